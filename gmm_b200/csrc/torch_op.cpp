// torch_op.cpp -- the `hopper_gmm_fwd::gmm` PyTorch operator over the C ABI.
//
// Drop-in for the reference's op registration (reference csrc/bindings.cc:13-19)
// and host entry point (reference csrc/hopper_gmm_forward.cu:372-486): same
// schema, same argument checks and messages, CUDA dispatch key only.  The
// tensor work is delegated to libgmm_sm100.so through include/gmm_sm100.h.
//
// Differences from the reference host layer, all deliberate:
//   * D is allocated uninitialised (at::empty): sum(batch_sizes) == T means
//     every row is written by exactly one expert, so the reference's memset
//     (hopper_gmm_forward.cu:440) is dead work.
//   * No per-expert tensor views or problem-table upload: the C ABI turns the
//     host batch_sizes into a tile schedule passed with the kernel launch.
//   * fp32 with trans_b=True multiplies by B[e]^T (B given as [E, dim_out, dim]),
//     as documented for trans_b; the reference transposed such a B a second
//     time (hopper_gmm_forward.cu:442-446).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "gmm_sm100.h"
#include "hopper_gmm_forward.h"

namespace hpc_ops_hopper {

// Declared in include/hopper_gmm_forward.h with the reference's signature
// (reference csrc/hopper_gmm_forward.h:23-25).
at::Tensor hopper_gmm_forward(at::Tensor A, at::Tensor B, at::Tensor batch_sizes, bool transb) {
  TORCH_CHECK(A.is_cuda() && A.is_contiguous(), "A must be a contiguous CUDA tensor");
  TORCH_CHECK(B.is_cuda() && B.is_contiguous(), "B must be a contiguous CUDA tensor");
  TORCH_CHECK(A.dim() == 2, "A must be 2D");
  TORCH_CHECK(B.dim() == 3, "B must be 3D [num_experts, dim, dim_out] (forward-only build)");
  TORCH_CHECK(batch_sizes.is_cpu() && batch_sizes.dim() == 1 &&
                  batch_sizes.scalar_type() == at::kLong,
              "batch_sizes must be a 1D CPU int64 tensor");
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "A and B must have the same dtype");
  TORCH_CHECK(A.get_device() == B.get_device(), "A and B must be on the same device");

  const int device = A.get_device();
  c10::cuda::CUDAGuard guard(device);
  {
    const int rc = gmm_sm100_check_device(device);
    TORCH_CHECK(rc == GMM_OK, "hopper_gmm_forward: ", gmm_sm100_last_error());
  }

  const int64_t num_experts = batch_sizes.size(0);
  const int64_t dim = A.size(1);
  const int64_t dim_out = transb ? B.size(1) : B.size(2);
  TORCH_CHECK(B.size(0) == num_experts, "B.size(0) must equal num_experts (batch_sizes.size(0))");
  TORCH_CHECK((transb ? B.size(2) : B.size(1)) == dim, "B.", (transb ? "size(2)" : "size(1)"),
              " must equal A.size(1) (dim), got ", (transb ? B.size(2) : B.size(1)), " vs ", dim);

  int dtype;
  switch (A.scalar_type()) {
    case at::kFloat: dtype = GMM_DTYPE_F32; break;
    case at::kBFloat16: dtype = GMM_DTYPE_BF16; break;
    case at::kHalf: dtype = GMM_DTYPE_F16; break;
    default: TORCH_CHECK(false, "Unsupported dtype: only FP32 / BF16 / FP16 are supported");
  }

  auto bs = batch_sizes.contiguous();
  const int64_t* bs_ptr = bs.data_ptr<int64_t>();
  at::Tensor D = at::empty({A.size(0), dim_out}, A.options());
  const size_t ws_bytes =
      gmm_sm100_workspace_size(bs_ptr, num_experts, A.size(0), dim, dim_out, dtype, transb ? 1 : 0);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({static_cast<int64_t>(ws_bytes)}, A.options().dtype(at::kByte));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  const int rc = gmm_sm100_forward(A.data_ptr(), B.data_ptr(), bs_ptr, num_experts, A.size(0), dim,
                                   dim_out, dtype, transb ? 1 : 0, D.data_ptr(),
                                   ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream);
  TORCH_CHECK(rc == GMM_OK, gmm_sm100_last_error());
  return D;
}

}  // namespace hpc_ops_hopper

namespace gmm_b200 {

// Fused MoE gate/up projection + SwiGLU: B holds [gate | up] (2*I output
// columns); returns silu(A @ Bgate) * (A @ Bup), [T, I].  No reference
// counterpart (the reference's caller would run two GEMM segments with the
// activation in between).
at::Tensor gmm_swiglu(at::Tensor A, at::Tensor B, at::Tensor batch_sizes, bool transb) {
  TORCH_CHECK(A.is_cuda() && A.is_contiguous(), "A must be a contiguous CUDA tensor");
  TORCH_CHECK(B.is_cuda() && B.is_contiguous(), "B must be a contiguous CUDA tensor");
  TORCH_CHECK(A.dim() == 2, "A must be 2D");
  TORCH_CHECK(B.dim() == 3, "B must be 3D [num_experts, dim, 2*inter] (or [num_experts, 2*inter, dim])");
  TORCH_CHECK(batch_sizes.is_cpu() && batch_sizes.dim() == 1 &&
                  batch_sizes.scalar_type() == at::kLong,
              "batch_sizes must be a 1D CPU int64 tensor");
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "A and B must have the same dtype");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 || A.scalar_type() == at::kHalf,
              "gmm_swiglu supports bf16 / fp16");
  const int device = A.get_device();
  c10::cuda::CUDAGuard guard(device);
  TORCH_CHECK(gmm_sm100_check_device(device) == GMM_OK, "gmm_swiglu: ", gmm_sm100_last_error());
  const int64_t num_experts = batch_sizes.size(0);
  const int64_t dim = A.size(1);
  const int64_t dim_out = transb ? B.size(1) : B.size(2);
  TORCH_CHECK(B.size(0) == num_experts, "B.size(0) must equal num_experts (batch_sizes.size(0))");
  TORCH_CHECK((transb ? B.size(2) : B.size(1)) == dim, "B's contraction size must equal A.size(1) (dim)");
  TORCH_CHECK(dim_out % 2 == 0, "B must hold gate and up projections of equal width");
  const int dtype = A.scalar_type() == at::kBFloat16 ? GMM_DTYPE_BF16 : GMM_DTYPE_F16;
  auto bs = batch_sizes.contiguous();
  const int64_t* bs_ptr = bs.data_ptr<int64_t>();
  at::Tensor D = at::empty({A.size(0), dim_out / 2}, A.options());
  const size_t ws_bytes =
      gmm_sm100_workspace_size(bs_ptr, num_experts, A.size(0), dim, dim_out, dtype, transb ? 1 : 0);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({static_cast<int64_t>(ws_bytes)}, A.options().dtype(at::kByte));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(device).stream();
  const int rc = gmm_sm100_forward_swiglu(A.data_ptr(), B.data_ptr(), bs_ptr, num_experts, A.size(0),
                                          dim, dim_out, dtype, transb ? 1 : 0, D.data_ptr(),
                                          ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream);
  TORCH_CHECK(rc == GMM_OK, gmm_sm100_last_error());
  return D;
}

}  // namespace gmm_b200

TORCH_LIBRARY(hopper_gmm_fwd, m) {
  m.def("gmm(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor");
  m.def("gmm_swiglu(Tensor A, Tensor B, Tensor batch_sizes, bool trans_b) -> Tensor");
}

TORCH_LIBRARY_IMPL(hopper_gmm_fwd, CUDA, m) {
  m.impl("gmm", &hpc_ops_hopper::hopper_gmm_forward);
  m.impl("gmm_swiglu", &gmm_b200::gmm_swiglu);
}
