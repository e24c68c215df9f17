/*
 * hopper_gmm_forward.h -- the C++ entry point of the grouped-GEMM forward, as
 * declared by the reference (reference csrc/hopper_gmm_forward.h:23-25), for
 * C++ code written against that header.  Defined in gmm_b200/_C.so (the same
 * function the hopper_gmm_fwd::gmm operator registers for the CUDA key), which
 * calls libgmm_sm100.so through the C ABI of gmm_sm100.h.
 *
 *   A : [num_tokens, dim]            contiguous CUDA, fp32 / bf16 / fp16
 *   B : [num_experts, dim, dim_out]  ([num_experts, dim_out, dim] if transb),
 *                                    contiguous CUDA, same dtype as A
 *   batch_sizes : [num_experts]      CPU int64, sum == num_tokens
 * Returns D : [num_tokens, dim_out], same dtype and device as A, with
 *   D[rows_e] = A[rows_e] @ B[e]     (B[e]^T when transb)
 * accumulated in fp32 (fp32 inputs: three TF32 tensor-core products).
 * Bad arguments raise c10::Error (RuntimeError in Python) with the
 * reference's messages.  Asynchronous on the current CUDA stream of A's device.
 *
 * torch::Tensor is at::Tensor, so the symbol is the reference's.
 */
#pragma once

#include <ATen/core/Tensor.h>

namespace hpc_ops_hopper {

at::Tensor hopper_gmm_forward(at::Tensor A, at::Tensor B, at::Tensor batch_sizes, bool transb = false);

}  // namespace hpc_ops_hopper
