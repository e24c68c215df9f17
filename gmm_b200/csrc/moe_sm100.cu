// moe_sm100.cu -- the MoE steps on either side of the grouped GEMM, on device:
// top-k routing, permutation of token rows into expert order, and the
// weighted un-permutation of the expert outputs.  No reference counterpart:
// the reference's benchmark times the grouped GEMM alone and leaves routing
// and gather/scatter out (reference tests/bench_moe_forward.py:216-217).
//
// Together with the device-batch-sizes grouped GEMM (gmm_sm100_forward_dev)
// these make an MoE layer that never synchronises with the host.
//
// All index work is deterministic: the permutation is a stable counting
// sort of the (token, slot) pairs by expert, so row i of the permuted
// matrix is the i-th pair of its expert in (token, slot) order.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "gmm_sm100.h"

namespace {

constexpr int kMaxExperts = 1024;
constexpr int kChunk = 4096;  // (token, slot) pairs per counting block

thread_local std::string t_moe_error;

int moe_fail(int code, const std::string& msg) {
  t_moe_error = msg;
  return code;
}

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }

// ------------------------------------------------------------------ routing
// One warp per token: softmax over E logits, then the k largest (ties go to
// the lower expert index), selected by the logits themselves so the choice
// does not depend on exp rounding.  weights = softmax probabilities of the
// selected experts, renormalised to sum 1 when `renorm`.
template <typename T>
__global__ void __launch_bounds__(256) moe_topk_kernel(const T* __restrict__ logits, int num_tokens,
                                                       int E, int k, int renorm,
                                                       int32_t* __restrict__ ids,
                                                       float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const int token = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (token >= num_tokens) return;
  const T* row = logits + static_cast<long long>(token) * E;
  float v[kMaxExperts / 32];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll 4
  for (int i = 0; i < per; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? to_float(row[e]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int i = 0; i < per; ++i) {
    const int e = lane + 32 * i;
    if (e < E) sum += __expf(v[i] - mx);
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  float sel_sum = 0.f;
  float sel_p[8];
  int sel_e[8];
  for (int j = 0; j < k; ++j) {
    // warp arg-max over the remaining logits, lowest index on ties
    float best = -INFINITY;
    int best_e = 0x7fffffff;
    for (int i = 0; i < per; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < best_e))) {
        best = v[i];
        best_e = e;
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    if ((best_e & 31) == lane) v[best_e >> 5] = -INFINITY;  // remove it
    const float pr = __expf(best - mx) / sum;
    sel_p[j] = pr;
    sel_e[j] = best_e;
    sel_sum += pr;
  }
  if (lane == 0) {
    for (int j = 0; j < k; ++j) {
      ids[static_cast<long long>(token) * k + j] = sel_e[j];
      weights[static_cast<long long>(token) * k + j] = renorm ? sel_p[j] / sel_sum : sel_p[j];
    }
  }
}

// --------------------------------------------------------------- permutation
// Per-chunk expert histogram.
__global__ void __launch_bounds__(256) moe_count_kernel(const int32_t* __restrict__ ids, int n_pairs,
                                                        int E, int32_t* __restrict__ counts) {
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * kChunk;
  const int p1 = min(p0 + kChunk, n_pairs);
  for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const int e = ids[p];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);  // out-of-range ids belong to no expert
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[blockIdx.x * E + e] = hist[e];
}

// One block: expert totals (batch sizes), their exclusive scan, and the
// first row of every (chunk, expert) run.
__global__ void __launch_bounds__(1024) moe_scan_kernel(const int32_t* __restrict__ counts, int n_chunks,
                                                        int E, int32_t* __restrict__ base,
                                                        int32_t* __restrict__ batch_sizes) {
  __shared__ int tot[kMaxExperts];
  const int e = threadIdx.x;
  int t = 0;
  if (e < E)
    for (int c = 0; c < n_chunks; ++c) t += counts[c * E + e];
  tot[e] = e < E ? t : 0;
  __syncthreads();
  // exclusive scan of tot (Hillis-Steele, 1024 entries)
  for (int d = 1; d < kMaxExperts; d <<= 1) {
    const int add = e >= d ? tot[e - d] : 0;
    __syncthreads();
    tot[e] += add;
    __syncthreads();
  }
  if (e < E) {
    int run = tot[e] - t;  // exclusive prefix
    batch_sizes[e] = t;
    for (int c = 0; c < n_chunks; ++c) {
      base[c * E + e] = run;
      run += counts[c * E + e];
    }
  }
}

// One warp per chunk walks its pairs in order, 32 at a time: pairs of the
// same expert within a group are ranked by lane (match_any + popc), so the
// assignment is the stable order.
__global__ void __launch_bounds__(32) moe_assign_kernel(const int32_t* __restrict__ ids, int n_pairs,
                                                        int E, int k, const int32_t* __restrict__ base,
                                                        int32_t* __restrict__ dst_pos,
                                                        int32_t* __restrict__ src_token) {
  __shared__ int next[kMaxExperts];
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) next[e] = base[blockIdx.x * E + e];
  __syncwarp();
  const int p0 = blockIdx.x * kChunk;
  const int p1 = min(p0 + kChunk, n_pairs);
  const unsigned lt = (1u << lane) - 1u;
  for (int g = p0; g < p1; g += 32) {
    const int p = g + lane;
    const int id = p < p1 ? ids[p] : -1;
    const bool live = p < p1 && id >= 0 && id < E;
    if (p < p1 && !live) dst_pos[p] = -1;  // an out-of-range id has no row
    const int e = live ? id : -1 - lane;  // dead lanes never match a real expert
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt);
    const int start = live ? next[e] : 0;
    __syncwarp();
    if (live) {
      const int pos = start + rank;
      dst_pos[p] = pos;
      src_token[pos] = p / k;
      if (rank == 0) next[e] = start + __popc(peers);
    }
    __syncwarp();
  }
}

// x_perm[i] = x[src_token[i]], one warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) moe_gather_kernel(const char* __restrict__ x,
                                                         const int32_t* __restrict__ src_token,
                                                         int n_rows, int num_tokens, long long row_bytes,
                                                         const int32_t* __restrict__ batch_sizes, int E,
                                                         char* __restrict__ x_perm) {
  __shared__ int live_rows;
  if (threadIdx.x == 0) {  // rows past the experts' total were never assigned a token
    int t = 0;
    for (int e = 0; e < E; ++e) t += batch_sizes[e];
    live_rows = t;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int n16 = static_cast<int>(row_bytes >> 4);
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < live_rows && r < n_rows; r += warps) {
    const int tok = src_token[r];
    if (tok < 0 || tok >= num_tokens) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<long long>(tok) * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(x_perm + static_cast<long long>(r) * row_bytes);
    for (int i = lane; i < n16; i += 32) dst[i] = src[i];
  }
}

// ---------------------------------------------------------------- combine
template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<__half> {
  static __device__ __forceinline__ void load(const __half* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static __device__ __forceinline__ void store(__half* p, const float (&f)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&f)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

// out[t] = sum_j w[t, j] * y[dst_pos[t, j]] (fp32 accumulation), one warp per token.
template <typename T>
__global__ void __launch_bounds__(256) moe_unpermute_kernel(const T* __restrict__ y,
                                                            const int32_t* __restrict__ dst_pos,
                                                            const float* __restrict__ weights,
                                                            int num_tokens, int k, int dim_out,
                                                            int n_rows, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < num_tokens; t += warps) {
    for (int c = lane * 8; c < dim_out; c += 256) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < k; ++j) {
        const long long pos = dst_pos[static_cast<long long>(t) * k + j];
        if (pos < 0 || pos >= n_rows) continue;  // a slot routed to no expert contributes nothing
        const float w = weights ? weights[static_cast<long long>(t) * k + j] : 1.0f;
        float f[8];
        Vec8<T>::load(y + pos * dim_out + c, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(w, f[i], acc[i]);
      }
      Vec8<T>::store(out + static_cast<long long>(t) * dim_out + c, acc);
    }
  }
}

int sm_count_current() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return moe_fail(GMM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return GMM_OK;
}

}  // namespace

extern "C" {

const char* gmm_sm100_moe_last_error(void) { return t_moe_error.c_str(); }

int gmm_sm100_moe_topk(const void* logits, int logits_dtype, int64_t num_tokens, int num_experts, int k,
                       int renormalize, int32_t* ids, float* weights, void* stream) {
  if (num_tokens < 0 || num_experts < 1 || num_experts > kMaxExperts || k < 1 || k > 8 || k > num_experts)
    return moe_fail(GMM_ERR_INVALID_ARGUMENT, "need 1 <= k <= min(8, num_experts) and num_experts <= 1024");
  if (num_tokens == 0) return GMM_OK;
  if (!logits || !ids || !weights) return moe_fail(GMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (num_tokens > (1LL << 31) / 32) return moe_fail(GMM_ERR_TOO_LARGE, "too many tokens");
  const int blocks = static_cast<int>((num_tokens * 32 + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int T = static_cast<int>(num_tokens);
  switch (logits_dtype) {
    case GMM_DTYPE_F32:
      moe_topk_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(logits), T, num_experts, k,
                                                     renormalize, ids, weights);
      break;
    case GMM_DTYPE_BF16:
      moe_topk_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), T,
                                                             num_experts, k, renormalize, ids, weights);
      break;
    case GMM_DTYPE_F16:
      moe_topk_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(logits), T, num_experts, k,
                                                      renormalize, ids, weights);
      break;
    default:
      return moe_fail(GMM_ERR_DTYPE, "logits must be fp32, bf16 or fp16");
  }
  return launch_status("moe_topk launch");
}

size_t gmm_sm100_moe_permute_workspace_size(int64_t num_pairs, int num_experts) {
  if (num_pairs <= 0 || num_experts <= 0) return 0;
  const int64_t chunks = (num_pairs + kChunk - 1) / kChunk;
  return static_cast<size_t>((2 * chunks * num_experts * 4 + 255) / 256 * 256);
}

int gmm_sm100_moe_permute(const void* x, int64_t num_tokens, int64_t row_bytes, const int32_t* ids, int k,
                          int num_experts, void* x_perm, int32_t* batch_sizes, int32_t* dst_pos,
                          int32_t* src_token, void* workspace, size_t workspace_bytes, void* stream) {
  if (num_tokens < 0 || k < 1 || num_experts < 1 || num_experts > kMaxExperts)
    return moe_fail(GMM_ERR_INVALID_ARGUMENT, "bad permute sizes");
  if (row_bytes < 0 || row_bytes % 16 != 0)
    return moe_fail(GMM_ERR_ALIGNMENT, "row bytes must be a multiple of 16");
  const int64_t n_pairs = num_tokens * k;
  if (n_pairs > INT32_MAX) return moe_fail(GMM_ERR_TOO_LARGE, "too many (token, slot) pairs");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_pairs == 0) {
    if (cudaMemsetAsync(batch_sizes, 0, sizeof(int32_t) * num_experts, s) != cudaSuccess)
      return moe_fail(GMM_ERR_CUDA, "cudaMemsetAsync");
    return GMM_OK;
  }
  const size_t need = gmm_sm100_moe_permute_workspace_size(n_pairs, num_experts);
  if (!workspace || workspace_bytes < need)
    return moe_fail(GMM_ERR_WORKSPACE, "permute workspace needs " + std::to_string(need) + " bytes");
  if (!ids || !batch_sizes || !dst_pos || !src_token)
    return moe_fail(GMM_ERR_INVALID_ARGUMENT, "null index pointer");
  const int chunks = static_cast<int>((n_pairs + kChunk - 1) / kChunk);
  int32_t* counts = static_cast<int32_t*>(workspace);
  int32_t* base = counts + static_cast<int64_t>(chunks) * num_experts;
  const int np = static_cast<int>(n_pairs);
  moe_count_kernel<<<chunks, 256, 0, s>>>(ids, np, num_experts, counts);
  moe_scan_kernel<<<1, 1024, 0, s>>>(counts, chunks, num_experts, base, batch_sizes);
  moe_assign_kernel<<<chunks, 32, 0, s>>>(ids, np, num_experts, k, base, dst_pos, src_token);
  int rc = launch_status("moe permute launch");
  if (rc != GMM_OK || row_bytes == 0 || !x) return rc;
  if (!x_perm) return moe_fail(GMM_ERR_INVALID_ARGUMENT, "x_perm is null");
  const int blocks = static_cast<int>(std::min<int64_t>((n_pairs + 7) / 8, 4LL * sm_count_current()));
  moe_gather_kernel<<<std::max(blocks, 1), 256, 0, s>>>(static_cast<const char*>(x), src_token, np,
                                                        static_cast<int>(num_tokens), row_bytes, batch_sizes,
                                                        num_experts, static_cast<char*>(x_perm));
  return launch_status("moe gather launch");
}

int gmm_sm100_moe_unpermute(const void* y, const int32_t* dst_pos, const float* weights, int64_t num_tokens,
                            int k, int64_t dim_out, int dtype, void* out, void* stream) {
  if (num_tokens < 0 || k < 1 || dim_out < 0) return moe_fail(GMM_ERR_INVALID_ARGUMENT, "bad sizes");
  if (num_tokens == 0 || dim_out == 0) return GMM_OK;
  if (dim_out % 8 != 0) return moe_fail(GMM_ERR_ALIGNMENT, "dim_out must be a multiple of 8");
  if (!y || !dst_pos || !out) return moe_fail(GMM_ERR_INVALID_ARGUMENT, "null pointer");
  if (num_tokens * k > INT32_MAX || dim_out > INT32_MAX) return moe_fail(GMM_ERR_TOO_LARGE, "too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = static_cast<int>(std::min<int64_t>((num_tokens + 7) / 8, 8LL * sm_count_current()));
  const int T = static_cast<int>(num_tokens), N = static_cast<int>(dim_out);
  switch (dtype) {
    case GMM_DTYPE_BF16:
      moe_unpermute_kernel<__nv_bfloat16><<<std::max(blocks, 1), 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(y), dst_pos, weights, T, k, N, T * k, static_cast<__nv_bfloat16*>(out));
      break;
    case GMM_DTYPE_F16:
      moe_unpermute_kernel<__half><<<std::max(blocks, 1), 256, 0, s>>>(
          static_cast<const __half*>(y), dst_pos, weights, T, k, N, T * k, static_cast<__half*>(out));
      break;
    case GMM_DTYPE_F32:
      moe_unpermute_kernel<float><<<std::max(blocks, 1), 256, 0, s>>>(
          static_cast<const float*>(y), dst_pos, weights, T, k, N, T * k, static_cast<float*>(out));
      break;
    default:
      return moe_fail(GMM_ERR_DTYPE, "unsupported dtype");
  }
  return launch_status("moe unpermute launch");
}

}  // extern "C"
