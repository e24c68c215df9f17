/*
 * gmm_sm100.h -- C ABI of the B200 (sm_100a) grouped-GEMM forward.
 *
 * One library, libgmm_sm100.so, exports these symbols.  Signatures carry only
 * plain pointers, integers and sizes (no C++ or torch types), so the library
 * can be bound from C, C++ (the torch operator in gmm_b200/csrc/torch_op.cpp),
 * Python ctypes, or any other FFI.  No exception crosses the boundary: every
 * entry point returns 0 or a negative gmm_status code.
 *
 * Semantics (the reference's forward, reference csrc/hopper_gmm_forward.h:9-25):
 *   A : [num_tokens, dim]            row-major, device memory
 *   B : [num_experts, dim, dim_out]  row-major (trans_b = 0), or
 *       [num_experts, dim_out, dim]  row-major (trans_b = 1), device memory
 *   batch_sizes : [num_experts] int64 in HOST memory, sum == num_tokens
 *   D : [num_tokens, dim_out]        row-major, device memory, same dtype as A
 * For each expert e with rows [off_e, off_e + batch_sizes[e]):
 *   D[rows] = A[rows] @ B[e]        (B[e]^T when trans_b)
 * accumulated in fp32.  Zero-row experts are skipped.  fp32 inputs are
 * multiplied on the tensor cores as three TF32 products (hi*hi + hi*lo +
 * lo*hi, the split made in shared memory inside the GEMM kernel) which gives
 * close to fp32 accuracy.
 */
#ifndef GMM_SM100_H_
#define GMM_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (A, B and D share one). */
enum gmm_dtype {
  GMM_DTYPE_F32 = 0,  /* fp32 in/out, 3xTF32 tensor-core products */
  GMM_DTYPE_BF16 = 1, /* bf16 in/out, fp32 accumulate */
  GMM_DTYPE_F16 = 2   /* fp16 in/out, fp32 accumulate */
};

/* Status codes. */
enum gmm_status {
  GMM_OK = 0,
  GMM_ERR_INVALID_ARGUMENT = -1, /* null pointer, negative size, bad shape */
  GMM_ERR_BATCH_SUM = -2,        /* sum(batch_sizes) != num_tokens */
  GMM_ERR_DTYPE = -3,            /* dtype not one of gmm_dtype */
  GMM_ERR_ALIGNMENT = -4,        /* pointer or row pitch not 16-byte aligned */
  GMM_ERR_ARCH = -5,             /* device is not compute capability 10.0 */
  GMM_ERR_CUDA = -6,             /* a CUDA runtime / driver call failed */
  GMM_ERR_WORKSPACE = -7,        /* workspace missing or smaller than required */
  GMM_ERR_TOO_LARGE = -8,        /* a size exceeds the kernel's index range */
  GMM_ERR_DEVICE_TIMEOUT = -9    /* a kernel wait ran out (see gmm_sm100_device_error) */
};

/* Human-readable text for a status code (static storage). */
const char* gmm_sm100_errstr(int status);

/* Detail of the last failure on the calling thread (thread-local storage). */
const char* gmm_sm100_last_error(void);

/* Kernel family override for 16-bit problems.  No reference counterpart (the
 * reference has one CUTLASS configuration per dtype).  GMM_TILE_AUTO picks
 * per problem (CTA-pair 256-row tiles when the non-empty experts average at
 * least 384 rows, swap-AB tiles when no expert has more than 64 rows, else
 * 128-row tiles); the others force one family (swap falls back to 128-row
 * tiles for the SwiGLU and expert-parallel epilogues).  Process-wide; the
 * initial value comes from the environment variable GMM_SM100_TILE
 * (128 / 256 / swap), read once.  Takes effect for plans made afterwards.
 * Returns the previous kind, or GMM_ERR_INVALID_ARGUMENT. */
enum gmm_tile_kind { GMM_TILE_AUTO = 0, GMM_TILE_128 = 1, GMM_TILE_PAIR = 2, GMM_TILE_SWAP = 3 };
int gmm_sm100_set_tile_kind(int kind);

/* GMM_OK if `device` is a compute-capability 10.0 (B200-class) GPU.
 * Replaces the reference's compute-capability check
 * (reference csrc/hopper_gmm_forward.cu:389-397). */
int gmm_sm100_check_device(int device);

/* Bytes of device workspace gmm_sm100_forward needs for this problem: the
 * tile table when more than 1024 experts are non-empty, else 0.  Replaces the reference's
 * workspace sizing (reference csrc/hopper_gmm_forward.cu:210-222, 411-427). */
size_t gmm_sm100_workspace_size(const int64_t* batch_sizes, int64_t num_experts,
                                int64_t num_tokens, int64_t dim, int64_t dim_out, int dtype,
                                int trans_b);

/* The grouped-GEMM forward: validates, builds the tile schedule from the host
 * batch_sizes and launches the persistent tcgen05 kernel on `stream` (a
 * cudaStream_t; NULL = legacy default stream).  Asynchronous: returns once the
 * work is enqueued.  `workspace` must hold gmm_sm100_workspace_size() bytes,
 * 256-byte aligned (may be NULL when that size is 0); it must stay allocated
 * until the work on `stream` completes.  Every row of D is written (D need
 * not be initialised).  Replaces the reference's entry point
 * hpc_ops_hopper::hopper_gmm_forward (reference csrc/hopper_gmm_forward.cu:372-486)
 * and its launcher CutlassGroupedGemm (reference csrc/hopper_gmm_forward.cu:230-325). */
int gmm_sm100_forward(const void* A, const void* B, const int64_t* batch_sizes,
                      int64_t num_experts, int64_t num_tokens, int64_t dim, int64_t dim_out,
                      int dtype, int trans_b, void* D, void* workspace, size_t workspace_bytes,
                      void* stream);

/* The same forward in two steps.  gmm_sm100_plan does the host half of
 * gmm_sm100_forward -- validation, the tile table and the kernel choice from
 * the host batch_sizes -- without any CUDA call; gmm_sm100_launch does the
 * device half on given operands.  A plan is built once per routing and can be
 * launched for every GEMM that shares the batch sizes (a layer's gate/up and
 * down projections), from any thread and stream at once (it is never
 * modified after creation).  Replaces the reference's host-side problem
 * building, done again on every call (reference csrc/hopper_gmm_forward.cu:
 * 230-316 CutlassGroupedGemm, :454-471 segmentation).  The kernel override
 * (gmm_sm100_set_tile_kind) in force when the plan is made applies to it. */
typedef struct gmm_sm100_plan_s gmm_sm100_plan_t;
int gmm_sm100_plan(const int64_t* batch_sizes, int64_t num_experts, int64_t num_tokens, int64_t dim,
                   int64_t dim_out, int dtype, int trans_b, gmm_sm100_plan_t** plan_out);
/* Workspace bytes gmm_sm100_launch needs for this plan (0 for most 16-bit plans). */
size_t gmm_sm100_plan_workspace_size(const gmm_sm100_plan_t* plan);
/* A, B, D as in gmm_sm100_forward, with the plan's shapes and dtype. */
int gmm_sm100_launch(const gmm_sm100_plan_t* plan, const void* A, const void* B, void* D, void* workspace,
                     size_t workspace_bytes, void* stream);
void gmm_sm100_plan_free(gmm_sm100_plan_t* plan);

/* Fused MoE gate/up projection with SwiGLU.  No reference counterpart: the
 * reference stops at the grouped GEMM, and its MoE layer would call it twice
 * (gate+up, then down) with the activation in between.  B holds each
 * expert's gate and up projections side by side -- [E, dim, 2*I] with
 * columns [gate | up] (trans_b = 0) or [E, 2*I, dim] with rows [gate | up]
 * (trans_b = 1); dim_out = 2*I, a multiple of 16.  D is [num_tokens, I]:
 *   D[rows_e] = silu(A[rows_e] @ Bgate[e]) * (A[rows_e] @ Bup[e])
 * computed from the fp32 accumulators and rounded once; bf16 / fp16 only.
 * Workspace as gmm_sm100_forward. */
int gmm_sm100_forward_swiglu(const void* A, const void* B, const int64_t* batch_sizes,
                             int64_t num_experts, int64_t num_tokens, int64_t dim, int64_t dim_out,
                             int dtype, int trans_b, void* D, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Variable-K grouped GEMM (MoE backward weight gradient): for each expert e
 * with rows [off_e, off_e + batch_sizes[e]) of A [num_tokens, dim_a] and
 * B [num_tokens, dim_b] (both row-major),
 *   D[e] = A[rows_e]^T @ B[rows_e]      D is [num_experts, dim_a, dim_b]
 * accumulated in fp32; an expert with no rows gets D[e] = 0.  bf16 / fp16;
 * num_experts <= 3073.  Restores the kernel family the reference removed
 * from its forward-only extract (reference csrc/hopper_gmm_forward.cu:16-21,
 * CutlassGroupedGemmVariableK). */
int gmm_sm100_forward_vark(const void* A, const void* B, const int64_t* batch_sizes,
                           int64_t num_experts, int64_t num_tokens, int64_t dim_a, int64_t dim_b,
                           int dtype, void* D, void* stream);

/* ------------------------------------------------ device-resident MoE layer
 * No reference counterpart (the reference's caller routes and permutes on its
 * own; its benchmark leaves them out).  Every entry below only enqueues work
 * on `stream` and never waits for the device, so a whole MoE layer can run
 * without a host synchronisation. */

/* Grouped GEMM whose batch sizes live in device memory: int32
 * batch_sizes_dev[num_experts] (num_experts <= 1024).  A has rows_cap rows
 * of which the first sum(batch_sizes) are used; D rows beyond the sum are not
 * written.  If a size is negative or the sum exceeds rows_cap the kernel does
 * no work and records GMM_ERR_INVALID_ARGUMENT / GMM_ERR_BATCH_SUM in the
 * device error word.  swiglu != 0 selects the fused SwiGLU epilogue (see
 * gmm_sm100_forward_swiglu).  Needs no workspace: the group table is built in
 * shared memory (workspace / workspace_bytes are accepted and ignored). */
int gmm_sm100_forward_dev(const void* A, const void* B, const int32_t* batch_sizes_dev,
                          int64_t num_experts, int64_t rows_cap, int64_t dim, int64_t dim_out,
                          int dtype, int trans_b, int swiglu, void* D, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Workspace bytes gmm_sm100_forward_dev needs: 0 for every problem. */
size_t gmm_sm100_dev_workspace_size(int64_t num_experts, int64_t rows_cap, int64_t dim,
                                    int64_t dim_out, int dtype);

/* Top-k routing: per token, softmax over the num_experts logits (fp32, bf16
 * or fp16, row-major [num_tokens, num_experts]) and the k largest (ties to
 * the lower expert index; k <= 8).  ids[t*k + j] (int32) in descending order;
 * weights[t*k + j] (fp32) their probabilities, renormalised to sum 1 when
 * renormalize != 0. */
int gmm_sm100_moe_topk(const void* logits, int logits_dtype, int64_t num_tokens, int num_experts,
                       int k, int renormalize, int32_t* ids, float* weights, void* stream);

/* Permutation into expert order: a stable counting sort of the
 * num_tokens * k (token, slot) pairs by ids[t*k + j].  Writes batch_sizes
 * (int32[num_experts], rows per expert), dst_pos[t*k + j] (row of the pair
 * in the permuted matrix; -1 for an id outside [0, num_experts)),
 * src_token[row] (token of each permuted row) and, when x is non-null,
 * x_perm[row] = x[src_token[row]] (rows of row_bytes bytes, a multiple of 16). */
int gmm_sm100_moe_permute(const void* x, int64_t num_tokens, int64_t row_bytes, const int32_t* ids,
                          int k, int num_experts, void* x_perm, int32_t* batch_sizes,
                          int32_t* dst_pos, int32_t* src_token, void* workspace,
                          size_t workspace_bytes, void* stream);

size_t gmm_sm100_moe_permute_workspace_size(int64_t num_pairs, int num_experts);

/* Combine: out[t] = sum_j weights[t*k + j] * y[dst_pos[t*k + j]] with fp32
 * accumulation (weights may be NULL: plain sum); y is [num_tokens*k, dim_out]
 * in expert order, dim_out a multiple of 8. */
int gmm_sm100_moe_unpermute(const void* y, const int32_t* dst_pos, const float* weights,
                            int64_t num_tokens, int k, int64_t dim_out, int dtype, void* out,
                            void* stream);

/* Detail of the last failure of a gmm_sm100_moe_* call on this thread. */
const char* gmm_sm100_moe_last_error(void);

/* Reads (and with clear != 0, resets) the device-side error word of the
 * current device: 0, or a gmm_status recorded by a kernel whose bounded wait
 * ran out.  Synchronises the device.  No reference counterpart (the
 * reference kernel has no device-side error path). */
int gmm_sm100_device_error(int* status_out, int clear);

/* Test hook of the bounded-wait path; no reference counterpart (the
 * reference kernel has no device-side timeout).  Runs gmm_sm100_forward
 * (bf16 / fp16, no workspace; the 128-row or CTA-pair kernel, per the tile
 * kind in force) with two changes: every pipeline wait gives up after wait_s
 * seconds (0 < wait_s <= 2) instead of 2 s, and the TMA producer of the first
 * tile of CTA (pair) 0 skips the loads of k-block drop_k_block.  The MMA
 * warp's wait for that stage then runs out, the CTA drains the copies it has
 * in flight, frees its tensor memory and returns, and the device error word
 * reads GMM_ERR_DEVICE_TIMEOUT (gmm_sm100_device_error).  D is left partly
 * unwritten.  Nothing faults or hangs: the failure is the one the bounded
 * waits exist for, made on purpose. */
int gmm_sm100_forward_inject_timeout(const void* A, const void* B, const int64_t* batch_sizes,
                                     int64_t num_experts, int64_t num_tokens, int64_t dim,
                                     int64_t dim_out, int dtype, int trans_b, void* D,
                                     int drop_k_block, double wait_s, void* stream);

/* ---------------------------------------------------------------- expert parallelism
 * No reference counterpart (the reference runs on one GPU).  A rank owning
 * num_local_experts experts receives, for local expert e, world segments of
 * rows stored expert-major in X: segment j (j = 0..world-1) comes from rank
 * s = (rank_base + j) % world and holds counts[e*world + j] rows.  Passing
 * its own rank as rank_base makes every rank start with a different peer, so
 * at any moment the ranks read from / write to distinct peers.  The pointers
 * in out_peers / src_peers (indexed by rank) are device addresses valid on
 * the calling device (peer memory of the other ranks, e.g. symmetric-memory
 * buffers); world <= 8. */

/* Dispatch: copy every (expert, segment) chunk of rows into X, reading
 * src_peers[s] + src_rows[e*world + j] * row_bytes over NVLink. */
int gmm_sm100_ep_gather(void* X, const void* const* src_peers, const int64_t* counts,
                        const int64_t* src_rows, int64_t num_local_experts, int world,
                        int rank_base, int64_t row_bytes, void* stream);

/* Cross-rank barrier of the layer, over peer memory (one small kernel; no
 * NCCL call).  flag_peers[s] points at rank s's `world` int32 flag slots (a
 * symmetric-memory buffer, zeroed before first use); every rank calls it
 * with the same, growing epoch.  Each rank posts epoch into every peer's slot
 * with release semantics at system scope -- so all the writes this rank
 * enqueued on `stream` before the barrier (its token rows, its peer stores)
 * are visible to the peers -- and waits for every peer's post with acquire.
 * The wait is bounded by timeout_s: past it the kernel records
 * GMM_ERR_DEVICE_TIMEOUT in the device error word (gmm_sm100_device_error)
 * and returns, so a rank that never arrives is reported instead of hanging
 * the GPU. */
int gmm_sm100_ep_barrier(int* const* flag_peers, int world, int rank, int epoch, double timeout_s,
                         void* stream);

/* Local grouped GEMM with the combine fused into its epilogue: the result of
 * row i of segment j of local expert e goes straight to row
 * dst_rows[e*world + j] + i of out_peers[s] (s = the rank the row came
 * from).  B holds the local experts' weights ([E_local, dim, dim_out], or
 * [E_local, dim_out, dim] if trans_b).  The caller orders the peers'
 * reads/writes with a cross-rank barrier before and after. */
int gmm_sm100_forward_ep(const void* X, const void* B, const int64_t* counts, const int64_t* dst_rows,
                         int64_t num_local_experts, int world, int rank_base, void* const* out_peers,
                         int64_t num_rows, int64_t dim, int64_t dim_out, int dtype, int trans_b,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes gmm_sm100_forward_ep needs (fp32 splits, large tables). */
size_t gmm_sm100_ep_workspace_size(const int64_t* counts, int64_t num_local_experts, int world,
                                   int64_t num_rows, int64_t dim, int64_t dim_out, int dtype);

/* Size of the fixed scratch area used by gmm_sm100_forward_f32_noalloc. */
#define GMM_SM100_NOALLOC_SCRATCH_BYTES (8u << 20) /* 8 MiB */

/* fp32 grouped-GEMM forward that allocates no memory at all.  No counterpart
 * in the reference; it exists for callers that cannot allocate device memory
 * themselves -- for example a plugin running inside a host engine that owns
 * every device allocation and its budget, or a latency-critical caller that
 * cannot afford cudaMalloc / cudaFree, which may synchronise the whole device.
 *
 * Same arguments and results as gmm_sm100_forward with dtype GMM_DTYPE_F32
 * (three TF32 tensor-core products, split into TF32 hi/lo parts in shared
 * memory), minus the workspace: the one device buffer that path needs, the
 * tile table of more than 1024 non-empty experts, goes to a scratch array of
 * GMM_SM100_NOALLOC_SCRATCH_BYTES compiled into the library, which every GPU
 * that loads the library keeps until the process exits.  Problems whose table
 *   (3 * non-empty experts + 2) * 4 bytes, rounded up to 256
 * exceeds that size (about 699,000 non-empty experts) are rejected with
 * GMM_ERR_TOO_LARGE before any GPU work.
 *
 * The first call on a device that needs the scratch looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture.  The address is kept per device
 * ordinal, so it belongs to the device's primary context, the one every CUDA
 * runtime call works in; a caller that makes a different driver-API context
 * current on the device (cuCtxSetCurrent) must not use this entry point.
 * All calls share the one scratch array; each call writes the part it reads
 * before its kernel runs (stream-ordered), so calls whose GPU work overlaps
 * (different streams, or different host threads, on one device) race on it
 * and must be serialised by the caller. */
int gmm_sm100_forward_f32_noalloc(const float* A, const float* B, const int64_t* batch_sizes,
                                  int64_t num_experts, int64_t num_tokens, int64_t dim,
                                  int64_t dim_out, int trans_b, float* D, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GMM_SM100_H_ */
