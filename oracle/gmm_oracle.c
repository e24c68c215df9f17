/*
 * gmm_oracle.c -- CPU parity oracle for the grouped-GEMM forward.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or
 * calls this file; it is the checker the CUDA kernels are compared against.
 *
 * Restates the reference's own oracle `ref_gmm` (reference
 * tests/test_forward.py:8-15) and the row segmentation of the reference host
 * entry point (reference csrc/hopper_gmm_forward.cu:454-471):
 *
 *   for each expert i in order, with rows [start, start + batch_sizes[i]):
 *       out[start:start+m_i] = a[start:start+m_i] @ (b[i]^T if trans_b else b[i])
 *   sum(batch_sizes) must equal the number of rows of a; zero-row experts
 *   contribute no rows.
 *
 * Inputs are fp32 (16-bit inputs are widened exactly by the caller).
 * Products are accumulated in fp64 so the oracle is at least as accurate as
 * the reference kernel's fp32 accumulator (reference hopper_gmm_forward.cu:80);
 * the caller rounds the result to the output dtype.
 */
#include <stdint.h>
#include <stddef.h>

/* Return codes: 0 ok, -1 bad argument, -2 sum(batch_sizes) != num_rows. */
int gmm_oracle_f64acc(const float* a, const float* b, const int64_t* batch_sizes,
                      int64_t num_experts, int64_t num_rows, int64_t dim,
                      int64_t dim_out, int trans_b, double* out) {
  if (!a || !b || !batch_sizes || !out || num_experts < 0 || num_rows < 0 ||
      dim <= 0 || dim_out <= 0)
    return -1;
  int64_t total = 0;
  for (int64_t e = 0; e < num_experts; ++e) {
    if (batch_sizes[e] < 0) return -1;
    total += batch_sizes[e];
  }
  if (total != num_rows) return -2;

  int64_t start = 0;
  for (int64_t e = 0; e < num_experts; ++e) {
    const int64_t m = batch_sizes[e];
    const float* be = b + e * dim * dim_out;
#pragma omp parallel for schedule(static)
    for (int64_t r = start; r < start + m; ++r) {
      const float* ar = a + r * dim;
      double* orow = out + r * dim_out;
      if (trans_b) {
        /* b[e] is [dim_out, dim]: out[r][n] = sum_k a[r][k] * b[e][n][k] */
        for (int64_t n = 0; n < dim_out; ++n) {
          const float* bn = be + n * dim;
          double acc = 0.0;
          for (int64_t k = 0; k < dim; ++k) acc += (double)ar[k] * (double)bn[k];
          orow[n] = acc;
        }
      } else {
        /* b[e] is [dim, dim_out]: out[r][n] = sum_k a[r][k] * b[e][k][n] */
        for (int64_t n = 0; n < dim_out; ++n) orow[n] = 0.0;
        for (int64_t k = 0; k < dim; ++k) {
          const double av = (double)ar[k];
          const float* bk = be + k * dim_out;
          for (int64_t n = 0; n < dim_out; ++n) orow[n] += av * (double)bk[n];
        }
      }
    }
    start += m;
  }
  return 0;
}
