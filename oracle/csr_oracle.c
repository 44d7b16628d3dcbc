/*
 * CPU restatement of the reference engine's CSR build and CSR SpMM.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels (tests/,
 * the smoke check and bench.py's CPU-baseline leg).  The product never links
 * or calls this file.
 *
 * orc_csr_plane   follows csr_build_kernel / scan / csr_compact
 *                 (spikestack_lite/sparse/src/sparse_linear.cu:251-369):
 *                 predicate v > 0, columns ascending within a row, int32
 *                 row offsets with row_offsets[0] = 0, values copied from S.
 * orc_spmm_csr    follows csr_coalesced_kernel (sparse_linear.cu:59-90):
 *                 out[b, o] = sum over the row's entries in order of
 *                 values[k] * weightT[col[k], o], one fused multiply-add per
 *                 term starting from 0 (nvcc contracts `sum += v * w`).
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared -o liboracle.so csr_oracle.c -lm
 */
#include <math.h>
#include <stdint.h>

int64_t orc_csr_plane(const float* S, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx,
                      float* values, int64_t capacity) {
  int64_t pos = 0;
  row_ptr[0] = 0;
  for (int64_t b = 0; b < M; ++b) {
    const float* r = S + b * (int64_t)K;
    int32_t n = 0;
    for (int k = 0; k < K; ++k) {
      const float v = r[k];
      if (v > 0.0f) {
        if (pos < capacity) {
          col_idx[pos] = k;
          if (values) values[pos] = v;
        }
        ++pos;
        ++n;
      }
    }
    if (nnz_row) nnz_row[b] = n;
    row_ptr[b + 1] = (int32_t)pos;
  }
  return pos;
}

void orc_spmm_csr(int64_t M, const int32_t* row_ptr, const int32_t* col_idx, const float* values,
                  const float* weightT, int N, float* out) {
  for (int64_t b = 0; b < M; ++b) {
    for (int o = 0; o < N; ++o) {
      float sum = 0.0f;
      for (int32_t p = row_ptr[b]; p < row_ptr[b + 1]; ++p) {
        const float v = values ? values[p] : 1.0f;
        sum = fmaf(v, weightT[(int64_t)col_idx[p] * N + o], sum);
      }
      out[b * (int64_t)N + o] = sum;
    }
  }
}
