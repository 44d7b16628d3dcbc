// CSR branch of spike-linear: Y = CSR(S) x W with the weight tile held in
// shared memory and reused by every row of all T planes.
//
// Reference: csr_coalesced_kernel (sparse_linear.cu:59-90), which sums the
// row's nonzeros in ascending column order with one fp32 fused multiply-add
// per term.  This kernel keeps exactly that order and rounding (fmaf from
// 0.0f), so its output is bit-identical to the reference engine's; what it
// changes is the data movement: the reference re-reads W from global memory
// for every nonzero of every plane (the multistep loop launches one SpMM per
// plane, sparse_linear.cu:667-688), here each CTA stages a [K x NT] slice of
// W in shared memory once and each warp-row gathers 16-byte weight vectors
// from it.
#include "spk_common.cuh"

namespace spk {

struct SpmmArgs {
  const int32_t* row_ptr;    // [T*(M+1)], relative to the plane
  const int64_t* plane_ptr;  // [T+1]
  const int32_t* col_idx;
  const float* values;       // may be null: unit values unless the tile flag says otherwise
  const float* S;            // source spikes (value gather for non-unit tiles)
  const uint8_t* tile_flags; // per scan tile: 1 if the tile holds positive values != 1
  int rows_per_tile;
  int64_t tiles_per_plane;
  const void* W;
  int64_t w_sk, w_sn;
  const float* bias;
  float* Y;
  int T;
  int64_t M;
  int K, N, NT;
  int64_t rows_per_cta;
  int64_t col_capacity;  // entries readable in col_idx / values
};

template <typename WT, int VEC>
__global__ void __launch_bounds__(256) spmm_csr_kernel(SpmmArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  WT* ws = reinterpret_cast<WT*>(smem_raw);  // [K][NT]
  const int NT = a.NT;
  const int n0 = blockIdx.x * NT;
  const WT* W = static_cast<const WT*>(a.W);

  // stage the weight slice once
  for (int64_t i = threadIdx.x; i < (int64_t)a.K * NT; i += blockDim.x) {
    const int k = (int)(i / NT), j = (int)(i % NT);
    const int n = n0 + j;
    ws[i] = (n < a.N) ? W[(int64_t)k * a.w_sk + (int64_t)n * a.w_sn] : WT(0.0f);
  }
  __syncthreads();

  const int LPR = NT / VEC;            // lanes per row
  const int RPW = 32 / LPR;            // rows per warp in flight
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, li = lane % LPR;
  const int nwarps = blockDim.x >> 5;
  const int64_t R = (int64_t)a.T * a.M;
  const int64_t r_begin = (int64_t)blockIdx.y * a.rows_per_cta;
  const int64_t r_end = min(R, r_begin + a.rows_per_cta);
  const int c0 = li * VEC;

  for (int64_t rb = r_begin + (int64_t)warp * RPW; rb < r_end; rb += (int64_t)nwarps * RPW) {
    const int64_t r = rb + sub;
    const bool active = (sub < RPW) && (r < r_end);
    float acc[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
    if (active) {
      const int t = (int)(r / a.M);
      const int64_t m = r - (int64_t)t * a.M;
      const int32_t* rp = a.row_ptr + (int64_t)t * (a.M + 1) + m;
      const int64_t p0 = a.plane_ptr[t] + rp[0];
      const int64_t p1 = min64(a.plane_ptr[t] + rp[1], a.col_capacity);  // an overflowed scan is reported, never over-read
      const bool unit = (a.values == nullptr) &&
                        (a.tile_flags == nullptr ||
                         a.tile_flags[(int64_t)t * a.tiles_per_plane + m / a.rows_per_tile] == 0);
      const float* srow = a.S + r * a.K;
      for (int64_t p = p0; p < p1; ++p) {
        const int col = a.col_idx[p];
        if ((unsigned)col >= (unsigned)a.K) continue;
        const float v = a.values ? a.values[p] : (unit ? 1.0f : srow[col]);
        const WT* wr = ws + (size_t)col * NT + c0;
        float w[VEC];
        if constexpr (sizeof(WT) == 4) {
          if constexpr (VEC == 4) {
            const float4 q = *reinterpret_cast<const float4*>(wr);
            w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) w[i] = (float)wr[i];
          }
        } else {
          const uint4 q = *reinterpret_cast<const uint4*>(wr);  // 8 bf16
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            w[2 * i] = f.x;
            w[2 * i + 1] = f.y;
          }
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = fmaf(v, w[i], acc[i]);
      }
      float* y = a.Y + r * a.N;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const int n = n0 + c0 + i;
        if (n < a.N) y[n] = a.bias ? acc[i] + a.bias[n] : acc[i];
      }
    }
  }
}

int launch_spmm_csr(const int32_t* row_ptr, const int64_t* plane_ptr, const int32_t* col_idx, const float* values,
                    const float* S, const uint8_t* tile_flags, int rows_per_tile, int64_t tiles_per_plane,
                    const void* W, int w_dtype, int64_t w_sk, int64_t w_sn, const float* bias, float* Y, int T,
                    int64_t M, int K, int N, int64_t col_capacity, cudaStream_t stream) {
  const size_t esz = (w_dtype == SPK_BF16) ? 2 : 4;
  const int vec = (w_dtype == SPK_BF16) ? 8 : 4;
  const size_t budget = 200 * 1024;
  int NT = 128;
  while (NT > vec && (size_t)K * NT * esz > budget) NT >>= 1;
  SPK_REQUIRE((size_t)K * NT * esz <= budget, "K=%d too large for the CSR branch weight tile", K);
  if (NT > 32 * vec) NT = 32 * vec;
  const int n_tiles = (int)ceil_div(N, NT);
  const int64_t R = (int64_t)T * M;
  const int sms = sm_count();
  int64_t groups = ceil_div(2 * sms, n_tiles);
  groups = groups < 1 ? 1 : groups;
  int64_t rows_per_cta = ceil_div(R, groups);
  groups = ceil_div(R, rows_per_cta);
  SPK_REQUIRE(groups <= 65535, "too many row groups");
  SpmmArgs a{row_ptr, plane_ptr, col_idx, values, S, tile_flags, rows_per_tile, tiles_per_plane,
             W, w_sk, w_sn, bias, Y, T, M, K, N, NT, rows_per_cta, col_capacity};
  const size_t smem = (size_t)K * NT * esz;
  dim3 grid((unsigned)n_tiles, (unsigned)groups);
  auto kern = (w_dtype == SPK_BF16) ? spmm_csr_kernel<__nv_bfloat16, 8> : spmm_csr_kernel<float, 4>;
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  prof_before(SPK_KERNEL_SPMM_CSR, stream);
  kern<<<grid, 256, smem, stream>>>(a);
  prof_after(SPK_KERNEL_SPMM_CSR, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

}  // namespace spk
