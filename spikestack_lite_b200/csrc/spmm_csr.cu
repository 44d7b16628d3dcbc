// CSR branch of spike-linear: Y = CSR(S) x W with a slice of W held in shared
// memory and reused by every row of all T planes.
//
// Reference: csr_coalesced_kernel (sparse_linear.cu:59-90), which sums the
// row's nonzeros in ascending column order with one fp32 fused multiply-add
// per term.  This kernel keeps exactly that order and rounding (fmaf from
// 0.0f, then + bias), so for fp32 W its output is bit-identical to the
// reference engine's.  What it changes is the data movement: the reference
// re-reads W^T from global memory for every nonzero of every plane (the
// multistep loop launches one SpMM per plane, sparse_linear.cu:667-688).
//
// Here a CTA owns one slice of NT output columns and a range of rows (all
// planes).  It stages W[:, slice] ([K][NT], K-major) in shared memory once --
// by TMA boxes of 256 rows when W is [K, N] row-major (the reference's
// weightT), by plain loads for other strides -- and then streams rows: a row
// is served by LPR = NT / VEC lanes, each owning VEC consecutive columns
// (one 16-byte gather of the weight row per nonzero).  The row's column
// indices are read LPR at a time with one coalesced load and broadcast to
// the row's lanes by shuffles, the next batch requested before the current
// one is consumed, so every lane keeps several gathers in flight; sixteen
// warps per CTA hide the remaining latency.  Cost: nnz x N fused
// multiply-adds fed from shared memory (2 bytes per FMA for bf16 W, 4 for
// fp32), plus the CSR read once per slice (from L2) and Y written once.
#include "tma.cuh"

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
  int n_tiles;           // column slices
  int64_t units_per_cta; // (slice, row) pairs per CTA, slice-major
  int64_t col_capacity;  // entries readable in col_idx / values
  int w_tma;             // 1: stage the slice with TMA boxes of w_box_rows rows
  int w_box_rows;
  int y_vec;             // Y 16-byte aligned and N % 4 == 0: vector stores
  const int* gate;       // automatic branch choice: run only when *gate == SPK_BRANCH_CSR (null: always)
};

constexpr int kSpmmThreads = 512;
constexpr size_t kSpmmSliceBudget = 200 * 1024;

// W [K, N] row-major (N contiguous), element size esz, boxes of box_cols x box_rows.
inline int make_map_weight(CUtensorMap* map, const void* W, int w_dtype, int64_t K, int64_t N, int64_t pitch,
                           int box_cols, int box_rows) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(SPK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const size_t esz = (w_dtype == SPK_BF16) ? 2 : 4;
  const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
  const cuuint64_t strides[1] = {(cuuint64_t)(pitch * esz)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, w_dtype == SPK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                         2, const_cast<void*>(W), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPK_ECUDA, "cuTensorMapEncodeTiled failed (%d) for the CSR weight slice", (int)r);
  return SPK_OK;
}

// Stage W[:, n0 : n0 + NT] as ws[k][j] (zero past N); row K (zero) is not touched.
// With TMA, `bar` (initialised by the caller) completes once per staging;
// `parity` is the staging's phase.
template <typename WT>
__device__ __forceinline__ bool stage_weight_slice(const CUtensorMap* wmap, const SpmmArgs& a, WT* ws, int n0,
                                                   uint64_t* bar, uint32_t parity) {
  const int NT = a.NT;
  if (a.w_tma) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)((size_t)a.K * NT * sizeof(WT)));
      for (int k0 = 0; k0 < a.K; k0 += a.w_box_rows)
        tma_load_2d(ws + (size_t)k0 * NT, wmap, n0, k0, bar);
    }
    if (mbar_wait(bar, parity, nullptr, SPK_DEV_PIPE_TIMEOUT)) return true;
    // gave up (reported): the boxes already issued still land before the CTA leaves
    mbar_wait(bar, parity, nullptr, SPK_DEV_PIPE_TIMEOUT);
    return false;
  }
  const WT* W = static_cast<const WT*>(a.W);
  const int64_t total = (int64_t)a.K * NT;
  if (a.w_sn <= a.w_sk) {  // n is the faster index in memory: consecutive threads take consecutive n
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
      const int k = (int)(i / NT), j = (int)(i % NT);
      const int n = n0 + j;
      ws[i] = (n < a.N) ? W[(int64_t)k * a.w_sk + (int64_t)n * a.w_sn] : WT(0.0f);
    }
  } else {  // k is the faster index (an nn.Linear weight [N, K]): consecutive threads take consecutive k
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
      const int j = (int)(i / a.K), k = (int)(i % a.K);
      const int n = n0 + j;
      ws[(size_t)k * NT + j] = (n < a.N) ? W[(int64_t)k * a.w_sk + (int64_t)n * a.w_sn] : WT(0.0f);
    }
  }
  return true;
}

template <typename WT, int VEC>
__device__ __forceinline__ void load_wvec(const WT* wr, float (&w)[VEC]) {
  if constexpr (sizeof(WT) == 4) {
    static_assert(VEC == 4, "fp32 weights: 4 per 16-byte gather");
    const float4 q = *reinterpret_cast<const float4*>(wr);
    w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
  } else {
    static_assert(VEC == 8, "bf16 weights: 8 per 16-byte gather");
    const uint4 q = *reinterpret_cast<const uint4*>(wr);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      w[2 * i] = f.x;
      w[2 * i + 1] = f.y;
    }
  }
}

// acc += w for unit spikes, VEC columns from one 16-byte gather, bit-identical
// to fmaf(1.0f, w, acc): bf16 W by the mixed-precision fma.rn.f32.bf16 on the
// packed halves (the product 1 x w is exact, so no conversion instructions),
// fp32 W by plain adds (1 x w + acc rounds once either way).
template <typename WT, int VEC>
__device__ __forceinline__ void acc_unit(const WT* wr, float (&acc)[VEC]) {
  const uint4 q = *reinterpret_cast<const uint4*>(wr);
  const uint32_t word[4] = {q.x, q.y, q.z, q.w};
  if constexpr (sizeof(WT) == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm("{\n\t.reg .b16 lo, hi, one;\n\t"
          "mov.b16 one, 0x3f80;\n\t"
          "mov.b32 {lo, hi}, %2;\n\t"
          "fma.rn.f32.bf16 %0, one, lo, %0;\n\t"
          "fma.rn.f32.bf16 %1, one, hi, %1;\n\t}"
          : "+f"(acc[2 * i]), "+f"(acc[2 * i + 1])
          : "r"(word[i]));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += __uint_as_float(word[i]);  // fmaf(1, w, acc) == acc + w
  }
}

// LPR lanes per row (VEC columns each), 32 / LPR rows per warp.  The warp
// walks its rows' nonzeros in lockstep, batch by batch up to the longest of
// its rows (a shorter row's lanes are predicated off), so the rows never
// diverge into serialised loops.
template <typename WT, int VEC, int LPR>
__global__ void __launch_bounds__(kSpmmThreads, 1) spmm_csr_kernel(const __grid_constant__ CUtensorMap wmap, SpmmArgs a) {
  if (gated_off(a.gate, SPK_BRANCH_CSR)) return;  // the automatic choice took the dense branch
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar;
  WT* ws = reinterpret_cast<WT*>(smem_aligned_1024(smem_raw));  // [K][NT]
  constexpr int RPW = 32 / LPR;  // rows per warp
  constexpr int NT = LPR * VEC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPR, li = lane % LPR;
  const int nwarps = blockDim.x >> 5;
  const int64_t R = (int64_t)a.T * a.M;
  const int c0 = li * VEC;
  if (a.w_tma && threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  for (int j = threadIdx.x; j < NT; j += blockDim.x) ws[(size_t)a.K * NT + j] = WT(0.0f);  // zero row K
  __syncthreads();
  // this CTA's work: the (slice, row) pairs [u, u_end) in slice-major order,
  // at most two slices, each staged once
  const int64_t total = (int64_t)a.n_tiles * R;
  int64_t u = (int64_t)blockIdx.x * a.units_per_cta;
  const int64_t u_end = min64(total, u + a.units_per_cta);
  uint32_t stagings = 0;
  while (u < u_end) {
    const int slice = (int)(u / R);
    const int64_t r_begin = u - (int64_t)slice * R;
    const int64_t r_end = min64(R, r_begin + (u_end - u));
    u += r_end - r_begin;
    const int n0 = slice * NT;
    __syncthreads();  // every gather of the previous slice is done
    const bool staged = stage_weight_slice<WT>(&wmap, a, ws, n0, &bar, stagings & 1u);
    ++stagings;
    if (!__syncthreads_and(staged)) return;  // a staging that gave up ends the whole CTA

    // Warp-uniform loop over row blocks of RPW rows, software-pipelined: the
    // next block's row pointers are requested while this block computes, and
    // each lane keeps SB batches of column indices in flight.
    constexpr int SB = 4;
    struct RowInfo {
      int64_t p0, n_r;
      int unit;
    };
    auto row_info = [&](int64_t rb) {
      RowInfo ri{0, 0, 1};
      const int64_t r = rb + sub;
      if (r < r_end) {
        const int t = (int)(r / a.M);
        const int64_t m = r - (int64_t)t * a.M;
        const int32_t* rp = a.row_ptr + (int64_t)t * (a.M + 1) + m;
        const int64_t pbase = a.plane_ptr[t];
        ri.p0 = pbase + rp[0];
        const int64_t p1 = min64(pbase + rp[1], a.col_capacity);  // an overflowed scan is reported, never over-read
        ri.n_r = p1 > ri.p0 ? p1 - ri.p0 : 0;
        ri.unit = (a.values == nullptr) &&
                  (a.tile_flags == nullptr || a.tile_flags[(int64_t)t * a.tiles_per_plane + m / a.rows_per_tile] == 0);
      }
      return ri;
    };
    auto load_cols = [&](const RowInfo& ri, int b, int (&c)[SB]) {
#pragma unroll
      for (int g = 0; g < SB; ++g) {
        const int e = b + g * LPR + li;
        c[g] = (e < ri.n_r) ? a.col_idx[ri.p0 + e] : -1;
      }
    };
    const int64_t stride = (int64_t)nwarps * RPW;
    int64_t rb = r_begin + (int64_t)warp * RPW;
    RowInfo cur = row_info(rb);
    int ci[SB];
    load_cols(cur, 0, ci);
    for (; rb < r_end; rb += stride) {
      const RowInfo nxt = row_info(rb + stride);  // requested now, used after this block
      const int64_t r = rb + sub;
      const bool live = r < r_end;
      const float* srow = a.S + (live ? r : 0) * (int64_t)a.K;
      const int n_max = __reduce_max_sync(0xffffffffu, (unsigned)cur.n_r);
      const bool any_real = __any_sync(0xffffffffu, !cur.unit);
      float acc[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
      for (int b = 0; b < n_max; b += SB * LPR) {
        int cn[SB];
        load_cols(cur, b + SB * LPR, cn);  // the next SB batches
        if (!any_real) {  // unit spikes (every row of the warp): no value shuffles, fused conversions
#pragma unroll
          for (int g = 0; g < SB; ++g) {
#pragma unroll
            for (int j = 0; j < LPR; ++j) {  // ascending column order
              const int col = __shfl_sync(0xffffffffu, ci[g], sub * LPR + j);
              const unsigned kr = min((unsigned)col, (unsigned)a.K);  // padding (-1) -> zero row K
              acc_unit<WT, VEC>(ws + (size_t)kr * NT + c0, acc);
            }
          }
#pragma unroll
          for (int g = 0; g < SB; ++g) ci[g] = cn[g];
          continue;
        }
#pragma unroll
        for (int g = 0; g < SB; ++g) {
          float vv = 1.0f;
          if (any_real && !cur.unit && ci[g] >= 0)
            vv = a.values ? a.values[cur.p0 + b + g * LPR + li]
                          : ((unsigned)ci[g] < (unsigned)a.K ? srow[ci[g]] : 0.0f);
#pragma unroll
          for (int j = 0; j < LPR; ++j) {  // ascending column order, one fmaf per term
            // branch-free: a padding entry reads the zero row K and adds v * (+0) with v = 1, which
            // leaves the accumulator bit-identical (it starts at +0 and never becomes -0)
            const int col = __shfl_sync(0xffffffffu, ci[g], sub * LPR + j);
            const float v = any_real ? __shfl_sync(0xffffffffu, vv, sub * LPR + j) : 1.0f;
            const int kr = (unsigned)col < (unsigned)a.K ? col : a.K;
            float w[VEC];
            load_wvec<WT, VEC>(ws + (size_t)kr * NT + c0, w);
#pragma unroll
            for (int i = 0; i < VEC; ++i) acc[i] = fmaf(v, w[i], acc[i]);
          }
        }
#pragma unroll
        for (int g = 0; g < SB; ++g) ci[g] = cn[g];
      }
      cur = nxt;
      load_cols(cur, 0, ci);  // the next block's first indices, before this block's stores
      if (!live) continue;
      float* y = a.Y + r * a.N + n0 + c0;
      if (a.y_vec && n0 + c0 + VEC <= a.N) {
        float o[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = a.bias ? acc[i] + a.bias[n0 + c0 + i] : acc[i];
#pragma unroll
        for (int i = 0; i < VEC; i += 4) *reinterpret_cast<float4*>(y + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const int n = n0 + c0 + i;
          if (n < a.N) y[i] = a.bias ? acc[i] + a.bias[n] : acc[i];
        }
      }
    }
  }
}

int launch_spmm_csr(const int32_t* row_ptr, const int64_t* plane_ptr, const int32_t* col_idx, const float* values,
                    const float* S, const uint8_t* tile_flags, int rows_per_tile, int64_t tiles_per_plane,
                    const void* W, int w_dtype, int64_t w_sk, int64_t w_sn, const float* bias, float* Y, int T,
                    int64_t M, int K, int N, int64_t col_capacity, cudaStream_t stream, const int* gate = nullptr) {
  const size_t esz = (w_dtype == SPK_BF16) ? 2 : 4;
  const int vec = (w_dtype == SPK_BF16) ? 8 : 4;
  // widest power-of-two slice (at most 32 lanes x VEC columns, at most N rounded up) that fits the budget
  int NT = 32 * vec;
  while (NT > vec && (NT / 2 >= N || (size_t)(K + 1) * NT * esz > kSpmmSliceBudget)) NT >>= 1;
  SPK_REQUIRE((size_t)(K + 1) * NT * esz <= kSpmmSliceBudget, "K=%d too large for the CSR branch weight slice", K);
  const int n_tiles = (int)ceil_div(N, NT);
  const int64_t R = (int64_t)T * M;
  const int sms = sm_count();
  // one CTA per SM, each with an equal share of the (slice, row) pairs
  const int64_t total = (int64_t)n_tiles * R;
  const int64_t per = ceil_div(total, (int64_t)sms);
  const int64_t grid_x = ceil_div(total, per);
  SpmmArgs a{row_ptr, plane_ptr, col_idx, values, S, tile_flags, rows_per_tile, tiles_per_plane,
             W, w_sk, w_sn, bias, Y, T, M, K, N, NT, n_tiles, per, col_capacity, 0, 0,
             ((reinterpret_cast<uintptr_t>(Y) & 15) == 0 && N % 4 == 0) ? 1 : 0, gate};
  // TMA staging when W is [K, N] row-major with a 16-byte aligned base and pitch, and the boxes tile K exactly
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  const int box_rows = K >= 256 ? 256 : K;
  if (w_sn == 1 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 && ((size_t)w_sk * esz) % 16 == 0 && K % box_rows == 0 &&
      w_sk >= N) {
    int rc = make_map_weight(&map, W, w_dtype, K, N, w_sk, NT, box_rows);
    if (rc) return rc;
    a.w_tma = 1;
    a.w_box_rows = box_rows;
  }
  const size_t smem = (size_t)(K + 1) * NT * esz + 1024;  // the slice, its zero row, alignment slack
  dim3 grid((unsigned)grid_x);
  void (*kern)(CUtensorMap, SpmmArgs) = nullptr;
  const int lpr = NT / vec;
#define SPK_SPMM_PICK(L)                                                                                    \
  if (lpr == L) kern = (w_dtype == SPK_BF16) ? spmm_csr_kernel<__nv_bfloat16, 8, L> : spmm_csr_kernel<float, 4, L>;
  SPK_SPMM_PICK(1) SPK_SPMM_PICK(2) SPK_SPMM_PICK(4) SPK_SPMM_PICK(8) SPK_SPMM_PICK(16) SPK_SPMM_PICK(32)
#undef SPK_SPMM_PICK
  SPK_REQUIRE(kern != nullptr, "no CSR kernel for %d lanes per row", lpr);
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  prof_before(SPK_KERNEL_SPMM_CSR, stream);
  kern<<<grid, kSpmmThreads, smem, stream>>>(map, a);
  prof_after(SPK_KERNEL_SPMM_CSR, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

}  // namespace spk
