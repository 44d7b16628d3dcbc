// Dense branch of spike-linear for fp32 weights: spikes straight from the TMA
// staging slot into the tensor cores (tcgen05 kind::tf32).
//
// Y[r, n] = sum_k relu'(S[r, k]) * W[k, n] (+ bias[n]) with relu'(x) = x if
// x > 0 else 0 (the reference engine's predicate, sparse_linear.cu:268).
// S arrives fp32 and spikes (0/1) are exact in tf32, so the A operand is the
// staging slot itself: TMA writes S with the 128-byte swizzle of a K-major
// UMMA operand (32 fp32 per swizzle row) and the MMA reads it from there.  W
// is split once per call into tf32 hi + lo halves (W = hi + lo to ~2^-22
// relative), two MMAs per k-step.  The converter warps no longer build the A
// operand; they read each slot once for the spike masks / row counts of the
// CSR pass and to screen it: a slot holding a value that tf32 does not carry
// exactly (low mantissa bits, negative, Inf/NaN) is rewritten in place by its
// warps as relu'(x) rounded to tf32 (hi pass), then as the remainder (lo pass,
// one more MMA with W hi), so every input is exact to ~2^-22 as well.
//
// Per slot: [128 rows x 64 columns] fp32 = two 16 KB swizzle-atom columns.
// Warp roles (704 threads): warp 0 TMA producer (S boxes of 32 columns x 128
// rows, weight chunks by 1-D bulk copy), warp 1 TMEM owner + MMA issuer,
// warps 2-17 converters (8 rows each), warps 18-21 epilogue (+ bias, store Y).
// Slot protocol: stg_full (TMA) -> chk (all converters screened; hi rewritten
// if needed) -> hi MMAs -> lo_go [-> the non-exact warps write lo -> lo_full
// -> lo MMAs] -> stg_empty (converters done reading/writing + the MMAs that
// read the slot).  Converter warps whose rows are exact never wait inside a
// slot: they arrive on chk, lo_full and stg_empty and move on.
// Every wait is bounded (2 s) and reports SPK_DEV_PIPE_TIMEOUT; issued copies
// and MMAs are drained and TMEM is freed on every exit.
#include "tma.cuh"

namespace spk {

namespace t32 {

constexpr int kRows = 128;                 // MMA M: one row tile
constexpr int kKChunk = 64;                // columns per staging slot
constexpr int kAtomBytes = kRows * 128;    // one swizzle-atom column of a slot: 128 rows x 32 fp32 = 16 KB
constexpr int kStgBytes = 2 * kAtomBytes;  // 32 KB
constexpr int kBoxRows = 32;              // TMA box: 32 fp32 columns x 32 rows = 4 KB (4 swizzle atoms)
constexpr int kBoxBytes = kBoxRows * 128;
constexpr int kConvWarps = 16;
constexpr int kThreads = 32 * (2 + kConvWarps + 4);
constexpr int kNS = 3;                     // staging slots
constexpr int kNB = 2;                     // weight chunk slots

template <int NT>
struct Cfg {
  static constexpr int kTileCols = ((NT + 31) / 32) * 32;
  static constexpr int kG = (256 / kTileCols) > 4 ? 4 : (256 / kTileCols);
  static constexpr int kAccCols = kG * kTileCols;
  static constexpr int kTmemCols = tc::pow2_at_least(2 * kAccCols, 32);
  static constexpr int kBAtom = NT * 128;            // one swizzle-atom column of the weight chunk
  static constexpr int kBBytes = 4 * kBAtom;         // hi (2 atoms) + lo (2 atoms)
  static constexpr size_t kRing = (size_t)kNS * kStgBytes + (size_t)kNB * kBBytes;
  // barriers (5 NS + 2 NB + 5), lo flags [NS][16] bytes, row counts [G][128], TMEM slot, abort flag
  static constexpr size_t kTail = 8 * (5 * kNS + 2 * kNB + 5) + kConvWarps * kNS + 4 * 128 * kG + 16;
  static_assert((8 * (5 * kNS + 2 * kNB + 5)) % 16 == 0, "lo flags 16-byte aligned");
  static constexpr size_t kSmemBytes = 1024 + kRing + ((kTail + 255) / 256) * 256;
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 128, "NT must be a multiple of 16 in [16, 128]");
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

}  // namespace t32

// Round to the nearest tf32 (ties away); values past the tf32 range keep
// their truncation so that hi stays finite.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  const float h = __uint_as_float(r);
  return isfinite(h) || !isfinite(x) ? h : __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

// Instruction descriptor: kind::tf32, A = B = tf32, D = f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_tf32_f32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Byte offset of (row r, 16-byte chunk c in [0, 8)) in a 128-byte-swizzled
// K-major atom column (rows of 128 bytes, 8-row atoms of 1024 bytes).
__host__ __device__ __forceinline__ uint32_t sw128_chunk(uint32_t r, uint32_t c) {
  return r * 128u + (((c ^ (r & 7u)) & 7u) << 4);
}

// Four fp32 values rounded to bf16 (nearest even), packed in memory order.
__device__ __forceinline__ uint2 bf16x4(float a, float b, float c, float d) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// ---------------------------------------------------------------- converters
// Converter warps of the tf32 dense kernels (both operand orders share the
// staging layout: 128 rows x 64 fp32 per slot, two 128-byte-swizzled atom
// columns).  Warp cw of CW = 16 screens rows [8cw, 8cw+8) of every slot,
// rewrites them for the exact hi/lo pass when needed, and emits the planar
// spike masks, row counts and block sums of the CSR pass.  kRelu: the
// spike-linear predicate relu'(x) (x if x > 0, else 0) is applied to S; the
// linear-activation op passes its input through unchanged (hi = x rounded
// to tf32, lo = the remainder).
template <int NS, int G, bool kRelu = true, bool kRev = false>
__device__ __forceinline__ void tf32_converter(const int cw, const int lane, unsigned char* stg, uint64_t* stg_full,
                                               uint64_t* chk, uint64_t* stg_empty, uint64_t* lo_go,
                                               uint64_t* lo_full, uint8_t* lo_flag, int* row_count,
                                               volatile int* abort_flag, const TcArgs& a, const int64_t r_begin,
                                               const int64_t r_end, const int n_tile, const int nk,
                                               const int groups, const int tiles) {
  constexpr int CW = t32::kConvWarps;
  // Warp cw screens rows [8cw, 8cw+8) of each slot; in load i a lane holds
  // columns 4(lane & 15) .. +3 of row 8cw + 2i + (lane >> 4) (16-byte chunk
  // lane & 7 of atom column (lane >> 3) & 1).  The masks keep the planar
  // format of the CSR pass: per row and 64-column chunk P0 = M0 | M1 << 16,
  // P1 = M2 | M3 << 16, bit m of plane Me = column 4m + e.
  const int half = lane >> 4;
  const int cl = lane & 15;
  const bool emit = (a.bitmap != nullptr) && n_tile == 0;
  const bool check_unit = emit && a.nonunit != nullptr;
  constexpr int RPW = t32::kRows / CW;  // rows per converter warp
  constexpr int NL = RPW / 2;           // 16-byte loads per lane and slot
  uint32_t soff[NL];
  int rls[NL];
#pragma unroll
  for (int i = 0; i < NL; ++i) {
    rls[i] = cw * RPW + 2 * i + half;
    soff[i] = (uint32_t)((cl >> 3) * t32::kAtomBytes) + sw128_chunk((uint32_t)rls[i], (uint32_t)(cl & 7));
  }
  const int my_i = (lane >> 1) & (NL - 1);
  const uint32_t my_sel = (lane & 1) ? 0x7632u : 0x5410u;
  int j = 0, s = 0;
  uint32_t ps = 0u;  // phase parity of the current use of slot s
  bool ok = true;
  for (int g = 0; g < groups && ok; ++g) {
    const int pg = kRev ? groups - 1 - g : g;  // the caller's group order
    const int tg = min(G, tiles - pg * G);
    for (int kc = 0; kc < nk && ok; ++kc) {
      for (int t = 0; t < tg; ++t) {
        if (!(ok = mbar_wait(&stg_full[s], ps, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        const int64_t row0 = r_begin + (int64_t)(pg * G + t) * t32::kRows;
        const int nrows = (int)min64(t32::kRows, r_end - row0);
        unsigned char* st = stg + s * t32::kStgBytes;
        uint4 v[NL];  // raw fp32 bits; rows past nrows count as zero
#pragma unroll
        for (int i = 0; i < NL; ++i) {
          v[i] = *reinterpret_cast<const uint4*>(st + soff[i]);
          if (rls[i] >= nrows) v[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        // Screen: a sign bit, low 13 mantissa bits or an all-ones exponent
        // (Inf/NaN; the OR of two other exponents can also give it, which
        // only costs speed) anywhere in the warp's rows -> exact path.
        uint32_t bits_or = 0u;
        bool nonunit = false;
        uint32_t m[NL][4];
#pragma unroll
        for (int i = 0; i < NL; ++i) {
          const uint4 b = v[i];
          bits_or |= b.x | b.y | b.z | b.w;
          if (check_unit) {
            nonunit |= (b.x != 0u && b.x != 0x3f800000u) || (b.y != 0u && b.y != 0x3f800000u) ||
                       (b.z != 0u && b.z != 0x3f800000u) || (b.w != 0u && b.w != 0x3f800000u);
          }
          if (emit) {
            m[i][0] = __ballot_sync(0xffffffffu, __uint_as_float(b.x) > 0.0f);
            m[i][1] = __ballot_sync(0xffffffffu, __uint_as_float(b.y) > 0.0f);
            m[i][2] = __ballot_sync(0xffffffffu, __uint_as_float(b.z) > 0.0f);
            m[i][3] = __ballot_sync(0xffffffffu, __uint_as_float(b.w) > 0.0f);
          }
        }
        const bool warp_lo =
            __any_sync(0xffffffffu, (bits_or & 0x80001fffu) != 0u || (bits_or & 0x7f800000u) == 0x7f800000u);
        float lo_v[NL][4];
        if (warp_lo) {
          // hi pass in place: relu'(x) rounded to tf32; the remainders wait in registers
#pragma unroll
          for (int i = 0; i < NL; ++i) {
            const float x[4] = {__uint_as_float(v[i].x), __uint_as_float(v[i].y), __uint_as_float(v[i].z),
                                __uint_as_float(v[i].w)};
            float h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float xr = (!kRelu || x[e] > 0.0f) ? x[e] : 0.0f;
              h[e] = tf32_rna(xr);
              lo_v[i][e] = isfinite(xr) ? tf32_rna(xr - h[e]) : 0.0f;
            }
            *reinterpret_cast<float4*>(st + soff[i]) = make_float4(h[0], h[1], h[2], h[3]);
          }
          fence_proxy_async_smem();
        }
        if (lane == 0) lo_flag[s * CW + cw] = warp_lo ? 1u : 0u;
        __syncwarp();
        if (lane == 0) mbar_arrive(&chk[s]);
        if (warp_lo) {
          // Lo pass, run by the warps whose rows were not exact: once every
          // warp has screened (chk) and the hi MMAs have read the slot
          // (lo_go), each writes its remainders, and the first of them
          // zeroes the rows of the exact warps, which have moved on.
          if (!(ok = mbar_wait(&chk[s], ps, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          uint32_t lo_mask = 0u;
#pragma unroll
          for (int w = 0; w < CW; ++w) lo_mask |= lo_flag[s * CW + w] ? (1u << w) : 0u;
          if (!(ok = mbar_wait(&lo_go[s], ps, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
#pragma unroll
          for (int i = 0; i < NL; ++i)
            *reinterpret_cast<float4*>(st + soff[i]) = make_float4(lo_v[i][0], lo_v[i][1], lo_v[i][2], lo_v[i][3]);
          if (cw == __ffs((int)lo_mask) - 1) {
            for (int w = 0; w < CW; ++w) {
              if ((lo_mask >> w) & 1u) continue;
#pragma unroll
              for (int i = 0; i < NL; ++i) {
                const uint32_t off = (uint32_t)((cl >> 3) * t32::kAtomBytes) +
                                     sw128_chunk((uint32_t)(w * RPW + 2 * i + half), (uint32_t)(cl & 7));
                *reinterpret_cast<float4*>(st + off) = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        // lo_full completes on every slot use (the MMA waits for it only on
        // a lo pass); the slot's data is consumed (the ballots used every
        // loaded value)
        if (lane == 0) {
          mbar_arrive(&lo_full[s]);
          mbar_arrive(&stg_empty[s]);
        }
        if (j == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (emit) {
          uint32_t q[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t x = m[0][e];
#pragma unroll
            for (int i = 1; i < NL; ++i) x = (my_i == i) ? m[i][e] : x;
            q[e] = x;
          }
          const uint32_t keep0 = __byte_perm(q[0], q[1], my_sel);
          const uint32_t keep1 = __byte_perm(q[2], q[3], my_sel);
          const int rl = cw * RPW + lane;
          if (lane < RPW && rl < nrows) {
            const int64_t grow = row0 + rl;
            const int idx = t * t32::kRows + rl;
            const int c = __popc(keep0) + __popc(keep1);
            const int total = (kc == 0 ? 0 : row_count[idx]) + c;
            row_count[idx] = total;
            *reinterpret_cast<uint2*>(a.bitmap + grow * a.KWP + 2 * kc) = make_uint2(keep0, keep1);
            if (kc == nk - 1 && a.row_cnt) a.row_cnt[grow] = total;
          }
          if (kc == nk - 1 && a.blk_sum) {
            // the warp's 8 rows lie in one 128-row block: one atomic per warp and level
            int cnt = (lane < RPW && rl < nrows) ? row_count[t * t32::kRows + rl] : 0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
            const int64_t g0 = row0 + cw * RPW;
            if (lane == 0 && cw * RPW < nrows && cnt) {
              atomicAdd(&a.blk_sum[g0 >> 7], cnt);
              atomicAdd(&a.sup_sum[g0 >> 14], (unsigned long long)cnt);
            }
          }
        }
        if (check_unit && __any_sync(0xffffffffu, nonunit) && lane == 0) atomicOr(a.nonunit, 1);
        ++j;
        if (++s == NS) {
          s = 0;
          ps ^= 1u;
        }
      }
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(t32::kThreads, 1)
    spike_linear_tf32_kernel(const __grid_constant__ CUtensorMap tmap_s, TcArgs a) {
  if (gated_off(a.gate, SPK_BRANCH_DENSE)) return;  // the automatic choice took the CSR branch
  using C = t32::Cfg<NT>;
  constexpr int G = C::kG, NS = t32::kNS, NB = t32::kNB, CW = t32::kConvWarps;
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  unsigned char* base = smem_aligned_1024(smem_dyn);
  unsigned char* stg = base;                                   // [NS][2 atoms x 16 KB] fp32 staging = A operand
  unsigned char* bst = stg + NS * t32::kStgBytes;               // [NB][hi 2 atoms | lo 2 atoms]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bst + NB * C::kBBytes);
  uint64_t* stg_full = bars;
  uint64_t* chk = stg_full + NS;
  uint64_t* stg_empty = chk + NS;
  uint64_t* lo_go = stg_empty + NS;
  uint64_t* lo_full = lo_go + NS;
  uint64_t* b_full = lo_full + NS;
  uint64_t* b_empty = b_full + NB;
  uint64_t* acc_full = b_empty + NB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint8_t* lo_flag = reinterpret_cast<uint8_t*>(drain + 1);      // [NS][CW] bytes, 16-byte aligned
  int* row_count = reinterpret_cast<int*>(lo_flag + NS * CW);      // [G][128]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(row_count + G * t32::kRows);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r_begin = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t r_end = min64(a.R, r_begin + a.rows_per_cta);
  const int n_tile = blockIdx.y;
  const int n0 = n_tile * NT;
  const int nk = a.nk;
  const int tiles = r_end > r_begin ? (int)ceil_div(r_end - r_begin, t32::kRows) : 0;
  const int groups = (tiles + G - 1) / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&stg_full[s], 1);
      mbar_init(&chk[s], CW);
      mbar_init(&stg_empty[s], CW + 1);
      mbar_init(&lo_go[s], 1);
      mbar_init(&lo_full[s], CW);
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent of the kernel before it.  When that is the
  // weight-image kernel (a plain launch, so S was complete before it
  // started; a.early_s) the producer requests the first slots of S before its
  // wait, and the converters screen them before theirs (ahead of their first
  // global write); otherwise (a prepared image: the previous kernel may be
  // the one writing S) every warp waits first.
  const bool late_dep = a.early_s && ((warp == 0 && lane == 0) || (warp >= 2 && warp < 2 + CW));
  if (!late_dep) asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_map(&tmap_s);
      auto load_s = [&](int s, int64_t row0, int kc) {
        // 32-row boxes up to the tile's last valid row: no reads past the CTA's range
        // (rows a box leaves out keep stale data; the converters and the epilogue ignore them)
        const int nbox = (int)ceil_div(min64(t32::kRows, r_end - row0), t32::kBoxRows);
        mbar_arrive_expect_tx(&stg_full[s], (uint32_t)(2 * nbox * t32::kBoxBytes));
        for (int b = 0; b < nbox; ++b) {
          unsigned char* dst = stg + s * t32::kStgBytes + b * t32::kBoxBytes;
          const int y = (int)row0 + b * t32::kBoxRows;
          tma_load_2d(dst, &tmap_s, kc * t32::kKChunk, y, &stg_full[s]);
          tma_load_2d(dst + t32::kAtomBytes, &tmap_s, kc * t32::kKChunk + 32, y, &stg_full[s]);
        }
      };
      int pre = 0;  // slots requested before the wait: the first NS (or all), only when S is known complete
      for (int g = 0; g < groups && pre < NS && a.early_s; ++g) {
        const int tg = min(G, tiles - g * G);
        for (int kc = 0; kc < nk && pre < NS; ++kc)
          for (int t = 0; t < tg && pre < NS; ++t, ++pre) load_s(pre, r_begin + (int64_t)(g * G + t) * t32::kRows, kc);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int j = 0, jb = 0;
      bool ok = true;
      for (int g = 0; g < groups && ok; ++g) {
        const int tg = min(G, tiles - g * G);
        for (int kc = 0; kc < nk && ok; ++kc) {
          const int sb = jb % NB;
          if (jb >= NB && !(ok = mbar_wait(&b_empty[sb], ((jb / NB) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
            break;
          mbar_arrive_expect_tx(&b_full[sb], C::kBBytes);
          bulk_g2s(bst + (size_t)sb * C::kBBytes, a.wimg + ((size_t)n_tile * nk + kc) * C::kBBytes, C::kBBytes,
                   &b_full[sb]);
          ++jb;
          for (int t = 0; t < tg; ++t, ++j) {
            if (j < pre) continue;
            const int s = j % NS;
            if (j >= NS && !(ok = mbar_wait(&stg_empty[s], ((j / NS) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
              break;
            load_s(s, r_begin + (int64_t)(g * G + t) * t32::kRows, kc);
          }
        }
      }
      // copies still in flight land before the CTA exits (early exits included)
      const int issued = max(j, pre);
      for (int i = (issued > NS ? issued - NS : 0); i < issued; ++i)
        mbar_wait(&stg_full[i % NS], (i / NS) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
      for (int i = (jb > NB ? jb - NB : 0); i < jb; ++i)
        mbar_wait(&b_full[i % NB], (i / NB) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_tf32_f32(t32::kRows, NT);
      int j = 0, jb = 0;
      bool ok = true;
      for (int g = 0; g < groups && ok; ++g) {
        const int tg = min(G, tiles - g * G);
        const int ab = g & 1;
        if (g >= 2 && !(ok = mbar_wait(&acc_empty[ab], ((g / 2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        tc_fence_after();
        for (int kc = 0; kc < nk && ok; ++kc) {
          const int sb = jb % NB;
          if (!(ok = mbar_wait(&b_full[sb], (jb / NB) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          const uint32_t bsm = smem_u32(bst + (size_t)sb * C::kBBytes);
          for (int t = 0; t < tg; ++t) {
            const int s = j % NS;
            if (!(ok = mbar_wait(&chk[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
            tc_fence_after();
            const uint4 lf = *reinterpret_cast<const uint4*>(lo_flag + s * CW);  // the 16 warps' flags
            const bool lo_any = (lf.x | lf.y | lf.z | lf.w) != 0u;
            const uint32_t d = tmem + (uint32_t)(ab * C::kAccCols + t * C::kTileCols);
            const uint32_t asm_ = smem_u32(stg + s * t32::kStgBytes);
#pragma unroll
            for (int kk = 0; kk < t32::kKChunk / 8; ++kk) {
              const uint32_t atom = (uint32_t)(kk >> 2), kof = (uint32_t)(kk & 3) * 32u;
              const uint64_t da = umma_desc_sw128_kmajor(asm_ + atom * t32::kAtomBytes + kof);
              const uint64_t dbh = umma_desc_sw128_kmajor(bsm + atom * C::kBAtom + kof);
              const uint64_t dbl = umma_desc_sw128_kmajor(bsm + (2 + atom) * C::kBAtom + kof);
              umma_tf32_ss(d, da, dbh, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
              umma_tf32_ss(d, da, dbl, idesc, 1u);
            }
            // lo_go and lo_full complete once per slot use, lo pass or not, so
            // that the phase parity of a use is (j / NS) & 1 for every waiter
            umma_commit(&lo_go[s]);
            if (lo_any) {
              // the slot's warps rewrite it with the remainders once the hi MMAs have read it
              if (!(ok = mbar_wait(&lo_full[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < t32::kKChunk / 8; ++kk) {
                const uint32_t atom = (uint32_t)(kk >> 2), kof = (uint32_t)(kk & 3) * 32u;
                const uint64_t da = umma_desc_sw128_kmajor(asm_ + atom * t32::kAtomBytes + kof);
                const uint64_t dbh = umma_desc_sw128_kmajor(bsm + atom * C::kBAtom + kof);
                umma_tf32_ss(d, da, dbh, idesc, 1u);
              }
            }
            umma_commit(&stg_empty[s]);
            ++j;
          }
          if (!ok) break;
          umma_commit(&b_empty[sb]);
          ++jb;
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      if (!ok) {  // issued MMAs finish before TMEM and shared memory are released
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);
      }
    }
  } else if (warp < 2 + CW) {
    tf32_converter<NS, G>(warp - 2, lane, stg, stg_full, chk, stg_empty, lo_go, lo_full, lo_flag, row_count, abort_flag,
                          a, r_begin, r_end, n_tile, nk, groups, tiles);
  } else {
    // ---------------------------------------------------------------- epilogue (warps 18-21)
    // 16-lane x 256-bit TMEM loads: four threads per row, so every store
    // instruction writes whole 32-byte sectors of eight rows (one row per lane
    // would touch 32 lines per instruction and hold up the converters' loads).
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int ar = lane >> 2, cp = (lane & 3) * 2;
    for (int g = 0; g < groups; ++g) {
      const int tg = min(G, tiles - g * G);
      const int ab = g & 1;
      if (!mbar_wait(&acc_full[ab], (g / 2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
      tc_fence_after();
      for (int t = 0; t < tg; ++t) {
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {
          const int64_t rowA = r_begin + (int64_t)(g * G + t) * t32::kRows + q * 32 + h2 * 16 + ar;
          const int64_t rowB = rowA + 8;
          const uint32_t tb = tmem + ((uint32_t)(q * 32 + h2 * 16) << 16) +
                              (uint32_t)(ab * C::kAccCols + t * C::kTileCols);
#pragma unroll 1
          for (int cb = 0; cb < NT; cb += 32) {
            float v[16];
            if (cb + 32 <= NT) tmem_ld_16x256b_x4(tb + (uint32_t)cb, v);
            else tmem_ld_16x256b_x2(tb + (uint32_t)cb, v);
            tmem_wait_ld();
            tmem_reg_fence(v);
#pragma unroll
            for (int jb = 0; jb < 4; ++jb) {
              const int n = n0 + cb + 8 * jb + cp;
              if (cb + 8 * jb >= NT) break;
#pragma unroll
              for (int rr = 0; rr < 2; ++rr) {
                const int64_t row = rr ? rowB : rowA;
                if (row >= r_end) continue;
                float x0 = v[4 * jb + 2 * rr], x1 = v[4 * jb + 2 * rr + 1];
                float* y = a.Y + row * a.N + n;
                if (a.y_vec && n + 2 <= a.N) {
                  if (a.bias) {
                    x0 += a.bias[n];
                    x1 += a.bias[n + 1];
                  }
                  *reinterpret_cast<float2*>(y) = make_float2(x0, x1);
                } else {
                  if (n < a.N) y[0] = a.bias ? x0 + a.bias[n] : x0;
                  if (n + 1 < a.N) y[1] = a.bias ? x1 + a.bias[n + 1] : x1;
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }
  role_join();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Weight image for the tf32 kernels: for N-tile t and 64-wide K-chunk c,
// [hi atom 0 | hi atom 1 | lo atom 0 | lo atom 1], each NT rows x 32 tf32 in
// the 128-byte-swizzled K-major layout (one bulk copy per chunk), hi =
// rna_tf32(w), lo = rna_tf32(w - hi).  A second region at img_b16 holds the
// bf16 operand of the linear op's correction pass: per (t, c) [bf16(w - hi)
// k0..63 | bf16(hi) k0..63], NT rows x 64 bf16 each in the same swizzle (hi
// of a non-finite w is 0 there: the tf32 pass carries it).  A third region at
// img_b16x3 holds the packed-spike kernel's operand: per (t, c) [b1 k0..63 |
// b2 k0..63 | b3 k0..63] with b1 = bf16(w), b2 = bf16(w - b1), b3 = bf16(w -
// b1 - b2) (w to ~2^-24 relative; the remainders are exact in fp32; b2 = b3 =
// 0 for non-finite w).  Also clears `zero_words` words at `zero` (the CSR
// pass state of the same call).
template <typename WT>
__global__ void w_image_tf32_kernel(const WT* W, int64_t sk, int64_t sn, int K, int N, int NT, int nk,
                                    unsigned char* img, unsigned char* img_b16, unsigned char* img_b16x3,
                                    uint32_t* zero, int64_t zero_words) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t npad = (int64_t)((N + NT - 1) / NT) * NT;
  const int64_t total = npad * nk * 16;  // one thread per (n, 4 k); n fastest: coalesced along W rows
  const size_t atom = (size_t)NT * 128;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < zero_words; i += nthr) zero[i] = 0u;
  for (int64_t i = tid; i < total; i += nthr) {
    const int64_t ng = i % npad;
    const int64_t kq = i / npad;         // global 4-column group
    const int kc = (int)(kq / 16), k4 = (int)(kq % 16);
    const int t = (int)(ng / NT), nl = (int)(ng % NT);
    float h[4], l[4], r[4], hb[4], b1[4], b2[4], b3[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = kc * 64 + k4 * 4 + e;
      float x = 0.0f;
      if (k < K && ng < N) x = static_cast<float>(W[(int64_t)k * sk + ng * sn]);
      h[e] = tf32_rna(x);
      const bool fin = isfinite(x);
      r[e] = fin ? x - h[e] : 0.0f;  // exact in fp32
      l[e] = tf32_rna(r[e]);
      hb[e] = fin ? h[e] : 0.0f;
      b1[e] = __bfloat162float(__float2bfloat16_rn(x));
      const float r1 = fin ? x - b1[e] : 0.0f;  // exact in fp32
      b2[e] = __bfloat162float(__float2bfloat16_rn(r1));
      b3[e] = r1 - b2[e];                        // exact; rounded below
    }
    unsigned char* blk = img + ((size_t)t * nk + kc) * 4 * atom;
    const uint32_t off = (uint32_t)((k4 >> 3) * atom) + sw128_chunk((uint32_t)nl, (uint32_t)(k4 & 7));
    *reinterpret_cast<float4*>(blk + off) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(blk + 2 * atom + off) = make_float4(l[0], l[1], l[2], l[3]);
    // bf16: columns 4 k4 .. 4 k4 + 3 are the half chunk (k4 & 1) of 16-byte chunk k4 >> 1
    unsigned char* b16 = img_b16 + ((size_t)t * nk + kc) * 2 * atom;
    const uint32_t off16 = sw128_chunk((uint32_t)nl, (uint32_t)(k4 >> 1)) + (uint32_t)(k4 & 1) * 8u;
    *reinterpret_cast<uint2*>(b16 + off16) = bf16x4(r[0], r[1], r[2], r[3]);
    *reinterpret_cast<uint2*>(b16 + atom + off16) = bf16x4(hb[0], hb[1], hb[2], hb[3]);
    unsigned char* b3x = img_b16x3 + ((size_t)t * nk + kc) * 3 * atom;
    *reinterpret_cast<uint2*>(b3x + off16) = bf16x4(b1[0], b1[1], b1[2], b1[3]);
    *reinterpret_cast<uint2*>(b3x + atom + off16) = bf16x4(b2[0], b2[1], b2[2], b2[3]);
    *reinterpret_cast<uint2*>(b3x + 2 * atom + off16) = bf16x4(b3[0], b3[1], b3[2], b3[3]);
  }
}

// ---------------------------------------------------------------- host side
// The tf32 region (hi and lo, 4 atoms per tile and chunk), the bf16 region of
// the linear op's correction pass (2 atoms), the three-way bf16 split (3 atoms).
inline size_t tf32_img_region_bytes(const TcPlan& p) { return (size_t)p.n_tiles * p.nk * p.NT * 512; }
inline size_t img_b16_region_bytes(const TcPlan& p) { return (size_t)p.n_tiles * p.nk * p.NT * 256; }
inline size_t img_b16x3_offset(const TcPlan& p) { return tf32_img_region_bytes(p) + img_b16_region_bytes(p); }
inline size_t tf32_img_bytes(const TcPlan& p) { return img_b16x3_offset(p) + (size_t)p.n_tiles * p.nk * p.NT * 384; }

template <int NT>
int launch_tf32_inst(const CUtensorMap& map, TcArgs a, int n_tiles, cudaStream_t stream) {
  using C = t32::Cfg<NT>;
  auto kern = spike_linear_tf32_kernel<NT>;
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes));
  const int sms = sm_count();
  const int ranges = sms / n_tiles > 0 ? sms / n_tiles : 1;
  a.rows_per_cta = ceil_div(ceil_div(a.R, ranges), 32) * 32;
  const int64_t gx = ceil_div(a.R, a.rows_per_cta);
  dim3 grid((unsigned)gx, (unsigned)n_tiles);
  prof_before(SPK_KERNEL_DENSE, stream);
  SPK_CUDA_TRY(launch_dependent(kern, grid, dim3(t32::kThreads), C::kSmemBytes, stream, map, a));
  prof_after(SPK_KERNEL_DENSE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_w_image_tf32(const void* W, int64_t sk, int64_t sn, int K, int N, const TcPlan& p, unsigned char* img,
                        uint32_t* zero, int64_t zero_words, cudaStream_t stream) {
  const int64_t total = (int64_t)p.n_tiles * p.NT * p.nk * 16;
  const int threads = 256;
  const int blocks = (int)min64(ceil_div(max64(total, zero_words), threads), 8192);
  prof_before(SPK_KERNEL_W_IMAGE, stream);
  w_image_tf32_kernel<float><<<blocks, threads, 0, stream>>>(static_cast<const float*>(W), sk, sn, K, N, p.NT, p.nk,
                                                             img, img + tf32_img_region_bytes(p),
                                                             img + img_b16x3_offset(p), zero, zero_words);
  prof_after(SPK_KERNEL_W_IMAGE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_tf32(const float* S, int64_t R, int K, int N, const TcPlan& p, const unsigned char* img, const TcOut& o,
                cudaStream_t stream) {
  CUtensorMap map;
  int rc = make_map_2d_swizzled_f32(&map, S, R, K, K, 32, t32::kBoxRows, "S");
  if (rc) return rc;
  TcArgs a{};
  a.R = R;
  a.K = K;
  a.N = N;
  a.nk = p.nk;
  a.KWP = 2 * p.nk;
  a.wimg = img;
  a.bias = o.bias;
  a.Y = o.Y;
  a.y_vec = ((N & 3) == 0 && (reinterpret_cast<uintptr_t>(o.Y) & 15) == 0) ? 1 : 0;
  a.bitmap = o.bitmap;
  a.row_cnt = o.row_cnt;
  a.nonunit = o.nonunit;
  a.blk_sum = o.blk_sum;
  a.sup_sum = o.sup_sum;
  a.gate = o.gate;
  a.early_s = o.early_s;
  switch (p.NT) {
    case 16: return launch_tf32_inst<16>(map, a, p.n_tiles, stream);
    case 32: return launch_tf32_inst<32>(map, a, p.n_tiles, stream);
    case 48: return launch_tf32_inst<48>(map, a, p.n_tiles, stream);
    case 64: return launch_tf32_inst<64>(map, a, p.n_tiles, stream);
    case 128: return launch_tf32_inst<128>(map, a, p.n_tiles, stream);
    default: break;
  }
  return fail(SPK_EUNSUPPORTED, "no tf32 dense tile for N=%d", N);
}

}  // namespace spk
