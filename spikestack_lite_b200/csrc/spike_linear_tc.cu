// Dense branch of spike-linear on the 5th-generation tensor cores.
//
// Y[r, n] = sum_k relu'(S[r, k]) * W[k, n] (+ bias[n]), relu'(x) = x if x > 0
// else 0 -- the reference engine's predicate (sparse_linear.cu:268) -- as a
// K-major bf16 x bf16 -> fp32 tcgen05 contraction with TMEM accumulators.
// Spikes are exact in bf16; fp32 operands are split into hi + lo bf16 halves
// so that products keep ~2^-17 relative accuracy:
//   W (fp32)  ->  W_hi + W_lo        two MMAs per k-step
//   S (fp32)  ->  S_hi [+ S_lo]      S_lo only for a stage holding a value that
//                                    bf16 does not represent (never for spikes)
//
// Work split: CTA (x, y) owns a contiguous range of rows (multiple of 32,
// balanced over all SMs) for N-tile y.  Its rows are processed in groups of
// G row tiles of 128; inside a group the K loop is outermost, so each weight
// chunk is brought in once and used by all G tiles, whose accumulators sit
// side by side in TMEM.  Two accumulator buffers let the epilogue of group g
// overlap the MMAs of group g+1.
//
// Warp roles (704 threads):
//   warp 0     TMA producer: S tiles via a 2-D tensor map (fp32, 32-row x
//              64-column boxes, zero fill past the tensor edge) into a 3-slot
//              staging ring; weight chunks of the pre-split image by 1-D bulk
//              copy.  Every copy lands in this CTA's own shared memory.
//   warp 1     TMEM owner and MMA issuer (one thread).
//   warps 2-17 converters: staging fp32 -> predicate -> bf16 hi [/lo] in the
//              128-byte-swizzled K-major A layout; optionally the packed spike
//              bitmap and per-row counts the CSR pass consumes.
//   warps 18-21 epilogue: tcgen05.ld (16 lanes x 256 bits) of their TMEM lane
//              quarter, + bias, sector-filling stores of Y.
// Every wait is bounded (2 s) and reports SPK_DEV_PIPE_TIMEOUT; each role then
// leaves its loop, issued copies and MMAs are drained, TMEM is freed.
#include "tma.cuh"

namespace spk {

namespace tc {

constexpr int kRows = 128;              // MMA M: one row tile
constexpr int kKChunk = 64;             // bf16 elements per 128-byte swizzle row
constexpr int kABytes = kRows * 128;    // one A half (hi or lo) of a stage: 16 KB
constexpr int kStgBytes = kRows * 256;  // fp32 staging of one stage: 32 KB
constexpr int kBoxRows = 32;            // TMA box: 32 rows x 64 fp32 = 8 KB
constexpr int kBoxBytes = kBoxRows * 256;
constexpr int kConvWarps = 16;          // converter warps (8 rows each per stage)
constexpr int kThreads = 32 * (2 + kConvWarps + 4);
constexpr int kNS = 3;                  // staging slots
constexpr int kNA = 2;                  // A slots (hi + lo each)
constexpr int kNB = 2;                  // weight chunk slots

__host__ __device__ constexpr int pow2_at_least(int x, int lo) {
  int p = lo;
  while (p < x) p <<= 1;
  return p;
}

template <int NT, bool WSPLIT>
struct Cfg {
  static constexpr int kTileCols = ((NT + 31) / 32) * 32;          // TMEM columns per row tile
  static constexpr int kG = (256 / kTileCols) > 4 ? 4 : (256 / kTileCols);  // row tiles per group
  static constexpr int kAccCols = kG * kTileCols;                    // one accumulator buffer
  static constexpr int kTmemCols = pow2_at_least(2 * kAccCols, 32);
  static constexpr int kBHalf = NT * 128;
  static constexpr int kBBytes = kBHalf * (WSPLIT ? 2 : 1);
  static constexpr size_t kRing = (size_t)kNS * kStgBytes + (size_t)kNA * 2 * kABytes + (size_t)kNB * kBBytes;
  // barriers (2NS + 2NA + 2NB + 5 words), lo flags [NA][4], row counts [G][128], TMEM slot, abort flag
  static constexpr size_t kTail = 8 * (2 * kNS + 2 * kNA + 2 * kNB + 5) + 4 * kConvWarps * kNA + 4 * 128 * kG + 16;
  static constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + kRing + ((kTail + 255) / 256) * 256;
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "NT must be a multiple of 16 in [16, 256]");
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

}  // namespace tc

struct TcArgs {
  int64_t R;              // rows (T*M)
  int K, N, nk, KWP;      // nk: 64-wide K chunks; KWP = 2*nk: planar bitmap words per row
  const unsigned char* wimg;
  const unsigned char* wimg_b16;  // the image's bf16 region (the linear op's correction pass), or null
  const unsigned char* wimg_b16x3;  // the image's three-way bf16 split (the packed-spike kernel), or null
  const float* bias;
  float* Y;
  int y_vec;              // Y 16-byte aligned and N % 4 == 0
  int64_t rows_per_cta;   // multiple of 32
  uint32_t* bitmap;       // [R][KWP] planar spike masks (see the converter), or null
  int32_t* row_cnt;       // [R] spikes per row, or null
  int* nonunit;           // set to 1 when a positive value other than 1 is seen
  int32_t* blk_sum;       // spikes per 128-row block (for the CSR scan's prefixes)
  unsigned long long* sup_sum;  // spikes per 16384-row super-block
  float thr;              // threshold of the spiking epilogues of the linear-activation op
  const int* gate;        // automatic branch choice: run only when *gate == SPK_BRANCH_DENSE (null: always)
  const uint32_t* bits_in;  // packed spikes [R][K/32] (the weights-in-TMEM kernel's packed input), or null
  GsmcCell cell;          // the GSMC recurrence's epilogue (weights-in-TMEM kernel, kEpiGsmc)
  int early_s;            // 1: the weight-image kernel (a plain launch) directly precedes this programmatic
                          // dependent, so S is complete and may be read before griddepcontrol.wait
};

template <int NT, bool WSPLIT>
__global__ void __launch_bounds__(tc::kThreads, 1)
    spike_linear_tc_kernel(const __grid_constant__ CUtensorMap tmap_s, TcArgs a) {
  if (gated_off(a.gate, SPK_BRANCH_DENSE)) return;  // the automatic choice took the CSR branch
  using C = tc::Cfg<NT, WSPLIT>;
  constexpr int G = C::kG, NS = tc::kNS, NA = tc::kNA, NB = tc::kNB;
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  unsigned char* base = smem_aligned_1024(smem_dyn);
  unsigned char* stg = base;                                     // [NS][32 KB] fp32 staging
  unsigned char* a_hi = stg + NS * tc::kStgBytes;                // [NA][16 KB]
  unsigned char* a_lo = a_hi + NA * tc::kABytes;                 // [NA][16 KB]
  unsigned char* bst = a_lo + NA * tc::kABytes;                  // [NB][kBBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bst + (size_t)NB * C::kBBytes);
  uint64_t* stg_full = bars;
  uint64_t* stg_empty = stg_full + NS;
  uint64_t* a_full = stg_empty + NS;
  uint64_t* a_empty = a_full + NA;
  uint64_t* b_full = a_empty + NA;
  uint64_t* b_empty = b_full + NB;
  uint64_t* acc_full = b_empty + NB;   // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* drain = acc_empty + 2;
  int* lo_flag = reinterpret_cast<int*>(drain + 1);              // [NA][kConvWarps]
  int* row_count = lo_flag + NA * tc::kConvWarps;               // [G][128]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(row_count + G * tc::kRows);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r_begin = (int64_t)blockIdx.x * a.rows_per_cta;
  const int64_t r_end = min64(a.R, r_begin + a.rows_per_cta);
  const int n_tile = blockIdx.y;
  const int n0 = n_tile * NT;
  const int nk = a.nk;
  const int tiles = r_end > r_begin ? (int)ceil_div(r_end - r_begin, tc::kRows) : 0;
  const int groups = (tiles + G - 1) / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&stg_full[s], 1);
      mbar_init(&stg_empty[s], tc::kConvWarps);
    }
    for (int s = 0; s < NA; ++s) {
      mbar_init(&a_full[s], tc::kConvWarps);
      mbar_init(&a_empty[s], 1);
      for (int w = 0; w < tc::kConvWarps; ++w) lo_flag[tc::kConvWarps * s + w] = 0;
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
  // Launched as a programmatic dependent of the weight-image kernel: the
  // prologue above overlaps its tail; its outputs (image, cleared scan state)
  // are read only after this wait.  The CSR scan may launch early in turn.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_map(&tmap_s);
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
          for (int t = 0; t < tg; ++t) {
            const int s = j % NS;
            if (j >= NS && !(ok = mbar_wait(&stg_empty[s], ((j / NS) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
              break;
            const int64_t row0 = r_begin + (int64_t)(g * G + t) * tc::kRows;
            const int nrows = (int)min64(tc::kRows, r_end - row0);
            const int nbox = (nrows + tc::kBoxRows - 1) / tc::kBoxRows;
            mbar_arrive_expect_tx(&stg_full[s], nbox * tc::kBoxBytes);
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(stg + s * tc::kStgBytes + b * tc::kBoxBytes, &tmap_s, kc * tc::kKChunk,
                          (int)(row0 + b * tc::kBoxRows), &stg_full[s]);
            ++j;
          }
        }
      }
      // every issued copy lands before the CTA can leave
      for (int i = (j > NS ? j - NS : 0); i < j; ++i)
        mbar_wait(&stg_full[i % NS], (i / NS) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
      for (int i = (jb > NB ? jb - NB : 0); i < jb; ++i)
        mbar_wait(&b_full[i % NB], (i / NB) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(tc::kRows, NT);
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
          const uint64_t db_hi = umma_desc_sw128_kmajor(smem_u32(bst + (size_t)sb * C::kBBytes));
          const uint64_t db_lo = umma_desc_sw128_kmajor(smem_u32(bst + (size_t)sb * C::kBBytes + C::kBHalf));
          for (int t = 0; t < tg; ++t) {
            const int sa = j % NA;
            if (!(ok = mbar_wait(&a_full[sa], (j / NA) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
            tc_fence_after();
            const uint64_t da_hi = umma_desc_sw128_kmajor(smem_u32(a_hi + sa * tc::kABytes));
            const uint64_t da_lo = umma_desc_sw128_kmajor(smem_u32(a_lo + sa * tc::kABytes));
            int lo_any = 0;
#pragma unroll
            for (int w = 0; w < tc::kConvWarps; ++w) lo_any |= lo_flag[tc::kConvWarps * sa + w];
            const bool lo = lo_any != 0;
            const uint32_t d = tmem + (uint32_t)(ab * C::kAccCols + t * C::kTileCols);
#pragma unroll
            for (int kk = 0; kk < tc::kKChunk / 16; ++kk) {
              const uint64_t adv = (uint64_t)(2 * kk);  // 32 bytes per 16-element k-step
              umma_f16_ss(d, da_hi + adv, db_hi + adv, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
              if (WSPLIT) umma_f16_ss(d, da_hi + adv, db_lo + adv, idesc, 1u);
              if (lo) umma_f16_ss(d, da_lo + adv, db_hi + adv, idesc, 1u);
            }
            umma_commit(&a_empty[sa]);
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
  } else if (warp < 2 + tc::kConvWarps) {
    // ---------------------------------------------------------------- converters
    // Warp cw owns rows [8cw, 8cw+8) of each tile; in load i a lane holds
    // 4 columns of row 8cw + 2i + (lane >> 4).  Fast path: the upper halves
    // of the fp32 bits (exact for non-negative values with zero low halves,
    // e.g. spikes) plus a bit test.  Only a warp holding another value (needs
    // the predicate, rounding or a lo half) takes the exact hi/lo split; the
    // lo share of an A slot is written then, and zero-filled once otherwise
    // ("dirty" tracks slots that may hold nonzero lo data), so a slot whose
    // other warps need the lo MMA sees zeros here.
    const int cw = warp - 2;
    const int half = lane >> 4;
    const int kq = (lane & 15) * 4;
    const bool emit = (a.bitmap != nullptr) && n_tile == 0;
    const bool check_unit = emit && a.nonunit != nullptr;
    constexpr int RPW = tc::kRows / tc::kConvWarps;  // rows per converter warp
    constexpr int NL = RPW / 2;                       // 16-byte loads per lane and slot
    // per-thread offsets, the same for every slot: staging row / A (swizzled) row
    uint32_t soff[NL], aoff[NL];
    int rls[NL];
#pragma unroll
    for (int i = 0; i < NL; ++i) {
      rls[i] = cw * RPW + 2 * i + half;
      soff[i] = (uint32_t)(rls[i] * 256 + kq * 4);
      aoff[i] = sw128_offset_bf16((uint32_t)rls[i], (uint32_t)kq);
    }
    // lane L < RPW packs the planar masks of local row L = 2i + h from the
    // warp-uniform ballots of load i: P0 = M0 | M1 << 16 (row 2i: low halves,
    // row 2i+1: high halves), P1 = M2 | M3 << 16
    const int my_i = (lane >> 1) & (NL - 1);
    const uint32_t my_sel = (lane & 1) ? 0x7632u : 0x5410u;
    uint32_t dirty = (1u << NA) - 1u;
    int j = 0, s = 0, sa = 0;
    uint32_t ps = 0u, pa = 0u;  // phase parities of the current staging / A slot
    bool ok = true;
    for (int g = 0; g < groups && ok; ++g) {
      const int tg = min(G, tiles - g * G);
      for (int kc = 0; kc < nk && ok; ++kc) {
        for (int t = 0; t < tg; ++t) {
          if (!(ok = mbar_wait(&stg_full[s], ps, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          if (j >= NA && !(ok = mbar_wait(&a_empty[sa], pa ^ 1u, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          const int64_t row0 = r_begin + (int64_t)(g * G + t) * tc::kRows;
          const int nrows = (int)min64(tc::kRows, r_end - row0);
          const unsigned char* st = stg + s * tc::kStgBytes;
          uint4 v[NL];  // raw fp32 bits
          if (nrows == tc::kRows) {
#pragma unroll
            for (int i = 0; i < NL; ++i) v[i] = *reinterpret_cast<const uint4*>(st + soff[i]);
          } else {
#pragma unroll
            for (int i = 0; i < NL; ++i)
              v[i] = (rls[i] < nrows) ? *reinterpret_cast<const uint4*>(st + soff[i]) : make_uint4(0u, 0u, 0u, 0u);
          }
          // Fast path: a non-negative value whose low 16 bits are zero is exactly
          // its upper half in bf16 (spikes 0/1 always are), so the A operand is
          // two byte permutes per 4 values.  One OR over the raw bits screens the
          // slot: a sign bit, low bits or an all-ones exponent field (Inf/NaN; the
          // OR of two other exponents can also give it, which only costs speed)
          // sends the warp down the exact path below.
          uint32_t bits_or = 0u;
          bool nonunit = false;
          uint32_t m[NL][4];  // ballots (warp-uniform)
          unsigned char* ahi = a_hi + sa * tc::kABytes;
#pragma unroll
          for (int i = 0; i < NL; ++i) {
            const uint4 b = v[i];
            bits_or |= b.x | b.y | b.z | b.w;
            *reinterpret_cast<uint2*>(ahi + aoff[i]) = make_uint2(__byte_perm(b.x, b.y, 0x7632), __byte_perm(b.z, b.w, 0x7632));
            if (check_unit) {
              nonunit |= (b.x != 0u && b.x != 0x3f800000u) || (b.y != 0u && b.y != 0x3f800000u) ||
                         (b.z != 0u && b.z != 0x3f800000u) || (b.w != 0u && b.w != 0x3f800000u);
            }
            if (emit) {
              // ballot e: bit m of lanes 0-15 = column 4m+e of row 2i, of lanes
              // 16-31 = column 4m+e of row 2i+1
              m[i][0] = __ballot_sync(0xffffffffu, __uint_as_float(b.x) > 0.0f);
              m[i][1] = __ballot_sync(0xffffffffu, __uint_as_float(b.y) > 0.0f);
              m[i][2] = __ballot_sync(0xffffffffu, __uint_as_float(b.z) > 0.0f);
              m[i][3] = __ballot_sync(0xffffffffu, __uint_as_float(b.w) > 0.0f);
            }
          }
          // The staging slot is released only now: every lane has stored values
          // computed from its loads, so those loads have completed (a release
          // right after issuing them could let the next TMA copy overwrite data
          // that a lane had not read yet).
          __syncwarp();
          if (lane == 0) mbar_arrive(&stg_empty[s]);
          if (emit) {
            // Planar spike masks per row and 64-column chunk: the 4 16-bit planes
            // packed into 2 words; the CSR pass converts them to column order.
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
              const int idx = t * tc::kRows + rl;
              const int c = __popc(keep0) + __popc(keep1);
              const int total = (kc == 0 ? 0 : row_count[idx]) + c;
              row_count[idx] = total;
              *reinterpret_cast<uint2*>(a.bitmap + grow * a.KWP + 2 * kc) = make_uint2(keep0, keep1);
              if (kc == nk - 1 && a.row_cnt) a.row_cnt[grow] = total;
            }
            if (kc == nk - 1 && a.blk_sum) {
              // the warp's 8 rows lie in one 128-row block: one atomic per warp and level
              int v = (lane < RPW && rl < nrows) ? row_count[t * tc::kRows + rl] : 0;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
              const int64_t g0 = row0 + cw * RPW;
              if (lane == 0 && cw * RPW < nrows && v) {
                atomicAdd(&a.blk_sum[g0 >> 7], v);
                atomicAdd(&a.sup_sum[g0 >> 14], (unsigned long long)v);
              }
            }
          }
          const bool warp_lo =
              __any_sync(0xffffffffu, (bits_or & 0x8000ffffu) != 0u || (bits_or & 0x7f800000u) == 0x7f800000u);
          if (warp_lo || ((dirty >> sa) & 1u)) {
            unsigned char* alo = a_lo + sa * tc::kABytes;
#pragma unroll
            for (int i = 0; i < NL; ++i) {
              uint2 lo_pk = make_uint2(0u, 0u);
              if (warp_lo) {  // exact path: predicate, round-to-nearest hi, lo remainder
                const float x[4] = {__uint_as_float(v[i].x), __uint_as_float(v[i].y), __uint_as_float(v[i].z),
                                    __uint_as_float(v[i].w)};
                __nv_bfloat16 h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split_bf16(x[e] > 0.0f ? x[e] : 0.0f, h[e], l[e]);
                *reinterpret_cast<uint2*>(ahi + aoff[i]) =
                    make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
                lo_pk = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
              }
              *reinterpret_cast<uint2*>(alo + aoff[i]) = lo_pk;
            }
            dirty = warp_lo ? (dirty | (1u << sa)) : (dirty & ~(1u << sa));
          }
          if (check_unit && __any_sync(0xffffffffu, nonunit) && lane == 0) atomicOr(a.nonunit, 1);
          if (lane == 0) lo_flag[sa * tc::kConvWarps + cw] = warp_lo ? 1 : 0;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[sa]);
          ++j;
          if (++s == NS) { s = 0; ps ^= 1u; }
          if (++sa == NA) { sa = 0; pa ^= 1u; }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 18-21)
    // 16-lane x 256-bit TMEM loads: four threads per row, so every store
    // instruction writes whole 32-byte sectors of eight rows.
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
          const int64_t rowA = r_begin + (int64_t)(g * G + t) * tc::kRows + q * 32 + h2 * 16 + ar;
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

// Pre-split weight image: for N-tile t and K-chunk c, an [NT x 64] bf16 hi
// block followed (fp32 W) by the lo block, each in the 128-byte-swizzled
// K-major layout of the B operand, so one bulk copy moves a whole chunk.
// The first thread also clears `zero_words` 32-bit words at `zero` (the CSR
// scan state and the non-unit flag of the same call), saving a memset node.
template <typename WT, bool WSPLIT>
__global__ void w_image_kernel(const WT* W, int64_t sk, int64_t sn, int K, int N, int NT, int nk, unsigned char* img,
                               uint32_t* zero, int64_t zero_words) {
  // the dense kernel (launched as a programmatic dependent) may start its
  // prologue now; it waits for this grid before it reads the image
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t total = (int64_t)((N + NT - 1) / NT) * NT * nk * 32;  // one thread per (n, 2 k)
  const size_t half = (size_t)NT * 128;
  const size_t stage = half * (WSPLIT ? 2 : 1);
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < zero_words; i += nthr) zero[i] = 0u;
  for (int64_t i = tid; i < total; i += nthr) {
    const int k2 = (int)(i % 32);        // pair of columns within the 64-wide chunk
    const int64_t rest = i / 32;
    const int64_t ng = rest / nk;        // global n index (padded)
    const int kc = (int)(rest % nk);
    const int t = (int)(ng / NT), nl = (int)(ng % NT);
    __nv_bfloat16 h[2], l[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int k = kc * 64 + k2 * 2 + e;
      float x = 0.0f;
      if (k < K && ng < N) x = static_cast<float>(W[(int64_t)k * sk + ng * sn]);
      if (WSPLIT) {
        split_bf16(x, h[e], l[e]);
      } else {
        h[e] = __float2bfloat16_rn(x);
      }
    }
    unsigned char* blk = img + ((size_t)t * nk + kc) * stage;
    const uint32_t off = sw128_offset_bf16((uint32_t)nl, (uint32_t)(k2 * 2));
    *reinterpret_cast<uint32_t*>(blk + off) = pack_bf16x2(h[0], h[1]);
    if (WSPLIT) *reinterpret_cast<uint32_t*>(blk + half + off) = pack_bf16x2(l[0], l[1]);
  }
}

// ---------------------------------------------------------------- host side
struct TcPlan {
  int NT;
  bool split;
  int nk, n_tiles;
  size_t img_bytes;
};

inline TcPlan tc_plan(int K, int N, int w_dtype) {
  TcPlan p{};
  p.split = (w_dtype == SPK_F32);
  p.NT = p.split ? 128 : 256;
  if (N <= 64) p.NT = (N + 15) / 16 * 16;
  else if (N <= 128) p.NT = 128;
  p.nk = (int)ceil_div(K, 64);
  p.n_tiles = (int)ceil_div(N, p.NT);
  p.img_bytes = (size_t)p.n_tiles * p.nk * p.NT * 128 * (p.split ? 2 : 1);
  return p;
}

inline bool tc_supported(int K, int N, const void* S) {
  return K >= 1 && N >= 1 && (K % 4) == 0 && (reinterpret_cast<uintptr_t>(S) % 16) == 0;
}

// S [R, K] fp32 as a 2-D tensor: boxes of 64 columns x 32 rows, zero fill
// outside the tensor (partial row tiles and K not a multiple of 64).
static int make_s_map(CUtensorMap* map, const float* S, int64_t R, int K) {
  return make_map_2d_f32(map, S, R, K, K, tc::kKChunk, tc::kBoxRows, "S");
}

struct TcOut {
  const float* bias;
  float* Y;
  uint32_t* bitmap;
  int32_t* row_cnt;
  int* nonunit;
  int32_t* blk_sum;
  unsigned long long* sup_sum;
  const int* gate = nullptr;  // automatic branch choice (see TcArgs::gate)
  int early_s = 1;            // the weight-image kernel precedes the launch (see TcArgs::early_s)
};

template <int NT, bool WSPLIT>
int launch_tc_inst(const CUtensorMap& map, TcArgs a, int n_tiles, cudaStream_t stream) {
  using C = tc::Cfg<NT, WSPLIT>;
  auto kern = spike_linear_tc_kernel<NT, WSPLIT>;
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes));
  const int sms = sm_count();
  const int ranges = sms / n_tiles > 0 ? sms / n_tiles : 1;
  a.rows_per_cta = ceil_div(ceil_div(a.R, ranges), 32) * 32;
  const int64_t gx = ceil_div(a.R, a.rows_per_cta);
  dim3 grid((unsigned)gx, (unsigned)n_tiles);
  prof_before(SPK_KERNEL_DENSE, stream);
  SPK_CUDA_TRY(launch_dependent(kern, grid, dim3(tc::kThreads), C::kSmemBytes, stream, map, a));
  prof_after(SPK_KERNEL_DENSE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_w_image(const void* W, int w_dtype, int64_t sk, int64_t sn, int K, int N, const TcPlan& p,
                   unsigned char* img, uint32_t* zero, int64_t zero_words, cudaStream_t stream) {
  const int64_t total = (int64_t)p.n_tiles * p.NT * p.nk * 32;
  const int threads = 256;
  const int blocks = (int)min64(ceil_div(max64(total, zero_words), threads), 8192);
  prof_before(SPK_KERNEL_W_IMAGE, stream);
  if (w_dtype == SPK_BF16) {
    w_image_kernel<__nv_bfloat16, false><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(W), sk, sn, K, N, p.NT, p.nk, img, zero, zero_words);
  } else {
    w_image_kernel<float, true><<<blocks, threads, 0, stream>>>(static_cast<const float*>(W), sk, sn, K, N, p.NT,
                                                               p.nk, img, zero, zero_words);
  }
  prof_after(SPK_KERNEL_W_IMAGE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_tc(const float* S, int64_t R, int K, int N, const TcPlan& p, const unsigned char* img, const TcOut& o,
              cudaStream_t stream) {
  CUtensorMap map;
  int rc = make_s_map(&map, S, R, K);
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
  if (p.split) {
    switch (p.NT) {
      case 16: return launch_tc_inst<16, true>(map, a, p.n_tiles, stream);
      case 32: return launch_tc_inst<32, true>(map, a, p.n_tiles, stream);
      case 48: return launch_tc_inst<48, true>(map, a, p.n_tiles, stream);
      case 64: return launch_tc_inst<64, true>(map, a, p.n_tiles, stream);
      case 128: return launch_tc_inst<128, true>(map, a, p.n_tiles, stream);
      default: break;
    }
  } else {
    switch (p.NT) {
      case 16: return launch_tc_inst<16, false>(map, a, p.n_tiles, stream);
      case 32: return launch_tc_inst<32, false>(map, a, p.n_tiles, stream);
      case 48: return launch_tc_inst<48, false>(map, a, p.n_tiles, stream);
      case 64: return launch_tc_inst<64, false>(map, a, p.n_tiles, stream);
      case 128: return launch_tc_inst<128, false>(map, a, p.n_tiles, stream);
      case 256: return launch_tc_inst<256, false>(map, a, p.n_tiles, stream);
      default: break;
    }
  }
  return fail(SPK_EUNSUPPORTED, "no dense-branch tile for N=%d", N);
}

}  // namespace spk
