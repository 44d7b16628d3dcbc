// Dense branch of spike-linear for fp32 weights and N > 64: the weights live
// in tensor memory as the A operand and the spikes stream through shared
// memory as the B operand (tcgen05.mma kind::tf32, A from TMEM).
//
// Per 128-column N tile the kernel computes Y^T[n, r] = sum_k W^T[n, k] *
// relu'(S[r, k]) (+ bias[n]) with relu'(x) = x if x > 0 else 0 (the reference
// engine's predicate, sparse_linear.cu:268): MMA M = the 128 output columns
// (TMEM lanes), MMA N = 128 rows of S, K = 64 per staging slot.  W is split
// into tf32 hi + lo halves (W = hi + lo to ~2^-22 relative), two MMAs per
// k-step; S arrives fp32 straight from TMA into the staging slot, which is
// the K-major B operand as it lies.  Non-exact S values (low mantissa bits,
// negative, Inf/NaN) take the same hi pass / lo pass in place as in the
// S-as-A kernel (spike_linear_tf32.cu), with the converter warps shared.
//
// The linear-activation op (general fp32 X) computes W X as one tf32 pass
// w_hi * x_t (x_t = x truncated to tf32 by the tensor core) plus one bf16
// pass over a doubled K: bf16(w - w_hi) * bf16(x) + bf16(w_hi) * bf16(x - x_t).
// The bf16 pass costs the tensor core what one tf32 pass does (twice the
// rate, twice the K), so two pass-times instead of the three of a 3xTF32
// split; each product is within ~2^-18 of w x relative (~1e-6 of max |y| in
// the tests), the dropped (w - w_hi)(x - x_t) is below 2^-21.
//
// Why this operand order: the S-as-A kernel keeps two 64 KB weight chunks in
// shared memory for the whole time the MMAs read them, leaving room for three
// 32 KB S slots, too few to cover the DRAM latency of a slot.  Here a weight
// chunk passes through shared memory only briefly (16 KB pieces, copied into
// TMEM by four warps), so five S slots fit.
//
// TMEM (512 columns): [0, 256) two weight chunks, each [hi k0..63 | lo k0..63]
// (one tf32 per column, lane = output column n; for the linear op the lo half
// holds the 128 bf16 [w - w_hi | w_hi] of the correction pass, two per
// column); [256, 512) the accumulators of a group of two row tiles (column =
// row, lane = n), single-buffered.
//
// Warp roles (736 threads): warp 0 S producer (TMA, boxes of 32 columns x 32
// rows), warp 1 TMEM owner + MMA issuer, warp 2 weight-piece producer (1-D
// bulk copies), warps 3-18 converters, warps 19-22 weight loaders (shared
// memory piece -> tcgen05.st into TMEM).  The epilogue (TMEM -> + bias -> Y)
// runs on the loader warps for spike-linear, and on the sixteen converter
// warps for the linear op, whose correction pass leaves the tensor core less
// work per row: the MMAs wait for the single-buffered accumulators to drain,
// so the drain is spread over four warps per TMEM lane quarter.
// Every wait is bounded (2 s) and reports SPK_DEV_PIPE_TIMEOUT; issued copies
// and MMAs are drained and TMEM is freed on every exit.
#include "tma.cuh"

namespace spk {

namespace wt {

constexpr int kRows = 128;                  // rows of S per tile (MMA N)
constexpr int kLanes = 128;                 // output columns per tile (MMA M, TMEM lanes)
constexpr int kKChunk = 64;                 // columns of S per staging slot
constexpr int kAtomBytes = kRows * 128;     // one swizzle-atom column of a slot: 16 KB
constexpr int kStgBytes = 2 * kAtomBytes;   // 32 KB
constexpr int kBoxRows = 32;
constexpr int kBoxBytes = kBoxRows * 128;
constexpr int kPieceBytes = kLanes * 128;   // 128 n x 32 k of hi or lo: 16 KB
constexpr int kPieces = 4;                  // per 64-wide K chunk: hi k0-31, hi k32-63, lo k0-31, lo k32-63
constexpr int kConvWarps = t32::kConvWarps;
constexpr int kNP = 4;                      // weight-piece slots
constexpr int kG = 2;                       // row tiles per accumulator group
constexpr int kWarps = 3 + kConvWarps + 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kTmemCols = 512;
constexpr uint32_t kAcol = 0;               // weight chunk buffers: 2 x 128 columns
constexpr uint32_t kDcol = 256;             // accumulators: kG x 128 columns
// Rows of a 128-row tile that one CTA stages: all of them, or half in a CTA
// pair (tcgen05 cta_group::2 splits the B operand by rows between the pair).
template <bool kPair>
struct Geo {
  static constexpr int kRowsC = kPair ? kRows / 2 : kRows;
  static constexpr int kAtom = kRowsC * 128;  // one swizzle-atom column of a slot
  static constexpr int kStg = 2 * kAtom;      // a slot: 64 fp32 columns
};
// Shared-memory rings per mode.  Spike-linear: five S slots.  Linear op:
// three X slots and two bf16 correction-operand buffers (the X slot itself is
// the tf32 pass's operand); a CTA pair stages half-height slots, four and
// three of them.  The GSMC recurrence (kXchg) gives one S slot to the
// epilogue's 16 KB gate exchange buffer.
template <bool kRelu, bool kXchg = false, bool kPair = false>
struct Ring {
  static constexpr int NS = kPair ? 4 : kRelu ? (kXchg ? 4 : 5) : 3;  // staging slots
  static constexpr int NL = kPair ? 3 : kRelu ? 0 : 2;  // correction-operand buffers (linear op)
  static constexpr size_t kXchgBytes = kXchg ? 2 * 4 * 16 * 32 * sizeof(float) : 0;  // [2][4 gates][16 rows][32]
  static constexpr size_t kRing =
      (size_t)(NS + NL) * Geo<kPair>::kStg + (size_t)kNP * kPieceBytes + kXchgBytes;
  // barriers, lo flags [NS][16] bytes, row counts [G][128], TMEM slot, abort flag
  static constexpr int kBarsUsed = 5 * NS + 2 * NL + 2 * kNP + 8;
  static constexpr int kBars = kBarsUsed + (kBarsUsed & 1);  // even: the lo flags after them stay 16-byte aligned
  static constexpr size_t kTail = 8 * kBars + kConvWarps * NS + 4 * kRows * kG + 16;
  static constexpr size_t kSmemBytes = 1024 + kRing + ((kTail + 255) / 256) * 256;
  static_assert((8 * kBars) % 16 == 0, "lo flags 16-byte aligned");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};
static_assert(kDcol + kG * kRows <= kTmemCols && kAcol + 2 * 2 * kKChunk <= kDcol, "TMEM budget");
static_assert(kRows == t32::kRows && kStgBytes == t32::kStgBytes, "staging layout shared with the converters");

}  // namespace wt

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::tf32.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 with A = B = bf16 (K = 16).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same for a CTA pair (cta_group::2, issued by CTA 0; M = 256 across the
// pair's TMEM, B split by rows between their shared memories), with an
// all-zero disable-output-lane mask.
__device__ __forceinline__ void umma_tf32_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u)
      : "memory");
}

// Epilogue of the weights-in-TMEM kernel, per element y = D + bias[n].
enum WtEpilogue : int {
  kEpiLinear = 0,     // y
  kEpiHeaviside = 1,  // 1 if y - thr > 0 else 0 (spike_fn(fc1(x) - thr); q, k spikes with thr = 0)
  kEpiVSpike = 2,     // 1 if (tanh(y) + 1) / 2 - thr > 0 else 0 (the v spikes, thr = tau)
  kEpiHeavisideBits = 3,  // the Heaviside spikes packed: bit b of word w of a row = column 32w + b
  kEpiVSpikeBits = 4,     // the v spikes packed the same way
  kEpiGsmc = 5            // the GSMC cell update from the recurrent gate projections (a.cell)
};

template <int kEpi>
__device__ __forceinline__ float wt_epilogue(float y, float thr) {
  if (kEpi == kEpiHeaviside) return (y - thr > 0.0f) ? 1.0f : 0.0f;
  if (kEpi == kEpiVSpike) return ((tanhf(y) + 1.0f) / 2.0f - thr > 0.0f) ? 1.0f : 0.0f;
  return y;
}

// Epilogue share of one converter warp of the linear op: the group iterated
// g-th (accumulators of its tg row tiles in TMEM columns kDcol + 16b for the
// 16-row blocks b) once its MMAs have committed.  The four converter warps of
// TMEM lane quarter q take every fourth block, so sixteen warps drain the
// accumulators while the tensor core waits for them.
template <int kEpi, int G, bool kPair = false>
__device__ __forceinline__ bool converter_group_epilogue(const int cw, const int lane, const TcArgs& a, const uint32_t tmem,
                                                      const int n0, const float bias_n, uint64_t* acc_full,
                                                      uint64_t* acc_empty, volatile int* abort_flag,
                                                      const int64_t r_begin, const int64_t r_end, const int g,
                                                      const int groups, const int tiles) {
  const int q = (cw + 3) & 3;  // warp 3 + cw may access TMEM lanes [32q, 32q + 32)
  const int sq = cw >> 2;      // its rank among the quarter's four converter warps
  if (!mbar_wait<kPair>(acc_full, g & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) return false;
  tc_fence_after();
  // with a.early_s these warps skipped the dependency wait at the start; only the weight-image
  // kernel can still be running then, and it never touches Y, but the first store waits anyway
  if (a.early_s && g == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
  const int pg = groups - 1 - g;
  const int tg = min(G, tiles - pg * G);
  const int64_t grow0 = r_begin + (int64_t)(pg * G) * wt::kRows;  // the tiles lie back to back in rows and columns
  const int nb = (int)ceil_div(min64((int64_t)tg * wt::kRows, r_end - grow0), 16);
  const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + wt::kDcol;
  const int n = n0 + q * 32 + lane;
  // tile by tile (blocks of tile t: 8t .. 8t + 7), each tile released on its own barrier as soon as
  // it is drained, so the next group's MMAs into tile 0 start while tile 1 drains
  bool released0 = false;
  for (int b = sq; b < nb; b += 4) {  // warp-uniform bounds
    if (b >= 8 && !released0) {       // first block of tile 1 for this warp: its part of tile 0 is done
      released0 = true;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_rank0(&acc_empty[0]);
        else mbar_arrive(&acc_empty[0]);
      }
    }
    float v[16];
    tmem_ld16(tacc + (uint32_t)(16 * b), v);
    tmem_wait_ld();
    tmem_reg_fence(v);
    const int64_t rowb = grow0 + (int64_t)b * 16;
    if constexpr (kEpi == kEpiHeavisideBits || kEpi == kEpiVSpikeBits) {
      // one ballot per row gives the row's word of this warp's 32 columns (N % 32 == 0: a
      // warp's columns are all in range or all out); lane jj stores row rowb + jj's word
      if (n0 + q * 32 < a.N) {
        uint32_t word = 0u;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const float spike =
              wt_epilogue<kEpi == kEpiHeavisideBits ? kEpiHeaviside : kEpiVSpike>(v[jj] + bias_n, a.thr);
          const uint32_t bal = __ballot_sync(0xffffffffu, spike > 0.0f);
          if (lane == jj) word = bal;
        }
        const int NW = a.N / 32;
        if (lane < 16 && rowb + lane < r_end)
          reinterpret_cast<uint32_t*>(a.Y)[(rowb + lane) * NW + (n0 / 32 + q)] = word;
      }
    } else if (n < a.N) {
      float* y = a.Y + rowb * a.N + n;
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        if (rowb + jj < r_end) y[(int64_t)jj * a.N] = wt_epilogue<kEpi>(v[jj] + bias_n, a.thr);
    }
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {  // the tiles not released above (every warp releases both once per group)
    for (int t = released0 ? 1 : 0; t < 2; ++t) {
      if constexpr (kPair) mbar_arrive_rank0(&acc_empty[t]);  // the pair's MMAs wait on CTA 0's barriers
      else mbar_arrive(&acc_empty[t]);
    }
  }
  return true;
}

// Converter warps of the linear op.  The tensor core reads the X slot's fp32
// values truncated to tf32 (the hi part, x_t); each warp reads its 8 rows once
// and writes the B operand of the correction pass into a buffer of the same
// size: per row [bf16(x) k0..63 | bf16(x - x_t) k0..63] in the 128-byte
// swizzle (x - x_t is exact in fp32; non-finite x gives 0 in both: the tf32
// pass carries it).  The slot itself is never rewritten, so a warp never
// waits for the MMAs inside a slot, only for a free buffer.  The converters
// also run the epilogue: that of group g - 1 after the first NL slots of group
// g (the ones the MMAs take first once the accumulators are free), the last
// group's after its slots.
template <int kEpi, int NS, int NL, int G, bool kPair = false>
__device__ __forceinline__ void linear_converter(const int cw, const int lane, unsigned char* stg,
                                                 unsigned char* lob, uint64_t* stg_full, uint64_t* stg_empty,
                                                 uint64_t* lof, uint64_t* loe, uint64_t* acc_full,
                                                 uint64_t* acc_empty, volatile int* abort_flag, const TcArgs& a,
                                                 const uint32_t tmem, const int n0, const int64_t r_begin,
                                                 const int64_t r_end, const int nk, const int groups,
                                                 const int tiles, const int rank) {
  using GE = wt::Geo<kPair>;
  constexpr int RPW = GE::kRowsC / wt::kConvWarps;  // rows per converter warp
  constexpr int NLD = RPW / 2;                      // 16-byte loads per lane and slot
  const int half = lane >> 4, cl = lane & 15;
  uint32_t soff[NLD], boff[NLD];
  int rls[NLD];
#pragma unroll
  for (int i = 0; i < NLD; ++i) {
    rls[i] = cw * RPW + 2 * i + half;
    // fp32 chunk cl holds columns 4cl .. 4cl+3: in bf16 half (cl & 1) of 16-byte chunk cl >> 1
    soff[i] = (uint32_t)((cl >> 3) * GE::kAtom) + sw128_chunk((uint32_t)rls[i], (uint32_t)(cl & 7));
    boff[i] = sw128_chunk((uint32_t)rls[i], (uint32_t)(cl >> 1)) + (uint32_t)(cl & 1) * 8u;
  }
  auto xv = [](uint32_t b) -> float {
    const float x = __uint_as_float(b);
    return isfinite(x) ? x : 0.0f;
  };
  auto rem = [](uint32_t b) -> float {
    const float x = __uint_as_float(b);
    return isfinite(x) ? x - __uint_as_float(b & 0xffffe000u) : 0.0f;
  };
  const int n = n0 + ((cw + 3) & 3) * 32 + lane;
  const float bias_n = (a.bias != nullptr && n < a.N) ? a.bias[n] : 0.0f;
  int j = 0;
  bool ok = true;
  for (int g = 0; g < groups && ok; ++g) {
    const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
    const int tg = min(G, tiles - pg * G);
    // slots of this group converted before the previous group's epilogue: at most NS (converting
    // slot NS + 1 would need a slot that only this group's MMAs free, which wait for the epilogue)
    const int trig = min(min(NL, NS), nk * tg);
    int js = 0;  // slot index within the group
    for (int kc = 0; kc < nk && ok; ++kc) {
      for (int t = 0; t < tg; ++t, ++j, ++js) {
        const int s = j % NS, l = j % NL;
        if (!(ok = mbar_wait<kPair>(&stg_full[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        // rows of this CTA's part of the tile (the second CTA of a pair stages rows 64 .. 127)
        const int nrows = (int)min64(
            GE::kRowsC, r_end - (r_begin + (int64_t)(pg * G + t) * wt::kRows + (int64_t)rank * GE::kRowsC));
        const unsigned char* st = stg + s * GE::kStg;
        uint2 xb[NLD], lo[NLD];
#pragma unroll
        for (int i = 0; i < NLD; ++i) {
          const uint4 b = rls[i] < nrows ? *reinterpret_cast<const uint4*>(st + soff[i]) : make_uint4(0u, 0u, 0u, 0u);
          xb[i] = bf16x4(xv(b.x), xv(b.y), xv(b.z), xv(b.w));
          lo[i] = bf16x4(rem(b.x), rem(b.y), rem(b.z), rem(b.w));
        }
        if (j >= NL && !(ok = mbar_wait<kPair>(&loe[l], ((j / NL) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        unsigned char* lb = lob + l * GE::kStg;
#pragma unroll
        for (int i = 0; i < NLD; ++i) {
          *reinterpret_cast<uint2*>(lb + boff[i]) = xb[i];
          *reinterpret_cast<uint2*>(lb + GE::kAtom + boff[i]) = lo[i];
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) mbar_arrive_rank0(&lof[l]);  // the pair's MMAs wait on CTA 0's barrier
          else mbar_arrive(&lof[l]);
          mbar_arrive(&stg_empty[s]);  // this warp has read the slot
        }
        if (g >= 1 && js + 1 == trig &&
            !(ok = converter_group_epilogue<kEpi, G, kPair>(cw, lane, a, tmem, n0, bias_n, acc_full, acc_empty, abort_flag,
                                                  r_begin, r_end, g - 1, groups, tiles)))
          break;
      }
    }
  }
  if (ok && groups > 0)
    converter_group_epilogue<kEpi, G, kPair>(cw, lane, a, tmem, n0, bias_n, acc_full, acc_empty, abort_flag, r_begin, r_end,
                                   groups - 1, groups, tiles);
}

// Converter warps of the packed-spike input (kBits).  The spikes arrive as
// 32-bit words, bit b of word w of a row = column 32w + b; each slot (128
// rows x 64 columns = two words per row) is expanded into bf16 0 / 1 in the
// K-major 128-byte swizzle of the B operand (one 16 KB atom column: the MMAs
// multiply it by the three-way bf16 split of W).  Warp cw fills rows
// 8cw..8cw+7; lane l takes row 8cw + l/4 and columns 16(l%4) .. +15 (two
// 16-byte chunks; the 8 lanes of a quarter warp cover distinct bank groups).
// The slot is free again when the MMAs that read it committed (stg_empty),
// and ready for them when every converter arrived on chk.  The converters
// also run the epilogue, as in the linear op.
template <int NS, int G>
__device__ __forceinline__ void bits_converter(const int cw, const int lane, unsigned char* stg, uint64_t* chk,
                                               uint64_t* stg_empty, uint64_t* acc_full, uint64_t* acc_empty,
                                               volatile int* abort_flag, const TcArgs& a, const uint32_t tmem,
                                               const int n0, const int64_t r_begin, const int64_t r_end,
                                               const int nk, const int groups, const int tiles) {
  constexpr int CW = wt::kConvWarps;
  const int KW = a.K / 32;
  const int rl = cw * (wt::kRows / CW) + (lane >> 2);  // row within the tile
  const int q = lane & 3;                               // 16-column group of the slot
  const int n = n0 + ((cw + 3) & 3) * 32 + lane;
  const float bias_n = (a.bias != nullptr && n < a.N) ? a.bias[n] : 0.0f;
  auto bf16x4_bits = [](uint32_t nib) -> uint2 {  // 4 spikes -> bf16 1.0 (0x3f80) / 0
    return make_uint2(((nib & 1u) ? 0x3f80u : 0u) | ((nib & 2u) ? 0x3f800000u : 0u),
                      ((nib & 4u) ? 0x3f80u : 0u) | ((nib & 8u) ? 0x3f800000u : 0u));
  };
  int j = 0;
  bool ok = true;
  for (int g = 0; g < groups && ok; ++g) {
    const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
    const int tg = min(G, tiles - pg * G);
    const int trig = min(min(2, NS), nk * tg);  // slots converted before the previous group's epilogue (<= NS)
    int js = 0;
    for (int kc = 0; kc < nk && ok; ++kc) {
      for (int t = 0; t < tg; ++t, ++j, ++js) {
        const int s = j % NS;
        if (j >= NS && !(ok = mbar_wait(&stg_empty[s], ((j / NS) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        const int64_t row = r_begin + (int64_t)(pg * G + t) * wt::kRows + rl;
        const uint32_t w = row < r_end ? a.bits_in[row * KW + 2 * kc + (q >> 1)] : 0u;
        const uint32_t h = (w >> ((q & 1) * 16)) & 0xffffu;
        unsigned char* st = stg + s * wt::kStgBytes;
        const uint2 c0 = bf16x4_bits(h), c1 = bf16x4_bits(h >> 4), c2 = bf16x4_bits(h >> 8), c3 = bf16x4_bits(h >> 12);
        *reinterpret_cast<uint4*>(st + sw128_chunk((uint32_t)rl, (uint32_t)(2 * q))) = make_uint4(c0.x, c0.y, c1.x, c1.y);
        *reinterpret_cast<uint4*>(st + sw128_chunk((uint32_t)rl, (uint32_t)(2 * q + 1))) =
            make_uint4(c2.x, c2.y, c3.x, c3.y);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&chk[s]);
        if (g >= 1 && js + 1 == trig &&
            !(ok = converter_group_epilogue<kEpiLinear, G>(cw, lane, a, tmem, n0, bias_n, acc_full, acc_empty,
                                                           abort_flag, r_begin, r_end, g - 1, groups, tiles)))
          break;
      }
    }
  }
  if (ok && groups > 0)
    converter_group_epilogue<kEpiLinear, G>(cw, lane, a, tmem, n0, bias_n, acc_full, acc_empty, abort_flag, r_begin,
                                            r_end, groups - 1, groups, tiles);
}

// kRelu: spike-linear (relu'(S)); false: the linear-activation op (plain X).
// kBits (with kRelu): the spikes come packed, 1 bit each (a.bits_in).
// kPair (linear op): launched in clusters of two CTAs along N, the pair's
// MMAs run as tcgen05 cta_group::2 (M = 256: the two CTAs' 128-column weight
// tiles in their TMEM; N = 128 rows: each CTA stages 64 of them), issued by
// CTA 0; every barrier the MMAs wait on lives in CTA 0 and collects both
// CTAs' arrivals, every MMA commit arrives in both CTAs.  Each SM then reads
// half the B operand per FLOP and converts half the rows.
template <int kEpi, bool kRelu, bool kBits = false, bool kPair = false>
__global__ void __launch_bounds__(wt::kThreads, 1)
    spike_linear_wt_kernel(const __grid_constant__ CUtensorMap tmap_s, TcArgs a) {
  static_assert(!kPair || !kRelu, "CTA pairs: the linear op only");
  if (!kPair && gated_off(a.gate, SPK_BRANCH_DENSE)) return;  // the automatic choice took the CSR branch
  using RG = wt::Ring<kRelu, kEpi == kEpiGsmc, kPair>;
  using GE = wt::Geo<kPair>;
  constexpr int G = wt::kG, NS = RG::NS, NL = RG::NL, NP = wt::kNP, CW = wt::kConvWarps;
  constexpr int PPC = kBits ? 3 : wt::kPieces;  // weight pieces per K chunk
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  unsigned char* base = smem_aligned_1024(smem_dyn);
  unsigned char* stg = base;                                  // [NS][2 atoms] fp32 staging = B operand
  unsigned char* lob = stg + NS * GE::kStg;                   // [NL][2 atoms] bf16 correction operand (linear op)
  unsigned char* pcs = lob + NL * GE::kStg;                   // [NP][16 KB] weight pieces
  float* xbuf = reinterpret_cast<float*>(pcs + NP * wt::kPieceBytes);  // GSMC gate exchange (kXchgBytes)
  uint64_t* bars = reinterpret_cast<uint64_t*>(pcs + NP * wt::kPieceBytes + RG::kXchgBytes);
  uint64_t* stg_full = bars;
  uint64_t* chk = stg_full + NS;
  uint64_t* stg_empty = chk + NS;
  uint64_t* lo_go = stg_empty + NS;
  uint64_t* lo_full = lo_go + NS;
  uint64_t* pc_full = lo_full + NS;
  uint64_t* pc_empty = pc_full + NP;
  uint64_t* a_full = pc_empty + NP;   // [2] weight chunk in TMEM
  uint64_t* a_empty = a_full + 2;     // [2]
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + 1;  // [2] row tile t of the accumulators drained
  uint64_t* drain = acc_empty + 2;
  uint64_t* lof = drain + 1;   // [NL] correction buffer written (linear op)
  uint64_t* loe = lof + NL;    // [NL] correction buffer read by the MMAs
  static_assert(5 * NS + 2 * NP + 8 + 2 * NL == RG::kBarsUsed, "the barriers above fill the barrier block");
  uint8_t* lo_flag = reinterpret_cast<uint8_t*>(bars + RG::kBars);  // [NS][CW] bytes, 16-byte aligned
  int* row_count = reinterpret_cast<int*>(lo_flag + NS * CW);       // [G][128]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(row_count + G * wt::kRows);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = kPair ? (int)cluster_ctarank() : 0;  // CTA 0 of a pair issues the MMAs
  // a pair's grid is (N tiles, row ranges) with clusters of (2, 1, 1); otherwise (row ranges, N tiles)
  const int64_t r_begin = (int64_t)(kPair ? blockIdx.y : blockIdx.x) * a.rows_per_cta;
  const int64_t r_end = min64(a.R, r_begin + a.rows_per_cta);
  const int n_tile = kPair ? blockIdx.x : blockIdx.y;
  const int n0 = n_tile * wt::kLanes;
  const int nk = a.nk;
  const int tiles = r_end > r_begin ? (int)ceil_div(r_end - r_begin, wt::kRows) : 0;
  const int groups = (tiles + G - 1) / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&stg_full[s], 1);
      mbar_init(&chk[s], CW);
      mbar_init(&stg_empty[s], kBits ? 1 : CW + 1);  // packed spikes: the MMAs' commit only
      mbar_init(&lo_go[s], 1);
      mbar_init(&lo_full[s], CW);
    }
    for (int p = 0; p < NP; ++p) {
      mbar_init(&pc_full[p], 1);
      mbar_init(&pc_empty[p], 4);
    }
    constexpr int kCtas = kPair ? 2 : 1;  // CTAs arriving on the barriers the MMAs wait on
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a_full[b], 4 * kCtas);
      mbar_init(&a_empty[b], 1);
    }
    mbar_init(acc_full, 1);
    for (int t = 0; t < 2; ++t)  // the epilogue warps: loaders or converters
      mbar_init(&acc_empty[t], (kRelu && !kBits) ? 4 : CW * kCtas);
    mbar_init(drain, 1);
    for (int l = 0; l < NL; ++l) {
      mbar_init(&lof[l], CW * kCtas);
      mbar_init(&loe[l], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_slot, wt::kTmemCols);  // warp 1 of both CTAs, the same slot offset
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, wt::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (kPair) cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent of the kernel before it.  When that is the
  // weight-image kernel (a plain launch, so S was complete before it started;
  // a.early_s) the S producer requests the first slots before its wait, and
  // the converters screen them before theirs (ahead of their first global
  // write); otherwise (a prepared image: the previous kernel may be the one
  // writing S) every warp waits first.
  const bool late_dep = a.early_s && ((warp == 0 && lane == 0) || (warp >= 3 && warp < 3 + CW));
  if (!late_dep) asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- S producer
    // (none for packed spikes: the converter warps build the slots)
    if (lane == 0 && !kBits) {
      tma_prefetch_map(&tmap_s);
      auto load_s = [&](int s, int64_t tile_row0, int kc) {
        // this CTA's rows of the tile (a pair's second CTA stages rows 64 .. 127), in 32-row
        // boxes up to the last valid row: no reads past the CTA's range (rows a box leaves out
        // keep stale data; the converters and the epilogue ignore them)
        const int64_t row0 = tile_row0 + (int64_t)rank * GE::kRowsC;
        const int nbox = row0 < r_end ? (int)ceil_div(min64(GE::kRowsC, r_end - row0), wt::kBoxRows) : 0;
        if (nbox == 0) {
          mbar_arrive(&stg_full[s]);
          return;
        }
        mbar_arrive_expect_tx(&stg_full[s], (uint32_t)(2 * nbox * wt::kBoxBytes));
        for (int b = 0; b < nbox; ++b) {
          unsigned char* dst = stg + s * GE::kStg + b * wt::kBoxBytes;
          const int y = (int)row0 + b * wt::kBoxRows;
          tma_load_2d(dst, &tmap_s, kc * wt::kKChunk, y, &stg_full[s]);
          tma_load_2d(dst + GE::kAtom, &tmap_s, kc * wt::kKChunk + 32, y, &stg_full[s]);
        }
      };
      int pre = 0;  // slots requested before the wait: the first NS (or all), only when S is known complete
      for (int g = 0; g < groups && pre < NS && a.early_s; ++g) {
        const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
    const int tg = min(G, tiles - pg * G);
        for (int kc = 0; kc < nk && pre < NS; ++kc)
          for (int t = 0; t < tg && pre < NS; ++t, ++pre) load_s(pre, r_begin + (int64_t)(pg * G + t) * wt::kRows, kc);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      int j = 0;
      bool ok = true;
      for (int g = 0; g < groups && ok; ++g) {
        const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
    const int tg = min(G, tiles - pg * G);
        for (int kc = 0; kc < nk && ok; ++kc) {
          for (int t = 0; t < tg; ++t, ++j) {
            if (j < pre) continue;
            const int s = j % NS;
            if (j >= NS &&
                !(ok = mbar_wait<kPair>(&stg_empty[s], ((j / NS) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
              break;
            load_s(s, r_begin + (int64_t)(pg * G + t) * wt::kRows, kc);
          }
        }
      }
      // copies still in flight land before the CTA exits (early exits included)
      const int issued = max(j, pre);
      for (int i = (issued > NS ? issued - NS : 0); i < issued; ++i)
        mbar_wait(&stg_full[i % NS], (i / NS) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr int kM = kPair ? 2 * wt::kLanes : wt::kLanes;  // a pair: M = 256 over both CTAs' TMEM
      constexpr uint32_t idesc = umma_idesc_tf32_f32(kM, wt::kRows);
      constexpr uint32_t idesc_b16 = umma_idesc_bf16_f32(kM, wt::kRows);
      auto commit = [](uint64_t* bar) {  // a pair's commits arrive in both CTAs
        if constexpr (kPair) umma_commit_pair(bar);
        else umma_commit(bar);
      };
      int j = 0, ja = 0;
      bool ok = true;
      for (int g = 0; g < groups && ok; ++g) {
        const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
    const int tg = min(G, tiles - pg * G);
        // the accumulators are single-buffered: before its first MMA into row tile t the group
        // waits until the previous group's epilogue has released that tile (below, at kc == 0)
        for (int kc = 0; kc < nk && ok; ++kc) {
          const int ab = ja & 1;
          if (!(ok = mbar_wait<kPair>(&a_full[ab], (ja >> 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          tc_fence_after();
          const uint32_t a_hi = tmem + wt::kAcol + (uint32_t)ab * 128u;
          const uint32_t a_lo = a_hi + 64u;
          for (int t = 0; t < tg; ++t) {
            const int s = j % NS;
            if (g >= 1 && kc == 0) {
              if (!(ok = mbar_wait<kPair>(&acc_empty[t], (g - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
              tc_fence_after();
            }
            if constexpr (!kRelu) {
              // linear op: the tf32 pass w_hi * x_t (the slot as the tensor core reads it), then the
              // bf16 correction pass over K = 128: [bf16(w - w_hi) | bf16(w_hi)] (TMEM columns
              // a_lo .. a_lo + 63, two bf16 per column) times [bf16(x) | bf16(x - x_t)] (the
              // converters' buffer).  Both passes step 32 bytes of a 128-byte row per MMA.
              const int l = j % NL;
              if (!(ok = mbar_wait<kPair>(&lof[l], (j / NL) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
              tc_fence_after();
              const uint32_t d = tmem + wt::kDcol + (uint32_t)(t * wt::kRows);
              // a pair: the same offsets in both CTAs' shared memory hold their halves of the rows
              const uint64_t db0 = umma_desc_sw128_kmajor(smem_u32(stg + s * GE::kStg));
              const uint64_t dl0 = umma_desc_sw128_kmajor(smem_u32(lob + l * GE::kStg));
#pragma unroll
              for (int kk = 0; kk < wt::kKChunk / 8; ++kk) {
                const uint64_t off = (uint64_t)(((kk >> 2) * GE::kAtom + (kk & 3) * 32) >> 4);
                const uint32_t acc = (kc > 0 || kk > 0) ? 1u : 0u;
                if constexpr (kPair) umma_tf32_ts_pair(d, a_hi + (uint32_t)kk * 8u, db0 + off, idesc, acc);
                else umma_tf32_ts(d, a_hi + (uint32_t)kk * 8u, db0 + off, idesc, acc);
              }
#pragma unroll
              for (int kk = 0; kk < 2 * wt::kKChunk / 16; ++kk) {
                const uint64_t off = (uint64_t)(((kk >> 2) * GE::kAtom + (kk & 3) * 32) >> 4);
                if constexpr (kPair) umma_bf16_ts_pair(d, a_lo + (uint32_t)kk * 8u, dl0 + off, idesc_b16, 1u);
                else umma_bf16_ts(d, a_lo + (uint32_t)kk * 8u, dl0 + off, idesc_b16, 1u);
              }
              commit(&stg_empty[s]);
              commit(&loe[l]);
              ++j;
              continue;
            }
            if constexpr (kBits) {
              // packed spikes: the slot holds bf16 0 / 1 (one 16 KB atom column); the chunk's
              // TMEM columns a_hi + [0, 96) hold the three-way bf16 split b1 | b2 | b3 of W (two
              // per column), so each 16-column step is three kind::f16 MMAs, exact per product
              if (!(ok = mbar_wait(&chk[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
              tc_fence_after();
              const uint32_t d = tmem + wt::kDcol + (uint32_t)(t * wt::kRows);
              const uint64_t db0 = umma_desc_sw128_kmajor(smem_u32(stg + s * wt::kStgBytes));
#pragma unroll
              for (int kk = 0; kk < wt::kKChunk / 16; ++kk)
#pragma unroll
                for (int p = 0; p < 3; ++p)
                  umma_bf16_ts(d, a_hi + (uint32_t)(p * 32 + kk * 8), db0 + (uint64_t)(2 * kk), idesc_b16,
                               (kc > 0 || kk > 0 || p > 0) ? 1u : 0u);
              umma_commit(&stg_empty[s]);
              ++j;
              continue;
            }
            if (!(ok = mbar_wait(&chk[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
            tc_fence_after();
            const uint4 lf = *reinterpret_cast<const uint4*>(lo_flag + s * CW);  // the 16 warps' flags
            const bool lo_any = (lf.x | lf.y | lf.z | lf.w) != 0u;
            const uint32_t d = tmem + wt::kDcol + (uint32_t)(t * wt::kRows);
            // k-step kk starts (kk >> 2) atoms + 32 (kk & 3) bytes into the slot: the descriptor's
            // address field (bytes >> 4, no carry out for shared-memory addresses) advances by that
            const uint64_t db0 = umma_desc_sw128_kmajor(smem_u32(stg + s * wt::kStgBytes));
#pragma unroll
            for (int kk = 0; kk < wt::kKChunk / 8; ++kk) {
              const uint64_t db = db0 + (uint64_t)(((kk >> 2) * wt::kAtomBytes + (kk & 3) * 32) >> 4);
              umma_tf32_ts(d, a_hi + (uint32_t)kk * 8u, db, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
              umma_tf32_ts(d, a_lo + (uint32_t)kk * 8u, db, idesc, 1u);
            }
            // lo_go and lo_full complete once per slot use, lo pass or not
            umma_commit(&lo_go[s]);
            if (lo_any) {
              // the slot's warps rewrite it with the remainders once the hi MMAs have read it
              if (!(ok = mbar_wait(&lo_full[s], (j / NS) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < wt::kKChunk / 8; ++kk) {
                const uint64_t db = db0 + (uint64_t)(((kk >> 2) * wt::kAtomBytes + (kk & 3) * 32) >> 4);
                umma_tf32_ts(d, a_hi + (uint32_t)kk * 8u, db, idesc, 1u);
              }
            }
            umma_commit(&stg_empty[s]);
            ++j;
          }
          if (!ok) break;
          commit(&a_empty[ab]);
          ++ja;
        }
        if (ok) commit(acc_full);
      }
      if (!ok) {  // issued MMAs finish before TMEM and shared memory are released
        commit(drain);
        mbar_wait<kPair>(drain, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- weight-piece producer
    if (lane == 0) {
      int jp = 0;
      bool ok = true;
      // pieces 0, 1: tf32 hi; 2, 3: tf32 lo (spike-linear) or the two bf16 atoms (linear op);
      // packed spikes: the three bf16 atoms b1, b2, b3
      const unsigned char* img = a.wimg + (size_t)n_tile * nk * wt::kPieces * wt::kPieceBytes;
      const unsigned char* img16 = kRelu ? nullptr : a.wimg_b16 + (size_t)n_tile * nk * 2 * wt::kPieceBytes;
      const unsigned char* img3 = kBits ? a.wimg_b16x3 + (size_t)n_tile * nk * 3 * wt::kPieceBytes : nullptr;
      for (int c = 0; c < groups * nk && ok; ++c) {
        const int kc = c % nk;
        for (int p = 0; p < PPC; ++p, ++jp) {
          const int sp = jp % NP;
          if (jp >= NP && !(ok = mbar_wait(&pc_empty[sp], ((jp / NP) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
            break;
          const unsigned char* src = kBits                ? img3 + ((size_t)kc * 3 + p) * wt::kPieceBytes
                                     : (kRelu || p < 2) ? img + ((size_t)kc * wt::kPieces + p) * wt::kPieceBytes
                                                        : img16 + ((size_t)kc * 2 + (p - 2)) * wt::kPieceBytes;
          mbar_arrive_expect_tx(&pc_full[sp], wt::kPieceBytes);
          bulk_g2s(pcs + (size_t)sp * wt::kPieceBytes, src, wt::kPieceBytes, &pc_full[sp]);
        }
      }
      for (int i = (jp > NP ? jp - NP : 0); i < jp; ++i)
        mbar_wait(&pc_full[i % NP], (i / NP) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp < 3 + CW) {
    if constexpr (!kRelu) {
      linear_converter<kEpi, NS, NL, G, kPair>(warp - 3, lane, stg, lob, stg_full, stg_empty, lof, loe, acc_full,
                                               acc_empty, abort_flag, a, tmem, n0, r_begin, r_end, nk, groups, tiles,
                                               rank);
    } else if constexpr (kBits) {
      bits_converter<NS, G>(warp - 3, lane, stg, chk, stg_empty, acc_full, acc_empty, abort_flag, a, tmem, n0, r_begin,
                            r_end, nk, groups, tiles);
    } else {
      tf32_converter<NS, G, kRelu, true>(warp - 3, lane, stg, stg_full, chk, stg_empty, lo_go, lo_full, lo_flag, row_count,
                                   abort_flag, a, r_begin, r_end, n_tile, nk, groups, tiles);
    }
  } else {
    // ---------------------------------------------------------------- weight loaders + epilogue (warps 19-22)
    // Warp q = warp & 3 owns TMEM lanes [32q, 32q+32): output columns n0 + 32q + lane.
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int nl = q * 32 + lane;
    const int n = n0 + nl;
    const float bias_n = (a.bias != nullptr && n < a.N) ? a.bias[n] : 0.0f;
    const int total_chunks = groups * nk;
    int ja = 0, jp = 0;
    bool ok = true;
    // one 64-wide K chunk of the weights: four 16 KB pieces -> TMEM buffer ja & 1
    auto load_chunk = [&]() -> bool {
      const int ab = ja & 1;
      if (ja >= 2 && !mbar_wait<kPair>(&a_empty[ab], ((ja >> 1) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))
        return false;
      tc_fence_after();
      for (int p = 0; p < PPC; ++p, ++jp) {
        const int sp = jp % NP;
        if (!mbar_wait(&pc_full[sp], (jp / NP) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) return false;
        const unsigned char* src = pcs + (size_t)sp * wt::kPieceBytes;
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(src + sw128_chunk((uint32_t)nl, (uint32_t)c));
          r[4 * c] = v.x;
          r[4 * c + 1] = v.y;
          r[4 * c + 2] = v.z;
          r[4 * c + 3] = v.w;
        }
        tmem_st_32x32b_x32(tmem + lane_base + wt::kAcol + (uint32_t)(ab * 128 + p * 32), r);
        __syncwarp();
        if (lane == 0) mbar_arrive(&pc_empty[sp]);  // the piece's words are in registers / issued
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_rank0(&a_full[ab]);  // the pair's MMAs wait on CTA 0's barrier
        else mbar_arrive(&a_full[ab]);
      }
      ++ja;
      return true;
    };
    // linear op and packed spikes: the converters run the epilogue, the loaders only stream the weight chunks
    constexpr bool kConvEpi = !kRelu || kBits;
    if constexpr (kConvEpi) {
      while (ok && ja < total_chunks) ok = load_chunk();
    }
    for (int g = 0; g < groups && ok && !kConvEpi; ++g) {
      const int pg = groups - 1 - g;  // groups in reverse order: the partial group first
      const int tg = min(G, tiles - pg * G);
      // this group's chunks, then the next group's first two (their buffers
      // free up with this group's last MMAs), then this group's epilogue
      while (ok && ja < min(total_chunks, (g + 1) * nk + 2)) ok = load_chunk();
      if (!ok) break;
      if (!(ok = mbar_wait(acc_full, g & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
      tc_fence_after();
      for (int t = 0; t < tg; ++t) {
        const int64_t row0 = r_begin + (int64_t)(pg * G + t) * wt::kRows;
#pragma unroll 1
        for (int rb = 0; rb < wt::kRows; rb += 16) {
          if (row0 + rb >= r_end) break;
          GsmcIn cin[4];  // GSMC: the inputs of this warp's 4 rows, requested before the accumulators are read
          if constexpr (kEpi == kEpiGsmc) {
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
              const int64_t row = row0 + rb + q * 4 + r4;
              if (row < r_end) cin[r4] = gsmc_load(a.cell, row, n_tile * 32 + lane);
            }
          }
          float v[16];
          tmem_ld16(tmem + lane_base + wt::kDcol + (uint32_t)(t * wt::kRows + rb), v);
          tmem_wait_ld();
          tmem_reg_fence(v);
          if constexpr (kEpi == kEpiGsmc) {
            // The tile's 128 columns are the f, i, o, g projections (lane quarters 0-3) of the
            // 32 channels 32 * n_tile + lane.  Each warp publishes its gate for 16 rows, then
            // updates the cells of 4 of those rows for the 32 channels (all four gates at hand).
            float* xb = xbuf + ((rb >> 4) & 1) * (4 * 16 * 32);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) xb[(q * 16 + jj) * 32 + lane] = v[jj];
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
            const int ch = n_tile * 32 + lane;
#pragma unroll
            for (int r4 = 0; r4 < 4; ++r4) {
              const int rr = q * 4 + r4;
              const int64_t row = row0 + rb + rr;
              if (row < r_end)
                gsmc_update(a.cell, row, ch, cin[r4], xb[(0 * 16 + rr) * 32 + lane], xb[(1 * 16 + rr) * 32 + lane],
                            xb[(2 * 16 + rr) * 32 + lane], xb[(3 * 16 + rr) * 32 + lane]);
            }
          } else if constexpr (kEpi == kEpiHeavisideBits || kEpi == kEpiVSpikeBits) {
            // one ballot per row gives the row's word of this warp's 32 columns (N % 32 == 0:
            // a warp's columns are all in range or all out); lane jj stores row rb + jj's word
            if (n0 + q * 32 < a.N) {
              uint32_t word = 0u;
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const float spike = wt_epilogue<kEpi == kEpiHeavisideBits ? kEpiHeaviside : kEpiVSpike>(
                    v[jj] + bias_n, a.thr);
                const uint32_t b = __ballot_sync(0xffffffffu, spike > 0.0f);
                if (lane == jj) word = b;
              }
              const int NW = a.N / 32;
              if (lane < 16 && row0 + rb + lane < r_end)
                reinterpret_cast<uint32_t*>(a.Y)[(row0 + rb + lane) * NW + (n0 / 32 + q)] = word;
            }
          } else if (n < a.N) {
            float* y = a.Y + (row0 + rb) * a.N + n;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              if (row0 + rb + jj < r_end) y[(int64_t)jj * a.N] = wt_epilogue<kEpi>(v[jj] + bias_n, a.thr);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[0]);
        mbar_arrive(&acc_empty[1]);
      }
    }
    tmem_wait_st();
  }

  role_join();
  if constexpr (kPair) cluster_sync_all();  // neither CTA frees TMEM or exits while the pair still works
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem, wt::kTmemCols);
    else tmem_dealloc(tmem, wt::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
// The weight image is the tf32 kernel's (tf32_img_bytes, w_image_tf32_kernel)
// with NT = 128: per N tile and K chunk the pieces hi k0-31 | hi k32-63 |
// lo k0-31 | lo k32-63, each 128 rows x 128 B in the 128-byte swizzle, and in
// the bf16 region (a.wimg_b16) the linear op's pieces bf16(w - hi) k0-63 |
// bf16(hi) k0-63 of the same size.
template <int kEpi, bool kRelu, bool kBits = false, bool kPair = false>
int launch_wt_inst(const CUtensorMap& map, TcArgs a, int n_tiles, cudaStream_t stream) {
  auto kern = spike_linear_wt_kernel<kEpi, kRelu, kBits, kPair>;
  constexpr size_t smem = wt::Ring<kRelu, kEpi == kEpiGsmc, kPair>::kSmemBytes;
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int pairs_fit = 0;
  if constexpr (kPair) {
    // as many row ranges as keep every pair resident at once (pairs need two SMs of one
    // cluster-capable group, so fewer than SMs / 2 may fit): no second wave
    static std::atomic<int> max_pairs[64];  // per device; host threads may launch concurrently
    int dev = 0;
    SPK_CUDA_TRY(cudaGetDevice(&dev));
    int mp = max_pairs[dev & 63].load(std::memory_order_relaxed);
    if (mp <= 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)n_tiles, 1);
      cfg.blockDim = dim3(wt::kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      SPK_CUDA_TRY(cudaOccupancyMaxActiveClusters(&mp, kern, &cfg));
      if (mp <= 0) return fail(SPK_ECUDA, "the CTA-pair kernel fits no cluster on this device");
      max_pairs[dev & 63].store(mp, std::memory_order_relaxed);
    }
    pairs_fit = mp;
    const int ranges = mp / (n_tiles / 2) > 0 ? mp / (n_tiles / 2) : 1;
    a.rows_per_cta = ceil_div(ceil_div(a.R, ranges), 32) * 32;
  }
  const int64_t gx = ceil_div(a.R, a.rows_per_cta);
  const dim3 grid = kPair ? dim3((unsigned)n_tiles, (unsigned)gx) : dim3((unsigned)gx, (unsigned)n_tiles);
  prof_before(SPK_KERNEL_DENSE, stream);
  if constexpr (kPair) {
    const cudaError_t e = launch_dependent_cluster(kern, grid, dim3(wt::kThreads), smem, stream, 2u, true, map, a);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(SPK_ECUDA, "CTA-pair launch failed: %s (grid %u x %u, %zu B shared, %d pairs fit)",
                  cudaGetErrorString(e), grid.x, grid.y, smem, pairs_fit);
    }
  } else {
    SPK_CUDA_TRY(launch_dependent(kern, grid, dim3(wt::kThreads), smem, stream, map, a));
  }
  prof_after(SPK_KERNEL_DENSE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

// CTA pairs for the linear op: SPK_WT_PAIR=1 in the environment turns them on
// (read at every launch, so a test can compare both forms in one process).
// Off by default: bit-identical to the single-CTA form but slower at the
// model's geometries (the pair's MMAs wait for the slower CTA's converters and
// for both CTAs' epilogues every group).
inline bool wt_pair_enabled() {
  const char* e = getenv("SPK_WT_PAIR");
  return e != nullptr && atoi(e) != 0;
}

inline TcArgs wt_args(int64_t R, int K, int N, const TcPlan& p, const unsigned char* img, const TcOut& o, float thr) {
  TcArgs a{};
  a.R = R;
  a.K = K;
  a.N = N;
  a.nk = p.nk;
  a.KWP = 2 * p.nk;
  a.wimg = img;
  a.wimg_b16 = img + tf32_img_region_bytes(p);
  a.wimg_b16x3 = img + img_b16x3_offset(p);
  a.bias = o.bias;
  a.Y = o.Y;
  a.y_vec = 0;
  a.bitmap = o.bitmap;
  a.row_cnt = o.row_cnt;
  a.nonunit = o.nonunit;
  a.blk_sum = o.blk_sum;
  a.sup_sum = o.sup_sum;
  a.gate = o.gate;
  a.early_s = o.early_s;
  a.thr = thr;
  const int sms = sm_count();
  const int ranges = sms / p.n_tiles > 0 ? sms / p.n_tiles : 1;
  a.rows_per_cta = ceil_div(ceil_div(a.R, ranges), 32) * 32;
  return a;
}

// act < 0: spike-linear (relu'(S) with the CSR outputs of `o`); act >= 0: the
// linear-activation op with epilogue `act` (WtEpilogue) and threshold `thr`;
// kEpiHeavisideBits writes the spikes packed into o.Y as uint32 [R][N/32].
int launch_wt(const float* S, int64_t R, int K, int N, const TcPlan& p, const unsigned char* img, const TcOut& o,
              cudaStream_t stream, int act = -1, float thr = 0.0f) {
  if (p.NT != wt::kLanes) return fail(SPK_EINVAL, "weights-in-TMEM kernel needs 128-column N tiles (NT=%d)", p.NT);
  if ((act == kEpiHeavisideBits || act == kEpiVSpikeBits) && N % 32 != 0)
    return fail(SPK_EINVAL, "packed spikes need N %% 32 == 0 (N=%d)", N);
  CUtensorMap map;
  int rc = make_map_2d_swizzled_f32(&map, S, R, K, K, 32, wt::kBoxRows, "S");
  if (rc) return rc;
  const TcArgs a = wt_args(R, K, N, p, img, o, thr);
  // the linear op in CTA pairs when the N tiles pair up (no automatic-choice gate on this op)
  const bool pair = act >= 0 && p.n_tiles % 2 == 0 && o.gate == nullptr && wt_pair_enabled();
  switch (act) {
    case -1: return launch_wt_inst<kEpiLinear, true>(map, a, p.n_tiles, stream);
    case kEpiLinear:
      return pair ? launch_wt_inst<kEpiLinear, false, false, true>(map, a, p.n_tiles, stream)
                  : launch_wt_inst<kEpiLinear, false>(map, a, p.n_tiles, stream);
    case kEpiHeaviside:
      return pair ? launch_wt_inst<kEpiHeaviside, false, false, true>(map, a, p.n_tiles, stream)
                  : launch_wt_inst<kEpiHeaviside, false>(map, a, p.n_tiles, stream);
    case kEpiVSpike:
      return pair ? launch_wt_inst<kEpiVSpike, false, false, true>(map, a, p.n_tiles, stream)
                  : launch_wt_inst<kEpiVSpike, false>(map, a, p.n_tiles, stream);
    case kEpiHeavisideBits:
      return pair ? launch_wt_inst<kEpiHeavisideBits, false, false, true>(map, a, p.n_tiles, stream)
                  : launch_wt_inst<kEpiHeavisideBits, false>(map, a, p.n_tiles, stream);
    case kEpiVSpikeBits:
      return pair ? launch_wt_inst<kEpiVSpikeBits, false, false, true>(map, a, p.n_tiles, stream)
                  : launch_wt_inst<kEpiVSpikeBits, false>(map, a, p.n_tiles, stream);
    default: break;
  }
  return fail(SPK_EINVAL, "unknown activation %d", act);
}

// One plane of the GSMC recurrence: the gate projections gr = s_prev W_rec^T
// of the rows s_prev [R][K = d] on the tensor cores (img: the image of W_rec
// with its rows permuted so that N tile c holds the f, i, o, g rows of the
// channels 32c .. 32c+31) and the cell update in the epilogue; gr never
// leaves the SM.
int launch_wt_gsmc(const float* s_prev, int64_t R, int d, const TcPlan& p, const unsigned char* img,
                   const GsmcCell& cell, cudaStream_t stream) {
  if (p.NT != wt::kLanes || p.n_tiles * 32 != d) return fail(SPK_EINVAL, "GSMC recurrence: d %% 32 == 0 required");
  CUtensorMap map;
  int rc = make_map_2d_swizzled_f32(&map, s_prev, R, d, d, 32, wt::kBoxRows, "s");
  if (rc) return rc;
  TcOut o{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  o.early_s = 0;  // the previous plane's kernel writes s_prev
  TcArgs a = wt_args(R, d, 4 * d, p, img, o, 0.0f);
  a.cell = cell;
  return launch_wt_inst<kEpiGsmc, true>(map, a, p.n_tiles, stream);
}

// Spike-linear over packed spikes bits [R][K/32] (K % 64 == 0): Y = S W (+ bias), fp32 W.
int launch_wt_bits(const uint32_t* bits, int64_t R, int K, int N, const TcPlan& p, const unsigned char* img,
                   const TcOut& o, cudaStream_t stream) {
  if (p.NT != wt::kLanes) return fail(SPK_EINVAL, "weights-in-TMEM kernel needs 128-column N tiles (NT=%d)", p.NT);
  if (K % 64 != 0) return fail(SPK_EINVAL, "packed spikes need K %% 64 == 0 (K=%d)", K);
  CUtensorMap map;
  memset(&map, 0, sizeof(map));  // no tensor map: the converters read the words themselves
  TcArgs a = wt_args(R, K, N, p, img, o, 0.0f);
  a.bits_in = bits;
  return launch_wt_inst<kEpiLinear, true, true>(map, a, p.n_tiles, stream);
}

}  // namespace spk
