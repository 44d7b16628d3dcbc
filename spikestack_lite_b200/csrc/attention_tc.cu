// Spiking linear attention on the 5th-generation tensor cores.
//
// AstrocyteHebbianAttention (attention.py:105-136) per (bt, head h), with
// k_w[n, i] = k[n, i] * lam_i^(L-1-n):
//   kv[i, j]  = sum_n k_w[n, i] v[n, j]      key_mass[i] = sum_n k_w[n, i]
//   out[n, j] = (sum_i q[n, i] kv[i, j]) / ((sum_i q[n, i] key_mass[i]) + eps)
// q, k, v and out stay in the d_model layout [BT, L, d] (channel c = h*dh + i).
// Heads are processed in groups of 128 channels (128 / dh heads per group), so
// d must be a multiple of 128 and dh one of 16, 32, 64.
//
// Pass 1 (attn_kv_tc_kernel), one unit = (bt, group): the tensor cores form
// kv^T = v^T k_w over the whole sequence (M = 128 v channels, N = 128 k
// channels, K = positions), both operands MN-major straight from the
// row-major sequence; cross-head blocks of the product are computed and
// discarded.  k_w = k * decay (decay table from powf, as the reference
// engine) is split into bf16 hi + lo; v is exact in bf16 for spikes (any
// other value adds a v_lo pass).  key_mass is summed in fp32 by the
// converter threads.  The epilogue writes, per unit, the B operand of pass 2
// as a ready-to-copy image: [hi | lo] x [2 K-chunks] x [144 rows x 128 B],
// K-major, 128-byte swizzled, with row j = the block-diagonal column j of kv
// (nonzero only for k channels of j's head) and rows 128 + h = key_mass of
// head h.
// Pass 2 (attn_out_tc_kernel), one item = (unit, 128-position tile):
// D[n, 0:144] = q_tile x image^T (q exact in bf16 for spikes), then
// out = D[:, j] / (D[:, 128 + head(j)] + eps) in the epilogue.
//
// Warp roles of both kernels (448 threads, one CTA per SM): warp 0 TMA
// producer, warp 1 TMEM owner + MMA issuer, warps 2-9 converters, warps
// 10-13 epilogue.  Every wait is bounded (2 s) and reports
// SPK_DEV_PIPE_TIMEOUT; issued copies and MMAs are drained before exit and
// TMEM is always freed.  Every copy lands in this CTA's own shared memory.
#include "tma.cuh"

namespace spk {

namespace at {

constexpr int kGrp = 128;                        // channels per head group
constexpr int kBoxCols = 64, kBoxRows = 32;      // TMA box: 64 fp32 columns x 32 rows
constexpr int kBoxBytes = kBoxCols * kBoxRows * 4;
// packed spikes (32 channels per word): a head group's 128 channels are 4 words = 16 bytes per position
constexpr int kBitWords = kGrp / 32;
constexpr int kBitBox1 = kBitWords * 32 * 4;     // pass 1: 32 positions
constexpr int kBitBox2 = kBitWords * 128 * 4;    // pass 2: one 128-position tile
constexpr int kConvWarps = 8;
constexpr int kThreads = 32 * (2 + kConvWarps + 4);

// pass 1
constexpr int kP1 = 32;                          // positions per chunk = two MMA k-steps
constexpr int kNS1 = 3;                          // staging slots: k, v, decay (2 boxes each)
constexpr int kStg1 = 6 * kBoxBytes;             // 48 KB
constexpr int kOp1 = kP1 * kGrp * 2;             // one MN-major bf16 operand: 8 KB
constexpr int kNA1 = 2;                          // operand slots: vT_hi, vT_lo, kw_hi, kw_lo
constexpr uint32_t kMnStride1 = 1024;            // atom stride along channels
constexpr uint32_t kKStride1 = 2048;             // atom stride along positions (2 channel atoms)

// B image of pass 2
constexpr int kImgRows = kGrp + 16;              // 128 kv columns + 16 key-mass / zero rows
constexpr int kImgChunk = kImgRows * 128;        // one 64-wide K chunk of one half: 18 KB
constexpr int kImgPart = 2 * kImgChunk;          // K = 128: 36 KB
constexpr int kImgBytes = 2 * kImgPart;          // hi + lo: 72 KB per unit

// pass 2
constexpr int kRows2 = 128;                      // positions per item (MMA M)
constexpr int kStg2 = kRows2 * 256;              // staging slot: 128 rows x 64 fp32 = 32 KB
constexpr int kNS2 = 2;                          // every converter warp consumes every slot
constexpr int kA2 = kRows2 * 128;                // A half (hi or lo) of one K chunk: 16 KB
constexpr int kNA2 = 2;
constexpr int kAcc2 = 256;                       // TMEM column stride of the two accumulators

constexpr size_t kTail1 = 8 * (2 * kNS1 + 2 * kNA1 + 2 + 2 + 2 + 2 + 1) + 4 * kNA1 * kConvWarps +
                          4 * 2 * kConvWarps * kGrp + 16;
constexpr size_t kSmem1 = 1024 + (size_t)kNS1 * kStg1 + (size_t)kNA1 * 4 * kOp1 + ((kTail1 + 255) / 256) * 256;
constexpr size_t kTail2 = 8 * (2 * kNS2 + 2 * kNA2 + 2 + 2 + 2 + 1) + 4 * kNA2 * kConvWarps + 16;
constexpr size_t kSmem2 =
    1024 + (size_t)kImgBytes + (size_t)kNS2 * kStg2 + (size_t)kNA2 * 2 * kA2 + ((kTail2 + 255) / 256) * 256;
static_assert(kSmem1 <= 232448 && kSmem2 <= 232448, "shared memory budget");

}  // namespace at

struct AttnKvArgs {
  int64_t units;   // BT * groups
  int groups;      // d / 128
  int L;           // positions per bt
  int nch;         // ceil(L / 32)
  unsigned char* img;
};

struct AttnOutArgs {
  int64_t items;   // units * tiles
  int64_t per_cta; // contiguous items per CTA
  int groups, L, tiles, d;
  float eps;
  const unsigned char* img;
  float* out;
};

// Byte offset of (position p in [0, 32), channel c in [0, 128)) in a pass-1
// MN-major operand: atom (p / 8, c / 64), line p % 8, element c % 64.
__device__ __forceinline__ uint32_t p1_offset(int p, int c) {
  return (uint32_t)(((p >> 3) * 2 + (c >> 6)) * 1024) + sw128_offset_bf16((uint32_t)(p & 7), (uint32_t)(c & 63));
}

__device__ __forceinline__ uint32_t upper_halves(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x7632); }

// kBits: k and v arrive packed (uint32 words [BT*L][d/32]); the converters
// expand them to the same fp32 0 / 1 patterns the fp32 staging would hold.
template <int DH, bool kBits = false>
__global__ void __launch_bounds__(at::kThreads, 1)
    attn_kv_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_tab, AttnKvArgs a) {
  using namespace at;
  constexpr int G = kGrp / DH;  // heads per group
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  unsigned char* base = smem_aligned_1024(smem_dyn);
  unsigned char* stg = base;
  unsigned char* ops = stg + kNS1 * kStg1;
  float* km_part = reinterpret_cast<float*>(ops + kNA1 * 4 * kOp1);  // [2][kConvWarps][128], 16-byte aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(km_part + 2 * kConvWarps * kGrp);
  uint64_t* stg_full = bars;
  uint64_t* stg_empty = stg_full + kNS1;
  uint64_t* a_full = stg_empty + kNS1;
  uint64_t* a_empty = a_full + kNA1;
  uint64_t* acc_full = a_empty + kNA1;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* km_full = acc_empty + 2;
  uint64_t* km_empty = km_full + 2;
  uint64_t* drain = km_empty + 2;
  int* lo_flag = reinterpret_cast<int*>(drain + 1);  // [kNA1][kConvWarps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lo_flag + kNA1 * kConvWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t my_units =
      blockIdx.x < a.units ? (a.units - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS1; ++s) {
      mbar_init(&stg_full[s], 1);
      mbar_init(&stg_empty[s], kConvWarps);
    }
    for (int s = 0; s < kNA1; ++s) {
      mbar_init(&a_full[s], kConvWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 4);
      mbar_init(&km_full[s], kConvWarps);
      mbar_init(&km_empty[s], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the decay table comes from the previous kernel on the stream; pass 2 may
  // be scheduled now (it waits for this grid before reading the images)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_map(&tm_k);
      tma_prefetch_map(&tm_v);
      tma_prefetch_map(&tm_tab);
      int j = 0;
      bool ok = true;
      for (int64_t ul = 0; ul < my_units && ok; ++ul) {
        const int64_t u = blockIdx.x + ul * gridDim.x;
        const int64_t bt = u / a.groups;
        const int col = (int)(u % a.groups) * kGrp;
        for (int c = 0; c < a.nch; ++c) {
          const int s = j % kNS1;
          if (j >= kNS1 && !(ok = mbar_wait(&stg_empty[s], ((j / kNS1) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
            break;
          unsigned char* st = stg + s * kStg1;
          const int row = (int)(bt * a.L) + c * kP1;
          if constexpr (kBits) {  // one 16-byte-wide box of words each for k and v
            mbar_arrive_expect_tx(&stg_full[s], 2 * kBitBox1 + 2 * kBoxBytes);
            tma_load_2d(st + 0 * kBoxBytes, &tm_k, col / 32, row, &stg_full[s]);
            tma_load_2d(st + 2 * kBoxBytes, &tm_v, col / 32, row, &stg_full[s]);
          } else {
            mbar_arrive_expect_tx(&stg_full[s], kStg1);
            tma_load_2d(st + 0 * kBoxBytes, &tm_k, col, row, &stg_full[s]);
            tma_load_2d(st + 1 * kBoxBytes, &tm_k, col + 64, row, &stg_full[s]);
            tma_load_2d(st + 2 * kBoxBytes, &tm_v, col, row, &stg_full[s]);
            tma_load_2d(st + 3 * kBoxBytes, &tm_v, col + 64, row, &stg_full[s]);
          }
          tma_load_2d(st + 4 * kBoxBytes, &tm_tab, col, c * kP1, &stg_full[s]);
          tma_load_2d(st + 5 * kBoxBytes, &tm_tab, col + 64, c * kP1, &stg_full[s]);
          ++j;
        }
      }
      for (int i = (j > kNS1 ? j - kNS1 : 0); i < j; ++i)
        mbar_wait(&stg_full[i % kNS1], (i / kNS1) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(128, 128, true, true);
      int j = 0;
      bool ok = true;
      for (int64_t ul = 0; ul < my_units && ok; ++ul) {
        const int ab = (int)(ul & 1);
        if (ul >= 2 && !(ok = mbar_wait(&acc_empty[ab], ((ul / 2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * 128);
        for (int c = 0; c < a.nch; ++c) {
          const int sa = j % kNA1;
          if (!(ok = mbar_wait(&a_full[sa], (j / kNA1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          tc_fence_after();
          int lo_any = 0;
#pragma unroll
          for (int w = 0; w < kConvWarps; ++w) lo_any |= lo_flag[sa * kConvWarps + w];
          const uint32_t o = smem_u32(ops + sa * 4 * kOp1);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            const uint32_t adv = (uint32_t)ks * 2 * kKStride1;  // 16 positions = two K atoms
            const uint64_t va_hi = umma_desc_sw128_mnmajor(o + adv, kMnStride1, kKStride1);
            const uint64_t va_lo = umma_desc_sw128_mnmajor(o + kOp1 + adv, kMnStride1, kKStride1);
            const uint64_t kb_hi = umma_desc_sw128_mnmajor(o + 2 * kOp1 + adv, kMnStride1, kKStride1);
            const uint64_t kb_lo = umma_desc_sw128_mnmajor(o + 3 * kOp1 + adv, kMnStride1, kKStride1);
            umma_f16_ss(d, va_hi, kb_hi, idesc, (c > 0 || ks > 0) ? 1u : 0u);
            umma_f16_ss(d, va_hi, kb_lo, idesc, 1u);
            if (lo_any) umma_f16_ss(d, va_lo, kb_hi, idesc, 1u);
          }
          umma_commit(&a_empty[sa]);
          ++j;
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      if (!ok) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);
      }
    }
  } else if (warp < 2 + kConvWarps) {
    // ---------------------------------------------------------------- converters
    // Warp cw owns positions 4cw..4cw+3 of each chunk; lane l owns channels
    // 4l..4l+3 (box l / 16, column 4 (l % 16)).
    const int cw = warp - 2;
    const int box = lane >> 4;
    const int cc = (lane & 15) * 4;
    const int ch = box * 64 + cc;
    uint32_t dirty = (1u << kNA1) - 1u;  // operand slots whose vT_lo may hold nonzero data
    int j = 0;
    bool ok = true;
    for (int64_t ul = 0; ul < my_units && ok; ++ul) {
      float km[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < a.nch; ++c) {
        const int s = j % kNS1, sa = j % kNA1;
        if (!(ok = mbar_wait(&stg_full[s], (j / kNS1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        if (j >= kNA1 && !(ok = mbar_wait(&a_empty[sa], ((j / kNA1) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
          break;
        const unsigned char* st = stg + s * kStg1;
        uint4 kk[4], vv[4];
        float4 ww[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int off = box * kBoxBytes + (4 * cw + i) * 256 + cc * 4;
          if constexpr (kBits) {
            const int wi = (4 * cw + i) * kBitWords + (ch >> 5);
            kk[i] = nibble_f32x4(reinterpret_cast<const uint32_t*>(st)[wi] >> (ch & 31));
            vv[i] = nibble_f32x4(reinterpret_cast<const uint32_t*>(st + 2 * kBoxBytes)[wi] >> (ch & 31));
          } else {
            kk[i] = *reinterpret_cast<const uint4*>(st + off);
            vv[i] = *reinterpret_cast<const uint4*>(st + 2 * kBoxBytes + off);
          }
          ww[i] = *reinterpret_cast<const float4*>(st + 4 * kBoxBytes + off);
        }
        const int nvalid = min(kP1, a.L - c * kP1);
        unsigned char* op = ops + sa * 4 * kOp1;
        uint32_t vlow = 0u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int p = 4 * cw + i;
          if (p >= nvalid) {  // rows past the sequence belong to the next bt
            kk[i] = make_uint4(0u, 0u, 0u, 0u);
            vv[i] = make_uint4(0u, 0u, 0u, 0u);
          }
          const float x0 = __uint_as_float(kk[i].x) * ww[i].x, x1 = __uint_as_float(kk[i].y) * ww[i].y;
          const float x2 = __uint_as_float(kk[i].z) * ww[i].z, x3 = __uint_as_float(kk[i].w) * ww[i].w;
          km[0] += x0;
          km[1] += x1;
          km[2] += x2;
          km[3] += x3;
          __nv_bfloat16 h[4], l[4];
          split_bf16(x0, h[0], l[0]);
          split_bf16(x1, h[1], l[1]);
          split_bf16(x2, h[2], l[2]);
          split_bf16(x3, h[3], l[3]);
          const uint32_t off = p1_offset(p, ch);
          *reinterpret_cast<uint2*>(op + 2 * kOp1 + off) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
          *reinterpret_cast<uint2*>(op + 3 * kOp1 + off) = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
          vlow |= (vv[i].x | vv[i].y | vv[i].z | vv[i].w) & 0xffffu;
          *reinterpret_cast<uint2*>(op + off) =
              make_uint2(upper_halves(vv[i].x, vv[i].y), upper_halves(vv[i].z, vv[i].w));
        }
        // release the staging slot only after every lane stored values computed
        // from its loads (so the loads are complete before the next copy lands)
        __syncwarp();
        if (lane == 0) mbar_arrive(&stg_empty[s]);
        // v values that bf16 does not hold exactly: exact hi/lo split for this warp
        const bool warp_lo = __any_sync(0xffffffffu, vlow != 0u);
        if (warp_lo || ((dirty >> sa) & 1u)) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t off = p1_offset(4 * cw + i, ch);
            uint2 lo_pk = make_uint2(0u, 0u);
            if (warp_lo) {
              __nv_bfloat16 h[4], l[4];
              split_bf16(__uint_as_float(vv[i].x), h[0], l[0]);
              split_bf16(__uint_as_float(vv[i].y), h[1], l[1]);
              split_bf16(__uint_as_float(vv[i].z), h[2], l[2]);
              split_bf16(__uint_as_float(vv[i].w), h[3], l[3]);
              *reinterpret_cast<uint2*>(op + off) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
              lo_pk = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
            }
            *reinterpret_cast<uint2*>(op + kOp1 + off) = lo_pk;
          }
          dirty = warp_lo ? (dirty | (1u << sa)) : (dirty & ~(1u << sa));
        }
        if (lane == 0) lo_flag[sa * kConvWarps + cw] = warp_lo ? 1 : 0;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
        ++j;
      }
      if (!ok) break;
      // key-mass partials of this unit
      const int kb = (int)(ul & 1);
      if (ul >= 2 && !(ok = mbar_wait(&km_empty[kb], ((ul / 2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
      *reinterpret_cast<float4*>(km_part + (kb * kConvWarps + cw) * kGrp + ch) = make_float4(km[0], km[1], km[2], km[3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&km_full[kb]);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 10-13)
    const int q = warp & 3;
    const int jr = 32 * q + lane;          // v channel j: D row and image row
    constexpr int WC = DH < 32 ? 32 : DH;  // TMEM columns one warp loads
    const int c0 = (32 * q / WC) * WC;     // first of them (warp-uniform)
    const int hb = (jr / DH) * DH;         // k channels of j's head: [hb, hb + DH)
    for (int64_t ul = 0; ul < my_units; ++ul) {
      const int ab = (int)(ul & 1);
      if (!mbar_wait(&acc_full[ab], (ul / 2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
      if (!mbar_wait(&km_full[ab], (ul / 2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
      tc_fence_after();
      const int64_t u = blockIdx.x + ul * gridDim.x;
      unsigned char* img = a.img + u * (int64_t)kImgBytes;
      // kv^T row jr restricted to the loaded columns
      float vals[WC];
      const uint32_t tb = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * 128 + c0);
#pragma unroll
      for (int t = 0; t < WC / 16; ++t) tmem_ld16(tb + 16u * t, *reinterpret_cast<float(*)[16]>(&vals[16 * t]));
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < WC / 16; ++t) tmem_reg_fence(*reinterpret_cast<float(*)[16]>(&vals[16 * t]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      // image row jr: the head block from the loaded columns, zeros elsewhere
#pragma unroll
      for (int t = 0; t < WC / 8; ++t) {
        const int k0 = c0 + 8 * t;
        uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
        if (k0 >= hb && k0 < hb + DH) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat16 h0, l0, h1, l1;
            split_bf16(vals[8 * t + 2 * e], h0, l0);
            split_bf16(vals[8 * t + 2 * e + 1], h1, l1);
            hw[e] = pack_bf16x2(h0, h1);
            lw[e] = pack_bf16x2(l0, l1);
          }
          hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        const uint32_t off = (uint32_t)((k0 >> 6) * kImgChunk) + sw128_offset_bf16((uint32_t)jr, (uint32_t)(k0 & 63));
        *reinterpret_cast<uint4*>(img + off) = hi;
        *reinterpret_cast<uint4*>(img + kImgPart + off) = lo;
      }
#pragma unroll
      for (int k0 = 0; k0 < kGrp; k0 += 8) {
        if (k0 >= c0 && k0 < c0 + WC) continue;
        const uint32_t off = (uint32_t)((k0 >> 6) * kImgChunk) + sw128_offset_bf16((uint32_t)jr, (uint32_t)(k0 & 63));
        *reinterpret_cast<uint4*>(img + off) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(img + kImgPart + off) = make_uint4(0u, 0u, 0u, 0u);
      }
      // key-mass rows 128 + h (h < G): key_mass of head h's channels (partials
      // of the converter warps summed in warp order), zeros elsewhere
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int piece = jr + 128 * r;     // 256 pieces of 16 B per half
        const int row = kGrp + piece / 16;
        const int k0 = (piece % 16) * 8;
        uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
        if (row - kGrp < G && k0 / DH == row - kGrp) {
          float kmv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) kmv[e] = 0.f;
#pragma unroll
          for (int w = 0; w < kConvWarps; ++w) {
            const float4 p0 = *reinterpret_cast<const float4*>(km_part + (ab * kConvWarps + w) * kGrp + k0);
            const float4 p1 = *reinterpret_cast<const float4*>(km_part + (ab * kConvWarps + w) * kGrp + k0 + 4);
            kmv[0] += p0.x; kmv[1] += p0.y; kmv[2] += p0.z; kmv[3] += p0.w;
            kmv[4] += p1.x; kmv[5] += p1.y; kmv[6] += p1.z; kmv[7] += p1.w;
          }
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat16 h0, l0, h1, l1;
            split_bf16(kmv[2 * e], h0, l0);
            split_bf16(kmv[2 * e + 1], h1, l1);
            hw[e] = pack_bf16x2(h0, h1);
            lw[e] = pack_bf16x2(l0, l1);
          }
          hi = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          lo = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        const uint32_t off = (uint32_t)((k0 >> 6) * kImgChunk) + sw128_offset_bf16((uint32_t)row, (uint32_t)(k0 & 63));
        *reinterpret_cast<uint4*>(img + off) = hi;
        *reinterpret_cast<uint4*>(img + kImgPart + off) = lo;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&km_empty[ab]);
    }
  }
  role_join();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// kBits: q arrives packed (uint32 words [BT*L][d/32]), expanded by the converters.
template <int DH, bool kBits = false>
__global__ void __launch_bounds__(at::kThreads, 1)
    attn_out_tc_kernel(const __grid_constant__ CUtensorMap tm_q, AttnOutArgs a) {
  using namespace at;
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  unsigned char* base = smem_aligned_1024(smem_dyn);
  unsigned char* bimg = base;                        // [hi | lo][2 K chunks][144 rows x 128 B]
  unsigned char* stg = bimg + kImgBytes;             // [kNS2][32 KB]
  unsigned char* a_hi = stg + kNS2 * kStg2;          // [kNA2][16 KB]
  unsigned char* a_lo = a_hi + kNA2 * kA2;           // [kNA2][16 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(a_lo + kNA2 * kA2);
  uint64_t* stg_full = bars;
  uint64_t* stg_empty = stg_full + kNS2;
  uint64_t* a_full = stg_empty + kNS2;
  uint64_t* a_empty = a_full + kNA2;
  uint64_t* acc_full = a_empty + kNA2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* b_full = acc_empty + 2;
  uint64_t* b_empty = b_full + 1;
  uint64_t* drain = b_empty + 1;
  int* lo_flag = reinterpret_cast<int*>(drain + 1);  // [kNA2][kConvWarps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lo_flag + kNA2 * kConvWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = (int64_t)blockIdx.x * a.per_cta;
  const int64_t i1 = min64(a.items, i0 + a.per_cta);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS2; ++s) {
      mbar_init(&stg_full[s], 1);
      mbar_init(&stg_empty[s], kConvWarps);
    }
    for (int s = 0; s < kNA2; ++s) {
      mbar_init(&a_full[s], kConvWarps);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 4);
    }
    mbar_init(b_full, 1);
    mbar_init(b_empty, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_map(&tm_q);
      int js = 0, jb = 0;
      int64_t cur = -1;
      bool ok = true;
      for (int64_t it = i0; it < i1 && ok; ++it) {
        const int64_t u = it / a.tiles;
        const int tile = (int)(it % a.tiles);
        const int64_t bt = u / a.groups;
        const int col = (int)(u % a.groups) * kGrp;
        const int nrows = min(kRows2, a.L - tile * kRows2);
        const int nbox = (nrows + kBoxRows - 1) / kBoxRows;
        for (int kc = 0; kc < 2 && ok; ++kc) {
          const int s = js % kNS2;
          if (js >= kNS2 && !(ok = mbar_wait(&stg_empty[s], ((js / kNS2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
            break;
          if constexpr (kBits) {  // the tile's 128 positions x 4 words (both K chunks read their half)
            mbar_arrive_expect_tx(&stg_full[s], (uint32_t)kBitBox2);
            tma_load_2d(stg + s * kStg2, &tm_q, col / 32, (int)(bt * a.L) + tile * kRows2, &stg_full[s]);
          } else {
            mbar_arrive_expect_tx(&stg_full[s], (uint32_t)(nbox * kBoxBytes));
            for (int b = 0; b < nbox; ++b)
              tma_load_2d(stg + s * kStg2 + b * kBoxBytes, &tm_q, col + 64 * kc,
                          (int)(bt * a.L) + tile * kRows2 + kBoxRows * b, &stg_full[s]);
          }
          ++js;
          if (kc == 0 && u != cur) {
            // a new unit: its kv image replaces the old one once every MMA on it is done
            if (jb > 0 && !(ok = mbar_wait(b_empty, (jb - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
            mbar_arrive_expect_tx(b_full, kImgBytes);
            bulk_g2s(bimg, a.img + u * (int64_t)kImgBytes, kImgPart, b_full);
            bulk_g2s(bimg + kImgPart, a.img + u * (int64_t)kImgBytes + kImgPart, kImgPart, b_full);
            ++jb;
            cur = u;
          }
        }
      }
      for (int i = (js > kNS2 ? js - kNS2 : 0); i < js; ++i)
        mbar_wait(&stg_full[i % kNS2], (i / kNS2) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
      if (jb > 0) mbar_wait(b_full, (jb - 1) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kRows2, kImgRows);
      int jt = 0, jb = 0, ti = 0;
      int64_t cur = -1;
      bool ok = true;
      for (int64_t it = i0; it < i1 && ok; ++it) {
        const int64_t u = it / a.tiles;
        if (u != cur) {
          if (cur >= 0) umma_commit(b_empty);  // fires once the MMAs on the old image are done
          if (!(ok = mbar_wait(b_full, jb & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          ++jb;
          cur = u;
        }
        const int ab = ti & 1;
        if (ti >= 2 && !(ok = mbar_wait(&acc_empty[ab], ((ti / 2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * kAcc2);
        for (int kc = 0; kc < 2; ++kc) {
          const int sa = jt % kNA2;
          if (!(ok = mbar_wait(&a_full[sa], (jt / kNA2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
          tc_fence_after();
          int lo_any = 0;
#pragma unroll
          for (int w = 0; w < kConvWarps; ++w) lo_any |= lo_flag[sa * kConvWarps + w];
          const uint64_t da_hi = umma_desc_sw128_kmajor(smem_u32(a_hi + sa * kA2));
          const uint64_t da_lo = umma_desc_sw128_kmajor(smem_u32(a_lo + sa * kA2));
          const uint64_t db_hi = umma_desc_sw128_kmajor(smem_u32(bimg + kc * kImgChunk));
          const uint64_t db_lo = umma_desc_sw128_kmajor(smem_u32(bimg + kImgPart + kc * kImgChunk));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adv = (uint64_t)(2 * kk);
            umma_f16_ss(d, da_hi + adv, db_hi + adv, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
            umma_f16_ss(d, da_hi + adv, db_lo + adv, idesc, 1u);
            if (lo_any) umma_f16_ss(d, da_lo + adv, db_hi + adv, idesc, 1u);
          }
          umma_commit(&a_empty[sa]);
          ++jt;
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
        ++ti;
      }
      if (!ok) {
        umma_commit(drain);
        mbar_wait(drain, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);
      }
    }
  } else if (warp < 2 + kConvWarps) {
    // ---------------------------------------------------------------- converters
    // Warp cw owns rows 16cw..16cw+15 of each 128-position tile; in load i a
    // lane holds 4 channels of row 16cw + 2i + lane / 16.  Every warp waits
    // on every phase of every staging slot (a warp that skipped phases could
    // not tell phase k from phase k + 2 of the same parity).
    const int cw = warp - 2;
    const int kq = (lane & 15) * 4;
    uint32_t dirty = (1u << kNA2) - 1u;
    int jt = 0;
    bool ok = true;
    for (int64_t it = i0; it < i1 && ok; ++it) {
      const int tile = (int)(it % a.tiles);
      const int nrows = min(kRows2, a.L - tile * kRows2);
      for (int kc = 0; kc < 2; ++kc) {
        const int s = jt % kNS2, sa = jt % kNA2;
        if (!(ok = mbar_wait(&stg_full[s], (jt / kNS2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT))) break;
        if (jt >= kNA2 && !(ok = mbar_wait(&a_empty[sa], ((jt / kNA2) - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)))
          break;
        uint4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rl = 16 * cw + 2 * i + (lane >> 4);
          if constexpr (kBits) {
            const int c = 64 * kc + kq;  // channel within the group
            v[i] = (rl < nrows) ? nibble_f32x4(reinterpret_cast<const uint32_t*>(stg + s * kStg2)[rl * kBitWords + (c >> 5)] >>
                                               (c & 31))
                                : make_uint4(0u, 0u, 0u, 0u);
          } else {
            v[i] = (rl < nrows) ? *reinterpret_cast<const uint4*>(stg + s * kStg2 + rl * 256 + kq * 4)
                                : make_uint4(0u, 0u, 0u, 0u);
          }
        }
        unsigned char* ahi = a_hi + sa * kA2;
        uint32_t low = 0u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rl = 16 * cw + 2 * i + (lane >> 4);
          low |= (v[i].x | v[i].y | v[i].z | v[i].w) & 0xffffu;
          *reinterpret_cast<uint2*>(ahi + sw128_offset_bf16((uint32_t)rl, (uint32_t)kq)) =
              make_uint2(upper_halves(v[i].x, v[i].y), upper_halves(v[i].z, v[i].w));
        }
        // release the staging slot only after every lane stored values computed
        // from its loads (so the loads are complete before the next copy lands)
        __syncwarp();
        if (lane == 0) mbar_arrive(&stg_empty[s]);
        const bool warp_lo = __any_sync(0xffffffffu, low != 0u);
        if (warp_lo || ((dirty >> sa) & 1u)) {
          unsigned char* alo = a_lo + sa * kA2;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rl = 16 * cw + 2 * i + (lane >> 4);
            const uint32_t off = sw128_offset_bf16((uint32_t)rl, (uint32_t)kq);
            uint2 lo_pk = make_uint2(0u, 0u);
            if (warp_lo) {
              __nv_bfloat16 h[4], l[4];
              split_bf16(__uint_as_float(v[i].x), h[0], l[0]);
              split_bf16(__uint_as_float(v[i].y), h[1], l[1]);
              split_bf16(__uint_as_float(v[i].z), h[2], l[2]);
              split_bf16(__uint_as_float(v[i].w), h[3], l[3]);
              *reinterpret_cast<uint2*>(ahi + off) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
              lo_pk = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
            }
            *reinterpret_cast<uint2*>(alo + off) = lo_pk;
          }
          dirty = warp_lo ? (dirty | (1u << sa)) : (dirty & ~(1u << sa));
        }
        if (lane == 0) lo_flag[sa * kConvWarps + cw] = warp_lo ? 1 : 0;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
        ++jt;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 10-13)
    // 16-lane x 256-bit TMEM loads: four threads per position, so every
    // store instruction writes whole 32-byte sectors of eight output rows.
    constexpr int G = kGrp / DH;
    const int q = warp & 3;
    const int ar = lane >> 2, cp = (lane & 3) * 2;
    int ti = 0;
    for (int64_t it = i0; it < i1; ++it) {
      const int64_t u = it / a.tiles;
      const int tile = (int)(it % a.tiles);
      const int ab = ti & 1;
      if (!mbar_wait(&acc_full[ab], (ti / 2) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
      tc_fence_after();
      float* obase = a.out + (u / a.groups) * a.L * (int64_t)a.d + (u % a.groups) * kGrp;
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        const int posA = tile * kRows2 + 32 * q + 16 * h2 + ar;  // this thread's rows: posA, posA + 8
        const uint32_t tb = tmem + ((uint32_t)(32 * q + 16 * h2) << 16) + (uint32_t)(ab * kAcc2);
        // key-mass products (columns 128 + h) of both rows, gathered from the quad
        float dn[16];
        tmem_ld_16x256b_x2(tb + kGrp, dn);
        tmem_wait_ld();
        tmem_reg_fence(dn);
        float inv[2][G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          // column 128 + h (h < 8) sits in quad member h / 2, element h % 2
          const int src = (lane & ~3) | (h >> 1);
          const float d0 = __shfl_sync(0xffffffffu, (h & 1) ? dn[1] : dn[0], src);
          const float d1 = __shfl_sync(0xffffffffu, (h & 1) ? dn[3] : dn[2], src);
          inv[0][h] = __frcp_rn(d0 + a.eps);
          inv[1][h] = __frcp_rn(d1 + a.eps);
        }
#pragma unroll
        for (int cb = 0; cb < kGrp; cb += 32) {  // unrolled: the head of each 8-column block is static
          float v[16];
          tmem_ld_16x256b_x4(tb + (uint32_t)cb, v);
          tmem_wait_ld();
          tmem_reg_fence(v);
#pragma unroll
          for (int jb = 0; jb < 4; ++jb) {
            const int col = cb + 8 * jb;
            const int hd = col / DH;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int pos = posA + 8 * rr;
              if (pos < a.L)
                *reinterpret_cast<float2*>(obase + (int64_t)pos * a.d + col + cp) =
                    make_float2(v[4 * jb + 2 * rr] * inv[rr][hd], v[4 * jb + 2 * rr + 1] * inv[rr][hd]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      ++ti;
    }
  }
  role_join();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

inline bool attn_tc_supported(int64_t BT, int L, int H, int dh, const float* q, const float* k, const float* v,
                              const float* out) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  const int64_t d = (int64_t)H * dh;
  return (dh == 16 || dh == 32 || dh == 64) && d % at::kGrp == 0 && (al & 15) == 0 && BT * (int64_t)L < (1ll << 31) &&
         L >= 1;
}

inline size_t attn_tc_image_bytes(int64_t BT, int H, int dh) {
  return (size_t)BT * (size_t)((int64_t)H * dh / at::kGrp) * at::kImgBytes;
}

template <int DH, bool kBits = false>
int launch_attention_tc_inst(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const CUtensorMap& mt, AttnKvArgs ka, AttnOutArgs oa, cudaStream_t st) {
  auto k1 = attn_kv_tc_kernel<DH, kBits>;
  auto k2 = attn_out_tc_kernel<DH, kBits>;
  SPK_CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)at::kSmem1));
  SPK_CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)at::kSmem2));
  const int sms = sm_count();
  const unsigned g1 = (unsigned)min64(ka.units, sms);
  prof_before(SPK_KERNEL_ATTN_KV, st);
  SPK_CUDA_TRY(launch_dependent(k1, dim3(g1), dim3(at::kThreads), at::kSmem1, st, mk, mv, mt, ka));
  prof_after(SPK_KERNEL_ATTN_KV, st);
  const int64_t g2 = min64(oa.items, sms);
  oa.per_cta = ceil_div(oa.items, g2);
  const unsigned grid2 = (unsigned)ceil_div(oa.items, oa.per_cta);
  prof_before(SPK_KERNEL_ATTN_OUT, st);
  SPK_CUDA_TRY(launch_dependent(k2, dim3(grid2), dim3(at::kThreads), at::kSmem2, st, mq, oa));
  prof_after(SPK_KERNEL_ATTN_OUT, st);
  return SPK_OK;
}

// tab: [L, d] decay table (written here), img: per-unit kv images.  bits:
// q, k, v are packed uint32 words [BT*L][d/32] instead of fp32.
inline int launch_attention_tc(const void* q, const void* k, const void* v, const float* lam, int64_t BT, int L,
                               int H, int dh, float eps, float* out, float* tab, unsigned char* img,
                               cudaStream_t st, bool bits = false) {
  const int d = H * dh;
  const int64_t R = BT * (int64_t)L;
  CUtensorMap mq, mk, mv, mt;
  int rc;
  if (bits) {
    const int W = d / 32;
    rc = make_map_2d_u32(&mq, static_cast<const uint32_t*>(q), R, W, W, at::kBitWords, at::kRows2, "q bits");
    if (!rc) rc = make_map_2d_u32(&mk, static_cast<const uint32_t*>(k), R, W, W, at::kBitWords, at::kP1, "k bits");
    if (!rc) rc = make_map_2d_u32(&mv, static_cast<const uint32_t*>(v), R, W, W, at::kBitWords, at::kP1, "v bits");
  } else {
    rc = make_map_2d_f32(&mq, static_cast<const float*>(q), R, d, d, at::kBoxCols, at::kBoxRows, "q");
    if (!rc) rc = make_map_2d_f32(&mk, static_cast<const float*>(k), R, d, d, at::kBoxCols, at::kBoxRows, "k");
    if (!rc) rc = make_map_2d_f32(&mv, static_cast<const float*>(v), R, d, d, at::kBoxCols, at::kBoxRows, "v");
  }
  if (!rc) rc = make_map_2d_f32(&mt, tab, L, d, d, at::kBoxCols, at::kBoxRows, "decay table");
  if (rc) return rc;
  decay_table_kernel<<<grid_for((int64_t)L * d, 256), 256, 0, st>>>(lam, L, d, tab);
  SPK_LAUNCH_CHECK();
  AttnKvArgs ka{};
  ka.groups = d / at::kGrp;
  ka.units = BT * ka.groups;
  ka.L = L;
  ka.nch = (int)ceil_div(L, at::kP1);
  ka.img = img;
  AttnOutArgs oa{};
  oa.groups = ka.groups;
  oa.L = L;
  oa.tiles = (int)ceil_div(L, at::kRows2);
  oa.items = ka.units * oa.tiles;
  oa.d = d;
  oa.eps = eps;
  oa.img = img;
  oa.out = out;
  if (bits) {
    switch (dh) {
      case 16: rc = launch_attention_tc_inst<16, true>(mq, mk, mv, mt, ka, oa, st); break;
      case 32: rc = launch_attention_tc_inst<32, true>(mq, mk, mv, mt, ka, oa, st); break;
      default: rc = launch_attention_tc_inst<64, true>(mq, mk, mv, mt, ka, oa, st); break;
    }
  } else {
    switch (dh) {
      case 16: rc = launch_attention_tc_inst<16>(mq, mk, mv, mt, ka, oa, st); break;
      case 32: rc = launch_attention_tc_inst<32>(mq, mk, mv, mt, ka, oa, st); break;
      default: rc = launch_attention_tc_inst<64>(mq, mk, mv, mt, ka, oa, st); break;
    }
  }
  if (rc) return rc;
  count_launch(3);
  return SPK_OK;
}

}  // namespace spk

extern "C" size_t spk_attention_workspace_bytes(int64_t BT, int L, int H, int dh) {
  if (BT < 1 || L < 1 || H < 1 || dh < 1) return 0;
  return spk::attn_layout(BT, L, H, dh).total;
}

extern "C" int spk_spiking_attention(const float* q, const float* k, const float* v, const float* lam, int64_t BT,
                                     int L, int H, int dh, float eps, float* out, void* workspace,
                                     size_t workspace_bytes, spk_stream_t stream) {
  SPK_REQUIRE(q && k && v && lam && out, "q, k, v, lam and out must be non-null");
  SPK_REQUIRE(BT >= 1 && L >= 1 && H >= 1, "invalid shape");
  SPK_REQUIRE(dh == 16 || dh == 32 || dh == 64, "head width %d not supported (16, 32 or 64)", dh);
  const spk::AttnLayout A = spk::attn_layout(BT, L, H, dh);
  if (workspace == nullptr || workspace_bytes < A.total)
    return spk::fail(SPK_EWORKSPACE, "workspace of %zu bytes required", A.total);
  const uintptr_t align_bits = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                               reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  SPK_REQUIRE((align_bits & 15) == 0, "q, k, v and out must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  float* tab = reinterpret_cast<float*>(static_cast<char*>(workspace) + A.tab);
  char* work = static_cast<char*>(workspace) + A.kv;
  if (spk::attn_tc_supported(BT, L, H, dh, q, k, v, out))
    return spk::launch_attention_tc(q, k, v, lam, BT, L, H, dh, eps, out, tab,
                                    reinterpret_cast<unsigned char*>(work), st);
  // heads that do not tile into 128-channel groups: SIMT passes
  SPK_REQUIRE(BT <= 65535, "BT=%lld exceeds the grid limit of 65535", (long long)BT);
  float* kv = reinterpret_cast<float*>(work);
  const int d = H * dh;
  spk::decay_table_kernel<<<spk::grid_for((int64_t)L * d, 256), 256, 0, st>>>(lam, L, d, tab);
  SPK_LAUNCH_CHECK();
  dim3 g1((unsigned)H, (unsigned)BT);
  dim3 g2((unsigned)spk::ceil_div(L, 64), (unsigned)H, (unsigned)BT);
  spk::prof_before(SPK_KERNEL_ATTN_KV, st);
  switch (dh) {
    case 16: spk::attn_kv_kernel<16><<<g1, 32, 0, st>>>(k, v, tab, L, H, kv); break;
    case 32: spk::attn_kv_kernel<32><<<g1, 64, 0, st>>>(k, v, tab, L, H, kv); break;
    default: spk::attn_kv_kernel<64><<<g1, 256, 0, st>>>(k, v, tab, L, H, kv); break;
  }
  spk::prof_after(SPK_KERNEL_ATTN_KV, st);
  SPK_LAUNCH_CHECK();
  spk::prof_before(SPK_KERNEL_ATTN_OUT, st);
  switch (dh) {
    case 16: spk::attn_out_kernel<16><<<g2, 256, 0, st>>>(q, kv, L, H, eps, out); break;
    case 32: spk::attn_out_kernel<32><<<g2, 256, 0, st>>>(q, kv, L, H, eps, out); break;
    default: spk::attn_out_kernel<64><<<g2, 256, 0, st>>>(q, kv, L, H, eps, out); break;
  }
  spk::prof_after(SPK_KERNEL_ATTN_OUT, st);
  SPK_LAUNCH_CHECK();
  spk::count_launch(3);
  return SPK_OK;
}

// The same attention over packed q, k, v spikes (uint32 words [BT*L][d/32],
// bit b of word w = channel 32w + b), as the model's projections write them:
// 32x fewer input bytes, results bit-identical to spk_spiking_attention on the
// unpacked spikes.  Tensor-core path only: d % 128 == 0, dh in {16, 32, 64}.
extern "C" int spk_spiking_attention_bits(const uint32_t* q_bits, const uint32_t* k_bits, const uint32_t* v_bits,
                                          const float* lam, int64_t BT, int L, int H, int dh, float eps, float* out,
                                          void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  SPK_REQUIRE(q_bits && k_bits && v_bits && lam && out, "q_bits, k_bits, v_bits, lam and out must be non-null");
  SPK_REQUIRE(BT >= 1 && L >= 1 && H >= 1, "invalid shape");
  SPK_REQUIRE(dh == 16 || dh == 32 || dh == 64, "head width %d not supported (16, 32 or 64)", dh);
  SPK_REQUIRE(((int64_t)H * dh) % spk::at::kGrp == 0, "packed attention needs d %% 128 == 0 (d=%d)", H * dh);
  SPK_REQUIRE(BT * (int64_t)L < (1ll << 31), "BT*L must stay below 2^31 rows");
  const uintptr_t al = reinterpret_cast<uintptr_t>(q_bits) | reinterpret_cast<uintptr_t>(k_bits) |
                       reinterpret_cast<uintptr_t>(v_bits) | reinterpret_cast<uintptr_t>(out);
  SPK_REQUIRE((al & 15) == 0, "q_bits, k_bits, v_bits and out must be 16-byte aligned");
  const spk::AttnLayout A = spk::attn_layout(BT, L, H, dh);
  if (workspace == nullptr || workspace_bytes < A.total)
    return spk::fail(SPK_EWORKSPACE, "workspace of %zu bytes required", A.total);
  float* tab = reinterpret_cast<float*>(static_cast<char*>(workspace) + A.tab);
  unsigned char* img = reinterpret_cast<unsigned char*>(static_cast<char*>(workspace) + A.kv);
  return spk::launch_attention_tc(q_bits, k_bits, v_bits, lam, BT, L, H, dh, eps, out, tab, img,
                                  (cudaStream_t)stream, true);
}
