// Spike -> CSR compaction for T planes in one launch (single pass over S).
//
// Replaces the reference engine's csr_build_kernel + scan_blocks_kernel +
// offscan_add_kernel + csr_compact_kernel (sparse_linear.cu:251-369).  Same
// predicate (S > 0, so negatives and NaN are dropped), same ascending column
// order, same int32 row_offsets per plane; unlike the reference it is correct
// for any number of rows (its block-offset scan stops at 65536 rows) and it
// reads S exactly once:
//
//   phase A  each warp ballots its rows 32 columns at a time into a bitmap
//            held in shared memory and counts the nonzeros per row;
//   phase B  the tile total is published and the tile's exclusive prefix is
//            found by a decoupled look-back over earlier tiles (tile ids are
//            handed out in launch order by an atomic counter, so every tile a
//            CTA waits on is already resident; every wait is bounded);
//   phase C  row_ptr / nnz_row are written and the bitmap is expanded into
//            column indices with coalesced stores (one 32-column word per
//            warp step), values gathered from S.
//
// Tiles never straddle planes; the first tile of plane t publishes the plane
// base so that row_ptr is relative to the plane (as in the reference) while
// col_idx holds the planes back to back.
//
// After the dense spike-linear kernel, which already packed the spike masks
// and counted the spikes per row, 128-row block and 16384-row super-block,
// csr_from_masks_kernel builds the same CSR without touching S: every prefix
// is a sum of finished counts (no look-back) and each lane expands one row.
#include "spk_common.cuh"

namespace spk {

struct ScanState {
  unsigned int tile_counter;
  int nonunit;  // set by the dense kernel when it saw a positive value other than 1
  unsigned int pad[62];
  // followed by: uint64_t tile_desc[num_tiles]; uint64_t plane_desc[T]; uint8_t tile_flags[num_tiles]
};

constexpr uint64_t kDescAgg = 1ull << 62;
constexpr uint64_t kDescIncl = 2ull << 62;
constexpr uint64_t kDescValueMask = (1ull << 62) - 1;

struct CsrLayout {
  int T;
  int64_t M;
  int K, KW;
  int rows_per_tile;
  int64_t tiles_per_plane, num_tiles;
  size_t desc_off, plane_desc_off, flags_off, total;
};

inline CsrLayout csr_layout(int T, int64_t M, int K) {
  CsrLayout L{};
  L.T = T;
  L.M = M;
  L.K = K;
  L.KW = (K + 31) / 32;
  int rt = 16384 / (L.KW > 0 ? L.KW : 1);
  rt = rt > 128 ? 128 : rt;
  rt = rt < 8 ? 8 : rt;
  L.rows_per_tile = rt & ~7;
  L.tiles_per_plane = ceil_div(M, L.rows_per_tile);
  L.num_tiles = L.tiles_per_plane * T;
  L.desc_off = sizeof(ScanState);
  L.plane_desc_off = L.desc_off + sizeof(uint64_t) * L.num_tiles;
  L.flags_off = L.plane_desc_off + sizeof(uint64_t) * T;
  L.total = align_up(L.flags_off + L.num_tiles, 256);
  return L;
}

struct CsrArgs {
  const float* S;          // [T*M, K]
  int T;
  int64_t M;
  int K, KW, rows_per_tile;
  int64_t tiles_per_plane, num_tiles;
  int32_t* nnz_row;        // [T*M] or null
  int32_t* row_ptr;        // [T*(M+1)]
  int32_t* col_idx;        // capacity col_capacity
  float* values;           // capacity col_capacity or null
  int64_t* plane_ptr;      // [T+1]
  int64_t col_capacity;
  ScanState* state;
  uint64_t* tile_desc;
  uint64_t* plane_desc;
  uint8_t* tile_flags;     // [num_tiles]: 1 if the tile holds a positive value != 1
  const uint32_t* bitmap;  // bitmap source: [T*M][KWP] planar spike masks written by the dense kernel
  const int32_t* row_cnt;  // bitmap source: [T*M] spikes per row
  int KWP;                 // planar words per row (2 per 64-column chunk)
  int vec4;                // S rows 16-byte aligned (K % 4 == 0, aligned base): phase A reads float4
  const int32_t* blk_sum;                // bitmap source: spikes per 128-row block of the T*M rows
  const unsigned long long* sup_sum;     // bitmap source: spikes per 16384-row super-block
  const int* gate;         // automatic branch choice: run only when *gate == gate_value (null: always)
  int gate_value;
  int* decide;             // scan under the automatic choice: the last tile writes SPK_BRANCH_CSR when the
  int64_t decide_limit;    // total number of spikes is <= decide_limit, else SPK_BRANCH_DENSE (null: none)
};

// 8 bits -> bits 0, 4, 8, ..., 28
__device__ __forceinline__ uint32_t spread8_stride4(uint32_t x) {
  x = (x | (x << 12)) & 0x000f000fu;
  x = (x | (x << 6)) & 0x03030303u;
  x = (x | (x << 3)) & 0x11111111u;
  return x;
}

__device__ __forceinline__ uint64_t spin_desc(const uint64_t* p, bool& ok) {
  uint64_t d = ld_relaxed_u64(p);
  if ((d >> 62) != 0) return d;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(64);  // back off: polling costs issue slots of the working warps
    d = ld_relaxed_u64(p);
    if ((d >> 62) != 0) return d;
    if ((it & 31u) == 0 && global_ns() - t0 > kSpinLimitNs) {
      report_device_error(SPK_DEV_SCAN_TIMEOUT);
      ok = false;
      return kDescIncl;  // value 0
    }
  }
}

__global__ void __launch_bounds__(256) csr_scan_kernel(CsrArgs a) {
  if (gated_off(a.gate, a.gate_value)) return;  // before the tile counter: every block leaves
  extern __shared__ __align__(16) uint32_t smem_u32buf[];
  const int RT = a.rows_per_tile;
  uint32_t* bm = smem_u32buf;                    // [RT][KW]
  int32_t* cnt = reinterpret_cast<int32_t*>(bm + (size_t)RT * a.KW);  // [RT]
  int32_t* pre = cnt + RT;                       // [RT] exclusive prefix inside the tile
  __shared__ int64_t s_excl, s_base;
  __shared__ unsigned int s_tile;
  __shared__ int s_nonunit;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    s_tile = atomicAdd(&a.state->tile_counter, 1u);
    s_nonunit = 0;
  }
  __syncthreads();
  const int64_t tile = s_tile;
  const bool valid_tile = tile < a.num_tiles;
  const int plane = valid_tile ? (int)(tile / a.tiles_per_plane) : 0;
  const int64_t tip = valid_tile ? tile % a.tiles_per_plane : 0;
  const int64_t row0 = tip * RT;  // row within plane
  const int rows = valid_tile ? (int)min64(RT, a.M - row0) : 0;
  const float* Sp = a.S + ((int64_t)plane * a.M + row0) * a.K;

  // ---- phase A: ballot rows into the shared bitmap
  bool nonunit = false;
  if (a.vec4) {
    // 16-byte loads: lane l holds columns 4l .. 4l+3 of a 128-column block, so
    // ballot e has bit l = column 4l + e; lane i < 4 interleaves byte i of the
    // four ballots into the block's column-order word i (bit b = column 32i + b)
    const int sh = (lane & 3) * 8;
    for (int r = warp; r < RT; r += 8) {
      int c = 0;
      if (r < rows) {
        const float4* row = reinterpret_cast<const float4*>(Sp + (int64_t)r * a.K);
        const int nb = (a.K + 127) / 128;
        for (int b0 = 0; b0 < nb; b0 += 4) {
          float4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int col = (b0 + u) * 128 + 4 * lane;
            v[u] = (b0 + u < nb && col < a.K) ? __ldg(row + (b0 + u) * 32 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float4 x = v[u];
            nonunit |= (x.x > 0.0f && x.x != 1.0f) || (x.y > 0.0f && x.y != 1.0f) || (x.z > 0.0f && x.z != 1.0f) ||
                       (x.w > 0.0f && x.w != 1.0f);
            const uint32_t m0 = __ballot_sync(0xffffffffu, x.x > 0.0f);
            const uint32_t m1 = __ballot_sync(0xffffffffu, x.y > 0.0f);
            const uint32_t m2 = __ballot_sync(0xffffffffu, x.z > 0.0f);
            const uint32_t m3 = __ballot_sync(0xffffffffu, x.w > 0.0f);
            c += __popc(m0) + __popc(m1) + __popc(m2) + __popc(m3);
            const uint32_t word = spread8_stride4((m0 >> sh) & 0xffu) | (spread8_stride4((m1 >> sh) & 0xffu) << 1) |
                                  (spread8_stride4((m2 >> sh) & 0xffu) << 2) |
                                  (spread8_stride4((m3 >> sh) & 0xffu) << 3);
            const int w = (b0 + u) * 4 + (lane & 3);
            if (lane < 4 && b0 + u < nb && w < a.KW) bm[r * a.KW + w] = word;
          }
        }
      }
      if (lane == 0) cnt[r] = c;
    }
  } else
  for (int r = warp; r < RT; r += 8) {
    int c = 0;
    if (r < rows) {
      const float* row = Sp + (int64_t)r * a.K;
      for (int w0 = 0; w0 < a.KW; w0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = (w0 + j) * 32 + lane;
          v[j] = (w0 + j < a.KW && col < a.K) ? __ldg(row + col) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool nz = v[j] > 0.0f;
          nonunit |= nz && (v[j] != 1.0f);
          const uint32_t bits = __ballot_sync(0xffffffffu, nz);
          if (w0 + j < a.KW) {
            if (lane == 0) bm[r * a.KW + w0 + j] = bits;
            c += __popc(bits);
          }
        }
      }
    }
    if (lane == 0) cnt[r] = c;
  }
  if (__any_sync(0xffffffffu, nonunit) && lane == 0) s_nonunit = 1;
  __syncthreads();

  // ---- phase B: in-tile exclusive prefix (warp 0), then the look-back (thread 0)
  if (warp == 0) {
    int64_t running = 0;
    for (int base = 0; base < RT; base += 32) {
      const int r = base + lane;
      const int v = (r < RT) ? cnt[r] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (r < RT) pre[r] = (int)running + incl - v;
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    const int64_t agg = running;
    bool ok = true;
    int64_t excl = 0;
    if (valid_tile && tile > 0) {
      // warp-wide look-back: lane l probes tile j - l, 32 predecessors per
      // round; the nearest inclusive prefix ends the walk.
      if (lane == 0) st_relaxed_u64(&a.tile_desc[tile], kDescAgg | (uint64_t)agg);
      __syncwarp();
      for (int64_t j = tile - 1;; j -= 32) {
        const int64_t idx = j - lane;
        const uint64_t d = (idx >= 0) ? spin_desc(&a.tile_desc[idx], ok) : kDescIncl;  // before tile 0: prefix 0
        const uint32_t incl = __ballot_sync(0xffffffffu, (d >> 62) == 2);
        const int last = incl ? __ffs(incl) - 1 : 31;  // lanes 0..last contribute
        int64_t v = (lane <= last) ? (int64_t)(d & kDescValueMask) : 0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        excl += v;
        if (incl) break;
      }
      ok = __all_sync(0xffffffffu, ok);
    }
    if (lane == 0 && valid_tile) {
      int64_t base;
      st_relaxed_u64(&a.tile_desc[tile], kDescIncl | (uint64_t)(excl + agg));
      if (tip == 0) {
        base = excl;
        st_relaxed_u64(&a.plane_desc[plane], kDescIncl | (uint64_t)base);
        a.plane_ptr[plane] = base;
        a.row_ptr[(int64_t)plane * (a.M + 1)] = 0;
      } else {
        const uint64_t d = spin_desc(&a.plane_desc[plane], ok);
        base = (int64_t)(d & kDescValueMask);
      }
      if (plane == a.T - 1 && tip == a.tiles_per_plane - 1) {
        a.plane_ptr[a.T] = excl + agg;
        if (a.decide) *a.decide = (excl + agg <= a.decide_limit) ? SPK_BRANCH_CSR : SPK_BRANCH_DENSE;
      }
      a.tile_flags[tile] = s_nonunit ? 1 : 0;
      s_excl = excl;
      s_base = base;
    }
  }
  __syncthreads();

  // ---- phase C: row pointers and column indices
  if (valid_tile) {
    const int64_t excl = s_excl, rel = s_excl - s_base;
    int32_t* rp = a.row_ptr + (int64_t)plane * (a.M + 1) + row0 + 1;
    int32_t* nr = a.nnz_row ? a.nnz_row + (int64_t)plane * a.M + row0 : nullptr;
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
      rp[r] = (int32_t)(rel + pre[r] + cnt[r]);
      if (nr) nr[r] = cnt[r];
    }
    // Expansion: a segment of LPR lanes (LPR = words per row rounded up to a
    // power of two, at most 32) takes one row; lane l of the segment takes
    // word w0 + l, a segmented scan of the word popcounts gives its output
    // offset, and the lane writes its word's columns in ascending order.
    bool overflow = false;
    int LPR = 1;
    while (LPR < a.KW && LPR < 32) LPR <<= 1;
    const int seg = lane / LPR, sl = lane % LPR, nseg = 32 / LPR;
    for (int rb = warp * nseg; rb < rows; rb += 8 * nseg) {
      const int r = rb + seg;
      const bool active = r < rows;
      int64_t pos = active ? excl + pre[r] : 0;
      const uint32_t* bw = bm + (active ? r : 0) * a.KW;
      const float* row = Sp + (int64_t)(active ? r : 0) * a.K;
      for (int w0 = 0; w0 < a.KW; w0 += LPR) {
        const int w = w0 + sl;
        uint32_t bits = (active && w < a.KW) ? bw[w] : 0u;
        const int c = __popc(bits);
        int incl = c;
        for (int o = 1; o < LPR; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o, LPR);
          if (sl >= o) incl += y;
        }
        const int64_t p0 = pos + (incl - c);
        if (p0 + c <= a.col_capacity) {  // common case: 32-bit offsets, no per-entry checks
          int32_t* dst = a.col_idx + p0;
          int k = 0;
          if (a.values == nullptr) {
            while (bits) {
              dst[k++] = w * 32 + __ffs(bits) - 1;
              bits &= bits - 1u;
            }
          } else {
            float* vdst = a.values + p0;
            while (bits) {
              const int col = w * 32 + __ffs(bits) - 1;
              bits &= bits - 1u;
              dst[k] = col;
              vdst[k++] = row[col];
            }
          }
        } else {
          int64_t p = p0;
          while (bits) {
            const int col = w * 32 + __ffs(bits) - 1;
            bits &= bits - 1u;
            if (p < a.col_capacity) {
              a.col_idx[p] = col;
              if (a.values) a.values[p] = row[col];
            } else {
              overflow = true;
            }
            ++p;
          }
        }
        pos += __shfl_sync(0xffffffffu, incl, LPR - 1, LPR);
      }
    }
    // under the automatic choice an overflow only means "above the crossover" (the dense branch runs)
    if (__any_sync(0xffffffffu, overflow) && lane == 0 && a.decide == nullptr) report_device_error(SPK_DEV_CSR_OVERFLOW);
  }

}

// Launch helper shared by every entry point that emits CSR.  With `bitmap`
// set, the scan reads the packed spikes and row counts of a preceding dense
// pass instead of S (S is then only read for values of non-unit spikes), and
// `state_zeroed` says that pass already cleared the scan state.
// Spikes before global rows r0 and r1 of the T*M rows, from the dense
// kernel's sums: whole 16384-row super-blocks, whole 128-row blocks, then
// single rows (at most R/16384 + 127 + 127 reads each), reduced over the CTA
// in one pass.  Call from every thread; `red` is [2][warps] shared scratch.
__device__ __forceinline__ void prefix_from_sums(const CsrArgs& a, int64_t r0, int64_t r1, int64_t* red,
                                                 int64_t& p0, int64_t& p1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (int)(blockDim.x >> 5);
  int64_t part[2] = {0, 0};
  const int64_t at[2] = {r0, r1};
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int64_t r = at[q];
    const int64_t s_end = r >> 14, b0 = s_end << 7, b1 = r >> 7;
    for (int64_t i = threadIdx.x; i < s_end; i += blockDim.x) part[q] += (int64_t)a.sup_sum[i];
    for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) part[q] += a.blk_sum[i];
    for (int64_t i = (b1 << 7) + threadIdx.x; i < r; i += blockDim.x) part[q] += a.row_cnt[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
    part[1] += __shfl_xor_sync(0xffffffffu, part[1], o);
  }
  if (lane == 0) {
    red[warp] = part[0];
    red[nw + warp] = part[1];
  }
  __syncthreads();
  p0 = 0;
  p1 = 0;
  for (int w = 0; w < nw; ++w) {
    p0 += red[w];
    p1 += red[nw + w];
  }
}

// CSR from the dense kernel's planar spike masks (row counts and block sums
// come with them): one row per lane, 128 rows per CTA.  For every 64-column
// chunk a lane rebuilds the two column-order words from the four 16-bit
// planes (8-bit groups spread to every 4th bit) and writes the set columns in
// ascending order to its row's segment.  No look-back and no waiting: every
// prefix is a sum of counts that are complete when the grid starts.
// Column indices of a warp's 32 rows are contiguous in col_idx: lanes expand
// into a per-warp shared buffer and the warp copies it out with coalesced
// stores (a warp whose rows hold more than kWarpBuf spikes, or whose values
// are requested, writes straight to global memory).
// Four lanes per row, each taking a quarter of the row's 64-column chunks:
// the lanes are ordered (row, quarter), so one warp-wide scan of the quarter
// counts gives every quarter its first slot, each lane's serial expansion is
// a quarter row long, and twice as many warps are in flight as with two lanes
// per row (the pass is latency-bound).
// A warp's 8 rows are contiguous in col_idx: lanes expand into a per-warp
// shared buffer, placed at the same offset modulo 16 bytes as the warp's
// segment of col_idx, and the warp copies it out with 16-byte stores (a warp
// whose rows hold more than kWarpBuf - 3 spikes, or whose values are
// requested, writes straight to global memory).
constexpr int kLanesPerRow = 4;
constexpr int kMaskRows = 64;                              // rows per CTA
constexpr int kMaskThreads = kLanesPerRow * kMaskRows;
constexpr int kMaskWarps = kMaskThreads / 32;
constexpr int kRowsPerWarp = 32 / kLanesPerRow;
constexpr int kWarpBuf = 1024;                              // column slots staged per warp
constexpr size_t kMaskSmem = sizeof(int32_t) * kMaskWarps * kWarpBuf;

// Six CTAs per SM (at most 42 registers a thread, the largest shared-memory
// carveout): 888 resident CTAs, so the 768 of the isolated config's 3 x 16384
// rows run in one wave instead of five per SM plus a tail.
constexpr int kMaskCtasPerSm = 6;
__global__ void __launch_bounds__(kMaskThreads, kMaskCtasPerSm) csr_from_masks_kernel(CsrArgs a, int64_t tiles_pp) {
  if (gated_off(a.gate, a.gate_value)) return;
  extern __shared__ __align__(16) int32_t s_buf_all[];  // [kMaskWarps][kWarpBuf]
  __shared__ int64_t s_red[2 * kMaskWarps];
  __shared__ int s_wtot[kMaskWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // programmatic dependent of the dense kernel: its outputs are complete after this
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int plane = (int)(blockIdx.x / tiles_pp);
  const int64_t row0 = (blockIdx.x % tiles_pp) * kMaskRows;  // row within the plane
  const int64_t grow0 = (int64_t)plane * a.M + row0;
  const int rl = warp * kRowsPerWarp + lane / kLanesPerRow;  // row in the CTA
  const int qr = lane % kLanesPerRow;                          // quarter of its chunks
  const int64_t r = row0 + rl;
  const bool valid = r < a.M;
  const int64_t grow = grow0 + rl;
  const int nch = a.KWP / 2, per = (nch + kLanesPerRow - 1) / kLanesPerRow;
  const int c0 = min(nch, qr * per), c1 = min(nch, c0 + per);
  const uint2* src = reinterpret_cast<const uint2*>(a.bitmap + grow * a.KWP);
  // All loads of the prologue go out together: this thread's share of the
  // CTA's two prefix sums (spikes before the CTA's first row in the whole
  // grid and before its plane: super-block, block and row counts) and the
  // row's first mask chunks.
  int64_t part[2] = {0, 0};
  {
    const int64_t at[2] = {grow0, (int64_t)plane * a.M};
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int64_t rr = at[q];
      const int64_t s_end = rr >> 14, b0 = s_end << 7, b1 = rr >> 7;
      for (int64_t i = threadIdx.x; i < s_end; i += blockDim.x) part[q] += (int64_t)a.sup_sum[i];
      for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) part[q] += a.blk_sum[i];
      for (int64_t i = (b1 << 7) + threadIdx.x; i < rr; i += blockDim.x) part[q] += a.row_cnt[i];
    }
  }
  constexpr int kPre = 4;  // mask chunks fetched ahead
  uint2 pre_w[kPre];
  int cnt = 0;            // spikes in this quarter of the row
#pragma unroll
  for (int c = 0; c < kPre; ++c) {
    pre_w[c] = (valid && c0 + c < c1) ? __ldg(src + c0 + c) : make_uint2(0u, 0u);
    cnt += __popc(pre_w[c].x) + __popc(pre_w[c].y);
  }
  for (int c = c0 + kPre; valid && c < c1; ++c) {
    const uint2 pw = __ldg(src + c);
    cnt += __popc(pw.x) + __popc(pw.y);
  }
  // warp-level: the prefix partials and the scan of the quarter counts, then
  // one CTA barrier for both
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    part[0] += __shfl_xor_sync(0xffffffffu, part[0], o);
    part[1] += __shfl_xor_sync(0xffffffffu, part[1], o);
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) {
    s_wtot[warp] = incl;
    s_red[warp] = part[0];
    s_red[kMaskWarps + warp] = part[1];
  }
  __syncthreads();
  int64_t pre_tile = 0, pre_plane = 0;
  int wbase = 0, ctot = 0;
#pragma unroll
  for (int w = 0; w < kMaskWarps; ++w) {
    pre_tile += s_red[w];
    pre_plane += s_red[kMaskWarps + w];
    wbase += (w < warp) ? s_wtot[w] : 0;
    ctot += s_wtot[w];
  }
  const int64_t pos = pre_tile + wbase + incl - cnt;
  const int64_t rel = pre_tile - pre_plane;
  int cnt_row = cnt;  // all quarters of the row
#pragma unroll
  for (int o = 1; o < kLanesPerRow; o <<= 1) cnt_row += __shfl_xor_sync(0xffffffffu, cnt_row, o);
  if (valid && qr == kLanesPerRow - 1) {
    a.row_ptr[(int64_t)plane * (a.M + 1) + r + 1] = (int32_t)(rel + wbase + incl);
    if (a.nnz_row) a.nnz_row[grow] = cnt_row;
  }
  if (threadIdx.x == 0) {
    if (row0 == 0) {
      a.row_ptr[(int64_t)plane * (a.M + 1)] = 0;
      a.plane_ptr[plane] = pre_plane;
    }
    if (plane == a.T - 1 && row0 + kMaskRows >= a.M) a.plane_ptr[a.T] = pre_tile + ctot;
  }
  const int wtot = s_wtot[warp];
  const int64_t wstart = pre_tile + wbase;
  // the warp's segment starts `sh` ints past a 16-byte boundary of col_idx
  const int sh = (int)((reinterpret_cast<uintptr_t>(a.col_idx + wstart) >> 2) & 3u);
  const bool staged = a.values == nullptr && wtot + 3 <= kWarpBuf && wstart + wtot <= a.col_capacity;
  int32_t* wbuf = s_buf_all + warp * kWarpBuf;
  // Calls emit(col) for the set columns of chunks [c0, c1) in ascending order.
  auto expand = [&](auto&& emit) {
    for (int c = c0; c < c1; ++c) {
      uint2 pw = make_uint2(0u, 0u);
      if (c - c0 < kPre) {
#pragma unroll
        for (int e = 0; e < kPre; ++e)
          if (e == c - c0) pw = pre_w[e];
      } else {
        pw = __ldg(src + c);
      }
      if ((pw.x | pw.y) == 0u) continue;
      // column 64c + 4m + e is bit m of plane e (planes: pw.x lo/hi, pw.y lo/hi)
      const uint32_t words[2] = {
          spread8_stride4(pw.x & 0xffu) | (spread8_stride4((pw.x >> 16) & 0xffu) << 1) |
              (spread8_stride4(pw.y & 0xffu) << 2) | (spread8_stride4((pw.y >> 16) & 0xffu) << 3),
          spread8_stride4((pw.x >> 8) & 0xffu) | (spread8_stride4(pw.x >> 24) << 1) |
              (spread8_stride4((pw.y >> 8) & 0xffu) << 2) | (spread8_stride4(pw.y >> 24) << 3)};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t bits = words[h];
        const int cb = 64 * c + 32 * h;
        while (bits) {
          emit(cb + __ffs(bits) - 1);
          bits &= bits - 1u;
        }
      }
    }
  };
  if (cnt > 0) {
    if (staged) {
      // shared-memory staging (a shared pointer throughout: no generic stores)
      int32_t* sdst = wbuf + sh + (incl - cnt);
      expand([&](int col) { *sdst++ = col; });
    } else {
      const bool unit_values = a.state->nonunit == 0;
      const float* row = a.S + grow * a.K;
      int64_t p = pos;
      bool overflow = false;
      expand([&](int col) {
        if (p < a.col_capacity) {
          a.col_idx[p] = col;
          if (a.values) a.values[p] = unit_values ? 1.0f : row[col];
        } else {
          overflow = true;
        }
        ++p;
      });
      if (overflow) report_device_error(SPK_DEV_CSR_OVERFLOW);
    }
  }
  if (staged) {
    __syncwarp();
    int32_t* g = a.col_idx + wstart;
    // g[i] = wbuf[sh + i]: a head of up to 3 ints, 16-byte vectors, a tail
    const int head = min(wtot, (4 - sh) & 3);
    if (lane < head) g[lane] = wbuf[sh + lane];
    const int nvec = (wtot - head) >> 2;
    const int4* s4 = reinterpret_cast<const int4*>(wbuf + sh + head);
    int4* g4 = reinterpret_cast<int4*>(g + head);
    for (int q = lane; q < nvec; q += 32) g4[q] = s4[q];
    const int done = head + 4 * nvec;
    if (lane < wtot - done) g[done + lane] = wbuf[sh + done + lane];
  }
}

// Gates of the automatic branch choice for the CSR launches (all null: none).
struct CsrGate {
  const int* gate = nullptr;
  int gate_value = 0;
  int* decide = nullptr;
  int64_t decide_limit = 0;
};

int launch_csr_scan_ex(const float* S, const uint32_t* bitmap, const int32_t* row_cnt, const int32_t* blk_sum,
                       const unsigned long long* sup_sum, bool state_zeroed, int T,
                       int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx, float* values,
                       int64_t* plane_ptr, int64_t col_capacity, void* ws, cudaStream_t stream,
                       const uint8_t** tile_flags_out, CsrLayout* layout_out, const CsrGate& gate = CsrGate()) {
  const CsrLayout L = csr_layout(T, M, K);
  CsrArgs a{};
  a.S = S;
  a.T = T;
  a.M = M;
  a.K = K;
  a.KW = L.KW;
  a.rows_per_tile = L.rows_per_tile;
  a.tiles_per_plane = L.tiles_per_plane;
  a.num_tiles = L.num_tiles;
  a.nnz_row = nnz_row;
  a.row_ptr = row_ptr;
  a.col_idx = col_idx;
  a.values = values;
  a.plane_ptr = plane_ptr;
  a.col_capacity = col_capacity;
  char* base = static_cast<char*>(ws);
  a.state = reinterpret_cast<ScanState*>(base);
  a.tile_desc = reinterpret_cast<uint64_t*>(base + L.desc_off);
  a.plane_desc = reinterpret_cast<uint64_t*>(base + L.plane_desc_off);
  a.tile_flags = reinterpret_cast<uint8_t*>(base + L.flags_off);
  a.bitmap = bitmap;
  a.row_cnt = row_cnt;
  a.KWP = 2 * (int)ceil_div(K, 64);
  a.blk_sum = blk_sum;
  a.sup_sum = sup_sum;
  a.vec4 = (S != nullptr && K % 4 == 0 && (reinterpret_cast<uintptr_t>(S) & 15) == 0) ? 1 : 0;
  a.gate = gate.gate;
  a.gate_value = gate.gate_value;
  a.decide = gate.decide;
  a.decide_limit = gate.decide_limit;
  if (bitmap) {
    // follows the dense kernel on the stream: programmatic dependent launch
    const int64_t tpp = ceil_div(M, kMaskRows);
    prof_before(SPK_KERNEL_CSR_SCAN, stream);
    SPK_CUDA_TRY(cudaFuncSetAttribute(csr_from_masks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kMaskSmem));
    SPK_CUDA_TRY(cudaFuncSetAttribute(csr_from_masks_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      (int)cudaSharedmemCarveoutMaxShared));
    SPK_CUDA_TRY(launch_dependent(csr_from_masks_kernel, dim3((unsigned)(tpp * T)), dim3(kMaskThreads), kMaskSmem,
                                  stream, a, tpp));
    prof_after(SPK_KERNEL_CSR_SCAN, stream);
    SPK_LAUNCH_CHECK();
    count_launch(1);
    if (tile_flags_out) *tile_flags_out = nullptr;
    if (layout_out) *layout_out = L;
    return SPK_OK;
  }
  const size_t smem = (size_t)L.rows_per_tile * L.KW * 4 + (size_t)L.rows_per_tile * 8;
  auto kern = csr_scan_kernel;
  if (smem > 48 * 1024) {
    SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  // The tile counter and the look-back descriptors start from zero on every
  // launch (stream-ordered), so the workspace needs no persistent state and
  // can be shared with any other use between calls.
  if (!state_zeroed) SPK_CUDA_TRY(cudaMemsetAsync(base, 0, L.flags_off, stream));
  prof_before(SPK_KERNEL_CSR_SCAN, stream);
  kern<<<(unsigned)L.num_tiles, 256, smem, stream>>>(a);
  prof_after(SPK_KERNEL_CSR_SCAN, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  if (tile_flags_out) *tile_flags_out = a.tile_flags;
  if (layout_out) *layout_out = L;
  return SPK_OK;
}

int launch_csr_scan(const float* S, int T, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr,
                    int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity, void* ws,
                    cudaStream_t stream, const uint8_t** tile_flags_out, CsrLayout* layout_out,
                    const CsrGate& gate = CsrGate()) {
  return launch_csr_scan_ex(S, nullptr, nullptr, nullptr, nullptr, false, T, M, K, nnz_row, row_ptr, col_idx, values, plane_ptr,
                            col_capacity, ws, stream, tile_flags_out, layout_out, gate);
}

int check_csr_shape(int T, int64_t M, int K) {
  SPK_REQUIRE(T >= 1 && M >= 1 && K >= 1, "invalid shape T=%d M=%lld K=%d", T, (long long)M, K);
  SPK_REQUIRE(K <= 131072, "K=%d exceeds the supported maximum of 131072 columns", K);
  SPK_REQUIRE((int64_t)M * K < (int64_t)INT32_MAX, "a plane of M*K=%lld entries overflows int32 row offsets",
              (long long)M * K);
  SPK_REQUIRE(csr_layout(T, M, K).num_tiles < (int64_t)INT32_MAX, "too many row tiles");
  return SPK_OK;
}

}  // namespace spk

extern "C" size_t spk_csr_workspace_bytes(int T, int64_t M, int K) {
  if (T < 1 || M < 1 || K < 1) return 0;
  return spk::csr_layout(T, M, K).total;
}

extern "C" int spk_csr_compact(const float* S, int T, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr,
                               int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity,
                               void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  int rc = spk::check_csr_shape(T, M, K);
  if (rc) return rc;
  SPK_REQUIRE(S && row_ptr && col_idx && plane_ptr, "S, row_ptr, col_idx and plane_ptr must be non-null");
  if (workspace == nullptr || workspace_bytes < spk::csr_layout(T, M, K).total)
    return spk::fail(SPK_EWORKSPACE, "workspace of %zu bytes required", spk::csr_layout(T, M, K).total);
  return spk::launch_csr_scan(S, T, M, K, nnz_row, row_ptr, col_idx, values, plane_ptr, col_capacity, workspace,
                              (cudaStream_t)stream, nullptr, nullptr);
}
