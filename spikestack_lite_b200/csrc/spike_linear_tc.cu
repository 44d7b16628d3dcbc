// Dense branch of spike-linear on the 5th-generation tensor cores.
//
// Y[r, n] = sum_k relu'(S[r, k]) * W[k, n] where relu'(x) = x if x > 0 else 0
// (the reference engine's predicate, sparse_linear.cu:268), computed as a
// K-major bf16 x bf16 -> fp32 tcgen05 contraction with the accumulator in
// TMEM.  Spikes are exact in bf16; an fp32 operand is split into hi + lo bf16
// halves so that the products keep ~2^-17 relative accuracy:
//   W (fp32)  ->  W_hi + W_lo       (two MMAs per k-step)
//   S (fp32)  ->  S_hi [+ S_lo]     (S_lo only for a k-chunk that holds a value
//                                    not exact in bf16; spikes never need it)
//
// CTA = one 128-row x NT-column output tile, 10 warps:
//   warps 0-3  producers: load S (fp32, 16 B per lane, coalesced), apply the
//              predicate, convert to bf16 and store into the 128-byte-swizzled
//              K-major A stage; per-warp flags tell the MMA issuer whether
//              the stage needs the lo half;
//   warp 8     allocates TMEM and streams the pre-split W image into the B
//              stage with 1-D bulk copies (no multicast);
//   warp 9     one thread issues tcgen05.mma and commits stage releases;
//   warps 4-7  epilogue: tcgen05.ld of their 32-lane TMEM quarter, + bias,
//              vectorised stores of Y.
// All waits are bounded (2 s); a timeout raises SPK_DEV_PIPE_TIMEOUT, every
// role drains what it issued, TMEM is freed and the kernel returns.
#include "spk_common.cuh"

namespace spk {

namespace tc {

constexpr int kRows = 128;          // MMA M
constexpr int kKChunk = 64;         // bf16 elements per 128-byte swizzle row
constexpr int kABytes = kRows * 128;  // one A stage half (hi or lo): 16 KB
constexpr int kThreads = 320;

template <int NT, bool WSPLIT>
struct Cfg {
  static constexpr int kBHalf = NT * 128;
  static constexpr int kBBytes = kBHalf * (WSPLIT ? 2 : 1);
  static constexpr int kStageBytes = 2 * kABytes + kBBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes >= 4 ? 4 : ((200 * 1024) / kStageBytes);
  static constexpr int kTmemCols = NT <= 32 ? 32 : (NT <= 64 ? 64 : (NT <= 128 ? 128 : 256));
  static constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(kStages >= 2, "stage ring too small");
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 256, "NT must be a multiple of 16 in [16, 256]");
};

}  // namespace tc

struct TcArgs {
  const float* S;
  int64_t R;       // rows (T*M)
  int K, N;
  int nk;          // k-chunks of 64
  const unsigned char* wimg;  // pre-split W image
  const float* bias;
  float* Y;
  int y_vec;       // Y is 16-byte aligned and N % 4 == 0: float4 stores
};

template <int NT, bool WSPLIT>
__global__ void __launch_bounds__(tc::kThreads, 1) spike_linear_tc_kernel(TcArgs a) {
  using C = tc::Cfg<NT, WSPLIT>;
  constexpr int ST = C::kStages;
  extern __shared__ __align__(1024) unsigned char smem_dyn[];
  // 1024-byte align the operand ring (required by the 128-byte swizzle)
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  unsigned char* a_hi = base;                          // [ST][16 KB]
  unsigned char* a_lo = base + ST * tc::kABytes;       // [ST][16 KB]
  unsigned char* bstg = base + 2 * ST * tc::kABytes;   // [ST][kBBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bstg + (size_t)ST * C::kBBytes);
  uint64_t* a_full = bars;            // [ST] 4 producer-warp arrivals
  uint64_t* b_full = bars + ST;       // [ST] 1 arrival + tx bytes
  uint64_t* empty = bars + 2 * ST;    // [ST] tcgen05.commit
  uint64_t* acc_full = bars + 3 * ST; // [1]
  uint64_t* drain = bars + 3 * ST + 1;
  int* lo_flag = reinterpret_cast<int*>(bars + 3 * ST + 2);  // [ST][4 producer warps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lo_flag + 4 * ST);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)blockIdx.x * tc::kRows;
  const int n_tile = blockIdx.y;
  const int n0 = n_tile * NT;
  const int nk = a.nk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
      for (int w = 0; w < 4; ++w) lo_flag[4 * s + w] = 0;
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // ------------------------------------------------------------ producers
    // Each warp owns rows [32w, 32w+32) of the tile.  Its share of the lo
    // stage is written only when it holds a value that is not exact in bf16;
    // otherwise it is zero-filled once per ring slot ("dirty" tracks slots
    // that may still hold nonzero lo data) so that a stage whose other warps
    // need the lo MMA still sees zeros here.
    const int half = lane >> 4;            // which of the 2 rows this lane loads
    const int kq = (lane & 15) * 4;        // first of the 4 columns within the chunk
    uint32_t dirty = (1u << ST) - 1u;      // ring slots whose lo share is not known to be zero
    for (int kc = 0; kc < nk; ++kc) {
      const int s = kc % ST, u = kc / ST;
      if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
      const int k = kc * tc::kKChunk + kq;
      float4 v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rl = warp * 32 + 2 * i + half;
        const int64_t row = r0 + rl;
        if (row < a.R && k < a.K) {
          v[i] = __ldg(reinterpret_cast<const float4*>(a.S + row * a.K + k));
        } else {
          v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      bool any_lo = false;
      uint2 lo_pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int rl = warp * 32 + 2 * i + half;
        float x[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        __nv_bfloat16 h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float xr = x[j] > 0.0f ? x[j] : 0.0f;
          split_bf16(xr, h[j], l[j]);
          any_lo |= (__bfloat16_as_ushort(l[j]) & 0x7fffu) != 0;
        }
        const uint32_t off = sw128_offset_bf16((uint32_t)rl, (uint32_t)kq);
        *reinterpret_cast<uint2*>(a_hi + s * tc::kABytes + off) =
            make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
        lo_pk[i] = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
      }
      const bool warp_lo = __any_sync(0xffffffffu, any_lo);
      if (warp_lo || ((dirty >> s) & 1u)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int rl = warp * 32 + 2 * i + half;
          const uint32_t off = sw128_offset_bf16((uint32_t)rl, (uint32_t)kq);
          *reinterpret_cast<uint2*>(a_lo + s * tc::kABytes + off) = warp_lo ? lo_pk[i] : make_uint2(0u, 0u);
        }
        dirty = warp_lo ? (dirty | (1u << s)) : (dirty & ~(1u << s));
      }
      if (lane == 0) lo_flag[s * 4 + warp] = warp_lo ? 1 : 0;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ B loader
    if (lane == 0) {
      int issued = 0;
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % ST, u = kc / ST;
        if (u > 0 && !mbar_wait(&empty[s], (u - 1) & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT)) break;
        mbar_arrive_expect_tx(&b_full[s], C::kBBytes);
        bulk_g2s(bstg + (size_t)s * C::kBBytes, a.wimg + ((size_t)n_tile * nk + kc) * C::kBBytes, C::kBBytes,
                 &b_full[s]);
        issued = kc + 1;
      }
      // drain: every issued copy must land before shared memory is released
      for (int kc = (issued > ST ? issued - ST : 0); kc < issued; ++kc) {
        mbar_wait(&b_full[kc % ST], (kc / ST) & 1, nullptr, SPK_DEV_PIPE_TIMEOUT);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(tc::kRows, NT);
      bool ok = true;
      for (int kc = 0; kc < nk && ok; ++kc) {
        const int s = kc % ST, u = kc / ST;
        ok = mbar_wait(&a_full[s], u & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT) &&
             mbar_wait(&b_full[s], u & 1, abort_flag, SPK_DEV_PIPE_TIMEOUT);
        if (!ok) break;
        tc_fence_after();
        const uint64_t da_hi = umma_desc_sw128_kmajor(smem_u32(a_hi + s * tc::kABytes));
        const uint64_t da_lo = umma_desc_sw128_kmajor(smem_u32(a_lo + s * tc::kABytes));
        const uint64_t db_hi = umma_desc_sw128_kmajor(smem_u32(bstg + (size_t)s * C::kBBytes));
        const uint64_t db_lo = umma_desc_sw128_kmajor(smem_u32(bstg + (size_t)s * C::kBBytes + C::kBHalf));
        const bool lo = (lo_flag[4 * s] | lo_flag[4 * s + 1] | lo_flag[4 * s + 2] | lo_flag[4 * s + 3]) != 0;
#pragma unroll
        for (int j = 0; j < tc::kKChunk / 16; ++j) {
          const uint64_t adv = (uint64_t)(2 * j);  // 32 bytes per 16-element k-step
          umma_f16_ss(tmem, da_hi + adv, db_hi + adv, idesc, (kc > 0 || j > 0) ? 1u : 0u);
          if (WSPLIT) umma_f16_ss(tmem, da_hi + adv, db_lo + adv, idesc, 1u);
          if (lo) umma_f16_ss(tmem, da_lo + adv, db_hi + adv, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(ok ? acc_full : drain);
      if (!ok) mbar_wait(drain, 0, nullptr, SPK_DEV_PIPE_TIMEOUT);  // issued MMAs finish before exit
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 4-7)
    const int q = warp & 3;
    const bool ok = mbar_wait(acc_full, 0, abort_flag, SPK_DEV_PIPE_TIMEOUT);
    tc_fence_after();
    if (ok) {
      const int64_t row = r0 + q * 32 + lane;
      const bool vec_ok = a.y_vec != 0;
#pragma unroll 1
      for (int c = 0; c < NT / 16; ++c) {
        float acc[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 16), acc);
        tmem_wait_ld();
        const int n = n0 + c * 16;
        if (row < a.R) {
          float* y = a.Y + row * a.N + n;
          if (vec_ok && n + 16 <= a.N) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float4 o = make_float4(acc[4 * g], acc[4 * g + 1], acc[4 * g + 2], acc[4 * g + 3]);
              if (a.bias) {
                o.x += a.bias[n + 4 * g];
                o.y += a.bias[n + 4 * g + 1];
                o.z += a.bias[n + 4 * g + 2];
                o.w += a.bias[n + 4 * g + 3];
              }
              *reinterpret_cast<float4*>(y + 4 * g) = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (n + j < a.N) y[j] = a.bias ? acc[j] + a.bias[n + j] : acc[j];
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Pre-split weight image: for n-tile t and k-chunk c, an [NT x 64] bf16 hi
// block followed (fp32 W) by the lo block, each in the 128-byte-swizzled
// K-major layout the B operand uses, so one bulk copy moves a whole stage.
template <typename WT, bool WSPLIT>
__global__ void w_image_kernel(const WT* W, int64_t sk, int64_t sn, int K, int N, int NT, int nk,
                               unsigned char* img) {
  const int64_t total = (int64_t)((N + NT - 1) / NT) * NT * nk * 8;  // one thread per (n, 8 k)
  const size_t half = (size_t)NT * 128;
  const size_t stage = half * (WSPLIT ? 2 : 1);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int k8 = (int)(i % 8);
    const int64_t rest = i / 8;
    const int kc = (int)(rest % nk);
    const int64_t ng = rest / nk;  // global n index (padded)
    const int t = (int)(ng / NT), nl = (int)(ng % NT);
    __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = kc * 64 + k8 * 8 + j;
      float x = 0.0f;
      if (k < K && ng < N) x = static_cast<float>(W[(int64_t)k * sk + ng * sn]);
      if (WSPLIT) {
        split_bf16(x, h[j], l[j]);
      } else {
        h[j] = __float2bfloat16_rn(x);
      }
    }
    unsigned char* blk = img + ((size_t)t * nk + kc) * stage;
    const uint32_t off = sw128_offset_bf16((uint32_t)nl, (uint32_t)(k8 * 8));
    *reinterpret_cast<uint4*>(blk + off) =
        make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]), pack_bf16x2(h[6], h[7]));
    if (WSPLIT) {
      *reinterpret_cast<uint4*>(blk + half + off) =
          make_uint4(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]), pack_bf16x2(l[6], l[7]));
    }
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

template <int NT, bool WSPLIT>
int launch_tc_inst(const TcArgs& a, int n_tiles, cudaStream_t stream) {
  using C = tc::Cfg<NT, WSPLIT>;
  auto kern = spike_linear_tc_kernel<NT, WSPLIT>;
  SPK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes));
  dim3 grid((unsigned)ceil_div(a.R, tc::kRows), (unsigned)n_tiles);
  SPK_REQUIRE(grid.x <= 2147483647u, "too many rows");
  prof_before(SPK_KERNEL_DENSE, stream);
  kern<<<grid, tc::kThreads, C::kSmemBytes, stream>>>(a);
  prof_after(SPK_KERNEL_DENSE, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_w_image(const void* W, int w_dtype, int64_t sk, int64_t sn, int K, int N, const TcPlan& p,
                   unsigned char* img, cudaStream_t stream) {
  const int64_t total = (int64_t)p.n_tiles * p.NT * p.nk * 8;
  const int threads = 256;
  const int blocks = (int)min64(ceil_div(total, threads), 4096);
  if (w_dtype == SPK_BF16) {
    w_image_kernel<__nv_bfloat16, false><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(W), sk, sn, K, N, p.NT, p.nk, img);
  } else {
    w_image_kernel<float, true><<<blocks, threads, 0, stream>>>(static_cast<const float*>(W), sk, sn, K, N, p.NT,
                                                               p.nk, img);
  }
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

int launch_tc(const float* S, int64_t R, int K, int N, const TcPlan& p, const unsigned char* img,
              const float* bias, float* Y, cudaStream_t stream) {
  const int y_vec = ((N & 3) == 0 && (reinterpret_cast<uintptr_t>(Y) & 15) == 0) ? 1 : 0;
  TcArgs a{S, R, K, N, p.nk, img, bias, Y, y_vec};
  if (p.split) {
    switch (p.NT) {
      case 16: return launch_tc_inst<16, true>(a, p.n_tiles, stream);
      case 32: return launch_tc_inst<32, true>(a, p.n_tiles, stream);
      case 48: return launch_tc_inst<48, true>(a, p.n_tiles, stream);
      case 64: return launch_tc_inst<64, true>(a, p.n_tiles, stream);
      case 128: return launch_tc_inst<128, true>(a, p.n_tiles, stream);
      default: break;
    }
  } else {
    switch (p.NT) {
      case 16: return launch_tc_inst<16, false>(a, p.n_tiles, stream);
      case 32: return launch_tc_inst<32, false>(a, p.n_tiles, stream);
      case 48: return launch_tc_inst<48, false>(a, p.n_tiles, stream);
      case 64: return launch_tc_inst<64, false>(a, p.n_tiles, stream);
      case 128: return launch_tc_inst<128, false>(a, p.n_tiles, stream);
      case 256: return launch_tc_inst<256, false>(a, p.n_tiles, stream);
      default: break;
    }
  }
  return fail(SPK_EUNSUPPORTED, "no dense-branch tile for N=%d", N);
}

}  // namespace spk
