// Shared host/device helpers for the spikestack-lite B200 engine.
//
// Host side: status codes and the thread-local last-error string that every
// extern "C" entry point reports through (see include/spikestack_b200.h).
// Device side: thin inline-PTX wrappers for the sm_100a features the kernels
// use -- mbarriers, 1-D bulk copies (cp.async.bulk into this CTA only),
// tcgen05 (TMEM alloc / MMA / commit / ld) and the UMMA shared-memory and
// instruction descriptors.  Every spin-wait is bounded by wall-clock time and
// reports a device error code instead of hanging.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <utility>

#include "../../include/spikestack_b200.h"

namespace spk {

// ---------------------------------------------------------------- host side
int fail(int code, const char* fmt, ...);   // records the message, returns code
void clear_error();

#define SPK_REQUIRE(cond, ...)                                                   \
  do {                                                                           \
    if (!(cond)) return ::spk::fail(SPK_EINVAL, __VA_ARGS__);                    \
  } while (0)

#define SPK_CUDA_TRY(call)                                                       \
  do {                                                                           \
    cudaError_t e_ = (call);                                                     \
    if (e_ != cudaSuccess)                                                       \
      return ::spk::fail(SPK_ECUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define SPK_LAUNCH_CHECK()                                                       \
  do {                                                                           \
    cudaError_t e_ = cudaGetLastError();                                         \
    if (e_ != cudaSuccess)                                                       \
      return ::spk::fail(SPK_ECUDA, "kernel launch failed: %s (%s:%d)",          \
                         cudaGetErrorString(e_), __FILE__, __LINE__);            \
  } while (0)

inline int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Launch `kern` as a programmatic dependent of the previous kernel on `stream`:
// it may start while that kernel drains and must execute griddepcontrol.wait
// before reading the previous kernel's results.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                    Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// As launch_dependent, in clusters of (cx, 1, 1) CTAs; pdl = false launches
// it as an ordinary successor of the previous kernel.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                            cudaStream_t stream, unsigned cx, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cx;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ inline int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Device error word (per device; read and cleared by spk_device_error()).
// Defined here: the library is built as one translation unit (engine.cu).
__device__ int g_device_error = 0;
// Where the first timed-out pipeline wait gave up: block << 40 | warp << 32 |
// shared-memory address of the mbarrier (0 = none).
__device__ unsigned long long g_timeout_site = 0ull;

// ----------------------------------------------------------- device helpers
#ifdef __CUDACC__

// Wall-clock bound for every spin-wait (nanoseconds).  A wait that runs out
// sets a SPK_DEV_* bit in g_device_error and returns false; callers then
// drain what they issued and leave the kernel.
constexpr uint64_t kSpinLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void report_device_error(int code) { atomicOr(&g_device_error, code); }

// One GSMC cell update (FusedGSMC._step_gates / gsmc_step_kernel order,
// gsmc_cuda.cu:11-77): pre = (gi + gr) / gate_scale + bias (the bias a second
// time on top of the W_in bias inside gi), f, i, o = 1 / (1 + expf(-pre)),
// g = tanhf(pre), a = f*m + i*g, v = o*tanhf(a) + wd, theta = v_th*(1 + heat)
// (adaptive), s = v > theta, m = a - s*v_th, heat = beta*heat + s; and the
// pooled output (mode 0: first plane of a mean, 1: middle, 2: last plane,
// scaled, 3: "last" pooling, 4: mean over one plane).  Shared by the step
// kernel and the fused recurrence so that both give the same bits.
struct GsmcCell {
  const float* gi;    // [M, 4d] this plane's input projection (with the W_in bias)
  const float* wd;    // [M, d]
  const float* bias;  // [4d] the W_in bias
  float* m;           // [M, d] state, updated in place
  float* heat;        // [M, d] state, updated in place
  float* s_out;       // [M, d] this plane's spikes
  float* out_t;       // [M, d] or null
  float* pooled;      // [M, d] or null
  int d;
  float v_th, gate_scale, beta, pool_scale;
  int adaptive, pool_mode;
};

__device__ __forceinline__ float gsmc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// The cell's inputs, loaded ahead of its update (they do not depend on the
// recurrent projection, so a caller can have them in flight meanwhile).
struct GsmcIn {
  float gi[4], wd, m, heat, pooled;
};

__device__ __forceinline__ GsmcIn gsmc_load(const GsmcCell& c, int64_t row, int col) {
  const int d = c.d;
  const int64_t idx = row * d + col;
  const float* gir = c.gi + row * 4 * d;
  GsmcIn in;
  in.gi[0] = gir[col];
  in.gi[1] = gir[d + col];
  in.gi[2] = gir[2 * d + col];
  in.gi[3] = gir[3 * d + col];
  in.wd = c.wd[idx];
  in.m = c.m[idx];
  in.heat = c.heat[idx];
  in.pooled = (c.pooled != nullptr && (c.pool_mode == 1 || c.pool_mode == 2)) ? c.pooled[idx] : 0.0f;
  return in;
}

__device__ __forceinline__ void gsmc_update(const GsmcCell& c, int64_t row, int col, const GsmcIn& in, float gr_f,
                                            float gr_i, float gr_o, float gr_g) {
  const int d = c.d;
  const int64_t idx = row * d + col;
  const float f = gsmc_sigmoid((in.gi[0] + gr_f) / c.gate_scale + c.bias[col]);
  const float i = gsmc_sigmoid((in.gi[1] + gr_i) / c.gate_scale + c.bias[d + col]);
  const float o = gsmc_sigmoid((in.gi[2] + gr_o) / c.gate_scale + c.bias[2 * d + col]);
  const float g = tanhf((in.gi[3] + gr_g) / c.gate_scale + c.bias[3 * d + col]);
  const float a = f * in.m + i * g;
  const float v = o * tanhf(a) + in.wd;
  const float h = in.heat;
  const float theta = c.adaptive ? c.v_th * (1.0f + h) : c.v_th;
  const float sn = (v > theta) ? 1.0f : 0.0f;
  c.m[idx] = a - sn * c.v_th;
  c.s_out[idx] = sn;
  c.heat[idx] = c.adaptive ? c.beta * h + sn : 0.0f;
  if (c.out_t != nullptr) c.out_t[idx] = sn;
  if (c.pooled != nullptr) {
    float* p = c.pooled + idx;
    if (c.pool_mode == 0) *p = sn;
    else if (c.pool_mode == 1) *p = in.pooled + sn;
    else if (c.pool_mode == 2) *p = (in.pooled + sn) * c.pool_scale;
    else if (c.pool_mode == 3) *p = sn;
    else *p = sn * c.pool_scale;
  }
}

__device__ __forceinline__ void gsmc_cell(const GsmcCell& c, int64_t row, int col, float gr_f, float gr_i, float gr_o,
                                          float gr_g) {
  gsmc_update(c, row, col, gsmc_load(c, row, col), gr_f, gr_i, gr_o, gr_g);
}

// Device-side branch choice of spike-linear's automatic mode: a kernel given a
// gate word runs only when the word holds its value (written by earlier
// kernels of the same stream), otherwise it returns at once.
constexpr int kGateTryCsr = 3;  // probe word: density may be below the crossover, let the CSR scan decide
__device__ __forceinline__ bool gated_off(const int* gate, int value) {
  return gate != nullptr && *reinterpret_cast<const volatile int*>(gate) != value;
}

// First 1024-byte-aligned byte of a dynamic shared array.  Offsetting the
// __shared__ array itself (rather than rounding an integer address) keeps the
// pointer in the shared state space, so accesses through it compile to
// shared-memory loads and stores instead of generic ones.
__device__ __forceinline__ unsigned char* smem_aligned_1024(unsigned char* smem) {
  return smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
}

// ---- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps in hardware until it completes or `hint_ns` passes, instead of
// re-issuing the test (which would take issue slots from working warps).
// kCl: acquire at cluster scope (barriers that the peer CTA of a pair, or a
// commit multicast to both CTAs, arrives on).
template <bool kCl = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 500000u) {
  uint32_t ok;
  if constexpr (kCl) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
  }
  return ok != 0;
}
// Bounded wait on the given phase parity (each try sleeps up to 0.5 ms).
// Also gives up early when *abort (a shared-memory flag other roles set after
// their own timeout) is raised.
template <bool kCl = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_try_wait<kCl>(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait<kCl>(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (global_ns() - t0 > kSpinLimitNs) {
      report_device_error(code);
      atomicCAS(&g_timeout_site, 0ull,
                ((unsigned long long)blockIdx.x << 40) | ((unsigned long long)(threadIdx.x >> 5) << 32) | smem_u32(bar));
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}

// ---- 1-D bulk copy global -> this CTA's shared memory, completes on an mbarrier
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 (cta_group::1 only)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// End of a warp-specialised kernel, before TMEM is released.  Roles run by one
// lane leave their warp diverged, and an aligned CTA barrier must be reached
// by whole warps (a warp whose other lanes arrive first can count as arrived
// while its working lane is still in its loop), so each warp reconverges
// first.
__device__ __forceinline__ void role_join() {
  __syncwarp();
  tc_fence_before();
  __syncthreads();
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16/f16 inputs, fp32 accumulate)
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- CTA pairs (cluster of two, tcgen05 cta_group::2) ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Arrive on the barrier at the same shared-memory offset in CTA 0 of the
// cluster (this CTA's own when it is CTA 0), release at cluster scope.
__device__ __forceinline__ void mbar_arrive_rank0(uint64_t* bar) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(smem_u32(bar)));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(r) : "memory");
}
// Every thread of both CTAs (unbounded: all paths of the kernel reach it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Collective over the pair: the same warp of both CTAs, the same destination offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Completion of the pair's MMAs issued so far: one arrive on the barrier at
// this offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 data-path lanes x 32 bit, 32 consecutive columns: thread i of the warp
// writes r[0..31] to columns [col, col+32) of TMEM lane (lane_base + i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// tcgen05.ld fills its destination registers asynchronously; the compiler sees
// them as written by the ld statement and may schedule their uses before
// tcgen05.wait::ld.  Passing them through an empty volatile statement placed
// after the wait makes every use depend on it.
__device__ __forceinline__ void tmem_reg_fence(float (&v)[16]) {
  asm volatile(""
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                 "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]),
                 "+f"(v[15]));
}

// 32 data-path lanes x 32 bit, 16 consecutive columns: thread i of the warp
// receives columns [col, col+16) of TMEM lane (lane_base + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 TMEM lanes x 256 bits, 4 (x4) or 2 (x2) repetitions along the columns:
// thread t holds, for repetition j, columns 8j + 2(t % 4) + {0, 1} of lane
// base + t / 4 (v[4j], v[4j+1]) and of lane base + t / 4 + 8 (v[4j+2],
// v[4j+3]) -- four threads share a row, so row stores fill whole sectors.
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, float (&v)[16]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
#pragma unroll
  for (int i = 8; i < 16; ++i) v[i] = 0.0f;
}

// UMMA shared-memory matrix descriptor for a K-major operand stored in the
// canonical 128-byte-swizzled layout: rows of 128 bytes, 8-row groups 1024
// bytes apart, the 16-byte chunk c of row r stored at chunk (c ^ (r & 7)).
// The operand base must be 1024-byte aligned; advancing along K by 16 bf16
// elements (32 bytes) adds 2 to the start-address field.
__device__ __forceinline__ uint64_t umma_desc_sw128_kmajor(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);   // start address  [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                      // swizzle mode: 128 B
  return d;
}

// Shared-memory descriptor of an MN-major bf16 operand with 128-byte swizzle:
// swizzle atoms of 8 K-lines x 64 MN-elements (1024 B, each line 128 B of
// consecutive MN elements); `mn_stride` = bytes between atoms along MN
// (leading byte offset), `k_stride` = bytes between atoms along K (stride
// byte offset).  Atoms start on 1024-byte boundaries.
__device__ __forceinline__ uint64_t umma_desc_sw128_mnmajor(uint32_t smem_addr, uint32_t mn_stride,
                                                            uint32_t k_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((mn_stride >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((k_stride >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32; A and B K-major
// unless a_mn / b_mn select the MN-major (transposed) operand layout.
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int M, int N, bool a_mn = false, bool b_mn = false) {
  return (1u << 4)                                // D format f32
         | (1u << 7)                              // A format bf16
         | (1u << 10)                             // B format bf16
         | (a_mn ? (1u << 15) : 0u)               // A major: MN
         | (b_mn ? (1u << 16) : 0u)               // B major: MN
         | (static_cast<uint32_t>(N >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24); // M / 16
}

// Byte offset of element (r, k) (k in [0, 64)) of a bf16 K-major SW128 block.
// The swizzle is a function of the address alone, so the same offset serves an
// MN-major atom with r = the K-line (0-7) and k = the MN element (0-63).
__host__ __device__ __forceinline__ uint32_t sw128_offset_bf16(uint32_t r, uint32_t k) {
  return r * 128u + ((((k >> 3) ^ (r & 7u)) & 7u) << 4) + ((k & 7u) << 1);
}

// fp32 -> (hi, lo) bf16 pair with hi + lo == x to ~2^-17 relative.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  float h = __bfloat162float(hi);
  if (!isfinite(h)) {  // rounding overflowed: keep the representable part
    hi = __float2bfloat16_rz(x);
    h = __bfloat162float(hi);
  }
  lo = isfinite(x) ? __float2bfloat16_rn(x - h) : __float2bfloat16_rn(0.0f);
}

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 a, __nv_bfloat16 b) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(a)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b)) << 16);
}

// relaxed 64-bit loads / stores at GPU scope for the look-back descriptors
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

#endif  // __CUDACC__

}  // namespace spk
