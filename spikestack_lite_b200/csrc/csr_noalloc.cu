// spk_csr_compact_noalloc: the spike -> CSR compaction for callers that
// cannot allocate device memory.
//
// Some hosts own every byte of device memory themselves and hand plugins no
// workspace: an FFI host without a CUDA allocator of its own, or a serving
// loop that forbids cudaMalloc after start-up because an allocation can
// synchronise the device and stall the other streams.  Such a caller cannot
// provide the scratch that spk_csr_compact's look-back scan needs, so this
// entry point keeps that scratch in a fixed array in the library itself.
//
// The array below (kNoAllocScratchBytes = 1 MiB) is part of the library's
// device image: every GPU that loads the library holds it until the process
// exits.  It bounds the problem size: the scan needs 256 bytes of state, 9
// bytes per row tile (a tile is up to 128 rows of one plane) and 8 bytes per
// plane, rounded up to 256 -- exactly spk_csr_workspace_bytes(T, M, K), so a
// problem fits when that is <= 1 MiB (about 116 000 row tiles with few planes,
// e.g. T*M up to ~14.8 million rows when K <= 4096; fewer with many small
// planes).  Larger requests are rejected with SPK_EWORKSPACE and a message;
// use spk_csr_compact then.
//
// Host code never touches the array through its name (on the host that name
// is only a stand-in, not a device address): the first call on each device
// looks its device address up with cudaGetSymbolAddress, with that device
// current, and caches it together with the CUDA context it was found in.  That
// first call therefore does a runtime query and should come before any stream
// capture on that device.  If the context changes (cudaDeviceReset, or the
// primary context torn down and created again) the module is loaded anew and
// the next call looks the address up again instead of using a stale one.
//
// Every call shares the one array, and the array keeps whatever the last call
// left in it; the scan clears the part that must start at zero (its tile
// counter and look-back descriptors) with a stream-ordered memset at the start
// of every call.  Calls that overlap on the GPU -- on two streams, or from two
// host threads -- race on the array; issue them on one stream.
// The call allocates nothing: no cudaMalloc, no cudaFree, no library routine
// that allocates.
#include <mutex>

#include "spk_common.cuh"

namespace spk {

constexpr size_t kNoAllocScratchBytes = 1u << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* g_noalloc_ptr[kNoAllocMaxDevices] = {};
static void* g_noalloc_ctx[kNoAllocMaxDevices] = {};
static std::mutex g_noalloc_mu;

// The current CUDA context (driver cuCtxGetCurrent, reached through the
// runtime's entry-point query so the library needs no -lcuda).
static void* current_context() {
  using GetCurrent = int (*)(void**);
  static GetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<GetCurrent>(p);
    return static_cast<GetCurrent>(nullptr);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the scratch array on the current device, looked up once
// per device and context.
static int noalloc_scratch(void** out) {
  int dev = 0;
  SPK_CUDA_TRY(cudaGetDevice(&dev));
  SPK_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "device ordinal %d out of range", dev);
  void* ctx = current_context();  // null before the runtime has made a context current on this thread
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also makes the context current
    if (e != cudaSuccess || p == nullptr)
      return fail(SPK_ECUDA, "cudaGetSymbolAddress of the fixed scratch array failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = current_context();
  }
  *out = g_noalloc_ptr[dev];
  return SPK_OK;
}

}  // namespace spk

extern "C" int spk_csr_compact_noalloc(const float* S, int T, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr,
                                       int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity,
                                       spk_stream_t stream) {
  int rc = spk::check_csr_shape(T, M, K);
  if (rc) return rc;
  SPK_REQUIRE(S && row_ptr && col_idx && plane_ptr, "S, row_ptr, col_idx and plane_ptr must be non-null");
  const size_t need = spk::csr_layout(T, M, K).total;
  if (need > spk::kNoAllocScratchBytes)
    return spk::fail(SPK_EWORKSPACE,
                     "spk_csr_compact_noalloc: T=%d x M=%lld rows need %zu bytes of scan scratch, above the fixed "
                     "%zu-byte limit of this entry point; call spk_csr_compact with a workspace instead",
                     T, (long long)M, need, spk::kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = spk::noalloc_scratch(&scratch);
  if (rc) return rc;
  return spk::launch_csr_scan(S, T, M, K, nnz_row, row_ptr, col_idx, values, plane_ptr, col_capacity, scratch,
                              (cudaStream_t)stream, nullptr, nullptr);
}
