// Error reporting, version and device-error plumbing shared by all entry points.
#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "spk_common.cuh"

namespace spk {

static thread_local char t_last_error[1024] = "";
static std::atomic<int64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { t_last_error[0] = '\0'; }

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// ---- per-kernel CUDA-event timing (spk_profile_begin / spk_profile_end)
struct EventPair {
  cudaEvent_t start, stop;
};
static std::mutex g_prof_mu;
static int g_prof_kernel = 0;
static std::vector<EventPair> g_prof_events;

void prof_before(int kernel_id, cudaStream_t stream) {
  if (g_prof_kernel != kernel_id) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  EventPair p{};
  if (cudaEventCreate(&p.start) != cudaSuccess || cudaEventCreate(&p.stop) != cudaSuccess) return;
  cudaEventRecord(p.start, stream);
  g_prof_events.push_back(p);
}

void prof_after(int kernel_id, cudaStream_t stream) {
  if (g_prof_kernel != kernel_id) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof_events.empty()) cudaEventRecord(g_prof_events.back().stop, stream);
}

}  // namespace spk

extern "C" int spk_profile_begin(int kernel_id) {
  std::lock_guard<std::mutex> lk(spk::g_prof_mu);
  for (auto& p : spk::g_prof_events) {
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  spk::g_prof_events.clear();
  spk::g_prof_kernel = kernel_id;
  return SPK_OK;
}

extern "C" int spk_profile_end(double* total_ms, int64_t* launches) {
  std::lock_guard<std::mutex> lk(spk::g_prof_mu);
  double sum = 0.0;
  int64_t n = 0;
  int rc = SPK_OK;
  for (auto& p : spk::g_prof_events) {
    float ms = 0.f;
    if (cudaEventSynchronize(p.stop) == cudaSuccess && cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
      sum += ms;
      ++n;
    } else {
      rc = spk::fail(SPK_ECUDA, "profiling event could not be read");
    }
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  spk::g_prof_events.clear();
  spk::g_prof_kernel = 0;
  if (total_ms) *total_ms = sum;
  if (launches) *launches = n;
  return rc;
}

extern "C" const char* spk_last_error(void) { return spk::t_last_error; }

extern "C" int spk_version(void) { return 10000; }  // 1.0.0

extern "C" int64_t spk_launch_count(void) { return spk::g_launches.load(std::memory_order_relaxed); }

extern "C" int spk_device_error(int clear, int* out_bits) {
  int bits = 0;
  SPK_CUDA_TRY(cudaDeviceSynchronize());
  SPK_CUDA_TRY(cudaMemcpyFromSymbol(&bits, spk::g_device_error, sizeof(int)));
  if (clear) {
    const int zero = 0;
    const unsigned long long none = 0ull;
    SPK_CUDA_TRY(cudaMemcpyToSymbol(spk::g_device_error, &zero, sizeof(int)));
    SPK_CUDA_TRY(cudaMemcpyToSymbol(spk::g_timeout_site, &none, sizeof(none)));
  }
  if (out_bits != nullptr) *out_bits = bits;
  return SPK_OK;
}

extern "C" int spk_timeout_site(uint64_t* out_site) {
  unsigned long long site = 0ull;
  SPK_CUDA_TRY(cudaDeviceSynchronize());
  SPK_CUDA_TRY(cudaMemcpyFromSymbol(&site, spk::g_timeout_site, sizeof(site)));
  if (out_site != nullptr) *out_site = site;
  return SPK_OK;
}
