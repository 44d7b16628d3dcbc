// Readout pooling of SpikingTransformer.forward (models/transformer.py:159-192):
// over the temporal context x [T, B, N, d] (T = 1 for the GSMC-pooled
// [B, N, d]), per sample b and channel c, the mean over (t, n) of x (the
// latency head's pooled input) and of spike(x) = (x > 0) (the classifier's
// input), both in one pass.
//
// Bound: HBM (4 bytes per element read once).  The composition it replaces
// reads the context three times (spike, mean of the spikes, mean of x) and
// writes the spike tensor once.
#include "spk_common.cuh"

namespace spk {

constexpr int kMeanWarps = 8;

// One CTA per (sample b, 128-channel group): lane l of warp w sums channels
// 4l .. 4l + 3 of the group over rows w, w + 8, ... of the T*N rows of b.
__global__ void __launch_bounds__(kMeanWarps * 32) temporal_mean_kernel(const float* __restrict__ x, int T, int64_t B,
                                                                        int N, int d, float inv_n,
                                                                        float* __restrict__ mean_x,
                                                                        float* __restrict__ mean_spike) {
  __shared__ float4 s_sum[kMeanWarps][32];
  __shared__ float4 s_cnt[kMeanWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.x;
  const int c = blockIdx.y * 128 + 4 * lane;
  const bool active = c < d;
  float4 sum = make_float4(0.f, 0.f, 0.f, 0.f), cnt = make_float4(0.f, 0.f, 0.f, 0.f);
  const int rows = T * N;
  if (active) {
#pragma unroll 4
    for (int i = warp; i < rows; i += kMeanWarps) {
      const int t = i / N, n = i - t * N;
      const float4 v = *reinterpret_cast<const float4*>(x + (((int64_t)t * B + b) * N + n) * d + c);
      sum.x += v.x;
      sum.y += v.y;
      sum.z += v.z;
      sum.w += v.w;
      cnt.x += v.x > 0.f ? 1.f : 0.f;  // exact: counts stay below 2^24
      cnt.y += v.y > 0.f ? 1.f : 0.f;
      cnt.z += v.z > 0.f ? 1.f : 0.f;
      cnt.w += v.w > 0.f ? 1.f : 0.f;
    }
  }
  s_sum[warp][lane] = sum;
  s_cnt[warp][lane] = cnt;
  __syncthreads();
  if (warp == 0 && active) {
    float4 a = s_sum[0][lane], k = s_cnt[0][lane];
    for (int w = 1; w < kMeanWarps; ++w) {
      const float4 p = s_sum[w][lane], q = s_cnt[w][lane];
      a.x += p.x;
      a.y += p.y;
      a.z += p.z;
      a.w += p.w;
      k.x += q.x;
      k.y += q.y;
      k.z += q.z;
      k.w += q.w;
    }
    if (mean_x != nullptr)
      *reinterpret_cast<float4*>(mean_x + b * d + c) = make_float4(a.x * inv_n, a.y * inv_n, a.z * inv_n, a.w * inv_n);
    if (mean_spike != nullptr)
      *reinterpret_cast<float4*>(mean_spike + b * d + c) =
          make_float4(k.x * inv_n, k.y * inv_n, k.z * inv_n, k.w * inv_n);
  }
}

}  // namespace spk

extern "C" int spk_temporal_mean(const float* x, int T, int64_t B, int N, int d, float* mean_x, float* mean_spike,
                                 spk_stream_t stream) {
  SPK_REQUIRE(T >= 1 && B >= 0 && N >= 1 && d >= 1, "invalid shape (T=%d, B=%lld, N=%d, d=%d)", T, (long long)B, N,
              d);
  SPK_REQUIRE(d % 4 == 0, "d must be a multiple of 4 (d=%d)", d);
  SPK_REQUIRE((int64_t)T * N < (1 << 24), "T*N must stay below 2^24 (exact spike counts)");
  SPK_REQUIRE(B < 2147483648ll, "too many samples");
  if (B == 0) return SPK_OK;
  SPK_REQUIRE(x != nullptr && (mean_x != nullptr || mean_spike != nullptr), "x and an output must be non-null");
  SPK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(mean_x) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(mean_spike) & 15u) == 0,
              "tensors must be 16-byte aligned");
  const float inv_n = 1.0f / (float)((int64_t)T * N);
  const dim3 grid((unsigned)B, (unsigned)((d + 127) / 128));
  spk::temporal_mean_kernel<<<grid, spk::kMeanWarps * 32, 0, (cudaStream_t)stream>>>(x, T, B, N, d, inv_n, mean_x,
                                                                                    mean_spike);
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}
