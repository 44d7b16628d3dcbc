// Spire time-repetition planes (SpireEncoder.forward in temporal mode,
// encode/spire.py:60-69, and the reference's spire_dither_kernel,
// encode/src/spire_cuda.cu:7-26): from the projection u [B, N, d],
//   v = (u - frontier[c]) - temporal_frontier[n]      (the reference's fp32 order)
//   planes[t, b, n, c] = (v - dither[t] > 0) ? 1 : 0,  t < T,
// written in (T, B, N, d) order.  One pass: u read once, the T planes written
// once; the reference composition makes two broadcast subtractions, the
// comparison and a bool -> float copy over the full tensors.
//
// Bound: HBM (4 bytes read, 4 T bytes written per element of u).
#include "spk_common.cuh"

namespace spk {

// Thread i handles the 4 channels 4 (i % d4) .. +3 of row i / d4 (row = b N + n).
__global__ void __launch_bounds__(256) spire_planes_kernel(const float4* __restrict__ u,
                                                           const float* __restrict__ frontier,
                                                           const float* __restrict__ tfront,
                                                           const float* __restrict__ dither, int T, int64_t rows,
                                                           int N, int d4, float4* __restrict__ planes) {
  const int64_t total = rows * d4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / d4;
    const int c4 = (int)(i - r * d4);
    float4 v = u[i];
    if (frontier != nullptr) {
      const float4 f = reinterpret_cast<const float4*>(frontier)[c4];
      v.x -= f.x;
      v.y -= f.y;
      v.z -= f.z;
      v.w -= f.w;
    }
    if (tfront != nullptr) {
      const float tf = tfront[r % N];
      v.x -= tf;
      v.y -= tf;
      v.z -= tf;
      v.w -= tf;
    }
    for (int t = 0; t < T; ++t) {
      const float dt = dither[t];
      float4 o;
      o.x = (v.x - dt > 0.0f) ? 1.0f : 0.0f;
      o.y = (v.y - dt > 0.0f) ? 1.0f : 0.0f;
      o.z = (v.z - dt > 0.0f) ? 1.0f : 0.0f;
      o.w = (v.w - dt > 0.0f) ? 1.0f : 0.0f;
      planes[(int64_t)t * total + i] = o;
    }
  }
}

}  // namespace spk

extern "C" int spk_spire_planes(const float* u, const float* frontier, const float* temporal_frontier,
                                const float* dither, int T, int64_t B, int N, int d, float* planes,
                                spk_stream_t stream) {
  SPK_REQUIRE(T >= 1 && B >= 0 && N >= 1 && d >= 1, "invalid shape (T=%d, B=%lld, N=%d, d=%d)", T, (long long)B, N,
              d);
  SPK_REQUIRE(d % 4 == 0, "d must be a multiple of 4 (d=%d)", d);
  if (B == 0) return SPK_OK;
  SPK_REQUIRE(u != nullptr && dither != nullptr && planes != nullptr, "u, dither and planes must be non-null");
  SPK_REQUIRE((reinterpret_cast<uintptr_t>(u) & 15u) == 0 && (reinterpret_cast<uintptr_t>(planes) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(frontier) & 15u) == 0,
              "u, planes and frontier must be 16-byte aligned");
  const int64_t rows = B * (int64_t)N;
  const int64_t total = rows * (d / 4);
  const int64_t want = spk::ceil_div(total, (int64_t)256);
  const int64_t cap = (int64_t)spk::sm_count() * 16;
  const int blocks = (int)(want < cap ? want : cap);
  spk::spire_planes_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const float4*>(u), frontier, temporal_frontier, dither, T, rows, N, d / 4,
      reinterpret_cast<float4*>(planes));
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}
