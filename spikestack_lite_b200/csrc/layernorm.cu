// Residual add + layer norm of the pre-norm block (AstrocyteHebbianBlock,
// nn/attention.py:174-177): x + branch(...) followed by nn.LayerNorm(d) of
// the sum, as one pass over HBM: H = X + D and Y = LayerNorm(H) over the last
// dimension (biased variance, eps inside the square root, affine gamma/beta).
//
// Bound: HBM.  Bytes per row: 4d (X) + 4d (D) read, 4d (H) + 4d (Y) written;
// with D null (a plain layer norm) 4d read and 4d written.  The composition it
// replaces moves 12d (add) + 8d (layer norm) bytes per row in two launches.
#include "spk_common.cuh"

namespace spk {

constexpr int kLnWarps = 8;  // rows per CTA (one warp per row)

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Lane l holds the float4 vectors l, l + 32, ... (< d / 4) of its warp's row
// in registers: loads, both statistics passes and the stores touch each
// element once.  NV = float4 vectors per lane (d <= 128 NV).
template <int NV>
__global__ void __launch_bounds__(kLnWarps * 32) add_layernorm_kernel(const float* X, const float* D,
                                                                     const float* __restrict__ gamma,
                                                                     const float* __restrict__ beta, int64_t rows,
                                                                     int d, float eps, float* H, float* Y) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = d >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(X + row * d);
  const float4* d4 = D != nullptr ? reinterpret_cast<const float4*>(D + row * d) : nullptr;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < nv) v[i] = x4[c];
  }
  if (d4 != nullptr) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        const float4 b = d4[c];
        v[i].x += b.x;
        v[i].y += b.y;
        v[i].z += b.z;
        v[i].w += b.w;
      }
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);  // padding lanes hold zeros
  const float mean = warp_sum_f32(sum) / (float)d;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (lane + 32 * i < nv) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
      sq += (a * a + b * b) + (c * c + e * e);
    }
  }
  const float rstd = rsqrtf(warp_sum_f32(sq) / (float)d + eps);
  float4* h4 = (d4 != nullptr && H != nullptr) ? reinterpret_cast<float4*>(H + row * d) : nullptr;
  float4* y4 = reinterpret_cast<float4*>(Y + row * d);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c >= nv) continue;
    if (h4 != nullptr) h4[c] = v[i];
    const float4 g = g4 != nullptr ? g4[c] : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 b = b4 != nullptr ? b4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 y;
    y.x = fmaf((v[i].x - mean) * rstd, g.x, b.x);
    y.y = fmaf((v[i].y - mean) * rstd, g.y, b.y);
    y.z = fmaf((v[i].z - mean) * rstd, g.z, b.z);
    y.w = fmaf((v[i].w - mean) * rstd, g.w, b.w);
    y4[c] = y;
  }
}

}  // namespace spk

extern "C" int spk_add_layernorm(const float* X, const float* D, const float* gamma, const float* beta,
                                 int64_t rows, int d, float eps, float* H, float* Y, spk_stream_t stream) {
  SPK_REQUIRE(rows >= 0 && d > 0, "invalid shape (rows=%lld, d=%d)", (long long)rows, d);
  SPK_REQUIRE(d % 4 == 0, "d must be a multiple of 4 (d=%d)", d);
  if (d > 1024) return spk::fail(SPK_EUNSUPPORTED, "layer norm width d=%d above 1024", d);
  SPK_REQUIRE(eps >= 0.0f, "eps must be non-negative");
  if (rows == 0) return SPK_OK;
  SPK_REQUIRE(X != nullptr && Y != nullptr, "X and Y must be non-null");
  SPK_REQUIRE(D == nullptr || H != nullptr, "H must be non-null when D is given");
  const void* ptrs[6] = {X, D, gamma, beta, H, Y};
  for (const void* p : ptrs)
    SPK_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15u) == 0, "tensors must be 16-byte aligned");
  const int64_t blocks = spk::ceil_div(rows, (int64_t)spk::kLnWarps);
  SPK_REQUIRE(blocks < (1ll << 31), "too many rows (%lld)", (long long)rows);
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)blocks), block(spk::kLnWarps * 32);
  const int nv = d / 4;
  if (nv <= 32)
    spk::add_layernorm_kernel<1><<<grid, block, 0, st>>>(X, D, gamma, beta, rows, d, eps, H, Y);
  else if (nv <= 64)
    spk::add_layernorm_kernel<2><<<grid, block, 0, st>>>(X, D, gamma, beta, rows, d, eps, H, Y);
  else if (nv <= 128)
    spk::add_layernorm_kernel<4><<<grid, block, 0, st>>>(X, D, gamma, beta, rows, d, eps, H, Y);
  else
    spk::add_layernorm_kernel<8><<<grid, block, 0, st>>>(X, D, gamma, beta, rows, d, eps, H, Y);
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}
