// GSMC cell (FusedGSMC, gsmc.py:47-148).
//
// spk_gsmc_step keeps the reference engine's step arithmetic exactly
// (gsmc_step_kernel, gsmc_cuda.cu:11-77): pre = (gi + gr) / gate_scale + bias
// (bias added a second time on top of the W_in bias inside gi, as in the
// reference), f,i,o = 1/(1+expf(-pre)), g = tanhf(pre), a = f*m + i*g,
// v = o*tanhf(a) + wd, theta = v_th*(1+heat) (adaptive), s = v > theta,
// m = a - s*v_th, heat = beta*heat + s.
//
// spk_gsmc_forward runs the whole eval-mode recurrence: per plane t the
// recurrent projection gr = W_rec s_{t-1} goes through the spike-linear dense
// branch (s is binary, so bf16 is exact for it; W_rec is split hi/lo), then
// the step kernel updates the state and accumulates the pooled output.  At
// t = 0 the state is zero, so the projection is skipped.
#include "spk_common.cuh"

namespace spk {

__device__ __forceinline__ float gsmc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// One thread per (row, col); when pooled != null the new spike is also added
// into pooled (scaled by pool_scale on the last plane, or copied for "last").
__global__ void gsmc_step_kernel(const float* __restrict__ gi, const float* __restrict__ gr,
                                 const float* __restrict__ wd, const float* __restrict__ bias, float* __restrict__ m,
                                 float* __restrict__ s, float* __restrict__ heat, float* __restrict__ out_t,
                                 int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta,
                                 float* __restrict__ pooled, int pool_mode, float pool_scale) {
  const int64_t total = M * d;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / d;
    const int col = (int)(idx % d);
    const float* gir = gi + row * 4 * d;
    const float gi_f = gir[col], gi_i = gir[d + col], gi_o = gir[2 * d + col], gi_g = gir[3 * d + col];
    float gr_f = 0.f, gr_i = 0.f, gr_o = 0.f, gr_g = 0.f;
    if (gr != nullptr) {
      const float* grr = gr + row * 4 * d;
      gr_f = grr[col];
      gr_i = grr[d + col];
      gr_o = grr[2 * d + col];
      gr_g = grr[3 * d + col];
    }
    const float f = gsmc_sigmoid((gi_f + gr_f) / gate_scale + bias[col]);
    const float i = gsmc_sigmoid((gi_i + gr_i) / gate_scale + bias[d + col]);
    const float o = gsmc_sigmoid((gi_o + gr_o) / gate_scale + bias[2 * d + col]);
    const float g = tanhf((gi_g + gr_g) / gate_scale + bias[3 * d + col]);
    const float a = f * m[idx] + i * g;
    const float v = o * tanhf(a) + wd[idx];
    const float h = heat[idx];
    const float theta = adaptive ? v_th * (1.0f + h) : v_th;
    const float sn = (v > theta) ? 1.0f : 0.0f;
    m[idx] = a - sn * v_th;
    s[idx] = sn;
    heat[idx] = adaptive ? beta * h + sn : 0.0f;
    if (out_t != nullptr) out_t[idx] = sn;
    if (pooled != nullptr) {
      if (pool_mode == 0) pooled[idx] = sn;                       // first plane of a mean: start the count
      else if (pool_mode == 1) pooled[idx] += sn;                 // middle plane
      else if (pool_mode == 2) pooled[idx] = (pooled[idx] + sn) * pool_scale;  // last plane: finish the mean
      else if (pool_mode == 3) pooled[idx] = sn;                  // "last" pooling
      else pooled[idx] = sn * pool_scale;                         // mean over a single plane
    }
  }
}

int launch_gsmc_step(const float* gi, const float* gr, const float* wd, const float* bias, float* m, float* s,
                     float* heat, float* out_t, int64_t M, int d, float v_th, float gs, int adaptive, float beta,
                     float* pooled, int pool_mode, float pool_scale, cudaStream_t stream) {
  const int64_t total = M * d;
  const int blocks = (int)min64(ceil_div(total, 256), 148 * 32);
  prof_before(SPK_KERNEL_GSMC_STEP, stream);
  gsmc_step_kernel<<<blocks, 256, 0, stream>>>(gi, gr, wd, bias, m, s, heat, out_t, M, d, v_th, gs, adaptive, beta,
                                               pooled, pool_mode, pool_scale);
  prof_after(SPK_KERNEL_GSMC_STEP, stream);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

// spike_linear_impl (spike_linear.cu, earlier in this translation unit) runs the recurrent projection.

struct GsmcLayout {
  size_t m, s, heat, gr, sl, sl_bytes, total;
};
inline GsmcLayout gsmc_layout(int64_t M, int d) {
  GsmcLayout G{};
  const size_t st = align_up(sizeof(float) * (size_t)M * d, 256);
  G.m = 0;
  G.s = st;
  G.heat = 2 * st;
  G.gr = 3 * st;
  G.sl = G.gr + align_up(sizeof(float) * (size_t)M * 4 * d, 256);
  G.sl_bytes = spk_spike_linear_workspace_bytes(1, M, d, 4 * d, SPK_F32);
  G.total = G.sl + align_up(G.sl_bytes, 256);
  return G;
}

}  // namespace spk

extern "C" int spk_gsmc_step(const float* gi, const float* gr, const float* wd, const float* bias, float* m, float* s,
                             float* heat, float* out_t, int64_t M, int d, float v_th, float gate_scale, int adaptive,
                             float beta, spk_stream_t stream) {
  SPK_REQUIRE(gi && gr && wd && bias && m && s && heat && out_t, "all tensors must be non-null");
  SPK_REQUIRE(M >= 0 && d > 0, "invalid shape");
  if (M == 0) return SPK_OK;
  return spk::launch_gsmc_step(gi, gr, wd, bias, m, s, heat, out_t, M, d, v_th, gate_scale, adaptive, beta, nullptr,
                               0, 1.0f, (cudaStream_t)stream);
}

extern "C" size_t spk_gsmc_workspace_bytes(int64_t M, int d) {
  if (M < 1 || d < 1) return 0;
  return spk::gsmc_layout(M, d).total;
}

extern "C" int spk_gsmc_forward(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias,
                                int T, int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta,
                                int pool_mean, float* out_all, float* pooled, void* workspace,
                                size_t workspace_bytes, spk_stream_t stream) {
  SPK_REQUIRE(gi_all && wd_all && w_rec && bias && pooled, "gi_all, wd_all, w_rec, bias and pooled must be non-null");
  SPK_REQUIRE(T >= 1 && M >= 1 && d >= 1, "invalid shape");
  const spk::GsmcLayout G = spk::gsmc_layout(M, d);
  if (workspace == nullptr || workspace_bytes < G.total)
    return spk::fail(SPK_EWORKSPACE, "workspace of %zu bytes required", G.total);
  cudaStream_t st = (cudaStream_t)stream;
  char* w = static_cast<char*>(workspace);
  float* m = reinterpret_cast<float*>(w + G.m);
  float* s = reinterpret_cast<float*>(w + G.s);
  float* heat = reinterpret_cast<float*>(w + G.heat);
  float* gr = reinterpret_cast<float*>(w + G.gr);
  SPK_CUDA_TRY(cudaMemsetAsync(w, 0, G.gr, st));  // m = s = heat = 0
  const float inv_t = 1.0f / (float)T;
  for (int t = 0; t < T; ++t) {
    const float* gi = gi_all + (int64_t)t * M * 4 * d;
    const float* wd = wd_all + (int64_t)t * M * d;
    float* out_t = out_all ? out_all + (int64_t)t * M * d : nullptr;
    const float* grp = nullptr;
    if (t > 0) {
      // gr[m, n] = sum_k s[m, k] * W_rec[n, k]   (nn.Linear weight, [4d, d])
      int rc = spk::spike_linear_impl(s, 1, M, d, w_rec, SPK_F32, 1, d, 4 * d, nullptr, gr, nullptr, nullptr,
                                      nullptr, nullptr, nullptr, 0, SPK_BRANCH_AUTO, w + G.sl, G.sl_bytes, st);
      if (rc) return rc;
      grp = gr;
    }
    int mode;
    float scale = 1.0f;
    if (!pool_mean) {
      mode = 3;
    } else if (T == 1) {
      mode = 4;
      scale = inv_t;
    } else if (t == 0) {
      mode = 0;
    } else if (t == T - 1) {
      mode = 2;
      scale = inv_t;
    } else {
      mode = 1;
    }
    int rc = spk::launch_gsmc_step(gi, grp, wd, bias, m, s, heat, out_t, M, d, v_th, gate_scale, adaptive, beta,
                                   pooled, mode, scale, st);
    if (rc) return rc;
  }
  return SPK_OK;
}
