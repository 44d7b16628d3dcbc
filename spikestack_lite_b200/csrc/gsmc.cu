// GSMC cell (FusedGSMC, gsmc.py:47-148).
//
// spk_gsmc_step keeps the reference engine's step arithmetic exactly
// (gsmc_step_kernel, gsmc_cuda.cu:11-77): pre = (gi + gr) / gate_scale + bias
// (bias added a second time on top of the W_in bias inside gi, as in the
// reference), f,i,o = 1/(1+expf(-pre)), g = tanhf(pre), a = f*m + i*g,
// v = o*tanhf(a) + wd, theta = v_th*(1+heat) (adaptive), s = v > theta,
// m = a - s*v_th, heat = beta*heat + s.
//
// spk_gsmc_forward runs the whole eval-mode recurrence (gsmc.py:119-142).
// At t = 0 the state is zero, so the recurrent projection is skipped and the
// step kernel runs alone.  For t >= 1 (d % 32 == 0) one tensor-core kernel per
// plane does both halves of the reference's loop body: gr = W_rec s_{t-1}
// (s binary, exact in tf32; W_rec split tf32 hi + lo, as the spike-linear
// dense branch) accumulates in tensor memory, with W_rec's rows regrouped so
// that each 128-column tile holds the f, i, o and g rows of 32 channels, and
// the epilogue applies the gates, the state update and the pooling to those
// channels -- gr never reaches global memory.  The spikes of consecutive
// planes alternate between two buffers (every column tile reads all of
// s_{t-1} while others write s_t).  That fused form (SPK_GSMC_FUSED) is
// correct and bit-identical to the two-kernel form, but slower at the model's
// geometry: its cell updates (48 bytes of state traffic per cell) run on the
// four epilogue warps of each SM while the single-buffered accumulators hold
// the next MMAs back, so the default is the two-kernel form -- gr through the
// spike-linear dense branch, then the step kernel over the whole GPU.
#include "spk_common.cuh"

namespace spk {

// One thread per (row, col); when pooled != null the new spike is also added
// into pooled (scaled by pool_scale on the last plane, or copied for "last").
__global__ void gsmc_step_kernel(const float* __restrict__ gi, const float* __restrict__ gr,
                                 const float* __restrict__ wd, const float* __restrict__ bias, float* __restrict__ m,
                                 float* __restrict__ s, float* __restrict__ heat, float* __restrict__ out_t,
                                 int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta,
                                 float* __restrict__ pooled, int pool_mode, float pool_scale) {
  const GsmcCell c{gi, wd, bias, m, heat, s, out_t, pooled, d, v_th, gate_scale, beta, pool_scale, adaptive, pool_mode};
  const int64_t total = M * d;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / d;
    const int col = (int)(idx % d);
    float gr_f = 0.f, gr_i = 0.f, gr_o = 0.f, gr_g = 0.f;
    if (gr != nullptr) {
      const float* grr = gr + row * 4 * d;
      gr_f = grr[col];
      gr_i = grr[d + col];
      gr_o = grr[2 * d + col];
      gr_g = grr[3 * d + col];
    }
    gsmc_cell(c, row, col, gr_f, gr_i, gr_o, gr_g);
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
  size_t m, s, heat, s2, wperm, img, gr, sl, sl_bytes, total;
};
inline GsmcLayout gsmc_layout(int64_t M, int d) {
  GsmcLayout G{};
  const size_t st = align_up(sizeof(float) * (size_t)M * d, 256);
  G.m = 0;
  G.s = st;
  G.heat = 2 * st;
  G.s2 = 3 * st;  // the fused recurrence's second spike buffer (planes alternate)
  G.wperm = 4 * st;
  G.img = align_up(G.wperm + sizeof(float) * (size_t)4 * d * d, 1024);
  G.gr = align_up(G.img + tf32_img_bytes(tc_plan(d, 4 * d, SPK_F32)), 256);
  G.sl = G.gr + align_up(sizeof(float) * (size_t)M * 4 * d, 256);
  G.sl_bytes = spk_spike_linear_workspace_bytes(1, M, d, 4 * d, SPK_F32);
  G.total = G.sl + align_up(G.sl_bytes, 256);
  return G;
}

// The fused recurrence takes d % 32 == 0 (whole 128-column gate tiles) with
// 16-byte aligned state rows; other shapes run the two-kernel form.
inline bool gsmc_fused_ok(int64_t M, int d) { return d % 32 == 0 && M < (int64_t(1) << 31); }

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

static int gsmc_forward_impl(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias, int T,
                             int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta, int pool_mean,
                             float* out_all, float* pooled, void* workspace, size_t workspace_bytes,
                             spk_stream_t stream, int form);

extern "C" int spk_gsmc_forward(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias,
                                int T, int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta,
                                int pool_mean, float* out_all, float* pooled, void* workspace,
                                size_t workspace_bytes, spk_stream_t stream) {
  return gsmc_forward_impl(gi_all, wd_all, w_rec, bias, T, M, d, v_th, gate_scale, adaptive, beta, pool_mean, out_all,
                           pooled, workspace, workspace_bytes, stream, SPK_GSMC_TWO_KERNEL);
}

extern "C" int spk_gsmc_forward_ex(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias,
                                   int T, int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta,
                                   int pool_mean, float* out_all, float* pooled, void* workspace,
                                   size_t workspace_bytes, int form, spk_stream_t stream) {
  SPK_REQUIRE(form == SPK_GSMC_TWO_KERNEL || form == SPK_GSMC_FUSED, "unknown GSMC form %d", form);
  return gsmc_forward_impl(gi_all, wd_all, w_rec, bias, T, M, d, v_th, gate_scale, adaptive, beta, pool_mean, out_all,
                           pooled, workspace, workspace_bytes, stream, form);
}

static int gsmc_forward_impl(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias, int T,
                             int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta, int pool_mean,
                             float* out_all, float* pooled, void* workspace, size_t workspace_bytes,
                             spk_stream_t stream, int form) {
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
  SPK_CUDA_TRY(cudaMemsetAsync(w, 0, G.s2, st));  // m = s = heat = 0
  const float inv_t = 1.0f / (float)T;
  const bool fused = form == SPK_GSMC_FUSED && T >= 2 && spk::gsmc_fused_ok(M, d);
  const spk::TcPlan p = spk::tc_plan(d, 4 * d, SPK_F32);
  unsigned char* img = reinterpret_cast<unsigned char*>(w + G.img);
  if (fused) {
    // W_rec [4d, d] with its rows regrouped: tile c (rows 128c .. 128c+127) holds the f, i, o, g rows of
    // channels 32c .. 32c+31, i.e. row 128c + 32q + l = W_rec row q*d + 32c + l (four strided copies)
    float* wperm = reinterpret_cast<float*>(w + G.wperm);
    const size_t blk = sizeof(float) * 32 * (size_t)d;  // 32 rows
    for (int q = 0; q < 4; ++q)
      SPK_CUDA_TRY(cudaMemcpy2DAsync(reinterpret_cast<char*>(wperm) + q * blk, 4 * blk,
                                     reinterpret_cast<const char*>(w_rec) + (size_t)q * d * d * sizeof(float), blk, blk,
                                     (size_t)d / 32, cudaMemcpyDeviceToDevice, st));
    int rc = spk::launch_w_image_tf32(wperm, 1, d, d, 4 * d, p, img, nullptr, 0, st);
    if (rc) return rc;
  }
  for (int t = 0; t < T; ++t) {
    const float* gi = gi_all + (int64_t)t * M * 4 * d;
    const float* wd = wd_all + (int64_t)t * M * d;
    float* out_t = out_all ? out_all + (int64_t)t * M * d : nullptr;
    const float* grp = nullptr;
    if (fused && t > 0) {
      int mode;
      float scale = 1.0f;
      if (!pool_mean) mode = 3;
      else if (t == T - 1) { mode = 2; scale = inv_t; }
      else mode = 1;
      float* s_prev = reinterpret_cast<float*>(w + ((t - 1) % 2 ? G.s2 : G.s));
      float* s_next = reinterpret_cast<float*>(w + (t % 2 ? G.s2 : G.s));
      const spk::GsmcCell cell{gi, wd, bias, m, heat, s_next, out_t, pooled, d, v_th, gate_scale, beta, scale,
                               adaptive, mode};
      int rc = spk::launch_wt_gsmc(s_prev, M, d, p, img, cell, st);
      if (rc) return rc;
      continue;
    }
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
