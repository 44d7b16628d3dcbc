// Spiking linear attention (AstrocyteHebbianAttention, attention.py:105-136).
//
// Compat ops with the reference engine's exact arithmetic:
//   apply_channel_decay        k * powf(lam_c, N-1-n)      (attention_cuda.cu:7-27)
//   fused_normalize_attention  numer / (denom + eps)        (attention_cuda.cu:29-40)
//
// Fused path (replaces decay -> head split -> two matmuls -> normalize, which
// makes ~10 full-tensor passes in the reference): per (bt, head)
//   pass 1  kv[j1, j2] = sum_n k[n,j1] w[n,j1] v[n,j2],  key_mass[j1] = sum_n k[n,j1] w[n,j1]
//           with w[n, c] = powf(lam_c, L-1-n) from a per-call table (L x d);
//   pass 2  out[n, j2] = (sum_j1 q[n,j1] kv[j1,j2]) / ((sum_j1 q[n,j1] key_mass[j1]) + eps)
// so q, k and v are each read once and the output written once, in d_model
// layout (no head transposes).
#include "spk_common.cuh"

namespace spk {

__global__ void channel_decay_kernel(const float* __restrict__ k, const float* __restrict__ lam, int64_t total,
                                     int N, int d, float* __restrict__ kw) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % d);
    const int n = (int)((i / d) % N);
    kw[i] = k[i] * powf(lam[c], (float)(N - 1 - n));
  }
}

__global__ void normalize_kernel(const float* __restrict__ numer, const float* __restrict__ denom, int64_t total,
                                 float eps, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = numer[i] / (denom[i] + eps);
}

__global__ void decay_table_kernel(const float* __restrict__ lam, int L, int d, float* __restrict__ tab) {
  // a programmatic dependent (the tensor-core kv pass) may start its prologue
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t total = (int64_t)L * d;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % d);
    const int n = (int)(i / d);
    tab[i] = powf(lam[c], (float)(L - 1 - n));
  }
}

// Pass 1: one CTA per (head, bt); (DH/4)^2 threads, each owning a 4x4 block of kv.
template <int DH>
__global__ void __launch_bounds__((DH / 4) * (DH / 4) < 32 ? 32 : (DH / 4) * (DH / 4))
attn_kv_kernel(const float* __restrict__ k, const float* __restrict__ v, const float* __restrict__ tab, int L,
               int H, float* __restrict__ kvout) {
  constexpr int B4 = DH / 4;
  constexpr int CH = 32;  // sequence rows staged per step
  __shared__ __align__(16) float skw[CH][DH];
  __shared__ __align__(16) float sv[CH][DH];
  const int h = blockIdx.x;
  const int64_t bt = blockIdx.y;
  const int d = H * DH;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int a = tid / B4, b = tid % B4;  // j1 block, j2 block
  const bool owner = tid < B4 * B4;
  float acc[4][4];
  float km[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    km[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }
  const float* kb = k + bt * (int64_t)L * d + h * DH;
  const float* vb = v + bt * (int64_t)L * d + h * DH;
  const float* tb = tab + h * DH;
  for (int n0 = 0; n0 < L; n0 += CH) {
    const int rows = min(CH, L - n0);
    __syncthreads();
    for (int i = tid; i < CH * B4; i += nthr) {
      const int r = i / B4, c4 = (i % B4) * 4;
      float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk, ww = kk;
      if (r < rows) {
        kk = *reinterpret_cast<const float4*>(kb + (int64_t)(n0 + r) * d + c4);
        vv = *reinterpret_cast<const float4*>(vb + (int64_t)(n0 + r) * d + c4);
        ww = *reinterpret_cast<const float4*>(tb + (int64_t)(n0 + r) * d + c4);
      }
      *reinterpret_cast<float4*>(&skw[r][c4]) = make_float4(kk.x * ww.x, kk.y * ww.y, kk.z * ww.z, kk.w * ww.w);
      *reinterpret_cast<float4*>(&sv[r][c4]) = vv;
    }
    __syncthreads();
    if (owner) {
      for (int r = 0; r < rows; ++r) {
        const float4 x = *reinterpret_cast<const float4*>(&skw[r][4 * a]);
        const float4 y = *reinterpret_cast<const float4*>(&sv[r][4 * b]);
        const float xs[4] = {x.x, x.y, x.z, x.w};
        const float ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          km[i] += xs[i];
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xs[i], ys[j], acc[i][j]);
        }
      }
    }
  }
  if (owner) {
    // kv block layout per (bt, h): [DH rows j1][DH + 1 cols]; col DH = key_mass
    float* o = kvout + ((int64_t)bt * H + h) * DH * (DH + 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) o[(4 * a + i) * (DH + 1) + 4 * b + j] = acc[i][j];
      if (b == 0) o[(4 * a + i) * (DH + 1) + DH] = km[i];
    }
  }
}

// Pass 2: one CTA per (row block of 64, head, bt).
template <int DH>
__global__ void __launch_bounds__(256) attn_out_kernel(const float* __restrict__ q, const float* __restrict__ kvin,
                                                       int L, int H, float eps, float* __restrict__ out) {
  constexpr int B4 = DH / 4;         // threads per row
  constexpr int RB = 64;             // rows per CTA
  __shared__ __align__(16) float skv[DH][DH + 4];
  __shared__ float skm[DH];
  __shared__ __align__(16) float sq[RB][DH];
  const int h = blockIdx.y;
  const int64_t bt = blockIdx.z;
  const int n0 = blockIdx.x * RB;
  const int d = H * DH;
  const int tid = threadIdx.x;
  const float* kvp = kvin + ((int64_t)bt * H + h) * DH * (DH + 1);
  for (int i = tid; i < DH * (DH + 1); i += blockDim.x) {
    const int r = i / (DH + 1), c = i % (DH + 1);
    if (c < DH) skv[r][c] = kvp[i];
    else skm[r] = kvp[i];
  }
  const int rows = min(RB, L - n0);
  for (int i = tid; i < RB * B4; i += blockDim.x) {
    const int r = i / B4, c4 = (i % B4) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) x = *reinterpret_cast<const float4*>(q + (bt * L + n0 + r) * (int64_t)d + h * DH + c4);
    *reinterpret_cast<float4*>(&sq[r][c4]) = x;
  }
  __syncthreads();
  const int per_pass = blockDim.x / B4;
  const int jb = tid % B4;
  for (int r = tid / B4; r < rows; r += per_pass) {
    float num[4] = {0.f, 0.f, 0.f, 0.f};
    float den = 0.f;
    for (int j1 = 0; j1 < DH; ++j1) {
      const float qq = sq[r][j1];
      const float4 kv4 = *reinterpret_cast<const float4*>(&skv[j1][4 * jb]);
      num[0] = fmaf(qq, kv4.x, num[0]);
      num[1] = fmaf(qq, kv4.y, num[1]);
      num[2] = fmaf(qq, kv4.z, num[2]);
      num[3] = fmaf(qq, kv4.w, num[3]);
      den = fmaf(qq, skm[j1], den);
    }
    const float de = den + eps;
    float4 o = make_float4(num[0] / de, num[1] / de, num[2] / de, num[3] / de);
    *reinterpret_cast<float4*>(out + (bt * L + n0 + r) * (int64_t)d + h * DH + 4 * jb) = o;
  }
}

inline int grid_for(int64_t total, int threads) {
  return (int)min64(ceil_div(total, threads), 148 * 32);
}

// Workspace: the decay table [L, d], then either the SIMT path's kv blocks
// [BT, H, dh, dh + 1] or the tensor-core path's per-(bt, head group) images
// (72 KB each, see attention_tc.cu) -- sized for the larger of the two.
struct AttnLayout {
  size_t tab, kv, total;
};
inline AttnLayout attn_layout(int64_t BT, int L, int H, int dh) {
  AttnLayout A{};
  A.tab = 0;
  A.kv = align_up(sizeof(float) * (size_t)L * H * dh, 256);
  const size_t simt = sizeof(float) * (size_t)BT * H * dh * (dh + 1);
  const size_t tc = (H * dh) % 128 == 0 ? (size_t)BT * (size_t)(H * dh / 128) * 73728 : 0;
  A.total = A.kv + align_up(simt > tc ? simt : tc, 256);
  return A;
}

}  // namespace spk

extern "C" int spk_apply_channel_decay(const float* k, const float* lam, int64_t B_total, int N, int d, float* k_w,
                                       spk_stream_t stream) {
  SPK_REQUIRE(k && lam && k_w, "k, lam and k_w must be non-null");
  SPK_REQUIRE(B_total >= 0 && N > 0 && d > 0, "invalid shape");
  const int64_t total = B_total * N * d;
  if (total == 0) return SPK_OK;
  spk::channel_decay_kernel<<<spk::grid_for(total, 256), 256, 0, (cudaStream_t)stream>>>(k, lam, total, N, d, k_w);
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}

extern "C" int spk_normalize_attention(const float* numer, const float* denom, int64_t total, float eps, float* out,
                                       spk_stream_t stream) {
  SPK_REQUIRE(numer && denom && out, "numer, denom and out must be non-null");
  SPK_REQUIRE(total >= 0, "invalid size");
  if (total == 0) return SPK_OK;
  spk::normalize_kernel<<<spk::grid_for(total, 256), 256, 0, (cudaStream_t)stream>>>(numer, denom, total, eps, out);
  SPK_LAUNCH_CHECK();
  spk::count_launch(1);
  return SPK_OK;
}
