// Entry points of the spike-linear path: the new multi-plane C ABI and the
// two reference-compatible ops (sparse_forward / sparse_multistep_forward).
//
// Orchestration per call (one stream, no host synchronisation):
//   dense branch:  W image (tf32 hi/lo for fp32 W, bf16 for bf16 W; pre-
//                  swizzled)  ->  tcgen05 kernel
//                  [-> CSR scan when CSR outputs are requested]
//   CSR branch:    CSR scan of all planes  ->  CSR SpMM with the weight tile
//                  held in shared memory across all planes
#include "spk_common.cuh"

namespace spk {

struct SlLayout {
  size_t csr_state;     // look-back state of the CSR scan (cleared every call)
  size_t blk_sum;       // spikes per 128-row block (dense path; cleared every call)
  size_t sup_sum;       // spikes per 16384-row super-block
  size_t zero_end;      // [csr_state, zero_end) is cleared by the weight-image kernel
  size_t img;           // W image (dense branch)
  size_t bitmap;        // packed spikes [T*M][ceil(K/32)] written by the dense kernel for the scan
  size_t row_cnt;       // spikes per row [T*M]
  size_t csr_rowptr;    // internal CSR when the caller did not ask for it (CSR branch)
  size_t csr_planeptr;
  size_t csr_cols;
  int64_t csr_capacity;
  size_t gate;          // GateWords of the automatic choice
  size_t total;
};

// ---------------------------------------------------------------- automatic branch choice
// Cost model of the two branches on one B200, from the density sweep and the
// isolated spike-linear measurements of bench.py (rates of whole launches):
//   dense:  max(HBM bytes / 2.8 TB/s, 2*R*K*N / R_tc), R_tc = 500 TFLOP/s for
//           bf16 W (one bf16 pass), 290 TFLOP/s for fp32 W (two tf32 passes);
//   CSR:    the scan reads S at 3.3 TB/s, the SpMM writes Y at 5 TB/s and
//           performs nnz*N fused multiply-adds at F_csr per second.
// The CSR branch wins when nnz stays below nnz_limit = (t_dense - t_fixed) *
// F_csr / N.  The choice is made on the device, without a host round trip
// (the reference reads the density back with .item(), sparse/__init__.py:268-271).
constexpr double kDenseHbm = 2.8e12, kTcBf16 = 5.0e14, kTcTf32 = 2.9e14;
constexpr double kScanHbm = 3.3e12, kYHbm = 5.0e12;
constexpr double kCsrFmaBf16 = 7.0e12, kCsrFmaF32 = 4.2e12;

inline double csr_nnz_limit(int T, int64_t M, int K, int N, int w_dtype) {
  const double R = (double)T * (double)M;
  const double t_dense = fmax(4.0 * R * (K + N) / kDenseHbm, 2.0 * R * K * N / (w_dtype == SPK_BF16 ? kTcBf16 : kTcTf32));
  const double t_fixed = 4.0 * R * K / kScanHbm + 4.0 * R * N / kYHbm;
  return (t_dense - t_fixed) * (w_dtype == SPK_BF16 ? kCsrFmaBf16 : kCsrFmaF32) / (double)N;
}

// Words of the device-side choice in the workspace.
struct GateWords {
  int probe;                 // SPK_BRANCH_DENSE or kGateTryCsr (written by the probe)
  int final_branch;          // SPK_BRANCH_DENSE or SPK_BRANCH_CSR (probe, or the CSR scan's last tile)
  unsigned long long count;  // positives in the sampled rows
  unsigned int ticket;       // blocks of the probe that finished
};
constexpr int kProbeRows = 1024;

// Counts the positive values of n_rows rows of S spread over all planes (row
// i * stride), one warp per row; the last block to finish scales the count to
// the whole input and writes the probe word: clearly above the limit (twice
// it, far outside the sampling error) -> the dense branch at once, else the
// CSR scan counts exactly and decides.
__global__ void __launch_bounds__(256) density_probe_kernel(const float* S, int64_t R, int K, int64_t stride,
                                                            int n_rows, GateWords* g, double nnz_limit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  unsigned c = 0;
  if (row < n_rows) {
    const float* src = S + (int64_t)row * stride * K;
    for (int k = lane; k < K; k += 32) c += src[k] > 0.0f ? 1u : 0u;
  }
  c = __reduce_add_sync(0xffffffffu, c);
  if (lane == 0 && c) atomicAdd(&g->count, (unsigned long long)c);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(&g->ticket, 1u) == gridDim.x - 1) {
    __threadfence();
    const double est = (double)atomicAdd(&g->count, 0ull) * ((double)R / (double)n_rows);
    const bool dense = est > 2.0 * nnz_limit;
    g->probe = dense ? SPK_BRANCH_DENSE : kGateTryCsr;
    if (dense) g->final_branch = SPK_BRANCH_DENSE;
  }
}

inline int launch_density_probe(const float* S, int64_t R, int K, GateWords* g, double nnz_limit,
                                cudaStream_t stream) {
  SPK_CUDA_TRY(cudaMemsetAsync(g, 0, sizeof(GateWords), stream));
  const int n_rows = (int)min64(R, kProbeRows);
  const int64_t stride = R / n_rows;
  density_probe_kernel<<<(unsigned)ceil_div(n_rows, 8), 256, 0, stream>>>(S, R, K, stride, n_rows, g, nnz_limit);
  SPK_LAUNCH_CHECK();
  count_launch(1);
  return SPK_OK;
}

// Branch for this call; *gated = true when the choice is left to the device.
inline int resolve_branch(int branch, int T, int64_t M, int K, int N, int w_dtype, const void* S, bool* gated) {
  *gated = false;
  if (branch == SPK_BRANCH_DENSE || branch == SPK_BRANCH_CSR) return branch;
  if (!tc_supported(K, N, S)) return SPK_BRANCH_CSR;  // the tcgen05 path cannot take the shape
  const double limit = csr_nnz_limit(T, M, K, N, w_dtype);
  if (limit <= 0.0) return SPK_BRANCH_DENSE;  // the dense branch wins at any density
  if (limit >= (double)T * (double)M * (double)K) return SPK_BRANCH_CSR;
  *gated = true;
  return SPK_BRANCH_AUTO;
}

inline SlLayout sl_layout(int T, int64_t M, int K, int N, int w_dtype, bool internal_csr) {
  SlLayout L{};
  size_t off = 0;
  L.csr_state = off;
  off += align_up(csr_layout(T, M, K).total, 256);
  L.blk_sum = off;
  off += align_up(sizeof(int32_t) * (size_t)ceil_div((int64_t)T * M, 128), 256);
  L.sup_sum = off;
  off += align_up(sizeof(uint64_t) * (size_t)ceil_div((int64_t)T * M, 16384), 256);
  L.zero_end = off;
  L.img = off;
  {
    const TcPlan p = tc_plan(K, N, w_dtype);
    off += align_up(w_dtype == SPK_F32 ? tf32_img_bytes(p) : p.img_bytes, 1024);
  }
  L.bitmap = off;
  off += align_up(sizeof(uint32_t) * (size_t)T * M * (2 * ((K + 63) / 64)), 256);  // planar masks
  L.row_cnt = off;
  off += align_up(sizeof(int32_t) * (size_t)T * M, 256);
  if (internal_csr) {
    L.csr_rowptr = off;
    off += align_up(sizeof(int32_t) * (size_t)T * (M + 1), 256);
    L.csr_planeptr = off;
    off += align_up(sizeof(int64_t) * (size_t)(T + 1), 256);
    L.csr_cols = off;
    L.csr_capacity = (int64_t)T * M * K;
    off += align_up(sizeof(int32_t) * (size_t)L.csr_capacity, 256);
  }
  L.gate = off;
  off += align_up(sizeof(GateWords), 256);
  L.total = off;
  return L;
}

// The CSR branch: the scan builds the CSR of all planes (the caller's buffers,
// or the workspace's), then the SpMM.  Under the automatic choice (gw non-null)
// the scan runs only when the probe left the choice to it and writes the final
// branch from the exact spike count; the SpMM runs only when that is the CSR.
int csr_branch(const float* S, int T, int64_t M, int K, const void* W, int w_dtype, int64_t sk, int64_t sn, int N,
               const float* bias, float* Y, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx, float* values,
               int64_t* plane_ptr, int64_t col_capacity, bool internal_csr, const SlLayout& L, char* wsb,
               cudaStream_t stream, GateWords* gw, double nnz_limit) {
  int32_t* rp = row_ptr;
  int32_t* ci = col_idx;
  int64_t* pp = plane_ptr;
  int64_t cap = col_capacity;
  if (internal_csr) {
    rp = reinterpret_cast<int32_t*>(wsb + L.csr_rowptr);
    pp = reinterpret_cast<int64_t*>(wsb + L.csr_planeptr);
    ci = reinterpret_cast<int32_t*>(wsb + L.csr_cols);
    cap = L.csr_capacity;
  }
  CsrGate cg;
  if (gw) {
    cg.gate = &gw->probe;
    cg.gate_value = kGateTryCsr;
    cg.decide = &gw->final_branch;
    cg.decide_limit = (int64_t)fmin(nnz_limit, (double)cap);  // the CSR branch only when its CSR fits
  }
  const uint8_t* flags = nullptr;
  CsrLayout cl{};
  int rc = launch_csr_scan(S, T, M, K, nnz_row, rp, ci, values, pp, cap, wsb + L.csr_state, stream, &flags, &cl, cg);
  if (rc) return rc;
  return launch_spmm_csr(rp, pp, ci, values, S, flags, cl.rows_per_tile, cl.tiles_per_plane, W, w_dtype, sk, sn,
                         bias, Y, T, M, K, N, cap, stream, gw ? &gw->final_branch : nullptr);
}

int spike_linear_impl(const float* S, int T, int64_t M, int K, const void* W, int w_dtype, int64_t sk, int64_t sn,
                      int N, const float* bias, float* Y, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx,
                      float* values, int64_t* plane_ptr, int64_t col_capacity, int branch, void* ws,
                      size_t ws_bytes, cudaStream_t stream, const unsigned char* w_img = nullptr) {
  int rc = check_csr_shape(T, M, K);
  if (rc) return rc;
  SPK_REQUIRE(N >= 1, "N must be positive");
  SPK_REQUIRE(S && W && Y, "S, W and Y must be non-null");
  SPK_REQUIRE(w_dtype == SPK_F32 || w_dtype == SPK_BF16, "w_dtype must be SPK_F32 or SPK_BF16");
  const bool want_csr = row_ptr != nullptr || col_idx != nullptr || plane_ptr != nullptr;
  SPK_REQUIRE(!want_csr || (row_ptr && col_idx && plane_ptr), "CSR outputs need row_ptr, col_idx and plane_ptr");
  bool gated = false;
  branch = resolve_branch(branch, T, M, K, N, w_dtype, S, &gated);
  if (branch == SPK_BRANCH_DENSE || gated) {
    SPK_REQUIRE(tc_supported(K, N, S), "dense branch needs K %% 4 == 0 and a 16-byte aligned S");
    SPK_REQUIRE((int64_t)T * M < (int64_t(1) << 31), "dense branch: T*M must stay below 2^31 rows (TMA coordinates)");
  }
  const bool internal_csr = (branch == SPK_BRANCH_CSR || gated) && !want_csr;
  const SlLayout L = sl_layout(T, M, K, N, w_dtype, internal_csr);
  if (ws == nullptr || ws_bytes < L.total)
    return fail(SPK_EWORKSPACE, "workspace of %zu bytes required (got %zu)", L.total, ws_bytes);
  char* wsb = static_cast<char*>(ws);
  GateWords* gw = reinterpret_cast<GateWords*>(wsb + L.gate);
  double nnz_limit = 0.0;
  if (gated) {
    // automatic choice on the device: the probe, then both branches, each
    // of whose kernels returns at once unless the choice is its own
    nnz_limit = csr_nnz_limit(T, M, K, N, w_dtype);
    rc = launch_density_probe(S, (int64_t)T * M, K, gw, nnz_limit, stream);
    if (rc) return rc;
    rc = csr_branch(S, T, M, K, W, w_dtype, sk, sn, N, bias, Y, nnz_row, row_ptr, col_idx, values, plane_ptr,
                    col_capacity, internal_csr, L, wsb, stream, gw, nnz_limit);
    if (rc) return rc;
  }

  if (branch == SPK_BRANCH_DENSE || gated) {
    // w_image also clears the scan state (tile counter, look-back
    // descriptors, non-unit flag); the dense kernel writes the packed spike
    // bitmap and row counts; the scan expands them (no second read of S).
    const TcPlan p = tc_plan(K, N, w_dtype);
    unsigned char* img = reinterpret_cast<unsigned char*>(wsb + L.img);
    uint32_t* state = reinterpret_cast<uint32_t*>(wsb + L.csr_state);
    const int64_t zero_words = want_csr ? (int64_t)((L.zero_end - L.csr_state) / 4) : 0;
    // fp32 W: tf32 kernel (spikes read by the tensor cores straight from the
    // TMA staging); bf16 W: bf16 kernel (one MMA per k-step, no W split)
    const bool tf32 = w_dtype == SPK_F32;
    if (w_img != nullptr) {  // prepared by spk_weight_image: only the CSR pass state needs clearing
      img = const_cast<unsigned char*>(w_img);
      if (zero_words) SPK_CUDA_TRY(cudaMemsetAsync(state, 0, (size_t)zero_words * 4, stream));
    } else {
      rc = tf32 ? launch_w_image_tf32(W, sk, sn, K, N, p, img, want_csr ? state : nullptr, zero_words, stream)
                : launch_w_image(W, w_dtype, sk, sn, K, N, p, img, want_csr ? state : nullptr, zero_words, stream);
      if (rc) return rc;
    }
    TcOut o{bias, Y, nullptr, nullptr, nullptr, nullptr, nullptr};
    o.gate = gated ? &gw->final_branch : nullptr;
    o.early_s = w_img == nullptr ? 1 : 0;
    if (want_csr) {
      o.bitmap = reinterpret_cast<uint32_t*>(wsb + L.bitmap);
      o.row_cnt = reinterpret_cast<int32_t*>(wsb + L.row_cnt);
      o.blk_sum = reinterpret_cast<int32_t*>(wsb + L.blk_sum);
      o.sup_sum = reinterpret_cast<unsigned long long*>(wsb + L.sup_sum);
      // value check only when CSR values are requested (spikes of 1 need no gather)
      if (values) o.nonunit = reinterpret_cast<int*>(wsb + L.csr_state) + 1;  // ScanState::nonunit
    }
    // fp32 W with 128-column N tiles: weights in tensor memory (deeper S
    // ring); narrower N: the S-as-A tf32 kernel with an N tile of N
    if (tf32 && p.NT == 128) rc = launch_wt(S, (int64_t)T * M, K, N, p, img, o, stream);
    else if (tf32) rc = launch_tf32(S, (int64_t)T * M, K, N, p, img, o, stream);
    else rc = launch_tc(S, (int64_t)T * M, K, N, p, img, o, stream);
    if (rc) return rc;
    if (want_csr) {
      CsrGate cg;
      if (gated) {
        cg.gate = &gw->final_branch;
        cg.gate_value = SPK_BRANCH_DENSE;
      }
      rc = launch_csr_scan_ex(S, o.bitmap, o.row_cnt, o.blk_sum, o.sup_sum, true, T, M, K, nnz_row, row_ptr, col_idx, values, plane_ptr,
                              col_capacity, wsb + L.csr_state, stream, nullptr, nullptr, cg);
    }
    return rc;
  }
  return csr_branch(S, T, M, K, W, w_dtype, sk, sn, N, bias, Y, nnz_row, row_ptr, col_idx, values, plane_ptr,
                    col_capacity, internal_csr, L, wsb, stream, nullptr, 0.0);
}
}  // namespace spk

extern "C" size_t spk_spike_linear_workspace_bytes(int T, int64_t M, int K, int N, int w_dtype) {
  if (T < 1 || M < 1 || K < 1 || N < 1) return 0;
  // enough for either branch, including the CSR branch's internal CSR
  return spk::sl_layout(T, M, K, N, w_dtype, true).total;
}

extern "C" int spk_spike_linear(const float* S, int T, int64_t M, int K, const void* W, int w_dtype,
                                int64_t w_stride_k, int64_t w_stride_n, int N, const float* bias, float* Y,
                                int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx, float* values,
                                int64_t* plane_ptr, int64_t col_capacity, int branch, void* workspace,
                                size_t workspace_bytes, spk_stream_t stream) {
  return spk::spike_linear_impl(S, T, M, K, W, w_dtype, w_stride_k, w_stride_n, N, bias, Y, nnz_row, row_ptr,
                                col_idx, values, plane_ptr, col_capacity, branch, workspace, workspace_bytes,
                                (cudaStream_t)stream);
}

// ---------------------------------------------------------------- prepared weights
// The dense branch reads W through a weight image (tf32 hi + lo pieces for
// fp32 W, the bf16 K-major blocks for bf16 W), rebuilt from W on every call
// by default.  A caller whose weights do not change between calls (inference)
// builds it once and passes it to the *_img entry points.
extern "C" size_t spk_weight_image_bytes(int K, int N, int w_dtype) {
  if (K < 1 || N < 1 || (w_dtype != SPK_F32 && w_dtype != SPK_BF16)) return 0;
  const spk::TcPlan p = spk::tc_plan(K, N, w_dtype);
  return spk::align_up(w_dtype == SPK_F32 ? spk::tf32_img_bytes(p) : p.img_bytes, 1024);
}

extern "C" int spk_weight_image(const void* W, int w_dtype, int64_t w_stride_k, int64_t w_stride_n, int K, int N,
                                void* image, size_t image_bytes, spk_stream_t stream) {
  using namespace spk;
  SPK_REQUIRE(W && image, "W and image must be non-null");
  SPK_REQUIRE(K >= 1 && N >= 1, "bad shape K=%d N=%d", K, N);
  SPK_REQUIRE(w_dtype == SPK_F32 || w_dtype == SPK_BF16, "w_dtype must be SPK_F32 or SPK_BF16");
  const size_t need = spk_weight_image_bytes(K, N, w_dtype);
  if (image_bytes < need) return fail(SPK_EWORKSPACE, "weight image of %zu bytes required (got %zu)", need, image_bytes);
  SPK_REQUIRE((reinterpret_cast<uintptr_t>(image) & 1023) == 0, "the weight image must be 1024-byte aligned");
  const TcPlan p = tc_plan(K, N, w_dtype);
  unsigned char* img = static_cast<unsigned char*>(image);
  cudaStream_t st = (cudaStream_t)stream;
  return w_dtype == SPK_F32 ? launch_w_image_tf32(W, w_stride_k, w_stride_n, K, N, p, img, nullptr, 0, st)
                            : launch_w_image(W, w_dtype, w_stride_k, w_stride_n, K, N, p, img, nullptr, 0, st);
}

extern "C" int spk_spike_linear_img(const float* S, int T, int64_t M, int K, const void* W, int w_dtype,
                                    int64_t w_stride_k, int64_t w_stride_n, int N, const void* w_image,
                                    const float* bias, float* Y, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx,
                                    float* values, int64_t* plane_ptr, int64_t col_capacity, int branch,
                                    void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  SPK_REQUIRE(w_image == nullptr || (reinterpret_cast<uintptr_t>(w_image) & 1023) == 0,
              "the weight image must be 1024-byte aligned");
  return spk::spike_linear_impl(S, T, M, K, W, w_dtype, w_stride_k, w_stride_n, N, bias, Y, nnz_row, row_ptr,
                                col_idx, values, plane_ptr, col_capacity, branch, workspace, workspace_bytes,
                                (cudaStream_t)stream, static_cast<const unsigned char*>(w_image));
}

extern "C" size_t spk_sparse_forward_workspace_bytes(int T, int64_t B, int I, int O) {
  if (T < 1 || B < 1 || I < 1 || O < 1) return 0;
  return spk_spike_linear_workspace_bytes(T, B, I, O, SPK_F32) + 1024;
}

// The reference ops leave the CSR of plane T-1 in the caller's buffers: the
// product runs over all planes, then the last plane's CSR is written into
// nnz_per_row / row_offsets / col_indices / values.
static int reference_multistep(const float* x, int T, int64_t B, int I, const float* weightT, int O,
                               int32_t* nnz_per_row, int32_t* row_offsets, int32_t* col_indices, float* values,
                               int64_t col_capacity, float* out, int branch, void* ws, size_t ws_bytes,
                               cudaStream_t stream) {
  int rc = spk::check_csr_shape(T, B, I);
  if (rc) return rc;
  SPK_REQUIRE(x && weightT && out, "input, weightT and output must be non-null");
  SPK_REQUIRE(nnz_per_row && row_offsets && col_indices && values, "CSR buffers must be non-null");
  SPK_REQUIRE(O >= 1, "O must be positive");
  const size_t need = spk_sparse_forward_workspace_bytes(T, B, I, O);
  if (ws == nullptr || ws_bytes < need) return spk::fail(SPK_EWORKSPACE, "workspace of %zu bytes required", need);
  // plane pointer pair of the last plane lives at the end of the workspace
  int64_t* pp = reinterpret_cast<int64_t*>(static_cast<char*>(ws) + need - 1024);
  rc = spk::spike_linear_impl(x, T, B, I, weightT, SPK_F32, O, 1, O, nullptr, out, nullptr, nullptr, nullptr,
                              nullptr, nullptr, 0, branch, ws, need - 1024, stream);
  if (rc) return rc;
  const float* last = x + (int64_t)(T - 1) * B * I;
  return spk::launch_csr_scan(last, 1, B, I, nnz_per_row, row_offsets, col_indices, values, pp, col_capacity, ws,
                              stream, nullptr, nullptr);
}

extern "C" int spk_sparse_forward(const float* input, int64_t B, int I, const float* weightT, int O,
                                  int32_t* nnz_per_row, int32_t* row_offsets, int32_t* col_indices, float* values,
                                  int64_t col_capacity, float* output, int branch, void* workspace,
                                  size_t workspace_bytes, spk_stream_t stream) {
  return reference_multistep(input, 1, B, I, weightT, O, nnz_per_row, row_offsets, col_indices, values,
                             col_capacity, output, branch, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int spk_sparse_multistep_forward(const float* dense_input, int T, int64_t B, int I,
                                            const float* weightT, int O, int32_t* nnz_per_row,
                                            int32_t* row_offsets, int32_t* col_indices, float* values,
                                            int64_t col_capacity, float* output, int branch, void* workspace,
                                            size_t workspace_bytes, spk_stream_t stream) {
  return reference_multistep(dense_input, T, B, I, weightT, O, nnz_per_row, row_offsets, col_indices, values,
                             col_capacity, output, branch, workspace, workspace_bytes, (cudaStream_t)stream);
}

// ------------------------------------------------------------ linear + activation
// Y = act(X W^T + bias) for the projections around the path (the SpikingFFN
// fc1 with its threshold spike, attention.py:156; the q/k/v spikes and the
// o_proj of the attention, attention.py:110-118, 136).  fp32-accurate on the
// tensor cores: W tf32 hi + lo, X rounded to tf32 in shared memory with its
// remainder in a second pass (~2^-22 relative per product, as fp32).
extern "C" size_t spk_linear_act_workspace_bytes(int K, int N) {
  if (K < 1 || N < 1) return 0;
  return spk::align_up(spk::tf32_img_bytes(spk::tc_plan(K, N, SPK_F32)), 1024);
}

static int linear_act_impl(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k, int64_t w_stride_n,
                           int N, const void* w_image, const float* bias, int act, float thr, float* Y, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream);

extern "C" int spk_linear_act(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k,
                              int64_t w_stride_n, int N, const float* bias, int act, float thr, float* Y,
                              void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  return linear_act_impl(X, R, K, W, w_stride_k, w_stride_n, N, nullptr, bias, act, thr, Y, workspace,
                         workspace_bytes, (cudaStream_t)stream);
}

extern "C" int spk_linear_act_img(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k,
                                  int64_t w_stride_n, int N, const void* w_image, const float* bias, int act,
                                  float thr, float* Y, void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  SPK_REQUIRE(w_image == nullptr || (reinterpret_cast<uintptr_t>(w_image) & 1023) == 0,
              "the weight image must be 1024-byte aligned");
  return linear_act_impl(X, R, K, W, w_stride_k, w_stride_n, N, w_image, bias, act, thr, Y, workspace,
                         workspace_bytes, (cudaStream_t)stream);
}

static int linear_act_impl(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k, int64_t w_stride_n,
                           int N, const void* w_image, const float* bias, int act, float thr, float* Y, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream) {
  using namespace spk;
  SPK_REQUIRE(R >= 0 && K >= 1 && N >= 1, "bad shape R=%lld K=%d N=%d", (long long)R, K, N);
  SPK_REQUIRE(R < (int64_t(1) << 31), "linear_act: at most 2^31 - 1 rows per call (TMA row coordinates)");
  SPK_REQUIRE(W && (R == 0 || (X && Y)), "X, W and Y must be non-null");
  SPK_REQUIRE(act >= SPK_ACT_NONE && act <= SPK_ACT_VSPIKE_BITS, "unknown activation %d", act);
  SPK_REQUIRE((act != SPK_ACT_HEAVISIDE_BITS && act != SPK_ACT_VSPIKE_BITS) || N % 32 == 0,
              "packed spikes need N %% 32 == 0 (N=%d)", N);
  SPK_REQUIRE(N > 64, "linear_act needs N > 64 (128-column tiles on the tensor cores)");
  SPK_REQUIRE(K % 4 == 0 && (R == 0 || tc_supported(K, N, X)), "linear_act needs K %% 4 == 0 and a 16-byte aligned X");
  const TcPlan p = tc_plan(K, N, SPK_F32);
  const size_t need = align_up(tf32_img_bytes(p), 1024);
  if (w_image == nullptr && (workspace == nullptr || workspace_bytes < need))
    return fail(SPK_EWORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  if (R == 0) return SPK_OK;
  unsigned char* img = static_cast<unsigned char*>(workspace);
  cudaStream_t st = stream;
  if (w_image != nullptr) {
    img = static_cast<unsigned char*>(const_cast<void*>(w_image));
  } else {
    int rc = launch_w_image_tf32(W, w_stride_k, w_stride_n, K, N, p, img, nullptr, 0, st);
    if (rc) return rc;
  }
  TcOut o{bias, Y, nullptr, nullptr, nullptr, nullptr, nullptr};
  o.early_s = w_image == nullptr ? 1 : 0;
  return launch_wt(X, R, K, N, p, img, o, st, act, thr);
}

extern "C" int spk_spike_linear_bits(const uint32_t* bits, int T, int64_t M, int K, const float* W, int64_t w_stride_k,
                                     int64_t w_stride_n, int N, const void* w_image, const float* bias, float* Y,
                                     void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  using namespace spk;
  SPK_REQUIRE(T >= 1 && M >= 0 && K >= 1 && N >= 1, "bad shape T=%d M=%lld K=%d N=%d", T, (long long)M, K, N);
  const int64_t R = (int64_t)T * M;
  SPK_REQUIRE(R < (int64_t(1) << 31), "packed spike-linear: at most 2^31 - 1 rows per call");
  SPK_REQUIRE(W && (R == 0 || (bits && Y)), "bits, W and Y must be non-null");
  SPK_REQUIRE(K % 64 == 0, "packed spikes need K %% 64 == 0 (K=%d)", K);
  SPK_REQUIRE(N > 64, "packed spike-linear needs N > 64 (128-column tiles on the tensor cores)");
  SPK_REQUIRE((reinterpret_cast<uintptr_t>(bits) & 3) == 0, "bits must be 4-byte aligned");
  SPK_REQUIRE(w_image == nullptr || (reinterpret_cast<uintptr_t>(w_image) & 1023) == 0,
              "the weight image must be 1024-byte aligned");
  const TcPlan p = tc_plan(K, N, SPK_F32);
  const size_t need = align_up(tf32_img_bytes(p), 1024);
  if (w_image == nullptr && (workspace == nullptr || workspace_bytes < need))
    return fail(SPK_EWORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  if (R == 0) return SPK_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned char* img = static_cast<const unsigned char*>(w_image);
  if (img == nullptr) {
    unsigned char* wimg = static_cast<unsigned char*>(workspace);
    int rc = launch_w_image_tf32(W, w_stride_k, w_stride_n, K, N, p, wimg, nullptr, 0, st);
    if (rc) return rc;
    img = wimg;
  }
  TcOut o{bias, Y, nullptr, nullptr, nullptr, nullptr, nullptr};
  o.early_s = w_image == nullptr ? 1 : 0;
  return launch_wt_bits(bits, R, K, N, p, img, o, st);
}
