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
  size_t total;
};

inline int resolve_branch(int branch, int K, int N, const void* S) {
  if (branch == SPK_BRANCH_DENSE || branch == SPK_BRANCH_CSR) return branch;
  // Dense unless the tcgen05 path cannot take the shape.  The dense branch is
  // HBM-bound for the narrow layers of the model (N <= 512) at any density,
  // so it never loses there; the CSR branch only wins on wide layers at very
  // low density, which a caller selects explicitly.
  return tc_supported(K, N, S) ? SPK_BRANCH_DENSE : SPK_BRANCH_CSR;
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
  L.total = off;
  return L;
}

int spike_linear_impl(const float* S, int T, int64_t M, int K, const void* W, int w_dtype, int64_t sk, int64_t sn,
                      int N, const float* bias, float* Y, int32_t* nnz_row, int32_t* row_ptr, int32_t* col_idx,
                      float* values, int64_t* plane_ptr, int64_t col_capacity, int branch, void* ws,
                      size_t ws_bytes, cudaStream_t stream) {
  int rc = check_csr_shape(T, M, K);
  if (rc) return rc;
  SPK_REQUIRE(N >= 1, "N must be positive");
  SPK_REQUIRE(S && W && Y, "S, W and Y must be non-null");
  SPK_REQUIRE(w_dtype == SPK_F32 || w_dtype == SPK_BF16, "w_dtype must be SPK_F32 or SPK_BF16");
  const bool want_csr = row_ptr != nullptr || col_idx != nullptr || plane_ptr != nullptr;
  SPK_REQUIRE(!want_csr || (row_ptr && col_idx && plane_ptr), "CSR outputs need row_ptr, col_idx and plane_ptr");
  branch = resolve_branch(branch, K, N, S);
  if (branch == SPK_BRANCH_DENSE) {
    SPK_REQUIRE(tc_supported(K, N, S), "dense branch needs K %% 4 == 0 and a 16-byte aligned S");
    SPK_REQUIRE((int64_t)T * M < (int64_t(1) << 31), "dense branch: T*M must stay below 2^31 rows (TMA coordinates)");
  }
  const bool internal_csr = (branch == SPK_BRANCH_CSR) && !want_csr;
  const SlLayout L = sl_layout(T, M, K, N, w_dtype, internal_csr);
  if (ws == nullptr || ws_bytes < L.total)
    return fail(SPK_EWORKSPACE, "workspace of %zu bytes required (got %zu)", L.total, ws_bytes);
  char* wsb = static_cast<char*>(ws);

  if (branch == SPK_BRANCH_DENSE) {
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
    rc = tf32 ? launch_w_image_tf32(W, sk, sn, K, N, p, img, want_csr ? state : nullptr, zero_words, stream)
              : launch_w_image(W, w_dtype, sk, sn, K, N, p, img, want_csr ? state : nullptr, zero_words, stream);
    if (rc) return rc;
    TcOut o{bias, Y, nullptr, nullptr, nullptr, nullptr, nullptr};
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
      rc = launch_csr_scan_ex(S, o.bitmap, o.row_cnt, o.blk_sum, o.sup_sum, true, T, M, K, nnz_row, row_ptr, col_idx, values, plane_ptr,
                              col_capacity, wsb + L.csr_state, stream, nullptr, nullptr);
    }
    return rc;
  }
  // CSR branch
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
  const uint8_t* flags = nullptr;
  CsrLayout cl{};
  rc = launch_csr_scan(S, T, M, K, nnz_row, rp, ci, values, pp, cap, wsb + L.csr_state, stream, &flags, &cl);
  if (rc) return rc;
  return launch_spmm_csr(rp, pp, ci, values, S, flags, cl.rows_per_tile, cl.tiles_per_plane, W, w_dtype, sk, sn,
                         bias, Y, T, M, K, N, cap, stream);
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

extern "C" int spk_linear_act(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k,
                              int64_t w_stride_n, int N, const float* bias, int act, float thr, float* Y,
                              void* workspace, size_t workspace_bytes, spk_stream_t stream) {
  using namespace spk;
  SPK_REQUIRE(R >= 0 && K >= 1 && N >= 1, "bad shape R=%lld K=%d N=%d", (long long)R, K, N);
  SPK_REQUIRE(R < (int64_t(1) << 31), "linear_act: at most 2^31 - 1 rows per call (TMA row coordinates)");
  SPK_REQUIRE(W && (R == 0 || (X && Y)), "X, W and Y must be non-null");
  SPK_REQUIRE(act >= SPK_ACT_NONE && act <= SPK_ACT_VSPIKE, "unknown activation %d", act);
  SPK_REQUIRE(N > 64, "linear_act needs N > 64 (128-column tiles on the tensor cores)");
  SPK_REQUIRE(K % 4 == 0 && (R == 0 || tc_supported(K, N, X)), "linear_act needs K %% 4 == 0 and a 16-byte aligned X");
  const TcPlan p = tc_plan(K, N, SPK_F32);
  const size_t need = align_up(tf32_img_bytes(p), 1024);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(SPK_EWORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);
  if (R == 0) return SPK_OK;
  unsigned char* img = static_cast<unsigned char*>(workspace);
  cudaStream_t st = (cudaStream_t)stream;
  int rc = launch_w_image_tf32(W, w_stride_k, w_stride_n, K, N, p, img, nullptr, 0, st);
  if (rc) return rc;
  TcOut o{bias, Y, nullptr, nullptr, nullptr, nullptr, nullptr};
  return launch_wt(X, R, K, N, p, img, o, st, act, thr);
}
