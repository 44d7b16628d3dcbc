/*
 * spikestack_b200.h -- C ABI of the B200 (sm_100a) engine for the temporal
 * forward hot path of SpikeStack Lite's SpikingTransformer.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream,
 * launches asynchronously on that stream and returns SPK_OK or an error code;
 * spk_last_error() gives the message of the last failure on the calling host
 * thread.  Nothing here allocates device memory: scratch space is a caller-
 * owned "workspace" whose size the matching *_workspace_bytes() query gives.
 * A workspace needs no initialisation and holds nothing between calls (the
 * CSR scan clears its own counters with a stream-ordered memset), so one
 * buffer may serve every entry point.  Calls that share one workspace must
 * not overlap on the GPU (issue them on one stream).
 *
 * Layouts are row-major and contiguous unless a stride argument says
 * otherwise.  A "plane" is one time step t of a [T, M, K] spike tensor.
 *
 * The reference interface each entry point replaces is cited as
 * file:line within the reference project (Griffith-7/spikestack-lite).
 */
#ifndef SPIKESTACK_B200_H
#define SPIKESTACK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* spk_stream_t; /* identical to cudaStream_t */

/* status codes */
enum {
  SPK_OK = 0,
  SPK_EINVAL = 1,        /* bad argument (shape, pointer, alignment, dtype) */
  SPK_EUNSUPPORTED = 2,  /* valid request the library does not implement */
  SPK_ECUDA = 3,         /* CUDA runtime error (launch or attribute) */
  SPK_EWORKSPACE = 4,    /* workspace missing or too small */
  SPK_EDEVICE = 5        /* a kernel reported a device-side error (spk_device_error) */
};

/* weight element types */
enum { SPK_F32 = 0, SPK_BF16 = 1 };

/* spike-linear branch selection */
enum {
  SPK_BRANCH_AUTO = 0,  /* dense tcgen05 branch above the density crossover, CSR branch below */
  SPK_BRANCH_DENSE = 1, /* tcgen05 / TMEM dense contraction (bf16 hi/lo split of fp32 operands) */
  SPK_BRANCH_CSR = 2    /* sparse branch: exact fp32 sums in ascending column order */
};

/* device error bits (spk_device_error) */
enum {
  SPK_DEV_PIPE_TIMEOUT = 1,    /* an mbarrier wait in a pipelined kernel ran out of time */
  SPK_DEV_SCAN_TIMEOUT = 2,    /* a look-back wait of the CSR scan ran out of time */
  SPK_DEV_CSR_OVERFLOW = 4,    /* the CSR column buffer was smaller than nnz */
  SPK_DEV_TMEM = 8             /* TMEM allocation returned an unusable address */
};

/* ------------------------------------------------------------------ misc */
const char* spk_last_error(void);
int spk_version(void);
/* Reads (and with clear != 0 resets) the device error word of the current
 * device.  Synchronizes the device. */
int spk_device_error(int clear, int* out_bits);
/* Diagnostic for SPK_DEV_PIPE_TIMEOUT: where the first timed-out pipeline
 * wait gave up since the last clearing spk_device_error call, as
 * block << 40 | warp << 32 | shared-memory address of the mbarrier (0 when no
 * wait timed out).  Synchronizes the device. */
int spk_timeout_site(uint64_t* out_site);
/* Self-test of the failure detection: launches one thread that waits on an
 * mbarrier nothing completes; after the wait's bound (2 s) the kernel records
 * SPK_DEV_PIPE_TIMEOUT and its site (spk_device_error, spk_timeout_site) and
 * exits, leaving the context usable.  No reference counterpart. */
int spk_selftest_wait_timeout(spk_stream_t stream);
/* Number of this library's kernel launches issued so far from this process
 * (all threads, all devices).  Used to report gpu_launches. */
int64_t spk_launch_count(void);

/* Kernel-level timing: after spk_profile_begin(id), every launch of kernel
 * `id` is bracketed by CUDA events recorded on its own launch stream;
 * spk_profile_end() waits for them and returns the summed device time and the
 * number of launches, then stops profiling.  No reference counterpart (the
 * reference times whole steps with a host clock, bench.py:57-61). */
enum {
  SPK_KERNEL_DENSE = 1,     /* tcgen05 spike-linear */
  SPK_KERNEL_CSR_SCAN = 2,  /* spike -> CSR compaction */
  SPK_KERNEL_SPMM_CSR = 3,  /* CSR branch SpMM */
  SPK_KERNEL_ATTN_KV = 4,   /* attention pass 1 */
  SPK_KERNEL_ATTN_OUT = 5,  /* attention pass 2 */
  SPK_KERNEL_GSMC_STEP = 6, /* GSMC cell step */
  SPK_KERNEL_W_IMAGE = 7    /* weight split / swizzle */
};
int spk_profile_begin(int kernel_id);
int spk_profile_end(double* total_ms, int64_t* launches);

/* ------------------------------------------------------- spike -> CSR
 * Replaces the CSR build of the reference engine: csr_build_kernel,
 * scan_blocks_kernel/offscan_add_kernel and csr_compact_kernel
 * (spikestack_lite/sparse/src/sparse_linear.cu:251-369), generalised to T
 * planes in one launch and to any M (the reference's offset scan is wrong
 * above 65536 rows).
 *
 * For every plane t of S[T, M, K]: nnz_row[t*M + m] = #{k : S > 0};
 * row_ptr[t*(M+1) + m] = exclusive prefix of nnz_row within the plane
 * (row_ptr[t*(M+1)] = 0); the column indices of the nonzeros of plane t, in
 * ascending k per row, start at col_idx[plane_ptr[t]] and values[] (optional,
 * may be NULL) holds S at those positions.  plane_ptr[T] is the total nnz.
 * Positions >= col_capacity are not written and raise SPK_DEV_CSR_OVERFLOW.
 * nnz_row may be NULL. */
size_t spk_csr_workspace_bytes(int T, int64_t M, int K);
int spk_csr_compact(const float* S, int T, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr,
                    int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity, void* workspace,
                    size_t workspace_bytes, spk_stream_t stream);

/* The same compaction for callers that cannot allocate device memory (hosts
 * that own all device memory and give plugins no workspace, or serving loops
 * that forbid cudaMalloc after start-up): no workspace argument, the scan's
 * scratch lives in a fixed 1 MiB array inside the library, held by every GPU
 * that loads it.  No counterpart in the reference.  Limit: a problem fits
 * when spk_csr_workspace_bytes(T, M, K) <= 1 MiB (256 bytes of state + 9
 * bytes per row tile of up to 128 rows of one plane + 8 bytes per plane,
 * rounded up to 256: about 116 000 tiles with few planes); larger requests
 * return SPK_EWORKSPACE.  The first call on a device (and the first after its
 * context was reset) looks the array's device address up
 * (cudaGetSymbolAddress) and should come before any stream capture there.  All calls share the
 * array: calls that overlap on the GPU race, so issue them on one stream. */
int spk_csr_compact_noalloc(const float* S, int T, int64_t M, int K, int32_t* nnz_row, int32_t* row_ptr,
                            int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity,
                            spk_stream_t stream);

/* ------------------------------------------------------- spike-linear
 * Y[r, n] = sum_{k : S[r,k] > 0} S[r,k] * W[k, n]  (+ bias[n] when bias != NULL)
 * for the R = T*M rows of S[T, M, K]; Y is [T, M, N] fp32.  W element (k, n)
 * is at W[k*w_stride_k + n*w_stride_n] (the reference passes weightT, i.e.
 * w_stride_k = N, w_stride_n = 1; an nn.Linear weight [N, K] is
 * w_stride_k = 1, w_stride_n = K).  w_dtype is SPK_F32 or SPK_BF16.
 * The CSR outputs follow spk_csr_compact and are optional (all NULL = none).
 * Replaces the multistep loop of sparse_multistep_forward
 * (sparse_linear.cu:645-691) with one pass whose weight tiles are reused
 * across the T planes. */
size_t spk_spike_linear_workspace_bytes(int T, int64_t M, int K, int N, int w_dtype);
int spk_spike_linear(const float* S, int T, int64_t M, int K, const void* W, int w_dtype, int64_t w_stride_k,
                     int64_t w_stride_n, int N, const float* bias, float* Y, int32_t* nnz_row, int32_t* row_ptr,
                     int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity, int branch,
                     void* workspace, size_t workspace_bytes, spk_stream_t stream);

/* Prepared weights.  The dense branch reads W through a weight image (tf32
 * hi + lo pieces for fp32 W, K-major bf16 blocks for bf16 W) that
 * spk_spike_linear and spk_linear_act rebuild from W on every call.  A caller
 * whose weights stay fixed between calls (inference) builds the image once
 * with spk_weight_image (image: 1024-byte aligned, spk_weight_image_bytes
 * bytes) and passes it to the *_img variants, which skip the rebuild; W is
 * still read by the CSR branch.  w_image = NULL behaves as the plain entry
 * point.  No counterpart in the reference (its ops take weightT on every call,
 * sparse/__init__.py:148-162); it replaces the per-call weight transpose. */
size_t spk_weight_image_bytes(int K, int N, int w_dtype);
int spk_weight_image(const void* W, int w_dtype, int64_t w_stride_k, int64_t w_stride_n, int K, int N, void* image,
                     size_t image_bytes, spk_stream_t stream);
int spk_spike_linear_img(const float* S, int T, int64_t M, int K, const void* W, int w_dtype, int64_t w_stride_k,
                         int64_t w_stride_n, int N, const void* w_image, const float* bias, float* Y, int32_t* nnz_row,
                         int32_t* row_ptr, int32_t* col_idx, float* values, int64_t* plane_ptr, int64_t col_capacity,
                         int branch, void* workspace, size_t workspace_bytes, spk_stream_t stream);

/* Reference-compatible ops.  Same arguments and results as the reference's
 * pybind ops sparse_forward (sparse_linear.cu:594-631) and
 * sparse_multistep_forward (sparse_linear.cu:645-691): input [B, I] /
 * [T, B, I], weightT [I, O], output [B, O] / [T, B, O]; the caller's CSR
 * buffers (nnz_per_row[B], row_offsets[B+1], col_indices/values of capacity
 * col_capacity >= nnz) receive the CSR of plane T-1 (the only plane the
 * reference leaves in them). */
size_t spk_sparse_forward_workspace_bytes(int T, int64_t B, int I, int O);
int spk_sparse_forward(const float* input, int64_t B, int I, const float* weightT, int O, int32_t* nnz_per_row,
                       int32_t* row_offsets, int32_t* col_indices, float* values, int64_t col_capacity,
                       float* output, int branch, void* workspace, size_t workspace_bytes, spk_stream_t stream);
int spk_sparse_multistep_forward(const float* dense_input, int T, int64_t B, int I, const float* weightT, int O,
                                 int32_t* nnz_per_row, int32_t* row_offsets, int32_t* col_indices, float* values,
                                 int64_t col_capacity, float* output, int branch, void* workspace,
                                 size_t workspace_bytes, spk_stream_t stream);

/* ------------------------------------------------------- linear + activation
 * Y[r, n] = act(sum_k X[r, k] * W[k, n] + bias[n]) for X [R, K] fp32 row-major,
 * W element (k, n) at W[k*w_stride_k + n*w_stride_n] (an nn.Linear weight
 * [N, K]: w_stride_k = 1, w_stride_n = K), bias optional, Y [R, N] fp32:
 *   SPK_ACT_NONE       y
 *   SPK_ACT_HEAVISIDE  1 if y - thr > 0 else 0  (spike_fn(fc1(x) - threshold),
 *                      attention.py:156; q, k spikes with thr = 0, :110-111)
 *   SPK_ACT_VSPIKE     1 if (tanh(y) + 1) / 2 - thr > 0 else 0  (the v spikes
 *                      with thr = tau[0], attention.py:112-115)
 * fp32-accurate on the tensor cores (tf32 hi/lo splits of W and X).  Needs
 * N > 64, K % 4 == 0 and a 16-byte aligned X.  Replaces the nn.Linear +
 * threshold + Heaviside pairs around the spike-linear path. */
enum { SPK_ACT_NONE = 0, SPK_ACT_HEAVISIDE = 1, SPK_ACT_VSPIKE = 2, SPK_ACT_HEAVISIDE_BITS = 3, SPK_ACT_VSPIKE_BITS = 4 };
/* SPK_ACT_HEAVISIDE_BITS: the Heaviside spikes of SPK_ACT_HEAVISIDE packed one
 * bit each, Y read as uint32 [R][N/32] (bit b of word w of a row = column
 * 32w + b; N % 32 == 0): 32x fewer bytes than the fp32 spike tensor for the
 * layer that consumes them (spk_spike_linear_bits).  Replaces the dense fp32
 * act tensor of SpikingFFN (attention.py:156), which the reference writes
 * and fc2 reads back.  SPK_ACT_VSPIKE_BITS packs the SPK_ACT_VSPIKE spikes the
 * same way (the attention's v, attention.py:114-115; q and k use
 * SPK_ACT_HEAVISIDE_BITS with thr 0) for spk_spiking_attention_bits. */
size_t spk_linear_act_workspace_bytes(int K, int N);
int spk_linear_act(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k, int64_t w_stride_n, int N,
                   const float* bias, int act, float thr, float* Y, void* workspace, size_t workspace_bytes,
                   spk_stream_t stream);
/* Spike-linear over packed spikes: bits [T*M][K/32] as written by
 * SPK_ACT_HEAVISIDE_BITS (K % 64 == 0), fp32 W with strides as for
 * spk_spike_linear (N > 64), Y [T, M, N] fp32 = S W (+ bias), bit-identical to
 * spk_spike_linear's dense branch on the unpacked spikes.  w_image: optional,
 * from spk_weight_image; the workspace (spk_linear_act_workspace_bytes(K, N)
 * bytes) may be NULL with an image.  The fc2 of SpikingFFN
 * (attention.py:158) on fc1's packed spikes. */
int spk_spike_linear_bits(const uint32_t* bits, int T, int64_t M, int K, const float* W, int64_t w_stride_k,
                          int64_t w_stride_n, int N, const void* w_image, const float* bias, float* Y,
                          void* workspace, size_t workspace_bytes, spk_stream_t stream);
/* spk_linear_act with a weight image prepared by spk_weight_image (fp32 W);
 * the workspace may then be NULL. */
int spk_linear_act_img(const float* X, int64_t R, int K, const float* W, int64_t w_stride_k, int64_t w_stride_n,
                       int N, const void* w_image, const float* bias, int act, float thr, float* Y, void* workspace,
                       size_t workspace_bytes, spk_stream_t stream);

/* ------------------------------------------------------- attention
 * apply_channel_decay (attention_cuda.cu:7-77, attention.py:30-44):
 * k_w[b, n, c] = k[b, n, c] * lam[c]^(N-1-n) over k [B_total, N, d]. */
int spk_apply_channel_decay(const float* k, const float* lam, int64_t B_total, int N, int d, float* k_w,
                            spk_stream_t stream);
/* fused_normalize_attention (attention_cuda.cu:29-107): out = numer / (denom + eps),
 * elementwise over `total` elements. */
int spk_normalize_attention(const float* numer, const float* denom, int64_t total, float eps, float* out,
                            spk_stream_t stream);
/* Spiking linear attention, the middle of AstrocyteHebbianAttention.forward
 * (attention.py:120-135): q, k, v are [BT, L, H*dh] spike tensors in d_model
 * layout (channel c = h*dh + j), lam [H*dh].  Per (bt, h):
 *   k_w[n, j] = k[n, c] * lam[c]^(L-1-n),  kv = k_w^T v,  key_mass = sum_n k_w,
 *   out[n, c'] = (q kv)[n, j'] / ((q key_mass)[n] + eps),
 * written back in d_model layout [BT, L, H*dh] (the o_proj input). */
size_t spk_attention_workspace_bytes(int64_t BT, int L, int H, int dh);
int spk_spiking_attention(const float* q, const float* k, const float* v, const float* lam, int64_t BT, int L,
                          int H, int dh, float eps, float* out, void* workspace, size_t workspace_bytes,
                          spk_stream_t stream);
/* The same over packed spikes: q_bits, k_bits, v_bits uint32 [BT*L][d/32]
 * (bit b of word w = channel 32w + b, as SPK_ACT_HEAVISIDE_BITS /
 * SPK_ACT_VSPIKE_BITS write them), 32x fewer input bytes; out as above,
 * bit-identical to spk_spiking_attention on the unpacked spikes.  Needs
 * d % 128 == 0 and dh in {16, 32, 64}; workspace as spk_attention_workspace_bytes.
 * Replaces the three fp32 spike tensors between the reference's q/k/v
 * projections and its attention (attention.py:110-117). */
int spk_spiking_attention_bits(const uint32_t* q_bits, const uint32_t* k_bits, const uint32_t* v_bits,
                               const float* lam, int64_t BT, int L, int H, int dh, float eps, float* out,
                               void* workspace, size_t workspace_bytes, spk_stream_t stream);

/* ------------------------------------------------------- GSMC
 * fused_gsmc_step (gsmc_cuda.cu:11-127): one cell step over M rows of width d;
 * gi, gr [M, 4d] (gate order f, i, o, g), wd [M, d], bias [4d]; m, s, heat
 * [M, d] are updated in place and out_t [M, d] receives the new spikes. */
int spk_gsmc_step(const float* gi, const float* gr, const float* wd, const float* bias, float* m, float* s,
                  float* heat, float* out_t, int64_t M, int d, float v_th, float gate_scale, int adaptive,
                  float beta, spk_stream_t stream);
/* The whole recurrence of FusedGSMC.forward in eval mode (gsmc.py:96-148)
 * given the batched input projections gi_all [T, M, 4d] (= W_in x, bias
 * included) and wd_all [T, M, d]: zero state, for each t the recurrent
 * projection gr = W_rec s_{t-1} (w_rec is the nn.Linear weight [4d, d]) and the
 * cell step.  out_all [T, M, d] (optional) receives every step's spikes and
 * pooled [M, d] their mean over T (pool_mean != 0) or the last step. */
size_t spk_gsmc_workspace_bytes(int64_t M, int d);
/* Forms of the recurrence for spk_gsmc_forward_ex.  SPK_GSMC_TWO_KERNEL (the
 * default of spk_gsmc_forward): per plane gr = W_rec s_{t-1} through the
 * spike-linear dense branch, then the step kernel.  SPK_GSMC_FUSED: one
 * tensor-core kernel per plane with the gates, state update and pooling in
 * its epilogue (gr stays on chip; d % 32 == 0, else the two-kernel form);
 * bit-identical results.  No counterpart in the reference (its loop,
 * gsmc.py:119-142, runs W_rec then fused_gsmc_step). */
enum { SPK_GSMC_TWO_KERNEL = 0, SPK_GSMC_FUSED = 1 };
int spk_gsmc_forward_ex(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias, int T,
                        int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta, int pool_mean,
                        float* out_all, float* pooled, void* workspace, size_t workspace_bytes, int form,
                        spk_stream_t stream);
int spk_gsmc_forward(const float* gi_all, const float* wd_all, const float* w_rec, const float* bias, int T,
                     int64_t M, int d, float v_th, float gate_scale, int adaptive, float beta, int pool_mean,
                     float* out_all, float* pooled, void* workspace, size_t workspace_bytes, spk_stream_t stream);

/* ------------------------------------------------------- residual add + layer norm
 * The pre-norm block's residual add and the layer norm of its result
 * (AstrocyteHebbianBlock.forward, nn/attention.py:174-177: x + attn(norm1(x)),
 * then norm2 of that sum; the block's output sum and the next block's norm1)
 * in one pass, per row of width d:
 *   H = X + D,  Y = (H - mean(H)) / sqrt(var(H) + eps) * gamma + beta,
 * with the biased variance of nn.LayerNorm.  D null: Y = LayerNorm(X) and H
 * is not written.  gamma / beta null: 1 / 0.  All pointers 16-byte aligned,
 * d % 4 == 0, d <= 1024 (SPK_EUNSUPPORTED above); H may alias X. */
int spk_add_layernorm(const float* X, const float* D, const float* gamma, const float* beta, int64_t rows, int d,
                      float eps, float* H, float* Y, spk_stream_t stream);

/* ------------------------------------------------------- Spire planes
 * The Spire encoder's temporal planes (SpireEncoder.forward, encode/spire.py:
 * 60-69; spire_dither_kernel, encode/src/spire_cuda.cu:7-58) from the
 * projection u [B, N, d]:
 *   v = (u - frontier[c]) - temporal_frontier[n],
 *   planes[t, b, n, c] = (v - dither[t] > 0) ? 1 : 0   for t < T,
 * planes [T, B, N, d] contiguous.  frontier [d] and temporal_frontier [N] may be
 * null (the term is then left out: spire_dither(v, dither) of the reference
 * engine).  d % 4 == 0; u, planes and frontier 16-byte aligned. */
int spk_spire_planes(const float* u, const float* frontier, const float* temporal_frontier, const float* dither,
                     int T, int64_t B, int N, int d, float* planes, spk_stream_t stream);

/* ------------------------------------------------------- readout pooling
 * The pooling before SpikingTransformer's classifier (models/transformer.py:
 * 159-192): over x [T, B, N, d] (T = 1 for the GSMC-pooled [B, N, d]), per
 * sample b and channel c, mean_x[b, c] = mean over (t, n) of x and
 * mean_spike[b, c] = mean over (t, n) of (x > 0), each (sum) * (1 / (T N)) as
 * torch's mean; either output may be null.  d % 4 == 0, T*N < 2^24, tensors
 * 16-byte aligned. */
int spk_temporal_mean(const float* x, int T, int64_t B, int N, int d, float* mean_x, float* mean_spike,
                      spk_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SPIKESTACK_B200_H */
