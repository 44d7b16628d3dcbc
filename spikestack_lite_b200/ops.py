"""Tensor-level ops over the C ABI (torch tensors in, torch tensors out).

Every op validates its tensors (CUDA, float32, contiguous where the kernel
needs it), passes raw pointers and the current stream of the tensors' device
to libspk_b200.so and raises ``EngineError`` (a RuntimeError) on any failure.
"""
import weakref

import torch

from . import _lib
from ._lib import EngineError, check, ptr, require_cuda, require_f32, stream_of


def _branch(b):
    if isinstance(b, int):
        return b
    try:
        return _lib.BRANCHES[b]
    except KeyError:
        raise EngineError(f"unknown branch {b!r} (auto, dense or csr)") from None


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


# (op, rows, K, N) of every dense contraction issued while a tally is open
_TALLY = None


class tally:
    """Records (op, rows, K, N) of each tensor-core contraction the ops issue
    inside the ``with`` block -- spike_linear, linear_act and the recurrent
    projections of gsmc_forward -- so that a caller can count their
    algorithmic FLOPs (2 * rows * K * N each).  Bookkeeping only."""

    def __enter__(self):
        global _TALLY
        self.calls = []
        _TALLY = self.calls
        return self

    def __exit__(self, *exc):
        global _TALLY
        _TALLY = None
        return False

    def flops(self):
        return sum(2.0 * r * k * n for _, r, k, n in self.calls)


def _record(op, rows, K, N):
    if _TALLY is not None:
        _TALLY.append((op, int(rows), int(K), int(N)))


# ------------------------------------------------------------ prepared weights
# The dense branch reads W through a weight image (spk_weight_image) that the
# plain entry points rebuild from W on every call.  Weights that stay fixed
# between calls (inference) get theirs built once: the cache holds one image
# per live weight tensor, valid while the tensor object, its version counter
# (bumped by every in-place change), pointer, shape, strides and dtype are
# unchanged, and drops it when the tensor is freed.  A weight changed through
# `.data` escapes the version counter: call clear_weight_cache() after that.
_IMG = {}
_IMG_ENABLED = True


def set_weight_cache(enabled):
    """Turn the prepared-weight cache on or off (on by default)."""
    global _IMG_ENABLED
    _IMG_ENABLED = bool(enabled)
    if not _IMG_ENABLED:
        _IMG.clear()


def clear_weight_cache():
    _IMG.clear()


def _weight_image(W, K, N, sk, sn, wdt):
    """The cached weight image of W (a 1024-byte aligned uint8 view), or None
    (cache off, or a stream capture in progress: an image built there would
    hold nothing until the graph is replayed)."""
    if not _IMG_ENABLED:
        return None
    key = (W.data_ptr(), tuple(W.shape), tuple(W.stride()), W.dtype, int(sk), int(sn), int(K), int(N))
    ent = _IMG.get(id(W))
    if ent is not None:
        ref, ver, k, img = ent
        if ref() is W and ver == W._version and k == key:
            return img
    if torch.cuda.is_current_stream_capturing():
        return None
    lib = _lib.load()
    nbytes = int(lib.spk_weight_image_bytes(K, N, wdt))
    buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=W.device)
    off = (-buf.data_ptr()) % 1024
    img = buf[off:off + nbytes]
    check(lib.spk_weight_image(ptr(W), wdt, sk, sn, K, N, ptr(img), nbytes, stream_of(W)), "spk_weight_image")
    wid = id(W)
    _IMG[wid] = (weakref.ref(W, lambda _r, i=wid: _IMG.pop(i, None)), W._version, key, img)
    return img


# ----------------------------------------------------------------- spike -> CSR
def csr_compact(S, values=True, capacity=None):
    """Per-plane CSR of S [T, M, K] (or [M, K] as one plane).

    Returns a dict with nnz_row [T, M], row_ptr [T, M+1] (int32, relative to
    each plane), col_idx (int32, planes back to back), values (float32 or
    None) and plane_ptr [T+1] (int64).  One launch for all planes, into
    buffers of `capacity` entries (default T*M*K, enough for any input), then
    an 8-byte device->host read of the total to size the returned views."""
    require_cuda(S, what="csr_compact")
    require_f32(S, what="csr_compact")
    S = _contig(S)
    if S.dim() == 2:
        S = S.unsqueeze(0)
    T, M, K = S.shape
    lib = _lib.load()
    dev = S.device
    nnz_row = torch.empty(T, M, dtype=torch.int32, device=dev)
    row_ptr = torch.empty(T, M + 1, dtype=torch.int32, device=dev)
    plane_ptr = torch.empty(T + 1, dtype=torch.int64, device=dev)
    cap = int(capacity) if capacity is not None else T * M * K
    col_idx = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    vals = torch.empty(max(cap, 1), dtype=torch.float32, device=dev) if values else None
    ws, wsn = _lib.workspace(dev, lib.spk_csr_workspace_bytes(T, M, K))
    check(lib.spk_csr_compact(ptr(S), T, M, K, ptr(nnz_row), ptr(row_ptr), ptr(col_idx), ptr(vals),
                              ptr(plane_ptr), cap, ws, wsn, stream_of(S)), "spk_csr_compact")
    nnz = int(plane_ptr[T].item())
    if nnz > cap:
        raise EngineError(f"csr_compact: {nnz} spikes exceed the capacity of {cap}")
    return {"nnz_row": nnz_row, "row_ptr": row_ptr, "col_idx": col_idx[:nnz],
            "values": None if vals is None else vals[:nnz], "plane_ptr": plane_ptr}


# ------------------------------------------------------------------ spike-linear
def spike_linear(S, weight=None, weightT=None, bias=None, branch="auto", csr=None):
    """Y[..., n] = sum_{k: S[..., k] > 0} S[..., k] W[k, n] (+ bias) for S [T, M, K]
    (or [M, K]).  W is given either as an nn.Linear ``weight`` [N, K] or as
    ``weightT`` [K, N] (the reference op layout), float32 or bfloat16.

    ``csr``: None, or a dict with preallocated int32/int64 buffers
    {nnz_row [T*M], row_ptr [T*(M+1)], col_idx [cap], plane_ptr [T+1],
    values [cap] (optional)} that receive the per-plane CSR."""
    require_cuda(S, weight, weightT, bias, what="spike_linear")
    require_f32(S, bias, what="spike_linear")
    if (weight is None) == (weightT is None):
        raise EngineError("spike_linear: pass exactly one of weight [N, K] or weightT [K, N]")
    squeeze = S.dim() == 2
    S = _contig(S)
    if squeeze:
        S = S.unsqueeze(0)
    if S.dim() != 3:
        raise EngineError(f"spike_linear: S must be [T, M, K] or [M, K], got {tuple(S.shape)}")
    T, M, K = S.shape
    W = weight if weight is not None else weightT
    if W.dtype not in (torch.float32, torch.bfloat16):
        raise EngineError(f"spike_linear: weight dtype {W.dtype} not supported (float32 or bfloat16)")
    if weight is not None:
        N, Kw = weight.shape
        sk, sn = weight.stride(1), weight.stride(0)
    else:
        Kw, N = weightT.shape
        sk, sn = weightT.stride(0), weightT.stride(1)
    if Kw != K:
        raise EngineError(f"spike_linear: weight K={Kw} does not match input K={K}")
    if bias is not None:
        bias = _contig(bias)
        if bias.numel() != N:
            raise EngineError("spike_linear: bias must have N elements")
    wdt = _lib.SPK_BF16 if W.dtype == torch.bfloat16 else _lib.SPK_F32
    lib = _lib.load()
    Y = torch.empty(T, M, N, dtype=torch.float32, device=S.device)
    c = csr or {}
    cap = c["col_idx"].numel() if c else 0
    ws, wsn = _lib.workspace(S.device, lib.spk_spike_linear_workspace_bytes(T, M, K, N, wdt))
    _record("spike_linear", T * M, K, N)
    img = _weight_image(W, K, N, sk, sn, wdt) if _branch(branch) != _lib.BRANCH_CSR else None
    check(lib.spk_spike_linear_img(ptr(S), T, M, K, ptr(W), wdt, sk, sn, N, ptr(img), ptr(bias), ptr(Y),
                                   ptr(c.get("nnz_row")), ptr(c.get("row_ptr")), ptr(c.get("col_idx")),
                                   ptr(c.get("values")), ptr(c.get("plane_ptr")), cap, _branch(branch), ws, wsn,
                                   stream_of(S)), "spk_spike_linear")
    return Y[0] if squeeze else Y


_ACTS = {"none": 0, "heaviside": 1, "vspike": 2, "heaviside_bits": 3, "vspike_bits": 4}


def linear_act(x, weight, bias=None, act="none", thr=0.0):
    """act(x @ weight.T + bias) for x [..., K] fp32 and an nn.Linear weight
    [N, K] fp32 on the tensor cores, fp32-accurate (spk_linear_act):

      "none"       y
      "heaviside"  (y - thr > 0).float()               spike_fn(fc1(x) - thr); q, k spikes (thr 0)
      "vspike"     ((tanh(y) + 1) / 2 - thr > 0).float()  v spikes (thr = tau)
      "heaviside_bits"  the "heaviside" spikes packed 32 to an int32 word:
                   [..., N/32], bit b of word w = column 32w + b (N % 32 == 0)
      "vspike_bits"     the "vspike" spikes packed the same way

    Needs N > 64 and K % 4 == 0."""
    require_cuda(x, weight, bias, what="linear_act")
    require_f32(x, weight, bias, what="linear_act")
    if act not in _ACTS:
        raise EngineError(f"linear_act: act must be one of {sorted(_ACTS)}")
    x = _contig(x)
    K = x.shape[-1]
    N, Kw = weight.shape
    if Kw != K:
        raise EngineError(f"linear_act: weight K={Kw} does not match input K={K}")
    if bias is not None:
        bias = _contig(bias)
        if bias.numel() != N:
            raise EngineError("linear_act: bias must have N elements")
    R = x.numel() // K if K else 0
    if act in ("heaviside_bits", "vspike_bits"):
        if N % 32:
            raise EngineError(f"linear_act: packed spikes need N % 32 == 0 (N={N})")
        Y = torch.empty(*x.shape[:-1], N // 32, dtype=torch.int32, device=x.device)
    else:
        Y = torch.empty(*x.shape[:-1], N, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws, wsn = _lib.workspace(x.device, lib.spk_linear_act_workspace_bytes(K, N))
    _record("linear_act", R, K, N)
    img = _weight_image(weight, K, N, weight.stride(1), weight.stride(0), _lib.SPK_F32)
    check(lib.spk_linear_act_img(ptr(x), R, K, ptr(weight), weight.stride(1), weight.stride(0), N, ptr(img),
                                 ptr(bias), _ACTS[act], float(thr), ptr(Y), ws, wsn, stream_of(x)), "spk_linear_act")
    return Y


def engine_linear(lin, x, act="none", thr=0.0):
    """act(lin(x)) through the engine's fp32-accurate tensor-core linear
    (spk_linear_act) when autograd is off and the shape is one it takes
    (out_features > 64, in_features % 4 == 0); None otherwise, and the caller
    runs the module (the reference's own nn.Linear, which training needs)."""
    if torch.is_grad_enabled() or not x.is_cuda or lin.out_features <= 64 or lin.in_features % 4:
        return None
    return linear_act(x, lin.weight, lin.bias, act, thr)


def spike_linear_bits(bits, K, weight, bias=None):
    """Spike-linear over packed spikes: bits int32 [..., K/32] (bit b of word w
    = column 32w + b, as linear_act(act="heaviside_bits") writes them), an
    nn.Linear weight [N, K] fp32, optional bias -> [..., N] fp32; the same
    values as spike_linear(unpack_spikes(bits, K), weight, bias,
    branch="dense").  Needs K % 64 == 0 and N > 64."""
    require_cuda(bits, weight, bias, what="spike_linear_bits")
    require_f32(weight, bias, what="spike_linear_bits")
    if bits.dtype != torch.int32:
        raise EngineError(f"spike_linear_bits: bits must be int32, got {bits.dtype}")
    bits = _contig(bits)
    N, Kw = weight.shape
    if Kw != K or bits.shape[-1] * 32 != K:
        raise EngineError(f"spike_linear_bits: K={K}, weight K={Kw}, bits hold {bits.shape[-1] * 32} columns")
    if bias is not None:
        bias = _contig(bias)
        if bias.numel() != N:
            raise EngineError("spike_linear_bits: bias must have N elements")
    R = bits.numel() // bits.shape[-1]
    Y = torch.empty(*bits.shape[:-1], N, dtype=torch.float32, device=bits.device)
    lib = _lib.load()
    _record("spike_linear_bits", R, K, N)
    img = _weight_image(weight, K, N, weight.stride(1), weight.stride(0), _lib.SPK_F32)
    ws, wsn = (None, 0) if img is not None else _lib.workspace(bits.device, lib.spk_linear_act_workspace_bytes(K, N))
    check(lib.spk_spike_linear_bits(ptr(bits), 1, R, K, ptr(weight), weight.stride(1), weight.stride(0), N, ptr(img),
                                    ptr(bias), ptr(Y), ws, wsn, stream_of(bits)), "spk_spike_linear_bits")
    return Y


def unpack_spikes(bits, K):
    """fp32 0 / 1 spikes [..., K] from packed words [..., K/32] (inspection and
    tests; the engine consumes the packed form directly)."""
    shifts = torch.arange(32, device=bits.device, dtype=torch.int32)
    b = (bits.unsqueeze(-1) >> shifts) & 1
    return b.reshape(*bits.shape[:-1], bits.shape[-1] * 32)[..., :K].float()


def alloc_csr(T, M, K, device, capacity=None, values=False):
    """Preallocated per-plane CSR buffers for spike_linear(csr=...)."""
    cap = int(capacity if capacity is not None else T * M * K)
    d = {
        "nnz_row": torch.empty(T * M, dtype=torch.int32, device=device),
        "row_ptr": torch.empty(T * (M + 1), dtype=torch.int32, device=device),
        "col_idx": torch.empty(max(cap, 1), dtype=torch.int32, device=device),
        "plane_ptr": torch.empty(T + 1, dtype=torch.int64, device=device),
    }
    if values:
        d["values"] = torch.empty(max(cap, 1), dtype=torch.float32, device=device)
    return d


def sparse_multistep_forward(dense_input, weightT, nnz_per_row, row_offsets, col_indices, values, T,
                             branch="auto"):
    """The reference op (sparse_linear.cu:645-691): dense_input [T, B, I],
    weightT [I, O] -> [T, B, O]; the CSR buffers receive plane T-1's CSR."""
    require_cuda(dense_input, weightT, nnz_per_row, row_offsets, col_indices, values,
                 what="sparse_multistep_forward")
    require_f32(dense_input, weightT, values, what="sparse_multistep_forward")
    x = _contig(dense_input)
    T = int(T)
    if x.dim() != 3 or x.shape[0] != T:
        x = x.reshape(T, -1, x.shape[-1])
    _, B, I = x.shape
    wT = _contig(weightT)
    O = wT.shape[1]
    if wT.shape[0] != I:
        raise EngineError(f"sparse_multistep_forward: weightT has {wT.shape[0]} rows, input has {I} features")
    cap = min(col_indices.numel(), values.numel())
    out = torch.empty(T, B, O, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws, wsn = _lib.workspace(x.device, lib.spk_sparse_forward_workspace_bytes(T, B, I, O))
    check(lib.spk_sparse_multistep_forward(ptr(x), T, B, I, ptr(wT), O, ptr(nnz_per_row), ptr(row_offsets),
                                           ptr(col_indices), ptr(values), cap, ptr(out), _branch(branch), ws, wsn,
                                           stream_of(x)), "spk_sparse_multistep_forward")
    return out


def sparse_forward(input, weightT, nnz_per_row, row_offsets, col_indices, values, branch="auto"):
    """The reference op (sparse_linear.cu:594-631): input [B, I] -> [B, O]."""
    require_cuda(input, weightT, nnz_per_row, row_offsets, col_indices, values, what="sparse_forward")
    require_f32(input, weightT, values, what="sparse_forward")
    x = _contig(input)
    B, I = x.shape
    wT = _contig(weightT)
    O = wT.shape[1]
    if wT.shape[0] != I:
        raise EngineError(f"sparse_forward: weightT has {wT.shape[0]} rows, input has {I} features")
    cap = min(col_indices.numel(), values.numel())
    out = torch.empty(B, O, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws, wsn = _lib.workspace(x.device, lib.spk_sparse_forward_workspace_bytes(1, B, I, O))
    check(lib.spk_sparse_forward(ptr(x), B, I, ptr(wT), O, ptr(nnz_per_row), ptr(row_offsets), ptr(col_indices),
                                 ptr(values), cap, ptr(out), _branch(branch), ws, wsn, stream_of(x)),
          "spk_sparse_forward")
    return out


def dense_to_csr_gpu(dense_input):
    """The reference op dense_to_csr_gpu (sparse_linear.cu:563-588):
    [B, I] -> [row_offsets [B+1], col_indices [B*I], values [B*I]]."""
    require_cuda(dense_input, what="dense_to_csr_gpu")
    require_f32(dense_input, what="dense_to_csr_gpu")
    x = _contig(dense_input)
    B, I = x.shape
    dev = x.device
    row_ptr = torch.empty(B + 1, dtype=torch.int32, device=dev)
    col_idx = torch.empty(B * I, dtype=torch.int32, device=dev)
    vals = torch.empty(B * I, dtype=torch.float32, device=dev)
    plane_ptr = torch.empty(2, dtype=torch.int64, device=dev)
    lib = _lib.load()
    ws, wsn = _lib.workspace(dev, lib.spk_csr_workspace_bytes(1, B, I))
    check(lib.spk_csr_compact(ptr(x), 1, B, I, None, ptr(row_ptr), ptr(col_idx), ptr(vals), ptr(plane_ptr), B * I,
                              ws, wsn, stream_of(x)), "spk_csr_compact")
    return [row_ptr, col_idx, vals]


# ---------------------------------------------------------------------- attention
def apply_channel_decay(k, lam):
    """k_w = k * lam ** (N-1-n) (attention_cuda.cu:42-77)."""
    require_cuda(k, lam, what="apply_channel_decay")
    require_f32(k, lam, what="apply_channel_decay")
    if k.dim() < 2:
        raise EngineError("apply_channel_decay: k must have at least 2 dimensions")
    k = _contig(k)
    lam = _contig(lam)
    d, N = k.shape[-1], k.shape[-2]
    if lam.dim() != 1 or lam.numel() != d:
        raise EngineError("apply_channel_decay: lam must be 1D tensor of size d matching k.size(-1)")
    out = torch.empty_like(k)
    if k.numel() == 0:
        return out
    check(_lib.load().spk_apply_channel_decay(ptr(k), ptr(lam), k.numel() // (N * d), N, d, ptr(out), stream_of(k)),
          "spk_apply_channel_decay")
    return out


def fused_normalize_attention(numer, denom, eps):
    """numer / (denom + eps) elementwise (attention_cuda.cu:79-107)."""
    require_cuda(numer, denom, what="fused_normalize_attention")
    require_f32(numer, denom, what="fused_normalize_attention")
    if denom.numel() < numer.numel():
        raise EngineError("fused_normalize_attention: denom must have at least as many elements as numer")
    numer = _contig(numer)
    denom = _contig(denom)
    out = torch.empty_like(numer)
    check(_lib.load().spk_normalize_attention(ptr(numer), ptr(denom), numer.numel(), float(eps), ptr(out),
                                              stream_of(numer)), "spk_normalize_attention")
    return out


def spiking_attention(q, k, v, lam, heads, eps=1e-6):
    """Fused spiking linear attention: q, k, v spikes [..., L, d] (d = heads*dh)
    -> normalised attention [..., L, d] (the o_proj input of
    AstrocyteHebbianAttention, attention.py:120-135)."""
    require_cuda(q, k, v, lam, what="spiking_attention")
    require_f32(q, k, v, lam, what="spiking_attention")
    shape = q.shape
    L, d = shape[-2], shape[-1]
    if k.shape != shape or v.shape != shape:
        raise EngineError("spiking_attention: q, k and v must have the same shape")
    if d % heads:
        raise EngineError("spiking_attention: d_model must be divisible by heads")
    dh = d // heads
    q, k, v, lam = (_contig(t) for t in (q, k, v, lam))
    BT = q.numel() // (L * d)
    out = torch.empty(shape, dtype=torch.float32, device=q.device)
    lib = _lib.load()
    ws, wsn = _lib.workspace(q.device, lib.spk_attention_workspace_bytes(BT, L, heads, dh))
    check(lib.spk_spiking_attention(ptr(q), ptr(k), ptr(v), ptr(lam), BT, L, heads, dh, float(eps), ptr(out), ws,
                                    wsn, stream_of(q)), "spk_spiking_attention")
    return out


def spiking_attention_bits(q_bits, k_bits, v_bits, lam, heads, eps=1e-6):
    """spiking_attention over packed spikes: q_bits, k_bits, v_bits int32
    [..., L, d/32] (bit b of word w = channel 32w + b, as linear_act's
    "heaviside_bits" / "vspike_bits" write them) -> [..., L, d] fp32, the same
    values as spiking_attention on the unpacked spikes.  Needs d % 128 == 0."""
    require_cuda(q_bits, k_bits, v_bits, lam, what="spiking_attention_bits")
    require_f32(lam, what="spiking_attention_bits")
    shape = q_bits.shape
    if k_bits.shape != shape or v_bits.shape != shape:
        raise EngineError("spiking_attention_bits: q, k and v must have the same shape")
    for t in (q_bits, k_bits, v_bits):
        if t.dtype != torch.int32:
            raise EngineError("spiking_attention_bits: packed spikes must be int32")
    L, d = shape[-2], shape[-1] * 32
    if d % heads:
        raise EngineError("spiking_attention_bits: d_model must be divisible by heads")
    dh = d // heads
    q_bits, k_bits, v_bits, lam = (_contig(t) for t in (q_bits, k_bits, v_bits, lam))
    BT = q_bits.numel() // (L * (d // 32))
    out = torch.empty(*shape[:-1], d, dtype=torch.float32, device=q_bits.device)
    lib = _lib.load()
    ws, wsn = _lib.workspace(q_bits.device, lib.spk_attention_workspace_bytes(BT, L, heads, dh))
    check(lib.spk_spiking_attention_bits(ptr(q_bits), ptr(k_bits), ptr(v_bits), ptr(lam), BT, L, heads, dh,
                                         float(eps), ptr(out), ws, wsn, stream_of(q_bits)),
          "spk_spiking_attention_bits")
    return out


# --------------------------------------------------------------------------- GSMC
def fused_gsmc_step(gi, gr, wd, bias, m, s, heat, v_th, gate_scale, adaptive_threshold, beta_adapt):
    """One GSMC step (gsmc_cuda.cu:79-127); updates m, s, heat in place and
    returns the new spikes [M, d]."""
    require_cuda(gi, gr, wd, bias, m, s, heat, what="fused_gsmc_step")
    require_f32(gi, gr, wd, bias, m, s, heat, what="fused_gsmc_step")
    for t in (gi, gr, wd, bias, m, s, heat):
        if not t.is_contiguous():
            raise EngineError("fused_gsmc_step: inputs and state tensors must be contiguous")
    M, d = gi.shape[0], wd.shape[-1]
    if gi.shape[-1] != 4 * d or gr.shape[-1] != 4 * d:
        raise EngineError("fused_gsmc_step: gi and gr must be of shape (M, 4*d)")
    if bias.numel() != 4 * d:
        raise EngineError("fused_gsmc_step: bias must have 4*d elements")
    if m.numel() != M * d or s.numel() != M * d or heat.numel() != M * d:
        raise EngineError("fused_gsmc_step: m, s and heat must be of size (M, d)")
    out = torch.empty(M, d, dtype=torch.float32, device=gi.device)
    check(_lib.load().spk_gsmc_step(ptr(gi), ptr(gr), ptr(wd), ptr(bias), ptr(m), ptr(s), ptr(heat), ptr(out), M, d,
                                    float(v_th), float(gate_scale), int(bool(adaptive_threshold)),
                                    float(beta_adapt), stream_of(gi)), "spk_gsmc_step")
    return out


def gsmc_forward(gi_all, wd_all, w_rec, bias, v_th=1.0, gate_scale=4.0, adaptive=True, beta=0.8, pool="mean",
                 return_planes=False, fused=False):
    """The eval-mode GSMC recurrence (gsmc.py:96-148) over precomputed input
    projections gi_all [T, M, 4d] and wd_all [T, M, d]; w_rec is the W_rec
    nn.Linear weight [4d, d].  Returns pooled [M, d] (and the planes [T, M, d]).
    fused=True: the recurrent projection and the cell update in one kernel per
    plane (SPK_GSMC_FUSED; same results, slower at the model's geometry)."""
    require_cuda(gi_all, wd_all, w_rec, bias, what="gsmc_forward")
    require_f32(gi_all, wd_all, w_rec, bias, what="gsmc_forward")
    gi_all, wd_all, w_rec, bias = (_contig(t) for t in (gi_all, wd_all, w_rec, bias))
    T, M, d = wd_all.shape
    pooled = torch.empty(M, d, dtype=torch.float32, device=gi_all.device)
    planes = torch.empty(T, M, d, dtype=torch.float32, device=gi_all.device) if return_planes else None
    lib = _lib.load()
    ws, wsn = _lib.workspace(gi_all.device, lib.spk_gsmc_workspace_bytes(M, d))
    _record("gsmc_recurrent", (T - 1) * M, d, 4 * d)  # W_rec s_{t-1} for t >= 1 (s_{-1} = 0 is skipped)
    check(lib.spk_gsmc_forward_ex(ptr(gi_all), ptr(wd_all), ptr(w_rec), ptr(bias), T, M, d, float(v_th),
                                  float(gate_scale), int(bool(adaptive)), float(beta), 1 if pool == "mean" else 0,
                                  ptr(planes), ptr(pooled), ws, wsn, 1 if fused else 0, stream_of(gi_all)),
          "spk_gsmc_forward")
    return (pooled, planes) if return_planes else pooled


# --------------------------------------------------------------------------- residual add + layer norm
def add_layernorm(x, delta, weight=None, bias=None, eps=1e-5):
    """h = x + delta and y = layer_norm(h) over the last dimension in one pass
    (spk_add_layernorm): the pre-norm block's residual add followed by the
    nn.LayerNorm of the sum (nn/attention.py:174-177).  delta None: h = x and
    y = layer_norm(x).  weight / bias: the nn.LayerNorm affine parameters [d]
    (None: 1 / 0).  Returns (h, y).  Needs d % 4 == 0 and d <= 1024."""
    require_cuda(x, delta, weight, bias, what="add_layernorm")
    require_f32(x, delta, weight, bias, what="add_layernorm")
    x = _contig(x)
    d = x.shape[-1]
    if delta is not None:
        if delta.shape != x.shape:
            raise EngineError(f"add_layernorm: delta shape {tuple(delta.shape)} != x shape {tuple(x.shape)}")
        delta = _contig(delta)
    for name, p in (("weight", weight), ("bias", bias)):
        if p is not None and p.numel() != d:
            raise EngineError(f"add_layernorm: {name} must have d={d} elements")
    weight = _contig(weight) if weight is not None else None
    bias = _contig(bias) if bias is not None else None
    rows = x.numel() // d if d else 0
    h = torch.empty_like(x) if delta is not None else x
    y = torch.empty_like(x)
    check(_lib.load().spk_add_layernorm(ptr(x), ptr(delta), ptr(weight), ptr(bias), rows, d, float(eps),
                                        ptr(h) if delta is not None else None, ptr(y), stream_of(x)),
          "spk_add_layernorm")
    return h, y


# --------------------------------------------------------------------------- Spire planes
def spire_planes(u, dither, frontier=None, temporal_frontier=None):
    """The Spire encoder's temporal planes (encode/spire.py:60-69) in one pass
    (spk_spire_planes): for u [B, N, d] and dither [T],
    planes[t] = ((u - frontier) - temporal_frontier[n]) - dither[t] > 0 as
    float32 [T, B, N, d]; frontier [d] and temporal_frontier [N] (any shape
    with those element counts) may be None."""
    require_cuda(u, dither, frontier, temporal_frontier, what="spire_planes")
    require_f32(u, dither, frontier, temporal_frontier, what="spire_planes")
    if u.dim() != 3:
        raise EngineError("spire_planes: u must be (B, N, d)")
    B, N, d = u.shape
    u = _contig(u)
    dither = _contig(dither).view(-1)
    if frontier is not None:
        frontier = _contig(frontier).view(-1)
        if frontier.numel() != d:
            raise EngineError(f"spire_planes: frontier must have d={d} elements")
    if temporal_frontier is not None:
        temporal_frontier = _contig(temporal_frontier).view(-1)
        if temporal_frontier.numel() != N:
            raise EngineError(f"spire_planes: temporal_frontier must have N={N} elements")
    T = dither.numel()
    planes = torch.empty(T, B, N, d, dtype=torch.float32, device=u.device)
    check(_lib.load().spk_spire_planes(ptr(u), ptr(frontier), ptr(temporal_frontier), ptr(dither), T, B, N, d,
                                       ptr(planes), stream_of(u)), "spk_spire_planes")
    return planes


def spire_dither(v, dither):
    """spire_dither(v [B, N, d], dither [T]) -> (v - dither[t] > 0) as float32
    [T, B, N, d]: the reference Spire engine's entry point (spire_cuda.cu:28-58)."""
    return spire_planes(v, dither)


# --------------------------------------------------------------------------- readout pooling
def temporal_mean(x):
    """(mean of x, mean of (x > 0)) over (t, n) per sample and channel for a
    temporal context x [T, B, N, d], or over n for [B, N, d] (the pooling in
    front of SpikingTransformer's classifier, models/transformer.py:159-192),
    in one pass (spk_temporal_mean).  Both results [B, d] float32."""
    require_cuda(x, what="temporal_mean")
    require_f32(x, what="temporal_mean")
    if x.dim() == 3:
        T, (B, N, d) = 1, x.shape
    elif x.dim() == 4:
        T, B, N, d = x.shape
    else:
        raise EngineError("temporal_mean: x must be (T, B, N, d) or (B, N, d)")
    x = _contig(x)
    mean_x = torch.empty(B, d, dtype=torch.float32, device=x.device)
    mean_s = torch.empty(B, d, dtype=torch.float32, device=x.device)
    check(_lib.load().spk_temporal_mean(ptr(x), T, B, N, d, ptr(mean_x), ptr(mean_s), stream_of(x)),
          "spk_temporal_mean")
    return mean_x, mean_s
