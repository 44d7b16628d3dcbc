"""CPU oracle for the SpikeStack Lite temporal forward hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: tests/, the smoke check
in __graft_entry__.py and the CPU-baseline leg of bench.py use it to produce
expected results on the CPU.  The product (package ``spikestack_lite_b200``)
never imports it and has no CPU fallback.

Every function restates the reference implementation (Griffith-7/spikestack-lite,
cited by file:line inside that project) in plain numpy / PyTorch-CPU code:

* integer / index work (CSR build) in numpy and in ``csr_oracle.c`` (bit-exact);
* floating point in PyTorch fp32 on the CPU, which is the reference's own CPU
  arithmetic (its CPU fallbacks are ``torch.matmul`` / elementwise torch ops).

Pinning: ``tests/test_oracle.py`` checks these functions against the golden
vectors in ``tests/golden/`` (produced by the reference itself, see
``tests/golden/make_golden.py``); the CSR restatement, for which the reference
has no CPU path, is pinned on the GPU box against the reference's own CUDA
engine compiled from its sources into ``oracle/_ref`` (``oracle/build_ref.py``).
"""

import ctypes
import math
import os

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def _lib():
    """ctypes handle of csr_oracle.c built into oracle/_build/liboracle.so."""
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            from oracle.build_oracle import build_oracle

            build_oracle()
        lib = ctypes.CDLL(path)
        lib.orc_csr_plane.restype = ctypes.c_int64
        lib.orc_csr_plane.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        lib.orc_spmm_csr.restype = None
        lib.orc_spmm_csr.argtypes = [ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        _LIB = lib
    return _LIB


def _ptr(a):
    return a.ctypes.data if a is not None else None


# ----------------------------------------------------------------------------- CSR
def csr_plane(S2):
    """CSR of one plane S2 [M, K] (numpy float32).

    Follows sparse_linear.cu:251-278 (predicate ``v > 0``: negatives and NaN
    dropped; nonzeros in ascending column order), :315-369 (int32 row
    offsets, row_offsets[0] = 0) and :281-299 (values copied from the input).
    Returns (nnz_row[M], row_ptr[M+1], col_idx[nnz], values[nnz]).
    """
    S2 = np.ascontiguousarray(S2, dtype=np.float32)
    mask = S2 > 0
    nnz = mask.sum(axis=1).astype(np.int32)
    row_ptr = np.zeros(S2.shape[0] + 1, dtype=np.int32)
    np.cumsum(nnz, out=row_ptr[1:])
    rows, cols = np.nonzero(mask)  # row-major order = ascending column per row
    return nnz, row_ptr, cols.astype(np.int32), S2[rows, cols].astype(np.float32)


def csr_plane_c(S2):
    """Same as csr_plane, computed by the C restatement (csr_oracle.c)."""
    S2 = np.ascontiguousarray(S2, dtype=np.float32)
    M, K = S2.shape
    cap = int((S2 > 0).sum())
    nnz = np.empty(M, np.int32)
    rp = np.empty(M + 1, np.int32)
    ci = np.empty(max(cap, 1), np.int32)
    vals = np.empty(max(cap, 1), np.float32)
    n = _lib().orc_csr_plane(_ptr(S2), M, K, _ptr(nnz), _ptr(rp), _ptr(ci), _ptr(vals), cap)
    return nnz, rp, ci[:n], vals[:n]


def csr_planes(S3):
    """Per-plane CSR of S3 [T, M, K] in the layout of spk_csr_compact:
    nnz_row [T, M], row_ptr [T, M+1] (relative to each plane), col_idx and
    values of all planes back to back, plane_ptr [T+1] (int64)."""
    T = S3.shape[0]
    parts = [csr_plane(S3[t]) for t in range(T)]
    nnz = np.stack([p[0] for p in parts])
    rp = np.stack([p[1] for p in parts])
    ci = np.concatenate([p[2] for p in parts])
    vals = np.concatenate([p[3] for p in parts])
    pp = np.zeros(T + 1, np.int64)
    np.cumsum([len(p[2]) for p in parts], out=pp[1:])
    return nnz, rp, ci, vals, pp


def spmm_csr_exact(row_ptr, col_idx, values, weightT):
    """CSR x weightT with the reference engine's exact summation
    (csr_coalesced_kernel, sparse_linear.cu:59-90): ascending entries, one
    fused multiply-add per term from 0.  Bit-exact restatement in C."""
    weightT = np.ascontiguousarray(weightT, dtype=np.float32)
    M = len(row_ptr) - 1
    N = weightT.shape[1]
    out = np.empty((M, N), np.float32)
    rp = np.ascontiguousarray(row_ptr, np.int32)
    ci = np.ascontiguousarray(col_idx, np.int32) if len(col_idx) else np.zeros(1, np.int32)
    vv = np.ascontiguousarray(values, np.float32) if values is not None and len(values) else None
    if values is not None and len(values) == 0:
        vv = np.zeros(1, np.float32)
    _lib().orc_spmm_csr(M, _ptr(rp), _ptr(ci), _ptr(vv), _ptr(weightT), N, _ptr(out))
    return out


# ---------------------------------------------------------------- spike-linear
def spike_linear(S, weightT, bias=None):
    """Y = relu'(S) @ weightT (+ bias), fp32 on the CPU.

    The reference engine only accumulates entries with S > 0
    (sparse_linear.cu:268); its CPU fallback is ``torch.matmul(dense_input,
    weightT)`` (sparse/__init__.py:104-105), which agrees for the non-negative
    spike inputs of the path.  SparseLinear adds the bias afterwards
    (sparse/__init__.py:260-261)."""
    X = torch.as_tensor(np.asarray(S, dtype=np.float32))
    X = torch.where(X > 0, X, torch.zeros((), dtype=X.dtype))
    W = torch.as_tensor(np.asarray(weightT, dtype=np.float32))
    Y = torch.matmul(X, W)
    if bias is not None:
        Y = Y + torch.as_tensor(np.asarray(bias, dtype=np.float32))
    return Y.numpy()


def reference_cpu_step(S, weightT):
    """The reference's CPU implementation of the spike-linear step exactly as it
    runs without an engine: ``torch.matmul(dense_input, weightT)``
    (sparse/__init__.py:104-105); S and weightT are CPU float32 tensors.  Used
    as the timed CPU baseline (it equals spike_linear for spike inputs)."""
    return torch.matmul(S, weightT)


def sparse_multistep_forward(S, weightT):
    """The reference op ``sparse_multistep_forward`` (sparse_linear.cu:645-691):
    returns (Y [T, M, N], CSR of plane T-1 as left in the caller's buffers)."""
    S = np.asarray(S, dtype=np.float32)
    return spike_linear(S, weightT), csr_plane(S[-1])


# ------------------------------------------------------------------- attention
def channel_decay(k, lam):
    """k_w = k * lam ** pos, pos = N-1 .. 0 along the sequence axis (-2)
    (attention.py:30-44, CPU branch)."""
    k = torch.as_tensor(k, dtype=torch.float32)
    lam = torch.as_tensor(lam, dtype=torch.float32)
    N = k.size(-2)
    pos = torch.arange(N - 1, -1, -1, dtype=torch.float32)
    w = lam.unsqueeze(0) ** pos.unsqueeze(1)
    return k * w.unsqueeze(0) if k.dim() >= 3 else k * w


def normalize_attention(numer, denom, eps):
    """numer / (denom + eps) (attention.py:57-73, CPU branch)."""
    return torch.as_tensor(numer) / (torch.as_tensor(denom) + eps)


def spiking_attention(q, k, v, lam, heads, eps=1e-6):
    """Middle of AstrocyteHebbianAttention.forward (attention.py:120-135):
    q, k, v spikes [..., N, d] -> normalised attention [..., N, d] (the o_proj
    input), heads merged back in d_model layout."""
    q = torch.as_tensor(q, dtype=torch.float32)
    k = torch.as_tensor(k, dtype=torch.float32)
    v = torch.as_tensor(v, dtype=torch.float32)
    leading = q.shape[:-1]
    d = q.shape[-1]
    dh = d // heads
    k_w = channel_decay(k, lam)
    qh = q.view(*leading, heads, dh).transpose(-3, -2)
    kh = k_w.view(*leading, heads, dh).transpose(-3, -2)
    vh = v.view(*leading, heads, dh).transpose(-3, -2)
    kv = torch.matmul(kh.transpose(-2, -1), vh)
    key_mass = kh.sum(dim=-2, keepdim=True).transpose(-2, -1)
    numer = torch.matmul(qh, kv)
    denom = torch.matmul(qh, key_mass)
    out = normalize_attention(numer, denom, eps)
    return out.transpose(-3, -2).contiguous().view(*leading, d)


# ------------------------------------------------------------------------ GSMC
def gsmc_step(gi, gr, wd, bias, m, s, heat, v_th=1.0, gate_scale=4.0, adaptive=True, beta=0.8):
    """One step of the reference engine's fused_gsmc_step (gsmc_cuda.cu:11-77):
    pre = (gi + gr) / gate_scale + bias.  Returns (s_new, m_new, heat_new)."""
    d = wd.shape[-1]
    pre = (gi + gr) / gate_scale + bias
    f = 1.0 / (1.0 + torch.exp(-pre[:, :d]))
    i = 1.0 / (1.0 + torch.exp(-pre[:, d:2 * d]))
    o = 1.0 / (1.0 + torch.exp(-pre[:, 2 * d:3 * d]))
    g = torch.tanh(pre[:, 3 * d:])
    a = f * m + i * g
    vv = o * torch.tanh(a) + wd
    theta = v_th * (1.0 + heat) if adaptive else torch.full_like(heat, v_th)
    s_new = (vv > theta).float()
    m_new = a - s_new * v_th
    heat_new = beta * heat + s_new if adaptive else torch.zeros_like(heat)
    return s_new, m_new, heat_new


def gsmc_forward(x, sd, v_th=1.0, gate_scale=4.0, adaptive=True, beta=0.8, pool="mean", step="module"):
    """FusedGSMC.forward in eval mode (gsmc.py:96-148).  ``sd`` holds W_in.*,
    W_rec.weight, W_d.*.  step="module" uses the module's CPU gate order
    (gsmc.py:86-94: gi/gs + gr/gs + bias), step="engine" the CUDA engine's
    ((gi + gr)/gs + bias).  Returns (pooled [B, N, d], planes [T, B*N, d])."""
    x = torch.as_tensor(x, dtype=torch.float32)
    T, B, N, d = x.shape
    flat = x.reshape(T, -1, d)
    W_in, b_in = _t(sd["W_in.weight"]), _t(sd["W_in.bias"])
    W_rec = _t(sd["W_rec.weight"])
    W_d, b_d = _t(sd["W_d.weight"]), _t(sd["W_d.bias"])
    gi_all = F.linear(flat, W_in, b_in)
    wd_all = F.linear(flat, W_d, b_d)
    M = B * N
    m = torch.zeros(M, d)
    s = torch.zeros(M, d)
    heat = torch.zeros(M, d)
    out = torch.empty(T, M, d)
    for t in range(T):
        gr = F.linear(s, W_rec)
        if step == "engine":
            s_new, m, heat = gsmc_step(gi_all[t], gr, wd_all[t], b_in, m, s, heat, v_th, gate_scale, adaptive, beta)
        else:
            pre = (gi_all[t] / gate_scale + gr / gate_scale) + b_in
            f = torch.sigmoid(pre[:, :d])
            i = torch.sigmoid(pre[:, d:2 * d])
            o = torch.sigmoid(pre[:, 2 * d:3 * d])
            g = torch.tanh(pre[:, 3 * d:])
            a = f * m + i * g
            vv = o * torch.tanh(a) + wd_all[t]
            theta = v_th * (1.0 + heat) if adaptive else v_th
            s_new = (vv - theta > 0).float()
            m = a - s_new * v_th
            if adaptive:
                heat = beta * heat + s_new
        s = s_new
        out[t] = s_new
    pooled = out.mean(dim=0) if pool == "mean" else out[-1]
    return pooled.view(B, N, d), out


# ----------------------------------------------------------------------- model
def _t(a):
    return torch.as_tensor(np.asarray(a), dtype=torch.float32)


def _lin(sd, prefix, x):
    w = _t(sd[prefix + ".weight"])
    b = sd.get(prefix + ".bias")
    return F.linear(x, w, None if b is None else _t(b))


def fc2_key(sd, prefix):
    """SparseLinear keeps its weight under fc2.linear.*, nn.Linear under fc2.*
    (sparse/__init__.py:209 vs attention.py:151)."""
    return prefix + ".linear" if (prefix + ".linear.weight") in sd else prefix


def spire_forward(sd, x, temporal=True):
    """SpireEncoder.forward (spire.py:60-69) with the PyTorch dither branch
    (spire.py:21-24): planes (R, B, N, d) of (v - dither_r > 0)."""
    u = _lin(sd, "embedding.projection", _t(x))
    d = u.shape[-1]
    v = (u - _t(sd["embedding.frontier"]).view(1, 1, d) - _t(sd["embedding.temporal_frontier"])).float()
    dither = _t(sd["embedding.dither"])
    spikes = (v.unsqueeze(-1) - dither > 0).float().permute(3, 0, 1, 2)
    return spikes if temporal else spikes.mean(dim=0)


def attention_forward(sd, p, x, heads, eps=1e-6):
    """AstrocyteHebbianAttention.forward (attention.py:105-136), v_levels = 1."""
    q = (_lin(sd, p + ".q_proj", x) > 0).float()
    k = (_lin(sd, p + ".k_proj", x) > 0).float()
    u01 = (torch.tanh(_lin(sd, p + ".v_proj", x)) + 1.0) / 2.0
    tau = float(np.asarray(sd[p + ".tau"]).reshape(-1)[0])
    v = (u01 - tau > 0).float()
    lam = torch.sigmoid(_t(sd[p + ".decay_logit"]))
    out = spiking_attention(q, k, v, lam, heads, eps)
    return _lin(sd, p + ".o_proj", out)


def ffn_forward(sd, p, x, threshold=0.0):
    """SpikingFFN.forward (attention.py:153-159): spike(fc1(x) - thr) -> fc2."""
    act = (_lin(sd, p + ".fc1", x) - threshold > 0).float()
    return _lin(sd, fc2_key(sd, p + ".fc2"), act)


def block_forward(sd, p, x, heads, threshold=0.0):
    """AstrocyteHebbianBlock.forward (attention.py:174-177), pre-norm."""
    d = x.shape[-1]
    h = F.layer_norm(x, (d,), _t(sd[p + ".norm1.weight"]), _t(sd[p + ".norm1.bias"]))
    x = x + attention_forward(sd, p + ".attn", h, heads)
    h = F.layer_norm(x, (d,), _t(sd[p + ".norm2.weight"]), _t(sd[p + ".norm2.bias"]))
    return x + ffn_forward(sd, p + ".ffn", h, threshold)


def block_stages(sd, p, x, heads, threshold=0.0):
    """block_forward with its intermediate stages (attention.py:110-117,
    153-159, 174-177): the two layer-norm outputs h1 and h2, the fp32
    pre-activations of the q, k, v projections and of fc1, their spikes, the
    mid-block residual x_mid and the block output.  Spike-flip accounting
    compares an implementation's spikes, computed from these same h1 / h2,
    with the ones here."""
    d = x.shape[-1]
    st = {}
    with torch.no_grad():
        h1 = F.layer_norm(x, (d,), _t(sd[p + ".norm1.weight"]), _t(sd[p + ".norm1.bias"]))
        st["h1"] = h1
        a = p + ".attn"
        st["q_pre"] = _lin(sd, a + ".q_proj", h1)
        st["k_pre"] = _lin(sd, a + ".k_proj", h1)
        st["v_pre"] = _lin(sd, a + ".v_proj", h1)
        st["tau"] = float(np.asarray(sd[a + ".tau"]).reshape(-1)[0])
        st["q"] = (st["q_pre"] > 0).float()
        st["k"] = (st["k_pre"] > 0).float()
        st["v"] = ((torch.tanh(st["v_pre"]) + 1.0) / 2.0 - st["tau"] > 0).float()
        lam = torch.sigmoid(_t(sd[a + ".decay_logit"]))
        st["attn"] = spiking_attention(st["q"], st["k"], st["v"], lam, heads)
        x_mid = x + _lin(sd, a + ".o_proj", st["attn"])
        st["x_mid"] = x_mid
        h2 = F.layer_norm(x_mid, (d,), _t(sd[p + ".norm2.weight"]), _t(sd[p + ".norm2.bias"]))
        st["h2"] = h2
        st["fc1_pre"] = _lin(sd, p + ".ffn.fc1", h2) - threshold
        st["act"] = (st["fc1_pre"] > 0).float()
        st["out"] = x_mid + _lin(sd, fc2_key(sd, p + ".ffn.fc2"), st["act"])
    return st


def block_from_spikes(sd, p, x, heads, q, k, v, act):
    """The arithmetic of one block (attention.py:119-136, 158, 174-177) from
    given q, k, v and fc1 spikes: attn = the normalised attention of (q, k, v),
    x_mid = x + o_proj(attn), out = x_mid + fc2(act).  With an implementation's
    own spikes this isolates its arithmetic from its threshold decisions."""
    a = p + ".attn"
    with torch.no_grad():
        lam = torch.sigmoid(_t(sd[a + ".decay_logit"]))
        attn = spiking_attention(_t(q), _t(k), _t(v), lam, heads)
        x_mid = _t(x) + _lin(sd, a + ".o_proj", attn)
        out = x_mid + _lin(sd, fc2_key(sd, p + ".ffn.fc2"), _t(act))
    return {"attn": attn, "x_mid": x_mid, "out": out}


def transformer_forward(sd, x, num_heads, num_layers, use_gsmc=False, spike_readout=True, threshold=0.0,
                        gsmc_pool="mean", capture=None):
    """SpikingTransformer.forward in temporal mode (transformer.py:159-192).
    ``capture`` (dict) receives the Spire planes, each block's output and the
    GSMC output for per-stage (teacher-forced) comparisons."""
    with torch.no_grad():
        ctx = spire_forward(sd, x, temporal=True)
        if capture is not None:
            capture["planes"] = ctx
        for i in range(num_layers):
            ctx = block_forward(sd, f"blocks.{i}", ctx, num_heads, threshold)
            if capture is not None:
                capture[f"block{i}_out"] = ctx
        if use_gsmc:
            gsd = {k[len("gsmc."):]: v for k, v in sd.items() if k.startswith("gsmc.")}
            ctx, _ = gsmc_forward(ctx, gsd, pool=gsmc_pool)
            if capture is not None:
                capture["gsmc_out"] = ctx
        if spike_readout:
            ctx = (ctx > 0).float()
        pooled = ctx.mean(dim=(0, 2)) if not use_gsmc else ctx.mean(dim=1)
        return _lin(sd, "classifier", pooled)


def model_config_from_golden(z):
    """Constructor keyword arguments stored in a golden model fixture."""
    import ast

    return dict(ast.literal_eval(str(z["config"])))


def state_dict_from_golden(z):
    return {k[3:]: np.asarray(z[k]) for k in z.files if k.startswith("sd_")}


def rel_err(a, b):
    """max |a - b| / max |b| (the parity tolerance metric: fp32 outputs within 1e-4 of it)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    scale = max(float(np.abs(b).max()) if b.size else 0.0, 1e-30)
    return float(np.abs(a - b).max()) / scale if b.size else 0.0


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("ctypes", "math", "os", "np", "torch", "F")]
