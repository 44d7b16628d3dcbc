"""Mirror of ``spikestack_lite.nn.attention`` on the B200 engine.

Same classes, constructor arguments and parameter names as the reference
(nn/attention.py): SurrogateHeaviside / spike_fn, AstrocyteHebbianAttention,
SpikingFFN, AstrocyteHebbianBlock.  Parameters are created in the reference's
order with the reference's initialisers, so a given torch seed yields the same
weights and reference state dicts load unchanged.

Forward without autograd (inference, the hot path) runs the fused spiking
attention kernel: q/k/v spikes -> decay -> K^T V trace + key mass ->
normalise, one pass per input, output already in d_model layout.  With
autograd on, the engine's decay / normalise ops run between dense torch
matmuls and the backward stays the reference's exact dense formulas.
"""
import torch
import torch.nn as nn

from . import ops
from .ops import engine_linear
from ._lib import EngineError
from .engine import attention_engine
from .sparse import SparseLinear

_attn_cuda_engine = attention_engine


def _engine_norm_ok(norm, x):
    """True when the engine's residual add + layer norm (spk_add_layernorm) can
    stand in for `norm` on x: autograd off, CUDA fp32 input, a layer norm over
    the last dimension of width d % 4 == 0, d <= 1024."""
    d = x.shape[-1]
    return (not torch.is_grad_enabled() and x.is_cuda and x.dtype == torch.float32
            and tuple(norm.normalized_shape) == (d,) and d % 4 == 0 and d <= 1024)


class SurrogateHeaviside(torch.autograd.Function):
    """(x > 0) forward, sigmoid-derivative surrogate backward (attention.py:13-24)."""

    @staticmethod
    def forward(ctx, input):
        ctx.save_for_backward(input)
        return (input > 0).float()

    @staticmethod
    def backward(ctx, grad_output):
        (input,) = ctx.saved_tensors
        sig = torch.sigmoid(10.0 * input)
        return grad_output * sig * (1 - sig) * 10.0


spike_fn = SurrogateHeaviside.apply


class _ChannelDecayAutograd(torch.autograd.Function):
    """Engine decay forward, exact dense backward (attention.py:30-54)."""

    @staticmethod
    def forward(ctx, k, lam, engine):
        N = k.size(-2)
        pos = torch.arange(N - 1, -1, -1, device=k.device, dtype=torch.float32)
        w = lam.unsqueeze(0) ** pos.unsqueeze(1)
        ctx.save_for_backward(k, lam, w, pos)
        return engine.apply_channel_decay(k.contiguous(), lam.contiguous())

    @staticmethod
    def backward(ctx, grad_k_w):
        k, lam, w, pos = ctx.saved_tensors
        grad_k = grad_k_w * w.unsqueeze(0)
        p = pos.unsqueeze(1)
        dw = p * torch.pow(lam.unsqueeze(0), (p - 1.0).clamp(min=0.0))
        grad_lam = (grad_k_w * k * dw.unsqueeze(0)).sum(dim=tuple(range(grad_k_w.dim() - 2)) + (-2,))
        return grad_k, grad_lam, None


class _NormalizeAttentionAutograd(torch.autograd.Function):
    """Engine normalise forward, exact dense backward (attention.py:57-81)."""

    @staticmethod
    def forward(ctx, numer, denom, eps, engine):
        denom_eps = denom + eps
        out = engine.fused_normalize_attention(numer.contiguous(), denom.expand_as(numer).contiguous(), float(eps))
        ctx.save_for_backward(numer, denom_eps, out)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        numer, denom_eps, out = ctx.saved_tensors
        return grad_out / denom_eps, -grad_out * out / denom_eps, None, None


class AstrocyteHebbianAttention(nn.Module):
    """Multi-head spiking linear attention with learnable per-channel decay
    (attention.py:84-136)."""

    def __init__(self, d_model=128, num_heads=4, v_levels=1):
        super().__init__()
        if d_model % num_heads:
            raise ValueError("d_model must be divisible by num_heads")
        self.h = num_heads
        self.dh = d_model // num_heads
        self.L = max(1, int(v_levels))
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.o_proj = nn.Linear(d_model, d_model)
        self.register_buffer("tau", torch.arange(1, self.L + 1).float() / (self.L + 1))
        self.decay_logit = nn.Parameter(torch.empty(d_model).uniform_(5.0, 8.0))
        self.eps = 1e-6

    def spikes(self, x):
        """q, k, v spike tensors of x (attention.py:110-118)."""
        if self.L == 1:
            q = engine_linear(self.q_proj, x, "heaviside")
            if q is not None:  # v: (tanh(v_proj(x)) + 1) / 2 - tau[0] > 0, tau[0] = 1 / (L + 1)
                return q, engine_linear(self.k_proj, x, "heaviside"), engine_linear(self.v_proj, x, "vspike", 0.5)
        q = spike_fn(self.q_proj(x))
        k = spike_fn(self.k_proj(x))
        u01 = (torch.tanh(self.v_proj(x)) + 1.0) / 2.0
        if self.L == 1:
            v = spike_fn(u01 - self.tau[0])
        else:
            v = spike_fn(u01.unsqueeze(-1) - self.tau.view(*([1] * u01.dim()), -1)).mean(dim=-1)
        return q, k, v

    def attend(self, q, k, v):
        """Normalised attention (the o_proj input), heads merged."""
        lam = torch.sigmoid(self.decay_logit)
        if not torch.is_grad_enabled() and self.L == 1:
            return ops.spiking_attention(q, k, v, lam, self.h, self.eps)
        leading = q.shape[:-1]
        d = q.shape[-1]
        k_w = _ChannelDecayAutograd.apply(k, lam, _attn_cuda_engine)
        qh = q.view(*leading, self.h, self.dh).transpose(-3, -2)
        kh = k_w.view(*leading, self.h, self.dh).transpose(-3, -2)
        vh = v.view(*leading, self.h, self.dh).transpose(-3, -2)
        kv = torch.matmul(kh.transpose(-2, -1), vh)
        key_mass = kh.sum(dim=-2, keepdim=True).transpose(-2, -1)
        out = _NormalizeAttentionAutograd.apply(torch.matmul(qh, kv), torch.matmul(qh, key_mass), self.eps,
                                                _attn_cuda_engine)
        return out.transpose(-3, -2).contiguous().view(*leading, d)

    def _packed_ok(self, x):
        """Inference on shapes the packed tensor-core attention takes."""
        d = self.h * self.dh
        return (not torch.is_grad_enabled() and x.is_cuda and x.dtype == torch.float32 and self.L == 1
                and d % 128 == 0 and self.dh in (16, 32, 64))

    def forward(self, x, record=None):
        """``record`` (a dict, optional) receives the q, k, v spikes and the
        normalised attention ("attn") this call computed.

        At inference the q, k and v spikes go from their projections to the
        attention packed one bit each (linear_act "heaviside_bits" /
        "vspike_bits" -> spiking_attention_bits): the reference's three fp32
        spike tensors (attention.py:110-117) are never written."""
        if x.device.type != "cuda":
            raise EngineError("AstrocyteHebbianAttention: CUDA input required (no CPU path)")
        if self._packed_ok(x):
            qb = engine_linear(self.q_proj, x, "heaviside_bits")
            if qb is not None:
                kb = engine_linear(self.k_proj, x, "heaviside_bits")
                vb = engine_linear(self.v_proj, x, "vspike_bits", 0.5)  # tau[0] = 1 / (L + 1), L = 1
                a = ops.spiking_attention_bits(qb, kb, vb, torch.sigmoid(self.decay_logit), self.h, self.eps)
                if record is not None:
                    d = self.h * self.dh
                    record.update(q=ops.unpack_spikes(qb, d), k=ops.unpack_spikes(kb, d), v=ops.unpack_spikes(vb, d),
                                  attn=a)
                y = engine_linear(self.o_proj, a)
                return y if y is not None else self.o_proj(a)
        q, k, v = self.spikes(x)
        a = self.attend(q, k, v)
        if record is not None:
            record.update(q=q, k=k, v=v, attn=a)
        y = engine_linear(self.o_proj, a)
        return y if y is not None else self.o_proj(a)


class SpikingFFN(nn.Module):
    """spike(fc1(x) - threshold) -> fc2 (attention.py:141-159); with SpikeSkip
    and a temporal (T, B, N, d) input, fc2 is the multi-plane spike-linear."""

    def __init__(self, d_model=128, expansion=4, use_spikeskip=False, spike_threshold=0.0):
        super().__init__()
        self.threshold = float(spike_threshold)
        self.fc1 = nn.Linear(d_model, d_model * expansion)
        self.use_spikeskip = use_spikeskip
        if use_spikeskip:
            self.fc2 = SparseLinear(d_model * expansion, d_model, bias=True)
        else:
            self.fc2 = nn.Linear(d_model * expansion, d_model)

    def forward(self, x, record=None):
        """``record`` (a dict, optional) receives the fc1 spikes ("act").

        At inference on a temporal input with the SpikeSkip fc2, fc1's spikes
        go to fc2 packed one bit each (ops.linear_act "heaviside_bits" ->
        SparseLinear.forward_bits): the reference's dense fp32 act tensor
        (attention.py:156) is never written."""
        if (self.use_spikeskip and x.dim() == 4 and self.fc1.out_features % 64 == 0
                and self.fc2.out_features > 64 and x.dtype == torch.float32):
            bits = engine_linear(self.fc1, x, "heaviside_bits", self.threshold)
            if bits is not None:
                if record is not None:
                    record["act"] = ops.unpack_spikes(bits, self.fc1.out_features)
                return self.fc2.forward_bits(bits)
        act = engine_linear(self.fc1, x, "heaviside", self.threshold)
        if act is None:
            act = spike_fn(self.fc1(x) - self.threshold)
        if record is not None:
            record["act"] = act
        if self.use_spikeskip and x.dim() == 4:
            return self.fc2.forward_multistep(act)
        return self.fc2(act)


class AstrocyteHebbianBlock(nn.Module):
    """Pre-norm block: x + attn(LN(x)), then x + ffn(LN(x)) (attention.py:162-177)."""

    def __init__(self, d_model=128, num_heads=4, expansion=4, v_levels=1, use_spikeskip=False,
                 spike_threshold=0.0):
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attn = AstrocyteHebbianAttention(d_model, num_heads, v_levels)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn = SpikingFFN(d_model, expansion, use_spikeskip=use_spikeskip, spike_threshold=spike_threshold)

    def forward(self, x):
        return self.forward_fused(x)[0]

    def forward_fused(self, x, x_norm=None, next_norm=None, record=None):
        """(block(x), next_norm(block(x)) or None).  At inference each residual
        add runs together with the layer norm of its result (ops.add_layernorm):
        x + attn(.) with norm2, and the block output with `next_norm` (the next
        block's norm1), whose result the caller hands back as `x_norm`.
        ``record`` (a dict, optional) receives the stages: q, k, v, attn, the
        mid-block residual "x_mid" and the fc1 spikes "act"."""
        if not _engine_norm_ok(self.norm1, x):  # the reference's composition (autograd, CPU)
            x = x + self.attn(self.norm1(x), record)
            if record is not None:
                record["x_mid"] = x
            return x + self.ffn(self.norm2(x), record), None
        if x_norm is None:
            x_norm = ops.add_layernorm(x, None, self.norm1.weight, self.norm1.bias, self.norm1.eps)[1]
        h, h_norm = ops.add_layernorm(x, self.attn(x_norm, record), self.norm2.weight, self.norm2.bias,
                                      self.norm2.eps)
        if record is not None:
            record["x_mid"] = h
        f = self.ffn(h_norm, record)
        if next_norm is None:
            return h + f, None
        return ops.add_layernorm(h, f, next_norm.weight, next_norm.bias, next_norm.eps)
