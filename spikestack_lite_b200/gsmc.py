"""Mirror of ``spikestack_lite.nn.gsmc.FusedGSMC`` on the B200 engine.

Same constructor, parameters (W_in, W_rec, W_d; created and initialised in the
reference's order, nn/gsmc.py:50-84) and forward contract:
x (T, B, N, d) -> (B, N, d).  In eval mode without autograd the whole
recurrence runs in the engine (spk_gsmc_forward: the recurrent projection of
each plane through the spike-linear dense branch, then the fused cell step,
pooling accumulated in place).  With autograd the reference's own tensor
formulas run (gsmc.py:119-142), as the reference does: its engine is
inference-only (gsmc.py:111-116).
"""
import torch
import torch.nn as nn

from . import ops
from ._lib import EngineError
from .attention import SurrogateHeaviside, engine_linear
from .engine import gsmc_engine

_gsmc_cuda_engine = gsmc_engine


class FusedGSMC(nn.Module):
    def __init__(self, d_model: int, v_th: float = 1.0, forget_bias: float = 8.0, output_bias: float = -2.0,
                 recurrent_scale: float = 0.5, gate_scale: float = 4.0, pool: str = "mean",
                 adaptive_threshold: bool = True, beta_adapt: float = 0.8):
        super().__init__()
        self.d_model = d_model
        self.v_th = float(v_th)
        self.pool = pool
        self.adaptive_threshold = bool(adaptive_threshold)
        self.beta_adapt = float(beta_adapt)
        self.W_in = nn.Linear(d_model, 4 * d_model)
        nn.init.xavier_uniform_(self.W_in.weight)
        nn.init.zeros_(self.W_in.bias)
        self.W_rec = nn.Linear(d_model, 4 * d_model, bias=False)
        nn.init.orthogonal_(self.W_rec.weight)
        self.W_rec.weight.data.mul_(recurrent_scale)
        with torch.no_grad():
            self.W_in.bias[:d_model].fill_(forget_bias)
            self.W_in.bias[2 * d_model:3 * d_model].fill_(output_bias)
        self.gate_scale = float(gate_scale)
        self.W_d = nn.Linear(d_model, d_model)
        nn.init.xavier_uniform_(self.W_d.weight)
        nn.init.zeros_(self.W_d.bias)
        self.spike_fn = SurrogateHeaviside.apply

    def forward(self, x, T):
        if x.device.type != "cuda":
            raise EngineError("FusedGSMC: CUDA input required (no CPU path)")
        T_len, B, N, d = x.shape
        flat = x.reshape(T_len, -1, d)
        if not self.training and not torch.is_grad_enabled():
            # input projections on the engine's tensor-core linear when it takes the shape
            gi_all = engine_linear(self.W_in, flat)
            gi_all = self.W_in(flat) if gi_all is None else gi_all
            wd_all = engine_linear(self.W_d, flat)
            wd_all = self.W_d(flat) if wd_all is None else wd_all
            pooled = ops.gsmc_forward(gi_all, wd_all, self.W_rec.weight, self.W_in.bias, self.v_th, self.gate_scale,
                                      self.adaptive_threshold, self.beta_adapt, self.pool)
            return pooled.view(B, N, d)
        return self._forward_autograd(self.W_in(flat), self.W_d(flat), B, N, d, T_len)

    def _forward_autograd(self, gi_all, wd_all, B, N, d, T_len):
        M = B * N
        dev = gi_all.device
        m = torch.zeros(M, d, device=dev)
        s = torch.zeros(M, d, device=dev)
        heat = torch.zeros(M, d, device=dev)
        outs = []
        for t in range(T_len):
            pre = (gi_all[t] / self.gate_scale + self.W_rec(s) / self.gate_scale) + self.W_in.bias
            f = torch.sigmoid(pre[:, :d])
            i = torch.sigmoid(pre[:, d:2 * d])
            o = torch.sigmoid(pre[:, 2 * d:3 * d])
            g = torch.tanh(pre[:, 3 * d:])
            a = f * m + i * g
            v = o * torch.tanh(a) + wd_all[t]
            theta = self.v_th * (1.0 + heat) if self.adaptive_threshold else self.v_th
            s = self.spike_fn(v - theta)
            m = a - s * self.v_th
            if self.adaptive_threshold:
                heat = self.beta_adapt * heat + s
            outs.append(s)
        out = torch.stack(outs)
        pooled = out.mean(dim=0) if self.pool == "mean" else out[-1]
        return pooled.view(B, N, d)
