"""Host composition of the temporal SpikingTransformer forward on the B200 engine.

Mirrors ``spikestack_lite.models.transformer.SpikingTransformer`` and
``spikestack_lite.encode.spire.SpireEncoder`` (models/transformer.py:41-192,
encode/spire.py:40-69): same constructor arguments, the same submodules and
parameter names (so reference state dicts load), created in the reference's
order so that one torch seed yields the same weights.  The host stays PyTorch;
the hot path runs in the engine (fc2 spike-linear, fused spiking attention,
fused GSMC recurrence).

Not mirrored (outside the forward hot path): the conv and text stems
(``use_conv_stem``, ``text_vocab`` raise), ``forward_text`` and the
exact-SNN latency loss; with ``use_exact=True`` the head's parameters exist
(for state-dict compatibility) but, as in the reference, forward() does not
use them.
"""
import torch
import torch.nn as nn

from . import ops
from ._lib import EngineError
from .attention import AstrocyteHebbianBlock, spike_fn
from .gsmc import FusedGSMC


class SpireEncoder(nn.Module):
    """Spire time-repetition encoder (encode/spire.py:40-69); in temporal mode
    returns the R binary planes (R, B, N, d) of (v - dither_r > 0)."""

    def __init__(self, input_dim, d_model, seq_len=784, n_repeats=3, threshold=0.5, temporal=False):
        super().__init__()
        self.d_model = d_model
        self.n_repeats = max(1, int(n_repeats))
        self.temporal = bool(temporal)
        self.projection = nn.Linear(input_dim, d_model)
        self.frontier = nn.Parameter(torch.ones(d_model) * threshold)
        self.temporal_frontier = nn.Parameter(torch.randn(1, seq_len, 1) * 0.02)
        self.dither = nn.Parameter(torch.linspace(-0.05, 0.05, self.n_repeats).view(1, 1, 1, self.n_repeats))

    def forward(self, x):
        # inference: the projection on the engine's tensor-core linear (as the blocks' projections)
        u = ops.engine_linear(self.projection, x)
        if u is None:
            u = self.projection(x)
        if (self.temporal and not torch.is_grad_enabled() and u.is_cuda and u.dtype == torch.float32
                and self.d_model % 4 == 0):
            # inference: the planes in one engine pass from u, (R, B, N, d)
            # contiguous as the reference engine's spire_dither returns them
            return ops.spire_planes(u, self.dither.float(), self.frontier, self.temporal_frontier)
        v = (u - self.frontier.view(1, 1, self.d_model) - self.temporal_frontier).float()
        if self.n_repeats == 1 and not self.temporal:
            return spike_fn(v)
        if self.temporal:
            return spike_fn(v.unsqueeze(0) - self.dither.float().view(-1, 1, 1, 1))
        return spike_fn(v.unsqueeze(-1) - self.dither.float()).permute(3, 0, 1, 2).mean(dim=0)


class _LatencyHeadParams(nn.Module):
    """Parameters of the exact-SNN SoftLatencyHead (nn/exact_head.py:55-71),
    kept for state-dict compatibility; not used by forward()."""

    def __init__(self, d_model, num_classes, t_max=40.0, time_steps=32):
        super().__init__()
        self.proj = nn.Linear(d_model, num_classes)
        self.theta = nn.Parameter(torch.zeros(num_classes))
        self.register_buffer("t_grid", torch.linspace(0.0, float(t_max), time_steps))


class SpikingTransformer(nn.Module):
    def __init__(self, input_dim=48, d_model=128, seq_len=64, num_classes=10, num_heads=4, v_levels=1,
                 num_layers=1, n_repeats=3, use_spikeskip=False, expansion=None, spike_readout=True,
                 temporal=False, spike_threshold=0.0, use_gsmc=False, gsmc_pool="mean", gsmc_readout=False,
                 use_exact=False, exact_weight=1.0, exact_beta_init=1.0, exact_beta_end=8.0,
                 use_conv_stem=False, conv_kernels=32, text_vocab=None, padding_idx=0):
        super().__init__()
        if use_conv_stem or text_vocab is not None:
            raise EngineError("SpikingTransformer: the conv and text stems are not part of this engine")
        self.d_model = d_model
        self.spike_readout = spike_readout
        self.temporal = bool(temporal)
        self.use_gsmc = bool(use_gsmc)
        self.use_exact = bool(use_exact)
        self.embedding = SpireEncoder(input_dim, d_model, seq_len, n_repeats=n_repeats, temporal=temporal)
        if expansion is None:
            expansion = 8 if use_spikeskip else 4  # models/transformer.py:93-96 (engine present)
        self.blocks = nn.ModuleList([
            AstrocyteHebbianBlock(d_model=d_model, num_heads=num_heads, expansion=expansion, v_levels=v_levels,
                                  use_spikeskip=use_spikeskip, spike_threshold=spike_threshold)
            for _ in range(num_layers)
        ])
        self.gsmc = None
        self.gsmc_readout = bool(gsmc_readout)
        if self.use_gsmc:
            if not self.temporal:
                raise ValueError("use_gsmc=True requires temporal=True (GSMC consumes the Spire T-planes).")
            self.gsmc = FusedGSMC(d_model=d_model, pool=gsmc_pool)
        self.use_spikeskip = use_spikeskip
        self.spike_threshold = float(spike_threshold)
        self.classifier = nn.Linear(d_model, num_classes)
        self.exact_head = _LatencyHeadParams(d_model, num_classes) if self.use_exact else None
        self.exact_weight = float(exact_weight)

    def load_reference_state_dict(self, sd, strict=True):
        """Load a reference state dict; maps fc2.* <-> fc2.linear.* between the
        dense and SpikeSkip FFN layouts (sparse/__init__.py:209)."""
        own = self.state_dict()
        fixed = {}
        for k, v in sd.items():
            if k not in own and ".ffn.fc2." in k:
                alt = k.replace(".ffn.fc2.", ".ffn.fc2.linear.")
                if alt not in own:
                    alt = k.replace(".ffn.fc2.linear.", ".ffn.fc2.")
                k = alt
            fixed[k] = torch.as_tensor(v)
        return self.load_state_dict(fixed, strict=strict)

    def encode(self, x):
        return self.embedding(x)

    def readout(self, context):
        if self.spike_readout:
            context = spike_fn(context)
        if self.temporal and self.gsmc is None:
            return self.classifier(context.mean(dim=(0, 2)))
        return self.classifier(context.mean(dim=1))

    def forward(self, x):
        if x.device.type != "cuda":
            raise EngineError("SpikingTransformer: CUDA input required (no CPU path)")
        context = self.embedding(x)
        context_norm = None  # the next block's norm1 of the context, when the engine computed it
        for i, block in enumerate(self.blocks):
            nxt = self.blocks[i + 1].norm1 if i + 1 < len(self.blocks) else None
            context, context_norm = block.forward_fused(context, context_norm, nxt)
        if self.gsmc is not None:
            context = self.gsmc(context, T=context.shape[0])
        pooled_over_time = self.temporal and self.gsmc is None
        if (self.spike_readout and not torch.is_grad_enabled() and context.dtype == torch.float32
                and context.dim() == (4 if pooled_over_time else 3) and context.shape[-1] % 4 == 0):
            # inference: both poolings (the latency head's and the classifier's) in one pass
            self._pooled_for_latency, pooled_spikes = ops.temporal_mean(context)
            return self.classifier(pooled_spikes)
        self._pooled_for_latency = context.mean(dim=(0, 2)) if pooled_over_time else context.mean(dim=1)
        return self.readout(context)
