"""Spike-flip accounting shared by the model parity tests.

A spike is a threshold decision, so an implementation whose pre-activation
differs from the reference's by rounding alone flips the spikes whose
reference pre-activation lies within that rounding of the threshold, and no
others.  count() separates the two kinds: flips inside a band around the
threshold (rounding, reported) and flips outside it (a real discrepancy, which
the tests require to be zero)."""
import torch

# Half-width of the rounding band, relative to max |pre-activation|: far above
# the fp32 rounding of a K <= 2048 dot product (~1e-6 relative), far below the
# distance of a genuinely wrong decision.
BAND_REL = 1e-4


def count(ours, ref, margin):
    """(flips, flips_outside_band) of spike tensor `ours` against `ref`, where
    `margin` is the reference's signed distance from the threshold (fp32)."""
    ours = torch.as_tensor(ours).float().cpu()
    ref = torch.as_tensor(ref).float().cpu()
    margin = torch.as_tensor(margin).float().cpu()
    diff = ours != ref
    band = BAND_REL * float(margin.abs().max()) if margin.numel() else 0.0
    far = margin.abs() > band
    return int(diff.sum()), int((diff & far).sum())


def block_spike_flips(blk, st):
    """Spike flips of one engine block's q, k, v and fc1 spikes, each computed
    by the engine from the reference's own layer-norm outputs (h1, h2) so
    that every flip is charged to the kernel that made the decision.
    Returns {name: (flips, flips_outside_band)}."""
    from spikestack_lite_b200 import ops

    dev = next(blk.parameters()).device
    h1 = st["h1"].to(dev)
    h2 = st["h2"].to(dev)
    a = blk.attn
    out = {}
    with torch.no_grad():
        q = ops.linear_act(h1, a.q_proj.weight, a.q_proj.bias, "heaviside", 0.0)
        k = ops.linear_act(h1, a.k_proj.weight, a.k_proj.bias, "heaviside", 0.0)
        v = ops.linear_act(h1, a.v_proj.weight, a.v_proj.bias, "vspike", st["tau"])
        act = ops.linear_act(h2, blk.ffn.fc1.weight, blk.ffn.fc1.bias, "heaviside", blk.ffn.threshold)
    out["q"] = count(q, st["q"], st["q_pre"])
    out["k"] = count(k, st["k"], st["k_pre"])
    out["v"] = count(v, st["v"], (torch.tanh(st["v_pre"]) + 1.0) / 2.0 - st["tau"])
    out["act"] = count(act, st["act"], st["fc1_pre"])
    return out
