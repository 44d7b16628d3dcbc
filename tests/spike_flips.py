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
    by the block's own spike path from the reference's own layer-norm outputs
    (h1, h2), so that every flip is charged to the kernel that made the
    decision.  Returns {name: (flips, flips_outside_band)}."""
    dev = next(blk.parameters()).device
    out = {}
    rec = {}
    with torch.no_grad():
        q, k, v = blk.attn.spikes(st["h1"].to(dev))
        blk.ffn(st["h2"].to(dev), rec)
    out["q"] = count(q, st["q"], st["q_pre"])
    out["k"] = count(k, st["k"], st["k_pre"])
    out["v"] = count(v, st["v"], (torch.tanh(st["v_pre"]) + 1.0) / 2.0 - st["tau"])
    out["act"] = count(rec["act"], st["act"], st["fc1_pre"])
    return out


def block_stage_errors(blk, sd, prefix, x_in, heads):
    """The engine block on x_in with its stages recorded, against the oracle's
    block arithmetic fed the engine's own q, k, v and fc1 spikes: relative
    errors (max |a - b| / max |b|) of the attention, the mid-block residual and
    the block output -- rounding only, whatever spikes flipped."""
    from oracle import spk_oracle as O

    dev = next(blk.parameters()).device
    rec = {}
    with torch.no_grad():
        out = blk.forward_fused(x_in.to(dev), record=rec)[0]
        assert torch.equal(out, blk(x_in.to(dev))), "the recorded forward differs from the block's forward"
    cpu = {k: v.float().cpu() for k, v in rec.items()}
    ref = O.block_from_spikes(sd, prefix, x_in, heads, cpu["q"], cpu["k"], cpu["v"], cpu["act"])
    return {"attn": O.rel_err(cpu["attn"].numpy(), ref["attn"].numpy()),
            "x_mid": O.rel_err(cpu["x_mid"].numpy(), ref["x_mid"].numpy()),
            "out": O.rel_err(out.cpu().numpy(), ref["out"].numpy())}
