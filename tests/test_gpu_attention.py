"""Spiking linear attention on the GPU against the oracle, the golden vectors
produced by the reference, and the reference's own CUDA engine."""
import numpy as np
import pytest
import torch

from oracle import spk_oracle as O
from spikestack_lite_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _spk(shape, p, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.rand(*shape, generator=g, device="cuda") < p).float()


def _lam(d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.sigmoid(torch.empty(d, device="cuda").uniform_(5.0, 8.0, generator=g))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_fused_attention_golden(golden, tag):
    z = golden("attention")
    q, k, v = (torch.from_numpy(z[f"{tag}_{n}"]).cuda() for n in "qkv")
    out = ops.spiking_attention(q, k, v, torch.from_numpy(z[f"{tag}_lam"]).cuda(), int(z[f"{tag}_heads"]),
                                float(z[f"{tag}_eps"]))
    assert O.rel_err(out.cpu().numpy(), z[f"{tag}_attn"]) < TOL


@pytest.mark.parametrize("shape,heads", [
    ((4, 2, 256, 256), 4),     # dh = 64
    ((3, 4, 64, 128), 4),      # the CPU model geometry: dh = 32
    ((2, 1, 100, 32), 2),      # dh = 16, ragged sequence length
    ((4, 8, 4096, 512), 8),    # the attention config's per-sample shape at B = 8
])
def test_fused_attention_vs_oracle(shape, heads):
    q, k, v = (_spk(shape, 0.15, s) for s in (1, 2, 3))
    lam = _lam(shape[-1], 4)
    out = ops.spiking_attention(q, k, v, lam, heads)
    ref = O.spiking_attention(q.cpu(), k.cpu(), v.cpu(), lam.cpu(), heads)
    assert O.rel_err(out.cpu().numpy(), ref.numpy()) < TOL


def test_decay_and_normalize_ops(ref_engine):
    ref = ref_engine("attention_ref")
    k = _spk((2, 3, 300, 64), 0.3, 5)
    lam = _lam(64, 6)
    ours = ops.apply_channel_decay(k, lam)
    torch.testing.assert_close(ours, ref.apply_channel_decay(k, lam), rtol=0, atol=0)
    assert O.rel_err(ours.cpu().numpy(), O.channel_decay(k.cpu(), lam.cpu()).numpy()) < 1e-6
    numer = torch.rand(5, 7, 9, device="cuda")
    denom = torch.rand(5, 7, 9, device="cuda")
    n1 = ops.fused_normalize_attention(numer, denom, 1e-6)
    torch.testing.assert_close(n1, ref.fused_normalize_attention(numer, denom, 1e-6), rtol=0, atol=0)


def test_attention_zero_keys_give_zero_output():
    q = _spk((1, 2, 64, 64), 0.5, 7)
    k = torch.zeros_like(q)
    v = _spk((1, 2, 64, 64), 0.5, 8)
    out = ops.spiking_attention(q, k, v, _lam(64, 9), 2)
    assert torch.count_nonzero(out).item() == 0
