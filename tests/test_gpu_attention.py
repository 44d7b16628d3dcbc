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


@pytest.mark.parametrize("shape,heads", [
    ((4, 64, 64, 512), 8),     # 1024 (bt, head group) units: several per CTA, both accumulator buffers
    ((2, 3, 100, 128), 2),     # ragged sequence (not a multiple of 32 or 128), dh = 64
    ((1, 2, 37, 256), 16),     # dh = 16: eight heads per 128-channel group, 37 positions
    ((1, 1, 300, 384), 12),    # dh = 32, three groups, partial last tile
])
def test_tensor_core_attention_geometries(shape, heads):
    q, k, v = (_spk(shape, 0.15, s) for s in (11, 12, 13))
    lam = _lam(shape[-1], 14)
    out = ops.spiking_attention(q, k, v, lam, heads)
    ref = O.spiking_attention(q.cpu(), k.cpu(), v.cpu(), lam.cpu(), heads)
    assert O.rel_err(out.cpu().numpy(), ref.numpy()) < TOL


def test_tensor_core_attention_real_valued_inputs():
    """q and v that bf16 does not hold exactly take the hi/lo split passes (k is always split).
    k stays positive so that the key mass, and so the denominator, is well conditioned."""
    g = torch.Generator(device="cuda").manual_seed(21)
    shape = (2, 2, 200, 256)
    q = torch.rand(*shape, generator=g, device="cuda")
    k = torch.rand(*shape, generator=g, device="cuda")
    v = torch.randn(*shape, generator=g, device="cuda")
    lam = _lam(256, 22)
    out = ops.spiking_attention(q, k, v, lam, 4)
    ref = O.spiking_attention(q.cpu(), k.cpu(), v.cpu(), lam.cpu(), 4)
    assert O.rel_err(out.cpu().numpy(), ref.numpy()) < TOL


def test_tensor_core_attention_mixed_exactness():
    """Only some positions hold non-bf16 values: per-warp exact paths next to fast ones."""
    shape = (1, 4, 256, 128)
    q, k, v = (_spk(shape, 0.2, s) for s in (31, 32, 33))
    q[0, 1, 37, 5] = 0.3
    v[0, 2, 200, 100] = 0.7
    lam = _lam(128, 34)
    out = ops.spiking_attention(q, k, v, lam, 2)
    ref = O.spiking_attention(q.cpu(), k.cpu(), v.cpu(), lam.cpu(), 2)
    assert O.rel_err(out.cpu().numpy(), ref.numpy()) < TOL


def test_tensor_core_attention_zero_keys():
    q = _spk((1, 3, 130, 128), 0.5, 41)
    k = torch.zeros_like(q)
    v = _spk((1, 3, 130, 128), 0.5, 42)
    out = ops.spiking_attention(q, k, v, _lam(128, 43), 2)
    assert torch.count_nonzero(out).item() == 0


def _pack(S):
    """fp32 0 / 1 spikes [..., d] -> int32 words [..., d/32] (bit b of word w = channel 32w + b)."""
    shifts = torch.arange(32, device=S.device, dtype=torch.int64)
    words = (S.view(*S.shape[:-1], S.shape[-1] // 32, 32).long() << shifts).sum(-1)
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)


@pytest.mark.parametrize("shape,heads", [
    ((4, 2, 256, 256), 4),     # dh = 64
    ((2, 1, 100, 128), 4),     # dh = 32, ragged sequence length
    ((1, 3, 130, 128), 8),     # dh = 16, a partial last tile
    ((4, 8, 4096, 512), 8),    # the attention config's per-sample shape at B = 8
])
def test_packed_attention_matches_the_fp32_form(shape, heads):
    """Attention over packed q, k, v gives the fp32-input attention's output bit
    for bit (the kernels expand the words into the same staging values)."""
    q, k, v = (_spk(shape, 0.15, s) for s in (11, 12, 13))
    lam = _lam(shape[-1], 14)
    want = ops.spiking_attention(q, k, v, lam, heads)
    got = ops.spiking_attention_bits(_pack(q), _pack(k), _pack(v), lam, heads)
    assert torch.equal(ops.unpack_spikes(_pack(q), shape[-1]), q)
    assert torch.equal(got, want)
