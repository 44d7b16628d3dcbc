"""Residual add + layer norm (spk_add_layernorm) against PyTorch fp32.

The pre-norm block computes x + branch(...) and nn.LayerNorm of the sum
(nn/attention.py:174-177); the engine does both in one pass.  The sum is the
same fp32 addition (bit-exact); the normalised output is within rounding of
torch's layer norm (a different order of the mean / variance sums)."""
import pytest
import torch
import torch.nn.functional as F

from spikestack_lite_b200 import ops
from spikestack_lite_b200._lib import EngineError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(4, 64, 1024, 512), (3, 256, 64, 128), (7, 96), (5, 1024), (3, 4), (1000, 36)])
@pytest.mark.parametrize("with_delta", [True, False])
def test_matches_torch(shape, with_delta):
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    d = shape[-1]
    x = torch.randn(*shape, generator=g, device="cuda") * 3 + 1
    delta = torch.randn(*shape, generator=g, device="cuda") if with_delta else None
    w = torch.randn(d, generator=g, device="cuda")
    b = torch.randn(d, generator=g, device="cuda")
    h, y = ops.add_layernorm(x, delta, w, b, 1e-5)
    h_ref = x + delta if with_delta else x
    assert torch.equal(h, h_ref)
    y_ref = F.layer_norm(h_ref, (d,), w, b, 1e-5)
    torch.testing.assert_close(y, y_ref, rtol=1e-5, atol=1e-5)


def test_no_affine_and_spike_inputs():
    # binary inputs (the Spire planes entering the first block), identity affine
    x = (torch.rand(4, 32, 100, 128, device="cuda") < 0.3).float()
    _, y = ops.add_layernorm(x, None)
    torch.testing.assert_close(y, F.layer_norm(x, (128,), eps=1e-5), rtol=1e-5, atol=1e-5)
    # a constant row: zero variance -> (x - mean) = 0 exactly, y = beta
    c = torch.full((2, 128), 0.75, device="cuda")
    beta = torch.randn(128, device="cuda")
    _, yc = ops.add_layernorm(c, None, torch.ones(128, device="cuda"), beta)
    assert torch.equal(yc, beta.expand_as(yc))


def test_block_forward_matches_reference_composition():
    from spikestack_lite_b200.attention import AstrocyteHebbianBlock

    torch.manual_seed(0)
    blk = AstrocyteHebbianBlock(d_model=128, num_heads=4, expansion=4, use_spikeskip=True).cuda().eval()
    x = torch.randn(3, 2, 64, 128, device="cuda")
    with torch.no_grad():
        fused, nrm = blk.forward_fused(x, None, blk.norm2)
        ln1 = blk.norm1(x)
        h = x + blk.attn(ln1)
        ref = h + blk.ffn(blk.norm2(h))
    # outputs differ only where an internal spike flipped on a rounding-level difference
    bad = ((fused - ref).abs() > 1e-4 * ref.abs().max()).float().mean().item()
    assert bad < 1e-3
    torch.testing.assert_close(nrm, blk.norm2(fused), rtol=1e-5, atol=1e-5)


def test_rejects_unsupported():
    x = torch.randn(4, 2048, device="cuda")
    with pytest.raises(EngineError):
        ops.add_layernorm(x, None)                        # d above 1024
    with pytest.raises(EngineError):
        ops.add_layernorm(torch.randn(4, 6, device="cuda"), None)  # d % 4 != 0
    with pytest.raises(EngineError):
        ops.add_layernorm(x, torch.randn(4, 1024, device="cuda"))  # shape mismatch
