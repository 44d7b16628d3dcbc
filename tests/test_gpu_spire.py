"""Spire planes (spk_spire_planes) against the reference's PyTorch composition.

SpireEncoder.forward in temporal mode (encode/spire.py:60-69) computes
v = (u - frontier) - temporal_frontier and the planes (v - dither[t] > 0); the
engine does it in one pass with the same fp32 operations, so the planes are
bit-identical, including values that sit exactly on a threshold."""
import pytest
import torch

from spikestack_lite_b200 import ops
from spikestack_lite_b200._lib import EngineError
from spikestack_lite_b200.engine import spire_engine

pytestmark = pytest.mark.gpu


def _reference(u, dither, frontier=None, tfront=None):
    v = u
    if frontier is not None:
        v = v - frontier.view(1, 1, -1)
    if tfront is not None:
        v = v - tfront.view(1, -1, 1)
    return (v.unsqueeze(-1) - dither.view(1, 1, 1, -1) > 0).float().permute(3, 0, 1, 2)


@pytest.mark.parametrize("B,N,d,T", [(8, 64, 128, 3), (4, 1024, 512, 4), (3, 7, 4, 1), (2, 33, 36, 5)])
def test_planes_bit_exact(B, N, d, T):
    g = torch.Generator(device="cuda").manual_seed(B * N + d)
    u = torch.randn(B, N, d, generator=g, device="cuda") * 0.3 + 0.5
    frontier = torch.ones(d, device="cuda") * 0.5 + torch.randn(d, generator=g, device="cuda") * 0.01
    tfront = torch.randn(1, N, 1, generator=g, device="cuda") * 0.02
    dither = torch.linspace(-0.05, 0.05, T, device="cuda").view(1, 1, 1, T)
    # a few values exactly on a threshold: v - dither == 0 gives no spike
    u[0, 0, :4] = frontier[:4] + tfront[0, 0, 0] + dither.view(-1)[0]
    planes = ops.spire_planes(u, dither, frontier, tfront)
    assert planes.shape == (T, B, N, d) and planes.is_contiguous()
    assert torch.equal(planes, _reference(u, dither.view(-1), frontier, tfront))


def test_reference_engine_entry_point():
    v = torch.randn(2, 16, 64, device="cuda") * 0.05
    dither = torch.linspace(-0.05, 0.05, 3, device="cuda")
    assert torch.equal(spire_engine.spire_dither(v, dither), _reference(v, dither))


def test_rejects_bad_arguments():
    with pytest.raises(EngineError):
        ops.spire_planes(torch.randn(2, 4, 6, device="cuda"), torch.zeros(2, device="cuda"))   # d % 4
    with pytest.raises(EngineError):
        ops.spire_planes(torch.randn(2, 4, 8, device="cuda"), torch.zeros(2, device="cuda"),
                         frontier=torch.zeros(4, device="cuda"))                                 # frontier size
    with pytest.raises(EngineError, match="CUDA"):
        ops.spire_planes(torch.randn(2, 4, 8), torch.zeros(2))
