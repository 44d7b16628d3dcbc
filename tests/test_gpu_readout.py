"""Readout pooling (spk_temporal_mean) against PyTorch.

SpikingTransformer's classifier input is the mean of spike(context) over time
and positions (models/transformer.py:159-192; over positions only after GSMC),
and the latency head's input the mean of the context itself.  Spike counts are
exact in fp32 and scaled by the same 1/n as torch's mean, so the classifier's
input is bit-identical; the plain mean differs only in summation order."""
import pytest
import torch

from spikestack_lite_b200 import ops
from spikestack_lite_b200._lib import EngineError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(3, 256, 64, 128), (4, 8, 1024, 512), (1, 5, 7, 36), (2, 3, 50, 1024)])
def test_temporal_context(shape):
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = torch.randn(*shape, generator=g, device="cuda")
    mx, ms = ops.temporal_mean(x)
    assert torch.equal(ms, (x > 0).float().mean(dim=(0, 2)))
    torch.testing.assert_close(mx, x.mean(dim=(0, 2)), rtol=1e-5, atol=1e-6)


def test_gsmc_pooled_context():
    x = torch.randn(16, 300, 64, device="cuda")
    mx, ms = ops.temporal_mean(x)
    assert torch.equal(ms, (x > 0).float().mean(dim=1))
    torch.testing.assert_close(mx, x.mean(dim=1), rtol=1e-5, atol=1e-6)


def test_rejects_bad_arguments():
    with pytest.raises(EngineError):
        ops.temporal_mean(torch.randn(2, 3, 4, 6, device="cuda"))     # d % 4
    with pytest.raises(EngineError):
        ops.temporal_mean(torch.randn(2, 8, device="cuda"))           # rank
    with pytest.raises(EngineError, match="CUDA"):
        ops.temporal_mean(torch.randn(2, 3, 8))
