"""The batch-512 model's true geometry -- seq 1024, input 256, d 512, 8 heads,
6 layers, T = 4 Spire planes, FFN x4, GSMC on, exact head on -- on a
two-sample slice of its batch (samples are independent through the whole
forward, so a slice runs every kernel at the geometry of the full batch: the
same K, N, sequence length, head split and row partition per sample).

Random-init weights from torch.manual_seed(0), as the benchmark builds them;
the oracle (oracle/spk_oracle.py, pinned to the reference's golden models)
runs the same state dict on the CPU.  The gates, stage by stage with teacher
forcing (each stage fed the oracle's own input for it):
  * Spire planes: flips only within rounding of the threshold;
  * per block: the engine's q, k, v and fc1 spikes computed from the oracle's
    layer-norm outputs -- zero flips outside the rounding band, count printed;
    the attention, mid-block residual and block output within 1e-4 x max|ref|
    of the oracle's block arithmetic fed the engine's own spikes;
  * GSMC: the pooled output against the oracle's cell;
  * logits end to end: within 1e-4 x max|ref| when no stage flipped a spike,
    else within 5e-2 (a flipped q, k or v spike changes a whole head's
    attention, and the change propagates through six blocks and the GSMC)."""
import numpy as np
import pytest
import torch

import spike_flips
from oracle import spk_oracle as O
from spikestack_lite_b200.transformer import SpikingTransformer

pytestmark = pytest.mark.gpu

C5 = dict(input_dim=256, d_model=512, seq_len=1024, num_classes=10, num_heads=8, num_layers=6, n_repeats=4,
          temporal=True, expansion=4, use_gsmc=True, use_exact=True, use_spikeskip=True)
SLICE = 2


@pytest.fixture(scope="module")
def c5():
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    m = SpikingTransformer(**C5).to(dev).eval()
    sd = {k: v.detach().cpu() for k, v in m.state_dict().items()}
    x = torch.randn(SLICE, C5["seq_len"], C5["input_dim"], generator=torch.Generator().manual_seed(1))
    cap = {}
    logits = O.transformer_forward(sd, x, C5["num_heads"], C5["num_layers"], use_gsmc=True, capture=cap)
    return {"m": m, "sd": sd, "x": x, "cap": cap, "logits": logits, "flips": {}}


def _block_input(cap, i):
    return cap["planes"] if i == 0 else cap[f"block{i - 1}_out"]


def test_c5_spire_planes(c5):
    m, cap, sd = c5["m"], c5["cap"], c5["sd"]
    with torch.no_grad():
        planes = m.encode(c5["x"].cuda()).cpu()
    assert planes.shape == cap["planes"].shape
    u = O._lin(sd, "embedding.projection", c5["x"])
    v = u - sd["embedding.frontier"].view(1, 1, -1) - sd["embedding.temporal_frontier"]
    margin = (v.unsqueeze(-1) - sd["embedding.dither"]).permute(3, 0, 1, 2)
    flips, far = spike_flips.count(planes, cap["planes"], margin)
    c5["flips"]["planes"] = flips
    print(f"\nC5 Spire planes: {planes.numel()} spikes, {flips} flipped ({far} outside the rounding band)")
    assert far == 0


@pytest.mark.parametrize("i", range(C5["num_layers"]))
def test_c5_block_spikes_teacher_forced(c5, i):
    m, cap, sd = c5["m"], c5["cap"], c5["sd"]
    x_in = _block_input(cap, i)
    st = O.block_stages(sd, f"blocks.{i}", x_in, C5["num_heads"])
    res = spike_flips.block_spike_flips(m.blocks[i], st)
    c5["flips"][f"block{i}"] = sum(f for f, _ in res.values())
    print(f"\nC5 block {i} spike flips (total, outside band): {res}")
    for name, (_, far) in res.items():
        assert far == 0, f"block {i} {name}: {far} spikes flipped away from the threshold"
    assert torch.equal(st["out"], cap[f"block{i}_out"])
    errs = spike_flips.block_stage_errors(m.blocks[i], sd, f"blocks.{i}", x_in, C5["num_heads"])
    print(f"C5 block {i}: stage errors given the engine's own spikes {errs}")
    for stage, e in errs.items():
        assert e < 1e-4, f"block {i} {stage}: rel err {e:.2e} with identical spikes"


def test_c5_gsmc_teacher_forced(c5):
    m, cap = c5["m"], c5["cap"]
    with torch.no_grad():
        pooled = m.gsmc(cap["block5_out"].cuda(), T=C5["n_repeats"]).cpu().numpy()
    ref = cap["gsmc_out"].numpy()
    off = int((np.abs(pooled - ref) > 1e-6).sum())
    c5["flips"]["gsmc"] = off
    print(f"\nC5 GSMC pooled output: {off} of {ref.size} values differ (spike flips / state rounding)")
    assert off <= max(2, ref.size // 10000)


def test_c5_logits_end_to_end(c5):
    m = c5["m"]
    with torch.no_grad():
        logits = m(c5["x"].cuda()).cpu().numpy()
    err = O.rel_err(logits, c5["logits"].numpy())
    total = sum(c5["flips"].values())
    print(f"\nC5 logits rel err {err:.2e}; spike flips by stage {c5['flips']} (total {total})")
    assert err < (1e-4 if total == 0 else 5e-2)
