"""Two-rank (gloo, CPU) tests of the batch-sharded multi-process path:
collectives, sharded model forward against the single-process result and the
reference's golden logits, uneven batches, and a rank that leaves early."""
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import dist_workers as W
from spikestack_lite_b200.dist import shard_bounds

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, tmp_path, *extra, world=2):
    """Run fn(rank, world, port, out_dir, *extra) as `world` spawned processes."""
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path)) + extra) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode is not None, "worker did not finish"
    return [json.load(open(os.path.join(tmp_path, f"rank{r}.json"))) for r in range(world)]


def test_shard_bounds():
    assert shard_bounds(512, 0, 8) == (0, 64)
    assert shard_bounds(512, 7, 8) == (448, 512)
    with pytest.raises(ValueError):
        shard_bounds(10, 0, 4)


def test_max_over_ranks_and_row_gather(tmp_path):
    res = _run(W.collectives, tmp_path)
    for r in res:
        assert r["max"] == 11.5
        assert r["rows"] == [[0.0] * 3, [0.0] * 3, [1.0] * 3, [1.0] * 3]


def test_sharded_model_matches_single_process(tmp_path, golden):
    path = os.path.join(HERE, "golden", "model_c5_tiny.npz")
    res = _run(W.sharded_model, tmp_path, path)
    z = golden("model_c5_tiny")
    for r in res:
        logits = np.asarray(r["logits"], dtype=np.float32)
        assert logits.shape == z["logits"].shape
        np.testing.assert_allclose(logits, z["logits"], rtol=0, atol=1e-6 * float(np.abs(z["logits"]).max()))
    np.testing.assert_array_equal(np.asarray(res[0]["logits"]), np.asarray(res[1]["logits"]))


def test_rank_leaving_early_fails_the_collective(tmp_path):
    res = _run(W.dead_peer, tmp_path)
    assert res[1] == {"left": True}
    assert res[0]["error"] is not None
