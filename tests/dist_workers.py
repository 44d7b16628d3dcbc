"""Worker bodies for the two-rank gloo tests (spawned processes; CPU only).

Each worker sets up the torchrun-style environment for its rank, runs one
scenario and writes its result to <out_dir>/rank<r>.json."""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _env(rank, world, port):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)


def _write(out_dir, rank, obj):
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(obj, f)


def collectives(rank, world, port, out_dir):
    _env(rank, world, port)
    import torch

    from spikestack_lite_b200.dist import RankGroup

    g = RankGroup("gloo", timeout_s=30).init()
    res = {"max": g.max(10 * rank + 1.5)}
    rows = g.gather_rows(torch.full((2, 3), float(rank)))
    res["rows"] = rows.tolist()
    g.barrier()
    g.close()
    _write(out_dir, rank, res)


def sharded_model(rank, world, port, out_dir, golden_path):
    """Batch-sharded oracle forward of a reference golden model: each rank runs
    its slice, the logits are gathered in batch order."""
    _env(rank, world, port)
    import numpy as np
    import torch

    from oracle import spk_oracle as O
    from spikestack_lite_b200.dist import RankGroup, sharded_forward

    torch.set_num_threads(1)
    z = np.load(golden_path)
    cfg = O.model_config_from_golden(z)
    sd = O.state_dict_from_golden(z)

    def fn(xs):
        return O.transformer_forward(sd, xs.numpy(), cfg["num_heads"], cfg["num_layers"],
                                     use_gsmc=cfg.get("use_gsmc", False))

    g = RankGroup("gloo", timeout_s=60).init()
    logits = sharded_forward(fn, torch.from_numpy(np.asarray(z["x"])), g)
    g.close()
    _write(out_dir, rank, {"logits": logits.tolist()})


def dead_peer(rank, world, port, out_dir):
    """Rank 1 leaves before the collective; rank 0's gather must fail, not hang."""
    _env(rank, world, port)
    import torch

    from spikestack_lite_b200.dist import RankGroup

    g = RankGroup("gloo", timeout_s=5).init()
    if rank == 1:
        _write(out_dir, rank, {"left": True})
        os._exit(0)  # leaves between steps, with nothing in flight
    try:
        g.gather_rows(torch.zeros(1, 2))
        _write(out_dir, rank, {"error": None})
    except Exception as e:  # noqa: BLE001 -- any collective failure is the expected outcome
        _write(out_dir, rank, {"error": type(e).__name__})
    os._exit(0)
