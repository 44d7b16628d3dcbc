"""Multi-process plumbing for the batch-sharded forward (one process per GPU).

The forward shards by batch: samples are independent through every layer
(per-token LayerNorm and GSMC, per-sample attention and readout), so rank r
runs the model on its contiguous slice of the batch and one all-gather of
the logits rebuilds the full batch -- the only collective on the path.

Rank, world size and local rank come from the torchrun environment
(RANK / WORLD_SIZE / LOCAL_RANK, MASTER_ADDR / MASTER_PORT).  With backend
"nccl" tensors live on cuda:LOCAL_RANK; with "gloo" (CPU tests) on the CPU.
"""
import datetime
import os

import torch


class RankGroup:
    """This process's place in the job plus the few collectives the path uses."""

    def __init__(self, backend="nccl", timeout_s=120):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.timeout_s = timeout_s
        self.pg = False

    @property
    def device(self):
        return torch.device("cuda", self.local) if self.backend == "nccl" else torch.device("cpu")

    def init(self):
        if self.world > 1 and not self.pg:
            import torch.distributed as dist

            kw = {"timeout": datetime.timedelta(seconds=self.timeout_s)}
            if self.backend == "nccl":
                kw["device_id"] = self.device
            dist.init_process_group(self.backend, **kw)
            self.pg = True
        return self

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x):
        """Max of a Python number over all ranks (every rank gets the result)."""
        if not self.pg:
            return x
        import torch.distributed as dist

        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_rows(self, local):
        """Concatenate every rank's [n_r, ...] block in rank order (equal n_r)."""
        if not self.pg:
            return local
        import torch.distributed as dist

        local = local.contiguous()
        out = torch.empty((local.shape[0] * self.world,) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        if self.backend == "nccl":
            dist.all_gather_into_tensor(out, local)
        else:
            dist.all_gather(list(out.chunk(self.world)), local)
        return out

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()
            self.pg = False


def shard_bounds(batch, rank, world):
    """[lo, hi) of rank's contiguous batch slice; the batch must split evenly."""
    if batch % world:
        raise ValueError(f"batch {batch} does not split evenly over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def sharded_forward(fn, x, group, chunk=None):
    """fn over this rank's slice of x (optionally in chunks of `chunk` samples),
    then the logits of all ranks gathered in batch order."""
    lo, hi = shard_bounds(x.shape[0], group.rank, group.world)
    xs = x[lo:hi]
    step = chunk or xs.shape[0]
    local = torch.cat([fn(xs[i:i + step]) for i in range(0, xs.shape[0], step)])
    return group.gather_rows(local)
