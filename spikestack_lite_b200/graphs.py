"""Inference forward of a model captured in one CUDA graph.

The small configurations of the forward (one layer, d = 128) are bound by
launch and host overhead: some thirty launches, each behind Python-side
argument checks.  CapturedForward records the whole eager forward once into a
CUDA graph and replays it: the engine's entry points only enqueue kernels and
stream-ordered memsets on the current stream (no host synchronisation, no
allocation of their own), so the recording holds every launch of the forward.

The reference has no counterpart (its forward is eager PyTorch,
models/transformer.py:159-192); the outputs are the eager forward's, bit for
bit, because the same kernels run on the same buffers.
"""
import torch

from ._lib import EngineError


class CapturedForward:
    """`model(x)` for inputs of `example`'s shape, dtype and device, replayed
    from a CUDA graph.  An eager warm-up call first sizes the engine's
    workspace and PyTorch's caches, so nothing is allocated outside the graph's
    memory pool during capture.  Calling copies x into the graph's static input
    and returns the graph's static output (overwritten by the next call)."""

    def __init__(self, model, example):
        if not example.is_cuda:
            raise EngineError("CapturedForward: CUDA input required")
        self.model = model
        self.x = example.detach().clone()
        with torch.no_grad():
            model(self.x)
            torch.cuda.synchronize(self.x.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.y = model(self.x)
        torch.cuda.synchronize(self.x.device)

    def __call__(self, x):
        if x.shape != self.x.shape or x.dtype != self.x.dtype or x.device != self.x.device:
            raise EngineError(f"CapturedForward: input {tuple(x.shape)} {x.dtype} on {x.device} does not match the "
                              f"captured {tuple(self.x.shape)} {self.x.dtype} on {self.x.device}")
        self.x.copy_(x)
        self.graph.replay()
        return self.y
