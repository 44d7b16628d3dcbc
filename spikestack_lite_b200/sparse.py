"""Mirror of ``spikestack_lite.sparse`` (sparse/__init__.py) on the B200 engine.

Same public names and argument meanings: ``sparse_linear_forward``,
``sparse_multistep_forward``, ``alloc_csr_buffers``, ``SparseLinear`` (with
``.linear`` holding the nn.Linear parameters, so reference state dicts load
unchanged) and the patchable module attribute ``_cuda_engine``.

Differences, all deliberate:
* CUDA only.  The reference silently computes CPU tensors with nn.Linear;
  here a CPU tensor raises (the engine has no CPU path).
* ``forward_multistep`` hands the nn.Linear weight [N, K] to the kernel as is
  (the reference copies ``weight.t().contiguous()`` every call,
  sparse/__init__.py:166) and adds the bias in the kernel epilogue.
* The CSR of the layer's input is only materialised when asked for
  (``emit_csr=True``); the reference always rebuilds it, though nothing reads it.
"""
import torch

from . import ops
from .ops import engine_linear
from ._lib import EngineError
from .engine import sparse_engine

_cuda_engine = sparse_engine


def sparse_linear_forward(input, weightT, nnz_per_row, row_offsets, col_indices, values):
    """Fused CSR conversion + multiply (sparse/__init__.py:93-99)."""
    if _cuda_engine is None:
        raise EngineError("spikestack_lite_b200.sparse: engine unavailable")
    return _cuda_engine.sparse_forward(input, weightT, nnz_per_row, row_offsets, col_indices, values)


def sparse_multistep_forward(dense_input, weightT, nnz_per_row, row_offsets, col_indices, values, T):
    """Multi-timestep spike-linear (sparse/__init__.py:102-106)."""
    if _cuda_engine is None:
        raise EngineError("spikestack_lite_b200.sparse: engine unavailable")
    return _cuda_engine.sparse_multistep_forward(dense_input, weightT, nnz_per_row, row_offsets, col_indices, values,
                                                 T)


def alloc_csr_buffers(batch_size, in_features, device=None):
    """Reusable CSR buffers (sparse/__init__.py:180-188): nnz_per_row [B],
    row_offsets [B+1], col_indices [B*I] int32, values [B*I] float32."""
    device = device or "cuda"
    return (
        torch.empty(batch_size, dtype=torch.int32, device=device),
        torch.empty(batch_size + 1, dtype=torch.int32, device=device),
        torch.empty(batch_size * in_features, dtype=torch.int32, device=device),
        torch.empty(batch_size * in_features, dtype=torch.float32, device=device),
    )


class _SparseMatmulAutograd(torch.autograd.Function):
    """Engine forward, exact dense backward (sparse/__init__.py:116-145)."""

    @staticmethod
    def forward(ctx, flat, weight, engine, csr):
        nnz_per_row, row_offsets, col_indices, values = csr
        out = engine.sparse_forward(flat, weight.t().contiguous(), nnz_per_row, row_offsets, col_indices, values)
        ctx.save_for_backward(flat, weight)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        flat, weight = ctx.saved_tensors
        return grad_out @ weight, grad_out.t() @ flat, None, None


class _SpikeLinearAutograd(torch.autograd.Function):
    """Multi-plane spike-linear: engine forward (weight and bias passed to the
    kernel as they are), exact dense backward (sparse/__init__.py:148-177)."""

    @staticmethod
    def forward(ctx, inp, weight, bias, csr):
        out = ops.spike_linear(inp, weight=weight, bias=bias, csr=csr)
        ctx.save_for_backward(inp, weight)
        ctx.has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, grad_out):
        inp, weight = ctx.saved_tensors
        grad_inp = torch.matmul(grad_out, weight)
        grad_weight = torch.einsum("...bo,...bf->of", grad_out, inp)
        grad_bias = grad_out.reshape(-1, grad_out.shape[-1]).sum(0) if ctx.has_bias else None
        return grad_inp, grad_weight, grad_bias, None


class SparseLinear(torch.nn.Module):
    """Drop-in for spikestack_lite.sparse.SparseLinear (sparse/__init__.py:191-280)."""

    def __init__(self, in_features, out_features, bias=False, device=None, sparse_threshold=1024):
        super().__init__()
        self.linear = torch.nn.Linear(in_features, out_features, bias=bias, device=device or "cpu")
        self.in_features = in_features
        self.out_features = out_features
        self.sparse_threshold = sparse_threshold
        self.emit_csr = False
        self.csr = None  # per-plane CSR of the last forward_multistep input when emit_csr is set
        self._buf = None

    def _check(self, x):
        if x.device.type != "cuda":
            raise EngineError("SparseLinear: CUDA input required (the B200 engine has no CPU path)")

    def _csr_buffers(self, B, device):
        if self._buf is None or self._buf[0].device != device or self._buf[0].numel() < B:
            cap = max(int(B), 2048)
            self._buf = alloc_csr_buffers(cap, self.in_features, device)
        return self._buf

    def forward_single(self, input):
        """One plane (*, in_features) -> (*, out_features) (sparse/__init__.py:225-238)."""
        self._check(input)
        leading = input.shape[:-1]
        flat = input.reshape(-1, self.in_features).contiguous()
        if torch.is_grad_enabled() and (flat.requires_grad or self.linear.weight.requires_grad):
            out = _SparseMatmulAutograd.apply(flat, self.linear.weight, _cuda_engine,
                                              self._csr_buffers(flat.size(0), flat.device))
            if self.linear.bias is not None:
                out = out + self.linear.bias
        else:
            out = ops.spike_linear(flat, weight=self.linear.weight, bias=self.linear.bias)
        return out.view(*leading, self.out_features)

    def forward_multistep(self, dense_input, T=None):
        """(T, ..., in_features) -> (T, ..., out_features) (sparse/__init__.py:240-262)."""
        if dense_input.dim() == 2:
            return self.forward_single(dense_input)
        self._check(dense_input)
        if T is None:
            T = dense_input.size(0)
        leading = dense_input.shape[1:-1]
        flat = dense_input.reshape(T, -1, self.in_features).contiguous()
        csr = None
        if self.emit_csr:
            csr = ops.alloc_csr(T, flat.size(1), self.in_features, flat.device)
        out = _SpikeLinearAutograd.apply(flat, self.linear.weight, self.linear.bias, csr)
        self.csr = csr
        return out.view(T, *leading, self.out_features)

    def forward_bits(self, bits):
        """(*, in_features / 32) int32 packed spikes (bit b of word w = input
        column 32w + b) -> (*, out_features), on the engine's dense branch,
        inference only: the fc2 of SpikingFFN on fc1's packed spikes."""
        self._check(bits)
        return ops.spike_linear_bits(bits, self.in_features, self.linear.weight, self.linear.bias)

    def forward(self, x):
        """Density-dispatched forward (sparse/__init__.py:264-280): the
        spike-linear engine for wide layers (in_features >= sparse_threshold) at
        >= 90 % sparsity, as the reference; otherwise the reference's dense
        nn.Linear, run at inference on the engine's fp32-accurate tensor-core
        linear (spk_linear_act; all values count, negatives included, as in
        nn.Linear) and through nn.Linear itself under autograd or for shapes
        that op does not take (out_features <= 64, in_features % 4 != 0)."""
        self._check(x)
        if self.in_features >= self.sparse_threshold:
            with torch.no_grad():
                nnz = (x != 0).sum().item()
            if 1.0 - nnz / max(1, x.numel()) >= 0.90:
                return self.forward_multistep(x) if x.dim() >= 3 else self.forward_single(x)
        y = engine_linear(self.linear, x) if x.dtype == torch.float32 else None
        return y if y is not None else self.linear(x)
