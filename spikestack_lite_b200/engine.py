"""Engine objects with the reference's pybind names.

The reference loads four torch extensions and keeps them in module globals
that its Python layer calls (and its tests monkeypatch):

    spikestack_lite.sparse._cuda_engine          sparse_forward, sparse_multistep_forward, dense_to_csr_gpu
                                                 (sparse_linear.cu:728-739)
    spikestack_lite.nn.attention._attn_cuda_engine  apply_channel_decay, fused_normalize_attention
                                                 (attention_cuda.cu:109-112)
    spikestack_lite.nn.gsmc._gsmc_cuda_engine    fused_gsmc_step (gsmc_cuda.cu:129-132)
    spikestack_lite.encode.spire._spire_cuda_engine  spire_dither (encode/src/spire_cuda.cu:60-62)

The objects below answer to the same names and argument lists, backed by
libspk_b200.so.  ``install(spikestack_lite)`` swaps them into an imported
reference package, which is the literal drop-in; the package's own mirror
modules (sparse, attention, gsmc, transformer) use them directly.
"""
from . import ops


class SparseEngine:
    """Replacement for the SpikeSkip engine module (``sparse._cuda_engine``)."""

    name = "spikestack_lite_b200.sparse"

    def __init__(self, branch="auto"):
        self.branch = branch

    def sparse_forward(self, input, weightT, nnz_per_row, row_offsets, col_indices, values):
        return ops.sparse_forward(input, weightT, nnz_per_row, row_offsets, col_indices, values, branch=self.branch)

    def sparse_multistep_forward(self, dense_input, weightT, nnz_per_row, row_offsets, col_indices, values, T):
        return ops.sparse_multistep_forward(dense_input, weightT, nnz_per_row, row_offsets, col_indices, values, T,
                                            branch=self.branch)

    def dense_to_csr_gpu(self, dense_input):
        return ops.dense_to_csr_gpu(dense_input)


class AttentionEngine:
    """Replacement for ``nn.attention._attn_cuda_engine``."""

    name = "spikestack_lite_b200.attention"

    def apply_channel_decay(self, k, lam):
        return ops.apply_channel_decay(k, lam)

    def fused_normalize_attention(self, numer, denom, eps):
        return ops.fused_normalize_attention(numer, denom, eps)

    # new fused entry point (no reference counterpart)
    def spiking_attention(self, q, k, v, lam, heads, eps=1e-6):
        return ops.spiking_attention(q, k, v, lam, heads, eps)


class SpireEngine:
    """Replacement for ``encode.spire._spire_cuda_engine``."""

    name = "spikestack_lite_b200.spire"

    def spire_dither(self, v, dither):
        return ops.spire_dither(v, dither)


class GsmcEngine:
    """Replacement for ``nn.gsmc._gsmc_cuda_engine``."""

    name = "spikestack_lite_b200.gsmc"

    def fused_gsmc_step(self, gi, gr, wd, bias, m, s, heat, v_th, gate_scale, adaptive_threshold, beta_adapt):
        return ops.fused_gsmc_step(gi, gr, wd, bias, m, s, heat, v_th, gate_scale, adaptive_threshold, beta_adapt)

    # new fused entry point (no reference counterpart)
    def gsmc_forward(self, gi_all, wd_all, w_rec, bias, v_th, gate_scale, adaptive, beta, pool="mean"):
        return ops.gsmc_forward(gi_all, wd_all, w_rec, bias, v_th, gate_scale, adaptive, beta, pool)


sparse_engine = SparseEngine()
attention_engine = AttentionEngine()
gsmc_engine = GsmcEngine()
spire_engine = SpireEngine()


def install(reference_pkg):
    """Point an imported reference package (``import spikestack_lite``) at this
    engine: its SparseLinear, attention and GSMC modules then run on the B200
    kernels with no other change."""
    import importlib

    sparse = importlib.import_module(reference_pkg.__name__ + ".sparse")
    attn = importlib.import_module(reference_pkg.__name__ + ".nn.attention")
    gsmc = importlib.import_module(reference_pkg.__name__ + ".nn.gsmc")
    sparse._cuda_engine = sparse_engine
    attn._attn_cuda_engine = attention_engine
    gsmc._gsmc_cuda_engine = gsmc_engine
    try:
        spire = importlib.import_module(reference_pkg.__name__ + ".encode.spire")
    except ImportError:
        spire = None
    if spire is not None:
        spire._spire_cuda_engine = spire_engine
    return reference_pkg
