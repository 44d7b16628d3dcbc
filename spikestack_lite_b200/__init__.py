"""B200 (sm_100a) engine for the temporal forward hot path of SpikeStack Lite.

Hand-written CUDA kernels behind a C ABI (include/spikestack_b200.h,
libspk_b200.so) with a thin PyTorch host that mirrors the reference's own
API: ``sparse`` (spike-linear ops, SparseLinear), ``attention``
(AstrocyteHebbianAttention, SpikingFFN, AstrocyteHebbianBlock), ``gsmc``
(FusedGSMC) and ``transformer`` (SpikingTransformer host composition);
``engine`` holds drop-in engine objects with the reference's pybind names and
``engine.install(spikestack_lite)`` swaps them into an imported reference.
"""
from . import _lib, ops  # noqa: F401
from ._lib import EngineError, launch_count  # noqa: F401

__version__ = "1.0.0"


def load():
    """Load the native library (raises EngineError when it is not built)."""
    return _lib.load()
