"""The C ABI library: it loads, exports every entry point include/spikestack_b200.h
declares, answers the size queries and rejects bad arguments with a status
and a message -- all without a GPU (no compute call is made)."""
import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "spikestack_b200.h")


@pytest.fixture(scope="module")
def lib():
    from spikestack_lite_b200 import build, _lib

    build.build()
    return _lib.load()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spk_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "spk_spike_linear" in names and "spk_csr_compact" in names and len(names) >= 18


def test_library_exports_every_declared_symbol(lib):
    from spikestack_lite_b200 import _lib

    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string(lib):
    assert lib.spk_version() >= 10000
    assert isinstance(lib.spk_last_error(), bytes)


def test_workspace_queries(lib):
    assert lib.spk_csr_workspace_bytes(3, 16384, 512) > 256
    assert lib.spk_csr_workspace_bytes(0, 1, 1) == 0
    assert lib.spk_spike_linear_workspace_bytes(3, 16384, 512, 128, 0) >= lib.spk_csr_workspace_bytes(3, 16384, 512)
    assert lib.spk_sparse_forward_workspace_bytes(3, 16384, 512, 128) > 0
    assert lib.spk_attention_workspace_bytes(256, 4096, 8, 64) >= 4 * 256 * 8 * 64 * 65
    assert lib.spk_gsmc_workspace_bytes(1024, 64) >= 3 * 4 * 1024 * 64


def test_invalid_arguments_are_rejected(lib):
    from spikestack_lite_b200._lib import SPK_EINVAL, SPK_EWORKSPACE

    rc = lib.spk_spike_linear(None, 1, 4, 8, None, 0, 8, 1, 8, None, None, None, None, None, None, None, 0, 0, None,
                              0, None)
    assert rc == SPK_EINVAL
    assert b"non-null" in lib.spk_last_error()
    rc = lib.spk_csr_compact(ctypes.c_void_p(16), 1, 4, 0, None, None, None, None, None, 0, None, 0, None)
    assert rc == SPK_EINVAL
    rc = lib.spk_csr_compact(ctypes.c_void_p(16), 1, 4, 8, None, ctypes.c_void_p(16), ctypes.c_void_p(16), None,
                             ctypes.c_void_p(16), 32, None, 0, None)
    assert rc == SPK_EWORKSPACE
    rc = lib.spk_spiking_attention(*([ctypes.c_void_p(16)] * 4), 1, 8, 2, 24, 1e-6, ctypes.c_void_p(16), None, 0,
                                   None)
    assert rc == SPK_EINVAL and b"head width" in lib.spk_last_error()
    rc = lib.spk_csr_compact(ctypes.c_void_p(16), 1, 1 << 20, 1 << 12, None, *([ctypes.c_void_p(16)] * 2), None,
                             ctypes.c_void_p(16), 0, None, 0, None)
    assert rc == SPK_EINVAL and b"int32" in lib.spk_last_error()


def test_python_ops_refuse_cpu_tensors(lib):
    import torch

    from spikestack_lite_b200 import ops
    from spikestack_lite_b200._lib import EngineError

    with pytest.raises(EngineError, match="CUDA"):
        ops.spike_linear(torch.zeros(2, 8), weight=torch.zeros(4, 8))
    with pytest.raises(EngineError, match="CUDA"):
        ops.csr_compact(torch.zeros(2, 8))
    with pytest.raises(EngineError, match="CUDA"):
        ops.spiking_attention(*(torch.zeros(1, 4, 8) for _ in range(3)), torch.ones(8), 2)


def test_add_layernorm_rejects_bad_arguments(lib):
    from spikestack_lite_b200._lib import SPK_EINVAL, SPK_EUNSUPPORTED, SPK_OK

    p = ctypes.c_void_p(256)
    assert lib.spk_add_layernorm(None, None, None, None, 0, 512, 1e-5, None, None, None) == SPK_OK  # no rows
    assert lib.spk_add_layernorm(p, None, None, None, 4, 510, 1e-5, None, p, None) == SPK_EINVAL
    assert b"multiple of 4" in lib.spk_last_error()
    assert lib.spk_add_layernorm(p, None, None, None, 4, 2048, 1e-5, None, p, None) == SPK_EUNSUPPORTED
    assert lib.spk_add_layernorm(p, p, None, None, 4, 512, 1e-5, None, p, None) == SPK_EINVAL  # D without H
    assert lib.spk_add_layernorm(ctypes.c_void_p(260), None, None, None, 4, 512, 1e-5, None, p, None) == SPK_EINVAL
    assert b"aligned" in lib.spk_last_error()
    assert lib.spk_add_layernorm(p, None, None, None, 4, 512, -1.0, None, p, None) == SPK_EINVAL
