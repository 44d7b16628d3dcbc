"""Spike -> CSR compaction on the GPU: bit-exact against the oracle (and against
the reference's own CUDA engine where it is valid), across the edge cases the
reference code is exposed to."""
import numpy as np
import pytest
import torch

from oracle import spk_oracle as O
from spikestack_lite_b200 import ops

pytestmark = pytest.mark.gpu


def _check_csr(S, out):
    exp = O.csr_planes(S)
    np.testing.assert_array_equal(out["nnz_row"].cpu().numpy(), exp[0])
    np.testing.assert_array_equal(out["row_ptr"].cpu().numpy(), exp[1])
    np.testing.assert_array_equal(out["col_idx"].cpu().numpy(), exp[2])
    np.testing.assert_array_equal(out["values"].cpu().numpy(), exp[3])
    np.testing.assert_array_equal(out["plane_ptr"].cpu().numpy(), exp[4])


@pytest.mark.parametrize("T,M,K,p", [
    (1, 1, 1, 1.0),          # smallest
    (3, 257, 512, 0.10),     # the isolated spike-linear geometry, odd M
    (2, 303, 100, 0.3),      # K not a multiple of 32
    (4, 1000, 2048, 0.05),   # wide rows (smaller row tiles)
    (1, 64, 33, 0.0),        # empty plane
    (2, 130, 64, 1.0),       # full planes
    (1, 70000, 32, 0.2),     # beyond the reference's 65536-row scan limit
])
def test_csr_bit_exact(T, M, K, p):
    g = torch.Generator(device="cuda").manual_seed(T * 7 + M + K)
    S = (torch.rand(T, M, K, generator=g, device="cuda") < p).float()
    _check_csr(S.cpu().numpy(), ops.csr_compact(S))


def test_csr_predicate_negative_nan_real_values():
    g = torch.Generator(device="cuda").manual_seed(5)
    S = torch.randn(2, 129, 96, generator=g, device="cuda")
    S[0, 3, 5] = float("nan")
    S[1, 7, 9] = float("inf")
    S[1, 8, 10] = -0.0
    _check_csr(S.cpu().numpy(), ops.csr_compact(S))


def test_csr_many_tiles_lookback():
    # 2 planes x 4096 tiles: the decoupled look-back crosses many tiles and a plane
    g = torch.Generator(device="cuda").manual_seed(9)
    S = (torch.rand(2, 131072, 32, generator=g, device="cuda") < 0.5).float()
    out = ops.csr_compact(S)
    exp = O.csr_planes(S.cpu().numpy())
    np.testing.assert_array_equal(out["row_ptr"].cpu().numpy(), exp[1])
    np.testing.assert_array_equal(out["plane_ptr"].cpu().numpy(), exp[4])
    np.testing.assert_array_equal(out["col_idx"].cpu().numpy(), exp[2])


def test_csr_matches_reference_engine(ref_engine):
    ref = ref_engine("spikeskip_ref")
    g = torch.Generator(device="cuda").manual_seed(2)
    x = (torch.rand(4097, 640, generator=g, device="cuda") < 0.12).float()
    roff, ci, vals = ref.dense_to_csr_gpu(x)
    ours = ops.dense_to_csr_gpu(x)
    n = int(roff[-1].item())
    torch.testing.assert_close(ours[0], roff, rtol=0, atol=0)
    torch.testing.assert_close(ours[1][:n], ci[:n], rtol=0, atol=0)
    torch.testing.assert_close(ours[2][:n], vals[:n], rtol=0, atol=0)


def test_csr_repeated_calls_share_workspace():
    # the scan state is reset by every launch: interleave shapes on one workspace
    for T, M, K in [(3, 1000, 64), (1, 5, 7), (2, 4000, 256), (3, 1000, 64)]:
        S = (torch.rand(T, M, K, device="cuda") < 0.2).float()
        _check_csr(S.cpu().numpy(), ops.csr_compact(S))
