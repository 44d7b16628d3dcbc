"""Parity at the full sizes of the density sweep and the attention config.

Density sweep: S[4, 65536, 2048] ~ Bernoulli(p) per plane, p in {0.01, 0.1,
0.5}, W[2048, 2048] bf16 ~ N(0, 1/K), fp32 accumulate.  The CSR of all four
planes is compared bit-exact with the oracle over the whole tensor; Y is
compared with the oracle (W.float(), fp32) on the first and last 512 rows of
every plane and on 512 rows drawn at random, within 1e-4 x max|ref|.

Attention: B = 64, H = 8, L = 4096, d_head = 64, T = 4, q, k, v ~
Bernoulli(0.15).  Each (t, b) unit is independent, so the oracle runs on a
sample of eight units (every plane of two samples drawn at random, plus the
first and last sample of plane 0) and the output is compared there within
1e-4 x max|ref|; the whole output is checked for finiteness and for zero rows
exactly where a query row has no spike."""
import numpy as np
import pytest
import torch

from oracle import spk_oracle as O
from spikestack_lite_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _sample_rows(M, n, seed):
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(512, M - 512), size=n, replace=False)
    return np.unique(np.concatenate([np.arange(512), np.sort(mid), np.arange(M - 512, M)]))


@pytest.mark.parametrize("p,branches", [(0.01, ("dense", "csr")), (0.1, ("dense", "csr")), (0.5, ("dense",))])
def test_density_sweep_full_size(p, branches):
    T, M, K, N = 4, 65536, 2048, 2048
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(int(p * 1000))
    S = (torch.rand(T, M, K, generator=g, device=dev) < p).float()
    W = (torch.randn(K, N, generator=g, device=dev) / K ** 0.5).to(torch.bfloat16)  # weightT [K, N]
    nnz = int((S > 0).sum().item())
    rows = _sample_rows(M, 512, seed=int(p * 1000))
    S_rows = S[:, rows].cpu().numpy()
    ref = O.spike_linear(S_rows, W.float().cpu().numpy())
    exp = None
    for branch in branches:
        csr = ops.alloc_csr(T, M, K, dev, capacity=nnz + 1024)
        Y = ops.spike_linear(S, weightT=W, csr=csr, branch=branch)
        err = O.rel_err(Y[:, rows].cpu().numpy(), ref)
        assert err < TOL, f"p={p} {branch}: rel err {err}"
        assert bool(torch.isfinite(Y).all())
        del Y
        if exp is None:
            exp = O.csr_planes(S.cpu().numpy())
        pp = csr["plane_ptr"].cpu().numpy()
        np.testing.assert_array_equal(pp, exp[4])
        np.testing.assert_array_equal(csr["nnz_row"].cpu().numpy().reshape(T, M), exp[0])
        np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy().reshape(T, M + 1), exp[1])
        np.testing.assert_array_equal(csr["col_idx"][:nnz].cpu().numpy(), exp[2])
        assert int(pp[-1]) == nnz
        del csr
        _free()
    del S
    _free()


def test_attention_full_size():
    T, B, L, H, dh = 4, 64, 4096, 8, 64
    d = H * dh
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4096)
    q, k, v = ((torch.rand(T, B, L, d, generator=g, device=dev) < 0.15).float() for _ in range(3))
    lam = torch.sigmoid(torch.empty(d, device=dev).uniform_(5.0, 8.0, generator=g))
    out = ops.spiking_attention(q, k, v, lam, H)
    assert out.shape == (T, B, L, d)
    assert bool(torch.isfinite(out).all())
    # a query row without spikes gives a zero output row, and only then (every
    # key mass is positive here: the first position's keys all decay to > 0)
    q_empty = q.view(T, B, L, H, dh).sum(-1) == 0
    o_zero = out.view(T, B, L, H, dh).abs().sum(-1) == 0
    assert torch.equal(q_empty, o_zero)
    rng = np.random.default_rng(7)
    bs = sorted(rng.choice(np.arange(1, B - 1), size=2, replace=False).tolist())
    units = [(t, b) for t in range(T) for b in bs] + [(0, 0), (0, B - 1)]
    for t, b in units:
        sl = (slice(t, t + 1), slice(b, b + 1))
        ref = O.spiking_attention(q[sl].cpu(), k[sl].cpu(), v[sl].cpu(), lam.cpu(), H)
        err = O.rel_err(out[sl].cpu().numpy(), ref.numpy())
        assert err < TOL, f"unit (t={t}, b={b}): rel err {err}"
    del q, k, v, out
    _free()
