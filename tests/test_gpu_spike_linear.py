"""Spike-linear on the GPU against the oracle.

Tolerance: fp32 outputs within max-abs 1e-4 x max|ref|.  The CSR
branch keeps the reference engine's summation order and is checked bit-exact
(against the C restatement of csr_coalesced_kernel and against the reference
engine itself); CSR indices and counts are always bit-exact."""
import numpy as np
import pytest
import torch

from oracle import spk_oracle as O
from spikestack_lite_b200 import ops

pytestmark = pytest.mark.gpu
TOL = 1e-4  # max |y - ref| / max |ref|


def _spikes(T, M, K, p, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.rand(T, M, K, generator=g, device="cuda") < p).float()


def _weight(N, K, seed, dtype=torch.float32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(dtype)


@pytest.mark.parametrize("branch", ["dense", "csr"])
@pytest.mark.parametrize("T,M,K,N,p", [
    (3, 257, 512, 128, 0.10),
    (3, 16384, 512, 128, 0.10),   # the isolated spike-linear config, full size
    (2, 300, 2048, 512, 0.5),     # the model's fc2 geometry at its density
    (1, 1, 64, 16, 1.0),
    (2, 129, 96, 48, 0.3),        # N tile of 48, partial row tile
    (1, 200, 128, 300, 0.2),      # N not a multiple of 16
])
def test_spike_linear_vs_oracle(branch, T, M, K, N, p):
    S = _spikes(T, M, K, p, seed=M + K)
    W = _weight(N, K, seed=N)
    Y = ops.spike_linear(S, weight=W, branch=branch)
    ref = O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy())
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("T,M,K,N,p", [
    (3, 16384, 512, 128, 0.10),   # the isolated spike-linear config
    (2, 300, 96, 200, 0.3),       # K not a multiple of 64, partial N tile, partial row tile
    (1, 1000, 2048, 512, 0.5),    # four N tiles
])
def test_weightT_layout_dense_branch(T, M, K, N, p):
    # weightT [K, N] contiguous (the reference ops' layout) on the dense branch:
    # the same results as the nn.Linear layout, CSR outputs included
    S = _spikes(T, M, K, p, seed=M + 7)
    WT = _weight(N, K, seed=N + 7).t().contiguous()
    b = torch.randn(N, device="cuda")
    csr = ops.alloc_csr(T, M, K, "cuda")
    Y = ops.spike_linear(S, weightT=WT, bias=b, csr=csr, branch="dense")
    ref = O.spike_linear(S.cpu().numpy(), WT.cpu().numpy()) + b.cpu().numpy()
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL
    assert torch.equal(Y, ops.spike_linear(S, weight=WT.t(), bias=b, branch="dense"))
    exp = O.csr_planes(S.cpu().numpy())
    assert np.array_equal(csr["row_ptr"].cpu().numpy().reshape(-1), exp[1].reshape(-1))
    assert np.array_equal(csr["col_idx"][: exp[2].size].cpu().numpy(), exp[2])


def test_weightT_layout_real_valued_inputs():
    g = torch.Generator(device="cuda").manual_seed(31)
    S = torch.randn(2, 260, 512, generator=g, device="cuda")
    WT = _weight(192, 512, seed=32).t().contiguous()
    Y = ops.spike_linear(S, weightT=WT, branch="dense")
    assert O.rel_err(Y.cpu().numpy(), O.spike_linear(S.cpu().numpy(), WT.cpu().numpy())) < TOL


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_bf16_weight_sweep_shape(branch):
    # the density-sweep geometry (K = N = 2048, bf16 W, fp32 accumulate), row slice
    S = _spikes(2, 512, 2048, 0.05, seed=1)
    W = _weight(2048, 2048, seed=2, dtype=torch.bfloat16)
    Y = ops.spike_linear(S, weightT=W.t(), branch=branch)
    ref = O.spike_linear(S.cpu().numpy(), W.float().t().cpu().numpy())
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("T,M,K,N,p", [(2, 300, 512, 200, 0.2), (1, 130, 64, 65, 0.5), (3, 1000, 256, 128, 0.1)])
def test_bf16_weight_partial_tiles_bias_csr(T, M, K, N, p):
    # bf16 weights on the dense branch: partial N tile, bias, CSR outputs
    S = _spikes(T, M, K, p, seed=M + 3)
    W = _weight(N, K, seed=N + 3, dtype=torch.bfloat16)
    b = torch.randn(N, device="cuda")
    csr = ops.alloc_csr(T, M, K, "cuda")
    Y = ops.spike_linear(S, weight=W, bias=b, csr=csr, branch="dense")
    ref = O.spike_linear(S.cpu().numpy(), W.float().t().cpu().numpy()) + b.cpu().numpy()
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL
    exp = O.csr_planes(S.cpu().numpy())
    assert np.array_equal(csr["row_ptr"].cpu().numpy().reshape(-1), exp[1].reshape(-1))
    assert np.array_equal(csr["col_idx"][: exp[2].size].cpu().numpy(), exp[2])


def test_bf16_weight_real_valued_inputs():
    # real-valued S with bf16 W: the converters split non-exact S values into hi + lo
    g = torch.Generator(device="cuda").manual_seed(12)
    S = torch.randn(2, 260, 512, generator=g, device="cuda")
    W = _weight(192, 512, seed=13, dtype=torch.bfloat16)
    Y = ops.spike_linear(S, weight=W, branch="dense")
    ref = O.spike_linear(S.cpu().numpy(), W.float().t().cpu().numpy())
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL


def test_csr_branch_bit_exact_with_reference_order():
    S = _spikes(2, 300, 512, 0.1, seed=4)
    W = _weight(128, 512, seed=5)
    Y = ops.spike_linear(S, weight=W, branch="csr").cpu().numpy()
    Sn, WT = S.cpu().numpy(), W.t().contiguous().cpu().numpy()
    for t in range(2):
        _, rp, ci, vals = O.csr_plane(Sn[t])
        np.testing.assert_array_equal(Y[t], O.spmm_csr_exact(rp, ci, vals, WT))


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_real_valued_negative_and_nan_inputs(branch):
    g = torch.Generator(device="cuda").manual_seed(8)
    S = torch.randn(2, 200, 256, generator=g, device="cuda")
    S[0, 1, 2] = float("nan")
    W = _weight(64, 256, seed=9)
    Y = ops.spike_linear(S, weight=W, branch=branch)
    ref = O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy())  # only S > 0 contributes
    assert O.rel_err(Y.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("stride", [37, 300])
def test_mixed_exact_and_real_rows(stride):
    # spike rows with a few real-valued rows: within one 128-row tile some
    # 8-row groups need the remainder pass and the others are exact, so the
    # remainder pass has to clear the exact groups' rows
    T, M, K = 2, 1500, 512
    S = _spikes(T, M, K, 0.1, seed=stride)
    g = torch.Generator(device="cuda").manual_seed(stride + 1)
    rows = torch.arange(5, M, stride, device="cuda")
    S[:, rows] = torch.randn(T, rows.numel(), K, generator=g, device="cuda") * 0.7
    W = _weight(128, K, seed=stride + 2)
    csr = ops.alloc_csr(T, M, K, "cuda", values=True)
    Y = ops.spike_linear(S, weight=W, csr=csr, branch="dense")
    Sn = S.cpu().numpy()
    assert O.rel_err(Y.cpu().numpy(), O.spike_linear(Sn, W.t().cpu().numpy())) < TOL
    exp = O.csr_planes(Sn)
    n = int(exp[4][-1])
    np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy(), exp[1].reshape(-1))
    np.testing.assert_array_equal(csr["col_idx"][:n].cpu().numpy(), exp[2])
    np.testing.assert_array_equal(csr["values"][:n].cpu().numpy(), exp[3])


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_bias_and_golden(golden, branch):
    z = golden("spike_linear")
    S = torch.from_numpy(z["bin_x"]).cuda()
    Y = ops.spike_linear(S, weight=torch.from_numpy(z["mod_w"]).cuda(), bias=torch.from_numpy(z["mod_b"]).cuda(),
                         branch=branch)
    assert O.rel_err(Y.cpu().numpy(), z["mod_y"]) < TOL
    S2 = torch.from_numpy(z["real_x"]).cuda()
    Y2 = ops.spike_linear(S2, weightT=torch.from_numpy(z["real_w"]).t().cuda(), branch=branch)
    assert O.rel_err(Y2.cpu().numpy(), z["real_y"]) < TOL


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_csr_outputs_with_product(branch):
    T, M, K = 3, 1000, 512
    S = _spikes(T, M, K, 0.1, seed=11)
    W = _weight(128, K, seed=12)
    csr = ops.alloc_csr(T, M, K, "cuda", values=True)
    Y = ops.spike_linear(S, weight=W, csr=csr, branch=branch)
    exp = O.csr_planes(S.cpu().numpy())
    n = int(exp[4][-1])
    np.testing.assert_array_equal(csr["nnz_row"].cpu().numpy(), exp[0].reshape(-1))
    np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy(), exp[1].reshape(-1))
    np.testing.assert_array_equal(csr["plane_ptr"].cpu().numpy(), exp[4])
    np.testing.assert_array_equal(csr["col_idx"][:n].cpu().numpy(), exp[2])
    np.testing.assert_array_equal(csr["values"][:n].cpu().numpy(), exp[3])
    assert O.rel_err(Y.cpu().numpy(), O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy())) < TOL


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_csr_outputs_real_valued(branch):
    # values other than 1 must be gathered from S (the dense pass flags them)
    g = torch.Generator(device="cuda").manual_seed(13)
    T, M, K = 2, 700, 200
    S = torch.randn(T, M, K, generator=g, device="cuda")
    W = _weight(96, K, seed=14)
    csr = ops.alloc_csr(T, M, K, "cuda", values=True)
    Y = ops.spike_linear(S, weight=W, csr=csr, branch=branch)
    exp = O.csr_planes(S.cpu().numpy())
    n = int(exp[4][-1])
    np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy(), exp[1].reshape(-1))
    np.testing.assert_array_equal(csr["col_idx"][:n].cpu().numpy(), exp[2])
    np.testing.assert_array_equal(csr["values"][:n].cpu().numpy(), exp[3])
    assert O.rel_err(Y.cpu().numpy(), O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy())) < TOL


@pytest.mark.parametrize("rows", [1, 31, 33, 129, 4000, 50001])
def test_dense_row_partition_edges(rows):
    # row ranges are split over the SMs in multiples of 32 rows; tiles and boxes at the edges
    S = _spikes(1, rows, 512, 0.1, seed=rows)
    W = _weight(128, 512, seed=3)
    csr = ops.alloc_csr(1, rows, 512, "cuda")
    Y = ops.spike_linear(S, weight=W, csr=csr, branch="dense")
    assert O.rel_err(Y.cpu().numpy(), O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy())) < TOL
    exp = O.csr_planes(S.cpu().numpy())
    np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy(), exp[1].reshape(-1))
    np.testing.assert_array_equal(csr["col_idx"][:int(exp[4][-1])].cpu().numpy(), exp[2])


@pytest.mark.parametrize("branch", ["dense", "csr"])
def test_reference_multistep_op_semantics(branch):
    # raw engine op as the reference tests call it (test_sparse.py:128-144)
    torch.manual_seed(11)
    B, T, I, O_ = 257, 3, 2048, 128
    x = torch.rand(T, B, I, device="cuda").round()
    w = torch.randn(O_, I, device="cuda")
    from spikestack_lite_b200.sparse import alloc_csr_buffers

    nnz, roff, ci, vals = alloc_csr_buffers(B, I, device="cuda")
    out = ops.sparse_multistep_forward(x, w.t().contiguous(), nnz, roff, ci, vals, T, branch=branch)
    assert torch.allclose(out, x @ w.t(), atol=1e-3, rtol=1e-3)
    exp = O.csr_plane(x[-1].cpu().numpy())  # the buffers hold plane T-1
    n = int(exp[1][-1])
    np.testing.assert_array_equal(nnz.cpu().numpy(), exp[0])
    np.testing.assert_array_equal(roff.cpu().numpy(), exp[1])
    np.testing.assert_array_equal(ci[:n].cpu().numpy(), exp[2])
    np.testing.assert_array_equal(vals[:n].cpu().numpy(), exp[3])
    out1 = ops.sparse_forward(x[0].contiguous(), w.t().contiguous(), nnz, roff, ci, vals, branch=branch)
    assert torch.allclose(out[0], out1, atol=1e-3, rtol=1e-3)


def test_reference_engine_parity(ref_engine):
    """Against the reference's own CUDA engine on the same inputs: CSR of the
    last plane bit-exact, Y bit-exact on the CSR branch."""
    ref = ref_engine("spikeskip_ref")
    torch.manual_seed(3)
    T, B, I, O_ = 3, 1000, 512, 128
    x = (torch.rand(T, B, I, device="cuda") < 0.1).float()
    wT = (torch.randn(O_, I, device="cuda") / I ** 0.5).t().contiguous()
    from spikestack_lite_b200.sparse import alloc_csr_buffers

    bufs_r = alloc_csr_buffers(B, I, device="cuda")
    bufs_o = alloc_csr_buffers(B, I, device="cuda")
    y_r = ref.sparse_multistep_forward(x, wT, *bufs_r, T)
    y_o = ops.sparse_multistep_forward(x, wT, *bufs_o, T, branch="csr")
    n = int(bufs_r[1][-1].item())
    for a, b in zip(bufs_o[:2], bufs_r[:2]):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    torch.testing.assert_close(bufs_o[2][:n], bufs_r[2][:n], rtol=0, atol=0)
    torch.testing.assert_close(bufs_o[3][:n], bufs_r[3][:n], rtol=0, atol=0)
    torch.testing.assert_close(y_o, y_r, rtol=0, atol=0)
    y_d = ops.sparse_multistep_forward(x, wT, *bufs_o, T, branch="dense")
    assert O.rel_err(y_d.cpu().numpy(), y_r.cpu().numpy()) < TOL


def test_full_size_properties():
    """Full isolated-config size: linearity in the weight and plane
    independence (size-independent properties) on the dense branch."""
    S = _spikes(3, 16384, 512, 0.1, seed=21)
    W1, W2 = _weight(128, 512, seed=22), _weight(128, 512, seed=23)
    Y1 = ops.spike_linear(S, weight=W1)
    Y2 = ops.spike_linear(S, weight=W2)
    Y12 = ops.spike_linear(S, weight=W1 + W2)
    scale = Y12.abs().max().item()
    assert (Y12 - Y1 - Y2).abs().max().item() / scale < 3e-5
    Yp = ops.spike_linear(S[1:2].contiguous(), weight=W1)
    torch.testing.assert_close(Yp[0], Y1[1], rtol=0, atol=0)


def test_sparselinear_forward_dense_side_golden(golden):
    """SparseLinear.forward below its width threshold (in_features 512 < 1024)
    takes the reference's dense path -- here the engine's tensor-core linear --
    and gives the reference module's output (golden mod_y; binary input, so the
    dense and spike paths agree)."""
    from spikestack_lite_b200.sparse import SparseLinear

    z = golden("spike_linear")
    lin = SparseLinear(512, 128, bias=True).cuda()
    with torch.no_grad():
        lin.linear.weight.copy_(torch.from_numpy(z["mod_w"]))
        lin.linear.bias.copy_(torch.from_numpy(z["mod_b"]))
        x = torch.from_numpy(z["bin_x"]).cuda()
        y = lin(x)
        y1 = lin(x[1])  # 2-D input, one plane
    assert O.rel_err(y.cpu().numpy(), z["mod_y"]) < TOL
    assert O.rel_err(y1.cpu().numpy(), z["mod_y"][1]) < TOL


def test_sparselinear_forward_dense_side_keeps_negative_inputs():
    """The dense side is nn.Linear's arithmetic: negative inputs count (the
    spike-linear engine's predicate drops them)."""
    from spikestack_lite_b200.sparse import SparseLinear

    torch.manual_seed(5)
    lin = SparseLinear(1024, 96, bias=True).cuda()
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(2, 40, 1024, generator=g, device="cuda")  # dense: sparsity 0 < 0.90
    with torch.no_grad():
        y = lin(x)
    ref = x.cpu().double() @ lin.linear.weight.detach().cpu().double().t() + lin.linear.bias.detach().cpu().double()
    assert O.rel_err(y.cpu().numpy(), ref.numpy()) < TOL


def test_sparselinear_forward_sparse_side_uses_engine():
    """>= 90 % sparsity at in_features >= 1024: the spike-linear engine, as the
    reference's forward_multistep / forward_single."""
    from spikestack_lite_b200 import _lib
    from spikestack_lite_b200.sparse import SparseLinear

    torch.manual_seed(7)
    lin = SparseLinear(1024, 128, bias=True).cuda()
    S = _spikes(3, 200, 1024, 0.05, seed=8)
    n0 = _lib.launch_count()
    with torch.no_grad():
        y = lin(S)
        y1 = lin(S[0])
    assert _lib.launch_count() > n0
    ref = O.spike_linear(S.cpu().numpy(), lin.linear.weight.detach().t().cpu().numpy()) + \
        lin.linear.bias.detach().cpu().numpy()
    assert O.rel_err(y.cpu().numpy(), ref) < TOL
    assert O.rel_err(y1.cpu().numpy(), ref[0]) < TOL


@pytest.mark.parametrize("p,expect", [(0.004, "csr"), (0.5, "dense")])
@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
def test_auto_branch_choice_on_device(p, expect, wdtype):
    """branch="auto" decides on the device (density probe, then the CSR scan's
    exact count against the crossover): far below the crossover it runs the
    CSR branch, far above it the dense branch.  The two branches round
    differently, so bit-equality with the explicit branch's output shows which
    one ran; the per-plane CSR outputs are exact either way."""
    T, M, K, N = 2, 3000, 2048, 512
    S = _spikes(T, M, K, p, seed=int(p * 1e4))
    W = _weight(N, K, seed=9, dtype=wdtype)
    b = torch.randn(N, device="cuda")
    want = ops.spike_linear(S, weight=W, bias=b, branch=expect)
    other = ops.spike_linear(S, weight=W, bias=b, branch="dense" if expect == "csr" else "csr")
    assert not torch.equal(want, other)  # the test can tell the branches apart
    csr = ops.alloc_csr(T, M, K, "cuda")
    got = ops.spike_linear(S, weight=W, bias=b, branch="auto", csr=csr)
    assert torch.equal(got, want), f"auto did not take the {expect} branch at p={p}"
    got2 = ops.spike_linear(S, weight=W, bias=b, branch="auto")  # internal CSR
    assert torch.equal(got2, want)
    exp = O.csr_planes(S.cpu().numpy())
    n = int(exp[4][-1])
    assert csr["plane_ptr"].cpu().numpy().tolist() == exp[4].tolist()
    np.testing.assert_array_equal(csr["row_ptr"].cpu().numpy().reshape(T, M + 1), exp[1])
    np.testing.assert_array_equal(csr["col_idx"][:n].cpu().numpy(), exp[2])
    ref = O.spike_linear(S.cpu().numpy(), W.float().t().cpu().numpy()) + b.cpu().numpy()
    assert O.rel_err(got.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_prepared_weight_image_cache(wdtype):
    """The dense branch with a weight image prepared once (ops' cache) gives
    exactly the per-call rebuild's output, and an in-place weight change (a new
    version) rebuilds it."""
    S = _spikes(3, 700, 512, 0.1, seed=31)
    W = _weight(256, 512, seed=32, dtype=wdtype)
    b = torch.randn(256, device="cuda")
    ops.set_weight_cache(False)
    try:
        y0 = ops.spike_linear(S, weight=W, bias=b, branch="dense")
    finally:
        ops.set_weight_cache(True)
    y1 = ops.spike_linear(S, weight=W, bias=b, branch="dense")
    y2 = ops.spike_linear(S, weight=W, bias=b, branch="dense")  # cache hit
    assert torch.equal(y0, y1) and torch.equal(y1, y2)
    with torch.no_grad():
        W.mul_(-0.5)
    y3 = ops.spike_linear(S, weight=W, bias=b, branch="dense")
    ops.set_weight_cache(False)
    try:
        y4 = ops.spike_linear(S, weight=W, bias=b, branch="dense")
    finally:
        ops.set_weight_cache(True)
    assert torch.equal(y3, y4) and not torch.equal(y3, y1)
    if wdtype == torch.float32:
        x = torch.randn(900, 512, device="cuda")
        a1 = ops.linear_act(x, W, b, act="heaviside")
        ops.set_weight_cache(False)
        try:
            a0 = ops.linear_act(x, W, b, act="heaviside")
        finally:
            ops.set_weight_cache(True)
        assert torch.equal(a0, a1)


def test_prepared_weight_image_through_the_c_abi():
    """spk_weight_image once, then spk_spike_linear_img twice: identical to
    spk_spike_linear, which rebuilds the image itself."""
    import ctypes

    from spikestack_lite_b200 import _lib

    lib = _lib.load()
    T, M, K, N = 2, 513, 256, 192
    S = _spikes(T, M, K, 0.2, seed=41)
    WT = _weight(N, K, seed=42).t().contiguous()  # weightT [K, N]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nb = lib.spk_weight_image_bytes(K, N, _lib.SPK_F32)
    buf = torch.empty(nb + 1024, dtype=torch.uint8, device="cuda")
    off = (-buf.data_ptr()) % 1024
    img = buf[off:off + nb]
    _lib.check(lib.spk_weight_image(WT.data_ptr(), _lib.SPK_F32, N, 1, K, N, img.data_ptr(), nb, stream),
               "spk_weight_image")
    wsn = lib.spk_spike_linear_workspace_bytes(T, M, K, N, _lib.SPK_F32)
    ws = torch.empty(wsn, dtype=torch.uint8, device="cuda")
    ys = []
    for use_img in (False, True, True):
        Y = torch.empty(T, M, N, device="cuda")
        if use_img:
            rc = lib.spk_spike_linear_img(S.data_ptr(), T, M, K, WT.data_ptr(), _lib.SPK_F32, N, 1, N, img.data_ptr(),
                                          None, Y.data_ptr(), None, None, None, None, None, 0, _lib.BRANCH_DENSE,
                                          ws.data_ptr(), wsn, stream)
        else:
            rc = lib.spk_spike_linear(S.data_ptr(), T, M, K, WT.data_ptr(), _lib.SPK_F32, N, 1, N, None, Y.data_ptr(),
                                      None, None, None, None, None, 0, _lib.BRANCH_DENSE, ws.data_ptr(), wsn, stream)
        _lib.check(rc, "spike_linear")
        ys.append(Y)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])
    assert O.rel_err(ys[1].cpu().numpy(), O.spike_linear(S.cpu().numpy(), WT.cpu().numpy())) < TOL


def test_weight_cache_never_serves_a_freed_weights_image():
    """A new weight tensor allocated at a freed weight's address (the caching
    allocator reuses blocks) with version 0 and the same shape must not be
    given the old tensor's image: the cache holds the tensor by weak reference
    and drops the image when the tensor dies."""
    S = _spikes(2, 600, 256, 0.2, seed=51)
    outs, refs = [], []
    for seed in (52, 53, 54):
        W = _weight(192, 256, seed=seed)
        outs.append(ops.spike_linear(S, weight=W, branch="dense"))
        refs.append(O.spike_linear(S.cpu().numpy(), W.t().cpu().numpy()))
        del W
    for y, ref in zip(outs, refs):
        assert O.rel_err(y.cpu().numpy(), ref) < TOL
    assert not torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("T,M", [(1, 5), (2, 700)])
def test_auto_branch_small_inputs(T, M):
    """The automatic choice on inputs with fewer rows than the probe samples:
    the result is one of the two branches' outputs exactly."""
    K, N = 2048, 512
    S = _spikes(T, M, K, 0.003, seed=M)
    W = _weight(N, K, seed=3, dtype=torch.bfloat16)
    got = ops.spike_linear(S, weight=W, branch="auto")
    assert torch.equal(got, ops.spike_linear(S, weight=W, branch="csr")) or \
        torch.equal(got, ops.spike_linear(S, weight=W, branch="dense"))
    ref = O.spike_linear(S.cpu().numpy(), W.float().t().cpu().numpy())
    assert O.rel_err(got.cpu().numpy(), ref) < TOL
