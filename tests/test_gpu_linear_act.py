"""Linear + activation on the tensor cores (spk_linear_act) against fp64.

The projections around the spike-linear path (SpikingFFN fc1 + threshold
spike, attention q/k/v spikes, o_proj) are fp32 nn.Linear layers in the
reference.  The engine computes them to fp32-class accuracy (a tf32 pass
w_hi * x_t plus a bf16 correction pass bf16(w - w_hi) * bf16(x) + bf16(w_hi) *
bf16(x - x_t)): outputs within 1e-5 x max|ref| of the fp64 product (~1e-6 in
practice); spikes equal to the fp64 decision except where the pre-activation
lies within rounding distance of the threshold."""
import pytest
import torch

from spikestack_lite_b200 import ops
from spikestack_lite_b200._lib import EngineError

pytestmark = pytest.mark.gpu


def _data(R, K, N, seed, bias=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(R, K, generator=g, device="cuda")
    w = torch.randn(N, K, generator=g, device="cuda") / K ** 0.5
    b = torch.randn(N, generator=g, device="cuda") * 0.1 if bias else None
    return x, w, b


def _ref64(x, w, b):
    y = x.double() @ w.double().t()
    return y + b.double() if b is not None else y


@pytest.mark.parametrize("R,K,N,bias", [
    (1000, 512, 2048, True),    # fc1 geometry (d 512 -> 4d)
    (4096, 512, 512, True),     # q/k/v/o projection geometry
    (257, 96, 300, False),      # partial row tile, partial N tile, K not a multiple of 64
    (3, 4, 65, True),           # smallest K, N just above the narrow-N limit
])
def test_linear_fp32_accuracy(R, K, N, bias):
    x, w, b = _data(R, K, N, seed=R + K + N, bias=bias)
    y = ops.linear_act(x, w, b)
    ref = _ref64(x, w, b)
    scale = ref.abs().max().item()
    err = (y.double() - ref).abs().max().item()
    cublas = torch.nn.functional.linear(x, w, b)
    err_cublas = (cublas.double() - ref).abs().max().item()
    assert err <= max(1e-5 * scale, 4 * err_cublas), (err, err_cublas, scale)


def test_real_world_scale_inputs():
    # wide dynamic range and negative values (no relu on this op)
    x, w, b = _data(512, 256, 384, seed=7)
    x = x * torch.logspace(-3, 3, 256, device="cuda")
    y = ops.linear_act(x, w, b)
    ref = _ref64(x, w, b)
    assert (y.double() - ref).abs().max().item() <= 1e-5 * ref.abs().max().item()


@pytest.mark.parametrize("thr", [0.0, 0.25])
def test_heaviside_spikes(thr):
    x, w, b = _data(2048, 512, 2048, seed=11)
    s = ops.linear_act(x, w, b, act="heaviside", thr=thr)
    pre = _ref64(x, w, b) - thr
    want = (pre > 0).float()
    near = pre.abs() < 1e-5 * pre.abs().max()
    assert set(s.unique().tolist()) <= {0.0, 1.0}
    assert torch.equal(s[~near], want[~near])
    # the reference op on the GPU (cuBLAS fp32 + threshold): flips only near the threshold
    ref_gpu = ((torch.nn.functional.linear(x, w, b) - thr) > 0).float()
    assert (s != ref_gpu).float().mean().item() < 1e-4


def test_vspike():
    x, w, b = _data(1024, 512, 512, seed=13)
    tau = 0.5
    s = ops.linear_act(x, w, b, act="vspike", thr=tau)
    y = _ref64(x, w, b)
    u = (torch.tanh(y) + 1.0) / 2.0 - tau
    want = (u > 0).float()
    near = u.abs() < 1e-5
    assert torch.equal(s[~near], want[~near])


def test_leading_dims_and_empty():
    x, w, b = _data(4 * 3 * 50, 128, 256, seed=17)
    x4 = x.view(4, 3, 50, 128)
    y4 = ops.linear_act(x4, w, b)
    assert y4.shape == (4, 3, 50, 256)
    torch.testing.assert_close(y4.view(-1, 256), ops.linear_act(x, w, b), rtol=0, atol=0)
    e = ops.linear_act(torch.empty(0, 128, device="cuda"), w, b)
    assert e.shape == (0, 256)


def test_rejects_unsupported():
    x, w, b = _data(8, 128, 64, seed=19)
    with pytest.raises(EngineError):
        ops.linear_act(x, w, b)                                   # N <= 64
    x, w, b = _data(8, 126, 128, seed=21)
    with pytest.raises(EngineError):
        ops.linear_act(x, w, b)                                   # K % 4 != 0
    with pytest.raises(EngineError):
        ops.linear_act(x.cpu(), w.cpu(), None)                    # no CPU path
    with pytest.raises(EngineError):
        ops.linear_act(x, w, b, act="relu")


@pytest.mark.parametrize("act", ["heaviside", "vspike"])
@pytest.mark.parametrize("R,K,N", [(1000, 512, 2048), (4097, 64, 96), (300, 256, 160)])
def test_packed_epilogues_pack_the_spikes(R, K, N, act):
    """act="heaviside_bits" / "vspike_bits" write the same decisions as
    "heaviside" / "vspike", packed one bit each (bit b of word w = column
    32w + b), partial row tiles included."""
    g = torch.Generator(device="cuda").manual_seed(R + N)
    x = torch.randn(R, K, generator=g, device="cuda")
    w = torch.randn(N, K, generator=g, device="cuda") / K ** 0.5
    b = torch.randn(N, generator=g, device="cuda") * 0.1
    thr = 0.05 if act == "heaviside" else 0.5
    spikes = ops.linear_act(x, w, b, act=act, thr=thr)
    bits = ops.linear_act(x, w, b, act=act + "_bits", thr=thr)
    assert 0.05 < float(spikes.mean()) < 0.95
    assert bits.dtype == torch.int32 and bits.shape == (R, N // 32)
    assert torch.equal(ops.unpack_spikes(bits, N), spikes)


@pytest.mark.parametrize("T,M,K,N", [(4, 1000, 2048, 512), (2, 4097, 128, 96), (1, 129, 64, 200)])
def test_spike_linear_bits_matches_the_unpacked_dense_branch(T, M, K, N):
    """fc2 on packed spikes against the dense branch on the unpacked fp32
    spikes and the float64 product.  The packed kernel multiplies bf16 0 / 1
    by the three-way bf16 split of W (exact products, fp32 accumulation), the
    dense branch by the tf32 hi + lo split (W to ~2^-22): both lie within fp32
    accumulation error of the exact sum."""
    g = torch.Generator(device="cuda").manual_seed(T * M + K)
    S = (torch.rand(T, M, K, generator=g, device="cuda") < 0.5).float()
    shifts = torch.arange(32, device="cuda", dtype=torch.int64)
    words = (S.view(T, M, K // 32, 32).long() << shifts).sum(-1)
    bits = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    assert torch.equal(ops.unpack_spikes(bits, K), S)
    w = torch.randn(N, K, generator=g, device="cuda") / K ** 0.5
    b = torch.randn(N, generator=g, device="cuda")
    y_bits = ops.spike_linear_bits(bits, K, w, b)
    y_dense = ops.spike_linear(S, weight=w, bias=b, branch="dense")
    ref = S.cpu().double() @ w.cpu().double().t() + b.cpu().double()
    scale = float(ref.abs().max())
    err_bits = float((y_bits.cpu().double() - ref).abs().max()) / scale
    err_dense = float((y_dense.cpu().double() - ref).abs().max()) / scale
    assert err_bits < 1e-5 and err_dense < 1e-5, (err_bits, err_dense)  # ~3e-6 at K = 2048


def test_packed_paths_with_no_rows():
    """Empty inputs: the packed epilogue and the packed spike-linear return
    empty outputs without launching."""
    w = torch.randn(128, 64, device="cuda")
    x = torch.empty(0, 64, device="cuda")
    assert ops.linear_act(x, w, None, act="heaviside_bits").shape == (0, 4)
    bits = torch.empty(3, 0, 2, dtype=torch.int32, device="cuda")
    assert ops.spike_linear_bits(bits, 64, w).shape == (3, 0, 128)


@pytest.mark.parametrize("R,K,N,act", [(1000, 512, 512, "none"), (257, 96, 256, "none"),
                                       (4097, 64, 256, "heaviside_bits"), (3, 4, 256, "vspike"),
                                       (65536, 512, 2048, "heaviside")])
def test_cta_pair_form_is_bit_identical(R, K, N, act, monkeypatch):
    """SPK_WT_PAIR=1 runs the linear op in CTA pairs (clusters of two CTAs
    along N, tcgen05 cta_group::2 with M = 256: the two N tiles' weights in the
    pair's TMEM, each CTA staging half of every 128-row tile): the same
    products summed in the same order as the single-CTA form, so the output is
    bit-identical, partial tiles and a rank whose half lies past the last row
    included."""
    g = torch.Generator(device="cuda").manual_seed(R + K + N)
    x = torch.randn(R, K, generator=g, device="cuda")
    w = torch.randn(N, K, generator=g, device="cuda") / K ** 0.5
    b = torch.randn(N, generator=g, device="cuda") * 0.1
    thr = 0.5 if act == "vspike" else 0.0
    monkeypatch.setenv("SPK_WT_PAIR", "0")
    single = ops.linear_act(x, w, b, act=act, thr=thr)
    monkeypatch.setenv("SPK_WT_PAIR", "1")
    pair = ops.linear_act(x, w, b, act=act, thr=thr)
    assert torch.equal(single, pair)
