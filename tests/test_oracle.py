"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz,
produced by tests/golden/make_golden.py from the reference's CPU paths) and
check the CSR restatement's internal consistency.  CPU only."""
import numpy as np
import pytest
import torch

from oracle import spk_oracle as O


# ------------------------------------------------------------------ spike-linear
def test_spike_linear_matches_reference_binary(golden):
    z = golden("spike_linear")
    y = O.spike_linear(z["bin_x"], z["bin_w"].T)
    assert O.rel_err(y, z["bin_y"]) < 1e-6


def test_spike_linear_matches_reference_real_valued(golden):
    z = golden("spike_linear")
    y = O.spike_linear(z["real_x"], z["real_w"].T)
    assert O.rel_err(y, z["real_y"]) < 1e-6


def test_sparselinear_module_bias(golden):
    z = golden("spike_linear")
    y = O.spike_linear(z["bin_x"], z["mod_w"].T, z["mod_b"])
    assert O.rel_err(y, z["mod_y"]) < 1e-6


def test_spmm_exact_restatement_close_to_matmul(golden):
    z = golden("spike_linear")
    x = z["bin_x"][0]
    nnz, rp, ci, vals = O.csr_plane(x)
    y = O.spmm_csr_exact(rp, ci, vals, z["bin_w"].T)
    assert O.rel_err(y, z["bin_y"][0]) < 1e-5


# --------------------------------------------------------------------------- CSR
@pytest.mark.parametrize("M,K,p", [(1, 1, 0.5), (7, 33, 0.3), (257, 512, 0.1), (64, 100, 0.0), (64, 100, 1.0)])
def test_csr_numpy_equals_c_restatement(M, K, p):
    rng = np.random.default_rng(M * 1000 + K)
    S = (rng.random((M, K)) < p).astype(np.float32)
    a, b = O.csr_plane(S), O.csr_plane_c(S)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_csr_predicate_drops_negative_nan_and_zero():
    S = np.array([[0.0, -1.0, np.nan, 2.5, 1.0, -0.0, np.inf]], np.float32)
    nnz, rp, ci, vals = O.csr_plane(S)
    assert nnz.tolist() == [3]
    assert rp.tolist() == [0, 3]
    assert ci.tolist() == [3, 4, 6]
    assert vals[:2].tolist() == [2.5, 1.0] and np.isinf(vals[2])
    c = O.csr_plane_c(S)
    np.testing.assert_array_equal(c[2], ci)


def test_csr_structure_properties():
    rng = np.random.default_rng(3)
    S = (rng.random((3, 300, 77)) < 0.2).astype(np.float32)
    nnz, rp, ci, vals, pp = O.csr_planes(S)
    assert pp[0] == 0 and pp[-1] == int((S > 0).sum())
    for t in range(3):
        assert rp[t, 0] == 0
        np.testing.assert_array_equal(np.diff(rp[t]), nnz[t])
        cols = ci[pp[t]:pp[t + 1]]
        for m in range(0, 300, 37):  # ascending, and exactly the nonzeros
            row = cols[rp[t, m]:rp[t, m + 1]]
            np.testing.assert_array_equal(row, np.nonzero(S[t, m] > 0)[0])
    assert np.all(vals == 1.0)


def test_multistep_leaves_last_plane_csr(golden):
    z = golden("spike_linear")
    y, (nnz, rp, ci, vals) = O.sparse_multistep_forward(z["bin_x"], z["bin_w"].T)
    assert O.rel_err(y, z["bin_y"]) < 1e-6
    ref = O.csr_plane(z["bin_x"][-1])
    for a, b in zip((nnz, rp, ci, vals), ref):
        np.testing.assert_array_equal(a, b)


# --------------------------------------------------------------------- attention
@pytest.mark.parametrize("tag", ["a", "b"])
def test_attention_matches_reference(golden, tag):
    z = golden("attention")
    out = O.spiking_attention(z[f"{tag}_q"], z[f"{tag}_k"], z[f"{tag}_v"], z[f"{tag}_lam"], int(z[f"{tag}_heads"]),
                              float(z[f"{tag}_eps"]))
    assert O.rel_err(out.numpy(), z[f"{tag}_attn"]) < 1e-6


def test_channel_decay_definition():
    k = torch.ones(2, 5, 3)
    lam = torch.tensor([0.5, 0.9, 1.0])
    kw = O.channel_decay(k, lam)
    assert torch.allclose(kw[0, :, 0], torch.tensor([0.5 ** 4, 0.5 ** 3, 0.25, 0.5, 1.0]))
    assert torch.allclose(kw[1, :, 2], torch.ones(5))


# -------------------------------------------------------------------------- GSMC
@pytest.mark.parametrize("pool", ["mean", "last"])
def test_gsmc_matches_reference(golden, pool):
    z = golden("gsmc")
    sd = {k[len(pool) + 4:]: z[k] for k in z.files if k.startswith(f"{pool}_sd_")}
    out, _ = O.gsmc_forward(z[f"{pool}_x"], sd, pool=pool, step="module")
    np.testing.assert_array_equal(out.numpy(), z[f"{pool}_out"])
    out_e, _ = O.gsmc_forward(z[f"{pool}_x"], sd, pool=pool, step="engine")
    assert np.abs(out_e.numpy() - z[f"{pool}_out"]).max() <= 1.0 / 3 + 1e-6  # at most a rare spike flip


# ------------------------------------------------------------------------- model
@pytest.mark.parametrize("name", ["model_c1", "model_c5_tiny"])
def test_transformer_matches_reference(golden, name):
    z = golden(name)
    cfg = O.model_config_from_golden(z)
    sd = O.state_dict_from_golden(z)
    cap = {}
    logits = O.transformer_forward(sd, z["x"], cfg["num_heads"], cfg["num_layers"], use_gsmc=cfg.get("use_gsmc", False),
                                   capture=cap)
    np.testing.assert_array_equal(cap["planes"].numpy(), z["cap_planes"])
    for i in range(cfg["num_layers"]):
        assert O.rel_err(cap[f"block{i}_out"].numpy(), z[f"cap_block{i}_out"]) < 1e-6
    assert O.rel_err(logits.numpy(), z["logits"]) < 1e-6


@pytest.mark.parametrize("name", ["model_c1", "model_c5_tiny"])
def test_block_stages_match_reference_blocks(golden, name):
    """The staged block restatement gives the reference's block outputs, and its
    spikes are the threshold decisions of its own pre-activations."""
    z = golden(name)
    cfg = O.model_config_from_golden(z)
    sd = O.state_dict_from_golden(z)
    for i in range(cfg["num_layers"]):
        st = O.block_stages(sd, f"blocks.{i}", torch.from_numpy(z[f"cap_block{i}_in"]), cfg["num_heads"],
                            cfg.get("spike_threshold", 0.0))
        np.testing.assert_allclose(st["out"].numpy(), z[f"cap_block{i}_out"], rtol=0, atol=1e-6)
        assert torch.equal(st["act"], (st["fc1_pre"] > 0).float())
        assert torch.equal(st["q"], (st["q_pre"] > 0).float())
