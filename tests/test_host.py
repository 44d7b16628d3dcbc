"""Host-side mirror of the reference API, on CPU: module structure, seeded
initialisation equal to the reference's (via the golden state dicts), state
dict loading, engine installation and the no-CPU-path contract."""
import types

import numpy as np
import pytest
import torch

from oracle import spk_oracle as O
from spikestack_lite_b200 import engine as E
from spikestack_lite_b200._lib import EngineError
from spikestack_lite_b200.sparse import SparseLinear, alloc_csr_buffers
from spikestack_lite_b200.transformer import SpikingTransformer


@pytest.mark.parametrize("name", ["model_c1", "model_c5_tiny"])
def test_seeded_init_equals_reference(golden, name):
    z = golden(name)
    cfg = O.model_config_from_golden(z)
    # the fixtures were made single-threaded; the QR inside orthogonal_ (GSMC
    # W_rec) rounds differently with other thread counts
    nthreads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        torch.manual_seed(0)
        m = SpikingTransformer(**cfg)
    finally:
        torch.set_num_threads(nthreads)
    ref = O.state_dict_from_golden(z)
    own = m.state_dict()
    for k, v in ref.items():
        k2 = k if k in own else k.replace(".ffn.fc2.", ".ffn.fc2.linear.")
        np.testing.assert_array_equal(own[k2].numpy(), v, err_msg=k)
    assert len(own) == len(ref)


def test_load_reference_state_dict_both_fc2_layouts(golden):
    z = golden("model_c1")
    cfg = O.model_config_from_golden(z)
    sd = {k: torch.as_tensor(v) for k, v in O.state_dict_from_golden(z).items()}
    m = SpikingTransformer(**cfg)
    m.load_reference_state_dict(sd)
    assert torch.equal(m.blocks[0].ffn.fc2.linear.weight, sd["blocks.0.ffn.fc2.weight"])
    dense = SpikingTransformer(**{**cfg, "use_spikeskip": False})
    sd2 = {k.replace(".ffn.fc2.", ".ffn.fc2.linear."): v for k, v in sd.items()}
    dense.load_reference_state_dict(sd2)
    assert torch.equal(dense.blocks[0].ffn.fc2.weight, sd["blocks.0.ffn.fc2.weight"])


def test_expansion_default_follows_engine_presence():
    assert SpikingTransformer(use_spikeskip=True).blocks[0].ffn.fc2.in_features == 1024
    assert SpikingTransformer(use_spikeskip=False).blocks[0].ffn.fc2.in_features == 512


def test_cpu_inputs_raise_instead_of_falling_back():
    m = SpikingTransformer(temporal=True, n_repeats=3, use_spikeskip=True, expansion=4)
    with pytest.raises(EngineError, match="CUDA"):
        m(torch.randn(2, 64, 48))
    with pytest.raises(EngineError, match="CUDA"):
        SparseLinear(1024, 16)(torch.zeros(2, 1024))


def test_linear_act_host_checks():
    from spikestack_lite_b200 import ops
    from spikestack_lite_b200.attention import engine_linear

    x, w = torch.randn(4, 128), torch.randn(256, 128)
    with pytest.raises(EngineError, match="CUDA"):
        ops.linear_act(x, w)
    # autograd on, or a CPU input: the module's own nn.Linear runs (None = not taken)
    lin = torch.nn.Linear(128, 256)
    assert engine_linear(lin, x) is None
    with torch.no_grad():
        assert engine_linear(lin, x) is None                  # CPU input
        assert engine_linear(torch.nn.Linear(128, 64), x) is None  # narrow N


def test_add_layernorm_host_checks():
    from spikestack_lite_b200 import ops
    from spikestack_lite_b200.attention import AstrocyteHebbianBlock, _engine_norm_ok

    x = torch.randn(2, 8, 128)
    with pytest.raises(EngineError, match="CUDA"):
        ops.add_layernorm(x, x)
    ln = torch.nn.LayerNorm(128)
    with torch.no_grad():
        assert not _engine_norm_ok(ln, x)                      # CPU input: the reference's composition
    # off the engine path the block runs the reference's composition, whose
    # attention has no CPU path either
    torch.manual_seed(0)
    blk = AstrocyteHebbianBlock(d_model=128, num_heads=4)
    with torch.no_grad(), pytest.raises(EngineError, match="CUDA"):
        blk.forward_fused(x, None, blk.norm1)


def test_spire_and_readout_ops_host_checks():
    from spikestack_lite_b200 import ops
    from spikestack_lite_b200.graphs import CapturedForward
    from spikestack_lite_b200.transformer import SpireEncoder

    with pytest.raises(EngineError, match="CUDA"):
        ops.spire_planes(torch.randn(2, 4, 8), torch.zeros(3))
    with pytest.raises(EngineError, match="CUDA"):
        ops.temporal_mean(torch.randn(3, 2, 4, 8))
    with pytest.raises(EngineError, match="CUDA"):
        CapturedForward(torch.nn.Identity(), torch.randn(2, 3))
    # off the engine path (CPU, or autograd on) the encoder runs the reference's composition
    torch.manual_seed(0)
    enc = SpireEncoder(input_dim=6, d_model=8, seq_len=5, n_repeats=3, temporal=True)
    x = torch.randn(2, 5, 6)
    planes = enc(x)
    u = enc.projection(x)
    v = u - enc.frontier.view(1, 1, 8) - enc.temporal_frontier
    want = (v.unsqueeze(-1) - enc.dither > 0).float().permute(3, 0, 1, 2)
    assert planes.shape == (3, 2, 5, 8) and torch.equal(planes, want)


def test_unsupported_stems_are_rejected():
    with pytest.raises(EngineError):
        SpikingTransformer(use_conv_stem=True)
    with pytest.raises(EngineError):
        SpikingTransformer(text_vocab=64)
    with pytest.raises(ValueError):
        SpikingTransformer(use_gsmc=True, temporal=False)


def test_alloc_csr_buffers_shapes():
    nnz, roff, ci, vals = alloc_csr_buffers(5, 7, device="cpu")
    assert nnz.shape == (5,) and roff.shape == (6,) and ci.shape == (35,) and vals.shape == (35,)
    assert nnz.dtype == torch.int32 and vals.dtype == torch.float32


def test_install_swaps_engines_into_a_reference_package():
    pkg = types.ModuleType("fakeref")
    mods = {n: types.ModuleType(n) for n in ("fakeref.sparse", "fakeref.nn", "fakeref.nn.attention",
                                             "fakeref.nn.gsmc", "fakeref.encode", "fakeref.encode.spire")}
    import sys

    sys.modules["fakeref"] = pkg
    sys.modules.update(mods)
    try:
        E.install(pkg)
        assert mods["fakeref.sparse"]._cuda_engine is E.sparse_engine
        assert mods["fakeref.nn.attention"]._attn_cuda_engine is E.attention_engine
        assert mods["fakeref.nn.gsmc"]._gsmc_cuda_engine is E.gsmc_engine
        assert mods["fakeref.encode.spire"]._spire_cuda_engine is E.spire_engine
    finally:
        for n in ["fakeref", *mods]:
            sys.modules.pop(n, None)


def test_engine_objects_expose_reference_names():
    for name in ("sparse_forward", "sparse_multistep_forward", "dense_to_csr_gpu"):
        assert callable(getattr(E.sparse_engine, name))
    for name in ("apply_channel_decay", "fused_normalize_attention"):
        assert callable(getattr(E.attention_engine, name))
    assert callable(E.gsmc_engine.fused_gsmc_step)
    assert callable(E.spire_engine.spire_dither)


def test_install_into_the_reference_package_when_available():
    """With a checkout of the reference named by SPIKESTACK_REFERENCE, install
    the engine into the real `spikestack_lite` package: its sparse, attention,
    GSMC and Spire modules then hold this engine's objects, and the reference's
    own SparseLinear reports the engine present.  Skipped without a checkout."""
    import importlib
    import os
    import sys

    ref = os.environ.get("SPIKESTACK_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "spikestack_lite")):
        pytest.skip("no reference checkout (set SPIKESTACK_REFERENCE)")
    sys.path.insert(0, ref)
    try:
        pkg = importlib.import_module("spikestack_lite")
        E.install(pkg)
        sparse = importlib.import_module("spikestack_lite.sparse")
        attn = importlib.import_module("spikestack_lite.nn.attention")
        gsmc = importlib.import_module("spikestack_lite.nn.gsmc")
        assert sparse._cuda_engine is E.sparse_engine
        assert attn._attn_cuda_engine is E.attention_engine
        assert gsmc._gsmc_cuda_engine is E.gsmc_engine
    finally:
        sys.path.remove(ref)
        for n in [m for m in sys.modules if m == "spikestack_lite" or m.startswith("spikestack_lite.")]:
            sys.modules.pop(n, None)
