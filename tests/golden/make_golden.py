"""Generate the golden input/output vectors under ``tests/golden/``.

These fixtures are produced by the REFERENCE implementation itself (its own
PyTorch CPU code paths), imported from a local checkout given by
``--reference`` (default: the SPIKESTACK_REFERENCE environment variable).  They exist so that the oracle
restatement in ``oracle/`` can be pinned against the reference on machines
where the reference is not available (the GPU box has no checkout).

Every fixture is small (a few hundred KB at most).  Run:

    python tests/golden/make_golden.py [--reference PATH]

What each file holds (all arrays float32 unless noted):

* ``spike_linear.npz`` -- ``spikestack_lite.sparse.sparse_multistep_forward``
  with no engine (``sparse/__init__.py:102-105``: ``torch.matmul``), for a
  binary Bernoulli(0.1) case and a non-negative real-valued case, plus
  ``SparseLinear.forward_multistep`` with bias (``sparse/__init__.py:240-262``).
* ``attention.npz`` -- ``AstrocyteHebbianAttention.forward``
  (``nn/attention.py:105-136``) with the q/k/v spikes, lambda, the o_proj
  input (normalised attention, heads merged) and the module output.
* ``gsmc.npz`` -- ``FusedGSMC.forward`` eval path (``nn/gsmc.py:96-148``),
  pooled ``mean`` and ``last``.
* ``model_c1.npz`` / ``model_c5_tiny.npz`` -- ``SpikingTransformer.forward``
  (``models/transformer.py:159-192``) logits, the full state dict and the
  per-stage intermediates (Spire planes, every block output, GSMC output).
"""

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return t.detach().cpu().numpy()


def make_spike_linear(out_dir):
    from spikestack_lite import sparse as S

    assert S._cuda_engine is None, "golden vectors must come from the reference CPU path"
    res = {}
    g = torch.Generator().manual_seed(0)
    # binary spikes, Bernoulli(0.1): the isolated spike-linear geometry at small M
    T, M, K, N = 3, 257, 512, 128
    x = (torch.rand(T, M, K, generator=g) < 0.10).float()
    w = torch.randn(N, K, generator=g) / K ** 0.5
    y = S.sparse_multistep_forward(x, w.t().contiguous(), None, None, None, None, T)
    res.update(bin_x=_np(x), bin_w=_np(w), bin_y=_np(y))
    # non-negative real-valued input (the reference tests use torch.rand)
    T2, M2, K2, N2 = 2, 24, 1024, 96
    x2 = torch.rand(T2, M2, K2, generator=g)
    x2 = torch.where(torch.rand(T2, M2, K2, generator=g) < 0.3, x2, torch.zeros(()))
    w2 = torch.randn(N2, K2, generator=g) * 0.5
    y2 = S.sparse_multistep_forward(x2, w2.t().contiguous(), None, None, None, None, T2)
    res.update(real_x=_np(x2), real_w=_np(w2), real_y=_np(y2))
    # module path with bias
    torch.manual_seed(3)
    lin = S.SparseLinear(K, N, bias=True)
    y3 = lin.forward_multistep(x)
    res.update(mod_w=_np(lin.linear.weight), mod_b=_np(lin.linear.bias), mod_y=_np(y3))
    np.savez_compressed(os.path.join(out_dir, "spike_linear.npz"), **res)


def _capture_attention(attn, x):
    cap = {}

    def hook(name):
        def _h(mod, inp, out):
            cap[name + "_in"] = inp[0].detach().clone()
            cap[name + "_out"] = out.detach().clone()
        return _h

    hs = [getattr(attn, n).register_forward_hook(hook(n)) for n in ("q_proj", "k_proj", "v_proj", "o_proj")]
    with torch.no_grad():
        y = attn(x)
    for h in hs:
        h.remove()
    q = (cap["q_proj_out"] > 0).float()
    k = (cap["k_proj_out"] > 0).float()
    u01 = (torch.tanh(cap["v_proj_out"]) + 1.0) / 2.0
    v = (u01 - attn.tau.item() > 0).float()
    return q, k, v, cap["o_proj_in"], y


def make_attention(out_dir):
    from spikestack_lite.nn.attention import AstrocyteHebbianAttention

    res = {}
    for tag, (d, h, shape) in {
        "a": (64, 4, (3, 2, 16, 64)),    # temporal (T, B, N, d), dh = 16
        "b": (128, 2, (2, 1, 96, 128)),  # dh = 64 like the attention config
    }.items():
        torch.manual_seed(11)
        attn = AstrocyteHebbianAttention(d_model=d, num_heads=h).eval()
        x = torch.randn(*shape)
        q, k, v, o_in, y = _capture_attention(attn, x)
        res[f"{tag}_q"], res[f"{tag}_k"], res[f"{tag}_v"] = _np(q), _np(k), _np(v)
        res[f"{tag}_lam"] = _np(torch.sigmoid(attn.decay_logit))
        res[f"{tag}_attn"] = _np(o_in)
        res[f"{tag}_y"] = _np(y)
        res[f"{tag}_heads"] = np.int64(h)
        res[f"{tag}_eps"] = np.float64(attn.eps)
    np.savez_compressed(os.path.join(out_dir, "attention.npz"), **res)


def make_gsmc(out_dir):
    from spikestack_lite.nn.gsmc import FusedGSMC

    res = {}
    for pool in ("mean", "last"):
        torch.manual_seed(5)
        cell = FusedGSMC(d_model=32, pool=pool).eval()
        g = torch.Generator().manual_seed(6)
        x = (torch.rand(3, 2, 8, 32, generator=g) < 0.4).float() * 1.5
        with torch.no_grad():
            out = cell(x, T=3)
        res[f"{pool}_x"] = _np(x)
        res[f"{pool}_out"] = _np(out)
        for k_, v_ in cell.state_dict().items():
            res[f"{pool}_sd_{k_}"] = _np(v_)
    np.savez_compressed(os.path.join(out_dir, "gsmc.npz"), **res)


def _capture_model(model, x):
    cap = {}
    hs = [model.embedding.register_forward_hook(lambda m, i, o: cap.__setitem__("planes", o.detach().clone()))]
    for bi, blk in enumerate(model.blocks):
        def _blk(m, i, o, bi=bi):
            cap[f"block{bi}_in"] = i[0].detach().clone()
            cap[f"block{bi}_out"] = o.detach().clone()
        hs.append(blk.register_forward_hook(_blk))
    if model.gsmc is not None:
        hs.append(model.gsmc.register_forward_hook(lambda m, i, o: cap.__setitem__("gsmc_out", o.detach().clone())))
    with torch.no_grad():
        logits = model(x)
    for h in hs:
        h.remove()
    return logits, cap


def make_models(out_dir):
    from spikestack_lite.models.transformer import SpikingTransformer

    cfgs = {
        # the CPU-runnable model geometry (batch reduced from 256 to 4)
        "model_c1": (dict(input_dim=48, d_model=128, seq_len=64, num_classes=10, num_heads=4, num_layers=1,
                          n_repeats=3, temporal=True, expansion=4, use_spikeskip=True), (4, 64, 48)),
        # the full-model geometry shrunk (GSMC + exact head on, 2 layers, dh = 32)
        "model_c5_tiny": (dict(input_dim=32, d_model=64, seq_len=32, num_classes=10, num_heads=2, num_layers=2,
                               n_repeats=4, temporal=True, expansion=4, use_gsmc=True, use_exact=True,
                               use_spikeskip=True), (2, 32, 32)),
    }
    for name, (kw, xshape) in cfgs.items():
        torch.manual_seed(0)
        model = SpikingTransformer(**kw).eval()
        g = torch.Generator().manual_seed(1)
        x = torch.randn(*xshape, generator=g)
        logits, cap = _capture_model(model, x)
        res = {"x": _np(x), "logits": _np(logits)}
        for k_, v_ in cap.items():
            res["cap_" + k_] = _np(v_)
        for k_, v_ in model.state_dict().items():
            res["sd_" + k_] = _np(v_)
        res["config"] = np.array(repr(sorted(kw.items())))
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **res)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPIKESTACK_REFERENCE"),
                    help="reference checkout (default: $SPIKESTACK_REFERENCE)")
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference PATH or set SPIKESTACK_REFERENCE")
    sys.path.insert(0, a.reference)
    torch.set_num_threads(1)
    make_spike_linear(a.out)
    make_attention(a.out)
    make_gsmc(a.out)
    make_models(a.out)
    for f in sorted(os.listdir(a.out)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(a.out, f)))


if __name__ == "__main__":
    main()
