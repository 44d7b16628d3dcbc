"""Build the reference's own CUDA engines from its sources, as a second checker.

Compiles, from a checkout of Griffith-7/spikestack-lite (``--reference PATH``
or the SPIKESTACK_REFERENCE environment variable; read-only), the three
engines on the hot path

    spikestack_lite/sparse/src/sparse_linear.cu   -> oracle/_ref/spikeskip_ref/
    spikestack_lite/nn/src/attention_cuda.cu      -> oracle/_ref/attention_ref/
    spikestack_lite/nn/src/gsmc_cuda.cu           -> oracle/_ref/gsmc_ref/

as PyTorch extensions for sm_100a with torch.utils.cpp_extension (not the
reference's own setup.py).  Outputs go only to oracle/_ref/ (git-ignored; the
built .so files travel to the GPU box with the working tree, the sources do
not).  TEST INFRASTRUCTURE ONLY: tests load these modules to compare against
the reference engine on the GPU; the product never touches them.
"""
import argparse
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
ENGINES = {
    "spikeskip_ref": "spikestack_lite/sparse/src/sparse_linear.cu",
    "attention_ref": "spikestack_lite/nn/src/attention_cuda.cu",
    "gsmc_ref": "spikestack_lite/nn/src/gsmc_cuda.cu",
}


def build_ref(reference=None, verbose=False):
    """Compile the reference engines from the checkout at ``reference`` (or the
    directory named by the SPIKESTACK_REFERENCE environment variable)."""
    from torch.utils.cpp_extension import load

    reference = reference or os.environ.get("SPIKESTACK_REFERENCE")
    if not reference:
        raise RuntimeError("no reference checkout given: pass --reference PATH or set SPIKESTACK_REFERENCE")

    built = {}
    for name, rel in ENGINES.items():
        src = os.path.join(reference, rel)
        if not os.path.exists(src):
            continue
        bdir = os.path.join(REF_DIR, name)
        os.makedirs(bdir, exist_ok=True)
        load(name=name, sources=[src], build_directory=bdir, verbose=verbose,
             extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
             extra_cflags=["-O3"])
        built[name] = os.path.join(bdir, name + ".so")
    return built


def load_ref(name):
    """Import a reference engine built by build_ref() (no rebuild, no sources
    needed).  Returns None when it was not built."""
    path = os.path.join(REF_DIR, name, name + ".so")
    if not os.path.exists(path):
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SPIKESTACK_REFERENCE"),
                    help="reference checkout (default: $SPIKESTACK_REFERENCE)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference PATH or set SPIKESTACK_REFERENCE")
    print(build_ref(a.reference, verbose=True))
    sys.exit(0)
