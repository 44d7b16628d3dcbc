"""Build recipe for the oracle's C restatement (oracle/csr_oracle.c).

Output: oracle/_build/liboracle.so (git-ignored; it travels to the GPU box with
the working tree).  Test infrastructure only.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build_oracle(force=False):
    out_dir = os.path.join(HERE, "_build")
    os.makedirs(out_dir, exist_ok=True)
    src = os.path.join(HERE, "csr_oracle.c")
    out = os.path.join(out_dir, "liboracle.so")
    if force or not os.path.exists(out) or os.path.getmtime(out) < os.path.getmtime(src):
        subprocess.check_call(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", out, src, "-lm"])
    return out


if __name__ == "__main__":
    print(build_oracle(force=True))
