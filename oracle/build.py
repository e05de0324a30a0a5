"""Build recipe for the CPU oracle (test infrastructure, never the product).

`build()` compiles moe_oracle.cpp into oracle/_build/<variant>/liboracle_moe.so:
  - "portable": -march=x86-64-v3 (AVX2), the copy built by __graft_entry__.build()
    and shipped to GPU hosts, whose CPUs are unknown in advance;
  - "native":   -march=native, built on the machine that times the CPU baseline.
Both use -ffp-contract=off so the oracle's float operations round exactly as
written (see the header of moe_oracle.cpp).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "moe_oracle.cpp")

FLAGS = {
    "portable": ["-march=x86-64-v3"],
    "native": ["-march=native"],
}


def lib_path(variant="portable"):
    return os.path.join(HERE, "_build", variant, "liboracle_moe.so")


def build(variant="portable", force=False):
    out = lib_path(variant)
    if (not force and os.path.exists(out)
            and os.path.getmtime(out) >= os.path.getmtime(SRC)):
        return out
    os.makedirs(os.path.dirname(out), exist_ok=True)
    cmd = (["g++", "-O3", "-std=c++17", "-fopenmp", "-ffp-contract=off",
            "-fno-fast-math", "-shared", "-fPIC"] + FLAGS[variant]
           + [SRC, "-o", out + ".tmp"])
    subprocess.check_call(cmd)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    for v in (sys.argv[1:] or ["portable"]):
        print(build(v, force=True))
