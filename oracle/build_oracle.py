"""TEST INFRASTRUCTURE ONLY: compile the C oracle (oracle/trident_oracle.c).

Two builds are made, one for x86-64-v3 (AVX2/FMA) and one for x86-64-v4 (AVX-512), because the
GPU box's host CPU is not known here; oracle.py picks the one the running CPU supports. The
outputs are git-ignored shared objects next to this file; they travel to the GPU box with the
snapshot. -ffp-contract=off keeps every float operation exactly as written (no implicit fusing).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "trident_oracle.c")
LEVELS = ("x86-64-v3", "x86-64-v4")


def lib_path(level: str) -> str:
    return os.path.join(HERE, f"liboracle_{level}.so")


def build(force: bool = False, quiet: bool = True) -> None:
    cc = os.environ.get("TRIDENT_ORACLE_CC", "/usr/bin/gcc")
    for level in LEVELS:
        out = lib_path(level)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(SRC):
            continue
        cmd = [cc, "-O3", f"-march={level}", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
               "-fPIC", "-shared", "-o", out + ".tmp", SRC, "-lm"]
        if not quiet:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        os.replace(out + ".tmp", out)


if __name__ == "__main__":
    build(force="--force" in sys.argv, quiet=False)
