"""Build the trident_b200 CUDA library (sm_100a) in-tree: trident_b200/libtrident_b200.so.

nvcc compiles every csrc/*.cu for `-gencode arch=compute_100a,code=sm_100a` (one process per source,
in parallel) and links one shared library exporting the C ABI of include/trident_b200.h. No fast-math: the exact-distance path must
keep IEEE fmaf/add semantics (the CPU oracle reproduces it bit for bit).
"""
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libtrident_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile each source to an object in parallel (trident_b200/_build/), then link the library."""
    if not force and not _stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC]
    if ptxas_info:
        flags.insert(0, "-Xptxas=-v")

    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    newest_header = max([os.path.getmtime(h) for h in headers] + [os.path.getmtime(__file__)])

    def compile_one(src):
        obj = os.path.join(objdir, os.path.splitext(os.path.basename(src))[0] + ".o")
        if not force and not ptxas_info and os.path.exists(obj) and \
                os.path.getmtime(obj) > max(os.path.getmtime(src), newest_header):
            return obj  # up to date
        cmd = [nvcc(), *flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        return obj

    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    out_tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", out_tmp, *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(out_tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
