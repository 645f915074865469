"""TEST INFRASTRUCTURE ONLY: build the reference's own CPU IVF-Flat into oracle/_ref/.

The reference keeps its exact CPU IVF-Flat (`omp_cpu_ivfflat_f32`, plus three helpers) as a C++
string, CPP_100M_HELPER, inside benchmarks/phase8_ooc_100m_4080.py:43-212, and JIT-builds it with
torch.utils.cpp_extension.load_inline (:214-225). This recipe does the same from the source where
it lies, with one textual change: the hard-coded `num_threads(24)` clauses (:63, :78, :103, :163)
become `num_threads(trident_ref_threads())`, which reads TRIDENT_REF_THREADS or else uses every
host core, so that the baseline uses the box's cores instead of 24.

Nothing is copied into the repository: the extracted source and the built module are written only
under oracle/_ref/, which git ignores. The module is built twice (x86-64-v3 and x86-64-v4) because
the host CPU that will run it is not known at build time; ref_cpu.py loads the one the running CPU
supports.
It runs only where the reference checkout is present (TRIDENT_REFERENCE_ROOT, else a `reference`
directory beside the repository root); machines without it use the prebuilt files.

build_gpu() also compiles the reference's GPU search, src/trident_v4_kernels.cu, unchanged, as the
torch extension its own suite JIT-builds (benchmarks/phase4a_suite.py:65-72, same flags: -O3
--use_fast_math -lineinfo) for sm_100a, into oracle/_ref/gpu/. ref_gpu.py drives it; tests use it to
pin the reference's GPU summation order against the oracle on the B200.
"""
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
REF_ROOT = os.environ.get("TRIDENT_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
REF_FILE = os.path.join(REF_ROOT, "benchmarks", "phase8_ooc_100m_4080.py")
REF_GPU_FILE = os.path.join(REF_ROOT, "src", "trident_v4_kernels.cu")
GPU_NAME = "trident_ref_v4"
GPU_DIR = os.path.join(OUT, "gpu")
LEVELS = {"x86-64-v3": "trident_ref_cpu_v3", "x86-64-v4": "trident_ref_cpu_v4"}

_THREADS_HELPER = """
#include <cstdlib>
static int trident_ref_threads() {
    const char* s = std::getenv("TRIDENT_REF_THREADS");
    int n = s ? std::atoi(s) : 0;
    return n > 0 ? n : omp_get_num_procs();
}
"""


def extract_source() -> str:
    with open(REF_FILE) as f:
        text = f.read()
    m = re.search(r'CPP_100M_HELPER\s*=\s*r"""(.*?)"""', text, re.S)
    if not m:
        raise RuntimeError(f"CPP_100M_HELPER not found in {REF_FILE}")
    src = m.group(1)
    n_sub = len(re.findall(r"num_threads\(24\)", src))
    src = src.replace("num_threads(24)", "num_threads(trident_ref_threads())")
    lines = src.split("\n")
    last_inc = max(i for i, l in enumerate(lines) if l.startswith("#include"))
    lines.insert(last_inc + 1, _THREADS_HELPER)
    if n_sub != 4:
        raise RuntimeError(f"expected 4 num_threads(24) clauses, found {n_sub}")
    return "\n".join(lines)


def available() -> bool:
    return os.path.exists(REF_FILE)


def module_path(level: str) -> str:
    name = LEVELS[level]
    return os.path.join(OUT, level, f"{name}.so")


def build(force: bool = False, quiet: bool = True) -> bool:
    """Build both variants; returns False when the reference is not mounted."""
    if not available():
        return False
    if not force and all(os.path.exists(module_path(l)) and os.path.getmtime(module_path(l)) >= os.path.getmtime(REF_FILE)
                         for l in LEVELS):
        return True
    os.environ["CXX"] = "/usr/bin/g++"  # the /opt/gcc wrapper lacks libgomp.spec
    from torch.utils.cpp_extension import load_inline

    src = extract_source()
    for level, name in LEVELS.items():
        bdir = os.path.join(OUT, level)
        os.makedirs(bdir, exist_ok=True)
        load_inline(name=name, cpp_sources=src,
                    extra_cflags=["-O3", "-fopenmp", f"-march={level}"],
                    extra_ldflags=["-fopenmp"], build_directory=bdir, verbose=not quiet)
    return True


def gpu_module_path() -> str:
    return os.path.join(GPU_DIR, f"{GPU_NAME}.so")


def build_gpu(force: bool = False, quiet: bool = True) -> bool:
    """Compile the reference GPU extension for sm_100a (nvcc cross-compiles; no GPU needed).
    Returns False when the reference is not mounted."""
    if not os.path.exists(REF_GPU_FILE):
        return False
    out = gpu_module_path()
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(REF_GPU_FILE):
        return True
    os.makedirs(GPU_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load

    # an explicit -gencode makes torch add no arch flags of its own
    load(name=GPU_NAME, sources=[REF_GPU_FILE], build_directory=GPU_DIR,
         extra_cflags=["-O3"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"],
         verbose=not quiet)
    return True


if __name__ == "__main__":
    ok = build(force="--force" in sys.argv, quiet=False)
    ok_gpu = build_gpu(force="--force" in sys.argv, quiet=False)
    print("built" if ok and ok_gpu else "reference not mounted; nothing built")
