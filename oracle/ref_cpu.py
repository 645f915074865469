"""TEST INFRASTRUCTURE ONLY: load the reference's CPU IVF-Flat built by ref_build.py.

The module exposes the reference functions unchanged (omp_cpu_ivfflat_f32 and helpers). It is used
to pin the oracle (tests) and as the timed CPU baseline (bench.py --impl reference). Loading needs
only the prebuilt module under oracle/_ref/, not the reference sources.
"""
import importlib.machinery
import importlib.util
import os

from . import ref_build
from .oracle import _cpu_has_avx512

_MOD = None


def load():
    """Return the reference CPU module, or raise FileNotFoundError if it was never built."""
    global _MOD
    if _MOD is not None:
        return _MOD
    import torch  # noqa: F401  (the module links against libtorch)

    level = "x86-64-v4" if _cpu_has_avx512() else "x86-64-v3"
    path = ref_build.module_path(level)
    if not os.path.exists(path):
        if ref_build.available():
            ref_build.build()
        if not os.path.exists(path):
            raise FileNotFoundError(f"reference CPU module not built: {path}")
    name = ref_build.LEVELS[level]
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _MOD = mod
    return mod
