"""The C-ABI library loads and exports every symbol include/*.h declares; host-only entry points
behave as documented (no GPU needed: nothing here launches a kernel)."""
import ctypes
import glob
import os
import re

import pytest

from helpers import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(trident_[a-z_0-9]+)\s*\(", text, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def L():
    from trident_b200 import _lib, build

    build.build()
    return _lib.lib()


def test_header_declares_the_path():
    names = declared_functions()
    for n in ("trident_search", "trident_coarse", "trident_workspace_size", "trident_merge_shards"):
        assert n in names


def test_every_declared_symbol_is_exported(L):
    from trident_b200 import _lib

    for n in declared_functions():
        assert hasattr(L, n), f"{n} declared in include/ but not exported"
    assert set(_lib.EXPORTED) <= set(declared_functions())


def test_version(L):
    assert L.trident_version() == 2


def test_noalloc_size_matches_the_header(L):
    from trident_b200 import _lib

    text = open(os.path.join(ROOT, "include", "trident_b200.h")).read()
    m = re.search(r"#define TRIDENT_NOALLOC_WORKSPACE_BYTES \((\d+)u \* (\d+)u \* (\d+)u\)", text)
    assert m, "macro not found"
    assert _lib.noalloc_workspace_bytes() == int(m.group(1)) * int(m.group(2)) * int(m.group(3))


def test_wait_limits_and_status_arguments(L):
    from trident_b200 import _lib

    assert L.trident_set_wait_limits(0, 0) == 0
    assert L.trident_set_wait_limits(-1, -1) == 0  # back to the defaults
    st = ctypes.c_int32(7)
    assert L.trident_workspace_status(None, None, ctypes.byref(st)) == _lib.TRIDENT_ERR_INVALID
    assert L.trident_workspace_status(4097 * 256 + 16, None, ctypes.byref(st)) == _lib.TRIDENT_ERR_INVALID
    assert "aligned" in _lib.last_error()


@pytest.mark.parametrize("B,K,nprobe,expect", [
    (1000, 10, 16, 2), (1000, 10, 64, 3), (1, 10, 64, 1), (1, 50, 64, 3), (1000, 10, 1, 0), (100, 10, 2, 2),
])
def test_p_init_rule(L, B, K, nprobe, expect):
    # the reference's warm-up split (src/trident_v4_kernels.cu:1269-1274)
    assert L.trident_p_init(2, B, K, nprobe) == expect
    assert L.trident_p_init(10, B, K, nprobe) == 0


def _desc(N=100_000, D=128, nlist=256, tile=128):
    from trident_b200 import _lib

    d = _lib.TridentIndexDesc()
    d.N, d.D, d.D_pad, d.nlist = N, D, ((D + 31) // 32) * 32, nlist
    d.tile_size, d.num_blocks = tile, d.D_pad // 32
    for f in ("xb_sorted", "orig_ids_sorted", "list_row_off", "list_tile_off", "codes", "vmin", "delta", "eps",
              "centroids", "centroid_norm_sq", "pca_mean", "pca_rot"):
        setattr(d, f, 4096)  # placeholder addresses: never dereferenced by host-only calls
    d.centroid_norm_max = 1.0
    d.lb_rel_slack = 1e-5
    return d


@pytest.mark.parametrize("cfg,B,nprobe,mode", [
    # W = B * nprobe * (N / nlist) * D against W0 = 9e8 (phase4a_suite.py:1013-1035, 1079) at C1-C4
    ((100_000, 128, 256), 1000, 16, 10),
    ((1_000_000, 960, 1024), 1000, 64, 2),
    ((10_000_000, 96, 4096), 1, 32, 10),
    ((10_000_000, 96, 4096), 100, 32, 10),
    ((10_000_000, 96, 4096), 100, 128, 2),
    ((10_000_000, 96, 4096), 10_000, 32, 2),
    ((100_000_000, 128, 65_536), 10_000, 256, 2),
])
def test_router(L, cfg, B, nprobe, mode):
    """The reference's rule with its A100 threshold gives the reference's decisions; the library
    default (the B200 calibration, where the cascade won at every measured batch) picks the cascade
    for every one of these workloads."""
    N, D, nlist = cfg
    d = _desc(N, D, nlist)
    assert L.trident_route(ctypes.byref(d), B, nprobe, 9.0e8) == mode
    assert L.trident_route(ctypes.byref(d), B, nprobe, 0.0) == 2


def test_index_check_errors(L):
    from trident_b200 import _lib

    assert L.trident_index_check(None) == _lib.TRIDENT_ERR_INVALID
    d = _desc()
    assert L.trident_index_check(ctypes.byref(d)) == 0
    d.D_pad = 100
    assert L.trident_index_check(ctypes.byref(d)) == _lib.TRIDENT_ERR_INVALID
    assert "D_pad" in _lib.last_error()
    d = _desc(tile=64)
    assert L.trident_index_check(ctypes.byref(d)) == _lib.TRIDENT_ERR_UNSUPPORTED
    d = _desc()
    d.codes = 4097
    assert L.trident_index_check(ctypes.byref(d)) == _lib.TRIDENT_ERR_INVALID


def test_workspace_size_is_monotone(L):
    d = _desc()
    sz = ctypes.c_size_t(0)
    prev = 0
    for B, K, np_ in [(1, 1, 1), (10, 10, 16), (1000, 10, 16), (1000, 100, 16), (1000, 100, 256)]:
        assert L.trident_workspace_size(ctypes.byref(d), B, K, np_, ctypes.byref(sz)) == 0
        assert sz.value >= prev
        prev = sz.value


def test_search_argument_errors(L):
    from trident_b200 import _lib

    d = _desc()
    sz = ctypes.c_size_t(0)
    L.trident_workspace_size(ctypes.byref(d), 4, 10, 8, ctypes.byref(sz))
    ws = 1 << 20  # fake 256-aligned address; B = 0 or a rejected argument never touches it
    args = lambda B, K, np_, mode, ub, wsb: L.trident_search(ctypes.byref(d), 4096, B, K, np_, mode, ub, ws, wsb,
                                                            4096, 4096, None, None)
    assert args(0, 10, 8, 2, 0, sz.value) == 0                                   # empty batch: no work
    assert args(4, 0, 8, 2, 0, sz.value) == _lib.TRIDENT_ERR_UNSUPPORTED          # K < 1
    assert args(4, 101, 8, 2, 0, sz.value) == _lib.TRIDENT_ERR_UNSUPPORTED        # K > 100
    assert args(4, 10, 300, 2, 0, sz.value) == _lib.TRIDENT_ERR_INVALID           # nprobe > nlist
    assert args(4, 10, 8, 2, 0, sz.value - 1) == _lib.TRIDENT_ERR_WORKSPACE       # workspace too small
    assert args(4, 10, 8, 2, 3, sz.value) == _lib.TRIDENT_ERR_INVALID             # ub_seed
    assert args(4, 10, 8, 0, 0, sz.value) == _lib.TRIDENT_ERR_UNSUPPORTED         # ablation mode 0
    assert args(4, 10, 8, 11, 0, sz.value) == _lib.TRIDENT_ERR_UNSUPPORTED        # Tribase mode 11
