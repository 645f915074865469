"""TEST INFRASTRUCTURE ONLY: numpy front end of the C oracle (trident_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, and
only as the checker. The product package (trident_b200) never imports it.

Definitions (each restates the reference; see trident_oracle.c for the reference lines):
  * probe set: the nprobe smallest float64 direct ||q - c||^2 (fma, d ascending), ties to the
    smaller list id, ascending;
  * exact distance: FP32 in the reference GPU summation order;
  * top-K: total order (distance asc, id asc); missing slots are (+inf, -1).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = set()
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    break
        return {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags
    except OSError:
        return False


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    from . import build_oracle

    level = "x86-64-v4" if _cpu_has_avx512() else "x86-64-v3"
    path = build_oracle.lib_path(level)
    if not os.path.exists(path):
        build_oracle.build()
    L = ctypes.CDLL(path)
    P = ctypes.c_void_p
    i64, i32, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_float
    L.oracle_version.restype = i32
    L.oracle_max_threads.restype = i32
    L.oracle_l2_ref_order.restype = f32
    L.oracle_l2_ref_order.argtypes = [P, P, i32]
    L.oracle_l2_f64.restype = ctypes.c_double
    L.oracle_l2_f64.argtypes = [P, P, i32]
    L.oracle_probe_select_f64.restype = i32
    L.oracle_probe_select_f64.argtypes = [P, P, i64, i32, i32, i32, P, P, i32]
    L.oracle_ivf_search.restype = i32
    L.oracle_ivf_search.argtypes = [P, i64, i32, P, i32, P, P, P, i32, P, P, i32]
    L.oracle_rotate_f64.restype = i32
    L.oracle_rotate_f64.argtypes = [P, i64, i32, i32, P, P, P, i32]
    L.oracle_stage_y_profile.restype = i32
    L.oracle_stage_y_profile.argtypes = [i64, i32, i32, P, P, P, i32, P, P, P, P, P, P, P, P, P, P, i32]
    _LIB = L
    return L


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data_as(ctypes.c_void_p)


def l2_ref_order(x, q) -> np.float32:
    x, px = _c(x, np.float32)
    q, pq = _c(q, np.float32)
    return np.float32(lib().oracle_l2_ref_order(px, pq, int(x.shape[-1])))


def l2_f64(a, b) -> float:
    a, pa = _c(a, np.float32)
    b, pb = _c(b, np.float32)
    return float(lib().oracle_l2_f64(pa, pb, int(a.shape[-1])))


def probe_select_f64(xq, centroids, nprobe, nthreads=0):
    xq, pq = _c(xq, np.float32)
    cent, pc = _c(centroids, np.float32)
    B, D = xq.shape
    nlist = cent.shape[0]
    cids = np.empty((B, nprobe), np.int32)
    d64 = np.empty((B, nprobe), np.float64)
    rc = lib().oracle_probe_select_f64(pq, pc, B, D, nlist, nprobe, cids.ctypes.data_as(ctypes.c_void_p),
                                       d64.ctypes.data_as(ctypes.c_void_p), int(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle_probe_select_f64 failed ({rc})")
    return cids, d64


def ivf_search(xq, probe_cids, vec_off, xb_sorted, orig_ids_sorted, K, nthreads=0):
    xq, pq = _c(xq, np.float32)
    pc, ppc = _c(probe_cids, np.int32)
    vo, pvo = _c(vec_off, np.int64)
    xb, pxb = _c(xb_sorted, np.float32)
    oi, poi = _c(orig_ids_sorted, np.int32)
    B, D = xq.shape
    out_d = np.empty((B, K), np.float32)
    out_i = np.empty((B, K), np.int64)
    rc = lib().oracle_ivf_search(pq, B, D, ppc, int(pc.shape[1]), pvo, pxb, poi, int(K),
                                 out_d.ctypes.data_as(ctypes.c_void_p),
                                 out_i.ctypes.data_as(ctypes.c_void_p), int(nthreads))
    if rc != 0:
        raise RuntimeError(f"oracle_ivf_search failed ({rc})")
    return out_d, out_i


def rotate_f64(xq, mean64, R64, D_pad, nthreads=0):
    xq, pq = _c(xq, np.float32)
    mu, pmu = _c(mean64, np.float64)
    R, pR = _c(R64, np.float64)
    B, D = xq.shape
    out = np.empty((B, D_pad), np.float32)
    lib().oracle_rotate_f64(pq, B, D, int(D_pad), pmu, pR, out.ctypes.data_as(ctypes.c_void_p), int(nthreads))
    return out


def stage_y_profile(probe_cids, vec_off, tile_off, T, codes, vmin, delta, eps, qrot, tau_safe,
                    want_rows=False, nthreads=0):
    pc, ppc = _c(probe_cids, np.int32)
    vo, pvo = _c(vec_off, np.int64)
    to, pto = _c(tile_off, np.int64)
    cd, pcd = _c(codes, np.uint8)
    vm, pvm = _c(vmin, np.float32)
    dl, pdl = _c(delta, np.float32)
    ep, pep = _c(eps, np.float32)
    qr, pqr = _c(qrot, np.float32)
    ts, pts = _c(tau_safe, np.float32)
    B, nprobe = pc.shape
    D_pad = qr.shape[1]
    cand = np.zeros(B, np.int64)
    blocks = np.zeros(B, np.int64)
    surv = np.zeros(B, np.int64)
    rows = np.zeros(int(vo[-1]), np.int32) if want_rows else None
    lib().oracle_stage_y_profile(B, int(D_pad), int(nprobe), ppc, pvo, pto, int(T), pcd, pvm, pdl, pep, pqr, pts,
                                 cand.ctypes.data_as(ctypes.c_void_p), blocks.ctypes.data_as(ctypes.c_void_p),
                                 surv.ctypes.data_as(ctypes.c_void_p),
                                 rows.ctypes.data_as(ctypes.c_void_p) if want_rows else None, int(nthreads))
    return cand, blocks, surv, rows


def exact_search(xq, centroids, nprobe, vec_off, xb_sorted, orig_ids_sorted, K, nthreads=0):
    """The whole oracle: float64 probe selection, then exact IVF-Flat top-K."""
    cids, _ = probe_select_f64(xq, centroids, nprobe, nthreads)
    d, i = ivf_search(xq, cids, vec_off, xb_sorted, orig_ids_sorted, K, nthreads)
    return d, i, cids
