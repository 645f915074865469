"""Stage Y on the tensor cores (tb_filter.cu) against the oracle and the CUDA-core Stage Y (needs a
B200 for the searches; the row_p check runs anywhere).

The tensor-core filter bounds each (query, row) pair from an exact int8 MMA of the row's SQ8 codes
with the query's split weights, and refines the survivors in the reference's FP32 order, so its
results must be bit-identical to the oracle's exact IVF-Flat and to the CUDA-core path's. The
library picks it by size (TRIDENT_INDEX_TENSOR_STAGE_Y_ALWAYS forces it, which the small cases here
need); the status-word checks repeat the wait-limit tests on this kernel.
"""
import numpy as np
import pytest

from helpers import CASE_NAMES, assert_same_topk, build_config_index, build_index, load_case, oracle_search


def _search(idx, xq, nprobe, K, mode=2):
    import torch

    d, i, _ = idx.search(torch.from_numpy(xq).cuda(), nprobe, mode=mode, k=K)
    torch.cuda.synchronize()
    return d.cpu().numpy().copy(), i.cpu().numpy().copy()


def _stats(idx, xq, nprobe, K):
    import torch

    st = torch.zeros(8, dtype=torch.int64, device="cuda")
    idx.search(torch.from_numpy(xq).cuda(), nprobe, mode=2, k=K, stats_buf=st)
    torch.cuda.synchronize()
    return st.cpu().numpy()


def test_row_p_is_the_rounded_down_row_term():
    """row_p[slot] = sum_d (code_d delta_d)^2 of the slot's row, in float64 rounded down to float32."""
    from helpers import sorted_storage  # noqa: F401

    f = load_case("g2_decay_c2")
    idx = build_index(f, device="cpu")
    h = idx.host_arrays()
    T, D_pad, nb = idx.tile_size, idx.D_pad, idx.num_blocks
    codes = h["codes"].reshape(-1, nb, T, 32).transpose(0, 2, 1, 3).reshape(-1, T, D_pad).astype(np.float64)
    toff = h["tile_off"]
    lists = np.repeat(np.arange(idx.nlist), np.diff(toff))
    p64 = ((codes * h["delta"][lists][:, None, :].astype(np.float64)) ** 2).sum(-1).reshape(-1)
    rp = idx.row_p().numpy().astype(np.float64)
    assert rp.shape == p64.shape
    assert (rp <= p64).all()
    assert np.allclose(rp, p64, rtol=1e-6, atol=0)


def test_set_stage_y_rejects_unknown_modes():
    f = load_case("g1_int_c1")
    idx = build_index(f, device="cpu")
    with pytest.raises(ValueError):
        idx.set_stage_y("sometimes")
    idx.set_stage_y("off")
    assert idx.stage_y == "off"


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASE_NAMES)
@pytest.mark.parametrize("K", [10, 100])
def test_forced_tensor_stage_y_equals_oracle_on_fixtures(name, K):
    f = load_case(name)
    idx = build_index(f, max_k=100)
    idx.set_stage_y("always")
    nprobe = int(f["nprobe"])
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"], nprobe, K)
    d, i = _search(idx, f["xq"], nprobe, K)
    assert idx.status() == 0
    assert_same_topk(d, i, od, oi)


@pytest.mark.gpu
@pytest.mark.parametrize("cfg_name,over", [
    # c4 shape: integer rows, D = 128, 1,526 rows per list, nprobe 256 (about 39 queries per list)
    ("c4", dict(N=1_000_000, nlist=656, nprobe=256, B=1000, K=10, n_comp=41)),
    # c3 shape: unit-norm real rows, D = 96 (D_pad 96: three code blocks)
    ("c3", dict(N=500_000, nlist=1024, nprobe=32, B=2000, K=10)),
    # c2 shape: D = 960, the wide variant (Hi and Lo converted separately), 256-row tiles
    ("c2", dict(N=200_000, nlist=1024, nprobe=64, B=1000, K=10)),
    # c3 shape at K = 100: 128-entry lists, every query's item lists filling past K
    ("c3", dict(N=500_000, nlist=1024, nprobe=32, B=2000, K=100)),
])
def test_tensor_and_cuda_core_stage_y_agree_at_config_shapes(cfg_name, over):
    from trident_b200 import datasets as ds

    ncomp = over.pop("n_comp", None)
    cfg = ds.scaled(ds.CONFIGS[cfg_name], **over)
    if ncomp:
        cfg = ds.Config(**{**cfg.__dict__, "n_comp": ncomp})
    xb, xq, cent, lids, idx = build_config_index(cfg, "kmeans")
    od, oi, _ = oracle_search(xb, lids, cent, xq[:64], cfg.nprobe, cfg.K)
    results = {}
    for mode in ("off", "always", "auto"):
        idx.set_stage_y(mode)
        results[mode] = _search(idx, xq, cfg.nprobe, cfg.K)
        assert idx.status() == 0
        assert_same_topk(results[mode][0][:64], results[mode][1][:64], od, oi)
    for mode in ("always", "auto"):
        assert np.array_equal(results[mode][1], results["off"][1])
        assert np.array_equal(results[mode][0].view(np.uint32), results["off"][0].view(np.uint32))
    # the same candidates enter Stage Y on both paths; the tensor-core filter scans all dims of each
    idx.set_stage_y("off")
    s_off = _stats(idx, xq, cfg.nprobe, cfg.K)
    idx.set_stage_y("always")
    s_on = _stats(idx, xq, cfg.nprobe, cfg.K)
    assert s_on[0] == s_off[0]
    assert s_on[1] == s_on[0] * idx.D_pad
    assert 0 < s_on[2] < 0.05 * s_on[0]  # survivors: a small share of the candidates


@pytest.mark.gpu
def test_tensor_stage_y_waits_that_give_up_mark_every_result():
    import torch

    from trident_b200 import _lib

    f = load_case("g3_norm_c3")
    idx = build_index(f)
    idx.set_stage_y("always")
    nprobe, K = int(f["nprobe"]), int(f["K"])
    try:
        for limits, status in (((0, -1), _lib.STATUS_LOCK_TIMEOUT), ((-1, 0), _lib.STATUS_MMA_TIMEOUT)):
            _lib.set_wait_limits(*limits)
            d, i = _search(idx, f["xq"], nprobe, K)
            assert np.isnan(d).all() and (i == -2).all()
            assert idx.status() & status
            _lib.set_wait_limits(-1, -1)
            d, i = _search(idx, f["xq"], nprobe, K)
            assert idx.status() == 0
            od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"], nprobe, K)
            assert_same_topk(d, i, od, oi)
    finally:
        _lib.set_wait_limits(-1, -1)
    torch.cuda.synchronize()


def test_stage_y_path_query():
    """trident_stage_y_tensor: the size rule (D_pad <= 256, B * nprobe >= 32768), the flag that forces
    the tensor cores, and what keeps the CUDA cores (no row_p, UB seeding inside items, K > 128)."""
    from trident_b200 import _lib

    f = load_case("g1_int_c1")  # D = 128
    idx = build_index(f, device="cpu")
    assert not idx.stage_y_tensor(48, 4)
    assert idx.stage_y_tensor(1000, 64)
    assert not idx.stage_y_tensor(1000, 64, ub_seed=2)
    assert not idx.stage_y_tensor(1000, 64, k=129)
    assert idx.stage_y_tensor(1000, 64, k=100)
    idx.set_stage_y("always")
    assert idx.stage_y_tensor(48, 4)
    idx.set_stage_y("off")
    assert not idx.stage_y_tensor(1000, 64)
    idx.set_stage_y("auto")
    d = idx.desc()
    wide = type(d).from_buffer_copy(d)
    wide.D, wide.D_pad, wide.num_blocks = 960, 960, 30
    assert _lib.lib().trident_stage_y_tensor(wide, 1000, 10, 64, 0) == 0


def _f32(x):
    return np.asarray(x, np.float64).astype(np.float32)


def _f32_down(x):
    """The largest float32 <= x (x >= 0)."""
    f = np.float32(x)
    return np.nextafter(f, np.float32(0)) if float(f) > x else f


def _fma32(a, b, c):
    """float32 fma: the exact float64 product of two float32 values, plus c, rounded once."""
    return _f32(np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64))


def _check_tensor_bound(idx, xq, centroids, mean64, R64, nprobe):
    """Restates filter_kernel's value v (float64 split weights with a measured residual, exact integer
    dot products, the kernel's float32 evaluation order) and asserts v - slack <= ||x^ - q~||^2 for
    every probed (query, row) pair. Returns the number of pairs checked."""
    from oracle import oracle as O

    h = idx.host_arrays()
    T, D_pad, nb = idx.tile_size, idx.D_pad, idx.num_blocks
    vec_off, tile_off = h["vec_off"], h["tile_off"]
    codes = h["codes"].reshape(-1, nb, T, 32).transpose(0, 2, 1, 3).reshape(-1, T, D_pad)
    rowp = idx.row_p().numpy()
    qrot = O.rotate_f64(xq, mean64, R64, D_pad)
    probe, _ = O.probe_select_f64(xq, centroids, nprobe)
    u = 2.0 ** -24
    checked = 0
    for qi in range(qrot.shape[0]):
        for c in probe[qi]:
            L = int(vec_off[c + 1] - vec_off[c])
            if L == 0:
                continue
            nt = (L + T - 1) // T
            cd = codes[tile_off[c]:tile_off[c] + nt].reshape(-1, D_pad)[:L].astype(np.int64)
            P = rowp[tile_off[c] * T + np.arange(L)]
            vm = h["vmin"][c].astype(np.float64)
            dl = h["delta"][c].astype(np.float64)
            b = vm - qrot[qi].astype(np.float64)
            w = dl * b
            sig = np.abs(w).max() / 127.0 if np.abs(w).max() > 0 else 1.0
            hi = np.clip(np.rint(w * (1.0 / sig)), -127, 127)
            r = w - sig * hi
            lo = np.clip(np.rint(r * (1.0 / sig) * 254.0), -127, 127)
            rmax = np.abs(r - sig * lo / 254.0).max() * (1 + 1e-9) + sig * 1e-12
            Hi, Lo = cd @ hi.astype(np.int64), cd @ lo.astype(np.int64)
            bsq = float((b * b).sum())
            pcap = float(((255.0 * dl) ** 2).sum())
            cmax = 255.0 * D_pad
            slack = 8 * u * (pcap + bsq + 2 * sig * 127 * cmax * (1 + 1 / 254)) + 2 * rmax * cmax
            base = _f32_down(bsq * (1 - 1e-12))
            s1 = _f32(P.astype(np.float64) + float(base))
            if D_pad <= 256:
                v = _fma32(_f32(2 * sig / 254), _f32(254 * Hi + Lo), s1)
            else:
                v = _fma32(_f32(2 * sig / 254), _f32(Lo), _fma32(_f32(2 * sig), _f32(Hi), s1))
            xhat = vm + cd * dl
            exact = ((xhat - qrot[qi].astype(np.float64)) ** 2).sum(axis=1)
            assert (v.astype(np.float64) - slack <= exact).all(), (qi, c)
            checked += L
    return checked


@pytest.mark.parametrize("name", CASE_NAMES)
def test_tensor_bound_never_exceeds_the_dequantised_distance(name):
    """On every fixture, v - slack of the tensor-core Stage Y is a lower bound of ||x^ - q~||^2."""
    f = load_case(name)
    idx = build_index(f, device="cpu")
    assert _check_tensor_bound(idx, f["xq"], f["centroids"], f["mean64"], f["R64"], int(f["nprobe"])) > 0


@pytest.mark.parametrize("D,offset,spread", [
    (960, 0.0, 1.0),      # the wide evaluation (Hi and Lo converted separately)
    (128, 3.0e4, 0.05),   # far from the origin, tiny spread: P, ||b||^2 and the cross term cancel
    (256, -1.0e3, 40.0),  # the largest narrow D_pad, mixed signs
])
def test_tensor_bound_holds_under_cancellation_and_wide_rows(D, offset, spread):
    from trident_b200 import SharedClusterStorage, TridentV4Index

    rng = np.random.default_rng(11)
    nlist, N = 8, 1600
    cent = (offset + spread * 20 * rng.standard_normal((nlist, D))).astype(np.float32)
    lids = rng.integers(0, nlist, N).astype(np.int32)
    xb = (cent[lids] + spread * rng.standard_normal((N, D))).astype(np.float32)
    xq = (cent[rng.integers(0, nlist, 12)] + spread * rng.standard_normal((12, D))).astype(np.float32)
    mean64 = np.zeros(D)
    R64 = np.linalg.qr(rng.standard_normal((D, D)))[0]
    st = SharedClusterStorage(xb, lids, None, nlist, device="cpu")
    idx = TridentV4Index(st, cent, mean64, R64, tile_size=128 if D < 256 else 256, device="cpu", max_batch=12,
                         max_nprobe=4)
    assert _check_tensor_bound(idx, xq, cent, mean64, R64, 4) > 0
