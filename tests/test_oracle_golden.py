"""Pins the CPU oracle against the reference itself (CPU only).

The fixtures hold the reference's own results: its exact CPU IVF-Flat (omp_cpu_ivfflat_f32) on
the oracle's float64 probe sets, and its Python index build. See tests/golden/make_golden.py.
"""
import numpy as np
import pytest

from helpers import CASE_NAMES, load_case, sorted_storage
from oracle import oracle as O


@pytest.mark.parametrize("name", CASE_NAMES)
def test_probe_selection_is_deterministic(name):
    f = load_case(name)
    cids, d64 = O.probe_select_f64(f["xq"], f["centroids"], int(f["nprobe"]))
    assert np.array_equal(cids, f["probe"])
    assert np.array_equal(d64, f["probe_d64"])
    # ascending by (d64, cid) and equal to a brute-force float64 numpy ranking
    q = f["xq"].astype(np.float64)
    c = f["centroids"].astype(np.float64)
    full = ((q[:, None, :] - c[None, :, :]) ** 2).sum(-1)
    for j in range(q.shape[0]):
        order = np.lexsort((np.arange(c.shape[0]), full[j]))[: int(f["nprobe"])]
        assert np.array_equal(order, cids[j])


@pytest.mark.parametrize("name", CASE_NAMES)
def test_oracle_matches_reference_cpu_ivfflat(name):
    """Oracle top-K == the reference's omp_cpu_ivfflat_f32 on the same probes."""
    f = load_case(name)
    xs, perm, off = sorted_storage(f["xb"], f["list_ids"], int(f["nlist"]))
    assert np.array_equal(perm, f["ref_sort_perm"])
    od, oi = O.ivf_search(f["xq"], f["probe"], off, xs, perm, int(f["K"]))
    rd, ri = f["ref_topk_d"], f["ref_topk_i"]
    integer_valued = np.array_equal(f["xb"], np.rint(f["xb"])) and np.array_equal(f["xq"], np.rint(f["xq"]))
    if integer_valued:
        # every summation order is exact below 2^24: bit-identical results, ties by id
        assert np.array_equal(oi, ri)
        assert np.array_equal(od, rd)
    else:
        # the reference CPU loop sums in a different order: distances agree to float32 rounding and
        # ids agree except where two candidates are within that rounding (the reference's audit
        # class "f32_ulps", benchmarks/phase3a_lossless_audit.py:99-114)
        np.testing.assert_allclose(od, rd, rtol=1e-5)
        for j in range(od.shape[0]):
            if not np.array_equal(oi[j], ri[j]):
                gap = np.abs(np.diff(od[j])).min()
                assert gap <= 1e-5 * od[j].max(), f"query {j}: id mismatch without a near tie"


def test_ties_are_broken_by_id():
    f = load_case("g4_ties")
    xs, perm, off = sorted_storage(f["xb"], f["list_ids"], int(f["nlist"]))
    od, oi = O.ivf_search(f["xq"], f["probe"], off, xs, perm, int(f["K"]))
    n_ties = 0
    for j in range(od.shape[0]):
        for k in range(od.shape[1] - 1):
            assert od[j, k] <= od[j, k + 1]
            if od[j, k] == od[j, k + 1]:
                assert oi[j, k] < oi[j, k + 1]
                n_ties += 1
    assert n_ties > 50  # the fixture really exercises ties


def _round_f32(fr):
    """Correctly rounded (ties to even) float32 of an exact rational (normal range only)."""
    from fractions import Fraction

    if fr == 0:
        return np.float32(0.0)
    sign = -1 if fr < 0 else 1
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    scaled = a / Fraction(2) ** (e - 23)  # in [2^23, 2^24)
    m = scaled.numerator // scaled.denominator
    rem = scaled - m
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and m % 2 == 1):
        m += 1
    return np.float32(sign * float(Fraction(m) * Fraction(2) ** (e - 23)))


def _fmaf(a, b, c):
    from fractions import Fraction

    return _round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def _warp_order_python(x, q):
    """Pure-Python simulation of 32 lanes + shfl_down butterfly (small sizes only), with an exact
    single-rounding fmaf."""
    D = len(x)
    f32 = np.float32
    parts = []
    for lane in range(32):
        p = f32(0.0)
        d = 4 * lane
        while d + 3 < D:
            for j in range(4):
                df = f32(x[d + j]) - f32(q[d + j])
                p = _fmaf(df, df, p)
            d += 128
        dr = d
        while dr < d + 4 and dr < D:
            df = f32(x[dr]) - f32(q[dr])
            p = _fmaf(df, df, p)
            dr += 1
        parts.append(p)
    off = 16
    while off > 0:
        for lane in range(off):
            parts[lane] = f32(parts[lane] + parts[lane + off])
        off //= 2
    return parts[0]


@pytest.mark.parametrize("D", [1, 3, 4, 17, 96, 128, 130, 200, 300])
def test_reference_summation_order(D):
    rng = np.random.default_rng(D)
    for _ in range(20):
        x = (rng.standard_normal(D) * rng.choice([1e-3, 1.0, 1e3], D)).astype(np.float32)
        q = (rng.standard_normal(D) * rng.choice([1e-3, 1.0, 1e3], D)).astype(np.float32)
        assert O.l2_ref_order(x, q) == _warp_order_python(x, q)


def test_rotation_oracle_is_float64_rounded_once():
    f = load_case("g2_decay_c2")
    D = int(f["D"])
    D_pad = ((D + 31) // 32) * 32
    qr = O.rotate_f64(f["xq"], f["mean64"], f["R64"], D_pad)
    ref = (f["xq"].astype(np.float64) - f["mean64"]) @ f["R64"]
    assert np.all(qr[:, D:] == 0)
    np.testing.assert_allclose(qr[:, :D], ref, rtol=1e-6, atol=1e-12)
