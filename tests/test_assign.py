"""trident_assign, the index build's list assignment on the tensor cores (needs a B200).

The kernel is the coarse stage's TMA-fed tcgen05 GEMM with an argmin epilogue and TF32 products.
The assignment is an input of the index, so it is checked against the float64 nearest centroid up
to the TF32 rounding: each row's chosen centroid is within the product error bound of the nearest,
|a - exact| <= 2^-9 * 2 sum_d |x_d c_d| + 2^-22 (D + 2) (||c||^2 + 2 sum_d |x_d c_d|) (operands
rounded to 10 mantissa bits, any accumulation order), and almost every row gets exactly it.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,D,nlist", [(5000, 128, 300), (20000, 96, 4096), (3000, 128, 65_536), (1, 8, 1)])
def test_assign_is_the_nearest_up_to_tf32_rounding(n, D, nlist):
    import torch

    from trident_b200.clustering import assign_tc

    rng = np.random.default_rng(n + D)
    cent = rng.standard_normal((nlist, D)).astype(np.float32) * 3
    x = (cent[rng.integers(0, nlist, n)] + rng.standard_normal((n, D))).astype(np.float32)
    got = assign_tc(torch.from_numpy(x).cuda(), torch.from_numpy(cent).cuda()).cpu().numpy()
    assert got.dtype == np.int32 and got.shape == (n,)
    assert ((got >= 0) & (got < nlist)).all()
    c64, x64 = cent.astype(np.float64), x.astype(np.float64)
    cn = (c64 ** 2).sum(1)
    for s in range(0, n, 1000):
        xs = x64[s:s + 1000]
        a = cn[None, :] - 2.0 * xs @ c64.T
        best = a.argmin(1)
        mag = np.abs(xs) @ np.abs(c64).T
        tol = 2.0 ** -9 * 2.0 * mag + 2.0 ** -22 * (D + 2) * (cn[None, :] + 2.0 * mag)
        rows = np.arange(len(xs))
        g = got[s:s + 1000]
        assert (a[rows, g] <= a[rows, best] + tol[rows, g] + tol[rows, best]).all()
    exact = 0
    for s in range(0, n, 1000):
        xs = x64[s:s + 1000]
        exact += int((got[s:s + 1000] == (cn[None, :] - 2.0 * xs @ c64.T).argmin(1)).sum())
    assert exact >= 0.98 * n


def test_assign_integer_rows_match_exact_argmin():
    """Small integers are exact in TF32, and with values in [0, 63] every partial sum stays below 2^22,
    so any accumulation the tensor core uses is exact: the assignment equals the exact argmin with
    ties to the smaller id."""
    import torch

    from trident_b200.clustering import assign_tc

    rng = np.random.default_rng(3)
    cent = rng.integers(0, 64, (1000, 128)).astype(np.float32)
    x = np.clip(cent[rng.integers(0, 1000, 20000)] + rng.integers(-8, 9, (20000, 128)), 0, 63).astype(np.float32)
    x[:10] = cent[:10]            # exact ties with other centroids are impossible; zero distance
    cent[500] = cent[7]           # a duplicate centroid: rows nearest to it must pick 7
    got = assign_tc(torch.from_numpy(x).cuda(), torch.from_numpy(cent).cuda()).cpu().numpy()
    c64 = cent.astype(np.int64)
    a = (c64 ** 2).sum(1)[None, :] - 2 * x.astype(np.int64) @ c64.T
    want = a.argmin(1)  # first minimum: the smaller id
    assert np.array_equal(got, want)


def test_assign_wait_limit_reports_status():
    import torch

    from trident_b200 import _lib
    from trident_b200.clustering import assign_tc

    x = torch.randn(4096, 64, device="cuda")
    c = torch.randn(512, 64, device="cuda")
    _lib.set_wait_limits(-1, 0)
    try:
        with pytest.raises(RuntimeError, match="bounded wait"):
            assign_tc(x, c)
    finally:
        _lib.set_wait_limits(-1, -1)
    got = assign_tc(x, c)
    assert int(got.min()) >= 0
