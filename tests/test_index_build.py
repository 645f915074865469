"""Index build (host side, CPU): same array semantics as the reference's TridentV4Index build, the
B200 blocked code layout, and soundness of the Stage-Y bound's eps."""
import numpy as np
import pytest

from helpers import CASE_NAMES, build_index, load_case


def _unblock(codes, tile_off, vec_off, T, D_pad):
    """[tiles][nb][T][32] -> [N, D_pad] in sorted-row order."""
    nb = D_pad // 32
    tiles = codes.reshape(-1, nb, T, 32).transpose(0, 2, 1, 3).reshape(-1, T, D_pad)
    N = int(vec_off[-1])
    out = np.zeros((N, D_pad), np.uint8)
    for c in range(len(vec_off) - 1):
        for v in range(vec_off[c], vec_off[c + 1]):
            loc = v - vec_off[c]
            out[v] = tiles[tile_off[c] + loc // T, loc % T]
    return out


@pytest.mark.parametrize("name", CASE_NAMES)
def test_build_matches_reference_arrays(name):
    f = load_case(name)
    idx = build_index(f, device="cpu")
    h = idx.host_arrays()
    assert np.array_equal(h["orig_ids_sorted"], f["ref_sort_perm"])
    nz = idx.storage.counts > 0
    # vmin / delta: the reference rotates with NumPy's float64 matmul, this build with torch's;
    # after rounding to float32 they agree to an ulp at most
    np.testing.assert_array_max_ulp(h["vmin"][nz], f["ref_vmin"][nz], maxulp=1)
    np.testing.assert_array_max_ulp(h["delta"][nz], f["ref_delta"][nz], maxulp=2)
    mine = _unblock(h["codes"], h["tile_off"], h["vec_off"], idx.tile_size, idx.D_pad)
    ref = f["ref_codes"]
    diff = mine.astype(np.int32) - ref.astype(np.int32)
    assert np.abs(diff).max() <= 1
    assert (diff != 0).mean() < 1e-4


@pytest.mark.parametrize("name", CASE_NAMES)
def test_eps_bounds_quantisation_error(name):
    f = load_case(name)
    idx = build_index(f, device="cpu")
    h = idx.host_arrays()
    D, D_pad = idx.D, idx.D_pad
    xs = h["xb_sorted"].astype(np.float64)
    x_rot = np.zeros((xs.shape[0], D_pad))
    x_rot[:, :D] = (xs - f["mean64"]) @ f["R64"]
    codes = _unblock(h["codes"], h["tile_off"], h["vec_off"], idx.tile_size, D_pad)
    lid = np.repeat(np.arange(idx.nlist), np.diff(h["vec_off"]))
    xhat = h["vmin"][lid].astype(np.float64) + codes * h["delta"][lid].astype(np.float64)
    err = np.abs(x_rot - xhat)
    assert (err <= h["eps"][lid]).all()
    # not needlessly loose: about half a quantisation step, except on degenerate dims whose range
    # is at the float32 rounding level of the coordinate (e.g. the zero-variance direction of
    # rows normalised to unit sum), where the rounding terms dominate
    nz = idx.storage.counts > 0
    vm, dl, ep = h["vmin"][nz][:, :D], h["delta"][nz][:, :D], h["eps"][nz][:, :D]
    normal = dl > 1e-4 * np.abs(vm)
    if name != "g4_ties":  # the tie fixture has many single-valued dims per list
        assert normal.mean() > 0.9
    assert (ep[normal] / dl[normal]).max() < 0.51


@pytest.mark.parametrize("name", ["g1_int_c1", "g2_decay_c2", "g3_norm_c3"])
def test_stage_y_bound_never_exceeds_exact_distance(name):
    """LB soundness: the float32 bound the kernel evaluates, on every (query, row), stays below the
    exact distance once the query-side slack sigma and rho are applied."""
    from oracle import oracle as O

    f = load_case(name)
    idx = build_index(f, device="cpu")
    h = idx.host_arrays()
    D, D_pad = idx.D, idx.D_pad
    qrot = O.rotate_f64(f["xq"], f["mean64"], f["R64"], D_pad)
    codes = _unblock(h["codes"], h["tile_off"], h["vec_off"], idx.tile_size, D_pad)
    lid = np.repeat(np.arange(idx.nlist), np.diff(h["vec_off"]))
    rho = idx.lb_rel_slack
    u = 2.0 ** -24
    for j in range(0, f["xq"].shape[0], 4):
        qn = np.linalg.norm(f["xq"][j].astype(np.float64) - f["mean64"])
        sigma = 3.0001 * u * qn * (1 + 1e-6) + np.sqrt(D_pad) * (D + 2) * 2.0 ** -52 * qn
        base = (h["vmin"][lid] - qrot[j]).astype(np.float32)
        uu = np.abs(codes.astype(np.float32) * h["delta"][lid] + base)  # float32 like the kernel (up to fma)
        l = np.maximum(uu - h["eps"][lid], 0).astype(np.float64)
        lb = (l * l).sum(1)
        exact = ((h["xb_sorted"].astype(np.float64) - f["xq"][j].astype(np.float64)) ** 2).sum(1)
        ok = np.sqrt(lb) <= np.sqrt(exact * (1 + rho)) + sigma + 1e-12
        assert ok.all(), f"query {j}: bound above the exact distance on {np.count_nonzero(~ok)} rows"
        assert (lb > 0).any()  # the bound is not trivially zero
