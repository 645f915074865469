"""The arrays oracle/ref_gpu.py restates for the reference's GPU search, checked on the CPU against
the arrays the reference's own Python index build made for the golden fixtures
(benchmarks/phase4a_suite.py:110-255, saved by tests/golden/make_golden.py).

The packed codes are unpacked with the fixtures' own unpacker, so the tile / warp / lane layout is
checked along with the values."""
import numpy as np
import pytest

from helpers import CASE_NAMES, load_case, sorted_storage


def _ref_index(f, **kw):
    import torch

    from oracle.ref_gpu import RefGpuIndex

    xs, perm, off = sorted_storage(f["xb"], f["list_ids"], int(f["nlist"]))
    return RefGpuIndex(torch.from_numpy(xs), torch.from_numpy(perm), off, f["centroids"], f["mean64"], f["R64"],
                       tile_size=int(f["tile"]), max_batch=int(f["B"]), max_nprobe=int(f["nprobe"]), **kw), off


@pytest.mark.parametrize("name", CASE_NAMES)
def test_restated_reference_arrays_match_the_reference_build(name):
    import make_golden

    f = load_case(name)
    r, off = _ref_index(f)
    assert np.array_equal(r.orig_ids_sorted.numpy(), f["ref_sort_perm"])
    nz = np.diff(off) > 0
    np.testing.assert_array_max_ulp(r.vmin_pad.numpy()[nz], f["ref_vmin"][nz], maxulp=1)
    np.testing.assert_array_max_ulp(r.delta_pad.numpy()[nz], f["ref_delta"][nz], maxulp=2)
    codes = make_golden.unpack_codes(r.sq8_packed.numpy(), r.tile_orig_ids.numpy(), off, np.diff(off), r.D_pad,
                                     r.tile_size)
    diff = codes.astype(np.int32) - f["ref_codes"].astype(np.int32)
    assert np.abs(diff).max() <= 1 and (diff != 0).mean() < 1e-4
    # ids in tile order, -1 past each list's last row
    ids = r.tile_orig_ids.numpy()
    assert (ids >= 0).sum() == r.N
    assert np.array_equal(np.sort(ids[ids >= 0]), np.arange(r.N))
    b = r.blk_bounds4.numpy()
    assert b[0] == 0 and b[-1] == r.D_pad // 4 and (np.diff(b) == 8).all()


def test_reference_search_refuses_what_its_kernels_cannot_hold():
    import torch

    f = load_case("g1_int_c1")
    r, _ = _ref_index(f, build_sq8=False)
    xq = torch.from_numpy(f["xq"])
    with pytest.raises(ValueError, match="K = 10"):
        r.search(xq, 4, mode=10, k=5)
    with pytest.raises(ValueError, match="SQ8"):
        r.search(xq, 4, mode=2)
    with pytest.raises(ValueError, match="nprobe"):
        r.search(xq, int(f["nlist"]) + 1, mode=10)
    with pytest.raises(ValueError, match="modes"):
        r.search(xq, 4, mode=1)
