"""On-disk index artifacts (trident_b200.artifacts): a saved index loads back with every array equal,
without repeating the SQ8 build. The CPU tests build and load on the host; the GPU test checks that
the loaded index searches bit for bit like the one that was saved."""
import numpy as np
import pytest

from helpers import build_index, load_case

ARRAYS = ("centroids", "centroid_norm_sq", "codes", "vmin_pad", "delta_pad", "eps_pad", "cluster_tile_off",
          "pca_mean", "pca_rot")


@pytest.mark.parametrize("name,rows_dtype", [("g1_int_c1", "u8"), ("g3_norm_c3", "f32")])
def test_save_load_round_trip_on_the_host(tmp_path, name, rows_dtype):
    from trident_b200 import load_index, save_index

    f = load_case(name)
    idx = build_index(f, device="cpu")
    save_index(idx, str(tmp_path))
    meta = np.load(tmp_path / "meta.npz")
    assert str(meta["rows_dtype"]) == rows_dtype
    got = load_index(str(tmp_path), device="cpu")
    for a in ARRAYS:
        assert np.array_equal(getattr(got, a).numpy(), getattr(idx, a).numpy()), a
    for a in ("xb_sorted", "orig_ids_sorted", "cluster_vec_off", "list_ids_sorted"):
        assert np.array_equal(getattr(got.storage, a).numpy(), getattr(idx.storage, a).numpy()), a
    assert np.array_equal(got.storage.counts, idx.storage.counts)
    for k in ("N", "D", "D_pad", "nlist", "tile_size", "num_blocks", "total_tiles", "centroid_norm_max",
              "lb_rel_slack"):
        assert getattr(got, k) == getattr(idx, k), k
    # the tensor-core Stage Y's row terms come out the same from the loaded codes and deltas
    assert np.array_equal(got.row_p().numpy(), idx.row_p().numpy())
    # the C ABI accepts the loaded descriptor
    d = got.desc()
    assert d.N == idx.N and d.nlist == idx.nlist


def test_load_rejects_another_format(tmp_path):
    from trident_b200 import load_index, save_index

    f = load_case("g1_int_c1")
    save_index(build_index(f, device="cpu"), str(tmp_path))
    meta = dict(np.load(tmp_path / "meta.npz"))
    meta["format_version"] = np.array(99)
    np.savez(tmp_path / "meta.npz", **meta)
    with pytest.raises(ValueError, match="artifact format"):
        load_index(str(tmp_path), device="cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["g1_int_c1", "g2_decay_c2"])
def test_loaded_index_searches_bit_for_bit(tmp_path, name):
    import torch

    from trident_b200 import load_index, save_index

    f = load_case(name)
    idx = build_index(f, device="cuda:0")
    save_index(idx, str(tmp_path))
    got = load_index(str(tmp_path), device="cuda:0")
    xq = torch.from_numpy(f["xq"]).cuda()
    for mode in (2, 10):
        d0, i0, _ = idx.search(xq, int(f["nprobe"]), mode=mode, k=int(f["K"]))
        d0, i0 = d0.cpu().numpy().copy(), i0.cpu().numpy().copy()
        d1, i1, _ = got.search(xq, int(f["nprobe"]), mode=mode, k=int(f["K"]))
        torch.cuda.synchronize()
        assert np.array_equal(i1.cpu().numpy(), i0)
        assert np.array_equal(d1.cpu().numpy().view(np.uint32), d0.view(np.uint32))
