"""Shared test helpers: golden fixtures, index construction and result comparison."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GOLDEN = os.path.join(HERE, "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

CASE_NAMES = ("g1_int_c1", "g2_decay_c2", "g3_norm_c3", "g4_ties")


def load_case(name):
    """Fixture arrays plus the regenerated base rows / queries (checksums verified)."""
    import make_golden  # tests/golden/make_golden.py

    f = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    cfg, tile, xb, xq = make_golden.case_data(name)
    assert make_golden.checksum(xb) == str(f["xb_sha"]), f"{name}: base-row generator drifted"
    assert make_golden.checksum(xq) == str(f["xq_sha"]), f"{name}: query generator drifted"
    f.update(cfg=cfg, xb=xb, xq=xq)
    return f


def build_index(f, device="cuda:0", tile_size=None, host_rows=False, **kw):
    from trident_b200 import SharedClusterStorage, TridentV4Index, choose_tile

    xb = f["xb"]
    st = SharedClusterStorage(xb, f["list_ids"], None, int(f["nlist"]), device=device, host_rows=host_rows)
    ts = tile_size or choose_tile(xb.shape[1])
    return TridentV4Index(st, f["centroids"], f["mean64"], f["R64"], tile_size=ts, device=device, **kw)


def sorted_storage(xb, list_ids, nlist):
    perm = np.argsort(list_ids, kind="stable").astype(np.int32)
    counts = np.bincount(list_ids, minlength=nlist)
    off = np.zeros(nlist + 1, np.int64)
    off[1:] = np.cumsum(counts)
    return np.ascontiguousarray(xb[perm]), perm, off


def oracle_search(xb, list_ids, centroids, xq, nprobe, K):
    from oracle import oracle as O

    nlist = centroids.shape[0]
    xs, perm, off = sorted_storage(xb, np.asarray(list_ids), nlist)
    d, i, cids = O.exact_search(xq, centroids, nprobe, off, xs, perm, K)
    return d, i, cids


def assert_same_topk(d, i, od, oi, exact_dist=True, rtol=1e-5):
    """ids identical; distances bit-identical (exact_dist) or within rtol."""
    d = np.asarray(d)
    i = np.asarray(i)
    bad = np.nonzero((i != oi).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} queries differ, first q={bad[0]}: got {i[bad[0]]} {d[bad[0]]} " \
                          f"want {oi[bad[0]]} {od[bad[0]]}"
    fin = np.isfinite(od)
    assert (np.isfinite(d) == fin).all()
    if exact_dist:
        assert np.array_equal(d[fin].view(np.uint32), od[fin].view(np.uint32)), \
            f"max |dd| = {np.abs(d[fin] - od[fin]).max()}"
    else:
        np.testing.assert_allclose(d[fin], od[fin], rtol=rtol)


def build_config_index(cfg, centroid_mode, seed=7, tile_size=None):
    """Rows and queries of cfg's distribution and an index over them (needs a GPU). Centroids from a
    short k-means ("kmeans") or sampled rows ("rows": integer-valued for the integer mixtures, so
    exact float64 ties occur at the nprobe boundary). Returns (xb, xq, centroids, list_ids, index)."""
    import torch

    from trident_b200 import SharedClusterStorage, TridentV4Index, choose_tile, datasets as ds
    from trident_b200.clustering import assign, train_clustering

    xb = ds.generate_np(cfg, cfg.N, ds.SEED_BASE)
    xq = ds.generate_np(cfg, cfg.B, ds.SEED_QUERY)
    if centroid_mode == "kmeans":
        cent, lids, _, mu, R, _ = train_clustering(xb, cfg.nlist, sample_size=min(cfg.N, 16 * cfg.nlist), niter=4,
                                                   device="cuda:0")
    else:
        rng = np.random.default_rng(seed)
        cent = np.ascontiguousarray(xb[rng.choice(cfg.N, cfg.nlist, replace=False)])
        xg = torch.from_numpy(xb).cuda()
        lids = assign(xg, torch.from_numpy(cent).cuda()).to(torch.int32).cpu().numpy()
        del xg
        mu = np.zeros(cfg.D)
        R = np.linalg.qr(rng.standard_normal((cfg.D, cfg.D)))[0]
    st = SharedClusterStorage(xb, lids, None, cfg.nlist, device="cuda:0")
    idx = TridentV4Index(st, cent, mu, R, tile_size=tile_size or choose_tile(cfg.D), device="cuda:0",
                         max_batch=cfg.B, max_nprobe=cfg.nprobe)
    return xb, xq, cent, lids, idx
