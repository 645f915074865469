"""Exact probe selection at the configs' list counts (needs a B200), through the C ABI.

probe_select_kernel has three ways to find the nprobe-th approximate coarse value before the exact
float64 re-check of the boundary:
  * nlist <= 1024: each thread's keys in registers (c1, c2; covered by test_gpu_search);
  * nlist <= 8192: the query's row cached in shared memory (c3: nlist 4096);
  * above that: an upper bound from the coarse GEMM's row minima over 64-list spans, then one pass
    over the row (c4: nlist 65,536; c5: 262,144), or, when nprobe exceeds the number of spans, an
    exact per-bit search that re-reads the row.
Each case checks the probe lists and their float64 distances bit for bit against the oracle
(oracle_probe_select_f64: the nprobe smallest float64 ||q - c||^2, ties to the smaller list id), and
the search's top-K (ids identical, distances bit-identical) against the oracle's exact IVF-Flat.
"""
import numpy as np
import pytest

from helpers import assert_same_topk, build_config_index, oracle_search

pytestmark = pytest.mark.gpu


def _build(cfg, centroid_mode, seed=7):
    return build_config_index(cfg, centroid_mode, seed)


def _coarse_matches_oracle(idx, xq, cent, nprobe):
    import torch

    from oracle import oracle as O

    cids, d64, _ = idx.coarse(torch.from_numpy(xq).cuda(), nprobe)
    torch.cuda.synchronize()
    oc, od = O.probe_select_f64(xq, cent, nprobe)
    got_c, got_d = cids.cpu().numpy(), d64.cpu().numpy()
    bad = np.nonzero((got_c != oc).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} probe lists differ, first q={bad[0]}"
    assert np.array_equal(got_d.view(np.uint64), od.view(np.uint64))
    return oc, od


def _search(idx, xq, nprobe, K, mode):
    import torch

    d, i, _ = idx.search(torch.from_numpy(xq).cuda(), nprobe, mode=mode, k=K)
    torch.cuda.synchronize()
    return d.cpu().numpy(), i.cpu().numpy()


@pytest.mark.parametrize("cfg_name,over,centroids,modes", [
    # c3 shape: real-valued rows, 4096 lists, the row cached in shared memory
    ("c3", dict(N=500_000, nlist=4096, nprobe=128, B=1000, K=10), "kmeans", (2, 10)),
    # c4 shape: 65,536 lists, the per-tile minimum bound; integer centroids give exact ties
    ("c4", dict(N=1_000_000, nlist=65_536, nprobe=256, B=1000, K=10), "rows", (2, 10)),
    # 16,384 lists from k-means (real-valued centroids), the per-tile minimum bound
    ("c4", dict(N=400_000, nlist=16_384, nprobe=64, B=1000, K=10), "kmeans", (2,)),
])
def test_probe_sets_and_topk_at_config_list_counts(cfg_name, over, centroids, modes):
    from trident_b200 import datasets as ds

    cfg = ds.scaled(ds.CONFIGS[cfg_name], **over)
    xb, xq, cent, lids, idx = _build(cfg, centroids)
    oc, _ = _coarse_matches_oracle(idx, xq, cent, cfg.nprobe)
    od, oi, ocids = oracle_search(xb, lids, cent, xq, cfg.nprobe, cfg.K)
    assert np.array_equal(ocids, oc)
    for mode in modes:
        d, i = _search(idx, xq, cfg.nprobe, cfg.K, mode)
        assert_same_topk(d, i, od, oi)


def test_probe_sets_when_nprobe_exceeds_the_span_count():
    """16,384 lists give 256 row minima over 64-list spans; nprobe = 300 cannot be bounded by them, so
    the exact per-bit search over the row in global memory runs."""
    from trident_b200 import datasets as ds

    cfg = ds.scaled(ds.CONFIGS["c4"], N=200_000, nlist=16_384, nprobe=300, B=300, K=10)
    _, xq, cent, _, idx = _build(cfg, "rows")
    _coarse_matches_oracle(idx, xq, cent, cfg.nprobe)
