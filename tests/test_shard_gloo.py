"""List sharding across two processes with the gloo backend, on the CPU.

Each rank owns the lists `partition_lists` gives it and holds only their rows, and brings its own
half of the queries. ShardedSearch then runs the staged protocol:
  - all-gather of the probe lists and queries;
  - threshold seed lists, gathered and merged into each query's threshold;
  - local scan, where nothing above the threshold is emitted;
  - all-to-all and merge.
The CPU oracle stands in for the GPU stages. Every rank's merged top-K must equal the unsharded
oracle's for its own queries. The bench runs the same protocol over NCCL with one GPU per rank.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from helpers import assert_same_topk, load_case, oracle_search, sorted_storage


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _OracleShard:
    """This rank's rows behind the staged-search methods of TridentV4Index (CPU oracle)."""

    def __init__(self, f, owner, rank):
        nlist = int(f["nlist"])
        xs, perm, off = sorted_storage(f["xb"], f["list_ids"], nlist)
        keep = np.concatenate([np.arange(off[c], off[c + 1]) for c in range(nlist) if owner[c] == rank]
                              + [np.zeros(0, np.int64)]).astype(np.int64)
        counts = np.array([off[c + 1] - off[c] if owner[c] == rank else 0 for c in range(nlist)], np.int64)
        self.off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
        self.xs = np.ascontiguousarray(xs[keep])
        self.perm = np.ascontiguousarray(perm[keep])
        self.centroids = f["centroids"]
        self.D_pad = (f["xb"].shape[1] + 31) // 32 * 32

    def _local(self, xq, probe, k):
        from oracle import oracle as O

        return O.ivf_search(xq.numpy(), np.ascontiguousarray(probe.numpy()), self.off, self.xs, self.perm, k)

    def search_prep(self, xq, nprobe):
        import torch

        from oracle import oracle as O

        cids, _ = O.probe_select_f64(xq.numpy(), self.centroids, nprobe)
        B = xq.shape[0]
        return (torch.from_numpy(np.ascontiguousarray(cids).astype(np.int32)),
                torch.zeros((B, self.D_pad), dtype=torch.float32), torch.zeros((B, 4), dtype=torch.float32))

    def search_seed(self, xq_all, probe, qrot, qinfo, nprobe, k=10, mode=2, ub_seed=0):
        import torch

        d, i = self._local(xq_all, probe, k)  # exact distances of distinct local rows
        return torch.from_numpy(np.ascontiguousarray(d)), torch.from_numpy(np.ascontiguousarray(i).astype(np.int64))

    def search_finish(self, xq_all, tau, nprobe, k=10, mode=2, ub_seed=0):
        import torch

        probe = torch.from_numpy(np.ascontiguousarray(self._probe_all(xq_all, nprobe)))
        d, i = self._local(xq_all, probe, k)
        drop = d > tau.numpy()[:, None]  # what the scan emits: nothing above the threshold
        d, i = d.copy(), i.astype(np.int64)
        d[drop], i[drop] = np.inf, -1
        return torch.from_numpy(d), torch.from_numpy(i)

    def _probe_all(self, xq_all, nprobe):
        from oracle import oracle as O

        cids, _ = O.probe_select_f64(xq_all.numpy(), self.centroids, nprobe)
        return cids.astype(np.int32)


def _merge_host(d_all, i_all):
    import torch

    from trident_b200.shard import merge_topk_host

    d, i = merge_topk_host(d_all.numpy(), i_all.numpy(), d_all.shape[2])
    return torch.from_numpy(d), torch.from_numpy(i)


def _rank(rank, world, port, name, K, out_path):
    import torch
    import torch.distributed as dist

    from trident_b200.shard import ShardedSearch, partition_lists

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        f = load_case(name)
        counts = np.bincount(f["list_ids"], minlength=int(f["nlist"]))
        owner = partition_lists(counts, world)
        ss = ShardedSearch(_OracleShard(f, owner, rank), merge=_merge_host)
        xq = f["xq"]
        B = xq.shape[0] // world  # every rank brings its own slice of the queries
        d, i = ss.search(torch.from_numpy(np.ascontiguousarray(xq[rank * B:(rank + 1) * B])), int(f["nprobe"]), k=K)
        np.savez(out_path + f".{rank}.npz", d=d.numpy(), i=i.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,K", [("g1_int_c1", 10), ("g3_norm_c3", 37)])
def test_two_rank_list_sharding_matches_unsharded(tmp_path, name, K):
    import torch.multiprocessing as mp

    out = str(tmp_path / "merged")
    mp.start_processes(_rank, args=(2, _free_port(), name, K, out), nprocs=2, join=True, start_method="spawn")
    parts = [np.load(out + f".{r}.npz") for r in range(2)]
    f = load_case(name)
    B = f["xq"].shape[0] // 2
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"][:2 * B], int(f["nprobe"]), K)
    assert_same_topk(np.concatenate([p["d"] for p in parts]), np.concatenate([p["i"] for p in parts]), od, oi)


def test_partition_is_balanced_and_total():
    from trident_b200.shard import partition_lists

    counts = np.random.default_rng(0).integers(0, 1000, 257)
    for R in (2, 3, 8):
        owner = partition_lists(counts, R)
        assert owner.min() >= 0 and owner.max() < R
        load = np.bincount(owner, weights=counts, minlength=R)
        assert load.sum() == counts.sum()
        assert load.max() - load.min() <= counts.max()  # greedy longest-first bound


def test_list_work_estimate_and_balanced_partition():
    """Work = rows x (1 + probes of the sample); the partition balances that work across ranks."""
    import torch

    from trident_b200.shard import list_work_estimate, partition_lists

    rng = np.random.default_rng(4)
    nlist, D, R = 64, 16, 4
    cent = rng.standard_normal((nlist, D)).astype(np.float32) * 4
    counts = rng.integers(1, 200, nlist)
    # a sample concentrated near the first 8 centroids: those lists are probed far more often
    hot = rng.integers(0, 8, 500)
    sample = (cent[hot] + 0.1 * rng.standard_normal((500, D))).astype(np.float32)
    work = list_work_estimate(torch.from_numpy(sample), torch.from_numpy(cent), counts, nprobe=2)
    d = ((sample[:, None, :].astype(np.float64) - cent[None]) ** 2).sum(-1)
    freq = np.bincount(np.argsort(d, axis=1, kind="stable")[:, :2].ravel(), minlength=nlist)
    assert np.array_equal(work, counts * (freq + 1))
    owner = partition_lists(work, R)
    load = np.bincount(owner, weights=work, minlength=R)
    assert load.max() <= load.mean() + work.max()  # greedy bound: within one list of the mean
