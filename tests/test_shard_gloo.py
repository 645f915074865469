"""List sharding across two processes with the gloo backend, on the CPU.

Each rank owns the lists `partition_lists` gives it and holds only their rows, selects the same
probe set from all centroids, searches its own rows (the CPU oracle stands in for the GPU index
here) and takes part in the all-gather of `ShardedSearch`. The merged top-K must equal the
unsharded oracle's. The bench runs the same protocol over NCCL with one GPU per rank.
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
    """This rank's rows behind the search() signature of TridentV4Index (CPU oracle)."""

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

    def search(self, xq, nprobe, mode=2, k=10, ub_seed=0, phase_ms=None):
        import torch

        from oracle import oracle as O

        xq = xq.numpy()
        cids, _ = O.probe_select_f64(xq, self.centroids, nprobe)
        d, i = O.ivf_search(xq, cids, self.off, self.xs, self.perm, k)
        return torch.from_numpy(np.ascontiguousarray(d)), torch.from_numpy(np.ascontiguousarray(i).astype(np.int64)), 0.0


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
        d, i = ss.search(torch.from_numpy(f["xq"]), int(f["nprobe"]), k=K)
        if rank == 0:
            np.savez(out_path, d=d.numpy(), i=i.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,K", [("g1_int_c1", 10), ("g3_norm_c3", 37)])
def test_two_rank_list_sharding_matches_unsharded(tmp_path, name, K):
    import torch.multiprocessing as mp

    out = str(tmp_path / "merged.npz")
    mp.start_processes(_rank, args=(2, _free_port(), name, K, out), nprocs=2, join=True, start_method="spawn")
    got = np.load(out)
    f = load_case(name)
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"], int(f["nprobe"]), K)
    assert_same_topk(got["d"], got["i"], od, oi)


def test_partition_is_balanced_and_total():
    from trident_b200.shard import partition_lists

    counts = np.random.default_rng(0).integers(0, 1000, 257)
    for R in (2, 3, 8):
        owner = partition_lists(counts, R)
        assert owner.min() >= 0 and owner.max() < R
        load = np.bincount(owner, weights=counts, minlength=R)
        assert load.sum() == counts.sum()
        assert load.max() - load.min() <= counts.max()  # greedy longest-first bound
