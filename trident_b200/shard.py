"""Multi-GPU list sharding (one process per GPU; new relative to the single-GPU reference).

The IVF lists are split across R ranks (greedy longest-first on list length, ties by list id).
Every rank holds ALL centroids, mean64 and R64 but only the rows of its own lists: lists owned by
other ranks are empty in its index. So every rank runs the identical coarse stage and selects the
identical probe set with no communication, scans only its own lists, and produces a per-query
top-K. The R lists are exchanged with one all-gather of [B, K] (float32 distance, int64 id) and
merged by trident_merge_shards under the same (distance, id) order, which makes the sharded result
identical to the single-GPU one.

Optional threshold exchange (min-all-reduce of each query's K-th distance after the warm-up pass)
is not needed for correctness; any rank's K-th distance bounds the global one.
"""
from typing import List

import numpy as np


def partition_lists(counts, R: int) -> np.ndarray:
    """owner[c] in [0, R): longest list first onto the least-loaded rank (ties: lower rank)."""
    counts = np.asarray(counts, np.int64)
    order = np.lexsort((np.arange(len(counts)), -counts))
    load = np.zeros(R, np.int64)
    owner = np.empty(len(counts), np.int32)
    for c in order:
        r = int(np.argmin(load))
        owner[c] = r
        load[r] += counts[c]
    return owner


def shard_rows(list_ids, owner, rank: int) -> np.ndarray:
    """Row indices (original ids) of the lists that `rank` owns."""
    list_ids = np.asarray(list_ids)
    return np.nonzero(owner[list_ids] == rank)[0]


def merge_topk_host(d_all, i_all, K: int):
    """NumPy reference of the shard merge: d_all/i_all [R, B, K] -> [B, K] by (d asc, id asc)."""
    R, B, _ = d_all.shape
    d = np.transpose(d_all, (1, 0, 2)).reshape(B, -1)
    i = np.transpose(i_all, (1, 0, 2)).reshape(B, -1)
    out_d = np.full((B, K), np.inf, np.float32)
    out_i = np.full((B, K), -1, np.int64)
    for q in range(B):
        valid = i[q] >= 0
        dq, iq = d[q][valid], i[q][valid]
        o = np.lexsort((iq, dq))[:K]
        out_d[q, : len(o)] = dq[o]
        out_i[q, : len(o)] = iq[o]
    return out_d, out_i


class ShardedSearch:
    """Search over a list-sharded index with torch.distributed (NCCL on GPUs, gloo in tests).

    `index` is this rank's TridentV4Index, built over the rows of its own lists (shard_rows) and the
    full set of centroids. search() runs the local query path, all-gathers the [B, K] lists and
    merges them on the device.
    """

    def __init__(self, index, group=None, merge=None):
        import torch.distributed as dist

        self.index = index
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.merge = merge  # (d_all [R,B,K], i_all [R,B,K]) -> (d, i); None: the device merge

    def search(self, xq_gpu, nprobe: int, k: int = 10, mode: int = 2, ub_seed: int = 0, phase_ms=None):
        import torch
        import torch.distributed as dist

        d_loc, i_loc, _ = self.index.search(xq_gpu, nprobe, mode=mode, k=k, ub_seed=ub_seed, phase_ms=phase_ms)
        B = d_loc.shape[0]
        # rank-major [R * B, K] (the shape every backend accepts), viewed as [R, B, K]
        d_all = torch.empty((self.world * B, k), dtype=torch.float32, device=d_loc.device)
        i_all = torch.empty((self.world * B, k), dtype=torch.int64, device=d_loc.device)
        dist.all_gather_into_tensor(d_all, d_loc.contiguous(), group=self.group)
        dist.all_gather_into_tensor(i_all, i_loc.contiguous(), group=self.group)
        d_all = d_all.view(self.world, B, k)
        i_all = i_all.view(self.world, B, k)
        if self.merge is not None:
            return self.merge(d_all, i_all)
        from .index import merge_shards

        return merge_shards(d_all, i_all)
