"""Multi-GPU list sharding (one process per GPU; new relative to the single-GPU reference).

The IVF lists are split across R ranks (greedy largest-first onto the least-loaded rank, ties by list
id), weighing each list by its length or, better, by its expected scan work (list_work_estimate).
Every rank holds ALL centroids, mean64 and R64 but only the rows of its own lists: lists owned by
other ranks are empty in its index. Each rank brings its own B queries; a step over the R * B
queries of all ranks runs the staged search:

  1. coarse stage on the rank's own queries (probe lists, rotated queries, side info);
  2. all-gather of those and of the query vectors over all ranks (NVLink);
  3. pairs + Stage X seed of the whole batch over the local lists -> each query's K smallest
     seed values of the local rows;
  4. all-gather + merge of those lists -> each query's threshold: the K-th smallest over
     distinct rows of all ranks, which bounds the final K-th distance;
  5. Stage Y/Z over the local lists -> per-query top-K of the local rows [R * B, K];
  6. all-to-all: rank r receives every rank's lists for its own B queries, and
     trident_merge_shards merges them under the (distance, id) order.

Per-rank work stays constant as R grows (1/R of the lists for R times the queries), so the
bench reports weak scaling. The merged result is identical to the single-GPU one.
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


def list_work_estimate(sample, centroids, counts, nprobe: int, chunk: int = 4096) -> np.ndarray:
    """Expected scan work of each list, for balancing the partition: rows x (1 + how many of the
    `sample` rows probe the list among their nprobe nearest centroids). A list's scan cost grows with
    the queries that probe it, not only with its length; rows of the dataset stand in for queries
    (they come from the same distribution). `sample` and `centroids` are float32 tensors on one
    device (float32 products: only the counts matter). Returns int64 [nlist]."""
    import torch

    nlist = int(centroids.shape[0])
    cn = (centroids.double() ** 2).sum(1).float()
    freq = torch.zeros(nlist, dtype=torch.int64, device=sample.device)
    ct = centroids.t().contiguous()
    k = min(int(nprobe), nlist)
    for s in range(0, int(sample.shape[0]), chunk):
        d = torch.addmm(cn.unsqueeze(0), sample[s:s + chunk], ct, beta=1.0, alpha=-2.0)
        idx = torch.topk(d, k, dim=1, largest=False).indices
        freq += torch.bincount(idx.flatten(), minlength=nlist)
    counts = torch.as_tensor(np.asarray(counts, np.int64), device=sample.device)
    return (counts * (freq + 1)).cpu().numpy()


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

    `index` is this rank's TridentV4Index, built over the rows of its own lists (shard_rows) and
    the full set of centroids (any object with search_prep / search_seed / search_finish works).
    search() takes this rank's own queries and returns their merged top-k. Every rank must call it
    with the same batch size, k, nprobe and mode.
    """

    def __init__(self, index, group=None, merge=None):
        import torch.distributed as dist

        self.index = index
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.merge = merge  # (d_all [R,B,K], i_all [R,B,K]) -> (d, i); None: the device merge

    def _merge(self, d_all, i_all):
        if self.merge is not None:
            return self.merge(d_all, i_all)
        from .index import merge_shards

        return merge_shards(d_all, i_all)

    @staticmethod
    def _pack(d, i):
        """[n, k] float32 distances + [n, k] int64 ids -> one [n, 3k] int32 tensor."""
        import torch

        return torch.cat([d.contiguous().view(torch.int32), i.contiguous().view(torch.int32)], dim=1)

    @staticmethod
    def _unpack(p, R, n, k):
        """[R * n, 3k] int32 -> ([R, n, k] float32, [R, n, k] int64), both contiguous."""
        import torch

        d = p[:, :k].contiguous().view(torch.float32).view(R, n, k)
        i = p[:, k:].contiguous().view(torch.int64).view(R, n, k)
        return d, i

    def _gather(self, t):
        import torch
        import torch.distributed as dist

        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        return out

    def search(self, xq, nprobe: int, k: int = 10, mode: int = 2, ub_seed: int = 0, phase_ms=None, stats_buf=None):
        import torch
        import torch.distributed as dist

        R, B = self.world, int(xq.shape[0])
        timed = phase_ms is not None and xq.is_cuda
        evs = []

        def mark(name):
            if timed:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                evs.append((name, e))

        mark("coarse")
        probe, qrot, qinfo = self.index.search_prep(xq, nprobe)
        mark("gather")
        # one all-gather of each query's [xq | q~ | qinfo | probe ids] as 32-bit words
        D, Dp, Q = int(xq.shape[1]), int(qrot.shape[1]), int(qinfo.shape[1])
        pack = torch.cat([xq.view(torch.int32), qrot.view(torch.int32), qinfo.view(torch.int32), probe], dim=1)
        allp = self._gather(pack)
        xq_all = allp[:, :D].contiguous().view(torch.float32)
        qrot_all = allp[:, D:D + Dp].contiguous().view(torch.float32)
        qinfo_all = allp[:, D + Dp:D + Dp + Q].contiguous().view(torch.float32)
        probe_all = allp[:, D + Dp + Q:].contiguous()
        mark("seed")
        seed_d, seed_i = self.index.search_seed(xq_all, probe_all, qrot_all, qinfo_all, nprobe, k=k, mode=mode,
                                                ub_seed=ub_seed)
        mark("tau")
        sd_all, si_all = self._unpack(self._gather(self._pack(seed_d, seed_i)), R, R * B, k)
        tau = self._merge(sd_all, si_all)[0][:, k - 1].contiguous()
        mark("scan")
        kw = {} if stats_buf is None else {"stats_buf": stats_buf}  # counters of this rank's scan
        d_loc, i_loc = self.index.search_finish(xq_all, tau, nprobe, k=k, mode=mode, ub_seed=ub_seed, **kw)
        mark("exchange")
        # rank-major chunks of B queries: rank r receives chunk r of every rank -> [R, B, k]
        loc = self._pack(d_loc, i_loc)
        inc = torch.empty_like(loc)
        dist.all_to_all_single(inc, loc, group=self.group)
        d_in, i_in = self._unpack(inc, R, B, k)
        mark("merge")
        out = self._merge(d_in, i_in)
        mark("end")
        if timed:
            evs[-1][1].synchronize()
            phase_ms.clear()
            for (n, a), (_, b) in zip(evs[:-1], evs[1:]):
                phase_ms[n] = a.elapsed_time(b)
        return out
