"""Coarse clustering and residual PCA for the index build (host side, off the query path).

Mirrors the reference's `load_or_train_clustering` (benchmarks/phase4a_suite.py:389-439): train
nlist centroids, assign every row to its list, take r_vec = ||x - c(x)||, then PCA on the residuals
of a 50k-row sample (mean64, R64 with components in descending variance). The reference trains with
faiss k-means, which is not installed here; this module runs seeded Lloyd k-means on the given
device instead (same role: the centroids are inputs of the index, and search results given fixed
centroids do not depend on how they were trained).
"""
import os
import time
from typing import Optional, Tuple

import numpy as np

from .datasets import SEED_KMEANS, SEED_PCA


def _torch():
    import torch

    return torch


def _as_tensor(x, device):
    torch = _torch()
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.float32)
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device)


def assign_tc(x, centroids):
    """Nearest centroid of every row on the tensor cores (trident_assign: the coarse stage's TMA-fed
    tcgen05 GEMM with an argmin epilogue, TF32 products). x and centroids: contiguous float32 CUDA
    tensors with D % 4 == 0. Returns int32 list ids."""
    torch = _torch()
    from . import _lib

    n, D = (int(v) for v in x.shape)
    cn = (centroids.double() ** 2).sum(1).float().contiguous()
    out = torch.empty(n, dtype=torch.int32, device=x.device)
    status = torch.zeros(1, dtype=torch.int32, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    _lib.check(_lib.lib().trident_assign(x.data_ptr(), n, D, centroids.data_ptr(), cn.data_ptr(),
                                         int(centroids.shape[0]), out.data_ptr(), status.data_ptr(),
                                         stream.cuda_stream))
    if int(status.item()) != 0:
        raise RuntimeError(f"trident_assign: a bounded wait gave up (status {int(status.item())})")
    return out


def _tc_ok(x, centroids) -> bool:
    return (x.is_cuda and x.dtype == centroids.dtype == _torch().float32 and x.is_contiguous()
            and centroids.is_contiguous() and x.shape[1] % 4 == 0 and x.data_ptr() % 16 == 0
            and centroids.data_ptr() % 16 == 0)


def assign(x, centroids, chunk: int = 1 << 16, tf32: bool = False):
    """Nearest centroid (squared L2 via ||c||^2 - 2 x.c; ties to the smaller id). Returns int64 list
    ids on x's device. With tf32 the products run on the TF32 tensor cores (trident_assign on CUDA
    when the layout allows, else torch with TF32 matmuls): the list assignment is an input of the
    index (the search is exact for whatever assignment it is given), so it does not need float32
    rounding, and large builds run many times faster."""
    torch = _torch()
    if tf32 and _tc_ok(x, centroids):
        return assign_tc(x, centroids).long()
    cn = (centroids.double() ** 2).sum(1).float()
    out = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    ct = centroids.t().contiguous()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32) and x.is_cuda
    try:
        for s in range(0, x.shape[0], chunk):
            e = min(x.shape[0], s + chunk)
            d = torch.addmm(cn.unsqueeze(0), x[s:e], ct, beta=1.0, alpha=-2.0)
            out[s:e] = torch.argmin(d, dim=1)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out


def kmeans(sample, nlist: int, niter: int = 20, seed: int = SEED_KMEANS, tf32: bool = False):
    """Seeded Lloyd k-means on a float32 tensor; empty clusters are re-seeded by splitting the
    largest one (the faiss rule). Returns float32 centroids [nlist, D] on the sample's device."""
    torch = _torch()
    n, D = sample.shape
    if n < nlist:
        raise ValueError(f"k-means needs at least nlist={nlist} rows, got {n}")
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    init = torch.randperm(n, generator=g)[:nlist].to(sample.device)
    cent = sample[init].clone()
    for _ in range(niter):
        a = assign(sample, cent, tf32=tf32)
        sums = torch.zeros((nlist, D), dtype=torch.float64, device=sample.device)
        sums.index_add_(0, a, sample.double())
        cnt = torch.bincount(a, minlength=nlist)
        nz = cnt > 0
        cent_new = cent.clone()
        cent_new[nz] = (sums[nz] / cnt[nz].unsqueeze(1).double()).float()
        empty = torch.nonzero(~nz).flatten().tolist()
        if empty:
            cntl = cnt.clone()
            for e in empty:
                big = int(torch.argmax(cntl))
                eps = 1.0 / 1024.0
                base = cent_new[big].clone()
                cent_new[e] = base * (1 + eps)
                cent_new[big] = base * (1 - eps)
                half = int(cntl[big]) // 2
                cntl[e] = half
                cntl[big] -= half
        cent = cent_new
    return cent.contiguous()


def residual_pca(x, centroids, list_ids, sample_size: int = 50_000, seed: int = SEED_PCA):
    """Mean and eigenvectors (descending eigenvalue) of the residuals of a row sample, in float64."""
    torch = _torch()
    n = x.shape[0]
    m = min(sample_size, n)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    idx = torch.randperm(n, generator=g)[:m].to(x.device)
    r = x[idx].double() - centroids[list_ids[idx]].double()
    mean64 = r.mean(0)
    rc = r - mean64
    cov = rc.t() @ rc / max(m - 1, 1)
    evals, evecs = torch.linalg.eigh(cov)
    order = torch.argsort(evals, descending=True)
    R64 = evecs[:, order].contiguous()
    return mean64.cpu().numpy(), R64.cpu().numpy()


def train_clustering(xb, nlist: int, sample_size: Optional[int] = None, niter: int = 20, device=None,
                     seed: int = 0, tf32: Optional[bool] = None, chunk: int = 1 << 20):
    """(centroids, list_ids, r_vec, mean64, R64, train_s) as NumPy arrays, the reference's tuple.

    tf32 (default: on for more than 10^7 rows) runs the k-means and assignment products on the TF32
    tensor cores. Residual norms are computed in chunks, so no temporary of the rows' size exists."""
    torch = _torch()
    if device is None:
        device = xb.device if isinstance(xb, torch.Tensor) else "cpu"
    t0 = time.perf_counter()
    x = _as_tensor(xb, device)
    n = x.shape[0]
    if tf32 is None:
        tf32 = n > 10_000_000
    ss = min(n, sample_size or 64 * nlist)
    g = torch.Generator(device="cpu")
    g.manual_seed(SEED_KMEANS + 1000 * seed)
    sidx = torch.randperm(n, generator=g)[:ss].to(x.device)
    cent = kmeans(x[sidx].contiguous(), nlist, niter=niter, seed=SEED_KMEANS + 1000 * seed, tf32=tf32)
    del sidx
    lids = assign(x, cent, tf32=tf32)
    r_vec = torch.empty(n, dtype=torch.float32, device=x.device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        r_vec[s:e] = torch.linalg.norm(x[s:e] - cent[lids[s:e]], dim=1)
    mean64, R64 = residual_pca(x, cent, lids, seed=SEED_PCA + 1000 * seed)
    if x.is_cuda:
        torch.cuda.synchronize(x.device)
    train_s = time.perf_counter() - t0
    return (cent.cpu().numpy(), lids.to(torch.int32).cpu().numpy(), r_vec.float().cpu().numpy(),
            mean64, R64, train_s)


def load_or_train_clustering(dataset: str, xb, nlist: int, seed: int, cache_dir: Optional[str] = None,
                             device=None, sample_size: Optional[int] = None):
    """Drop-in for the reference helper of the same name: returns
    (centroids, list_ids, r_vec, mean64, R64, train_s), cached as .npz with an atomic rename."""
    cache_file = None
    if cache_dir:
        os.makedirs(cache_dir, exist_ok=True)
        cache_file = os.path.join(cache_dir, f"{dataset}_nlist{nlist}_s{seed}.npz")
        if os.path.exists(cache_file):
            d = np.load(cache_file)
            return (d["centroids"], d["list_ids"], d["r_vec"], d["mean64"], d["R64"], float(d["train_time_s"]))
    out = train_clustering(xb, nlist, sample_size=sample_size, device=device, seed=seed)
    if cache_file:
        tmp = cache_file + f".tmp_{os.getpid()}.npz"
        np.savez(tmp, centroids=out[0], list_ids=out[1], r_vec=out[2], mean64=out[3], R64=out[4],
                 train_time_s=out[5])
        os.replace(tmp, cache_file)
    return out
