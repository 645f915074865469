"""On-disk index artifacts: save a built index once, load it without rebuilding.

The reference caches its 100M index as `meta.npz` plus raw memory-mapped `.bin` files of the codes,
tile ids and u8 rows (benchmarks/phase8_ooc_100m_4080.py:228-248), and widens the u8 rows to float32
on the CPU at every load (:354). The same idea in this build's layout, one directory per index (a
list-sharded deployment saves each rank's shard into its own directory; row ids stay global):

  meta.npz      format version, shapes and scalars, centroids, ||c||^2, the PCA mean and rotation
                (float64), the list row and tile offsets, the per-list vmin / delta / eps
  rows.bin      the list-sorted rows [N, D]: uint8 when every value is an integer in [0, 255]
                (SIFT-shaped data, 4x smaller), float32 otherwise; uint8 rows are widened on the
                device while loading, so no host pass over the rows is needed
  ids.bin       [N] int32 original row ids
  codes.bin     the blocked SQ8 codes [tiles][blocks][tile rows][32] uint8, exactly as searched

Loading copies the files to the device in chunks (or, with host_rows=True, the rows into pinned host
memory for the out-of-core mode) and assembles the index without repeating the SQ8 build.
"""
import os

import numpy as np

FORMAT_VERSION = 1
_CHUNK_ROWS = 1 << 20


def _torch():
    import torch

    return torch


def _rows_fit_u8(xs) -> bool:
    """Whether every row value is an integer in [0, 255] (checked chunk by chunk on the rows' device)."""
    torch = _torch()
    for s in range(0, xs.shape[0], _CHUNK_ROWS):
        x = xs[s:s + _CHUNK_ROWS]
        if bool(((x < 0) | (x > 255) | (x != torch.round(x))).any()):
            return False
    return True


def _write(f, t, dtype=None):
    """Append tensor t (any device) to the open binary file f, in row chunks."""
    n = t.shape[0]
    step = max(1, _CHUNK_ROWS if t.dim() > 1 else _CHUNK_ROWS * 64)
    for s in range(0, n, step):
        a = t[s:s + step]
        if dtype is not None:
            a = a.to(dtype)
        a.cpu().numpy().tofile(f)


def save_index(index, path: str) -> None:
    """Write `index` (a built TridentV4Index) into directory `path` (created if missing)."""
    torch = _torch()
    os.makedirs(path, exist_ok=True)
    st = index.storage
    rows_u8 = _rows_fit_u8(st.xb_sorted)
    meta = dict(
        format_version=FORMAT_VERSION, N=index.N, D=index.D, nlist=index.nlist, tile_size=index.tile_size,
        num_blocks=index.num_blocks, total_tiles=index.total_tiles, per_cluster_sq8=index.per_cluster_sq8,
        use_pca=index.use_pca, centroid_norm_max=index.centroid_norm_max, lb_rel_slack=index.lb_rel_slack,
        rows_dtype="u8" if rows_u8 else "f32", codes_bytes=int(index.codes.numel()),
        centroids=index.centroids.cpu().numpy(), centroid_norm_sq=index.centroid_norm_sq.cpu().numpy(),
        mean64=np.asarray(index.mean64, np.float64), R64=np.asarray(index.R64, np.float64),
        vec_off=st.cluster_vec_off.cpu().numpy(), tile_off=index.cluster_tile_off.cpu().numpy(),
        vmin=index.vmin_pad.cpu().numpy(), delta=index.delta_pad.cpu().numpy(), eps=index.eps_pad.cpu().numpy(),
        counts=np.asarray(st.counts, np.int32),
    )
    tmp = os.path.join(path, "meta.tmp.npz")
    np.savez(tmp, **meta)
    with open(os.path.join(path, "rows.bin"), "wb") as f:
        _write(f, st.xb_sorted, torch.uint8 if rows_u8 else torch.float32)
    with open(os.path.join(path, "ids.bin"), "wb") as f:
        _write(f, st.orig_ids_sorted, torch.int32)
    with open(os.path.join(path, "codes.bin"), "wb") as f:
        _write(f, index.codes.view(-1), torch.uint8)
    os.replace(tmp, os.path.join(path, "meta.npz"))  # written last: a complete directory has it


def _to_device(mm, out, device):
    """Copy memmap rows into the preallocated tensor `out` chunk by chunk (widening uint8 to float32
    on the device when out is float32 and mm is uint8)."""
    torch = _torch()
    step = _CHUNK_ROWS if mm.ndim > 1 else _CHUNK_ROWS * 64
    for s in range(0, mm.shape[0], step):
        a = torch.from_numpy(np.array(mm[s:s + step]))  # a writable copy of the chunk
        if out.device.type == "cuda":
            a = a.to(out.device, non_blocking=False)
        out[s:s + a.shape[0]].copy_(a.to(out.dtype))


def load_index(path: str, device="cuda:0", host_rows: bool = False, max_batch: int = 1024,
               max_nprobe: int = 512, max_k: int = 100):
    """The index saved in `path`, on `device` (rows in pinned host memory with host_rows=True)."""
    torch = _torch()
    from .index import SharedClusterStorage, TridentV4Index

    meta = np.load(os.path.join(path, "meta.npz"))
    if int(meta["format_version"]) != FORMAT_VERSION:
        raise ValueError(f"{path}: artifact format {int(meta['format_version'])}, expected {FORMAT_VERSION}")
    dev = torch.device(device)
    N, D, nlist = int(meta["N"]), int(meta["D"]), int(meta["nlist"])
    rows_u8 = str(meta["rows_dtype"]) == "u8"
    rows_mm = np.memmap(os.path.join(path, "rows.bin"), dtype=np.uint8 if rows_u8 else np.float32, mode="r",
                        shape=(N, D)) if N else np.zeros((0, D), np.float32)
    ids_mm = np.memmap(os.path.join(path, "ids.bin"), dtype=np.int32, mode="r", shape=(N,)) if N else \
        np.zeros(0, np.int32)
    codes_mm = np.memmap(os.path.join(path, "codes.bin"), dtype=np.uint8, mode="r",
                         shape=(int(meta["codes_bytes"]),))

    st = SharedClusterStorage.__new__(SharedClusterStorage)
    st.dev, st.nlist, st.N, st.D = dev, nlist, N, D
    st.host_rows = bool(host_rows)
    if host_rows:
        st.xb_sorted = torch.empty((N, D), dtype=torch.float32, pin_memory=True)
        for s in range(0, N, _CHUNK_ROWS):
            st.xb_sorted[s:s + _CHUNK_ROWS].copy_(torch.from_numpy(np.array(rows_mm[s:s + _CHUNK_ROWS])))
    else:
        st.xb_sorted = torch.empty((N, D), dtype=torch.float32, device=dev)
        _to_device(rows_mm, st.xb_sorted, dev)
    st.orig_ids_sorted = torch.empty(N, dtype=torch.int32, device=dev)
    _to_device(ids_mm, st.orig_ids_sorted, dev)
    st.cluster_vec_off = torch.from_numpy(np.asarray(meta["vec_off"], np.int64)).to(dev)
    st.counts = np.asarray(meta["counts"], np.int32)
    st.list_ids_sorted = torch.repeat_interleave(torch.arange(nlist, device=dev),
                                                 torch.from_numpy(st.counts.astype(np.int64)).to(dev))
    st.sort_perm = np.asarray(ids_mm)
    st.r_vec_sorted = None

    codes = torch.empty(int(meta["codes_bytes"]), dtype=torch.uint8, device=dev)
    _to_device(codes_mm, codes, dev)
    f64 = lambda k: torch.from_numpy(np.ascontiguousarray(meta[k], np.float64)).to(dev)
    f32 = lambda k: torch.from_numpy(np.ascontiguousarray(meta[k], np.float32)).to(dev)
    arrays = dict(centroids=f32("centroids"), centroid_norm_sq=f32("centroid_norm_sq"), codes=codes,
                  vmin=f32("vmin"), delta=f32("delta"), eps=f32("eps"),
                  tile_off=torch.from_numpy(np.asarray(meta["tile_off"], np.int64)).to(dev),
                  pca_mean=f64("mean64"), pca_rot=f64("R64"))
    params = dict(tile_size=int(meta["tile_size"]), per_cluster_sq8=int(meta["per_cluster_sq8"]),
                  use_pca=int(meta["use_pca"]), centroid_norm_max=float(meta["centroid_norm_max"]),
                  lb_rel_slack=float(meta["lb_rel_slack"]), total_tiles=int(meta["total_tiles"]),
                  mean64=np.asarray(meta["mean64"], np.float64), R64=np.asarray(meta["R64"], np.float64))
    return TridentV4Index.from_arrays(st, arrays, params, device=dev, max_batch=max_batch, max_nprobe=max_nprobe,
                                     max_k=max_k)
