"""Drop-in host API of the TRIDENT query path: SharedClusterStorage and TridentV4Index.

Mirrors the reference classes of benchmarks/phase4a_suite.py:75-342 (same constructor arguments,
same `search` signature and return order: distances, ids, kernel ms) on top of the B200 C ABI
(include/trident_b200.h). PyTorch only allocates and hands over device memory; every search-path
computation runs in the CUDA library, and there is no CPU fallback.

Index build (off the query path, host side; reference :75-255):
  * rows are stably sorted by list id (cluster-major storage);
  * each row is rotated, x~ = (x - mean64) R64 in float64, and rounded to float32;
  * per list and dim: vmin = min x~, delta = max((max - min)/255, 1e-12) (float32 arithmetic),
    codes = clip(round((x~ - vmin)/delta), 0, 255);
  * eps, the bound on |x~ - (vmin + code * delta)| that keeps the Stage-Y lower bound sound, is
    measured per list and dim in float64 and widened by the float32 rounding of the kernel's bound
    arithmetic (the reference used eps = 0.5001 * delta, :179, without such an argument);
  * codes are stored in 32-dim blocks per tile: [tile][block][row in tile][32 bytes].
"""
import math
import time
from typing import Optional

import numpy as np

from . import _lib

U32 = 2.0 ** -24  # float32 unit roundoff
U64 = 2.0 ** -53


def _torch():
    import torch

    return torch


def choose_tile(dim: int) -> int:
    """Rows per tile. The reference picks 256 for D >= 256 else 64 (phase4a_suite.py:61-62); the
    B200 kernels run one thread per row and use 256 or 128."""
    return 256 if dim >= 256 else 128


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


class SharedClusterStorage:
    """Rows sorted by list id (stable), their original ids and the list row offsets.

    Same role and attribute names as the reference class (phase4a_suite.py:75-92). `xb_raw` may be
    a NumPy array or a torch tensor (on any device). With `host_rows=True` the sorted rows are kept
    in pinned host memory and read by the kernels through UVA (the zero-copy out-of-core mode).
    cluster_vec_off is int64 here (the reference used int32).
    """

    def __init__(self, xb_raw, list_ids, r_vec, nlist: int, device="cuda:0", host_rows: bool = False):
        torch = _torch()
        self.dev = torch.device(device)
        self.nlist = int(nlist)
        x = xb_raw if isinstance(xb_raw, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(xb_raw, np.float32))
        lid = list_ids if isinstance(list_ids, torch.Tensor) else torch.from_numpy(np.asarray(list_ids))
        self.N, self.D = int(x.shape[0]), int(x.shape[1])
        work = x.device if x.is_cuda else (self.dev if self.dev.type == "cuda" else torch.device("cpu"))
        lid_w = lid.to(work, torch.int64)
        if lid_w.numel() and (int(lid_w.min()) < 0 or int(lid_w.max()) >= self.nlist):
            raise ValueError("list id out of range")
        perm = torch.sort(lid_w, stable=True).indices
        counts = torch.bincount(lid_w, minlength=self.nlist)
        vec_off = torch.zeros(self.nlist + 1, dtype=torch.int64, device=work)
        vec_off[1:] = torch.cumsum(counts, 0)
        self.sort_perm = perm.to(torch.int32).cpu().numpy()
        self.counts = counts.cpu().numpy().astype(np.int32)
        self.host_rows = bool(host_rows)
        xs = x.to(work, torch.float32)[perm] if x.device != work else x[perm]
        if host_rows:
            self.xb_sorted = torch.empty((self.N, self.D), dtype=torch.float32, pin_memory=True)
            self.xb_sorted.copy_(xs)
        else:
            self.xb_sorted = xs.to(self.dev).contiguous()
        del xs
        self.orig_ids_sorted = perm.to(self.dev, torch.int32).contiguous()
        self.cluster_vec_off = vec_off.to(self.dev).contiguous()
        self.list_ids_sorted = torch.repeat_interleave(torch.arange(self.nlist, device=work), counts).to(self.dev)
        if r_vec is not None:
            rv = r_vec if isinstance(r_vec, torch.Tensor) else torch.from_numpy(np.asarray(r_vec, np.float32))
            self.r_vec_sorted = rv.to(work)[perm].cpu().numpy()
        else:
            self.r_vec_sorted = None


class TridentV4Index:
    """The searchable index (reference: phase4a_suite.py:95-342).

    Arguments mirror the reference: tile_size (rows per tile; 64 maps to 128 on B200),
    per_cluster_sq8 (0 = one global SQ8 interval, stored per list), use_pca (0 = identity rotation),
    var_block (variable block widths are an ablation of the reference and are not supported),
    max_batch / max_nprobe (workspace sizing). max_k bounds K (1..100).
    """

    def __init__(self, storage: SharedClusterStorage, centroids, mean64, R64, tile_size: int = 256,
                 per_cluster_sq8: int = 1, use_pca: int = 1, var_block: int = 0, max_batch: int = 1024,
                 max_nprobe: int = 512, device="cuda:0", max_k: int = 100, build_chunk: int = 1 << 16):
        torch = _torch()
        if var_block:
            raise NotImplementedError("var_block=1 (variable Stage-Y block widths) is an ablation of the "
                                      "reference and is not part of the B200 layout (32-dim blocks)")
        self.storage = storage
        self.dev = torch.device(device)
        self.N, self.D, self.nlist = storage.N, storage.D, storage.nlist
        self.tile_size = 128 if tile_size < 128 else (256 if tile_size > 128 else 128)
        self.per_cluster_sq8 = int(per_cluster_sq8)
        self.use_pca = int(use_pca)
        self.var_block = 0
        self.D_pad = ((self.D + 31) // 32) * 32
        self.num_blocks = self.D_pad // 32
        self.max_batch, self.max_nprobe, self.max_k = int(max_batch), int(max_nprobe), int(max_k)
        t0 = time.perf_counter()
        work = self.dev if self.dev.type == "cuda" else torch.device("cpu")

        D, D_pad, nlist, T = self.D, self.D_pad, self.nlist, self.tile_size
        if use_pca:
            mean64 = np.asarray(mean64, np.float64).reshape(D)
            R64 = np.asarray(R64, np.float64).reshape(D, D)
            orth = np.abs(R64.T @ R64 - np.eye(D)).max()
            if orth > 1e-9:
                raise ValueError(f"R64 is not orthogonal (max |R^T R - I| = {orth:.3e}); the lower bound "
                                 "needs a distance-preserving rotation")
        else:
            mean64 = np.zeros(D, np.float64)
            R64 = np.eye(D, dtype=np.float64)
        self.mean64, self.R64 = mean64, R64
        mu_w = torch.from_numpy(mean64).to(work)
        R_w = torch.from_numpy(R64).to(work)

        # ---- centroids
        cent = torch.from_numpy(np.ascontiguousarray(centroids, np.float32)).to(work)
        if cent.shape != (nlist, D):
            raise ValueError(f"centroids shape {tuple(cent.shape)} != ({nlist}, {D})")
        cn64 = (cent.double() ** 2).sum(1)
        self.centroids = cent.to(self.dev).contiguous()
        self.centroid_norm_sq = cn64.float().to(self.dev).contiguous()
        self.centroid_norm_max = float(np.nextafter(np.float32(math.sqrt(float(cn64.max())) * (1 + 1e-7)),
                                                    np.float32(np.inf)))

        # ---- rotation, per-list SQ8 intervals, codes and eps
        xs = storage.xb_sorted
        lids = storage.list_ids_sorted.to(work)
        vec_off = storage.cluster_vec_off.to(work)
        N = self.N

        def rotated(s, e):
            xc = xs[s:e].to(work, non_blocking=True).double()
            x64 = (xc - mu_w) @ R_w
            if D_pad > D:
                x64 = torch.nn.functional.pad(x64, (0, D_pad - D))
            return x64, torch.linalg.norm(xc - mu_w, dim=1)

        vmin = torch.full((nlist, D_pad), float("inf"), dtype=torch.float32, device=work)
        vmax = torch.full((nlist, D_pad), float("-inf"), dtype=torch.float32, device=work)
        rnorm = torch.zeros(nlist, dtype=torch.float64, device=work)
        for s in range(0, N, build_chunk):
            e = min(N, s + build_chunk)
            x64, nrm = rotated(s, e)
            x32 = x64.float()
            idx = lids[s:e].unsqueeze(1).expand(-1, D_pad)
            if per_cluster_sq8:
                vmin.scatter_reduce_(0, idx, x32, "amin", include_self=True)
                vmax.scatter_reduce_(0, idx, x32, "amax", include_self=True)
            else:
                vmin[0] = torch.minimum(vmin[0], x32.min(0).values)
                vmax[0] = torch.maximum(vmax[0], x32.max(0).values)
            rnorm.scatter_reduce_(0, lids[s:e], nrm, "amax", include_self=True)
        if not per_cluster_sq8:
            vmin[:] = vmin[0]
            vmax[:] = vmax[0]
        empty = torch.from_numpy(storage.counts == 0).to(work) if per_cluster_sq8 else torch.zeros(nlist, dtype=torch.bool, device=work)
        delta = torch.clamp((vmax - vmin) / 255.0, min=1e-12)
        vmin = torch.where(empty.unsqueeze(1), torch.zeros_like(vmin), vmin)
        delta = torch.where(empty.unsqueeze(1), torch.ones_like(delta), delta)
        if N == 0:
            vmin.zero_()
            delta.fill_(1.0)

        total_tiles_per = (torch.from_numpy(storage.counts.astype(np.int64)).to(work) + T - 1) // T
        tile_off = torch.zeros(nlist + 1, dtype=torch.int64, device=work)
        tile_off[1:] = torch.cumsum(total_tiles_per, 0)
        total_tiles = int(tile_off[-1])
        nb = self.num_blocks
        codes_tiles = torch.zeros((max(total_tiles, 1), nb, T, 32), dtype=torch.uint8, device=work)
        qerr = torch.zeros((nlist, D_pad), dtype=torch.float64, device=work)
        vmin64, delta64 = vmin.double(), delta.double()
        for s in range(0, N, build_chunk):
            e = min(N, s + build_chunk)
            x64, _ = rotated(s, e)
            x32 = x64.float()
            lc = lids[s:e]
            vm, dl = vmin[lc], delta[lc]
            code = torch.clamp(torch.round((x32 - vm) / dl), 0.0, 255.0)
            xhat = vmin64[lc] + code.double() * delta64[lc]
            err = (x64 - xhat).abs()
            qerr.scatter_reduce_(0, lc.unsqueeze(1).expand(-1, D_pad), err, "amax", include_self=True)
            rows = torch.arange(s, e, device=work)
            local = rows - vec_off[lc]
            tile = tile_off[lc] + local // T
            slot = local % T
            cu8 = code.to(torch.uint8).view(e - s, nb, 32)
            codes_tiles[tile, :, slot, :] = cu8
        self.codes = codes_tiles.reshape(-1).to(self.dev).contiguous()
        # eps: measured quantisation error, the float64 rotation error of the rows, and the
        # float32 roundings of u = fma(code, delta, vmin - q~) that do not scale with the query.
        rot_err = (D + 2) * 2.0 * U64 * rnorm
        eps64 = (qerr + rot_err.unsqueeze(1) + U32 * (2.0 * vmin64.abs() + 256.0 * delta64)) * (1.0 + 4.0 * U32)
        eps32 = eps64.float()
        eps32 = torch.where(eps32.double() < eps64, torch.nextafter(eps32, torch.full_like(eps32, float("inf"))), eps32)
        self.vmin_pad = vmin.to(self.dev).contiguous()
        self.delta_pad = delta.to(self.dev).contiguous()
        self.eps_pad = eps32.to(self.dev).contiguous()
        self.cluster_tile_off = tile_off.to(self.dev).contiguous()
        self.total_tiles = total_tiles
        self.pca_mean = torch.from_numpy(mean64.copy()).to(self.dev)
        self.pca_rot = torch.from_numpy(np.ascontiguousarray(R64)).to(self.dev)
        # relative slack of the prune test: float32 accumulation of the bound over D_pad terms and
        # of the exact distance (4 ceil(D/128) chained fma + 5 tree adds + the subtraction).
        self.lb_rel_slack = float((D_pad + 4 * math.ceil(D / 128) + 32) * U32 * 1.01)
        self.build_s = time.perf_counter() - t0
        self._reset_runtime()

    def _reset_runtime(self):
        """Per-index state of the search calls (descriptor, workspace, output buffers)."""
        self._desc = None
        self._ws = None
        self._ws_key = None
        self._out = {}
        self._stats_tmp = None

    @classmethod
    def from_arrays(cls, storage: SharedClusterStorage, arrays: dict, params: dict, device="cuda:0",
                    max_batch: int = 1024, max_nprobe: int = 512, max_k: int = 100):
        """An index from already-built arrays (trident_b200.artifacts.load_index), without the SQ8
        build. `arrays` holds device tensors: centroids, centroid_norm_sq, codes, vmin, delta, eps,
        tile_off, pca_mean, pca_rot; `params` the scalars tile_size, per_cluster_sq8, use_pca,
        centroid_norm_max, lb_rel_slack, total_tiles, plus mean64 and R64 (NumPy float64)."""
        torch = _torch()
        self = cls.__new__(cls)
        self.storage = storage
        self.dev = torch.device(device)
        self.N, self.D, self.nlist = storage.N, storage.D, storage.nlist
        self.tile_size = int(params["tile_size"])
        self.per_cluster_sq8 = int(params["per_cluster_sq8"])
        self.use_pca = int(params["use_pca"])
        self.var_block = 0
        self.D_pad = ((self.D + 31) // 32) * 32
        self.num_blocks = self.D_pad // 32
        self.max_batch, self.max_nprobe, self.max_k = int(max_batch), int(max_nprobe), int(max_k)
        self.mean64, self.R64 = params["mean64"], params["R64"]
        self.centroids = arrays["centroids"]
        self.centroid_norm_sq = arrays["centroid_norm_sq"]
        self.centroid_norm_max = float(params["centroid_norm_max"])
        self.codes = arrays["codes"]
        self.vmin_pad, self.delta_pad, self.eps_pad = arrays["vmin"], arrays["delta"], arrays["eps"]
        self.cluster_tile_off = arrays["tile_off"]
        self.total_tiles = int(params["total_tiles"])
        self.pca_mean, self.pca_rot = arrays["pca_mean"], arrays["pca_rot"]
        self.lb_rel_slack = float(params["lb_rel_slack"])
        self.build_s = 0.0
        self._reset_runtime()
        return self

    # ------------------------------------------------------------------------------------------
    # Stage Y on the tensor cores (the library's tcgen05 8-bit filter) needs each code slot's
    # sum_d (code_d delta_d)^2 (row_p). "auto" lets the library pick it where it is the faster
    # (D_pad <= 256, B * nprobe >= 32768), "always" for every cascade search, "off" never. The
    # results are identical in every setting.
    stage_y = "auto"

    def set_stage_y(self, mode: str) -> None:
        if mode not in ("auto", "always", "off"):
            raise ValueError(f"stage_y mode {mode!r}: expected 'auto', 'always' or 'off'")
        self.stage_y = mode
        self._desc = None

    def row_p(self):
        """[total_tiles * tile_size] float32 in code-slot order: sum_d (code_d delta_d)^2 of the slot's
        row in float64, rounded down (0 for empty slots). Computed once from the codes and deltas."""
        if getattr(self, "_row_p", None) is not None:
            return self._row_p
        torch = _torch()
        T, nb, D_pad = self.tile_size, self.num_blocks, self.D_pad
        tiles = max(self.total_tiles, 1)
        out = torch.zeros(tiles * T, dtype=torch.float32, device=self.codes.device)
        if self.total_tiles > 0:
            toff = self.cluster_tile_off.to(out.device).long()
            tile_list = torch.repeat_interleave(torch.arange(self.nlist, device=out.device), toff[1:] - toff[:-1])
            codes = self.codes.view(tiles, nb, T, 32)
            dl = self.delta_pad.to(out.device).double()
            step = max(1, (1 << 25) // (T * D_pad))  # about 256 MB of float64 per chunk
            for s in range(0, self.total_tiles, step):
                e = min(self.total_tiles, s + step)
                x = codes[s:e].permute(0, 2, 1, 3).reshape(e - s, T, D_pad).double() * dl[tile_list[s:e]].unsqueeze(1)
                p64 = (x * x).sum(-1) * (1.0 - 1e-12)
                p32 = p64.float()
                p32 = torch.where(p32.double() > p64, torch.nextafter(p32, torch.zeros_like(p32)), p32)
                out[s * T:e * T] = p32.reshape(-1)
                del x, p64, p32
        self._row_p = out
        return out

    def desc(self) -> _lib.TridentIndexDesc:
        if self._desc is None:
            s = self.storage
            d = _lib.TridentIndexDesc()
            d.N, d.D, d.D_pad, d.nlist = self.N, self.D, self.D_pad, self.nlist
            d.tile_size, d.num_blocks = self.tile_size, self.num_blocks
            d.flags = _lib.INDEX_TENSOR_STAGE_Y_ALWAYS if self.stage_y == "always" else 0
            d.xb_sorted = _ptr(s.xb_sorted)
            d.orig_ids_sorted = _ptr(s.orig_ids_sorted)
            d.list_row_off = _ptr(s.cluster_vec_off)
            d.list_tile_off = _ptr(self.cluster_tile_off)
            d.codes = _ptr(self.codes)
            d.vmin, d.delta, d.eps = _ptr(self.vmin_pad), _ptr(self.delta_pad), _ptr(self.eps_pad)
            d.centroids, d.centroid_norm_sq = _ptr(self.centroids), _ptr(self.centroid_norm_sq)
            d.pca_mean, d.pca_rot = _ptr(self.pca_mean), _ptr(self.pca_rot)
            d.centroid_norm_max = self.centroid_norm_max
            d.lb_rel_slack = self.lb_rel_slack
            d.row_p = _ptr(self.row_p()) if self.stage_y != "off" else None
            _lib.check(_lib.lib().trident_index_check(d))
            self._desc = d
        return self._desc

    def workspace_bytes(self, B: int, K: int, nprobe: int) -> int:
        import ctypes

        n = ctypes.c_size_t(0)
        _lib.check(_lib.lib().trident_workspace_size(self.desc(), int(B), int(K), int(nprobe), ctypes.byref(n)))
        return int(n.value)

    def _workspace(self, B: int, K: int, nprobe: int):
        torch = _torch()
        need = self.workspace_bytes(B, K, nprobe)
        if self._ws is None or self._ws.numel() < need:
            cap = max(need, self.workspace_bytes(max(B, self.max_batch), max(K, 10), max(nprobe, min(self.max_nprobe, self.nlist))))
            self._ws = torch.empty(cap, dtype=torch.uint8, device=self.dev)
        return self._ws

    def _outputs(self, B: int, K: int):
        torch = _torch()
        cap = max(B, self.max_batch)
        buf = self._out.get(K)
        if buf is None or buf[0].shape[0] < cap:
            buf = (torch.empty((cap, K), dtype=torch.float32, device=self.dev),
                   torch.empty((cap, K), dtype=torch.int64, device=self.dev))
            self._out[K] = buf
        return buf[0][:B], buf[1][:B]

    def status(self) -> int:
        """Device-side status word of this index's workspace after its last search (waits for the
        current stream): 0, or an OR of _lib.STATUS_LOCK_TIMEOUT / _lib.STATUS_MMA_TIMEOUT when a
        bounded wait gave up and the results were marked (NaN, -2)."""
        import ctypes

        torch = _torch()
        if self._ws is None:
            return 0
        st = ctypes.c_int32(0)
        _lib.check(_lib.lib().trident_workspace_status(_ptr(self._ws), torch.cuda.current_stream(self.dev).cuda_stream,
                                                       ctypes.byref(st)))
        return int(st.value)

    def route(self, B: int, nprobe: int, w0: float = 0.0) -> int:
        """The cost router: 10 (CM-FP32) if W = B * nprobe * (N / nlist) * D < w0 else 2 (cascade).
        w0 <= 0 uses the library's B200 calibration (TRIDENT_ROUTE_W0_B200); the reference's A100
        value was 9e8."""
        return int(_lib.lib().trident_route(self.desc(), int(B), int(nprobe), float(w0)))

    def stage_y_tensor(self, B: int, nprobe: int, k: int = 10, ub_seed: int = 0) -> bool:
        """Whether a cascade search of this shape runs Stage Y on the tensor cores (else CUDA cores)."""
        return bool(_lib.lib().trident_stage_y_tensor(self.desc(), int(B), int(k), int(nprobe), int(ub_seed)))

    def search(self, xq_gpu, nprobe: int, mode: int = 2, use_l1: int = 0, rerank_m: int = 0, tile_override: int = 0,
               warp_refine: int = 1, stats_buf=None, record_kernel_ms: bool = False, k: int = 10, ub_seed: int = 0,
               out=None, phase_ms: Optional[dict] = None):
        """Top-k search. Returns (topk_d [B, k] float32 squared distances, topk_i [B, k] int64 ids, kern_ms).

        mode: 2 = TRIDENT cascade (K2), 10 = CM-FP32 exact scan, -1 = cost router. The reference's
        ablation modes (0 CM-SQ8+RR, 1 K1, 11 Tribase), use_l1 and rerank_m are not implemented.
        ub_seed replaces the reference's TRIDENT_UB_SEED environment variable. phase_ms (a dict)
        receives CUDA-event times of each phase (coarse, pairs, seed, scan, merge); the
        call then synchronises the stream.
        """
        torch = _torch()
        if mode not in (-1, 2, 10):
            raise NotImplementedError(f"mode {mode} is a reference ablation/baseline mode; supported: 2, 10, -1")
        if use_l1 or rerank_m:
            raise NotImplementedError("use_l1 / rerank_m belong to the reference's ablation modes")
        if tile_override and (128 if tile_override < 128 else tile_override) != self.tile_size:
            raise ValueError(f"tile_override={tile_override} differs from the built tile size {self.tile_size}")
        if not warp_refine:
            raise NotImplementedError("warp_refine=0 (serial refine ablation) is not implemented")
        if xq_gpu.device != self.dev or xq_gpu.dtype != torch.float32 or not xq_gpu.is_contiguous():
            raise ValueError("queries must be a contiguous float32 tensor on the index device")
        if xq_gpu.dim() != 2 or xq_gpu.shape[1] != self.D:
            raise ValueError(f"queries must be [B, {self.D}]")
        B, K = int(xq_gpu.shape[0]), int(k)
        ws = self._workspace(B, K, nprobe)
        if out is not None:
            topk_d, topk_i = out
        else:
            topk_d, topk_i = self._outputs(B, K)
        stream = torch.cuda.current_stream(self.dev)
        sptr = 0
        if stats_buf is not None:
            if stats_buf.numel() >= _lib.STATS_LEN:
                sptr = _ptr(stats_buf)
            else:
                if self._stats_tmp is None:
                    self._stats_tmp = torch.zeros(_lib.STATS_LEN, dtype=torch.int64, device=self.dev)
                self._stats_tmp.zero_()
                sptr = _ptr(self._stats_tmp)
        ev0 = ev1 = None
        if record_kernel_ms:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        if phase_ms is not None:
            import ctypes

            buf = (ctypes.c_float * len(_lib.PHASES))()
            rc = _lib.lib().trident_search_profiled(self.desc(), _ptr(xq_gpu), B, K, int(nprobe), int(mode),
                                                    int(ub_seed), _ptr(ws), ws.numel(), _ptr(topk_d), _ptr(topk_i),
                                                    sptr, stream.cuda_stream, buf)
            _lib.check(rc)
            phase_ms.clear()
            phase_ms.update({n: float(buf[i]) for i, n in enumerate(_lib.PHASES)})
        else:
            rc = _lib.lib().trident_search(self.desc(), _ptr(xq_gpu), B, K, int(nprobe), int(mode), int(ub_seed),
                                           _ptr(ws), ws.numel(), _ptr(topk_d), _ptr(topk_i), sptr, stream.cuda_stream)
            _lib.check(rc)
        if stats_buf is not None and stats_buf.numel() < _lib.STATS_LEN:
            stats_buf += self._stats_tmp[: stats_buf.numel()]
        ms = 0.0
        if record_kernel_ms:
            ev1.record(stream)
            ev1.synchronize()
            ms = ev0.elapsed_time(ev1)
        return topk_d, topk_i, ms

    def search_stream(self, xq_host, nprobe: int, k: int = 10, batch: Optional[int] = None, mode: int = -1,
                      ub_seed: int = 0, timing: Optional[dict] = None):
        """Top-k of many host queries, streamed through the search in sub-batches of `batch` (default
        max_batch): a copy stream uploads sub-batch s + 1 into the second of two device buffers and
        downloads sub-batch s - 1's results into pinned host memory while sub-batch s is searched
        (events order the streams). mode = -1 routes each sub-batch on its own size. Returns pinned
        host tensors (distances [Q, k] float32, ids [Q, k] int64). timing (a dict) receives 'ms': CUDA
        events from before the first upload to after the last download.

        Caller-side streaming of the reference's drivers, which copy each batch and call search on it
        (benchmarks/phase4a_suite.py:280-342), moved into the index."""
        torch = _torch()
        x = xq_host if isinstance(xq_host, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(xq_host, np.float32))
        if x.is_cuda or x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != self.D:
            raise ValueError(f"xq_host must be a float32 host array [Q, {self.D}]")
        x = x.contiguous()
        if not x.is_pinned():
            x = x.pin_memory()
        Q, K = int(x.shape[0]), int(k)
        bs = int(batch or self.max_batch)
        out_d = torch.empty((Q, K), dtype=torch.float32, pin_memory=True)
        out_i = torch.empty((Q, K), dtype=torch.int64, pin_memory=True)
        if Q == 0:
            return out_d, out_i
        comp = torch.cuda.current_stream(self.dev)
        copy = getattr(self, "_copy_stream", None)
        if copy is None:
            copy = self._copy_stream = torch.cuda.Stream(device=self.dev)
        qbuf = [torch.empty((bs, self.D), dtype=torch.float32, device=self.dev) for _ in range(2)]
        rbuf = [(torch.empty((bs, K), dtype=torch.float32, device=self.dev),
                 torch.empty((bs, K), dtype=torch.int64, device=self.dev)) for _ in range(2)]
        ev = lambda t=False: torch.cuda.Event(enable_timing=t)
        h2d, done, d2h = [ev(), ev()], [ev(), ev()], [ev(), ev()]
        t0, t1 = ev(True), ev(True)
        nb = (Q + bs - 1) // bs
        t0.record(copy)
        with torch.cuda.stream(copy):
            b0 = min(bs, Q)
            qbuf[0][:b0].copy_(x[:b0], non_blocking=True)
            h2d[0].record(copy)
        for s in range(nb):
            cur, lo = s & 1, s * bs
            b = min(bs, Q - lo)
            comp.wait_event(h2d[cur])
            if s >= 2:
                comp.wait_event(d2h[cur])  # rbuf[cur] of sub-batch s - 2 is on its way to the host
            m = self.route(b, nprobe) if mode == -1 else mode
            self.search(qbuf[cur][:b], nprobe, mode=m, k=K, ub_seed=ub_seed,
                        out=(rbuf[cur][0][:b], rbuf[cur][1][:b]))
            done[cur].record(comp)
            with torch.cuda.stream(copy):
                if s + 1 < nb:  # the next sub-batch, once search s - 1 has released its buffer
                    if s >= 1:
                        copy.wait_event(done[cur ^ 1])
                    nlo = lo + bs
                    b2 = min(bs, Q - nlo)
                    qbuf[cur ^ 1][:b2].copy_(x[nlo:nlo + b2], non_blocking=True)
                    h2d[cur ^ 1].record(copy)
                copy.wait_event(done[cur])
                out_d[lo:lo + b].copy_(rbuf[cur][0][:b], non_blocking=True)
                out_i[lo:lo + b].copy_(rbuf[cur][1][:b], non_blocking=True)
                d2h[cur].record(copy)
        t1.record(copy)
        t1.synchronize()
        if timing is not None:
            timing["ms"] = t0.elapsed_time(t1)
        return out_d, out_i

    # ---- the search in three stages, for list sharding over GPUs (trident_b200.shard)
    def search_prep(self, xq_gpu, nprobe: int):
        """Stage 1 on this rank's own queries: (probe [B, nprobe] int32, qrot [B, D_pad] float32,
        qinfo [B, 4] float32)."""
        torch = _torch()
        B = int(xq_gpu.shape[0])
        ws = self._workspace(B, 1, nprobe)
        probe = torch.empty((B, nprobe), dtype=torch.int32, device=self.dev)
        qrot = torch.empty((B, self.D_pad), dtype=torch.float32, device=self.dev)
        qinfo = torch.empty((B, _lib.QINFO_LEN), dtype=torch.float32, device=self.dev)
        stream = torch.cuda.current_stream(self.dev)
        _lib.check(_lib.lib().trident_search_prep(self.desc(), _ptr(xq_gpu), B, int(nprobe), _ptr(ws), ws.numel(),
                                                  _ptr(probe), _ptr(qrot), _ptr(qinfo), stream.cuda_stream))
        return probe, qrot, qinfo

    def search_seed(self, xq_all, probe, qrot, qinfo, nprobe: int, k: int = 10, mode: int = 2, ub_seed: int = 0):
        """Stage 2 on the gathered batch: work items over this rank's lists and each query's k
        smallest seed values from this rank's rows. Returns (seed_d [B_all, k] float32, seed_i
        [B_all, k] int64), ascending and padded with (+inf, -1); merged over the ranks, column k-1
        is the threshold for search_finish. The workspace keeps the items for search_finish."""
        torch = _torch()
        B, K = int(xq_all.shape[0]), int(k)
        ws = self._workspace(B, K, nprobe)
        seed_d = torch.empty((B, K), dtype=torch.float32, device=self.dev)
        seed_i = torch.empty((B, K), dtype=torch.int64, device=self.dev)
        stream = torch.cuda.current_stream(self.dev)
        _lib.check(_lib.lib().trident_search_seed(self.desc(), _ptr(xq_all), B, K, int(nprobe), int(mode),
                                                  int(ub_seed), _ptr(probe), _ptr(qrot), _ptr(qinfo), _ptr(ws),
                                                  ws.numel(), _ptr(seed_d), _ptr(seed_i), stream.cuda_stream))
        return seed_d, seed_i

    def search_finish(self, xq_all, tau, nprobe: int, k: int = 10, mode: int = 2, ub_seed: int = 0, stats_buf=None):
        """Stage 3: the per-query top-k [B_all, k] of this rank's rows under the thresholds tau."""
        torch = _torch()
        B, K = int(xq_all.shape[0]), int(k)
        ws = self._workspace(B, K, nprobe)
        out_d = torch.empty((B, K), dtype=torch.float32, device=self.dev)
        out_i = torch.empty((B, K), dtype=torch.int64, device=self.dev)
        stream = torch.cuda.current_stream(self.dev)
        sptr = _ptr(stats_buf) if stats_buf is not None else 0
        _lib.check(_lib.lib().trident_search_finish(self.desc(), _ptr(xq_all), B, K, int(nprobe), int(mode),
                                                    int(ub_seed), _ptr(tau), _ptr(ws), ws.numel(), _ptr(out_d),
                                                    _ptr(out_i), sptr, stream.cuda_stream))
        return out_d, out_i

    def coarse(self, xq_gpu, nprobe: int):
        """Exact probe lists (ascending by (float64 distance, list id)), their float64 distances and
        the float32 rotated queries."""
        torch = _torch()
        B = int(xq_gpu.shape[0])
        ws = self._workspace(B, 1, nprobe)
        cids = torch.empty((B, nprobe), dtype=torch.int32, device=self.dev)
        d64 = torch.empty((B, nprobe), dtype=torch.float64, device=self.dev)
        qrot = torch.empty((B, self.D_pad), dtype=torch.float32, device=self.dev)
        stream = torch.cuda.current_stream(self.dev)
        rc = _lib.lib().trident_coarse(self.desc(), _ptr(xq_gpu), B, int(nprobe), _ptr(ws), ws.numel(), _ptr(cids),
                                       _ptr(d64), _ptr(qrot), 0, stream.cuda_stream)
        _lib.check(rc)
        return cids, d64, qrot

    # host copies of the index arrays (tests, oracle counters)
    def host_arrays(self) -> dict:
        s = self.storage
        return {
            "xb_sorted": s.xb_sorted.cpu().numpy(), "orig_ids_sorted": s.orig_ids_sorted.cpu().numpy(),
            "vec_off": s.cluster_vec_off.cpu().numpy(), "tile_off": self.cluster_tile_off.cpu().numpy(),
            "codes": self.codes.cpu().numpy(), "vmin": self.vmin_pad.cpu().numpy(),
            "delta": self.delta_pad.cpu().numpy(), "eps": self.eps_pad.cpu().numpy(),
            "centroids": self.centroids.cpu().numpy(),
        }


def merge_shards(d_in, i_in, out_d=None, out_i=None):
    """Global top-K from per-shard lists d_in/i_in [R, B, K] (device tensors)."""
    torch = _torch()
    R, B, K = (int(x) for x in d_in.shape)
    if out_d is None:
        out_d = torch.empty((B, K), dtype=torch.float32, device=d_in.device)
        out_i = torch.empty((B, K), dtype=torch.int64, device=d_in.device)
    stream = torch.cuda.current_stream(d_in.device)
    _lib.check(_lib.lib().trident_merge_shards(_ptr(d_in), _ptr(i_in), R, B, K, _ptr(out_d), _ptr(out_i),
                                               stream.cuda_stream))
    return out_d, out_i
