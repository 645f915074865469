"""TEST INFRASTRUCTURE ONLY: run the reference's own GPU search on a B200.

ref_build.build_gpu() compiles the reference's src/trident_v4_kernels.cu unchanged (entry point
launch_trident_v4_search, :1171-1604). This module loads that build and feeds it the arrays that the
reference's Python index makes (benchmarks/phase4a_suite.py:110-280). The arrays are restated here on
the GPU from the same sorted rows that this library searches, so both read identical data:
  * W_coarse_only = -2 C^T and b_coarse_only = ||c||^2 (:135-137). W_combined / b_combined append the
    float32 PCA rotation R and -mean.R (:139-145);
  * per-list SQ8 (:147-172): vmin = min, delta = max((max - min) / 255, 1e-12), codes =
    clip(round((x - vmin) / delta), 0, 255), eps = 0.5001 * delta. The rows are rotated in float64 on
    the GPU, where the reference uses NumPy (:148-150); the float32 results agree to an ulp;
  * tiles of tile_size rows, codes packed [tile, D_pad/4, tile_size/32, 32] as u32 words of four
    dimensions, ids padded with -1 (:185-227);
  * uniform 32-dimension blocks, bounds in units of four dimensions (:246-255).
Only what the launch reads for modes 10 (exact cluster-major FP32) and 2 (the lossless cascade) is
built; the L1 band is off (use_l1 = 0, the suite's default), so tile_r_minmax stays zero.

The reference kernels accept only K = 10: their shared top-K arrays hold ten entries
(trident_v4_kernels.cu:293-294, :977-978, :581-582). Probe selection keeps a query's whole coarse
row in shared memory (:1249-1253). Rows are read as float4 (:318-324), so D must be a multiple of 4.
search() checks all of these before it launches anything.

Users: tests/test_ref_gpu_kernel.py (the reference's distances against the oracle, and against this
library) and bench.py --impl reference-gpu (the reference's kernels timed on the same B200).
"""
import importlib.machinery
import importlib.util
import os

import numpy as np

from . import ref_build

MAX_CANDS = 16384       # the reference's per-query candidate buffer (phase4a_suite.py:276)
REF_K = 10
MAX_NLIST = 32768       # (nlist + 64) * 4 bytes of shared memory must stay below 227 KB
_MOD = None


def available() -> bool:
    return os.path.exists(ref_build.gpu_module_path()) or os.path.exists(ref_build.REF_GPU_FILE)


def load():
    """The reference GPU extension, or FileNotFoundError if it was never built."""
    global _MOD
    if _MOD is not None:
        return _MOD
    import torch  # noqa: F401  (the module links against libtorch)

    path = ref_build.gpu_module_path()
    if not os.path.exists(path):
        ref_build.build_gpu()
        if not os.path.exists(path):
            raise FileNotFoundError(f"reference GPU module not built: {path}")
    name = ref_build.GPU_NAME
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _MOD = mod
    return mod


class RefGpuIndex:
    """The reference's device arrays and work buffers over already sorted rows.

    xb_sorted [N, D] float32 and orig_ids_sorted [N] int32 are CUDA tensors in list order; vec_off
    is the [nlist + 1] row offset of each list. mean64 / R64 are the float64 PCA (None: no PCA,
    as the reference with use_pca = 0). build_sq8=False skips the cascade arrays (mode 10 only).
    """

    def __init__(self, xb_sorted, orig_ids_sorted, vec_off, centroids, mean64=None, R64=None, tile_size=256,
                 max_batch=1024, max_nprobe=512, build_sq8=True):
        import torch

        dev = xb_sorted.device
        N, D = xb_sorted.shape
        nlist = int(centroids.shape[0])
        if D % 4 != 0:
            raise ValueError(f"the reference kernels read rows as float4; D = {D} is not a multiple of 4")
        if nlist > MAX_NLIST:
            raise ValueError(f"nlist {nlist} exceeds the reference's shared-memory coarse row ({MAX_NLIST})")
        if tile_size not in (64, 256):
            raise ValueError("the reference kernels are built for tile sizes 64 and 256")
        if N >= 2 ** 31:
            raise ValueError("the reference offsets are int32")
        self.dev, self.N, self.D, self.nlist = dev, N, D, nlist
        self.tile_size, self.W_tile = tile_size, tile_size // 32
        self.D_pad = ((D + 31) // 32) * 32
        self.D4 = self.D_pad // 4
        self.max_batch, self.max_nprobe = int(max_batch), int(max_nprobe)
        self.xb_sorted = xb_sorted.contiguous()
        self.orig_ids_sorted = orig_ids_sorted.to(torch.int32).contiguous()
        vec_off = np.asarray(vec_off, np.int64)
        self.vec_off_np = vec_off
        self.cluster_vec_off = torch.from_numpy(vec_off.astype(np.int32)).to(dev)
        f32 = dict(device=dev, dtype=torch.float32)

        C = torch.as_tensor(np.asarray(centroids, np.float32)).to(dev)
        c_norm_sq = (C ** 2).sum(dim=1)
        self.W_coarse_only = (-2.0 * C.t()).contiguous()
        self.b_coarse_only = c_norm_sq.unsqueeze(0).contiguous()
        use_pca = mean64 is not None
        mean64_g = torch.as_tensor(np.asarray(mean64, np.float64)).to(dev) if use_pca else \
            torch.zeros(D, device=dev, dtype=torch.float64)
        R64_g = torch.as_tensor(np.asarray(R64, np.float64)).to(dev) if use_pca else \
            torch.eye(D, device=dev, dtype=torch.float64)
        mean_f32, R_f32 = mean64_g.float(), R64_g.float()
        total_cols = nlist + self.D_pad
        self.W_combined = torch.zeros((D, total_cols), **f32)
        self.b_combined = torch.zeros((1, total_cols), **f32)
        self.W_combined[:, :nlist] = self.W_coarse_only
        self.W_combined[:, nlist:nlist + D] = R_f32
        self.b_combined[0, :nlist] = c_norm_sq
        self.b_combined[0, nlist:nlist + D] = -torch.matmul(mean_f32, R_f32)

        counts = np.diff(vec_off)
        tile_counts = (counts + tile_size - 1) // tile_size
        tile_off = np.zeros(nlist + 1, np.int64)
        tile_off[1:] = np.cumsum(tile_counts)
        self.total_tiles = int(tile_off[-1])
        self.cluster_tile_off = torch.from_numpy(tile_off.astype(np.int32)).to(dev)
        i32 = dict(device=dev, dtype=torch.int32)
        if build_sq8:
            self._build_sq8(mean64_g, R64_g, counts, tile_off)
        else:
            self.sq8_packed = torch.zeros(1, **i32)
            self.tile_orig_ids = torch.full((1,), -1, **i32)
            self.vmin_pad = torch.zeros((nlist, self.D_pad), **f32)
            self.delta_pad = torch.ones((nlist, self.D_pad), **f32)
            self.eps_pad = torch.zeros((nlist, self.D_pad), **f32)
        self.has_sq8 = bool(build_sq8)
        self.tile_r_minmax = torch.zeros((max(self.total_tiles, 1), 2), **f32)
        self.blk_bounds4 = torch.arange(0, self.D4 + 1, 8, **i32)

        B, P = self.max_batch, self.max_nprobe
        self.proj_buf = torch.zeros((B, total_cols), **f32)
        self.cdists_buf = torch.zeros((B, nlist), **f32)
        self.probe_cids_buf = torch.zeros((B, P), **i32)
        self.probe_dqcs_buf = torch.zeros((B, P), **f32)
        self.pair_bufs = [torch.zeros(B * P, **(i32 if j % 3 != 2 else f32)) for j in range(6)]
        self.topk_d = torch.zeros((B, REF_K), **f32)
        self.topk_i = torch.zeros((B, REF_K), device=dev, dtype=torch.int64)
        self.topm_d = torch.zeros((B, 100), **f32)
        self.topm_i = torch.zeros((B, 100), device=dev, dtype=torch.int64)
        self.tau_sq = torch.zeros(B, **f32)
        self.cand_d = torch.zeros((B, MAX_CANDS), **f32)
        self.cand_i = torch.zeros((B, MAX_CANDS), device=dev, dtype=torch.int64)
        self.cand_cnt = torch.zeros(B, **i32)

    def _build_sq8(self, mean64_g, R64_g, counts, tile_off):
        import torch

        dev, N, D, D_pad, T, nlist = self.dev, self.N, self.D, self.D_pad, self.tile_size, self.nlist
        xr = torch.zeros((N, D_pad), device=dev, dtype=torch.float32)
        for a in range(0, N, 1 << 17):  # bounded float64 temporaries
            b = min(N, a + (1 << 17))
            xr[a:b, :D] = ((self.xb_sorted[a:b].double() - mean64_g) @ R64_g).float()
        codes = torch.zeros((N, D_pad), device=dev, dtype=torch.uint8)
        vmin = torch.zeros((nlist, D_pad), device=dev, dtype=torch.float32)
        delta = torch.ones((nlist, D_pad), device=dev, dtype=torch.float32)
        off = self.vec_off_np
        for c in range(nlist):
            s, e = int(off[c]), int(off[c + 1])
            if s == e:
                continue
            c_vecs = xr[s:e]
            c_min = c_vecs.amin(0)
            c_delta = torch.clamp_min((c_vecs.amax(0) - c_min) / 255.0, 1e-12)
            vmin[c], delta[c] = c_min, c_delta
            codes[s:e] = torch.clamp(torch.round((c_vecs - c_min) / c_delta), 0, 255).to(torch.uint8)
        del xr
        self.vmin_pad, self.delta_pad = vmin, delta
        self.eps_pad = (delta * 0.5001).contiguous()

        total = max(self.total_tiles, 1)
        packed = torch.zeros((total, self.D4, self.W_tile, 32), device=dev, dtype=torch.int32)
        tile_ids = torch.full((total * T,), -1, device=dev, dtype=torch.int32)
        lid = torch.repeat_interleave(torch.arange(nlist, device=dev),
                                      torch.from_numpy(counts.astype(np.int64)).to(dev))
        start = torch.from_numpy(off[:-1].astype(np.int64)).to(dev)
        t0 = torch.from_numpy(tile_off[:-1].astype(np.int64)).to(dev)
        words = codes.view(torch.int32)  # [N, D_pad / 4], four dimensions per word, little-endian
        for a in range(0, N, 1 << 20):
            b = min(N, a + (1 << 20))
            r = torch.arange(a, b, device=dev)
            j = r - start[lid[a:b]]
            tile = t0[lid[a:b]] + j // T
            w, ln = (j % T) // 32, j % 32
            packed[tile, :, w, ln] = words[a:b]
            tile_ids[tile * T + j % T] = self.orig_ids_sorted[a:b]
        self.sq8_packed = packed
        self.tile_orig_ids = tile_ids.view(total, T)

    def search(self, xq, nprobe, mode=2, k=REF_K, record_events=False):
        """launch_trident_v4_search on xq [B, D] (CUDA float32). Returns (topk_d [B, 10] float32,
        topk_i [B, 10] int64, probe_cids [B, nprobe] int32, kernel ms or 0), all on the device."""
        import torch

        B = int(xq.shape[0])
        if k != REF_K:
            raise ValueError(f"the reference kernels support only K = {REF_K}")
        if mode not in (2, 10):
            raise ValueError("only modes 2 (cascade) and 10 (exact FP32 scan) are driven here")
        if mode == 2 and not self.has_sq8:
            raise ValueError("mode 2 needs the SQ8 arrays (build_sq8=True)")
        if not (1 <= B <= self.max_batch) or not (1 <= nprobe <= min(self.max_nprobe, self.nlist)):
            raise ValueError(f"B = {B} / nprobe = {nprobe} outside this index's buffers")
        if nprobe * REF_K > MAX_CANDS:
            raise ValueError("nprobe * K exceeds the reference's candidate buffer")
        if xq.dtype != torch.float32 or xq.device != self.dev or tuple(xq.shape[1:]) != (self.D,):
            raise ValueError("xq must be [B, D] float32 on the index's device")
        xq = xq.contiguous()
        p = self.pair_bufs
        ms = load().launch_trident_v4_search(
            int(mode), int(self.tile_size), 0, 1, 0, int(nprobe), xq,
            self.W_combined, self.b_combined, self.W_coarse_only, self.b_coarse_only,
            self.proj_buf, self.cdists_buf, self.probe_cids_buf, self.probe_dqcs_buf,
            p[0], p[1], p[2], p[3], p[4], p[5],
            self.sq8_packed, self.tile_orig_ids, self.tile_r_minmax, self.cluster_tile_off,
            self.cluster_vec_off, self.xb_sorted, self.orig_ids_sorted,
            self.vmin_pad, self.delta_pad, self.eps_pad, self.blk_bounds4,
            self.topk_d[:B], self.topk_i[:B], self.topm_d, self.topm_i, self.tau_sq,
            self.cand_d, self.cand_i, self.cand_cnt, bool(record_events), 1, None, None)
        cids = self.probe_cids_buf.view(-1)[:B * nprobe].view(B, nprobe)
        return self.topk_d[:B], self.topk_i[:B], cids, float(ms)
