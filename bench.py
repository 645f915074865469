#!/usr/bin/env python3
"""Benchmark of the TRIDENT lossless IVF query path on B200: QPS at K=10.

Default workload: "c4", the configuration on which the metric's 1/2/4/8-GPU scaling is
quoted: N = 100,000,000 rows, D = 128, nlist = 65,536, nprobe = 256, K = 10, B = 10,000 queries in
total; SIFT-shaped integer rows (a 4096-component Gaussian mixture, sigma 25, rounded and clipped to
[0, 255]) generated on the GPU from fixed seeds (the real dataset is not used). It fits one B200
(about 106 GB at the build's peak). With --gpus N the IVF lists are sharded across N ranks (one
process per GPU) and the 10,000 queries are split between them (strong scaling):
  - each rank runs the coarse stage for its own queries; one NCCL all-gather shares the queries,
    rotated queries, side information and probe lists;
  - each rank seeds every query from its own lists; an all-gather of the seed lists and a device
    merge give each query's threshold;
  - each rank scans its own lists for every query;
  - an all-to-all of the per-rank top-K lists and a device merge.
--config c1 | c2 | c3 run the other configurations; their B is per rank (weak scaling).

One step = one search of the batch. `value` = all ranks' queries / step time with the queries already
in HBM (device time by CUDA events per step, L2 flushed between steps, max over ranks). `e2e` = the
same through the public API with the queries copied from pinned host memory and the results copied
back inside the timed region. Every run checks a sample of queries against the CPU oracle first.

`--impl reference` times the reference's own CPU exact IVF-Flat (omp_cpu_ivfflat_f32, built from
the reference sources into oracle/_ref) with float64 probe selection, on the box's host cores.
`--config c3 --sweep` times the cascade, CM-FP32 and the router over the c3 sweep.
`--impl reference-gpu --config c1|c2|c3` times the reference's own GPU kernels (built unchanged for
sm_100a) on the same B200 and data; c4's 65,536 lists do not fit its probe selection.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QPS at K=10 (lossless vs IVF-Flat) at 1/2/4/8 B200; % HBM roofline"
UNIT = "queries/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    p.add_argument("--ref-tile", type=int, default=0, help="reference-gpu: tile size 64 or 256 (default by D)")
    p.add_argument("--config", default="c4")
    p.add_argument("--batch", type=int, default=0, help="queries per step (default: the config's B)")
    p.add_argument("--nprobe", type=int, default=0)
    p.add_argument("--k", type=int, default=0)
    p.add_argument("--mode", type=int, default=-1, help="-1 router, 2 cascade, 10 CM-FP32")
    p.add_argument("--ub-seed", type=int, default=-1, help="0/1/2 (default: 0, or 1 with --ooc)")
    p.add_argument("--ooc", action="store_true",
                   help="zero-copy out-of-core: FP32 rows in pinned host memory, read over PCIe by Stage Z")
    p.add_argument("--check", type=int, default=64, help="queries verified against the CPU oracle")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU seconds of the CPU baseline")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-roofline", action="store_true")
    p.add_argument("--n", type=int, default=0, help="override N (rows) for quick runs")
    p.add_argument("--nlist", type=int, default=0, help="override nlist")
    p.add_argument("--n-comp", type=int, default=0, help="override the mixture's component count")
    p.add_argument("--sweep", action="store_true",
                   help="c3: time both modes and the router over B x nprobe x K, oracle-checking every cell")
    a = p.parse_args()
    if a.ub_seed < 0:  # out of core, seed from SQ8 upper bounds: the seed then reads no FP32 row
        a.ub_seed = 1 if a.ooc else 0
    return a


# ----------------------------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))

    def init(self):
        import torch

        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            # stdout carries exactly one JSON line: NCCL's version banner goes to stderr
            os.environ.setdefault("NCCL_DEBUG", "WARN")
            sys.stdout.flush()
            saved = os.dup(1)
            os.dup2(2, 1)
            try:
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=self.dev)
                dist.barrier()
            finally:
                sys.stdout.flush()
                os.dup2(saved, 1)
                os.close(saved)
        return self

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def bcast(self, t):
        if self.world > 1:
            import torch.distributed as dist

            dist.broadcast(t, 0)
        return t

    def close(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


# ----------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks and throttle reasons of this GPU, sampled in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index: int):
        import torch

        self.proc = None
        self.lines = []
        self.err = None
        try:
            uuid = str(torch.cuda.get_device_properties(dev_index).uuid)
            self.sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception as e:  # pragma: no cover
            self.sel = None
            self.err = f"uuid: {e}"

    def start(self):
        if not self.sel:
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.sel, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception as e:  # pragma: no cover
            self.err = str(e)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        time.sleep(0.05)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0, "note": self.err or "no samples"}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------------------------
STRONG = ("c4", "c5")  # configs whose query count is the job's total (split across ranks)
# CPU-baseline query prefix for the 10^4-query configs: the sample's probes decide how many rows must
# be copied to host memory (100 queries at C4 probe about 32% of the lists, 16 GB of rows)
CPU_SAMPLE_CAP = {"c4": 100, "c5": 100}


def workload_config(args):
    from trident_b200 import datasets as ds

    cfg = ds.CONFIGS[args.config]
    over = {}
    if args.batch:
        over["B"] = args.batch
    if args.nprobe:
        over["nprobe"] = args.nprobe
    if args.k:
        over["K"] = args.k
    if args.n:
        over["N"] = args.n
    if args.nlist:
        over["nlist"] = args.nlist
    if over:
        cfg = ds.scaled(cfg, **over)
    if args.n_comp:
        cfg = ds.Config(**{**cfg.__dict__, "n_comp": args.n_comp, "name": cfg.name.split("_")[0] + "_small"})
    return cfg


def make_clustering(args, d: Dist, cfg):
    """Rows generated on the GPU (every rank the same rows), clustered on rank 0 and broadcast.
    Returns (xb on the device, own queries, c_np, l_np, mu_np, R_np, strong)."""
    import numpy as np
    import torch

    from trident_b200 import datasets as ds
    from trident_b200.clustering import train_clustering

    strong = cfg.name.split("_")[0] in STRONG
    xb = ds.generate_torch(cfg, cfg.N, ds.SEED_BASE, device=d.dev)
    if strong:  # the config's B queries are the job's; rank r takes its slice
        if cfg.B % d.world:
            raise SystemExit(f"B={cfg.B} does not split over {d.world} ranks")
        per = cfg.B // d.world
        xq = ds.generate_np(cfg, cfg.B, ds.SEED_QUERY)[d.rank * per:(d.rank + 1) * per]
    else:  # each rank brings its own B queries; rank r holds rows [r B, (r + 1) B)
        xq = ds.generate_np(cfg, cfg.B * d.world, ds.SEED_QUERY)[d.rank * cfg.B:(d.rank + 1) * cfg.B]
    xq = np.ascontiguousarray(xq)
    cent = torch.empty((cfg.nlist, cfg.D), dtype=torch.float32, device=d.dev)
    lids = torch.empty(cfg.N, dtype=torch.int32, device=d.dev)
    mu = torch.empty(cfg.D, dtype=torch.float64, device=d.dev)
    R = torch.empty((cfg.D, cfg.D), dtype=torch.float64, device=d.dev)
    if d.rank == 0:
        t0 = time.perf_counter()
        c_np, l_np, _, mu_np, R_np, _ = train_clustering(xb, cfg.nlist, sample_size=cfg.sample_size(), device=d.dev)
        cent.copy_(torch.from_numpy(c_np))
        lids.copy_(torch.from_numpy(l_np))
        mu.copy_(torch.from_numpy(mu_np))
        R.copy_(torch.from_numpy(R_np))
        log(f"[rank 0] clustering of {cfg.N} rows into {cfg.nlist} lists: {time.perf_counter() - t0:.1f}s")
    for t in (cent, lids, mu, R):
        d.bcast(t)
    torch.cuda.synchronize()
    return xb, xq, lids, cent.cpu().numpy(), lids.cpu().numpy(), mu.cpu().numpy(), R.cpu().numpy(), strong


def make_workload(args, d: Dist):
    """Generate the config's rows/queries, cluster (rank 0, broadcast) and build this rank's shard.
    The full row array is dropped once the shard's storage is built."""
    import numpy as np
    import torch

    from trident_b200 import SharedClusterStorage, TridentV4Index, choose_tile
    from trident_b200.shard import list_work_estimate, partition_lists

    cfg = workload_config(args)
    t0 = time.perf_counter()
    xb, xq, lids, c_np, l_np, mu_np, R_np, strong = make_clustering(args, d, cfg)
    if d.world > 1:
        # lists weighed by expected scan work: rows x (1 + probes among 8192 base rows used as
        # stand-in queries), estimated on rank 0 and broadcast so every rank takes the same partition
        counts = np.bincount(l_np, minlength=cfg.nlist)
        work = torch.zeros(cfg.nlist, dtype=torch.int64, device=d.dev)
        if d.rank == 0:
            g = torch.Generator(device="cpu")
            g.manual_seed(ds_seed_balance())
            samp = xb[torch.randperm(cfg.N, generator=g)[:8192].to(d.dev)].contiguous()
            work.copy_(torch.from_numpy(list_work_estimate(samp, torch.from_numpy(c_np).to(d.dev), counts,
                                                           cfg.nprobe)))
            del samp
        d.bcast(work)
        owner = torch.from_numpy(partition_lists(work.cpu().numpy(), d.world)).to(d.dev)
        rows = torch.nonzero(owner[lids.long()] == d.rank).flatten()
        st = SharedClusterStorage(xb[rows], lids[rows], None, cfg.nlist, device=d.dev, host_rows=args.ooc)
        st.orig_ids_sorted = rows.to(torch.int32)[st.orig_ids_sorted.long()].contiguous()
        del rows, owner
    else:
        st = SharedClusterStorage(xb, lids, None, cfg.nlist, device=d.dev, host_rows=args.ooc)
    del xb, lids
    torch.cuda.empty_cache()
    idx = TridentV4Index(st, c_np, mu_np, R_np, tile_size=choose_tile(cfg.D), device=d.dev,
                         max_batch=max(1, xq.shape[0]) * d.world,
                         max_nprobe=cfg.nprobe, max_k=cfg.K)
    torch.cuda.synchronize()
    log(f"[rank {d.rank}] built {cfg.name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist} shard rows={st.N} "
        f"in {time.perf_counter() - t0:.1f}s (index build {idx.build_s:.1f}s, peak device memory "
        f"{torch.cuda.max_memory_allocated(d.dev) / 1e9:.1f} GB)")
    return cfg, xq, c_np, l_np, idx, strong


def ds_seed_balance() -> int:
    """Seed of the base-row sample that estimates list work for the partition."""
    from trident_b200 import datasets as ds

    return ds.SEED_PCA + 100


def host_storage(cfg, l_np, lists, device):
    """Host copies of the rows of `lists` in the index's order (list-major, original ids ascending
    within a list), regenerated on `device` chunk by chunk from the seeded generator, so that no
    process keeps the whole row array. Other lists are empty in the returned offsets, so a search
    whose probes all lie in `lists` sees exactly the full dataset's lists.
    Returns (xs [n, D] float32 torch CPU tensor, perm [n] int32 original ids, off [nlist + 1] int64)."""
    import numpy as np
    import torch

    from trident_b200 import datasets as ds

    need = np.zeros(cfg.nlist, bool)
    need[np.asarray(lists, np.int64)] = True
    counts = np.bincount(l_np, minlength=cfg.nlist)
    counts[~need] = 0
    off = np.zeros(cfg.nlist + 1, np.int64)
    off[1:] = np.cumsum(counts)
    sel = np.nonzero(need[l_np])[0]                       # original ids, ascending
    order = np.argsort(l_np[sel], kind="stable")          # list-major
    perm = sel[order].astype(np.int32)
    dest = np.empty(len(sel), np.int64)
    dest[order] = np.arange(len(sel))                     # destination row of sel[k]
    # the rows are put in order on the device (one scatter per generated chunk), then copied to
    # pageable host memory in one piece
    xs_dev = torch.empty((len(sel), cfg.D), dtype=torch.float32, device=device)
    sel_dev = torch.from_numpy(sel).to(device)
    dest_dev = torch.from_numpy(dest).to(device)
    for s, e, x in ds.iter_torch_chunks(cfg, cfg.N, ds.SEED_BASE, device=device):
        a, b = (int(v) for v in np.searchsorted(sel, [s, e]))
        if b > a:
            xs_dev.index_copy_(0, dest_dev[a:b], x[sel_dev[a:b] - s])
    del sel_dev, dest_dev
    xs = xs_dev.cpu()
    del xs_dev
    if str(device).startswith("cuda"):
        torch.cuda.empty_cache()
    return xs, perm, off


def cpu_reference_run(xq, cent, nprobe, K, xs, perm, off, n, threads):
    """One timed call of the reference CPU path on n queries: float64 probe selection (stands in for
    the faiss quantizer the reference times, phase8_ooc_100m_4080.py:570-574) + omp_cpu_ivfflat_f32."""
    import numpy as np
    import torch

    from oracle import oracle as O
    from oracle import ref_cpu

    ref = ref_cpu.load()
    q = np.ascontiguousarray(xq[:n])
    out_d = torch.empty((n, K), dtype=torch.float32)
    out_i = torch.empty((n, K), dtype=torch.int64)
    off32 = torch.from_numpy(off.astype(np.int32))
    oid = torch.from_numpy(perm)
    t0 = time.perf_counter()
    cids, _ = O.probe_select_f64(q, cent, nprobe, nthreads=threads)
    ref.omp_cpu_ivfflat_f32(torch.from_numpy(q), torch.from_numpy(cids.astype(np.int64)), off32, xs, oid, out_d, out_i)
    dt = time.perf_counter() - t0
    return dt, out_d.numpy(), out_i.numpy()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def data_desc(cfg) -> str:
    kind = {"int_mixture": f"SIFT-shaped integer rows in [0, 255] ({cfg.n_comp}-component mixture, sigma={cfg.sigma})",
            "decay": "GIST1M-shaped decay-spectrum rows",
            "norm_mixture": f"Deep-shaped L2-normalised rows ({cfg.n_comp}-component mixture, sigma={cfg.sigma})"}
    return f"synthetic (seeded {kind.get(cfg.kind, cfg.kind)}, generated on the GPU)"


def cpu_baseline(args, cfg, xq, c_np, xs, perm, off, n_max):
    """The reference's CPU path on the first n queries of rank 0 (n sized for about
    args.cpu_seconds of CPU work, at most n_max)."""
    threads = host_threads()
    os.environ["TRIDENT_REF_THREADS"] = str(threads)
    probe_n = min(n_max, 8)
    dt, _, _ = cpu_reference_run(xq, c_np, cfg.nprobe, cfg.K, xs, perm, off, probe_n, threads)
    per_q = dt / probe_n
    n = int(max(min(16, n_max), min(n_max, args.cpu_seconds / max(per_q, 1e-6))))
    dt, _, _ = cpu_reference_run(xq, c_np, cfg.nprobe, cfg.K, xs, perm, off, n, threads)
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"first {n} of rank 0's {xq.shape[0]} queries (one call: float64 probe selection + "
                      f"omp_cpu_ivfflat_f32 with {threads} threads), {dt:.2f}s"}


def roofline(idx, cfg, xq_dev, out_d, scan_ms, peaks, list_stride=0, tensor=False):
    """Algorithmic bytes of the scan launch under each query's final K-th distance, divided by its
    measured duration. bytes = B*D_pad*4 (rotated queries) + per distinct probed list (4 B per row id
    + 3*D_pad*4 B of vmin/delta/eps) + per row 32 B x the largest number of 32-dim blocks any query
    must scan + D*4 B per distinct surviving row + 8 B per candidate slot written.
    list_stride > 1 profiles only the lists c with c % list_stride == 0 (all queries probing them)
    and scales the per-row terms by the probed rows' total over the sampled lists' rows.
    tensor: the scan ran Stage Y on the tensor cores (filter_kernel), which reads every code block of
    a probed row where the algorithm needs only the blocks above; the bytes stay the algorithm's."""
    import numpy as np
    import torch

    from oracle import oracle as O

    cids, _, qrot = idx.coarse(xq_dev, cfg.nprobe)
    torch.cuda.synchronize()
    p1 = np.ascontiguousarray(cids.cpu().numpy())
    vec_off = idx.storage.cluster_vec_off.cpu().numpy()
    tile_off = idx.cluster_tile_off.cpu().numpy()
    L = np.diff(vec_off)
    lists = np.unique(p1[p1 >= 0])
    nb, T = idx.num_blocks, idx.tile_size
    tau = out_d[:, cfg.K - 1].astype(np.float32)
    t0 = time.perf_counter()
    if list_stride > 1:  # compact copies of the sampled lists' codes, other lists empty
        samp = lists[lists % list_stride == 0]
        keep = np.zeros(idx.nlist, bool)
        keep[samp] = True
        p1s = np.where(keep[np.maximum(p1, 0)] & (p1 >= 0), p1, -1).astype(np.int32)
        cnt = np.where(keep, L, 0)
        s_off = np.zeros(idx.nlist + 1, np.int64)
        s_off[1:] = np.cumsum(cnt)
        tiles = np.where(keep, np.diff(tile_off), 0)
        s_toff = np.zeros(idx.nlist + 1, np.int64)
        s_toff[1:] = np.cumsum(tiles)
        tile_ids = np.concatenate([np.arange(tile_off[c], tile_off[c + 1]) for c in samp]) if len(samp) else \
            np.zeros(0, np.int64)
        per_tile = nb * T * 32
        codes = idx.codes.view(-1, per_tile)[torch.from_numpy(tile_ids).to(idx.codes.device)].cpu().numpy()
        scale = float(L[lists].sum()) / max(1.0, float(L[samp].sum()))
        prof_lists, prof_off = samp, s_off
    else:
        p1s, s_off, s_toff, codes, scale = p1, vec_off, tile_off, idx.codes.cpu().numpy(), 1.0
        prof_lists, prof_off = lists, vec_off
    cand, blocks, surv, rows = O.stage_y_profile(
        p1s, s_off, s_toff, T, codes.reshape(-1), idx.vmin_pad.cpu().numpy(), idx.delta_pad.cpu().numpy(),
        idx.eps_pad.cpu().numpy(), qrot.cpu().numpy(), tau, want_rows=True)
    prof_s = time.perf_counter() - t0
    in_lists = np.zeros(int(prof_off[-1]), bool)
    for c in prof_lists:
        in_lists[prof_off[c]:prof_off[c + 1]] = True
    rb = rows[in_lists]
    surv_rows = int(round((rb > nb).sum() * scale))
    code_bytes = int(round(32 * np.minimum(rb, nb).astype(np.int64).sum() * scale))
    bytes_alg = (cfg.B * idx.D_pad * 4 + int(L[lists].sum()) * 4 + len(lists) * 3 * idx.D_pad * 4 + code_bytes
                 + surv_rows * idx.D * 4 + int((p1 >= 0).sum()) * cfg.K * 8)
    B_here = int(xq_dev.shape[0])
    bytes_alg += (B_here - cfg.B) * idx.D_pad * 4
    achieved = bytes_alg / (scan_ms * 1e-3) / 1e9
    peak = float(peaks.get("hbm_gbs", 6650.0))
    out = {
        "bound": "hbm",
        "kernel": ("filter_kernel (Stage Y on the tensor cores, Stage Z, every probe)" if tensor
                   else "scan_kernel (Stage Y/Z over every probe)"),
        "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
        "traffic": traffic_from_profile(cfg.name, "filter_kernel" if tensor else "scan_kernel"),
        "algorithmic_bytes": int(bytes_alg), "launch_ms": round(scan_ms, 4),
        "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback 6.65 TB/s",
        "pairs": int((p1 >= 0).sum()), "candidates": int(round(cand.sum() * scale)),
        "blocks": int(round(blocks.sum() * scale)), "survivor_pairs": int(round(surv.sum() * scale)),
        "survivor_rows": surv_rows, "profile_s": round(prof_s, 2),
    }
    if list_stride > 1:
        out["profile_sample"] = (f"lists c with c % {list_stride} == 0 ({len(prof_lists)} of {len(lists)} probed "
                                 f"lists), per-row terms scaled by {scale:.3f}")
    return out


def pcie_accounting(idx, cfg, xq_dev, nprobe, K, mode, ub_seed, ms_per_step, d=None, sharded=None):
    """Out-of-core PCIe traffic of one step. Every Stage-Z refine reads one FP32 row (D x 4 bytes) from
    pinned host memory through UVA. The seed then reads no row (ub_seed >= 1: SQ8 upper bounds), so
    the rows crossing PCIe are the scan's survivors (statistics slot TRIDENT_STAT_SURVIVORS). With
    ub_seed = 0 the seed's refined rows come on top. They are bounded here by B x seed rows. Under
    list sharding every rank runs one step with statistics (a collective step) and the counts are
    summed over the ranks; each rank's PCIe link carries its own rows."""
    import torch

    st = torch.zeros(8, dtype=torch.int64, device=xq_dev.device)
    if sharded is not None:
        sharded.search(xq_dev, nprobe, k=K, mode=mode, ub_seed=ub_seed, stats_buf=st)
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.all_reduce(st)
    else:
        idx.search(xq_dev, nprobe, mode=mode, k=K, ub_seed=ub_seed, stats_buf=st)
    torch.cuda.synchronize()
    surv = int(st[2].item())
    cand = int(st[0].item())
    row = cfg.D * 4
    seed_rows = 0 if ub_seed >= 1 or mode != 2 else cfg.B * max(64, 32 * ((K + 31) // 32))
    by = (surv + seed_rows) * row
    gbs = by / (ms_per_step * 1e-3) / 1e9
    # the box's PCIe peak: a 1 GiB copy from pinned host memory to the device (copy engine), best of 5
    src = torch.empty(1 << 28, dtype=torch.float32, pin_memory=True)
    dst = torch.empty(1 << 28, dtype=torch.float32, device=xq_dev.device)
    best = 0.0
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, src.numel() * 4 / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return {"rows_in": "pinned host memory (zero-copy, read through UVA)", "survivor_rows": surv,
            "candidates": cand, "survivor_fraction": round(surv / max(cand, 1), 8),
            "seed_rows_bound": seed_rows, "pcie_bytes_per_step": by, "pcie_gbs": round(gbs, 2),
            "pcie_peak_gbs": round(best, 2), "pcie_peak_source": "measured: 1 GiB pinned host -> device copy",
            "pcie_frac": round(gbs / best, 4) if best > 0 else None}


def traffic_from_profile(workload: str, kernel: str = "scan_kernel"):
    """DRAM bytes per launch of `kernel` at `workload` from the committed ncu summary of that kernel
    (a line `dram_bytes_per_launch[<workload>]: <bytes>`), or None when no capture of it is committed."""
    import glob

    key = f"dram_bytes_per_launch[{workload}]:"
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", f"{kernel}_*.md"))):
        for line in open(path):
            if line.strip().startswith(key):
                try:
                    return int(float(line.split(":", 1)[1].strip()))
                except ValueError:
                    return None
    return None


def check_against_oracle(cfg, xq, c_np, xs, perm, off, got_d, got_i, n):
    import numpy as np

    from oracle import oracle as O

    n = min(n, cfg.B)
    od, oi, _ = O.exact_search(xq[:n], c_np, cfg.nprobe, off, xs.numpy(), perm, cfg.K)
    ok_i = np.array_equal(got_i[:n], oi)
    ok_d = np.array_equal(got_d[:n].view(np.uint32), od.view(np.uint32))
    return {"queries": n, "ids_identical": bool(ok_i), "distances_bit_identical": bool(ok_d)}


# ----------------------------------------------------------------------------------------------
def run_ours(args, d: Dist):
    import numpy as np
    import torch

    from trident_b200 import _lib
    from trident_b200.shard import ShardedSearch

    from oracle import oracle as O

    cfg, xq, c_np, l_np, idx, strong = make_workload(args, d)
    B, K, nprobe = int(xq.shape[0]), cfg.K, cfg.nprobe  # B: this rank's queries per step
    # the scan of a step covers every rank's queries over this rank's lists
    mode = args.mode if args.mode != -1 else idx.route(B * d.world, nprobe)
    xq_pin = torch.from_numpy(xq).pin_memory()
    xq_dev = xq_pin.to(d.dev)
    sharded = ShardedSearch(idx) if d.world > 1 else None

    def step(xdev, phase=None, out=None):
        if sharded is not None:
            return sharded.search(xdev, nprobe, k=K, mode=mode, ub_seed=args.ub_seed, phase_ms=phase)
        dd, ii, _ = idx.search(xdev, nprobe, mode=mode, k=K, ub_seed=args.ub_seed, phase_ms=phase, out=out)
        return dd, ii

    # correctness first (rank 0 checks a sample of queries against the CPU oracle)
    d_out, i_out = step(xq_dev)
    torch.cuda.synchronize()
    got_d, got_i = d_out.cpu().numpy(), i_out.cpu().numpy()
    if d.world > 1:  # every rank's queries and results, for rank 0's roofline of its scan
        import torch.distributed as dist

        xq_all_dev = torch.empty((B * d.world, cfg.D), dtype=torch.float32, device=d.dev)
        dist.all_gather_into_tensor(xq_all_dev, xq_dev)
        d_all_dev = torch.empty((B * d.world, K), dtype=torch.float32, device=d.dev)
        dist.all_gather_into_tensor(d_all_dev, d_out.contiguous())
        d_all = d_all_dev.cpu().numpy()
    else:
        xq_all_dev, d_all = xq_dev, got_d
    xs = perm = off = None
    check = None
    n_cpu = 0 if args.no_cpu_baseline else min(B, CPU_SAMPLE_CAP.get(cfg.name.split("_")[0], B))
    if d.rank == 0:
        # host rows of every list that the checked queries and the CPU-baseline sample probe
        t0 = time.perf_counter()
        n_need = min(B, max(args.check, n_cpu))
        cids_need, _ = O.probe_select_f64(xq[:n_need], c_np, nprobe)
        xs, perm, off = host_storage(cfg, l_np, np.unique(cids_need[cids_need >= 0]), d.dev)
        log(f"[rank 0] host rows of the {n_need} sample queries' lists: {xs.shape[0]} rows in "
            f"{time.perf_counter() - t0:.1f}s")
        check = check_against_oracle(cfg, xq, c_np, xs, perm, off, got_d, got_i, args.check)
        log(f"[rank 0] oracle check: {check}")
        if not (check["ids_identical"] and check["distances_bit_identical"]):
            raise SystemExit("results differ from the CPU oracle; refusing to report a number")

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=d.dev)  # > 126 MB L2
    stream = torch.cuda.current_stream(d.dev)
    for _ in range(args.warmup):
        step(xq_dev)
    torch.cuda.synchronize()

    clocks = ClockSampler(d.local)
    clocks.start()
    time.sleep(0.3)
    # ---- device-timed region: K steps, queries resident in HBM, L2 flushed between steps
    phase_tot = {}
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches0 = int(_lib.lib().trident_launch_count())
    d.barrier()
    torch.cuda.synchronize()
    # TRIDENT_PROFILE_REGION=1: the timed steps alone are the profiler's region (ncu --profile-from-start off)
    region = bool(os.environ.get("TRIDENT_PROFILE_REGION"))
    if region:
        torch.cuda.profiler.start()
    for s in range(args.steps):
        flush.fill_(s & 0xFF)
        ph = {}
        evs[s][0].record(stream)
        step(xq_dev, phase=ph)
        evs[s][1].record(stream)
        for n, v in ph.items():
            phase_tot[n] = phase_tot.get(n, 0.0) + v
    torch.cuda.synchronize()
    if region:
        torch.cuda.profiler.stop()
    d.barrier()
    launches = int(_lib.lib().trident_launch_count()) - launches0
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = d.max(sum(step_ms))
    scan_per_rank = [phase_tot.get("scan", 0.0) / args.steps]
    if d.world > 1:  # every rank's scan time: the load balance of the list partition
        import torch.distributed as dist

        t = torch.tensor([scan_per_rank[0]], dtype=torch.float64, device=d.dev)
        allt = torch.empty(d.world, dtype=torch.float64, device=d.dev)
        dist.all_gather_into_tensor(allt, t)
        scan_per_rank = [round(float(v), 4) for v in allt.cpu().tolist()]
    # ---- end to end through the public API: pinned host queries in, host results out.
    #  * one GPU: TridentV4Index.search_stream over the steps' queries in sub-batches of B (a copy
    #    stream uploads the next sub-batch and downloads the previous results while the current one is
    #    searched), timed by its CUDA events from the first upload to the last download;
    #  * several GPUs: the staged search exchanges data between ranks inside every step, so each step
    #    runs its H2D copy, search and D2H copy in order on the compute stream.
    # There is no L2 flush inside; the index (codes + rows) is larger than L2.
    d.barrier()
    torch.cuda.synchronize()
    if d.world > 1:
        out_h = [(torch.empty((B, K), dtype=torch.float32, pin_memory=True),
                  torch.empty((B, K), dtype=torch.int64, pin_memory=True)) for _ in range(2)]
        xq_bufs = [torch.empty_like(xq_dev), torch.empty_like(xq_dev)]
        e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_start.record(stream)
        last = 0
        for s in range(args.steps):
            cur = s & 1
            xq_bufs[cur].copy_(xq_pin, non_blocking=True)
            dd, ii = step(xq_bufs[cur])
            out_h[cur][0].copy_(dd, non_blocking=True)
            out_h[cur][1].copy_(ii, non_blocking=True)
            last = cur
        e2e_end.record(stream)
        torch.cuda.synchronize()
        e2e_local = e2e_start.elapsed_time(e2e_end)
        out_d_h, out_i_h = out_h[last]
    else:
        xq_steps = xq_pin.repeat(args.steps, 1).pin_memory()
        tm = {}
        sd, si = idx.search_stream(xq_steps, nprobe, k=K, batch=B, mode=mode, ub_seed=args.ub_seed, timing=tm)
        e2e_local = tm["ms"]
        out_d_h, out_i_h = sd[-B:], si[-B:]
    d.barrier()
    clk = clocks.stop()
    e2e_ms = d.max(e2e_local)
    assert np.array_equal(out_i_h.numpy(), got_i)

    ooc_acc = None
    if args.ooc:  # every rank takes part (a collective step under list sharding)
        ooc_acc = pcie_accounting(idx, cfg, xq_dev, nprobe, K, mode, args.ub_seed, total_ms / args.steps, d=d,
                                  sharded=sharded)
        if d.world > 1:
            per = ooc_acc["pcie_gbs"] / d.world
            ooc_acc["pcie_gbs_per_rank"] = round(per, 2)
            ooc_acc["pcie_frac"] = round(per / ooc_acc["pcie_peak_gbs"], 4) if ooc_acc["pcie_peak_gbs"] else None
            ooc_acc["note"] = ("bytes and survivors summed over the ranks; each rank's PCIe link carries its own "
                               "rows, so pcie_frac is one rank's share over one link's measured peak")
    result = None
    if d.rank == 0:
        peaks = {}
        pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
        if os.path.exists(pp):
            peaks = json.load(open(pp))
        ms_per_step = total_ms / args.steps
        scan_ms = phase_tot.get("scan", 0.0) / args.steps
        roof = None
        if not args.no_roofline and mode == 2:
            # rank 0's scan covers every rank's queries over rank 0's lists
            stride = 64 if cfg.nlist > 8192 else 1
            roof = roofline(idx, cfg, xq_all_dev, d_all, scan_ms, peaks, list_stride=stride,
                            tensor=idx.stage_y_tensor(B * d.world, nprobe, K, args.ub_seed))
            if d.world > 1:
                roof["scope"] = f"rank 0's scan: all {B * d.world} queries over rank 0's lists"
        cpu = None
        if n_cpu:
            cpu = cpu_baseline(args, cfg, xq, c_np, xs, perm, off, n_cpu)
        ooc = ooc_acc
        result = {
            "metric": METRIC, "value": round(B * d.world / (ms_per_step * 1e-3), 1), "unit": UNIT,
            "n_gpus": d.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "f32",
            "data": data_desc(cfg),
            "config": {
                "workload": f"{cfg.name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist} nprobe={nprobe} K={K} " +
                            (f"B={B * d.world} in total" if strong else f"B={B} per GPU"),
                "global_batch": B * d.world,
                "mode": {2: "cascade", 10: "cm_fp32"}[mode] + (" (router)" if args.mode == -1 else ""),
                "ub_seed": args.ub_seed, "tile_size": idx.tile_size,
                "l2": f"a 512 MB L2 flush between timed steps (outside the step events); this GPU's shard "
                      f"holds {idx.codes.numel() / 1e9:.2f} GB SQ8 codes + "
                      f"{idx.storage.xb_sorted.numel() * 4 / 1e9:.2f} GB FP32 rows",
                "parallelism": f"list-sharded x{d.world}" if d.world > 1 else "single GPU",
                "phase_ms_per_step": {n: round(v / args.steps, 4) for n, v in phase_tot.items()},
                **({"scan_ms_per_rank": scan_per_rank,
                    "partition": "lists weighed by rows x (1 + probes of 8192 base rows)"} if d.world > 1 else {}),
                "step_ms_min_max": [round(min(step_ms), 4), round(max(step_ms), 4)],
            },
            "e2e": {"value": round(B * d.world / (e2e_ms / args.steps * 1e-3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": int(xq_pin.numel() * 4) * d.world,
                    "d2h_bytes_per_step": int(out_d_h.numel() * 4 + out_i_h.numel() * 8) * d.world,
                    "method": ("TridentV4Index.search_stream over the steps' queries in sub-batches of B: H2D "
                               "of the next sub-batch and D2H of the previous results on a copy stream beside the "
                               "search; its CUDA events from the first H2D to the last D2H; no L2 flush inside "
                               "(index larger than L2)") if d.world == 1 else
                              ("ShardedSearch.search per batch: H2D of this rank's queries, the staged search, D2H "
                               "of its merged results, in order on the compute stream; CUDA events around all "
                               "steps, max over ranks; no L2 flush inside")},
            "gpu_launches": launches, "clocks": clk, "lossless_check": check,
            "roofline": roof, "cpu_baseline": cpu,
            **({"ooc": ooc} if ooc is not None else {}),
        }
    d.barrier()  # rank 0's post-timing checks end before any rank leaves the process group
    return result


def run_sweep(args, d: Dist):
    """The config's sweep (c3: B in {1, 100, 10^4}, nprobe in {32, 128}, K in {1, 10, 50, 100}) on one
    GPU: per cell, the median step time of the cascade, the CM-FP32 scan and the router's choice
    (CUDA events, L2 flushed between steps), an oracle check of up to 16 queries, and for the
    cascade at B <= 100 the HBM roofline fraction of its scan phase."""
    import numpy as np
    import torch

    from oracle import oracle as O

    cfg, xq, c_np, l_np, idx, _ = make_workload(args, d)
    ex = cfg.extra or {}
    Bs, nps, Ks = ex.get("B", (cfg.B,)), ex.get("nprobe", (cfg.nprobe,)), ex.get("K", (cfg.K,))
    xq_dev = torch.from_numpy(xq).to(d.dev)
    n_chk = 16
    cids_need, _ = O.probe_select_f64(xq[:n_chk], c_np, max(nps))
    xs, perm, off = host_storage(cfg, l_np, np.unique(cids_need), d.dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=d.dev)
    peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}

    def timed(q, nprobe, K, mode, iters=10):
        for _ in range(3):
            idx.search(q, nprobe, mode=mode, k=K)
        ms, phases = [], {}
        for i in range(iters):
            flush.fill_(i & 0xFF)
            ph = {}
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            idx.search(q, nprobe, mode=mode, k=K, phase_ms=ph)
            b.record()
            b.synchronize()
            ms.append(a.elapsed_time(b))
            for k, v in ph.items():
                phases[k] = phases.get(k, 0.0) + v / iters
        return statistics.median(ms), phases

    cells = []
    for B in Bs:
        q = xq_dev[:B].contiguous()
        for nprobe in nps:
            for K in Ks:
                row = {"B": B, "nprobe": nprobe, "K": K}
                for mode, name in ((2, "cascade"), (10, "cm_fp32")):
                    ms, ph = timed(q, nprobe, K, mode)
                    row[f"qps_{name}"] = round(B / (ms * 1e-3), 1)
                    row[f"ms_{name}"] = round(ms, 4)
                    if mode == 2:
                        scan_ms = ph.get("scan", 0.0)
                    dd, ii, _ = idx.search(q, nprobe, mode=mode, k=K)
                    torch.cuda.synchronize()
                    m = min(B, n_chk)
                    od, oi, _ = O.exact_search(xq[:m], c_np, nprobe, off, xs.numpy(), perm, K)
                    row[f"check_{name}"] = bool(np.array_equal(ii[:m].cpu().numpy(), oi) and
                                                np.array_equal(dd[:m].cpu().numpy().view(np.uint32), od.view(np.uint32)))
                    if mode == 2 and B <= 100:
                        r = roofline(idx, ds_cfg_with(cfg, B=B, nprobe=nprobe, K=K), q, dd.cpu().numpy(), scan_ms, peaks,
                                     tensor=idx.stage_y_tensor(B, nprobe, K))
                        row["cascade_scan_roofline_frac"] = r["frac"]
                        row["cascade_scan_alg_bytes"] = r["algorithmic_bytes"]
                        row["cascade_scan_ms"] = round(scan_ms, 4)
                routed = idx.route(B, nprobe)
                row["router"] = {2: "cascade", 10: "cm_fp32"}[routed]
                row["router_picked_faster"] = bool((routed == 2) == (row["ms_cascade"] <= row["ms_cm_fp32"]))
                cells.append(row)
                log(f"[sweep] {row}")
    ok = all(c["check_cascade"] and c["check_cm_fp32"] for c in cells)
    return {"metric": METRIC, "unit": UNIT, "n_gpus": 1, "sweep_of": cfg.name, "data": data_desc(cfg),
            "config": {"workload": f"{cfg.name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist}"},
            "all_cells_match_oracle": ok, "cells": cells}


def ds_cfg_with(cfg, **kw):
    from trident_b200 import datasets as ds

    return ds.Config(**{**cfg.__dict__, **kw})


def run_reference(args, d: Dist):
    if d.rank != 0:
        return None
    import torch

    from oracle import ref_cpu

    try:
        ref_cpu.load()
    except Exception as e:
        return {"impl": "reference", "unavailable": f"reference CPU module not built: {e}"}
    import numpy as np

    from oracle import oracle as O

    cfg = workload_config(args)
    xb, xq, lids, c_np, l_np, _, _, strong = make_clustering(args, d, cfg)
    del xb, lids
    torch.cuda.empty_cache()
    n_max = min(xq.shape[0], CPU_SAMPLE_CAP.get(cfg.name.split("_")[0], xq.shape[0]))
    cids_need, _ = O.probe_select_f64(xq[:n_max], c_np, cfg.nprobe)
    xs, perm, off = host_storage(cfg, l_np, np.unique(cids_need[cids_need >= 0]), d.dev)
    threads = host_threads()
    os.environ["TRIDENT_REF_THREADS"] = str(threads)
    dt, _, _ = cpu_reference_run(xq, c_np, cfg.nprobe, cfg.K, xs, perm, off, min(n_max, 8), threads)
    budget_s = 150.0 / max(args.steps + args.warmup, 1)
    n = int(max(min(8, n_max), min(n_max, budget_s / max(dt / min(n_max, 8), 1e-6))))
    for _ in range(args.warmup):
        cpu_reference_run(xq, c_np, cfg.nprobe, cfg.K, xs, perm, off, n, threads)
    times = []
    for _ in range(args.steps):
        t, _, _ = cpu_reference_run(xq, c_np, cfg.nprobe, cfg.K, xs, perm, off, n, threads)
        times.append(t)
    tot = sum(times)
    qps = n * args.steps / tot
    return {
        "metric": METRIC, "value": round(qps, 2), "unit": UNIT, "n_gpus": getattr(d, "launched", d.world), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(tot / args.steps * 1e3, 2), "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32", "data": data_desc(cfg),
        "impl": "reference",
        "config": {"workload": f"{cfg.name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist} nprobe={cfg.nprobe} "
                               f"K={cfg.K} " + (f"B={cfg.B} in total" if strong else f"B={cfg.B} per GPU"),
                   "global_batch": cfg.B if strong else cfg.B * getattr(d, "launched", d.world),
                   "host": "rank 0's host cores only: the reference's CPU path does not use the GPUs",
                   "sample_queries_per_step": n},
        "cpu_baseline": {"value": round(qps, 2), "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"each step: first {n} queries, float64 probe selection + omp_cpu_ivfflat_f32"},
        "e2e": {"value": round(qps, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference_gpu(args, d: Dist):
    """The reference's own GPU search (src/trident_v4_kernels.cu, built unchanged for sm_100a into
    oracle/_ref/gpu) on this B200, over the same rows, lists and queries as this library's arm.
    `value` is its mode 2 (the lossless cascade); its mode 10 (exact cluster-major FP32) is reported
    beside it. The same timing rules as this library's arm: W warm-up steps, K device-timed steps
    with a 512 MB L2 flush between them. A sample of queries is checked against the oracle's exact
    IVF-Flat over the reference's own probe sets (float32 coarse distances)."""
    if d.rank != 0:
        return None
    import numpy as np
    import torch

    from oracle import oracle as O
    from oracle import ref_gpu
    from trident_b200 import SharedClusterStorage

    try:
        ref_gpu.load()
    except Exception as e:
        return {"impl": "reference-gpu", "unavailable": f"reference GPU module not built: {e}"}
    cfg = workload_config(args)
    if cfg.nlist > ref_gpu.MAX_NLIST:
        return {"impl": "reference-gpu",
                "unavailable": f"{cfg.name}: nlist {cfg.nlist} does not fit the reference's probe selection, which "
                               f"holds a query's whole coarse row in shared memory (at most {ref_gpu.MAX_NLIST} lists "
                               f"in 227 KB)"}
    if cfg.K != ref_gpu.REF_K:
        return {"impl": "reference-gpu", "unavailable": "the reference's GPU kernels hold K = 10 only"}
    xb, xq, lids, c_np, l_np, mu_np, R_np, strong = make_clustering(args, d, cfg)
    st = SharedClusterStorage(xb, lids, None, cfg.nlist, device=d.dev)
    del xb, lids
    torch.cuda.empty_cache()
    B, nprobe = int(xq.shape[0]), cfg.nprobe
    tile = args.ref_tile or (256 if cfg.D >= 256 else 64)
    t0 = time.perf_counter()
    ref = ref_gpu.RefGpuIndex(st.xb_sorted, st.orig_ids_sorted, st.cluster_vec_off.cpu().numpy(), c_np, mu_np,
                              R_np, tile_size=tile, max_batch=B, max_nprobe=nprobe)
    torch.cuda.synchronize()
    log(f"[rank 0] reference arrays (tile {tile}) in {time.perf_counter() - t0:.1f}s")
    xq_pin = torch.from_numpy(xq).pin_memory()
    xq_dev = xq_pin.to(d.dev)

    # oracle check of a sample under each mode, over the reference's own probe sets
    n = min(B, args.check)
    off = st.cluster_vec_off.cpu().numpy().astype(np.int64)
    xs_h, perm_h = st.xb_sorted.cpu().numpy(), st.orig_ids_sorted.cpu().numpy()
    checks = {}
    for mode in (2, 10):
        dd, ii, cids, _ = ref.search(xq_dev, nprobe, mode=mode)
        torch.cuda.synchronize()
        dd, ii, cids = dd.cpu().numpy()[:n], ii.cpu().numpy()[:n], cids.cpu().numpy()[:n]
        od, oi = O.ivf_search(xq[:n], cids, off, xs_h, perm_h, cfg.K)
        fin = np.isfinite(od)
        checks[mode] = {"queries": n, "ids_identical": bool(np.array_equal(ii, oi)),
                        "distances_bit_identical": bool(np.array_equal(dd[fin].view(np.uint32),
                                                                       od[fin].view(np.uint32)))}
    del xs_h, perm_h
    log(f"[rank 0] reference vs oracle over its own probe sets: {checks}")

    flush = torch.empty(512 << 20, dtype=torch.uint8, device=d.dev)
    stream = torch.cuda.current_stream(d.dev)
    timed = {}
    clocks = ClockSampler(d.local)
    clocks.start()
    time.sleep(0.3)
    for mode in (2, 10):
        for _ in range(args.warmup):
            ref.search(xq_dev, nprobe, mode=mode)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for s in range(args.steps):
            flush.fill_(s & 0xFF)
            evs[s][0].record(stream)
            ref.search(xq_dev, nprobe, mode=mode)
            evs[s][1].record(stream)
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
        timed[mode] = {"qps": round(B / (ms * 1e-3), 1), "ms_per_step": round(ms, 4)}
    # end to end, mode 2: H2D of the pinned queries, the search, D2H of the top-K, per step in order
    out_d = torch.empty((B, cfg.K), dtype=torch.float32, pin_memory=True)
    out_i = torch.empty((B, cfg.K), dtype=torch.int64, pin_memory=True)
    xq_buf = torch.empty_like(xq_dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xq_buf.copy_(xq_pin, non_blocking=True)
        dd, ii, _, _ = ref.search(xq_buf, nprobe, mode=2)
        out_d.copy_(dd, non_blocking=True)
        out_i.copy_(ii, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    return {
        "metric": METRIC, "value": timed[2]["qps"], "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": timed[2]["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32", "data": data_desc(cfg),
        "impl": "reference-gpu",
        "config": {"workload": f"{cfg.name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist} nprobe={nprobe} K={cfg.K} B={B}",
                   "global_batch": B, "tile_size": tile,
                   "kernels": "the reference's src/trident_v4_kernels.cu, unchanged, -O3 --use_fast_math, sm_100a",
                   "l2": "a 512 MB L2 flush between timed steps (outside the step events)",
                   "modes": {"2 (cascade)": timed[2], "10 (cm_fp32)": timed[10]}},
        "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": int(xq_pin.numel() * 4),
                "d2h_bytes_per_step": int(out_d.numel() * 4 + out_i.numel() * 8),
                "method": "mode 2; per step H2D of the pinned queries, the search, D2H of the top-K, in order on "
                          "one stream; CUDA events around all steps"},
        "clocks": clk,
        "lossless_check": {"vs": "the oracle's exact IVF-Flat over the reference's own probe sets",
                           "mode_2": checks[2], "mode_10": checks[10]},
    }


def main():
    args = parse_args()
    d = Dist()
    if args.impl in ("reference", "reference-gpu"):
        # the reference arms run on rank 0 alone; other ranks exit without work
        if d.rank != 0:
            return 0
        d.launched = d.world  # the job's GPU count, reported; rank 0 alone runs, without a process group
        d.world = 1
    d.init()
    try:
        if args.impl == "reference":
            res = run_reference(args, d)
        elif args.impl == "reference-gpu":
            res = run_reference_gpu(args, d)
        elif args.sweep:
            res = run_sweep(args, d)
        else:
            res = run_ours(args, d)
    finally:
        if args.impl not in ("reference", "reference-gpu"):
            d.close()
    if d.rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
