"""Calibration of the cost router's threshold W0 on the GPU at hand.

The router (trident_route) runs the CM-FP32 exact scan when the work W = B * nprobe * (N / nlist) * D
is below W0 and the cascade otherwise. The reference calibrates W0 by timing both modes over batch
sizes B in {1, 4, ..., 1024} at each dataset's nprobe and taking the smallest W at which the cascade
is at least as fast (benchmarks/phase4a_suite.py:1013-1035; its A100 value is 9e8). This module does
the same on seeded synthetic stand-ins of the benchmark configurations, timing each search with CUDA
events (median of `iters` calls after `warmup`).

    python -m trident_b200.calibrate [--configs c1,c2,c3] [--out calib.json]
"""
import argparse
import json
import statistics
import sys
import time

BATCHES = (1, 4, 8, 16, 32, 64, 128, 256, 512, 1024)


def time_search(idx, xq, nprobe: int, mode: int, k: int = 10, warmup: int = 5, iters: int = 20) -> float:
    """Median milliseconds of one search (CUDA events on the current stream)."""
    import torch

    for _ in range(warmup):
        idx.search(xq, nprobe, mode=mode, k=k)
    ms = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        idx.search(xq, nprobe, mode=mode, k=k)
        b.record()
        b.synchronize()
        ms.append(a.elapsed_time(b))
    return statistics.median(ms)


def calibrate(idx, xq_pool, nprobe: int, batches=BATCHES, k: int = 10, name: str = ""):
    """Rows {B, W, ms_cm, ms_cascade, cascade_faster} and the smallest W at which the cascade wins
    (None if it never does)."""
    rows = []
    avg_len = idx.N / float(idx.nlist)
    for B in batches:
        if B > xq_pool.shape[0]:
            break
        q = xq_pool[:B].contiguous()
        W = float(B) * nprobe * avg_len * idx.D
        ms_cm = time_search(idx, q, nprobe, 10, k)
        ms_k2 = time_search(idx, q, nprobe, 2, k)
        rows.append({"config": name, "B": B, "nprobe": nprobe, "W": W, "ms_cm_fp32": round(ms_cm, 4),
                     "ms_cascade": round(ms_k2, 4), "cascade_faster": bool(ms_k2 <= ms_cm)})
    wins = [r["W"] for r in rows if r["cascade_faster"]]
    return rows, (min(wins) if wins else None)


def _build(name: str, device):
    import torch

    from . import SharedClusterStorage, TridentV4Index, choose_tile, datasets as ds
    from .clustering import train_clustering

    cfg = ds.CONFIGS[name]
    xb = ds.generate_torch(cfg, cfg.N, ds.SEED_BASE, device=device)
    cent, lids, _, mu, R, _ = train_clustering(xb, cfg.nlist, sample_size=cfg.sample_size(), device=device)
    st = SharedClusterStorage(xb, torch.from_numpy(lids).to(device), None, cfg.nlist, device=device)
    del xb
    idx = TridentV4Index(st, cent, mu, R, tile_size=choose_tile(cfg.D), device=device, max_batch=max(BATCHES),
                         max_nprobe=cfg.nprobe)
    xq = torch.from_numpy(ds.generate_np(cfg, max(BATCHES), ds.SEED_QUERY)).to(device)
    return cfg, idx, xq


def main(argv=None):
    import torch

    p = argparse.ArgumentParser()
    p.add_argument("--configs", default="c1,c2,c3")
    p.add_argument("--out", default="")
    a = p.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    all_rows, per_cfg = [], {}
    for name in a.configs.split(","):
        t0 = time.perf_counter()
        cfg, idx, xq = _build(name, dev)
        rows, w = calibrate(idx, xq, cfg.nprobe, name=name)
        all_rows += rows
        per_cfg[name] = w
        print(f"[calibrate] {name}: crossover W = {w} ({time.perf_counter() - t0:.1f}s)", file=sys.stderr, flush=True)
        del idx
        torch.cuda.empty_cache()
    found = [w for w in per_cfg.values() if w is not None]
    res = {"w0": min(found) if found else None, "per_config": per_cfg, "rows": all_rows,
           "gpu": torch.cuda.get_device_name(dev), "rule": "smallest W at which the cascade is at least as fast "
                                                          "(phase4a_suite.py:1013-1035)"}
    line = json.dumps(res)
    print(line, flush=True)
    if a.out:
        with open(a.out, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
