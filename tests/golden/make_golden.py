"""Generate the golden fixtures under tests/golden/ from the reference itself.

Runs only where the reference checkout is present (see oracle/ref_build.py); other machines use the
committed .npz files. For each case it:
  1. draws a small seeded dataset with trident_b200.datasets (NumPy PCG64) and clusters it;
  2. builds the reference's own index on the CPU by importing benchmarks/phase4a_suite.py
     (SharedClusterStorage + TridentV4Index, device="cpu") and records its per-list SQ8 arrays
     (vmin_pad, delta_pad) and codes (unpacked from sq8_packed to one row per sorted vector);
  3. selects probes with the oracle's float64 rule and runs the reference's own exact CPU IVF-Flat,
     omp_cpu_ivfflat_f32 (benchmarks/phase8_ooc_100m_4080.py:141-204, built by oracle/ref_build.py),
     recording its top-K ids and distances.
The fixture stores the clustering (centroids, list ids, mean64, R64) so that tests do not depend
on k-means reproducing bit for bit, plus checksums of the regenerated base rows and queries.

Usage: python tests/golden/make_golden.py
"""
import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from oracle import ref_build, ref_cpu  # noqa: E402
from trident_b200 import datasets as ds  # noqa: E402
from trident_b200.clustering import train_clustering  # noqa: E402

REF_ROOT = ref_build.REF_ROOT

# name -> (base config, overrides, tile size used for the reference build)
CASES = {
    "g1_int_c1": (ds.CONFIGS["c1"], dict(N=2000, nlist=16, B=48, nprobe=4, K=10), 64),
    "g2_decay_c2": (ds.CONFIGS["c2"], dict(N=2000, D=200, nlist=16, B=48, nprobe=4, K=10), 256),
    "g3_norm_c3": (ds.CONFIGS["c3"], dict(N=2000, nlist=32, B=48, nprobe=8, K=10), 64),
    "g4_ties": (ds.Config("ties", 2000, 16, 8, 0, 0, 0, "int_mixture", n_comp=4, sigma=0.6), dict(B=48, nprobe=3, K=10), 64),
}


def checksum(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def case_config(name):
    base, ov, tile = CASES[name]
    if name == "g4_ties":
        cfg = ds.Config("ties", 2000, 16, 8, ov["nprobe"], ov["K"], ov["B"], "int_mixture", n_comp=4, sigma=0.6)
    else:
        cfg = ds.scaled(base, **ov)
    return cfg, tile


def case_data(name):
    cfg, tile = case_config(name)
    xb = ds.generate_np(cfg, cfg.N, ds.SEED_BASE)
    xq = ds.generate_np(cfg, cfg.B, ds.SEED_QUERY)
    if name == "g4_ties":
        # values in {0..3}: many exact distance ties between different rows
        xb = np.clip(np.rint(xb / 85.0), 0, 3).astype(np.float32)
        xq = np.clip(np.rint(xq / 85.0), 0, 3).astype(np.float32)
    return cfg, tile, xb, xq


def import_reference_suite():
    # The reference module creates result/cache folders under $HOME at import time; point HOME at
    # a git-ignored folder inside this repository.
    home = os.path.join(HERE, ".refhome")
    os.makedirs(home, exist_ok=True)
    os.environ["HOME"] = home
    path = os.path.join(REF_ROOT, "benchmarks", "phase4a_suite.py")
    spec = importlib.util.spec_from_file_location("ref_phase4a_suite", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def unpack_codes(sq8_packed, tile_orig_ids, vec_off, counts, D_pad, tile):
    """Reference layout [tiles][D4][W][32] u32 -> codes [N, D_pad] u8 in sorted-row order."""
    W = tile // 32
    D4 = D_pad // 4
    packed = sq8_packed.reshape(-1, D4, W, 32).view(np.uint32)
    tiles = np.ascontiguousarray(packed.transpose(0, 2, 3, 1)).reshape(-1, tile, D4)  # [tiles][row][D4]
    bytes_ = tiles.view(np.uint8).reshape(-1, tile, D_pad)
    N = int(vec_off[-1])
    out = np.zeros((N, D_pad), np.uint8)
    tile_cnt = (counts + tile - 1) // tile
    t = 0
    for c in range(len(counts)):
        s = vec_off[c]
        for k in range(tile_cnt[c]):
            n = min(tile, counts[c] - k * tile)
            out[s + k * tile: s + k * tile + n] = bytes_[t, :n]
            t += 1
    return out


def make_case(name, suite, refmod):
    import torch

    cfg, tile, xb, xq = case_data(name)
    cent, lids, r_vec, mean64, R64, _ = train_clustering(xb, cfg.nlist, device="cpu")
    storage = suite.SharedClusterStorage(xb, lids.astype(np.int64), r_vec, cfg.nlist, device="cpu")
    idx = suite.TridentV4Index(storage, cent, mean64, R64, tile_size=tile, per_cluster_sq8=1, use_pca=1,
                               var_block=0, max_batch=8, max_nprobe=cfg.nprobe, device="cpu")
    D_pad = idx.D_pad
    vec_off = storage.cluster_vec_off.numpy().astype(np.int64)
    codes = unpack_codes(idx.sq8_packed.numpy(), idx.tile_orig_ids.numpy(), vec_off, storage.counts, D_pad, tile)
    probe, probe_d64 = O.probe_select_f64(xq, cent, cfg.nprobe)
    out_d = torch.empty((cfg.B, cfg.K), dtype=torch.float32)
    out_i = torch.empty((cfg.B, cfg.K), dtype=torch.int64)
    refmod.omp_cpu_ivfflat_f32(torch.from_numpy(xq), torch.from_numpy(probe.astype(np.int64)),
                               torch.from_numpy(vec_off.astype(np.int32)), storage.xb_sorted.contiguous(),
                               storage.orig_ids_sorted.contiguous(), out_d, out_i)
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        N=cfg.N, D=cfg.D, nlist=cfg.nlist, B=cfg.B, nprobe=cfg.nprobe, K=cfg.K, tile=tile,
        xb_sha=checksum(xb), xq_sha=checksum(xq),
        centroids=cent, list_ids=lids.astype(np.int32), mean64=mean64, R64=R64,
        ref_sort_perm=storage.sort_perm.astype(np.int32),
        ref_vmin=idx.vmin_pad.numpy(), ref_delta=idx.delta_pad.numpy(), ref_codes=codes,
        probe=probe, probe_d64=probe_d64,
        ref_topk_d=out_d.numpy(), ref_topk_i=out_i.numpy(),
    )
    print(f"{name}: N={cfg.N} D={cfg.D} nlist={cfg.nlist} B={cfg.B} nprobe={cfg.nprobe} K={cfg.K}")


def main():
    if not os.path.exists(REF_ROOT):
        print("reference not mounted; fixtures unchanged")
        return
    ref_build.build()
    refmod = ref_cpu.load()
    suite = import_reference_suite()
    for name in CASES:
        make_case(name, suite, refmod)


if __name__ == "__main__":
    main()
