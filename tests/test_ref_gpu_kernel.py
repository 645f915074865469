"""The reference's own GPU search run on the B200, pinned against the oracle and compared with this
library (test infrastructure: the reference's src/trident_v4_kernels.cu built unchanged for sm_100a
by oracle/ref_build.py, driven by oracle/ref_gpu.py over the same sorted rows this library searches).

The oracle restates the reference's FP32 summation order (trident_v4_kernels.cu:11-17, :318-330).
Here the reference's compiled kernels check that restatement on real-valued data, on the GPU:
  * the reference's mode 10 (exact cluster-major FP32 scan, :269-378) over the probe set it selects
    itself (float32 coarse distances, :68-162) equals the oracle's exact IVF-Flat over that same
    probe set: ids identical, distances bit-identical;
  * the same for its mode 2 (the SQ8 cascade with FP32 refinement, :530-960);
  * on every query whose reference probe set equals the float64 one this library uses, this
    library's result in modes 10 and 2 equals the reference's, ids and distances bit for bit.
The reference kernels hold K = 10 only (their shared top-K arrays have ten entries).
"""
import numpy as np
import pytest

from helpers import CASE_NAMES, assert_same_topk, build_config_index, build_index, load_case

pytestmark = pytest.mark.gpu


def _ref_gpu():
    from oracle import ref_gpu

    if not ref_gpu.available():
        pytest.skip("reference GPU module not built (oracle/ref_build.py needs the reference sources)")
    ref_gpu.load()
    return ref_gpu


def _check(idx, xq, nprobe, tile_size, min_same):
    """Runs the reference's modes 10 and 2 and this library's on xq; returns the share of queries
    whose reference probe set equals the float64 one."""
    import torch

    from oracle import oracle as O

    ref_gpu = _ref_gpu()
    st = idx.storage
    off = st.cluster_vec_off.cpu().numpy().astype(np.int64)
    cent = idx.centroids.cpu().numpy()
    ref = ref_gpu.RefGpuIndex(st.xb_sorted, st.orig_ids_sorted, off, cent, idx.mean64, idx.R64,
                              tile_size=tile_size, max_batch=xq.shape[0], max_nprobe=nprobe)
    xs = st.xb_sorted.cpu().numpy()
    perm = st.orig_ids_sorted.cpu().numpy()
    xq_dev = torch.from_numpy(xq).cuda()
    oc, _ = O.probe_select_f64(xq, cent, nprobe)
    share = None
    for mode in (10, 2):
        d, i, cids, _ = ref.search(xq_dev, nprobe, mode=mode)
        torch.cuda.synchronize()
        d, i, cids = d.cpu().numpy(), i.cpu().numpy(), cids.cpu().numpy()
        od, oi = O.ivf_search(xq, cids, off, xs, perm, 10)
        assert_same_topk(d, i, od, oi)
        same = (np.sort(cids, axis=1) == np.sort(oc, axis=1)).all(axis=1)
        share = float(same.mean())
        assert share >= min_same, f"only {share:.3f} of the reference's probe sets equal the float64 ones"
        md, mi, _ = idx.search(xq_dev, nprobe, mode=mode, k=10)
        torch.cuda.synchronize()
        assert_same_topk(md.cpu().numpy()[same], mi.cpu().numpy()[same], d[same], i[same])
    return share


@pytest.mark.parametrize("name", CASE_NAMES)
def test_reference_gpu_kernels_equal_the_oracle_on_the_fixtures(name):
    f = load_case(name)
    idx = build_index(f)
    _check(idx, f["xq"], int(f["nprobe"]), int(f["tile"]), min_same=0.9)


@pytest.mark.parametrize("cfg_name,over,tile", [
    # c2 shape: real-valued, decaying spectrum, D = 960
    ("c2", dict(N=200_000, nlist=1024, nprobe=64, B=1000), 256),
    # c3 shape: unit-norm real-valued rows, D = 96, 4096 lists
    ("c3", dict(N=500_000, nlist=4096, nprobe=32, B=1000), 64),
])
def test_reference_gpu_kernels_equal_the_oracle_at_config_shapes(cfg_name, over, tile):
    from trident_b200 import datasets as ds

    cfg = ds.scaled(ds.CONFIGS[cfg_name], K=10, **over)
    _, xq, _, _, idx = build_config_index(cfg, "rows")
    _check(idx, xq, cfg.nprobe, tile, min_same=0.5)
