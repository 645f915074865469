"""The bounded waits of the kernels give up cleanly, and the failure reaches the host (needs a B200).

Every wait inside the kernels has a limit: the scan's per-query insertion lock and the coarse GEMM's
tensor-core completion barrier. A wait that runs out must not hang or fault the GPU: the kernel
records why in the workspace's status word, every result it may have spoiled reads (NaN, -2), and
the next search with the default limits is correct again. The tests set a limit of 0 through the C
ABI (trident_set_wait_limits), so each such wait gives up at its first check; the tensor-core
drain before tensor memory is freed keeps its full limit, so no MMA is left in flight.
"""
import numpy as np
import pytest

from helpers import build_index, load_case, oracle_search

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def case():
    f = load_case("g3_norm_c3")
    f["index"] = build_index(f, device="cuda:0")
    return f


@pytest.fixture(autouse=True)
def default_limits():
    from trident_b200 import _lib

    _lib.set_wait_limits(-1, -1)
    yield
    _lib.set_wait_limits(-1, -1)


def _marked(d, i):
    return bool(np.isnan(d).all() and (i == -2).all())


def _run(idx, xq, nprobe, K, mode=2):
    import torch

    d, i, _ = idx.search(xq, nprobe, mode=mode, k=K)
    torch.cuda.synchronize()
    return d.cpu().numpy().copy(), i.cpu().numpy().copy()


def _check_oracle(f, d, i):
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"], int(f["nprobe"]), int(f["K"]))
    assert np.array_equal(i, oi) and np.array_equal(d.view(np.uint32), od.view(np.uint32))


def test_lock_wait_that_gives_up_marks_every_result(case):
    import torch

    from trident_b200 import _lib

    f, idx = case, case["index"]
    xq = torch.from_numpy(f["xq"]).cuda()
    _lib.set_wait_limits(0, -1)
    d, i = _run(idx, xq, int(f["nprobe"]), int(f["K"]), mode=2)
    assert _marked(d, i)
    assert idx.status() == _lib.STATUS_LOCK_TIMEOUT
    _lib.set_wait_limits(-1, -1)
    for mode in (2, 10):
        d, i = _run(idx, xq, int(f["nprobe"]), int(f["K"]), mode=mode)
        assert idx.status() == _lib.STATUS_OK
        _check_oracle(f, d, i)


def test_tensor_core_wait_that_gives_up_marks_probes_and_results(case):
    import torch

    from trident_b200 import _lib

    f, idx = case, case["index"]
    xq = torch.from_numpy(f["xq"]).cuda()
    nprobe = int(f["nprobe"])
    _lib.set_wait_limits(-1, 0)
    for mode in (2, 10):
        d, i = _run(idx, xq, nprobe, int(f["K"]), mode=mode)
        assert _marked(d, i)
        assert idx.status() == _lib.STATUS_MMA_TIMEOUT
    cids, d64, _ = idx.coarse(xq, nprobe)
    torch.cuda.synchronize()
    assert (cids.cpu().numpy() == -1).all() and np.isnan(d64.cpu().numpy()).all()
    assert idx.status() == _lib.STATUS_MMA_TIMEOUT
    _lib.set_wait_limits(-1, -1)
    cids, _, _ = idx.coarse(xq, nprobe)
    torch.cuda.synchronize()
    assert np.array_equal(cids.cpu().numpy(), f["probe"])
    assert idx.status() == _lib.STATUS_OK
    d, i = _run(idx, xq, nprobe, int(f["K"]))
    _check_oracle(f, d, i)


@pytest.mark.parametrize("where", ["prep", "finish"])
def test_staged_search_carries_a_timeout_to_every_rank(case, where):
    """The multi-GPU protocol emulated with R = 3 shard indexes on one GPU (as in test_gpu_search):
    a tensor-core timeout in one rank's coarse stage, or a lock timeout in one rank's scan, must mark
    every merged result (NaN, -2) and show in the status of every rank it reaches."""
    import torch

    from test_gpu_search import _shard_indexes
    from trident_b200 import _lib, merge_shards

    f = case
    R, nprobe, K = 3, int(f["nprobe"]), int(f["K"])
    shards = _shard_indexes(f, R)
    B = f["xq"].shape[0] // R
    xq_all = torch.from_numpy(np.ascontiguousarray(f["xq"][:R * B])).cuda()
    parts = []
    for r in range(R):
        _lib.set_wait_limits(-1, 0 if (where == "prep" and r == 0) else -1)
        parts.append(shards[r].search_prep(xq_all[r * B:(r + 1) * B].contiguous(), nprobe))
    _lib.set_wait_limits(-1, -1)
    probe, qrot, qinfo = (torch.cat([p[k] for p in parts]).contiguous() for k in range(3))
    seeds = [s.search_seed(xq_all, probe, qrot, qinfo, nprobe, k=K, mode=2) for s in shards]
    sd, _ = merge_shards(torch.stack([x[0] for x in seeds]).contiguous(), torch.stack([x[1] for x in seeds]).contiguous())
    tau = sd[:, K - 1].contiguous()
    outs = []
    for r in range(R):
        _lib.set_wait_limits(0 if (where == "finish" and r == 1) else -1, -1)
        outs.append(shards[r].search_finish(xq_all, tau, nprobe, k=K, mode=2))
    _lib.set_wait_limits(-1, -1)
    torch.cuda.synchronize()
    want = _lib.STATUS_MMA_TIMEOUT if where == "prep" else _lib.STATUS_LOCK_TIMEOUT
    statuses = [s.status() for s in shards]
    if where == "prep":
        assert statuses == [want] * R  # the status travelled with the gathered qinfo rows
    else:
        assert statuses == [0, want, 0]
    for r in range(R):
        d_in = torch.stack([o[0][r * B:(r + 1) * B] for o in outs]).contiguous()
        i_in = torch.stack([o[1][r * B:(r + 1) * B] for o in outs]).contiguous()
        gd, gi = merge_shards(d_in, i_in)
        assert _marked(gd.cpu().numpy(), gi.cpu().numpy())
