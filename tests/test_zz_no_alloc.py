"""trident_search_noalloc, the search entry point that allocates nothing, called through the C ABI.

Some callers of this library cannot allocate device memory: cudaMalloc is unavailable or not
allowed where they run, so they cannot provide the workspace that trident_search needs. For them,
trident_search_noalloc keeps its workspace in a fixed array inside the library. This file checks
three things through the C ABI:
  * two calls in a row return exactly what trident_search returns for the same queries (the bar of
    every parity test here: identical ids, bit-identical distances);
  * the calls do not depend on what the previous call left in the shared array;
  * a batch too large for the fixed array is rejected with a clear error.
The file is named to be collected last, so that a run stopping at the first failure has already run
every other test. It builds its own index and passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from helpers import build_index, load_case

pytestmark = pytest.mark.gpu


def _noalloc(idx, xq_dev, nprobe, K, mode, out=None):
    import torch

    from trident_b200 import _lib

    B = int(xq_dev.shape[0])
    if out is None:
        out = (torch.empty((B, K), dtype=torch.float32, device=xq_dev.device),
               torch.empty((B, K), dtype=torch.int64, device=xq_dev.device))
    out_d, out_i = out
    out_d.fill_(-7.0)
    out_i.fill_(-7)
    stream = torch.cuda.current_stream(xq_dev.device)
    rc = _lib.lib().trident_search_noalloc(ctypes.byref(idx.desc()), xq_dev.data_ptr(), B, K, nprobe, mode, 0,
                                           out_d.data_ptr(), out_i.data_ptr(), None, stream.cuda_stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    return out_d.cpu().numpy(), out_i.cpu().numpy()


@pytest.mark.parametrize("name", ["g1_int_c1", "g2_decay_c2", "g3_norm_c3"])
def test_noalloc_matches_search_on_two_calls_in_a_row(name):
    import torch

    f = load_case(name)
    idx = build_index(f, device="cuda:0")
    xq = torch.from_numpy(f["xq"]).cuda()
    nprobe, K = int(f["nprobe"]), int(f["K"])
    for mode in (2, 10):
        ref_d, ref_i, _ = idx.search(xq, nprobe, mode=mode, k=K)
        torch.cuda.synchronize()
        ref_d, ref_i = ref_d.cpu().numpy().copy(), ref_i.cpu().numpy().copy()
        for _ in range(2):
            d, i = _noalloc(idx, xq, nprobe, K, mode)
            assert np.array_equal(i, ref_i)
            assert np.array_equal(d.view(np.uint32), ref_d.view(np.uint32))
    # after a first call on this thread and device, further calls take no device memory: the free
    # memory of the device (cudaMemGetInfo) stays the same across them
    out = (torch.empty((xq.shape[0], K), dtype=torch.float32, device="cuda"),
           torch.empty((xq.shape[0], K), dtype=torch.int64, device="cuda"))
    _noalloc(idx, xq, nprobe, K, 2, out=out)
    free0 = torch.cuda.mem_get_info()[0]
    for mode in (2, 10, 2):
        _noalloc(idx, xq, nprobe, K, mode, out=out)
    assert torch.cuda.mem_get_info()[0] == free0
    # a different, smaller problem right after: leftovers of the previous call must not matter
    d, i = _noalloc(idx, xq[:5].contiguous(), 2, 3, 2)
    ref_d, ref_i, _ = idx.search(xq[:5].contiguous(), 2, mode=2, k=3)
    torch.cuda.synchronize()
    assert np.array_equal(i, ref_i.cpu().numpy())
    assert np.array_equal(d.view(np.uint32), ref_d.cpu().numpy().view(np.uint32))


def test_noalloc_rejects_a_batch_beyond_its_fixed_workspace():
    import torch

    from trident_b200 import _lib

    f = load_case("g2_decay_c2")
    idx = build_index(f, device="cuda:0")
    nprobe, K = int(f["nprobe"]), 100
    B = 1
    while idx.workspace_bytes(B, K, nprobe) <= _lib.noalloc_workspace_bytes():
        B *= 2
    xq = torch.zeros((1, idx.D), dtype=torch.float32, device="cuda")  # never read: the size check comes first
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    outi = torch.empty(1, dtype=torch.int64, device="cuda")
    rc = _lib.lib().trident_search_noalloc(ctypes.byref(idx.desc()), xq.data_ptr(), B, K, nprobe, 2, 0,
                                           out.data_ptr(), outi.data_ptr(), None, None)
    assert rc == _lib.TRIDENT_ERR_WORKSPACE
    assert "no-alloc workspace" in _lib.last_error()
