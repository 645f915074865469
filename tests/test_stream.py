"""TridentV4Index.search_stream: host queries streamed through the search in sub-batches (needs a B200).

The stream overlaps the upload of the next sub-batch and the download of the previous results with the
current search, and routes each sub-batch on its own size. Its results must equal one search over all
the queries (and the oracle) for every sub-batch size, including a last sub-batch smaller than the rest.
"""
import numpy as np
import pytest

from helpers import assert_same_topk, build_index, load_case, oracle_search

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [7, 16, 48, 1000])
@pytest.mark.parametrize("mode", [-1, 2, 10])
def test_stream_equals_one_search(batch, mode):
    import torch

    f = load_case("g3_norm_c3")
    idx = build_index(f, device="cuda:0")
    xq = f["xq"]
    nprobe, K = int(f["nprobe"]), int(f["K"])
    timing = {}
    sd, si = idx.search_stream(xq, nprobe, k=K, batch=batch, mode=mode, timing=timing)
    assert sd.is_pinned() and si.is_pinned() and timing["ms"] > 0.0
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], xq, nprobe, K)
    assert_same_topk(sd.numpy(), si.numpy(), od, oi)
    d1, i1, _ = idx.search(torch.from_numpy(xq).cuda(), nprobe, mode=2 if mode == -1 else mode, k=K)
    torch.cuda.synchronize()
    assert np.array_equal(si.numpy(), i1.cpu().numpy())


def test_stream_routes_each_sub_batch():
    """48 queries in sub-batches of 20: on this fixture the router sends the two full sub-batches to
    the cascade and the last 8 queries to the CM-FP32 scan; the merged results are exact either way."""
    f = load_case("g1_int_c1")
    idx = build_index(f, device="cuda:0")
    nprobe, K = int(f["nprobe"]), int(f["K"])
    assert f["xq"].shape[0] == 48
    assert idx.route(20, nprobe) == 2 and idx.route(8, nprobe) == 10
    sd, si = idx.search_stream(f["xq"], nprobe, k=K, batch=20, mode=-1)
    od, oi, _ = oracle_search(f["xb"], f["list_ids"], f["centroids"], f["xq"], nprobe, K)
    assert_same_topk(sd.numpy(), si.numpy(), od, oi)
