"""The reference's adversarial top-16 route cases, restated for the moments
router of this path (kernels/cuda_sm90/benchmark_hopper_route.py:62-75).

Each unit has one query head equal to the unit vector e0 and routes with the
mean term only, so bucket f's logit is mean[f, 0] / sqrt(d): the test sets
mean[f, 0] = s_f * sqrt(d) to give the scores of each case.  The cases:
  empty          no live bucket;
  fewer_than_16  13 live buckets;
  all_equal      every logit 0 (ties -> ascending feature id);
  near_tie       logits ~ N(0, 1e-6);
  masked_random  bucket sizes uniform in [0, 150), every third bucket empty,
                 logits ~ N(0, 2);
  large_range    as masked_random with logits ~ N(0, 100): most softmax
                 weights underflow to zero, and zero-score live buckets
                 follow in ascending feature id.
The routed order is exact given the device's scores; against the oracle's
order it may differ only between scores within the 1e-5 relative tolerance
the moments scores are compared at.  The unbudgeted union is bit-exact
against the oracle's greedy on the routed order.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
F, U, K_ROUTE, D, H = 3000, 4, 16, 128, 256
CASES = ("empty", "fewer_than_16", "all_equal", "near_tie", "masked_random", "large_range")


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    import prismkv_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return prismkv_b200


def case_inputs(name, rs):
    counts = np.ones((U, F), np.int64)
    logits = np.zeros((U, F), np.float32)
    if name == "empty":
        counts[:] = 0
    elif name == "fewer_than_16":
        counts[:, 13:] = 0
    elif name == "near_tie":
        logits = (rs.standard_normal((U, F)) * 1e-6).astype(np.float32)
    elif name in ("masked_random", "large_range"):
        counts = rs.randint(0, 150, size=(U, F)).astype(np.int64)
        counts[:, ::3] = 0
        logits = (rs.standard_normal((U, F)) * (100.0 if name == "large_range" else 2.0)).astype(np.float32)
    return counts, logits


@pytest.mark.parametrize("name", CASES)
def test_adversarial_route_case(pk, oracle, name):
    dev = torch.device("cuda")
    rs = np.random.RandomState(CASES.index(name) + 62)
    counts, logits = case_inputs(name, rs)
    lists = [[np.arange(c, dtype=np.int64) for c in counts[u]] for u in range(U)]
    mean = np.zeros((U, F, D), np.float32)
    mean[:, :, 0] = logits * np.float32(math.sqrt(D))
    var = np.zeros((U, F, D), np.float32)
    q = np.zeros((U, 1, D), np.float32)
    q[:, :, 0] = 1.0

    idx = pk.index.from_lists([[torch.from_numpy(x) for x in lu] for lu in lists], H, D, dev)
    idx.mean = torch.from_numpy(mean).to(dev)
    idx.var = torch.from_numpy(var).to(dev)
    sae = pk.SAEParams(torch.zeros(F, D, device=dev), torch.zeros(F, device=dev), key_mean=8, query_topk=K_ROUTE)
    op = pk.SparseDecode(idx, sae, heads_per_unit=1, router="moments", query_topk=K_ROUTE, terms=("mean",),
                         exact_encode=True)
    op.route(torch.from_numpy(q).to(dev).bfloat16().contiguous())
    op.check()

    score = op.score.cpu().numpy()
    n_order = op.n_order.cpu().numpy()
    count = op.count.cpu().numpy()
    for u in range(U):
        oi = oracle.index_from_lists(H, np.zeros(D, np.float32), lists[u], mean=mean[u], variance=var[u])
        oscore, oorder = oracle.bucket_scores(q[u], oi, router="moments", query_topk=K_ROUTE, terms=("mean",))
        np.testing.assert_allclose(score[u], oscore, rtol=1e-5, atol=1e-7)
        got = op.order[u, :n_order[u]].cpu().numpy().astype(np.int64)
        assert np.array_equal(got, oracle.order_live(score[u], counts[u], K_ROUTE)), (name, u)
        assert len(got) == len(oorder) == min(K_ROUTE, int((counts[u] > 0).sum()))
        if not np.array_equal(got, oorder):
            i = int(np.flatnonzero(got != oorder)[0])
            a, b = oscore[got[i]], oscore[oorder[i]]
            assert abs(a - b) <= 1e-5 * max(abs(a), abs(b)), (name, u, i, a, b)
        ids, feats, _ = oracle.select_from_order(got, oi, H)
        assert np.array_equal(op.ids[u, :count[u]].cpu().numpy().astype(np.int64), ids), (name, u)
        if name == "all_equal":
            assert got.tolist() == list(range(K_ROUTE))
        if name == "empty":
            assert n_order[u] == 0 and count[u] == 0
