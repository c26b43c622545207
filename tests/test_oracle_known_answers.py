"""The reference's closed-form expectations (tests/test_core.py of the
reference, lines cited per test) evaluated on the oracle."""
import numpy as np
import pytest


def test_global_budget_cardinality_and_zero(oracle):  # test_core.py:12-17
    a = np.array([[10., 9., 8., 7.], [1., .9, .8, .7]], np.float32)
    ids = oracle.positive_global_topk(a, 4)
    assert (ids // 4).tolist() == [0, 0, 0, 0]
    assert len(oracle.positive_global_topk(np.zeros_like(a), 4)) == 0
    assert oracle.positive_global_topk(np.ones((2, 4), np.float32), 3).tolist() == [0, 1, 2]


def test_moments_of_original_keys_and_empty_bucket(oracle):  # test_core.py:26-33
    k = np.array([[2., 4.], [4., 8.], [9., 0.]], np.float32)
    idx = oracle.summarize(k, [np.array([0, 1]), np.array([2]), np.array([], np.int64)])
    np.testing.assert_allclose(idx.mean[0], [3., 6.])
    np.testing.assert_allclose(idx.variance[0], [1., 4.])
    assert idx.counts.tolist() == [2, 1, 0]
    score, _ = oracle.bucket_scores(np.ones((1, 2), np.float32), idx)
    assert score[-1] == 0


def test_gqa_normalize_before_aggregation(oracle):  # test_core.py:35-42
    k = np.array([[10., 0.], [0., 2.], [-3., -1.]], np.float32)
    idx = oracle.summarize(k, [np.array([0]), np.array([1]), np.array([2])])
    q = np.array([[1., 0.], [0., 1.]], np.float32)
    score, _ = oracle.bucket_scores(q, idx, terms=("mean",), query_topk=3)
    logits = q @ k.T / np.sqrt(2)
    e = np.exp(logits - logits.max(-1, keepdims=True))
    wanted = (e / e.sum(-1, keepdims=True)).mean(0)
    np.testing.assert_allclose(score, wanted, rtol=1e-5)


def test_overlap_unique_budget_skips_overflow(oracle):  # test_core.py:44-53
    keys = np.zeros((10, 2), np.float32)
    idx = oracle.summarize(keys, [np.array([0, 1, 2, 3]), np.array([2, 3]), np.array([4])])
    ids, meta = oracle.select_buckets(np.ones((1, 2), np.float32), idx, unique_cap=.3, query_topk=3,
                                      terms=("count",))
    assert ids.tolist() == [2, 3, 4]
    assert meta["features"] == [1, 2]
    assert meta["raw"] == 3
    full_ids, meta = oracle.select_buckets(np.ones((1, 2), np.float32), idx, query_topk=2, terms=("count",))
    assert full_ids.tolist() == [0, 1, 2, 3]
    assert meta["raw"] == 6


def test_attention_with_dense_tail_and_duplicates(oracle):  # test_core.py:55-63
    rs = np.random.RandomState(0)
    k, v, q = (rs.standard_normal(s).astype(np.float32) for s in ((9, 4), (9, 4), (3, 4)))
    def ref(rows):
        lg = q @ k[rows].T / 2
        e = np.exp(lg - lg.max(-1, keepdims=True))
        return (e / e.sum(-1, keepdims=True)) @ v[rows]
    np.testing.assert_allclose(oracle.attend(q, k, v, np.arange(6), 6), ref(np.arange(9)), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(oracle.attend(q, k, v, np.array([1, 3]), 6), ref(np.array([1, 3, 6, 7, 8])),
                               rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        oracle.attend(q, k, v, np.array([1, 1]), 6)


def test_empty_index_and_zero_budget(oracle):  # test_core.py:65-72
    k = np.random.RandomState(1).standard_normal((5, 2)).astype(np.float32)
    idx = oracle.summarize(k, [np.array([], np.int64)])
    ids, _ = oracle.select_buckets(np.ones((1, 2), np.float32), idx)
    assert len(ids) == 0
    idx = oracle.summarize(k, [np.arange(5)])
    ids, _ = oracle.select_buckets(np.ones((1, 2), np.float32), idx, unique_cap=0)
    assert len(ids) == 0


def test_incremental_moments_preserve_old_memberships(oracle):  # test_core.py:74-86
    rs = np.random.RandomState(2)
    k = rs.standard_normal((17, 4)).astype(np.float32)
    new = (rs.standard_normal((7, 4)) + 4).astype(np.float32)
    W = (rs.uniform(-.5, .5, (12, 4))).astype(np.float32)
    sae = oracle.SAE(W, np.zeros(12, np.float32), key_mean=2, query_topk=3)
    index = oracle.build_index(k, sae, 1)
    before = [x.copy() for x in index.lists]
    merged = oracle.append_index(index, new, sae, 1)
    wanted = oracle.summarize(np.concatenate((k, new)), merged.lists, index.center)
    np.testing.assert_allclose(merged.mean, wanted.mean, atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(merged.variance, wanted.variance, atol=1e-5, rtol=1e-5)
    for old, new_ids in zip(before, merged.lists):
        assert np.array_equal(new_ids[:len(old)], old)
    assert merged.memberships - index.memberships == 7 * 2
    assert np.array_equal(merged.center, index.center)


def test_query_feature_shared_weighted_route(oracle):  # test_core.py:88-96
    sae = oracle.SAE(np.array([[3., 0.], [0., 2.], [-2., 0.], [0., -1.]], np.float32), np.zeros(4, np.float32),
                     key_mean=1, query_topk=1)
    rs = np.random.RandomState(3)
    idx = oracle.summarize(rs.standard_normal((4, 2)).astype(np.float32), [np.array([i]) for i in range(4)])
    score, order = oracle.bucket_scores(np.eye(2, dtype=np.float32), idx, router="q_activation", sae=sae,
                                        query_scale=1, query_topk=1)
    np.testing.assert_allclose(score, [.5, .5, 0., 0.])
    assert order.tolist() == [0, 1]


def test_tied_witness_routes_by_feature_id(oracle):  # kernels/cuda_sm90/validate.py:21-37
    """The seeded decode witness's expectation: with every bucket mean and
    variance zero, all live buckets tie and the route takes the first
    min(16, count) by feature id; the union is their sorted unique tokens."""
    F, d, H = 3000, 128, 257
    q = np.random.RandomState(0).standard_normal((6, d)).astype(np.float32)
    for count in (17, 9, 1, 0):
        lists = [[0, f + 1, H // 2, H - 1] if f < count else [] for f in range(F)]
        idx = oracle.index_from_lists(H, np.zeros(d, np.float32), lists, mean=np.zeros((F, d), np.float32),
                                      variance=np.zeros((F, d), np.float32))
        ids, meta = oracle.select_buckets(q, idx, router="moments", query_topk=16)
        n = min(16, count)
        assert meta["features"] == list(range(n))
        want = sorted({t for f in range(n) for t in (0, f + 1, H // 2, H - 1)})
        assert ids.tolist() == want


@pytest.mark.parametrize("kind", ["random", "rounded", "sparse", "zeros"])
def test_positive_topk_witness(oracle, kind):  # kernels/cuda_sm90/validate.py:64-74
    """The positive global top-k witness: the kept coordinates are the
    largest positive values (as many as the count allows), none twice."""
    rs = np.random.RandomState(5)
    a = rs.random_sample((93, 3000)).astype(np.float32)
    if kind == "rounded":
        a = np.round(a * 8).astype(np.float32)
    elif kind == "sparse":
        a = np.zeros_like(a)
        a.reshape(-1)[:11] = 1.0
    elif kind == "zeros":
        a = np.zeros_like(a)
    ids = oracle.positive_global_topk(a, 744)
    assert len(np.unique(ids)) == len(ids)
    flat = a.reshape(-1)
    target = np.sort(flat)[::-1][:744]
    np.testing.assert_array_equal(np.sort(flat[ids])[::-1], target[target > 0])
