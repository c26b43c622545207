"""The oracle's blocked build (orc_build_index_stream) equals its direct build.

build_index at the GPU configurations' sizes (n * F up to 2^31 activations)
cannot hold the [n, F] activation matrix, so the oracle evaluates it in token
blocks with a two-pass threshold search.  These cases check, on the CPU, that
the blocked form returns the same index as the direct restatement of
core.py:92-103 -- including the regimes where the global BatchTopK's
threshold is decided by ties (integer activations), where fewer activations
are positive than the budget (threshold zero), where every activation is
zero, and where n and F are not multiples of the block and vector widths.
The large fixtures (cfg2, cfg3u, cfg4c in tests/test_oracle_golden.py) pin
the blocked form to the reference itself.
"""
import numpy as np
import pytest

from gen import unit_case


def same(a, b):
    return (np.array_equal(a.counts, b.counts) and np.array_equal(a.ids, b.ids)
            and np.array_equal(a.mean.view(np.uint32), b.mean.view(np.uint32))
            and np.array_equal(a.variance.view(np.uint32), b.variance.view(np.uint32))
            and np.array_equal(a.center.view(np.uint32), b.center.view(np.uint32)))


@pytest.mark.parametrize("seed,n,F,key_mean", [(1, 6, 64, 8), (2, 7, 17, 3), (3, 100, 100, 8), (4, 257, 256, 8),
                                               (5, 1000, 512, 4), (6, 33, 2000, 8), (7, 129, 531, 1)])
def test_stream_equals_direct_on_clustered_keys(oracle, seed, n, F, key_mean):
    c = unit_case(seed, n, 128, 4, F, 4, bf16=True, key_mean=key_mean)
    sae = oracle.SAE(c["W"], c["b"], key_mean=key_mean, query_topk=4)
    a = oracle.build_index(c["keys"], sae, 1.0, stream=False)
    b = oracle.build_index(c["keys"], sae, 1.0, stream=True)
    assert same(a, b)


def one_hot_case(acts):
    """Encoder rows e_f make the centered keys' activations equal to `acts`
    (F <= d): keys = acts, center = 0, W = I[:F]."""
    n, F = acts.shape
    d = 128
    keys = np.zeros((n, d), np.float32)
    keys[:, :F] = acts
    W = np.eye(F, d, dtype=np.float32)
    return keys, W, np.zeros(F, np.float32)


@pytest.mark.parametrize("kind", ["int_ties", "few_positive", "zeros", "negative_bias", "one_value"])
def test_stream_equals_direct_on_tie_regimes(oracle, kind):
    rs = np.random.RandomState(42)
    n, F = 93, 96
    if kind == "int_ties":
        acts = rs.randint(0, 9, size=(n, F)).astype(np.float32)
    elif kind == "few_positive":
        acts = np.where(rs.rand(n, F) < 0.02, rs.rand(n, F) + 0.5, 0).astype(np.float32)
    elif kind == "zeros":
        acts = np.zeros((n, F), np.float32)
    elif kind == "negative_bias":
        acts = rs.standard_normal((n, F)).astype(np.float32)
    else:
        acts = np.full((n, F), 0.75, np.float32)
    keys, W, b = one_hot_case(acts)
    if kind == "negative_bias":
        b = np.full(F, -1.0, np.float32)
    sae = oracle.SAE(W, b, key_mean=8, query_topk=4)
    center = np.zeros(128, np.float32)
    a = oracle.build_index(keys, sae, 1.0, center=center, stream=False)
    s = oracle.build_index(keys, sae, 1.0, center=center, stream=True)
    assert same(a, s)
    if kind == "zeros":
        assert a.memberships == 0
    if kind == "one_value":
        # every activation ties at the threshold: the first n * 8 entries in
        # flat (token-major) order are the members
        flat = np.arange(n * 8)
        assert a.memberships == n * 8
        assert np.array_equal(a.counts, np.bincount(flat % F, minlength=F))
