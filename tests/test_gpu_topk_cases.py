"""The reference's positive global top-k witness, restated for the index
build (kernels/cuda_sm90/validate.py:64-74, ``top_check``: 93 rows, count
744 = 93 x 8, random / rounded / sparse / zero activations).

The build's activations are relu(W (k - center) + b); with zero center and
bias and one-hot encoder rows W_f = e_(f mod 128), key n's activation of
bucket f is key[n, f mod 128], so the keys set the activation pattern:
  random   keys ~ N(0, 1);
  rounded  integer keys in 0..8: every value repeats across the features
           that share f mod 128, so the cut falls inside long runs of ties,
           which go by ascending flat index (core.py:24);
  sparse   one key with 11 unit coordinates: 176 positive activations,
           fewer than the count, all kept;
  zeros    no positive activation: an empty index.
The device index must equal the oracle's build, bucket for bucket, with no
duplicate membership.  F is 2048 here (the witness's matrix has 3000
columns); d is the path's 128.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
N, D, F, KEY_MEAN = 93, 128, 2048, 8
CASES = ("random", "rounded", "sparse", "zeros")


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    import prismkv_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return prismkv_b200


def keys_for(name, rs):
    if name == "random":
        return rs.standard_normal((N, D)).astype(np.float32)
    if name == "rounded":
        return np.round(rs.random_sample((N, D)) * 8).astype(np.float32)
    keys = np.zeros((N, D), np.float32)
    if name == "sparse":
        keys[0, :11] = 1.0
    return keys


@pytest.mark.parametrize("name", CASES)
def test_positive_global_topk_case(pk, oracle, name):
    dev = torch.device("cuda")
    rs = np.random.RandomState(CASES.index(name) + 64)
    keys = keys_for(name, rs)
    W = np.zeros((F, D), np.float32)
    W[np.arange(F), np.arange(F) % D] = 1.0
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.zeros(F, device=dev), key_mean=KEY_MEAN, query_topk=16)
    idx = pk.build_index(torch.from_numpy(keys).to(dev), sae, 1.0, center=torch.zeros(D, device=dev))
    counts, ids = idx.dev.csr(0)
    osae = oracle.SAE(W, np.zeros(F, np.float32), key_mean=KEY_MEAN, query_topk=16)
    oidx = oracle.build_index(keys, osae, 1.0, center=np.zeros(D, np.float32))
    assert np.array_equal(counts, oidx.counts), name
    assert np.array_equal(ids, oidx.ids), name
    total = int(counts.sum())
    positives = int((np.maximum(keys[:, np.arange(F) % D], 0) > 0).sum())
    assert total == min(N * KEY_MEAN, positives), (name, total, positives)
    # No membership twice: each bucket's list is strictly increasing.
    off = np.concatenate([[0], np.cumsum(counts)])
    for f in range(F):
        assert np.all(np.diff(ids[off[f]:off[f + 1]]) > 0)
