"""The reference's seeded decode witness, restated for this path
(kernels/cuda_sm90/validate.py:8-62, ``tail_check``).

Four units, one per KV group of the witness.  Unit g holds (17, 9, 1, 0)[g]
live buckets of F = 3000, bucket f listing tokens (0, f+1, H//2, H-1): the
buckets overlap on the first and last old tokens, one unit has a single
bucket and one has none, and the ids reach the bitmap's last (partial) word.
Every bucket mean and variance is zero, so every live bucket's moments score
ties and the route must take them by ascending feature id
(validate.py:31-37): the first min(16, count) buckets, whose unbudgeted union
is the sorted unique of their tokens.  Attention over that union plus the
dense tail is checked against the CPU oracle for the default, a clustered
and an over-8 split count (the witness checks 32, 64 and 128 splits).  The
witness's head_dim is 256; this path is compiled for 128, which is used
here.  Histories and tails follow the witness's cases (257, 1) and
(32768, 1024).
"""
import numpy as np
import pytest
import torch

from gen import bf16_round

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2
PATTERN = (17, 9, 1, 0)
F, G, K_ROUTE, D = 3000, 6, 16, 128


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    import prismkv_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return prismkv_b200


@pytest.mark.parametrize("H,tail", [(257, 1), (32768, 1024)])
def test_tied_moments_route_union_and_attention(pk, oracle, H, tail):
    dev = torch.device("cuda")
    U = len(PATTERN)
    rs = np.random.RandomState(20261109)
    keys = bf16_round(rs.standard_normal((U, H + tail, D)).astype(np.float32))
    vals = bf16_round(rs.standard_normal((U, H + tail, D)).astype(np.float32))
    q = bf16_round(rs.standard_normal((U, G, D)).astype(np.float32))
    lists = [[[0, f + 1, H // 2, H - 1] if f < count else [] for f in range(F)] for count in PATTERN]

    idx = pk.index.from_lists([[torch.tensor(x, dtype=torch.int64) for x in lu] for lu in lists], H, D, dev)
    idx.mean = torch.zeros(U, F, D, device=dev)
    idx.var = torch.zeros(U, F, D, device=dev)
    sae = pk.SAEParams(torch.zeros(F, D, device=dev), torch.zeros(F, device=dev), key_mean=8, query_topk=K_ROUTE)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, router="moments", query_topk=K_ROUTE, exact_encode=True)
    Q = torch.from_numpy(q).to(dev).bfloat16().contiguous()
    Kd = torch.from_numpy(keys).to(dev).bfloat16()
    Vd = torch.from_numpy(vals).to(dev).bfloat16()
    op.route(Q)
    op.check()

    n_order = op.n_order.cpu().numpy()
    n_feat = op.n_features.cpu().numpy()
    count = op.count.cpu().numpy()
    expected_ids = []
    for u, c in enumerate(PATTERN):
        n = min(K_ROUTE, c)
        assert n_order[u] == n and n_feat[u] == n
        assert op.order[u, :n].cpu().tolist() == list(range(n))
        assert op.features[u, :n].cpu().tolist() == list(range(n))
        want = np.unique(np.array([t for f in range(n) for t in (0, f + 1, H // 2, H - 1)], np.int64))
        assert np.array_equal(op.ids[u, :count[u]].cpu().numpy().astype(np.int64), want)
        # The oracle restatement of core.py takes the same buckets and tokens.
        oidx = oracle.index_from_lists(H, np.zeros(D, np.float32), lists[u], mean=np.zeros((F, D), np.float32),
                                       variance=np.zeros((F, D), np.float32))
        oids, meta = oracle.select_buckets(q[u], oidx, router="moments", query_topk=K_ROUTE)
        assert np.array_equal(oids, want) and list(meta["features"]) == list(range(n))
        expected_ids.append(want)

    refs = np.stack([oracle.attend(q[u], keys[u], vals[u], expected_ids[u], H) for u in range(U)])
    for splits in (None, 3, 12):
        out = op.attention(Q, Kd, Vd, length=H + tail, splits=splits)
        torch.cuda.synchronize()
        err = rel_l2(out.float().cpu().numpy(), refs)
        assert err < TOL_BF16, (splits, err)
