"""The reference's standalone decode witness over four index kinds, restated
for this path (examples/check_native8b.py:13-66, cases at :80).

Eight units (the witness's eight KV groups), F = 3000 buckets, 4 query heads,
moments routing to 16 buckets, unbudgeted union, attention over the union
plus a dense tail.  Index kinds (check_native8b.py:16-23):
  empty   no memberships;
  ties    token t in bucket t % min(H, 64), bucket means and variances zero;
  few     token t in bucket (t + g) % 7;
  random  token t in buckets (t + 17g + o) % 3000, o in {0, 137, 811}.
Bucket moments are the raw (uncentred) mean and clamped variance of the
member keys, as the witness computes them.  The routed order is exact given
the device's scores and equals the oracle's order except between scores
within rounding of each other; the union is bit-exact against the oracle's
greedy on that order; attention is within the bf16 tolerance of the oracle.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2
F, U, G, K_ROUTE, D = 3000, 8, 4, 16, 128
CASES = [(32, 1, "ties"), (65, 7, "few"), (257, 31, "random"), (257, 129, "empty"), (1025, 3, "random"),
         (65536, 17, "random")]


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


def memberships(H, g, kind):
    if kind == "empty":
        return np.empty(0, np.int64), np.empty(0, np.int64)
    if kind == "ties":
        tid = np.arange(H, dtype=np.int64)
        return tid, tid % min(H, 64)
    if kind == "few":
        tid = np.arange(H, dtype=np.int64)
        return tid, (tid + g) % 7
    tid = np.repeat(np.arange(H, dtype=np.int64), 3)
    fid = np.stack([(np.arange(H) + g * 17 + o) % F for o in (0, 137, 811)], axis=-1).reshape(-1)
    return tid, fid


@pytest.mark.parametrize("H,tail,kind", CASES)
def test_index_kind_route_union_and_attention(pk, oracle, H, tail, kind):
    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(90 + H)

    def bf16_randn(*shape):   # bf16 values (round to nearest even), held in fp32
        return torch.randn(*shape, generator=gen).bfloat16().float().numpy()

    keys = bf16_randn(U, H + tail, D)
    vals = bf16_randn(U, H + tail, D)
    q = bf16_randn(U, G, D)

    lists, means, variances, oidx = [], [], [], []
    for g in range(U):
        tid, fid = memberships(H, g, kind)
        order = np.lexsort((tid, fid))
        tid_s, fid_s = tid[order], fid[order]
        bounds = np.searchsorted(fid_s, np.arange(F + 1))
        lists.append([tid_s[bounds[f]:bounds[f + 1]] for f in range(F)])
        n = torch.from_numpy(np.bincount(fid, minlength=F))
        sums = torch.zeros(F, D, dtype=torch.float32)
        squares = torch.zeros(F, D, dtype=torch.float32)
        if len(tid):
            raw = torch.from_numpy(keys[g, tid])
            sums.index_add_(0, torch.from_numpy(fid), raw)
            squares.index_add_(0, torch.from_numpy(fid), raw.square())
        mu = sums / n.clamp_min(1)[:, None].float()
        var = (squares / n.clamp_min(1)[:, None].float() - mu.square()).clamp_min(0)
        if kind == "ties":
            mu.zero_()
            var.zero_()
        means.append(mu.numpy())
        variances.append(var.numpy())
        oidx.append(oracle.index_from_lists(H, np.zeros(D, np.float32), lists[g], mean=means[-1],
                                            variance=variances[-1]))

    idx = pk.index.from_lists([[torch.from_numpy(x) for x in lu] for lu in lists], H, D, dev)
    idx.mean = torch.from_numpy(np.stack(means)).to(dev)
    idx.var = torch.from_numpy(np.stack(variances)).to(dev)
    sae = pk.SAEParams(torch.zeros(F, D, device=dev), torch.zeros(F, device=dev), key_mean=8, query_topk=K_ROUTE)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, router="moments", query_topk=K_ROUTE, exact_encode=True)
    Q = torch.from_numpy(q).to(dev).bfloat16().contiguous()
    op.route(Q)
    op.check()

    score = op.score.cpu().numpy()
    n_order = op.n_order.cpu().numpy()
    n_feat = op.n_features.cpu().numpy()
    count = op.count.cpu().numpy()
    union = []
    for g in range(U):
        oscore, oorder = oracle.bucket_scores(q[g], oidx[g], router="moments", query_topk=K_ROUTE)
        np.testing.assert_allclose(score[g], oscore, rtol=1e-5, atol=1e-7)
        got = op.order[g, :n_order[g]].cpu().numpy().astype(np.int64)
        # Exact given the device's own scores.
        assert np.array_equal(got, oracle.order_live(score[g], oidx[g].counts, K_ROUTE))
        # Equal to the oracle's order unless two scores sit within rounding.
        if not np.array_equal(got, oorder):
            assert len(got) == len(oorder)
            i = int(np.flatnonzero(got != oorder)[0])
            a, b = oscore[got[i]], oscore[oorder[i]]
            assert abs(a - b) <= 1e-6 * max(abs(a), abs(b)), (kind, g, i, a, b)
        ids, feats, raw = oracle.select_from_order(got, oidx[g], H)
        assert n_feat[g] == len(feats) and op.features[g, :n_feat[g]].cpu().tolist() == feats
        assert np.array_equal(op.ids[g, :count[g]].cpu().numpy().astype(np.int64), ids)
        if kind == "empty":
            assert n_order[g] == 0 and count[g] == 0
        union.append(ids)

    refs = np.stack([oracle.attend(q[g], keys[g], vals[g], union[g], H) for g in range(U)])
    Kd = torch.from_numpy(keys).to(dev).bfloat16()
    Vd = torch.from_numpy(vals).to(dev).bfloat16()
    for splits in (None, 12):
        out = op.attention(Q, Kd, Vd, length=H + tail, splits=splits)
        torch.cuda.synchronize()
        err = rel_l2(out.float().cpu().numpy(), refs)
        assert np.isfinite(out.float().cpu().numpy()).all() and err < TOL_BF16, (kind, H, splits, err)
