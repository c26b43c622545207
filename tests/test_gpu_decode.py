"""GPU tests of the batched decode operator and the edge cases of the path,
checked against the CPU oracle on the same seeded inputs (integer outputs
exact; attention within 2e-2 relative L2 in bf16, 1e-3 in fp32)."""
import numpy as np
import pytest
import torch

from gen import bf16_round

pytestmark = pytest.mark.gpu
TOL_F32, TOL_BF16 = 1e-3, 2e-2


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


def clustered(rs, U, n, d, C, G):
    centers = rs.standard_normal((U, C, d)).astype(np.float32)
    cid = rs.randint(0, C, size=(U, n))
    uu = np.arange(U)[:, None]
    keys = centers[uu, cid] + np.float32(0.3) * rs.standard_normal((U, n, d))
    vals = rs.standard_normal((U, n, d))
    qc = rs.randint(0, C, size=(U, G))
    q = centers[uu, qc] + np.float32(0.3) * rs.standard_normal((U, G, d))
    return (bf16_round(keys.astype(np.float32)), bf16_round(vals.astype(np.float32)),
            bf16_round(q.astype(np.float32)))


@pytest.fixture(scope="module")
def batch(pk, oracle):
    rs = np.random.RandomState(7)
    U, N, tail, d, C, F, G, k = 8, 4096, 16, 128, 64, 512, 4, 16
    keys, vals, q = clustered(rs, U, N + tail, d, C, G)
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    b = np.zeros(F, np.float32)
    dev = torch.device("cuda")
    K = torch.from_numpy(keys).to(dev).to(torch.bfloat16)
    V = torch.from_numpy(vals).to(dev).to(torch.bfloat16)
    Q = torch.from_numpy(q).to(dev).to(torch.bfloat16).contiguous()
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.from_numpy(b).to(dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=True)
    osae = oracle.SAE(W, b, key_mean=8, query_topk=k)
    oidx = [oracle.build_index(keys[u, :N], osae, 1.0) for u in range(U)]
    return dict(U=U, N=N, tail=tail, d=d, F=F, G=G, k=k, keys=keys, vals=vals, q=q, K=K, V=V, Q=Q, sae=sae,
                idx=idx, osae=osae, oidx=oidx)


@pytest.mark.parametrize("budget", [None, 256, 1024])
def test_batched_decode_matches_oracle(pk, oracle, batch, budget):
    B = batch
    cap = None if budget is None else budget / B["N"]
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], query_scale=1.0, unique_cap=cap)
    out = op(B["Q"], B["K"], B["V"])
    torch.cuda.synchronize()
    op.check()
    for u in range(B["U"]):
        counts, ids = B["idx"].csr(u)
        assert np.array_equal(counts, B["oidx"][u].counts)
        assert np.array_equal(ids, B["oidx"][u].ids)
        oids, meta = oracle.select_buckets(B["q"][u], B["oidx"][u], unique_cap=cap, router="q_activation",
                                           sae=B["osae"], query_scale=1.0, query_topk=B["k"])
        c = int(op.count[u])
        assert np.array_equal(op.ids[u, :c].cpu().numpy().astype(np.int64), oids)
        assert op.features[u, :int(op.n_features[u])].cpu().tolist() == meta["features"]
        assert int(op.raw[u]) == meta["raw"]
        ref = oracle.attend(B["q"][u], B["keys"][u], B["vals"][u], oids, B["N"])
        assert rel_l2(out[u].float().cpu().numpy(), ref) < TOL_BF16


def test_splits_agree(pk, batch):
    B = batch
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], unique_cap=512 / B["N"])
    op.route(B["Q"])
    outs = [op.attention(B["Q"], B["K"], B["V"], splits=s).float().clone() for s in (1, 3, 16, 64)]
    # The attention weights enter the PV product in bf16 (relative rounding
    # 2^-9, renormalised per split) and the outputs are bf16, so split trees
    # agree to a few 1e-3 -- an order below the bf16 parity tolerance.
    for o in outs[1:]:
        assert rel_l2(o.cpu().numpy(), outs[0].cpu().numpy()) < 5e-3


def test_split_counts_in_any_order(pk, batch):
    """Cluster launches of different split counts share one shared-memory
    limit per kernel; a larger split count after a smaller one (the limit
    set lower in between) must still launch."""
    B = batch
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], unique_cap=512 / B["N"])
    op.route(B["Q"])
    ref = op.attention(B["Q"], B["K"], B["V"], splits=1).float().clone()
    for s in (16, 3, 16, 8, 2, 12, 16):
        out = op.attention(B["Q"], B["K"], B["V"], splits=s).float()
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 5e-3, s


def test_sequence_shard_partials_merge(pk, batch):
    """Emulates the sequence-sharded decode on one GPU: each shard attends
    over its own id range and the LSE merge of the partials equals the
    unsharded result."""
    B = batch
    U, G, d = B["U"], B["G"], B["d"]
    from prismkv_b200 import native as nv
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=G, unique_cap=None)
    op.route(B["Q"])
    one = torch.empty(1, U * G, d + 2, device="cuda")
    op.attention(B["Q"], B["K"], B["V"], partial=one[0])
    full = torch.empty(U * G, d, dtype=torch.float32, device="cuda")
    nv.call("pk_lse_merge", one, 1, U * G, d, full, nv.PK_F32)
    full = full.view(U, G, d)
    ids = op.ids.clone()
    count = op.count.clone()
    P = 3
    parts = torch.empty(P, U * G, d + 2, device="cuda")
    for r in range(P):
        lo, hi = r * B["N"] // P, (r + 1) * B["N"] // P
        sel = [(ids[u, :count[u]][(ids[u, :count[u]] >= lo) & (ids[u, :count[u]] < hi)]) for u in range(U)]
        op.ids.zero_()
        for u in range(U):
            op.ids[u, :len(sel[u])] = sel[u]
            op.count[u] = len(sel[u])
        # The dense tail belongs to the last shard only.
        length = torch.full((U,), B["N"] + B["tail"] if r == P - 1 else B["N"], dtype=torch.int32, device="cuda")
        op.attention(B["Q"], B["K"], B["V"], length=length, partial=parts[r])
    merged = torch.empty(U * G, d, dtype=torch.float32, device="cuda")
    nv.call("pk_lse_merge", parts, P, U * G, d, merged, nv.PK_F32)
    # Each shard's online softmax rounds its weights to bf16 against its own
    # running maximum, so shard and full partials differ by that rounding
    # (~1e-4 relative); the fp32 merge itself adds no error.
    assert rel_l2(merged.view(U, G, d).cpu().numpy(), full.cpu().numpy()) < 2e-3


def test_slot_major_layout_and_inactive_unit(pk, batch):
    B = batch
    U, G, d = B["U"], B["G"], B["d"]
    Hkv = 4
    K4 = B["K"].view(U // Hkv, Hkv, -1, d).transpose(1, 2).contiguous()  # [B, T, Hkv, d]
    V4 = B["V"].view(U // Hkv, Hkv, -1, d).transpose(1, 2).contiguous()
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=G, unique_cap=512 / B["N"])
    op.route(B["Q"])
    ref = op.attention(B["Q"], B["K"], B["V"]).float().clone()
    got = op.attention(B["Q"], K4, V4).float().clone()
    assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < 1e-6
    length = torch.full((U,), B["N"] + B["tail"], dtype=torch.int32, device="cuda")
    length[-1] = 0
    masked = op.attention(B["Q"], K4, V4, length=length)
    assert torch.count_nonzero(masked[-1]).item() == 0
    assert rel_l2(masked[:-1].float().cpu().numpy(), ref[:-1].cpu().numpy()) < 1e-6


def test_fp32_decode_path(pk, oracle, batch):
    B = batch
    K, V, Q = B["K"].float(), B["V"].float(), B["Q"].float().contiguous()
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], unique_cap=256 / B["N"])
    out = op(Q, K, V)
    for u in range(B["U"]):
        oids, _ = oracle.select_buckets(B["q"][u], B["oidx"][u], unique_cap=256 / B["N"], router="q_activation",
                                        sae=B["osae"], query_scale=1.0, query_topk=B["k"])
        ref = oracle.attend(B["q"][u], B["keys"][u], B["vals"][u], oids, B["N"])
        assert rel_l2(out[u].cpu().numpy(), ref) < TOL_F32


def test_empty_index_zero_budget_and_tail_only(pk, oracle):
    dev = torch.device("cuda")
    rs = np.random.RandomState(3)
    n, d, F = 300, 128, 64
    keys = bf16_round(rs.standard_normal((n + 5, d)).astype(np.float32))
    vals = bf16_round(rs.standard_normal((n + 5, d)).astype(np.float32))
    q = bf16_round(rs.standard_normal((4, d)).astype(np.float32))
    W = -np.abs(rs.standard_normal((F, d))).astype(np.float32) * 0
    b = np.full(F, -1.0, np.float32)  # every activation <= 0: empty index
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.from_numpy(b).to(dev), key_mean=8, query_topk=8)
    K = torch.from_numpy(keys).to(dev).bfloat16()
    V = torch.from_numpy(vals).to(dev).bfloat16()
    Q = torch.from_numpy(q).to(dev).bfloat16()
    idx = pk.build_index(K[:n], sae, 1.0)
    assert int(idx.counts.sum()) == 0
    ids, meta = pk.select_buckets(Q, idx, router="q_activation", sae=sae, query_scale=1.0, query_topk=8)
    assert len(ids) == 0 and meta["features"] == [] and meta["candidate_buckets"] == 0
    out = pk.attend(Q, K, V, ids, n)
    ref = oracle.attend(q, keys, vals, np.zeros(0, np.int64), n)
    assert rel_l2(out.float().cpu().numpy(), ref) < TOL_BF16
    # zero budget on a populated index
    W2 = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    sae2 = pk.SAEParams(torch.from_numpy(W2).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=8)
    idx2 = pk.build_index(K[:n], sae2, 1.0)
    ids2, meta2 = pk.select_buckets(Q, idx2, unique_cap=0.0, router="q_activation", sae=sae2, query_scale=1.0,
                                    query_topk=8)
    assert len(ids2) == 0 and meta2["raw"] == 0 and meta2["limit"] == 0
    # no old rows and no tail: zeros (core.py:180-181)
    out0 = pk.attend(Q, K[:n], V[:n], ids2, n)
    assert torch.count_nonzero(out0).item() == 0


def test_tied_activations_follow_flat_index_order(pk, oracle):
    """All activations equal: the budget takes ties by ascending flat index
    (core.py:24), as the reference's own tie fixture."""
    dev = torch.device("cuda")
    d = 128
    W = np.zeros((3, d), np.float32)
    W[0, 0] = W[1, 0] = W[2, 1] = 1.0
    keys = np.ones((9, d), np.float32)
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.zeros(3, device=dev), key_mean=2, query_topk=2)
    idx = pk.build_index(torch.from_numpy(keys).to(dev), sae, 1.0, center=torch.zeros(d, device=dev))
    osae = oracle.SAE(W, np.zeros(3, np.float32), key_mean=2, query_topk=2)
    oidx = oracle.build_index(keys, osae, 1.0, center=np.zeros(d, np.float32))
    counts, ids = idx.dev.csr(0)
    assert counts.tolist() == [6, 6, 6] == oidx.counts.tolist()
    assert np.array_equal(ids, oidx.ids)


def test_append_grows_regions_when_full(pk, oracle):
    """Appends that overflow a bucket region repack the index and retry;
    the result equals the oracle's append_index."""
    dev = torch.device("cuda")
    rs = np.random.RandomState(11)
    n, d, F = 512, 128, 64
    keys = bf16_round((rs.standard_normal((n + 256, d)) + 1).astype(np.float32))
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=8)
    K = torch.from_numpy(keys).to(dev).bfloat16()
    idx = pk.DeviceIndex.build(K[:n], sae, 1.0, moments=True, slack_frac=0.0, slack_min=0)
    osae = oracle.SAE(W, np.zeros(F, np.float32), key_mean=8, query_topk=8)
    oidx = oracle.build_index(keys[:n], osae, 1.0)
    for lo in range(n, n + 256, 64):
        idx.append(K[lo:lo + 64], sae, 1.0)
        oidx = oracle.append_index(oidx, keys[lo:lo + 64], osae, 1.0)
    counts, ids = idx.csr(0)
    assert idx.history == oidx.history
    assert np.array_equal(counts, oidx.counts)
    assert np.array_equal(ids, oidx.ids)
    assert np.array_equal(idx.mean[0].cpu().numpy().view(np.uint32), oidx.mean.view(np.uint32))
    assert np.array_equal(idx.var[0].cpu().numpy().view(np.uint32), oidx.variance.view(np.uint32))


def test_bound_filtered_routing_equals_exact_encode(pk, batch):
    """The tensor-core-filtered router and the all-features exact encode
    give identical candidate orders and unions on many queries."""
    B = batch
    fast = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], unique_cap=512 / B["N"])
    exact = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=B["G"], unique_cap=512 / B["N"], exact_encode=True)
    g = torch.Generator(device="cuda").manual_seed(9)
    for rep in range(20):
        q = (B["Q"].float() + 0.5 * torch.randn(B["Q"].shape, device="cuda", generator=g)).bfloat16().contiguous()
        fast.route(q)
        exact.route(q)
        torch.cuda.synchronize()
        assert torch.equal(fast.n_order, exact.n_order), rep
        for u in range(B["U"]):
            n = int(exact.n_order[u])
            assert torch.equal(fast.order[u, :n], exact.order[u, :n]), (rep, u)
            c = int(exact.count[u])
            assert int(fast.count[u]) == c
            assert torch.equal(fast.ids[u, :c], exact.ids[u, :c])


def _union_case(pk, oracle, rs, U, H, F, n_cand, sizes_from, probs, hot_n, limits, hist_u=None, n_u=None):
    """Random CSR indexes (buckets drawn from a shared hot set plus random
    tokens, so they overlap), a random candidate order per unit; every limit
    through pk_union against the oracle's greedy."""
    from prismkv_b200 import native as nv
    dev = torch.device("cuda")
    hist_u = hist_u or [H] * U
    n_u = n_u if n_u is not None else [n_cand] * U
    lists_all, orders = [], []
    for u in range(U):
        Hu = hist_u[u]
        sizes = rs.choice(sizes_from, size=F, p=probs)
        hot = rs.randint(0, Hu, size=hot_n)
        lists = []
        for f in range(F):
            pool = np.concatenate([hot, rs.randint(0, Hu, size=int(sizes[f]))])
            lists.append(np.unique(rs.choice(pool, size=min(len(pool), int(sizes[f])), replace=False)))
        lists_all.append(lists)
        orders.append(rs.permutation(F)[:n_cand])
    dindex = pk.index.from_lists([[torch.from_numpy(x) for x in l] for l in lists_all], H, 128, dev)
    order = torch.tensor(np.stack(orders), dtype=torch.int32, device=dev)
    n_order = torch.tensor(n_u, dtype=torch.int32, device=dev)
    hist = torch.tensor(hist_u, dtype=torch.int32, device=dev)
    for lim in limits:
        limit = torch.full((U,), lim, dtype=torch.int64, device=dev)
        out = torch.empty(U, H, dtype=torch.int32, device=dev)
        cnt = torch.empty(U, dtype=torch.int32, device=dev)
        feats = torch.empty(U, n_cand, dtype=torch.int32, device=dev)
        nf = torch.empty(U, dtype=torch.int32, device=dev)
        raw = torch.empty(U, dtype=torch.int64, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        nv.call("pk_union", dindex.offsets, dindex.lens, dindex.ids, dindex.ids.stride(0), order, n_order,
                n_cand, hist, limit, U, F, H, out, H, cnt, feats, nf, raw, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for u in range(U):
            oi = oracle.index_from_lists(hist_u[u], np.zeros(128, np.float32), lists_all[u])
            ids, fts, rw = oracle.select_from_order(orders[u][:n_u[u]], oi, lim)
            c = int(cnt[u])
            assert np.array_equal(out[u, :c].cpu().numpy().astype(np.int64), ids), (lim, u)
            assert feats[u, :int(nf[u])].cpu().tolist() == fts, (lim, u)
            assert int(raw[u]) == rw, (lim, u)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_union_matches_oracle_on_config3_like_buckets(pk, oracle, seed):
    """Buckets of config-3-like sizes that overlap, against the oracle: the
    unbudgeted path, prefixes that stop at the first skip, and tail walks
    with accepted buckets after it.  Units differ in history (the bitmap's
    last partial word at several widths) and one unit has no candidates."""
    rs = np.random.RandomState(200 + seed)
    U, H, F, n_cand = 5, 70001, 400, 160
    _union_case(pk, oracle, rs, U, H, F, n_cand, [2, 30, 120, 400], [0.2, 0.4, 0.3, 0.1], 2000,
                (0, 300, 2500, 4096, 9000, 10 ** 9),
                hist_u=[70001, 65536, 1000, 70001, 33], n_u=[160, 160, 160, 0, 160])


def test_union_matches_oracle_when_tokens_are_mostly_distinct(pk, oracle):
    """About 18,000 list entries over a 200,000-token history with almost no
    overlap between the candidates' lists."""
    rs = np.random.RandomState(7)
    _union_case(pk, oracle, rs, 3, 200000, 300, 120, [150], [1.0], 10, (0, 5000, 12000, 10 ** 9))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_union_greedy_matches_oracle_on_large_buckets(pk, oracle, seed):
    """Budgeted union on synthetic CSR indexes whose buckets are large and
    overlap heavily (multi-round hash path, single-bucket rounds, accepted
    buckets after the first skip), against the oracle's greedy."""
    rs = np.random.RandomState(100 + seed)
    _union_case(pk, oracle, rs, 6, 60000, 300, 200, [3, 40, 300, 2000, 9000], [0.2, 0.4, 0.3, 0.08, 0.02], 3000,
                (0, 500, 4096, 20000, 10 ** 9))


def test_union_matches_oracle_at_a_million_token_history(pk, oracle):
    """Config 4's union size: a 2^20-token history, whose bitmap leaves room
    to stage only part of the 256 candidates' lists, so the tail runs the
    windowed recount rounds; against the oracle's greedy."""
    rs = np.random.RandomState(41)
    _union_case(pk, oracle, rs, 2, 1 << 20, 600, 256, [64, 256, 1024], [0.3, 0.5, 0.2], 4000,
                (0, 8192, 30000, 10 ** 9))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_bound_filtered_build_equals_exact_build(pk, dtype):
    """Tensor-core bounds + exact recompute of the undecided band give the
    same memberships as computing every activation exactly."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(21)
    U, N, d, F, C = 4, 6000, 128, 1024, 48
    centers = torch.randn(U, C, d, device=dev, generator=g)
    cid = torch.randint(0, C, (U, N), device=dev, generator=g)
    keys = (torch.gather(centers, 1, cid[..., None].expand(U, N, d)) +
            0.3 * torch.randn(U, N, d, device=dev, generator=g)).to(dtype)
    W = torch.randn(F, d, device=dev, generator=g) / d ** 0.5
    b = 0.05 * torch.randn(F, device=dev, generator=g)
    sae = pk.SAEParams(W, b, key_mean=8, query_topk=16)
    fast = pk.DeviceIndex.build(keys, sae, 1.3, moments=False)
    exact = pk.DeviceIndex.build(keys, sae, 1.3, moments=False, exact=True)
    # The tensor-core bounds decided (no fallback to the exact path).
    assert fast.encode_path == "bounds" and exact.encode_path == "exact"
    assert torch.equal(fast.center, exact.center)
    for u in range(U):
        cf, idf = fast.csr(u)
        ce, ide = exact.csr(u)
        assert np.array_equal(cf, ce), u
        assert np.array_equal(idf, ide), u


@pytest.mark.parametrize("G", [1, 3, 8, 12, 16])
def test_attention_head_counts_and_split_forms_match_oracle(pk, oracle, G):
    """Both bf16 attention kernels -- heads in the MMA's N for G <= 8, in its
    M for 9..16 -- with one split, a cluster of splits merged on chip, more
    splits than one cluster holds (for G <= 8: clusters of 8, 6 or 5 merged
    on chip and then across clusters through global memory; a prime count
    takes the last-CTA merge of every split), against the oracle's attend
    (core.py:170-183) on the same bf16 inputs.  Each workspace is used twice
    in a row (the arrival counters must be left at zero)."""
    from prismkv_b200 import native as nv
    rs = np.random.RandomState(11 + G)
    U, N, tail, d = 3, 2048, 5, 128
    keys = bf16_round(rs.standard_normal((U, N + tail, d)).astype(np.float32))
    vals = bf16_round(rs.standard_normal((U, N + tail, d)).astype(np.float32))
    q = bf16_round(rs.standard_normal((U, G, d)).astype(np.float32))
    counts = [700, 0, 1531]
    width = 1536
    ids = np.zeros((U, width), np.int32)
    sel = []
    for u, c in enumerate(counts):
        s = np.sort(rs.choice(N, c, replace=False)).astype(np.int32)
        ids[u, :c] = s
        sel.append(s)
    dev = torch.device("cuda")
    K = torch.from_numpy(keys).to(dev).to(torch.bfloat16)
    V = torch.from_numpy(vals).to(dev).to(torch.bfloat16)
    Q = torch.from_numpy(q).to(dev).to(torch.bfloat16).contiguous()
    tid = torch.from_numpy(ids).to(dev)
    count = torch.tensor(counts, dtype=torch.int32, device=dev)
    hist = torch.full((U,), N, dtype=torch.int32, device=dev)
    length = torch.full((U,), N + tail, dtype=torch.int32, device=dev)
    refs = [oracle.attend(q[u], keys[u], vals[u], sel[u], N) for u in range(U)]
    for splits in (1, 4, 8, 13, 12, 16, 20, 24, 64):
        nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, splits)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        first = None
        for rep in range(2):
            out = torch.full((U, G, d), float("nan"), dtype=torch.bfloat16, device=dev)
            nv.call("pk_sparse_av", Q, K, V, nv.PK_BF16, 1, K.stride(0), 0, K.stride(1), tid, width, count, hist,
                    length, U, G, d, splits, ws, nbytes, out, None)
            torch.cuda.synchronize()
            if first is None:
                first = out.clone()
            else:
                assert torch.equal(out, first), (G, splits)
        got = out.float().cpu().numpy()
        for u in range(U):
            assert rel_l2(got[u], refs[u]) < TOL_BF16, (G, splits, u)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kv_append_matches_indexed_assignment(pk, dtype):
    """The decode KV append (batch_append, kernels/cuda_sm90/native_sources/
    av.cu:70-90) into a slot-major and a unit-major cache equals indexed
    assignment; positions outside [0, capacity) leave their slot untouched."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(3)
    S, cap, Hkv, d = 5, 40, 4, 128
    pos = torch.tensor([0, 17, cap - 1, -1, cap], dtype=torch.int32, device=dev)
    for shape, new_shape in (((S, cap, Hkv, d), (S, Hkv, d)), ((S, cap, d), (S, d))):
        Kc = torch.randn(*shape, device=dev, generator=g).to(dtype)
        Vc = torch.randn(*shape, device=dev, generator=g).to(dtype)
        kn = torch.randn(*new_shape, device=dev, generator=g).to(dtype)
        vn = torch.randn(*new_shape, device=dev, generator=g).to(dtype)
        refK, refV = Kc.clone(), Vc.clone()
        for s in range(S):
            p = int(pos[s])
            if 0 <= p < cap:
                refK[s, p] = kn[s]
                refV[s, p] = vn[s]
        pk.kv_append(kn, vn, Kc, Vc, pos)
        torch.cuda.synchronize()
        assert torch.equal(Kc, refK) and torch.equal(Vc, refV)
    with pytest.raises(ValueError):
        pk.kv_append(kn, vn, Kc, Vc, pos.long())


@pytest.mark.parametrize("G,dtype", [(4, torch.bfloat16), (12, torch.bfloat16), (4, torch.float32)])
def test_fused_append_equals_append_then_attention(pk, G, dtype):
    """pk_sparse_av_append (the KV append fused into the attention launch)
    gives the output and caches of writing the new rows first and attending
    after (batch_append then batch_av, kernels/cuda_sm90/model.py:109-137),
    bit for bit: both attention kernels and the fp32 one, with one split, a
    cluster of splits and more than 8 splits; an inactive unit and a unit
    without a tail row are left alone."""
    from prismkv_b200 import native as nv
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(21 + G)
    U, N, tail, d = 6, 1024, 9, 128
    total = N + tail + 4
    K = torch.randn(U, total, d, device=dev, generator=g).to(dtype)
    V = torch.randn(U, total, d, device=dev, generator=g).to(dtype)
    Q = torch.randn(U, G, d, device=dev, generator=g).to(dtype).contiguous()
    kn = torch.randn(U, d, device=dev, generator=g).to(dtype)
    vn = torch.randn(U, d, device=dev, generator=g).to(dtype)
    width = 320
    ids = torch.zeros(U, width, dtype=torch.int32, device=dev)
    count = torch.full((U,), 300, dtype=torch.int32, device=dev)
    count[2] = 0
    for u in range(U):
        ids[u, :300] = torch.randperm(N, device=dev, generator=g)[:300].sort().values.int()
    hist = torch.full((U,), N, dtype=torch.int32, device=dev)
    length = torch.full((U,), N + tail, dtype=torch.int32, device=dev)
    length[4] = 0          # inactive unit
    length[5] = N          # no tail row: nothing appended
    for splits in (1, 8, 12):
        nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, splits)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        K1, V1 = K.clone(), V.clone()
        for u in range(U):
            if int(length[u]) > N:
                K1[u, int(length[u]) - 1] = kn[u]
                V1[u, int(length[u]) - 1] = vn[u]
        out1 = torch.empty(U, G, d, dtype=dtype, device=dev)
        code = nv.dtype_code(Q)
        nv.call("pk_sparse_av", Q, K1, V1, code, 1, K1.stride(0), 0, K1.stride(1), ids, width, count, hist, length,
                U, G, d, splits, ws, nbytes, out1, None)
        K2, V2 = K.clone(), V.clone()
        out2 = torch.empty(U, G, d, dtype=dtype, device=dev)
        nv.call("pk_sparse_av_append", Q, K2, V2, code, 1, K2.stride(0), 0, K2.stride(1), ids, width, count, hist,
                length, U, G, d, splits, ws, nbytes, out2, None, kn, vn)
        torch.cuda.synchronize()
        assert torch.equal(out1, out2), splits
        assert torch.equal(K1, K2) and torch.equal(V1, V2), splits


@pytest.mark.parametrize("G", [3, 8, 12])
def test_routing_head_counts_match_oracle(pk, oracle, batch, G):
    """q_activation routing (core.py:131-139) for G heads per unit, bit-exact
    against the oracle: G <= 8 builds the unit's order in a cluster of its
    head CTAs, G = 12 in the unit's last CTA; G = 3 takes the interleaved dot
    order of F.linear, G >= 6 the sequential one."""
    B = batch
    U, d, k = B["U"], B["d"], B["k"]
    rs = np.random.RandomState(40 + G)
    q = bf16_round(rs.standard_normal((U, G, d)).astype(np.float32))
    Q = torch.from_numpy(q).cuda().to(torch.bfloat16).contiguous()
    op = pk.SparseDecode(B["idx"], B["sae"], heads_per_unit=G, unique_cap=512 / B["N"])
    op.route(Q)
    torch.cuda.synchronize()
    for u in range(U):
        _, ref = oracle.bucket_scores(q[u], B["oidx"][u], router="q_activation", sae=B["osae"], query_scale=1.0,
                                      query_topk=k)
        n = int(op.n_order[u])
        assert n == len(ref), (G, u)
        assert np.array_equal(op.order[u, :n].cpu().numpy(), ref), (G, u)
