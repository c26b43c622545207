"""GPU tests of the sequence-sharded decode.

On one GPU the P shards are emulated: a built index is cut into token shards
(shard_index), each shard routes and attends over its own rows and exports
its (m, l, o) partial, and pk_lse_merge combines them; the unbudgeted union
of every shard must be the global union cut at the shard boundaries (bit
exact) and the merged output must match the unsharded one.  With two or
more GPUs the same path runs as two NCCL ranks (ShardedDecode), compared
with a single-GPU run of the whole history."""
import os
import socket

import numpy as np
import pytest
import torch

from gen import bf16_round

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_case(seed, U=4, N=6000, tail=12, d=128, C=48, F=1024, G=4, k=16):
    rs = np.random.RandomState(seed)
    centers = rs.standard_normal((U, C, d)).astype(np.float32)
    cid = rs.randint(0, C, size=(U, N + tail))
    uu = np.arange(U)[:, None]
    keys = bf16_round((centers[uu, cid] + np.float32(0.3) * rs.standard_normal((U, N + tail, d))).astype(np.float32))
    vals = bf16_round(rs.standard_normal((U, N + tail, d)).astype(np.float32))
    q = bf16_round((centers[uu, rs.randint(0, C, size=(U, G))] +
                    np.float32(0.3) * rs.standard_normal((U, G, d))).astype(np.float32))
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    return dict(U=U, N=N, tail=tail, d=d, F=F, G=G, k=k, keys=keys, vals=vals, q=q, W=W)


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    import prismkv_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return prismkv_b200


@pytest.mark.parametrize("P", [2, 3])
def test_emulated_shards_match_unsharded(pk, P):
    from prismkv_b200 import native as nv
    from prismkv_b200.shard import shard_index, token_ranges
    c = make_case(11)
    U, N, G, d = c["U"], c["N"], c["G"], c["d"]
    dev = torch.device("cuda")
    K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
    V = torch.from_numpy(c["vals"]).to(dev).bfloat16()
    Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(c["F"], device=dev), key_mean=8,
                       query_topk=c["k"])
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    full_op = pk.SparseDecode(idx, sae, heads_per_unit=G, unique_cap=None)
    full_op.route(Q)
    one = torch.empty(1, U * G, d + 2, device=dev)
    full_op.attention(Q, K, V, partial=one[0])
    ref = torch.empty(U * G, d, device=dev)
    nv.call("pk_lse_merge", one, 1, U * G, d, ref, nv.PK_F32)
    parts = torch.empty(P, U * G, d + 2, device=dev)
    for r, (lo, hi) in enumerate(token_ranges(N, P)):
        sh = shard_index(idx, lo, hi)
        op = pk.SparseDecode(sh, sae, heads_per_unit=G, unique_cap=None)
        op.route(Q)
        torch.cuda.synchronize()
        op.check()
        for u in range(U):
            glob = full_op.ids[u, :int(full_op.count[u])].long()
            want = glob[(glob >= lo) & (glob < hi)] - lo
            got = op.ids[u, :int(op.count[u])].long()
            assert torch.equal(got, want)
        # The shard's rows, the last shard followed by the dense tail.
        rows = slice(lo, hi + c["tail"]) if r == P - 1 else slice(lo, hi)
        op.attention(Q, K[:, rows].contiguous(), V[:, rows].contiguous(), partial=parts[r])
    merged = torch.empty(U * G, d, device=dev)
    nv.call("pk_lse_merge", parts, P, U * G, d, merged, nv.PK_F32)
    # bf16 weights are rounded against each shard's own running maximum.
    assert rel_l2(merged.cpu().numpy(), ref.cpu().numpy()) < 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, exchange="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import prismkv_b200 as pk
        from prismkv_b200.shard import ShardedDecode, shard_index, token_ranges
        c = make_case(5)
        U, N, G, d = c["U"], c["N"], c["G"], c["d"]
        K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
        V = torch.from_numpy(c["vals"]).to(dev).bfloat16()
        Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
        sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(c["F"], device=dev), key_mean=8,
                           query_topk=c["k"])
        idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
        lo, hi = token_ranges(N, world)[rank]
        sd = ShardedDecode(shard_index(idx, lo, hi), sae, heads_per_unit=G, budget=None, exchange=exchange,
                           split_route=True)
        assert sd.exchange == exchange and sd.split_route
        rows = slice(lo, hi + c["tail"]) if sd.is_tail_rank else slice(lo, hi)
        Ks, Vs = K[:, rows].contiguous(), V[:, rows].contiguous()
        ref = pk.SparseDecode(idx, sae, heads_per_unit=G, unique_cap=None)(Q, K, V).float()
        errs = []
        for rep in range(3):   # repeated steps (both parities of the peer exchange)
            out = sd(Q, Ks, Vs).float()
            torch.cuda.synchronize()
            sd.check()
            errs.append(float((out - ref).norm() / ref.norm()))
        q.put((rank, max(errs)))
        sd.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_two_rank_nccl_sharded_decode(exchange):
    """Two ranks (NCCL process group), the step's all-gathers by NCCL or over
    NVLink peer memory (pk_p2p_allgather)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(e < 2e-2 for e in res.values()), res


@pytest.mark.parametrize("P", [2, 4])
def test_emulated_shards_moments_router(pk, oracle, P):
    """The moments router on sequence shards: each shard's moments folded in
    token order with the append merge (core.py:194-199) equal the oracle's
    fold bit for bit; with them and the whole sequence's bucket sizes every
    shard routes the buckets the oracle routes from those moments
    (core.py:117-130), the unbudgeted shard unions are the global union cut
    at the shard boundaries, and the merged attention matches the oracle."""
    from prismkv_b200 import native as nv
    from prismkv_b200.shard import fold_moments, shard_index, shard_moments, token_ranges, ShardedDecode
    c = make_case(17)
    U, N, G, d, F, k = c["U"], c["N"], c["G"], c["d"], c["F"], c["k"]
    dev = torch.device("cuda")
    K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
    V = torch.from_numpy(c["vals"]).to(dev).bfloat16()
    Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    ranges = token_ranges(N, P)
    shards = [shard_index(idx, lo, hi) for lo, hi in ranges]
    parts = [shard_moments(sh, K[:, lo:hi].contiguous()) for sh, (lo, hi) in zip(shards, ranges)]
    counts, mean, var = fold_moments(parts)
    torch.cuda.synchronize()
    assert torch.equal(counts, idx.lens)
    osae = oracle.SAE(c["W"], np.zeros(F, np.float32), key_mean=8, query_topk=k)
    fulls = [oracle.build_index(c["keys"][u, :N], osae, 1.0, moments=False) for u in range(U)]
    for u in range(U):
        # The oracle's fold: per shard, summarize its keys over its part of
        # every bucket, then merge in token order.
        om = ov = oc = None
        for lo, hi in ranges:
            lists = [x[(x >= lo) & (x < hi)] - lo for x in fulls[u].lists]
            part = oracle.summarize(c["keys"][u, lo:hi], lists)
            if om is None:
                om, ov, oc = part.mean, part.variance, part.counts
            else:
                om, ov = oracle.merge_moments(oc, om, ov, part.counts, part.mean, part.variance)
                oc = oc + part.counts
        assert np.array_equal(mean[u].cpu().numpy().view(np.uint32), om.view(np.uint32)), u
        assert np.array_equal(var[u].cpu().numpy().view(np.uint32), ov.view(np.uint32)), u
    # Level 1: the order the oracle takes from the device's own scores of
    # the folded moments and the whole sequence's sizes.
    orders = []
    for u in range(U):
        s_dev = torch.empty(1, F, device=dev)
        o1 = torch.empty(1, k, dtype=torch.int32, device=dev)
        n1 = torch.empty(1, dtype=torch.int32, device=dev)
        ws = torch.empty(int(nv.query("pk_route_moments_workspace_bytes", 1, G, F)), dtype=torch.uint8, device=dev)
        nv.call("pk_route_moments", Q[u:u + 1].contiguous(), nv.PK_BF16, mean[u:u + 1].contiguous(),
                var[u:u + 1].contiguous(), counts[u:u + 1].contiguous(), 7, 1, G, d, F, k, ws, ws.numel(), s_dev,
                o1, n1, k)
        orders.append(oracle.order_live(s_dev[0].cpu().numpy(), counts[u].long().cpu().numpy(), k))
    out_parts = torch.empty(P, U * G, d + 2, device=dev)
    for r, (sh, (lo, hi)) in enumerate(zip(shards, ranges)):
        sh.mean, sh.var, sh.global_counts = mean, var, counts
        sd = ShardedDecode(sh, sae, heads_per_unit=G, router="moments", query_topk=k, budget=None)
        sd.op.route(Q)
        torch.cuda.synchronize()
        sd.check()
        for u in range(U):
            n = int(sd.op.n_order[u])
            assert np.array_equal(sd.op.order[u, :n].long().cpu().numpy(), orders[u]), (r, u)
            local = oracle.index_from_lists(hi - lo, np.zeros(d, np.float32),
                                            [x[(x >= lo) & (x < hi)] - lo for x in fulls[u].lists])
            ids, _, _ = oracle.select_from_order(orders[u], local, hi - lo)
            cnt = int(sd.op.count[u])
            assert np.array_equal(sd.op.ids[u, :cnt].long().cpu().numpy(), ids), (r, u)
        rows = slice(lo, hi + c["tail"]) if r == P - 1 else slice(lo, hi)
        sd.op.attention(Q, K[:, rows].contiguous(), V[:, rows].contiguous(), partial=out_parts[r])
    merged = torch.empty(U * G, d, device=dev)
    nv.call("pk_lse_merge", out_parts, P, U * G, d, merged, nv.PK_F32)
    merged = merged.view(U, G, d).cpu().numpy()
    for u in range(U):
        gids, _, _ = oracle.select_from_order(orders[u], fulls[u], N)
        ref = oracle.attend(c["q"][u], c["keys"][u], c["vals"][u], gids, N)
        assert rel_l2(merged[u], ref) < 2e-2, u


def _rank_main_moments(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import prismkv_b200 as pk
        from prismkv_b200.shard import ShardedDecode, attach_global_moments, fold_moments, shard_index, \
            shard_moments, token_ranges
        c = make_case(23)
        U, N, G, d, F, k = c["U"], c["N"], c["G"], c["d"], c["F"], c["k"]
        K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
        V = torch.from_numpy(c["vals"]).to(dev).bfloat16()
        Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
        sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=k)
        idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
        ranges = token_ranges(N, world)
        lo, hi = ranges[rank]
        sh = attach_global_moments(shard_index(idx, lo, hi), K[:, lo:hi].contiguous(), gather_bytes=1 << 20)
        # Every rank's moments equal the in-process fold of all shards.
        _, m_ref, v_ref = fold_moments([shard_moments(shard_index(idx, a, b), K[:, a:b].contiguous())
                                        for a, b in ranges])
        same = torch.equal(sh.mean, m_ref) and torch.equal(sh.var, v_ref) and torch.equal(sh.global_counts, idx.lens)
        sd = ShardedDecode(sh, sae, heads_per_unit=G, router="moments", query_topk=k, budget=None)
        rows = slice(lo, hi + c["tail"]) if sd.is_tail_rank else slice(lo, hi)
        out = sd(Q, K[:, rows].contiguous(), V[:, rows].contiguous()).float()
        full = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
        full.mean, full.var = m_ref, v_ref
        ref = pk.SparseDecode(full, sae, heads_per_unit=G, router="moments", query_topk=k,
                              unique_cap=None)(Q, K, V).float()
        torch.cuda.synchronize()
        err = float((out - ref).norm() / ref.norm())
        q.put((rank, (same, err)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_nccl_sharded_moments_router():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_moments, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(s and e < 2e-2 for s, e in res.values()), res


@pytest.mark.parametrize("P", [2, 3, 8])
def test_feature_split_route_equals_unsharded(pk, P):
    """The feature-sharded q_activation route: each feature range's picks
    (pk_route_qact_shard), stacked as an all-gather would, merged on one
    device (pk_route_qact_merge) give the unsharded route's order and, with
    it, the same budgeted union (integer outputs, bit-exact)."""
    from prismkv_b200.shard import feature_ranges
    c = make_case(23)
    U, N, G, d, F, k = c["U"], c["N"], c["G"], c["d"], c["F"], c["k"]
    dev = torch.device("cuda")
    K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
    Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    ref = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=1500)
    ref.route(Q)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=1500)
    gathered = torch.empty(P, U * G, k, 2, dtype=torch.int32, device=dev)
    for r, (lo, hi) in enumerate(feature_ranges(F, P)):
        op.route_shard_picks(Q, lo, hi, gathered[r])
    op.route_merge(gathered)
    op.union()
    torch.cuda.synchronize()
    ref.check()
    op.check()
    assert torch.equal(op.n_order, ref.n_order)
    for u in range(U):
        n = int(ref.n_order[u])
        assert torch.equal(op.order[u, :n], ref.order[u, :n]), u
        c_ = int(ref.count[u])
        assert int(op.count[u]) == c_ and torch.equal(op.ids[u, :c_], ref.ids[u, :c_]), u


def test_feature_split_route_config4_shape(pk):
    """The feature-sharded route at config 4's routing shape (F = 32768,
    64 features per query head, 8 units of 4 heads) over 8 feature ranges
    equals the unsharded route's order bit for bit."""
    from prismkv_b200.shard import feature_ranges
    rs = np.random.RandomState(29)
    U, G, d, F, k, N, C = 8, 4, 128, 32768, 64, 16384, 256
    centers = rs.standard_normal((U, C, d)).astype(np.float32)
    cid = rs.randint(0, C, size=(U, N))
    keys = (centers[np.arange(U)[:, None], cid] + np.float32(0.3) * rs.standard_normal((U, N, d))).astype(np.float32)
    q = (centers[np.arange(U)[:, None], rs.randint(0, C, size=(U, G))]
         + np.float32(0.3) * rs.standard_normal((U, G, d))).astype(np.float32)
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    dev = torch.device("cuda")
    K = torch.from_numpy(keys).to(dev).bfloat16()
    Q = torch.from_numpy(q).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K, sae, 1.0, moments=False)
    ref = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=8192)
    ref.route(Q)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=8192)
    P = 8
    gathered = torch.empty(P, U * G, k, 2, dtype=torch.int32, device=dev)
    for r, (lo, hi) in enumerate(feature_ranges(F, P)):
        op.route_shard_picks(Q, lo, hi, gathered[r])
    op.route_merge(gathered)
    op.union()
    torch.cuda.synchronize()
    assert torch.equal(op.n_order, ref.n_order) and torch.equal(op.count, ref.count)
    for u in range(U):
        n, c_ = int(ref.n_order[u]), int(ref.count[u])
        assert torch.equal(op.order[u, :n], ref.order[u, :n]), u
        assert torch.equal(op.ids[u, :c_], ref.ids[u, :c_]), u


def _p2p_rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        from prismkv_b200.shard import PeerExchange
        n = 1040   # floats: not a multiple of the 256-byte slot
        px = PeerExchange(n * 4, device=dev)
        ok = True
        out = torch.empty(world, n, device=dev)
        src = torch.empty(n, device=dev)
        for step in range(5):
            src.copy_(torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * rank + 10.0 * step)
            px.all_gather(src, out)
            torch.cuda.synchronize()
            px.check()
            want = torch.stack([torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * r + 10.0 * step
                                for r in range(world)])
            ok = ok and torch.equal(out, want)
        # The same exchange replayed from a CUDA graph.
        g = torch.cuda.CUDAGraph()
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(g, stream=s_cap):
                px.all_gather(src, out)
        torch.cuda.current_stream().wait_stream(s_cap)
        for step in range(5, 9):
            src.copy_(torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * rank + 10.0 * step)
            g.replay()
            torch.cuda.synchronize()
            px.check()
            want = torch.stack([torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * r + 10.0 * step
                                for r in range(world)])
            ok = ok and torch.equal(out, want)
        del g
        px.close()
        q.put((rank, ok))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_peer_exchange_all_gather():
    """pk_p2p_allgather between two ranks: every rank receives every rank's
    buffer, over repeated epochs (both parity slots), eager and replayed from
    a CUDA graph."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_p2p_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(res.values()), res


def test_peer_exchange_wait_runs_out_and_reports(pk):
    """Failure detection without a GPU fault: a two-rank exchange issued on
    one GPU against a stand-in peer region that nothing publishes into.
    The wait for the missing peer gives up after its poll limit, the status
    word reports PK_STATUS_EXCHANGE_TIMEOUT, this rank's own slot is still
    gathered, and the device stays usable."""
    import ctypes
    from prismkv_b200 import native as nv
    dev = torch.device("cuda")
    n = 256   # floats
    region = int(nv.query("pk_p2p_region_bytes", 2, n * 4))
    ptrs = []
    for _ in range(2):
        p = ctypes.c_uint64(0)
        assert nv.query("pk_p2p_alloc", region, ctypes.addressof(p)) == 0
        ptrs.append(int(p.value))
    try:
        bases = (ctypes.c_uint64 * 2)(*ptrs)
        src = torch.arange(n, device=dev, dtype=torch.float32)
        out = torch.full((2, n), -1.0, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        nv.call("pk_p2p_allgather", src, n * 4, 0, 2, ctypes.addressof(bases), ptrs[0], out, status, 2000)
        torch.cuda.synchronize()
        assert int(status.item()) == nv.STATUS_EXCHANGE_TIMEOUT
        assert torch.equal(out[0], src)
        with pytest.raises(RuntimeError, match="peer exchange timed out"):
            nv.check_status(status, "exchange")
        # The context is intact: ordinary work still runs.
        x = torch.randn(1024, device=dev)
        assert torch.allclose((x * 2).sum(), 2 * x.sum())
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            nv.query("pk_p2p_free", p)


def test_peer_exchange_single_rank_gathers_itself(pk):
    """With one rank the exchange is a copy into out[0], epoch after epoch."""
    from prismkv_b200.shard import PeerExchange
    dev = torch.device("cuda")
    px = PeerExchange(64 * 4, device=dev)
    out = torch.empty(1, 64, device=dev)
    try:
        for step in range(4):
            src = torch.randn(64, device=dev)
            px.all_gather(src, out)
            torch.cuda.synchronize()
            px.check()
            assert torch.equal(out[0], src)
    finally:
        px.close()


def test_feature_split_merge_ignores_repeated_and_out_of_range_picks(pk):
    """pk_route_qact_merge ignores ids outside [0, F), ranks a list out of
    rank order by the quadratic path and ranks repeated ids without gaps
    (the lists it expects are disjoint and in rank order; this keeps a
    malformed input from steering its memory accesses): the picks of the
    whole feature range followed by copies with their ids pushed out of
    range, or reversed, merge into the one-device route's order, and the
    same picks repeated three times merge without a fault."""
    c = make_case(31)
    U, N, G, d, F, k = c["U"], c["N"], c["G"], c["d"], c["F"], c["k"]
    dev = torch.device("cuda")
    K = torch.from_numpy(c["keys"]).to(dev).bfloat16()
    Q = torch.from_numpy(c["q"]).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(c["W"]).to(dev), torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    ref = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=1500)
    ref.route(Q)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=1500)
    picks = torch.empty(U * G, k, 2, dtype=torch.int32, device=dev)
    op.route_shard_picks(Q, 0, F, picks)
    bad = picks.clone()
    bad[..., 1] += F
    worse = picks.clone()
    worse[..., 1] = -worse[..., 1] - 1
    op.route_merge(torch.stack([picks, bad, worse]).contiguous())
    torch.cuda.synchronize()
    assert torch.equal(op.n_order, ref.n_order)
    for u in range(U):
        n = int(ref.n_order[u])
        assert torch.equal(op.order[u, :n], ref.order[u, :n]), u
    # A list out of rank order takes the quadratic rank: the same order.
    op.route_merge(picks.flip(1).contiguous().unsqueeze(0))
    torch.cuda.synchronize()
    assert torch.equal(op.n_order, ref.n_order)
    for u in range(U):
        n = int(ref.n_order[u])
        assert torch.equal(op.order[u, :n], ref.order[u, :n]), u
    op.route_merge(torch.stack([picks, picks, picks]).contiguous())
    torch.cuda.synchronize()
    assert bool((op.n_order >= 0).all()) and bool((op.n_order <= op.width).all())
