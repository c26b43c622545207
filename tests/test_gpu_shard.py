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


def _rank_main(rank, world, port, q):
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
        sd = ShardedDecode(shard_index(idx, lo, hi), sae, heads_per_unit=G, budget=None)
        rows = slice(lo, hi + c["tail"]) if sd.is_tail_rank else slice(lo, hi)
        out = sd(Q, K[:, rows].contiguous(), V[:, rows].contiguous()).float()
        ref = pk.SparseDecode(idx, sae, heads_per_unit=G, unique_cap=None)(Q, K, V).float()
        torch.cuda.synchronize()
        err = float((out - ref).norm() / ref.norm())
        q.put((rank, err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_nccl_sharded_decode():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(e < 2e-2 for e in res.values()), res
