"""GPU tests of the sequence-sharded build with the exact global BatchTopK
(prismkv_b200.shard: ShardBuilder, drive_build, global_center,
build_sharded).  The shards' global center is bit-identical to the
one-device center, and every shard's index (lens and bucket lists) equals the
one-device index of the whole sequence cut at the shard (shard_index): the
memberships of the reference's single build, core.py:13-26, over all N
tokens.  P shards are emulated in one process (the collectives become sums,
maxima and stacks over the shards); with two GPUs the same build runs as two
NCCL ranks."""
import os
import socket

import pytest
import torch

from gen import bf16_round

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prismkv_b200
    return prismkv_b200


def make(seed, U=4, N=16384, d=128, C=64, F=1024):
    g = torch.Generator().manual_seed(seed)
    centers = torch.randn(U, C, d, generator=g)
    cid = torch.randint(0, C, (U, N), generator=g)
    keys = centers[torch.arange(U)[:, None], cid] + 0.3 * torch.randn(U, N, d, generator=g)
    keys = torch.from_numpy(bf16_round(keys.numpy()))
    W = torch.randn(F, d, generator=g) / d ** 0.5
    b = 0.02 * torch.randn(F, generator=g)
    return keys.cuda().bfloat16(), W.cuda(), b.cuda()


def pairs(idx, u):
    """(bucket, token) pairs of unit u as sorted int64 codes."""
    offs = idx.offsets[u].long()
    lens = idx.lens[u].long()
    F = lens.numel()
    tot = int(lens.sum())
    if tot == 0:
        return torch.empty(0, dtype=torch.int64, device=lens.device)
    seg = torch.repeat_interleave(torch.arange(F, device=lens.device), lens)
    start = torch.cumsum(lens, 0) - lens
    slot = torch.arange(tot, device=lens.device) - torch.repeat_interleave(start, lens)
    ids = idx.ids[u, offs[seg] + slot].long()
    return seg * (1 << 32) + ids


def emulated_collectives():
    def allreduce_sum(ts):
        tot = torch.stack([t.clone() for t in ts]).sum(0).to(ts[0].dtype)
        for t in ts:
            t.copy_(tot)

    def allreduce_max(ts):
        tot = torch.stack([t.clone() for t in ts]).max(0).values
        for t in ts:
            t.copy_(tot)

    return allreduce_sum, allreduce_max, lambda ts: torch.stack(ts)


@pytest.mark.parametrize("P", [2, 4])
def test_emulated_sharded_build_equals_global_build(pk, P):
    from prismkv_b200.shard import ShardBuilder, drive_build, global_center, shard_index, token_ranges
    K, W, b = make(21)
    U, N = K.shape[0], K.shape[1]
    sae = pk.SAEParams(W, b, key_mean=8, query_topk=16)
    full = pk.DeviceIndex.build(K, sae, 1.0, moments=False)
    assert full.encode_path == "bounds"
    ranges = token_ranges(N, P)
    center = global_center([K[:, lo:hi] for lo, hi in ranges], N)
    assert torch.equal(center, full.center)
    builders = [ShardBuilder(K[:, lo:hi], sae, 1.0, lo=lo, N_total=N, center=center) for lo, hi in ranges]
    shards = drive_build(builders, *emulated_collectives())
    for (lo, hi), got in zip(ranges, shards):
        want = shard_index(full, lo, hi)
        assert got.history == hi - lo
        assert torch.equal(got.lens, want.lens)
        for u in range(U):
            assert torch.equal(pairs(got, u), pairs(want, u)), (lo, u)


def test_sharded_union_equals_global_union(pk):
    """Decoding on the sharded indexes selects the global union cut at each
    shard (unbudgeted), as with indexes cut from the one-device build."""
    from prismkv_b200.shard import ShardBuilder, drive_build, global_center, token_ranges
    K, W, b = make(22, U=4)
    U, N, G = K.shape[0], K.shape[1], 4
    sae = pk.SAEParams(W, b, key_mean=8, query_topk=16)
    full = pk.DeviceIndex.build(K, sae, 1.0, moments=False)
    g = torch.Generator().manual_seed(5)
    Q = torch.from_numpy(bf16_round(torch.randn(U, G, 128, generator=g).numpy())).cuda().bfloat16().contiguous()
    ref = pk.SparseDecode(full, sae, heads_per_unit=G, unique_cap=None)
    ref.route(Q)
    ranges = token_ranges(N, 2)
    center = global_center([K[:, lo:hi] for lo, hi in ranges], N)
    shards = drive_build([ShardBuilder(K[:, lo:hi], sae, 1.0, lo=lo, N_total=N, center=center) for lo, hi in ranges],
                         *emulated_collectives())
    for (lo, hi), idx in zip(ranges, shards):
        op = pk.SparseDecode(idx, sae, heads_per_unit=G, unique_cap=None)
        op.route(Q)
        for u in range(U):
            glob = ref.ids[u, :int(ref.count[u])].long()
            want = glob[(glob >= lo) & (glob < hi)] - lo
            assert torch.equal(op.ids[u, :int(op.count[u])].long(), want)


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
        from prismkv_b200.shard import build_sharded, shard_index, token_ranges
        K, W, b = (t.to(dev) for t in make(23))
        U, N = K.shape[0], K.shape[1]
        sae = pk.SAEParams(W, b, key_mean=8, query_topk=16)
        lo, hi = token_ranges(N, world)[rank]
        got = build_sharded(K[:, lo:hi].contiguous(), sae, 1.0, lo=lo, N_total=N)
        want = shard_index(pk.DeviceIndex.build(K, sae, 1.0, moments=False), lo, hi)
        ok = torch.equal(got.lens, want.lens) and all(torch.equal(pairs(got, u), pairs(want, u)) for u in range(U))
        q.put((rank, bool(ok)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_nccl_sharded_build(pk):
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
    assert all(res.values()), res
