"""Host-side logic of the sequence-sharded decode, on the CPU: shard ranges,
cutting an index into token shards, the all-gather of partials over a gloo
group of two ranks, and -- through the oracle -- the two facts the sharded
path rests on: the unbudgeted union of a global index is the union of its
shards' unions, and the log-sum-exp merge of per-shard partials is the
attention over the whole selection."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gen import bf16_round, unit_case


def test_token_ranges_partition():
    from prismkv_b200.shard import token_ranges
    for N in (0, 1, 7, 1000, 1 << 20):
        for P in (1, 2, 3, 8):
            r = token_ranges(N, P)
            assert len(r) == P and r[0][0] == 0 and r[-1][1] == N
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            sizes = [hi - lo for lo, hi in r]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        token_ranges(10, 0)


def random_lists(rs, U, F, N, mean_len):
    out = []
    for _ in range(U):
        lu = []
        for _ in range(F):
            n = rs.randint(0, 2 * mean_len + 1)
            lu.append(np.sort(rs.choice(N, size=min(n, N), replace=False)).astype(np.int64))
        out.append(lu)
    return out


def test_shard_index_cuts_every_bucket():
    from prismkv_b200.index import from_lists
    from prismkv_b200.shard import shard_index, token_ranges
    rs = np.random.RandomState(0)
    U, F, N, d = 3, 40, 500, 8
    lists = random_lists(rs, U, F, N, 12)
    idx = from_lists(lists, N, d, "cpu")
    rebuilt = [[[] for _ in range(F)] for _ in range(U)]
    for lo, hi in token_ranges(N, 3):
        sh = shard_index(idx, lo, hi)
        assert sh.history == hi - lo
        for u in range(U):
            got = sh.lists(u)
            for f in range(F):
                want = lists[u][f][(lists[u][f] >= lo) & (lists[u][f] < hi)] - lo
                assert np.array_equal(got[f].numpy(), want)
                rebuilt[u][f].extend((got[f].numpy() + lo).tolist())
    for u in range(U):
        for f in range(F):
            assert rebuilt[u][f] == lists[u][f].tolist()


def test_shard_of_empty_index():
    from prismkv_b200.index import from_lists
    from prismkv_b200.shard import shard_index
    idx = from_lists([[[] for _ in range(5)]], 10, 4, "cpu")
    sh = shard_index(idx, 3, 7)
    assert sh.history == 4 and int(sh.lens.sum()) == 0


def test_unbudgeted_union_is_union_of_shard_unions(oracle):
    rs = np.random.RandomState(3)
    N, F = 2000, 64
    lists = random_lists(rs, 1, F, N, 30)[0]
    idx = oracle.index_from_lists(N, np.zeros(4, np.float32), lists)
    order = rs.permutation(F)[:20].astype(np.int64)
    full = oracle.select_from_order(order, idx, oracle.budget_limit(N, None))[0]
    from prismkv_b200.shard import token_ranges
    parts = []
    for lo, hi in token_ranges(N, 4):
        sl = [x[(x >= lo) & (x < hi)] - lo for x in lists]
        sidx = oracle.index_from_lists(hi - lo, np.zeros(4, np.float32), sl)
        ids = oracle.select_from_order(order, sidx, oracle.budget_limit(hi - lo, None))[0]
        parts.append(ids + lo)
    assert np.array_equal(np.concatenate(parts), full)


def partial_np(q, keys, vals, rows):
    """(m, l, o) of softmax(q k^T / sqrt(d)) v over `rows`, natural log."""
    s = (q.astype(np.float64) @ keys[rows].T.astype(np.float64)) / np.sqrt(q.shape[-1])
    if s.shape[1] == 0:
        return np.full(q.shape[0], -np.inf), np.zeros(q.shape[0]), np.zeros(q.shape)
    m = s.max(1)
    p = np.exp(s - m[:, None])
    return m, p.sum(1), p @ vals[rows].astype(np.float64)


def test_lse_merge_of_shard_partials_is_full_attention(oracle):
    c = unit_case(11, n=1200, d=128, clusters=16, F=256, G=4, tail=9, bf16=True, key_mean=8)
    keys, vals, q = c["keys"], c["values"], c["q"]
    N = c["history"]
    rs = np.random.RandomState(5)
    ids = np.sort(rs.choice(N, size=300, replace=False)).astype(np.int64)
    ref = oracle.attend(q, keys, vals, ids, N)
    from prismkv_b200.shard import token_ranges
    P = 3
    ms, ls, os_ = [], [], []
    for r, (lo, hi) in enumerate(token_ranges(N, P)):
        rows = ids[(ids >= lo) & (ids < hi)]
        if r == P - 1:
            rows = np.concatenate([rows, np.arange(N, keys.shape[0])])
        m, l, o = partial_np(q, keys, vals, rows)
        ms.append(m); ls.append(l); os_.append(o)
    M = np.max(ms, 0)
    w = [np.where(np.isneginf(m), 0.0, np.exp(m - M)) for m in ms]
    L = sum(wi * li for wi, li in zip(w, ls))
    O = sum(wi[:, None] * oi for wi, oi in zip(w, os_))
    out = O / L[:, None]
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from prismkv_b200.shard import gather_partials
        part = torch.full((6, 10), float(rank + 1))
        part[:, 0] = -float("inf") if rank == 0 else 0.5
        out = torch.empty(world, 6, 10)
        gather_partials(part, out)
        ok = all(torch.equal(out[r, :, 1:], torch.full((6, 9), float(r + 1))) for r in range(world))
        ok = ok and bool(torch.isneginf(out[0, :, 0]).all()) and bool((out[1, :, 0] == 0.5).all())
        with pytest.raises(ValueError):
            gather_partials(part, torch.empty(world + 1, 6, 10))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_gather_partials_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}


def test_shard_budget():
    from prismkv_b200.shard import shard_budget
    assert shard_budget(None, 4) is None
    assert shard_budget(8192, 8) == 1024
    assert shard_budget(10, 3) == 3


def test_unit_views_share_storage():
    from prismkv_b200.index import from_lists
    rs = np.random.RandomState(1)
    lists = random_lists(rs, 4, 16, 300, 6)
    idx = from_lists(lists, 300, 8, "cpu")
    sub = idx.units(1, 3)
    assert sub.U == 2 and sub.history == idx.history
    assert sub.ids.data_ptr() == idx.ids[1].data_ptr()
    for u in range(2):
        assert all(torch.equal(a, b) for a, b in zip(sub.lists(u), idx.lists(u + 1)))
    with pytest.raises(ValueError):
        idx.units(2, 2)
