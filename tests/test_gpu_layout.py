"""GPU tests of the KV layout diagnostic (prismkv_b200.layout): the packed
copy holds exactly the routed rows and then the dense tail, attention over it
with identity ids equals the in-place sparse attention bit for bit (as the
reference's layout probe asserts, single.py:42-53), for unit-major and
slot-major K/V and both dtypes; a packed buffer too short is flagged."""
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


def make(seed, dtype, U=8, N=5000, tail=37, d=128, C=48, F=1024, G=4, k=16):
    g = torch.Generator().manual_seed(seed)
    centers = torch.randn(U, C, d, generator=g)
    cid = torch.randint(0, C, (U, N + tail), generator=g)
    keys = centers[torch.arange(U)[:, None], cid] + 0.3 * torch.randn(U, N + tail, d, generator=g)
    vals = torch.randn(U, N + tail, d, generator=g)
    q = centers[torch.arange(U)[:, None], torch.randint(0, C, (U, G), generator=g)] + 0.3 * torch.randn(U, G, d,
                                                                                                          generator=g)
    W = torch.randn(F, d, generator=g) / d ** 0.5
    if dtype == torch.bfloat16:
        keys, vals, q = (torch.from_numpy(bf16_round(x.numpy())) for x in (keys, vals, q))
    dev = torch.device("cuda")
    return (keys.to(dev, dtype), vals.to(dev, dtype), q.to(dev, dtype).contiguous(), W.to(dev), N, tail, G, k)


@pytest.mark.parametrize("dtype,slot_major,budget", [(torch.bfloat16, False, 512), (torch.bfloat16, True, None),
                                                     (torch.float32, False, 256)])
def test_packed_attention_is_identical(pk, dtype, slot_major, budget):
    from prismkv_b200.layout import layout_probe
    K, V, Q, W, N, tail, G, k = make(3, dtype)
    U = K.shape[0]
    sae = pk.SAEParams(W, torch.zeros(W.shape[0], device=W.device), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=budget)
    op.route(Q)
    length = torch.full((U,), N + tail, dtype=torch.int32, device=K.device)
    length[1] = 0          # an inactive unit: no rows
    length[2] = N + 1      # a one-row tail
    if slot_major:
        # [B, total, H_kv, d] with B * H_kv = U (H_kv = 2).
        K = K.view(U // 2, 2, N + tail, -1).transpose(1, 2).contiguous()
        V = V.view(U // 2, 2, N + tail, -1).transpose(1, 2).contiguous()
    res = layout_probe(op, Q, K, V, length, reps=3)
    assert res["identical"]
    counts = op.count.tolist()
    want = sum(counts[u] + max(int(length[u]) - N, 0) for u in range(U) if int(length[u]) > 0)
    assert res["rows"] == want
    assert all(t > 0 for t in res["us"].values())


def test_short_packed_buffer_is_flagged(pk):
    from prismkv_b200 import native as nv
    from prismkv_b200.layout import gather_kv
    K, V, Q, W, N, tail, G, k = make(4, torch.bfloat16, U=4)
    U = K.shape[0]
    ids = torch.arange(64, dtype=torch.int32, device=K.device).repeat(U, 1).contiguous()
    count = torch.full((U,), 64, dtype=torch.int32, device=K.device)
    hist = torch.full((U,), N, dtype=torch.int32, device=K.device)
    length = torch.full((U,), N + tail, dtype=torch.int32, device=K.device)
    status = torch.zeros(1, dtype=torch.int32, device=K.device)
    pk_, pv_ = gather_kv(K, V, ids, count, hist, length, 64 + tail - 1, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & nv.STATUS_OUT_FULL
    # The slots that fit are still the right rows.
    assert torch.equal(pk_[:, :64], K[:, :64])
    assert torch.equal(pv_[:, 64:], V[:, N:N + tail - 1])
