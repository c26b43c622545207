"""The allocation-free sparse-attention entry point, checked against the
workspace entry point it mirrors and against the CPU oracle.

pk_sparse_av_noalloc serves callers that cannot allocate device memory -- a
host whose device memory is all pre-reserved for its own pool, or a
foreign-language caller of the C ABI without a device allocator -- by keeping
its split scratch in a library-owned device array.  Both entry points run the
same kernel with the same split count on the same inputs, so their outputs
must be bitwise equal; each case calls the allocation-free one twice in a
row, because the shared array keeps the previous call's partials and arrival
counters.  The cases cover the paths that read and write that array: fp32
(global partials merged by the unit's last CTA), bf16 with more than eight
heads and more splits than one cluster holds (the same last-CTA merge), and
bf16 with the on-chip cluster merge.  The oracle's attend (core.py:170-183)
bounds the error: 1e-3 relative L2 for fp32, 2e-2 for bf16.  The file sorts
last so that pytest collects it after every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = {"f32": 1e-3, "bf16": 2e-2}

# (dtype, heads per unit, splits)
CASES = [("f32", 4, 12), ("bf16", 12, 20), ("bf16", 4, 12), ("bf16", 4, 6)]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("dtype,G,splits", CASES)
def test_noalloc_sparse_attention_equals_workspace_entry_point(oracle, dtype, G, splits):
    from prismkv_b200 import build as b
    b.build()
    from prismkv_b200 import native as nv
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    dev = torch.device("cuda")
    dt, code = (torch.float32, nv.PK_F32) if dtype == "f32" else (torch.bfloat16, nv.PK_BF16)
    g = torch.Generator(device=dev).manual_seed(5 + G + splits)
    U, d, H, tail, sel = 16, 128, 4096, 24, 700
    total = H + tail
    K = torch.randn(U, total, d, device=dev, generator=g).to(dt)
    V = torch.randn(U, total, d, device=dev, generator=g).to(dt)
    Q = torch.randn(U, G, d, device=dev, generator=g).to(dt)
    ids = torch.stack([torch.randperm(H, device=dev, generator=g)[:sel].sort().values for _ in range(U)]).int()
    count = torch.full((U,), sel, dtype=torch.int32, device=dev)
    count[3] = 0                       # a unit with only the dense tail
    hist = torch.full((U,), H, dtype=torch.int32, device=dev)
    length = torch.full((U,), total, dtype=torch.int32, device=dev)
    length[5] = 0                      # an inactive unit
    args = (Q, K, V, code, 1, K.stride(0), 0, K.stride(1), ids, ids.shape[1], count, hist, length, U, G, d, splits)
    nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, splits)
    assert nbytes <= 4 << 20          # PK_SPARSE_AV_NOALLOC_SCRATCH_BYTES
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    ref = torch.empty(U, G, d, dtype=dt, device=dev)
    nv.call("pk_sparse_av", *args, ws, nbytes, ref, None)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full((U, G, d), float("nan"), dtype=dt, device=dev)
        nv.call("pk_sparse_av_noalloc", *args, out)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.count_nonzero(out[5]).item() == 0
    # Against the oracle, unit by unit (the inactive unit is all zeros).
    qh, kh, vh = Q.float().cpu().numpy(), K.float().cpu().numpy(), V.float().cpu().numpy()
    ih, ch = ids.long().cpu().numpy(), count.cpu().numpy()
    got = out.float().cpu().numpy()
    for u in range(U):
        if u == 5:
            continue
        want = oracle.attend(qh[u], kh[u], vh[u], ih[u, :ch[u]], H)
        assert rel_l2(got[u], want) < TOL[dtype], (u, rel_l2(got[u], want))


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from prismkv_b200 import native as nv
    fn = nv.lib().pk_sparse_av_noalloc
    # 1024 units x 4 heads x 64 splits of (m, l, o[128]) needs ~136 MB > 4 MiB.
    rc = fn(1, 1, 1, nv.PK_BF16, 1, 0, 0, 128, 1, 1, 1, 1, 1, 1024, 4, 128, 64, 1, 0)
    assert rc == -4
