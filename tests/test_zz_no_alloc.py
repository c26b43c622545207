"""The allocation-free sparse-attention entry point, checked against the
workspace entry point it mirrors.

pk_sparse_av_noalloc serves callers that cannot allocate device memory -- a
host whose device memory is all pre-reserved for its own pool, or a
foreign-language caller of the C ABI without a device allocator -- by keeping
its split scratch in a library-owned device array.  This test calls both
entry points through the C ABI on the same inputs and requires the same
output (within the bf16 attention tolerance the other tests use, 2e-2
relative L2) on two calls in a row, since the shared array keeps the previous
call's contents.  It lives in its own file so that pytest collects it last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_noalloc_sparse_attention_matches_workspace_entry_point():
    from prismkv_b200 import build as b
    b.build()
    from prismkv_b200 import native as nv
    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(5)
    U, G, d, H, tail, sel = 16, 4, 128, 4096, 24, 700
    total = H + tail
    K = torch.randn(U, total, d, device=dev, generator=g).bfloat16()
    V = torch.randn(U, total, d, device=dev, generator=g).bfloat16()
    Q = torch.randn(U, G, d, device=dev, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(H, device=dev, generator=g)[:sel].sort().values for _ in range(U)]).int()
    count = torch.full((U,), sel, dtype=torch.int32, device=dev)
    count[3] = 0                       # a unit with only the dense tail
    hist = torch.full((U,), H, dtype=torch.int32, device=dev)
    length = torch.full((U,), total, dtype=torch.int32, device=dev)
    length[5] = 0                      # an inactive unit
    splits = 12
    args = (Q, K, V, nv.PK_BF16, 1, K.stride(0), 0, K.stride(1), ids, ids.shape[1], count, hist, length, U, G, d,
            splits)
    nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, splits)
    assert nbytes <= 4 << 20
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    ref = torch.empty(U, G, d, dtype=torch.bfloat16, device=dev)
    nv.call("pk_sparse_av", *args, ws, nbytes, ref, None)
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full((U, G, d), float("nan"), dtype=torch.bfloat16, device=dev)
        nv.call("pk_sparse_av_noalloc", *args, out)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_l2(out.float().cpu().numpy(), ref.float().cpu().numpy()) < TOL_BF16
        assert torch.count_nonzero(out[5]).item() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from prismkv_b200 import native as nv
    fn = nv.lib().pk_sparse_av_noalloc
    # 1024 units x 4 heads x 64 splits of (m, l, o[128]) needs ~136 MB > 4 MiB.
    rc = fn(1, 1, 1, nv.PK_BF16, 1, 0, 0, 128, 1, 1, 1, 1, 1, 1024, 4, 128, 64, 1, 0)
    assert rc == -4
