"""KV layout control: the explicit gather of the selected rows and the dense
tail into a packed layout, and the probe that compares sparse attention on
the rows in place with attention on the packed copy (the reference's
kernels/cuda_sm90/native_sources/gather.cu and single.py:24-67
``layout_probe``).  A diagnostic beside the decode path, not part of it."""
from __future__ import annotations

import torch

from . import native as nv
from .decode import SparseDecode, default_splits, kv_layout


def gather_kv(k: torch.Tensor, v: torch.Tensor, ids: torch.Tensor, count: torch.Tensor, history: torch.Tensor,
              length: torch.Tensor, packed_rows: int, *, status: torch.Tensor | None = None):
    """Packed K/V [U, packed_rows, d]: unit u's rows ids[u, :count[u]], then
    its tail rows [history[u], length[u]); later slots are left unwritten.
    k, v as for sparse attention ([U, total, d] or slot-major)."""
    U, d = ids.shape[0], k.shape[-1]
    kv_heads, bs, hs, rs, _ = kv_layout(k, v, U, d)
    for t in (count, history, length):
        if t.dtype != torch.int32 or tuple(t.shape) != (U,):
            raise ValueError(f"count/history/length must be int32 [{U}]")
    out_k = torch.empty(U, packed_rows, d, dtype=k.dtype, device=k.device)
    out_v = torch.empty_like(out_k)
    nv.call("pk_gather_kv", k, v, nv.dtype_code(k), kv_heads, bs, hs, rs, ids, ids.stride(0), count, history, length,
            U, d, packed_rows, out_k, out_v, status)
    return out_k, out_v


def _graph_us(fn, reps: int) -> float:
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(reps):
                fn()
    torch.cuda.current_stream().wait_stream(stream)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / reps


@torch.no_grad()
def layout_probe(op: SparseDecode, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, length: torch.Tensor, *,
                 splits: int | None = None, reps: int = 20) -> dict:
    """After ``op.route(q)``: pack the routed rows and the tail, check the
    packing against the rows in place, check that attention over the packed
    copy (identity ids, the same splits) equals the in-place attention bit
    for bit, and time both attentions, the gather, and gather + packed
    attention (CUDA-graph replay of ``reps`` calls each, single.py:54-66)."""
    U, G, d = op.U, op.G, op.d
    # An inactive unit (length 0) has no rows.
    rows = torch.where(length > 0, op.count + (length - op.history).clamp(min=0), torch.zeros_like(op.count)).long()
    P = int(rows.max().item())
    status = torch.zeros(1, dtype=torch.int32, device=q.device)
    pk_, pv_ = gather_kv(k, v, op.ids, op.count, op.history, length, P, status=status)
    nv.check_status(status, "gather_kv")
    kv_heads, bs, hs, rs, _ = kv_layout(k, v, U, d)
    cnt, hist = op.count.tolist(), op.history.tolist()
    for u in range(U):
        c = min(cnt[u], int(rows[u]))   # an inactive unit packs nothing
        h, t = hist[u], int(rows[u]) - c
        pos = torch.cat([op.ids[u, :c].long(), torch.arange(h, h + t, device=q.device)])
        ku = k[u] if k.dim() == 3 else k[u // kv_heads, :, u % kv_heads]
        vu = v[u] if v.dim() == 3 else v[u // kv_heads, :, u % kv_heads]
        if not torch.equal(pk_[u, :c + t], ku[pos]) or not torch.equal(pv_[u, :c + t], vu[pos]):
            raise RuntimeError("packed rows differ from the selection and tail")
    S = splits or default_splits(U, P, q.device)
    ident = torch.arange(max(P, 1), dtype=torch.int32, device=q.device).repeat(U, 1).contiguous()
    p_len = rows.int()
    nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, S)
    ws = op.ws.get(("av", U, G, d, S), nbytes)
    packed_out = torch.empty(U, G, d, dtype=q.dtype, device=q.device)

    def indexed():
        return op.attention(q, k, v, length=length, splits=S)

    def gather():
        nv.call("pk_gather_kv", k, v, nv.dtype_code(k), kv_heads, bs, hs, rs, op.ids, op.ids.stride(0), op.count,
                op.history, length, U, d, P, pk_, pv_, None)

    def prepacked():
        nv.call("pk_sparse_av", q, pk_, pv_, nv.dtype_code(q), 1, pk_.stride(0), 0, pk_.stride(1), ident,
                ident.shape[1], op.count, op.count, p_len, U, G, d, S, ws, nbytes, packed_out, None)

    left = indexed().clone()
    prepacked()
    torch.cuda.synchronize()
    identical = bool(torch.equal(left, packed_out))
    esz = k.element_size()
    moved = int(rows.sum().item()) * d * esz * 2
    times = {name: _graph_us(fn, reps) for name, fn in
             (("indexed_av", indexed), ("prepacked_av", prepacked), ("explicit_gather", gather),
              ("gather_and_av", lambda: (gather(), prepacked())))}
    return dict(rows=int(rows.sum().item()), packed_rows=P, identical=identical, us=times,
                gather_read_GB_s=moved / times["explicit_gather"] / 1e3,
                temporary_bytes=2 * pk_.numel() * pk_.element_size())
