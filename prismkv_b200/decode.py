"""Batched decode-time retrieval over the U units of one layer.

The device operator of the reference (src/prismkv/native8b.py:34-111
``Native8B``; kernels/cuda_sm90/native.py:122-189 ``DecodeOps``), shape-
parametric: a constructor that takes the layer's index and preallocates every
output, ``route(q)`` (router + budgeted union), ``attention(q, k, v)`` (sparse
attention with split-KV), ``__call__`` (both) and ``buffer_bytes()``.  Every
call is asynchronous on the current stream with no host synchronisation, so a
whole decode step can be captured in a CUDA graph.
"""
from __future__ import annotations

import torch

from . import native as nv
from .index import DeviceIndex, SAEParams, budget_limit


def kv_layout(k: torch.Tensor, v: torch.Tensor, U: int, d: int):
    """(kv_heads, batch_stride, head_stride, row_stride, total) of K/V given as
    [U, total, d] (rows of each unit contiguous) or slot-major
    [B, total, H_kv, d] with U = B * H_kv (native8b.py:83-84,92-101 checks)."""
    if k.shape != v.shape or k.stride() != v.stride():
        raise ValueError("K and V must share shape and strides")
    if k.dim() == 3:
        if k.shape[0] != U or k.shape[2] != d:
            raise ValueError(f"K/V[{U},total,{d}] required")
        kv = (1, k.stride(0), 0, k.stride(1), k.shape[1])
    elif k.dim() == 4:
        B, total, Hkv, dd = k.shape
        if B * Hkv != U or dd != d:
            raise ValueError("slot-major K/V[B,total,H_kv,d] with B*H_kv == U required")
        kv = (Hkv, k.stride(0), k.stride(2), k.stride(1), total)
    else:
        raise ValueError("K/V must be 3-D or 4-D")
    if k.stride(-1) != 1:
        raise ValueError("K/V with contiguous head dimension required")
    return kv


def default_splits(U: int, rows: int | None, device) -> int:
    """Split count of the sparse attention for U units of about ``rows`` rows
    each: one wave of two CTAs per SM over all units, at least two 64-row
    tiles per split, and above 8 splits whole clusters of 8 (at most 64),
    the library's own default (pk_sparse_av with splits <= 0) when rows is
    None."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    s = (2 * sms) // max(1, U)
    if rows is not None:
        s = min(s, max(1, (rows + 63) // 64 // 2))
    if s > 8:
        s = min(64, s // 8 * 8)
    return max(1, s)


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              positions: torch.Tensor) -> None:
    """Decode KV append (the reference's ``batch_append``,
    kernels/cuda_sm90/native_sources/av.cu:70-90, called from
    kernels/cuda_sm90/model.py:109-115): slot s's new rows
    k_new/v_new[s] ([H_kv, d], or [d] for a unit-major cache) are written at
    row positions[s] of the caches, given as slot-major [slots, capacity,
    H_kv, d] or unit-major [slots, capacity, d].  positions: int32 [slots] on
    the device; a position outside [0, capacity) leaves its slot untouched.
    Asynchronous on the current stream; graph-capturable."""
    if k_cache.dim() == 4:
        slots, capacity, kv_heads, d = k_cache.shape
    elif k_cache.dim() == 3:
        slots, capacity, d = k_cache.shape
        kv_heads = 1
    else:
        raise ValueError("caches must be [slots, capacity, H_kv, d] or [slots, capacity, d]")
    _, bs, hs, rs, _ = kv_layout(k_cache, v_cache, slots * kv_heads, d)
    for t in (k_new, v_new):
        if t.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
            raise ValueError("new rows and caches must share a dtype")
        if t.numel() != slots * kv_heads * d or not t.is_contiguous():
            raise ValueError(f"new rows must be contiguous [{slots}, {kv_heads}, {d}]")
    if positions.dtype != torch.int32 or tuple(positions.shape) != (slots,) or not positions.is_cuda:
        raise ValueError(f"positions must be a device int32 tensor [{slots}]")
    nv.call("pk_kv_append", k_new, v_new, k_cache, v_cache, nv.dtype_code(k_cache), kv_heads, bs, hs, rs, positions,
            slots, capacity, d)


class SparseDecode:
    def __init__(self, index: DeviceIndex, sae, *, heads_per_unit: int = 4, router: str = "q_activation",
                 query_scale: float = 1.0, query_topk: int | None = None, unique_cap: float | None = None,
                 budget: int | None = None, terms=("count", "mean", "variance"), splits: int | None = None,
                 max_history: int | None = None, workspace: nv.Workspace | None = None,
                 exact_encode: bool = False, route_counts: torch.Tensor | None = None):
        if router not in ("q_activation", "moments"):
            raise ValueError("router must be 'q_activation' or 'moments'")
        if unique_cap is not None and budget is not None:
            raise ValueError("give unique_cap or budget, not both")
        if unique_cap is not None and not 0 <= unique_cap <= 1:
            raise ValueError("unique_cap must be a fraction in [0,1]")
        nv.require_head_dim(index.d)
        self.index = index
        self.sae = SAEParams.of(sae, index.device)
        self.router = router
        self.G = heads_per_unit
        self.U, self.F, self.d = index.U, index.F, index.d
        self.k = min(query_topk or self.sae.query_topk, self.F)
        self.query_scale = float(query_scale)
        self.terms = terms
        self.splits = splits
        self.ws = workspace or nv.Workspace(index.device)
        dev = index.device
        U, G, k = self.U, self.G, self.k
        self.width = G * k if router == "q_activation" else k
        self.max_history = int(max_history or index.history)
        self.order = torch.zeros(U, self.width, dtype=torch.int32, device=dev)
        self.n_order = torch.zeros(U, dtype=torch.int32, device=dev)
        self.features = torch.zeros(U, self.width, dtype=torch.int32, device=dev)
        self.n_features = torch.zeros(U, dtype=torch.int32, device=dev)
        self.raw = torch.zeros(U, dtype=torch.int64, device=dev)
        self.count = torch.zeros(U, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.history = torch.full((U,), index.history, dtype=torch.int32, device=dev)
        self.unique_cap, self.budget = unique_cap, budget
        lim = budget if budget is not None else budget_limit(index.history, unique_cap)
        self.limit = torch.full((U,), int(lim), dtype=torch.int64, device=dev)
        self.id_width = int(min(self.max_history, lim)) if (budget is not None or unique_cap is not None) \
            else self.max_history
        self.ids = torch.zeros(U, max(1, self.id_width), dtype=torch.int32, device=dev)
        self.score = torch.zeros(U, self.F, device=dev) if router == "moments" else None
        self.out = None
        # Bound-filtered routing (tensor-core approximation + exact recompute
        # of the candidates) unless the all-features exact encode is asked for.
        self.prep = (None, None) if exact_encode else self.sae.prepared()
        # Bucket sizes the moments router reads (count term and liveness):
        # the index's own unless given (a sequence shard routes with the
        # whole sequence's sizes).
        if route_counts is not None and (route_counts.dtype != torch.int32 or tuple(route_counts.shape) != (U, self.F)):
            raise ValueError(f"route_counts must be int32 [{U}, {self.F}]")
        self.route_counts = route_counts

    def sync_history(self) -> None:
        """Refresh per-unit history and limits after the index grew (append)."""
        H = self.index.history
        if H > self.max_history:
            raise ValueError("index history exceeds max_history given at construction")
        self.history.fill_(H)
        lim = self.budget if self.budget is not None else budget_limit(H, self.unique_cap)
        self.limit.fill_(int(lim))

    # ---------------------------------------------------------------- route
    def route(self, q: torch.Tensor) -> None:
        """Router + budgeted union for every unit (core.py:142-167)."""
        U, G, d, F, k = self.U, self.G, self.d, self.F, self.k
        if q.shape != (U, G, d) or not q.is_contiguous():
            raise ValueError(f"contiguous Q[{U},{G},{d}] required")
        idx = self.index
        if self.router == "q_activation":
            nbytes = nv.query("pk_route_qact_workspace_bytes", U, G, F, k)
            nv.call("pk_route_qact", q, nv.dtype_code(q), None, U, self.sae.W_enc, self.sae.b_enc, self.prep[0],
                    self.prep[1], self.query_scale, idx.lens, U, G, d, F, k, self.ws.get(("qact", U, G, F, k), nbytes), nbytes, self.order,
                    self.n_order, self.width, None, None)
        else:
            bits = ((nv.PK_TERM_COUNT if "count" in self.terms else 0)
                    | (nv.PK_TERM_MEAN if "mean" in self.terms else 0)
                    | (nv.PK_TERM_VARIANCE if "variance" in self.terms else 0))
            nbytes = nv.query("pk_route_moments_workspace_bytes", U, G, F)
            counts = self.route_counts if self.route_counts is not None else idx.lens
            nv.call("pk_route_moments", q, nv.dtype_code(q), idx.mean, idx.var, counts, bits, U, G, d, F, k,
                    self.ws.get(("moments", U, G, F), nbytes), nbytes, self.score, self.order, self.n_order,
                    self.width)
        self.union()

    def union(self) -> None:
        """The budgeted union of the routed order (core.py:152-164) for every
        unit: ids, accepted buckets, raw sizes and counts."""
        idx = self.index
        nv.call("pk_union", idx.offsets, idx.lens, idx.ids, idx.ids.stride(0), self.order, self.n_order, self.width,
                self.history, self.limit, self.U, self.F, self.max_history, self.ids, self.ids.shape[1], self.count,
                self.features, self.n_features, self.raw, self.status)

    # ---------------------------------------------- feature-sharded routing
    def route_shard_picks(self, q: torch.Tensor, f_lo: int, f_hi: int, picks: torch.Tensor) -> torch.Tensor:
        """q_activation routing over the features [f_lo, f_hi) only: each
        head's positive top-k among them, exact, in rank order, as int32
        (value bits, feature id) pairs in picks [U*G, k, 2] (unused slots
        (0, INT32_MAX)).  The first half of the feature-sharded route; the
        picks of every feature range go to route_merge."""
        U, G, d, F, k = self.U, self.G, self.d, self.F, self.k
        if self.router != "q_activation" or self.prep[0] is None:
            raise ValueError("feature-sharded routing needs the bound-filtered q_activation router")
        if q.shape != (U, G, d) or not q.is_contiguous():
            raise ValueError(f"contiguous Q[{U},{G},{d}] required")
        if tuple(picks.shape) != (U * G, k, 2) or picks.dtype != torch.int32 or not picks.is_contiguous():
            raise ValueError(f"picks must be a contiguous int32 [{U * G}, {k}, 2] tensor")
        nbytes = nv.query("pk_route_qact_shard_workspace_bytes", U, G, f_hi - f_lo, k)
        nv.call("pk_route_qact_shard", q, nv.dtype_code(q), self.sae.W_enc, self.sae.b_enc, self.prep[0], self.prep[1],
                self.query_scale, U, G, d, F, k, f_lo, f_hi,
                self.ws.get(("qact_shard", U, G, f_hi - f_lo, k), nbytes), nbytes, picks)
        return picks

    def route_merge(self, gathered: torch.Tensor) -> None:
        """The second half of the feature-sharded route: gathered [P, U*G,
        k, 2] holds the picks of P disjoint feature ranges covering all F
        features; every head's exact top-k over them, then the unit's
        normalisation, aggregation and order (core.py:134-139), equal to the
        unsharded route's.  Bucket liveness comes from this index."""
        U, G, F, k = self.U, self.G, self.F, self.k
        P = gathered.shape[0]
        if tuple(gathered.shape[1:]) != (U * G, k, 2) or gathered.dtype != torch.int32 or not gathered.is_contiguous():
            raise ValueError(f"gathered picks must be a contiguous int32 [P, {U * G}, {k}, 2] tensor")
        nbytes = nv.query("pk_route_qact_merge_workspace_bytes", U, G, k)
        nv.call("pk_route_qact_merge", gathered, P, self.index.lens, U, G, F, k,
                self.ws.get(("qact_merge", U, G, k), nbytes), nbytes, self.order, self.n_order, self.width, None)

    # ------------------------------------------------------------ attention
    def attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, length=None, splits=None,
                  partial: torch.Tensor | None = None, append=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sparse attention over the routed ids plus the dense tail.

        k, v: [U, total, d] (rows of each unit contiguous) or slot-major
        [B, total, H_kv, d] with U = B * H_kv.  length: rows per unit
        (history + tail), an int or an int32 tensor [U]; default all rows.
        With ``partial`` ([U*G, d+2] fp32) the per-head (m, l, o) partial is
        written instead of the output (for the sequence-sharded merge).
        ``append=(k_new, v_new)`` (contiguous, U*d elements each, unit u =
        slot * H_kv + head) fuses the decode KV append: each unit's new rows
        are attended as row length[u] - 1, the newest tail row, and written
        into k and v there (one launch; as kv_append then attention).
        ``out`` (contiguous [U, G, d] of Q's dtype) receives the output
        instead of the operator's own buffer."""
        U, G, d = self.U, self.G, self.d
        if k.dtype != q.dtype or v.dtype != q.dtype:
            raise ValueError("Q, K and V must share a dtype")
        kv_heads, bs, hs, rs, total = kv_layout(k, v, U, d)
        if total < self.index.history:
            raise ValueError("K/V shorter than the indexed history")
        if length is None:
            length = total
        if isinstance(length, int):
            if not self.index.history <= length <= total and length != 0:
                raise ValueError("length must lie in [history, K/V rows] (0 marks an inactive unit)")
            lt = self._length_buf(length)
        else:
            # Device lengths are the caller's contract: each in [history, rows] or 0.
            if length.dtype != torch.int32 or tuple(length.shape) != (U,):
                raise ValueError(f"length tensor must be int32 [{U}]")
            lt = length
        S = splits or self.splits or 0
        if S <= 0:
            # Rows per unit: at most the id width plus the tail.
            S = default_splits(U, self.id_width + max(0, total - self.index.history), q.device)
        nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, S)
        if partial is not None:
            out = None
        elif out is not None:
            if tuple(out.shape) != (U, G, d) or out.dtype != q.dtype or not out.is_contiguous():
                raise ValueError(f"out must be a contiguous [{U},{G},{d}] {q.dtype} tensor")
        else:
            if self.out is None or self.out.dtype != q.dtype:
                self.out = torch.empty(U, G, d, dtype=q.dtype, device=q.device)
            out = self.out
        args = (q, k, v, nv.dtype_code(q), kv_heads, bs, hs, rs, self.ids, self.ids.shape[1], self.count,
                self.history, lt, U, G, d, S, self.ws.get(("av", U, G, d, S), nbytes), nbytes, out, partial)
        if append is None:
            nv.call("pk_sparse_av", *args)
        else:
            k_new, v_new = append
            for t in (k_new, v_new):
                if t.dtype != q.dtype or t.numel() != U * d or not t.is_contiguous() or not t.is_cuda:
                    raise ValueError(f"append rows must be contiguous device tensors of {U}x{d} {q.dtype}")
            nv.call("pk_sparse_av_append", *args, k_new, v_new)
        return out if partial is None else partial

    def _length_buf(self, n: int) -> torch.Tensor:
        buf = getattr(self, "_len", None)
        if buf is None:
            buf = self._len = torch.empty(self.U, dtype=torch.int32, device=self.index.device)
            self._len_val = None
        if self._len_val != n:
            buf.fill_(n)
            self._len_val = n
        return buf

    def __call__(self, q, k, v, **kwargs):
        self.route(q)
        return self.attention(q, k, v, **kwargs)

    def check(self) -> None:
        """Synchronise and raise on any condition the kernels flagged."""
        nv.check_status(self.status, "decode")

    def buffer_bytes(self) -> dict:
        """Live tensors owned here (index, K/V and model weights excluded)."""
        out = {name: t.numel() * t.element_size() for name, t in vars(self).items() if isinstance(t, torch.Tensor)}
        out["workspace"] = self.ws.bytes()
        return out
