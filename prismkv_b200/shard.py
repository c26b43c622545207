"""Sequence-sharded decode: the KV cache and the bucket lists of every unit
split along the token axis over the ranks of a process group.

Rank r of P owns tokens [lo_r, hi_r) of the history (``token_ranges``); the
dense tail of generated tokens lives on the last rank.  One decode step is:

1. routing, replicated on every rank (the q_activation scores depend only on
   the query and the SAE, core.py:131-139; bucket liveness is local);
2. the union of the routed buckets' shard-local lists (core.py:152-164) with
   the per-shard budget ``budget // P`` -- in the unbudgeted mode the shards'
   unions are exactly the global union cut at the shard boundaries;
3. sparse attention over the shard's rows, exported as the per-head
   log-sum-exp partial (m, l, o[d]);
4. one all-gather of the P partials (NCCL over NVLink on GPUs) and the exact
   log-sum-exp merge on every rank (pk_lse_merge), the split-KV merge of the
   reference's kernels (kernels/ppu_8b/av_tuned.cu) applied across ranks.

There is no other collective on the path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import native as nv
from .decode import SparseDecode
from .index import DeviceIndex


def token_ranges(N: int, P: int) -> list:
    """Contiguous shard ranges [lo, hi) covering tokens 0..N-1 (sizes differ
    by at most one; rank order = token order = flat-index order)."""
    if P < 1 or N < 0:
        raise ValueError("P >= 1 and N >= 0 required")
    return [(r * N // P, (r + 1) * N // P) for r in range(P)]


def shard_index(index: DeviceIndex, lo: int, hi: int) -> DeviceIndex:
    """The part of ``index`` that covers tokens [lo, hi), with token ids made
    relative to lo.  Each bucket's entries in the range form one contiguous,
    still ascending run of its list; counts are the shard-local list sizes.
    Moments are not carried (the sharded path routes with q_activation)."""
    if not 0 <= lo <= hi <= index.history:
        raise ValueError("shard range must lie within the index history")
    U, F, dev = index.U, index.F, index.device
    lens = index.lens.long()
    flat_lens = lens.flatten()
    total = int(flat_lens.sum().item())
    new_lens = torch.zeros(U * F, dtype=torch.long, device=dev)
    out = DeviceIndex(U, F, index.d, 1, dev, moments=False)
    if total:
        seg = torch.repeat_interleave(torch.arange(U * F, device=dev), flat_lens)
        uu = seg // F
        start = torch.cumsum(flat_lens, 0) - flat_lens
        slot = torch.arange(total, device=dev) - torch.repeat_interleave(start, flat_lens)
        tok = index.ids[uu, index.offsets.long()[uu, seg % F] + slot].long()
        keep = (tok >= lo) & (tok < hi)
        new_lens.scatter_add_(0, seg[keep], torch.ones_like(seg[keep]))
        lens_u = new_lens.view(U, F)
        offs = torch.zeros(U, F + 1, dtype=torch.long, device=dev)
        offs[:, 1:] = torch.cumsum(lens_u, 1)
        cap = int(offs[:, -1].max().item())
        ids = torch.zeros(U, max(1, cap), dtype=torch.int32, device=dev)
        k_seg, k_tok = seg[keep], tok[keep]
        k_start = torch.cumsum(new_lens, 0) - new_lens
        k_slot = torch.arange(k_seg.numel(), device=dev) - k_start[k_seg]
        ids[k_seg // F, offs[k_seg // F, k_seg % F] + k_slot] = (k_tok - lo).int()
        out.offsets = offs.int()
        out.lens = lens_u.int()
        out.ids = ids
    out.center.copy_(index.center)
    out.history = hi - lo
    return out


def gather_partials(part: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather of every rank's [U*G, d+2] partial into out[P, U*G, d+2]
    (rank order).  NCCL gathers into the flat buffer; gloo (CPU) by list.
    Without a process group there is one shard and nothing to exchange."""
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    if out.shape[0] != P or out.shape[1:] != part.shape:
        raise ValueError("out must be [world, *part.shape]")
    if P == 1:
        out[0].copy_(part)
        return out
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, part, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), part, group=group)
    return out


def shard_budget(budget, P: int):
    """Per-shard union budget: floor(budget / P) (None stays unbudgeted)."""
    return None if budget is None else int(budget) // P


class ShardedDecode:
    """Decode over this rank's sequence shard of every unit, merged across
    the group.  ``local_index`` covers this rank's token range (built on the
    shard, or cut from a full index by ``shard_index``); K/V passed to the
    call hold the shard's rows, the last rank's followed by the dense tail."""

    def __init__(self, local_index: DeviceIndex, sae, *, group=None, heads_per_unit: int = 4,
                 query_scale: float = 1.0, query_topk: int | None = None, budget: int | None = None,
                 splits: int | None = None, max_history: int | None = None,
                 workspace: nv.Workspace | None = None):
        self.group = group
        init = dist.is_initialized()
        self.P = dist.get_world_size(group) if init else 1
        self.rank = dist.get_rank(group) if init else 0
        self.budget = budget
        self.op = SparseDecode(local_index, sae, heads_per_unit=heads_per_unit, router="q_activation",
                               query_scale=query_scale, query_topk=query_topk,
                               budget=shard_budget(budget, self.P), splits=splits, max_history=max_history,
                               workspace=workspace)
        U, G, d = self.op.U, self.op.G, self.op.d
        dev = local_index.device
        self.part = torch.empty(U * G, d + 2, dtype=torch.float32, device=dev)
        self.gathered = torch.empty(self.P, U * G, d + 2, dtype=torch.float32, device=dev)
        self.out = None

    @property
    def is_tail_rank(self) -> bool:
        return self.rank == self.P - 1

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, length=None) -> torch.Tensor:
        U, G, d = self.op.U, self.op.G, self.op.d
        self.op.route(q)
        self.op.attention(q, k, v, length=length, partial=self.part)
        gather_partials(self.part, self.gathered, self.group)
        if self.out is None or self.out.dtype != q.dtype:
            self.out = torch.empty(U, G, d, dtype=q.dtype, device=q.device)
        nv.call("pk_lse_merge", self.gathered, self.P, U * G, d, self.out, nv.dtype_code(q))
        return self.out

    def check(self) -> None:
        self.op.check()
