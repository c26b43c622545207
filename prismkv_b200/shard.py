"""Sequence-sharded decode: the KV cache and the bucket lists of every unit
split along the token axis over the ranks of a process group.

Rank r of P owns tokens [lo_r, hi_r) of the history (``token_ranges``); the
dense tail of generated tokens lives on the last rank.  One decode step is:

1. routing, replicated on every rank by default (the q_activation scores
   depend only on the query and the SAE, core.py:131-139, bucket liveness
   being local; the moments router, core.py:117-130, reads the whole
   sequence's bucket moments and sizes, attach_global_moments, so every rank
   takes the same buckets).  With split_route=True, q_activation is split by
   features instead: rank r encodes the features of its range
   (``feature_ranges``) for every query head and keeps each head's exact
   positive top-k among them; one all-gather of those picks (a few KB) and
   an exact merge give every rank the unsharded per-head top-k and the same
   order;
2. the union of the routed buckets' shard-local lists (core.py:152-164) with
   the per-shard budget ``budget // P`` -- in the unbudgeted mode the shards'
   unions are exactly the global union cut at the shard boundaries;
3. sparse attention over the shard's rows, exported as the per-head
   log-sum-exp partial (m, l, o[d]);
4. one all-gather of the P partials (NCCL over NVLink on GPUs) and the exact
   log-sum-exp merge on every rank (pk_lse_merge), the split-KV merge of the
   reference's kernels (kernels/ppu_8b/av_tuned.cu) applied across ranks.

The two all-gathers (routing picks, attention partials) are the only
exchanges on the path.  Between GPUs of one node they run over NVLink peer
memory (``PeerExchange``: plain peer stores and one flag per rank, a kernel
of the library); with exchange="nccl", or on CPU process groups, they are
library all-gathers.
"""
from __future__ import annotations

import ctypes
import math

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
    Moments are not carried: attach_global_moments gives the shard the whole
    sequence's."""
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


def feature_ranges(F: int, P: int) -> list:
    """Contiguous feature ranges [lo, hi) of the feature-sharded route, in
    rank order (sizes differ by at most one)."""
    return token_ranges(F, P)


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


class PeerExchange:
    """All-gather of a fixed-size device buffer between the P <= 8 ranks of
    one node over NVLink peer memory (pk_p2p_allgather).  Each rank
    allocates an exchange region in its own device memory and opens every
    peer's through a CUDA IPC handle (handles are exchanged once, at
    construction, over the process group).  ``all_gather(src, out)`` copies
    every rank's ``src`` into ``out[P, ...]``: one kernel, graph-capturable,
    no host synchronisation; every rank must make the same sequence of
    calls.  A peer that does not publish within ``max_spins`` polls (~64 ns
    each) sets a status bit that ``check()`` raises on."""

    def __init__(self, nbytes: int, group=None, device=None, max_spins: int = 1 << 23):
        if nbytes <= 0 or nbytes % 16:
            raise ValueError("the exchanged buffer must be a positive multiple of 16 bytes")
        self.group = group
        self.P = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.P > 8:
            raise ValueError("PeerExchange joins at most 8 ranks")
        self.nbytes = int(nbytes)
        self.max_spins = int(max_spins)
        self.device = torch.device(device or "cuda")
        region = int(nv.query("pk_p2p_region_bytes", self.P, self.nbytes))
        ptr = ctypes.c_uint64(0)
        with torch.cuda.device(self.device):
            _check(nv.query("pk_p2p_alloc", region, ctypes.addressof(ptr)), "pk_p2p_alloc")
        self.base = int(ptr.value)
        self._opened = []
        try:
            handle = (ctypes.c_uint8 * 64)()
            _check(nv.query("pk_p2p_handle", self.base, ctypes.addressof(handle)), "pk_p2p_handle")
            handles = [bytes(handle)]
            if self.P > 1:
                handles = [None] * self.P
                dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for q, h in enumerate(handles):
                if q == self.rank:
                    bases.append(self.base)
                    continue
                hb = (ctypes.c_uint8 * 64).from_buffer_copy(h)
                p = ctypes.c_uint64(0)
                with torch.cuda.device(self.device):
                    _check(nv.query("pk_p2p_open", ctypes.addressof(hb), ctypes.addressof(p)), "pk_p2p_open")
                self._opened.append(int(p.value))
                bases.append(int(p.value))
        except Exception:
            self.close(collective=False)
            raise
        self._bases = (ctypes.c_uint64 * self.P)(*bases)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def all_gather(self, src: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if src.numel() * src.element_size() != self.nbytes or not src.is_contiguous():
            raise ValueError(f"src must be a contiguous buffer of {self.nbytes} bytes")
        if out.shape[0] != self.P or out.numel() * out.element_size() != self.P * self.nbytes \
                or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous [{self.P}, ...] buffer of {self.P * self.nbytes} bytes")
        nv.call("pk_p2p_allgather", src, self.nbytes, self.rank, self.P, ctypes.addressof(self._bases), self.base,
                out, self.status, self.max_spins)
        return out

    def check(self) -> None:
        nv.check_status(self.status, "peer exchange")

    def close(self, collective: bool = True) -> None:
        """Unmaps the peers' regions and frees this rank's: a collective call
        (every rank, nothing in flight); the barriers keep any rank from
        freeing its region while a peer may still write to it."""
        if not getattr(self, "base", 0) and not getattr(self, "_opened", None):
            return
        torch.cuda.synchronize(self.device)
        sync = collective and self.P > 1 and dist.is_initialized()
        if sync:
            dist.barrier(group=self.group)
        for p in getattr(self, "_opened", []):
            nv.query("pk_p2p_close", p)
        self._opened = []
        if sync:
            dist.barrier(group=self.group)
        if getattr(self, "base", 0):
            nv.query("pk_p2p_free", self.base)
            self.base = 0


def _check(rc: int, what: str) -> None:
    if rc:
        raise RuntimeError(f"{what}: {'argument error' if rc < 0 else 'CUDA error'} {rc}")


def shard_budget(budget, P: int):
    """Per-shard union budget: floor(budget / P) (None stays unbudgeted)."""
    return None if budget is None else int(budget) // P


# ---------------------------------------------------------------------------
# Bucket moments of the whole sequence on every rank (the moments router)
# ---------------------------------------------------------------------------

def shard_moments(index: DeviceIndex, keys: torch.Tensor):
    """(bucket sizes int32 [U, F], mean, var fp32 [U, F, d]) of this shard:
    the population moments of its own keys over its own part of every
    bucket (core.py:76-89 on the shard)."""
    from .index import _unit_view
    keys, U, N, d, us, rs = _unit_view(keys)
    if (U, d) != (index.U, index.d) or N < index.history:
        raise ValueError("keys must be the shard's [U, N, d] rows of the index")
    F = index.F
    mean = torch.zeros(U, F, d, dtype=torch.float32, device=keys.device)
    var = torch.zeros_like(mean)
    nv.call("pk_summarize", keys, nv.dtype_code(keys), us, rs, index.offsets, index.lens, index.ids,
            index.ids.stride(0), U, d, F, mean, var)
    return index.lens.clone(), mean, var


def fold_moments(parts):
    """Moments of consecutive blocks folded in order with the reference's
    append merge (core.py:194-199, pk_merge_moments): parts is a list of
    (sizes int32 [U, F], mean, var [U, F, d]) in token order; returns the
    folded (sizes, mean, var)."""
    counts, mean, var = (t.clone() for t in parts[0])
    U, F, d = mean.shape
    for lens, m, v in parts[1:]:
        nv.call("pk_merge_moments", counts, mean, var, lens.contiguous(), m.contiguous(), v.contiguous(), U, F, d)
        counts += lens
    return counts, mean, var


def attach_global_moments(index: DeviceIndex, keys: torch.Tensor, *, group=None,
                          gather_bytes: int = 256 << 20) -> DeviceIndex:
    """Gives this rank's shard index the bucket moments and sizes of the
    whole sequence, so that the moments router (core.py:117-130) routes the
    same on every rank: each shard's moments (shard_moments) all-gathered
    and folded in token order with the append merge.  The result is the
    moments the reference's append_index would hold after indexing the
    shards one after another with these memberships.  Features are gathered
    in chunks of at most ``gather_bytes``.  index.mean / index.var /
    index.global_counts are set; returns the index."""
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    lens, mean, var = shard_moments(index, keys)
    if P == 1:
        index.mean, index.var, index.global_counts = mean, var, lens
        return index
    U, F, d = mean.shape
    all_lens = _gather(lens, torch.empty((P, U, F), dtype=lens.dtype, device=lens.device), group)
    fc = max(1, min(F, gather_bytes // (2 * P * U * d * 4)))
    out_mean, out_var = torch.empty_like(mean), torch.empty_like(var)
    for f0 in range(0, F, fc):
        f1 = min(F, f0 + fc)
        m_all = _gather(mean[:, f0:f1].contiguous(), torch.empty((P, U, f1 - f0, d), device=mean.device), group)
        v_all = _gather(var[:, f0:f1].contiguous(), torch.empty((P, U, f1 - f0, d), device=var.device), group)
        _, m, v = fold_moments([(all_lens[r, :, f0:f1].contiguous(), m_all[r], v_all[r]) for r in range(P)])
        out_mean[:, f0:f1] = m
        out_var[:, f0:f1] = v
    index.mean, index.var = out_mean, out_var
    index.global_counts = all_lens.sum(0, dtype=torch.int32)
    return index


class ShardedDecode:
    """Decode over this rank's sequence shard of every unit, merged across
    the group.  ``local_index`` covers this rank's token range (built on the
    shard, or cut from a full index by ``shard_index``); K/V passed to the
    call hold the shard's rows, the last rank's followed by the dense tail.
    router="moments" needs the whole sequence's moments on the index
    (attach_global_moments): every rank then routes with the global bucket
    moments and sizes and takes the same buckets."""

    def __init__(self, local_index: DeviceIndex, sae, *, group=None, heads_per_unit: int = 4,
                 router: str = "q_activation", query_scale: float = 1.0, query_topk: int | None = None,
                 budget: int | None = None, splits: int | None = None, max_history: int | None = None,
                 workspace: nv.Workspace | None = None, split_route: bool | None = None,
                 exchange: str | None = None):
        self.group = group
        init = dist.is_initialized()
        self.P = dist.get_world_size(group) if init else 1
        self.rank = dist.get_rank(group) if init else 0
        self.budget = budget
        route_counts = None
        if router == "moments":
            route_counts = getattr(local_index, "global_counts", None)
            if local_index.mean is None or route_counts is None:
                raise ValueError("the sharded moments router needs attach_global_moments on the shard index")
        self.op = SparseDecode(local_index, sae, heads_per_unit=heads_per_unit, router=router,
                               query_scale=query_scale, query_topk=query_topk,
                               budget=shard_budget(budget, self.P), splits=splits, max_history=max_history,
                               workspace=workspace, route_counts=route_counts)
        U, G, d = self.op.U, self.op.G, self.op.d
        dev = local_index.device
        self.part = torch.empty(U * G, d + 2, dtype=torch.float32, device=dev)
        self.gathered = torch.empty(self.P, U * G, d + 2, dtype=torch.float32, device=dev)
        self.out = None
        # q_activation routing split by features over the ranks on request;
        # replicated by default (measured faster on B200s at config 4: the
        # split's merge and exchange cost more than the encode it saves).
        if split_route is None:
            split_route = False
        if split_route and (router != "q_activation" or self.op.prep[0] is None):
            raise ValueError("split_route needs the bound-filtered q_activation router")
        self.split_route = bool(split_route)
        if self.split_route:
            self.f_range = feature_ranges(self.op.F, self.P)[self.rank]
            self.picks = torch.empty(U * G, self.op.k, 2, dtype=torch.int32, device=dev)
            self.all_picks = torch.empty(self.P, U * G, self.op.k, 2, dtype=torch.int32, device=dev)
        # The exchanges: NVLink peer memory between the GPUs of one node
        # (default with more than one CUDA rank), or the group's all-gather.
        if exchange is None:
            exchange = "p2p" if self.P > 1 and dev.type == "cuda" and dist.get_backend(group) == "nccl" else "nccl"
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.exchange = exchange
        self._px_part = self._px_picks = None
        if exchange == "p2p" and self.P > 1:
            self._px_part = PeerExchange(self.part.numel() * 4, group, dev)
            if self.split_route:
                self._px_picks = PeerExchange(self.picks.numel() * 4, group, dev)

    @property
    def is_tail_rank(self) -> bool:
        return self.rank == self.P - 1

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, length=None) -> torch.Tensor:
        U, G, d = self.op.U, self.op.G, self.op.d
        if self.split_route:
            self.op.route_shard_picks(q, *self.f_range, self.picks)
            if self._px_picks is not None:
                self._px_picks.all_gather(self.picks, self.all_picks)
            else:
                _gather(self.picks, self.all_picks, self.group)
            self.op.route_merge(self.all_picks)
            self.op.union()
        else:
            self.op.route(q)
        self.op.attention(q, k, v, length=length, partial=self.part)
        if self._px_part is not None:
            self._px_part.all_gather(self.part, self.gathered)
        else:
            gather_partials(self.part, self.gathered, self.group)
        if self.out is None or self.out.dtype != q.dtype:
            self.out = torch.empty(U, G, d, dtype=q.dtype, device=q.device)
        nv.call("pk_lse_merge", self.gathered, self.P, U * G, d, self.out, nv.dtype_code(q))
        return self.out

    def check(self) -> None:
        self.op.check()
        for px in (self._px_part, self._px_picks):
            if px is not None:
                px.check()

    def close(self) -> None:
        """Releases the peer-memory exchanges (every rank, nothing in flight)."""
        for px in (self._px_part, self._px_picks):
            if px is not None:
                px.close()
        self._px_part = self._px_picks = None


# ---------------------------------------------------------------------------
# Sequence-sharded build with the exact global BatchTopK
# ---------------------------------------------------------------------------

class ShardBuilder:
    """This shard's side of the sequence-sharded build (pk_build_shard_phase):
    keys [U, N, d] of tokens [lo, lo + N) of a sequence of N_total tokens,
    with the global center.  The phases are driven by ``drive_build`` with the
    collectives between them; the result is the shard-local index (token ids
    relative to lo) whose memberships are exactly those of the whole
    sequence's index cut at the shard (the reference's one-device build)."""

    def __init__(self, keys: torch.Tensor, sae, key_scale: float, *, lo: int, N_total: int, center: torch.Tensor,
                 slack_frac: float = 0.25, slack_min: int = 4, boundary_capacity: int | None = None,
                 workspace: nv.Workspace | None = None):
        from .index import SAEParams, _unit_view
        keys, U, N, d, us, rs = _unit_view(keys)
        self.keys, self.U, self.N, self.d, self.us, self.rs = keys, U, N, d, us, rs
        self.sae = SAEParams.of(sae, keys.device)
        self.F = self.sae.features
        self.key_scale = float(key_scale)
        self.lo, self.N_total = int(lo), int(N_total)
        self.global_count = self.N_total * self.sae.key_mean
        self.slack_frac, self.slack_min = float(slack_frac), int(slack_min)
        self.bcap = int(boundary_capacity or (4 * N * self.sae.key_mean + 65536))
        # Under the global threshold a shard may hold more than its own
        # N * key_mean members: the member list is sized for all of them.
        self.mcap = int(min(self.global_count, N * self.F))
        self.ws = workspace or nv.Workspace(keys.device)
        dev = keys.device
        self.index = DeviceIndex(U, self.F, d, 1, dev, moments=False)
        self.index.slack_frac, self.index.slack_min = self.slack_frac, self.slack_min
        self.index.center.copy_(torch.as_tensor(center, dtype=torch.float32, device=dev).reshape(-1, d).expand(U, d))
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.sample_info = torch.zeros(2, dtype=torch.int32, device=dev)
        self._alloc()

    def _alloc(self):
        U, N, F = self.U, self.N, self.F
        self.nbytes = int(nv.query("pk_build_shard_workspace_bytes", U, N, F, self.mcap, self.bcap))
        self.buf = self.ws.get(("shard_build", U, N, F, self.mcap, self.bcap), self.nbytes)
        lay = torch.zeros(8, dtype=torch.int64)
        rc = nv.query("pk_build_shard_layout", U, N, F, self.mcap, self.bcap, lay.data_ptr())
        if rc:
            raise RuntimeError(f"pk_build_shard_layout: argument error {rc}")
        o = lay.tolist()

        def view(k, n, dtype):
            nb = n * torch.empty(0, dtype=dtype).element_size()
            return self.buf[o[k]:o[k] + nb].view(dtype)

        self.histS = view(0, U * 8192, torch.int32).view(U, 8192)
        self.histL = view(1, U * 1024, torch.int32).view(U, 1024)
        self.histU = view(2, U * 1024, torch.int32).view(U, 1024)
        self.n_members = view(3, U, torch.int32)
        self.n_boundary = view(4, U, torch.int32)
        self.bkeys = view(5, U * self.bcap, torch.int64).view(U, self.bcap)

    def _phase(self, phase, *, sample_frac=0.0, all_keys=None, key_counts=None, P=1, key_cap=1, need=None):
        wh, wn = self.sae.prepared_half()
        idx = self.index
        nv.call("pk_build_shard_phase", phase, self.keys, nv.dtype_code(self.keys), self.us, self.rs, idx.center,
                self.key_scale, self.sae.W_enc, self.sae.b_enc, wh, wn, self.U, self.N, self.d, self.F,
                self.sae.key_mean, self.mcap, self.bcap, self.buf, self.nbytes, self.global_count, float(sample_frac),
                self.lo * self.F, idx.lens, idx.offsets, idx.ids, idx.ids.stride(0), 0, self.slack_frac,
                self.slack_min, all_keys, key_counts, P, key_cap, need, self.sample_info, self.status)

    def sample(self) -> torch.Tensor:
        self.status.zero_()
        self._phase(0)
        return self.histS

    def sample_fraction(self) -> float:
        """This shard's share of the sampled fraction of all N_total * F entries."""
        ns, fts = self.sample_info.tolist()
        return min(ns * 128, self.N) / self.N_total / max(1, fts)

    def bounds(self, sample_frac: float):
        self._phase(1, sample_frac=sample_frac)
        return self.histL, self.histU

    def classify(self):
        self._phase(2)
        return self.n_members, self.n_boundary, self.bkeys

    def finish(self, all_keys: torch.Tensor, key_counts: torch.Tensor, need: torch.Tensor) -> DeviceIndex:
        P, U, key_cap = all_keys.shape
        # CSR room for this shard's members: those decided so far plus, at
        # most, all of its boundary keys, each bucket with its slack.
        ub = int((self.n_members.long() + self.n_boundary.long()).max().item())
        cap = ub + int(math.ceil(ub * self.slack_frac)) + self.F * (self.slack_min + 1) + 64
        self.index.ids = torch.zeros(U, max(1, cap), dtype=torch.int32, device=self.keys.device)
        self._phase(3, all_keys=all_keys, key_counts=key_counts, P=P, key_cap=key_cap, need=need)
        self.index.history = self.N
        self.index.encode_path = "bounds"
        return self.index


def drive_build(builders, allreduce_sum, allreduce_max, allgather):
    """Runs the phases of the local builders (one per rank, or every shard
    when emulated in one process) with the given collectives over the lists
    of per-builder tensors: allreduce_sum / allreduce_max in place,
    allgather -> [P, ...] stacked in rank order."""
    def check(what):
        st = [b.status for b in builders]
        allreduce_max(st)
        v = int(st[0].item())
        if v:
            msgs = [m for bit, m in nv.STATUS_BITS.items() if v & bit]
            raise RuntimeError(f"sharded build ({what}): " + "; ".join(msgs))

    allreduce_sum([b.sample() for b in builders])
    fr = [torch.tensor([b.sample_fraction()], dtype=torch.float64, device=b.keys.device) for b in builders]
    allreduce_sum(fr)
    check("sample")
    hs = [b.bounds(float(fr[0].item())) for b in builders]
    allreduce_sum([h[0] for h in hs])
    allreduce_sum([h[1] for h in hs])
    check("bounds")
    cl = [b.classify() for b in builders]
    check("classify")
    members = [c[0].long().clone() for c in cl]
    allreduce_sum(members)
    caps = [c[1].max().long().reshape(1).clone() for c in cl]
    allreduce_max(caps)
    key_cap = max(1, min(int(caps[0].item()), min(b.bcap for b in builders)))
    all_keys = allgather([c[2][:, :key_cap].contiguous() for c in cl])
    counts = allgather([c[1].clone() for c in cl])
    out = []
    for b, m in zip(builders, members):
        need = (b.global_count - m).contiguous()
        out.append(b.finish(all_keys, counts, need))
    check("finish")
    return out


def global_center(keys_shards, N_total: int, gather=None) -> torch.Tensor:
    """Key center [U, d] of a sequence split into shards of whole cascade
    chunks (pk_key_center_chunks): the in-order fp32 sum of all chunk sums
    over N_total, bit-identical to the one-device torch-order mean.
    ``keys_shards``: this rank's keys [U, N, d] (with ``gather`` an
    all-gather over ranks) or the list of every shard's keys in order."""
    from .index import _unit_view
    local = keys_shards if isinstance(keys_shards, (list, tuple)) else [keys_shards]
    rows = int(nv.query("pk_key_center_chunk_rows", int(N_total)))
    if N_total % rows:
        raise ValueError(f"the sequence length must be a multiple of the cascade chunk ({rows} rows)")
    parts = []
    for k in local:
        k, U, N, d, us, rs = _unit_view(k)
        if N % rows:
            raise ValueError(f"every shard must hold whole cascade chunks of {rows} rows")
        out = torch.empty(U, N // rows, d, dtype=torch.float32, device=k.device)
        nv.call("pk_key_center_chunks", k, nv.dtype_code(k), us, rs, U, N, d, int(N_total), out)
        parts.append(out)
    chunks = torch.cat(parts, 1) if gather is None else torch.cat(list(gather(parts[0]).unbind(0)), 1)
    acc = torch.zeros_like(chunks[:, 0])
    for c in range(chunks.shape[1]):
        acc = acc + chunks[:, c]
    return acc / float(N_total)


def build_sharded(keys: torch.Tensor, sae, key_scale: float, *, lo: int, N_total: int, group=None, center=None,
                  slack_frac: float = 0.25, slack_min: int = 4, workspace: nv.Workspace | None = None) -> DeviceIndex:
    """This rank's index of tokens [lo, lo + N) under the whole sequence's
    exact BatchTopK (one SUM all-reduce of the sampled histogram, of the
    bound histograms and of the member counts, one MAX all-reduce of the
    status and key counts, one all-gather of the boundary keys).  The center
    defaults to the global key mean (global_center, all-gathered chunk sums).
    Without an initialised process group the shard is the whole sequence."""
    init = dist.is_initialized()
    P = dist.get_world_size(group) if init else 1

    def gather(t):
        out = torch.empty((P,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        return _gather(t, out, group)

    if center is None:
        center = global_center(keys, N_total, gather if P > 1 else None)
    b = ShardBuilder(keys, sae, key_scale, lo=lo, N_total=N_total, center=center, slack_frac=slack_frac,
                     slack_min=slack_min, workspace=workspace)

    def red(ts, op):
        if P > 1:
            dist.all_reduce(ts[0], op=op, group=group)

    def allgather(ts):
        t = ts[0]
        out = torch.empty((P,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        return _gather(t, out, group)

    return drive_build([b], lambda ts: red(ts, dist.ReduceOp.SUM), lambda ts: red(ts, dist.ReduceOp.MAX),
                       allgather)[0]


def _gather(t: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    P = out.shape[0]
    if P == 1:
        out[0].copy_(t)
    elif dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out
