"""Device-resident bucket index for U units of one layer, and SAE parameters.

Layout (see include/prismkv_b200.h): offsets[U, F+1] int32 bucket regions,
lens[U, F] int32 bucket sizes, ids[U, capacity] int32 token ids ascending per
bucket, center[U, d] fp32, optional mean/var[U, F, d] fp32.  Regions keep
spare slots so append_index extends buckets in place; a full region makes the
append refuse (all or nothing) and the index repacks itself with more room.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import native as nv


@dataclass
class SAEParams:
    """The encoder fields the path reads (the reference's SharedSAE,
    src/prismkv/core.py:29-48): W_enc[F, d], b_enc[F], key_mean, query_topk."""
    W_enc: torch.Tensor
    b_enc: torch.Tensor
    key_mean: int = 8
    query_topk: int = 16

    def __post_init__(self):
        self.W_enc = self.W_enc.detach().float().contiguous()
        self.b_enc = self.b_enc.detach().float().contiguous()
        F, d = self.W_enc.shape
        if self.b_enc.shape != (F,):
            raise ValueError("b_enc must have shape [features]")
        if not 1 <= self.key_mean <= F or not 1 <= self.query_topk <= F:
            raise ValueError("invalid sparsity")

    @property
    def features(self) -> int:
        return int(self.W_enc.shape[0])

    @property
    def head_dim(self) -> int:
        return int(self.W_enc.shape[1])

    def to(self, device) -> "SAEParams":
        return SAEParams(self.W_enc.to(device), self.b_enc.to(device), self.key_mean, self.query_topk)

    def prepared(self):
        """(W_bf16[F, d], w_norm[F]) for the bound-filtered routing path,
        computed once on the device (pk_sae_prepare)."""
        cached = getattr(self, "_prep", None)
        if cached is None or cached[0].device != self.W_enc.device:
            wb = torch.empty(self.W_enc.shape, dtype=torch.bfloat16, device=self.W_enc.device)
            wn = torch.empty(self.features, dtype=torch.float32, device=self.W_enc.device)
            nv.call("pk_sae_prepare", self.W_enc, self.features, self.head_dim, wb, wn)
            cached = self._prep = (wb, wn)
        return cached

    def prepared_half(self):
        """(W_half[F, d], w_norm[F]) for the bound-filtered build and append:
        W_enc rounded to fp16 on the device (pk_sae_prepare_half)."""
        cached = getattr(self, "_prep_half", None)
        if cached is None or cached[0].device != self.W_enc.device:
            wh = torch.empty(self.W_enc.shape, dtype=torch.float16, device=self.W_enc.device)
            nv.call("pk_sae_prepare_half", self.W_enc, self.features, self.head_dim, wh)
            cached = self._prep_half = (wh, self.prepared()[1])
        return cached

    @classmethod
    def of(cls, sae, device=None) -> "SAEParams":
        """Accepts an SAEParams or any object with the reference SharedSAE's
        fields (W_enc, b_enc, key_mean, query_topk)."""
        if isinstance(sae, SAEParams):
            p = sae
        else:
            p = cls(sae.W_enc, sae.b_enc, int(sae.key_mean), int(sae.query_topk))
        if device is not None and p.W_enc.device != torch.device(device):
            p = p.to(device)
        return p


def _unit_view(keys: torch.Tensor):
    """keys [U, N, d] or [N, d] -> (tensor, U, N, d, unit_stride, row_stride)."""
    if keys.dim() == 2:
        keys = keys.unsqueeze(0)
    if keys.dim() != 3:
        raise ValueError("keys must be [N, d] or [U, N, d]")
    if keys.stride(-1) != 1:
        keys = keys.contiguous()
    U, N, d = keys.shape
    return keys, U, N, d, keys.stride(0), keys.stride(1)


class DeviceIndex:
    """Bucket index of U units (one layer) resident in HBM."""

    def __init__(self, U: int, F: int, d: int, capacity: int, device, moments: bool = False):
        self.U, self.F, self.d = U, F, d
        self.device = torch.device(device)
        self.offsets = torch.zeros(U, F + 1, dtype=torch.int32, device=self.device)
        self.lens = torch.zeros(U, F, dtype=torch.int32, device=self.device)
        self.ids = torch.zeros(U, max(1, capacity), dtype=torch.int32, device=self.device)
        self.center = torch.zeros(U, d, dtype=torch.float32, device=self.device)
        self.mean = torch.zeros(U, F, d, device=self.device) if moments else None
        self.var = torch.zeros(U, F, d, device=self.device) if moments else None
        self.history = 0
        self.slack_frac = 0.0
        self.slack_min = 0
        self.encode_path = None   # "bounds" (tensor-core bounds) or "exact", set by build
        self.global_counts = None  # a sequence shard's whole-sequence bucket sizes (attach_global_moments)

    # ------------------------------------------------------------------ build
    @classmethod
    def build(cls, keys: torch.Tensor, sae, key_scale: float = 1.0, *, center=None, moments: bool = True,
              slack_frac: float = 0.0, slack_min: int = 0, workspace: nv.Workspace | None = None,
              boundary_capacity: int | None = None, exact: bool = False) -> "DeviceIndex":
        """Index every unit's keys (core.py:92-103 per unit).  By default the
        activations are bounded on the tensor cores and only undecided
        entries recomputed; exact=True computes every activation in fp32."""
        keys, U, N, d, us, rs = _unit_view(keys)
        if N == 0 or key_scale <= 0:
            raise ValueError("nonempty [history,head_dim] keys and positive scale required")
        sae = SAEParams.of(sae, keys.device)
        if d != sae.head_dim:
            raise ValueError("SAE and attention head dimensions differ")
        nv.require_head_dim(d)
        F = sae.features
        cap = int(nv.query("pk_build_ids_capacity", N, F, sae.key_mean, float(slack_frac), int(slack_min)))
        idx = cls(U, F, d, cap, keys.device, moments)
        idx.slack_frac, idx.slack_min = float(slack_frac), int(slack_min)
        dt = nv.dtype_code(keys)
        if center is None:
            nv.call("pk_key_center", keys, dt, us, rs, U, N, d, idx.center)
        else:
            c = torch.as_tensor(center, dtype=torch.float32, device=keys.device).reshape(-1, d)
            idx.center.copy_(c.expand(U, d))
        idx._encode(keys, dt, us, rs, N, sae, key_scale, token_base=0, workspace=workspace,
                    boundary_capacity=boundary_capacity, exact=exact)
        idx.history = N
        if moments:
            nv.call("pk_summarize", keys, dt, us, rs, idx.offsets, idx.lens, idx.ids, idx.ids.stride(0), U, d, F,
                    idx.mean, idx.var)
        return idx

    def _encode(self, keys, dt, us, rs, N, sae, key_scale, token_base, workspace, boundary_capacity, exact=False):
        U, F, d = self.U, self.F, self.d
        ws = workspace or nv.Workspace(keys.device)
        status = torch.zeros(1, dtype=torch.int32, device=keys.device)
        bcap = boundary_capacity or (4 * N * sae.key_mean + 65536)
        wb, wn = (None, None) if exact else sae.prepared_half()
        for _ in range(6):
            nbytes = nv.query("pk_build_workspace_bytes", U, N, F, sae.key_mean, bcap)
            buf = ws.get(("build", U, N, F, bcap), nbytes)
            status.zero_()
            nv.call("pk_build_index", keys, dt, us, rs, self.center, float(key_scale), sae.W_enc, sae.b_enc, wb, wn, U,
                    N, d, F, sae.key_mean, token_base, self.slack_frac, self.slack_min, self.offsets, self.lens,
                    self.ids, self.ids.stride(0), bcap, buf, nbytes, status)
            v = int(status.item())
            if v & nv.STATUS_BOUNDARY_FULL:
                bcap *= 4
                continue
            if v & nv.STATUS_NEEDS_EXACT and wb is not None:
                # The bounds could not bracket the threshold: exact encode.
                wb, wn = None, None
                continue
            nv.check_status(status, "build_index")
            self.encode_path = "bounds" if wb is not None else "exact"
            return
        nv.check_status(status, "build_index")

    # ----------------------------------------------------------------- append
    def append(self, new_keys: torch.Tensor, sae, key_scale: float = 1.0, *,
               workspace: nv.Workspace | None = None) -> None:
        """In-place append_index (core.py:186-201) of a block of keys per unit."""
        new_keys, U, n, d, us, rs = _unit_view(new_keys)
        if U != self.U or d != self.d:
            raise ValueError("new keys must be [U, n, d] matching the index")
        if n == 0:
            return
        sae = SAEParams.of(sae, new_keys.device)
        ws = workspace or nv.Workspace(new_keys.device)
        status = torch.zeros(1, dtype=torch.int32, device=new_keys.device)
        bcap = 4 * n * sae.key_mean + 65536
        dt = nv.dtype_code(new_keys)
        wb, wn = sae.prepared_half()
        for _ in range(8):
            nbytes = nv.query("pk_append_workspace_bytes", U, n, d, self.F, sae.key_mean, bcap)
            buf = ws.get(("append", U, n, self.F, bcap), nbytes)
            status.zero_()
            nv.call("pk_append_index", new_keys, dt, us, rs, n, self.center, float(key_scale), sae.W_enc, sae.b_enc,
                    wb, wn, U, d, self.F, sae.key_mean, self.history, self.offsets, self.lens, self.ids,
                    self.ids.stride(0), self.mean, self.var, bcap, buf, nbytes, status)
            v = int(status.item())
            if v & nv.STATUS_BOUNDARY_FULL:
                bcap *= 4
                continue
            if v & nv.STATUS_NEEDS_EXACT and wb is not None:
                wb, wn = None, None
                continue
            if v & nv.STATUS_BUCKET_FULL:
                # Nothing was written: make room and retry.
                self.repack(max(0.25, 2 * self.slack_frac), max(2 * n * sae.key_mean // max(1, self.F) + 8,
                                                                 2 * self.slack_min))
                continue
            nv.check_status(status, "append_index")
            self.history += n
            return
        nv.check_status(status, "append_index")

    def repack(self, slack_frac: float, slack_min: int) -> None:
        """Rewrite the bucket regions with more spare slots (device copy)."""
        lens = self.lens.long()
        slack = torch.ceil(lens.float() * slack_frac).long() + slack_min
        size = lens + slack
        new_off = torch.zeros(self.U, self.F + 1, dtype=torch.long, device=self.device)
        new_off[:, 1:] = torch.cumsum(size, 1)
        cap = int(new_off[:, -1].max().item())
        new_ids = torch.zeros(self.U, max(1, cap), dtype=torch.int32, device=self.device)
        old_off = self.offsets.long()
        # Gather every live entry: (unit, bucket, slot) -> positions.
        total = int(lens.sum().item())
        if total:
            uu = torch.repeat_interleave(torch.arange(self.U, device=self.device).repeat_interleave(self.F),
                                         lens.flatten())
            ff = torch.repeat_interleave(torch.arange(self.F, device=self.device).repeat(self.U), lens.flatten())
            start = torch.cumsum(lens.flatten(), 0) - lens.flatten()
            slot = torch.arange(total, device=self.device) - torch.repeat_interleave(start, lens.flatten())
            src = old_off[uu, ff] + slot
            dst = new_off[uu, ff] + slot
            new_ids[uu, dst] = self.ids[uu, src]
        self.offsets = new_off.int()
        self.ids = new_ids
        self.slack_frac, self.slack_min = float(slack_frac), int(slack_min)

    # ------------------------------------------------------------- utilities
    def clone(self) -> "DeviceIndex":
        c = DeviceIndex.__new__(DeviceIndex)
        c.__dict__.update(self.__dict__)
        for name in ("offsets", "lens", "ids", "center", "mean", "var"):
            t = getattr(self, name)
            setattr(c, name, None if t is None else t.clone())
        return c

    def units(self, u0: int, u1: int) -> "DeviceIndex":
        """Units [u0, u1) as an index over views of this one's tensors (no
        copy): operators on disjoint unit ranges can run concurrently, for
        example one per CUDA stream.  Appends must go through the full index."""
        if not 0 <= u0 < u1 <= self.U:
            raise ValueError("unit range must lie within [0, U)")
        c = DeviceIndex.__new__(DeviceIndex)
        c.__dict__.update(self.__dict__)
        c.U = u1 - u0
        for name in ("offsets", "lens", "ids", "center", "mean", "var"):
            t = getattr(self, name)
            setattr(c, name, None if t is None else t[u0:u1])
        return c

    def lists(self, u: int = 0) -> list:
        """The reference's FeatureIndex.lists for unit u (int64 tensors)."""
        off = self.offsets[u].long().cpu()
        ln = self.lens[u].long().cpu()
        ids = self.ids[u].long()
        return [ids[int(off[f]):int(off[f]) + int(ln[f])] for f in range(self.F)]

    def csr(self, u: int = 0):
        """(counts int64 [F], ids int64 [memberships]) of unit u on the host."""
        off = self.offsets[u].long().cpu().numpy()
        ln = self.lens[u].long().cpu().numpy()
        ids = self.ids[u].cpu().numpy()
        import numpy as np
        out = np.concatenate([ids[off[f]:off[f] + ln[f]] for f in range(self.F)]) if ln.sum() else \
            np.zeros(0, np.int32)
        return ln.astype(np.int64), out.astype(np.int64)

    @property
    def memberships(self) -> int:
        return int(self.lens.sum().item())

    def buffer_bytes(self) -> dict:
        return {name: t.numel() * t.element_size() for name, t in self.__dict__.items()
                if isinstance(t, torch.Tensor)}


def from_lists(lists_per_unit, history: int, d: int, device, center=None) -> DeviceIndex:
    """Device index from explicit bucket lists (list over units of lists of
    token-id sequences), as the reference's summarize() takes them."""
    U = len(lists_per_unit)
    F = len(lists_per_unit[0])
    lens = torch.tensor([[len(x) for x in lu] for lu in lists_per_unit], dtype=torch.long)
    cap = int(lens.sum(1).max().item()) if U else 0
    idx = DeviceIndex(U, F, d, cap, device, moments=False)
    off = torch.zeros(U, F + 1, dtype=torch.long)
    off[:, 1:] = torch.cumsum(lens, 1)
    ids = torch.zeros(U, max(1, cap), dtype=torch.int32)
    for u, lu in enumerate(lists_per_unit):
        flat = [int(t) for x in lu for t in (x.tolist() if hasattr(x, "tolist") else x)]
        if flat:
            ids[u, :len(flat)] = torch.tensor(flat, dtype=torch.int32)
    idx.offsets.copy_(off.int())
    idx.lens.copy_(lens.int())
    idx.ids.copy_(ids)
    idx.history = int(history)
    if center is not None:
        idx.center.copy_(torch.as_tensor(center, dtype=torch.float32).reshape(-1, d).expand(U, d))
    return idx


def budget_limit(history: int, unique_cap) -> int:
    """core.py:153: floor(history * unique_cap) in Python float arithmetic."""
    return history if unique_cap is None else math.floor(history * unique_cap)
