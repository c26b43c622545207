"""The reference's portable operator API (src/prismkv/core.py) on the B200.

Same names, arguments, return values and errors as the reference; the
arithmetic runs in the CUDA library (prismkv_b200/csrc).  Inputs are CUDA
tensors; results stay on the device.

    build_index      core.py:92-103    -> pk_key_center + pk_build_index + pk_summarize
    append_index     core.py:186-201   -> pk_append_index
    summarize        core.py:76-89     -> pk_summarize
    bucket_scores    core.py:106-139   -> pk_route_qact / pk_route_moments
    select_buckets   core.py:142-167   -> routing + pk_union
    attend           core.py:170-183   -> pk_sparse_av
"""
from __future__ import annotations

import torch

from . import native as nv
from .index import DeviceIndex, SAEParams, budget_limit, from_lists

# Spare slots kept per bucket by build_index so append_index extends in place.
APPEND_SLACK_FRAC = 0.25
APPEND_SLACK_MIN = 4

_ws: dict = {}


def _workspace(device) -> nv.Workspace:
    key = torch.device(device)
    if key not in _ws:
        _ws[key] = nv.Workspace(key)
    return _ws[key]


class FeatureIndex:
    """core.py:62-73: history, center, counts, mean, variance, lists, backed
    by a one-unit DeviceIndex."""

    def __init__(self, dev: DeviceIndex):
        self.dev = dev

    @property
    def history(self) -> int:
        return self.dev.history

    @property
    def center(self) -> torch.Tensor:
        return self.dev.center[0]

    @property
    def counts(self) -> torch.Tensor:
        return self.dev.lens[0].long()

    @property
    def mean(self):
        return None if self.dev.mean is None else self.dev.mean[0]

    @property
    def variance(self):
        return None if self.dev.var is None else self.dev.var[0]

    @property
    def lists(self) -> list:
        return self.dev.lists(0)

    @property
    def memberships(self) -> int:
        return self.dev.memberships


SharedSAE = SAEParams  # parameter holder with the SharedSAE fields the path reads


@torch.no_grad()
def build_index(keys, sae, key_scale, *, center=None) -> FeatureIndex:
    if keys.ndim != 2 or len(keys) == 0 or key_scale <= 0:
        raise ValueError("nonempty [history,head_dim] keys and positive scale required")
    p = SAEParams.of(sae, keys.device)
    if keys.shape[-1] != p.head_dim:
        raise ValueError("SAE and attention head dimensions differ")
    dev = DeviceIndex.build(keys, p, float(key_scale), center=center, moments=True,
                            slack_frac=APPEND_SLACK_FRAC, slack_min=APPEND_SLACK_MIN,
                            workspace=_workspace(keys.device))
    return FeatureIndex(dev)


@torch.no_grad()
def append_index(index: FeatureIndex, new_keys, sae, key_scale) -> FeatureIndex:
    """Returns a new index; the given one is left as it was (as core.py)."""
    dev = index.dev.clone()
    dev.append(new_keys, SAEParams.of(sae, new_keys.device), float(key_scale),
               workspace=_workspace(new_keys.device))
    return FeatureIndex(dev)


@torch.no_grad()
def summarize(keys, lists, center=None) -> FeatureIndex:
    n, d = keys.shape
    center = keys.float().mean(0) if center is None else center
    dev = from_lists([lists], n, d, keys.device, center=center)
    F = dev.F
    dev.mean = torch.zeros(1, F, d, device=keys.device)
    dev.var = torch.zeros(1, F, d, device=keys.device)
    k = keys.contiguous()
    nv.call("pk_summarize", k, nv.dtype_code(k), 0, k.stride(0), dev.offsets, dev.lens, dev.ids, dev.ids.stride(0),
            1, d, F, dev.mean, dev.var)
    return FeatureIndex(dev)


def _route(q, dev: DeviceIndex, *, router, sae, query_scale, query_topk, terms, want_score=True):
    """Runs the router for unit 0; returns (score[F], order int32 [n])."""
    if q.ndim != 2:
        raise ValueError("q must be [heads, head_dim]")
    G, d = q.shape
    nv.require_head_dim(d)
    F = dev.F
    device = q.device
    qc = q.contiguous()
    if qc.dtype not in (torch.float32, torch.bfloat16):
        qc = qc.float()
    ws = _workspace(device)
    score = torch.empty(1, F, device=device)
    if router == "moments":
        if not terms or set(terms) - {"count", "mean", "variance"}:
            raise ValueError("specify exact estimator components")
        if dev.mean is None:
            raise ValueError("the moments router needs an index built with moments")
        bits = ((nv.PK_TERM_COUNT if "count" in terms else 0) | (nv.PK_TERM_MEAN if "mean" in terms else 0)
                | (nv.PK_TERM_VARIANCE if "variance" in terms else 0))
        k = min(int(query_topk), F)
        order = torch.empty(1, max(1, k), dtype=torch.int32, device=device)
        n = torch.empty(1, dtype=torch.int32, device=device)
        nbytes = nv.query("pk_route_moments_workspace_bytes", 1, G, F)
        nv.call("pk_route_moments", qc, nv.dtype_code(qc), dev.mean, dev.var, dev.lens, bits, 1, G, d, F, k,
                ws.get(("moments", 1, G, F), nbytes), nbytes, score, order, n, order.shape[1])
        return score[0], order[0, :int(n.item())]
    if router != "q_activation" or sae is None or query_scale is None or query_scale <= 0:
        raise ValueError("q_activation requires SAE and saved positive query scale")
    p = SAEParams.of(sae, device)
    k = min(int(query_topk), F)
    order = torch.empty(1, max(1, G * k), dtype=torch.int32, device=device)
    n = torch.empty(1, dtype=torch.int32, device=device)
    nbytes = nv.query("pk_route_qact_workspace_bytes", 1, G, F, k)
    wb, wn = p.prepared()
    nv.call("pk_route_qact", qc, nv.dtype_code(qc), None, 1, p.W_enc, p.b_enc, wb, wn, float(query_scale), dev.lens, 1,
            G, d, F, k, ws.get(("qact", 1, G, F, k), nbytes), nbytes, order, n, order.shape[1],
            score if want_score else None, None)
    return score[0], order[0, :int(n.item())]


@torch.no_grad()
def bucket_scores(q, index: FeatureIndex, *, router="moments", sae=None, query_scale=None, query_topk=16,
                  terms=("count", "mean", "variance")):
    score, order = _route(q, index.dev, router=router, sae=sae, query_scale=query_scale, query_topk=query_topk,
                          terms=terms)
    return score, order.long()


@torch.no_grad()
def select_buckets(q, index: FeatureIndex, *, unique_cap=None, **kwargs):
    if unique_cap is not None and not 0 <= unique_cap <= 1:
        raise ValueError("unique_cap must be a fraction in [0,1]")
    kw = dict(router="moments", sae=None, query_scale=None, query_topk=16, terms=("count", "mean", "variance"))
    kw.update(kwargs)
    dev = index.dev
    score, order = _route(q, dev, **kw)
    device = q.device
    H = dev.history
    limit = budget_limit(H, unique_cap)
    n = torch.tensor([len(order)], dtype=torch.int32, device=device)
    order_buf = order.reshape(1, -1).contiguous() if len(order) else torch.zeros(1, 1, dtype=torch.int32,
                                                                                  device=device)
    hist = torch.tensor([H], dtype=torch.int32, device=device)
    lim = torch.tensor([limit], dtype=torch.int64, device=device)
    out = torch.empty(1, max(1, H), dtype=torch.int32, device=device)
    cnt = torch.empty(1, dtype=torch.int32, device=device)
    feats = torch.empty(1, order_buf.shape[1], dtype=torch.int32, device=device)
    nf = torch.empty(1, dtype=torch.int32, device=device)
    raw = torch.empty(1, dtype=torch.int64, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    nv.call("pk_union", dev.offsets, dev.lens, dev.ids, dev.ids.stride(0), order_buf, n, order_buf.shape[1], hist,
            lim, 1, dev.F, max(1, H), out, out.shape[1], cnt, feats, nf, raw, status)
    nv.check_status(status, "select_buckets")
    c = int(cnt.item())
    ids = out[0, :c].long()
    assert len(ids) <= limit
    return ids, dict(features=feats[0, :int(nf.item())].long().tolist(), raw=int(raw.item()), unique=c,
                     limit=limit, candidate_buckets=len(order), scores=score)


@torch.no_grad()
def attend(q, keys, values, old_ids, history):
    if keys.shape != values.shape or not 0 <= history <= len(keys):
        raise ValueError("invalid KV/history")
    if len(old_ids) and (old_ids.min() < 0 or old_ids.max() >= history):
        raise ValueError("old_ids must address old history only")
    if len(old_ids.unique()) != len(old_ids):
        raise ValueError("deduplicate history before attention")
    G, d = q.shape
    nv.require_head_dim(d)
    device = q.device
    dt = q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32
    qc = q.to(dt).contiguous()
    k = keys.to(dt).contiguous()
    v = values.to(dt).contiguous()
    ids = old_ids.to(torch.int32).reshape(1, -1).contiguous() if len(old_ids) else \
        torch.zeros(1, 1, dtype=torch.int32, device=device)
    count = torch.tensor([len(old_ids)], dtype=torch.int32, device=device)
    hist = torch.tensor([history], dtype=torch.int32, device=device)
    total = len(keys)
    rows = len(old_ids) + (total - history)
    if rows == 0:
        return q.new_zeros(q.shape)
    length = torch.tensor([total], dtype=torch.int32, device=device)
    out = torch.empty(1, G, d, dtype=dt, device=device)
    splits = max(1, min(64, rows // 256))
    nbytes = nv.query("pk_sparse_av_workspace_bytes", 1, G, d, splits)
    ws = _workspace(device)
    nv.call("pk_sparse_av", qc, k, v, nv.dtype_code(qc), 1, 0, 0, k.stride(0), ids, ids.shape[1], count, hist, length,
            1, G, d, splits, ws.get(("av", 1, G, d, splits), nbytes), nbytes, out, None)
    return out[0].to(q.dtype)
