"""Hugging Face attention integration for unpadded, batch-one causal decode.

The reference's adapter (src/prismkv/hf_reference.py:66-240, ``HFReference``)
with its decode path on this library's device operator:

* prefill runs the model's own attention backend (SDPA or eager), exactly as
  the reference (hf_reference.py:173-185);
* each decode token routes, unions and attends every KV group of the layer
  at once: the groups that share an encoder form the units of one
  ``DeviceIndex`` / ``SparseDecode`` (one kernel chain per layer instead of
  one Python loop iteration per group, hf_reference.py:193-217);
* the index of a layer is built from the prefix at its first decode token
  and grows by complete blocks of ``update_interval`` keys, the current
  token always staying in the dense tail (hf_reference.py:202-213);
* ``mode="all_read"`` is the dense-equivalence control: every history row
  through the same sparse-attention kernel.

Routing, union and attention run asynchronously on the current stream; the
per-group records (history, unique, raw, buckets, tail) are kept as device
tensors and read when ``records`` is accessed.  Supported attention modules:
Qwen3Attention, Qwen3_5Attention (the reference's) and LlamaAttention (the
Llama-3-8B-shaped decode loop); K/V in bf16 or fp32.
"""
from __future__ import annotations

import importlib
import math
from contextlib import contextmanager
from dataclasses import dataclass

import torch

from . import native as nv
from .decode import SparseDecode
from .index import DeviceIndex, SAEParams

SUPPORTED_MODULES = ("Qwen3Attention", "Qwen3_5Attention", "LlamaAttention")
BACKEND = "prismkv_b200"
BACKEND_EAGER = "prismkv_b200_eager"


@dataclass
class Encoder:
    """hf_reference.py:16-20: one encoder per (layer, KV group)."""
    sae: object
    key_scale: float
    query_scale: float


def _dispatch(module, q, k, v, attention_mask, **kwargs):
    session = getattr(module, "_prismkv_b200_session", None)
    if session is None:
        raise RuntimeError("PrismKV B200 backend selected without an attached session")
    return session.forward(module, q, k, v, attention_mask, **kwargs)


class _Batch:
    """The KV groups of one layer that share an encoder: one index, one
    operator, U = len(groups) units."""

    def __init__(self, groups, encoder: Encoder):
        self.groups = list(groups)
        self.encoder = encoder
        g0 = self.groups[0]
        self.span = slice(g0, g0 + len(self.groups)) if self.groups == list(range(g0, g0 + len(self.groups))) \
            else None
        self.sae = None
        self.index: DeviceIndex | None = None
        self.op: SparseDecode | None = None
        self.dense_ids = None
        self.len_dev = None   # rows per unit (history + tail), read by the attention on the device
        self.kv = None        # the layer's K/V cache tensors of the last decode step

    def rows(self, t: torch.Tensor) -> torch.Tensor:
        """t[0, groups] ([B, H_kv, T, d] -> [U, T, d]); a view for a run of groups."""
        return t[0, self.span] if self.span is not None else t[0, self.groups]


class HFReference:
    """A stateful, all-group adapter; one session per model, one request at a
    time (hf_reference.py:66-128).

    mode='all_read' is the dense-equivalence control; the main method is
    mode='sparse', router='moments', selected_buckets=16, unique_cap=None.
    Call begin_request() when starting a new KV cache; close() restores the
    model's attention backends."""

    def __init__(self, model, encoders, *, mode="sparse", router="moments", selected_buckets=16, unique_cap=None,
                 update_interval=4096, detailed_records=False):
        if mode not in ("sparse", "all_read"):
            raise ValueError("mode must be sparse or all_read")
        if router not in ("moments", "q_activation") or selected_buckets <= 0:
            raise ValueError("unsupported router/bucket count")
        if unique_cap is not None and not 0 <= unique_cap <= 1:
            raise ValueError("unique cap must be a fraction")
        if update_interval <= 0:
            raise ValueError("positive update interval required")
        if detailed_records:
            raise NotImplementedError("detailed records (per-list old/new splits) are not kept on the device path")
        self.model, self.encoders = model, encoders
        self.mode, self.router = mode, router
        self.selected_buckets, self.unique_cap = selected_buckets, unique_cap
        self.update_interval, self.force_prefill = update_interval, False
        self.detailed_records = detailed_records
        self.modules, self.original, self.configs = {}, {}, {}
        expected = set()
        for module in model.modules():
            if type(module).__name__ not in SUPPORTED_MODULES:
                continue
            if hasattr(module, "_prismkv_b200_session"):
                raise ValueError("model already has a PrismKV B200 session")
            layer = module.layer_idx
            if layer in self.modules:
                raise ValueError("duplicate attention-layer IDs")
            cfg = module.config
            expected.update((layer, g) for g in range(cfg.num_key_value_heads))
            self.modules[layer] = module
            implementation = cfg._attn_implementation
            if implementation not in ("sdpa", "eager"):
                raise ValueError("the adapter is validated for SDPA/eager prefill only")
            namespace = vars(importlib.import_module(type(module).__module__))
            registry = namespace["ALL_ATTENTION_FUNCTIONS"]
            self.original[layer] = (namespace["eager_attention_forward"] if implementation == "eager"
                                    else registry[implementation])
            self.configs[id(cfg)] = (cfg, implementation)
        if not self.modules or set(encoders) != expected:
            raise ValueError(f"provide exactly all standard-attention KV encoders; missing={expected - set(encoders)}, "
                             f"extra={set(encoders) - expected}")
        from transformers import AttentionInterface, AttentionMaskInterface
        from transformers.masking_utils import eager_mask, sdpa_mask
        AttentionInterface.register(BACKEND, _dispatch)
        AttentionMaskInterface.register(BACKEND, sdpa_mask)
        # Eager attention does not infer causality from a missing mask.
        AttentionInterface.register(BACKEND_EAGER, _dispatch)
        AttentionMaskInterface.register(BACKEND_EAGER, eager_mask)
        for module in self.modules.values():
            module._prismkv_b200_session = self
        for cfg, old in self.configs.values():
            cfg._attn_implementation = BACKEND_EAGER if old == "eager" else BACKEND
        self.workspaces = {}
        self.begin_request()

    # ----------------------------------------------------------- lifecycle
    def begin_request(self):
        self.prefix_lengths, self.layers, self._records = {}, {}, []
        self._graph_total = None

    @contextmanager
    def prefill(self):
        """Explicitly mark chunked prefill, including one-token chunks."""
        previous = self.force_prefill
        self.force_prefill = True
        try:
            yield self
        finally:
            self.force_prefill = previous

    def close(self):
        for module in self.modules.values():
            if getattr(module, "_prismkv_b200_session", None) is self:
                del module._prismkv_b200_session
        for cfg, implementation in self.configs.values():
            cfg._attn_implementation = implementation
        self.layers.clear()

    def generate(self, *args, **kwargs):
        """Reset for a new model.generate call/cache. Existing cache reuse is manual."""
        if kwargs.get("past_key_values") is not None:
            raise ValueError("use manual model calls and session state for an existing cache")
        self.begin_request()
        return self.model.generate(*args, **kwargs)

    @property
    def records(self) -> list:
        """Per (decode token, layer, group) records as in hf_reference.py:218-232
        (read from the device here, not during decode)."""
        out = []
        for rec in self._records:
            layer, groups, history, tail, count, raw, nfeat = rec
            c, r, nf = count.tolist(), raw.tolist(), nfeat.tolist()
            for i, g in enumerate(groups):
                out.append(dict(layer=layer, group=g, history=history, unique=int(c[i]), raw=int(r[i]),
                                buckets=int(nf[i]), tail=tail, routing_policy=self.mode))
        return out

    # ------------------------------------------------------------- forward
    def _workspace(self, device) -> nv.Workspace:
        key = torch.device(device)
        if key not in self.workspaces:
            self.workspaces[key] = nv.Workspace(key)
        return self.workspaces[key]

    def _batches(self, layer: int, groups: int):
        """The layer's groups partitioned by encoder (SAE object and scales)."""
        state = self.layers.get(layer)
        if state is None:
            by_key = {}
            for g in range(groups):
                enc = self.encoders[(layer, g)]
                by_key.setdefault((id(enc.sae), float(enc.key_scale), float(enc.query_scale)), []).append(g)
            state = self.layers[layer] = [_Batch(gs, self.encoders[(layer, gs[0])]) for gs in by_key.values()]
        return state

    @torch.no_grad()
    def forward(self, module, q, k, v, attention_mask, **kwargs):
        if q.shape[0] != 1 or k.shape[0] != 1:
            raise NotImplementedError("the adapter supports unpadded batch-one requests")
        if q.shape[-2] < 1 or q.shape[-1] != k.shape[-1] or k.shape != v.shape:
            raise ValueError("invalid QKV shapes")
        d = q.shape[-1]
        if not math.isclose(kwargs.get("scaling", 1 / math.sqrt(d)), 1 / math.sqrt(d)):
            raise NotImplementedError("nonstandard attention scale")
        if kwargs.get("sliding_window") is not None or kwargs.get("softcap") is not None:
            raise NotImplementedError("sliding-window/soft-capped attention is outside this adapter")
        if kwargs.get("dropout", 0) != 0:
            raise ValueError("inference only: disable dropout")
        layer, steps = module.layer_idx, q.shape[-2]
        graph = self._graph_total is not None
        if graph:
            # Replayed decode (GraphDecoder): the length comes from the host,
            # nothing is read back from the device while capturing.
            total = self._graph_total
        else:
            total = k.shape[-2]
            if attention_mask is not None:
                if attention_mask.ndim != 4:
                    raise NotImplementedError("padding/arbitrary attention masks are unsupported")
                # The last row must see a prefix of the cache: all of it (a
                # growing cache) or its first `total` slots (a static cache).
                last = attention_mask[..., -1, :total].reshape(-1, total)[0]
                visible = last if last.dtype == torch.bool else last == 0
                n = int(visible.sum().item())
                if n == 0 or not bool(visible[:n].all()):
                    raise NotImplementedError("padding/arbitrary attention masks are unsupported")
                total = n
        is_prefill = self.force_prefill or layer not in self.prefix_lengths or steps > 1
        if is_prefill:
            self.prefix_lengths[layer] = total
            self.layers.pop(layer, None)
            if attention_mask is None and 1 < steps < total:
                positions = torch.arange(total - steps, total, device=q.device)
                visible = torch.arange(total, device=q.device)[None] <= positions[:, None]
                attention_mask = torch.zeros((1, 1, steps, total), device=q.device, dtype=q.dtype)
                attention_mask.masked_fill_(~visible[None, None], -torch.inf)
            return self.original[layer](module, q, k, v, attention_mask, **kwargs)
        if steps != 1:
            raise NotImplementedError("decode is one token per forward")
        if not q.is_cuda:
            raise RuntimeError("the PrismKV B200 decode path needs CUDA tensors")
        groups, queries = k.shape[1], q.shape[1]
        if queries % groups:
            raise ValueError("Q heads must form equal-sized KV groups")
        per_group = queries // groups
        if k.stride(-1) != 1 or v.stride() != k.stride():
            k, v = k.contiguous(), v.contiguous()
        answer = torch.empty((1, 1, queries, d), dtype=q.dtype, device=q.device)
        qh = q[0, :, 0].reshape(groups, per_group, d)
        ws = self._workspace(q.device)
        for batch in self._batches(layer, groups):
            Qb = (qh[batch.span] if batch.span is not None else qh[batch.groups]).contiguous()
            Kb, Vb = batch.rows(k), batch.rows(v)
            batch.kv = (k, v)
            if self.mode == "all_read":
                history = self.prefix_lengths[layer]
                out, count, raw, nfeat = self._dense(batch, Qb, Kb, Vb, history, total, ws)
            else:
                if not graph:
                    history = self._advance(batch, layer, per_group, Kb, total, ws)
                    batch.len_dev.fill_(total)
                else:
                    history = batch.index.history
                op = batch.op
                op.route(Qb)
                out = op.attention(Qb, Kb, Vb, length=batch.len_dev)
                count, raw, nfeat = op.count, op.raw, op.n_features
            for i, g in enumerate(batch.groups):
                answer[0, 0, g * per_group:(g + 1) * per_group] = out[i]
            if not graph:
                self._records.append((layer, tuple(batch.groups), history, total - history, count.clone(),
                                      raw.clone(), nfeat.clone()))
        return answer, None

    def _advance(self, batch: _Batch, layer: int, per_group: int, Kb: torch.Tensor, total: int,
                 ws: nv.Workspace) -> int:
        """Build the batch's index from the prefix on first use, then index
        complete old tail blocks, keeping the current token in the dense
        tail (hf_reference.py:202-213); returns the indexed history."""
        enc = batch.encoder
        if batch.index is None:
            h = self.prefix_lengths[layer]
            batch.sae = SAEParams.of(enc.sae, Kb.device)
            batch.index = DeviceIndex.build(Kb[:, :h], batch.sae, float(enc.key_scale),
                                            moments=self.router == "moments", slack_frac=0.25, slack_min=4,
                                            workspace=ws)
        index = batch.index
        grew = False
        while total - index.history > self.update_interval:
            new = Kb[:, index.history:index.history + self.update_interval]
            index.append(new, batch.sae, float(enc.key_scale), workspace=ws)
            grew = True
        op = batch.op
        if op is None or index.history > op.max_history:
            batch.op = SparseDecode(index, batch.sae, heads_per_unit=per_group, router=self.router,
                                    query_scale=float(enc.query_scale), query_topk=self.selected_buckets,
                                    unique_cap=self.unique_cap, max_history=index.history + 8 * self.update_interval,
                                    workspace=ws)
            batch.len_dev = torch.zeros(len(batch.groups), dtype=torch.int32, device=Kb.device)
        elif grew:
            op.sync_history()
        return index.history

    def _dense(self, batch: _Batch, Qb, Kb, Vb, history: int, total: int, ws: nv.Workspace):
        """all_read: every history row (ids 0..history-1) plus the tail,
        through the sparse-attention kernel."""
        U, G, d = Qb.shape
        if batch.dense_ids is None or batch.dense_ids.shape[1] < history:
            batch.dense_ids = torch.arange(history, dtype=torch.int32, device=Qb.device).repeat(U, 1).contiguous()
        ids = batch.dense_ids
        count = torch.full((U,), history, dtype=torch.int32, device=Qb.device)
        hist = torch.full((U,), history, dtype=torch.int32, device=Qb.device)
        length = torch.full((U,), total, dtype=torch.int32, device=Qb.device)
        sms = torch.cuda.get_device_properties(Qb.device).multi_processor_count
        S = max(1, min(8, (2 * sms) // U))
        nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, S)
        out = torch.empty(U, G, d, dtype=Qb.dtype, device=Qb.device)
        nv.call("pk_sparse_av", Qb, Kb, Vb, nv.dtype_code(Qb), 1, Kb.stride(0), 0, Kb.stride(1), ids, ids.shape[1],
                count, hist, length, U, G, d, S, ws.get(("av", U, G, d, S), nbytes), nbytes, out, None)
        zeros = torch.zeros(U, dtype=torch.int64, device=Qb.device)
        return out, count, torch.full((U,), history, dtype=torch.int64, device=Qb.device), zeros


class GraphDecoder:
    """One-token decode of a model over a transformers StaticCache, replayed
    as one CUDA graph per step (the reference's serving loop,
    kernels/cuda_sm90/serving.py:71-125: a captured decode step whose inputs
    are refreshed before each replay).

    The first call runs eagerly (building every layer's index from the
    prefix) and then captures the step.  Before each replay the host writes
    the token and its position, indexes complete ``update_interval`` blocks
    (appends run outside the graph; the index and operator update in place),
    and refreshes the per-unit lengths.  If an append had to reallocate an
    index, the step is captured again.  Records are not kept for replayed
    steps.  mode='sparse' only."""

    def __init__(self, session: "HFReference", model, cache):
        if session.mode != "sparse":
            raise ValueError("graph decode needs mode='sparse'")
        self.s, self.model, self.cache = session, model, cache
        dev = next(model.parameters()).device
        self.tok = torch.zeros(1, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.graph = None
        self.logits = None
        self._ptrs = None
        self.captures = 0
        self.replays = 0

    def _buffers(self):
        return [(b.index.ids.data_ptr(), b.index.offsets.data_ptr(), b.index.lens.data_ptr(),
                 b.op.ids.data_ptr()) for st in self.s.layers.values() for b in st]

    @torch.no_grad()
    def step(self, token: int, position: int) -> torch.Tensor:
        """Logits of the next token after ``token`` at cache slot
        ``position`` (the positions continue the prefilled cache)."""
        s = self.s
        total = position + 1
        if self.graph is not None:
            ws = None
            for layer, st in s.layers.items():
                for b in st:
                    k, _ = b.kv
                    ws = ws or s._workspace(k.device)
                    s._advance(b, layer, b.op.G, b.rows(k), total, ws)
                    b.len_dev.fill_(total)
            if self._buffers() != self._ptrs:
                self.graph = None    # an index was reallocated: capture again
        if self.graph is None:
            self.tok.fill_(token)
            self.pos.fill_(position)
            out = self.model(input_ids=self.tok, past_key_values=self.cache, cache_position=self.pos, use_cache=True)
            eager = out.logits[:, -1].clone()
            self._capture(total + 1)
            return eager
        self.tok.fill_(token)
        self.pos.fill_(position)
        s._graph_total = total
        try:
            self.graph.replay()
        finally:
            s._graph_total = None
        self.replays += 1
        return self.logits[:, -1]

    def _capture(self, total_next: int):
        s = self.s
        self.graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        s._graph_total = total_next
        try:
            with torch.cuda.stream(stream):
                with torch.cuda.graph(self.graph, stream=stream):
                    self.logits = self.model(input_ids=self.tok, past_key_values=self.cache,
                                             cache_position=self.pos, use_cache=True).logits
        finally:
            s._graph_total = None
        torch.cuda.current_stream().wait_stream(stream)
        self._ptrs = self._buffers()
        self.captures += 1
