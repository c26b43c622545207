"""Hugging Face attention integration for unpadded, batch-one causal decode.

The drop-in for the reference's adapter (src/prismkv/hf_reference.py:66-240,
``HFReference``): the same constructor arguments, refusals (their exception
types), lifecycle calls and records, with the decode path on this library's
device operator.  Its contract, restated:

* every standard attention module of the model (Qwen3Attention,
  Qwen3_5Attention; LlamaAttention here as well) must have one encoder per
  (layer, KV group), no more and no fewer;
* the model's attention backend is replaced by a dispatcher that sends each
  call to the session; prefill calls (several query rows, a layer's first
  call, or any call inside ``prefill()``) run the backend the model was
  configured with (SDPA or eager), with a causal mask offset to the cache
  when a chunk arrives without one; ``close()`` puts the backends back;
* a decode call (one query row) routes, unions and attends every KV group of
  the layer: the groups that share an encoder form the units of one
  ``DeviceIndex`` / ``SparseDecode`` (one kernel chain per layer instead of
  one loop iteration per group, hf_reference.py:193-217);
* the index of a layer is built from the prefix at its first decode token
  and grows by complete blocks of ``update_interval`` keys, the current
  token always staying in the dense tail (hf_reference.py:202-213);
* ``mode="all_read"`` is the dense-equivalence control: every history row
  through the same sparse-attention kernel.

Routing, union and attention run asynchronously on the current stream; the
per-group records (history, unique, raw, buckets, tail, and with
``detailed_records`` the split between the prefix and indexed generated
tokens) are kept as device tensors and read when ``records`` is accessed.
K/V in bf16 or fp32.
"""
from __future__ import annotations

import math
import sys
from contextlib import contextmanager
from dataclasses import dataclass

import torch

from . import native as nv
from .decode import SparseDecode, default_splits
from .index import DeviceIndex, SAEParams

SUPPORTED_MODULES = ("Qwen3Attention", "Qwen3_5Attention", "LlamaAttention")
BACKEND = "prismkv_b200"
BACKEND_EAGER = "prismkv_b200_eager"
SESSION_ATTR = "_prismkv_b200_session"


@dataclass
class Encoder:
    """hf_reference.py:16-20: one encoder per (layer, KV group)."""
    sae: object
    key_scale: float
    query_scale: float


def _dispatch(module, q, k, v, attention_mask, **kwargs):
    """The registered attention function: hands the call to the module's
    session."""
    session = getattr(module, SESSION_ATTR, None)
    if session is None:
        raise RuntimeError(f"attention backend {BACKEND!r} called on a module with no PrismKV B200 session")
    return session.forward(module, q, k, v, attention_mask, **kwargs)


def _check_options(mode, router, selected_buckets, unique_cap, update_interval) -> None:
    """The constructor's refusals of bad options (ValueError, as the
    reference's adapter)."""
    problems = []
    if mode not in ("sparse", "all_read"):
        problems.append(f"mode {mode!r} (expected 'sparse' or 'all_read')")
    if router not in ("moments", "q_activation"):
        problems.append(f"router {router!r} (expected 'moments' or 'q_activation')")
    if not selected_buckets > 0:
        problems.append(f"selected_buckets {selected_buckets!r} (expected a positive count)")
    if unique_cap is not None and not 0 <= unique_cap <= 1:
        problems.append(f"unique_cap {unique_cap!r} (expected None or a fraction in [0, 1])")
    if not update_interval > 0:
        problems.append(f"update_interval {update_interval!r} (expected a positive token count)")
    if problems:
        raise ValueError("invalid adapter options: " + "; ".join(problems))


def _prefill_backend(module, implementation: str):
    """The attention function the model would call for `implementation`:
    the registry entry for SDPA, the modeling file's own eager function for
    eager."""
    if implementation == "eager":
        return getattr(sys.modules[type(module).__module__], "eager_attention_forward")
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    return ALL_ATTENTION_FUNCTIONS[implementation]


def _causal_chunk_mask(steps: int, total: int, like: torch.Tensor) -> torch.Tensor:
    """Additive mask [1, 1, steps, total] for the last `steps` positions of a
    `total`-slot cache: query row i sits at position total - steps + i and
    sees the slots up to it."""
    mask = torch.full((steps, total), -torch.inf, dtype=like.dtype, device=like.device)
    return torch.triu(mask, diagonal=total - steps + 1)[None, None]


def _check_call(q, k, v, kwargs) -> int:
    """Refusals of an attention call outside the adapter's contract
    (unpadded batch one, standard scale, no sliding window, soft cap or
    dropout); returns the head dimension."""
    if q.shape[0] != 1 or k.shape[0] != 1:
        raise NotImplementedError(f"batch {q.shape[0]}: only unpadded batch-one requests are supported")
    d = q.shape[-1]
    if q.shape[-2] < 1 or k.shape[-1] != d or v.shape != k.shape:
        raise ValueError(f"attention shapes q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)} do not agree")
    if not math.isclose(kwargs.get("scaling", d ** -0.5), d ** -0.5):
        raise NotImplementedError(f"attention scale {kwargs['scaling']} differs from 1/sqrt({d})")
    for name in ("sliding_window", "softcap"):
        if kwargs.get(name) is not None:
            raise NotImplementedError(f"{name} attention is not supported")
    if kwargs.get("dropout", 0) != 0:
        raise ValueError("attention dropout must be 0 (inference only)")
    return d


def _visible_length(mask, slots: int) -> int:
    """Cache slots the last query row sees.  Without a mask it is every slot;
    a 4-D mask must let the last row see a prefix of the cache (all of a
    growing cache, the filled part of a static one) -- anything else is
    padding or a custom mask, which the adapter refuses."""
    if mask is None:
        return slots
    if mask.ndim != 4:
        raise NotImplementedError("only 4-D causal masks are supported (no padding or custom masks)")
    row = mask[..., -1, :slots].reshape(-1, slots)[0]
    sees = row if row.dtype == torch.bool else row == 0
    n = int(sees.sum().item())
    if n == 0 or not bool(sees[:n].all()):
        raise NotImplementedError("only 4-D causal masks are supported (no padding or custom masks)")
    return n


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
        self.prefix_lens = None   # per-unit bucket sizes over the prefix (detailed records)

    def rows(self, t: torch.Tensor) -> torch.Tensor:
        """t[0, groups] ([B, H_kv, T, d] -> [U, T, d]); a view for a run of groups."""
        return t[0, self.span] if self.span is not None else t[0, self.groups]


class HFReference:
    """One session per model and one request at a time (the reference's
    hf_reference.py:66-128 interface).

    mode='all_read' is the dense-equivalence control; the reference's main
    method is mode='sparse', router='moments', selected_buckets=16,
    unique_cap=None.  Call begin_request() when starting a new KV cache;
    close() gives the model its attention backends back."""

    def __init__(self, model, encoders, *, mode="sparse", router="moments", selected_buckets=16, unique_cap=None,
                 update_interval=4096, detailed_records=False):
        _check_options(mode, router, selected_buckets, unique_cap, update_interval)
        # Discover the attention modules and check the encoder coverage
        # before anything on the model changes.
        modules, backends, configs = {}, {}, {}
        for name, module in model.named_modules():
            if type(module).__name__ not in SUPPORTED_MODULES:
                continue
            if hasattr(module, SESSION_ATTR):
                raise ValueError(f"{name} is already attached to a PrismKV B200 session")
            layer = module.layer_idx
            if layer in modules:
                raise ValueError(f"attention layer id {layer} appears twice ({name})")
            cfg = module.config
            implementation = cfg._attn_implementation
            if implementation not in ("sdpa", "eager"):
                raise ValueError(f"{name}: prefill backend {implementation!r} is not supported (sdpa or eager)")
            modules[layer] = module
            backends[layer] = _prefill_backend(module, implementation)
            configs[id(cfg)] = (cfg, implementation)
        wanted = {(layer, g) for layer, m in modules.items() for g in range(m.config.num_key_value_heads)}
        given = set(encoders)
        if not modules or given != wanted:
            raise ValueError(f"encoders must cover exactly the (layer, KV group) pairs of the model's attention: "
                             f"missing={sorted(wanted - given)}, extra={sorted(given - wanted)}")
        self.model, self.encoders = model, encoders
        self.mode, self.router = mode, router
        self.selected_buckets, self.unique_cap = selected_buckets, unique_cap
        self.update_interval = update_interval
        self.detailed_records = bool(detailed_records)
        self.modules, self.original, self.configs = modules, backends, configs
        self._prefill_depth = 0
        self._attach()
        self.workspaces = {}
        self.begin_request()

    # ----------------------------------------------------------- lifecycle
    def _attach(self) -> None:
        from transformers import AttentionInterface, AttentionMaskInterface
        from transformers.masking_utils import eager_mask, sdpa_mask
        # Two registry names: an eager model keeps the eager mask builder,
        # which always materialises the causal mask.
        for name, mask_fn in ((BACKEND, sdpa_mask), (BACKEND_EAGER, eager_mask)):
            AttentionInterface.register(name, _dispatch)
            AttentionMaskInterface.register(name, mask_fn)
        for module in self.modules.values():
            setattr(module, SESSION_ATTR, self)
        for cfg, implementation in self.configs.values():
            cfg._attn_implementation = BACKEND_EAGER if implementation == "eager" else BACKEND

    def begin_request(self):
        """Forget every layer's prefix and index (a new KV cache)."""
        self.prefix_lengths, self.layers, self._records = {}, {}, []
        self._graph_total = None

    @property
    def force_prefill(self) -> bool:
        return self._prefill_depth > 0

    @contextmanager
    def prefill(self):
        """Within this block every call is prefill (chunked prefill,
        one-token chunks included)."""
        self._prefill_depth += 1
        try:
            yield self
        finally:
            self._prefill_depth -= 1

    def close(self):
        """Detach from the model and restore its attention backends."""
        for module in self.modules.values():
            if getattr(module, SESSION_ATTR, None) is self:
                delattr(module, SESSION_ATTR)
        for cfg, implementation in self.configs.values():
            cfg._attn_implementation = implementation
        self.layers.clear()

    def generate(self, *args, **kwargs):
        """model.generate on a fresh request; continuing an existing cache is
        done with manual model calls."""
        if kwargs.get("past_key_values") is not None:
            raise ValueError("generate() starts a new request; drive an existing cache with manual model calls")
        self.begin_request()
        return self.model.generate(*args, **kwargs)

    @property
    def records(self) -> list:
        """Per (decode token, layer, group) records as in hf_reference.py:218-232
        (read from the device here, not during decode)."""
        out = []
        for rec in self._records:
            layer, groups, history, tail, count, raw, nfeat, detail = rec
            c, r, nf = count.tolist(), raw.tolist(), nfeat.tolist()
            if detail is not None:
                initial, old_unique, old_raw = detail
                ou, orw = old_unique.tolist(), old_raw.tolist()
            for i, g in enumerate(groups):
                row = dict(layer=layer, group=g, history=history, unique=int(c[i]), raw=int(r[i]),
                           buckets=int(nf[i]), tail=tail, routing_policy=self.mode)
                if detail is not None:
                    row.update(initial_history=initial, old_unique=int(ou[i]), old_raw=int(orw[i]),
                               generated_indexed_unique=int(c[i]) - int(ou[i]),
                               generated_indexed_raw=int(r[i]) - int(orw[i]))
                out.append(row)
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
        d = _check_call(q, k, v, kwargs)
        layer, steps = module.layer_idx, q.shape[-2]
        graph = self._graph_total is not None
        # Replayed decode (GraphDecoder) takes the length from the host, so
        # nothing is read back from the device while capturing.
        total = self._graph_total if graph else _visible_length(attention_mask, k.shape[-2])
        if self.force_prefill or steps > 1 or layer not in self.prefix_lengths:
            # Prefill: the model's own backend over the whole chunk; the
            # layer's decode state starts again from this prefix.
            self.prefix_lengths[layer] = total
            self.layers.pop(layer, None)
            if attention_mask is None and 1 < steps < total:
                attention_mask = _causal_chunk_mask(steps, total, q)
            return self.original[layer](module, q, k, v, attention_mask, **kwargs)
        if not q.is_cuda:
            raise RuntimeError("the PrismKV B200 decode path runs on CUDA tensors only")
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
                detail = self._detail(batch, layer, count) if self.detailed_records else None
                self._records.append((layer, tuple(batch.groups), history, total - history, count.clone(),
                                      raw.clone(), nfeat.clone(), detail))
        return answer, None

    def _detail(self, batch: _Batch, layer: int, count: torch.Tensor):
        """The detailed record's split (hf_reference.py:218-231) on the
        device: of the union's ids, those inside the prefix the index was
        built from (ids are ascending, so the ones below its length); of the
        accepted buckets' raw entries, those from that prefix -- a bucket's
        size at build time, since appends only add later tokens."""
        initial = self.prefix_lengths[layer]
        if self.mode == "all_read":
            n = count.to(torch.int64)
            return initial, n, n
        op = batch.op
        width = op.ids.shape[1]
        slot = torch.arange(width, device=op.ids.device)
        old_unique = ((op.ids < initial) & (slot[None] < count[:, None])).sum(1)
        picks = torch.gather(batch.prefix_lens, 1, op.features.long())
        taken = torch.arange(op.features.shape[1], device=op.ids.device)[None] < op.n_features[:, None]
        old_raw = (picks * taken).sum(1)
        return initial, old_unique, old_raw

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
            if self.detailed_records:
                batch.prefix_lens = batch.index.lens.to(torch.int64)
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
        S = default_splits(U, total, Qb.device)
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
