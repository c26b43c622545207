"""GPU tests of the Hugging Face adapter (prismkv_b200.hf_reference) on tiny
random-init Qwen3 / Llama models.

* all_read mode (every history row through the sparse-attention kernel)
  reproduces the model's own decode logits;
* sparse mode, for both routers: every decode step of every layer and KV
  group selects exactly the ids the CPU oracle selects on the same keys and
  query (the index built from the prefix at the first decode token, then
  grown by update_interval blocks), and attends to within the fp32
  tolerance of the oracle; with one encoder shared by a layer's groups the
  groups run as the units of one batched operator."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")

TOL_F32 = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def tiny_model(kind, layers=2, heads=4, kv_heads=2):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    Cfg, Model = (Qwen3Config, Qwen3ForCausalLM) if kind == "qwen3" else (LlamaConfig, LlamaForCausalLM)
    cfg = Cfg(vocab_size=96, hidden_size=512, intermediate_size=256, num_hidden_layers=layers,
              num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128, max_position_embeddings=2048)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return Model(cfg).eval().cuda()


def make_encoders(layers, kv_heads, F, shared, seed=3):
    from prismkv_b200.hf_reference import Encoder
    from prismkv_b200.index import SAEParams
    g = torch.Generator().manual_seed(seed)
    out = {}
    for layer in range(layers):
        common = None
        for grp in range(kv_heads):
            if common is None or not shared:
                W = torch.randn(F, 128, generator=g) / 128 ** 0.5
                b = 0.01 * torch.randn(F, generator=g)
                common = Encoder(SAEParams(W.cuda(), b.cuda(), key_mean=8, query_topk=8), 1.0, 1.0)
            out[(layer, grp)] = common
    return out


def decode(model, prompt, steps):
    """Greedy decode; logits of every decode step."""
    logits = []
    with torch.no_grad():
        out = model(input_ids=prompt, use_cache=True)
        nxt = out.logits[:, -1].argmax(-1, keepdim=True)
        for _ in range(steps):
            out = model(input_ids=nxt, past_key_values=out.past_key_values, use_cache=True)
            logits.append(out.logits[:, -1].float().cpu())
            nxt = out.logits[:, -1].argmax(-1, keepdim=True)
    return logits


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import prismkv_b200
    return prismkv_b200


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_all_read_matches_model_decode(pk, kind):
    from prismkv_b200.hf_reference import HFReference
    model = tiny_model(kind)
    prompt = torch.randint(0, 96, (1, 150), generator=torch.Generator().manual_seed(5)).cuda()
    ref = decode(model, prompt, 6)
    s = HFReference(model, make_encoders(2, 2, 256, shared=False), mode="all_read")
    try:
        got = decode(model, prompt, 6)
    finally:
        s.close()
    for a, b in zip(got, ref):
        assert rel_l2(a.numpy(), b.numpy()) < TOL_F32
    recs = s.records
    assert len(recs) == 6 * 2 * 2
    assert all(r["unique"] == r["history"] == 150 and r["tail"] >= 1 for r in recs)


@pytest.mark.parametrize("router,shared,kind", [("q_activation", False, "qwen3"), ("q_activation", True, "llama"),
                                                ("moments", False, "qwen3"), ("moments", True, "qwen3")])
def test_sparse_decode_matches_oracle(pk, oracle, router, shared, kind):
    orc = oracle
    from prismkv_b200.hf_reference import HFReference
    layers, kv_heads, per_group, F, ui, prefix, steps = 2, 2, 2, 256, 16, 160, 24
    model = tiny_model(kind)
    encs = make_encoders(layers, kv_heads, F, shared)
    s = HFReference(model, encs, router=router, selected_buckets=8, update_interval=ui, detailed_records=True)
    caps = []
    inner = s.forward

    def capture(module, q, k, v, mask, **kw):
        out = inner(module, q, k, v, mask, **kw)
        layer = module.layer_idx
        if layer in s.layers:   # a decode step (prefill drops the layer's state)
            ids = {}
            for b in s.layers[layer]:
                assert len(b.groups) == (kv_heads if shared else 1)
                for i, g in enumerate(b.groups):
                    c = int(b.op.count[i])
                    ids[g] = (b.op.ids[i, :c].long().cpu().numpy(), b.index.history)
            caps.append((layer, q[0, :, 0].float().cpu().numpy(), k[0].float().cpu().numpy(),
                         v[0].float().cpu().numpy(), out[0][0, 0].float().cpu().numpy(), ids))
        return out

    s.forward = capture
    prompt = torch.randint(0, 96, (1, prefix), generator=torch.Generator().manual_seed(7)).cuda()
    try:
        decode(model, prompt, steps)
    finally:
        s.close()
    assert len(caps) == steps * layers
    recs = s.records
    assert len(recs) == steps * layers * kv_heads
    oidx = {}
    saes = {key: orc.SAE(e.sae.W_enc.cpu().numpy(), e.sae.b_enc.cpu().numpy(), 8, 8) for key, e in encs.items()}
    appended = False
    for ci, (layer, q, k, v, out, ids) in enumerate(caps):
        total = k.shape[1]
        for g in range(kv_heads):
            sae = saes[(layer, g)]
            K, V = k[g], v[g]
            if (layer, g) not in oidx:
                oidx[(layer, g)] = orc.build_index(K[:prefix], sae, 1.0, moments=router == "moments")
            idx = oidx[(layer, g)]
            while total - idx.history > ui:
                idx = orc.append_index(idx, K[idx.history:idx.history + ui], sae, 1.0)
                appended = True
            oidx[(layer, g)] = idx
            Q = q[g * per_group:(g + 1) * per_group]
            want, meta = orc.select_buckets(Q, idx, router=router, sae=sae, query_scale=1.0, query_topk=8,
                                            unique_cap=None)
            got, hist = ids[g]
            assert hist == idx.history
            assert np.array_equal(got, want), (layer, g, total)
            ref = orc.attend(Q, K, V, want, idx.history)
            assert rel_l2(out[g * per_group:(g + 1) * per_group], ref) < TOL_F32
            # The record, detailed split included (hf_reference.py:218-231).
            rec = next(r for r in recs[ci * kv_heads:(ci + 1) * kv_heads] if r["group"] == g)
            assert (rec["layer"], rec["history"], rec["tail"]) == (layer, idx.history, total - idx.history)
            assert (rec["unique"], rec["raw"], rec["buckets"]) == (len(want), meta["raw"], len(meta["features"]))
            old_unique = int((want < prefix).sum())
            old_raw = sum(int((idx.lists[b] < prefix).sum()) for b in meta["features"])
            assert (rec["initial_history"], rec["old_unique"], rec["old_raw"]) == (prefix, old_unique, old_raw)
            assert rec["generated_indexed_unique"] == len(want) - old_unique
            assert rec["generated_indexed_raw"] == meta["raw"] - old_raw
    assert appended


def _run_static(model, encs, prompt, steps, ui, graph):
    """Greedy decode over a StaticCache, eager or replayed (GraphDecoder)."""
    from transformers import StaticCache
    from prismkv_b200.hf_reference import GraphDecoder, HFReference
    s = HFReference(model, encs, router="q_activation", selected_buckets=8, update_interval=ui)
    cache = StaticCache(config=model.config, max_cache_len=256)
    n = prompt.shape[1]
    logits = []
    try:
        with torch.no_grad():
            out = model(input_ids=prompt, past_key_values=cache, cache_position=torch.arange(n, device="cuda"),
                        use_cache=True)
            tok = int(out.logits[0, -1].argmax())
            gd = GraphDecoder(s, model, cache) if graph else None
            for i in range(steps):
                pos = n + i
                if graph:
                    lg = gd.step(tok, pos).clone()
                else:
                    o = model(input_ids=torch.tensor([[tok]], device="cuda"), past_key_values=cache,
                              cache_position=torch.tensor([pos], device="cuda"), use_cache=True)
                    lg = o.logits[:, -1].clone()
                logits.append(lg.float().cpu())
                tok = int(lg.argmax())
            appended = any(b.index.history > n for st in s.layers.values() for b in st)
            if graph:
                # Steps replay one captured graph (a new capture only when an
                # append reallocated an index).
                assert gd.captures <= 3 and gd.replays >= steps - 3, (gd.captures, gd.replays)
    finally:
        s.close()
    return logits, appended


def test_static_cache_and_graph_decode(pk):
    """A static cache (full-length K/V, the length from the mask) decodes as
    the growing cache does, and the replayed CUDA-graph step (appends between
    replays) reproduces the eager static-cache steps."""
    model = tiny_model("qwen3")
    encs = make_encoders(2, 2, 256, shared=False)
    prompt = torch.randint(0, 96, (1, 150), generator=torch.Generator().manual_seed(9)).cuda()
    steps, ui = 30, 16
    from prismkv_b200.hf_reference import HFReference
    s = HFReference(model, encs, router="q_activation", selected_buckets=8, update_interval=ui)
    try:
        dynamic = decode(model, prompt, steps)
    finally:
        s.close()
    eager, app_e = _run_static(model, encs, prompt, steps, ui, graph=False)
    graphed, app_g = _run_static(model, encs, prompt, steps, ui, graph=True)
    assert app_e and app_g
    for a, b in zip(eager, dynamic):
        assert rel_l2(a.numpy(), b.numpy()) < 1e-5
    for a, b in zip(graphed, eager):
        assert rel_l2(a.numpy(), b.numpy()) < 1e-6
