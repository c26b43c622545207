"""Host-side behaviour of the Hugging Face adapter (prismkv_b200.hf_reference),
on CPU: argument validation and encoder coverage (hf_reference.py:77-113),
backend registration and restoration, prefill through the model's own
attention (identical logits), and a loud failure for decode without CUDA
(there is no CPU path)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")

from prismkv_b200.hf_reference import BACKEND, Encoder, HFReference  # noqa: E402
from prismkv_b200.index import SAEParams  # noqa: E402


def tiny_model(kind="qwen3", layers=2, kv_heads=1, heads=2):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    Cfg, Model = (Qwen3Config, Qwen3ForCausalLM) if kind == "qwen3" else (LlamaConfig, LlamaForCausalLM)
    cfg = Cfg(vocab_size=96, hidden_size=256, intermediate_size=128, num_hidden_layers=layers,
              num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128, max_position_embeddings=1024)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    return Model(cfg).eval()


def encoders(layers, kv_heads, F=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = {}
    for layer in range(layers):
        for grp in range(kv_heads):
            W = torch.randn(F, 128, generator=g) / 128 ** 0.5
            out[(layer, grp)] = Encoder(SAEParams(W, torch.zeros(F), key_mean=8, query_topk=8), 1.0, 1.0)
    return out


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_validation_registration_and_close(kind):
    m = tiny_model(kind)
    enc = encoders(2, 1)
    with pytest.raises(ValueError):
        HFReference(m, enc, mode="dense")
    with pytest.raises(ValueError):
        HFReference(m, enc, router="random")
    with pytest.raises(ValueError):
        HFReference(m, enc, unique_cap=1.5)
    with pytest.raises(ValueError):
        HFReference(m, enc, update_interval=0)
    missing = dict(enc)
    missing.pop((1, 0))
    with pytest.raises(ValueError, match="missing"):
        HFReference(m, missing)
    extra = dict(enc)
    extra[(5, 0)] = enc[(0, 0)]
    with pytest.raises(ValueError, match="extra"):
        HFReference(m, extra)
    # Nothing was attached by the failed constructions.
    assert m.config._attn_implementation == "sdpa"
    s = HFReference(m, enc)
    assert m.config._attn_implementation == BACKEND
    with pytest.raises(ValueError, match="already"):
        HFReference(m, enc)
    s.close()
    assert m.config._attn_implementation == "sdpa"
    assert not any(hasattr(mod, "_prismkv_b200_session") for mod in m.modules())


@pytest.mark.parametrize("kind", ["qwen3", "llama"])
def test_prefill_passthrough_and_cpu_decode_refused(kind):
    m = tiny_model(kind)
    ids = torch.randint(0, 96, (1, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = m(input_ids=ids).logits
    s = HFReference(m, encoders(2, 1), router="q_activation")
    try:
        with torch.no_grad():
            out = m(input_ids=ids, use_cache=True)
        assert torch.equal(out.logits, ref)
        assert s.prefix_lengths == {0: 24, 1: 24}
        # A one-token decode step reaches the device path, which needs CUDA.
        with pytest.raises(RuntimeError, match="CUDA"), torch.no_grad():
            m(input_ids=ids[:, :1], past_key_values=out.past_key_values, use_cache=True)
        # Batch > 1 is refused as in the reference.
        with pytest.raises(NotImplementedError), torch.no_grad():
            m(input_ids=torch.cat([ids, ids]), use_cache=True)
    finally:
        s.close()


def test_detailed_records_accepted():
    """detailed_records=True is a supported option (the split is computed on
    the device at decode time; tests/test_gpu_hf.py checks its values)."""
    m = tiny_model()
    s = HFReference(m, encoders(2, 1), detailed_records=True)
    try:
        assert s.detailed_records and s.records == []
    finally:
        s.close()
    assert m.config._attn_implementation == "sdpa"


def test_chunked_prefill_mask_and_prefill_block():
    """A chunk that arrives without a mask gets the causal mask offset to the
    cache (its row i sees slots up to total - steps + i); inside prefill()
    even one-token calls are prefill."""
    from prismkv_b200.hf_reference import _causal_chunk_mask
    mask = _causal_chunk_mask(3, 7, torch.zeros(1))[0, 0]
    want = torch.tensor([[0 if j <= 4 + i else float("-inf") for j in range(7)] for i in range(3)])
    assert torch.equal(mask, want)
    m = tiny_model()
    s = HFReference(m, encoders(2, 1))
    try:
        ids = torch.randint(0, 96, (1, 9), generator=torch.Generator().manual_seed(2))
        with torch.no_grad():
            out = m(input_ids=ids[:, :8], use_cache=True)
            with s.prefill():
                assert s.force_prefill
                m(input_ids=ids[:, 8:], past_key_values=out.past_key_values, use_cache=True)
            assert not s.force_prefill
        assert s.prefix_lengths == {0: 9, 1: 9}
    finally:
        s.close()
