"""Encoder bundles (prismkv_b200.weights), on CPU: the reference's contracts
(tests/test_weights.py of the reference: round trip of weights, scales and
metadata without touching the random-number stream; tampered and
out-of-directory files rejected) plus the other refusals of
src/prismkv/weights.py:39-70, and loading a bundle written by the
reference's own save_encoders (tests/golden/bundle_ref, made by
tests/golden/make_bundle.py)."""
import json
from pathlib import Path

import pytest
import torch

from prismkv_b200.hf_reference import Encoder
from prismkv_b200.index import SAEParams
from prismkv_b200.weights import load_encoders, save_encoders

GOLDEN = Path(__file__).resolve().parent / "golden"


def enc(d, F, key_mean, topk, ks, qs, seed=0):
    g = torch.Generator().manual_seed(seed)
    return Encoder(SAEParams(torch.randn(F, d, generator=g), torch.randn(F, generator=g), key_mean, topk), ks, qs)


def test_roundtrip_scales_metadata_and_rng(tmp_path):
    bundle = {(2, 0): enc(8, 32, 2, 4, 2.5, 1.25), (0, 1): enc(8, 32, 3, 5, 1.0, 0.5, seed=1)}
    root = tmp_path / "weights"
    save_encoders(bundle, root, metadata={"purpose": "unit test"})
    rng = torch.random.get_rng_state().clone()
    loaded, manifest = load_encoders(root)
    assert torch.equal(rng, torch.random.get_rng_state())
    assert set(loaded) == set(bundle)
    for key, e in bundle.items():
        got = loaded[key]
        assert torch.equal(got.sae.W_enc, e.sae.W_enc) and torch.equal(got.sae.b_enc, e.sae.b_enc)
        assert (got.sae.key_mean, got.sae.query_topk) == (e.sae.key_mean, e.sae.query_topk)
        assert (got.key_scale, got.query_scale) == (e.key_scale, e.query_scale)
    assert manifest["metadata"]["purpose"] == "unit test"
    assert [r["file"] for r in manifest["groups"]] == ["l00_g01.pt", "l02_g00.pt"]
    with pytest.raises(FileExistsError):
        save_encoders(bundle, root)          # never overwrites


def test_tampered_and_outside_files_rejected(tmp_path):
    root = tmp_path / "weights"
    save_encoders({(0, 0): enc(4, 16, 2, 4, 1, 1)}, root)
    data = root / "l00_g00.pt"
    with data.open("ab") as stream:
        stream.write(b"tamper")
    with pytest.raises(ValueError):
        load_encoders(root)
    manifest = json.loads((root / "manifest.json").read_text())
    manifest["groups"][0]["file"] = "../outside.pt"
    (root / "manifest.json").write_text(json.dumps(manifest))
    with pytest.raises(ValueError):
        load_encoders(root)


def _rewrite(root, edit):
    m = json.loads((root / "manifest.json").read_text())
    edit(m)
    (root / "manifest.json").write_text(json.dumps(m))


def test_other_refusals(tmp_path):
    def fresh(name, e=None):
        root = tmp_path / name
        save_encoders({(0, 0): e or enc(4, 16, 2, 4, 1, 1)}, root)
        return root

    root = fresh("schema")
    _rewrite(root, lambda m: m.update(schema=2))
    with pytest.raises(ValueError, match="schema"):
        load_encoders(root)
    root = fresh("dup")
    _rewrite(root, lambda m: m["groups"].append(dict(m["groups"][0])))
    with pytest.raises(ValueError, match="duplicate"):
        load_encoders(root)
    root = fresh("shape")
    _rewrite(root, lambda m: m["groups"][0].update(features=17))
    with pytest.raises(ValueError, match="shape"):
        load_encoders(root)
    root = fresh("scale")
    _rewrite(root, lambda m: m["groups"][0].update(query_scale=0.0))
    with pytest.raises(ValueError, match="scale"):
        load_encoders(root)
    bad = enc(4, 16, 2, 4, 1, 1)
    bad.sae.W_enc[0, 0] = float("nan")
    root = fresh("nan", bad)
    with pytest.raises(ValueError, match="nonfinite"):
        load_encoders(root)
    root = fresh("contents")
    torch.save({"W_enc": torch.zeros(16, 4), "b_enc": torch.zeros(16), "extra": torch.zeros(1)}, root / "l00_g00.pt")
    from prismkv_b200.weights import file_digest
    _rewrite(root, lambda m: m["groups"][0].update(sha256=file_digest(root / "l00_g00.pt")))
    with pytest.raises(ValueError, match="contents"):
        load_encoders(root)
    with pytest.raises(ValueError):
        save_encoders({(-1, 0): enc(4, 16, 2, 4, 1, 1)}, tmp_path / "neg")


def test_loads_a_bundle_saved_by_the_reference():
    loaded, manifest = load_encoders(GOLDEN / "bundle_ref")
    expect = json.loads((GOLDEN / "bundle_ref_expect.json").read_text())
    assert manifest["schema"] == 1
    assert set(loaded) == {(0, 1), (3, 0)}
    for key, e in expect.items():
        l, g = map(int, key.split(","))
        got = loaded[(l, g)]
        assert torch.equal(got.sae.W_enc, torch.tensor(e["W"], dtype=torch.float32))
        assert torch.equal(got.sae.b_enc, torch.tensor(e["b"], dtype=torch.float32))
        assert (got.key_scale, got.query_scale) == (e["key_scale"], e["query_scale"])
        assert (got.sae.key_mean, got.sae.query_topk) == (2, 4)
