"""Inference-only encoder bundles: one tensor-only file per (layer, KV group)
plus a manifest with shapes, sparsities, scales and SHA-256 file hashes.

The reference's bundle format and checks (src/prismkv/weights.py:18-70,
manifest schema 1), kept alike so that bundles move between the two
libraries: ``save_encoders`` writes the same file names and manifest;
``load_encoders`` rejects an unknown schema, a file outside the bundle
directory, a hash mismatch, a duplicate (layer, group), unexpected file
contents, shapes that disagree with the manifest, non-finite weights and
non-positive scales.  Loading builds the encoders from the stored tensors
(no random initialisation), so the caller's random-number stream is left
as it was."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .hf_reference import Encoder
from .index import SAEParams

SCHEMA = 1
FORMAT = "PrismKV inference encoder bundle; decoder/optimizer omitted"


def _sha(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as stream:
        for chunk in iter(lambda: stream.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def save_encoders(encoders, directory, *, metadata=None) -> None:
    """Write one tensor-only file per (layer, KV group) and the manifest
    into a new directory (never overwrites one)."""
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=False)
    records = []
    for (layer, group), bundle in sorted(encoders.items()):
        if layer < 0 or group < 0 or bundle.key_scale <= 0 or bundle.query_scale <= 0:
            raise ValueError("invalid group or saved scale")
        sae = bundle.sae
        W = sae.W_enc.detach().float().cpu()
        b = sae.b_enc.detach().float().cpu()
        name = f"l{layer:02d}_g{group:02d}.pt"
        path = root / name
        torch.save(dict(W_enc=W, b_enc=b), path)
        records.append(dict(layer=layer, group=group, file=name, sha256=_sha(path), head_dim=int(W.shape[1]),
                            features=int(W.shape[0]), key_mean=int(sae.key_mean), query_topk=int(sae.query_topk),
                            key_scale=float(bundle.key_scale), query_scale=float(bundle.query_scale)))
    (root / "manifest.json").write_text(json.dumps(dict(schema=SCHEMA, format=FORMAT, metadata=metadata or {},
                                                        groups=records), indent=2), encoding="utf8")


def load_encoders(directory, *, device="cpu"):
    """(encoders {(layer, group): Encoder}, manifest) from a bundle directory;
    each encoder's SAE parameters on ``device``."""
    root = Path(directory).resolve()
    manifest = json.loads((root / "manifest.json").read_text(encoding="utf8"))
    if manifest.get("schema") != SCHEMA:
        raise ValueError("unsupported encoder-bundle schema")
    result = {}
    for row in manifest["groups"]:
        path = (root / row["file"]).resolve()
        if path.parent != root or not path.is_file() or _sha(path) != row["sha256"]:
            raise ValueError("encoder path/hash mismatch")
        unit = (row["layer"], row["group"])
        if unit in result:
            raise ValueError("duplicate layer/KV group")
        tensors = torch.load(path, map_location="cpu", weights_only=True)
        if not isinstance(tensors, dict) or set(tensors) != {"W_enc", "b_enc"}:
            raise ValueError("unexpected checkpoint contents")
        F, d = int(row["features"]), int(row["head_dim"])
        W, b = tensors["W_enc"], tensors["b_enc"]
        if tuple(W.shape) != (F, d) or tuple(b.shape) != (F,):
            raise ValueError("encoder shape mismatch")
        if not (torch.isfinite(W).all() and torch.isfinite(b).all()):
            raise ValueError("nonfinite encoder")
        if row["key_scale"] <= 0 or row["query_scale"] <= 0:
            raise ValueError("positive Q/K scales required")
        sae = SAEParams(W.to(device), b.to(device), int(row["key_mean"]), int(row["query_topk"]))
        result[unit] = Encoder(sae, float(row["key_scale"]), float(row["query_scale"]))
    return result, manifest
