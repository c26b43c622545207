"""Encoder bundles: the inference-only encoders of a model, one per
(layer, KV group), as a directory that moves between this library and the
reference (src/prismkv/weights.py, manifest schema 1).

Format (schema 1):

* ``manifest.json`` -- a JSON object: ``schema`` (the integer 1),
  ``format`` (a description string), ``metadata`` (a free JSON object) and
  ``groups``, one record per encoder with the fields of ``GroupRecord``:
  ``layer`` and ``group`` (non-negative integers), ``file`` (the tensor
  file's name, ``l{layer:02d}_g{group:02d}.pt``, inside the bundle
  directory), ``sha256`` (hex digest of that file's bytes), ``head_dim``,
  ``features``, ``key_mean``, ``query_topk`` (integers) and ``key_scale``,
  ``query_scale`` (positive numbers).
* one tensor file per record: a ``torch.save`` dict holding exactly
  ``W_enc`` (fp32 ``[features, head_dim]``) and ``b_enc`` (fp32
  ``[features]``); decoder and optimizer state are not part of a bundle.

``load_encoders`` refuses, with ``ValueError``: another schema; a record
whose file lies outside the directory or whose bytes do not hash to its
digest; a (layer, group) listed twice; non-positive scales; a tensor file
with other contents; tensors whose shapes disagree with the record; and
non-finite weights.  It builds each encoder straight from the stored
tensors, so the caller's random-number streams are not touched.
``save_encoders`` writes a new directory only (``FileExistsError`` if it
exists) and refuses negative ids and non-positive scales.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import asdict, dataclass
from pathlib import Path

import torch

from .hf_reference import Encoder
from .index import SAEParams

SCHEMA = 1
FORMAT = "PrismKV inference encoder bundle; decoder/optimizer omitted"
MANIFEST = "manifest.json"
TENSORS = ("W_enc", "b_enc")


def file_digest(path) -> str:
    """SHA-256 hex digest of a file's bytes."""
    with open(path, "rb") as stream:
        return hashlib.file_digest(stream, "sha256").hexdigest()


@dataclass(frozen=True)
class GroupRecord:
    """One encoder's manifest record."""
    layer: int
    group: int
    file: str
    sha256: str
    head_dim: int
    features: int
    key_mean: int
    query_topk: int
    key_scale: float
    query_scale: float

    @staticmethod
    def file_name(layer: int, group: int) -> str:
        return f"l{layer:02d}_g{group:02d}.pt"

    @classmethod
    def parse(cls, row: dict) -> "GroupRecord":
        try:
            rec = cls(int(row["layer"]), int(row["group"]), str(row["file"]), str(row["sha256"]),
                      int(row["head_dim"]), int(row["features"]), int(row["key_mean"]), int(row["query_topk"]),
                      float(row["key_scale"]), float(row["query_scale"]))
        except (KeyError, TypeError, ValueError) as err:
            raise ValueError(f"malformed manifest record {row!r}: {err}") from None
        if not (rec.key_scale > 0 and rec.query_scale > 0):
            raise ValueError(f"{rec.file}: key_scale and query_scale must be positive "
                             f"(got {rec.key_scale}, {rec.query_scale})")
        return rec

    @property
    def unit(self) -> tuple:
        return self.layer, self.group


def save_encoders(encoders, directory, *, metadata=None) -> None:
    """Write ``encoders`` ({(layer, group): Encoder}) as a bundle into the new
    directory ``directory``."""
    items = sorted(encoders.items())
    for (layer, group), enc in items:
        if min(layer, group) < 0:
            raise ValueError(f"layer and group ids must be non-negative (got {layer}, {group})")
        if not (enc.key_scale > 0 and enc.query_scale > 0):
            raise ValueError(f"encoder ({layer}, {group}): scales must be positive")
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=False)
    records = []
    for (layer, group), enc in items:
        sae = enc.sae
        W = sae.W_enc.detach().to("cpu", torch.float32).contiguous()
        b = sae.b_enc.detach().to("cpu", torch.float32).contiguous()
        name = GroupRecord.file_name(layer, group)
        torch.save({"W_enc": W, "b_enc": b}, root / name)
        records.append(GroupRecord(layer, group, name, file_digest(root / name), int(W.shape[1]), int(W.shape[0]),
                                   int(sae.key_mean), int(sae.query_topk), float(enc.key_scale),
                                   float(enc.query_scale)))
    manifest = {"schema": SCHEMA, "format": FORMAT, "metadata": dict(metadata or {}),
                "groups": [asdict(r) for r in records]}
    # The manifest goes last and whole (written aside, then renamed), so a
    # directory with a manifest always holds every file it lists.
    tmp = root / (MANIFEST + ".tmp")
    tmp.write_text(json.dumps(manifest, indent=2), encoding="utf8")
    os.replace(tmp, root / MANIFEST)


def _read_manifest(root: Path):
    manifest = json.loads((root / MANIFEST).read_text(encoding="utf8"))
    if manifest.get("schema") != SCHEMA:
        raise ValueError(f"bundle schema {manifest.get('schema')!r} is not supported (this loader reads {SCHEMA})")
    records = [GroupRecord.parse(row) for row in manifest.get("groups", [])]
    seen = set()
    for rec in records:
        if rec.unit in seen:
            raise ValueError(f"layer {rec.layer}, group {rec.group} appears twice in the manifest (duplicate)")
        seen.add(rec.unit)
    return manifest, records


def _read_tensors(root: Path, rec: GroupRecord):
    path = (root / rec.file).resolve()
    if path.parent != root or not path.is_file():
        raise ValueError(f"{rec.file}: not a file inside the bundle directory")
    if file_digest(path) != rec.sha256:
        raise ValueError(f"{rec.file}: SHA-256 differs from the manifest's")
    blob = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(blob, dict) or sorted(blob) != sorted(TENSORS):
        keys = sorted(blob) if isinstance(blob, dict) else type(blob).__name__
        raise ValueError(f"{rec.file}: contents {keys} are not exactly {list(TENSORS)}")
    W, b = blob["W_enc"], blob["b_enc"]
    if tuple(W.shape) != (rec.features, rec.head_dim) or tuple(b.shape) != (rec.features,):
        raise ValueError(f"{rec.file}: tensor shape W_enc{tuple(W.shape)} b_enc{tuple(b.shape)} disagrees with "
                         f"the manifest ({rec.features} features x {rec.head_dim})")
    if not (bool(torch.isfinite(W).all()) and bool(torch.isfinite(b).all())):
        raise ValueError(f"{rec.file}: nonfinite encoder weights")
    return W, b


def load_encoders(directory, *, device="cpu"):
    """(encoders {(layer, group): Encoder}, manifest) from a bundle
    directory, the encoders' parameters on ``device``."""
    root = Path(directory).resolve()
    manifest, records = _read_manifest(root)
    out = {}
    for rec in records:
        W, b = _read_tensors(root, rec)
        sae = SAEParams(W.to(device), b.to(device), rec.key_mean, rec.query_topk)
        out[rec.unit] = Encoder(sae, rec.key_scale, rec.query_scale)
    return out, manifest
