"""Realistic-weight fixtures: two of the reference's pretrained Qwen3-8B SAE
encoders (F = 3000, d = 128; src/prismkv/weights.py bundle, schema 1) run
through the reference's own core.py on seeded clustered keys, with the
bundle's key and query scales.

Run in a container that has the reference checkout (read-only):

    PRISMKV_REFERENCE=/path/to/reference python tests/golden/make_realweights.py

Writes tests/golden/bundle_qwen3_8b/ (the two encoder files copied byte for
byte, their manifest records, the reference's MIT notice) and
tests/golden/real_l00_g00.npz, real_l20_g05.npz: the same outputs as
make_golden.py's fixtures (index digests, q_activation and moments routes,
budgeted and unbudgeted unions for both routers, attention, append).  The
reference runs on one thread (see the note at the bottom).
"""
import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from gen import unit_case  # noqa: E402
import make_golden as mg  # noqa: E402
from make_golden import SAE, core, digest, lists_csr  # noqa: E402

REF = Path(os.environ.get("PRISMKV_REFERENCE", "/root/reference"))
SRC = REF / "pretrained" / "Qwen3-8B"
OUT = HERE / "bundle_qwen3_8b"
PICK = [(0, 0), (20, 5)]
NOTICE = ("The encoder files in this directory are two of the pretrained Qwen3-8B SAE encoders of the PrismKV\n"
          "reference (pretrained/Qwen3-8B), copied unchanged as test fixtures.  MIT License,\n"
          "Copyright (c) 2026 PrismKV authors.\n")


def copy_bundle():
    manifest = json.loads((SRC / "manifest.json").read_text())
    rows = [r for r in manifest["groups"] if (r["layer"], r["group"]) in PICK]
    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir()
    for r in rows:
        shutil.copyfile(SRC / r["file"], OUT / r["file"])
    small = dict(schema=manifest["schema"], format=manifest["format"],
                 metadata={"model_label": manifest["metadata"].get("model_label"),
                           "subset_of": "pretrained/Qwen3-8B of the PrismKV reference"},
                 groups=rows)
    (OUT / "manifest.json").write_text(json.dumps(small, indent=2))
    (OUT / "NOTICE").write_text(NOTICE)
    return rows


def run_real(row, seed, n=16384, clusters=256, G=4, tail=16, append_n=64, caps=(0.0625, None)):
    t = torch.load(OUT / row["file"], map_location="cpu", weights_only=True)
    W, b = t["W_enc"].float().numpy(), t["b_enc"].float().numpy()
    F, d, k, km = row["features"], row["head_dim"], row["query_topk"], row["key_mean"]
    ks, qs = float(row["key_scale"]), float(row["query_scale"])
    c = unit_case(seed, n, d, clusters, F, G, tail=tail + append_n, bf16=True, key_mean=km)
    keys, values, q = (torch.from_numpy(c[x]) for x in ("keys", "values", "q"))
    sae = SAE(W, b, km, k)
    out = {}
    idx = core.build_index(keys[:n], sae, ks)
    counts, ids = lists_csr(idx.lists)
    out["center"] = idx.center.numpy()
    out["counts"] = counts
    out["ids_sha"] = digest(ids.astype(np.int64))
    out["n_members"] = np.int64(len(ids))
    out["mean_sha"] = digest(idx.mean.numpy())
    out["var_sha"] = digest(idx.variance.numpy())
    score, order = core.bucket_scores(q, idx, router="q_activation", sae=sae, query_scale=qs, query_topk=k)
    out["qact_order"] = order.numpy().astype(np.int32)
    out["qact_score_sha"] = digest(score.numpy())
    mscore, morder = core.bucket_scores(q, idx, router="moments", query_topk=k)
    out["mom_order"] = morder.numpy().astype(np.int32)
    out["mom_score"] = mscore.numpy()
    total = n + tail
    for router in ("q_activation", "moments"):
        for j, cap in enumerate(caps):
            kw = dict(router=router, query_topk=k)
            if router == "q_activation":
                kw.update(sae=sae, query_scale=qs)
            sel, meta = core.select_buckets(q, idx, unique_cap=cap, **kw)
            tag = f"{router[0]}{j}"
            out[f"{tag}_ids"] = sel.numpy().astype(np.int32)
            out[f"{tag}_features"] = np.array(meta["features"], np.int32)
            out[f"{tag}_raw"] = np.int64(meta["raw"])
            out[f"{tag}_attend"] = core.attend(q, keys[:total], values[:total], sel, n).numpy()
    merged = core.append_index(idx, keys[n:n + append_n], sae, ks)
    mc, mids = lists_csr(merged.lists)
    out["app_counts"] = mc
    out["app_ids_sha"] = digest(mids.astype(np.int64))
    meta = dict(file=row["file"], seed=seed, n=n, d=d, clusters=clusters, F=F, G=G, k=k, tail=tail,
                append_n=append_n, key_mean=km, key_scale=ks, query_scale=qs,
                caps=[(-1.0 if c_ is None else c_) for c_ in caps], torch=torch.__version__,
                cpu=torch.backends.cpu.get_cpu_capability())
    out["meta"] = np.array(json.dumps(meta))
    name = "real_" + row["file"][:-3]
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, "members", len(ids), "qact order", len(order), "sel", [len(out[f"q{j}_ids"]) for j in range(len(caps))])


if __name__ == "__main__":
    # One thread: F.linear of a 2-5-row query block then takes MKL's sixteen
    # interleaved chains for every F.  With several threads and F not a
    # multiple of 256 (F = 3000 here) MKL switches to one sequential chain,
    # so the reference's fp32 scores depend on the thread count; the
    # single-thread order is the one the oracle and the kernels restate.
    torch.set_num_threads(1)
    rows = copy_bundle()
    for i, row in enumerate(rows):
        run_real(row, seed=31 + i)
