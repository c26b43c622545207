"""Generate golden fixtures by running the reference implementation itself.

Run in a container that has the reference checkout (read-only):

    PRISMKV_REFERENCE=/path/to/reference python tests/golden/make_golden.py

It imports the reference's portable path (src/prismkv/core.py) and evaluates
build_index, append_index, bucket_scores (q_activation and moments),
select_buckets and attend on seeded inputs from tests/golden/gen.py, writing
tests/golden/*.npz.  Large integer/fp32 outputs are stored as SHA-256 digests
of their little-endian bytes; small ones are stored whole.  The fixtures record
the torch version and CPU capability they were produced with.
"""
import hashlib
import json
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from gen import unit_case  # noqa: E402

REF = Path(os.environ.get("PRISMKV_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REF / "src"))
from prismkv import core  # noqa: E402


def digest(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


class SAE(torch.nn.Module):
    """Parameter holder with the fields core.py reads (W_enc, b_enc, ...)."""
    def __init__(self, W, b, key_mean, query_topk):
        super().__init__()
        self.W_enc = torch.nn.Parameter(torch.from_numpy(W))
        self.b_enc = torch.nn.Parameter(torch.from_numpy(b))
        self.features, self.head_dim = W.shape
        self.key_mean, self.query_topk = key_mean, query_topk

    dense = core.SharedSAE.dense


def lists_csr(lists):
    counts = np.array([len(x) for x in lists], np.int64)
    ids = torch.cat(lists).numpy().astype(np.int64) if len(lists) else np.zeros(0, np.int64)
    return counts, ids


# (name, seed, n, d, clusters, F, G, k, tail, bf16, caps, append_n, key_mean)
CASES = [
    ("u17", 11, 17, 128, 4, 64, 4, 4, 3, False, (None, 0.5), 5, 8),
    ("u64", 12, 64, 128, 8, 128, 4, 16, 0, True, (None, 0.25), 4, 8),
    ("u257", 13, 257, 128, 16, 256, 4, 16, 31, True, (None, 0.1, 0.0), 64, 8),
    ("u512", 14, 512, 128, 32, 256, 4, 32, 7, False, (None, 0.125, 0.03), 37, 8),
    ("u1000", 15, 1000, 128, 64, 512, 4, 16, 129, True, (None, 0.05), 24, 4),
    ("u2048", 16, 2048, 128, 64, 512, 4, 32, 1, True, (None, 0.0625, 1.0), 96, 8),
    ("u4096g8", 17, 4096, 128, 128, 1024, 8, 16, 16, True, (None, 0.125), 64, 8),
    ("cfg1", 18, 8192, 128, 256, 2048, 4, 16, 0, False, (0.125,), 256, 8),
]

# Units at the GPU configurations' shapes.  cfg2: one unit of config 2
# (N 32768, 1024 clusters, F 8192, k 32, budget 2048 tokens); cfg3u: one unit
# of config 3 (N 131072, F 16384, k 32, budget 4096, a 64-token tail); cfg4c:
# a 65536-token cut of a config-4 unit (F 32768, k 64, 4096 clusters, budget
# 8192 tokens).  They take minutes of reference CPU time each, so they are
# generated only when named on the command line.
LARGE = [
    ("cfg2", 19, 32768, 128, 1024, 8192, 4, 32, 0, True, (2048 / 32768, None), 128, 8),
    ("cfg3u", 20, 131072, 128, 1024, 16384, 4, 32, 64, True, (4096 / 131072,), 64, 8),
    ("cfg4c", 21, 65536, 128, 4096, 32768, 4, 64, 0, True, (8192 / 65536,), 32, 8),
]


def run_case(name, seed, n, d, clusters, F, G, k, tail, bf16, caps, append_n, key_mean):
    c = unit_case(seed, n, d, clusters, F, G, tail=tail + append_n, bf16=bf16, key_mean=key_mean)
    keys = torch.from_numpy(c["keys"])
    values = torch.from_numpy(c["values"])
    q = torch.from_numpy(c["q"])
    sae = SAE(c["W"], c["b"], key_mean, k)
    out = {}
    idx = core.build_index(keys[:n], sae, 1.0)
    counts, ids = lists_csr(idx.lists)
    out["center"] = idx.center.numpy()
    out["counts"] = counts
    out["ids_sha"] = digest(ids.astype(np.int64))
    out["n_members"] = np.int64(len(ids))
    out["mean_sha"] = digest(idx.mean.numpy())
    out["var_sha"] = digest(idx.variance.numpy())
    if len(ids) <= 20000:
        out["ids"] = ids.astype(np.int32)
    # q_activation route
    score, order = core.bucket_scores(q, idx, router="q_activation", sae=sae, query_scale=1.0, query_topk=k)
    out["qact_order"] = order.numpy().astype(np.int32)
    out["qact_score_sha"] = digest(score.numpy())
    nz = score.nonzero().flatten()
    out["qact_score_nz_ids"] = nz.numpy().astype(np.int32)
    out["qact_score_nz"] = score[nz].numpy()
    # moments route
    mscore, morder = core.bucket_scores(q, idx, router="moments", query_topk=k)
    out["mom_order"] = morder.numpy().astype(np.int32)
    out["mom_score"] = mscore.numpy()
    # select + attend per cap (q_activation router)
    for j, cap in enumerate(caps):
        sel, meta = core.select_buckets(q, idx, unique_cap=cap, router="q_activation", sae=sae,
                                        query_scale=1.0, query_topk=k)
        out[f"sel{j}_ids"] = sel.numpy().astype(np.int32)
        out[f"sel{j}_features"] = np.array(meta["features"], np.int32)
        out[f"sel{j}_raw"] = np.int64(meta["raw"])
        out[f"sel{j}_limit"] = np.int64(meta["limit"])
        out[f"sel{j}_cap"] = np.float64(-1.0 if cap is None else cap)
        total = n + tail
        att = core.attend(q, keys[:total], values[:total], sel, n)
        out[f"sel{j}_attend"] = att.numpy()
    # moments router select (unbudgeted) -- the native path's rule
    msel, mmeta = core.select_buckets(q, idx, unique_cap=None, router="moments", query_topk=k)
    out["msel_ids"] = msel.numpy().astype(np.int32)
    # append
    new = keys[n:n + append_n]
    merged = core.append_index(idx, new, sae, 1.0)
    mc, mids = lists_csr(merged.lists)
    out["app_counts"] = mc
    out["app_ids_sha"] = digest(mids.astype(np.int64))
    out["app_mean_sha"] = digest(merged.mean.numpy())
    out["app_var_sha"] = digest(merged.variance.numpy())
    if len(mids) <= 20000:
        out["app_ids"] = mids.astype(np.int32)
    meta = dict(name=name, seed=seed, n=n, d=d, clusters=clusters, F=F, G=G, k=k, tail=tail, bf16=bf16,
                caps=[(-1.0 if c is None else c) for c in caps], append_n=append_n, key_mean=key_mean,
                torch=torch.__version__, cpu=torch.backends.cpu.get_cpu_capability())
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, "members", len(ids), "order", len(order), "sel", [len(out[f'sel{j}_ids']) for j in range(len(caps))])


def run_edge():
    """Edge cases: ties in the global budget, an empty index, zero budget."""
    out = {}
    # all-equal activations -> tie order by flat index (core.py:24)
    keys = torch.ones(9, 4)
    W = torch.tensor([[1., 0, 0, 0], [1., 0, 0, 0], [0, 1., 0, 0]]).numpy()
    sae = SAE(W, np.zeros(3, np.float32), 2, 2)
    idx = core.build_index(keys + torch.arange(9.)[:, None] * 0, sae, 1.0, center=torch.zeros(4))
    c, ids = lists_csr(idx.lists)
    out["tie_counts"], out["tie_ids"] = c, ids
    # every activation <= 0 -> empty index
    sae2 = SAE(np.full((5, 4), -1.0, np.float32), np.full(5, -1.0, np.float32), 3, 2)
    idx2 = core.build_index(torch.randn(6, 4, generator=torch.Generator().manual_seed(0)), sae2, 1.0)
    out["empty_counts"] = lists_csr(idx2.lists)[0]
    np.savez_compressed(HERE / "edge.npz", **out)
    print("edge", out["tie_counts"], out["tie_ids"])


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count())
    names = sys.argv[1:]
    if not names:
        for case in CASES:
            run_case(*case)
        run_edge()
    for case in CASES + LARGE:
        if case[0] in names:
            run_case(*case)
