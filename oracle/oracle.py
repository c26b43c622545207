"""CPU oracle for the PrismKV decode-time retrieval path (TEST INFRASTRUCTURE).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, and only as the checker.  The product (prismkv_b200) never imports
it.

It mirrors the public functions of the reference's portable path,
src/prismkv/core.py, on numpy arrays:

    positive_global_topk  core.py:13-26
    summarize             core.py:76-89
    build_index           core.py:92-103
    bucket_scores         core.py:106-139
    select_buckets        core.py:142-167
    attend                core.py:170-183
    append_index          core.py:186-201

The arithmetic runs in oracle/prismkv_oracle.c, which restates the fp32
reduction orders of the reference's runtime; tests/test_oracle_golden.py pins
the results against fixtures generated from the reference itself
(tests/golden/make_golden.py).  Parity status: pinned bit-exact for integer
outputs and for the fp32 activations, centers, moments and q_activation scores;
the moments router's softmax and ``attend`` are pinned to a tolerance.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
SOURCE = HERE / "prismkv_oracle.c"

_lib = None


def build(force: bool = False) -> Path:
    """Compile the C restatement (gcc; no fast-math, no FMA contraction)."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SOURCE.stat().st_mtime:
        cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared",
               "-fPIC", str(SOURCE), "-o", str(LIB_PATH) + ".tmp", "-lm"]
        subprocess.run(cmd, check=True)
        os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I64, I, F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.orc_colmean.argtypes = [P, I64, I, P]
        L.orc_rowsum.argtypes = [P, I64]
        L.orc_rowsum.restype = F32
        L.orc_dense.argtypes = [P, I64, I, P, P, I, P]
        L.orc_positive_global_topk.argtypes = [P, I64, I64, P]
        L.orc_positive_global_topk.restype = I64
        L.orc_summarize.argtypes = [P, I, P, P, I, P, P]
        L.orc_build_index.argtypes = [P, I64, I, P, F32, P, P, I, I, P, P, P, P, I64, P, P]
        L.orc_build_index.restype = I64
        L.orc_build_index_stream.argtypes = L.orc_build_index.argtypes
        L.orc_build_index_stream.restype = I64
        L.orc_merge_moments.argtypes = [P, P, P, P, P, P, I, I, P, P]
        L.orc_route_qact.argtypes = [P, I, I, P, P, I, F32, I, P, P, P, P]
        L.orc_route_qact.restype = I
        L.orc_order_live.argtypes = [P, P, I, I, P]
        L.orc_order_live.restype = I
        L.orc_moments_score.argtypes = [P, I, I, P, P, P, I, I, P]
        L.orc_select.argtypes = [P, I, P, P, I64, I64, P, P, P, P]
        L.orc_select.restype = I64
        L.orc_attend.argtypes = [P, I, I, P, P, I64, P, I64, I64, P]
        L.orc_num_threads.restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# --------------------------------------------------------------------------
# Types
# --------------------------------------------------------------------------

@dataclass
class SAE:
    """Encoder parameters the path reads (core.py:29-45): W_enc[F,d], b_enc[F]."""
    W_enc: np.ndarray
    b_enc: np.ndarray
    key_mean: int = 8
    query_topk: int = 16

    def __post_init__(self):
        self.W_enc = _f32(self.W_enc)
        self.b_enc = _f32(self.b_enc)
        if not 1 <= self.key_mean <= self.features or not 1 <= self.query_topk <= self.features:
            raise ValueError("invalid sparsity")

    @property
    def features(self) -> int:
        return int(self.W_enc.shape[0])

    @property
    def head_dim(self) -> int:
        return int(self.W_enc.shape[1])

    def dense(self, normalized) -> np.ndarray:
        """core.py:47-48."""
        x = _f32(normalized)
        rows = x.shape[0]
        out = np.empty((rows, self.features), np.float32)
        lib().orc_dense(_p(x), rows, x.shape[1], _p(self.W_enc), _p(self.b_enc), self.features, _p(out))
        return out


@dataclass
class FeatureIndex:
    """core.py:62-73, held as CSR (offsets[F+1], ids) instead of a list."""
    history: int
    center: np.ndarray
    counts: np.ndarray
    mean: np.ndarray | None
    variance: np.ndarray | None
    offsets: np.ndarray
    ids: np.ndarray

    @property
    def lists(self):
        return [self.ids[self.offsets[b]:self.offsets[b + 1]] for b in range(len(self.counts))]

    @property
    def memberships(self) -> int:
        return int(self.offsets[-1])


def index_from_lists(history, center, lists, mean=None, variance=None) -> FeatureIndex:
    counts = np.array([len(x) for x in lists], np.int64)
    offsets = np.zeros(len(lists) + 1, np.int64)
    np.cumsum(counts, out=offsets[1:])
    ids = _i64(np.concatenate([np.asarray(x, np.int64) for x in lists])) if len(lists) else np.zeros(0, np.int64)
    return FeatureIndex(int(history), _f32(center) if center is not None else None, counts,
                        mean, variance, offsets, ids)


# --------------------------------------------------------------------------
# Functions (core.py)
# --------------------------------------------------------------------------

def positive_global_topk(a, count: int) -> np.ndarray:
    a = _f32(a)
    if a.ndim != 2 or count < 0:
        raise ValueError("expected a matrix and nonnegative activation budget")
    n = a.size
    out = np.empty(max(1, min(count, n)), np.int64)
    m = lib().orc_positive_global_topk(_p(a), n, count, _p(out))
    return out[:m].copy()


def colmean(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape[1], np.float32)
    lib().orc_colmean(_p(x), x.shape[0], x.shape[1], _p(out))
    return out


def rowsum(x) -> np.float32:
    x = _f32(x)
    return np.float32(lib().orc_rowsum(_p(x), x.size))


def summarize(keys, lists, center=None) -> FeatureIndex:
    keys = _f32(keys)
    n, d = keys.shape
    center = colmean(keys) if center is None else _f32(center)
    idx = index_from_lists(n, center, lists)
    F = len(lists)
    mean = np.empty((F, d), np.float32)
    var = np.empty((F, d), np.float32)
    lib().orc_summarize(_p(keys), d, _p(idx.offsets), _p(idx.ids), F, _p(mean), _p(var))
    idx.mean, idx.variance = mean, var
    return idx


# Above this many activations (n * F) build_index evaluates them in token
# blocks (orc_build_index_stream) instead of holding the [n, F] matrix.
STREAM_ACTIVATIONS = 1 << 25


def build_index(keys, sae: SAE, key_scale: float, *, center=None, moments: bool = True,
                stream: bool | None = None) -> FeatureIndex:
    """core.py:92-103.  ``stream`` picks the blocked evaluation (same result);
    by default it is used above STREAM_ACTIVATIONS activations."""
    keys = _f32(keys)
    if keys.ndim != 2 or len(keys) == 0 or key_scale <= 0:
        raise ValueError("nonempty [history,head_dim] keys and positive scale required")
    if keys.shape[-1] != sae.head_dim:
        raise ValueError("SAE and attention head dimensions differ")
    n, d = keys.shape
    F = sae.features
    cap = min(n * sae.key_mean, n * F)
    center_out = np.empty(d, np.float32)
    counts = np.empty(F, np.int64)
    offsets = np.empty(F + 1, np.int64)
    ids = np.empty(max(cap, 1), np.int64)
    mean = np.empty((F, d), np.float32) if moments else None
    var = np.empty((F, d), np.float32) if moments else None
    c_in = _f32(center) if center is not None else None
    if stream is None:
        stream = n * F > STREAM_ACTIVATIONS
    fn = lib().orc_build_index_stream if stream else lib().orc_build_index
    m = fn(_p(keys), n, d, _p(c_in), float(key_scale), _p(sae.W_enc), _p(sae.b_enc),
                              F, sae.key_mean, _p(center_out), _p(counts), _p(offsets), _p(ids), cap,
                              _p(mean), _p(var))
    if m < 0:
        raise RuntimeError(f"oracle build_index failed ({m})")
    return FeatureIndex(n, center_out, counts, mean, var, offsets, ids[:m].copy())


def append_index(index: FeatureIndex, new_keys, sae: SAE, key_scale: float) -> FeatureIndex:
    nxt = build_index(new_keys, sae, key_scale, center=index.center, moments=index.mean is not None)
    F = len(index.counts)
    total = index.counts + nxt.counts
    if index.mean is not None:
        d = index.mean.shape[1]
        mean = np.empty_like(index.mean)
        var = np.empty_like(index.variance)
        lib().orc_merge_moments(_p(_i64(index.counts)), _p(index.mean), _p(index.variance),
                                _p(_i64(nxt.counts)), _p(nxt.mean), _p(nxt.variance), F, d,
                                _p(mean), _p(var))
    else:
        mean = var = None
    lists = [np.concatenate((old, new + index.history)) for old, new in zip(index.lists, nxt.lists)]
    out = index_from_lists(index.history + len(new_keys), index.center, lists, mean, var)
    return out


def merge_moments(counts_a, mean_a, var_a, counts_b, mean_b, var_b):
    """The moments half of append_index (core.py:194-199): blocks a and b of
    bucket sizes counts_* and moments [F, d] merged; returns (mean, var)."""
    counts_a, counts_b = _i64(counts_a), _i64(counts_b)
    mean_a, var_a, mean_b, var_b = _f32(mean_a), _f32(var_a), _f32(mean_b), _f32(var_b)
    F, d = mean_a.shape
    mean = np.empty_like(mean_a)
    var = np.empty_like(var_a)
    lib().orc_merge_moments(_p(counts_a), _p(mean_a), _p(var_a), _p(counts_b), _p(mean_b), _p(var_b), F, d,
                            _p(mean), _p(var))
    return mean, var


def bucket_scores(q, index: FeatureIndex, *, router="moments", sae: SAE | None = None,
                  query_scale=None, query_topk=16, terms=("count", "mean", "variance")):
    q = _f32(q)
    F = len(index.counts)
    G, d = q.shape
    counts = _i64(index.counts)
    if router == "moments":
        if not terms or set(terms) - {"count", "mean", "variance"}:
            raise ValueError("specify exact estimator components")
        bits = (1 if "count" in terms else 0) | (2 if "mean" in terms else 0) | (4 if "variance" in terms else 0)
        score = np.empty(F, np.float32)
        lib().orc_moments_score(_p(q), G, d, _p(_f32(index.mean)), _p(_f32(index.variance)), _p(counts), F,
                                bits, _p(score))
        order = np.empty(max(1, min(query_topk, F)), np.int32)
        n = lib().orc_order_live(_p(score), _p(counts), F, query_topk, _p(order))
        return score, order[:n].astype(np.int64)
    if router != "q_activation" or sae is None or query_scale is None or query_scale <= 0:
        raise ValueError("q_activation requires SAE and saved positive query scale")
    k = min(query_topk, F)
    score = np.empty(F, np.float32)
    order = np.empty(max(1, G * k), np.int32)
    topk = np.empty(G * k, np.int32)
    n = lib().orc_route_qact(_p(q), G, d, _p(sae.W_enc), _p(sae.b_enc), F, float(query_scale), k,
                             _p(counts), _p(score), _p(order), _p(topk))
    return score, order[:n].astype(np.int64)


def order_live(score, counts, k: int) -> np.ndarray:
    """Ordering half of the moments router (core.py:127-130) on given scores."""
    score, counts = _f32(score), _i64(counts)
    order = np.empty(max(1, k), np.int32)
    n = lib().orc_order_live(_p(score), _p(counts), len(score), k, _p(order))
    return order[:n].astype(np.int64)


def select_from_order(order, index: FeatureIndex, limit: int):
    """The greedy of core.py:152-164 on a given candidate order."""
    order = np.ascontiguousarray(np.asarray(order, np.int32))
    out = np.empty(max(1, index.history), np.int64)
    feats = np.empty(max(1, len(order)), np.int32)
    nf = ctypes.c_int(0)
    raw = ctypes.c_int64(0)
    m = lib().orc_select(_p(order), len(order), _p(_i64(index.offsets)), _p(_i64(index.ids)),
                         index.history, int(limit), _p(out), _p(feats), ctypes.byref(nf), ctypes.byref(raw))
    return out[:m].copy(), feats[:nf.value].astype(np.int64).tolist(), int(raw.value)


def budget_limit(history: int, unique_cap) -> int:
    """core.py:153 (python float arithmetic, then floor)."""
    return history if unique_cap is None else math.floor(history * unique_cap)


def select_buckets(q, index: FeatureIndex, *, unique_cap=None, **kwargs):
    if unique_cap is not None and not 0 <= unique_cap <= 1:
        raise ValueError("unique_cap must be a fraction in [0,1]")
    scores, order = bucket_scores(q, index, **kwargs)
    limit = budget_limit(index.history, unique_cap)
    ids, features, raw = select_from_order(order, index, limit)
    assert len(ids) <= limit
    return ids, dict(features=features, raw=raw, unique=len(ids), limit=limit,
                     candidate_buckets=len(order), scores=scores)


def attend(q, keys, values, old_ids, history: int) -> np.ndarray:
    q, keys, values = _f32(q), _f32(keys), _f32(values)
    old = _i64(old_ids).reshape(-1)
    if keys.shape != values.shape or not 0 <= history <= len(keys):
        raise ValueError("invalid KV/history")
    if len(old) and (old.min() < 0 or old.max() >= history):
        raise ValueError("old_ids must address old history only")
    if len(np.unique(old)) != len(old):
        raise ValueError("deduplicate history before attention")
    G, d = q.shape
    out = np.empty((G, d), np.float32)
    lib().orc_attend(_p(q), G, d, _p(keys), _p(values), len(keys), _p(old), len(old), history, _p(out))
    return out
