"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Uses numpy's legacy RandomState, whose streams are stable across numpy
versions, so the fixtures' inputs regenerate identically on any host.
Distributions follow the benchmark configs: keys from a Gaussian-mixture
(centers ~ N(0,1), per-token noise sigma 0.3), values iid N(0,1), queries a
random center plus N(0, 0.3) noise, W_enc ~ N(0, 1/d), b_enc = 0.
"""
import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def unit_case(seed, n, d, clusters, F, G, tail=0, bf16=False, key_mean=8):
    rs = np.random.RandomState(seed)
    centers = rs.standard_normal((clusters, d)).astype(np.float32)
    cid = rs.randint(0, clusters, size=n + tail)
    keys = (centers[cid] + np.float32(0.3) * rs.standard_normal((n + tail, d)).astype(np.float32)).astype(np.float32)
    values = rs.standard_normal((n + tail, d)).astype(np.float32)
    qc = rs.randint(0, clusters, size=G)
    q = (centers[qc] + np.float32(0.3) * rs.standard_normal((G, d)).astype(np.float32)).astype(np.float32)
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    b = np.zeros(F, np.float32)
    if bf16:
        keys, values, q = bf16_round(keys), bf16_round(values), bf16_round(q)
    return dict(keys=keys, values=values, q=q, W=W, b=b, history=n, key_mean=key_mean)
