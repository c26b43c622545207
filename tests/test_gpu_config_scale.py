"""The batched decode operator at the GPU configurations' sizes, against the
CPU oracle on identical seeded inputs.

Two units of config 3 (history 131072, F 16384, query top-32, budget 4096
tokens, a short generated tail) and two 65536-token cuts of config-4 units
(F 32768, query top-64, budget 8192 tokens, 4096 clusters) run through the
path the bench times: DeviceIndex.build (bound-filtered tensor-core build),
SparseDecode.route (bound-filtered q_activation routing + budgeted union) and
SparseDecode.attention.  The oracle recomputes each unit with the reference's
rules (core.py:13-26, 92-103, 131-139, 142-167, 170-183): memberships,
routed order, union ids and accepted buckets must be bit-exact, attention
within 2e-2 relative L2 (bf16).  The units share one SAE, as the units of a
layer do.
"""
import numpy as np
import pytest
import torch

from gen import unit_case

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def pk():
    from prismkv_b200 import build as b
    b.build()
    import prismkv_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return prismkv_b200


def run_case(pk, oracle, seeds, N, F, k, budget, clusters, tail):
    G, d = 4, 128
    dev = torch.device("cuda")
    cases = [unit_case(s, N, d, clusters, F, G, tail=tail, bf16=True) for s in seeds]
    W, b = cases[0]["W"], cases[0]["b"]
    U = len(cases)
    K = torch.stack([torch.from_numpy(c["keys"]) for c in cases]).to(dev).bfloat16()
    V = torch.stack([torch.from_numpy(c["values"]) for c in cases]).to(dev).bfloat16()
    Q = torch.stack([torch.from_numpy(c["q"]) for c in cases]).to(dev).bfloat16().contiguous()
    sae = pk.SAEParams(torch.from_numpy(W).to(dev), torch.from_numpy(b).to(dev), key_mean=8, query_topk=k)
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False)
    assert idx.encode_path == "bounds"
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, query_scale=1.0, budget=budget, max_history=N)
    op.route(Q)
    out = op.attention(Q, K, V, length=N + tail)
    torch.cuda.synchronize()
    op.check()
    osae = oracle.SAE(W, b, key_mean=8, query_topk=k)
    for u, c in enumerate(cases):
        oidx = oracle.build_index(c["keys"][:N], osae, 1.0, moments=False)
        counts, mem = idx.csr(u)
        assert np.array_equal(counts, oidx.counts), u
        assert np.array_equal(mem, oidx.ids), u
        _, order = oracle.bucket_scores(c["q"], oidx, router="q_activation", sae=osae, query_scale=1.0,
                                        query_topk=k)
        n = int(op.n_order[u].item())
        assert np.array_equal(op.order[u, :n].long().cpu().numpy(), order), u
        ids, feats, raw = oracle.select_from_order(order, oidx, budget)
        cnt = int(op.count[u].item())
        assert np.array_equal(op.ids[u, :cnt].long().cpu().numpy(), ids), u
        nf = int(op.n_features[u].item())
        assert op.features[u, :nf].long().cpu().tolist() == feats, u
        assert int(op.raw[u].item()) == raw, u
        assert 0 < cnt <= budget
        ref = oracle.attend(c["q"], c["keys"], c["values"], ids, N)
        got = out[u].float().cpu().numpy().astype(np.float64)
        err = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        assert err < TOL_BF16, (u, err)


def test_config3_units_match_oracle(pk, oracle):
    run_case(pk, oracle, seeds=(301, 302), N=131072, F=16384, k=32, budget=4096, clusters=1024, tail=5)


def test_config4_cut_units_match_oracle(pk, oracle):
    run_case(pk, oracle, seeds=(401, 402), N=65536, F=32768, k=64, budget=8192, clusters=4096, tail=0)
