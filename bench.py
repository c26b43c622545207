#!/usr/bin/env python
"""Decode-attention benchmark: tokens/s at 128K context, config-3 shapes.

One decode step = for each of 32 layers: q_activation routing (SAE encode +
per-head top-32 + aggregation), budgeted bucket union (4096 tokens), and
sparse attention over the selected rows plus the dense generated tail, for
B=4 sequences x 8 KV heads (U = 32 units) with 4 query heads each, history
131072 tokens, F = 16384 SAE features.  Inputs are seeded synthetic tensors
with the config's shapes (clustered keys, iid values); the index is built by
this library's own build kernels before timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): the config's 32 units are split over
the ranks (2 and 4 ranks split the batch, 8 ranks split the batch 4 ways and
the KV heads 2 ways); the job still decodes the same B=4 sequences, so this
is strong scaling with no collective on the path.  The line's ``seqshard``
object measures config 4 on the same ranks: the 1M-token context split
along the sequence, with one NCCL all-gather of the attention partials per
step.  Timing is on the device with CUDA events, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode attn tokens/s/GPU at 128K ctx; sparse-AV HBM GB/s vs 8 TB/s peak"
L2_BYTES = 126 * 1024 * 1024


def parse():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=3,
                   help="3: Llama-3-8B-shaped 32-layer decode (default); 2: isolated stage times of one 128-unit "
                        "layer; 4: 1M-token sequence-sharded decode; 5: prefill bucket build + decode budget sweep")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--batch", type=int, default=4)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--q-per-kv", type=int, default=4)
    p.add_argument("--history", type=int, default=131072)
    p.add_argument("--features", type=int, default=16384)
    p.add_argument("--query-topk", type=int, default=32)
    p.add_argument("--key-mean", type=int, default=8)
    p.add_argument("--budget", type=int, default=4096)
    p.add_argument("--clusters", type=int, default=1024)
    p.add_argument("--max-steps", type=int, default=256, help="decode positions the KV cache holds")
    p.add_argument("--update-interval", type=int, default=4096, help="index append cadence (tokens)")
    p.add_argument("--no-graph", action="store_true", help="eager launches instead of CUDA-graph replay")
    p.add_argument("--layout", action="store_true",
                   help="layout diagnostic: in-place sparse attention vs explicit gather + packed attention")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-seqshard", action="store_true", help="skip the config-4 sub-measurement")
    p.add_argument("--parity-units", type=int, default=1,
                   help="units of layer 0 recomputed by the CPU oracle after timing (0: none)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--exchange", choices=["p2p", "nccl"], default=None,
                   help="config 4 on several GPUs: the step's all-gathers over NVLink peer memory (default) or NCCL")
    p.add_argument("--split-route", action="store_true",
                   help="config 4 on several GPUs: q_activation routing split by features over the ranks")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampler
# ---------------------------------------------------------------------------

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self):
        return time.time()

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0, t1):
        rows = [s for t, s in self.samples if t0 - 0.05 <= t <= t1 + 0.05]
        if not rows:
            rows = [s for t, s in self.samples][-3:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = sorted(v for v in (num(r[1]) for r in rows) if v is not None)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": num(rows[0][2]),
                "power_w_max": max((num(r[3]) or 0) for r in rows), "reasons": sorted(reasons),
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

GRAPH_INSPECT_ERRORS: list = []


def graph_kernel_launches(graph):
    """Kernel nodes of this library (C++ namespace pk) in a captured CUDA
    graph, through the driver API, or None when the graph cannot be
    inspected (the reason goes to GRAPH_INSPECT_ERRORS)."""
    try:
        from cuda.bindings import driver as drv
        ok = drv.CUresult.CUDA_SUCCESS
        handle = drv.CUgraph(int(graph.raw_cuda_graph()))
        err, _, n = drv.cuGraphGetNodes(handle, 0)
        if err != ok:
            GRAPH_INSPECT_ERRORS.append(f"cuGraphGetNodes: {err}")
            return None
        err, nodes, n = drv.cuGraphGetNodes(handle, n)
        if err != ok:
            GRAPH_INSPECT_ERRORS.append(f"cuGraphGetNodes: {err}")
            return None
        count = 0
        for node in nodes[:n]:
            err, kind = drv.cuGraphNodeGetType(node)
            if err != ok or kind != drv.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            err, params = drv.cuGraphKernelNodeGetParams(node)
            if err != ok or params is None:
                GRAPH_INSPECT_ERRORS.append(f"cuGraphKernelNodeGetParams: {err}")
                return None
            err, name = drv.cuFuncGetName(params.func)
            if err != ok:
                GRAPH_INSPECT_ERRORS.append(f"cuFuncGetName: {err}")
                return None
            name = name.decode() if isinstance(name, bytes) else str(name)
            count += name.startswith("_ZN2pk")
        return count
    except Exception as err:  # noqa: BLE001 -- an inspection aid, never fatal
        GRAPH_INSPECT_ERRORS.append(f"{type(err).__name__}: {err}")
        return None


def gen_layer(torch, dev, g, U, T, d, C):
    """Clustered keys (centers ~ N(0,1), noise sigma 0.3) and iid values, bf16."""
    centers = torch.randn(U, C, d, device=dev, generator=g)
    cid = torch.randint(0, C, (U, T), device=dev, generator=g)
    K = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    V = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    chunk = 16384
    for lo in range(0, T, chunk):
        hi = min(T, lo + chunk)
        c = torch.gather(centers, 1, cid[:, lo:hi, None].expand(U, hi - lo, d))
        K[:, lo:hi] = (c + 0.3 * torch.randn(U, hi - lo, d, device=dev, generator=g)).to(torch.bfloat16)
        V[:, lo:hi] = torch.randn(U, hi - lo, d, device=dev, generator=g).to(torch.bfloat16)
    return centers, K, V


def gen_queries(torch, dev, g, centers, n, G):
    U, C, d = centers.shape
    cid = torch.randint(0, C, (n, U, G), device=dev, generator=g)
    c = centers[torch.arange(U, device=dev)[None, :, None], cid]
    return (c + 0.3 * torch.randn(n, U, G, d, device=dev, generator=g)).to(torch.bfloat16)


class Ranks:
    """One process per GPU (torchrun's RANK / LOCAL_RANK / WORLD_SIZE), NCCL
    between them; device timings are reduced as the max over ranks."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def unit_partition(B: int, Hkv: int, world: int, rank: int):
    """The config's U = B * Hkv units (unit id b * Hkv + h) split over the
    ranks batch-first: 2 and 4 ranks split the batch, 8 ranks split the
    batch 4 ways and the KV heads 2 ways.  Returns this rank's unit ids."""
    U = B * Hkv
    if U % world:
        raise SystemExit(f"{U} units do not split evenly over {world} ranks")
    per = U // world
    return list(range(rank * per, (rank + 1) * per))


def gen_units(torch, dev, seed, layer, units, T, d, C, steps, G):
    """K, V [U, T, d] and every step's queries [steps, U, G, d] (bf16) of the
    given global unit ids of one layer: clustered keys (centers ~ N(0,1),
    noise sigma 0.3), iid values, queries a random center plus noise.  Each
    unit has its own seed, so a unit's data does not depend on how the units
    are spread over ranks."""
    U = len(units)
    K = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    V = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    Q = torch.empty(steps, U, G, d, device=dev, dtype=torch.bfloat16)
    g = torch.Generator(device=dev)
    for i, u in enumerate(units):
        g.manual_seed(seed * 1_000_003 + layer * 4099 + u)
        centers = torch.randn(C, d, device=dev, generator=g)
        for lo in range(0, T, 32768):
            hi = min(T, lo + 32768)
            cid = torch.randint(0, C, (hi - lo,), device=dev, generator=g)
            K[i, lo:hi] = (centers[cid] + 0.3 * torch.randn(hi - lo, d, device=dev, generator=g)).to(torch.bfloat16)
            V[i, lo:hi] = torch.randn(hi - lo, d, device=dev, generator=g).to(torch.bfloat16)
        qc = torch.randint(0, C, (steps, G), device=dev, generator=g)
        Q[:, i] = (centers[qc] + 0.3 * torch.randn(steps, G, d, device=dev, generator=g)).to(torch.bfloat16)
    return K, V, Q


def run_ours(a):
    import torch
    import prismkv_b200 as pk
    from prismkv_b200 import native as nv

    ctx = Ranks()
    world, rank, dev = ctx.world, ctx.rank, ctx.dev
    L, B, Hkv, G, d = a.layers, a.batch, a.kv_heads, a.q_per_kv, 128
    units = unit_partition(B, Hkv, world, rank)
    U = len(units)
    N, F, k = a.history, a.features, a.query_topk
    T = N + a.max_steps
    total_steps = a.warmup + a.steps
    if total_steps > a.max_steps:
        raise SystemExit("warmup + steps exceeds the KV cache's decode positions (--max-steps)")
    t_setup = time.time()
    layers = []
    ws = nv.Workspace(dev)
    build_s = 0.0
    for l in range(L):
        K, V, Q = gen_units(torch, dev, a.seed, l, units, T, d, a.clusters, total_steps, G)
        gw = torch.Generator(device=dev)
        gw.manual_seed(a.seed * 1_000_003 + l * 4099 + 999_983)   # one SAE per layer, shared by its units
        W = torch.randn(F, d, device=dev, generator=gw) / math.sqrt(d)
        sae = pk.SAEParams(W, torch.zeros(F, device=dev), key_mean=a.key_mean, query_topk=k)
        torch.cuda.synchronize()
        tb = time.time()
        idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws, slack_frac=0.25, slack_min=4)
        torch.cuda.synchronize()
        build_s += time.time() - tb
        op = pk.SparseDecode(idx, sae, heads_per_unit=G, query_scale=1.0, budget=a.budget,
                             max_history=N + a.max_steps, workspace=ws)
        layers.append(dict(K=K, V=V, idx=idx, op=op, Q=Q))
    for key in [k_ for k_ in ws.buffers if isinstance(k_, tuple) and k_[0] == "build"]:
        del ws.buffers[key]
    torch.cuda.empty_cache()
    # Per-step lengths: history + the tokens generated so far (dense tail).
    lens = torch.stack([torch.full((U,), N + s + 1, dtype=torch.int32, device=dev) for s in range(total_steps)])
    # Each step appends its token's K/V rows at position N + s of every layer's
    # cache (the reference's decode append, model.py:109-115); the rows are the
    # generated cache rows themselves, so the attention sees the same data.
    kv_steps = torch.stack([torch.stack([torch.stack([lay["K"][:, N + s], lay["V"][:, N + s]]) for lay in layers])
                            for s in range(total_steps)]).contiguous()   # [steps, L, 2, U, d]
    setup_s = time.time() - t_setup

    # Static inputs for graph replay.
    # Every step's queries for all layers, stacked so one copy loads a step.
    q_steps = torch.stack([torch.stack([lay["Q"][s] for lay in layers]) for s in range(total_steps)]).contiguous()
    for lay in layers:
        del lay["Q"]
    q_static = q_steps[0].clone()   # [L, U, G, d]
    kv_static = kv_steps[0].clone()  # [L, 2, U, d]
    len_static = lens[0].clone()
    outs = torch.empty(L, U, G, d, dtype=torch.bfloat16, device=dev)

    def step_body():
        for l, lay in enumerate(layers):
            q = q_static[l]
            lay["op"].route(q)
            # The token's KV append fused into the attention launch: its rows
            # are attended as the newest tail row and written into the cache.
            lay["op"].attention(q, lay["K"], lay["V"], length=len_static,
                                append=(kv_static[l, 0], kv_static[l, 1]), out=outs[l])

    def load_step(s):
        q_static.copy_(q_steps[s])
        kv_static.copy_(kv_steps[s])
        len_static.copy_(lens[s])

    # Warm up eagerly once (creates every workspace), then capture.
    load_step(0)
    step_body()
    torch.cuda.synchronize()
    for lay in layers:
        lay["op"].check()
    graph = None
    graph_launches = None
    if not a.no_graph:
        graph = torch.cuda.CUDAGraph(keep_graph=True)
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(graph, stream=s_cap):
                step_body()
        torch.cuda.current_stream().wait_stream(s_cap)
        graph.instantiate()
        torch.cuda.synchronize()
        graph_launches = graph_kernel_launches(graph)

    def run_step(s):
        load_step(s)
        if graph is not None:
            graph.replay()
        else:
            step_body()

    for s in range(a.warmup):
        run_step(s)
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = Clocks(ctx.local)
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ctx.barrier()
    t0 = time.time()
    e0.record()
    for s in range(a.warmup, total_steps):
        run_step(s)
    e1.record()
    torch.cuda.synchronize()
    t1 = time.time()
    ctx.barrier()
    ms = ctx.max(e0.elapsed_time(e1))
    for lay in layers:
        lay["op"].check()

    # Per-launch sparse-attention timing.  After each step's routing, a CUDA
    # graph holding only the layers' attention launches is replayed between
    # two events on the launching stream (no host gaps inside), and each
    # launch's algorithmic bytes come from that step's routed counts.
    def av_body():
        for l, lay in enumerate(layers):
            lay["op"].attention(q_static[l], lay["K"], lay["V"], length=len_static)

    av_graph = None
    if graph is not None:
        av_graph = torch.cuda.CUDAGraph()
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(av_graph, stream=s_cap):
                av_body()
        torch.cuda.current_stream().wait_stream(s_cap)
        torch.cuda.synchronize()
    av_ms, av_bytes = 0.0, []
    for s in range(a.warmup, total_steps):
        run_step(s)
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record()
        if av_graph is not None:
            av_graph.replay()
        else:
            av_body()
        eb.record()
        torch.cuda.synchronize()
        av_ms += ea.elapsed_time(eb)
        tail = s + 1
        for lay in layers:
            c = int(lay["op"].count.long().sum().item())
            av_bytes.append((c + U * tail) * d * 2 * 2 + 4 * c + 2 * U * G * d * 2)

    # End to end through the public API with host buffers: pinned host
    # queries -> device, full step, outputs -> pinned host, every step.
    h_q = q_steps.cpu().pin_memory()
    h_kv = kv_steps.cpu().pin_memory()
    h_out = torch.empty(L, U, G, d, dtype=torch.bfloat16).pin_memory()
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ctx.barrier()
    ee0.record()
    for s in range(a.warmup, total_steps):
        q_static.copy_(h_q[s], non_blocking=True)
        kv_static.copy_(h_kv[s], non_blocking=True)
        len_static.copy_(lens[s])
        if graph is not None:
            graph.replay()
        else:
            step_body()
        h_out.copy_(outs, non_blocking=True)
    ee1.record()
    torch.cuda.synchronize()
    e2e_ms = ctx.max(ee0.elapsed_time(ee1))
    # Index append (core.py:186-201) at the reference's cadence: a block of
    # update_interval keys per layer every update_interval decode steps.  It
    # is timed on a clone of each layer's index (the decode index stays as
    # built) and its per-step share is added to the step time below.
    append_block_ms = 0.0
    if a.update_interval > 0:
        blk = min(a.update_interval, N)
        sae0 = layers[0]["op"].sae
        warm = layers[0]["idx"].clone()
        warm.append(layers[0]["K"][:, :blk], sae0, 1.0, workspace=ws)   # allocates the append workspace
        del warm
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for lay in layers:
            idx_c = lay["idx"].clone()
            torch.cuda.synchronize()
            ea.record()
            idx_c.append(lay["K"][:, :blk], lay["op"].sae, 1.0, workspace=ws)
            eb.record()
            torch.cuda.synchronize()
            append_block_ms += ea.elapsed_time(eb)
            del idx_c
        torch.cuda.empty_cache()
    append_ms_per_step = append_block_ms / a.update_interval if a.update_interval > 0 else 0.0
    append_ms_per_step = ctx.max(append_ms_per_step)
    clocks.stop()
    clk = clocks.summary(t0, t1)
    encode_paths = sorted({lay["idx"].encode_path for lay in layers})
    parity = None
    if rank == 0 and a.parity_units > 0:
        # Outside every timed region: one decode step of sampled units of
        # layer 0, recomputed by the CPU oracle on this run's own inputs.
        s_last = total_steps - 1
        load_step(s_last)
        lay = layers[0]
        lay["op"].route(q_static[0])
        o = lay["op"].attention(q_static[0], lay["K"], lay["V"], length=len_static)
        torch.cuda.synchronize()
        sample = sorted({0, U - 1})[:a.parity_units]
        parity = sample_parity(lay, q_static[0], o, int(lens[s_last][0].item()), sample, N, F, k, a)
        parity["units"] = [units[u] for u in sample]

    tokens = B * a.steps          # the job decodes the config's B sequences
    decode_ms = ms
    ms = ms + append_ms_per_step * a.steps        # amortised append included
    e2e_ms = e2e_ms + append_ms_per_step * a.steps
    value = tokens / (ms / 1e3)
    e2e = tokens / (e2e_ms / 1e3)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs", 6650.0)
    mean_av_ms = av_ms / len(av_bytes)
    mean_bytes = sum(av_bytes) / len(av_bytes)
    achieved = mean_bytes / (mean_av_ms / 1e3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "sparse_av_traffic.json"
    if tfile.exists():
        try:
            tj = json.loads(tfile.read_text())
            # One ncu capture's DRAM bytes per algorithmic byte, applied to
            # this run's mean launch (same kernel, same per-row traffic).
            traffic = round(tj["dram_bytes_per_algorithmic_byte"] * mean_bytes)
        except (OSError, ValueError, KeyError):
            traffic = None
    # This library's kernels per step, counted in the captured step graph
    # (kernel nodes whose function lives in namespace pk); eager runs fall
    # back to the four launches per layer the step issues.
    launches_per_step = graph_launches if graph_launches is not None else L * 4
    if world == 1:
        partition = "all 32 units on one GPU"
    else:
        partition = f"{U} units per rank ({B * Hkv} units split batch-first over {world} ranks)"
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms / a.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded clustered keys, iid values, random-init SAE)",
        "config": {"workload": "config3: Llama-3-8B-shaped decode attention path, 32 layers",
                   "layers": L, "batch": B, "kv_heads": Hkv, "q_per_kv": G, "head_dim": d,
                   "history": N, "features": F, "query_topk": k, "budget": a.budget, "key_mean": a.key_mean,
                   "router": "q_activation", "update_interval": a.update_interval,
                   "graph": graph is not None, "l2": "inputs larger than L2 (KV and index per step >> 126 MB)",
                   "parallelism": f"batch x kv-heads over {world} GPU(s): {partition}",
                   "units_per_gpu": U, "setup_s": round(setup_s, 1), "build_s": round(build_s, 1),
                   "decode_ms_per_step": round(decode_ms / a.steps, 4),
                   "append_ms_per_block": round(append_block_ms, 3),
                   "append_ms_per_step": round(append_ms_per_step, 5),
                   "step": "32 x (route + union + sparse attention with the token's KV append) per token of each "
                           "of the B sequences, plus the amortised index append of an update_interval block per "
                           "layer every update_interval tokens"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "sparse_av_bf16_kernel", "avg_launch_us": round(mean_av_ms * 1e3, 2),
                     "algorithmic_bytes_per_launch": int(mean_bytes),
                     "share_of_step": round(av_ms / a.steps / (ms / a.steps), 3),
                     "peak_source": "measured" if "hbm_gbs" in peaks else "fallback"},
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(L * U * G * d * 2 + L * 2 * U * d * 2) * world,
                "d2h_bytes_per_step": int(L * U * G * d * 2) * world},
        "gpu_launches": launches_per_step * a.steps,
        "gpu_launches_source": "graph kernel nodes" if graph_launches is not None else
                               "per-layer launch count" + (f" ({GRAPH_INSPECT_ERRORS[0]})" if GRAPH_INSPECT_ERRORS
                                                           else ""),
        "clocks": clk,
        "encode_path": encode_paths[0] if len(encode_paths) == 1 else encode_paths,
        "parity": parity,
    }
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_rate(a, seconds=a.cpu_seconds)
    # The config-4 sequence-sharded step on the same ranks (its NCCL
    # all-gather is the path's one collective), after this config's memory
    # is released.
    del graph, av_graph, layers, kv_steps, q_steps, outs, h_q, h_kv
    ws.buffers.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if not a.no_seqshard:
        line["seqshard"] = seqshard_measure(a, ctx)
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


# ---------------------------------------------------------------------------
# sampled-unit parity against the CPU oracle (outside the timed region)
# ---------------------------------------------------------------------------

def sample_parity(lay, q, out, length, units, N, F, k, a) -> dict:
    """Recomputes one decode step of `units` of one layer with the CPU
    oracle on the bench's own inputs: the unit's index from its keys (the
    whole-history global BatchTopK, core.py:92-103), the q_activation order
    (core.py:131-139), the budgeted union (core.py:142-167) and the attention
    over the union and the dense tail (core.py:170-183).  Memberships, order,
    union ids and accepted buckets must be bit-exact; the attention within
    2e-2 relative L2 (bf16)."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import oracle

    op, idx = lay["op"], lay["idx"]
    t0 = time.time()
    sae = oracle.SAE(op.sae.W_enc.float().cpu().numpy(), op.sae.b_enc.float().cpu().numpy(), key_mean=a.key_mean,
                     query_topk=k)
    res = {"units": list(units), "layer": 0, "memberships": True, "order": True, "ids": True, "features": True,
           "attn_rel_l2": 0.0}
    for u in units:
        keys = lay["K"][u, :length].float().cpu().numpy()
        vals = lay["V"][u, :length].float().cpu().numpy()
        qu = q[u].float().cpu().numpy()
        oidx = oracle.build_index(keys[:N], sae, 1.0, moments=False)
        counts, mem = idx.csr(u)
        res["memberships"] &= bool(np.array_equal(counts, oidx.counts) and np.array_equal(mem, oidx.ids))
        _, order = oracle.bucket_scores(qu, oidx, router="q_activation", sae=sae, query_scale=1.0, query_topk=k)
        n_order = int(op.n_order[u].item())
        res["order"] &= bool(np.array_equal(op.order[u, :n_order].long().cpu().numpy(), order))
        ids, feats, _ = oracle.select_from_order(order, oidx, int(op.limit[u].item()))
        c = int(op.count[u].item())
        res["ids"] &= bool(np.array_equal(op.ids[u, :c].long().cpu().numpy(), ids))
        nf = int(op.n_features[u].item())
        res["features"] &= op.features[u, :nf].long().cpu().tolist() == feats
        ref = oracle.attend(qu, keys, vals, ids, N)
        got = out[u].float().cpu().numpy().astype(np.float64)
        err = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
        res["attn_rel_l2"] = max(res["attn_rel_l2"], round(err, 6))
    res["ok"] = bool(res["memberships"] and res["order"] and res["ids"] and res["features"]
                     and res["attn_rel_l2"] < 2e-2)
    res["oracle_s"] = round(time.time() - t0, 1)
    return res


# ---------------------------------------------------------------------------
# CPU: the reference path restated by the oracle, on a bounded sample
# ---------------------------------------------------------------------------

def _oracle_decode_time(N, F, d, G, k, C, key_mean, budget, tail, n_units, seconds, seed=1234):
    """Seconds per batch of n_units units for the oracle's route + select +
    attend (q_activation), one unit per host thread.  Each unit's bucket
    index is a synthetic CSR with key_mean memberships per token (its build
    is not timed).  Returns (seconds per batch, reps)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import oracle
    from gen import bf16_round

    rs = np.random.RandomState(seed)
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    sae = oracle.SAE(W, np.zeros(F, np.float32), key_mean=key_mean, query_topk=k)
    units = []
    for u in range(n_units):
        centers = rs.standard_normal((C, d)).astype(np.float32)
        cid = rs.randint(0, C, N + tail)
        keys = bf16_round(centers[cid] + np.float32(0.3) * rs.standard_normal((N + tail, d)).astype(np.float32))
        vals = bf16_round(rs.standard_normal((N + tail, d)).astype(np.float32))
        q = bf16_round(centers[rs.randint(0, C, G)] + np.float32(0.3) * rs.standard_normal((G, d)).astype(np.float32))
        feats = rs.randint(0, F, size=(N, key_mean))
        tok = np.repeat(np.arange(N), key_mean)
        order = np.lexsort((tok, feats.reshape(-1)))
        fs, ts = feats.reshape(-1)[order], tok[order]
        keep = np.ones(len(fs), bool)
        keep[1:] = (fs[1:] != fs[:-1]) | (ts[1:] != ts[:-1])
        fs, ts = fs[keep], ts[keep]
        counts = np.bincount(fs, minlength=F).astype(np.int64)
        offsets = np.zeros(F + 1, np.int64)
        np.cumsum(counts, out=offsets[1:])
        idx = oracle.FeatureIndex(N, np.zeros(d, np.float32), counts, None, None, offsets, ts.astype(np.int64))
        units.append((q, keys, vals, idx))
    cap = budget / N

    def one(unit):
        q, keys, vals, idx = unit
        ids, _ = oracle.select_buckets(q, idx, unique_cap=cap, router="q_activation", sae=sae, query_scale=1.0,
                                       query_topk=k)
        oracle.attend(q, keys, vals, ids, N)

    reps, t_total = 0, 0.0
    with ThreadPoolExecutor(max_workers=n_units) as ex:
        list(ex.map(one, units))  # warm
        while t_total < seconds or reps == 0:
            t0 = time.perf_counter()
            list(ex.map(one, units))
            t_total += time.perf_counter() - t0
            reps += 1
    return t_total / reps, reps


def cpu_rate(a, seconds: float = 10.0) -> dict:
    """Times the oracle's route + select + attend for a sample of config-3
    units on the host cores (one unit per thread) and scales to a full
    decode step (all units x layers).  The sample's bucket index is a
    synthetic CSR with key_mean memberships per token (its build is not
    timed)."""
    cores = os.cpu_count() or 1
    n_units = max(1, min(cores, a.batch * a.kv_heads))
    N, F, d, G, k = a.history, a.features, 128, a.q_per_kv, a.query_topk
    tail = 128
    per_batch, reps = _oracle_decode_time(N, F, d, G, k, a.clusters, a.key_mean, a.budget, tail, n_units, seconds)
    U_total = a.batch * a.kv_heads * a.layers
    step_s = per_batch * U_total / n_units
    return {"value": round(a.batch / step_s, 4), "unit": "tokens/s", "cores": n_units, "kind": "port",
            "sample": f"{n_units} config-3 units (history {N}, F {F}, k {k}, budget {a.budget}, tail {tail}) "
                      f"x {reps} reps, one unit per thread, scaled to {U_total} units per step; synthetic CSR "
                      f"index, build not timed"}


def cpu_stage_rate(seconds: float = 10.0, build_keys: int = 4096) -> dict:
    """Config 2 on the host cores through the oracle port: one decode
    layer-step (route + select + attend of all 128 units, timed on a sample
    of units, one unit per thread, scaled to 128) and the index build of one
    unit on a sample of build_keys keys (the C restatement's own threads),
    reported as keys/s."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import oracle

    cores = os.cpu_count() or 1
    U, N, F, d, G, k, Bt, C, tail = 128, 32768, 8192, 128, 4, 32, 2048, 1024, 16
    n_units = max(1, min(cores, U))
    per_batch, reps = _oracle_decode_time(N, F, d, G, k, C, 8, Bt, tail, n_units, seconds)
    layer_us = per_batch * U / n_units * 1e6
    rs = np.random.RandomState(4321)
    W = (rs.standard_normal((F, d)) / np.sqrt(d)).astype(np.float32)
    sae = oracle.SAE(W, np.zeros(F, np.float32), key_mean=8, query_topk=k)
    centers = rs.standard_normal((C, d)).astype(np.float32)
    keys = centers[rs.randint(0, C, build_keys)] + np.float32(0.3) * rs.standard_normal((build_keys, d)).astype(
        np.float32)
    t0 = time.perf_counter()
    oracle.build_index(keys, sae, 1.0, moments=False)
    build_s = time.perf_counter() - t0
    return {"value": round(layer_us, 1), "unit": "us", "cores": n_units, "kind": "port",
            "build_keys_per_s": round(build_keys / build_s, 1), "build_threads": oracle.num_threads(),
            "sample": f"decode: {n_units} config-2 units (history {N}, F {F}, k {k}, budget {Bt}, tail {tail}) x "
                      f"{reps} reps, one unit per thread, scaled to {U} units per layer-step, synthetic CSR index; "
                      f"build: one unit of {build_keys} clustered keys, F {F}, key_mean 8, "
                      f"{oracle.num_threads()} threads"}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = cpu_rate(a, seconds=max(1.0, a.cpu_seconds))
    line = {"metric": METRIC, "value": base["value"], "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config3: Llama-3-8B-shaped decode attention path, 32 layers",
                       "history": a.history, "features": a.features, "budget": a.budget},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# config 4: million-token single-layer decode, KV cache sequence-sharded
# ---------------------------------------------------------------------------

def seqshard_measure(a, ctx) -> dict:
    """Config 4: B=1, 32/8 heads (U = 8 units of 4 query heads), context
    1048576, F = 32768, 64 features per query, budget 8192, clustered keys
    with 4096 clusters.  Rank r of P holds tokens [r*N/P, (r+1)*N/P) of every
    unit and its shard of the bucket index (built with the whole sequence's
    exact BatchTopK, build_sharded); a decode step routes (replicated),
    unions its shard's buckets with budget 8192/P, attends over its rows and
    merges the P log-sum-exp partials after one NCCL all-gather.  The total
    context is fixed: strong scaling.  Returns the measurement as a dict."""
    import torch
    import prismkv_b200 as pk
    from prismkv_b200 import native as nv
    from prismkv_b200.shard import ShardedDecode, build_sharded, token_ranges

    world, rank, local, dev = ctx.world, ctx.rank, ctx.local, ctx.dev
    barrier, max_over_ranks = ctx.barrier, ctx.max
    B, Hkv, G, d = 1, 8, 4, 128
    U = B * Hkv
    N, F, k, budget, C = 1 << 20, 32768, 64, 8192, 4096
    steps_total = a.warmup + a.steps
    lo, hi = token_ranges(N, world)[rank]
    tail = steps_total if rank == world - 1 else 0
    n_local = hi - lo
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed * 7919 + 1)
    centers = torch.randn(U, C, d, device=dev, generator=g)
    W = torch.randn(F, d, device=dev, generator=g) / math.sqrt(d)
    Q = (centers[torch.arange(U, device=dev)[None, :, None],
                 torch.randint(0, C, (steps_total, U, G), device=dev, generator=g)]
         + 0.3 * torch.randn(steps_total, U, G, d, device=dev, generator=g)).to(torch.bfloat16)
    g.manual_seed(a.seed * 7919 + 1000 + rank)
    T = n_local + tail
    K = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    V = torch.empty(U, T, d, device=dev, dtype=torch.bfloat16)
    for c0 in range(0, T, 16384):
        c1 = min(T, c0 + 16384)
        cid = torch.randint(0, C, (U, c1 - c0), device=dev, generator=g)
        cc = torch.gather(centers, 1, cid[:, :, None].expand(U, c1 - c0, d))
        K[:, c0:c1] = (cc + 0.3 * torch.randn(U, c1 - c0, d, device=dev, generator=g)).to(torch.bfloat16)
        V[:, c0:c1] = torch.randn(U, c1 - c0, d, device=dev, generator=g).to(torch.bfloat16)
    sae = pk.SAEParams(W, torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    ws = nv.Workspace(dev)
    torch.cuda.synchronize()
    tb = time.time()
    # The exact global BatchTopK over all N tokens (one device's build),
    # each rank keeping its shard: histogram all-reduces and one all-gather.
    idx = build_sharded(K[:, :n_local], sae, 1.0, lo=lo, N_total=N, workspace=ws)
    torch.cuda.synchronize()
    build_s = time.time() - tb
    for key in [k_ for k_ in ws.buffers if isinstance(k_, tuple) and k_[0] in ("build", "shard_build")]:
        del ws.buffers[key]
    torch.cuda.empty_cache()
    sd = ShardedDecode(idx, sae, heads_per_unit=G, budget=budget, max_history=n_local, workspace=ws,
                       exchange=a.exchange, split_route=a.split_route or None)
    q_static = Q[0].clone()
    len_static = torch.full((U,), n_local + (1 if tail else 0), dtype=torch.int32, device=dev)

    out_static = [None]

    def body():
        out_static[0] = sd(q_static, K, V, length=len_static)

    # The step (route, union, attention, the all-gather of partials, the
    # merge) replayed as one CUDA graph, captured after eager warm-up steps
    # (which also set up the NCCL communicator).
    graph = [None]

    def step(s):
        q_static.copy_(Q[s])
        len_static.fill_(n_local + (s + 1 if tail else 0))
        if graph[0] is not None:
            graph[0].replay()
        else:
            body()
        return out_static[0]

    for s_ in range(a.warmup):
        step(s_)
    torch.cuda.synchronize()
    sd.check()
    barrier()
    launches = None
    if not a.no_graph:
        graph[0] = torch.cuda.CUDAGraph(keep_graph=True)
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(graph[0], stream=s_cap):
                body()
        torch.cuda.current_stream().wait_stream(s_cap)
        graph[0].instantiate()
        torch.cuda.synchronize()
        launches = graph_kernel_launches(graph[0])
        barrier()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    t0 = time.time()
    e0.record()
    for s_ in range(a.warmup, steps_total):
        out = step(s_)
    e1.record()
    torch.cuda.synchronize()
    t1 = time.time()
    ms = max_over_ranks(e0.elapsed_time(e1))
    # End to end with host buffers: the query in, the merged output out.
    h_q = Q.cpu().pin_memory()
    h_out = torch.empty(U, G, d, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    barrier()
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ee0.record()
    for s_ in range(a.warmup, steps_total):
        q_static.copy_(h_q[s_], non_blocking=True)
        len_static.fill_(n_local + (s_ + 1 if tail else 0))
        if graph[0] is not None:
            graph[0].replay()
        else:
            body()
        h_out.copy_(out_static[0], non_blocking=True)
    ee1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(ee0.elapsed_time(ee1))
    clocks.stop()
    sd.check()
    tokens = B * a.steps
    out = {
        "metric": "config4 decode tokens/s at 1M ctx (sequence-sharded)", "value": round(tokens / (ms / 1e3), 2),
        "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True, "scaling": "strong",
        "config": {"workload": "config4: 1M-token single-layer decode, KV cache sequence-sharded",
                   "batch": B, "kv_heads": Hkv, "q_per_kv": G, "history": N, "features": F, "query_topk": k,
                   "budget": budget, "budget_per_shard": budget // world, "clusters": C,
                   "tokens_per_shard": n_local, "build_s": round(build_s, 2),
                   "index_build": "exact BatchTopK over the whole sequence (build_sharded)",
                   "routing": "split by features over the ranks" if sd.split_route else "replicated on every rank",
                   "parallelism": f"seq{world}", "graph": graph[0] is not None,
                   "collective": (("all-gathers of the routing picks and of the (m, l, o) partials, one of each "
                                   "per step" if sd.split_route else "one all-gather of the (m, l, o) partials per step")
                                  + f", over {'NVLink peer memory (pk_p2p_allgather)' if sd.exchange == 'p2p' else 'NCCL'}")
                                 if world > 1 else None,
                   "l2": "KV rows gathered per step are scattered over >> L2"},
        "e2e": {"value": round(tokens / (e2e_ms / 1e3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(U * G * d * 2) * world, "d2h_bytes_per_step": int(U * G * d * 2) * world},
        "gpu_launches": launches * a.steps if launches is not None else None,
        "clocks": clocks.summary(t0, t1),
    }
    graph[0] = None   # a graph holding NCCL calls is released before the group
    sd.close()        # the peer-memory exchanges (collective)
    del sd, idx, K, V
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def run_seqshard(a):
    """bench.py --config 4: the config-4 step alone, as its own JSON line."""
    ctx = Ranks()
    line = seqshard_measure(a, ctx)
    line.update(vs_baseline=None, dtype="bf16", data="synthetic (seeded clustered keys, iid values, random-init SAE)")
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


# ---------------------------------------------------------------------------
# config 5: prefill bucket build of a 32-layer x 8-KV-head cache, budget sweep
# ---------------------------------------------------------------------------

def run_build_sweep(a):
    """Config 5: every layer's keys (B = 8 sequences x 8 KV heads = 64 units,
    context 65536, bf16) are SAE-encoded (F = 16384, a 128 x 16384 product
    per key) and bucketed with the global top-8 per key; then one layer
    decodes with union budgets 512..8192 and its sparse attention is timed
    per budget.  Build throughput is reported as keys/s and as the tensor
    work of the encode (2*N*F*d FLOP per unit) per second."""
    import torch
    import prismkv_b200 as pk
    from prismkv_b200 import native as nv

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L, B, Hkv, G, d = a.layers, 8, 8, 4, 128
    U = B * Hkv
    N, F, k, C = 65536, 16384, 32, a.clusters
    g = torch.Generator(device=dev)
    ws = nv.Workspace(dev)
    build_ms = []
    K = V = centers = idx = sae = None
    for l in range(L):
        g.manual_seed(a.seed * 1_000_003 + 500 + l)
        centers, K, V = gen_layer(torch, dev, g, U, N + 16, d, C)
        W = torch.randn(F, d, device=dev, generator=g) / math.sqrt(d)
        sae = pk.SAEParams(W, torch.zeros(F, device=dev), key_mean=8, query_topk=k)
        sae.prepared_half()
        if l == 0:   # allocate the build workspace untimed
            pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws)
        e1.record()
        torch.cuda.synchronize()
        build_ms.append(e0.elapsed_time(e1))
        if idx.encode_path != "bounds":
            raise SystemExit("build fell back to the exact path")
    total_ms = sum(build_ms)
    flop = 2.0 * U * N * F * d * L
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    # Decode budget sweep on the last layer.
    q = gen_queries(torch, dev, g, centers, 1, G)[0].contiguous()
    sweep = []
    for budget in (512, 1024, 2048, 4096, 8192):
        op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=budget, workspace=nv.Workspace(dev))
        op.route(q)
        op.attention(q, K, V)
        torch.cuda.synchronize()
        op.check()
        graph = torch.cuda.CUDAGraph()
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        reps = 20
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(graph, stream=s_cap):
                for _ in range(reps):
                    op.attention(q, K, V)
        torch.cuda.current_stream().wait_stream(s_cap)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        cnt = int(op.count.long().sum().item())
        byts = (cnt + U * 16) * d * 2 * 2 + 4 * cnt + 2 * U * G * d * 2
        sweep.append({"budget": budget, "attention_us": round(us, 2), "rows": cnt + U * 16,
                      "GB_s": round(byts / us / 1e3, 1),
                      "frac_of_measured_hbm": round(byts / us / 1e3 / peaks.get("hbm_gbs", 6650.0), 4)})
        del graph
    line = {
        "metric": "config5 prefill bucket build keys/s; decode sparse-AV GB/s per budget",
        "value": round(U * N * L / (total_ms / 1e3), 1), "unit": "keys/s", "n_gpus": 1, "steps": L,
        "warmup": 1, "ms_per_step": round(total_ms / L, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded clustered keys, iid values, random-init SAE)",
        "config": {"workload": "config5: 32 layers x 64 units x 65536 keys, F=16384, top-8 per key; budget sweep",
                   "layers": L, "units_per_layer": U, "context": N, "features": F, "key_mean": 8,
                   "build_ms_per_layer": [round(x, 2) for x in build_ms[:4]],
                   "encode_tflops": round(flop / (total_ms / 1e3) / 1e12, 1),
                   "encode_frac_of_measured_bf16": round(flop / (total_ms / 1e3) / 1e12 /
                                                         (peaks.get("bf16_tflops", 1590.0)), 4),
                   "decode_sweep": sweep},
        "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


def run_stages(a):
    """Config 2: one bf16 layer of B = 16 sequences x 8 KV heads (128 units),
    context 32768, F = 8192, 8 features per key, 32 per query, budget 2048;
    routing (q_activation encode + top-k + aggregation), union and sparse
    attention are each timed alone (CUDA-graph replay of 20 calls), then the
    layer's index build.  Attention is reported against the measured HBM
    copy peak; routing as the FP32-equivalent encode rate (2*F*d FLOP per
    query head) and its W read."""
    import torch
    import prismkv_b200 as pk
    from prismkv_b200 import native as nv

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    B, Hkv, G, d = 16, 8, 4, 128
    U = B * Hkv
    N, F, k, Bt, C, tail = 32768, 8192, 32, 2048, 1024, 16
    g = torch.Generator(device=dev)
    g.manual_seed(a.seed * 1_000_003 + 200)
    centers, K, V = gen_layer(torch, dev, g, U, N + tail, d, C)
    W = torch.randn(F, d, device=dev, generator=g) / math.sqrt(d)
    sae = pk.SAEParams(W, torch.zeros(F, device=dev), key_mean=8, query_topk=k)
    sae.prepared_half()
    ws = nv.Workspace(dev)
    pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws)   # workspace, untimed
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws)
    e1.record()
    torch.cuda.synchronize()
    build_ms = e0.elapsed_time(e1)
    if idx.encode_path != "bounds":
        raise SystemExit("build fell back to the exact path")
    q = gen_queries(torch, dev, g, centers, 1, G)[0].contiguous()
    op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=Bt, workspace=ws)
    lt = torch.full((U,), N + tail, dtype=torch.int32, device=dev)
    Wb, wn = op.prep
    nbytes = nv.query("pk_route_qact_workspace_bytes", U, G, F, k)
    rws = ws.get(("qact", U, G, F, k), nbytes)

    def route_only():
        nv.call("pk_route_qact", q, nv.dtype_code(q), None, U, sae.W_enc, sae.b_enc, Wb, wn, 1.0, idx.lens, U, G, d,
                F, k, rws, nbytes, op.order, op.n_order, op.width, None, None)

    def union_only():
        nv.call("pk_union", idx.offsets, idx.lens, idx.ids, idx.ids.stride(0), op.order, op.n_order, op.width,
                op.history, op.limit, U, F, op.max_history, op.ids, op.ids.shape[1], op.count, op.features,
                op.n_features, op.raw, op.status)

    def attn_only():
        op.attention(q, K, V, length=lt)

    def timed(fn, reps=20):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(graph, stream=s_cap):
                for _ in range(reps):
                    fn()
        torch.cuda.current_stream().wait_stream(s_cap)
        graph.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(max(3, a.steps // 10)):
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e3 / reps)
        del graph
        return best

    route_us = timed(route_only)
    union_us = timed(union_only)
    attn_us = timed(attn_only)
    layer_us = timed(lambda: (route_only(), union_only(), attn_only()))
    op.check()
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    cnt = int(op.count.long().sum().item())
    av_bytes = (cnt + U * tail) * d * 2 * 2 + 4 * cnt + 2 * U * G * d * 2
    route_flop = 2.0 * F * d * U * G
    line = {
        "metric": "config2 isolated stage times (routing, union, sparse-AV) per layer-step",
        "value": round(layer_us, 2), "unit": "us", "n_gpus": 1, "steps": 20, "warmup": 1,
        "ms_per_step": round(layer_us / 1e3, 4), "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded clustered keys, iid values, random-init SAE)",
        "config": {"workload": "config2: 128 units, context 32768, F=8192, k=32, budget 2048 (CUDA-graph replay, "
                               "20 calls per stage)",
                   "route_us": round(route_us, 2), "union_us": round(union_us, 2),
                   "attention_us": round(attn_us, 2), "attention_rows": cnt + U * tail,
                   "attention_GB_s": round(av_bytes / attn_us / 1e3, 1),
                   "attention_frac_of_measured_hbm": round(av_bytes / attn_us / 1e3 / hbm, 4),
                   "routing_fp32_equiv_tflops": round(route_flop / route_us / 1e6, 2),
                   "routing_W_read_GB_s": round(F * d * 2 / route_us / 1e3, 1),
                   "union_unique_tokens_per_unit": round(cnt / U, 1),
                   "build_ms": round(build_ms, 2), "build_keys_per_s": round(U * N / (build_ms / 1e3), 1)},
        "gpu_launches": None,
    }
    if not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_stage_rate(seconds=a.cpu_seconds)
    print(json.dumps(line), flush=True)


def run_layout(a):
    """Layout diagnostic at config-3 shape (single.py:24-67): per layer, route
    once, then CUDA-graph replay over the layers of the in-place sparse
    attention, the explicit gather of the routed rows and tail into a packed
    copy (pk_gather_kv), attention over the packed copy, and both together.
    Eight layers (the selected rows of a pass, ~540 MB, far exceed L2).  The
    gather's read rate is the HBM rate of random 256-byte rows: the ceiling
    of the in-place attention's traffic."""
    import torch
    import prismkv_b200 as pk
    from prismkv_b200 import native as nv
    from prismkv_b200.layout import layout_probe, gather_kv

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L = min(a.layers, 8)
    U, G, d = a.batch * a.kv_heads, a.q_per_kv, 128
    N, F, k, tail = a.history, a.features, a.query_topk, 128
    g = torch.Generator(device=dev)
    ws = nv.Workspace(dev)
    layers = []
    for l in range(L):
        g.manual_seed(a.seed * 1_000_003 + 700 + l)
        centers, K, V = gen_layer(torch, dev, g, U, N + tail, d, a.clusters)
        W = torch.randn(F, d, device=dev, generator=g) / math.sqrt(d)
        sae = pk.SAEParams(W, torch.zeros(F, device=dev), key_mean=a.key_mean, query_topk=k)
        idx = pk.DeviceIndex.build(K[:, :N], sae, 1.0, moments=False, workspace=ws)
        op = pk.SparseDecode(idx, sae, heads_per_unit=G, budget=a.budget, workspace=nv.Workspace(dev))
        q = gen_queries(torch, dev, g, centers, 1, G)[0].contiguous()
        op.route(q)
        layers.append((op, q, K, V))
    torch.cuda.synchronize()
    length = torch.full((U,), N + tail, dtype=torch.int32, device=dev)
    checks = [layout_probe(op, q, K, V, length, reps=2) for op, q, K, V in layers]   # bit-exact check per layer
    rows = sum(c["rows"] for c in checks)
    P = max(c["packed_rows"] for c in checks)
    packed = [gather_kv(K, V, op.ids, op.count, op.history, length, P) for op, q, K, V in layers]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    S = max(1, min(8, (2 * sms) // U))
    ident = torch.arange(P, dtype=torch.int32, device=dev).repeat(U, 1).contiguous()
    nbytes = nv.query("pk_sparse_av_workspace_bytes", U, G, d, S)
    out = torch.empty(U, G, d, dtype=torch.bfloat16, device=dev)

    def indexed():
        for op, q, K, V in layers:
            op.attention(q, K, V, length=length, splits=S)

    def gather():
        for (op, q, K, V), (pk_, pv_) in zip(layers, packed):
            nv.call("pk_gather_kv", K, V, nv.PK_BF16, 1, K.stride(0), 0, K.stride(1), op.ids, op.ids.stride(0),
                    op.count, op.history, length, U, d, P, pk_, pv_, None)

    def prepacked():
        for (op, q, K, V), (pk_, pv_) in zip(layers, packed):
            p_len = op.count + (length - op.history)
            nv.call("pk_sparse_av", q, pk_, pv_, nv.PK_BF16, 1, pk_.stride(0), 0, pk_.stride(1), ident, P, op.count,
                    op.count, p_len, U, G, d, S, op.ws.get(("av", U, G, d, S), nbytes), nbytes, out, None)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        s_cap = torch.cuda.Stream()
        s_cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s_cap):
            with torch.cuda.graph(graph, stream=s_cap):
                fn()
        torch.cuda.current_stream().wait_stream(s_cap)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(max(3, a.steps // 10)):
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) * 1e3 / L)
        del graph
        return best

    us = {"indexed_av": timed(indexed), "prepacked_av": timed(prepacked), "explicit_gather": timed(gather),
          "gather_and_av": timed(lambda: (gather(), prepacked()))}
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    row_bytes = rows / L * d * 2 * 2            # K + V rows per layer
    line = {
        "metric": "layout probe: in-place sparse attention vs explicit gather + packed attention per layer",
        "value": round(us["indexed_av"], 2), "unit": "us", "n_gpus": 1, "steps": L, "warmup": 1,
        "ms_per_step": round(us["indexed_av"] / 1e3, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded clustered keys, iid values, random-init SAE)",
        "config": {"workload": f"config-3 layer shape x {L} layers (U={U}, history {N}, tail {tail}, budget "
                               f"{a.budget}); CUDA-graph replay over the layers",
                   "us_per_layer": {k_: round(v_, 2) for k_, v_ in us.items()},
                   "identical_outputs": all(c["identical"] for c in checks),
                   "rows_per_layer": rows // L,
                   "gather_read_GB_s": round(row_bytes / us["explicit_gather"] / 1e3, 1),
                   "gather_read_plus_write_GB_s": round(2 * row_bytes / us["explicit_gather"] / 1e3, 1),
                   "gather_read_plus_write_frac_of_measured_hbm":
                       round(2 * row_bytes / us["explicit_gather"] / 1e3 / hbm, 4),
                   "indexed_av_GB_s": round(row_bytes / us["indexed_av"] / 1e3, 1),
                   "indexed_av_frac_of_gather_rate": round(us["explicit_gather"] / us["indexed_av"], 4)},
        "gpu_launches": None,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    args = parse()
    if args.impl == "ours" and args.layout:
        run_layout(args)
        sys.exit(0)
    if args.impl == "ours" and args.config == 2:
        run_stages(args)
        sys.exit(0)
    if args.impl == "ours" and args.config == 4:
        run_seqshard(args)
        sys.exit(0)
    if args.impl == "ours" and args.config == 5:
        run_build_sweep(args)
        sys.exit(0)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
