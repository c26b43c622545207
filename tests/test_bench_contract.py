"""bench.py's reference arm (CPU): the JSON line the driver reads, and the
torchrun contract that only rank 0 runs and prints it.  Small shapes keep the
oracle's sample to a second or two."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
SMALL = ["--history", "4096", "--features", "1024", "--query-topk", "16", "--budget", "512", "--clusters", "64",
         "--batch", "1", "--kv-heads", "2", "--layers", "2", "--steps", "1", "--warmup", "0", "--cpu-seconds", "0.2"]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *SMALL], cwd=ROOT,
                          env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0"})
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tokens/s"
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_unit_partition_splits_batch_then_kv_heads():
    """bench.py --gpus N spreads config 3's 4 x 8 units batch-first: 2 and 4
    ranks split the batch, 8 ranks split it 4 ways and the KV heads 2 ways."""
    import bench
    B, H = 4, 8
    for world in (1, 2, 4, 8):
        parts = [bench.unit_partition(B, H, world, r) for r in range(world)]
        assert sorted(u for p in parts for u in p) == list(range(B * H))
        assert all(len(p) == B * H // world for p in parts)
    eight = [bench.unit_partition(B, H, 8, r) for r in range(8)]
    for r, p in enumerate(eight):
        assert {u // H for u in p} == {r // 2}                     # one sequence
        assert {u % H for u in p} == set(range(4 * (r % 2), 4 * (r % 2) + 4))   # half its KV heads
