"""Host logic of bench.py, on CPU: the per-rank workload draw behind sequence sharding (every
rank owns an independent, reproducible set of 64 sequences, so no data crosses GPUs), the
algorithmic byte count the headline metric divides by, and the reference arm's JSON line
(rank 0 prints it; other ranks exit 0 without work)."""
import json
import os
import subprocess
import sys

import numpy as np

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_workload_draw_per_rank():
    for rank in range(8):
        lens, layers = bench.workload_lengths("config4", rank, 0)
        assert layers == 8 and len(lens) == 64
        assert lens.min() >= 1024 and lens.max() <= 65536
        again, _ = bench.workload_lengths("config4", rank, 0)
        assert np.array_equal(lens, again)  # reproducible
    draws = [tuple(bench.workload_lengths("config4", r, 0)[0]) for r in range(8)]
    assert len(set(draws)) == 8  # independent sequences per rank
    total = sum(sum(d) for d in draws)  # 512 sequences: the config-5a job at N=8
    assert 14e6 < total < 20e6  # E = 512 * 33280 = 17.04 M tokens


def test_step_bytes_is_the_kv_formula_plus_row_io():
    lens = np.array([1024, 4097, 65536], dtype=np.int64)
    total, kv = bench.step_bytes(lens, 8)
    assert kv == 8 * sum(int(L) + 1 for L in lens) * 4 * 256 * 2 * 2
    per_seq_io = 16 * 512 * 2 + 2 * 4 * 256 * 2 + 16 * 256 * 2 + 16 * 256 * 2 + 4 * 256 * 2 * 2
    assert total - kv == 8 * len(lens) * per_seq_io


def _run_reference(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "small",
                           "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_line():
    r = _run_reference({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"]
    for key in ("metric", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_reference_arm_other_ranks_are_silent():
    r = _run_reference({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
