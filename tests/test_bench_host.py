"""Host logic of bench.py, on CPU: the workload draw behind sequence sharding (one seeded draw
of 64 sequences per GPU, split across ranks balanced by tokens, so no data crosses GPUs), the
algorithmic byte count the headline metric divides by, and the reference arm's JSON line
(rank 0 prints it; other ranks exit 0 without work)."""
import json
import os
import subprocess
import sys

import numpy as np

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_workload_draw_is_one_job_split_by_tokens():
    one, layers = bench.workload_lengths("config4", 0, 0, 1)
    assert layers == 8 and len(one) == 64 and one.min() >= 1024 and one.max() <= 65536
    again, _ = bench.workload_lengths("config4", 0, 0, 1)
    assert np.array_equal(one, again)  # reproducible
    for world in (2, 4, 8):
        parts = [bench.workload_lengths("config4", r, 0, world)[0] for r in range(world)]
        assert all(len(p) == 64 for p in parts)  # 64 sequences per GPU: weak scaling
        allx = np.sort(np.concatenate(parts))
        draw = np.sort(np.random.default_rng(0).integers(1024, 65537, 64 * world))
        assert np.array_equal(allx, draw)  # one global draw, every sequence on exactly one rank
        tokens = [int(p.sum()) for p in parts]
        # largest-first onto the lightest rank: the heaviest rank is within one sequence's
        # length of the lightest
        assert max(tokens) - min(tokens) <= 65536
        assert max(tokens) / (sum(tokens) / world) < 1.01
    total = sum(int(bench.workload_lengths("config4", r, 0, 8)[0].sum()) for r in range(8))
    assert 14e6 < total < 20e6  # 512 sequences (config 5a): E = 512 * 33280 = 17.04 M tokens


def test_balanced_partition_caps_and_balances():
    lens = np.array([10, 9, 8, 7, 6, 5, 4, 3], dtype=np.int64)
    owner = bench.balanced_partition(lens, 2, 4)
    assert sorted(np.bincount(owner)) == [4, 4]
    assert abs(lens[owner == 0].sum() - lens[owner == 1].sum()) <= 2


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
    # the same metric, unit and direction as our arm's line, so the two compare
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert "all 8 sequences" in line["cpu_baseline"]["sample"]


def test_reference_arm_other_ranks_are_silent():
    r = _run_reference({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
