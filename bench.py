"""Benchmark of the Peregrine KV-cache decode hot path on B200 (one JSON line on rank 0).

Workload ("batched paged decode"): per GPU 64 sequences with context
lengths ~ U[1024, 65536] (seeded per rank), 8 full-attention layers, 16q/4kv heads, d=256,
bf16 K/V in 16-token pages whose block tables are a random permutation over one pool per
layer sized to the total tokens. One step = for each of the 8 layers: append one new K/V row
per sequence with RMSNorm + partial RoPE (pgc_append_kv_rope, packed q|gate input), then
split-K paged decode attention with the sigmoid gate (pgc_decode_attn). At N GPUs every rank
runs its own 64 sequences with its own pools (sequence sharding, BASELINE config 5a at N=8:
512 sequences), no collective on the data path: weak scaling.

Metric: achieved HBM GB/s of the step's algorithmic bytes (K+V read of every cached token
incl. the appended one, plus q/gate/out and the appended rows), whole job, and decode tok/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config4|small]

--impl reference times the reference path's CPU restatement (the Zig/Metal reference cannot
be built or run on Linux) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D, NQ, NKV, PAGE = 256, 16, 4, 16
LAYERS = 8
SCALE = 1.0 / 16
KV_BYTES_PER_TOKEN = NKV * D * 2 * 2  # K + V per layer


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4", choices=["config4", "small"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def workload_lengths(workload: str, rank: int, seed: int):
    import numpy as np
    rng = np.random.default_rng(seed * 1000003 + rank)
    if workload == "small":
        return rng.integers(1024, 8193, 8).astype(np.int64), 2
    return rng.integers(1024, 65537, 64).astype(np.int64), LAYERS


def step_bytes(lens, layers):
    B = len(lens)
    kv = int(sum(int(L) + 1 for L in lens)) * KV_BYTES_PER_TOKEN
    per_layer_io = B * (NQ * 2 * D * 2      # packed q|gate in (append)
                        + 2 * NKV * D * 2  # k_in, v_in
                        + NQ * D * 2       # rotated q (append write, decode read x2)
                        + NQ * D * 2       # out
                        + NKV * D * 2 * 2)  # appended K/V rows written
    return layers * (kv + per_layer_io), layers * kv


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the decode split kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "decode_split_kernel_config4.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch_config4:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(f"/tmp/pgc_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ CPU legs

def cpu_sample(lens, threads: int, max_tokens: int = 24576, min_seconds: float = 0.0):
    """Times the CPU restatement of the decode path (oracle, test infrastructure) on a bounded
    sample of the workload: the first sequences of this rank's draw, up to `max_tokens` cached
    tokens in total, one layer, OpenMP over (sequence, kv head). Returns (GB/s, seconds, desc)."""
    import numpy as np
    from oracle import oracle
    oracle.set_threads(threads)
    chosen, total = [], 0
    for L in lens:
        L = int(min(L, max_tokens - total)) if total + int(L) > max_tokens else int(L)
        if L <= 0:
            break
        chosen.append(L + 1)
        total += L + 1
    pages = [(L + PAGE - 1) // PAGE for L in chosen]
    npages = sum(pages)
    kp = oracle.normal_bf16(npages * NKV * PAGE * D, 11).reshape(npages, NKV, PAGE, D)
    vp = oracle.normal_bf16(npages * NKV * PAGE * D, 12).reshape(npages, NKV, PAGE, D)
    table = np.zeros((len(chosen), max(pages)), np.int32)
    o = 0
    for b, p in enumerate(pages):
        table[b, :p] = np.arange(o, o + p)
        o += p
    q = oracle.normal_bf16(len(chosen) * NQ * D, 13).reshape(len(chosen), 1, NQ, D)
    seq = np.array(chosen, np.int32)
    reps = 0
    t0 = time.perf_counter()
    while True:  # layer repeats until the sample is long enough (at most the 8 layers)
        oracle.decode_paged(q, kp, vp, table, seq, SCALE)
        reps += 1
        if time.perf_counter() - t0 >= min_seconds or reps >= LAYERS:
            break
    dt = time.perf_counter() - t0
    nbytes = reps * sum(chosen) * KV_BYTES_PER_TOKEN
    desc = (f"decode attention of {len(chosen)} sequence(s) of the workload draw "
            f"({sum(chosen)} cached tokens) x {reps} layer(s), oracle C port, {threads} thread(s)")
    return nbytes / dt / 1e9, dt, desc


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the path timed on the host cores."""
    if rank != 0:
        return
    lens, layers = workload_lengths(args.workload, 0, args.seed)
    threads = os.cpu_count() or 1
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, dt, desc = cpu_sample(lens, threads, max_tokens=65536)
        if i >= args.warmup:
            vals.append((gbs, dt))
    gbs = statistics.median(v[0] for v in vals)
    ms = statistics.median(v[1] for v in vals) * 1e3
    line = {
        "impl": "reference", "metric": "decode-attn achieved HBM GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"{args.workload}: batched paged decode sample on host cores",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference (Zig + Metal) cannot be built or run on Linux; this arm times its "
                "CPU restatement (oracle/pgo_oracle.c) of the same decode semantics",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ GPU arm

def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    from peregrine_b200 import capi

    torch.cuda.set_device(local_rank)
    capi.lib()  # fails loudly when the CUDA library is not built
    lens, layers = workload_lengths(args.workload, rank, args.seed)
    B = len(lens)
    pages = [(int(L) + 1 + PAGE - 1) // PAGE for L in lens]  # +1: the appended row
    total_pages = sum(pages)
    max_len = int(max(lens)) + 1
    g = torch.Generator(device="cuda")
    g.manual_seed(args.seed * 7919 + rank)
    bf = torch.bfloat16
    kpool = [torch.randn((total_pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    vpool = [torch.randn((total_pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    perm = torch.randperm(total_pages, device="cuda", generator=g).to(torch.int32)
    table = torch.zeros((B, max(pages)), dtype=torch.int32, device="cuda")
    o = 0
    for b, p in enumerate(pages):
        table[b, :p] = perm[o:o + p]
        o += p
    lens_t = torch.tensor(lens, dtype=torch.int64, device="cuda")
    seq_lens = (lens_t + 1).to(torch.int32)
    positions = lens_t.to(torch.int32)
    slots = table.gather(1, (lens_t // PAGE).view(-1, 1)).view(-1).to(torch.int64) * PAGE + lens_t % PAGE
    rope = torch.from_numpy(capi.rope_table(max_len + 1)).cuda()
    qw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    kw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    q_in = [torch.randn((B, NQ, 2 * D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    k_in = [torch.randn((B, NKV, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    v_in = [torch.randn((B, NKV, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    q_rot = [torch.empty((B, NQ, D), dtype=bf, device="cuda") for _ in range(layers)]
    gate = [torch.empty((B, NQ, D), dtype=bf, device="cuda") for _ in range(layers)]
    out = [torch.empty((B, NQ, D), dtype=bf, device="cuda") for _ in range(layers)]
    ws = torch.empty(capi.decode_workspace_bytes(B, 1, max_len), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    n_ev = layers * args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_ev)]

    def layer(l, timing=None):
        capi.append_kv_rope(q_in[l], q_rot[l], k_in[l], v_in[l], rope, positions, slots, kpool[l],
                            vpool[l], mode=capi.APPEND_DECODE, gate_out=gate[l], q_norm_w=qw,
                            k_norm_w=kw, stream=stream)
        if timing is not None:
            timing[0].record(stream)
        capi.decode_attn(q_rot[l], kpool[l], vpool[l], table, seq_lens, max_len, SCALE, out[l], ws,
                         gate=gate[l], stream=stream)
        if timing is not None:
            timing[1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        for l in range(layers):
            layer(l)
    barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.25)  # first sample lands inside the timed region
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    i = 0
    for _ in range(args.steps):
        for l in range(layers):
            layer(l, ev[i])
            i += 1
    t1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    dec_ms = sorted(a.elapsed_time(b) for a, b in ev)
    dec_avg = sum(dec_ms) / len(dec_ms)
    code, detail = capi.device_error()
    assert code == 0, f"device error {code} ({detail})"

    # ---- end-to-end through the C ABI with host buffers (pinned), copies inside the region
    q_h = [t.cpu().pin_memory() for t in q_in]
    k_h = [t.cpu().pin_memory() for t in k_in]
    v_h = [t.cpu().pin_memory() for t in v_in]
    out_h = [torch.empty(t.shape, dtype=bf).pin_memory() for t in out]
    h2d = sum(t.numel() * 2 for t in q_h + k_h + v_h)
    d2h = sum(t.numel() * 2 for t in out_h)

    def e2e_step():
        for l in range(layers):
            q_in[l].copy_(q_h[l], non_blocking=True)
            k_in[l].copy_(k_h[l], non_blocking=True)
            v_in[l].copy_(v_h[l], non_blocking=True)
            layer(l)
            out_h[l].copy_(out[l], non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    t = torch.tensor([ms, e2e_ms, dec_avg], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dec_avg = (float(x) for x in t.tolist())
    total_b, kv_b = step_bytes(lens, layers)
    tb = torch.tensor([total_b, kv_b, B], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tb)
    all_bytes, all_kv, all_seqs = (float(x) for x in tb.tolist())
    if rank != 0:
        return
    step_ms = ms / args.steps
    value = all_bytes / (step_ms * 1e-3) / 1e9
    e2e_value = all_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    # dominant kernel: pgc_decode_attn (split kernel + merge) of one layer on this rank
    launch_bytes = kv_b / layers + B * NQ * D * 2 * 3  # K/V + q + gate + out
    achieved = launch_bytes / (dec_avg * 1e-3) / 1e9
    traffic = profiled_traffic() if args.workload == "config4" else None
    line = {
        "metric": "decode-attn achieved HBM GB/s (% of 8 TB/s); decode tok/s",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1) bf16 K/V/Q, random page permutation)",
        "config": {"workload": f"{args.workload}: batched paged decode, {int(all_seqs)} sequences "
                               f"({B} per GPU), L~U[1024,65536], {layers} full-attention layers, "
                               "16q/4kv d256, 16-token pages, 1 query + 1 append per sequence",
                   "global_batch": int(all_seqs), "parallelism": f"sequence-sharded x{world}",
                   "l2": "inputs larger than L2 (K/V pools ~70 GB per GPU)"},
        "pct_of_8TBs": round(100 * value / world / 8000.0, 2),
        "tok_s": round(all_seqs / (step_ms * 1e-3), 1),
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "tok_s": round(all_seqs / (e2e_ms / args.steps * 1e-3), 1)},
        "roofline": {"bound": "hbm", "kernel": "pgc_decode_attn (decode_split_kernel + merge_kernel)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "launch_ms": round(dec_avg, 4),
                     "algorithmic_bytes_per_launch": launch_bytes},
        "gpu_launches": args.steps * layers * 3,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        gbs, dt, desc = cpu_sample(lens, threads, max_tokens=1 << 30, min_seconds=10.0)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                "kind": "port", "sample": desc + f", {dt:.1f} s"}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    assert args.warmup >= 3 or args.impl == "reference", "at least 3 warm-up steps"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
