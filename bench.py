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
# One metric string for both arms (ours and --impl reference), so the two lines compare.
METRIC = "decode-attn achieved HBM GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4", choices=["config4", "small"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1-3 side figures")
    ap.add_argument("--profile-kernels", choices=["q4", "linear", "restore", "verify", "projection"],
                    default=None,
                    help="small cases for ncu captures: the q4 decode projection, the gated-delta "
                         "prefill, the config-2 restore, one config-3 verify layer (fused and two-call), "
                         "one layer's prefill projections")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="profiling aid: config 2's causal prefill on one layer, 3 launches")
    return ap.parse_args()


def workload_lengths(workload: str, rank: int, seed: int, world: int = 1):
    """This rank's sequence lengths and the layer count. One seeded draw for the whole job
    (64 sequences per GPU, L ~ U[1024, 65536]; 512 at 8 GPUs, BASELINE config 5a), split
    across the ranks balanced by tokens: longest first onto the rank with the fewest tokens
    among those still below 64 sequences. A rank's lengths keep their draw order, so at one
    GPU the workload is exactly config 4's draw."""
    import numpy as np
    rng = np.random.default_rng(seed * 1000003)
    per, lo, hi, layers = (8, 1024, 8193, 2) if workload == "small" else (64, 1024, 65537, LAYERS)
    lens = rng.integers(lo, hi, per * world).astype(np.int64)
    owner = balanced_partition(lens, world, per)
    return lens[owner == rank], layers


def balanced_partition(lens, world: int, per_rank: int):
    """Owner rank of every sequence: greedy longest-processing-time assignment with a cap of
    `per_rank` sequences per rank (ties go to the lower rank)."""
    import numpy as np
    owner = np.full(len(lens), -1, np.int64)
    load = [0] * world
    count = [0] * world
    for i in sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i)):
        r = min((r for r in range(world) if count[r] < per_rank), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += int(lens[i])
        count[r] += 1
    return owner


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

class CpuSample:
    """The CPU restatement of the decode path (oracle, test infrastructure) over this rank's
    whole draw: every sequence of the workload, one layer's K/V (random pages, seeded), OpenMP
    over (sequence, kv head). `run` times decode passes of that layer; the same sample serves
    the cpu_baseline leg of our arm and every step of the reference arm."""

    def __init__(self, lens, threads: int):
        import numpy as np
        from oracle import oracle
        self.oracle = oracle
        self.threads = threads
        oracle.set_threads(threads)
        self.chosen = [int(L) + 1 for L in lens]  # + the appended row
        pages = [(L + PAGE - 1) // PAGE for L in self.chosen]
        npages = sum(pages)
        self.kp = oracle.normal_bf16(npages * NKV * PAGE * D, 11).reshape(npages, NKV, PAGE, D)
        self.vp = oracle.normal_bf16(npages * NKV * PAGE * D, 12).reshape(npages, NKV, PAGE, D)
        self.table = np.zeros((len(self.chosen), max(pages)), np.int32)
        o = 0
        for b, p in enumerate(pages):
            self.table[b, :p] = np.arange(o, o + p)
            o += p
        self.q = oracle.normal_bf16(len(self.chosen) * NQ * D, 13).reshape(len(self.chosen), 1, NQ, D)
        self.seq = np.array(self.chosen, np.int32)
        self.tokens = sum(self.chosen)

    def run(self, min_seconds: float = 0.0, max_layers: int = 1):
        """Decode passes until `min_seconds` have elapsed or `max_layers` passes ran.
        Returns (GB/s of K+V, seconds, passes)."""
        reps = 0
        t0 = time.perf_counter()
        while True:
            self.oracle.decode_paged(self.q, self.kp, self.vp, self.table, self.seq, SCALE)
            reps += 1
            if time.perf_counter() - t0 >= min_seconds or reps >= max_layers:
                break
        dt = time.perf_counter() - t0
        return reps * self.tokens * KV_BYTES_PER_TOKEN / dt / 1e9, dt, reps

    def desc(self, reps: int) -> str:
        return (f"decode attention of all {len(self.chosen)} sequences of rank 0's workload draw "
                f"({self.tokens} cached tokens) x {reps} layer pass(es), oracle C port, "
                f"{self.threads} thread(s)")


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the path timed on the host cores, on rank 0's
    sequences of the same draw our arm decodes (one layer of all of them per step)."""
    if rank != 0:
        return
    lens, layers = workload_lengths(args.workload, 0, args.seed, world)
    threads = os.cpu_count() or 1
    sample = CpuSample(lens, threads)
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, dt, _ = sample.run()
        if i >= args.warmup:
            vals.append((gbs, dt))
    gbs = statistics.median(v[0] for v in vals)
    ms = statistics.median(v[1] for v in vals) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in, fp32 accumulate", "data": "synthetic",
        "config": {"workload": f"{args.workload}: batched paged decode of rank 0's {len(lens)} "
                               "sequences on host cores, one layer per step",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample.desc(1) + " per step"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference (Zig + Metal) cannot be built or run on Linux; this arm times its "
                "CPU restatement (oracle/pgo_oracle.c) of the same decode semantics",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------ output checks
# The timed configurations are checked in the same run, after their timed regions: the CPU
# oracle (test infrastructure, fp32 accumulate) is the checker, never the thing measured.

ATOL, RTOL = 2e-2, 1e-2


def _u16(t):
    """bf16 (or int16) device tensor -> host uint16 bits."""
    import numpy as np
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf(a):
    import numpy as np
    return (a.astype(np.uint32) << 16).view(np.float32)


def _close(got_u16, ref_f32):
    import numpy as np
    g = _bf(got_u16)
    err = np.abs(g - ref_f32)
    bad = int(((err > ATOL + RTOL * np.abs(ref_f32)) | ~np.isfinite(g)).sum())
    return float(err.max()) if err.size else 0.0, bad


def check_decode_against_oracle(capi, seqs, q, gate, out, kpool, vpool, table, seq_lens, nq=1):
    """Decode output of sequences `seqs` (indices into the batch) against the oracle: their
    pages are copied out of the pools into compact host pools in block-table order."""
    import numpy as np
    import torch
    from oracle import oracle
    oracle.set_threads(os.cpu_count() or 1)
    worst, bad = 0.0, 0
    for b in seqs:
        L = int(seq_lens[b].item())
        npg = (L + PAGE - 1) // PAGE
        idx = table[b, :npg].long()
        kp = _u16(kpool.index_select(0, idx))
        vp = _u16(vpool.index_select(0, idx))
        tb = np.arange(npg, dtype=np.int32).reshape(1, -1)
        qb = _u16(q[b * nq:(b + 1) * nq]).reshape(1, nq, NQ, D)
        gb = None if gate is None else _u16(gate[b * nq:(b + 1) * nq]).reshape(1, nq, NQ, D)
        ref, _ = oracle.decode_paged(qb, kp, vp, tb, np.array([L], np.int32), SCALE, num_queries=nq,
                                     gate=gb)
        e, n = _close(_u16(out.reshape(-1, nq, NQ, D)[b]).reshape(1, nq, NQ, D), ref)
        worst, bad = max(worst, e), bad + n
        del kp, vp
    torch.cuda.synchronize()
    return {"max_abs_err": worst, "bad": bad}


# ------------------------------------------------------------------------------ other configs
# BASELINE configs 1-3 are timed in the same run (single GPU, rank 0) and reported under
# "configs"; the headline line stays config 4.

def _ev_time(fn, iters, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def bench_config1(capi, iters=20):
    """Config 1: one layer, batch 1, 4096 cached tokens + 1 appended at position 4096 (RoPE on
    64 dims, no norm), decode over 4097 tokens; output bf16 [16x256]. The 16.8 MB cache fits in
    L2, so the step rotates over 16 copies of it (269 MB, larger than L2) and every step reads
    its K/V from HBM. Timed as direct launches and as a replayed CUDA graph of 16 steps."""
    import torch
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    L, copies = 4096, 16
    pages = (L + 1 + PAGE - 1) // PAGE
    kps = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(copies)]
    vps = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(copies)]
    table = torch.arange(pages, dtype=torch.int32, device="cuda").view(1, -1)
    q_in = torch.randn((1, NQ, D), dtype=bf, device="cuda", generator=g)
    k_in = torch.randn((1, NKV, D), dtype=bf, device="cuda", generator=g)
    v_in = torch.randn((1, NKV, D), dtype=bf, device="cuda", generator=g)
    q = torch.empty_like(q_in)
    out = torch.empty((1, 1, NQ, D), dtype=bf, device="cuda")
    rope = torch.from_numpy(capi.rope_table(L + 1)).cuda()
    pos = torch.tensor([L], dtype=torch.int32, device="cuda")
    slot = torch.tensor([L], dtype=torch.int64, device="cuda")
    seq = torch.tensor([L + 1], dtype=torch.int32, device="cuda")
    ws = torch.empty(capi.decode_workspace_bytes(1, 1, L + 1), dtype=torch.uint8, device="cuda")

    def fused_step(st, c):
        capi.decode_attn_append(q_in, k_in, v_in, rope, pos, slot, kps[c], vps[c], table, seq, L + 1,
                                SCALE, out, ws, stream=st)

    def two_call_step(st, c):
        capi.append_kv_rope(q_in, q, k_in, v_in, rope, pos, slot, kps[c], vps[c], stream=st)
        capi.decode_attn(q, kps[c], vps[c], table, seq, L + 1, SCALE, out, ws, stream=st)

    s = torch.cuda.current_stream()

    def timed(step):
        def all_copies(st):
            for c in range(copies):
                step(st, c)
        direct = _ev_time(lambda: all_copies(s), iters) / copies
        graph_ms = None
        try:
            gr = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(s)
            with torch.cuda.graph(gr, stream=cap):
                all_copies(cap)
            s.wait_stream(cap)
            graph_ms = _ev_time(gr.replay, iters) / copies
        except Exception as e:  # the graph figure is optional
            print(f"config1 graph capture failed: {e}", file=sys.stderr)
        return direct, graph_ms

    direct, graph_ms = timed(fused_step)
    direct2, graph2 = timed(two_call_step)
    # output check: the fused launch against the two calls (bit for bit), and against the oracle
    fused_step(s, 0)
    out_f = out.clone()
    two_call_step(s, 0)
    torch.cuda.synchronize()
    parity = check_decode_against_oracle(capi, [0], q, None, out, kps[0], vps[0], table, seq)
    parity.update(fused_equals_two_calls=bool(torch.equal(out_f, out)),
                  check="fused append+decode vs append then decode (bit-exact); decode vs the "
                        "CPU oracle (abs 2e-2 + rel 1e-2)")
    parity["ok"] = parity["bad"] == 0 and parity["fused_equals_two_calls"]
    nbytes = (L + 1) * KV_BYTES_PER_TOKEN + 3 * NQ * D * 2 + 2 * NKV * D * 2
    best = direct if graph_ms is None else min(direct, graph_ms)
    return {"workload": "config1: 1 layer, 4097-token decode + 1 append at pos 4096, fused in one "
                        "launch (pgc_decode_attn_append); 16 cache copies in rotation: K/V read from "
                        "HBM, not L2",
            "us_per_step": round(direct * 1e3, 2),
            "us_per_step_graph": None if graph_ms is None else round(graph_ms * 1e3, 2),
            "us_per_step_two_calls": round(direct2 * 1e3, 2),
            "us_per_step_graph_two_calls": None if graph2 is None else round(graph2 * 1e3, 2),
            "GB_s": round(nbytes / (best * 1e-3) / 1e9, 1), "algorithmic_bytes": nbytes,
            "parity": parity}


def bench_config2(capi, iters=5):
    """Config 2: restore of a 24576-token prefix from an HBM prefix store (8 layers of
    dense-layout K/V into 16-token pages under a random permutation, MTP hidden rows
    [24576x4096] bf16, 24 gated-delta fp32 states [32x128x128], 24 conv fp32 states [3x8192], the
    reference's conv state type (state.zig, prefix_persist.zig); BASELINE's text says bf16, the
    copy is byte-agnostic),
    then a 1600-token chunk: K/V append with RMSNorm + RoPE, causal attention over
    prefix + chunk. The q4 projections are out of scope: the chunk's N(0,1) hidden rows
    [1600x4096] serve directly as Q."""
    import numpy as np
    import torch
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    P, T, layers = 24576, 1600, LAYERS
    n = P + T
    pages = (n + PAGE - 1) // PAGE
    stride = capi.full_cache_stride_for_max_seq(P)
    store_k = [torch.randn((NKV, stride, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    store_v = [torch.randn((NKV, D, stride), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    store_h = torch.randn((P, 4096), dtype=bf, device="cuda", generator=g)
    store_gd = [torch.randn(32 * 128 * 128, device="cuda", generator=g) for _ in range(24)]
    store_cv = [torch.randn(3 * 8192, device="cuda", generator=g) for _ in range(24)]
    kp = [torch.empty((pages, NKV, PAGE, D), dtype=bf, device="cuda") for _ in range(layers)]
    vp = [torch.empty((pages, NKV, PAGE, D), dtype=bf, device="cuda") for _ in range(layers)]
    live_h = torch.empty((n, 4096), dtype=bf, device="cuda")
    live = [torch.empty_like(t) for t in store_gd + store_cv]
    table = torch.randperm(pages, device="cuda", generator=g).to(torch.int32)
    hidden = torch.randn((T, NQ, D), dtype=bf, device="cuda", generator=g)
    k_in = torch.randn((T, NKV, D), dtype=bf, device="cuda", generator=g)
    v_in = torch.randn((T, NKV, D), dtype=bf, device="cuda", generator=g)
    qw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    kw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    rope = torch.from_numpy(capi.rope_table(n)).cuda()
    pos = torch.arange(P, n, dtype=torch.int32, device="cuda")
    slots = table.long()[pos.long() // PAGE] * PAGE + pos.long() % PAGE
    q = torch.empty_like(hidden)
    out = torch.empty_like(hidden)
    regions = [(d, s_, s_.numel() * s_.element_size()) for d, s_ in zip(live, store_gd + store_cv)]
    s = torch.cuda.current_stream()

    def restore():
        for l in range(layers):
            capi.kv_restore_dense(store_k[l], store_v[l], stride, 0, kp[l], vp[l], table, 0, P, stream=s)
        capi.copy_rows(live_h, store_h, P, 4096 * 2, 4096 * 2, 4096 * 2, stream=s)
        capi.copy_regions(regions, stream=s)

    def chunk_append():
        for l in range(layers):
            capi.append_kv_rope(hidden, q, k_in, v_in, rope, pos, slots, kp[l], vp[l],
                                mode=capi.APPEND_PREFILL, q_norm_w=qw, k_norm_w=kw, stream=s)

    pws_bytes = capi.prefill_workspace_bytes(P, T)
    pws = torch.empty(max(pws_bytes, 16), dtype=torch.uint8, device="cuda")

    def prefill():
        for l in range(layers):
            capi.prefill_attn(q, kp[l], vp[l], table, P, T, SCALE, out, pws, stream=s)

    # The same prefix as a cache hit on the page-refcounted prefix cache: the entry's pages
    # are forked into the request's block table (host refcounts, KV and hidden rows are not
    # copied), the partial boundary page (none here: 24576 is page aligned) is copied on write,
    # and the 24 GD + conv linear states are copied into the request's state, as the
    # reference's hit path copies them (copyLinearStateFrom).
    from peregrine_b200 import prefix_cache as pcm
    ppool = pcm.PagePool(pages)
    pcache = pcm.PrefixCache(ppool, 65536, T, state_slots=2)
    ids = np.arange(P, dtype=np.uint32)
    hit_entry = pcache.start_direct_entry(ids)
    pcache.finish_direct_entry(hit_entry, 0)
    hit_pools = kp + vp

    def hit_share():
        m = pcache.find_prefix(ids)
        t = pcache.fork(m)
        if m.len % PAGE:
            src, dst = ppool.make_writable(t, len(t) - 1)
            pcm.copy_page(hit_pools, src, dst, stream=s)
        capi.copy_regions(regions, stream=s)
        pcache.touch(m)
        ppool.release(t)

    h_ms = _ev_time(hit_share, iters)
    hit_bytes = 24 * (32 * 128 * 128 * 4 + 3 * 8192 * 4)
    pcache.close()
    ppool.close()
    r_ms = _ev_time(restore, iters)

    # The same restore from a prefix store in pinned host memory (a snapshot file read into
    # host RAM): the kernels read the store over the host link, so its bytes cross it once.
    def pinned(t):
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h

    hk, hv = [pinned(t) for t in store_k], [pinned(t) for t in store_v]
    hh = pinned(store_h)
    hregions = [(d, pinned(s_), nb) for d, (_, s_, nb) in zip(live, regions)]

    def restore_pinned():
        for l in range(layers):
            capi.kv_restore_dense(hk[l], hv[l], stride, 0, kp[l], vp[l], table, 0, P, stream=s)
        capi.copy_rows(live_h, hh, P, 4096 * 2, 4096 * 2, 4096 * 2, stream=s)
        capi.copy_regions(hregions, stream=s)

    rp_ms = _ev_time(restore_pinned, 3)

    # Staged: the copy engines move each layer's dense K/V from the pinned store into one of two
    # device staging buffers on a copy stream (cudaMemcpyAsync), and the restore kernel scatters
    # layer l into pages while layer l + 1 is in flight; hidden rows and states go by DMA
    # straight to their destinations.
    cs = torch.cuda.Stream()
    stage_k = [torch.empty_like(store_k[0]) for _ in range(2)]
    stage_v = [torch.empty_like(store_v[0]) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def restore_staged():
        cs.wait_stream(s)
        for l in range(layers):
            b = l % 2
            with torch.cuda.stream(cs):
                if l >= 2:
                    cs.wait_event(freed[b])
                stage_k[b].copy_(hk[l], non_blocking=True)
                stage_v[b].copy_(hv[l], non_blocking=True)
                copied[b].record(cs)
            s.wait_event(copied[b])
            capi.kv_restore_dense(stage_k[b], stage_v[b], stride, 0, kp[l], vp[l], table, 0, P,
                                  stream=s)
            freed[b].record(s)
        with torch.cuda.stream(cs):
            live_h[:P].copy_(hh, non_blocking=True)
            for d, h, _ in hregions:
                d.copy_(h, non_blocking=True)
        s.wait_stream(cs)

    rs_ms = _ev_time(restore_staged, 3)
    # the staged path must write what the HBM-store restore writes: zero, stage, compare
    for t in kp + vp + [live_h] + live:
        t.zero_()
    restore_staged()
    torch.cuda.synchronize()
    got = [t.clone() for t in (kp[0], vp[0], kp[-1], vp[-1], live_h, live[0], live[-1])]
    restore()
    torch.cuda.synchronize()
    staged_ok = all(torch.equal(a, b) for a, b in zip(got, (kp[0], vp[0], kp[-1], vp[-1], live_h,
                                                            live[0], live[-1])))
    del got
    del hk, hv, hh, hregions, stage_k, stage_v
    a_ms = _ev_time(chunk_append, iters)
    p_ms = _ev_time(prefill, iters)
    restore_bytes = layers * P * KV_BYTES_PER_TOKEN + P * 4096 * 2 + 24 * (32 * 128 * 128 * 4 + 3 * 8192 * 4)
    flops = layers * 4 * NQ * D * (T * P + T * (T + 1) / 2)
    append_bytes = layers * T * (NQ * D * 2 * 2 + NKV * D * 2 * 4)
    return {"workload": "config2: restore 24576-token prefix (8 layers KV + MTP hidden + 24 GD/conv "
                        "states) from an HBM store (and, timed apart, from a pinned host store), then 1600-token "
                        "chunk append + causal prefill",
            "restore_ms": round(r_ms, 3), "restore_bytes": restore_bytes,
            "restore_GB_s_read_plus_write": round(2 * restore_bytes / (r_ms * 1e-3) / 1e9, 1),
            "restore_pinned_store_ms": round(rp_ms, 3),
            "restore_pinned_store_GB_s_host_link": round(restore_bytes / (rp_ms * 1e-3) / 1e9, 1),
            "restore_pinned_store_staged_ms": round(rs_ms, 3),
            "restore_pinned_store_staged_GB_s_host_link": round(restore_bytes / (rs_ms * 1e-3) / 1e9, 1),
            "restore_pinned_store_staged_matches": staged_ok,
            "hit_share_ms": round(h_ms, 3), "hit_share_bytes_copied": hit_bytes,
            "append_ms": round(a_ms, 3), "append_GB_s": round(append_bytes / (a_ms * 1e-3) / 1e9, 1),
            "prefill_ms": round(p_ms, 3), "prefill_flop": flops,
            "prefill_TFLOP_s": round(flops / (p_ms * 1e-3) / 1e12, 1)}


def bench_config3(capi, iters=10):
    """Config 3: MTP verify over a 32768-token cache on 8 layers, 2 query tokens (draft + bonus)
    attending in one pass, state snapshot of 24 gated-delta + conv states before the step, a
    seeded Bernoulli(0.7) acceptance flag, and on reject the device-side truncation of the last
    KV row plus bit-exact state restore (pgc_rollback)."""
    import numpy as np
    import torch
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    L, layers = 32768, LAYERS
    pages = (L + 2 + PAGE - 1) // PAGE
    kp = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    vp = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    table = torch.randperm(pages, device="cuda", generator=g).to(torch.int32).view(1, -1)
    live = ([torch.randn(32 * 128 * 128, device="cuda", generator=g) for _ in range(24)]
            + [torch.randn(3 * 8192, device="cuda", generator=g) for _ in range(24)])
    snap = [torch.empty_like(t) for t in live]
    q_in = [torch.randn((2, NQ, 2 * D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    k_in = [torch.randn((2, NKV, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    v_in = [torch.randn((2, NKV, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    q = torch.empty((2, NQ, D), dtype=bf, device="cuda")
    gate = torch.empty((2, NQ, D), dtype=bf, device="cuda")
    out = torch.empty((1, 2, NQ, D), dtype=bf, device="cuda")
    qw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    kw = torch.randn(D, dtype=bf, device="cuda", generator=g)
    rope = torch.from_numpy(capi.rope_table(L + 2)).cuda()
    pos = torch.tensor([L, L + 1], dtype=torch.int32, device="cuda")
    slots = table[0].long()[pos.long() // PAGE] * PAGE + pos.long() % PAGE
    seq = torch.tensor([L + 2], dtype=torch.int32, device="cuda")
    ws = torch.empty(capi.decode_workspace_bytes(1, 2, L + 2), dtype=torch.uint8, device="cuda")
    flags = (np.random.default_rng(0).random(4096) < 0.7).astype(np.int32)
    accept = torch.from_numpy(flags).cuda()
    nb = [t.numel() * t.element_size() for t in live]
    snap_regions = list(zip(snap, live, nb))
    back_regions = list(zip(live, snap, nb))
    s = torch.cuda.current_stream()
    counter = {"i": 0}

    def layer_ops(st, fused):
        for l in range(layers):
            if fused:
                capi.decode_attn_append(q_in[l], k_in[l], v_in[l], rope, pos, slots, kp[l], vp[l], table,
                                        seq, L + 2, SCALE, out, ws, num_queries=2, q_norm_w=qw, k_norm_w=kw,
                                        stream=st)
            else:
                capi.append_kv_rope(q_in[l], q, k_in[l], v_in[l], rope, pos, slots, kp[l], vp[l],
                                    gate_out=gate, q_norm_w=qw, k_norm_w=kw, stream=st)
                capi.decode_attn(q, kp[l], vp[l], table, seq, L + 2, SCALE, out, ws, num_queries=2,
                                 gate=gate, stream=st)

    def step():
        i = counter["i"] % len(flags)
        counter["i"] += 1
        seq.fill_(L + 2)
        capi.copy_regions(snap_regions, stream=s)
        layer_ops(s, True)
        capi.rollback(accept[i:i + 1], seq, 0, 1, back_regions, stream=s)

    ms_direct = _ev_time(step, iters)
    # the same step as one CUDA graph (launch overhead removed); the acceptance flag of each
    # replay is copied into the captured flag buffer first. The two-call form (append, then
    # decode) is timed the same way for comparison.
    acc = torch.zeros(1, dtype=torch.int32, device="cuda")

    def graph_ms(fused):
        try:
            gr = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(s)
            with torch.cuda.graph(gr, stream=cap):
                seq.fill_(L + 2)
                capi.copy_regions(snap_regions, stream=cap)
                layer_ops(cap, fused)
                capi.rollback(acc, seq, 0, 1, back_regions, stream=cap)
            s.wait_stream(cap)

            def replay():
                i = counter["i"] % len(flags)
                counter["i"] += 1
                acc.copy_(accept[i:i + 1])
                gr.replay()

            return _ev_time(replay, iters)
        except Exception as e:
            print(f"config3 graph capture failed: {e}", file=sys.stderr)
            return None

    ms_graph = graph_ms(True)
    ms_two = graph_ms(False)
    # output check on the last layer: fused vs two calls (bit for bit), two calls vs the oracle
    seq.fill_(L + 2)
    lt = layers - 1
    capi.decode_attn_append(q_in[lt], k_in[lt], v_in[lt], rope, pos, slots, kp[lt], vp[lt], table, seq,
                            L + 2, SCALE, out, ws, num_queries=2, q_norm_w=qw, k_norm_w=kw, stream=s)
    out_f = out.clone()
    capi.append_kv_rope(q_in[lt], q, k_in[lt], v_in[lt], rope, pos, slots, kp[lt], vp[lt],
                        gate_out=gate, q_norm_w=qw, k_norm_w=kw, stream=s)
    capi.decode_attn(q, kp[lt], vp[lt], table, seq, L + 2, SCALE, out, ws, num_queries=2, gate=gate,
                     stream=s)
    torch.cuda.synchronize()
    parity = check_decode_against_oracle(capi, [0], q, gate, out, kp[lt], vp[lt], table, seq, nq=2)
    parity.update(fused_equals_two_calls=bool(torch.equal(out_f, out)),
                  check="last layer, 2 queries: fused append+decode vs append then decode "
                        "(bit-exact); decode vs the CPU oracle (abs 2e-2 + rel 1e-2)")
    parity["ok"] = parity["bad"] == 0 and parity["fused_equals_two_calls"]
    ms = ms_direct if ms_graph is None else min(ms_direct, ms_graph)
    kv = layers * (L + 2) * KV_BYTES_PER_TOKEN
    state = sum(nb)
    reject_rate = 1.0 - float(flags.mean())
    moved = kv + 2 * state + reject_rate * 2 * state  # KV read, snapshot r+w, expected restore r+w
    return {"workload": "config3: MTP verify, 2 queries over 32768 tokens x 8 layers (append fused "
                        "into the decode, pgc_decode_attn_append), state snapshot + device-side "
                        "Bernoulli(0.7) rollback",
            "ms_per_verify": round(ms, 3), "ms_per_verify_direct": round(ms_direct, 3),
            "ms_per_verify_graph": None if ms_graph is None else round(ms_graph, 3),
            "ms_per_verify_graph_two_calls": None if ms_two is None else round(ms_two, 3),
            "kv_bytes": kv, "state_bytes": state,
            "GB_s": round(moved / (ms * 1e-3) / 1e9, 1), "parity": parity}


def bench_linear(capi, iters=10):
    """The linear-attention state producers (24 Gated-DeltaNet layers; no BASELINE config names
    them, they write the states configs 2-3 restore). Decode: 64 sequences, one token each, per
    layer a conv1d step and a gated delta-rule step over slot-indexed states (each sequence's
    2 MiB recurrent state read and written once, conv state 96 KiB). Prefill: one 1600-token
    chunk of one sequence through both. The q4 projections around them are out of scope:
    conv inputs, a/b and the gate parameters are seeded N(0,1) bf16."""
    import torch
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    B, LAYERS_LIN, T = 64, 24, 1600
    C, HV = capi.LIN_CONV_DIM, capi.LIN_VALUE_HEADS
    rec = [torch.randn((B, HV, 128, 128), device="cuda", generator=g) * 0.05 for _ in range(LAYERS_LIN)]
    conv = [torch.randn((B, 3, C), device="cuda", generator=g) for _ in range(LAYERS_LIN)]
    w = torch.randn((C, 4), dtype=bf, device="cuda", generator=g)
    x = torch.randn((B, C), dtype=bf, device="cuda", generator=g)
    co = torch.empty_like(x)
    a = torch.randn((B, HV), dtype=bf, device="cuda", generator=g)
    b = torch.randn((B, HV), dtype=bf, device="cuda", generator=g)
    a_log = torch.randn(HV, device="cuda", generator=g) * 0.5 - 1.0
    dtb = torch.randn(HV, dtype=bf, device="cuda", generator=g)
    y = torch.empty((B, HV * 128), dtype=bf, device="cuda")
    s = torch.cuda.current_stream()

    def decode_step():
        for l in range(LAYERS_LIN):
            capi.conv1d_decode(conv[l], x, w, co, stream=s)
            capi.gated_delta_decode(rec[l], True, co, a, b, a_log, dtb, y, stream=s)

    dec_ms = _ev_time(decode_step, iters)
    dec_bytes = LAYERS_LIN * B * (2 * HV * 128 * 128 * 4 + 2 * 3 * C * 4 + 3 * C * 2 + 2 * HV * 128 * 2)
    xs = torch.randn((T, C), dtype=bf, device="cuda", generator=g)
    cs = torch.empty_like(xs)
    at = torch.randn((T, HV), dtype=bf, device="cuda", generator=g)
    bt = torch.randn((T, HV), dtype=bf, device="cuda", generator=g)
    yt = torch.empty((T, HV * 128), dtype=bf, device="cuda")
    ws = torch.empty(capi.gated_delta_prefill_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    st1 = [r[0] for r in rec]
    cv1 = [c_[0] for c_ in conv]

    def prefill_chunk():
        for l in range(LAYERS_LIN):
            capi.conv1d_prefill(cv1[l], True, xs, w, cs, stream=s)
            capi.gated_delta_prefill(st1[l], True, cs, at, bt, a_log, dtb, yt, ws, stream=s)

    pf_ms = _ev_time(prefill_chunk, max(2, iters // 4))
    return {"workload": "24 linear layers: decode of 64 sequences (conv1d + gated delta rule over "
                        "slot-indexed states); prefill of one 1600-token chunk",
            "decode_ms_per_step": round(dec_ms, 4), "decode_state_bytes": dec_bytes,
            "decode_GB_s": round(dec_bytes / (dec_ms * 1e-3) / 1e9, 1),
            "prefill_ms_per_chunk": round(pf_ms, 3)}


def bench_q4(capi, iters=20):
    """The q4 projections of the 8 full-attention layers (q|gate 4096 -> 8192, k and v 4096 ->
    1024, o 4096 -> 4096; seeded random packed weights): decode of 64 tokens through
    pgc_q4_linear (bytes = packed weights + scales/biases + activations), and the prefill path
    of a 1600-token chunk: the weights dequantised once by pgc_q4_dequantize (not timed, as the
    reference prepares its dense RHS once), then the library's tcgen05 GEMM (pgc_prefill_linear:
    q | gate, k and v in one launch, o in another), with cuBLAS (torch.matmul) timed beside it."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    shapes = [(8192, 4096), (1024, 4096), (1024, 4096), (4096, 4096)]
    w = [[torch.randint(-2 ** 31, 2 ** 31 - 1, (o, i // 8), dtype=torch.int32, device="cuda", generator=g)
          for o, i in shapes] for _ in range(LAYERS)]
    sc = [[(torch.rand((o, i // 64), device="cuda", generator=g) * 0.02).to(torch.bfloat16) for o, i in shapes]
          for _ in range(LAYERS)]
    bi = [[(torch.randn((o, i // 64), device="cuda", generator=g) * 0.05).to(torch.bfloat16) for o, i in shapes]
          for _ in range(LAYERS)]
    s = torch.cuda.current_stream()

    def decode_ms(T):
        x = torch.randn((T, 4096), dtype=torch.bfloat16, device="cuda", generator=g)
        ys = [torch.empty((T, o), dtype=torch.bfloat16, device="cuda") for o, _ in shapes]

        def decode_step():
            # per layer: q | gate, k and v share x (pgc_q4_linear_multi: one launch at 1-2
            # tokens), then o
            st = torch.cuda.current_stream()
            for l in range(LAYERS):
                capi.q4_linear_multi(x, w[l][:3], sc[l][:3], bi[l][:3], ys[:3], stream=st)
                capi.q4_linear(x, w[l][3], sc[l][3], bi[l][3], ys[3], stream=st)

        # 16 (1-2 tokens) or 32 small launches per step: replayed as one CUDA graph, so the figure is device time
        # and not the Python launch rate
        decode_step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            decode_step()
        ms = _ev_time(graph.replay, iters)
        by = LAYERS * sum(o * i // 2 + 2 * (o * i // 64) * 2 + T * (i + o) * 2 for o, i in shapes)
        return ms, by

    dec_ms, dec_bytes = decode_ms(64)
    one_ms, one_bytes = decode_ms(1)
    dense = [[torch.empty((o, i), dtype=torch.bfloat16, device="cuda") for o, i in shapes] for _ in range(LAYERS)]
    for l in range(LAYERS):
        for j in range(4):
            capi.q4_dequantize(w[l][j], sc[l][j], bi[l][j], dense[l][j], stream=s)
    Tp = 1600
    xp = torch.randn((Tp, 4096), dtype=torch.bfloat16, device="cuda", generator=g)
    att = torch.randn((Tp, 4096), dtype=torch.bfloat16, device="cuda", generator=g)
    yp = [torch.empty((Tp, o), dtype=torch.bfloat16, device="cuda") for o, _ in shapes]

    def prefill_step():
        # per layer: q | gate, k and v share the chunk's hidden rows (one launch); o projects the
        # attention output
        for l in range(LAYERS):
            capi.prefill_linear(xp, dense[l][:3], yp[:3], stream=s)
            capi.prefill_linear(att, dense[l][3:], yp[3:], stream=s)

    def prefill_step_cublas():
        for l in range(LAYERS):
            for j in range(3):
                torch.matmul(xp, dense[l][j].t(), out=yp[j])
            torch.matmul(att, dense[l][3].t(), out=yp[3])

    pf_ms = _ev_time(prefill_step, max(3, iters // 4))
    pf_cublas_ms = _ev_time(prefill_step_cublas, max(3, iters // 4))
    # output check: the last layer's four projections against cuBLAS on the same operands
    prefill_step()
    ours = [y.clone() for y in yp]
    prefill_step_cublas()
    torch.cuda.synchronize()
    rel = max(float(((a.float() - b.float()).abs().max() / b.float().abs().max()).item())
              for a, b in zip(ours, yp))
    flops = LAYERS * sum(2 * Tp * o * i for o, i in shapes)
    return {"workload": "q4 projections of 8 full-attention layers: decode of 64 tokens and of 1 token "
                        "(pgc_q4_linear), prefill of a 1600-token chunk (dequantised weights + "
                        "pgc_prefill_linear tcgen05 GEMM; cuBLAS timed beside it)",
            "decode_ms_per_step": round(dec_ms, 4), "decode_bytes": dec_bytes,
            "decode_GB_s": round(dec_bytes / (dec_ms * 1e-3) / 1e9, 1),
            "decode_1tok_ms_per_step": round(one_ms, 4),
            "decode_1tok_GB_s": round(one_bytes / (one_ms * 1e-3) / 1e9, 1),
            "prefill_ms_per_chunk": round(pf_ms, 3),
            "prefill_TFLOP_s": round(flops / (pf_ms * 1e-3) / 1e12, 1),
            "prefill_cublas_ms_per_chunk": round(pf_cublas_ms, 3),
            "prefill_cublas_TFLOP_s": round(flops / (pf_cublas_ms * 1e-3) / 1e12, 1),
            "parity": {"check": "last layer's q|gate, k, v, o projections: pgc_prefill_linear vs "
                                "cuBLAS on the same bf16 operands (max |diff| / max |y|)",
                       "max_rel_diff": rel, "ok": rel < 1e-2}}


def bench_config5b(capi, rank, world, iters=20, warmup=3):
    """Config 5b: one 262144-token sequence (8 layers, 16q/4kv, d=256), context-parallel across
    the ranks in contiguous page-aligned KV shards; per layer: q/k RoPE (the new K/V row lands
    on the rank owning position 262144), split-K decode over the local shard, exchange of the
    (m, l, o) partials and LSE merge + gate on every rank. Timed twice: with the library's
    peer-memory exchange kernel and the append fused into the split kernel
    (pgc_cp_decode_attn_append, the reported figure), and with the library's NCCL path after a
    separate append (pgc_append_kv_rope, then pgc_cp_decode_attn_nccl: partials, in-place
    ncclAllGather, merge)."""
    import torch
    import torch.distributed as dist
    from peregrine_b200 import cp
    bf = torch.bfloat16
    L, layers = 262144, LAYERS
    cap = L + 1
    s0, e0 = cp.shard_bounds(cap, world, rank)
    n = e0 - s0
    tail = cp.owner_of(L, cap, world)
    pages = max(1, (n + PAGE - 1) // PAGE)
    g = torch.Generator(device="cuda")
    g.manual_seed(5000 + rank)
    kp = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    vp = [torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
    table = torch.arange(pages, dtype=torch.int32, device="cuda").view(1, -1)
    local_len = torch.tensor([n], dtype=torch.int32, device="cuda")
    gq = torch.Generator(device="cuda")
    gq.manual_seed(77)  # the query side is identical on every rank
    q_in = [torch.randn((1, NQ, 2 * D), dtype=bf, device="cuda", generator=gq) for _ in range(layers)]
    k_in = [torch.randn((1, NKV, D), dtype=bf, device="cuda", generator=gq) for _ in range(layers)]
    v_in = [torch.randn((1, NKV, D), dtype=bf, device="cuda", generator=gq) for _ in range(layers)]
    q = torch.empty((1, NQ, D), dtype=bf, device="cuda")
    gate = torch.empty((1, NQ, D), dtype=bf, device="cuda")
    out = torch.empty((NQ, D), dtype=bf, device="cuda")
    gathered = torch.empty((world, NQ, 258), dtype=torch.float32, device="cuda")
    ws = torch.empty(capi.decode_workspace_bytes(1, 1, max(n, 1)), dtype=torch.uint8, device="cuda")
    rope = torch.from_numpy(capi.rope_table(cap)).cuda()
    pos = torch.tensor([L], dtype=torch.int32, device="cuda")
    slot_val = (L - s0) if rank == tail else -1
    slot = torch.tensor([slot_val], dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream()

    ex = cp.PeerExchange(world, rank)
    grp = cp.NcclGroup(world, rank)

    def step_peer():
        # the append fused into the split kernel (pgc_cp_decode_attn_append): one launch pair
        # (split + exchange) per layer
        for l in range(layers):
            ex.decode_layer_append(q_in[l], k_in[l], v_in[l], rope, pos, slot, s0, kp[l], vp[l], table,
                                   local_len, n, SCALE, ws, out, stream=s)

    def step_nccl():
        for l in range(layers):
            capi.append_kv_rope(q_in[l], q, k_in[l], v_in[l], rope, pos, slot, kp[l], vp[l],
                                gate_out=gate, stream=s)
            grp.decode_layer(q.view(1, 1, NQ, D), kp[l], vp[l], table, local_len, n, SCALE,
                             gathered, ws, out, gate=gate.view(NQ, D), stream=s)

    def timed(step):
        for _ in range(warmup):
            step()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a_.record(s)
        for _ in range(iters):
            step()
        b_.record(s)
        torch.cuda.synchronize()
        t = torch.tensor([a_.elapsed_time(b_) / iters], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def step_local():
        # this rank's shard decoded alone (split + merge launches, no append, no exchange): the
        # single-sequence part of a context-parallel layer
        for l in range(layers):
            capi.decode_attn(q.view(1, 1, NQ, D), kp[l], vp[l], table, local_len, n, SCALE, out, ws,
                             gate=gate.view(NQ, D), stream=s)

    ms = timed(step_peer)
    code, _ = capi.device_error()
    ms_nccl = timed(step_nccl)
    ms_local = timed(step_local)
    # Output check (last layer of one more step of each path): the peer-exchange output against
    # the NCCL path's, against every other rank's, and against the oracle, which decodes each
    # rank's shard on the host into (m, l, o) partials that are gathered and LSE-merged with the
    # gate. The paths merge in different orders, so they agree to rounding, not bit for bit.
    import numpy as np
    from oracle import oracle
    step_peer()
    torch.cuda.synchronize()
    out_peer = out.clone()
    step_nccl()
    torch.cuda.synchronize()
    out_nccl, q_last, g_last = out.clone(), q.clone(), gate.clone()
    code2, _ = capi.device_error()
    diff_paths = (out_peer.float() - out_nccl.float()).abs().max().item()
    if world > 1:
        outs = [torch.empty_like(out_peer) for _ in range(world)]
        dist.all_gather(outs, out_peer)
        ranks_equal = all(torch.equal(o_, outs[0]) for o_ in outs)
    else:
        ranks_equal = True
    oracle.set_threads(max(1, (os.cpu_count() or 1) // world))
    kp_h, vp_h = _u16(kp[-1]), _u16(vp[-1])
    tb = np.arange(pages, dtype=np.int32).reshape(1, -1)
    qh = _u16(q_last).reshape(1, 1, NQ, D)
    part = oracle.decode_partials_paged(qh, kp_h, vp_h, tb, np.array([n], np.int32), SCALE)[0]
    del kp_h, vp_h
    part_t = torch.from_numpy(np.ascontiguousarray(part)).cuda()
    if world > 1:
        parts = [torch.empty_like(part_t) for _ in range(world)]
        dist.all_gather(parts, part_t)
    else:
        parts = [part_t]
    allp = np.ascontiguousarray(torch.stack(parts).cpu().numpy())  # [world][16][258]
    ref, _ = oracle.merge_partials(allp, NQ, world, NQ * 258, _u16(g_last).reshape(NQ, D).copy())
    err, bad = _close(_u16(out_peer).reshape(NQ, D), ref)
    chk = torch.tensor([err, float(bad), diff_paths, float(not ranks_equal), float(code2 != 0)],
                       dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(chk, op=dist.ReduceOp.MAX)
    err, bad, diff_paths, ranks_differ, dev_err = chk.tolist()
    parity = {"check": "last layer: peer-exchange output (append fused) vs the oracle (per-rank shard "
                       "partials on the host, gathered, LSE-merged, gated), vs the NCCL path (separate "
                       "append), and across ranks",
              "tolerance": "abs 2e-2 + rel 1e-2 vs oracle; paths within 1 bf16 ulp",
              "max_abs_err_vs_oracle": err, "bad_elements": int(bad),
              "max_abs_diff_peer_vs_nccl": diff_paths, "ranks_identical": ranks_differ == 0,
              "ranks": world}
    parity["ok"] = bad == 0 and ranks_differ == 0 and dev_err == 0 and diff_paths <= 1.6e-2
    if world > 1:
        dist.barrier()
    ex.close()
    grp.close()
    kv = layers * cap * KV_BYTES_PER_TOKEN
    return {"workload": f"config5b: one 262144-token sequence, 8 layers, context-parallel over "
                        f"{world} GPU(s) ({n} tokens on rank {rank}); partials exchanged by the "
                        f"library's peer-memory exchange kernel (the library's NCCL all-gather path, "
                        f"pgc_cp_decode_attn_nccl, timed beside it)",
            "ms_per_token": round(ms, 4), "tok_s": round(1e3 / ms, 1),
            "GB_s_aggregate": round(kv / (ms * 1e-3) / 1e9, 1), "kv_bytes": kv,
            "ms_per_token_nccl": round(ms_nccl, 4), "device_error": code,
            "per_layer_us": {"cp_peer_fused": round(ms * 1e3 / layers, 2),
                             "cp_nccl": round(ms_nccl * 1e3 / layers, 2),
                             "local_shard_decode": round(ms_local * 1e3 / layers, 2),
                             "shard_hbm_floor": round(n * KV_BYTES_PER_TOKEN / (measured_peaks()[0] * 1e9) * 1e6, 2),
                             "note": "local_shard_decode: the slowest rank's shard through pgc_decode_attn "
                                     "alone (split + merge, no append, no exchange); cp_peer_fused minus it "
                                     "is the append and the exchange"},
            "parity": parity}


# ------------------------------------------------------------------------------ GPU arm

def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    from peregrine_b200 import capi

    torch.cuda.set_device(local_rank)
    capi.lib()  # fails loudly when the CUDA library is not built
    lens, layers = workload_lengths(args.workload, rank, args.seed, world)
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

    # The copies run on their own stream, as a serving loop would issue them: layer l + 1's
    # inputs upload while layer l decodes, and each output downloads behind its layer. Events
    # keep a layer's buffers from being overwritten while the previous step still uses them.
    cs = torch.cuda.Stream()
    in_ready = [torch.cuda.Event() for _ in range(layers)]
    used = [torch.cuda.Event() for _ in range(layers)]
    out_read = [torch.cuda.Event() for _ in range(layers)]
    for l in range(layers):
        used[l].record(stream)
        out_read[l].record(cs)

    def e2e_step():
        with torch.cuda.stream(cs):
            for l in range(layers):
                cs.wait_event(used[l])
                q_in[l].copy_(q_h[l], non_blocking=True)
                k_in[l].copy_(k_h[l], non_blocking=True)
                v_in[l].copy_(v_h[l], non_blocking=True)
                in_ready[l].record(cs)
        for l in range(layers):
            stream.wait_event(in_ready[l])
            stream.wait_event(out_read[l])
            layer(l)
            used[l].record(stream)
            with torch.cuda.stream(cs):
                cs.wait_event(used[l])
                out_h[l].copy_(out[l], non_blocking=True)
                out_read[l].record(cs)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    cs.wait_stream(stream)
    for _ in range(args.steps):
        e2e_step()
    stream.wait_stream(cs)  # the last step's downloads are inside the region
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # Output check of the timed workload, on every rank: layer 0 of this rank's shortest and
    # longest sequence against the CPU oracle (fp32 accumulate), the gate applied.
    parity4 = check_decode_against_oracle(
        capi, [int(np.argmin(lens)), int(np.argmax(lens))], q_rot[0], gate[0], out[0],
        kpool[0], vpool[0], table, seq_lens)
    total_b, kv_b = step_bytes(lens, layers)
    launch_bytes = kv_b / layers + B * NQ * D * 2 * 3  # K/V + q + gate + out of one launch
    mine = [ms, e2e_ms, dec_avg, float(total_b), float(kv_b), float(B), launch_bytes,
            float(sum(int(L) for L in lens)), parity4["max_abs_err"], float(parity4["bad"])]
    t = torch.tensor(mine, dtype=torch.float64, device="cuda")
    if world > 1:
        allr = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allr, t)
        per_rank = [x.tolist() for x in allr]
    else:
        per_rank = [t.tolist()]
    ms = max(r[0] for r in per_rank)
    e2e_ms = max(r[1] for r in per_rank)
    all_bytes = sum(r[3] for r in per_rank)
    all_seqs = sum(r[5] for r in per_rank)
    # the dominant kernel's roofline per rank: that rank's launch bytes over its own launch time
    achieved_rank = [r[6] / (r[2] * 1e-3) / 1e9 for r in per_rank]
    parity_all = {"config4": {"check": "layer 0 output of each rank's shortest and longest "
                                       "sequence vs the CPU oracle (fp32 accumulate, gate applied)",
                              "tolerance": "abs 2e-2 + rel 1e-2",
                              "max_abs_err": max(r[8] for r in per_rank),
                              "bad_elements": int(sum(r[9] for r in per_rank)),
                              "ranks": world}}
    parity_all["config4"]["ok"] = parity_all["config4"]["bad_elements"] == 0
    cfg5b = None
    if args.workload == "config4" and not args.no_configs:
        kpool.clear()
        vpool.clear()
        torch.cuda.empty_cache()
        cfg5b = bench_config5b(capi, rank, world)
    if rank != 0:
        return
    step_ms = ms / args.steps
    value = all_bytes / (step_ms * 1e-3) / 1e9
    e2e_value = all_bytes / (e2e_ms / args.steps * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()
    achieved = min(achieved_rank)
    dec_avg = per_rank[achieved_rank.index(achieved)][2]
    launch_bytes = per_rank[achieved_rank.index(achieved)][6]
    traffic = profiled_traffic() if args.workload == "config4" else None
    line = {
        "metric": METRIC,
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
                     "rank_rule": "the slowest rank's launch (min over ranks of own bytes / own time)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "launch_ms": round(dec_avg, 4),
                     "algorithmic_bytes_per_launch": launch_bytes},
        "gpu_launches": args.steps * layers * 3,
        "clocks": clk,
        "per_rank": [{"rank": i, "sequences": int(r[5]), "cached_tokens": int(r[7]),
                      "step_ms": round(r[0] / args.steps, 4),
                      "decode_launch_ms": round(r[2], 4),
                      "decode_launch_GB_s": round(achieved_rank[i], 1)}
                     for i, r in enumerate(per_rank)],
        "parity": parity_all,
    }
    if cfg5b is not None:
        line["configs"] = {"config5b": cfg5b}
        if world == 1:
            line["configs"].update({"config1": bench_config1(capi), "config2": bench_config2(capi),
                                    "config3": bench_config3(capi), "linear": bench_linear(capi),
                                    "q4": bench_q4(capi)})
    for name, c in line.get("configs", {}).items():
        if isinstance(c, dict) and "parity" in c:
            line["parity"][name] = c["parity"]
    line["parity_ok"] = all(v.get("ok", False) for v in line["parity"].values())
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sample = CpuSample(lens, threads)
        gbs, dt, reps = sample.run(min_seconds=10.0, max_layers=layers)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                "kind": "port", "sample": sample.desc(reps) + f", {dt:.1f} s"}
    print(json.dumps(line), flush=True)


def profile_prefill():
    """One full-attention layer of config 2's prefill (1600-token chunk over a 24576-token
    prefix, pages under a random permutation), launched 3 times: the small case for ncu
    captures of prefill_pair_kernel (about 1 GB on the device)."""
    import torch
    from peregrine_b200 import capi
    bf = torch.bfloat16
    P, T = 24576, 1600
    pages = (P + T + PAGE - 1) // PAGE
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    kp = torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g)
    vp = torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g)
    table = torch.randperm(pages, device="cuda", generator=g).to(torch.int32)
    q = torch.randn((T, NQ, D), dtype=bf, device="cuda", generator=g)
    out = torch.empty_like(q)
    ws = torch.empty(max(capi.prefill_workspace_bytes(P, T), 16), dtype=torch.uint8, device="cuda")
    for _ in range(3):
        capi.prefill_attn(q, kp, vp, table, P, T, SCALE, out, ws)
    torch.cuda.synchronize()
    print(json.dumps({"profile": "prefill", "prefix": P, "chunk": T, "launches": 3}), flush=True)


def profile_kernels(which):
    """Small cases for ncu captures (3 launches each unless stated).
    q4: the 4096 -> 8192 q|gate projection of 64 decode tokens (q4_tc_kernel; 18 MB of packed
    weights, scales and biases; four weight copies so that launches read from HBM).
    linear: one gated-delta prefill layer over a 1600-token chunk (gated_delta_prep_kernel,
    gated_delta_chunk_kernel, gated_delta_chunk_scan_kernel)."""
    import torch
    from peregrine_b200 import capi
    bf = torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    if which == "q4":
        o, i, T = 8192, 4096, 64
        ws = [torch.randint(-2 ** 31, 2 ** 31 - 1, (o, i // 8), dtype=torch.int32, device="cuda", generator=g)
              for _ in range(4)]
        sc = (torch.rand((o, i // 64), device="cuda", generator=g) * 0.02).to(bf)
        bi = (torch.randn((o, i // 64), device="cuda", generator=g) * 0.05).to(bf)
        x = torch.randn((T, i), dtype=bf, device="cuda", generator=g)
        y = torch.empty((T, o), dtype=bf, device="cuda")
        for k in range(3):
            capi.q4_linear(x, ws[k], sc, bi, y)
    elif which == "linear":
        T, C, HV = 1600, capi.LIN_CONV_DIM, capi.LIN_VALUE_HEADS
        xs = torch.randn((T, C), dtype=bf, device="cuda", generator=g)
        at = torch.randn((T, HV), dtype=bf, device="cuda", generator=g)
        bt = torch.randn((T, HV), dtype=bf, device="cuda", generator=g)
        a_log = torch.randn(HV, device="cuda", generator=g) * 0.5 - 1.0
        dtb = torch.randn(HV, dtype=bf, device="cuda", generator=g)
        rec = torch.randn((HV, 128, 128), device="cuda", generator=g) * 0.05
        yt = torch.empty((T, HV * 128), dtype=bf, device="cuda")
        ws = torch.empty(capi.gated_delta_prefill_workspace_bytes(T), dtype=torch.uint8, device="cuda")
        for _ in range(3):
            capi.gated_delta_prefill(rec, True, xs, at, bt, a_log, dtb, yt, ws)
    elif which == "restore":
        # config 2's restore, once: 8 layers of dense K/V into permuted pages, the hidden rows and
        # the 48 linear states (about 1.1 GB each way on the device)
        P, layers = 24576, LAYERS
        pages = (P + 1600 + PAGE - 1) // PAGE
        stride = capi.full_cache_stride_for_max_seq(P)
        sk = [torch.randn((NKV, stride, D), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
        sv = [torch.randn((NKV, D, stride), dtype=bf, device="cuda", generator=g) for _ in range(layers)]
        sh = torch.randn((P, 4096), dtype=bf, device="cuda", generator=g)
        sgd = [torch.randn(32 * 128 * 128, device="cuda", generator=g) for _ in range(24)]
        scv = [torch.randn(3 * 8192, device="cuda", generator=g) for _ in range(24)]
        kp = [torch.empty((pages, NKV, PAGE, D), dtype=bf, device="cuda") for _ in range(layers)]
        vp = [torch.empty((pages, NKV, PAGE, D), dtype=bf, device="cuda") for _ in range(layers)]
        lh = torch.empty((P + 1600, 4096), dtype=bf, device="cuda")
        live = [torch.empty_like(t) for t in sgd + scv]
        table = torch.randperm(pages, device="cuda", generator=g).to(torch.int32)
        regions = [(d, s_, s_.numel() * s_.element_size()) for d, s_ in zip(live, sgd + scv)]
        for l in range(layers):
            capi.kv_restore_dense(sk[l], sv[l], stride, 0, kp[l], vp[l], table, 0, P)
        capi.copy_rows(lh, sh, P, 4096 * 2, 4096 * 2, 4096 * 2)
        capi.copy_regions(regions)
    elif which == "verify":
        # one config-3 layer (2 queries over 32768 cached tokens, RMSNorm weights, packed q | gate):
        # the fused append + decode, then the two-call form
        L = 32768
        pages = (L + 2 + PAGE - 1) // PAGE
        kp = torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g)
        vp = torch.randn((pages, NKV, PAGE, D), dtype=bf, device="cuda", generator=g)
        table = torch.randperm(pages, device="cuda", generator=g).to(torch.int32).view(1, -1)
        q_in = torch.randn((2, NQ, 2 * D), dtype=bf, device="cuda", generator=g)
        k_in = torch.randn((2, NKV, D), dtype=bf, device="cuda", generator=g)
        v_in = torch.randn((2, NKV, D), dtype=bf, device="cuda", generator=g)
        qw = torch.randn(D, dtype=bf, device="cuda", generator=g)
        kw = torch.randn(D, dtype=bf, device="cuda", generator=g)
        rope = torch.from_numpy(capi.rope_table(L + 2)).cuda()
        pos = torch.tensor([L, L + 1], dtype=torch.int32, device="cuda")
        slots = table[0].long()[pos.long() // PAGE] * PAGE + pos.long() % PAGE
        seq = torch.tensor([L + 2], dtype=torch.int32, device="cuda")
        ws = torch.empty(capi.decode_workspace_bytes(1, 2, L + 2), dtype=torch.uint8, device="cuda")
        q = torch.empty((2, NQ, D), dtype=bf, device="cuda")
        gate = torch.empty_like(q)
        out = torch.empty((1, 2, NQ, D), dtype=bf, device="cuda")
        for _ in range(3):
            capi.decode_attn_append(q_in, k_in, v_in, rope, pos, slots, kp, vp, table, seq, L + 2, SCALE, out, ws,
                                    num_queries=2, q_norm_w=qw, k_norm_w=kw)
        for _ in range(3):
            capi.append_kv_rope(q_in, q, k_in, v_in, rope, pos, slots, kp, vp, gate_out=gate, q_norm_w=qw,
                                k_norm_w=kw)
            capi.decode_attn(q, kp, vp, table, seq, L + 2, SCALE, out, ws, num_queries=2, gate=gate)
    elif which == "projection":
        # one layer's prefill projections at a 1600-token chunk (q | gate, k, v in one launch, then
        # o), 3 times: 117 MB of bf16 weights, about 0.2 GB on the device
        T, i = 1600, 4096
        ws = [torch.randn((o, i), dtype=bf, device="cuda", generator=g) for o in (8192, 1024, 1024, 4096)]
        x = torch.randn((T, i), dtype=bf, device="cuda", generator=g)
        ys = [torch.empty((T, w.shape[0]), dtype=bf, device="cuda") for w in ws]
        for _ in range(3):
            capi.prefill_linear(x, ws[:3], ys[:3])
            capi.prefill_linear(x, ws[3:], ys[3:])
    torch.cuda.synchronize()
    print(json.dumps({"profile": which}), flush=True)


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
    if args.profile_kernels:
        profile_kernels(args.profile_kernels)
        return
    if args.profile_prefill:
        profile_prefill()
        return
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
