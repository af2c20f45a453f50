"""GPU parity of the split-K paged decode attention against the CPU oracle, through the C ABI.
Tolerance (from the path's contract): |gpu - oracle| <= 2e-2 + 1e-2 * |oracle|, oracle fp32."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, assert_attn_close, dev, host_u16, paged_pools

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 16


def _case(oracle, lens, nq=1, seed=0, gate=False, spare_pages=7, nan_fill=False):
    rng = np.random.default_rng(seed)
    ks = [oracle.normal_bf16(L * NKV * D, seed * 1000 + 2 * b + 1).reshape(L, NKV, D) for b, L in enumerate(lens)]
    vs = [oracle.normal_bf16(L * NKV * D, seed * 1000 + 2 * b + 2).reshape(L, NKV, D) for b, L in enumerate(lens)]
    npages = sum((L + PAGE - 1) // PAGE for L in lens) + spare_pages
    kp, vp, table = paged_pools(rng, ks, vs, npages)
    if nan_fill:
        # slots past each sequence end hold NaN bit patterns (stale memory)
        for b, L in enumerate(lens):
            if L % PAGE:
                kp[table[b, L // PAGE], :, L % PAGE:] = 0x7FC0
                vp[table[b, L // PAGE], :, L % PAGE:] = 0x7FC0
    q = oracle.normal_bf16(len(lens) * nq * NQ * D, seed + 77).reshape(len(lens), nq, NQ, D)
    g = oracle.normal_bf16(q.size, seed + 78).reshape(q.shape) if gate else None
    seq = np.array(lens, np.int32)
    return q, kp, vp, table, seq, g


def _run(cuda, q, kp, vp, table, seq, nq, g=None, max_len=None):
    import torch
    max_len = max_len or int(seq.max())
    B = seq.shape[0]
    ws = torch.empty(cuda.decode_workspace_bytes(B, nq, max_len), dtype=torch.uint8, device="cuda")
    out = torch.empty((B, nq, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(dev(q), dev(kp), dev(vp), dev(table), dev(seq), max_len, SCALE, out, ws,
                     num_queries=nq, gate=None if g is None else dev(g))
    torch.cuda.synchronize()
    return host_u16(out)


def test_config1_single_layer_decode(cuda, oracle):
    # BASELINE config 1 shape: 1 sequence, 4097 tokens (4096 cached + the appended row)
    q, kp, vp, table, seq, _ = _case(oracle, [4097], spare_pages=0)
    got = _run(cuda, q, kp, vp, table, seq, 1)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE)
    err = assert_attn_close(got, ref)
    assert err < 2e-3


@pytest.mark.parametrize("nq", [1, 2, 3, 4])
def test_ragged_batch(cuda, oracle, nq):
    lens = [max(nq, L) for L in [1, 15, 16, 17, 100, 1023, 1025, 3000]]
    q, kp, vp, table, seq, g = _case(oracle, lens, nq=nq, seed=nq, gate=(nq == 2))
    got = _run(cuda, q, kp, vp, table, seq, nq, g)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE, nq, g)
    assert_attn_close(got, ref)


@pytest.mark.parametrize("nq", [1, 2])
def test_empty_sequence_slots_give_zero_rows(cuda, oracle, nq):
    # a serving batch with padding slots (seq_lens 0): their rows come out as zeros (gate or
    # not) and the other sequences are unaffected
    lens = [0, 37, 0, 1500, 0]
    q, kp, vp, table, seq, g = _case(oracle, lens, nq=nq, seed=21, gate=(nq == 2))
    got = _run(cuda, q, kp, vp, table, seq, nq, g)
    live = [b for b, L in enumerate(lens) if L > 0]
    ref, _ = oracle.decode_paged(q[live], kp, vp, np.ascontiguousarray(table[live]), seq[live], SCALE,
                                 nq, None if g is None else g[live])
    assert_attn_close(got[live], ref)
    assert (got[[b for b, L in enumerate(lens) if L == 0]] == 0).all()


def test_long_sequences_many_splits(cuda, oracle):
    lens = [20001, 40000, 1111]
    q, kp, vp, table, seq, _ = _case(oracle, lens, seed=9)
    got = _run(cuda, q, kp, vp, table, seq, 1, max_len=table.shape[1] * PAGE)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE)
    assert_attn_close(got, ref)


def test_stale_nan_slots_do_not_leak(cuda, oracle):
    lens = [5, 33, 250]
    q, kp, vp, table, seq, _ = _case(oracle, lens, seed=4, nan_fill=True)
    got = _run(cuda, q, kp, vp, table, seq, 1)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE)
    assert_attn_close(got, ref)


def test_partials_and_cross_shard_merge(cuda, oracle):
    """Context-parallel form on one GPU: the cache split in 3 contiguous shards, per-shard
    partials, then the LSE merge equals attention over the whole cache."""
    import torch
    L, S = 9000, 3
    q, kp, vp, table, seq, g = _case(oracle, [L], seed=5, gate=True)
    k_log = oracle.normal_bf16(L * NKV * D, 5 * 1000 + 1).reshape(L, NKV, D)
    v_log = oracle.normal_bf16(L * NKV * D, 5 * 1000 + 2).reshape(L, NKV, D)
    bounds = np.linspace(0, L, S + 1).astype(int)
    parts = torch.empty((S, NQ, 258), dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(6)
    for s, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        skp, svp, st = paged_pools(rng, [k_log[a:b]], [v_log[a:b]], (b - a) // 16 + 5)
        sl = np.array([b - a], np.int32)
        ws = torch.empty(cuda.decode_workspace_bytes(1, 1, int(b - a)), dtype=torch.uint8, device="cuda")
        cuda.decode_attn_partials(dev(q), dev(skp), dev(svp), dev(st), dev(sl), int(b - a), SCALE,
                                  parts[s], ws)
        ref_p = oracle.decode_partials_paged(q, skp, svp, st, sl, SCALE)
        torch.cuda.synchronize()
        gp = parts[s].cpu().numpy()
        assert np.abs(gp[:, 0] - ref_p[0, :, 0]).max() < 1e-3                 # m
        assert np.allclose(gp[:, 1], ref_p[0, :, 1], rtol=2e-2)               # l
    out = torch.empty((NQ, D), dtype=torch.int16, device="cuda")
    cuda.merge_partials(parts, NQ, S, NQ * 258, out, gate=dev(g.reshape(NQ, D)))
    torch.cuda.synchronize()
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE, 1, g)
    assert_attn_close(host_u16(out).reshape(1, 1, NQ, D), ref)


def test_bad_page_id_is_recorded_not_faulted(cuda, oracle):
    import torch
    q, kp, vp, table, seq, _ = _case(oracle, [64], seed=7)
    cuda.device_error(clear=True)
    table = table.copy()
    table[0, 1] = kp.shape[0] + 1000  # out of range: the kernel substitutes page 0 and records
    _run(cuda, q, kp, vp, table, seq, 1)
    code, detail = cuda.device_error(clear=True)
    assert code == 1 and detail == kp.shape[0] + 1000
    assert cuda.device_error(clear=True) == (0, 0)


def test_host_validation(cuda):
    import torch
    from peregrine_b200.capi import PgcError
    z = torch.zeros(1 << 16, dtype=torch.int16, device="cuda")
    pool = torch.zeros((4, NKV, PAGE, D), dtype=torch.int16, device="cuda")
    tbl = torch.zeros((1, 4), dtype=torch.int32, device="cuda")
    sl = torch.tensor([10], dtype=torch.int32, device="cuda")
    out = torch.empty((1, 1, NQ, D), dtype=torch.int16, device="cuda")
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(PgcError, match="WORKSPACE"):
        cuda.decode_attn(z, pool, pool, tbl, sl, 10, SCALE, out, small)
    ws = torch.empty(cuda.decode_workspace_bytes(1, 1, 64), dtype=torch.uint8, device="cuda")
    with pytest.raises(PgcError, match="BOUNDS"):
        cuda.decode_attn(z, pool, pool, tbl, sl, 65, SCALE, out, ws)   # 4 pages < 65 tokens
    with pytest.raises(PgcError, match="INVALID"):
        cuda.decode_attn(z, pool, pool, tbl, sl, 10, SCALE, out, ws, num_queries=5)
    with pytest.raises(PgcError, match="ALIGN"):
        cuda.decode_attn(z[1:], pool, pool, tbl, sl, 10, SCALE, out, ws)


def test_single_long_sequence_merge_over_80_parts(cuda, oracle):
    """A 100000-token sequence beside a short one: the batch's splits are capped at 64 pages, so
    the long row has 98 key-range splits, more than the merge keeps in registers (80 per row),
    and the merge takes its streaming path."""
    lens = [100000, 3000]
    q, kp, vp, table, seq, g = _case(oracle, lens, seed=11, gate=True, spare_pages=0)
    got = _run(cuda, q, kp, vp, table, seq, 1, g)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE, 1, g)
    assert_attn_close(got, ref)


@pytest.mark.parametrize("num_parts", [20, 80, 81, 130])
def test_merge_partials_part_counts(cuda, oracle, num_parts):
    """pgc_merge_partials across the merge's register path (up to 80 parts per row) and its
    streaming path, with empty parts (m = -inf, l = 0, o = 0) mixed in."""
    import torch
    rng = np.random.default_rng(num_parts)
    rows = 16
    parts = np.zeros((num_parts, rows, 258), np.float32)
    parts[:, :, 0] = rng.standard_normal((num_parts, rows)) * 3.0
    parts[:, :, 1] = rng.random((num_parts, rows)) * 50.0 + 1.0
    parts[:, :, 2:] = rng.standard_normal((num_parts, rows, 256)) * parts[:, :, 1:2]
    empty = rng.random((num_parts, rows)) < 0.2
    parts[empty, 0] = -np.inf
    parts[empty, 1:] = 0.0
    g = oracle.normal_bf16(rows * D, 3).reshape(rows, D)
    ref, _ = oracle.merge_partials(parts, rows, num_parts, rows * 258, g)
    out = torch.empty((rows, D), dtype=torch.int16, device="cuda")
    cuda.merge_partials(torch.from_numpy(parts).cuda(), rows, num_parts, rows * 258, out, gate=dev(g))
    torch.cuda.synchronize()
    assert_attn_close(host_u16(out).reshape(1, 1, rows, D), ref.reshape(1, 1, rows, D))


def test_single_sequence_one_wave_long_splits(cuda, oracle):
    """One 150000-token sequence alone: its splits are not capped (a one-wave plan of long
    splits, over 64 pages each)."""
    lens = [150000]
    q, kp, vp, table, seq, g = _case(oracle, lens, seed=12, gate=True, spare_pages=0)
    got = _run(cuda, q, kp, vp, table, seq, 1, g)
    ref, _ = oracle.decode_paged(q, kp, vp, table, seq, SCALE, 1, g)
    assert_attn_close(got, ref)
