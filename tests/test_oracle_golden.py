"""Pins the CPU oracle against the reference's own fixtures (tests/golden/) and checks its
arithmetic against independent float64 restatements. CPU only."""
import numpy as np
import pytest

D, NQ, NKV, PAGE = 256, 16, 4, 16


def test_stride_golden_values(oracle, fixtures):
    # src/model/state.zig:244-254
    assert len(fixtures["stride_cases"]) == 9
    for max_seq, expected in fixtures["stride_cases"]:
        assert oracle.full_cache_stride_for_max_seq(max_seq) == expected, max_seq


def test_topology_fixture(fixtures):
    t = fixtures["topology"]
    assert sum(t["is_linear"]) == 24 and t["is_linear"].count(False) == 8
    assert [i for i, lin in enumerate(t["is_linear"]) if not lin] == [3, 7, 11, 15, 19, 23, 27, 31]
    assert (t["num_kv"], t["head_dim"], t["hidden"]) == (4, 256, 4096)
    assert (t["conv_k"] - 1) * t["conv_dim"] * 4 == 96 * 1024          # conv state bytes (f32)
    assert t["hv"] * t["dv"] * t["dk"] * 4 == 2 * 1024 * 1024          # recurrent state bytes


def _persist_runs(cache_k, cache_v, stride, count):
    """The v3 snapshot run order (src/server/prefix_persist.zig:85-137): 4 K runs of
    count*256 values, then 4*256 V runs of count values."""
    out = []
    for h in range(NKV):
        out.append(cache_k[h * stride * D:(h * stride + count) * D])
    for h in range(NKV):
        for d in range(D):
            base = (h * D + d) * stride
            out.append(cache_v[base:base + count])
    return np.concatenate(out)


@pytest.mark.parametrize("distinct", [False, True])
def test_persist_roundtrip_fixture(oracle, fixtures, distinct):
    # src/server/prefix_persist.zig:457-541: fill every full layer's K/V with the fixture's byte
    # pattern, compact to token_count runs, restore into a fresh cache, compare every run.
    p = fixtures["persist"]
    count = p["roundtrip_token_count"]
    max_seq = max(count, p["roundtrip_cache_init"][1])
    stride = oracle.full_cache_stride_for_max_seq(max_seq)
    fill = p["fill_start"]
    for is_lin in fixtures["topology"]["is_linear"]:
        if is_lin:
            fill = (fill + 2) & 0xFF
            continue
        n = NKV * stride * D
        if distinct:
            rng = np.random.default_rng(fill)
            k = rng.integers(0, 65535, n, dtype=np.uint16)
            v = rng.integers(0, 65535, n, dtype=np.uint16)
        else:
            k = np.full(n, fill | (fill << 8), dtype=np.uint16)
            v = np.full(n, ((fill + 1) & 0xFF) * 0x0101, dtype=np.uint16)
        fill = (fill + 2) & 0xFF
        # compaction = copyFullAttentionRangeFrom into a dense cache of stride `count`
        ck = np.zeros(NKV * count * D, np.uint16)
        cv = np.zeros(NKV * count * D, np.uint16)
        oracle.copy_full_attention_range(ck, cv, count, 0, k, v, stride, 0, count)
        assert np.array_equal(np.concatenate([ck, cv]), _persist_runs(k, v, stride, count))
        rk = np.zeros_like(k)
        rv = np.zeros_like(v)
        oracle.copy_full_attention_range(rk, rv, stride, 0, ck, cv, count, 0, count)
        assert np.array_equal(_persist_runs(rk, rv, stride, count), _persist_runs(k, v, stride, count))


def test_expected_file_bytes_fixture(fixtures):
    # src/server/prefix_persist.zig:443-455
    t, p = fixtures["topology"], fixtures["persist"]
    n = p["expected_file_bytes_token_count"]
    conv = (t["conv_k"] - 1) * t["conv_dim"] * 4
    recur = t["hv"] * t["dv"] * t["dk"] * 4
    kv = NKV * n * D * 2
    total = p["header_bytes"] + n * 4 + 24 * (conv + recur) + 8 * 2 * kv + n * t["hidden"] * 2
    assert p["header_bytes"] == 48 and p["version"] == 3
    assert p["magic"].to_bytes(8, "little") == b"PRGPFXS1"
    assert total == 48 + n * 4 + 24 * (98304 + 2097152) + 16 * kv + n * 8192


def test_hidden_row_fixtures(oracle, fixtures):
    # src/server/prefix_state_cache.zig:935-1023: hidden rows are [rows, 4096] bf16 = 8 KiB rows
    row = fixtures["topology"]["hidden"] * 2
    c0, c1 = fixtures["hidden_cases"]
    work = np.full(c0["rows"] * row, c0["fill"], np.uint8)
    entry = np.zeros(16 * row, np.uint8)
    oracle.copy_rows(entry, work, c0["rows"], row, row, row)
    assert (entry[:c0["rows"] * row] == c0["fill"]).all() and (entry[c0["rows"] * row:] == 0).all()
    # extend: rows [0, 3) kept from the reused entry, suffix rows copied from work rows 3..5
    entry = np.zeros(16 * row, np.uint8)
    entry[:c1["prefix_rows"] * row] = c1["prefix_fill"]
    work = np.zeros(c1["total_rows"] * row, np.uint8)
    work[c1["work_base_row"] * row:c1["total_rows"] * row] = c1["suffix_fill"]
    n = c1["total_rows"] - c1["prefix_rows"]
    dst_rows = np.arange(c1["prefix_rows"], c1["total_rows"], dtype=np.int32)
    src_rows = np.arange(c1["work_base_row"], c1["work_base_row"] + n, dtype=np.int32)
    oracle.copy_rows(entry, work, n, row, row, row, dst_rows, src_rows)
    for r, val in c1["checks"]:
        assert entry[r * row] == val


# ----------------------------------------------------------------- oracle arithmetic checks

def _paged_from_dense(rng, k_logical, v_logical, num_pages):
    """k_logical [L][4][256] -> pools with a random page permutation; returns pools, table."""
    L = k_logical.shape[0]
    npg = (L + PAGE - 1) // PAGE
    table = rng.permutation(num_pages)[:npg].astype(np.int32)
    kp = np.zeros((num_pages, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    for t in range(L):
        kp[table[t // PAGE], :, t % PAGE] = k_logical[t]
        vp[table[t // PAGE], :, t % PAGE] = v_logical[t]
    return kp, vp, table


def _ref_decode(q, k, v, L, nq, scale):
    """float64 definition: query j sees tokens [0, L - nq + j]."""
    out = np.zeros((nq, NQ, D))
    qf = oracle_bf(q).astype(np.float64).reshape(nq, NQ, D)
    kf = oracle_bf(k).astype(np.float64)
    vf = oracle_bf(v).astype(np.float64)
    for j in range(nq):
        vis = L - nq + j + 1
        for h in range(NQ):
            s = kf[:vis, h // 4] @ qf[j, h] * scale
            w = np.exp(s - s.max())
            out[j, h] = (w[:, None] * vf[:vis, h // 4]).sum(0) / w.sum()
    return out


def oracle_bf(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("L,nq", [(1, 1), (37, 1), (1024, 1), (1500, 2), (2049, 3)])
def test_oracle_decode_matches_float64(oracle, L, nq):
    rng = np.random.default_rng(L)
    q = oracle.normal_bf16(nq * NQ * D, seed=L).reshape(1, nq, NQ, D)
    k = oracle.normal_bf16(L * NKV * D, seed=L + 1).reshape(L, NKV, D)
    v = oracle.normal_bf16(L * NKV * D, seed=L + 2).reshape(L, NKV, D)
    kp, vp, table = _paged_from_dense(rng, k, v, (L + 15) // 16 + 3)
    out, outb = oracle.decode_paged(q, kp, vp, table.reshape(1, -1), np.array([L], np.int32),
                                    1 / 16, nq)
    ref = _ref_decode(q, k, v, L, nq, 1 / 16)
    assert np.abs(out[0] - ref).max() < 1e-4
    assert np.array_equal(outb, oracle.f32_to_bf16(out))


def test_oracle_dense_two_source_equals_paged(oracle):
    # attention_decode.metal:89-93: prefix buffers for t < prefix_len, local after
    L, P = 3000, 1234
    rng = np.random.default_rng(0)
    q = oracle.normal_bf16(NQ * D, 5)
    k = oracle.normal_bf16(L * NKV * D, 6).reshape(L, NKV, D)
    v = oracle.normal_bf16(L * NKV * D, 7).reshape(L, NKV, D)
    ps = oracle.full_cache_stride_for_max_seq(P)
    ls = oracle.full_cache_stride_for_max_seq(L - P)
    pk = np.zeros((NKV, ps, D), np.uint16)
    pv = np.zeros((NKV, D, ps), np.uint16)
    lk = np.zeros((NKV, ls, D), np.uint16)
    lv = np.zeros((NKV, D, ls), np.uint16)
    pk[:, :P] = k[:P].transpose(1, 0, 2)
    pv[:, :, :P] = v[:P].transpose(1, 2, 0)
    lk[:, :L - P] = k[P:].transpose(1, 0, 2)
    lv[:, :, :L - P] = v[P:].transpose(1, 2, 0)
    dense = oracle.decode_dense_prefix(q, pk, pv, lk, lv, L, P, 1 / 16, ps, ls)
    kp, vp, table = _paged_from_dense(rng, k, v, 200)
    paged, _ = oracle.decode_paged(q.reshape(1, 1, NQ, D), kp, vp, table.reshape(1, -1),
                                   np.array([L], np.int32), 1 / 16)
    assert np.array_equal(dense, paged[0, 0])


def test_oracle_partials_merge(oracle):
    # splitting a cache into shards and LSE-merging the shard partials equals the whole
    L, S = 4000, 3
    rng = np.random.default_rng(1)
    q = oracle.normal_bf16(NQ * D, 11).reshape(1, 1, NQ, D)
    k = oracle.normal_bf16(L * NKV * D, 12).reshape(L, NKV, D)
    v = oracle.normal_bf16(L * NKV * D, 13).reshape(L, NKV, D)
    kp, vp, t = _paged_from_dense(rng, k, v, 300)
    full, _ = oracle.decode_paged(q, kp, vp, t.reshape(1, -1), np.array([L], np.int32), 1 / 16)
    bounds = np.linspace(0, L, S + 1).astype(int)
    parts = []
    for a, b in zip(bounds[:-1], bounds[1:]):
        kp, vp, t = _paged_from_dense(rng, k[a:b], v[a:b], 120)
        parts.append(oracle.decode_partials_paged(q, kp, vp, t.reshape(1, -1), np.array([b - a], np.int32), 1 / 16))
    parts = np.ascontiguousarray(np.stack(parts))  # [S][1][16][258]
    merged, _ = oracle.merge_partials(parts, NQ, S, NQ * 258)
    assert np.abs(merged - full[0, 0]).max() < 1e-5


def test_oracle_append_matches_float64(oracle):
    T = 5
    rope = oracle.rope_table(4200)
    q_in = oracle.normal_bf16(T * NQ * 2 * D, 21).reshape(T, NQ, 2 * D)
    k_in = oracle.normal_bf16(T * NKV * D, 22).reshape(T, NKV, D)
    v_in = oracle.normal_bf16(T * NKV * D, 23).reshape(T, NKV, D)
    qw = oracle.normal_bf16(D, 24)
    kw = oracle.normal_bf16(D, 25)
    pos = np.array([0, 1, 17, 4096, 4199], np.int32)
    slots = np.array([5, 16, 33, -1, 47], np.int64)
    kp = np.zeros((4, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    q_out, gate = oracle.append_kv_rope(q_in, k_in, v_in, rope, pos, slots, kp, vp, 1, qw, kw, True)
    assert np.array_equal(gate, q_in[:, :, D:])
    for t in range(T):
        for h in range(NQ + NKV):
            x = oracle_bf(q_in[t, h, :D] if h < NQ else k_in[t, h - NQ]).astype(np.float64)
            w = oracle_bf(qw if h < NQ else kw).astype(np.float64)
            y = x / np.sqrt((x * x).mean() + 1e-6) * w
            ang = pos[t] * 1e7 ** (-np.arange(32) * 2 / 64)
            r = y.copy()
            r[:32] = y[:32] * np.cos(ang) - y[32:64] * np.sin(ang)
            r[32:64] = y[32:64] * np.cos(ang) + y[:32] * np.sin(ang)
            if h < NQ:
                got = oracle_bf(q_out[t, h])
            else:
                if slots[t] < 0:
                    continue
                got = oracle_bf(kp[slots[t] // 16, h - NQ, slots[t] % 16])
                assert np.array_equal(vp[slots[t] // 16, h - NQ, slots[t] % 16], v_in[t, h - NQ])
            assert np.abs(got - r).max() <= 2 ** -7 * np.abs(r).max() + 1e-6


def test_oracle_prefill_matches_float64(oracle):
    P, T = 40, 9
    n = P + T
    rng = np.random.default_rng(3)
    q = oracle.normal_bf16(T * NQ * D, 31).reshape(T, NQ, D)
    k = oracle.normal_bf16(n * NKV * D, 32).reshape(n, NKV, D)
    v = oracle.normal_bf16(n * NKV * D, 33).reshape(n, NKV, D)
    kp, vp, table = _paged_from_dense(rng, k, v, 8)
    out, _ = oracle.prefill_paged(q, kp, vp, table, P, T, 1 / 16)
    for t in range(T):
        ref = _ref_decode(q[t].reshape(1, 1, NQ, D), k[:P + t + 1], v[:P + t + 1], P + t + 1, 1, 1 / 16)
        assert np.abs(out[t] - ref[0]).max() < 1e-4


def test_oracle_dense_restore_snapshot_roundtrip(oracle):
    rng = np.random.default_rng(4)
    stride, count, src_tok, dst_tok = 256, 70, 9, 13
    kd = rng.integers(0, 65535, NKV * stride * D, dtype=np.uint16)
    vd = rng.integers(0, 65535, NKV * D * stride, dtype=np.uint16)
    table = rng.permutation(12).astype(np.int32)
    kp = np.zeros((12, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    assert oracle.kv_restore_dense(kd, vd, stride, src_tok, kp, vp, table, dst_tok, count) == 0
    k2 = np.zeros_like(kd)
    v2 = np.zeros_like(vd)
    assert oracle.kv_snapshot_dense(kp, vp, table, dst_tok, k2, v2, stride, src_tok, count) == 0
    ek = np.zeros_like(kd)
    ev = np.zeros_like(vd)
    oracle.copy_full_attention_range(ek, ev, stride, src_tok, kd, vd, stride, src_tok, count)
    assert np.array_equal(k2, ek) and np.array_equal(v2, ev)
    # out-of-range table is reported, not written
    assert oracle.kv_restore_dense(kd, vd, stride, 0, kp, vp, table[:2], 0, 40) == -2


def test_oracle_rollback(oracle):
    live = np.arange(100, dtype=np.float32)
    snap = np.full(100, 7, np.float32)
    seq = np.array([10, 20], np.int32)
    oracle.rollback(np.array([1], np.int32), seq, 1, 1, [(live, snap)])
    assert seq[1] == 20 and live[5] == 5
    oracle.rollback(np.array([0], np.int32), seq, 1, 1, [(live, snap)])
    assert seq[1] == 19 and (live == 7).all()
