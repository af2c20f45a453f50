"""GPU parity of the append (RMSNorm + partial RoPE) and every cache-copy kernel against the
CPU oracle, through the C ABI. All of these are bit-exact."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, dev, host_u16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("packed", [False, True])
def test_append_bit_exact(cuda, oracle, mode, norm, packed):
    import torch
    T = 37
    rope = oracle.rope_table(70000)
    q_in = oracle.normal_bf16(T * NQ * (2 if packed else 1) * D, 101).reshape(T, NQ, -1)
    k_in = oracle.normal_bf16(T * NKV * D, 102).reshape(T, NKV, D)
    v_in = oracle.normal_bf16(T * NKV * D, 103).reshape(T, NKV, D)
    qw = oracle.normal_bf16(D, 104) if norm else None
    kw = oracle.normal_bf16(D, 105) if norm else None
    rng = np.random.default_rng(7)
    pos = rng.integers(0, 70000, T).astype(np.int32)
    pos[0], pos[1] = 0, 4096
    npages = 8
    slots = rng.permutation(npages * PAGE)[:T].astype(np.int64)
    slots[3] = -1
    kp = oracle.normal_bf16(npages * NKV * PAGE * D, 106).reshape(npages, NKV, PAGE, D)
    vp = oracle.normal_bf16(npages * NKV * PAGE * D, 107).reshape(npages, NKV, PAGE, D)
    kp_d, vp_d = dev(kp), dev(vp)
    q_out = torch.zeros((T, NQ, D), dtype=torch.int16, device="cuda")
    gate = torch.zeros((T, NQ, D), dtype=torch.int16, device="cuda") if packed else None
    cuda.append_kv_rope(dev(q_in), q_out, dev(k_in), dev(v_in), dev(rope), dev(pos), dev(slots),
                        kp_d, vp_d, mode=mode, gate_out=gate,
                        q_norm_w=None if qw is None else dev(qw),
                        k_norm_w=None if kw is None else dev(kw))
    torch.cuda.synchronize()
    rq, rg = oracle.append_kv_rope(q_in, k_in, v_in, rope, pos, slots, kp, vp, mode, qw, kw, packed)
    assert np.array_equal(host_u16(q_out), rq)
    assert np.array_equal(host_u16(kp_d), kp)
    assert np.array_equal(host_u16(vp_d), vp)
    if packed:
        assert np.array_equal(host_u16(gate), rg)


def test_config1_append_at_4096(cuda, oracle):
    """one new K/V row at position 4096, RoPE theta 1e7 on dims [0, 64) of
    Q and K, no norm."""
    import torch
    rope = oracle.rope_table(4097)
    q_in = oracle.normal_bf16(NQ * D, 0).reshape(1, NQ, D)
    k_in = oracle.normal_bf16(NKV * D, 1).reshape(1, NKV, D)
    v_in = oracle.normal_bf16(NKV * D, 2).reshape(1, NKV, D)
    pos = np.array([4096], np.int32)
    slots = np.array([4096], np.int64)
    kp = np.zeros((257, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    kd, vd = dev(kp), dev(vp)
    q_out = torch.zeros((1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.append_kv_rope(dev(q_in), q_out, dev(k_in), dev(v_in), dev(rope), dev(pos), dev(slots), kd, vd)
    torch.cuda.synchronize()
    rq, _ = oracle.append_kv_rope(q_in, k_in, v_in, rope, pos, slots, kp, vp, 0)
    assert np.array_equal(host_u16(q_out), rq)
    assert np.array_equal(host_u16(kd)[256], kp[256]) and np.array_equal(host_u16(vd)[256], vp[256])
    assert np.array_equal(host_u16(q_out)[0, :, 64:], q_in[0, :, 64:])  # tail dims untouched


def test_copy_rows_gather_scatter(cuda, oracle):
    import torch
    rng = np.random.default_rng(1)
    for row_bytes, pitch in [(8192, 8192), (4096 * 2, 8192 + 16), (12, 20), (6, 7)]:
        n_src = 50
        src = rng.integers(0, 255, n_src * pitch, dtype=np.uint8)
        dst = rng.integers(0, 255, 64 * pitch, dtype=np.uint8)
        sr = rng.permutation(n_src)[:30].astype(np.int32)
        dr = rng.permutation(64)[:30].astype(np.int32)
        sd, dd = torch.from_numpy(src).cuda(), torch.from_numpy(dst).cuda()
        cuda.copy_rows(dd, sd, 30, row_bytes, pitch, pitch, dst_rows=dev(dr), src_rows=dev(sr))
        torch.cuda.synchronize()
        oracle.copy_rows(dst, src, 30, row_bytes, pitch, pitch, dr, sr)
        assert np.array_equal(dd.cpu().numpy(), dst), row_bytes


def test_copy_rows_from_pinned_host_store(cuda):
    """Restore from a host-resident (pinned) prefix store: 16-token pages straight into HBM."""
    import torch
    pages = 96
    store = torch.randint(-30000, 30000, (pages, NKV * PAGE * D), dtype=torch.int16).pin_memory()
    pool = torch.zeros((200, NKV * PAGE * D), dtype=torch.int16, device="cuda")
    table = torch.randperm(200, dtype=torch.int32)[:pages]
    cuda.copy_rows(pool, store.data_ptr(), pages, NKV * PAGE * D * 2, NKV * PAGE * D * 2,
                   NKV * PAGE * D * 2, dst_rows=table.cuda())
    torch.cuda.synchronize()
    assert torch.equal(pool.cpu()[table.long()], store)


# (restore dense token, page token, count, snapshot dense token, snapshot count): the first case
# takes the element-wise kernel (dense token not a multiple of 8), the others the vector kernel
# with ragged 64-token tiles and 8-token chunks
@pytest.mark.parametrize("src_tok,dst_tok,count,snap_tok,snap_count",
                         [(100, 21, 777, 3, 900), (96, 21, 777, 8, 901), (0, 0, 1000, 0, 1000),
                          (8, 5, 7, 16, 63)])
def test_dense_restore_snapshot_bit_exact(cuda, oracle, src_tok, dst_tok, count, snap_tok,
                                          snap_count):
    import torch
    rng = np.random.default_rng(2)
    stride = oracle.full_cache_stride_for_max_seq(1000)
    kd = rng.integers(0, 65535, NKV * stride * D, dtype=np.uint16)
    vd = rng.integers(0, 65535, NKV * D * stride, dtype=np.uint16)
    npages = 90
    table = rng.permutation(npages).astype(np.int32)
    kp = rng.integers(0, 65535, (npages, NKV, PAGE, D), dtype=np.uint16)
    vp = rng.integers(0, 65535, (npages, NKV, PAGE, D), dtype=np.uint16)
    kpd, vpd = dev(kp), dev(vp)
    cuda.kv_restore_dense(dev(kd), dev(vd), stride, src_tok, kpd, vpd, dev(table), dst_tok, count)
    assert oracle.kv_restore_dense(kd, vd, stride, src_tok, kp, vp, table, dst_tok, count) == 0
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(kpd), kp) and np.array_equal(host_u16(vpd), vp)
    k2 = np.zeros_like(kd)
    v2 = np.zeros_like(vd)
    k2d, v2d = dev(k2), dev(v2)
    cuda.kv_snapshot_dense(kpd, vpd, dev(table), 5, k2d, v2d, stride, snap_tok, snap_count)
    assert oracle.kv_snapshot_dense(kp, vp, table, 5, k2, v2, stride, snap_tok, snap_count) == 0
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(k2d), k2) and np.array_equal(host_u16(v2d), v2)


def test_kv_copy_tokens_bit_exact(cuda, oracle):
    import torch
    rng = np.random.default_rng(3)
    sk = rng.integers(0, 65535, (20, NKV, PAGE, D), dtype=np.uint16)
    sv = rng.integers(0, 65535, (20, NKV, PAGE, D), dtype=np.uint16)
    dk = rng.integers(0, 65535, (30, NKV, PAGE, D), dtype=np.uint16)
    dv = rng.integers(0, 65535, (30, NKV, PAGE, D), dtype=np.uint16)
    st = rng.permutation(20).astype(np.int32)
    dt = rng.permutation(30)[:20].astype(np.int32)
    dkd, dvd = dev(dk), dev(dv)
    cuda.kv_copy_tokens(dev(sk), dev(sv), dev(st), 7, dkd, dvd, dev(dt), 30, 250)
    assert oracle.kv_copy_tokens(sk, sv, st, 7, dk, dv, dt, 30, 250) == 0
    torch.cuda.synchronize()
    assert np.array_equal(host_u16(dkd), dk) and np.array_equal(host_u16(dvd), dv)


def _linear_state(rng, layers=24, conv_bytes=3 * 8192 * 2):
    recur = [rng.standard_normal(32 * 128 * 128).astype(np.float32) for _ in range(layers)]
    conv = [rng.integers(0, 255, conv_bytes, dtype=np.uint8) for _ in range(layers)]
    return recur, conv


@pytest.mark.parametrize("conv_bytes", [3 * 8192 * 2, 3 * 8192 * 4, 1001])
def test_copy_and_zero_regions(cuda, conv_bytes):
    import torch
    rng = np.random.default_rng(4)
    recur, conv = _linear_state(rng, conv_bytes=conv_bytes)
    src = [torch.from_numpy(a).cuda() for a in recur + conv]
    dst = [torch.zeros_like(t) for t in src]
    cuda.copy_regions([(d, s, s.numel() * s.element_size()) for d, s in zip(dst, src)])
    torch.cuda.synchronize()
    assert all(torch.equal(d, s) for d, s in zip(dst, src))
    cuda.zero_regions([(d, d.numel() * d.element_size()) for d in dst[:5]])
    torch.cuda.synchronize()
    assert all(int(d.count_nonzero()) == 0 for d in dst[:5]) and torch.equal(dst[5], src[5])


def test_rollback_device_side(cuda, oracle):
    """MTP verify rollback (BASELINE config 3 semantics): snapshot before the step; a seeded
    Bernoulli(0.7) acceptance flag decides; on reject the sequence loses its last KV row and the
    recurrent + conv state returns to the snapshot bit for bit."""
    import torch
    rng = np.random.default_rng(5)
    recur, conv = _linear_state(rng, layers=24)
    live = [torch.from_numpy(a).cuda() for a in recur + conv]
    snap = [torch.empty_like(t) for t in live]
    flags = (np.random.default_rng(0).random(12) < 0.7).astype(np.int32)
    seq = torch.tensor([0, 500], dtype=torch.int32, device="cuda")
    for step, accept in enumerate(flags):
        cuda.copy_regions([(s, l, l.numel() * l.element_size()) for s, l in zip(snap, live)])
        before = [t.clone() for t in live]
        for t in live:  # the verify step mutates the state and appends draft + bonus rows
            t.add_(1) if t.dtype == torch.float32 else t.bitwise_xor_(0x5A)
        after = [t.clone() for t in live]
        seq[0] = 32768 + 2 + step
        acc = torch.tensor([int(accept)], dtype=torch.int32, device="cuda")
        cuda.rollback(acc, seq, 0, 1, [(l, s, l.numel() * l.element_size()) for l, s in zip(live, snap)])
        torch.cuda.synchronize()
        expect = after if accept else before
        assert all(torch.equal(a, b) for a, b in zip(live, expect))
        assert int(seq[0]) == 32768 + 2 + step - (0 if accept else 1) and int(seq[1]) == 500
