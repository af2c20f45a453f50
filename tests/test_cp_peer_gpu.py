"""Peer-memory context-parallel exchange (pgc_cp_decode_attn) on one GPU.

1. world = 1: split decode + exchange kernel over several back-to-back calls (both epoch
   parities) against the oracle over the same cache, within the attention tolerance.
2. The append fused in (pgc_cp_decode_attn_append), world = 1 over a cache whose first global
   position is not 0, bit for bit against pgc_append_kv_rope followed by pgc_cp_decode_attn
   (output and pools) over several layers.
3. A rank that never arrives: world = 2 where the second rank's buffer is a local stand-in that
   nobody publishes to. The exchange kernel's flag wait runs out after its bound (~2 s), the
   library reports PGC_ERR_TIMEOUT's device code through pgc_device_error, and the context stays
   usable: the next world = 1 call is correct. No GPU fault is involved: the wait is bounded and
   the kernel returns."""
import ctypes as C
import time

import numpy as np
import pytest

from _util import D, NKV, NQ, PAGE, assert_attn_close, dev, host_u16

pytestmark = pytest.mark.gpu


def _cache(oracle, L, seed):
    k = oracle.normal_bf16(L * NKV * D, seed).reshape(L, NKV, D)
    v = oracle.normal_bf16(L * NKV * D, seed + 1).reshape(L, NKV, D)
    pages = (L + PAGE - 1) // PAGE
    kp = np.zeros((pages, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    for t in range(L):
        kp[t // PAGE, :, t % PAGE] = k[t]
        vp[t // PAGE, :, t % PAGE] = v[t]
    return kp, vp, np.arange(pages, dtype=np.int32).reshape(1, -1)


def _buffer(capi, world):
    p = C.c_void_p()
    capi.check(capi.lib().pgc_cp_buffer_alloc(world, C.byref(p)), "pgc_cp_buffer_alloc")
    return p.value


def _call(capi, q, kp, vp, table, L, gate, out, ws, bufs, world, rank, epoch):
    """Launches one exchange call; returns the device seq_len tensor, which the caller keeps
    alive until the stream has synchronised."""
    import torch
    arr = (C.c_void_p * world)(*bufs)
    seq = torch.tensor([L], dtype=torch.int32, device="cuda")
    capi.check(capi.lib().pgc_cp_decode_attn(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), kp.shape[0], table.data_ptr(), table.shape[-1],
        seq.data_ptr(), L, 1 / 16, gate.data_ptr(), out.data_ptr(),
        ws.data_ptr(), ws.numel(), arr, world, rank, epoch, None), "pgc_cp_decode_attn")
    return seq


def test_peer_exchange_single_rank_matches_oracle(cuda, oracle):
    import torch
    L = 3000
    kp, vp, table = _cache(oracle, L, 3)
    q = oracle.normal_bf16(NQ * D, 1).reshape(1, 1, NQ, D)
    g = oracle.normal_bf16(NQ * D, 2).reshape(NQ, D)
    ref, _ = oracle.decode_paged(q, kp, vp, table, np.array([L], np.int32), 1 / 16, 1, g.reshape(1, 1, NQ, D))
    kd, vd, td, qd, gd = dev(kp), dev(vp), dev(table), dev(q), dev(g)
    ws = torch.empty(cuda.decode_workspace_bytes(1, 1, L), dtype=torch.uint8, device="cuda")
    out = torch.empty((NQ, D), dtype=torch.int16, device="cuda")
    buf = _buffer(cuda, 1)
    try:
        for epoch in range(1, 5):
            out.zero_()
            seq = _call(cuda, qd, kd, vd, td, L, gd, out, ws, [buf], 1, 0, epoch)
            torch.cuda.synchronize()
            del seq
            assert_attn_close(host_u16(out), ref[0, 0])
        assert cuda.device_error() == (0, 0)
    finally:
        cuda.lib().pgc_cp_buffer_free(buf)


def test_peer_exchange_times_out_when_a_rank_never_arrives(cuda, oracle):
    import torch
    L = 200
    kp, vp, table = _cache(oracle, L, 5)
    q = oracle.normal_bf16(NQ * D, 6).reshape(1, 1, NQ, D)
    g = oracle.normal_bf16(NQ * D, 7).reshape(NQ, D)
    kd, vd, td, qd, gd = dev(kp), dev(vp), dev(table), dev(q), dev(g)
    ws = torch.empty(cuda.decode_workspace_bytes(1, 1, L), dtype=torch.uint8, device="cuda")
    out = torch.empty((NQ, D), dtype=torch.int16, device="cuda")
    own, absent = _buffer(cuda, 2), _buffer(cuda, 2)
    solo = _buffer(cuda, 1)
    try:
        cuda.device_error(clear=True)
        t0 = time.time()
        seq = _call(cuda, qd, kd, vd, td, L, gd, out, ws, [own, absent], 2, 0, 1)
        torch.cuda.synchronize()
        del seq
        waited = time.time() - t0
        code, detail = cuda.device_error(clear=True)
        assert code == 4 and detail == 1001, (code, detail)  # decode unit, wait timeout, rank 1's records
        assert 1.0 < waited < 30.0, waited
        # the context is still usable
        ref, _ = oracle.decode_paged(q, kp, vp, table, np.array([L], np.int32), 1 / 16, 1,
                                     g.reshape(1, 1, NQ, D))
        seq = _call(cuda, qd, kd, vd, td, L, gd, out, ws, [solo], 1, 0, 1)
        torch.cuda.synchronize()
        del seq
        assert_attn_close(host_u16(out), ref[0, 0])
        assert cuda.device_error() == (0, 0)
    finally:
        for b in (own, absent, solo):
            cuda.lib().pgc_cp_buffer_free(b)


def test_fused_append_matches_append_then_exchange(cuda, oracle):
    """A shard whose first global position is 40000 (so RoPE positions and pool indices differ)
    with the new token at its end: the fused call and the two calls give the same bits."""
    import torch
    from peregrine_b200 import cp
    L, start = 2500, 40000  # L cached tokens + the new one
    kp, vp, table = _cache(oracle, L + 1, 8)
    kp[(L) // PAGE, :, L % PAGE] = 0
    vp[(L) // PAGE, :, L % PAGE] = 0
    rope = torch.from_numpy(cuda.rope_table(start + L + 1)).cuda()
    qw = dev(oracle.normal_bf16(D, 9))
    kw = dev(oracle.normal_bf16(D, 10))
    pos = torch.tensor([start + L], dtype=torch.int32, device="cuda")
    slot = torch.tensor([L], dtype=torch.int64, device="cuda")
    seq = torch.tensor([L + 1], dtype=torch.int32, device="cuda")
    ws = torch.empty(cuda.decode_workspace_bytes(1, 1, L + 1), dtype=torch.uint8, device="cuda")
    outs = {}
    pools = {}
    for mode in ("fused", "two_calls"):
        kd, vd, td = dev(kp), dev(vp), dev(table)
        ex = cp.PeerExchange(1, 0)
        res = []
        try:
            for layer in range(3):
                q_in = dev(oracle.normal_bf16(NQ * 2 * D, 20 + layer).reshape(1, NQ, 2 * D))
                k_in = dev(oracle.normal_bf16(NKV * D, 30 + layer).reshape(1, NKV, D))
                v_in = dev(oracle.normal_bf16(NKV * D, 40 + layer).reshape(1, NKV, D))
                out = torch.empty((NQ, D), dtype=torch.int16, device="cuda")
                if mode == "fused":
                    ex.decode_layer_append(q_in, k_in, v_in, rope, pos, slot, start, kd, vd, td, seq, L + 1,
                                           1 / 16, ws, out, q_norm_w=qw, k_norm_w=kw)
                else:
                    q = torch.empty((1, NQ, D), dtype=torch.int16, device="cuda")
                    gate = torch.empty((1, NQ, D), dtype=torch.int16, device="cuda")
                    cuda.append_kv_rope(q_in, q, k_in, v_in, rope, pos, slot, kd, vd, gate_out=gate,
                                        q_norm_w=qw, k_norm_w=kw)
                    ex.decode_layer(q.view(1, 1, NQ, D), kd, vd, td, seq, L + 1, 1 / 16, ws, out,
                                    gate=gate.view(NQ, D))
                torch.cuda.synchronize()
                res.append(out.clone())
        finally:
            ex.close()
        outs[mode] = res
        pools[mode] = (kd.clone(), vd.clone())
    for a, b in zip(outs["fused"], outs["two_calls"]):
        assert torch.equal(a, b)
    assert torch.equal(pools["fused"][0], pools["two_calls"][0])
    assert torch.equal(pools["fused"][1], pools["two_calls"][1])
    assert cuda.device_error() == (0, 0)
