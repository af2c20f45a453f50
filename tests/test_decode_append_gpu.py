"""pgc_decode_attn_append (the decode append fused into the split-K decode) against the two
calls it replaces, pgc_append_kv_rope (decode mode) then pgc_decode_attn, on the same inputs:
the attention output and the pools after the call are bit-exact, and the output is also checked
against the oracle within the attention tolerance. Cases: BASELINE config 1 (one row at position
4096), ragged batches at 1-4 queries per sequence whose new tokens straddle page and split
boundaries, q with and without the packed gate and norm weights, a padding token (slot -1) and
an out-of-range position (recorded in the decode unit of pgc_device_error)."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, assert_attn_close, dev, host_u16, paged_pools

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 16


def _setup(oracle, lens, nq, seed, packed, norm, spare_pages=6):
    """Pools whose sequences already hold every token but the last nq (those rows hold stale
    data that the append overwrites); returns host arrays."""
    rng = np.random.default_rng(seed)
    ks = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b + 1).reshape(L, NKV, D) for b, L in enumerate(lens)]
    vs = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b + 2).reshape(L, NKV, D) for b, L in enumerate(lens)]
    npages = sum((L + PAGE - 1) // PAGE for L in lens) + spare_pages
    kp, vp, table = paged_pools(rng, ks, vs, npages)
    B = len(lens)
    T = B * nq
    q_in = oracle.normal_bf16(T * NQ * (2 if packed else 1) * D, seed + 11).reshape(T, NQ, -1)
    k_in = oracle.normal_bf16(T * NKV * D, seed + 12).reshape(T, NKV, D)
    v_in = oracle.normal_bf16(T * NKV * D, seed + 13).reshape(T, NKV, D)
    qw = oracle.normal_bf16(D, seed + 14) if norm else None
    kw = oracle.normal_bf16(D, seed + 15) if norm else None
    pos = np.array([L - nq + j for L in lens for j in range(nq)], np.int32)
    slots = np.array([table[b, p // PAGE] * PAGE + p % PAGE
                      for b in range(B) for p in pos[b * nq:(b + 1) * nq]], np.int64)
    seq = np.array(lens, np.int32)
    return dict(kp=kp, vp=vp, table=table, q_in=q_in, k_in=k_in, v_in=v_in, qw=qw, kw=kw, pos=pos,
                slots=slots, seq=seq, rope=oracle.rope_table(max(lens) + 8))


def _two_calls(cuda, c, nq, max_len):
    import torch
    T = c["pos"].shape[0]
    kp, vp = dev(c["kp"]), dev(c["vp"])
    q = torch.zeros((T, NQ, D), dtype=torch.int16, device="cuda")
    packed = c["q_in"].shape[-1] == 2 * D
    gate = torch.zeros((T, NQ, D), dtype=torch.int16, device="cuda") if packed else None
    opt = lambda a: None if a is None else dev(a)
    cuda.append_kv_rope(dev(c["q_in"]), q, dev(c["k_in"]), dev(c["v_in"]), dev(c["rope"]), dev(c["pos"]),
                        dev(c["slots"]), kp, vp, gate_out=gate, q_norm_w=opt(c["qw"]), k_norm_w=opt(c["kw"]))
    B = c["seq"].shape[0]
    ws = torch.empty(cuda.decode_workspace_bytes(B, nq, max_len), dtype=torch.uint8, device="cuda")
    out = torch.empty((B, nq, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(q, kp, vp, dev(c["table"]), dev(c["seq"]), max_len, SCALE, out, ws, num_queries=nq,
                     gate=gate)
    torch.cuda.synchronize()
    return host_u16(out), host_u16(kp), host_u16(vp), host_u16(q), None if gate is None else host_u16(gate)


def _fused(cuda, c, nq, max_len):
    import torch
    kp, vp = dev(c["kp"]), dev(c["vp"])
    B = c["seq"].shape[0]
    ws = torch.empty(cuda.decode_workspace_bytes(B, nq, max_len), dtype=torch.uint8, device="cuda")
    out = torch.empty((B, nq, NQ, D), dtype=torch.int16, device="cuda")
    opt = lambda a: None if a is None else dev(a)
    cuda.decode_attn_append(dev(c["q_in"]), dev(c["k_in"]), dev(c["v_in"]), dev(c["rope"]), dev(c["pos"]),
                            dev(c["slots"]), kp, vp, dev(c["table"]), dev(c["seq"]), max_len, SCALE, out, ws,
                            num_queries=nq, q_norm_w=opt(c["qw"]), k_norm_w=opt(c["kw"]))
    torch.cuda.synchronize()
    return host_u16(out), host_u16(kp), host_u16(vp)


def _check(cuda, oracle, c, nq):
    max_len = int(c["seq"].max())
    ref_out, ref_kp, ref_vp, q_rot, gate = _two_calls(cuda, c, nq, max_len)
    out, kp, vp = _fused(cuda, c, nq, max_len)
    assert np.array_equal(kp, ref_kp)
    assert np.array_equal(vp, ref_vp)
    assert np.array_equal(out, ref_out)
    B = c["seq"].shape[0]
    g = None if gate is None else gate.reshape(B, nq, NQ, D)
    ref, _ = oracle.decode_paged(q_rot.reshape(B, nq, NQ, D), kp, vp, c["table"], c["seq"], SCALE, nq, g)
    assert_attn_close(out, ref)


@pytest.mark.parametrize("packed,norm", [(False, False), (True, True)])
def test_config1_fused_matches_two_calls(cuda, oracle, packed, norm):
    c = _setup(oracle, [4097], 1, 1, packed, norm, spare_pages=0)
    _check(cuda, oracle, c, 1)


@pytest.mark.parametrize("nq", [1, 2, 3, 4])
def test_ragged_batch_fused_matches_two_calls(cuda, oracle, nq):
    # new tokens at page starts, page ends and across page boundaries; 1040 and 4097 cross
    # split boundaries (4-page splits at this batch)
    lens = [max(nq, L) for L in [1, 16, 17, 33, 64, 1040, 4097, 20001]]
    c = _setup(oracle, lens, nq, 10 + nq, packed=(nq % 2 == 0), norm=(nq >= 3))
    _check(cuda, oracle, c, nq)


def test_padding_token_and_bad_position(cuda, oracle):
    c = _setup(oracle, [300, 47], 2, 5, packed=True, norm=True)
    c["slots"][1] = -1  # padding: nothing appended, the row keeps its bytes
    max_len = int(c["seq"].max())
    ref_out, ref_kp, ref_vp, _, _ = _two_calls(cuda, c, 2, max_len)
    out, kp, vp = _fused(cuda, c, 2, max_len)
    assert np.array_equal(kp, ref_kp) and np.array_equal(vp, ref_vp) and np.array_equal(out, ref_out)
    cuda.device_error(clear=True)
    bad = dict(c)
    bad["pos"] = c["pos"].copy()
    bad["pos"][2] = 1 << 30  # beyond the RoPE table: recorded, not faulted
    _fused(cuda, bad, 2, max_len)
    code, detail = cuda.device_error(clear=True)
    assert code == 3 and detail == 2, (code, detail)  # decode unit, position out of range, token 2
    assert cuda.device_error() == (0, 0)
