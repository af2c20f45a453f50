"""pgc_decode_attn_static: the decode entry point for callers that cannot allocate device
memory (a host whose allocator owns the GPU, a serving loop that forbids allocation after
start-up, a plugin handed only its input and output buffers). It takes no workspace and keeps
its split partials in the library's fixed device array. Checked through the C ABI: bit for bit
against the workspace entry point pgc_decode_attn (the same kernels and split plan), and
against the CPU oracle within the attention tolerance (2e-2 abs + 1e-2 rel), on two calls in a
row; a second call reserves no device memory; shapes beyond the array are rejected. Named to
be collected last."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, assert_attn_close, dev, host_u16, paged_pools

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 16


def _inputs(oracle, lens, seed, nq):
    rng = np.random.default_rng(seed)
    ks = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b).reshape(L, NKV, D) for b, L in enumerate(lens)]
    vs = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b + 1).reshape(L, NKV, D) for b, L in enumerate(lens)]
    kp, vp, table = paged_pools(rng, ks, vs, sum((L + PAGE - 1) // PAGE for L in lens) + 3)
    q = oracle.normal_bf16(len(lens) * nq * NQ * D, seed + 50).reshape(len(lens), nq, NQ, D)
    g = oracle.normal_bf16(q.size, seed + 51).reshape(q.shape)
    host = (q, kp, vp, table, np.array(lens, np.int32), g)
    return host, [dev(x) for x in host]


def test_static_scratch_matches_workspace_entry(cuda, oracle):
    import torch
    cases = [([4097], 1, 1), ([3000, 17, 1025, 800], 2, 2)]  # two calls in a row
    for lens, nq, seed in cases:
        host, (q, kp, vp, table, seq, g) = _inputs(oracle, lens, seed, nq)
        max_len = max(lens)
        out_static = torch.full((len(lens), nq, NQ, D), -1, dtype=torch.int16, device="cuda")
        cuda.decode_attn_static(q, kp, vp, table, seq, max_len, SCALE, out_static,
                                num_queries=nq, gate=g)
        ws = torch.empty(cuda.decode_workspace_bytes(len(lens), nq, max_len), dtype=torch.uint8,
                         device="cuda")
        out_ws = torch.empty_like(out_static)
        cuda.decode_attn(q, kp, vp, table, seq, max_len, SCALE, out_ws, ws, num_queries=nq, gate=g)
        torch.cuda.synchronize()
        a, b = host_u16(out_static), host_u16(out_ws)
        assert np.array_equal(a, b), f"{int((a != b).sum())} elements differ from pgc_decode_attn"
        hq, hkp, hvp, htable, hseq, hg = host
        ref, _ = oracle.decode_paged(hq, hkp, hvp, htable, hseq, SCALE, num_queries=nq, gate=hg)
        assert_attn_close(a, ref)


def test_static_scratch_allocates_nothing(cuda, oracle):
    import torch
    _, (q, kp, vp, table, seq, g) = _inputs(oracle, [2048, 513], 3, 1)
    out = torch.empty((2, 1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn_static(q, kp, vp, table, seq, 2048, SCALE, out, gate=g)  # set-up call
    first = out.clone()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    cuda.decode_attn_static(q, kp, vp, table, seq, 2048, SCALE, out, gate=g)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device memory changed by {free0 - free1} bytes"
    assert torch.equal(first, out)


def test_static_scratch_rejects_oversize(cuda):
    import torch
    from peregrine_b200.capi import PgcError
    batch, max_len = 64, 65536
    assert cuda.decode_workspace_bytes(batch, 1, max_len) > 16 << 20
    q = torch.zeros((batch, 1, NQ, D), dtype=torch.int16, device="cuda")
    pool = torch.zeros((8, NKV, PAGE, D), dtype=torch.int16, device="cuda")
    table = torch.zeros((batch, max_len // PAGE), dtype=torch.int32, device="cuda")
    seq = torch.ones(batch, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(PgcError, match="WORKSPACE"):
        cuda.decode_attn_static(q, pool, pool, table, seq, max_len, SCALE, out)
