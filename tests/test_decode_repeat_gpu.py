"""Decode calls that reuse one workspace, through the C ABI: a workspace full of garbage
(finite bytes, or all-ones words that read as NaN, which splits past a sequence's end leave in
place under their empty partials) needs no initialisation, repeated calls and replays of one captured CUDA graph give identical
bits, and a batch too large for one wave of CTAs agrees with the same sequences decoded alone
(one wave), all against the CPU oracle (2e-2 abs + 1e-2 rel)."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, assert_attn_close, dev, host_u16, paged_pools

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 16


def _case(oracle, lens, nq, seed):
    rng = np.random.default_rng(seed)
    ks = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b).reshape(L, NKV, D) for b, L in enumerate(lens)]
    vs = [oracle.normal_bf16(L * NKV * D, seed * 100 + 2 * b + 1).reshape(L, NKV, D) for b, L in enumerate(lens)]
    kp, vp, table = paged_pools(rng, ks, vs, sum((L + PAGE - 1) // PAGE for L in lens) + 5)
    q = oracle.normal_bf16(len(lens) * nq * NQ * D, seed + 7).reshape(len(lens), nq, NQ, D)
    g = oracle.normal_bf16(q.size, seed + 8).reshape(q.shape)
    return (q, kp, vp, table, np.array(lens, np.int32), g)


@pytest.mark.parametrize("lens,nq,fill", [([4097], 1, 0xA5), ([32770], 2, 0xA5), ([65536], 1, 0xA5),
                                          ([5000, 3, 70, 12000], 3, 0xA5), ([5000, 3, 70, 12000], 3, 0xFF),
                                          ([40000, 1, 16, 17], 1, 0xFF)])
def test_garbage_workspace_and_repeated_calls(cuda, oracle, lens, nq, fill):
    import torch
    host = _case(oracle, lens, nq, len(lens) + nq)
    q, kp, vp, table, seq, g = [dev(x) for x in host]
    max_len = max(lens)
    ws = torch.full((cuda.decode_workspace_bytes(len(lens), nq, max_len),), fill, dtype=torch.uint8,
                    device="cuda")
    outs = []
    for _ in range(3):
        out = torch.full((len(lens), nq, NQ, D), -1, dtype=torch.int16, device="cuda")
        cuda.decode_attn(q, kp, vp, table, seq, max_len, SCALE, out, ws, num_queries=nq, gate=g)
        outs.append(out)
    torch.cuda.synchronize()
    ref, _ = oracle.decode_paged(host[0], host[1], host[2], host[3], host[4], SCALE, nq, host[5])
    assert_attn_close(host_u16(outs[0]), ref)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    code, _ = cuda.device_error()
    assert code == 0


def test_graph_replays_are_identical(cuda, oracle):
    import torch
    host = _case(oracle, [8000, 300], 1, 11)
    q, kp, vp, table, seq, g = [dev(x) for x in host]
    ws = torch.empty(cuda.decode_workspace_bytes(2, 1, 8000), dtype=torch.uint8, device="cuda")
    out = torch.empty((2, 1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(q, kp, vp, table, seq, 8000, SCALE, out, ws, gate=g)  # warm-up outside capture
    torch.cuda.synchronize()
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=s):
        cuda.decode_attn(q, kp, vp, table, seq, 8000, SCALE, out, ws, gate=g, stream=s)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        out.fill_(-1)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, first)
    code, _ = cuda.device_error()
    assert code == 0


def test_one_wave_and_many_wave_paths_agree(cuda, oracle):
    """A 24-sequence batch of long contexts takes several waves of split CTAs; its first two
    sequences alone take one wave with a different split size. Both match the oracle."""
    import torch
    lens = [30000, 9000] + [20000] * 22
    host = _case(oracle, lens, 1, 21)
    q, kp, vp, table, seq, g = [dev(x) for x in host]
    ws = torch.empty(cuda.decode_workspace_bytes(len(lens), 1, 30000), dtype=torch.uint8, device="cuda")
    big = torch.empty((len(lens), 1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(q, kp, vp, table, seq, 30000, SCALE, big, ws, gate=g)
    ws2 = torch.empty(cuda.decode_workspace_bytes(2, 1, 30000), dtype=torch.uint8, device="cuda")
    small = torch.empty((2, 1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(q[:2], kp, vp, table[:2], seq[:2], 30000, SCALE, small, ws2, gate=g[:2])
    torch.cuda.synchronize()
    ref, _ = oracle.decode_paged(host[0][:2].copy(), host[1], host[2], host[3][:2].copy(), host[4][:2].copy(),
                                 SCALE, 1, host[5][:2].copy())
    assert_attn_close(host_u16(small), ref)
    assert_attn_close(host_u16(big)[:2], ref)
    code, _ = cuda.device_error()
    assert code == 0
