"""GPU parity of the tcgen05 chunked-prefill attention against the CPU oracle, through the C
ABI. Tolerance: |gpu - oracle| <= 2e-2 + 1e-2 |oracle| (fp32 oracle)."""
import numpy as np
import pytest

from _util import NKV, NQ, D, PAGE, assert_attn_close, dev, host_u16, paged_pools

pytestmark = pytest.mark.gpu
SCALE = 1.0 / 16


def _setup(oracle, P, T, seed, spare=5, nan_tail=False):
    n = P + T
    rng = np.random.default_rng(seed)
    k = oracle.normal_bf16(n * NKV * D, seed * 10 + 1).reshape(n, NKV, D)
    v = oracle.normal_bf16(n * NKV * D, seed * 10 + 2).reshape(n, NKV, D)
    kp, vp, table = paged_pools(rng, [k], [v], (n + PAGE - 1) // PAGE + spare)
    if nan_tail and n % PAGE:
        kp[table[0, n // PAGE], :, n % PAGE:] = 0x7FC0
        vp[table[0, n // PAGE], :, n % PAGE:] = 0x7FC0
    q = oracle.normal_bf16(T * NQ * D, seed * 10 + 3).reshape(T, NQ, D)
    return q, kp, vp, table[0]


def _gpu(cuda, q, kp, vp, table, P, T):
    import torch
    out = torch.full((T, NQ, D), -1, dtype=torch.int16, device="cuda")
    nbytes = cuda.prefill_workspace_bytes(P, T)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda") if nbytes else None
    cuda.prefill_attn(dev(q), dev(kp), dev(vp), dev(table), P, T, SCALE, out, ws)
    torch.cuda.synchronize()
    return host_u16(out)


@pytest.mark.parametrize("P,T", [(0, 1), (0, 40), (100, 70), (1000, 33), (777, 129), (64, 64),
                                 (5, 300), (3000, 37), (9000, 96)])
def test_prefill_small(cuda, oracle, P, T):
    q, kp, vp, table = _setup(oracle, P, T, seed=P + T, nan_tail=True)
    got = _gpu(cuda, q, kp, vp, table, P, T)
    ref, _ = oracle.prefill_paged(q, kp, vp, table, P, T, SCALE)
    assert_attn_close(got, ref)


def config2_rows(T=1600):
    """Query rows checked at the config-2 shape: one row in every 64-token pair tile (at a
    different offset in each, covering both CTAs of a pair), the edges of the first pair and of
    its two 32-token halves, and the last rows of the chunk (the causal diagonal's end)."""
    rows = {64 * c + (c * 23) % 64 for c in range(T // 64)}
    rows |= {0, 1, 31, 32, 63, 64, T - 4, T - 3, T - 2, T - 1}
    return sorted(r for r in rows if r < T)


def test_prefill_config2_shape(cuda, oracle):
    """BASELINE config 2 attention shape: 1600-token chunk over a 24576-token prefix, which the
    kernel runs as 25 pair tiles x 4 kv heads x 2 key-range shares merged afterwards (every
    row's keys straddle the share boundary, which sits inside the prefix). Rows of
    config2_rows() are checked against the oracle restricted to that query position, and the
    last token against the decode kernel over the same cache."""
    import torch
    P, T = 24576, 1600
    assert cuda.prefill_workspace_bytes(P, T) == 2 * T * NQ * 258 * 4  # the two-share plan
    q, kp, vp, table = _setup(oracle, P, T, seed=2, spare=0)
    got = _gpu(cuda, q, kp, vp, table, P, T)
    rows = config2_rows(T)
    assert len(rows) >= 25 + 8
    for t in rows:
        ref, _ = oracle.prefill_paged(np.ascontiguousarray(q[t:t + 1]), kp, vp, table, P + t, 1, SCALE)
        assert_attn_close(got[t:t + 1], ref)
    n = P + T
    ws = torch.empty(cuda.decode_workspace_bytes(1, 1, n), dtype=torch.uint8, device="cuda")
    out = torch.empty((1, 1, NQ, D), dtype=torch.int16, device="cuda")
    cuda.decode_attn(dev(np.ascontiguousarray(q[-1:])), dev(kp), dev(vp), dev(table.reshape(1, -1)),
                     dev(np.array([n], np.int32)), n, SCALE, out, ws)
    torch.cuda.synchronize()
    dec = (host_u16(out).reshape(NQ, D).astype(np.uint32) << 16).view(np.float32)
    assert_attn_close(got[-1], dec)
    code, _ = cuda.device_error()
    assert code == 0


def test_prefill_workspace_rules(cuda):
    import torch
    from peregrine_b200.capi import PgcError
    # T=1152: 18 pair columns x 4 kv heads = 72 pairs, one nearly full wave on 74 pair slots
    assert cuda.prefill_workspace_bytes(24576, 1152) == 0
    # config 2: 100 pairs fill 68 % of two waves; two key-range shares fill 90 % of three
    assert cuda.prefill_workspace_bytes(24576, 1600) == 2 * 1600 * NQ * 258 * 4
    P, T = 24576, 96  # 12 CTAs: the key range is split, partials need a workspace
    nbytes = cuda.prefill_workspace_bytes(P, T)
    assert nbytes > 0 and nbytes % (T * NQ * 258 * 4) == 0
    q = torch.zeros((T, NQ, D), dtype=torch.int16, device="cuda")
    pool = torch.zeros(((P + T) // PAGE + 1, NKV, PAGE, D), dtype=torch.int16, device="cuda")
    table = torch.arange(pool.shape[0], dtype=torch.int32, device="cuda")
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(PgcError, match="WORKSPACE"):
        cuda.prefill_attn(q, pool, pool, table, P, T, SCALE, q, small)
