"""Linear-attention state producers: causal conv1d + SiLU and the gated delta-rule recurrence.

CPU: the oracle (oracle/pgo_linear.c) against an independent numpy statement of the same
mathematics (different summation order: agreement to float rounding), conv1d prefill against
repeated decode steps (bit-exact: same products in the same order), and gated-delta prefill
against repeated decode steps (the reference's two q/k norm reductions differ in order only).
GPU: every entry point against the oracle on the same seeded inputs. Tolerances: conv state
bit-exact (a copy of inputs); conv output and y within 1 bf16 ulp plus 1e-6 (decode: only
CUDA's expf/logf differ from libm's; prefill also regroups the recurrence into 64-token chunks,
the same fp32 arithmetic in another order); recurrent state within 1e-5 relative + 1e-6
absolute after up to 1600 tokens."""
import numpy as np
import pytest

CONV, K, HK, HV, DK, DV = 8192, 4, 16, 32, 128, 128
KEY = HK * DK


def _inputs(oracle, seed, T=1):
    rng = np.random.default_rng(seed)
    conv_out = oracle.normal_bf16(T * CONV, seed).reshape(T, CONV)
    a = oracle.normal_bf16(T * HV, seed + 1).reshape(T, HV)
    b = oracle.normal_bf16(T * HV, seed + 2).reshape(T, HV)
    a_log = (rng.standard_normal(HV) * 0.5 - 1.0).astype(np.float32)
    dt_bias = oracle.normal_bf16(HV, seed + 3)
    return conv_out, a, b, a_log, dt_bias


def _bf(oracle, x):
    return oracle.bf16_to_f32(np.ascontiguousarray(x))


def _close_bf16(got, ref, what):
    """Within one bf16 ulp of the reference value (plus 1e-6 for values near zero)."""
    g = got.astype(np.float32)
    r = ref.astype(np.float32)
    ulp = np.abs(r) * 2.0 ** -7
    bad = np.abs(g - r) > ulp + 1e-6
    assert not bad.any(), f"{what}: {bad.sum()} values beyond 1 bf16 ulp, max {np.abs(g - r).max():.3e}"


# ---------------------------------------------------------------- CPU: oracle self-consistency

def test_gated_delta_oracle_matches_numpy_statement(oracle):
    """One decode step of the oracle against the textbook recurrence in float64."""
    conv_out, a, b, a_log, dt_bias = _inputs(oracle, 10)
    rng = np.random.default_rng(11)
    state0 = (rng.standard_normal((HV, DV, DK)) * 0.1).astype(np.float32)
    st = state0.copy()
    y = oracle.gated_delta_decode(st, 1, conv_out[0], a[0], b[0], a_log, dt_bias)
    x = _bf(oracle, conv_out[0]).astype(np.float64)
    af, bf_, dtb = (_bf(oracle, a[0]).astype(np.float64), _bf(oracle, b[0]).astype(np.float64),
                    _bf(oracle, dt_bias).astype(np.float64))
    S = state0.astype(np.float64)
    y_ref = np.zeros(HV * DV)
    for hv in range(HV):
        hk = hv // 2
        q = x[hk * DK:(hk + 1) * DK]
        k = x[KEY + hk * DK:KEY + (hk + 1) * DK]
        q = q / np.sqrt((q * q).sum() + 1e-6) / np.sqrt(DK)
        k = k / np.sqrt((k * k).sum() + 1e-6)
        g = af[hv] + dtb[hv]
        decay = np.exp(-np.exp(a_log[hv]) * np.logaddexp(0.0, g))
        beta = 1.0 / (1.0 + np.exp(-bf_[hv]))
        v = x[2 * KEY + hv * DV:2 * KEY + (hv + 1) * DV]
        Sd = S[hv] * decay
        delta = (v - Sd @ k) * beta
        S[hv] = Sd + np.outer(delta, k)
        y_ref[hv * DV:(hv + 1) * DV] = S[hv] @ q
    assert np.allclose(st, S, rtol=1e-5, atol=1e-6)
    _close_bf16(_bf(oracle, y), oracle.bf16_to_f32(oracle.f32_to_bf16(y_ref.astype(np.float32))), "y")


def test_conv1d_prefill_equals_repeated_decode(oracle):
    rng = np.random.default_rng(3)
    w = oracle.normal_bf16(CONV * K, 4)
    for has_state, T in [(1, 9), (0, 2), (1, 1)]:
        st0 = rng.standard_normal((K - 1, CONV)).astype(np.float32)
        x = oracle.normal_bf16(T * CONV, 5 + T).reshape(T, CONV)
        s_pref = st0.copy() if has_state else np.zeros_like(st0)
        out_p = oracle.conv1d_prefill(s_pref, has_state, x, w)
        s_dec = st0.copy() if has_state else np.zeros_like(st0)
        outs = [oracle.conv1d_decode(s_dec, x[t], w) for t in range(T)]
        assert np.array_equal(out_p, np.stack(outs))
        assert np.array_equal(s_pref, s_dec)


def test_gated_delta_prefill_tracks_repeated_decode(oracle):
    T = 12
    conv_out, a, b, a_log, dt_bias = _inputs(oracle, 20, T)
    s_p = np.zeros((HV, DV, DK), np.float32)
    y_p = oracle.gated_delta_prefill(s_p, 0, conv_out, a, b, a_log, dt_bias)
    s_d = np.zeros_like(s_p)
    ys = []
    for t in range(T):
        ys.append(oracle.gated_delta_decode(s_d, 1 if t else 0, conv_out[t], a[t], b[t], a_log, dt_bias))
    assert np.allclose(s_p, s_d, rtol=1e-5, atol=1e-6)
    _close_bf16(_bf(oracle, y_p), _bf(oracle, np.stack(ys)), "y")


# ---------------------------------------------------------------- GPU parity

@pytest.mark.gpu
def test_conv1d_decode_batch_with_slots(cuda, oracle):
    import torch
    from _util import dev
    rng = np.random.default_rng(7)
    B, slots_n = 5, 9
    w = oracle.normal_bf16(CONV * K, 8)
    states = rng.standard_normal((slots_n, K - 1, CONV)).astype(np.float32)
    slots = np.array([7, 0, 3, 8, 2], np.int32)
    x = oracle.normal_bf16(B * CONV, 9).reshape(B, CONV)
    st_d = torch.from_numpy(states.copy()).cuda()
    out = torch.empty((B, CONV), dtype=torch.int16, device="cuda")
    cuda.conv1d_decode(st_d, dev(x), dev(w), out, slots=dev(slots))
    torch.cuda.synchronize()
    ref_states = states.copy()
    for i, s in enumerate(slots):
        ref = oracle.conv1d_decode(ref_states[s], x[i], w)
        _close_bf16(_bf(oracle, out[i].cpu().numpy().view(np.uint16)), _bf(oracle, ref), "conv out")
    assert np.array_equal(st_d.cpu().numpy(), ref_states)  # untouched slots included


@pytest.mark.gpu
@pytest.mark.parametrize("has_state,T", [(1, 1), (1, 2), (0, 3), (1, 130), (0, 1600)])
def test_conv1d_prefill(cuda, oracle, has_state, T):
    import torch
    from _util import dev
    rng = np.random.default_rng(T)
    w = oracle.normal_bf16(CONV * K, 30)
    st0 = rng.standard_normal((K - 1, CONV)).astype(np.float32)
    x = oracle.normal_bf16(T * CONV, 31).reshape(T, CONV)
    st_d = torch.from_numpy(st0.copy()).cuda()
    out = torch.empty((T, CONV), dtype=torch.int16, device="cuda")
    cuda.conv1d_prefill(st_d, has_state, dev(x), dev(w), out)
    torch.cuda.synchronize()
    st_ref = st0.copy()
    ref = oracle.conv1d_prefill(st_ref, has_state, x, w)
    _close_bf16(_bf(oracle, out.cpu().numpy().view(np.uint16)), _bf(oracle, ref), "conv out")
    assert np.array_equal(st_d.cpu().numpy(), st_ref)


@pytest.mark.gpu
def test_gated_delta_decode_batch_with_slots(cuda, oracle):
    import torch
    from _util import dev
    rng = np.random.default_rng(12)
    B, nslots = 3, 4
    conv_out, a, b, a_log, dt_bias = _inputs(oracle, 40, B)
    states = (rng.standard_normal((nslots, HV, DV, DK)) * 0.1).astype(np.float32)
    slots = np.array([2, 0, 3], np.int32)
    st_d = torch.from_numpy(states.copy()).cuda()
    y = torch.empty((B, HV * DV), dtype=torch.int16, device="cuda")
    cuda.gated_delta_decode(st_d, True, dev(conv_out), dev(a), dev(b), torch.from_numpy(a_log).cuda(),
                            dev(dt_bias), y, slots=dev(slots))
    torch.cuda.synchronize()
    ref_states = states.copy()
    got = st_d.cpu().numpy()
    for i, s in enumerate(slots):
        yr = oracle.gated_delta_decode(ref_states[s], 1, conv_out[i], a[i], b[i], a_log, dt_bias)
        _close_bf16(_bf(oracle, y[i].cpu().numpy().view(np.uint16)), _bf(oracle, yr), "y")
    assert np.allclose(got, ref_states, rtol=1e-5, atol=1e-6)
    assert np.array_equal(got[1], states[1])  # slot 1 not in the batch


@pytest.mark.gpu
@pytest.mark.parametrize("has_state,T", [(0, 1), (1, 5), (0, 257), (1, 1600)])
def test_gated_delta_prefill(cuda, oracle, has_state, T):
    import torch
    from _util import dev
    rng = np.random.default_rng(50 + T)
    conv_out, a, b, a_log, dt_bias = _inputs(oracle, 60 + T, T)
    st0 = (rng.standard_normal((HV, DV, DK)) * 0.1).astype(np.float32)
    st_d = torch.from_numpy(st0.copy()).cuda()
    y = torch.empty((T, HV * DV), dtype=torch.int16, device="cuda")
    ws = torch.empty(cuda.gated_delta_prefill_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    cuda.gated_delta_prefill(st_d, has_state, dev(conv_out), dev(a), dev(b),
                             torch.from_numpy(a_log).cuda(), dev(dt_bias), y, ws)
    torch.cuda.synchronize()
    st_ref = st0.copy()
    yr = oracle.gated_delta_prefill(st_ref, has_state, conv_out, a, b, a_log, dt_bias)
    assert np.allclose(st_d.cpu().numpy(), st_ref, rtol=1e-5, atol=1e-6)
    _close_bf16(_bf(oracle, y.cpu().numpy().view(np.uint16)), _bf(oracle, yr), "y")


@pytest.mark.gpu
@pytest.mark.parametrize("cut", [128, 100])
def test_gated_delta_prefill_across_calls(cuda, oracle, cut):
    """The state carries across calls: prefill of 160 tokens against `cut` + the rest. At a
    64-token chunk boundary (128) the arithmetic is the same, so the results are bitwise equal;
    elsewhere (100) the chunks regroup the same fp32 recurrence, within the state tolerance."""
    import torch
    from _util import dev
    T = 160
    conv_out, a, b, a_log, dt_bias = _inputs(oracle, 70, T)
    al = torch.from_numpy(a_log).cuda()
    ws = torch.empty(cuda.gated_delta_prefill_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    s1 = torch.zeros((HV, DV, DK), dtype=torch.float32, device="cuda")
    y1 = torch.empty((T, HV * DV), dtype=torch.int16, device="cuda")
    cuda.gated_delta_prefill(s1, 0, dev(conv_out), dev(a), dev(b), al, dev(dt_bias), y1, ws)
    s2 = torch.zeros_like(s1)
    y2 = torch.empty_like(y1)
    for lo, hi, has in [(0, cut, 0), (cut, T, 1)]:
        cuda.gated_delta_prefill(s2, has, dev(conv_out[lo:hi]), dev(a[lo:hi]), dev(b[lo:hi]), al,
                                 dev(dt_bias), y2[lo:hi], ws)
    torch.cuda.synchronize()
    if cut % 64 == 0:
        assert torch.equal(s1, s2) and torch.equal(y1, y2)
    else:
        assert np.allclose(s2.cpu().numpy(), s1.cpu().numpy(), rtol=1e-5, atol=1e-6)
        _close_bf16(_bf(oracle, y2.cpu().numpy().view(np.uint16)), _bf(oracle, y1.cpu().numpy().view(np.uint16)), "y")
