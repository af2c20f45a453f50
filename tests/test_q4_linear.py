"""q4 (group-64 affine) projections: the weight format of shaders/linear.metal:12-20.

CPU: the oracle's dequantisation against a numpy statement of the format (nibble order, group
scale and bias), and its projection against float64 sums over the unrounded weights.
GPU: pgc_q4_dequantize bit-exact against the oracle; pgc_q4_linear against the oracle (the
reference decode path's algebra: per group scale * sum(q x) + bias * sum(x), fp32) for the
model's projection shapes (q|gate 4096 -> 8192, k/v 4096 -> 1024, o 4096 -> 4096), token
counts 1-2 (the CUDA-core GEMV) and across the tcgen05 kernel's 16/32/64-token tiles plus a
multi-tile count, a partial 128-row tile
(out 192, 64) and in_dim 2048 and 8192 (every split-K cluster size). Tolerance for the projection: the GPU sums in the tensor
cores' order, so |y - y_ref| <= 1 bf16 ulp of |y_ref| + 1e-3 * rms(y_ref)."""
import numpy as np
import pytest


def _weights(oracle, out_dim, in_dim, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 2 ** 32, (out_dim, in_dim // 8), dtype=np.uint64).astype(np.uint32)
    sc = oracle.f32_to_bf16((rng.random((out_dim, in_dim // 64)) * 0.02 + 0.001).astype(np.float32))
    bi = oracle.f32_to_bf16((rng.standard_normal((out_dim, in_dim // 64)) * 0.05).astype(np.float32))
    return w, sc, bi


def _numpy_dequant(oracle, w, sc, bi):
    out_dim, words = w.shape
    q = np.stack([(w >> (4 * j)) & 0xF for j in range(8)], axis=-1).reshape(out_dim, words * 8)
    s = np.repeat(oracle.bf16_to_f32(sc), 64, axis=1)
    b = np.repeat(oracle.bf16_to_f32(bi), 64, axis=1)
    return (s * q.astype(np.float32)).astype(np.float32) + b


def test_oracle_dequant_matches_format(oracle):
    w, sc, bi = _weights(oracle, 16, 512, 1)
    d = oracle.q4_dequantize(w, sc, bi)
    ref = oracle.f32_to_bf16(_numpy_dequant(oracle, w, sc, bi).astype(np.float32))
    assert np.array_equal(d, ref)


def test_oracle_linear_matches_float64(oracle):
    """The decode projection keeps the weights unrounded (scale * sum(q x) + bias * sum(x))."""
    w, sc, bi = _weights(oracle, 64, 512, 2)
    x = oracle.normal_bf16(3 * 512, 3).reshape(3, 512)
    y = oracle.bf16_to_f32(oracle.q4_linear(x, w, sc, bi))
    q = np.stack([(w >> (4 * j)) & 0xF for j in range(8)], axis=-1).reshape(64, 512).astype(np.float64)
    wd = (np.repeat(oracle.bf16_to_f32(sc), 64, axis=1).astype(np.float64) * q
          + np.repeat(oracle.bf16_to_f32(bi), 64, axis=1))
    ref = oracle.bf16_to_f32(x).astype(np.float64) @ wd.T
    assert np.allclose(y, ref, rtol=2 ** -7, atol=1e-3 * np.sqrt((ref ** 2).mean()))


@pytest.mark.gpu
def test_q4_dequantize_bit_exact(cuda, oracle):
    import torch
    w, sc, bi = _weights(oracle, 1024, 4096, 4)
    out = torch.empty((1024, 4096), dtype=torch.int16, device="cuda")
    cuda.q4_dequantize(torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(sc.view(np.int16)).cuda(),
                       torch.from_numpy(bi.view(np.int16)).cuda(), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint16), oracle.q4_dequantize(w, sc, bi))


@pytest.mark.gpu
@pytest.mark.parametrize("out_dim,T,in_dim", [
    (8192, 1, 4096), (1024, 2, 4096), (4096, 3, 4096), (1024, 4, 8192), (64, 1, 2048),
    (1024, 7, 4096), (1024, 16, 4096), (1024, 17, 4096), (1024, 32, 4096),
    (4096, 33, 4096), (1024, 48, 4096), (1024, 64, 4096), (1024, 130, 4096),
    (192, 5, 2048), (64, 64, 2048), (1024, 9, 8192), (4096, 64, 8192), (1024, 1000, 2048)])
def test_q4_linear_matches_oracle(cuda, oracle, out_dim, T, in_dim):
    import torch
    w, sc, bi = _weights(oracle, out_dim, in_dim, 10 + T)
    x = oracle.normal_bf16(T * in_dim, 20 + T).reshape(T, in_dim)
    y = torch.empty((T, out_dim), dtype=torch.int16, device="cuda")
    cuda.q4_linear(torch.from_numpy(x.view(np.int16)).cuda(), torch.from_numpy(w.view(np.int32)).cuda(),
                   torch.from_numpy(sc.view(np.int16)).cuda(), torch.from_numpy(bi.view(np.int16)).cuda(), y)
    torch.cuda.synchronize()
    got = oracle.bf16_to_f32(y.cpu().numpy().view(np.uint16))
    ref = oracle.bf16_to_f32(oracle.q4_linear(x, w, sc, bi))
    tol = np.abs(ref) * 2 ** -7 + 1e-3 * np.sqrt((ref ** 2).mean())
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} beyond tolerance, max {np.abs(got - ref).max():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 2, 5, 64])
def test_q4_linear_multi_matches_single(cuda, oracle, T):
    """pgc_q4_linear_multi over the decode step's weights that share x (q | gate 8192, k 1024,
    v 1024): at 1-2 tokens one grouped GEMV launch, beyond that one tensor-core pass per
    weight; each output bit-identical to pgc_q4_linear on that weight alone and within the
    projection tolerance of the oracle."""
    import torch
    in_dim = 4096
    outs = [8192, 1024, 1024]
    ws = [_weights(oracle, o, in_dim, 30 + i) for i, o in enumerate(outs)]
    x = oracle.normal_bf16(T * in_dim, 40 + T).reshape(T, in_dim)

    def dv(a, dt):
        return torch.from_numpy(a.view(dt)).cuda()

    xd = dv(x, np.int16)
    wd = [(dv(w, np.int32), dv(sc, np.int16), dv(bi, np.int16)) for w, sc, bi in ws]
    multi = [torch.empty((T, o), dtype=torch.int16, device="cuda") for o in outs]
    cuda.q4_linear_multi(xd, [a for a, _, _ in wd], [b for _, b, _ in wd], [c for _, _, c in wd], multi)
    single = [torch.empty((T, o), dtype=torch.int16, device="cuda") for o in outs]
    for (a, b, c), y in zip(wd, single):
        cuda.q4_linear(xd, a, b, c, y)
    torch.cuda.synchronize()
    for i, (m, s1) in enumerate(zip(multi, single)):
        assert torch.equal(m, s1), i
    w0, sc0, bi0 = ws[1]
    got = oracle.bf16_to_f32(multi[1].cpu().numpy().view(np.uint16))
    ref = oracle.bf16_to_f32(oracle.q4_linear(x, w0, sc0, bi0))
    tol = np.abs(ref) * 2 ** -7 + 1e-3 * np.sqrt((ref ** 2).mean())
    assert not (np.abs(got - ref) > tol).any()
