"""pgc_prefill_linear: the prefill projections' dense GEMM (tcgen05, two-SM tiles of 256 x 256),
through the C ABI. The reference path dequantises each q4 weight once (checked bit-exact in
test_q4_linear.py) and multiplies the chunk by it with fp32 accumulation and a bf16 result
(src/model/block_attn.zig:96-108, src/model/mlx_nt.zig). The check is a float64 product of the
same bf16 operands, rounded only at the end; the GPU sums in the tensor cores' order, so the
tolerance is 1 bf16 ulp of |y_ref| + 1e-3 * rms(y_ref), the q4 decode tests' bound. Shapes: the
model's fused q | gate, k, v projections and its o projection at the 1600-token chunk, row and
column tails (tokens not a multiple of 256, outputs not a multiple of 256), one token, in_dim
64, and one to four weights per call."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bf(a):
    return (a.astype(np.uint32) << 16).view(np.float32)


def _close(got_u16, ref64):
    got = _bf(got_u16).astype(np.float64)
    tol = np.abs(ref64) * 2 ** -7 + 1e-3 * np.sqrt((ref64 ** 2).mean()) + 1e-30
    bad = np.abs(got - ref64) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} beyond tolerance, max {np.abs(got - ref64).max():.3e}"


def _run(cuda, oracle, T, in_dim, out_dims, seed, scale=1.0):
    import torch
    x = oracle.normal_bf16(T * in_dim, seed).reshape(T, in_dim)
    ws = [oracle.f32_to_bf16(_bf(oracle.normal_bf16(o * in_dim, seed + 1 + i)).reshape(o, in_dim) * scale)
          for i, o in enumerate(out_dims)]
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    wd = [torch.from_numpy(w.view(np.int16)).cuda() for w in ws]
    outs = [torch.full((T, o), -1, dtype=torch.int16, device="cuda") for o in out_dims]
    cuda.prefill_linear(xd, wd, outs)
    torch.cuda.synchronize()
    xf = _bf(x).astype(np.float64)
    for w, o in zip(ws, outs):
        _close(o.cpu().numpy().view(np.uint16), xf @ _bf(w).astype(np.float64).T)
    code, _ = cuda.device_error()
    assert code == 0


@pytest.mark.parametrize("T,in_dim,out_dims", [
    (1600, 4096, [8192, 1024, 1024]),   # the fused q | gate, k, v projections of a chunk
    (1600, 4096, [4096]),               # the o projection
    (1, 4096, [256]), (257, 1024, [520, 8]), (300, 64, [136, 264, 16, 2048]),
    (513, 2048, [1000]), (2048, 512, [768, 256])])
def test_prefill_linear_matches_float64(cuda, oracle, T, in_dim, out_dims):
    _run(cuda, oracle, T, in_dim, out_dims, seed=T + in_dim, scale=1.0 / 32)


def test_q4_prefill_path(cuda, oracle):
    """Dequantise on the GPU (bit-exact), then project: the reference's prefill path for a q4
    weight, against the float64 product with the oracle's dequantised weight."""
    import torch
    rng = np.random.default_rng(5)
    out_dim, in_dim, T = 1024, 4096, 700
    w = rng.integers(0, 2 ** 32, (out_dim, in_dim // 8), dtype=np.uint64).astype(np.uint32)
    sc = oracle.f32_to_bf16((rng.random((out_dim, in_dim // 64)) * 0.02 + 0.001).astype(np.float32))
    bi = oracle.f32_to_bf16((rng.standard_normal((out_dim, in_dim // 64)) * 0.05).astype(np.float32))
    x = oracle.normal_bf16(T * in_dim, 6).reshape(T, in_dim)
    dense = torch.empty((out_dim, in_dim), dtype=torch.int16, device="cuda")
    cuda.q4_dequantize(torch.from_numpy(w.view(np.int32)).cuda(), torch.from_numpy(sc.view(np.int16)).cuda(),
                       torch.from_numpy(bi.view(np.int16)).cuda(), dense)
    y = torch.empty((T, out_dim), dtype=torch.int16, device="cuda")
    cuda.prefill_linear(torch.from_numpy(x.view(np.int16)).cuda(), [dense], [y])
    torch.cuda.synchronize()
    wd = oracle.q4_dequantize(w, sc, bi)
    assert np.array_equal(dense.cpu().numpy().view(np.uint16), wd)
    _close(y.cpu().numpy().view(np.uint16), _bf(x).astype(np.float64) @ _bf(wd).astype(np.float64).T)


def test_prefill_linear_rejects_bad_shapes(cuda):
    import torch
    from peregrine_b200.capi import PgcError
    x = torch.zeros((4, 100), dtype=torch.int16, device="cuda")  # in_dim not a multiple of 64
    w = torch.zeros((8, 100), dtype=torch.int16, device="cuda")
    y = torch.zeros((4, 8), dtype=torch.int16, device="cuda")
    with pytest.raises(PgcError, match="INVALID"):
        cuda.prefill_linear(x, [w], [y])
    x = torch.zeros((4, 64), dtype=torch.int16, device="cuda")
    w = torch.zeros((12, 64), dtype=torch.int16, device="cuda")  # out_dim not a multiple of 8
    y = torch.zeros((4, 12), dtype=torch.int16, device="cuda")
    with pytest.raises(PgcError, match="INVALID"):
        cuda.prefill_linear(x, [w], [y])
