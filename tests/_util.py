"""Shared helpers for the GPU parity tests: numpy (uint16 bf16 bits) <-> torch device tensors,
and the attention tolerance max-abs 2e-2 / rel 1e-2 against the fp32-accumulated oracle."""
import numpy as np

D, NQ, NKV, PAGE = 256, 16, 4, 16
ATOL, RTOL = 2e-2, 1e-2


def dev(a: np.ndarray):
    import torch
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host_u16(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def bf(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def assert_attn_close(got_bf16: np.ndarray, ref_f32: np.ndarray):
    g = bf(got_bf16)
    err = np.abs(g - ref_f32)
    bad = err > ATOL + RTOL * np.abs(ref_f32)
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, max abs err {err.max():.3e}"
    assert np.isfinite(g).all()
    return float(err.max())


def paged_pools(rng, logical_k, logical_v, num_pages, tables_out=None):
    """Scatter per-sequence logical K/V [L][4][256] into pools under a random page permutation.
    Returns (k_pool, v_pool, block_tables [B][max_pages])."""
    B = len(logical_k)
    pages = [(k.shape[0] + PAGE - 1) // PAGE for k in logical_k]
    assert sum(pages) <= num_pages
    perm = rng.permutation(num_pages).astype(np.int32)
    maxp = max(pages)
    table = np.zeros((B, maxp), np.int32)
    kp = np.zeros((num_pages, NKV, PAGE, D), np.uint16)
    vp = np.zeros_like(kp)
    o = 0
    for b in range(B):
        table[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
        L = logical_k[b].shape[0]
        full = L // PAGE * PAGE
        idx = table[b, :L // PAGE]
        kp[idx] = logical_k[b][:full].reshape(-1, PAGE, NKV, D).transpose(0, 2, 1, 3)
        vp[idx] = logical_v[b][:full].reshape(-1, PAGE, NKV, D).transpose(0, 2, 1, 3)
        for t in range(full, L):
            kp[table[b, t // PAGE], :, t % PAGE] = logical_k[b][t]
            vp[table[b, t // PAGE], :, t % PAGE] = logical_v[b][t]
    return kp, vp, table
