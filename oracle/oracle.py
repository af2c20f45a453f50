"""ctypes binding of the CPU ORACLE (oracle/pgo_oracle.c) — TEST INFRASTRUCTURE ONLY.

Used as the parity checker by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs. Never imported by the product (peregrine_b200). Parity status is stated
in pgo_oracle.h: copy semantics pinned by the reference's own tests, attention/append values
parity-unpinned (no numeric golden vectors exist in the reference).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libpgo_oracle.so"

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F32 = C.c_float
F64 = C.c_double
SZ = C.c_size_t

_SIG = {
    "pgo_bf16_to_f32": (F32, [C.c_uint16]),
    "pgo_f32_to_bf16": (C.c_uint16, [F32]),
    "pgo_f32_to_bf16_array": (None, [P, P, SZ]),
    "pgo_bf16_to_f32_array": (None, [P, P, SZ]),
    "pgo_fill_normal_bf16": (None, [P, SZ, U64, U64]),
    "pgo_set_threads": (None, [I32]),
    "pgo_get_threads": (I32, []),
    "pgo_full_cache_stride_for_max_seq": (I32, [U64, C.POINTER(U64)]),
    "pgo_rope_table": (None, [P, I64, I32, F64]),
    "pgo_append_kv_rope": (I32, [P, I32, P, P, P, P, P, P, P, I64, P, P, I64, P, P, I64, I32]),
    "pgo_decode_paged": (I32, [P, P, P, I64, P, I32, P, I32, I32, F32, P, P, P]),
    "pgo_decode_partials_paged": (I32, [P, P, P, I64, P, I32, P, I32, I32, F32, P]),
    "pgo_decode_dense_prefix": (I32, [P, P, P, P, P, I32, I32, F32, I32, I32, P, P]),
    "pgo_merge_partials": (I32, [P, I64, I32, I64, P, P, P]),
    "pgo_prefill_paged": (I32, [P, P, P, I64, P, I32, I32, F32, P, P]),
    "pgo_copy_full_attention_range": (None, [P, P, I64, I64, P, P, I64, I64, I64]),
    "pgo_kv_restore_dense": (I32, [P, P, I64, I64, P, P, I64, P, I64, I64, I64]),
    "pgo_kv_snapshot_dense": (I32, [P, P, I64, P, I64, I64, P, P, I64, I64, I64]),
    "pgo_kv_copy_tokens": (I32, [P, P, I64, P, I64, I64, P, P, I64, P, I64, I64, I64]),
    "pgo_copy_rows": (None, [P, P, P, P, I64, I64, I64, I64]),
    "pgo_rollback": (None, [P, P, I32, I32, P, P, P, I32]),
    "pgo_conv1d_decode": (None, [P, P, P, P, I32, I32]),
    "pgo_conv1d_prefill": (None, [P, I32, P, I32, P, P, I32, I32]),
    "pgo_gated_delta_decode": (None, [P, I32, P, P, P, P, P, P]),
    "pgo_gated_delta_prefill": (None, [P, I32, P, P, P, P, P, I32, P]),
    "pgo_q4_dequantize": (None, [P, P, P, P, I32, I32]),
    "pgo_q4_linear": (None, [P, P, P, P, P, I32, I32, I32]),
}

_lib = None


def build() -> Path:
    newest = max((HERE / f).stat().st_mtime for f in ("pgo_oracle.c", "pgo_linear.c", "pgo_oracle.h"))
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < newest:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIG.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def _p(a):
    if a is None:
        return None
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"], "oracle wants C-contiguous numpy"
    return a.ctypes.data


def set_threads(n: int) -> None:
    lib().pgo_set_threads(n)


def normal_bf16(n: int, seed: int, first_index: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().pgo_fill_normal_bf16(_p(out), n, seed, first_index)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().pgo_f32_to_bf16_array(_p(a), _p(out), a.size)
    return out


def full_cache_stride_for_max_seq(max_seq: int) -> int | None:
    out = U64(0)
    rc = lib().pgo_full_cache_stride_for_max_seq(max_seq, C.byref(out))
    return None if rc != 0 else out.value


def rope_table(max_pos: int, rot_dim: int = 64, theta: float = 1e7) -> np.ndarray:
    t = np.empty((max_pos, rot_dim), dtype=np.float32)
    lib().pgo_rope_table(_p(t), max_pos, rot_dim, theta)
    return t


def append_kv_rope(q_in, k_in, v_in, rope, positions, slots, k_pages, v_pages, mode,
                   q_norm_w=None, k_norm_w=None, want_gate=False):
    tokens = positions.shape[0]
    q_out = np.zeros((tokens, 16, 256), dtype=np.uint16)
    gate = np.zeros((tokens, 16, 256), dtype=np.uint16) if want_gate else None
    rc = lib().pgo_append_kv_rope(_p(q_in), q_in.shape[-1], _p(q_out), _p(gate), _p(k_in), _p(v_in),
                                  _p(q_norm_w), _p(k_norm_w), _p(rope), rope.shape[0], _p(positions),
                                  _p(slots), tokens, _p(k_pages), _p(v_pages), k_pages.shape[0], mode)
    assert rc == 0, rc
    return q_out, gate


def decode_paged(q, k_pages, v_pages, block_tables, seq_lens, scale, num_queries=1, gate=None):
    batch = seq_lens.shape[0]
    out = np.zeros((batch, num_queries, 16, 256), dtype=np.float32)
    outb = np.zeros((batch, num_queries, 16, 256), dtype=np.uint16)
    rc = lib().pgo_decode_paged(_p(q), _p(k_pages), _p(v_pages), k_pages.shape[0],
                                _p(block_tables), block_tables.shape[1], _p(seq_lens), batch,
                                num_queries, scale, _p(gate), _p(out), _p(outb))
    assert rc == 0, rc
    return out, outb


def decode_partials_paged(q, k_pages, v_pages, block_tables, seq_lens, scale, num_queries=1):
    batch = seq_lens.shape[0]
    parts = np.zeros((batch, num_queries * 16, 258), dtype=np.float32)
    rc = lib().pgo_decode_partials_paged(_p(q), _p(k_pages), _p(v_pages), k_pages.shape[0],
                                         _p(block_tables), block_tables.shape[1], _p(seq_lens),
                                         batch, num_queries, scale, _p(parts))
    assert rc == 0, rc
    return parts


def decode_dense_prefix(q, pk, pv, lk, lv, seq_len, prefix_len, scale, prefix_stride, local_stride,
                        gate=None):
    out = np.zeros((16, 256), dtype=np.float32)
    rc = lib().pgo_decode_dense_prefix(_p(q), _p(pk), _p(pv), _p(lk), _p(lv), seq_len, prefix_len,
                                       scale, prefix_stride, local_stride, _p(gate), _p(out))
    assert rc == 0, rc
    return out


def merge_partials(parts, rows, num_parts, part_stride, gate=None):
    out = np.zeros((rows, 256), dtype=np.float32)
    outb = np.zeros((rows, 256), dtype=np.uint16)
    lib().pgo_merge_partials(_p(parts), rows, num_parts, part_stride, _p(gate), _p(out), _p(outb))
    return out, outb


def prefill_paged(q, k_pages, v_pages, block_table, prefix_len, chunk_len, scale):
    out = np.zeros((chunk_len, 16, 256), dtype=np.float32)
    outb = np.zeros((chunk_len, 16, 256), dtype=np.uint16)
    rc = lib().pgo_prefill_paged(_p(q), _p(k_pages), _p(v_pages), k_pages.shape[0], _p(block_table),
                                 prefix_len, chunk_len, scale, _p(out), _p(outb))
    assert rc == 0, rc
    return out, outb


def copy_full_attention_range(dst_k, dst_v, dst_stride, dst_token, src_k, src_v, src_stride,
                              src_token, count):
    lib().pgo_copy_full_attention_range(_p(dst_k), _p(dst_v), dst_stride, dst_token, _p(src_k),
                                        _p(src_v), src_stride, src_token, count)


def kv_restore_dense(k_dense, v_dense, src_stride, src_token, k_pages, v_pages, table, dst_token,
                     count):
    return lib().pgo_kv_restore_dense(_p(k_dense), _p(v_dense), src_stride, src_token, _p(k_pages),
                                      _p(v_pages), k_pages.shape[0], _p(table), table.shape[-1],
                                      dst_token, count)


def kv_snapshot_dense(k_pages, v_pages, table, src_token, k_dense, v_dense, dst_stride, dst_token,
                      count):
    return lib().pgo_kv_snapshot_dense(_p(k_pages), _p(v_pages), k_pages.shape[0], _p(table),
                                       table.shape[-1], src_token, _p(k_dense), _p(v_dense),
                                       dst_stride, dst_token, count)


def kv_copy_tokens(sk, sv, st, s_tok, dk, dv, dt, d_tok, count):
    return lib().pgo_kv_copy_tokens(_p(sk), _p(sv), sk.shape[0], _p(st), st.shape[-1], s_tok,
                                    _p(dk), _p(dv), dk.shape[0], _p(dt), dt.shape[-1], d_tok, count)


def copy_rows(dst, src, n_rows, row_bytes, dst_pitch, src_pitch, dst_rows=None, src_rows=None):
    lib().pgo_copy_rows(_p(dst), _p(src), _p(dst_rows), _p(src_rows), n_rows, row_bytes, dst_pitch,
                        src_pitch)


def rollback(accept, seq_lens, seq_index, reject_tokens, pairs):
    n = len(pairs)
    dsts = (C.c_void_p * max(1, n))(*[_p(d) for d, _ in pairs])
    srcs = (C.c_void_p * max(1, n))(*[_p(s) for _, s in pairs])
    nbytes = (C.c_uint64 * max(1, n))(*[d.nbytes for d, _ in pairs])
    lib().pgo_rollback(_p(accept), _p(seq_lens), seq_index, reject_tokens, dsts, srcs, nbytes, n)


# ------------------------------------------------------------------ linear attention (pgo_linear.c)
LIN_CONV, LIN_K, LIN_HV, LIN_DV, LIN_DK = 8192, 4, 32, 128, 128


def conv1d_decode(state, x, w):
    """state f32 [3][8192] (updated in place), x bf16 [8192], w bf16 [8192][4] -> out bf16."""
    out = np.empty(LIN_CONV, np.uint16)
    lib().pgo_conv1d_decode(_p(state), _p(x), _p(w), _p(out), LIN_CONV, LIN_K)
    return out


def conv1d_prefill(state, has_state, x, w):
    """x bf16 [T][8192] -> out bf16 [T][8192]; state published in place."""
    T = x.shape[0]
    out = np.empty((T, LIN_CONV), np.uint16)
    lib().pgo_conv1d_prefill(_p(state), int(has_state), _p(x), T, _p(w), _p(out), LIN_CONV, LIN_K)
    return out


def gated_delta_decode(state, has_state, conv_out, a, b, a_log, dt_bias):
    """state f32 [32][128][128] in place; returns y bf16 [4096]."""
    y = np.empty(LIN_HV * LIN_DV, np.uint16)
    lib().pgo_gated_delta_decode(_p(state), int(has_state), _p(conv_out), _p(a), _p(b), _p(a_log),
                                 _p(dt_bias), _p(y))
    return y


def gated_delta_prefill(state, has_state, conv_out, a, b, a_log, dt_bias):
    """conv_out bf16 [T][8192], a/b bf16 [T][32]; returns y bf16 [T][4096]."""
    T = conv_out.shape[0]
    y = np.empty((T, LIN_HV * LIN_DV), np.uint16)
    lib().pgo_gated_delta_prefill(_p(state), int(has_state), _p(conv_out), _p(a), _p(b), _p(a_log),
                                  _p(dt_bias), T, _p(y))
    return y


# ------------------------------------------------------------------ q4 projections (pgo_linear.c)
def q4_dequantize(w, scales, biases):
    """w u32 [out][in/8], scales/biases bf16 [out][in/64] -> bf16 [out][in]."""
    out_dim, in_dim = w.shape[0], w.shape[1] * 8
    out = np.empty((out_dim, in_dim), np.uint16)
    lib().pgo_q4_dequantize(_p(w), _p(scales), _p(biases), _p(out), out_dim, in_dim)
    return out


def q4_linear(x, w, scales, biases):
    """x bf16 [T][in] -> y bf16 [T][out]."""
    T, out_dim, in_dim = x.shape[0], w.shape[0], w.shape[1] * 8
    y = np.empty((T, out_dim), np.uint16)
    lib().pgo_q4_linear(_p(x), _p(w), _p(scales), _p(biases), _p(y), T, out_dim, in_dim)
    return y

