"""ctypes binding of libperegrine_cuda.so (the C ABI in include/peregrine_cuda.h).

This module only loads the native library and forwards raw pointers; it holds no compute of
its own. Loading fails loudly when the library has not been built: there is no Python or CPU
fallback for any operation.

The thin tensor helpers at the bottom accept torch CUDA tensors (torch is used only as the
device-memory allocator and stream source) and raise PgcError on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libperegrine_cuda.so"

HEAD_DIM = 256
NUM_Q_HEADS = 16
NUM_KV_HEADS = 4
GQA_GROUP = 4
ROTARY_DIM = 64
PAGE_TOKENS = 16
HIDDEN = 4096
MAX_CONTEXT_TOKENS = 65536
PARTIAL_FLOATS = HEAD_DIM + 2
MAX_QUERIES = 4
MAX_REGIONS = 128
APPEND_DECODE = 0
APPEND_PREFILL = 1

STATUS = {
    0: "PGC_OK", -1: "PGC_ERR_INVALID", -2: "PGC_ERR_BOUNDS", -3: "PGC_ERR_WORKSPACE",
    -4: "PGC_ERR_CUDA", -5: "PGC_ERR_ALIGN", -6: "PGC_ERR_DEVICE", -7: "PGC_ERR_TIMEOUT",
    -8: "PGC_ERR_CONTEXT", -9: "PGC_ERR_FILE", -10: "PGC_ERR_FORMAT", -11: "PGC_ERR_CAPACITY",
    -12: "PGC_ERR_NCCL",
}


STATUS_INVALID = -1


class PgcError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {STATUS.get(status, status)}")


class Region(C.Structure):
    _fields_ = [("dst", C.c_void_p), ("src", C.c_void_p), ("bytes", C.c_uint64)]


class PrefixLayout(C.Structure):
    _fields_ = [("token_count", C.c_uint64), ("tokens", C.c_uint64),
                ("conv", C.c_uint64 * 24), ("recur", C.c_uint64 * 24),
                ("k_runs", C.c_uint64 * 8), ("v_runs", C.c_uint64 * 8),
                ("hidden", C.c_uint64), ("total_bytes", C.c_uint64)]


class PrefixInfo(C.Structure):
    _fields_ = [("token_count", C.c_uint64), ("next_token", C.c_uint32),
                ("next_token_valid", C.c_uint32), ("hidden_valid", C.c_uint32),
                ("file_bytes", C.c_uint64)]


class Match(C.Structure):
    _fields_ = [("index", C.c_int64), ("len", C.c_int64)]

    def __eq__(self, other):
        return isinstance(other, Match) and (self.index, self.len) == (other.index, other.len)

    def __repr__(self):
        return f"Match(index={self.index}, len={self.len})"


class PrefixStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "hits", "misses", "hit_tokens", "computed_tokens", "reserved_tokens", "resident_tokens",
        "max_tokens", "entry_count", "pinned_count", "evictions", "trie_nodes")] + [
        ("active_index", C.c_int64)]


class PrefixEntry(C.Structure):
    _fields_ = [("token_count", C.c_uint64), ("page_count", C.c_int64), ("capacity", C.c_uint64),
                ("state_slot", C.c_int32), ("pinned", C.c_int32), ("hidden_valid", C.c_int32),
                ("next_token_valid", C.c_int32), ("next_token", C.c_uint32),
                ("last_access", C.c_uint64), ("hits", C.c_uint64)]


P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F32 = C.c_float
F64 = C.c_double
SZ = C.c_size_t

SIGNATURES = {
    "pgc_status_string": (C.c_char_p, [I32]),
    "pgc_version": (I32, []),
    "pgc_device_error": (I32, [C.POINTER(I32), C.POINTER(I64), I32]),
    "pgc_full_cache_stride_for_max_seq": (I32, [U64, C.POINTER(U64)]),
    "pgc_rope_table_fill": (I32, [P, I64, I32, F64]),
    "pgc_append_kv_rope": (I32, [P, I32, P, P, P, P, P, P, P, I64, P, P, I64, P, P, I64, I32, P]),
    "pgc_decode_workspace_bytes": (SZ, [I32, I32, I32]),
    "pgc_decode_attn": (I32, [P, P, P, I64, P, I32, P, I32, I32, I32, F32, P, P, P, SZ, P]),
    "pgc_decode_attn_static": (I32, [P, P, P, I64, P, I32, P, I32, I32, I32, F32, P, P, P]),
    "pgc_decode_attn_append": (I32, [P, I32, P, P, P, P, P, I64, P, P, P, P, I64, P, I32, P, I32, I32, I32,
                                     F32, P, P, SZ, P]),
    "pgc_decode_attn_partials": (I32, [P, P, P, I64, P, I32, P, I32, I32, I32, F32, P, P, SZ, P]),
    "pgc_merge_partials": (I32, [P, I64, I32, I64, P, P, P]),
    "pgc_prefill_workspace_bytes": (SZ, [I32, I32]),
    "pgc_prefill_attn": (I32, [P, P, P, I64, P, I32, I32, F32, P, P, SZ, P]),
    "pgc_copy_rows": (I32, [P, P, P, P, I64, I64, I64, I64, P]),
    "pgc_kv_restore_dense": (I32, [P, P, I64, I64, P, P, I64, P, I64, I64, I64, P]),
    "pgc_kv_snapshot_dense": (I32, [P, P, I64, P, I64, I64, P, P, I64, I64, I64, P]),
    "pgc_kv_copy_tokens": (I32, [P, P, I64, P, I64, I64, P, P, I64, P, I64, I64, I64, P]),
    "pgc_copy_regions": (I32, [C.POINTER(Region), I32, P]),
    "pgc_zero_regions": (I32, [C.POINTER(Region), I32, P]),
    "pgc_rollback": (I32, [P, P, I32, I32, C.POINTER(Region), I32, P]),
    "pgc_prefix_file_layout": (I32, [U64, C.POINTER(PrefixLayout)]),
    "pgc_prefix_file_inspect": (I32, [C.c_char_p, U64, U64, U64, C.POINTER(PrefixInfo)]),
    "pgc_prefix_file_read": (I32, [C.c_char_p, U64, U64, U64, P, U64, C.POINTER(PrefixInfo)]),
    "pgc_prefix_file_header": (I32, [P, U64, U64, U64, C.c_uint32, I32, I32]),
    "pgc_prefix_file_write": (I32, [C.c_char_p, P, U64]),
    "pgc_conv1d_decode": (I32, [P, I64, P, I32, P, P, P, P]),
    "pgc_conv1d_prefill": (I32, [P, I32, P, I32, P, P, P]),
    "pgc_gated_delta_decode": (I32, [P, I64, P, I32, I32, P, P, P, P, P, P, P]),
    "pgc_gated_delta_prefill_workspace_bytes": (SZ, [I32]),
    "pgc_gated_delta_prefill": (I32, [P, I32, P, P, P, P, P, I32, P, P, SZ, P]),
    "pgc_cp_buffer_bytes": (SZ, [I32]),
    "pgc_cp_buffer_alloc": (I32, [I32, C.POINTER(P)]),
    "pgc_cp_buffer_free": (I32, [P]),
    "pgc_ipc_get_handle": (I32, [P, P]),
    "pgc_ipc_open_handle": (I32, [P, C.POINTER(P)]),
    "pgc_ipc_close": (I32, [P]),
    "pgc_cp_decode_attn": (I32, [P, P, P, I64, P, I32, P, I32, F32, P, P, P, SZ, C.POINTER(P), I32, I32,
                                 C.c_uint32, P]),
    "pgc_q4_dequantize": (I32, [P, P, P, P, I32, I32, P]),
    "pgc_q4_linear": (I32, [P, I32, P, P, P, P, I32, I32, P]),
    "pgc_prefill_linear": (I32, [P, I32, I32, I32, P, P, P, P]),
    "pgc_q4_linear_multi": (I32, [P, I32, I32, I32, P, P, P, P, P, P]),
    "pgc_nccl_get_unique_id": (I32, [P]),
    "pgc_nccl_comm_init": (I32, [I32, I32, P, P]),
    "pgc_nccl_comm_destroy": (I32, [P]),
    "pgc_cp_decode_attn_nccl": (I32, [P, P, P, I64, P, I32, P, I32, F32, P, P, P, P, SZ, P, P]),
    "pgc_cp_decode_attn_append": (I32, [P, I32, P, P, P, P, P, I64, P, P, I64, P, P, I64, P, I32, P, I32, F32,
                                        P, P, SZ, C.POINTER(P), I32, I32, C.c_uint32, P]),
    "pgc_page_pool_create": (P, [I32]),
    "pgc_page_pool_destroy": (None, [P]),
    "pgc_page_pool_alloc": (I32, [P, I32, P]),
    "pgc_page_pool_retain": (I32, [P, P, I32]),
    "pgc_page_pool_release": (I32, [P, P, I32]),
    "pgc_page_pool_refcount": (I32, [P, I32]),
    "pgc_page_pool_free_pages": (I32, [P]),
    "pgc_page_pool_make_writable": (I32, [P, P, I32, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "pgc_prefix_cache_create": (P, [P, I32, U64, U64, I32]),
    "pgc_prefix_cache_destroy": (None, [P]),
    "pgc_prefix_cache_clear_all": (None, [P]),
    "pgc_prefix_cache_enable_hidden_tracking": (None, [P]),
    "pgc_prefix_cache_find": (I32, [P, P, U64, C.POINTER(Match)]),
    "pgc_prefix_cache_contains": (I32, [P, P, U64, U64]),
    "pgc_prefix_cache_touch": (None, [P, Match]),
    "pgc_prefix_cache_record_hit": (None, [P, U64]),
    "pgc_prefix_cache_record_miss": (None, [P]),
    "pgc_prefix_cache_record_computed": (None, [P, U64]),
    "pgc_prefix_cache_stats": (I32, [P, C.POINTER(PrefixStats)]),
    "pgc_prefix_cache_entry": (I32, [P, I64, C.POINTER(PrefixEntry), P, U64, P, I64]),
    "pgc_prefix_cache_remove": (I32, [P, I64]),
    "pgc_prefix_cache_start_direct": (I32, [P, P, U64, I32, C.POINTER(Match)]),
    "pgc_prefix_cache_finish_direct": (I32, [P, Match, C.c_uint32]),
    "pgc_prefix_cache_set_hidden_valid": (I32, [P, Match, I32]),
    "pgc_prefix_cache_store": (I32, [P, P, U64, C.POINTER(Match), P, I64, I32,
                                     C.POINTER(C.c_uint32), I32, C.POINTER(Match),
                                     C.POINTER(C.c_int)]),
    "pgc_prefix_cache_fork": (I32, [P, Match, P, I64, C.POINTER(C.c_int64)]),
    "pgc_prefix_cache_evict_for_pages": (I32, [P, I32]),
    "pgc_prefix_cache_load_slot": (I32, [P, P, U64, C.POINTER(Match)]),
    "pgc_prefix_cache_finish_loaded": (I32, [P, Match]),
    "pgc_prefix_cache_persisted": (I32, [P, C.POINTER(Match)]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the native library (raises if it is missing: no fallback exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is not built; run `python -m peregrine_b200.build` "
                "(the CUDA library is the only implementation)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        raise PgcError(status, what)


# ----------------------------------------------------------------------------- host helpers

def full_cache_stride_for_max_seq(max_seq: int) -> int:
    out = U64(0)
    check(lib().pgc_full_cache_stride_for_max_seq(max_seq, C.byref(out)),
          "pgc_full_cache_stride_for_max_seq")
    return out.value


def rope_table(max_pos: int, rot_dim: int = ROTARY_DIM, theta: float = 1e7):
    import numpy as np
    t = np.empty((max_pos, rot_dim), dtype=np.float32)
    check(lib().pgc_rope_table_fill(t.ctypes.data, max_pos, rot_dim, theta), "pgc_rope_table_fill")
    return t


def device_error(clear: bool = True) -> tuple[int, int]:
    code, detail = I32(0), I64(0)
    check(lib().pgc_device_error(C.byref(code), C.byref(detail), int(clear)), "pgc_device_error")
    return code.value, detail.value


# ----------------------------------------------------------------------------- torch helpers

def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def decode_workspace_bytes(batch: int, num_queries: int, max_seq_len: int) -> int:
    return int(lib().pgc_decode_workspace_bytes(batch, num_queries, max_seq_len))


def decode_attn(q, k_pages, v_pages, block_tables, seq_lens, max_seq_len, scale, out,
                workspace, num_queries=1, gate=None, stream=None) -> None:
    batch = seq_lens.shape[0]
    check(lib().pgc_decode_attn(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], _ptr(block_tables),
        block_tables.shape[1], _ptr(seq_lens), batch, num_queries, max_seq_len, scale, _ptr(gate),
        _ptr(out), _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream)),
        "pgc_decode_attn")


def decode_attn_append(q_in, k_in, v_in, rope, positions, slots, k_pages, v_pages, block_tables,
                       seq_lens, max_seq_len, scale, out, workspace, num_queries=1, q_norm_w=None,
                       k_norm_w=None, stream=None) -> None:
    """pgc_decode_attn_append: the decode append (RMSNorm + RoPE, new K/V rows into the pool) and
    the attention in one launch. q_in [tokens][16][256 or 512 (q | gate)]."""
    batch = seq_lens.shape[0]
    check(lib().pgc_decode_attn_append(
        _ptr(q_in), q_in.shape[-1], _ptr(k_in), _ptr(v_in), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope),
        rope.shape[0], _ptr(positions), _ptr(slots), _ptr(k_pages), _ptr(v_pages), k_pages.shape[0],
        _ptr(block_tables), block_tables.shape[1], _ptr(seq_lens), batch, num_queries, max_seq_len,
        scale, _ptr(out), _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream)),
        "pgc_decode_attn_append")


def decode_attn_static(q, k_pages, v_pages, block_tables, seq_lens, max_seq_len, scale, out,
                       num_queries=1, gate=None, stream=None) -> None:
    """pgc_decode_attn_static: same attention, scratch in the library's fixed device array."""
    batch = seq_lens.shape[0]
    check(lib().pgc_decode_attn_static(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], _ptr(block_tables),
        block_tables.shape[1], _ptr(seq_lens), batch, num_queries, max_seq_len, scale, _ptr(gate),
        _ptr(out), _stream(stream)), "pgc_decode_attn_static")


def decode_attn_partials(q, k_pages, v_pages, block_tables, seq_lens, max_seq_len, scale,
                         partials, workspace, num_queries=1, stream=None) -> None:
    batch = seq_lens.shape[0]
    check(lib().pgc_decode_attn_partials(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], _ptr(block_tables),
        block_tables.shape[1], _ptr(seq_lens), batch, num_queries, max_seq_len, scale,
        _ptr(partials), _ptr(workspace), workspace.numel() * workspace.element_size(),
        _stream(stream)), "pgc_decode_attn_partials")


def merge_partials(partials, rows, num_parts, part_stride, out, gate=None, stream=None) -> None:
    check(lib().pgc_merge_partials(_ptr(partials), rows, num_parts, part_stride, _ptr(gate),
                                   _ptr(out), _stream(stream)), "pgc_merge_partials")


def append_kv_rope(q_in, q_out, k_in, v_in, rope, positions, slots, k_pages, v_pages,
                   mode=APPEND_DECODE, gate_out=None, q_norm_w=None, k_norm_w=None,
                   stream=None) -> None:
    tokens = positions.shape[0]
    q_head_stride = q_in.shape[-1]
    check(lib().pgc_append_kv_rope(
        _ptr(q_in), q_head_stride, _ptr(q_out), _ptr(gate_out), _ptr(k_in), _ptr(v_in),
        _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope), rope.shape[0], _ptr(positions), _ptr(slots),
        tokens, _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], mode, _stream(stream)),
        "pgc_append_kv_rope")


def prefill_workspace_bytes(prefix_len: int, chunk_len: int) -> int:
    return int(lib().pgc_prefill_workspace_bytes(prefix_len, chunk_len))


def prefill_attn(q, k_pages, v_pages, block_table, prefix_len, chunk_len, scale, out, workspace,
                 stream=None) -> None:
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().pgc_prefill_attn(
        _ptr(q), _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], _ptr(block_table), prefix_len,
        chunk_len, scale, _ptr(out), _ptr(workspace), ws_bytes, _stream(stream)),
        "pgc_prefill_attn")


def copy_rows(dst, src, n_rows, row_bytes, dst_pitch, src_pitch, dst_rows=None, src_rows=None,
              stream=None) -> None:
    d = dst if isinstance(dst, int) else dst.data_ptr()
    s = src if isinstance(src, int) else src.data_ptr()
    check(lib().pgc_copy_rows(d, s, _ptr(dst_rows), _ptr(src_rows), n_rows, row_bytes, dst_pitch,
                              src_pitch, _stream(stream)), "pgc_copy_rows")


def kv_restore_dense(k_dense, v_dense, src_stride, src_token, k_pages, v_pages, block_table,
                     dst_token, count, stream=None) -> None:
    check(lib().pgc_kv_restore_dense(
        _ptr(k_dense), _ptr(v_dense), src_stride, src_token, _ptr(k_pages), _ptr(v_pages),
        k_pages.shape[0], _ptr(block_table), block_table.shape[-1], dst_token, count,
        _stream(stream)), "pgc_kv_restore_dense")


def kv_snapshot_dense(k_pages, v_pages, block_table, src_token, k_dense, v_dense, dst_stride,
                      dst_token, count, stream=None) -> None:
    check(lib().pgc_kv_snapshot_dense(
        _ptr(k_pages), _ptr(v_pages), k_pages.shape[0], _ptr(block_table),
        block_table.shape[-1], src_token, _ptr(k_dense), _ptr(v_dense), dst_stride, dst_token,
        count, _stream(stream)), "pgc_kv_snapshot_dense")


def kv_copy_tokens(src_k, src_v, src_table, src_token, dst_k, dst_v, dst_table, dst_token, count,
                   stream=None) -> None:
    check(lib().pgc_kv_copy_tokens(
        _ptr(src_k), _ptr(src_v), src_k.shape[0], _ptr(src_table), src_table.shape[-1],
        src_token, _ptr(dst_k), _ptr(dst_v), dst_k.shape[0], _ptr(dst_table),
        dst_table.shape[-1], dst_token, count, _stream(stream)), "pgc_kv_copy_tokens")


def _regions(pairs):
    arr = (Region * max(1, len(pairs)))()
    for i, (dst, src, nbytes) in enumerate(pairs):
        arr[i].dst = dst if isinstance(dst, int) else dst.data_ptr()
        arr[i].src = (src if isinstance(src, int) else src.data_ptr()) if src is not None else None
        arr[i].bytes = nbytes
    return arr


def copy_regions(pairs, stream=None) -> None:
    """pairs: [(dst, src, nbytes)] with tensors or raw addresses."""
    check(lib().pgc_copy_regions(_regions(pairs), len(pairs), _stream(stream)), "pgc_copy_regions")


def zero_regions(pairs, stream=None) -> None:
    check(lib().pgc_zero_regions(_regions([(d, None, n) for d, n in pairs]), len(pairs),
                                 _stream(stream)), "pgc_zero_regions")


def rollback(accept, seq_lens, seq_index, reject_tokens, pairs, stream=None) -> None:
    check(lib().pgc_rollback(_ptr(accept), _ptr(seq_lens), seq_index, reject_tokens,
                             _regions(pairs), len(pairs), _stream(stream)), "pgc_rollback")


# ----------------------------------------------------------------------------- prefix-state file

def prefix_file_layout(token_count: int) -> PrefixLayout:
    lay = PrefixLayout()
    check(lib().pgc_prefix_file_layout(token_count, C.byref(lay)), "pgc_prefix_file_layout")
    return lay


def prefix_file_inspect(path, fingerprint: int, vocab: int, max_tokens: int) -> PrefixInfo:
    info = PrefixInfo()
    check(lib().pgc_prefix_file_inspect(str(path).encode(), fingerprint, vocab, max_tokens,
                                        C.byref(info)), "pgc_prefix_file_inspect")
    return info


def prefix_file_read(path, fingerprint: int, vocab: int, max_tokens: int, image_ptr: int,
                     image_bytes: int) -> PrefixInfo:
    info = PrefixInfo()
    check(lib().pgc_prefix_file_read(str(path).encode(), fingerprint, vocab, max_tokens,
                                     image_ptr, image_bytes, C.byref(info)), "pgc_prefix_file_read")
    return info


def prefix_file_header(image_ptr: int, image_bytes: int, fingerprint: int, token_count: int,
                       next_token: int = 0, next_token_valid: bool = False,
                       hidden_valid: bool = False) -> None:
    check(lib().pgc_prefix_file_header(image_ptr, image_bytes, fingerprint, token_count,
                                       next_token, int(next_token_valid), int(hidden_valid)),
          "pgc_prefix_file_header")


def prefix_file_write(path, image_ptr: int, image_bytes: int) -> None:
    check(lib().pgc_prefix_file_write(str(path).encode(), image_ptr, image_bytes),
          "pgc_prefix_file_write")


# ----------------------------------------------------------------------------- linear attention
LIN_CONV_DIM = 8192
LIN_VALUE_HEADS = 32
LIN_HEAD_DIM = 128


def conv1d_decode(conv_states, x, weight, out, slots=None, stream=None) -> None:
    """conv_states f32 [num_slots][3][8192]; x/out [batch][8192] bf16; slots [batch] int32."""
    batch = x.shape[0]
    check(lib().pgc_conv1d_decode(_ptr(conv_states), conv_states.shape[0], _ptr(slots), batch,
                                  _ptr(x), _ptr(weight), _ptr(out), _stream(stream)),
          "pgc_conv1d_decode")


def conv1d_prefill(conv_state, has_previous_state, x, weight, out, stream=None) -> None:
    check(lib().pgc_conv1d_prefill(_ptr(conv_state), int(has_previous_state), _ptr(x), x.shape[0],
                                   _ptr(weight), _ptr(out), _stream(stream)), "pgc_conv1d_prefill")


def gated_delta_decode(states, has_previous_state, conv_out, a, b, a_log, dt_bias, y, slots=None,
                       stream=None) -> None:
    """states f32 [num_slots][32][128][128]; conv_out [batch][8192]; a/b [batch][32]; y
    [batch][4096]."""
    batch = conv_out.shape[0]
    check(lib().pgc_gated_delta_decode(_ptr(states), states.shape[0], _ptr(slots), batch,
                                       int(has_previous_state), _ptr(conv_out), _ptr(a), _ptr(b),
                                       _ptr(a_log), _ptr(dt_bias), _ptr(y), _stream(stream)),
          "pgc_gated_delta_decode")


def gated_delta_prefill_workspace_bytes(tokens: int) -> int:
    return lib().pgc_gated_delta_prefill_workspace_bytes(tokens)


def gated_delta_prefill(state, has_previous_state, conv_out, a, b, a_log, dt_bias, y, workspace,
                        stream=None) -> None:
    check(lib().pgc_gated_delta_prefill(_ptr(state), int(has_previous_state), _ptr(conv_out), _ptr(a),
                                        _ptr(b), _ptr(a_log), _ptr(dt_bias), conv_out.shape[0], _ptr(y),
                                        _ptr(workspace), workspace.numel() * workspace.element_size(),
                                        _stream(stream)), "pgc_gated_delta_prefill")


# ----------------------------------------------------------------------------- q4 projections
def q4_dequantize(weight, scales, biases, out, stream=None) -> None:
    """weight int32/uint32 [out][in/8], scales/biases bf16 [out][in/64] -> out bf16 [out][in]."""
    check(lib().pgc_q4_dequantize(_ptr(weight), _ptr(scales), _ptr(biases), _ptr(out), out.shape[0],
                                  out.shape[1], _stream(stream)), "pgc_q4_dequantize")


LINEAR_MAX_WEIGHTS = 4


def prefill_linear(x, weights, outs, stream=None) -> None:
    """pgc_prefill_linear: outs[i] = x @ weights[i]^T (bf16, fp32 accumulate) for the weights that
    share the input x [tokens][in]; weights[i] bf16 [out_i][in], outs[i] bf16 [tokens][out_i]."""
    n = len(weights)
    assert n == len(outs) and 1 <= n <= LINEAR_MAX_WEIGHTS
    wp = (C.c_void_p * n)(*[w.data_ptr() for w in weights])
    op = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    dims = (C.c_int * n)(*[int(w.shape[0]) for w in weights])
    check(lib().pgc_prefill_linear(_ptr(x), x.shape[0], x.shape[1], n, C.cast(wp, C.c_void_p),
                                   C.cast(dims, C.c_void_p), C.cast(op, C.c_void_p), _stream(stream)),
          "pgc_prefill_linear")


def q4_linear_multi(x, weights, scales, biases, ys, stream=None) -> None:
    """pgc_q4_linear_multi: ys[i] = x @ w_i^T for the q4 weights that share x [tokens][in]."""
    n = len(weights)
    assert n == len(scales) == len(biases) == len(ys) and 1 <= n <= LINEAR_MAX_WEIGHTS

    def arr(ts):
        return C.cast((C.c_void_p * n)(*[t.data_ptr() for t in ts]), C.c_void_p)

    dims = (C.c_int * n)(*[int(y.shape[1]) for y in ys])
    check(lib().pgc_q4_linear_multi(_ptr(x), x.shape[0], x.shape[1], n, arr(weights), arr(scales),
                                    arr(biases), arr(ys), C.cast(dims, C.c_void_p), _stream(stream)),
          "pgc_q4_linear_multi")


def q4_linear(x, weight, scales, biases, y, stream=None) -> None:
    """x bf16 [tokens][in] -> y bf16 [tokens][out]."""
    check(lib().pgc_q4_linear(_ptr(x), x.shape[0], _ptr(weight), _ptr(scales), _ptr(biases), _ptr(y),
                              y.shape[1], x.shape[1], _stream(stream)), "pgc_q4_linear")

