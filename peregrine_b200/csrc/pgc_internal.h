// pgc_internal.h — host-side launchers shared between the C-ABI layer (capi.cpp) and the
// kernel translation units. Arguments are validated by capi.cpp before these run.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

#include "../../include/peregrine_cuda.h"

namespace pgc {

struct DevErrorHost {
    int code;
    int pad;
    long long detail;
};

// Tensor map over one paged pool viewed as [num_pages * 4 * 16 rows][256] bf16, 64 x 16 boxes,
// 128-byte swizzle. Cached per (device, base pointer, num_pages).
int pool_tensor_map(const void *pool, int64_t num_pages, CUtensorMap *out);
int current_sm_count();
// Tensor map over a chunk's queries [tokens][16][256] bf16 viewed as (dim, head, token),
// 64 x 4 x 32 boxes, 128-byte swizzle. Cached per (device, pointer, tokens).
int q_tensor_map(const void *q, int tokens, CUtensorMap *out);
int tiled_map_2d(const void *ptr, int elem_bytes, int64_t inner, int64_t outer, int box_inner,
                 int box_outer, bool swizzle128, CUtensorMap *out);

// decode_attn.cu
struct DecodePlan {
    int pages_per_split;
    int max_splits;
    int prefetch_pre;    // L2 prefetch before the programmatic-launch wait, pages per CTA
    int prefetch_ahead;  // L2 prefetch distance past the ring, pages
};
DecodePlan decode_plan(int batch, int max_seq_len, int sm_count);
size_t decode_workspace_bytes(int batch, int num_queries, int max_seq_len, int sm_count);
// The decode append fused into the split kernel (pgc_decode_attn_append): the inputs of
// pgc_append_kv_rope in decode mode, token t = seq * num_queries + j.
struct DecodeAppend {
    const uint16_t *q_in = nullptr;  // [tokens][16][q_head_stride] bf16 (q, or q | gate)
    int q_head_stride = 0;
    const uint16_t *k_in = nullptr, *v_in = nullptr;  // [tokens][4][256]
    const uint16_t *q_norm_w = nullptr, *k_norm_w = nullptr;
    const float *rope = nullptr;  // [rope_max_pos][64] cos | sin
    int64_t rope_max_pos = 0;
    const int32_t *positions = nullptr;
    const int64_t *slots = nullptr;
    uint16_t *k_pages = nullptr, *v_pages = nullptr;
    int64_t num_pages = 0;
    // context-parallel shard: positions (RoPE) minus pos_offset give the token's index in this
    // rank's cache; 0 otherwise
    int64_t pos_offset = 0;
};
cudaError_t launch_decode(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                          int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                          const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                          float scale, const uint16_t *gate, uint16_t *out, float *partials_out,
                          void *workspace, int sm_count, cudaStream_t stream,
                          const DecodeAppend *app = nullptr, int64_t gate_stride = 256,
                          const void *k_pages = nullptr, const void *v_pages = nullptr);
cudaError_t launch_merge_partials(const float *partials, int64_t rows, int num_parts,
                                  int64_t part_stride, const uint16_t *gate, uint16_t *out,
                                  cudaStream_t stream);
cudaError_t decode_read_error(DevErrorHost *e, bool clear);
// context-parallel exchange buffer: [2][world][16][8][34] u64 epoch-tagged words
size_t cp_buffer_bytes(int world);
cudaError_t launch_cp_decode(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                             int64_t num_pages, const int32_t *block_table, int max_pages,
                             const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                             uint16_t *out, void *workspace, float *const *bufs, int world, int rank,
                             uint32_t epoch, int sm_count, cudaStream_t stream,
                             const void *k_pages = nullptr, const void *v_pages = nullptr,
                             const DecodeAppend *app = nullptr, int64_t gate_stride = 256);
int decode_static_scratch(void **ptr_out);

// kv_append.cu
cudaError_t launch_append(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                          uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                          const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                          const float *rope_table, int64_t rope_max_pos, const int32_t *positions,
                          const int64_t *slot_mapping, int64_t tokens, uint16_t *k_pages,
                          uint16_t *v_pages, int64_t num_pages, int mode, cudaStream_t stream);
cudaError_t append_read_error(DevErrorHost *e, bool clear);

// cache_copy.cu
cudaError_t launch_copy_rows(void *dst, const void *src, const int32_t *dst_rows,
                             const int32_t *src_rows, int64_t n_rows, int64_t row_bytes,
                             int64_t dst_pitch, int64_t src_pitch, cudaStream_t stream);
cudaError_t launch_kv_dense(bool restore, uint16_t *dense_k, uint16_t *dense_v,
                            int64_t dense_stride, int64_t dense_token, uint16_t *k_pages,
                            uint16_t *v_pages, int64_t num_pages, const int32_t *table,
                            int64_t n_table, int64_t page_token, int64_t count,
                            cudaStream_t stream);
cudaError_t launch_kv_copy_tokens(const uint16_t *sk, const uint16_t *sv, int64_t s_pages,
                                  const int32_t *s_table, int64_t s_n, int64_t s_tok,
                                  uint16_t *dk, uint16_t *dv, int64_t d_pages,
                                  const int32_t *d_table, int64_t d_n, int64_t d_tok,
                                  int64_t count, cudaStream_t stream);
cudaError_t launch_regions(const pgc_region *regions, int n, bool zero, const int32_t *accept,
                           int32_t *seq_lens, int seq_index, int reject_tokens,
                           cudaStream_t stream);
cudaError_t copy_read_error(DevErrorHost *e, bool clear);

// prefill_attn.cu
int prefill_nsplit(int prefix_len, int chunk_len, int sm_count);
size_t prefill_workspace_bytes(int prefix_len, int chunk_len, int sm_count);
cudaError_t launch_prefill(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                           const uint16_t *v_pages, int64_t num_pages, const int32_t *block_table, int prefix_len,
                           int chunk_len, float scale, uint16_t *out, void *workspace,
                           int sm_count, cudaStream_t stream);
cudaError_t prefill_read_error(DevErrorHost *e, bool clear);

// linear_attn.cu
size_t gated_delta_prefill_workspace_bytes(int tokens);
cudaError_t launch_conv1d_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                                 const uint16_t *x, const uint16_t *w, uint16_t *out,
                                 cudaStream_t stream);
cudaError_t launch_conv1d_prefill(float *state, int has_state, const uint16_t *x, int T,
                                  const uint16_t *w, uint16_t *out, cudaStream_t stream);
cudaError_t launch_gated_delta_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                                      int has_state, const uint16_t *conv_out, const uint16_t *a,
                                      const uint16_t *b, const float *a_log, const uint16_t *dt_bias,
                                      uint16_t *y, cudaStream_t stream);
cudaError_t launch_gated_delta_prefill(float *state, int has_state, const uint16_t *conv_out,
                                       const uint16_t *a, const uint16_t *b, const float *a_log,
                                       const uint16_t *dt_bias, int T, uint16_t *y, void *ws,
                                       cudaStream_t stream);
cudaError_t linear_read_error(DevErrorHost *e, bool clear);

// q4_linear.cu
cudaError_t launch_q4_dequantize(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                                 uint16_t *out, int out_dim, int in_dim, cudaStream_t stream);
// Token rows per q4 projection tile (the MMA's N): 16, 32 or 64.
inline int q4_token_tile(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : 64; }
cudaError_t launch_q4_linear(const CUtensorMap &tx, const CUtensorMap &tw, int T, const uint16_t *scales,
                             const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                             cudaStream_t stream);
// 1-2 tokens: the CUDA-core stream over the packed words (q4_gemv_kernel); from 3 tokens on
// the tcgen05 kernel is faster.
constexpr int kQ4GemvMaxTokens = 2;
struct Q4Weight {
    const uint32_t *w;
    const uint16_t *scales, *biases;
    uint16_t *y;
    int out_dim;
};
// n (<= PGC_LINEAR_MAX_WEIGHTS) weights that share x, one launch
cudaError_t launch_q4_gemv(const uint16_t *x, int T, const Q4Weight *ws, int n, int in_dim, cudaStream_t stream);
cudaError_t q4_read_error(DevErrorHost *e, bool clear);

// prefill_linear.cu
struct LinearOut {
    uint16_t *y;
    int out_dim;
};
// x: [T][in_dim] bf16 (64 x 128 boxes, 128-byte swizzle); tw[i]: weight i [out_dim][in_dim]
// (same boxes). in_dim % 64 == 0, out_dim % 8 == 0.
cudaError_t launch_prefill_linear(const CUtensorMap &tx, const CUtensorMap *tw, const LinearOut *outs,
                                  int n_weights, int T, int in_dim, int sm_count, cudaStream_t stream);
cudaError_t prefill_linear_read_error(DevErrorHost *e, bool clear);

}  // namespace pgc
