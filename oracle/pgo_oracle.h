/*
 * pgo_oracle.h — CPU ORACLE for the Peregrine KV / prefix-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a scalar C11 restatement of the reference's semantics
 * (XiaoConstantine/peregrine, Zig + Metal) used as the parity checker by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference legs. It is never
 * part of the product path: libperegrine_cuda.so does not link it and has no CPU fallback.
 *
 * Parity status:
 *   - layout rules (stride alignment) and byte-copy semantics: PINNED against the reference's
 *     own tests (src/model/state.zig:244-254 stride golden values; the byte-pattern fixtures of
 *     src/server/prefix_state_cache.zig:935-1164 and src/server/prefix_persist.zig:457-639),
 *     transcribed in tests/golden/.
 *   - attention, RoPE and append VALUES: PARITY UNPINNED. The reference holds no numeric golden
 *     vectors for them (its kernel comments cite off-tree MLX checks only) and its Metal/Zig
 *     code cannot be built or run on Linux (no zig, no Metal). The oracle restates the kernels'
 *     arithmetic, each function citing the file:line it follows.
 *
 * Conventions: bf16 values are uint16_t bit patterns; compiled with -ffp-contract=off so each
 * fp32 operation rounds exactly once, in source order.
 */
#ifndef PGO_ORACLE_H
#define PGO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* --- numerics helpers --- */
float pgo_bf16_to_f32(uint16_t b);
uint16_t pgo_f32_to_bf16(float f); /* round to nearest even, quiet NaN kept */
void pgo_f32_to_bf16_array(const float *src, uint16_t *dst, size_t n);
void pgo_bf16_to_f32_array(const uint16_t *src, float *dst, size_t n);
/* SplitMix64-seeded Box-Muller N(0,1) in double, rounded to fp32 then bf16. Element i of a
 * (seed) stream is a pure function of (seed, i), so any slice can be regenerated. */
void pgo_fill_normal_bf16(uint16_t *out, size_t n, uint64_t seed, uint64_t first_index);
void pgo_set_threads(int n);
int pgo_get_threads(void);

/* --- layout rules --- */
int pgo_full_cache_stride_for_max_seq(uint64_t max_seq, uint64_t *stride_out);
void pgo_rope_table(float *table, int64_t max_pos, int rot_dim, double theta);

/* --- A3/A4 append --- */
int pgo_append_kv_rope(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                       uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                       const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                       const float *rope_table, int64_t rope_max_pos,
                       const int32_t *positions, const int64_t *slot_mapping, int64_t tokens,
                       uint16_t *k_pages, uint16_t *v_pages, int64_t num_pages, int mode);

/* --- A1/A2 decode attention --- */
/* Paged: same arguments as pgc_decode_attn; fp32 result in out_f32 [batch][nq][16][256]
 * (un-rounded) and, if out_bf16 != NULL, the bf16 rounding. */
int pgo_decode_paged(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                     int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                     const int32_t *seq_lens, int batch, int num_queries, float scale,
                     const uint16_t *gate, float *out_f32, uint16_t *out_bf16);
/* Partials of one paged cache (the CP shard form): [batch][nq*16][258]. */
int pgo_decode_partials_paged(const uint16_t *q, const uint16_t *k_pages,
                              const uint16_t *v_pages, int64_t num_pages,
                              const int32_t *block_tables, int max_pages_per_seq,
                              const int32_t *seq_lens, int batch, int num_queries,
                              float scale, float *partials);
/* Dense two-source form of attention_decode.metal:24-243 (one sequence, one query):
 * K [4][stride][256], V [4][256][stride] for prefix (t < prefix_len) and local tokens. */
int pgo_decode_dense_prefix(const uint16_t *q, const uint16_t *prefix_k,
                            const uint16_t *prefix_v, const uint16_t *local_k,
                            const uint16_t *local_v, int seq_len, int prefix_len, float scale,
                            int prefix_stride, int local_stride, const uint16_t *gate,
                            float *out_f32);
int pgo_merge_partials(const float *partials, int64_t rows, int num_parts, int64_t part_stride,
                       const uint16_t *gate, float *out_f32, uint16_t *out_bf16);

/* --- A5 prefill attention --- */
int pgo_prefill_paged(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                      int64_t num_pages, const int32_t *block_table, int prefix_len,
                      int chunk_len, float scale, float *out_f32, uint16_t *out_bf16);

/* --- A6-A9, A11 copies --- */
void pgo_copy_full_attention_range(uint16_t *dst_k, uint16_t *dst_v, int64_t dst_stride,
                                   int64_t dst_token, const uint16_t *src_k,
                                   const uint16_t *src_v, int64_t src_stride,
                                   int64_t src_token, int64_t count);
int pgo_kv_restore_dense(const uint16_t *k_dense, const uint16_t *v_dense, int64_t src_stride,
                         int64_t src_token, uint16_t *k_pages, uint16_t *v_pages,
                         int64_t num_pages, const int32_t *block_table, int64_t n_table,
                         int64_t dst_token, int64_t count);
int pgo_kv_snapshot_dense(const uint16_t *k_pages, const uint16_t *v_pages, int64_t num_pages,
                          const int32_t *block_table, int64_t n_table, int64_t src_token,
                          uint16_t *k_dense, uint16_t *v_dense, int64_t dst_stride,
                          int64_t dst_token, int64_t count);
int pgo_kv_copy_tokens(const uint16_t *src_k, const uint16_t *src_v, int64_t src_num_pages,
                       const int32_t *src_table, int64_t src_n_table, int64_t src_token,
                       uint16_t *dst_k, uint16_t *dst_v, int64_t dst_num_pages,
                       const int32_t *dst_table, int64_t dst_n_table, int64_t dst_token,
                       int64_t count);
void pgo_copy_rows(void *dst, const void *src, const int32_t *dst_rows, const int32_t *src_rows,
                   int64_t n_rows, int64_t row_bytes, int64_t dst_pitch, int64_t src_pitch);

/* --- A10 rollback --- */
void pgo_rollback(const int32_t *accept, int32_t *seq_lens, int seq_index, int reject_tokens,
                  void *const *dsts, const void *const *srcs, const uint64_t *bytes, int n);

/* Linear attention (pgo_linear.c): conv1d + SiLU, gated delta-rule recurrence. Shapes fixed to
 * the model's (Hk 16, Hv 32, Dk = Dv = 128, conv_dim 8192). */
void pgo_conv1d_decode(float *state, const uint16_t *x, const uint16_t *w, uint16_t *out, int C,
                       int K);
void pgo_conv1d_prefill(float *state, int has_state, const uint16_t *x, int T, const uint16_t *w,
                        uint16_t *out, int C, int K);
void pgo_gated_delta_decode(float *state, int has_state, const uint16_t *conv_out, const uint16_t *a,
                            const uint16_t *b, const float *A_log, const uint16_t *dt_bias,
                            uint16_t *y);
void pgo_gated_delta_prefill(float *state, int has_state, const uint16_t *conv_out, const uint16_t *a,
                             const uint16_t *b, const float *A_log, const uint16_t *dt_bias, int T,
                             uint16_t *y);

/* q4 group-64 affine projections (pgo_linear.c). */
void pgo_q4_dequantize(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                       uint16_t *out, int out_dim, int in_dim);
void pgo_q4_linear(const uint16_t *x, const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                   uint16_t *y, int T, int out_dim, int in_dim);

#ifdef __cplusplus
}
#endif
#endif
