/*
 * pgo_oracle.c — CPU ORACLE (test infrastructure only; see pgo_oracle.h for the parity status).
 *
 * Scalar restatement of the reference's KV / prefix-cache semantics. Every function cites the
 * reference file:line (paths within XiaoConstantine/peregrine) whose arithmetic it follows.
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fopenmp -shared -fPIC (see oracle/Makefile).
 */
#include "pgo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define D 256
#define NQH 16
#define NKV 4
#define GRP 4
#define PAGE 16
#define ROT 64
#define PF (D + 2)

static int g_threads = 1;

void pgo_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int pgo_get_threads(void) { return g_threads; }

/* ---------------------------------------------------------------- numerics */

float pgo_bf16_to_f32(uint16_t b) {
    /* shaders/bf16.h:8-11: bf16 is the high half of an fp32. */
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t pgo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void pgo_f32_to_bf16_array(const float *src, uint16_t *dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = pgo_f32_to_bf16(src[i]);
}

void pgo_bf16_to_f32_array(const uint16_t *src, float *dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = pgo_bf16_to_f32(src[i]);
}

static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

static double u01(uint64_t bits) { return ((double)(bits >> 11) + 0.5) * (1.0 / 9007199254740992.0); }

void pgo_fill_normal_bf16(uint16_t *out, size_t n, uint64_t seed, uint64_t first_index) {
    /* Box-Muller over pairs: elements 2k and 2k+1 share one pair of uniforms. */
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static) if (n > (1u << 20)) num_threads(g_threads)
    for (size_t i = 0; i < n; i++) {
        uint64_t idx = first_index + i;
        uint64_t pair = idx >> 1;
        uint64_t base = splitmix64(seed ^ 0xD1B54A32D192ED03ull) + 2 * pair;
        double u1 = u01(splitmix64(base));
        double u2 = u01(splitmix64(base + 1));
        double r = sqrt(-2.0 * log(u1));
        double v = (idx & 1) ? r * sin(two_pi * u2) : r * cos(two_pi * u2);
        out[i] = pgo_f32_to_bf16((float)v);
    }
}

/* ---------------------------------------------------------------- layout rules */

int pgo_full_cache_stride_for_max_seq(uint64_t max_seq, uint64_t *stride_out) {
    /* src/model/state.zig:25-32 */
    if (max_seq == 0 || max_seq > 65536) return -8;
    uint64_t a = max_seq >= 16000 ? 64 : 256;
    uint64_t r = max_seq % a;
    *stride_out = r == 0 ? max_seq : max_seq + (a - r);
    return 0;
}

void pgo_rope_table(float *table, int64_t max_pos, int rot_dim, double theta) {
    /* inv_freq_i = theta^(-2i/rot), angle = pos * inv_freq_i (shaders/rope.metal:5-10,
     * attention.metal:391-396), evaluated in double and rounded once to fp32. */
    const int half = rot_dim / 2;
    for (int64_t p = 0; p < max_pos; p++) {
        for (int i = 0; i < half; i++) {
            double inv_freq = pow(theta, -(2.0 * (double)i) / (double)rot_dim);
            double ang = (double)p * inv_freq;
            table[p * rot_dim + i] = (float)cos(ang);
            table[p * rot_dim + half + i] = (float)sin(ang);
        }
    }
}

/* ---------------------------------------------------------------- A3/A4 append */

/* Sum of squares in the order of the reference's 256-thread tree reduction
 * (shaders/attention.metal:370-375 / :178-183): p[i] = x[i]^2, then p[i] += p[i + s] for
 * s = 128, 64, ..., 1; the result is p[0]. */
static float tree_sum_sq(const float *x) {
    float p[D];
    for (int i = 0; i < D; i++) p[i] = x[i] * x[i];
    for (int s = D / 2; s > 0; s >>= 1)
        for (int i = 0; i < s; i++) p[i] = p[i] + p[i + s];
    return p[0];
}

/* One head row: attention.metal:327-421 (mode 0) / :146-219 (mode 1). */
static void prepare_row(const uint16_t *src, const uint16_t *w, const float *cs, int mode,
                        uint16_t *dst) {
    float x[D];
    for (int d = 0; d < D; d++) x[d] = pgo_bf16_to_f32(src[d]);
    float y[D];
    if (w) {
        float ss = tree_sum_sq(x);
        float t = ss / 256.0f + 1e-6f;
        float inv = 1.0f / sqrtf(t);
        for (int d = 0; d < D; d++) y[d] = (x[d] * inv) * pgo_bf16_to_f32(w[d]);
    } else {
        for (int d = 0; d < D; d++) y[d] = x[d];
    }
    const int half = ROT / 2;
    for (int i = 0; i < half; i++) {
        float x1 = y[i], x2 = y[i + half];
        if (mode == 0) { /* decode: normalised pair rounded to bf16 first (:389-390) */
            x1 = pgo_bf16_to_f32(pgo_f32_to_bf16(x1));
            x2 = pgo_bf16_to_f32(pgo_f32_to_bf16(x2));
        }
        float c = cs[i], s = cs[half + i];
        float r1 = x1 * c - x2 * s;
        float r2 = x2 * c + x1 * s;
        dst[i] = pgo_f32_to_bf16(r1);
        dst[i + half] = pgo_f32_to_bf16(r2);
    }
    for (int d = ROT; d < D; d++) dst[d] = pgo_f32_to_bf16(y[d]);
}

int pgo_append_kv_rope(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                       uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                       const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                       const float *rope_table, int64_t rope_max_pos,
                       const int32_t *positions, const int64_t *slot_mapping, int64_t tokens,
                       uint16_t *k_pages, uint16_t *v_pages, int64_t num_pages, int mode) {
    for (int64_t t = 0; t < tokens; t++) {
        int32_t pos = positions[t];
        if (pos < 0 || pos >= rope_max_pos) return -2;
        const float *cs = rope_table + (int64_t)pos * ROT;
        for (int h = 0; h < NQH; h++) {
            const uint16_t *src = q_in + (t * NQH + h) * (int64_t)q_head_stride;
            prepare_row(src, q_norm_w, cs, mode, q_out + (t * NQH + h) * D);
            if (gate_out) memcpy(gate_out + (t * NQH + h) * D, src + D, D * 2);
        }
        int64_t slot = slot_mapping[t];
        if (slot < 0) continue;
        int64_t page = slot / PAGE, s = slot % PAGE;
        if (page >= num_pages) return -2;
        for (int h = 0; h < NKV; h++) {
            int64_t off = ((page * NKV + h) * PAGE + s) * D;
            prepare_row(k_in + (t * NKV + h) * D, k_norm_w, cs, mode, k_pages + off);
            memcpy(v_pages + off, v_in + (t * NKV + h) * D, D * 2);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- A1/A2 decode */

typedef struct {
    const uint16_t *k;
    const uint16_t *v;
    int64_t k_tok_stride; /* elements between consecutive tokens of K (contiguous dims) */
    int64_t v_tok_stride; /* elements between consecutive tokens of V */
    int64_t v_dim_stride; /* elements between consecutive dims of V */
} kv_row;

typedef void (*row_fn)(const void *ctx, int64_t t, kv_row *out);

typedef struct {
    const uint16_t *k_pages, *v_pages;
    const int32_t *table;
    int kvh;
} paged_ctx;

static void paged_row(const void *c, int64_t t, kv_row *r) {
    const paged_ctx *p = (const paged_ctx *)c;
    int64_t page = p->table[t / PAGE];
    int64_t off = ((page * NKV + p->kvh) * PAGE + t % PAGE) * D;
    r->k = p->k_pages + off;
    r->v = p->v_pages + off;
    r->v_dim_stride = 1;
}

typedef struct {
    const uint16_t *pk, *pv, *lk, *lv;
    int64_t ps, ls;
    int prefix_len, kvh;
} dense_ctx;

static void dense_row(const void *c, int64_t t, kv_row *r) {
    /* attention_decode.metal:57-60, :89-93: tokens < prefix_len read the prefix buffers. */
    const dense_ctx *p = (const dense_ctx *)c;
    if (t < p->prefix_len) {
        r->k = p->pk + ((int64_t)p->kvh * p->ps + t) * D;
        r->v = p->pv + (int64_t)p->kvh * D * p->ps + t;
        r->v_dim_stride = p->ps;
    } else {
        int64_t lt = t - p->prefix_len;
        r->k = p->lk + ((int64_t)p->kvh * p->ls + lt) * D;
        r->v = p->lv + (int64_t)p->kvh * D * p->ls + lt;
        r->v_dim_stride = p->ls;
    }
}

/* Split-context partials for one kv head and `nrows` query rows (row r = query j * 4 + g,
 * query j seeing `visible[j]` tokens), over tokens [t_begin, t_end):
 * attention_decode.metal:79-209. The 1024-token chunk is walked as 8 interleaved 64-token
 * tile streams (:79), each with its own online softmax (:108-130), merged at the end
 * (:170-209). Output per row: (m, l, o[256]). */
static void chunk_partial(const float qf[][D], int nrows, const int *visible, float scale,
                          row_fn rf, const void *ctx, int64_t t_begin, int64_t t_end,
                          float out[][PF]) {
    enum { SG = 8, TILE = 64, CHUNK = 1024 };
    float m[SG][NQH], den[SG][NQH];
    static __thread float acc[SG][NQH][D];
    for (int s = 0; s < SG; s++)
        for (int r = 0; r < nrows; r++) {
            m[s][r] = -INFINITY;
            den[s][r] = 0.0f;
            memset(acc[s][r], 0, sizeof(acc[s][r]));
        }
    kv_row kr;
    for (int sg = 0; sg < SG; sg++) {
        for (int tile = sg; tile < CHUNK / TILE; tile += SG) {
            int64_t tb = t_begin + (int64_t)tile * TILE;
            if (tb >= t_end) break;
            int64_t valid = t_end - tb < TILE ? t_end - tb : TILE;
            float sc[TILE][NQH];
            for (int tt = 0; tt < TILE; tt++) {
                for (int r = 0; r < nrows; r++) sc[tt][r] = -INFINITY;
                if (tt >= valid) continue;
                int64_t t = tb + tt;
                rf(ctx, t, &kr);
                for (int r = 0; r < nrows; r++) {
                    if (t >= visible[r / GRP]) continue;
                    float dot = 0.0f;
                    for (int d = 0; d < D; d++) dot += qf[r][d] * pgo_bf16_to_f32(kr.k[d]);
                    sc[tt][r] = dot * scale;
                }
            }
            for (int r = 0; r < nrows; r++) {
                float tmax = -INFINITY;
                for (int tt = 0; tt < TILE; tt++) tmax = fmaxf(tmax, sc[tt][r]);
                float mn = fmaxf(m[sg][r], tmax);
                float corr = m[sg][r] == -INFINITY ? 0.0f : expf(m[sg][r] - mn);
                float wsum = 0.0f;
                float w[TILE];
                for (int tt = 0; tt < TILE; tt++) {
                    w[tt] = sc[tt][r] == -INFINITY ? 0.0f : expf(sc[tt][r] - mn);
                    wsum += w[tt];
                }
                den[sg][r] = den[sg][r] * corr + wsum;
                m[sg][r] = mn;
                for (int d = 0; d < D; d++) acc[sg][r][d] *= corr;
                for (int tt = 0; tt < valid; tt++) {
                    if (w[tt] == 0.0f) continue;
                    rf(ctx, tb + tt, &kr);
                    for (int d = 0; d < D; d++)
                        acc[sg][r][d] += w[tt] * pgo_bf16_to_f32(kr.v[d * kr.v_dim_stride]);
                }
            }
        }
    }
    for (int r = 0; r < nrows; r++) {
        float ma = -INFINITY;
        for (int s = 0; s < SG; s++) ma = fmaxf(ma, m[s][r]);
        float da = 0.0f;
        float o[D];
        memset(o, 0, sizeof(o));
        for (int s = 0; s < SG; s++) {
            float w = m[s][r] == -INFINITY ? 0.0f : expf(m[s][r] - ma);
            da += den[s][r] * w;
            for (int d = 0; d < D; d++) o[d] += acc[s][r][d] * w;
        }
        out[r][0] = ma;
        out[r][1] = da;
        memcpy(&out[r][2], o, sizeof(o));
    }
}

/* attention_decode.metal:215-243 for one row over `n` partials (stride in floats). */
static void merge_row(const float *p, int n, int64_t stride, const uint16_t *gate, float *o) {
    float ma = -INFINITY;
    for (int c = 0; c < n; c++) ma = fmaxf(ma, p[c * stride]);
    float den = 0.0f;
    float acc[D];
    memset(acc, 0, sizeof(acc));
    for (int c = 0; c < n; c++) {
        const float *pc = p + c * stride;
        float w = pc[0] == -INFINITY ? 0.0f : expf(pc[0] - ma);
        den += pc[1] * w;
        for (int d = 0; d < D; d++) acc[d] += pc[2 + d] * w;
    }
    for (int d = 0; d < D; d++) {
        /* An empty row (no visible token) is defined as 0 here; the reference would
         * produce 0/0. */
        float v = den == 0.0f ? 0.0f : acc[d] / den;
        if (gate) v = v * (1.0f / (1.0f + expf(-pgo_bf16_to_f32(gate[d]))));
        o[d] = v;
    }
}

/* All chunk partials of one (sequence, kv head): rows nq*4, chunks of 1024 tokens
 * (attention_decode.metal:17, block_attn.zig:336-349). */
static void kvhead_partials(const uint16_t *qrows_base, int nq, int kvh, const int *visible,
                            int64_t seq_len, float scale, row_fn rf, const void *ctx,
                            float *part /* [nrows][nchunks][PF] */, int nchunks) {
    float qf[NQH][D];
    int nrows = nq * GRP;
    for (int j = 0; j < nq; j++)
        for (int g = 0; g < GRP; g++)
            for (int d = 0; d < D; d++)
                qf[j * GRP + g][d] =
                    pgo_bf16_to_f32(qrows_base[((int64_t)j * NQH + kvh * GRP + g) * D + d]);
    float out[NQH][PF];
    for (int c = 0; c < nchunks; c++) {
        int64_t tb = (int64_t)c * 1024, te = tb + 1024 < seq_len ? tb + 1024 : seq_len;
        chunk_partial((const float(*)[D])qf, nrows, visible, scale, rf, ctx, tb, te, out);
        for (int r = 0; r < nrows; r++) memcpy(part + ((int64_t)r * nchunks + c) * PF, out[r], sizeof(out[r]));
    }
}

static int decode_common(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                         int64_t num_pages, const int32_t *block_tables, int max_pages,
                         const int32_t *seq_lens, int batch, int nq, float scale,
                         const uint16_t *gate, float *out_f32, uint16_t *out_bf16,
                         float *partials_out) {
    if (nq < 1 || nq > 4) return -1;
    for (int b = 0; b < batch; b++) {
        int64_t L = seq_lens[b];
        if (L < nq || L > (int64_t)max_pages * PAGE) return -2;
        for (int64_t p = 0; p < (L + PAGE - 1) / PAGE; p++) {
            int32_t pg = block_tables[(int64_t)b * max_pages + p];
            if (pg < 0 || pg >= num_pages) return -2;
        }
    }
    int err = 0;
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(g_threads)
    for (int b = 0; b < batch; b++) {
        for (int kvh = 0; kvh < NKV; kvh++) {
            int64_t L = seq_lens[b];
            int visible[4];
            for (int j = 0; j < nq; j++) visible[j] = (int)(L - nq + j + 1);
            int nchunks = (int)((L + 1023) / 1024);
            int nrows = nq * GRP;
            float *part = (float *)malloc(sizeof(float) * nrows * nchunks * PF);
            if (!part) { err = -1; continue; }
            paged_ctx ctx = {k_pages, v_pages, block_tables + (int64_t)b * max_pages, kvh};
            kvhead_partials(q + (int64_t)b * nq * NQH * D, nq, kvh, visible, L, scale, paged_row,
                            &ctx, part, nchunks);
            for (int r = 0; r < nrows; r++) {
                int j = r / GRP, g = r % GRP;
                int64_t orow = ((int64_t)b * nq + j) * NQH + kvh * GRP + g;
                if (partials_out) {
                    float *dst = partials_out + orow * PF;
                    /* shard-level partial: merge chunks but keep (m, l, o) un-normalised */
                    float ma = -INFINITY;
                    for (int c = 0; c < nchunks; c++) ma = fmaxf(ma, part[((int64_t)r * nchunks + c) * PF]);
                    float den = 0.0f, acc[D];
                    memset(acc, 0, sizeof(acc));
                    for (int c = 0; c < nchunks; c++) {
                        const float *pc = part + ((int64_t)r * nchunks + c) * PF;
                        float w = pc[0] == -INFINITY ? 0.0f : expf(pc[0] - ma);
                        den += pc[1] * w;
                        for (int d = 0; d < D; d++) acc[d] += pc[2 + d] * w;
                    }
                    dst[0] = ma;
                    dst[1] = den;
                    memcpy(dst + 2, acc, sizeof(acc));
                } else {
                    float o[D];
                    merge_row(part + (int64_t)r * nchunks * PF, nchunks, PF,
                              gate ? gate + orow * D : NULL, o);
                    if (out_f32) memcpy(out_f32 + orow * D, o, sizeof(o));
                    if (out_bf16)
                        for (int d = 0; d < D; d++) out_bf16[orow * D + d] = pgo_f32_to_bf16(o[d]);
                }
            }
            free(part);
        }
    }
    return err;
}

int pgo_decode_paged(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                     int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                     const int32_t *seq_lens, int batch, int num_queries, float scale,
                     const uint16_t *gate, float *out_f32, uint16_t *out_bf16) {
    return decode_common(q, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                         seq_lens, batch, num_queries, scale, gate, out_f32, out_bf16, NULL);
}

int pgo_decode_partials_paged(const uint16_t *q, const uint16_t *k_pages,
                              const uint16_t *v_pages, int64_t num_pages,
                              const int32_t *block_tables, int max_pages_per_seq,
                              const int32_t *seq_lens, int batch, int num_queries,
                              float scale, float *partials) {
    return decode_common(q, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                         seq_lens, batch, num_queries, scale, NULL, NULL, NULL, partials);
}

int pgo_decode_dense_prefix(const uint16_t *q, const uint16_t *prefix_k,
                            const uint16_t *prefix_v, const uint16_t *local_k,
                            const uint16_t *local_v, int seq_len, int prefix_len, float scale,
                            int prefix_stride, int local_stride, const uint16_t *gate,
                            float *out_f32) {
    if (seq_len <= 0 || prefix_len < 0 || prefix_len > seq_len) return -1;
    int nchunks = (seq_len + 1023) / 1024;
    int visible[1] = {seq_len};
    for (int kvh = 0; kvh < NKV; kvh++) {
        float *part = (float *)malloc(sizeof(float) * GRP * nchunks * PF);
        if (!part) return -1;
        dense_ctx ctx = {prefix_k, prefix_v, local_k, local_v, prefix_stride, local_stride,
                         prefix_len, kvh};
        kvhead_partials(q, 1, kvh, visible, seq_len, scale, dense_row, &ctx, part, nchunks);
        for (int g = 0; g < GRP; g++) {
            int h = kvh * GRP + g;
            merge_row(part + (int64_t)g * nchunks * PF, nchunks, PF, gate ? gate + h * D : NULL,
                      out_f32 + h * D);
        }
        free(part);
    }
    return 0;
}

int pgo_merge_partials(const float *partials, int64_t rows, int num_parts, int64_t part_stride,
                       const uint16_t *gate, float *out_f32, uint16_t *out_bf16) {
    for (int64_t r = 0; r < rows; r++) {
        float o[D];
        merge_row(partials + r * PF, num_parts, part_stride, gate ? gate + r * D : NULL, o);
        if (out_f32) memcpy(out_f32 + r * D, o, sizeof(o));
        if (out_bf16)
            for (int d = 0; d < D; d++) out_bf16[r * D + d] = pgo_f32_to_bf16(o[d]);
    }
    return 0;
}

/* ---------------------------------------------------------------- A5 prefill */

int pgo_prefill_paged(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                      int64_t num_pages, const int32_t *block_table, int prefix_len,
                      int chunk_len, float scale, float *out_f32, uint16_t *out_bf16) {
    /* Scalar causal attention in fp32 (attention.metal:567-707 semantics) with the
     * prefix-aware mask col <= (n - tokens) + t (attention.metal:729-737, :1347-1353). */
    int64_t n = (int64_t)prefix_len + chunk_len;
    for (int64_t p = 0; p < (n + PAGE - 1) / PAGE; p++)
        if (block_table[p] < 0 || block_table[p] >= num_pages) return -2;
#pragma omp parallel for collapse(2) schedule(dynamic, 4) num_threads(g_threads)
    for (int t = 0; t < chunk_len; t++) {
        for (int h = 0; h < NQH; h++) {
            int kvh = h / GRP;
            int64_t vis = (int64_t)prefix_len + t + 1;
            float qf[D];
            for (int d = 0; d < D; d++) qf[d] = pgo_bf16_to_f32(q[((int64_t)t * NQH + h) * D + d]);
            float *s = (float *)malloc(sizeof(float) * vis);
            float mx = -INFINITY;
            for (int64_t c = 0; c < vis; c++) {
                int64_t off = (((int64_t)block_table[c / PAGE] * NKV + kvh) * PAGE + c % PAGE) * D;
                float dot = 0.0f;
                for (int d = 0; d < D; d++) dot += qf[d] * pgo_bf16_to_f32(k_pages[off + d]);
                s[c] = dot * scale;
                mx = fmaxf(mx, s[c]);
            }
            float den = 0.0f, acc[D];
            memset(acc, 0, sizeof(acc));
            for (int64_t c = 0; c < vis; c++) {
                float w = expf(s[c] - mx);
                den += w;
                int64_t off = (((int64_t)block_table[c / PAGE] * NKV + kvh) * PAGE + c % PAGE) * D;
                for (int d = 0; d < D; d++) acc[d] += w * pgo_bf16_to_f32(v_pages[off + d]);
            }
            free(s);
            int64_t orow = ((int64_t)t * NQH + h) * D;
            for (int d = 0; d < D; d++) {
                float o = acc[d] / den;
                if (out_f32) out_f32[orow + d] = o;
                if (out_bf16) out_bf16[orow + d] = pgo_f32_to_bf16(o);
            }
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- copies */

void pgo_copy_full_attention_range(uint16_t *dst_k, uint16_t *dst_v, int64_t dst_stride,
                                   int64_t dst_token, const uint16_t *src_k,
                                   const uint16_t *src_v, int64_t src_stride,
                                   int64_t src_token, int64_t count) {
    /* src/model/state.zig:182-230: K as 4 runs of count*256 values, V as 4*256 runs of
     * count values. */
    if (count == 0) return;
    for (int64_t h = 0; h < NKV; h++)
        memcpy(dst_k + (h * dst_stride + dst_token) * D, src_k + (h * src_stride + src_token) * D,
               (size_t)count * D * 2);
    for (int64_t h = 0; h < NKV; h++)
        for (int64_t d = 0; d < D; d++)
            memcpy(dst_v + (h * D + d) * dst_stride + dst_token,
                   src_v + (h * D + d) * src_stride + src_token, (size_t)count * 2);
}

static int64_t page_off(const int32_t *table, int64_t n_table, int64_t num_pages, int64_t t,
                        int kvh) {
    if (t / PAGE >= n_table) return -1;
    int64_t pg = table[t / PAGE];
    if (pg < 0 || pg >= num_pages) return -1;
    return ((pg * NKV + kvh) * PAGE + t % PAGE) * D;
}

int pgo_kv_restore_dense(const uint16_t *k_dense, const uint16_t *v_dense, int64_t src_stride,
                         int64_t src_token, uint16_t *k_pages, uint16_t *v_pages,
                         int64_t num_pages, const int32_t *block_table, int64_t n_table,
                         int64_t dst_token, int64_t count) {
    for (int64_t i = 0; i < count; i++)
        for (int h = 0; h < NKV; h++) {
            int64_t off = page_off(block_table, n_table, num_pages, dst_token + i, h);
            if (off < 0) return -2;
            memcpy(k_pages + off, k_dense + ((int64_t)h * src_stride + src_token + i) * D, D * 2);
            for (int d = 0; d < D; d++)
                v_pages[off + d] = v_dense[((int64_t)h * D + d) * src_stride + src_token + i];
        }
    return 0;
}

int pgo_kv_snapshot_dense(const uint16_t *k_pages, const uint16_t *v_pages, int64_t num_pages,
                          const int32_t *block_table, int64_t n_table, int64_t src_token,
                          uint16_t *k_dense, uint16_t *v_dense, int64_t dst_stride,
                          int64_t dst_token, int64_t count) {
    for (int64_t i = 0; i < count; i++)
        for (int h = 0; h < NKV; h++) {
            int64_t off = page_off(block_table, n_table, num_pages, src_token + i, h);
            if (off < 0) return -2;
            memcpy(k_dense + ((int64_t)h * dst_stride + dst_token + i) * D, k_pages + off, D * 2);
            for (int d = 0; d < D; d++)
                v_dense[((int64_t)h * D + d) * dst_stride + dst_token + i] = v_pages[off + d];
        }
    return 0;
}

int pgo_kv_copy_tokens(const uint16_t *src_k, const uint16_t *src_v, int64_t src_num_pages,
                       const int32_t *src_table, int64_t src_n_table, int64_t src_token,
                       uint16_t *dst_k, uint16_t *dst_v, int64_t dst_num_pages,
                       const int32_t *dst_table, int64_t dst_n_table, int64_t dst_token,
                       int64_t count) {
    for (int64_t i = 0; i < count; i++)
        for (int h = 0; h < NKV; h++) {
            int64_t so = page_off(src_table, src_n_table, src_num_pages, src_token + i, h);
            int64_t dof = page_off(dst_table, dst_n_table, dst_num_pages, dst_token + i, h);
            if (so < 0 || dof < 0) return -2;
            memcpy(dst_k + dof, src_k + so, D * 2);
            memcpy(dst_v + dof, src_v + so, D * 2);
        }
    return 0;
}

void pgo_copy_rows(void *dst, const void *src, const int32_t *dst_rows, const int32_t *src_rows,
                   int64_t n_rows, int64_t row_bytes, int64_t dst_pitch, int64_t src_pitch) {
    for (int64_t i = 0; i < n_rows; i++) {
        int64_t dr = dst_rows ? dst_rows[i] : i;
        int64_t sr = src_rows ? src_rows[i] : i;
        memcpy((char *)dst + dr * dst_pitch, (const char *)src + sr * src_pitch, (size_t)row_bytes);
    }
}

/* ---------------------------------------------------------------- A10 rollback */

void pgo_rollback(const int32_t *accept, int32_t *seq_lens, int seq_index, int reject_tokens,
                  void *const *dsts, const void *const *srcs, const uint64_t *bytes, int n) {
    /* src/server/decode_loop.zig:216-258: on reject the committed state is the pre-step state,
     * so the live recurrent/conv state returns to the snapshot and the rejected KV rows are
     * dropped by shortening the sequence. */
    if (*accept) return;
    seq_lens[seq_index] -= reject_tokens;
    for (int i = 0; i < n; i++) memcpy(dsts[i], srcs[i], (size_t)bytes[i]);
}
