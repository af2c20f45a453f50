/*
 * pgo_linear.c — CPU ORACLE (test infrastructure only) for the linear-attention (Gated-DeltaNet)
 * state producers: the depthwise causal conv1d + SiLU and the gated delta-rule recurrence.
 *
 * Also the q4 (group-64 affine) projections around the attention kernels.
 *
 * Scalar restatement of the reference shaders, each function citing the file:line it follows
 * (paths within XiaoConstantine/peregrine). Shapes are the model's (src/model/block_linear.zig:
 * 18-26): Hk = 16 key heads, Hv = 32 value heads, Dk = Dv = 128, conv_dim = 2*Hk*Dk + Hv*Dv =
 * 8192, kernel size 4. Sums follow the reference order: a lane-local loop over the dk chunks
 * {lane, lane+32, lane+64, lane+96}, then a 32-lane butterfly (xor 16, 8, 4, 2, 1) for its
 * simd_sum; the 128-thread tree for qk_l2norm_prefill_bf16. rsqrt is taken as 1/sqrtf (the
 * CUDA kernels do the same); exp/log come from libm, so the GPU comparison is within a
 * tolerance, not bit-exact. Parity unpinned: the reference holds no numeric vectors for these
 * kernels (its comments cite MLX checks only, gated_delta.metal:5-6, conv1d.metal:5-6).
 */
#include "pgo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define LHK 16
#define LHV 32
#define LDK 128
#define LDV 128
#define LKEY (LHK * LDK)
#define LVAL (LHV * LDV)
#define LCONV (2 * LKEY + LVAL)

static float silu(float x) { return x / (1.0f + expf(-x)); }

/* 32-lane butterfly sum, the value lane 0 ends with (all lanes agree). */
static float simd_sum32(const float *v) {
    float s[32];
    memcpy(s, v, sizeof(s));
    for (int o = 16; o > 0; o >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ o];
        memcpy(s, t, sizeof(s));
    }
    return s[0];
}

/* conv1d.metal:49-66 (conv1d_silu_decode_bf16): out = silu(sum_j w[c,j] * window_j), then the
 * f32 state [K-1][C] rolls (oldest first). */
void pgo_conv1d_decode(float *state, const uint16_t *x, const uint16_t *w, uint16_t *out, int C,
                       int K) {
    const int km1 = K - 1;
    for (int c = 0; c < C; ++c) {
        const float xnew = pgo_bf16_to_f32(x[c]);
        float acc = 0.0f;
        for (int j = 0; j < km1; ++j) acc += pgo_bf16_to_f32(w[(size_t)c * K + j]) * state[(size_t)j * C + c];
        acc += pgo_bf16_to_f32(w[(size_t)c * K + km1]) * xnew;
        out[c] = pgo_f32_to_bf16(silu(acc));
        for (int j = 0; j + 1 < km1; ++j) state[(size_t)j * C + c] = state[(size_t)(j + 1) * C + c];
        if (km1 > 0) state[(size_t)(km1 - 1) * C + c] = xnew;
    }
}

/* conv1d.metal:128-164 (conv1d_silu_prefill_vec4_bf16) then :166-186 (state publish). */
void pgo_conv1d_prefill(float *state, int has_state, const uint16_t *x, int T, const uint16_t *w,
                        uint16_t *out, int C, int K) {
    const int km1 = K - 1;
    for (int t = 0; t < T; ++t) {
        for (int c = 0; c < C; ++c) {
            float acc = 0.0f;
            for (int j = 0; j < K; ++j) {
                const int src = t + j;
                float v = 0.0f;
                if (src < km1) {
                    if (has_state) v = state[(size_t)src * C + c];
                } else if (src - km1 < T) {
                    v = pgo_bf16_to_f32(x[(size_t)(src - km1) * C + c]);
                }
                acc += pgo_bf16_to_f32(w[(size_t)c * K + j]) * v;
            }
            out[(size_t)t * C + c] = pgo_f32_to_bf16(silu(acc));
        }
    }
    for (int c = 0; c < C; ++c) {
        float nw[8];
        for (int j = 0; j < km1; ++j) {
            const int src = T + j;
            float v = 0.0f;
            if (src < km1) {
                if (has_state) v = state[(size_t)src * C + c];
            } else if (src - km1 < T) {
                v = pgo_bf16_to_f32(x[(size_t)(src - km1) * C + c]);
            }
            nw[j] = v;
        }
        for (int j = 0; j < km1; ++j) state[(size_t)j * C + c] = nw[j];
    }
}

/* gated_norm.metal:247-263 (gating_many_bf16): decay and beta of value head h. */
static void gates(const uint16_t *a, const uint16_t *b, const float *A_log, const uint16_t *dt_bias,
                  int h, float *decay, float *beta) {
    const float x = pgo_bf16_to_f32(a[h]) + pgo_bf16_to_f32(dt_bias[h]);
    const float sp = fmaxf(x, 0.0f) + logf(1.0f + expf(-fabsf(x)));
    *decay = expf(-expf(A_log[h]) * sp);
    *beta = 1.0f / (1.0f + expf(-pgo_bf16_to_f32(b[h])));
}

/* One token of the recurrence for value head hv (gated_delta.metal:83-129 and :213-253): rows
 * dv of state [Dv][Dk] decay, take the rank-1 delta update and produce y[dv]. q and k are the
 * normalised key-head vectors. */
static void delta_token(float *st, const float *q, const float *k, const uint16_t *v_row,
                        float decay, float beta, uint16_t *y) {
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float s = 0.0f;
        for (int ch = 0; ch < 4; ++ch) s += k[l + 32 * ch] * q[l + 32 * ch];
        lane[l] = s;
    }
    const float kq = simd_sum32(lane);
    for (int dv = 0; dv < LDV; ++dv) {
        float *row = st + (size_t)dv * LDK;
        float dec[LDK];
        float lk[32], lq[32];
        for (int l = 0; l < 32; ++l) {
            float sk = 0.0f, sq = 0.0f;
            for (int ch = 0; ch < 4; ++ch) {
                const int dk = l + 32 * ch;
                dec[dk] = row[dk] * decay;
                sk += dec[dk] * k[dk];
                sq += dec[dk] * q[dk];
            }
            lk[l] = sk;
            lq[l] = sq;
        }
        const float kv_mem = simd_sum32(lk);
        const float out_base = simd_sum32(lq);
        const float delta = (pgo_bf16_to_f32(v_row[dv]) - kv_mem) * beta;
        for (int dk = 0; dk < LDK; ++dk) row[dk] = dec[dk] + k[dk] * delta;
        y[dv] = pgo_f32_to_bf16(out_base + delta * kq);
    }
}

/* gated_delta.metal:146-261 (gated_delta_decode_h128_fused_bf16): one token, q/k L2 norms and
 * gates inline. state [Hv][Dv][Dk] f32, conv_out [conv_dim] bf16, y [Hv*Dv] bf16. */
void pgo_gated_delta_decode(float *state, int has_state, const uint16_t *conv_out, const uint16_t *a,
                            const uint16_t *b, const float *A_log, const uint16_t *dt_bias,
                            uint16_t *y) {
    if (!has_state) memset(state, 0, sizeof(float) * LHV * LDV * LDK);
    for (int hv = 0; hv < LHV; ++hv) {
        const int hk = hv / (LHV / LHK);
        float decay, beta;
        gates(a, b, A_log, dt_bias, hv, &decay, &beta);
        float qr[LDK], kr[LDK], lq[32], lk[32];
        for (int l = 0; l < 32; ++l) {
            float sq = 0.0f, sk = 0.0f;
            for (int ch = 0; ch < 4; ++ch) {
                const int dk = l + 32 * ch;
                qr[dk] = pgo_bf16_to_f32(conv_out[hk * LDK + dk]);
                kr[dk] = pgo_bf16_to_f32(conv_out[LKEY + hk * LDK + dk]);
                sq += qr[dk] * qr[dk];
                sk += kr[dk] * kr[dk];
            }
            lq[l] = sq;
            lk[l] = sk;
        }
        const float q_inv = (1.0f / sqrtf(simd_sum32(lq) + 1.0e-6f)) * (1.0f / sqrtf((float)LDK));
        const float k_inv = 1.0f / sqrtf(simd_sum32(lk) + 1.0e-6f);
        float q[LDK], k[LDK];
        for (int dk = 0; dk < LDK; ++dk) {
            q[dk] = qr[dk] * q_inv;
            k[dk] = kr[dk] * k_inv;
        }
        delta_token(state + (size_t)hv * LDV * LDK, q, k, conv_out + 2 * LKEY + hv * LDV, decay, beta,
                    y + hv * LDV);
    }
}

/* qk_l2norm_prefill_bf16 (gated_norm.metal:191-245) for one token and key head: 128-thread tree. */
static void qk_norm_prefill(const uint16_t *conv_row, int hk, float *q, float *k) {
    float pq[128], pk[128];
    for (int t = 0; t < 128; ++t) {
        const float qv = pgo_bf16_to_f32(conv_row[hk * LDK + t]);
        const float kv = pgo_bf16_to_f32(conv_row[LKEY + hk * LDK + t]);
        pq[t] = qv * qv;
        pk[t] = kv * kv;
    }
    for (int s = 64; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t) {
            pq[t] += pq[t + s];
            pk[t] += pk[t + s];
        }
    const float q_inv = 1.0f / sqrtf(pq[0] + 1.0e-6f);
    const float k_inv = 1.0f / sqrtf(pk[0] + 1.0e-6f);
    const float q_scale = 1.0f / sqrtf((float)LDK);
    for (int t = 0; t < 128; ++t) {
        q[t] = pgo_bf16_to_f32(conv_row[hk * LDK + t]) * q_inv * q_scale;
        k[t] = pgo_bf16_to_f32(conv_row[LKEY + hk * LDK + t]) * k_inv;
    }
}

/* block_linear.zig:335-346: qk_l2norm_prefill_bf16 + gating_many_bf16 per token, then
 * gated_delta_prefill_h128_norm_prepared_value_major_r8_bf16 (gated_delta.metal:35-138) over
 * the T tokens of one sequence. conv_out [T][conv_dim] bf16, a/b [T][Hv] bf16, y [T][Hv*Dv]. */
void pgo_gated_delta_prefill(float *state, int has_state, const uint16_t *conv_out, const uint16_t *a,
                             const uint16_t *b, const float *A_log, const uint16_t *dt_bias, int T,
                             uint16_t *y) {
    if (!has_state) memset(state, 0, sizeof(float) * LHV * LDV * LDK);
    for (int t = 0; t < T; ++t) {
        const uint16_t *row = conv_out + (size_t)t * LCONV;
        float q[LHK][LDK], k[LHK][LDK];
        for (int hk = 0; hk < LHK; ++hk) qk_norm_prefill(row, hk, q[hk], k[hk]);
        for (int hv = 0; hv < LHV; ++hv) {
            const int hk = hv / (LHV / LHK);
            float decay, beta;
            gates(a + (size_t)t * LHV, b + (size_t)t * LHV, A_log, dt_bias, hv, &decay, &beta);
            delta_token(state + (size_t)hv * LDV * LDK, q[hk], k[hk], row + 2 * LKEY + hv * LDV, decay,
                        beta, y + (size_t)t * LVAL + hv * LDV);
        }
    }
}

/* ---------------------------------------------------------------- q4 projections
 * Format of shaders/linear.metal:12-20: weight u32 [out][in/8] (8 nibbles, low nibble = lowest
 * column), scales and biases bf16 [out][in/64]; w = scale * q + bias. */

/* q4_affine_group64_dequantize_bf16 (linear.metal:422-444): bf16(scale * q + bias), the product
 * and the sum each rounded to fp32. */
void pgo_q4_dequantize(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                       uint16_t *out, int out_dim, int in_dim) {
    const int words = in_dim / 8, groups = in_dim / 64;
    for (int o = 0; o < out_dim; ++o)
        for (int k = 0; k < in_dim; ++k) {
            const uint32_t q = (w[(size_t)o * words + k / 8] >> ((k & 7) * 4)) & 0xFu;
            const float s = pgo_bf16_to_f32(scales[(size_t)o * groups + k / 64]);
            const float b = pgo_bf16_to_f32(biases[(size_t)o * groups + k / 64]);
            const float p = s * (float)q;
            out[(size_t)o * in_dim + k] = pgo_f32_to_bf16(p + b);
        }
}

/* The decode projection of linear.metal:64-123 (q4_affine_group64_qmv_fast_compute4_bf16): per
 * 64-input group g of row o, y += scale * sum_k(q_k * x_k) + bias * sum_k(x_k), everything in
 * fp32 (the weights are never rounded to bf16 on this path), then one bf16 rounding of y. Sums
 * run in k order. x [T][in] bf16, y [T][out] bf16. */
void pgo_q4_linear(const uint16_t *x, const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                   uint16_t *y, int T, int out_dim, int in_dim) {
    const int words = in_dim / 8, groups = in_dim / 64;
    for (int t = 0; t < T; ++t) {
        const uint16_t *xr = x + (size_t)t * in_dim;
        for (int o = 0; o < out_dim; ++o) {
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float qx = 0.0f, xs = 0.0f;
                for (int k = g * 64; k < g * 64 + 64; ++k) {
                    const uint32_t q = (w[(size_t)o * words + k / 8] >> ((k & 7) * 4)) & 0xFu;
                    const float xv = pgo_bf16_to_f32(xr[k]);
                    qx += (float)q * xv;
                    xs += xv;
                }
                const float sc = pgo_bf16_to_f32(scales[(size_t)o * groups + g]);
                const float bi = pgo_bf16_to_f32(biases[(size_t)o * groups + g]);
                acc += sc * qx + bi * xs;
            }
            y[(size_t)t * out_dim + o] = pgo_f32_to_bf16(acc);
        }
    }
}
