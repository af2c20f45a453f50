// linear_attn.cu — the linear-attention (Gated-DeltaNet) state producers on sm_100a: the
// depthwise causal conv1d + SiLU and the gated delta-rule recurrence, decode and prefill.
//
// Behaviour follows shaders/conv1d.metal:49-186 (conv1d_silu_decode_bf16,
// conv1d_silu_prefill_vec4_bf16, conv1d_silu_prefill_state_bf16), shaders/gated_delta.metal:
// 35-261 (the r8 prefill scan and the fused decode step) and shaders/gated_norm.metal:191-263
// (q/k L2 norms, gates), as composed by src/model/block_linear.zig:202-466. Shapes are the
// model's: Hk = 16, Hv = 32, Dk = Dv = 128, conv_dim 8192, kernel 4; the recurrent state is
// [Hv][Dv][Dk] f32 (2 MiB) and the conv state [3][8192] f32 per sequence.
//
// B200 layout: decode is batched over state slots (the same slot index the prefix cache hands an
// entry), so one launch updates every sequence's state in place; it streams each 2 MiB state
// once per token and is HBM-bound (4 MiB moved per sequence per layer). Each CTA is 4 warps x 8
// value rows of one head; a lane owns key dims {l, l+32, l+64, l+96}, so every state access is a
// 128-byte coalesced row chunk and the dot products keep the reference's order (lane-local
// chunk loop, then a 32-lane xor butterfly). Products and sums use round-to-nearest intrinsics
// in that order, so only expf/logf differ from the CPU restatement.
#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_linear_err);

namespace {

constexpr int kHk = PGC_LIN_KEY_HEADS, kHv = PGC_LIN_VALUE_HEADS;
constexpr int kDk = PGC_LIN_HEAD_DIM, kDv = PGC_LIN_HEAD_DIM;
constexpr int kKeyDim = kHk * kDk, kValDim = kHv * kDv;
constexpr int kConv = PGC_LIN_CONV_DIM, kKer = PGC_LIN_CONV_KERNEL;
constexpr int kRowsPerWarp = 8, kWarps = 4, kRowsPerCta = kRowsPerWarp * kWarps;
constexpr int kStateFloats = kHv * kDv * kDk;
static_assert(kConv == 2 * kKeyDim + kValDim, "conv_dim = q + k + v");
static_assert(kDv % kRowsPerCta == 0, "row tiles cover a head");

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float inv_sqrt(float x) { return __fdiv_rn(1.0f, __fsqrt_rn(x)); }

// gating_many_bf16 (gated_norm.metal:247-263)
__device__ __forceinline__ void gates(float a, float dt_bias, float a_log, float b, float *decay,
                                      float *beta) {
    const float x = __fadd_rn(a, dt_bias);
    const float sp = __fadd_rn(fmaxf(x, 0.0f), logf(__fadd_rn(1.0f, expf(-fabsf(x)))));
    *decay = expf(__fmul_rn(-expf(a_log), sp));
    *beta = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b)));
}

// ---------------------------------------------------------------- conv1d
// conv1d_silu_decode_bf16 (conv1d.metal:49-66) over a batch of sequences: thread per (channel,
// sequence); state [slot][3][8192] f32 rolls in place.
__global__ void __launch_bounds__(256) conv1d_decode_kernel(float *states, int64_t num_slots,
                                                            const int32_t *slots, const uint16_t *x,
                                                            const uint16_t *w, uint16_t *out) {
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int s = blockIdx.y;
    if (c >= kConv) return;
    const int64_t slot = slots ? slots[s] : s;
    if (slot < 0 || slot >= num_slots) {
        if (c == 0) record_error(&g_linear_err, kErrPageOutOfRange, slot);
        return;
    }
    float *st = states + slot * (int64_t)(kKer - 1) * kConv;
    const uint2 wq = *reinterpret_cast<const uint2 *>(w + (int64_t)c * kKer);
    const float w0 = bf((uint16_t)wq.x), w1 = bf((uint16_t)(wq.x >> 16));
    const float w2 = bf((uint16_t)wq.y), w3 = bf((uint16_t)(wq.y >> 16));
    const float s0 = st[c], s1 = st[kConv + c], s2 = st[2 * kConv + c];
    const float xn = bf(x[(int64_t)s * kConv + c]);
    float acc = 0.0f;
    acc = __fadd_rn(acc, __fmul_rn(w0, s0));
    acc = __fadd_rn(acc, __fmul_rn(w1, s1));
    acc = __fadd_rn(acc, __fmul_rn(w2, s2));
    acc = __fadd_rn(acc, __fmul_rn(w3, xn));
    out[(int64_t)s * kConv + c] = f32_to_bf16_bits(silu(acc));
    st[c] = s1;
    st[kConv + c] = s2;
    st[2 * kConv + c] = xn;
}

// conv1d_silu_prefill_vec4_bf16 (conv1d.metal:128-164): thread per (channel, 64-token chunk)
// with the 3-input window in registers.
constexpr int kConvChunk = 64;
__global__ void __launch_bounds__(256) conv1d_prefill_kernel(const float *state, int has_state,
                                                             const uint16_t *x, int T,
                                                             const uint16_t *w, uint16_t *out) {
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= kConv) return;
    const int t0 = blockIdx.y * kConvChunk;
    const int t1 = min(T, t0 + kConvChunk);
    const uint2 wq = *reinterpret_cast<const uint2 *>(w + (int64_t)c * kKer);
    const float w0 = bf((uint16_t)wq.x), w1 = bf((uint16_t)(wq.x >> 16));
    const float w2 = bf((uint16_t)wq.y), w3 = bf((uint16_t)(wq.y >> 16));
    // window = inputs t-3, t-2, t-1 (source indices t, t+1, t+2 of the reference's loop)
    float win[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int src = t0 - 3 + j;  // input index; < 0 reads the state row src + 3
        win[j] = src >= 0 ? bf(x[(int64_t)src * kConv + c])
                          : (has_state ? state[(int64_t)(src + 3) * kConv + c] : 0.0f);
    }
    for (int t = t0; t < t1; ++t) {
        const float xn = bf(x[(int64_t)t * kConv + c]);
        float acc = 0.0f;
        acc = __fadd_rn(acc, __fmul_rn(w0, win[0]));
        acc = __fadd_rn(acc, __fmul_rn(w1, win[1]));
        acc = __fadd_rn(acc, __fmul_rn(w2, win[2]));
        acc = __fadd_rn(acc, __fmul_rn(w3, xn));
        out[(int64_t)t * kConv + c] = f32_to_bf16_bits(silu(acc));
        win[0] = win[1];
        win[1] = win[2];
        win[2] = xn;
    }
}

// conv1d_silu_prefill_state_bf16 (conv1d.metal:166-186): the last three inputs (or, for chunks
// shorter than three, the tail of the old state) become the new state.
__global__ void __launch_bounds__(256) conv1d_publish_kernel(float *state, int has_state,
                                                             const uint16_t *x, int T) {
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= kConv) return;
    float nw[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int src = T + j;  // source index of the reference; input index src - 3
        nw[j] = src >= 3 ? bf(x[(int64_t)(src - 3) * kConv + c])
                         : (has_state ? state[(int64_t)src * kConv + c] : 0.0f);
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) state[(int64_t)j * kConv + c] = nw[j];
}

// ---------------------------------------------------------------- gated delta rule
// One warp's 8 value rows of head hv for one token: decay, rank-1 delta update, y. q/k are this
// lane's 4 normalised key values, kq their full dot product; state rows in registers.
//
// The 16 row sums (kv_mem and the y base of 8 rows) are reduced with a reduce-scatter over the
// warp instead of 16 butterflies: at each xor stage (16, 8, 4, 2) a lane keeps half of its
// values and adds the partner's copy of that half, then xor 1 completes the sum. Every stage
// adds the same operand pairs a butterfly would (fp addition is commutative), so each result is
// bitwise the butterfly's; lane l ends with value 8*b4 + 4*b3 + 2*b2 + b1 of its bits. The lane
// holding kv_mem[r] forms delta[r], the y lane (l ^ 16) receives it, and the 8 deltas are then
// broadcast for the state update: 25 shuffles per token instead of 80.
template <int R>
__device__ __forceinline__ void delta_rows(float (&st)[R][4], const float (&q)[4], const float (&k)[4],
                                           float kq, const float (&v)[R], float decay, float beta,
                                           uint16_t *y, int lane) {
    // S scatter stages (xor 16, 8, ...) halve 2R values to one; the remaining xor offsets finish
    // as a butterfly. Lane l then holds value idx = sum_i bit(16 >> i) * 2^(S-1-i): kv_mem[idx]
    // when b4 = 0, the y base of row idx - R when b4 = 1.
    constexpr int S = R == 8 ? 4 : (R == 4 ? 3 : (R == 2 ? 2 : 1));
    static_assert((2 << (S - 1)) == 2 * R, "R is 1, 2, 4 or 8");
    float acc[2 * R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float sk = 0.0f, sq = 0.0f;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            st[r][ch] = __fmul_rn(st[r][ch], decay);
            sk = __fadd_rn(sk, __fmul_rn(st[r][ch], k[ch]));
            sq = __fadd_rn(sq, __fmul_rn(st[r][ch], q[ch]));
        }
        acc[r] = sk;
        acc[R + r] = sq;
    }
#pragma unroll
    for (int st_i = 0; st_i < S; ++st_i) {
        const int n = (2 * R) >> st_i, o = 16 >> st_i;
        const bool hi = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = hi ? acc[i] : acc[i + n / 2];
            const float keep = hi ? acc[i + n / 2] : acc[i];
            acc[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
        }
    }
    float sum = acc[0];
#pragma unroll
    for (int o = 16 >> S; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    int r_mine = 0;
#pragma unroll
    for (int i = 1; i < S; ++i) r_mine |= ((lane >> (4 - i)) & 1) << (S - 1 - i);
    float vr = v[0];
#pragma unroll
    for (int r = 1; r < R; ++r) vr = r == r_mine ? v[r] : vr;
    const float delta_mine = __fmul_rn(__fsub_rn(vr, sum), beta);  // meaningful on b4 = 0 lanes
    const float delta_y = __shfl_xor_sync(0xffffffffu, delta_mine, 16);
    if ((lane & 16) && (lane & ((16 >> (S - 1)) - 1)) == 0)
        y[r_mine] = f32_to_bf16_bits(__fadd_rn(sum, __fmul_rn(delta_y, kq)));
#pragma unroll
    for (int r = 0; r < R; ++r) {
        int src = 0;
#pragma unroll
        for (int i = 1; i < S; ++i) src |= ((r >> (S - 1 - i)) & 1) << (4 - i);
        const float delta = __shfl_sync(0xffffffffu, delta_mine, src);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) st[r][ch] = __fadd_rn(st[r][ch], __fmul_rn(k[ch], delta));
    }
}

// gated_delta_decode_h128_fused_bf16 (gated_delta.metal:146-261) over a batch: grid
// (Dv / 32 row tiles, Hv, batch), 4 warps x 8 rows.
__global__ void __launch_bounds__(kWarps * 32) gated_delta_decode_kernel(
    float *states, int64_t num_slots, const int32_t *slots, int has_state,
    const uint16_t *conv_out, const uint16_t *a, const uint16_t *b, const float *a_log,
    const uint16_t *dt_bias, uint16_t *y) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int hv = blockIdx.y, s = blockIdx.z;
    const int hk = hv / (kHv / kHk);
    const int dv0 = blockIdx.x * kRowsPerCta + warp * kRowsPerWarp;
    const int64_t slot = slots ? slots[s] : s;
    if (slot < 0 || slot >= num_slots) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && hv == 0) record_error(&g_linear_err, kErrPageOutOfRange, slot);
        return;
    }
    const uint16_t *row = conv_out + (int64_t)s * kConv;
    float decay, beta;
    gates(bf(a[(int64_t)s * kHv + hv]), bf(dt_bias[hv]), a_log[hv], bf(b[(int64_t)s * kHv + hv]), &decay, &beta);

    float q[4], k[4], qss = 0.0f, kss = 0.0f;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        q[ch] = bf(row[hk * kDk + lane + 32 * ch]);
        k[ch] = bf(row[kKeyDim + hk * kDk + lane + 32 * ch]);
        qss = __fadd_rn(qss, __fmul_rn(q[ch], q[ch]));
        kss = __fadd_rn(kss, __fmul_rn(k[ch], k[ch]));
    }
    const float q_inv = __fmul_rn(inv_sqrt(__fadd_rn(warp_sum(qss), 1.0e-6f)), inv_sqrt((float)kDk));
    const float k_inv = inv_sqrt(__fadd_rn(warp_sum(kss), 1.0e-6f));
    float kq = 0.0f;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
        q[ch] = __fmul_rn(q[ch], q_inv);
        k[ch] = __fmul_rn(k[ch], k_inv);
        kq = __fadd_rn(kq, __fmul_rn(k[ch], q[ch]));
    }
    kq = warp_sum(kq);

    float *st_g = states + slot * (int64_t)kStateFloats + ((int64_t)hv * kDv + dv0) * kDk;
    float st[kRowsPerWarp][4];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
            st[r][ch] = has_state ? st_g[r * kDk + lane + 32 * ch] : 0.0f;
    float v[kRowsPerWarp];
    const uint4 vq = *reinterpret_cast<const uint4 *>(row + 2 * kKeyDim + hv * kDv + dv0);
    const uint32_t vw[4] = {vq.x, vq.y, vq.z, vq.w};
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) v[r] = bf((uint16_t)(vw[r >> 1] >> ((r & 1) * 16)));
    delta_rows<kRowsPerWarp>(st, q, k, kq, v, decay, beta, y + (int64_t)s * kValDim + hv * kDv + dv0, lane);
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) st_g[r * kDk + lane + 32 * ch] = st[r][ch];
}

// qk_l2norm_prefill_bf16 (gated_norm.metal:191-245) and gating_many_bf16 (:247-263) for one
// sequence: block (token, key head) of 128 threads with the same shared-memory tree. Outputs are
// head-major so that the scan stages a chunk of tokens with contiguous copies: q, k f32
// [16][T][128]; kq f32 [16][T] (q.k of the normalised vectors, lane-chunk order then the warp
// butterfly, as the scan would form it); g, beta f32 [32][T] (value heads 2hk and 2hk+1).
__global__ void __launch_bounds__(128) gated_delta_prep_kernel(const uint16_t *conv_out,
                                                               const uint16_t *a, const uint16_t *b,
                                                               const float *a_log,
                                                               const uint16_t *dt_bias, int T,
                                                               float *qn, float *kn, float *kqn,
                                                               float *g, float *beta) {
    pdl_trigger();
    pdl_wait();
    __shared__ float pq[128], pk[128];
    const int t = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
    const uint16_t *row = conv_out + (int64_t)t * kConv;
    const float qv = bf(row[hk * kDk + tid]);
    const float kv = bf(row[kKeyDim + hk * kDk + tid]);
    pq[tid] = __fmul_rn(qv, qv);
    pk[tid] = __fmul_rn(kv, kv);
    __syncthreads();
    for (int s = 64; s > 0; s >>= 1) {
        if (tid < s) {
            pq[tid] = __fadd_rn(pq[tid], pq[tid + s]);
            pk[tid] = __fadd_rn(pk[tid], pk[tid + s]);
        }
        __syncthreads();
    }
    const float q_inv = inv_sqrt(__fadd_rn(pq[0], 1.0e-6f));
    const float k_inv = inv_sqrt(__fadd_rn(pk[0], 1.0e-6f));
    const float q_scale = inv_sqrt((float)kDk);
    const float qo = __fmul_rn(__fmul_rn(qv, q_inv), q_scale);
    const float ko = __fmul_rn(kv, k_inv);
    const int64_t o = ((int64_t)hk * T + t) * kDk + tid;
    qn[o] = qo;
    kn[o] = ko;
    __syncthreads();  // the tree is done with pq: reuse it for q.k
    pq[tid] = __fmul_rn(ko, qo);
    __syncthreads();
    if (tid < 32) {
        float sacc = 0.0f;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) sacc = __fadd_rn(sacc, pq[tid + 32 * ch]);
        sacc = warp_sum(sacc);
        if (tid == 0) kqn[(int64_t)hk * T + t] = sacc;
        if (tid < 2) {
            const int hv = 2 * hk + tid;
            float d, bt;
            gates(bf(a[(int64_t)t * kHv + hv]), bf(dt_bias[hv]), a_log[hv], bf(b[(int64_t)t * kHv + hv]), &d, &bt);
            g[(int64_t)hv * T + t] = d;
            beta[(int64_t)hv * T + t] = bt;
        }
    }
}

// gated_delta_prefill_h128_norm_prepared_value_major_r8_bf16 (gated_delta.metal:35-138): the
// scan over T tokens of one sequence, state rows in registers. The token loop is sequential, so
// what bounds it is the latency of one token's update; the inputs every warp of a head needs
// (q, k, q.k, gates) are staged once per CTA in shared memory, 64 tokens at a time and double
// buffered with cp.async, instead of being re-read from L2 by each warp. CTA = 32 value rows of
// one head (8 warps x 4 rows); grid 4 x 32 = 128 CTAs, one per SM: per token each SM issues the
// ~180 instructions of each of its 8 warps, and more rows per SM would make issue the bound.
constexpr int kScanRows = 4;
constexpr int kScanWarps = 8;
constexpr int kScanRowsPerCta = kScanRows * kScanWarps;
constexpr int kScanChunk = 64;
struct ScanStage {
    float q[kScanChunk][kDk];
    float k[kScanChunk][kDk];
    float kq[kScanChunk];
    float g[kScanChunk];
    float beta[kScanChunk];
    uint16_t v[kScanChunk][kScanRowsPerCta];
};
constexpr int kScanSmem = 2 * (int)sizeof(ScanStage);

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem_dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(kScanWarps * 32) gated_delta_scan_kernel(
    float *state, int has_state, const uint16_t *conv_out, const float *qn, const float *kn,
    const float *kqn, const float *g, const float *beta, int T, uint16_t *y) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t scan_smem[];
    ScanStage *stage = reinterpret_cast<ScanStage *>(scan_smem);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
    const int hv = blockIdx.y;
    const int hk = hv / (kHv / kHk);
    const int row0 = blockIdx.x * kScanRowsPerCta;
    const int dv0 = row0 + warp * kScanRows;
    float *st_g = state + ((int64_t)hv * kDv + dv0) * kDk;
    float st[kScanRows][4];
#pragma unroll
    for (int r = 0; r < kScanRows; ++r)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) st[r][ch] = has_state ? st_g[r * kDk + lane + 32 * ch] : 0.0f;

    const int n_chunks = (T + kScanChunk - 1) / kScanChunk;
    auto issue = [&](int c) {
        ScanStage &sg = stage[c & 1];
        const int t0 = c * kScanChunk;
        const int n = min(kScanChunk, T - t0);
        const float *qs = qn + ((int64_t)hk * T + t0) * kDk;
        const float *ks = kn + ((int64_t)hk * T + t0) * kDk;
        for (int i = tid; i < n * (kDk / 4); i += kScanWarps * 32) {
            cp_async16(&sg.q[0][0] + 4 * i, qs + 4 * i);
            cp_async16(&sg.k[0][0] + 4 * i, ks + 4 * i);
        }
        for (int i = tid; i < n; i += kScanWarps * 32) {
            cp_async4(&sg.kq[i], kqn + (int64_t)hk * T + t0 + i);
            cp_async4(&sg.g[i], g + (int64_t)hv * T + t0 + i);
            cp_async4(&sg.beta[i], beta + (int64_t)hv * T + t0 + i);
        }
        // v: this CTA's 64 rows of each token = 128 contiguous bytes of conv_out
        for (int i = tid; i < n * (kScanRowsPerCta / 8); i += kScanWarps * 32) {
            const int tt = i / (kScanRowsPerCta / 8), u = i % (kScanRowsPerCta / 8);
            cp_async16(&sg.v[tt][8 * u],
                       conv_out + (int64_t)(t0 + tt) * kConv + 2 * kKeyDim + hv * kDv + row0 + 8 * u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (n_chunks > 0) issue(0);
    for (int c = 0; c < n_chunks; ++c) {
        if (c + 1 < n_chunks) {
            issue(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // chunk c is in shared memory for every warp
        const ScanStage &sg = stage[c & 1];
        const int t0 = c * kScanChunk;
        const int n = min(kScanChunk, T - t0);
        for (int i = 0; i < n; ++i) {
            float q[4], k[4];
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                q[ch] = sg.q[i][lane + 32 * ch];
                k[ch] = sg.k[i][lane + 32 * ch];
            }
            const uint2 vv = *reinterpret_cast<const uint2 *>(&sg.v[i][warp * kScanRows]);
            const float v[kScanRows] = {bf((uint16_t)vv.x), bf((uint16_t)(vv.x >> 16)), bf((uint16_t)vv.y),
                                        bf((uint16_t)(vv.y >> 16))};
            delta_rows<kScanRows>(st, q, k, sg.kq[i], v, sg.g[i], sg.beta[i],
                                  y + (int64_t)(t0 + i) * kValDim + hv * kDv + dv0, lane);
        }
        __syncthreads();  // every warp is done with stage c & 1 before chunk c + 2 refills it
    }
#pragma unroll
    for (int r = 0; r < kScanRows; ++r)
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) st_g[r * kDk + lane + 32 * ch] = st[r][ch];
}

}  // namespace

size_t gated_delta_prefill_workspace_bytes(int tokens) {
    if (tokens <= 0) return 0;
    return (size_t)tokens * (2 * kKeyDim + kHk + 2 * kHv) * sizeof(float);
}

cudaError_t launch_conv1d_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                                 const uint16_t *x, const uint16_t *w, uint16_t *out,
                                 cudaStream_t stream) {
    return launch_pdl(conv1d_decode_kernel, dim3(kConv / 256, batch), dim3(256), 0, stream, states,
                      num_slots, slots, x, w, out);
}

cudaError_t launch_conv1d_prefill(float *state, int has_state, const uint16_t *x, int T,
                                  const uint16_t *w, uint16_t *out, cudaStream_t stream) {
    cudaError_t e = launch_pdl(conv1d_prefill_kernel, dim3(kConv / 256, (T + kConvChunk - 1) / kConvChunk),
                               dim3(256), 0, stream, (const float *)state, has_state, x, T, w, out);
    if (e != cudaSuccess) return e;
    return launch_pdl(conv1d_publish_kernel, dim3(kConv / 256), dim3(256), 0, stream, state, has_state, x, T);
}

cudaError_t launch_gated_delta_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                                      int has_state, const uint16_t *conv_out, const uint16_t *a,
                                      const uint16_t *b, const float *a_log, const uint16_t *dt_bias,
                                      uint16_t *y, cudaStream_t stream) {
    return launch_pdl(gated_delta_decode_kernel, dim3(kDv / kRowsPerCta, kHv, batch), dim3(kWarps * 32), 0,
                      stream, states, num_slots, slots, has_state, conv_out, a, b, a_log, dt_bias, y);
}

cudaError_t launch_gated_delta_prefill(float *state, int has_state, const uint16_t *conv_out,
                                       const uint16_t *a, const uint16_t *b, const float *a_log,
                                       const uint16_t *dt_bias, int T, uint16_t *y, void *ws,
                                       cudaStream_t stream) {
    float *qn = static_cast<float *>(ws);
    float *kn = qn + (size_t)T * kKeyDim;
    float *kqn = kn + (size_t)T * kKeyDim;
    float *g = kqn + (size_t)T * kHk;
    float *beta = g + (size_t)T * kHv;
    cudaError_t e = launch_pdl(gated_delta_prep_kernel, dim3(T, kHk), dim3(128), 0, stream, conv_out, a, b,
                               a_log, dt_bias, T, qn, kn, kqn, g, beta);
    if (e != cudaSuccess) return e;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(gated_delta_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    return launch_pdl(gated_delta_scan_kernel, dim3(kDv / kScanRowsPerCta, kHv), dim3(kScanWarps * 32),
                      kScanSmem, stream, state, has_state, conv_out, (const float *)qn, (const float *)kn,
                      (const float *)kqn, (const float *)g, (const float *)beta, T, y);
}

cudaError_t linear_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_linear_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_linear_err, &z, sizeof(DevError));
}

}  // namespace pgc
