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
// head-major so that a chunk of tokens is contiguous: q, k f32 [16][T][128]; the log of the
// decay (-exp(A_log) * softplus(a + dt_bias), whose exp is gating_many's g) and beta f32
// [32][T] for value heads 2hk and 2hk+1.
__global__ void __launch_bounds__(128) gated_delta_prep_kernel(const uint16_t *conv_out,
                                                               const uint16_t *a, const uint16_t *b,
                                                               const float *a_log,
                                                               const uint16_t *dt_bias, int T,
                                                               float *qn, float *kn, float *lgd,
                                                               float *beta) {
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
    const int64_t o = ((int64_t)hk * T + t) * kDk + tid;
    qn[o] = __fmul_rn(__fmul_rn(qv, q_inv), q_scale);
    kn[o] = __fmul_rn(kv, k_inv);
    if (tid < 2) {
        const int hv = 2 * hk + tid;
        const float x = __fadd_rn(bf(a[(int64_t)t * kHv + hv]), bf(dt_bias[hv]));
        const float sp = __fadd_rn(fmaxf(x, 0.0f), logf(__fadd_rn(1.0f, expf(-fabsf(x)))));
        lgd[(int64_t)hv * T + t] = __fmul_rn(-expf(a_log[hv]), sp);
        beta[(int64_t)hv * T + t] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bf(b[(int64_t)t * kHv + hv]))));
    }
}

// ---------------------------------------------------------------- chunked recurrence
// The prefill recurrence over T tokens in chunks of C = 64, the standard chunked form of the
// gated delta rule. Within a chunk, with lg_i the cumulative log-decay from the chunk start
// (log space, so products of decays cannot underflow) and S_0 the state entering the chunk:
//   delta = T_c (beta * (V - e^{lg} * (K S_0^T))),  T_c = (I + A)^{-1},
//   A_ij = beta_i e^{lg_i - lg_j} (k_i . k_j) for j < i,
// so with U = T_c (beta * V) and W = T_c (beta * e^{lg} * K) (no state in either):
//   delta = U - W S_0^T
//   y     = e^{lg} * (Q S_0^T) + QKm delta,   QKm_ij = e^{lg_i - lg_j} (q_i . k_j) for j <= i
//   S_C   = e^{lg_C} S_0 + delta^T (e^{lg_C - lg} * K).
// This is the sequential recurrence of gated_delta.metal:35-138 regrouped: the same fp32
// arithmetic in a different order. gated_delta_chunk_kernel computes U, W, QKm and lg for every
// (chunk, value head) in parallel; gated_delta_chunk_scan_kernel then walks the chunks with the
// state, each CTA owning 32 value rows of one head (the rows are independent given K, beta, g).
constexpr int kChunk = 64;
constexpr int kRowP = kDk + 4;      // f32 rows of 128 padded by 16 B: float4 rows 4 banks apart
constexpr int kQKP = kChunk + 4;    // f32 rows of 64, same padding

struct ChunkWs {
    // per (value head, chunk): U, W [64][128], QKm [64][64], lg [64]
    static constexpr int64_t kUW = (int64_t)kChunk * kDk;
    static constexpr int64_t kQK = (int64_t)kChunk * kChunk;
    static constexpr int64_t kPer = 2 * kUW + kQK + kChunk;
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(src) : "memory");
}
// 16-byte copy that writes zeros without reading when `valid` is false
__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float dot4(const float4 &a, const float4 &b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    return fmaf(a.w, b.w, acc);
}

// Per (chunk, value head): A, QKm, then U and W by forward substitution. 256 threads.
// Shared memory (~101 KB, two CTAs per SM): K, Q [64][132] (later the U and W solutions
// [64][128] each), A transposed At[j][i] [64][68], lg, beta [64], the V slice [64][128] bf16.
constexpr int kChunkSmemFloats = 2 * kChunk * kRowP + kChunk * kQKP + 2 * kChunk + kChunk * kDv / 2;
__global__ void __launch_bounds__(256, 2) gated_delta_chunk_kernel(const float *qn, const float *kn,
                                                                const float *lgd, const float *beta,
                                                                const uint16_t *conv_out, int T,
                                                                float *cw) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float ck_smem[];
    float *Ks = ck_smem;                 // [64][132]
    float *Qs = Ks + kChunk * kRowP;     // [64][132]
    float *At = Qs + kChunk * kRowP;     // [64][68]: At[j][i] = A[i][j]
    float *lg = At + kChunk * kQKP;      // [64]
    float *bt = lg + kChunk;             // [64]
    uint16_t *vst = reinterpret_cast<uint16_t *>(bt + kChunk);  // [64][128] bf16
    const int c = blockIdx.x, hv = blockIdx.y, tid = threadIdx.x;
    const int hk = hv / (kHv / kHk);
    const int nc = gridDim.x;
    const int t0 = c * kChunk;
    const int n = min(kChunk, T - t0);
    {
        const float *ksrc = kn + ((int64_t)hk * T + t0) * kDk;
        const float *qsrc = qn + ((int64_t)hk * T + t0) * kDk;
        for (int i = tid; i < kChunk * kDk / 4; i += 256) {
            const int r = i / (kDk / 4), k4 = i % (kDk / 4);
            const bool ok = r < n;
            cp_async16_zfill(Ks + r * kRowP + 4 * k4, ok ? ksrc + r * kDk + 4 * k4 : ksrc, ok);
            cp_async16_zfill(Qs + r * kRowP + 4 * k4, ok ? qsrc + r * kDk + 4 * k4 : qsrc, ok);
        }
        cp_async_commit();
    }
    // beta and the per-token log decays (the decays go through `lg` first, then each of the 64
    // threads sums its own prefix in token order, the same order as one running sum)
    if (tid < kChunk) {
        bt[tid] = tid < n ? beta[(int64_t)hv * T + t0 + tid] : 0.f;
        lg[tid] = tid < n ? lgd[(int64_t)hv * T + t0 + tid] : 0.f;
    }
    // V slice of the chunk (bf16), coalesced
    for (int i = tid; i < kChunk * kDv; i += 256) {
        const int r = i / kDv, k = i % kDv;
        vst[i] = r < n ? conv_out[(int64_t)(t0 + r) * kConv + 2 * kKeyDim + hv * kDv + k] : 0;
    }
    __syncthreads();
    float lgi = 0.f;
    if (tid < kChunk)
        for (int j = 0; j <= tid; ++j) lgi += lg[j];
    __syncthreads();
    if (tid < kChunk) lg[tid] = lgi;
    cp_async_wait<0>();
    __syncthreads();
    float *out = cw + ((int64_t)hv * nc + c) * ChunkWs::kPer;
    float *U = out, *W = out + ChunkWs::kUW, *QK = out + 2 * ChunkWs::kUW, *LG = QK + ChunkWs::kQK;
    // A (strictly lower) and QKm (lower incl. diagonal): 4x4 (i, j) per thread, i = bi + 16 ii,
    // j = bj + 16 jj, dot products over k in order k = 0..127.
    {
        const int bi = tid >> 4, bj = tid & 15;
        float kk[4][4] = {}, qk[4][4] = {};
#pragma unroll 2
        for (int k = 0; k < kDk; k += 4) {
            float4 ki[4], qi[4], kj[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                ki[x] = ld4(Ks + (bi + 16 * x) * kRowP + k);
                qi[x] = ld4(Qs + (bi + 16 * x) * kRowP + k);
                kj[x] = ld4(Ks + (bj + 16 * x) * kRowP + k);
            }
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) {
                    kk[x][y] = dot4(ki[x], kj[y], kk[x][y]);
                    qk[x][y] = dot4(qi[x], kj[y], qk[x][y]);
                }
        }
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int i = bi + 16 * x, j = bj + 16 * y;
                const bool in = j <= i && i < n;
                const float dec = in ? expf(lg[i] - lg[j]) : 0.f;
                At[j * kQKP + i] = j < i ? bt[i] * dec * kk[x][y] : 0.f;
                QK[i * kChunk + j] = dec * qk[x][y];
            }
    }
    if (tid < kChunk) LG[tid] = lg[tid];
    // right-hand sides: column `col` of beta * V (threads 0-127) or beta * e^{lg} * K (128-255)
    const int col = tid & 127;
    const bool is_w = tid >= 128;
    float *us = is_w ? Qs : Ks;  // [64][128], free once the right-hand sides are in registers
    float rhs[kChunk];
#pragma unroll
    for (int i = 0; i < kChunk; ++i)
        rhs[i] = is_w ? bt[i] * expf(lg[i]) * Ks[i * kRowP + col] : bt[i] * bf(vst[i * kDv + col]);
    __syncthreads();  // At complete; every thread has read K and Q
#pragma unroll
    for (int i = 0; i < kChunk; ++i) us[i * kDk + col] = rhs[i];
    // forward substitution u_i = r_i - sum_{j<i} A_ij u_j in 16-row blocks: the earlier blocks
    // enter as independent dot products, then a 16-step solve inside the block. Each thread
    // touches only its own column of `us`.
    for (int blk = 0; blk < kChunk / 16; ++blk) {
        float r[16];
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) r[ii] = us[(blk * 16 + ii) * kDk + col];
        for (int j = 0; j < blk * 16; ++j) {
            const float uj = us[j * kDk + col];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 a = ld4(At + j * kQKP + blk * 16 + 4 * q);
                r[4 * q + 0] = fmaf(-a.x, uj, r[4 * q + 0]);
                r[4 * q + 1] = fmaf(-a.y, uj, r[4 * q + 1]);
                r[4 * q + 2] = fmaf(-a.z, uj, r[4 * q + 2]);
                r[4 * q + 3] = fmaf(-a.w, uj, r[4 * q + 3]);
            }
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
            for (int ii = jj + 1; ii < 16; ++ii)
                r[ii] = fmaf(-At[(blk * 16 + jj) * kQKP + blk * 16 + ii], r[jj], r[ii]);
        }
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) us[(blk * 16 + ii) * kDk + col] = r[ii];
    }
    float *dst = is_w ? W : U;
    for (int i = 0; i < kChunk; ++i) dst[i * kDk + col] = us[i * kDk + col];
}

// 3xTF32 products on the tensor cores (mma.sync m16n8k8): each fp32 operand x is split into
// big = tf32(x) and small = tf32(x - big), and a*b is accumulated as a_small*b_big +
// a_big*b_small + a_big*b_big, which keeps about 22 bits of every product (the small*small term
// is below fp32 rounding).
__device__ __forceinline__ uint32_t tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t &big, uint32_t &small) {
    big = tf32_rna(x);
    small = tf32_rna(x - __uint_as_float(big));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// A fragment (16 x 8, row-major) of rows r0 + g and r0 + g + 8, columns c + t and c + t + 4,
// read from f32 rows of `ld` floats, split into big and small parts
__device__ __forceinline__ void frag_a(const float *m, int ld, int r0, int c, int g, int t, uint32_t (&big)[4],
                                       uint32_t (&small)[4]) {
    split_tf32(m[(r0 + g) * ld + c + t], big[0], small[0]);
    split_tf32(m[(r0 + g + 8) * ld + c + t], big[1], small[1]);
    split_tf32(m[(r0 + g) * ld + c + t + 4], big[2], small[2]);
    split_tf32(m[(r0 + g + 8) * ld + c + t + 4], big[3], small[3]);
}
__device__ __forceinline__ void mma3(float (&d)[4], const uint32_t (&ab)[4], const uint32_t (&as)[4], uint32_t bb0,
                                     uint32_t bb1, uint32_t bs0, uint32_t bs1) {
    mma_tf32(d, as, bb0, bb1);
    mma_tf32(d, ab, bs0, bs1);
    mma_tf32(d, ab, bb0, bb1);
}

// The state walk: CTA = (32 value rows, value head), 256 threads; the 32 x 128 state slice stays
// in shared memory across chunks. Each chunk's tiles are staged in shared memory with cp.async
// in two groups, A = {W, Q, U slice} and B = {K, QKm, lg}: A of chunk c+1 loads during phase 2
// of chunk c (after phase 1 has released W, Q, U), B of chunk c+1 during phase 1 of chunk c+1.
// The three products run on the tensor cores in 3xTF32 (g = lane / 4, t = lane % 4 below):
//   phase 1   delta = U - W S^T, QS = Q S^T    warp w: rows 16 (w / 2).., value rows 16 (w % 2)..
//   phase 2a  y = e^{lg} QS + QKm delta        same tile (QS stays in registers)
//   phase 2b  S = e^{lg_C} S + (e^{lg_C - lg} delta)^T K   warp w: value rows 16 (w / 4)..,
//                                                           keys 32 (w % 4)..
// Shared-memory rows are padded to 4 mod 32 floats, so every fragment read is conflict-free.

constexpr int kRowsScan = 32;
constexpr int kDP = kRowsScan + 4;
struct ScanSmem {
    static constexpr int S = 0;                              // [32][132]
    static constexpr int W = S + kRowsScan * kRowP;          // [64][132]
    static constexpr int Q = W + kChunk * kRowP;             // [64][132]
    static constexpr int U = Q + kChunk * kRowP;             // [64][32]
    static constexpr int K = U + kChunk * kRowsScan;         // [64][132]
    static constexpr int QK = K + kChunk * kRowP;            // [64][68]
    static constexpr int LG = QK + kChunk * kQKP;            // [64]
    static constexpr int D = LG + kChunk;                    // [64][36]
    static constexpr int Ds = D + kChunk * kDP;              // [64][36], scaled by e^{lg_C - lg}
    static constexpr int kFloats = Ds + kChunk * kDP;
};

__global__ void __launch_bounds__(256) gated_delta_chunk_scan_kernel(float *state, int has_state,
                                                                     const float *qn, const float *kn,
                                                                     const float *cw, int T,
                                                                     uint16_t *y) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) float cs_smem[];
    float *S = cs_smem + ScanSmem::S, *Ws = cs_smem + ScanSmem::W, *Qs = cs_smem + ScanSmem::Q;
    float *Us = cs_smem + ScanSmem::U, *Ks = cs_smem + ScanSmem::K, *QKs = cs_smem + ScanSmem::QK;
    float *LGs = cs_smem + ScanSmem::LG, *Dl = cs_smem + ScanSmem::D, *Dsc = cs_smem + ScanSmem::Ds;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
    const int hv = blockIdx.y, hk = hv / (kHv / kHk);
    const int r0 = blockIdx.x * kRowsScan;
    const int nc = (T + kChunk - 1) / kChunk;
    float *st_g = state + ((int64_t)hv * kDv + r0) * kDk;

    auto issue_a = [&](int c) {
        const int t0 = c * kChunk, n = min(kChunk, T - t0);
        const float *base = cw + ((int64_t)hv * nc + c) * ChunkWs::kPer;
        const float *Wg = base + ChunkWs::kUW;
        const float *Qg = qn + ((int64_t)hk * T + t0) * kDk;
        for (int i = tid; i < kChunk * kDk / 4; i += 256) {
            const int r = i >> 5, k4 = i & 31;
            cp_async16(Ws + r * kRowP + 4 * k4, Wg + r * kDk + 4 * k4);
            const bool ok = r < n;
            cp_async16_zfill(Qs + r * kRowP + 4 * k4, ok ? Qg + r * kDk + 4 * k4 : Qg, ok);
        }
        for (int i = tid; i < kChunk * kRowsScan / 4; i += 256) {
            const int r = i >> 3, q = i & 7;
            cp_async16(Us + r * kRowsScan + 4 * q, base + r * kDk + r0 + 4 * q);
        }
        cp_async_commit();
    };
    auto issue_b = [&](int c) {
        const int t0 = c * kChunk, n = min(kChunk, T - t0);
        const float *base = cw + ((int64_t)hv * nc + c) * ChunkWs::kPer;
        const float *QKg = base + 2 * ChunkWs::kUW;
        const float *Kg = kn + ((int64_t)hk * T + t0) * kDk;
        for (int i = tid; i < kChunk * kDk / 4; i += 256) {
            const int r = i >> 5, k4 = i & 31;
            const bool ok = r < n;
            cp_async16_zfill(Ks + r * kRowP + 4 * k4, ok ? Kg + r * kDk + 4 * k4 : Kg, ok);
        }
        for (int i = tid; i < kChunk * kChunk / 4; i += 256) {
            const int r = i >> 4, q = i & 15;
            cp_async16(QKs + r * kQKP + 4 * q, QKg + r * kChunk + 4 * q);
        }
        if (tid < kChunk / 4) cp_async16(LGs + 4 * tid, QKg + ChunkWs::kQK + 4 * tid);
        cp_async_commit();
    };

    issue_a(0);
    issue_b(0);
    for (int i = tid; i < kRowsScan * kDk; i += 256)
        S[(i / kDk) * kRowP + i % kDk] = has_state ? st_g[i] : 0.f;
    const int i0 = (w >> 1) * 16, n0 = (w & 1) * 16;  // phase 1 / 2a tile
    const int rb = (w >> 2) * 16, kb = (w & 3) * 32;   // phase 2b tile
    for (int c = 0; c < nc; ++c) {
        const int t0 = c * kChunk, n = min(kChunk, T - t0);
        cp_async_wait<1>();  // A(c) landed (B(c) may still be in flight)
        __syncthreads();
        // phase 1: dacc = W S^T, qacc = Q S^T over the 128 keys
        float dacc[2][4] = {}, qacc[2][4] = {};
#pragma unroll 2
        for (int k = 0; k < kDk; k += 8) {
            uint32_t wb[4], wsm[4], qb[4], qsm[4];
            frag_a(Ws, kRowP, i0, k, g, t, wb, wsm);
            frag_a(Qs, kRowP, i0, k, g, t, qb, qsm);
#pragma unroll
            for (int nn = 0; nn < 2; ++nn) {
                // B[k][r] = S[r][k]: column r = n0 + 8 nn + g, rows k + t and k + t + 4
                const float *sr = S + (n0 + 8 * nn + g) * kRowP + k + t;
                uint32_t bb0, bs0, bb1, bs1;
                split_tf32(sr[0], bb0, bs0);
                split_tf32(sr[4], bb1, bs1);
                mma3(dacc[nn], wb, wsm, bb0, bb1, bs0, bs1);
                mma3(qacc[nn], qb, qsm, bb0, bb1, bs0, bs1);
            }
        }
        // delta = U - W S^T at rows i0 + g (+8), value rows n0 + 8 nn + 2t (+1)
#pragma unroll
        for (int nn = 0; nn < 2; ++nn) {
            const int col = n0 + 8 * nn + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = i0 + g + 8 * h;
                dacc[nn][2 * h] = Us[i * kRowsScan + col] - dacc[nn][2 * h];
                dacc[nn][2 * h + 1] = Us[i * kRowsScan + col + 1] - dacc[nn][2 * h + 1];
                *reinterpret_cast<float2 *>(Dl + i * kDP + col) = make_float2(dacc[nn][2 * h], dacc[nn][2 * h + 1]);
            }
        }
        __syncthreads();  // W, Q, U released; delta complete
        if (c + 1 < nc) {
            issue_a(c + 1);
            cp_async_wait<1>();  // B(c)
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float lgC = LGs[n - 1];
        // phase 2a: y = e^{lg} QS + QKm delta (QKm is zero above the diagonal: j <= i0 + 15)
        {
            float yacc[2][4];
            const float e0 = expf(LGs[i0 + g]), e1 = expf(LGs[i0 + g + 8]);
            const float c0 = expf(lgC - LGs[i0 + g]), c1 = expf(lgC - LGs[i0 + g + 8]);
#pragma unroll
            for (int nn = 0; nn < 2; ++nn) {
                yacc[nn][0] = e0 * qacc[nn][0];
                yacc[nn][1] = e0 * qacc[nn][1];
                yacc[nn][2] = e1 * qacc[nn][2];
                yacc[nn][3] = e1 * qacc[nn][3];
                const int col = n0 + 8 * nn + 2 * t;
                *reinterpret_cast<float2 *>(Dsc + (i0 + g) * kDP + col) =
                    make_float2(dacc[nn][0] * c0, dacc[nn][1] * c0);
                *reinterpret_cast<float2 *>(Dsc + (i0 + g + 8) * kDP + col) =
                    make_float2(dacc[nn][2] * c1, dacc[nn][3] * c1);
            }
            for (int j = 0; j < i0 + 16; j += 8) {
                uint32_t ab[4], as[4];
                frag_a(QKs, kQKP, i0, j, g, t, ab, as);
#pragma unroll
                for (int nn = 0; nn < 2; ++nn) {
                    // B[j][r] = delta[j][r]: column n0 + 8 nn + g, rows j + t and j + t + 4
                    const float *dr = Dl + (j + t) * kDP + n0 + 8 * nn + g;
                    uint32_t bb0, bs0, bb1, bs1;
                    split_tf32(dr[0], bb0, bs0);
                    split_tf32(dr[4 * kDP], bb1, bs1);
                    mma3(yacc[nn], ab, as, bb0, bb1, bs0, bs1);
                }
            }
#pragma unroll
            for (int nn = 0; nn < 2; ++nn) {
                const int col = r0 + n0 + 8 * nn + 2 * t;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = i0 + g + 8 * h;
                    if (i < n)
                        *reinterpret_cast<uint32_t *>(y + (int64_t)(t0 + i) * kValDim + hv * kDv + col) =
                            pack_bf16x2(yacc[nn][2 * h], yacc[nn][2 * h + 1]);
                }
            }
        }
        __syncthreads();  // the scaled delta is complete
        // phase 2b: S[r][k] = e^{lg_C} S[r][k] + sum_j Dsc[j][r] K[j][k] for this warp's tile
        {
            const float eC = expf(lgC);
            float sacc[4][4];
#pragma unroll
            for (int nn = 0; nn < 4; ++nn) {
                const int col = kb + 8 * nn + 2 * t;
                const float2 s0 = *reinterpret_cast<const float2 *>(S + (rb + g) * kRowP + col);
                const float2 s1 = *reinterpret_cast<const float2 *>(S + (rb + g + 8) * kRowP + col);
                sacc[nn][0] = eC * s0.x;
                sacc[nn][1] = eC * s0.y;
                sacc[nn][2] = eC * s1.x;
                sacc[nn][3] = eC * s1.y;
            }
#pragma unroll 2
            for (int j = 0; j < kChunk; j += 8) {
                // A[r][j] = Dsc[j][r]: rows rb + g (+8), columns j + t (+4)
                uint32_t ab[4], as[4];
                split_tf32(Dsc[(j + t) * kDP + rb + g], ab[0], as[0]);
                split_tf32(Dsc[(j + t) * kDP + rb + g + 8], ab[1], as[1]);
                split_tf32(Dsc[(j + t + 4) * kDP + rb + g], ab[2], as[2]);
                split_tf32(Dsc[(j + t + 4) * kDP + rb + g + 8], ab[3], as[3]);
#pragma unroll
                for (int nn = 0; nn < 4; ++nn) {
                    const float *kr = Ks + (j + t) * kRowP + kb + 8 * nn + g;
                    uint32_t bb0, bs0, bb1, bs1;
                    split_tf32(kr[0], bb0, bs0);
                    split_tf32(kr[4 * kRowP], bb1, bs1);
                    mma3(sacc[nn], ab, as, bb0, bb1, bs0, bs1);
                }
            }
            // every thread has finished reading S (phase 1) before this point; each element
            // below has one owner
#pragma unroll
            for (int nn = 0; nn < 4; ++nn) {
                const int col = kb + 8 * nn + 2 * t;
                *reinterpret_cast<float2 *>(S + (rb + g) * kRowP + col) = make_float2(sacc[nn][0], sacc[nn][1]);
                *reinterpret_cast<float2 *>(S + (rb + g + 8) * kRowP + col) = make_float2(sacc[nn][2], sacc[nn][3]);
            }
        }
        __syncthreads();  // K, QKm, lg, delta released
        if (c + 1 < nc) issue_b(c + 1);
    }
    __syncthreads();
    for (int i = tid; i < kRowsScan * kDk; i += 256) st_g[i] = S[(i / kDk) * kRowP + i % kDk];
}

}  // namespace

size_t gated_delta_prefill_workspace_bytes(int tokens) {
    if (tokens <= 0) return 0;
    const int64_t nc = (tokens + kChunk - 1) / kChunk;
    return ((size_t)tokens * (2 * kKeyDim + 2 * kHv) + (size_t)kHv * nc * ChunkWs::kPer) * sizeof(float);
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
    float *lgd = kn + (size_t)T * kKeyDim;
    float *beta = lgd + (size_t)T * kHv;
    float *cw = beta + (size_t)T * kHv;
    const int nc = (T + kChunk - 1) / kChunk;
    cudaError_t e = launch_pdl(gated_delta_prep_kernel, dim3(T, kHk), dim3(128), 0, stream, conv_out, a, b,
                               a_log, dt_bias, T, qn, kn, lgd, beta);
    if (e != cudaSuccess) return e;
    constexpr int kChunkSmem = kChunkSmemFloats * (int)sizeof(float);
    constexpr int kScanSmemC = ScanSmem::kFloats * (int)sizeof(float);
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(gated_delta_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kChunkSmem);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(gated_delta_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kScanSmemC);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    e = launch_pdl(gated_delta_chunk_kernel, dim3(nc, kHv), dim3(256), kChunkSmem, stream, (const float *)qn,
                   (const float *)kn, (const float *)lgd, (const float *)beta, conv_out, T, cw);
    if (e != cudaSuccess) return e;
    return launch_pdl(gated_delta_chunk_scan_kernel, dim3(kDv / kRowsScan, kHv), dim3(256), kScanSmemC, stream,
                      state, has_state, (const float *)qn, (const float *)kn, (const float *)cw, T, y);
}

cudaError_t linear_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_linear_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_linear_err, &z, sizeof(DevError));
}

}  // namespace pgc
