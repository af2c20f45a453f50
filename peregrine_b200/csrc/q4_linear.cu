// q4_linear.cu — the q4 (group-64 affine) projections around the attention kernels, sm_100a.
//
// Format of shaders/linear.metal:12-20 (MLX's affine quantisation): weight u32 [out][in/8],
// 8 nibbles per word with the low nibble at the lowest input column; scales and biases bf16
// [out][in/64]; w = scale * q + bias.
//
// Two entry points, mirroring the reference's two paths (src/model/linear_q4.zig:77-150,
// src/model/mlx_nt.zig): decode multiplies by the packed weights directly
// (linear_q4_affine_group64_qmv_fast_bf16), prefill dequantises each weight once into a dense
// bf16 matrix (q4_affine_group64_dequantize_bf16, linear.metal:422-444) and runs a dense GEMM.
//
// q4_tc_kernel is the decode projection on the tcgen05 tensor cores: the packed weights are read
// once (0.5 byte per weight) and unpacked in shared memory into the MMA's A operand, the tokens
// are its B operand, and the per-group scale and bias are applied to the fp32 partial sums in
// TMEM as the reference's decode kernel applies them (linear.metal:64-123).
#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {
namespace {

constexpr int kQ4Group = 64;

__device__ __forceinline__ void cp_async16_zfill_q4(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ uint32_t q4_cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void q4_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// q as an exact float without an integer conversion: 2^23 + q has q in the low mantissa bits.
__device__ __forceinline__ float q_f32(uint32_t q) { return __uint_as_float(0x4B000000u | q) - 8388608.0f; }

// q4_affine_group64_dequantize_bf16: thread per packed word -> 8 bf16 (one 16-byte store). The
// product and the sum are each rounded to fp32 and the pair rounded to bf16 by the hardware's
// round-to-nearest-even conversion (all values are finite).
__global__ void __launch_bounds__(256) q4_dequant_kernel(const uint32_t *w, const uint16_t *scales,
                                                         const uint16_t *biases, uint16_t *out,
                                                         int64_t words_total, int in_dim) {
    pdl_trigger();
    pdl_wait();
    const int words = in_dim / 8, groups = in_dim / kQ4Group;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < words_total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = i / words;
        const int kw = (int)(i - o * words);
        const uint32_t p = w[i];
        const int64_t gi = o * groups + (kw * 8) / kQ4Group;
        const float s = bf16_bits_to_f32(scales[gi]), b = bf16_bits_to_f32(biases[gi]);
        uint32_t r[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            r[j] = pack_bf16x2(__fadd_rn(__fmul_rn(s, q_f32((p >> (8 * j)) & 0xFu)), b),
                               __fadd_rn(__fmul_rn(s, q_f32((p >> (8 * j + 4)) & 0xFu)), b));
        *reinterpret_cast<uint4 *>(out + o * in_dim + kw * 8) = make_uint4(r[0], r[1], r[2], r[3]);
    }
}


// Decode projection for 1-2 tokens (the reference's single-sequence GEMV,
// linear_q4_affine_group64_qmv_fast_bf16, linear.metal:64-123) on the CUDA cores: at this batch
// a weight feeds T FMAs, so the kernel is a stream of packed words. Each warp owns 2 (one
// token) or 4 (two tokens) output rows; lane l takes words 4l..4l+3 of every 128-word run of a
// row (16 bytes, half a group), so a warp reads 512 contiguous bytes per row and run, and
// issues the loads of 4 runs before any arithmetic. x and the CTA's scales and biases are
// copied to shared memory once per CTA; x serves the rows of every warp. Per half
// group the lane accumulates sum((128 + q) x) (each nibble as the float 128 + q, exact) and
// sum(x), then adds scale * that + (bias - 128 scale) * sum(x); the lanes' sums meet in a
// butterfly at the end. Each nibble becomes the float 128 + q with one byte permute, and the
// products run as paired fp32 FMAs, so a weight costs about two issue slots at one token.
// Output rows per warp: 2 at one token (more warps in flight: the 8-layer step 0.156 -> 0.134 ms),
// 4 at two tokens (each weight word then feeds more FMAs).
template <int T>
constexpr int gemv_rows() { return T == 1 ? 2 : 4; }
// Byte k of `nibbles` (a nibble in its low 4 bits) as the float 128 + q: the byte lands in bits
// 16-23 under the exponent byte 0x43 (2^7), so q sits in the top mantissa bits, worth 1 each.
__device__ __forceinline__ float q128_f32(uint32_t nibbles, int k) {
    return __uint_as_float(__byte_perm(nibbles, 0x43000000u, 0x7054u | (k << 8)));
}
// Up to PGC_LINEAR_MAX_WEIGHTS weights that share the input (the q | gate, k and v projections)
// run as one launch: their 32-row CTA blocks form one grid.
struct Q4GemvGroups {
    const uint32_t *w[PGC_LINEAR_MAX_WEIGHTS];
    const uint16_t *scales[PGC_LINEAR_MAX_WEIGHTS];
    const uint16_t *biases[PGC_LINEAR_MAX_WEIGHTS];
    uint16_t *y[PGC_LINEAR_MAX_WEIGHTS];
    int out_dim[PGC_LINEAR_MAX_WEIGHTS];
    int block_begin[PGC_LINEAR_MAX_WEIGHTS];  // first CTA of each weight
    int n;
};

template <int T>
__global__ void __launch_bounds__(256) q4_gemv_kernel(const uint16_t *x, const Q4GemvGroups gp, int in_dim) {
    constexpr int kGemvRows = gemv_rows<T>();
    pdl_trigger();
    pdl_wait();
    // this CTA's weight (constant parameter indices only: a dynamically indexed parameter array
    // would be copied to local memory)
    const int b = blockIdx.x;
    const int gi = (gp.n > 1 && b >= gp.block_begin[1]) + (gp.n > 2 && b >= gp.block_begin[2]) +
                   (gp.n > 3 && b >= gp.block_begin[3]);
#define Q4_PICK(field) (gi == 0 ? gp.field[0] : gi == 1 ? gp.field[1] : gi == 2 ? gp.field[2] : gp.field[3])
    const uint32_t *w = Q4_PICK(w);
    const uint16_t *scales = Q4_PICK(scales);
    const uint16_t *biases = Q4_PICK(biases);
    uint16_t *y = Q4_PICK(y);
    const int out_dim = Q4_PICK(out_dim);
    const int block0 = Q4_PICK(block_begin);
#undef Q4_PICK
    // shared memory: x [T][in_dim] bf16, then this CTA's 32 rows of scales and of biases
    // ([32][groups] each, one contiguous block of the [out][groups] arrays)
    extern __shared__ __align__(16) uint16_t gx[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rc = (b - block0) * 8 * kGemvRows;  // first row of the CTA within its weight
    const int r0 = rc + warp * kGemvRows;
    const int words = in_dim / 8, groups = in_dim / kQ4Group;
    const int runs = words / 128;
    uint16_t *gsc = gx + T * in_dim, *gbi = gsc + 8 * kGemvRows * groups;
    // x, scales and biases to shared memory once per CTA; the copies overlap the first batch of
    // weight loads
    for (int i = threadIdx.x; i < T * in_dim / 8; i += 256) cp_async16_zfill_q4(gx + 8 * i, x + 8 * i, true);
    const int nrows = min(8 * kGemvRows, out_dim - rc);
    for (int i = threadIdx.x; i < nrows * groups / 8; i += 256) {
        cp_async16_zfill_q4(gsc + 8 * i, scales + (int64_t)rc * groups + 8 * i, true);
        cp_async16_zfill_q4(gbi + 8 * i, biases + (int64_t)rc * groups + 8 * i, true);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    const bool live = r0 < out_dim;
    float acc[kGemvRows][T];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) acc[r][t] = 0.f;
    // all packed words of kRuns runs in flight before any arithmetic (16 loads of 16 bytes per
    // lane at one token): the stream is latency-bound per warp otherwise
    constexpr int kRuns = 4;
    uint4 wq[kRuns][kGemvRows];
    auto load_batch = [&](int it0) {
#pragma unroll
        for (int j = 0; j < kRuns; ++j)
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r)
                if (live && it0 + j < runs)
                    wq[j][r] = __ldcs(reinterpret_cast<const uint4 *>(w + (int64_t)(r0 + r) * words +
                                                                       (it0 + j) * 128 + lane * 4));
    };
    load_batch(0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (!live) return;
    for (int it0 = 0; it0 < runs; it0 += kRuns) {
        if (it0 > 0) load_batch(it0);
#pragma unroll
        for (int j = 0; j < kRuns; ++j) {
            if (it0 + j >= runs) break;
            const int wo = (it0 + j) * 128 + lane * 4;  // first word of this lane's half group
            const int g = wo / 8;
            float sc[kGemvRows], e[kGemvRows];
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r) {
                const int rl = warp * kGemvRows + r;
                sc[r] = bf16_bits_to_f32(gsc[rl * groups + g]);
                e[r] = bf16_bits_to_f32(gbi[rl * groups + g]) - 128.0f * sc[r];
            }
            // per (row, token): even and odd partial sums of (128 + q) x as one float2; x sums
            float2 tmp[kGemvRows][T], xs[T];
#pragma unroll
            for (int t = 0; t < T; ++t) {
                xs[t] = make_float2(0.f, 0.f);
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) tmp[r][t] = make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                float2 xp[T][4];  // x pairs (2k, 2k + 1) of the word's 8 inputs
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const uint4 xv = *reinterpret_cast<const uint4 *>(gx + t * in_dim + (wo + wd) * 8);
                    const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        xp[t][k] = make_float2(__uint_as_float(xw[k] << 16), __uint_as_float(xw[k] & 0xFFFF0000u));
                        xs[t] = __fadd2_rn(xs[t], xp[t][k]);
                    }
                }
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) {
                    const uint32_t word = wd == 0 ? wq[j][r].x : wd == 1 ? wq[j][r].y : wd == 2 ? wq[j][r].z : wq[j][r].w;
                    const uint32_t lo = word & 0x0F0F0F0Fu, hi = (word >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 wp = make_float2(q128_f32(lo, k), q128_f32(hi, k));
#pragma unroll
                        for (int t = 0; t < T; ++t) tmp[r][t] = __ffma2_rn(wp, xp[t][k], tmp[r][t]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
                for (int t = 0; t < T; ++t)
                    acc[r][t] = fmaf(sc[r], tmp[r][t].x + tmp[r][t].y, fmaf(e[r], xs[t].x + xs[t].y, acc[r][t]));
        }
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) y[(int64_t)t * out_dim + r0 + r] = f32_to_bf16_bits(v);
        }
}

// The four bf16 pairs (128 + q_{2j}, 128 + q_{2j+1}) of a packed word, j = 0..3: the even and
// odd nibbles are split into bytes once, then one byte permute per pair places them in bytes 0
// and 2 (selector nibble 8 = the sign of byte 0 of `lo`, which is 0) and one OR adds 0x4300.
__device__ __forceinline__ void nib_pairs_bf16(uint32_t word, uint32_t (&pr)[4]) {
    const uint32_t lo = word & 0x0F0F0F0Fu, hi = (word >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t r;
        asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(lo), "r"(hi), "r"(0x8480u | (4u + j) << 8 | j));
        pr[j] = r | 0x43004300u;
    }
}

// ------------------------------------------------------------------ tcgen05 pieces (cta_group::1)
__device__ __forceinline__ uint64_t q4_sdesc(uint32_t saddr) {
    // K-major operand, SWIZZLE_128B: 128-byte rows, 8-row atoms of 1024 B (SBO), version 1
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)(16 >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: f32 accumulate, bf16 A and B, both K-major
__host__ __device__ constexpr uint32_t q4_idesc(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void q4_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void q4_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void q4_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void q4_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// N consecutive fp32 columns of this warp's 32 TMEM lanes (thread i: lane quarter*32 + i)
template <int N>
__device__ __forceinline__ void q4_tmem_ld(uint32_t taddr, float *v);
template <>
__device__ __forceinline__ void q4_tmem_ld<8>(uint32_t taddr, float *v) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
template <>
__device__ __forceinline__ void q4_tmem_ld<16>(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
                 "%11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
                   "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

PGC_DEFINE_ERROR_WORD(g_q4_err);

__device__ __forceinline__ bool q4_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int where) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > 2000000000ull || i > (1u << 30)) {
                record_error(&g_q4_err, kErrWaitTimeout, where);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// q4 projection on the 5th-generation tensor cores. y[t][o] = sum_k x[t][k] w[o][k] with the
// reference decode path's algebra per 64-input group g (linear.metal:64-123):
//   y += scale_g * sum_g(q x) + bias_g * sum_g(x).
// The weights are the MMA's A operand (M = 128 output rows per CTA) as bf16 128 + q (exact), the
// tokens its B operand (N = NP, the batch padded to 16, 32 or 64). Per group the tensor cores
// give tmp = sum_g((128 + q) x) in fp32 in TMEM; the epilogue adds scale * tmp + (bias -
// 128 scale) * sum_g(x) to fp32 registers. Grid (S, out / 128, ceil(T / NP)); the S CTAs of a
// cluster split K and their fp32 tiles are summed through distributed shared memory in rank
// order.
// Warps: 0-7 epilogue (warp w reads TMEM lanes 32 (w % 4).. and token half w / 4), 8 MMA issue
// and TMEM owner, 9-16 converters (thread c: output row c % 128, words 4 (c / 128)..+3 of a
// group), 17-18 x sums (token halves), 19 TMA producer. The pipeline moves in steps of two
// groups (a step's waits, proxy fence and commits are paid once per 128 inputs):
//   - W ring: the packed words of 4 groups (2 steps) per slot ([128 rows][128 B], 128-byte
//     swizzle, so a request moves 128 contiguous bytes of a row), 2 slots ahead; the converters
//     release a slot when they have unpacked its last step;
//   - X ring: one step's two x tiles (the MMA's B operands, [NP][64] bf16 swizzled, rows past T
//     read as zero) and their sums per slot; released by the MMA's commit and the epilogue;
//   - bf16 slots: one step's two weight tiles (the MMA's A operands, [128][64] swizzled), 3 or 4
//     of them, so converting step s does not wait on the MMAs of step s - 2;
//   - TMEM: two buffers of a step's two partial-sum tiles [128 lanes][NP].
// Each converter warp unpacks its rows on its own (no barrier across the converters) and issues
// no copies, so the proxy fence that hands its stores to the tensor cores has nothing in flight
// to wait for.
template <int NP>
struct Q4TcCfg {
    static constexpr int kGW = 4;                       // groups per W slot
    static constexpr int kNW = 3;                       // W slots
    static constexpr int kLAW = kNW - 1;                // W slots loaded ahead
    static constexpr int kNX = NP == 64 ? 3 : 4;        // X slots (steps)
    static constexpr int kLAX = kNX - 1;                // steps of x loaded ahead
    static constexpr int kNB = NP == 16 ? 4 : 3;        // bf16 slots (steps)
    static constexpr int kTB = 2;                       // TMEM buffers (steps)
    static constexpr int kXBytes = NP * 128;            // one x tile [NP][64] bf16, swizzled
    static constexpr int kXSum = 2 * kXBytes;           // offset of the x sums [2][NP] in a slot
    static constexpr int kXStride = (2 * kXBytes + 2 * NP * 4 + 1023) / 1024 * 1024;
    static constexpr int kBf = 0;                       // [kNB][2][128][64] bf16
    static constexpr int kW = kBf + kNB * 32768;        // [kNW][128][32] u32
    static constexpr int kX = kW + kNW * 16384;         // [kNX] x slots
    static constexpr int kSc = kX + kNX * kXStride;     // scales, then biases
    static constexpr int kTmemCols = kTB * 2 * NP < 32 ? 32 : kTB * 2 * NP;
    static constexpr int kMaxG = 32;  // groups per CTA slice (scales and biases in shared memory)
    static constexpr int kThreads = 20 * 32;
    static_assert(NP * 128 * 4 <= kNB * 32768, "split-K tile fits in the bf16 slots");
    // scales/biases: [128][G] u16 rows padded to 16 bytes; barriers after them
    __host__ __device__ static int sc_ld(int G) { return G * 2 + 16; }
    __host__ __device__ static int bars(int G) { return kSc + 2 * 128 * sc_ld(G); }
    __host__ __device__ static int bytes(int G) { return bars(G) + 1024; }
};

template <int NP>
__global__ void __launch_bounds__(20 * 32, 1)
    q4_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int T,
                 const uint16_t *scales, const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                 int S) {
    using C = Q4TcCfg<NP>;
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(1024) uint8_t q4_smem[];
    if ((smem_u32(q4_smem) & 1023u) != 0) {
        if (threadIdx.x == 0) record_error(&g_q4_err, kErrSmemAlign, 0);
        return;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x;  // rank in the cluster
    const int o0 = blockIdx.y * 128;
    const int t0 = blockIdx.z * NP;
    const int nt = min(NP, T - t0);
    const int groups = in_dim / kQ4Group;
    const int G = groups / S;  // groups of this CTA's K slice (a multiple of 8)
    const int nsteps = G / 2;
    const int g0 = split * G;
    const int ldsc = C::sc_ld(G);
    uint16_t *scs = reinterpret_cast<uint16_t *>(q4_smem + C::kSc);
    uint16_t *bis = reinterpret_cast<uint16_t *>(q4_smem + C::kSc + 128 * ldsc);
    uint64_t *bar = reinterpret_cast<uint64_t *>(q4_smem + C::bars(G));
    uint64_t *conv_full = bar, *bf_empty = conv_full + C::kNB;
    uint64_t *tmem_full = bf_empty + C::kNB, *tmem_empty = tmem_full + C::kTB;
    uint64_t *w_full = tmem_empty + C::kTB, *w_empty = w_full + C::kNW;
    uint64_t *x_full = w_empty + C::kNW, *x_empty = x_full + C::kNX, *xs_full = x_empty + C::kNX;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xs_full + C::kNX);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(xs_full + C::kNX + 1);
    if (tid == 0) {
        for (int i = 0; i < C::kNB; ++i) {
            mbar_init(&conv_full[i], 8);
            mbar_init(&bf_empty[i], 1);
        }
        for (int i = 0; i < C::kTB; ++i) {
            mbar_init(&tmem_full[i], 1);
            mbar_init(&tmem_empty[i], 8);
        }
        for (int i = 0; i < C::kNW; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 8);
        }
        for (int i = 0; i < C::kNX; ++i) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], 9);
            mbar_init(&xs_full[i], 2);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    q4_tc_fence_before();
    __syncthreads();
    q4_tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t sbase = smem_u32(q4_smem);
    auto x_slot = [&](int st) { return C::kX + (st % C::kNX) * C::kXStride; };

    constexpr int kHalf = NP / 2;                 // tokens per epilogue warp
    constexpr int kCh = kHalf < 16 ? kHalf : 16;  // TMEM columns per load
    float acc[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) acc[i] = 0.f;
    const int q = warp & 3, h = (warp >> 2) & 1;
    const int erow = 32 * q + lane;  // epilogue: output row within the tile

    if (warp < 8) {
        // ------------------------------------------------ epilogue
        {
            // this slice's scales (token half 0) or biases (half 1) of row erow
            const bool ok = o0 + erow < out_dim;
            const uint16_t *src = (h == 0 ? scales : biases) + (int64_t)(o0 + erow) * groups + g0;
            uint8_t *dst = q4_smem + C::kSc + h * 128 * ldsc + erow * ldsc;
            for (int u = 0; u < G / 8; ++u)
                cp_async16_zfill_q4(dst + 16 * u, ok ? src + 8 * u : scales, ok);
            asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
            asm volatile("bar.sync 2, 256;" ::: "memory");
        }
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + h * kHalf;
        for (int st = 0; st < nsteps; ++st) {
            const int b = st % C::kTB;
            if (!q4_wait(&tmem_full[b], (st / C::kTB) & 1, abort_flag, 30)) break;
            if (!q4_wait(&xs_full[st % C::kNX], (st / C::kNX) & 1, abort_flag, 31)) break;
            q4_tc_fence_after();
#pragma unroll
            for (int jg = 0; jg < 2; ++jg) {
                const int g = 2 * st + jg;
                const float sc = bf16_bits_to_f32(scs[erow * (ldsc / 2) + g]);
                const float e = bf16_bits_to_f32(bis[erow * (ldsc / 2) + g]) - 128.0f * sc;
                const float *xs = reinterpret_cast<const float *>(q4_smem + x_slot(st) + C::kXSum) + jg * NP + h * kHalf;
#pragma unroll
                for (int c0 = 0; c0 < kHalf; c0 += kCh) {
                    float tmp[kCh];
                    q4_tmem_ld<kCh>(lane_addr + (b * 2 + jg) * NP + c0, tmp);
#pragma unroll
                    for (int i = 0; i < kCh; i += 4) {
                        const float4 v = *reinterpret_cast<const float4 *>(xs + c0 + i);
                        acc[c0 + i] = fmaf(sc, tmp[i], fmaf(e, v.x, acc[c0 + i]));
                        acc[c0 + i + 1] = fmaf(sc, tmp[i + 1], fmaf(e, v.y, acc[c0 + i + 1]));
                        acc[c0 + i + 2] = fmaf(sc, tmp[i + 2], fmaf(e, v.z, acc[c0 + i + 2]));
                        acc[c0 + i + 3] = fmaf(sc, tmp[i + 3], fmaf(e, v.w, acc[c0 + i + 3]));
                    }
                }
            }
            q4_tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tmem_empty[b]);
                mbar_arrive(&x_empty[st % C::kNX]);
            }
        }
        if (S == 1 && o0 + erow < out_dim) {
#pragma unroll
            for (int i = 0; i < kHalf; ++i) {
                const int t = h * kHalf + i;
                if (t < nt) y[(int64_t)(t0 + t) * out_dim + o0 + erow] = f32_to_bf16_bits(acc[i]);
            }
        }
    } else if (warp == 8) {
        // ------------------------------------------------ MMA issue (one thread)
        int last = -1;
        if (lane == 0) {
            constexpr uint32_t idesc = q4_idesc(128, NP);
            for (int st = 0; st < nsteps; ++st) {
                const int bs = st % C::kNB, b = st % C::kTB, xs = st % C::kNX;
                if (!q4_wait(&conv_full[bs], (st / C::kNB) & 1, abort_flag, 20)) break;
                if (!q4_wait(&x_full[xs], (st / C::kNX) & 1, abort_flag, 22)) break;
                if (!q4_wait(&tmem_empty[b], ((st / C::kTB) & 1) ^ 1, abort_flag, 21)) break;
                q4_tc_fence_after();
#pragma unroll
                for (int jg = 0; jg < 2; ++jg) {
                    const uint32_t a_addr = sbase + C::kBf + bs * 32768 + jg * 16384;
                    const uint32_t x_addr = sbase + x_slot(st) + jg * C::kXBytes;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        q4_mma(tmem + (b * 2 + jg) * NP, q4_sdesc(a_addr + kk * 32), q4_sdesc(x_addr + kk * 32),
                               idesc, kk > 0 ? 1u : 0u);
                }
                q4_commit(&bf_empty[bs]);
                q4_commit(&x_empty[xs]);
                q4_commit(&tmem_full[b]);
                last = st;
            }
            // the tensor cores are done with everything issued before TMEM is released
            if (last >= 0 && *abort_flag) mbar_wait_bounded(&tmem_full[last % C::kTB], (last / C::kTB) & 1);
        }
        __syncwarp();
    } else if (warp < 17) {
        // ------------------------------------------------ converters (each warp on its own)
        const int c = tid - 9 * 32;
        const int row = c & 127, hh = c >> 7;
        for (int st = 0; st < nsteps; ++st) {
            const int bs = st % C::kNB, ws = st / 2;
            bool ok = q4_wait(&w_full[ws % C::kNW], (ws / C::kNW) & 1, abort_flag, 12);
            if (lane == 0 && ok) ok = q4_wait(&bf_empty[bs], ((st / C::kNB) & 1) ^ 1, abort_flag, 10);
            if (__any_sync(0xffffffffu, !ok)) break;
            // group j of the W slot: words 4 hh..4 hh+3 are 16-byte chunk 2 j + hh of the row
            const uint8_t *wrow = q4_smem + C::kW + (ws % C::kNW) * 16384 + row * 128;
            uint4 wq[2];
#pragma unroll
            for (int jg = 0; jg < 2; ++jg) {
                const int j = 2 * (st & 1) + jg;
                wq[jg] = *reinterpret_cast<const uint4 *>(wrow + (((2 * j + hh) ^ (row & 7)) << 4));
            }
#pragma unroll
            for (int jg = 0; jg < 2; ++jg) {
                uint8_t *bf = q4_smem + C::kBf + bs * 32768 + jg * 16384 + row * 128;
                const uint32_t wv[4] = {wq[jg].x, wq[jg].y, wq[jg].z, wq[jg].w};
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int u = 4 * hh + jj;
                    uint32_t pr[4];
                    nib_pairs_bf16(wv[jj], pr);
                    *reinterpret_cast<uint4 *>(bf + ((u ^ (row & 7)) << 4)) = make_uint4(pr[0], pr[1], pr[2], pr[3]);
                }
            }
            fence_proxy_async_smem();  // the bf16 tiles are read by the tensor cores
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&conv_full[bs]);
                if (st & 1) mbar_arrive(&w_empty[ws % C::kNW]);
            }
        }
    } else if (warp < 19) {
        // ------------------------------------------------ x sums: warp 17 + hx, tokens of half hx
        const int hx = warp - 17;
        constexpr int kLpt = 64 / NP;      // lanes per token
        constexpr int kChunks = 8 / kLpt;  // 16-byte chunks per lane
        const int t = hx * kHalf + lane / kLpt, part = lane % kLpt;
        for (int st = 0; st < nsteps; ++st) {
            const bool ok = q4_wait(&x_full[st % C::kNX], (st / C::kNX) & 1, abort_flag, 13);
            if (__any_sync(0xffffffffu, !ok)) break;
            uint8_t *xsl = q4_smem + x_slot(st);
            float sx[2] = {0.f, 0.f};
#pragma unroll
            for (int jg = 0; jg < 2; ++jg)
#pragma unroll
                for (int i = 0; i < kChunks; ++i) {
                    const int u = part * kChunks + i;
                    const uint4 v = *reinterpret_cast<const uint4 *>(xsl + jg * C::kXBytes + t * 128 + ((u ^ (t & 7)) << 4));
                    sx[jg] += (bf16_bits_to_f32(v.x & 0xFFFFu) + bf16_bits_to_f32(v.x >> 16)) +
                              (bf16_bits_to_f32(v.y & 0xFFFFu) + bf16_bits_to_f32(v.y >> 16)) +
                              (bf16_bits_to_f32(v.z & 0xFFFFu) + bf16_bits_to_f32(v.z >> 16)) +
                              (bf16_bits_to_f32(v.w & 0xFFFFu) + bf16_bits_to_f32(v.w >> 16));
                }
#pragma unroll
            for (int jg = 0; jg < 2; ++jg) {
#pragma unroll
                for (int o = kLpt / 2; o > 0; o >>= 1) sx[jg] += __shfl_xor_sync(0xffffffffu, sx[jg], o);
                if (part == 0) reinterpret_cast<float *>(xsl + C::kXSum)[jg * NP + t] = sx[jg];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xs_full[st % C::kNX]);
        }
    } else if (lane == 0) {
        // ------------------------------------------------ TMA producer (one thread)
        tma_prefetch_desc(&tmx);
        tma_prefetch_desc(&tmw);
        const uint64_t pol_w = l2_policy_evict_first(), pol_x = l2_policy_evict_last();
        const int nws = G / C::kGW;  // W slots of the slice
        auto issue_w = [&](int ws) {
            if (ws >= nws) return true;
            const int prev = ws - C::kNW;  // the W slot's previous contents
            if (prev >= 0 && !q4_wait(&w_empty[prev % C::kNW], (prev / C::kNW) & 1, abort_flag, 14)) return false;
            uint64_t *fb = &w_full[ws % C::kNW];
            mbar_arrive_expect_tx(fb, 16384);
            tma_load_2d(q4_smem + C::kW + (ws % C::kNW) * 16384, &tmw, (g0 + ws * C::kGW) * 8, o0, fb, pol_w);
            return true;
        };
        auto issue_x = [&](int st) {
            if (st >= nsteps) return true;
            const int prev = st - C::kNX;
            if (prev >= 0 && !q4_wait(&x_empty[prev % C::kNX], (prev / C::kNX) & 1, abort_flag, 11)) return false;
            uint64_t *fb = &x_full[st % C::kNX];
            mbar_arrive_expect_tx(fb, 2 * C::kXBytes);
            tma_load_2d(q4_smem + x_slot(st), &tmx, (g0 + 2 * st) * kQ4Group, t0, fb, pol_x);
            tma_load_2d(q4_smem + x_slot(st) + C::kXBytes, &tmx, (g0 + 2 * st + 1) * kQ4Group, t0, fb, pol_x);
            return true;
        };
        // W slots are consumed one per two steps, x slots one per step: issue in consumption
        // order, each as soon as its slot is free
        int nw = 0, nx = 0;
        bool ok = true;
        while (ok && (nw < nws || nx < nsteps)) {
            if (nw < nws && (nx >= nsteps || 2 * nw <= nx + 2 * C::kLAW - C::kLAX)) ok = issue_w(nw++);
            else ok = issue_x(nx++);
        }
    }

    if (S > 1) {
        // split-K: every CTA parks its fp32 tile [NP][128] in the (now idle) bf16 slots, then
        // CTA `split` sums rows [split * 128 / S, ...) over the cluster in rank order
        float *red = reinterpret_cast<float *>(q4_smem + C::kBf);
        if (warp < 8) {
#pragma unroll
            for (int i = 0; i < kHalf; ++i) red[(h * kHalf + i) * 128 + erow] = acc[i];
        }
        q4_cluster_sync();
        const int rows = 128 / S;
        const uint32_t base = smem_u32(red);
        for (int i = tid; i < rows * nt; i += C::kThreads) {
            const int t = i / rows, r = split * rows + i % rows;
            if (o0 + r >= out_dim) continue;
            float sum = 0.f;
            for (int qq = 0; qq < S; ++qq) sum += ld_dsmem(q4_cluster_map(base + (uint32_t)(t * 128 + r) * 4, qq));
            y[(int64_t)(t0 + t) * out_dim + o0 + r] = f32_to_bf16_bits(sum);
        }
        q4_cluster_sync();  // no CTA leaves while a peer may still read its tile
    }
    q4_tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        q4_tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols)
                     : "memory");
    }
}

}  // namespace

cudaError_t launch_q4_dequantize(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                                 uint16_t *out, int out_dim, int in_dim, cudaStream_t stream) {
    const int64_t words = (int64_t)out_dim * (in_dim / 8);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t blocks = (words + 255) / 256;
    if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
    return launch_pdl(q4_dequant_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, w, scales, biases, out,
                      words, in_dim);
}

// K splits: the smallest S in {1, 2, 4, 8} that gives ~0.8 of a wave of CTAs, keeping each
// CTA's slice a whole number of 8-group units (16-byte scale and bias copies).
static int q4_splits(int tiles, int groups, int sms, int max_g) {
    int S = 1;
    while (groups / S > max_g) S *= 2;
    while (S < 8 && tiles * S < sms * 4 / 5 && (groups / (2 * S)) % 8 == 0 && groups % (2 * S) == 0) S *= 2;
    return S;
}

template <int NP>
static cudaError_t launch_q4_tc(const CUtensorMap &tx, const CUtensorMap &tw, int T, const uint16_t *scales,
                                const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                                cudaStream_t stream) {
    using C = Q4TcCfg<NP>;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int groups = in_dim / kQ4Group;
    const int row_tiles = (out_dim + 127) / 128, tok_tiles = (T + NP - 1) / NP;
    const int S = q4_splits(row_tiles * tok_tiles, groups, sms, C::kMaxG);
    const int bytes = C::bytes(groups / S);
    static std::atomic<int> attr_bytes[64] = {};
    if (dev < 0 || dev >= 64 || attr_bytes[dev] < bytes) {
        cudaError_t e = cudaFuncSetAttribute(q4_tc_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_bytes[dev] = bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, row_tiles, tok_tiles);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
#ifndef PGC_NO_PDL
    cfg.numAttrs = 2;
#else
    cfg.numAttrs = 1;
#endif
    return cudaLaunchKernelEx(&cfg, q4_tc_kernel<NP>, tx, tw, T, scales, biases, y, out_dim, in_dim, S);
}

cudaError_t launch_q4_linear(const CUtensorMap &tx, const CUtensorMap &tw, int T, const uint16_t *scales,
                             const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                             cudaStream_t stream) {
    switch (q4_token_tile(T)) {
        case 16: return launch_q4_tc<16>(tx, tw, T, scales, biases, y, out_dim, in_dim, stream);
        case 32: return launch_q4_tc<32>(tx, tw, T, scales, biases, y, out_dim, in_dim, stream);
        default: return launch_q4_tc<64>(tx, tw, T, scales, biases, y, out_dim, in_dim, stream);
    }
}

cudaError_t launch_q4_gemv(const uint16_t *x, int T, const Q4Weight *ws, int n, int in_dim, cudaStream_t stream) {
    if (T < 1 || T > kQ4GemvMaxTokens || n < 1 || n > PGC_LINEAR_MAX_WEIGHTS) return cudaErrorInvalidValue;
    const int cta_rows = 8 * (T == 1 ? gemv_rows<1>() : gemv_rows<2>());
    Q4GemvGroups gp = {};
    int blocks = 0;
    for (int i = 0; i < n; ++i) {
        gp.w[i] = ws[i].w;
        gp.scales[i] = ws[i].scales;
        gp.biases[i] = ws[i].biases;
        gp.y[i] = ws[i].y;
        gp.out_dim[i] = ws[i].out_dim;
        gp.block_begin[i] = blocks;
        blocks += (ws[i].out_dim + cta_rows - 1) / cta_rows;
    }
    gp.n = n;
    const dim3 grid((unsigned)blocks);
    const size_t smem = ((size_t)T * in_dim + 2 * cta_rows * (in_dim / kQ4Group)) * 2;
    static std::atomic<bool> attr_set[64][kQ4GemvMaxTokens] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    auto go = [&](auto kernel) {
        if (dev < 0 || dev >= 64 || !attr_set[dev][T - 1]) {
            // largest: T tokens of 8192 inputs + 2 x 32 rows of 128 groups
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (T * 8192 + 2 * cta_rows * 128) * 2);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) attr_set[dev][T - 1] = true;
        }
        return launch_pdl(kernel, grid, dim3(256), smem, stream, x, gp, in_dim);
    };
    switch (T) {
        case 1: return go(q4_gemv_kernel<1>);
        case 2: return go(q4_gemv_kernel<2>);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t q4_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_q4_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_q4_err, &z, sizeof(DevError));
}

}  // namespace pgc
