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
// q4_linear_kernel is the decode projection, 64 tokens per CTA row of the grid. It is HBM-bound
// on the packed weights (0.5 byte per weight, read once), so what matters is bytes in flight:
// an 8-CTA cluster splits K, every CTA loads its whole slice (64 output rows x in/8 inputs) at
// once, and the slices are summed through distributed shared memory. Each warp owns 8 output
// rows (one n8 tile) and all token tiles, dequantises its B fragments straight from the packed
// words with one OR per pair (bf16 128 + q) and accumulates with bf16 mma.sync in fp32; per
// 64-input group it applies scale and bias algebraically, as the reference's decode kernel
// does (linear.metal:64-123). At 64 tokens each weight feeds 64 FMAs, more than the CUDA cores
// could sustain at HBM speed.
#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {
namespace {

constexpr int kQ4Group = 64;
// A CTA has W warps of 8 output rows each: 64 rows for small batches, 128 above 16 tokens
// (the activation block is re-read once per row tile, so wider tiles cut its L2 traffic).
constexpr int kQ4Tokens = 64;       // token rows per CTA (4 m16 tiles)
constexpr int kQ4Splits = 8;        // K splits = CTAs of a cluster

// Token rows per CTA: the batch rounded up to whole m16 tiles, at most 64.
__host__ __device__ inline int q4_tokens_per_cta(int T) {
    const int r = (T + 15) / 16 * 16;
    return r < kQ4Tokens ? r : kQ4Tokens;
}

// Shared memory of one CTA for a K slice of ks inputs and tp token rows.
template <int W>
struct Q4Layout {
    static constexpr int kRows = 8 * W;
    int xld, wld, x, w, sc, bi, xsum, red, bytes;
    __host__ __device__ Q4Layout(int ks, int tp) {
        xld = ks + 8;      // padded activation row (bf16): conflict-free ldmatrix
        wld = ks / 8 + 4;  // padded packed-word row: a warp's 8 rows fall 4 banks apart
        x = 0;
        w = x + tp * xld * 2;
        sc = w + kRows * wld * 4;
        bi = sc + kRows * (ks / kQ4Group) * 2;
        xsum = (bi + kRows * (ks / kQ4Group) * 2 + 15) & ~15;
        red = xsum + tp * (ks / kQ4Group) * 4;
        bytes = red + tp * kRows * 4;
    }
};

__device__ __forceinline__ void cpa16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
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

// Two nibbles of a packed word (k = 2j, 2j + 1) as a bf16 pair 128 + q: 0x4300 is 128.0 in
// bf16 and its last mantissa bit is worth 1, so OR-ing q in gives 128 + q exactly.
__device__ __forceinline__ uint32_t nib2_bf16(uint32_t word, int j) {
    const uint32_t t = word >> (8 * j);
    return ((t & 0xFu) | ((t & 0xF0u) << 12)) | 0x43004300u;
}

// y[t][o] = sum_k x[t][k] * w[o][k], with the reference decode path's algebra per 64-input
// group: y += scale * sum(q * x) + bias * sum(x). The mma sees the nibbles as bf16 128 + q (exact)
// against the bf16 activations, so it accumulates sum((128 + q) x) exactly in fp32 per group;
// then acc += scale * tmp + (bias - 128 scale) * sum(x). Grid (8 K splits, out_dim / 64,
// ceil(T / 64)); the 8 CTAs of a cluster split K. Each CTA issues every load of its slice at
// once (no loop-carried pipeline: the whole slice in flight), parks its fp32 tile
// [tokens][64 rows] in shared memory, and after a cluster barrier CTA r sums output rows
// [8r, 8r + 8) over the 8 tiles through distributed shared memory, in rank order.
template <int W>
__global__ void __cluster_dims__(kQ4Splits, 1, 1) __launch_bounds__(W * 32)
    q4_linear_kernel(const uint16_t *x, int T, const uint32_t *w, const uint16_t *scales,
                     const uint16_t *biases, uint16_t *y, int out_dim, int in_dim) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) uint8_t q4_smem[];
    const int ks_len = in_dim / kQ4Splits;
    const int tp = q4_tokens_per_cta(T);
    constexpr int kQ4RowsPerCta = 8 * W;
    constexpr int kQ4Warps = W;
    const Q4Layout<W> L(ks_len, tp);
    uint16_t *xs = reinterpret_cast<uint16_t *>(q4_smem + L.x);
    uint32_t *ws_ = reinterpret_cast<uint32_t *>(q4_smem + L.w);
    uint16_t *scs = reinterpret_cast<uint16_t *>(q4_smem + L.sc);
    uint16_t *bis = reinterpret_cast<uint16_t *>(q4_smem + L.bi);
    float *xsum = reinterpret_cast<float *>(q4_smem + L.xsum);
    float *red = reinterpret_cast<float *>(q4_smem + L.red);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x;  // == rank in the cluster
    const int o0 = blockIdx.y * kQ4RowsPerCta;
    const int t0 = blockIdx.z * tp;
    const int nt = min(tp, T - t0);
    const int mtiles = (nt + 15) / 16;
    const int words = in_dim / 8, groups = in_dim / kQ4Group;
    const int k0 = split * ks_len;
    const int wpr = ks_len / 8, gpr = ks_len / kQ4Group;  // words and groups per row in the slice

    for (int i = tid; i < nt * (ks_len / 8); i += kQ4Warps * 32) {
        const int r = i / (ks_len / 8), u = i % (ks_len / 8);
        cpa16(xs + r * L.xld + u * 8, x + (int64_t)(t0 + r) * in_dim + k0 + u * 8);
    }
    for (int i = tid; i < kQ4RowsPerCta * (wpr / 4); i += kQ4Warps * 32) {
        const int r = i / (wpr / 4), u = i % (wpr / 4);
        cpa16(ws_ + r * L.wld + u * 4, w + (int64_t)(o0 + r) * words + k0 / 8 + u * 4);
    }
    for (int i = tid; i < kQ4RowsPerCta * (gpr / 4); i += kQ4Warps * 32) {
        const int r = i / (gpr / 4), u = i % (gpr / 4);
        const int64_t gi = (int64_t)(o0 + r) * groups + k0 / kQ4Group + u * 4;
        cpa8(scs + r * gpr + u * 4, scales + gi);
        cpa8(bis + r * gpr + u * 4, biases + gi);
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // sum(x) of every (token, group) of the slice: a warp per pair, each lane one bf16 pair
    for (int i = warp; i < tp * gpr; i += kQ4Warps) {
        const int r = i / gpr, g = i % gpr;
        float sx = 0.f;
        if (r < nt) {
            const uint32_t v = *reinterpret_cast<const uint32_t *>(xs + r * L.xld + g * kQ4Group + 2 * lane);
            sx = bf16_bits_to_f32(v & 0xFFFFu) + bf16_bits_to_f32(v >> 16);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
        }
        if (lane == 0) xsum[i] = sx;
    }
    __syncthreads();

    float acc[4][4];
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][i] = 0.f;
    const int n_local = warp * 8 + (lane >> 2);  // this thread's B column (output row)
    const int tq = lane & 3;
    const int c0 = warp * 8 + 2 * tq;            // this thread's two C columns (output rows)
    const uint32_t *wrow = ws_ + n_local * L.wld;
    for (int g = 0; g < gpr; ++g) {
        float tmp[4][4];
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i) tmp[m][i] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kQ4Group / 16; ++kk) {
            const int ks = g * (kQ4Group / 16) + kk;
            const uint2 wq = *reinterpret_cast<const uint2 *>(wrow + 2 * ks);  // one 8-byte load
            const uint32_t b0 = nib2_bf16(wq.x, tq), b1 = nib2_bf16(wq.y, tq);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                if (m < mtiles) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(smem_u32(xs + (m * 16 + (lane & 15)) * L.xld + ks * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
                    mma_bf16_16816(tmp[m], a0, a1, a2, a3, b0, b1);
                }
            }
        }
        const float s0 = bf16_bits_to_f32(scs[c0 * gpr + g]), s1 = bf16_bits_to_f32(scs[(c0 + 1) * gpr + g]);
        const float e0 = bf16_bits_to_f32(bis[c0 * gpr + g]) - 128.0f * s0;
        const float e1 = bf16_bits_to_f32(bis[(c0 + 1) * gpr + g]) - 128.0f * s1;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            if (m < mtiles) {
                const int r0 = m * 16 + (lane >> 2);
                const float x0 = xsum[r0 * gpr + g], x1 = xsum[(r0 + 8) * gpr + g];
                acc[m][0] += s0 * tmp[m][0] + e0 * x0;
                acc[m][1] += s1 * tmp[m][1] + e1 * x0;
                acc[m][2] += s0 * tmp[m][2] + e0 * x1;
                acc[m][3] += s1 * tmp[m][3] + e1 * x1;
            }
        }
    }
    // C fragment: tokens lane/4 and lane/4 + 8 of the m tile, rows 2*(lane%4) + {0, 1} of the n8
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        if (m < mtiles) {
            const int r0 = m * 16 + (lane >> 2);
            red[r0 * kQ4RowsPerCta + c0] = acc[m][0];
            red[r0 * kQ4RowsPerCta + c0 + 1] = acc[m][1];
            red[(r0 + 8) * kQ4RowsPerCta + c0] = acc[m][2];
            red[(r0 + 8) * kQ4RowsPerCta + c0 + 1] = acc[m][3];
        }
    }
    q4_cluster_sync();  // every CTA's tile is in its shared memory
    {
        // CTA `split` reduces its eighth of the output rows for all nt tokens
        constexpr int kSlice = kQ4RowsPerCta / kQ4Splits;
        constexpr int kTokPass = kQ4Warps * 32 / kSlice;
        const int rr = tid % kSlice, tk = tid / kSlice;
        const int col = split * kSlice + rr;
        const uint32_t base = smem_u32(red);
        for (int t = tk; t < nt; t += kTokPass) {
            float sum = 0.f;
#pragma unroll
            for (int q = 0; q < kQ4Splits; ++q)
                sum += ld_dsmem(q4_cluster_map(base + (uint32_t)(t * kQ4RowsPerCta + col) * 4, q));
            y[(int64_t)(t0 + t) * out_dim + o0 + col] = f32_to_bf16_bits(sum);
        }
    }
    q4_cluster_sync();  // no CTA leaves while a peer may still read its tile
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

template <int W>
cudaError_t launch_q4_linear_w(const uint16_t *x, int T, const uint32_t *w, const uint16_t *scales,
                               const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                               cudaStream_t stream) {
    const int tp = q4_tokens_per_cta(T);
    const Q4Layout<W> L(in_dim / kQ4Splits, tp);
    static int attr_bytes[64] = {};  // largest dynamic shared memory set per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || attr_bytes[dev] < L.bytes) {
        cudaError_t e = cudaFuncSetAttribute(q4_linear_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, L.bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_bytes[dev] = L.bytes;
    }
    return launch_pdl(q4_linear_kernel<W>, dim3(kQ4Splits, out_dim / (8 * W), (T + tp - 1) / tp), dim3(W * 32),
                      (size_t)L.bytes, stream, x, T, w, scales, biases, y, out_dim, in_dim);
}

cudaError_t launch_q4_linear(const uint16_t *x, int T, const uint32_t *w, const uint16_t *scales,
                             const uint16_t *biases, uint16_t *y, int out_dim, int in_dim,
                             cudaStream_t stream) {
    if (T > 16 && out_dim % 128 == 0)
        return launch_q4_linear_w<16>(x, T, w, scales, biases, y, out_dim, in_dim, stream);
    return launch_q4_linear_w<8>(x, T, w, scales, biases, y, out_dim, in_dim, stream);
}

}  // namespace pgc
