// pgc_common.cuh — shared device helpers for libperegrine_cuda (sm_100a only).
//
// Fixed Qwen3.5-9B full-attention geometry, bf16 bit helpers with one rounding rule shared
// with the CPU checker, the per-translation-unit device error word, and inline-PTX wrappers
// for mbarriers, TMA tiled loads, ldmatrix and bf16 mma.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libperegrine_cuda targets sm_100a only"
#endif

namespace pgc {

constexpr int kHeadDim = 256;
constexpr int kNumQHeads = 16;
constexpr int kNumKvHeads = 4;
constexpr int kGroup = 4;
constexpr int kPage = 16;
constexpr int kRot = 64;
constexpr int kPartial = kHeadDim + 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device error word. Each translation unit owns one (static, so no relocatable device code is
// needed); kernels record the first fault instead of trapping and the host reads every unit's
// word through pgc_device_error.
struct DevError {
    int code;
    int pad;
    long long detail;
};

enum ErrCode : int {
    kErrNone = 0,
    kErrPageOutOfRange = 1,
    kErrSlotOutOfRange = 2,
    kErrPosOutOfRange = 3,
    kErrWaitTimeout = 4,
    kErrTableOutOfRange = 5,
    kErrSmemAlign = 6,
};

#define PGC_DEFINE_ERROR_WORD(name) static __device__ pgc::DevError name

__device__ __forceinline__ void record_error(DevError *e, int code, long long detail) {
    if (atomicCAS(&e->code, 0, code) == 0) e->detail = detail;
}

// ---------------------------------------------------------------- bf16 bits
// Round-to-nearest-even with quiet-NaN passthrough; identical to the CPU checker's rule.
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
#endif
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---------------------------------------------------------------- shared-memory addressing
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch. A kernel launched with launch_pdl may start while the
// previous kernel in its stream is still running; pdl_wait() blocks until that kernel has
// completed and its memory is visible, so every such kernel calls it before its first global
// memory access (whatever precedes it in the stream). pdl_trigger() lets the next kernel
// launch once every CTA of this grid has started.
#ifndef PGC_NO_PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#else  // build option: plain stream-ordered launches
__device__ __forceinline__ void pdl_wait() {}
__device__ __forceinline__ void pdl_trigger() {}
#endif

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
#ifndef PGC_NO_PDL
    cfg.numAttrs = 1;
#else
    cfg.numAttrs = 0;
#endif
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: gives up after ~2 s (or 2^30 polls) and returns false. Callers record
// kErrWaitTimeout and leave the kernel instead of spinning forever on a shared GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0; i < (1u << 30); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 0 && global_timer_ns() - t0 > 2000000000ull) return false;
    }
    return false;
}

// ---------------------------------------------------------------- TMA (no multicast)
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 2-D tiled TMA load global -> shared, completion signalled on `bar` (complete_tx bytes).
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, int32_t x,
                                            int32_t y, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// ---------------------------------------------------------------- ldmatrix / mma
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One appended row (a q head or a k head, 256 dims) held by a warp, lane l owning dims l + 32 j:
// optional RMSNorm x * (1 / sqrt(mean(x^2) + 1e-6)) * w with the sum in a fixed order, then RoPE
// on the pairs (l, l + 32) of dims [0, 64) with the host's cos/sin row; in decode mode the pair is
// rounded to bf16 first (attention.metal:377,389-396). out[j] is dim l + 32 j as bf16. Every
// step is an explicitly rounded fp32 operation, so the append kernel and the fused decode
// produce the same bits. append_row_compute takes the row already loaded (x and w as floats).
__device__ __forceinline__ void append_row_compute(const float (&x)[8], const float *w, float c, float s,
                                                   bool decode_mode, uint16_t (&out)[8]) {
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = x[j];
    if (w != nullptr) {
        float e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = __fmul_rn(y[j], y[j]);
        const float a0 = __fadd_rn(e[0], e[4]), a1 = __fadd_rn(e[1], e[5]);
        const float a2 = __fadd_rn(e[2], e[6]), a3 = __fadd_rn(e[3], e[7]);
        float ss = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_down_sync(0xffffffffu, ss, o));
        ss = __shfl_sync(0xffffffffu, ss, 0);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 256.0f), 1e-6f)));
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(__fmul_rn(y[j], inv), w[j]);
    }
    float x1 = y[0], x2 = y[1];  // dims lane and lane + 32: one RoPE pair
    if (decode_mode) {
        x1 = bf16_bits_to_f32(f32_to_bf16_bits(x1));
        x2 = bf16_bits_to_f32(f32_to_bf16_bits(x2));
    }
    out[0] = f32_to_bf16_bits(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
    out[1] = f32_to_bf16_bits(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
#pragma unroll
    for (int j = 2; j < 8; ++j) out[j] = f32_to_bf16_bits(y[j]);
}

// The same row with its loads: src and w rows of 256 bf16, rope_row the position's cos | sin.
__device__ __forceinline__ void append_row_warp(const uint16_t *src, const uint16_t *w, const float *rope_row,
                                                bool decode_mode, int lane, uint16_t (&out)[8]) {
    float x[8], wf[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        x[j] = bf16_bits_to_f32(src[lane + 32 * j]);
        wf[j] = w != nullptr ? bf16_bits_to_f32(w[lane + 32 * j]) : 0.f;
    }
    append_row_compute(x, w != nullptr ? wf : nullptr, rope_row[lane], rope_row[32 + lane], decode_mode, out);
}

// Byte offset of element (row, dim) inside a [4 boxes][16 rows][128 B] page tile written by
// TMA with 128-byte swizzling: 16-byte unit index XOR (row mod 8).
__device__ __forceinline__ uint32_t swz_page_offset(int row, int dim) {
    const int box = dim >> 6;
    const int unit = (dim & 63) >> 3;
    return box * 2048 + row * 128 + ((unit ^ (row & 7)) << 4) + ((dim & 7) << 1);
}

}  // namespace pgc
