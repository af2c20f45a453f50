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

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Byte offset of element (row, dim) inside a [4 boxes][16 rows][128 B] page tile written by
// TMA with 128-byte swizzling: 16-byte unit index XOR (row mod 8).
__device__ __forceinline__ uint32_t swz_page_offset(int row, int dim) {
    const int box = dim >> 6;
    const int unit = (dim & 63) >> 3;
    return box * 2048 + row * 128 + ((unit ^ (row & 7)) << 4) + ((dim & 7) << 1);
}

}  // namespace pgc
