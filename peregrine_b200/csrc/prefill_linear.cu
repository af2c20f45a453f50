// prefill_linear.cu — dense bf16 projections of a prefill chunk on the 5th-gen tensor cores
// (tcgen05.mma cta_group::2, accumulators in TMEM, operands staged by TMA), sm_100a.
//
// The reference's prefill projections dequantise each q4 weight once into a dense bf16 matrix
// (q4_affine_group64_dequantize_bf16, shaders/linear.metal:422-444; pgc_q4_dequantize here) and
// multiply the chunk's rows by it with an NT GEMM (src/model/block_attn.zig:96-108,
// src/model/mlx_nt.zig; MLX steel GEMM, shaders/mlx_gemm.metal): y[t][o] = sum_k x[t][k] w[o][k],
// fp32 accumulation, bf16 output. This kernel is that GEMM.
//
// Design: a persistent grid of CTA pairs (clusters of two, one pair per two SMs). A pair owns a
// 256 x 256 output tile at a time: each CTA stages 128 rows of x and 128 rows of w per 64-wide
// K block (two 16 KiB TMA boxes, 128-byte swizzle) into a 6-stage ring, the pair leader issues
// M256 N256 K16 MMAs that read both CTAs' halves, and each CTA's TMEM holds its 128 rows x 256
// fp32 columns. TMEM holds two accumulators, so the epilogue of tile i (TMEM -> registers ->
// bf16 -> global) overlaps the MMAs of tile i + 1. Up to four weights that share the input
// (the q | gate, k and v projections) are one launch: the tiles of all of them form one queue.
//
// Per CTA: warp 0 TMA producer, warp 1 MMA issuer (leader only), warps 2-5 epilogue (one TMEM
// lane quarter each).
#include <cuda.h>

#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_plin_err);

namespace {

constexpr int kTileM = 256;   // rows of x per pair tile (128 per CTA)
constexpr int kTileN = 256;   // rows of w per pair tile (128 per CTA)
constexpr int kBlockK = 64;   // one 128-byte swizzle row of bf16
constexpr int kStages = 6;
constexpr int kHalfBytes = 128 * kBlockK * 2;      // 16 KiB: one CTA's half of A or of B
constexpr int kStageBytes = 2 * kHalfBytes;
constexpr uint32_t kTmemCols = 512;                // two 256-column accumulators
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps);

struct Smem {
    static constexpr int kRing = 0;
    static constexpr int kBar = kRing + kStages * kStageBytes;
    // full[kStages] (leader), empty[kStages], tfull[2], tempty[2] (leader)
    static constexpr int kNumBars = 2 * kStages + 4;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kAbort = kTmemSlot + 8;
    static constexpr int kBytes = kAbort + 8;
};
constexpr int kSmemBytes = Smem::kBytes + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "prefill projection shared memory exceeds the sm_100 limit");

__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    // K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO);
    // start >> 4 [0,14), LBO >> 4 [16,30) (unused for swizzled K-major), SBO >> 4 [32,46),
    // version 1 [46,48), layout SWIZZLE_128B (2) [61,64).
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)(16 >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 D, bf16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void pair_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void arrive_expect_tx_remote(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait (~2 s), cluster-scope acquire. Gives up early once another role of this CTA has
// timed out; records the first timeout with the waiting role in the detail.
__device__ __forceinline__ bool wait_bounded(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int where) {
    if (try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (try_wait_cluster(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > 2000000000ull || i > (1u << 30)) {
                record_error(&g_plin_err, kErrWaitTimeout, where);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// 2-D TMA load into this CTA's shared memory, bytes counted on the pair leader's barrier.
__device__ __forceinline__ void tma_load_pair(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                              uint32_t bar_leader, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_leader), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// Completion of the leader's earlier MMAs arrives on the barrier at this offset in both CTAs.
__device__ __forceinline__ void commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"((uint16_t)3)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

struct LinGroup {
    uint16_t *y;      // [T][out_dim] bf16
    int out_dim;
    int tile_begin;   // first tile of this weight in the launch's queue
};

struct LinParams {
    int T, in_dim, m_tiles, k_blocks, n_groups, total_tiles;
    LinGroup g[PGC_LINEAR_MAX_WEIGHTS];
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    prefill_linear_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw0,
                          const __grid_constant__ CUtensorMap tw1, const __grid_constant__ CUtensorMap tw2,
                          const __grid_constant__ CUtensorMap tw3, const LinParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    pdl_trigger();
    const uint32_t rank = cta_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem::kBar);
    uint64_t *full = bars;                 // leader: both CTAs' bytes of a stage
    uint64_t *empty = full + kStages;      // each: the stage's MMAs are done
    uint64_t *tfull = empty + kStages;     // each [2]: an accumulator is complete
    uint64_t *tempty = tfull + 2;          // leader [2]: both CTAs' epilogues drained it
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Smem::kTmemSlot);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Smem::kAbort);
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 2);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * kEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before();
    pair_sync();  // barriers and TMEM of both CTAs are ready
    fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // x may be the previous kernel's output

    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int n_local = pair < p.total_tiles ? (p.total_tiles - 1 - pair) / n_pairs + 1 : 0;
    // tile -> (weight, row tile, column tile); row tiles vary fastest so that the pairs running
    // at once share the weight tiles they read
    // (constant indices only: a dynamically indexed parameter array would be copied to local
    // memory)
    auto tile_coords = [&](int t, int &g, int &m0, int &n0) {
        g = (p.n_groups > 1 && t >= p.g[1].tile_begin) + (p.n_groups > 2 && t >= p.g[2].tile_begin) +
            (p.n_groups > 3 && t >= p.g[3].tile_begin);
        const int begin = g == 0 ? 0 : g == 1 ? p.g[1].tile_begin : g == 2 ? p.g[2].tile_begin : p.g[3].tile_begin;
        const int local = t - begin;
        m0 = (local % p.m_tiles) * kTileM;
        n0 = (local / p.m_tiles) * kTileN;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            tma_prefetch_desc(&tx);
            const uint64_t pol_x = l2_policy_evict_last();   // x is re-read by every column tile
            const uint64_t pol_w = l2_policy_evict_normal();
            const uint32_t full0 = map_to_rank(smem_u32(&full[0]), 0);
            int it = 0;
            for (int lt = 0; lt < n_local; ++lt) {
                int g, m0, n0;
                tile_coords(pair + lt * n_pairs, g, m0, n0);
                const CUtensorMap *tw = g == 0 ? &tw0 : g == 1 ? &tw1 : g == 2 ? &tw2 : &tw3;
                for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !wait_bounded(&empty[s], ((it / kStages) - 1) & 1, abort_flag, 1)) {
                        lt = n_local;
                        break;
                    }
                    uint8_t *st = smem + Smem::kRing + s * kStageBytes;
                    const uint32_t fb = full0 + s * 8;
                    arrive_expect_tx_remote(fb, kStageBytes);
                    tma_load_pair(st, &tx, kb * kBlockK, m0 + (int)rank * 128, fb, pol_x);
                    tma_load_pair(st + kHalfBytes, tw, kb * kBlockK, n0 + (int)rank * 128, fb, pol_w);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (pair leader)
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kTileM, kTileN);
            int it = 0;
            bool ok = true;
            for (int lt = 0; ok && lt < n_local; ++lt) {
                const int b = lt & 1;
                if (lt >= 2 && !wait_bounded(&tempty[b], ((lt >> 1) - 1) & 1, abort_flag, 2)) break;
                fence_after();
                const uint32_t d = tmem + b * kTileN;
                for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!wait_bounded(&full[s], (it / kStages) & 1, abort_flag, 3)) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint32_t a_addr = smem_u32(smem + Smem::kRing + s * kStageBytes);
                    const uint32_t b_addr = a_addr + kHalfBytes;
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 16; ++kk)
                        mma_pair(d, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), idesc,
                                 (kb > 0 || kk > 0) ? 1u : 0u);
                    commit_pair(&empty[s]);  // the stage may be refilled in both CTAs
                }
                if (ok) commit_pair(&tfull[b]);  // the accumulator is complete in both CTAs
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // warp w reads TMEM lanes 32 * (w % 4) .. +31: rows of this CTA's 128-row half
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        const uint32_t tempty0 = map_to_rank(smem_u32(&tempty[0]), 0);
        for (int lt = 0; lt < n_local; ++lt) {
            const int b = lt & 1;
            if (!wait_bounded(&tfull[b], (lt >> 1) & 1, abort_flag, 4)) break;
            fence_after();
            int g, m0, n0;
            tile_coords(pair + lt * n_pairs, g, m0, n0);
            const int row = m0 + (int)rank * 128 + q * 32 + lane;
            const int out_dim = g == 0 ? p.g[0].out_dim : g == 1 ? p.g[1].out_dim : g == 2 ? p.g[2].out_dim : p.g[3].out_dim;
            uint16_t *ybase = g == 0 ? p.g[0].y : g == 1 ? p.g[1].y : g == 2 ? p.g[2].y : p.g[3].y;
            uint16_t *yrow = ybase + (int64_t)row * out_dim;
#pragma unroll 1
            for (int c = 0; c < kTileN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32cols(tmem + lane_base + b * kTileN + c * 32, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int col = n0 + c * 32;
                if (row < p.T) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        if (col + i + 8 <= out_dim) {
                            uint4 o;
                            o.x = pack_bf16x2(__uint_as_float(v[i]), __uint_as_float(v[i + 1]));
                            o.y = pack_bf16x2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
                            o.z = pack_bf16x2(__uint_as_float(v[i + 4]), __uint_as_float(v[i + 5]));
                            o.w = pack_bf16x2(__uint_as_float(v[i + 6]), __uint_as_float(v[i + 7]));
                            *reinterpret_cast<uint4 *>(yrow + col + i) = o;
                        }
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) arrive_remote(tempty0 + b * 8);  // the leader may reuse accumulator b
        }
    }
    // no CTA frees TMEM or leaves while the pair's MMAs or the peer may still use it
    fence_before();
    pair_sync();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

}  // namespace

cudaError_t launch_prefill_linear(const CUtensorMap &tx, const CUtensorMap *tw, const LinearOut *outs,
                                  int n_weights, int T, int in_dim, int sm_count, cudaStream_t stream) {
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    LinParams lp = {};
    lp.T = T;
    lp.in_dim = in_dim;
    lp.m_tiles = (T + kTileM - 1) / kTileM;
    lp.k_blocks = in_dim / kBlockK;
    lp.n_groups = n_weights;
    int tiles = 0;
    for (int g = 0; g < n_weights; ++g) {
        lp.g[g].y = outs[g].y;
        lp.g[g].out_dim = outs[g].out_dim;
        lp.g[g].tile_begin = tiles;
        tiles += lp.m_tiles * ((outs[g].out_dim + kTileN - 1) / kTileN);
    }
    lp.total_tiles = tiles;
    if (tiles == 0) return cudaSuccess;
    int pairs = sm_count / 2;
    if (pairs > tiles) pairs = tiles;
    if (pairs < 1) pairs = 1;
    const CUtensorMap &w1 = n_weights > 1 ? tw[1] : tw[0];
    const CUtensorMap &w2 = n_weights > 2 ? tw[2] : tw[0];
    const CUtensorMap &w3 = n_weights > 3 ? tw[3] : tw[0];
    return launch_pdl(prefill_linear_kernel, dim3(2 * pairs), dim3(kThreads), kSmemBytes, stream, tx, tw[0], w1,
                      w2, w3, lp);
}

cudaError_t prefill_linear_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_plin_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_plin_err, &z, sizeof(DevError));
}

}  // namespace pgc
