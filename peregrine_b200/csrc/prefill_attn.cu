// prefill_attn.cu — chunked-prefill causal GQA attention over prefix + chunk on the 5th-gen
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA) for sm_100a.
//
// Behaviour follows the reference's prefix-aware prefill chain
// (prefill_score_prefix_head_major_bf16 -> prefill_softmax_bf16 ->
// prefill_value_prefix_head_major_value_dim_major_bf16, shaders/attention.metal:1204-1964,
// dispatched at src/model/block_attn.zig:633-703): query t of a `tokens`-row chunk sees cache
// columns c <= (n - tokens) + t (attention.metal:1347-1353), with scale 1/16. The reference
// materialises S and P in bf16 per kv head; here they never leave the SM: S lives in TMEM, P
// in shared memory, and the softmax is online (fp32), so only Q, K, V and O touch HBM.
//
// Two-SM design (tcgen05 cta_group::2): a cluster of two CTAs runs one kv head for two adjacent
// 32-token query tiles. The 4 GQA heads of the kv head are stacked into each CTA's 128 rows
// (row r = token r/4, head r%4), so the pair's MMAs have M = 256 and every K/V tile serves 64
// tokens x 4 heads. The leader CTA issues S = Q K^T (M256 N128 K256) and O += P V (M256 N256
// K128) for both; each CTA stages its own Q, 64 of the tile's 128 keys and 128 of the 256 value
// dims, so each SM fetches half of every K/V tile. Per CTA (672 threads): warps 0-15 softmax +
// epilogue (four warps per TMEM lane quarter, splitting key columns and O dims), warp 16 the MMA
// issuer (leader only), warps 17-18 the Q/K TMA producers, warps 19-20 the V producers. TMEM: O in columns
// [0,256), two S tiles in [256,512); P(j) is written over the first 64 columns of S(j).
#include <cuda.h>

#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_prefill_err);

namespace {

constexpr int kBM = 128;           // rows = 32 tokens x 4 heads
constexpr int kTokTile = 32;
constexpr uint32_t kTmemCols = 512;
constexpr float kLazyRescale = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

struct PrefillParams {
    const int32_t *block_table;
    const uint16_t *v_pages;  // V pool (the pair kernel copies a partial final page directly)
    uint16_t *out;
    float *ws;  // nsplit > 1: partials [nsplit][chunk_len * 16][258] (m natural log, l, o)
    int64_t num_pages;
    int prefix_len;
    int chunk_len;
    int nsplit;
    float scale_log2;
};

// ---------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // sm_100 shared-memory matrix descriptor: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46),
    // version 1 at [46,48), layout SWIZZLE_128B (2) at [61,64).
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
           ((uint64_t)(sbo >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: f32 accumulate, bf16 A and B.
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
           ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 columns of fp32: thread i of the warp gets lane (quarter*32 + i), 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
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
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
          "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])),
          "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
          "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
          "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
          "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
          "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
          "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
          "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
          "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
          "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// Bounded wait that also gives up as soon as another role of the CTA has recorded a timeout.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              int where) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > 2000000000ull || i > (1u << 30)) {
                record_error(&g_prefill_err, kErrWaitTimeout, where);
#ifndef PGC_PREFILL_NO_ABORT
                *abort_flag = 1;
#endif
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- two-SM (cta_group::2) helpers
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
          "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]),
          "r"(v[14]), "r"(v[15])
        : "memory");
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    // non-.aligned forms: producer and MMA warps arrive with diverged lanes
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Arrive (with transaction bytes) on an mbarrier that may live in another CTA of the cluster.
// The release is CTA-scoped: what an arrival publishes was produced and ordered inside this CTA
// (TMA bytes are counted by the barrier itself; P in TMEM is ordered by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync). A cluster-scoped release measured ~1400 cycles per
// arrival here, on the critical path of every tile.
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t bar_cluster, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;"
                 ::"r"(bar_cluster), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
                 : "memory");
}

// Waits with acquire at cluster scope (the barrier is signalled from the peer CTA too).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
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

// 2-D tiled TMA load into this CTA's shared memory whose completion bytes are counted on the
// pair leader's mbarrier (`bar_leader`: a shared::cluster address in CTA 0).
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap, int32_t x,
                                                 int32_t y, uint32_t bar_leader, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_leader), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void *smem_dst, const void *tmap, int32_t x,
                                                 int32_t y, int32_t z, uint32_t bar_leader) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar_leader)
        : "memory");
}

__device__ __forceinline__ void umma2_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma2_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Completion of this thread's earlier pair MMAs arrives once on the mbarrier at this shared
// offset in BOTH CTAs of the pair (commit arrive with CTA mask 0b11; an mbarrier signal, not a
// data load).
__device__ __forceinline__ void umma2_commit_pair(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"((uint16_t)3)
        : "memory");
}

// Bounded wait with cluster-scope acquire, for barriers that the peer CTA arrives on.
__device__ __forceinline__ bool wait_or_abort_cluster(uint64_t *bar, uint32_t parity,
                                                      volatile int *abort_flag, int where) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > 2000000000ull || i > (1u << 30)) {
                record_error(&g_prefill_err, kErrWaitTimeout, where);
#ifndef PGC_PREFILL_NO_ABORT
                *abort_flag = 1;
#endif
                return false;
            }
        }
    }
}

// =============================================================================================
// Two-SM prefill (tcgen05 cta_group::2). A cluster of two CTAs runs one kv head for two adjacent
// 32-token query tiles: M = 256 rows (each CTA's 128 rows = its 32 tokens x 4 heads). Every
// MMA is issued by the pair leader (cluster rank 0) and reads each CTA's half of both operands
// from that CTA's shared memory or TMEM: for S = Q K^T (M256 N128) each CTA stages its own Q and
// 64 of the tile's 128 keys; for O += P V (M256 N256) each CTA holds its P rows in TMEM and 128
// of the 256 value dims. Each SM therefore fetches half of every K/V tile that a one-SM CTA
// would, for the same tensor work.
// =============================================================================================
namespace pair {

constexpr int kSoftmaxWarps = 16;
// warps 0-15 softmax, 16 MMA, 17-18 K (+Q) TMA, 19-20 V TMA. TMA boxes here are one page high
// (2 KiB); an SM retires them roughly twice as fast when two warps issue in parallel, so each
// operand has two producer warps.
constexpr int kProducerWarps = 2;
constexpr int kThreads = 32 * (kSoftmaxWarps + 1 + 2 * kProducerWarps);
constexpr int kBNp = 128;             // keys per tile
constexpr int kQBytesP = kBM * kHeadDim * 2;      // [4 dim blocks][128 rows][128 B] = 64 KiB
constexpr int kKHalf = 64 * kHeadDim * 2;         // this CTA's 64 keys: [4][64][128 B] = 32 KiB
constexpr int kVHalf = kBNp * 128 * 2;            // this CTA's 128 dims: [2][128][128 B] = 32 KiB
constexpr int kKSlotsP = 3;
constexpr int kVSlotsP = 2;
constexpr uint32_t kTO = 0;           // O: 256 columns
constexpr uint32_t kTS = 256;         // S tiles: 2 x 128 columns; P(j) over the first 64 of S(j)

struct Smem2 {
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kQBytesP;
    static constexpr int kV = kK + kKSlotsP * kKHalf;
    static constexpr int kBar = kV + kVSlotsP * kVHalf;
    // leader-side: q_full, k_full[3], v_full[2], p_full[2]; both sides: k_empty[3],
    // v_empty[2], s_full[2], pv_done[2]
    static constexpr int kNumBars = 1 + kKSlotsP + kVSlotsP + 2 + kKSlotsP + kVSlotsP + 2 + 2;
    static constexpr int kRed = kBar + kNumBars * 8;
    static constexpr int kTmemSlot = kRed + 4 * kBM * 4;  // red: [4 key quarters][128 rows] fp32
    static constexpr int kAbort = kTmemSlot + 8;
    static constexpr int kBytes = kTmemSlot + 16;
};
static_assert(Smem2::kBytes <= 232448, "pair prefill shared memory exceeds the sm_100 limit");

}  // namespace pair

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::kThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const PrefillParams p) {
    using namespace pair;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    // The two CTAs of a pair must agree on the layout; a misaligned window would break it, and
    // both CTAs see the same alignment, so both leave together.
    if ((smem_u32(smem) & 1023u) != 0) {
        if (threadIdx.x == 0) record_error(&g_prefill_err, kErrSmemAlign, 0);
        return;
    }

    const int qt = blockIdx.x;  // this CTA's 32-token tile; the pair is (2c, 2c+1)
    const int kvh = blockIdx.y;
    const int T = p.chunk_len, P = p.prefix_len;
    const int tok0 = qt * kTokTile;
    const int pair_last = min(((qt >> 1) << 1) * kTokTile + 2 * kTokTile - 1, T - 1);
    const int n_keys = P + pair_last + 1;  // keys any row of the pair may see
    const int n_tiles = (n_keys + kBNp - 1) / kBNp;
    const int total_keys = P + T;
    const int tb = (int)((int64_t)n_tiles * blockIdx.z / p.nsplit);
    const int n_loc = (int)((int64_t)n_tiles * (blockIdx.z + 1) / p.nsplit) - tb;

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Smem2::kBar);
    uint64_t *q_full = bars;                       // leader: both CTAs' Q bytes
    uint64_t *k_full = q_full + 1;                 // leader [3]: both CTAs' K halves
    uint64_t *v_full = k_full + kKSlotsP;          // leader [2]: both CTAs' V halves
    uint64_t *p_full = v_full + kVSlotsP;          // leader [2]: both CTAs' softmax warps
    uint64_t *k_empty = p_full + 2;                // each [3]
    uint64_t *v_empty = k_empty + kKSlotsP;        // each [2]
    uint64_t *s_full = v_empty + kVSlotsP;         // each [2]
    uint64_t *pv_done = s_full + 2;                // each [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Smem2::kTmemSlot);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + Smem2::kAbort);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        mbar_init(q_full, 2);
        for (int s = 0; s < kKSlotsP; ++s) {
            mbar_init(&k_full[s], 2 * kProducerWarps);  // leader: both CTAs' K producers
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < kVSlotsP; ++s) {
            mbar_init(&v_full[s], 2 * kProducerWarps);  // leader: both CTAs' V producers
            mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&p_full[b], 2 * kSoftmaxWarps);
            mbar_init(&s_full[b], 1);
            mbar_init(&pv_done[b], 1);
        }
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers are initialised before anyone signals them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto leader_addr = [&](uint64_t *bar) { return cluster_map(smem_u32(bar), 0); };

    if (warp >= kSoftmaxWarps + 1 && warp < kSoftmaxWarps + 1 + kProducerWarps) {
        // ------------------------------------------------------------ TMA: Q and this CTA's K half
        // producer kw loads pages {2kw, 2kw+1} of this CTA's 64 keys (4 boxes of 64 dims each)
        const int kw = warp - (kSoftmaxWarps + 1);
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_last();
            if (kw == 0) {
                tma_prefetch_desc(&tmq);
                tma_prefetch_desc(&tmk);
                const uint32_t qbar = leader_addr(q_full);
                mbar_arrive_expect_tx_cluster(qbar, kQBytesP);
                for (int c = 0; c < 4; ++c)
                    tma_load_3d_pair(smem + Smem2::kQ + c * (kBM * 128), &tmq, c * 64, kvh * kGroup, tok0, qbar);
            }
            for (int j = 0; j < n_loc; ++j) {
                const int sl = j % kKSlotsP;
                if (j >= kKSlotsP &&
                    !wait_or_abort(&k_empty[sl], ((j / kKSlotsP) - 1) & 1, abort_flag, 1))
                    break;
                const int key0 = (tb + j) * kBNp + (int)rank * 64;  // this CTA's 64 keys
                int npg = 0;
                for (int pp = 2 * kw; pp < 2 * kw + 2; ++pp)
                    if (key0 + pp * kPage < total_keys) ++npg;
                const uint32_t kbar = leader_addr(&k_full[sl]);
                mbar_arrive_expect_tx_cluster(kbar, (uint32_t)npg * 4 * 2048);
                uint8_t *dst = smem + Smem2::kK + sl * kKHalf;
                for (int pp = 2 * kw; pp < 2 * kw + npg; ++pp) {
                    int page = p.block_table[(key0 >> 4) + pp];
                    if (page < 0 || page >= p.num_pages) {
                        record_error(&g_prefill_err, kErrPageOutOfRange, page);
                        page = 0;
                    }
                    const int row = (page * kNumKvHeads + kvh) * kPage;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tma_load_2d_pair(dst + c * (64 * 128) + pp * 2048, &tmk, c * 64, row, kbar, pol);
                }
            }
        }
    } else if (warp >= kSoftmaxWarps + 1 + kProducerWarps) {
        // ------------------------------------------------------------ TMA: this CTA's V half
        // (value dims [128 * rank, +128) of all 128 keys), counted on the leader's barrier like
        // K. Producer vw owns keys [64 vw, +64) (pages 4vw..4vw+3). Rows past the cache end are
        // zeroed here and a partial final page is copied row by row by the whole warp, so no
        // stale slot (possibly a NaN pattern) meets a zero probability in P.V, and the softmax
        // warps never wait on V.
        const int vw = warp - (kSoftmaxWarps + 1 + kProducerWarps);
        const int r0 = vw * 64, r1 = r0 + 64;  // this producer's key rows of the tile
        {
            if (lane == 0 && vw == 0) tma_prefetch_desc(&tmv);
            const uint64_t pol = l2_policy_evict_last();
            for (int j = 0; j < n_loc; ++j) {
                const int sl = j % kVSlotsP;
                bool go = true;
                if (lane == 0 && j >= kVSlotsP)
                    go = wait_or_abort(&v_empty[sl], ((j / kVSlotsP) - 1) & 1, abort_flag, 11);
                if (!__shfl_sync(0xffffffffu, go ? 1 : 0, 0)) break;
                const int key0 = (tb + j) * kBNp;
                const int valid = min(kBNp, total_keys - key0);  // keys of this tile in the cache
                const int full_pages = valid / kPage;            // loaded by TMA
                uint8_t *dst = smem + Smem2::kV + sl * kVHalf;
                const int first = max(full_pages * kPage, r0);   // first row not loaded by TMA
                if (first < r1) {
                    // rows [first, r1): zero, then copy the partial page's valid rows
                    for (int i = lane; i < (r1 - first) * 2 * 8; i += 32) {
                        const int row = first + i / 16;
                        const int u = i % 16;
                        *reinterpret_cast<uint4 *>(dst + (u >> 3) * (kBNp * 128) + row * 128 + (u & 7) * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                    __syncwarp();
                    const int tail = valid - full_pages * kPage;  // valid rows in the partial page
                    if (tail > 0 && full_pages * kPage >= r0 && full_pages * kPage < r1) {
                        int page = p.block_table[(key0 >> 4) + full_pages];
                        if (page < 0 || page >= p.num_pages) {
                            if (lane == 0) record_error(&g_prefill_err, kErrPageOutOfRange, page);
                            page = 0;
                        }
                        const uint16_t *src = p.v_pages + ((int64_t)(page * kNumKvHeads + kvh) * kPage) * kHeadDim;
                        for (int i = lane; i < tail * 2 * 8; i += 32) {
                            const int rr = i / 16, u = i % 16;  // row in page, 16-B unit of 2 blocks
                            const int db = u >> 3, unit = u & 7;
                            const uint4 v = *reinterpret_cast<const uint4 *>(
                                src + (int64_t)rr * kHeadDim + ((int)rank * 2 + db) * 64 + unit * 8);
                            const int row = full_pages * kPage + rr;
                            *reinterpret_cast<uint4 *>(dst + db * (kBNp * 128) + row * 128 +
                                                       ((unit ^ (row & 7)) << 4)) = v;
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                if (lane == 0) {
                    const int pp0 = r0 / kPage, pp1 = min(full_pages, r1 / kPage);
                    const uint32_t vbar = leader_addr(&v_full[sl]);
                    mbar_arrive_expect_tx_cluster(vbar, (uint32_t)max(pp1 - pp0, 0) * 2 * 2048);
                    for (int pp = pp0; pp < pp1; ++pp) {
                        int page = p.block_table[(key0 >> 4) + pp];
                        if (page < 0 || page >= p.num_pages) {
                            record_error(&g_prefill_err, kErrPageOutOfRange, page);
                            page = 0;
                        }
                        const int row = (page * kNumKvHeads + kvh) * kPage;
#pragma unroll
                        for (int db = 0; db < 2; ++db)
                            tma_load_2d_pair(dst + db * (kBNp * 128) + pp * 2048, &tmv,
                                             ((int)rank * 2 + db) * 64, row, vbar, pol);
                    }
                }
                __syncwarp();
            }
        }
    } else if (warp == kSoftmaxWarps) {
        // ------------------------------------------------------------ pair MMA issuer (leader)
        if (leader && lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc(2 * kBM, kBNp, false, false);
            constexpr uint32_t idesc_o = umma_idesc(2 * kBM, kHeadDim, false, true);
            const uint32_t q_addr = smem_u32(smem + Smem2::kQ);
            auto both = [&](uint64_t *bar) { umma2_commit_pair(bar); };
            auto issue_s = [&](int jj) -> bool {
                const int b = jj & 1;
                const int sl = jj % kKSlotsP;
                if (!wait_or_abort(&k_full[sl], (jj / kKSlotsP) & 1, abort_flag, 3)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(smem + Smem2::kK + sl * kKHalf);
#pragma unroll
                for (int kk = 0; kk < kHeadDim / 16; ++kk)
                    umma2_ss(tmem + kTS + b * kBNp,
                             umma_desc(q_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024),
                             umma_desc(k_addr + (kk >> 2) * (64 * 128) + (kk & 3) * 32, 16, 1024),
                             idesc_s, kk > 0 ? 1u : 0u);
                both(&k_empty[sl]);
                both(&s_full[b]);
                return true;
            };
            bool ok = wait_or_abort(q_full, 0, abort_flag, 2);
            if (ok) ok = issue_s(0);
            if (ok && n_loc > 1) ok = issue_s(1);
            for (int j = 0; ok && j < n_loc; ++j) {
                const int b = j & 1;
                const int sl = j % kVSlotsP;
                if (!wait_or_abort_cluster(&p_full[b], (j >> 1) & 1, abort_flag, 4) ||
                    !wait_or_abort_cluster(&v_full[sl], (j / kVSlotsP) & 1, abort_flag, 5)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t v_addr = smem_u32(smem + Smem2::kV + sl * kVHalf);
#pragma unroll
                for (int kk = 0; kk < kBNp / 16; ++kk)
                    umma2_ts(tmem + kTO, tmem + kTS + b * kBNp + kk * 8,
                             umma_desc(v_addr + kk * 2048, kBNp * 128, 1024), idesc_o,
                             (j > 0 || kk > 0) ? 1u : 0u);
                both(&v_empty[sl]);
                both(&pv_done[b]);
                if (j + 2 < n_loc) ok = issue_s(j + 2);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        // Warps w, w+4, w+8 and w+12 share TMEM lanes 32*(w%4)..+31 (one accumulator row per
        // thread) and split each 128-key S tile into key quarters [32*cg, +32) and O into dims
        // [64*cg, +64). Four warps per lane quarter keep four independent load -> max -> exp2 ->
        // store chains in flight on every SM sub-partition. The row maximum is taken on the raw
        // scores and the 1/16 * log2(e) scale is folded into the exp2 argument (one FMA).
        const int qd = warp & 3;
        const int cg = warp >> 2;
        const int r = qd * 32 + lane;
        const int t = tok0 + r / kGroup;
        const int g = r % kGroup;
        const bool row_ok = t < T;
        const int vis = P + t;
        const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
        const int64_t orow = (int64_t)t * kNumQHeads + kvh * kGroup + g;
        float *red = reinterpret_cast<float *>(smem + Smem2::kRed);  // [4 key quarters][128 rows]
        const uint32_t pbar[2] = {leader_addr(&p_full[0]), leader_addr(&p_full[1])};
        const float c = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_loc; ++j) {
            const int b = j & 1;
            if (!wait_or_abort(&s_full[b], (j >> 1) & 1, abort_flag, 6)) { ok = false; break; }
            tc_fence_after();
            float sv[32];
            tmem_ld32(tmem + lane_addr + kTS + b * kBNp + cg * 32, sv);
            tmem_wait_ld();
            const int key0 = (tb + j) * kBNp + cg * 32;
            if (!(key0 + 31 <= vis && row_ok)) {
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[i] = (row_ok && key0 + i <= vis) ? sv[i] : -INFINITY;
            }
            // four independent chains of 3-input maxima
            float mq[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
            for (int i = 4; i < 32; i += 8)
#pragma unroll
                for (int k = 0; k < 4; ++k) mq[k] = fmax3(mq[k], sv[i + 2 * k], sv[i + 2 * k + 1]);
            float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
            red[cg * kBM + r] = mx;
            // all four quarters have read S tile b (so P may overwrite it) and posted their max
            asm volatile("bar.sync %0, 128;" ::"r"(1 + qd) : "memory");
            mx = fmaxf(fmaxf(red[r], red[kBM + r]), fmaxf(red[2 * kBM + r], red[3 * kBM + r]));
            // and have read the maxima before the next tile rewrites them
            asm volatile("bar.sync %0, 128;" ::"r"(1 + qd) : "memory");
            const float m_new = fmaxf(m, mx * c);
            float corr = 1.f;
            if (m_new > m + kLazyRescale) {
                corr = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
                m = m_new;
            }
            const float m_use = (m == -INFINITY) ? 0.f : m;
            // paired fp32 FMAs and adds (sm_100 f32x2): half the issue slots of scalar ones
            const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_use, -m_use);
            float2 ps2 = make_float2(0.f, 0.f);
            uint32_t pw[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const float2 x = __ffma2_rn(make_float2(sv[i], sv[i + 1]), c2, nm2);
                const float2 a = make_float2(fast_exp2(x.x), fast_exp2(x.y));
                ps2 = __fadd2_rn(ps2, a);
                pw[i >> 1] = pack_bf16x2(a.x, a.y);
            }
            l = l * corr + (ps2.x + ps2.y);
            if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                if (!wait_or_abort(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, 7)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < 2; ++cc) {
                    float o[32];
                    const uint32_t col = kTO + cg * 64 + cc * 32;
                    tmem_ld32(tmem + lane_addr + col, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const float2 v = __fmul2_rn(make_float2(o[i], o[i + 1]), make_float2(corr, corr));
                        o[i] = v.x;
                        o[i + 1] = v.y;
                    }
                    tmem_st32(tmem + lane_addr + col, o);
                }
            }
            tmem_st16u(tmem + lane_addr + kTS + b * kBNp + cg * 16, pw);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(pbar[b]);
        }
        const int jl = n_loc - 1;
        if (ok && wait_or_abort(&pv_done[jl & 1], (jl >> 1) & 1, abort_flag, 9)) {
            tc_fence_after();
            red[cg * kBM + r] = l;
            asm volatile("bar.sync %0, 128;" ::"r"(1 + qd) : "memory");
            const float l_row = (red[r] + red[kBM + r]) + (red[2 * kBM + r] + red[3 * kBM + r]);
            const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
            uint16_t *dst = p.out + orow * kHeadDim;
            float *part = p.nsplit > 1
                              ? p.ws + ((int64_t)blockIdx.z * T * kNumQHeads + orow) * kPartial
                              : nullptr;
            if (part != nullptr && row_ok && cg == 0) {
                part[0] = (m == -INFINITY) ? -INFINITY : m * kLn2;
                part[1] = l_row;
            }
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                float o[32];
                const int col = cg * 64 + cc * 32;
                tmem_ld32(tmem + lane_addr + kTO + col, o);
                tmem_wait_ld();
                if (!row_ok) continue;
                if (part != nullptr) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        *reinterpret_cast<float2 *>(part + 2 + col + i) = make_float2(o[i], o[i + 1]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
                        v.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
                        v.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
                        v.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
                        *reinterpret_cast<uint4 *>(dst + col + i) = v;
                    }
                }
            }
        }
    }
    // neither CTA may leave (or free TMEM) while the pair MMA or the peer can still touch it
    tc_fence_before();
    cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

// Key-range splits per CTA. The kernel's K/V fetch path, not SM occupancy, limits it once
// the grid covers every SM (one CTA per SM: 225 KiB of shared memory each), so the key range
// is split only when the grid has fewer CTAs than SMs: then nsplit ~ SMs / CTAs (at most 8,
// and never more shares than the smallest CTA has key tiles); the shares are merged by
// merge_kernel.
int prefill_nsplit(int prefix_len, int chunk_len, int sm_count) {
    // Work items are CTA pairs x key-range splits; sm_count / 2 pairs are resident at once, so
    // items run in waves of `slots`. The split count is the smallest one (at most 8, and never
    // more shares than the smallest pair has 128-key tiles) whose waves are >= 85 % full, else
    // the one with the fullest waves. Each extra share costs a Q load, a pipeline fill and
    // partials for the merge, which is why a nearly full wave is not split further. Config 2
    // (100 pairs on 74 slots): 2 shares, 90 % full waves, 1193 TFLOP/s against 1023 unsplit.
    const int qtiles = (chunk_len + kTokTile - 1) / kTokTile;
    const int pairs = ((qtiles + 1) / 2) * kNumKvHeads;
    const int slots = sm_count / 2 > 0 ? sm_count / 2 : 1;
    const int min_tiles = (prefix_len + (chunk_len < kTokTile ? chunk_len : kTokTile) + 127) / 128;
    const int max_ns = min_tiles < 8 ? (min_tiles < 1 ? 1 : min_tiles) : 8;
    int best = 1;
    double best_fill = 0.0;
    for (int ns = 1; ns <= max_ns; ++ns) {
        const int64_t items = (int64_t)pairs * ns;
        const int64_t waves = (items + slots - 1) / slots;
        const double fill = (double)items / (double)(waves * slots);
        if (fill >= 0.85) return ns;
        if (fill > best_fill + 1e-9) {
            best_fill = fill;
            best = ns;
        }
    }
    return best;
}

size_t prefill_workspace_bytes(int prefix_len, int chunk_len, int sm_count) {
    const int ns = prefill_nsplit(prefix_len, chunk_len, sm_count);
    if (ns <= 1) return 0;
    return (size_t)ns * chunk_len * kNumQHeads * kPartial * sizeof(float);
}

cudaError_t launch_prefill(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                           const uint16_t *v_pages, int64_t num_pages, const int32_t *block_table, int prefix_len,
                           int chunk_len, float scale, uint16_t *out, void *workspace,
                           int sm_count, cudaStream_t stream) {
    auto kern = prefill_pair_kernel;
    const int smem_bytes = pair::Smem2::kBytes, threads = pair::kThreads, xmul = 2;
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem_bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    CUtensorMap tq;
    if (q_tensor_map(q, chunk_len, &tq) != PGC_OK) return cudaErrorInvalidValue;
    const int ns = prefill_nsplit(prefix_len, chunk_len, sm_count);
    PrefillParams pp;
    pp.block_table = block_table;
    pp.v_pages = v_pages;
    pp.out = out;
    pp.ws = static_cast<float *>(workspace);
    pp.num_pages = num_pages;
    pp.prefix_len = prefix_len;
    pp.chunk_len = chunk_len;
    pp.nsplit = ns;
    pp.scale_log2 = scale * kLog2e;
    const int qtiles = (chunk_len + kTokTile - 1) / kTokTile;
    dim3 grid((qtiles + xmul - 1) / xmul * xmul, kNumKvHeads, ns);
    kern<<<grid, threads, smem_bytes, stream>>>(tq, tk, tv, pp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || ns == 1) return e;
    const int64_t rows = (int64_t)chunk_len * kNumQHeads;
    return launch_merge_partials(pp.ws, rows, ns, rows * kPartial, nullptr, out, stream);
}

cudaError_t prefill_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_prefill_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_prefill_err, &z, sizeof(DevError));
}

}  // namespace pgc
