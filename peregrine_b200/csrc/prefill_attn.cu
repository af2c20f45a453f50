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
// CTA = one kv head x 32 query tokens. The 4 GQA heads of the kv head are stacked into the
// MMA's M = 128 rows (row r = token r/4, head r%4), so every K/V tile is loaded once for 4
// heads. Warp roles (224 threads):
//   warps 0-3  softmax + epilogue, thread r owns accumulator row r (TMEM lane r);
//   warp 4     MMA issuer (one lane): S = Q K^T (M128 N64 K256), O += P V (M128 N256);
//   warp 5     TMA producer of Q and of the K tiles (64 keys = 4 pages) into a 2-slot ring;
//   warp 6     TMA producer of the V tiles into their own 2-slot ring.
// S and P are double-buffered (TMEM S columns [0,64) and [64,128), O at [128,384) of a
// 512-column allocation; two P tiles in shared memory), so the tensor core computes S(j+2) and
// P.V(j) while the softmax warps turn S(j+1) into probabilities.
#include <cuda.h>

#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_prefill_err);

namespace {

constexpr int kBM = 128;           // rows = 32 tokens x 4 heads
constexpr int kTokTile = 32;
constexpr int kBN = 64;            // keys per tile (4 pages)
constexpr int kThreadsP = 224;
constexpr int kQBytes = kBM * kHeadDim * 2;      // 64 KiB: [4 dim blocks][128 rows][128 B]
constexpr int kKVTileBytes = kBN * kHeadDim * 2;  // 32 KiB: [4 dim blocks][64 keys][128 B]
constexpr int kPBytes = kBM * kBN * 2;            // 16 KiB: [128 rows][128 B]
constexpr int kStagesP = 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 128;
constexpr float kLazyRescale = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

struct SmemP {
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + kQBytes;                   // K ring [2]
    static constexpr int kV = kK + kStagesP * kKVTileBytes;   // V ring [2]
    static constexpr int kP = kV + kStagesP * kKVTileBytes;   // P [2]
    static constexpr int kBar = kP + 2 * kPBytes;
    // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full[2], p_free[2]
    static constexpr int kNumBars = 15;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kBytes = kTmemSlot + 16;
};
constexpr int kSmemBytesP = SmemP::kBytes + 1024;

struct PrefillParams {
    const int32_t *block_table;
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

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar))
                 : "memory");
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

// 3-D tiled TMA load (Q tile: 64 dims x 4 heads x 32 tokens).
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const void *tmap, int32_t x, int32_t y,
                                            int32_t z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
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
                *abort_flag = 1;
                return false;
            }
        }
    }
}

__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, const PrefillParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ int abort_flag_s;

    const int qt = blockIdx.x;
    const int kvh = blockIdx.y;
    const int T = p.chunk_len, P = p.prefix_len;
    const int tok0 = qt * kTokTile;
    const int t_last = min(tok0 + kTokTile - 1, T - 1);
    const int n_keys = P + t_last + 1;  // keys any row of this tile may see
    const int n_tiles = (n_keys + kBN - 1) / kBN;
    const int total_keys = P + T;       // keys present in the cache
    // this CTA's share of the key tiles (split z of nsplit; the host keeps every share >= 1)
    const int tb = (int)((int64_t)n_tiles * blockIdx.z / p.nsplit);
    const int n_loc = (int)((int64_t)n_tiles * (blockIdx.z + 1) / p.nsplit) - tb;

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + SmemP::kBar);
    uint64_t *q_full = bars + 0;
    uint64_t *k_full = bars + 1;   // [2]
    uint64_t *k_empty = bars + 3;  // [2]
    uint64_t *v_full = bars + 5;   // [2]
    uint64_t *v_empty = bars + 7;  // [2]
    uint64_t *s_full = bars + 9;   // [2] S buffer b holds a finished S tile
    uint64_t *p_full = bars + 11;  // [2] P buffer b written (128 arrivals)
    uint64_t *p_free = bars + 13;  // [2] P.V that read P buffer b has completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + SmemP::kTmemSlot);
    volatile int *abort_flag = &abort_flag_s;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        abort_flag_s = 0;
        mbar_init(q_full, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&k_full[b], 1);
            mbar_init(&k_empty[b], 1);
            mbar_init(&v_full[b], 1);
            mbar_init(&v_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], kBM);
            mbar_init(&p_free[b], 1);
        }
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    uint8_t *q_s = smem + SmemP::kQ;

    if (warp == 5 || warp == 6) {
        // ------------------------------------------------------------ TMA producers
        // warp 5 streams Q and the K tiles, warp 6 the V tiles; each ring slot is refilled as
        // soon as the MMA that read it has completed (S for K, P.V for V).
        if (lane == 0) {
            const bool is_k = warp == 5;
            const CUtensorMap *tm = is_k ? &tmk : &tmv;
            tma_prefetch_desc(tm);
            // every q-tile CTA of a kv head streams the same K/V: ask L2 to keep it
            const uint64_t pol = l2_policy_evict_last();
            if (is_k) {
                tma_prefetch_desc(&tmq);
                mbar_arrive_expect_tx(q_full, kQBytes);
                for (int c = 0; c < 4; ++c)
                    tma_load_3d(q_s + c * (kBM * 128), &tmq, c * 64, kvh * kGroup, tok0, q_full);
            }
            uint64_t *full = is_k ? k_full : v_full;
            uint64_t *empty = is_k ? k_empty : v_empty;
            uint8_t *ring = smem + (is_k ? SmemP::kK : SmemP::kV);
            for (int j = 0; j < n_loc; ++j) {
                const int b = j & 1;
                if (j >= 2 && !wait_or_abort(&empty[b], ((j >> 1) - 1) & 1, abort_flag, 1)) break;
                const int key0 = (tb + j) * kBN;
                int npg = 0;
                for (int pp = 0; pp < kBN / kPage; ++pp)
                    if (key0 + pp * kPage < total_keys) ++npg;
                mbar_arrive_expect_tx(&full[b], (uint32_t)npg * kPage * kHeadDim * 2);
                uint8_t *tile = ring + b * kKVTileBytes;
                for (int pp = 0; pp < npg; ++pp) {
                    int page = p.block_table[(key0 >> 4) + pp];
                    if (page < 0 || page >= p.num_pages) {
                        record_error(&g_prefill_err, kErrPageOutOfRange, page);
                        page = 0;
                    }
                    const int row = (page * kNumKvHeads + kvh) * kPage;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tma_load_2d(tile + c * (kBN * 128) + pp * 2048, tm, c * 64, row, &full[b], pol);
                }
            }
        }
    } else if (warp == 4) {
        // ------------------------------------------------------------ MMA issuer
        // Issue order S0 S1 PV0 S2 PV1 S3 ...: S(j+2) and P.V(j) run while the softmax
        // warps work on S(j+1).
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc(kBM, kBN, false, false);
            constexpr uint32_t idesc_o = umma_idesc(kBM, kHeadDim, false, true);
            const uint32_t q_addr = smem_u32(q_s);
            auto issue_s = [&](int jj) -> bool {
                const int b = jj & 1;
                if (!wait_or_abort(&k_full[b], (jj >> 1) & 1, abort_flag, 3)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(smem + SmemP::kK + b * kKVTileBytes);
#pragma unroll
                for (int kk = 0; kk < kHeadDim / 16; ++kk)
                    umma_f16(tmem + kTmemS + b * kBN,
                             umma_desc(q_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024),
                             umma_desc(k_addr + (kk >> 2) * (kBN * 128) + (kk & 3) * 32, 16, 1024),
                             idesc_s, kk > 0 ? 1u : 0u);
                umma_commit(&k_empty[b]);
                umma_commit(&s_full[b]);
                return true;
            };
            bool ok = wait_or_abort(q_full, 0, abort_flag, 2);
            if (ok) ok = issue_s(0);
            if (ok && n_loc > 1) ok = issue_s(1);
            for (int j = 0; ok && j < n_loc; ++j) {
                const int b = j & 1;
                if (!wait_or_abort(&p_full[b], (j >> 1) & 1, abort_flag, 4) ||
                    !wait_or_abort(&v_full[b], (j >> 1) & 1, abort_flag, 5)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t p_addr = smem_u32(smem + SmemP::kP + b * kPBytes);
                const uint32_t v_addr = smem_u32(smem + SmemP::kV + b * kKVTileBytes);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_f16(tmem + kTmemO, umma_desc(p_addr + kk * 32, 16, 1024),
                             umma_desc(v_addr + kk * 2048, kBN * 128, 1024), idesc_o,
                             (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&v_empty[b]);
                umma_commit(&p_free[b]);
                if (j + 2 < n_loc) ok = issue_s(j + 2);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        const int r = threadIdx.x;  // accumulator row = TMEM lane
        const int t = tok0 + r / kGroup;
        const int g = r % kGroup;
        const bool row_ok = t < T;
        const int vis = P + t;  // keys c <= vis are visible
        const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_loc; ++j) {
            const int b = j & 1;
            if (!wait_or_abort(&s_full[b], (j >> 1) & 1, abort_flag, 6)) { ok = false; break; }
            tc_fence_after();
            float sv[64];
            {
                float a[32], c2[32];
                tmem_ld32(tmem + lane_addr + kTmemS + b * kBN, a);
                tmem_ld32(tmem + lane_addr + kTmemS + b * kBN + 32, c2);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) { sv[i] = a[i]; sv[32 + i] = c2[i]; }
            }
            const int key0 = (tb + j) * kBN;
            float mx = -INFINITY;
            if (key0 + kBN - 1 <= vis && row_ok) {  // tile entirely visible: no per-key test
#pragma unroll
                for (int i = 0; i < kBN; ++i) {
                    sv[i] *= p.scale_log2;
                    mx = fmaxf(mx, sv[i]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < kBN; ++i) {
                    sv[i] = (row_ok && key0 + i <= vis) ? sv[i] * p.scale_log2 : -INFINITY;
                    mx = fmaxf(mx, sv[i]);
                }
            }
            const float m_new = fmaxf(m, mx);
            float corr = 1.f;
            if (m_new > m + kLazyRescale) {  // also true the first time a row sees a key
                corr = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
                m = m_new;
            }
            const float m_use = (m == -INFINITY) ? 0.f : m;
            float ps = 0.f;
#pragma unroll
            for (int i = 0; i < kBN; ++i) {
                sv[i] = fast_exp2(sv[i] - m_use);
                ps += sv[i];
            }
            l = l * corr + ps;
            if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                // O must be stable: wait for P.V(j-1), the last MMA writing it
                if (!wait_or_abort(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, 7)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < kHeadDim / 32; ++cc) {
                    float o[32];
                    tmem_ld32(tmem + lane_addr + kTmemO + cc * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= corr;
                    tmem_st32(tmem + lane_addr + kTmemO + cc * 32, o);
                }
                tmem_wait_st();
            }
            // P buffer b is free once P.V(j-2), the previous reader, has completed
            if (j >= 2 && !wait_or_abort(&p_free[b], ((j >> 1) - 1) & 1, abort_flag, 10)) {
                ok = false;
                break;
            }
            uint8_t *p_s = smem + SmemP::kP + b * kPBytes;
#pragma unroll
            for (int ch = 0; ch < kBN / 8; ++ch) {
                uint4 v;
                v.x = pack_bf16x2(sv[ch * 8 + 0], sv[ch * 8 + 1]);
                v.y = pack_bf16x2(sv[ch * 8 + 2], sv[ch * 8 + 3]);
                v.z = pack_bf16x2(sv[ch * 8 + 4], sv[ch * 8 + 5]);
                v.w = pack_bf16x2(sv[ch * 8 + 6], sv[ch * 8 + 7]);
                *reinterpret_cast<uint4 *>(p_s + r * 128 + ((ch ^ (r & 7)) << 4)) = v;
            }
            if (key0 + kBN > total_keys) {
                // Keys past the cache end (stale slots, or pages not loaded) get zero V rows so
                // that a NaN pattern cannot reach the P.V product through a zero probability.
                if (!wait_or_abort(&v_full[b], (j >> 1) & 1, abort_flag, 8)) { ok = false; break; }
                uint8_t *vt = smem + SmemP::kV + b * kKVTileBytes;
                const int first = total_keys - key0;
                const int nz = (kBN - first) * 4 * 8;  // rows x 4 dim blocks x 8 units of 16 B
                for (int i = r; i < nz; i += kBM) {
                    const int row = first + i / 32;
                    const int u = i % 32;
                    *reinterpret_cast<uint4 *>(vt + (u >> 3) * (kBN * 128) + row * 128 + (u & 7) * 16) =
                        make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&p_full[b]);
        }
        const int jl = n_loc - 1;
        if (ok && wait_or_abort(&p_free[jl & 1], (jl >> 1) & 1, abort_flag, 9)) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const int64_t orow = (int64_t)t * kNumQHeads + kvh * kGroup + g;
            uint16_t *dst = p.out + orow * kHeadDim;
            float *part = p.nsplit > 1
                              ? p.ws + ((int64_t)blockIdx.z * T * kNumQHeads + orow) * kPartial
                              : nullptr;
            if (part != nullptr && row_ok) {
                part[0] = (m == -INFINITY) ? -INFINITY : m * kLn2;  // natural-log units
                part[1] = l;
            }
#pragma unroll 1
            for (int cc = 0; cc < kHeadDim / 32; ++cc) {
                float o[32];
                tmem_ld32(tmem + lane_addr + kTmemO + cc * 32, o);
                tmem_wait_ld();
                if (!row_ok) continue;
                if (part != nullptr) {
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        *reinterpret_cast<float2 *>(part + 2 + cc * 32 + i) = make_float2(o[i], o[i + 1]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
                        v.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
                        v.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
                        v.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
                        *reinterpret_cast<uint4 *>(dst + cc * 32 + i) = v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
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
    const int ctas = ((chunk_len + kTokTile - 1) / kTokTile) * kNumKvHeads;
    const int min_tiles = (prefix_len + (chunk_len < kTokTile ? chunk_len : kTokTile) + kBN - 1) / kBN;
    int ns = sm_count / ctas;
    if (ns > 8) ns = 8;
    if (ns > min_tiles) ns = min_tiles;
    return ns < 1 ? 1 : ns;
}

size_t prefill_workspace_bytes(int prefix_len, int chunk_len, int sm_count) {
    const int ns = prefill_nsplit(prefix_len, chunk_len, sm_count);
    if (ns <= 1) return 0;
    return (size_t)ns * chunk_len * kNumQHeads * kPartial * sizeof(float);
}

cudaError_t launch_prefill(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                           int64_t num_pages, const int32_t *block_table, int prefix_len,
                           int chunk_len, float scale, uint16_t *out, void *workspace,
                           int sm_count, cudaStream_t stream) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytesP);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    CUtensorMap tq;
    if (q_tensor_map(q, chunk_len, &tq) != PGC_OK) return cudaErrorInvalidValue;
    const int ns = prefill_nsplit(prefix_len, chunk_len, sm_count);
    PrefillParams pp;
    pp.block_table = block_table;
    pp.out = out;
    pp.ws = static_cast<float *>(workspace);
    pp.num_pages = num_pages;
    pp.prefix_len = prefix_len;
    pp.chunk_len = chunk_len;
    pp.nsplit = ns;
    pp.scale_log2 = scale * kLog2e;
    dim3 grid((chunk_len + kTokTile - 1) / kTokTile, kNumKvHeads, ns);
    prefill_kernel<<<grid, kThreadsP, kSmemBytesP, stream>>>(tq, tk, tv, pp);
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
