// decode_attn.cu — split-K flash-decode attention over the paged bf16 KV cache (sm_100a).
//
// Behaviour follows sdpa_decode_prefix_flash_partials_bf16 + ..._reduce_gated_bf16
// (shaders/attention_decode.metal:24-243): per (kv head, context split) the 4 GQA query heads
// are scored against every token, an online softmax keeps (m, l, o[256]) in fp32, and a
// log-sum-exp merge combines the splits and applies the optional sigmoid gate.
//
// B200 design:
//   * one CTA per (split, kv head, sequence); 1 producer warp + 4 consumer warps;
//   * the producer streams each 16-token page of K and V (8 KiB each, contiguous in the pool)
//     into a 4-stage shared-memory ring with 2-D TMA loads (64 x 16 boxes, 128-byte swizzle,
//     L2 evict-first), completion on mbarriers;
//   * consumer warp w takes pages w, w+4, ...; scores and P.V run on the bf16 tensor cores
//     (mma.m16n8k16, fp32 accumulate) with the query rows (4 heads x up to 4 query tokens) as
//     the M dimension, so the online softmax stays in registers;
//   * the 4 warp states are merged in shared memory and each split writes one fp32 partial
//     per query row; a second small kernel merges splits (and, for context parallelism,
//     partials gathered from other GPUs).
#include <cuda.h>

#include <mutex>

#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_decode_err);

namespace {

constexpr int kConsumers = 4;
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kStages = 4;
// Page i goes to stage i % kStages and to consumer warp i % kConsumers. The stage count must be
// a multiple of the consumer count so that every stage has exactly one consumer, which waits
// on it phase after phase; with a stage shared by two warps, a warp running ahead would wait
// on the parity of a phase two steps ahead, which an mbarrier reports as already complete.
static_assert(kStages % kConsumers == 0, "each stage must belong to one consumer warp");
constexpr int kTileBytes = kPage * kHeadDim * 2;  // one (page, kv head) of K or V: 8 KiB
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kQRowBytes = kHeadDim * 2 + 16;  // padded row: conflict-free ldmatrix
constexpr int kMinPagesPerSplit = 4;
constexpr int kMaxPagesPerSplit = 64;
constexpr int kPrefetchPre = 4;    // pages prefetched into L2 before the programmatic-launch wait
constexpr int kPrefetchAhead = 0;  // pages prefetched past the ring while streaming

struct SplitParams {
    const uint16_t *q;           // rotated query rows, or nullptr with `app` set
    DecodeAppend app;            // fused decode append (app.q_in != nullptr)
    const int32_t *block_tables;
    const int32_t *seq_lens;
    float *ws;  // [rows][max_splits][258], row = (seq * nq + j) * 16 + head
    int64_t num_pages;
    int max_pages_per_seq;
    int num_queries;
    int pages_per_split;
    int max_splits;
    float scale_log2;
    // L2 prefetch hints (0: none): `prefetch_pre` pages of this CTA's range are prefetched
    // before the programmatic-launch wait, from a block-table and length read that may predate
    // the previous kernel's writes (hints only: the TMA loads after the wait read the pool
    // coherently through L2); `prefetch_ahead` pages past the ring while streaming.
    int prefetch_pre, prefetch_ahead;
    const uint8_t *k_base, *v_base;
};

struct SmemLayout {
    static constexpr int kStageOff = 0;                            // 1024-aligned
    static constexpr int kQOff = kStageOff + kStages * kStageBytes;
    static constexpr int kMOff = kQOff + 16 * kQRowBytes;
    static constexpr int kLOff = kMOff + kConsumers * 16 * 4;
    static constexpr int kBarOff = kLOff + kConsumers * 16 * 4;
    static constexpr int kBytes = kBarOff + (2 * kStages + 1) * 8;  // + kv_ready (fused append)
};
constexpr int kSmemBytes = SmemLayout::kBytes + 1024;  // + alignment slack

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) from global memory into L2.
__device__ __forceinline__ void prefetch_l2(const void *ptr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

template <bool kFused>
__global__ void __launch_bounds__(kThreads, 2)
    decode_split_kernel(const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const SplitParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    pdl_trigger();
    const int split = blockIdx.x;
    const int kvh = blockIdx.y;
    const int seq = blockIdx.z;
    const int nq = p.num_queries;
    const int nrows = nq * kGroup;

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + SmemLayout::kBarOff);
    uint64_t *empty = full + kStages;
    uint8_t *q_s = smem + SmemLayout::kQOff;
    float *m_s = reinterpret_cast<float *>(smem + SmemLayout::kMOff);
    float *l_s = reinterpret_cast<float *>(smem + SmemLayout::kLOff);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Shared-memory barriers and the tensor-map prefetch touch no global memory that an earlier
    // kernel writes, so they run before the programmatic-launch wait, overlapping its tail.
    uint64_t *kv_ready = empty + kStages;  // fused append: the new K/V rows are in the pool
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        if (kFused) mbar_init(kv_ready, nq);
        fence_mbar_init();
    }
    if (threadIdx.x == kConsumers * 32) {
        tma_prefetch_desc(&tmk);
        tma_prefetch_desc(&tmv);
        // Start HBM -> L2 traffic for this CTA's first pages while the previous kernel in the
        // stream drains (its tail and the merge before this launch): page ids outside the pool
        // are skipped, so a stale table costs bandwidth, never correctness.
        if (p.prefetch_pre > 0) {
            const int Lg = p.seq_lens[seq];
            const int tb = split * p.pages_per_split * kPage;
            if (tb < Lg) {
                const int np = min(p.prefetch_pre, (min(Lg, tb + p.pages_per_split * kPage) - tb + kPage - 1) / kPage);
                const int32_t *tbl = p.block_tables + (int64_t)seq * p.max_pages_per_seq + split * p.pages_per_split;
                for (int i = 0; i < np; ++i) {
                    const int pg = tbl[i];
                    if (pg >= 0 && pg < p.num_pages) {
                        const int64_t off = ((int64_t)pg * kNumKvHeads + kvh) * kTileBytes;
                        prefetch_l2(p.k_base + off, kTileBytes);
                        prefetch_l2(p.v_base + off, kTileBytes);
                    }
                }
            }
        }
    }
    pdl_wait();
    const int L = p.seq_lens[seq];
    const int tok_begin = split * p.pages_per_split * kPage;
    if (tok_begin >= L) {
        // A split past the sequence end leaves an empty partial (m = -inf, l = 0; its o is never
        // summed), so the merges take every planned split without reading the lengths again.
        if (threadIdx.x < nrows) {
            const int j = threadIdx.x / kGroup, g = threadIdx.x % kGroup;
            const int64_t row = (int64_t)(seq * nq + j) * kNumQHeads + kvh * kGroup + g;
            float *dst = p.ws + (row * p.max_splits + split) * kPartial;
            dst[0] = -INFINITY;
            dst[1] = 0.f;
        }
        return;  // uniform across the CTA
    }
    const int tok_end = min(L, tok_begin + p.pages_per_split * kPage);
    const int n_pages = (tok_end - tok_begin + kPage - 1) / kPage;
    __syncthreads();  // barriers initialised: the producer may start streaming K/V now

    if (warp == kConsumers) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            // fused append: the pages holding a new token are loaded only after this CTA has
            // written the token's K/V rows into the pool (kv_ready), so the tile carries them
            int32_t newpos[PGC_MAX_QUERIES];
#pragma unroll
            for (int j = 0; j < PGC_MAX_QUERIES; ++j)
                newpos[j] = (kFused && j < nq) ? (int32_t)(p.app.positions[(int64_t)seq * nq + j] - p.app.pos_offset) : -1;
            const int32_t *table =
                p.block_tables + (int64_t)seq * p.max_pages_per_seq + split * p.pages_per_split;
            auto prefetch_page = [&](int i) {
                const int pg = table[i];
                if (pg >= 0 && pg < p.num_pages) {
                    const int64_t off = ((int64_t)pg * kNumKvHeads + kvh) * kTileBytes;
                    prefetch_l2(p.k_base + off, kTileBytes);
                    prefetch_l2(p.v_base + off, kTileBytes);
                }
            };
            for (int i = max(kStages, p.prefetch_pre); i < min(n_pages, kStages + p.prefetch_ahead); ++i)
                prefetch_page(i);
            for (int i = 0; i < n_pages; ++i) {
                if (i + kStages + p.prefetch_ahead < n_pages && p.prefetch_ahead > 0 &&
                    i + kStages + p.prefetch_ahead >= p.prefetch_pre)
                    prefetch_page(i + kStages + p.prefetch_ahead);
                const int s = i % kStages;
                const int round = i / kStages;
                if (round > 0 && !mbar_wait_bounded(&empty[s], (round - 1) & 1)) {
                    record_error(&g_decode_err, kErrWaitTimeout, 1);
                    return;
                }
                int page = table[i];
                if (page < 0 || page >= p.num_pages) {
                    record_error(&g_decode_err, kErrPageOutOfRange, page);
                    page = 0;
                }
                if (kFused) {
                    const int tok0 = tok_begin + i * kPage;
                    bool holds_new = false;
#pragma unroll
                    for (int j = 0; j < PGC_MAX_QUERIES; ++j)
                        holds_new |= newpos[j] >= tok0 && newpos[j] < tok0 + kPage && newpos[j] < tok_end;
                    if (holds_new && !mbar_wait_bounded(kv_ready, 0)) {
                        record_error(&g_decode_err, kErrWaitTimeout, 3);
                        return;
                    }
                }
                uint8_t *stage = smem + SmemLayout::kStageOff + s * kStageBytes;
                mbar_arrive_expect_tx(&full[s], kStageBytes);
                const int row = (page * kNumKvHeads + kvh) * kPage;
#pragma unroll
                for (int c = 0; c < 4; ++c) tma_load_2d(stage + c * 2048, &tmk, c * 64, row, &full[s], pol);
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    tma_load_2d(stage + kTileBytes + c * 2048, &tmv, c * 64, row, &full[s], pol);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    constexpr bool fused = kFused;
    if (!fused) {
        // Query rows (loaded while the first K/V pages are in flight): r = j * 4 + g (query
        // token j, head kvh * 4 + g); rows >= nrows are zero.
        for (int i = threadIdx.x; i < 16 * (kHeadDim / 8); i += kConsumers * 32) {
            const int r = i / (kHeadDim / 8);
            const int c = i % (kHeadDim / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < nrows) {
                const int j = r / kGroup, g = r % kGroup;
                const uint16_t *src =
                    p.q + ((int64_t)(seq * nq + j) * kNumQHeads + kvh * kGroup + g) * kHeadDim;
                v = reinterpret_cast<const uint4 *>(src)[c];
            }
            *reinterpret_cast<uint4 *>(q_s + r * kQRowBytes + c * 16) = v;
        }
    } else {
        // Fused decode append, the arithmetic of pgc_append_kv_rope in decode mode: the query
        // rows (RMSNorm + RoPE) go straight into the tile; the new K and V rows of this kv head
        // are written into the pool by the CTA whose token range holds them, before its producer
        // loads those pages (kv_ready), so the attention reads them as after a separate append.
        const DecodeAppend &a = p.app;
        // warp g: query head kvh * 4 + g of every token j (tile row j * 4 + g); warp j < nq also
        // the new K and V rows of token j. All loads are issued in two rounds (positions, then
        // rows, weights and RoPE rows) before any arithmetic.
        const int g = warp;
        const int64_t tb = (int64_t)seq * nq;
        int32_t pos[PGC_MAX_QUERIES];
#pragma unroll
        for (int j = 0; j < PGC_MAX_QUERIES; ++j) pos[j] = j < nq ? a.positions[tb + j] : -1;
        const int64_t slot = warp < nq ? a.slots[tb + warp] : -1;
        const int32_t kpos = warp < nq ? a.positions[tb + warp] : -1;  // the K/V token's position
        // its index in this sequence's cache (a context-parallel shard starts at pos_offset)
        const int64_t klocal = (int64_t)kpos - a.pos_offset;
        // The appended tokens normally sit at L - nq + j: their RoPE rows are fetched for that
        // guess in the same round as the positions, and fetched again only where a position
        // differs.
        float xq[PGC_MAX_QUERIES][8], cq[PGC_MAX_QUERIES], sq[PGC_MAX_QUERIES], qwf[8];
#pragma unroll
        for (int j = 0; j < PGC_MAX_QUERIES; ++j) {
            const int32_t guess = (int32_t)(L - nq + j + a.pos_offset);
            const bool gok = j < nq && guess >= 0 && guess < a.rope_max_pos;
            cq[j] = gok ? a.rope[(int64_t)guess * kRot + lane] : 0.f;
            sq[j] = gok ? a.rope[(int64_t)guess * kRot + 32 + lane] : 0.f;
            const uint16_t *src = a.q_in + ((tb + j) * kNumQHeads + kvh * kGroup + g) * a.q_head_stride;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) xq[j][jj] = j < nq ? bf16_bits_to_f32(src[lane + 32 * jj]) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < PGC_MAX_QUERIES; ++j) {
            const bool ok = j < nq && pos[j] >= 0 && pos[j] < a.rope_max_pos;
            if (ok && pos[j] != (int32_t)(L - nq + j + a.pos_offset)) {
                cq[j] = a.rope[(int64_t)pos[j] * kRot + lane];
                sq[j] = a.rope[(int64_t)pos[j] * kRot + 32 + lane];
            }
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) qwf[jj] = a.q_norm_w != nullptr ? bf16_bits_to_f32(a.q_norm_w[lane + 32 * jj]) : 0.f;
        // the K/V token's rows and its RoPE row (for the guessed position) in the same round
        float xk[8], kwf[8], ck = 0.f, sk = 0.f;
        uint16_t vv[8];
        const int32_t kguess = (int32_t)(L - nq + warp + a.pos_offset);
        if (warp < nq) {
            const int64_t t = tb + warp;
            const uint16_t *ks = a.k_in + (t * kNumKvHeads + kvh) * kHeadDim;
            const uint16_t *vs = a.v_in + (t * kNumKvHeads + kvh) * kHeadDim;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                xk[jj] = bf16_bits_to_f32(ks[lane + 32 * jj]);
                kwf[jj] = a.k_norm_w != nullptr ? bf16_bits_to_f32(a.k_norm_w[lane + 32 * jj]) : 0.f;
                vv[jj] = vs[lane + 32 * jj];
            }
            if (kguess >= 0 && kguess < a.rope_max_pos) {
                ck = a.rope[(int64_t)kguess * kRot + lane];
                sk = a.rope[(int64_t)kguess * kRot + 32 + lane];
            }
        }
        const bool kv_ok = warp < nq && kpos >= 0 && kpos < a.rope_max_pos && slot >= 0;
        const bool page_ok = kv_ok && slot / kPage < a.num_pages;
        if (page_ok && kpos != kguess) {
            ck = a.rope[(int64_t)kpos * kRot + lane];
            sk = a.rope[(int64_t)kpos * kRot + 32 + lane];
        }
        // query rows
#pragma unroll
        for (int j = 0; j < PGC_MAX_QUERIES; ++j) {
            uint16_t *qrow = reinterpret_cast<uint16_t *>(q_s + (j * kGroup + g) * kQRowBytes);
            uint16_t o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (j < nq) {
                if (pos[j] >= 0 && pos[j] < a.rope_max_pos)
                    append_row_compute(xq[j], a.q_norm_w != nullptr ? qwf : nullptr, cq[j], sq[j], true, o);
                else if (lane == 0 && kvh == 0 && split == 0 && g == 0)
                    record_error(&g_decode_err, kErrPosOutOfRange, tb + j);
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) qrow[lane + 32 * jj] = o[jj];
        }
        // the new K and V rows of token `warp`, written into the pool by the CTA whose token
        // range holds its position (split 0 for a position past the sequence); every warp
        // j < nq then releases kv_ready after a proxy fence, so the producer's TMA loads see them
        if (warp < nq) {
            if (kv_ok && !page_ok) {
                if (lane == 0 && kvh == 0 && split == 0) record_error(&g_decode_err, kErrSlotOutOfRange, slot);
            } else if (page_ok && ((klocal >= tok_begin && klocal < tok_end) || (split == 0 && klocal >= L))) {
                uint16_t ko[8];
                append_row_compute(xk, a.k_norm_w != nullptr ? kwf : nullptr, ck, sk, true, ko);
                const int64_t off = (((slot / kPage) * kNumKvHeads + kvh) * kPage + slot % kPage) * kHeadDim;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    a.k_pages[off + lane + 32 * jj] = ko[jj];
                    a.v_pages[off + lane + 32 * jj] = vv[jj];
                }
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(kv_ready);
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");

    const int r0 = lane >> 2;          // C-fragment rows r0 and r0 + 8
    const int cpair = (lane & 3) * 2;  // C-fragment column pair
    // visible token bound per C row: query j sees tokens < L - nq + j + 1
    const int vis0 = (r0 < nrows) ? L - nq + (r0 / kGroup) + 1 : L;
    const int vis1 = (r0 + 8 < nrows) ? L - nq + ((r0 + 8) / kGroup) + 1 : L;

    float o[32][4];
#pragma unroll
    for (int n = 0; n < 32; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    const uint32_t q_base = smem_u32(q_s) + (lane & 15) * kQRowBytes + (lane >> 4) * 16;
    // ldmatrix lane roles: matrix mi = lane / 8, row-in-matrix = lane % 8
    const int mi = lane >> 3;
    const int k_tok = (mi >> 1) * 8 + (lane & 7);  // K: matrices (tok 0-7|8-15) x (k lo|hi)
    const int k_dim_off = (mi & 1) * 8;
    const int v_tok = (mi & 1) * 8 + (lane & 7);   // V: matrices (tok lo|hi) x (dim lo|hi)
    const int v_dim_off = (mi >> 1) * 8;

    bool ok = true;
    for (int i = warp; i < n_pages; i += kConsumers) {
        const int s = i % kStages;
        if (!mbar_wait_bounded(&full[s], (i / kStages) & 1)) {
            record_error(&g_decode_err, kErrWaitTimeout, 2);
            ok = false;
            break;
        }
        uint8_t *kt = smem + SmemLayout::kStageOff + s * kStageBytes;
        uint8_t *vt = kt + kTileBytes;
        const uint32_t k_base = smem_u32(kt);
        const uint32_t v_base = smem_u32(vt);
        const int tok0 = tok_begin + i * kPage;
        const int nvalid = min(kPage, tok_end - tok0);

        // S[16 rows x 16 tokens] = Q K^T
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            ldsm_x4(q_base + kk * 32, a0, a1, a2, a3);
            ldsm_x4(k_base + swz_page_offset(k_tok, kk * 16 + k_dim_off), b0, b1, b2, b3);
            mma_bf16_16816(sacc[0], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(sacc[1], a0, a1, a2, a3, b2, b3);
        }

        // masked, log2-scaled scores; online softmax in registers
        float sc[2][4];
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int t = tok0 + n * 8 + cpair + e;
                sc[n][e] = (t < vis0) ? sacc[n][e] * p.scale_log2 : -INFINITY;
                sc[n][2 + e] = (t < vis1) ? sacc[n][2 + e] * p.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, sc[n][e]);
                mx1 = fmaxf(mx1, sc[n][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float mu0 = (mn0 == -INFINITY) ? 0.f : mn0;
        const float mu1 = (mn1 == -INFINITY) ? 0.f : mn1;
        const float corr0 = fast_exp2(m0 - mu0);  // m = -inf -> 0
        const float corr1 = fast_exp2(m1 - mu1);
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[n][e] = fast_exp2(sc[n][e] - mu0);
                sc[n][2 + e] = fast_exp2(sc[n][2 + e] - mu1);
                ps0 += sc[n][e];
                ps1 += sc[n][2 + e];
            }
        }
        l0 = l0 * corr0 + ps0;
        l1 = l1 * corr1 + ps1;
        if (__any_sync(0xffffffffu, corr0 != 1.f || corr1 != 1.f)) {
#pragma unroll
            for (int n = 0; n < 32; ++n) {
                o[n][0] *= corr0;
                o[n][1] *= corr0;
                o[n][2] *= corr1;
                o[n][3] *= corr1;
            }
        }
        const uint32_t pa0 = pack_bf16x2(sc[0][0], sc[0][1]);
        const uint32_t pa1 = pack_bf16x2(sc[0][2], sc[0][3]);
        const uint32_t pa2 = pack_bf16x2(sc[1][0], sc[1][1]);
        const uint32_t pa3 = pack_bf16x2(sc[1][2], sc[1][3]);

        if (nvalid < kPage) {
            // Slots past the sequence end hold stale bytes; zero their V rows so that a
            // NaN pattern cannot leak through a zero probability.
            for (int idx = lane; idx < (kPage - nvalid) * 4 * 8; idx += 32) {
                const int row = nvalid + idx / 32;
                const int unit = idx % 32;  // 4 boxes x 8 units of 16 B
                *reinterpret_cast<uint4 *>(vt + (unit >> 3) * 2048 + row * 128 + (unit & 7) * 16) =
                    make_uint4(0, 0, 0, 0);
            }
            fence_proxy_async_smem();  // generic writes before any later async-proxy refill
            __syncwarp();
        }

        // O[16 x 256] += P[16 x 16] V[16 x 256]
#pragma unroll
        for (int nd = 0; nd < 16; ++nd) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_trans(v_base + swz_page_offset(v_tok, nd * 16 + v_dim_off), b0, b1, b2, b3);
            mma_bf16_16816(o[2 * nd], pa0, pa1, pa2, pa3, b0, b1);
            mma_bf16_16816(o[2 * nd + 1], pa0, pa1, pa2, pa3, b2, b3);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---------------------------------------------------------------- merge 4 warp states
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    // all consumers are past their last stage read: reuse the ring as fp32 scratch
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
    float *o_s = reinterpret_cast<float *>(smem + SmemLayout::kStageOff);  // [4][16][256]
    if ((lane & 3) == 0) {
        m_s[warp * 16 + r0] = m0;
        l_s[warp * 16 + r0] = l0;
        m_s[warp * 16 + r0 + 8] = m1;
        l_s[warp * 16 + r0 + 8] = l1;
    }
    if (r0 < nrows) {
#pragma unroll
        for (int n = 0; n < 32; ++n)
            *reinterpret_cast<float2 *>(&o_s[(warp * 16 + r0) * kHeadDim + n * 8 + cpair]) =
                make_float2(o[n][0], o[n][1]);
    }
    if (r0 + 8 < nrows) {
#pragma unroll
        for (int n = 0; n < 32; ++n)
            *reinterpret_cast<float2 *>(&o_s[(warp * 16 + r0 + 8) * kHeadDim + n * 8 + cpair]) =
                make_float2(o[n][2], o[n][3]);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
    if (!ok) return;

    const int tid = threadIdx.x;  // 0..127
    for (int r = 0; r < nrows; ++r) {
        float ma = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) ma = fmaxf(ma, m_s[w * 16 + r]);
        float wt[kConsumers];
        float den = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumers; ++w) {
            const float mw = m_s[w * 16 + r];
            wt[w] = (mw == -INFINITY) ? 0.f : fast_exp2(mw - ma);
            den += l_s[w * 16 + r] * wt[w];
        }
        const int j = r / kGroup, g = r % kGroup;
        const int64_t row = (int64_t)(seq * nq + j) * kNumQHeads + kvh * kGroup + g;
        float *dst = p.ws + (row * p.max_splits + split) * kPartial;
        for (int d = tid; d < kHeadDim; d += kConsumers * 32) {
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumers; ++w) acc += o_s[(w * 16 + r) * kHeadDim + d] * wt[w];
            dst[2 + d] = acc;
        }
        if (tid == 0) {
            dst[0] = (ma == -INFINITY) ? -INFINITY : ma * kLn2;  // natural-log units
            dst[1] = den;
        }
    }
}

// Log-sum-exp merge of a row's partials (attention_decode.metal:215-243). One CTA per
// (row, 32-dim chunk): lane = dim, so every partial row read is a coalesced 128-byte run, and
// the 8 warps take every 8th partial, so the reads of different partials are independent and
// overlap instead of forming one serial chain. A part with m = -inf (a split past the sequence
// end) has weight 0 and its o is not summed.
struct MergeParams {
    const float *parts;
    int64_t row_stride;   // floats between rows
    int64_t part_stride;  // floats between parts of a row
    int nparts;
    const uint16_t *gate;
    int64_t gate_stride;  // elements between gate rows
    uint16_t *out;      // bf16 output, or
    float *out_partial; // merged (m, l, o) partial
};

constexpr int kMergeWarps = 8;

constexpr int kMergeCached = 10;  // parts per warp held in registers: rows of up to 80 parts

__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeParams p) {
    pdl_trigger();
    pdl_wait();
    __shared__ float red_m[kMergeWarps];
    __shared__ float red_acc[kMergeWarps][32];
    __shared__ float red_den[kMergeWarps];
    const int64_t row = blockIdx.x;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int d = blockIdx.y * 32 + lane;
    const float *base = p.parts + row * p.row_stride;
    float ma = -INFINITY;
    float den = 0.f, acc = 0.f;
    const int np = p.nparts;
    if (np <= kMergeWarps * kMergeCached) {
        // one round of loads: every (m, l, o[d]) of this warp's parts, then the maximum, the
        // weights and the sums from registers
        float mc[kMergeCached], lc[kMergeCached], oc[kMergeCached];
#pragma unroll
        for (int i = 0; i < kMergeCached; ++i) {
            const int c = warp + kMergeWarps * i;
            mc[i] = -INFINITY;
            lc[i] = oc[i] = 0.f;
            if (c < np) {
                const float *pc = base + c * p.part_stride;
                mc[i] = pc[0];
                lc[i] = pc[1];
                oc[i] = pc[2 + d];  // read even for an empty part: it is not summed
            }
        }
#pragma unroll
        for (int i = 0; i < kMergeCached; ++i)
            if (warp + kMergeWarps * i < np) ma = fmaxf(ma, mc[i]);
        if (lane == 0) red_m[warp] = ma;  // m is the same in every lane of the warp
        __syncthreads();
        ma = red_m[0];
#pragma unroll
        for (int w = 1; w < kMergeWarps; ++w) ma = fmaxf(ma, red_m[w]);
#pragma unroll
        for (int i = 0; i < kMergeCached; ++i) {
            if (warp + kMergeWarps * i < np && mc[i] != -INFINITY) {
                const float w = exp2f((mc[i] - ma) * kLog2e);
                den += lc[i] * w;
                acc += oc[i] * w;
            }
        }
    } else {
        for (int c = threadIdx.x; c < np; c += kMergeWarps * 32) ma = fmaxf(ma, base[c * p.part_stride]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
        if (lane == 0) red_m[warp] = ma;
        __syncthreads();
        ma = red_m[0];
#pragma unroll
        for (int w = 1; w < kMergeWarps; ++w) ma = fmaxf(ma, red_m[w]);
#pragma unroll 4
        for (int c = warp; c < np; c += kMergeWarps) {
            const float *pc = base + c * p.part_stride;
            const float mcv = pc[0];
            if (mcv == -INFINITY) continue;
            const float w = exp2f((mcv - ma) * kLog2e);
            den += pc[1] * w;
            acc += pc[2 + d] * w;
        }
    }
    red_acc[warp][lane] = acc;
    if (lane == 0) red_den[warp] = den;
    __syncthreads();
    if (warp != 0) return;
    acc = 0.f;
    den = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
        acc += red_acc[w][lane];
        den += red_den[w];
    }
    if (p.out_partial) {
        float *dst = p.out_partial + row * kPartial;
        dst[2 + d] = acc;
        if (blockIdx.y == 0 && lane == 0) {
            dst[0] = ma;
            dst[1] = den;
        }
        return;
    }
    float v = (den == 0.f) ? 0.f : acc / den;
    if (p.gate) {
        const float g = bf16_bits_to_f32(p.gate[row * p.gate_stride + d]);
        v = v * (1.0f / (1.0f + expf(-g)));
    }
    p.out[row * kHeadDim + d] = f32_to_bf16_bits(v);
}


// Merge for many rows with few parts (prefill key-range splits, context-parallel shards): one
// warp per row, grid-stride; lane l owns dims [8l, 8l + 8). The same arithmetic and part order
// as merge_kernel. A partial row is 258 floats, so its o[] is 8-byte aligned: float2 loads.
constexpr int kMergeRowsMaxParts = 16;

__global__ void __launch_bounds__(256) merge_rows_kernel(const float *parts, int64_t rows, int np,
                                                         int64_t part_stride, const uint16_t *gate,
                                                         uint16_t *out) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * 8;
    for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += nw) {
        const float *base = parts + row * kPartial;
        float ma = -INFINITY;
        for (int c = 0; c < np; ++c) ma = fmaxf(ma, base[c * part_stride]);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float den = 0.f;
        for (int c = 0; c < np; ++c) {
            const float *pc = base + c * part_stride;
            const float mc = pc[0];
            const float w = (mc == -INFINITY) ? 0.f : exp2f((mc - ma) * kLog2e);
            den += pc[1] * w;
            const float2 *o = reinterpret_cast<const float2 *>(pc + 2 + 8 * lane);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 v = o[k];
                acc[2 * k] += v.x * w;
                acc[2 * k + 1] += v.y * w;
            }
        }
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = (den == 0.f) ? 0.f : acc[k] / den;
        if (gate) {
            const uint4 gq = *reinterpret_cast<const uint4 *>(gate + row * kHeadDim + 8 * lane);
            const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float g = bf16_bits_to_f32((uint16_t)(gw[k >> 1] >> ((k & 1) * 16)));
                v[k] = v[k] * (1.0f / (1.0f + expf(-g)));
            }
        }
        uint4 q;
        q.x = (uint32_t)f32_to_bf16_bits(v[0]) | ((uint32_t)f32_to_bf16_bits(v[1]) << 16);
        q.y = (uint32_t)f32_to_bf16_bits(v[2]) | ((uint32_t)f32_to_bf16_bits(v[3]) << 16);
        q.z = (uint32_t)f32_to_bf16_bits(v[4]) | ((uint32_t)f32_to_bf16_bits(v[5]) << 16);
        q.w = (uint32_t)f32_to_bf16_bits(v[6]) | ((uint32_t)f32_to_bf16_bits(v[7]) << 16);
        *reinterpret_cast<uint4 *>(out + row * kHeadDim + 8 * lane) = q;
    }
}

}  // namespace

DecodePlan decode_plan(int batch, int max_seq_len, int sm_count) {
    const int64_t max_pages = (max_seq_len + kPage - 1) / kPage;
    const int64_t units = (int64_t)batch * kNumKvHeads * max_pages;
    // One wave of resident CTAs (2 per SM): fewer, longer splits amortise each CTA's prologue
    // and epilogue; long batches hit the 64-page cap anyway.
    const int64_t target_ctas = (int64_t)sm_count * 2;
    int64_t pps = (units + target_ctas - 1) / target_ctas;
    if (pps < kMinPagesPerSplit) pps = kMinPagesPerSplit;
    // The cap keeps a ragged batch's longest sequence from stretching the wave; one sequence has
    // no such spread, so its splits grow until one wave covers it (a 262144-token context-parallel
    // shard: 74 splits of 222 pages per kv head instead of 257 of 64).
    if (pps > kMaxPagesPerSplit && batch > 1) pps = kMaxPagesPerSplit;
    DecodePlan plan;
    plan.pages_per_split = (int)pps;
    plan.max_splits = (int)((max_pages + pps - 1) / pps);
    if (plan.max_splits < 1) plan.max_splits = 1;
    // The pre-wait prefetch pays where one wave of CTAs covers the grid (its ramp then
    // overlaps the previous kernel's tail); a many-wave grid keeps HBM busy on its own, and
    // there the extra hints cost bandwidth (config 4: 6388 -> 6251 GB/s with them).
    plan.prefetch_pre = (int64_t)batch * kNumKvHeads * plan.max_splits <= target_ctas ? kPrefetchPre : 0;
    plan.prefetch_ahead = kPrefetchAhead;
    return plan;
}

size_t decode_workspace_bytes(int batch, int num_queries, int max_seq_len, int sm_count) {
    const DecodePlan plan = decode_plan(batch, max_seq_len, sm_count);
    const size_t rows = (size_t)batch * num_queries * kNumQHeads;
    return rows * plan.max_splits * kPartial * sizeof(float);
}

cudaError_t launch_decode(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                          int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                          const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                          float scale, const uint16_t *gate, uint16_t *out, float *partials_out,
                          void *workspace, int sm_count, cudaStream_t stream,
                          const DecodeAppend *app, int64_t gate_stride, const void *k_pages,
                          const void *v_pages) {
    static std::atomic<bool> attr_set[64] = {};  // the attribute is per device context
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const DecodePlan plan = decode_plan(batch, max_seq_len, sm_count);
    SplitParams sp;
    sp.q = q;
    if (app != nullptr) sp.app = *app;
    sp.block_tables = block_tables;
    sp.seq_lens = seq_lens;
    sp.ws = static_cast<float *>(workspace);
    sp.num_pages = num_pages;
    sp.max_pages_per_seq = max_pages_per_seq;
    sp.num_queries = num_queries;
    sp.pages_per_split = plan.pages_per_split;
    sp.max_splits = plan.max_splits;
    sp.scale_log2 = scale * kLog2e;
    const bool pf = k_pages != nullptr && v_pages != nullptr;
    sp.prefetch_pre = pf ? plan.prefetch_pre : 0;
    sp.prefetch_ahead = pf ? plan.prefetch_ahead : 0;
    sp.k_base = static_cast<const uint8_t *>(k_pages);
    sp.v_base = static_cast<const uint8_t *>(v_pages);
    dim3 grid(plan.max_splits, kNumKvHeads, batch);
    cudaError_t le = app != nullptr
                         ? launch_pdl(decode_split_kernel<true>, grid, dim3(kThreads), kSmemBytes, stream, tk, tv, sp)
                         : launch_pdl(decode_split_kernel<false>, grid, dim3(kThreads), kSmemBytes, stream, tk, tv, sp);
    if (le != cudaSuccess) return le;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    MergeParams mp;
    mp.parts = sp.ws;
    mp.row_stride = (int64_t)plan.max_splits * kPartial;
    mp.part_stride = kPartial;
    mp.nparts = plan.max_splits;  // splits past a sequence's end left empty partials
    mp.gate = gate;
    mp.gate_stride = gate_stride;
    mp.out = out;
    mp.out_partial = partials_out;
    const int64_t rows = (int64_t)batch * num_queries * kNumQHeads;
    return launch_pdl(merge_kernel, dim3((unsigned)rows, kHeadDim / 32), dim3(kMergeWarps * 32), 0,
                      stream, mp);
}

cudaError_t launch_merge_partials(const float *partials, int64_t rows, int num_parts,
                                  int64_t part_stride, const uint16_t *gate, uint16_t *out,
                                  cudaStream_t stream) {
    MergeParams mp;
    mp.parts = partials;
    mp.row_stride = kPartial;
    mp.part_stride = part_stride;
    mp.nparts = num_parts;
    mp.gate = gate;
    mp.gate_stride = kHeadDim;
    mp.out = out;
    mp.out_partial = nullptr;
    if (num_parts <= kMergeRowsMaxParts && part_stride % 2 == 0 &&
        (reinterpret_cast<uintptr_t>(partials) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(gate) & 15) == 0) {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        int64_t blocks = (rows + 7) / 8;
        if (blocks > (int64_t)sms * 16) blocks = (int64_t)sms * 16;
        return launch_pdl(merge_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, partials,
                          rows, num_parts, part_stride, gate, out);
    }
    return launch_pdl(merge_kernel, dim3((unsigned)rows, kHeadDim / 32), dim3(kMergeWarps * 32), 0,
                      stream, mp);
}

// ------------------------------------------------------------------------------------------
// Context-parallel exchange over peer memory (BASELINE config 5b). Rank g holds one contiguous
// KV shard of a long sequence; the split kernel leaves its per-split partials in the
// workspace. The exchange kernel (one CTA per row and 32-dim chunk) then (1) LSE-merges those
// splits into the rank's partial slice (m, l, o[32 dims]), (2) stores the slice straight into
// every rank's exchange buffer over NVLink as 8-byte words that carry the value in the low half
// and the call's epoch in the high half, (3) polls its own buffer until every source rank's
// words of this slice carry the epoch (bounded) and (4) merges the world partials with the gate
// into the bf16 output. A 64-bit store is single-copy atomic, so a word whose flag is current
// holds the current value: no fence and no arrival counter sit between the stores and the
// reads (a system-scope fence after the remote stores cost 7-14 us per call). This replaces
// merge kernel + all-gather + merge kernel: launched right behind the split kernel
// (programmatic dependent launch), it is resident when the last split finishes.
// Exchange buffer per rank: [2 parities][world sources][16 rows][8 chunks][34 words] u64
// (o[32], m, l). It starts zeroed and epochs start at 1, so no stale word matches. Parity
// epoch & 1 double-buffers the records: rank r cannot start call e + 2 before every rank has
// sent it call e + 1, which each does only after finishing its reads of call e.
constexpr int kCpRows = kNumQHeads;

struct CpParams {
    const float *parts;  // split partials [16][max_splits][258]
    int max_splits;
    float *bufs[PGC_CP_MAX_RANKS];  // every rank's exchange buffer, as mapped in this process
    int world, rank;
    uint32_t epoch;
    const uint16_t *gate;
    int64_t gate_stride;  // elements between gate rows
    uint16_t *out;
};

constexpr int kCpWords = 34;  // one record: o[32], m, l

__device__ __forceinline__ int64_t cp_record(int parity, int world, int src, int row, int chunk) {
    return ((((int64_t)parity * world + src) * kCpRows + row) * (kHeadDim / 32) + chunk) * kCpWords;
}
__device__ __forceinline__ void cp_store_word(unsigned long long *a, float v, uint32_t epoch) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long cp_load_word(const unsigned long long *a) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

// One CTA per (row, 32-dim chunk), 128 CTAs: the 8 warps stride over the local splits (lane =
// dim), as the merge kernel does, so the L2 reads of up to 256 split partials per row overlap.
// Warp w stores the CTA's record (o slice, m, l) into rank w's buffer over NVLink; warp 0 then
// polls the records of every source rank in this rank's buffer and merges them.
__global__ void __launch_bounds__(256) cp_exchange_kernel(const CpParams p) {
    pdl_trigger();
    pdl_wait();
    __shared__ float wm[8], wden[8], wacc[8][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r = blockIdx.x, d0 = blockIdx.y * 32;
    const int np = p.max_splits;  // splits past the shard's end left empty partials
    const float *base = p.parts + (int64_t)r * p.max_splits * kPartial;
    float ma = -INFINITY;
    float den = 0.f, acc = 0.f;
    constexpr int kCached = 16;  // parts per warp held in registers: rows of up to 128 splits
    if (np <= 8 * kCached) {
        // one round of loads: every (m, l, o[d]) of this warp's splits, then the maximum, the
        // weights and the sums from registers (the order of the sums is the streaming path's)
        float mc[kCached], lc[kCached], oc[kCached];
#pragma unroll
        for (int i = 0; i < kCached; ++i) {
            const int c = warp + 8 * i;
            mc[i] = -INFINITY;
            lc[i] = oc[i] = 0.f;
            if (c < np) {
                const float *pc = base + (int64_t)c * kPartial;
                mc[i] = pc[0];
                lc[i] = pc[1];
                oc[i] = pc[2 + d0 + lane];  // read even for an empty part: it is not summed
            }
        }
#pragma unroll
        for (int i = 0; i < kCached; ++i) ma = fmaxf(ma, mc[i]);
        if (lane == 0) wm[warp] = ma;  // m is the same in every lane of the warp
        __syncthreads();
        ma = wm[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) ma = fmaxf(ma, wm[w]);
#pragma unroll
        for (int i = 0; i < kCached; ++i) {
            if (mc[i] != -INFINITY) {
                const float w = exp2f((mc[i] - ma) * kLog2e);
                den += lc[i] * w;
                acc += oc[i] * w;
            }
        }
    } else {
        for (int c = tid; c < np; c += 256) ma = fmaxf(ma, base[(int64_t)c * kPartial]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
        if (lane == 0) wm[warp] = ma;
        __syncthreads();
        ma = wm[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) ma = fmaxf(ma, wm[w]);
#pragma unroll 4
        for (int c = warp; c < np; c += 8) {
            const float *pc = base + (int64_t)c * kPartial;
            const float mc = pc[0];
            if (mc == -INFINITY) continue;
            const float w = exp2f((mc - ma) * kLog2e);
            den += pc[1] * w;
            acc += pc[2 + d0 + lane] * w;
        }
    }
    if (lane == 0) wden[warp] = den;
    wacc[warp][lane] = acc;
    __syncthreads();
    if (p.world == 1) {
        // nothing to exchange: the rank partial is the result (the same arithmetic as the
        // one-part merge below: weight exp2(0) = 1)
        if (warp == 0) {
            float sacc = 0.f, sden = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                sacc += wacc[w][lane];
                sden += wden[w];
            }
            const int dd = d0 + lane;
            const float d2 = (ma == -INFINITY) ? 0.f : sden;
            float v = (d2 == 0.f) ? 0.f : ((ma == -INFINITY) ? 0.f : sacc) / d2;
            if (p.gate) {
                const float g = bf16_bits_to_f32(p.gate[r * p.gate_stride + dd]);
                v = v * (1.0f / (1.0f + expf(-g)));
            }
            p.out[r * kHeadDim + dd] = f32_to_bf16_bits(v);
        }
        return;
    }
    // this CTA's record of the rank partial -> [parity][rank][r][chunk] of every rank's buffer
    const uint32_t epoch = p.epoch;
    const int parity = (int)(epoch & 1u);
    const int chunk = blockIdx.y;
    if (warp < p.world) {
        float sacc = 0.f, sden = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            sacc += wacc[w][lane];
            sden += wden[w];
        }
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(p.bufs[warp]) +
                                  cp_record(parity, p.world, p.rank, r, chunk);
        cp_store_word(dst + lane, sacc, epoch);
        if (lane == 0) cp_store_word(dst + 32, ma, epoch);
        if (lane == 1) cp_store_word(dst + 33, sden, epoch);
    }
    // Warp c polls source c's record of this slice in this rank's buffer until its words carry
    // this epoch (bounded), so the world's records are awaited in parallel rather than as one
    // chain of dependent round trips; warp 0 then merges them from shared memory in source order.
    __shared__ float xm[PGC_CP_MAX_RANKS], xl[PGC_CP_MAX_RANKS], xo[PGC_CP_MAX_RANKS][32];
    if (warp < p.world) {
        const int c = warp;
        const unsigned long long *rec =
            reinterpret_cast<const unsigned long long *>(p.bufs[p.rank]) + cp_record(parity, p.world, c, r, chunk);
        const uint64_t t0 = global_timer_ns();
        unsigned long long wo, wm, wl;
        for (uint32_t it = 0;; ++it) {
            wo = cp_load_word(rec + lane);
            wm = cp_load_word(rec + 32);
            wl = cp_load_word(rec + 33);
            const bool ready = (uint32_t)(wo >> 32) == epoch && (uint32_t)(wm >> 32) == epoch &&
                               (uint32_t)(wl >> 32) == epoch;
            if (__all_sync(0xffffffffu, ready)) break;
            if ((it & 63u) == 0) {
                // lane 0's clock decides, so the warp leaves the loop together
                const bool late = __shfl_sync(0xffffffffu, global_timer_ns() - t0 > 2000000000ull, 0);
                if (late) {
                    if (lane == 0) record_error(&g_decode_err, kErrWaitTimeout, 1000 + c);
                    break;
                }
            }
        }
        if (lane == 0) {
            xm[c] = __uint_as_float((uint32_t)wm);
            xl[c] = __uint_as_float((uint32_t)wl);
        }
        xo[c][lane] = __uint_as_float((uint32_t)wo);
    }
    __syncthreads();
    if (warp == 0) {
        float mv[PGC_CP_MAX_RANKS], lv[PGC_CP_MAX_RANKS], ov[PGC_CP_MAX_RANKS];
#pragma unroll
        for (int c = 0; c < PGC_CP_MAX_RANKS; ++c) {
            mv[c] = c < p.world ? xm[c] : -INFINITY;
            lv[c] = c < p.world ? xl[c] : 0.f;
            ov[c] = c < p.world ? xo[c][lane] : 0.f;
        }
        float m2 = -INFINITY;
        for (int c = 0; c < p.world; ++c) m2 = fmaxf(m2, mv[c]);
        float d2 = 0.f, a2 = 0.f;
        for (int c = 0; c < p.world; ++c) {
            const float mc = mv[c];
            const float w = (mc == -INFINITY) ? 0.f : exp2f((mc - m2) * kLog2e);
            d2 += lv[c] * w;
            a2 += ov[c] * w;
        }
        const int dd = d0 + lane;
        float v = (d2 == 0.f) ? 0.f : a2 / d2;
        if (p.gate) {
            const float g = bf16_bits_to_f32(p.gate[r * p.gate_stride + dd]);
            v = v * (1.0f / (1.0f + expf(-g)));
        }
        p.out[r * kHeadDim + dd] = f32_to_bf16_bits(v);
    }
}

size_t cp_buffer_bytes(int world) {
    return (size_t)2 * world * kCpRows * (kHeadDim / 32) * kCpWords * sizeof(unsigned long long);
}

cudaError_t launch_cp_decode(const uint16_t *q, const CUtensorMap &tk, const CUtensorMap &tv,
                             int64_t num_pages, const int32_t *block_table, int max_pages,
                             const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                             uint16_t *out, void *workspace, float *const *bufs, int world, int rank,
                             uint32_t epoch, int sm_count, cudaStream_t stream, const void *k_pages,
                             const void *v_pages, const DecodeAppend *app, int64_t gate_stride) {
    static std::atomic<bool> attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_split_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBytes);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const DecodePlan plan = decode_plan(1, max_seq_len, sm_count);
    SplitParams sp = {};
    sp.q = q;
    if (app != nullptr) sp.app = *app;
    sp.block_tables = block_table;
    sp.seq_lens = seq_len;
    sp.ws = static_cast<float *>(workspace);
    sp.num_pages = num_pages;
    sp.max_pages_per_seq = max_pages;
    sp.num_queries = 1;
    sp.pages_per_split = plan.pages_per_split;
    sp.max_splits = plan.max_splits;
    sp.scale_log2 = scale * kLog2e;
    const bool pf = k_pages != nullptr && v_pages != nullptr;
    sp.prefetch_pre = pf ? plan.prefetch_pre : 0;
    sp.prefetch_ahead = pf ? plan.prefetch_ahead : 0;
    sp.k_base = static_cast<const uint8_t *>(k_pages);
    sp.v_base = static_cast<const uint8_t *>(v_pages);
    const dim3 grid(plan.max_splits, kNumKvHeads, 1);
    cudaError_t e = app != nullptr
                        ? launch_pdl(decode_split_kernel<true>, grid, dim3(kThreads), kSmemBytes, stream, tk, tv, sp)
                        : launch_pdl(decode_split_kernel<false>, grid, dim3(kThreads), kSmemBytes, stream, tk, tv, sp);
    if (e != cudaSuccess) return e;
    CpParams cp;
    cp.parts = sp.ws;
    cp.max_splits = plan.max_splits;
    for (int i = 0; i < PGC_CP_MAX_RANKS; ++i) cp.bufs[i] = i < world ? bufs[i] : nullptr;
    cp.world = world;
    cp.rank = rank;
    cp.epoch = epoch;
    cp.gate = gate;
    cp.gate_stride = gate_stride;
    cp.out = out;
    return launch_pdl(cp_exchange_kernel, dim3(kCpRows, kHeadDim / 32), dim3(256), 0, stream, cp);
}

cudaError_t decode_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_decode_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_decode_err, &z, sizeof(DevError));
}

}  // namespace pgc

// ------------------------------------------------------------------------------------------
// Allocation-free decode entry (pgc_decode_attn_static). For callers that cannot call
// cudaMalloc at all, the split partials live in this fixed array. A GPU holds it from the
// library module's load on that device (with CUDA's lazy module loading: the first library
// call there) until the process exits. Every call shares it and it keeps the last
// call's contents; nothing in it needs to start at zero, because each call's split kernel
// writes every partial value its merge kernel uses. Two calls that overlap on the GPU (different
// streams, or different host threads on one device) race on it.
namespace pgc {

constexpr size_t kStaticScratchBytes = (size_t)PGC_DECODE_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_decode_static_scratch[kStaticScratchBytes];

int decode_static_scratch(void **ptr_out) {
    // Host code cannot use the array's name as a device address: resolve it once per device,
    // with that device current. The first call on a device does this set-up.
    static std::mutex mu;
    static void *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PGC_ERR_CUDA;
    std::lock_guard<std::mutex> lk(mu);
    if (addr[dev] == nullptr) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_decode_static_scratch) != cudaSuccess || p == nullptr)
            return PGC_ERR_CUDA;
        addr[dev] = p;
    }
    *ptr_out = addr[dev];
    return PGC_OK;
}

}  // namespace pgc
