// cache_copy.cu — byte-exact cache movement for prefix snapshot/restore, hidden rows, linear
// state and MTP rollback (sm_100a).
//
// The reference does all of this as host memcpy on CPU-visible Metal buffers
// (src/model/state.zig:124-230, src/server/prefix_state_cache.zig:584-629,
// src/server/decode_loop.zig:295-311). Here every copy is one kernel launch of 16-byte
// vector loads/stores, HBM-bound, reading and writing any memory the GPU can address
// (HBM, or pinned host memory for a host-resident prefix store).
#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_copy_err);

namespace {

int launch_blocks(int64_t work_items, int threads) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t want = (work_items + threads - 1) / threads;
    const int64_t cap = (int64_t)sms * 16;
    if (want > cap) want = cap;
    if (want < 1) want = 1;
    return (int)want;
}

// ---------------------------------------------------------------- row gather / scatter
template <typename V>
__global__ void __launch_bounds__(256)
    copy_rows_kernel(uint8_t *dst, const uint8_t *src, const int32_t *dst_rows,
                     const int32_t *src_rows, int64_t n_rows, int64_t units_per_row,
                     int64_t dst_pitch, int64_t src_pitch) {
    const int64_t total = n_rows * units_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / units_per_row;
        const int64_t u = i - r * units_per_row;
        const int64_t dr = dst_rows ? dst_rows[r] : r;
        const int64_t sr = src_rows ? src_rows[r] : r;
        reinterpret_cast<V *>(dst + dr * dst_pitch)[u] =
            reinterpret_cast<const V *>(src + sr * src_pitch)[u];
    }
}

// ---------------------------------------------------------------- dense <-> paged KV
// Resolves logical token t of a paged sequence to the element offset of its (kvh) row, or -1
// (recorded) when the table entry or the page id is out of range.
__device__ __forceinline__ int64_t paged_row(const int32_t *table, int64_t n_table,
                                             int64_t num_pages, int64_t t, int kvh) {
    const int64_t pi = t / kPage;
    if (t < 0 || pi >= n_table) {
        record_error(&g_copy_err, kErrTableOutOfRange, t);
        return -1;
    }
    const int64_t page = table[pi];
    if (page < 0 || page >= num_pages) {
        record_error(&g_copy_err, kErrPageOutOfRange, page);
        return -1;
    }
    return ((page * kNumKvHeads + kvh) * kPage + t % kPage) * kHeadDim;
}

constexpr int kDenseTile = 32;  // tokens per CTA

// One CTA per (32-token tile, kv head). K rows are 512 B in both layouts (uint4 copies);
// V is value-dim-major in the dense layout and token-major in the pages, so it is
// transposed through shared memory: coalesced 64-byte runs on the dense side, whole 512-byte
// rows on the page side.
template <typename KV>
__global__ void __launch_bounds__(256)
    kv_dense_kernel(bool restore, uint16_t *dk, uint16_t *dv, int64_t dstride, int64_t dtok,
                    uint16_t *kp, uint16_t *vp, int64_t num_pages, const int32_t *table,
                    int64_t n_table, int64_t ptok, int64_t count) {
    __shared__ uint16_t vt[kHeadDim][kDenseTile + 2];
    __shared__ int64_t rows[kDenseTile];
    const int kvh = blockIdx.y;
    const int64_t base = (int64_t)blockIdx.x * kDenseTile;
    const int n = (int)(count - base < kDenseTile ? count - base : kDenseTile);
    const int tid = threadIdx.x;
    if (tid < kDenseTile) rows[tid] = tid < n ? paged_row(table, n_table, num_pages, ptok + base + tid, kvh) : -1;
    __syncthreads();

    // K: 32 tokens x one 512-byte row each, in units of KV (16 B when the dense side is
    // 16-byte aligned; a file image's runs may only be 4- or 2-byte aligned)
    constexpr int kUnits = kHeadDim * 2 / (int)sizeof(KV);
    for (int i = tid; i < n * kUnits; i += 256) {
        const int tt = i / kUnits, u = i % kUnits;
        const int64_t pr = rows[tt];
        if (pr < 0) continue;
        KV *prow = reinterpret_cast<KV *>(kp + pr);
        KV *drow = reinterpret_cast<KV *>(dk + ((int64_t)kvh * dstride + dtok + base + tt) * kHeadDim);
        if (restore) prow[u] = drow[u];
        else drow[u] = prow[u];
    }
    // V
    if (restore) {
        for (int i = tid; i < kHeadDim * kDenseTile; i += 256) {
            const int d = i / kDenseTile, tt = i % kDenseTile;
            if (tt < n) vt[d][tt] = dv[((int64_t)kvh * kHeadDim + d) * dstride + dtok + base + tt];
        }
        __syncthreads();
        for (int i = tid; i < n * kHeadDim; i += 256) {
            const int tt = i / kHeadDim, d = i % kHeadDim;
            const int64_t pr = rows[tt];
            if (pr >= 0) vp[pr + d] = vt[d][tt];
        }
    } else {
        for (int i = tid; i < n * kHeadDim; i += 256) {
            const int tt = i / kHeadDim, d = i % kHeadDim;
            const int64_t pr = rows[tt];
            vt[d][tt] = pr >= 0 ? vp[pr + d] : 0;
        }
        __syncthreads();
        for (int i = tid; i < kHeadDim * kDenseTile; i += 256) {
            const int d = i / kDenseTile, tt = i % kDenseTile;
            if (tt < n && rows[tt] >= 0)
                dv[((int64_t)kvh * kHeadDim + d) * dstride + dtok + base + tt] = vt[d][tt];
        }
    }
}

// Vector form of kv_dense_kernel for a 16-byte aligned dense side (dense stride and first
// token multiples of 8): one CTA per (64-token tile, kv head), no shared-memory staging.
// Each thread moves one 8x8 block of V (8 value dims x 8 tokens): eight 16-byte loads along
// the source's contiguous axis, an in-register transpose of 16-bit elements (byte permutes),
// eight 16-byte stores along the destination's contiguous axis. A warp covers 2 token chunks x
// 16 dim blocks, so the dense side moves whole 32-byte sectors and the page side 256-byte row
// halves. K rows are 512 B in both layouts: eight independent 16-byte copies per thread.
constexpr int kVecTile = 64;

__device__ __forceinline__ void transpose8x8_u16(const uint32_t (&in)[8][4], uint32_t (&out)[8][4]) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int m = 0; m < 4; ++m)
            out[k][m] = __byte_perm(in[2 * m][k >> 1], in[2 * m + 1][k >> 1],
                                    (k & 1) ? 0x7632u : 0x5410u);
}

__device__ __forceinline__ void ld4(uint32_t (&r)[4], const uint16_t *p) {
    const uint4 v = *reinterpret_cast<const uint4 *>(p);
    r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
}

__device__ __forceinline__ void st4(uint16_t *p, const uint32_t (&r)[4]) {
    *reinterpret_cast<uint4 *>(p) = make_uint4(r[0], r[1], r[2], r[3]);
}

__global__ void __launch_bounds__(256)
    kv_dense_vec_kernel(bool restore, uint16_t *dk, uint16_t *dv, int64_t dstride, int64_t dtok,
                        uint16_t *kp, uint16_t *vp, int64_t num_pages, const int32_t *table,
                        int64_t n_table, int64_t ptok, int64_t count) {
    __shared__ int64_t rows[kVecTile];
    const int kvh = blockIdx.y;
    const int64_t base = (int64_t)blockIdx.x * kVecTile;
    const int n = (int)(count - base < kVecTile ? count - base : kVecTile);
    const int tid = threadIdx.x;
    if (tid < kVecTile) rows[tid] = tid < n ? paged_row(table, n_table, num_pages, ptok + base + tid, kvh) : -1;
    __syncthreads();

    // K: 64 tokens x 32 uint4, loads first for memory-level parallelism
    {
        uint4 buf[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + j * 256, tt = i >> 5, u = i & 31;
            if (tt < n && rows[tt] >= 0) {
                const uint4 *src = restore
                    ? reinterpret_cast<const uint4 *>(dk + ((int64_t)kvh * dstride + dtok + base + tt) * kHeadDim) + u
                    : reinterpret_cast<const uint4 *>(kp + rows[tt]) + u;
                buf[j] = *src;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + j * 256, tt = i >> 5, u = i & 31;
            if (tt < n && rows[tt] >= 0) {
                uint4 *dst = restore
                    ? reinterpret_cast<uint4 *>(kp + rows[tt]) + u
                    : reinterpret_cast<uint4 *>(dk + ((int64_t)kvh * dstride + dtok + base + tt) * kHeadDim) + u;
                *dst = buf[j];
            }
        }
    }

    // V: one 8x8 block per thread
    const int w = tid >> 5, l = tid & 31;
    const int d0 = ((l & 15) + 16 * (w >> 2)) * 8;
    const int t0 = (2 * (w & 3) + (l >> 4)) * 8;
    if (t0 >= n) return;
    bool full = t0 + 8 <= n;
#pragma unroll
    for (int k = 0; k < 8; ++k) full = full && rows[t0 + k] >= 0;
    uint16_t *dcol = dv + ((int64_t)kvh * kHeadDim + d0) * dstride + dtok + base + t0;
    if (full) {
        uint32_t a[8][4], b[8][4];
        if (restore) {
#pragma unroll
            for (int r = 0; r < 8; ++r) ld4(a[r], dcol + (int64_t)r * dstride);
            transpose8x8_u16(a, b);
#pragma unroll
            for (int k = 0; k < 8; ++k) st4(vp + rows[t0 + k] + d0, b[k]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) ld4(a[k], vp + rows[t0 + k] + d0);
            transpose8x8_u16(a, b);
#pragma unroll
            for (int r = 0; r < 8; ++r) st4(dcol + (int64_t)r * dstride, b[r]);
        }
        return;
    }
    // ragged tail chunk (or a token whose row failed to resolve): element by element
    const int m = n - t0 < 8 ? n - t0 : 8;
    for (int k = 0; k < m; ++k) {
        const int64_t pr = rows[t0 + k];
        if (pr < 0) continue;
        for (int r = 0; r < 8; ++r) {
            if (restore) vp[pr + d0 + r] = dcol[(int64_t)r * dstride + k];
            else dcol[(int64_t)r * dstride + k] = vp[pr + d0 + r];
        }
    }
}

// paged -> paged, one warp per (token, kv head): 512 B of K and 512 B of V
__global__ void __launch_bounds__(256)
    kv_copy_tokens_kernel(const uint16_t *sk, const uint16_t *sv, int64_t s_pages,
                          const int32_t *s_table, int64_t s_n, int64_t s_tok, uint16_t *dk,
                          uint16_t *dv, int64_t d_pages, const int32_t *d_table, int64_t d_n,
                          int64_t d_tok, int64_t count) {
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= count * kNumKvHeads) return;
    const int64_t i = gw / kNumKvHeads;
    const int kvh = (int)(gw % kNumKvHeads);
    int64_t so = 0, dof = 0;
    if (lane == 0) {
        so = paged_row(s_table, s_n, s_pages, s_tok + i, kvh);
        dof = paged_row(d_table, d_n, d_pages, d_tok + i, kvh);
    }
    so = __shfl_sync(0xffffffffu, so, 0);
    dof = __shfl_sync(0xffffffffu, dof, 0);
    if (so < 0 || dof < 0) return;
    reinterpret_cast<uint4 *>(dk + dof)[lane] = reinterpret_cast<const uint4 *>(sk + so)[lane];
    reinterpret_cast<uint4 *>(dv + dof)[lane] = reinterpret_cast<const uint4 *>(sv + so)[lane];
}

// ---------------------------------------------------------------- batched regions
struct RegionTable {
    uint8_t *dst[PGC_MAX_REGIONS];
    const uint8_t *src[PGC_MAX_REGIONS];
    int64_t begin[PGC_MAX_REGIONS + 1];  // prefix sums of units
    int32_t unit[PGC_MAX_REGIONS];       // 16 (vector) or 1 (byte) bytes per unit
    int n;
    int zero;
    const int32_t *accept;  // rollback: skip everything when *accept != 0
    int32_t *seq_lens;
    int seq_index;
    int reject_tokens;
};

__global__ void __launch_bounds__(256) regions_kernel(const __grid_constant__ RegionTable rt) {
    if (rt.accept != nullptr) {
        if (*rt.accept != 0) return;
        if (blockIdx.x == 0 && threadIdx.x == 0) rt.seq_lens[rt.seq_index] -= rt.reject_tokens;
    }
    const int64_t total = rt.begin[rt.n];
    int r = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        while (i >= rt.begin[r + 1]) ++r;  // i only grows within a thread
        const int64_t u = i - rt.begin[r];
        if (rt.unit[r] == 16) {
            uint4 v = rt.zero ? make_uint4(0, 0, 0, 0) : reinterpret_cast<const uint4 *>(rt.src[r])[u];
            reinterpret_cast<uint4 *>(rt.dst[r])[u] = v;
        } else {
            rt.dst[r][u] = rt.zero ? 0 : rt.src[r][u];
        }
    }
}

}  // namespace

cudaError_t launch_copy_rows(void *dst, const void *src, const int32_t *dst_rows,
                             const int32_t *src_rows, int64_t n_rows, int64_t row_bytes,
                             int64_t dst_pitch, int64_t src_pitch, cudaStream_t stream) {
    if (n_rows == 0 || row_bytes == 0) return cudaSuccess;
    auto aligned = [](int64_t v, int64_t a) { return v % a == 0; };
    const int64_t ad = (int64_t)(uintptr_t)dst, as = (int64_t)(uintptr_t)src;
    int vec = 1;
    if (aligned(ad, 16) && aligned(as, 16) && aligned(row_bytes, 16) && aligned(dst_pitch, 16) &&
        aligned(src_pitch, 16))
        vec = 16;
    else if (aligned(ad, 4) && aligned(as, 4) && aligned(row_bytes, 4) && aligned(dst_pitch, 4) &&
             aligned(src_pitch, 4))
        vec = 4;
    const int64_t upr = row_bytes / vec;
    const int blocks = launch_blocks(n_rows * upr, 256);
    uint8_t *d = static_cast<uint8_t *>(dst);
    const uint8_t *s = static_cast<const uint8_t *>(src);
    if (vec == 16)
        copy_rows_kernel<uint4><<<blocks, 256, 0, stream>>>(d, s, dst_rows, src_rows, n_rows, upr, dst_pitch, src_pitch);
    else if (vec == 4)
        copy_rows_kernel<uint32_t><<<blocks, 256, 0, stream>>>(d, s, dst_rows, src_rows, n_rows, upr, dst_pitch, src_pitch);
    else
        copy_rows_kernel<uint8_t><<<blocks, 256, 0, stream>>>(d, s, dst_rows, src_rows, n_rows, upr, dst_pitch, src_pitch);
    return cudaGetLastError();
}

cudaError_t launch_kv_dense(bool restore, uint16_t *dense_k, uint16_t *dense_v,
                            int64_t dense_stride, int64_t dense_token, uint16_t *k_pages,
                            uint16_t *v_pages, int64_t num_pages, const int32_t *table,
                            int64_t n_table, int64_t page_token, int64_t count,
                            cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    dim3 grid((unsigned)((count + kDenseTile - 1) / kDenseTile), kNumKvHeads);
    const uintptr_t a = reinterpret_cast<uintptr_t>(dense_k);
    const uintptr_t av = reinterpret_cast<uintptr_t>(dense_v);
    if (a % 16 == 0 && av % 16 == 0 && dense_stride % 8 == 0 && dense_token % 8 == 0) {
        dim3 vgrid((unsigned)((count + kVecTile - 1) / kVecTile), kNumKvHeads);
        kv_dense_vec_kernel<<<vgrid, 256, 0, stream>>>(restore, dense_k, dense_v, dense_stride,
                                                       dense_token, k_pages, v_pages, num_pages,
                                                       table, n_table, page_token, count);
    } else if (a % 16 == 0)
        kv_dense_kernel<uint4><<<grid, 256, 0, stream>>>(restore, dense_k, dense_v, dense_stride,
                                                         dense_token, k_pages, v_pages, num_pages,
                                                         table, n_table, page_token, count);
    else if (a % 4 == 0)
        kv_dense_kernel<uint32_t><<<grid, 256, 0, stream>>>(restore, dense_k, dense_v, dense_stride,
                                                            dense_token, k_pages, v_pages, num_pages,
                                                            table, n_table, page_token, count);
    else
        kv_dense_kernel<uint16_t><<<grid, 256, 0, stream>>>(restore, dense_k, dense_v, dense_stride,
                                                            dense_token, k_pages, v_pages, num_pages,
                                                            table, n_table, page_token, count);
    return cudaGetLastError();
}

cudaError_t launch_kv_copy_tokens(const uint16_t *sk, const uint16_t *sv, int64_t s_pages,
                                  const int32_t *s_table, int64_t s_n, int64_t s_tok,
                                  uint16_t *dk, uint16_t *dv, int64_t d_pages,
                                  const int32_t *d_table, int64_t d_n, int64_t d_tok,
                                  int64_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const int64_t blocks = (count * kNumKvHeads + 7) / 8;
    kv_copy_tokens_kernel<<<(unsigned)blocks, 256, 0, stream>>>(sk, sv, s_pages, s_table, s_n, s_tok,
                                                                dk, dv, d_pages, d_table, d_n, d_tok, count);
    return cudaGetLastError();
}

cudaError_t launch_regions(const pgc_region *regions, int n, bool zero, const int32_t *accept,
                           int32_t *seq_lens, int seq_index, int reject_tokens,
                           cudaStream_t stream) {
    RegionTable rt;
    memset(&rt, 0, sizeof(rt));
    rt.n = n;
    rt.zero = zero ? 1 : 0;
    rt.accept = accept;
    rt.seq_lens = seq_lens;
    rt.seq_index = seq_index;
    rt.reject_tokens = reject_tokens;
    int64_t acc = 0;
    for (int i = 0; i < n; ++i) {
        rt.dst[i] = static_cast<uint8_t *>(regions[i].dst);
        rt.src[i] = static_cast<const uint8_t *>(regions[i].src);
        const uintptr_t a = (uintptr_t)regions[i].dst | (zero ? 0 : (uintptr_t)regions[i].src);
        const bool v16 = (a % 16 == 0) && (regions[i].bytes % 16 == 0);
        rt.unit[i] = v16 ? 16 : 1;
        rt.begin[i] = acc;
        acc += (int64_t)(regions[i].bytes / rt.unit[i]);
    }
    rt.begin[n] = acc;
    if (acc == 0 && accept == nullptr) return cudaSuccess;
    const int blocks = launch_blocks(acc, 256);
    regions_kernel<<<blocks, 256, 0, stream>>>(rt);
    return cudaGetLastError();
}

cudaError_t copy_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_copy_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_copy_err, &z, sizeof(DevError));
}

}  // namespace pgc
