// capi.cpp — the extern "C" boundary of libperegrine_cuda.so (declared in
// include/peregrine_cuda.h).
//
// Role of the reference's Objective-C bridge (src/runtime/bridge.h:1-103, bridge.m): a flat
// C ABI that a Zig host binds with @cImport / extern. Each entry validates shapes, bounds and
// alignment on the host (the reference's kernels only early-return on bad shapes,
// attention_decode.metal:45-48), resolves per-device state (SM count, cached TMA
// descriptors) and enqueues the kernels on the caller's stream. No entry allocates device
// memory: workspaces are caller-owned, as buffers are in the reference (bridge.h:14-16).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>

#include "pgc_internal.h"

namespace pgc {
namespace {

std::mutex g_mu;

struct MapKey {
    int dev;
    const void *ptr;
    int64_t pages;
    bool operator==(const MapKey &o) const { return dev == o.dev && ptr == o.ptr && pages == o.pages; }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.ptr) ^ (std::hash<int64_t>()(k.pages) * 31) ^ (size_t)k.dev;
    }
};
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    // resolved once; a function-local static is initialised exactly once across threads
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return nullptr;
    }();
    return fn;
}

// per-device facts, cached on first use (atomics: host threads may make first calls at once;
// racing writers store the same values)
std::atomic<int> g_sm_count[64] = {};
std::atomic<int> g_arch_ok[64] = {};  // 0 unknown, 1 ok, -1 not sm_100

int check_device(int *dev_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return PGC_ERR_CUDA;
    if (dev < 0 || dev >= 64) return PGC_ERR_DEVICE;
    if (g_arch_ok[dev] == 0) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return PGC_ERR_CUDA;
        g_sm_count[dev] = sms;
        g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
    }
    if (g_arch_ok[dev] != 1) return PGC_ERR_DEVICE;
    if (dev_out) *dev_out = dev;
    return PGC_OK;
}

inline bool al16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? PGC_OK : PGC_ERR_CUDA; }

}  // namespace

int current_sm_count() {
    int dev = 0;
    if (check_device(&dev) != PGC_OK) return 148;
    return g_sm_count[dev];
}

int pool_tensor_map(const void *pool, int64_t num_pages, CUtensorMap *out) {
    int dev = 0;
    int st = check_device(&dev);
    if (st != PGC_OK) return st;
    std::lock_guard<std::mutex> lk(g_mu);
    MapKey key{dev, pool, num_pages};
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return PGC_OK;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return PGC_ERR_CUDA;
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)PGC_HEAD_DIM, (cuuint64_t)num_pages * 4 * 16};
    const cuuint64_t strides[1] = {(cuuint64_t)PGC_HEAD_DIM * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(pool), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return PGC_ERR_CUDA;
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return PGC_OK;
}

int q_tensor_map(const void *q, int tokens, CUtensorMap *out) {
    int dev = 0;
    int st = check_device(&dev);
    if (st != PGC_OK) return st;
    std::lock_guard<std::mutex> lk(g_mu);
    MapKey key{dev, q, -(int64_t)tokens - 1};  // negative: distinct from pool keys
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return PGC_OK;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return PGC_ERR_CUDA;
    CUtensorMap m;
    const cuuint64_t dims[3] = {(cuuint64_t)PGC_HEAD_DIM, (cuuint64_t)PGC_NUM_Q_HEADS,
                                (cuuint64_t)tokens};
    const cuuint64_t strides[2] = {(cuuint64_t)PGC_HEAD_DIM * 2,
                                   (cuuint64_t)PGC_HEAD_DIM * PGC_NUM_Q_HEADS * 2};
    const cuuint32_t box[3] = {64, 4, 32};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(q), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return PGC_ERR_CUDA;
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return PGC_OK;
}

// 2-D tiled tensor map over a row-major [outer][inner] array (elem_bytes 2 or 4), cached by
// pointer and shape. Used by the q4 projection for its activations and packed weights.
int tiled_map_2d(const void *ptr, int elem_bytes, int64_t inner, int64_t outer, int box_inner,
                 int box_outer, bool swizzle128, CUtensorMap *out) {
    int dev = 0;
    int st = check_device(&dev);
    if (st != PGC_OK) return st;
    struct Key {
        int dev;
        const void *ptr;
        int64_t a, b, c;
        bool operator<(const Key &o) const {
            return std::tie(dev, ptr, a, b, c) < std::tie(o.dev, o.ptr, o.a, o.b, o.c);
        }
    };
    static std::map<Key, CUtensorMap> cache;
    const Key key{dev, ptr, inner * 8 + elem_bytes, outer, (int64_t)box_inner << 32 | box_outer << 1 | (swizzle128 ? 1 : 0)};
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return PGC_OK;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return PGC_ERR_CUDA;
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)(inner * elem_bytes)};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&m, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 2,
                    const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return PGC_ERR_CUDA;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return PGC_OK;
}

}  // namespace pgc

using namespace pgc;

extern "C" {

const char *pgc_status_string(int status) {
    switch (status) {
        case PGC_OK: return "ok";
        case PGC_ERR_INVALID: return "invalid argument";
        case PGC_ERR_BOUNDS: return "index or length out of bounds";
        case PGC_ERR_WORKSPACE: return "workspace too small";
        case PGC_ERR_CUDA: return "CUDA error";
        case PGC_ERR_ALIGN: return "misaligned pointer or size";
        case PGC_ERR_DEVICE: return "current device is not sm_100";
        case PGC_ERR_TIMEOUT: return "bounded device wait timed out";
        case PGC_ERR_CONTEXT: return "invalid context length";
        case PGC_ERR_FILE: return "file missing or not accessible";
        case PGC_ERR_FORMAT: return "prefix-state file failed validation";
        case PGC_ERR_CAPACITY: return "page pool or state slots exhausted";
        case PGC_ERR_NCCL: return "NCCL unavailable or an NCCL call failed";
        default: return "unknown status";
    }
}

int pgc_version(void) { return 100; }

int pgc_device_error(int *code_out, int64_t *detail_out, int clear) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (cudaDeviceSynchronize() != cudaSuccess) return PGC_ERR_CUDA;
    DevErrorHost e[7] = {};
    cudaError_t r = decode_read_error(&e[0], clear != 0);
    if (r == cudaSuccess) r = append_read_error(&e[1], clear != 0);
    if (r == cudaSuccess) r = copy_read_error(&e[2], clear != 0);
    if (r == cudaSuccess) r = prefill_read_error(&e[3], clear != 0);
    if (r == cudaSuccess) r = linear_read_error(&e[4], clear != 0);
    if (r == cudaSuccess) r = q4_read_error(&e[5], clear != 0);
    if (r == cudaSuccess) r = prefill_linear_read_error(&e[6], clear != 0);
    if (r != cudaSuccess) return PGC_ERR_CUDA;
    int code = 0;
    long long detail = 0;
    for (int i = 0; i < 7 && code == 0; ++i)
        if (e[i].code != 0) {
            code = e[i].code + 100 * i;  // unit in the hundreds digit
            detail = e[i].detail;
        }
    if (code_out) *code_out = code;
    if (detail_out) *detail_out = detail;
    return PGC_OK;
}

int pgc_full_cache_stride_for_max_seq(uint64_t max_seq, uint64_t *stride_out) {
    if (!stride_out) return PGC_ERR_INVALID;
    if (max_seq == 0 || max_seq > PGC_MAX_CONTEXT_TOKENS) return PGC_ERR_CONTEXT;
    const uint64_t a = max_seq >= 16000 ? 64 : 256;
    const uint64_t r = max_seq % a;
    *stride_out = r == 0 ? max_seq : max_seq + (a - r);
    return PGC_OK;
}

int pgc_rope_table_fill(float *table_host, int64_t max_pos, int rot_dim, double theta) {
    if (!table_host || max_pos <= 0 || rot_dim <= 0 || (rot_dim & 1) || !(theta > 0.0))
        return PGC_ERR_INVALID;
    const int half = rot_dim / 2;
    for (int64_t p = 0; p < max_pos; ++p)
        for (int i = 0; i < half; ++i) {
            const double inv_freq = std::pow(theta, -(2.0 * (double)i) / (double)rot_dim);
            const double ang = (double)p * inv_freq;
            table_host[p * rot_dim + i] = (float)std::cos(ang);
            table_host[p * rot_dim + half + i] = (float)std::sin(ang);
        }
    return PGC_OK;
}

int pgc_append_kv_rope(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                       uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                       const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                       const float *rope_table, int64_t rope_max_pos,
                       const int32_t *positions, const int64_t *slot_mapping, int64_t tokens,
                       uint16_t *k_pages, uint16_t *v_pages, int64_t num_pages, int mode,
                       void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (tokens < 0 || num_pages <= 0 || rope_max_pos <= 0) return PGC_ERR_INVALID;
    if (mode != PGC_APPEND_DECODE && mode != PGC_APPEND_PREFILL) return PGC_ERR_INVALID;
    if (q_head_stride != PGC_HEAD_DIM && q_head_stride != 2 * PGC_HEAD_DIM) return PGC_ERR_INVALID;
    if (gate_out && q_head_stride != 2 * PGC_HEAD_DIM) return PGC_ERR_INVALID;
    if (tokens == 0) return PGC_OK;
    if (!q_in || !q_out || !k_in || !v_in || !rope_table || !positions || !slot_mapping ||
        !k_pages || !v_pages)
        return PGC_ERR_INVALID;
    if (!al16(v_in) || !al16(v_pages) || !al16(k_pages)) return PGC_ERR_ALIGN;
    return cuda_status(launch_append(q_in, q_head_stride, q_out, gate_out, k_in, v_in, q_norm_w,
                                     k_norm_w, rope_table, rope_max_pos, positions, slot_mapping,
                                     tokens, k_pages, v_pages, num_pages, mode,
                                     static_cast<cudaStream_t>(stream)));
}

size_t pgc_decode_workspace_bytes(int batch, int num_queries, int max_seq_len) {
    if (batch <= 0 || num_queries <= 0 || max_seq_len <= 0) return 0;
    return decode_workspace_bytes(batch, num_queries, max_seq_len, current_sm_count());
}

static int decode_checks(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                         int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                         const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                         void *workspace, size_t workspace_bytes) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!q || !k_pages || !v_pages || !block_tables || !seq_lens) return PGC_ERR_INVALID;
    if (batch <= 0 || num_queries < 1 || num_queries > PGC_MAX_QUERIES || max_seq_len <= 0 ||
        num_pages <= 0 || max_pages_per_seq <= 0)
        return PGC_ERR_INVALID;
    if ((int64_t)max_pages_per_seq * PGC_PAGE_TOKENS < max_seq_len) return PGC_ERR_BOUNDS;
    if (num_pages * 4 * 16 > INT32_MAX) return PGC_ERR_BOUNDS;  // TMA row coordinate is int32
    if (!al16(q) || !al16(k_pages) || !al16(v_pages) || !al16(workspace)) return PGC_ERR_ALIGN;
    if (workspace_bytes < decode_workspace_bytes(batch, num_queries, max_seq_len, current_sm_count()))
        return PGC_ERR_WORKSPACE;
    if (!workspace) return PGC_ERR_WORKSPACE;
    return PGC_OK;
}

int pgc_decode_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                    int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                    const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                    float scale, const uint16_t *gate, uint16_t *out, void *workspace,
                    size_t workspace_bytes, void *stream) {
    int st = decode_checks(q, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                           seq_lens, batch, num_queries, max_seq_len, workspace, workspace_bytes);
    if (st != PGC_OK) return st;
    if (!out || !std::isfinite(scale)) return PGC_ERR_INVALID;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    return cuda_status(launch_decode(q, tk, tv, num_pages, block_tables, max_pages_per_seq, seq_lens,
                                     batch, num_queries, max_seq_len, scale, gate, out, nullptr,
                                     workspace, current_sm_count(),
                                     static_cast<cudaStream_t>(stream), nullptr, PGC_HEAD_DIM,
                                     k_pages, v_pages));
}

int pgc_decode_attn_append(const uint16_t *q_in, int q_head_stride, const uint16_t *k_in,
                           const uint16_t *v_in, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                           const float *rope_table, int64_t rope_max_pos, const int32_t *positions,
                           const int64_t *slot_mapping, uint16_t *k_pages, uint16_t *v_pages,
                           int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                           const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                           float scale, uint16_t *out, void *workspace, size_t workspace_bytes,
                           void *stream) {
    int st = decode_checks(q_in, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                           seq_lens, batch, num_queries, max_seq_len, workspace, workspace_bytes);
    if (st != PGC_OK) return st;
    if (!out || !std::isfinite(scale) || !k_in || !v_in || !rope_table || !positions || !slot_mapping ||
        rope_max_pos <= 0)
        return PGC_ERR_INVALID;
    if (q_head_stride != PGC_HEAD_DIM && q_head_stride != 2 * PGC_HEAD_DIM) return PGC_ERR_INVALID;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    DecodeAppend app;
    app.q_in = q_in;
    app.q_head_stride = q_head_stride;
    app.k_in = k_in;
    app.v_in = v_in;
    app.q_norm_w = q_norm_w;
    app.k_norm_w = k_norm_w;
    app.rope = rope_table;
    app.rope_max_pos = rope_max_pos;
    app.positions = positions;
    app.slots = slot_mapping;
    app.k_pages = k_pages;
    app.v_pages = v_pages;
    app.num_pages = num_pages;
    // packed q | gate rows: the gate is the second half of each 512-wide head row
    const uint16_t *gate = q_head_stride == 2 * PGC_HEAD_DIM ? q_in + PGC_HEAD_DIM : nullptr;
    return cuda_status(launch_decode(nullptr, tk, tv, num_pages, block_tables, max_pages_per_seq, seq_lens,
                                     batch, num_queries, max_seq_len, scale, gate, out, nullptr, workspace,
                                     current_sm_count(), static_cast<cudaStream_t>(stream), &app,
                                     q_head_stride, k_pages, v_pages));
}

int pgc_decode_attn_static(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                           int64_t num_pages, const int32_t *block_tables,
                           int max_pages_per_seq, const int32_t *seq_lens, int batch,
                           int num_queries, int max_seq_len, float scale, const uint16_t *gate,
                           uint16_t *out, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (batch <= 0 || num_queries < 1 || num_queries > PGC_MAX_QUERIES || max_seq_len <= 0)
        return PGC_ERR_INVALID;
    const size_t need = decode_workspace_bytes(batch, num_queries, max_seq_len, current_sm_count());
    if (need > (size_t)PGC_DECODE_STATIC_SCRATCH_BYTES) return PGC_ERR_WORKSPACE;
    void *scratch = nullptr;
    if ((st = decode_static_scratch(&scratch)) != PGC_OK) return st;
    return pgc_decode_attn(q, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                           seq_lens, batch, num_queries, max_seq_len, scale, gate, out, scratch,
                           (size_t)PGC_DECODE_STATIC_SCRATCH_BYTES, stream);
}

int pgc_decode_attn_partials(const uint16_t *q, const uint16_t *k_pages,
                             const uint16_t *v_pages, int64_t num_pages,
                             const int32_t *block_tables, int max_pages_per_seq,
                             const int32_t *seq_lens, int batch, int num_queries,
                             int max_seq_len, float scale, float *partials, void *workspace,
                             size_t workspace_bytes, void *stream) {
    int st = decode_checks(q, k_pages, v_pages, num_pages, block_tables, max_pages_per_seq,
                           seq_lens, batch, num_queries, max_seq_len, workspace, workspace_bytes);
    if (st != PGC_OK) return st;
    if (!partials || !std::isfinite(scale)) return PGC_ERR_INVALID;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    return cuda_status(launch_decode(q, tk, tv, num_pages, block_tables, max_pages_per_seq, seq_lens,
                                     batch, num_queries, max_seq_len, scale, nullptr, nullptr,
                                     partials, workspace, current_sm_count(),
                                     static_cast<cudaStream_t>(stream), nullptr, PGC_HEAD_DIM,
                                     k_pages, v_pages));
}

int pgc_merge_partials(const float *partials, int64_t rows, int num_parts, int64_t part_stride,
                       const uint16_t *gate, uint16_t *out, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!partials || !out || rows < 0 || num_parts < 1) return PGC_ERR_INVALID;
    if (num_parts > 1 && part_stride < rows * PGC_PARTIAL_FLOATS) return PGC_ERR_INVALID;
    if (rows == 0) return PGC_OK;
    if (rows > INT32_MAX) return PGC_ERR_BOUNDS;
    return cuda_status(launch_merge_partials(partials, rows, num_parts, part_stride, gate, out,
                                             static_cast<cudaStream_t>(stream)));
}

size_t pgc_prefill_workspace_bytes(int prefix_len, int chunk_len) {
    if (chunk_len <= 0 || prefix_len < 0) return 0;
    return prefill_workspace_bytes(prefix_len, chunk_len, current_sm_count());
}

int pgc_prefill_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                     int64_t num_pages, const int32_t *block_table, int prefix_len,
                     int chunk_len, float scale, uint16_t *out, void *workspace,
                     size_t workspace_bytes, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!q || !k_pages || !v_pages || !block_table || !out) return PGC_ERR_INVALID;
    if (prefix_len < 0 || chunk_len < 0 || num_pages <= 0 || !std::isfinite(scale))
        return PGC_ERR_INVALID;
    if (chunk_len == 0) return PGC_OK;
    if (num_pages * 4 * 16 > INT32_MAX) return PGC_ERR_BOUNDS;
    if (!al16(q) || !al16(out) || !al16(k_pages) || !al16(v_pages)) return PGC_ERR_ALIGN;
    const size_t need = prefill_workspace_bytes(prefix_len, chunk_len, current_sm_count());
    if (workspace_bytes < need || (need > 0 && !workspace)) return PGC_ERR_WORKSPACE;
    if (((uintptr_t)workspace & 15u) != 0) return PGC_ERR_ALIGN;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    return cuda_status(launch_prefill(q, tk, tv, v_pages, num_pages, block_table, prefix_len, chunk_len,
                                      scale, out, workspace, current_sm_count(),
                                      static_cast<cudaStream_t>(stream)));
}

int pgc_copy_rows(void *dst, const void *src, const int32_t *dst_rows, const int32_t *src_rows,
                  int64_t n_rows, int64_t row_bytes, int64_t dst_pitch, int64_t src_pitch,
                  void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (n_rows < 0 || row_bytes < 0 || dst_pitch < 0 || src_pitch < 0) return PGC_ERR_INVALID;
    if (n_rows == 0 || row_bytes == 0) return PGC_OK;
    if (!dst || !src) return PGC_ERR_INVALID;
    if (!dst_rows && row_bytes > dst_pitch && n_rows > 1) return PGC_ERR_INVALID;
    if (!src_rows && row_bytes > src_pitch && n_rows > 1) return PGC_ERR_INVALID;
    return cuda_status(launch_copy_rows(dst, src, dst_rows, src_rows, n_rows, row_bytes, dst_pitch,
                                        src_pitch, static_cast<cudaStream_t>(stream)));
}

static int dense_checks(const void *kd, const void *vd, int64_t stride, int64_t tok,
                        const void *kp, const void *vp, int64_t num_pages, const int32_t *table,
                        int64_t n_table, int64_t ptok, int64_t count) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (count < 0 || stride <= 0 || tok < 0 || ptok < 0 || num_pages <= 0 || n_table < 0)
        return PGC_ERR_INVALID;
    if (count == 0) return PGC_OK;
    if (!kd || !vd || !kp || !vp || !table) return PGC_ERR_INVALID;
    if (tok + count > stride) return PGC_ERR_BOUNDS;
    if ((ptok + count + PGC_PAGE_TOKENS - 1) / PGC_PAGE_TOKENS > n_table) return PGC_ERR_BOUNDS;
    // the dense side may be a file image (2-byte aligned bf16 runs); pools are 16-byte aligned
    if (((uintptr_t)kd & 1u) || ((uintptr_t)vd & 1u) || !al16(kp) || !al16(vp)) return PGC_ERR_ALIGN;
    return PGC_OK;
}

int pgc_kv_restore_dense(const uint16_t *k_dense, const uint16_t *v_dense, int64_t src_stride,
                         int64_t src_token, uint16_t *k_pages, uint16_t *v_pages,
                         int64_t num_pages, const int32_t *block_table, int64_t n_table,
                         int64_t dst_token, int64_t count, void *stream) {
    int st = dense_checks(k_dense, v_dense, src_stride, src_token, k_pages, v_pages, num_pages,
                          block_table, n_table, dst_token, count);
    if (st != PGC_OK || count == 0) return st;
    return cuda_status(launch_kv_dense(true, const_cast<uint16_t *>(k_dense),
                                       const_cast<uint16_t *>(v_dense), src_stride, src_token,
                                       k_pages, v_pages, num_pages, block_table, n_table, dst_token,
                                       count, static_cast<cudaStream_t>(stream)));
}

int pgc_kv_snapshot_dense(const uint16_t *k_pages, const uint16_t *v_pages, int64_t num_pages,
                          const int32_t *block_table, int64_t n_table, int64_t src_token,
                          uint16_t *k_dense, uint16_t *v_dense, int64_t dst_stride,
                          int64_t dst_token, int64_t count, void *stream) {
    int st = dense_checks(k_dense, v_dense, dst_stride, dst_token, k_pages, v_pages, num_pages,
                          block_table, n_table, src_token, count);
    if (st != PGC_OK || count == 0) return st;
    return cuda_status(launch_kv_dense(false, k_dense, v_dense, dst_stride, dst_token,
                                       const_cast<uint16_t *>(k_pages),
                                       const_cast<uint16_t *>(v_pages), num_pages, block_table,
                                       n_table, src_token, count, static_cast<cudaStream_t>(stream)));
}

int pgc_kv_copy_tokens(const uint16_t *src_k_pages, const uint16_t *src_v_pages,
                       int64_t src_num_pages, const int32_t *src_table, int64_t src_n_table,
                       int64_t src_token, uint16_t *dst_k_pages, uint16_t *dst_v_pages,
                       int64_t dst_num_pages, const int32_t *dst_table, int64_t dst_n_table,
                       int64_t dst_token, int64_t count, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (count < 0 || src_token < 0 || dst_token < 0 || src_num_pages <= 0 || dst_num_pages <= 0)
        return PGC_ERR_INVALID;
    if (count == 0) return PGC_OK;
    if (!src_k_pages || !src_v_pages || !src_table || !dst_k_pages || !dst_v_pages || !dst_table)
        return PGC_ERR_INVALID;
    if ((src_token + count + 15) / 16 > src_n_table || (dst_token + count + 15) / 16 > dst_n_table)
        return PGC_ERR_BOUNDS;
    if (!al16(src_k_pages) || !al16(src_v_pages) || !al16(dst_k_pages) || !al16(dst_v_pages))
        return PGC_ERR_ALIGN;
    return cuda_status(launch_kv_copy_tokens(src_k_pages, src_v_pages, src_num_pages, src_table,
                                             src_n_table, src_token, dst_k_pages, dst_v_pages,
                                             dst_num_pages, dst_table, dst_n_table, dst_token,
                                             count, static_cast<cudaStream_t>(stream)));
}

static int region_checks(const pgc_region *r, int n, bool need_src) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (n < 0 || n > PGC_MAX_REGIONS) return PGC_ERR_INVALID;
    if (n > 0 && !r) return PGC_ERR_INVALID;
    for (int i = 0; i < n; ++i) {
        if (r[i].bytes == 0) continue;
        if (!r[i].dst || (need_src && !r[i].src)) return PGC_ERR_INVALID;
    }
    return PGC_OK;
}

int pgc_copy_regions(const pgc_region *regions_host, int n, void *stream) {
    int st = region_checks(regions_host, n, true);
    if (st != PGC_OK || n == 0) return st;
    return cuda_status(launch_regions(regions_host, n, false, nullptr, nullptr, 0, 0,
                                      static_cast<cudaStream_t>(stream)));
}

int pgc_zero_regions(const pgc_region *regions_host, int n, void *stream) {
    int st = region_checks(regions_host, n, false);
    if (st != PGC_OK || n == 0) return st;
    return cuda_status(launch_regions(regions_host, n, true, nullptr, nullptr, 0, 0,
                                      static_cast<cudaStream_t>(stream)));
}

int pgc_rollback(const int32_t *accept, int32_t *seq_lens, int seq_index, int reject_tokens,
                 const pgc_region *regions_host, int n, void *stream) {
    int st = region_checks(regions_host, n, true);
    if (st != PGC_OK) return st;
    if (!accept || !seq_lens || seq_index < 0 || reject_tokens < 0) return PGC_ERR_INVALID;
    return cuda_status(launch_regions(regions_host, n, false, accept, seq_lens, seq_index,
                                      reject_tokens, static_cast<cudaStream_t>(stream)));
}

// ------------------------------------------------------------------ linear attention
int pgc_conv1d_decode(float *conv_states, int64_t num_slots, const int32_t *slots, int batch,
                      const uint16_t *x, const uint16_t *weight, uint16_t *out, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (batch < 0 || num_slots <= 0) return PGC_ERR_INVALID;
    if (batch == 0) return PGC_OK;
    if (!conv_states || !x || !weight || !out) return PGC_ERR_INVALID;
    if (!slots && batch > num_slots) return PGC_ERR_BOUNDS;
    if (((uintptr_t)weight & 7u) != 0 || ((uintptr_t)conv_states & 3u) != 0) return PGC_ERR_ALIGN;
    return cuda_status(launch_conv1d_decode(conv_states, num_slots, slots, batch, x, weight, out,
                                            static_cast<cudaStream_t>(stream)));
}

int pgc_conv1d_prefill(float *conv_state, int has_previous_state, const uint16_t *x, int tokens,
                       const uint16_t *weight, uint16_t *out, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (tokens < 0) return PGC_ERR_INVALID;
    if (tokens == 0) return PGC_OK;
    if (!conv_state || !x || !weight || !out) return PGC_ERR_INVALID;
    if (((uintptr_t)weight & 7u) != 0 || ((uintptr_t)conv_state & 3u) != 0) return PGC_ERR_ALIGN;
    return cuda_status(launch_conv1d_prefill(conv_state, has_previous_state != 0, x, tokens, weight, out,
                                             static_cast<cudaStream_t>(stream)));
}

int pgc_gated_delta_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                           int has_previous_state, const uint16_t *conv_out, const uint16_t *a,
                           const uint16_t *b, const float *a_log, const uint16_t *dt_bias,
                           uint16_t *y, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (batch < 0 || num_slots <= 0) return PGC_ERR_INVALID;
    if (batch == 0) return PGC_OK;
    if (!states || !conv_out || !a || !b || !a_log || !dt_bias || !y) return PGC_ERR_INVALID;
    if (!slots && batch > num_slots) return PGC_ERR_BOUNDS;
    if (!al16(conv_out) || ((uintptr_t)states & 3u) != 0) return PGC_ERR_ALIGN;
    return cuda_status(launch_gated_delta_decode(states, num_slots, slots, batch, has_previous_state != 0,
                                                 conv_out, a, b, a_log, dt_bias, y,
                                                 static_cast<cudaStream_t>(stream)));
}

size_t pgc_gated_delta_prefill_workspace_bytes(int tokens) {
    return gated_delta_prefill_workspace_bytes(tokens);
}

int pgc_gated_delta_prefill(float *state, int has_previous_state, const uint16_t *conv_out,
                            const uint16_t *a, const uint16_t *b, const float *a_log,
                            const uint16_t *dt_bias, int tokens, uint16_t *y, void *workspace,
                            size_t workspace_bytes, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (tokens < 0) return PGC_ERR_INVALID;
    if (tokens == 0) return PGC_OK;
    if (!state || !conv_out || !a || !b || !a_log || !dt_bias || !y || !workspace) return PGC_ERR_INVALID;
    if (workspace_bytes < gated_delta_prefill_workspace_bytes(tokens)) return PGC_ERR_WORKSPACE;
    if (!al16(conv_out) || !al16(workspace) || ((uintptr_t)state & 3u) != 0) return PGC_ERR_ALIGN;
    return cuda_status(launch_gated_delta_prefill(state, has_previous_state != 0, conv_out, a, b, a_log,
                                                  dt_bias, tokens, y, workspace,
                                                  static_cast<cudaStream_t>(stream)));
}

// ------------------------------------------------------------------ context parallel
size_t pgc_cp_buffer_bytes(int world) {
    if (world < 1 || world > PGC_CP_MAX_RANKS) return 0;
    return cp_buffer_bytes(world);
}

int pgc_cp_buffer_alloc(int world, void **buffer_out) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!buffer_out || world < 1 || world > PGC_CP_MAX_RANKS) return PGC_ERR_INVALID;
    void *p = nullptr;
    if (cudaMalloc(&p, cp_buffer_bytes(world)) != cudaSuccess) return PGC_ERR_CUDA;
    if (cudaMemset(p, 0, cp_buffer_bytes(world)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return PGC_ERR_CUDA;
    }
    *buffer_out = p;
    return PGC_OK;
}

int pgc_cp_buffer_free(void *buffer) {
    if (!buffer) return PGC_ERR_INVALID;
    return cuda_status(cudaFree(buffer));
}

int pgc_ipc_get_handle(void *buffer, void *handle_out) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!buffer || !handle_out) return PGC_ERR_INVALID;
    static_assert(sizeof(cudaIpcMemHandle_t) == PGC_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, buffer) != cudaSuccess) return PGC_ERR_CUDA;
    memcpy(handle_out, &h, sizeof(h));
    return PGC_OK;
}

int pgc_ipc_open_handle(const void *handle, void **buffer_out) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (!handle || !buffer_out) return PGC_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PGC_ERR_CUDA;
    *buffer_out = p;
    return PGC_OK;
}

int pgc_ipc_close(void *buffer) {
    if (!buffer) return PGC_ERR_INVALID;
    return cuda_status(cudaIpcCloseMemHandle(buffer));
}

int pgc_cp_decode_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                       int64_t num_pages, const int32_t *block_table, int max_pages,
                       const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                       uint16_t *out, void *workspace, size_t workspace_bytes,
                       void *const *buffers, int world, int rank, uint32_t epoch, void *stream) {
    int st = decode_checks(q, k_pages, v_pages, num_pages, block_table, max_pages, seq_len, 1, 1,
                           max_seq_len, workspace, workspace_bytes);
    if (st != PGC_OK) return st;
    if (!out || !buffers || !std::isfinite(scale)) return PGC_ERR_INVALID;
    if (world < 1 || world > PGC_CP_MAX_RANKS || rank < 0 || rank >= world || epoch == 0)
        return PGC_ERR_INVALID;
    float *bufs[PGC_CP_MAX_RANKS] = {};
    for (int i = 0; i < world; ++i) {
        if (!buffers[i] || !al16(buffers[i])) return PGC_ERR_INVALID;
        bufs[i] = static_cast<float *>(buffers[i]);
    }
    if (!al16(out) || (gate && !al16(gate))) return PGC_ERR_ALIGN;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    return cuda_status(launch_cp_decode(q, tk, tv, num_pages, block_table, max_pages, seq_len, max_seq_len,
                                        scale, gate, out, workspace, bufs, world, rank, epoch,
                                        current_sm_count(), static_cast<cudaStream_t>(stream), k_pages,
                                        v_pages));
}

int pgc_cp_decode_attn_append(const uint16_t *q_in, int q_head_stride, const uint16_t *k_in,
                              const uint16_t *v_in, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                              const float *rope_table, int64_t rope_max_pos, const int32_t *position,
                              const int64_t *slot, int64_t shard_start, uint16_t *k_pages,
                              uint16_t *v_pages, int64_t num_pages, const int32_t *block_table, int max_pages,
                              const int32_t *seq_len, int max_seq_len, float scale, uint16_t *out,
                              void *workspace, size_t workspace_bytes, void *const *buffers, int world,
                              int rank, uint32_t epoch, void *stream) {
    int st = decode_checks(q_in, k_pages, v_pages, num_pages, block_table, max_pages, seq_len, 1, 1,
                           max_seq_len, workspace, workspace_bytes);
    if (st != PGC_OK) return st;
    if (!out || !buffers || !std::isfinite(scale) || !k_in || !v_in || !rope_table || !position || !slot ||
        rope_max_pos <= 0 || shard_start < 0)
        return PGC_ERR_INVALID;
    if (q_head_stride != PGC_HEAD_DIM && q_head_stride != 2 * PGC_HEAD_DIM) return PGC_ERR_INVALID;
    if (world < 1 || world > PGC_CP_MAX_RANKS || rank < 0 || rank >= world || epoch == 0)
        return PGC_ERR_INVALID;
    float *bufs[PGC_CP_MAX_RANKS] = {};
    for (int i = 0; i < world; ++i) {
        if (!buffers[i] || !al16(buffers[i])) return PGC_ERR_INVALID;
        bufs[i] = static_cast<float *>(buffers[i]);
    }
    if (!al16(out)) return PGC_ERR_ALIGN;
    CUtensorMap tk, tv;
    if ((st = pool_tensor_map(k_pages, num_pages, &tk)) != PGC_OK) return st;
    if ((st = pool_tensor_map(v_pages, num_pages, &tv)) != PGC_OK) return st;
    DecodeAppend app;
    app.q_in = q_in;
    app.q_head_stride = q_head_stride;
    app.k_in = k_in;
    app.v_in = v_in;
    app.q_norm_w = q_norm_w;
    app.k_norm_w = k_norm_w;
    app.rope = rope_table;
    app.rope_max_pos = rope_max_pos;
    app.positions = position;
    app.slots = slot;
    app.k_pages = k_pages;
    app.v_pages = v_pages;
    app.num_pages = num_pages;
    app.pos_offset = shard_start;
    // packed q | gate rows: the gate is the second half of each 512-wide head row
    const uint16_t *gate = q_head_stride == 2 * PGC_HEAD_DIM ? q_in + PGC_HEAD_DIM : nullptr;
    return cuda_status(launch_cp_decode(nullptr, tk, tv, num_pages, block_table, max_pages, seq_len, max_seq_len,
                                        scale, gate, out, workspace, bufs, world, rank, epoch,
                                        current_sm_count(), static_cast<cudaStream_t>(stream), k_pages,
                                        v_pages, &app, q_head_stride));
}

// ------------------------------------------------------------------ q4 projections
int pgc_q4_dequantize(const uint32_t *weight, const uint16_t *scales, const uint16_t *biases,
                      uint16_t *out, int out_dim, int in_dim, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (out_dim < 0 || in_dim <= 0 || in_dim % 64 != 0) return PGC_ERR_INVALID;
    if (out_dim == 0) return PGC_OK;
    if (!weight || !scales || !biases || !out) return PGC_ERR_INVALID;
    if (!al16(out) || ((uintptr_t)weight & 3u) != 0) return PGC_ERR_ALIGN;
    return cuda_status(launch_q4_dequantize(weight, scales, biases, out, out_dim, in_dim,
                                            static_cast<cudaStream_t>(stream)));
}

int pgc_q4_linear(const uint16_t *x, int tokens, const uint32_t *weight, const uint16_t *scales,
                  const uint16_t *biases, uint16_t *y, int out_dim, int in_dim, void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (tokens < 0 || out_dim <= 0 || in_dim <= 0) return PGC_ERR_INVALID;
    // K slices of whole 8-group units (16-byte scale and bias copies); the scale and bias
    // slices of a CTA stay in shared memory, which bounds in_dim
    if (in_dim % 2048 != 0 || in_dim > 8192 || out_dim % 64 != 0) return PGC_ERR_INVALID;
    if (tokens == 0) return PGC_OK;
    if (!x || !weight || !scales || !biases || !y) return PGC_ERR_INVALID;
    if (!al16(x) || !al16(weight) || !al16(scales) || !al16(biases) || ((uintptr_t)y & 1u) != 0)
        return PGC_ERR_ALIGN;
    if (tokens <= kQ4GemvMaxTokens) {
        const Q4Weight q4w = {weight, scales, biases, y, out_dim};
        return cuda_status(launch_q4_gemv(x, tokens, &q4w, 1, in_dim, static_cast<cudaStream_t>(stream)));
    }
    const int np = q4_token_tile(tokens);
    CUtensorMap tx, tw;
    if ((st = tiled_map_2d(x, 2, in_dim, tokens, 64, np, true, &tx)) != PGC_OK) return st;
    if ((st = tiled_map_2d(weight, 4, in_dim / 8, out_dim, 32, 128, true, &tw)) != PGC_OK) return st;
    return cuda_status(launch_q4_linear(tx, tw, tokens, scales, biases, y, out_dim, in_dim,
                                        static_cast<cudaStream_t>(stream)));
}

int pgc_q4_linear_multi(const uint16_t *x, int tokens, int in_dim, int n_weights,
                        const uint32_t *const *weights, const uint16_t *const *scales,
                        const uint16_t *const *biases, uint16_t *const *outs, const int *out_dims,
                        void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (n_weights < 1 || n_weights > PGC_LINEAR_MAX_WEIGHTS || !weights || !scales || !biases || !outs ||
        !out_dims)
        return PGC_ERR_INVALID;
    if (tokens > kQ4GemvMaxTokens) {
        // the tensor-core projection: one launch per weight, each a pass over its packed words
        for (int i = 0; i < n_weights; ++i)
            if ((st = pgc_q4_linear(x, tokens, weights[i], scales[i], biases[i], outs[i], out_dims[i], in_dim,
                                    stream)) != PGC_OK)
                return st;
        return PGC_OK;
    }
    if (tokens < 0 || in_dim <= 0 || in_dim % 2048 != 0 || in_dim > 8192) return PGC_ERR_INVALID;
    Q4Weight q4w[PGC_LINEAR_MAX_WEIGHTS];
    for (int i = 0; i < n_weights; ++i) {
        if (out_dims[i] <= 0 || out_dims[i] % 64 != 0) return PGC_ERR_INVALID;
        if (!weights[i] || !scales[i] || !biases[i] || !outs[i]) return PGC_ERR_INVALID;
        if (!al16(weights[i]) || !al16(scales[i]) || !al16(biases[i]) || ((uintptr_t)outs[i] & 1u) != 0)
            return PGC_ERR_ALIGN;
        q4w[i] = {weights[i], scales[i], biases[i], outs[i], out_dims[i]};
    }
    if (tokens == 0) return PGC_OK;
    if (!x) return PGC_ERR_INVALID;
    if (!al16(x)) return PGC_ERR_ALIGN;
    return cuda_status(launch_q4_gemv(x, tokens, q4w, n_weights, in_dim, static_cast<cudaStream_t>(stream)));
}

int pgc_prefill_linear(const uint16_t *x, int tokens, int in_dim, int n_weights,
                       const uint16_t *const *weights, const int *out_dims, uint16_t *const *outs,
                       void *stream) {
    int st = check_device(nullptr);
    if (st != PGC_OK) return st;
    if (tokens < 0 || in_dim <= 0 || in_dim % 64 != 0 || n_weights < 1 ||
        n_weights > PGC_LINEAR_MAX_WEIGHTS || !weights || !out_dims || !outs)
        return PGC_ERR_INVALID;
    for (int i = 0; i < n_weights; ++i) {
        if (!weights[i] || !outs[i] || out_dims[i] <= 0 || out_dims[i] % 8 != 0) return PGC_ERR_INVALID;
        if (!al16(weights[i]) || !al16(outs[i])) return PGC_ERR_ALIGN;
    }
    if (tokens == 0) return PGC_OK;
    if (!x) return PGC_ERR_INVALID;
    if (!al16(x)) return PGC_ERR_ALIGN;
    CUtensorMap tx, tw[PGC_LINEAR_MAX_WEIGHTS];
    LinearOut lo[PGC_LINEAR_MAX_WEIGHTS];
    if ((st = tiled_map_2d(x, 2, in_dim, tokens, 64, 128, true, &tx)) != PGC_OK) return st;
    for (int i = 0; i < n_weights; ++i) {
        if ((st = tiled_map_2d(weights[i], 2, in_dim, out_dims[i], 64, 128, true, &tw[i])) != PGC_OK) return st;
        lo[i].y = outs[i];
        lo[i].out_dim = out_dims[i];
    }
    return cuda_status(launch_prefill_linear(tx, tw, lo, n_weights, tokens, in_dim, current_sm_count(),
                                             static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
