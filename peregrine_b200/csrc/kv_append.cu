// kv_append.cu — KV append with fused RMSNorm + partial NeoX RoPE (sm_100a).
//
// Behaviour follows qwen35_q_gate_prepare_kv_append_pair_head_major_value_dim_major_bf16
// (shaders/attention.metal:327-421; decode) and qwen35_qk_norm_rope_append_many_bf16
// (shaders/attention.metal:146-219; prefill): per head row, optional RMSNorm
// x * rsqrt(mean(x^2) + 1e-6) * w, RoPE on pairs (i, i + 32) for i < 32 with the angle table of
// pgc_rope_table_fill, q to q_out, k and v into the paged pools.
//
// One warp per (token, head row), 20 rows per token (16 q + 4 k). Lane l owns dims l + 32j,
// j = 0..7, so the RoPE pair (l, l + 32) is in-thread and the sum of squares reproduces the
// reference's 256-thread tree (strides 128, 64, 32 in registers, then 16..1 by shuffle).
// Every fp32 operation is an explicitly rounded intrinsic, so results are bit-identical to
// the same operations done in order on the CPU.
#include "pgc_common.cuh"
#include "pgc_internal.h"

namespace pgc {

PGC_DEFINE_ERROR_WORD(g_append_err);

namespace {

struct AppendParams {
    const uint16_t *q_in;
    uint16_t *q_out;
    uint16_t *gate_out;
    const uint16_t *k_in;
    const uint16_t *v_in;
    const uint16_t *q_norm_w;
    const uint16_t *k_norm_w;
    const float *rope;
    const int32_t *positions;
    const int64_t *slots;
    uint16_t *k_pages;
    uint16_t *v_pages;
    int64_t rope_max_pos;
    int64_t tokens;
    int64_t num_pages;
    int q_head_stride;
    int mode;
};

constexpr int kRowsPerToken = kNumQHeads + kNumKvHeads;

__global__ void __launch_bounds__(256) append_kernel(const AppendParams p) {
    pdl_trigger();
    pdl_wait();
    const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= p.tokens * kRowsPerToken) return;
    const int64_t t = gw / kRowsPerToken;
    const int hr = (int)(gw % kRowsPerToken);
    const bool is_q = hr < kNumQHeads;
    const int kvh = hr - kNumQHeads;

    const int32_t pos = p.positions[t];
    if (pos < 0 || pos >= p.rope_max_pos) {
        if (lane == 0) record_error(&g_append_err, kErrPosOutOfRange, t);
        return;
    }
    uint16_t *dst;
    uint16_t *vdst = nullptr;
    if (is_q) {
        dst = p.q_out + (t * kNumQHeads + hr) * kHeadDim;
    } else {
        const int64_t slot = p.slots[t];
        if (slot < 0) return;  // padding token: nothing to append
        const int64_t page = slot / kPage;
        if (page >= p.num_pages) {
            if (lane == 0) record_error(&g_append_err, kErrSlotOutOfRange, slot);
            return;
        }
        const int64_t off = ((page * kNumKvHeads + kvh) * kPage + slot % kPage) * kHeadDim;
        dst = p.k_pages + off;
        vdst = p.v_pages + off;
    }
    const uint16_t *src = is_q ? p.q_in + (t * kNumQHeads + hr) * (int64_t)p.q_head_stride
                               : p.k_in + (t * kNumKvHeads + kvh) * kHeadDim;
    const uint16_t *w = is_q ? p.q_norm_w : p.k_norm_w;

    uint16_t o[8];
    append_row_warp(src, w, p.rope + (int64_t)pos * kRot, p.mode == PGC_APPEND_DECODE, lane, o);
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[lane + 32 * j] = o[j];

    if (is_q) {
        if (p.gate_out != nullptr) {
            uint16_t *g = p.gate_out + (t * kNumQHeads + hr) * kHeadDim;
#pragma unroll
            for (int j = 0; j < 8; ++j) g[lane + 32 * j] = src[kHeadDim + lane + 32 * j];
        }
    } else {
        const uint4 *vs = reinterpret_cast<const uint4 *>(p.v_in + (t * kNumKvHeads + kvh) * kHeadDim);
        reinterpret_cast<uint4 *>(vdst)[lane] = vs[lane];
    }
}

}  // namespace

cudaError_t launch_append(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                          uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                          const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                          const float *rope_table, int64_t rope_max_pos, const int32_t *positions,
                          const int64_t *slot_mapping, int64_t tokens, uint16_t *k_pages,
                          uint16_t *v_pages, int64_t num_pages, int mode, cudaStream_t stream) {
    AppendParams p;
    p.q_in = q_in;
    p.q_out = q_out;
    p.gate_out = gate_out;
    p.k_in = k_in;
    p.v_in = v_in;
    p.q_norm_w = q_norm_w;
    p.k_norm_w = k_norm_w;
    p.rope = rope_table;
    p.positions = positions;
    p.slots = slot_mapping;
    p.k_pages = k_pages;
    p.v_pages = v_pages;
    p.rope_max_pos = rope_max_pos;
    p.tokens = tokens;
    p.num_pages = num_pages;
    p.q_head_stride = q_head_stride;
    p.mode = mode;
    const int64_t warps = tokens * kRowsPerToken;
    const int64_t blocks = (warps + 7) / 8;
    cudaError_t e = launch_pdl(append_kernel, dim3((unsigned)blocks), dim3(256), 0, stream, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t append_read_error(DevErrorHost *e, bool clear) {
    cudaError_t r = cudaMemcpyFromSymbol(e, g_append_err, sizeof(DevError));
    if (r != cudaSuccess || !clear) return r;
    DevErrorHost z = {0, 0, 0};
    return cudaMemcpyToSymbol(g_append_err, &z, sizeof(DevError));
}

}  // namespace pgc
