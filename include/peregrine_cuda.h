/*
 * peregrine_cuda.h — C ABI of libperegrine_cuda.so, the B200 (sm_100a) KV / prefix-cache
 * hot path of the Peregrine Qwen3.5-9B server.
 *
 * The reference binds its GPU work through the Objective-C Metal bridge
 * (src/runtime/bridge.h:1-103) and through Zig helpers that copy cache state with host
 * memcpy (src/model/state.zig:124-230). Each entry point below names the reference
 * interface it replaces.
 *
 * Conventions (mirroring src/runtime/bridge.h):
 *   - plain pointers and sizes only; bf16 tensors are passed as uint16_t bit patterns;
 *   - the caller owns every device, pinned-host and workspace buffer;
 *   - every operation is enqueued asynchronously on the caller's CUDA stream
 *     (a cudaStream_t passed as void*; NULL = legacy default stream);
 *   - every entry returns an int status: 0 = ok, negative = PGC_ERR_* (the reference's
 *     encode calls return void and report GPU failure at commit time, bridge.m:376;
 *     here shape and bounds errors are caught on the host before the launch);
 *   - device-side faults never trap: kernels that find an out-of-range index record it
 *     in a device error word (read with pgc_device_error) and skip the access.
 *
 * Fixed geometry (Qwen3.5-9B full-attention layers, src/model/block_attn.zig:21-28):
 * 16 query heads, 4 KV heads (GQA group 4), head_dim 256, rotary_dim 64, hidden 4096.
 *
 * Paged KV layout (new design; the reference cache is a dense strided buffer, see
 * state.zig:41-44): per layer one K pool and one V pool, each
 *     pool[page][kv_head 4][slot 16][dim 256]  bf16
 * so one (page, kv head) is an 8 KiB contiguous run of 16 token rows of 512 B. A token at
 * logical position t of a sequence lives in page block_table[t / 16], slot t % 16.
 */
#ifndef PEREGRINE_CUDA_H
#define PEREGRINE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PGC_NUM_Q_HEADS 16
#define PGC_NUM_KV_HEADS 4
#define PGC_GQA_GROUP 4
#define PGC_HEAD_DIM 256
#define PGC_ROTARY_DIM 64
#define PGC_PAGE_TOKENS 16
#define PGC_HIDDEN 4096
#define PGC_MAX_CONTEXT_TOKENS 65536 /* state.zig:11 (per-sequence dense cache limit) */
#define PGC_PARTIAL_FLOATS (PGC_HEAD_DIM + 2) /* one (m, l, o[256]) partial */
#define PGC_MAX_QUERIES 4                     /* query tokens per sequence per decode call */
#define PGC_MAX_REGIONS 128                   /* regions per pgc_copy_regions call */

enum pgc_status {
    PGC_OK = 0,
    PGC_ERR_INVALID = -1,   /* null pointer, bad shape or unsupported parameter */
    PGC_ERR_BOUNDS = -2,    /* index or length outside the buffer it addresses */
    PGC_ERR_WORKSPACE = -3, /* workspace smaller than the *_workspace_bytes query */
    PGC_ERR_CUDA = -4,      /* a CUDA runtime/driver call failed */
    PGC_ERR_ALIGN = -5,     /* a pointer or size lacks the required alignment */
    PGC_ERR_DEVICE = -6,    /* current device is not sm_100 */
    PGC_ERR_TIMEOUT = -7,   /* a bounded device wait gave up (reported by pgc_device_error) */
    PGC_ERR_CONTEXT = -8,   /* length outside (0, PGC_MAX_CONTEXT_TOKENS] */
    PGC_ERR_FILE = -9,      /* file missing, unreadable or not writable */
    PGC_ERR_FORMAT = -10,   /* prefix-state file fails validation (wrong model, size, ...) */
    PGC_ERR_CAPACITY = -11, /* page pool or linear-state slots exhausted after eviction */
    PGC_ERR_NCCL = -12      /* NCCL missing from the process or an NCCL call failed */
};

/* Status text for an error code (static storage). */
const char *pgc_status_string(int status);
/* Library ABI version (major*10000 + minor*100 + patch). */
int pgc_version(void);
/* Reads and optionally clears the device error word of the current device: 0 when no kernel
 * recorded a fault, else code + 100 * unit (units: 0 decode and context-parallel exchange,
 * 1 append, 2 copies, 3 prefill, 4 linear attention, 5 q4 projection, 6 prefill projection). Synchronises the device. Replaces the reference's
 * MTLCommandBufferStatusError check at commit time (bridge.m:376). */
int pgc_device_error(int *code_out, int64_t *detail_out, int clear);

/* ---------------------------------------------------------------------------------------
 * Layout rules
 * ------------------------------------------------------------------------------------- */

/* Dense-cache token stride for a sequence capacity; replaces fullCacheStrideForMaxSeq
 * (src/model/state.zig:25-32): align(max_seq, 256), or align(max_seq, 64) once
 * max_seq >= 16000; PGC_ERR_CONTEXT for 0 or > 65536. Used by the dense snapshot format. */
int pgc_full_cache_stride_for_max_seq(uint64_t max_seq, uint64_t *stride_out);

/* Fills a RoPE cos/sin table [max_pos][rot_dim] fp32 on the HOST: row p holds
 * cos(p * theta^(-2i/rot_dim)) for i < rot_dim/2 followed by the matching sines, each
 * computed in double and rounded once to fp32. Replaces the per-thread pow/cos/sin of
 * shaders/rope.metal:5-10 and attention.metal:391-396 with a table built once per model;
 * the append kernel reads it, so device and host agree bit for bit. */
int pgc_rope_table_fill(float *table_host, int64_t max_pos, int rot_dim, double theta);

/* ---------------------------------------------------------------------------------------
 * A3/A4: KV append with fused RMSNorm + partial RoPE
 * ------------------------------------------------------------------------------------- */

#define PGC_APPEND_DECODE 0  /* qwen35_q_gate_prepare_kv_append_pair_..._bf16 rounding */
#define PGC_APPEND_PREFILL 1 /* qwen35_qk_norm_rope_append_many_bf16 rounding */

/* Prepares `tokens` new rows: for each token t, each of the 16 q heads and the 4 k heads is
 * optionally RMS-normalised (x * rsqrt(mean(x^2) + 1e-6) * w, tree-ordered sum of
 * squares), then its first 64 dims get NeoX half-split RoPE at positions[t]; q goes to
 * q_out, k to the K pool at slot_mapping[t] (= page * 16 + slot), v is copied unchanged
 * to the V pool at the same slot. A negative slot skips the K/V write of that token.
 *   q_in       [tokens][16][q_head_stride] bf16; q_head_stride 256, or 512 for the packed
 *              q|gate projection of the decode path (attention.metal:362-366)
 *   gate_out   nullable [tokens][16][256]: receives the gate half of a packed q_in
 *   k_in, v_in [tokens][4][256]
 *   q_norm_w, k_norm_w  nullable [256] bf16 RMSNorm weights (NULL = no norm)
 *   rope_table [rope_max_pos][64] from pgc_rope_table_fill, in device memory
 *   mode       PGC_APPEND_DECODE rounds the normalised pair to bf16 before rotating
 *              (attention.metal:389-390); PGC_APPEND_PREFILL does not (attention.metal:196-197)
 * Replaces: qwen35_q_gate_prepare_kv_append_pair_head_major_value_dim_major_bf16
 * (shaders/attention.metal:327-421, launched at src/model/block_attn.zig:322-327) and
 * qwen35_qk_norm_rope_append_many_bf16 (shaders/attention.metal:146-219, launched at
 * src/model/block_attn.zig:435-441). */
int pgc_append_kv_rope(const uint16_t *q_in, int q_head_stride, uint16_t *q_out,
                       uint16_t *gate_out, const uint16_t *k_in, const uint16_t *v_in,
                       const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                       const float *rope_table, int64_t rope_max_pos,
                       const int32_t *positions, const int64_t *slot_mapping, int64_t tokens,
                       uint16_t *k_pages, uint16_t *v_pages, int64_t num_pages, int mode,
                       void *stream);

/* ---------------------------------------------------------------------------------------
 * A1/A2: split-K flash-decode attention over the paged cache
 * ------------------------------------------------------------------------------------- */

/* Workspace bytes pgc_decode_attn / pgc_decode_attn_partials need for this shape. */
size_t pgc_decode_workspace_bytes(int batch, int num_queries, int max_seq_len);

/* Decode SDPA for `batch` sequences, each with `num_queries` (1..4) consecutive query
 * tokens (1 for a decode step, 2 for the MTP verify of draft + bonus). Query j of sequence
 * b sits at position seq_lens[b] - num_queries + j and attends causally to tokens
 * [0, seq_lens[b] - num_queries + j]. Scores are scale * q.k (fp32), softmax and the
 * weighted V sum accumulate in fp32 and the output is rounded once to bf16; with a gate,
 * out = attn * sigmoid(gate) (attention_decode.metal:240-242).
 *   q            [batch][num_queries][16][256] bf16 (device)
 *   k/v_pages    paged pools of `num_pages` pages (layout in the file header)
 *   block_tables [batch][max_pages_per_seq] int32 page ids (device)
 *   seq_lens     [batch] int32 tokens in cache including the queries (device); 0 marks an
 *                empty slot, whose output rows are written as zeros
 *   max_seq_len  host-side upper bound of seq_lens (sizes the split grid)
 *   gate         nullable [batch][num_queries][16][256] bf16
 *   out          [batch][num_queries][16][256] bf16
 * Replaces: sdpa_decode_prefix_flash_partials_bf16 (shaders/attention_decode.metal:24-210)
 * + sdpa_decode_prefix_flash_reduce_gated_bf16 (:215-243), dispatched at
 * src/model/block_attn.zig:331-356. The reference's two KV sources (prefix entry for
 * t < prefix_len, request-local cache after, attention_decode.metal:89-93) become block
 * table entries: shared prefix pages followed by request-local pages. */
int pgc_decode_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                    int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                    const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                    float scale, const uint16_t *gate, uint16_t *out, void *workspace,
                    size_t workspace_bytes, void *stream);

/* Same attention, but emits the un-normalised per-row partial (m, l, o[256]) fp32 of this
 * cache instead of bf16 output: partials [batch][num_queries*16][258], m in natural-log
 * units, l = sum exp(s - m), o = sum exp(s - m) v. Used for context-parallel shards, whose
 * partials are exchanged and combined with pgc_merge_partials. Same partial format as
 * attention_decode.metal:198-206. */
int pgc_decode_attn_partials(const uint16_t *q, const uint16_t *k_pages,
                             const uint16_t *v_pages, int64_t num_pages,
                             const int32_t *block_tables, int max_pages_per_seq,
                             const int32_t *seq_lens, int batch, int num_queries,
                             int max_seq_len, float scale, float *partials, void *workspace,
                             size_t workspace_bytes, void *stream);

/* Size of the fixed scratch array behind pgc_decode_attn_static (16 MiB per GPU). */
#define PGC_DECODE_STATIC_SCRATCH_BYTES (16u << 20)

/* block_attn.zig:322-356 in one launch: pgc_append_kv_rope in decode mode (RMSNorm + RoPE of the
 * q and k heads, the new K/V rows written at slot_mapping) fused into pgc_decode_attn, the same
 * bits as the two calls in sequence. q_in [batch * num_queries][16][q_head_stride] bf16, either q
 * (256) or the packed q | gate rows (512: the gate gates the output as in pgc_decode_attn); k_in,
 * v_in [batch * num_queries][4][256]; token t = seq * num_queries + j at positions[t] (the last
 * num_queries tokens of its sequence, counted in seq_lens). The rotated q is not written out.
 * Position and slot errors are recorded in the decode unit of pgc_device_error. */
int pgc_decode_attn_append(const uint16_t *q_in, int q_head_stride, const uint16_t *k_in,
                           const uint16_t *v_in, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                           const float *rope_table, int64_t rope_max_pos, const int32_t *positions,
                           const int64_t *slot_mapping, uint16_t *k_pages, uint16_t *v_pages,
                           int64_t num_pages, const int32_t *block_tables, int max_pages_per_seq,
                           const int32_t *seq_lens, int batch, int num_queries, int max_seq_len,
                           float scale, uint16_t *out, void *workspace, size_t workspace_bytes,
                           void *stream);

/* pgc_decode_attn without a caller workspace, for callers that cannot allocate device memory
 * at all: code running where cudaMalloc is unavailable or forbidden (a host whose allocator
 * owns all device memory, a real-time serving loop that bans allocation after start-up, a
 * plugin that is handed only its input and output buffers). The split partials go to a
 * file-scope device array of PGC_DECODE_STATIC_SCRATCH_BYTES per GPU, held until the process
 * exits. Under CUDA's default lazy module loading the array is reserved on a device when the
 * library's module is first loaded there, i.e. by the first library call on that device; that
 * first call also resolves the array's device address (cudaGetSymbolAddress) with the device
 * current. So make the first call at start-up, before the caller's allocator claims the
 * device's memory and before any stream capture. Inputs, outputs and their meaning are
 * exactly those of pgc_decode_attn. Returns PGC_ERR_WORKSPACE when
 * pgc_decode_workspace_bytes(batch, num_queries, max_seq_len) exceeds the array. All calls
 * share the array: calls that overlap on the GPU race. Calls
 * no cudaMalloc, cudaFree or allocating library routine. This entry point has no counterpart
 * in the reference. */
int pgc_decode_attn_static(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                           int64_t num_pages, const int32_t *block_tables,
                           int max_pages_per_seq, const int32_t *seq_lens, int batch,
                           int num_queries, int max_seq_len, float scale, const uint16_t *gate,
                           uint16_t *out, void *stream);

/* Log-sum-exp merge of `num_parts` partials per row: m* = max m_p, w_p = exp(m_p - m*),
 * out = sum w_p o_p / sum w_p l_p, times sigmoid(gate) when gate is non-NULL, rounded to
 * bf16. A part with m = -inf has weight 0. Row r, part p lives at
 * partials + p * part_stride + r * 258 (floats). Replaces
 * sdpa_decode_prefix_flash_reduce_gated_bf16 (shaders/attention_decode.metal:215-243) for
 * partials that came from several GPUs. */
int pgc_merge_partials(const float *partials, int64_t rows, int num_parts,
                       int64_t part_stride, const uint16_t *gate, uint16_t *out,
                       void *stream);

/* ---------------------------------------------------------------------------------------
 * A5: chunked-prefill causal attention (tcgen05 / TMEM)
 * ------------------------------------------------------------------------------------- */

/* Workspace bytes pgc_prefill_attn needs for this shape (0 when the grid fills whole waves of
 * SMs without splitting the key range; otherwise the fp32 partials of the key splits). */
size_t pgc_prefill_workspace_bytes(int prefix_len, int chunk_len);

/* Causal GQA attention of a `chunk_len`-token chunk of ONE sequence over prefix + chunk:
 * query t (position prefix_len + t) sees cache tokens [0, prefix_len + t]. The chunk's K/V
 * must already be in the cache (pgc_append_kv_rope). q [chunk_len][16][256] bf16,
 * out [chunk_len][16][256] bf16, block_table [ceil((prefix_len+chunk_len)/16)] int32.
 * Replaces the prefix-aware materialised chain prefill_score_prefix_head_major_bf16 →
 * prefill_softmax_bf16 → prefill_value_prefix_head_major_value_dim_major_bf16
 * (shaders/attention.metal:1204-1358, 1413-1461, 1816-1964; dispatched at
 * src/model/block_attn.zig:633-703) and the non-prefix MLX-GEMM route (block_attn.zig:500-566),
 * with the mask col <= (n - tokens) + t of attention.metal:1347-1353. */
int pgc_prefill_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                     int64_t num_pages, const int32_t *block_table, int prefix_len,
                     int chunk_len, float scale, uint16_t *out, void *workspace,
                     size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------------
 * A6-A9, A11: cache copies (prefix snapshot / restore, hidden rows, state)
 * ------------------------------------------------------------------------------------- */

/* Row gather/scatter: for i < n_rows, copies row_bytes from src + src_rows[i]*src_pitch to
 * dst + dst_rows[i]*dst_pitch (a NULL index array means the identity). Any pointer the GPU
 * can address: HBM, or pinned host memory (the host-resident prefix store). 16-byte vector
 * path when pointers, pitches and row_bytes are 16-byte aligned, else a 4- or 1-byte path.
 * Replaces the hidden-row memcpys of src/server/prefix_state_cache.zig:592-629, :477-487,
 * :265-289 and src/server.zig:1263-1270, and serves page-granular KV copies
 * (row = one (page) of a pool: 4 * 16 * 256 * 2 = 32 KiB). */
int pgc_copy_rows(void *dst, const void *src, const int32_t *dst_rows,
                  const int32_t *src_rows, int64_t n_rows, int64_t row_bytes,
                  int64_t dst_pitch, int64_t src_pitch, void *stream);

/* Restores `count` tokens from a dense reference-layout cache (K [4][src_stride][256]
 * head-major, V [4][256][src_stride] value-dim-major, state.zig:41-44 and the v3 snapshot
 * runs of src/server/prefix_persist.zig:85-137) starting at src_token into the paged pools
 * at logical positions [dst_token, dst_token + count) of the sequence whose page ids are
 * block_table[0 .. n_table). Replaces copyFullAttentionRangeFrom
 * (src/model/state.zig:143-230) when the destination is the paged cache. */
int pgc_kv_restore_dense(const uint16_t *k_dense, const uint16_t *v_dense,
                         int64_t src_stride, int64_t src_token, uint16_t *k_pages,
                         uint16_t *v_pages, int64_t num_pages, const int32_t *block_table,
                         int64_t n_table, int64_t dst_token, int64_t count, void *stream);

/* The inverse of pgc_kv_restore_dense: paged tokens [src_token, src_token + count) →
 * dense reference layout at dst_token (storePrefixFromWork into a prefix entry,
 * src/server/prefix_state_cache.zig:584-588, and the v3 persist writer). */
int pgc_kv_snapshot_dense(const uint16_t *k_pages, const uint16_t *v_pages,
                          int64_t num_pages, const int32_t *block_table, int64_t n_table,
                          int64_t src_token, uint16_t *k_dense, uint16_t *v_dense,
                          int64_t dst_stride, int64_t dst_token, int64_t count, void *stream);

/* Copies logical tokens [src_token, src_token + count) of one paged sequence into logical
 * tokens [dst_token, dst_token + count) of another (possibly the same pools). Replaces
 * copyFullAttentionRangeFrom (src/model/state.zig:143-179) between two paged states, e.g.
 * the verifier re-sync of src/server/decode_loop.zig:295-311. */
int pgc_kv_copy_tokens(const uint16_t *src_k_pages, const uint16_t *src_v_pages,
                       int64_t src_num_pages, const int32_t *src_table, int64_t src_n_table,
                       int64_t src_token, uint16_t *dst_k_pages, uint16_t *dst_v_pages,
                       int64_t dst_num_pages, const int32_t *dst_table, int64_t dst_n_table,
                       int64_t dst_token, int64_t count, void *stream);

/* One contiguous byte region. */
typedef struct pgc_region {
    void *dst;
    const void *src; /* ignored by pgc_zero_regions */
    uint64_t bytes;
} pgc_region;

/* Copies up to PGC_MAX_REGIONS regions in ONE launch (the descriptors travel as a kernel
 * argument; no device descriptor buffer). Replaces copyLinearStateFrom
 * (src/model/state.zig:130-141): 24 linear layers × (conv, recurrent) state. */
int pgc_copy_regions(const pgc_region *regions_host, int n, void *stream);

/* Zero-fills up to PGC_MAX_REGIONS regions in one launch. Replaces resetForNewSequence
 * (src/model/state.zig:110-118) and the zero-fill of initBf16FullCaches (:51-83). */
int pgc_zero_regions(const pgc_region *regions_host, int n, void *stream);

/* ---------------------------------------------------------------------------------------
 * A10: MTP verify rollback
 * ------------------------------------------------------------------------------------- */

/* Device-side accept/reject of a speculative verify step, with no host round trip.
 * Reads *accept (device int32). When it is 0 (draft rejected): seq_lens[seq_index] -= reject_tokens
 * (the rejected KV rows are truncated; attention is bounded by seq_len, so the rows need no
 * clearing, state.zig:107-109) and every region is copied snapshot → live (regions[i].src =
 * snapshot taken before the step, .dst = live recurrent/conv state). When *accept != 0
 * nothing changes. Replaces the double-buffered swap + prepareVerifierState re-sync of
 * src/server/decode_loop.zig:216-258,295-311. */
int pgc_rollback(const int32_t *accept, int32_t *seq_lens, int seq_index, int reject_tokens,
                 const pgc_region *regions_host, int n, void *stream);

/* ---------------------------------------------------------------------------------------
 * Prefix-state snapshot file (format v3 of src/server/prefix_persist.zig:31-137)
 * ------------------------------------------------------------------------------------- */

/* Byte offsets of every section of a v3 file holding `token_count` tokens. Linear layers are
 * numbered in model order (24: conv f32 [3][8192], recurrent f32 [32][128][128]); full layers
 * too (8: K runs [4][count][256] bf16 = a dense K of stride count, V runs [4][256][count] bf16
 * = a dense V of stride count). Replaces expectedFileBytes / fullCacheRuns
 * (prefix_persist.zig:64-137). */
typedef struct pgc_prefix_layout {
    uint64_t token_count;
    uint64_t tokens;      /* u32 [count] */
    uint64_t conv[24];
    uint64_t recur[24];
    uint64_t k_runs[8];
    uint64_t v_runs[8];
    uint64_t hidden;      /* bf16 [count][4096] */
    uint64_t total_bytes; /* exact file size */
} pgc_prefix_layout;

typedef struct pgc_prefix_info {
    uint64_t token_count;
    uint32_t next_token;
    uint32_t next_token_valid;
    uint32_t hidden_valid;
    uint64_t file_bytes;
} pgc_prefix_info;

int pgc_prefix_file_layout(uint64_t token_count, pgc_prefix_layout *out);

/* Validates a v3 file without reading its payload: magic, version, dtype, model fingerprint,
 * flags, cached next token < vocab, 0 < token_count <= max_tokens and the exact file size.
 * PGC_ERR_FILE when it cannot be opened, PGC_ERR_FORMAT when it must be ignored (the caller
 * then cold-prefills). Replaces the checks of load() (src/server/prefix_persist.zig:329-356). */
int pgc_prefix_file_inspect(const char *path, uint64_t model_fingerprint, uint64_t vocab,
                            uint64_t max_tokens, pgc_prefix_info *info);

/* Validates, then reads the whole file into `image` (ideally pinned host memory: the restore
 * kernels then read it directly). Section offsets from pgc_prefix_file_layout. */
int pgc_prefix_file_read(const char *path, uint64_t model_fingerprint, uint64_t vocab,
                         uint64_t max_tokens, void *image, uint64_t image_bytes,
                         pgc_prefix_info *info);

/* Writes the 48-byte header into a file image whose sections the caller has filled (token
 * ids, linear states, pgc_kv_snapshot_dense into the K/V runs with dst_stride = count, hidden
 * rows). */
int pgc_prefix_file_header(void *image, uint64_t image_bytes, uint64_t model_fingerprint,
                           uint64_t token_count, uint32_t next_token, int next_token_valid,
                           int hidden_valid);

/* Atomically replaces `path` with the image (temporary file, fsync, rename), as save() does
 * (src/server/prefix_persist.zig:255-326). */
int pgc_prefix_file_write(const char *path, const void *image, uint64_t image_bytes);

/* ---------------------------------------------------------------------------------------
 * Page pool and page-refcounted prefix cache (host side, no device work).
 *
 * Replaces the resident prompt-prefix cache (src/server/prefix_state_cache.zig:21-567). The
 * reference entry owns a private model state and every hit or store copies KV rows
 * (state.zig:124-230); here every KV page of every full layer, and the MTP hidden-row pool, is
 * indexed by one page id, an entry is a list of page ids, and sharing is a refcount:
 *   hit:    pgc_prefix_cache_fork -> the request's block table starts with the entry's pages;
 *           before writing into a page it does not own alone (the partial page at the end of a
 *           match) the request calls pgc_page_pool_make_writable and copies that one page on
 *           the device (pgc_copy_regions over each per-page pool);
 *   store:  pgc_prefix_cache_store adopts the work sequence's pages (no KV copy);
 *   linear state (recurrent + conv) is not paged: each entry owns a state slot and the caller
 *           copies it where the reference does (copy_linear_state reports when).
 * The policy is the reference's: token-level longest-prefix match, reserved-token budget with
 * capacity max(len, prefill chunk), LRU eviction of unpinned entries, entry indexes that shift
 * down when an earlier entry is removed (a pgc_match is valid until the next mutation).
 * Constructors return NULL on failure (bridge.h convention); one thread per cache.
 * ------------------------------------------------------------------------------------- */
typedef struct pgc_page_pool pgc_page_pool;
typedef struct pgc_prefix_cache pgc_prefix_cache;

/* The reference's Match (prefix_state_cache.zig:16-19); index -1 = no match. */
typedef struct pgc_match {
    int64_t index;
    int64_t len;
} pgc_match;

/* Cache.Stats (prefix_state_cache.zig:200-229) plus resident/pinned/active/trie counters. */
typedef struct pgc_prefix_stats {
    uint64_t hits, misses, hit_tokens, computed_tokens;
    uint64_t reserved_tokens, resident_tokens, max_tokens;
    uint64_t entry_count, pinned_count, evictions, trie_nodes;
    int64_t active_index;
} pgc_prefix_stats;

typedef struct pgc_prefix_entry {
    uint64_t token_count;
    int64_t page_count;
    uint64_t capacity;      /* reserved tokens */
    int32_t state_slot;     /* linear-state slot owned by the entry */
    int32_t pinned, hidden_valid, next_token_valid;
    uint32_t next_token;
    uint64_t last_access, hits;
} pgc_prefix_entry;

pgc_page_pool *pgc_page_pool_create(int32_t num_pages);
/* A pool destroyed while caches are built on it is freed with the last of them. */
void pgc_page_pool_destroy(pgc_page_pool *pool);
/* n fresh pages with one reference each; PGC_ERR_CAPACITY (nothing taken) when fewer are free. */
int pgc_page_pool_alloc(pgc_page_pool *pool, int32_t n, int32_t *pages_out);
int pgc_page_pool_retain(pgc_page_pool *pool, const int32_t *pages, int32_t n);
/* Drops one reference per listed page; a page reaching 0 returns to the free list. */
int pgc_page_pool_release(pgc_page_pool *pool, const int32_t *pages, int32_t n);
int32_t pgc_page_pool_refcount(const pgc_page_pool *pool, int32_t page);
int32_t pgc_page_pool_free_pages(const pgc_page_pool *pool);
/* Copy-on-write for table[slot]: if the page has other holders, a fresh page replaces it in
 * the table (this holder's reference moves to it) and *src != *dst names the device copy to
 * issue before writing; otherwise *src == *dst and nothing is to be copied. */
int pgc_page_pool_make_writable(pgc_page_pool *pool, int32_t *table, int32_t slot,
                                int32_t *src_page, int32_t *dst_page);

/* Cache.init (prefix_state_cache.zig:312-320) over `pool`, with `state_slots` linear-state
 * slots. */
pgc_prefix_cache *pgc_prefix_cache_create(pgc_page_pool *pool, int32_t page_tokens,
                                          uint64_t max_tokens, uint64_t prefill_chunk_tokens,
                                          int32_t state_slots);
void pgc_prefix_cache_destroy(pgc_prefix_cache *cache);
void pgc_prefix_cache_clear_all(pgc_prefix_cache *cache);
void pgc_prefix_cache_enable_hidden_tracking(pgc_prefix_cache *cache);
/* findPrefix: 1 and the longest cached prefix of the prompt, or 0 (out->index = -1). */
int pgc_prefix_cache_find(const pgc_prefix_cache *cache, const uint32_t *prompt, uint64_t n,
                          pgc_match *out);
/* containsPromptPrefix: 1 when an entry holds exactly prompt[0, prefix_len). */
int pgc_prefix_cache_contains(const pgc_prefix_cache *cache, const uint32_t *prompt, uint64_t n,
                              uint64_t prefix_len);
void pgc_prefix_cache_touch(pgc_prefix_cache *cache, pgc_match match);
void pgc_prefix_cache_record_hit(pgc_prefix_cache *cache, uint64_t reused_tokens);
void pgc_prefix_cache_record_miss(pgc_prefix_cache *cache);
void pgc_prefix_cache_record_computed(pgc_prefix_cache *cache, uint64_t tokens);
int pgc_prefix_cache_stats(const pgc_prefix_cache *cache, pgc_prefix_stats *out);
/* Entry metadata; tokens_out / pages_out (nullable) receive its token ids and page ids. */
int pgc_prefix_cache_entry(const pgc_prefix_cache *cache, int64_t index, pgc_prefix_entry *out,
                           uint32_t *tokens_out, uint64_t tokens_cap, int32_t *pages_out,
                           int64_t pages_cap);
/* removeEntry: releases the entry's pages and state slot; later indexes shift down. */
int pgc_prefix_cache_remove(pgc_prefix_cache *cache, int64_t index);
/* startDirectEntry (:315-328): an entry with fresh pages for n tokens that the caller prefills
 * in place; finishDirectEntry (:330-337) records the next token and touches it. */
int pgc_prefix_cache_start_direct(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                                  int pinned, pgc_match *out);
int pgc_prefix_cache_finish_direct(pgc_prefix_cache *cache, pgc_match match, uint32_t next_token);
/* setEntryHidden (:258-268): the entry's hidden rows (in its pages) are now real. */
int pgc_prefix_cache_set_hidden_valid(pgc_prefix_cache *cache, pgc_match match, int valid);
/* storePrefixFromWork (:344-424): caches ids[0, n) whose rows the work sequence's block table
 * holds (work_table, >= ceil(n / page_tokens) live pages). reuse (nullable) is the match the
 * work sequence forked from; that entry is extended in place. suffix_hidden != 0: the work
 * pages hold real hidden rows for [reuse.len, n). next_token (nullable) caches the next token.
 * *copy_linear_state (nullable) = 1 when the caller must copy the work sequence's linear state
 * into the entry's state slot. */
int pgc_prefix_cache_store(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                           const pgc_match *reuse, const int32_t *work_table, int64_t work_pages,
                           int suffix_hidden, const uint32_t *next_token, int pinned,
                           pgc_match *out, int *copy_linear_state);
/* prefixState (:278-283) for paged KV: the first ceil(match.len / page_tokens) pages of the
 * entry, one reference each taken for the caller, written to table_out. */
int pgc_prefix_cache_fork(pgc_prefix_cache *cache, pgc_match match, int32_t *table_out,
                          int64_t table_cap, int64_t *pages_out);
/* Evicts LRU unpinned entries until `need_free` pages are free (pages still held by running
 * sequences are not freed by evicting their entry); PGC_ERR_CAPACITY when nothing is left. */
int pgc_prefix_cache_evict_for_pages(pgc_prefix_cache *cache, int32_t need_free);
/* loadEntrySlot + finishLoadedEntry (:426-453): clears the cache, then one pinned entry with
 * fresh pages for a snapshot file's tokens (restore the file image into them), then indexed. */
int pgc_prefix_cache_load_slot(pgc_prefix_cache *cache, const uint32_t *ids, uint64_t n,
                               pgc_match *out);
int pgc_prefix_cache_finish_loaded(pgc_prefix_cache *cache, pgc_match match);
/* persistedEntryConst (:153-163): the active entry, else the most recently used one. */
int pgc_prefix_cache_persisted(const pgc_prefix_cache *cache, pgc_match *out);

/* ---------------------------------------------------------------------------------------
 * Linear attention (Gated-DeltaNet) state producers: the causal conv1d + SiLU and the gated
 * delta-rule recurrence, for the 24 linear layers whose states pgc_copy_regions snapshots,
 * restores and rolls back. Shapes are the model's (src/model/block_linear.zig:18-26).
 * Per sequence: conv state f32 [3][8192] (oldest first), recurrent state f32 [32][128][128]
 * ([Hv][Dv][Dk]); conv_out rows are [q 2048 | k 2048 | v 4096] bf16. Decode entries take a
 * batch of sequences whose states live in slot arrays (`slots` [batch] int32 device indices;
 * NULL = sequence i uses slot i) and update them in place.
 * ------------------------------------------------------------------------------------- */
#define PGC_LIN_KEY_HEADS 16
#define PGC_LIN_VALUE_HEADS 32
#define PGC_LIN_HEAD_DIM 128
#define PGC_LIN_CONV_DIM 8192
#define PGC_LIN_CONV_KERNEL 4

/* conv1d_silu_decode_bf16 (shaders/conv1d.metal:49-66): x [batch][8192] bf16, weight
 * [8192][4] bf16 (8-byte aligned), out [batch][8192] bf16; conv_states [num_slots][3][8192]. */
int pgc_conv1d_decode(float *conv_states, int64_t num_slots, const int32_t *slots, int batch,
                      const uint16_t *x, const uint16_t *weight, uint16_t *out, void *stream);

/* conv1d_silu_prefill_vec4_bf16 + conv1d_silu_prefill_state_bf16 (conv1d.metal:128-186) for one
 * sequence: x/out [tokens][8192] bf16; the state is read (has_previous_state) then published. */
int pgc_conv1d_prefill(float *conv_state, int has_previous_state, const uint16_t *x, int tokens,
                       const uint16_t *weight, uint16_t *out, void *stream);

/* gated_delta_decode_h128_fused_bf16 (shaders/gated_delta.metal:146-261) over a batch: conv_out
 * [batch][8192] bf16 (16-byte aligned), a/b [batch][32] bf16, a_log [32] f32, dt_bias [32] bf16,
 * y [batch][4096] bf16; states [num_slots][32][128][128] f32 updated in place. */
int pgc_gated_delta_decode(float *states, int64_t num_slots, const int32_t *slots, int batch,
                           int has_previous_state, const uint16_t *conv_out, const uint16_t *a,
                           const uint16_t *b, const float *a_log, const uint16_t *dt_bias,
                           uint16_t *y, void *stream);

/* Prefill of one sequence (src/model/block_linear.zig:335-346: qk_l2norm_prefill_bf16,
 * gating_many_bf16, gated_delta_prefill_h128_norm_prepared_value_major_r8_bf16): conv_out
 * [tokens][8192], a/b [tokens][32], y [tokens][4096]. Workspace: normalised q/k and gates. */
size_t pgc_gated_delta_prefill_workspace_bytes(int tokens);
int pgc_gated_delta_prefill(float *state, int has_previous_state, const uint16_t *conv_out,
                            const uint16_t *a, const uint16_t *b, const float *a_log,
                            const uint16_t *dt_bias, int tokens, uint16_t *y, void *workspace,
                            size_t workspace_bytes, void *stream);

/* ---------------------------------------------------------------------------------------
 * Context-parallel decode over NVLink peer memory (BASELINE config 5b; the reference is single
 * device). Rank g of `world` (<= PGC_CP_MAX_RANKS) GPUs holds a contiguous KV shard of one
 * sequence. pgc_cp_decode_attn runs the split decode over the local shard and then one exchange
 * kernel that merges the splits, stores the rank's (m, l, o) partial into every rank's exchange
 * buffer as 8-byte words tagged with the call's epoch, polls its own buffer (bounded, ~2 s, then
 * PGC_ERR_TIMEOUT through pgc_device_error) until every rank's words for this call have landed,
 * and merges the world partials (+ sigmoid gate) into the bf16 output on every rank. No
 * collective library and no fence is involved.
 * Setup: each rank allocates its buffer with pgc_cp_buffer_alloc, exports it with
 * pgc_ipc_get_handle, the handles are exchanged by the caller (any host channel) and opened
 * with pgc_ipc_open_handle; `buffers[i]` is rank i's buffer as mapped in this process (its own
 * at [rank]). `epoch` starts at 1 on freshly allocated (zeroed) buffers and increases by one per
 * call, identically on every rank (2^32 - 1 calls per allocation).
 * ------------------------------------------------------------------------------------- */
#define PGC_CP_MAX_RANKS 8
#define PGC_IPC_HANDLE_BYTES 64
size_t pgc_cp_buffer_bytes(int world);
int pgc_cp_buffer_alloc(int world, void **buffer_out);  /* device memory, zeroed */
int pgc_cp_buffer_free(void *buffer);
int pgc_ipc_get_handle(void *buffer, void *handle_out);
int pgc_ipc_open_handle(const void *handle, void **buffer_out);
int pgc_ipc_close(void *buffer);
int pgc_cp_decode_attn(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                       int64_t num_pages, const int32_t *block_table, int max_pages,
                       const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                       uint16_t *out, void *workspace, size_t workspace_bytes,
                       void *const *buffers, int world, int rank, uint32_t epoch, void *stream);

/* pgc_cp_decode_attn with the decode append of the step fused in, as pgc_decode_attn_append does
 * for one GPU: every rank computes the query rows (RMSNorm + RoPE at the global `position`) from
 * the packed q | gate input (q_head_stride 512; 256 for q alone, ungated), and the rank whose
 * shard holds the new token writes its K/V rows at `slot` (its index in this rank's pool; -1 on
 * the other ranks). `shard_start` is the global position of this rank's first cached token, so
 * position - shard_start is the token's index in the shard (seq_len counts it on the owner).
 * One token per call; the rest as pgc_cp_decode_attn. */
int pgc_cp_decode_attn_append(const uint16_t *q_in, int q_head_stride, const uint16_t *k_in,
                              const uint16_t *v_in, const uint16_t *q_norm_w, const uint16_t *k_norm_w,
                              const float *rope_table, int64_t rope_max_pos, const int32_t *position,
                              const int64_t *slot, int64_t shard_start, uint16_t *k_pages,
                              uint16_t *v_pages, int64_t num_pages, const int32_t *block_table, int max_pages,
                              const int32_t *seq_len, int max_seq_len, float scale, uint16_t *out,
                              void *workspace, size_t workspace_bytes, void *const *buffers, int world,
                              int rank, uint32_t epoch, void *stream);

/* The same context-parallel decode with the partials exchanged by an NCCL all-gather (the
 * reference is single device; BASELINE config 5b names this collective). One layer:
 * pgc_decode_attn_partials over the local shard into this rank's slot of `gathered`
 * ([world][16][258] fp32, device), an in-place ncclAllGather on `stream`, then
 * pgc_merge_partials with the gate into `out` [16][256] bf16 on every rank. `comm` is an
 * ncclComm_t of the context-parallel group (rank and size are read from it). NCCL is loaded at
 * run time (libnccl.so.2, the copy already in the process if any); PGC_ERR_NCCL when it is
 * missing or a call fails. Setup without another NCCL binding: rank 0 calls
 * pgc_nccl_get_unique_id, the 128 bytes travel to the other ranks over any host channel, and
 * every rank calls pgc_nccl_comm_init with its device current; pgc_nccl_comm_destroy at the end. */
#define PGC_NCCL_UNIQUE_ID_BYTES 128
int pgc_nccl_get_unique_id(void *id_out);
int pgc_nccl_comm_init(int world, int rank, const void *id, void **comm_out);
int pgc_nccl_comm_destroy(void *comm);
int pgc_cp_decode_attn_nccl(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                            int64_t num_pages, const int32_t *block_table, int max_pages,
                            const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                            uint16_t *out, float *gathered, void *workspace, size_t workspace_bytes,
                            void *comm, void *stream);

/* ---------------------------------------------------------------------------------------
 * q4 (group-64 affine) projections around the attention kernels: weight u32 [out][in/8], 8
 * nibbles per word with the low nibble at the lowest input column; scales and biases bf16
 * [out][in/64]; w = scale * q + bias (shaders/linear.metal:12-20).
 * ------------------------------------------------------------------------------------- */
/* q4_affine_group64_dequantize_bf16 (linear.metal:422-444): out bf16 [out][in], bit-exact
 * bf16(scale * q + bias). The prefill projections use it once per weight (the reference's
 * prepared dense RHS, src/model/mlx_nt.zig) followed by a dense bf16 GEMM. in_dim % 64 == 0. */
int pgc_q4_dequantize(const uint32_t *weight, const uint16_t *scales, const uint16_t *biases,
                      uint16_t *out, int out_dim, int in_dim, void *stream);

/* The prefill projections' dense GEMM (src/model/block_attn.zig:96-108: the prepared dense RHS
 * of each q4 weight, src/model/mlx_nt.zig, multiplied by MLX's NT GEMM, shaders/mlx_gemm.metal):
 * y_i[t][o] = sum_k x[t][k] * weights_i[o][k] for i < n_weights, fp32 accumulation, bf16
 * output rounded to nearest. x [tokens][in_dim], weights_i [out_dims[i]][in_dim] (for example
 * pgc_q4_dequantize's output), outs[i] [tokens][out_dims[i]], all bf16 and 16-byte aligned;
 * in_dim % 64 == 0, out_dims[i] % 8 == 0, 1 <= n_weights <= PGC_LINEAR_MAX_WEIGHTS. The weights
 * that share an input (the q | gate, k and v projections) go in one call: their tiles form one
 * work queue on the tensor cores. Timeouts are recorded in unit 6 of pgc_device_error. */
#define PGC_LINEAR_MAX_WEIGHTS 4
int pgc_prefill_linear(const uint16_t *x, int tokens, int in_dim, int n_weights,
                       const uint16_t *const *weights, const int *out_dims, uint16_t *const *outs,
                       void *stream);

/* linear_q4_affine_group64_qmv_fast_bf16 (linear.metal:158-194) for decode batches:
 * y[t][o] = sum_k x[t][k] * w[o][k], x [tokens][in] bf16, y [tokens][out] bf16, in fp32 with the
 * reference decode algebra per 64-input group (scale * sum(q x) + bias * sum(x), unrounded
 * weights). in_dim a multiple of 2048 up to 8192, out_dim % 64 == 0; x, weight, scales and
 * biases 16-byte aligned. Up to 64 tokens share one pass over the packed weights; larger
 * batches take one pass per 64 tokens. */
int pgc_q4_linear(const uint16_t *x, int tokens, const uint32_t *weight, const uint16_t *scales,
                  const uint16_t *biases, uint16_t *y, int out_dim, int in_dim, void *stream);

/* pgc_q4_linear for up to PGC_LINEAR_MAX_WEIGHTS weights that share the input x (the q | gate, k
 * and v projections of a decode step, block_attn.zig:309-320): outs[i] = x w_i^T with the same
 * algebra and rules per weight. At 1-2 tokens all of them run as one launch of the CUDA-core
 * GEMV (their row blocks form one grid); at more tokens each weight is its own tensor-core pass. */
int pgc_q4_linear_multi(const uint16_t *x, int tokens, int in_dim, int n_weights,
                        const uint32_t *const *weights, const uint16_t *const *scales,
                        const uint16_t *const *biases, uint16_t *const *outs, const int *out_dims,
                        void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PEREGRINE_CUDA_H */
