// prefix_persist.cpp — the on-disk prefix-state snapshot (format v3) on the host side.
//
// Same file format as src/server/prefix_persist.zig:31-137 so that a snapshot written by the
// reference server loads here and the other way round:
//   header (48 B: magic "PRGPFXS1", version 3, dtype 0 = bf16, model fingerprint, token count,
//   cached next token + valid flag, hidden-valid flag), token ids (u32), then per layer in model
//   order (layer i is linear unless (i + 1) % 4 == 0, src/model/decoder_layer.zig:29-31):
//     linear: conv state f32 [3][8192] and recurrent state f32 [32][128][128];
//     full:   K runs [4][count][256] bf16 then V runs [4][256][count] bf16 (the reference's
//             head-major K and value-dim-major V compacted to `count` tokens, :85-137);
//   then the MTP hidden rows [count][4096] bf16.
// The K and V runs are exactly a dense cache of stride `count`, so pgc_kv_restore_dense with
// src_stride = count moves a file image straight into the paged pools (and
// pgc_kv_snapshot_dense writes one). The file is read into / written from a caller buffer —
// pinned host memory, so the restore kernels read it over the host link without a staging copy.
// Validation mirrors load() (:329-413): any mismatch makes the file "not usable"
// (PGC_ERR_FORMAT) and the caller cold-prefills, as the reference does.
#include <cstdio>
#include <cstring>
#include <string>

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/peregrine_cuda.h"

namespace {

constexpr uint64_t kMagic = 0x3153584650475250ull;  // "PRGPFXS1" little-endian
constexpr uint32_t kVersion = 3;
constexpr uint32_t kDtypeBf16 = 0;
constexpr int kLayers = 32;
constexpr uint64_t kConvBytes = 3ull * 8192 * 4;
constexpr uint64_t kRecurBytes = 32ull * 128 * 128 * 4;
constexpr uint64_t kHidden = 4096;

struct Header {
    uint64_t magic;
    uint32_t version;
    uint32_t dtype;
    uint64_t model_fingerprint;
    uint64_t token_count;
    uint32_t next_token;
    uint32_t next_token_valid;
    uint32_t hidden_valid;
    uint32_t pad;  // the extern struct's trailing alignment
};
static_assert(sizeof(Header) == 48, "header is 48 bytes");

inline bool is_linear(int layer) { return (layer + 1) % 4 != 0; }

bool read_all(int fd, void *dst, uint64_t bytes) {
    uint8_t *p = static_cast<uint8_t *>(dst);
    while (bytes > 0) {
        const size_t chunk = bytes > (1u << 30) ? (1u << 30) : (size_t)bytes;
        const ssize_t n = ::read(fd, p, chunk);
        if (n <= 0) return false;
        p += n;
        bytes -= (uint64_t)n;
    }
    return true;
}

bool write_all(int fd, const void *src, uint64_t bytes) {
    const uint8_t *p = static_cast<const uint8_t *>(src);
    while (bytes > 0) {
        const size_t chunk = bytes > (1u << 30) ? (1u << 30) : (size_t)bytes;
        const ssize_t n = ::write(fd, p, chunk);
        if (n <= 0) return false;
        p += n;
        bytes -= (uint64_t)n;
    }
    return true;
}

}  // namespace

extern "C" {

int pgc_prefix_file_layout(uint64_t token_count, pgc_prefix_layout *out) {
    if (!out || token_count == 0 || token_count > (1ull << 32)) return PGC_ERR_INVALID;
    memset(out, 0, sizeof(*out));
    uint64_t off = sizeof(Header);
    out->tokens = off;
    off += token_count * 4;
    int li = 0, fi = 0;
    const uint64_t kv_bytes = 4ull * token_count * 256 * 2;
    for (int l = 0; l < kLayers; ++l) {
        if (is_linear(l)) {
            out->conv[li] = off;
            off += kConvBytes;
            out->recur[li] = off;
            off += kRecurBytes;
            ++li;
        } else {
            out->k_runs[fi] = off;
            off += kv_bytes;
            out->v_runs[fi] = off;
            off += kv_bytes;
            ++fi;
        }
    }
    out->hidden = off;
    off += token_count * kHidden * 2;
    out->total_bytes = off;
    out->token_count = token_count;
    return PGC_OK;
}

int pgc_prefix_file_inspect(const char *path, uint64_t model_fingerprint, uint64_t vocab,
                            uint64_t max_tokens, pgc_prefix_info *info) {
    if (!path || !info) return PGC_ERR_INVALID;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return PGC_ERR_FILE;
    Header h;
    struct stat st;
    const bool ok_read = read_all(fd, &h, sizeof(h)) && ::fstat(fd, &st) == 0;
    ::close(fd);
    if (!ok_read) return PGC_ERR_FORMAT;
    if (h.magic != kMagic || h.version != kVersion || h.dtype != kDtypeBf16) return PGC_ERR_FORMAT;
    if (h.model_fingerprint != model_fingerprint) return PGC_ERR_FORMAT;
    if (h.next_token_valid > 1 || h.hidden_valid > 1) return PGC_ERR_FORMAT;
    if (h.next_token_valid == 1 && h.next_token >= vocab) return PGC_ERR_FORMAT;
    if (h.token_count == 0 || h.token_count > max_tokens) return PGC_ERR_FORMAT;
    pgc_prefix_layout lay;
    if (pgc_prefix_file_layout(h.token_count, &lay) != PGC_OK) return PGC_ERR_FORMAT;
    if ((uint64_t)st.st_size != lay.total_bytes) return PGC_ERR_FORMAT;
    info->token_count = h.token_count;
    info->next_token = h.next_token;
    info->next_token_valid = h.next_token_valid;
    info->hidden_valid = h.hidden_valid;
    info->file_bytes = lay.total_bytes;
    return PGC_OK;
}

int pgc_prefix_file_read(const char *path, uint64_t model_fingerprint, uint64_t vocab,
                         uint64_t max_tokens, void *image, uint64_t image_bytes,
                         pgc_prefix_info *info) {
    if (!image) return PGC_ERR_INVALID;
    pgc_prefix_info local;
    int st = pgc_prefix_file_inspect(path, model_fingerprint, vocab, max_tokens, &local);
    if (st != PGC_OK) return st;
    if (image_bytes < local.file_bytes) return PGC_ERR_BOUNDS;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return PGC_ERR_FILE;
    const bool ok = read_all(fd, image, local.file_bytes);
    ::close(fd);
    if (!ok) return PGC_ERR_FILE;
    if (info) *info = local;
    return PGC_OK;
}

int pgc_prefix_file_header(void *image, uint64_t image_bytes, uint64_t model_fingerprint,
                           uint64_t token_count, uint32_t next_token, int next_token_valid,
                           int hidden_valid) {
    if (!image || token_count == 0) return PGC_ERR_INVALID;
    pgc_prefix_layout lay;
    if (pgc_prefix_file_layout(token_count, &lay) != PGC_OK) return PGC_ERR_INVALID;
    if (image_bytes < lay.total_bytes) return PGC_ERR_BOUNDS;
    Header h;
    memset(&h, 0, sizeof(h));
    h.magic = kMagic;
    h.version = kVersion;
    h.dtype = kDtypeBf16;
    h.model_fingerprint = model_fingerprint;
    h.token_count = token_count;
    h.next_token = next_token;
    h.next_token_valid = next_token_valid ? 1 : 0;
    h.hidden_valid = hidden_valid ? 1 : 0;
    memcpy(image, &h, sizeof(h));
    return PGC_OK;
}

int pgc_prefix_file_write(const char *path, const void *image, uint64_t image_bytes) {
    if (!path || !image || image_bytes < sizeof(Header)) return PGC_ERR_INVALID;
    Header h;
    memcpy(&h, image, sizeof(h));
    pgc_prefix_layout lay;
    if (h.magic != kMagic || pgc_prefix_file_layout(h.token_count, &lay) != PGC_OK ||
        image_bytes != lay.total_bytes)
        return PGC_ERR_FORMAT;
    // atomic replace: write a temporary file in the same directory, fsync, rename
    const std::string tmp = std::string(path) + ".tmp." + std::to_string((long)::getpid());
    const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return PGC_ERR_FILE;
    bool ok = write_all(fd, image, image_bytes) && ::fsync(fd) == 0;
    ok = (::close(fd) == 0) && ok;
    if (!ok || ::rename(tmp.c_str(), path) != 0) {
        ::unlink(tmp.c_str());
        return PGC_ERR_FILE;
    }
    return PGC_OK;
}

}  // extern "C"
