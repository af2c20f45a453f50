// cp_nccl.cpp — context-parallel decode with the partials exchanged by an NCCL all-gather
// (BASELINE config 5b's "NCCL all-gather over NVLink" path), behind the C ABI.
//
// Rank g of the communicator holds a contiguous KV shard of one sequence. One layer:
//   1. pgc_decode_attn_partials over the local shard -> this rank's (m, l, o[256]) for the 16
//      query heads, written straight into its slot of the gathered buffer;
//   2. an in-place ncclAllGather of the 16 x 258 fp32 partials on the caller's stream;
//   3. pgc_merge_partials: the log-sum-exp combine of attention_decode.metal:215-243 over the
//      ranks' partials, the sigmoid gate, bf16 output on every rank.
// NCCL is loaded at run time (libnccl.so.2; the copy already in the process if there is one),
// so the library itself has no link-time NCCL dependency and loads on hosts without it.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "pgc_internal.h"

namespace {

// The few NCCL entry points used here, with NCCL's C signatures (nccl.h): the communicator is
// an opaque pointer, the unique id 128 bytes passed by value, results are ints (0 = success).
struct NcclUniqueId {
    char internal[PGC_NCCL_UNIQUE_ID_BYTES];
};
using GetUniqueIdFn = int (*)(NcclUniqueId *);
using CommInitRankFn = int (*)(void **, int, NcclUniqueId, int);
using CommDestroyFn = int (*)(void *);
using CommCountFn = int (*)(void *, int *);
using CommUserRankFn = int (*)(void *, int *);
using AllGatherFn = int (*)(const void *, void *, size_t, int, void *, cudaStream_t);
constexpr int kNcclFloat32 = 7;

struct Nccl {
    GetUniqueIdFn get_unique_id = nullptr;
    CommInitRankFn comm_init_rank = nullptr;
    CommDestroyFn comm_destroy = nullptr;
    CommCountFn comm_count = nullptr;
    CommUserRankFn comm_user_rank = nullptr;
    AllGatherFn all_gather = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.get_unique_id = reinterpret_cast<GetUniqueIdFn>(dlsym(h, "ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<CommInitRankFn>(dlsym(h, "ncclCommInitRank"));
        n.comm_destroy = reinterpret_cast<CommDestroyFn>(dlsym(h, "ncclCommDestroy"));
        n.comm_count = reinterpret_cast<CommCountFn>(dlsym(h, "ncclCommCount"));
        n.comm_user_rank = reinterpret_cast<CommUserRankFn>(dlsym(h, "ncclCommUserRank"));
        n.all_gather = reinterpret_cast<AllGatherFn>(dlsym(h, "ncclAllGather"));
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.comm_count &&
               n.comm_user_rank && n.all_gather;
    });
    return n;
}

}  // namespace

extern "C" {

int pgc_nccl_get_unique_id(void *id_out) {
    if (!id_out) return PGC_ERR_INVALID;
    const Nccl &n = nccl();
    if (!n.ok) return PGC_ERR_NCCL;
    NcclUniqueId id;
    if (n.get_unique_id(&id) != 0) return PGC_ERR_NCCL;
    memcpy(id_out, &id, sizeof(id));
    return PGC_OK;
}

int pgc_nccl_comm_init(int world, int rank, const void *id, void **comm_out) {
    if (!id || !comm_out || world < 1 || rank < 0 || rank >= world) return PGC_ERR_INVALID;
    const Nccl &n = nccl();
    if (!n.ok) return PGC_ERR_NCCL;
    NcclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    void *comm = nullptr;
    if (n.comm_init_rank(&comm, world, uid, rank) != 0 || comm == nullptr) return PGC_ERR_NCCL;
    *comm_out = comm;
    return PGC_OK;
}

int pgc_nccl_comm_destroy(void *comm) {
    if (!comm) return PGC_ERR_INVALID;
    const Nccl &n = nccl();
    if (!n.ok) return PGC_ERR_NCCL;
    return n.comm_destroy(comm) == 0 ? PGC_OK : PGC_ERR_NCCL;
}

int pgc_cp_decode_attn_nccl(const uint16_t *q, const uint16_t *k_pages, const uint16_t *v_pages,
                            int64_t num_pages, const int32_t *block_table, int max_pages,
                            const int32_t *seq_len, int max_seq_len, float scale, const uint16_t *gate,
                            uint16_t *out, float *gathered, void *workspace, size_t workspace_bytes,
                            void *comm, void *stream) {
    if (!gathered || !comm || !out) return PGC_ERR_INVALID;
    const Nccl &n = nccl();
    if (!n.ok) return PGC_ERR_NCCL;
    int world = 0, rank = 0;
    if (n.comm_count(comm, &world) != 0 || n.comm_user_rank(comm, &rank) != 0 || world < 1 ||
        rank < 0 || rank >= world)
        return PGC_ERR_NCCL;
    const size_t count = (size_t)PGC_NUM_Q_HEADS * PGC_PARTIAL_FLOATS;
    float *mine = gathered + (size_t)rank * count;
    int st = pgc_decode_attn_partials(q, k_pages, v_pages, num_pages, block_table, max_pages, seq_len, 1, 1,
                                      max_seq_len, scale, mine, workspace, workspace_bytes, stream);
    if (st != PGC_OK) return st;
    // in place: rank r's slot is gathered + r * count on every rank
    if (n.all_gather(mine, gathered, count, kNcclFloat32, comm, static_cast<cudaStream_t>(stream)) != 0)
        return PGC_ERR_NCCL;
    return pgc_merge_partials(gathered, PGC_NUM_Q_HEADS, world, (int64_t)count, gate, out, stream);
}

}  // extern "C"
