"""Context-parallel decode over several GPUs (one long sequence, KV sharded by position).

The reference has no multi-GPU path; this is the B200 design for sequences beyond one GPU's
HBM or latency budget (BASELINE config 5b): rank g holds the contiguous, page-aligned KV shard
[start_g, end_g) of every full-attention layer. A decode step on one layer is
  1. pgc_decode_attn_partials over the local shard -> (m, l, o[256]) per query row (fp32),
  2. an all-gather of those partials across ranks (NCCL over NVLink; 16 rows x 258 floats =
     16.5 KB per rank per layer per query token),
  3. pgc_merge_partials: the log-sum-exp combine of attention_decode.metal:215-243 applied to
     the gathered shard partials, optional sigmoid gate, bf16 output on every rank.
The new token's K/V row is appended only on the rank owning its position (the tail shard).
Three exchange paths: `NcclGroup.decode_layer` runs the library's NCCL path
(pgc_cp_decode_attn_nccl: partials, in-place ncclAllGather, merge, all behind the C ABI, on a
communicator the library creates), `cp_decode_layer` all-gathers through torch.distributed (the
same steps composed in Python), and `PeerExchange.decode_layer` moves the partials with the
library's own exchange kernel over NVLink peer memory (merge, stores into every rank's buffer,
epoch flags, final merge in one kernel).
"""
from __future__ import annotations

from . import capi

PAGE = capi.PAGE_TOKENS


def shard_bounds(total_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous shard of positions for `rank`; boundaries are page aligned so every shard's
    block table starts on a page edge. The last shard takes the remainder."""
    per = -(-total_tokens // world)
    per = -(-per // PAGE) * PAGE
    start = min(rank * per, total_tokens)
    end = min(start + per, total_tokens)
    return start, end


def owner_of(position: int, total_capacity: int, world: int) -> int:
    """Rank whose shard holds `position` under shard_bounds(total_capacity, world, .)."""
    for r in range(world):
        s, e = shard_bounds(total_capacity, world, r)
        if s <= position < e:
            return r
    return world - 1


def gather_partials(local, gathered, group=None) -> None:
    """All-gather the local partials [rows, 258] into gathered [world, rows, 258]. A single
    rank (no process group) simply copies its own partials."""
    import torch.distributed as dist
    if not dist.is_initialized() or gathered.shape[0] == 1:
        gathered[0].copy_(local)
        return
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local, group=group)
    else:
        parts = list(gathered.unbind(0))
        dist.all_gather(parts, local, group=group)


class PeerExchange:
    """Exchange buffers of the context-parallel group, mapped into this process.

    Every rank allocates its buffer in the library (pgc_cp_buffer_alloc), exports a CUDA IPC
    handle, and the handles travel over the process group as host objects (the only use of
    torch.distributed here); each rank then maps every peer's buffer. Decode steps then move
    their partials with the library's exchange kernel, GPU to GPU over NVLink."""

    def __init__(self, world: int, rank: int, group=None):
        import ctypes as C

        import torch.distributed as dist
        self.world, self.rank = world, rank
        own = C.c_void_p()
        capi.check(capi.lib().pgc_cp_buffer_alloc(world, C.byref(own)), "pgc_cp_buffer_alloc")
        self._own = own.value
        handle = (C.c_uint8 * 64)()
        capi.check(capi.lib().pgc_ipc_get_handle(self._own, handle), "pgc_ipc_get_handle")
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        else:
            handles[0] = bytes(handle)
        self._opened = []
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            h = (C.c_uint8 * 64).from_buffer_copy(handles[r])
            p = C.c_void_p()
            capi.check(capi.lib().pgc_ipc_open_handle(h, C.byref(p)), "pgc_ipc_open_handle")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.buffers = (C.c_void_p * world)(*ptrs)
        self.epoch = 0

    def close(self) -> None:
        for p in self._opened:
            capi.lib().pgc_ipc_close(p)
        self._opened = []
        if self._own:
            capi.lib().pgc_cp_buffer_free(self._own)
            self._own = None

    def decode_layer(self, q, k_pages, v_pages, block_table, local_len_dev, local_max_len, scale,
                     workspace, out, gate=None, stream=None) -> None:
        """One layer of context-parallel decode for one query token: split decode over the
        local shard, then the peer exchange + merge kernel; out [16, 256] bf16 on every rank.
        Every rank calls it once per layer in the same order (the epoch counts calls)."""
        self.epoch += 1
        capi.check(capi.lib().pgc_cp_decode_attn(
            q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), k_pages.shape[0],
            block_table.data_ptr(), block_table.shape[-1], local_len_dev.data_ptr(),
            max(local_max_len, 1), scale, None if gate is None else gate.data_ptr(), out.data_ptr(),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), self.buffers,
            self.world, self.rank, self.epoch, capi._stream(stream)), "pgc_cp_decode_attn")


    def decode_layer_append(self, q_in, k_in, v_in, rope, position, slot, shard_start, k_pages, v_pages,
                            block_table, local_len_dev, local_max_len, scale, workspace, out,
                            q_norm_w=None, k_norm_w=None, stream=None) -> None:
        """decode_layer with the step's append fused in (pgc_cp_decode_attn_append): q_in is
        the packed q | gate [1, 16, 512] (or q alone [1, 16, 256]), position [1] the global
        position (RoPE), slot [1] the new token's index in this rank's pool or -1 where another
        rank owns it, shard_start this rank's first global position."""
        self.epoch += 1
        capi.check(capi.lib().pgc_cp_decode_attn_append(
            q_in.data_ptr(), q_in.shape[-1], k_in.data_ptr(), v_in.data_ptr(),
            None if q_norm_w is None else q_norm_w.data_ptr(),
            None if k_norm_w is None else k_norm_w.data_ptr(), rope.data_ptr(), rope.shape[0],
            position.data_ptr(), slot.data_ptr(), shard_start, k_pages.data_ptr(), v_pages.data_ptr(),
            k_pages.shape[0], block_table.data_ptr(), block_table.shape[-1], local_len_dev.data_ptr(),
            max(local_max_len, 1), scale, out.data_ptr(), workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), self.buffers, self.world, self.rank, self.epoch,
            capi._stream(stream)), "pgc_cp_decode_attn_append")


class NcclGroup:
    """An NCCL communicator of the context-parallel group, made through the library's C ABI:
    rank 0 draws the unique id (pgc_nccl_get_unique_id), the 128 bytes travel over the process
    group as a host object, and every rank joins with pgc_nccl_comm_init on its current device.
    A host without torch does the same with any channel for the id."""

    def __init__(self, world: int, rank: int, group=None):
        import ctypes as C

        import torch.distributed as dist
        self.world, self.rank = world, rank
        uid = (C.c_uint8 * 128)()
        if rank == 0:
            capi.check(capi.lib().pgc_nccl_get_unique_id(uid), "pgc_nccl_get_unique_id")
        if world > 1:
            obj = [bytes(uid)]
            dist.broadcast_object_list(obj, src=0, group=group)
            uid = (C.c_uint8 * 128).from_buffer_copy(obj[0])
        comm = C.c_void_p()
        capi.check(capi.lib().pgc_nccl_comm_init(world, rank, uid, C.byref(comm)), "pgc_nccl_comm_init")
        self.comm = comm.value

    def close(self) -> None:
        if self.comm:
            capi.check(capi.lib().pgc_nccl_comm_destroy(self.comm), "pgc_nccl_comm_destroy")
            self.comm = None

    def decode_layer(self, q, k_pages, v_pages, block_table, local_len_dev, local_max_len, scale,
                     gathered, workspace, out, gate=None, stream=None) -> None:
        """One layer for one query token: partials of the local shard, in-place all-gather into
        gathered [world, 16, 258] fp32, merge + gate into out [16, 256] bf16 on every rank."""
        capi.check(capi.lib().pgc_cp_decode_attn_nccl(
            q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), k_pages.shape[0],
            block_table.data_ptr(), block_table.shape[-1], local_len_dev.data_ptr(),
            max(local_max_len, 1), scale, None if gate is None else gate.data_ptr(), out.data_ptr(),
            gathered.data_ptr(), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            self.comm, capi._stream(stream)), "pgc_cp_decode_attn_nccl")


def cp_decode_layer(q, k_pages, v_pages, block_table, local_len_dev, local_max_len, scale,
                    partial, gathered, workspace, out, gate=None, group=None, stream=None):
    """One layer of context-parallel decode for one sequence and one query token.

    q [1, 1, 16, 256] bf16 (same on every rank), block_table [1, pages] of the local shard,
    local_len_dev [1] int32 (tokens of the shard, may be 0), partial [16, 258] fp32,
    gathered [world, 16, 258] fp32, out [16, 256] bf16 (written on every rank)."""
    capi.decode_attn_partials(q, k_pages, v_pages, block_table, local_len_dev,
                              max(local_max_len, 1), scale, partial, workspace, stream=stream)
    gather_partials(partial, gathered, group)
    rows = partial.shape[0]
    capi.merge_partials(gathered, rows, gathered.shape[0], rows * capi.PARTIAL_FLOATS, out,
                        gate=gate, stream=stream)
