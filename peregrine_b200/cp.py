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
The collective runs through torch.distributed (the process-group plumbing); the attention and
the merge are the library's kernels.
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
