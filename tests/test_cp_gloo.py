"""Context-parallel decode host logic on CPU: world_size-2 gloo ranks, each holding one KV
shard, exchange their (m, l, o) partials with the same gather the GPU path uses, and the LSE
merge of the gathered partials must equal attention over the whole cache (oracle)."""
import os
import socket

import numpy as np
import pytest

D, NQ, NKV, PAGE = 256, 16, 4, 16


def test_shard_bounds_cover_and_align():
    from peregrine_b200.cp import owner_of, shard_bounds
    for total in (1, 15, 16, 17, 4097, 262144, 262145):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
            for a, _ in spans:
                assert a % PAGE == 0 or a == total
            for pos in (0, total - 1):
                r = owner_of(pos, total, world)
                assert spans[r][0] <= pos < spans[r][1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, L, result_path):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from oracle import oracle
    from peregrine_b200.cp import gather_partials, shard_bounds

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q = oracle.normal_bf16(NQ * D, 1).reshape(1, 1, NQ, D)
        k = oracle.normal_bf16(L * NKV * D, 2).reshape(L, NKV, D)
        v = oracle.normal_bf16(L * NKV * D, 3).reshape(L, NKV, D)
        s, e = shard_bounds(L, world, rank)
        n = e - s
        pages = max(1, (n + PAGE - 1) // PAGE)
        kp = np.zeros((pages, NKV, PAGE, D), np.uint16)
        vp = np.zeros_like(kp)
        for t in range(n):
            kp[t // PAGE, :, t % PAGE] = k[s + t]
            vp[t // PAGE, :, t % PAGE] = v[s + t]
        table = np.arange(pages, dtype=np.int32).reshape(1, -1)
        if n > 0:
            local = oracle.decode_partials_paged(q, kp, vp, table, np.array([n], np.int32), 1 / 16)[0]
        else:
            local = np.zeros((NQ, 258), np.float32)
            local[:, 0] = -np.inf
        gathered = torch.empty((world, NQ, 258), dtype=torch.float32)
        gather_partials(torch.from_numpy(np.ascontiguousarray(local)), gathered)
        merged, _ = oracle.merge_partials(np.ascontiguousarray(gathered.numpy()), NQ, world, NQ * 258)
        if rank == 0:
            kf, vf, tf = np.zeros((L // PAGE + 1, NKV, PAGE, D), np.uint16), None, None
            vf = np.zeros_like(kf)
            for t in range(L):
                kf[t // PAGE, :, t % PAGE] = k[t]
                vf[t // PAGE, :, t % PAGE] = v[t]
            tf = np.arange(kf.shape[0], dtype=np.int32).reshape(1, -1)
            full, _ = oracle.decode_paged(q, kf, vf, tf, np.array([L], np.int32), 1 / 16)
            np.save(result_path, np.abs(merged - full[0, 0]).max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L", [3000, 16])  # 16 tokens: the second shard is empty
def test_cp_merge_two_gloo_ranks(tmp_path, L):
    import torch.multiprocessing as mp
    world = 2
    out = str(tmp_path / "err.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), L, out), nprocs=world, join=True,
                       start_method="spawn")
    assert float(np.load(out)) < 1e-5
