"""Context-parallel decode on 2 GPUs through the library: each rank holds one KV shard on its
own GPU. Three exchange paths: pgc_cp_decode_attn_nccl (partials, in-place ncclAllGather and
merge behind the C ABI, on a communicator made by pgc_nccl_comm_init), the same steps composed
through torch.distributed (pgc_decode_attn_partials + all-gather + pgc_merge_partials),
and pgc_cp_decode_attn, whose exchange kernel stores the partials into the peers' buffers over
NVLink and waits on epoch flags. Every rank's output must match the oracle over the whole cache
within the attention tolerance (2e-2 abs + 1e-2 rel). Skipped when fewer than 2 GPUs are
visible; the peer path runs 5 layers back to back (epoch parity buffers)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
D, NQ, NKV, PAGE = 256, 16, 4, 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, L, result_dir, path="torch"):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    from oracle import oracle
    from peregrine_b200 import capi, cp

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        q = oracle.normal_bf16(NQ * D, 1).reshape(1, 1, NQ, D)
        g = oracle.normal_bf16(NQ * D, 4).reshape(NQ, D)
        k = oracle.normal_bf16(L * NKV * D, 2).reshape(L, NKV, D)
        v = oracle.normal_bf16(L * NKV * D, 3).reshape(L, NKV, D)
        s, e = cp.shard_bounds(L, world, rank)
        n = e - s
        pages = max(1, (n + PAGE - 1) // PAGE)
        kp = np.zeros((pages, NKV, PAGE, D), np.uint16)
        vp = np.zeros_like(kp)
        for t in range(n):
            kp[t // PAGE, :, t % PAGE] = k[s + t]
            vp[t // PAGE, :, t % PAGE] = v[s + t]

        def dv(a):
            return torch.from_numpy(np.ascontiguousarray(a.view(np.int16) if a.dtype == np.uint16 else a)).cuda()

        table = dv(np.arange(pages, dtype=np.int32).reshape(1, -1))
        partial = torch.empty((NQ, 258), dtype=torch.float32, device="cuda")
        gathered = torch.empty((world, NQ, 258), dtype=torch.float32, device="cuda")
        ws = torch.empty(capi.decode_workspace_bytes(1, 1, max(n, 1)), dtype=torch.uint8, device="cuda")
        out = torch.empty((NQ, D), dtype=torch.int16, device="cuda")
        if path == "capi_nccl":
            grp = cp.NcclGroup(world, rank)
            for _ in range(3):  # several layers on one communicator
                grp.decode_layer(dv(q), dv(kp), dv(vp), table, dv(np.array([n], np.int32)), n, 1 / 16,
                                 gathered, ws, out, gate=dv(g))
            torch.cuda.synchronize()
            grp.close()
        elif path == "peer":
            ex = cp.PeerExchange(world, rank)
            dist.barrier()
            # several layers in a row: exercises the epoch parity double buffer
            for _ in range(5):
                ex.decode_layer(dv(q), dv(kp), dv(vp), table, dv(np.array([n], np.int32)), n, 1 / 16,
                                ws, out, gate=dv(g))
            torch.cuda.synchronize()
            code, _ = capi.device_error()
            assert code == 0, code
            dist.barrier()
            ex.close()
        else:
            cp.cp_decode_layer(dv(q), dv(kp), dv(vp), table, dv(np.array([n], np.int32)), n, 1 / 16,
                               partial, gathered, ws, out, gate=dv(g))
        torch.cuda.synchronize()
        got = (out.cpu().numpy().view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        kf = np.zeros((L // PAGE + 1, NKV, PAGE, D), np.uint16)
        vf = np.zeros_like(kf)
        for t in range(L):
            kf[t // PAGE, :, t % PAGE] = k[t]
            vf[t // PAGE, :, t % PAGE] = v[t]
        tf = np.arange(kf.shape[0], dtype=np.int32).reshape(1, -1)
        ref, _ = oracle.decode_paged(q, kf, vf, tf, np.array([L], np.int32), 1 / 16, 1, g.reshape(1, 1, NQ, D))
        err = np.abs(got - ref[0, 0])
        ok = bool((err <= 2e-2 + 1e-2 * np.abs(ref[0, 0])).all())
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([float(ok), err.max()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("path", ["capi_nccl", "torch", "peer"])
@pytest.mark.parametrize("L", [5000, 16])
def test_cp_decode_two_gpus(tmp_path, L, path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), L, str(tmp_path), path), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        ok, err = np.load(tmp_path / f"rank{r}.npy")
        assert ok == 1.0, (r, err)
