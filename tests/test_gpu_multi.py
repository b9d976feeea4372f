"""Multi-GPU row-block sharding on real GPUs (NCCL), when more than one GPU
is visible; skipped otherwise.

Every rank computes its rows of C for a W=64 signed product, B is
all-gathered from the ranks' row blocks and C's rows reach rank 0 -- by NCCL
point-to-point transfers, and again by the final kernel of every rank storing
into rank 0's buffer through a CUDA IPC mapping -- and rank 0 compares each
assembled product with a one-GPU product of the same inputs, bit for bit.
NVLS is switched off for this test.
"""
import os
import socket
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime

        import torch
        import torch.distributed as dist

        import mfft_bench_b200 as m
        from mfft_bench_b200 import dist as D
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        ctx = m.Context(rank, stream=torch.cuda.current_stream())
        ranges = D.all_ranges(n, world)
        r0, r1 = ranges[rank]
        A = torch.empty(n * n, dtype=torch.int64, device=dev)
        Bfull = torch.empty_like(A)
        ctx.gen_int64(A, 777)
        ctx.gen_int64(Bfull, 888)
        ctx.sync()
        B = torch.zeros_like(A)
        D.allgather_rows(Bfull.view(n, n)[r0:r1].contiguous().view(-1), B, n, ranges)
        out = ctx.mm_i64(A, B, n, RL=9, rows=(r0, r1))
        full = torch.empty(9 * n * n, dtype=torch.uint16, device=dev) if rank == 0 else None
        ctx.sync()
        D.gather_planes_to_root(out, full, n, 9, ranges)
        want = None
        if rank == 0:
            want = ctx.mm_i64(A, Bfull, n, RL=9)
            ctx.sync()
            assert torch.equal(full.view(torch.int16), want.view(torch.int16)), "sharded != 1 GPU"
        # the same product with every rank's final kernel storing its rows
        # straight into rank 0's buffer through a CUDA IPC mapping
        peer = D.PeerOutput(9 * n * n, "uint16")
        ctx.set_output_plane_stride(n * n)
        ctx.mm_i64(A, B, n, RL=9, out=peer.ptr + r0 * n * 2, rows=(r0, r1))
        ctx.set_output_plane_stride(0)
        ctx.sync()
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.all_reduce(flag)
        torch.cuda.synchronize()
        if rank == 0:
            assert torch.equal(peer.tensor.view(torch.int16), want.view(torch.int16)), \
                "peer-stored rows != 1 GPU"
        peer.close()
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_sharded_product_matches_single_gpu():
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    n = 2048 + 64  # rows not divisible into whole 128-row tiles per rank
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, n, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), msgs
