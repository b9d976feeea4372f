"""Multi-GPU row-block sharding on real GPUs (NCCL), when more than one GPU
is visible; skipped otherwise.

Three products are sharded over every visible GPU (up to 8), one process per
GPU: the W=64 signed int64 path (configs[4]'s kind), the W=1024 unsigned
limb-plane path (configs[2]'s kind, `mm_u16`) and the fp32 embedding on the
512-bit grid (configs[3]'s kind).  Every rank computes its rows of C; B is
all-gathered from the ranks' row blocks, and C's rows reach rank 0 twice --
by NCCL point-to-point transfers, and by the final kernel of every rank
storing into rank 0's buffer through a CUDA IPC mapping.  Rank 0 compares
both assembled products with a one-GPU product of the same inputs, bit for
bit, and checks entries of every shard's first and last rows against the CPU
oracle.  NVLS is switched off for this test.
"""
import os
import socket
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# kind -> (n, planes of an input, output planes, output element)
CASES = {
    # rows not divisible into whole 128-row tiles per rank
    "i64": dict(n=2048 + 64, planes=1, RL=9),
    # W = 1024 unsigned: 64 limbs in, 129 limb planes out
    "u16": dict(n=1024 + 64, planes=64, RL=129),
    # fp32 N(0,1) * 2^k on the 512-bit grid
    "f32": dict(n=1024 + 64, planes=1, RL=1),
}


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(ctx, kind, n, dev):
    import torch
    if kind == "i64":
        A = torch.empty(n * n, dtype=torch.int64, device=dev)
        B = torch.empty_like(A)
        ctx.gen_int64(A, 777)
        ctx.gen_int64(B, 888)
    elif kind == "u16":
        A = torch.empty(64 * n * n, dtype=torch.uint16, device=dev)
        B = torch.empty_like(A)
        ctx.gen_bigmat(A, n, 64, 777)
        ctx.gen_bigmat(B, n, 64, 888)
    else:
        from mfft_bench_b200 import gen_normal_f32
        hA, hB = gen_normal_f32(n, 777)
        A = torch.from_numpy(hA).to(dev)
        B = torch.from_numpy(hB).to(dev)
    ctx.sync()
    return A, B


def _product(ctx, kind, A, B, n, RL, rows, out=None):
    if kind == "i64":
        return ctx.mm_i64(A, B, n, RL=RL, out=out, rows=rows)
    if kind == "u16":
        return ctx.mm_u16(A, B, n, 64, RL=RL, out=out, rows=rows)
    return ctx.fp32(A, B, n, 512, out=out, rows=rows)


def _oracle_entries(kind, A, B, n, RL, rows, cols):
    """Exact entries (rows[i], cols[i]) from the CPU oracle, as the same bytes
    the GPU writes ([RL] uint16 limbs, or one fp32 word)."""
    import numpy as np

    from oracle.oracle import Oracle
    o = Oracle()
    r = np.ascontiguousarray(rows, np.int32)
    c = np.ascontiguousarray(cols, np.int32)
    if kind == "f32":
        return o.fpx_entries(A.cpu().numpy(), B.cpu().numpy(), n, 512, r, c).view(np.uint32)
    if kind == "i64":
        Ap = o.int64_to_planes(A.cpu().numpy(), n)
        Bp = o.int64_to_planes(B.cpu().numpy(), n)
        return o.entries(Ap, Bp, n, 4, True, r, c, RL)
    u16 = lambda t: t.view(__import__("torch").int16).cpu().numpy().view(np.uint16)  # noqa: E731
    return o.entries(u16(A), u16(B), n, 64, False, r, c, RL)


def _rank(rank, world, port, kind, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime

        import numpy as np
        import torch
        import torch.distributed as dist

        import mfft_bench_b200 as m
        from mfft_bench_b200 import dist as D
        cfg = CASES[kind]
        n, P, RL = cfg["n"], cfg["planes"], cfg["RL"]
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        ctx = m.Context(rank, stream=torch.cuda.current_stream())
        ranges = D.all_ranges(n, world)
        r0, r1 = ranges[rank]
        A, Bfull = _inputs(ctx, kind, n, dev)
        # B as this rank holds it before the exchange: its own row block of
        # every plane, the rest zero
        B = torch.zeros_like(Bfull)
        gat = (lambda t: t.view(torch.int16)) if kind == "u16" else (lambda t: t)
        Bv, Bfv = B.view(P, n * n), Bfull.view(P, n, n)
        for u in range(P):
            D.allgather_rows(gat(Bfv[u, r0:r1].contiguous().view(-1)), gat(Bv[u]), n, ranges)
        out = _product(ctx, kind, A, B, n, RL, (r0, r1))
        full = torch.empty(RL * n * n, dtype=out.dtype, device=dev) if rank == 0 else None
        ctx.sync()
        D.gather_planes_to_root(out, full, n, RL, ranges)
        want = None
        bits = (lambda t: t.view(torch.int32)) if kind == "f32" else (lambda t: t.view(torch.int16))
        if rank == 0:
            want = _product(ctx, kind, A, Bfull, n, RL, None)
            ctx.sync()
            assert torch.equal(bits(full), bits(want)), f"{kind}: NCCL-gathered shards != 1 GPU"
            # every shard's first and last row, 8 columns each, against the oracle
            rows = [r for a, b in ranges if b > a for r in (a, b - 1) for _ in range(8)]
            rng = np.random.default_rng(5)
            cols = rng.integers(0, n, len(rows))
            ri = torch.tensor(rows, device=dev)
            ci = torch.tensor(cols, device=dev)
            got = bits(want).view(RL, n, n)[:, ri, ci].cpu().numpy()  # [RL][samples]
            got = got.view(np.uint32 if kind == "f32" else np.uint16).ravel()
            exp = _oracle_entries(kind, A, Bfull, n, RL, rows, cols)
            assert np.array_equal(got, exp.ravel()), f"{kind}: entries differ from the oracle"
        # the same product with every rank's final kernel storing its rows
        # straight into rank 0's buffer through a CUDA IPC mapping
        dt = {"i64": "uint16", "u16": "uint16", "f32": "float32"}[kind]
        peer = D.PeerOutput(RL * n * n, dt)
        ctx.set_output_plane_stride(n * n)
        _product(ctx, kind, A, B, n, RL, (r0, r1), out=peer.ptr + r0 * n * out.element_size())
        ctx.set_output_plane_stride(0)
        ctx.sync()
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        dist.all_reduce(flag)
        torch.cuda.synchronize()
        if rank == 0:
            got = peer.tensor.view(torch.int32 if kind == "f32" else torch.int16)
            assert torch.equal(got, bits(want)), f"{kind}: peer-stored rows != 1 GPU"
        peer.close()
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("kind", sorted(CASES))
def test_sharded_product_matches_single_gpu(kind):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, kind, errq)) for r in range(world)]
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
