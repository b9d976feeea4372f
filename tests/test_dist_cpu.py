"""Multi-process (gloo, world size 2) tests of the row-block sharding logic.

The GPU compute of a rank is replaced here by the CPU oracle computing that
rank's rows; what is under test is the orchestration of mfft_bench_b200.dist:
the row split, the all-gather of B's row blocks (equal and unequal blocks),
and the plane-by-plane gather of C's rows into the plane-major [RL][n][n]
layout on rank 0.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, L, align, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from mfft_bench_b200 import dist as D
        from oracle.oracle import Oracle
        o = Oracle()
        ranges = D.all_ranges(n, world, align)
        r0, r1 = ranges[rank]
        rows = r1 - r0
        RL = 2 * L + 1
        A = o.signed_planes(n, L, 11)
        B = o.signed_planes(n, L, 12)
        # 1. B all-gather, plane by plane, from this rank's row blocks
        Bv = B.reshape(L, n, n)
        gathered = torch.zeros(L * n * n, dtype=torch.int16)
        for u in range(L):
            loc = torch.from_numpy(Bv[u, r0:r1, :].copy().view(np.int16).ravel())
            D.allgather_rows(loc, gathered.view(L, n * n)[u], n, ranges)
        assert np.array_equal(gathered.numpy().view(np.uint16), B), "B all-gather"
        # 2. this rank's rows of C (oracle stands in for the GPU), gather to rank 0
        ii = np.repeat(np.arange(r0, r1), n)
        jj = np.tile(np.arange(n), rows)
        mine = o.entries(A, B, n, L, True, ii, jj, RL) if rows else np.zeros((RL, 0), np.uint16)
        local = torch.from_numpy(np.ascontiguousarray(mine).view(np.int16).ravel())
        full = torch.zeros(RL * n * n, dtype=torch.int16) if rank == 0 else None
        D.gather_planes_to_root(local, full, n, RL, ranges)
        want = o.mm_signed(A, B, n, L) if rank == 0 else None
        if rank == 0:
            assert np.array_equal(full.numpy().view(np.uint16), want), "C gather"
        # 3. sub-blocks shipped asynchronously while the next one is computed
        subs = D.plan_subblocks(ranges, 2, align=16)
        nsub = len(subs[0])
        assert all(len(x) == nsub for x in subs)
        full2 = torch.zeros(RL * n * n, dtype=torch.int16) if rank == 0 else None
        works, keep = [], []
        for si in range(nsub):
            a, b = subs[rank][si]
            ii = np.repeat(np.arange(a, b), n)
            jj = np.tile(np.arange(n), b - a)
            blk = o.entries(A, B, n, L, True, ii, jj, RL) if b > a else np.zeros((RL, 0), np.uint16)
            t = torch.from_numpy(np.ascontiguousarray(blk).view(np.int16).ravel())
            keep.append(t)
            works += D.gather_sub_to_root_async(t, full2, n, RL, [x[si] for x in subs])
        for wk in works:
            wk.wait()
        if rank == 0:
            assert np.array_equal(full2.numpy().view(np.uint16), want), "async sub-block gather"
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, never hang it
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("n,L,align", [(64, 4, 16), (100, 2, 16), (40, 3, 128)])
def test_sharded_product_orchestration(n, L, align):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, L, align, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), msgs


def test_subblock_plan_covers_every_row():
    sys.path.insert(0, ROOT)
    from mfft_bench_b200 import dist as D
    for n in (100, 1000, 2048, 16384):
        for world in (1, 2, 3, 8):
            rng = D.all_ranges(n, world)
            for nsub in (1, 2, 3):
                subs = D.plan_subblocks(rng, nsub)
                assert len({len(x) for x in subs}) == 1
                for (a, b), x in zip(rng, subs):
                    assert x[0][0] == a and x[-1][1] == b
                    for (p, q), (r, t) in zip(x, x[1:]):
                        assert q == r


def test_row_ranges_cover_and_align():
    sys.path.insert(0, ROOT)
    from mfft_bench_b200 import dist as D
    for n in (1, 100, 128, 1000, 16384):
        for world in (1, 2, 3, 4, 8):
            rs = D.all_ranges(n, world)
            assert rs[0][0] == 0 and rs[-1][1] == n
            for (a, b), (c, d) in zip(rs, rs[1:]):
                assert b == c and a <= b
            for a, b in rs[:-1]:
                assert a % 128 == 0 and (b % 128 == 0 or b == n)
    rs = D.all_ranges(16384, 8)
    assert {b - a for a, b in rs} == {2048}


class _FakeIpcLib:
    """Stand-in for the library's CUDA IPC entry points: fixed device
    addresses, optional failure codes, and a log of the calls of this rank."""

    def __init__(self, fail_alloc=False, fail_open=False):
        self.fail_alloc, self.fail_open, self.calls = fail_alloc, fail_open, []

    def mfftgpu_ipc_alloc(self, nbytes, pptr, handle):
        self.calls.append(("alloc", nbytes))
        if self.fail_alloc:
            return 2
        pptr._obj.value = 0x7000
        handle[0:8] = b"peer-out"
        return 0

    def mfftgpu_ipc_open(self, handle, pptr):
        self.calls.append(("open", bytes(handle[0:8])))
        if self.fail_open:
            return 3
        pptr._obj.value = 0x9000
        return 0

    def mfftgpu_ipc_close(self, ptr):
        self.calls.append(("close", ptr))
        return 0

    def mfftgpu_ipc_free(self, ptr):
        self.calls.append(("free", ptr))
        return 0


def _peer_worker(rank, world, port, case, errq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from mfft_bench_b200 import dist as D
        lib = _FakeIpcLib(fail_alloc=(case == "alloc" and rank == 0),
                          fail_open=(case == "open" and rank == 1))
        if case == "ok":
            peer = D.PeerOutput(100, "uint16", lib=lib)
            assert peer.ptr == (0x7000 if rank == 0 else 0x9000)
            if rank != 0:
                assert peer.tensor is None
            peer.close()
            peer.close()  # a second close is a no-op
            want = ([("alloc", 200), ("free", 0x7000)] if rank == 0 else
                    [("open", b"peer-out"), ("close", 0x9000)])
            assert lib.calls == want, lib.calls
        else:
            try:
                D.PeerOutput(100, "float64", lib=lib)
            except RuntimeError:
                pass
            else:
                raise AssertionError("a failed setup must raise on every rank")
            if case == "alloc":
                want = [("alloc", 800)] if rank == 0 else []
            else:  # the mapping failed on rank 1: the root frees what it allocated
                want = [("alloc", 800), ("free", 0x7000)] if rank == 0 else [("open", b"peer-out")]
            assert lib.calls == want, lib.calls
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent, never hang it
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("case", ["ok", "alloc", "open"])
def test_peer_output_setup_and_failures(case):
    """The shared output of the sharded product: its collective setup and
    teardown, and that a failed allocation on the root or a failed mapping on
    another rank makes every rank raise instead of waiting."""
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, case, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), msgs


def _leaver_worker(rank, world, port, errq, outq):
    try:
        sys.path.insert(0, ROOT)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        import time
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        from mfft_bench_b200 import dist as D
        n = 64
        ranges = D.all_ranges(n, world, 16)
        r0, r1 = ranges[rank]
        full = torch.zeros(n * n, dtype=torch.int16)
        local = torch.ones((r1 - r0) * n, dtype=torch.int16)
        D.allgather_rows(local, full, n, ranges)  # step 1: everybody takes part
        if rank == 1:
            outq.put("rank 1 left")
            os._exit(0)  # leaves between steps, with nothing in flight
        t0 = time.monotonic()
        try:
            D.allgather_rows(local, full, n, ranges)  # step 2: rank 1 is gone
        except Exception as e:  # the collective must end with an error
            outq.put(f"rank 0 error after {time.monotonic() - t0:.1f}s: {type(e).__name__}")
            os._exit(0)
        outq.put("rank 0 completed a collective without its peer")
        os._exit(0)
    except Exception as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_rank_that_leaves_ends_the_next_collective_with_an_error():
    """A rank that leaves between steps: the remaining rank's next exchange
    step (the B all-gather) ends with an error inside the process group's
    short timeout instead of waiting for good."""
    ctx = mp.get_context("spawn")
    errq, outq = ctx.SimpleQueue(), ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, 2, port, errq, outq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not outq.empty():
        msgs.append(outq.get())
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank waited for good"
    assert not errs, errs
    assert "rank 1 left" in msgs
    assert any(m.startswith("rank 0 error after") for m in msgs), msgs
