"""The allocation-free entry point (mfftgpu_mm_i64_noalloc).

It exists for callers that may not allocate device memory themselves (a
framework that owns every device byte through its own pool, or a
latency-critical path that cannot take cudaMalloc's implicit device
synchronisation): they pass their own inputs and output, and the library
runs the whole product in a fixed static scratch array instead of its
workspace.  This file is collected last on purpose, so that a run that stops
at the first failure has already run every other test.

The checks: its output equals the allocating entry point's output bit for
bit, on two calls in a row with different inputs (the shared array keeps
the previous call's contents, so stale state would show), and sizes beyond
the array are refused with MFFTGPU_ERR_ARG.
"""
import ctypes as C

import pytest

import mfft_bench_b200 as m
from mfft_bench_b200._lib import lib

pytestmark = pytest.mark.gpu


def _noalloc(A, B, n, out, RL, stream):
    return lib.mfftgpu_mm_i64_noalloc(C.c_void_p(A.data_ptr()), C.c_void_p(B.data_ptr()), n,
                                      C.c_void_p(out.data_ptr()), RL, C.c_void_p(stream))


@pytest.mark.parametrize("sizes", [(256, 96), (100, 256)])
def test_noalloc_matches_allocating_path_twice(sizes):
    import torch
    ctx = m.Context(0)
    stream = torch.cuda.current_stream()
    ctx.set_stream(stream)
    try:
        for call, n in enumerate(sizes):
            A = torch.empty(n * n, dtype=torch.int64, device="cuda")
            B = torch.empty(n * n, dtype=torch.int64, device="cuda")
            ctx.gen_int64(A, 1000 + 7 * call + n)
            ctx.gen_int64(B, 2000 + 11 * call + n)
            want = ctx.mm_i64(A, B, n, RL=9)
            ctx.sync()
            got = torch.full((9 * n * n,), 0x5A5A, dtype=torch.int16, device="cuda")
            rc = _noalloc(A, B, n, got, 9, stream.cuda_stream)
            assert rc == 0, m.api.lib.mfftgpu_status_string(rc)
            assert torch.equal(got, want.view(torch.int16)), f"call {call} (n={n}) differs"
    finally:
        ctx.close()


def test_noalloc_rejects_sizes_beyond_the_scratch():
    import torch
    n = 272
    A = torch.zeros(n * n, dtype=torch.int64, device="cuda")
    out = torch.zeros(9 * n * n, dtype=torch.int16, device="cuda")
    assert _noalloc(A, A, n, out, 9, torch.cuda.current_stream().cuda_stream) == 1
