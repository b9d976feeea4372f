"""Failure detection on the GPU without a GPU fault.

* every mbarrier wait in the tcgen05 kernel is bounded: with a producer that
  never loads, the kernel gives up after the configured timeout, reports
  MFFTGPU_ERR_TIMEOUT and the context stays usable;
* inputs outside the documented range come back as MFFTGPU_ERR_RANGE;
* bad shapes and row ranges are rejected before any launch.
"""
import numpy as np
import pytest

import mfft_bench_b200 as m

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(ctx, oracle):
    assert ctx.selftest_timeout(50_000_000) == 4  # MFFTGPU_ERR_TIMEOUT
    n, L = 32, 4
    A, B = oracle.bigmat_rand(n, L, 1), oracle.bigmat_rand(n, L, 2)
    assert np.array_equal(ctx.mm_u16(A, B, n, L), oracle.mm_mfft(A, B, n, L))


def test_limb_out_of_range_is_reported(ctx):
    n, L = 16, 2
    A32 = np.zeros(L * n * n, np.int32)
    A32[5] = 70000
    with pytest.raises(m.MfftError) as e:
        ctx.conv_i32(A32, A32, n, L)
    assert e.value.status == 5  # MFFTGPU_ERR_RANGE


def test_bad_arguments_rejected(ctx):
    import torch
    A = np.zeros(4 * 16, np.uint16)
    with pytest.raises(m.MfftError) as e:
        ctx.mm_u16(A, A, 4, 4, RL=-1)
    assert e.value.status == 1
    dA = torch.zeros(4 * 16, dtype=torch.int16, device="cuda")
    with pytest.raises(m.MfftError):
        ctx.mm_u16(dA, dA, 4, 4, rows=(3, 9))
