"""GPU parity of the fp64 fixed-point embedding (fpx_init_d / fpx_encode_d /
conv / fpx_decode_f64, src/fpfixed.c:109-172, 308-322): every output double
compared as bits with the reference's own outputs (tests/golden) and with the
oracle's restatement, through the native ABI, the fused drop-in and the
reference's own call sequence, on both product methods.
"""
import numpy as np
import pytest

import mfft_bench_b200 as m
from conftest import load_fixture

pytestmark = pytest.mark.gpu
CASES = [("fp64_n64_w512", 512), ("fp64_n64_w0", 0), ("fp64_n48_w0_tiny", 0)]


@pytest.mark.parametrize("name,fb", CASES)
@pytest.mark.parametrize("method", ["mfft", "schoolbook"])
def test_fp64_fixture(ctx, name, fb, method):
    f = load_fixture(name + ".npz")
    n = int(round(np.sqrt(f["A"].size)))
    ctx.set_method(method)
    try:
        got = ctx.fp64(f["A"], f["B"], n, fb)
        assert ctx.last_plan()["kind"] == (1 if method == "schoolbook" else 0)
    finally:
        ctx.set_method("mfft")
    assert np.array_equal(got.view(np.uint64), f["C"].view(np.uint64))


@pytest.mark.parametrize("name,fb", CASES)
def test_fp64_dropins(name, fb):
    f = load_fixture(name + ".npz")
    n = int(round(np.sqrt(f["A"].size)))
    want = f["C"].view(np.uint64)
    assert np.array_equal(m.fpx_gemm_f64(f["A"], f["B"], n, fb).view(np.uint64), want)
    assert np.array_equal(m.fpx_gemm_f64_limbplane(f["A"], f["B"], n, fb).view(np.uint64), want)
    fx = m.Fpx64(f["A"], f["B"], n, fb)  # the reference's own sequence, conv on the GPU
    fx.encode()
    fx.conv()
    got = fx.decode_f64()
    fx.free()
    assert np.array_equal(got.view(np.uint64), want)


def test_fp64_random_ranges(ctx, oracle):
    rng = np.random.default_rng(8)
    n = 72
    for fb, lo, hi in ((512, -20, 20), (0, -20, 20), (0, -60, 60), (128, -30, 30),
                       (0, -1000, -980), (0, 900, 1000)):
        A = rng.standard_normal(n * n) * np.exp2(rng.integers(lo, hi, n * n))
        B = rng.standard_normal(n * n) * np.exp2(rng.integers(lo, hi, n * n))
        A[::11] = 0.0
        B[3::7] = -0.0
        A[5] = np.inf
        B[9] = np.nan
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        want = oracle.fpx64_entries(A, B, n, fb, rows, cols)
        got = ctx.fp64(A, B, n, fb)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), (fb, lo, hi)


def test_fp64_large_sampled(ctx, oracle):
    """n = 4096 on the 512-bit grid: sampled entries vs the oracle, and the
    error vs the fp64 GEMM within half an ulp plus the fp64 GEMM's own error."""
    import torch
    n = 4096
    rng = np.random.default_rng(21)
    A = rng.standard_normal(n * n) * np.exp2(rng.integers(-8, 9, n * n))
    B = rng.standard_normal(n * n) * np.exp2(rng.integers(-8, 9, n * n))
    C = ctx.fp64(A, B, n, 512)
    srows = np.concatenate([np.array([0, 1, 127, 128, 2047, 2048, 4095]), rng.integers(0, n, 150)])
    scols = np.concatenate([np.array([4095, 0, 128, 127, 2048, 2047, 1]), rng.integers(0, n, 150)])
    want = oracle.fpx64_entries(A, B, n, 512, srows.astype(np.int32), scols.astype(np.int32))
    assert np.array_equal(C.reshape(n, n)[srows, scols].view(np.uint64), want.view(np.uint64))
    tA = torch.from_numpy(A).cuda().view(n, n)
    tB = torch.from_numpy(B).cuda().view(n, n)
    ref = (tA @ tB).cpu().numpy().ravel()
    mag = (tA.abs() @ tB.abs()).cpu().numpy().ravel()
    err = np.abs(C - ref)
    assert (err <= 2.0 ** -53 * np.abs(ref) * (1 + 2.0 ** -20) + n * 2.0 ** -52 * mag).all()


@pytest.mark.parametrize("dtype,fb,lo,hi", [
    ("f64", 0, -20, 20), ("f64", 0, -45, 45), ("f64", 512, -8, 8), ("f64", 0, -90, 90),
    ("f32", 0, -45, 45), ("f32", 0, -70, 70), ("f32", 512, -8, 8),
])
def test_float_outputs_all_inverse_kernels(ctx, oracle, dtype, fb, lo, hi):
    """fp32 / fp64 outputs through the lane inverse (NB*K >= 64 plans) and the
    generic kernel agree bit for bit with each other and with the oracle."""
    rng = np.random.default_rng(1000 + 7 * abs(lo) + hi)
    n = 72
    A = rng.standard_normal(n * n) * np.exp2(rng.integers(lo, hi, n * n))
    B = rng.standard_normal(n * n) * np.exp2(rng.integers(lo, hi, n * n))
    rows = np.repeat(np.arange(n), n)
    cols = np.tile(np.arange(n), n)
    if dtype == "f32":
        A, B = A.astype(np.float32), B.astype(np.float32)
        run, want = ctx.fp32, oracle.fpx_entries(A, B, n, fb, rows, cols)
        view = np.uint32
    else:
        run, want = ctx.fp64, oracle.fpx64_entries(A, B, n, fb, rows, cols)
        view = np.uint64
    got = run(A, B, n, fb)
    plan = ctx.last_plan()
    ctx.set_kernel_variant("inverse", 1)
    try:
        gen = run(A, B, n, fb)
    finally:
        ctx.set_kernel_variant("inverse", 0)
    assert np.array_equal(got.view(view), gen.view(view)), plan
    assert np.array_equal(got.view(view), want.view(view)), plan
