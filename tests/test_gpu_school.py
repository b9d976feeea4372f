"""GPU parity of the limb-plane schoolbook method (the reference's
mm_limbplane / conv_limbplane and limb-*-exact comparator rows) on the same
tcgen05 kernel: its job table against a CUDA-core evaluation, its products
against the oracle and the reference's fixtures, and bit-identity with the
MFFT path at the full sizes of the benchmark configurations c3-c5.
"""
import numpy as np
import pytest

import mfft_bench_b200 as m
from conftest import load_fixture

pytestmark = pytest.mark.gpu
SA, SB = 12345, 12345 ^ 0xABCDEF


@pytest.fixture
def school(ctx):
    ctx.set_method("schoolbook")
    yield ctx
    ctx.set_method("mfft")


# ---------------------------------------------------------------- the job table alone
@pytest.mark.parametrize("rows,cols,kdim,LbA,LbB,U", [
    (256, 128, 128, 10, 10, 8),     # the c5 shape of the job table (2 chunks)
    (300, 272, 144, 7, 5, 3),       # ragged tiles, 3 chunks
    (64, 64, 64, 3, 9, 2),          # smaller than one pair tile in both dimensions
    (16, 16, 16, 1, 1, 1),          # a single plane product
    (130, 48, 40, 4, 6, 2),
    (1000, 1008, 1000, 10, 10, 4),
    (512, 512, 512, 37, 37, 37),    # the c2 shape (one chunk, 73 positions)
])
def test_school_job_table_vs_cuda_cores(ctx, rows, cols, kdim, LbA, LbB, U):
    assert ctx.selftest_school(rows, cols, kdim, LbA, LbB, U) == 0


# ---------------------------------------------------------------- products vs the oracle
@pytest.mark.parametrize("n,L,signed", [
    (1, 1, False), (3, 2, True), (17, 3, False), (64, 4, True), (100, 4, False),
    (128, 16, True), (256, 16, False), (48, 64, False), (300, 8, True), (33, 40, True),
])
def test_school_products_vs_oracle(school, oracle, n, L, signed):
    gen = oracle.signed_planes if signed else oracle.bigmat_rand
    A, B = gen(n, L, 5 + n), gen(n, L, 9 + L)
    RL = 2 * L + 1
    got = school.mm_u16(A, B, n, L, signed=signed)
    pi = school.last_plan()
    assert pi["kind"] == 1 and pi["pw_kernel"] == 3
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 2000)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 2000)]
    want = oracle.entries(A, B, n, L, signed, rows, cols)
    assert np.array_equal(got.reshape(RL, n, n)[:, rows, cols], want)
    for rl in (1, L, RL + 2):  # truncated and sign-extended outputs
        out = school.mm_u16(A, B, n, L, signed=signed, RL=rl)
        full = oracle.entries(A, B, n, L, signed, rows, cols, max(rl, RL))
        assert np.array_equal(out.reshape(rl, n, n)[:, rows, cols], full[:rl]), rl


def test_school_int64_extremes(school, oracle):
    n = 200
    x = np.full(n * n, np.iinfo(np.int64).min, np.int64)
    y = np.full(n * n, np.iinfo(np.int64).max, np.int64)
    x[1::3] = np.iinfo(np.int64).max
    y[::5] = np.iinfo(np.int64).min
    x[7::11] = 0
    got = school.mm_i64(x, y, n, RL=9)
    want = oracle.mm_signed(oracle.int64_to_planes(x, n), oracle.int64_to_planes(y, n), n, 4)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n,L", [(8, 8), (16, 64), (48, 16)])
def test_school_unsigned_fixture_and_dropin(school, n, L):
    f = load_fixture(f"mm_mfft_u_n{n}_L{L}.npz")
    assert np.array_equal(school.mm_u16(f["A"], f["B"], n, L), f["out"])
    assert np.array_equal(m.mm_limbplane(f["A"], f["B"], n, L), f["out"])


@pytest.mark.parametrize("n,L", [(32, 4), (64, 4), (48, 16)])
def test_school_signed_fixture_and_conv_dropin(n, L):
    f = load_fixture(f"signed_n{n}_L{L}.npz")
    assert np.array_equal(m.mm_limbplane_signed(f["A"], f["B"], n, L), f["out"])
    assert np.array_equal(m.conv_limbplane(f["A32"], f["B32"], n, L), f["cw"])


@pytest.mark.parametrize("n,fb", [(64, 512), (64, 0), (96, 512)])
def test_school_fp32_fixture(school, n, fb):
    f = load_fixture(f"fp32_n{n}_w{fb}.npz")
    got = school.fp32(f["A"], f["B"], n, fb)
    assert np.array_equal(got.view(np.uint32), f["C"].view(np.uint32))
    assert np.array_equal(m.fpx_gemm_f32_limbplane(f["A"], f["B"], n, fb).view(np.uint32),
                          f["C"].view(np.uint32))


def test_school_c1_digest(school, oracle, golden):
    """n=64, W=8192 (1171 digits per entry, 2341 output positions)."""
    n, L = 64, 512
    out = school.mm_u16(m.bigmat_rand(n, L, SA), m.bigmat_rand(n, L, SB), n, L)
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


def test_school_c2_shape_digest(school, oracle, golden):
    n, L = 1024, 16
    out = school.mm_u16(m.bigmat_rand(n, L, SA), m.bigmat_rand(n, L, SB), n, L)
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


# ---------------------------------------------------------------- full sizes: school == MFFT
def _both(ctx, fn):
    import torch
    ctx.set_method("mfft")
    a = fn()
    ctx.sync()
    ctx.set_method("schoolbook")
    try:
        b = fn()
        ctx.sync()
        assert ctx.last_plan()["kind"] == 1
    finally:
        ctx.set_method("mfft")
    return bool(torch.equal(a.view(torch.int16), b.view(torch.int16))) if hasattr(a, "view") \
        else np.array_equal(a, b)


def test_school_equals_mfft_c5(ctx):
    import torch
    n = 16384
    dA = torch.empty(n * n, dtype=torch.int64, device="cuda")
    dB = torch.empty_like(dA)
    ctx.gen_int64(dA, SA)
    ctx.gen_int64(dB, SB)
    assert _both(ctx, lambda: ctx.mm_i64(dA, dB, n, RL=9))


def test_school_equals_mfft_c3(ctx):
    import torch
    n, L = 4096, 64
    dA = torch.empty(L * n * n, dtype=torch.uint16, device="cuda")
    dB = torch.empty_like(dA)
    ctx.gen_bigmat(dA, n, L, SA)
    ctx.gen_bigmat(dB, n, L, SB)
    assert _both(ctx, lambda: ctx.mm_u16(dA, dB, n, L))


def test_school_equals_mfft_c4(ctx):
    n = 8192
    A, B = m.gen_normal_f32(n, SA)
    ctx.set_method("mfft")
    a = ctx.fp32(A, B, n, 512)
    ctx.set_method("schoolbook")
    try:
        b = ctx.fp32(A, B, n, 512)
        assert ctx.last_plan()["kind"] == 1
    finally:
        ctx.set_method("mfft")
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
