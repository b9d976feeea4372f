"""GPU parity: the B200 path through its C ABI vs the reference's outputs.

Bit-exact equality is required everywhere (integer path: every output limb;
fp32 path: every output float, compared as bits).
"""
import numpy as np
import pytest

import mfft_bench_b200 as m
from conftest import load_fixture

pytestmark = pytest.mark.gpu
SA, SB = 12345, 12345 ^ 0xABCDEF


# ---------------------------------------------------------------- the tcgen05 kernel alone
@pytest.mark.parametrize("rows,cols,kdim,NB,K,dA,dB,nchunk,bn", [
    (256, 256, 256, 2, 1, 1, 1, 1, 256),
    (128, 64, 128, 1, 1, 1, 1, 1, 64),
    (200, 208, 144, 2, 4, 2, 2, 2, 128),
    (64, 64, 64, 4, 8, 1, 1, 1, 64),
    (1000, 1008, 1000, 2, 4, 3, 2, 3, 256),
    (384, 512, 520, 8, 8, 1, 1, 1, 256),
])
def test_pointwise_kernel_vs_cuda_cores(ctx, rows, cols, kdim, NB, K, dA, dB, nchunk, bn):
    assert ctx.selftest_pointwise(rows, cols, kdim, NB, K, dA, dB, nchunk, bn, variant=1) == 0


@pytest.mark.parametrize("rows,cols,kdim,NB,K,dA,dB,nchunk", [
    (256, 256, 256, 2, 1, 1, 1, 1),
    (512, 256, 128, 1, 2, 1, 1, 1),
    (300, 272, 144, 2, 4, 2, 2, 2),
    (1000, 1008, 1000, 2, 4, 3, 2, 3),
    (768, 1024, 520, 8, 8, 1, 1, 1),
    (2048, 2048, 2048, 2, 8, 1, 1, 1),
])
def test_pointwise_pair_kernel_vs_cuda_cores(ctx, rows, cols, kdim, NB, K, dA, dB, nchunk):
    """The CTA-pair (tcgen05 cta_group::2, 256 x 256 tiles) variant."""
    assert ctx.selftest_pointwise(rows, cols, kdim, NB, K, dA, dB, nchunk, 256, variant=2) == 0


@pytest.mark.parametrize("rows,cols,kdim,NB,K,dA,dB", [
    (256, 128, 128, 1, 4, 1, 1),
    (256, 256, 256, 2, 8, 1, 1),
    (300, 272, 144, 2, 4, 1, 1),
    (1000, 1008, 1000, 2, 8, 1, 1),
    (768, 1024, 520, 8, 8, 1, 1),
    (2048, 2048, 2048, 4, 16, 1, 1),
    (512, 384, 256, 2, 8, 2, 2),
    (300, 272, 144, 2, 4, 3, 2),
    (1024, 1024, 512, 2, 16, 2, 2),
])
def test_pointwise_grouped_kernel_vs_cuda_cores(ctx, rows, cols, kdim, NB, K, dA, dB):
    """The t-grouped CTA-pair variant (4 jobs per tile, shared A and F tiles),
    single- and multi-digit plans."""
    assert ctx.selftest_pointwise(rows, cols, kdim, NB, K, dA, dB, 1, 256, variant=3) == 0


@pytest.mark.parametrize("half", [0, 1])
@pytest.mark.parametrize("rows,cols,kdim,NB,K,dA,dB", [
    (256, 256, 256, 8, 8, 1, 1),
    (512, 384, 256, 16, 16, 1, 1),
    (300, 272, 144, 4, 4, 3, 2),
    (512, 256, 384, 32, 16, 2, 2),
])
def test_pointwise_grouped_half_points(ctx, half, rows, cols, kdim, NB, K, dA, dB):
    """Points 0 and NB/2 with operands that vanish above coefficient K/2 (as
    the forward transform leaves them): the t-grouped kernel skipping their
    zero terms (half=1) and computing them (half=0) both match the CUDA-core
    sum over every term."""
    ctx.set_half_points(half)
    try:
        assert ctx.selftest_pointwise(rows, cols, kdim, NB, K, dA, dB, 1, 256, variant=3) == 0
    finally:
        ctx.set_half_points(1)


@pytest.mark.parametrize("n,L,signed", [
    (256, 16, True),    # b4 NB16 K16
    (300, 4, True),     # b4 NB8 K8 (the W=64 plan), ragged n
    (256, 64, False),   # b8 NB32 K16, 3 digit classes
    (512, 8, False),    # b4 NB16 K8
])
def test_half_points_skip_is_exact(ctx, oracle, n, L, signed):
    """Whole products with the half-point terms skipped and computed are the
    same bits, and match the oracle's exact entries."""
    gen = oracle.signed_planes if signed else oracle.bigmat_rand
    A, B = gen(n, L, 71 + n), gen(n, L, 73 + L)
    ctx.set_karatsuba(0)  # the t-grouped kernel's own half-point skip
    ctx.set_half_points(0)
    try:
        dense = ctx.mm_u16(A, B, n, L, signed=signed).reshape(2 * L + 1, n, n)
        pd = ctx.last_plan()
        ctx.set_half_points(1)
        got = ctx.mm_u16(A, B, n, L, signed=signed).reshape(2 * L + 1, n, n)
        ph = ctx.last_plan()
    finally:
        ctx.set_half_points(1)
        ctx.set_karatsuba(3)
    assert ph["pw_kernel"] == 3 and ph["half_points"] == 1 and pd["half_points"] == 0
    NB, K, S = ph["NB"], ph["K"], ph["S"]
    assert ph["int8_macs"] == pytest.approx(pd["int8_macs"] * ((NB - 2) * K * K + 2 * S * S)
                                            / (NB * K * K))
    assert np.array_equal(got, dense)
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 3000)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 3000)]
    assert np.array_equal(got[:, rows, cols], oracle.entries(A, B, n, L, signed, rows, cols))


# ---------------------------------------------------------------- the forward kernels
@pytest.mark.parametrize("n,L,signed", [
    (256, 64, False),   # b8 NB32 K16 d2, int16 digits (the c3 plan shape)
    (130, 32, True),    # b4 NB16 K32, int8 digits
    (64, 128, False),   # b8 NB32 K32 d2
    (40, 17, False),    # b9 NB16 K8 d2
    (96, 41, True),     # b11 NB8 K32 d2
    (256, 12, False),   # b6 NB4 K32
    (20, 49, True),     # b7 NB32 K16 d2, int8 digits
    (300, 16, True),    # b4 NB16 K16: the byte-SIMD kernel
    (24, 25, True),     # b13: sums too wide for int16 lanes, generic kernel either way
    (300, 4, True),     # b4 NB8 K8, Karatsuba level 3: the 18 operand planes per point
])
def test_forward_kernels_vs_generic(ctx, oracle, n, L, signed):
    """The one-point-per-warp and byte-SIMD forward kernels against the
    generic forward kernel (whole products, bit for bit) and the oracle."""
    gen = oracle.signed_planes if signed else oracle.bigmat_rand
    A, B = gen(n, L, 41 + n), gen(n, L, 43 + L)
    got = ctx.mm_u16(A, B, n, L, signed=signed)
    ctx.set_kernel_variant("forward", 1)
    try:
        ref = ctx.mm_u16(A, B, n, L, signed=signed)
    finally:
        ctx.set_kernel_variant("forward", 0)
    assert np.array_equal(got, ref)
    RL = 2 * L + 1
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 1500)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 1500)]
    want = oracle.entries(A, B, n, L, signed, rows, cols)
    assert np.array_equal(got.reshape(RL, n, n)[:, rows, cols], want)


# ---------------------------------------------------------------- the inverse kernels
@pytest.mark.parametrize("kind,n", [("i64", 256), ("i64", 130), ("f32", 96), ("f32w0", 80),
                                    ("f64", 72)])
def test_inverse_lane_kernel_on_small_plans(ctx, oracle, kind, n):
    """The lane inverse (inverse variant 2) on plans with NB*K <= 64, which
    the register kernel serves by default: the W=64 (c5 plan NB8 K8), fp32
    and fp64 products, bit-identical to the register kernel and to the
    oracle."""
    def run():
        if kind == "i64":
            return ctx.mm_i64(A, B, n, RL=9)
        if kind == "f64":
            return ctx.fp64(A, B, n, 512)
        return ctx.fp32(A, B, n, 0 if kind == "f32w0" else 512)
    if kind == "i64":
        A, B = oracle.int64_entries(n, 71), oracle.int64_entries(n, 73)
    elif kind == "f64":
        g = np.random.default_rng(n)
        A = g.standard_normal(n * n) * np.exp2(g.integers(-8, 9, n * n))
        B = g.standard_normal(n * n) * np.exp2(g.integers(-8, 9, n * n))
    else:
        A, B = oracle.normal_f32(n, 79 + n)
    ref = run()
    plan = ctx.last_plan()
    assert plan["NB"] * plan["K"] <= 64
    ctx.set_kernel_variant("inverse", 2)
    try:
        got = run()
    finally:
        ctx.set_kernel_variant("inverse", 0)
    assert np.array_equal(got.view(np.uint8), ref.view(np.uint8))
    if kind == "i64":
        rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 1500)]
        cols = np.tile(np.arange(n), n)[:: max(1, n * n // 1500)]
        want = oracle.entries(oracle.int64_to_planes(A, n), oracle.int64_to_planes(B, n), n, 4,
                              True, rows, cols, 9)
        assert np.array_equal(got.reshape(9, n, n)[:, rows, cols], want)
    elif kind != "f64":
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        want = oracle.fpx_entries(A, B, n, 0 if kind == "f32w0" else 512, rows, cols)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n,L,signed", [
    (256, 16, True),    # b4 NB16 K16
    (128, 64, False),   # b8 NB32 K16, 3 digit classes
    (130, 32, True),    # b4 NB16 K32, padded rows (scalar stores)
    (64, 128, False),   # b8 NB32 K32
    (33, 9, True),      # b5 NB8 K16
    (40, 17, False),    # b9 NB16 K8
    (24, 25, True),     # b13 NB16 K8, 5 digit classes
    (17, 113, False),   # b15 NB32 K16
    (96, 41, True),     # b11 NB8 K32
    (256, 12, False),   # b6 NB4 K32
    (20, 49, True),     # b7 NB32 K16
])
def test_inverse_lane_kernel_vs_generic_and_oracle(ctx, oracle, n, L, signed):
    """The lane-parallel inverse (warp-shuffle DFT, segmented carry) against
    the generic shared-memory kernel and the oracle's exact entries."""
    plan = m.plan_info(n, 0, 16 * L, 16 * L)
    assert plan["NB"] * plan["K"] > 64 and plan["K"] in (8, 16, 32) and plan["NB"] <= 32
    gen = oracle.signed_planes if signed else oracle.bigmat_rand
    A, B = gen(n, L, 31 + n), gen(n, L, 37 + L)
    RL = 2 * L + 1
    got = ctx.mm_u16(A, B, n, L, signed=signed)
    ctx.set_kernel_variant("inverse", 1)
    try:
        ref = ctx.mm_u16(A, B, n, L, signed=signed)
    finally:
        ctx.set_kernel_variant("inverse", 0)
    assert np.array_equal(got, ref)
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 1500)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 1500)]
    want = oracle.entries(A, B, n, L, signed, rows, cols)
    assert np.array_equal(got.reshape(RL, n, n)[:, rows, cols], want)
    # truncated and sign-extended outputs through the lane kernel
    for rl in (1, L, RL + 3):
        out = ctx.mm_u16(A, B, n, L, signed=signed, RL=rl)
        full = oracle.entries(A, B, n, L, signed, rows, cols, max(rl, RL))
        assert np.array_equal(out.reshape(rl, n, n)[:, rows, cols], full[:rl]), rl


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("n,L", [(8, 8), (16, 64), (48, 16)])
def test_unsigned_fixture(ctx, n, L):
    f = load_fixture(f"mm_mfft_u_n{n}_L{L}.npz")
    assert np.array_equal(ctx.mm_u16(f["A"], f["B"], n, L), f["out"])
    # the same product through the reference-named drop-in symbol
    assert np.array_equal(m.mm_mfft(f["A"], f["B"], n, L), f["out"])


def test_c1_digest(ctx, oracle, golden):
    n, L = 64, 512
    A, B = m.bigmat_rand(n, L, SA), m.bigmat_rand(n, L, SB)
    out = ctx.mm_u16(A, B, n, L)
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


@pytest.mark.parametrize("n,L", [(32, 4), (64, 4), (48, 16)])
def test_signed_fixture(ctx, n, L):
    f = load_fixture(f"signed_n{n}_L{L}.npz")
    assert np.array_equal(ctx.mm_u16(f["A"], f["B"], n, L, signed=True), f["out"])
    assert np.array_equal(m.mm_mfft_signed(f["A"], f["B"], n, L), f["out"])
    # conv_mfft: the unnormalised int64 planes, bit for bit
    assert np.array_equal(ctx.conv_i32(f["A32"], f["B32"], n, L), f["cw"])
    assert np.array_equal(m.conv_mfft(f["A32"], f["B32"], n, L), f["cw"])
    if L == 4:
        x = f["A"].reshape(4, n * n).astype(np.uint64)
        y = f["B"].reshape(4, n * n).astype(np.uint64)
        xa = sum(x[u] << np.uint64(16 * u) for u in range(4)).view(np.int64)
        ya = sum(y[u] << np.uint64(16 * u) for u in range(4)).view(np.int64)
        assert np.array_equal(ctx.mm_i64(xa, ya, n, RL=9), f["out"])


@pytest.mark.parametrize("n,fb", [(64, 512), (64, 0), (96, 512)])
def test_fp32_fixture(ctx, n, fb):
    f = load_fixture(f"fp32_n{n}_w{fb}.npz")
    got = ctx.fp32(f["A"], f["B"], n, fb)
    assert np.array_equal(got.view(np.uint32), f["C"].view(np.uint32))
    assert np.array_equal(m.fpx_gemm_f32(f["A"], f["B"], n, fb).view(np.uint32),
                          f["C"].view(np.uint32))
    # the reference's own call sequence through the drop-in symbols
    fx = m.Fpx(f["A"], f["B"], n, fb)
    fx.encode()
    fx.conv()
    out = fx.decode_f32()
    fx.free()
    assert np.array_equal(out.view(np.uint32), f["C"].view(np.uint32))


# ---------------------------------------------------------------- vs the oracle, random shapes
@pytest.mark.parametrize("n,L", [(1, 1), (1, 4), (3, 2), (17, 3), (100, 4), (128, 16), (200, 8),
                                 (33, 64), (256, 2)])
def test_unsigned_random(ctx, oracle, n, L):
    A, B = oracle.bigmat_rand(n, L, 7 + n), oracle.bigmat_rand(n, L, 9 + L)
    got = ctx.mm_u16(A, B, n, L).reshape(2 * L + 1, n, n)
    if oracle.plan(L) is not None and n <= 128:
        assert np.array_equal(got.ravel(), oracle.mm_mfft(A, B, n, L))
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 3000)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 3000)]
    want = oracle.entries(A, B, n, L, False, rows, cols)
    assert np.array_equal(got[:, rows, cols], want)


@pytest.mark.parametrize("n,L", [(5, 1), (40, 4), (96, 16), (130, 5), (64, 32)])
def test_signed_random(ctx, oracle, n, L):
    A, B = oracle.signed_planes(n, L, 3 + n), oracle.signed_planes(n, L, 5 + L)
    got = ctx.mm_u16(A, B, n, L, signed=True).reshape(2 * L + 1, n, n)
    assert np.array_equal(got.ravel(), oracle.mm_signed(A, B, n, L)) if n <= 96 else True
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 3000)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 3000)]
    assert np.array_equal(got[:, rows, cols], oracle.entries(A, B, n, L, True, rows, cols))


def test_extreme_values(ctx, oracle):
    """All-ones (max unsigned), INT64_MIN / INT64_MAX, zeros."""
    n, L = 48, 4
    A = np.full(L * n * n, 0xFFFF, np.uint16)
    B = np.full(L * n * n, 0xFFFF, np.uint16)
    assert np.array_equal(ctx.mm_u16(A, B, n, L), oracle.mm_mfft(A, B, n, L))
    x = np.full(n * n, np.iinfo(np.int64).min, np.int64)
    y = np.full(n * n, np.iinfo(np.int64).max, np.int64)
    x[1::3] = np.iinfo(np.int64).max
    y[::5] = np.iinfo(np.int64).min
    got = ctx.mm_i64(x, y, n, RL=9)
    want = oracle.mm_signed(oracle.int64_to_planes(x, n), oracle.int64_to_planes(y, n), n, 4)
    assert np.array_equal(got, want)
    z = np.zeros(L * n * n, np.uint16)
    assert not ctx.mm_u16(z, A, n, L).any()


@pytest.mark.parametrize("RL", [1, 3, 8, 12])
def test_short_and_long_output(ctx, oracle, RL):
    """RL below 2L+1 truncates mod 2^(16 RL); above it sign-extends."""
    n, L = 32, 4
    A, B = oracle.signed_planes(n, L, 1), oracle.signed_planes(n, L, 2)
    full = oracle.mm_signed(A, B, n, L, RL=12)
    got = ctx.mm_u16(A, B, n, L, signed=True, RL=RL)
    assert np.array_equal(got, full[: RL * n * n])


@pytest.mark.parametrize("n,L", [(8, 2), (24, 8), (16, 32), (70, 3)])
def test_conv_mixed_sign_limbs(ctx, oracle, n, L):
    """conv_mfft semantics on arbitrary-sign limbs in [-65535, 65535]."""
    rng = np.random.default_rng(n * L)
    A32 = rng.integers(-65535, 65536, L * n * n).astype(np.int32)
    B32 = rng.integers(-65535, 65536, L * n * n).astype(np.int32)
    assert np.array_equal(ctx.conv_i32(A32, B32, n, L), oracle.conv_limbplane(A32, B32, n, L))


def test_fp32_random_ranges(ctx, oracle):
    rng = np.random.default_rng(4)
    n = 72
    for fb, spread in ((512, 20), (0, 20), (0, 60), (128, 30), (96, 5)):
        A = (rng.standard_normal(n * n) * np.exp2(rng.integers(-spread, spread, n * n))).astype(np.float32)
        B = (rng.standard_normal(n * n) * np.exp2(rng.integers(-spread, spread, n * n))).astype(np.float32)
        A[::11] = 0.0
        B[3::7] = -0.0
        A[5] = np.inf
        B[9] = np.nan
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        want = oracle.fpx_entries(A, B, n, fb, rows, cols)
        got = ctx.fp32(A, B, n, fb)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), fb


# ---------------------------------------------------------------- device-resident entry points
def test_device_pointer_path_and_row_ranges(ctx, oracle):
    import torch
    n, L = 200, 4
    A, B = oracle.signed_planes(n, L, 21), oracle.signed_planes(n, L, 22)
    full = ctx.mm_u16(A, B, n, L, signed=True).reshape(9, n, n)
    dA = torch.from_numpy(A.view(np.int16)).cuda().view(torch.uint16)
    dB = torch.from_numpy(B.view(np.int16)).cuda().view(torch.uint16)
    for r0, r1 in ((0, n), (0, 64), (64, 130), (130, 200), (199, 200)):
        out = ctx.mm_u16(dA, dB, n, L, signed=True, rows=(r0, r1))
        ctx.sync()
        got = out.view(torch.int16).cpu().numpy().view(np.uint16).reshape(9, r1 - r0, n)
        assert np.array_equal(got, full[:, r0:r1, :]), (r0, r1)


def test_device_generators_match_host(ctx):
    import torch
    n, L = 33, 5
    dm = torch.empty(n * n * L, dtype=torch.uint16, device="cuda")
    ctx.gen_bigmat(dm, n, L, 12345)
    ctx.sync()
    assert np.array_equal(dm.view(torch.int16).cpu().numpy().view(np.uint16),
                          m.bigmat_rand(n, L, 12345))


def test_host_entry_points_chunked_readback(ctx):
    """n >= 4096: the host-pointer calls compute C in row chunks and read each
    chunk back while the next computes; the result equals the one-shot
    device-pointer product."""
    import torch
    n = 4096
    dA = torch.empty(n * n, dtype=torch.int64, device="cuda")
    dB = torch.empty_like(dA)
    ctx.gen_int64(dA, 101)
    ctx.gen_int64(dB, 202)
    want = ctx.mm_i64(dA, dB, n, RL=9)
    ctx.sync()
    got = ctx.mm_i64(dA.cpu().numpy(), dB.cpu().numpy(), n, RL=9)
    assert np.array_equal(got, want.view(torch.int16).cpu().numpy().view(np.uint16))
    L = 3
    uA = torch.empty(L * n * n, dtype=torch.uint16, device="cuda")
    uB = torch.empty_like(uA)
    ctx.gen_bigmat(uA, n, L, 7)
    ctx.gen_bigmat(uB, n, L, 8)
    want = ctx.mm_u16(uA, uB, n, L, signed=True, RL=5)
    ctx.sync()
    h = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    got = ctx.mm_u16(h(uA), h(uB), n, L, signed=True, RL=5)
    assert np.array_equal(got, h(want))


@pytest.mark.parametrize("rows,cols,kdim,NB", [
    (256, 128, 512, 8),
    (300, 272, 1000, 8),   # ragged rows, columns and contraction
    (512, 256, 2048, 4),
    (100, 128, 256, 2),    # fewer rows than one pair tile
    (256, 144, 640, 8),    # 5 k-blocks: level 2's last stage holds one
    (300, 128, 100, 4),    # a single, partial k-block
])
@pytest.mark.parametrize("level", [1, 2, 3])
def test_karatsuba_pointwise_kernel(ctx, rows, cols, kdim, NB, level):
    """The Karatsuba plane-product kernel on random int8 operand planes
    against a CUDA-core evaluation of its job table.  Level 1 (NB * 12 planes
    per side): P0, P1, P2 of every ordinary point, P0 of the half points.
    Level 2 (NB * 16): the length-2 convolutions Q0, Q1, Q2 of P0 and P1 (two
    k-blocks per pipeline stage, an odd k-block count included) and P2.
    Level 3 (NB * 18): those of P2 as well."""
    assert ctx.selftest_pointwise(rows, cols, kdim, NB, 8, 1, 1, 1, 256,
                                  variant=3 + level) == 0


@pytest.mark.parametrize("rows,cols,kdim,NB,K,nchunk,bn", [
    (256, 256, 512, 32, 16, 1, 256),
    (300, 272, 1000, 8, 16, 2, 256),   # ragged, two contraction chunks per class
    (128, 64, 256, 4, 64, 1, 64),      # the c1 shape of plan (K = 64)
])
def test_digit_sum_pointwise_kernel(ctx, rows, cols, kdim, NB, K, nchunk, bn):
    """A digit-sum job table (class w multiplies digit w of A by digit w of B)
    on the kernel the product path picks -- t-grouped (one chunk, 256 rows),
    CTA pairs (two chunks), one CTA per tile (the small c1 shape) -- against a
    CUDA-core evaluation of the table."""
    assert ctx.selftest_pointwise(rows, cols, kdim, NB, K, 3, 3, nchunk, bn, variant=7) == 0


@pytest.mark.parametrize("n,L,signed", [(256, 64, False), (300, 64, True), (64, 512, False),
                                        (130, 128, False)])
def test_digit_sums_are_exact(ctx, oracle, n, L, signed):
    """Two-digit plans with digit sums (the default) and without them give the
    same bits, and match the oracle's exact entries."""
    gen = oracle.signed_planes if signed else oracle.bigmat_rand
    A, B = gen(n, L, 91 + n), gen(n, L, 93 + L)
    got = ctx.mm_u16(A, B, n, L, signed=signed)
    p = ctx.last_plan()
    assert p["dsum"] == 1 and p["dA"] == p["dB"] == 3 and p["nW"] == 3
    ctx.set_digit_sums(0)
    try:
        ref = ctx.mm_u16(A, B, n, L, signed=signed)
        q = ctx.last_plan()
    finally:
        ctx.set_digit_sums(1)
    assert q["dsum"] == 0 and q["dA"] == q["dB"] == 2
    assert p["int8_macs"] * 4 == q["int8_macs"] * 3
    assert np.array_equal(got, ref)
    RL = 2 * L + 1
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 1500)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 1500)]
    want = oracle.entries(A, B, n, L, signed, rows, cols, RL)
    assert np.array_equal(got.reshape(RL, n, n)[:, rows, cols], want)


def test_karatsuba_four_stage_pipeline(monkeypatch):
    """The opt-in four-stage pipeline of the level-3 kernel (one k-block per
    48 KB stage) on the same job-table check."""
    monkeypatch.setenv("MFFTGPU_KARA_STAGES", "4")
    c = m.Context(0)
    try:
        for rows, cols, kdim, NB in ((256, 128, 512, 8), (300, 144, 640, 4)):
            assert c.selftest_pointwise(rows, cols, kdim, NB, 8, 1, 1, 1, 256, variant=6) == 0
    finally:
        c.close()


@pytest.mark.parametrize("n,kind", [(256, "i64"), (300, "i64"), (1000, "i64"), (2112, "i64"),
                                    (512, "u16s"), (384, "u16")])
def test_karatsuba_products_are_exact(ctx, oracle, n, kind):
    """Whole W=64 products with the Karatsuba pointwise at level 3 (the
    default for this plan), 2, 1 (also through the lane inverse) and without
    it are the same bits, and match the oracle."""
    if kind == "i64":
        A, B = oracle.int64_entries(n, 5 + n), oracle.int64_entries(n, 7 + n)
        run = lambda: ctx.mm_i64(A, B, n, RL=9)  # noqa: E731
        Ap, Bp, signed = oracle.int64_to_planes(A, n), oracle.int64_to_planes(B, n), True
    else:
        signed = kind == "u16s"
        gen = oracle.signed_planes if signed else oracle.bigmat_rand
        Ap, Bp = gen(n, 4, 11 + n), gen(n, 4, 13 + n)
        run = lambda: ctx.mm_u16(Ap, Bp, n, 4, signed=signed)  # noqa: E731
    got = run()
    pk = ctx.last_plan()
    assert pk["kara"] == 3 and pk["pw_kernel"] == 4
    assert pk["int8_macs"] == 240 * float(pk["n_int"]) ** 3
    ctx.set_karatsuba(2)
    try:
        two = run()
        assert ctx.last_plan()["kara"] == 2
        assert ctx.last_plan()["int8_macs"] == 264 * float(pk["n_int"]) ** 3
        ctx.set_karatsuba(1)
        one = run()
        assert ctx.last_plan()["kara"] == 1
        assert ctx.last_plan()["int8_macs"] == 320 * float(pk["n_int"]) ** 3
        ctx.set_kernel_variant("inverse", 2)  # the lane inverse on level-1 job planes
        lane = run()
        assert ctx.last_plan()["kara"] == 1
        ctx.set_karatsuba(0)
        ref = run()
        assert ctx.last_plan()["kara"] == 0
    finally:
        ctx.set_kernel_variant("inverse", 0)
        ctx.set_karatsuba(3)
    assert np.array_equal(two, got)
    assert np.array_equal(one, got)
    assert np.array_equal(lane, got)
    assert np.array_equal(got, ref)
    rows = np.repeat(np.arange(n), n)[:: max(1, n * n // 2000)]
    cols = np.tile(np.arange(n), n)[:: max(1, n * n // 2000)]
    want = oracle.entries(Ap, Bp, n, 4, signed, rows, cols, 9)
    assert np.array_equal(got.reshape(9, n, n)[:, rows, cols], want)
