"""Pin the CPU oracle (oracle/mfft_oracle.c) before trusting it as the checker.

Golden fixtures in tests/golden/ were produced by running the reference's own
C (compiled from source into oracle/_ref) -- see tests/golden/make_golden.py.
When oracle/_ref is present the oracle is also compared with it directly on
fresh random inputs.
"""
import numpy as np
import pytest

from conftest import load_fixture

SA, SB = 12345, 12345 ^ 0xABCDEF


@pytest.mark.parametrize("n,L", [(8, 8), (16, 64), (48, 16)])
def test_unsigned_fixture(oracle, golden, n, L):
    f = load_fixture(f"mm_mfft_u_n{n}_L{L}.npz")
    A = oracle.bigmat_rand(n, L, SA)
    B = oracle.bigmat_rand(n, L, SB)
    assert np.array_equal(A, f["A"]) and np.array_equal(B, f["B"])
    out = oracle.mm_mfft(A, B, n, L)
    assert np.array_equal(out, f["out"])
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


def test_c1_digest(oracle, golden):
    """Benchmark configuration c1 (n=64, W=8192): the oracle's restated MFFT reproduces
    the digest of the reference's own mm_mfft output."""
    n, L = 64, 512
    out = oracle.mm_mfft(oracle.bigmat_rand(n, L, SA), oracle.bigmat_rand(n, L, SB), n, L)
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


@pytest.mark.parametrize("n,L", [(32, 4), (64, 4), (48, 16)])
def test_signed_fixture(oracle, n, L):
    f = load_fixture(f"signed_n{n}_L{L}.npz")
    A32 = oracle.signlimb(f["A"], n, L)
    B32 = oracle.signlimb(f["B"], n, L)
    assert np.array_equal(A32, f["A32"]) and np.array_equal(B32, f["B32"])
    cw = oracle.conv_mfft(A32, B32, n, L)
    assert np.array_equal(cw, f["cw"])
    assert np.array_equal(oracle.conv_limbplane(A32, B32, n, L), f["cw"])
    assert np.array_equal(oracle.mm_signed(f["A"], f["B"], n, L), f["out"])


def test_signed_generators(oracle):
    x = oracle.int64_entries(32, SA)
    f = load_fixture("signed_n32_L4.npz")
    assert np.array_equal(oracle.int64_to_planes(x, 32), f["A"])
    g = load_fixture("signed_n48_L16.npz")
    assert np.array_equal(oracle.signed_planes(48, 16, SA), g["A"])


@pytest.mark.parametrize("n,L,signed", [(32, 4, True), (48, 16, True), (48, 16, False)])
def test_entry_product_matches_full(oracle, n, L, signed):
    if signed:
        f = load_fixture(f"signed_n{n}_L{L}.npz")
    else:
        f = load_fixture(f"mm_mfft_u_n{n}_L{L}.npz")
    rng = np.random.default_rng(1)
    rows = rng.integers(0, n, 40)
    cols = rng.integers(0, n, 40)
    ent = oracle.entries(f["A"], f["B"], n, L, signed, rows, cols)
    full = f["out"].reshape(2 * L + 1, n, n)
    assert np.array_equal(ent, full[:, rows, cols])


@pytest.mark.parametrize("n,fb", [(64, 512), (64, 0), (96, 512)])
def test_fp32_fixture(oracle, n, fb):
    f = load_fixture(f"fp32_n{n}_w{fb}.npz")
    A, B = oracle.normal_f32(n, SA)
    assert np.array_equal(A, f["A"]) and np.array_equal(B, f["B"])
    rows = np.repeat(np.arange(n), n)
    cols = np.tile(np.arange(n), n)
    C = oracle.fpx_entries(A, B, n, fb, rows, cols)
    assert np.array_equal(C.view(np.uint32), f["C"].view(np.uint32))


@pytest.mark.parametrize("name", ["fp64_n64_w512", "fp64_n64_w0", "fp64_n48_w0_tiny"])
def test_fp64_fixture(oracle, name):
    """The oracle's fp64 restatement equals the reference's fpx_*_d path on
    every entry (the _tiny case has ~2000 subnormal results)."""
    f = load_fixture(name + ".npz")
    n = int(round(np.sqrt(f["A"].size)))
    fb = 512 if "w512" in name else 0
    rows = np.repeat(np.arange(n), n)
    cols = np.tile(np.arange(n), n)
    C = oracle.fpx64_entries(f["A"], f["B"], n, fb, rows, cols)
    assert np.array_equal(C.view(np.uint64), f["C"].view(np.uint64))


def test_checksum_detects_single_limb_error(oracle):
    f = load_fixture("signed_n48_L16.npz")
    out = f["out"].copy()
    assert oracle.checksum(f["A"], f["B"], 48, 16, True, out, 33) == 0
    out[30 * 48 * 48 + 7] ^= 0x100  # a high limb of one entry
    assert oracle.checksum(f["A"], f["B"], 48, 16, True, out, 33) == 2


# ---------------------------------------------------------------- vs the reference itself
def test_oracle_vs_reference_mixed_sign_limbs(oracle, reflib):
    """conv_mfft on arbitrary-sign int32 limbs (not just sign*magnitude)."""
    rng = np.random.default_rng(7)
    for n, L in ((8, 2), (24, 8), (16, 32)):
        A32 = rng.integers(-65535, 65536, L * n * n).astype(np.int32)
        B32 = rng.integers(-65535, 65536, L * n * n).astype(np.int32)
        assert np.array_equal(oracle.conv_mfft(A32, B32, n, L), reflib.conv_mfft(A32, B32, n, L))


def test_oracle_vs_reference_fp32_random(oracle, reflib):
    rng = np.random.default_rng(3)
    n = 40
    for fb in (512, 0, 128):
        A = (rng.standard_normal(n * n) * np.exp2(rng.integers(-20, 20, n * n))).astype(np.float32)
        B = (rng.standard_normal(n * n) * np.exp2(rng.integers(-20, 20, n * n))).astype(np.float32)
        A[::17] = 0.0
        B[5::13] = -0.0
        ref, _ = reflib.fp32_gemm(A, B, n, fb)
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        got = oracle.fpx_entries(A, B, n, fb, rows, cols)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), fb


def test_plan_init_matches_reference(oracle, reflib):
    for L in range(1, 70):
        for sigma in range(0, 8):
            a, b = oracle.plan(L, sigma), reflib.plan(L, sigma)
            assert (a is None) == (b is None)
            if a is not None:
                assert (a.S, a.NB, a.K, a.g, a.nprod) == (b.S, b.NB, b.K, b.g, b.nprod)


def test_plan_init_rec_matches_reference(reflib):
    """The drop-in recursive planner against the reference's (its Karatsuba /
    block-split cost model and int64 refusals), over powers of two and
    non-powers, matrix sizes from 1 to 2^20 and every sigma override."""
    import mfft_bench_b200 as m
    for L in (1, 2, 3, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096):
        for n in (1, 2, 3, 64, 100, 1024, 4096, 16384, 65536, 1 << 20):
            for sigma in range(0, 13):
                a, b = m.mfft_plan_init_rec(L, n, sigma), reflib.plan_rec(L, n, sigma)
                assert (a is None) == (b is None), (L, n, sigma)
                if a is not None:
                    assert (a.S, a.NB, a.K, a.g, a.nprod, a.rec) == \
                        (b.S, b.NB, b.K, b.g, b.nprod, b.rec), (L, n, sigma)


def test_oracle_vs_reference_unsigned_random(oracle, reflib):
    """mm_mfft of the restatement against the reference's mm_mfft and
    mm_limbplane on the reference's own generator, including outputs shorter
    and longer than 2L+1 limbs.  (The reference plans L = 2, 4, ..., 64.)"""
    for n, L, seed in ((5, 2, 1), (12, 4, 2), (20, 8, 3), (9, 32, 4), (3, 64, 5)):
        A, B = reflib.bigmat_rand(n, L, seed), reflib.bigmat_rand(n, L, seed ^ 0xABCDEF)
        for RL in (2 * L + 1, L, 2 * L + 4):
            want = reflib.mm_mfft(A, B, n, L, RL)
            assert np.array_equal(oracle.mm_mfft(A, B, n, L, RL), want), (n, L, RL)
            assert np.array_equal(reflib.mm_limbplane(A, B, n, L, RL), want), (n, L, RL)


def test_sampled_entries_vs_reference(oracle, reflib):
    """The per-entry checker the full-size GPU tests rely on, against the
    reference itself: signed entries through conv_mfft + normalize_planes
    (sign * limb planes, as the reference's signed route does), unsigned
    through mm_mfft."""
    rng = np.random.default_rng(11)
    for n, L in ((16, 4), (24, 16), (10, 32)):  # L the reference plans (powers of two)
        A, B = oracle.signed_planes(n, L, 21 + n), oracle.signed_planes(n, L, 22 + L)
        RL = 2 * L + 1
        cw = reflib.conv_mfft(oracle.signlimb(A, n, L), oracle.signlimb(B, n, L), n, L)
        want = reflib.normalize_planes(cw, 2 * L - 1, n, RL).reshape(RL, n * n)
        rows = rng.integers(0, n, 200)
        cols = rng.integers(0, n, 200)
        got = oracle.entries(A, B, n, L, True, rows, cols)
        assert np.array_equal(got, want[:, rows * n + cols]), (n, L)
        A, B = reflib.bigmat_rand(n, L, 5), reflib.bigmat_rand(n, L, 6)
        want = reflib.mm_mfft(A, B, n, L).reshape(RL, n * n)
        got = oracle.entries(A, B, n, L, False, rows, cols)
        assert np.array_equal(got, want[:, rows * n + cols]), (n, L)


def test_oracle_vs_reference_fp64_random(oracle, reflib):
    """The fp64 embedding's per-entry restatement against the reference's
    fpx_*_d path on random magnitudes, zeros and signed zeros, several grids."""
    rng = np.random.default_rng(5)
    n = 32
    for fb in (512, 0, 256):
        A = rng.standard_normal(n * n) * np.exp2(rng.integers(-30, 30, n * n))
        B = rng.standard_normal(n * n) * np.exp2(rng.integers(-30, 30, n * n))
        A[::19] = 0.0
        B[3::11] = -0.0
        ref, _ = reflib.fp64_gemm(A, B, n, fb)
        rows = np.repeat(np.arange(n), n)
        cols = np.tile(np.arange(n), n)
        got = oracle.fpx64_entries(A, B, n, fb, rows, cols)
        assert np.array_equal(got.view(np.uint64), ref.view(np.uint64)), fb
