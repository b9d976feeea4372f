"""C-ABI and host-logic tests that need no GPU.

* the library loads and exports every symbol include/*.h declares;
* reference-compatible host helpers (mfft_plan_init, bigmat_rand,
  normalize_planes, fpx_decode_f32) behave like the reference;
* the int8 planner's exactness invariants hold over a sweep of shapes;
* the fp32 rounding rule shared with the device matches the oracle,
  including ties, sticky bits, subnormal results and overflow;
* without a GPU every product entry point returns a status, never crashes.
"""
import ctypes as C

import numpy as np
import pytest

import mfft_bench_b200 as m
from mfft_bench_b200 import _lib


def test_exports_every_declared_symbol():
    names = _lib.declared_functions()
    assert len(names) > 40
    missing = [s for s in names if not hasattr(_lib.lib, s)]
    assert not missing, missing


def test_product_library_is_not_the_oracle():
    import os
    assert os.path.basename(m.LIB_PATH) == "libmfftb200.so"
    assert not hasattr(_lib.lib, "orc_conv_mfft")


def test_plan_init_semantics(oracle):
    for L in range(1, 80):
        for sigma in range(0, 9):
            p = m.mfft_plan_init(L, sigma)
            q = oracle.plan(L, sigma)
            assert (p is None) == (q is None), (L, sigma)
            if p is not None:
                assert (p.S, p.NB, p.K, p.g, p.nprod, p.rec) == (q.S, q.NB, q.K, q.g, q.nprod, 0)


def test_plan_init_rec_known_answers():
    """The recursive plans of the benchmark shapes, as the reference's own
    mfft_plan_init_rec (src/mfft.c:665-686) gives them: (L, n) -> S, NB, K,
    products."""
    for (L, n), want in {(512, 64): (16, 64, 32, 15552), (16, 1024): (4, 8, 8, 216),
                         (64, 4096): (8, 16, 16, 1296), (4, 16384): (2, 4, 4, 36),
                         (32, 8192): (4, 16, 8, 432)}.items():
        p = m.mfft_plan_init_rec(L, n)
        assert (p.S, p.NB, p.K, p.nprod, p.rec, p.g) == want + (1, 2 * want[2] // want[1])
    assert m.mfft_plan_init_rec(3, 64) is None and m.mfft_plan_init_rec(2, 64) is None


def test_bigmat_rand_matches_reference_stream(oracle):
    for n, L, seed in ((5, 3, 12345), (16, 64, 12345 ^ 0xABCDEF), (1, 1, 0)):
        assert np.array_equal(m.bigmat_rand(n, L, seed), oracle.bigmat_rand(n, L, seed))


def test_normalize_planes_matches_reference(oracle):
    rng = np.random.default_rng(0)
    n = 9
    for P, RL in ((1, 3), (7, 9), (15, 33), (15, 4)):
        acc = rng.integers(-(1 << 50), 1 << 50, P * n * n, dtype=np.int64)
        assert np.array_equal(m.normalize_planes(acc, P, n, RL),
                              oracle.normalize_planes(acc, P, n, RL))


def test_kernel_names():
    assert _lib.lib.kernel_name(2) == b"packed"
    assert _lib.lib.kernel_name(12) == b"sm100"
    assert _lib.lib.kernel_from_name(b"sm100") == 12
    assert _lib.lib.kernel_from_name(b"nope") == -1


# ---------------------------------------------------------------- planner invariants
def _split_ok(M, d, bounds):
    """Brute-force the digit split of every |x| <= M at the extremes."""
    for x in (M, -M, M - 1, -(M - 1), 0, 64, -64, 63, -65, 8191, -8191):
        if abs(x) > M:
            continue
        v = x
        for i in range(d):
            if i < d - 1:
                lo = ((v + 64) & 127) - 64
                if abs(lo) > bounds[i]:
                    return False
                v = (v - lo) >> 7
            else:
                if abs(v) > bounds[i] or abs(v) > 127:
                    return False
    return True


@pytest.mark.parametrize("n", [1, 16, 64, 200, 1024, 4096, 16384])
@pytest.mark.parametrize("mode,w", [(0, 8), (0, 64), (0, 256), (0, 1024), (0, 8192), (0, 68),
                                    (1, 1), (1, 4), (1, 16), (1, 64), (1, 512)])
def test_plan_exactness_invariants(n, mode, w):
    try:
        pi = m.plan_info(n, mode, w)
    except m.MfftError:
        # only acceptable when no int8 plan can be exact (huge limb mode)
        assert mode == 1 and w >= 512 and n >= 4096
        return
    dmax = 65535 if mode == 1 else (1 << pi["b"]) - 1
    assert pi["acc_bound"] < 2 ** 31
    assert pi["inv_bound_log2"] <= 62
    assert pi["NB"] >= pi["ncA"] + pi["ncB"] and (2 * pi["K"]) % pi["NB"] == 0
    assert pi["K"] == 2 * pi["S"]
    if mode == 0:
        assert pi["LbA"] * pi["b"] >= w
    else:
        assert pi["LbA"] == w and pi["b"] == 16
    MA = pi["ncA"] * dmax
    # recompute the split bounds independently (digit sums: the two digits of
    # the split, whose sum lo + hi must also be an int8)
    nsplit = 2 if pi["dsum"] else pi["dA"]
    T, bounds = MA, []
    for i in range(nsplit - 1):
        bounds.append(min(64, T))
        T = (T + 64) // 128
    bounds.append(T)
    assert T <= 127 and _split_ok(MA, nsplit, bounds)
    if pi["dsum"]:
        # lo in [-64, 63] and |hi| <= 64 keep lo + hi in [-128, 127]; three
        # digit-pair classes (lo*lo, hi*hi, sum*sum) of K terms each
        MB = pi["ncB"] * dmax
        TB = (MB + 64) // 128
        assert pi["dA"] == pi["dB"] == 3 and pi["nW"] == 3 and T <= 64 and TB <= 64
        per = -(-pi["K"] // pi["nchunk"]) * pi["n_int"]
        assert per * (64 + T) * (64 + TB) < 2 ** 31
        assert pi["njobs"] == pi["NB"] * pi["K"] * 3 * pi["nchunk"]
        assert pi["int8_macs"] == pi["NB"] * pi["K"] ** 2 * 3 * float(pi["n_int"]) ** 3
        return
    if pi["kara"]:
        # Karatsuba pointwise: three full length-S convolutions per ordinary
        # point, one per half point.  The operands a0 + a1 take one digit per
        # transform block, so they are bounded like the values (MA), and P2's
        # accumulators sum S terms of length n.  Level 3 (the default where
        # it fits) takes P0, P1 and P2 as three length-S/2 convolutions each:
        # their sums take two digits per block (2 MA <= 127), with at most
        # S/2 terms per accumulator; otherwise the plan stays at level 1.
        NB, S = pi["NB"], pi["S"]
        MB = pi["ncB"] * dmax
        assert pi["K"] == 8 and pi["dA"] == pi["dB"] == 1 and pi["nchunk"] == 1 and NB <= 8
        assert MA <= 127 and MB <= 127 and S * pi["n_int"] * MA * MB < 2 ** 31
        nh = min(NB, 2)
        if 2 * MA <= 127 and 2 * MB <= 127 and 2 * pi["n_int"] * (2 * MA) * (2 * MB) < 2 ** 31:
            assert pi["kara"] == 3 and pi["njobs"] == NB * 27
            q = 3 * (S // 2) ** 2
            assert pi["int8_macs"] == (3 * q * (NB - nh) + q * nh) * float(pi["n_int"]) ** 3
        else:
            assert pi["kara"] == 1 and pi["njobs"] == NB * 21
            assert pi["int8_macs"] == (3 * S * S * (NB - nh) + S * S * nh) * float(pi["n_int"]) ** 3
    else:
        assert pi["njobs"] == pi["NB"] * pi["K"] * pi["nW"] * pi["nchunk"]
        assert pi["int8_macs"] == (pi["NB"] * pi["K"] ** 2 * pi["dA"] * pi["dB"]
                                   * float(pi["n_int"]) ** 3)


@pytest.mark.parametrize("n", [1, 16, 100, 1024, 4096, 16384])
@pytest.mark.parametrize("mode,w", [(2, 8), (2, 64), (2, 68), (2, 256), (2, 1024), (2, 8192),
                                    (3, 64)])
def test_school_plan_invariants(n, mode, w):
    """Schoolbook plans: int8 digit planes, every chunk's int32 accumulator
    bounded by the worst digit product, chunks covering all of A's digits."""
    pi = m.plan_info(n, mode, w)
    assert pi["kind"] == 1 and pi["NB"] == 1 and pi["dA"] == pi["dB"] == pi["nW"] == 1
    b, LbA, LbB, U = pi["b"], pi["LbA"], pi["LbB"], pi["U"]
    bal = pi["balanced"]
    assert bal in (0, 1) and (mode == 3 or not bal)
    assert 2 <= b <= (8 if bal else 7) and LbA * b >= w + bal and LbB * b >= w + bal
    assert pi["positions"] == LbA + LbB - 1
    assert pi["K"] % 4 == 0 and pi["K"] >= pi["positions"]
    assert pi["nchunk"] * U >= LbA > (pi["nchunk"] - 1) * U
    dmax = (1 << (b - 1)) if bal else (1 << b) - 1
    worst = min(U, LbA, LbB) * pi["n_int"] * dmax * dmax
    assert worst == pi["acc_bound"] and worst < 2 ** 31
    assert pi["int8_macs"] == LbA * LbB * float(pi["n_int"]) ** 3
    assert pi["njobs"] == pi["K"] * pi["nchunk"]


def test_balanced_digits_restate_the_value():
    """The balanced digit rule of the int64 pack kernel, restated: byte m of
    x + sum 2^(8i+7), minus 128, over 9 digits gives back x exactly."""
    H = sum(1 << (8 * i + 7) for i in range(9))
    for x in (0, 1, -1, 2**63 - 1, -2**63, 0x7F7F7F7F7F7F7F7F, -0x8080808080808080, 12345678901234):
        z = x + H
        assert 0 <= z < 1 << 72
        d = [((z >> (8 * i)) & 255) - 128 for i in range(9)]
        assert all(-128 <= v <= 127 for v in d)
        assert sum(v << (8 * i) for i, v in enumerate(d)) == x
    pi = m.plan_info(16384, 3, 64)
    assert pi["balanced"] == 1 and pi["b"] == 8 and pi["LbA"] == 9
    assert pi["int8_macs"] == 81 * 16384.0 ** 3


def test_school_plan_fewer_products_at_the_bench_widths():
    """The comparison the reference's GPU planner makes: at W=64 and W=256
    schoolbook needs fewer plane products than flat MFFT."""
    for n, w in ((16384, 64), (1024, 256), (8192, 68)):
        s, f = m.plan_info(n, 2, w), m.plan_info(n, 0, w)
        assert s["int8_macs"] < f["int8_macs"] / 2


def test_bench_plans_are_single_digit():
    """The bench configurations run with one int8 digit per transformed value."""
    for n, w in ((16384, 64), (1024, 256)):
        pi = m.plan_info(n, 0, w)
        assert pi["dA"] == pi["dB"] == 1 and pi["nchunk"] == 1


# ---------------------------------------------------------------- fp32 rounding rule
def _words_from_cw(cw, nw):
    carry, words = 0, [0] * nw
    for k in range(2 * nw):
        v = (int(cw[k]) if k < len(cw) else 0) + carry
        words[k >> 1] |= (v & 0xFFFF) << (16 * (k & 1))
        carry = v >> 16
    return words


def test_decode_rule_matches_oracle(oracle):
    rng = np.random.default_rng(11)
    L = 32
    cases = []
    for _ in range(3000):
        cw = np.zeros(2 * L - 1, np.int64)
        k = rng.integers(1, 6)
        pos = rng.integers(0, 2 * L - 1, k)
        for p in pos:
            cw[p] += int(rng.integers(-(1 << 40), 1 << 40))
        S = int(rng.integers(0, 1100))
        cases.append((cw, S))
    # exact ties and near-ties around the 24-bit rounding point, with and without sticky
    for top in (0x1000001, 0x1000003, 0x1FFFFFF, 0xFFFFFF8, 0x2000001):
        for lowbits in (0, 1, 0x8000, 0x4000):
            cw = np.zeros(2 * L - 1, np.int64)
            cw[3] = top
            cw[2] = lowbits
            for S in (100, 0, 250, 400, 900, 1030):
                cases.append((cw.copy(), S))
                cases.append((-cw, S))
    cases.append((np.zeros(2 * L - 1, np.int64), 512))
    for cw, S in cases:
        want = np.float32(oracle.decode_f32_entry(cw, L, S))
        got = np.float32(m.decode_words_f32(_words_from_cw(cw, 36), 0, S))
        assert want.view(np.uint32) == got.view(np.uint32), (cw.nonzero(), S, want, got)


def test_decode_rule_f64_matches_oracle(oracle):
    """The fp64 rule (53-bit round, binary64 ldexp incl. subnormals and
    overflow) vs the oracle's restatement of fpx_decode_f64."""
    rng = np.random.default_rng(13)
    L = 32
    cases = []
    for _ in range(3000):
        cw = np.zeros(2 * L - 1, np.int64)
        for p in rng.integers(0, 2 * L - 1, rng.integers(1, 6)):
            cw[p] += int(rng.integers(-(1 << 45), 1 << 45))
        cases.append((cw, int(rng.integers(0, 2300))))  # reaches subnormal results
    for top in ((1 << 53) + 1, (1 << 53) + 3, (1 << 54) - 1, (1 << 60) - 8, (1 << 54) + 1):
        for lowbits in (0, 1, 0x8000, 0x4000):
            cw = np.zeros(2 * L - 1, np.int64)
            cw[3] = top
            cw[2] = lowbits
            for S in (100, 0, 1100, 2100, 2150, 20):
                cases.append((cw.copy(), S))
                cases.append((-cw, S))
    big = np.zeros(2 * L - 1, np.int64)
    big[2 * L - 2] = 1 << 40  # ~2^1032 on the grid: overflows binary64 at S = 0
    cases += [(big, 0), (-big, 0), (np.zeros(2 * L - 1, np.int64), 512)]
    for cw, S in cases:
        want = np.float64(oracle.decode_f64_entry(cw, L, S))
        got = np.float64(m.decode_words_f64(_words_from_cw(cw, 36), 0, S))
        assert want.view(np.uint64) == got.view(np.uint64), (cw.nonzero(), S, want, got)


def test_decode_rule_bit_offset_equivalence():
    """Shifting the integer by 2^k and passing bit_off = k is the same number."""
    rng = np.random.default_rng(5)
    for _ in range(500):
        v = int(rng.integers(1, 1 << 62)) * int(rng.integers(1, 1 << 40))
        if rng.integers(0, 2):
            v = -v
        k = int(rng.integers(0, 40))
        S = int(rng.integers(0, 300))
        w1 = [(v << k) >> (32 * i) & 0xFFFFFFFF for i in range(6)]
        w2 = [v >> (32 * i) & 0xFFFFFFFF for i in range(6)]
        a = np.float32(m.decode_words_f32(w1, 0, S))
        b = np.float32(m.decode_words_f32(w2, k, S))
        assert a.view(np.uint32) == b.view(np.uint32)


def test_fpx_host_decode_matches_reference(reflib):
    """Drop-in fpx_encode / fpx_decode_f32 (host side) vs the reference's own."""
    from mfft_bench_b200._lib import FpxCtx, lib
    from oracle.oracle import RefFpx
    rng = np.random.default_rng(2)
    n = 24
    A = (rng.standard_normal(n * n) * np.exp2(rng.integers(-30, 30, n * n))).astype(np.float32)
    B = (rng.standard_normal(n * n)).astype(np.float32)
    for fb in (512, 0):
        ours, ref = FpxCtx(), RefFpx()
        assert lib.fpx_init(C.byref(ours), A.ctypes.data, B.ctypes.data, n, fb) == 0
        assert reflib.lib.fpx_init(C.byref(ref), A, B, n, fb) == 0
        assert (ours.L, ours.SA, ours.SB, ours.spreadA) == (ref.L, ref.SA, ref.SB, ref.spreadA)
        lib.fpx_encode(C.byref(ours), A.ctypes.data, B.ctypes.data)
        reflib.lib.fpx_encode(C.byref(ref), A, B)
        nn = n * n
        a32 = np.ctypeslib.as_array(ours.A32, shape=(ours.L * nn,))
        assert np.array_equal(a32, np.ctypeslib.as_array(ref.A32, shape=(ref.L * nn,)))
        # same random Cw planes into both, decode both
        cw = rng.integers(-(1 << 45), 1 << 45, (2 * ours.L - 1) * nn, dtype=np.int64)
        np.ctypeslib.as_array(ours.Cw, shape=cw.shape)[:] = cw
        np.ctypeslib.as_array(ref.Cw, shape=cw.shape)[:] = cw
        o1 = np.empty(nn, np.float32)
        o2 = np.empty(nn, np.float32)
        lib.fpx_decode_f32(C.byref(ours), o1.ctypes.data)
        reflib.lib.fpx_decode_f32(C.byref(ref), o2)
        assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
        lib.fpx_free(C.byref(ours))
        reflib.lib.fpx_free(C.byref(ref))


def test_fpx64_host_matches_reference(reflib):
    """Drop-in fpx_init_d / fpx_encode_d / fpx_decode_f64 / fpx_decode_ld
    (host side) vs the reference's own."""
    from mfft_bench_b200._lib import FpxCtx, lib
    from oracle.oracle import RefFpx
    rng = np.random.default_rng(3)
    n = 20
    A = rng.standard_normal(n * n) * np.exp2(rng.integers(-40, 40, n * n))
    B = rng.standard_normal(n * n) * np.exp2(rng.integers(-600, -560, n * n))
    A[3] = 0.0
    B[4] = np.inf
    ldp = np.ctypeslib.ndpointer(np.longdouble, flags="C_CONTIGUOUS")
    reflib.lib.fpx_decode_ld.argtypes = [C.POINTER(RefFpx), ldp]
    for fb in (512, 0):
        ours, ref = FpxCtx(), RefFpx()
        assert lib.fpx_init_d(C.byref(ours), A.ctypes.data, B.ctypes.data, n, fb) == 0
        assert reflib.lib.fpx_init_d(C.byref(ref), A, B, n, fb) == 0
        assert (ours.L, ours.SA, ours.SB, ours.sig, ours.spreadB) == \
            (ref.L, ref.SA, ref.SB, ref.sig, ref.spreadB)
        lib.fpx_encode_d(C.byref(ours), A.ctypes.data, B.ctypes.data)
        reflib.lib.fpx_encode_d(C.byref(ref), A, B)
        nn = n * n
        for x, y in ((ours.A32, ref.A32), (ours.B32, ref.B32)):
            assert np.array_equal(np.ctypeslib.as_array(x, shape=(ours.L * nn,)),
                                  np.ctypeslib.as_array(y, shape=(ref.L * nn,)))
        cw = rng.integers(-(1 << 45), 1 << 45, (2 * ours.L - 1) * nn, dtype=np.int64)
        np.ctypeslib.as_array(ours.Cw, shape=cw.shape)[:] = cw
        np.ctypeslib.as_array(ref.Cw, shape=cw.shape)[:] = cw
        o1, o2 = np.empty(nn, np.float64), np.empty(nn, np.float64)
        lib.fpx_decode_f64(C.byref(ours), o1.ctypes.data)
        reflib.lib.fpx_decode_f64(C.byref(ref), o2)
        assert np.array_equal(o1.view(np.uint64), o2.view(np.uint64))
        l1, l2 = np.empty(nn, np.longdouble), np.empty(nn, np.longdouble)
        lib.fpx_decode_ld(C.byref(ours), l1.ctypes.data)
        reflib.lib.fpx_decode_ld(C.byref(ref), l2)
        assert np.array_equal(l1, l2)
        lib.fpx_free(C.byref(ours))
        reflib.lib.fpx_free(C.byref(ref))


# ---------------------------------------------------------------- no GPU: statuses, not crashes
def test_no_device_statuses():
    if m.device_count() > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(m.MfftError) as e:
        m.Context(0)
    assert e.value.status == 6  # MFFTGPU_ERR_NODEVICE
    A = m.bigmat_rand(4, 2, 1)
    with pytest.raises(m.MfftError):
        m.mm_mfft(A, A, 4, 2)
