"""The recursive plan (mfft-rec) and ssa_negconv through the drop-in symbols.

The reference's recursive plan (src/mfft.c:665-686) changes how the CPU
solves each point's negacyclic convolution (src/mfft.c:560-662), not the
result: mm_mfft / conv_mfft under a recursive plan must give the same bits as
the reference's own recursive run.  ssa_negconv itself is the exact product
A * B mod (y^K + 1) of two K-plane int32 matrix polynomials.
"""
import numpy as np
import pytest

import mfft_bench_b200 as m

pytestmark = pytest.mark.gpu


def _negacyclic_exact(A, B, K, n):
    """C[w] = sum over u + v = w (mod K) of +-A[u] @ B[v], in Python integers
    reduced modulo 2^64 to int64 (the drop-in's contract where the reference's
    int64 would wrap)."""
    Ao = A.reshape(K, n, n).astype(object)
    Bo = B.reshape(K, n, n).astype(object)
    C = [np.zeros((n, n), dtype=object) for _ in range(K)]
    for u in range(K):
        for v in range(K):
            t, sg = (u + v, 1) if u + v < K else (u + v - K, -1)
            C[t] = C[t] + sg * Ao[u].dot(Bo[v])
    wrap = np.vectorize(lambda x: ((int(x) + (1 << 63)) % (1 << 64)) - (1 << 63), otypes=[object])
    return np.stack([wrap(c) for c in C]).astype(np.int64).ravel()


@pytest.mark.parametrize("K,n,bits", [(4, 16, 20), (8, 12, 24), (16, 8, 26), (2, 33, 30), (1, 5, 31)])
def test_ssa_negconv_exact(K, n, bits):
    rng = np.random.default_rng(K * 100 + n)
    hi = (1 << bits) - 1 if bits < 31 else (1 << 31) - 1
    A = rng.integers(-hi, hi + 1, K * n * n, dtype=np.int64).astype(np.int32)
    B = rng.integers(-hi, hi + 1, K * n * n, dtype=np.int64).astype(np.int32)
    A[:n] = -(1 << 31) if bits == 31 else -hi  # the extreme value, one row
    got = m.ssa_negconv(A, B, K, n, bits)
    assert np.array_equal(got, _negacyclic_exact(A, B, K, n))


def test_ssa_negconv_matches_reference(reflib):
    """Against the reference's own recursive ssa_negconv on inputs whose
    product fits its int64 planning (Mbits = 18, the top-level bound of an
    NB = 4 plan)."""
    for K, n in ((4, 9), (8, 16), (16, 6)):
        rng = np.random.default_rng(K + n)
        A = rng.integers(-(1 << 18), 1 << 18, K * n * n).astype(np.int32)
        B = rng.integers(-(1 << 18), 1 << 18, K * n * n).astype(np.int32)
        assert np.array_equal(m.ssa_negconv(A, B, K, n, 18), reflib.ssa_negconv(A, B, K, n, 18))


@pytest.mark.parametrize("n,L", [(5, 4), (12, 16), (9, 64), (4, 256)])
def test_mm_mfft_recursive_plan_matches_reference(reflib, n, L):
    """mm_mfft under the recursive plan: the drop-in (B200) against the
    reference's recursive CPU run, same inputs, same plan."""
    A, B = reflib.bigmat_rand(n, L, 7 + L), reflib.bigmat_rand(n, L, (7 + L) ^ 0xABCDEF)
    mine, ref = m.mfft_plan_init_rec(L, n), reflib.plan_rec(L, n)
    assert mine.rec == ref.rec == 1 and mine.nprod == ref.nprod
    want = reflib.mm_mfft(A, B, n, L, plan=ref)
    assert np.array_equal(m.mm_mfft(A, B, n, L, plan=mine), want)
    assert np.array_equal(m.mm_mfft(A, B, n, L), want)  # the flat plan, same bits


def test_conv_mfft_recursive_plan_signed_limbs(oracle):
    """conv_mfft under a recursive plan on signed limbs (the fpfixed
    embedding's input form): the exact limb convolution."""
    n, L = 16, 32
    rng = np.random.default_rng(3)
    A = rng.integers(-(1 << 15), 1 << 15, L * n * n).astype(np.int32)
    B = rng.integers(-(1 << 15), 1 << 15, L * n * n).astype(np.int32)
    plan = m.mfft_plan_init_rec(L, n)
    got = m.conv_mfft(A, B, n, L, plan=plan)
    Ao, Bo = A.reshape(L, n, n).astype(np.int64), B.reshape(L, n, n).astype(np.int64)
    want = np.zeros((2 * L - 1, n, n), np.int64)
    for u in range(L):
        for v in range(L):
            want[u + v] += Ao[u] @ Bo[v]
    assert np.array_equal(got, want.ravel())
