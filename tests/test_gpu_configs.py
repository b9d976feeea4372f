"""Parity at the full sizes of the benchmark configurations c2-c5 (bit-exact).

Full CPU runs of the reference are infeasible beyond n = 1024 (hours), so
full-size parity uses size-independent properties and sampled entries:
* c2: the full n=1024, W=256 output digests equal the digests of the
  reference's own outputs (tests/golden, ~100 s of reference CPU each):
  unsigned through mm_mfft, signed through its signed route
  conv_mfft + normalize_planes; the signed product is also checked on
  sampled entries and by checksum;
* every row and column sum of C equals A*(B*1) and (1^T A)*B modulo the
  prime 2^61-1, computed from all limbs of every entry (oracle checksum);
* sampled entries -- including the first/last rows of every 128-row tile
  group and of every multi-GPU shard boundary -- equal the oracle's exact
  per-entry products;
* c4 (fp32): sampled entries bit-exact vs the oracle's fpfixed path, plus the
  max relative error vs an fp64 GEMM, which must be a half-ulp of fp32.
"""
import numpy as np
import pytest

import mfft_bench_b200 as m

pytestmark = pytest.mark.gpu
SA, SB = 12345, 12345 ^ 0xABCDEF


def _sample(n, count, seed=0):
    rng = np.random.default_rng(seed)
    special = [0, 1, 127, 128, 255, 256, n // 2 - 1, n // 2, n - 2, n - 1]
    for k in (2, 4, 8):
        special += [n * r // k for r in range(k)] + [n * r // k - 1 for r in range(1, k)]
    special = [s for s in special if 0 <= s < n]
    rows = np.concatenate([np.array(special), rng.integers(0, n, count)])
    cols = np.concatenate([np.array(special[::-1]), rng.integers(0, n, count)])
    return rows.astype(np.int32), cols.astype(np.int32)


def test_c2_shape_unsigned_full_digest(ctx, oracle, golden):
    """n=1024, W=256 unsigned: the whole output vs the reference's digest."""
    n, L = 1024, 16
    A, B = m.bigmat_rand(n, L, SA), m.bigmat_rand(n, L, SB)
    out = ctx.mm_u16(A, B, n, L)
    rec = next(c for c in golden["unsigned"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]


def test_c2_signed(ctx, oracle, golden):
    """n=1024, W=256 signed; the whole output vs the digest of the
    reference's conv_mfft + normalize_planes on the same inputs."""
    n, L = 1024, 16
    A, B = oracle.signed_planes(n, L, SA), oracle.signed_planes(n, L, SB)
    out = ctx.mm_u16(A, B, n, L, signed=True)
    RL = 2 * L + 1
    rec = next(c for c in golden["signed"] if c["n"] == n and c["L"] == L)
    assert f"{oracle.digest(out):016x}" == rec["digest"]
    assert oracle.checksum(A, B, n, L, True, out, RL) == 0
    rows, cols = _sample(n, 1500)
    got = out.reshape(RL, n, n)[:, rows, cols]
    assert np.array_equal(got, oracle.entries(A, B, n, L, True, rows, cols))


def test_c3_unsigned_1024bit(ctx, oracle):
    """n=4096, W=1024 unsigned (2-digit split plan)."""
    import torch
    n, L = 4096, 64
    dA = torch.empty(L * n * n, dtype=torch.uint16, device="cuda")
    dB = torch.empty_like(dA)
    ctx.gen_bigmat(dA, n, L, SA)
    ctx.gen_bigmat(dB, n, L, SB)
    out = ctx.mm_u16(dA, dB, n, L)
    ctx.sync()
    RL = 2 * L + 1
    h = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    A, B, C = h(dA), h(dB), h(out)
    del dA, dB, out
    assert np.array_equal(A[:1024], oracle.bigmat_rand(32, 1, SA))  # same stream prefix
    assert oracle.checksum(A, B, n, L, False, C, RL) == 0
    rows, cols = _sample(n, 200)
    got = C.reshape(RL, n, n)[:, rows, cols]
    assert np.array_equal(got, oracle.entries(A, B, n, L, False, rows, cols))


def test_c4_fp32_512bit_grid(ctx, oracle):
    """n=8192 fp32 N(0,1)*2^k, fixed 512-bit grid."""
    import torch
    n = 8192
    A, B = m.gen_normal_f32(n, SA)
    C = ctx.fp32(A, B, n, 512)
    rows, cols = _sample(n, 400)
    want = oracle.fpx_entries(A, B, n, 512, rows, cols)
    assert np.array_equal(C.reshape(n, n)[rows, cols].view(np.uint32), want.view(np.uint32))
    # accuracy vs an fp64 GEMM.  The result is the exact product rounded once,
    # so |C - exact| <= 2^-24 |exact|; the fp64 GEMM itself is off by at most
    # ~n * 2^-53 * (|A||B|), which dominates where entries cancel.
    tA = torch.from_numpy(A).cuda().double().view(n, n)
    tB = torch.from_numpy(B).cuda().double().view(n, n)
    ref = (tA @ tB).cpu().numpy().ravel()
    mag = (tA.abs() @ tB.abs()).cpu().numpy().ravel()
    err = np.abs(C.astype(np.float64) - ref)
    bound = 2.0 ** -24 * np.abs(ref) * (1 + 2.0 ** -20) + n * 2.0 ** -52 * mag
    assert (err <= bound).all()
    rel = err / np.maximum(np.abs(ref), 1e-300)
    print(f"c4 max relative error vs fp64 GEMM: {rel[np.abs(ref) > 0].max():.3e} "
          f"(median {np.median(rel):.3e})")


def test_c5_signed_64bit(ctx, oracle):
    """c5: n=16384, W=64 signed (the headline configuration)."""
    import torch
    n = 16384
    dA = torch.empty(n * n, dtype=torch.int64, device="cuda")
    dB = torch.empty_like(dA)
    ctx.gen_int64(dA, SA)
    ctx.gen_int64(dB, SB)
    out = ctx.mm_i64(dA, dB, n, RL=9)
    ctx.sync()
    A, B = dA.cpu().numpy(), dB.cpu().numpy()
    C = out.view(torch.int16).cpu().numpy().view(np.uint16)
    del dA, dB, out
    # the host-buffer entry point: chunked uploads and read-backs overlapped
    # with the row blocks' compute, the same bits
    assert np.array_equal(ctx.mm_i64(A, B, n, RL=9), C)
    assert np.array_equal(A[:4096], oracle.int64_entries(64, SA))
    assert oracle.checksum(A, B, n, 4, True, C, 9) == 0
    rows, cols = _sample(n, 3000)
    Ap, Bp = oracle.int64_to_planes(A, n), oracle.int64_to_planes(B, n)
    got = C.reshape(9, n, n)[:, rows, cols]
    assert np.array_equal(got, oracle.entries(Ap, Bp, n, 4, True, rows, cols))
