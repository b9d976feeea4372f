"""The invariant behind the half-point skip of the t-grouped plane-product
kernel, checked on the CPU for the GPU planner's plans of the benchmark
configurations: a block holds coefficients 0..S-1 of Z[y]/(y^K+1) (K = 2S),
and the points j = 0 and j = NB/2 evaluate at y^0 and y^K = -1, so the
transformed blocks there vanish above coefficient S-1 and the products of
that point can be non-zero only on the triangle c1 < S, 0 <= t - c1 < S.

The forward transform is restated here from its definition (the same sum
the forward kernels evaluate: Xhat_j[c] = sum_beta s * X[beta S + c'],
c' = (c - g j beta) mod 2K, s = -1 past K)."""
import numpy as np
import pytest

import mfft_bench_b200 as m


def forward(X, NB, K, S, nc):
    g = 2 * K // NB
    out = np.zeros((NB, K), np.int64)
    for j in range(NB):
        for c in range(K):
            acc = 0
            for beta in range(nc):
                r = (c - g * j * beta) % (2 * K)
                sg = 1
                if r >= K:
                    r, sg = r - K, -1
                if r < S and beta * S + r < len(X):
                    acc += sg * int(X[beta * S + r])
            out[j, c] = acc
    return out


def point_range(half, t, K, S):
    """c1 range of the terms of job (j, t) that can be non-zero (the kernel's
    pw_point_range)."""
    if not half:
        return 0, K - 1
    return max(0, t - (S - 1)), min(t, S - 1)


@pytest.mark.parametrize("n,W", [(1024, 256), (4096, 1024), (16384, 64), (8192, 80),
                                 (256, 64), (512, 128)])
def test_half_point_terms(n, W):
    p = m.plan_info(n, 0, W, W)
    NB, K, S = p["NB"], p["K"], p["S"]
    assert K == 2 * S
    rng = np.random.default_rng(W + n)
    nc = NB // 2
    X = rng.integers(-(1 << 7), 1 << 7, nc * S)
    Y = rng.integers(-(1 << 7), 1 << 7, nc * S)
    Ah, Bh = forward(X, NB, K, S, nc), forward(Y, NB, K, S, nc)
    for j in range(NB):
        half = j == 0 or 2 * j == NB
        if half:
            assert not Ah[j, S:].any() and not Bh[j, S:].any(), j
        for t in range(K):
            lo, hi = point_range(half, t, K, S)
            # negacyclic product of point j, coefficient t, over every c1 ...
            full = sum((1 if c1 <= t else -1) * int(Ah[j, c1]) * int(Bh[j, (t - c1) % K])
                       for c1 in range(K))
            # ... equals the sum over the kernel's range (at a half point it has
            # no wrapped term: c1 <= t throughout)
            part = sum((1 if c1 <= t else -1) * int(Ah[j, c1]) * int(Bh[j, (t - c1) % K])
                       for c1 in range(lo, hi + 1))
            if half:
                assert hi <= t
            assert full == part, (j, t)
            if half and t == K - 1:
                assert lo > hi and full == 0
