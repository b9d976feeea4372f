"""The Karatsuba pointwise step, on the CPU: the algebra the kernels rely on
and the planner's choice of it.

At an evaluation point the MFFT multiplies two ring elements of
Z[y]/(y^8 + 1) (src/mfft.c:383-396: 64 plane products per point).  With
a = a0 + y^4 a1 and b = b0 + y^4 b1 (a0, a1, b0, b1 of degree < 4), and
y^8 = -1:

    a b = P0 - P1 + y^4 (P2 - P0 - P1)      P0 = a0 b0, P1 = a1 b1,
                                            P2 = (a0 + a1)(b0 + b1)

so three full convolutions of length 4 (48 plane products) give the same
coefficients; at the points 0 and NB/2 the blocks have a1 = b1 = 0 and P0 is
the whole product.  The inverse kernel recombines the 21 job planes of a
point with exactly the formulas restated here.
"""
import random

import pytest

import mfft_bench_b200 as m


def _negacyclic(a, b, K=8):
    c = [0] * K
    for i in range(K):
        for j in range(K):
            if i + j < K:
                c[i + j] += a[i] * b[j]
            else:
                c[i + j - K] -= a[i] * b[j]
    return c


def _conv4(a, b):
    c = [0] * 7
    for i in range(4):
        for j in range(4):
            c[i + j] += a[i] * b[j]
    return c


def _recombine(P0, P1, P2):
    """Chat from the job planes, as the register inverse kernel forms it."""
    M = [P2[s] - P0[s] - P1[s] for s in range(7)]
    y = [0] * 8
    for t in range(3):
        y[t] = P0[t] - P1[t] - M[t + 4]
    y[3] = P0[3] - P1[3]
    for t in range(4, 7):
        y[t] = P0[t] - P1[t] + M[t - 4]
    y[7] = M[3]
    return y


@pytest.mark.parametrize("half", [False, True])
def test_karatsuba_identity(half):
    rng = random.Random(7 + half)
    for _ in range(2000):
        a = [rng.randint(-60, 60) for _ in range(8)]
        b = [rng.randint(-60, 60) for _ in range(8)]
        if half:
            a[4:] = b[4:] = [0] * 4
        sa = [a[i] + a[i + 4] for i in range(4)]
        sb = [b[i] + b[i + 4] for i in range(4)]
        assert max(map(abs, sa + sb)) <= 120  # the int8 operands of P2
        P0, P1, P2 = _conv4(a[:4], b[:4]), _conv4(a[4:], b[4:]), _conv4(sa, sb)
        want = _negacyclic(a, b)
        assert _recombine(P0, P1, P2) == want
        if half:
            assert P0 + [0] == want  # the half points read P0 alone


def _expand2(Q0, Q1, Q2):
    """A length-4 convolution from its three length-2 ones, as the register
    inverse kernel forms it: P = Q0 + y^2 (Q2 - Q0 - Q1) + y^4 Q1."""
    M = [Q2[s] - Q0[s] - Q1[s] for s in range(3)]
    return [Q0[0], Q0[1], Q0[2] + M[0], M[1], Q1[0] + M[2], Q1[1], Q1[2]]


def _conv2(a, b):
    return [a[0] * b[0], a[0] * b[1] + a[1] * b[0], a[1] * b[1]]


@pytest.mark.parametrize("half", [False, True])
def test_two_level_karatsuba_identity(half):
    """Level 2: P0 and P1 from three length-2 convolutions each (their
    operands are single transformed digits, |x| <= 60, so the sums fit int8);
    P2's operands are sums already and stay one level deep."""
    rng = random.Random(11 + half)
    for _ in range(2000):
        a = [rng.randint(-60, 60) for _ in range(8)]
        b = [rng.randint(-60, 60) for _ in range(8)]
        if half:
            a[4:] = b[4:] = [0] * 4
        P = []
        for lo in (0, 4):
            u0, u1 = a[lo:lo + 2], a[lo + 2:lo + 4]
            v0, v1 = b[lo:lo + 2], b[lo + 2:lo + 4]
            su = [u0[i] + u1[i] for i in range(2)]
            sv = [v0[i] + v1[i] for i in range(2)]
            assert max(map(abs, su + sv)) <= 120  # the int8 operands of Q2
            P.append(_expand2(_conv2(u0, v0), _conv2(u1, v1), _conv2(su, sv)))
            assert P[-1] == _conv4(a[lo:lo + 4], b[lo:lo + 4])
        sa = [a[i] + a[i + 4] for i in range(4)]
        sb = [b[i] + b[i + 4] for i in range(4)]
        assert _recombine(P[0], P[1], _conv4(sa, sb)) == _negacyclic(a, b)


def test_three_way_split_identity():
    """Level 3: P2 as three length-2 convolutions too (its operands a0 + a1
    are single-term sums per block, so (a0+a1)[c] + (a0+a1)[c+2] fits int8
    like x[c] + x[c+2])."""
    rng = random.Random(13)
    for _ in range(2000):
        a = [rng.randint(-60, 60) for _ in range(8)]
        b = [rng.randint(-60, 60) for _ in range(8)]
        sa = [a[i] + a[i + 4] for i in range(4)]
        sb = [b[i] + b[i + 4] for i in range(4)]
        P = []
        for u, v in ((a[:4], b[:4]), (a[4:], b[4:]), (sa, sb)):
            su, sv = [u[0] + u[2], u[1] + u[3]], [v[0] + v[2], v[1] + v[3]]
            P.append(_expand2(_conv2(u[:2], v[:2]), _conv2(u[2:], v[2:]), _conv2(su, sv)))
            assert P[-1] == _conv4(u, v)
        assert _recombine(*P) == _negacyclic(a, b)


def _point_terms(K, S, NB, nc, j):
    """Digit terms of the transformed coefficients x[0..K-1] at point j:
    block beta (beta < nc) holds digits at ring positions 0..S-1 and is
    multiplied by y^(g j beta), a signed permutation of Z[y]/(y^K + 1)."""
    g = 2 * K // NB
    xs = []
    for k in range(K):
        t = {}
        for beta in range(nc):
            r, sgn = (k - g * j * beta) % (2 * K), 1
            if r >= K:
                r, sgn = r - K, -1
            if r < S:
                t[(beta, r)] = t.get((beta, r), 0) + sgn
        xs.append(t)
    return xs


def _nterms(*ts):
    out = {}
    for t in ts:
        for key, v in t.items():
            out[key] = out.get(key, 0) + v
    return sum(abs(v) for v in out.values())


@pytest.mark.parametrize("NB", [2, 4, 8])
def test_karatsuba_operand_bounds(NB):
    """The bounds every Karatsuba level relies on, counted from the transform
    itself at every evaluation point: x[c] and (a0+a1)[c] = x[c] + x[c+4]
    take one digit per block (|.| <= nc * dmax = boundA); the second-level
    sums x[c] + x[c+2] and (a0+a1)[c] + (a0+a1)[c+2] take two (<= 2 boundA,
    the int8 check of the planner); a third level on Q2 would need four."""
    K, S = 8, 4
    nc = NB // 2 if NB > 2 else 1
    for j in range(NB):
        x = _point_terms(K, S, NB, nc, j)
        s = [_merge(x[c], x[c + 4]) for c in range(4)]
        assert max(_nterms(v) for v in x) <= nc
        assert max(_nterms(v) for v in s) <= nc
        assert max(_nterms(x[c], x[c + 2]) for c in (0, 1, 4, 5)) <= 2 * nc
        assert max(_nterms(s[c], s[c + 2]) for c in (0, 1)) <= 2 * nc
    if NB == 8:  # the reason a Q2 stays a length-2 convolution
        x = _point_terms(K, S, NB, nc, 0)
        assert _nterms(x[0], x[1], x[2], x[3]) == 4 * nc


def _merge(a, b):
    out = dict(a)
    for key, v in b.items():
        out[key] = out.get(key, 0) + v
    return out


def test_digit_sum_identity():
    """Digit sums: with x = lo + 2^7 hi (lo in [-64, 63]) on both sides,
    xa xb = (1 - 2^7) lo_a lo_b + (2^14 - 2^7) hi_a hi_b
            + 2^7 (lo_a + hi_a)(lo_b + hi_b),
    the class weights the inverse kernels apply; |hi| <= 64 keeps lo + hi an
    int8.  Checked at the extremes of the c1 plan's values (|x| <= 8160)."""
    rng = random.Random(17)

    def split(x):
        lo = ((x + 64) & 127) - 64
        return lo, (x - lo) >> 7

    for _ in range(20000):
        xa, xb = rng.randint(-8160, 8160), rng.randint(-8160, 8160)
        (la, ha), (lb, hb) = split(xa), split(xb)
        assert -128 <= la + ha <= 127 and -128 <= lb + hb <= 127
        got = (1 - 128) * la * lb + (16384 - 128) * ha * hb + 128 * (la + ha) * (lb + hb)
        assert got == xa * xb
    for xa in (-8160, 8160, -8097, 8095):
        la, ha = split(xa)
        assert -128 <= la + ha <= 127


def test_karatsuba_extremes():
    """All-extreme operands: every job value and the recombined coefficients
    stay within the int32 accumulator and int64 inverse bounds the planner
    proves (|digit sum| <= 60, 4 terms of a length-n contraction)."""
    n = 16384
    for sa in (60, -60):
        for sb in (60, -60):
            a, b = [sa] * 8, [sb] * 8
            ha = [a[i] + a[i + 4] for i in range(4)]
            hb = [b[i] + b[i + 4] for i in range(4)]
            P2 = _conv4(ha, hb)
            assert max(abs(v) * n for v in P2) < 2 ** 31
            got = _recombine(_conv4(a[:4], b[:4]), _conv4(a[4:], b[4:]), P2)
            assert got == _negacyclic(a, b)


def test_planner_uses_karatsuba_on_the_w64_plan():
    pi = m.plan_info(16384, 0, 64)
    assert (pi["b"], pi["S"], pi["NB"], pi["K"], pi["dA"]) == (4, 4, 8, 8, 1)
    assert pi["kara"] == 3 and pi["njobs"] == 8 * 27
    # 6 ordinary points x 3 x 12 + 2 half points x 12 = 240 plane products
    # (P2 one level deep: 264; one level: 6 x 48 + 2 x 16 = 320; none: 512)
    assert pi["int8_macs"] == 240 * 16384.0 ** 3
    # the level-3 accumulators (2 terms of sums <= 120) fit int32 up to
    # n ~ 74565; the W = 64 plan changes beyond that
    assert m.plan_info(40000, 0, 64)["kara"] == 3
    assert m.plan_info(74560, 0, 64)["kara"] == 3
    # b = 5 (values <= 124, c4's plan): a0 + a1 still fits int8 (one digit per
    # block), the second level's sums (<= 248) do not -- one level
    pi = m.plan_info(8192, 0, 68)
    assert (pi["b"], pi["kara"], pi["njobs"]) == (5, 1, 8 * 21)
    # plans with K != 8 or two digits keep the negacyclic pointwise
    assert m.plan_info(4096, 0, 1024)["kara"] == 0
