// fwd.cu -- Kernel 2a: forward MFFT transform of digit planes.
//
// Reference semantics: pack blocks of S digits into ring coefficients
// 0..S-1 of Z[y]/(y^K+1) (src/mfft.c:322-336) and evaluate the block
// polynomial at the NB points omega^j = y^(g j) (src/mfft.c:339-351 with the
// op lists of :163-258).  Every twiddle is a signed permutation (a
// negacyclic shift, src/roots.c:14-24), so each transformed coefficient is
// a signed sum of one digit from each of the nc non-zero blocks:
//
//     Xhat_j[c] = sum_beta  s * X[beta*S + c'],   c' = (c - g j beta) mod 2K
//                                                 (s = -1 when c' lands in [K, 2K))
//
// The kernels evaluate these sums directly for 4 consecutive elements per
// thread and write each value as d signed int8 digits: forward_simd_kernel
// (one-digit plans, int8 digit planes) keeps the digits in registers as
// packed bytes with compile-time twiddles; forward_pt_kernel (K = 8/16/32
// otherwise, while the sums fit int16) gives each warp one point and adds
// packed int16 pairs, the shift picked by a warp-uniform switch;
// forward_kernel (the rest: K = 64, wide digits) reads the digits through L1
// and spreads the evaluation points over gridDim.y when the operand is small.
// For B they write the F stack the pointwise kernel expects:
// F[K-1-c] = +Bhat[c] and F[2K-1-c] = -Bhat[c].  In Karatsuba mode
// (f_stack = 2, one digit) both operands are written as K + S planes per
// point: Xhat[0..K-1], then Xhat[c] + Xhat[c+S] for c < S; with the second
// Karatsuba level (f_stack = 3) S more follow: Xhat[c] + Xhat[c+S/2] for the
// first S/2 coefficients c of each half (c = 0..S/2-1, then S..S+S/2-1); with
// f_stack = 4 S/2 more: s[c] + s[c+S/2] (c < S/2) of the sums s[c] =
// Xhat[c] + Xhat[c+S].
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "runtime.h"

namespace mfftb {

template <int DB>
__device__ __forceinline__ void load4(const void* D, long long off, int (&v)[4]) {
    if (DB == 1) {
        char4 c = __ldg(reinterpret_cast<const char4*>(reinterpret_cast<const int8_t*>(D) + off));
        v[0] = c.x;
        v[1] = c.y;
        v[2] = c.z;
        v[3] = c.w;
    } else if (DB == 2) {
        short4 c = __ldg(reinterpret_cast<const short4*>(reinterpret_cast<const int16_t*>(D) + off));
        v[0] = c.x;
        v[1] = c.y;
        v[2] = c.z;
        v[3] = c.w;
    } else {
        int4 c = __ldg(reinterpret_cast<const int4*>(reinterpret_cast<const int32_t*>(D) + off));
        v[0] = c.x;
        v[1] = c.y;
        v[2] = c.z;
        v[3] = c.w;
    }
}

__device__ __forceinline__ void store4(int8_t* p, int a, int b, int c, int d) {
    char4 v;
    v.x = (signed char)a;
    v.y = (signed char)b;
    v.z = (signed char)c;
    v.w = (signed char)d;
    *reinterpret_cast<char4*>(p) = v;
}

template <int DB>
__global__ void __launch_bounds__(256) forward_kernel(const FwdArgs a) {
    const long long e0 = 4 * (blockIdx.x * (long long)blockDim.x + threadIdx.x);
    if (e0 >= a.nelem) return;
    const int mask2K = 2 * a.K - 1;  // 2K is a power of two
    const int nplanes_j = a.f_stack ? (2 * a.K - 1) : a.K;
    // small operands (few elements, many points) spread the points over
    // gridDim.y so that every SM gets work
    for (int j = blockIdx.y; j < a.NB; j += gridDim.y) {
        const int step = (a.g * j) & mask2K;
        if (a.f_stack >= 2) {
            // Karatsuba operands (one digit): planes x[c], then x[c] + x[c+S]
            // (and for f_stack = 3 the half-block sums)
            auto coef = [&](int c, int (&x)[4]) {
                x[0] = x[1] = x[2] = x[3] = 0;
                int e = 0;
                for (int beta = 0; beta < a.nc; ++beta, e = (e + step) & mask2K) {
                    int r = (c - e) & mask2K;
                    int sgn = 1;
                    if (r >= a.K) {
                        r -= a.K;
                        sgn = -1;
                    }
                    if (r >= a.S) continue;
                    const int m = (beta << a.lgS) + r;
                    if (m >= a.Lb) continue;
                    int v[4];
                    load4<DB>(a.D, (long long)m * a.dplane + e0, v);
                    for (int q = 0; q < 4; ++q) x[q] += sgn * v[q];
                }
            };
            const int per_j = a.f_stack == 4   ? a.K + 2 * a.S + a.S / 2
                              : a.f_stack == 3 ? a.K + 2 * a.S
                                               : a.K + a.S;
            const long long base = (long long)j * per_j;
            for (int c = 0; c < a.S; ++c) {
                int lo[4], hi[4];
                coef(c, lo);
                coef(c + a.S, hi);
                store4(a.out + (base + c) * a.oplane + e0, lo[0], lo[1], lo[2], lo[3]);
                store4(a.out + (base + c + a.S) * a.oplane + e0, hi[0], hi[1], hi[2], hi[3]);
                store4(a.out + (base + a.K + c) * a.oplane + e0, lo[0] + hi[0], lo[1] + hi[1],
                       lo[2] + hi[2], lo[3] + hi[3]);
            }
            if (a.f_stack >= 3) {
                const int h = a.S / 2;
                for (int i = 0; i < a.S; ++i) {
                    const int c = (i / h) * a.S + i % h;  // first coefficient of the pair
                    int x0[4], x1[4];
                    coef(c, x0);
                    coef(c + h, x1);
                    store4(a.out + (base + a.K + a.S + i) * a.oplane + e0, x0[0] + x1[0],
                           x0[1] + x1[1], x0[2] + x1[2], x0[3] + x1[3]);
                }
            }
            if (a.f_stack == 4) {
                const int h = a.S / 2;
                for (int c = 0; c < h; ++c) {
                    int t[4] = {0, 0, 0, 0}, v[4];
                    const int idx[4] = {c, c + a.S, c + h, c + h + a.S};
                    for (int q = 0; q < 4; ++q) {
                        coef(idx[q], v);
                        for (int e = 0; e < 4; ++e) t[e] += v[e];
                    }
                    store4(a.out + (base + a.K + 2 * a.S + c) * a.oplane + e0, t[0], t[1], t[2],
                           t[3]);
                }
            }
            continue;
        }
        for (int c = 0; c < a.K; ++c) {
            int x[4] = {0, 0, 0, 0};
            int e = 0;  // g * j * beta mod 2K
            for (int beta = 0; beta < a.nc; ++beta, e = (e + step) & mask2K) {
                int r = (c - e) & mask2K;
                int sgn = 1;
                if (r >= a.K) {
                    r -= a.K;
                    sgn = -1;
                }
                if (r >= a.S) continue;
                const int m = (beta << a.lgS) + r;
                if (m >= a.Lb) continue;
                int v[4];
                load4<DB>(a.D, (long long)m * a.dplane + e0, v);
                x[0] += sgn * v[0];
                x[1] += sgn * v[1];
                x[2] += sgn * v[2];
                x[3] += sgn * v[3];
            }
            // d signed int8 digits: balanced 7-bit low digits, top digit
            // rest; with digit sums the two digits of the split, then their sum
            const int nsplit = a.dsum ? 2 : a.d;
            int dsum4[4] = {0, 0, 0, 0};
            for (int dd = 0; dd < a.d; ++dd) {
                int dg[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (dd >= nsplit) {
                        dg[q] = dsum4[q];
                    } else if (dd < nsplit - 1) {
                        int lo = ((x[q] + 64) & 127) - 64;
                        dg[q] = lo;
                        x[q] = (x[q] - lo) >> 7;
                    } else {
                        dg[q] = x[q];
                    }
                    dsum4[q] += dd < nsplit ? dg[q] : 0;
                }
                if (!a.f_stack) {
                    long long plane = ((long long)j * a.d + dd) * nplanes_j + c;
                    store4(a.out + plane * a.oplane + e0, dg[0], dg[1], dg[2], dg[3]);
                } else {
                    long long base = ((long long)j * a.d + dd) * nplanes_j;
                    store4(a.out + (base + (a.K - 1 - c)) * a.oplane + e0, dg[0], dg[1], dg[2],
                           dg[3]);
                    if (c >= 1)
                        store4(a.out + (base + (2 * a.K - 1 - c)) * a.oplane + e0, -dg[0], -dg[1],
                               -dg[2], -dg[3]);
                }
            }
        }
    }
}

// Single-digit plans (every transformed coefficient fits int8, so every
// partial sum does too) with int8 digit planes: 4 elements per thread as
// packed bytes, byte-wise SIMD adds, all twiddle indices resolved at compile
// time.  Same outputs as forward_kernel.  NBLK: blocks that may be non-zero
// (NB, or NB/2 when nc <= NB/2, which NB = next_pow2(ncA + ncB) gives for
// operands of equal width -- half the digit registers).
template <int NB, int K, int NBLK = NB>
__global__ void __launch_bounds__(256) forward_simd_kernel(const FwdArgs a) {
    constexpr int S = K / 2, G = 2 * K / NB, TWO_K = 2 * K;
    const long long e0 = 4 * (blockIdx.x * 256LL + threadIdx.x);
    if (e0 >= a.nelem) return;
    const int8_t* D = reinterpret_cast<const int8_t*>(a.D);
    uint32_t dg[NBLK * S];
#pragma unroll
    for (int m = 0; m < NBLK * S; ++m)
        dg[m] = (m < a.Lb && m / S < a.nc)
                    ? __ldg(reinterpret_cast<const uint32_t*>(D + (long long)m * a.dplane + e0))
                    : 0u;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        if (a.f_stack >= 2) {
            // Karatsuba operands: x[0..S-1], x[S..K-1], x[c] + x[c+S] (and
            // for f_stack = 3 the half-block sums x[c] + x[c+S/2])
            uint32_t xs[K];
#pragma unroll
            for (int c = 0; c < K; ++c) {
                uint32_t x = 0;
#pragma unroll
                for (int beta = 0; beta < NBLK; ++beta) {
                    const int e = (G * j * beta) % TWO_K;
                    int r = ((c - e) % TWO_K + TWO_K) % TWO_K;
                    const bool neg = r >= K;
                    if (neg) r -= K;
                    if (r < S)
                        x = neg ? __vsub4(x, dg[beta * S + r]) : __vadd4(x, dg[beta * S + r]);
                }
                xs[c] = x;
            }
            const long long base =
                (long long)j * (a.f_stack == 4 ? K + 2 * S + S / 2
                                               : (a.f_stack == 3 ? K + 2 * S : K + S));
#pragma unroll
            for (int c = 0; c < K; ++c)
                *reinterpret_cast<uint32_t*>(a.out + (base + c) * a.oplane + e0) = xs[c];
#pragma unroll
            for (int c = 0; c < S; ++c)
                *reinterpret_cast<uint32_t*>(a.out + (base + K + c) * a.oplane + e0) =
                    __vadd4(xs[c], xs[c + S]);
            if (a.f_stack >= 3) {
                constexpr int H = S / 2 > 0 ? S / 2 : 1;
#pragma unroll
                for (int i = 0; i < S; ++i) {
                    const int c = (i / H) * S + i % H;
                    *reinterpret_cast<uint32_t*>(a.out + (base + K + S + i) * a.oplane + e0) =
                        __vadd4(xs[c], xs[c + H]);
                }
            }
            if (a.f_stack == 4) {
                constexpr int H = S / 2 > 0 ? S / 2 : 1;
#pragma unroll
                for (int c = 0; c < H; ++c)
                    *reinterpret_cast<uint32_t*>(a.out + (base + K + 2 * S + c) * a.oplane + e0) =
                        __vadd4(__vadd4(xs[c], xs[c + S]), __vadd4(xs[c + H], xs[c + H + S]));
            }
            continue;
        }
#pragma unroll
        for (int c = 0; c < K; ++c) {
            uint32_t x = 0;
#pragma unroll
            for (int beta = 0; beta < NBLK; ++beta) {
                const int e = (G * j * beta) % TWO_K;
                int r = ((c - e) % TWO_K + TWO_K) % TWO_K;
                const bool neg = r >= K;
                if (neg) r -= K;
                if (r < S) x = neg ? __vsub4(x, dg[beta * S + r]) : __vadd4(x, dg[beta * S + r]);
            }
            if (!a.f_stack) {
                *reinterpret_cast<uint32_t*>(a.out + (long long)(j * K + c) * a.oplane + e0) = x;
            } else {
                const long long base = (long long)j * (2 * K - 1);
                *reinterpret_cast<uint32_t*>(a.out + (base + (K - 1 - c)) * a.oplane + e0) = x;
                if (c >= 1)
                    *reinterpret_cast<uint32_t*>(a.out + (base + (2 * K - 1 - c)) * a.oplane + e0) =
                        __vsub4(0u, x);
            }
        }
    }
}

// One evaluation point per warp (multi-digit plans and int16 digit planes,
// K = 8, 16 or 32).  Lane l holds elements e0..e0+3 (e0 = 4l + 128 x block)
// as two packed int16 pairs per coefficient; block beta enters point j
// shifted by e = g j beta mod 2K, which is warp-uniform, so a switch on e
// picks a fully unrolled shift-and-add with constant register indices.  Every
// partial sum is a signed sum of at most nc digits of at most 2^b, which the
// launcher checks stays below 2^15.  The digits a warp loads are the ones
// the other warps of the CTA (other points, same elements) load too, so they
// come from L1 after the first.
template <int K, int E>
__device__ __forceinline__ void fwd_pt_shift_add(uint32_t (&acc)[K][2],
                                                 const uint32_t (&x)[K / 2][2]) {
    if constexpr (E < 2 * K) {
        constexpr int S = K / 2;
#pragma unroll
        for (int c = 0; c < K; ++c) {
            const int r = (c - E + 2 * K) % (2 * K);  // X coefficient landing on c
            if (r < S) {
                acc[c][0] = __vadd2(acc[c][0], x[r][0]);
                acc[c][1] = __vadd2(acc[c][1], x[r][1]);
            } else if (r >= K && r < K + S) {  // wrapped past y^K: negated
                acc[c][0] = __vsub2(acc[c][0], x[r - K][0]);
                acc[c][1] = __vsub2(acc[c][1], x[r - K][1]);
            }
        }
    }
}

template <int DB>
__device__ __forceinline__ void load4_pairs(const void* D, long long off, uint32_t& p01,
                                            uint32_t& p23) {
    if (DB == 2) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const int16_t*>(D) + off));
        p01 = v.x;
        p23 = v.y;
    } else {
        const char4 c = __ldg(reinterpret_cast<const char4*>(reinterpret_cast<const int8_t*>(D) + off));
        p01 = (uint32_t)(uint16_t)(int16_t)c.x | ((uint32_t)(uint16_t)(int16_t)c.y << 16);
        p23 = (uint32_t)(uint16_t)(int16_t)c.z | ((uint32_t)(uint16_t)(int16_t)c.w << 16);
    }
}

#define FWD_PT_CASE(E)                      \
    case E:                                 \
        fwd_pt_shift_add<K, E>(acc, x);     \
        break;

template <int K, int DB>
__global__ void __launch_bounds__(256) forward_pt_kernel(const FwdArgs a, int npg) {
    constexpr int S = K / 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the npg point groups of one 128-element slice are consecutive blocks,
    // so they run together and read the slice's digit planes from L2 once
    const int pg = (int)(blockIdx.x % npg);
    const long long eb = blockIdx.x / npg;
    const int j = pg * (blockDim.x >> 5) + warp;
    const long long e0 = eb * 128 + 4 * lane;
    if (j >= a.NB || e0 >= a.nelem) return;
    const int step = (a.g * j) & (2 * K - 1);
    uint32_t acc[K][2];
#pragma unroll
    for (int c = 0; c < K; ++c) acc[c][0] = acc[c][1] = 0u;
    int e = 0;
    for (int beta = 0; beta < a.nc; ++beta, e = (e + step) & (2 * K - 1)) {
        uint32_t x[S][2];
#pragma unroll
        for (int r = 0; r < S; ++r) {
            const int m = beta * S + r;
            x[r][0] = x[r][1] = 0u;
            if (m < a.Lb) load4_pairs<DB>(a.D, (long long)m * a.dplane + e0, x[r][0], x[r][1]);
        }
        switch (e) {
            FWD_PT_CASE(0) FWD_PT_CASE(1) FWD_PT_CASE(2) FWD_PT_CASE(3)
            FWD_PT_CASE(4) FWD_PT_CASE(5) FWD_PT_CASE(6) FWD_PT_CASE(7)
            FWD_PT_CASE(8) FWD_PT_CASE(9) FWD_PT_CASE(10) FWD_PT_CASE(11)
            FWD_PT_CASE(12) FWD_PT_CASE(13) FWD_PT_CASE(14) FWD_PT_CASE(15)
            FWD_PT_CASE(16) FWD_PT_CASE(17) FWD_PT_CASE(18) FWD_PT_CASE(19)
            FWD_PT_CASE(20) FWD_PT_CASE(21) FWD_PT_CASE(22) FWD_PT_CASE(23)
            FWD_PT_CASE(24) FWD_PT_CASE(25) FWD_PT_CASE(26) FWD_PT_CASE(27)
            FWD_PT_CASE(28) FWD_PT_CASE(29) FWD_PT_CASE(30) FWD_PT_CASE(31)
            FWD_PT_CASE(32) FWD_PT_CASE(33) FWD_PT_CASE(34) FWD_PT_CASE(35)
            FWD_PT_CASE(36) FWD_PT_CASE(37) FWD_PT_CASE(38) FWD_PT_CASE(39)
            FWD_PT_CASE(40) FWD_PT_CASE(41) FWD_PT_CASE(42) FWD_PT_CASE(43)
            FWD_PT_CASE(44) FWD_PT_CASE(45) FWD_PT_CASE(46) FWD_PT_CASE(47)
            FWD_PT_CASE(48) FWD_PT_CASE(49) FWD_PT_CASE(50) FWD_PT_CASE(51)
            FWD_PT_CASE(52) FWD_PT_CASE(53) FWD_PT_CASE(54) FWD_PT_CASE(55)
            FWD_PT_CASE(56) FWD_PT_CASE(57) FWD_PT_CASE(58) FWD_PT_CASE(59)
            FWD_PT_CASE(60) FWD_PT_CASE(61) FWD_PT_CASE(62) FWD_PT_CASE(63)
            default: break;
        }
    }
    // d signed int8 digits per value (balanced 7-bit low digits, top digit
    // the rest), the same split as forward_kernel
    const long long plane0 = (long long)j * a.d * (a.f_stack ? (2 * K - 1) : K);
    if (a.d <= 2 || a.dsum) {
        // the same split on the packed int16 pairs: lo = ((x + 64) & 127) - 64
        // per halfword (only its low 7 bits matter, so a wrapping add is
        // exact), hi = (x - lo) / 128, whose byte is bits 7..14 of each
        // halfword (the plan bounds |hi| <= 127, so x - lo does not wrap);
        // bytes of four elements gathered with one byte permute each
        auto store_planes = [&](int dd, int c, uint32_t v) {
            if (!a.f_stack) {
                *reinterpret_cast<uint32_t*>(a.out + (plane0 + (long long)dd * K + c) * a.oplane +
                                             e0) = v;
            } else {
                const long long base = plane0 + (long long)dd * (2 * K - 1);
                *reinterpret_cast<uint32_t*>(a.out + (base + (K - 1 - c)) * a.oplane + e0) = v;
                if (c >= 1)
                    *reinterpret_cast<uint32_t*>(a.out + (base + (2 * K - 1 - c)) * a.oplane + e0) =
                        __vsub4(0u, v);
            }
        };
#pragma unroll
        for (int c = 0; c < K; ++c) {
            const uint32_t p01 = acc[c][0], p23 = acc[c][1];
            if (a.d == 1) {
                store_planes(0, c, __byte_perm(p01, p23, 0x6420));
                continue;
            }
            const uint32_t lo01 = __vsub2(__vadd2(p01, 0x00400040u) & 0x007F007Fu, 0x00400040u);
            const uint32_t lo23 = __vsub2(__vadd2(p23, 0x00400040u) & 0x007F007Fu, 0x00400040u);
            const uint32_t lo = __byte_perm(lo01, lo23, 0x6420);
            const uint32_t hi =
                __byte_perm(__vsub2(p01, lo01) >> 7, __vsub2(p23, lo23) >> 7, 0x6420);
            store_planes(0, c, lo);
            store_planes(1, c, hi);
            // digit sums: lo + hi per byte (in [-128, 127] by the plan, so
            // the byte-wise wrapping add is exact)
            if (a.dsum) store_planes(2, c, __vadd4(lo, hi));
        }
        return;
    }
#pragma unroll
    for (int c = 0; c < K; ++c) {
        int x[4] = {(int)(int16_t)(acc[c][0] & 0xffffu), (int)(int16_t)(acc[c][0] >> 16),
                    (int)(int16_t)(acc[c][1] & 0xffffu), (int)(int16_t)(acc[c][1] >> 16)};
        for (int dd = 0; dd < a.d; ++dd) {
            int dg[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (dd < a.d - 1) {
                    const int lo = ((x[q] + 64) & 127) - 64;
                    dg[q] = lo;
                    x[q] = (x[q] - lo) >> 7;
                } else {
                    dg[q] = x[q];
                }
            }
            if (!a.f_stack) {
                store4(a.out + (plane0 + (long long)dd * K + c) * a.oplane + e0, dg[0], dg[1],
                       dg[2], dg[3]);
            } else {
                const long long base = plane0 + (long long)dd * (2 * K - 1);
                store4(a.out + (base + (K - 1 - c)) * a.oplane + e0, dg[0], dg[1], dg[2], dg[3]);
                if (c >= 1)
                    store4(a.out + (base + (2 * K - 1 - c)) * a.oplane + e0, -dg[0], -dg[1],
                           -dg[2], -dg[3]);
            }
        }
    }
}
#undef FWD_PT_CASE

template <int K>
static int launch_pt(const FwdArgs& a, cudaStream_t stream) {
    const int wpb = a.NB < 8 ? a.NB : 8;  // warps (points) per CTA
    const int npg = (a.NB + wpb - 1) / wpb;
    const long long blocks = (a.nelem + 127) / 128 * npg;
    if (blocks > 0x7fffffffLL) return MFFTB_ERR_ARG;
    if (a.dbytes == 1) forward_pt_kernel<K, 1><<<(unsigned)blocks, 32 * wpb, 0, stream>>>(a, npg);
    else forward_pt_kernel<K, 2><<<(unsigned)blocks, 32 * wpb, 0, stream>>>(a, npg);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

template <int NB, int K>
static int launch_simd(const FwdArgs& a, cudaStream_t stream) {
    long long blocks = (a.nelem / 4 + 255) / 256;
    if (blocks <= 0) return MFFTB_OK;
    if (a.nc <= NB / 2) {
        forward_simd_kernel<NB, K, NB / 2><<<(unsigned)blocks, 256, 0, stream>>>(a);
    } else {
        // all NB blocks in registers only while they fit (NB*S <= 64 words)
        if constexpr (NB * K / 2 <= 64)
            forward_simd_kernel<NB, K><<<(unsigned)blocks, 256, 0, stream>>>(a);
        else
            return MFFTB_ERR_UNSUPPORTED;
    }
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int forward_launch(const FwdArgs& a, cudaStream_t stream) {
    if (a.nelem % 4 || a.d < 1 || a.d > 4) return MFFTB_ERR_ARG;
    if (a.dsum && (a.d != 3 || a.f_stack >= 2)) return MFFTB_ERR_ARG;
    // Karatsuba operands: one int8 digit per value, blocks of S = K/2
    if (a.f_stack >= 2 && (a.d != 1 || 2 * a.S != a.K)) return MFFTB_ERR_ARG;
    if (a.f_stack >= 3 && a.S < 2) return MFFTB_ERR_ARG;
    const int threads = 256;
    long long blocks = (a.nelem / 4 + threads - 1) / threads;
    if (blocks <= 0) return MFFTB_OK;
    if ((1 << a.lgS) != a.S || (1 << a.lgK) != a.K) return MFFTB_ERR_ARG;
    if (a.variant == 0 && a.d == 1 && a.dbytes == 1 && 2 * a.S == a.K) {
        int rc = MFFTB_ERR_UNSUPPORTED;
        if (a.NB == 8 && a.K == 8) rc = launch_simd<8, 8>(a, stream);
        else if (a.NB == 4 && a.K == 4) rc = launch_simd<4, 4>(a, stream);
        else if (a.NB == 8 && a.K == 4) rc = launch_simd<8, 4>(a, stream);
        else if (a.NB == 4 && a.K == 8) rc = launch_simd<4, 8>(a, stream);
        else if (a.NB == 16 && a.K == 16) rc = launch_simd<16, 16>(a, stream);
        else if (a.NB == 16 && a.K == 8) rc = launch_simd<16, 8>(a, stream);
        else if (a.NB == 8 && a.K == 16) rc = launch_simd<8, 16>(a, stream);
        if (rc != MFFTB_ERR_UNSUPPORTED) return rc;
    }
    // one point per warp with int16 lanes when every partial sum fits them:
    // |sum| <= nc * 2^b < 2^15
    if (a.variant == 0 && a.f_stack < 2 && (a.dbytes == 1 || a.dbytes == 2) && 2 * a.S == a.K &&
        a.b >= 1 &&
        a.b <= 14 && ((long long)a.nc << a.b) < 32768 && a.NB >= 1 && a.nelem % 4 == 0) {
        if (a.K == 8) return launch_pt<8>(a, stream);
        if (a.K == 16) return launch_pt<16>(a, stream);
        if (a.K == 32) return launch_pt<32>(a, stream);
    }
    long long jsplit = (4 * 148 + blocks - 1) / blocks;  // aim at >= 4 CTAs per SM
    if (jsplit > a.NB) jsplit = a.NB;
    if (jsplit < 1) jsplit = 1;
    const dim3 grid((unsigned)blocks, (unsigned)jsplit);
    if (a.dbytes == 1) forward_kernel<1><<<grid, threads, 0, stream>>>(a);
    else if (a.dbytes == 2) forward_kernel<2><<<grid, threads, 0, stream>>>(a);
    else forward_kernel<4><<<grid, threads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

}  // namespace mfftb
