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
// Both kernels evaluate these sums directly for 4 consecutive elements per
// thread and write each value as d signed int8 digits; forward_simd_kernel
// (one-digit plans, int8 digit planes) keeps the digits in registers as
// packed bytes with compile-time twiddles, forward_kernel (the rest) reads
// them through L1 and spreads the evaluation points over gridDim.y when the
// operand is small.  For B they write the F stack the pointwise kernel
// expects: F[K-1-c] = +Bhat[c] and F[2K-1-c] = -Bhat[c].
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
            // d signed int8 digits: balanced 7-bit low digits, top digit rest
            for (int dd = 0; dd < a.d; ++dd) {
                int dg[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (dd < a.d - 1) {
                        int lo = ((x[q] + 64) & 127) - 64;
                        dg[q] = lo;
                        x[q] = (x[q] - lo) >> 7;
                    } else {
                        dg[q] = x[q];
                    }
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
    const int threads = 256;
    long long blocks = (a.nelem / 4 + threads - 1) / threads;
    if (blocks <= 0) return MFFTB_OK;
    if ((1 << a.lgS) != a.S || (1 << a.lgK) != a.K) return MFFTB_ERR_ARG;
    if (a.d == 1 && a.dbytes == 1 && 2 * a.S == a.K) {
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
