// inv.cu -- Kernel 2b + Kernel 4: inverse MFFT transform, /NB, fold onto
// radix-2^b positions, carry propagation and output formatting, fused.
//
// Reference semantics:
//   * Chat_j[t] = sum over digit classes w and chunks of 2^(7w) * acc
//     (the int8 digit split of the pointwise step, undone exactly in int64);
//   * inverse transform NB * C_beta = sum_j y^(-g j beta) Chat_j
//     (src/mfft.c:398-404 with the op list of :262-299);
//   * fold: position beta*S + c receives C_beta[c] / NB (src/mfft.c:407-418);
//   * INV_U16: carry into 16-bit two's complement limbs, normalize_planes
//     (src/bigmat.c:48-60);
//   * INV_I64: the unnormalised int64 planes conv_mfft returns (limb mode);
//   * INV_F32 / INV_F64: extract + round_to + ldexpf / ldexp of
//     fpx_decode_f32 / fpx_decode_f64 (src/fpfixed.c:212-322), see decode.cuh.
//
// Kernels: inverse_kernel (below; any plan) -- a CTA owns E consecutive
// elements (E <= 32) and keeps their NB*K int64 transformed values in shared
// memory; 256 threads cooperate on the loads and on the inverse DFT, then E
// threads fold and carry one element each.  inverse_reg_kernel (NB*K <= 64)
// and inverse_lane_kernel (K in {8,16,32}, NB <= 32) are the fast paths for
// the common plans; school_carry*_kernel finish schoolbook plans.
#include <cuda_runtime.h>

#include <cstdint>

#include "decode.cuh"
#include "kernels.h"
#include "runtime.h"

namespace mfftb {

// fp output of one element from its exact product words
__device__ __forceinline__ void store_float(const InvArgs& a, long long o, uint32_t* words, int nw) {
    if (a.out_kind == INV_F64)
        reinterpret_cast<double*>(a.out)[o] = decode_words_f64(words, nw, a.bit_off, a.S_scale);
    else
        reinterpret_cast<float*>(a.out)[o] = decode_words_f32(words, nw, a.bit_off, a.S_scale);
}

constexpr int INV_THREADS = 256;
constexpr int INV_VPT = 16;     // inverse-DFT outputs per thread (registers)
constexpr int INV_MAXW = 40;    // 32-bit words of an fp32-path product (1280 bits)

__global__ void __launch_bounds__(INV_THREADS) inverse_kernel(const InvArgs a) {
    extern __shared__ int64_t sm[];  // [NB*K][E]
    const int E = a.elems;
    const int NK = a.NB * a.K;
    const long long per_row = a.lda;
    const long long e_base = (long long)blockIdx.x * E;
    const long long total = (long long)a.rows * per_row;

    // ---- phase 1: Chat values for the CTA's elements (smem index q*E + i)
    const int lgE = a.lgE, emask = E - 1;
    for (int idx = threadIdx.x; idx < NK * E; idx += INV_THREADS) {
        const int q = idx >> lgE, i = idx & emask;
        const long long e = e_base + i;
        int64_t v = 0;
        if (e < total) {
            const int32_t* src = a.acc + (long long)q * a.nW * a.nchunk * a.acc_plane + e;
            for (int w = 0; w < a.nW; ++w) {
                int64_t s = 0;
                for (int ch = 0; ch < a.nchunk; ++ch, src += a.acc_plane) s += (int64_t)__ldg(src);
                v += s * inv_class_weight(a.dsum, w);
            }
        }
        sm[idx] = v;
    }
    __syncthreads();

    // ---- phase 2: inverse DFT, outputs (beta, c, i) -> registers -> smem
    {
        const int mask2K = 2 * a.K - 1, kmask = a.K - 1;
        int64_t outv[INV_VPT];
#pragma unroll
        for (int k = 0; k < INV_VPT; ++k) {
            const int idx = threadIdx.x + k * INV_THREADS;
            int64_t acc = 0;
            if (idx < NK * E) {
                const int i = idx & emask;
                const int bc = idx >> lgE;
                const int beta = bc >> a.lgK, c = bc & kmask;
                const int step = (a.g * beta) & mask2K;
                int e = 0;  // g * j * beta mod 2K
                const int64_t* col = sm + i;
                for (int j = 0; j < a.NB; ++j, e = (e + step) & mask2K) {
                    // y^(-e) * Chat_j: coefficient c takes Chat_j[(c + e) mod 2K]
                    int r = (c + e) & mask2K;
                    const int64_t v = col[((j << a.lgK) + (r & kmask)) << lgE];
                    acc += r >= a.K ? -v : v;
                }
                acc >>= a.log2NB;  // exact: acc is a multiple of NB
            }
            outv[k] = acc;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < INV_VPT; ++k) {
            const int idx = threadIdx.x + k * INV_THREADS;
            if (idx < NK * E) sm[idx] = outv[k];
        }
    }
    __syncthreads();

    // ---- phase 3: fold + carry + output, one thread per element
    if (threadIdx.x >= E) return;
    const long long e = e_base + threadIdx.x;
    if (e >= total) return;
    const int row = (int)(e / per_row), col = (int)(e % per_row);
    if (row >= a.rows || col >= a.cols) return;
    const int i = threadIdx.x;
    const int S = a.S, lgS = a.lgS, smask = S - 1;
    auto pos_value = [&](int p) -> int64_t {
        const int beta = p >> lgS, c = p & smask;
        int64_t v = 0;
        if (beta < a.NB) v += sm[(((beta << a.lgK) + c) << lgE) + i];
        if (beta >= 1 && beta - 1 < a.NB) v += sm[((((beta - 1) << a.lgK) + c + S) << lgE) + i];
        return v;
    };

    if (a.out_kind == INV_I64) {
        int64_t* out = reinterpret_cast<int64_t*>(a.out);
        for (int p = 0; p < a.RL; ++p)
            out[(long long)p * a.out_plane + (long long)row * a.ldo + col] =
                p < a.positions ? pos_value(p) : 0;
        return;
    }

    const uint64_t mask = (1ULL << a.b) - 1ULL;
    int64_t carry = 0;
    uint64_t bits = 0;
    int nb = 0;
    if (a.out_kind == INV_U16) {
        uint16_t* out = reinterpret_cast<uint16_t*>(a.out);
        int w = 0;
        const long long o = (long long)row * a.ldo + col;
        for (int p = 0; p < a.positions && w < a.RL; ++p) {
            const int64_t v = pos_value(p) + carry;
            bits |= ((uint64_t)v & mask) << nb;
            nb += a.b;
            carry = v >> a.b;
            while (nb >= 16 && w < a.RL) {
                out[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
                bits >>= 16;
                nb -= 16;
                ++w;
            }
        }
        while (w < a.RL) {
            const int need = 16 - nb;
            bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
            carry >>= need;
            out[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
            bits = 0;
            nb = 0;
            ++w;
        }
        return;
    }

    // INV_F32: two's complement words of the exact product, then round once
    uint32_t words[INV_MAXW];
    int nw = 0;
    for (int p = 0; p < a.positions; ++p) {
        const int64_t v = pos_value(p) + carry;
        bits |= ((uint64_t)v & mask) << nb;
        nb += a.b;
        carry = v >> a.b;
        if (nb >= 32) {
            if (nw < INV_MAXW) words[nw++] = (uint32_t)bits;
            bits >>= 32;
            nb -= 32;
        }
    }
    // the remaining carry is the sign-extended top part: two more words
    // always cover it (|carry| < 2^62)
    for (int k = 0; k < 3 && nw < INV_MAXW; ++k) {
        const int need = 32 - nb;
        bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
        carry >>= need;
        words[nw++] = (uint32_t)bits;
        bits = 0;
        nb = 0;
    }
    store_float(a, (long long)row * a.ldo + col, words, nw);
}

// ---------------------------------------------------------------- register variant
// For plans with NB*K <= 64 (the W=64, fp32 and fp64 configurations) one thread
// owns one element and keeps its NB ring elements in registers: a radix-2
// decimation-in-time inverse FFT whose twiddles y^-e are compile-time signed
// permutations, then fold, carry and output.  Same semantics as
// inverse_kernel.
template <int NB, int K>
__device__ __forceinline__ void ring_mul_pow(const int64_t (&v)[K], int64_t (&o)[K], int e) {
    // o = y^e * v in Z[y]/(y^K + 1), e in [0, 2K) (compile-time after unrolling)
#pragma unroll
    for (int c = 0; c < K; ++c) {
        int r = c - e;
        r = ((r % (2 * K)) + 2 * K) % (2 * K);
        o[c] = r < K ? v[r] : -v[r - K];
    }
}

// kara = 2: a length-4 convolution P from the 9 job planes of its three
// length-2 convolutions Q0, Q1, Q2 (3 coefficients each):
// P = Q0 + y^2 (Q2 - Q0 - Q1) + y^4 Q1
__device__ __forceinline__ void kara2_expand(const int32_t* src, long long plane,
                                             int64_t (&P)[7]) {
    int64_t q0[3], q1[3], m[3];
#pragma unroll
    for (int s = 0; s < 3; ++s) {
        q0[s] = __ldg(src + s * plane);
        q1[s] = __ldg(src + (3 + s) * plane);
    }
#pragma unroll
    for (int s = 0; s < 3; ++s) m[s] = (int64_t)__ldg(src + (6 + s) * plane) - q0[s] - q1[s];
    P[0] = q0[0];
    P[1] = q0[1];
    P[2] = q0[2] + m[0];
    P[3] = m[1];
    P[4] = q1[0] + m[2];
    P[5] = q1[1];
    P[6] = q1[2];
}

// KARA: the Karatsuba level of the job planes (0: NB*K negacyclic planes),
// a template argument so that every load of a point is issued back to back.
// Levels 2 and 3 (25 / 27 planes per point) are held to three blocks per SM
// (168 registers, a small spill): the loads in flight per SM matter more
// than the spill (c5, level 2: 44.6 ms against 53.8 ms at two blocks per SM).
template <int NB, int K, int KARA>
__global__ void __launch_bounds__(128, KARA >= 2 ? 3 : 1) inverse_reg_kernel(const InvArgs a) {
    constexpr int S = K / 2, LGNB = NB == 2 ? 1 : (NB == 4 ? 2 : 3);
    const long long e = blockIdx.x * 128LL + threadIdx.x;
    const long long total = (long long)a.rows * a.lda;
    if (e >= total) return;
    const int row = (int)(e / a.lda), col = (int)(e % a.lda);
    if (row >= a.rows || col >= a.cols) return;

    int64_t x[NB][K];
    // load Chat_j into bit-reversed position for the in-place DIT.  With one
    // digit class and one chunk (the single-digit plans) all NB*K loads are
    // independent and issued back to back.
    auto bitrev = [](int j) {
        return LGNB == 1 ? j : (LGNB == 2 ? (((j & 1) << 1) | (j >> 1))
                                          : (((j & 1) << 2) | (j & 2) | (j >> 2)));
    };
    if constexpr (K == 8 && KARA > 0) {
        {
            // Chat_j = P0 - P1 + y^4 (P2 - P0 - P1) mod y^8 + 1, with
            // M = P2 - P0 - P1: Chat[t] = D[t] - M[t+4] (t < 3), D[3] (t = 3),
            // D[t] + M[t-4] (t = 4..6), M[3] (t = 7), D = P0 - P1.  Level 2
            // first forms P0 and P1 from their length-2 convolutions.
            constexpr int NQ = KARA == 3 ? 27 : (KARA == 2 ? 25 : 21);
            constexpr int P2 = KARA == 1 ? 14 : 18;
#pragma unroll
            for (int j = 0; j < NB; ++j) {
                const int32_t* src = a.acc + (long long)j * NQ * a.acc_plane + e;
                int64_t P0[7];
                if constexpr (KARA >= 2) {
                    kara2_expand(src, a.acc_plane, P0);
                } else {
#pragma unroll
                    for (int s = 0; s < 7; ++s) P0[s] = __ldg(src + (long long)s * a.acc_plane);
                }
                if (j == 0 || 2 * j == NB) {  // half point: P0 only
#pragma unroll
                    for (int t = 0; t < 7; ++t) x[bitrev(j)][t] = P0[t];
                    x[bitrev(j)][7] = 0;
                    continue;
                }
                int64_t P1[7], M[7];
                if constexpr (KARA >= 2) {
                    kara2_expand(src + 9 * a.acc_plane, a.acc_plane, P1);
                } else {
#pragma unroll
                    for (int s = 0; s < 7; ++s)
                        P1[s] = __ldg(src + (long long)(7 + s) * a.acc_plane);
                }
                if constexpr (KARA == 3) {
                    kara2_expand(src + 18 * a.acc_plane, a.acc_plane, M);
#pragma unroll
                    for (int s = 0; s < 7; ++s) M[s] -= P0[s] + P1[s];
                } else {
#pragma unroll
                    for (int s = 0; s < 7; ++s)
                        M[s] = (int64_t)__ldg(src + (long long)(P2 + s) * a.acc_plane) - P0[s] -
                               P1[s];
                }
                int64_t(&y)[K] = x[bitrev(j)];
#pragma unroll
                for (int t = 0; t < 3; ++t) y[t] = P0[t] - P1[t] - M[t + 4];
                y[3] = P0[3] - P1[3];
#pragma unroll
                for (int t = 4; t < 7; ++t) y[t] = P0[t] - P1[t] + M[t - 4];
                y[7] = M[3];
            }
            goto loaded;
        }
    }
    if (a.nW == 1 && a.nchunk == 1) {
        int32_t raw[NB * K];
#pragma unroll
        for (int q = 0; q < NB * K; ++q) raw[q] = __ldg(a.acc + (long long)q * a.acc_plane + e);
#pragma unroll
        for (int j = 0; j < NB; ++j)
#pragma unroll
            for (int t = 0; t < K; ++t) x[bitrev(j)][t] = raw[j * K + t];
    } else {
#pragma unroll
        for (int j = 0; j < NB; ++j) {
#pragma unroll
            for (int t = 0; t < K; ++t) {
                const int32_t* src =
                    a.acc + (long long)(j * K + t) * a.nW * a.nchunk * a.acc_plane + e;
                int64_t v = 0;
                for (int w = 0; w < a.nW; ++w) {
                    int64_t s = 0;
                    for (int ch = 0; ch < a.nchunk; ++ch, src += a.acc_plane)
                        s += (int64_t)__ldg(src);
                    v += s * inv_class_weight(a.dsum, w);
                }
                x[bitrev(j)][t] = v;
            }
        }
    }
loaded:
    // DIT stages with W = omega^-1 = y^-g
#pragma unroll
    for (int len = 2; len <= NB; len <<= 1) {
#pragma unroll
        for (int st = 0; st < NB; st += len) {
#pragma unroll
            for (int k = 0; k < len / 2; ++k) {
                const int e0 = (2 * K / NB) * (NB / len) * k;           // g * (NB/len) * k
                const int ee = (2 * K - (e0 % (2 * K))) % (2 * K);     // inverse twiddle
                int64_t tw[K];
                ring_mul_pow<NB, K>(x[st + k + len / 2], tw, ee);
#pragma unroll
                for (int c = 0; c < K; ++c) {
                    const int64_t u = x[st + k][c];
                    x[st + k][c] = u + tw[c];
                    x[st + k + len / 2][c] = u - tw[c];
                }
            }
        }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int c = 0; c < K; ++c) x[b][c] >>= LGNB;  // exact division by NB

    auto pos_value = [&](int p) -> int64_t {
        int64_t v = 0;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
            for (int c = 0; c < K; ++c)
                if (b * S + c == p) v += x[b][c];
        }
        return v;
    };

    if (a.out_kind == INV_I64) {
        int64_t* out = reinterpret_cast<int64_t*>(a.out);
        const long long o = (long long)row * a.ldo + col;
#pragma unroll
        for (int p = 0; p < (NB + 1) * S; ++p)
            if (p < a.RL) out[(long long)p * a.out_plane + o] = p < a.positions ? pos_value(p) : 0;
        for (int p = (NB + 1) * S; p < a.RL; ++p) out[(long long)p * a.out_plane + o] = 0;
        return;
    }
    const uint64_t mask = (1ULL << a.b) - 1ULL;
    int64_t carry = 0;
    uint64_t bits = 0;
    int nb = 0;
    if (a.out_kind == INV_U16) {
        uint16_t* out = reinterpret_cast<uint16_t*>(a.out);
        int w = 0;
        const long long o = (long long)row * a.ldo + col;
#pragma unroll
        for (int p = 0; p < (NB + 1) * S; ++p) {
            if (p < a.positions) {
                const int64_t v = pos_value(p) + carry;
                bits |= ((uint64_t)v & mask) << nb;
                nb += a.b;
                carry = v >> a.b;
                while (nb >= 16 && w < a.RL) {
                    out[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
                    bits >>= 16;
                    nb -= 16;
                    ++w;
                }
            }
        }
        while (w < a.RL) {
            const int need = 16 - nb;
            bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
            carry >>= need;
            out[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
            bits = 0;
            nb = 0;
            ++w;
        }
        return;
    }
    uint32_t words[INV_MAXW];
    int nw = 0;
#pragma unroll
    for (int p = 0; p < (NB + 1) * S; ++p) {
        if (p < a.positions) {
            const int64_t v = pos_value(p) + carry;
            bits |= ((uint64_t)v & mask) << nb;
            nb += a.b;
            carry = v >> a.b;
            if (nb >= 32) {
                if (nw < INV_MAXW) words[nw++] = (uint32_t)bits;
                bits >>= 32;
                nb -= 32;
            }
        }
    }
    for (int k = 0; k < 3 && nw < INV_MAXW; ++k) {
        const int need = 32 - nb;
        bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
        carry >>= need;
        words[nw++] = (uint32_t)bits;
        bits = 0;
        nb = 0;
    }
    store_float(a, (long long)row * a.ldo + col, words, nw);
}

// ---------------------------------------------------------------- lane variant
// For integer-output plans with K in {8, 16, 32} and NB <= 32 (the W = 256 and
// W = 1024 configurations).  K lanes own one element: lane c holds coefficient
// c of all NB transformed ring elements in registers, so the radix-2 DIT
// butterflies run in registers and each twiddle y^-e (a signed rotation of the
// coefficients) is one warp shuffle.  The CTA stages its E elements' NB*K
// values through shared memory first (coalesced 16-byte loads per plane).
//
// Carry propagation is split over the element's K lanes: lane s ripples the
// positions [s*SEG, (s+1)*SEG) with carry-in 0 (pass 1).  With D_s the
// segment's digits and M = SEG*b, the true carry-out is co_s + delta_s where
// delta_s = floor((D_s + ci_s) / 2^M) and ci_s = co_{s-1} + delta_{s-1} is the
// true carry-in.  Because every carry is below 2^(63-b) <= 2^(b*L) with
// L = floor(62/b) and each segment has more than L digits, delta_s is -1, 0
// or +1 and is fixed by the low L digits plus whether the higher digits are
// all ones / all zeros; each lane tabulates delta_s for delta_{s-1} in
// {-1, 0, 1} and a K-step shuffle chain resolves them.  Pass 2 ripples each
// segment again from its exact carry-in and emits its 16-bit limbs (segment
// boundaries sit on limb boundaries: SEG*b is a multiple of 16).
constexpr int INVL_THREADS = 256;

template <int LG>
__host__ __device__ constexpr int bitrev_c(int j) {
    int r = 0;
    for (int i = 0; i < LG; ++i) r |= ((j >> i) & 1) << (LG - 1 - i);
    return r;
}
__host__ __device__ constexpr int ilog2_c(int v) { return v <= 1 ? 0 : 1 + ilog2_c(v >> 1); }

// Shared-memory layouts of the lane kernel's carry stage, padded so that the
// K lanes of an element, each walking its own segment of positions / limbs,
// hit different banks (without the pad every lane of a 16-position segment
// maps position p to the same bank).  Fold buffer of a warp: [PMAX][EPW]
// int64 with one extra word per 16 positions; limb buffer: [RL][E] uint16
// with 8 extra limbs (16 bytes, keeping 16-byte vectors aligned) per 8 rows.
__host__ __device__ constexpr int invl_pidx(int p, int epw) { return p * epw + (p >> 4); }
__host__ __device__ constexpr int invl_pbw(int pmax, int epw) { return pmax * epw + (pmax >> 4) + 1; }
__host__ __device__ constexpr int invl_oidx(int w, int e) { return w * e + 8 * (w >> 3); }
__host__ __device__ constexpr int invl_obsize(int rl, int e) { return invl_oidx(rl, e) + 8; }

struct InvLaneGeom {
    int seg;   // positions per lane
    int pmax;  // (NB + 1) * S fold positions
};

__host__ __device__ inline int invl_seg(int positions, int K, int b) {
    const int L = 62 / b;
    int seg = (positions + K - 1) / K;
    if (seg < L + 1) seg = L + 1;
    int tz = 0;
    while (tz < 4 && !((b >> tz) & 1)) ++tz;
    const int m = 16 >> tz;  // SEG * b must be a multiple of 16
    return (seg + m - 1) / m * m;
}

// One radix-2 DIT stage of butterfly span LEN over the lane's NB values,
// then the next stage (compile-time recursion keeps every index constant).
template <int NB, int K, int LEN>
__device__ __forceinline__ void lane_dit(int64_t (&x)[NB], int c) {
    if constexpr (LEN <= NB) {
#pragma unroll
        for (int st = 0; st < NB; st += LEN) {
#pragma unroll
            for (int k = 0; k < LEN / 2; ++k) {
                const int e0 = (2 * K / LEN) * k;  // twiddle y^-(g (NB/LEN) k), e0 < K
                int64_t t = x[st + k + LEN / 2];
                if (e0 != 0) {
                    // (y^-e0 v)[c] = v[c + e0], negated when c + e0 wraps past K
                    t = __shfl_sync(0xffffffffu, t, (c + e0) & (K - 1), K);
                    if (c + e0 >= K) t = -t;
                }
                const int64_t u = x[st + k];
                x[st + k] = u + t;
                x[st + k + LEN / 2] = u - t;
            }
        }
        lane_dit<NB, K, 2 * LEN>(x, c);
    }
}

// RL: 16-bit limbs the carry stage emits per element (a.RL for INV_U16; for
// fp outputs enough limbs to hold the product plus its sign extension).
template <int NB, int K>
__global__ void __launch_bounds__(INVL_THREADS, 2) inverse_lane_kernel(const InvArgs a, int seg,
                                                                       int vec_out, int RL) {
    constexpr int EPW = 32 / K;                  // elements per warp
    constexpr int E = (INVL_THREADS / 32) * EPW;  // elements per CTA
    constexpr int NK = NB * K;
    constexpr int LD = E + 1;                    // odd stride: conflict-free column reads
    constexpr int VE = E / 4;
    constexpr int S = K / 2;
    constexpr int LGNB = ilog2_c(NB);
    constexpr int PMAX = (NB + 1) * S;
    constexpr unsigned FULL = 0xffffffffu;
    extern __shared__ int64_t sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long e_base = (long long)blockIdx.x * E;
    const long long total = (long long)a.rows * a.lda;
    const int ncls = a.nW * a.nchunk;
    // Karatsuba job planes (K = 8): 21 per point, staged as they are; the
    // P1 / P2 planes of the half points are never written and not loaded
    const bool kara = K == 8 && a.kara == 1;
    const int NQ = kara ? NB * 21 : NK;

    // ---- phase 1: stage [NQ][E] int64 = sum over digit classes w and chunks
    // of 2^(7w) * acc.  The planes of up to INVL_KB (class, chunk) pairs are
    // loaded together -- INVL_UB x INVL_KB 16-byte loads in flight per thread
    // -- and summed before one smem update per element.  Each thread revisits
    // only its own smem words across batches, so no barrier is needed between
    // them.
    constexpr int INVL_UB = 4, INVL_KB = 3;
    for (int k0 = 0; k0 < ncls; k0 += INVL_KB) {
        const int kn = ncls - k0 < INVL_KB ? ncls - k0 : INVL_KB;
        for (int idx0 = threadIdx.x; idx0 < NQ * VE; idx0 += INVL_UB * INVL_THREADS) {
            int4 r[INVL_UB][INVL_KB];
#pragma unroll
            for (int u = 0; u < INVL_UB; ++u) {
                const int idx = idx0 + u * INVL_THREADS;
                const int q = idx / VE, v = idx % VE;
                const long long e = e_base + 4 * v;
                bool live = idx < NQ * VE && e < total;
                if (kara) {
                    const int jq = q / 21;
                    live = live && (q % 21 < 7 || !(jq == 0 || 2 * jq == NB));
                }
#pragma unroll
                for (int kk = 0; kk < INVL_KB; ++kk) {
                    r[u][kk] = make_int4(0, 0, 0, 0);
                    if (live && kk < kn)
                        r[u][kk] = __ldg(reinterpret_cast<const int4*>(
                            a.acc + (long long)(q * ncls + k0 + kk) * a.acc_plane + e));
                }
            }
#pragma unroll
            for (int u = 0; u < INVL_UB; ++u) {
                const int idx = idx0 + u * INVL_THREADS;
                if (idx < NQ * VE) {
                    const int q = idx / VE, v = idx % VE;
                    int64_t* d = sm + q * LD + 4 * v;
                    int64_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
                    for (int kk = 0; kk < INVL_KB; ++kk) {
                        if (kk >= kn) break;
                        const int64_t f = inv_class_weight(a.dsum, (k0 + kk) / a.nchunk);
                        s0 += (int64_t)r[u][kk].x * f;
                        s1 += (int64_t)r[u][kk].y * f;
                        s2 += (int64_t)r[u][kk].z * f;
                        s3 += (int64_t)r[u][kk].w * f;
                    }
                    if (k0 == 0) {
                        d[0] = s0;
                        d[1] = s1;
                        d[2] = s2;
                        d[3] = s3;
                    } else {
                        d[0] += s0;
                        d[1] += s1;
                        d[2] += s2;
                        d[3] += s3;
                    }
                }
            }
        }
    }
    __syncthreads();

    // ---- phase 2: inverse DFT in registers, lane c = coefficient c
    const int es = lane / K, c = lane % K;
    const int ei = warp * EPW + es;
    int64_t x[NB];
    if (kara) {
        // coefficient c of Chat_j = P0 - P1 + y^4 (P2 - P0 - P1) mod y^8 + 1:
        // (P0 - P1)[c] + sign * M[c ^ 4], M = P2 - P0 - P1, sign -1 for c < 4
        // (the wrapped half), no M term for c = 3; half points: P0[c]
        const int cx = c ^ 4;
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const int64_t* pj = sm + (bitrev_c<LGNB>(j) * 21) * LD + ei;
            const bool half = bitrev_c<LGNB>(j) == 0 || 2 * bitrev_c<LGNB>(j) == NB;
            int64_t v = c < 7 ? pj[c * LD] : 0;
            if (!half) {
                if (c < 7) v -= pj[(7 + c) * LD];
                if (cx < 7) {
                    const int64_t Mx = pj[(14 + cx) * LD] - pj[cx * LD] - pj[(7 + cx) * LD];
                    v += c < 4 ? -Mx : Mx;
                }
            }
            x[j] = v;
        }
    } else {
#pragma unroll
        for (int j = 0; j < NB; ++j) x[j] = sm[(bitrev_c<LGNB>(j) * K + c) * LD + ei];  // DIT order
    }
    lane_dit<NB, K, 2>(x, c);
#pragma unroll
    for (int j = 0; j < NB; ++j) x[j] >>= LGNB;  // exact division by NB
    __syncthreads();  // staging reads done: the buffer is reused below

    // ---- fold: position beta*S + c (c < S) = C_beta[c] + C_{beta-1}[c + S]
    constexpr int PBW = invl_pbw(PMAX, EPW);
    int64_t* pb = sm + (long long)warp * PBW;  // this warp's [PMAX][EPW], padded
#pragma unroll
    for (int beta = 0; beta <= NB; ++beta) {
        const int64_t hi = beta >= 1 ? __shfl_down_sync(FULL, x[beta - 1], S, K) : 0;
        const int64_t lo = beta < NB ? x[beta] : 0;
        if (c < S) pb[invl_pidx(beta * S + c, EPW) + es] = lo + hi;
    }
    __syncwarp();

    // ---- carry: segment c of the element, two passes and a +-1 chain
    const int P = a.positions, b = a.b, L = 62 / b;
    const int64_t mask = (int64_t)((1ULL << b) - 1ULL);
    const int p0 = c * seg;
    const int p1 = min(P, p0 + seg);
    const int64_t* mine = pb + es;
    int64_t carry = 0, dlo = 0;
    bool ones = true, zeros = true;
    for (int p = p0, i = 0; p < p1; ++p, ++i) {
        const int64_t v = mine[invl_pidx(p, EPW)] + carry;
        const int64_t d = v & mask;
        carry = v >> b;
        if (i < L) {
            dlo |= d << (b * i);
        } else {
            ones &= d == mask;
            zeros &= d == 0;
        }
    }
    int64_t co_prev = __shfl_up_sync(FULL, carry, 1, K);
    if (c == 0) co_prev = 0;
    int tab = 0;
#pragma unroll
    for (int xi = 0; xi < 3; ++xi) {
        const int64_t sum = dlo + co_prev + (xi - 1);
        const int64_t q = sum >> (b * L);
        const int d = q >= 1 ? (ones ? 1 : 0) : (q <= -1 ? (zeros ? -1 : 0) : 0);
        tab |= (d + 1) << (2 * xi);
    }
    int delta = 0, delta_prev = 0;
#pragma unroll
    for (int s = 1; s < K; ++s) {
        const int t = __shfl_sync(FULL, tab, s, K);
        if (c == s) delta_prev = delta;
        delta = ((t >> (2 * (delta + 1))) & 3) - 1;
    }
    carry = c == 0 ? 0 : co_prev + delta_prev;

    uint16_t* ob = reinterpret_cast<uint16_t*>(sm + (long long)(INVL_THREADS / 32) * PBW);  // [RL][E]
    int w = p0 * b / 16;
    uint64_t bits = 0;
    int nb = 0;
    for (int p = p0; p < p1; ++p) {
        const int64_t v = mine[invl_pidx(p, EPW)] + carry;
        bits |= ((uint64_t)v & (uint64_t)mask) << nb;
        nb += b;
        carry = v >> b;
        while (nb >= 16) {
            if (w < RL) ob[invl_oidx(w, E) + ei] = (uint16_t)(bits & 0xFFFFu);
            bits >>= 16;
            nb -= 16;
            ++w;
        }
    }
    if (p0 < P && p1 == P) {  // the top segment: sign-extend from the final carry
        while (w < RL) {
            const int need = 16 - nb;
            bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
            carry >>= need;
            ob[invl_oidx(w, E) + ei] = (uint16_t)(bits & 0xFFFFu);
            bits = 0;
            nb = 0;
            ++w;
        }
    }
    __syncthreads();

    if (a.out_kind == INV_F32 || a.out_kind == INV_F64) {
        // one thread per element: the limbs as 32-bit words, rounded once
        if (threadIdx.x >= E) return;
        const long long e = e_base + threadIdx.x;
        if (e >= total) return;
        const int row = (int)(e / a.lda), col = (int)(e % a.lda);
        if (row >= a.rows || col >= a.cols) return;
        uint32_t words[INV_MAXW];
        const int nw = RL / 2;
        for (int k = 0; k < nw; ++k)
            words[k] = (uint32_t)ob[invl_oidx(2 * k, E) + threadIdx.x] |
                       ((uint32_t)ob[invl_oidx(2 * k + 1, E) + threadIdx.x] << 16);
        store_float(a, (long long)row * a.ldo + col, words, nw);
        return;
    }

    // ---- store the CTA's limbs, plane by plane
    uint16_t* out = reinterpret_cast<uint16_t*>(a.out);
    if (vec_out) {  // element e is output index e: 16-byte stores of 8 elements
        for (int idx = threadIdx.x; idx < RL * (E / 8); idx += INVL_THREADS) {
            const int wv = idx / (E / 8), v = idx % (E / 8);
            const long long e = e_base + 8 * v;
            if (e < total)
                *reinterpret_cast<uint4*>(out + (long long)wv * a.out_plane + e) =
                    *reinterpret_cast<const uint4*>(ob + invl_oidx(wv, E) + 8 * v);
        }
    } else {
        for (int idx = threadIdx.x; idx < RL * E; idx += INVL_THREADS) {
            const int wv = idx / E, i = idx % E;
            const long long e = e_base + i;
            if (e >= total) continue;
            const int row = (int)(e / a.lda), col = (int)(e % a.lda);
            if (row >= a.rows || col >= a.cols) continue;
            out[(long long)wv * a.out_plane + (long long)row * a.ldo + col] = ob[invl_oidx(wv, E) + i];
        }
    }
}

template <int NB, int K>
static int launch_lane(const InvArgs& a, cudaStream_t stream) {
    constexpr int E = (INVL_THREADS / 32) * (32 / K);
    constexpr int PMAX = (NB + 1) * (K / 2);
    // fp outputs: the product's limbs plus 64 bits of sign extension, in whole
    // 32-bit words (the register and generic kernels append the same margin)
    int RL = a.RL;
    if (a.out_kind == INV_F32 || a.out_kind == INV_F64) {
        RL = ((a.positions * a.b + 15) / 16 + 4 + 1) / 2 * 2;
        if (RL > 2 * INV_MAXW) return MFFTB_ERR_UNSUPPORTED;
    }
    const size_t stage = (size_t)(a.kara == 1 ? NB * 21 : NB * K) * (E + 1) * sizeof(int64_t);
    const size_t carry = (size_t)(INVL_THREADS / 32) * invl_pbw(PMAX, 32 / K) * sizeof(int64_t) +
                         (size_t)invl_obsize(RL, E) * sizeof(uint16_t);
    const size_t smem = (stage > carry ? stage : carry + 16);
    if (smem > 200 * 1024) return MFFTB_ERR_UNSUPPORTED;
    static int attr_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev != dev) {
        if (cudaFuncSetAttribute(inverse_lane_kernel<NB, K>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 200 * 1024) != cudaSuccess)
            return MFFTB_ERR_CUDA;
        attr_dev = dev;
    }
    const int seg = invl_seg(a.positions, K, a.b);
    const long long total = (long long)a.rows * a.lda;
    const int vec_out = a.lda == a.ldo && a.cols == a.lda && a.lda % 8 == 0 &&
                        a.out_plane % 8 == 0 && reinterpret_cast<uintptr_t>(a.out) % 16 == 0;
    const long long blocks = (total + E - 1) / E;
    if (blocks > 0)
        inverse_lane_kernel<NB, K><<<(unsigned)blocks, INVL_THREADS, smem, stream>>>(a, seg, vec_out,
                                                                                 RL);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

// MFFTB_ERR_UNSUPPORTED when the lane variant does not cover the plan
static int try_lane(const InvArgs& a, cudaStream_t stream) {
    if (a.out_kind == INV_I64) return MFFTB_ERR_UNSUPPORTED;
    if (a.kara && (a.kara != 1 || a.K != 8 || a.nW != 1 || a.nchunk != 1))
        return MFFTB_ERR_UNSUPPORTED;
    if (a.positions > (a.NB + 1) * a.S || a.b < 2 || a.b > 15) return MFFTB_ERR_UNSUPPORTED;
    if (a.lda % 4 || a.acc_plane % 4 || reinterpret_cast<uintptr_t>(a.acc) % 16)
        return MFFTB_ERR_UNSUPPORTED;
    if (invl_seg(a.positions, a.K, a.b) * a.K < a.positions) return MFFTB_ERR_UNSUPPORTED;
#define INVL_CASE(nb, k) \
    if (a.NB == nb && a.K == k) return launch_lane<nb, k>(a, stream);
    INVL_CASE(8, 8) INVL_CASE(16, 8) INVL_CASE(32, 8)
    INVL_CASE(4, 16) INVL_CASE(8, 16) INVL_CASE(16, 16) INVL_CASE(32, 16)
    INVL_CASE(4, 32) INVL_CASE(8, 32) INVL_CASE(16, 32) INVL_CASE(32, 32)
#undef INVL_CASE
    return MFFTB_ERR_UNSUPPORTED;
}

template <int NB, int K, int KARA = 0>
static int launch_reg(const InvArgs& a, cudaStream_t stream) {
    const long long total = (long long)a.rows * a.lda;
    const long long blocks = (total + 127) / 128;
    if (blocks > 0) inverse_reg_kernel<NB, K, KARA><<<(unsigned)blocks, 128, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

template <int NB>
static int launch_reg_kara(const InvArgs& a, cudaStream_t stream) {
    if (a.kara == 3) return launch_reg<NB, 8, 3>(a, stream);
    return a.kara == 2 ? launch_reg<NB, 8, 2>(a, stream) : launch_reg<NB, 8, 1>(a, stream);
}

static int school_carry_launch(const InvArgs& a, cudaStream_t stream);

int inverse_launch(const InvArgs& a, cudaStream_t stream) {
    if (a.school) return school_carry_launch(a, stream);
    if (a.kara) {
        if (a.K != 8 || a.nW != 1 || a.nchunk != 1 || a.positions > (a.NB + 1) * a.S ||
            a.kara > 3)
            return MFFTB_ERR_ARG;
        if (a.variant == 2) {
            const int rc = try_lane(a, stream);
            if (rc != MFFTB_ERR_UNSUPPORTED) return rc;
        }
        if (a.NB == 8) return launch_reg_kara<8>(a, stream);
        if (a.NB == 4) return launch_reg_kara<4>(a, stream);
        if (a.NB == 2) return launch_reg_kara<2>(a, stream);
        return MFFTB_ERR_ARG;
    }
    const int NK = a.NB * a.K;
    if (a.elems < 1 || a.elems > 32 || NK * a.elems > INV_VPT * INV_THREADS) return MFFTB_ERR_ARG;
    if ((1 << a.log2NB) != a.NB || (1 << a.lgS) != a.S || (1 << a.lgK) != a.K ||
        (1 << a.lgE) != a.elems)
        return MFFTB_ERR_ARG;
    if ((a.out_kind == INV_F32 || a.out_kind == INV_F64) &&
        (long long)a.positions * a.b + 96 > 32LL * INV_MAXW)
        return MFFTB_ERR_UNSUPPORTED;
    if (a.variant == 2) {  // the lane kernel first where it covers the plan
        const int rc = try_lane(a, stream);
        if (rc != MFFTB_ERR_UNSUPPORTED) return rc;
    }
    if (a.positions <= (a.NB + 1) * a.S) {
        if (a.NB == 8 && a.K == 8) return launch_reg<8, 8>(a, stream);
        if (a.NB == 4 && a.K == 4) return launch_reg<4, 4>(a, stream);
        if (a.NB == 8 && a.K == 4) return launch_reg<8, 4>(a, stream);
        if (a.NB == 4 && a.K == 8) return launch_reg<4, 8>(a, stream);
        if (a.NB == 2 && a.K == 4) return launch_reg<2, 4>(a, stream);
        if (a.NB == 2 && a.K == 2) return launch_reg<2, 2>(a, stream);
        if (a.NB == 4 && a.K == 2) return launch_reg<4, 2>(a, stream);
        if (a.NB == 2 && a.K == 8) return launch_reg<2, 8>(a, stream);
        if (a.NB == 4 && a.K == 16) return launch_reg<4, 16>(a, stream);
        if (a.NB == 2 && a.K == 16) return launch_reg<2, 16>(a, stream);
        if (a.NB == 2 && a.K == 32) return launch_reg<2, 32>(a, stream);
    }
    if (a.variant != 1) {
        const int rc = try_lane(a, stream);
        if (rc != MFFTB_ERR_UNSUPPORTED) return rc;
    }
    const size_t smem = (size_t)NK * a.elems * sizeof(int64_t);
    if (smem > 200 * 1024) return MFFTB_ERR_ARG;
    static size_t attr = 0;
    if (smem > 48 * 1024 && smem > attr) {
        if (cudaFuncSetAttribute(inverse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(200 * 1024)) != cudaSuccess)
            return MFFTB_ERR_CUDA;
        attr = 200 * 1024;
    }
    const long long total = (long long)a.rows * a.lda;
    const long long blocks = (total + a.elems - 1) / a.elems;
    if (blocks <= 0) return MFFTB_OK;
    inverse_kernel<<<(unsigned)blocks, INV_THREADS, smem, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

// ---------------------------------------------------------------- schoolbook carry
// Schoolbook plans have no transform: position t of the product is
// C_t = sum over the live chunks of job plane (t, ch).  One thread per
// element streams the positions (coalesced across the warp), carries in
// radix 2^b and formats the output as the other inverse kernels do.
constexpr int SC_THREADS = 256;
constexpr int SC_UNROLL = 8;

__device__ __forceinline__ bool school_live(const InvArgs& a, int t, int ch) {
    int lo = ch * a.U;
    if (t - (a.LbB - 1) > lo) lo = t - (a.LbB - 1);
    int hi = ch * a.U + a.U - 1;
    if (t < hi) hi = t;
    if (a.LbA - 1 < hi) hi = a.LbA - 1;
    return lo <= hi;
}

__global__ void __launch_bounds__(SC_THREADS) school_carry_kernel(const InvArgs a) {
    const long long e = blockIdx.x * (long long)SC_THREADS + threadIdx.x;
    const long long total = (long long)a.rows * a.lda;
    if (e >= total) return;
    const int row = (int)(e / a.lda), col = (int)(e % a.lda);
    if (row >= a.rows || col >= a.cols) return;
    const long long o = (long long)row * a.ldo + col;
    const int P = a.positions, b = a.b;
    const uint64_t mask = (1ULL << b) - 1ULL;
    int64_t carry = 0;
    uint64_t bits = 0;
    int nb = 0, w = 0;
    uint32_t words[INV_MAXW];
    int nw = 0;
    uint16_t* out16 = reinterpret_cast<uint16_t*>(a.out);
    for (int t0 = 0; t0 < P; t0 += SC_UNROLL) {
        int64_t v[SC_UNROLL];
#pragma unroll
        for (int i = 0; i < SC_UNROLL; ++i) {
            v[i] = 0;
            const int t = t0 + i;
            if (t < P)
                for (int ch = 0; ch < a.nchunk; ++ch)
                    if (school_live(a, t, ch))
                        v[i] += __ldg(a.acc + (long long)(t * a.nchunk + ch) * a.acc_plane + e);
        }
#pragma unroll
        for (int i = 0; i < SC_UNROLL; ++i) {
            if (t0 + i >= P) break;
            const int64_t x = v[i] + carry;
            bits |= ((uint64_t)x & mask) << nb;
            nb += b;
            carry = x >> b;
            if (a.out_kind == INV_U16) {
                while (nb >= 16 && w < a.RL) {
                    out16[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
                    bits >>= 16;
                    nb -= 16;
                    ++w;
                }
                if (nb >= 16) {  // past RL: drop the bits
                    bits >>= 16;
                    nb -= 16;
                }
            } else if (nb >= 32) {
                if (nw < INV_MAXW) words[nw++] = (uint32_t)bits;
                bits >>= 32;
                nb -= 32;
            }
        }
    }
    if (a.out_kind == INV_U16) {
        while (w < a.RL) {
            const int need = 16 - nb;
            bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
            carry >>= need;
            out16[(long long)w * a.out_plane + o] = (uint16_t)(bits & 0xFFFFu);
            bits = 0;
            nb = 0;
            ++w;
        }
        return;
    }
    for (int k = 0; k < 3 && nw < INV_MAXW; ++k) {
        const int need = 32 - nb;
        bits |= ((uint64_t)carry & ((1ULL << need) - 1ULL)) << nb;
        carry >>= need;
        words[nw++] = (uint32_t)bits;
        bits = 0;
        nb = 0;
    }
    store_float(a, o, words, nw);
}

// Integer output, 4 consecutive elements per thread: 16-byte loads of every
// job plane (512 contiguous bytes per warp and plane) and 8-byte limb stores.
constexpr int SC4_UNROLL = 4;

__global__ void __launch_bounds__(SC_THREADS) school_carry4_kernel(const InvArgs a, int vec_out) {
    const long long e = (blockIdx.x * (long long)SC_THREADS + threadIdx.x) * 4;
    const long long total = (long long)a.rows * a.lda;
    if (e >= total) return;
    const int row = (int)(e / a.lda), col = (int)(e % a.lda);  // lda % 4 == 0: one row
    if (row >= a.rows || col >= a.cols) return;
    const int P = a.positions, b = a.b;
    const uint64_t mask = (1ULL << b) - 1ULL;
    int64_t carry[4] = {0, 0, 0, 0};
    uint64_t bits[4] = {0, 0, 0, 0};
    int nb = 0, w = 0;  // same for the 4 elements
    uint16_t* out16 = reinterpret_cast<uint16_t*>(a.out);
    const long long o = (long long)row * a.ldo + col;
    const bool full = vec_out && col + 3 < a.cols;
    auto store = [&](int wv, const uint16_t (&h)[4]) {
        uint16_t* dst = out16 + (long long)wv * a.out_plane + o;
        if (full) {
            ushort4 q;
            q.x = h[0];
            q.y = h[1];
            q.z = h[2];
            q.w = h[3];
            *reinterpret_cast<ushort4*>(dst) = q;
        } else {
            for (int i = 0; i < 4; ++i)
                if (col + i < a.cols) dst[i] = h[i];
        }
    };
    for (int t0 = 0; t0 < P; t0 += SC4_UNROLL) {
        int64_t v[SC4_UNROLL][4];
#pragma unroll
        for (int u = 0; u < SC4_UNROLL; ++u) {
            v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0;
            const int t = t0 + u;
            if (t < P)
                for (int ch = 0; ch < a.nchunk; ++ch)
                    if (school_live(a, t, ch)) {
                        const int4 r = __ldg(reinterpret_cast<const int4*>(
                            a.acc + (long long)(t * a.nchunk + ch) * a.acc_plane + e));
                        v[u][0] += r.x;
                        v[u][1] += r.y;
                        v[u][2] += r.z;
                        v[u][3] += r.w;
                    }
        }
#pragma unroll
        for (int u = 0; u < SC4_UNROLL; ++u) {
            if (t0 + u >= P) break;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t x = v[u][i] + carry[i];
                bits[i] |= ((uint64_t)x & mask) << nb;
                carry[i] = x >> b;
            }
            nb += b;
            while (nb >= 16) {
                if (w < a.RL) {
                    uint16_t h[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) h[i] = (uint16_t)(bits[i] & 0xFFFFu);
                    store(w, h);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) bits[i] >>= 16;
                nb -= 16;
                ++w;
            }
        }
    }
    while (w < a.RL) {  // sign-extend from the final carries
        const int need = 16 - nb;
        uint16_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            bits[i] |= ((uint64_t)carry[i] & ((1ULL << need) - 1ULL)) << nb;
            carry[i] >>= need;
            h[i] = (uint16_t)(bits[i] & 0xFFFFu);
            bits[i] = 0;
        }
        store(w, h);
        nb = 0;
        ++w;
    }
}

static int school_carry_launch(const InvArgs& a, cudaStream_t stream) {
    if (a.out_kind == INV_I64) return MFFTB_ERR_UNSUPPORTED;
    if (a.out_kind == INV_U16 && a.lda % 4 == 0 && a.acc_plane % 4 == 0 &&
        reinterpret_cast<uintptr_t>(a.acc) % 16 == 0 && a.b >= 1 && a.b <= 15 && a.nchunk >= 1 &&
        a.U >= 1) {
        const int vec_out = a.ldo % 4 == 0 && a.out_plane % 4 == 0 &&
                            reinterpret_cast<uintptr_t>(a.out) % 8 == 0;
        const long long total4 = ((long long)a.rows * a.lda) / 4;
        const long long blocks = (total4 + SC_THREADS - 1) / SC_THREADS;
        if (blocks > 0) school_carry4_kernel<<<(unsigned)blocks, SC_THREADS, 0, stream>>>(a, vec_out);
        return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
    }
    if (a.b < 1 || a.b > 15 || a.nchunk < 1 || a.U < 1) return MFFTB_ERR_ARG;
    if ((a.out_kind == INV_F32 || a.out_kind == INV_F64) &&
        (long long)a.positions * a.b + 96 > 32LL * INV_MAXW)
        return MFFTB_ERR_UNSUPPORTED;
    const long long total = (long long)a.rows * a.lda;
    const long long blocks = (total + SC_THREADS - 1) / SC_THREADS;
    if (blocks > 0) school_carry_kernel<<<(unsigned)blocks, SC_THREADS, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

// ---------------------------------------------------------------- fp32 exponent scan
__device__ __forceinline__ int frexp_e(float x) {
    int e;
    frexpf(x, &e);
    return e;
}
__device__ __forceinline__ int frexp_e(double x) {
    int e;
    frexp(x, &e);
    return e;
}

template <typename T, int SIG>
__global__ void scan_fp_kernel(const T* X, long long count, int* out3) {
    int lo = 1 << 30, hi = -(1 << 30), any = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        T x = __ldg(X + i);
        if (x == (T)0 || !isfinite(x)) continue;
        int e2 = frexp_e(x) - SIG;
        lo = min(lo, e2);
        hi = max(hi, e2);
        any = 1;
    }
    for (int o = 16; o > 0; o >>= 1) {
        lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        any |= __shfl_xor_sync(0xffffffffu, any, o);
    }
    if ((threadIdx.x & 31) == 0 && any) {
        atomicMin(out3 + 0, lo);
        atomicMax(out3 + 1, hi);
        atomicOr(out3 + 2, 1);
    }
}

template <typename T, int SIG>
static int scan_launch(const T* X, long long count, int* out3, cudaStream_t stream) {
    int init[3] = {1 << 30, -(1 << 30), 0};
    if (cudaMemcpyAsync(out3, init, sizeof init, cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return MFFTB_ERR_CUDA;
    long long blocks = (count + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    scan_fp_kernel<T, SIG><<<(unsigned)blocks, 256, 0, stream>>>(X, count, out3);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int scan_f32_launch(const float* X, long long count, int* out3, cudaStream_t stream) {
    return scan_launch<float, 24>(X, count, out3, stream);
}
int scan_f64_launch(const double* X, long long count, int* out3, cudaStream_t stream) {
    return scan_launch<double, 53>(X, count, out3, stream);
}

float decode_words_host(uint32_t* w, int nw, int bit_off, int S) {
    return decode_words_f32(w, nw, bit_off, S);
}
double decode_words_host_f64(uint32_t* w, int nw, int bit_off, int S) {
    return decode_words_f64(w, nw, bit_off, S);
}

}  // namespace mfftb
