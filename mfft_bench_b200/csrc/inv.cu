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
//   * INV_F32: extract + round_to + ldexpf of fpx_decode_f32
//     (src/fpfixed.c:212-285), see decode.cuh.
//
// A CTA owns E consecutive elements (E <= 32) and keeps their NB*K int64
// transformed values in shared memory; 256 threads cooperate on the loads
// and on the inverse DFT, then E threads fold and carry one element each.
#include <cuda_runtime.h>

#include <cstdint>

#include "decode.cuh"
#include "kernels.h"
#include "runtime.h"

namespace mfftb {

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
                v += s * ((int64_t)1 << (7 * w));
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
    float* out = reinterpret_cast<float*>(a.out);
    out[(long long)row * a.ldo + col] = decode_words_f32(words, nw, a.bit_off, a.S_scale);
}

// ---------------------------------------------------------------- register variant
// For plans with NB*K <= 64 (the W=64 and fp32 configurations) one thread
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

template <int NB, int K>
__global__ void __launch_bounds__(128) inverse_reg_kernel(const InvArgs a) {
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
                    v += s * ((int64_t)1 << (7 * w));
                }
                x[bitrev(j)][t] = v;
            }
        }
    }
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
    float* out = reinterpret_cast<float*>(a.out);
    out[(long long)row * a.ldo + col] = decode_words_f32(words, nw, a.bit_off, a.S_scale);
}

template <int NB, int K>
static int launch_reg(const InvArgs& a, cudaStream_t stream) {
    const long long total = (long long)a.rows * a.lda;
    const long long blocks = (total + 127) / 128;
    if (blocks > 0) inverse_reg_kernel<NB, K><<<(unsigned)blocks, 128, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int inverse_launch(const InvArgs& a, cudaStream_t stream) {
    const int NK = a.NB * a.K;
    if (a.elems < 1 || a.elems > 32 || NK * a.elems > INV_VPT * INV_THREADS) return MFFTB_ERR_ARG;
    if ((1 << a.log2NB) != a.NB || (1 << a.lgS) != a.S || (1 << a.lgK) != a.K ||
        (1 << a.lgE) != a.elems)
        return MFFTB_ERR_ARG;
    if (a.out_kind == INV_F32 && (long long)a.positions * a.b + 96 > 32LL * INV_MAXW)
        return MFFTB_ERR_UNSUPPORTED;
    if (a.positions <= (a.NB + 1) * a.S) {
        if (a.NB == 8 && a.K == 8) return launch_reg<8, 8>(a, stream);
        if (a.NB == 4 && a.K == 4) return launch_reg<4, 4>(a, stream);
        if (a.NB == 8 && a.K == 4) return launch_reg<8, 4>(a, stream);
        if (a.NB == 4 && a.K == 8) return launch_reg<4, 8>(a, stream);
        if (a.NB == 2 && a.K == 4) return launch_reg<2, 4>(a, stream);
        if (a.NB == 2 && a.K == 2) return launch_reg<2, 2>(a, stream);
        if (a.NB == 4 && a.K == 2) return launch_reg<4, 2>(a, stream);
        if (a.NB == 2 && a.K == 8) return launch_reg<2, 8>(a, stream);
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

// ---------------------------------------------------------------- fp32 exponent scan
__global__ void scan_f32_kernel(const float* X, long long count, int* out3) {
    int lo = 1 << 30, hi = -(1 << 30), any = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        float x = __ldg(X + i);
        if (x == 0.0f || !isfinite(x)) continue;
        int e;
        frexpf(x, &e);
        int e2 = e - 24;
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

int scan_f32_launch(const float* X, long long count, int* out3, cudaStream_t stream) {
    int init[3] = {1 << 30, -(1 << 30), 0};
    if (cudaMemcpyAsync(out3, init, sizeof init, cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return MFFTB_ERR_CUDA;
    long long blocks = (count + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    scan_f32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(X, count, out3);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

float decode_words_host(uint32_t* w, int nw, int bit_off, int S) {
    return decode_words_f32(w, nw, bit_off, S);
}

}  // namespace mfftb
