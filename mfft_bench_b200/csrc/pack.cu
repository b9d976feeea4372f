// pack.cu -- Kernel 1: split matrix entries into signed digit planes.
//
// Reference semantics: the entry-to-limb-plane layout of src/mfftbench.h:74-82
// (plane-major, limbs LSB first), the widening in mm_mfft (src/mfft.c:433-434),
// the signed limb convention and the fp32 grid encoding of src/fpfixed.c:
// 175-193.  The B200 path re-radixes every entry into b-bit digits (b <= 8)
// so a transformed coefficient fits a small number of int8 tensor-core
// digits:
//   * integers (u16 limb planes, int64): digit m is the bit field
//     [m*b, m*b+b) of the two's complement value; the top digit is
//     sign-extended, all others are unsigned.  Local bit extraction, no carry
//     chain, identical value.
//   * fp32: digit m of |x| * 2^(off - lo_bit) (the entry's position on the
//     fixed-point grid relative to the live window), times sign(x).
//   * limb mode (conv_mfft): the caller's int32 limbs are the digits.
// Output planes are [Lb][rows][ld] (row r of the operand, contraction index
// contiguous), int8 for b <= 7 and int16 for wider digits.  B is written transposed (row = output column) so both GEMM
// operands are K-major.  Rows/columns beyond n are zero.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "runtime.h"

namespace mfftb {

// ---------------------------------------------------------------- digit of one entry
__device__ __forceinline__ int digit_u16pl(const uint16_t* src, long long nn, long long idx, int L,
                                           int m, int b, int W, int is_signed) {
    const int p = m * b;
    const int u = p >> 4, sh = p & 15;
    const uint32_t lo = u < L ? __ldg(src + (long long)u * nn + idx) : 0u;
    const uint32_t hi = (u + 1) < L ? __ldg(src + (long long)(u + 1) * nn + idx) : 0u;
    const uint32_t v = ((hi << 16) | lo) >> sh;
    if (is_signed && p + b >= W) {
        // top digit: bits [p, W) sign-extended (W - p is in [1, b])
        const int keep = W - p;
        return (int32_t)(v << (32 - keep)) >> (32 - keep);
    }
    return (int)(v & ((1u << b) - 1u));
}

__device__ __forceinline__ int digit_f32(float x, int m, int b, int S_grid, int lo_bit,
                                         int trunc_rel) {
    if (x == 0.0f || !isfinite(x)) return 0;
    int e;
    float mf = frexpf(x, &e);
    uint32_t mi = (uint32_t)(fabsf(mf) * 16777216.0f);
    int off = e - 24 + S_grid;
    if (off < 0) return 0;                // below the grid (src/fpfixed.c:184)
    const int rel = off - lo_bit;         // >= 0 by construction of lo_bit
    const int p = m * b;
    int lim = trunc_rel - p;              // bits of this digit inside the grid
    if (lim <= 0) return 0;
    uint64_t field;
    if (p >= rel) {
        int s = p - rel;
        field = s >= 24 ? 0 : ((uint64_t)mi >> s);
    } else {
        int s = rel - p;
        field = s >= b ? 0 : ((uint64_t)mi << s);
    }
    uint32_t mask = lim >= b ? ((1u << b) - 1u) : ((1u << lim) - 1u);
    int d = (int)(field & mask);
    return x < 0.0f ? -d : d;
}

// fp64 on the same grid (encode_one_d, src/fpfixed.c:141-160): the 53-bit
// significand mi = |m| * 2^53 placed at bit off = e - 53 + S, bits at or above
// the grid top dropped, digit m of the window starting at lo_bit.
__device__ __forceinline__ int digit_f64(double x, int m, int b, int S_grid, int lo_bit,
                                         int trunc_rel) {
    if (x == 0.0 || !isfinite(x)) return 0;
    int e;
    double mf = frexp(x, &e);
    const uint64_t mi = (uint64_t)(fabs(mf) * 9007199254740992.0);  // 2^53, exact
    const int off = e - 53 + S_grid;
    if (off < 0) return 0;                // below the grid (src/fpfixed.c:149)
    const int rel = off - lo_bit;
    const int p = m * b;
    const int lim = trunc_rel - p;
    if (lim <= 0) return 0;
    uint64_t field;
    if (p >= rel) {
        const int s = p - rel;
        field = s >= 53 ? 0 : (mi >> s);
    } else {
        const int s = rel - p;            // only the low b - s bits of mi reach the field
        field = s >= b ? 0 : ((mi & ((1ull << (b - s)) - 1ull)) << s);
    }
    const uint64_t mask = lim >= b ? ((1ull << b) - 1ull) : ((1ull << lim) - 1ull);
    const int d = (int)(field & mask);
    return x < 0.0 ? -d : d;
}

template <int FMT>
__device__ __forceinline__ int entry_digit(const PackArgs& a, int i, int j, int m) {
    if (i < 0 || i >= a.n || j >= a.n) return 0;
    const long long idx = (long long)i * a.n + j;
    if (FMT == PACK_U16PL) {
        return digit_u16pl(reinterpret_cast<const uint16_t*>(a.src), (long long)a.n * a.n, idx,
                           a.L16, m, a.b, a.W, a.is_signed);
    } else if (FMT == PACK_I64) {
        int64_t x = __ldg(reinterpret_cast<const long long*>(a.src) + idx);
        const int p = m * a.b;
        if (p + a.b >= a.W) {
            // top digit: bits [p, W) sign-extended (W <= 64)
            int64_t t = (int64_t)((uint64_t)x << (64 - a.W)) >> (64 - a.W);
            return (int)(t >> p);
        }
        return (int)(((uint64_t)x >> p) & ((1u << a.b) - 1u));
    } else if (FMT == PACK_F64) {
        double x = __ldg(reinterpret_cast<const double*>(a.src) + idx);
        return digit_f64(x, m, a.b, a.S_grid, a.lo_bit, a.trunc_rel);
    } else {
        float x = __ldg(reinterpret_cast<const float*>(a.src) + idx);
        return digit_f32(x, m, a.b, a.S_grid, a.lo_bit, a.trunc_rel);
    }
}

// 32x32 element tile, PACK_MCH digit planes per block.  Straight: out row =
// source row.  Transposed: out row = source column (B^T for the GEMM).
constexpr int PACK_MCH = 8;

template <int FMT, bool TRANSPOSE, typename OT>
__global__ void __launch_bounds__(256) pack_digits_kernel(const PackArgs a) {
    __shared__ OT tile[PACK_MCH][32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;     // output tile origin
    const int m0 = blockIdx.z * PACK_MCH;
    const int mcount = a.Lb - m0 < PACK_MCH ? a.Lb - m0 : PACK_MCH;
    OT* out = reinterpret_cast<OT*>(a.dst);
    if (!TRANSPOSE) {
        for (int q = 0; q < 4; ++q) {
            const int r = r0 + ty + 8 * q, c = c0 + tx;
            if (r >= a.rows || c >= a.ld) continue;
            for (int mm = 0; mm < mcount; ++mm) {
                int d = entry_digit<FMT>(a, a.row0 + r, c, m0 + mm);
                out[(long long)(m0 + mm) * a.plane + (long long)r * a.ld + c] = (OT)d;
            }
        }
    } else {
        // source element (i = c0 + ty + 8q [contraction index k], j = r0 + tx [output column])
        for (int q = 0; q < 4; ++q) {
            const int i = c0 + ty + 8 * q, j = r0 + tx;
            for (int mm = 0; mm < mcount; ++mm)
                tile[mm][ty + 8 * q][tx] = (OT)entry_digit<FMT>(a, i, j, m0 + mm);
        }
        __syncthreads();
        for (int q = 0; q < 4; ++q) {
            const int r = r0 + ty + 8 * q, c = c0 + tx;  // out row = j, out col = i
            if (r >= a.rows || c >= a.ld) continue;
            for (int mm = 0; mm < mcount; ++mm)
                out[(long long)(m0 + mm) * a.plane + (long long)r * a.ld + c] = tile[mm][tx][ty + 8 * q];
        }
    }
}

// Limb mode: int32 limb planes [L][n][n] -> int32 digit planes, range-checked
// (|limb| <= 65535 is the documented input contract of conv_mfft).
template <bool TRANSPOSE>
__global__ void __launch_bounds__(256) pack_limbs_kernel(const PackArgs a) {
    __shared__ int32_t tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32, m = blockIdx.z;
    const int32_t* src = reinterpret_cast<const int32_t*>(a.src) + (long long)m * a.n * a.n;
    int32_t* out = reinterpret_cast<int32_t*>(a.dst) + (long long)m * a.plane;
    bool bad = false;
    if (!TRANSPOSE) {
        for (int q = 0; q < 4; ++q) {
            const int r = r0 + ty + 8 * q, c = c0 + tx;
            if (r >= a.rows || c >= a.ld) continue;
            const int i = a.row0 + r;
            int32_t v = (i < a.n && c < a.n) ? __ldg(src + (long long)i * a.n + c) : 0;
            if (v > 65535 || v < -65535) bad = true;
            out[(long long)r * a.ld + c] = v;
        }
    } else {
        for (int q = 0; q < 4; ++q) {
            const int i = c0 + ty + 8 * q, j = r0 + tx;
            int32_t v = (i < a.n && j < a.n) ? __ldg(src + (long long)i * a.n + j) : 0;
            if (v > 65535 || v < -65535) bad = true;
            tile[ty + 8 * q][tx] = v;
        }
        __syncthreads();
        for (int q = 0; q < 4; ++q) {
            const int r = r0 + ty + 8 * q, c = c0 + tx;
            if (r >= a.rows || c >= a.ld) continue;
            out[(long long)r * a.ld + c] = tile[tx][ty + 8 * q];
        }
    }
    if (bad) atomicCAS(a.err, 0, MFFTB_ERR_RANGE);
}

// int64 entries into int8 digit planes, 4 digits per 32-bit store.
// Straight (A): a thread owns 4 consecutive columns of one row.
// Transposed (B): a 64 x 64 tile of entries is staged in shared memory and a
// thread emits 4 consecutive contraction indices of one output row.
__device__ __forceinline__ int digit_of_i64(int64_t x, int p, int b, int W) {
    if (p + b >= W) {
        int64_t t = (int64_t)((uint64_t)x << (64 - W)) >> (64 - W);
        return (int)(t >> p);
    }
    return (int)(((uint64_t)x >> p) & ((1u << b) - 1u));
}

// Balanced digits: with H = sum_{i < Lb} 2^(b*i + b-1), the value
// z = x + H is non-negative and below 2^(b*Lb) (Lb >= ceil((64+1)/b)), and
// digit m = field m of z minus 2^(b-1) -- so x = sum_m digit_m 2^(b*m) with
// every digit in [-2^(b-1), 2^(b-1)), still a local bit-field extraction.
__device__ __forceinline__ unsigned __int128 balanced_offset(int b, int Lb) {
    unsigned __int128 h = 0;
    for (int i = 0; i < Lb; ++i) h |= (unsigned __int128)1 << (b * i + b - 1);
    return h;
}
__device__ __forceinline__ int digit_balanced(unsigned __int128 z, int p, int b) {
    return (int)((unsigned)(z >> p) & ((1u << b) - 1u)) - (1 << (b - 1));
}
__device__ __forceinline__ unsigned __int128 balanced_z(int64_t x, unsigned __int128 H) {
    return (unsigned __int128)(__int128)x + H;
}

__device__ __forceinline__ uint32_t pack4(int d0, int d1, int d2, int d3) {
    return (uint32_t)(d0 & 0xFF) | ((uint32_t)(d1 & 0xFF) << 8) | ((uint32_t)(d2 & 0xFF) << 16) |
           ((uint32_t)(d3 & 0xFF) << 24);
}

__global__ void __launch_bounds__(256) pack_i64_straight_kernel(const PackArgs a) {
    const long long t = blockIdx.x * 256LL + threadIdx.x;
    const int groups = a.ld / 4;
    const int r = (int)(t / groups), c0 = (int)(t % groups) * 4;
    if (r >= a.rows) return;
    const int i = a.row0 + r;
    const long long* src = reinterpret_cast<const long long*>(a.src);
    int64_t x[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
        x[q] = (i < a.n && c0 + q < a.n) ? __ldg(src + (long long)i * a.n + c0 + q) : 0;
    uint8_t* out = reinterpret_cast<uint8_t*>(a.dst) + (long long)r * a.ld + c0;
    if (a.balanced) {
        const unsigned __int128 H = balanced_offset(a.b, a.Lb);
        unsigned __int128 z[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) z[q] = balanced_z(x[q], H);
        for (int m = 0; m < a.Lb; ++m) {
            const int p = m * a.b;
            *reinterpret_cast<uint32_t*>(out + (long long)m * a.plane) =
                pack4(digit_balanced(z[0], p, a.b), digit_balanced(z[1], p, a.b),
                      digit_balanced(z[2], p, a.b), digit_balanced(z[3], p, a.b));
        }
        return;
    }
    for (int m = 0; m < a.Lb; ++m) {
        const int p = m * a.b;
        *reinterpret_cast<uint32_t*>(out + (long long)m * a.plane) =
            pack4(digit_of_i64(x[0], p, a.b, a.W), digit_of_i64(x[1], p, a.b, a.W),
                  digit_of_i64(x[2], p, a.b, a.W), digit_of_i64(x[3], p, a.b, a.W));
    }
}

__global__ void __launch_bounds__(256) pack_i64_transposed_kernel(const PackArgs a) {
    __shared__ int64_t tile[64][65];
    const int k0 = blockIdx.x * 64, j0 = blockIdx.y * 64;  // contraction / output-row origin
    const long long* src = reinterpret_cast<const long long*>(a.src);
    for (int e = threadIdx.x; e < 64 * 64; e += 256) {
        const int kk = e >> 6, jj = e & 63;  // coalesced along j
        const int k = k0 + kk, j = j0 + jj;
        tile[kk][jj] = (k < a.n && j < a.n) ? __ldg(src + (long long)k * a.n + j) : 0;
    }
    __syncthreads();
    uint8_t* out = reinterpret_cast<uint8_t*>(a.dst);
    for (int w = threadIdx.x; w < 64 * 16; w += 256) {
        const int jj = w >> 4, kq = (w & 15) * 4;  // 16 threads per output row
        const int r = j0 + jj, c = k0 + kq;
        if (r >= a.rows || c >= a.ld) continue;
        const int64_t x0 = tile[kq][jj], x1 = tile[kq + 1][jj], x2 = tile[kq + 2][jj],
                      x3 = tile[kq + 3][jj];
        uint8_t* o = out + (long long)r * a.ld + c;
        if (a.balanced) {
            const unsigned __int128 H = balanced_offset(a.b, a.Lb);
            const unsigned __int128 z0 = balanced_z(x0, H), z1 = balanced_z(x1, H),
                                    z2 = balanced_z(x2, H), z3 = balanced_z(x3, H);
            for (int m = 0; m < a.Lb; ++m) {
                const int p = m * a.b;
                *reinterpret_cast<uint32_t*>(o + (long long)m * a.plane) =
                    pack4(digit_balanced(z0, p, a.b), digit_balanced(z1, p, a.b),
                          digit_balanced(z2, p, a.b), digit_balanced(z3, p, a.b));
            }
            continue;
        }
        for (int m = 0; m < a.Lb; ++m) {
            const int p = m * a.b;
            *reinterpret_cast<uint32_t*>(o + (long long)m * a.plane) =
                pack4(digit_of_i64(x0, p, a.b, a.W), digit_of_i64(x1, p, a.b, a.W),
                      digit_of_i64(x2, p, a.b, a.W), digit_of_i64(x3, p, a.b, a.W));
        }
    }
}

int pack_launch(const PackArgs& a, cudaStream_t stream) {
    if (a.ld % 16 || a.rows <= 0 || a.Lb <= 0 || a.b < 1 || (a.b > 15 && a.fmt != PACK_I32LIMB))
        return MFFTB_ERR_ARG;
    dim3 block(256);
    if (a.balanced && (a.fmt != PACK_I64 || a.b > 8 || a.plane % 4 || a.W != 64 ||
                       a.b * a.Lb < 65 || a.b * a.Lb > 120))
        return MFFTB_ERR_ARG;
    if (a.fmt == PACK_I64 && (a.b <= 7 || a.balanced) && a.plane % 4 == 0) {
        if (a.transpose) {
            dim3 grid((a.ld + 63) / 64, (a.rows + 63) / 64);
            pack_i64_transposed_kernel<<<grid, block, 0, stream>>>(a);
        } else {
            const long long threads = (long long)a.rows * (a.ld / 4);
            pack_i64_straight_kernel<<<(unsigned)((threads + 255) / 256), block, 0, stream>>>(a);
        }
        return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
    }
    if (a.fmt == PACK_I32LIMB) {
        dim3 grid((a.ld + 31) / 32, (a.rows + 31) / 32, a.Lb);
        if (a.transpose) pack_limbs_kernel<true><<<grid, block, 0, stream>>>(a);
        else pack_limbs_kernel<false><<<grid, block, 0, stream>>>(a);
    } else {
        dim3 grid((a.ld + 31) / 32, (a.rows + 31) / 32, (a.Lb + PACK_MCH - 1) / PACK_MCH);
#define MFFTB_PACK(F)                                                                       \
    if (a.b <= 7) {                                                                         \
        if (a.transpose) pack_digits_kernel<F, true, int8_t><<<grid, block, 0, stream>>>(a);  \
        else pack_digits_kernel<F, false, int8_t><<<grid, block, 0, stream>>>(a);             \
    } else {                                                                                \
        if (a.transpose) pack_digits_kernel<F, true, int16_t><<<grid, block, 0, stream>>>(a); \
        else pack_digits_kernel<F, false, int16_t><<<grid, block, 0, stream>>>(a);            \
    }
        if (a.fmt == PACK_U16PL) {
            MFFTB_PACK(PACK_U16PL)
        } else if (a.fmt == PACK_I64) {
            MFFTB_PACK(PACK_I64)
        } else if (a.fmt == PACK_F32) {
            MFFTB_PACK(PACK_F32)
        } else if (a.fmt == PACK_F64) {
            MFFTB_PACK(PACK_F64)
        } else {
            return MFFTB_ERR_ARG;
        }
#undef MFFTB_PACK
    }
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

}  // namespace mfftb
