// decode.cuh -- exact big-integer -> fp32 / fp64 rounding of the fixed-point
// embeddings, shared by the GPU kernels and the host self-test entry points.
//
// Semantics follow fpx_decode_f32 (src/fpfixed.c:212-285): the exact product
// is carried into 16-bit limbs (two's complement), negated if negative, the
// top (at most four) limbs that hold the leading bit are gathered as `top`,
// everything below is the sticky bit, and round_to() rounds `top` to 24 bits
// half-to-even with the sticky bit breaking ties.  The result is
// sgn * ldexpf(sig, shift - S).  ldexpf is evaluated here from its IEEE-754
// definition (exact scaling of a <=24-bit integer, one round-to-nearest-even
// step into the subnormal range, infinity on overflow); no libm is called.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define MFFTB_HD __host__ __device__ __forceinline__
#else
#define MFFTB_HD inline
#endif

namespace mfftb {

MFFTB_HD int bitlen64(uint64_t v) {
    int n = 0;
    while (v) {
        ++n;
        v >>= 1;
    }
    return n;
}

// sig * 2^e rounded to the nearest fp32 (ties to even), sig < 2^24.
MFFTB_HD uint32_t scale_to_f32_bits(uint32_t sig, int e) {
    if (sig == 0) return 0u;
    const int nb = bitlen64(sig);
    const int E = e + nb - 1;  // value in [2^E, 2^(E+1))
    if (E > 127) return 0x7F800000u;
    if (E >= -126) {
        uint32_t mant = sig << (24 - nb);
        return ((uint32_t)(E + 127) << 23) | (mant & 0x7FFFFFu);
    }
    // subnormal: units of 2^-149
    const int sh = e + 149;
    if (sh >= 0) return sig << sh;  // exact, < 2^23
    const int r = -sh;
    if (r >= 32) return 0u;
    uint32_t q = sig >> r;
    uint32_t rem = sig & ((1u << r) - 1u);
    uint32_t half = 1u << (r - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return q;  // may carry into the smallest normal, which is the right encoding
}

// Bits [lo, lo+cnt) (cnt <= 64) of the little-endian word array w[0..nw);
// positions below 0 or past the array read as 0.  Three words are enough:
// a 64-bit field starting at bit (lo mod 32) ends inside the third.
MFFTB_HD uint64_t get_bits(const uint32_t* w, int nw, int lo, int cnt) {
    if (cnt <= 0) return 0;
    int lead = 0;  // zero bits contributed by positions below 0
    if (lo < 0) {
        lead = -lo;
        if (lead >= cnt) return 0;
        cnt -= lead;
        lo = 0;
    }
    const int wi = lo >> 5, sh = lo & 31;
    const uint64_t x0 = wi < nw ? w[wi] : 0u;
    const uint64_t x1 = wi + 1 < nw ? w[wi + 1] : 0u;
    const uint64_t x2 = wi + 2 < nw ? w[wi + 2] : 0u;
    uint64_t r = ((x1 << 32) | x0) >> sh;
    if (sh) r |= x2 << (64 - sh);
    if (cnt < 64) r &= (1ull << cnt) - 1ull;
    return r << lead;
}

MFFTB_HD bool any_bits_below(const uint32_t* w, int nw, int lim) {
    if (lim <= 0) return false;
    int full = lim >> 5;
    for (int i = 0; i < full && i < nw; ++i)
        if (w[i]) return true;
    int rem = lim & 31;
    if (rem && full < nw && (w[full] & ((1u << rem) - 1u))) return true;
    return false;
}

// sig * 2^e rounded to the nearest fp64 (ties to even), sig < 2^53; the
// IEEE-754 binary64 counterpart of scale_to_f32_bits (ldexp of fpx_decode_f64,
// src/fpfixed.c:308-322).
MFFTB_HD uint64_t scale_to_f64_bits(uint64_t sig, int e) {
    if (sig == 0) return 0ull;
    const int nb = bitlen64(sig);
    const int E = e + nb - 1;  // value in [2^E, 2^(E+1))
    if (E > 1023) return 0x7FF0000000000000ull;
    if (E >= -1022) {
        uint64_t mant = sig << (53 - nb);
        return ((uint64_t)(E + 1023) << 52) | (mant & 0xFFFFFFFFFFFFFull);
    }
    // subnormal: units of 2^-1074
    const int sh = e + 1074;
    if (sh >= 0) return sig << sh;  // exact, < 2^52
    const int r = -sh;
    if (r >= 64) return 0ull;
    uint64_t q = sig >> r;
    uint64_t rem = sig & ((1ull << r) - 1ull);
    uint64_t half = 1ull << (r - 1);
    if (rem > half || (rem == half && (q & 1ull))) ++q;
    return q;
}

// Shared front half of the decode (extract + round_to of src/fpfixed.c:
// 212-265): negate a negative value in place, locate its top 16-bit limb on
// the grid, gather at most four limbs as `top`, round to `bits` significant
// bits half-to-even with the sticky bit breaking ties.  Returns 0 for an
// exact zero, else -1 / +1 with *sig and *shift set (value = sig * 2^shift).
MFFTB_HD int decode_words_round(uint32_t* w, int nw, int bit_off, int bits, uint64_t* sig_out,
                                int* shift_out) {
    const bool neg = (w[nw - 1] >> 31) & 1u;
    if (neg) {
        uint32_t c = 1;
        for (int i = 0; i < nw; ++i) {
            uint64_t t = (uint64_t)(~w[i]) + c;
            w[i] = (uint32_t)t;
            c = (uint32_t)(t >> 32);
        }
    }
    int top_word = -1;
    for (int i = nw - 1; i >= 0; --i)
        if (w[i]) {
            top_word = i;
            break;
        }
    if (top_word < 0) return 0;
    const int bitlen_int = 32 * top_word + bitlen64(w[top_word]);
    const int bitlen = bitlen_int + bit_off;
    const int h = (bitlen - 1) >> 4;
    const int k = h + 1 < 4 ? h + 1 : 4;
    const int base = 16 * (h - k + 1);
    const int tb = bitlen - base;
    const uint64_t top = get_bits(w, nw, base - bit_off, tb);
    const bool sticky = any_bits_below(w, nw, base - bit_off);
    int shift = base;
    uint64_t sig = top;
    if (tb > bits) {
        int drop = tb - bits;
        uint64_t q = top >> drop;
        uint64_t rem = top & ((1ULL << drop) - 1);
        uint64_t half = 1ULL << (drop - 1);
        int up = rem > half ? 1 : (rem < half ? 0 : (sticky ? 1 : (int)(q & 1)));
        q += up;
        if (q >> bits) {
            q >>= 1;
            ++drop;
        }
        shift += drop;
        sig = q;
    }
    *sig_out = sig;
    *shift_out = shift;
    return neg ? -1 : 1;
}

// fpx_decode_f64's rule on the same word array (53-bit significand).
MFFTB_HD double decode_words_f64(uint32_t* w, int nw, int bit_off, int S) {
    uint64_t sig;
    int shift;
    const int sgn = decode_words_round(w, nw, bit_off, 53, &sig, &shift);
    uint64_t bits = sgn ? scale_to_f64_bits(sig, shift - S) : 0ull;
    if (sgn < 0) bits |= 0x8000000000000000ull;
    union {
        uint64_t u;
        double d;
    } cv;
    cv.u = bits;
    return cv.d;
}

// w: the exact product as nw 32-bit words of two's complement (little
// endian), worth w * 2^bit_off on the grid of scale 2^S.  w is modified
// (negated in place when negative).
MFFTB_HD float decode_words_f32(uint32_t* w, int nw, int bit_off, int S) {
    const bool neg = (w[nw - 1] >> 31) & 1u;
    if (neg) {
        uint32_t c = 1;
        for (int i = 0; i < nw; ++i) {
            uint64_t t = (uint64_t)(~w[i]) + c;
            w[i] = (uint32_t)t;
            c = (uint32_t)(t >> 32);
        }
    }
    int top_word = -1;
    for (int i = nw - 1; i >= 0; --i)
        if (w[i]) {
            top_word = i;
            break;
        }
    if (top_word < 0) return 0.0f;  // exact zero -> +0.0f
    const int bitlen_int = 32 * top_word + bitlen64(w[top_word]);
    const int bitlen = bitlen_int + bit_off;          // true bit length on the grid
    const int h = (bitlen - 1) >> 4;                  // top non-zero 16-bit limb
    const int k = h + 1 < 4 ? h + 1 : 4;              // limbs gathered
    const int base = 16 * (h - k + 1);
    const int tb = bitlen - base;
    const uint64_t top = get_bits(w, nw, base - bit_off, tb);
    const bool sticky = any_bits_below(w, nw, base - bit_off);
    int shift = base;
    uint64_t sig = top;
    if (tb > 24) {
        int drop = tb - 24;
        uint64_t q = top >> drop;
        uint64_t rem = top & ((1ULL << drop) - 1);
        uint64_t half = 1ULL << (drop - 1);
        int up = rem > half ? 1 : (rem < half ? 0 : (sticky ? 1 : (int)(q & 1)));
        q += up;
        if (q >> 24) {
            q >>= 1;
            ++drop;
        }
        shift += drop;
        sig = q;
    }
    uint32_t bits = scale_to_f32_bits((uint32_t)sig, shift - S);
    if (neg) bits |= 0x80000000u;
    union {
        uint32_t u;
        float f;
    } cv;
    cv.u = bits;
    return cv.f;
}

}  // namespace mfftb
