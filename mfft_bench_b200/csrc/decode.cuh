// decode.cuh -- exact big-integer -> fp32 rounding of the fp32 embedding,
// shared by the GPU kernel and the host self-test entry point.
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

// Bits [lo, lo+cnt) (cnt <= 64) of the little-endian word array w[0..nw).
MFFTB_HD uint64_t get_bits(const uint32_t* w, int nw, int lo, int cnt) {
    uint64_t r = 0;
    for (int i = 0; i < cnt; ++i) {
        int p = lo + i;
        if (p < 0) continue;
        int wi = p >> 5;
        if (wi >= nw) break;
        r |= (uint64_t)((w[wi] >> (p & 31)) & 1u) << i;
    }
    return r;
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
