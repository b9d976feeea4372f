// plan.h -- MFFT plan for the B200 path: limb radix, block size, transform
// length, int8 digit split of the transformed planes and contraction chunks.
//
// The reference plans a fixed 16-bit limb radix with S = 2^floor(log2(L)/2)
// (src/mfft.c:77-95) and multiplies transformed planes as int32 x int32 ->
// int64 on CPU cores.  Here every product must run on tcgen05 kind::i8, so
// the planner searches the limb radix b, the block size S and the int8 digit
// split jointly, minimising issued int8 MACs subject to exactness:
//   * every transformed coefficient (a signed sum of nc digits) is split
//     into d signed int8 digits (balanced 7-bit low digits, top digit <=127);
//   * every int32 TMEM accumulator stays below 2^31 (chunked contraction);
//   * the inverse transform stays below 2^62 in int64.
// Exactness never depends on the plan; only speed does.
#pragma once
#include <cstdint>

namespace mfftb {

enum PlanMode {
    PLAN_VALUE = 0,  // entries re-radixed into b-bit digits of |x| (sign applied)
    PLAN_LIMB = 1,   // the caller's 16-bit limbs are the coefficients (conv_mfft)
};

enum PlanKind {
    KIND_MFFT = 0,    // transform, pointwise NB*K^2 plane products, inverse
    KIND_SCHOOL = 1,  // limb-plane schoolbook: LbA*LbB digit-plane products, no transform
};

struct Plan {
    int kind;       // PlanKind
    int n;          // matrix dimension
    int n_int;      // internal dimension: n rounded up to a multiple of 16
    int mode;       // PlanMode
    int b;          // digit bits (16 in PLAN_LIMB)
    int LbA, LbB;   // digits (coefficients) per entry of A / B
    int wA, wB;     // bits per entry of A / B: magnitude bits (PLAN_VALUE),
                    // 16 x limbs (PLAN_LIMB)
    int S, NB, K, g;
    int ncA, ncB;   // nonzero input blocks of A / B
    int dA, dB;     // int8 digits per transformed value
    int nW;         // digit-weight classes dA + dB - 1
    int nchunk;     // contraction chunks per job
    int njobs;      // NB * K * nW * nchunk
    int boundA[4], boundB[4];  // |digit| bounds of the split transformed values
    int positions;  // radix-2^b output positions produced (LbA + LbB - 1)
    long long acc_bound;       // worst int32 accumulator magnitude
    double inv_bound_log2;     // log2 of the worst inverse-transform magnitude
    double macs_per_elem;      // int8 MACs per output element = NB*K*K*dA*dB*n
    // KIND_SCHOOL: job t (t < K, K = positions rounded up to 4) of chunk ch
    // sums A_u * B_(t-u) over u in [ch*U, ch*U+U) with 0 <= t-u < LbB;
    // NB = 1, dA = dB = nW = 1, njobs = K * nchunk.
    int U;
    // balanced digits (int64 entries only): digit m of x is byte m of
    // x + sum_i 2^(b*i + b-1), minus 2^(b-1), so digits lie in
    // [-2^(b-1), 2^(b-1)) and b = 8 still fits int8
    int balanced;
    // Karatsuba pointwise (KIND_MFFT, K = 8): each point's ring product is
    // three full convolutions of length S = 4 instead of the K^2 negacyclic
    // terms -- 48 plane products per point, 16 at the half points; njobs is
    // then the NB * 21 job planes, macs_per_elem the issued MACs.  kara = 2
    // splits P0 and P1 once more into three length-2 convolutions each (40
    // plane products per point, 12 at the half points, NB * 25 job planes);
    // kara = 3 splits P2 as well (36 per point, NB * 27 job planes).
    int kara;
    // Digit sums (two-digit plans): each transformed value x = lo + 2^7 hi
    // also gets the digit lo + hi, and the product's middle class
    // lo_A hi_B + hi_A lo_B comes from (lo_A + hi_A)(lo_B + hi_B) - lo_A lo_B -
    // hi_A hi_B: three digit-pair products per term instead of four.  The
    // plan then has dA = dB = 3 digits and nW = 3 classes (lo*lo, hi*hi,
    // sum*sum), one digit pair each.
    int dsum;
};

// Returns 0 and fills *p on success.  wA / wB: magnitude bits per entry in
// PLAN_VALUE, limb counts in PLAN_LIMB.  force_b > 0 pins the digit width
// (PLAN_VALUE only); force_S > 0 pins the block size.
// Bytes per element of the digit planes the pack kernel writes.
inline int plan_digit_bytes(const Plan& p) {
    return p.mode == PLAN_LIMB ? 4 : ((p.b <= 7 || p.balanced) ? 1 : 2);
}
int plan_search(int n, int mode, int wA, int wB, int force_b, int force_S, Plan* p);
// Schoolbook limb-plane plan (PLAN_VALUE only): digit width b in [2, 7] so
// the digit planes are the int8 tensor-core operands themselves; the
// contraction over u is chunked so every int32 accumulator stays < 2^31.
// Minimises plane products plus the job-plane traffic.  force_b > 0 pins b.
// balanced_ok: the operands are two's complement int64 entries, which may use
// balanced 8-bit digits (ceil((W+1)/8) of them).
int plan_search_school(int n, int wA, int wB, int force_b, Plan* p, int balanced_ok = 0);
// The deepest Karatsuba level that keeps the plan exact (0: none).  Every
// level needs K = 8, one int8 digit per transformed value and one
// contraction chunk.  A block of the transform holds S coefficients in a
// ring of K = 2S, so a signed permutation y^e puts each block's digit in
// exactly one of the positions c and c+S: (a0 + a1)[c] = x[c] + x[c+S] has
// one digit term per block, as x[c] has, and |a0 + a1| <= boundA (level 1;
// P2's int32 accumulators sum up to 4 terms of length n).  Every sum the
// second level forms -- x[c] + x[c+2] (P0, P1) or (a0+a1)[c] +
// (a0+a1)[c+2] (P2) -- has at most two terms per block, so levels 2 and 3
// need 2 boundA <= 127 (accumulators of at most 2 terms of such sums).
int plan_kara_max_level(const Plan& p);
bool plan_kara_ok(const Plan& p);
// Whether a plan can take digit sums: two int8 digits per value on both
// sides, lo in [-64, 63] and |hi| <= 64, so lo + hi lies in [-128, 127]; and
// chunks that keep every class's accumulators below 2^31.
bool plan_dsum_ok(const Plan& p);
// Switch a two-digit plan to digit sums (dA = dB = 3, nW = 3, chunks, job
// planes and issued MACs); a plan that cannot take them is left unchanged.
void plan_set_dsum(Plan& p);
// Set a plan's Karatsuba level (0 = negacyclic; 1; 2, P0 and P1 split once
// more; 3, P2 as well; job planes and issued MACs), capped at the deepest
// level the plan can take.
void plan_set_kara(Plan& p, int level);
// Whether job (t, ch) of a schoolbook plan has any term.
inline bool school_job_live(const Plan& p, int t, int ch) {
    const int lo = t - (p.LbB - 1) > ch * p.U ? t - (p.LbB - 1) : ch * p.U;
    int hi = t < p.LbA - 1 ? t : p.LbA - 1;
    if (hi > ch * p.U + p.U - 1) hi = ch * p.U + p.U - 1;
    return lo <= hi;
}

}  // namespace mfftb
