// pointwise.cuh -- the MFFT pointwise step as one persistent tcgen05 kernel.
//
// Reference semantics (src/mfft.c:383-396, leaf src/kernel.c:160-191): for
// every evaluation point j and output ring coefficient t,
//
//     Chat[j][t] = sum_{c1} sign(c1,t) * Ahat[j][c1] * Bhat[j][(t-c1) mod K]
//
// with sign -1 where c1 > t (the negacyclic wrap of Z[y]/(y^K+1)).  Here the
// K plane products of one (j,t) are a single GEMM whose contraction is the
// K operand planes laid end to end (length K*n).  The B operand of (j,t) is a
// window of the "F" stack the forward transform writes for B:
//
//     F[r] = +Bhat[K-1-r]   for r <  K
//     F[r] = -Bhat[2K-1-r]  for r >= K            (r = 0 .. 2K-2)
//
// so the B plane paired with Ahat[j][c1] is F[K-1-t+c1]: no sign handling
// inside the kernel.  Transformed values wider than int8 are split into dA/dB
// signed 7-bit digits; a job then also carries a digit-weight class
// w = da + db, and its contraction runs over every (da, db) pair of that
// class.  Long contractions are split into nchunk chunks so that the int32
// TMEM accumulator provably cannot overflow (bounds are checked on the host
// when the plan is built).
#pragma once
#include <cstdint>

namespace mfftb {

constexpr int PW_BM = 128;          // rows of a tile (MMA M)
constexpr int PW_BK = 128;          // contraction bytes per pipeline stage
constexpr int PW_STAGES = 4;        // smem pipeline depth
constexpr int PW_MAX_BN = 256;      // widest tile (MMA N)
constexpr int PW_THREADS = 192;     // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int PW_TMEM_COLS = 512;   // two accumulator buffers of up to 256 columns
constexpr int PW_GROUP_M = 16;      // tile raster: 16 row-tiles per group for L2 reuse

constexpr int PW_A_STAGE_BYTES = PW_BM * PW_BK;
constexpr int PW_B_STAGE_BYTES = PW_MAX_BN * PW_BK;
constexpr int PW_SMEM_BYTES =
    1024 /*alignment slack*/ + PW_STAGES * (PW_A_STAGE_BYTES + PW_B_STAGE_BYTES) + 256;

struct PwJobs {
    int K;        // ring dimension
    int dA, dB;   // int8 digits per transformed A / B value
    int nW;       // digit-weight classes = dA + dB - 1
    int nchunk;   // contraction chunks per (j, t, w)
    int njobs;    // NB * K * nW * nchunk
    // Schoolbook limb-plane mode (school = 1): job q = t * nchunk + ch is
    //     C_t = sum_u A_u * B_(t-u),  u in [ch*U, ch*U+U), 0 <= u < LbA,
    //                                 0 <= t-u < LbB
    // over the digit planes themselves (the "F" operand holds B's LbB digit
    // planes in order; no transform, no signs).  K = number of t's (a
    // multiple of 4), dA = dB = nW = 1.
    int school;
    int LbA, LbB, U;
    // Half points (MFFT mode): the points j = 0 and j = NB/2 evaluate the
    // blocks at y^0 and y^K = -1, which moves no coefficient, so there
    // Ahat_j and Bhat_j vanish above coefficient zpS - 1 (zpS = S = K/2, the
    // coefficients one block holds).  zpS > 0 tells the t-grouped kernel it
    // may skip the terms that are zero for that reason; 0 = no skipping.
    int NB;
    int zpS;
    // Karatsuba mode (kara = 1; K = 8, one digit, one chunk): point j's ring
    // product is taken as three full convolutions of length S = 4 --
    // P0 = a0*b0, P1 = a1*b1, P2 = (a0+a1)*(b0+b1), with a = a0 + y^4 a1 --
    // 3*16 plane products instead of K^2 = 64; the half points need only P0
    // (a1 = b1 = 0 there).  The operands are 12 planes per point, in order
    // a0[0..3], a1[0..3], (a0+a1)[0..3] (the same for B), and product p's
    // output coefficient s (s = 0..6) goes to job plane j*21 + p*7 + s; the
    // inverse combines them into Chat_j.
    //
    // kara = 2 applies the same split once more to P0 and P1, whose operands
    // are single digits (|x| <= 60, so x[c] + x[c+2] still fits int8): with
    // a0 = u0 + z^2 u1 (z = y), P0 = Q0 + z^2 (Q2 - Q0 - Q1) + z^4 Q1 for the
    // three length-2 convolutions Q0 = u0*v0, Q1 = u1*v1,
    // Q2 = (u0+u1)*(v0+v1), 12 plane products instead of 16 (P2's operands
    // are already sums and stay one level deep).  The operands are 16 planes
    // per point: the 12 above, then a0[0]+a0[2], a0[1]+a0[3], a1[0]+a1[2],
    // a1[1]+a1[3]; the job planes are 25 per point: Q0, Q1, Q2 of P0
    // (3 coefficients each, planes j*25 + 0..8), of P1 (9..17), then P2's 7
    // (18..24).
    //
    // kara = 3 splits P2 the same way.  Its operands (a0+a1)[c] are no larger
    // than a single transformed value: every block of the transform holds S
    // coefficients in a ring of K = 2S, so of the two positions c and c+S a
    // signed permutation y^e fills exactly one from each block, and
    // (a0+a1)[c] = x[c] + x[c+S] has one digit term per block, like x[c];
    // (a0+a1)[c] + (a0+a1)[c+2] then has two per block, like x[c] + x[c+2].
    // 18 operand planes per point: the 16 above, then (a0+a1)[0]+(a0+a1)[2],
    // (a0+a1)[1]+(a0+a1)[3]; 27 job planes: the Q0, Q1, Q2 of P0 (0..8), of
    // P1 (9..17) and of P2 (18..26).
    int kara;
    // digit sums (dA = dB = 3, nW = 3): the three digits of a transformed
    // value are lo, hi and lo + hi, and class w multiplies digit w of A by
    // digit w of B only (one digit pair per class instead of up to two); the
    // inverse weighs the classes (1 - 2^7, 2^14 - 2^7, 2^7)
    int dsum;
};

constexpr int PWK_OPS = 12;    // operand planes per point, kara = 1
constexpr int PWK_JOBS = 21;   // job planes per point, kara = 1
constexpr int PWK2_OPS = 16;   // operand planes per point, kara = 2
constexpr int PWK2_JOBS = 25;  // job planes per point, kara = 2
constexpr int PWK3_OPS = 18;   // operand planes per point, kara = 3
constexpr int PWK3_JOBS = 27;  // job planes per point, kara = 3

__host__ __device__ inline int pw_kara_level_ops(int level) {
    return level == 3 ? PWK3_OPS : (level == 2 ? PWK2_OPS : PWK_OPS);
}
__host__ __device__ inline int pw_kara_ops(const PwJobs& J) { return pw_kara_level_ops(J.kara); }
__host__ __device__ inline int pw_kara_jobs(const PwJobs& J) {
    return J.kara == 3 ? PWK3_JOBS : (J.kara == 2 ? PWK2_JOBS : PWK_JOBS);
}
// kara >= 2: the first operand plane of length-2 convolution g within a
// point's operand planes (g = 0..2: Q0, Q1, Q2 of P0; 3..5: of P1; 6..8, at
// kara = 3: of P2)
__host__ __device__ inline int pw_kara2_qplane(int g) {
    switch (g) {
        case 0: return 0;
        case 1: return 2;
        case 2: return 12;
        case 3: return 4;
        case 4: return 6;
        case 5: return 14;
        case 6: return 8;
        case 7: return 10;
        default: return 16;
    }
}

// Karatsuba mode: the half points (j = 0, NB/2) need P0 only
__host__ __device__ inline bool pw_kara_half(const PwJobs& J, int j) {
    return j == 0 || 2 * j == J.NB;
}
// tile groups per point: kara = 1, (product p, output half hi), 6 per
// ordinary point, 2 per half point; kara = 2, the six length-2 convolutions
// and P2's two halves, 8 per ordinary point, 3 per half point; kara = 3,
// nine length-2 convolutions per ordinary point, 3 per half point
__host__ __device__ inline int pw_kara_point_groups(const PwJobs& J, bool half) {
    if (half) return J.kara >= 2 ? 3 : 2;
    return J.kara == 3 ? 9 : (J.kara == 2 ? 8 : 6);
}
__host__ __device__ inline int pw_kara_groups(const PwJobs& J) {
    const int nhalf = J.NB <= 2 ? J.NB : 2;
    return nhalf * pw_kara_point_groups(J, true) + (J.NB - nhalf) * pw_kara_point_groups(J, false);
}

__host__ __device__ inline bool pw_half_point(const PwJobs& J, int j) {
    return !J.school && J.zpS > 0 && (j == 0 || 2 * j == J.NB);
}

// c1 range [lo, hi] of the terms of job (j, t) that can be non-zero: every c1
// at an ordinary point; at a half point only c1 < zpS with 0 <= t - c1 < zpS
// (no wrap, since t - c1 + K >= zpS); empty when lo > hi (t > 2 zpS - 2).
__host__ __device__ inline void pw_point_range(const PwJobs& J, int j, int t, int& lo, int& hi) {
    if (!pw_half_point(J, j)) {
        lo = 0;
        hi = J.K - 1;
        return;
    }
    lo = t - (J.zpS - 1);
    if (lo < 0) lo = 0;
    hi = t < J.zpS - 1 ? t : J.zpS - 1;
}

// u range [lo, hi] of schoolbook job (t, ch); empty when lo > hi
__host__ __device__ inline void pw_school_range(const PwJobs& J, int t, int ch, int& lo, int& hi) {
    lo = ch * J.U;
    if (t - (J.LbB - 1) > lo) lo = t - (J.LbB - 1);
    hi = ch * J.U + J.U - 1;
    if (t < hi) hi = t;
    if (J.LbA - 1 < hi) hi = J.LbA - 1;
}

struct PwParams {
    PwJobs jobs;
    int rows;          // valid rows of A (and of the output planes)
    int cols;          // valid columns of the output planes (= rows of B^T)
    int kdim;          // valid contraction length of one plane pair
    int kblocks;       // ceil(kdim / PW_BK)
    int block_n;       // MMA N: 64, 128 or 256
    int tiles_m, tiles_n;
    long long num_tiles;
    int32_t* out;      // [job][rows][ldo] int32
    long long out_plane;  // elements between job planes
    int ldo;           // output row stride (elements)
    int* err;          // device status word (0 = ok)
    unsigned long long timeout_ns;
    int stall_producer;  // self-test of the bounded waits: the producer issues nothing
    int raster;          // 0: job-major; 1: point-major, the K*nW*nchunk jobs of a tile innermost
    int group_m;         // row tiles per raster group
    // Wave alignment (t-grouped kernel): before each full wave of tiles the
    // producers meet at this zeroed counter so CTAs that share operand tiles
    // read them at about the same time (L2 reuse).  A timing hint only: a
    // wait that runs past its deadline switches the alignment off.
    unsigned int* wave_counter;
};

// Segment s of job q: which A plane and which F plane feed it.  Shared by
// the kernel and the host-side checker so both read the same job table.
__host__ __device__ inline void pw_job_decode(const PwJobs& J, int q, int& j, int& t, int& w,
                                              int& ch) {
    ch = q % J.nchunk;
    int r = q / J.nchunk;
    w = r % J.nW;
    r /= J.nW;
    t = r % J.K;
    j = r / J.K;
}

__host__ __device__ inline int pw_class_first_da(const PwJobs& J, int w) {
    if (J.dsum) return w;
    int lo = w - (J.dB - 1);
    return lo > 0 ? lo : 0;
}
__host__ __device__ inline int pw_class_pairs(const PwJobs& J, int w) {
    if (J.dsum) return 1;
    int lo = pw_class_first_da(J, w);
    int hi = w < J.dA - 1 ? w : J.dA - 1;
    return hi - lo + 1;
}
// B's digit paired with A's digit da in class w
__host__ __device__ inline int pw_class_db(const PwJobs& J, int w, int da) {
    return J.dsum ? w : w - da;
}
// segments [s0, s1) of job q's class that chunk ch covers; the split is
// balanced so no chunk is empty while nchunk <= K (checked by the planner)
__host__ __device__ inline void pw_chunk_range(const PwJobs& J, int w, int ch, int& s0, int& s1) {
    int total = pw_class_pairs(J, w) * J.K;
    s0 = (int)((long long)ch * total / J.nchunk);
    s1 = (int)((long long)(ch + 1) * total / J.nchunk);
}
__host__ __device__ inline void pw_segment_planes(const PwJobs& J, int j, int t, int w, int s,
                                                  int& planeA, int& planeF) {
    int pair = s / J.K, c1 = s % J.K;
    int da = pw_class_first_da(J, w) + pair;
    int db = pw_class_db(J, w, da);
    planeA = (j * J.dA + da) * J.K + c1;
    planeF = (j * J.dB + db) * (2 * J.K - 1) + (J.K - 1 - t + c1);
}

}  // namespace mfftb
