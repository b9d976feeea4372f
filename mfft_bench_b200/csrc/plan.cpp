// plan.cpp -- exact-plan search; see plan.h.
#include "plan.h"

#include <cmath>
#include <cstring>

namespace mfftb {

static int next_pow2(int x) {
    int r = 1;
    while (r < x) r <<= 1;
    return r;
}

// Split |x| <= M into d signed digits: d-1 balanced low digits in [-64, 63]
// and a top digit; returns d (0 if more than 4 would be needed) and the
// per-digit magnitude bounds.
static int split_bounds(long long M, int bounds[4]) {
    for (int d = 1; d <= 4; ++d) {
        long long T = M;
        for (int i = 0; i < d - 1; ++i) {
            bounds[i] = (int)(T < 64 ? T : 64);
            T = (T + 64) / 128;
        }
        if (T <= 127) {
            bounds[d - 1] = (int)T;
            for (int i = d; i < 4; ++i) bounds[i] = 0;
            return d;
        }
    }
    return 0;
}

static bool fill(Plan& p) {
    const long long dmax = p.mode == PLAN_LIMB ? 65535 : (1LL << p.b) - 1;
    p.ncA = (p.LbA + p.S - 1) / p.S;
    p.ncB = (p.LbB + p.S - 1) / p.S;
    p.NB = next_pow2(p.ncA + p.ncB);
    if (p.NB < 2) p.NB = 2;
    p.K = 2 * p.S;
    if ((2 * p.K) % p.NB) return false;
    p.g = 2 * p.K / p.NB;
    const long long MA = p.ncA * dmax, MB = p.ncB * dmax;
    p.dA = split_bounds(MA, p.boundA);
    p.dB = split_bounds(MB, p.boundB);
    if (!p.dA || !p.dB) return false;
    p.nW = p.dA + p.dB - 1;
    // int32 accumulator: a chunk of one class holds at most ceil(total/nchunk)
    // segments, each a length-n contraction of two digit planes.
    const long long lim = 2147483647LL;
    int nchunk = 0;
    for (int c = 1; c <= p.K && !nchunk; ++c) {
        bool ok = true;
        long long worst = 0;
        for (int w = 0; w < p.nW && ok; ++w) {
            int lo = w - (p.dB - 1) > 0 ? w - (p.dB - 1) : 0;
            int hi = w < p.dA - 1 ? w : p.dA - 1;
            int total = (hi - lo + 1) * p.K;
            long long segmax = 0;
            for (int da = lo; da <= hi; ++da) {
                long long s = (long long)p.n_int * p.boundA[da] * p.boundB[w - da];
                if (s > segmax) segmax = s;
            }
            long long per = (total + c - 1) / c;
            long long bnd = per * segmax;
            if (bnd > lim) ok = false;
            if (bnd > worst) worst = bnd;
        }
        if (ok) {
            nchunk = c;
            p.acc_bound = worst;
        }
    }
    if (!nchunk) return false;
    p.nchunk = nchunk;
    p.njobs = p.NB * p.K * p.nW * p.nchunk;
    // inverse transform: |Chat| <= K * n * MA * MB, summed over NB points
    p.inv_bound_log2 = std::log2((double)p.NB) + std::log2((double)p.K) +
                       std::log2((double)p.n_int) + std::log2((double)MA) +
                       std::log2((double)MB) + 1.0;
    if (p.inv_bound_log2 > 62.0) return false;
    p.positions = p.LbA + p.LbB - 1;
    p.macs_per_elem = (double)p.NB * p.K * p.K * p.dA * p.dB * p.n_int;
    return true;
}

static bool better(const Plan& a, const Plan& b) {
    if (a.macs_per_elem != b.macs_per_elem) return a.macs_per_elem < b.macs_per_elem;
    if (a.njobs != b.njobs) return a.njobs < b.njobs;
    return a.NB * (2 * a.K - 1) * a.dB < b.NB * (2 * b.K - 1) * b.dB;
}

int plan_search(int n, int mode, int wA, int wB, int force_b, int force_S, Plan* out) {
    if (n <= 0 || wA <= 0 || wB <= 0 || !out) return 1;
    Plan best;
    bool have = false;
    // value-mode digit planes are int8 for b <= 7 and int16 up to b = 15 (they
    // feed only the forward transform; the tensor-core operands are the
    // split transformed planes, always int8)
    int b_lo = 2, b_hi = 15;
    if (mode == PLAN_LIMB) b_lo = b_hi = 16;
    else if (force_b > 0) {
        if (force_b > 15) return 1;
        b_lo = b_hi = force_b;
    }
    for (int b = b_lo; b <= b_hi; ++b) {
        for (int sigma = 0; sigma <= 13; ++sigma) {
            int S = 1 << sigma;
            if (force_S > 0 && S != force_S) continue;
            Plan p;
            std::memset(&p, 0, sizeof p);
            p.n = n;
            p.n_int = (n + 15) / 16 * 16;
            p.mode = mode;
            p.b = b;
            p.LbA = mode == PLAN_LIMB ? wA : (wA + b - 1) / b;
            p.LbB = mode == PLAN_LIMB ? wB : (wB + b - 1) / b;
            p.wA = mode == PLAN_LIMB ? 16 * wA : wA;
            p.wB = mode == PLAN_LIMB ? 16 * wB : wB;
            p.S = S;
            if (S > 2 * (p.LbA > p.LbB ? p.LbA : p.LbB) && S > 1) continue;
            if (!fill(p)) continue;
            if (!have || better(p, best)) {
                best = p;
                have = true;
            }
        }
    }
    if (!have) return 2;
    *out = best;
    return 0;
}

int plan_kara_max_level(const Plan& p) {
    if (p.kind != KIND_MFFT || p.mode != PLAN_VALUE || p.K != 8 || p.S != 4 || p.dA != 1 ||
        p.dB != 1 || p.nchunk != 1 || p.NB < 2 || p.NB > 8 || p.dsum)
        return 0;
    const long long lim = 2147483647LL;
    const long long A = p.boundA[0], B = p.boundB[0];
    // level 1: the operands of P2, one digit term per block, are int8 like
    // the values; P2's accumulators sum up to 4 terms of length n
    if (A > 127 || B > 127 || 4LL * p.n_int * A * B > lim) return 0;
    // levels 2 and 3: sums of two terms per block, accumulators of at most
    // 2 terms of such sums
    if (2 * A > 127 || 2 * B > 127 || 2LL * p.n_int * (2 * A) * (2 * B) > lim) return 1;
    return 3;
}

bool plan_kara_ok(const Plan& p) { return plan_kara_max_level(p) > 0; }

void plan_set_kara(Plan& p, int level) {
    if (level < 0 || level > 3) level = 0;
    const int top = plan_kara_max_level(p);
    if (level > top) level = top;
    p.kara = level;
    const double S2 = (double)p.S * p.S;
    const double pts = p.NB <= 2 ? 0.0 : (double)p.NB - 2.0;  // ordinary points
    const double half = p.NB <= 2 ? (double)p.NB : 2.0;
    if (level == 1) {  // P0, P1, P2: S^2 plane products each
        p.njobs = p.NB * 21;
        p.macs_per_elem = (3.0 * S2 * pts + S2 * half) * p.n_int;
    } else if (level == 2) {  // P0, P1 as three length-S/2 convolutions each
        const double q = 3.0 * S2 / 4.0;
        p.njobs = p.NB * 25;
        p.macs_per_elem = ((2.0 * q + S2) * pts + q * half) * p.n_int;
    } else if (level == 3) {  // P0, P1 and P2 as three length-S/2 convolutions each
        const double q = 3.0 * S2 / 4.0;
        p.njobs = p.NB * 27;
        p.macs_per_elem = (3.0 * q * pts + q * half) * p.n_int;
    } else {
        p.njobs = p.NB * p.K * p.nW * p.nchunk;
        p.macs_per_elem = (double)p.NB * p.K * p.K * p.dA * p.dB * p.n_int;
    }
}

// chunks per class of a digit-sum plan (0: none fits); *worst receives the
// largest accumulator bound
static int dsum_chunks(const Plan& p, long long* worst) {
    const long long lim = 2147483647LL;
    const long long bA[3] = {p.boundA[0], p.boundA[1], (long long)p.boundA[0] + p.boundA[1]};
    const long long bB[3] = {p.boundB[0], p.boundB[1], (long long)p.boundB[0] + p.boundB[1]};
    for (int c = 1; c <= p.K; ++c) {
        long long w = 0;
        bool ok = true;
        for (int cls = 0; cls < 3 && ok; ++cls) {
            const long long bnd = (long long)((p.K + c - 1) / c) * p.n_int * bA[cls] * bB[cls];
            if (bnd > lim) ok = false;
            if (bnd > w) w = bnd;
        }
        if (ok) {
            *worst = w;
            return c;
        }
    }
    return 0;
}

bool plan_dsum_ok(const Plan& p) {
    if (p.kind != KIND_MFFT || p.kara || p.dsum || p.dA != 2 || p.dB != 2) return false;
    if (p.boundA[0] > 64 || p.boundB[0] > 64 || p.boundA[1] > 64 || p.boundB[1] > 64)
        return false;
    long long worst = 0;
    return dsum_chunks(p, &worst) > 0;
}

void plan_set_dsum(Plan& p) {
    if (!plan_dsum_ok(p)) return;
    long long worst = 0;
    p.nchunk = dsum_chunks(p, &worst);
    p.acc_bound = worst;
    p.dsum = 1;
    p.dA = p.dB = 3;
    p.nW = 3;
    p.boundA[2] = p.boundA[0] + p.boundA[1];
    p.boundB[2] = p.boundB[0] + p.boundB[1];
    p.njobs = p.NB * p.K * p.nW * p.nchunk;
    p.macs_per_elem = (double)p.NB * p.K * p.K * 3 * p.n_int;
}

int plan_search_school(int n, int wA, int wB, int force_b, Plan* out, int balanced_ok) {
    if (n <= 0 || wA <= 0 || wB <= 0 || !out) return 1;
    if (force_b > 8 || (force_b == 8 && !balanced_ok)) return 1;
    Plan best;
    double best_cost = 0;
    bool have = false;
    const long long lim = 2147483647LL;
    const int b_lo = force_b > 0 ? force_b : 2;
    const int b_hi = force_b > 0 ? force_b : (balanced_ok ? 8 : 7);
    for (int cand = 0; cand < 2 * (b_hi - b_lo + 1); ++cand) {
        const int b = b_lo + cand / 2;
        const int bal = cand & 1;
        if (bal && !balanced_ok) continue;
        if (!bal && b > 7) continue;
        Plan p;
        std::memset(&p, 0, sizeof p);
        p.kind = KIND_SCHOOL;
        p.n = n;
        p.n_int = (n + 15) / 16 * 16;
        p.mode = PLAN_VALUE;
        p.b = b;
        p.balanced = bal;
        // balanced digits of a W-bit two's complement value: ceil((W+1)/b)
        p.LbA = bal ? (wA + b) / b : (wA + b - 1) / b;
        p.LbB = bal ? (wB + b) / b : (wB + b - 1) / b;
        p.wA = wA;
        p.wB = wB;
        p.positions = p.LbA + p.LbB - 1;
        p.NB = 1;
        p.K = (p.positions + 3) / 4 * 4;
        p.S = p.K / 2;
        p.g = 2;
        p.ncA = p.LbA;
        p.ncB = p.LbB;
        p.dA = p.dB = p.nW = 1;
        const long long dmax = bal ? (1LL << (b - 1)) : (1LL << b) - 1;
        p.boundA[0] = p.boundB[0] = (int)dmax;
        const long long seg = (long long)p.n_int * dmax * dmax;  // one plane product
        long long U = lim / seg;
        if (U < 1) continue;
        const int terms = p.LbA < p.LbB ? p.LbA : p.LbB;
        if (U > p.LbA) U = p.LbA;
        p.U = (int)U;
        p.nchunk = (p.LbA + p.U - 1) / p.U;
        p.acc_bound = (long long)(p.U < terms ? p.U : terms) * seg;
        p.njobs = p.K * p.nchunk;
        p.inv_bound_log2 = std::log2((double)terms) + std::log2((double)seg) + 1.0;
        p.macs_per_elem = (double)p.LbA * p.LbB * p.n_int;
        int live = 0;
        for (int t = 0; t < p.positions; ++t)
            for (int ch = 0; ch < p.nchunk; ++ch) live += school_job_live(p, t, ch);
        // one int8 MAC ~ 1/250 of an HBM byte at the measured rates; a live job
        // plane costs 8 B per element (written, then read by the carry)
        const double cost = p.macs_per_elem + 2000.0 * live;
        if (!have || cost < best_cost) {
            best = p;
            best_cost = cost;
            have = true;
        }
    }
    if (!have) return 2;
    *out = best;
    return 0;
}

}  // namespace mfftb
