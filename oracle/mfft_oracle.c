/* mfft_oracle.c -- TEST INFRASTRUCTURE ONLY (see mfft_oracle.h).
 *
 * Plain-C restatement of the reference hot path, written for clarity, not
 * speed: int64 everywhere, direct ring DFTs instead of the reference's fused
 * op lists, an ikj leaf instead of the packed kernel.  Every function cites
 * the reference lines (paths inside hadilq/mfft-bench) whose behaviour it
 * restates.  The product library never calls this code.
 */
#include "mfft_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* splitmix64, src/bigmat.c:21-27 */
uint64_t orc_sm64(uint64_t *s)
{
    uint64_t z = (*s += 0x9E3779B97F4A7C15ULL);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* one 16-bit limb per draw, plane-major order: src/bigmat.c:29-35 */
void orc_bigmat_rand(uint16_t *m, int n, int L, uint64_t seed)
{
    uint64_t s = seed;
    size_t total = (size_t)n * n * L;
    for (size_t i = 0; i < total; i++) m[i] = (uint16_t)(orc_sm64(&s) & 0xFFFFu);
}

/* Signed W=16L-bit inputs (the reference has no signed generator): the
 * bigmat_rand stream read as L-limb two's complement per entry.  The single
 * value -2^(16L-1) lies outside the open range (-2^(W-1), 2^(W-1)); it is
 * mapped to 0 (probability 2^-W per entry). */
void orc_gen_signed_planes(uint16_t *m, int n, int L, uint64_t seed)
{
    orc_bigmat_rand(m, n, L, seed);
    size_t nn = (size_t)n * n;
    for (size_t idx = 0; idx < nn; idx++) {
        if (m[(size_t)(L - 1) * nn + idx] != 0x8000u) continue;
        int low_zero = 1;
        for (int u = 0; u < L - 1; u++)
            if (m[(size_t)u * nn + idx]) { low_zero = 0; break; }
        if (low_zero) m[(size_t)(L - 1) * nn + idx] = 0;
    }
}

/* W=64 signed entries: raw splitmix64 draws, row-major */
void orc_gen_int64(int64_t *x, size_t count, uint64_t seed)
{
    uint64_t s = seed;
    for (size_t i = 0; i < count; i++) x[i] = (int64_t)orc_sm64(&s);
}

/* int64 row-major -> four 16-bit two's complement limb planes */
void orc_int64_to_planes(const int64_t *x, int n, uint16_t *planes)
{
    size_t nn = (size_t)n * n;
    for (size_t i = 0; i < nn; i++)
        for (int u = 0; u < 4; u++)
            planes[(size_t)u * nn + i] = (uint16_t)(((uint64_t)x[i] >> (16 * u)) & 0xFFFFu);
}

/* fp32 N(0,1) * 2^k, k uniform in [-8, 8] (the reference ML track only has
 * U(-1,1), src/mlgemm.c:657-680).  One splitmix64 stream from `seed`: all of
 * A, then all of B; per entry u1, u2 (open (0,1)), then k.  Box-Muller. */
static float normal_draw(uint64_t *s)
{
    double u1 = ((double)(orc_sm64(s) >> 11) + 0.5) * 0x1.0p-53;
    double u2 = ((double)(orc_sm64(s) >> 11) + 0.5) * 0x1.0p-53;
    int k = (int)(orc_sm64(s) % 17u) - 8;
    double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    return ldexpf((float)z, k);
}
void orc_gen_normal_f32(float *A, float *B, size_t count, uint64_t seed)
{
    uint64_t s = seed;
    for (size_t i = 0; i < count; i++) A[i] = normal_draw(&s);
    for (size_t i = 0; i < count; i++) B[i] = normal_draw(&s);
}

/* two's complement u16 planes -> sign * limb(|x|) int32 planes, the signed
 * limb convention of src/fpfixed.c:187-192 */
void orc_planes_to_signlimb(const uint16_t *pl, int n, int L, int32_t *out)
{
    size_t nn = (size_t)n * n;
    uint32_t *mag = malloc((size_t)L * sizeof(uint32_t));
    for (size_t idx = 0; idx < nn; idx++) {
        int neg = (pl[(size_t)(L - 1) * nn + idx] & 0x8000u) != 0;
        uint32_t borrow = 1;
        for (int u = 0; u < L; u++) {
            uint32_t v = pl[(size_t)u * nn + idx];
            if (neg) { v = (~v & 0xFFFFu) + borrow; borrow = v >> 16; v &= 0xFFFFu; }
            mag[u] = v;
        }
        for (int u = 0; u < L; u++)
            out[(size_t)u * nn + idx] = neg ? -(int32_t)mag[u] : (int32_t)mag[u];
    }
    free(mag);
}

/* src/mfft.c:77-95 */
int orc_plan_init(orc_plan *p, int L, int sigma_override)
{
    if (L < 2 || (L & (L - 1))) return -1;
    int l = 0;
    while ((1 << l) < L) l++;
    int sigma = sigma_override > 0 ? sigma_override : l / 2;
    if (sigma < 1) sigma = 1;
    if (sigma > l) return -1;
    int S = 1 << sigma, NB = 2 * L / S, K = 2 * S;
    if (2 * S * S < L) return -1;
    if ((2 * K) % NB) return -1;
    if (NB < 2) return -1;
    p->L = L; p->S = S; p->NB = NB; p->K = K; p->g = 2 * K / NB;
    p->nprod = (long long)NB * K * K;
    return 0;
}

/* dst += y^e * src in Z[y]/(y^K+1), every coefficient an nn-plane:
 * coefficient c moves to (c+e) mod 2K, negated when it passes y^K = -1
 * (src/mfft.c:124-141, src/roots.c:14-21) */
static void ring_axpy_shift(int64_t *dst, const int64_t *src, int K, size_t nn, int e)
{
    for (int c = 0; c < K; c++) {
        int m = (c + e) % (2 * K);
        int sgn = 1;
        if (m >= K) { m -= K; sgn = -1; }
        const int64_t *s = src + (size_t)c * nn;
        int64_t *d = dst + (size_t)m * nn;
        if (sgn > 0) for (size_t i = 0; i < nn; i++) d[i] += s[i];
        else         for (size_t i = 0; i < nn; i++) d[i] -= s[i];
    }
}

/* C += sign * A * B, int64 n x n, the ikj leaf of src/kernel.c:39-53 */
static void leaf_ikj(int64_t *C, const int64_t *A, const int64_t *B, int n, int sign)
{
    for (int i = 0; i < n; i++) {
        int64_t *Cr = C + (size_t)i * n;
        for (int k = 0; k < n; k++) {
            int64_t a = A[(size_t)i * n + k] * sign;
            if (!a) continue;
            const int64_t *Br = B + (size_t)k * n;
            for (int j = 0; j < n; j++) Cr[j] += a * Br[j];
        }
    }
}

/* conv_mfft, src/mfft.c:302-422: pack, evaluate at the NB roots omega^j =
 * y^(g j), pointwise negacyclic convolutions, interpolate, divide by NB,
 * fold onto limb planes.  The evaluations are computed as direct DFTs in
 * natural order (the reference's fused Gentleman-Sande / Cooley-Tukey op
 * lists produce the same values in bit-reversed order). */
void orc_conv_mfft(int64_t *Cout, const int32_t *A, const int32_t *B, int n, int L,
                   const orc_plan *p)
{
    size_t nn = (size_t)n * n;
    int NB = p->NB, K = p->K, S = p->S, g = p->g;
    size_t blk = (size_t)K * nn;
    int64_t *Ab = calloc((size_t)NB * blk, 8), *Bb = calloc((size_t)NB * blk, 8);
    int64_t *Ah = calloc((size_t)NB * blk, 8), *Bh = calloc((size_t)NB * blk, 8);
    int64_t *Ch = calloc((size_t)NB * blk, 8), *Cb = calloc((size_t)NB * blk, 8);
    int64_t *Cw = calloc((size_t)(2 * L + S) * nn, 8);
    /* pack: block b holds limbs b*S .. b*S+S-1 in coefficients 0..S-1
     * (src/mfft.c:329-336) */
    for (int b = 0; b < L / S; b++)
        for (int c = 0; c < S; c++)
            for (size_t i = 0; i < nn; i++) {
                Ab[((size_t)b * K + c) * nn + i] = A[(size_t)(b * S + c) * nn + i];
                Bb[((size_t)b * K + c) * nn + i] = B[(size_t)(b * S + c) * nn + i];
            }
    /* forward: Xhat_j = sum_b y^(g j b) X_b */
    for (int j = 0; j < NB; j++)
        for (int b = 0; b < NB; b++) {
            int e = (int)(((long long)g * j * b) % (2 * K));
            ring_axpy_shift(Ah + (size_t)j * blk, Ab + (size_t)b * blk, K, nn, e);
            ring_axpy_shift(Bh + (size_t)j * blk, Bb + (size_t)b * blk, K, nn, e);
        }
    /* pointwise: Chat_j[t] = sum over c1 + c2 = t (mod K) of +-Ahat_j[c1] Bhat_j[c2]
     * (src/mfft.c:383-396) */
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int j = 0; j < NB; j++)
        for (int t = 0; t < K; t++)
            for (int c1 = 0; c1 < K; c1++) {
                int c2 = t - c1, sgn = 1;
                if (c2 < 0) { c2 += K; sgn = -1; }
                leaf_ikj(Ch + ((size_t)j * K + t) * nn, Ah + ((size_t)j * K + c1) * nn,
                         Bh + ((size_t)j * K + c2) * nn, n, sgn);
            }
    /* inverse: NB * C_b = sum_j y^(-g j b) Chat_j */
    for (int b = 0; b < NB; b++)
        for (int j = 0; j < NB; j++) {
            int e = (int)(((long long)g * j * b) % (2 * K));
            ring_axpy_shift(Cb + (size_t)b * blk, Ch + (size_t)j * blk, K, nn, (2 * K - e) % (2 * K));
        }
    /* fold: Cw[b*S + c] += C_b[c] / NB (src/mfft.c:409-415), keep 2L-1 planes (:418) */
    for (int b = 0; b < NB; b++)
        for (int c = 0; c < K; c++) {
            int w = b * S + c;
            const int64_t *src = Cb + ((size_t)b * K + c) * nn;
            int64_t *dst = Cw + (size_t)w * nn;
            for (size_t i = 0; i < nn; i++) dst[i] += src[i] / NB;
        }
    memcpy(Cout, Cw, (size_t)(2 * L - 1) * nn * 8);
    free(Ab); free(Bb); free(Ah); free(Bh); free(Ch); free(Cb); free(Cw);
}

/* schoolbook over limb planes, src/methods.c:94-104 -- an independent check */
void orc_conv_limbplane(int64_t *Cw, const int32_t *A, const int32_t *B, int n, int L)
{
    size_t nn = (size_t)n * n;
    memset(Cw, 0, (size_t)(2 * L - 1) * nn * 8);
    int64_t *a = malloc(nn * 8), *b = malloc(nn * 8);
    for (int w = 0; w < 2 * L - 1; w++)
        for (int u = 0; u < L; u++) {
            int v = w - u;
            if (v < 0 || v >= L) continue;
            for (size_t i = 0; i < nn; i++) a[i] = A[(size_t)u * nn + i];
            for (size_t i = 0; i < nn; i++) b[i] = B[(size_t)v * nn + i];
            leaf_ikj(Cw + (size_t)w * nn, a, b, n, 1);
        }
    free(a); free(b);
}

/* src/bigmat.c:48-60 */
void orc_normalize_planes(const int64_t *acc, int nplanes, int n, uint16_t *out, int RL)
{
    size_t nn = (size_t)n * n;
    for (size_t idx = 0; idx < nn; idx++) {
        int64_t carry = 0;
        for (int w = 0; w < RL; w++) {
            int64_t v = (w < nplanes ? acc[(size_t)w * nn + idx] : 0) + carry;
            out[(size_t)w * nn + idx] = (uint16_t)(v & 0xFFFF);
            carry = v >> 16;
        }
    }
}

/* src/mfft.c:424-438 */
void orc_mm_mfft(const uint16_t *A, const uint16_t *B, int n, int L, const orc_plan *p,
                 uint16_t *out, int RL)
{
    size_t nn = (size_t)n * n;
    int P = 2 * L - 1;
    int32_t *A32 = malloc((size_t)L * nn * 4), *B32 = malloc((size_t)L * nn * 4);
    int64_t *Cw = calloc((size_t)P * nn, 8);
    for (size_t i = 0; i < (size_t)L * nn; i++) { A32[i] = A[i]; B32[i] = B[i]; }
    orc_conv_mfft(Cw, A32, B32, n, L, p);
    orc_normalize_planes(Cw, P, n, out, RL);
    free(A32); free(B32); free(Cw);
}

/* signed path: sign*limb planes -> conv_mfft -> normalize_planes, which
 * yields two's complement (the fpfixed convention applied to integers) */
void orc_mm_signed(const uint16_t *A, const uint16_t *B, int n, int L, uint16_t *out, int RL)
{
    size_t nn = (size_t)n * n;
    int P = 2 * L - 1;
    orc_plan p;
    int32_t *A32 = malloc((size_t)L * nn * 4), *B32 = malloc((size_t)L * nn * 4);
    int64_t *Cw = calloc((size_t)P * nn, 8);
    orc_planes_to_signlimb(A, n, L, A32);
    orc_planes_to_signlimb(B, n, L, B32);
    if (orc_plan_init(&p, L, 0) == 0) orc_conv_mfft(Cw, A32, B32, n, L, &p);
    else orc_conv_limbplane(Cw, A32, B32, n, L);
    orc_normalize_planes(Cw, P, n, out, RL);
    free(A32); free(B32); free(Cw);
}

/* Exact product of selected entries by the textbook per-entry limb
 * convolution of src/methods.c:30-50 (generalised to signed limbs), then
 * carried into RL limbs like src/bigmat.c:48-60.  out is [RL][nsamp]. */
void orc_entry_product(const uint16_t *A, const uint16_t *B, int n, int L, int is_signed,
                       int nsamp, const int *rows, const int *cols, uint16_t *out, int RL)
{
    size_t nn = (size_t)n * n;
#pragma omp parallel
    {
        int64_t *acc = malloc((size_t)(2 * L) * 8);
        int32_t *a = malloc((size_t)L * 4), *b = malloc((size_t)L * 4);
        uint32_t *mag = malloc((size_t)L * 4);
#pragma omp for schedule(dynamic)
        for (int s = 0; s < nsamp; s++) {
            int i = rows[s], j = cols[s];
            memset(acc, 0, (size_t)(2 * L) * 8);
            for (int k = 0; k < n; k++) {
                for (int side = 0; side < 2; side++) {
                    const uint16_t *pl = side ? B : A;
                    size_t idx = side ? (size_t)k * n + j : (size_t)i * n + k;
                    int32_t *dst = side ? b : a;
                    int neg = is_signed && (pl[(size_t)(L - 1) * nn + idx] & 0x8000u);
                    uint32_t borrow = 1;
                    for (int u = 0; u < L; u++) {
                        uint32_t v = pl[(size_t)u * nn + idx];
                        if (neg) { v = (~v & 0xFFFFu) + borrow; borrow = v >> 16; v &= 0xFFFFu; }
                        mag[u] = v;
                    }
                    for (int u = 0; u < L; u++) dst[u] = neg ? -(int32_t)mag[u] : (int32_t)mag[u];
                }
                for (int u = 0; u < L; u++) {
                    if (!a[u]) continue;
                    for (int v = 0; v < L; v++) acc[u + v] += (int64_t)a[u] * b[v];
                }
            }
            int64_t carry = 0;
            for (int w = 0; w < RL; w++) {
                int64_t v = (w < 2 * L - 1 ? acc[w] : 0) + carry;
                out[(size_t)w * nsamp + s] = (uint16_t)(v & 0xFFFF);
                carry = v >> 16;
            }
        }
        free(acc); free(a); free(b); free(mag);
    }
}

/* FNV-1a style digest over uint16 words, the golden-digest definition */
uint64_t orc_digest_u16(const uint16_t *v, size_t count)
{
    uint64_t h = 0xcbf29ce484222325ULL;
    for (size_t i = 0; i < count; i++) { h ^= v[i]; h *= 0x100000001b3ULL; }
    return h;
}

/* ------------------------------------------------------------------ *
 * fp32 fixed-point embedding, src/fpfixed.c
 * ------------------------------------------------------------------ */
static int next_pow2(int x) { int r = 1; while (r < x) r <<= 1; return r; }

/* src/fpfixed.c:40-54 */
static void fscan(const float *X, size_t nn, int *lo, int *hi, int *any)
{
    int l = 1 << 30, h = -(1 << 30), seen = 0;
    for (size_t i = 0; i < nn; i++) {
        float x = X[i];
        if (x == 0.0f || !isfinite(x)) continue;
        int e;
        frexpf(x, &e);
        int e2 = e - 24;
        if (e2 < l) l = e2;
        if (e2 > h) h = e2;
        seen = 1;
    }
    if (!seen) { l = 0; h = 0; }
    *lo = l; *hi = h; *any = seen;
}

/* src/fpfixed.c:59-78 (fp32: sig 24, three limbs touched) + :80-94 + :96-108 */
int orc_fpx_init(orc_fpx *c, const float *A, const float *B, int n, int force_bits)
{
    size_t nn = (size_t)n * n;
    int loA, hiA, loB, hiB, anyA, anyB;
    fscan(A, nn, &loA, &hiA, &anyA);
    fscan(B, nn, &loB, &hiB, &anyB);
    memset(c, 0, sizeof *c);
    int spreadA = anyA ? hiA - loA : 0, spreadB = anyB ? hiB - loB : 0, L;
    if (force_bits > 0) {
        c->SA = c->SB = force_bits / 2;
        L = next_pow2(force_bits / 16);
    } else {
        c->SA = -loA;
        c->SB = -loB;
        int bitsA = 24 + spreadA + 1, bitsB = 24 + spreadB + 1;
        int bits = bitsA > bitsB ? bitsA : bitsB;
        int spread = spreadA > spreadB ? spreadA : spreadB;
        int need = (bits + 15) / 16, need2 = spread / 16 + 3;
        L = next_pow2(need > need2 ? need : need2);
        if (L < 2) L = 2;
    }
    c->n = n; c->L = L;
    if ((double)n * L * 65535.0 * 65535.0 > 4.0e18) return -1;
    c->A32 = calloc((size_t)L * nn, 4);
    c->B32 = calloc((size_t)L * nn, 4);
    c->Cw = calloc((size_t)(2 * L - 1) * nn, 8);
    return (c->A32 && c->B32 && c->Cw) ? 0 : -1;
}

/* src/fpfixed.c:175-193 */
static void encode_one(int32_t *plane, size_t nn, size_t idx, float x, int L, int S)
{
    if (x == 0.0f || !isfinite(x)) return;
    int e;
    float m = frexpf(x, &e);
    int32_t mi = (int32_t)(fabsf(m) * 16777216.0f);
    int off = e - 24 + S;
    if (off < 0) return;
    int lo = off >> 4, sh = off & 15;
    uint64_t v = (uint64_t)mi << sh;
    int sgn = x < 0.0f ? -1 : 1;
    for (int t = 0; t < 3; t++) {
        int w = lo + t;
        if (w >= L) break;
        plane[(size_t)w * nn + idx] = sgn * (int32_t)((v >> (16 * t)) & 0xFFFFu);
    }
}

/* src/fpfixed.c:195-204 */
void orc_fpx_encode(orc_fpx *c, const float *A, const float *B)
{
    size_t nn = (size_t)c->n * c->n;
    memset(c->A32, 0, (size_t)c->L * nn * 4);
    memset(c->B32, 0, (size_t)c->L * nn * 4);
    for (size_t i = 0; i < nn; i++) encode_one(c->A32, nn, i, A[i], c->L, c->SA);
    for (size_t i = 0; i < nn; i++) encode_one(c->B32, nn, i, B[i], c->L, c->SB);
}

/* extract + round_to + ldexpf for one entry: src/fpfixed.c:214-285.
 * cw holds the entry's 2L-1 unnormalised int64 planes. */
float orc_decode_f32_entry(const int64_t *cw, int L, int S)
{
    int RL = 2 * L + 2, P = 2 * L - 1;
    int32_t *limb = malloc((size_t)RL * 4);
    int64_t carry = 0;
    for (int w = 0; w < RL; w++) {
        int64_t t = (w < P ? cw[w] : 0) + carry;
        limb[w] = (int32_t)(t & 0xFFFF);
        carry = t >> 16;
    }
    int neg = carry < 0;
    if (neg) {
        int32_t borrow = 1;
        for (int w = 0; w < RL; w++) {
            int32_t t = (~limb[w] & 0xFFFF) + borrow;
            limb[w] = t & 0xFFFF;
            borrow = t >> 16;
        }
    }
    int h = -1;
    for (int w = RL - 1; w >= 0; w--) if (limb[w]) { h = w; break; }
    if (h < 0) { free(limb); return 0.0f; }
    int bl = 0;
    { int32_t v = limb[h]; while (v) { bl++; v >>= 1; } }
    int bitlen = 16 * h + bl;
    int k = h + 1 < 4 ? h + 1 : 4;
    uint64_t top = 0;
    for (int w = h; w > h - k; w--) top = (top << 16) | (uint64_t)limb[w];
    int base = 16 * (h - k + 1);
    int sticky = 0;
    for (int w = h - k; w >= 0; w--) if (limb[w]) { sticky = 1; break; }
    int tb = bitlen - base, shift = base;
    uint64_t sig = top;
    if (tb > 24) {
        int drop = tb - 24;
        uint64_t q = top >> drop, rem = top & ((1ULL << drop) - 1), half = 1ULL << (drop - 1);
        int up = rem > half ? 1 : rem < half ? 0 : (sticky ? 1 : (int)(q & 1));
        q += up;
        if (q >> 24) { q >>= 1; drop++; }
        shift += drop;
        sig = q;
    }
    free(limb);
    return (float)(neg ? -1 : 1) * ldexpf((float)sig, shift - S);
}

/* src/fpfixed.c:269-285 */
void orc_fpx_decode_f32(const orc_fpx *c, float *C)
{
    size_t nn = (size_t)c->n * c->n;
    int P = 2 * c->L - 1;
    int64_t *cw = malloc((size_t)P * 8);
    for (size_t i = 0; i < nn; i++) {
        for (int w = 0; w < P; w++) cw[w] = c->Cw[(size_t)w * nn + i];
        C[i] = orc_decode_f32_entry(cw, c->L, c->SA + c->SB);
    }
    free(cw);
}

void orc_fpx_free(orc_fpx *c)
{
    free(c->A32); free(c->B32); free(c->Cw);
    c->A32 = c->B32 = NULL; c->Cw = NULL;
}

/* Sampled entries of the fp32 path: the exact per-entry limb convolution of
 * the encoded row/column (grid sizing as orc_fpx_init), then the reference
 * decode.  out[s] = C[rows[s]][cols[s]]. */
void orc_fpx_entries(const float *A, const float *B, int n, int force_bits, int nsamp,
                     const int *rows, const int *cols, float *out)
{
    orc_fpx c;
    size_t nn = (size_t)n * n;
    /* sizing only: scan the full matrices exactly as fpx_init does */
    int loA, hiA, loB, hiB, anyA, anyB;
    fscan(A, nn, &loA, &hiA, &anyA);
    fscan(B, nn, &loB, &hiB, &anyB);
    memset(&c, 0, sizeof c);
    if (force_bits > 0) {
        c.SA = c.SB = force_bits / 2;
        c.L = next_pow2(force_bits / 16);
    } else {
        int spreadA = anyA ? hiA - loA : 0, spreadB = anyB ? hiB - loB : 0;
        c.SA = -loA; c.SB = -loB;
        int bitsA = 24 + spreadA + 1, bitsB = 24 + spreadB + 1;
        int bits = bitsA > bitsB ? bitsA : bitsB;
        int spread = spreadA > spreadB ? spreadA : spreadB;
        int need = (bits + 15) / 16, need2 = spread / 16 + 3;
        c.L = next_pow2(need > need2 ? need : need2);
        if (c.L < 2) c.L = 2;
    }
    int L = c.L, P = 2 * L - 1;
#pragma omp parallel
    {
        int32_t *a = calloc((size_t)L, 4), *b = calloc((size_t)L, 4);
        int64_t *cw = malloc((size_t)P * 8);
#pragma omp for schedule(dynamic)
        for (int s = 0; s < nsamp; s++) {
            memset(cw, 0, (size_t)P * 8);
            for (int k = 0; k < n; k++) {
                memset(a, 0, (size_t)L * 4);
                memset(b, 0, (size_t)L * 4);
                encode_one(a, 1, 0, A[(size_t)rows[s] * n + k], L, c.SA);
                encode_one(b, 1, 0, B[(size_t)k * n + cols[s]], L, c.SB);
                for (int u = 0; u < L; u++) {
                    if (!a[u]) continue;
                    for (int v = 0; v < L; v++) cw[u + v] += (int64_t)a[u] * b[v];
                }
            }
            out[s] = orc_decode_f32_entry(cw, L, c.SA + c.SB);
        }
        free(a); free(b); free(cw);
    }
}

/* ------------------------------------------------------------------ *
 * fp64 on the same grid (src/fpfixed.c:109-172, 308-322): 53-bit
 * significand, up to five limbs per entry through 128-bit staging, round once
 * to 53 bits, ldexp.
 * ------------------------------------------------------------------ */
/* src/fpfixed.c:115-128 */
static void dscan(const double *X, size_t nn, int *lo, int *hi, int *any)
{
    int l = 1 << 30, h = -(1 << 30), seen = 0;
    for (size_t i = 0; i < nn; i++) {
        double x = X[i];
        if (x == 0.0 || !isfinite(x)) continue;
        int e;
        frexp(x, &e);
        int e2 = e - 53;
        if (e2 < l) l = e2;
        if (e2 > h) h = e2;
        seen = 1;
    }
    if (!seen) { l = 0; h = 0; }
    *lo = l; *hi = h; *any = seen;
}

/* src/fpfixed.c:141-160 */
static void encode_one_d(int32_t *plane, size_t nn, size_t idx, double x, int L, int S)
{
    if (x == 0.0 || !isfinite(x)) return;
    int e;
    double m = frexp(x, &e);
    int64_t mi = (int64_t)(fabs(m) * 9007199254740992.0);
    int off = e - 53 + S;
    if (off < 0) return;
    int lo = off >> 4, sh = off & 15;
    unsigned __int128 v = (unsigned __int128)mi << sh;
    int sgn = x < 0.0 ? -1 : 1;
    for (int t = 0; t < 5; t++) {
        int w = lo + t;
        if (w >= L) break;
        uint64_t chunk = (uint64_t)(v >> (16 * t));
        plane[(size_t)w * nn + idx] = sgn * (int32_t)(chunk & 0xFFFFu);
    }
}

/* extract + round_to(53) + ldexp for one entry (src/fpfixed.c:214-265,
 * 308-322) */
double orc_decode_f64_entry(const int64_t *cw, int L, int S)
{
    int RL = 2 * L + 2, P = 2 * L - 1;
    int32_t *limb = malloc((size_t)RL * 4);
    int64_t carry = 0;
    for (int w = 0; w < RL; w++) {
        int64_t t = (w < P ? cw[w] : 0) + carry;
        limb[w] = (int32_t)(t & 0xFFFF);
        carry = t >> 16;
    }
    int neg = carry < 0;
    if (neg) {
        int32_t borrow = 1;
        for (int w = 0; w < RL; w++) {
            int32_t t = (~limb[w] & 0xFFFF) + borrow;
            limb[w] = t & 0xFFFF;
            borrow = t >> 16;
        }
    }
    int h = -1;
    for (int w = RL - 1; w >= 0; w--) if (limb[w]) { h = w; break; }
    if (h < 0) { free(limb); return 0.0; }
    int bl = 0;
    { int32_t v = limb[h]; while (v) { bl++; v >>= 1; } }
    int bitlen = 16 * h + bl;
    int k = h + 1 < 4 ? h + 1 : 4;
    uint64_t top = 0;
    for (int w = h; w > h - k; w--) top = (top << 16) | (uint64_t)limb[w];
    int base = 16 * (h - k + 1);
    int sticky = 0;
    for (int w = h - k; w >= 0; w--) if (limb[w]) { sticky = 1; break; }
    int tb = bitlen - base, shift = base;
    uint64_t sig = top;
    if (tb > 53) {
        int drop = tb - 53;
        uint64_t q = top >> drop, rem = top & ((1ULL << drop) - 1), half = 1ULL << (drop - 1);
        int up = rem > half ? 1 : rem < half ? 0 : (sticky ? 1 : (int)(q & 1));
        q += up;
        if (q >> 53) { q >>= 1; drop++; }
        shift += drop;
        sig = q;
    }
    free(limb);
    return (double)(neg ? -1 : 1) * ldexp((double)sig, shift - S);
}

/* Sampled entries of the fp64 path (grid sizing of src/fpfixed.c:59-78 with
 * sig 53, five limbs touched) */
void orc_fpx64_entries(const double *A, const double *B, int n, int force_bits, int nsamp,
                       const int *rows, const int *cols, double *out)
{
    size_t nn = (size_t)n * n;
    int loA, hiA, loB, hiB, anyA, anyB, SA, SB, L;
    dscan(A, nn, &loA, &hiA, &anyA);
    dscan(B, nn, &loB, &hiB, &anyB);
    if (force_bits > 0) {
        SA = SB = force_bits / 2;
        L = next_pow2(force_bits / 16);
    } else {
        int spreadA = anyA ? hiA - loA : 0, spreadB = anyB ? hiB - loB : 0;
        SA = -loA; SB = -loB;
        int bitsA = 53 + spreadA + 1, bitsB = 53 + spreadB + 1;
        int bits = bitsA > bitsB ? bitsA : bitsB;
        int spread = spreadA > spreadB ? spreadA : spreadB;
        int need = (bits + 15) / 16, need2 = spread / 16 + 5;
        L = next_pow2(need > need2 ? need : need2);
        if (L < 2) L = 2;
    }
    int P = 2 * L - 1;
#pragma omp parallel
    {
        int32_t *a = calloc((size_t)L, 4), *b = calloc((size_t)L, 4);
        int64_t *cw = malloc((size_t)P * 8);
#pragma omp for schedule(dynamic)
        for (int s = 0; s < nsamp; s++) {
            memset(cw, 0, (size_t)P * 8);
            for (int k = 0; k < n; k++) {
                memset(a, 0, (size_t)L * 4);
                memset(b, 0, (size_t)L * 4);
                encode_one_d(a, 1, 0, A[(size_t)rows[s] * n + k], L, SA);
                encode_one_d(b, 1, 0, B[(size_t)k * n + cols[s]], L, SB);
                for (int u = 0; u < L; u++) {
                    if (!a[u]) continue;
                    for (int v = 0; v < L; v++) cw[u + v] += (int64_t)a[u] * b[v];
                }
            }
            out[s] = orc_decode_f64_entry(cw, L, SA + SB);
        }
        free(a); free(b); free(cw);
    }
}

/* ------------------------------------------------------------------ *
 * Size-independent property for full-size runs: every row and column sum
 * of C = A*B must match the matrix-vector products A*(B*1) and (1^T A)*B,
 * all taken modulo the Mersenne prime M = 2^61 - 1.  Entries of A, B, C
 * are reduced mod M from their full limb representation, so an error in
 * any limb of any entry changes a sum (up to a 2^-61 coincidence).
 * fmt 0: A, B are L uint16 limb planes (two's complement if is_signed);
 * fmt 1: A, B are int64 row-major.  C: RL two's complement uint16 planes.
 * Returns the number of mismatching rows plus columns.
 * ------------------------------------------------------------------ */
#define MP ((1ULL << 61) - 1)
static uint64_t mp_red(unsigned __int128 x)
{
    uint64_t lo = (uint64_t)(x & MP), hi = (uint64_t)(x >> 61);
    uint64_t r = lo + hi;
    while (r >= MP) r -= MP;
    return r;
}
static uint64_t mp_mul(uint64_t a, uint64_t b) { return mp_red((unsigned __int128)a * b); }
static uint64_t mp_add(uint64_t a, uint64_t b) { uint64_t r = a + b; return r >= MP ? r - MP : r; }
static uint64_t mp_pow2(int k) { return 1ULL << (k % 61); }
static uint64_t mp_neg(uint64_t a) { return a ? MP - a : 0; }

static uint64_t planes_mod(const uint16_t *p, size_t nn, size_t idx, int L, int is_signed)
{
    uint64_t v = 0;
    for (int u = 0; u < L; u++) v = mp_add(v, mp_mul(p[(size_t)u * nn + idx], mp_pow2(16 * u)));
    if (is_signed && (p[(size_t)(L - 1) * nn + idx] & 0x8000u)) v = mp_add(v, mp_neg(mp_pow2(16 * L)));
    return v;
}
static uint64_t entry_mod(const void *X, int fmt, size_t nn, size_t idx, int L, int is_signed)
{
    if (fmt == 1) {
        int64_t x = ((const int64_t *)X)[idx];
        if (x >= 0) return (uint64_t)x % MP;
        uint64_t mag = (uint64_t)(-(x + 1)) + 1;   /* |x|, exact also for INT64_MIN */
        return mp_neg(mag % MP);
    }
    return planes_mod((const uint16_t *)X, nn, idx, L, is_signed);
}

long long orc_checksum_modp(const void *A, const void *B, int fmt, int n, int L, int is_signed,
                            const uint16_t *Cp, int RL)
{
    size_t nn = (size_t)n * n;
    uint64_t *colA = calloc((size_t)n, 8), *rowB = calloc((size_t)n, 8);
    uint64_t *colC = calloc((size_t)n, 8), *rowC = calloc((size_t)n, 8);
    uint64_t *expC = calloc((size_t)n, 8), *expR = calloc((size_t)n, 8);
    long long bad = 0;
#pragma omp parallel for schedule(static)
    for (int k = 0; k < n; k++) {
        uint64_t sa = 0, sb = 0;
        for (int i = 0; i < n; i++) sa = mp_add(sa, entry_mod(A, fmt, nn, (size_t)i * n + k, L, is_signed));
        for (int j = 0; j < n; j++) sb = mp_add(sb, entry_mod(B, fmt, nn, (size_t)k * n + j, L, is_signed));
        colA[k] = sa;
        rowB[k] = sb;
    }
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        uint64_t e = 0, c = 0;
        for (int k = 0; k < n; k++)
            e = mp_add(e, mp_mul(colA[k], entry_mod(B, fmt, nn, (size_t)k * n + j, L, is_signed)));
        for (int i = 0; i < n; i++) c = mp_add(c, planes_mod(Cp, nn, (size_t)i * n + j, RL, 1));
        expC[j] = e;
        colC[j] = c;
    }
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        uint64_t e = 0, c = 0;
        for (int k = 0; k < n; k++)
            e = mp_add(e, mp_mul(entry_mod(A, fmt, nn, (size_t)i * n + k, L, is_signed), rowB[k]));
        for (int j = 0; j < n; j++) c = mp_add(c, planes_mod(Cp, nn, (size_t)i * n + j, RL, 1));
        expR[i] = e;
        rowC[i] = c;
    }
    for (int t = 0; t < n; t++) bad += (expC[t] != colC[t]) + (expR[t] != rowC[t]);
    free(colA); free(rowB); free(colC); free(rowC); free(expC); free(expR);
    return bad;
}
