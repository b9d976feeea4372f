/* refapi.c -- the reference's hot-path API (include/mfftbench_b200.h) on top
 * of the native B200 library (include/mfftgpu.h).
 *
 * The products run on the GPU through one process-wide context.  The
 * host-side helpers of the same header (bigmat_*, normalize_planes,
 * bigres_equal, fpx_encode/fpx_decode_f32) keep the reference's semantics
 * on caller-owned host buffers; each cites the reference lines it matches.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../../include/mfftbench_b200.h"
#include "../../include/mfftgpu.h"

long long g_kernel_calls = 0;
int g_mfft_profile = 0;
mfft_profile_t g_mfft_prof;

static mfftgpu_ctx *g_ctx = NULL;
static int g_status = 0;

int mfftb_last_status(void) { return g_status; }

static mfftgpu_ctx *default_ctx(void)
{
    if (g_ctx) return g_ctx;
    int dev = 0;
    const char *s = getenv("MFFTGPU_DEVICE");
    if (s) dev = atoi(s);
    int rc = mfftgpu_create(&g_ctx, dev);
    if (rc) {
        fprintf(stderr, "mfft: no usable B200 device (%s)\n", mfftgpu_status_string(rc));
        g_status = rc;
        g_ctx = NULL;
    }
    return g_ctx;
}

static int finish(mfftgpu_ctx *c, int rc, const char *what)
{
    g_status = rc;
    if (rc)
        fprintf(stderr, "mfft: %s failed: %s (%s)\n", what, mfftgpu_status_string(rc),
                c ? mfftgpu_last_error(c) : "");
    return rc;
}

static void account(mfftgpu_ctx *c, int n, int mode, int wA, int wB)
{
    mfftgpu_plan_info pi;
    /* plane products of the plan that ran (src/kernel.c:13 counts leaf calls) */
    if ((c && mfftgpu_last_plan(c, &pi) == 0) || mfftgpu_plan_info_get(n, mode, wA, wB, &pi) == 0)
        g_kernel_calls = pi.kind == 1 ? (long long)pi.LbA * pi.LbB
                                      : (long long)pi.NB * pi.K * pi.K * pi.dA * pi.dB;
    if (g_mfft_profile && c) {
        float ms[5];
        mfftgpu_last_phase_ms(c, ms);
        g_mfft_prof.pack += ms[0] * 1e-3;
        g_mfft_prof.transform += ms[1] * 1e-3;
        g_mfft_prof.pointwise += ms[2] * 1e-3;
        g_mfft_prof.fold += ms[3] * 1e-3;
        g_mfft_prof.n_fft += 3;
    }
}

/* ------------------------------------------------------------------ kernel names */
static const char *knames[KERNEL__COUNT] = {"ikj",      "blocked",  "packed",       "strassen",
                                            "winograd", "bitplane", "convk",        "convkara",
                                            "boolpack", "bitpack",  "boolstrassen", "booltiled",
                                            "sm100"};

const char *kernel_name(kernel_t k)
{
    if ((int)k < 0 || k >= KERNEL__COUNT) return "?";
    return knames[k];
}

int kernel_from_name(const char *s)
{
    for (int i = 0; i < KERNEL__COUNT; i++)
        if (s && strcmp(s, knames[i]) == 0) return i;
    return -1;
}

/* ------------------------------------------------------------------ profile */
void mfft_profile_reset(void) { memset(&g_mfft_prof, 0, sizeof g_mfft_prof); }

void mfft_profile_print(const char *label)
{
    double tot = g_mfft_prof.pack + g_mfft_prof.build_ops + g_mfft_prof.transform +
                 g_mfft_prof.pointwise + g_mfft_prof.fold;
    if (tot <= 0) tot = 1e-30;
    printf("profile %s (B200):\n"
           "  pack        %8.4f s  (%5.1f%%)\n"
           "  transform   %8.4f s  (%5.1f%%)  launches %lld\n"
           "  pointwise   %8.4f s  (%5.1f%%)\n"
           "  fold+carry  %8.4f s  (%5.1f%%)\n"
           "  total       %8.4f s\n",
           label ? label : "mfft", g_mfft_prof.pack, 100.0 * g_mfft_prof.pack / tot,
           g_mfft_prof.transform, 100.0 * g_mfft_prof.transform / tot, g_mfft_prof.n_fft,
           g_mfft_prof.pointwise, 100.0 * g_mfft_prof.pointwise / tot, g_mfft_prof.fold,
           100.0 * g_mfft_prof.fold / tot, tot);
}

/* ------------------------------------------------------------------ bigmat helpers */
double now_sec(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

uint16_t *bigmat_alloc(int n, int L) { return calloc((size_t)n * n * L, sizeof(uint16_t)); }

/* splitmix64 stream, one 16-bit limb per draw (src/bigmat.c:20-35) */
void bigmat_rand(uint16_t *m, int n, int L, uint64_t seed)
{
    uint64_t s = seed;
    size_t total = (size_t)n * n * L;
    for (size_t i = 0; i < total; i++) {
        uint64_t z = (s += 0x9E3779B97F4A7C15ULL);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        m[i] = (uint16_t)((z ^ (z >> 31)) & LIMB_MASK);
    }
}

uint16_t *bigmat_to_entry_major(const uint16_t *plane, int n, int L)
{
    uint16_t *e = bigmat_alloc(n, L);
    if (!e) return NULL;
    size_t nn = (size_t)n * n;
    for (int u = 0; u < L; u++)
        for (size_t idx = 0; idx < nn; idx++) e[idx * L + u] = plane[(size_t)u * nn + idx];
    return e;
}

/* carry with arithmetic shifts into RL 16-bit limbs (src/bigmat.c:48-60) */
void normalize_planes(const int64_t *acc, int nplanes, int n, uint16_t *out, int RL)
{
    size_t nn = (size_t)n * n;
#pragma omp parallel for schedule(static)
    for (long long idx = 0; idx < (long long)nn; idx++) {
        int64_t carry = 0;
        for (int w = 0; w < RL; w++) {
            int64_t v = (w < nplanes ? acc[(size_t)w * nn + idx] : 0) + carry;
            out[(size_t)w * nn + idx] = (uint16_t)(v & LIMB_MASK);
            carry = v >> LIMB_BITS;
        }
    }
}

int bigres_equal(const uint16_t *a, const uint16_t *b, int n, int RL, int *bad_i, int *bad_j,
                 int *bad_w)
{
    size_t nn = (size_t)n * n;
    for (int w = 0; w < RL; w++)
        for (size_t idx = 0; idx < nn; idx++)
            if (a[(size_t)w * nn + idx] != b[(size_t)w * nn + idx]) {
                if (bad_w) *bad_w = w;
                if (bad_i) *bad_i = (int)(idx / n);
                if (bad_j) *bad_j = (int)(idx % n);
                return 0;
            }
    return 1;
}

/* ------------------------------------------------------------------ workload generators */
static uint64_t sm64_at(uint64_t seed, uint64_t t)
{
    uint64_t z = seed + (t + 1) * 0x9E3779B97F4A7C15ULL; /* draw t of the splitmix64 stream */
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static float normal_at(uint64_t seed, uint64_t t)
{
    double u1 = ((double)(sm64_at(seed, t) >> 11) + 0.5) * 0x1.0p-53;
    double u2 = ((double)(sm64_at(seed, t + 1) >> 11) + 0.5) * 0x1.0p-53;
    int k = (int)(sm64_at(seed, t + 2) % 17u) - 8;
    double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    return ldexpf((float)z, k);
}

void mfftgpu_gen_normal_f32(float *A, float *B, size_t count, uint64_t seed)
{
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)count; i++) {
        A[i] = normal_at(seed, 3 * (uint64_t)i);
        B[i] = normal_at(seed, 3 * ((uint64_t)count + (uint64_t)i));
    }
}

/* ------------------------------------------------------------------ plan */
static int ilog2i(int x)
{
    int r = 0;
    while ((1 << r) < x) r++;
    return r;
}

/* same acceptance rules and fields as src/mfft.c:77-95 */
int mfft_plan_init(mfft_plan *p, int L, int sigma_override)
{
    if (!p || L < 2 || (L & (L - 1))) return -1;
    int l = ilog2i(L);
    int sigma = sigma_override > 0 ? sigma_override : l / 2;
    if (sigma < 1) sigma = 1;
    if (sigma > l) return -1;
    int S = 1 << sigma, NB = 2 * L / S, K = 2 * S;
    if (2 * S * S < L) return -1;
    if ((2 * K) % NB) return -1;
    if (NB < 2) return -1;
    p->L = L;
    p->S = S;
    p->NB = NB;
    p->K = K;
    p->g = 2 * K / NB;
    p->rec = 0;
    p->nprod = (long long)NB * K * K;
    return 0;
}

long long mfft_plan_products(const mfft_plan *p)
{
    return p->nprod ? p->nprod : (long long)p->NB * p->K * p->K;
}

/* src/mfft.c:102-110: worst-case bits of the reference's int64 intermediates */
double mfft_plan_maxbits(const mfft_plan *p, int n)
{
    return 3.0 * log2((double)p->NB) + log2((double)p->K) + log2((double)n) + 2.0 * LIMB_BITS;
}

void mfft_plan_describe(const mfft_plan *p, int n)
{
    mfftgpu_plan_info pi;
    printf("MFFT plan: L=%d limbs per entry (scalar width %d bits)  S=%d  NB=%d  K=%d  "
           "omega=I_%d^%d\n",
           p->L, p->L * LIMB_BITS, p->S, p->NB, p->K, ilog2i(p->K), p->g);
    if (mfftgpu_plan_info_get(n, 0, 16 * p->L, 16 * p->L, &pi) == 0)
        printf("           B200 plan: %d-bit digits S=%d NB=%d K=%d int8 split %dx%d -> %lld "
               "int8 plane products (limb-plane schoolbook %d)\n",
               pi.b, pi.S, pi.NB, pi.K, pi.dA, pi.dB,
               (long long)pi.NB * pi.K * pi.K * pi.dA * pi.dB, pi.LbA * pi.LbB);
}

/* ------------------------------------------------------------------ recursive plan
 * src/mfft.c:449-527,665-686.  The reference's recursive plan solves each
 * point's negacyclic convolution of length 2^k either by Karatsuba (3^k
 * products) or by splitting it into 2^nu blocks carried in a ring of length
 * 2^(k+1-nu) whose block products recurse one level down (2^nu times the
 * cost below); a choice whose int64 intermediates could pass 62 bits is
 * refused.  The cost model and its tie rules are kept so that a recursive plan
 * has the reference's S, NB, K and product count.  The product itself runs on
 * the B200 path like every other plan: the exact result does not depend on
 * the plan, and the GPU's own planner picks the int8 schedule (whose ring
 * products are themselves split by Karatsuba on the W = 64 plan). */
enum { NEG_KMAX = 26, NEG_MMAX = 74 }; /* the reference's table bounds, mfft.c:480-481 */

typedef struct {
    long long cost;
    int outbits, maxbits, ok;
} negcost;

typedef struct {
    negcost v[NEG_KMAX][NEG_MMAX];
    unsigned char done[NEG_KMAX][NEG_MMAX];
    int ln; /* ceil(log2 n) */
} negmemo;

static negcost neg_cost(negmemo *m, int k, int mbits)
{
    negcost none = {0, 0, 0, 0};
    if (k < 0 || k >= NEG_KMAX || mbits < 0 || mbits >= NEG_MMAX) return none;
    if (m->done[k][mbits]) return m->v[k][mbits];
    negcost best = none;
    /* Karatsuba on the whole convolution: the folded result needs
     * 1 + k + ln + 2 mbits bits, its intermediates one more */
    const int kbits = 2 + k + m->ln + 2 * mbits;
    if (kbits <= 62) {
        long long c = 1;
        for (int i = 0; i < k; i++) c *= 3;
        best.cost = c;
        best.outbits = kbits - 1;
        best.maxbits = kbits;
        best.ok = 1;
    }
    for (int nu = 2; 2 * nu <= k + 1; nu++) {
        negcost sub = neg_cost(m, k + 1 - nu, mbits + nu);
        if (!sub.ok) continue;
        const int top = sub.maxbits > nu + sub.outbits ? sub.maxbits : nu + sub.outbits;
        if (top > 62) continue;
        const long long c = ((long long)1 << nu) * sub.cost;
        if (!best.ok || c < best.cost) {
            best.cost = c;
            best.outbits = sub.outbits + 1;
            best.maxbits = top;
            best.ok = 1;
        }
    }
    m->done[k][mbits] = 1;
    m->v[k][mbits] = best;
    return best;
}

int mfft_plan_init_rec(mfft_plan *p, int L, int n, int sigma_override)
{
    if (!p || L < 2 || (L & (L - 1))) return -1;
    negmemo *m = calloc(1, sizeof *m);
    if (!m) return -1;
    m->ln = ilog2i(n);
    const int l = ilog2i(L);
    long long best = -1;
    int pick = 0;
    for (int sigma = 1; sigma < l; sigma++) {
        const int S = 1 << sigma, NB = 2 * L / S, K = 2 * S;
        if (2 * S * S < L || (2 * K) % NB || NB < 2) continue;
        if (sigma_override > 0 && sigma != sigma_override) continue;
        const negcost c = neg_cost(m, sigma + 1, LIMB_BITS + ilog2i(NB));
        if (!c.ok) continue;
        const long long total = (long long)NB * c.cost;
        if (best < 0 || total < best) {
            best = total;
            pick = sigma;
        }
    }
    free(m);
    if (best < 0) return -1;
    p->L = L;
    p->S = 1 << pick;
    p->NB = 2 * L / p->S;
    p->K = 2 * p->S;
    p->g = 2 * p->K / p->NB;
    p->rec = 1;
    p->nprod = best;
    return 0;
}

/* src/mfft.c:560-662: C = A * B mod (y^K + 1), A and B K int32 planes of
 * n x n matrices, C K int64 planes.  It runs on the GPU as one limb
 * convolution: every int32 entry x splits into signed 16-bit limbs
 * x = 2^16 h + l, coefficient u of A (and of B) becomes limbs 3u (l) and
 * 3u + 1 (h), with limb 3u + 2 left zero so that the limb products of
 * different coefficient pairs never share a slot; then
 * lin[t] = Cw[3t] + 2^16 Cw[3t+1] + 2^32 Cw[3t+2] (modulo 2^64, exact where
 * the product fits int64, as the reference requires) and
 * C[w] = lin[w] - lin[w + K]. */
void ssa_negconv(int64_t *C, const int32_t *A, const int32_t *B, int K, int n, int Mbits,
                 kernel_t kern)
{
    (void)Mbits;
    (void)kern;
    if (!C || !A || !B || K < 1 || n < 1) {
        finish(NULL, MFFTGPU_ERR_ARG, "ssa_negconv");
        return;
    }
    const size_t nn = (size_t)n * n;
    const int Lx = 3 * K - 1, P = 2 * Lx - 1;
    int32_t *As = calloc((size_t)Lx * nn, sizeof(int32_t));
    int32_t *Bs = calloc((size_t)Lx * nn, sizeof(int32_t));
    int64_t *Cw = malloc((size_t)P * nn * sizeof(int64_t));
    mfftgpu_ctx *c = (As && Bs && Cw) ? default_ctx() : NULL;
    int rc = !(As && Bs && Cw) ? MFFTGPU_ERR_NOMEM : (c ? 0 : g_status);
    if (c) {
        for (int u = 0; u < K; u++)
            for (size_t i = 0; i < nn; i++) {
                const int32_t a = A[(size_t)u * nn + i], b = B[(size_t)u * nn + i];
                const int32_t al = (int16_t)(uint16_t)((uint32_t)a & 0xFFFFu);
                const int32_t bl = (int16_t)(uint16_t)((uint32_t)b & 0xFFFFu);
                As[(size_t)(3 * u) * nn + i] = al;
                As[(size_t)(3 * u + 1) * nn + i] = (int32_t)(((int64_t)a - al) >> 16);
                Bs[(size_t)(3 * u) * nn + i] = bl;
                Bs[(size_t)(3 * u + 1) * nn + i] = (int32_t)(((int64_t)b - bl) >> 16);
            }
        mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
        rc = mfftgpu_conv_i32(c, As, Bs, n, Lx, Cw);
    }
    if (!finish(c, rc, "ssa_negconv")) {
        for (int w = 0; w < K; w++)
            for (size_t i = 0; i < nn; i++) {
                uint64_t v = 0;
                for (int hi = 0; hi < 2; hi++) {
                    const int t = w + hi * K;
                    if (t > 2 * K - 2) break;
                    const uint64_t lin = (uint64_t)Cw[(size_t)(3 * t) * nn + i] +
                                         ((uint64_t)Cw[(size_t)(3 * t + 1) * nn + i] << 16) +
                                         ((uint64_t)Cw[(size_t)(3 * t + 2) * nn + i] << 32);
                    v = hi ? v - lin : v + lin;
                }
                C[(size_t)w * nn + i] = (int64_t)v;
            }
        account(c, n, 1, Lx, Lx);
    } else {
        memset(C, 0, (size_t)K * nn * sizeof(int64_t));
    }
    free(As);
    free(Bs);
    free(Cw);
}

/* ------------------------------------------------------------------ products */
void mm_mfft(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, const mfft_plan *p,
             kernel_t k, uint16_t *out, int RL)
{
    (void)k;
    if (p && p->L != L) {
        finish(NULL, MFFTGPU_ERR_ARG, "mm_mfft (plan L mismatch)");
        return;
    }
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int rc = mfftgpu_mm_u16(c, Apl, Bpl, n, L, 0, out, RL);
    if (finish(c, rc, "mm_mfft")) {
        memset(out, 0, (size_t)RL * n * n * sizeof(uint16_t));
        return;
    }
    account(c, n, 0, 16 * L, 16 * L);
}

void mm_mfft_signed(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, uint16_t *out, int RL)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int rc = mfftgpu_mm_u16(c, Apl, Bpl, n, L, 1, out, RL);
    if (finish(c, rc, "mm_mfft_signed")) {
        memset(out, 0, (size_t)RL * n * n * sizeof(uint16_t));
        return;
    }
    account(c, n, 0, 16 * L, 16 * L);
}

void conv_mfft(int64_t *Cw, const int32_t *A32, const int32_t *B32, int n, int L,
               const mfft_plan *p, kernel_t k)
{
    (void)k;
    if (p && p->L != L) {
        finish(NULL, MFFTGPU_ERR_ARG, "conv_mfft (plan L mismatch)");
        return;
    }
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int rc = mfftgpu_conv_i32(c, A32, B32, n, L, Cw);
    if (finish(c, rc, "conv_mfft")) {
        memset(Cw, 0, (size_t)(2 * L - 1) * n * n * sizeof(int64_t));
        return;
    }
    account(c, n, 1, L, L);
}

/* Limb-plane schoolbook (src/methods.c:94-123): the same exact products as
 * mm_mfft / conv_mfft, computed as digit-plane GEMMs A_u B_v on the tensor
 * cores without a transform. */
static int with_school(mfftgpu_ctx *c, int on)
{
    int prev = mfftgpu_get_method(c);
    mfftgpu_set_method(c, on);
    return prev;
}

void mm_limbplane(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, kernel_t k,
                  uint16_t *out, int RL)
{
    (void)k;
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int prev = with_school(c, 1);
    int rc = mfftgpu_mm_u16(c, Apl, Bpl, n, L, 0, out, RL);
    with_school(c, prev);
    if (finish(c, rc, "mm_limbplane")) {
        memset(out, 0, (size_t)RL * n * n * sizeof(uint16_t));
        return;
    }
    account(c, n, 2, 16 * L, 16 * L);
}

void mm_limbplane_signed(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, uint16_t *out,
                         int RL)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int prev = with_school(c, 1);
    int rc = mfftgpu_mm_u16(c, Apl, Bpl, n, L, 1, out, RL);
    with_school(c, prev);
    if (finish(c, rc, "mm_limbplane_signed")) {
        memset(out, 0, (size_t)RL * n * n * sizeof(uint16_t));
        return;
    }
    account(c, n, 2, 16 * L, 16 * L);
}

/* conv_limbplane's unnormalised planes Cw[w] = sum_{u+v=w} A_u B_v depend on
 * the caller's limb split, so they come from the limb-mode plan (the same
 * values conv_mfft returns). */
void conv_limbplane(int64_t *Cw, const int32_t *A32, const int32_t *B32, int n, int L,
                    kernel_t k)
{
    (void)k;
    mfftgpu_ctx *c = default_ctx();
    if (!c) return;
    mfftgpu_set_profile(c, g_mfft_profile ? 1 : 0);
    int rc = mfftgpu_conv_i32(c, A32, B32, n, L, Cw);
    if (finish(c, rc, "conv_limbplane")) {
        memset(Cw, 0, (size_t)(2 * L - 1) * n * n * sizeof(int64_t));
        return;
    }
    account(c, n, 1, L, L);
}

int fpx_gemm_f32_limbplane(const float *A, const float *B, int n, int force_bits, float *C)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return g_status;
    int prev = with_school(c, 1);
    int rc = mfftgpu_fp32(c, A, B, n, force_bits, C);
    with_school(c, prev);
    return finish(c, rc, "fpx_gemm_f32_limbplane");
}

int fpx_gemm_f32(const float *A, const float *B, int n, int force_bits, float *C)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return g_status;
    return finish(c, mfftgpu_fp32(c, A, B, n, force_bits, C), "fpx_gemm_f32");
}

/* ------------------------------------------------------------------ fp32 embedding (host side) */
static int next_pow2(int x)
{
    int r = 1;
    while (r < x) r <<= 1;
    return r;
}

/* exponent range of finite non-zero fp64 entries, e2 = frexp exponent - 53
 * (src/fpfixed.c:115-128) */
static void dscan(const double *X, size_t nn, int *lo, int *hi, int *any)
{
    int l = 1 << 30, h = -(1 << 30), seen = 0;
    for (size_t i = 0; i < nn; i++) {
        double x = X[i];
        if (x == 0.0 || !isfinite(x)) continue;
        int e;
        frexp(x, &e);
        if (e - 53 < l) l = e - 53;
        if (e - 53 > h) h = e - 53;
        seen = 1;
    }
    if (!seen) l = h = 0;
    *lo = l;
    *hi = h;
    *any = seen;
}

/* exponent range of finite non-zero entries, e2 = frexp exponent - 24
 * (src/fpfixed.c:40-54) */
static void fscan(const float *X, size_t nn, int *lo, int *hi, int *any)
{
    int l = 1 << 30, h = -(1 << 30), seen = 0;
    for (size_t i = 0; i < nn; i++) {
        float x = X[i];
        if (x == 0.0f || !isfinite(x)) continue;
        int e;
        frexpf(x, &e);
        if (e - 24 < l) l = e - 24;
        if (e - 24 > h) h = e - 24;
        seen = 1;
    }
    if (!seen) l = h = 0;
    *lo = l;
    *hi = h;
    *any = seen;
}

/* grid sizing and allocation shared by both precisions (src/fpfixed.c:59-94):
 * sig = significand bits, wr = limbs one shifted significand can touch */
static int fpx_setup(fpx_ctx *c, int n, int force_bits, int sig, int wr, int loA, int hiA,
                     int anyA, int loB, int hiB, int anyB)
{
    size_t nn = (size_t)n * n;
    memset(c, 0, sizeof *c);
    c->sig = sig;
    c->spreadA = anyA ? hiA - loA : 0;
    c->spreadB = anyB ? hiB - loB : 0;
    int L;
    if (force_bits > 0) {
        c->SA = c->SB = force_bits / 2;
        L = next_pow2(force_bits / LIMB_BITS);
    } else {
        c->SA = -loA;
        c->SB = -loB;
        int bitsA = sig + c->spreadA + 1, bitsB = sig + c->spreadB + 1;
        int bits = bitsA > bitsB ? bitsA : bitsB;
        int spread = c->spreadA > c->spreadB ? c->spreadA : c->spreadB;
        int need = (bits + LIMB_BITS - 1) / LIMB_BITS, need2 = spread / LIMB_BITS + wr;
        L = next_pow2(need > need2 ? need : need2);
        if (L < 2) L = 2;
    }
    c->n = n;
    c->L = L;
    if ((double)n * L * 65535.0 * 65535.0 > 4.0e18) {
        fprintf(stderr, "fpx: n=%d L=%d would overflow int64 accumulators\n", n, L);
        return -1;
    }
    c->A32 = calloc((size_t)L * nn, sizeof(int32_t));
    c->B32 = calloc((size_t)L * nn, sizeof(int32_t));
    c->Cw = calloc((size_t)(2 * L - 1) * nn, sizeof(int64_t));
    if (!c->A32 || !c->B32 || !c->Cw) {
        fpx_free(c);
        return -1;
    }
    return 0;
}

/* src/fpfixed.c:96-108 */
int fpx_init(fpx_ctx *c, const float *A, const float *B, int n, int force_bits)
{
    size_t nn = (size_t)n * n;
    int loA, hiA, loB, hiB, anyA, anyB;
    fscan(A, nn, &loA, &hiA, &anyA);
    fscan(B, nn, &loB, &hiB, &anyB);
    return fpx_setup(c, n, force_bits, 24, 3, loA, hiA, anyA, loB, hiB, anyB);
}

/* src/fpfixed.c:130-140: a 53-bit significand shifted by up to 15 touches
 * five limbs */
int fpx_init_d(fpx_ctx *c, const double *A, const double *B, int n, int force_bits)
{
    size_t nn = (size_t)n * n;
    int loA, hiA, loB, hiB, anyA, anyB;
    dscan(A, nn, &loA, &hiA, &anyA);
    dscan(B, nn, &loB, &hiB, &anyB);
    return fpx_setup(c, n, force_bits, 53, 5, loA, hiA, anyA, loB, hiB, anyB);
}

/* significand shifted onto the grid, up to three signed 16-bit limbs
 * (src/fpfixed.c:175-193) */
static void encode_entry(int32_t *plane, size_t nn, size_t idx, float x, int L, int S)
{
    if (x == 0.0f || !isfinite(x)) return;
    int e;
    float m = frexpf(x, &e);
    uint64_t mi = (uint64_t)(fabsf(m) * 16777216.0f);
    int off = e - 24 + S;
    if (off < 0) return;
    int lo = off >> 4;
    uint64_t v = mi << (off & 15);
    int32_t sgn = x < 0.0f ? -1 : 1;
    for (int t = 0; t < 3 && lo + t < L; t++)
        plane[(size_t)(lo + t) * nn + idx] = sgn * (int32_t)((v >> (16 * t)) & 0xFFFFu);
}

/* fp64 significand on the grid through 128-bit staging, up to five signed
 * 16-bit limbs (src/fpfixed.c:141-160) */
static void encode_entry_d(int32_t *plane, size_t nn, size_t idx, double x, int L, int S)
{
    if (x == 0.0 || !isfinite(x)) return;
    int e;
    double m = frexp(x, &e);
    uint64_t mi = (uint64_t)(fabs(m) * 9007199254740992.0);
    int off = e - 53 + S;
    if (off < 0) return;
    int lo = off >> 4;
    unsigned __int128 v = (unsigned __int128)mi << (off & 15);
    int32_t sgn = x < 0.0 ? -1 : 1;
    for (int t = 0; t < 5 && lo + t < L; t++)
        plane[(size_t)(lo + t) * nn + idx] = sgn * (int32_t)((uint64_t)(v >> (16 * t)) & 0xFFFFu);
}

void fpx_encode_d(fpx_ctx *c, const double *A, const double *B)
{
    size_t nn = (size_t)c->n * c->n;
    double t0 = now_sec();
    memset(c->A32, 0, (size_t)c->L * nn * sizeof(int32_t));
    memset(c->B32, 0, (size_t)c->L * nn * sizeof(int32_t));
    for (size_t i = 0; i < nn; i++) encode_entry_d(c->A32, nn, i, A[i], c->L, c->SA);
    for (size_t i = 0; i < nn; i++) encode_entry_d(c->B32, nn, i, B[i], c->L, c->SB);
    c->enc_secs = now_sec() - t0;
}

void fpx_encode(fpx_ctx *c, const float *A, const float *B)
{
    size_t nn = (size_t)c->n * c->n;
    double t0 = now_sec();
    memset(c->A32, 0, (size_t)c->L * nn * sizeof(int32_t));
    memset(c->B32, 0, (size_t)c->L * nn * sizeof(int32_t));
    for (size_t i = 0; i < nn; i++) encode_entry(c->A32, nn, i, A[i], c->L, c->SA);
    for (size_t i = 0; i < nn; i++) encode_entry(c->B32, nn, i, B[i], c->L, c->SB);
    c->enc_secs = now_sec() - t0;
}

/* carry the 2L-1 planes of one entry into 32-bit two's complement words,
 * then the shared device rounding rule (extract + round_to + ldexpf,
 * src/fpfixed.c:212-285) */
void fpx_decode_f32(fpx_ctx *c, float *C)
{
    size_t nn = (size_t)c->n * c->n;
    int P = 2 * c->L - 1, RL = 2 * c->L + 2;
    int nw = (RL + 1) / 2 + 1;
    int S = c->SA + c->SB;
    double t0 = now_sec();
#pragma omp parallel
    {
        uint32_t *w = malloc((size_t)nw * sizeof(uint32_t));
#pragma omp for schedule(static)
        for (long long i = 0; i < (long long)nn; i++) {
            int64_t carry = 0;
            memset(w, 0, (size_t)nw * sizeof(uint32_t));
            for (int k = 0; k < 2 * nw; k++) {
                int64_t v = (k < P ? c->Cw[(size_t)k * nn + i] : 0) + carry;
                w[k >> 1] |= (uint32_t)(v & 0xFFFF) << (16 * (k & 1));
                carry = v >> 16;
            }
            C[i] = mfftgpu_decode_words_f32(w, nw, 0, S);
        }
        free(w);
    }
    c->dec_secs = now_sec() - t0;
}

/* the exact value of entry i as 32-bit two's complement words */
static void entry_words(const fpx_ctx *c, size_t nn, long long i, uint32_t *w, int nw)
{
    int P = 2 * c->L - 1;
    int64_t carry = 0;
    memset(w, 0, (size_t)nw * sizeof(uint32_t));
    for (int k = 0; k < 2 * nw; k++) {
        int64_t v = (k < P ? c->Cw[(size_t)k * nn + i] : 0) + carry;
        w[k >> 1] |= (uint32_t)(v & 0xFFFF) << (16 * (k & 1));
        carry = v >> 16;
    }
}

/* src/fpfixed.c:308-322: round once to 53 bits */
void fpx_decode_f64(fpx_ctx *c, double *C)
{
    size_t nn = (size_t)c->n * c->n;
    int RL = 2 * c->L + 2;
    int nw = (RL + 1) / 2 + 1;
    int S = c->SA + c->SB;
    double t0 = now_sec();
#pragma omp parallel
    {
        uint32_t *w = malloc((size_t)nw * sizeof(uint32_t));
#pragma omp for schedule(static)
        for (long long i = 0; i < (long long)nn; i++) {
            entry_words(c, nn, i, w, nw);
            C[i] = mfftgpu_decode_words_f64(w, nw, 0, S);
        }
        free(w);
    }
    c->dec_secs = now_sec() - t0;
}

/* src/fpfixed.c:291-306: the reference-precision decode, rounded to the
 * 64-bit significand of x86 long double (ldexpl of the host libm) */
void fpx_decode_ld(fpx_ctx *c, long double *C)
{
    size_t nn = (size_t)c->n * c->n;
    int RL = 2 * c->L + 2;
    int nw = (RL + 1) / 2 + 1;
    int S = c->SA + c->SB;
    uint32_t *w = malloc((size_t)nw * sizeof(uint32_t));
    if (!w) return;
    for (long long i = 0; i < (long long)nn; i++) {
        entry_words(c, nn, i, w, nw);
        uint64_t sig;
        int shift;
        int sgn = mfftgpu_decode_words_round(w, nw, 0, 63, &sig, &shift);
        C[i] = sgn ? (long double)sgn * ldexpl((long double)sig, shift - S) : 0.0L;
    }
    free(w);
}

int fpx_gemm_f64(const double *A, const double *B, int n, int force_bits, double *C)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return g_status;
    return finish(c, mfftgpu_fp64(c, A, B, n, force_bits, C), "fpx_gemm_f64");
}

int fpx_gemm_f64_limbplane(const double *A, const double *B, int n, int force_bits, double *C)
{
    mfftgpu_ctx *c = default_ctx();
    if (!c) return g_status;
    int prev = with_school(c, 1);
    int rc = mfftgpu_fp64(c, A, B, n, force_bits, C);
    with_school(c, prev);
    return finish(c, rc, "fpx_gemm_f64_limbplane");
}

void fpx_free(fpx_ctx *c)
{
    free(c->A32);
    free(c->B32);
    free(c->Cw);
    c->A32 = c->B32 = NULL;
    c->Cw = NULL;
}
