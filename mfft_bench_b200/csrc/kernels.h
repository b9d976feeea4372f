// kernels.h -- argument blocks and launchers of the HBM-bound kernels
// (pack, forward transform, inverse transform + fold + carry, fp32 scan).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace mfftb {

enum PackFmt {
    PACK_U16PL = 0,    // uint16 limb planes [L16][n][n] (unsigned or two's complement)
    PACK_I64 = 1,      // int64 row-major [n][n]
    PACK_F32 = 2,      // fp32 row-major [n][n] on a fixed-point grid
    PACK_I32LIMB = 3,  // int32 limb planes [L][n][n], limbs are the digits (conv_mfft)
    PACK_F64 = 4,      // fp64 row-major [n][n] on a fixed-point grid (53-bit significand)
};

struct PackArgs {
    int fmt;
    const void* src;
    int n;             // source matrix dimension
    int row0;          // first source row (straight layout; row-block sharding)
    int L16;           // PACK_U16PL / PACK_I32LIMB: limb planes in the source
    int W;             // two's complement / magnitude width of integer entries
    int is_signed;
    int S_grid;        // PACK_F32: grid scale SA or SB
    int lo_bit;        // PACK_F32: first live bit of the window on the grid
    int trunc_rel;     // PACK_F32: 16*L_grid - lo_bit (bits at/above the grid top are dropped)
    int b;             // digit bits
    int Lb;            // digit planes to produce
    void* dst;         // int8 (or int32 for PACK_I32LIMB) planes [Lb][rows][ld]
    int rows, ld;      // output plane geometry
    long long plane;   // elements per output plane
    int transpose;     // 1: output row = source column
    int* err;
    int balanced;      // PACK_I64 only: balanced digits in [-2^(b-1), 2^(b-1)), b <= 8
};
int pack_launch(const PackArgs& a, cudaStream_t stream);

struct FwdArgs {
    const void* D;     // digit planes [Lb][..]: int8, int16 or int32 (dbytes 1, 2, 4)
    int dbytes;
    long long dplane;  // elements per digit plane
    int Lb;
    long long nelem;   // elements per plane to transform (rows * ld), multiple of 4
    int S, NB, K, g, nc, d;
    int lgS, lgK;      // log2 of S and K (all plan sizes are powers of two)
    int f_stack;       // 0: write Ahat [j][da][c]; 1: write F [j][db][r] (2K-1 planes);
                       // 2: Karatsuba operands [j][K + S]: Xhat[c], then Xhat[c] + Xhat[c+S];
                       // 3: two levels [j][K + 2S]: those, then Xhat[c] + Xhat[c+S/2] for
                       //    c = 0..S/2-1 and S..S+S/2-1;
                       // 4: [j][K + 2S + S/2]: those, then s[c] + s[c+S/2] (c < S/2) of
                       //    s[c] = Xhat[c] + Xhat[c+S]
    int8_t* out;
    long long oplane;  // bytes per output plane
    int* err;
    int b;             // digit width: every digit has |digit| <= 2^b
    int variant;       // 0 auto, 1 the generic kernel only (for comparisons)
    int dsum;          // digit sums (d = 3): digits lo, hi of the two-digit split, then
                       // lo + hi (the plan bounds it to int8)
};
int forward_launch(const FwdArgs& a, cudaStream_t stream);

enum InvOut {
    INV_U16 = 0,   // normalised two's complement 16-bit limb planes [RL][rows][ldo]
    INV_I64 = 1,   // unnormalised int64 limb-convolution planes [P][rows][ldo] (limb mode)
    INV_F32 = 2,   // fp32 [rows][ldo], rounded once (fpx_decode_f32 semantics)
    INV_F64 = 3,   // fp64 [rows][ldo], rounded once (fpx_decode_f64 semantics)
};

struct InvArgs {
    const int32_t* acc;   // [njobs][rows][lda] int32 job planes of the pointwise step
    long long acc_plane;
    int lda;
    int rows, cols;       // valid output rows / columns
    int S, NB, K, g, nW, nchunk;
    int log2NB, lgS, lgK, lgE;
    int b;                // radix bits of the output positions
    int positions;        // radix-2^b positions to fold and carry
    int out_kind;
    void* out;
    long long out_plane;  // elements between output planes
    int ldo;
    int RL;               // INV_U16: limbs to emit; INV_I64: planes to emit
    int bit_off;          // INV_F32 / INV_F64: true grid position of internal bit 0
    int S_scale;          // INV_F32 / INV_F64: SA + SB
    int elems;            // elements per CTA (power of two, <= 32)
    int* err;
    int variant;          // 0 auto, 1 the generic shared-memory kernel only, 2 the lane
                          // kernel wherever it covers the plan
    // schoolbook plans: acc holds job planes q = t * nchunk + ch (t < positions)
    // of C_t = sum_u A_u B_(t-u); planes of jobs without terms are not read
    int school;
    int LbA, LbB, U;
    // Karatsuba mode (K = 8, one digit class, one chunk): acc holds 21 job
    // planes per point j, q = j*21 + p*7 + s, coefficient s of the full
    // convolutions P0 = a0*b0, P1 = a1*b1, P2 = (a0+a1)*(b0+b1) (a = a0 +
    // y^4 a1); the half points (j = 0, NB/2) hold P0 only.  kara = 2: 25
    // job planes per point, q = j*25 + ...: the length-2 convolutions Q0, Q1,
    // Q2 of P0 (3 coefficients each, 0..8) and of P1 (9..17), from which
    // P = Q0 + y^2 (Q2 - Q0 - Q1) + y^4 Q1, then P2 (18..24).  kara = 3: 27,
    // the Q's of P2 at 18..26.  The register kernel reads every layout, the
    // lane kernel kara = 1 only.
    int kara;
    // digit sums (nW = 3): class w holds the products of digit w of A with
    // digit w of B -- lo*lo, hi*hi, (lo+hi)*(lo+hi) -- so Chat = (1 - 2^7) acc0
    // + (2^14 - 2^7) acc1 + 2^7 acc2 instead of the sum over w of 2^(7w) acc_w
    int dsum;
};
int inverse_launch(const InvArgs& a, cudaStream_t stream);

// weight of digit class w in Chat (see InvArgs::dsum)
__host__ __device__ inline int64_t inv_class_weight(int dsum, int w) {
    if (dsum) return w == 0 ? 1 - 128 : (w == 1 ? 16384 - 128 : 128);
    return (int64_t)1 << (7 * w);
}

// fp32 exponent scan of src/fpfixed.c:40-54: out[0] = min e2, out[1] = max e2,
// out[2] = any finite non-zero (e2 = frexp exponent - 24).
int scan_f32_launch(const float* X, long long count, int* out3, cudaStream_t stream);
// fp64 counterpart (src/fpfixed.c:115-128, e2 = frexp exponent - 53)
int scan_f64_launch(const double* X, long long count, int* out3, cudaStream_t stream);

// test-only host entries: the device decode rules run on the CPU
float decode_words_host(uint32_t* w, int nw, int bit_off, int S);
double decode_words_host_f64(uint32_t* w, int nw, int bit_off, int S);

}  // namespace mfftb
