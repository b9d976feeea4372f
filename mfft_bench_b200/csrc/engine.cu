// engine.cu -- host orchestration of the B200 MFFT path and the native C ABI
// (include/mfftgpu.h).
//
// One product = pack(B, transposed) -> forward(F stack) once, then for each
// row block of A: pack(A) -> forward(Ahat) -> tcgen05 pointwise -> inverse +
// fold + carry straight into the caller's output rows.  Row blocks bound the
// device workspace (the reference mallocs NB*K full planes per call,
// src/mfft.c:310-316; here only F is kept whole) and are also the unit of
// multi-GPU sharding: a rank computes rows [row_begin, row_end).  Schoolbook
// plans skip both transforms (the digit planes are the tensor-core operands)
// and finish with the streaming carry.  The host-pointer entry points
// overlap their uploads and read-backs with the compute of row chunks.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>

#include "../../include/mfftgpu.h"
#include "decode.cuh"
#include "kernels.h"
#include "plan.h"
#include "runtime.h"

using namespace mfftb;

// Karatsuba level of the pointwise step where a plan allows it (the W = 64
// plans): 2 splits P0 and P1 into length-2 convolutions as well, 3 also P2
constexpr int kDefaultKara = 3;

struct mfftgpu_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    cudaStream_t copy_stream = nullptr;  // device->host reads of the host-pointer entry points
    cudaStream_t up_stream = nullptr;    // host->device uploads of the host-pointer entry points
    cudaEvent_t chunk_ev[8] = {};
    cudaEvent_t up_ev[9] = {};
    int* d_err = nullptr;    // device status word
    int* d_scan = nullptr;   // fp32 exponent scan results
    char* ws = nullptr;      // grow-only workspace
    size_t ws_bytes = 0;
    size_t ws_limit = 0;
    char* io = nullptr;      // grow-only staging for the host-pointer entry points
    size_t io_bytes = 0;
    unsigned long long timeout_ns = 4000000000ull;
    int profile = 0;  // 0 off, 1 last product, 2 accumulate across products
    // profiling: start/end events per launch, recorded without host syncs;
    // times are read back lazily by mfftgpu_last_phase_ms
    // (2 events per launch: 2048 launches, e.g. 100 products of 14 launches)
    static constexpr int kMaxEv = 4096;
    cudaEvent_t ev[kMaxEv] = {};
    int ev_phase[kMaxEv / 2] = {};
    int ev_used = 0;
    int ev_dropped = 0;  // launches past the event capacity, not in the phase times
    float phase_ms[5] = {};
    bool phase_valid = true;
    int launches = 0;
    int raster = 0, group_m = 0;  // pointwise tile order (tuning)
    int pw_variant = 0;           // pointwise kernel: 0 auto, 1 single CTA, 2 CTA pairs, 3 grouped
    int wave_sync = 1;            // wave alignment of the t-grouped kernel
    int half_points = 1;          // skip the zero terms of points 0 and NB/2 (t-grouped kernel)
    int inv_variant = 0;          // inverse kernel: 0 auto, 1 generic shared-memory kernel,
                                  // 2 the lane kernel wherever it covers the plan
    int fwd_variant = 0;          // forward kernel: 0 auto, 1 generic kernel
    int method = 0;               // 0 MFFT, 1 limb-plane schoolbook (value-mode products)
    int kara = kDefaultKara;      // Karatsuba level where the plan allows it
    int dsum = 1;                 // digit sums on the two-digit plans
    int kara_stages = 0;          // level-3 pipeline: 4 four 48 KB stages; 0 / 2 two of 96 KB
    long long out_plane_stride = 0;  // _dev integer outputs: elements between planes (0: compact)
    // transformed-B cache: valid while the workspace is not reallocated
    int reuse_b = 0;
    bool b_valid = false;
    const void* b_ptr = nullptr;
    int b_fmt = -1, b_n = 0, b_b = 0, b_Lb = 0, b_S = 0, b_NB = 0, b_dB = 0, b_lo = 0, b_sgrid = 0,
        b_trunc = 0, b_kind = 0, b_kara = 0, b_dsum = 0;
    Plan last_plan{};
    bool have_plan = false;
    int last_pw_kernel = 0;
    int last_rblock = 0;  // rows per row block of the last product
    int last_half = 0;  // the last product's plane-product kernel skipped the half-point terms
    char msg[512] = {};
};

namespace {

int set_err(mfftgpu_ctx* c, int code, const char* fmt, ...) {
    if (c) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(c->msg, sizeof c->msg, fmt, ap);
        va_end(ap);
    }
    return code;
}

#define CUDA_OK(call)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return set_err(C, MFFTB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

int ensure(mfftgpu_ctx* C, char** buf, size_t* have, size_t need) {
    if (need <= *have) return MFFTB_OK;
    if (*buf) {
        cudaStreamSynchronize(C->stream);
        cudaFree(*buf);
        *buf = nullptr;
        *have = 0;
    }
    size_t sz = (need + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
    if (cudaMalloc(buf, sz) != cudaSuccess) {
        cudaGetLastError();
        return set_err(C, MFFTB_ERR_NOMEM, "cudaMalloc(%zu bytes) failed", sz);
    }
    *have = sz;
    return MFFTB_OK;
}

struct Operand {
    int fmt;
    const void* p;
    int n, L16, W, is_signed;
    int S_grid, lo_bit, trunc_rel;
};

struct OutSpec {
    int kind;   // INV_*
    void* p;
    long long plane;
    int ld;
    int RL;
    int bit_off, S_scale;
    int esize;  // bytes per output element
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int inv_elems(const Plan& P) {
    int nk = P.NB * P.K;
    int e = 32;
    while (e > 1 && (nk * e > 16 * 256 || (size_t)nk * e * 8 > 200 * 1024)) e >>= 1;
    return e;
}

int log2i(int x) {
    int r = 0;
    while ((1 << r) < x) ++r;
    return r;
}

int run_product(mfftgpu_ctx* C, const Plan& plan, const Operand& A, const Operand& B,
                int row_begin, int row_end, const OutSpec& O) {
    Plan P = plan;
    // the Karatsuba pointwise runs on 256-row CTA-pair tiles; its job planes
    // are read by the register and lane inverse kernels
    if (P.kara && (C->inv_variant == 1 || C->pw_variant != 0 || P.n_int < 128 ||
                   row_end - row_begin < 256 || C->num_sms < 2))
        plan_set_kara(P, 0);
    const int n_int = P.n_int;
    const int dbytes = plan_digit_bytes(P);
    const long long nn_int = (long long)n_int * n_int;
    const int rows = row_end - row_begin;
    if (rows <= 0) return MFFTB_OK;
    // schoolbook plans multiply the digit planes themselves: no transform,
    // no F stack, no A-hat planes
    const bool school = P.kind == KIND_SCHOOL;
    int fpl = 0, apl = 0;
    size_t szDB = 0, szF = 0, per_row = 0;
    long long R = 0;
    const size_t limit = C->ws_limit;
    const int rows_pad = (rows + 15) / 16 * 16;
    // row block R from the workspace limit: B's digit planes and operand
    // planes whole, A's digit and operand planes and the job planes per row
    auto size_blocks = [&]() {
        const int kops = pw_kara_level_ops(P.kara);
        fpl = school ? 0 : (P.kara ? P.NB * kops : P.NB * P.dB * (2 * P.K - 1));
        apl = school ? 0 : (P.kara ? P.NB * kops : P.NB * P.dA * P.K);
        szDB = align256((size_t)P.LbB * nn_int * dbytes);
        szF = align256((size_t)fpl * nn_int);
        per_row = (size_t)n_int * ((size_t)P.LbA * dbytes + apl + 4 * (size_t)P.njobs);
        if (limit > szDB + szF + per_row * 128)
            R = (long long)((limit - szDB - szF) / per_row) / 128 * 128;
        else
            R = 128;
        if (R > rows_pad) R = rows_pad;
        if (R < 16) R = 16;
        // several blocks: equal blocks of whole 256-row CTA-pair tiles (a
        // block ending half-way through a pair tile leaves that tile's other
        // 128 rows idle in every plane product)
        if (R >= 256 && R < rows_pad) {
            const long long nblk = (rows_pad + R - 1) / R;
            const long long even = (rows_pad + nblk - 1) / nblk;
            const long long r256 = (even + 255) / 256 * 256;
            R = r256 <= R ? r256 : R / 256 * 256;
        }
    };
    size_blocks();
    if (P.kara && R < 256) {  // every row block's tiles read 256 rows of each plane
        plan_set_kara(P, 0);
        size_blocks();
    }
    const size_t szDA = align256((size_t)P.LbA * R * n_int * dbytes);
    const size_t szAh = align256((size_t)apl * R * n_int);
    const size_t szAcc = align256((size_t)P.njobs * R * n_int * 4);
    const size_t had = C->ws_bytes;
    int rc = ensure(C, &C->ws, &C->ws_bytes, szDB + szF + szDA + szAh + szAcc);
    if (rc) return rc;
    if (C->ws_bytes != had) C->b_valid = false;  // reallocated: the cached F is gone
    const bool b_cached = C->reuse_b && C->b_valid && C->b_kind == P.kind && C->b_ptr == B.p &&
                          C->b_fmt == B.fmt &&
                          C->b_n == P.n && C->b_b == P.b && C->b_Lb == P.LbB && C->b_S == P.S &&
                          C->b_NB == P.NB && C->b_dB == P.dB && C->b_lo == B.lo_bit &&
                          C->b_sgrid == B.S_grid && C->b_trunc == B.trunc_rel &&
                          C->b_kara == P.kara && C->b_dsum == P.dsum;
    char* DB = C->ws;
    int8_t* F = reinterpret_cast<int8_t*>(DB + szDB);
    char* DA = DB + szDB + szF;
    int8_t* Ah = reinterpret_cast<int8_t*>(DA + szDA);
    int32_t* acc = reinterpret_cast<int32_t*>(DA + szDA + szAh);
    cudaStream_t st = C->stream;
    C->launches = 0;
    C->last_plan = P;
    C->last_rblock = (int)R;
    C->have_plan = true;
    CUDA_OK(cudaMemsetAsync(C->d_err, 0, sizeof(int), st));
    if (C->profile != 2) {
        C->ev_used = 0;
        C->ev_dropped = 0;
    }
    C->phase_valid = false;
    // phase ids: 0 pack, 1 forward, 2 pointwise, 3 inverse
    int cur_phase = 0;
    auto tick = [&](int phase) {
        cur_phase = phase;
        if (C->profile && C->ev_used + 2 <= mfftgpu_ctx::kMaxEv)
            cudaEventRecord(C->ev[C->ev_used], st);
    };
    auto tock = [&]() {
        if (C->profile && C->ev_used + 2 <= mfftgpu_ctx::kMaxEv) {
            cudaEventRecord(C->ev[C->ev_used + 1], st);
            C->ev_phase[C->ev_used / 2] = cur_phase;
            C->ev_used += 2;
        } else if (C->profile) {
            ++C->ev_dropped;
        }
    };

    // ---- B: digits (transposed) and the F stack, once per product
    PackArgs pb{};
    pb.fmt = B.fmt;
    pb.src = B.p;
    pb.n = B.n;
    pb.row0 = 0;
    pb.L16 = B.L16;
    pb.W = B.W;
    pb.is_signed = B.is_signed;
    pb.S_grid = B.S_grid;
    pb.lo_bit = B.lo_bit;
    pb.trunc_rel = B.trunc_rel;
    pb.b = P.b;
    pb.Lb = P.LbB;
    pb.dst = DB;
    pb.rows = n_int;
    pb.ld = n_int;
    pb.plane = nn_int;
    pb.transpose = 1;
    pb.err = C->d_err;
    pb.balanced = P.balanced;
    FwdArgs fb{};
    fb.D = DB;
    fb.dbytes = dbytes;
    fb.dplane = nn_int;
    fb.Lb = P.LbB;
    fb.nelem = nn_int;
    fb.S = P.S;
    fb.NB = P.NB;
    fb.K = P.K;
    fb.g = P.g;
    fb.nc = P.ncB;
    fb.d = P.dB;
    fb.lgS = log2i(P.S);
    fb.lgK = log2i(P.K);
    fb.f_stack = P.kara ? 1 + P.kara : 1;
    fb.out = F;
    fb.oplane = nn_int;
    fb.err = C->d_err;
    fb.b = P.b;
    fb.variant = C->fwd_variant;
    fb.dsum = P.dsum;
    if (!b_cached) {
        C->b_valid = false;
        tick(0);
        if ((rc = pack_launch(pb, st))) return set_err(C, rc, "pack(B) launch failed");
        ++C->launches;
        tock();
        if (!school) {
            tick(1);
            if ((rc = forward_launch(fb, st))) return set_err(C, rc, "forward(B) launch failed");
            ++C->launches;
            tock();
        }
        C->b_valid = true;
        C->b_kind = P.kind;
        C->b_ptr = B.p;
        C->b_fmt = B.fmt;
        C->b_n = P.n;
        C->b_b = P.b;
        C->b_Lb = P.LbB;
        C->b_S = P.S;
        C->b_NB = P.NB;
        C->b_dB = P.dB;
        C->b_lo = B.lo_bit;
        C->b_sgrid = B.S_grid;
        C->b_trunc = B.trunc_rel;
        C->b_kara = P.kara;
        C->b_dsum = P.dsum;
    }

    // ---- A row blocks
    for (int r = 0; r < rows; r += (int)R) {
        const int rb = (int)std::min<long long>(R, rows - r);
        PackArgs pa = pb;
        pa.fmt = A.fmt;
        pa.src = A.p;
        pa.n = A.n;
        pa.row0 = row_begin + r;
        pa.L16 = A.L16;
        pa.W = A.W;
        pa.is_signed = A.is_signed;
        pa.S_grid = A.S_grid;
        pa.lo_bit = A.lo_bit;
        pa.trunc_rel = A.trunc_rel;
        pa.Lb = P.LbA;
        pa.dst = DA;
        pa.rows = rb;
        pa.plane = R * n_int;
        pa.transpose = 0;
        tick(0);
        if ((rc = pack_launch(pa, st))) return set_err(C, rc, "pack(A) launch failed");
        ++C->launches;
        tock();
        FwdArgs fa = fb;
        fa.D = DA;
        fa.dplane = R * n_int;
        fa.Lb = P.LbA;
        fa.nelem = (long long)rb * n_int;
        fa.nc = P.ncA;
        fa.d = P.dA;
        fa.f_stack = P.kara ? 1 + P.kara : 0;
        fa.out = Ah;
        fa.oplane = R * n_int;
        if (!school) {
            tick(1);
            if ((rc = forward_launch(fa, st))) return set_err(C, rc, "forward(A) launch failed");
            ++C->launches;
            tock();
        }

        PwLaunch L{};
        L.A = school ? reinterpret_cast<const int8_t*>(DA) : Ah;
        L.lda = n_int;
        L.a_plane_bytes = R * n_int;
        L.a_planes = school ? P.LbA : apl;
        L.F = school ? reinterpret_cast<const int8_t*>(DB) : F;
        L.ldf = n_int;
        L.f_plane_bytes = nn_int;
        L.f_planes = school ? P.LbB : fpl;
        L.rows = rb;
        L.cols = n_int;
        L.kdim = n_int;
        L.jobs = PwJobs{P.K, P.dA, P.dB, P.nW, P.nchunk, P.njobs, school ? 1 : 0, P.LbA, P.LbB, P.U,
                        P.NB, (!school && !P.kara && C->half_points && P.K == 2 * P.S) ? P.S : 0,
                        P.kara, P.dsum};
        L.map_rows = (int)std::max<long long>(rb, 256);
        L.kara_stages = C->kara_stages;
        L.block_n = n_int <= 64 ? 64 : (n_int <= 128 ? 128 : 256);
        L.out = acc;
        L.out_plane = R * n_int;
        L.ldo = n_int;
        L.err = C->d_err;
        L.timeout_ns = C->timeout_ns;
        L.num_sms = C->num_sms;
        L.raster = C->raster;
        L.group_m = C->group_m;
        L.variant = C->pw_variant;
        L.wave_counter = C->wave_sync ? reinterpret_cast<unsigned int*>(C->d_err + 32) : nullptr;
        L.chosen = &C->last_pw_kernel;
        tick(2);
        if ((rc = pointwise_launch(L, st))) return set_err(C, rc, "pointwise launch failed");
        C->last_half = L.jobs.zpS > 0 && C->last_pw_kernel == 3;
        ++C->launches;
        tock();

        InvArgs ia{};
        ia.acc = acc;
        ia.acc_plane = R * n_int;
        ia.lda = n_int;
        ia.rows = rb;
        ia.cols = P.n;
        ia.S = P.S;
        ia.NB = P.NB;
        ia.K = P.K;
        ia.g = P.g;
        ia.nW = P.nW;
        ia.nchunk = P.nchunk;
        ia.log2NB = log2i(P.NB);
        ia.lgS = log2i(P.S);
        ia.lgK = log2i(P.K);
        ia.b = P.b;
        ia.positions = P.positions;
        ia.out_kind = O.kind;
        ia.out = static_cast<char*>(O.p) + (size_t)r * O.ld * O.esize;
        ia.out_plane = O.plane;
        ia.ldo = O.ld;
        ia.RL = O.RL;
        ia.bit_off = O.bit_off;
        ia.S_scale = O.S_scale;
        ia.elems = inv_elems(P);
        ia.lgE = log2i(ia.elems);
        ia.err = C->d_err;
        ia.variant = C->inv_variant;
        ia.school = school ? 1 : 0;
        ia.LbA = P.LbA;
        ia.LbB = P.LbB;
        ia.U = P.U;
        ia.kara = P.kara;
        ia.dsum = P.dsum;
        tick(3);
        if ((rc = inverse_launch(ia, st))) return set_err(C, rc, "inverse launch failed (%d)", rc);
        ++C->launches;
        tock();
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_err(C, MFFTB_ERR_CUDA, "%s", cudaGetErrorString(e));
    return MFFTB_OK;
}

// plane stride of a _dev integer output: compact [RL][rows][n] unless the
// caller asked for another layout (e.g. its rows of a full [RL][n][n] array)
long long out_plane(const mfftgpu_ctx* C, int n, int row_begin, int row_end) {
    return C->out_plane_stride ? C->out_plane_stride : (long long)(row_end - row_begin) * n;
}

int check_rows(int n, int row_begin, int row_end) {
    return (row_begin < 0 || row_end > n || row_begin > row_end) ? MFFTB_ERR_ARG : MFFTB_OK;
}

int plan_or_err(mfftgpu_ctx* C, int n, int mode, int wA, int wB, Plan* P,
                int balanced_ok = 0) {
    // the schoolbook method covers value-mode products; limb mode (conv)
    // always runs the MFFT plan
    if (C->method == 1 && mode == PLAN_VALUE &&
        plan_search_school(n, wA, wB, 0, P, balanced_ok) == 0)
        return MFFTB_OK;
    int rc = plan_search(n, mode, wA, wB, 0, 0, P);
    if (rc)
        return set_err(C, MFFTB_ERR_PLAN, "no exact int8 plan for n=%d mode=%d widths %d/%d", n,
                       mode, wA, wB);
    plan_set_kara(*P, C->kara);
    if (C->dsum) plan_set_dsum(*P);
    return MFFTB_OK;
}

__global__ void gen_u16_kernel(uint16_t* m, long long count, uint64_t seed) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        uint64_t z = seed + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ULL;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        m[i] = (uint16_t)((z ^ (z >> 31)) & 0xFFFFu);
    }
}

__global__ void gen_i64_kernel(int64_t* x, long long count, uint64_t seed) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
         i += (long long)gridDim.x * blockDim.x) {
        uint64_t z = seed + (uint64_t)(i + 1) * 0x9E3779B97F4A7C15ULL;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        x[i] = (int64_t)(z ^ (z >> 31));
    }
}

int next_pow2i(int x) {
    int r = 1;
    while (r < x) r <<= 1;
    return r;
}

}  // namespace

// =====================================================================================
extern "C" {

const char* mfftgpu_status_string(int s) {
    switch (s) {
        case MFFTGPU_OK: return "ok";
        case MFFTGPU_ERR_ARG: return "invalid argument";
        case MFFTGPU_ERR_NOMEM: return "out of device memory";
        case MFFTGPU_ERR_CUDA: return "CUDA error";
        case MFFTGPU_ERR_TIMEOUT: return "device-side wait timed out";
        case MFFTGPU_ERR_RANGE: return "input limb out of range";
        case MFFTGPU_ERR_NODEVICE: return "no usable sm_100 device";
        case MFFTGPU_ERR_PLAN: return "no exact plan";
        case MFFTGPU_ERR_UNSUPPORTED: return "unsupported";
        default: return "unknown status";
    }
}

int mfftgpu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int mfftgpu_create(mfftgpu_ctx** out, int device) {
    if (!out) return MFFTB_ERR_ARG;
    *out = nullptr;
    int ndev = mfftgpu_device_count();
    if (device < 0 || device >= ndev) return MFFTB_ERR_NODEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return MFFTB_ERR_CUDA;
    if (prop.major != 10 || prop.minor != 0) return MFFTB_ERR_NODEVICE;
    mfftgpu_ctx* C = new (std::nothrow) mfftgpu_ctx();
    if (!C) return MFFTB_ERR_NOMEM;
    C->device = device;
    C->num_sms = prop.multiProcessorCount;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete C;
        return MFFTB_ERR_CUDA;
    }
    if (cudaStreamCreateWithFlags(&C->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&C->d_err, 256) != cudaSuccess) {
        delete C;
        return MFFTB_ERR_CUDA;
    }
    C->own_stream = true;
    C->d_scan = C->d_err + 4;
    for (auto& e : C->ev) {
        if (cudaEventCreate(&e) != cudaSuccess) {
            e = nullptr;
            C->profile = 0;
        }
    }
    size_t fr = 0, tot = 0;
    cudaMemGetInfo(&fr, &tot);
    C->ws_limit = (size_t)(0.55 * (double)fr);
    if (const char* s = getenv("MFFTGPU_WS_GB")) C->ws_limit = (size_t)(atof(s) * 1073741824.0);
    if (const char* s = getenv("MFFTGPU_RASTER")) C->raster = atoi(s);
    if (const char* s = getenv("MFFTGPU_GROUP_M")) C->group_m = atoi(s);
    if (const char* s = getenv("MFFTGPU_PW_VARIANT")) C->pw_variant = atoi(s);
    if (const char* s = getenv("MFFTGPU_WAVE_SYNC")) C->wave_sync = atoi(s);
    if (const char* s = getenv("MFFTGPU_KARA_STAGES")) C->kara_stages = atoi(s);
    if (const char* s = getenv("MFFTGPU_DSUM")) C->dsum = atoi(s) != 0;
    if (const char* s = getenv("MFFTGPU_HALF_POINTS")) C->half_points = atoi(s) != 0;
    if (const char* s = getenv("MFFTGPU_INV_VARIANT")) C->inv_variant = atoi(s);
    if (const char* s = getenv("MFFTGPU_FWD_VARIANT")) C->fwd_variant = atoi(s) == 1 ? 1 : 0;
    if (const char* s = getenv("MFFTGPU_METHOD")) C->method = atoi(s);
    if (const char* s = getenv("MFFTGPU_KARA")) {
        const int v = atoi(s);
        C->kara = v < 0 ? 0 : (v > 3 ? 3 : v);
    }
    cudaMemset(C->d_err, 0, 256);
    *out = C;
    return MFFTB_OK;
}

int mfftgpu_destroy(mfftgpu_ctx* C) {
    if (!C) return MFFTB_OK;
    cudaSetDevice(C->device);
    if (C->stream) cudaStreamSynchronize(C->stream);
    cudaFree(C->ws);
    cudaFree(C->io);
    cudaFree(C->d_err);
    for (auto& e : C->ev)
        if (e) cudaEventDestroy(e);
    for (cudaStream_t s : {C->copy_stream, C->up_stream})
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    for (auto& e : C->chunk_ev)
        if (e) cudaEventDestroy(e);
    for (auto& e : C->up_ev)
        if (e) cudaEventDestroy(e);
    if (C->own_stream && C->stream) cudaStreamDestroy(C->stream);
    delete C;
    return MFFTB_OK;
}

int mfftgpu_set_stream(mfftgpu_ctx* C, void* s) {
    if (!C) return MFFTB_ERR_ARG;
    if (C->own_stream && C->stream) cudaStreamDestroy(C->stream);
    C->stream = static_cast<cudaStream_t>(s);
    C->own_stream = false;
    return MFFTB_OK;
}

int mfftgpu_set_workspace_limit(mfftgpu_ctx* C, size_t bytes) {
    if (!C) return MFFTB_ERR_ARG;
    C->ws_limit = bytes;
    return MFFTB_OK;
}

int mfftgpu_set_timeout_ns(mfftgpu_ctx* C, unsigned long long ns) {
    if (!C || ns == 0) return MFFTB_ERR_ARG;
    C->timeout_ns = ns;
    return MFFTB_OK;
}

int mfftgpu_set_reuse_b(mfftgpu_ctx* C, int on) {
    if (!C) return MFFTB_ERR_ARG;
    C->reuse_b = on != 0;
    if (!on) C->b_valid = false;
    return MFFTB_OK;
}

int mfftgpu_set_method(mfftgpu_ctx* C, int method) {
    if (!C || method < 0 || method > 1) return MFFTB_ERR_ARG;
    C->method = method;
    return MFFTB_OK;
}

int mfftgpu_get_method(mfftgpu_ctx* C) { return C ? C->method : -1; }

int mfftgpu_set_output_plane_stride(mfftgpu_ctx* C, long long elems) {
    if (!C || elems < 0) return MFFTB_ERR_ARG;
    C->out_plane_stride = elems;
    return MFFTB_OK;
}

// --------------------------------------------------------------------- peer buffers (CUDA IPC)
int mfftgpu_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return MFFTB_ERR_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return MFFTB_ERR_NOMEM;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return MFFTB_ERR_CUDA;
    }
    std::memcpy(handle, &h, sizeof h);
    *ptr = p;
    return MFFTB_OK;
}

int mfftgpu_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return MFFTB_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
               ? MFFTB_OK
               : MFFTB_ERR_CUDA;
}

int mfftgpu_ipc_close(void* ptr) {
    return ptr && cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int mfftgpu_ipc_free(void* ptr) {
    return ptr && cudaFree(ptr) == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int mfftgpu_set_half_points(mfftgpu_ctx* C, int on) {
    if (!C || on < 0 || on > 1) return MFFTB_ERR_ARG;
    C->half_points = on;
    return MFFTB_OK;
}

int mfftgpu_set_digit_sums(mfftgpu_ctx* C, int on) {
    if (!C || on < 0 || on > 1) return MFFTB_ERR_ARG;
    C->dsum = on;
    return MFFTB_OK;
}

int mfftgpu_set_karatsuba(mfftgpu_ctx* C, int level) {
    if (!C || level < 0 || level > 3) return MFFTB_ERR_ARG;
    C->kara = level;
    return MFFTB_OK;
}

int mfftgpu_set_kernel_variant(mfftgpu_ctx* C, int stage, int variant) {
    if (!C) return MFFTB_ERR_ARG;
    if (stage == 2 && variant >= 0 && variant <= 3) {
        C->pw_variant = variant;
        return MFFTB_OK;
    }
    if (stage == 3 && variant >= 0 && variant <= 2) {
        C->inv_variant = variant;
        return MFFTB_OK;
    }
    if (stage == 1 && variant >= 0 && variant <= 1) {
        C->fwd_variant = variant;
        return MFFTB_OK;
    }
    return MFFTB_ERR_ARG;
}

int mfftgpu_set_profile(mfftgpu_ctx* C, int mode) {
    if (!C || mode < 0 || mode > 2) return MFFTB_ERR_ARG;
    C->profile = mode;
    C->ev_used = 0;
    C->ev_dropped = 0;
    C->phase_valid = false;
    return MFFTB_OK;
}

int mfftgpu_last_phase_dropped(mfftgpu_ctx* C) { return C ? C->ev_dropped : 0; }

int mfftgpu_last_phase_ms(mfftgpu_ctx* C, float out[5]) {
    if (!C || !out) return MFFTB_ERR_ARG;
    if (!C->phase_valid) {
        for (float& v : C->phase_ms) v = 0.0f;
        if (C->ev_used >= 2) {
            cudaSetDevice(C->device);
            CUDA_OK(cudaEventSynchronize(C->ev[C->ev_used - 1]));
            for (int k = 0; k < C->ev_used; k += 2) {
                float ms = 0;
                CUDA_OK(cudaEventElapsedTime(&ms, C->ev[k], C->ev[k + 1]));
                C->phase_ms[C->ev_phase[k / 2]] += ms;
            }
            float tot = 0;
            CUDA_OK(cudaEventElapsedTime(&tot, C->ev[0], C->ev[C->ev_used - 1]));
            C->phase_ms[4] = tot;
        }
        C->phase_valid = true;
    }
    memcpy(out, C->phase_ms, sizeof C->phase_ms);
    return MFFTB_OK;
}

int mfftgpu_last_launches(mfftgpu_ctx* C) { return C ? C->launches : 0; }

const char* mfftgpu_last_error(mfftgpu_ctx* C) { return C ? C->msg : "no context"; }

int mfftgpu_sync(mfftgpu_ctx* C) {
    if (!C) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    CUDA_OK(cudaStreamSynchronize(C->stream));
    int h = 0;
    CUDA_OK(cudaMemcpy(&h, C->d_err, sizeof h, cudaMemcpyDeviceToHost));
    if (h) return set_err(C, h, "device reported: %s", mfftgpu_status_string(h));
    return MFFTB_OK;
}

static void fill_info(const Plan& P, mfftgpu_plan_info* o);

int mfftgpu_plan_info_get(int n, int mode, int wA, int wB, mfftgpu_plan_info* o) {
    if (!o) return MFFTB_ERR_ARG;
    Plan P;
    if (mode == 2 || mode == 3) {  // 3: int64 operands, balanced digits allowed
        if (plan_search_school(n, wA, wB, 0, &P, mode == 3)) return MFFTB_ERR_PLAN;
    } else if (plan_search(n, mode, wA, wB, 0, 0, &P)) {
        return MFFTB_ERR_PLAN;
    } else {
        plan_set_kara(P, kDefaultKara);  // the default context settings
        plan_set_dsum(P);
    }
    fill_info(P, o);
    return MFFTB_OK;
}

int mfftgpu_last_plan(mfftgpu_ctx* C, mfftgpu_plan_info* o) {
    if (!C || !o || !C->have_plan) return MFFTB_ERR_ARG;
    fill_info(C->last_plan, o);
    o->pw_kernel = C->last_pw_kernel;
    o->rblock = C->last_rblock;
    const Plan& P = C->last_plan;
    if (C->last_half && P.kind == KIND_MFFT && P.NB >= 2) {
        // points 0 and NB/2 issue S^2 of their K^2 plane products
        o->half_points = 1;
        o->int8_macs *= ((double)(P.NB - 2) * P.K * P.K + 2.0 * P.S * P.S) / ((double)P.NB * P.K * P.K);
    }
    return MFFTB_OK;
}

static void fill_info(const Plan& P, mfftgpu_plan_info* o) {
    const int n = P.n;
    o->n = P.n;
    o->n_int = P.n_int;
    o->mode = P.mode;
    o->b = P.b;
    o->LbA = P.LbA;
    o->LbB = P.LbB;
    o->S = P.S;
    o->NB = P.NB;
    o->K = P.K;
    o->g = P.g;
    o->ncA = P.ncA;
    o->ncB = P.ncB;
    o->dA = P.dA;
    o->dB = P.dB;
    o->nW = P.nW;
    o->nchunk = P.nchunk;
    o->njobs = P.njobs;
    o->positions = P.positions;
    o->acc_bound = P.acc_bound;
    o->inv_bound_log2 = P.inv_bound_log2;
    o->int8_macs = P.macs_per_elem * (double)P.n_int * P.n_int;
    o->schoolbook_macs = (double)n * n * (double)n * P.LbA * P.LbB;
    o->wA = P.wA;
    o->wB = P.wB;
    o->schoolbook7_macs = (double)n * n * (double)n * ((P.wA + 6) / 7) * ((P.wB + 6) / 7);
    o->kara = P.kara;
    o->dsum = P.dsum;
    o->rblock = 0;
    o->pw_kernel = 0;
    o->kind = P.kind;
    o->U = P.U;
    o->balanced = P.balanced;
    o->half_points = 0;
}

// --------------------------------------------------------------------- integers
int mfftgpu_mm_u16_dev(mfftgpu_ctx* C, const uint16_t* A, const uint16_t* B, int n, int L,
                       int is_signed, uint16_t* out, int RL, int row_begin, int row_end) {
    if (!C || !A || !B || !out || n <= 0 || L <= 0 || RL <= 0) return MFFTB_ERR_ARG;
    if (check_rows(n, row_begin, row_end)) return set_err(C, MFFTB_ERR_ARG, "bad row range");
    cudaSetDevice(C->device);
    Plan P;
    int rc = plan_or_err(C, n, PLAN_VALUE, 16 * L, 16 * L, &P);
    if (rc) return rc;
    Operand a{PACK_U16PL, A, n, L, 16 * L, is_signed ? 1 : 0, 0, 0, 0};
    Operand b = a;
    b.p = B;
    OutSpec o{INV_U16, out, out_plane(C, n, row_begin, row_end), n, RL, 0, 0, 2};
    return run_product(C, P, a, b, row_begin, row_end, o);
}

int mfftgpu_mm_i64_dev(mfftgpu_ctx* C, const int64_t* A, const int64_t* B, int n, uint16_t* out,
                       int RL, int row_begin, int row_end) {
    if (!C || !A || !B || !out || n <= 0 || RL <= 0) return MFFTB_ERR_ARG;
    if (check_rows(n, row_begin, row_end)) return set_err(C, MFFTB_ERR_ARG, "bad row range");
    cudaSetDevice(C->device);
    Plan P;
    int rc = plan_or_err(C, n, PLAN_VALUE, 64, 64, &P, 1);
    if (rc) return rc;
    Operand a{PACK_I64, A, n, 4, 64, 1, 0, 0, 0};
    Operand b = a;
    b.p = B;
    OutSpec o{INV_U16, out, out_plane(C, n, row_begin, row_end), n, RL, 0, 0, 2};
    return run_product(C, P, a, b, row_begin, row_end, o);
}

int mfftgpu_conv_i32_dev(mfftgpu_ctx* C, const int32_t* A32, const int32_t* B32, int n, int L,
                         int64_t* Cw) {
    if (!C || !A32 || !B32 || !Cw || n <= 0 || L <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    Plan P;
    int rc = plan_or_err(C, n, PLAN_LIMB, L, L, &P);
    if (rc) return rc;
    Operand a{PACK_I32LIMB, A32, n, L, 0, 1, 0, 0, 0};
    Operand b = a;
    b.p = B32;
    OutSpec o{INV_I64, Cw, (long long)n * n, n, 2 * L - 1, 0, 0, 8};
    return run_product(C, P, a, b, 0, n, o);
}

// --------------------------------------------------------------------- fp32 / fp64
// The fixed-point embeddings of src/fpfixed.c: fp32 (sig 24, an entry touches
// wr = 3 limbs) and fp64 (sig 53, wr = 5), same grid rules, same product,
// decode rounded once to the output precision.
static int fp_dev(mfftgpu_ctx* C, const void* A, const void* B, int n, int force_bits, void* Cout,
                  int row_begin, int row_end, bool is64) {
    if (!C || !A || !B || !Cout || n <= 0 || force_bits < 0) return MFFTB_ERR_ARG;
    if (check_rows(n, row_begin, row_end)) return set_err(C, MFFTB_ERR_ARG, "bad row range");
    cudaSetDevice(C->device);
    cudaStream_t st = C->stream;
    const long long nn = (long long)n * n;
    const int sig = is64 ? 53 : 24, wr = is64 ? 5 : 3;
    int rc;
    if (is64) {
        if ((rc = scan_f64_launch(static_cast<const double*>(A), nn, C->d_scan, st)))
            return set_err(C, rc, "scan(A) failed");
        if ((rc = scan_f64_launch(static_cast<const double*>(B), nn, C->d_scan + 3, st)))
            return set_err(C, rc, "scan(B) failed");
    } else {
        if ((rc = scan_f32_launch(static_cast<const float*>(A), nn, C->d_scan, st)))
            return set_err(C, rc, "scan(A) failed");
        if ((rc = scan_f32_launch(static_cast<const float*>(B), nn, C->d_scan + 3, st)))
            return set_err(C, rc, "scan(B) failed");
    }
    int h[6];
    CUDA_OK(cudaMemcpyAsync(h, C->d_scan, sizeof h, cudaMemcpyDeviceToHost, st));
    CUDA_OK(cudaStreamSynchronize(st));
    const int loA = h[2] ? h[0] : 0, hiA = h[2] ? h[1] : 0, anyA = h[2];
    const int loB = h[5] ? h[3] : 0, hiB = h[5] ? h[4] : 0, anyB = h[5];
    // grid sizing of fpx_size (src/fpfixed.c:59-78)
    int SA, SB, L;
    const int spreadA = anyA ? hiA - loA : 0, spreadB = anyB ? hiB - loB : 0;
    if (force_bits > 0) {
        SA = SB = force_bits / 2;
        L = next_pow2i(force_bits / 16);
    } else {
        SA = -loA;
        SB = -loB;
        int bits = std::max(sig + spreadA + 1, sig + spreadB + 1);
        int spread = std::max(spreadA, spreadB);
        int need = (bits + 15) / 16, need2 = spread / 16 + wr;
        L = next_pow2i(std::max(need, need2));
        if (L < 2) L = 2;
    }
    // fpx_alloc's int64 headroom guard (src/fpfixed.c:84-88)
    if ((double)n * L * 65535.0 * 65535.0 > 4.0e18)
        return set_err(C, MFFTB_ERR_RANGE, "fpx: n=%d L=%d would overflow int64 accumulators", n, L);
    // live bit windows on the grid
    auto window = [&](int any, int lo, int hi, int S, int& lo_bit, int& width) {
        lo_bit = 0;
        width = 1;
        if (!any) return;
        int l = std::max(0, lo + S), t = std::min(16 * L, hi + S + sig);
        if (t <= l) return;
        lo_bit = l;
        width = t - l;
    };
    int loBitA, wA, loBitB, wB;
    window(anyA, loA, hiA, SA, loBitA, wA);
    window(anyB, loB, hiB, SB, loBitB, wB);
    Plan P;
    if ((rc = plan_or_err(C, n, PLAN_VALUE, wA, wB, &P))) return rc;
    const int fmt = is64 ? PACK_F64 : PACK_F32;
    Operand a{fmt, A, n, 0, wA, 1, SA, loBitA, 16 * L - loBitA};
    Operand b{fmt, B, n, 0, wB, 1, SB, loBitB, 16 * L - loBitB};
    OutSpec o{is64 ? INV_F64 : INV_F32, Cout, 0, n, 0, loBitA + loBitB, SA + SB, is64 ? 8 : 4};
    return run_product(C, P, a, b, row_begin, row_end, o);
}

int mfftgpu_fp32_dev(mfftgpu_ctx* C, const float* A, const float* B, int n, int force_bits,
                     float* Cout, int row_begin, int row_end) {
    return fp_dev(C, A, B, n, force_bits, Cout, row_begin, row_end, false);
}

int mfftgpu_fp64_dev(mfftgpu_ctx* C, const double* A, const double* B, int n, int force_bits,
                     double* Cout, int row_begin, int row_end) {
    return fp_dev(C, A, B, n, force_bits, Cout, row_begin, row_end, true);
}

// --------------------------------------------------------------------- host-pointer variants
static int stage(mfftgpu_ctx* C, size_t inA, size_t inB, size_t outb, char** dA, char** dB,
                 char** dO) {
    size_t a = align256(inA), b = align256(inB), o = align256(outb);
    int rc = ensure(C, &C->io, &C->io_bytes, a + b + o);
    if (rc) return rc;
    *dA = C->io;
    *dB = C->io + a;
    *dO = C->io + a + b;
    return MFFTB_OK;
}

}  // extern "C"

// Host-pointer products: B is uploaded first and A in row chunks on an
// upload stream; the rows of C are computed chunk by chunk as their rows of
// A arrive (B packed and transformed once, kept across chunks), and each
// chunk's rows of every output plane are read back on a third stream while
// the next chunk computes, so both copies hide behind the tensor-core work.
// The operands are row-major planes: A and B have a_planes planes of
// a_esize-byte elements ([planes][n][n]); compute(r0, r1, dst) writes rows
// [r0, r1) of C as [planes][r1-r0][n] at dst; host out is [planes][n][n]
// with elements of esize bytes.  whole_a: every chunk reads all of A (the
// fp embeddings scan A's exponent range first), so chunk 0 waits for the
// last upload.
template <typename F>
static int rows_pipelined(mfftgpu_ctx* C, int n, const void* hA, const void* hB, char* dA,
                          char* dB, int a_planes, size_t a_esize, int planes, size_t esize,
                          char* dO, void* out, bool whole_a, F compute) {
    // more chunks for the largest products: the first chunk's upload and the
    // last chunk's read-back are the copies no compute hides
    const int nchunks = n >= 16384 ? 8 : (n >= 4096 ? 4 : 1);
    // chunk c covers rows [bound(c), bound(c + 1)), boundaries on whole
    // 256-row CTA-pair tiles
    auto bound = [&](int c) {
        if (c >= nchunks) return n;
        return (int)(((long long)n * c / nchunks) / 256 * 256);
    };
    const size_t in = (size_t)a_planes * n * n * a_esize;
    if (nchunks == 1) {
        CUDA_OK(cudaMemcpyAsync(dA, hA, in, cudaMemcpyHostToDevice, C->stream));
        CUDA_OK(cudaMemcpyAsync(dB, hB, in, cudaMemcpyHostToDevice, C->stream));
    } else {
        if (!C->copy_stream) {
            CUDA_OK(cudaStreamCreateWithFlags(&C->copy_stream, cudaStreamNonBlocking));
            CUDA_OK(cudaStreamCreateWithFlags(&C->up_stream, cudaStreamNonBlocking));
            for (auto& e : C->chunk_ev) CUDA_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            for (auto& e : C->up_ev) CUDA_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        }
        // earlier work on the context stream may still read the staging buffers
        CUDA_OK(cudaEventRecord(C->up_ev[8], C->stream));
        CUDA_OK(cudaStreamWaitEvent(C->up_stream, C->up_ev[8], 0));
        CUDA_OK(cudaMemcpyAsync(dB, hB, in, cudaMemcpyHostToDevice, C->up_stream));
        for (int c = 0; c < nchunks; ++c) {
            const int r0 = bound(c), r1 = bound(c + 1);
            const size_t w = (size_t)(r1 - r0) * n * a_esize, off = (size_t)r0 * n * a_esize;
            CUDA_OK(cudaMemcpy2DAsync(dA + off, (size_t)n * n * a_esize,
                                      static_cast<const char*>(hA) + off, (size_t)n * n * a_esize,
                                      w, a_planes, cudaMemcpyHostToDevice, C->up_stream));
            CUDA_OK(cudaEventRecord(C->up_ev[c], C->up_stream));
        }
    }
    const bool keep = C->reuse_b;
    const long long keep_stride = C->out_plane_stride;
    C->out_plane_stride = 0;  // the chunks below are compact
    int rc = MFFTB_OK;
    C->b_valid = false;
    for (int c = 0; c < nchunks && !rc; ++c) {
        const int r0 = bound(c), r1 = bound(c + 1);
        if (r1 <= r0) continue;
        if (nchunks > 1)
            CUDA_OK(cudaStreamWaitEvent(C->stream, C->up_ev[whole_a ? nchunks - 1 : c], 0));
        char* dst = dO + (size_t)planes * r0 * n * esize;
        C->reuse_b = c > 0;  // same B buffer for every chunk
        rc = compute(r0, r1, dst);
        if (rc) break;
        const size_t w = (size_t)(r1 - r0) * n * esize;
        if (nchunks == 1) {
            CUDA_OK(cudaMemcpyAsync(out, dst, (size_t)planes * w, cudaMemcpyDeviceToHost, C->stream));
            continue;
        }
        CUDA_OK(cudaEventRecord(C->chunk_ev[c], C->stream));
        CUDA_OK(cudaStreamWaitEvent(C->copy_stream, C->chunk_ev[c], 0));
        CUDA_OK(cudaMemcpy2DAsync(static_cast<char*>(out) + (size_t)r0 * n * esize,
                                  (size_t)n * n * esize, dst, w, w, planes, cudaMemcpyDeviceToHost,
                                  C->copy_stream));
    }
    C->reuse_b = keep;
    C->out_plane_stride = keep_stride;
    C->b_valid = false;
    if (nchunks > 1) {
        cudaError_t e = cudaStreamSynchronize(C->copy_stream);
        if (!rc && e != cudaSuccess) rc = set_err(C, MFFTB_ERR_CUDA, "%s", cudaGetErrorString(e));
    }
    int rs = mfftgpu_sync(C);
    return rc ? rc : rs;
}

extern "C" {

int mfftgpu_mm_u16(mfftgpu_ctx* C, const uint16_t* A, const uint16_t* B, int n, int L,
                   int is_signed, uint16_t* out, int RL) {
    if (!C || !A || !B || !out || n <= 0 || L <= 0 || RL <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const size_t in = (size_t)L * n * n * 2, ob = (size_t)RL * n * n * 2;
    char *dA, *dB, *dO;
    int rc = stage(C, in, in, ob, &dA, &dB, &dO);
    if (rc) return rc;
    return rows_pipelined(C, n, A, B, dA, dB, L, 2, RL, 2, dO, out, false, [&](int r0, int r1, char* dst) {
        return mfftgpu_mm_u16_dev(C, (uint16_t*)dA, (uint16_t*)dB, n, L, is_signed,
                                  (uint16_t*)dst, RL, r0, r1);
    });
}

int mfftgpu_mm_i64(mfftgpu_ctx* C, const int64_t* A, const int64_t* B, int n, uint16_t* out,
                   int RL) {
    if (!C || !A || !B || !out || n <= 0 || RL <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const size_t in = (size_t)n * n * 8, ob = (size_t)RL * n * n * 2;
    char *dA, *dB, *dO;
    int rc = stage(C, in, in, ob, &dA, &dB, &dO);
    if (rc) return rc;
    return rows_pipelined(C, n, A, B, dA, dB, 1, 8, RL, 2, dO, out, false, [&](int r0, int r1, char* dst) {
        return mfftgpu_mm_i64_dev(C, (int64_t*)dA, (int64_t*)dB, n, (uint16_t*)dst, RL, r0, r1);
    });
}

int mfftgpu_conv_i32(mfftgpu_ctx* C, const int32_t* A32, const int32_t* B32, int n, int L,
                     int64_t* Cw) {
    if (!C || !A32 || !B32 || !Cw || n <= 0 || L <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const size_t in = (size_t)L * n * n * 4, ob = (size_t)(2 * L - 1) * n * n * 8;
    char *dA, *dB, *dO;
    int rc = stage(C, in, in, ob, &dA, &dB, &dO);
    if (rc) return rc;
    CUDA_OK(cudaMemcpyAsync(dA, A32, in, cudaMemcpyHostToDevice, C->stream));
    CUDA_OK(cudaMemcpyAsync(dB, B32, in, cudaMemcpyHostToDevice, C->stream));
    rc = mfftgpu_conv_i32_dev(C, (int32_t*)dA, (int32_t*)dB, n, L, (int64_t*)dO);
    if (rc) return rc;
    CUDA_OK(cudaMemcpyAsync(Cw, dO, ob, cudaMemcpyDeviceToHost, C->stream));
    return mfftgpu_sync(C);
}

int mfftgpu_fp64(mfftgpu_ctx* C, const double* A, const double* B, int n, int force_bits,
                 double* Cout) {
    if (!C || !A || !B || !Cout || n <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const size_t in = (size_t)n * n * 8;
    char *dA, *dB, *dO;
    int rc = stage(C, in, in, in, &dA, &dB, &dO);
    if (rc) return rc;
    return rows_pipelined(C, n, A, B, dA, dB, 1, 8, 1, 8, dO, Cout, true, [&](int r0, int r1, char* dst) {
        return mfftgpu_fp64_dev(C, (double*)dA, (double*)dB, n, force_bits, (double*)dst, r0, r1);
    });
}

int mfftgpu_fp32(mfftgpu_ctx* C, const float* A, const float* B, int n, int force_bits,
                 float* Cout) {
    if (!C || !A || !B || !Cout || n <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const size_t in = (size_t)n * n * 4;
    char *dA, *dB, *dO;
    int rc = stage(C, in, in, in, &dA, &dB, &dO);
    if (rc) return rc;
    return rows_pipelined(C, n, A, B, dA, dB, 1, 4, 1, 4, dO, Cout, true, [&](int r0, int r1, char* dst) {
        return mfftgpu_fp32_dev(C, (float*)dA, (float*)dB, n, force_bits, (float*)dst, r0, r1);
    });
}

// --------------------------------------------------------------------- generators
int mfftgpu_gen_bigmat_dev(mfftgpu_ctx* C, uint16_t* m, int n, int L, uint64_t seed) {
    if (!C || !m || n <= 0 || L <= 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    gen_u16_kernel<<<C->num_sms * 8, 256, 0, C->stream>>>(m, (long long)n * n * L, seed);
    CUDA_OK(cudaGetLastError());
    return MFFTB_OK;
}

int mfftgpu_gen_int64_dev(mfftgpu_ctx* C, int64_t* x, size_t count, uint64_t seed) {
    if (!C || !x) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    gen_i64_kernel<<<C->num_sms * 8, 256, 0, C->stream>>>(x, (long long)count, seed);
    CUDA_OK(cudaGetLastError());
    return MFFTB_OK;
}

int mfftgpu_selftest_pointwise(mfftgpu_ctx* C, int rows, int cols, int kdim, int NB, int K,
                               int dA, int dB, int nchunk, int block_n, int variant,
                               long long* mismatches) {
    if (!C || !mismatches || rows <= 0 || cols <= 0 || kdim <= 0 || cols % 16 || NB < 1 ||
        K < 1 || dA < 1 || dB < 1 || nchunk < 1 || nchunk > K)
        return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const int ld = (kdim + 15) / 16 * 16;
    PwJobs J{K, dA, dB, dA + dB - 1, nchunk, NB * K * (dA + dB - 1) * nchunk};
    // variants 4, 5, 6: the Karatsuba kernel (K = 8, one digit, one chunk)
    // at level 1 / 2 / 3 on random operand planes, NB * 12 / 16 / 18 per
    // side; A planes span at least 256 rows
    const bool kara = variant >= 4 && variant <= 6;
    if (kara && (K != 8 || dA != 1 || dB != 1 || nchunk != 1 || NB < 2 || NB > 8 || cols < 128))
        return MFFTB_ERR_ARG;
    const int arows = kara ? std::max(rows, 256) : rows;
    // variant 7: a digit-sum job table (dA = dB = 3, class w pairs digit w
    // with digit w) on the kernel the product path picks for the shape
    if (variant == 7) {
        if (dA != 3 || dB != 3) return MFFTB_ERR_ARG;
        J.nW = 3;
        J.njobs = NB * K * 3 * nchunk;
        J.dsum = 1;
        variant = 0;
    }
    if (kara) {
        J.NB = NB;
        J.kara = variant - 3;
        J.njobs = NB * pw_kara_jobs(J);
    } else if (C->half_points && K % 2 == 0) {
        J.NB = NB;
        J.zpS = K / 2;
    }
    const int apl = kara ? NB * pw_kara_ops(J) : NB * dA * K;
    const int fpl = kara ? NB * pw_kara_ops(J) : NB * dB * (2 * K - 1);
    const size_t szA = align256((size_t)apl * arows * ld), szF = align256((size_t)fpl * cols * ld);
    const size_t szO = align256((size_t)J.njobs * rows * cols * 4);
    int rc = ensure(C, &C->ws, &C->ws_bytes, szA + szF + szO + 256);
    if (rc) return rc;
    int8_t* A = reinterpret_cast<int8_t*>(C->ws);
    int8_t* F = A + szA;
    int32_t* out = reinterpret_cast<int32_t*>(F + szF);
    long long* dcnt = reinterpret_cast<long long*>(reinterpret_cast<char*>(out) + szO);
    int* mism = C->d_err + 8;
    // random digits in [-128, 127]: keep every class contraction inside int32
    if ((long long)kdim * K * std::min(dA, dB) * 16384LL > 2147483647LL) return MFFTB_ERR_ARG;
    gen_u16_kernel<<<C->num_sms * 4, 256, 0, C->stream>>>(reinterpret_cast<uint16_t*>(A),
                                                          (long long)(szA + szF) / 2, 0x5EEDull);
    CUDA_OK(cudaGetLastError());
    if (kara && (long long)kdim * 4 * 16384LL > 2147483647LL) return MFFTB_ERR_ARG;
    if (J.zpS > 0) {
        // operands as a forward transform leaves them: at j = 0 and j = NB/2
        // Ahat[c] = Bhat[c] = 0 for c >= K/2, i.e. F planes [0, K/2) and
        // [K, K + K/2) of every digit (the checker then sums those zeros)
        for (int j = 0; j < NB; ++j) {
            if (!pw_half_point(J, j)) continue;
            for (int da = 0; da < dA; ++da)
                CUDA_OK(cudaMemsetAsync(A + ((long long)(j * dA + da) * K + K / 2) * rows * ld, 0,
                                        (size_t)(K / 2) * rows * ld, C->stream));
            for (int db = 0; db < dB; ++db) {
                int8_t* f0 = F + (long long)(j * dB + db) * (2 * K - 1) * cols * ld;
                CUDA_OK(cudaMemsetAsync(f0, 0, (size_t)(K / 2) * cols * ld, C->stream));
                CUDA_OK(cudaMemsetAsync(f0 + (long long)K * cols * ld, 0, (size_t)(K / 2) * cols * ld,
                                        C->stream));
            }
        }
    }
    CUDA_OK(cudaMemsetAsync(C->d_err, 0, 64, C->stream));
    PwLaunch L{};
    L.A = A;
    L.lda = ld;
    L.a_plane_bytes = (long long)arows * ld;
    L.a_planes = apl;
    L.F = F;
    L.ldf = ld;
    L.f_plane_bytes = (long long)cols * ld;
    L.f_planes = fpl;
    L.rows = rows;
    L.cols = cols;
    L.kdim = kdim;
    L.jobs = J;
    L.map_rows = arows;
    L.kara_stages = C->kara_stages;
    L.block_n = block_n;
    L.out = out;
    L.out_plane = (long long)rows * cols;
    L.ldo = cols;
    L.err = C->d_err;
    L.timeout_ns = C->timeout_ns;
    L.num_sms = C->num_sms;
    L.variant = kara ? 0 : variant;
    L.wave_counter = reinterpret_cast<unsigned int*>(C->d_err + 32);
    if ((rc = pointwise_launch(L, C->stream))) return set_err(C, rc, "pointwise launch failed");
    if ((rc = pointwise_check_launch(L, mism, dcnt, C->stream))) return rc;
    rc = mfftgpu_sync(C);
    if (rc) return rc;
    int h = 0;
    CUDA_OK(cudaMemcpy(&h, mism, sizeof h, cudaMemcpyDeviceToHost));
    *mismatches = h;
    return MFFTB_OK;
}

int mfftgpu_selftest_school(mfftgpu_ctx* C, int rows, int cols, int kdim, int LbA, int LbB,
                            int U, long long* mismatches) {
    if (!C || !mismatches || rows <= 0 || cols <= 0 || kdim <= 0 || cols % 16 || LbA < 1 ||
        LbB < 1 || U < 1)
        return MFFTB_ERR_ARG;
    // random digits in [-128, 127]: a chunk of U plane products must fit int32
    if ((long long)kdim * U * 16384LL > 2147483647LL) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const int ld = (kdim + 15) / 16 * 16;
    const int T = (LbA + LbB - 1 + 3) / 4 * 4;
    const int nchunk = (LbA + U - 1) / U;
    PwJobs J{T, 1, 1, 1, nchunk, T * nchunk, 1, LbA, LbB, U};
    const size_t szA = align256((size_t)LbA * rows * ld), szF = align256((size_t)LbB * cols * ld);
    const size_t szO = align256((size_t)J.njobs * rows * cols * 4);
    int rc = ensure(C, &C->ws, &C->ws_bytes, szA + szF + szO + 256);
    if (rc) return rc;
    C->b_valid = false;
    int8_t* A = reinterpret_cast<int8_t*>(C->ws);
    int8_t* F = A + szA;
    int32_t* out = reinterpret_cast<int32_t*>(F + szF);
    long long* dcnt = reinterpret_cast<long long*>(reinterpret_cast<char*>(out) + szO);
    int* mism = C->d_err + 8;
    gen_u16_kernel<<<C->num_sms * 4, 256, 0, C->stream>>>(reinterpret_cast<uint16_t*>(A),
                                                          (long long)(szA + szF) / 2, 0x5C001ull);
    CUDA_OK(cudaGetLastError());
    CUDA_OK(cudaMemsetAsync(C->d_err, 0, 64, C->stream));
    PwLaunch L{};
    L.A = A;
    L.lda = ld;
    L.a_plane_bytes = (long long)rows * ld;
    L.a_planes = LbA;
    L.F = F;
    L.ldf = ld;
    L.f_plane_bytes = (long long)cols * ld;
    L.f_planes = LbB;
    L.rows = rows;
    L.cols = cols;
    L.kdim = kdim;
    L.jobs = J;
    L.block_n = 128;
    L.out = out;
    L.out_plane = (long long)rows * cols;
    L.ldo = cols;
    L.err = C->d_err;
    L.timeout_ns = C->timeout_ns;
    L.num_sms = C->num_sms;
    L.wave_counter = reinterpret_cast<unsigned int*>(C->d_err + 32);
    if ((rc = pointwise_launch(L, C->stream))) return set_err(C, rc, "pointwise launch failed");
    if ((rc = pointwise_check_launch(L, mism, dcnt, C->stream))) return rc;
    rc = mfftgpu_sync(C);
    if (rc) return rc;
    int h = 0;
    CUDA_OK(cudaMemcpy(&h, mism, sizeof h, cudaMemcpyDeviceToHost));
    *mismatches = h;
    return MFFTB_OK;
}

int mfftgpu_selftest_timeout(mfftgpu_ctx* C, unsigned long long timeout_ns) {
    if (!C || timeout_ns == 0) return MFFTB_ERR_ARG;
    cudaSetDevice(C->device);
    const int n = 256;
    int rc = ensure(C, &C->ws, &C->ws_bytes, (size_t)3 * n * n * 4);
    if (rc) return rc;
    CUDA_OK(cudaMemsetAsync(C->d_err, 0, sizeof(int), C->stream));
    PwLaunch L{};
    L.A = reinterpret_cast<int8_t*>(C->ws);
    L.lda = n;
    L.a_plane_bytes = (long long)n * n;
    L.a_planes = 1;
    L.F = reinterpret_cast<int8_t*>(C->ws) + (size_t)n * n;
    L.ldf = n;
    L.f_plane_bytes = (long long)n * n;
    L.f_planes = 1;
    L.rows = n;
    L.cols = n;
    L.kdim = n;
    L.jobs = PwJobs{1, 1, 1, 1, 1, 1};
    L.block_n = 256;
    L.out = reinterpret_cast<int32_t*>(C->ws + (size_t)2 * n * n);
    L.out_plane = (long long)n * n;
    L.ldo = n;
    L.err = C->d_err;
    L.timeout_ns = timeout_ns;
    L.num_sms = C->num_sms;
    L.stall_producer = 1;
    if ((rc = pointwise_launch(L, C->stream))) return rc;
    return mfftgpu_sync(C);  // expected: MFFTGPU_ERR_TIMEOUT, context still usable
}

float mfftgpu_decode_words_f32(uint32_t* w, int nw, int bit_off, int S) {
    return decode_words_host(w, nw, bit_off, S);
}

double mfftgpu_decode_words_f64(uint32_t* w, int nw, int bit_off, int S) {
    return decode_words_host_f64(w, nw, bit_off, S);
}

int mfftgpu_decode_words_round(uint32_t* w, int nw, int bit_off, int bits, uint64_t* sig,
                               int* shift) {
    if (!w || nw <= 0 || bits < 1 || bits > 63 || !sig || !shift) return 0;
    return decode_words_round(w, nw, bit_off, bits, sig, shift);
}

}  // extern "C"
