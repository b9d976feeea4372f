// noalloc.cu -- an exact 64-bit product that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a host framework that owns every
// device byte through its own pool and forbids side allocations, or a
// latency-critical caller that cannot afford cudaMalloc's implicit device
// synchronisation in the middle of its work.  mfftgpu_mm_i64_noalloc serves
// them: the caller passes device inputs and the device output, and every
// intermediate plane of the MFFT pipeline lives in one fixed scratch array in
// this file, a static __device__ array of kScratchBytes.  Every GPU that
// loads the library holds this array until the process exits.
//
// The same four kernels as the allocating path run on it (pack, forward
// transform, tcgen05 pointwise, inverse + carry); only where their buffers
// come from differs.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/mfftgpu.h"
#include "kernels.h"
#include "plan.h"
#include "runtime.h"

namespace {

constexpr size_t kScratchBytes = 32u << 20;  // 32 MiB per device: n <= 256 for W = 64

// the scratch; host code must not use this name as an address (see below)
static __device__ __align__(256) char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
// Per device, set up once with that device current: whether it is an sm_100
// GPU, its SM count, and the device address of g_noalloc_scratch (in host
// code g_noalloc_scratch is only a host-side stand-in for the symbol, not a
// device address).  Filled under g_setup_mutex, so concurrent first calls
// from several host threads are safe.  The cache assumes the device context
// lives as long as the process: after cudaDeviceReset the address is stale.
struct DeviceSetup {
    bool done = false;
    int status = 0;  // MFFTB_OK, or the error every later call returns
    int num_sms = 0;
    char* scratch = nullptr;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mutex;

int device_setup(int dev, int* num_sms, char** scratch) {
    using namespace mfftb;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceSetup& d = g_setup[dev];
    if (!d.done) {
        int major = 0, minor = 0, sms = 0;
        void* p = nullptr;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return MFFTB_ERR_CUDA;  // not cached: a later call may try again
        if (major != 10 || minor != 0) {
            d.status = MFFTB_ERR_NODEVICE;
        } else {
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p)
                return MFFTB_ERR_CUDA;
            d.scratch = static_cast<char*>(p);
            d.num_sms = sms;
        }
        d.done = true;
    }
    *num_sms = d.num_sms;
    *scratch = d.scratch;
    return d.status;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

int lg(int x) {
    int r = 0;
    while ((1 << r) < x) ++r;
    return r;
}

}  // namespace

extern "C" int mfftgpu_mm_i64_noalloc(const int64_t* A, const int64_t* B, int n, uint16_t* out,
                                      int RL, void* stream_handle) {
    using namespace mfftb;
    if (!A || !B || !out || n <= 0 || RL <= 0) return MFFTB_ERR_ARG;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MFFTB_ERR_CUDA;
    int num_sms = 0;
    char* scratch = nullptr;
    if (int rc0 = device_setup(dev, &num_sms, &scratch)) return rc0;
    cudaStream_t st = static_cast<cudaStream_t>(stream_handle);

    Plan P;
    if (plan_search(n, PLAN_VALUE, 64, 64, 0, 0, &P)) return MFFTB_ERR_PLAN;
    const int n_int = P.n_int;
    const long long nn = (long long)n_int * n_int;
    const int dbytes = plan_digit_bytes(P);
    const int fpl = P.NB * P.dB * (2 * P.K - 1), apl = P.NB * P.dA * P.K;
    const size_t szErr = 256;
    const size_t szDB = a256((size_t)P.LbB * nn * dbytes), szF = a256((size_t)fpl * nn);
    const size_t szDA = a256((size_t)P.LbA * nn * dbytes), szAh = a256((size_t)apl * nn);
    const size_t szAcc = a256((size_t)P.njobs * nn * 4);
    if (szErr + szDB + szF + szDA + szAh + szAcc > kScratchBytes) return MFFTB_ERR_ARG;  // too large
    int* err = reinterpret_cast<int*>(scratch);
    char* DB = scratch + szErr;
    int8_t* F = reinterpret_cast<int8_t*>(DB + szDB);
    char* DA = DB + szDB + szF;
    int8_t* Ah = reinterpret_cast<int8_t*>(DA + szDA);
    int32_t* acc = reinterpret_cast<int32_t*>(DA + szDA + szAh);

    // the array keeps the previous call's contents: the status word must start
    // at zero; every plane below is fully rewritten before it is read
    if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return MFFTB_ERR_CUDA;

    PackArgs pk{};
    pk.fmt = PACK_I64;
    pk.n = n;
    pk.L16 = 4;
    pk.W = 64;
    pk.is_signed = 1;
    pk.b = P.b;
    pk.ld = n_int;
    pk.plane = nn;
    pk.err = err;
    PackArgs pb = pk;
    pb.src = B;
    pb.Lb = P.LbB;
    pb.dst = DB;
    pb.rows = n_int;
    pb.transpose = 1;
    PackArgs pa = pk;
    pa.src = A;
    pa.Lb = P.LbA;
    pa.dst = DA;
    pa.rows = n_int;
    pa.transpose = 0;
    int rc;
    if ((rc = pack_launch(pb, st)) || (rc = pack_launch(pa, st))) return rc;

    FwdArgs f{};
    f.dbytes = dbytes;
    f.dplane = nn;
    f.nelem = nn;
    f.S = P.S;
    f.NB = P.NB;
    f.K = P.K;
    f.g = P.g;
    f.lgS = lg(P.S);
    f.lgK = lg(P.K);
    f.oplane = nn;
    f.err = err;
    f.b = P.b;
    FwdArgs fb = f;
    fb.D = DB;
    fb.Lb = P.LbB;
    fb.nc = P.ncB;
    fb.d = P.dB;
    fb.f_stack = 1;
    fb.out = F;
    FwdArgs fa = f;
    fa.D = DA;
    fa.Lb = P.LbA;
    fa.nc = P.ncA;
    fa.d = P.dA;
    fa.f_stack = 0;
    fa.out = Ah;
    if ((rc = forward_launch(fb, st)) || (rc = forward_launch(fa, st))) return rc;

    PwLaunch L{};
    L.A = Ah;
    L.lda = n_int;
    L.a_plane_bytes = nn;
    L.a_planes = apl;
    L.F = F;
    L.ldf = n_int;
    L.f_plane_bytes = nn;
    L.f_planes = fpl;
    L.rows = n_int;
    L.cols = n_int;
    L.kdim = n_int;
    L.jobs = PwJobs{P.K, P.dA, P.dB, P.nW, P.nchunk, P.njobs};
    L.block_n = n_int <= 64 ? 64 : (n_int <= 128 ? 128 : 256);
    L.out = acc;
    L.out_plane = nn;
    L.ldo = n_int;
    L.err = err;
    L.timeout_ns = 4000000000ull;
    L.num_sms = num_sms;
    if ((rc = pointwise_launch(L, st))) return rc;

    InvArgs ia{};
    ia.acc = acc;
    ia.acc_plane = nn;
    ia.lda = n_int;
    ia.rows = n;
    ia.cols = n;
    ia.S = P.S;
    ia.NB = P.NB;
    ia.K = P.K;
    ia.g = P.g;
    ia.nW = P.nW;
    ia.nchunk = P.nchunk;
    ia.log2NB = lg(P.NB);
    ia.lgS = lg(P.S);
    ia.lgK = lg(P.K);
    ia.b = P.b;
    ia.positions = P.positions;
    ia.out_kind = INV_U16;
    ia.out = out;
    ia.out_plane = (long long)n * n;
    ia.ldo = n;
    ia.RL = RL;
    int e = 32;
    while (e > 1 && (P.NB * P.K * e > 16 * 256 || (size_t)P.NB * P.K * e * 8 > 200 * 1024)) e >>= 1;
    ia.elems = e;
    ia.lgE = lg(e);
    ia.err = err;
    if ((rc = inverse_launch(ia, st))) return rc;

    // the status of the device-side checks (bounded waits, ranges): read back
    // into host stack memory, then the call returns
    int h = 0;
    if (cudaMemcpyAsync(&h, err, sizeof h, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return MFFTB_ERR_CUDA;
    return h;
}
