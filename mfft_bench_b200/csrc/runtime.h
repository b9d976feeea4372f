// runtime.h -- host-side declarations shared by the CUDA translation units of
// libmfftb200: status codes, kernel launch descriptors and the launchers.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "pointwise.cuh"

// Status codes returned by every mfftgpu_* entry point (see include/mfftgpu.h).
enum {
    MFFTB_OK = 0,
    MFFTB_ERR_ARG = 1,        // invalid argument / shape / plan
    MFFTB_ERR_NOMEM = 2,      // device or pinned allocation failed
    MFFTB_ERR_CUDA = 3,       // CUDA runtime error
    MFFTB_ERR_TIMEOUT = 4,    // a bounded device-side wait ran out
    MFFTB_ERR_RANGE = 5,      // an input limb outside the documented range
    MFFTB_ERR_NODEVICE = 6,   // no sm_100 device available
    MFFTB_ERR_PLAN = 7,       // no exact plan fits int32/int64 headroom
    MFFTB_ERR_UNSUPPORTED = 8,
    MFFTB_ERR_DIST = 9,       // distributed orchestration error
};

namespace mfftb {

struct PwLaunch {
    const int8_t* A;          // Ahat planes [a_planes][rows][lda]
    long long lda, a_plane_bytes;
    int a_planes;
    const int8_t* F;          // F planes [f_planes][cols][ldf]  (B transposed)
    long long ldf, f_plane_bytes;
    int f_planes;
    int rows, cols, kdim;
    PwJobs jobs;
    int block_n;
    int32_t* out;             // [njobs][rows][ldo]
    long long out_plane;
    int ldo;
    int* err;
    unsigned long long timeout_ns;
    int num_sms;
    int stall_producer;       // self-test only: see PwParams
    int raster, group_m;      // tile order (see PwParams); 0 = defaults
    int variant;              // 0 auto, 1 one CTA per tile, 2 CTA pairs, 3 t-grouped CTA pairs
    unsigned int* wave_counter;  // optional 4-byte device word for wave alignment (see PwParams)
    int* chosen;              // optional host out: kernel used (1 single CTA, 2 pair, 3 grouped,
                              // 4 Karatsuba)
    int map_rows;             // Karatsuba mode: rows the A tensor map spans (>= rows, >= 256;
                              // the rows past `rows` lie inside the plane stride)
    int kara_stages;          // Karatsuba level 3: 4 four 48 KB stages; 0 / 2 two of 96 KB
};

int pointwise_launch(const PwLaunch& L, cudaStream_t stream);

}  // namespace mfftb

namespace mfftb {
// test-only: compares L.out with a CUDA-core evaluation of the job table
int pointwise_check_launch(const PwLaunch& L, int* d_mismatch, long long* d_first_bad,
                           cudaStream_t stream);
}  // namespace mfftb
