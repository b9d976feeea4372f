// refgpu_mfft.cu -- TEST INFRASTRUCTURE ONLY: a command-line driver that
// runs ONE row of the reference's own CUDA benchmark, its GPU MFFT on the
// fp32 fixed-point embedding ("limb-mfft-fp32": mfft_float_gemm,
// cuda/gemm_bench.cu:1593-1701; CUDA-core int32 x int32 -> int64 plane
// products k_igemm32, cuda/mfft_gpu.cuh:197-250), on inputs given in a file,
// so that it can be timed and compared beside this repository's tcgen05
// path on the same B200 and the same inputs.
//
// The reference's gemm_bench.cu is compiled where it lies (oracle/Makefile,
// target refgpu: -I the reference's cuda/ directory); its own main() is
// renamed so that this file's main() picks the one row.  Nothing here is
// linked into the product library.
//
//   refgpu_mfft N REPS IN OUT
//     IN : 2*N*N float32, A then B, row-major
//     OUT: N*N float32, the product rounded by the reference's k_decode
//   prints the reference's own plan line, then one JSON line:
//     {"n":N,"ms":best-of-REPS,"gemms":plane products,"LA":..,"LB":..,"sms":..}
#define main gemm_bench_main
#include "gemm_bench.cu"
#undef main

int main(int argc, char** argv) {
    if (argc != 5) {
        fprintf(stderr, "usage: %s N REPS IN OUT\n", argv[0]);
        return 2;
    }
    const int n = atoi(argv[1]), reps = atoi(argv[2]);
    if (n <= 0 || reps <= 0) return 2;
    const size_t nn = (size_t)n * n;
    float* h = (float*)malloc(2 * nn * sizeof(float));
    if (!h) return 3;
    FILE* f = fopen(argv[3], "rb");
    if (!f || fread(h, sizeof(float), 2 * nn, f) != 2 * nn) {
        fprintf(stderr, "cannot read %s\n", argv[3]);
        return 3;
    }
    fclose(f);
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, 0));
    g_sms = prop.multiProcessorCount;
    float *dA, *dB, *dC;
    CK(cudaMalloc(&dA, nn * sizeof(float)));
    CK(cudaMalloc(&dB, nn * sizeof(float)));
    CK(cudaMalloc(&dC, nn * sizeof(float)));
    CK(cudaMemcpy(dA, h, nn * sizeof(float), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dB, h + nn, nn * sizeof(float), cudaMemcpyHostToDevice));
    cublasHandle_t hb;
    CB(cublasCreate(&hb));
    // the reference's grid for these inputs (24-bit significands, exponent
    // range scanned on the host), as its main() builds it for the fp32 rows
    LimbPlan pf = plan_limbs(h, h + nn, nn, 24);
    long long gemms = 0;
    double ms = mfft_float_gemm(hb, n, dA, dB, dC, pf, reps, &gemms);
    CK(cudaMemcpy(h, dC, nn * sizeof(float), cudaMemcpyDeviceToHost));
    f = fopen(argv[4], "wb");
    if (!f || fwrite(h, sizeof(float), nn, f) != nn) {
        fprintf(stderr, "cannot write %s\n", argv[4]);
        return 3;
    }
    fclose(f);
    printf("{\"n\": %d, \"ms\": %.3f, \"gemms\": %lld, \"LA\": %d, \"LB\": %d, \"sms\": %d}\n", n,
           ms, gemms, pf.LA, pf.LB, g_sms);
    cublasDestroy(hb);
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dC);
    free(h);
    return gemms > 0 ? 0 : 4;
}
