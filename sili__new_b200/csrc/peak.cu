// FP32 FMA peak of the device: the denominator of the FP32 fraction the
// bench reports beside the HBM fraction for the issue-bound kernels (the
// fused update, the batched forwards).  Every thread runs 16 independent
// fma chains so the FMA pipes never wait on a result; the grid fills every
// SM at full occupancy several times over.
#include <cuda_runtime.h>

#include <string>

#include "kernels.cuh"
#include "sili_b200.h"

namespace sili {
int set_error(int code, const std::string& msg);
}

namespace {

constexpr int kChains = 16;

__global__ void __launch_bounds__(256) k_fma_peak(float seed, int iters, float* __restrict__ out) {
    float a[kChains];
#pragma unroll
    for (int j = 0; j < kChains; ++j) a[j] = seed + (float)(threadIdx.x + j);
    const float m = 0.999999f, c = 1e-7f;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int j = 0; j < kChains; ++j) a[j] = __fmaf_rn(a[j], m, c);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kChains; ++j) s += a[j];
    // written only for an impossible value, so the chains cannot be removed
    if (s == -1.2345f) out[blockIdx.x] = s;
}

}  // namespace

extern "C" int sili_fp32_fma_peak(int device, int iters, double* tflops, double* ms) {
    if (!tflops || iters <= 0) return sili::set_error(SILI_EINVAL, "fp32_fma_peak: bad arguments");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return sili::set_error(SILI_ECUDA, std::string("fp32_fma_peak: ") + cudaGetErrorString(e));
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int blocks = sms * 8 * 4;   // 8 resident 256-thread blocks per SM, 4 waves
    float* out = nullptr;
    cudaStream_t s = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float best = 0.f;
    if ((e = cudaMalloc(&out, (size_t)blocks * sizeof(float))) != cudaSuccess ||
        (e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreate(&e0)) != cudaSuccess || (e = cudaEventCreate(&e1)) != cudaSuccess)
        goto done;
    for (int rep = 0; rep < 6; ++rep) {   // first two: warm-up (clocks up)
        cudaEventRecord(e0, s);
        k_fma_peak<<<blocks, 256, 0, s>>>(1.0f, iters, out);
        sili::count_launch();
        cudaEventRecord(e1, s);
        if ((e = cudaEventSynchronize(e1)) != cudaSuccess) goto done;
        float t = 0.f;
        cudaEventElapsedTime(&t, e0, e1);
        if (rep >= 2 && (best == 0.f || t < best)) best = t;
    }
    e = cudaGetLastError();
done:
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (s) cudaStreamDestroy(s);
    if (out) cudaFree(out);
    if (e != cudaSuccess) return sili::set_error(SILI_ECUDA, std::string("fp32_fma_peak: ") + cudaGetErrorString(e));
    const double flops = 2.0 * kChains * (double)iters * 256.0 * (double)blocks;
    *tflops = flops / ((double)best * 1e-3) / 1e12;
    if (ms) *ms = best;
    return SILI_OK;
}
