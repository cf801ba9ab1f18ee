// peak.cu -- FP32 FMA throughput of this device (no counterpart in the reference).
//
// The brute-force KNN scan and the FPS distance updates run on the FP32 pipe, whose peak the
// driver's measured peaks do not include. This kernel issues only independent fused
// multiply-adds (8 chains per thread, scalar fma.rn.f32 or packed fma.rn.f32x2), enough of
// them to hide the pipe's latency, on every SM, so a benchmark can state FP32 fractions against
// a measured number rather than a nominal one.
#include "common.cuh"

namespace gdl {

constexpr int kPeakThreads = 256;
constexpr int kPeakChains = 8;

template <bool PACKED>
__global__ void __launch_bounds__(kPeakThreads) fp32_peak_kernel(float *__restrict__ out, int64_t iters) {
    const float a = 1.0f + 1e-7f * (float)threadIdx.x, c = 1e-9f;
    if (PACKED) {
        uint64_t acc[kPeakChains];
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) acc[j] = pack2(0.5f * (float)j, 0.25f * (float)j);
        const uint64_t A = pack2(a, a), C = pack2(c, c);
        for (int64_t it = 0; it < iters; ++it)
#pragma unroll
            for (int j = 0; j < kPeakChains; ++j) asm volatile("fma.rn.f32x2 %0, %0, %1, %2;" : "+l"(acc[j]) : "l"(A), "l"(C));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) {
            float lo, hi;
            unpack2(acc[j], lo, hi);
            s += lo + hi;
        }
        if (s == 12345.0f) out[blockIdx.x * kPeakThreads + threadIdx.x] = s;  // keeps the chains live
    } else {
        float acc[kPeakChains];
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) acc[j] = 0.5f * (float)j;
        for (int64_t it = 0; it < iters; ++it)
#pragma unroll
            for (int j = 0; j < kPeakChains; ++j) asm volatile("fma.rn.f32 %0, %0, %1, %2;" : "+f"(acc[j]) : "f"(a), "f"(c));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < kPeakChains; ++j) s += acc[j];
        if (s == 12345.0f) out[blockIdx.x * kPeakThreads + threadIdx.x] = s;
    }
}

}  // namespace gdl

using namespace gdl;

extern "C" int64_t gdl_fp32_peak_flops(int64_t iters, int32_t packed, int32_t blocks) {
    return (int64_t)2 * kPeakChains * (packed ? 2 : 1) * iters * kPeakThreads * (int64_t)blocks;
}

extern "C" int gdl_fp32_peak(float *out, int64_t iters, int32_t packed, int32_t blocks, void *stream) {
    GDL_RETURN_IF(!out || iters <= 0 || blocks <= 0, GDL_ERR_INVALID);
    cudaStream_t st = (cudaStream_t)stream;
    if (packed) fp32_peak_kernel<true><<<blocks, kPeakThreads, 0, st>>>(out, iters);
    else fp32_peak_kernel<false><<<blocks, kPeakThreads, 0, st>>>(out, iters);
    return cudaGetLastError() == cudaSuccess ? GDL_OK : GDL_ERR_CUDA;
}
