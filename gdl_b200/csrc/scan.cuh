// scan.cuh -- device-wide exclusive prefix sums (reduce-then-scan, three short launches).
#pragma once

#include "common.cuh"

namespace gdl {

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;  // elements per block

template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T *warp_sums, T *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    T inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T w = lane < nwarps ? warp_sums[lane] : T(0);
        T wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            T t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < nwarps) warp_sums[lane] = wi - w;  // exclusive warp offsets
        if (lane == 31) *total = wi;
    }
    __syncthreads();
    T r = warp_sums[warp] + inc - v;
    __syncthreads();
    return r;
}

// Block-local exclusive scan of in[0, n) -> out (as TOut); block sums -> totals[blockIdx.x].
template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kScanThreads) scan_local_kernel(const TIn *__restrict__ in, TOut *__restrict__ out,
                                                                 TOut *__restrict__ totals, int64_t n) {
    __shared__ TOut warp_sums[32];
    __shared__ TOut total;
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    TOut v[kScanItems];
    TOut s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        v[i] = (base + i < n) ? (TOut)in[base + i] : TOut(0);
        s += v[i];
    }
    TOut off = block_exclusive_scan<TOut>(s, warp_sums, &total);
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        if (base + i < n) out[base + i] = off;
        off += v[i];
    }
    if (threadIdx.x == 0) totals[blockIdx.x] = total;
}

// In-place exclusive scan of totals[0, m) by one block (any m); grand total -> *grand.
template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_totals_kernel(T *__restrict__ totals, int64_t m,
                                                                  T *__restrict__ grand) {
    __shared__ T warp_sums[32];
    __shared__ T total;
    T carry = 0;
    for (int64_t b0 = 0; b0 < m; b0 += kScanTile) {
        const int64_t base = b0 + (int64_t)threadIdx.x * kScanItems;
        T v[kScanItems];
        T s = 0;
#pragma unroll
        for (int i = 0; i < kScanItems; ++i) {
            v[i] = (base + i < m) ? totals[base + i] : T(0);
            s += v[i];
        }
        T off = block_exclusive_scan<T>(s, warp_sums, &total) + carry;
#pragma unroll
        for (int i = 0; i < kScanItems; ++i) {
            if (base + i < m) totals[base + i] = off;
            off += v[i];
        }
        carry += total;
    }
    if (threadIdx.x == 0 && grand) *grand = carry;
}

template <typename T>
__global__ void scan_add_kernel(T *__restrict__ out, const T *__restrict__ totals, int64_t n, T *__restrict__ tail,
                                const T *__restrict__ grand) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] += totals[i / kScanTile];
    if (i == 0 && tail) *tail = *grand;
}

inline int64_t scan_blocks(int64_t n) { return (n + kScanTile - 1) / kScanTile; }

// scratch: scan_blocks(n) + 1 elements of TOut
template <typename TIn, typename TOut>
inline cudaError_t exclusive_scan(const TIn *in, TOut *out, int64_t n, TOut *scratch, TOut *tail,
                                  cudaStream_t stream) {
    const int64_t nb = scan_blocks(n);
    if (n > 0) scan_local_kernel<TIn, TOut><<<(unsigned)nb, kScanThreads, 0, stream>>>(in, out, scratch, n);
    scan_totals_kernel<TOut><<<1, kScanThreads, 0, stream>>>(scratch, nb, scratch + nb);
    const int64_t nt = n > 0 ? n : 1;
    scan_add_kernel<TOut><<<(unsigned)((nt + 255) / 256), 256, 0, stream>>>(out, scratch, n, tail, scratch + nb);
    return cudaGetLastError();
}

}  // namespace gdl
