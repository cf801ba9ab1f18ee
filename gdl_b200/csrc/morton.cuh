// morton.cuh -- per-cloud bounding boxes and 30-bit Morton codes of packed clouds (sm_100a).
//
// Used to group spatially close points: the bucketed FPS (buckets of consecutive points in
// Morton order, skipped per pick by an exact box bound) and the blocked KNN (source blocks and
// query tiles in Morton order). Only the grouping depends on this order, never a result.
#pragma once

#include "common.cuh"

namespace gdl {

// The quantisation below may round freely: the order only steers which points are grouped.
constexpr int kBoxThreads = 1024;

__device__ __forceinline__ uint32_t spread10(uint32_t v) {  // bits 0..9 -> bits 0, 3, ..., 27
    v &= 0x3ffu;
    v = (v | (v << 16)) & 0x030000ffu;
    v = (v | (v << 8)) & 0x0300f00fu;
    v = (v | (v << 4)) & 0x030c30c3u;
    v = (v | (v << 2)) & 0x09249249u;
    return v;
}

// Bounding box of each cloud: box[6b..6b+5] = (min x, y, z, max x, y, z); fminf / fmaxf skip NaN.
// bad (nullable): bad[b] = 1 if cloud b has a NaN or infinite coordinate, else 0.
static __global__ void __launch_bounds__(kBoxThreads) cloud_box_kernel(const float *__restrict__ pos,
                                                                       const int64_t *__restrict__ ptr,
                                                                       float *__restrict__ box,
                                                                       int32_t *__restrict__ bad) {
    __shared__ float part[6][kBoxThreads / 32];
    const int b = blockIdx.x;
    const int64_t start = ptr[b], n = ptr[b + 1] - start;
    float v[6] = {INFINITY, INFINITY, INFINITY, -INFINITY, -INFINITY, -INFINITY};
    bool nonfinite = false;
    for (int64_t i = threadIdx.x; i < n; i += kBoxThreads) {
        const float *p = pos + 3 * (start + i);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float x = p[c];
            v[c] = fminf(v[c], x);
            v[3 + c] = fmaxf(v[3 + c], x);
            nonfinite |= !isfinite(x);
        }
    }
    if (bad) {
        const int any = __syncthreads_or(nonfinite);
        if (threadIdx.x == 0) bad[b] = any ? 1 : 0;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            v[c] = fminf(v[c], __shfl_xor_sync(0xffffffffu, v[c], o));
            v[3 + c] = fmaxf(v[3 + c], __shfl_xor_sync(0xffffffffu, v[3 + c], o));
        }
    if (lane == 0)
#pragma unroll
        for (int c = 0; c < 6; ++c) part[c][warp] = v[c];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int c = 0; c < 6; ++c) {
            float x = part[c][lane];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float y = __shfl_xor_sync(0xffffffffu, x, o);
                x = c < 3 ? fminf(x, y) : fmaxf(x, y);
            }
            if (lane == 0) box[6 * b + c] = x;
        }
    }
}

__device__ __forceinline__ uint32_t morton_cell(float x, float lo, float scale) {
    const float t = (x - lo) * scale;
    if (!(t > 0.0f)) return 0u;  // below the box, NaN, or a degenerate axis
    return t >= 1023.0f ? 1023u : (uint32_t)t;
}

// 30-bit Morton code of every point over its cloud's box (1024 cells per axis). `ptr` gives the
// points' clouds, `box` one box per cloud (the points' own, or another set's with the same clouds).
// Codes go to keys[i] (or keys[i - ptr[0]] when `relative`), for indices below `limit` only.
// keys are 30-bit codes (10 bits per axis) shifted right by `shift` (a multiple of 3 keeps whole
// levels: 6 gives 24-bit codes, 8 bits per axis, for a three-pass 8-bit radix sort)
static __global__ void morton_code_kernel(const float *__restrict__ pos, const int64_t *__restrict__ ptr, int B,
                                          const float *__restrict__ box, uint32_t *__restrict__ keys,
                                          bool relative, int64_t limit, int shift = 0) {
    const int64_t first = ptr[0], last = ptr[B];
    for (int64_t i = first + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < last;
         i += (int64_t)gridDim.x * blockDim.x) {
        int lo = 0, hi = B - 1;  // the cloud of i: the last b with ptr[b] <= i
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (ptr[mid] <= i) lo = mid;
            else hi = mid - 1;
        }
        const float *bx = box + 6 * lo;
        uint32_t code = 0;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float ext = bx[3 + c] - bx[c];
            const float scale = (ext > 0.0f && ext < INFINITY) ? 1024.0f / ext : 0.0f;
            code |= spread10(morton_cell(pos[3 * i + c], bx[c], scale)) << c;
        }
        const int64_t at = relative ? i - first : i;  // relative: indexed from the first point of cloud 0
        if (at < limit) keys[at] = code >> shift;      // `keys` holds `limit` entries
    }
}

}  // namespace gdl
