// common.cuh -- shared device helpers for the gdl_b200 point-cloud graph kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gdl_b200.h"

#define GDL_RETURN_IF(cond, code) \
    do {                          \
        if (cond) return (code);  \
    } while (0)

#define GDL_CUDA_TRY(expr)                                \
    do {                                                  \
        cudaError_t _e = (expr);                          \
        if (_e != cudaSuccess) return GDL_ERR_CUDA;       \
    } while (0)

namespace gdl {

constexpr int kSmCount = 148;  // B200: 2 dies x 74 SMs

// ---------------------------------------------------------------- exact float ops
// The reference kernels are built with --use_fast_math (geoembodied/csrc/__init__.py:97-101),
// i.e. flush-to-zero single precision with FMA contraction. These wrappers pin each
// rounding step in PTX so the result does not depend on this library's own flags.
__device__ __forceinline__ float sub_ftz(float a, float b) {
    float r;
    asm("sub.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float mul_ftz(float a, float b) {
    float r;
    asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float add_ftz(float a, float b) {
    float r;
    asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float fma_ftz(float a, float b, float c) {
    float r;
    asm("fma.rn.ftz.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Squared distance with the rounding of the reference kernels' `dx*dx + dy*dy + dz*dz`
// (fps_kernel.cu:91-94, knn_kernel.cu:149-152, radius_graph_kernel.cu:224-227) as nvcc
// contracts it: fma(dz, dz, fma(dx, dx, dy*dy)), flush-to-zero. Pinned bit-for-bit against
// the distances the reference KNN kernel returns on a B200 (the other contractions differ).
__device__ __forceinline__ float dist2(float ax, float ay, float az, float bx, float by, float bz) {
    const float dx = sub_ftz(ax, bx);
    const float dy = sub_ftz(ay, by);
    const float dz = sub_ftz(az, bz);
    return fma_ftz(dz, dz, fma_ftz(dx, dx, mul_ftz(dy, dy)));
}

// ---------------------------------------------------------------- packed fp32x2 arithmetic
// sm_100a executes two fp32 lanes per instruction with the same IEEE rounding as the scalar
// forms (.rn, flush-to-zero), so the packed distance below is bit-identical to dist2().
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t dist2_x2(uint64_t qx, uint64_t qy, uint64_t qz, uint64_t sx, uint64_t sy,
                                             uint64_t sz) {
    uint64_t dx, dy, dz, r;
    asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(dx) : "l"(qx), "l"(sx));
    asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(dy) : "l"(qy), "l"(sy));
    asm("sub.rn.ftz.f32x2 %0, %1, %2;" : "=l"(dz) : "l"(qz), "l"(sz));
    asm("mul.rn.ftz.f32x2 %0, %1, %1;" : "=l"(r) : "l"(dy));
    asm("fma.rn.ftz.f32x2 %0, %1, %1, %2;" : "=l"(r) : "l"(dx), "l"(r));
    asm("fma.rn.ftz.f32x2 %0, %1, %1, %2;" : "=l"(r) : "l"(dz), "l"(r));
    return r;
}

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ unsigned warp_max_u32(unsigned v) { return __reduce_max_sync(0xffffffffu, v); }
__device__ __forceinline__ unsigned warp_min_u32(unsigned v) { return __reduce_min_sync(0xffffffffu, v); }

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// round-to-nearest-even float -> bfloat16 bits (NaN stays quiet NaN)
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

__host__ __device__ __forceinline__ int knn_bucket(int k) {  // knn_kernel.cu:253-288
    return k <= 4 ? 4 : k <= 8 ? 8 : k <= 16 ? 16 : k <= 32 ? 32 : 64;
}
__host__ __device__ __forceinline__ int radius_bucket(int k) {  // radius_graph_kernel.cu:372-420
    return k <= 16 ? 16 : k <= 32 ? 32 : 64;
}

// ---------------------------------------------------------------- MinK heap
// Restates MinK<K> (knn_kernel.cu:35-102, radius_graph_kernel.cu:34-85) with the capacity a
// runtime value: filled unsorted until full, heapified once, then the root is replaced by
// strictly smaller distances; `>` comparisons keep incumbents on ties. The arrays live in
// thread-local memory; the hot loops only touch them when a candidate beats the root.
struct MinKHeap {
    float d[64];
    int i[64];
    int count;
    int cap;

    __device__ __forceinline__ void init(int c) {
        count = 0;
        cap = c;
    }
    __device__ __forceinline__ float root_or_inf() const { return count >= cap ? d[0] : __int_as_float(0x7f800000); }
    __device__ __forceinline__ void sift_down(int at) {
        for (;;) {
            int l = 2 * at + 1, r = 2 * at + 2, g = at;
            if (l < cap && d[l] > d[g]) g = l;
            if (r < cap && d[r] > d[g]) g = r;
            if (g == at) break;
            float td = d[at];
            d[at] = d[g];
            d[g] = td;
            int ti = i[at];
            i[at] = i[g];
            i[g] = ti;
            at = g;
        }
    }
    __device__ __forceinline__ void add(float dist, int idx) {
        if (count >= cap) {
            if (dist >= d[0]) return;
            d[0] = dist;
            i[0] = idx;
            sift_down(0);
        } else {
            d[count] = dist;
            i[count] = idx;
            ++count;
            if (count == cap)
                for (int j = cap / 2 - 1; j >= 0; --j) sift_down(j);
        }
    }
    __device__ __forceinline__ void sort_ascending() {  // stable insertion sort, knn_kernel.cu:87-101
        for (int a = 1; a < count; ++a) {
            float kd = d[a];
            int ki = i[a];
            int b = a - 1;
            while (b >= 0 && d[b] > kd) {
                d[b + 1] = d[b];
                i[b + 1] = i[b];
                --b;
            }
            d[b + 1] = kd;
            i[b + 1] = ki;
        }
    }
};

// The same heap as free functions over caller-owned arrays, so the counter stays in a
// register while only the arrays live in local memory.
__device__ __forceinline__ void heap_sift_down(float *d, int *id, int cap, int at) {
    for (;;) {
        int l = 2 * at + 1, r = 2 * at + 2, g = at;
        if (l < cap && d[l] > d[g]) g = l;
        if (r < cap && d[r] > d[g]) g = r;
        if (g == at) break;
        const float td = d[at];
        d[at] = d[g];
        d[g] = td;
        const int ti = id[at];
        id[at] = id[g];
        id[g] = ti;
        at = g;
    }
}

__device__ __forceinline__ void heap_add(float *d, int *id, int &count, int cap, float dist, int idx) {
    if (count >= cap) {
        if (dist >= d[0]) return;
        d[0] = dist;
        id[0] = idx;
        heap_sift_down(d, id, cap, 0);
    } else {
        d[count] = dist;
        id[count] = idx;
        ++count;
        if (count == cap)
            for (int j = cap / 2 - 1; j >= 0; --j) heap_sift_down(d, id, cap, j);
    }
}

__device__ __forceinline__ void sort_ints(int *v, int count) {  // ascending insertion sort
    for (int a = 1; a < count; ++a) {
        const int x = v[a];
        int c = a - 1;
        while (c >= 0 && v[c] > x) {
            v[c + 1] = v[c];
            --c;
        }
        v[c + 1] = x;
    }
}

}  // namespace gdl
