// radius.cu -- radius graph for packed, variable-size clouds (sm_100a), emitted as a CSR
// over destinations with ascending sources.
//
// Reference: geoembodied/csrc/radius_graph_kernel.cu:91-467 (cell binning, CUB sort, cell
// offsets, find_neighbors_kernel<K>, per-cloud host loop in radius_graph_cuda_batched).
//
// The reference decides which <= K neighbours a point keeps by feeding candidates, in a fixed
// order, to a MinK heap; with ties at the cut the kept SET depends on that order. So the grid,
// the order and the heap are reproduced exactly:
//   * grid per cloud: bbox of all its points -/+ 1e-5f, cell = r, res = ceil(extent/r)+1
//     capped at 1024 (:280-299), computed on the device in the same float arithmetic;
//   * points binned with clamping, masked points last (:91-127); stable sort by cell with the
//     point index as tie order (CUB radix sort of (cell, index), :319-347);
//   * each query scans the 27 cells around its UNclamped cell in (dx, dy, dz) order (:199-235);
//     the three z-cells of a (dx, dy) column are consecutive keys, so a column is one
//     contiguous run of the sorted array, found by binary search (no dense cell table);
//   * MinK<bucket(max_num_neighbors)> heap on d2 < r2 (strict), self skipped unless loop.
// B200 layout: all clouds in one launch per stage (no host loop, no host syncs), sorted
// coordinates gathered once as float4 for 16-byte loads in the candidate loop.
#include "common.cuh"
#include "radix.cuh"

namespace gdl {

struct GridParams {
    float mn[3];
    int res[3];
    int ncells;  // also the sort key of masked points
    int ok;      // cloud has >= 2 points
};

__device__ __forceinline__ int find_cloud_i(const int64_t *__restrict__ ptr, int B, int64_t q) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (ptr[mid] <= q) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

constexpr int kGridThreads = 256;

__global__ void __launch_bounds__(kGridThreads) rg_grid_kernel(const float *__restrict__ x,
                                                               const int64_t *__restrict__ ptr, float inv_cell,
                                                               GridParams *__restrict__ gp,
                                                               int32_t *__restrict__ key_bits) {
    __shared__ float smin[3][kGridThreads / 32], smax[3][kGridThreads / 32];
    const int b = blockIdx.x;
    const int64_t s0 = ptr[b], s1 = ptr[b + 1];
    float lo[3] = {__int_as_float(0x7f800000), __int_as_float(0x7f800000), __int_as_float(0x7f800000)};
    float hi[3] = {__int_as_float(0xff800000), __int_as_float(0xff800000), __int_as_float(0xff800000)};
    for (int64_t i = s0 + threadIdx.x; i < s1; i += kGridThreads)
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const float v = x[3 * i + a];
            lo[a] = fminf(lo[a], v);
            hi[a] = fmaxf(hi[a], v);
        }
#pragma unroll
    for (int a = 0; a < 3; ++a)
        for (int o = 16; o > 0; o >>= 1) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0)
        for (int a = 0; a < 3; ++a) {
            smin[a][w] = lo[a];
            smax[a][w] = hi[a];
        }
    __syncthreads();
    if (threadIdx.x == 0) {
        GridParams g;
        int64_t cells = 1;
        for (int a = 0; a < 3; ++a) {
            float l = smin[a][0], h = smax[a][0];
            for (int j = 1; j < kGridThreads / 32; ++j) {
                l = fminf(l, smin[a][j]);
                h = fmaxf(h, smax[a][j]);
            }
            // host arithmetic of the reference, in IEEE single precision (:283-297)
            const float mn = __fsub_rn(l, 1e-5f), mx = __fadd_rn(h, 1e-5f);
            const float c = ceilf(__fmul_rn(__fsub_rn(mx, mn), inv_cell));
            const int r = (c >= 1023.0f) ? 1024 : (int)c + 1;
            g.mn[a] = mn;
            g.res[a] = r < 1 ? 1 : r;
            cells *= g.res[a];
        }
        g.ncells = (int)cells;
        g.ok = (s1 - s0) > 1;
        gp[b] = g;
        int bits = 0;
        while (bits < 31 && ((int64_t)1 << bits) <= cells) ++bits;  // keys go up to ncells
        atomicMax(key_bits, bits);
    }
}

__device__ __forceinline__ int cell_coord(float p, float mn, float inv) {
    // __float2int_rd((p - min) * inv) under --use_fast_math (:117-119, :192-194)
    return __float2int_rd(mul_ftz(sub_ftz(p, mn), inv));
}

__global__ void rg_keys_kernel(const float *__restrict__ x, const int64_t *__restrict__ ptr, int32_t B,
                               const uint8_t *__restrict__ mask, float inv, const GridParams *__restrict__ gp,
                               uint32_t *__restrict__ keys) {
    const int64_t i = ptr[0] + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ptr[B]) return;
    const int b = find_cloud_i(ptr, B, i);
    const GridParams g = gp[b];
    if (!g.ok || (mask && !mask[i])) {
        keys[i] = (uint32_t)g.ncells;
        return;
    }
    int c[3];
#pragma unroll
    for (int a = 0; a < 3; ++a) {
        int v = cell_coord(x[3 * i + a], g.mn[a], inv);
        c[a] = v < 0 ? 0 : (v > g.res[a] - 1 ? g.res[a] - 1 : v);
    }
    keys[i] = (uint32_t)((c[0] * g.res[1] + c[1]) * g.res[2] + c[2]);
}

__global__ void rg_gather_kernel(const float *__restrict__ x, const int64_t *__restrict__ ptr, int32_t B,
                                 const int32_t *__restrict__ sorted_idx, float4 *__restrict__ sorted_pts) {
    const int64_t j = ptr[0] + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= ptr[B]) return;
    const int64_t o = sorted_idx[j];
    sorted_pts[j] = make_float4(x[3 * o], x[3 * o + 1], x[3 * o + 2], 0.0f);
}

__device__ __forceinline__ int64_t lower_bound_u32(const uint32_t *__restrict__ a, int64_t lo, int64_t hi, uint32_t v) {
    while (lo < hi) {
        const int64_t m = (lo + hi) >> 1;
        if (a[m] < v) lo = m + 1;
        else hi = m;
    }
    return lo;
}

constexpr int kQueryThreads = 128;

__global__ void __launch_bounds__(kQueryThreads) rg_query_kernel(
    const float *__restrict__ x, const int64_t *__restrict__ ptr, int32_t B, int64_t n, const uint8_t *__restrict__ mask,
    float r_sq, float inv, int loop, int cap, const GridParams *__restrict__ gp,
    const uint32_t *__restrict__ sorted_keys, const int32_t *__restrict__ sorted_idx,
    const float4 *__restrict__ sorted_pts, int32_t *__restrict__ counts, int32_t *__restrict__ padded) {
    const int64_t q = (int64_t)blockIdx.x * kQueryThreads + threadIdx.x;
    if (q >= n) return;
    if (q < ptr[0] || q >= ptr[B] || (mask && !mask[q])) {
        counts[q] = 0;
        return;
    }
    const int b = find_cloud_i(ptr, B, q);
    const GridParams g = gp[b];
    if (!g.ok) {
        counts[q] = 0;
        return;
    }
    const int64_t cs0 = ptr[b], cs1 = ptr[b + 1];
    const float qx = x[3 * q], qy = x[3 * q + 1], qz = x[3 * q + 2];
    const int qc[3] = {cell_coord(qx, g.mn[0], inv), cell_coord(qy, g.mn[1], inv), cell_coord(qz, g.mn[2], inv)};
    const int zlo = qc[2] - 1 < 0 ? 0 : qc[2] - 1;
    const int zhi = qc[2] + 1 > g.res[2] - 1 ? g.res[2] - 1 : qc[2] + 1;
    MinKHeap h;
    h.init(cap);
    if (zlo <= zhi) {
        for (int dx = -1; dx <= 1; ++dx) {
            const int cx = qc[0] + dx;
            if (cx < 0 || cx >= g.res[0]) continue;
            for (int dy = -1; dy <= 1; ++dy) {
                const int cy = qc[1] + dy;
                if (cy < 0 || cy >= g.res[1]) continue;
                const uint32_t col = (uint32_t)((cx * g.res[1] + cy) * g.res[2]);
                const int64_t j0 = lower_bound_u32(sorted_keys, cs0, cs1, col + (uint32_t)zlo);
                const int64_t j1 = lower_bound_u32(sorted_keys, j0, cs1, col + (uint32_t)zhi + 1u);
                for (int64_t j = j0; j < j1; ++j) {
                    const int o = sorted_idx[j];
                    if (!loop && o == (int)q) continue;
                    const float4 s = sorted_pts[j];
                    const float d = dist2(qx, qy, qz, s.x, s.y, s.z);
                    if (d < r_sq) h.add(d, o);
                }
            }
        }
    }
    // kept set, ascending source index
    int *keep = h.i;
    for (int a = 1; a < h.count; ++a) {
        const int v = keep[a];
        int c = a - 1;
        while (c >= 0 && keep[c] > v) {
            keep[c + 1] = keep[c];
            --c;
        }
        keep[c + 1] = v;
    }
    int32_t *dst = padded + q * cap;
    for (int a = 0; a < h.count; ++a) dst[a] = keep[a];
    counts[q] = h.count;
}

__global__ void rg_compact_kernel(const int32_t *__restrict__ counts, const int32_t *__restrict__ padded, int64_t n,
                                  int cap, const int64_t *__restrict__ row_ptr, int64_t *__restrict__ src,
                                  int64_t *__restrict__ dst) {
    // one warp per query row: lanes copy the row's entries
    const int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (q >= n) return;
    const int c = counts[q];
    const int64_t o = row_ptr[q];
    for (int a = lane; a < c; a += 32) {
        src[o + a] = padded[q * cap + a];
        if (dst) dst[o + a] = q;
    }
}

struct RadiusWs {
    GridParams *gp;
    int32_t *key_bits;
    uint32_t *keys, *sorted_keys;
    int32_t *sorted_idx, *counts, *padded;
    float4 *sorted_pts;
    int64_t *scan_scratch;
    RadixScratch rs;
};

static size_t radius_ws(int64_t n, int32_t B, int cap, char *base, RadiusWs *w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + off : nullptr;
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t nn = n > 0 ? n : 1;
    RadiusWs t;
    t.gp = (GridParams *)take(sizeof(GridParams) * (B > 0 ? B : 1));
    t.key_bits = (int32_t *)take(sizeof(int32_t));
    t.keys = (uint32_t *)take(sizeof(uint32_t) * nn);
    t.sorted_keys = (uint32_t *)take(sizeof(uint32_t) * nn);
    t.sorted_idx = (int32_t *)take(sizeof(int32_t) * nn);
    t.counts = (int32_t *)take(sizeof(int32_t) * nn);
    t.padded = (int32_t *)take(sizeof(int32_t) * nn * cap);
    t.sorted_pts = (float4 *)take(sizeof(float4) * nn);
    t.scan_scratch = (int64_t *)take(sizeof(int64_t) * (scan_blocks(nn) + 1));
    const size_t rbytes = radix_scratch_bytes(nn, B > 0 ? B : 1);
    char *rb = take(rbytes);
    if (base) t.rs = radix_carve(rb, nn, B > 0 ? B : 1);
    if (w) *w = t;
    return off;
}

}  // namespace gdl

using namespace gdl;

extern "C" size_t gdl_radius_graph_workspace_size(int64_t n_points, int32_t num_clouds, int32_t max_num_neighbors) {
    return radius_ws(n_points, num_clouds, radius_bucket(max_num_neighbors), nullptr, nullptr);
}

extern "C" int gdl_radius_graph(const float *x, const int64_t *ptr, int32_t num_clouds, int64_t n_points,
                                double radius, int32_t max_num_neighbors, int32_t loop, const uint8_t *mask,
                                int64_t *out_row_ptr, int64_t *out_src, int64_t *out_dst, void *workspace,
                                size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || n_points < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(!out_row_ptr, GDL_ERR_INVALID);
    GDL_RETURN_IF(n_points >= INT32_MAX / 64, GDL_ERR_OVERFLOW);
    const float r = (float)radius;  // radius_graph_kernel.cu:266
    if (n_points == 0 || num_clouds == 0 || !(r > 0.0f)) {
        GDL_CUDA_TRY(cudaMemsetAsync(out_row_ptr, 0, sizeof(int64_t) * (n_points + 1), st));
        return GDL_OK;
    }
    GDL_RETURN_IF(!x || !ptr || !out_src, GDL_ERR_INVALID);
    const int cap = radius_bucket(max_num_neighbors);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_radius_graph_workspace_size(n_points, num_clouds, max_num_neighbors),
                  GDL_ERR_WORKSPACE);
    RadiusWs w;
    radius_ws(n_points, num_clouds, cap, (char *)workspace, &w);
    const float r_sq = r * r;           // :274
    const float inv = 1.0f / r;         // :276 (host IEEE division)
    const unsigned g256 = (unsigned)((n_points + 255) / 256);
    GDL_CUDA_TRY(cudaMemsetAsync(w.key_bits, 0, sizeof(int32_t), st));
    rg_grid_kernel<<<num_clouds, kGridThreads, 0, st>>>(x, ptr, inv, w.gp, w.key_bits);
    rg_keys_kernel<<<g256, 256, 0, st>>>(x, ptr, num_clouds, mask, inv, w.gp, w.keys);
    GDL_CUDA_TRY(radix_sort_pairs(w.keys, nullptr, w.sorted_keys, w.sorted_idx, n_points, ptr, num_clouds, 4,
                                  w.key_bits, w.rs, st));
    rg_gather_kernel<<<g256, 256, 0, st>>>(x, ptr, num_clouds, w.sorted_idx, w.sorted_pts);
    rg_query_kernel<<<(unsigned)((n_points + kQueryThreads - 1) / kQueryThreads), kQueryThreads, 0, st>>>(
        x, ptr, num_clouds, n_points, mask, r_sq, inv, loop, cap, w.gp, w.sorted_keys, w.sorted_idx, w.sorted_pts,
        w.counts, w.padded);
    GDL_CUDA_TRY((exclusive_scan<int32_t, int64_t>(w.counts, out_row_ptr, n_points, w.scan_scratch,
                                                   out_row_ptr + n_points, st)));
    rg_compact_kernel<<<(unsigned)((n_points * 32 + 255) / 256), 256, 0, st>>>(w.counts, w.padded, n_points, cap,
                                                                             out_row_ptr, out_src, out_dst);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
