// geom.cu -- edge geometry of COO edges and the per-cloud average degree (sm_100a).
//
// gdl_edge_geometry_coo replaces compute_edge_vectors + spherical_harmonics over an arbitrary
// edge list (functional/radius_graph.py:338-358, kernels/triton_sph_harm.py:200-240); the
// radius graph writes the same values from its emission kernel instead (radius.cu).
// gdl_cloud_avg_degree replaces the degree / scatter_add / per-cloud mean block of
// SpatialGraph.build and from_edge_index (nn/modules/spatial_graph.py:131-153, 225-239).
#include "common.cuh"
#include "geom.cuh"

namespace gdl {

// One warp per 32 consecutive edges; outputs staged per warp (warp_geom_emit).
__global__ void __launch_bounds__(256) edge_geom_coo_kernel(const float *__restrict__ x, int64_t n,
                                                            const int64_t *__restrict__ row,
                                                            const int64_t *__restrict__ col, int64_t E, EdgeGeom g) {
    __shared__ float stage[8 * kGeomStageFloats];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *st = stage + warp * kGeomStageFloats;
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    for (int64_t e0 = ((int64_t)blockIdx.x * 8 + warp) * 32; e0 < E; e0 += nwarps * 32) {
        const int cnt = (int)(E - e0 < 32 ? E - e0 : 32);
        float q3[3], s3[3];
        const float nan = __int_as_float(0x7fc00000);
        q3[0] = q3[1] = q3[2] = s3[0] = s3[1] = s3[2] = nan;
        if (lane < cnt) {
            const int64_t s = row[e0 + lane], q = col[e0 + lane];
            if (s >= 0 && s < n && q >= 0 && q < n) {
                q3[0] = x[3 * q], q3[1] = x[3 * q + 1], q3[2] = x[3 * q + 2];
                s3[0] = x[3 * s], s3[1] = x[3 * s + 1], s3[2] = x[3 * s + 2];
            }
        }
        warp_geom_emit(g, st, e0, cnt, lane, q3[0], q3[1], q3[2], s3[0], s3[1], s3[2]);
    }
}

// cloud of node i: batch[i], else the b with ptr[b] <= i < ptr[b+1], else 0 (one cloud); -1 outside
__device__ __forceinline__ int node_cloud(int64_t i, const int64_t *__restrict__ batch, const int64_t *__restrict__ ptr,
                                          int32_t B) {
    if (batch) {
        const int64_t b = batch[i];
        return (b >= 0 && b < B) ? (int)b : -1;
    }
    if (!ptr) return 0;
    if (i < ptr[0] || i >= ptr[B]) return -1;
    int lo = 0, hi = B - 1;  // largest b with ptr[b] <= i
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ptr[mid] <= i) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// sums[b] += degree, cnt[b] += 1 with 64-bit integer atomics (exact, order-free); a warp whose
// nodes share one cloud (contiguous clouds) adds its total once
__global__ void __launch_bounds__(256) cloud_degree_sum_kernel(const int32_t *__restrict__ node_start,
                                                               const int32_t *__restrict__ node_end, int64_t n,
                                                               const int64_t *__restrict__ batch,
                                                               const int64_t *__restrict__ ptr, int32_t B,
                                                               unsigned long long *__restrict__ sums,
                                                               unsigned long long *__restrict__ cnt) {
    const int lane = threadIdx.x & 31;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < n; base += stride) {
        const int64_t i = base + threadIdx.x;  // the whole warp iterates together
        const bool in = i < n;
        const int b = in ? node_cloud(i, batch, ptr, B) : -1;
        const long long deg = in ? (long long)node_end[i] - (long long)node_start[i] : 0;
        const int b0 = __shfl_sync(0xffffffffu, b, 0);
        if (__all_sync(0xffffffffu, !in || b == b0) && b0 >= 0) {
            long long t = deg;
            int c = in ? 1 : 0;
            for (int off = 16; off > 0; off >>= 1) {
                t += __shfl_xor_sync(0xffffffffu, t, off);
                c += __shfl_xor_sync(0xffffffffu, c, off);
            }
            if (lane == 0) {
                atomicAdd(&sums[b0], (unsigned long long)t);
                atomicAdd(&cnt[b0], (unsigned long long)c);
            }
        } else if (in && b >= 0) {
            atomicAdd(&sums[b], (unsigned long long)deg);
            atomicAdd(&cnt[b], 1ull);
        }
    }
}

__global__ void __launch_bounds__(256) cloud_avg_write_kernel(int64_t n, const int64_t *__restrict__ batch,
                                                              const int64_t *__restrict__ ptr, int32_t B,
                                                              const unsigned long long *__restrict__ sums,
                                                              const unsigned long long *__restrict__ cnt,
                                                              float *__restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = node_cloud(i, batch, ptr, B);
        float a = 1.0f;
        if (b >= 0) {
            const long long c = (long long)cnt[b];
            // cloud_sum / cloud_cnt.clamp(min=1), both exact in float below 2^24
            a = __fdiv_rn((float)(long long)sums[b], (float)(c > 1 ? c : 1));
            a = a < 1.0f ? 1.0f : a;  // clamp(min=1.0); NaN cannot occur
        }
        out[i] = a;
    }
}

// One pass over max(n, capacity) slots: the sort-free CSR fields of a destination-grouped edge
// list and, from the row pointer alone, each node's cloud average degree.
__global__ void __launch_bounds__(256) radius_csr_finish_kernel(const int64_t *__restrict__ row_ptr,
                                                                const int64_t *__restrict__ dst, int64_t n,
                                                                int64_t cap, const int64_t *__restrict__ ptr, int32_t B,
                                                                int32_t *__restrict__ col_sorted,
                                                                int32_t *__restrict__ perm,
                                                                int32_t *__restrict__ node_start,
                                                                int32_t *__restrict__ node_end,
                                                                float *__restrict__ avg) {
    const int64_t E = row_ptr[n];
    const int64_t m = n > E ? n : E;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        if (i < E && i < cap) {
            if (col_sorted) col_sorted[i] = (int32_t)dst[i];
            if (perm) perm[i] = (int32_t)i;
        }
        if (i < n) {
            const int64_t s = row_ptr[i], e = row_ptr[i + 1];
            const bool any = e > s;  // nodes without edges keep 0 / 0 (segment_reduce_kernel.cu:30-50)
            if (node_start) node_start[i] = any ? (int32_t)s : 0;
            if (node_end) node_end[i] = any ? (int32_t)e : 0;
            if (avg) {
                float a = 1.0f;
                long long edges = E, nodes = n;
                const int b = node_cloud(i, nullptr, ptr, B);
                if (ptr && b >= 0) {
                    edges = row_ptr[ptr[b + 1]] - row_ptr[ptr[b]];
                    nodes = ptr[b + 1] - ptr[b];
                }
                if (b >= 0) {
                    a = __fdiv_rn((float)edges, (float)(nodes > 1 ? nodes : 1));
                    a = a < 1.0f ? 1.0f : a;
                }
                avg[i] = a;
            }
        }
    }
}

inline unsigned grid_for(int64_t n) {
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = (int64_t)kSmCount * 8;
    return (unsigned)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace gdl

using namespace gdl;

extern "C" int gdl_edge_geometry_coo(const float *x, int64_t n_points, const int64_t *row, const int64_t *col,
                                     int64_t n_edges, const gdl_edge_geometry *geometry, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_points < 0 || n_edges < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(!edge_geom_valid(geometry), GDL_ERR_INVALID);
    const EdgeGeom g = edge_geom_from(x, geometry);
    if (n_edges == 0 || !g.x) return GDL_OK;
    GDL_RETURN_IF(!row || !col || (n_points > 0 && !x), GDL_ERR_INVALID);
    edge_geom_coo_kernel<<<grid_for(n_edges), 256, 0, st>>>(x, n_points, row, col, n_edges, g);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" size_t gdl_cloud_avg_degree_workspace_size(int32_t num_clouds) {
    const size_t b = num_clouds > 0 ? (size_t)num_clouds : 1;
    return (2 * b * sizeof(unsigned long long) + 255) & ~size_t(255);
}

extern "C" int gdl_cloud_avg_degree(const int32_t *node_start, const int32_t *node_end, int64_t n_nodes,
                                    const int64_t *batch, const int64_t *ptr, int32_t num_clouds, float *out,
                                    void *workspace, size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_nodes < 0 || num_clouds < 0, GDL_ERR_INVALID);
    if (n_nodes == 0) return GDL_OK;
    GDL_RETURN_IF(!node_start || !node_end || !out, GDL_ERR_INVALID);
    GDL_RETURN_IF((batch || ptr) && num_clouds < 1, GDL_ERR_INVALID);
    const int32_t B = (batch || ptr) ? num_clouds : 1;
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_cloud_avg_degree_workspace_size(B), GDL_ERR_WORKSPACE);
    unsigned long long *sums = (unsigned long long *)workspace, *cnt = sums + B;
    GDL_CUDA_TRY(cudaMemsetAsync(sums, 0, 2 * (size_t)B * sizeof(unsigned long long), st));
    cloud_degree_sum_kernel<<<grid_for(n_nodes), 256, 0, st>>>(node_start, node_end, n_nodes, batch, ptr, B, sums, cnt);
    cloud_avg_write_kernel<<<grid_for(n_nodes), 256, 0, st>>>(n_nodes, batch, ptr, B, sums, cnt, out);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_radius_csr_finish(const int64_t *row_ptr, const int64_t *dst, int64_t n_points, int64_t capacity,
                                     const int64_t *ptr, int32_t num_clouds, int32_t *col_sorted, int32_t *perm,
                                     int32_t *node_start, int32_t *node_end, float *avg_degree, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_points < 0 || capacity < 0 || num_clouds < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(!row_ptr || (ptr && num_clouds < 1), GDL_ERR_INVALID);
    GDL_RETURN_IF(col_sorted && !dst, GDL_ERR_INVALID);
    GDL_RETURN_IF(n_points >= INT32_MAX / 64, GDL_ERR_OVERFLOW);
    const int64_t slots = n_points > capacity ? n_points : capacity;
    if (slots == 0) return GDL_OK;
    radius_csr_finish_kernel<<<grid_for(slots), 256, 0, st>>>(row_ptr, dst, n_points, capacity, ptr, num_clouds,
                                                              col_sorted, perm, node_start, node_end, avg_degree);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
