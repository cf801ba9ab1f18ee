// hybrid.cu -- radius graph + symmetric KNN fallback edges, deduplicated, in the reference's
// edge order, with its segment-reduce CSR (sm_100a).
//
// The reference's _EncoderStage._build_hybrid_graph (nn/modules/multi_scale_se3_net.py:
// 126-219) takes the radius graph, finds the nodes with fewer than k incoming edges, adds
// both directions of an edge to each such node's k nearest neighbours (knn_self with k + 1,
// column 0 dropped), deduplicates the concatenation through a hash `unique()` -- which also
// sorts it by (row, col) -- and then sorts it again by col for the CSR (from_edge_index ->
// sort_and_build_csr). Here the union is built per destination from counts and offsets (no
// hash), each destination's sources are sorted and deduplicated by one warp, and one stable
// radix sort by source gives the reference's (row, col) order; the CSR by col is the
// destination-grouped list itself, and perm is the inverse of that sort. Everything stays on
// the device: the edge count is written at out_row_ptr[n].
#include "common.cuh"
#include "geom.cuh"
#include "radix.cuh"

namespace gdl {

constexpr int kHyWarpSortMax = 128;  // rows up to this many candidates are sorted by one warp

// own[q] = radius in-degree + (isolated ? its valid fallback neighbours : 0); tot[q] += own[q];
// every fallback neighbour m of an isolated q gets one reverse candidate: tot[m] += 1
__global__ void hy_count_kernel(const int64_t *__restrict__ row_ptr, const int64_t *__restrict__ knn, int64_t n,
                                int kf, int32_t *__restrict__ own, int32_t *__restrict__ tot) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n; q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t deg = row_ptr[q + 1] - row_ptr[q];
        int nv = 0;
        if (deg < kf) {
            for (int j = 1; j <= kf; ++j) {
                const int64_t m = knn[q * (kf + 1) + j];
                if (m >= 0 && m < n) {
                    ++nv;
                    atomicAdd(&tot[m], 1);
                }
            }
        }
        own[q] = (int32_t)deg + nv;
        atomicAdd(&tot[q], (int32_t)deg + nv);
    }
}

// one warp per destination: copy its radius sources, append its fallback neighbours when
// isolated, and hand each of those neighbours a reverse candidate (slot order within a row is
// settled by the sort that follows)
__global__ void __launch_bounds__(256) hy_fill_kernel(const int64_t *__restrict__ row_ptr,
                                                      const int64_t *__restrict__ src, const int64_t *__restrict__ knn,
                                                      int64_t n, int kf, const int32_t *__restrict__ own,
                                                      const int64_t *__restrict__ off, int32_t *__restrict__ fillc,
                                                      int32_t *__restrict__ buf) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < n; q += warps) {
        const int64_t r0 = row_ptr[q], deg = row_ptr[q + 1] - r0, o = off[q];
        for (int64_t j = lane; j < deg; j += 32) buf[o + j] = (int32_t)src[r0 + j];
        if (deg < kf && lane == 0) {
            int64_t p = o + deg;
            for (int j = 1; j <= kf; ++j) {
                const int64_t m = knn[q * (kf + 1) + j];
                if (m >= 0 && m < n) {
                    buf[p++] = (int32_t)m;
                    const int slot = atomicAdd(&fillc[m], 1);
                    buf[off[m] + own[m] + slot] = (int32_t)q;
                }
            }
        }
    }
}

// ascending bitonic sort of NR * 32 keys held as element lane + 32 r in register r
template <int NR>
__device__ __forceinline__ void warp_bitonic(int32_t (&v)[NR], int lane) {
    constexpr int M = NR * 32;
#pragma unroll
    for (int size = 2; size <= M; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {  // partner in another register of the same lane
                const int rs = stride >> 5;
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    if (r & rs) continue;
                    const int i = lane + 32 * r;
                    const bool asc = (i & size) == 0 || size == M;
                    const int32_t a = v[r], b = v[r + rs];
                    const int32_t lo = a < b ? a : b, hi = a < b ? b : a;
                    v[r] = asc ? lo : hi;
                    v[r + rs] = asc ? hi : lo;
                }
            } else {
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    const int i = lane + 32 * r;
                    const int32_t p = __shfl_xor_sync(0xffffffffu, v[r], stride);
                    const bool asc = (i & size) == 0 || size == M;
                    const bool lower = (i & stride) == 0;
                    v[r] = (lower == asc) ? (v[r] < p ? v[r] : p) : (v[r] < p ? p : v[r]);
                }
            }
        }
    }
}

// sort + deduplicate the c candidates at row[0, c) in place; returns the distinct count
template <int NR>
__device__ __forceinline__ int warp_sort_unique(int32_t *__restrict__ row, int c, int lane) {
    int32_t v[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) v[r] = lane + 32 * r < c ? row[lane + 32 * r] : 0x7fffffff;
    warp_bitonic<NR>(v, lane);
    int base = 0;
    int32_t prev_last = 0;  // element 32 r - 1 (lane 31 of register r - 1)
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int i = lane + 32 * r;
        int32_t before = __shfl_up_sync(0xffffffffu, v[r], 1);
        if (lane == 0) before = prev_last;
        const bool u = i < c && (i == 0 || v[r] != before);
        const unsigned m = __ballot_sync(0xffffffffu, u);
        if (u) row[base + __popc(m & ((1u << lane) - 1))] = v[r];
        base += __popc(m);
        prev_last = __shfl_sync(0xffffffffu, v[r], 31);
    }
    return base;
}

__global__ void __launch_bounds__(256) hy_unique_kernel(const int32_t *__restrict__ tot,
                                                        const int64_t *__restrict__ off, int64_t n,
                                                        int32_t *__restrict__ buf, int32_t *__restrict__ ucnt) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < n; q += warps) {
        const int c = tot[q];
        int32_t *row = buf + off[q];
        __syncwarp();
        int u;
        if (c <= 64) {
            u = warp_sort_unique<2>(row, c, lane);
        } else if (c <= kHyWarpSortMax) {
            u = warp_sort_unique<4>(row, c, lane);
        } else {  // rare (many equal-distance neighbours): one lane, insertion sort in place
            u = 0;
            if (lane == 0) {
                for (int i = 1; i < c; ++i) {
                    const int32_t key = row[i];
                    int j = i - 1;
                    while (j >= 0 && row[j] > key) {
                        row[j + 1] = row[j];
                        --j;
                    }
                    row[j + 1] = key;
                }
                for (int i = 0; i < c; ++i)
                    if (i == 0 || row[i] != row[i - 1]) row[u++] = row[i];
            }
            u = __shfl_sync(0xffffffffu, u, 0);
        }
        if (lane == 0) ucnt[q] = u;
    }
}

// destination-grouped union -> sort keys (source) and the segment-reduce CSR fields; seg = {0, E}
// bounds the sort that follows to the edges (the count is only known on the device)
__global__ void __launch_bounds__(256) hy_emit_kernel(const int32_t *__restrict__ buf, const int64_t *__restrict__ off,
                                                      const int32_t *__restrict__ ucnt,
                                                      const int64_t *__restrict__ rp, int64_t n,
                                                      uint32_t *__restrict__ keys, int32_t *__restrict__ col_sorted,
                                                      int32_t *__restrict__ src_sorted,
                                                      int32_t *__restrict__ node_start, int32_t *__restrict__ node_end,
                                                      int64_t *__restrict__ seg) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        seg[0] = 0;
        seg[1] = rp[n];
    }
    for (int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < n; q += warps) {
        const int64_t o = rp[q], u = ucnt[q], b = off[q];
        for (int64_t j = lane; j < u; j += 32) {
            keys[o + j] = (uint32_t)buf[b + j];
            col_sorted[o + j] = (int32_t)q;
            if (src_sorted) src_sorted[o + j] = buf[b + j];
        }
        if (lane == 0) {
            node_start[q] = u > 0 ? (int32_t)o : 0;  // empty nodes 0 / 0 (segment_reduce_kernel.cu:30-50)
            node_end[q] = u > 0 ? (int32_t)(o + u) : 0;
        }
    }
}

// position i of the (row, col) order: the edge at destination-grouped slot p = sorted_pos[i]; one
// warp per 32 positions, writing each edge's geometry (staged per warp) when g.x is set
__global__ void __launch_bounds__(256) hy_order_kernel(const uint32_t *__restrict__ skeys,
                                                       const int32_t *__restrict__ spos,
                                                       const int32_t *__restrict__ col_sorted,
                                                       const int64_t *__restrict__ rp, int64_t n,
                                                       int64_t *__restrict__ out_row, int64_t *__restrict__ out_col,
                                                       int32_t *__restrict__ perm, EdgeGeom g) {
    __shared__ float stage[8 * kGeomStageFloats];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t E = rp[n];
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    for (int64_t base = ((int64_t)blockIdx.x * 8 + warp) * 32; base < E; base += nwarps * 32) {
        const int cnt = (int)(E - base < 32 ? E - base : 32);
        int64_t r = 0, c = 0;
        if (lane < cnt) {
            const int64_t i = base + lane;
            const int32_t p = spos[i];
            r = (int64_t)skeys[i];
            c = col_sorted[p];
            out_row[i] = r;
            out_col[i] = c;
            perm[p] = (int32_t)i;
        }
        if (g.x)  // destination = col, source = row: diff = x[col] - x[row]
            warp_geom_emit(g, stage + warp * kGeomStageFloats, base, cnt, lane, g.x[3 * c], g.x[3 * c + 1],
                           g.x[3 * c + 2], g.x[3 * r], g.x[3 * r + 1], g.x[3 * r + 2]);
    }
}

struct HybridWs {
    int32_t *own, *tot, *fillc, *ucnt, *buf, *spos;
    int64_t *off, *scan_scratch, *seg;
    uint32_t *keys, *skeys;
    RadixScratch rs;
};

inline int64_t hybrid_capacity(int64_t n, int cap_r, int kf) { return n * ((int64_t)cap_r + 2 * (int64_t)kf); }

inline size_t hybrid_ws(int64_t n, int64_t cap, char *base, HybridWs *w) {
    size_t o = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + o : nullptr;
        o += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t nn = n > 0 ? n : 1, cc = cap > 0 ? cap : 1;
    HybridWs t;
    t.own = (int32_t *)take(4 * nn);
    t.tot = (int32_t *)take(4 * nn);
    t.fillc = (int32_t *)take(4 * nn);
    t.ucnt = (int32_t *)take(4 * nn);
    t.off = (int64_t *)take(8 * (nn + 1));
    t.scan_scratch = (int64_t *)take(8 * (scan_blocks(nn) + 1));
    t.seg = (int64_t *)take(8 * 2);
    t.buf = (int32_t *)take(4 * cc);
    t.keys = (uint32_t *)take(4 * cc);
    t.skeys = (uint32_t *)take(4 * cc);
    t.spos = (int32_t *)take(4 * cc);
    char *rb = take(radix_scratch_bytes(cc, 1));
    if (base) t.rs = radix_carve(rb, cc, 1);
    if (w) *w = t;
    return o;
}

inline unsigned hy_grid(int64_t work, int per_block) {
    int64_t b = (work + per_block - 1) / per_block;
    const int64_t capb = (int64_t)kSmCount * 8;
    return (unsigned)(b < 1 ? 1 : (b > capb ? capb : b));
}

}  // namespace gdl

using namespace gdl;

extern "C" int64_t gdl_hybrid_graph_capacity(int64_t n_points, int32_t max_num_neighbors, int32_t knn_fallback_k) {
    const int cap_r = max_num_neighbors <= 16 ? 16 : max_num_neighbors <= 32 ? 32 : 64;
    return hybrid_capacity(n_points, cap_r, knn_fallback_k > 0 ? knn_fallback_k : 0);
}

extern "C" size_t gdl_hybrid_graph_workspace_size(int64_t n_points, int32_t max_num_neighbors,
                                                  int32_t knn_fallback_k) {
    return hybrid_ws(n_points, gdl_hybrid_graph_capacity(n_points, max_num_neighbors, knn_fallback_k), nullptr,
                     nullptr);
}

extern "C" int gdl_hybrid_graph(const float *x, const int64_t *radius_row_ptr, const int64_t *radius_src,
                                const int64_t *knn_idx, int64_t n_points, int32_t max_num_neighbors,
                                int32_t knn_fallback_k, int64_t *out_row_ptr, int64_t *out_row, int64_t *out_col,
                                int32_t *col_sorted, int32_t *perm, int32_t *src_sorted, int32_t *node_start,
                                int32_t *node_end, const gdl_edge_geometry *geometry, void *workspace,
                                size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_points < 0 || knn_fallback_k < 0 || knn_fallback_k > 64, GDL_ERR_INVALID);
    GDL_RETURN_IF(!edge_geom_valid(geometry), GDL_ERR_INVALID);
    const EdgeGeom geom = edge_geom_from(x, geometry);
    GDL_RETURN_IF(geom.x == nullptr && geometry && (geometry->diff || geometry->dist || geometry->direction ||
                                                    geometry->sph) && n_points > 0,
                  GDL_ERR_INVALID);
    GDL_RETURN_IF(!out_row_ptr, GDL_ERR_INVALID);
    const int64_t n = n_points;
    const int64_t cap = gdl_hybrid_graph_capacity(n, max_num_neighbors, knn_fallback_k);
    GDL_RETURN_IF(cap >= INT32_MAX || n >= INT32_MAX, GDL_ERR_OVERFLOW);
    if (n == 0) {
        GDL_CUDA_TRY(cudaMemsetAsync(out_row_ptr, 0, sizeof(int64_t), st));
        return GDL_OK;
    }
    GDL_RETURN_IF(!radius_row_ptr || !radius_src || (knn_fallback_k > 0 && !knn_idx), GDL_ERR_INVALID);
    GDL_RETURN_IF(!out_row || !out_col || !col_sorted || !perm || !node_start || !node_end, GDL_ERR_INVALID);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_hybrid_graph_workspace_size(n, max_num_neighbors, knn_fallback_k),
                  GDL_ERR_WORKSPACE);
    HybridWs w;
    hybrid_ws(n, cap, (char *)workspace, &w);
    const int kf = knn_fallback_k;
    GDL_CUDA_TRY(cudaMemsetAsync(w.tot, 0, sizeof(int32_t) * n, st));
    GDL_CUDA_TRY(cudaMemsetAsync(w.fillc, 0, sizeof(int32_t) * n, st));
    hy_count_kernel<<<hy_grid(n, 256), 256, 0, st>>>(radius_row_ptr, knn_idx, n, kf, w.own, w.tot);
    GDL_CUDA_TRY((exclusive_scan<int32_t, int64_t>(w.tot, w.off, n, w.scan_scratch, w.off + n, st)));
    hy_fill_kernel<<<hy_grid(n, 8), 256, 0, st>>>(radius_row_ptr, radius_src, knn_idx, n, kf, w.own, w.off, w.fillc,
                                                  w.buf);
    hy_unique_kernel<<<hy_grid(n, 8), 256, 0, st>>>(w.tot, w.off, n, w.buf, w.ucnt);
    GDL_CUDA_TRY((exclusive_scan<int32_t, int64_t>(w.ucnt, out_row_ptr, n, w.scan_scratch, out_row_ptr + n, st)));
    hy_emit_kernel<<<hy_grid(n, 8), 256, 0, st>>>(w.buf, w.off, w.ucnt, out_row_ptr, n, w.keys, col_sorted,
                                                  src_sorted, node_start, node_end, w.seg);
    int bits = 1;
    while (bits < 32 && ((int64_t)1 << bits) < n) ++bits;  // keys 0 .. n - 1
    GDL_CUDA_TRY(radix_sort_pairs(w.keys, nullptr, w.skeys, w.spos, cap, w.seg, 1, (bits + 7) / 8, nullptr, w.rs,
                                  st));
    hy_order_kernel<<<hy_grid(cap, 256), 256, 0, st>>>(w.skeys, w.spos, col_sorted, out_row_ptr, n, out_row, out_col,
                                                       perm, geom);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
