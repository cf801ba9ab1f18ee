// aggregate.cu -- weighted sums of KNN-gathered neighbour rows, forward and backward (sm_100a).
//
// The consumers of a KNN graph in the reference reduce each query's k gathered rows with
// per-neighbour weights, materialising [n_query, k, dim] gathers with torch indexing first:
//   EquivariantPool      s_out = (w[..., None] * scalars[idx]).sum(1), v_out likewise
//                        (nn/modules/equivariant_pool.py:395-420)
//   EquivariantInterpolate  w = inverse-distance weights of the k nearest coarse points,
//                        s/v/t2 = sum_k w * feat[idx] (nn/modules/equivariant_interp.py:91-125)
// Here one pass reads each neighbour row once and writes the reduced row; nothing of size
// [n_query, k, dim] exists. Every output is an fp32 fold in k order starting from 0 with the
// product rounded first (w * f, then +), i.e. the reference's evaluation order for k <= 8.
// Neighbours with idx < 0 (KNN padding) or idx >= n_src are skipped; the reference multiplies
// them by a zero weight, which only differs when the skipped row holds inf or NaN.
//
// Backward w.r.t. the source rows is a segment sum over a transposed graph: the (query, slot)
// pairs are stably sorted by their source index (radix sort), and each source row folds
// w * grad_out[query] over its pairs in (query, slot) order -- deterministic, no atomics, and
// the order a sequential CPU index_add of the reference's autograd would use.
#include "common.cuh"
#include "radix.cuh"

namespace gdl {

// w[q, k] = inv_k / max(sum_k inv_k, 1e-8) with inv_k = 1 / sqrt(max(dist, 1e-4)), 0 where
// idx < 0 (equivariant_interp.py:92-96). One thread per query; the sum runs in k order.
__global__ void __launch_bounds__(256) knn_idw_weights_kernel(const int64_t *__restrict__ idx,
                                                              const float *__restrict__ dist, int64_t n_q, int K,
                                                              float *__restrict__ w) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n_q; q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t *iq = idx + q * K;
        const float *dq = dist + q * K;
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            float v = 0.0f;
            if (iq[k] >= 0) {
                float d = dq[k];
                d = d < 1e-4f ? 1e-4f : d;  // clamp(min=1e-4); NaN stays NaN
                v = __fdiv_rn(1.0f, __fsqrt_rn(d));
            }
            s = __fadd_rn(s, v);
        }
        s = s < 1e-8f ? 1e-8f : s;
        for (int k = 0; k < K; ++k) {
            float v = 0.0f;
            if (iq[k] >= 0) {
                float d = dq[k];
                d = d < 1e-4f ? 1e-4f : d;
                v = __fdiv_rn(1.0f, __fsqrt_rn(d));
            }
            w[q * K + k] = __fdiv_rn(v, s);
        }
    }
}

template <int VEC>
struct Vec;
template <>
struct Vec<4> {
    using T = float4;
    __device__ static float get(const T &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
    __device__ static void set(T &v, int i, float f) {
        if (i == 0) v.x = f;
        else if (i == 1) v.y = f;
        else if (i == 2) v.z = f;
        else v.w = f;
    }
};
template <>
struct Vec<1> {
    using T = float;
    __device__ static float get(const T &v, int) { return v; }
    __device__ static void set(T &v, int, float f) { v = f; }
};

// out[q, :] = sum_k w[q, k] * src[idx[q, k], :]. Consecutive threads cover consecutive VEC-float
// pieces of one output row, so the gathered source rows and the output row are read and written
// coalesced; the k indices and weights of a query are warp-broadcast loads.
template <int VEC>
__global__ void __launch_bounds__(256) knn_wsum_kernel(const float *__restrict__ src, int64_t n_src, int64_t vpr,
                                                       const int64_t *__restrict__ idx, const float *__restrict__ w,
                                                       int64_t n_q, int K, float *__restrict__ out) {
    using V = Vec<VEC>;
    using T = typename V::T;
    const T *s4 = reinterpret_cast<const T *>(src);
    T *o4 = reinterpret_cast<T *>(out);
    const int64_t total = n_q * vpr;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t q = t / vpr, v = t - q * vpr;
        const int64_t *iq = idx + q * K;
        const float *wq = w + q * K;
        float acc[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
#pragma unroll 4
        for (int k = 0; k < K; ++k) {
            const int64_t s = iq[k];
            if (s >= 0 && s < n_src) {
                const float wk = wq[k];
                const T f = s4[s * vpr + v];
#pragma unroll
                for (int i = 0; i < VEC; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(wk, V::get(f, i)));
            }
        }
        T r;
#pragma unroll
        for (int i = 0; i < VEC; ++i) V::set(r, i, acc[i]);
        o4[t] = r;
    }
}

// ------------------------------------------------------------------ backward
__global__ void knn_pair_keys_kernel(const int64_t *__restrict__ idx, int64_t m, int64_t n_src,
                                     uint32_t *__restrict__ keys) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t s = idx[i];
        keys[i] = (uint32_t)((s >= 0 && s < n_src) ? s : n_src);  // skipped pairs sort last
    }
}

// [ns[s], ne[s]) = the sorted pairs of source s (0 / 0 for sources without pairs)
__global__ void knn_pair_offsets_kernel(const uint32_t *__restrict__ sk, int64_t m, int64_t n_src,
                                        int32_t *__restrict__ ns, int32_t *__restrict__ ne) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t v = sk[i];
        if ((int64_t)v >= n_src) continue;
        if (i == 0 || sk[i - 1] != v) ns[v] = (int32_t)i;
        if (i == m - 1 || sk[i + 1] != v) ne[v] = (int32_t)(i + 1);
    }
}

// grad_src[s, :] = sum over the pairs p of s (ascending) of w[p] * grad_out[p / K, :]
template <int VEC>
__global__ void __launch_bounds__(256) knn_wsum_bwd_kernel(const float *__restrict__ gout, int64_t vpr,
                                                           const int32_t *__restrict__ perm,
                                                           const int32_t *__restrict__ ns,
                                                           const int32_t *__restrict__ ne,
                                                           const float *__restrict__ w, int K, int64_t n_src,
                                                           float *__restrict__ gsrc) {
    using V = Vec<VEC>;
    using T = typename V::T;
    const T *g4 = reinterpret_cast<const T *>(gout);
    T *o4 = reinterpret_cast<T *>(gsrc);
    const int64_t total = n_src * vpr;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t s = t / vpr, v = t - s * vpr;
        float acc[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
        const int32_t j1 = ne[s];
        for (int32_t j = ns[s]; j < j1; ++j) {
            const int32_t p = perm[j];
            const float wk = w[p];
            const T g = g4[(int64_t)(p / K) * vpr + v];
#pragma unroll
            for (int i = 0; i < VEC; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(wk, V::get(g, i)));
        }
        T r;
#pragma unroll
        for (int i = 0; i < VEC; ++i) V::set(r, i, acc[i]);
        o4[t] = r;
    }
}

// grad_w[q, k] (+)= sum_c grad_out[q, c] * src[idx[q, k], c]: one warp per (q, k), lanes over c
// (lane-strided partial sums, then a fixed butterfly), skipped pairs get 0.
__global__ void __launch_bounds__(256) knn_wsum_wgrad_kernel(const float *__restrict__ gout,
                                                             const float *__restrict__ src, int64_t n_src,
                                                             int64_t dim, const int64_t *__restrict__ idx,
                                                             int64_t m, int K, int accumulate,
                                                             float *__restrict__ gw) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t p = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < m; p += warps) {
        const int64_t s = idx[p];
        float acc = 0.0f;
        if (s >= 0 && s < n_src) {
            const float *g = gout + (p / K) * dim;
            const float *f = src + s * dim;
            for (int64_t c = lane; c < dim; c += 32) acc = __fadd_rn(acc, __fmul_rn(g[c], f[c]));
        }
        for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) gw[p] = accumulate ? __fadd_rn(gw[p], acc) : acc;
    }
}

inline unsigned agg_grid(int64_t work) {
    int64_t b = (work + 255) / 256;
    const int64_t cap = (int64_t)kSmCount * 8;
    return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

inline bool vec4_ok(const void *a, const void *b, int64_t dim) {
    return dim % 4 == 0 && ((uintptr_t)a % 16 == 0) && ((uintptr_t)b % 16 == 0);
}

struct KnnTransposeWs {
    uint32_t *keys, *sorted_keys;
    int32_t *perm, *ns, *ne;
    RadixScratch rs;
};

inline size_t knn_transpose_ws(int64_t m, int64_t n_src, char *base, KnnTransposeWs *w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + off : nullptr;
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t mm = m > 0 ? m : 1, nn = n_src > 0 ? n_src : 1;
    KnnTransposeWs t;
    t.keys = (uint32_t *)take(sizeof(uint32_t) * mm);
    t.sorted_keys = (uint32_t *)take(sizeof(uint32_t) * mm);
    t.perm = (int32_t *)take(sizeof(int32_t) * mm);
    t.ns = (int32_t *)take(sizeof(int32_t) * nn);
    t.ne = (int32_t *)take(sizeof(int32_t) * nn);
    char *rb = take(radix_scratch_bytes(mm, 1));
    if (base) t.rs = radix_carve(rb, mm, 1);
    if (w) *w = t;
    return off;
}

}  // namespace gdl

using namespace gdl;

extern "C" int gdl_knn_idw_weights(const int64_t *idx, const float *dist, int64_t n_query, int32_t k,
                                   float *out_weight, void *stream) {
    GDL_RETURN_IF(n_query < 0 || k < 0, GDL_ERR_INVALID);
    if (n_query == 0 || k == 0) return GDL_OK;
    GDL_RETURN_IF(!idx || !dist || !out_weight, GDL_ERR_INVALID);
    knn_idw_weights_kernel<<<agg_grid(n_query), 256, 0, (cudaStream_t)stream>>>(idx, dist, n_query, k, out_weight);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_knn_weighted_sum(const float *src, int64_t n_src, int64_t dim, const int64_t *idx,
                                    const float *weight, int64_t n_query, int32_t k, float *out, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_src < 0 || dim < 0 || n_query < 0 || k < 0, GDL_ERR_INVALID);
    if (n_query == 0 || dim == 0) return GDL_OK;
    GDL_RETURN_IF(!out, GDL_ERR_INVALID);
    if (k == 0) {
        GDL_CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * n_query * dim, st));
        return GDL_OK;
    }
    GDL_RETURN_IF(!idx || !weight || (n_src > 0 && !src), GDL_ERR_INVALID);
    if (vec4_ok(src, out, dim)) {
        const int64_t vpr = dim / 4;
        knn_wsum_kernel<4><<<agg_grid(n_query * vpr), 256, 0, st>>>(src, n_src, vpr, idx, weight, n_query, k, out);
    } else {
        knn_wsum_kernel<1><<<agg_grid(n_query * dim), 256, 0, st>>>(src, n_src, dim, idx, weight, n_query, k, out);
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" size_t gdl_knn_weighted_sum_backward_workspace_size(int64_t n_query, int32_t k, int64_t n_src) {
    return knn_transpose_ws(n_query * (k > 0 ? k : 0), n_src, nullptr, nullptr);
}

extern "C" int gdl_knn_weighted_sum_backward(const float *const *grad_out, float *const *grad_src,
                                             const int64_t *dims, int32_t n_tables, const int64_t *idx,
                                             const float *weight, int64_t n_query, int32_t k, int64_t n_src,
                                             void *workspace, size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_query < 0 || k < 0 || n_src < 0 || n_tables < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(n_tables > 0 && (!grad_out || !grad_src || !dims), GDL_ERR_INVALID);
    const int64_t m = n_query * k;
    GDL_RETURN_IF(m >= INT32_MAX || n_src >= INT32_MAX, GDL_ERR_OVERFLOW);
    if (n_src == 0 || n_tables == 0) return GDL_OK;
    for (int t = 0; t < n_tables; ++t) GDL_RETURN_IF(dims[t] < 0 || (dims[t] > 0 && !grad_src[t]), GDL_ERR_INVALID);
    if (m == 0) {
        for (int t = 0; t < n_tables; ++t)
            if (dims[t] > 0) GDL_CUDA_TRY(cudaMemsetAsync(grad_src[t], 0, sizeof(float) * n_src * dims[t], st));
        return GDL_OK;
    }
    GDL_RETURN_IF(!idx || !weight, GDL_ERR_INVALID);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_knn_weighted_sum_backward_workspace_size(n_query, k, n_src),
                  GDL_ERR_WORKSPACE);
    KnnTransposeWs w;
    knn_transpose_ws(m, n_src, (char *)workspace, &w);
    GDL_CUDA_TRY(cudaMemsetAsync(w.ns, 0, sizeof(int32_t) * n_src, st));
    GDL_CUDA_TRY(cudaMemsetAsync(w.ne, 0, sizeof(int32_t) * n_src, st));
    knn_pair_keys_kernel<<<agg_grid(m), 256, 0, st>>>(idx, m, n_src, w.keys);
    int bits = 1;
    while (bits < 32 && ((int64_t)1 << bits) <= n_src) ++bits;  // keys 0 .. n_src
    GDL_CUDA_TRY(radix_sort_pairs(w.keys, nullptr, w.sorted_keys, w.perm, m, nullptr, 1, (bits + 7) / 8, nullptr,
                                  w.rs, st));
    knn_pair_offsets_kernel<<<agg_grid(m), 256, 0, st>>>(w.sorted_keys, m, n_src, w.ns, w.ne);
    for (int t = 0; t < n_tables; ++t) {
        const int64_t dim = dims[t];
        if (dim == 0) continue;
        GDL_RETURN_IF(!grad_out[t], GDL_ERR_INVALID);
        if (vec4_ok(grad_out[t], grad_src[t], dim))
            knn_wsum_bwd_kernel<4><<<agg_grid(n_src * (dim / 4)), 256, 0, st>>>(grad_out[t], dim / 4, w.perm, w.ns, w.ne,
                                                                                weight, k, n_src, grad_src[t]);
        else
            knn_wsum_bwd_kernel<1><<<agg_grid(n_src * dim), 256, 0, st>>>(grad_out[t], dim, w.perm, w.ns, w.ne, weight,
                                                                          k, n_src, grad_src[t]);
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_knn_weighted_sum_weight_grad(const float *grad_out, const float *src, int64_t n_src, int64_t dim,
                                                const int64_t *idx, int64_t n_query, int32_t k, int32_t accumulate,
                                                float *grad_weight, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_src < 0 || dim < 0 || n_query < 0 || k < 0, GDL_ERR_INVALID);
    const int64_t m = n_query * k;
    if (m == 0) return GDL_OK;
    GDL_RETURN_IF(!idx || !grad_weight || (dim > 0 && (!grad_out || (n_src > 0 && !src))), GDL_ERR_INVALID);
    int64_t blocks = (m + 7) / 8;
    const int64_t cap = (int64_t)kSmCount * 8;
    knn_wsum_wgrad_kernel<<<(unsigned)(blocks > cap ? cap : blocks), 256, 0, st>>>(grad_out, src, n_src, dim, idx, m,
                                                                                  k, accumulate, grad_weight);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
