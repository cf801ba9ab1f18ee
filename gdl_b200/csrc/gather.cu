// gather.cu -- row gather out[i] = src[idx[i]] (sm_100a).
//
// The message materialisation that feeds a segment reduce over a KNN graph: the reference's
// pooling layer builds msg = feats[knn_idx] with torch indexing (nn/modules/
// equivariant_pool.py:277-300) before reducing over each query's k slots. Rows are moved
// as 16-byte vectors when the row size and both base addresses allow it (every bf16 row of
// 8k channels, every f32 row of 4k), otherwise as 4-byte words; consecutive threads cover
// consecutive vectors of a row, so reads of one source row and writes of one output row are
// coalesced. Indices outside [0, n_src) produce a zero row.
#include "common.cuh"

namespace gdl {

template <typename V>
__global__ void __launch_bounds__(256) gather_rows_kernel(const V *__restrict__ src, int64_t n_src,
                                                          int64_t vec_per_row, const int64_t *__restrict__ idx,
                                                          int64_t n_idx, V *__restrict__ out) {
    const int64_t total = n_idx * vec_per_row;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = t / vec_per_row, v = t - row * vec_per_row;
        const int64_t s = idx[row];
        V val;
        if (s >= 0 && s < n_src) val = src[s * vec_per_row + v];
        else memset(&val, 0, sizeof(V));
        out[t] = val;
    }
}

}  // namespace gdl

using namespace gdl;

extern "C" int gdl_gather_rows(const void *src, int64_t n_src, int64_t row_bytes, const int64_t *idx, int64_t n_idx,
                               void *out, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(n_src < 0 || n_idx < 0 || row_bytes < 0, GDL_ERR_INVALID);
    if (n_idx == 0 || row_bytes == 0) return GDL_OK;
    GDL_RETURN_IF(!idx || !out || (n_src > 0 && !src), GDL_ERR_INVALID);
    GDL_RETURN_IF(row_bytes % 4 != 0, GDL_ERR_INVALID);
    const bool v16 = row_bytes % 16 == 0 && ((uintptr_t)src % 16 == 0) && ((uintptr_t)out % 16 == 0);
    const int64_t vec = v16 ? 16 : 4;
    const int64_t per_row = row_bytes / vec;
    const int64_t total = n_idx * per_row;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = (int64_t)kSmCount * 8;  // 8 resident 256-thread CTAs per SM, grid-stride beyond
    if (blocks > cap) blocks = cap;
    if (v16)
        gather_rows_kernel<uint4><<<(unsigned)blocks, 256, 0, st>>>((const uint4 *)src, n_src, per_row, idx, n_idx,
                                                                    (uint4 *)out);
    else
        gather_rows_kernel<uint32_t><<<(unsigned)blocks, 256, 0, st>>>((const uint32_t *)src, n_src, per_row, idx,
                                                                       n_idx, (uint32_t *)out);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
