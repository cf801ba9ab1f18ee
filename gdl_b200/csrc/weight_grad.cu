// weight_grad.cu -- weight gradients of the per-row linear maps around SE3Conv's fused message
// kernels: the node projections (nn.Linear weights W [M, N] applied to [rows, N, sub] features,
// geoembodied/nn/modules/se3_conv.py:343-413) and the radial MLP's two nn.Linear layers
// (se3_conv.py:266-268). Their gradients contract over the rows (nodes or edges, up to hundreds
// of thousands) into an output of at most a few hundred x a few hundred:
//     C[m, n] = sum_r sum_j A[r, m, j] * B[r, n, j]
// A GEMM library tiles the output, so such shapes leave it a handful of tiles and a long K loop
// (a split-K of tens of CTAs). Here the rows are split into a fixed number of slices sized to
// fill the 148 SMs; each CTA folds one slice into one 64 x 64 tile of C (256 threads x 4 x 4
// accumulators; the slice's rows staged in shared memory with the sub components transposed so
// that every accumulate step reads two float4, the next stage's loads held in registers while the
// current one is folded), writes its partial tile, and a second launch adds the partials in a
// fixed order -- the result does not depend on scheduling.
#include "common.cuh"

namespace gdl {
namespace {

constexpr int kWgTile = 64;
constexpr int kWgRows = 8;  // slice lengths are multiples of this
constexpr int kWgThreads = 256;
constexpr int kWgTargetCtas = 3 * kSmCount;
constexpr int64_t kWgMinRowsPerSlice = 32;

struct WgPlan {
    int tiles_m, tiles_n;
    int64_t slices, rows_per_slice;
};

WgPlan wg_plan(int64_t rows, int M, int N) {
    WgPlan p;
    p.tiles_m = (M + kWgTile - 1) / kWgTile;
    p.tiles_n = (N + kWgTile - 1) / kWgTile;
    const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
    int64_t s = (kWgTargetCtas + tiles - 1) / tiles;
    const int64_t by_rows = (rows + kWgMinRowsPerSlice - 1) / kWgMinRowsPerSlice;
    s = s < by_rows ? s : by_rows;
    s = s < 1 ? 1 : s;
    int64_t per = (rows + s - 1) / s;
    per = (per + kWgRows - 1) / kWgRows * kWgRows;
    p.rows_per_slice = per < kWgRows ? kWgRows : per;
    p.slices = rows > 0 ? (rows + p.rows_per_slice - 1) / p.rows_per_slice : 0;
    return p;
}

// rows staged per step (32 k-steps for scalars, 24 / 40 for vectors / type-2) and the elements of
// one matrix each thread carries from global memory into a stage
template <int SUB>
struct WgStage {
    static constexpr int rows = SUB == 1 ? 32 : 8;
    static constexpr int elems = rows * kWgTile * SUB / kWgThreads;
};

template <int SUB>
__device__ __forceinline__ void wg_fetch(const float *__restrict__ X, int64_t ld, int c0, int cw, int64_t rb,
                                         int64_t r1, float (&v)[WgStage<SUB>::elems]) {
#pragma unroll
    for (int e = 0; e < WgStage<SUB>::elems; ++e) {
        const int i = threadIdx.x + e * kWgThreads;
        const int rr = i / (kWgTile * SUB);
        const int x = i - rr * (kWgTile * SUB);
        const int64_t r = rb + rr;
        v[e] = (r < r1 && x < cw * SUB) ? X[r * ld + (int64_t)c0 * SUB + x] : 0.0f;
    }
}

// element x of staged row rr's slab [64 * SUB) is channel x / SUB, component x % SUB
template <int SUB>
__device__ __forceinline__ void wg_store(float (*S)[kWgTile], const float (&v)[WgStage<SUB>::elems]) {
#pragma unroll
    for (int e = 0; e < WgStage<SUB>::elems; ++e) {
        const int i = threadIdx.x + e * kWgThreads;
        const int rr = i / (kWgTile * SUB);
        const int x = i - rr * (kWgTile * SUB);
        const int ch = x / SUB, j = x - ch * SUB;
        S[rr * SUB + j][ch] = v[e];
    }
}

template <int SUB>
__global__ void __launch_bounds__(kWgThreads) wg_partial_kernel(const float *__restrict__ A, int64_t lda,
                                                                const float *__restrict__ B, int64_t ldb,
                                                                int64_t rows, int M, int N, int tiles_n,
                                                                int64_t rows_per_slice, float *__restrict__ part,
                                                                float *__restrict__ part_sum) {
    constexpr int RR = WgStage<SUB>::rows;
    constexpr int EL = WgStage<SUB>::elems;
    __shared__ __align__(16) float As[RR * SUB][kWgTile];
    __shared__ __align__(16) float Bs[RR * SUB][kWgTile];
    const int m0 = (int)(blockIdx.x / tiles_n) * kWgTile;
    const int n0 = (int)(blockIdx.x % tiles_n) * kWgTile;
    const int64_t slice = blockIdx.y;
    const int64_t r0 = slice * rows_per_slice;
    const int64_t r1 = rows < r0 + rows_per_slice ? rows : r0 + rows_per_slice;
    const int t = threadIdx.x, ty = t >> 4, tx = t & 15;
    const int mw = M - m0 < kWgTile ? M - m0 : kWgTile;
    const int nw = N - n0 < kWgTile ? N - n0 : kWgTile;
    const bool want_sum = part_sum != nullptr && n0 == 0 && tx == 0;
    float acc[4][4];
    float csum[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        csum[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    }
    float va[EL], vb[EL];
    wg_fetch<SUB>(A, lda, m0, mw, r0, r1, va);
    wg_fetch<SUB>(B, ldb, n0, nw, r0, r1, vb);
    for (int64_t rb = r0; rb < r1; rb += RR) {
        wg_store<SUB>(As, va);
        wg_store<SUB>(Bs, vb);
        __syncthreads();
        if (rb + RR < r1) {  // the next stage's loads are in flight while this one is folded
            wg_fetch<SUB>(A, lda, m0, mw, rb + RR, r1, va);
            wg_fetch<SUB>(B, ldb, n0, nw, rb + RR, r1, vb);
        }
#pragma unroll 4
        for (int k = 0; k < RR * SUB; ++k) {
            const float4 a = *reinterpret_cast<const float4 *>(&As[k][ty * 4]);
            const float4 b = *reinterpret_cast<const float4 *>(&Bs[k][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w};
            const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
            }
            if (want_sum) {
#pragma unroll
                for (int i = 0; i < 4; ++i) csum[i] += av[i];
            }
        }
        __syncthreads();
    }
    float *P = part + slice * (int64_t)M * N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N) P[(int64_t)m * N + n] = acc[i][j];
        }
        if (want_sum) part_sum[slice * M + m] = csum[i];
    }
}

// C[i] = sum over slices of the partial tiles; col_sum likewise. A block owns 32 consecutive outputs
// (one per lane, coalesced); warp w adds slices w, w + 8, ... and the eight warp sums are added in
// warp order, so the order of additions is fixed.
constexpr int kWgReduceWarps = 8;

__global__ void __launch_bounds__(32 * kWgReduceWarps) wg_reduce_kernel(const float *__restrict__ part,
                                                                       const float *__restrict__ part_sum,
                                                                       int64_t slices, int64_t MN, int M,
                                                                       float *__restrict__ C,
                                                                       float *__restrict__ col_sum) {
    __shared__ float acc[kWgReduceWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t total = MN + (col_sum ? M : 0);
    const int64_t i = (int64_t)blockIdx.x * 32 + lane;
    float s = 0.0f;
    if (i < total) {
        const bool tile = i < MN;
        const float *src = tile ? part + i : part_sum + (i - MN);
        const int64_t stride = tile ? MN : M;
#pragma unroll 4
        for (int64_t k = w; k < slices; k += kWgReduceWarps) s += src[k * stride];
    }
    acc[w][lane] = s;
    __syncthreads();
    if (w == 0 && i < total) {
        float t = acc[0][lane];
#pragma unroll
        for (int k = 1; k < kWgReduceWarps; ++k) t += acc[k][lane];
        if (i < MN)
            C[i] = t;
        else
            col_sum[i - MN] = t;
    }
}

size_t wg_bytes(const WgPlan &p, int M, int N) {
    const size_t part = (size_t)p.slices * M * N * sizeof(float);
    const size_t sums = (size_t)p.slices * M * sizeof(float);
    return ((part + 255) & ~(size_t)255) + ((sums + 255) & ~(size_t)255);
}

}  // namespace
}  // namespace gdl

using namespace gdl;

namespace gdl {
// column sums of A alone (a layer without output columns still has a bias gradient): one
// thread per column, rows in order, double accumulator (deterministic)
static __global__ void wg_colsum_kernel(const float *__restrict__ A, int64_t lda, int64_t rows, int32_t M,
                                        float *__restrict__ col_sum) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    double s = 0.0;
    for (int64_t r = 0; r < rows; ++r) s += (double)A[r * lda + m];
    col_sum[m] = (float)s;
}
}  // namespace gdl

extern "C" size_t gdl_weight_grad_workspace_size(int64_t rows, int32_t M, int32_t N, int32_t sub) {
    if (rows <= 0 || M <= 0 || N <= 0 || (sub != 1 && sub != 3 && sub != 5)) return 256;
    return wg_bytes(wg_plan(rows, M, N), M, N);
}

extern "C" int gdl_weight_grad(const float *A, int64_t lda, const float *B, int64_t ldb, int64_t rows, int32_t M,
                               int32_t N, int32_t sub, float *C, float *col_sum, void *workspace,
                               size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(rows < 0 || M < 0 || N < 0 || (sub != 1 && sub != 3 && sub != 5), GDL_ERR_INVALID);
    GDL_RETURN_IF(col_sum && sub != 1, GDL_ERR_INVALID);
    if (M == 0) return GDL_OK;
    if (N == 0) {  // no C entries; the column sums of A (a bias gradient) do not depend on N
        if (col_sum) {
            if (rows == 0) {
                GDL_CUDA_TRY(cudaMemsetAsync(col_sum, 0, (size_t)M * sizeof(float), st));
            } else {
                GDL_RETURN_IF(!A || lda < (int64_t)M, GDL_ERR_INVALID);
                wg_colsum_kernel<<<(unsigned)((M + 127) / 128), 128, 0, st>>>(A, lda, rows, M, col_sum);
                GDL_CUDA_TRY(cudaGetLastError());
            }
        }
        return GDL_OK;
    }
    GDL_RETURN_IF(!C, GDL_ERR_INVALID);
    if (rows == 0) {
        GDL_CUDA_TRY(cudaMemsetAsync(C, 0, (size_t)M * N * sizeof(float), st));
        if (col_sum) GDL_CUDA_TRY(cudaMemsetAsync(col_sum, 0, (size_t)M * sizeof(float), st));
        return GDL_OK;
    }
    GDL_RETURN_IF(!A || !B || lda < (int64_t)M * sub || ldb < (int64_t)N * sub, GDL_ERR_INVALID);
    const WgPlan p = wg_plan(rows, M, N);
    GDL_RETURN_IF(p.slices > 65535 || (int64_t)p.tiles_m * p.tiles_n > (1 << 30), GDL_ERR_OVERFLOW);
    GDL_RETURN_IF(!workspace || workspace_bytes < wg_bytes(p, M, N), GDL_ERR_WORKSPACE);
    float *part = (float *)workspace;
    const size_t part_bytes = ((size_t)p.slices * M * N * sizeof(float) + 255) & ~(size_t)255;
    float *part_sum = col_sum ? (float *)((char *)workspace + part_bytes) : nullptr;
    const dim3 grid((unsigned)(p.tiles_m * p.tiles_n), (unsigned)p.slices);
    const int tn = p.tiles_n;
    if (sub == 1)
        wg_partial_kernel<1><<<grid, kWgThreads, 0, st>>>(A, lda, B, ldb, rows, M, N, tn, p.rows_per_slice, part, part_sum);
    else if (sub == 3)
        wg_partial_kernel<3><<<grid, kWgThreads, 0, st>>>(A, lda, B, ldb, rows, M, N, tn, p.rows_per_slice, part, part_sum);
    else
        wg_partial_kernel<5><<<grid, kWgThreads, 0, st>>>(A, lda, B, ldb, rows, M, N, tn, p.rows_per_slice, part, part_sum);
    const int64_t total = (int64_t)M * N + (col_sum ? M : 0);
    wg_reduce_kernel<<<(unsigned)((total + 31) / 32), 32 * kWgReduceWarps, 0, st>>>(part, part_sum, p.slices,
                                                                                 (int64_t)M * N, M, C, col_sum);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
