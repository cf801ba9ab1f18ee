// knn.cu -- brute-force k-nearest neighbours for packed clouds (sm_100a).
//
// Reference: geoembodied/csrc/knn_kernel.cu:113-291 (knn_kernel<MAX_K> + knn_cuda).
//
// What must match: the reference keeps a MinK<KB> heap (KB = 4/8/16/32/64 >= k) while
// scanning its cloud's sources in ascending index order, stable-sorts it and returns the
// first k. Whenever the k_eff + 1 smallest distances of a query (k_eff = min(k, 64)) are
// pairwise distinct, that output is simply "the k_eff nearest, ascending" -- independent of
// scan order or data structure (a heap that rejects d >= root keeps every value below its
// final root). So the fast path may scan in any order and split the scan: it keeps the
// k_eff + 1 smallest (distance, index) pairs per query, and a query whose list contains an
// equal pair is replayed by knn_exact_kernel, which runs the reference's heap verbatim.
//
// Fast path: 128 queries of one cloud per CTA (one per thread, coordinates in registers),
// the cloud's sources staged through shared memory as float4 in 2048-point chunks and read
// by broadcast; a thread only touches its (local-memory) list when a distance beats its
// current (k_eff+1)-th best, held in a register. Distances use the reference's rounding.
// Small query sets split each cloud's sources over `split` CTAs; knn_merge_kernel merges
// their sorted partial lists.
#include "common.cuh"
#include "radix.cuh"

namespace gdl {

constexpr int kKnnThreads = 128;
constexpr int kKnnChunk = 2048;
constexpr int kKnnMaxSplit = 32;

// query tiles per cloud -> exclusive prefix (one block)
__global__ void __launch_bounds__(kScanThreads) knn_tiles_kernel(const int64_t *__restrict__ ptr_q, int32_t B,
                                                                 int32_t *__restrict__ tile_base) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t total;
    int32_t carry = 0;
    for (int32_t b0 = 0; b0 < B; b0 += kScanThreads) {
        const int32_t b = b0 + threadIdx.x;
        int32_t t = 0;
        if (b < B) t = (int32_t)((ptr_q[b + 1] - ptr_q[b] + kKnnThreads - 1) / kKnnThreads);
        int32_t off = block_exclusive_scan<int32_t>(t, warp_sums, &total) + carry;
        if (b < B) tile_base[b] = off;
        carry += total;
    }
    if (threadIdx.x == 0) tile_base[B] = carry;
}

// The L smallest (distance, index) pairs seen so far, ascending; ties keep arrival order.
template <int CAP>
struct TopList {
    float d[CAP];
    int i[CAP];
    int cnt;
    int L;
    float thr;  // distance a candidate must beat (inf until the list is full)

    __device__ __forceinline__ void init(int l) {
        cnt = 0;
        L = l;
        thr = __int_as_float(0x7f800000);
    }
    __device__ __forceinline__ void insert(float dist, int idx) {
        int p = cnt < L ? cnt : L - 1;
        while (p > 0 && d[p - 1] > dist) {
            d[p] = d[p - 1];
            i[p] = i[p - 1];
            --p;
        }
        d[p] = dist;
        i[p] = idx;
        if (cnt < L) ++cnt;
        if (cnt == L) thr = d[L - 1];
    }
    __device__ __forceinline__ void offer(float dist, int idx) {
        if (dist < thr) insert(dist, idx);
    }
    __device__ __forceinline__ bool has_tie() const {
        for (int a = 1; a < cnt; ++a)
            if (d[a] == d[a - 1]) return true;
        return false;
    }
};

__device__ __forceinline__ void write_row(int64_t *__restrict__ oi, float *__restrict__ od, int k, int valid,
                                          const float *d, const int *i) {
    for (int j = 0; j < k; ++j) {
        if (j < valid) {
            oi[j] = i[j];
            od[j] = d[j];
        } else {
            oi[j] = -1;
            od[j] = 1e30f;
        }
    }
}

template <int KB>
__global__ void __launch_bounds__(kKnnThreads) knn_fast_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, int split, const int32_t *__restrict__ tile_base,
    int64_t *__restrict__ out_idx, float *__restrict__ out_dist, float *__restrict__ part_d,
    int32_t *__restrict__ part_i, int32_t *__restrict__ part_cnt, int32_t *__restrict__ flag_list,
    int32_t *__restrict__ flag_count) {
    __shared__ float4 sh[kKnnChunk];
    const int t = blockIdx.x;
    const int qt = t / split, sp = t - (t / split) * split;
    if (qt >= tile_base[B]) return;
    const int b = find_segment(tile_base, B, qt);
    const int64_t q = ptr_q[b] + (int64_t)(qt - tile_base[b]) * kKnnThreads + threadIdx.x;
    const bool valid = q < ptr_q[b + 1];
    const int64_t s0 = ptr_s[b], len = ptr_s[b + 1] - ptr_s[b];
    const int64_t ss = s0 + len * sp / split, se = s0 + len * (sp + 1) / split;
    const int ke = k < 64 ? k : 64;
    float qx = 0.0f, qy = 0.0f, qz = 0.0f;
    if (valid) {
        qx = query[3 * q];
        qy = query[3 * q + 1];
        qz = query[3 * q + 2];
    }
    TopList<KB + 1> tl;
    tl.init(ke + 1);
    for (int64_t c0 = ss; c0 < se; c0 += kKnnChunk) {
        const int m = (int)(se - c0 < kKnnChunk ? se - c0 : kKnnChunk);
        __syncthreads();
        for (int j = threadIdx.x; j < m; j += kKnnThreads) {
            const float *p = source + 3 * (c0 + j);
            sh[j] = make_float4(p[0], p[1], p[2], 0.0f);
        }
        __syncthreads();
        if (valid) {
#pragma unroll 4
            for (int j = 0; j < m; ++j) {
                const float4 s = sh[j];
                const float d = dist2(qx, qy, qz, s.x, s.y, s.z);
                if (d < tl.thr) tl.insert(d, (int)(c0 + j));
            }
        }
    }
    if (!valid) return;
    if (split == 1) {
        if (tl.has_tie()) {
            flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
            return;
        }
        write_row(out_idx + q * k, out_dist + q * k, k, tl.cnt < ke ? tl.cnt : ke, tl.d, tl.i);
    } else {
        const int64_t slot = (q - ptr_q[0]) * split + sp;
        float *pd = part_d + slot * (KB + 1);
        int32_t *pi = part_i + slot * (KB + 1);
        for (int j = 0; j < tl.cnt; ++j) {
            pd[j] = tl.d[j];
            pi[j] = tl.i[j];
        }
        part_cnt[slot] = tl.cnt;
    }
}

template <int KB>
__global__ void __launch_bounds__(kKnnThreads) knn_merge_kernel(
    const int64_t *__restrict__ ptr_q, int32_t B, int k, int split, const float *__restrict__ part_d,
    const int32_t *__restrict__ part_i, const int32_t *__restrict__ part_cnt, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count) {
    const int64_t q = ptr_q[0] + (int64_t)blockIdx.x * kKnnThreads + threadIdx.x;
    if (q >= ptr_q[B]) return;
    const int ke = k < 64 ? k : 64;
    TopList<KB + 1> tl;
    tl.init(ke + 1);
    const int64_t base = (q - ptr_q[0]) * split;
    for (int sp = 0; sp < split; ++sp) {
        const int c = part_cnt[base + sp];
        const float *pd = part_d + (base + sp) * (KB + 1);
        const int32_t *pi = part_i + (base + sp) * (KB + 1);
        for (int j = 0; j < c; ++j) {
            const float d = pd[j];
            if (d >= tl.thr) break;  // partial lists are ascending
            tl.insert(d, pi[j]);
        }
    }
    if (tl.has_tie()) {
        flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    write_row(out_idx + q * k, out_dist + q * k, k, tl.cnt < ke ? tl.cnt : ke, tl.d, tl.i);
}

__device__ __forceinline__ int find_cloud(const int64_t *__restrict__ ptr, int B, int64_t q) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (ptr[mid] <= q) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// The reference kernel verbatim for queries with tied candidate distances.
__global__ void __launch_bounds__(kKnnThreads) knn_exact_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, const int32_t *__restrict__ flag_list,
    const int32_t *__restrict__ flag_count, int64_t *__restrict__ out_idx, float *__restrict__ out_dist) {
    const int nflag = *flag_count;
    for (int f = blockIdx.x * kKnnThreads + threadIdx.x; f < nflag; f += gridDim.x * kKnnThreads) {
        const int64_t q = flag_list[f];
        const int b = find_cloud(ptr_q, B, q);
        const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
        MinKHeap h;
        h.init(knn_bucket(k));
        for (int64_t s = ptr_s[b]; s < ptr_s[b + 1]; ++s)
            h.add(dist2(qx, qy, qz, source[3 * s], source[3 * s + 1], source[3 * s + 2]), (int)s);
        h.sort_ascending();
        write_row(out_idx + q * k, out_dist + q * k, k, h.count < k ? h.count : k, h.d, h.i);
    }
}

// queries outside [ptr_q[0], ptr_q[B]) belong to no cloud: padding only
__global__ void knn_pad_kernel(const int64_t *__restrict__ ptr_q, int32_t B, int64_t n_q, int k,
                               int64_t *__restrict__ out_idx, float *__restrict__ out_dist) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_q * k) return;
    const int64_t q = i / k;
    if (q < ptr_q[0] || q >= ptr_q[B]) {
        out_idx[i] = -1;
        out_dist[i] = 1e30f;
    }
}

static int knn_split(int64_t n_q, int32_t B, int64_t max_src) {
    const int64_t tiles = n_q / kKnnThreads + B;
    int64_t split = (4 * kSmCount + tiles - 1) / (tiles > 0 ? tiles : 1);
    const int64_t by_src = max_src / 512;
    if (split > by_src) split = by_src;
    if (split > kKnnMaxSplit) split = kKnnMaxSplit;
    if (split < 1) split = 1;
    return (int)split;
}

struct KnnWs {
    int32_t *tile_base, *flag_count, *flag_list, *part_i, *part_cnt;
    float *part_d;
};

static size_t knn_ws(int64_t n_q, int32_t B, int32_t k, int64_t max_src, char *base, KnnWs *w) {
    const int split = knn_split(n_q, B, max_src);
    const int kb = knn_bucket(k);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + off : nullptr;
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t nq = n_q > 0 ? n_q : 1;
    KnnWs t;
    t.tile_base = (int32_t *)take(sizeof(int32_t) * (B + 1));
    t.flag_count = (int32_t *)take(sizeof(int32_t));
    t.flag_list = (int32_t *)take(sizeof(int32_t) * nq);
    const int64_t np = split > 1 ? nq * split : 1;
    t.part_cnt = (int32_t *)take(sizeof(int32_t) * np);
    t.part_d = (float *)take(sizeof(float) * np * (kb + 1));
    t.part_i = (int32_t *)take(sizeof(int32_t) * np * (kb + 1));
    if (w) *w = t;
    return off;
}

template <int KB>
static void knn_launch(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
                       int32_t B, int64_t n_q, int k, int split, const KnnWs &w, int64_t *oi, float *od,
                       cudaStream_t st) {
    const int64_t grid = (n_q / kKnnThreads + B) * split;
    knn_fast_kernel<KB><<<(unsigned)grid, kKnnThreads, 0, st>>>(query, source, ptr_q, ptr_s, B, k, split,
                                                               w.tile_base, oi, od, w.part_d, w.part_i, w.part_cnt,
                                                               w.flag_list, w.flag_count);
    if (split > 1)
        knn_merge_kernel<KB><<<(unsigned)((n_q + kKnnThreads - 1) / kKnnThreads), kKnnThreads, 0, st>>>(
            ptr_q, B, k, split, w.part_d, w.part_i, w.part_cnt, oi, od, w.flag_list, w.flag_count);
}

}  // namespace gdl

using namespace gdl;

extern "C" size_t gdl_knn_workspace_size(int64_t n_query, int32_t num_clouds, int32_t k, int64_t max_cloud_sources) {
    return knn_ws(n_query, num_clouds, k, max_cloud_sources, nullptr, nullptr);
}

extern "C" int gdl_knn(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
                       int32_t num_clouds, int64_t n_query, int32_t k, int64_t max_cloud_sources, int64_t *out_idx,
                       float *out_dist, void *workspace, size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || n_query < 0 || max_cloud_sources < 0, GDL_ERR_INVALID);
    if (n_query == 0 || k <= 0) return GDL_OK;
    GDL_RETURN_IF(!query || !ptr_q || !ptr_s || !out_idx || !out_dist, GDL_ERR_INVALID);
    GDL_RETURN_IF(n_query >= INT32_MAX || max_cloud_sources >= INT32_MAX, GDL_ERR_OVERFLOW);
    GDL_RETURN_IF(n_query * (int64_t)k >= ((int64_t)1 << 40), GDL_ERR_OVERFLOW);
    const size_t need = gdl_knn_workspace_size(n_query, num_clouds, k, max_cloud_sources);
    GDL_RETURN_IF(!workspace || workspace_bytes < need, GDL_ERR_WORKSPACE);
    KnnWs w;
    knn_ws(n_query, num_clouds, k, max_cloud_sources, (char *)workspace, &w);
    const unsigned padg = (unsigned)((n_query * k + 255) / 256);
    if (num_clouds == 0) {  // every query is outside all clouds
        GDL_CUDA_TRY(cudaMemsetAsync(out_idx, 0xff, sizeof(int64_t) * n_query * k, st));
        knn_pad_kernel<<<padg, 256, 0, st>>>(ptr_q, 0, n_query, k, out_idx, out_dist);
        return cudaGetLastError() == cudaSuccess ? GDL_OK : GDL_ERR_CUDA;
    }
    GDL_CUDA_TRY(cudaMemsetAsync(w.flag_count, 0, sizeof(int32_t), st));
    knn_tiles_kernel<<<1, kScanThreads, 0, st>>>(ptr_q, num_clouds, w.tile_base);
    knn_pad_kernel<<<padg, 256, 0, st>>>(ptr_q, num_clouds, n_query, k, out_idx, out_dist);
    const int split = knn_split(n_query, num_clouds, max_cloud_sources);
    switch (knn_bucket(k)) {
    case 4: knn_launch<4>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 8: knn_launch<8>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 16: knn_launch<16>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 32: knn_launch<32>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    default: knn_launch<64>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    }
    knn_exact_kernel<<<kSmCount, kKnnThreads, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.flag_list,
                                                       w.flag_count, out_idx, out_dist);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
