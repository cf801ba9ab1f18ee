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
// by broadcast; a thread only touches its (local-memory) heap when a distance beats its
// current (k_eff+1)-th best, held in a register. Distances use the reference's rounding.
// Small query sets split each cloud's sources over `split` CTAs; knn_merge_kernel merges
// their sorted partial lists.
#include "common.cuh"
#include "radix.cuh"

namespace gdl {

constexpr int kKnnThreads = 128;
constexpr int kKnnChunk = 1024;
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

// ---------------------------------------------------------------- per-thread lists in shared memory
// Every per-thread array lives in shared memory as [slot][thread] with a stride of
// kKnnThreads words, so the 32 lanes of a warp always hit 32 different banks whatever slot
// each of them touches.
constexpr int kKnnGroup = 8;  // sources per distance group (one vote, one group minimum)
constexpr int kKnnBuf = 16;   // buffered candidates per thread; a flush starts at > kKnnBuf - kKnnGroup

__device__ __forceinline__ void sheap_sift_down(float *d, int *id, int n, int at) {
    for (;;) {
        const int l = 2 * at + 1, r = l + 1;
        int g = at;
        float gd = d[at * kKnnThreads];
        if (l < n) {
            const float ld = d[l * kKnnThreads];
            if (ld > gd) { g = l; gd = ld; }
        }
        if (r < n) {
            const float rd = d[r * kKnnThreads];
            if (rd > gd) { g = r; gd = rd; }
        }
        if (g == at) return;
        const float td = d[at * kKnnThreads];
        const int ti = id[at * kKnnThreads];
        d[at * kKnnThreads] = gd;
        id[at * kKnnThreads] = id[g * kKnnThreads];
        d[g * kKnnThreads] = td;
        id[g * kKnnThreads] = ti;
        at = g;
    }
}

// Max-heap of the L smallest distances seen (filled unsorted, heapified when full, root
// replaced by strictly smaller distances). `thr` mirrors the root once full (+inf before).
__device__ __forceinline__ void sheap_add(float *d, int *id, int &cnt, int L, float &thr, float dist, int idx) {
    if (cnt < L) {
        d[cnt * kKnnThreads] = dist;
        id[cnt * kKnnThreads] = idx;
        if (++cnt == L) {
            for (int j = L / 2 - 1; j >= 0; --j) sheap_sift_down(d, id, L, j);
            thr = d[0];
        }
    } else {
        d[0] = dist;
        id[0] = idx;
        sheap_sift_down(d, id, L, 0);
        thr = d[0];
    }
}

// ascending by distance, into thread-local arrays
__device__ __forceinline__ void sheap_sorted(const float *d, const int *id, int cnt, float *od, int *oi) {
    for (int a = 0; a < cnt; ++a) {
        const float kd = d[a * kKnnThreads];
        const int ki = id[a * kKnnThreads];
        int b = a - 1;
        while (b >= 0 && od[b] > kd) {
            od[b + 1] = od[b];
            oi[b + 1] = oi[b];
            --b;
        }
        od[b + 1] = kd;
        oi[b + 1] = ki;
    }
}

__device__ __forceinline__ bool top_has_tie(const float *d, int cnt) {
    for (int a = 1; a < cnt; ++a)
        if (d[a] == d[a - 1]) return true;
    return false;
}

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

// ---------------------------------------------------------------- fast path
template <int KB>
struct KnnSmem {
    float sx[kKnnChunk], sy[kKnnChunk], sz[kKnnChunk];  // staged sources, SoA
    float hd[(KB + 1) * kKnnThreads];                    // heap of the k_eff + 1 best
    int hi[(KB + 1) * kKnnThreads];
    float bd[kKnnBuf * kKnnThreads];  // candidates that beat the threshold, not yet in the heap
    int bi[kKnnBuf * kKnnThreads];
    int nonfinite;                    // a staged source has a NaN/inf coordinate
};

template <int KB>
constexpr size_t knn_smem_bytes() {
    return sizeof(KnnSmem<KB>);
}

// Fast path: kKnnThreads queries of one cloud per CTA (one per thread, coordinates in
// registers); the cloud's sources (or this CTA's share of them, `split` > 1) are staged in
// shared memory in kKnnChunk-point chunks and read by broadcast, eight at a time. A thread
// keeps its k_eff + 1 best in a shared-memory max-heap; distances below the heap root go
// to a per-thread buffer first, and the warp drains all its buffers together once a vote
// finds one nearly full -- so heap work is paid per lane, not per union of lanes. Queries
// whose final list holds equal distances, or that met a non-finite coordinate, are handed
// to knn_exact_kernel.
template <int KB>
__global__ void __launch_bounds__(kKnnThreads) knn_fast_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, int split, const int32_t *__restrict__ tile_base,
    int64_t *__restrict__ out_idx, float *__restrict__ out_dist, float *__restrict__ part_d,
    int32_t *__restrict__ part_i, int32_t *__restrict__ part_cnt, int32_t *__restrict__ flag_list,
    int32_t *__restrict__ flag_count) {
    extern __shared__ __align__(16) unsigned char knn_smem_raw[];
    KnnSmem<KB> &S = *reinterpret_cast<KnnSmem<KB> *>(knn_smem_raw);
    const int t = blockIdx.x;
    const int qt = t / split, sp = t - (t / split) * split;
    if (qt >= tile_base[B]) return;  // uniform over the CTA
    const int b = find_segment(tile_base, B, qt);
    const int tid = threadIdx.x;
    const int64_t q = ptr_q[b] + (int64_t)(qt - tile_base[b]) * kKnnThreads + tid;
    const bool valid = q < ptr_q[b + 1];
    const int64_t s0 = ptr_s[b], len = ptr_s[b + 1] - ptr_s[b];
    const int64_t ss = s0 + len * sp / split, se = s0 + len * (sp + 1) / split;
    const int ke = k < 64 ? k : 64;
    const int L = ke + 1;
    float qx = 0.0f, qy = 0.0f, qz = 0.0f;
    bool nonfinite = false;
    if (valid) {
        qx = query[3 * q];
        qy = query[3 * q + 1];
        qz = query[3 * q + 2];
        nonfinite = !(isfinite(qx) && isfinite(qy) && isfinite(qz));
    }
    if (tid == 0) S.nonfinite = 0;
    const uint64_t QX = pack2(qx, qx), QY = pack2(qy, qy), QZ = pack2(qz, qz);
    float *hd = S.hd + tid;
    int *hi = S.hi + tid;
    float *bd = S.bd + tid;
    int *bi = S.bi + tid;
    int cnt = 0, nb = 0;
    // invalid threads run the loop (they vote) but never accept a candidate
    float thr = valid ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    const float kPadNaN = __int_as_float(0x7fffffff);
    for (int64_t c0 = ss; c0 < se; c0 += kKnnChunk) {
        const int m = (int)(se - c0 < kKnnChunk ? se - c0 : kKnnChunk);
        const int mg = (m + kKnnGroup - 1) & ~(kKnnGroup - 1);
        __syncthreads();
        bool bad = false;
        for (int j = tid; j < mg; j += kKnnThreads) {
            float x = kPadNaN, y = kPadNaN, z = kPadNaN;  // padding: NaN never passes `<`
            if (j < m) {
                const float *p = source + 3 * (c0 + j);
                x = p[0];
                y = p[1];
                z = p[2];
                bad |= !(isfinite(x) && isfinite(y) && isfinite(z));
            }
            S.sx[j] = x;
            S.sy[j] = y;
            S.sz[j] = z;
        }
        if (bad) S.nonfinite = 1;
        __syncthreads();
        for (int j = 0; j < mg; j += kKnnGroup) {
            if (__any_sync(0xffffffffu, nb > kKnnBuf - kKnnGroup)) {
                for (int e = 0; e < nb; ++e) {
                    const float d = bd[e * kKnnThreads];
                    if (d < thr) sheap_add(hd, hi, cnt, L, thr, d, bi[e * kKnnThreads]);
                }
                nb = 0;
            }
            const float4 x0 = *reinterpret_cast<const float4 *>(S.sx + j);
            const float4 x1 = *reinterpret_cast<const float4 *>(S.sx + j + 4);
            const float4 y0 = *reinterpret_cast<const float4 *>(S.sy + j);
            const float4 y1 = *reinterpret_cast<const float4 *>(S.sy + j + 4);
            const float4 z0 = *reinterpret_cast<const float4 *>(S.sz + j);
            const float4 z1 = *reinterpret_cast<const float4 *>(S.sz + j + 4);
            float d[kKnnGroup];
            unpack2(dist2_x2(QX, QY, QZ, pack2(x0.x, x0.y), pack2(y0.x, y0.y), pack2(z0.x, z0.y)), d[0], d[1]);
            unpack2(dist2_x2(QX, QY, QZ, pack2(x0.z, x0.w), pack2(y0.z, y0.w), pack2(z0.z, z0.w)), d[2], d[3]);
            unpack2(dist2_x2(QX, QY, QZ, pack2(x1.x, x1.y), pack2(y1.x, y1.y), pack2(z1.x, z1.y)), d[4], d[5]);
            unpack2(dist2_x2(QX, QY, QZ, pack2(x1.z, x1.w), pack2(y1.z, y1.w), pack2(z1.z, z1.w)), d[6], d[7]);
            const float mn = fminf(fminf(fminf(d[0], d[1]), fminf(d[2], d[3])), fminf(fminf(d[4], d[5]), fminf(d[6], d[7])));
            if (mn < thr) {
                const int base = (int)(c0 + j);  // global index of d[0]
#pragma unroll
                for (int e = 0; e < kKnnGroup; ++e) {
                    if (d[e] < thr) {
                        bd[nb * kKnnThreads] = d[e];
                        bi[nb * kKnnThreads] = base + e;
                        ++nb;
                    }
                }
            }
        }
    }
    for (int e = 0; e < nb; ++e) {
        const float d = bd[e * kKnnThreads];
        if (d < thr) sheap_add(hd, hi, cnt, L, thr, d, bi[e * kKnnThreads]);
    }
    __syncthreads();  // S.nonfinite is complete
    nonfinite |= S.nonfinite != 0;
    if (!valid) return;
    float td[KB + 1];
    int ti[KB + 1];
    sheap_sorted(hd, hi, cnt, td, ti);
    if (split == 1) {
        if (nonfinite || top_has_tie(td, cnt)) {
            flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
            return;
        }
        write_row(out_idx + q * k, out_dist + q * k, k, cnt < ke ? cnt : ke, td, ti);
    } else {
        const int64_t slot = (q - ptr_q[0]) * split + sp;
        float *pd = part_d + slot * (KB + 1);
        int32_t *pi = part_i + slot * (KB + 1);
        for (int j = 0; j < cnt; ++j) {
            pd[j] = td[j];
            pi[j] = ti[j];
        }
        part_cnt[slot] = nonfinite ? -1 : cnt;
    }
}

// Merges the `split` ascending partial lists of a query (two-pointer merges, first L kept).
template <int KB>
__global__ void __launch_bounds__(kKnnThreads) knn_merge_kernel(
    const int64_t *__restrict__ ptr_q, int32_t B, int k, int split, const float *__restrict__ part_d,
    const int32_t *__restrict__ part_i, const int32_t *__restrict__ part_cnt, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count) {
    const int64_t q = ptr_q[0] + (int64_t)blockIdx.x * kKnnThreads + threadIdx.x;
    if (q >= ptr_q[B]) return;
    const int ke = k < 64 ? k : 64;
    const int L = ke + 1;
    float ad[KB + 1], bdv[KB + 1];
    int ai[KB + 1], biv[KB + 1];
    float *cd = ad, *nd = bdv;
    int *ci = ai, *ni = biv;
    int cnt = 0;
    const int64_t base = (q - ptr_q[0]) * split;
    for (int sp = 0; sp < split; ++sp) {
        const int c = part_cnt[base + sp];
        if (c < 0) {  // a partial scan met a non-finite coordinate
            flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
            return;
        }
        const float *pd = part_d + (base + sp) * (KB + 1);
        const int32_t *pi = part_i + (base + sp) * (KB + 1);
        int a = 0, bb = 0, o = 0;
        while (o < L && (a < cnt || bb < c)) {
            const bool take_b = bb < c && (a >= cnt || pd[bb] < cd[a]);
            if (take_b) {
                nd[o] = pd[bb];
                ni[o] = pi[bb];
                ++bb;
            } else {
                nd[o] = cd[a];
                ni[o] = ci[a];
                ++a;
            }
            ++o;
        }
        cnt = o;
        float *tdp = cd; cd = nd; nd = tdp;
        int *tip = ci; ci = ni; ni = tip;
    }
    if (top_has_tie(cd, cnt)) {
        flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    write_row(out_idx + q * k, out_dist + q * k, k, cnt < ke ? cnt : ke, cd, ci);
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

// The reference kernel's heap, replayed exactly for flagged queries: one warp per query.
// The lanes compute 32 distances at a time; a candidate the heap would reject at the start
// of the batch (full and d >= root -- the root never grows) is rejected at its turn too, so
// only the ballot of the others is walked, in source order, and every lane applies the
// same MinKHeap::add to its own copy of the heap.
__global__ void __launch_bounds__(kKnnThreads) knn_exact_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, const int32_t *__restrict__ flag_list,
    const int32_t *__restrict__ flag_count, int64_t *__restrict__ out_idx, float *__restrict__ out_dist) {
    const int nflag = *flag_count;
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kKnnThreads / 32);
    for (int f = blockIdx.x * (kKnnThreads / 32) + (threadIdx.x >> 5); f < nflag; f += warps) {
        const int64_t q = flag_list[f];
        const int b = find_cloud(ptr_q, B, q);
        const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
        MinKHeap h;
        h.init(knn_bucket(k));
        for (int64_t c0 = ptr_s[b]; c0 < ptr_s[b + 1]; c0 += 32) {
            const int64_t s = c0 + lane;
            const bool in = s < ptr_s[b + 1];
            float d = 0.0f;
            if (in) d = dist2(qx, qy, qz, source[3 * s], source[3 * s + 1], source[3 * s + 2]);
            const bool full = h.count >= h.cap;
            unsigned live = __ballot_sync(0xffffffffu, in && !(full && d >= h.d[0]));
            while (live) {
                const int l = __ffs(live) - 1;
                live &= live - 1;
                h.add(__shfl_sync(0xffffffffu, d, l), (int)(c0 + l));
            }
        }
        h.sort_ascending();
        if (lane == 0) write_row(out_idx + q * k, out_dist + q * k, k, h.count < k ? h.count : k, h.d, h.i);
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
    const int64_t by_src = max_src / 256;
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
    const size_t smem = knn_smem_bytes<KB>();
    cudaFuncSetAttribute(knn_fast_kernel<KB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    knn_fast_kernel<KB><<<(unsigned)grid, kKnnThreads, smem, st>>>(query, source, ptr_q, ptr_s, B, k, split,
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
