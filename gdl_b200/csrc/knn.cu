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
#include "knn_grid.cuh"
#include "morton.cuh"
#include "radix.cuh"

namespace gdl {

constexpr int kKnnThreads = 128;
constexpr int kKnnChunk = 1024;
constexpr int kKnnMaxSplit = 32;

// query tiles per cloud -> exclusive prefix (one block)
__global__ void __launch_bounds__(kScanThreads) knn_tiles_kernel(const int64_t *__restrict__ ptr_q, int32_t B,
                                                                 int32_t tile, int32_t *__restrict__ tile_base) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t total;
    int32_t carry = 0;
    for (int32_t b0 = 0; b0 < B; b0 += kScanThreads) {
        const int32_t b = b0 + threadIdx.x;
        int32_t t = 0;
        if (b < B) t = (int32_t)((ptr_q[b + 1] - ptr_q[b] + tile - 1) / tile);
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
constexpr int kS = kKnnThreads;  // stride between the slots of one thread's list

// Entries are (distance, index bits) pairs. kheap_* is a max-heap of L entries over distance
// (filled unsorted, heapified when full, root replaced by strictly smaller distances); `thr`
// mirrors the root once full (+inf before). Sinks x from slot `at`.
template <int L>
__device__ __forceinline__ void kheap_sink(float2 *h, int at, float2 x) {
#pragma unroll
    for (int lvl = 0; lvl < 7; ++lvl) {  // 7 levels hold 127 >= L entries
        const int l = 2 * at + 1;
        if (l >= L) break;
        float2 c = h[l * kS];
        int g = l;
        if (l + 1 < L) {
            const float2 r = h[(l + 1) * kS];
            if (r.x > c.x) {
                c = r;
                g = l + 1;
            }
        }
        if (!(c.x > x.x)) break;
        h[at * kS] = c;
        at = g;
    }
    h[at * kS] = x;
}

template <int L>
__device__ __forceinline__ void kheap_add(float2 *h, int &cnt, float &thr, float2 x) {
    if (cnt < L) {
        h[cnt * kS] = x;
        if (++cnt == L) {
            for (int j = L / 2 - 1; j >= 0; --j) kheap_sink<L>(h, j, h[j * kS]);
            thr = h[0].x;
        }
    } else {
        kheap_sink<L>(h, 0, x);
        thr = h[0].x;
    }
}

// the heap's entries, ascending by distance, into thread-local arrays
__device__ __forceinline__ void kheap_sorted(const float2 *h, int cnt, float *od, int *oi) {
    for (int a = 0; a < cnt; ++a) {
        const float2 x = h[a * kS];
        int b = a - 1;
        while (b >= 0 && od[b] > x.x) {
            od[b + 1] = od[b];
            oi[b + 1] = oi[b];
            --b;
        }
        od[b + 1] = x.x;
        oi[b + 1] = __float_as_int(x.y);
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

// ---------------------------------------------------------------- fast path
template <int L>
struct KnnSmem {
    float sx[kKnnChunk], sy[kKnnChunk], sz[kKnnChunk];  // staged sources, SoA
    float2 heap[L * kKnnThreads];                        // the L best per thread
    float2 buf[kKnnBuf * kKnnThreads];  // candidates that beat the threshold, not yet in the heap
    int nonfinite;                      // a staged source has a NaN/inf coordinate
};

template <int L>
constexpr size_t knn_smem_bytes() {
    return sizeof(KnnSmem<L>);
}

// Fast path: kKnnThreads queries of one cloud per CTA (one per thread, coordinates in
// registers); the cloud's sources (or this CTA's share of them, `split` > 1) are staged in
// shared memory in kKnnChunk-point chunks and read by broadcast, eight at a time. A thread
// keeps its L best (L = KB + 1, KB = the reference's heap size >= k; L = 2 for k = 1) in a
// shared-memory max-heap, of which the first k_eff + 1 decide the output; distances below the
// heap root go
// to a per-thread buffer first, and the warp drains all its buffers together once a vote
// finds one nearly full -- so heap work is paid per lane, not per union of lanes. Queries
// whose final list holds equal distances, that met a non-finite coordinate or whose
// distances overflowed are handed to knn_exact_kernel.
template <int KB, int L>
__global__ void __launch_bounds__(kKnnThreads) knn_fast_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, int split, const int32_t *__restrict__ tile_base,
    int64_t *__restrict__ out_idx, float *__restrict__ out_dist, float *__restrict__ part_d,
    int32_t *__restrict__ part_i, int32_t *__restrict__ part_cnt, int32_t *__restrict__ flag_list,
    int32_t *__restrict__ flag_count, unsigned long long *__restrict__ pairs) {
    extern __shared__ __align__(16) unsigned char knn_smem_raw[];
    KnnSmem<L> &S = *reinterpret_cast<KnnSmem<L> *>(knn_smem_raw);
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
    float2 *heap = S.heap + tid;
    float2 *buf = S.buf + tid;
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
                    const float2 x = buf[e * kS];
                    if (x.x < thr) kheap_add<L>(heap, cnt, thr, x);
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
                // branch-free append: every candidate is written at slot nb, which advances only
                // when it is kept (nb <= kKnnBuf - kKnnGroup here, so slot nb stays in range)
                const int base = (int)(c0 + j);  // global index of d[0]
#pragma unroll
                for (int e = 0; e < kKnnGroup; ++e) {
                    buf[nb * kS] = make_float2(d[e], __int_as_float(base + e));
                    nb += d[e] < thr ? 1 : 0;
                }
            }
        }
    }
    for (int e = 0; e < nb; ++e) {
        const float2 x = buf[e * kS];
        if (x.x < thr) kheap_add<L>(heap, cnt, thr, x);
    }
    const int nvalid = __syncthreads_count(valid);  // also: S.nonfinite is complete
    if (tid == 0) atomicAdd(pairs, (unsigned long long)nvalid * (unsigned long long)(se - ss));
    nonfinite |= S.nonfinite != 0;
    if (!valid) return;
    float td[KB + 1];
    int ti[KB + 1];
    // Every finite distance enters a heap that is not full, so a short list means distances
    // that overflowed to +inf (or NaN): the reference's heap keeps those while it fills.
    nonfinite |= (int64_t)cnt < (se - ss < L ? se - ss : (int64_t)L);
    kheap_sorted(heap, cnt, td, ti);
    if (cnt > ke + 1) cnt = ke + 1;  // only the first k_eff + 1 decide the output
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

// Merges the `split` ascending partial lists of a query (at most k_eff + 1 entries each):
// one warp per query stages the lists in shared memory, lane s walks list s, and each step
// takes the smallest head (lowest list on equal heads) by a warp min-reduction.
constexpr int kMergeWarps = kKnnThreads / 32;

static size_t knn_merge_smem(int split, int k) {
    const int lm = (k < 64 ? k : 64) + 1;
    return sizeof(float2) * (size_t)kMergeWarps * (size_t)(split + 1) * lm;
}

__global__ void __launch_bounds__(kKnnThreads) knn_merge_kernel(
    const int64_t *__restrict__ ptr_q, int32_t B, int k, int split, int part_stride, const float *__restrict__ part_d,
    const int32_t *__restrict__ part_i, const int32_t *__restrict__ part_cnt, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count) {
    extern __shared__ float2 merge_smem[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t q = ptr_q[0] + (int64_t)blockIdx.x * kMergeWarps + w;
    if (q >= ptr_q[B]) return;  // uniform over the warp
    const int ke = k < 64 ? k : 64;
    const int lm = ke + 1;
    float2 *stage = merge_smem + (size_t)w * (split + 1) * lm;
    float2 *out = stage + (size_t)split * lm;
    const int64_t base = (q - ptr_q[0]) * split;
    int c = lane < split ? part_cnt[base + lane] : 0;
    if (__any_sync(0xffffffffu, c < 0)) {  // a partial scan met a non-finite coordinate
        if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    if (c > lm) c = lm;
    for (int sp = 0; sp < split; ++sp) {
        const int cs = __shfl_sync(0xffffffffu, c, sp);
        const float *pd = part_d + (base + sp) * part_stride;
        const int32_t *pi = part_i + (base + sp) * part_stride;
        for (int j = lane; j < cs; j += 32) stage[sp * lm + j] = make_float2(pd[j], __int_as_float(pi[j]));
    }
    __syncwarp();
    int p = 0;
    unsigned key = c > 0 ? __float_as_uint(stage[lane * lm].x) : 0xffffffffu;  // distances are >= 0
    int cnt = 0;
    for (; cnt < lm; ++cnt) {
        const unsigned m = __reduce_min_sync(0xffffffffu, key);
        if (m == 0xffffffffu) break;
        const int win = __ffs(__ballot_sync(0xffffffffu, key == m)) - 1;
        if (lane == win) {
            out[cnt] = stage[lane * lm + p];
            ++p;
            key = p < c ? __float_as_uint(stage[lane * lm + p].x) : 0xffffffffu;
        }
    }
    __syncwarp();
    bool tie = false;
    for (int j = 1 + lane; j < cnt; j += 32) tie |= out[j].x == out[j - 1].x;
    if (__any_sync(0xffffffffu, tie)) {
        if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    const int valid = cnt < ke ? cnt : ke;
    for (int j = lane; j < k; j += 32) {
        if (j < valid) {
            out_idx[q * k + j] = __float_as_int(out[j].y);
            out_dist[q * k + j] = out[j].x;
        } else {
            out_idx[q * k + j] = -1;
            out_dist[q * k + j] = 1e30f;
        }
    }
}

// ---------------------------------------------------------------- one warp per query (k >= 8, small clouds)
// For larger k the per-thread heaps above spend their time in lock-step sift-downs. Here a warp
// owns a query: its lanes test 32 sources at a time against the threshold (the (k_eff+1)-th best
// so far), and each accepted candidate is inserted into the warp's sorted list of the L = k_eff+1
// best, held as entry lane + 32 r in register set r of every lane: the insert position is one
// ballot/popc, the shift one shuffle. The CTA's 8 queries (warps) of one cloud share the sources
// staged in shared memory. Ties, non-finite coordinates and overflowed distances go to
// knn_exact_kernel as in the per-thread path.
constexpr int kWarpMinK = 8;
// Measured: faster than the per-thread heaps for k = 16 over 2048 sources (57 vs 73 us), slower
// for k = 32 over 8192 sources (1.59 vs 1.2 ms), where the serial insert chain dominates.
constexpr int64_t kWarpMaxSources = 4096;
constexpr int kWarpQ = 8;         // queries (warps) per CTA
constexpr int kWarpChunk = 2048;  // sources staged per pass

template <int NR>
__global__ void __launch_bounds__(kWarpQ * 32) knn_warp_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, const int32_t *__restrict__ tile_base,
    int64_t *__restrict__ out_idx, float *__restrict__ out_dist, int32_t *__restrict__ flag_list,
    int32_t *__restrict__ flag_count, unsigned long long *__restrict__ pairs) {
    __shared__ float4 sh[kWarpChunk];
    __shared__ int bad_s;
    const int t = blockIdx.x;
    if (t >= tile_base[B]) return;  // uniform over the CTA
    const int b = find_segment(tile_base, B, t);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t q = ptr_q[b] + (int64_t)(t - tile_base[b]) * kWarpQ + warp;
    const bool valid = q < ptr_q[b + 1];  // uniform over the warp
    const int64_t s0 = ptr_s[b], s1 = ptr_s[b + 1];
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
    const float kInf = __int_as_float(0x7f800000);
    float ed[NR];
    int ei[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        ed[r] = kInf;
        ei[r] = -1;
    }
    float thr = kInf;
    int cnt = 0;
    if (threadIdx.x == 0) bad_s = 0;
    for (int64_t c0 = s0; c0 < s1; c0 += kWarpChunk) {
        const int m = (int)(s1 - c0 < kWarpChunk ? s1 - c0 : kWarpChunk);
        __syncthreads();
        bool bad = false;
        for (int j = threadIdx.x; j < m; j += kWarpQ * 32) {
            const float *p = source + 3 * (c0 + j);
            const float x = p[0], y = p[1], z = p[2];
            bad |= !(isfinite(x) && isfinite(y) && isfinite(z));
            sh[j] = make_float4(x, y, z, 0.0f);
        }
        if (bad) bad_s = 1;
        __syncthreads();
        if (!valid) continue;  // uniform over the warp; the next pass's barrier is still reached
        for (int j0 = 0; j0 < m; j0 += 32) {
            const int j = j0 + lane;
            float d = kInf;
            if (j < m) {
                const float4 sp = sh[j];
                d = dist2(qx, qy, qz, sp.x, sp.y, sp.z);
            }
            unsigned acc = __ballot_sync(0xffffffffu, d < thr);
            while (acc) {
                const int l = __ffs(acc) - 1;
                acc &= acc - 1;
                const float dd = __shfl_sync(0xffffffffu, d, l);
                if (!(dd < thr)) continue;  // the threshold tightened since the ballot (uniform)
                warp_list_insert<NR>(ed, ei, dd, (int)(c0 + j0 + l), lane);
                ++cnt;
#pragma unroll
                for (int r = 0; r < NR; ++r)  // threshold = entry L - 1 (register set, lane uniform)
                    if ((L - 1) / 32 == r) thr = __shfl_sync(0xffffffffu, ed[r], (L - 1) & 31);
            }
        }
    }
    __syncthreads();  // bad_s is complete
    nonfinite |= bad_s != 0;
    if (!valid) return;
    if (lane == 0) atomicAdd(pairs, (unsigned long long)(s1 - s0));
    const int have = cnt < L ? cnt : L;
    // every finite distance enters a list that is not full: a short list means overflowed distances
    bool flag = nonfinite || (int64_t)have < (s1 - s0 < L ? s1 - s0 : (int64_t)L);
    if (!flag) {
        bool tie = false;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const float up = __shfl_up_sync(0xffffffffu, ed[r], 1);
            const float cross = r > 0 ? __shfl_sync(0xffffffffu, ed[r > 0 ? r - 1 : 0], 31) : 0.0f;
            const int i = lane + 32 * r;
            const float prev = lane > 0 ? up : cross;
            if (i >= 1 && i < have && prev == ed[r]) tie = true;
        }
        flag = __any_sync(0xffffffffu, tie);
    }
    if (flag) {
        if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    const int nv = have < ke ? have : ke;
    int64_t *oi = out_idx + q * k;
    float *od = out_dist + q * k;
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int i = lane + 32 * r;
        if (i < k) {
            oi[i] = i < nv ? (int64_t)ei[r] : -1;
            od[i] = i < nv ? ed[r] : 1e30f;
        }
    }
    for (int i = 32 * NR + lane; i < k; i += 32) {
        oi[i] = -1;
        od[i] = 1e30f;
    }
}

// ---------------------------------------------------------------- blocked path (mid-size clouds)
// Clouds of 4097 .. 32767 sources (and k below the warp path's range or clouds above its size):
// the sources of each cloud are put in Morton order and cut into blocks of 32 with a box each,
// the queries in Morton order and cut into tiles of 128 (one per thread). A tile orders its
// cloud's blocks by the lower bound of the distance between the tile's box and the block's box
// (coarse bins of the bound's float bits, a counting sort), then visits them nearest-first in
// stages of kKbStage blocks: a warp skips a block whose point-to-box bound is >= the current
// (k_eff+1)-th best distance of each of its lanes, and the tile stops once the next bin's lower
// edge is >= every lane's. The bounds are rounded like the distances (a difference of
// coordinates rounds to at least the rounding of the gap it covers; the fma chain keeps the
// order), so a skipped block holds no distance that could enter a list; the lists, the tie and
// overflow checks and the exact replay are those of the brute-force path, so the output is the
// reference's. Clouds with a non-finite coordinate are replayed exactly.
constexpr int kKbBlock = 32;        // sources per block
constexpr int kKbStage = 8;         // blocks staged in shared memory per pass
constexpr int kKbMaxBlocks = 1024;  // blocks a tile orders (32768 sources); larger clouds go in index order
constexpr int kKbBins = 64;
constexpr int kBwMinK = 8;          // k from which one warp serves one query (knn_bwarp_kernel)
constexpr int kBwBulk = 4;          // accepted candidates of a block above which they are merged in bulk

template <int L>
struct KbSmem {
    float2 heap[L * kKnnThreads];
    float2 buf[kKnnBuf * kKnnThreads];
    float4 pts[kKbStage * kKbBlock];
    float4 lo[kKbStage], hi[kKbStage];
    int32_t list[kKbMaxBlocks];
    uint32_t key[kKbMaxBlocks];  // block j's bound bits, then its bin
    int32_t hist[kKbBins + 1];
    float box[6][kKnnThreads / 32];
    uint32_t kmin;
};

// per-axis gap between [a_lo, a_hi] and [b_lo, b_hi], rounded no higher than any |a - b|
__device__ __forceinline__ float kb_gap(float alo, float ahi, float blo, float bhi) {
    return fmaxf(fmaxf(sub_ftz(blo, ahi), sub_ftz(alo, bhi)), 0.0f);
}
__device__ __forceinline__ float kb_lb(float gx, float gy, float gz) {
    return fma_ftz(gz, gz, fma_ftz(gx, gx, mul_ftz(gy, gy)));
}

// lower edge of a bin: bin 0 holds the bounds that are 0, bin i >= 1 the bounds whose bits >> 21
// exceed the smallest positive bound's by i - 1 (the last bin by at least that)
__device__ __forceinline__ float kb_bin_edge(uint32_t bin, uint32_t kmin) {
    return bin == 0 ? 0.0f : __uint_as_float(min(((kmin >> 21) + bin - 1) << 21, 0x7f800000u));
}

// Relative source offsets lptr[b] = ptr_s[b] - ptr_s[0]. If the sources outnumber the capacity
// the workspace was sized for (a max_cloud_sources below the true mean), every offset is 0 --
// nothing is sorted or gathered -- and `invalid` sends every query to the exact replay.
static __global__ void kb_lptr_kernel(const int64_t *__restrict__ ptr_s, int32_t B, int64_t cap,
                                      int64_t *__restrict__ lptr, int32_t *__restrict__ invalid) {
    const bool bad = ptr_s[B] - ptr_s[0] > cap || ptr_s[B] < ptr_s[0];
    for (int b = threadIdx.x; b <= B; b += blockDim.x) lptr[b] = bad ? 0 : ptr_s[b] - ptr_s[0];
    if (threadIdx.x == 0) *invalid = bad ? 1 : 0;
}

// sorted sources as float4 (x, y, z, global index bits) and each block's box: one warp per block
static __global__ void kb_blocks_kernel(const float *__restrict__ source, const int64_t *__restrict__ ptr_s,
                                        const int64_t *__restrict__ lptr, int32_t B,
                                        const int32_t *__restrict__ blk_base, const int32_t *__restrict__ order,
                                        const int32_t *__restrict__ invalid, float4 *__restrict__ pts,
                                        float4 *__restrict__ blk_lo, float4 *__restrict__ blk_hi) {
    if (*invalid) return;
    const int lane = threadIdx.x & 31;
    const int nblk = blk_base[B];
    for (int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < nblk; g += (gridDim.x * blockDim.x) >> 5) {
        const int b = find_segment(blk_base, B, g);
        const int64_t j = lptr[b] + (int64_t)(g - blk_base[b]) * kKbBlock + lane;  // sorted position
        float x = INFINITY, y = INFINITY, z = INFINITY, X = -INFINITY, Y = -INFINITY, Z = -INFINITY;
        if (j < lptr[b + 1]) {
            const int64_t v = ptr_s[0] + order[j];
            const float px = source[3 * v], py = source[3 * v + 1], pz = source[3 * v + 2];
            pts[j] = make_float4(px, py, pz, __int_as_float((int32_t)v));
            x = X = px;
            y = Y = py;
            z = Z = pz;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            x = fminf(x, __shfl_xor_sync(0xffffffffu, x, o));
            y = fminf(y, __shfl_xor_sync(0xffffffffu, y, o));
            z = fminf(z, __shfl_xor_sync(0xffffffffu, z, o));
            X = fmaxf(X, __shfl_xor_sync(0xffffffffu, X, o));
            Y = fmaxf(Y, __shfl_xor_sync(0xffffffffu, Y, o));
            Z = fmaxf(Z, __shfl_xor_sync(0xffffffffu, Z, o));
        }
        if (lane == 0) {
            blk_lo[g] = make_float4(x, y, z, 0.0f);
            blk_hi[g] = make_float4(X, Y, Z, 0.0f);
        }
    }
}

template <int KB, int L>
__global__ void __launch_bounds__(kKnnThreads) knn_block_kernel(
    const float *__restrict__ query, const int64_t *__restrict__ ptr_q, int32_t B, int k,
    const int32_t *__restrict__ tile_base, const int32_t *__restrict__ qorder, const int64_t *__restrict__ lptr,
    const int32_t *__restrict__ blk_base, const float4 *__restrict__ pts, const float4 *__restrict__ blk_lo,
    const float4 *__restrict__ blk_hi, const int32_t *__restrict__ bad, const int32_t *__restrict__ invalid,
    int64_t *__restrict__ out_idx, float *__restrict__ out_dist, int32_t *__restrict__ flag_list,
    int32_t *__restrict__ flag_count, unsigned long long *__restrict__ pairs) {
    extern __shared__ __align__(16) unsigned char kb_smem_raw[];
    KbSmem<L> &S = *reinterpret_cast<KbSmem<L> *>(kb_smem_raw);
    const int t = blockIdx.x;
    if (t >= tile_base[B]) return;  // uniform over the CTA
    const int b = find_segment(tile_base, B, t);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t qp = ptr_q[b] + (int64_t)(t - tile_base[b]) * kKnnThreads + tid;
    const bool valid = qp < ptr_q[b + 1];
    const int64_t q = valid ? (int64_t)qorder[qp] : 0;
    float qx = 0.0f, qy = 0.0f, qz = 0.0f;
    bool nonfinite = false;
    if (valid) {
        qx = query[3 * q];
        qy = query[3 * q + 1];
        qz = query[3 * q + 2];
        nonfinite = !(isfinite(qx) && isfinite(qy) && isfinite(qz));
    }
    if (*invalid || bad[b]) {  // uniform: the exact replay serves the whole tile
        if (valid) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    const int ke = k < 64 ? k : 64;
    const int64_t ns = lptr[b + 1] - lptr[b];
    const float4 *cp = pts + lptr[b];
    const int nb = blk_base[b + 1] - blk_base[b];
    const float4 *clo = blk_lo + blk_base[b], *chi = blk_hi + blk_base[b];

    // the tile's box (its finite queries)
    {
        float v[6];
        const bool in = valid && !nonfinite;
        v[0] = in ? qx : INFINITY;
        v[1] = in ? qy : INFINITY;
        v[2] = in ? qz : INFINITY;
        v[3] = in ? qx : -INFINITY;
        v[4] = in ? qy : -INFINITY;
        v[5] = in ? qz : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int c = 0; c < 6; ++c) {
                const float y = __shfl_xor_sync(0xffffffffu, v[c], o);
                v[c] = c < 3 ? fminf(v[c], y) : fmaxf(v[c], y);
            }
        if (lane == 0)
#pragma unroll
            for (int c = 0; c < 6; ++c) S.box[c][warp] = v[c];
        if (tid < kKbBins + 1) S.hist[tid] = 0;
        if (tid == 0) S.kmin = 0xffffffffu;
    }
    __syncthreads();
    float tb[6];
#pragma unroll
    for (int c = 0; c < 6; ++c) {
        float x = S.box[c][0];
#pragma unroll
        for (int w = 1; w < kKnnThreads / 32; ++w) x = c < 3 ? fminf(x, S.box[c][w]) : fmaxf(x, S.box[c][w]);
        tb[c] = x;
    }
    // blocks in ascending order of their bound to the tile (bins of the bound's bits)
    const bool ordered = nb <= kKbMaxBlocks;
    if (ordered) {
        for (int j = tid; j < nb; j += kKnnThreads) {
            const float4 lo = clo[j], hi = chi[j];
            const float lb = kb_lb(kb_gap(tb[0], tb[3], lo.x, hi.x), kb_gap(tb[1], tb[4], lo.y, hi.y),
                                   kb_gap(tb[2], tb[5], lo.z, hi.z));
            const uint32_t bits = __float_as_uint(lb);
            S.key[j] = bits;
            if (bits > 0u) atomicMin(&S.kmin, bits);
        }
        __syncthreads();
        const uint32_t kmin = S.kmin;
        for (int j = tid; j < nb; j += kKnnThreads) {
            const uint32_t bits = S.key[j];
            const uint32_t d = bits == 0u ? 0u : 1u + min((bits >> 21) - (kmin >> 21), (uint32_t)(kKbBins - 2));
            S.key[j] = d;
            atomicAdd(&S.hist[d + 1], 1);
        }
        __syncthreads();
        if (warp == 0) {  // exclusive offsets of the bins (hist[0] stays 0)
            int carry = 0;
            for (int c0 = 1; c0 <= kKbBins; c0 += 32) {
                int v = c0 + lane <= kKbBins ? S.hist[c0 + lane] : 0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int u = __shfl_up_sync(0xffffffffu, v, o);
                    if (lane >= o) v += u;
                }
                if (c0 + lane <= kKbBins) S.hist[c0 + lane] = v + carry;
                carry += __shfl_sync(0xffffffffu, v, 31);
            }
        }
        __syncthreads();
        for (int j = tid; j < nb; j += kKnnThreads) {
            const uint32_t d = S.key[j];
            S.list[atomicAdd(&S.hist[d], 1)] = j;
        }
        __syncthreads();  // S.key[j] keeps block j's bin for the early stop
    }
    const uint32_t kmin = S.kmin;

    const uint64_t QX = pack2(qx, qx), QY = pack2(qy, qy), QZ = pack2(qz, qz);
    float2 *heap = S.heap + tid;
    float2 *buf = S.buf + tid;
    int cnt = 0, nbuf = 0;
    float thr = valid ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
    const int wvalid = __popc(__ballot_sync(0xffffffffu, valid));
    unsigned long long tested = 0;  // distances this warp evaluates (its valid lanes x block sizes)
    for (int p0 = 0; p0 < nb; p0 += kKbStage) {
        if (ordered) {
            const float edge = kb_bin_edge(S.key[S.list[p0]], kmin);
            if (__syncthreads_and(!(thr > edge))) break;  // every later block is at least this far
        } else {
            __syncthreads();
        }
        const int m = nb - p0 < kKbStage ? nb - p0 : kKbStage;
        for (int i = tid; i < m * kKbBlock; i += kKnnThreads) {
            const int blk = ordered ? S.list[p0 + i / kKbBlock] : p0 + i / kKbBlock;
            const int64_t j = (int64_t)blk * kKbBlock + (i % kKbBlock);
            S.pts[i] = j < ns ? cp[j] : make_float4(__int_as_float(0x7fffffff), __int_as_float(0x7fffffff),
                                                    __int_as_float(0x7fffffff), 0.0f);  // NaN never passes `<`
        }
        if (tid < m) {
            const int blk = ordered ? S.list[p0 + tid] : p0 + tid;
            S.lo[tid] = clo[blk];
            S.hi[tid] = chi[blk];
        }
        __syncthreads();
        for (int g = 0; g < m; ++g) {
            const float4 lo = S.lo[g], hi = S.hi[g];
            const float lb = kb_lb(kb_gap(qx, qx, lo.x, hi.x), kb_gap(qy, qy, lo.y, hi.y), kb_gap(qz, qz, lo.z, hi.z));
            if (!__any_sync(0xffffffffu, lb < thr)) continue;  // no lane of this warp can gain from it
            tested += (unsigned long long)wvalid * kKbBlock;
#pragma unroll
            for (int e0 = 0; e0 < kKbBlock; e0 += kKnnGroup) {
                if (__any_sync(0xffffffffu, nbuf > kKnnBuf - kKnnGroup)) {
                    for (int e = 0; e < nbuf; ++e) {
                        const float2 x = buf[e * kS];
                        if (x.x < thr) kheap_add<L>(heap, cnt, thr, x);
                    }
                    nbuf = 0;
                }
                const float4 *sp = S.pts + g * kKbBlock + e0;
                float d[kKnnGroup];
#pragma unroll
                for (int e = 0; e < kKnnGroup; e += 2)
                    unpack2(dist2_x2(QX, QY, QZ, pack2(sp[e].x, sp[e + 1].x), pack2(sp[e].y, sp[e + 1].y),
                                     pack2(sp[e].z, sp[e + 1].z)),
                            d[e], d[e + 1]);
                const float mn = fminf(fminf(fminf(d[0], d[1]), fminf(d[2], d[3])),
                                       fminf(fminf(d[4], d[5]), fminf(d[6], d[7])));
                if (mn < thr) {
#pragma unroll
                    for (int e = 0; e < kKnnGroup; ++e) {
                        buf[nbuf * kS] = make_float2(d[e], sp[e].w);
                        nbuf += d[e] < thr ? 1 : 0;
                    }
                }
            }
        }
    }
    for (int e = 0; e < nbuf; ++e) {
        const float2 x = buf[e * kS];
        if (x.x < thr) kheap_add<L>(heap, cnt, thr, x);
    }
    if (lane == 0 && tested) atomicAdd(pairs, tested);
    if (!valid) return;
    float td[KB + 1];
    int ti[KB + 1];
    // every finite distance meets a list that is not full (a block is skipped only when its bound
    // is >= the threshold, +inf until the list is full): a short list means overflowed distances
    nonfinite |= (int64_t)cnt < (ns < L ? ns : (int64_t)L);
    kheap_sorted(heap, cnt, td, ti);
    if (cnt > ke + 1) cnt = ke + 1;
    if (nonfinite || top_has_tie(td, cnt)) {
        flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    write_row(out_idx + q * k, out_dist + q * k, k, cnt < ke ? cnt : ke, td, ti);
}

// One warp per query over the same blocks (k >= 8): the warp bounds its query's distance to every
// block of the cloud (the bounds in shared memory), then repeatedly takes the nearest unvisited
// block -- a warp minimum -- until that bound is >= the (k_eff+1)-th best distance so far; each
// visited block's 32 sources are tested one per lane against the threshold and accepted ones go
// into the warp's sorted list (as knn_warp_kernel). Nearest-first means few inserts; the stop rule
// is exact for the same reason as in knn_block_kernel.
constexpr int kBwWarps = 8;

__device__ __forceinline__ int kb_find_cloud(const int64_t *__restrict__ ptr, int B, int64_t q) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (ptr[mid] <= q) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

template <int NR>
__global__ void __launch_bounds__(kBwWarps * 32) knn_bwarp_kernel(
    const float *__restrict__ query, const int64_t *__restrict__ ptr_q, int32_t B, int k,
    const int32_t *__restrict__ qorder, const int64_t *__restrict__ lptr, const int32_t *__restrict__ blk_base,
    const float4 *__restrict__ pts, const float4 *__restrict__ blk_lo, const float4 *__restrict__ blk_hi,
    const int32_t *__restrict__ bad, const int32_t *__restrict__ invalid, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count,
    unsigned long long *__restrict__ pairs) {
    __shared__ float lbs[kBwWarps][kKbMaxBlocks];
    __shared__ float mrg_d[kBwWarps][32 * NR];  // the bulk merge's staging
    __shared__ int mrg_i[kBwWarps][32 * NR];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t p = ptr_q[0] + (int64_t)blockIdx.x * kBwWarps + warp;
    if (p >= ptr_q[B]) return;  // uniform over the warp; no block-wide barrier follows
    const int b = kb_find_cloud(ptr_q, B, p);
    const int64_t q = qorder[p];
    const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
    const int nb = blk_base[b + 1] - blk_base[b];
    if (*invalid || bad[b] || !(isfinite(qx) && isfinite(qy) && isfinite(qz)) || nb > kKbMaxBlocks) {
        if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;  // exact replay
        return;
    }
    const int64_t ns = lptr[b + 1] - lptr[b];
    const float4 *cp = pts + lptr[b];
    const float4 *clo = blk_lo + blk_base[b], *chi = blk_hi + blk_base[b];
    float *lb = lbs[warp];
    for (int j = lane; j < nb; j += 32) {
        const float4 lo = clo[j], hi = chi[j];
        lb[j] = kb_lb(kb_gap(qx, qx, lo.x, hi.x), kb_gap(qy, qy, lo.y, hi.y), kb_gap(qz, qz, lo.z, hi.z));
    }
    __syncwarp();
    const int ke = k < 64 ? k : 64;
    const int L = ke + 1;
    const float kInf = __int_as_float(0x7f800000);
    float ed[NR];
    int ei[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        ed[r] = kInf;
        ei[r] = -1;
    }
    float thr = kInf;
    int cnt = 0, visits = 0;
    for (int it = 0; it < nb; ++it) {
        // the nearest unvisited block (visited ones hold a NaN bound, which never wins)
        uint32_t best = 0xffffffffu;
        int bj = -1;
        for (int j = lane; j < nb; j += 32) {
            const float v = lb[j];
            const uint32_t key = v == v ? __float_as_uint(v) : 0xffffffffu;  // bounds are >= 0
            if (key < best) {
                best = key;
                bj = j;
            }
        }
        const uint32_t m = __reduce_min_sync(0xffffffffu, best);
        if (m == 0xffffffffu || !(__uint_as_float(m) < thr)) break;  // every unvisited block is this far
        const int wl = __ffs(__ballot_sync(0xffffffffu, best == m)) - 1;
        const int j = __shfl_sync(0xffffffffu, bj, wl);
        if (lane == 0) lb[j] = __int_as_float(0x7fffffff);
        ++visits;
        const int64_t sj = (int64_t)j * kKbBlock + lane;
        float d = kInf;
        int si = -1;
        if (sj < ns) {
            const float4 sp = cp[sj];
            d = dist2(qx, qy, qz, sp.x, sp.y, sp.z);
            si = __float_as_int(sp.w);
        }
        unsigned acc = __ballot_sync(0xffffffffu, d < thr);
        if (__popc(acc) > kBwBulk) {  // many candidates: one bulk merge
            const bool in = (acc >> lane) & 1u;
            warp_list_merge<NR>(ed, ei, in ? d : kInf, in ? si : -1, L, lane, mrg_d[warp], mrg_i[warp]);
            cnt += __popc(acc);
#pragma unroll
            for (int r = 0; r < NR; ++r)
                if ((L - 1) / 32 == r) thr = __shfl_sync(0xffffffffu, ed[r], (L - 1) & 31);
            acc = 0u;
        }
        while (acc) {
            const int l = __ffs(acc) - 1;
            acc &= acc - 1;
            const float dd = __shfl_sync(0xffffffffu, d, l);
            const int ii = __shfl_sync(0xffffffffu, si, l);
            if (!(dd < thr)) continue;  // the threshold tightened since the ballot (uniform)
            warp_list_insert<NR>(ed, ei, dd, ii, lane);
            ++cnt;
#pragma unroll
            for (int r = 0; r < NR; ++r)  // threshold = entry L - 1 (register set, lane uniform)
                if ((L - 1) / 32 == r) thr = __shfl_sync(0xffffffffu, ed[r], (L - 1) & 31);
        }
        __syncwarp();
    }
    if (lane == 0) atomicAdd(pairs, (unsigned long long)visits * kKbBlock);
    const int have = cnt < L ? cnt : L;
    // every finite distance meets a list that is not full: a short list means overflowed distances
    bool flag = (int64_t)have < (ns < L ? ns : (int64_t)L);
    if (!flag) {
        bool tie = false;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const float up = __shfl_up_sync(0xffffffffu, ed[r], 1);
            const float cross = r > 0 ? __shfl_sync(0xffffffffu, ed[r > 0 ? r - 1 : 0], 31) : 0.0f;
            const int i = lane + 32 * r;
            const float prev = lane > 0 ? up : cross;
            if (i >= 1 && i < have && prev == ed[r]) tie = true;
        }
        flag = __any_sync(0xffffffffu, tie);
    }
    if (flag) {
        if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        return;
    }
    const int nv = have < ke ? have : ke;
    int64_t *oi = out_idx + q * k;
    float *od = out_dist + q * k;
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int i = lane + 32 * r;
        if (i < k) {
            oi[i] = i < nv ? (int64_t)ei[r] : -1;
            od[i] = i < nv ? ed[r] : 1e30f;
        }
    }
    for (int i = 32 * NR + lane; i < k; i += 32) {
        oi[i] = -1;
        od[i] = 1e30f;
    }
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

// The reference kernel's heap, replayed exactly for flagged queries: one CTA per query. All its
// warps compute the distances of a stretch of kExactStretch sources into shared memory; then warp
// 0 walks them in source order, 32 at a time: a candidate the heap rejects now (full and d >= root
// -- the root never grows while distances are ordered) is rejected at its turn too, so only the
// ballot of the others is walked, and every lane applies the same MinKHeap::add to its own copy of
// the heap. A chunk with a NaN distance (or a NaN root) walks every candidate.
constexpr int kExactThreads = 256;
constexpr int kExactStretch = 4096;

__global__ void __launch_bounds__(kExactThreads) knn_exact_kernel(
    const float *__restrict__ query, const float *__restrict__ source, const int64_t *__restrict__ ptr_q,
    const int64_t *__restrict__ ptr_s, int32_t B, int k, const int32_t *__restrict__ flag_list,
    const int32_t *__restrict__ flag_count, int64_t *__restrict__ out_idx, float *__restrict__ out_dist,
    unsigned long long *__restrict__ pairs) {
    __shared__ float sd[kExactStretch];
    __shared__ float cmin[kExactStretch / 32];  // per 32-candidate chunk: smallest distance, NaN if any
    const int nflag = *flag_count;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int f = blockIdx.x; f < nflag; f += gridDim.x) {  // uniform over the CTA
        const int64_t q = flag_list[f];
        const int b = find_cloud(ptr_q, B, q);
        const float qx = query[3 * q], qy = query[3 * q + 1], qz = query[3 * q + 2];
        MinKHeap h;
        h.init(knn_bucket(k));
        const int64_t s0 = ptr_s[b], se = ptr_s[b + 1];
        for (int64_t c0 = s0; c0 < se; c0 += kExactStretch) {
            const int m = (int)(se - c0 < kExactStretch ? se - c0 : kExactStretch);
            __syncthreads();  // the previous stretch's walk is done
            for (int i0 = 0; i0 < m; i0 += kExactThreads) {  // whole warps: 32 consecutive candidates
                const int i = i0 + tid;
                float d = __int_as_float(0x7f800000);
                if (i < m) {
                    const float *p = source + 3 * (c0 + i);
                    d = dist2(qx, qy, qz, p[0], p[1], p[2]);
                    sd[i] = d;
                }
                float mn = d;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                const bool nan = __any_sync(0xffffffffu, d != d);
                if (lane == 0 && i0 + warp * 32 < m) cmin[(i0 >> 5) + warp] = nan ? __int_as_float(0x7fc00000) : mn;
            }
            __syncthreads();
            if (warp == 0) {
                // Chunks are walked in order; a chunk whose smallest distance is >= the heap's largest
                // (heap full, nothing NaN) holds no candidate the heap would take, and stays so as the
                // heap's largest only decreases -- 32 chunks are tested per ballot. The others are
                // walked candidate by candidate exactly as before.
                const int nch = (m + 31) >> 5;
                for (int g0 = 0; g0 < nch; g0 += 32) {
                    const bool have = g0 + lane < nch;
                    const float cm = have ? cmin[g0 + lane] : 0.0f;
                    const bool full0 = h.count >= h.cap;
                    const float root0 = full0 ? h.d[0] : 0.0f;
                    unsigned need =
                        __ballot_sync(0xffffffffu, have && !(full0 && root0 == root0 && cm >= root0));
                    while (need) {
                        const int j0 = (g0 + __ffs(need) - 1) << 5;
                        need &= need - 1;
                        const bool in = j0 + lane < m;
                        const float d = in ? sd[j0 + lane] : 0.0f;
                        const bool full = h.count >= h.cap;
                        const bool unordered = __any_sync(0xffffffffu, in && d != d) || (full && h.d[0] != h.d[0]);
                        unsigned live = __ballot_sync(0xffffffffu, in && (unordered || !(full && d >= h.d[0])));
                        while (live) {
                            const int l = __ffs(live) - 1;
                            live &= live - 1;
                            h.add(__shfl_sync(0xffffffffu, d, l), (int)(c0 + j0 + l));
                        }
                    }
                }
            }
        }
        if (tid == 0) {
            h.sort_ascending();
            write_row(out_idx + q * k, out_dist + q * k, k, h.count < k ? h.count : k, h.d, h.i);
            atomicAdd(pairs, (unsigned long long)(se - s0));
        }
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

struct KbWs {  // the blocked path's buffers
    int64_t *lptr;
    int32_t *invalid, *bad, *blk_base, *sorder, *qorder;
    float *box;
    uint32_t *skeys, *sskeys, *qkeys, *sqkeys;
    float4 *pts, *blk_lo, *blk_hi;
    RadixScratch rs;
};

struct KnnWs {
    int32_t *tile_base, *flag_count, *flag_list, *part_i, *part_cnt;
    unsigned long long *pairs;  // distances evaluated by the call (after flag_count, 8-byte aligned)
    float *part_d;
    bool grid;   // clouds large enough for the grid path (knn_grid.cu)
    bool block;  // mid-size clouds: the blocked path
    KgWs kg;
    KbWs kb;
};

// The grid path needs local source indices below 2^31.
static bool knn_use_grid(int32_t B, int64_t max_src) {
    return max_src >= kKgMinSources && (int64_t)B * max_src < ((int64_t)1 << 31) - 1;
}

// Clouds above the warp path's size that the grid path does not take go blocked, except for a
// single small query set per cloud (the split brute-force scan then fills the GPU better).
constexpr int64_t kKbMinSources = 4097;
static bool knn_use_block(int64_t n_q, int32_t B, int64_t max_src) {
    return max_src >= kKbMinSources && !knn_use_grid(B, max_src) && (int64_t)B * max_src < ((int64_t)1 << 31) - 1 &&
           n_q >= (int64_t)4 * kSmCount;
}



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
    t.flag_count = (int32_t *)take(sizeof(int32_t) + sizeof(unsigned long long));  // + the distance count
    t.pairs = t.flag_count ? (unsigned long long *)(t.flag_count + 2) : nullptr;
    t.flag_list = (int32_t *)take(sizeof(int32_t) * nq);
    const int64_t np = split > 1 ? nq * split : 1;
    t.part_cnt = (int32_t *)take(sizeof(int32_t) * np);
    t.part_d = (float *)take(sizeof(float) * np * (kb + 1));
    t.part_i = (int32_t *)take(sizeof(int32_t) * np * (kb + 1));
    t.grid = knn_use_grid(B, max_src);
    if (t.grid) {
        const size_t gbytes = knn_grid_ws((int64_t)B * max_src, B, nullptr, nullptr);
        char *gb = take(gbytes);
        if (base) knn_grid_ws((int64_t)B * max_src, B, gb, &t.kg);
    }
    t.block = knn_use_block(n_q, B, max_src);
    if (t.block) {
        const int64_t cap = (int64_t)B * max_src > 0 ? (int64_t)B * max_src : 1;
        const int64_t nblk = cap / kKbBlock + B + 1;
        const int32_t nb = B > 0 ? B : 1;
        t.kb.lptr = (int64_t *)take(sizeof(int64_t) * (nb + 1));
        t.kb.invalid = (int32_t *)take(sizeof(int32_t));
        t.kb.bad = (int32_t *)take(sizeof(int32_t) * nb);
        t.kb.blk_base = (int32_t *)take(sizeof(int32_t) * (nb + 1));
        t.kb.box = (float *)take(sizeof(float) * 6 * nb);
        t.kb.skeys = (uint32_t *)take(sizeof(uint32_t) * cap);
        t.kb.sskeys = (uint32_t *)take(sizeof(uint32_t) * cap);
        t.kb.sorder = (int32_t *)take(sizeof(int32_t) * cap);
        t.kb.qkeys = (uint32_t *)take(sizeof(uint32_t) * nq);
        t.kb.sqkeys = (uint32_t *)take(sizeof(uint32_t) * nq);
        t.kb.qorder = (int32_t *)take(sizeof(int32_t) * nq);
        t.kb.pts = (float4 *)take(sizeof(float4) * cap);
        t.kb.blk_lo = (float4 *)take(sizeof(float4) * nblk);
        t.kb.blk_hi = (float4 *)take(sizeof(float4) * nblk);
        const int64_t rn = cap > nq ? cap : nq;
        char *rb = take(radix_scratch_bytes(rn, nb));
        if (base) t.kb.rs = radix_carve(rb, rn, nb);
    }
    if (w) *w = t;
    return off;
}

template <int KB, int L>
static void knn_block_launch(const float *query, const int64_t *ptr_q, int32_t B, int64_t n_q, int k,
                             const KnnWs &w, int64_t *oi, float *od, cudaStream_t st) {
    const size_t smem = sizeof(KbSmem<L>);
    cudaFuncSetAttribute(knn_block_kernel<KB, L>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const KbWs &b = w.kb;
    knn_block_kernel<KB, L><<<(unsigned)(n_q / kKnnThreads + B), kKnnThreads, smem, st>>>(
        query, ptr_q, B, k, w.tile_base, b.qorder, b.lptr, b.blk_base, b.pts, b.blk_lo, b.blk_hi, b.bad, b.invalid,
        oi, od, w.flag_list, w.flag_count, w.pairs);
}

// Morton order of each cloud's sources (blocks of 32 with boxes) and queries (tiles of 128), then
// the blocked search; the tile offsets (tile_base) must already be built for kKnnThreads.
static cudaError_t knn_block_run(const float *query, const float *source, const int64_t *ptr_q,
                                 const int64_t *ptr_s, int32_t B, int64_t n_q, int k, int64_t max_src,
                                 const KnnWs &w, int64_t *oi, float *od, cudaStream_t st) {
    const KbWs &b = w.kb;
    const int64_t cap = (int64_t)B * max_src;
    kb_lptr_kernel<<<1, 256, 0, st>>>(ptr_s, B, cap, b.lptr, b.invalid);
    cloud_box_kernel<<<B, kBoxThreads, 0, st>>>(source, ptr_s, b.box, b.bad);
    const unsigned gs = (unsigned)((cap + 255) / 256 < 4 * kSmCount ? (cap + 255) / 256 : 4 * kSmCount);
    // 24-bit codes (256 cells per axis: far finer than a block of 32 points in clouds of up to 32767)
    // sort in three 8-bit passes; the order only groups nearby points -- every bound below comes
    // from the blocks' actual boxes
    morton_code_kernel<<<gs > 0 ? gs : 1, 256, 0, st>>>(source, ptr_s, B, b.box, b.skeys, true, cap, 6);
    const unsigned gq = (unsigned)((n_q + 255) / 256 < 4 * kSmCount ? (n_q + 255) / 256 : 4 * kSmCount);
    morton_code_kernel<<<gq > 0 ? gq : 1, 256, 0, st>>>(query, ptr_q, B, b.box, b.qkeys, false, n_q, 6);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // (with `invalid` set the offsets are all 0: the source sort sorts nothing)
    e = radix_sort_pairs(b.skeys, nullptr, b.sskeys, b.sorder, cap, b.lptr, B, 3, nullptr, b.rs, st);
    if (e != cudaSuccess) return e;
    e = radix_sort_pairs(b.qkeys, nullptr, b.sqkeys, b.qorder, n_q, ptr_q, B, 3, nullptr, b.rs, st);
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    knn_tiles_kernel<<<1, kScanThreads, 0, st>>>(ptr_s, B, kKbBlock, b.blk_base);
    const unsigned gb = (unsigned)((cap / kKbBlock + B + 7) / 8 < 8 * kSmCount ? (cap / kKbBlock + B + 7) / 8
                                                                              : 8 * kSmCount);
    kb_blocks_kernel<<<gb > 0 ? gb : 1, 256, 0, st>>>(source, ptr_s, b.lptr, B, b.blk_base, b.sorder, b.invalid,
                                                       b.pts, b.blk_lo, b.blk_hi);
    if (k >= kBwMinK) {  // one warp per query, nearest block first
        const int L = (k < 64 ? k : 64) + 1;
        const unsigned grid = (unsigned)((n_q + kBwWarps - 1) / kBwWarps);
        if (L <= 32)
            knn_bwarp_kernel<1><<<grid, kBwWarps * 32, 0, st>>>(query, ptr_q, B, k, b.qorder, b.lptr, b.blk_base,
                                                                b.pts, b.blk_lo, b.blk_hi, b.bad, b.invalid, oi, od,
                                                                w.flag_list, w.flag_count, w.pairs);
        else if (L <= 64)
            knn_bwarp_kernel<2><<<grid, kBwWarps * 32, 0, st>>>(query, ptr_q, B, k, b.qorder, b.lptr, b.blk_base,
                                                                b.pts, b.blk_lo, b.blk_hi, b.bad, b.invalid, oi, od,
                                                                w.flag_list, w.flag_count, w.pairs);
        else
            knn_bwarp_kernel<3><<<grid, kBwWarps * 32, 0, st>>>(query, ptr_q, B, k, b.qorder, b.lptr, b.blk_base,
                                                                b.pts, b.blk_lo, b.blk_hi, b.bad, b.invalid, oi, od,
                                                                w.flag_list, w.flag_count, w.pairs);
        return cudaGetLastError();
    }
    switch (knn_bucket(k)) {
    case 4:
        if (k == 1) knn_block_launch<4, 2>(query, ptr_q, B, n_q, k, w, oi, od, st);
        else knn_block_launch<4, 5>(query, ptr_q, B, n_q, k, w, oi, od, st);
        break;
    case 8: knn_block_launch<8, 9>(query, ptr_q, B, n_q, k, w, oi, od, st); break;
    case 16: knn_block_launch<16, 17>(query, ptr_q, B, n_q, k, w, oi, od, st); break;
    case 32: knn_block_launch<32, 33>(query, ptr_q, B, n_q, k, w, oi, od, st); break;
    default: knn_block_launch<64, 65>(query, ptr_q, B, n_q, k, w, oi, od, st); break;
    }
    return cudaGetLastError();
}

template <int KB>
static void knn_launch(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
                       int32_t B, int64_t n_q, int k, int split, const KnnWs &w, int64_t *oi, float *od,
                       cudaStream_t st) {
    const int64_t grid = (n_q / kKnnThreads + B) * split;
    if (KB == 4 && k == 1) {  // nearest neighbour: a list of two decides it
        const size_t smem = knn_smem_bytes<2>();
        cudaFuncSetAttribute(knn_fast_kernel<KB, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        knn_fast_kernel<KB, 2><<<(unsigned)grid, kKnnThreads, smem, st>>>(
            query, source, ptr_q, ptr_s, B, k, split, w.tile_base, oi, od, w.part_d, w.part_i, w.part_cnt,
            w.flag_list, w.flag_count, w.pairs);
    } else {
        const size_t smem = knn_smem_bytes<KB + 1>();
        cudaFuncSetAttribute(knn_fast_kernel<KB, KB + 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        knn_fast_kernel<KB, KB + 1><<<(unsigned)grid, kKnnThreads, smem, st>>>(
            query, source, ptr_q, ptr_s, B, k, split, w.tile_base, oi, od, w.part_d, w.part_i, w.part_cnt,
            w.flag_list, w.flag_count, w.pairs);
    }
    if (split > 1) {
        const size_t msm = knn_merge_smem(split, k);
        cudaFuncSetAttribute(knn_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msm);
        knn_merge_kernel<<<(unsigned)((n_q + kMergeWarps - 1) / kMergeWarps), kKnnThreads, msm, st>>>(
            ptr_q, B, k, split, KB + 1, w.part_d, w.part_i, w.part_cnt, oi, od, w.flag_list, w.flag_count);
    }
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
    GDL_CUDA_TRY(cudaMemsetAsync(w.flag_count, 0, 2 * sizeof(int32_t) + sizeof(unsigned long long), st));
    const bool warp_path = k >= kWarpMinK && max_cloud_sources <= kWarpMaxSources && !w.block;
    knn_tiles_kernel<<<1, kScanThreads, 0, st>>>(ptr_q, num_clouds, warp_path ? kWarpQ : kKnnThreads, w.tile_base);
    knn_pad_kernel<<<padg, 256, 0, st>>>(ptr_q, num_clouds, n_query, k, out_idx, out_dist);
    if (w.grid) {  // large clouds: exact search over a grid of each cloud's sources
        GDL_CUDA_TRY(knn_grid_run(query, source, ptr_q, ptr_s, num_clouds, n_query, k, max_cloud_sources, w.kg,
                                  out_idx, out_dist, w.flag_list, w.flag_count, st));
        knn_exact_kernel<<<kSmCount, kExactThreads, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.flag_list,
                                                           w.flag_count, out_idx, out_dist, w.pairs);
        GDL_CUDA_TRY(cudaGetLastError());
        return GDL_OK;
    }
    if (w.block) {  // mid-size clouds: Morton-ordered source blocks, nearest first
        GDL_CUDA_TRY(knn_block_run(query, source, ptr_q, ptr_s, num_clouds, n_query, k, max_cloud_sources, w,
                                   out_idx, out_dist, st));
        knn_exact_kernel<<<kSmCount, kExactThreads, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.flag_list,
                                                           w.flag_count, out_idx, out_dist, w.pairs);
        GDL_CUDA_TRY(cudaGetLastError());
        return GDL_OK;
    }
    if (warp_path) {
        const unsigned grid = (unsigned)(n_query / kWarpQ + num_clouds);
        const int L = (k < 64 ? k : 64) + 1;
        if (L <= 32)
            knn_warp_kernel<1><<<grid, kWarpQ * 32, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.tile_base,
                                                             out_idx, out_dist, w.flag_list, w.flag_count, w.pairs);
        else if (L <= 64)
            knn_warp_kernel<2><<<grid, kWarpQ * 32, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.tile_base,
                                                             out_idx, out_dist, w.flag_list, w.flag_count, w.pairs);
        else
            knn_warp_kernel<3><<<grid, kWarpQ * 32, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.tile_base,
                                                             out_idx, out_dist, w.flag_list, w.flag_count, w.pairs);
        knn_exact_kernel<<<kSmCount, kExactThreads, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.flag_list,
                                                           w.flag_count, out_idx, out_dist, w.pairs);
        GDL_CUDA_TRY(cudaGetLastError());
        return GDL_OK;
    }
    const int split = knn_split(n_query, num_clouds, max_cloud_sources);
    switch (knn_bucket(k)) {
    case 4: knn_launch<4>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 8: knn_launch<8>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 16: knn_launch<16>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    case 32: knn_launch<32>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    default: knn_launch<64>(query, source, ptr_q, ptr_s, num_clouds, n_query, k, split, w, out_idx, out_dist, st); break;
    }
    knn_exact_kernel<<<kSmCount, kExactThreads, 0, st>>>(query, source, ptr_q, ptr_s, num_clouds, k, w.flag_list,
                                                       w.flag_count, out_idx, out_dist, w.pairs);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_knn_distance_count(const void *workspace, int64_t n_query, int32_t num_clouds, int32_t k,
                                      int64_t max_cloud_sources, unsigned long long *out) {
    GDL_RETURN_IF(!workspace || !out, GDL_ERR_INVALID);
    KnnWs w;
    knn_ws(n_query, num_clouds, k, max_cloud_sources, (char *)workspace, &w);
    GDL_CUDA_TRY(cudaMemcpy(out, w.pairs, sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    return GDL_OK;
}
