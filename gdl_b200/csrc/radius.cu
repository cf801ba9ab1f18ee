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
#include "geom.cuh"
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
    const int64_t o = sorted_idx[j];  // .w carries the point's global index
    sorted_pts[j] = make_float4(x[3 * o], x[3 * o + 1], x[3 * o + 2], __int_as_float((int32_t)o));
}

__device__ __forceinline__ int64_t lower_bound_u32(const uint32_t *__restrict__ a, int64_t lo, int64_t hi, uint32_t v) {
    while (lo < hi) {
        const int64_t m = (lo + hi) >> 1;
        if (a[m] < v) lo = m + 1;
        else hi = m;
    }
    return lo;
}

// ------------------------------------------------------------------ small clouds, fused
// One CTA per cloud of at most kSmallMax points does the whole pipeline in shared memory:
// bbox + grid parameters, cell keys, a stable LSD radix sort of (cell, index) (warp match +
// per-warp digit counters, as in radix.cuh), the sorted coordinates, and every query with the
// exact MinK heap. A second kernel turns the per-query counts into the global CSR.
constexpr int kSmallThreads = 512;
constexpr int kSmallMax = 4096;
constexpr int kSmallWarps = kSmallThreads / 32;
constexpr int kSmallItems = kSmallMax / kSmallThreads;  // keys per thread in a pass

constexpr int kSmallCells = 16384;  // dense cell-start table when the grid has at most this many cells

struct SmallSmem {
    uint32_t key[2][kSmallMax];
    int32_t val[2][kSmallMax];
    float4 pts[kSmallMax];
    int32_t cell_start[kSmallCells + 1];
    uint32_t warp_cnt[kSmallWarps][256];
    uint32_t digit_base[256];
    float red[6][kSmallWarps];
    GridParams g;
    int32_t warp_tot[kSmallWarps];
};

__device__ __forceinline__ GridParams grid_from_bbox(const float *lo, const float *hi, float inv_cell, int64_t n) {
    GridParams g;
    int64_t cells = 1;
    for (int a = 0; a < 3; ++a) {
        // host arithmetic of the reference, in IEEE single precision (:283-297)
        const float mn = __fsub_rn(lo[a], 1e-5f), mx = __fadd_rn(hi[a], 1e-5f);
        const float c = ceilf(__fmul_rn(__fsub_rn(mx, mn), inv_cell));
        const int r = (c >= 1023.0f) ? 1024 : (int)c + 1;
        g.mn[a] = mn;
        g.res[a] = r < 1 ? 1 : r;
        cells *= g.res[a];
    }
    g.ncells = (int)cells;
    g.ok = n > 1;
    return g;
}

// grid = num_clouds * split: CTA (b, part) rebuilds cloud b's grid in shared memory and answers
// queries [part * chunk, (part + 1) * chunk). Rows go to `padded` row-major (cap entries per
// query), unsorted; counts[q] entries each.
__global__ void __launch_bounds__(kSmallThreads) rg_small_kernel(
    const float *__restrict__ x, const int64_t *__restrict__ ptr, const uint8_t *__restrict__ mask, float r_sq,
    float inv, int loop, int cap, int split, int64_t n_all, int32_t *__restrict__ counts,
    int32_t *__restrict__ padded, int32_t *__restrict__ cloud_tot) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SmallSmem &S = *reinterpret_cast<SmallSmem *>(smem_raw);
    const int b = blockIdx.x / split, part = blockIdx.x % split;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t s0 = ptr[b];
    const int n = (int)(ptr[b + 1] - s0);

    // 1. bbox of all points of the cloud (masked ones included, :281-288)
    float lo[3] = {__int_as_float(0x7f800000), __int_as_float(0x7f800000), __int_as_float(0x7f800000)};
    float hi[3] = {__int_as_float(0xff800000), __int_as_float(0xff800000), __int_as_float(0xff800000)};
    for (int i = tid; i < n; i += kSmallThreads)
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            const float v = x[3 * (s0 + i) + a];
            lo[a] = fminf(lo[a], v);
            hi[a] = fmaxf(hi[a], v);
        }
#pragma unroll
    for (int a = 0; a < 3; ++a)
        for (int o = 16; o > 0; o >>= 1) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    if (lane == 0)
        for (int a = 0; a < 3; ++a) {
            S.red[a][warp] = lo[a];
            S.red[3 + a][warp] = hi[a];
        }
    __syncthreads();
    if (tid == 0) {
        for (int a = 0; a < 3; ++a)
            for (int w = 1; w < kSmallWarps; ++w) {
                S.red[a][0] = fminf(S.red[a][0], S.red[a][w]);
                S.red[3 + a][0] = fmaxf(S.red[3 + a][0], S.red[3 + a][w]);
            }
        const float l3[3] = {S.red[0][0], S.red[1][0], S.red[2][0]};
        const float h3[3] = {S.red[3][0], S.red[4][0], S.red[5][0]};
        S.g = grid_from_bbox(l3, h3, inv, n);
    }
    __syncthreads();
    const GridParams g = S.g;

    // 2. cell keys (masked points last, :107-111), padded to items * kSmallThreads slots
    const int items = (n + kSmallThreads - 1) / kSmallThreads;  // keys per thread in a pass
    for (int i = tid; i < items * kSmallThreads; i += kSmallThreads) {
        uint32_t key = 0xffffffffu;  // padding sorts after everything
        if (i < n) {
            if (!g.ok || (mask && !mask[s0 + i])) {
                key = (uint32_t)g.ncells;
            } else {
                int c[3];
#pragma unroll
                for (int a = 0; a < 3; ++a) {
                    const int v = cell_coord(x[3 * (s0 + i) + a], g.mn[a], inv);
                    c[a] = v < 0 ? 0 : (v > g.res[a] - 1 ? g.res[a] - 1 : v);
                }
                key = (uint32_t)((c[0] * g.res[1] + c[1]) * g.res[2] + c[2]);
            }
        }
        S.key[0][i] = key;
        S.val[0][i] = i;
    }
    int bits = 0;
    while (bits < 31 && ((int64_t)1 << bits) <= (int64_t)g.ncells) ++bits;
    const int passes = (bits + 7) / 8;
    // padding keys are 0xffffffff: they stay last as long as the digits of the passes run
    // order them after every real key, which holds because real keys < 2^bits

    // 3. stable LSD radix sort in shared memory
    int src = 0;
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int p = 0; p < passes; ++p) {
        const int shift = 8 * p;
        __syncthreads();
        for (int d = tid; d < kSmallWarps * 256; d += kSmallThreads) (&S.warp_cnt[0][0])[d] = 0;
        __syncthreads();
        uint32_t key[kSmallItems], dig[kSmallItems], rank[kSmallItems];
        int32_t val[kSmallItems];
#pragma unroll
        for (int it = 0; it < kSmallItems; ++it) {
            if (it >= items) break;
            const int idx = warp * 32 * items + it * 32 + lane;
            key[it] = S.key[src][idx];
            val[it] = S.val[src][idx];
            dig[it] = (key[it] >> shift) & 255u;
            const unsigned peers = __match_any_sync(0xffffffffu, dig[it]);
            const unsigned before = __popc(peers & lt_mask);
            const uint32_t base = S.warp_cnt[warp][dig[it]];
            __syncwarp();
            if (before == 0) S.warp_cnt[warp][dig[it]] = base + __popc(peers);
            __syncwarp();
            rank[it] = base + before;
        }
        __syncthreads();
        if (tid < 256) {  // per digit: exclusive prefix over warps, digit total
            uint32_t run = 0;
            for (int w = 0; w < kSmallWarps; ++w) {
                const uint32_t c = S.warp_cnt[w][tid];
                S.warp_cnt[w][tid] = run;
                run += c;
            }
            S.digit_base[tid] = run;
        }
        __syncthreads();
        if (tid < 32) {  // exclusive scan of the 256 digit totals by one warp
            uint32_t v[8], t = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[j] = S.digit_base[tid * 8 + j];
                t += v[j];
            }
            uint32_t inc = t;
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
                if (tid >= o) inc += y;
            }
            uint32_t run = inc - t;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t c = v[j];
                S.digit_base[tid * 8 + j] = run;
                run += c;
            }
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < kSmallItems; ++it) {
            if (it >= items) break;
            const uint32_t dst = S.digit_base[dig[it]] + S.warp_cnt[warp][dig[it]] + rank[it];
            S.key[src ^ 1][dst] = key[it];
            S.val[src ^ 1][dst] = val[it];
        }
        src ^= 1;
    }
    __syncthreads();
    // 4. sorted coordinates; first sorted position of every cell (dense table: a cell's points
    // are [cell_start[c], cell_start[c+1]); empty cells take the next cell's start)
    const uint32_t *keys = S.key[src];
    const int32_t *vals = S.val[src];
    const bool dense = g.ncells < kSmallCells;
    if (dense)
        for (int c = tid; c <= g.ncells; c += kSmallThreads) S.cell_start[c] = n;
    for (int j = tid; j < n; j += kSmallThreads) {  // .w carries the point's local index
        const int v = vals[j];
        const int64_t o = s0 + v;
        S.pts[j] = make_float4(x[3 * o], x[3 * o + 1], x[3 * o + 2], __int_as_float(v));
    }
    __syncthreads();
    if (dense) {
        for (int j = tid; j < n; j += kSmallThreads)
            // masked points carry key ncells: their run start is the end of the last cell
            if (keys[j] <= (uint32_t)g.ncells && (j == 0 || keys[j - 1] != keys[j])) S.cell_start[keys[j]] = j;
        __syncthreads();
        // suffix minimum cell_start[c] = min(cell_start[c..ncells]): each thread folds a span of
        // consecutive cells from the top, then one block-wide suffix scan of the span minima
        const int total = g.ncells + 1, span = (total + kSmallThreads - 1) / kSmallThreads;
        const int c0 = tid * span, c1 = min(c0 + span, total);
        int m = 0x7fffffff;
        for (int c = c1 - 1; c >= c0; --c) m = min(m, S.cell_start[c]);
        // inclusive suffix scan over threads (higher tid = higher cells)
        const int lane_ = tid & 31, w = tid >> 5;
        int suf = m;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_down_sync(0xffffffffu, suf, o);
            if (lane_ + o < 32) suf = min(suf, y);
        }
        if (lane_ == 0) S.warp_tot[w] = suf;
        __syncthreads();
        int above = 0x7fffffff;  // minimum over all later threads
        for (int ww = w + 1; ww < kSmallWarps; ++ww) above = min(above, S.warp_tot[ww]);
        int after = __shfl_down_sync(0xffffffffu, suf, 1);
        if (lane_ == 31) after = 0x7fffffff;
        int run = min(above, after);
        for (int c = c1 - 1; c >= c0; --c) {
            run = min(run, S.cell_start[c]);
            S.cell_start[c] = run;
        }
    }
    __syncthreads();

    // 5. queries, one warp each. Lanes 0-8 fetch the sorted-position ranges of the 9 z-columns
    // of the 27-cell neighbourhood ((dx, dy) order, empty outside the grid); a warp scan makes
    // them one candidate list that the lanes test 32 at a time; ballot/popc place the accepted
    // sources, in scan order, into the query's padded row. Rows are sorted at compaction. A
    // query with more than `cap` sources in range replays the reference heap on lane 0.
    int my_total = 0;
    const int chunk = (n + split - 1) / split;
    const int qend = min(n, (part + 1) * chunk);
    for (int q = part * chunk + warp; q < qend; q += kSmallWarps) {
        int kept = 0;
        if (g.ok && !(mask && !mask[s0 + q])) {
            const float qx = x[3 * (s0 + q)], qy = x[3 * (s0 + q) + 1], qz = x[3 * (s0 + q) + 2];
            const int qc0 = cell_coord(qx, g.mn[0], inv), qc1 = cell_coord(qy, g.mn[1], inv),
                      qc2 = cell_coord(qz, g.mn[2], inv);
            const int zlo = qc2 - 1 < 0 ? 0 : qc2 - 1;
            const int zhi = qc2 + 1 > g.res[2] - 1 ? g.res[2] - 1 : qc2 + 1;
            int j0 = 0, len = 0;
            if (lane < 9) {
                const int cx = qc0 + lane / 3 - 1, cy = qc1 + lane % 3 - 1;
                if (zlo <= zhi && cx >= 0 && cx < g.res[0] && cy >= 0 && cy < g.res[1]) {
                    const int colc = (cx * g.res[1] + cy) * g.res[2];
                    int e;
                    if (dense) {
                        j0 = S.cell_start[colc + zlo];
                        e = S.cell_start[colc + zhi + 1];
                    } else {
                        const uint32_t klo = (uint32_t)(colc + zlo), khi = (uint32_t)(colc + zhi) + 1u;
                        int lo = 0, hi = n;
                        while (lo < hi) {
                            const int m = (lo + hi) >> 1;
                            if (keys[m] < klo) lo = m + 1;
                            else hi = m;
                        }
                        j0 = lo;
                        hi = n;
                        while (lo < hi) {
                            const int m = (lo + hi) >> 1;
                            if (keys[m] < khi) lo = m + 1;
                            else hi = m;
                        }
                        e = lo;
                    }
                    len = e - j0;
                }
            }
            int inc = len;  // inclusive prefix of the column lengths
            for (int o = 1; o < 16; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const int total = __shfl_sync(0xffffffffu, inc, 8);
            const int excl = inc - len;
            // every lane takes the 9 (first candidate number, start) pairs, full-warp shuffles
            // outside any divergent branch
            int cex[9], cj[9];
#pragma unroll
            for (int c = 0; c < 9; ++c) {
                cex[c] = __shfl_sync(0xffffffffu, excl, c);
                cj[c] = __shfl_sync(0xffffffffu, j0, c);
            }
            int32_t *row = padded + (s0 + q) * cap;
            for (int base = 0; base < total; base += 32) {
                const int t = base + lane;
                bool ok = false;
                int o = 0;
                if (t < total) {
                    int j = 0;
#pragma unroll
                    for (int c = 0; c < 9; ++c)  // column holding candidate t
                        if (t >= cex[c]) j = cj[c] + (t - cex[c]);
                    const float4 sp = S.pts[j];
                    o = __float_as_int(sp.w);
                    ok = (loop || o != q) && dist2(qx, qy, qz, sp.x, sp.y, sp.z) < r_sq;
                }
                const unsigned hits = __ballot_sync(0xffffffffu, ok);
                const int pos = kept + __popc(hits & lt_mask);
                if (ok && pos < cap) row[pos] = (int32_t)(s0 + o);
                kept += __popc(hits);
            }
            if (kept > cap) {  // the reference heap decides which `cap` stay, in scan order
                int cjl[9];
#pragma unroll
                for (int c = 0; c < 9; ++c) cjl[c] = __shfl_sync(0xffffffffu, len, c);
                if (lane == 0) {
                    float hd[64];
                    int hid[64];
                    int hc = 0;
#pragma unroll
                    for (int c = 0; c < 9; ++c)
                        for (int j = cj[c]; j < cj[c] + cjl[c]; ++j) {
                            const float4 sp = S.pts[j];
                            const int o = __float_as_int(sp.w);
                            if (!loop && o == q) continue;
                            const float d = dist2(qx, qy, qz, sp.x, sp.y, sp.z);
                            if (d < r_sq) heap_add(hd, hid, hc, cap, d, o);
                        }
                    for (int a2 = 0; a2 < hc; ++a2) row[a2] = (int32_t)(s0 + hid[a2]);
                }
                __syncwarp();
                kept = cap;
            }
        }
        if (lane == 0) {
            counts[s0 + q] = kept;
            my_total += kept;
        }
    }
    for (int o = 16; o > 0; o >>= 1) my_total += __shfl_xor_sync(0xffffffffu, my_total, o);
    if (lane == 0) S.warp_tot[warp] = my_total;
    __syncthreads();
    if (tid == 0) {
        int t = 0;
        for (int w = 0; w < kSmallWarps; ++w) t += S.warp_tot[w];
        atomicAdd(&cloud_tot[b], t);  // the parts of a cloud add up (integer: order-free)
    }
}

// Sort one query's kept sources (count <= 64, in padded[0, c)) ascending with a warp bitonic
// sort (two keys per lane) and write them at o, with their geometry when g.x is set (staged in
// the warp's kGeomStageFloats floats at geo_st).
__device__ __forceinline__ void warp_sort_emit(const int32_t *__restrict__ col, int64_t stride, int c, int64_t o,
                                               int64_t q, int64_t *__restrict__ src, int64_t *__restrict__ dstv,
                                               int32_t *__restrict__ src32, const EdgeGeom &g,
                                               float *__restrict__ geo_st) {
    const int lane = threadIdx.x & 31;
    int a = lane < c ? col[lane * stride] : 0x7fffffff;
    int b = lane + 32 < c ? col[(lane + 32) * stride] : 0x7fffffff;
    if (c > 1 && c <= 32) {  // one value per lane: bitonic sort over the 32 lanes
        for (int size = 2; size <= 32; size <<= 1)
            for (int stride2 = size >> 1; stride2 > 0; stride2 >>= 1) {
                const int p = __shfl_xor_sync(0xffffffffu, a, stride2);
                const bool asc = (lane & size) == 0 || size == 32;
                const bool lower = (lane & stride2) == 0;
                a = (lower == asc) ? min(a, p) : max(a, p);
            }
    } else if (c > 32) {
        // bitonic sort of the 64 values held as (a = element lane, b = element lane + 32)
        for (int size = 2; size <= 64; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                if (stride == 32) {  // partner is the other register of the same lane
                    const bool up = true;  // size == 64: whole sequence ascending
                    const int lo = min(a, b), hi = max(a, b);
                    a = up ? lo : hi;
                    b = up ? hi : lo;
                } else {
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        int v = r == 0 ? a : b;
                        const int idx = lane + 32 * r;
                        const int p = __shfl_xor_sync(0xffffffffu, v, stride);
                        const bool asc = ((idx & size) == 0);
                        const bool lower = (idx & stride) == 0;
                        v = (lower == asc) ? min(v, p) : max(v, p);
                        if (r == 0) a = v;
                        else b = v;
                    }
                }
            }
        }
    }
    if (lane < c) {
        src[o + lane] = a;
        if (src32) src32[o + lane] = a;
        if (dstv) dstv[o + lane] = q;
    }
    if (lane + 32 < c) {
        src[o + lane + 32] = b;
        if (src32) src32[o + lane + 32] = b;
        if (dstv) dstv[o + lane + 32] = q;
    }
    if (g.x && c > 0) {  // c is warp-uniform
        const float qx = g.x[3 * q], qy = g.x[3 * q + 1], qz = g.x[3 * q + 2];
        const int64_t sa = lane < c ? a : q, sb = lane + 32 < c ? b : q;
        warp_geom_emit(g, geo_st, o, c < 32 ? c : 32, lane, qx, qy, qz, g.x[3 * sa], g.x[3 * sa + 1],
                       g.x[3 * sa + 2]);
        if (c > 32)
            warp_geom_emit(g, geo_st, o + 32, c - 32, lane, qx, qy, qz, g.x[3 * sb], g.x[3 * sb + 1],
                           g.x[3 * sb + 2]);
    }
}

// grid = num_clouds * split. Every CTA of cloud b takes the cloud's global edge offset (sum of the
// earlier clouds' totals) and scans the cloud's counts; it writes row_ptr and the edges of its
// own query part, one warp per row: bitonic sort of the row's sources, then the copy.
__global__ void __launch_bounds__(kSmallThreads) rg_small_compact_kernel(
    const int64_t *__restrict__ ptr, int32_t B, int split, int64_t n_all, int cap, const int32_t *__restrict__ counts,
    const int32_t *__restrict__ padded, const int32_t *__restrict__ cloud_tot, int64_t *__restrict__ row_ptr,
    int64_t *__restrict__ src, int64_t *__restrict__ dstv, int32_t *__restrict__ row_ptr32,
    int32_t *__restrict__ src32, const EdgeGeom geom) {
    __shared__ int64_t warp_sums[32];
    __shared__ int64_t total;
    __shared__ int64_t offs[kSmallMax];
    extern __shared__ float geo_stage[];  // kSmallWarps * kGeomStageFloats when geometry is written
    const int b = blockIdx.x / split, part = blockIdx.x % split;
    const int tid = threadIdx.x, warp = tid >> 5;
    int64_t base = 0;
    for (int c = tid; c < b; c += kSmallThreads) base += cloud_tot[c];
    (void)block_exclusive_scan<int64_t>(base, warp_sums, &total);
    base = total;
    const int64_t s0 = ptr[b], s1 = ptr[b + 1];
    const int n = (int)(s1 - s0);
    int64_t carry = base;
    for (int q0 = 0; q0 < n; q0 += kSmallThreads) {  // offsets of the whole cloud
        const int q = q0 + tid;
        const int c = q < n ? counts[s0 + q] : 0;
        const int64_t off = block_exclusive_scan<int64_t>(c, warp_sums, &total) + carry;
        if (q < n) offs[q] = off;
        carry += total;
    }
    __syncthreads();
    const int chunk = (n + split - 1) / split;
    const int qb = part * chunk, qe = min(n, qb + chunk);
    for (int q = qb + tid; q < qe; q += kSmallThreads) {
        const int64_t gq = s0 + q;
        row_ptr[gq] = offs[q];
        if (row_ptr32) row_ptr32[gq] = (int32_t)offs[q];
    }
    for (int q = qb + warp; q < qe; q += kSmallWarps)  // one warp sorts and writes a row
        warp_sort_emit(padded + (s0 + q) * cap, 1, counts[s0 + q], offs[q], s0 + q, src, dstv, src32, geom,
                       geo_stage + warp * kGeomStageFloats);
    if (b == 0 && part == 0)  // points before the first cloud have no edges
        for (int64_t q = tid; q < ptr[0]; q += kSmallThreads) {
            row_ptr[q] = 0;
            if (row_ptr32) row_ptr32[q] = 0;
        }
    if (b == B - 1 && part == split - 1)  // the end of the last cloud, and points after it
        for (int64_t q = s1 + tid; q <= n_all; q += kSmallThreads) {
            row_ptr[q] = carry;
            if (row_ptr32) row_ptr32[q] = (int32_t)carry;
        }
}


// ------------------------------------------------------------------ any cloud size
// Cell table of cloud b, kCellBudget * n_b entries from cell_start[kCellBudget * ptr[b]]:
//   * dense: the grid has at most kCellBudget * n_b - 1 cells; entry c (c = 0..ncells) is the
//     first sorted position with key >= c, so a (dx, dy) column's z-cells zlo..zhi are
//     [entry col + zlo, entry col + zhi + 1);
//   * columns: a larger grid whose res_x * res_y (x, y) columns fit; entry k (k = 0..res_x res_y)
//     is the first sorted position with key >= k * res_z, so a query binary-searches only the
//     few points of each column for its z-range;
//   * neither: the query binary-searches the cloud's sorted keys.
constexpr int kCellBudget = 16;

__device__ __forceinline__ bool dense_cells(const GridParams &g, int64_t n_b) {
    return (int64_t)g.ncells + 1 <= kCellBudget * n_b;
}

__device__ __forceinline__ bool column_cells(const GridParams &g, int64_t n_b) {
    return (int64_t)g.res[0] * g.res[1] + 1 <= kCellBudget * n_b;
}

__global__ void rg_cells_kernel(const int64_t *__restrict__ ptr, int32_t B, const GridParams *__restrict__ gp,
                                const uint32_t *__restrict__ sorted_keys, int32_t *__restrict__ cell_start) {
    const int64_t t = kCellBudget * ptr[0] + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= kCellBudget * ptr[B]) return;
    int lo = 0, hi = B - 1;  // cloud whose table holds entry t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (kCellBudget * ptr[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    const int b = lo;
    const GridParams g = gp[b];
    const int64_t s0 = ptr[b], s1 = ptr[b + 1];
    const int64_t c = t - kCellBudget * s0;
    if (dense_cells(g, s1 - s0)) {
        if (c <= g.ncells) cell_start[t] = (int32_t)lower_bound_u32(sorted_keys, s0, s1, (uint32_t)c);
    } else if (column_cells(g, s1 - s0)) {
        if (c <= (int64_t)g.res[0] * g.res[1])
            cell_start[t] = (int32_t)lower_bound_u32(sorted_keys, s0, s1, (uint32_t)(c * g.res[2]));
    }
}

// One warp per query. Lanes 0-8 find the sorted ranges of the 9 z-columns of the 27-cell
// neighbourhood in the reference's (dx, dy) order (and, on grids with a dense cell table, where
// the query's own z-cell lies in each); the warp tests a column's candidates 32 at a time and
// ballot/popc append the sources in range to the query's padded row (rows are sorted at
// compaction). The reference keeps them all when at most `cap` are in range. Otherwise its heap
// keeps the `cap` smallest distances whenever the cap-th and the next are different, and the
// warp finds that cut in the same pass: the (distance, source) pairs in range also go to a shared
// buffer, and whenever the buffer has grown (or would overflow) a histogram of it yields a bound,
// the largest distance among its smallest >= cap pairs. No pair above the bound can be kept, so
// the buffer keeps the pairs at or below it, later candidates above it are dropped, and a column,
// or the outer z-cell of a column, whose cell box lies farther from the query than the bound (or
// than r, before there is a bound) is not scanned at all. The query's own column goes first,
// which makes the first bound tight. A radix select of the buffer gives the cap-th distance; a
// tie at the cut (or ties that fill the buffer) replays the reference heap on lane 0, fed in the
// reference's scan order.
constexpr int kQueryWarps = 8;
constexpr int kScanDepth = 4;  // candidate batches of 32 in flight per warp
constexpr int kOvfCap = 1024;  // candidates a warp can hold for the selection
constexpr int kHistBins = 256;
constexpr int kFlatMax = 256;  // queries with at most this many candidates load them as one list

struct QueryWarpSmem {
    float2 buf[kOvfCap];  // (distance, global index bits)
    int hist[kHistBins];
};

// The first bin at which the running count of the warp's histogram reaches `rank`, and the count
// before it (every lane returns both).
__device__ __forceinline__ int hist_rank_bin(const int *hist, int rank, int lane, int &before) {
    int v[kHistBins / 32], sum = 0;  // 8 consecutive bins per lane, warp scan
#pragma unroll
    for (int i = 0; i < kHistBins / 32; ++i) {
        v[i] = hist[lane * (kHistBins / 32) + i];
        sum += v[i];
    }
    int pre = sum;
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += y;
    }
    int run = pre - sum, found = -1, bef = 0;
#pragma unroll
    for (int i = 0; i < kHistBins / 32; ++i) {
        if (found < 0 && run + v[i] >= rank) {
            found = lane * (kHistBins / 32) + i;
            bef = run;
        }
        run += v[i];
    }
    const unsigned have = __ballot_sync(0xffffffffu, found >= 0);
    const int srcl = __ffs(have) - 1;  // lowest lane: the first bin reaching the rank
    before = __shfl_sync(0xffffffffu, bef, srcl);
    return __shfl_sync(0xffffffffu, found, srcl);
}

// Distances, in cell units, from a query at scaled coordinate u (cell qc = floor(u), the binning
// arithmetic of cell_coord) to the faces of its cell, less a rounding margin: a point binned into
// the cell below has u' < qc and one binned above has u' >= qc + 1, by the same arithmetic, whose
// relative error (three roundings) the margin covers many times over. The cell below is open to
// clamped points when the query's own cell lies past the grid (qc >= res): no bound then.
__device__ __forceinline__ void face_gaps(float u, int qc, int res, float &below, float &above) {
    const float eps = 0x1p-19f * (fabsf(u) + 2.0f);
    below = qc < res ? fmaxf(u - (float)qc - eps, 0.0f) : 0.0f;
    above = fmaxf((float)(qc + 1) - u - eps, 0.0f);
}

__global__ void __launch_bounds__(kQueryWarps * 32, 3) rg_query_warp_kernel(
    const int64_t *__restrict__ ptr, int32_t B, int64_t n, const uint8_t *__restrict__ mask,
    float r_sq, float inv, int loop, int cap, const GridParams *__restrict__ gp,
    const uint32_t *__restrict__ sorted_keys, const int32_t *__restrict__ cell_start,
    const float4 *__restrict__ sorted_pts, int32_t *__restrict__ counts, int32_t *__restrict__ padded) {
    // sorted_pts spans every cloud: a point's sorted position lies in its own cloud's range
    // (positions fit in int32: the host refuses n_points >= INT32_MAX / 64)
    extern __shared__ __align__(16) unsigned char query_smem[];  // kQueryWarps x QueryWarpSmem
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    QueryWarpSmem &W = reinterpret_cast<QueryWarpSmem *>(query_smem)[warp];
    const unsigned lt_mask = (1u << lane) - 1u;
    const int64_t nwarps = (int64_t)gridDim.x * kQueryWarps;
    const int64_t p0 = ptr[0], p1 = ptr[B];
    const int64_t gw = (int64_t)blockIdx.x * kQueryWarps + warp;
    // a box lower bound on a squared distance, scaled down by more than the rounding of dist2
    const float shrink = r_sq * (1.0f - 0x1p-19f);
    for (int64_t q = gw * 32 + lane; q < n; q += nwarps * 32)  // points outside every cloud
        if (q < p0 || q >= p1) counts[q] = 0;
    // queries in cell order (position j of the sorted points): warps running together share
    // most of their candidate columns in L1
    for (int64_t j = p0 + gw; j < p1; j += nwarps) {
        int kept = 0;
        const float4 qp = sorted_pts[j];  // the query's coordinates (copied from x) and index
        const int64_t q = __float_as_int(qp.w);
        const bool live = !(mask && !mask[q]);
        const int b = find_cloud_i(ptr, B, j);
        const GridParams g = gp[b];
        if (live && g.ok) {  // uniform over the warp
            const int64_t s0 = ptr[b], s1 = ptr[b + 1];
            const float qx = qp.x, qy = qp.y, qz = qp.z;
            const float ux = mul_ftz(sub_ftz(qx, g.mn[0]), inv), uy = mul_ftz(sub_ftz(qy, g.mn[1]), inv),
                        uz = mul_ftz(sub_ftz(qz, g.mn[2]), inv);
            const int qc0 = __float2int_rd(ux), qc1 = __float2int_rd(uy), qc2 = __float2int_rd(uz);  // cell_coord
            const int zlo = qc2 - 1 < 0 ? 0 : qc2 - 1;
            const int zhi = qc2 + 1 > g.res[2] - 1 ? g.res[2] - 1 : qc2 + 1;
            // lane c < 9: column c's sorted range [j0, j0 + len) and the query's z-cell within it,
            // [j0 + zm0, j0 + zm1) (the whole column when the grid has no dense cell table)
            int j0 = 0, len = 0, zm0 = 0, zm1 = 0;
            if (lane < 9) {
                const int cx = qc0 + lane / 3 - 1, cy = qc1 + lane % 3 - 1;
                if (zlo <= zhi && cx >= 0 && cx < g.res[0] && cy >= 0 && cy < g.res[1]) {
                    const int colc = (cx * g.res[1] + cy) * g.res[2];
                    int e;
                    if (dense_cells(g, s1 - s0)) {
                        const int32_t *cs = cell_start + kCellBudget * s0;
                        j0 = cs[colc + zlo];
                        e = cs[colc + zhi + 1];
                        if (zlo <= qc2 && qc2 <= zhi) {
                            zm0 = cs[colc + qc2] - j0;
                            zm1 = cs[colc + qc2 + 1] - j0;
                        } else {
                            zm1 = e - j0;
                        }
                    } else {
                        // the column's points (or the cloud's), then two independent searches
                        int64_t lo = s0, hi = s1;
                        if (column_cells(g, s1 - s0)) {
                            const int32_t *cs = cell_start + kCellBudget * s0;
                            const int col = cx * g.res[1] + cy;
                            lo = cs[col];
                            hi = cs[col + 1];
                        }
                        j0 = (int)lower_bound_u32(sorted_keys, lo, hi, (uint32_t)(colc + zlo));
                        e = (int)lower_bound_u32(sorted_keys, lo, hi, (uint32_t)(colc + zhi) + 1u);
                        zm1 = e - j0;
                    }
                    len = e - j0;
                }
            }
            float gxl, gxh, gyl, gyh, gzl, gzh;  // face gaps of the query's cell, cell units
            face_gaps(ux, qc0, g.res[0], gxl, gxh);
            face_gaps(uy, qc1, g.res[1], gyl, gyh);
            face_gaps(uz, qc2, g.res[2], gzl, gzh);
            int32_t *row = padded + q * cap;
            int m = 0;            // pairs in the buffer: every pair seen in range with d <= bound
            float bound = r_sq;   // in range is d < r_sq, so every such pair until the first bound
            bool bounded = false, replay = false;
            int next_tighten = 2 * cap;
            // keep the buffered pairs at or below the histogram bin where the running count
            // reaches cap; the bound becomes the largest distance kept (m >= cap on entry)
            auto tighten = [&]() {
                if (!(bound > 0x1p-100f)) {  // a zero bound: only ties remain, the heap decides
                    replay = true;
                    return;
                }
                const float scale = (float)kHistBins / bound;
                __syncwarp();
                for (int h = lane; h < kHistBins; h += 32) W.hist[h] = 0;
                __syncwarp();
                for (int i = lane; i < m; i += 32)
                    atomicAdd(&W.hist[min((int)(W.buf[i].x * scale), kHistBins - 1)], 1);
                __syncwarp();
                int before;
                const int cut = hist_rank_bin(W.hist, cap, lane, before);
                int w = 0;
                float top = 0.0f;
                for (int base = 0; base < m; base += 32) {
                    const int i = base + lane;
                    const float2 e = i < m ? W.buf[i] : make_float2(0.0f, 0.0f);
                    const bool keep = i < m && min((int)(e.x * scale), kHistBins - 1) <= cut;
                    const unsigned kh = __ballot_sync(0xffffffffu, keep);  // reads of the batch done
                    if (keep) {
                        W.buf[w + __popc(kh & lt_mask)] = e;  // position <= i
                        top = fmaxf(top, e.x);
                    }
                    w += __popc(kh);
                    __syncwarp();
                }
                for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
                m = w;
                bound = top;
                bounded = true;
                next_tighten = 2 * (m > cap ? m : cap);
            };
            // one batch of candidates: test them, append the sources in range to the row while at
            // most cap are, and the pairs at or below the bound to the buffer (room checked before)
            auto consume = [&](const float4 &sp, bool have) {
                bool ok = false;
                float d = 0.0f;
                int o = 0;
                if (have) {
                    o = __float_as_int(sp.w);
                    d = dist2(qx, qy, qz, sp.x, sp.y, sp.z);
                    ok = (loop || (int64_t)o != q) && d < r_sq;
                }
                const unsigned hits = __ballot_sync(0xffffffffu, ok);
                const int pos = kept + __popc(hits & lt_mask);
                if (ok && pos < cap) row[pos] = o;
                kept += __popc(hits);
                const bool put = ok && d <= bound;
                const unsigned ph = bounded ? __ballot_sync(0xffffffffu, put) : hits;
                if (put) W.buf[m + __popc(ph & lt_mask)] = make_float2(d, __int_as_float(o));
                m += __popc(ph);
            };
            // candidates of all 9 columns as one list (inclusive prefix of the lengths on lanes 0-8)
            int incl = len;
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int total = __shfl_sync(0xffffffffu, incl, 8);
            if (total <= kFlatMax) {
                // few candidates: load them all at once instead of column after column (the buffer
                // holds every pair in range, no bound needed)
                const int lbase = j0 - (incl - len);  // sorted position of list entry t, column lane
                int ends[9];
#pragma unroll
                for (int c = 0; c < 9; ++c) ends[c] = __shfl_sync(0xffffffffu, incl, c);
                for (int t0 = 0; t0 < total; t0 += 32 * kScanDepth) {
                    float4 sp[kScanDepth];
#pragma unroll
                    for (int u = 0; u < kScanDepth; ++u) {
                        const int t = t0 + 32 * u + lane;
                        int col = 0;
#pragma unroll
                        for (int c = 0; c < 8; ++c) col += t >= ends[c];
                        const int at = __shfl_sync(0xffffffffu, lbase, col) + t;
                        if (t < total) sp[u] = sorted_pts[at];
                    }
#pragma unroll
                    for (int u = 0; u < kScanDepth; ++u) {
                        if (t0 + 32 * u >= total) break;  // uniform over the warp
                        consume(sp[u], t0 + 32 * u + lane < total);
                    }
                }
            } else {
                // columns: the query's own first, then the rest; once the heap replay is decided
                // the scan stops (the replay rescans every column)
                for (int ci = 0; ci < 9 && !replay; ++ci) {
                    if (m >= next_tighten) tighten();  // m >= 2 cap: the row is over the cap
                    const int c = ci == 0 ? 4 : (ci <= 4 ? ci - 1 : ci);
                    const int cb = __shfl_sync(0xffffffffu, j0, c);
                    const int cl = __shfl_sync(0xffffffffu, len, c);
                    const int z0 = __shfl_sync(0xffffffffu, zm0, c), z1 = __shfl_sync(0xffffffffu, zm1, c);
                    const int cxo = c / 3, cyo = c - 3 * cxo;
                    const float gx = cxo == 0 ? gxl : (cxo == 2 ? gxh : 0.0f);
                    const float gy = cyo == 0 ? gyl : (cyo == 2 ? gyh : 0.0f);
                    const float gxy = gx * gx + gy * gy;
                    if (replay || cl == 0 || gxy * shrink > bound) continue;  // uniform: nothing to keep
                    const int a = (gxy + gzl * gzl) * shrink > bound ? z0 : 0;   // the z-cell below
                    const int e = (gxy + gzh * gzh) * shrink > bound ? z1 : cl;  // the z-cell above
                    for (int k0 = a; k0 < e; k0 += 32 * kScanDepth) {
                        if (m > kOvfCap - 32 * kScanDepth) {  // room for the batches below
                            tighten();
                            if (m > kOvfCap - 32 * kScanDepth) replay = true;  // ties fill the buffer
                            if (replay) break;
                        }
                        float4 sp[kScanDepth];
#pragma unroll
                        for (int u = 0; u < kScanDepth; ++u) {
                            const int k = k0 + 32 * u + lane;
                            if (k < e) sp[u] = sorted_pts[cb + k];
                        }
#pragma unroll
                        for (int u = 0; u < kScanDepth; ++u) {
                            if (k0 + 32 * u >= e) break;  // uniform over the warp
                            consume(sp[u], k0 + 32 * u + lane < e);
                        }
                    }
                }
            }
            if (kept > cap) {
                __syncwarp();
                if (!replay) {
                    // radix select of the cap-th smallest distance (rank cap, 1-based), 8 bits a
                    // pass, over the buffer: every pair in range at or below the bound, m >= cap
                    uint32_t prefix = 0, pmask = 0;
                    int rank = cap;  // rank within the candidates matching the prefix
                    for (int shift = 24; shift >= 0; shift -= 8) {
                        for (int h = lane; h < kHistBins; h += 32) W.hist[h] = 0;
                        __syncwarp();
                        for (int i = lane; i < m; i += 32) {
                            const uint32_t u = __float_as_uint(W.buf[i].x);
                            if ((u & pmask) == prefix) atomicAdd(&W.hist[(u >> shift) & 255u], 1);
                        }
                        __syncwarp();
                        int before;
                        const int digit = hist_rank_bin(W.hist, rank, lane, before);
                        rank -= before;
                        prefix |= (uint32_t)digit << shift;
                        pmask |= 255u << shift;
                        __syncwarp();
                    }
                    const float vcap = __uint_as_float(prefix);  // the cap-th smallest distance
                    // the kept set is {d <= vcap} when exactly cap candidates qualify
                    int le = 0;
                    for (int i = lane; i < m; i += 32) le += W.buf[i].x <= vcap;
                    for (int o = 16; o > 0; o >>= 1) le += __shfl_xor_sync(0xffffffffu, le, o);
                    if (le != cap) {
                        replay = true;  // tie at the cut: the scan order decides
                    } else {
                        int w = 0;
                        for (int base = 0; base < m; base += 32) {
                            const int i = base + lane;
                            const bool ok = i < m && W.buf[i].x <= vcap;
                            const unsigned hits = __ballot_sync(0xffffffffu, ok);
                            if (ok) row[w + __popc(hits & lt_mask)] = __float_as_int(W.buf[i].y);
                            w += __popc(hits);
                        }
                    }
                    __syncwarp();
                }
                if (replay) {  // the reference heap, fed in its scan order, on lane 0
                    int clen[9], cbeg[9];
#pragma unroll
                    for (int c = 0; c < 9; ++c) {
                        clen[c] = __shfl_sync(0xffffffffu, len, c);
                        cbeg[c] = __shfl_sync(0xffffffffu, j0, c);
                    }
                    if (lane == 0) {
                        float hd[64];
                        int hid[64];
                        int hc = 0;
#pragma unroll
                        for (int c = 0; c < 9; ++c)
                            for (int k = 0; k < clen[c]; ++k) {
                                const float4 sp = sorted_pts[cbeg[c] + k];
                                const int o = __float_as_int(sp.w);
                                if (!loop && (int64_t)o == q) continue;
                                const float d = dist2(qx, qy, qz, sp.x, sp.y, sp.z);
                                if (d < r_sq) heap_add(hd, hid, hc, cap, d, o);
                            }
                        for (int a2 = 0; a2 < hc; ++a2) row[a2] = hid[a2];
                    }
                    __syncwarp();
                }
                kept = cap;
            }
        }
        if (lane == 0) counts[q] = kept;
    }
}

// row_ptr from the exclusive scan of counts; one warp sorts each row ascending and writes it
__global__ void rg_compact_sort_kernel(const int32_t *__restrict__ counts, const int32_t *__restrict__ padded,
                                       int64_t n, int cap, const int64_t *__restrict__ row_ptr,
                                       int64_t *__restrict__ src, int64_t *__restrict__ dst,
                                       int32_t *__restrict__ row_ptr32, int32_t *__restrict__ src32,
                                       const EdgeGeom geom) {
    extern __shared__ float geo_stage[];  // (blockDim.x / 32) * kGeomStageFloats when geometry is written
    const int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (q > n) return;  // uniform over the warp
    if (row_ptr32 && lane == 0) row_ptr32[q] = (int32_t)row_ptr[q];
    if (q == n) return;
    warp_sort_emit(padded + q * cap, 1, counts[q], row_ptr[q], q, src, dst, src32, geom,
                   geo_stage + (threadIdx.x >> 5) * kGeomStageFloats);
}

struct RadiusWs {
    GridParams *gp;
    int32_t *key_bits;
    uint32_t *keys, *sorted_keys;
    int32_t *sorted_idx, *counts, *padded;
    float4 *sorted_pts;
    int32_t *cell_start;
    int64_t *scan_scratch;
    int32_t *cloud_tot;
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
    t.cell_start = (int32_t *)take(sizeof(int32_t) * kCellBudget * nn);
    t.scan_scratch = (int64_t *)take(sizeof(int64_t) * (scan_blocks(nn) + 1));
    t.cloud_tot = (int32_t *)take(sizeof(int32_t) * (B > 0 ? B : 1));
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

extern "C" int gdl_radius_graph_geometry(const float *x, const int64_t *ptr, int32_t num_clouds, int64_t n_points,
                                         int64_t max_cloud_points, double radius, int32_t max_num_neighbors,
                                         int32_t loop, const uint8_t *mask, int64_t *out_row_ptr, int64_t *out_src,
                                         int64_t *out_dst, int32_t *out_row_ptr32, int32_t *out_src32,
                                         const gdl_edge_geometry *geometry, void *workspace, size_t workspace_bytes,
                                         void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || n_points < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(!out_row_ptr, GDL_ERR_INVALID);
    GDL_RETURN_IF(!edge_geom_valid(geometry), GDL_ERR_INVALID);
    const EdgeGeom geom = edge_geom_from(x, geometry);
    GDL_RETURN_IF(n_points >= INT32_MAX / 64, GDL_ERR_OVERFLOW);
    const float r = (float)radius;  // radius_graph_kernel.cu:266
    if (n_points == 0 || num_clouds == 0 || !(r > 0.0f)) {
        GDL_CUDA_TRY(cudaMemsetAsync(out_row_ptr, 0, sizeof(int64_t) * (n_points + 1), st));
        if (out_row_ptr32) GDL_CUDA_TRY(cudaMemsetAsync(out_row_ptr32, 0, sizeof(int32_t) * (n_points + 1), st));
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
    if (max_cloud_points > 0 && max_cloud_points <= kSmallMax) {  // fused per-cloud path
        const size_t smem = sizeof(SmallSmem);
        // spread each cloud over several CTAs so that small batches still fill the GPU
        int split = (int)((2 * kSmCount) / num_clouds);
        split = split < 1 ? 1 : (split > 8 ? 8 : split);
        GDL_CUDA_TRY(cudaFuncSetAttribute(rg_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        GDL_CUDA_TRY(cudaMemsetAsync(w.cloud_tot, 0, sizeof(int32_t) * num_clouds, st));
        rg_small_kernel<<<num_clouds * split, kSmallThreads, smem, st>>>(x, ptr, mask, r_sq, inv, loop, cap, split,
                                                                         n_points, w.counts, w.padded, w.cloud_tot);
        const size_t geo_smem = geom.x ? sizeof(float) * kGeomStageFloats * kSmallWarps : 0;
        if (geo_smem)
            GDL_CUDA_TRY(cudaFuncSetAttribute(rg_small_compact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)geo_smem));
        rg_small_compact_kernel<<<num_clouds * split, kSmallThreads, geo_smem, st>>>(
            ptr, num_clouds, split, n_points, cap, w.counts, w.padded, w.cloud_tot, out_row_ptr, out_src, out_dst,
            out_row_ptr32, out_src32, geom);
        GDL_CUDA_TRY(cudaGetLastError());
        return GDL_OK;
    }
    const unsigned g256 = (unsigned)((n_points + 255) / 256);
    GDL_CUDA_TRY(cudaMemsetAsync(w.key_bits, 0, sizeof(int32_t), st));
    rg_grid_kernel<<<num_clouds, kGridThreads, 0, st>>>(x, ptr, inv, w.gp, w.key_bits);
    rg_keys_kernel<<<g256, 256, 0, st>>>(x, ptr, num_clouds, mask, inv, w.gp, w.keys);
    GDL_CUDA_TRY(radix_sort_pairs(w.keys, nullptr, w.sorted_keys, w.sorted_idx, n_points, ptr, num_clouds, 4,
                                  w.key_bits, w.rs, st));
    rg_gather_kernel<<<g256, 256, 0, st>>>(x, ptr, num_clouds, w.sorted_idx, w.sorted_pts);
    rg_cells_kernel<<<(unsigned)((kCellBudget * n_points + 255) / 256), 256, 0, st>>>(ptr, num_clouds, w.gp,
                                                                                    w.sorted_keys, w.cell_start);
    const int64_t qblocks = (n_points + kQueryWarps - 1) / kQueryWarps;
    const unsigned qgrid = (unsigned)(qblocks < 32 * kSmCount ? qblocks : 32 * kSmCount);
    const size_t qsmem = sizeof(QueryWarpSmem) * kQueryWarps;
    GDL_CUDA_TRY(cudaFuncSetAttribute(rg_query_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsmem));
    rg_query_warp_kernel<<<qgrid, kQueryWarps * 32, qsmem, st>>>(ptr, num_clouds, n_points, mask, r_sq, inv, loop, cap,
                                                             w.gp, w.sorted_keys, w.cell_start, w.sorted_pts,
                                                             w.counts, w.padded);
    GDL_CUDA_TRY((exclusive_scan<int32_t, int64_t>(w.counts, out_row_ptr, n_points, w.scan_scratch,
                                                   out_row_ptr + n_points, st)));
    const size_t geo_smem = geom.x ? sizeof(float) * kGeomStageFloats * (256 / 32) : 0;
    rg_compact_sort_kernel<<<(unsigned)(((n_points + 1) * 32 + 255) / 256), 256, geo_smem, st>>>(
        w.counts, w.padded, n_points, cap, out_row_ptr, out_src, out_dst, out_row_ptr32, out_src32, geom);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_radius_graph(const float *x, const int64_t *ptr, int32_t num_clouds, int64_t n_points,
                                int64_t max_cloud_points, double radius, int32_t max_num_neighbors, int32_t loop,
                                const uint8_t *mask, int64_t *out_row_ptr, int64_t *out_src, int64_t *out_dst,
                                int32_t *out_row_ptr32, int32_t *out_src32, void *workspace, size_t workspace_bytes,
                                void *stream) {
    return gdl_radius_graph_geometry(x, ptr, num_clouds, n_points, max_cloud_points, radius, max_num_neighbors, loop,
                                     mask, out_row_ptr, out_src, out_dst, out_row_ptr32, out_src32, nullptr,
                                     workspace, workspace_bytes, stream);
}
