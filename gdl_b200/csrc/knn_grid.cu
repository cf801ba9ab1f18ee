// knn_grid.cu -- exact KNN for large clouds over a uniform grid of the sources (sm_100a).
//
// Reference semantics: knn_kernel.cu:113-291 (see knn.cu). Whenever a query's k_eff + 1
// nearest distances are pairwise different, the reference's output is "the k_eff nearest,
// ascending", whatever order the sources are visited in. So for clouds of many points the
// sources of each cloud are bucketed into a uniform grid, and each query examines cells in
// growing shells around its own until the (k_eff+1)-th nearest distance found is provably below
// the distance to every unexamined cell. The result is exact: queries with equal distances
// among their k_eff + 1 nearest, with non-finite coordinates, or whose search runs out of room
// are handed to knn.cu's replay of the reference heap.
//
// Grid per cloud (one CTA): bbox; cell size h0 from the mean density (t points per cell, t
// growing with k); the occupancy a point actually sees at h0 (sum of squared cell counts / n)
// corrects h for clustered clouds; at most kKgCellBudget cells per point and 1024 per axis.
// Sources are radix-sorted by cell (stable), gathered as float4 (.w = local index), and a dense
// table gives each cell's [first, one-past-last) sorted position within its cloud.
//
// Query (one warp): shell s = 1 is the 3x3x3 block around the query's (clamped) cell; shell
// s > 1 adds the cells at Chebyshev distance s. A cell column's z-run is one contiguous sorted
// range. Candidates at or below the current (k_eff+1)-th distance T are appended to a shared
// buffer; when it fills, a radix select finds T and the buffer keeps d <= T. After each shell,
// the search stops once T (1 + 1e-5) < (b - delta)^2, b = the distance from the query to the
// nearest face of the examined block that is not the grid's edge, delta = the coordinate slack of
// cell assignment. The k_eff + 1 nearest are then sorted by a warp bitonic sort.
#include "knn_grid.cuh"

namespace gdl {

constexpr int kKgGridThreads = 1024;
constexpr int kKgWarps = 8;
constexpr int kKgBuf = 1024;
constexpr int kKgBins = 256;
constexpr int kKgMaxShell = 12;  // farther than this: the query goes to the exact replay

struct KgWarpSmem {
    float2 buf[kKgBuf];  // (distance, local source index bits)
    int hist[kKgBins];
};

static __device__ __forceinline__ int kg_find(const int64_t *__restrict__ p, int B, int64_t j) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p[mid] <= j) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

static __device__ __forceinline__ int kg_cell(float p, float mn, float inv, int res) {
    const int v = __float2int_rd(mul_ftz(sub_ftz(p, mn), inv));
    return v < 0 ? 0 : (v > res - 1 ? res - 1 : v);
}

// Local source offsets. If the sources outnumber the capacity the workspace was sized for (a
// max_cloud_sources below the true maximum), every offset is 0 -- nothing is sorted or written --
// and `invalid` sends every query to the exact replay, which does not depend on that capacity.
static __global__ void kg_lptr_kernel(const int64_t *__restrict__ ptr_s, int32_t B, int64_t nmax,
                                      int64_t *__restrict__ lptr, int32_t *__restrict__ invalid) {
    const bool bad = ptr_s[B] - ptr_s[0] > nmax || ptr_s[B] < ptr_s[0];
    for (int b = threadIdx.x; b <= B; b += blockDim.x) lptr[b] = bad ? 0 : ptr_s[b] - ptr_s[0];
    if (threadIdx.x == 0) *invalid = bad ? 1 : 0;
}

// grid resolution for cell size h within the budget; returns the cell count
static __device__ int64_t kg_resolve(const float *eff, int64_t n, float &h, int *res) {
    for (int it = 0; it < 64; ++it) {
        int64_t cells = 1;
        for (int a = 0; a < 3; ++a) {
            const float c = ceilf(eff[a] / h);
            res[a] = c >= 1024.0f ? 1024 : (c < 1.0f ? 1 : (int)c);
            cells *= res[a];
        }
        if (cells <= (int64_t)kKgCellBudget * n) return cells;
        h *= 1.25f;
    }
    res[0] = res[1] = res[2] = 1;
    return 1;
}

static __global__ void __launch_bounds__(kKgGridThreads) kg_grid_kernel(
    const float *__restrict__ src, const int64_t *__restrict__ ptr_s, const int64_t *__restrict__ lptr, int32_t B,
    int k, int32_t *__restrict__ scratch, KGrid *__restrict__ grids, int32_t *__restrict__ key_bits) {
    __shared__ float red[6][kKgGridThreads / 32];
    __shared__ unsigned long long sq[kKgGridThreads / 32];
    __shared__ int bad_s;
    __shared__ KGrid g0;
    __shared__ int64_t cells0_s;
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t base = ptr_s[0], s0 = lptr[b], s1 = lptr[b + 1], n = s1 - s0;
    if (n <= 0) {  // uniform over the CTA
        if (tid == 0) {
            KGrid g = {};
            g.ok = 0;
            grids[b] = g;
        }
        return;
    }
    if (tid == 0) bad_s = 0;
    float lo[3], hi[3];
    for (int a = 0; a < 3; ++a) {
        lo[a] = __int_as_float(0x7f800000);
        hi[a] = __int_as_float(0xff800000);
    }
    bool bad = false;
    for (int64_t i = s0 + tid; i < s1; i += kKgGridThreads)
        for (int a = 0; a < 3; ++a) {
            const float v = src[3 * (base + i) + a];
            bad |= !isfinite(v);
            lo[a] = fminf(lo[a], v);
            hi[a] = fmaxf(hi[a], v);
        }
    for (int a = 0; a < 3; ++a)
        for (int o = 16; o > 0; o >>= 1) {
            lo[a] = fminf(lo[a], __shfl_xor_sync(0xffffffffu, lo[a], o));
            hi[a] = fmaxf(hi[a], __shfl_xor_sync(0xffffffffu, hi[a], o));
        }
    if (lane == 0)
        for (int a = 0; a < 3; ++a) {
            red[a][warp] = lo[a];
            red[3 + a][warp] = hi[a];
        }
    __syncthreads();
    if (bad) bad_s = 1;
    if (tid == 0) {
        float l[3], h3[3], eff[3], maxe = 0.0f, maxabs = 0.0f;
        for (int a = 0; a < 3; ++a) {
            l[a] = red[a][0];
            h3[a] = red[3 + a][0];
            for (int w = 1; w < kKgGridThreads / 32; ++w) {
                l[a] = fminf(l[a], red[a][w]);
                h3[a] = fmaxf(h3[a], red[3 + a][w]);
            }
            maxe = fmaxf(maxe, h3[a] - l[a]);
            maxabs = fmaxf(maxabs, fmaxf(fabsf(l[a]), fabsf(h3[a])));
        }
        for (int a = 0; a < 3; ++a) eff[a] = fmaxf(fmaxf(h3[a] - l[a], 1e-3f * maxe), 1e-30f);
        const int ke = k < 64 ? k : 64;
        const float t = fmaxf(4.0f, 0.5f * (float)(ke + 1));  // target points per cell
        float h = maxe > 0.0f ? cbrtf(eff[0] * eff[1] * eff[2] * t / (float)n) : 1.0f;
        if (!(h > 0.0f) || !isfinite(h)) h = fmaxf(maxe, 1.0f);
        KGrid g = {};
        for (int a = 0; a < 3; ++a) g.mn[a] = l[a];
        cells0_s = kg_resolve(eff, n, h, g.res);
        g.h = h;
        g.inv = 1.0f / h;
        g.delta = 1e-5f * (maxabs + maxe + h);
        g.ok = 1;
        g0 = g;
    }
    __syncthreads();
    if (bad_s) {
        if (tid == 0) {
            KGrid g = g0;
            g.ok = -1;
            grids[b] = g;
        }
        return;
    }
    // occupancy a point sees at h0: sum over cells of count^2 / n
    const KGrid g = g0;
    const int64_t cells0 = cells0_s;
    int32_t *cnt = scratch + (int64_t)kKgCellBudget * s0;
    for (int64_t c = tid; c < cells0; c += kKgGridThreads) cnt[c] = 0;
    __syncthreads();
    for (int64_t i = s0 + tid; i < s1; i += kKgGridThreads) {
        const float *p = src + 3 * (base + i);
        const int cx = kg_cell(p[0], g.mn[0], g.inv, g.res[0]), cy = kg_cell(p[1], g.mn[1], g.inv, g.res[1]),
                  cz = kg_cell(p[2], g.mn[2], g.inv, g.res[2]);
        atomicAdd(&cnt[((int64_t)cx * g.res[1] + cy) * g.res[2] + cz], 1);
    }
    __syncthreads();
    unsigned long long acc = 0;
    for (int64_t c = tid; c < cells0; c += kKgGridThreads) {
        const unsigned long long v = (unsigned)cnt[c];
        acc += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sq[warp] = acc;
    __syncthreads();
    if (tid == 0) {
        unsigned long long s = 0;
        for (int w = 0; w < kKgGridThreads / 32; ++w) s += sq[w];
        const float occ = (float)((double)s / (double)n);
        const int ke = k < 64 ? k : 64;
        const float t = fmaxf(4.0f, 0.5f * (float)(ke + 1));
        KGrid gf = g;
        float h = g.h;
        if (occ > t) {  // clustered: shrink the cells toward t points seen per point
            float eff[3], maxe = 0.0f;
            for (int a = 0; a < 3; ++a) maxe = fmaxf(maxe, (float)g.res[a] * g.h);
            for (int a = 0; a < 3; ++a) eff[a] = fmaxf((float)g.res[a] * g.h, 1e-3f * maxe);
            h = g.h * cbrtf(t / occ);
            const int64_t cells = kg_resolve(eff, n, h, gf.res);
            (void)cells;
            gf.h = h;
            gf.inv = 1.0f / h;
            gf.delta = fmaxf(g.delta, 1e-5f * h);
        }
        grids[b] = gf;
        int64_t cells = (int64_t)gf.res[0] * gf.res[1] * gf.res[2];
        int bits = 0;
        while (bits < 31 && ((int64_t)1 << bits) < cells) ++bits;
        atomicMax(key_bits, bits);
    }
}

static __global__ void kg_keys_kernel(const float *__restrict__ src, const int64_t *__restrict__ ptr_s,
                                      const int64_t *__restrict__ lptr, int32_t B, const KGrid *__restrict__ grids,
                                      uint32_t *__restrict__ keys) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= lptr[B]) return;
    const KGrid g = grids[kg_find(lptr, B, j)];
    uint32_t key = 0;
    if (g.ok == 1) {
        const float *p = src + 3 * (ptr_s[0] + j);
        const int cx = kg_cell(p[0], g.mn[0], g.inv, g.res[0]), cy = kg_cell(p[1], g.mn[1], g.inv, g.res[1]),
                  cz = kg_cell(p[2], g.mn[2], g.inv, g.res[2]);
        key = (uint32_t)(((int64_t)cx * g.res[1] + cy) * g.res[2] + cz);
    }
    keys[j] = key;
}

static __global__ void kg_gather_kernel(const float *__restrict__ src, const int64_t *__restrict__ ptr_s,
                                        const int64_t *__restrict__ lptr, int32_t B,
                                        const int32_t *__restrict__ sorted_idx, float4 *__restrict__ pts) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= lptr[B]) return;
    const int32_t o = sorted_idx[j];
    const float *p = src + 3 * (ptr_s[0] + o);
    pts[j] = make_float4(p[0], p[1], p[2], __int_as_float(o));
}

static __global__ void kg_cells_kernel(const int64_t *__restrict__ lptr, int32_t B, const KGrid *__restrict__ grids,
                                       const uint32_t *__restrict__ skeys, int2 *__restrict__ cells) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= lptr[B]) return;
    const int b = kg_find(lptr, B, j);
    if (grids[b].ok != 1) return;
    const int64_t c0 = lptr[b], c1 = lptr[b + 1];
    const uint32_t key = skeys[j];
    int2 *tab = cells + (int64_t)kKgCellBudget * c0;
    // positions relative to the cloud's first sorted source
    if (j == c0 || skeys[j - 1] != key) tab[key].x = (int)(j - c0);
    if (j == c1 - 1 || skeys[j + 1] != key) tab[key].y = (int)(j - c0) + 1;
}

// rank-th smallest (1-based) of buf[0, m).x; the values are >= 0 or +inf, so their bit patterns
// order like the values. Radix select, 8 bits a pass, histogram in shared memory.
static __device__ float kg_kth(const float2 *buf, int m, int rank, int *hist, int lane) {
    uint32_t prefix = 0, pmask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int h = lane; h < kKgBins; h += 32) hist[h] = 0;
        __syncwarp();
        for (int i = lane; i < m; i += 32) {
            const uint32_t u = __float_as_uint(buf[i].x);
            if ((u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
        }
        __syncwarp();
        int v[kKgBins / 32], sum = 0;
#pragma unroll
        for (int i = 0; i < kKgBins / 32; ++i) {
            v[i] = hist[lane * (kKgBins / 32) + i];
            sum += v[i];
        }
        int pre = sum;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, pre, o);
            if (lane >= o) pre += y;
        }
        int run = pre - sum, found = -1, before = 0;
#pragma unroll
        for (int i = 0; i < kKgBins / 32; ++i) {
            if (found < 0 && run + v[i] >= rank) {
                found = lane * (kKgBins / 32) + i;
                before = run;
            }
            run += v[i];
        }
        const unsigned have = __ballot_sync(0xffffffffu, found >= 0);
        const int srcl = have ? __ffs(have) - 1 : 0;
        const int digit = __shfl_sync(0xffffffffu, found, srcl);
        rank -= __shfl_sync(0xffffffffu, before, srcl);
        prefix |= (uint32_t)(digit & 255) << shift;
        pmask |= 255u << shift;
        __syncwarp();
    }
    return __uint_as_float(prefix);
}

// keep buf entries with distance <= v, in place (every lane reads before any lane writes)
static __device__ int kg_compact(float2 *buf, int m, float v, int lane) {
    const unsigned lt = (1u << lane) - 1u;
    int w = 0;
    for (int base = 0; base < m; base += 32) {
        const int i = base + lane;
        float2 e = make_float2(0.0f, 0.0f);
        bool keep = false;
        if (i < m) {
            e = buf[i];
            keep = e.x <= v;
        }
        __syncwarp();
        const unsigned hb = __ballot_sync(0xffffffffu, keep);
        if (keep) buf[w + __popc(hb & lt)] = e;
        w += __popc(hb);
        __syncwarp();
    }
    return w;
}

// ascending bitonic sort of 128 keys, element r * 32 + lane in a[r]
static __device__ __forceinline__ void kg_sort128(uint64_t (&a)[4], int lane) {
#pragma unroll
    for (int size = 2; size <= 128; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int rs = stride >> 5;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int pr = r ^ rs;
                    if (pr > r) {
                        const bool up = ((r * 32 + lane) & size) == 0;
                        const uint64_t x = a[r], y = a[pr];
                        const uint64_t mn = x < y ? x : y, mx = x < y ? y : x;
                        a[r] = up ? mn : mx;
                        a[pr] = up ? mx : mn;
                    }
                }
            } else {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int e = r * 32 + lane;
                    const uint64_t p = __shfl_xor_sync(0xffffffffu, a[r], stride);
                    const bool up = (e & size) == 0, lower = (e & stride) == 0;
                    a[r] = (lower == up) ? (a[r] < p ? a[r] : p) : (a[r] < p ? p : a[r]);
                }
            }
        }
    }
}

static __global__ void __launch_bounds__(kKgWarps * 32) kg_query_kernel(
    const float *__restrict__ query, const int64_t *__restrict__ ptr_q, int32_t B, const int64_t *__restrict__ ptr_s,
    const int64_t *__restrict__ lptr, const KGrid *__restrict__ grids, const float4 *__restrict__ pts,
    const int2 *__restrict__ cells, int k, const int32_t *__restrict__ invalid, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count) {
    extern __shared__ __align__(16) unsigned char kg_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    KgWarpSmem &W = reinterpret_cast<KgWarpSmem *>(kg_smem)[warp];
    const unsigned lt = (1u << lane) - 1u;
    const int ke = k < 64 ? k : 64;
    const int64_t q0 = ptr_q[0], q1 = ptr_q[B], sbase = ptr_s[0];
    const int64_t nw = (int64_t)gridDim.x * kKgWarps;
    const float kInf = __int_as_float(0x7f800000);
    for (int64_t q = q0 + (int64_t)blockIdx.x * kKgWarps + warp; q < q1; q += nw) {
        if (*invalid) {  // sources beyond the workspace's capacity: exact replay of every query
            if (lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
            continue;
        }
        const int b = kg_find(ptr_q, B, q);
        const KGrid g = grids[b];
        const int64_t s0 = lptr[b], nb = lptr[b + 1] - s0;
        int64_t *oi = out_idx + q * k;
        float *od = out_dist + q * k;
        if (nb <= 0) {  // no sources: padding only (the reference's empty heap)
            for (int j = lane; j < k; j += 32) {
                oi[j] = -1;
                od[j] = 1e30f;
            }
            continue;
        }
        const float qp[3] = {query[3 * q], query[3 * q + 1], query[3 * q + 2]};
        bool flag = g.ok != 1 || !(isfinite(qp[0]) && isfinite(qp[1]) && isfinite(qp[2]));
        const int K1 = (int)(ke + 1 < nb ? ke + 1 : nb);
        int m = 0;
        float T = kInf;
        if (!flag) {
            int qc[3];
            for (int a = 0; a < 3; ++a) qc[a] = kg_cell(qp[a], g.mn[a], g.inv, g.res[a]);
            const int2 *tab = cells + (int64_t)kKgCellBudget * s0;
            bool done = false;
            for (int s = 1; !done; ++s) {
                if (s > kKgMaxShell) {
                    flag = true;
                    break;
                }
                const int side = 2 * s + 1, npairs = side * side;
                for (int p0 = 0; p0 < npairs && !flag; p0 += 32) {
                    const int p = p0 + lane;
                    int ra0 = 0, re0 = 0, ra1 = 0, re1 = 0;  // two sorted ranges [ra, re)
                    if (p < npairs) {
                        const int dx = p / side - s, dy = p % side - s;
                        const int cx = qc[0] + dx, cy = qc[1] + dy;
                        if (cx >= 0 && cx < g.res[0] && cy >= 0 && cy < g.res[1]) {
                            const int64_t col = ((int64_t)cx * g.res[1] + cy) * g.res[2];
                            // z-run [z0, z1] of cells: one contiguous sorted range
                            auto run = [&](int z0, int z1, int &a, int &e) {
                                z0 = z0 < 0 ? 0 : z0;
                                z1 = z1 > g.res[2] - 1 ? g.res[2] - 1 : z1;
                                for (int z = z0; z <= z1; ++z) {
                                    const int2 c = tab[col + z];
                                    if (c.y > c.x) {
                                        if (e == 0) a = c.x;
                                        e = c.y;
                                    }
                                }
                            };
                            if (s == 1 || max(abs(dx), abs(dy)) == s) {
                                run(qc[2] - s, qc[2] + s, ra0, re0);
                            } else {  // interior column of the shell: its two end cells
                                run(qc[2] - s, qc[2] - s, ra0, re0);
                                run(qc[2] + s, qc[2] + s, ra1, re1);
                            }
                        }
                    }
                    // candidates of every non-empty range, 32 at a time
                    auto take = [&](int ra, int re) {
                        unsigned busy = __ballot_sync(0xffffffffu, re > ra);
                        while (busy && !flag) {
                            const int l = __ffs(busy) - 1;
                            busy &= busy - 1;
                            const int a = __shfl_sync(0xffffffffu, ra, l), e = __shfl_sync(0xffffffffu, re, l);
                            for (int j0 = a; j0 < e; j0 += 32) {
                                const int j = j0 + lane;
                                bool acc = false;
                                float d = 0.0f;
                                int o = 0;
                                if (j < e) {
                                    const float4 sp = pts[s0 + j];
                                    o = __float_as_int(sp.w);
                                    d = dist2(qp[0], qp[1], qp[2], sp.x, sp.y, sp.z);
                                    acc = d <= T;
                                }
                                const unsigned hb = __ballot_sync(0xffffffffu, acc);
                                if (acc) W.buf[m + __popc(hb & lt)] = make_float2(d, __int_as_float(o));
                                m += __popc(hb);
                                if (m > kKgBuf - 32) {  // keep the K1 nearest (and their ties)
                                    __syncwarp();
                                    T = kg_kth(W.buf, m, K1, W.hist, lane);
                                    m = kg_compact(W.buf, m, T, lane);
                                    if (m > kKgBuf - 64) {  // a mass of equal distances: give up
                                        flag = true;
                                        break;
                                    }
                                }
                            }
                        }
                    };
                    take(ra0, re0);
                    if (!flag) take(ra1, re1);
                }
                if (flag) break;
                __syncwarp();
                if (m >= K1) T = kg_kth(W.buf, m, K1, W.hist, lane);
                // pruning bound: distance to the nearest face of the examined block that is not
                // the grid's edge (points lie inside the grid, the edge cells are open-ended)
                float bound = kInf;
                bool covered = true;
                for (int a = 0; a < 3; ++a) {
                    if (qc[a] - s > 0) {
                        covered = false;
                        bound = fminf(bound, qp[a] - (g.mn[a] + (float)(qc[a] - s) * g.h));
                    }
                    if (qc[a] + s < g.res[a] - 1) {
                        covered = false;
                        bound = fminf(bound, (g.mn[a] + (float)(qc[a] + s + 1) * g.h) - qp[a]);
                    }
                }
                if (covered) {
                    done = true;
                } else if (m >= K1) {
                    const float bb = bound - g.delta;
                    done = bb > 0.0f && T * 1.00001f < bb * bb;
                }
            }
        }
        if (!flag) {
            // the K1 nearest: entries at or below the K1-th distance, sorted
            __syncwarp();
            const float v = m > K1 ? kg_kth(W.buf, m, K1, W.hist, lane) : kInf;
            m = kg_compact(W.buf, m, v, lane);
            if (m > 128) flag = true;  // more than 128 at or below the K1-th: equal distances
        }
        if (!flag) {
            uint64_t key[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int i = r * 32 + lane;
                key[r] = ~0ull;
                if (i < m) {
                    const float2 e = W.buf[i];
                    key[r] = ((uint64_t)__float_as_uint(e.x) << 32) | (uint32_t)__float_as_int(e.y);
                }
            }
            kg_sort128(key, lane);
            // equal distances among the first K1 -> the reference heap decides their order
            bool tie = false;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint64_t up = __shfl_up_sync(0xffffffffu, key[r], 1);
                const uint64_t prev_last = r > 0 ? __shfl_sync(0xffffffffu, key[r - 1], 31) : 0ull;
                const int e = r * 32 + lane;
                const uint64_t prev = lane > 0 ? up : prev_last;
                if (e >= 1 && e < K1 && (prev >> 32) == (key[r] >> 32)) tie = true;
            }
            flag = __any_sync(0xffffffffu, tie);
            if (!flag) {
                const int valid = K1 < ke ? K1 : ke;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int e = r * 32 + lane;
                    if (e < valid) {
                        oi[e] = sbase + (int64_t)(uint32_t)key[r];
                        od[e] = __uint_as_float((uint32_t)(key[r] >> 32));
                    }
                }
                for (int j = valid + lane; j < k; j += 32) {
                    oi[j] = -1;
                    od[j] = 1e30f;
                }
            }
        }
        if (flag && lane == 0) flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        __syncwarp();
    }
}

size_t knn_grid_ws(int64_t nmax, int32_t B, char *base, KgWs *w) {
    size_t off = 0;
    auto take = [&](size_t bytes) {
        char *r = base ? base + off : nullptr;
        off += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t n = nmax > 0 ? nmax : 1;
    const int32_t nb = B > 0 ? B : 1;
    KgWs t;
    t.lptr = (int64_t *)take(sizeof(int64_t) * (nb + 1));
    t.invalid = (int32_t *)take(sizeof(int32_t));
    t.grid = (KGrid *)take(sizeof(KGrid) * nb);
    t.key_bits = (int32_t *)take(sizeof(int32_t));
    t.keys = (uint32_t *)take(sizeof(uint32_t) * n);
    t.sorted_keys = (uint32_t *)take(sizeof(uint32_t) * n);
    t.sorted_idx = (int32_t *)take(sizeof(int32_t) * n);
    t.pts = (float4 *)take(sizeof(float4) * n);
    t.cells = (int2 *)take(sizeof(int2) * kKgCellBudget * n);
    char *rb = take(radix_scratch_bytes(n, nb));
    if (base) t.rs = radix_carve(rb, n, nb);
    if (w) *w = t;
    return off;
}

cudaError_t knn_grid_run(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
                         int32_t B, int64_t n_q, int k, int64_t max_src, const KgWs &w, int64_t *out_idx,
                         float *out_dist, int32_t *flag_list, int32_t *flag_count, cudaStream_t st) {
    const int64_t nmax = (int64_t)B * max_src;
    const unsigned g256 = (unsigned)((nmax + 255) / 256);
    kg_lptr_kernel<<<1, 256, 0, st>>>(ptr_s, B, nmax, w.lptr, w.invalid);
    cudaError_t e = cudaMemsetAsync(w.key_bits, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return e;
    kg_grid_kernel<<<B, kKgGridThreads, 0, st>>>(source, ptr_s, w.lptr, B, k, (int32_t *)w.cells, w.grid,
                                                  w.key_bits);
    kg_keys_kernel<<<g256, 256, 0, st>>>(source, ptr_s, w.lptr, B, w.grid, w.keys);
    e = radix_sort_pairs(w.keys, nullptr, w.sorted_keys, w.sorted_idx, nmax, w.lptr, B, 4, w.key_bits, w.rs, st);
    if (e != cudaSuccess) return e;
    kg_gather_kernel<<<g256, 256, 0, st>>>(source, ptr_s, w.lptr, B, w.sorted_idx, w.pts);
    e = cudaMemsetAsync(w.cells, 0, sizeof(int2) * kKgCellBudget * nmax, st);
    if (e != cudaSuccess) return e;
    kg_cells_kernel<<<g256, 256, 0, st>>>(w.lptr, B, w.grid, w.sorted_keys, w.cells);
    const size_t smem = sizeof(KgWarpSmem) * kKgWarps;
    e = cudaFuncSetAttribute(kg_query_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int64_t blocks = (n_q + kKgWarps - 1) / kKgWarps;
    const unsigned grid = (unsigned)(blocks < 24 * kSmCount ? (blocks > 0 ? blocks : 1) : 24 * kSmCount);
    kg_query_kernel<<<grid, kKgWarps * 32, smem, st>>>(query, ptr_q, B, ptr_s, w.lptr, w.grid, w.pts, w.cells, k,
                                                        w.invalid, out_idx, out_dist, flag_list, flag_count);
    return cudaGetLastError();
}

}  // namespace gdl
