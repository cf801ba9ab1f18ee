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
// range. Candidates below the current (k_eff+1)-th distance T enter the warp's sorted list of the
// k_eff + 1 nearest (one ballot/popc and one shuffle per insert). After each shell the search
// stops once T (1 + 1e-5) < (b - delta)^2, b = the distance from the query to the nearest face of
// the examined block that is not the grid's edge, delta = the coordinate slack of cell assignment.
#include "knn_grid.cuh"

namespace gdl {

constexpr int kKgGridThreads = 1024;
constexpr int kKgWarps = 8;
constexpr int kKgMaxShell = 12;  // farther than this: the query goes to the exact replay
constexpr int kKgDepth = 4;      // candidate batches of 32 in flight per warp

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
        // clustered clouds: shrink the cells toward t points seen per point -- for k >= 8, whose
        // answers lie within a few points; for smaller k the density cell stays, so that queries
        // off the sources' clusters still end their search in the first shells
        if (occ > t && ke >= 8) {
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

template <int NR>
static __global__ void __launch_bounds__(kKgWarps * 32) kg_query_kernel(
    const float *__restrict__ query, const int64_t *__restrict__ ptr_q, int32_t B, const int64_t *__restrict__ ptr_s,
    const int64_t *__restrict__ lptr, const KGrid *__restrict__ grids, const float4 *__restrict__ pts,
    const int2 *__restrict__ cells, int k, const int32_t *__restrict__ invalid, int64_t *__restrict__ out_idx,
    float *__restrict__ out_dist, int32_t *__restrict__ flag_list, int32_t *__restrict__ flag_count) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
        // the warp's sorted list of the K1 nearest so far; thr = its K1-th entry (+inf until full)
        float ed[NR];
        int ei[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            ed[r] = kInf;
            ei[r] = -1;
        }
        float thr = kInf;
        int cnt = 0;
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
                for (int p0 = 0; p0 < npairs; p0 += 32) {
                    const int p = p0 + lane;
                    int ra0 = 0, re0 = 0, ra1 = 0, re1 = 0;  // two sorted ranges [ra, re) of the cloud
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
                        while (busy) {
                            const int l = __ffs(busy) - 1;
                            busy &= busy - 1;
                            const int a = __shfl_sync(0xffffffffu, ra, l), e = __shfl_sync(0xffffffffu, re, l);
                            for (int jb = a; jb < e; jb += 32 * kKgDepth) {
                              float4 sp[kKgDepth];  // loads of kKgDepth batches issued together
#pragma unroll
                              for (int u = 0; u < kKgDepth; ++u)
                                  if (jb + 32 * u + lane < e) sp[u] = pts[s0 + jb + 32 * u + lane];
#pragma unroll
                              for (int u = 0; u < kKgDepth; ++u) {
                                const int j0 = jb + 32 * u;
                                if (j0 >= e) break;  // uniform over the warp
                                const int j = j0 + lane;
                                float d = kInf;
                                int o = 0;
                                if (j < e) {
                                    o = __float_as_int(sp[u].w);
                                    d = dist2(qp[0], qp[1], qp[2], sp[u].x, sp[u].y, sp[u].z);
                                }
                                unsigned acc = __ballot_sync(0xffffffffu, d < thr);
                                while (acc) {
                                    const int l2 = __ffs(acc) - 1;
                                    acc &= acc - 1;
                                    const float dd = __shfl_sync(0xffffffffu, d, l2);
                                    const int oo = __shfl_sync(0xffffffffu, o, l2);
                                    if (!(dd < thr)) continue;  // tightened since the ballot (uniform)
                                    warp_list_insert<NR>(ed, ei, dd, oo, lane);
                                    ++cnt;
#pragma unroll
                                    for (int r = 0; r < NR; ++r)
                                        if ((K1 - 1) / 32 == r) thr = __shfl_sync(0xffffffffu, ed[r], (K1 - 1) & 31);
                                }
                              }
                            }
                        }
                    };
                    take(ra0, re0);
                    take(ra1, re1);
                }
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
                } else if (cnt >= K1) {
                    const float bb = bound - g.delta;
                    done = bb > 0.0f && thr * 1.00001f < bb * bb;
                }
            }
        }
        const int have = cnt < K1 ? cnt : K1;
        // every finite distance enters a list that is not full: a short list means overflowed distances
        if (!flag && have < K1) flag = true;
        if (!flag) {  // equal distances among the K1 nearest: the reference heap decides their order
            bool tie = false;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float up = __shfl_up_sync(0xffffffffu, ed[r], 1);
                const float cross = r > 0 ? __shfl_sync(0xffffffffu, ed[r > 0 ? r - 1 : 0], 31) : 0.0f;
                const int i = lane + 32 * r;
                const float prev = lane > 0 ? up : cross;
                if (i >= 1 && i < K1 && prev == ed[r]) tie = true;
            }
            flag = __any_sync(0xffffffffu, tie);
        }
        if (!flag) {
            const int nv = K1 < ke ? K1 : ke;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int i = lane + 32 * r;
                if (i < k) {
                    oi[i] = i < nv ? sbase + (int64_t)ei[r] : -1;
                    od[i] = i < nv ? ed[r] : 1e30f;
                }
            }
            for (int i = 32 * NR + lane; i < k; i += 32) {
                oi[i] = -1;
                od[i] = 1e30f;
            }
        } else if (lane == 0) {
            flag_list[atomicAdd(flag_count, 1)] = (int32_t)q;
        }
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
    const int64_t blocks = (n_q + kKgWarps - 1) / kKgWarps;
    const unsigned grid = (unsigned)(blocks < 24 * kSmCount ? (blocks > 0 ? blocks : 1) : 24 * kSmCount);
    const int K1 = (k < 64 ? k : 64) + 1;
    if (K1 <= 32)
        kg_query_kernel<1><<<grid, kKgWarps * 32, 0, st>>>(query, ptr_q, B, ptr_s, w.lptr, w.grid, w.pts, w.cells, k,
                                                          w.invalid, out_idx, out_dist, flag_list, flag_count);
    else if (K1 <= 64)
        kg_query_kernel<2><<<grid, kKgWarps * 32, 0, st>>>(query, ptr_q, B, ptr_s, w.lptr, w.grid, w.pts, w.cells, k,
                                                          w.invalid, out_idx, out_dist, flag_list, flag_count);
    else
        kg_query_kernel<3><<<grid, kKgWarps * 32, 0, st>>>(query, ptr_q, B, ptr_s, w.lptr, w.grid, w.pts, w.cells, k,
                                                          w.invalid, out_idx, out_dist, flag_list, flag_count);
    return cudaGetLastError();
}

}  // namespace gdl
