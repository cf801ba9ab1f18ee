// knn_grid.cuh -- exact KNN over a uniform grid of each cloud's sources (large clouds).
#pragma once

#include "common.cuh"
#include "radix.cuh"

namespace gdl {

// The grid path serves calls whose largest cloud has at least this many sources. Below it the
// brute-force scan wins: it is fp32-bound at ~3.6 T pairs/s, while one uniform cell size cannot fit
// both clustered sources and queries that sit away from them (measured on configurations 3 and 4:
// 1.44 ms vs 1.2 ms and 5.5 ms vs 4.8 ms), and the quadratic cost only bites for larger clouds.
constexpr int64_t kKgMinSources = 32768;
constexpr int kKgCellBudget = 16;  // grid cells per source point at most (dense cell table)

// Warp-distributed sorted list of the best (distance, index) pairs: entry lane + 32 r lives in
// register set r of every lane, ascending, +inf padded. Inserts (dd, ii) after the entries smaller
// than dd: the position is one ballot/popc per set, the shift one shuffle. All lanes call it.
template <int NR>
__device__ __forceinline__ void warp_list_insert(float (&ed)[NR], int (&ei)[NR], float dd, int ii, int lane) {
    int pos = 0;
#pragma unroll
    for (int r = 0; r < NR; ++r) pos += __popc(__ballot_sync(0xffffffffu, ed[r] < dd));
    float ud[NR], xd[NR];
    int ui[NR], xi[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {  // entry (lane + 32 r - 1), read before any entry changes
        ud[r] = __shfl_up_sync(0xffffffffu, ed[r], 1);
        ui[r] = __shfl_up_sync(0xffffffffu, ei[r], 1);
        xd[r] = r > 0 ? __shfl_sync(0xffffffffu, ed[r > 0 ? r - 1 : 0], 31) : 0.0f;
        xi[r] = r > 0 ? __shfl_sync(0xffffffffu, ei[r > 0 ? r - 1 : 0], 31) : 0;
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int i = lane + 32 * r;
        if (i > pos) {
            ed[r] = lane == 0 ? xd[r] : ud[r];
            ei[r] = lane == 0 ? xi[r] : ui[r];
        } else if (i == pos) {
            ed[r] = dd;
            ei[r] = ii;
        }
    }
}

// Bulk form of warp_list_insert: every lane offers one candidate (d, i) (d = +inf for none). The
// candidates are sorted across the warp (bitonic, ascending distance, then index), each one's
// place in the merged list is its rank plus the number of entries <= it, each entry's its index
// plus the number of candidates < it (a stable merge, entries first), and the L smallest are
// written through `stage` (2 * 32 * NR words of shared memory for this warp) back into the
// registers. For many candidates at once this costs a few dozen shuffles instead of one insert
// network per candidate.
template <int NR>
__device__ __forceinline__ void warp_list_merge(float (&ed)[NR], int (&ei)[NR], float d, int i, int L, int lane,
                                                float *stage_d, int *stage_i) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1)  // bitonic sort of the 32 candidates
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float od = __shfl_xor_sync(0xffffffffu, d, j);
            const int oi = __shfl_xor_sync(0xffffffffu, i, j);
            const bool up = (lane & k) == 0;          // this run ascends
            const bool low = (lane & j) == 0;         // this lane holds the smaller slot
            const bool other_less = od < d || (od == d && oi < i);
            if (other_less == (low == up)) {
                d = od;
                i = oi;
            }
        }
    // binary search range: a power of two above 32 * NR, since a candidate can follow every entry
    constexpr int P = NR == 1 ? 64 : 128;
    // entries <= d (the candidate's place among them)
    int le = 0;
#pragma unroll
    for (int half = P / 2; half >= 1; half >>= 1) {
        const int probe = le + half - 1;
        float v = __int_as_float(0x7f800000);
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const float x = __shfl_sync(0xffffffffu, ed[r], probe & 31);
            if ((probe >> 5) == r) v = x;
        }
        if (probe < 32 * NR && v <= d) le += half;
    }
    const int pc = lane + le;
    // candidates < entry (the entry's place among them): the candidates are sorted in lane order
    int pe[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        int lt = 0;
#pragma unroll
        for (int half = 32; half >= 1; half >>= 1) {  // lt runs 0..32
            const int probe = lt + half - 1;
            const float x = __shfl_sync(0xffffffffu, d, probe & 31);
            if (probe < 32 && x < ed[r]) lt += half;
        }
        pe[r] = lane + 32 * r + lt;
    }
    __syncwarp();
    if (pc < L) {
        stage_d[pc] = d;
        stage_i[pc] = i;
    }
#pragma unroll
    for (int r = 0; r < NR; ++r)
        if (pe[r] < L) {
            stage_d[pe[r]] = ed[r];
            stage_i[pe[r]] = ei[r];
        }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int at = lane + 32 * r;
        ed[r] = at < L ? stage_d[at] : __int_as_float(0x7f800000);
        ei[r] = at < L ? stage_i[at] : -1;
    }
    __syncwarp();
}

struct KGrid {
    float mn[3];
    float h, inv;
    float delta;  // coordinate slack of the pruning bound (rounding of cell assignment)
    int res[3];
    int ok;       // 1 grid built; 0 cloud without sources; -1 non-finite coordinates
};

struct KgWs {
    int64_t *lptr;      // [B + 1] source offsets relative to ptr_s[0]
    int32_t *invalid;   // [1] the sources exceed the capacity the workspace was sized for
    KGrid *grid;        // [B]
    int32_t *key_bits;  // [1]
    uint32_t *keys, *sorted_keys;
    int32_t *sorted_idx;
    float4 *pts;   // sorted sources, .w = local source index
    int2 *cells;   // [kKgCellBudget * nmax] (first, one-past-last) sorted position per cell
    RadixScratch rs;
};

// bytes of the grid path's workspace for at most `nmax` sources in `B` clouds (base == nullptr:
// size only); carves `w` from `base` otherwise
size_t knn_grid_ws(int64_t nmax, int32_t B, char *base, KgWs *w);

// Builds the grids and answers every query of [ptr_q[0], ptr_q[B]): rows are written, or the
// query is appended to flag_list for the exact heap replay (equal distances among its k+1
// nearest, non-finite coordinates, or a search that ran out of room).
cudaError_t knn_grid_run(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
                         int32_t B, int64_t n_q, int k, int64_t max_src, const KgWs &w, int64_t *out_idx,
                         float *out_dist, int32_t *flag_list, int32_t *flag_count, cudaStream_t st);

}  // namespace gdl
