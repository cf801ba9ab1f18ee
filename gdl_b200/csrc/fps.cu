// fps.cu -- farthest point sampling for packed clouds (sm_100a).
//
// Reference: geoembodied/csrc/fps_kernel.cu:40-209 (fps_kernel<512> + fps_cuda).
//
// Semantics kept bit-exact: seed = first point of the cloud; min_d starts at 1e30; each step
// min_d[p] = fminf(dist2(p, sel), min_d[p]) with the reference's rounding (common.cuh) and the
// next pick is the argmax. Ties go by a 32-bit priority: either the reference kernel's
// reduction order (GDL_TIE_REFERENCE, see fps_priority) or the lowest index.
//
// Design (B200). The step is a pure latency chain (one argmax per selected point), so the
// kernels minimise the work between two picks. The argmax is a single u64 key (min_d bits << 32
// | ~priority), so any grouping of the points gives the same winner.
//  * Clouds of at most 4096 points: one CTA per cloud, P points per thread in REGISTERS, a tree
//    max over the thread's keys, two redux.sync per warp, warp winners into a double-buffered
//    slot array, one __syncthreads per pick (fps_cta_kernel).
//  * Larger clouds (bucketed FPS): each cloud is first put in Morton order (bounding box, 30-bit
//    codes, segmented radix sort), so that every thread owns a compact run of P points -- a
//    bucket with an axis-aligned box. A thread first bounds the distance from a new sample to its
//    box with the same rounded operations as the point distances; the bound is <= every point's
//    rounded distance (rounding is monotone), so when it is >= the bucket's largest minimum no
//    minimum of the bucket can change and the thread skips its P updates. The points sit in shared
//    memory (SoA float2 pairs, each thread's in priority order so that a (min-distance, slot) key
//    reduced as a tree orders them exactly), the minima in registers. One CTA serves up to 8192
//    or 13824 points; larger clouds run on a thread-block cluster of up to 16 CTAs whose records
//    cross through distributed shared memory (st.async stores completing bytes on each receiver's
//    mbarrier, one bounded wait per round). The picks are made in rounds of up to eight: each
//    warp, and in a cluster each CTA, reports its best point with a bound on its other points,
//    and the records are taken in decreasing key order while each provably remains the next pick
//    of the one-at-a-time chain (its minimum survives the picks taken before it in the round, it
//    beats their bounds); the result is bit-identical to one pick per exchange, with about three
//    and a half picks per exchange on LiDAR clouds (fps_bucket_kernel).
//  * Clouds beyond 16 x 13824 points: a CTA that streams points from HBM with min_d in the
//    workspace (fps_stream_kernel).
#include <cooperative_groups.h>

#include "common.cuh"
#include "morton.cuh"
#include "radix.cuh"

namespace cg = cooperative_groups;

namespace gdl {

// Priority of local point i under the reference kernel's tie order (fps_kernel.cu:86-143):
// thread tid = i % 512 scans i = tid, tid+512, ... keeping the first maximum (`>`), the
// shuffle-down tree and the shared-memory tree keep their left operand on ties, i.e. prefer
// lane / warp indices in bit-reversed order. Smaller priority wins.
__device__ __forceinline__ uint32_t fps_priority(uint32_t i, int tie) {
    if (tie == GDL_TIE_LOWEST_INDEX) return i;
    const uint32_t tid = i & 511u, rj = i >> 9;
    const uint32_t w = tid >> 5, l = tid & 31u;
    return ((__brev(w) >> 28) << 27) | ((__brev(l) >> 27) << 22) | (rj & 0x3fffffu);
}

// inverse of fps_priority
__device__ __forceinline__ uint32_t fps_index(uint32_t prio, int tie) {
    if (tie == GDL_TIE_LOWEST_INDEX) return prio;
    const uint32_t w = __brev((prio >> 27) & 15u) >> 28, l = __brev((prio >> 22) & 31u) >> 27;
    return ((prio & 0x3fffffu) << 9) | (w << 5) | l;
}

__device__ __forceinline__ uint64_t make_key(float m, uint32_t np) {
    return ((uint64_t)__float_as_uint(m) << 32) | np;
}

__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }

// max over the warp of a u64 key (hi word first, then lo among the hi winners)
__device__ __forceinline__ uint64_t warp_max_key(uint64_t k) {
    const uint32_t hi = (uint32_t)(k >> 32);
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)k : 0u);
    return ((uint64_t)mhi << 32) | mlo;
}

// lane holding the warp's largest u64 key (the lowest such lane) and that key's high word: one
// redux on the high words, the low words only when several lanes share the largest high word
__device__ __forceinline__ int warp_argmax_key(uint64_t k, uint32_t &mhi) {
    const uint32_t hi = (uint32_t)(k >> 32);
    mhi = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t tied = __ballot_sync(0xffffffffu, hi == mhi);
    if ((tied & (tied - 1u)) == 0u) return __ffs(tied) - 1;
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (uint32_t)k : 0u);
    return __ffs(__ballot_sync(0xffffffffu, hi == mhi && (uint32_t)k == mlo)) - 1;
}

// out offset of cloud b = sum_{c<b} max(k_c, 0)
__device__ __forceinline__ int64_t block_out_offset(const int64_t *__restrict__ kpc, int b, int64_t *red) {
    int64_t s = 0;
    for (int c = threadIdx.x; c < b; c += blockDim.x) s += kpc[c] > 0 ? kpc[c] : 0;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    int64_t t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    __syncthreads();
    return t;
}

// one selection: global index (and, when requested, its coordinates)
__device__ __forceinline__ void emit(int64_t *__restrict__ out, float *__restrict__ out_pos, int64_t slot,
                                     int64_t start, int64_t idx, float x, float y, float z) {
    out[slot] = start + idx;
    if (out_pos) {
        out_pos[3 * slot] = x;
        out_pos[3 * slot + 1] = y;
        out_pos[3 * slot + 2] = z;
    }
}

// slots [actual, kb) of a cloud that asked for more points than it has: -1 (and 0 coordinates)
__device__ __forceinline__ void pad_outputs(int64_t *__restrict__ out, float *__restrict__ out_pos, int64_t o0,
                                            int64_t actual, int64_t kb, int threads) {
    for (int64_t j = actual + threadIdx.x; j < kb; j += threads) {
        out[o0 + j] = -1;
        if (out_pos) out_pos[3 * (o0 + j)] = out_pos[3 * (o0 + j) + 1] = out_pos[3 * (o0 + j) + 2] = 0.0f;
    }
}

// Per-thread register state: P points i = base + threadIdx.x + j * THREADS.
template <int THREADS, int P>
struct PointRegs {
    static_assert(P % 2 == 0, "points are held in pairs");
    uint64_t xp[P / 2], yp[P / 2], zp[P / 2];  // coordinates of points (2h, 2h+1), packed fp32x2
    float md[P];
    uint32_t np[P];  // ~priority; 0 marks a padding slot (never wins)

    __device__ __forceinline__ void load(const float *__restrict__ pos, int64_t start, int n, int base, int tie,
                                         float4 *__restrict__ sxyz) {
        float x[P], y[P], z[P];
#pragma unroll
        for (int j = 0; j < P; ++j) {
            const int i = base + (int)threadIdx.x + j * THREADS;
            if (i < n) {
                const float *p = pos + 3 * (start + i);
                x[j] = p[0];
                y[j] = p[1];
                z[j] = p[2];
                md[j] = 1e30f;
                np[j] = ~fps_priority((uint32_t)i, tie);
                sxyz[i - base] = make_float4(x[j], y[j], z[j], 0.0f);
            } else {
                x[j] = y[j] = z[j] = 0.0f;
                md[j] = 0.0f;
                np[j] = 0u;
            }
        }
#pragma unroll
        for (int h = 0; h < P / 2; ++h) {
            xp[h] = pack2(x[2 * h], x[2 * h + 1]);
            yp[h] = pack2(y[2 * h], y[2 * h + 1]);
            zp[h] = pack2(z[2 * h], z[2 * h + 1]);
        }
    }

    // update the minima against (sx, sy, sz); this thread's best key (tree max over P)
    __device__ __forceinline__ uint64_t step(float sx, float sy, float sz) {
        const uint64_t SX = pack2(sx, sx), SY = pack2(sy, sy), SZ = pack2(sz, sz);
        uint64_t k[P];
#pragma unroll
        for (int h = 0; h < P / 2; ++h) {
            float d0, d1;  // dist2(point, s) for both points of the pair, bit-identical to dist2()
            unpack2(dist2_x2(xp[h], yp[h], zp[h], SX, SY, SZ), d0, d1);
            const float m0 = fminf(d0, md[2 * h]), m1 = fminf(d1, md[2 * h + 1]);
            md[2 * h] = m0;
            md[2 * h + 1] = m1;
            k[2 * h] = np[2 * h] ? make_key(m0, np[2 * h]) : 0ull;
            k[2 * h + 1] = np[2 * h + 1] ? make_key(m1, np[2 * h + 1]) : 0ull;
        }
#pragma unroll
        for (int w = 1; w < P; w <<= 1)
#pragma unroll
            for (int j = 0; j + w < P; j += 2 * w) k[j] = umax64(k[j], k[j + w]);
        return k[0];
    }
};


// ------------------------------------------------------------------ one CTA per cloud
template <int THREADS, int P>
__global__ void __launch_bounds__(THREADS) fps_cta_kernel(const float *__restrict__ pos,
                                                          const int64_t *__restrict__ ptr,
                                                          const int64_t *__restrict__ kpc, int tie,
                                                          int64_t *__restrict__ out, float *__restrict__ out_pos) {
    constexpr int NW = THREADS / 32;
    extern __shared__ float4 sxyz[];  // [THREADS * P]
    __shared__ unsigned long long slots[2][NW];
    __shared__ int64_t red[NW];
    const int b = blockIdx.x;
    const int64_t start = ptr[b];
    const int n = (int)(ptr[b + 1] - start);
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    if (kb <= 0) return;
    const int64_t actual = n <= 0 ? 0 : (kb < n ? kb : n);
    pad_outputs(out, out_pos, o0, actual, kb, THREADS);
    if (actual <= 0) return;

    PointRegs<THREADS, P> pr;
    pr.load(pos, start, n, 0, tie, sxyz);
    __syncthreads();
    float4 s = sxyz[0];
    if (threadIdx.x == 0) emit(out, out_pos, o0, start, 0, s.x, s.y, s.z);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t k = 1; k < actual; ++k) {
        const uint64_t wk = warp_max_key(pr.step(s.x, s.y, s.z));
        const int par = (int)(k & 1);
        if (lane == 0) slots[par][warp] = wk;
        __syncthreads();
        // every warp reduces the warp winners itself: no second barrier; the other parity
        // buffer takes step k+1's writes while slow warps still read this one
        const uint64_t best = warp_max_key(lane < NW ? slots[par][lane] : 0ull);
        const uint32_t idx = fps_index(~(uint32_t)best, tie);
        s = sxyz[idx];
        if (threadIdx.x == 0) emit(out, out_pos, o0 + k, start, idx, s.x, s.y, s.z);
    }
}

// ------------------------------------------------------------------ bucketed FPS
constexpr int kMaxCluster = 16;
constexpr int kDefaultWaitPolls = 1 << 20;   // mbarrier polls before a wait gives up
constexpr int kMaxDynSmem = 227 * 1024;
constexpr int kRecBytes = 24;                // one record: key, x, y (16-B store) + z, bound (8-B store)
constexpr int kCtaRecords = 2;               // records a CTA of a cluster sends per round
// A record's bound: the largest minimum (float bits, >= 0) among the points it stands for other
// than its own, with the top bit set when its own coordinates are not finite (its distance to
// itself is then NaN, not 0, so no pick may follow it in the same round); either way, a later
// pick's minimum bits must exceed the bound.
constexpr uint32_t kNonFinite = 0x80000000u;
constexpr int kRoundPicks = 16;              // picks one round may make

__host__ __device__ constexpr size_t bucket_points_bytes(int T, int P) { return (size_t)16 * T * P; }
// records per round: one per CTA of the cluster, double-buffered
__host__ __device__ constexpr size_t bucket_smem_bytes(int T, int P, int cs) {
    return bucket_points_bytes(T, P) + (size_t)2 * kCtaRecords * cs * kRecBytes;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t mapa_u32(uint32_t a, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done;
}

// One warp record into a CTA's slot: (key, x, y) in 16 bytes and (z, bound) in 8, both completing
// bytes of a transaction on that CTA's mbarrier.
__device__ __forceinline__ void st_async_rec(uint32_t da, uint32_t db, uint32_t rb, uint64_t key, float x, float y,
                                             float z, uint32_t bound) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(da),
                 "r"((uint32_t)key), "r"((uint32_t)(key >> 32)), "r"(__float_as_uint(x)), "r"(__float_as_uint(y)),
                 "r"(rb)
                 : "memory");
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(db),
                 "r"(__float_as_uint(z)), "r"(bound), "r"(rb)
                 : "memory");
}

// Lower bound of dist2(p, s) over every p of the box [lo, hi]. Per axis the gap is the larger of
// lo - s, s - hi and 0, each difference rounded like the point differences: a point's
// |p - s| rounds to at least the gap's rounding (rounding is monotone), and the same fma chain
// keeps that order, so the bound never exceeds a point's rounded distance. A NaN sample gives gaps
// of 0 (fmaxf), and then every distance is NaN and no minimum changes anyway; an infinite box
// side gives an infinite gap only when every point of the box is infinite on that side.
__device__ __forceinline__ float box_dist2_lb(float sx, float sy, float sz, const float (&bx)[6]) {
    const float gx = fmaxf(fmaxf(sub_ftz(bx[0], sx), sub_ftz(sx, bx[3])), 0.0f);
    const float gy = fmaxf(fmaxf(sub_ftz(bx[1], sy), sub_ftz(sy, bx[4])), 0.0f);
    const float gz = fmaxf(fmaxf(sub_ftz(bx[2], sz), sub_ftz(sz, bx[5])), 0.0f);
    return fma_ftz(gz, gz, fma_ftz(gx, gx, mul_ftz(gy, gy)));
}

// the rounded distance of point (px, py, pz) to sample (sx, sy, sz), computed exactly as the
// bucket update computes it (packed, lane 0 of the pair)
__device__ __forceinline__ float pair_dist2(float px, float py, float pz, float sx, float sy, float sz) {
    float d0, d1;
    unpack2(dist2_x2(pack2(px, px), pack2(py, py), pack2(pz, pz), pack2(sx, sx), pack2(sy, sy), pack2(sz, sz)), d0,
            d1);
    return d0;
}

// T threads per CTA, P points per thread -- a bucket of consecutive points in Morton order, kept
// in priority order in shared memory, with its box, its minima in registers, its best key and the
// largest minimum among its other points; a cluster of cs CTAs serves one cloud of at most
// cs * T * P points, which `order` (global indices, Morton order within each cloud) lists.
// Warp-sized chunks of 32 threads' buckets go round-robin over the cluster's CTAs, so that the
// buckets around one pick (neighbours in Morton order) update on several SMs.
//
// The picks are made in rounds of up to M. Per round:
//  1. every bucket applies the previous round's picks (skipping each whose distance bound to the
//     bucket's box is >= the bucket's largest minimum);
//  2. every warp sends one record to every CTA of the cluster (st.async completing bytes on the
//     receiver's mbarrier; a lone CTA writes its own slots and meets one barrier): the warp's best
//     key, that point, and a bound on the keys of the warp's other points (the other lanes' best
//     keys and the winning bucket's second minimum);
//  3. after a bounded wait for the cluster's records every warp takes them in decreasing key
//     order. The first is the argmax, as in the one-pick chain. A later one, c, is the next pick
//     of the same chain exactly when every point other than c holds a smaller key once the
//     accepted picks a_1..a_j have updated the minima: c's own minimum must survive them
//     (!(dist2(c, a_i) < min(c))), c must beat the bound of each a_i's warp (the points that a_i
//     hid from the records), each a_i's minimum must drop to 0 (dist2(a_i, a_i) == 0: finite
//     coordinates) below c's (min(c) > 0); every other record's warp holds keys no larger than its
//     record, which is smaller than c. The first record that fails ends the round. Minima only
//     decrease and fminf over a set of samples does not depend on their order, so the result is
//     bit-identical to picking one point per exchange.
// status (nullable) receives GDL_ERR_TIMEOUT when a bounded wait gives up; the cloud's picks from
// that one on are then -2 (coordinates 0). hold_rank / hold_pick: the CTA of that rank in every
// cluster sends no records in the round that starts at that pick (rounds never cross it while a
// hold is set), which makes every wait of the round run out (the failure path's test); -1
// disables it. A lone CTA never waits, unless hold_rank asks it to exchange. rounds (nullable):
// the largest number of exchange rounds any cloud took (atomicMax), for the latency roofline.
template <int T, int P, int TIE, int M>
__global__ void __launch_bounds__(T, 1) fps_bucket_kernel(const float *__restrict__ pos,
                                                           const int32_t *__restrict__ order,
                                                           const int64_t *__restrict__ ptr,
                                                           const int64_t *__restrict__ kpc,
                                                           int64_t *__restrict__ out, float *__restrict__ out_pos,
                                                           int32_t *__restrict__ status, int wait_polls,
                                                           int hold_rank, int64_t hold_pick,
                                                           unsigned long long *__restrict__ rounds) {
    constexpr int NW = T / 32, PH = P / 2;
    static_assert(P % 2 == 0, "points are held in pairs");
    constexpr int kMaxRecords = NW > kCtaRecords * kMaxCluster ? NW : kCtaRecords * kMaxCluster;  // per round
    static_assert(M >= 1 && M <= 32 && kMaxRecords <= 32, "one record and one pick per lane");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ __align__(8) unsigned long long mbar[2];
    __shared__ int64_t red[NW];
    __shared__ uint4 slotA[NW];  // warp records: key, x, y
    __shared__ uint2 slotB[NW];  // z, bound
    __shared__ float4 s_pick[M];  // the round's picks
    __shared__ int s_count;       // how many (-1: a wait gave up)
    // small buckets (P <= 8) test the round's picks against their warp's box first: there a
    // lane's own tests cost about as much as its update (larger buckets measured slower with it)
    constexpr bool kWarpBox = P <= 8;
    __shared__ float s_wbox[kWarpBox ? NW : 1][6];  // each warp's box: the union of its lanes' boxes
    float2 *sx2 = reinterpret_cast<float2 *>(smem);  // pair h of thread t at h * T + t
    float2 *sy2 = sx2 + PH * T;
    float2 *sz2 = sy2 + PH * T;
    uint2 *sn2 = reinterpret_cast<uint2 *>(sz2 + PH * T);  // ~priority, 0 for padding

    cg::cluster_group cluster = cg::this_cluster();
    const int cs = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int RC = kCtaRecords * cs;                                             // records per round
    uint4 *recA = reinterpret_cast<uint4 *>(smem + bucket_points_bytes(T, P));  // [2][RC]: key, x, y
    uint2 *recB = reinterpret_cast<uint2 *>(recA + 2 * RC);                     // [2][RC]: z, bound

    const int b = blockIdx.x / cs;
    const int64_t start = ptr[b];
    const int n = (int)(ptr[b + 1] - start);
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    const int64_t actual = (kb <= 0 || n <= 0) ? 0 : (kb < n ? kb : n);
    if (rank == 0) pad_outputs(out, out_pos, o0, actual, kb, T);
    {  // the launch must give every CTA the shared memory this kernel indexes (the same for all
       // CTAs of the cluster, so they all leave here together, before any remote access)
        uint32_t dyn;
        asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        if ((size_t)dyn < bucket_smem_bytes(T, P, cs)) {
            if (threadIdx.x == 0 && status) atomicExch(status, (int32_t)GDL_ERR_INVALID);
            if (rank == 0)
                for (int64_t j = threadIdx.x; j < actual; j += T) out[o0 + j] = -2;
            return;
        }
    }

    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int q0 = ((warp * cs + rank) * 32 + lane) * P;  // this thread's first sorted position
    float md[P];
    float box[6] = {INFINITY, INFINITY, INFINITY, -INFINITY, -INFINITY, -INFINITY};
    {
        float x[P], y[P], z[P];
        uint32_t np[P];  // ~priority; 0 marks a padding slot (key 0, never wins)
#pragma unroll
        for (int j = 0; j < P; ++j) {
            const int q = q0 + j;
            x[j] = y[j] = z[j] = 0.0f;
            np[j] = 0u;
            if (q < n) {
                const int64_t v = order[start + q];
                x[j] = pos[3 * v];
                y[j] = pos[3 * v + 1];
                z[j] = pos[3 * v + 2];
                np[j] = ~fps_priority((uint32_t)(v - start), TIE);
            }
        }
        // the thread's points in priority order (slot 0 preferred, padding last): a thread-local
        // key (min-distance, P - 1 - slot) then orders them exactly as (min-distance, ~priority)
#pragma unroll
        for (int r = 0; r < P; ++r)
#pragma unroll
            for (int j = r & 1; j + 1 < P; j += 2)
                if (np[j] < np[j + 1]) {
                    const float tx = x[j], ty = y[j], tz = z[j];
                    const uint32_t tn = np[j];
                    x[j] = x[j + 1], y[j] = y[j + 1], z[j] = z[j + 1], np[j] = np[j + 1];
                    x[j + 1] = tx, y[j + 1] = ty, z[j + 1] = tz, np[j + 1] = tn;
                }
#pragma unroll
        for (int j = 0; j < P; ++j) {
            md[j] = np[j] ? 1e30f : 0.0f;
            if (np[j]) {
                box[0] = fminf(box[0], x[j]);
                box[1] = fminf(box[1], y[j]);
                box[2] = fminf(box[2], z[j]);
                box[3] = fmaxf(box[3], x[j]);
                box[4] = fmaxf(box[4], y[j]);
                box[5] = fmaxf(box[5], z[j]);
            }
            const int o = (j >> 1) * T + t, c = j & 1;
            reinterpret_cast<float *>(&sx2[o])[c] = x[j];
            reinterpret_cast<float *>(&sy2[o])[c] = y[j];
            reinterpret_cast<float *>(&sz2[o])[c] = z[j];
            reinterpret_cast<uint32_t *>(&sn2[o])[c] = np[j];
        }
    }
    // lkey: the bucket's best thread-local key (min-distance, P - 1 - slot), reduced as a tree;
    // bestkey: the same point's (min-distance, ~priority) key and (bx, by, bz) its coordinates;
    // sec: the largest minimum among the bucket's other slots (float bits; minima are >= 0)
    uint64_t lkey, bestkey;
    uint32_t sec;
    float bx, by, bz;
    auto rekey = [&]() {
        uint64_t kk[P];
#pragma unroll
        for (int j = 0; j < P; ++j) kk[j] = make_key(md[j], (uint32_t)(P - 1 - j));
#pragma unroll
        for (int w = 1; w < P; w <<= 1)
#pragma unroll
            for (int j = 0; j + w < P; j += 2 * w) kk[j] = umax64(kk[j], kk[j + w]);
        lkey = kk[0];
        const int bj = P - 1 - (int)(uint32_t)lkey;
        uint32_t sb[P];
#pragma unroll
        for (int j = 0; j < P; ++j) sb[j] = j == bj ? 0u : __float_as_uint(md[j]);
#pragma unroll
        for (int w = 1; w < P; w <<= 1)
#pragma unroll
            for (int j = 0; j + w < P; j += 2 * w) sb[j] = sb[j] > sb[j + w] ? sb[j] : sb[j + w];
        sec = sb[0];
        const int o = (bj >> 1) * T + t;
        const float2 X = sx2[o], Y = sy2[o], Z = sz2[o];
        const uint2 N = sn2[o];
        bestkey = (lkey & 0xffffffff00000000ull) | (uint64_t)((bj & 1) ? N.y : N.x);
        bx = (bj & 1) ? X.y : X.x;
        by = (bj & 1) ? Y.y : Y.x;
        bz = (bj & 1) ? Z.y : Z.x;
    };
    rekey();
    // the warp's box: redux.sync over an order-preserving integer image of each coordinate (the
    // boxes are built from +-inf by fminf / fmaxf, never NaN)
    if constexpr (kWarpBox) {
#pragma unroll
        for (int c = 0; c < 6; ++c) {
            const int b = __float_as_int(box[c]);
            const int key = b >= 0 ? b : (b ^ 0x7fffffff);
            const int r = c < 3 ? __reduce_min_sync(0xffffffffu, key) : __reduce_max_sync(0xffffffffu, key);
            if (lane == 0) s_wbox[warp][c] = __int_as_float(r >= 0 ? r : (r ^ 0x7fffffff));
        }
    }

    if (t == 0) {
        if (actual > 0) {  // the first pick: the cloud's first point
            const float x0 = pos[3 * start], y0 = pos[3 * start + 1], z0 = pos[3 * start + 2];
            s_pick[0] = make_float4(x0, y0, z0, 0.0f);
            if (rank == 0) emit(out, out_pos, o0, start, 0, x0, y0, z0);
        }
        s_count = actual > 0 ? 1 : 0;
        for (int p = 0; p < 2; ++p) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[p])));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    cluster.sync();  // every CTA resident, its points stored and its barriers initialised

    const bool exchange = cs > 1 || hold_rank >= 0;  // a lone CTA selects from its warps' records
    uint32_t phase = 0u;                              // bit p: parity of the next phase of mbar[p]
    int64_t k = 1;
    int par = 0;
    bool ok = true;
    unsigned long long nround = 0;
    while (k < actual) {
        ++nround;
        // 1. the bucket's minima against the previous round's picks (s_pick[0, s_count)): one pass
        // over the points per pick that some lane of the warp needs (a lane whose box is too far from
        // the pick -- bound >= its largest minimum -- gets fminf(d, m) == m, so computing it there
        // changes nothing)
        {
            const int npick = s_count;
            const float curmax = __uint_as_float((uint32_t)(lkey >> 32));
            // (small buckets) first lanes 0..npick-1 test one pick each against the warp's box and
            // its lanes' largest minimum (minima are >= 0, so their bits order as unsigned): the
            // bound to a box can only grow for a box inside it, so a pick that fails there fails
            // every lane's own test; the lanes then test only the picks that passed
            uint32_t need = 0u;
            if constexpr (kWarpBox) {
                const uint32_t wmax = __reduce_max_sync(0xffffffffu, (uint32_t)(lkey >> 32));
                bool near = false;
                if (lane < npick) {
                    const float4 p = s_pick[lane];
                    // read every round (volatile): held across the loop the box would cost registers
                    const volatile float *wbp = s_wbox[warp];
                    float wb[6];
#pragma unroll
                    for (int c = 0; c < 6; ++c) wb[c] = wbp[c];
                    near = !(box_dist2_lb(p.x, p.y, p.z, wb) >= __uint_as_float(wmax));
                }
                uint32_t cand = __ballot_sync(0xffffffffu, near);
#pragma unroll 1
                while (cand) {
                    const int i = __ffs(cand) - 1;
                    cand &= cand - 1u;
                    const float4 p = s_pick[i];
                    if (!(box_dist2_lb(p.x, p.y, p.z, box) >= curmax)) need |= 1u << i;
                }
            } else {
#pragma unroll 1
                for (int i = 0; i < npick; ++i) {
                    const float4 p = s_pick[i];
                    if (!(box_dist2_lb(p.x, p.y, p.z, box) >= curmax)) need |= 1u << i;
                }
            }
            uint32_t wneed = __reduce_or_sync(0xffffffffu, need);
            if (wneed) {
#pragma unroll 1
                while (wneed) {
                    const int i = __ffs(wneed) - 1;
                    wneed &= wneed - 1u;
                    const float4 p = s_pick[i];
                    const uint64_t SX = pack2(p.x, p.x), SY = pack2(p.y, p.y), SZ = pack2(p.z, p.z);
#pragma unroll
                    for (int h = 0; h < PH; ++h) {
                        const float2 X = sx2[h * T + t], Y = sy2[h * T + t], Z = sz2[h * T + t];
                        float d0, d1;
                        unpack2(dist2_x2(pack2(X.x, X.y), pack2(Y.x, Y.y), pack2(Z.x, Z.y), SX, SY, SZ), d0, d1);
                        md[2 * h] = fminf(d0, md[2 * h]);
                        md[2 * h + 1] = fminf(d1, md[2 * h + 1]);
                    }
                }
                rekey();
            }
        }
        // 2. the warp's record: its best key and point, and a bound on its other points' keys
        {
            uint32_t mhi;
            const int wl = warp_argmax_key(bestkey, mhi);
            const uint32_t wb = __reduce_max_sync(0xffffffffu, lane == wl ? sec : (uint32_t)(bestkey >> 32));
            if (lane == wl) {
                const bool fin = fabsf(bx) < INFINITY && fabsf(by) < INFINITY && fabsf(bz) < INFINITY;
                slotA[warp] = make_uint4((uint32_t)bestkey, (uint32_t)(bestkey >> 32), __float_as_uint(bx),
                                         __float_as_uint(by));
                slotB[warp] = make_uint2(__float_as_uint(bz), wb | (fin ? 0u : kNonFinite));
            }
        }
        __syncthreads();
        // 3. warp 0 makes the round's picks; the other warps wait at the next barrier
        if (warp == 0) {
            int64_t limit = actual - k;
            if (hold_pick > k && hold_pick - k < limit) limit = hold_pick - k;  // only while a hold is set
            // the records the picks are taken from, one per lane: a lone CTA's warp records, or the
            // cluster's CTA records (a CTA's best and a bound on its other points: the other warps'
            // best keys and the winning warp's bound), exchanged through st.async and a bounded wait
            uint4 ra = make_uint4(0u, 0u, 0u, 0u);
            uint2 rc = make_uint2(0u, 0u);
            const uint4 *SA = slotA;
            const uint2 *SB = slotB;
            int S = NW;
            bool got = true;
            if (lane < NW) {
                ra = slotA[lane];
                rc = slotB[lane];
            }
            if (exchange) {
                // the CTA's two best warp records: the first keeps its warp's bound, the second's also
                // covers the CTA's other warps (their best keys)
                static_assert(kCtaRecords == 2, "two records per CTA");
                const uint64_t sk = ((uint64_t)ra.y << 32) | ra.x;
                uint32_t mhi;
                const int w1 = warp_argmax_key(sk, mhi);
                const int w2 = warp_argmax_key(lane == w1 ? 0ull : sk, mhi);
                const uint32_t rest = __reduce_max_sync(0xffffffffu, (lane == w1 || lane == w2) ? 0u : ra.y);
                const uint32_t bar = smem_u32(&mbar[par]);
                if (lane == 0)
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                                 "r"(RC * kRecBytes)
                                 : "memory");
                // lane r * cs + d sends record r to CTA d (a CTA with one non-empty warp has no second
                // record: the second argmax then ties among empty keys and may return the first warp)
                const int which = lane >= cs ? 1 : 0, dst = lane - which * cs, wsrc = which ? w2 : w1;
                const bool empty = which && w2 == w1;
                uint4 w = slotA[wsrc];
                const uint2 wz = slotB[wsrc];
                if (empty) w = make_uint4(0u, 0u, 0u, 0u);
                const uint32_t wbnd = empty ? 0u : which ? (wz.y > rest ? wz.y : rest) : wz.y;
                const int slot = par * RC + kCtaRecords * rank + which;
                if (lane < RC && !(rank == hold_rank && k == hold_pick))
                    st_async_rec(mapa_u32(smem_u32(&recA[slot]), dst), mapa_u32(smem_u32(&recB[slot]), dst),
                                 mapa_u32(bar, dst), ((uint64_t)w.y << 32) | w.x, __uint_as_float(w.z),
                                 __uint_as_float(w.w), __uint_as_float(wz.x), wbnd);
                const uint32_t want = (phase >> par) & 1u;
                // the warp leaves the poll loop together (a lane-divergent exit would leave the warp
                // split for the code that follows)
                bool done = false;
                for (int it = 0; it < wait_polls && !done; ++it)
                    done = __all_sync(0xffffffffu, mbar_try_wait(bar, want));
                phase ^= 1u << par;
                got = done;
                ra = make_uint4(0u, 0u, 0u, 0u);
                rc = make_uint2(0u, 0u);
                SA = recA + par * RC;
                SB = recB + par * RC;
                S = RC;
                if (lane < RC) {
                    ra = SA[lane];
                    rc = SB[lane];
                }
            }
            if (!got) {
                if (lane == 0) s_count = -1;
            } else {
                // Every record's rank (how many records hold a larger key) and whether it may follow
                // every record ahead of it within the round: its minimum survives each of them and
                // exceeds each one's bound (which also rules out a non-finite record ahead: its own
                // distance is NaN, not 0, and would keep its key), and is > 0 (a taken record's minimum
                // drops to 0). The round takes the records ahead of the first that may not; the first
                // record (rank 0) is always taken.
                const uint64_t mk = ((uint64_t)ra.y << 32) | ra.x;
                const float mx = __uint_as_float(ra.z), my = __uint_as_float(ra.w), mz = __uint_as_float(rc.x);
                const uint32_t mhi = ra.y;
                const float mmd = __uint_as_float(mhi);
                int rnk = 0;
                bool bad = mhi == 0u;
#pragma unroll 4
                for (int j = 0; j < S; ++j) {
                    const uint4 a = SA[j];
                    const uint2 c = SB[j];
                    const uint64_t kj = ((uint64_t)a.y << 32) | a.x;
                    const float xj = __uint_as_float(a.z), yj = __uint_as_float(a.w), zj = __uint_as_float(c.x);
                    const bool ahead = kj > mk;
                    // (bitwise: no branch per record; a non-finite record's bound exceeds every minimum)
                    const bool clash = !(mhi > c.y) | (dist2(mx, my, mz, xj, yj, zj) < mmd);
                    rnk += ahead ? 1 : 0;
                    bad |= ahead & clash;
                }
                const int lim = (int64_t)M < limit ? M : (int)limit;
                int A = __reduce_min_sync(0xffffffffu, (mk != 0ull && bad && rnk > 0) ? rnk : 32);
                const int nrec = __popc(__ballot_sync(0xffffffffu, mk != 0ull));
                A = A < nrec ? A : nrec;
                A = A < lim ? A : lim;
                if (mk != 0ull && rnk < A) {
                    s_pick[rnk] = make_float4(mx, my, mz, 0.0f);
                    if (rank == 0) emit(out, out_pos, o0 + k + rnk, start, fps_index(~(uint32_t)mk, TIE), mx, my, mz);
                }
                if (lane == 0) s_count = A;
            }
        }
        __syncthreads();
        const int A = s_count;
        if (A < 0) {
            ok = false;
            break;
        }
        k += A;
        par ^= 1;
    }
    if (!ok) {
        if (t == 0 && status) atomicExch(status, (int32_t)GDL_ERR_TIMEOUT);
        if (rank == 0 && warp == 0)  // mark the picks this cloud did not make
            for (int64_t j = k + lane; j < actual; j += 32) {
                out[o0 + j] = -2;
                if (out_pos) out_pos[3 * (o0 + j)] = out_pos[3 * (o0 + j) + 1] = out_pos[3 * (o0 + j) + 2] = 0.0f;
            }
    }
    if (rounds && rank == 0 && t == 0) atomicMax(rounds, nround);
    cluster.sync();  // no CTA leaves while a peer may still write into it
}

// ------------------------------------------------------------------ streaming fallback
// Any cloud size: one 1024-thread CTA per cloud, coordinates streamed from HBM every step,
// running minima in the workspace (as the reference does, fps_kernel.cu:90-106).
constexpr int kStreamThreads = 1024;
__global__ void __launch_bounds__(kStreamThreads) fps_stream_kernel(const float *__restrict__ pos,
                                                                    const int64_t *__restrict__ ptr,
                                                                    const int64_t *__restrict__ kpc, int tie,
                                                                    float *__restrict__ mind,
                                                                    int64_t *__restrict__ out,
                                                                    float *__restrict__ out_pos) {
    constexpr int NW = kStreamThreads / 32;
    __shared__ unsigned long long slots[2][NW];
    __shared__ int64_t red[NW];
    const int b = blockIdx.x;
    const int64_t start = ptr[b];
    const int64_t n = ptr[b + 1] - start;
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    if (kb <= 0) return;
    const int64_t actual = n <= 0 ? 0 : (kb < n ? kb : n);
    pad_outputs(out, out_pos, o0, actual, kb, kStreamThreads);
    if (actual <= 0) return;
    float *md = mind + start;
    for (int64_t i = threadIdx.x; i < n; i += kStreamThreads) md[i] = 1e30f;
    __syncthreads();
    float sx = pos[3 * start], sy = pos[3 * start + 1], sz = pos[3 * start + 2];
    if (threadIdx.x == 0) emit(out, out_pos, o0, start, 0, sx, sy, sz);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t k = 1; k < actual; ++k) {
        uint64_t best = 0ull;
        for (int64_t i = threadIdx.x; i < n; i += kStreamThreads) {
            const float *p = pos + 3 * (start + i);
            const float m = fminf(dist2(p[0], p[1], p[2], sx, sy, sz), md[i]);
            md[i] = m;
            best = umax64(best, make_key(m, ~fps_priority((uint32_t)i, tie)));
        }
        const uint64_t wk = warp_max_key(best);
        const int par = (int)(k & 1);
        if (lane == 0) slots[par][warp] = wk;
        __syncthreads();
        const int64_t idx = fps_index(~(uint32_t)warp_max_key(slots[par][lane]), tie);
        sx = pos[3 * (start + idx)];
        sy = pos[3 * (start + idx) + 1];
        sz = pos[3 * (start + idx) + 2];
        if (threadIdx.x == 0) emit(out, out_pos, o0 + k, start, idx, sx, sy, sz);
    }
}

template <int T, int P>
static cudaError_t launch_cta(int B, const float *pos, const int64_t *ptr, const int64_t *kpc, int tie, int64_t *out,
                              float *out_pos, cudaStream_t st) {
    const size_t smem = sizeof(float4) * T * P;
    auto kern = fps_cta_kernel<T, P>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<B, T, smem, st>>>(pos, ptr, kpc, tie, out, out_pos);
    return cudaGetLastError();
}

constexpr int kCtaCapacity = 4096;            // fps_cta_kernel<256, 16>; larger clouds are bucketed
// Bucketed launch shapes, from sweeps on a B200 (configuration 5's LiDAR clouds, configuration 3's
// 8192-point level): CTAs of 256 x 4 = 1024 points (clusters of up to 8: configuration 3's first
// level 0.74 ms on 8-CTA clusters against 1.05 ms on one 512 x 16 CTA per cloud, which left most
// SMs idle), of 512 x 16 = 8192 points (one CTA, or clusters of up to 16), of 512 x 26 = 13312
// points (10 for a 131072-point cloud; 7.2 ms for configuration 5's FPS against 8.1 ms with
// 384 x 36) and of 384 x 36 = 13824 points (the largest clouds: up to 16 x 13824). A B200 holds 11
// clusters of 10 CTAs at once but only 7 of 11-16, so eight LiDAR clouds run in one wave only as
// 10-CTA clusters, while up to seven take the 16-CTA shape, whose smaller buckets update faster.
// The launch takes the shape that needs the fewest waves of clusters, the smallest buckets on a
// tie.
constexpr int kTinyT = 256, kTinyP = 4;
constexpr int kTinyMaxCluster = 8;  // the tiny shape serves clouds of up to 8 x 1024 points
constexpr int kSmallT = 512, kSmallP = 16;
constexpr int kMidT = 512, kMidP = 26;
constexpr int kBigT = 384, kBigP = 36;
constexpr int64_t kTinyCapacity = (int64_t)kTinyT * kTinyP;
constexpr int64_t kSmallCapacity = (int64_t)kSmallT * kSmallP;
constexpr int64_t kMidCapacity = (int64_t)kMidT * kMidP;
constexpr int64_t kBucketCapacity = (int64_t)kBigT * kBigP;
constexpr int kMaxDevices = 64;

// launch configuration of the bucketed kernel for B clouds on clusters of cs CTAs
template <int T, int P, int TIE, int M>
static cudaError_t bucket_config(int B, int cs, cudaStream_t st, cudaLaunchConfig_t &cfg, cudaLaunchAttribute &attr) {
    auto kern = fps_bucket_kernel<T, P, TIE, M>;
    const size_t smem = bucket_smem_bytes(T, P, cs);
    if (cs < 1 || cs > kMaxCluster || smem > (size_t)kMaxDynSmem) return cudaErrorInvalidConfiguration;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (cs > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cfg = {};
    cfg.gridDim = dim3((unsigned)(B * cs));
    cfg.blockDim = dim3(T);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)cs;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return cudaSuccess;
}

// clusters of cs CTAs of this shape resident at once on the current device (0: none), cached
template <int T, int P, int TIE, int M>
static int bucket_max_clusters(int cs) {
    static int cache[kMaxDevices][kMaxCluster + 1];  // 0: not asked yet; -1: none fit
    int dev = 0;
    if (cs < 1 || cs > kMaxCluster || cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (dev >= 0 && dev < kMaxDevices && cache[dev][cs] != 0) return cache[dev][cs] > 0 ? cache[dev][cs] : 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    int mc = 0;
    if (bucket_config<T, P, TIE, M>(1, cs, 0, cfg, attr) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&mc, fps_bucket_kernel<T, P, TIE, M>, &cfg) != cudaSuccess)
        mc = 0;
    (void)cudaGetLastError();
    if (dev >= 0 && dev < kMaxDevices) cache[dev][cs] = mc > 0 ? mc : -1;
    return mc > 0 ? mc : 0;
}

template <int T, int P, int TIE, int M>
static cudaError_t launch_bucket(int B, int cs, const float *pos, const int32_t *order, const int64_t *ptr,
                                 const int64_t *kpc, int64_t *out, float *out_pos, int32_t *status, int polls,
                                 int hold_rank, int64_t hold_pick, unsigned long long *rounds, cudaStream_t st) {
    if (bucket_max_clusters<T, P, TIE, M>(cs) < 1) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr;
    cudaError_t e = bucket_config<T, P, TIE, M>(B, cs, st, cfg, attr);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, fps_bucket_kernel<T, P, TIE, M>, pos, order, ptr, kpc, out, out_pos, status, polls,
                              hold_rank, hold_pick, rounds);
}

template <int T, int P, int M>
static cudaError_t launch_bucket_tie(int tie, int B, int cs, const float *pos, const int32_t *order,
                                     const int64_t *ptr, const int64_t *kpc, int64_t *out, float *out_pos,
                                     int32_t *status, int polls, int hold_rank, int64_t hold_pick,
                                     unsigned long long *rounds, cudaStream_t st) {
    return tie == GDL_TIE_LOWEST_INDEX
               ? launch_bucket<T, P, GDL_TIE_LOWEST_INDEX, M>(B, cs, pos, order, ptr, kpc, out, out_pos, status,
                                                               polls, hold_rank, hold_pick, rounds, st)
               : launch_bucket<T, P, GDL_TIE_REFERENCE, M>(B, cs, pos, order, ptr, kpc, out, out_pos, status, polls,
                                                            hold_rank, hold_pick, rounds, st);
}

template <int T, int P, int M>
static int bucket_max_clusters_tie(int tie, int cs) {
    return tie == GDL_TIE_LOWEST_INDEX ? bucket_max_clusters<T, P, GDL_TIE_LOWEST_INDEX, M>(cs)
                                       : bucket_max_clusters<T, P, GDL_TIE_REFERENCE, M>(cs);
}

// Workspace of the bucketed path: cloud boxes, Morton keys, sorted keys, the order, radix scratch.
struct FpsWork {
    unsigned long long *rounds;  // exchange rounds of the last bucketed launch (its longest cloud)
    float *box;
    uint32_t *keys, *sorted_keys;
    int32_t *order;
    RadixScratch rs;
};

static size_t fps_carve(char *base, int64_t n, int32_t B, FpsWork *w) {
    char *p = base;
    auto take = [&](size_t bytes) {
        char *r = p;
        p += (bytes + 255) & ~size_t(255);
        return r;
    };
    const int64_t nn = n > 0 ? n : 1;
    char *rounds = take(sizeof(unsigned long long));
    char *box = take(sizeof(float) * 6 * (size_t)(B > 0 ? B : 1));
    char *keys = take(sizeof(uint32_t) * nn);
    char *skeys = take(sizeof(uint32_t) * nn);
    char *ord = take(sizeof(int32_t) * nn);
    char *rb = take(radix_scratch_bytes(nn, B > 0 ? B : 1));
    if (base) {
        w->rounds = (unsigned long long *)rounds;
        w->box = (float *)box;
        w->keys = (uint32_t *)keys;
        w->sorted_keys = (uint32_t *)skeys;
        w->order = (int32_t *)ord;
        w->rs = radix_carve(rb, nn, B > 0 ? B : 1);
    }
    return (size_t)(p - base);
}

}  // namespace gdl

using namespace gdl;

extern "C" size_t gdl_fps_workspace_size(int64_t n_points, int32_t num_clouds, int64_t max_cloud_points) {
    if (max_cloud_points <= kCtaCapacity || n_points <= 0) return 0;
    FpsWork w;
    // (the streaming fallback keeps its n floats of running minima in the keys region)
    return fps_carve(nullptr, n_points, num_clouds, &w);
}

extern "C" int gdl_fps_round_count(const void *workspace, int64_t n_points, int32_t num_clouds,
                                   int64_t max_cloud_points, unsigned long long *out) {
    GDL_RETURN_IF(!out || num_clouds < 0 || n_points < 0, GDL_ERR_INVALID);
    *out = 0;
    if (max_cloud_points <= kCtaCapacity || n_points <= 0) return GDL_OK;  // one pick per exchange
    GDL_RETURN_IF(!workspace, GDL_ERR_INVALID);
    FpsWork w;
    fps_carve((char *)workspace, n_points, num_clouds, &w);
    GDL_CUDA_TRY(cudaMemcpy(out, w.rounds, sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    return GDL_OK;
}

extern "C" int gdl_fps_ex(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int32_t num_clouds,
                          int64_t n_points, int64_t max_cloud_points, int32_t tie_break, int64_t *out_idx,
                          float *out_pos, void *workspace, size_t workspace_bytes, int32_t *status, int32_t wait_polls,
                          int32_t hold_rank, int64_t hold_pick, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || max_cloud_points < 0 || n_points < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(tie_break != GDL_TIE_REFERENCE && tie_break != GDL_TIE_LOWEST_INDEX, GDL_ERR_INVALID);
    if (num_clouds == 0) return GDL_OK;
    GDL_RETURN_IF(!ptr || !k_per_cloud || !out_idx || (n_points > 0 && !pos), GDL_ERR_INVALID);
    GDL_RETURN_IF(max_cloud_points >= INT32_MAX || n_points >= INT32_MAX, GDL_ERR_OVERFLOW);
    const int64_t m = max_cloud_points;
    const int polls = wait_polls > 0 ? wait_polls : kDefaultWaitPolls;
    cudaError_t e;
    if (m <= 512) e = launch_cta<128, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= 1024) e = launch_cta<256, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= 2048) e = launch_cta<256, 8>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= kCtaCapacity) e = launch_cta<256, 16>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else {
        GDL_RETURN_IF(!workspace || workspace_bytes < gdl_fps_workspace_size(n_points, num_clouds, m),
                      GDL_ERR_WORKSPACE);
        FpsWork w;
        fps_carve((char *)workspace, n_points, num_clouds, &w);
        // the shape: 256 x 4 (clusters of up to 8), 512 x 16, 512 x 26 or 384 x 36 CTAs (clusters of up
        // to 16), whichever needs the fewest waves of resident clusters for these clouds, the
        // smallest buckets on a tie
        const int64_t caps[4] = {kTinyCapacity, kSmallCapacity, kMidCapacity, kBucketCapacity};
        const int cmax[4] = {kTinyMaxCluster, kMaxCluster, kMaxCluster, kMaxCluster};
        int shape = -1, cs = 0;
        int64_t best_waves = 0;
        for (int sh = 0; sh < 4; ++sh) {
            const int c = (int)((m + caps[sh] - 1) / caps[sh]);
            if (c > cmax[sh]) continue;
            const int mc = sh == 0 ? bucket_max_clusters_tie<kTinyT, kTinyP, kRoundPicks>(tie_break, c)
                         : sh == 1 ? bucket_max_clusters_tie<kSmallT, kSmallP, kRoundPicks>(tie_break, c)
                         : sh == 2 ? bucket_max_clusters_tie<kMidT, kMidP, kRoundPicks>(tie_break, c)
                                   : bucket_max_clusters_tie<kBigT, kBigP, kRoundPicks>(tie_break, c);
            if (mc <= 0) continue;
            const int64_t waves = (num_clouds + mc - 1) / mc;
            if (shape < 0 || waves < best_waves) shape = sh, cs = c, best_waves = waves;
        }
        e = cudaErrorInvalidConfiguration;
        if (shape >= 0) {
            // Morton order of every cloud (the buckets), then the bucketed kernel
            GDL_CUDA_TRY(cudaMemsetAsync(w.rounds, 0, sizeof(unsigned long long), st));
            cloud_box_kernel<<<num_clouds, kBoxThreads, 0, st>>>(pos, ptr, w.box, nullptr);
            const int64_t blocks = (n_points + 255) / 256;
            morton_code_kernel<<<(unsigned)(blocks < 4 * kSmCount ? (blocks > 0 ? blocks : 1) : 4 * kSmCount), 256, 0,
                                 st>>>(pos, ptr, num_clouds, w.box, w.keys, false, n_points);
            GDL_CUDA_TRY(cudaGetLastError());
            GDL_CUDA_TRY(radix_sort_pairs(w.keys, nullptr, w.sorted_keys, w.order, n_points, ptr, num_clouds, 4,
                                          nullptr, w.rs, st));
            if (shape == 0)
                e = launch_bucket_tie<kTinyT, kTinyP, kRoundPicks>(tie_break, num_clouds, cs, pos, w.order, ptr,
                                                                   k_per_cloud, out_idx, out_pos, status, polls,
                                                                   hold_rank, hold_pick, w.rounds, st);
            else if (shape == 1)
                e = launch_bucket_tie<kSmallT, kSmallP, kRoundPicks>(tie_break, num_clouds, cs, pos, w.order, ptr,
                                                                     k_per_cloud, out_idx, out_pos, status, polls,
                                                                     hold_rank, hold_pick, w.rounds, st);
            else if (shape == 2)
                e = launch_bucket_tie<kMidT, kMidP, kRoundPicks>(tie_break, num_clouds, cs, pos, w.order, ptr,
                                                                 k_per_cloud, out_idx, out_pos, status, polls,
                                                                 hold_rank, hold_pick, w.rounds, st);
            else
                e = launch_bucket_tie<kBigT, kBigP, kRoundPicks>(tie_break, num_clouds, cs, pos, w.order, ptr,
                                                                 k_per_cloud, out_idx, out_pos, status, polls,
                                                                 hold_rank, hold_pick, w.rounds, st);
        }
        if (e != cudaSuccess) {
            (void)cudaGetLastError();  // clear a refused cluster launch, use the streaming kernel
            fps_stream_kernel<<<num_clouds, kStreamThreads, 0, st>>>(pos, ptr, k_per_cloud, tie_break,
                                                                     (float *)w.keys, out_idx, out_pos);
            e = cudaGetLastError();
        }
    }
    return e == cudaSuccess ? GDL_OK : GDL_ERR_CUDA;
}

extern "C" int gdl_fps(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int32_t num_clouds,
                       int64_t n_points, int64_t max_cloud_points, int32_t tie_break, int64_t *out_idx,
                       float *out_pos, void *workspace, size_t workspace_bytes, void *stream) {
    return gdl_fps_ex(pos, ptr, k_per_cloud, num_clouds, n_points, max_cloud_points, tie_break, out_idx, out_pos,
                      workspace, workspace_bytes, nullptr, 0, -1, -1, stream);
}
