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
// kernel minimises the work between two picks:
//  * a cloud's coordinates and running minima stay in REGISTERS for the whole run (P points
//    per thread); a float4 copy of the coordinates in shared memory serves the winner lookup;
//  * the argmax is a single u64 key (min_d bits << 32 | ~priority): a tree max over the
//    thread's P keys, two redux.sync per warp, warp winners into a double-buffered slot
//    array, one __syncthreads, then every warp reduces the slots itself (no second barrier;
//    a shared-memory u64 atomicMax measured ~300 cycles slower per step here);
//  * the winner's local index is decoded from its priority (a bijection) and its coordinates
//    read back from shared memory.
// Clouds above one CTA's register budget run on a thread-block cluster (up to 16 CTAs of 13312
// points each, one per SM): each CTA's winner record goes to every CTA of the cluster through
// distributed shared memory (st.async + mbarrier per pick). A 131072-point cloud takes 10 CTAs,
// the largest cluster of which 8 fit on a B200 at once (11 of 10 CTAs, 7 of 11-16 CTAs), so a
// batch of 8 LiDAR clouds runs in one wave. Larger clouds fall back to a CTA that streams points
// from HBM with min_d in a workspace.
#include <cooperative_groups.h>

#include "common.cuh"

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

// Register state of the cluster kernel: P points per thread with NO stored priority, so that
// more points fit per CTA (a cluster of at most 10 CTAs per 131072-point cloud, the largest size
// at which 8 clusters are resident at once on a B200). With THREADS = 256 and the CTA's first
// point a multiple of 512, a thread's points i = base + tid + 256 j are ordered by either tie
// rule as a fixed permutation of j: lowest index = ascending j; the reference's order (see
// fps_priority) = even j ascending, then odd j ascending (its bit 27 is j's parity, its low bits
// j / 2). The running max uses that rank in the key's low word; the thread's winner then gets
// its true priority. Slots past the cloud (j >= nv) hold min_d = 0 and can only surface when
// every valid minimum is 0 too; that case rescans the valid slots.
template <int P, int TIE>
struct WidePoints {
    static_assert(P % 2 == 0, "points are held in pairs");
    static constexpr int THREADS = 256;
    uint64_t xp[P / 2], yp[P / 2], zp[P / 2];
    float md[P];
    int nv;    // slots j < nv hold points of the cloud
    int base;  // local index of this CTA's first point

    static __device__ __forceinline__ constexpr uint32_t pref(int j) {  // larger = preferred
        return (uint32_t)(P - 1 - (TIE == GDL_TIE_LOWEST_INDEX ? j : ((j & 1) ? P / 2 + j / 2 : j / 2)));
    }
    static __device__ __forceinline__ int unpref(uint32_t p) {
        const int q = P - 1 - (int)p;
        return TIE == GDL_TIE_LOWEST_INDEX ? q : (q < P / 2 ? 2 * q : 2 * (q - P / 2) + 1);
    }

    __device__ __forceinline__ void load(const float *__restrict__ pos, int64_t start, int n, int b, int,
                                         float4 *__restrict__ sxyz) {
        base = b;
        nv = 0;
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
                sxyz[i - base] = make_float4(x[j], y[j], z[j], 0.0f);
                nv = j + 1;
            } else {
                x[j] = y[j] = z[j] = 0.0f;
                md[j] = 0.0f;
            }
        }
#pragma unroll
        for (int h = 0; h < P / 2; ++h) {
            xp[h] = pack2(x[2 * h], x[2 * h + 1]);
            yp[h] = pack2(y[2 * h], y[2 * h + 1]);
            zp[h] = pack2(z[2 * h], z[2 * h + 1]);
        }
    }

    __device__ __forceinline__ uint64_t step(float sx, float sy, float sz) {
        const uint64_t SX = pack2(sx, sx), SY = pack2(sy, sy), SZ = pack2(sz, sz);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int h = 0; h < P / 2; ++h) {
            float d0, d1;
            unpack2(dist2_x2(xp[h], yp[h], zp[h], SX, SY, SZ), d0, d1);
            const float m0 = fminf(d0, md[2 * h]), m1 = fminf(d1, md[2 * h + 1]);
            md[2 * h] = m0;
            md[2 * h + 1] = m1;
            const uint64_t k0 = ((uint64_t)__float_as_uint(m0) << 32) | pref(2 * h);
            const uint64_t k1 = ((uint64_t)__float_as_uint(m1) << 32) | pref(2 * h + 1);
            acc[h & 3] = umax64(acc[h & 3], umax64(k0, k1));
        }
        if (nv == 0) return 0ull;
        uint64_t best = umax64(umax64(acc[0], acc[1]), umax64(acc[2], acc[3]));
        int j = unpref((uint32_t)best);
        if (j >= nv) {  // a padding slot won among zero minima: take the best valid slot
            best = 0ull;
#pragma unroll
            for (int t = 0; t < P; ++t)
                if (t < nv) best = umax64(best, ((uint64_t)__float_as_uint(md[t]) << 32) | pref(t));
            j = unpref((uint32_t)best);
        }
        const uint32_t prio = fps_priority((uint32_t)(base + (int)threadIdx.x + j * THREADS), TIE);
        return (best & 0xffffffff00000000ull) | (uint64_t)(~prio);
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

// ------------------------------------------------------------------ cluster per cloud
// Per pick, warp 0 of every CTA sends its winner record to every CTA of the cluster with
// st.async stores into distributed shared memory, each completing 24 bytes of a transaction on
// the receiving CTA's mbarrier; a CTA then waits on its own mbarrier only (no cluster-wide
// barrier per pick: 1.18 vs 1.63 us per pick at 16 CTAs). Two record buffers and two mbarriers
// alternate between picks: a CTA's record for pick k+2 can only be sent after the CTA received
// this CTA's record for pick k+1, which is sent after this CTA finished reading pick k's.
// Every wait is bounded; a CTA that gives up stops, and rank 0 then marks the cloud's remaining
// picks with -2 (never observed; a broken cluster exchange would show up there, not as a hang).
struct __align__(32) Rec {  // one CTA's best point
    unsigned long long key;
    float x, y, z, pad;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t mapa_u32(uint32_t a, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}

constexpr int kClusterWaitLimit = 1 << 20;  // mbarrier polls before a CTA gives up

template <int THREADS, int P, class PR>
__global__ void __launch_bounds__(THREADS) fps_cluster_kernel(const float *__restrict__ pos,
                                                              const int64_t *__restrict__ ptr,
                                                              const int64_t *__restrict__ kpc, int tie,
                                                              int64_t *__restrict__ out, float *__restrict__ out_pos) {
    constexpr int kMaxCluster = 16;
    constexpr int NW = THREADS / 32;
    extern __shared__ float4 sxyz[];  // this CTA's THREADS * P points
    __shared__ unsigned long long slots[2][NW];
    __shared__ Rec recs[2][kMaxCluster];
    __shared__ __align__(8) unsigned long long mbar[2];
    __shared__ int64_t red[NW];
    cg::cluster_group cluster = cg::this_cluster();
    const int cs = (int)cluster.num_blocks();
    const int rank = (int)cluster.block_rank();
    const int b = blockIdx.x / cs;
    const int64_t start = ptr[b];
    const int n = (int)(ptr[b + 1] - start);
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    const int64_t actual = (kb <= 0 || n <= 0) ? 0 : (kb < n ? kb : n);
    if (rank == 0) pad_outputs(out, out_pos, o0, actual, kb, THREADS);
    const int base = rank * THREADS * P;
    PR pr;
    pr.load(pos, start, n, base, tie, sxyz);
    float sx = 0.0f, sy = 0.0f, sz = 0.0f;
    if (actual > 0) {
        sx = pos[3 * start];
        sy = pos[3 * start + 1];
        sz = pos[3 * start + 2];
        if (rank == 0 && threadIdx.x == 0) emit(out, out_pos, o0, start, 0, sx, sy, sz);
    }
    if (threadIdx.x == 0) {
        for (int p = 0; p < 2; ++p) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar[p])));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t phase[2] = {0u, 0u};
    cluster.sync();  // every CTA resident, its barriers initialised, before any remote store
    int64_t k = 1;
    for (; k < actual; ++k) {
        const uint64_t wk = warp_max_key(pr.step(sx, sy, sz));
        const int par = (int)(k & 1);
        if (lane == 0) slots[par][warp] = wk;
        __syncthreads();
        if (warp == 0) {  // this CTA's winner, sent into every CTA's record slot [rank]
            const unsigned long long key = warp_max_key(lane < NW ? slots[par][lane] : 0ull);
            float rx = 0.0f, ry = 0.0f, rz = 0.0f;
            if (key != 0ull) {
                const float4 c = sxyz[fps_index(~(uint32_t)key, tie) - base];
                rx = c.x;
                ry = c.y;
                rz = c.z;
            }
            if (lane == 0)  // this CTA expects one 24-byte record from each CTA for this pick
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&mbar[par])),
                             "r"(cs * 24)
                             : "memory");
            if (lane < cs) {
                const uint32_t dst = mapa_u32(smem_u32(&recs[par][rank]), lane);
                const uint32_t bar = mapa_u32(smem_u32(&mbar[par]), lane);
                asm volatile(
                    "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                        dst),
                    "r"((uint32_t)key), "r"((uint32_t)(key >> 32)), "r"(__float_as_uint(rx)), "r"(__float_as_uint(ry)),
                    "r"(bar)
                    : "memory");
                asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(
                                 dst + 16),
                             "r"(__float_as_uint(rz)), "r"(0u), "r"(bar)
                             : "memory");
            }
        }
        uint32_t done = 0;
        for (int it = 0; it < kClusterWaitLimit && !done; ++it)
            asm volatile(
                "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, "
                "p;\n\t}"
                : "=r"(done)
                : "r"(smem_u32(&mbar[par])), "r"(phase[par])
                : "memory");
        phase[par] ^= 1u;
        if (!__syncthreads_and(done)) break;  // the whole CTA stops if any thread gave up
        const unsigned long long mine = lane < cs ? recs[par][lane].key : 0ull;
        const uint64_t best = warp_max_key(mine);
        const int src = __ffs(__ballot_sync(0xffffffffu, lane < cs && mine == best)) - 1;
        const Rec w = recs[par][src];
        sx = w.x;
        sy = w.y;
        sz = w.z;
        if (rank == 0 && threadIdx.x == 0) emit(out, out_pos, o0 + k, start, fps_index(~(uint32_t)best, tie), sx, sy, sz);
    }
    if (k < actual && rank == 0)  // a wait gave up: mark the picks this cloud did not make
        for (int64_t j = k + threadIdx.x; j < actual; j += THREADS) out[o0 + j] = -2;
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

constexpr int kCtaCapacity = 256 * 32;         // points per single-CTA cloud (fps_cta_kernel<256, 32>)
constexpr int kClusterThreads = 256;
constexpr int kClusterP = 52;                   // 13312 points per CTA: 10 CTAs for 131072 points
constexpr int64_t kClusterCapacity = (int64_t)kClusterThreads * kClusterP;

static cudaError_t launch_cluster(int B, int cs, const float *pos, const int64_t *ptr, const int64_t *kpc, int tie,
                                  int64_t *out, float *out_pos, cudaStream_t st) {
    auto kern = tie == GDL_TIE_LOWEST_INDEX
                    ? fps_cluster_kernel<kClusterThreads, kClusterP, WidePoints<kClusterP, GDL_TIE_LOWEST_INDEX>>
                    : fps_cluster_kernel<kClusterThreads, kClusterP, WidePoints<kClusterP, GDL_TIE_REFERENCE>>;
    const size_t smem = sizeof(float4) * kClusterCapacity;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (cs > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * cs));
    cfg.blockDim = dim3(kClusterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int max_clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg);
    if (e != cudaSuccess || max_clusters < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
    return cudaLaunchKernelEx(&cfg, kern, pos, ptr, kpc, tie, out, out_pos);
}

}  // namespace gdl

using namespace gdl;

extern "C" size_t gdl_fps_workspace_size(int64_t n_points, int64_t max_cloud_points) {
    // the cluster variant may be refused by the device; the streaming fallback needs n floats
    if (max_cloud_points <= kCtaCapacity) return 0;
    return sizeof(float) * (size_t)(n_points > 0 ? n_points : 1);
}

extern "C" int gdl_fps(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int32_t num_clouds,
                       int64_t n_points, int64_t max_cloud_points, int32_t tie_break, int64_t *out_idx,
                       float *out_pos, void *workspace, size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || max_cloud_points < 0 || n_points < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(tie_break != GDL_TIE_REFERENCE && tie_break != GDL_TIE_LOWEST_INDEX, GDL_ERR_INVALID);
    if (num_clouds == 0) return GDL_OK;
    GDL_RETURN_IF(!ptr || !k_per_cloud || !out_idx || (n_points > 0 && !pos), GDL_ERR_INVALID);
    GDL_RETURN_IF(max_cloud_points >= INT32_MAX, GDL_ERR_OVERFLOW);
    const int64_t m = max_cloud_points;
    cudaError_t e;
    if (m <= 512) e = launch_cta<128, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= 1024) e = launch_cta<256, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= 2048) e = launch_cta<256, 8>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= 4096) e = launch_cta<256, 16>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else if (m <= kCtaCapacity) e = launch_cta<256, 32>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
    else {
        const int cs = (int)((m + kClusterCapacity - 1) / kClusterCapacity);
        e = cudaErrorInvalidConfiguration;
        if (cs <= 16) e = launch_cluster(num_clouds, cs, pos, ptr, k_per_cloud, tie_break, out_idx, out_pos, st);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();  // clear a refused cluster launch, use the streaming kernel
            GDL_RETURN_IF(!workspace || workspace_bytes < sizeof(float) * (size_t)n_points, GDL_ERR_WORKSPACE);
            fps_stream_kernel<<<num_clouds, kStreamThreads, 0, st>>>(pos, ptr, k_per_cloud, tie_break,
                                                                     (float *)workspace, out_idx, out_pos);
            e = cudaGetLastError();
        }
    }
    return e == cudaSuccess ? GDL_OK : GDL_ERR_CUDA;
}
