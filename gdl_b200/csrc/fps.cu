// fps.cu -- farthest point sampling for packed clouds (sm_100a).
//
// Reference: geoembodied/csrc/fps_kernel.cu:40-209 (fps_kernel<512> + fps_cuda).
//
// Semantics kept bit-exact: seed = first point of the cloud; min_d starts at 1e30; each step
// min_d[p] = fminf(dist2(p, sel), min_d[p]) with the reference's rounding (common.cuh) and the
// next pick is the argmax. Ties go by a 32-bit priority: either the reference kernel's
// reduction order (GDL_TIE_REFERENCE, see fps_priority) or the lowest index.
//
// Design (B200): a cloud's points and running minima stay in REGISTERS for the whole run
// (P points per thread); the argmax is a packed 64-bit key (min_d bits, ~priority) reduced with
// two redux.sync per warp, the warp winners go to a double-buffered shared-memory slot array,
// one __syncthreads per step, and every warp then reduces the slots redundantly (no second
// barrier). Clouds above one CTA's register budget use a thread-block cluster (up to 16 CTAs,
// one per SM): each warp writes its winner straight into every CTA's slot array through
// distributed shared memory and one cluster barrier per step publishes them. Larger clouds
// fall back to a CTA that streams points from HBM with min_d in a workspace.
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

struct Cand {  // one warp's (or CTA's) best point
    uint32_t hi;  // bits of min_d (>= 0, so ordered like the float)
    uint32_t lo;  // ~priority
    float x, y, z;
    int32_t idx;  // local index
};

__device__ __forceinline__ bool key_gt(uint32_t ahi, uint32_t alo, uint32_t bhi, uint32_t blo) {
    return ahi > bhi || (ahi == bhi && alo > blo);
}

// Reduce a candidate across the warp; every lane returns the winner.
__device__ __forceinline__ Cand warp_argmax(Cand c) {
    const uint32_t mhi = __reduce_max_sync(0xffffffffu, c.hi);
    const uint32_t mlo = __reduce_max_sync(0xffffffffu, c.hi == mhi ? c.lo : 0u);
    const unsigned win = __ballot_sync(0xffffffffu, c.hi == mhi && c.lo == mlo);
    const int src = __ffs(win) - 1;
    Cand r;
    r.hi = mhi;
    r.lo = mlo;
    r.x = __shfl_sync(0xffffffffu, c.x, src);
    r.y = __shfl_sync(0xffffffffu, c.y, src);
    r.z = __shfl_sync(0xffffffffu, c.z, src);
    r.idx = __shfl_sync(0xffffffffu, c.idx, src);
    return r;
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

// Per-thread register state: P points (strided by THREADS inside a chunk of THREADS*P points).
template <int P>
struct PointRegs {
    float x[P], y[P], z[P], md[P];
    uint32_t np[P];  // ~priority, 0 for padding lanes

    __device__ __forceinline__ void load(const float *__restrict__ pos, int64_t start, int n, int chunk_base,
                                         int threads, int tie) {
#pragma unroll
        for (int j = 0; j < P; ++j) {
            const int i = chunk_base + (int)threadIdx.x + j * threads;
            if (i < n) {
                const float *p = pos + 3 * (start + i);
                x[j] = p[0];
                y[j] = p[1];
                z[j] = p[2];
                md[j] = 1e30f;
                np[j] = ~fps_priority((uint32_t)i, tie);
            } else {
                x[j] = y[j] = z[j] = 0.0f;
                md[j] = -1.0f;
                np[j] = 0u;
            }
        }
    }

    // update minima against (sx, sy, sz), return this thread's best candidate
    __device__ __forceinline__ Cand step(float sx, float sy, float sz, int chunk_base, int threads) {
        Cand c;
        c.hi = 0u;
        c.lo = 0u;
        c.x = c.y = c.z = 0.0f;
        c.idx = 0;
#pragma unroll
        for (int j = 0; j < P; ++j) {
            if (np[j] != 0u) {
                const float d = dist2(x[j], y[j], z[j], sx, sy, sz);
                const float m = fminf(d, md[j]);
                md[j] = m;
                const uint32_t h = __float_as_uint(m);
                if (key_gt(h, np[j], c.hi, c.lo)) {
                    c.hi = h;
                    c.lo = np[j];
                    c.x = x[j];
                    c.y = y[j];
                    c.z = z[j];
                    c.idx = chunk_base + (int)threadIdx.x + j * threads;
                }
            }
        }
        return c;
    }
};

// ------------------------------------------------------------------ one CTA per cloud
template <int THREADS, int P>
__global__ void __launch_bounds__(THREADS) fps_cta_kernel(const float *__restrict__ pos,
                                                          const int64_t *__restrict__ ptr,
                                                          const int64_t *__restrict__ kpc, int tie,
                                                          int64_t *__restrict__ out) {
    constexpr int NW = THREADS / 32;
    __shared__ Cand slots[2][NW];
    __shared__ int64_t red[NW];
    const int b = blockIdx.x;
    const int64_t start = ptr[b];
    const int n = (int)(ptr[b + 1] - start);
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    if (kb <= 0) return;
    const int64_t actual = n <= 0 ? 0 : (kb < n ? kb : n);
    for (int64_t j = actual + threadIdx.x; j < kb; j += THREADS) out[o0 + j] = -1;
    if (actual <= 0) return;

    PointRegs<P> pr;
    pr.load(pos, start, n, 0, THREADS, tie);
    if (threadIdx.x == 0) out[o0] = start;
    float sx = pos[3 * start], sy = pos[3 * start + 1], sz = pos[3 * start + 2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t k = 1; k < actual; ++k) {
        Cand c = warp_argmax(pr.step(sx, sy, sz, 0, THREADS));
        const int par = (int)(k & 1);
        if (lane == 0) slots[par][warp] = c;
        __syncthreads();
        Cand s = lane < NW ? slots[par][lane] : Cand{0u, 0u, 0.0f, 0.0f, 0.0f, 0};
        s = warp_argmax(s);
        sx = s.x;
        sy = s.y;
        sz = s.z;
        if (threadIdx.x == 0) out[o0 + k] = start + s.idx;
    }
}

// ------------------------------------------------------------------ cluster per cloud
template <int THREADS, int P>
__global__ void __launch_bounds__(THREADS) fps_cluster_kernel(const float *__restrict__ pos,
                                                              const int64_t *__restrict__ ptr,
                                                              const int64_t *__restrict__ kpc, int tie,
                                                              int64_t *__restrict__ out) {
    constexpr int NW = THREADS / 32;
    constexpr int kMaxCluster = 16;
    __shared__ Cand slots[2][kMaxCluster * NW];
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
    if (rank == 0)
        for (int64_t j = actual + threadIdx.x; j < kb; j += THREADS) out[o0 + j] = -1;
    // every CTA of the cluster runs the same number of steps (uniform exit)
    const int chunk_base = rank * THREADS * P;
    PointRegs<P> pr;
    pr.load(pos, start, n, chunk_base, THREADS, tie);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nslots = cs * NW;
    if (actual > 0 && rank == 0 && threadIdx.x == 0) out[o0] = start;
    float sx = actual > 0 ? pos[3 * start] : 0.0f, sy = actual > 0 ? pos[3 * start + 1] : 0.0f,
          sz = actual > 0 ? pos[3 * start + 2] : 0.0f;
    cluster.sync();  // all CTAs resident before remote shared-memory writes
    for (int64_t k = 1; k < actual; ++k) {
        Cand c = warp_argmax(pr.step(sx, sy, sz, chunk_base, THREADS));
        const int par = (int)(k & 1);
        if (lane < cs) {  // lane q publishes this warp's winner into CTA q's slot array
            Cand *dst = cluster.map_shared_rank(&slots[par][rank * NW + warp], lane);
            *dst = c;
        }
        cluster.sync();
        Cand s = Cand{0u, 0u, 0.0f, 0.0f, 0.0f, 0};
        for (int q = lane; q < nslots; q += 32) {
            const Cand t = slots[par][q];
            if (key_gt(t.hi, t.lo, s.hi, s.lo)) s = t;
        }
        s = warp_argmax(s);
        sx = s.x;
        sy = s.y;
        sz = s.z;
        if (rank == 0 && threadIdx.x == 0) out[o0 + k] = start + s.idx;
    }
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
                                                                    int64_t *__restrict__ out) {
    constexpr int NW = kStreamThreads / 32;
    __shared__ Cand slots[2][NW];
    __shared__ int64_t red[NW];
    const int b = blockIdx.x;
    const int64_t start = ptr[b];
    const int64_t n = ptr[b + 1] - start;
    const int64_t kb = kpc[b];
    const int64_t o0 = block_out_offset(kpc, b, red);
    if (kb <= 0) return;
    const int64_t actual = n <= 0 ? 0 : (kb < n ? kb : n);
    for (int64_t j = actual + threadIdx.x; j < kb; j += kStreamThreads) out[o0 + j] = -1;
    if (actual <= 0) return;
    float *md = mind + start;
    for (int64_t i = threadIdx.x; i < n; i += kStreamThreads) md[i] = 1e30f;
    if (threadIdx.x == 0) out[o0] = start;
    float sx = pos[3 * start], sy = pos[3 * start + 1], sz = pos[3 * start + 2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    for (int64_t k = 1; k < actual; ++k) {
        Cand c{0u, 0u, 0.0f, 0.0f, 0.0f, 0};
        for (int64_t i = threadIdx.x; i < n; i += kStreamThreads) {
            const float *p = pos + 3 * (start + i);
            const float px = p[0], py = p[1], pz = p[2];
            const float m = fminf(dist2(px, py, pz, sx, sy, sz), md[i]);
            md[i] = m;
            const uint32_t h = __float_as_uint(m), l = ~fps_priority((uint32_t)i, tie);
            if (key_gt(h, l, c.hi, c.lo)) c = Cand{h, l, px, py, pz, (int32_t)i};
        }
        c = warp_argmax(c);
        const int par = (int)(k & 1);
        if (lane == 0) slots[par][warp] = c;
        __syncthreads();
        Cand s = slots[par][lane];
        s = warp_argmax(s);
        sx = s.x;
        sy = s.y;
        sz = s.z;
        if (threadIdx.x == 0) out[o0 + k] = start + s.idx;
    }
}

template <int T, int P>
static cudaError_t launch_cta(int B, const float *pos, const int64_t *ptr, const int64_t *kpc, int tie, int64_t *out,
                              cudaStream_t st) {
    fps_cta_kernel<T, P><<<B, T, 0, st>>>(pos, ptr, kpc, tie, out);
    return cudaGetLastError();
}

constexpr int kClusterThreads = 512;
constexpr int kClusterP = 16;
constexpr int64_t kCtaCapacity = (int64_t)kClusterThreads * kClusterP;  // points per CTA

static cudaError_t launch_cluster(int B, int cs, const float *pos, const int64_t *ptr, const int64_t *kpc, int tie,
                                  int64_t *out, cudaStream_t st) {
    auto kern = fps_cluster_kernel<kClusterThreads, kClusterP>;
    if (cs > 8) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(B * cs));
    cfg.blockDim = dim3(kClusterThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int max_clusters = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg);
    if (e != cudaSuccess || max_clusters < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
    return cudaLaunchKernelEx(&cfg, kern, pos, ptr, kpc, tie, out);
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
                       void *workspace, size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_clouds < 0 || max_cloud_points < 0 || n_points < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(tie_break != GDL_TIE_REFERENCE && tie_break != GDL_TIE_LOWEST_INDEX, GDL_ERR_INVALID);
    if (num_clouds == 0) return GDL_OK;
    GDL_RETURN_IF(!ptr || !k_per_cloud || !out_idx || (n_points > 0 && !pos), GDL_ERR_INVALID);
    GDL_RETURN_IF(max_cloud_points >= INT32_MAX, GDL_ERR_OVERFLOW);
    const int64_t m = max_cloud_points;
    cudaError_t e;
    if (m <= 512) e = launch_cta<128, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, st);
    else if (m <= 1024) e = launch_cta<256, 4>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, st);
    else if (m <= 2048) e = launch_cta<256, 8>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, st);
    else if (m <= 4096) e = launch_cta<256, 16>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, st);
    else if (m <= kCtaCapacity) e = launch_cta<kClusterThreads, kClusterP>(num_clouds, pos, ptr, k_per_cloud, tie_break, out_idx, st);
    else {
        const int cs = (int)((m + kCtaCapacity - 1) / kCtaCapacity);
        e = cudaErrorInvalidConfiguration;
        if (cs <= 16) e = launch_cluster(num_clouds, cs, pos, ptr, k_per_cloud, tie_break, out_idx, st);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();  // clear a refused cluster launch, use the streaming kernel
            GDL_RETURN_IF(!workspace || workspace_bytes < sizeof(float) * (size_t)n_points, GDL_ERR_WORKSPACE);
            fps_stream_kernel<<<num_clouds, kStreamThreads, 0, st>>>(pos, ptr, k_per_cloud, tie_break,
                                                                     (float *)workspace, out_idx);
            e = cudaGetLastError();
        }
    }
    return e == cudaSuccess ? GDL_OK : GDL_ERR_CUDA;
}
