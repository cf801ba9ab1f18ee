// se3_aggregate.cu -- SE3Conv messages computed inside the segment reduction (sm_100a).
//
// The reference's SE3Conv (nn/modules/se3_conv.py:61-235, 487-545) gathers the source features
// of every edge, runs the nine tensor-product paths per edge (matmuls over the input channels,
// products with the radial weights R, the direction d, Y_0 and the l = 2 harmonics Y_2), writes
// the [E, C_s + 3 C_v + 5 C_t2] messages, reduces them per target with segment_reduce and
// divides by the cloud's average degree. Every path is linear in the source features, so the
// channel mixing can run once per NODE instead of once per edge: with node projections
//   P0 = s W_ss^T [N,Cs]     P1 = s W_sv^T [N,Cv]     P2 = W_vv v [N,Cv,3]    P3 = W_vs v [N,Cs,3]
//   P4 = W_x v [N,Cv,3]      P5 = s W_st2^T [N,Ct2]   P6 = W_t2t2 t2 [N,Ct2,5]
//   P7 = W_vt2 v [N,Ct2,3]   P8 = |t2|^2 W_t2s^T [N,Cs]
// (plain GEMMs, done by the caller), an edge's message is a handful of products of its source's
// projections with (R, d, Y_0, Y_2), e.g. path 3 (d . v -> s): R3 sum_k d_k P3[o, k]; path 4
// (d x v -> v): R4 (d x P4[o]); path 7 (d (x) v -> t2 through CG(1,1,2)): R7 sum_ij d_i P7[o, j]
// CG[i, j, m]. This kernel forms those messages while it reduces each target's segment, so no
// [E, C] message exists. Backward: gradients w.r.t. the projections (grouped by source over a
// source-sorted edge list, deterministic) and w.r.t. R (one warp per edge).
#include "common.cuh"

namespace gdl {

struct Se3Paths {
    const float *p[9];
    int rc[9];      // R column of each path (-1: path off)
    int64_t ld[9];  // floats between consecutive nodes' rows of each projection
    int cs, cv, ct2;
};

struct Se3Edge {  // per-edge values shared by all channels of the edge
    float r[9];
    float d[3];
    float y0;
    float y2[5];
};

__device__ __forceinline__ void load_edge(const Se3Paths &P, const float *__restrict__ R, int64_t rs,
                                          const float *__restrict__ dir, const float *__restrict__ sph, int sd,
                                          int64_t e, Se3Edge &x) {
#pragma unroll
    for (int p = 0; p < 9; ++p) x.r[p] = P.rc[p] >= 0 ? R[e * rs + P.rc[p]] : 0.0f;
    x.d[0] = dir[3 * e];
    x.d[1] = dir[3 * e + 1];
    x.d[2] = dir[3 * e + 2];
    x.y0 = sph[e * sd];
#pragma unroll
    for (int m = 0; m < 5; ++m) x.y2[m] = sd >= 9 ? sph[e * sd + 4 + m] : 0.0f;
}

// lane t's edge values, to every lane (the edges of a segment are loaded 32 at a time, one per
// lane, so that their loads overlap instead of forming a dependent chain per edge)
__device__ __forceinline__ void shfl_edge(const Se3Edge &m, int t, Se3Edge &x) {
#pragma unroll
    for (int p = 0; p < 9; ++p) x.r[p] = __shfl_sync(0xffffffffu, m.r[p], t);
#pragma unroll
    for (int k = 0; k < 3; ++k) x.d[k] = __shfl_sync(0xffffffffu, m.d[k], t);
    x.y0 = __shfl_sync(0xffffffffu, m.y0, t);
#pragma unroll
    for (int k = 0; k < 5; ++k) x.y2[k] = __shfl_sync(0xffffffffu, m.y2[k], t);
}

__device__ __forceinline__ void zero_edge(Se3Edge &x) {
#pragma unroll
    for (int p = 0; p < 9; ++p) x.r[p] = 0.0f;
    x.d[0] = x.d[1] = x.d[2] = x.y0 = 0.0f;
#pragma unroll
    for (int k = 0; k < 5; ++k) x.y2[k] = 0.0f;
}

// Term of path p in the message of an edge from source s: scalar channel o (paths 0, 3, 8),
// vector channel (o, k) (paths 1, 2, 4), type-2 channel (o, m) (paths 5, 6, 7).
__device__ __forceinline__ float se3_term_s(const Se3Paths &P, const Se3Edge &x, int64_t s, int o, int p) {
    if (p == 0) return __fmul_rn(__fmul_rn(x.r[0], x.y0), P.p[0][s * P.ld[0] + o]);
    if (p == 3) {
        const float *q = P.p[3] + s * P.ld[3] + o * 3;
        const float dot =
            __fadd_rn(__fadd_rn(__fmul_rn(x.d[0], q[0]), __fmul_rn(x.d[1], q[1])), __fmul_rn(x.d[2], q[2]));
        return __fmul_rn(x.r[3], dot);
    }
    if (p == 8) return __fmul_rn(x.r[8], P.p[8][s * P.ld[8] + o]);
    return 0.0f;
}

__device__ __forceinline__ float se3_term_v(const Se3Paths &P, const Se3Edge &x, int64_t s, int o, int k, int p) {
    if (p == 1) return __fmul_rn(__fmul_rn(x.r[1], P.p[1][s * P.ld[1] + o]), x.d[k]);
    if (p == 2) return __fmul_rn(__fmul_rn(x.r[2], x.y0), P.p[2][s * P.ld[2] + o * 3 + k]);
    if (p == 4) {
        const float *q = P.p[4] + s * P.ld[4] + o * 3;
        const int k1 = k == 2 ? 0 : k + 1, k2 = k == 0 ? 2 : k - 1;  // (d x q)_k = d_k1 q_k2 - d_k2 q_k1
        return __fmul_rn(x.r[4], __fsub_rn(__fmul_rn(x.d[k1], q[k2]), __fmul_rn(x.d[k2], q[k1])));
    }
    return 0.0f;
}

__device__ __forceinline__ float se3_term_t(const Se3Paths &P, const float *__restrict__ cg, const Se3Edge &x,
                                            int64_t s, int o, int m, int p) {
    if (p == 5) return __fmul_rn(__fmul_rn(x.r[5], P.p[5][s * P.ld[5] + o]), x.y2[m]);
    if (p == 6) return __fmul_rn(__fmul_rn(x.r[6], x.y0), P.p[6][s * P.ld[6] + o * 5 + m]);
    if (p == 7) {
        const float *q = P.p[7] + s * P.ld[7] + o * 3;
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) t = __fadd_rn(t, __fmul_rn(__fmul_rn(x.d[i], q[j]), cg[(i * 3 + j) * 5 + m]));
        return __fmul_rn(x.r[7], t);
    }
    return 0.0f;
}

// the message of one channel of kind KIND (0 scalar, 1 vector, 2 type-2; fl indexes that kind's
// channels): the active paths' terms added in the reference's path order (scalars 0, 3, 8;
// vectors 1, 2, 4; type-2 5, 6, 7)
template <int KIND>
__device__ __forceinline__ float se3_message_kind(const Se3Paths &P, const float *__restrict__ cg, const Se3Edge &x,
                                                  int64_t s, int fl) {
    float msg = 0.0f;
    if constexpr (KIND == 0) {
        if (P.p[0]) msg = __fadd_rn(msg, se3_term_s(P, x, s, fl, 0));
        if (P.p[3]) msg = __fadd_rn(msg, se3_term_s(P, x, s, fl, 3));
        if (P.p[8]) msg = __fadd_rn(msg, se3_term_s(P, x, s, fl, 8));
    } else if constexpr (KIND == 1) {
        const int o = fl / 3, k = fl - 3 * o;
        if (P.p[1]) msg = __fadd_rn(msg, se3_term_v(P, x, s, o, k, 1));
        if (P.p[2]) msg = __fadd_rn(msg, se3_term_v(P, x, s, o, k, 2));
        if (P.p[4]) msg = __fadd_rn(msg, se3_term_v(P, x, s, o, k, 4));
    } else {
        const int o = fl / 5, m = fl - 5 * o;
        if (P.p[5]) msg = __fadd_rn(msg, se3_term_t(P, cg, x, s, o, m, 5));
        if (P.p[6]) msg = __fadd_rn(msg, se3_term_t(P, cg, x, s, o, m, 6));
        if (P.p[7]) msg = __fadd_rn(msg, se3_term_t(P, cg, x, s, o, m, 7));
    }
    return msg;
}

constexpr int kSe3Chunks = 4;  // output channels per lane held in registers (128 per warp pass)

// the channels of one kind for target n: lanes over channels (kSe3Chunks per lane per pass), the
// segment's edges in slot order, each message formed on the fly, the fold divided by the degree
template <int KIND>
__device__ __forceinline__ void fwd_kind_pass(const Se3Paths &P, const float *__restrict__ R, int64_t rs,
                                              const float *__restrict__ dir, const float *__restrict__ sph, int sd,
                                              const float *__restrict__ cg, const int64_t *__restrict__ row,
                                              const int32_t *__restrict__ perm, int32_t j0, int32_t j1, bool single,
                                              Se3Edge &mine, int64_t &msrc, int64_t n, float a,
                                              float *__restrict__ out, int width, int lane) {
    for (int c0 = 0; c0 < width; c0 += 32 * kSe3Chunks) {
        float acc[kSe3Chunks];
#pragma unroll
        for (int i = 0; i < kSe3Chunks; ++i) acc[i] = 0.0f;
        for (int32_t jb = j0; jb < j1; jb += 32) {  // up to 32 edges: lane t loads edge jb + t
            const int cnt = j1 - jb < 32 ? (int)(j1 - jb) : 32;
            if (!single) {
                msrc = 0;
                zero_edge(mine);
                if (lane < cnt) {
                    const int64_t e = perm[jb + lane];
                    msrc = row[e];
                    load_edge(P, R, rs, dir, sph, sd, e, mine);
                }
            }
            for (int t = 0; t < cnt; ++t) {  // slot order is kept: edges are folded one by one
                Se3Edge x;
                shfl_edge(mine, t, x);
                const int64_t s = __shfl_sync(0xffffffffu, msrc, t);
#pragma unroll
                for (int i = 0; i < kSe3Chunks; ++i) {
                    const int f = c0 + lane + 32 * i;
                    if (f < width) acc[i] = __fadd_rn(acc[i], se3_message_kind<KIND>(P, cg, x, s, f));
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kSe3Chunks; ++i) {
            const int f = c0 + lane + 32 * i;
            if (f < width) out[n * width + f] = __fdiv_rn(acc[i], a);
        }
    }
}

// one warp per target node; its three channel kinds in turn, edges of the segment in sorted-slot
// order, messages formed on the fly
__global__ void __launch_bounds__(256, 3) se3_agg_fwd_kernel(Se3Paths P, const float *__restrict__ R, int64_t rs,
                                                          const float *__restrict__ dir, const float *__restrict__ sph,
                                                          int sd, const float *__restrict__ cg,
                                                          const int64_t *__restrict__ row,
                                                          const int32_t *__restrict__ perm,
                                                          const int32_t *__restrict__ ns,
                                                          const int32_t *__restrict__ ne,
                                                          const float *__restrict__ avg, int64_t N,
                                                          float *__restrict__ os, float *__restrict__ ov,
                                                          float *__restrict__ ot) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t n = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
        const int32_t j0 = ns[n], j1 = ne[n];
        const float a = avg[n];
        // a segment of at most 32 edges (the usual case) is loaded once for all channel passes
        const bool single = j1 - j0 <= 32;
        Se3Edge mine;
        int64_t msrc = 0;
        zero_edge(mine);
        if (single && lane < j1 - j0) {
            const int64_t e = perm[j0 + lane];
            msrc = row[e];
            load_edge(P, R, rs, dir, sph, sd, e, mine);
        }
        fwd_kind_pass<0>(P, R, rs, dir, sph, sd, cg, row, perm, j0, j1, single, mine, msrc, n, a, os, P.cs, lane);
        fwd_kind_pass<1>(P, R, rs, dir, sph, sd, cg, row, perm, j0, j1, single, mine, msrc, n, a, ov, 3 * P.cv,
                         lane);
        fwd_kind_pass<2>(P, R, rs, dir, sph, sd, cg, row, perm, j0, j1, single, mine, msrc, n, a, ot, 5 * P.ct2,
                         lane);
    }
}

// -------------------------------------------------------------------- backward
// g = grad_out[target] / avg[target] for channel f of the flattened output
__device__ __forceinline__ float grad_at(const float *__restrict__ gs, const float *__restrict__ gv,
                                         const float *__restrict__ gt, const Se3Paths &P, int64_t t, int f) {
    if (f < P.cs) return gs[t * P.cs + f];
    f -= P.cs;
    if (f < 3 * P.cv) return gv[t * 3 * P.cv + f];
    f -= 3 * P.cv;
    return gt[t * 5 * P.ct2 + f];
}

// grad_R[e, rc[p]] = sum over output channels f of g[f] * (path p's term of channel f without R_p).
// One warp per edge; the nine sums are lane-strided, then reduced with a fixed butterfly.
template <bool DIV>
__global__ void __launch_bounds__(256) se3_agg_grad_r_kernel(Se3Paths P, const float *__restrict__ R, int64_t rs,
                                                             const float *__restrict__ dir,
                                                             const float *__restrict__ sph, int sd,
                                                             const float *__restrict__ cg,
                                                             const int64_t *__restrict__ row,
                                                             const int64_t *__restrict__ col,
                                                             const float *__restrict__ avg, int64_t E,
                                                             const float *__restrict__ gs,
                                                             const float *__restrict__ gv,
                                                             const float *__restrict__ gt, float *__restrict__ gR) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t e = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < E; e += warps) {
        const int64_t s = row[e], t = col[e];
        const float a = DIV ? avg[t] : 1.0f;
        Se3Edge x;
        load_edge(P, R, rs, dir, sph, sd, e, x);
        Se3Edge one = x;  // unit radial weights: each path's term without its R
#pragma unroll
        for (int p = 0; p < 9; ++p) one.r[p] = 1.0f;
        float part[9];
#pragma unroll
        for (int p = 0; p < 9; ++p) part[p] = 0.0f;
        // lane-strided over each channel kind in turn; a kind feeds only its three paths
        for (int o = lane; o < P.cs; o += 32) {
            const float g = DIV ? __fdiv_rn(gs[t * P.cs + o], a) : gs[t * P.cs + o];
            if (P.p[0]) part[0] = __fadd_rn(part[0], __fmul_rn(g, se3_term_s(P, one, s, o, 0)));
            if (P.p[3]) part[3] = __fadd_rn(part[3], __fmul_rn(g, se3_term_s(P, one, s, o, 3)));
            if (P.p[8]) part[8] = __fadd_rn(part[8], __fmul_rn(g, se3_term_s(P, one, s, o, 8)));
        }
        for (int f = lane; f < 3 * P.cv; f += 32) {
            const float g = DIV ? __fdiv_rn(gv[t * 3 * P.cv + f], a) : gv[t * 3 * P.cv + f];
            const int o = f / 3, k = f - 3 * o;
            if (P.p[1]) part[1] = __fadd_rn(part[1], __fmul_rn(g, se3_term_v(P, one, s, o, k, 1)));
            if (P.p[2]) part[2] = __fadd_rn(part[2], __fmul_rn(g, se3_term_v(P, one, s, o, k, 2)));
            if (P.p[4]) part[4] = __fadd_rn(part[4], __fmul_rn(g, se3_term_v(P, one, s, o, k, 4)));
        }
        for (int f = lane; f < 5 * P.ct2; f += 32) {
            const float g = DIV ? __fdiv_rn(gt[t * 5 * P.ct2 + f], a) : gt[t * 5 * P.ct2 + f];
            const int o = f / 5, m = f - 5 * o;
            if (P.p[5]) part[5] = __fadd_rn(part[5], __fmul_rn(g, se3_term_t(P, cg, one, s, o, m, 5)));
            if (P.p[6]) part[6] = __fadd_rn(part[6], __fmul_rn(g, se3_term_t(P, cg, one, s, o, m, 6)));
            if (P.p[7]) part[7] = __fadd_rn(part[7], __fmul_rn(g, se3_term_t(P, cg, one, s, o, m, 7)));
        }
#pragma unroll
        for (int p = 0; p < 9; ++p) {
            if (P.rc[p] < 0) continue;
            float v = part[p];
            for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0) gR[e * rs + P.rc[p]] = v;
        }
    }
}

struct Se3Grads {
    float *g[9];
};

// sizes of the nine projection rows: 0 cs, 1 cv, 2 3cv, 3 3cs, 4 3cv, 5 ct2, 6 5ct2, 7 3ct2, 8 cs
__device__ __forceinline__ int proj_width(const Se3Paths &P, int p) {
    switch (p) {
        case 0: return P.cs;
        case 1: return P.cv;
        case 2: return 3 * P.cv;
        case 3: return 3 * P.cs;
        case 4: return 3 * P.cv;
        case 5: return P.ct2;
        case 6: return 5 * P.ct2;
        case 7: return 3 * P.ct2;
        default: return P.cs;
    }
}

// d(message) / d(projection p entry q) contracted with g over the channels that entry feeds
template <bool DIV>
__device__ __forceinline__ float proj_grad_term(const Se3Paths &P, const float *__restrict__ cg, const Se3Edge &x,
                                                const float *__restrict__ gs, const float *__restrict__ gv,
                                                const float *__restrict__ gt, int64_t t, float a, int p, int q) {
    auto G = [&](int f) {
        const float g = grad_at(gs, gv, gt, P, t, f);
        return DIV ? __fdiv_rn(g, a) : g;
    };
    switch (p) {
        case 0: return __fmul_rn(__fmul_rn(x.r[0], x.y0), G(q));
        case 3: {
            const int o = q / 3, k = q - 3 * o;
            return __fmul_rn(__fmul_rn(x.r[3], x.d[k]), G(o));
        }
        case 8: return __fmul_rn(x.r[8], G(q));
        case 1: {
            const int b = P.cs + 3 * q;
            float sacc = 0.0f;
#pragma unroll
            for (int k = 0; k < 3; ++k) sacc = __fadd_rn(sacc, __fmul_rn(x.d[k], G(b + k)));
            return __fmul_rn(x.r[1], sacc);
        }
        case 2: return __fmul_rn(__fmul_rn(x.r[2], x.y0), G(P.cs + q));
        case 4: {  // (g_v[o] x d)_j
            const int o = q / 3, j = q - 3 * o;
            const int j1 = j == 2 ? 0 : j + 1, j2 = j == 0 ? 2 : j - 1;
            const int b = P.cs + 3 * o;
            const float cr = __fsub_rn(__fmul_rn(G(b + j1), x.d[j2]), __fmul_rn(G(b + j2), x.d[j1]));
            return __fmul_rn(x.r[4], cr);
        }
        case 5: {
            const int b = P.cs + 3 * P.cv + 5 * q;
            float sacc = 0.0f;
#pragma unroll
            for (int m = 0; m < 5; ++m) sacc = __fadd_rn(sacc, __fmul_rn(x.y2[m], G(b + m)));
            return __fmul_rn(x.r[5], sacc);
        }
        case 6: return __fmul_rn(__fmul_rn(x.r[6], x.y0), G(P.cs + 3 * P.cv + q));
        default: {  // 7: sum_m (sum_i d_i CG[i, j, m]) g_t[o, m]
            const int o = q / 3, j = q - 3 * o;
            const int b = P.cs + 3 * P.cv + 5 * o;
            float sacc = 0.0f;
#pragma unroll
            for (int m = 0; m < 5; ++m) {
                float c = 0.0f;
#pragma unroll
                for (int i = 0; i < 3; ++i) c = __fadd_rn(c, __fmul_rn(x.d[i], cg[(i * 3 + j) * 5 + m]));
                sacc = __fadd_rn(sacc, __fmul_rn(c, G(b + m)));
            }
            return __fmul_rn(x.r[7], sacc);
        }
    }
}

// one projection's gradient rows for source s (PI fixed at compile time, so that the inner loop
// holds only that projection's term)
template <int PI, bool DIV>
__device__ __forceinline__ void grad_p_pass(const Se3Paths &P, float *__restrict__ gp, const float *__restrict__ R,
                                            int64_t rs, const float *__restrict__ dir,
                                            const float *__restrict__ sph, int sd, const float *__restrict__ cg,
                                            const int64_t *__restrict__ col, const int32_t *__restrict__ sperm,
                                            const float *__restrict__ avg, const float *__restrict__ gs,
                                            const float *__restrict__ gv, const float *__restrict__ gt,
                                            int64_t s, int32_t j0, int32_t j1, bool single, Se3Edge &mine,
                                            int64_t &mt, float &ma, int lane) {
    const int w = proj_width(P, PI);
    for (int q0 = 0; q0 < w; q0 += 32 * kSe3Chunks) {
        float acc[kSe3Chunks];
#pragma unroll
        for (int i = 0; i < kSe3Chunks; ++i) acc[i] = 0.0f;
        for (int32_t jb = j0; jb < j1; jb += 32) {  // lane u loads out-edge jb + u
            const int cnt = j1 - jb < 32 ? (int)(j1 - jb) : 32;
            if (!single) {
                mt = 0;
                ma = 1.0f;
                zero_edge(mine);
                if (lane < cnt) {
                    const int64_t e = sperm[jb + lane];
                    mt = col[e];
                    ma = DIV ? avg[mt] : 1.0f;
                    load_edge(P, R, rs, dir, sph, sd, e, mine);
                }
            }
            for (int u = 0; u < cnt; ++u) {
                Se3Edge x;
                shfl_edge(mine, u, x);
                const int64_t t = __shfl_sync(0xffffffffu, mt, u);
                const float a = __shfl_sync(0xffffffffu, ma, u);
#pragma unroll
                for (int i = 0; i < kSe3Chunks; ++i) {
                    const int q = q0 + lane + 32 * i;
                    if (q < w) acc[i] = __fadd_rn(acc[i], proj_grad_term<DIV>(P, cg, x, gs, gv, gt, t, a, PI, q));
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kSe3Chunks; ++i) {
            const int q = q0 + lane + 32 * i;
            if (q < w) gp[s * P.ld[PI] + q] = acc[i];
        }
    }
}

// grad of every projection entry of source node s: one warp per source, its out-edges in
// source-sorted order (deterministic), lanes over the entries of one projection at a time
template <bool DIV>
__global__ void __launch_bounds__(256, 3) se3_agg_grad_p_kernel(Se3Paths P, Se3Grads Gp, const float *__restrict__ R,
                                                             int64_t rs, const float *__restrict__ dir,
                                                             const float *__restrict__ sph, int sd,
                                                             const float *__restrict__ cg,
                                                             const int64_t *__restrict__ col,
                                                             const int32_t *__restrict__ sperm,
                                                             const int32_t *__restrict__ sns,
                                                             const int32_t *__restrict__ sne,
                                                             const float *__restrict__ avg, int64_t N,
                                                             const float *__restrict__ gs,
                                                             const float *__restrict__ gv,
                                                             const float *__restrict__ gt) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t s = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); s < N; s += warps) {
        const int32_t j0 = sns[s], j1 = sne[s];
        // at most 32 out-edges (the usual case): loaded once for all projections and passes
        const bool single = j1 - j0 <= 32;
        Se3Edge mine;
        int64_t mt = 0;
        float ma = 1.0f;
        zero_edge(mine);
        if (single && lane < j1 - j0) {
            const int64_t e = sperm[j0 + lane];
            mt = col[e];
            ma = DIV ? avg[mt] : 1.0f;
            load_edge(P, R, rs, dir, sph, sd, e, mine);
        }
#define GDL_SE3_PASS(PI)                                                                                          \
    if (Gp.g[PI])                                                                                                 \
        grad_p_pass<PI, DIV>(P, Gp.g[PI], R, rs, dir, sph, sd, cg, col, sperm, avg, gs, gv, gt, s, j0, j1, single, mine, \
                        mt, ma, lane);
        GDL_SE3_PASS(0)
        GDL_SE3_PASS(1)
        GDL_SE3_PASS(2)
        GDL_SE3_PASS(3)
        GDL_SE3_PASS(4)
        GDL_SE3_PASS(5)
        GDL_SE3_PASS(6)
        GDL_SE3_PASS(7)
        GDL_SE3_PASS(8)
#undef GDL_SE3_PASS
    }
}

inline unsigned se3_grid(int64_t warps_needed) {
    int64_t b = (warps_needed + 7) / 8;
    const int64_t cap = (int64_t)kSmCount * 16;
    return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

inline bool se3_paths_ok(const gdl_se3_paths *g, Se3Paths *P) {
    if (!g || g->cs < 0 || g->cv < 0 || g->ct2 < 0) return false;
    P->cs = (int)g->cs;
    P->cv = (int)g->cv;
    P->ct2 = (int)g->ct2;
    const int64_t dense[9] = {g->cs, g->cv, 3 * g->cv, 3 * g->cs, 3 * g->cv, g->ct2, 5 * g->ct2, 3 * g->ct2, g->cs};
    for (int p = 0; p < 9; ++p) {
        P->p[p] = g->p[p];
        P->rc[p] = g->p[p] ? g->r_col[p] : -1;
        P->ld[p] = g->ld[p] > 0 ? g->ld[p] : dense[p];
        if (g->p[p] && (g->r_col[p] < 0 || P->ld[p] < dense[p])) return false;
    }
    return true;
}

}  // namespace gdl

using namespace gdl;

extern "C" int gdl_se3_aggregate(const gdl_se3_paths *paths, const float *R, int64_t r_stride, const float *direction,
                                 const float *sph, int32_t sph_dim, const float *cg, const int64_t *row,
                                 const int32_t *perm, const int32_t *node_start, const int32_t *node_end,
                                 const float *avg_degree, int64_t n_nodes, int64_t n_edges, float *out_s, float *out_v,
                                 float *out_t2, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    Se3Paths P;
    GDL_RETURN_IF(!se3_paths_ok(paths, &P) || n_nodes < 0 || n_edges < 0 || sph_dim < 1, GDL_ERR_INVALID);
    for (int p = 0; p < 9; ++p) GDL_RETURN_IF(P.rc[p] >= r_stride, GDL_ERR_INVALID);
    if (n_nodes == 0) return GDL_OK;
    GDL_RETURN_IF(!node_start || !node_end || !avg_degree, GDL_ERR_INVALID);
    GDL_RETURN_IF((P.cs && !out_s) || (P.cv && !out_v) || (P.ct2 && !out_t2), GDL_ERR_INVALID);
    GDL_RETURN_IF(n_edges > 0 && (!R || !direction || !sph || !row || !perm), GDL_ERR_INVALID);
    GDL_RETURN_IF((P.p[7] && !cg) || ((P.p[5]) && sph_dim < 9), GDL_ERR_INVALID);
    se3_agg_fwd_kernel<<<se3_grid(n_nodes), 256, 0, st>>>(P, R, r_stride, direction, sph, sph_dim, cg, row, perm,
                                                          node_start, node_end, avg_degree, n_nodes, out_s, out_v,
                                                          out_t2);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_se3_aggregate_backward(const gdl_se3_paths *paths, float *const *grad_proj, float *grad_R,
                                          const float *grad_s, const float *grad_v, const float *grad_t2,
                                          const float *R, int64_t r_stride, const float *direction, const float *sph,
                                          int32_t sph_dim, const float *cg, const int64_t *row, const int64_t *col,
                                          const int32_t *src_perm, const int32_t *src_start, const int32_t *src_end,
                                          const float *avg_degree, int64_t n_nodes, int64_t n_edges, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    Se3Paths P;
    GDL_RETURN_IF(!se3_paths_ok(paths, &P) || n_nodes < 0 || n_edges < 0 || sph_dim < 1, GDL_ERR_INVALID);
    GDL_RETURN_IF((P.cs && !grad_s) || (P.cv && !grad_v) || (P.ct2 && !grad_t2), GDL_ERR_INVALID);
    if (n_nodes == 0) return GDL_OK;
    GDL_RETURN_IF((P.p[7] && !cg) || ((P.p[5]) && sph_dim < 9), GDL_ERR_INVALID);
    if (grad_R && n_edges > 0) {
        GDL_RETURN_IF(!R || !direction || !sph || !row || !col, GDL_ERR_INVALID);
        if (avg_degree)
            se3_agg_grad_r_kernel<true><<<se3_grid(n_edges), 256, 0, st>>>(
                P, R, r_stride, direction, sph, sph_dim, cg, row, col, avg_degree, n_edges, grad_s, grad_v, grad_t2, grad_R);
        else
            se3_agg_grad_r_kernel<false><<<se3_grid(n_edges), 256, 0, st>>>(
                P, R, r_stride, direction, sph, sph_dim, cg, row, col, avg_degree, n_edges, grad_s, grad_v, grad_t2, grad_R);
    }
    if (grad_proj) {
        Se3Grads G;
        bool any = false;
        for (int p = 0; p < 9; ++p) {
            G.g[p] = P.p[p] ? grad_proj[p] : nullptr;
            any = any || G.g[p];
        }
        if (any) {
            GDL_RETURN_IF(!src_perm || !src_start || !src_end || (n_edges > 0 && (!R || !direction || !sph || !col)),
                          GDL_ERR_INVALID);
            if (avg_degree)
                se3_agg_grad_p_kernel<true><<<se3_grid(n_nodes), 256, 0, st>>>(
                    P, G, R, r_stride, direction, sph, sph_dim, cg, col, src_perm, src_start, src_end, avg_degree, n_nodes,
                    grad_s, grad_v, grad_t2);
            else
                se3_agg_grad_p_kernel<false><<<se3_grid(n_nodes), 256, 0, st>>>(
                    P, G, R, r_stride, direction, sph, sph_dim, cg, col, src_perm, src_start, src_end, avg_degree, n_nodes,
                    grad_s, grad_v, grad_t2);
        }
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
