// geom.cuh -- edge geometry written where an edge is emitted (sm_100a).
//
// For an edge (src -> dst) of a point graph the reference computes, with torch ops after the
// graph is built (functional/radius_graph.py:338-358, nn/modules/spatial_graph.py:126-129):
//   diff = x[dst] - x[src]
//   dist = |diff| clamped below at 1e-8
//   dir  = diff / dist
//   Y    = real spherical harmonics of dir up to degree 2 (kernels/triton_sph_harm.py:200-240)
// Each value below is rounded exactly as that torch evaluation rounds it on the CPU: IEEE
// single precision, no flush to zero, |diff| = sqrt(fma(dz, dz, fma(dy, dy, dx * dx))) (the
// accumulation torch's 2-norm performs over a row of three), one rounding per torch op of the
// harmonics, constants rounded to float before use.
#pragma once

#include "common.cuh"

namespace gdl {

struct EdgeGeom {
    const float *x;  // [n_points, 3]; nullptr: no geometry is written
    float *diff;     // [E, 3] (nullable)
    float *dist;     // [E] (nullable)
    float *dir;      // [E, 3] (nullable)
    float *sph;      // [E, sph_dim] (nullable)
    int sph_dim;     // 1, 4 or 9 when sph is set
};

// float(sqrt((2l+1)/(4 pi) * (l-|m|)!/(l+|m|)!)) for the components l <= 2 uses
constexpr float kShC0 = 0x1.20dd76p-2f;   // l = 0
constexpr float kShC1 = 0x1.f45438p-2f;   // l = 1
constexpr float kShC20 = 0x1.42f602p-2f;  // l = 2, m = 0: sqrt(5 / (16 pi))
constexpr float kShC21 = 0x1.17b142p+0f;  // l = 2, |m| = 1 (and the xy term): sqrt(15 / (4 pi))
constexpr float kShC22 = 0x1.17b142p-1f;  // l = 2, m = 2: sqrt(15 / (16 pi))

// Channel layout [Y00 | Y1-1 Y10 Y11 | Y2-2 Y2-1 Y20 Y21 Y22] = [c0 | c1 y, c1 z, c1 x |
// c21 x y, c21 y z, c20 (3 z z - 1), c21 x z, c22 (x x - y y)], evaluated left to right.
__device__ __forceinline__ void sph_store(float *__restrict__ o, int dim, float x, float y, float z) {
    o[0] = kShC0;
    if (dim == 1) return;
    o[1] = __fmul_rn(kShC1, y);
    o[2] = __fmul_rn(kShC1, z);
    o[3] = __fmul_rn(kShC1, x);
    if (dim == 4) return;
    o[4] = __fmul_rn(__fmul_rn(kShC21, x), y);
    o[5] = __fmul_rn(__fmul_rn(kShC21, y), z);
    o[6] = __fmul_rn(kShC20, __fsub_rn(__fmul_rn(__fmul_rn(3.0f, z), z), 1.0f));
    o[7] = __fmul_rn(__fmul_rn(kShC21, x), z);
    o[8] = __fmul_rn(kShC22, __fsub_rn(__fmul_rn(x, x), __fmul_rn(y, y)));
}

// Per-warp staging for warp_geom_emit: dist [32] | direction [32 x 3] | diff [32 x 3] |
// harmonics [32 x 9] floats.
constexpr int kGeomStageFloats = 32 + 96 + 96 + 288;

// Geometry of `cnt` <= 32 consecutive edge slots e0 .. e0 + cnt - 1, lane i holding slot e0 + i
// (destination q, source s). The values go through the warp's staging area `st` so that every
// output array is written by consecutive lanes at consecutive addresses: the rows of the [E, 3]
// and [E, 9] arrays are 12 and 36 bytes long, and lane-per-row stores would touch up to eight
// times the 32-byte sectors they fill. All lanes call it (warp-uniform e0, cnt).
__device__ __forceinline__ void warp_geom_emit(const EdgeGeom &g, float *__restrict__ st, int64_t e0, int cnt,
                                               int lane, float qx, float qy, float qz, float sx, float sy,
                                               float sz) {
    float *s_dist = st, *s_dir = st + 32, *s_diff = st + 128, *s_sph = st + 224;
    if (lane < cnt) {
        const float dx = __fsub_rn(qx, sx), dy = __fsub_rn(qy, sy), dz = __fsub_rn(qz, sz);
        const float n = __fsqrt_rn(__fmaf_rn(dz, dz, __fmaf_rn(dy, dy, __fmul_rn(dx, dx))));
        const float d = n < 1e-8f ? 1e-8f : n;  // clamp(min=1e-8); NaN stays NaN
        const float ux = __fdiv_rn(dx, d), uy = __fdiv_rn(dy, d), uz = __fdiv_rn(dz, d);
        s_dist[lane] = d;
        s_dir[3 * lane] = ux;
        s_dir[3 * lane + 1] = uy;
        s_dir[3 * lane + 2] = uz;
        s_diff[3 * lane] = dx;
        s_diff[3 * lane + 1] = dy;
        s_diff[3 * lane + 2] = dz;
        if (g.sph) sph_store(s_sph + g.sph_dim * lane, g.sph_dim, ux, uy, uz);
    }
    __syncwarp();
    if (g.dist)
        for (int f = lane; f < cnt; f += 32) g.dist[e0 + f] = s_dist[f];
    if (g.dir)
        for (int f = lane; f < 3 * cnt; f += 32) g.dir[3 * e0 + f] = s_dir[f];
    if (g.diff)
        for (int f = lane; f < 3 * cnt; f += 32) g.diff[3 * e0 + f] = s_diff[f];
    if (g.sph)
        for (int f = lane; f < g.sph_dim * cnt; f += 32) g.sph[g.sph_dim * e0 + f] = s_sph[f];
    __syncwarp();
}

// Builds the device-side descriptor from the C-ABI one (nullptr: no geometry).
inline EdgeGeom edge_geom_from(const float *x, const gdl_edge_geometry *g) {
    EdgeGeom r{nullptr, nullptr, nullptr, nullptr, nullptr, 0};
    if (!g || !(g->diff || g->dist || g->direction || g->sph)) return r;
    r.x = x;
    r.diff = g->diff;
    r.dist = g->dist;
    r.dir = g->direction;
    r.sph = g->sph;
    r.sph_dim = g->sph ? (g->sph_max_l + 1) * (g->sph_max_l + 1) : 0;
    return r;
}

inline bool edge_geom_valid(const gdl_edge_geometry *g) {
    return !g || !g->sph || (g->sph_max_l >= 0 && g->sph_max_l <= 2);
}

}  // namespace gdl
