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

// Writes edge e's geometry from the destination position (qx, qy, qz) and the source's.
__device__ __forceinline__ void edge_geom_store(const EdgeGeom &g, int64_t e, float qx, float qy, float qz, float sx,
                                                float sy, float sz) {
    const float dx = __fsub_rn(qx, sx), dy = __fsub_rn(qy, sy), dz = __fsub_rn(qz, sz);
    const float n = __fsqrt_rn(__fmaf_rn(dz, dz, __fmaf_rn(dy, dy, __fmul_rn(dx, dx))));
    const float d = n < 1e-8f ? 1e-8f : n;  // clamp(min=1e-8); NaN stays NaN
    if (g.diff) {
        g.diff[3 * e] = dx;
        g.diff[3 * e + 1] = dy;
        g.diff[3 * e + 2] = dz;
    }
    if (g.dist) g.dist[e] = d;
    if (g.dir || g.sph) {
        const float ux = __fdiv_rn(dx, d), uy = __fdiv_rn(dy, d), uz = __fdiv_rn(dz, d);
        if (g.dir) {
            g.dir[3 * e] = ux;
            g.dir[3 * e + 1] = uy;
            g.dir[3 * e + 2] = uz;
        }
        if (g.sph) sph_store(g.sph + e * g.sph_dim, g.sph_dim, ux, uy, uz);
    }
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
