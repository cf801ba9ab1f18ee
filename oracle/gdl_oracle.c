/*
 * gdl_oracle.c -- CPU restatement of GeoEmbodied's point-cloud graph operators.
 *
 * TEST INFRASTRUCTURE ONLY: this is the parity checker for the sm_100a kernels in
 * gdl_b200/csrc. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference leg may load it. The product never links or calls it.
 *
 * Every function restates the arithmetic of the reference CUDA kernels
 * (the .cu files under geoembodied/csrc in illusionaryshelter/GDL), including their rounding,
 * flush-to-zero (the reference builds with --use_fast_math, geoembodied/csrc/__init__.py:97-101),
 * heap tie behaviour and scan order, so that integer outputs are bit-identical.
 *
 * Squared-distance rounding is a parameter (dist_mode) because the reference has two
 * implementations whose rounding differs:
 *   GDL_DIST_TORCH  : the PyTorch CPU fallbacks, (dx*dx + dy*dy) + dz*dz, every op
 *                     rounded, no flush-to-zero (csrc/__init__.py:480-483, :645).
 *   GDL_DIST_FMA_*  : candidate contractions of `dx*dx + dy*dy + dz*dz` in the CUDA
 *                     kernels (fps_kernel.cu:91-94, knn_kernel.cu:149-152,
 *                     radius_graph_kernel.cu:224-227) with flush-to-zero; which one
 *                     nvcc produced is pinned on the GPU box against the reference's
 *                     returned KNN distances (tests/test_gpu_ref_pin.py).
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off -fno-fast-math, pthreads).
 */
#include <float.h>
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>
#include <stdatomic.h>
#include <unistd.h>

/* ---------------------------------------------------------------- thread pool
 * A dynamic parallel-for over [0, n) in chunks; the thread count defaults to the
 * online cores and can be set with gdl_oracle_set_num_threads().
 */
static int g_threads = 0;

typedef void (*body_fn)(int64_t i, void *ctx);
typedef struct {
    _Atomic int64_t next;
    int64_t n, chunk;
    body_fn fn;
    void *ctx;
} PoolJob;

static void *pool_worker(void *arg) {
    PoolJob *job = (PoolJob *)arg;
    for (;;) {
        int64_t i0 = atomic_fetch_add(&job->next, job->chunk);
        if (i0 >= job->n) break;
        int64_t i1 = i0 + job->chunk < job->n ? i0 + job->chunk : job->n;
        for (int64_t i = i0; i < i1; ++i) job->fn(i, job->ctx);
    }
    return NULL;
}

int gdl_oracle_num_threads(void) {
    if (g_threads <= 0) {
        long c = sysconf(_SC_NPROCESSORS_ONLN);
        g_threads = c > 0 ? (int)c : 1;
    }
    return g_threads;
}

void gdl_oracle_set_num_threads(int n) { g_threads = n; }

static void parallel_for(int64_t n, int64_t chunk, body_fn fn, void *ctx) {
    if (n <= 0) return;
    int t = gdl_oracle_num_threads();
    if ((int64_t)t > (n + chunk - 1) / chunk) t = (int)((n + chunk - 1) / chunk);
    PoolJob job;
    atomic_init(&job.next, 0);
    job.n = n; job.chunk = chunk; job.fn = fn; job.ctx = ctx;
    if (t <= 1) { pool_worker(&job); return; }
    pthread_t th[256];
    if (t > 256) t = 256;
    for (int j = 1; j < t; ++j) pthread_create(&th[j], NULL, pool_worker, &job);
    pool_worker(&job);
    for (int j = 1; j < t; ++j) pthread_join(th[j], NULL);
}

enum {
    GDL_DIST_TORCH = 0,     /* ((dx*dx + dy*dy) + dz*dz), no FTZ                  */
    GDL_DIST_FMA_ZYX = 1,   /* fma(dz,dz, fma(dy,dy, dx*dx)), FTZ                 */
    GDL_DIST_FMA_ZXY = 2,   /* fma(dz,dz, fma(dx,dx, dy*dy)), FTZ                 */
    GDL_DIST_FMA_Z_SUM = 3, /* fma(dz,dz, dx*dx + dy*dy), FTZ                      */
    GDL_DIST_NOFMA_FTZ = 4, /* ((dx*dx + dy*dy) + dz*dz), FTZ                      */
    GDL_DIST_FMA_XYZ = 5,   /* fma(dx,dx, fma(dy,dy, dz*dz)), FTZ                 */
};

enum { GDL_TIE_REFERENCE = 0, GDL_TIE_LOWEST_INDEX = 1 };
enum { GDL_REDUCE_SUM = 0, GDL_REDUCE_MEAN = 1, GDL_REDUCE_MAX = 2 };
enum { GDL_DTYPE_F32 = 0, GDL_DTYPE_BF16 = 1 };

/* ---------------------------------------------------------------- float helpers */

/* flush a subnormal to a signed zero (what .ftz does to operands and results) */
static inline float ftz(float x) { return (fabsf(x) < FLT_MIN) ? copysignf(0.0f, x) : x; }
static inline float sub_ftz(float a, float b) { return ftz(ftz(a) - ftz(b)); }
static inline float mul_ftz(float a, float b) { return ftz(ftz(a) * ftz(b)); }
static inline float add_ftz(float a, float b) { return ftz(ftz(a) + ftz(b)); }
static inline float fma_ftz(float a, float b, float c) { return ftz(fmaf(ftz(a), ftz(b), ftz(c))); }

static inline float dist2(float ax, float ay, float az, float bx, float by, float bz, int mode) {
    if (mode == GDL_DIST_TORCH) {
        float dx = ax - bx, dy = ay - by, dz = az - bz;
        float t = dx * dx, u = dy * dy, v = dz * dz;
        float s = t + u;
        return s + v;
    }
    float dx = sub_ftz(ax, bx), dy = sub_ftz(ay, by), dz = sub_ftz(az, bz);
    switch (mode) {
    case GDL_DIST_FMA_ZYX: return fma_ftz(dz, dz, fma_ftz(dy, dy, mul_ftz(dx, dx)));
    case GDL_DIST_FMA_ZXY: return fma_ftz(dz, dz, fma_ftz(dx, dx, mul_ftz(dy, dy)));
    case GDL_DIST_FMA_Z_SUM: return fma_ftz(dz, dz, add_ftz(mul_ftz(dx, dx), mul_ftz(dy, dy)));
    case GDL_DIST_NOFMA_FTZ: return add_ftz(add_ftz(mul_ftz(dx, dx), mul_ftz(dy, dy)), mul_ftz(dz, dz));
    case GDL_DIST_FMA_XYZ: return fma_ftz(dx, dx, fma_ftz(dy, dy, mul_ftz(dz, dz)));
    default: return NAN;
    }
}

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline int max_k_bucket_knn(int k) { /* knn_kernel.cu:253-288 */
    return k <= 4 ? 4 : k <= 8 ? 8 : k <= 16 ? 16 : k <= 32 ? 32 : 64;
}
static inline int max_k_bucket_radius(int k) { /* radius_graph_kernel.cu:372-420 */
    return k <= 16 ? 16 : k <= 32 ? 32 : 64;
}

/* ---------------------------------------------------------------- MinK heap
 * Restates MinK<K> (knn_kernel.cu:35-102, radius_graph_kernel.cu:34-85): a max-heap
 * that is filled unsorted until it holds K entries, heapified once, then replaces its
 * root when a strictly smaller distance arrives; ties keep the incumbent.
 */
typedef struct {
    float d[64];
    int i[64];
    int count;
    int cap;
} MinK;

static inline void mink_init(MinK *h, int cap) {
    h->count = 0;
    h->cap = cap;
    for (int j = 0; j < cap; ++j) { h->d[j] = 1e30f; h->i[j] = -1; }
}

static inline void mink_sift_down(MinK *h, int i) {
    const int K = h->cap;
    for (;;) {
        int l = 2 * i + 1, r = 2 * i + 2, g = i;
        if (l < K && h->d[l] > h->d[g]) g = l;
        if (r < K && h->d[r] > h->d[g]) g = r;
        if (g == i) break;
        float td = h->d[i]; h->d[i] = h->d[g]; h->d[g] = td;
        int ti = h->i[i]; h->i[i] = h->i[g]; h->i[g] = ti;
        i = g;
    }
}

static inline void mink_add(MinK *h, float d, int idx) {
    const int K = h->cap;
    if (h->count >= K && d >= h->d[0]) return;
    if (h->count >= K) {
        h->d[0] = d; h->i[0] = idx;
        mink_sift_down(h, 0);
    } else {
        h->d[h->count] = d; h->i[h->count] = idx;
        ++h->count;
        if (h->count == K)
            for (int j = K / 2 - 1; j >= 0; --j) mink_sift_down(h, j);
    }
}

static inline void mink_sort(MinK *h) { /* knn_kernel.cu:87-101, stable insertion sort */
    for (int a = 1; a < h->count; ++a) {
        float kd = h->d[a]; int ki = h->i[a];
        int b = a - 1;
        while (b >= 0 && h->d[b] > kd) { h->d[b + 1] = h->d[b]; h->i[b + 1] = h->i[b]; --b; }
        h->d[b + 1] = kd; h->i[b + 1] = ki;
    }
}

/* ---------------------------------------------------------------- FPS
 * fps_kernel.cu:54-152 (+ host :160-209). Seed = first point of the cloud; each step
 * min_d[p] = fminf(dist2(p, sel), min_d[p]) starting from 1e30, then sel = argmax.
 * Tie rule GDL_TIE_REFERENCE reproduces the kernel's reduction order: per thread
 * (tid = i % 512) the first strided point wins (`>` in ascending order, :102), the
 * shuffle-down tree (:111-118) and the shared-memory tree (:134-143) keep the left
 * operand on ties, which prefers lanes/warps in bit-reversed index order.
 * GDL_TIE_LOWEST_INDEX is torch.argmax's rule (csrc/__init__.py:648).
 * Output slots are laid out by cumsum(k) (fps_kernel.cu:177-180); a cloud with k > n
 * writes n indices and the remaining slots hold -1 (the reference leaves them unset).
 */
static inline uint32_t brev_bits(uint32_t v, int bits) {
    uint32_t r = 0;
    for (int b = 0; b < bits; ++b) r |= ((v >> b) & 1u) << (bits - 1 - b);
    return r;
}

uint32_t gdl_oracle_fps_priority(int64_t i, int tie_mode) {
    if (tie_mode == GDL_TIE_LOWEST_INDEX) return (uint32_t)i;
    uint32_t tid = (uint32_t)(i & 511), rj = (uint32_t)(i >> 9);
    uint32_t w = tid >> 5, l = tid & 31;
    return (brev_bits(w, 4) << 27) | (brev_bits(l, 5) << 22) | (rj & 0x3fffffu);
}

typedef struct {
    const float *pos; const int64_t *ptr, *k, *out_off; int tie_mode, dist_mode; int64_t *out;
} FpsCtx;

static void fps_cloud(int64_t b, void *vctx) {
    FpsCtx *c = (FpsCtx *)vctx;
    const int64_t start = c->ptr[b], n = c->ptr[b + 1] - c->ptr[b], kb = c->k[b];
    const int64_t out_start = c->out_off[b];
    if (n <= 0 || kb <= 0) return;
    const int64_t actual = kb < n ? kb : n;
    float *md = (float *)malloc(sizeof(float) * (size_t)n);
    uint32_t *prio = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) { md[i] = 1e30f; prio[i] = gdl_oracle_fps_priority(i, c->tie_mode); }
    int64_t sel = 0;
    c->out[out_start] = start;
    const float *P = c->pos + 3 * start;
    for (int64_t step = 1; step < actual; ++step) {
        const float sx = P[3 * sel], sy = P[3 * sel + 1], sz = P[3 * sel + 2];
        float bd = -1.0f; uint32_t bp = 0xffffffffu; int64_t bi = 0;
        for (int64_t i = 0; i < n; ++i) {
            float d = dist2(P[3 * i], P[3 * i + 1], P[3 * i + 2], sx, sy, sz, c->dist_mode);
            float m = fminf(d, md[i]);
            md[i] = m;
            if (m > bd || (m == bd && prio[i] < bp)) { bd = m; bp = prio[i]; bi = i; }
        }
        sel = bi;
        c->out[out_start + step] = start + sel;
    }
    free(md); free(prio);
}

int gdl_oracle_fps(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int B,
                   int tie_mode, int dist_mode, int64_t *out) {
    int64_t *off = (int64_t *)malloc(sizeof(int64_t) * (size_t)(B + 1));
    off[0] = 0;
    for (int b = 0; b < B; ++b) off[b + 1] = off[b] + (k_per_cloud[b] > 0 ? k_per_cloud[b] : 0);
    for (int64_t j = 0; j < off[B]; ++j) out[j] = -1;
    FpsCtx ctx = {pos, ptr, k_per_cloud, off, tie_mode, dist_mode, out};
    parallel_for(B, 1, fps_cloud, &ctx);
    free(off);
    return 0;
}

/* ---------------------------------------------------------------- KNN
 * knn_kernel.cu:113-172: per query, scan the sources of its cloud in ascending global
 * index, MinK<bucket(k)> heap, stable sort, write the first k (pad -1 / 1e30).
 * Queries outside every [ptr_q[b], ptr_q[b+1]) keep the padding.
 */
typedef struct {
    const float *query, *source; const int64_t *ptr_q, *ptr_s; int B, k, cap, dist_mode;
    const int32_t *qcloud; int64_t *out_idx; float *out_dist;
} KnnCtx;

static void knn_query(int64_t q, void *vctx) {
    KnnCtx *c = (KnnCtx *)vctx;
    const int b = c->qcloud[q];
    if (b < 0) return;
    const int64_t s0 = c->ptr_s[b], s1 = c->ptr_s[b + 1];
    MinK h;
    mink_init(&h, c->cap);
    const float qx = c->query[3 * q], qy = c->query[3 * q + 1], qz = c->query[3 * q + 2];
    for (int64_t s = s0; s < s1; ++s) {
        float d = dist2(qx, qy, qz, c->source[3 * s], c->source[3 * s + 1], c->source[3 * s + 2], c->dist_mode);
        mink_add(&h, d, (int)s);
    }
    mink_sort(&h);
    for (int j = 0; j < c->k && j < h.count; ++j) {
        c->out_idx[q * c->k + j] = h.i[j];
        c->out_dist[q * c->k + j] = h.d[j];
    }
}

int gdl_oracle_knn(const float *query, const float *source, const int64_t *ptr_q,
                   const int64_t *ptr_s, int B, int64_t n_q, int k, int dist_mode,
                   int64_t *out_idx, float *out_dist) {
    if (k <= 0 || n_q <= 0) return 0;
    for (int64_t j = 0; j < n_q * (int64_t)k; ++j) { out_idx[j] = -1; out_dist[j] = 1e30f; }
    int32_t *qc = (int32_t *)malloc(sizeof(int32_t) * (size_t)n_q);
    for (int64_t q = 0; q < n_q; ++q) qc[q] = -1;
    for (int b = 0; b < B; ++b)
        for (int64_t q = ptr_q[b]; q < ptr_q[b + 1] && q < n_q; ++q) qc[q] = b;
    KnnCtx ctx = {query, source, ptr_q, ptr_s, B, k, max_k_bucket_knn(k), dist_mode, qc, out_idx, out_dist};
    parallel_for(n_q, 16, knn_query, &ctx);
    free(qc);
    return 0;
}

/* ---------------------------------------------------------------- radius graph
 * radius_graph_kernel.cu:253-430 applied per cloud (the batched entry point loops over
 * clouds, :437-467). Grid: bbox over all points of the cloud (masked ones included,
 * :281-288) widened by 1e-5f, cell = r, resolution ceil(extent/r)+1 capped at 1024
 * (:290-297); points are binned with clamping (:117-124) and stably sorted by cell
 * (CUB radix sort on (cell, index), :325-347); a query scans the 27 cells around its
 * UNclamped cell in (dx, dy, dz) order (:200-235), keeps the bucket(max_nn) nearest with
 * d2 < r2 in a MinK heap. Output here is the kept set of every query, emitted as a CSR
 * over destinations (queries) with ascending sources; edge (row=src, col=dst).
 *
 * row_ptr: [N+1], src: capacity N*bucket. Returns the number of edges.
 */
static inline int f2i_rd(float v) { /* __float2int_rd: round down, saturate, NaN -> 0 */
    if (v != v) return 0;
    float f = floorf(v);
    if (f >= 2147483648.0f) return INT_MAX;
    if (f < -2147483648.0f) return INT_MIN;
    return (int)f;
}

typedef struct { int key; int idx; } KeyIdx;
static int cmp_keyidx(const void *a, const void *b) {
    const KeyIdx *x = (const KeyIdx *)a, *y = (const KeyIdx *)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx);
}
static int cmp_int(const void *a, const void *b) {
    int x = *(const int *)a, y = *(const int *)b;
    return x < y ? -1 : (x > y);
}

/* grid parameters exactly as the reference host computes them (float arithmetic) */
void gdl_oracle_radius_grid(const float *x, int64_t n, float inv_cell, float *mins, int *res) {
    float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
    for (int64_t i = 0; i < n; ++i)
        for (int a = 0; a < 3; ++a) {
            float v = x[3 * i + a];
            if (v < lo[a]) lo[a] = v;
            if (v > hi[a]) hi[a] = v;
        }
    for (int a = 0; a < 3; ++a) {
        float mn = lo[a] - 1e-5f, mx = hi[a] + 1e-5f;
        float ext = (mx - mn) * inv_cell;
        float c = ceilf(ext);
        int r = (c >= 1023.0f) ? 1024 : (int)c + 1; /* cap at 1024 (:295-297) */
        mins[a] = mn;
        res[a] = r;
    }
}

typedef struct {
    const float *P; const uint8_t *M; int64_t s0, n; const KeyIdx *ki;
    float mn[3]; int res[3]; float inv, r_sq; int loop, cap, dist_mode;
    int *kept; int64_t *cnt;
} RadCtx;

static void radius_query(int64_t q, void *vctx) {
    RadCtx *c = (RadCtx *)vctx;
    if (c->M && !c->M[q]) return;
    const float *P = c->P;
    const int rx = c->res[0], ry = c->res[1], rz = c->res[2];
    const float qx = P[3 * q], qy = P[3 * q + 1], qz = P[3 * q + 2];
    const int qcx = f2i_rd(mul_ftz(sub_ftz(qx, c->mn[0]), c->inv));
    const int qcy = f2i_rd(mul_ftz(sub_ftz(qy, c->mn[1]), c->inv));
    const int qcz = f2i_rd(mul_ftz(sub_ftz(qz, c->mn[2]), c->inv));
    MinK h;
    mink_init(&h, c->cap);
    for (int dx = -1; dx <= 1; ++dx) {
        int cx = qcx + dx;
        if (cx < 0 || cx >= rx) continue;
        for (int dy = -1; dy <= 1; ++dy) {
            int cy = qcy + dy;
            if (cy < 0 || cy >= ry) continue;
            for (int dz = -1; dz <= 1; ++dz) {
                int cz = qcz + dz;
                if (cz < 0 || cz >= rz) continue;
                int cell = (cx * ry + cy) * rz + cz;
                int64_t lo = 0, hi = c->n;
                while (lo < hi) { int64_t m = (lo + hi) / 2; if (c->ki[m].key < cell) lo = m + 1; else hi = m; }
                for (int64_t j = lo; j < c->n && c->ki[j].key == cell; ++j) {
                    int o = c->ki[j].idx;
                    if (!c->loop && o == (int)q) continue;
                    float d = dist2(qx, qy, qz, P[3 * o], P[3 * o + 1], P[3 * o + 2], c->dist_mode);
                    if (d < c->r_sq) mink_add(&h, d, o);
                }
            }
        }
    }
    int *dst = c->kept + (c->s0 + q) * c->cap;
    for (int j = 0; j < h.count; ++j) dst[j] = h.i[j] + (int)c->s0;
    qsort(dst, (size_t)h.count, sizeof(int), cmp_int);
    c->cnt[c->s0 + q] = h.count;
}

int64_t gdl_oracle_radius_graph(const float *x, const int64_t *ptr, int B, double radius,
                                int max_num_neighbors, int loop, const uint8_t *mask,
                                int dist_mode, int64_t *row_ptr, int64_t *src) {
    const float r = (float)radius;
    const int64_t N = ptr[B];
    const int cap = max_k_bucket_radius(max_num_neighbors);
    int64_t *cnt = (int64_t *)calloc((size_t)(N > 0 ? N : 1), sizeof(int64_t));
    int *kept = (int *)malloc(sizeof(int) * (size_t)(N > 0 ? N : 1) * cap);
    if (r > 0.0f) {
        for (int b = 0; b < B; ++b) {
            const int64_t s0 = ptr[b], n = ptr[b + 1] - ptr[b];
            if (n <= 1) continue;
            RadCtx c;
            c.P = x + 3 * s0; c.M = mask ? mask + s0 : NULL; c.s0 = s0; c.n = n;
            c.r_sq = r * r; c.inv = 1.0f / r; c.loop = loop; c.cap = cap; c.dist_mode = dist_mode;
            c.kept = kept; c.cnt = cnt;
            gdl_oracle_radius_grid(c.P, n, c.inv, c.mn, c.res);
            KeyIdx *ki = (KeyIdx *)malloc(sizeof(KeyIdx) * (size_t)n);
            for (int64_t i = 0; i < n; ++i) {
                ki[i].idx = (int)i;
                if (c.M && !c.M[i]) { ki[i].key = INT_MAX; continue; }
                const float *p = c.P + 3 * i;
                int cx = f2i_rd(mul_ftz(sub_ftz(p[0], c.mn[0]), c.inv));
                int cy = f2i_rd(mul_ftz(sub_ftz(p[1], c.mn[1]), c.inv));
                int cz = f2i_rd(mul_ftz(sub_ftz(p[2], c.mn[2]), c.inv));
                cx = cx < 0 ? 0 : (cx > c.res[0] - 1 ? c.res[0] - 1 : cx);
                cy = cy < 0 ? 0 : (cy > c.res[1] - 1 ? c.res[1] - 1 : cy);
                cz = cz < 0 ? 0 : (cz > c.res[2] - 1 ? c.res[2] - 1 : cz);
                ki[i].key = (cx * c.res[1] + cy) * c.res[2] + cz;
            }
            qsort(ki, (size_t)n, sizeof(KeyIdx), cmp_keyidx); /* == stable sort by key */
            c.ki = ki;
            parallel_for(n, 32, radius_query, &c);
            free(ki);
        }
    }
    int64_t e = 0;
    for (int64_t q = 0; q < N; ++q) {
        row_ptr[q] = e;
        for (int64_t j = 0; j < cnt[q]; ++j) src[e++] = kept[q * cap + j];
    }
    row_ptr[N] = e;
    free(cnt); free(kept);
    return e;
}

/* ---------------------------------------------------------------- CSR build
 * segment_reduce_kernel.cu:100-169: stable sort of destinations (CUB radix sort of
 * int32 keys carrying the original edge id), node_start/node_end set only for nodes
 * that occur (empty nodes keep 0/0, :30-50, :155-156). Returns 1 on an index outside
 * [0, N).
 */
int gdl_oracle_sort_and_build_csr(const int64_t *col, int64_t E, int64_t N, int32_t *col_sorted,
                                  int32_t *perm, int32_t *node_start, int32_t *node_end) {
    for (int64_t n = 0; n < N; ++n) { node_start[n] = 0; node_end[n] = 0; }
    if (E == 0) return 0;
    int64_t *cnt = (int64_t *)calloc((size_t)N + 1, sizeof(int64_t));
    for (int64_t e = 0; e < E; ++e) {
        if (col[e] < 0 || col[e] >= N) { free(cnt); return 1; }
        cnt[col[e] + 1]++;
    }
    for (int64_t n = 0; n < N; ++n) cnt[n + 1] += cnt[n];
    int64_t *fill = (int64_t *)malloc(sizeof(int64_t) * (size_t)(N > 0 ? N : 1));
    for (int64_t n = 0; n < N; ++n) fill[n] = cnt[n];
    for (int64_t e = 0; e < E; ++e) {
        int64_t p = fill[col[e]]++;
        col_sorted[p] = (int32_t)col[e];
        perm[p] = (int32_t)e;
    }
    for (int64_t n = 0; n < N; ++n)
        if (cnt[n + 1] > cnt[n]) { node_start[n] = (int32_t)cnt[n]; node_end[n] = (int32_t)cnt[n + 1]; }
    free(cnt); free(fill);
    return 0;
}

/* ---------------------------------------------------------------- segment reduce
 * sum : segment_reduce_kernel.cu:66-93, acc = 0.0f; acc += msg[perm[e]][c] in sorted
 *       order with FTZ adds.
 * mean: sum / deg (IEEE division); max: elementwise max, NaN propagates; empty -> 0.
 *       (semantics of torch.scatter_reduce(include_self=False) used by the reference's
 *       callers, nn/modules/invariant_attention.py:215-220, nn/modules/se3_net.py:262-268)
 * perm may be NULL (identity: rows already in segment order).
 */
static inline float load_msg(const void *msg, int dtype, int64_t idx) {
    return dtype == GDL_DTYPE_BF16 ? bf16_to_f32(((const uint16_t *)msg)[idx]) : ((const float *)msg)[idx];
}

typedef struct {
    const void *msg; int dtype; const int32_t *perm, *ns, *ne; int64_t C; int reduce; float *out;
} SegCtx;

static void seg_node(int64_t n, void *vctx) {
    SegCtx *c = (SegCtx *)vctx;
    const int64_t s = c->ns[n], e = c->ne[n], C = c->C;
    for (int64_t ch = 0; ch < C; ++ch) {
        float v;
        if (s >= e) {
            v = 0.0f;
        } else if (c->reduce == GDL_REDUCE_MAX) {
            v = -INFINITY;
            int nan = 0;
            for (int64_t j = s; j < e; ++j) {
                int64_t row = c->perm ? c->perm[j] : j;
                float m = load_msg(c->msg, c->dtype, row * C + ch);
                if (m != m) nan = 1;
                else if (m > v) v = m;
            }
            if (nan) v = NAN;
        } else {
            float acc = 0.0f;
            for (int64_t j = s; j < e; ++j) {
                int64_t row = c->perm ? c->perm[j] : j;
                acc = add_ftz(acc, load_msg(c->msg, c->dtype, row * C + ch));
            }
            v = (c->reduce == GDL_REDUCE_MEAN) ? acc / (float)(e - s) : acc;
        }
        c->out[n * C + ch] = v;
    }
}

int gdl_oracle_segment_reduce(const void *msg, int dtype, const int32_t *perm, const int32_t *node_start,
                              const int32_t *node_end, int64_t N, int64_t C, int reduce, float *out) {
    SegCtx ctx = {msg, dtype, perm, node_start, node_end, C, reduce, out};
    parallel_for(N, 64, seg_node, &ctx);
    return 0;
}

/* backward: grad_msg[perm[j]] for j in [s, e) of node n.
 * sum  : grad_out[n]              (functional/segment_reduce.py:142-158)
 * mean : grad_out[n] / deg
 * max  : grad_out[n] / t at each of the t entries equal to out[n], else 0 * that share
 *        (torch scatter_reduce 'amax' backward: grad split evenly among ties, the mask
 *        applied by a multiply so non-maxima carry the share's sign on a zero).
 * Rows of msg not covered by any segment are written as 0.
 */
int gdl_oracle_segment_reduce_backward(const float *grad_out, const void *msg, int dtype,
                                       const float *out, const int32_t *perm, const int32_t *node_start,
                                       const int32_t *node_end, int64_t N, int64_t C, int64_t E,
                                       int reduce, void *grad_msg) {
    float *g = (float *)calloc((size_t)(E * C > 0 ? E * C : 1), sizeof(float));
    for (int64_t n = 0; n < N; ++n) {
        const int64_t s = node_start[n], e = node_end[n];
        if (s >= e) continue;
        for (int64_t c = 0; c < C; ++c) {
            const float go = grad_out[n * C + c];
            if (reduce == GDL_REDUCE_MAX) {
                const float mx = out[n * C + c];
                int64_t t = 0;
                for (int64_t j = s; j < e; ++j) {
                    int64_t row = perm ? perm[j] : j;
                    if (load_msg(msg, dtype, row * C + c) == mx) ++t;
                }
                const float share = t > 0 ? go / (float)t : 0.0f;
                for (int64_t j = s; j < e; ++j) {
                    int64_t row = perm ? perm[j] : j;
                    /* mask * share as torch computes it: non-maxima get 0 * share (a signed zero) */
                    g[row * C + c] = ((load_msg(msg, dtype, row * C + c) == mx) ? 1.0f : 0.0f) * share;
                }
            } else {
                const float v = (reduce == GDL_REDUCE_MEAN) ? go / (float)(e - s) : go;
                for (int64_t j = s; j < e; ++j) {
                    int64_t row = perm ? perm[j] : j;
                    g[row * C + c] = v;
                }
            }
        }
    }
    if (dtype == GDL_DTYPE_BF16) {
        uint16_t *o = (uint16_t *)grad_msg;
        for (int64_t i = 0; i < E * C; ++i) o[i] = f32_to_bf16_rne(g[i]);
    } else {
        memcpy(grad_msg, g, sizeof(float) * (size_t)(E * C));
    }
    free(g);
    return 0;
}

/* ---------------------------------------------------------------- edge geometry
 * compute_edge_vectors (functional/radius_graph.py:338-358) and spherical_harmonics
 * (kernels/triton_sph_harm.py:200-240, normalize=False) as the reference's torch CPU path
 * rounds them: diff = x[col] - x[row]; |diff| = sqrtf(fmaf(dz, dz, fmaf(dy, dy, dx * dx)))
 * (torch's 2-norm accumulation over a row of three, pinned against torch 2.11 on the CPU);
 * dist = clamp(|diff|, min=1e-8) keeping NaN; dir = diff / dist; harmonics with one rounding
 * per torch op, constants (double) rounded to float first. Any output may be NULL. An edge
 * with an index outside [0, n) gets NaN everywhere.
 */
static void sph_row(float *o, int dim, float x, float y, float z) {
    const float c0 = (float)0.28209479177387814, c1 = (float)0.4886025119029199;
    const float c20 = (float)0.31539156525252005, c21 = (float)1.0925484305920792;
    const float c22 = (float)0.5462742152960396;
    o[0] = c0 * 1.0f;
    if (dim == 1) return;
    o[1] = c1 * y; o[2] = c1 * z; o[3] = c1 * x;
    if (dim == 4) return;
    o[4] = (c21 * x) * y;
    o[5] = (c21 * y) * z;
    o[6] = c20 * ((3.0f * z) * z - 1.0f);
    o[7] = (c21 * x) * z;
    o[8] = c22 * (x * x - y * y);
}

int gdl_oracle_edge_geometry(const float *x, int64_t n, const int64_t *row, const int64_t *col, int64_t E,
                             float *diff, float *dist, float *dir, float *sph, int max_l) {
    const int dim = (max_l + 1) * (max_l + 1);
    for (int64_t e = 0; e < E; ++e) {
        const int64_t s = row[e], q = col[e];
        float dx, dy, dz;
        if (s >= 0 && s < n && q >= 0 && q < n) {
            dx = x[3 * q] - x[3 * s]; dy = x[3 * q + 1] - x[3 * s + 1]; dz = x[3 * q + 2] - x[3 * s + 2];
        } else {
            dx = dy = dz = NAN;
        }
        const float nrm = sqrtf(fmaf(dz, dz, fmaf(dy, dy, dx * dx)));
        const float d = nrm < 1e-8f ? 1e-8f : nrm;
        if (diff) { diff[3 * e] = dx; diff[3 * e + 1] = dy; diff[3 * e + 2] = dz; }
        if (dist) dist[e] = d;
        const float ux = dx / d, uy = dy / d, uz = dz / d;
        if (dir) { dir[3 * e] = ux; dir[3 * e + 1] = uy; dir[3 * e + 2] = uz; }
        if (sph) sph_row(sph + e * dim, dim, ux, uy, uz);
    }
    return 0;
}

/* Per-node average degree of its cloud, clamped below at 1 (nn/modules/spatial_graph.py:
 * 131-153): cloud_sum / max(cloud_cnt, 1) over degree = node_end - node_start, clouds from
 * batch (if given), else ptr (if given), else one cloud; sums in exact integers, converted to
 * float once (equal to the reference's float scatter_add while sums stay below 2^24). Nodes
 * outside every cloud get 1. */
int gdl_oracle_cloud_avg_degree(const int32_t *ns, const int32_t *ne, int64_t n, const int64_t *batch,
                                const int64_t *ptr, int B, float *out) {
    if (!batch && !ptr) B = 1;
    int64_t *sum = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    int64_t *cnt = (int64_t *)calloc((size_t)(B > 0 ? B : 1), sizeof(int64_t));
    int *cl = (int *)malloc(sizeof(int) * (size_t)(n > 0 ? n : 1));
    for (int64_t i = 0; i < n; ++i) {
        int b = 0;
        if (batch) b = (batch[i] >= 0 && batch[i] < B) ? (int)batch[i] : -1;
        else if (ptr) {
            b = -1;
            for (int c = 0; c < B; ++c)
                if (ptr[c] <= i && i < ptr[c + 1]) { b = c; break; }
        }
        cl[i] = b;
        if (b >= 0) { sum[b] += (int64_t)ne[i] - ns[i]; cnt[b] += 1; }
    }
    for (int64_t i = 0; i < n; ++i) {
        const int b = cl[i];
        float a = 1.0f;
        if (b >= 0) {
            a = (float)sum[b] / (float)(cnt[b] > 1 ? cnt[b] : 1);
            if (a < 1.0f) a = 1.0f;
        }
        out[i] = a;
    }
    free(sum); free(cnt); free(cl);
    return 0;
}

/* ---------------------------------------------------------------- KNN aggregation
 * EquivariantInterpolate (nn/modules/equivariant_interp.py:91-125) and the weighted sums of
 * EquivariantPool (nn/modules/equivariant_pool.py:395-420):
 *   idw:  inv_j = 1 / sqrtf(max(dist, 1e-4)) (0 where idx < 0), s = sum_j inv_j in j order,
 *         w_j = inv_j / max(s, 1e-8)
 *   sum:  out[q] = sum_j w[q,j] * src[idx[q,j]] in j order from 0, product rounded first;
 *         neighbours outside [0, n_src) are skipped
 *   bwd:  grad_src[s] = sum over (q, j) ascending with idx = s of w[q,j] * grad_out[q]
 *   wgrad: per (q, j), 32 lane-strided partial sums over c then a xor butterfly (16, 8, 4, 2, 1)
 *         -- the fixed order the GPU kernel uses (the reference's order is torch's).
 */
int gdl_oracle_knn_idw_weights(const int64_t *idx, const float *dist, int64_t n_q, int K, float *w) {
    for (int64_t q = 0; q < n_q; ++q) {
        float s = 0.0f;
        for (int k = 0; k < K; ++k) {
            float v = 0.0f;
            if (idx[q * K + k] >= 0) {
                float d = dist[q * K + k];
                d = d < 1e-4f ? 1e-4f : d;
                v = 1.0f / sqrtf(d);
            }
            s = s + v;
            w[q * K + k] = v;
        }
        s = s < 1e-8f ? 1e-8f : s;
        for (int k = 0; k < K; ++k) w[q * K + k] = w[q * K + k] / s;
    }
    return 0;
}

int gdl_oracle_knn_weighted_sum(const float *src, int64_t n_src, int64_t dim, const int64_t *idx, const float *w,
                                int64_t n_q, int K, float *out) {
    for (int64_t q = 0; q < n_q; ++q)
        for (int64_t c = 0; c < dim; ++c) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) {
                const int64_t s = idx[q * K + k];
                if (s >= 0 && s < n_src) acc = acc + w[q * K + k] * src[s * dim + c];
            }
            out[q * dim + c] = acc;
        }
    return 0;
}

int gdl_oracle_knn_weighted_sum_backward(const float *gout, int64_t dim, const int64_t *idx, const float *w,
                                         int64_t n_q, int K, int64_t n_src, float *gsrc) {
    for (int64_t i = 0; i < n_src * dim; ++i) gsrc[i] = 0.0f;
    for (int64_t q = 0; q < n_q; ++q)
        for (int k = 0; k < K; ++k) {
            const int64_t s = idx[q * K + k];
            if (s < 0 || s >= n_src) continue;
            for (int64_t c = 0; c < dim; ++c) gsrc[s * dim + c] = gsrc[s * dim + c] + w[q * K + k] * gout[q * dim + c];
        }
    return 0;
}

int gdl_oracle_knn_weighted_sum_weight_grad(const float *gout, const float *src, int64_t n_src, int64_t dim,
                                            const int64_t *idx, int64_t n_q, int K, int accumulate, float *gw) {
    for (int64_t p = 0; p < n_q * K; ++p) {
        float lanes[32];
        const int64_t s = idx[p];
        for (int l = 0; l < 32; ++l) {
            float a = 0.0f;
            if (s >= 0 && s < n_src)
                for (int64_t c = l; c < dim; c += 32) a = a + gout[(p / K) * dim + c] * src[s * dim + c];
            lanes[l] = a;
        }
        for (int off = 16; off > 0; off >>= 1) {
            float nxt[32];
            for (int l = 0; l < 32; ++l) nxt[l] = lanes[l] + lanes[l ^ off];
            for (int l = 0; l < 32; ++l) lanes[l] = nxt[l];
        }
        gw[p] = accumulate ? gw[p] + lanes[0] : lanes[0];
    }
    return 0;
}

/* ---------------------------------------------------------------- hybrid graph
 * _EncoderStage._build_hybrid_graph (nn/modules/multi_scale_se3_net.py:126-219): the radius
 * edges (src -> q) plus, for every q with fewer than kf radius in-edges, (q -> m) and (m -> q)
 * for each valid m of knn[q, 1..kf]; deduplicated and ordered by row * n + col, as the
 * reference's `unique()` of the edge hashes returns them. Returns E; out_row / out_col need
 * room for the radius edges + 2 n kf.
 */
static int cmp_i64(const void *a, const void *b) {
    const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

int64_t gdl_oracle_hybrid_graph(const int64_t *row_ptr, const int64_t *src, const int64_t *knn, int64_t n, int kf,
                                int64_t *out_row, int64_t *out_col) {
    const int64_t er = row_ptr[n] - row_ptr[0];
    int64_t *h = (int64_t *)malloc(sizeof(int64_t) * (size_t)(er + 2 * n * kf + 1));
    int64_t m = 0;
    for (int64_t q = 0; q < n; ++q)
        for (int64_t j = row_ptr[q]; j < row_ptr[q + 1]; ++j) h[m++] = src[j] * n + q;
    for (int64_t q = 0; q < n; ++q) {
        if (row_ptr[q + 1] - row_ptr[q] >= kf) continue;
        for (int j = 1; j <= kf; ++j) {
            const int64_t v = knn[q * (kf + 1) + j];
            if (v < 0 || v >= n) continue;
            h[m++] = q * n + v;
            h[m++] = v * n + q;
        }
    }
    qsort(h, (size_t)m, sizeof(int64_t), cmp_i64);
    int64_t E = 0;
    for (int64_t i = 0; i < m; ++i) {
        if (i > 0 && h[i] == h[i - 1]) continue;
        out_row[E] = h[i] / n;
        out_col[E] = h[i] % n;
        ++E;
    }
    free(h);
    return E;
}
