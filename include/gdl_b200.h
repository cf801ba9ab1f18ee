/*
 * gdl_b200.h -- C ABI of the B200 (sm_100a) point-cloud graph operators.
 *
 * Drop-in native layer for GeoEmbodied's hot path (illusionaryshelter/GDL,
 * geoembodied/csrc): farthest-point sampling, KNN, radius graph, CSR build and
 * segment reduce (sum / mean / max, forward and backward).
 *
 * Conventions
 *  - Every pointer argument is DEVICE memory unless the comment says otherwise. Inputs
 *    are borrowed; outputs are written in place; nothing is freed.
 *  - `stream` is a cudaStream_t passed as void*; every kernel runs on it and no entry
 *    point synchronises the host, except where a comment says so.
 *  - Scratch memory is caller-provided (`workspace`, `workspace_bytes`); each operator
 *    that needs it has a *_workspace_size() query evaluated on the host. A workspace
 *    must be 256-byte aligned and may be reused once the stream has moved past the call.
 *  - Return value: a gdl_status for argument and launch errors. Launches are asynchronous,
 *    so execution faults surface at the caller's next synchronisation like any CUDA error.
 *    The only device-side waits (FPS's exchange between warps and CTAs) are bounded.
 *  - Clouds are packed CSR-style: cloud b owns points [ptr[b], ptr[b+1]); ptr is int64.
 */
#ifndef GDL_B200_H
#define GDL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    GDL_OK = 0,
    GDL_ERR_INVALID = 1,     /* bad argument: null pointer, negative size, bad enum       */
    GDL_ERR_WORKSPACE = 2,   /* workspace smaller than *_workspace_size()                  */
    GDL_ERR_CUDA = 3,        /* CUDA runtime / launch error                                */
    GDL_ERR_UNSUPPORTED = 4, /* device is not sm_100 (B200) or configuration not supported */
    GDL_ERR_OVERFLOW = 5,    /* a size exceeds the 32-bit index range of a kernel          */
    GDL_ERR_TIMEOUT = 6      /* a bounded device-side wait gave up                         */
} gdl_status;

enum { GDL_TIE_REFERENCE = 0, GDL_TIE_LOWEST_INDEX = 1 };
enum { GDL_REDUCE_SUM = 0, GDL_REDUCE_MEAN = 1, GDL_REDUCE_MAX = 2 };
enum { GDL_DTYPE_F32 = 0, GDL_DTYPE_BF16 = 1 };

/* Library version (major*10000 + minor*100 + patch). */
int gdl_version(void);

/* Human-readable name of a gdl_status. */
const char *gdl_status_string(int status);

/* GDL_OK if `device` is an sm_100 GPU this library was built for. */
int gdl_check_device(int device);

/* FP32 FMA throughput probe (no counterpart in the reference): `blocks` CTAs of 256 threads each
 * run `iters` rounds of 8 independent FMAs (scalar fma.rn.f32, or packed fma.rn.f32x2 when
 * `packed`), so that a benchmark can state FP32 fractions (KNN's distance scan) against a number
 * measured on this device. out [blocks * 256] f32 is written only to keep the work live.
 * gdl_fp32_peak_flops: the floating-point operations one such launch performs (2 per FMA lane). */
int64_t gdl_fp32_peak_flops(int64_t iters, int32_t packed, int32_t blocks);
int gdl_fp32_peak(float *out, int64_t iters, int32_t packed, int32_t blocks, void *stream);

/* ------------------------------------------------------------------------------ FPS
 * Replaces fps_cuda(pos, ptr, k_per_batch) -- geoembodied/csrc/fps_kernel.cu:160-209,
 * Python dispatch geoembodied/csrc/__init__.py:566-597.
 *
 * pos          [n_points, 3] f32
 * ptr          [num_clouds + 1] i64
 * k_per_cloud  [num_clouds] i64, samples requested per cloud
 * out_idx      [sum(max(k_b, 0))] i64: cloud b's picks start at sum_{c<b} max(k_c, 0);
 *              min(k_b, n_b) global indices in selection order, then -1 padding.
 * n_points     rows of pos.
 * max_cloud_points  host-side upper bound of max_b n_b. It selects the kernel variant: one CTA
 *              per cloud with the points in registers up to 4096 points; above that the clouds
 *              are put in Morton order (in the workspace) and run bucketed, one CTA of up to 8192
 *              points or a thread-block cluster of up to 8 CTAs of 1024 points or of up to 16 CTAs of
 *              8192, 13312 or 13824 points (up to 221184; the shape that needs the fewest waves of
 *              resident clusters for num_clouds, the smallest buckets on a tie), in
 *              exact rounds of up to 16 picks; beyond that, or if the device refuses the cluster,
 *              a streaming CTA that keeps the running minima in the workspace.
 * tie_break    GDL_TIE_REFERENCE: the reference kernel's argmax reduction order
 *              (bit-identical to fps_kernel<512>); GDL_TIE_LOWEST_INDEX: torch.argmax.
 * out_pos      [same slots, 3] f32 (nullable): coordinates of each pick (0 for padding), which
 *              saves the caller a gather of pos[out_idx].
 * Seed is the first point of each cloud; distances use the reference's rounding.
 * The bucketed kernel's CTAs (a cluster's, or one CTA's warps) exchange each round's records
 * through shared-memory barriers with a bounded wait; a wait that gives up (never observed)
 * writes -2 into the cloud's remaining picks (coordinates 0) -- gdl_fps_ex also reports it.
 */
size_t gdl_fps_workspace_size(int64_t n_points, int32_t num_clouds, int64_t max_cloud_points);
int gdl_fps(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int32_t num_clouds, int64_t n_points,
            int64_t max_cloud_points, int32_t tie_break, int64_t *out_idx, float *out_pos, void *workspace,
            size_t workspace_bytes, void *stream);

/* gdl_fps with the bounded waits exposed (same reference interface as gdl_fps).
 * status      [1] i32 device (nullable): set to GDL_ERR_TIMEOUT when a wait of the bucketed
 *             kernel gave up (the caller zeroes it; read it after the stream has run the call).
 * wait_polls  mbarrier polls before a wait gives up (<= 0: 2^20).
 * hold_rank, hold_pick  failure injection for tests (-1: off): in every cluster the CTA of this
 *             rank sends no records at this pick, so every wait of that pick runs out and
 *             the call takes its failure path (status, -2 picks) without faulting anything.
 */
int gdl_fps_ex(const float *pos, const int64_t *ptr, const int64_t *k_per_cloud, int32_t num_clouds,
               int64_t n_points, int64_t max_cloud_points, int32_t tie_break, int64_t *out_idx, float *out_pos,
               void *workspace, size_t workspace_bytes, int32_t *status, int32_t wait_polls, int32_t hold_rank,
               int64_t hold_pick, void *stream);

/* Exchange rounds the last bucketed gdl_fps / gdl_fps_ex call on this workspace took for its
 * longest cloud, read back synchronously into *out (host); 0 for clouds of <= 4096 points, whose
 * kernel makes one pick per exchange. For rooflines: the picks per round, and the round count a
 * pure exchange chain would need. No counterpart in the reference. */
int gdl_fps_round_count(const void *workspace, int64_t n_points, int32_t num_clouds, int64_t max_cloud_points,
                        unsigned long long *out);

/* ------------------------------------------------------------------------------ KNN
 * Replaces knn_cuda(query, source, ptr_q, ptr_s, k) and knn_self_cuda(points, ptr, k)
 * -- geoembodied/csrc/knn_kernel.cu:200-308, dispatch csrc/__init__.py:376-432.
 *
 * query [n_query, 3] f32, source [*, 3] f32, ptr_q / ptr_s [num_clouds + 1] i64.
 * out_idx [n_query, k] i64 global source indices, -1 padded; out_dist [n_query, k] f32
 * squared distances, 1e30 padded. At most min(k, 64) neighbours per query (the reference's
 * MinK<64> bucket), ascending distance; equal distances are ordered exactly as the
 * reference's heap orders them. Queries outside every [ptr_q[b], ptr_q[b+1]) keep padding.
 * max_cloud_sources: host-side bound of the sources per cloud, max_b (ptr_s[b+1] - ptr_s[b]),
 * or any value with num_clouds * max_cloud_sources >= ptr_s[num_clouds] - ptr_s[0] (e.g. the mean
 * rounded up). Calls with max_cloud_sources >= 32768 search a grid of each cloud's sources (exact;
 * knn_grid.cu); if the bound is violated there, every query falls back to the exact heap replay.
 * Calls with 4097 <= max_cloud_sources < 32768 and at least 592 queries put each cloud's sources
 * in Morton order, in blocks of 32 with a box each, and visit them nearest-first per tile of 128
 * Morton-ordered queries, skipping blocks by an exact distance bound (the workspace holds the
 * orders and boxes).
 */
size_t gdl_knn_workspace_size(int64_t n_query, int32_t num_clouds, int32_t k, int64_t max_cloud_sources);
/* Distances (query, source pairs) the last gdl_knn call with this workspace and these sizes
 * evaluated, read back synchronously into *out (host): the work a roofline counts once clouds of
 * 4097 .. 32767 sources skip blocks of sources (brute force evaluates every pair). The grid path
 * (clouds of >= 32768 sources) does not count its searches. No counterpart in the reference. */
int gdl_knn_distance_count(const void *workspace, int64_t n_query, int32_t num_clouds, int32_t k,
                           int64_t max_cloud_sources, unsigned long long *out);
int gdl_knn(const float *query, const float *source, const int64_t *ptr_q, const int64_t *ptr_s,
            int32_t num_clouds, int64_t n_query, int32_t k, int64_t max_cloud_sources, int64_t *out_idx,
            float *out_dist, void *workspace, size_t workspace_bytes, void *stream);

/* ----------------------------------------------------------------------- radius graph
 * Replaces radius_graph_cuda(points, radius, max_num_neighbors, mask, loop) and
 * radius_graph_cuda_batched(...) -- geoembodied/csrc/radius_graph_kernel.cu:253-467,
 * dispatch csrc/__init__.py:130-186 -- for any number of variable-size clouds at once.
 *
 * x [n_points, 3] f32, ptr [num_clouds + 1] i64, mask [n_points] u8 (nullable, 0 = padding).
 * Per query: the bucket(max_num_neighbors) in {16, 32, 64} nearest points of its own
 * cloud with squared distance < r^2 (r = (float)radius), found on the reference's
 * per-cloud cell grid with its scan order and heap, so the edge SET equals the
 * reference's. Edges are emitted as a CSR over destinations:
 *   out_row_ptr [n_points + 1] i64  (edges of destination q: [row_ptr[q], row_ptr[q+1]))
 *   out_src     [capacity] i64      (row: the neighbour, ascending within a destination)
 *   out_dst     [capacity] i64      (col: the query; nullable)
 *   out_row_ptr32 [n_points + 1], out_src32 [capacity] i32 (nullable): the same CSR in the
 *               int32 layout the segment reduce consumes (node_start = row_ptr32[:-1],
 *               node_end = row_ptr32[1:], perm = src32 to gather source rows).
 * capacity = n_points * bucket(max_num_neighbors). The edge count is out_row_ptr[n_points].
 * max_cloud_points: host-side upper bound of the largest cloud, or 0 if unknown; clouds of at
 * most 4096 points take a fused path (one CTA per cloud, 2 launches in total).
 */
size_t gdl_radius_graph_workspace_size(int64_t n_points, int32_t num_clouds, int32_t max_num_neighbors);
int gdl_radius_graph(const float *x, const int64_t *ptr, int32_t num_clouds, int64_t n_points,
                     int64_t max_cloud_points, double radius, int32_t max_num_neighbors, int32_t loop,
                     const uint8_t *mask, int64_t *out_row_ptr, int64_t *out_src, int64_t *out_dst,
                     int32_t *out_row_ptr32, int32_t *out_src32, void *workspace, size_t workspace_bytes,
                     void *stream);

/* ------------------------------------------------------------------------ edge geometry
 * Replaces compute_edge_vectors(x, row, col) -- geoembodied/functional/radius_graph.py:338-358 --
 * and spherical_harmonics(direction, max_l, normalize=False) -- kernels/triton_sph_harm.py:
 * 200-240, 322-369 -- as SpatialGraph.build / from_edge_index call them
 * (nn/modules/spatial_graph.py:126-129, 222-223). Per edge (src -> dst):
 *   diff      [E, 3] x[dst] - x[src]
 *   dist      [E]    |diff| clamped below at 1e-8
 *   direction [E, 3] diff / dist
 *   sph       [E, (sph_max_l + 1)^2] real spherical harmonics of direction, l <= sph_max_l,
 *             channels [Y00 | Y1-1 Y10 Y11 | Y2-2 Y2-1 Y20 Y21 Y22]
 * Every pointer is nullable (nothing written). Rounding: IEEE single precision as the
 * reference's torch CPU evaluation of the same formulas.
 */
typedef struct gdl_edge_geometry {
    float *diff;
    float *dist;
    float *direction;
    float *sph;
    int32_t sph_max_l; /* 0, 1 or 2 when sph is set */
} gdl_edge_geometry;

/* The radius graph of gdl_radius_graph with the geometry of each edge written by the kernel
 * that emits the edge (edge slot j of out_src gets slot j of every geometry array; capacity
 * as for out_src). Same workspace as gdl_radius_graph. No counterpart kernel in the reference,
 * whose radius graph and geometry are separate passes. */
int gdl_radius_graph_geometry(const float *x, const int64_t *ptr, int32_t num_clouds, int64_t n_points,
                              int64_t max_cloud_points, double radius, int32_t max_num_neighbors, int32_t loop,
                              const uint8_t *mask, int64_t *out_row_ptr, int64_t *out_src, int64_t *out_dst,
                              int32_t *out_row_ptr32, int32_t *out_src32, const gdl_edge_geometry *geometry,
                              void *workspace, size_t workspace_bytes, void *stream);

/* Geometry of COO edges (row = src, col = dst, int64, any order) over x [n_points, 3].
 * An edge with an index outside [0, n_points) gets NaN in every output. */
int gdl_edge_geometry_coo(const float *x, int64_t n_points, const int64_t *row, const int64_t *col,
                          int64_t n_edges, const gdl_edge_geometry *geometry, void *stream);

/* Per-node average degree of the node's cloud, clamped below at 1 -- the avg_degree of
 * SpatialGraph.build / from_edge_index (nn/modules/spatial_graph.py:131-153, 225-239):
 * degree[n] = node_end[n] - node_start[n]; the cloud of node n is batch[n] (batch given, any
 * order, values in [0, num_clouds)), else the b with ptr[b] <= n < ptr[b+1] (ptr given), else
 * one cloud of all nodes. out[n] = float(sum of the cloud's degrees) / float(max(nodes, 1)),
 * then max(., 1). Nodes outside every cloud get 1. Sums are exact (integer atomics). */
size_t gdl_cloud_avg_degree_workspace_size(int32_t num_clouds);
int gdl_cloud_avg_degree(const int32_t *node_start, const int32_t *node_end, int64_t n_nodes, const int64_t *batch,
                         const int64_t *ptr, int32_t num_clouds, float *out, void *workspace, size_t workspace_bytes,
                         void *stream);

/* SpatialGraph's CSR fields for a radius graph from gdl_radius_graph(_geometry), without a sort:
 * its edges already come grouped by ascending destination, so sort_and_build_csr(col, N)
 * (segment_reduce_kernel.cu:100-169) of them is the identity permutation. With
 * E = row_ptr[n_points] (read on the device, E <= capacity):
 *   col_sorted [capacity] i32: first E = dst;  perm [capacity] i32: first E = 0 .. E-1
 *   node_start / node_end [n_points] i32 (0 / 0 for nodes without edges, as the reference)
 *   avg_degree [n_points] f32: edges of the node's cloud / its nodes, clamped below at 1,
 *              clouds from ptr [num_clouds + 1] (nullable: one cloud of all n_points nodes)
 * Every output is nullable. No counterpart kernel in the reference. */
int gdl_radius_csr_finish(const int64_t *row_ptr, const int64_t *dst, int64_t n_points, int64_t capacity,
                          const int64_t *ptr, int32_t num_clouds, int32_t *col_sorted, int32_t *perm,
                          int32_t *node_start, int32_t *node_end, float *avg_degree, void *stream);

/* ------------------------------------------------------------------------ hybrid graph
 * Replaces _EncoderStage._build_hybrid_graph (geoembodied/nn/modules/multi_scale_se3_net.py:
 * 126-219) up to its SpatialGraph: radius edges, plus both directions of (q, m) for every node
 * q with fewer than knn_fallback_k radius in-edges and each valid m of knn_idx[q, 1 ..
 * knn_fallback_k] (knn_self with k = knn_fallback_k + 1, column 0 dropped), deduplicated and --
 * like the reference's hash unique() -- ordered by (row, col); then from_edge_index's geometry
 * and sort_and_build_csr(col) (segment_reduce_kernel.cu:100-169) without a second sort.
 *   x              [n_points, 3] f32 (read only for the geometry)
 *   radius_row_ptr / radius_src: gdl_radius_graph's destination CSR, built with the same
 *                  max_num_neighbors (it sizes the buffers here)
 *   knn_idx        [n_points, knn_fallback_k + 1] i64 (gdl_knn of the points against themselves)
 * Outputs (capacity = gdl_hybrid_graph_capacity(...) slots; the edge count E is written at
 * out_row_ptr[n_points], on the device):
 *   out_row / out_col [capacity] i64: the edges in (row, col) order (first E valid)
 *   out_row_ptr [n_points + 1] i64: destination CSR of the same edges
 *   col_sorted / perm [capacity] i32, node_start / node_end [n_points] i32: the segment-reduce CSR
 *   src_sorted [capacity] i32 (nullable): the source of each col-sorted slot, row[perm[j]]
 *   geometry (nullable): per edge in (row, col) order, as gdl_edge_geometry_coo
 * No counterpart kernel in the reference. */
int64_t gdl_hybrid_graph_capacity(int64_t n_points, int32_t max_num_neighbors, int32_t knn_fallback_k);
size_t gdl_hybrid_graph_workspace_size(int64_t n_points, int32_t max_num_neighbors, int32_t knn_fallback_k);
int gdl_hybrid_graph(const float *x, const int64_t *radius_row_ptr, const int64_t *radius_src, const int64_t *knn_idx,
                     int64_t n_points, int32_t max_num_neighbors, int32_t knn_fallback_k, int64_t *out_row_ptr,
                     int64_t *out_row, int64_t *out_col, int32_t *col_sorted, int32_t *perm, int32_t *src_sorted,
                     int32_t *node_start, int32_t *node_end, const gdl_edge_geometry *geometry, void *workspace,
                     size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------ SE3Conv message aggregation
 * Replaces SE3Conv's per-edge messages + segment_reduce + degree normalisation
 * (geoembodied/nn/modules/se3_conv.py:61-235 _compute_messages, :487-545 forward) for the
 * nine tensor-product paths, without materialising the [E, C] messages. The channel mixing of
 * each path is linear in the source features and is passed in per NODE (GEMMs run by the
 * caller); the kernel forms each edge's message from its source's projections and the edge's
 * radial weights R, direction d and harmonics while it reduces the edges of each target:
 *   p[0] [N,Cs]    = s W_ss^T       scalar  += (R0 Y0) p0[o]
 *   p[1] [N,Cv]    = s W_sv^T       vector  += (R1 p1[o]) d_k
 *   p[2] [N,Cv,3]  = W_vv v         vector  += (R2 Y0) p2[o,k]
 *   p[3] [N,Cs,3]  = W_vs v         scalar  += R3 (d . p3[o])
 *   p[4] [N,Cv,3]  = W_x v          vector  += R4 (d x p4[o])_k
 *   p[5] [N,Ct2]   = s W_st2^T      type-2  += (R5 p5[o]) Y2_m
 *   p[6] [N,Ct2,5] = W_t2t2 t2      type-2  += (R6 Y0) p6[o,m]
 *   p[7] [N,Ct2,3] = W_vt2 v        type-2  += R7 sum_ij d_i p7[o,j] cg[i,j,m]
 *   p[8] [N,Cs]    = |t2|^2 W_t2s^T scalar  += R8 p8[o]
 * out = (sum over the target's edges in CSR slot order) / avg_degree[target].
 * p[i] == NULL switches path i off; r_col[i] = its column of R [E, r_stride]. Y0 = sph[e, 0],
 * Y2 = sph[e, 4:9] (sph [E, sph_dim]); cg [3, 3, 5] Cartesian CG(1,1,2) (path 7 only).
 * Edges: row [E] (source of edge e), perm [E] (edge of CSR slot j), node_start/node_end [N].
 * Backward: grad_R [E, r_stride] (nullable) and grad_proj[i] (nullable array / entries, shapes and
 * row strides ld[i] of p[i]; every entry of each row is written) from grad_s/v/t2 [N, ...]; grad_proj needs the edges grouped by source: src_perm /
 * src_start / src_end = gdl_sort_and_build_csr(row) (perm, node_start, node_end), and col [E].
 * avg_degree may be NULL in the backward: grad_s/v/t2 then come already divided by their target's
 * average degree (one division per node and channel instead of one per edge term).
 * No counterpart kernel in the reference. */
typedef struct gdl_se3_paths {
    const float *p[9];
    int32_t r_col[9];
    int64_t ld[9]; /* floats from one node's row of p[i] to the next (0: the dense row width above),
                      so that projections of one input can be column slices of one GEMM result */
    int64_t cs, cv, ct2;
} gdl_se3_paths;

int gdl_se3_aggregate(const gdl_se3_paths *paths, const float *R, int64_t r_stride, const float *direction,
                      const float *sph, int32_t sph_dim, const float *cg, const int64_t *row, const int32_t *perm,
                      const int32_t *node_start, const int32_t *node_end, const float *avg_degree, int64_t n_nodes,
                      int64_t n_edges, float *out_s, float *out_v, float *out_t2, void *stream);
int gdl_se3_aggregate_backward(const gdl_se3_paths *paths, float *const *grad_proj, float *grad_R,
                               const float *grad_s, const float *grad_v, const float *grad_t2, const float *R,
                               int64_t r_stride, const float *direction, const float *sph, int32_t sph_dim,
                               const float *cg, const int64_t *row, const int64_t *col, const int32_t *src_perm,
                               const int32_t *src_start, const int32_t *src_end, const float *avg_degree,
                               int64_t n_nodes, int64_t n_edges, void *stream);

/* ------------------------------------------------------------ channel-mixing weight gradient
 * Replaces the weight gradients torch autograd takes through SE3Conv's nn.Linear layers: the node
 * projections W [M, N] (geoembodied/nn/modules/se3_conv.py:343-413, applied to [rows, N, sub]
 * features: sub = 1 scalars, 3 vectors, 5 type-2) and the radial MLP (se3_conv.py:266-268, sub = 1).
 * The rows (nodes or edges) run to the hundreds of thousands, M and N to a few hundred:
 *   C[m, n]    = sum_{r < rows} sum_{j < sub} A[r * lda + m * sub + j] * B[r * ldb + n * sub + j]
 *   col_sum[m] = sum_{r < rows} A[r * lda + m]   (nullable, sub == 1 only: the bias gradient)
 * A = the layer's output gradient, B = its input (lda >= M * sub, ldb >= N * sub, in floats); C [M, N]
 * dense row-major and col_sum [M] are overwritten (zeros when rows == 0; col_sum is still written
 * when N == 0). The rows are split into a fixed number of slices and the partial results added in
 * slice order: deterministic.
 */
size_t gdl_weight_grad_workspace_size(int64_t rows, int32_t M, int32_t N, int32_t sub);
int gdl_weight_grad(const float *A, int64_t lda, const float *B, int64_t ldb, int64_t rows, int32_t M, int32_t N,
                    int32_t sub, float *C, float *col_sum, void *workspace, size_t workspace_bytes, void *stream);

/* -------------------------------------------------------------------- KNN aggregation
 * Replaces the weighted neighbour sums of the reference's KNN consumers, which gather
 * [n_query, k, dim] rows with torch indexing and reduce them over k:
 *   EquivariantPool         s_out = (w[..., None] * scalars[idx]).sum(1), v_out likewise
 *                           (nn/modules/equivariant_pool.py:395-420)
 *   EquivariantInterpolate  inverse-distance weights + the same sums for s, v, t2
 *                           (nn/modules/equivariant_interp.py:91-125)
 * idx [n_query, k] i64 (KNN output; entries < 0 or >= n_src are skipped), rows f32.
 *
 * gdl_knn_idw_weights: out_weight[q, j] = inv_j / max(sum_j inv_j, 1e-8) with
 *   inv_j = 1 / sqrt(max(dist[q, j], 1e-4)), 0 where idx[q, j] < 0 (dist = squared distances).
 * gdl_knn_weighted_sum: out[q, :] = sum_j weight[q, j] * src[idx[q, j], :], src [n_src, dim],
 *   out [n_query, dim]; an fp32 fold in j order from 0, products rounded first.
 * gdl_knn_weighted_sum_backward: grad_src[t][s, :] = sum over the (q, j) with idx[q, j] = s, in
 *   (q, j) order, of weight[q, j] * grad_out[t][q, :], for n_tables tables sharing idx/weight
 *   (host arrays of device pointers and dims). Deterministic (sorted pairs, no atomics).
 * gdl_knn_weighted_sum_weight_grad: grad_weight[q, j] (+= if accumulate) sum_c grad_out[q, c] *
 *   src[idx[q, j], c]; 0 for skipped pairs.
 * No counterpart kernels in the reference (torch indexing, mul and sum there).
 */
int gdl_knn_idw_weights(const int64_t *idx, const float *dist, int64_t n_query, int32_t k, float *out_weight,
                        void *stream);
int gdl_knn_weighted_sum(const float *src, int64_t n_src, int64_t dim, const int64_t *idx, const float *weight,
                         int64_t n_query, int32_t k, float *out, void *stream);
size_t gdl_knn_weighted_sum_backward_workspace_size(int64_t n_query, int32_t k, int64_t n_src);
int gdl_knn_weighted_sum_backward(const float *const *grad_out, float *const *grad_src, const int64_t *dims,
                                  int32_t n_tables, const int64_t *idx, const float *weight, int64_t n_query,
                                  int32_t k, int64_t n_src, void *workspace, size_t workspace_bytes, void *stream);
int gdl_knn_weighted_sum_weight_grad(const float *grad_out, const float *src, int64_t n_src, int64_t dim,
                                     const int64_t *idx, int64_t n_query, int32_t k, int32_t accumulate,
                                     float *grad_weight, void *stream);

/* -------------------------------------------------------------------------- CSR build
 * Replaces sort_and_build_csr(col, N) -- geoembodied/csrc/segment_reduce_kernel.cu:100-169.
 * col [num_edges] i64 in [0, num_nodes). Stable sort by destination:
 * col_sorted / perm [num_edges] i32 (perm = original edge id of each sorted slot),
 * node_start / node_end [num_nodes] i32; nodes without edges get 0 / 0.
 */
size_t gdl_sort_and_build_csr_workspace_size(int64_t num_edges, int64_t num_nodes);
int gdl_sort_and_build_csr(const int64_t *col, int64_t num_edges, int64_t num_nodes, int32_t *col_sorted,
                           int32_t *perm, int32_t *node_start, int32_t *node_end, void *workspace,
                           size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------- segment reduce
 * Replaces segment_reduce_sum(msg, perm, node_start, node_end, N) --
 * geoembodied/csrc/segment_reduce_kernel.cu:176-210 -- and adds mean and max
 * (torch.scatter_reduce(include_self=False) semantics, used by the reference's callers
 * at nn/modules/invariant_attention.py:215-220 and nn/modules/se3_net.py:226-270).
 *
 * msg [num_rows, C] f32 or bf16 (dtype); perm [*] i32 row of each sorted slot (nullable:
 * slot j is row j); node_start / node_end [num_nodes] i32. out [num_nodes, C] f32:
 *   sum  : ((0 + m_0) + m_1) + ... in slot order (bit-identical to the reference kernel)
 *          for segments of up to 4096 slots; longer ones use a fixed-order tree.
 *   mean : sum / degree;  max : elementwise maximum (NaN propagates); empty -> 0.
 * arg_out [num_nodes, C] i32 (max only, nullable): slot of the unique maximum, -1 when
 * tied (or empty); consumed by the backward.
 */
size_t gdl_segment_reduce_workspace_size(int64_t num_rows, int64_t num_nodes);
int gdl_segment_reduce(const void *msg, int32_t dtype, int64_t num_rows, int64_t C, const int32_t *perm,
                       const int32_t *node_start, const int32_t *node_end, int64_t num_nodes, int32_t reduce,
                       float *out, int32_t *arg_out, void *workspace, size_t workspace_bytes, void *stream);

/* Backward of gdl_segment_reduce (the reference's autograd: gather grad_out by destination,
 * un-permute -- geoembodied/functional/segment_reduce.py:142-158, 259-270): for every slot j
 * of node n,
 *   grad_msg[perm[j]] = grad_out[n]                              (sum)
 *                     = grad_out[n] / degree(n)                  (mean)
 *                     = (msg == out[n]) * grad_out[n] / ties     (max; ties = #maxima)
 * `arg`/`out` come from the max forward (msg is re-read only for tied maxima). Rows that no
 * slot references are left untouched. grad_msg has msg's dtype (bf16 rounded to nearest even).
 * Uses the same workspace size as gdl_segment_reduce.
 */
int gdl_segment_reduce_backward(const float *grad_out, const void *msg, int32_t dtype, const float *out,
                                const int32_t *arg, int64_t num_rows, int64_t C, const int32_t *perm,
                                const int32_t *node_start, const int32_t *node_end, int64_t num_nodes, int32_t reduce,
                                void *grad_msg, void *workspace, size_t workspace_bytes, void *stream);

/* Segment reduce that allocates nothing (no counterpart in the reference).
 * For callers that may not allocate device memory while they run -- a CUDA graph being
 * captured under a fixed memory plan, plugin or real-time hosts whose enqueue path forbids
 * cudaMalloc / cudaFree, programs without an allocator for the device. Same arguments and
 * results as gdl_segment_reduce, minus the workspace: its scratch (the queue of segments longer
 * than 4096 slots) lives in a 64 KiB array built into the library, which every GPU that loads
 * the library keeps until the process exits.
 *  - num_rows must not exceed 66,863,040 (16,320 queued segments x 4,097 slots); larger inputs
 *    return GDL_ERR_OVERFLOW.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 *    that device current; make that first call before any stream capture. The address is kept
 *    for the life of the process: after a cudaDeviceReset() on that device (which destroys the
 *    context owning the array) this entry point must not be called again in that process.
 *  - All calls on a device share the array. Each call clears the part that must start at zero,
 *    but calls whose kernels may overlap on the GPU (unordered streams) race and must not be
 *    issued; order them on one stream or with events.
 */
int gdl_segment_reduce_noalloc(const void *msg, int32_t dtype, int64_t num_rows, int64_t C, const int32_t *perm,
                               const int32_t *node_start, const int32_t *node_end, int64_t num_nodes, int32_t reduce,
                               float *out, int32_t *arg_out, void *stream);

/* ------------------------------------------------------------------------ row gather
 * out[i, :] = src[idx[i], :] -- the msg = feats[knn_idx] materialisation of the reference's
 * pooling layer (geoembodied/nn/modules/equivariant_pool.py:277-300, torch indexing there;
 * no counterpart in geoembodied/csrc).
 *
 * src        [n_src, row_bytes] any element type; row_bytes a multiple of 4
 * idx        [n_idx] i64; an index outside [0, n_src) yields a zero row
 * out        [n_idx, row_bytes]
 */
int gdl_gather_rows(const void *src, int64_t n_src, int64_t row_bytes, const int64_t *idx, int64_t n_idx, void *out,
                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDL_B200_H */
