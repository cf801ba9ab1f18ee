// segment.cu -- CSR build and deterministic segment reduce (sum / mean / max, fwd + bwd).
//
// Reference: geoembodied/csrc/segment_reduce_kernel.cu (sort_and_build_csr :100-169,
// segment_reduce_sum_kernel :66-93) and the autograd in
// geoembodied/functional/segment_reduce.py:112-158, 211-279.
//
// Layout in HBM: msg [rows, C] row-major (f32 or bf16), out [N, C] f32, CSR as int32
// node_start / node_end over "slots" (sorted positions), perm[slot] = msg row.
//
// Forward, short segments (<= kLongSegment slots): a group of G lanes owns one segment; each
// lane owns VEC consecutive channels and folds the segment's rows in slot order, so a sum is
// ((0 + m0) + m1) + ... exactly like the reference kernel (one thread per channel). Rows are
// fetched with 8/16-byte vector loads, U slots in flight. Long segments are queued and
// handled one CTA each: row groups fold contiguous slot ranges, partials combined in a fixed
// order (deterministic, not the reference's rounding).
// Backward: the same segment-to-group mapping; each group writes its segment's gradient rows
// grad_msg[perm[j]] (what the reference's gather + un-permute computes, segment_reduce.py:
// 142-158), VEC channels per lane. Max uses the forward's arg and re-reads msg only for
// tied maxima, whose gradient is shared evenly (torch's amax rule).
#include <initializer_list>
#include <type_traits>
#include <mutex>

#include "common.cuh"
#include "radix.cuh"

namespace gdl {

constexpr int kLongSegment = 4096;
constexpr int kSegThreads = 256;
constexpr int kUnroll = 4;       // rows in flight per lane, long segments
// rows in flight per lane, short segments: 64 bytes at 16-byte vectors, 8 rows below that
template <int VEC>
struct ShortUnroll {
    static constexpr int value = VEC >= 8 ? 4 : 8;
};

// ----------------------------------------------------------------- vector loads as f32
// VecIO<T, VEC>: VEC consecutive elements of type T. `load_raw` issues one vector load
// (kept raw so that many rows can be in flight in few registers), `cvt` widens it to f32;
// `store` narrows f32 values back to T; `store_raw` writes VEC elements already in T.
template <typename T, int VEC>
struct VecIO;

template <>
struct VecIO<float, 8> {
    struct Raw { float4 a, b; };
    static __device__ __forceinline__ Raw load_raw(const float *p) {
        return {__ldg(reinterpret_cast<const float4 *>(p)), __ldg(reinterpret_cast<const float4 *>(p) + 1)};
    }
    static __device__ __forceinline__ void cvt(const Raw &r, float *v) {
        v[0] = r.a.x; v[1] = r.a.y; v[2] = r.a.z; v[3] = r.a.w;
        v[4] = r.b.x; v[5] = r.b.y; v[6] = r.b.z; v[7] = r.b.w;
    }
    static __device__ __forceinline__ void store(float *p, const float *v) {
        reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    static __device__ __forceinline__ void store_raw(float *p, const float *v) { store(p, v); }
};
template <>
struct VecIO<float, 4> {
    using Raw = float4;
    static __device__ __forceinline__ Raw load_raw(const float *p) { return __ldg(reinterpret_cast<const float4 *>(p)); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) { v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w; }
    static __device__ __forceinline__ void store(float *p, const float *v) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
    static __device__ __forceinline__ void store_raw(float *p, const float *v) { store(p, v); }
};
template <>
struct VecIO<float, 2> {
    using Raw = float2;
    static __device__ __forceinline__ Raw load_raw(const float *p) { return __ldg(reinterpret_cast<const float2 *>(p)); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) { v[0] = t.x; v[1] = t.y; }
    static __device__ __forceinline__ void store(float *p, const float *v) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    }
    static __device__ __forceinline__ void store_raw(float *p, const float *v) { store(p, v); }
};
template <>
struct VecIO<float, 1> {
    using Raw = float;
    static __device__ __forceinline__ Raw load_raw(const float *p) { return __ldg(p); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) { v[0] = t; }
    static __device__ __forceinline__ void store(float *p, const float *v) { *p = v[0]; }
    static __device__ __forceinline__ void store_raw(float *p, const float *v) { *p = v[0]; }
};
template <>
struct VecIO<uint16_t, 8> {
    using Raw = uint4;
    static __device__ __forceinline__ Raw load_raw(const uint16_t *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) {
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ void store_raw(uint16_t *p, const uint16_t *v) {
        *reinterpret_cast<uint4 *>(p) = make_uint4((uint32_t)v[0] | ((uint32_t)v[1] << 16), (uint32_t)v[2] | ((uint32_t)v[3] << 16),
                                                   (uint32_t)v[4] | ((uint32_t)v[5] << 16), (uint32_t)v[6] | ((uint32_t)v[7] << 16));
    }
};
template <>
struct VecIO<uint16_t, 4> {
    using Raw = uint2;
    static __device__ __forceinline__ Raw load_raw(const uint16_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) {
        v[0] = __uint_as_float(t.x << 16); v[1] = __uint_as_float(t.x & 0xffff0000u);
        v[2] = __uint_as_float(t.y << 16); v[3] = __uint_as_float(t.y & 0xffff0000u);
    }
    static __device__ __forceinline__ void store_raw(uint16_t *p, const uint16_t *v) {
        *reinterpret_cast<uint2 *>(p) = make_uint2((uint32_t)v[0] | ((uint32_t)v[1] << 16), (uint32_t)v[2] | ((uint32_t)v[3] << 16));
    }
};
template <>
struct VecIO<uint16_t, 2> {
    using Raw = uint32_t;
    static __device__ __forceinline__ Raw load_raw(const uint16_t *p) { return __ldg(reinterpret_cast<const unsigned int *>(p)); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) {
        v[0] = __uint_as_float(t << 16); v[1] = __uint_as_float(t & 0xffff0000u);
    }
    static __device__ __forceinline__ void store_raw(uint16_t *p, const uint16_t *v) {
        *reinterpret_cast<uint32_t *>(p) = (uint32_t)v[0] | ((uint32_t)v[1] << 16);
    }
};
template <>
struct VecIO<uint16_t, 1> {
    using Raw = uint16_t;
    static __device__ __forceinline__ Raw load_raw(const uint16_t *p) { return __ldg(p); }
    static __device__ __forceinline__ void cvt(const Raw &t, float *v) { v[0] = bf16_bits_to_f32(t); }
    static __device__ __forceinline__ void store_raw(uint16_t *p, const uint16_t *v) { *p = v[0]; }
};

template <typename T, int VEC>
__device__ __forceinline__ void vec_load(const T *p, float *v) {
    VecIO<T, VEC>::cvt(VecIO<T, VEC>::load_raw(p), v);
}

// f32 value -> element of type T (bf16 rounds to nearest even)
template <typename T>
__device__ __forceinline__ T to_elem(float f);
template <>
__device__ __forceinline__ float to_elem<float>(float f) { return f; }
template <>
__device__ __forceinline__ uint16_t to_elem<uint16_t>(float f) { return f32_to_bf16_bits(f); }

// ----------------------------------------------------------------- reduction state
// max keeps (best, slot of the first best, "another value equals best", NaN seen), branch-free;
// the first value pushed starts it (arg < 0 marks "no value yet"). NaN is tracked by a
// NaN-propagating max (max.NaN), so a NaN anywhere makes the result NaN.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

struct MaxState {
    float best, nanacc;
    int arg;  // -1: no value yet
    bool tie;
    __device__ __forceinline__ void init() {
        best = nanacc = __int_as_float(0xff800000);
        arg = -1;
        tie = false;
    }
    __device__ __forceinline__ void push(float v, int slot) {
        const bool gt = v > best || arg < 0;  // the first value always starts the maximum
        const bool eq = v == best;
        tie = !gt && (tie || eq);
        best = gt ? v : best;
        arg = gt ? slot : arg;
        nanacc = max_nan(nanacc, v);
    }
    __device__ __forceinline__ void merge(const MaxState &o) {  // o covers later slots
        if (o.arg < 0) return;
        if (arg < 0) {
            *this = o;
            return;
        }
        nanacc = max_nan(nanacc, o.nanacc);
        if (o.best > best) {
            best = o.best;
            arg = o.arg;
            tie = o.tie;
        } else if (o.best == best) {
            tie = true;
        }
    }
    __device__ __forceinline__ bool nan() const { return nanacc != nanacc; }
    __device__ __forceinline__ float value() const { return nan() ? __int_as_float(0x7fc00000) : (arg < 0 ? 0.0f : best); }
    __device__ __forceinline__ int arg_out() const { return (nan() || tie) ? -1 : arg; }
};

// Queue segment n for the one-CTA-per-segment kernel; true if it was queued. A full queue
// (a CSR with more slots than rows can hold more long segments than it was sized for) leaves
// the segment to its lane group. Called by all G lanes of the group.
template <int G>
__device__ __forceinline__ bool queue_long(int64_t n, int lig, int32_t *long_list, int32_t *long_count,
                                           int64_t max_long) {
    int queued = 0;
    if (lig == 0) {
        const int idx = atomicAdd(long_count, 1);
        queued = idx < max_long;
        if (queued) long_list[idx] = (int32_t)n;
    }
    const int lane = threadIdx.x & 31, leader = lane & ~(G - 1);
    const unsigned gmask = G == 32 ? 0xffffffffu : (((1u << G) - 1u) << leader);
    return __shfl_sync(gmask, queued, leader) != 0;
}

// ---------------------------------------------------------------- packed bf16 max
// Two bf16 channels per 32-bit word. Per channel: the maximum (max.NaN: a NaN anywhere makes it
// NaN), the largest of the other values (`second`, starts as NaN, which max ignores) and the slot
// of the first maximum (updated on strictly greater values). The maximum is tied exactly when
// second == best at the end. Three packed operations and two selects per pair of values.
struct MaxBf16x2 {
    uint32_t best, second;
    int arg_lo, arg_hi;
    __device__ __forceinline__ void first(uint32_t w, int slot) {
        best = w;
        second = 0x7fc07fc0u;  // NaN: no second value yet
        arg_lo = arg_hi = slot;
    }
    __device__ __forceinline__ void push(uint32_t w, int slot) {
        asm("{\n\t.reg .pred gl, gh;\n\t.reg .b32 lo;\n\t"
            "setp.gt.bf16x2 gl|gh, %4, %0;\n\t"
            "selp.b32 %2, %5, %2, gl;\n\t"
            "selp.b32 %3, %5, %3, gh;\n\t"
            "min.bf16x2 lo, %0, %4;\n\t"
            "max.bf16x2 %1, %1, lo;\n\t"
            "max.NaN.bf16x2 %0, %0, %4;\n\t}"
            : "+r"(best), "+r"(second), "+r"(arg_lo), "+r"(arg_hi)
            : "r"(w), "r"(slot));
    }
};

template <int W, typename Raw>
__device__ __forceinline__ void raw_words(const Raw &r, uint32_t (&w)[W]);
template <>
__device__ __forceinline__ void raw_words<4, uint4>(const uint4 &r, uint32_t (&w)[4]) {
    w[0] = r.x; w[1] = r.y; w[2] = r.z; w[3] = r.w;
}
template <>
__device__ __forceinline__ void raw_words<2, uint2>(const uint2 &r, uint32_t (&w)[2]) {
    w[0] = r.x; w[1] = r.y;
}
template <>
__device__ __forceinline__ void raw_words<1, uint32_t>(const uint32_t &r, uint32_t (&w)[1]) {
    w[0] = r;
}

// one channel of segment n by the scalar rules (value, first slot, tie): used when the maximum
// is a zero, whose sign the packed max may not keep from the first occurrence
template <typename T>
__device__ __noinline__ void seg_max_exact(const T *__restrict__ msg, int64_t C, const int32_t *__restrict__ perm,
                                           int s, int e, int64_t ch, float &val, int &argo) {
    MaxState m;
    m.init();
    for (int j = s; j < e; ++j) {
        float x;
        vec_load<T, 1>(msg + (perm ? (int64_t)__ldg(perm + j) : (int64_t)j) * C + ch, &x);
        m.push(x, j);
    }
    val = m.value();
    argo = m.arg_out();
}

// bf16 max of short segments, packed: VEC channels per lane (VEC even)
template <int VEC>
__device__ __forceinline__ void seg_fwd_bf16_max(const uint16_t *__restrict__ msg, int64_t C,
                                                 const int32_t *__restrict__ perm, int s, int e, int64_t n,
                                                 int64_t c, float *__restrict__ out, int32_t *__restrict__ arg) {
    using IO = VecIO<uint16_t, VEC>;
    constexpr int W = VEC / 2;
    constexpr int U = ShortUnroll<VEC>::value;
    MaxBf16x2 mx[W];
    float o[VEC];
    if (e <= s) {
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            o[v] = 0.0f;
            if (arg) arg[n * C + c + v] = -1;
        }
        VecIO<float, VEC>::store(out + n * C + c, o);
        return;
    }
    {  // the first row starts every channel
        uint32_t w[W];
        raw_words<W>(IO::load_raw(msg + (perm ? (int64_t)__ldg(perm + s) : (int64_t)s) * C + c), w);
#pragma unroll
        for (int i = 0; i < W; ++i) mx[i].first(w[i], s);
    }
    int j = s + 1;
    for (; j + U <= e; j += U) {
        typename IO::Raw r[U];
#pragma unroll
        for (int u = 0; u < U; ++u) r[u] = IO::load_raw(msg + (perm ? (int64_t)__ldg(perm + j + u) : (int64_t)(j + u)) * C + c);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            uint32_t w[W];
            raw_words<W>(r[u], w);
#pragma unroll
            for (int i = 0; i < W; ++i) mx[i].push(w[i], j + u);
        }
    }
    for (; j < e; ++j) {
        uint32_t w[W];
        raw_words<W>(IO::load_raw(msg + (perm ? (int64_t)__ldg(perm + j) : (int64_t)j) * C + c), w);
#pragma unroll
        for (int i = 0; i < W; ++i) mx[i].push(w[i], j);
    }
#pragma unroll
    for (int i = 0; i < W; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int v = 2 * i + h;
            const uint32_t bb = h ? (mx[i].best & 0xffff0000u) : (mx[i].best << 16);
            const uint32_t sb = h ? (mx[i].second & 0xffff0000u) : (mx[i].second << 16);
            const float best = __uint_as_float(bb), second = __uint_as_float(sb);
            int a = h ? mx[i].arg_hi : mx[i].arg_lo;
            float val;
            if (best != best) {  // a NaN in the segment
                val = __int_as_float(0x7fc00000);
                a = -1;
            } else if (best == 0.0f) {  // keep the first zero's sign, as the scalar rule does
                seg_max_exact<uint16_t>(msg, C, perm, s, e, c + v, val, a);
            } else {
                val = best;
                if (second == best) a = -1;  // tied maximum
            }
            o[v] = val;
            if (arg) arg[n * C + c + v] = a;
        }
    }
    VecIO<float, VEC>::store(out + n * C + c, o);
}

template <typename T, int VEC, int G, int RED>
__global__ void __launch_bounds__(kSegThreads) seg_fwd_short_kernel(
    const T *__restrict__ msg, int64_t C, const int32_t *__restrict__ perm, const int32_t *__restrict__ ns,
    const int32_t *__restrict__ ne, int64_t N, float *__restrict__ out, int32_t *__restrict__ arg,
    int32_t *__restrict__ long_list, int32_t *__restrict__ long_count, int64_t max_long) {
    constexpr int kGroups = kSegThreads / G;
    const int lig = threadIdx.x % G;
    const int64_t n = (int64_t)blockIdx.x * kGroups + threadIdx.x / G;
    if (n >= N) return;
    const int s = ns[n], e = ne[n];
    if (e - s > kLongSegment && queue_long<G>(n, lig, long_list, long_count, max_long)) return;
    using IO = VecIO<T, VEC>;
    if constexpr (std::is_same<T, uint16_t>::value && RED == GDL_REDUCE_MAX && VEC % 2 == 0) {
        for (int64_t c0 = 0; c0 < C; c0 += (int64_t)G * VEC) {
            const int64_t c = c0 + (int64_t)lig * VEC;
            if (c < C) seg_fwd_bf16_max<VEC>(msg, C, perm, s, e, n, c, out, arg);
        }
    } else {
        for (int64_t c0 = 0; c0 < C; c0 += (int64_t)G * VEC) {
            const int64_t c = c0 + (int64_t)lig * VEC;
            if (c >= C) continue;
            float acc[VEC];
            MaxState mx[RED == GDL_REDUCE_MAX ? VEC : 1];
    #pragma unroll
            for (int v = 0; v < VEC; ++v) {
                acc[v] = 0.0f;
                if (RED == GDL_REDUCE_MAX) mx[v].init();
            }
            // batches of U rows with their loads issued together: deg / U memory latencies
            constexpr int U = ShortUnroll<VEC>::value;
            int j = s;
            for (; j + U <= e; j += U) {
                typename IO::Raw r[U];
    #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int64_t row = perm ? (int64_t)__ldg(perm + j + u) : (int64_t)(j + u);
                    r[u] = IO::load_raw(msg + row * C + c);
                }
    #pragma unroll
                for (int u = 0; u < U; ++u) {
                    float x[VEC];
                    IO::cvt(r[u], x);
    #pragma unroll
                    for (int v = 0; v < VEC; ++v) {
                        if (RED == GDL_REDUCE_MAX) mx[v].push(x[v], j + u);
                        else acc[v] = add_ftz(acc[v], x[v]);
                    }
                }
            }
            for (; j < e; ++j) {
                float x[VEC];
                const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
                vec_load<T, VEC>(msg + row * C + c, x);
    #pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    if (RED == GDL_REDUCE_MAX) mx[v].push(x[v], j);
                    else acc[v] = add_ftz(acc[v], x[v]);
                }
            }
            float o[VEC];
    #pragma unroll
            for (int v = 0; v < VEC; ++v) {
                if (RED == GDL_REDUCE_MAX) {
                    o[v] = mx[v].value();
                    if (arg) arg[n * C + c + v] = mx[v].arg_out();
                } else if (RED == GDL_REDUCE_MEAN) {
                    o[v] = (e > s) ? __fdiv_rn(acc[v], (float)(e - s)) : 0.0f;
                } else {
                    o[v] = acc[v];
                }
            }
            VecIO<float, VEC>::store(out + n * C + c, o);
        }
    }
}

// one CTA per queued long segment; row group rg folds a contiguous slot range
template <typename T, int VEC, int G, int RED>
__global__ void __launch_bounds__(kSegThreads) seg_fwd_long_kernel(
    const T *__restrict__ msg, int64_t C, const int32_t *__restrict__ perm, const int32_t *__restrict__ ns,
    const int32_t *__restrict__ ne, float *__restrict__ out, int32_t *__restrict__ arg,
    const int32_t *__restrict__ long_list, const int32_t *__restrict__ long_count) {
    // launched with max_long CTAs: entries beyond the queue's capacity were handled in place
    constexpr int kRG = kSegThreads / G;
    __shared__ float part[kRG][G * VEC];
    __shared__ int part_arg[RED == GDL_REDUCE_MAX ? kRG : 1][RED == GDL_REDUCE_MAX ? G * VEC : 1];
    __shared__ unsigned char part_tie[RED == GDL_REDUCE_MAX ? kRG : 1][RED == GDL_REDUCE_MAX ? G * VEC : 1];
    __shared__ float part_nan[RED == GDL_REDUCE_MAX ? kRG : 1][RED == GDL_REDUCE_MAX ? G * VEC : 1];
    if ((int)blockIdx.x >= *long_count) return;
    const int64_t n = long_list[blockIdx.x];
    const int s = ns[n], e = ne[n];
    const int deg = e - s;
    const int rg = threadIdx.x / G, lig = threadIdx.x % G;
    const int chunk = (deg + kRG - 1) / kRG;
    const int j0 = s + rg * chunk;
    const int j1 = min(j0 + chunk, e);
    for (int64_t c0 = 0; c0 < C; c0 += (int64_t)G * VEC) {
        const int64_t c = c0 + (int64_t)lig * VEC;
        const bool active = c < C;
        float acc[VEC];
        MaxState mx[RED == GDL_REDUCE_MAX ? VEC : 1];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            acc[v] = 0.0f;
            if (RED == GDL_REDUCE_MAX) mx[v].init();
        }
        if (active) {
            int j = j0;
            for (; j + kUnroll <= j1; j += kUnroll) {
                float x[kUnroll][VEC];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int64_t row = perm ? (int64_t)__ldg(perm + j + u) : (int64_t)(j + u);
                    vec_load<T, VEC>(msg + row * C + c, x[u]);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u)
#pragma unroll
                    for (int v = 0; v < VEC; ++v) {
                        if (RED == GDL_REDUCE_MAX) mx[v].push(x[u][v], j + u);
                        else acc[v] = add_ftz(acc[v], x[u][v]);
                    }
            }
            for (; j < j1; ++j) {
                float x[VEC];
                const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
                vec_load<T, VEC>(msg + row * C + c, x);
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    if (RED == GDL_REDUCE_MAX) mx[v].push(x[v], j);
                    else acc[v] = add_ftz(acc[v], x[v]);
                }
            }
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            const int k = lig * VEC + v;
            if (RED == GDL_REDUCE_MAX) {
                part[rg][k] = mx[v].best;
                part_arg[rg][k] = mx[v].arg;
                part_tie[rg][k] = mx[v].tie;
                part_nan[rg][k] = mx[v].nanacc;
            } else {
                part[rg][k] = acc[v];
            }
        }
        __syncthreads();
        for (int k = threadIdx.x; k < G * VEC; k += kSegThreads) {
            const int64_t ch = c0 + k;
            if (ch < C) {
                if (RED == GDL_REDUCE_MAX) {
                    MaxState m;
                    m.init();
                    for (int r = 0; r < kRG; ++r) {
                        MaxState o;
                        o.best = part[r][k]; o.arg = part_arg[r][k]; o.tie = part_tie[r][k] != 0; o.nanacc = part_nan[r][k];
                        m.merge(o);
                    }
                    out[n * C + ch] = m.value();
                    if (arg) arg[n * C + ch] = m.arg_out();
                } else {
                    float a = 0.0f;
                    for (int r = 0; r < kRG; ++r) a = add_ftz(a, part[r][k]);
                    out[n * C + ch] = (RED == GDL_REDUCE_MEAN) ? __fdiv_rn(a, (float)deg) : a;
                }
            }
        }
        __syncthreads();
    }
}

// gradient of one (segment, VEC channels) for slots [j0, j1) of segment n. The values a slot
// can receive are fixed per segment (sum: g; mean: g / deg; max: g where the slot holds the
// maximum, 0 * g elsewhere -- torch's mask * share, signed zeros included), so they are converted
// to T once and the slots are a pure store stream. A max channel without a unique maximum (arg
// -1: tied or NaN) is written here too for f32 when arg was kept (its lane reads its row chunks to
// find the maxima), else by seg_bwd_max_fix_kernel afterwards.
template <typename T, int VEC, int RED>
__device__ __forceinline__ void seg_bwd_range(const float *__restrict__ grad_out, const T *__restrict__ msg,
                                              const float *__restrict__ out, const int32_t *__restrict__ arg,
                                              int64_t C, const int32_t *__restrict__ perm, int64_t n, int s, int e,
                                              int j0, int j1, int64_t c, T *__restrict__ grad_msg) {
    (void)msg;
    (void)out;
    float g[VEC];
    vec_load<float, VEC>(grad_out + n * C + c, g);
    T hit_v[VEC], miss_v[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
        const float base = RED == GDL_REDUCE_MEAN ? __fdiv_rn(g[v], (float)(e - s)) : g[v];
        hit_v[v] = to_elem<T>(1.0f * base);
        miss_v[v] = to_elem<T>(0.0f * base);
    }
    if constexpr (RED == GDL_REDUCE_MAX) {
        // Channels without a unique maximum (arg -1: tied, or a NaN maximum) share the gradient
        // evenly among the slots equal to the maximum (torch's amax rule; a NaN maximum equals no
        // slot, so every slot gets 0 * (g / 0)). With arg kept, a lane holding such a channel
        // counts those slots over the whole segment and writes every slot of its range itself --
        // its own row chunks only, read twice -- instead of leaving the channel to a separate pass
        // that would read one element per row per channel. For f32 only: ties are rare there,
        // while bf16 channels tie often enough that most warps would take the two extra row
        // passes (the separate pass is cheaper for them).
        if (arg && sizeof(T) == 4) {
            int a[VEC];
            bool tied = false;
#pragma unroll
            for (int v = 0; v < VEC; ++v) {
                a[v] = arg[n * C + c + v];
                tied |= a[v] < 0;
            }
            if (tied) {
                float mxv[VEC];
                int cnt[VEC];
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    mxv[v] = out[n * C + c + v];
                    cnt[v] = 0;
                }
#pragma unroll 4
                for (int j = s; j < e; ++j) {
                    float x[VEC];
                    vec_load<T, VEC>(msg + (perm ? (int64_t)__ldg(perm + j) : (int64_t)j) * C + c, x);
#pragma unroll
                    for (int v = 0; v < VEC; ++v) cnt[v] += (a[v] < 0 && x[v] == mxv[v]) ? 1 : 0;
                }
                T thit[VEC], tmiss[VEC];
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    const float base = __fdiv_rn(g[v], (float)cnt[v]);
                    thit[v] = to_elem<T>(1.0f * base);
                    tmiss[v] = to_elem<T>(0.0f * base);
                }
#pragma unroll 4
                for (int j = j0; j < j1; ++j) {
                    const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
                    float x[VEC];
                    vec_load<T, VEC>(msg + row * C + c, x);
                    T val[VEC];
#pragma unroll
                    for (int v = 0; v < VEC; ++v)
                        val[v] = a[v] >= 0 ? (a[v] == j ? hit_v[v] : miss_v[v]) : (x[v] == mxv[v] ? thit[v] : tmiss[v]);
                    VecIO<T, VEC>::store_raw(grad_msg + row * C + c, val);
                }
                return;
            }
        }
    }
    if constexpr (RED == GDL_REDUCE_MAX && sizeof(T) == 4) {
        // f32: select per slot and channel (every channel here has a unique maximum, or no arg was
        // kept and the fix-up pass rewrites them all)
        int a[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) a[v] = arg ? arg[n * C + c + v] : -1;
        for (int j = j0; j < j1; ++j) {
            const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
            T val[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) val[v] = a[v] == j ? hit_v[v] : miss_v[v];
            VecIO<T, VEC>::store_raw(grad_msg + row * C + c, val);
        }
        return;
    }
    // bf16 max (and sum / mean): one constant row for every slot -- for max the miss row, then
    // each channel's unique maximum written over it, which costs no per-value work per slot
    const T *row_v = RED == GDL_REDUCE_MAX ? miss_v : hit_v;
    for (int j = j0; j < j1; ++j) {
        const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
        VecIO<T, VEC>::store_raw(grad_msg + row * C + c, row_v);
    }
    if constexpr (RED == GDL_REDUCE_MAX) {
        if (!arg) return;  // every channel is fixed up afterwards
#pragma unroll
        for (int v = 0; v < VEC; ++v) {  // the unique maximum's slot, after its miss row (same thread)
            const int av = arg[n * C + c + v];
            if (av >= j0 && av < j1) {
                const int64_t row = perm ? (int64_t)__ldg(perm + av) : (int64_t)av;
                grad_msg[row * C + c + v] = hit_v[v];
            }
        }
    }
}

// Max channels without a unique maximum (arg -1, or no arg at all): the gradient is shared evenly
// among the slots equal to the maximum (torch's amax rule); a NaN maximum equals no slot, so every
// slot gets 0 * (g / 0). One warp per segment: the lanes read the segment's arg row, and for each
// channel to fix, every lane loads the value of one slot, a ballot counts the maxima, and the
// lanes write the shares (segments longer than 32 slots take their slots 32 at a time).
constexpr int kFixWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kFixWarps * 32) seg_bwd_max_fix_kernel(
    const float *__restrict__ grad_out, const T *__restrict__ msg, const float *__restrict__ out,
    const int32_t *__restrict__ arg, int64_t C, const int32_t *__restrict__ perm, const int32_t *__restrict__ ns,
    const int32_t *__restrict__ ne, int64_t N, T *__restrict__ grad_msg) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kFixWarps;
    for (int64_t n = (int64_t)blockIdx.x * kFixWarps + (threadIdx.x >> 5); n < N; n += nw) {
        const int s = ns[n], e = ne[n];
        if (e <= s) continue;  // uniform over the warp
        for (int64_t c0 = 0; c0 < C; c0 += 32) {
            const int64_t cl = c0 + lane;
            unsigned todo = __ballot_sync(0xffffffffu, cl < C && (!arg || arg[n * C + cl] < 0));
            while (todo) {
                const int64_t ch = c0 + __ffs(todo) - 1;
                todo &= todo - 1;
                const float mx = out[n * C + ch];
                int cnt = 0;
                for (int j0 = s; j0 < e; j0 += 32) {
                    const int j = j0 + lane;
                    bool eq = false;
                    if (j < e) {
                        float x;
                        vec_load<T, 1>(msg + (perm ? (int64_t)__ldg(perm + j) : (int64_t)j) * C + ch, &x);
                        eq = x == mx;
                    }
                    cnt += __popc(__ballot_sync(0xffffffffu, eq));
                }
                const float base = __fdiv_rn(grad_out[n * C + ch], (float)cnt);
                const T hit = to_elem<T>(1.0f * base), miss = to_elem<T>(0.0f * base);
                for (int j0 = s; j0 < e; j0 += 32) {
                    const int j = j0 + lane;
                    if (j < e) {
                        const int64_t row = perm ? (int64_t)__ldg(perm + j) : (int64_t)j;
                        float x;
                        vec_load<T, 1>(msg + row * C + ch, &x);
                        grad_msg[row * C + ch] = x == mx ? hit : miss;
                    }
                }
            }
        }
    }
}

template <typename T, int VEC, int G, int RED>
__global__ void __launch_bounds__(kSegThreads) seg_bwd_short_kernel(
    const float *__restrict__ grad_out, const T *__restrict__ msg, const float *__restrict__ out,
    const int32_t *__restrict__ arg, int64_t C, const int32_t *__restrict__ perm, const int32_t *__restrict__ ns,
    const int32_t *__restrict__ ne, int64_t N, T *__restrict__ grad_msg, int32_t *__restrict__ long_list,
    int32_t *__restrict__ long_count, int64_t max_long) {
    constexpr int kGroups = kSegThreads / G;
    const int lig = threadIdx.x % G;
    const int64_t n = (int64_t)blockIdx.x * kGroups + threadIdx.x / G;
    if (n >= N) return;
    const int s = ns[n], e = ne[n];
    if (e <= s) return;
    if (e - s > kLongSegment && queue_long<G>(n, lig, long_list, long_count, max_long)) return;
    for (int64_t c0 = 0; c0 < C; c0 += (int64_t)G * VEC) {
        const int64_t c = c0 + (int64_t)lig * VEC;
        if (c < C) seg_bwd_range<T, VEC, RED>(grad_out, msg, out, arg, C, perm, n, s, e, s, e, c, grad_msg);
    }
}

template <typename T, int VEC, int G, int RED>
__global__ void __launch_bounds__(kSegThreads) seg_bwd_long_kernel(
    const float *__restrict__ grad_out, const T *__restrict__ msg, const float *__restrict__ out,
    const int32_t *__restrict__ arg, int64_t C, const int32_t *__restrict__ perm, const int32_t *__restrict__ ns,
    const int32_t *__restrict__ ne, T *__restrict__ grad_msg, const int32_t *__restrict__ long_list,
    const int32_t *__restrict__ long_count) {
    constexpr int kRG = kSegThreads / G;
    if ((int)blockIdx.x >= *long_count) return;
    const int64_t n = long_list[blockIdx.x];
    const int s = ns[n], e = ne[n];
    const int rg = threadIdx.x / G, lig = threadIdx.x % G;
    const int chunk = (e - s + kRG - 1) / kRG;
    const int j0 = s + rg * chunk;
    const int j1 = min(j0 + chunk, e);
    if (j0 >= j1) return;
    for (int64_t c0 = 0; c0 < C; c0 += (int64_t)G * VEC) {
        const int64_t c = c0 + (int64_t)lig * VEC;
        if (c < C) seg_bwd_range<T, VEC, RED>(grad_out, msg, out, arg, C, perm, n, s, e, j0, j1, c, grad_msg);
    }
}

// ----------------------------------------------------------------- CSR build kernels
__global__ void csr_keys_kernel(const int64_t *__restrict__ col, int64_t E, uint32_t *__restrict__ keys) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < E) keys[i] = (uint32_t)(int32_t)col[i];
}

// segment_reduce_kernel.cu:30-50: boundaries of runs of equal destinations
__global__ void csr_offsets_kernel(const int32_t *__restrict__ cs, int64_t E, int64_t N, int32_t *__restrict__ ns,
                                   int32_t *__restrict__ ne) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= E) return;
    const int32_t v = cs[i];
    if (v < 0 || v >= N) return;
    if (i == 0 || cs[i - 1] != v) ns[v] = (int32_t)i;
    if (i == E - 1 || cs[i + 1] != v) ne[v] = (int32_t)(i + 1);
}

// ----------------------------------------------------------------- host dispatch
struct SegShape {
    int vec;
    int group;
};

template <typename T>
static SegShape seg_shape(int64_t C, uintptr_t align_bits) {
    // widest vector that divides C and the row alignment; lanes per segment = C / VEC
    const int maxv = 16 / (int)sizeof(T);
    int vec = 1;
    for (int v = maxv; v >= 1; v >>= 1) {
        if (C % v == 0 && (align_bits % (v * sizeof(T))) == 0) { vec = v; break; }
    }
    // the widest vector: 16-byte accesses keep the most bytes in flight per lane
    int64_t lanes = C / vec;
    int g = 1;
    while (g < lanes && g < 32) g <<= 1;
    return {vec, g};
}

// narrow a shape until its VEC-wide f32 accesses (out / grad_out rows) are aligned too
static SegShape fit_f32_side(SegShape sh, int64_t C, uintptr_t alf) {
    // f32 rows take VEC = 8 as two 16-byte accesses
    while (sh.vec > 1 && alf % (uintptr_t)(sh.vec * 4 < 16 ? sh.vec * 4 : 16) != 0) sh.vec >>= 1;
    int64_t lanes = C / sh.vec;
    int g = 1;
    while (g < lanes && g < 32) g <<= 1;
    sh.group = g;
    return sh;
}

// largest power of two dividing every address and row stride given (the vector width a
// kernel may use for all of them); null pointers do not constrain it
static uintptr_t common_align(std::initializer_list<uintptr_t> vals) {
    uintptr_t a = 0;
    for (uintptr_t v : vals) a |= v;
    if (a == 0) return 256;
    a &= (~a + 1);  // lowest set bit
    return a > 256 ? 256 : a;
}

template <typename T, int VEC, int G, int RED>
static void launch_fwd(const void *msg, int64_t C, const int32_t *perm, const int32_t *ns, const int32_t *ne,
                       int64_t N, float *out, int32_t *arg, int32_t *long_list, int32_t *long_count,
                       int64_t max_long, cudaStream_t st) {
    constexpr int groups = kSegThreads / G;
    const int64_t blocks = (N + groups - 1) / groups;
    seg_fwd_short_kernel<T, VEC, G, RED><<<(unsigned)blocks, kSegThreads, 0, st>>>(
        (const T *)msg, C, perm, ns, ne, N, out, arg, long_list, long_count, max_long);
    if (max_long > 0)
        seg_fwd_long_kernel<T, VEC, G, RED><<<(unsigned)max_long, kSegThreads, 0, st>>>(
            (const T *)msg, C, perm, ns, ne, out, arg, long_list, long_count);
}

template <typename T, int VEC, int RED>
static void launch_fwd_g(int G, const void *msg, int64_t C, const int32_t *perm, const int32_t *ns,
                         const int32_t *ne, int64_t N, float *out, int32_t *arg, int32_t *ll, int32_t *lc,
                         int64_t ml, cudaStream_t st) {
    switch (G) {
    case 1: launch_fwd<T, VEC, 1, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 2: launch_fwd<T, VEC, 2, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 4: launch_fwd<T, VEC, 4, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 8: launch_fwd<T, VEC, 8, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 16: launch_fwd<T, VEC, 16, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    default: launch_fwd<T, VEC, 32, RED>(msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    }
}

template <typename T, int RED>
static void launch_fwd_v(SegShape sh, const void *msg, int64_t C, const int32_t *perm, const int32_t *ns,
                         const int32_t *ne, int64_t N, float *out, int32_t *arg, int32_t *ll, int32_t *lc,
                         int64_t ml, cudaStream_t st) {
    switch (sh.vec) {
    case 8: launch_fwd_g<T, 8, RED>(sh.group, msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 4: launch_fwd_g<T, 4, RED>(sh.group, msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    case 2: launch_fwd_g<T, 2, RED>(sh.group, msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    default: launch_fwd_g<T, 1, RED>(sh.group, msg, C, perm, ns, ne, N, out, arg, ll, lc, ml, st); break;
    }
}

template <typename T, int VEC, int G, int RED>
static void launch_bwd(const float *go, const void *msg, const float *out, const int32_t *arg, int64_t C,
                       const int32_t *perm, const int32_t *ns, const int32_t *ne, int64_t N, void *gm, int32_t *ll,
                       int32_t *lc, int64_t ml, cudaStream_t st) {
    constexpr int groups = kSegThreads / G;
    const int64_t blocks = (N + groups - 1) / groups;
    seg_bwd_short_kernel<T, VEC, G, RED><<<(unsigned)blocks, kSegThreads, 0, st>>>(
        go, (const T *)msg, out, arg, C, perm, ns, ne, N, (T *)gm, ll, lc, ml);
    if (ml > 0)
        seg_bwd_long_kernel<T, VEC, G, RED><<<(unsigned)ml, kSegThreads, 0, st>>>(go, (const T *)msg, out, arg, C, perm,
                                                                                 ns, ne, (T *)gm, ll, lc);
    if (RED == GDL_REDUCE_MAX && (!arg || sizeof(T) != 4)) {  // f32 with arg: done above
        const int64_t fb = (N + kFixWarps - 1) / kFixWarps;
        seg_bwd_max_fix_kernel<T><<<(unsigned)(fb < 16 * kSmCount ? fb : 16 * kSmCount), kFixWarps * 32, 0, st>>>(
            go, (const T *)msg, out, arg, C, perm, ns, ne, N, (T *)gm);
    }
}

template <typename T, int VEC, int RED>
static void launch_bwd_g(int G, const float *go, const void *msg, const float *out, const int32_t *arg, int64_t C,
                         const int32_t *perm, const int32_t *ns, const int32_t *ne, int64_t N, void *gm, int32_t *ll,
                         int32_t *lc, int64_t ml, cudaStream_t st) {
    switch (G) {
    case 1: launch_bwd<T, VEC, 1, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 2: launch_bwd<T, VEC, 2, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 4: launch_bwd<T, VEC, 4, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 8: launch_bwd<T, VEC, 8, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 16: launch_bwd<T, VEC, 16, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    default: launch_bwd<T, VEC, 32, RED>(go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    }
}

template <typename T, int RED>
static void launch_bwd_v(SegShape sh, const float *go, const void *msg, const float *out, const int32_t *arg,
                         int64_t C, const int32_t *perm, const int32_t *ns, const int32_t *ne, int64_t N, void *gm,
                         int32_t *ll, int32_t *lc, int64_t ml, cudaStream_t st) {
    switch (sh.vec) {
    case 8: launch_bwd_g<T, 8, RED>(sh.group, go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 4: launch_bwd_g<T, 4, RED>(sh.group, go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    case 2: launch_bwd_g<T, 2, RED>(sh.group, go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    default: launch_bwd_g<T, 1, RED>(sh.group, go, msg, out, arg, C, perm, ns, ne, N, gm, ll, lc, ml, st); break;
    }
}

}  // namespace gdl

using namespace gdl;

static inline size_t al256(size_t b) { return (b + 255) & ~size_t(255); }

extern "C" size_t gdl_sort_and_build_csr_workspace_size(int64_t num_edges, int64_t num_nodes) {
    (void)num_nodes;
    const int64_t E = num_edges > 0 ? num_edges : 1;
    return al256(sizeof(uint32_t) * E) + radix_scratch_bytes(E, 1) + 256;
}

extern "C" int gdl_sort_and_build_csr(const int64_t *col, int64_t num_edges, int64_t num_nodes, int32_t *col_sorted,
                                      int32_t *perm, int32_t *node_start, int32_t *node_end, void *workspace,
                                      size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_edges < 0 || num_nodes < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(num_edges >= INT32_MAX || num_nodes >= INT32_MAX, GDL_ERR_OVERFLOW);
    if (num_nodes > 0) {
        GDL_RETURN_IF(!node_start || !node_end, GDL_ERR_INVALID);
        GDL_CUDA_TRY(cudaMemsetAsync(node_start, 0, sizeof(int32_t) * num_nodes, st));
        GDL_CUDA_TRY(cudaMemsetAsync(node_end, 0, sizeof(int32_t) * num_nodes, st));
    }
    if (num_edges == 0) return GDL_OK;
    GDL_RETURN_IF(!col || !col_sorted || !perm, GDL_ERR_INVALID);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_sort_and_build_csr_workspace_size(num_edges, num_nodes),
                  GDL_ERR_WORKSPACE);
    char *p = (char *)workspace;
    uint32_t *keys = (uint32_t *)p;
    p += al256(sizeof(uint32_t) * num_edges);
    RadixScratch rs = radix_carve(p, num_edges, 1);
    csr_keys_kernel<<<(unsigned)((num_edges + 255) / 256), 256, 0, st>>>(col, num_edges, keys);
    int bits = 1;
    while (bits < 32 && ((int64_t)1 << bits) < num_nodes) ++bits;
    const int passes = (bits + 7) / 8;
    GDL_CUDA_TRY(radix_sort_pairs(keys, nullptr, (uint32_t *)col_sorted, perm, num_edges, nullptr, 1, passes, nullptr,
                                  rs, st));
    csr_offsets_kernel<<<(unsigned)((num_edges + 255) / 256), 256, 0, st>>>(col_sorted, num_edges, num_nodes,
                                                                            node_start, node_end);
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" size_t gdl_segment_reduce_workspace_size(int64_t num_rows, int64_t num_nodes) {
    (void)num_nodes;
    const int64_t max_long = num_rows / (kLongSegment + 1) + 1;
    return al256(sizeof(int32_t)) + al256(sizeof(int32_t) * max_long);
}

extern "C" int gdl_segment_reduce(const void *msg, int32_t dtype, int64_t num_rows, int64_t C, const int32_t *perm,
                                  const int32_t *node_start, const int32_t *node_end, int64_t num_nodes,
                                  int32_t reduce, float *out, int32_t *arg_out, void *workspace,
                                  size_t workspace_bytes, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_rows < 0 || C <= 0 || num_nodes < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(dtype != GDL_DTYPE_F32 && dtype != GDL_DTYPE_BF16, GDL_ERR_INVALID);
    GDL_RETURN_IF(reduce < GDL_REDUCE_SUM || reduce > GDL_REDUCE_MAX, GDL_ERR_INVALID);
    GDL_RETURN_IF(num_rows >= INT32_MAX, GDL_ERR_OVERFLOW);
    if (num_nodes == 0) return GDL_OK;
    GDL_RETURN_IF(!out || !node_start || !node_end || (num_rows > 0 && !msg), GDL_ERR_INVALID);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_segment_reduce_workspace_size(num_rows, num_nodes),
                  GDL_ERR_WORKSPACE);
    int32_t *long_count = (int32_t *)workspace;
    int32_t *long_list = (int32_t *)((char *)workspace + al256(sizeof(int32_t)));
    const int64_t max_long = num_rows / (kLongSegment + 1) + 1;
    GDL_CUDA_TRY(cudaMemsetAsync(long_count, 0, sizeof(int32_t), st));
    const int64_t esz = dtype == GDL_DTYPE_BF16 ? 2 : 4;
    const uintptr_t al = common_align({(uintptr_t)msg, (uintptr_t)(C * esz), (uintptr_t)out, (uintptr_t)(C * 4)});
    if (dtype == GDL_DTYPE_F32) {
        SegShape sh = seg_shape<float>(C, al);
        if (reduce == GDL_REDUCE_SUM) launch_fwd_v<float, GDL_REDUCE_SUM>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_fwd_v<float, GDL_REDUCE_MEAN>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else launch_fwd_v<float, GDL_REDUCE_MAX>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
    } else {
        // out rows are f32: the vector width must also suit them
        SegShape sh = fit_f32_side(seg_shape<uint16_t>(C, al), C,
                                   common_align({(uintptr_t)out, (uintptr_t)(C * 4)}));
        if (reduce == GDL_REDUCE_SUM) launch_fwd_v<uint16_t, GDL_REDUCE_SUM>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_fwd_v<uint16_t, GDL_REDUCE_MEAN>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else launch_fwd_v<uint16_t, GDL_REDUCE_MAX>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

extern "C" int gdl_segment_reduce_backward(const float *grad_out, const void *msg, int32_t dtype, const float *out,
                                           const int32_t *arg, int64_t num_rows, int64_t C, const int32_t *perm,
                                           const int32_t *node_start, const int32_t *node_end, int64_t num_nodes,
                                           int32_t reduce, void *grad_msg, void *workspace, size_t workspace_bytes,
                                           void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_rows < 0 || C <= 0 || num_nodes < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(dtype != GDL_DTYPE_F32 && dtype != GDL_DTYPE_BF16, GDL_ERR_INVALID);
    GDL_RETURN_IF(reduce < GDL_REDUCE_SUM || reduce > GDL_REDUCE_MAX, GDL_ERR_INVALID);
    GDL_RETURN_IF(num_rows >= INT32_MAX, GDL_ERR_OVERFLOW);
    if (num_nodes == 0 || num_rows == 0) return GDL_OK;
    GDL_RETURN_IF(!grad_out || !grad_msg || !node_start || !node_end, GDL_ERR_INVALID);
    GDL_RETURN_IF(reduce == GDL_REDUCE_MAX && (!msg || !out), GDL_ERR_INVALID);
    GDL_RETURN_IF(!workspace || workspace_bytes < gdl_segment_reduce_workspace_size(num_rows, num_nodes),
                  GDL_ERR_WORKSPACE);
    int32_t *long_count = (int32_t *)workspace;
    int32_t *long_list = (int32_t *)((char *)workspace + al256(sizeof(int32_t)));
    const int64_t max_long = num_rows / (kLongSegment + 1) + 1;
    GDL_CUDA_TRY(cudaMemsetAsync(long_count, 0, sizeof(int32_t), st));
    const int64_t esz = dtype == GDL_DTYPE_BF16 ? 2 : 4;
    const uintptr_t al = common_align({(uintptr_t)grad_out, (uintptr_t)(C * 4), (uintptr_t)grad_msg,
                                       (uintptr_t)(C * esz), (uintptr_t)msg});
    SegShape sh = dtype == GDL_DTYPE_F32 ? seg_shape<float>(C, al) : seg_shape<uint16_t>(C, al);
    sh = fit_f32_side(sh, C, common_align({(uintptr_t)grad_out, (uintptr_t)(C * 4)}));
    const int32_t *a = arg;
    if (dtype == GDL_DTYPE_F32) {
        if (reduce == GDL_REDUCE_SUM) launch_bwd_v<float, GDL_REDUCE_SUM>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_bwd_v<float, GDL_REDUCE_MEAN>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
        else launch_bwd_v<float, GDL_REDUCE_MAX>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
    } else {
        if (reduce == GDL_REDUCE_SUM) launch_bwd_v<uint16_t, GDL_REDUCE_SUM>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_bwd_v<uint16_t, GDL_REDUCE_MEAN>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
        else launch_bwd_v<uint16_t, GDL_REDUCE_MAX>(sh, grad_out, msg, out, a, C, perm, node_start, node_end, num_nodes, grad_msg, long_list, long_count, max_long, st);
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}

// ---------------------------------------------------------------------------------------------
// Segment reduce without any allocation.
//
// Some callers cannot allocate device memory at the moment they reduce: code that runs while a
// CUDA graph is being captured with a static memory plan, plugin hosts (inference engines,
// real-time robot control loops) that forbid cudaMalloc / cudaFree on their enqueue path, or
// programs with no allocator bound to the device at all. gdl_segment_reduce asks them for a
// workspace; this variant instead keeps its only scratch -- the queue of segments longer than
// kLongSegment slots -- in a fixed array compiled into the library. Every GPU that loads the
// library holds that array (64 KiB) until the process exits.
//
// The array is shared by every call on a device and keeps whatever the last call left in it:
// the queue counter is cleared by each call, and two calls whose kernels overlap on the GPU
// (different streams, no ordering between them) race on it and must not be issued.
namespace gdl {

constexpr int kNoAllocSlots = 16384;  // the counter, padding to 256 bytes, then the queue
constexpr int kNoAllocQueue = kNoAllocSlots - 64;
// largest input whose long segments all fit the queue (with at most one slot per row)
constexpr int64_t kNoAllocMaxRows = (int64_t)kNoAllocQueue * (kLongSegment + 1);
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) int32_t g_seg_noalloc_scratch[kNoAllocSlots];

// device address of g_seg_noalloc_scratch, looked up once per device with that device current
// and kept for the process's life (a cudaDeviceReset() ends the context that owns the array;
// the header forbids calls after one)
static int32_t *g_noalloc_ptr[kNoAllocMaxDevices];
static std::mutex g_noalloc_mutex;

static int noalloc_scratch(int32_t **out) {
    int dev = 0;
    GDL_CUDA_TRY(cudaGetDevice(&dev));
    GDL_RETURN_IF(dev < 0 || dev >= kNoAllocMaxDevices, GDL_ERR_UNSUPPORTED);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        GDL_CUDA_TRY(cudaGetSymbolAddress(&p, g_seg_noalloc_scratch));
        g_noalloc_ptr[dev] = (int32_t *)p;
    }
    *out = g_noalloc_ptr[dev];
    return GDL_OK;
}

}  // namespace gdl

extern "C" int gdl_segment_reduce_noalloc(const void *msg, int32_t dtype, int64_t num_rows, int64_t C,
                                          const int32_t *perm, const int32_t *node_start, const int32_t *node_end,
                                          int64_t num_nodes, int32_t reduce, float *out, int32_t *arg_out,
                                          void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    GDL_RETURN_IF(num_rows < 0 || C <= 0 || num_nodes < 0, GDL_ERR_INVALID);
    GDL_RETURN_IF(num_rows > kNoAllocMaxRows, GDL_ERR_OVERFLOW);  // queue would not fit the array
    GDL_RETURN_IF(dtype != GDL_DTYPE_F32 && dtype != GDL_DTYPE_BF16, GDL_ERR_INVALID);
    GDL_RETURN_IF(reduce < GDL_REDUCE_SUM || reduce > GDL_REDUCE_MAX, GDL_ERR_INVALID);
    if (num_nodes == 0) return GDL_OK;
    GDL_RETURN_IF(!out || !node_start || !node_end || (num_rows > 0 && !msg), GDL_ERR_INVALID);
    int32_t *scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != GDL_OK) return rc;
    int32_t *long_count = scratch;
    int32_t *long_list = scratch + 64;  // 256-byte offset
    const int64_t want = num_rows / (kLongSegment + 1) + 1;
    const int64_t max_long = want < kNoAllocQueue ? want : kNoAllocQueue;
    GDL_CUDA_TRY(cudaMemsetAsync(long_count, 0, sizeof(int32_t), st));
    const int64_t esz = dtype == GDL_DTYPE_BF16 ? 2 : 4;
    const uintptr_t al = common_align({(uintptr_t)msg, (uintptr_t)(C * esz), (uintptr_t)out, (uintptr_t)(C * 4)});
    if (dtype == GDL_DTYPE_F32) {
        SegShape sh = seg_shape<float>(C, al);
        if (reduce == GDL_REDUCE_SUM) launch_fwd_v<float, GDL_REDUCE_SUM>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_fwd_v<float, GDL_REDUCE_MEAN>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else launch_fwd_v<float, GDL_REDUCE_MAX>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
    } else {
        SegShape sh = fit_f32_side(seg_shape<uint16_t>(C, al), C, common_align({(uintptr_t)out, (uintptr_t)(C * 4)}));
        if (reduce == GDL_REDUCE_SUM) launch_fwd_v<uint16_t, GDL_REDUCE_SUM>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else if (reduce == GDL_REDUCE_MEAN) launch_fwd_v<uint16_t, GDL_REDUCE_MEAN>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
        else launch_fwd_v<uint16_t, GDL_REDUCE_MAX>(sh, msg, C, perm, node_start, node_end, num_nodes, out, arg_out, long_list, long_count, max_long, st);
    }
    GDL_CUDA_TRY(cudaGetLastError());
    return GDL_OK;
}
