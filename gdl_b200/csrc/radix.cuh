// radix.cuh -- stable, segmented LSD radix sort of (uint32 key, int32 value) pairs.
//
// Segments are contiguous ranges [seg_ptr[b], seg_ptr[b+1]) sorted independently (one
// segment = a plain sort). Every pass handles 8 key bits in three steps:
//   upsweep   : per 2048-key tile (tiles never cross a segment) a 256-bin digit histogram,
//               stored at  tile_base(b)*256 + digit*ntiles(b) + local_tile
//   scan      : one exclusive scan over that array; because the layout is
//               [segment][digit][tile], each entry's prefix is exactly the output slot of
//               the tile's first key with that digit
//   downsweep : each tile ranks its keys stably (warp match + per-warp digit counters in
//               shared memory, in index order) and scatters them.
// Stability makes it equal to a sort by (segment, key, original position), which is the
// order CUB's DeviceRadixSort gives the reference (radius_graph_kernel.cu:325-347,
// segment_reduce_kernel.cu:130-152).
#pragma once

#include "scan.cuh"

namespace gdl {

constexpr int kRadixThreads = 256;
constexpr int kRadixItems = 8;
constexpr int kRadixTile = kRadixThreads * kRadixItems;
constexpr int kRadixBins = 256;
constexpr int kRadixWarps = kRadixThreads / 32;

struct RadixScratch {
    int32_t *seg_tile_base;  // [num_segments + 1]
    uint32_t *hist;          // [kRadixBins * max_tiles]
    uint32_t *hist_totals;   // [scan_blocks(kRadixBins * max_tiles) + 1]
    uint32_t *keys_tmp;      // [n]
    int32_t *vals_tmp;       // [n]
};

inline int64_t radix_max_tiles(int64_t n, int32_t num_segments) { return n / kRadixTile + num_segments + 1; }

inline size_t radix_scratch_bytes(int64_t n, int32_t num_segments) {
    const int64_t mt = radix_max_tiles(n, num_segments);
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    return al(sizeof(int32_t) * (num_segments + 1)) + al(sizeof(uint32_t) * kRadixBins * mt) +
           al(sizeof(uint32_t) * (scan_blocks(kRadixBins * mt) + 1)) + al(sizeof(uint32_t) * (n > 0 ? n : 1)) +
           al(sizeof(int32_t) * (n > 0 ? n : 1));
}

inline RadixScratch radix_carve(char *&p, int64_t n, int32_t num_segments) {
    const int64_t mt = radix_max_tiles(n, num_segments);
    auto take = [&](size_t b) {
        char *r = p;
        p += (b + 255) & ~size_t(255);
        return r;
    };
    RadixScratch s;
    s.seg_tile_base = (int32_t *)take(sizeof(int32_t) * (num_segments + 1));
    s.hist = (uint32_t *)take(sizeof(uint32_t) * kRadixBins * mt);
    s.hist_totals = (uint32_t *)take(sizeof(uint32_t) * (scan_blocks(kRadixBins * mt) + 1));
    s.keys_tmp = (uint32_t *)take(sizeof(uint32_t) * (n > 0 ? n : 1));
    s.vals_tmp = (int32_t *)take(sizeof(int32_t) * (n > 0 ? n : 1));
    return s;
}

__device__ __forceinline__ int64_t seg_begin(const int64_t *seg_ptr, int b, int64_t n) {
    return seg_ptr ? seg_ptr[b] : (b == 0 ? 0 : n);
}

// tiles per segment -> exclusive prefix (one block)
static __global__ void __launch_bounds__(kScanThreads) radix_tiles_kernel(const int64_t *__restrict__ seg_ptr, int32_t B,
                                                                   int64_t n, int32_t *__restrict__ seg_tile_base) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t total;
    int32_t carry = 0;
    for (int32_t b0 = 0; b0 < B; b0 += kScanThreads) {
        const int32_t b = b0 + threadIdx.x;
        int32_t t = 0;
        if (b < B) {
            const int64_t len = seg_begin(seg_ptr, b + 1, n) - seg_begin(seg_ptr, b, n);
            t = (int32_t)((len + kRadixTile - 1) / kRadixTile);
        }
        int32_t off = block_exclusive_scan<int32_t>(t, warp_sums, &total) + carry;
        if (b < B) seg_tile_base[b] = off;
        carry += total;
    }
    if (threadIdx.x == 0) seg_tile_base[B] = carry;
}

__device__ __forceinline__ int find_segment(const int32_t *__restrict__ base, int B, int t) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (base[mid] <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ bool pass_skipped(const int32_t *key_bits, int shift) {
    return key_bits != nullptr && shift >= *key_bits;
}

static __global__ void __launch_bounds__(kRadixThreads) radix_upsweep_kernel(
    const uint32_t *__restrict__ keys, const int64_t *__restrict__ seg_ptr, int32_t B, int64_t n,
    const int32_t *__restrict__ seg_tile_base, uint32_t *__restrict__ hist, int shift,
    const int32_t *__restrict__ key_bits) {
    __shared__ uint32_t cnt[kRadixBins];
    const int t = blockIdx.x;
    if (t >= seg_tile_base[B] || pass_skipped(key_bits, shift)) return;
    const int b = find_segment(seg_tile_base, B, t);
    const int lt = t - seg_tile_base[b];
    const int nt = seg_tile_base[b + 1] - seg_tile_base[b];
    const int64_t s0 = seg_begin(seg_ptr, b, n) + (int64_t)lt * kRadixTile;
    const int64_t se = seg_begin(seg_ptr, b + 1, n);
    const int64_t s1 = s0 + kRadixTile < se ? s0 + kRadixTile : se;
    cnt[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t i = s0 + threadIdx.x; i < s1; i += kRadixThreads) atomicAdd(&cnt[(keys[i] >> shift) & 255u], 1u);
    __syncthreads();
    const int d = threadIdx.x;
    hist[(int64_t)seg_tile_base[b] * kRadixBins + (int64_t)d * nt + lt] = cnt[d];
}

// vals_in == nullptr means identity values (the global key position).
static __global__ void __launch_bounds__(kRadixThreads) radix_downsweep_kernel(
    const uint32_t *__restrict__ keys_in, const int32_t *__restrict__ vals_in, uint32_t *__restrict__ keys_out,
    int32_t *__restrict__ vals_out, const int64_t *__restrict__ seg_ptr, int32_t B, int64_t n,
    const int32_t *__restrict__ seg_tile_base, const uint32_t *__restrict__ hist_scanned,
    const uint32_t *__restrict__ hist_totals, int shift, const int32_t *__restrict__ key_bits) {
    __shared__ uint32_t warp_cnt[kRadixWarps][kRadixBins];
    const int t = blockIdx.x;
    if (t >= seg_tile_base[B]) return;
    const int b = find_segment(seg_tile_base, B, t);
    const int lt = t - seg_tile_base[b];
    const int nt = seg_tile_base[b + 1] - seg_tile_base[b];
    const int64_t origin = seg_begin(seg_ptr, 0, n);
    const int64_t s0 = seg_begin(seg_ptr, b, n) + (int64_t)lt * kRadixTile;
    const int64_t se = seg_begin(seg_ptr, b + 1, n);
    const int64_t s1 = s0 + kRadixTile < se ? s0 + kRadixTile : se;

    if (pass_skipped(key_bits, shift)) {  // digit is zero everywhere: order unchanged
        for (int64_t i = s0 + threadIdx.x; i < s1; i += kRadixThreads) {
            keys_out[i] = keys_in[i];
            vals_out[i] = vals_in ? vals_in[i] : (int32_t)i;
        }
        return;
    }

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int d = threadIdx.x; d < kRadixWarps * kRadixBins; d += kRadixThreads) (&warp_cnt[0][0])[d] = 0;
    __syncthreads();

    uint32_t key[kRadixItems], dig[kRadixItems], rank[kRadixItems];
    int32_t val[kRadixItems];
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < kRadixItems; ++i) {
        const int64_t idx = s0 + (int64_t)warp * 32 * kRadixItems + i * 32 + lane;
        const bool valid = idx < s1;
        key[i] = valid ? keys_in[idx] : 0u;
        val[i] = valid ? (vals_in ? vals_in[idx] : (int32_t)idx) : 0;
        dig[i] = valid ? ((key[i] >> shift) & 255u) : 256u;
        const unsigned peers = __match_any_sync(0xffffffffu, dig[i]);
        const unsigned before = __popc(peers & lt_mask);
        uint32_t base = 0;
        if (valid) base = warp_cnt[warp][dig[i]];
        __syncwarp();
        if (valid && before == 0) warp_cnt[warp][dig[i]] = base + __popc(peers);
        __syncwarp();
        rank[i] = base + before;
    }
    __syncthreads();
    {
        const int d = threadIdx.x;  // kRadixThreads == kRadixBins
        const int64_t e = (int64_t)seg_tile_base[b] * kRadixBins + (int64_t)d * nt + lt;
        uint32_t running = (uint32_t)origin + hist_scanned[e] + hist_totals[e / kScanTile];
#pragma unroll
        for (int w = 0; w < kRadixWarps; ++w) {
            const uint32_t c = warp_cnt[w][d];
            warp_cnt[w][d] = running;
            running += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kRadixItems; ++i) {
        if (dig[i] < 256u) {
            const uint32_t dst = warp_cnt[warp][dig[i]] + rank[i];
            keys_out[dst] = key[i];
            vals_out[dst] = val[i];
        }
    }
}

// Sort keys (uint32, positions [seg_ptr[0], seg_ptr[B]) or [0, n) if seg_ptr is null) with
// values; `passes` 8-bit passes from bit 0. key_bits (device, nullable) lets passes at or
// above that many significant bits degrade to copies. Output lands in keys_out/vals_out.
// keys_in is not modified; it may alias neither output.
inline cudaError_t radix_sort_pairs(const uint32_t *keys_in, const int32_t *vals_in, uint32_t *keys_out,
                                    int32_t *vals_out, int64_t n, const int64_t *seg_ptr, int32_t B, int passes,
                                    const int32_t *key_bits, const RadixScratch &s, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (B < 1) B = 1;
    const int64_t mt = radix_max_tiles(n, B);
    const int64_t hn = (int64_t)kRadixBins * mt;
    radix_tiles_kernel<<<1, kScanThreads, 0, stream>>>(seg_ptr, B, n, s.seg_tile_base);
    if (passes < 1) passes = 1;
    // ping-pong so that the last pass writes the outputs
    const uint32_t *kin = keys_in;
    const int32_t *vin = vals_in;
    for (int p = 0; p < passes; ++p) {
        const bool last = p == passes - 1;
        uint32_t *kout = last ? keys_out : (((passes - 1 - p) & 1) ? s.keys_tmp : keys_out);
        int32_t *vout = last ? vals_out : (((passes - 1 - p) & 1) ? s.vals_tmp : vals_out);
        const int shift = 8 * p;
        radix_upsweep_kernel<<<(unsigned)mt, kRadixThreads, 0, stream>>>(kin, seg_ptr, B, n, s.seg_tile_base, s.hist,
                                                                        shift, key_bits);
        scan_local_kernel<uint32_t, uint32_t>
            <<<(unsigned)scan_blocks(hn), kScanThreads, 0, stream>>>(s.hist, s.hist, s.hist_totals, hn);
        scan_totals_kernel<uint32_t><<<1, kScanThreads, 0, stream>>>(s.hist_totals, scan_blocks(hn), nullptr);
        radix_downsweep_kernel<<<(unsigned)mt, kRadixThreads, 0, stream>>>(
            kin, vin, kout, vout, seg_ptr, B, n, s.seg_tile_base, s.hist, s.hist_totals, shift, key_bits);
        kin = kout;
        vin = vout;
    }
    return cudaGetLastError();
}

}  // namespace gdl
