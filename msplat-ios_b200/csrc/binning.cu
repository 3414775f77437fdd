// binning.cu — tile intersection counting, offsets, key emission and the
// per-tile depth sort.
//
// Replaces scatter_to_prealloc_bins_kernel (core/metal/msplat_metal.metal:
// 1557-1591), prefix_sum_kernel (:3093-3145) and the sort half of
// bitonic_sort_per_tile_2dgs_kernel (:1606-1664).
//
// The reference scatters into fixed 2048-slot bins with atomics, so which
// intersections survive in an overfull tile depends on the atomic race. Here
// every step is deterministic:
//   1. the projection adds each Gaussian's tile rectangle into a 2-D
//      difference array (4 atomics per Gaussian instead of one per tile);
//   2. one CTA integrates it into exact per-tile counts, clamps them to 2048
//      and scans both the raw and the kept counts;
//   3. each (Gaussian, tile) pair appends the key (depth_bits << 32) | id into
//      its tile's raw segment (slot order is irrelevant, the set is exact);
//   4. one CTA per tile keeps, for overfull tiles, the 2048 lowest Gaussian
//      ids (a three-pass radix select on the id bits) and sorts the kept keys
//      ascending in shared memory. Output: the sorted Gaussian ids.
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

constexpr int kCountThreads = 1024;
// Work estimate of a tile row for band balancing: kept intersections plus a
// fixed per-tile cost (launch, id loads, per-pixel outputs).
constexpr int kRowWorkPerTile = 64;

__global__ void __launch_bounds__(kCountThreads)
k_tile_counts(const int32_t* __restrict__ diff, int tx, int ty, int row0, int row1, int32_t* __restrict__ raw_counts,
              int64_t* __restrict__ raw_start, int2* __restrict__ tile_bins, int64_t* __restrict__ totals,
              int64_t* __restrict__ row_work) {
    const int dw = tx + 1;
    // Column prefix over y (one thread per tile column).
    for (int x = threadIdx.x; x < tx; x += blockDim.x) {
        int run = 0;
        for (int y = 0; y < ty; ++y) {
            run += diff[y * dw + x];
            raw_counts[y * tx + x] = run;
        }
    }
    __syncthreads();
    // Row prefix over x (one thread per tile row); rows outside the band
    // [row0, row1) get zero counts so that nothing is emitted for them.
    for (int y = threadIdx.x; y < ty; y += blockDim.x) {
        int run = 0;
        int64_t work = 0;
        int32_t* row = raw_counts + (size_t)y * tx;
        const bool in_band = y >= row0 && y < row1;
        for (int x = 0; x < tx; ++x) {
            run += row[x];
            row[x] = in_band ? run : 0;
            work += min(run, kMaxTileElems) + kRowWorkPerTile;
        }
        if (row_work) row_work[y] = work;
    }
    __syncthreads();
    // Exclusive scans of raw (int64) and kept = min(raw, 2048) (int32).
    const int T = tx * ty;
    const int chunk = (T + blockDim.x - 1) / blockDim.x;
    const int b = threadIdx.x * chunk;
    const int e = min(b + chunk, T);
    int64_t sraw = 0;
    int32_t skept = 0;
    for (int t = b; t < e; ++t) {
        int r = raw_counts[t];
        sraw += r;
        skept += min(r, kMaxTileElems);
    }
    __shared__ int64_t s_raw[kCountThreads];
    __shared__ int32_t s_kept[kCountThreads];
    s_raw[threadIdx.x] = sraw;
    s_kept[threadIdx.x] = skept;
    __syncthreads();
    // Hillis-Steele inclusive scan over the per-thread sums.
    for (int off = 1; off < (int)blockDim.x; off <<= 1) {
        int64_t vr = threadIdx.x >= off ? s_raw[threadIdx.x - off] : 0;
        int32_t vk = threadIdx.x >= off ? s_kept[threadIdx.x - off] : 0;
        __syncthreads();
        s_raw[threadIdx.x] += vr;
        s_kept[threadIdx.x] += vk;
        __syncthreads();
    }
    int64_t run_raw = s_raw[threadIdx.x] - sraw;
    int32_t run_kept = s_kept[threadIdx.x] - skept;
    for (int t = b; t < e; ++t) {
        int r = raw_counts[t];
        int k = min(r, kMaxTileElems);
        raw_start[t] = run_raw;
        tile_bins[t] = make_int2(run_kept, run_kept + k);
        run_raw += r;
        run_kept += k;
    }
    if (threadIdx.x == blockDim.x - 1) {
        totals[0] = s_raw[threadIdx.x];
        totals[1] = s_kept[threadIdx.x];
    }
}

// One warp per 32 consecutive Gaussians: their clipped tile rectangles are
// flattened into (Gaussian, tile) pairs by a warp prefix sum of the areas, and
// every lane takes one pair per round (owner found by a binary search over the
// lanes' exclusive offsets), so a warp keeps 32 independent slot atomics in
// flight whatever the rectangle sizes.
__global__ void __launch_bounds__(256)
k_emit_keys(int n, const uint2* __restrict__ rects, const float* __restrict__ depths, int tx, int row0, int row1,
            const int64_t* __restrict__ raw_start, int32_t* __restrict__ fill, uint64_t* __restrict__ keys) {
    constexpr unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    int x0 = 0, y0 = 0, w = 0, area = 0;
    uint64_t key = 0;
    if (i < n) {
        const uint2 r = rects[i];
        x0 = r.x & 0xFFFF;
        const int x1 = r.y & 0xFFFF;
        y0 = max((int)(r.x >> 16), row0);
        const int y1 = min((int)(r.y >> 16), row1);
        w = x1 - x0;
        if (w > 0 && y1 > y0) area = w * (y1 - y0);
        key = ((uint64_t)__float_as_uint(depths[i]) << 32) | (uint64_t)(uint32_t)i;
    }
    int incl = area;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(full, incl, d);
        if (lane >= d) incl += v;
    }
    const int total = __shfl_sync(full, incl, 31);
    const int excl = incl - area;
    for (int base = 0; base < total; base += 32) {
        const int j = base + lane;
        // owner: the last lane whose exclusive offset is <= j
        int lo = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const int e = __shfl_sync(full, excl, lo + step);
            if (lo + step < 32 && e <= j) lo += step;
        }
        const int o_excl = __shfl_sync(full, excl, lo);
        const int o_x0 = __shfl_sync(full, x0, lo);
        const int o_y0 = __shfl_sync(full, y0, lo);
        const int o_w = __shfl_sync(full, w, lo);
        const unsigned long long o_key = __shfl_sync(full, (unsigned long long)key, lo);
        if (j < total) {
            const int local = j - o_excl;
            const int ry = local / o_w;
            const int t = (o_y0 + ry) * tx + o_x0 + (local - ry * o_w);
            const int slot = atomicAdd(&fill[t], 1);
            keys[__ldg(raw_start + t) + slot] = o_key;
        }
    }
}

constexpr int kSortThreads = 256;

__device__ __forceinline__ void bitonic_sort(uint64_t* data, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int q = threadIdx.x; q < (n >> 1); q += kSortThreads) {
                const int lo = ((q & ~(j - 1)) << 1) | (q & (j - 1));
                const int hi = lo | j;
                const bool up = (lo & k) == 0;
                const uint64_t a = data[lo], b = data[hi];
                if ((a > b) == up) {
                    data[lo] = b;
                    data[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

__global__ void __launch_bounds__(kSortThreads)
k_tile_sort(const int32_t* __restrict__ raw_counts, const int64_t* __restrict__ raw_start,
            const uint64_t* __restrict__ keys, const int2* __restrict__ tile_bins,
            int32_t* __restrict__ gaussian_ids, int tile0, uint32_t* err) {
    __shared__ uint64_t data[kMaxTileElems];
    __shared__ int hist[256];
    __shared__ uint32_t s_prefix;
    __shared__ int s_need, s_count;
    const int t = tile0 + blockIdx.x;
    const int count = raw_counts[t];
    if (count <= 0) return;
    const uint64_t* src = keys + raw_start[t];
    const int out = tile_bins[t].x;
    int n;
    if (count <= kMaxTileElems) {
        n = 1;
        while (n < count) n <<= 1;
        for (int q = threadIdx.x; q < n; q += kSortThreads) data[q] = q < count ? src[q] : ~0ull;
        __syncthreads();
    } else {
        // Radix select on the 24-bit Gaussian id: find theta such that exactly
        // 2048 ids of this tile are <= theta.
        if (threadIdx.x == 0) {
            s_prefix = 0;
            s_need = kMaxTileElems;
            if (err) atomicOr(err, kErrTileOverflow);
        }
        for (int shift = 16; shift >= 0; shift -= 8) {
            hist[threadIdx.x] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix;
            for (int q = threadIdx.x; q < count; q += kSortThreads) {
                const uint32_t id = (uint32_t)src[q];
                if ((id >> (shift + 8)) == prefix) atomicAdd(&hist[(id >> shift) & 255], 1);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int need = s_need, cum = 0, d = 0;
                for (; d < 256; ++d) {
                    if (cum + hist[d] >= need) break;
                    cum += hist[d];
                }
                s_need = need - cum;
                s_prefix = (prefix << 8) | (uint32_t)d;
            }
            __syncthreads();
        }
        const uint32_t theta = s_prefix;
        if (threadIdx.x == 0) s_count = 0;
        __syncthreads();
        for (int q = threadIdx.x; q < count; q += kSortThreads) {
            const uint64_t key = src[q];
            if ((uint32_t)key <= theta) {
                const int slot = atomicAdd(&s_count, 1);
                if (slot < kMaxTileElems) data[slot] = key;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0 && s_count != kMaxTileElems && err) atomicOr(err, kErrCapacity);
        n = kMaxTileElems;
    }
    bitonic_sort(data, n);
    const int kept = min(count, kMaxTileElems);
    for (int q = threadIdx.x; q < kept; q += kSortThreads) gaussian_ids[out + q] = (int32_t)(uint32_t)data[q];
}

}  // namespace

void launch_tile_counts(const int32_t* tile_diff, int tiles_x, int tiles_y, int row0, int row1,
                        int32_t* raw_counts, int64_t* raw_start, int2* tile_bins, int64_t* totals,
                        int64_t* row_work, cudaStream_t s) {
    note_launches(1);
    k_tile_counts<<<1, kCountThreads, 0, s>>>(tile_diff, tiles_x, tiles_y, row0, row1, raw_counts, raw_start,
                                              tile_bins, totals, row_work);
}

void launch_emit_keys(int n, const uint2* rects, const float* depths, int tiles_x, int row0, int row1,
                      const int64_t* raw_start, int32_t* fill, uint64_t* raw_keys, cudaStream_t s) {
    if (n <= 0) return;
    note_launches(1);
    k_emit_keys<<<(n + 255) / 256, 256, 0, s>>>(n, rects, depths, tiles_x, row0, row1, raw_start, fill, raw_keys);
}

void launch_tile_sort(int tile0, int num_tiles, const int32_t* raw_counts, const int64_t* raw_start,
                      const uint64_t* raw_keys, const int2* tile_bins, int32_t* gaussian_ids, uint32_t* err,
                      cudaStream_t s) {
    if (num_tiles <= 0) return;
    note_launches(1);
    k_tile_sort<<<num_tiles, kSortThreads, 0, s>>>(raw_counts, raw_start, raw_keys, tile_bins, gaussian_ids, tile0,
                                                    err);
}

}  // namespace msplat
