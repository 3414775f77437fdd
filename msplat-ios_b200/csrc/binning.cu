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
//   1. the projection adds each Gaussian's tile rectangle into the 2-D
//      difference array of its id chunk (32 contiguous id ranges; 4 atomics
//      per Gaussian instead of one per tile);
//   2. one CTA per chunk integrates its array into per-tile counts; per tile,
//      the raw count and, for a tile over the 2048 cap, the id bound below
//      which its 2048 lowest ids lie (the end of the chunk where the
//      cumulative count reaches 2048); one CTA then clamps the emitted counts
//      to 2048 and scans both the emitted and the kept counts;
//   3. each (Gaussian, tile) pair under the tile's id bound appends the key
//      (depth_bits << 32) | id into its tile's segment (slot order is
//      irrelevant, the set is exact); Gaussians past the bounds of every
//      8x8-tile block they touch are skipped whole;
//   4. per tile, the kept keys are sorted ascending with a register-blocked
//      bitonic network (keys in registers; partners in the same warp reached
//      by shuffles, only cross-warp partners through shared memory): one warp
//      per tile up to 512 keys, one CTA above that; for an overfull tile the
//      CTA first keeps the 2048 lowest Gaussian ids among the emitted ones (a
//      radix select on the id bits). Output: the sorted Gaussian ids.
#include <climits>

#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

constexpr int kCountThreads = 1024;

// Per-tile intersection counts of one id chunk (blockIdx.x) from its 2-D
// difference array: column prefix over y (one thread per tile column), then
// row prefix over x (one warp per tile row, 32 columns at a time with a
// shuffle scan).
__global__ void __launch_bounds__(kCountThreads)
k_chunk_counts(const int32_t* __restrict__ diff, int tx, int ty, int32_t* __restrict__ chunk_counts) {
    const int dw = tx + 1;
    const int32_t* d = diff + (size_t)blockIdx.x * dw * (ty + 1);
    int32_t* out = chunk_counts + (size_t)blockIdx.x * tx * ty;
    for (int x = threadIdx.x; x < tx; x += blockDim.x) {
        int run = 0;
        for (int y = 0; y < ty; ++y) {
            run += d[y * dw + x];
            out[y * tx + x] = run;
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int y = warp; y < ty; y += nwarps) {
        int32_t* row = out + (size_t)y * tx;
        int carry = 0;
        for (int x0 = 0; x0 < tx; x0 += 32) {
            const int x = x0 + lane;
            int v = x < tx ? row[x] : 0;
#pragma unroll
            for (int dd = 1; dd < 32; dd <<= 1) {
                const int o = __shfl_up_sync(0xffffffffu, v, dd);
                if (lane >= dd) v += o;
            }
            const int run = carry + v;
            if (x < tx) row[x] = run;
            carry = __shfl_sync(0xffffffffu, run, 31);
        }
    }
}

// Per tile: the raw count (sum over the id chunks) and, for a tile over the
// 2048 cap, the first chunk k at which the cumulative count reaches 2048.
// The 2048 lowest ids of the tile (the ones it keeps) all lie in chunks
// 0..k, so only those chunks' intersections are emitted: emit_count[t] is
// their number and id_limit[t] = (k + 1) * id_chunk the exclusive id bound
// (INT_MAX for tiles within the cap, which emit everything). block_max
// (zeroed by the caller) receives the largest id_limit of each
// kLimitBlock x kLimitBlock block of tiles.
__global__ void __launch_bounds__(256)
k_tile_select(const int32_t* __restrict__ chunk_counts, int num_tiles, int tx, int num_chunks, int id_chunk,
              int32_t* __restrict__ raw_true, int32_t* __restrict__ emit_count, int32_t* __restrict__ id_limit,
              int32_t* __restrict__ block_max, uint32_t* err) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= num_tiles) return;
    const int bxn = (tx + kLimitBlock - 1) / kLimitBlock;
    int32_t* bmax = block_max + ((t / tx) / kLimitBlock) * bxn + (t % tx) / kLimitBlock;
    int64_t cum = 0;
    int cut = -1, emitted = 0;
    for (int c = 0; c < num_chunks; ++c) {
        cum += chunk_counts[(size_t)c * num_tiles + t];
        if (cut < 0 && cum >= kMaxTileElems) {
            cut = c;
            emitted = (int)cum;
        }
    }
    const int raw = (int)min(cum, (int64_t)INT_MAX);
    raw_true[t] = raw;
    int limit = INT_MAX;
    if (raw > kMaxTileElems) {
        emit_count[t] = emitted;
        limit = (int)min((int64_t)(cut + 1) * id_chunk, (int64_t)INT_MAX);
        if (err) atomicOr(err, kErrTileOverflow);
    } else {
        emit_count[t] = raw;
    }
    id_limit[t] = limit;
    atomicMax(bmax, limit);
}

constexpr int kWarpSortMax = 512;  // tiles up to this many keys are sorted by one warp

// From the per-tile emitted counts (k_tile_select): the row work, clamped
// kept counts and both exclusive scans, for tile rows [row0, row1) (other
// rows get zero counts). With world > 0 the rows are chosen here: band `rank`
// of `world` work-balanced bands [o0, o1) plus a one-row halo; the band goes
// to totals[2..3] next to the emitted and kept totals (totals[0..1]).
__global__ void __launch_bounds__(kCountThreads)
k_tile_counts(int tx, int ty, int row0, int row1, int32_t* __restrict__ raw_counts,
              int64_t* __restrict__ raw_start, unsigned long long* __restrict__ fill, int2* __restrict__ tile_bins,
              int64_t* __restrict__ totals, int64_t* __restrict__ row_work, int world, int rank,
              int32_t* __restrict__ big_tiles) {
    __shared__ int s_rows[2];
    __shared__ int s_big;
    // The work of each row (one warp per tile row).
    if (row_work) {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
        for (int y = warp; y < ty; y += nwarps) {
            const int32_t* row = raw_counts + (size_t)y * tx;
            int64_t work = 0;
            for (int x = lane; x < tx; x += 32) work += min(row[x], kMaxTileElems) + kRowWorkPerTile;
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) work += __shfl_xor_sync(0xffffffffu, work, d);
            if (lane == 0) row_work[y] = work;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int r0 = row0, r1 = row1;
        if (world > 0 && row_work) {
            double total = 0;
            for (int y = 0; y < ty; ++y) total += (double)row_work[y];
            const int o0 = band_cut(row_work, ty, total, rank, world);
            const int o1 = band_cut(row_work, ty, total, rank + 1, world);
            totals[2] = o0;
            totals[3] = o1;
            r0 = o1 > o0 ? max(0, o0 - 1) : 0;
            r1 = o1 > o0 ? min(ty, o1 + 1) : 0;
        }
        s_rows[0] = r0;
        s_rows[1] = r1;
        s_big = 0;
    }
    __syncthreads();
    // Rows outside [row0, row1) get zero counts so that nothing is emitted there.
    {
        const int r0 = s_rows[0], r1 = s_rows[1];
        for (int q = threadIdx.x; q < tx * ty; q += blockDim.x) {
            const int y = q / tx;
            if (y < r0 || y >= r1) raw_counts[q] = 0;
        }
    }
    __syncthreads();
    // Exclusive scans of raw (int64) and kept = min(raw, 2048) (int32): each
    // warp scans a contiguous segment of tiles 32 at a time (coalesced), then
    // the warps' segment totals are scanned and added.
    const int T = tx * ty;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int seg = ((T + nwarps - 1) / nwarps + 31) & ~31;
    const int b = min(warp * seg, T), e = min(b + seg, T);
    __shared__ int64_t s_raw[kCountThreads / 32];
    __shared__ int32_t s_kept[kCountThreads / 32];
    int64_t wraw = 0;
    int32_t wkept = 0;
    for (int t0 = b; t0 < e; t0 += 32) {
        const int t = t0 + lane;
        const int r = t < e ? raw_counts[t] : 0;
        int64_t vr = r;
        int32_t vk = min(r, kMaxTileElems);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            vr += __shfl_xor_sync(0xffffffffu, vr, d);
            vk += __shfl_xor_sync(0xffffffffu, vk, d);
        }
        wraw += vr;
        wkept += vk;
    }
    if (lane == 0) {
        s_raw[warp] = wraw;
        s_kept[warp] = wkept;
    }
    __syncthreads();
    int64_t run_raw = 0;
    int32_t run_kept = 0;
    for (int w = 0; w < warp; ++w) {
        run_raw += s_raw[w];
        run_kept += s_kept[w];
    }
    for (int t0 = b; t0 < e; t0 += 32) {
        const int t = t0 + lane;
        const int r = t < e ? raw_counts[t] : 0;
        const int k = min(r, kMaxTileElems);
        int64_t ir = r;
        int32_t ik = k;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int64_t orr = __shfl_up_sync(0xffffffffu, ir, d);
            const int32_t ok = __shfl_up_sync(0xffffffffu, ik, d);
            if (lane >= d) {
                ir += orr;
                ik += ok;
            }
        }
        if (t < e) {
            raw_start[t] = run_raw + ir - r;
            fill[t] = (unsigned long long)(run_raw + ir - r);
            tile_bins[t] = make_int2(run_kept + ik - k, run_kept + ik);
        }
        // tiles the CTA sort handles (more than kWarpSortMax keys), listed in
        // any order so that its grid covers just them
        const bool big = t < e && r > kWarpSortMax;
        const unsigned bb = __ballot_sync(0xffffffffu, big);
        if (bb) {
            int at = 0;
            if (lane == 0) at = atomicAdd(&s_big, __popc(bb));
            at = __shfl_sync(0xffffffffu, at, 0);
            if (big) big_tiles[at + __popc(bb & ((1u << lane) - 1u))] = t;
        }
        run_raw += __shfl_sync(0xffffffffu, ir, 31);
        run_kept += __shfl_sync(0xffffffffu, ik, 31);
    }
    if (threadIdx.x == blockDim.x - 1) {
        int64_t tr = 0;
        int32_t tk = 0;
        for (int w = 0; w < nwarps; ++w) {
            tr += s_raw[w];
            tk += s_kept[w];
        }
        totals[0] = tr;
        totals[1] = tk;
    }
    __syncthreads();
    if (threadIdx.x == 0) totals[4] = s_big;
}

// One warp per 32 consecutive Gaussians: their clipped tile rectangles are
// flattened into (Gaussian, tile) pairs by a warp prefix sum of the areas, and
// every lane takes four pairs per round (owners found by a binary search over
// the lanes' exclusive offsets), so a warp keeps 128 independent slot atomics
// in flight whatever the rectangle sizes.
__global__ void __launch_bounds__(256)
k_emit_keys(int n, const uint2* __restrict__ rects, const float* __restrict__ depths, int tx, int row0, int row1,
            const int32_t* __restrict__ id_limit, const int32_t* __restrict__ block_max,
            unsigned long long* __restrict__ fill, uint64_t* __restrict__ keys) {
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
        // a Gaussian at or past the id bound of every tile block it touches
        // emits nothing (those tiles keep lower ids only)
        if (area > 0) {
            const int bxn = (tx + kLimitBlock - 1) / kLimitBlock;
            bool any = false;
            for (int by = y0 / kLimitBlock; by <= (y1 - 1) / kLimitBlock && !any; ++by)
                for (int bx = x0 / kLimitBlock; bx <= (x1 - 1) / kLimitBlock; ++bx)
                    if (__ldg(block_max + by * bxn + bx) > i) {
                        any = true;
                        break;
                    }
            if (!any) area = 0;
        }
    }
    int incl = area;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(full, incl, d);
        if (lane >= d) incl += v;
    }
    const int total = __shfl_sync(full, incl, 31);
    const int excl = incl - area;
    // kPairsPerLane pairs per lane and round: their slot atomics are issued
    // back to back, so each lane keeps several round trips in flight
    constexpr int kPairsPerLane = 4;
    for (int base = 0; base < total; base += 32 * kPairsPerLane) {
        int tile[kPairsPerLane];
        unsigned long long okey[kPairsPerLane];
#pragma unroll
        for (int q = 0; q < kPairsPerLane; ++q) {
            const int j = base + q * 32 + lane;
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
            okey[q] = __shfl_sync(full, (unsigned long long)key, lo);
            tile[q] = -1;
            if (j < total) {
                const int local = j - o_excl;
                const int ry = local / o_w;
                tile[q] = (o_y0 + ry) * tx + o_x0 + (local - ry * o_w);
                // past the tile's id limit: not among its 2048 lowest ids
                if ((int)(uint32_t)okey[q] >= __ldg(id_limit + tile[q])) tile[q] = -1;
            }
        }
        // fill[t] starts at the tile's first key position (k_tile_counts),
        // so the atomic returns the key's position directly
        unsigned long long pos[kPairsPerLane];
#pragma unroll
        for (int q = 0; q < kPairsPerLane; ++q)
            if (tile[q] >= 0) pos[q] = atomicAdd(&fill[tile[q]], 1ull);
#pragma unroll
        for (int q = 0; q < kPairsPerLane; ++q)
            if (tile[q] >= 0) keys[pos[q]] = okey[q];
    }
}

constexpr int kSortThreads = 256;

// Compare-exchange for an ascending (up) or descending block.
__device__ __forceinline__ void cmp_swap(uint64_t& a, uint64_t& b, bool up) {
    const bool sw = (a > b) == up;
    const uint64_t lo = sw ? b : a, hi = sw ? a : b;
    a = lo;
    b = hi;
}

// v = min(v, o) when keep_min, else max(v, o).
__device__ __forceinline__ uint64_t keep_of(uint64_t v, uint64_t o, bool keep_min) {
    return ((v < o) == keep_min) ? v : o;
}

// Bitonic sort of G * E 64-bit keys held "blocked": thread t of the group
// holds elements [E t, E t + E) in v.
//  - block sizes k <= E stay inside the thread: a compile-time network;
//  - for k > E the direction (element & k) is the same for all of a thread's
//    elements; stages with partner distance j < E are register
//    compare-exchanges, j < 32 E shuffles within the warp, and larger j go
//    through shared memory (xchg, G * E keys, element (t, r) stored at
//    r * G + t so that a warp's accesses hit distinct banks).
template <int E, int G>
__device__ __forceinline__ void bitonic_blocked(uint64_t (&v)[E], int t, uint64_t* xchg) {
    const int lane = t & 31;
    const int base = t * E;
#pragma unroll
    for (int k = 2; k <= E; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int r = 0; r < E; ++r) {
                const int p = r ^ j;
                if (p > r) cmp_swap(v[r], v[p], (((base + r) & k) == 0));
            }
        }
    }
    for (int k = 2 * E; k <= G * E; k <<= 1) {
        const bool up = (base & k) == 0;
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j < E) {
#pragma unroll
                for (int jj = 1; jj < E; jj <<= 1) {
                    if (jj == j) {
#pragma unroll
                        for (int r = 0; r < E; ++r) {
                            const int p = r ^ jj;
                            if (p > r) cmp_swap(v[r], v[p], up);
                        }
                    }
                }
            } else if (G == 32 || j < 32 * E) {
                const int lm = j / E;
                const bool keep_min = ((lane & lm) == 0) == up;
#pragma unroll
                for (int r = 0; r < E; ++r) v[r] = keep_of(v[r], __shfl_xor_sync(0xffffffffu, v[r], lm), keep_min);
            } else if constexpr (G > 32) {
                const int pt = t ^ (j / E);
                const bool keep_min = ((base & j) == 0) == up;
                __syncthreads();
#pragma unroll
                for (int r = 0; r < E; ++r) xchg[r * G + t] = v[r];
                __syncthreads();
#pragma unroll
                for (int r = 0; r < E; ++r) v[r] = keep_of(v[r], xchg[r * G + pt], keep_min);
            }
        }
    }
}

template <int E, int G>
__device__ __forceinline__ void sort_and_store(const uint64_t* src, int count, int t, uint64_t* xchg, int32_t* dst,
                                               int kept) {
    uint64_t v[E];
#pragma unroll
    for (int r = 0; r < E; ++r) {
        const int e = t * E + r;
        v[r] = e < count ? src[e] : ~0ull;
    }
    bitonic_blocked<E, G>(v, t, xchg);
#pragma unroll
    for (int r = 0; r < E; ++r) {
        const int e = t * E + r;
        if (e < kept) dst[e] = (int32_t)(uint32_t)v[r];
    }
}

// Tiles with at most kWarpSortMax keys: one warp per tile, no barriers.
__global__ void __launch_bounds__(kSortThreads)
k_tile_sort_warp(const int32_t* __restrict__ raw_counts, const int64_t* __restrict__ raw_start,
                 const uint64_t* __restrict__ keys, const int2* __restrict__ tile_bins,
                 int32_t* __restrict__ gaussian_ids, int tile0, int num_tiles) {
    const int w = blockIdx.x * (kSortThreads / 32) + (threadIdx.x >> 5);
    if (w >= num_tiles) return;
    const int t = tile0 + w;
    const int count = raw_counts[t];
    if (count <= 0 || count > kWarpSortMax) return;
    const uint64_t* src = keys + raw_start[t];
    int32_t* dst = gaussian_ids + tile_bins[t].x;
    const int lane = threadIdx.x & 31;
    if (count <= 128)
        sort_and_store<4, 32>(src, count, lane, nullptr, dst, count);
    else if (count <= 256)
        sort_and_store<8, 32>(src, count, lane, nullptr, dst, count);
    else
        sort_and_store<16, 32>(src, count, lane, nullptr, dst, count);
}

constexpr int kSelectBins = 4096;

// Exclusive scan of one int per thread over the CTA.
__device__ __forceinline__ int cta_exclusive_scan(int v) {
    __shared__ int warp_sum[kSortThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += o;
    }
    if (lane == 31) warp_sum[warp] = inc;
    __syncthreads();
    int base = 0;
#pragma unroll
    for (int w = 0; w < kSortThreads / 32; ++w) base += (w < warp) ? warp_sum[w] : 0;
    __syncthreads();
    return base + inc - v;
}

// Smallest digit d of the histogram with sum(hist[0..d]) >= need; writes d
// and need - sum(hist[0..d-1]). Requires sum(hist) >= need.
__device__ __forceinline__ void find_digit(const int* hist, int need, int* s_digit, int* s_need) {
    constexpr int per = kSelectBins / kSortThreads;
    int local[per];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < per; ++i) {
        local[i] = hist[threadIdx.x * per + i];
        sum += local[i];
    }
    const int ex = cta_exclusive_scan(sum);
    if (ex < need && ex + sum >= need) {
        int cum = ex;
#pragma unroll
        for (int i = 0; i < per; ++i) {
            if (cum + local[i] >= need) {
                *s_digit = threadIdx.x * per + i;
                *s_need = need - cum;
                break;
            }
            cum += local[i];
        }
    }
    __syncthreads();
}

// Tiles with more than kWarpSortMax keys: one CTA per tile; for overfull
// tiles first the radix select of the 2048 lowest ids.
__global__ void __launch_bounds__(kSortThreads)
k_tile_sort(const int32_t* __restrict__ raw_counts, const int64_t* __restrict__ raw_start,
            const uint64_t* __restrict__ keys, const int2* __restrict__ tile_bins,
            int32_t* __restrict__ gaussian_ids, const int32_t* __restrict__ big_tiles, uint32_t* err, int num_ids) {
    __shared__ uint64_t data[kMaxTileElems];
    __shared__ int hist[kSelectBins];
    __shared__ uint32_t s_prefix;
    __shared__ int s_digit, s_need, s_count;
    const int t = big_tiles[blockIdx.x];
    const int count = raw_counts[t];
    if (count <= kWarpSortMax) return;
    const uint64_t* src = keys + raw_start[t];
    int32_t* dst = gaussian_ids + tile_bins[t].x;
    if (count <= kMaxTileElems) {
        if (count <= 4 * kSortThreads)
            sort_and_store<4, kSortThreads>(src, count, threadIdx.x, data, dst, count);
        else
            sort_and_store<8, kSortThreads>(src, count, threadIdx.x, data, dst, count);
        return;
    }
    // Radix select on the Gaussian id, most significant digit first: bits
    // 24..31 (only when there are more than 2^24 Gaussians), 12..23, 0..11.
    // Each pass histograms the ids that share the digits chosen so far and
    // picks the digit below which fewer than `need` ids remain; the result
    // theta is the id such that exactly 2048 ids of this tile are <= theta.
    if (threadIdx.x == 0 && err) atomicOr(err, kErrTileOverflow);
    uint32_t prefix = 0;  // digits chosen so far
    int need = kMaxTileElems;
    for (int level = num_ids > (1 << 24) ? 0 : 1; level < 3; ++level) {
        const int shift = level == 0 ? 24 : (level == 1 ? 12 : 0);
        const uint32_t mask = level == 0 ? 255u : 4095u;
        const int above = shift + (level == 0 ? 8 : 12);  // bits above this digit: fixed by prefix
        for (int q = threadIdx.x; q < kSelectBins; q += kSortThreads) hist[q] = 0;
        __syncthreads();
        for (int q = threadIdx.x; q < count; q += kSortThreads) {
            const uint32_t id = (uint32_t)src[q];
            if (((uint64_t)id >> above) == prefix) atomicAdd(&hist[(id >> shift) & mask], 1);
        }
        __syncthreads();
        find_digit(hist, need, &s_digit, &s_need);
        prefix = (prefix << (level == 0 ? 8 : 12)) | (uint32_t)s_digit;
        need = s_need;
        __syncthreads();
    }
    if (threadIdx.x == 0) s_prefix = prefix;
    __syncthreads();
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
    const int got = s_count;
    if (threadIdx.x == 0 && got != kMaxTileElems && err) atomicOr(err, kErrCapacity);
    // the selected keys sit in data[] in arbitrary order: any assignment to
    // threads will do, so read them bank-conflict free
    uint64_t v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const int e = r * kSortThreads + threadIdx.x;
        v[r] = e < got && e < kMaxTileElems ? data[e] : ~0ull;
    }
    bitonic_blocked<8, kSortThreads>(v, threadIdx.x, data);
#pragma unroll
    for (int r = 0; r < 8; ++r) dst[threadIdx.x * 8 + r] = (int32_t)(uint32_t)v[r];
}

}  // namespace

void launch_tile_counts(const int32_t* tile_diff, int id_chunk, int32_t* chunk_counts, int32_t* raw_true,
                        int32_t* id_limit, int32_t* block_max, int tiles_x, int tiles_y, int row0, int row1,
                        int32_t* raw_counts, int64_t* raw_start, uint64_t* fill, int2* tile_bins, int64_t* totals,
                        int64_t* row_work, uint32_t* err, cudaStream_t s, int world, int rank, int32_t* big_tiles) {
    const int T = tiles_x * tiles_y;
    note_launches(3);
    k_chunk_counts<<<kIdChunks, kCountThreads, 0, s>>>(tile_diff, tiles_x, tiles_y, chunk_counts);
    k_tile_select<<<(T + 255) / 256, 256, 0, s>>>(chunk_counts, T, tiles_x, kIdChunks, id_chunk, raw_true,
                                                  raw_counts, id_limit, block_max, err);
    k_tile_counts<<<1, kCountThreads, 0, s>>>(tiles_x, tiles_y, row0, row1, raw_counts, raw_start,
                                              reinterpret_cast<unsigned long long*>(fill), tile_bins, totals,
                                              row_work, world, rank, big_tiles);
}

void launch_emit_keys(int n, const uint2* rects, const float* depths, int tiles_x, int row0, int row1,
                      const int32_t* id_limit, const int32_t* block_max, uint64_t* fill, uint64_t* raw_keys,
                      cudaStream_t s) {
    if (n <= 0) return;
    note_launches(1);
    k_emit_keys<<<(n + 255) / 256, 256, 0, s>>>(n, rects, depths, tiles_x, row0, row1, id_limit, block_max,
                                                reinterpret_cast<unsigned long long*>(fill), raw_keys);
}

void launch_tile_sort(int tile0, int num_tiles, const int32_t* raw_counts, const int64_t* raw_start,
                      const uint64_t* raw_keys, const int2* tile_bins, int32_t* gaussian_ids, uint32_t* err,
                      int num_gaussians, const int32_t* big_tiles, int num_big, cudaStream_t s) {
    if (num_tiles <= 0) return;
    note_launches(num_big > 0 ? 2 : 1);
    const int warps = kSortThreads / 32;
    k_tile_sort_warp<<<(num_tiles + warps - 1) / warps, kSortThreads, 0, s>>>(raw_counts, raw_start, raw_keys,
                                                                              tile_bins, gaussian_ids, tile0,
                                                                              num_tiles);
    if (num_big > 0)
        k_tile_sort<<<num_big, kSortThreads, 0, s>>>(raw_counts, raw_start, raw_keys, tile_bins, gaussian_ids,
                                                      big_tiles, err, num_gaussians);
}

}  // namespace msplat
