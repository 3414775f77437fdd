// route.cu — multi-GPU exchange that routes projected surfels to the ranks
// whose image band they touch.
//
// Every rank owns a contiguous slice of Gaussians (its parameters and Adam
// state) and an image band of tile rows. A step:
//   1. the owner projects its own slice (geometry and SH colour; the
//      projection of msplat_render, so records are bit-identical) and writes
//      the slice's summary: per-tile intersection counts (from a 2-D
//      difference array) and two histograms of its tile rectangles' first and
//      last rows;
//   2. the summaries of all ranks are gathered (the caller's all-gather) and
//      every rank computes the same work-balanced bands (the least maximum
//      band cost over the summed counts, halo rows included) and, from the
//      histograms, how many Gaussians every rank sends to every rank, so the
//      all-to-all needs no count exchange;
//   3. each projected Gaussian goes, as a 128-byte payload (raster record,
//      cull record, tile rectangle, depth, global id), to every rank whose
//      band plus its one-tile-row halo its rectangle meets, in increasing id
//      order per destination: packed for the caller's all-to-all, or stored
//      by the pack kernel straight into the destination GPU's inbox (CUDA
//      IPC mapping, NVLink stores);
//   4. a rank bins, sorts and rasterises its band over what it received;
//      the received Gaussians are in increasing global id order (sources in
//      rank order, each in id order), so sorting by (depth, local index)
//      gives the single-GPU order and the overfull-tile policy keeps the
//      same 2048 ids;
//   5. the band's per-Gaussian raster-gradient records go back to their
//      owners (the reverse all-to-all, or peer stores into the owner's
//      return box), which add them up, run the projection VJP and Adam on
//      their slice. Parameters are never gathered.
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

constexpr int kRouteThreads = 256;

// Tile rectangle (x0, y0, x1, y1) of a packed rect.
__device__ __forceinline__ int4 unpack_rect(uint2 r) {
    return make_int4((int)(r.x & 0xffffu), (int)(r.x >> 16), (int)(r.y & 0xffffu), (int)(r.y >> 16));
}

// Per-tile counts of the slice from the 2-D difference array the projection
// filled ([(ty+1) x (tx+1)], one id chunk): counts[y][x] is the sum of
// diff[0..y][0..x]. Rows first (one warp per row, a shuffle scan over
// 32-column chunks with a carry), then columns (32 x 32 threads per block of
// 32 columns: each thread sums a segment of rows, the segment sums are
// scanned in shared memory, then each thread rewrites its segment).
__global__ void __launch_bounds__(256) k_route_prefix_rows(const int32_t* __restrict__ diff, int tx, int ty,
                                                           int32_t* __restrict__ rowsum) {
    const int lane = threadIdx.x & 31;
    const int y = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (y >= ty) return;
    const int dw = tx + 1;
    int carry = 0;
    for (int x0 = 0; x0 < tx; x0 += 32) {
        const int x = x0 + lane;
        int v = x < tx ? diff[(size_t)y * dw + x] : 0;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, d);
            if (lane >= d) v += u;
        }
        if (x < tx) rowsum[(size_t)y * tx + x] = carry + v;
        carry += __shfl_sync(0xffffffffu, v, 31);
    }
}
__global__ void __launch_bounds__(1024) k_route_prefix_cols(const int32_t* __restrict__ rowsum, int tx, int ty,
                                                            int32_t* __restrict__ counts) {
    __shared__ int seg_sum[32][33];
    const int lx = threadIdx.x, seg = threadIdx.y;
    const int x = blockIdx.x * 32 + lx;
    const int per = (ty + 31) / 32;
    const int ya = min(ty, seg * per), yb = min(ty, ya + per);
    int run = 0;
    if (x < tx)
        for (int y = ya; y < yb; ++y) run += rowsum[(size_t)y * tx + x];
    seg_sum[seg][lx] = run;
    __syncthreads();
    if (x >= tx) return;
    int off = 0;
    for (int k = 0; k < seg; ++k) off += seg_sum[k][lx];
    for (int y = ya; y < yb; ++y) {
        off += rowsum[(size_t)y * tx + x];
        counts[(size_t)y * tx + x] = off;
    }
}

// Whether a projected Gaussian takes part in the exchange (the rule of
// k_route_dest and of the rect-row histograms).
__device__ __forceinline__ bool routable(int32_t radius, int4 r) { return radius > 0 && r.z > r.x && r.w > r.y; }

// Rect-row histograms of the slice: starts[y] (+=) counts the routable
// Gaussians whose tile rectangle starts at row y, ends[y] those whose
// rectangle ends at row y (exclusive bound), y in [0, ty]; per-block
// histograms in shared memory (2 (ty + 1) ints), flushed with atomics.
__global__ void __launch_bounds__(kRouteThreads) k_route_hist(int n, const uint2* __restrict__ rects,
                                                              const int32_t* __restrict__ radii, int ty,
                                                              int32_t* __restrict__ starts,
                                                              int32_t* __restrict__ ends) {
    extern __shared__ int shist[];
    const int rows = ty + 1;
    for (int k = threadIdx.x; k < 2 * rows; k += blockDim.x) shist[k] = 0;
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const int4 r = unpack_rect(rects[i]);
        if (routable(radii[i], r)) {
            atomicAdd(&shist[r.y], 1);
            atomicAdd(&shist[rows + r.w], 1);
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < rows; k += blockDim.x) {
        if (shist[k]) atomicAdd(&starts[k], shist[k]);
        if (shist[rows + k]) atomicAdd(&ends[k], shist[rows + k]);
    }
}

// Row work of the summed per-tile counts of all ranks (the row work of
// k_tile_counts: kept = min(raw, 2048) plus the per-tile cost), one warp per
// row, the sum over ranks per tile.
__global__ void __launch_bounds__(256) k_route_row_work(const int32_t* __restrict__ summaries, int64_t len, int tx,
                                                        int ty, int world, int64_t* __restrict__ row_work) {
    const int lane = threadIdx.x & 31;
    const int y = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (y >= ty) return;
    int64_t work = 0;
    for (int x = lane; x < tx; x += 32) {
        int c = 0;
        for (int r = 0; r < world; ++r) c += summaries[(size_t)r * len + (size_t)y * tx + x];
        work += min(c, kMaxTileElems) + kRowWorkPerTile;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) work += __shfl_xor_sync(0xffffffffu, work, d);
    if (lane == 0) row_work[y] = work;
}

// Band cost in tenths of a row-work unit: the band's rows, plus 0.4 of each
// halo row it renders but does not own (forward and binning, about 0.4 of a
// row's step work). Integer arithmetic, so every rank (and a CPU restatement)
// computes identical cuts. P10[y] = 10 x the row work of rows [0, y);
// H[y] = 4 x the row work of row y.
constexpr int64_t kRowTenths = 10, kHaloTenths = 4;

// Greedy cover of rows [0, ty) by at most `world` bands of cost <= L, each
// band as long as possible: the largest end b1 whose rows alone fit (binary
// search over the increasing P10), then back while the halo rows push the
// cost over L. cuts[1..] receive the band ends (when given). Returns whether
// the rows are covered.
__device__ bool greedy_bands(const int64_t* P10, const int64_t* H, int ty, int world, int64_t L, int* cuts) {
    int b0 = 0;
    for (int r = 0; r < world; ++r) {
        if (b0 < ty) {
            int lo = b0, hi = ty;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (P10[mid] - P10[b0] <= L) lo = mid;
                else hi = mid - 1;
            }
            const int64_t left = b0 > 0 ? H[b0 - 1] : 0;
            int b1 = lo;
            while (b1 > b0 && P10[b1] - P10[b0] + left + (b1 < ty ? H[b1] : 0) > L) --b1;
            if (b1 == b0) return false;
            b0 = b1;
        }
        if (cuts) cuts[r + 1] = b0;
    }
    return b0 == ty;
}

// Bands of every rank: the least L (to within one unit) for which the greedy
// cover succeeds, found by kCutThreads-way search rounds (thread k tests
// lo + (hi - lo) (k + 1) / kCutThreads), then the greedy cover at that L.
// Then the items from rank r to rank q: r's routable Gaussians whose
// rectangle rows [y0, y1) meet q's band with its one-row halo [lo, hi),
// i.e. all of them but those with y0 >= hi and those with y1 <= lo (disjoint
// when y0 < y1 and lo < hi); 0 for an empty band.
constexpr int kCutThreads = 256;
__global__ void __launch_bounds__(kCutThreads) k_route_cuts(const int32_t* __restrict__ summaries, int64_t len,
                                                            int tx, int ty, int world,
                                                            const int64_t* __restrict__ row_work,
                                                            int32_t* __restrict__ bands, int64_t* __restrict__ matrix) {
    extern __shared__ int64_t sdyn[];
    int64_t* H = sdyn;            // [ty]
    int64_t* P10 = sdyn + ty;     // [ty + 1]
    __shared__ int sb[kMaxPeerRanks + 1];
    __shared__ int64_t s_lo, s_hi;
    __shared__ int s_kmin;
    for (int y = threadIdx.x; y < ty; y += blockDim.x) H[y] = kHaloTenths * row_work[y];
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t run = 0, wmax = 0;
        P10[0] = 0;
        for (int y = 0; y < ty; ++y) {
            const int64_t wy = H[y] / kHaloTenths;
            run += wy;
            P10[y + 1] = kRowTenths * run;
            wmax = max(wmax, wy);
        }
        s_lo = 0;
        s_hi = kRowTenths * run + 2 * kHaloTenths * wmax;  // one band over every row fits
    }
    __syncthreads();
    for (int round = 0; round < 12; ++round) {
        const int64_t lo = s_lo, hi = s_hi;
        if (hi - lo <= 1) break;
        if (threadIdx.x == 0) s_kmin = kCutThreads - 1;
        __syncthreads();
        const int64_t L = lo + ((hi - lo) * (threadIdx.x + 1)) / kCutThreads;
        if (greedy_bands(P10, H, ty, world, L, nullptr)) atomicMin(&s_kmin, (int)threadIdx.x);
        __syncthreads();
        if (threadIdx.x == 0) {
            const int k = s_kmin;
            s_hi = lo + ((hi - lo) * (k + 1)) / kCutThreads;
            s_lo = k > 0 ? lo + ((hi - lo) * k) / kCutThreads : lo;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        sb[0] = 0;
        if (!greedy_bands(P10, H, ty, world, s_hi, sb))
            for (int r = 1; r <= world; ++r) sb[r] = ty;  // not reached: s_hi stays feasible
        sb[world] = ty;
    }
    __syncthreads();
    if (threadIdx.x <= world) bands[threadIdx.x] = sb[threadIdx.x];
    for (int k = threadIdx.x; k < world * world; k += blockDim.x) {
        const int r = k / world, q = k % world;
        const int b0 = sb[q], b1 = sb[q + 1];
        int64_t items = 0;
        if (b1 > b0) {
            const int lo = max(0, b0 - 1), hi = min(ty, b1 + 1);
            const int32_t* starts = summaries + (size_t)r * len + (size_t)tx * ty;
            const int32_t* ends = starts + (ty + 1);
            int64_t all = 0, late = 0, early = 0;
            for (int y = 0; y <= ty; ++y) {
                const int64_t st = starts[y];
                all += st;
                if (y >= hi) late += st;
                if (y <= lo) early += ends[y];
            }
            items = all - late - early;
        }
        matrix[k] = items;
    }
}

// Destinations of each projected Gaussian of the slice: the ranks whose band
// with a one-tile-row halo ([b_r - 1, b_{r+1} + 1)) meets its rectangle's
// rows, a contiguous range [first, last] since bands are ordered (first =
// -1: none). Per block of kRouteThreads Gaussians, the number going to each
// rank (block_counts[block][rank]).
__global__ void __launch_bounds__(kRouteThreads) k_route_dest(int n, const uint2* __restrict__ rects,
                                                              const int32_t* __restrict__ radii,
                                                              const int32_t* __restrict__ bands, int world, int ty,
                                                              int2* __restrict__ dest,
                                                              int32_t* __restrict__ block_counts) {
    __shared__ int scount[kMaxPeerRanks];
    if (threadIdx.x < kMaxPeerRanks) scount[threadIdx.x] = 0;
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    int2 d = make_int2(-1, -2);
    if (i < n) {
        const int4 r = unpack_rect(rects[i]);
        if (routable(radii[i], r)) {
            for (int q = 0; q < world; ++q) {
                const int b0 = bands[q], b1 = bands[q + 1];
                if (b1 <= b0) continue;  // empty band: renders nothing
                const int lo = max(0, b0 - 1), hi = min(ty, b1 + 1);
                if (r.y < hi && r.w > lo) {
                    if (d.x < 0) d.x = q;
                    d.y = q;
                }
            }
        }
    }
    if (i < n) dest[i] = d;
    for (int q = d.x; q >= 0 && q <= d.y; ++q) atomicAdd(&scount[q], 1);
    __syncthreads();
    if (threadIdx.x < world) block_counts[(size_t)blockIdx.x * world + threadIdx.x] = scount[threadIdx.x];
}

// Exclusive scan of block_counts over blocks for every rank (one block of
// kScanThreads threads; per rank, each thread sums a contiguous segment of
// blocks, the segment sums are scanned across the block, then each thread
// rewrites its segment), the items per rank (total) and the first item of
// each rank in the packed buffer (base, exclusive scan of total).
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads) k_route_scan(int32_t* __restrict__ block_counts, int nblocks,
                                                             int world, int64_t* __restrict__ total,
                                                             int64_t* __restrict__ base) {
    __shared__ int64_t warp_sum[kScanThreads / 32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int per = (nblocks + kScanThreads - 1) / kScanThreads;
    const int ba = min(nblocks, t * per), bb = min(nblocks, ba + per);
    for (int q = 0; q < world; ++q) {
        int64_t mine = 0;
        for (int b = ba; b < bb; ++b) mine += block_counts[(size_t)b * world + q];
        // inclusive scan of the per-thread sums: warps, then the warp totals
        int64_t v = mine;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int64_t u = __shfl_up_sync(0xffffffffu, v, d);
            if (lane >= d) v += u;
        }
        if (lane == 31) warp_sum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int64_t w = warp_sum[lane];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int64_t u = __shfl_up_sync(0xffffffffu, w, d);
                if (lane >= d) w += u;
            }
            warp_sum[lane] = w;  // inclusive over warps
        }
        __syncthreads();
        int64_t run = v - mine + (warp > 0 ? warp_sum[warp - 1] : 0);
        for (int b = ba; b < bb; ++b) {
            const int c = block_counts[(size_t)b * world + q];
            block_counts[(size_t)b * world + q] = (int32_t)run;
            run += c;
        }
        if (t == kScanThreads - 1) total[q] = warp_sum[kScanThreads / 32 - 1];
        __syncthreads();  // warp_sum is rewritten for the next rank
    }
    if (t == 0) {
        int64_t run = 0;
        for (int r = 0; r < world; ++r) {
            base[r] = run;
            run += total[r];
        }
    }
}

// Payload of one routed Gaussian: raster record (5 float4), cull record
// (2 float4), then (rect.x, rect.y, depth bits, global id).
static_assert(kRoutePayloadF4 == kRecordF4 + kCullF4 + 1 && kRoutePayloadF4 * 16 == 128, "128-byte payload");

// Packs every projected Gaussian of the slice for each of its destinations:
// destination q's items go to d.dst[q] (this rank's send buffer at the
// group's offset, or the destination's inbox on its own GPU at this source's
// offset, written over NVLink) in increasing id order (block offsets from
// k_route_scan, ranks inside the block from ballots); src[d.send_base[q] + k]
// = local index of group q's item k. With `fence`, each thread's stores are
// made visible system-wide before the kernel ends (peer destinations).
__global__ void __launch_bounds__(kRouteThreads) k_route_pack(
    int n, int g0, const float4* __restrict__ records, const float4* __restrict__ cull,
    const uint2* __restrict__ rects, const float* __restrict__ depths, const int2* __restrict__ dest,
    const int32_t* __restrict__ block_offsets, int world, RouteDests d, int fence, int32_t* __restrict__ src) {
    __shared__ int wcount[kMaxPeerRanks][kRouteThreads / 32];
    __shared__ int slane[kRouteThreads / 32][32];  // per warp: t-th going lane
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int2 dq = i < n ? dest[i] : make_int2(-1, -2);
    for (int q = 0; q < world; ++q) {
        const unsigned b = __ballot_sync(0xffffffffu, q >= dq.x && q <= dq.y);
        if (lane == 0) wcount[q][warp] = __popc(b);
    }
    __syncthreads();
    const int i0 = blockIdx.x * blockDim.x + warp * 32;  // the warp's first local index
    for (int q = 0; q < world; ++q) {
        const bool goes = q >= dq.x && q <= dq.y;
        const unsigned b = __ballot_sync(0xffffffffu, goes);
        if (b == 0u) continue;
        // the warp's items for q are consecutive in the group, from k0
        int wbefore = 0;
        for (int w2 = 0; w2 < warp; ++w2) wbefore += wcount[q][w2];
        const int64_t k0 = block_offsets[(size_t)blockIdx.x * world + q] + wbefore;
        const int rk = __popc(b & ((1u << lane) - 1u));
        if (goes) {
            src[d.send_base[q] + k0 + rk] = i;
            slane[warp][rk] = lane;
        }
        __syncwarp();
        // the warp writes the run together: four whole payloads (512
        // contiguous bytes) per store instruction, lane l the float4 l % 8
        // of payload l / 8 (peer stores stay full-line over NVLink)
        const int cnt = __popc(b);
        float4* run = d.dst[q] + k0 * kRoutePayloadF4;
        for (int idx = lane; idx < cnt * kRoutePayloadF4; idx += 32) {
            const int t = idx / kRoutePayloadF4, c = idx % kRoutePayloadF4;
            const int j = i0 + slane[warp][t];  // t-th lane going to q (t < cnt)
            float4 v;
            if (c < kRecordF4) {
                v = records[(size_t)j * kRecordF4 + c];
            } else if (c < kRecordF4 + kCullF4) {
                v = cull[(size_t)j * kCullF4 + (c - kRecordF4)];
            } else {
                const uint2 r = rects[j];
                v = make_float4(__uint_as_float(r.x), __uint_as_float(r.y), depths[j], __int_as_float(g0 + j));
            }
            run[idx] = v;
        }
        __syncwarp();  // slane is rewritten for the next destination
    }
    if (fence) __threadfence_system();
}

// Band rank: pushes the raster-gradient record of every received item back
// to its owner: item j came from source r (recv_off[r] <= j < recv_off[r+1])
// as r's k-th item for this band, and goes to ret.dst[r] + k (the owner's
// return box at the offset of this band's group, written over NVLink).
__global__ void __launch_bounds__(kRouteThreads) k_route_push(int64_t m, const float4* __restrict__ grads, int world,
                                                              RouteReturns ret) {
    // a warp moves 32 items, eight whole records (512 bytes) per store
    // instruction: lane l the float4 l % 4 of item l / 4 of each group of 8
    constexpr int kF4 = kGradStride / 4;
    const int lane = threadIdx.x & 31;
    const int64_t j0 = ((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31));
    for (int idx = lane; idx < 32 * kF4; idx += 32) {
        const int64_t j = j0 + idx / kF4;
        if (j >= m) break;
        int r = 0;
        while (r + 1 < world && j >= ret.recv_off[r + 1]) ++r;
        ret.dst[r][(j - ret.recv_off[r]) * kF4 + idx % kF4] = grads[j * kF4 + idx % kF4];
    }
    __threadfence_system();
}

// Receiver: payloads (in increasing global id order) into the binning and
// rasteriser arrays at local index j, the global id in ids[j], and the tile
// rectangle into the per-id-chunk difference arrays the tile counts read
// (chunk j / id_chunk), as the projection does.
__global__ void __launch_bounds__(kRouteThreads) k_route_unpack(
    int64_t m, const float4* __restrict__ in, int tx, int ty, int id_chunk, float4* __restrict__ records,
    float4* __restrict__ cull, uint2* __restrict__ rects, float* __restrict__ depths, int32_t* __restrict__ ids,
    int32_t* __restrict__ radii, int32_t* __restrict__ tile_diff) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= m) return;
    const float4* p = in + j * kRoutePayloadF4;
#pragma unroll
    for (int k = 0; k < kRecordF4; ++k) records[j * kRecordF4 + k] = p[k];
#pragma unroll
    for (int k = 0; k < kCullF4; ++k) cull[j * kCullF4 + k] = p[kRecordF4 + k];
    const float4 t = p[kRecordF4 + kCullF4];
    const uint2 r = make_uint2(__float_as_uint(t.x), __float_as_uint(t.y));
    rects[j] = r;
    depths[j] = t.z;
    ids[j] = __float_as_int(t.w);
    radii[j] = 1;  // every received Gaussian is visible (its radius stays with its owner)
    const int4 q = unpack_rect(r);
    if (q.z <= q.x || q.w <= q.y) return;
    const int dw = tx + 1;
    int32_t* diff = tile_diff + (size_t)(j / id_chunk) * dw * (ty + 1);
    atomicAdd(&diff[q.y * dw + q.x], 1);
    atomicAdd(&diff[q.y * dw + q.z], -1);
    atomicAdd(&diff[q.w * dw + q.x], -1);
    atomicAdd(&diff[q.w * dw + q.z], 1);
}

// Owner: adds the raster-gradient records that came back (item p belongs to
// local Gaussian src[p]) into the slice's records.
__global__ void __launch_bounds__(kRouteThreads) k_route_gather(int64_t items, const float4* __restrict__ grads,
                                                                const int32_t* __restrict__ src,
                                                                float* __restrict__ slice_grads) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= items) return;
    float4* dst = reinterpret_cast<float4*>(slice_grads + (size_t)src[p] * kGradStride);
#pragma unroll
    for (int k = 0; k < kGradStride / 4; ++k) {
        const float4 v = grads[p * (kGradStride / 4) + k];
        if (v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f) atomicAdd(dst + k, v);
    }
}

}  // namespace

void launch_route_summary(const int32_t* diff, int tx, int ty, int n, const uint2* rects, const int32_t* radii,
                          int32_t* rowsum, int32_t* summary, cudaStream_t s) {
    if (tx <= 0 || ty <= 0) return;
    // the histograms (summary + tx * ty, 2 (ty + 1) ints) are zeroed by the caller
    int32_t* starts = summary + (size_t)tx * ty;
    note_launches(n > 0 ? 3 : 2);
    k_route_prefix_rows<<<(ty + 7) / 8, 256, 0, s>>>(diff, tx, ty, rowsum);
    k_route_prefix_cols<<<(tx + 31) / 32, dim3(32, 32), 0, s>>>(rowsum, tx, ty, summary);
    if (n > 0) {
        const size_t smem = 2 * (size_t)(ty + 1) * sizeof(int);
        if (smem > 48 * 1024)
            (void)cudaFuncSetAttribute(k_route_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_route_hist<<<(n + kRouteThreads - 1) / kRouteThreads, kRouteThreads, smem, s>>>(n, rects, radii, ty, starts,
                                                                                         starts + (ty + 1));
    }
}

void launch_route_plan(const int32_t* summaries, int tx, int ty, int world, int64_t* row_work, int32_t* bands,
                       int64_t* matrix, int n, const uint2* rects, const int32_t* radii, int2* dest,
                       int32_t* block_counts, int64_t* totals, int64_t* base, cudaStream_t s) {
    const int nblocks = (n + kRouteThreads - 1) / kRouteThreads;
    const int64_t len = route_summary_len(tx, ty);
    note_launches(nblocks > 0 ? 4 : 3);
    k_route_row_work<<<(ty + 7) / 8, 256, 0, s>>>(summaries, len, tx, ty, world, row_work);
    const size_t smem = (size_t)(2 * ty + 1) * sizeof(int64_t);
    if (smem > 48 * 1024)
        (void)cudaFuncSetAttribute(k_route_cuts, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_route_cuts<<<1, kCutThreads, smem, s>>>(summaries, len, tx, ty, world, row_work, bands, matrix);
    if (nblocks > 0)
        k_route_dest<<<nblocks, kRouteThreads, 0, s>>>(n, rects, radii, bands, world, ty, dest, block_counts);
    k_route_scan<<<1, kScanThreads, 0, s>>>(block_counts, nblocks, world, totals, base);
}

void launch_route_pack(int n, int g0, const float4* records, const float4* cull, const uint2* rects,
                       const float* depths, const int2* dest, const int32_t* block_offsets, int world,
                       const RouteDests& d, bool fence, int32_t* src, cudaStream_t s) {
    if (n <= 0) return;
    note_launches(1);
    k_route_pack<<<(n + kRouteThreads - 1) / kRouteThreads, kRouteThreads, 0, s>>>(
        n, g0, records, cull, rects, depths, dest, block_offsets, world, d, fence ? 1 : 0, src);
}

void launch_route_push(int64_t m, const float4* grads, int world, const RouteReturns& ret, cudaStream_t s) {
    if (m <= 0) return;
    note_launches(1);
    k_route_push<<<(unsigned)((m + kRouteThreads - 1) / kRouteThreads), kRouteThreads, 0, s>>>(m, grads, world, ret);
}

void launch_route_unpack(int64_t m, const float4* in, int tx, int ty, int id_chunk, float4* records, float4* cull,
                         uint2* rects, float* depths, int32_t* ids, int32_t* radii, int32_t* tile_diff,
                         cudaStream_t s) {
    if (m <= 0) return;
    note_launches(1);
    k_route_unpack<<<(unsigned)((m + kRouteThreads - 1) / kRouteThreads), kRouteThreads, 0, s>>>(
        m, in, tx, ty, id_chunk, records, cull, rects, depths, ids, radii, tile_diff);
}

void launch_route_gather(int64_t items, const float4* grads, const int32_t* src, float* slice_grads, cudaStream_t s) {
    if (items <= 0) return;
    note_launches(1);
    k_route_gather<<<(unsigned)((items + kRouteThreads - 1) / kRouteThreads), kRouteThreads, 0, s>>>(
        items, grads, src, slice_grads);
}

}  // namespace msplat
