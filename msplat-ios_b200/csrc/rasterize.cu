// rasterize.cu — 2DGS tile rasteriser, forward and backward.
//
// Forward follows nd_rasterize_forward_2dgs_kernel
// (core/metal/msplat_metal.metal:553-754): per pixel, front-to-back over the
// tile's depth-sorted surfels, ray/plane intersection through the surfel's
// homography, min(rho3d, 2 * d^2) falloff, alpha = min(0.99, o * exp(-rho/2)),
// skip below 1/255, stop when T would drop to 1e-4, plus depth, normal,
// median-depth and distortion outputs.
// Backward follows nd_rasterize_backward_2dgs_kernel (:1705-1979): reverse
// traversal recovering T as T / (1 - alpha).
//
// B200 design: one 256-thread CTA per 16x16 tile (the reference runs four
// 8x8 groups per tile, each re-reading the tile list); the tile's surfels are
// streamed in batches of 256: ids are read coalesced, the 80-byte per-Gaussian
// records (written once by the projection) are gathered into shared memory
// structure-of-arrays with cp.async (16-byte asynchronous copies, waited on
// before the batch barrier). Each warp owns an 8x4 pixel block: it tests 32
// surfels at a time (one per lane) against its block with the exact
// screen-space conic of rho3d <= rmax and the 2-D filter disc (32-byte cull
// records from the projection), and walks only the surfels that can reach
// the block. The forward records, per tile-list entry, which warps blended
// the surfel (one bit per warp); the backward drops entries no warp blended
// and each warp visits only its own, so pairs that were rejected in the
// forward are not evaluated again. In the backward the per-(pixel, surfel)
// gradients are summed across the warp through a per-warp transpose buffer in
// shared memory (13 stores, four 16-byte loads and one shuffle per lane),
// across warps in shared memory, and leave the CTA as four float4 atomics per
// surfel. The replayed pair evaluation follows the forward's operation
// sequence with the hardware reciprocal and exponential; the gradient
// arithmetic after it uses fast reciprocals.
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

constexpr int kThreads = 256;

struct Pair {
    float u, v, inv_z, rho3d, rho2d, depth, G, alpha;
    float kx, ky, kz, lx, ly, lz;
    float p_x, p_y, p_z;
};

// Per-(pixel, surfel) evaluation in two stages, both straight-line (every
// test is folded into the returned predicate, so that the lanes of a warp do
// not diverge inside them).
//
// Stage 1: the 2-D falloff, k = px Tw - Tu, l = py Tw - Tv and p = k x l.
// Returns false when both falloffs certainly exceed rmax: such a pair fails
// the alpha >= 1/255 test of stage 2 anyway. The forward uses it to skip a
// surfel for the whole warp when no lane passes.
__device__ __forceinline__ bool pair_stage1(float px, float py, float4 r0, float4 r1, float4 r2, float rmax, Pair& e) {
    // Tu = r0.xyz, Tv = (r0.w, r1.x, r1.y), Tw = (r1.z, r1.w, r2.x), xy = r2.yz, opacity = r2.w
    const float dx = fsub(r2.y, px), dy = fsub(r2.z, py);
    e.rho2d = fmul(kFilterInvSq, ffma(dx, dx, fmul(dy, dy)));
    e.kx = ffma(px, r1.z, -r0.x); e.ky = ffma(px, r1.w, -r0.y); e.kz = ffma(px, r2.x, -r0.z);
    e.lx = ffma(py, r1.z, -r0.w); e.ly = ffma(py, r1.w, -r1.x); e.lz = ffma(py, r2.x, -r1.y);
    e.p_x = ffma(e.ky, e.lz, -fmul(e.kz, e.ly));
    e.p_y = ffma(e.kz, e.lx, -fmul(e.kx, e.lz));
    e.p_z = ffma(e.kx, e.ly, -fmul(e.ky, e.lx));
    return !(e.rho2d > rmax && e.p_x * e.p_x + e.p_y * e.p_y > (rmax * 1.0001f) * (e.p_z * e.p_z));
}

// Stage 2: ray/plane intersection, falloff, depth and alpha; returns whether
// the pair is blended (p.z != 0, depth >= near, alpha >= 1/255). EXACT (the
// forward): a pinned IEEE operation sequence, identical in the CPU checker,
// with the IEEE reciprocal and the deterministic exponential. The backward
// replay uses the hardware reciprocal and exponential instead (a few ulp
// apart): its gradients are compared within a tolerance, and a pair whose
// alpha lies within those ulp of 1/255 is the only one whose decision can
// differ from the forward's. Lanes whose result is discarded may evaluate
// out-of-range arguments here; every operation stays defined for them.
template <bool EXACT>
__device__ __forceinline__ bool pair_stage2(float4 r1, float4 r2, Pair& e) {
    const float inv_z = EXACT ? __frcp_rn(e.p_z) : __fdividef(1.0f, e.p_z);
    const float u = fmul(e.p_x, inv_z), v = fmul(e.p_y, inv_z);
    const float rho3d = ffma(u, u, fmul(v, v));
    const float rho = (e.rho2d < rho3d) ? e.rho2d : rho3d;
    const float depth = ffma(u, r1.z, ffma(v, r1.w, r2.x));
    const float power = fmul(-0.5f, rho);
    // for a lane that passed stage 1, power is in [-5.6, 0] or NaN
    const float G = EXACT ? det_exp_nonpos(power) : __expf(power);
    const float og = fmul(r2.w, G);
    const float alpha = (og < 0.99f) ? og : 0.99f;
    e.u = u; e.v = v; e.inv_z = inv_z; e.rho3d = rho3d; e.depth = depth; e.G = G; e.alpha = alpha;
    return (e.p_z != 0.0f) & !(depth < kNearN) & !(power > 0.0f) & !(alpha < 1.0f / 255.0f);
}

// Pixel of thread t inside its 16x16 tile: each warp covers an 8x4 block, so
// a small surfel tends to be rejected by whole warps.
__device__ __forceinline__ int tile_lx(int t) { return ((t >> 5) & 1) * 8 + (t & 7); }
__device__ __forceinline__ int tile_ly(int t) { return (t >> 6) * 4 + ((t >> 3) & 3); }

// Whether a surfel can reach alpha >= 1/255 anywhere in the pixel rectangle
// [x0, x1] x [y0, y1] (bounds already grown by kCullMargin), from its cull
// record (common.cuh) and its 2-D centre m: the filter disc
// |p - m|^2 <= rd2 meets the rectangle, or the minimum of d^T E d over the
// rectangle (d = p - centre), evaluated as the sum of squares
// (s1 d.x + t1 d.y)^2 + (s2 d.y)^2, is at most 1. For a convex quadratic whose
// minimum lies outside the rectangle, the minimum over the rectangle is on
// the edge x = clamp(centre.x) or on the edge y = clamp(centre.y); along
// each, the best other coordinate is the clamped unconstrained one.
__device__ __forceinline__ bool block_hit(float4 c0, float4 c1, float mx, float my, float x0, float x1, float y0,
                                          float y1) {
    const float ddx = fmaxf(0.f, fmaxf(x0 - mx, mx - x1)), ddy = fmaxf(0.f, fmaxf(y0 - my, my - y1));
    const float lox = x0 - c0.x, hix = x1 - c0.x, loy = y0 - c0.y, hiy = y1 - c0.y;
    const float dx = fminf(fmaxf(0.f, lox), hix), dy = fminf(fmaxf(0.f, loy), hiy);
    const float dy1 = fminf(fmaxf(c1.y * dx, loy), hiy);
    const float dx2 = fminf(fmaxf(c1.z * dy, lox), hix);
    const float h1 = fmaf(c0.z, dx, c0.w * dy1), g1 = c1.x * dy1;
    const float h2 = fmaf(c0.z, dx2, c0.w * dy), g2 = c1.x * dy;
    const float q1 = fmaf(h1, h1, g1 * g1), q2 = fmaf(h2, h2, g2 * g2);
    return c1.w >= 0.f && (fminf(q1, q2) <= 1.f || fmaf(ddx, ddx, ddy * ddy) <= c1.w);
}

// Packs the per-warp blend flags of batch entry threadIdx.x (one byte per
// warp in sflag) into one bit per warp and stores it for tile-list entry
// b0 + threadIdx.x.
__device__ __forceinline__ void flush_blend_flags(uint8_t* mask, const uint2* sflag, int b0, int end) {
    const int idx = b0 + threadIdx.x;
    if (idx >= end) return;
    const uint2 f = sflag[threadIdx.x];
    uint32_t m = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) m |= (((f.x >> (8 * w)) & 1u) << w) | (((f.y >> (8 * w)) & 1u) << (w + 4));
    mask[idx] = (uint8_t)m;
}

// AUXOUT: every output of the reference's forward; otherwise only what a
// colour-only training step consumes (the image, the final transmittance and
// the last contributor), skipping depth, normal, median and distortion.
// COUNT: accumulate the work counters (a.counters); compiled out otherwise.
template <bool AUXOUT, bool COUNT>
__global__ void __launch_bounds__(kThreads, 4) k_raster_fwd(RasterFwdArgs a) {
    __shared__ float4 srec[kRecordF4][kThreads];
    __shared__ float4 scull[kCullF4][kThreads];
    __shared__ uint2 sflag[kThreads];  // per batch entry: byte w set when warp w blended it
    constexpr unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tile = (a.tile_row_begin + blockIdx.y) * a.tiles_x + blockIdx.x;
    const int lx = tile_lx(threadIdx.x), ly = tile_ly(threadIdx.x);
    // this warp's 8x4 pixel block, grown by the cull margin
    const float wx0 = (float)(blockIdx.x * kTile + (warp & 1) * 8) - kCullMargin, wx1 = wx0 + (7.f + 2.f * kCullMargin);
    const float wy0 = (float)((a.tile_row_begin + blockIdx.y) * kTile + (warp >> 1) * 4) - kCullMargin,
                wy1 = wy0 + (3.f + 2.f * kCullMargin);
    const int j = blockIdx.x * kTile + lx;
    const int i = (a.tile_row_begin + blockIdx.y) * kTile + ly;
    const bool inside = (i < a.height) && (j < a.width);
    const float px = (float)j, py = (float)i;
    const int2 range = a.tile_bins[tile];
    const float mscale = __fdiv_rn(kFarN, __fsub_rn(kFarN, kNearN));

    float T = 1.f, cr = 0.f, cg = 0.f, cb = 0.f, nx = 0.f, ny = 0.f, nz = 0.f, pdepth = 0.f;
    // contributor: 1-based position in the tile list of the surfel being
    // blended (the reference's per-pixel counter, metal:612-650)
    float M1 = 0.f, M2 = 0.f, dist = 0.f, median_depth = 0.f;
    int median_c = -1, contributor = 0, last_c = 0;
    bool done = !inside;

    int flush_b0 = -1;  // batch whose blend flags are still in sflag
    unsigned n_visits = 0, n_blend = 0;  // work counters (visits are warp-uniform)
    for (int b0 = range.x; b0 < range.y; b0 += kThreads) {
        const bool all_done = __syncthreads_count(done) == kThreads;
        if (flush_b0 >= 0) flush_blend_flags(a.blend_mask, sflag, flush_b0, range.y);
        flush_b0 = -1;
        if (all_done) break;
        const int idx = b0 + threadIdx.x;
        if (idx < range.y) {
            const int g = a.gaussian_ids[idx];
            const float4* r = a.records + (size_t)g * kRecordF4;
            const float4* cr = a.cull + (size_t)g * kCullF4;
#pragma unroll
            for (int k = 0; k < kRecordF4; ++k) cp_async16(&srec[k][threadIdx.x], r + k);
#pragma unroll
            for (int k = 0; k < kCullF4; ++k) cp_async16(&scull[k][threadIdx.x], cr + k);
        }
        sflag[threadIdx.x] = make_uint2(0u, 0u);
        cp_async_wait_all();
        __syncthreads();
        flush_b0 = b0;
        if (__all_sync(full, done)) continue;
        const int bs = min(kThreads, range.y - b0);
        const int base = b0 - range.x + 1;  // 1-based position of surfel 0 of this batch in the tile list
        // 32 surfels at a time: one cull test per lane, then the warp walks
        // the surfels that can reach its 8x4 pixel block
        for (int c = 0; c < bs; c += 32) {
            bool hit = false;
            if (c + lane < bs) {
                const int q = c + lane;
                const float4 r2 = srec[2][q];
                hit = block_hit(scull[0][q], scull[1][q], r2.y, r2.z, wx0, wx1, wy0, wy1);
            }
            unsigned bits = __ballot_sync(full, hit);
            while (bits) {
                const int s = c + __ffs(bits) - 1;
                bits &= bits - 1;
                // no per-pixel cull test: the surfel can reach this warp's
                // block; stage 1's rejection bound covers the pixels it
                // cannot reach, and the warp moves on when no lane is left
                Pair e;
                const float4 q1 = srec[1][s], q2 = srec[2][s];
                const bool cand = (!done) & pair_stage1(px, py, srec[0][s], q1, q2, srec[4][s].z, e);
                if (!__any_sync(full, cand)) continue;
                if (COUNT) ++n_visits;
                if (!(pair_stage2<true>(q1, q2, e) & cand)) continue;
                contributor = base + s;
                const float next_T = fmul(T, fsub(1.0f, e.alpha));
                if (next_T <= 1e-4f) {
                    done = true;
                    continue;
                }
                const float w = fmul(e.alpha, T);
                if constexpr (AUXOUT) {
                    const float A = fsub(1.f, T);
                    const float m = fmul(mscale, fsub(1.f, __fdiv_rn(kNearN, e.depth)));
                    const float mm = fmul(m, m);
                    dist = ffma(fsub(fadd(fmul(mm, A), M2), fmul(fmul(2.f, m), M1)), w, dist);
                    M1 = ffma(m, w, M1);
                    M2 = ffma(mm, w, M2);
                    if (T > 0.5f) {
                        median_depth = e.depth;
                        median_c = contributor;
                    }
                }
                const float4 r3 = srec[3][s];
                cr = ffma(r3.x, w, cr);
                cg = ffma(r3.y, w, cg);
                cb = ffma(r3.z, w, cb);
                if constexpr (AUXOUT) {
                    const float4 r4 = srec[4][s];
                    pdepth = ffma(e.depth, w, pdepth);
                    nx = ffma(r3.w, w, nx);
                    ny = ffma(r4.x, w, ny);
                    nz = ffma(r4.y, w, nz);
                }
                T = next_T;
                last_c = contributor;
                if (COUNT) ++n_blend;
                reinterpret_cast<uint8_t*>(&sflag[s])[warp] = 1;
            }
            if (__all_sync(full, done)) break;
        }
    }
    if (flush_b0 >= 0) {
        __syncthreads();
        flush_blend_flags(a.blend_mask, sflag, flush_b0, range.y);
    }
    if (COUNT && a.counters) {
        const unsigned blended = __reduce_add_sync(full, n_blend);
        if (lane == 0) {
            atomicAdd(a.counters + 0, (unsigned long long)blended);
            atomicAdd(a.counters + 1, (unsigned long long)n_visits);
        }
    }
    if (!inside) return;
    const size_t pix = (size_t)i * a.width + j;
    a.final_Ts[3 * pix + 0] = T;
    a.final_idx[2 * pix + 0] = last_c;
    a.out_img[3 * pix + 0] = ffma(a.bg[0], T, cr);
    a.out_img[3 * pix + 1] = ffma(a.bg[1], T, cg);
    a.out_img[3 * pix + 2] = ffma(a.bg[2], T, cb);
    if (!AUXOUT) return;
    a.final_Ts[3 * pix + 1] = M1;
    a.final_Ts[3 * pix + 2] = M2;
    a.final_idx[2 * pix + 1] = median_c;
    a.out_depth[pix] = pdepth;
    a.out_normal[3 * pix + 0] = nx;
    a.out_normal[3 * pix + 1] = ny;
    a.out_normal[3 * pix + 2] = nz;
    a.out_alpha[pix] = fsub(1.f, T);
    a.out_median_depth[pix] = median_depth;
    a.out_distortion[pix] = dist;
}

// Gradient values reduced per (warp, surfel): 13 for the colour-only kernel,
// 16 with the auxiliary (normal) gradients.
template <bool AUX>
constexpr int bwd_values() { return AUX ? 16 : 13; }
// Dynamic shared memory of k_raster_bwd: records [5][256] float4, the
// per-batch accumulator [256][16] and the per-warp transpose buffers
// [8][NV][36] of the warp reduction.
template <bool AUX>
constexpr size_t bwd_dynamic_smem() {
    return sizeof(float4) * kRecordF4 * kThreads + sizeof(float) * kThreads * kGradStride +
           sizeof(float) * (kThreads / 32) * bwd_values<AUX>() * 36;
}

// COUNT: accumulate the work counters (a.counters); compiled out otherwise.
template <bool AUX, bool COUNT>
__global__ void __launch_bounds__(kThreads, 4) k_raster_bwd(RasterBwdArgs a) {
    extern __shared__ __align__(16) unsigned char dsm[];
    constexpr int NV = bwd_values<AUX>();
    float4 (*srec)[kThreads] = reinterpret_cast<float4 (*)[kThreads]>(dsm);
    float (*sacc)[kGradStride] =
        reinterpret_cast<float (*)[kGradStride]>(dsm + sizeof(float4) * kRecordF4 * kThreads);
    // per-warp transpose buffer of the warp reduction: value k of lane L at
    // [k][L]; rows of 36 floats keep both the stores and the 16-byte loads
    // free of bank conflicts
    float (*sred)[NV][36] = reinterpret_cast<float (*)[NV][36]>(
        dsm + sizeof(float4) * kRecordF4 * kThreads + sizeof(float) * kThreads * kGradStride);
    __shared__ int sid[kThreads];
    __shared__ int srel[kThreads];       // 0-based position in the tile list
    __shared__ uint8_t smask[kThreads];  // warps that blended the surfel in the forward
    __shared__ int swarp_cnt[kThreads / 32];
    __shared__ int s_max_last;
    constexpr unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tile_row = a.tile_row_begin + blockIdx.y;
    const int tile = tile_row * a.tiles_x + blockIdx.x;
    const int j = blockIdx.x * kTile + tile_lx(threadIdx.x);
    const int i = tile_row * kTile + tile_ly(threadIdx.x);
    const bool inside = (i < a.height) && (j < a.width);
    const float px = (float)j, py = (float)i;
    const int2 range = a.tile_bins[tile];
    const size_t pix = inside ? (size_t)i * a.width + j : 0;
    const float mscale = __fdiv_rn(kFarN, __fsub_rn(kFarN, kNearN));

    float T_final = 0.f, final_D = 0.f, final_D2 = 0.f;
    int last_c = 0, median_c = -1;
    float dpix[3] = {0.f, 0.f, 0.f};
    float dL_ddepth = 0.f, dL_daccum = 0.f, dL_dmed = 0.f, dnorm2[3] = {0.f, 0.f, 0.f};
    const float dL_dreg = a.dL_dout_distortion;
    if (inside) {
        T_final = a.final_Ts[3 * pix];
        last_c = a.final_idx[2 * pix];
        if (AUX) {
            final_D = a.final_Ts[3 * pix + 1];
            final_D2 = a.final_Ts[3 * pix + 2];
            median_c = a.final_idx[2 * pix + 1];
        }
        dpix[0] = a.dL_dout_img[3 * pix];
        dpix[1] = a.dL_dout_img[3 * pix + 1];
        dpix[2] = a.dL_dout_img[3 * pix + 2];
        if (AUX) {
            if (a.dL_dout_depth) dL_ddepth = a.dL_dout_depth[pix];
            if (a.dL_dout_alpha) dL_daccum = a.dL_dout_alpha[pix];
            if (a.dL_dout_median_depth) dL_dmed = a.dL_dout_median_depth[pix];
            if (a.dL_dout_normal)
                for (int c = 0; c < 3; ++c) dnorm2[c] = a.dL_dout_normal[3 * pix + c];
        }
    }
    if (threadIdx.x == 0) s_max_last = 0;
    __syncthreads();
    if (last_c > 0) atomicMax(&s_max_last, last_c);
    __syncthreads();
    const int hi = range.x + s_max_last;  // surfels at or past this index never blended
    const float final_A = 1.0f - T_final;
    const float bg_dot = a.bg[0] * dpix[0] + a.bg[1] * dpix[1] + a.bg[2] * dpix[2];

    float T = T_final;
    float accum_rec[3] = {0.f, 0.f, 0.f}, last_color[3] = {0.f, 0.f, 0.f}, last_alpha = 0.f;
    float accum_depth_rec = 0.f, last_depth = 0.f, accum_alpha_rec = 0.f, last_dL_dT = 0.f;
    float accum_normal_rec[3] = {0.f, 0.f, 0.f}, last_normal[3] = {0.f, 0.f, 0.f};
    unsigned n_visits = 0, n_blend = 0;  // work counters (visits are warp-uniform)

    for (int bend = hi; bend > range.x; bend -= kThreads) {
        const int bs = min(kThreads, bend - range.x);
        __syncthreads();  // the previous batch is consumed
        // entries blended by no warp are dropped; the rest are compacted in
        // back-to-front order
        const int rel_t = bend - 1 - (int)threadIdx.x - range.x;
        const uint32_t m = ((int)threadIdx.x < bs) ? a.blend_mask[range.x + rel_t] : 0u;
        // the id is read with the flags (one round trip less before the copies)
        const int g_pre = ((int)threadIdx.x < bs) ? a.gaussian_ids[range.x + rel_t] : 0;
        const unsigned bal = __ballot_sync(full, m != 0u);
        if (lane == 0) swarp_cnt[warp] = __popc(bal);
        __syncthreads();
        int off = 0, total = 0;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) {
            const int c = swarp_cnt[w];
            off += (w < warp) ? c : 0;
            total += c;
        }
        if (m != 0u) {
            const int pos = off + __popc(bal & ((1u << lane) - 1u));
            const int g = g_pre;
            sid[pos] = g;
            srel[pos] = rel_t;
            smask[pos] = (uint8_t)m;
            const float4* r = a.records + (size_t)g * kRecordF4;
#pragma unroll
            for (int k = 0; k < kRecordF4; ++k) cp_async16(&srec[k][pos], r + k);
        }
        if ((int)threadIdx.x < total) {
#pragma unroll
            for (int k = 0; k < kGradStride; ++k) sacc[threadIdx.x][k] = 0.f;
        }
        cp_async_wait_all();
        __syncthreads();
        for (int c = 0; c < total; c += 32) {
            unsigned bits = __ballot_sync(full, c + lane < total && ((smask[c + lane] >> warp) & 1u));
            while (bits) {
                const int s = c + __ffs(bits) - 1;
                bits &= bits - 1;
                const int rel = srel[s];
                if (COUNT) ++n_visits;
                float g[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) g[k] = 0.f;
                Pair e;
                const float4 r0 = srec[0][s], r1 = srec[1][s], r2 = srec[2][s];
                pair_stage1(px, py, r0, r1, r2, 0.f, e);
                if ((rel < last_c) & pair_stage2<false>(r1, r2, e)) {
                    if (COUNT) ++n_blend;
                    const float4 r3 = srec[3][s], r4 = srec[4][s];
                    const float alpha = e.alpha, G = e.G, opa = r2.w;
                    const float r1ma = __fdividef(1.0f, 1.0f - alpha);
                    T = T * r1ma;
                    const float w = alpha * T;
                    float dL_dalpha = 0.f;
                    const float col[3] = {r3.x, r3.y, r3.z};
#pragma unroll
                    for (int c3 = 0; c3 < 3; ++c3) {
                        accum_rec[c3] = last_alpha * last_color[c3] + (1.f - last_alpha) * accum_rec[c3];
                        last_color[c3] = col[c3];
                        dL_dalpha += (col[c3] - accum_rec[c3]) * dpix[c3];
                        // the clamp mask (per surfel) is applied at the flush
                        // in the colour-only kernel
                        g[10 + c3] = (!AUX || col[c3] > 0.f) ? w * dpix[c3] : 0.f;
                    }
                    float dL_dz = 0.f;
                    if (AUX) {
                        const float rd = __fdividef(1.0f, e.depth);
                        const float m_d = mscale * (1.0f - kNearN * rd);
                        const float dmd_dd = ((kFarN * kNearN) / (kFarN - kNearN)) * rd * rd;
                        if (rel == median_c - 1) dL_dz += dL_dmed;
                        const float dL_dweight = (final_D2 + m_d * m_d * final_A - 2.0f * m_d * final_D) * dL_dreg;
                        dL_dalpha += dL_dweight - last_dL_dT;
                        last_dL_dT = dL_dweight * alpha + (1.0f - alpha) * last_dL_dT;
                        const float dL_dmd = 2.0f * (T * alpha) * (m_d * final_A - final_D) * dL_dreg;
                        dL_dz += dL_dmd * dmd_dd;
                        accum_depth_rec = last_alpha * last_depth + (1.f - last_alpha) * accum_depth_rec;
                        last_depth = e.depth;
                        dL_dalpha += (e.depth - accum_depth_rec) * dL_ddepth;
                        accum_alpha_rec = last_alpha + (1.f - last_alpha) * accum_alpha_rec;
                        dL_dalpha += (1.0f - accum_alpha_rec) * dL_daccum;
                        const float nrm[3] = {r3.w, r4.x, r4.y};
#pragma unroll
                        for (int c3 = 0; c3 < 3; ++c3) {
                            accum_normal_rec[c3] = last_alpha * last_normal[c3] + (1.f - last_alpha) * accum_normal_rec[c3];
                            last_normal[c3] = nrm[c3];
                            dL_dalpha += (nrm[c3] - accum_normal_rec[c3]) * dnorm2[c3];
                            g[13 + c3] = w * dnorm2[c3];
                        }
                    }
                    dL_dalpha *= T;
                    last_alpha = alpha;
                    dL_dalpha += (-T_final * r1ma) * bg_dot;
                    const float dL_dG = opa * dL_dalpha;
                    if (AUX) dL_dz += w * dL_ddepth;
                    if (e.rho3d <= e.rho2d) {
                        const float dsx = -dL_dG * G * e.u + dL_dz * r1.z;
                        const float dsy = -dL_dG * G * e.v + dL_dz * r1.w;
                        const float dpx = dsx * e.inv_z, dpy = dsy * e.inv_z;
                        const float dpz = -(dpx * e.u + dpy * e.v);
                        if constexpr (AUX) {
                            // dk = cross(l, dp), dl = cross(dp, k)
                            const float dkx = e.ly * dpz - e.lz * dpy, dky = e.lz * dpx - e.lx * dpz,
                                        dkz = e.lx * dpy - e.ly * dpx;
                            const float dlx = dpy * e.kz - dpz * e.ky, dly = dpz * e.kx - dpx * e.kz,
                                        dlz = dpx * e.ky - dpy * e.kx;
                            g[0] = -dkx; g[1] = -dky; g[2] = -dkz;
                            g[3] = -dlx; g[4] = -dly; g[5] = -dlz;
                            g[6] = px * dkx + py * dlx + dL_dz * e.u;
                            g[7] = px * dky + py * dly + dL_dz * e.v;
                            g[8] = px * dkz + py * dlz + dL_dz;
                        } else {
                            // k = px Tw - Tu and l = py Tw - Tv are affine in the
                            // pixel, so the warp's sums of dk = l x dp, dl = dp x k
                            // and px dk + py dl follow from the sums of dp, px dp and
                            // py dp; the cross products are taken once per surfel
                            // when the CTA flushes its accumulator
                            g[0] = dpx; g[1] = dpy; g[2] = dpz;
                            g[3] = px * dpx; g[4] = px * dpy; g[5] = px * dpz;
                            g[6] = py * dpx; g[7] = py * dpy; g[8] = py * dpz;
                        }
                    } else if (AUX) {
                        g[6] = e.u * dL_dz;
                        g[7] = e.v * dL_dz;
                        g[8] = dL_dz;
                    }
                    // colour-only kernel: the per-surfel factor o (1 - o) is
                    // applied at the flush
                    g[9] = AUX ? G * dL_dalpha * (opa * (1.0f - opa)) : G * dL_dalpha;
                }
                // the forward's flags guarantee a contributing lane here: sum
                // value vi over the warp, lanes 2 vi and 2 vi + 1 each adding
                // 16 of the 32 lanes' entries
                float* wb = &sred[warp][0][0];
#pragma unroll
                for (int k = 0; k < NV; ++k) wb[k * 36 + lane] = g[k];
                __syncwarp();
                const int vi = lane >> 1;
                float tot = 0.f;
                if (vi < NV) {
                    const float4* row = reinterpret_cast<const float4*>(wb + vi * 36 + (lane & 1) * 16);
                    const float4 q0 = row[0], q1 = row[1], q2 = row[2], q3 = row[3];
                    // pairwise tree with sm_100 packed FP32 adds
                    const float2 s0 = __fadd2_rn(make_float2(q0.x, q0.y), make_float2(q0.z, q0.w));
                    const float2 s1 = __fadd2_rn(make_float2(q1.x, q1.y), make_float2(q1.z, q1.w));
                    const float2 s2 = __fadd2_rn(make_float2(q2.x, q2.y), make_float2(q2.z, q2.w));
                    const float2 s3 = __fadd2_rn(make_float2(q3.x, q3.y), make_float2(q3.z, q3.w));
                    const float2 s = __fadd2_rn(__fadd2_rn(s0, s1), __fadd2_rn(s2, s3));
                    tot = s.x + s.y;
                }
                tot += __shfl_xor_sync(full, tot, 1);
                __syncwarp();
                if (!(lane & 1) && vi < NV && tot != 0.f) atomicAdd(&sacc[s][vi], tot);
            }
        }
        __syncthreads();
        if constexpr (AUX) {
            for (int q = threadIdx.x; q < total * 4; q += kThreads) {
                const int s = q >> 2, part = q & 3;
                const float4 v = make_float4(sacc[s][4 * part], sacc[s][4 * part + 1], sacc[s][4 * part + 2],
                                             sacc[s][4 * part + 3]);
                if (v.x != 0.f || v.y != 0.f || v.z != 0.f || v.w != 0.f)
                    atomicAdd(reinterpret_cast<float4*>(a.raster_grads + (size_t)sid[s] * kGradStride) + part, v);
            }
        } else {
            for (int s = threadIdx.x; s < total; s += kThreads) {
                const float* acc = sacc[s];
                const float4 r0 = srec[0][s], r1 = srec[1][s], r2 = srec[2][s];
                const float tux = r0.x, tuy = r0.y, tuz = r0.z, tvx = r0.w, tvy = r1.x, tvz = r1.y;
                const float twx = r1.z, twy = r1.w, twz = r2.x;
                const float sx = acc[0], sy = acc[1], sz = acc[2];   // sum dp
                const float ax = acc[3], ay = acc[4], az = acc[5];   // sum px dp
                const float bx = acc[6], by = acc[7], bz = acc[8];   // sum py dp
                // sum dk = Tw x (sum py dp) - Tv x (sum dp)
                const float dkx = (twy * bz - twz * by) - (tvy * sz - tvz * sy);
                const float dky = (twz * bx - twx * bz) - (tvz * sx - tvx * sz);
                const float dkz = (twx * by - twy * bx) - (tvx * sy - tvy * sx);
                // sum dl = (sum px dp) x Tw - (sum dp) x Tu
                const float dlx = (ay * twz - az * twy) - (sy * tuz - sz * tuy);
                const float dly = (az * twx - ax * twz) - (sz * tux - sx * tuz);
                const float dlz = (ax * twy - ay * twx) - (sx * tuy - sy * tux);
                // sum (px dk + py dl) = Tu x (sum py dp) - Tv x (sum px dp)
                const float ex = (tuy * bz - tuz * by) - (tvy * az - tvz * ay);
                const float ey = (tuz * bx - tux * bz) - (tvz * ax - tvx * az);
                const float ez = (tux * by - tuy * bx) - (tvx * ay - tvy * ax);
                float4* dst = reinterpret_cast<float4*>(a.raster_grads + (size_t)sid[s] * kGradStride);
                const float4 p0 = make_float4(-dkx, -dky, -dkz, -dlx);
                const float4 p1 = make_float4(-dly, -dlz, ex, ey);
                const float opa = r2.w;
                const float4 r3 = srec[3][s];
                const float4 p2 = make_float4(ez, acc[9] * (opa * (1.0f - opa)), r3.x > 0.f ? acc[10] : 0.f,
                                              r3.y > 0.f ? acc[11] : 0.f);
                const float4 p3 = make_float4(r3.z > 0.f ? acc[12] : 0.f, 0.f, 0.f, 0.f);
                if (p0.x != 0.f || p0.y != 0.f || p0.z != 0.f || p0.w != 0.f) atomicAdd(dst, p0);
                if (p1.x != 0.f || p1.y != 0.f || p1.z != 0.f || p1.w != 0.f) atomicAdd(dst + 1, p1);
                if (p2.x != 0.f || p2.y != 0.f || p2.z != 0.f || p2.w != 0.f) atomicAdd(dst + 2, p2);
                if (p3.x != 0.f) atomicAdd(dst + 3, p3);
            }
        }
    }
    if (COUNT && a.counters) {
        const unsigned blended = __reduce_add_sync(full, n_blend);
        if (lane == 0) {
            atomicAdd(a.counters + 2, (unsigned long long)n_visits);
            atomicAdd(a.counters + 3, (unsigned long long)blended);
        }
    }
}

}  // namespace

namespace {
template <bool AUXOUT, bool COUNT>
void fwd_launch(const RasterFwdArgs& a, int rows, cudaStream_t s) {
    k_raster_fwd<AUXOUT, COUNT><<<dim3(a.tiles_x, rows), kThreads, 0, s>>>(a);
}
template <bool AUX, bool COUNT>
void bwd_launch(const RasterBwdArgs& a, int rows, cudaStream_t s) {
    constexpr size_t smem = bwd_dynamic_smem<AUX>();
    cudaFuncSetAttribute(k_raster_bwd<AUX, COUNT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(k_raster_bwd<AUX, COUNT>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    k_raster_bwd<AUX, COUNT><<<dim3(a.tiles_x, rows), kThreads, smem, s>>>(a);
}
}  // namespace

void launch_rasterize_forward(const RasterFwdArgs& a, cudaStream_t s) {
    const int rows = a.tile_row_end - a.tile_row_begin;
    if (rows <= 0 || a.tiles_x <= 0) return;
    note_launches(1);
    const bool count = a.counters != nullptr;
    if (a.aux_outputs)
        count ? fwd_launch<true, true>(a, rows, s) : fwd_launch<true, false>(a, rows, s);
    else
        count ? fwd_launch<false, true>(a, rows, s) : fwd_launch<false, false>(a, rows, s);
}

void launch_rasterize_backward(const RasterBwdArgs& a, cudaStream_t s) {
    const int rows = a.tile_row_end - a.tile_row_begin;
    if (rows <= 0 || a.tiles_x <= 0) return;
    const bool aux = a.dL_dout_depth || a.dL_dout_alpha || a.dL_dout_normal || a.dL_dout_median_depth ||
                     a.dL_dout_distortion != 0.0f;
    note_launches(1);
    const bool count = a.counters != nullptr;
    if (aux)
        count ? bwd_launch<true, true>(a, rows, s) : bwd_launch<true, false>(a, rows, s);
    else
        count ? bwd_launch<false, true>(a, rows, s) : bwd_launch<false, false>(a, rows, s);
}

}  // namespace msplat
