// kernels.cuh — launch interfaces of the msplat B200 kernels (host side).
//
// Each kernel family lives in its own translation unit; backend.cu sequences
// them on one CUDA stream. All pointers are device pointers. Layouts follow
// the reference (core/metal/msplat_metal.mm:353-537) for every tensor that
// crosses the public boundary; the raster record and the raster-gradient
// record are internal (common.cuh).
#pragma once
#include <cstdint>
#include <string>
#include <cuda_runtime.h>

namespace msplat {

// Kernel-launch accounting (msplat_launch_count): every launcher records the
// kernels it enqueues.
void note_launches(int k);
// Sets the calling thread's msplat_last_error() text ("" clears it).
void set_last_error(const std::string& msg);

struct CameraDev {
    float viewmat[16];
    float projmat[16];
    float fx, fy, cx, cy;
    int width, height, tiles_x, tiles_y;
    float cam_pos[3];
};

// ---- projection (project.cu) ------------------------------------------------
constexpr int kMaxPeerRanks = 16;
// Gaussian ids are split into this many contiguous chunks for the per-tile
// counts, so that a tile over the 2048 cap emits only the chunks that can hold
// its 2048 lowest ids.
constexpr int kIdChunks = 32;
// Side of the square blocks of tiles over which the largest id bound is kept
// (block_max), letting key emission skip a Gaussian whose id is past the
// bounds of all the blocks it touches.
constexpr int kLimitBlock = 8;

struct ProjFwdArgs {
    int n;
    // 0: geometry and colour; 1: geometry only (record colour left unset);
    // 2: colour only, for the Gaussians pass 1 kept (radii > 0)
    int pass;
    const float* means; const float* scales; const float* quats; const float* opacities;
    const float* f_dc; const float* f_rest;
    int rest_bases;          // K = num_sh_bases(degree) - 1
    int degrees_to_use;
    float glob_scale, clip_thresh;
    CameraDev cam;
    // product outputs
    float4* records;         // [N, 5] float4
    float4* cull;            // [N, 2] float4 cull record (written with the geometry)
    uint2* rects;            // [N] packed tile rect (x0 | y0 << 16, x1 | y1 << 16)
    float* depths;           // [N] view-space depth (sort key)
    int32_t* radii;          // [N]
    int32_t* tile_diff;      // [kIdChunks][(tiles_y+1) * (tiles_x+1)] 2-D difference arrays (+=)
    int id_chunk;            // Gaussian i counts into difference array i / id_chunk
    // optional reference-shaped outputs (may be null)
    float* xys; float* transmats; int32_t* num_tiles_hit; float* normal_opacity;
    float* colors; float* aabb;
    // multi-GPU: with peer_world > 1, Gaussian i's colour coefficients
    // (features_dc, features_rest) are read from the buffer of its owner rank
    // i / peer_chunk (a peer's memory mapped here); the geometry groups are
    // local (all-gathered by the caller)
    int peer_world, peer_chunk;
    const float* peer_dc[kMaxPeerRanks];
    const float* peer_rest[kMaxPeerRanks];
    // pass 2: colour only for Gaussians whose tile rectangle meets tile rows
    // [color_row0, color_row1) (color_row1 <= color_row0: all)
    int color_row0, color_row1;
    // pass 2: with rgb_in ([N, 3], the clamped colours for this camera,
    // computed by launch_shard_colors on the owners and all-gathered) the
    // colour is copied instead of evaluated; raw colours are not available
    const float* rgb_in;
};
void launch_project_forward(const ProjFwdArgs& a, cudaStream_t s);
// Clamped colours max(SH + 0.5, 0) of Gaussians [g0, g1) for a.cam into
// rgb_out[3 i .. 3 i + 2], with the SH code of the forward (bit-identical).
void launch_shard_colors(const ProjFwdArgs& a, int g0, int g1, float* rgb_out, cudaStream_t s);

struct ProjBwdArgs {
    int g_begin, g_end;      // Gaussians handled by this launch (a shard)
    float* means; float* scales; float* quats; float* f_dc; float* f_rest; float* opacities;
    int rest_bases, degrees_to_use;
    float glob_scale;
    CameraDev cam;
    const int32_t* radii;
    const float* raster_grads;   // [N, 16]
    // optional reference-shaped gradient outputs (null = not written)
    float* dL_dmean3D; float* dL_dscale; float* dL_dquat; float* dL_dmean2D;
    float* dL_dfeatures_dc; float* dL_dfeatures_rest; float* dL_dopacity;
    // densify statistics (updated in place; may be null)
    float* xys_grad_norm; float* vis_counts; float* max_2d_size; float inv_max_dim;
    // Adam (applied when do_adam != 0); group order means, scales, quats,
    // f_dc, f_rest, opacities
    int do_adam;
    float* exp_avg[6]; float* exp_avg_sq[6];
    float step_size[6];
    float beta1, beta2, bc2_sqrt, eps;
};
void launch_project_backward(const ProjBwdArgs& a, cudaStream_t s);

// ---- binning (binning.cu) ---------------------------------------------------
// Tile counts from the per-chunk difference arrays (chunk_counts: scratch of
// kIdChunks * tiles), the true raw counts (raw_true), the emitted counts
// (raw_counts: all intersections of a tile within the cap, the chunks up to
// the one holding its 2048th lowest id otherwise) with the id bound of each
// tile (id_limit), kept counts, exclusive scans and the two totals.
// totals[0] = emitted intersections (int64), totals[1] = kept, totals[2..3]
// = the band (when balancing), totals[4] = tiles with more than 512 keys,
// listed in big_tiles (capacity: the tile count) for the CTA sort.
// fill[t] receives raw_start[t]: the key counter of k_emit_keys. Only
// tile rows [row0, row1) are binned; the other rows get empty ranges.
// row_work (optional, [tiles_y]) receives a per-row work estimate over all
// rows, for balancing tile-row bands across GPUs.
void launch_tile_counts(const int32_t* tile_diff, int id_chunk, int32_t* chunk_counts, int32_t* raw_true,
                        int32_t* id_limit, int32_t* block_max, int tiles_x, int tiles_y, int row0, int row1,
                        int32_t* raw_counts, int64_t* raw_start, uint64_t* fill, int2* tile_bins, int64_t* totals,
                        int64_t* row_work, uint32_t* err, cudaStream_t s,
                        int world, int rank, int32_t* big_tiles);
void launch_emit_keys(int n, const uint2* rects, const float* depths, int tiles_x, int row0, int row1,
                      const int32_t* id_limit, const int32_t* block_max, uint64_t* fill, uint64_t* raw_keys,
                      cudaStream_t s);
// num_gaussians bounds the ids (the overfull-tile select needs a third digit
// pass above 2^24 Gaussians).
void launch_tile_sort(int tile0, int num_tiles, const int32_t* raw_counts, const int64_t* raw_start,
                      const uint64_t* raw_keys, const int2* tile_bins, int32_t* gaussian_ids,
                      uint32_t* err, int num_gaussians, const int32_t* big_tiles, int num_big, cudaStream_t s);

// ---- rasterisation (rasterize.cu) -------------------------------------------
struct RasterFwdArgs {
    int width, height, tiles_x, tiles_y;
    int tile_row_begin, tile_row_end;   // tile rows rendered by this launch
    const int2* tile_bins; const int32_t* gaussian_ids; const float4* records;
    const float4* cull;                 // [N, 2] cull records of the projection
    float bg[3];
    float* final_Ts; int32_t* final_idx; float* out_img; float* out_depth; float* out_normal;
    float* out_alpha; float* out_median_depth; float* out_distortion;
    // [kept intersections] one byte per tile-list entry: bit w set when warp w
    // of the tile's CTA blended that surfel (read by the backward)
    uint8_t* blend_mask;
    // optional work counters (+=, may be null): [0] blended (pixel, surfel)
    // pairs, [1] (warp, surfel) visits evaluated past the cull
    unsigned long long* counters;
    // 1: every output of the reference's forward; 0: only out_img, final_Ts
    // channel 0 (T) and final_idx channel 0 (last contributor), which is all a
    // colour-only training step reads
    int aux_outputs;
};
void launch_rasterize_forward(const RasterFwdArgs& a, cudaStream_t s);

struct RasterBwdArgs {
    int width, height, tiles_x, tiles_y;
    int tile_row_begin, tile_row_end;
    const int2* tile_bins; const int32_t* gaussian_ids; const float4* records;
    float bg[3];
    const float* final_Ts; const int32_t* final_idx;
    const float* dL_dout_img;
    // auxiliary upstream gradients; all null (and dist_grad == 0) selects the
    // colour-only kernel used by training
    const float* dL_dout_depth; const float* dL_dout_alpha; const float* dL_dout_normal;
    const float* dL_dout_median_depth;
    float dL_dout_distortion;            // uniform per-pixel distortion gradient
    float* raster_grads;                 // [N, 16] (+=)
    const uint8_t* blend_mask;           // written by the forward over the same tiles
    // optional work counters (+=, may be null): [2] (warp, surfel) visits,
    // [3] blended (pixel, surfel) pairs replayed
    unsigned long long* counters;
};
void launch_rasterize_backward(const RasterBwdArgs& a, cudaStream_t s);

// ---- loss (ssim_loss.cu) ------------------------------------------------------
struct LossArgs {
    int width, height;
    int row_begin, row_end;              // pixel rows owned by this launch
    const float* out_img; const float* gt; const float* out_distortion;
    float lambda_l1, lambda_dist, lambda_dssim;
    float inv_num;                       // 1 / (3 * H * W) of the full image
    float* dL_dout_img;                  // written for owned rows
    double* partials;                    // [num_blocks * 3] (l1, ssim, dist) per block
};
// max_blocks > 0 caps the grid (strips x row segments) at that many CTAs.
int loss_num_blocks(int width, int row_begin, int row_end, int max_blocks = 0);
void launch_loss_ssim(const LossArgs& a, cudaStream_t s, int max_blocks = 0);
// Sums the block partials in a fixed order: out[0] = loss, out[1] = ssim sum,
// out[2] = l1 term, out[3] = distortion term (all double), loss_f = float loss.
void launch_loss_finalize(const double* partials, int num_blocks, float lambda_dssim, float inv_num,
                          double* out, float* loss_f, uint32_t* err, cudaStream_t s);

// Allocation-free loss forward/backward (scratch in fixed device arrays of
// ssim_loss.cu). Returns an MSPLAT_* code and fills *msg on failure.
int loss_ssim_noalloc(const float* out_img, const float* gt, const float* out_distortion, int width, int height,
                      float lambda_l1, float lambda_dist, float lambda_dssim, float* dL_dout_img, float* loss_out,
                      cudaStream_t s, std::string* msg);

// ---- routed multi-GPU exchange (route.cu) -------------------------------------
// Route summary of a slice ([tiles + 2 (ty + 1)] int32): per-tile counts
// from its projection's difference array, then the number of the slice's
// routable Gaussians whose tile rectangle starts at row y, then those whose
// rectangle ends at row y (y in [0, ty]). rowsum: scratch [ty * tx].
inline int64_t route_summary_len(int tx, int ty) { return (int64_t)tx * ty + 2 * (int64_t)(ty + 1); }
void launch_route_summary(const int32_t* diff, int tx, int ty, int n, const uint2* rects, const int32_t* radii,
                          int32_t* rowsum, int32_t* summary, cudaStream_t s);
// From the summaries of all ranks ([world][summary length]): the bands of all
// ranks (bands [world + 1]), the items from every rank to every rank
// (matrix [world][world], int64), the destination range of each projected
// Gaussian of this slice, per-block offsets per destination (block_counts,
// scanned in place) and this slice's items per destination (totals [world]).
void launch_route_plan(const int32_t* summaries, int tx, int ty, int world, int64_t* row_work, int32_t* bands,
                       int64_t* matrix, int n, const uint2* rects, const int32_t* radii, int2* dest,
                       int32_t* block_counts, int64_t* totals, int64_t* base, cudaStream_t s);
// A routed Gaussian: raster record (5 float4), cull record (2 float4), then
// (rect.x bits, rect.y bits, depth, global id bits).
constexpr int kRoutePayloadF4 = 8;
// Where the routed items go: group q (the items for destination rank q)
// starts at dst[q] (a local send buffer or a peer's inbox mapped here), and
// send_base[q] is its first item in this rank's packing order.
struct RouteDests {
    float4* dst[kMaxPeerRanks];
    int64_t send_base[kMaxPeerRanks];
};
// Where the band's records go back: items from source r (received items
// [recv_off[r], recv_off[r+1])) to dst[r] (the owner's return box at this
// band's group, mapped here).
struct RouteReturns {
    float4* dst[kMaxPeerRanks];
    int64_t recv_off[kMaxPeerRanks + 1];
};
// 128-byte payloads of the slice's Gaussians per destination;
// src[item] = local index (packing order). fence: system-scope fence after
// the stores (peer destinations).
void launch_route_pack(int n, int g0, const float4* records, const float4* cull, const uint2* rects,
                       const float* depths, const int2* dest, const int32_t* block_offsets, int world,
                       const RouteDests& d, bool fence, int32_t* src, cudaStream_t s);
// The band's records [m, 16] back to their owners' return boxes.
void launch_route_push(int64_t m, const float4* grads, int world, const RouteReturns& ret, cudaStream_t s);
// Received payloads into the binning and rasteriser arrays (radii = 1: the
// received set is visible) and the per-id-chunk difference arrays.
void launch_route_unpack(int64_t m, const float4* in, int tx, int ty, int id_chunk, float4* records, float4* cull,
                         uint2* rects, float* depths, int32_t* ids, int32_t* radii, int32_t* tile_diff,
                         cudaStream_t s);
void launch_route_gather(int64_t items, const float4* grads, const int32_t* src, float* slice_grads, cudaStream_t s);

// ---- image helpers of the trainer API (image_ops.cu) --------------------------
void launch_resize_area(const float* src, int sw, int sh, float* dst, int dw, int dh, cudaStream_t s);
void launch_rgba8(const float* src, uint8_t* dst, int64_t n, cudaStream_t s);

// ---- Adam (adam.cu) -----------------------------------------------------------
void launch_fused_adam(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, int64_t n,
                       float step_size, float beta1, float beta2, float bc2_sqrt, float eps, cudaStream_t s);
void launch_unpack_raster_grads(int n, const float* raster_grads, float* dL_dtransMat, float* dL_dnormal3D,
                                float* dL_dcolors, float* dL_dopacity, cudaStream_t s);

}  // namespace msplat
