/*
 * oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference (ken001111/msplat-ios) 2DGS training step:
 * the Metal kernels in core/metal/msplat_metal.metal and the host orchestration
 * in core/metal/msplat_metal.mm:935-1331 and core/src/model.cpp:500-544,762-829.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library, and only as the checker or the timed CPU baseline.
 * The product (msplat-ios_b200/) never links or calls it.
 *
 * Parity pin: the reference cannot execute here (Metal Shading Language plus
 * ObjC++, no Apple toolchain), and its own tests hold no golden vectors or
 * known-answer tests for this path. This oracle is therefore pinned by
 * (a) the reference's fixed constants (SH basis constants, SSIM window),
 * (b) analytic known-answer cases and finite-difference gradient checks in
 * tests/, and (c) an independent torch-autograd restatement of the SSIM loss.
 * Parity against the Metal binary itself is "unpinned".
 *
 * Conventions (all match the reference's tensor layouts):
 *   means [N,3], scales [N,2] (log), quats [N,4] (q0 stored first, used as w),
 *   opacities [N] (logit), f_dc [N,3], f_rest [N,K,3] with K = bases-1,
 *   images [H,W,3] row-major, tiles 16x16 row-major.
 */
#ifndef MSPLAT_ORACLE_H
#define MSPLAT_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MAX_TILE_ELEMS 2048

typedef struct {
    float viewmat[16];   /* row-major world->camera */
    float projmat[16];   /* row-major world->clip (proj * view) */
    float fx, fy, cx, cy;
    int width, height;
    float cam_pos[3];
} OrcCamera;

/* Model::prepareCam (model.cpp:500-544) with downscale factor 1. */
void orc_prepare_cam(const float camToWorld[16], float fx, float fy, float cx,
                     float cy, int width, int height, OrcCamera* out);

/* Deterministic exp used everywhere the reference calls exp() on the forward
 * path (scales, sigmoid, the rasteriser's Gaussian falloff). */
float orc_exp(float x);

/* project_and_sh_forward_2dgs_kernel (msplat_metal.metal:1413-1521). Culled
 * Gaussians get radii = 0, num_tiles_hit = 0 and zeroed side outputs. */
void orc_project_forward(int n, const float* means, const float* scales,
                         float glob_scale, const float* quats,
                         const float* opacities, const float* f_dc,
                         const float* f_rest, int degree, int degrees_to_use,
                         const OrcCamera* cam, float clip_thresh,
                         float* xys, float* depths, int32_t* radii,
                         float* transmats, int32_t* num_tiles_hit,
                         float* normal_opacity, float* colors, float* aabb);

/* scatter_to_prealloc_bins_kernel + prefix_sum_kernel + the sort half of
 * bitonic_sort_per_tile_2dgs_kernel (metal:1557-1591, 3093-3145, 1606-1664)
 * with a deterministic overflow policy: a tile with more than 2048
 * intersections keeps the 2048 lowest Gaussian ids, then every tile is sorted
 * by the key (depth_bits << 32) | id.
 * Outputs: raw_counts[T] (un-clamped), tile_bins[T*2] = (start, end),
 * gaussian_ids[<= capacity]. Returns the number of kept intersections, or -1
 * when capacity is too small (nothing written to gaussian_ids then). */
int64_t orc_bin_and_sort(int n, const float* xys, const float* depths,
                         const int32_t* radii, const float* aabb,
                         int tiles_x, int tiles_y, int64_t* raw_counts,
                         int32_t* tile_bins, int32_t* gaussian_ids,
                         int64_t capacity);

/* Raw (un-clamped) intersection counts per tile, as orc_bin_and_sort
 * reports them, without building the key lists (scales to the billions of
 * intersections of an overloaded scene). */
void orc_tile_counts(int n, const float* xys, const int32_t* radii, const float* aabb, int tiles_x,
                     int tiles_y, int64_t* raw_counts);

/* Sorted kept Gaussian ids of the listed tiles under orc_bin_and_sort's
 * overflow policy, without building the other tiles' lists. ids_out holds
 * 2048 entries per listed tile; counts_out[k] = kept count of tiles[k]. */
void orc_tile_kept_ids(int n, const float* xys, const float* depths, const int32_t* radii, const float* aabb,
                       int tiles_x, int tiles_y, int num_tiles, const int32_t* tiles, int32_t* ids_out,
                       int32_t* counts_out);

/* Pack half of bitonic_sort_per_tile_2dgs_kernel (metal:1666-1689). */
void orc_pack(int64_t kept, const int32_t* gaussian_ids, const float* xys,
              const float* transmats, const float* normal_opacity,
              const float* colors, float* packed_xy, float* packed_transmat,
              float* packed_normal_opac, float* packed_rgb);

/* nd_rasterize_forward_2dgs_kernel (metal:553-754). */
void orc_rasterize_forward(int width, int height, int tiles_x,
                           const int32_t* tile_bins, const float* packed_xy,
                           const float* packed_normal_opac,
                           const float* packed_transmat, const float* packed_rgb,
                           const float* background, float* final_Ts,
                           int32_t* final_idx, float* out_img, float* out_depth,
                           float* out_normal, float* out_alpha,
                           float* out_median_depth, float* out_distortion);

/* loss_l1_distortion_2dgs_kernel + the SSIM forward/backward kernel chain
 * (metal:2704-2762, 2823-3085; dispatch order msplat_metal.mm:1077-1212).
 * Writes dL_dout_img [H,W,3] and dL_dout_distortion [H,W]; returns the loss in
 * *loss and the SSIM-map sum in *ssim_sum. */
void orc_loss_ssim(int width, int height, const float* out_img, const float* gt,
                   const float* out_distortion, float lambda_l1,
                   float lambda_dist, float lambda_dssim, float* dL_dout_img,
                   float* dL_dout_distortion, double* loss, double* ssim_sum);

/* nd_rasterize_backward_2dgs_kernel (metal:1705-1979). Accumulators are
 * double precision (a fixed-order stand-in for the float atomics) and are
 * converted to float at the end; outputs are overwritten, not added to.
 * Any of the aux upstream gradient maps may be NULL (= zeros). */
void orc_rasterize_backward(int n, int width, int height, int tiles_x,
                            const int32_t* tile_bins, const int32_t* gaussian_ids,
                            const float* packed_xy, const float* packed_normal_opac,
                            const float* packed_transmat, const float* packed_rgb,
                            const float* final_Ts, const int32_t* final_idx,
                            const float* background, const float* dL_dout_img,
                            const float* dL_dout_depth, const float* dL_dout_alpha,
                            const float* dL_dout_normal,
                            const float* dL_dout_median_depth,
                            const float* dL_dout_distortion,
                            float* dL_dtransMat, float* dL_dmean2D,
                            float* dL_dnormal3D, float* dL_dopacity,
                            float* dL_dcolors);

/* project_and_sh_backward_2dgs_kernel (metal:2003-2209). dL_dmean2D is
 * overwritten with the densify proxy; the three stats are updated in place. */
void orc_project_backward(int n, const float* means, const float* scales,
                          float glob_scale, const float* quats,
                          const OrcCamera* cam, const int32_t* radii,
                          const float* dL_dtransMat, const float* dL_dnormal3D,
                          const float* dL_dcolors, int degree, int degrees_to_use,
                          const float* f_rest, float* dL_dmean3D, float* dL_dscale,
                          float* dL_dquat, float* dL_dmean2D, float* dL_dfeatures_dc,
                          float* dL_dfeatures_rest, float* xys_grad_norm,
                          float* vis_counts, float* max_2d_size, float inv_max_dim);

/* fused_adam_kernel (metal:1383-1406). */
void orc_fused_adam(float* params, const float* grads, float* exp_avg,
                    float* exp_avg_sq, int64_t n, float step_size, float beta1,
                    float beta2, float bc2_sqrt, float eps);

/* One full training step: msplat_train_step_2dgs (msplat_metal.mm:935-1331)
 * followed by the six Adam groups of Model::fullIteration (model.cpp:762-829).
 * Parameters and Adam moments are updated in place. grads_out (optional,
 * may be NULL) receives the per-group gradients concatenated in group order
 * (means, scales, quats, f_dc, f_rest, opacities) = 13N + 3KN floats.
 * out_img_out (optional) receives the rendered image. Returns the loss. */
typedef struct {
    int n, degree, degrees_to_use;
    float* means; float* scales; float* quats; float* f_dc; float* f_rest;
    float* opacities;
    float* exp_avg[6]; float* exp_avg_sq[6];
    float* xys_grad_norm; float* vis_counts; float* max_2d_size;
    const float* background; const float* gt;
    float lr[6]; int adam_step; /* step count after increment (>= 1) */
    float lambda_l1, lambda_dist, lambda_dssim;
} OrcStepArgs;

float orc_train_step(const OrcStepArgs* a, const OrcCamera* cam, float* grads_out,
                     float* out_img_out, int64_t* kept_out);

/* Render-only forward (forward_pipeline, msplat_metal.mm:545-754). */
void orc_render(int n, const float* means, const float* scales, const float* quats,
                const float* opacities, const float* f_dc, const float* f_rest,
                int degree, int degrees_to_use, const float* background,
                const OrcCamera* cam, float* out_img);

/* orc_render restricted to pixel rows [0, pixel_rows) (the other rows are
 * left at zero): the target band of orc_time_step_sample's loss. */
void orc_render_rows(int n, const float* means, const float* scales, const float* quats, const float* opacities,
                     const float* f_dc, const float* f_rest, int degree, int degrees_to_use,
                     const float* background, const OrcCamera* cam, int pixel_rows, float* out_img);

/* Times one training step on a bounded sample of the workload, for the CPU
 * baseline: projection, binning, projection VJP and Adam on all N Gaussians;
 * rasterisation forward/backward on every tile_row_stride-th row of tiles and
 * the loss on pixel rows [0, H / tile_row_stride), both scaled back by
 * the stride. Parameters are updated in place (values are not checked).
 * Returns the estimated seconds of one full step; stage_seconds[7] receives
 * project, bin+sort+pack, raster fwd, loss, raster bwd, projection VJP, Adam. */
double orc_time_step_sample(const OrcStepArgs* a, const OrcCamera* cam, int tile_row_stride,
                            double* stage_seconds);

/* Densification as the reference stages it (msplat_densify,
 * core/metal/msplat_metal.mm:1339-1594; kernels core/metal/msplat_metal.metal:
 * 3231-3491): classify, append split children at [n + 2 o, n + 2 o + 1],
 * shrink split parents, append duplicates at [n + 2 S + d], cull-classify the
 * grown set, compact. The buffers hold `cap` >= 3n rows (params[6], m[6],
 * v[6] in Model group order, rows of 3, 2, 4, 3, 3K, 1 floats); stats are
 * xys_grad_norm, vis_counts, max_2d_size [n]; random_samples [2n, 3]. One
 * deliberate difference: the compaction moves scales rows of 2 floats (the
 * reference's stride table says 3, msplat_metal.mm:1365, 1377). Returns the
 * new count; *num_splits and *num_dups receive the growth counts. */
typedef struct OrcDensifyArgs {
    float grad_thresh, size_thresh, screen_thresh;
    int check_screen;
    float cull_alpha_thresh, cull_scale_thresh, cull_screen_size;
    int check_huge;
    float half_max_dim, log_size_fac;
} OrcDensifyArgs;
int orc_densify(int n, int cap, int rest_bases, const OrcDensifyArgs* a, const float* xys_grad_norm,
                const float* vis_counts, const float* max_2d_size, float* const params[6], float* const m[6],
                float* const v[6], const float* random_samples, int* num_splits, int* num_dups);

/* The split samples of Model::afterTrain (model.cpp:254-259): `count` draws
 * of std::normal_distribution<float>(0, 1) from std::mt19937(seed). */
void orc_normal_samples(uint32_t seed, int64_t count, float* out);

/* Threads the oracle may use (OpenMP); <= 0 means all. Returns the count. */
int orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
