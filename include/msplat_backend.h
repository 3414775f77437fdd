/*
 * msplat_backend.h — C ABI of the B200 (sm_100a) training-step backend.
 *
 * Drop-in for the reference's backend boundary core/metal/bindings.h, whose
 * functions take MTensor (a Metal buffer plus shape). Here every tensor is a
 * plain CUDA device pointer with the reference's layout and the functions are
 * extern "C", so cgo/JNI/ctypes/Swift-C callers can bind them directly:
 *
 *   means [N,3]  scales [N,2] (log)  quats [N,4]  opacities [N] (logit)
 *   features_dc [N,3]  features_rest [N,K,3] (K = (degree+1)^2 - 1)
 *   images [H,W,3] float32, row-major; tiles are 16x16.
 *
 * Errors: every entry point returns MSPLAT_OK (0) or an error code and never
 * throws across the boundary; msplat_last_error() describes the last failure
 * of the calling thread. The reference prints to stderr and asserts instead
 * (core/metal/msplat_metal.mm:215-220, 560-575).
 *
 * Threading: one workspace per CUDA device, reused across calls and grown on
 * demand (the reference's FusedTensorCache, msplat_metal.mm:353-537). Calls on
 * the same device must not overlap; tensors returned by msplat_last_tensor
 * alias the workspace and are invalidated by the next call, as the reference's
 * msplat_last_* accessors are.
 */
#ifndef MSPLAT_BACKEND_H
#define MSPLAT_BACKEND_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MSPLAT_OK = 0,
    MSPLAT_ERR_ARGUMENT = 1,   /* bad pointer, size or degree */
    MSPLAT_ERR_CUDA = 2,       /* a CUDA runtime call failed */
    MSPLAT_ERR_CAPACITY = 3,   /* an intersection buffer could not be sized */
    MSPLAT_ERR_NONFINITE = 4   /* the loss came out NaN or infinite */
};

/* Status flags raised by the last step (msplat_last_status_flags). */
#define MSPLAT_FLAG_TILE_OVERFLOW 0x1u /* some tile had > 2048 intersections; the 2048 lowest ids were kept */

/* Camera prepared by the host (Model::prepareCam, core/src/model.cpp:500-544). */
typedef struct MsplatCamera {
    float viewmat[16]; /* row-major world -> camera */
    float projmat[16]; /* row-major world -> clip */
    float fx, fy, cx, cy;
    int32_t width, height;
    float cam_pos[3];
} MsplatCamera;

/* Gaussian parameters, device pointers in the reference layout. */
typedef struct MsplatGaussians {
    int32_t num_points; /* 0 .. 2^25 (MSPLAT_ERR_ARGUMENT above) */
    int32_t sh_degree; /* degree of the stored coefficients, 0..3 */
    float* means;
    float* scales;
    float* quats;
    float* opacities;
    float* features_dc;
    float* features_rest; /* may be NULL when sh_degree == 0 */
} MsplatGaussians;

/* Adam state for the six groups in Model order (means, scales, quats,
 * features_dc, features_rest, opacities): model.hpp:117-123. */
typedef struct MsplatAdamState {
    float* exp_avg[6];
    float* exp_avg_sq[6];
    float lr[6];
    int32_t step; /* step count AFTER this update (>= 1) */
    float beta1, beta2, eps;
} MsplatAdamState;

/* Reference-shaped tensor view returned by msplat_last_tensor. dtype: 0 f32,
 * 1 i32, 2 i64, 3 f64. */
typedef struct MsplatTensorRef {
    void* data;
    int64_t shape[4];
    int32_t ndim;
    int32_t dtype;
} MsplatTensorRef;

/* Model::prepareCam (core/src/model.cpp:500-544) for downscale factor 1: view
 * matrix from an OpenGL camToWorld (row-major 4x4) with the y/z flip,
 * perspective with znear 0.001 / zfar 1000 from the intrinsics, camera
 * position. Host-only; returns MSPLAT_ERR_ARGUMENT on bad input. */
int msplat_prepare_camera(const float camToWorld[16], float fx, float fy, float cx, float cy, int32_t width,
                          int32_t height, MsplatCamera* out);

/* Model::schedulersStep (core/src/model.cpp:183-186): log-linear means
 * learning rate at `step` of `max_steps`. */
float msplat_means_lr(int32_t step, int32_t max_steps, float lr_init, float lr_final);

/* Replaces msplat_render (core/metal/bindings.h:139-148, impl
 * msplat_metal.mm:545-772): projection, binning, sort and forward
 * rasterisation. The image and side outputs stay in the workspace
 * (msplat_last_tensor "out_img", "out_depth", ...); when out_img is non-NULL
 * the image is also copied there (device pointer). background is a host
 * float[3]. Asynchronous on `stream` apart from one small read of the
 * intersection count. */
int msplat_render(const MsplatGaussians* g, const MsplatCamera* cam, float glob_scale, float clip_thresh,
                  int32_t degrees_to_use, const float background[3], float* out_img, void* stream);

/* Replaces msplat_train_step_2dgs (core/metal/bindings.h:48-60, impl
 * msplat_metal.mm:935-1331): forward, L1 + DSSIM (+ distortion) loss,
 * backward. Per-Gaussian gradients are left in the workspace (names
 * "dL_dmean3D", "dL_dscale", "dL_dquat", "dL_dopacity", "dL_dfeatures_dc",
 * "dL_dfeatures_rest", "dL_dmean2D", "dL_dtransMat", "dL_dnormal3D",
 * "dL_dcolors"), the densify statistics are updated in place, and the loss is
 * returned in *loss after synchronising the stream (as the reference does).
 * gt is a device [H,W,3] image. */
int msplat_train_step_2dgs(const MsplatGaussians* g, const MsplatCamera* cam, float glob_scale,
                           float clip_thresh, int32_t degrees_to_use, const float background[3], const float* gt,
                           float lambda_l1, float lambda_dist, float lambda_dssim, float* xys_grad_norm,
                           float* vis_counts, float* max_2d_size, float inv_max_dim, float* loss, void* stream);

/* Replaces msplat_fused_adam (core/metal/bindings.h:100-105, impl
 * msplat_metal.mm:884-906): one Adam step on one flat group. Asynchronous. */
int msplat_fused_adam(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, uint32_t n,
                      float step_size, float beta1, float beta2, float bc2_sqrt, float eps, void* stream);

/* Model::fullIteration (core/src/model.cpp:762-829) as one device pipeline:
 * forward, loss, backward and Adam on all six groups, with the gradients kept
 * in registers between the projection VJP and the optimiser. Parameters and
 * moments are updated in place. The loss is written to loss_dev (a device
 * float) and the call does not wait for the GPU beyond one small read of the
 * intersection count. write_grads != 0 additionally materialises the
 * reference-shaped gradients in the workspace. With lambda_dist == 0 and
 * write_grads == 0 the forward computes only what the step reads (the
 * image, the final transmittance and the last contributor): the depth,
 * normal, alpha, median-depth and distortion outputs, final_Ts channels 1-2
 * and final_idx channel 1 are not produced (msplat_last_tensor reports them
 * as not produced by the last call). */
int msplat_train_step_fused(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                            const float background[3], const float* gt, float lambda_l1, float lambda_dist,
                            float lambda_dssim, const MsplatAdamState* adam, float* xys_grad_norm,
                            float* vis_counts, float* max_2d_size, float* loss_dev, int32_t write_grads,
                            void* stream);

/* Tile-sharded pieces of the step for multi-GPU runs (one process per GPU).
 * Part 1 projects all N Gaussians, bins and rasterises a band of tile rows
 * plus a one-tile-row halo (the SSIM window's reach), evaluates the loss on
 * the band's own rows and rasterises the backward there. With world > 0 the
 * band is chosen by the library: band `rank` of `world` contiguous bands of
 * about equal work (kept tile intersections), identical on every rank because
 * every rank projects the same Gaussians; the chosen [begin, end) is written
 * to tile_rows. With world <= 0, tile_rows[0..1] gives the band. It leaves the
 * raster-space gradient records [N,16] in raster_grads_out (device, zeroed by
 * the call) and the three loss partial sums (l1, ssim, distortion) in
 * loss_parts_dev (device double[3], may be NULL). After the caller sums the
 * records across ranks (reduce-scatter), part 2 runs the projection VJP and
 * Adam on Gaussians [g_begin, g_end); raster_grads must address the record of
 * Gaussian i at raster_grads + 16 * i for i in that range. */
int msplat_shard_forward_backward(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                  const float background[3], const float* gt, float lambda_l1, float lambda_dist,
                                  float lambda_dssim, int32_t world, int32_t rank, int32_t* tile_rows,
                                  float* raster_grads_out, double* loss_parts_dev, void* stream);
/* msplat_shard_forward_backward with the projection split around binning:
 * with split_color != 0 the geometry (homography, tile rectangles, depth,
 * opacity) is projected first and the SH colour only after the tile lists
 * are sorted, after `stream` has waited for features_ready (a cudaEvent_t,
 * may be NULL). A caller can therefore still be gathering features_dc and
 * features_rest from the other ranks when it makes this call; only means,
 * scales, quats and opacities must be in place. Same results as
 * msplat_shard_forward_backward. */
int msplat_shard_forward_backward_after(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                        const float background[3], const float* gt, float lambda_l1,
                                        float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                        int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                        void* features_ready, int32_t split_color, void* stream);
/* Peer colour access (one process per GPU on one node). Each rank keeps the
 * six parameter groups as [padded, w] device buffers indexed by the global
 * Gaussian id and owns rows [rank * chunk, (rank + 1) * chunk), which only it
 * updates (msplat_shard_project_backward_adam). The caller all-gathers the
 * geometry groups (means, scales, quats, opacities: 10 floats per Gaussian),
 * which every rank's projection needs for every Gaussian; the colour groups
 * (features_dc, features_rest: 48 floats) are not gathered: every rank maps
 * the other ranks' buffers (CUDA IPC) and, after binning, reads the colour
 * of just the Gaussians whose tile rectangle meets its band from their owner
 * over NVLink (plain loads, no multicast). Ordering across ranks comes from
 * the collectives of the step: the owners' Adam updates are complete before
 * any collective the caller issues after them (the geometry all-gather, the
 * loss all-reduce), and no owner updates again before every rank has joined
 * the next reduce-scatter. base[0..2] and base[5] are not read. */
#define MSPLAT_MAX_PEER_RANKS 16
typedef struct MsplatPeerParams {
    int32_t world;  /* ranks, 2..MSPLAT_MAX_PEER_RANKS */
    int32_t chunk;  /* Gaussians owned per rank */
    const float* base[6][MSPLAT_MAX_PEER_RANKS]; /* [group][rank]: that rank's buffer, mapped here (Model group order) */
} MsplatPeerParams;

/* Device buffers that can be shared with other processes: cudaMalloc'd and
 * zeroed (msplat_device_alloc), their IPC handle (64 bytes), a peer buffer
 * opened from a handle, and the matching release calls. */
int msplat_device_alloc(uint64_t bytes, void** ptr);
int msplat_device_free(void* ptr);
int msplat_ipc_handle(void* ptr, uint8_t handle[64]);
int msplat_ipc_open(const uint8_t handle[64], void** ptr);
int msplat_ipc_close(void* ptr);

/* msplat_shard_forward_backward with the colour coefficients read through
 * `peers` (Gaussian i from rank i / peers->chunk) and the geometry from g
 * (this rank's gathered buffers). */
int msplat_shard_forward_backward_peers(const MsplatGaussians* g, const MsplatPeerParams* peers,
                                        const MsplatCamera* cam, int32_t degrees_to_use,
                                        const float background[3], const float* gt, float lambda_l1,
                                        float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                        int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                        void* stream);
int msplat_shard_project_backward_adam(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                       const float* raster_grads, int32_t g_begin, int32_t g_end,
                                       const MsplatAdamState* adam, float* xys_grad_norm, float* vis_counts,
                                       float* max_2d_size, void* stream);

/* Routed multi-GPU exchange (one process per GPU; no counterpart in the
 * reference, which runs on one GPU). Rank r owns Gaussians [g_begin, g_end)
 * (parameters and Adam state, updated only by it; the rest of its parameter
 * buffers is never read) and one band of tile rows. A step, with the
 * caller's collectives in brackets:
 *   msplat_route_project   projection of the own slice; the slice's
 *                          summary (int32 [msplat_route_summary_len]): its
 *                          per-tile intersection counts, then the number of
 *                          its Gaussians whose tile rectangle starts at row
 *                          y, then those whose rectangle ends at row y
 *                          (y in [0, tiles_y])
 *   [all-gather the summaries, rank order]
 *   msplat_route_plan      the bands of all ranks and how many Gaussians
 *                          each rank sends to each rank (identical on every
 *                          rank): a Gaussian goes to every rank whose band
 *                          plus a one-tile-row halo its tile rectangle meets
 *   msplat_route_pack      128 bytes per (Gaussian, destination), grouped by
 *                          destination rank, increasing id within a group
 *   [all-to-all of the payloads, sources in rank order]
 *   msplat_route_band      binning, sort, forward rasteriser, loss and
 *                          backward over the received Gaussians for the
 *                          rank's band; raster-gradient records [recv, 16]
 *                          and the band's loss partial sums (l1, ssim, dist)
 *   [all-to-all of the records back; all-reduce of the loss sums]
 *   msplat_route_return    adds the returned records per own Gaussian
 *   msplat_route_project_backward_adam   projection VJP + Adam on the slice
 * Results equal the single-GPU step (same tile lists: the received set is in
 * increasing global id order). Per call state lives in the device workspace,
 * so one routed step runs at a time per device. */
int msplat_route_summary_len(const MsplatCamera* cam, int64_t* len_out);
int msplat_route_project(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use, int32_t g_begin,
                         int32_t g_end, int32_t* summary_out, void* stream);
/* summaries: device int32 [world][summary length], every rank's summary;
 * bands_out: host int32 [world + 1] (band of rank r: [bands[r], bands[r+1]));
 * send_counts_out / recv_counts_out: host int64 [world], the items this rank
 * sends to / receives from each rank. Waits for the stream; fails if this
 * slice's destinations disagree with the counts derived from the summaries. */
int msplat_route_plan(const int32_t* summaries, const MsplatCamera* cam, int32_t world, int32_t rank,
                      int32_t* bands_out, int64_t* send_counts_out, int64_t* recv_counts_out, void* stream);
/* send_payload: device buffer of sum(send_counts) x 128 bytes. */
int msplat_route_pack(void* send_payload, void* stream);
/* The routed exchange without collectives for the payloads: every rank's
 * inbox (the payloads it receives, sources in rank order) and return box
 * (the records of its own packed items, in packing order) are device
 * buffers that every rank maps (msplat_device_alloc + msplat_ipc_*). */
typedef struct MsplatRoutePeers {
    int32_t world, rank;      /* as in the last msplat_route_plan */
    int64_t inbox_items;      /* capacity of each inbox (128-byte items) */
    int64_t returnbox_items;  /* capacity of each return box (64-byte items) */
    void* inbox[MSPLAT_MAX_PEER_RANKS];     /* [rank]: that rank's inbox, mapped here */
    void* returnbox[MSPLAT_MAX_PEER_RANKS]; /* [rank]: that rank's return box, mapped here */
} MsplatRoutePeers;
/* msplat_route_pack writing each destination's group straight into that
 * rank's inbox (NVLink stores). Every rank must finish this call's kernel
 * before any rank reads its inbox (e.g. a one-element all-reduce on the
 * stream); then msplat_route_band reads inbox[rank], sum(recv_counts) items. */
int msplat_route_pack_peers(const MsplatRoutePeers* peers, void* stream);
/* The band's records ([sum(recv_counts), 16] from msplat_route_band) into
 * their owners' return boxes; after every rank's push (a one-element
 * all-reduce), msplat_route_return reads returnbox[rank], sum(send_counts)
 * items. */
int msplat_route_push_peers(const MsplatRoutePeers* peers, const float* raster_grads, void* stream);
/* recv_payload: num_recv x 128 bytes; raster_grads_out: device float
 * [num_recv, 16]; loss_parts_dev: device double [3]. */
int msplat_route_band(const MsplatCamera* cam, int32_t sh_degree, const void* recv_payload, int64_t num_recv,
                      int32_t band_begin, int32_t band_end, const float background[3], const float* gt,
                      float lambda_l1, float lambda_dist, float lambda_dssim, float* raster_grads_out,
                      double* loss_parts_dev, void* stream);
/* recv_grads: the records of this rank's packed items, returned in packing
 * order (sum(send_counts) x 16 floats); slice_grads: device float
 * [g_end - g_begin, 16] (overwritten). */
int msplat_route_return(const float* recv_grads, int64_t num_items, float* slice_grads, void* stream);
/* The projection VJP and Adam on the slice of the last msplat_route_project,
 * from slice_grads; densify statistics indexed by global id (may be NULL). */
int msplat_route_project_backward_adam(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                       const float* slice_grads, const MsplatAdamState* adam, float* xys_grad_norm,
                                       float* vis_counts, float* max_2d_size, void* stream);
/* Colour exchange by clamped colour instead of SH coefficients (no
 * reference counterpart; the colour evaluation is sh_coeffs_to_color,
 * core/metal/msplat_metal.metal:756-823, as in the projection). The colour a
 * Gaussian contributes to a step depends only on its own parameters and the
 * camera, so the owner of a slice, right after its Adam update, evaluates the
 * clamped colours max(SH + 0.5, 0) of its Gaussians [g_begin, g_end) for the
 * NEXT step's camera into rgb[3 i .. 3 i + 2] (msplat_shard_colors); the ranks
 * all-gather that [N, 3] buffer (12 B per Gaussian instead of 192 B of
 * coefficients at SH degree 3) and the next step copies it
 * (msplat_shard_forward_backward_rgb, after rgb_ready when non-null) where it
 * would evaluate the SH. The copied colours are bit-identical to the
 * evaluated ones. The colour coefficients then stay current only on their
 * owner: gather them before exporting or checkpointing. */
int msplat_shard_colors(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use, int32_t g_begin,
                        int32_t g_end, float* rgb, void* stream);
int msplat_shard_forward_backward_rgb(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                      const float background[3], const float* gt, float lambda_l1,
                                      float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                      int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                      const float* rgb, void* rgb_ready, void* stream);

/* Densification: replaces msplat_densify (core/metal/bindings.h:143-157, impl
 * core/metal/msplat_metal.mm:1339-1594, kernels core/metal/msplat_metal.metal:
 * 3231-3491) as driven by Model::afterTrain (core/src/model.cpp:240-306).
 * Same decisions: a Gaussian with vis_counts > 0 and average screen gradient
 * (xys_grad_norm / vis_counts) * half_max_dim > grad_thresh splits when its
 * largest scale exceeds size_thresh (or, with check_screen, its max_2d_size
 * exceeds screen_thresh), and is duplicated when its largest scale does not;
 * a split produces two children at parent + R(q) (n * scale, 0) with scales
 * shrunk by log_size_fac and zero moments, and the parent's own scale shrinks
 * too (a Gaussian that both splits and duplicates duplicates the shrunk
 * parent); duplicates copy the parent with zero moments. Then the grown set
 * [originals | children in split order | duplicates in duplicate order] is
 * culled: sigmoid(opacity) < cull_alpha_thresh, every split parent, and with
 * check_huge a largest scale above cull_scale_thresh or (originals, with
 * check_screen) max_2d_size above cull_screen_size; survivors keep their
 * order. The reference compacts the scales with a row stride of 3 although
 * 2DGS scales have 2 entries (msplat_metal.mm:1365, 1377), which scrambles
 * them; this build compacts every group with its true row size.
 * Two calls: msplat_densify_plan classifies on the device, reads back the
 * counts (synchronising `stream`) and keeps the per-Gaussian decisions in the
 * library's workspace; msplat_densify_apply then writes the new set into
 * caller-allocated arrays of plan->new_count rows (out, out_adam->exp_avg /
 * exp_avg_sq; other fields of out_adam are ignored). random_samples holds
 * 2 * num_splits * 3 standard normals (device): the values the reference
 * draws from std::mt19937(step) / std::normal_distribution<float> for split
 * ordinal o, child k at [(2 o + k) * 3, +3). Call apply right after plan with
 * the same g, adam and args; inputs are not modified. */
typedef struct MsplatDensifyArgs {
    float grad_thresh;         /* densifyGradThresh */
    float size_thresh;         /* densifySizeThresh */
    float screen_thresh;       /* splitScreenSize */
    int32_t check_screen;      /* step < stopScreenSizeAt */
    float cull_alpha_thresh;   /* 0.1 (model.cpp:270) */
    float cull_scale_thresh;   /* 0.5 */
    float cull_screen_size;    /* 0.15 */
    int32_t check_huge;        /* step > refineEvery * resetAlphaEvery */
    float half_max_dim;        /* 0.5 * max(width, height) of the last step */
    float log_size_fac;        /* log(1.6) */
    const float* xys_grad_norm; /* [N] device, accumulated by the steps */
    const float* vis_counts;    /* [N] device */
    const float* max_2d_size;   /* [N] device */
} MsplatDensifyArgs;

typedef struct MsplatDensifyPlan {
    int32_t num_splits;  /* Gaussians that split */
    int32_t num_dups;    /* Gaussians duplicated */
    int32_t new_count;   /* Gaussians after growth and culling */
} MsplatDensifyPlan;

int msplat_densify_plan(const MsplatGaussians* g, const MsplatDensifyArgs* args, MsplatDensifyPlan* plan,
                        void* stream);
int msplat_densify_apply(const MsplatGaussians* g, const MsplatAdamState* adam, const MsplatDensifyArgs* args,
                         const float* random_samples, const MsplatGaussians* out, const MsplatAdamState* out_adam,
                         void* stream);

/* The split samples of Model::afterTrain (core/src/model.cpp:254-259): the
 * first `count` draws of std::normal_distribution<float>(0, 1) from
 * std::mt19937(seed), written to host memory. Host-only. */
int msplat_normal_samples(uint32_t seed, int64_t count, float* out);

/* Opacity reset of Model::afterTrain (core/src/model.cpp:290-299): every
 * opacity logit above max_logit becomes max_logit, and the opacity group's
 * moments (n floats each, may be NULL) are zeroed. Asynchronous. */
int msplat_reset_opacity(float* opacities, float* exp_avg, float* exp_avg_sq, int32_t n, float max_logit,
                         void* stream);

/* Allocation-free L1 + DSSIM (+ distortion) loss, forward and backward. No
 * counterpart in the reference. For callers that may not allocate device
 * memory at run time (hosts whose GPU memory all comes from their own pool
 * allocator, or that fix their memory budget at start-up): it calls no
 * cudaMalloc/cudaFree and no allocating library routine. Its scratch lives in
 * fixed arrays inside the library's device image, about 192 KiB held by every
 * GPU that loads the library until the process exits. The scratch holds 8192
 * loss blocks; this entry point lays out at most that many (54-column strips,
 * fewer row segments per strip than the regular path for tall images), so it
 * accepts any height and widths up to 8192 x 54 = 442,368 pixels. Wider
 * images are rejected with MSPLAT_ERR_ARGUMENT. Inputs and outputs are
 * caller-owned device memory: out_img and gt [H,W,3], out_distortion [H,W]
 * (may be NULL when lambda_dist == 0), dL_dout_img [H,W,3] (written),
 * loss_out one float (written, may be NULL). A non-finite loss is not turned
 * into an error code on this path: it shows only as NaN or Inf in *loss_out.
 * The first call on a device looks up the scratch addresses; make that first
 * call before any stream capture. All calls share the scratch, so calls that
 * overlap on the GPU (other streams, other host threads) race; serialise
 * them. Asynchronous on `stream`. */
int msplat_loss_ssim_noalloc(const float* out_img, const float* gt, const float* out_distortion, int32_t width,
                             int32_t height, float lambda_l1, float lambda_dist, float lambda_dssim,
                             float* dL_dout_img, float* loss_out, void* stream);

/* Accessor for the workspace tensors of the last call (the msplat_last_*
 * family, core/metal/bindings.h:36-43, 107-131). Names: out_img, out_depth,
 * out_normal, out_alpha, out_median_depth, out_distortion, final_Ts,
 * final_idx, dL_dout_img, radii, depths, xys, transMats, normal_opacity,
 * colors, num_tiles_hit, tile_bins, gaussian_ids, raw_tile_counts, the
 * dL_d* gradients listed above, loss_partials (f64 [blocks,3]: l1, ssim,
 * distortion sums per loss block), loss_terms (f64 [4]: loss, ssim sum,
 * l1 term, distortion term), raster_counters (i64 [4]: blended
 * (pixel, surfel) pairs of the forward rasteriser, its (warp, surfel) visits
 * past the cull, the backward's (warp, surfel) visits and its blended pairs;
 * each visit evaluates 32 pixels; zeros unless msplat_set_raster_counters
 * enabled them) and intersection_totals (i64 [5]: emitted
 * keys, kept intersections, band begin and end, tiles with more than 512
 * keys). Returns MSPLAT_ERR_ARGUMENT for an unknown
 * name or a tensor the last call did not produce. */
int msplat_last_tensor(const char* name, MsplatTensorRef* out);

/* Number of kept tile intersections of the last call. */
int64_t msplat_last_num_intersections(void);
/* MSPLAT_FLAG_* bits raised by the last call. */
uint32_t msplat_last_status_flags(void);
/* Stage timing with CUDA events recorded on the launch stream at stage
 * boundaries (the reference's PROFILE_STAGES intent, msplat_metal.mm:84-129).
 * Enabling (or disabling) resets the totals. msplat_stage_times waits for the
 * recorded steps, writes the accumulated milliseconds and the number of
 * samples per stage, and returns the number of stages (or -1 on error). */
int msplat_set_stage_timing(int32_t enable);
int32_t msplat_stage_times(double* total_ms, int64_t* counts, int32_t max_stages);
/* Rasteriser work counters (off by default: the kernels are then launched
 * without the per-visit counting). While enabled, every forward/backward pair
 * leaves in msplat_last_tensor("raster_counters") (int64 [4]): forward
 * blended (pixel, surfel) pairs, forward (warp, surfel) visits past the cull,
 * backward visits, backward blended pairs. */
int msplat_set_raster_counters(int32_t enable);
const char* msplat_stage_name(int32_t i);
/* Kernel launches issued by this library since load (for launch accounting). */
int64_t msplat_launch_count(void);
/* Per-thread description of the last error ("" if none). */
const char* msplat_last_error(void);

/* msplat_commit / msplat_gpu_sync (core/metal/bindings.h:21-24). */
void msplat_commit(void);
void msplat_gpu_sync(void);
/* cleanup_msplat_metal (core/metal/bindings.h:8): frees every workspace. */
void msplat_backend_cleanup(void);

#ifdef __cplusplus
}
#endif
#endif
