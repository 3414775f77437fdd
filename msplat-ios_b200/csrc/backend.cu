// backend.cu — the C ABI of include/msplat_backend.h: per-device workspace,
// stage sequencing on one stream, reference-shaped accessors.
//
// Stage order of one training step (msplat_train_step_2dgs,
// core/metal/msplat_metal.mm:935-1331, plus Model::fullIteration's Adam loop,
// core/src/model.cpp:800-826):
//   project (+ tile difference array) -> tile counts/scans -> [read totals]
//   -> emit keys -> per-tile select/sort -> rasterise forward -> fused
//   L1+DSSIM loss fwd/bwd -> loss finalize -> rasterise backward ->
//   projection VJP (+ Adam on all groups).
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "msplat_backend.h"
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {

static std::atomic<int64_t> g_launches{0};
void note_launches(int k) { g_launches.fetch_add(k, std::memory_order_relaxed); }

namespace {
thread_local std::string t_last_error;
}  // namespace

void set_last_error(const std::string& msg) { t_last_error = msg; }

namespace {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(call)                                                                                    \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            throw Error(MSPLAT_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));       \
    } while (0)

// Device buffer that only grows.
struct Buf {
    void* p = nullptr;
    size_t cap = 0;
    void ensure(size_t bytes) {
        if (bytes <= cap) return;
        if (p) CK(cudaFree(p));
        p = nullptr;
        cap = 0;
        size_t want = bytes + bytes / 8 + 256;
        CK(cudaMalloc(&p, want));
        cap = want;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

struct Workspace {
    int device = -1;
    // per Gaussian
    Buf records, cull, rects, depths, radii, raster_grads;
    Buf xys, transmats, num_tiles_hit, normal_opacity, colors, aabb;
    Buf dL_dmean3D, dL_dscale, dL_dquat, dL_dmean2D, dL_dfeatures_dc, dL_dfeatures_rest, dL_dopacity;
    Buf dL_dtransMat, dL_dnormal3D, dL_dcolors;
    // per tile / intersection
    Buf tile_diff, chunk_counts, raw_true, id_limit, block_max, raw_counts, raw_start, tile_bins, fill, raw_keys, gaussian_ids,
        blend_mask;
    // per pixel
    Buf final_Ts, final_idx, out_img, out_depth, out_normal, out_alpha, out_median, out_dist, dL_dout_img;
    // scalars
    Buf loss_partials, loss_out, loss_f, err, totals, row_work, counters, big_tiles;
    // routed multi-GPU exchange (route.cu): the owner's projected slice, its
    // destinations and packing order, the received global ids
    Buf own_records, own_cull, own_rects, own_depths, own_radii, own_dest, route_diff, route_colsum, route_block,
        route_totals, route_base, route_bands, route_matrix, route_row_work, route_src, route_ids;
    // pinned: bands (int32 [17] in the first 9 slots), the slice's items per
    // rank [16], the count matrix [16 x 16]
    static constexpr int kHostRouteSlots = (kMaxPeerRanks + 2) / 2 + kMaxPeerRanks + kMaxPeerRanks * kMaxPeerRanks;
    int64_t* h_route = nullptr;
    int route_n = 0, route_g0 = 0, route_world = 0, route_rank = 0;
    std::vector<int64_t> route_matrix_h;  // the last plan's count matrix [world x world]
    int64_t route_items = 0;
    int64_t* h_totals = nullptr;  // pinned [5]: raw, kept, band begin, band end, large tiles
    uint32_t* h_err = nullptr;    // pinned [1]
    // shape bookkeeping of the last call
    int n = 0, K = 0, W = 0, H = 0, tx = 0, ty = 0;
    int64_t kept = 0;
    int64_t loss_blocks = 0;
    uint32_t flags = 0;
    bool flags_pending = false;       // err word not yet read back
    cudaStream_t last_stream = nullptr;
    // stage timing (msplat_set_stage_timing): per step, (stage id, event) at
    // each stage boundary; stage id -1 closes the step
    std::vector<std::vector<std::pair<int, cudaEvent_t>>> ev_pending;
    std::vector<cudaEvent_t> ev_pool;
    bool have_ref_proj = false, have_grads = false, have_pixels = false, have_dimg = false;
    // the last forward wrote every per-pixel output (not only the image, T and
    // the last contributor that a colour-only training step reads)
    bool have_aux = false;

    void release_all() {
        Buf* all[] = {&records, &cull, &rects, &depths, &radii, &raster_grads, &xys, &transmats, &num_tiles_hit,
                      &normal_opacity, &colors, &aabb, &dL_dmean3D, &dL_dscale, &dL_dquat, &dL_dmean2D,
                      &dL_dfeatures_dc, &dL_dfeatures_rest, &dL_dopacity, &dL_dtransMat, &dL_dnormal3D,
                      &dL_dcolors, &tile_diff, &chunk_counts, &raw_true, &id_limit, &block_max, &raw_counts, &raw_start, &tile_bins, &fill, &raw_keys,
                      &gaussian_ids, &blend_mask, &final_Ts, &final_idx, &out_img, &out_depth, &out_normal, &out_alpha,
                      &out_median, &out_dist, &dL_dout_img, &loss_partials, &loss_out, &loss_f, &err, &totals, &row_work, &counters, &big_tiles, &own_records, &own_cull, &own_rects, &own_depths,
                      &own_radii, &own_dest, &route_diff, &route_colsum, &route_block, &route_totals, &route_base,
                      &route_bands, &route_matrix, &route_row_work, &route_src, &route_ids};
        for (Buf* b : all) b->release();
        for (auto& set : ev_pending)
            for (auto& m : set) cudaEventDestroy(m.second);
        for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
        ev_pending.clear();
        ev_pool.clear();
        if (h_totals) cudaFreeHost(h_totals);
        if (h_route) cudaFreeHost(h_route);
        h_route = nullptr;
        if (h_err) cudaFreeHost(h_err);
        h_totals = nullptr;
        h_err = nullptr;
    }
};

std::mutex g_ws_mu;
std::vector<Workspace*> g_ws;

// Stage timing: CUDA events recorded on the launch stream at stage
// boundaries, read back only when msplat_stage_times() is called.
enum Stage { kStProject = 0, kStCounts, kStEmit, kStSort, kStRasterFwd, kStLoss, kStRasterBwd, kStProjectBwd,
             kStBetweenShardCalls, kStColor, kStRouteExchange, kStRouteUnpack, kNumStages };
// between_shard_calls: from the end of msplat_shard_forward_backward to the
// start of msplat_shard_project_backward_adam on the stream (the caller's
// reduce-scatter and any wait for slower ranks)
const char* kStageNames[kNumStages] = {"project_forward", "tile_counts", "emit_keys", "tile_sort",
                                       "rasterize_forward", "loss_ssim", "rasterize_backward",
                                       "project_backward_adam", "between_shard_calls",
                                       "project_color",   // colour pass of a split projection, incl. its wait
                                       // routed exchange: the slice summary, the plan and the payload
                                       // dispatch (from the end of the slice's projection to the band's
                                       // start, incl. the caller's collectives), then the unpack
                                       "route_exchange", "route_unpack"};
bool g_timing = false;
// rasteriser work counters (msplat_set_raster_counters): off, the kernels are
// built without the per-visit counting
bool g_counting = false;
double g_stage_ms[kNumStages] = {};
int64_t g_stage_n[kNumStages] = {};

Workspace& workspace() {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(g_ws_mu);
    if ((int)g_ws.size() <= dev) g_ws.resize(dev + 1, nullptr);
    if (!g_ws[dev]) {
        g_ws[dev] = new Workspace();
        g_ws[dev]->device = dev;
    }
    Workspace& w = *g_ws[dev];
    if (!w.h_totals) {
        CK(cudaHostAlloc(reinterpret_cast<void**>(&w.h_totals), 5 * sizeof(int64_t), cudaHostAllocDefault));
        CK(cudaHostAlloc(reinterpret_cast<void**>(&w.h_err), sizeof(uint32_t), cudaHostAllocDefault));
        CK(cudaHostAlloc(reinterpret_cast<void**>(&w.h_route), Workspace::kHostRouteSlots * sizeof(int64_t),
                         cudaHostAllocDefault));
    }
    return w;
}

cudaEvent_t take_event(Workspace& w) {
    if (!w.ev_pool.empty()) {
        cudaEvent_t e = w.ev_pool.back();
        w.ev_pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    return e;
}

// Marks the start of `stage` (stage -1 marks the end of the step).
void mark(Workspace& w, int stage, cudaStream_t s) {
    if (!g_timing) return;
    if (stage == kStProject) w.ev_pending.emplace_back();
    if (w.ev_pending.empty()) return;
    cudaEvent_t e = take_event(w);
    CK(cudaEventRecord(e, s));
    w.ev_pending.back().emplace_back(stage, e);
}

// Waits for every recorded step and adds its stage durations.
void flush_timing(Workspace& w) {
    for (auto& set : w.ev_pending) {
        if (set.size() >= 2) {
            CK(cudaEventSynchronize(set.back().second));
            for (size_t k = 0; k + 1 < set.size(); ++k) {
                const int st = set[k].first;
                if (st < 0 || st >= kNumStages) continue;
                float ms = 0.f;
                CK(cudaEventElapsedTime(&ms, set[k].second, set[k + 1].second));
                g_stage_ms[st] += ms;
                g_stage_n[st] += 1;
            }
        }
        for (auto& m : set) w.ev_pool.push_back(m.second);
    }
    w.ev_pending.clear();
}

int sh_rest_bases(int degree) { return (degree + 1) * (degree + 1) - 1; }

void check_inputs(const MsplatGaussians* g, const MsplatCamera* cam, int degrees_to_use) {
    if (!g || !cam) throw Error(MSPLAT_ERR_ARGUMENT, "null gaussians or camera");
    // ids take 25 bits at most (the overfull-tile select reads 32-bit ids in
    // three digits; per-Gaussian int offsets stay below 2^31 up to 2^25)
    if (g->num_points < 0 || g->num_points > (1 << 25))
        throw Error(MSPLAT_ERR_ARGUMENT, "num_points must be in [0, 2^25]");
    if (g->sh_degree < 0 || g->sh_degree > 3) throw Error(MSPLAT_ERR_ARGUMENT, "sh_degree must be 0..3");
    if (degrees_to_use < 0 || degrees_to_use > g->sh_degree)
        throw Error(MSPLAT_ERR_ARGUMENT, "degrees_to_use must be in [0, sh_degree]");
    if (cam->width <= 0 || cam->height <= 0 || cam->width > 65535 * 16 || cam->height > 65535 * 16)
        throw Error(MSPLAT_ERR_ARGUMENT, "bad image size");
    if (g->num_points > 0 && (!g->means || !g->scales || !g->quats || !g->opacities || !g->features_dc))
        throw Error(MSPLAT_ERR_ARGUMENT, "null parameter pointer");
    if (g->sh_degree > 0 && g->num_points > 0 && !g->features_rest)
        throw Error(MSPLAT_ERR_ARGUMENT, "features_rest is null for sh_degree > 0");
}

CameraDev make_cam(const MsplatCamera* c) {
    CameraDev d;
    std::memcpy(d.viewmat, c->viewmat, sizeof(d.viewmat));
    std::memcpy(d.projmat, c->projmat, sizeof(d.projmat));
    d.fx = c->fx; d.fy = c->fy; d.cx = c->cx; d.cy = c->cy;
    d.width = c->width; d.height = c->height;
    d.tiles_x = (c->width + kTile - 1) / kTile;
    d.tiles_y = (c->height + kTile - 1) / kTile;
    d.cam_pos[0] = c->cam_pos[0]; d.cam_pos[1] = c->cam_pos[1]; d.cam_pos[2] = c->cam_pos[2];
    return d;
}

// Projection, binning, sort and forward rasterisation of tile rows
// [row0, row1). When balance_world > 0 the rows are chosen here instead:
// band balance_rank of balance_world work-balanced bands, returned in
// *owned0/*owned1, rendered with a one-tile-row halo.
void stage_forward(Workspace& w, const MsplatGaussians* g, const CameraDev& cam, int degrees_to_use,
                   float glob_scale, float clip, const float bg[3], bool ref_outputs, int row0, int row1,
                   cudaStream_t s, int balance_world = 0, int balance_rank = 0, int* owned0 = nullptr,
                   int* owned1 = nullptr, bool split_color = false, cudaEvent_t features_ready = nullptr,
                   const MsplatPeerParams* peers = nullptr, const float* rgb_in = nullptr,
                   bool aux_out = true, bool prefilled = false) {
    const int n = g->num_points;
    const int K = sh_rest_bases(g->sh_degree);
    const int tx = cam.tiles_x, ty = cam.tiles_y, T = tx * ty;
    const size_t P = (size_t)cam.width * cam.height;
    w.n = n; w.K = K; w.W = cam.width; w.H = cam.height; w.tx = tx; w.ty = ty;
    w.flags = 0;
    w.have_ref_proj = ref_outputs;
    w.have_aux = aux_out;
    w.have_grads = false;
    w.have_dimg = false;
    const size_t nn = (size_t)(n > 0 ? n : 1);
    w.records.ensure(nn * kRecordF4 * sizeof(float4));
    w.cull.ensure(nn * kCullF4 * sizeof(float4));
    w.rects.ensure(nn * sizeof(uint2));
    w.depths.ensure(nn * sizeof(float));
    w.radii.ensure(nn * sizeof(int32_t));
    if (ref_outputs) {
        w.xys.ensure(nn * 2 * 4); w.transmats.ensure(nn * 9 * 4); w.num_tiles_hit.ensure(nn * 4);
        w.normal_opacity.ensure(nn * 4 * 4); w.colors.ensure(nn * 3 * 4); w.aabb.ensure(nn * 2 * 4);
    }
    const size_t diff_bytes = (size_t)kIdChunks * (tx + 1) * (ty + 1) * 4;
    w.tile_diff.ensure(diff_bytes);
    w.chunk_counts.ensure((size_t)kIdChunks * T * 4);
    w.raw_true.ensure((size_t)T * 4);
    w.id_limit.ensure((size_t)T * 4);
    const size_t bmax_bytes =
        (size_t)((tx + kLimitBlock - 1) / kLimitBlock) * ((ty + kLimitBlock - 1) / kLimitBlock) * 4;
    w.block_max.ensure(bmax_bytes);
    w.raw_counts.ensure((size_t)T * 4);
    w.raw_start.ensure((size_t)T * 8);
    w.tile_bins.ensure((size_t)T * sizeof(int2));
    w.fill.ensure((size_t)T * 8);
    w.totals.ensure(5 * sizeof(int64_t));
    w.big_tiles.ensure((size_t)T * sizeof(int32_t));
    w.err.ensure(sizeof(uint32_t));
    w.final_Ts.ensure(P * 3 * 4); w.final_idx.ensure(P * 2 * 4); w.out_img.ensure(P * 3 * 4);
    w.out_depth.ensure(P * 4); w.out_normal.ensure(P * 3 * 4); w.out_alpha.ensure(P * 4);
    w.out_median.ensure(P * 4); w.out_dist.ensure(P * 4);

    // prefilled: the records, cull records, rectangles, depths and the
    // per-id-chunk difference arrays already hold n Gaussians (the routed
    // exchange's received set), so the projection is skipped
    if (!prefilled) CK(cudaMemsetAsync(w.tile_diff.p, 0, diff_bytes, s));
    CK(cudaMemsetAsync(w.block_max.p, 0, bmax_bytes, s));
    CK(cudaMemsetAsync(w.err.p, 0, sizeof(uint32_t), s));

    ProjFwdArgs pa{};
    pa.n = n;
    pa.pass = split_color ? 1 : 0;
    if (peers) {
        // colour from the owners' buffers, after binning, for this band only
        split_color = true;
        pa.pass = 1;
    }
    pa.means = g->means; pa.scales = g->scales; pa.quats = g->quats; pa.opacities = g->opacities;
    pa.f_dc = g->features_dc; pa.f_rest = g->features_rest;
    pa.rest_bases = K; pa.degrees_to_use = degrees_to_use;
    pa.glob_scale = glob_scale; pa.clip_thresh = clip;
    pa.cam = cam;
    pa.records = w.records.as<float4>(); pa.cull = w.cull.as<float4>(); pa.rects = w.rects.as<uint2>(); pa.depths = w.depths.as<float>();
    pa.radii = w.radii.as<int32_t>(); pa.tile_diff = w.tile_diff.as<int32_t>();
    const int id_chunk = std::max(1, (n + kIdChunks - 1) / kIdChunks);
    pa.id_chunk = id_chunk;
    if (ref_outputs) {
        pa.xys = w.xys.as<float>(); pa.transmats = w.transmats.as<float>();
        pa.num_tiles_hit = w.num_tiles_hit.as<int32_t>(); pa.normal_opacity = w.normal_opacity.as<float>();
        pa.colors = w.colors.as<float>(); pa.aabb = w.aabb.as<float>();
    }
    // a prefilled (routed) band was projected by the owners: no projection
    // stage here, the caller marked its unpack
    if (!prefilled) {
        mark(w, kStProject, s);
        launch_project_forward(pa, s);
    }
    mark(w, kStCounts, s);
    if (balance_world > 0) w.row_work.ensure((size_t)ty * sizeof(int64_t));
    launch_tile_counts(w.tile_diff.as<int32_t>(), id_chunk, w.chunk_counts.as<int32_t>(), w.raw_true.as<int32_t>(),
                       w.id_limit.as<int32_t>(), w.block_max.as<int32_t>(), tx, ty, row0, row1, w.raw_counts.as<int32_t>(),
                       w.raw_start.as<int64_t>(), w.fill.as<uint64_t>(), w.tile_bins.as<int2>(), w.totals.as<int64_t>(),
                       balance_world > 0 ? w.row_work.as<int64_t>() : nullptr, w.err.as<uint32_t>(), s, balance_world,
                       balance_rank, w.big_tiles.as<int32_t>());
    // The one host read of the step: buffer sizes for the intersections (and
    // the band the kernel chose, when balancing).
    CK(cudaMemcpyAsync(w.h_totals, w.totals.p, 5 * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (balance_world > 0) {
        const int o0 = (int)w.h_totals[2], o1 = (int)w.h_totals[3];
        if (o0 < 0 || o1 > ty || o0 > o1) throw Error(MSPLAT_ERR_CAPACITY, "corrupt band");
        if (owned0) *owned0 = o0;
        if (owned1) *owned1 = o1;
        row0 = o1 > o0 ? std::max(0, o0 - 1) : 0;
        row1 = o1 > o0 ? std::min(ty, o1 + 1) : 0;
    }
    const int64_t raw_total = w.h_totals[0], kept = w.h_totals[1], num_big = w.h_totals[4];
    if (raw_total < 0 || kept < 0 || kept > raw_total || num_big < 0 || num_big > T)
        throw Error(MSPLAT_ERR_CAPACITY, "corrupt tile totals");
    w.kept = kept;
    w.raw_keys.ensure((size_t)(raw_total > 0 ? raw_total : 1) * sizeof(uint64_t));
    w.gaussian_ids.ensure((size_t)(kept > 0 ? kept : 1) * sizeof(int32_t));
    w.blend_mask.ensure((size_t)(kept > 0 ? kept : 1));
    mark(w, kStEmit, s);
    launch_emit_keys(n, w.rects.as<uint2>(), w.depths.as<float>(), tx, row0, row1, w.id_limit.as<int32_t>(),
                     w.block_max.as<int32_t>(), w.fill.as<uint64_t>(), w.raw_keys.as<uint64_t>(), s);
    mark(w, kStSort, s);
    launch_tile_sort(row0 * tx, (row1 - row0) * tx, w.raw_counts.as<int32_t>(), w.raw_start.as<int64_t>(), w.raw_keys.as<uint64_t>(),
                     w.tile_bins.as<int2>(), w.gaussian_ids.as<int32_t>(), w.err.as<uint32_t>(), n,
                     w.big_tiles.as<int32_t>(), (int)num_big, s);
    if (split_color) {
        // colour after binning: the caller may still be gathering features_dc /
        // features_rest until features_ready
        mark(w, kStColor, s);
        if (features_ready) CK(cudaStreamWaitEvent(s, features_ready, 0));
        ProjFwdArgs pc = pa;
        pc.pass = 2;
        pc.color_row0 = row0;
        pc.color_row1 = row1;
        pc.rgb_in = rgb_in;
        if (peers) {
            pc.peer_world = peers->world;
            pc.peer_chunk = peers->chunk;
            for (int q = 0; q < peers->world; ++q) {
                pc.peer_dc[q] = peers->base[3][q];
                pc.peer_rest[q] = peers->base[4][q];
            }
        }
        launch_project_forward(pc, s);
    }
    RasterFwdArgs ra{};
    ra.width = cam.width; ra.height = cam.height; ra.tiles_x = tx; ra.tiles_y = ty;
    ra.tile_row_begin = row0; ra.tile_row_end = row1;
    ra.tile_bins = w.tile_bins.as<int2>(); ra.gaussian_ids = w.gaussian_ids.as<int32_t>();
    ra.records = w.records.as<float4>();
    ra.cull = w.cull.as<float4>();
    ra.bg[0] = bg[0]; ra.bg[1] = bg[1]; ra.bg[2] = bg[2];
    ra.final_Ts = w.final_Ts.as<float>(); ra.final_idx = w.final_idx.as<int32_t>(); ra.out_img = w.out_img.as<float>();
    ra.out_depth = w.out_depth.as<float>(); ra.out_normal = w.out_normal.as<float>();
    ra.out_alpha = w.out_alpha.as<float>(); ra.out_median_depth = w.out_median.as<float>();
    ra.out_distortion = w.out_dist.as<float>();
    ra.blend_mask = w.blend_mask.as<uint8_t>();
    w.counters.ensure(4 * sizeof(unsigned long long));
    CK(cudaMemsetAsync(w.counters.p, 0, 4 * sizeof(unsigned long long), s));
    ra.counters = g_counting ? w.counters.as<unsigned long long>() : nullptr;
    ra.aux_outputs = aux_out ? 1 : 0;
    mark(w, kStRasterFwd, s);
    launch_rasterize_forward(ra, s);
    w.have_pixels = true;
    w.flags_pending = true;
    w.last_stream = s;
}

// Loss forward/backward over pixel rows [prow0, prow1); finalize into
// loss_out (double[4]) and loss_f (float).
void stage_loss(Workspace& w, const CameraDev& cam, const float* gt, float l1, float ldist, float ldssim, int prow0,
                int prow1, bool finalize, cudaStream_t s) {
    const size_t P = (size_t)cam.width * cam.height;
    w.dL_dout_img.ensure(P * 3 * 4);
    const int nb = loss_num_blocks(cam.width, prow0, prow1);
    w.loss_blocks = nb;
    w.loss_partials.ensure((size_t)(nb > 0 ? nb : 1) * 3 * sizeof(double));
    w.loss_out.ensure(4 * sizeof(double));
    w.loss_f.ensure(sizeof(float));
    LossArgs la{};
    la.width = cam.width; la.height = cam.height; la.row_begin = prow0; la.row_end = prow1;
    la.out_img = w.out_img.as<float>(); la.gt = gt; la.out_distortion = w.out_dist.as<float>();
    la.lambda_l1 = l1; la.lambda_dist = ldist; la.lambda_dssim = ldssim;
    la.inv_num = 1.0f / (float)((double)cam.height * (double)cam.width * 3.0);
    la.dL_dout_img = w.dL_dout_img.as<float>();
    la.partials = w.loss_partials.as<double>();
    mark(w, kStLoss, s);
    launch_loss_ssim(la, s);
    if (finalize)
        launch_loss_finalize(w.loss_partials.as<double>(), nb, ldssim, la.inv_num, w.loss_out.as<double>(),
                             w.loss_f.as<float>(), w.err.as<uint32_t>(), s);
    w.have_dimg = true;
}

void stage_raster_backward(Workspace& w, const CameraDev& cam, const float bg[3], float ldist, int row0, int row1,
                           float* raster_grads, cudaStream_t s) {
    RasterBwdArgs ba{};
    ba.width = cam.width; ba.height = cam.height; ba.tiles_x = cam.tiles_x; ba.tiles_y = cam.tiles_y;
    ba.tile_row_begin = row0; ba.tile_row_end = row1;
    ba.tile_bins = w.tile_bins.as<int2>(); ba.gaussian_ids = w.gaussian_ids.as<int32_t>();
    ba.records = w.records.as<float4>();
    ba.bg[0] = bg[0]; ba.bg[1] = bg[1]; ba.bg[2] = bg[2];
    ba.final_Ts = w.final_Ts.as<float>(); ba.final_idx = w.final_idx.as<int32_t>();
    ba.dL_dout_img = w.dL_dout_img.as<float>();
    ba.dL_dout_distortion = ldist * (1.0f / (float)((double)cam.height * (double)cam.width * 3.0)) * 3.0f;  // lambda_dist / HW
    ba.raster_grads = raster_grads;
    ba.blend_mask = w.blend_mask.as<uint8_t>();
    ba.counters = g_counting ? w.counters.as<unsigned long long>() : nullptr;
    mark(w, kStRasterBwd, s);
    launch_rasterize_backward(ba, s);
}

ProjBwdArgs make_proj_bwd(Workspace& w, const MsplatGaussians* g, const CameraDev& cam, int degrees_to_use,
                          float glob_scale, const float* raster_grads, int g0, int g1) {
    ProjBwdArgs pb{};
    pb.g_begin = g0; pb.g_end = g1;
    pb.means = g->means; pb.scales = g->scales; pb.quats = g->quats; pb.f_dc = g->features_dc;
    pb.f_rest = g->features_rest; pb.opacities = g->opacities;
    pb.rest_bases = sh_rest_bases(g->sh_degree); pb.degrees_to_use = degrees_to_use;
    pb.glob_scale = glob_scale; pb.cam = cam;
    pb.radii = w.radii.as<int32_t>();
    pb.raster_grads = raster_grads;
    pb.inv_max_dim = 1.0f / (float)std::max(cam.width, cam.height);
    return pb;
}

void set_adam(ProjBwdArgs& pb, const MsplatAdamState* adam) {
    if (!adam) throw Error(MSPLAT_ERR_ARGUMENT, "null adam state");
    if (adam->step < 1) throw Error(MSPLAT_ERR_ARGUMENT, "adam step must be >= 1");
    pb.do_adam = 1;
    // Model::fullIteration: bc1/bc2 from std::pow(float, int) (double), model.cpp:767-769, 815-818.
    const float bc1 = 1.0f - std::pow(adam->beta1, adam->step);
    const float bc2 = 1.0f - std::pow(adam->beta2, adam->step);
    for (int k = 0; k < 6; ++k) {
        pb.exp_avg[k] = adam->exp_avg[k];
        pb.exp_avg_sq[k] = adam->exp_avg_sq[k];
        pb.step_size[k] = adam->lr[k] / bc1;
    }
    pb.beta1 = adam->beta1; pb.beta2 = adam->beta2; pb.eps = adam->eps;
    pb.bc2_sqrt = std::sqrt(bc2);
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        t_last_error.clear();
        return MSPLAT_OK;
    } catch (const Error& e) {
        t_last_error = e.what();
        return e.code;
    } catch (const std::exception& e) {
        t_last_error = e.what();
        return MSPLAT_ERR_CUDA;
    }
}

int shard_forward_backward_impl(const MsplatGaussians* g, const MsplatPeerParams* peers, const MsplatCamera* cam,
                                int32_t degrees_to_use, const float background[3], const float* gt, float lambda_l1,
                                float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                void* features_ready, int32_t split_color, void* stream,
                                const float* rgb_in);

}  // namespace
}  // namespace msplat

using namespace msplat;

extern "C" {

int msplat_render(const MsplatGaussians* g, const MsplatCamera* cam, float glob_scale, float clip_thresh,
                  int32_t degrees_to_use, const float background[3], float* out_img, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (!background) throw Error(MSPLAT_ERR_ARGUMENT, "null background");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        CameraDev cd = make_cam(cam);
        stage_forward(w, g, cd, degrees_to_use, glob_scale, clip_thresh, background, true, 0, cd.tiles_y, s);
        mark(w, -1, s);
        if (out_img)
            CK(cudaMemcpyAsync(out_img, w.out_img.p, (size_t)cd.width * cd.height * 3 * 4, cudaMemcpyDeviceToDevice, s));
        CK(cudaGetLastError());
    });
}

int msplat_train_step_2dgs(const MsplatGaussians* g, const MsplatCamera* cam, float glob_scale, float clip_thresh,
                           int32_t degrees_to_use, const float background[3], const float* gt, float lambda_l1,
                           float lambda_dist, float lambda_dssim, float* xys_grad_norm, float* vis_counts,
                           float* max_2d_size, float inv_max_dim, float* loss, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (!background || !gt) throw Error(MSPLAT_ERR_ARGUMENT, "null background or gt");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        CameraDev cd = make_cam(cam);
        const int n = g->num_points;
        stage_forward(w, g, cd, degrees_to_use, glob_scale, clip_thresh, background, true, 0, cd.tiles_y, s);
        stage_loss(w, cd, gt, lambda_l1, lambda_dist, lambda_dssim, 0, cd.height, true, s);
        const size_t nn = (size_t)(n > 0 ? n : 1);
        w.raster_grads.ensure(nn * kGradStride * 4);
        CK(cudaMemsetAsync(w.raster_grads.p, 0, nn * kGradStride * 4, s));
        stage_raster_backward(w, cd, background, lambda_dist, 0, cd.tiles_y, w.raster_grads.as<float>(), s);
        const int K = sh_rest_bases(g->sh_degree);
        w.dL_dmean3D.ensure(nn * 12); w.dL_dscale.ensure(nn * 8); w.dL_dquat.ensure(nn * 16);
        w.dL_dmean2D.ensure(nn * 8); w.dL_dfeatures_dc.ensure(nn * 12);
        w.dL_dfeatures_rest.ensure(nn * (size_t)(K > 0 ? K : 1) * 12); w.dL_dopacity.ensure(nn * 4);
        w.dL_dtransMat.ensure(nn * 36); w.dL_dnormal3D.ensure(nn * 12); w.dL_dcolors.ensure(nn * 12);
        ProjBwdArgs pb = make_proj_bwd(w, g, cd, degrees_to_use, glob_scale, w.raster_grads.as<float>(), 0, n);
        pb.inv_max_dim = inv_max_dim;
        pb.dL_dmean3D = w.dL_dmean3D.as<float>(); pb.dL_dscale = w.dL_dscale.as<float>();
        pb.dL_dquat = w.dL_dquat.as<float>(); pb.dL_dmean2D = w.dL_dmean2D.as<float>();
        pb.dL_dfeatures_dc = w.dL_dfeatures_dc.as<float>();
        pb.dL_dfeatures_rest = K > 0 ? w.dL_dfeatures_rest.as<float>() : nullptr;
        pb.dL_dopacity = w.dL_dopacity.as<float>();
        pb.xys_grad_norm = xys_grad_norm; pb.vis_counts = vis_counts; pb.max_2d_size = max_2d_size;
        if ((xys_grad_norm == nullptr) != (vis_counts == nullptr) || (vis_counts == nullptr) != (max_2d_size == nullptr))
            throw Error(MSPLAT_ERR_ARGUMENT, "densify statistics must be all set or all null");
        mark(w, kStProjectBwd, s);
        launch_project_backward(pb, s);
        mark(w, -1, s);
        launch_unpack_raster_grads(n, w.raster_grads.as<float>(), w.dL_dtransMat.as<float>(),
                                   w.dL_dnormal3D.as<float>(), w.dL_dcolors.as<float>(), nullptr, s);
        w.have_grads = true;
        float lf = 0.f;
        CK(cudaMemcpyAsync(w.h_err, w.err.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(&lf, w.loss_f.p, sizeof(float), cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        CK(cudaGetLastError());
        w.flags = *w.h_err;
        w.flags_pending = false;
        if (loss) *loss = lf;
        if (w.flags & kErrCapacity) throw Error(MSPLAT_ERR_CAPACITY, "tile select kept a wrong count");
        if (w.flags & kErrNonFinite) throw Error(MSPLAT_ERR_NONFINITE, "loss is not finite");
    });
}

int msplat_fused_adam(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, uint32_t n,
                      float step_size, float beta1, float beta2, float bc2_sqrt, float eps, void* stream) {
    return guarded([&] {
        if (n > 0 && (!params || !grads || !exp_avg || !exp_avg_sq)) throw Error(MSPLAT_ERR_ARGUMENT, "null pointer");
        launch_fused_adam(params, grads, exp_avg, exp_avg_sq, (int64_t)n, step_size, beta1, beta2, bc2_sqrt, eps,
                          static_cast<cudaStream_t>(stream));
        CK(cudaGetLastError());
    });
}

int msplat_train_step_fused(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                            const float background[3], const float* gt, float lambda_l1, float lambda_dist,
                            float lambda_dssim, const MsplatAdamState* adam, float* xys_grad_norm,
                            float* vis_counts, float* max_2d_size, float* loss_dev, int32_t write_grads,
                            void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (!background || !gt) throw Error(MSPLAT_ERR_ARGUMENT, "null background or gt");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        CameraDev cd = make_cam(cam);
        const int n = g->num_points;
        // a colour-only step that returns no gradients reads only the image,
        // T and the last contributor of the forward
        const bool aux = write_grads != 0 || lambda_dist != 0.0f;
        stage_forward(w, g, cd, degrees_to_use, 1.0f, 0.01f, background, write_grads != 0, 0, cd.tiles_y, s, 0, 0,
                      nullptr, nullptr, false, nullptr, nullptr, nullptr, aux);
        stage_loss(w, cd, gt, lambda_l1, lambda_dist, lambda_dssim, 0, cd.height, true, s);
        const size_t nn = (size_t)(n > 0 ? n : 1);
        w.raster_grads.ensure(nn * kGradStride * 4);
        CK(cudaMemsetAsync(w.raster_grads.p, 0, nn * kGradStride * 4, s));
        stage_raster_backward(w, cd, background, lambda_dist, 0, cd.tiles_y, w.raster_grads.as<float>(), s);
        ProjBwdArgs pb = make_proj_bwd(w, g, cd, degrees_to_use, 1.0f, w.raster_grads.as<float>(), 0, n);
        set_adam(pb, adam);
        pb.xys_grad_norm = xys_grad_norm; pb.vis_counts = vis_counts; pb.max_2d_size = max_2d_size;
        if ((xys_grad_norm == nullptr) != (vis_counts == nullptr) || (vis_counts == nullptr) != (max_2d_size == nullptr))
            throw Error(MSPLAT_ERR_ARGUMENT, "densify statistics must be all set or all null");
        const int K = sh_rest_bases(g->sh_degree);
        if (write_grads) {
            w.dL_dmean3D.ensure(nn * 12); w.dL_dscale.ensure(nn * 8); w.dL_dquat.ensure(nn * 16);
            w.dL_dmean2D.ensure(nn * 8); w.dL_dfeatures_dc.ensure(nn * 12);
            w.dL_dfeatures_rest.ensure(nn * (size_t)(K > 0 ? K : 1) * 12); w.dL_dopacity.ensure(nn * 4);
            pb.dL_dmean3D = w.dL_dmean3D.as<float>(); pb.dL_dscale = w.dL_dscale.as<float>();
            pb.dL_dquat = w.dL_dquat.as<float>(); pb.dL_dmean2D = w.dL_dmean2D.as<float>();
            pb.dL_dfeatures_dc = w.dL_dfeatures_dc.as<float>();
            pb.dL_dfeatures_rest = K > 0 ? w.dL_dfeatures_rest.as<float>() : nullptr;
            pb.dL_dopacity = w.dL_dopacity.as<float>();
        }
        mark(w, kStProjectBwd, s);
        launch_project_backward(pb, s);
        mark(w, -1, s);
        if (write_grads) {
            w.dL_dtransMat.ensure(nn * 36); w.dL_dnormal3D.ensure(nn * 12); w.dL_dcolors.ensure(nn * 12);
            launch_unpack_raster_grads(n, w.raster_grads.as<float>(), w.dL_dtransMat.as<float>(),
                                       w.dL_dnormal3D.as<float>(), w.dL_dcolors.as<float>(), nullptr, s);
            w.have_grads = true;
        }
        if (loss_dev) CK(cudaMemcpyAsync(loss_dev, w.loss_f.p, sizeof(float), cudaMemcpyDeviceToDevice, s));
        CK(cudaGetLastError());
    });
}

int msplat_shard_forward_backward(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                  const float background[3], const float* gt, float lambda_l1, float lambda_dist,
                                  float lambda_dssim, int32_t world, int32_t rank, int32_t* tile_rows,
                                  float* raster_grads_out, double* loss_parts_dev, void* stream) {
    return shard_forward_backward_impl(g, nullptr, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist,
                                       lambda_dssim, world, rank, tile_rows, raster_grads_out, loss_parts_dev,
                                       nullptr, 0, stream, nullptr);
}

int msplat_shard_forward_backward_peers(const MsplatGaussians* g, const MsplatPeerParams* peers,
                                        const MsplatCamera* cam, int32_t degrees_to_use,
                                        const float background[3], const float* gt, float lambda_l1,
                                        float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                        int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                        void* stream) {
    return shard_forward_backward_impl(g, peers, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist,
                                       lambda_dssim, world, rank, tile_rows, raster_grads_out, loss_parts_dev,
                                       nullptr, 0, stream, nullptr);
}

int msplat_shard_forward_backward_after(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                        const float background[3], const float* gt, float lambda_l1,
                                        float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                        int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                        void* features_ready, int32_t split_color, void* stream) {
    return shard_forward_backward_impl(g, nullptr, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist,
                                       lambda_dssim, world, rank, tile_rows, raster_grads_out, loss_parts_dev,
                                       features_ready, split_color, stream, nullptr);
}

int msplat_shard_forward_backward_rgb(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                      const float background[3], const float* gt, float lambda_l1,
                                      float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                      int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                      const float* rgb, void* rgb_ready, void* stream) {
    if (!rgb) {
        msplat::set_last_error("null rgb");
        return MSPLAT_ERR_ARGUMENT;
    }
    return shard_forward_backward_impl(g, nullptr, cam, degrees_to_use, background, gt, lambda_l1, lambda_dist,
                                       lambda_dssim, world, rank, tile_rows, raster_grads_out, loss_parts_dev,
                                       rgb_ready, 1, stream, rgb);
}

int msplat_shard_colors(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use, int32_t g_begin,
                        int32_t g_end, float* rgb, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (!rgb) throw Error(MSPLAT_ERR_ARGUMENT, "null rgb");
        if (g_begin < 0 || g_end > g->num_points || g_begin > g_end) throw Error(MSPLAT_ERR_ARGUMENT, "bad slice");
        ProjFwdArgs pa{};
        pa.n = g->num_points;
        pa.means = g->means; pa.scales = g->scales; pa.quats = g->quats; pa.opacities = g->opacities;
        pa.f_dc = g->features_dc; pa.f_rest = g->features_rest;
        pa.rest_bases = sh_rest_bases(g->sh_degree);
        pa.degrees_to_use = degrees_to_use;
        pa.cam = make_cam(cam);
        launch_shard_colors(pa, g_begin, g_end, rgb, static_cast<cudaStream_t>(stream));
        CK(cudaGetLastError());
    });
}

}  // extern "C"

namespace msplat {
namespace {
int shard_forward_backward_impl(const MsplatGaussians* g, const MsplatPeerParams* peers, const MsplatCamera* cam,
                                int32_t degrees_to_use, const float background[3], const float* gt, float lambda_l1,
                                float lambda_dist, float lambda_dssim, int32_t world, int32_t rank,
                                int32_t* tile_rows, float* raster_grads_out, double* loss_parts_dev,
                                void* features_ready, int32_t split_color, void* stream,
                                const float* rgb_in) {
    return guarded([&] {
        if (peers) {
            if (peers->world < 2 || peers->world > MSPLAT_MAX_PEER_RANKS || peers->chunk <= 0 ||
                (int64_t)peers->world * peers->chunk < g->num_points)
                throw Error(MSPLAT_ERR_ARGUMENT, "bad peer parameter view");
            for (int gi = 0; gi < 6; ++gi)
                for (int q = 0; q < peers->world; ++q)
                    if (!peers->base[gi][q] && !(gi == 4 && g->sh_degree == 0))
                        throw Error(MSPLAT_ERR_ARGUMENT, "null peer buffer");
        }
        check_inputs(g, cam, degrees_to_use);
        if (!background || !gt || !raster_grads_out || !tile_rows) throw Error(MSPLAT_ERR_ARGUMENT, "null pointer");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        CameraDev cd = make_cam(cam);
        int o0 = tile_rows[0], o1 = tile_rows[1];
        if (world > 0) {
            if (rank < 0 || rank >= world) throw Error(MSPLAT_ERR_ARGUMENT, "rank out of range");
        } else if (o0 < 0 || o1 > cd.tiles_y || o0 > o1) {
            throw Error(MSPLAT_ERR_ARGUMENT, "bad tile row range");
        }
        const int n = g->num_points;
        const int r0 = std::max(0, o0 - 1), r1 = std::min(cd.tiles_y, o1 + 1);
        stage_forward(w, g, cd, degrees_to_use, 1.0f, 0.01f, background, false, r0, r1, s, world, rank, &o0, &o1,
                      split_color != 0, static_cast<cudaEvent_t>(features_ready), peers, rgb_in,
                      lambda_dist != 0.0f);
        tile_rows[0] = o0;
        tile_rows[1] = o1;
        const int p0 = std::min(cd.height, o0 * kTile), p1 = std::min(cd.height, o1 * kTile);
        const size_t nn = (size_t)(n > 0 ? n : 1);
        CK(cudaMemsetAsync(raster_grads_out, 0, nn * kGradStride * 4, s));
        if (p1 > p0) {
            stage_loss(w, cd, gt, lambda_l1, lambda_dist, lambda_dssim, p0, p1, false, s);
            stage_raster_backward(w, cd, background, lambda_dist, o0, o1, raster_grads_out, s);
        }
        if (loss_parts_dev) {
            if (p1 > p0) {
                // Sum the block partials (l1, ssim, dist) without the DSSIM offset.
                const int nb = loss_num_blocks(cd.width, p0, p1);
                launch_loss_finalize(w.loss_partials.as<double>(), nb, 0.0f, 0.0f, w.loss_out.as<double>(),
                                     nullptr, w.err.as<uint32_t>(), s);
                // loss_out = {l1 + dist, ssim, l1, dist} -> parts (l1, ssim, dist)
                CK(cudaMemcpyAsync(loss_parts_dev, w.loss_out.as<double>() + 2, sizeof(double), cudaMemcpyDeviceToDevice, s));
                CK(cudaMemcpyAsync(loss_parts_dev + 1, w.loss_out.as<double>() + 1, sizeof(double), cudaMemcpyDeviceToDevice, s));
                CK(cudaMemcpyAsync(loss_parts_dev + 2, w.loss_out.as<double>() + 3, sizeof(double), cudaMemcpyDeviceToDevice, s));
            } else {
                CK(cudaMemsetAsync(loss_parts_dev, 0, 3 * sizeof(double), s));
            }
        }
        mark(w, kStBetweenShardCalls, s);
        CK(cudaGetLastError());
    });
}
}  // namespace
}  // namespace msplat

extern "C" {

int msplat_device_alloc(uint64_t bytes, void** ptr) {
    return guarded([&] {
        if (!ptr) throw Error(MSPLAT_ERR_ARGUMENT, "null pointer");
        *ptr = nullptr;
        void* p = nullptr;
        CK(cudaMalloc(&p, bytes > 0 ? bytes : 1));
        CK(cudaMemset(p, 0, bytes > 0 ? bytes : 1));
        *ptr = p;
    });
}

int msplat_device_free(void* ptr) {
    return guarded([&] {
        if (ptr) CK(cudaFree(ptr));
    });
}

int msplat_ipc_handle(void* ptr, uint8_t handle[64]) {
    return guarded([&] {
        if (!ptr || !handle) throw Error(MSPLAT_ERR_ARGUMENT, "null pointer");
        static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
        cudaIpcMemHandle_t h;
        CK(cudaIpcGetMemHandle(&h, ptr));
        std::memcpy(handle, &h, 64);
    });
}

int msplat_ipc_open(const uint8_t handle[64], void** ptr) {
    return guarded([&] {
        if (!ptr || !handle) throw Error(MSPLAT_ERR_ARGUMENT, "null pointer");
        *ptr = nullptr;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle, 64);
        void* p = nullptr;
        CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        *ptr = p;
    });
}

int msplat_ipc_close(void* ptr) {
    return guarded([&] {
        if (ptr) CK(cudaIpcCloseMemHandle(ptr));
    });
}

int msplat_shard_project_backward_adam(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                       const float* raster_grads, int32_t g_begin, int32_t g_end,
                                       const MsplatAdamState* adam, float* xys_grad_norm, float* vis_counts,
                                       float* max_2d_size, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (!raster_grads) throw Error(MSPLAT_ERR_ARGUMENT, "null raster_grads");
        if (g_begin < 0 || g_end > g->num_points || g_begin > g_end) throw Error(MSPLAT_ERR_ARGUMENT, "bad shard");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        CameraDev cd = make_cam(cam);
        ProjBwdArgs pb = make_proj_bwd(w, g, cd, degrees_to_use, 1.0f, raster_grads, g_begin, g_end);
        set_adam(pb, adam);
        pb.xys_grad_norm = xys_grad_norm; pb.vis_counts = vis_counts; pb.max_2d_size = max_2d_size;
        mark(w, kStProjectBwd, s);
        launch_project_backward(pb, s);
        mark(w, -1, s);
        CK(cudaGetLastError());
    });
}

// ---- routed multi-GPU exchange (route.cu) -----------------------------------

int msplat_route_summary_len(const MsplatCamera* cam, int64_t* len_out) {
    return guarded([&] {
        if (!cam || !len_out) throw Error(MSPLAT_ERR_ARGUMENT, "null argument");
        const CameraDev cd = make_cam(cam);
        *len_out = route_summary_len(cd.tiles_x, cd.tiles_y);
    });
}

int msplat_route_project(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use, int32_t g_begin,
                         int32_t g_end, int32_t* summary_out, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        if (g_begin < 0 || g_end > g->num_points || g_begin > g_end) throw Error(MSPLAT_ERR_ARGUMENT, "bad slice");
        if (!summary_out) throw Error(MSPLAT_ERR_ARGUMENT, "null summary_out");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        const CameraDev cd = make_cam(cam);
        const int n = g_end - g_begin;
        const size_t nn = (size_t)(n > 0 ? n : 1);
        const int tx = cd.tiles_x, ty = cd.tiles_y;
        w.own_records.ensure(nn * kRecordF4 * sizeof(float4));
        w.own_cull.ensure(nn * kCullF4 * sizeof(float4));
        w.own_rects.ensure(nn * sizeof(uint2));
        w.own_depths.ensure(nn * sizeof(float));
        w.own_radii.ensure(nn * sizeof(int32_t));
        const size_t diff_bytes = (size_t)(tx + 1) * (ty + 1) * 4;
        w.route_diff.ensure(diff_bytes);
        w.route_colsum.ensure((size_t)tx * ty * 4);
        CK(cudaMemsetAsync(w.route_diff.p, 0, diff_bytes, s));
        const int K = sh_rest_bases(g->sh_degree);
        ProjFwdArgs pa{};
        pa.n = n;
        pa.pass = 0;
        pa.means = g->means + 3 * (size_t)g_begin;
        pa.scales = g->scales + 2 * (size_t)g_begin;
        pa.quats = g->quats + 4 * (size_t)g_begin;
        pa.opacities = g->opacities + (size_t)g_begin;
        pa.f_dc = g->features_dc + 3 * (size_t)g_begin;
        pa.f_rest = K > 0 ? g->features_rest + 3 * (size_t)K * g_begin : g->features_rest;
        pa.rest_bases = K; pa.degrees_to_use = degrees_to_use;
        pa.glob_scale = 1.0f; pa.clip_thresh = 0.01f;
        pa.cam = cd;
        pa.records = w.own_records.as<float4>(); pa.cull = w.own_cull.as<float4>();
        pa.rects = w.own_rects.as<uint2>(); pa.depths = w.own_depths.as<float>();
        pa.radii = w.own_radii.as<int32_t>(); pa.tile_diff = w.route_diff.as<int32_t>();
        pa.id_chunk = std::max(1, n);  // one difference array for the slice
        mark(w, kStProject, s);
        launch_project_forward(pa, s);
        mark(w, kStRouteExchange, s);
        CK(cudaMemsetAsync(summary_out + (size_t)tx * ty, 0, 2 * (size_t)(ty + 1) * sizeof(int32_t), s));
        launch_route_summary(w.route_diff.as<int32_t>(), tx, ty, n, w.own_rects.as<uint2>(), w.own_radii.as<int32_t>(),
                             w.route_colsum.as<int32_t>(), summary_out, s);
        w.route_n = n;
        w.route_g0 = g_begin;
        CK(cudaGetLastError());
    });
}

int msplat_route_plan(const int32_t* summaries, const MsplatCamera* cam, int32_t world, int32_t rank,
                      int32_t* bands_out, int64_t* send_counts_out, int64_t* recv_counts_out, void* stream) {
    return guarded([&] {
        if (!summaries || !cam || !bands_out || !send_counts_out || !recv_counts_out)
            throw Error(MSPLAT_ERR_ARGUMENT, "null argument");
        if (world < 1 || world > kMaxPeerRanks) throw Error(MSPLAT_ERR_ARGUMENT, "world must be in [1, 16]");
        if (rank < 0 || rank >= world) throw Error(MSPLAT_ERR_ARGUMENT, "rank out of range");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        const CameraDev cd = make_cam(cam);
        const int tx = cd.tiles_x, ty = cd.tiles_y, n = w.route_n;
        const int nblocks = (n + 255) / 256;
        w.own_dest.ensure((size_t)(n > 0 ? n : 1) * sizeof(int2));
        w.route_block.ensure((size_t)(nblocks > 0 ? nblocks : 1) * world * sizeof(int32_t));
        w.route_totals.ensure(kMaxPeerRanks * sizeof(int64_t));
        w.route_base.ensure(kMaxPeerRanks * sizeof(int64_t));
        w.route_bands.ensure((kMaxPeerRanks + 1) * sizeof(int32_t));
        w.route_matrix.ensure(kMaxPeerRanks * kMaxPeerRanks * sizeof(int64_t));
        w.route_row_work.ensure((size_t)(ty > 0 ? ty : 1) * sizeof(int64_t));
        launch_route_plan(summaries, tx, ty, world, w.route_row_work.as<int64_t>(), w.route_bands.as<int32_t>(),
                          w.route_matrix.as<int64_t>(), n, w.own_rects.as<uint2>(), w.own_radii.as<int32_t>(),
                          w.own_dest.as<int2>(), w.route_block.as<int32_t>(), w.route_totals.as<int64_t>(),
                          w.route_base.as<int64_t>(), s);
        // host: bands (int32, world + 1), this slice's totals (int64, world),
        // the count matrix (int64, world x world)
        int32_t* hb = reinterpret_cast<int32_t*>(w.h_route);
        int64_t* ht = w.h_route + (kMaxPeerRanks + 2) / 2;
        int64_t* hm = ht + kMaxPeerRanks;
        CK(cudaMemcpyAsync(hb, w.route_bands.p, (world + 1) * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(ht, w.route_totals.p, world * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
        CK(cudaMemcpyAsync(hm, w.route_matrix.p, (size_t)world * world * sizeof(int64_t), cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        for (int r = 0; r <= world; ++r) {
            if (hb[r] < 0 || hb[r] > ty || (r > 0 && hb[r] < hb[r - 1])) throw Error(MSPLAT_ERR_CAPACITY, "corrupt bands");
            bands_out[r] = hb[r];
        }
        int64_t items = 0;
        for (int q = 0; q < world; ++q) {
            const int64_t c = ht[q];
            // the slice's own destinations must agree with the count matrix
            // every rank computed from the gathered histograms
            if (c < 0 || c > n || c != hm[(size_t)rank * world + q])
                throw Error(MSPLAT_ERR_CAPACITY, "route counts disagree with the gathered summaries");
            send_counts_out[q] = c;
            items += c;
        }
        for (int r = 0; r < world; ++r) {
            const int64_t c = hm[(size_t)r * world + rank];
            if (c < 0) throw Error(MSPLAT_ERR_CAPACITY, "corrupt route counts");
            recv_counts_out[r] = c;
        }
        w.route_world = world;
        w.route_rank = rank;
        w.route_matrix_h.assign(hm, hm + (size_t)world * world);
        w.route_items = items;
        w.route_src.ensure((size_t)(items > 0 ? items : 1) * sizeof(int32_t));
    });
}

namespace {
// Items from rank r to rank q in the last plan.
int64_t route_count(const Workspace& w, int r, int q) { return w.route_matrix_h[(size_t)r * w.route_world + q]; }

RouteDests own_dests(const Workspace& w) {
    RouteDests d{};
    int64_t run = 0;
    for (int q = 0; q < w.route_world; ++q) {
        d.send_base[q] = run;
        run += route_count(w, w.route_rank, q);
    }
    return d;
}

void check_route_peers(const Workspace& w, const MsplatRoutePeers* peers) {
    if (!peers) throw Error(MSPLAT_ERR_ARGUMENT, "null peers");
    if (peers->world != w.route_world || peers->rank != w.route_rank)
        throw Error(MSPLAT_ERR_ARGUMENT, "peers world/rank differ from the last msplat_route_plan");
    for (int q = 0; q < w.route_world; ++q)
        if (!peers->inbox[q] || !peers->returnbox[q]) throw Error(MSPLAT_ERR_ARGUMENT, "null peer buffer");
}
}  // namespace

int msplat_route_pack(void* send_payload, void* stream) {
    return guarded([&] {
        Workspace& w = workspace();
        if (w.route_items > 0 && !send_payload) throw Error(MSPLAT_ERR_ARGUMENT, "null send_payload");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        RouteDests d = own_dests(w);
        for (int q = 0; q < w.route_world; ++q)
            d.dst[q] = static_cast<float4*>(send_payload) + (size_t)d.send_base[q] * kRoutePayloadF4;
        launch_route_pack(w.route_n, w.route_g0, w.own_records.as<float4>(), w.own_cull.as<float4>(),
                          w.own_rects.as<uint2>(), w.own_depths.as<float>(), w.own_dest.as<int2>(),
                          w.route_block.as<int32_t>(), w.route_world, d, false, w.route_src.as<int32_t>(), s);
        CK(cudaGetLastError());
    });
}

int msplat_route_pack_peers(const MsplatRoutePeers* peers, void* stream) {
    return guarded([&] {
        Workspace& w = workspace();
        check_route_peers(w, peers);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        RouteDests d = own_dests(w);
        for (int q = 0; q < w.route_world; ++q) {
            // q's inbox holds the sources in rank order
            int64_t off = 0;
            for (int r = 0; r < w.route_rank; ++r) off += route_count(w, r, q);
            if (off + route_count(w, w.route_rank, q) > peers->inbox_items)
                throw Error(MSPLAT_ERR_CAPACITY, "a peer inbox is too small for this step");
            d.dst[q] = static_cast<float4*>(peers->inbox[q]) + (size_t)off * kRoutePayloadF4;
        }
        launch_route_pack(w.route_n, w.route_g0, w.own_records.as<float4>(), w.own_cull.as<float4>(),
                          w.own_rects.as<uint2>(), w.own_depths.as<float>(), w.own_dest.as<int2>(),
                          w.route_block.as<int32_t>(), w.route_world, d, true, w.route_src.as<int32_t>(), s);
        CK(cudaGetLastError());
    });
}

int msplat_route_push_peers(const MsplatRoutePeers* peers, const float* raster_grads, void* stream) {
    return guarded([&] {
        Workspace& w = workspace();
        check_route_peers(w, peers);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        RouteReturns ret{};
        int64_t m = 0;
        for (int r = 0; r < w.route_world; ++r) {
            ret.recv_off[r] = m;
            m += route_count(w, r, w.route_rank);
            // r's return box holds its items in its packing order: groups by
            // destination rank
            int64_t off = 0, row = 0;
            for (int q = 0; q < w.route_world; ++q) {
                if (q < w.route_rank) off += route_count(w, r, q);
                row += route_count(w, r, q);
            }
            if (row > peers->returnbox_items) throw Error(MSPLAT_ERR_CAPACITY, "a peer return box is too small");
            ret.dst[r] = static_cast<float4*>(peers->returnbox[r]) + (size_t)off * (kGradStride / 4);
        }
        ret.recv_off[w.route_world] = m;
        if (m > 0 && !raster_grads) throw Error(MSPLAT_ERR_ARGUMENT, "null raster_grads");
        launch_route_push(m, reinterpret_cast<const float4*>(raster_grads), w.route_world, ret, s);
        CK(cudaGetLastError());
    });
}

int msplat_route_band(const MsplatCamera* cam, int32_t sh_degree, const void* recv_payload, int64_t num_recv,
                      int32_t band_begin, int32_t band_end, const float background[3], const float* gt,
                      float lambda_l1, float lambda_dist, float lambda_dssim, float* raster_grads_out,
                      double* loss_parts_dev, void* stream) {
    return guarded([&] {
        if (!cam || !background || !gt || !loss_parts_dev) throw Error(MSPLAT_ERR_ARGUMENT, "null argument");
        if (num_recv < 0 || num_recv > (1 << 25)) throw Error(MSPLAT_ERR_ARGUMENT, "num_recv must be in [0, 2^25]");
        if (num_recv > 0 && (!recv_payload || !raster_grads_out)) throw Error(MSPLAT_ERR_ARGUMENT, "null buffer");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        Workspace& w = workspace();
        const CameraDev cd = make_cam(cam);
        if (band_begin < 0 || band_end > cd.tiles_y || band_begin > band_end)
            throw Error(MSPLAT_ERR_ARGUMENT, "bad band");
        const int m = (int)num_recv;
        const size_t nn = (size_t)(m > 0 ? m : 1);
        const int tx = cd.tiles_x, ty = cd.tiles_y;
        // the arrays the binning and rasterisers read, filled from the payloads
        w.records.ensure(nn * kRecordF4 * sizeof(float4));
        w.cull.ensure(nn * kCullF4 * sizeof(float4));
        w.rects.ensure(nn * sizeof(uint2));
        w.depths.ensure(nn * sizeof(float));
        w.radii.ensure(nn * sizeof(int32_t));
        w.route_ids.ensure(nn * sizeof(int32_t));
        const size_t diff_bytes = (size_t)kIdChunks * (tx + 1) * (ty + 1) * 4;
        w.tile_diff.ensure(diff_bytes);
        CK(cudaMemsetAsync(w.tile_diff.p, 0, diff_bytes, s));
        const int id_chunk = std::max(1, (m + kIdChunks - 1) / kIdChunks);
        mark(w, kStRouteUnpack, s);
        launch_route_unpack(num_recv, static_cast<const float4*>(recv_payload), tx, ty, id_chunk,
                            w.records.as<float4>(), w.cull.as<float4>(), w.rects.as<uint2>(), w.depths.as<float>(),
                            w.route_ids.as<int32_t>(), w.radii.as<int32_t>(), w.tile_diff.as<int32_t>(), s);
        MsplatGaussians recv{};
        recv.num_points = m;
        recv.sh_degree = sh_degree;
        const int r0 = band_end > band_begin ? std::max(0, band_begin - 1) : 0;
        const int r1 = band_end > band_begin ? std::min(ty, band_end + 1) : 0;
        stage_forward(w, &recv, cd, 0, 1.0f, 0.01f, background, false, r0, r1, s, 0, 0, nullptr, nullptr, false,
                      nullptr, nullptr, nullptr, lambda_dist != 0.0f, /*prefilled=*/true);
        const int p0 = std::min(cd.height, band_begin * kTile), p1 = std::min(cd.height, band_end * kTile);
        if (m > 0) CK(cudaMemsetAsync(raster_grads_out, 0, nn * kGradStride * 4, s));
        if (p1 > p0) {
            stage_loss(w, cd, gt, lambda_l1, lambda_dist, lambda_dssim, p0, p1, false, s);
            if (m > 0) stage_raster_backward(w, cd, background, lambda_dist, band_begin, band_end, raster_grads_out, s);
            const int nb = loss_num_blocks(cd.width, p0, p1);
            launch_loss_finalize(w.loss_partials.as<double>(), nb, 0.0f, 0.0f, w.loss_out.as<double>(), nullptr,
                                 w.err.as<uint32_t>(), s);
            // loss_out = {l1 + dist, ssim, l1, dist} -> parts (l1, ssim, dist)
            CK(cudaMemcpyAsync(loss_parts_dev, w.loss_out.as<double>() + 2, sizeof(double), cudaMemcpyDeviceToDevice, s));
            CK(cudaMemcpyAsync(loss_parts_dev + 1, w.loss_out.as<double>() + 1, sizeof(double), cudaMemcpyDeviceToDevice,
                               s));
            CK(cudaMemcpyAsync(loss_parts_dev + 2, w.loss_out.as<double>() + 3, sizeof(double), cudaMemcpyDeviceToDevice,
                               s));
        } else {
            CK(cudaMemsetAsync(loss_parts_dev, 0, 3 * sizeof(double), s));
        }
        mark(w, kStBetweenShardCalls, s);
        CK(cudaGetLastError());
    });
}

int msplat_route_return(const float* recv_grads, int64_t num_items, float* slice_grads, void* stream) {
    return guarded([&] {
        Workspace& w = workspace();
        if (num_items != w.route_items) throw Error(MSPLAT_ERR_ARGUMENT, "num_items differs from the packed items");
        if (!slice_grads || (num_items > 0 && !recv_grads)) throw Error(MSPLAT_ERR_ARGUMENT, "null buffer");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (w.route_n > 0) CK(cudaMemsetAsync(slice_grads, 0, (size_t)w.route_n * kGradStride * 4, s));
        launch_route_gather(num_items, reinterpret_cast<const float4*>(recv_grads), w.route_src.as<int32_t>(),
                            slice_grads, s);
        CK(cudaGetLastError());
    });
}

int msplat_route_project_backward_adam(const MsplatGaussians* g, const MsplatCamera* cam, int32_t degrees_to_use,
                                       const float* slice_grads, const MsplatAdamState* adam, float* xys_grad_norm,
                                       float* vis_counts, float* max_2d_size, void* stream) {
    return guarded([&] {
        check_inputs(g, cam, degrees_to_use);
        Workspace& w = workspace();
        const int g0 = w.route_g0, g1 = w.route_g0 + w.route_n;
        if (g1 > g->num_points) throw Error(MSPLAT_ERR_ARGUMENT, "slice beyond num_points");
        if (w.route_n > 0 && !slice_grads) throw Error(MSPLAT_ERR_ARGUMENT, "null slice_grads");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        CameraDev cd = make_cam(cam);
        // the kernel indexes by global id: offset the slice buffers
        ProjBwdArgs pb = make_proj_bwd(w, g, cd, degrees_to_use, 1.0f, slice_grads - (size_t)g0 * kGradStride, g0, g1);
        pb.radii = w.own_radii.as<int32_t>() - g0;
        set_adam(pb, adam);
        pb.xys_grad_norm = xys_grad_norm; pb.vis_counts = vis_counts; pb.max_2d_size = max_2d_size;
        mark(w, kStProjectBwd, s);
        launch_project_backward(pb, s);
        mark(w, -1, s);
        CK(cudaGetLastError());
    });
}

int msplat_last_tensor(const char* name, MsplatTensorRef* out) {
    return guarded([&] {
        if (!name || !out) throw Error(MSPLAT_ERR_ARGUMENT, "null argument");
        Workspace& w = workspace();
        const std::string nm(name);
        const int64_t n = w.n, H = w.H, W = w.W, T = (int64_t)w.tx * w.ty;
        auto set = [&](const Buf& b, int dtype, std::initializer_list<int64_t> shape, bool ok) {
            if (!ok || !b.p) throw Error(MSPLAT_ERR_ARGUMENT, "tensor '" + nm + "' not produced by the last call");
            out->data = b.p;
            out->dtype = dtype;
            out->ndim = (int32_t)shape.size();
            int k = 0;
            for (int64_t d : shape) out->shape[k++] = d;
            for (; k < 4; ++k) out->shape[k] = 0;
        };
        const bool px = w.have_pixels, rp = w.have_ref_proj, gr = w.have_grads, ax = px && w.have_aux;
        if (nm == "out_img") set(w.out_img, 0, {H, W, 3}, px);
        else if (nm == "out_depth") set(w.out_depth, 0, {H, W}, ax);
        else if (nm == "out_normal") set(w.out_normal, 0, {H, W, 3}, ax);
        else if (nm == "out_alpha") set(w.out_alpha, 0, {H, W}, ax);
        else if (nm == "out_median_depth") set(w.out_median, 0, {H, W}, ax);
        else if (nm == "out_distortion") set(w.out_dist, 0, {H, W}, ax);
        else if (nm == "final_Ts") set(w.final_Ts, 0, {H, W, 3}, ax);
        else if (nm == "final_idx") set(w.final_idx, 1, {H, W, 2}, ax);
        else if (nm == "dL_dout_img") set(w.dL_dout_img, 0, {H, W, 3}, w.have_dimg);
        else if (nm == "radii") set(w.radii, 1, {n}, px);
        else if (nm == "depths") set(w.depths, 0, {n}, px);
        else if (nm == "tile_bins") set(w.tile_bins, 1, {T, 2}, px);
        else if (nm == "raw_tile_counts") set(w.raw_true, 1, {T}, px);
        else if (nm == "gaussian_ids") set(w.gaussian_ids, 1, {w.kept}, px);
        else if (nm == "raster_counters") set(w.counters, 2, {4}, px);
        else if (nm == "intersection_totals") set(w.totals, 2, {5}, px);
        else if (nm == "xys") set(w.xys, 0, {n, 2}, rp);
        else if (nm == "transMats") set(w.transmats, 0, {n, 9}, rp);
        else if (nm == "normal_opacity") set(w.normal_opacity, 0, {n, 4}, rp);
        else if (nm == "colors") set(w.colors, 0, {n, 3}, rp);
        else if (nm == "num_tiles_hit") set(w.num_tiles_hit, 1, {n}, rp);
        else if (nm == "dL_dmean3D") set(w.dL_dmean3D, 0, {n, 3}, gr);
        else if (nm == "dL_dscale") set(w.dL_dscale, 0, {n, 2}, gr);
        else if (nm == "dL_dquat") set(w.dL_dquat, 0, {n, 4}, gr);
        else if (nm == "dL_dopacity") set(w.dL_dopacity, 0, {n, 1}, gr);
        else if (nm == "dL_dfeatures_dc") set(w.dL_dfeatures_dc, 0, {n, 3}, gr);
        else if (nm == "dL_dfeatures_rest") set(w.dL_dfeatures_rest, 0, {n, w.K, 3}, gr && w.K > 0);
        else if (nm == "dL_dmean2D") set(w.dL_dmean2D, 0, {n, 2}, gr);
        else if (nm == "dL_dtransMat") set(w.dL_dtransMat, 0, {n, 9}, gr);
        else if (nm == "dL_dnormal3D") set(w.dL_dnormal3D, 0, {n, 3}, gr);
        else if (nm == "dL_dcolors") set(w.dL_dcolors, 0, {n, 3}, gr);
        else if (nm == "loss_partials") set(w.loss_partials, 3, {w.loss_blocks, 3}, w.have_dimg);
        else if (nm == "loss_terms") set(w.loss_out, 3, {4}, w.have_dimg);
        else throw Error(MSPLAT_ERR_ARGUMENT, "unknown tensor name '" + nm + "'");
    });
}

int msplat_loss_ssim_noalloc(const float* out_img, const float* gt, const float* out_distortion, int32_t width,
                             int32_t height, float lambda_l1, float lambda_dist, float lambda_dssim,
                             float* dL_dout_img, float* loss_out, void* stream) {
    std::string msg;
    const int rc = loss_ssim_noalloc(out_img, gt, out_distortion, width, height, lambda_l1, lambda_dist, lambda_dssim,
                                     dL_dout_img, loss_out, static_cast<cudaStream_t>(stream), &msg);
    t_last_error = rc == MSPLAT_OK ? std::string() : msg;
    return rc;
}

int64_t msplat_last_num_intersections(void) {
    try {
        return workspace().kept;
    } catch (...) {
        return -1;
    }
}

uint32_t msplat_last_status_flags(void) {
    try {
        Workspace& w = workspace();
        if (w.flags_pending) {
            CK(cudaMemcpyAsync(w.h_err, w.err.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, w.last_stream));
            CK(cudaStreamSynchronize(w.last_stream));
            w.flags = *w.h_err;
            w.flags_pending = false;
        }
        return w.flags & MSPLAT_FLAG_TILE_OVERFLOW;
    } catch (...) {
        return 0;
    }
}

int msplat_set_stage_timing(int32_t enable) {
    return guarded([&] {
        Workspace& w = workspace();
        flush_timing(w);
        g_timing = enable != 0;
        for (int k = 0; k < kNumStages; ++k) {
            g_stage_ms[k] = 0.0;
            g_stage_n[k] = 0;
        }
    });
}

int msplat_set_raster_counters(int32_t enable) {
    return guarded([&] { g_counting = enable != 0; });
}

int32_t msplat_stage_times(double* total_ms, int64_t* counts, int32_t max_stages) {
    try {
        Workspace& w = workspace();
        flush_timing(w);
        const int k = max_stages < kNumStages ? max_stages : kNumStages;
        for (int i = 0; i < k; ++i) {
            if (total_ms) total_ms[i] = g_stage_ms[i];
            if (counts) counts[i] = g_stage_n[i];
        }
        t_last_error.clear();
        return kNumStages;
    } catch (const std::exception& e) {
        t_last_error = e.what();
        return -1;
    }
}

const char* msplat_stage_name(int32_t i) { return (i >= 0 && i < kNumStages) ? kStageNames[i] : ""; }

int64_t msplat_launch_count(void) { return g_launches.load(); }

const char* msplat_last_error(void) { return t_last_error.c_str(); }

void msplat_commit(void) {}

void msplat_gpu_sync(void) { cudaDeviceSynchronize(); }

void msplat_backend_cleanup(void) {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    for (Workspace* w : g_ws)
        if (w) {
            w->release_all();
            delete w;
        }
    g_ws.clear();
}

}  // extern "C"
