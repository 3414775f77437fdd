// trainer.cu — the trainer-level C API of include/msplat_c_api.h: in-memory
// datasets, Model initialisation, the training step loop with its camera
// shuffle and learning-rate schedule, rendering and evaluation. Host code over
// the backend C ABI (include/msplat_backend.h) and the CUDA runtime.
//
// Follows core/src/msplat_api.mm (Dataset/Trainer, :20-280; C API :282-407),
// core/src/model.cpp (Model ctor :43-121, setupOptimizers :123-168,
// schedulersStep :183-186, getDownscaleFactor :235-238, afterTrain :240-306,
// checkpoints :341-498, prepareCam :500-544, fullIteration :762-829) and
// core/src/loaders/save_gaussians.cpp (PLY :11-58, .splat :60-111).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "kernels.cuh"
#include "msplat_backend.h"
#include "msplat_c_api.h"

namespace msplat {
namespace {

struct ApiError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define CKT(call)                                                                                     \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) throw ApiError(std::string(#call) + ": " + cudaGetErrorString(e_));    \
    } while (0)

void check_rc(int rc) {
    if (rc != MSPLAT_OK) throw ApiError(msplat_last_error());
}

struct Camera {
    float c2w[16];
    float fx, fy, cx, cy;
    int width, height;
    float* image = nullptr;  // pinned host [h][w][3] or null
};

struct Dataset {
    std::vector<Camera> train, test;
    std::vector<float> xyz;
    std::vector<uint8_t> rgb;
    std::vector<float*> pinned;
    // InputData::scale / translation (the loaders' normalisation); in-memory
    // datasets are used as given
    float scale = 1.0f;
    float translation[3] = {0.f, 0.f, 0.f};
    ~Dataset() {
        for (float* p : pinned) cudaFreeHost(p);
    }
};

template <typename T>
struct DevArray {
    T* p = nullptr;
    size_t n = 0;
    void alloc(size_t count) {
        release();
        if (count == 0) count = 1;
        CKT(cudaMalloc(&p, count * sizeof(T)));
        CKT(cudaMemset(p, 0, count * sizeof(T)));
        CKT(cudaDeviceSynchronize());  // zeroed before any stream of the trainer touches it
        n = count;
    }
    void ensure(size_t count) {
        if (count > n) alloc(count);
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    ~DevArray() { release(); }
};

constexpr double kC0 = 0.28209479177387814;

int num_sh_bases(int degree) { return (degree + 1) * (degree + 1); }

// Mean distance to the 3 nearest other points (PointsTensor::scales, k = 4
// including the point itself, kdtree_tensor.hpp:26-40), with a uniform grid.
std::vector<float> knn_mean_distance(const std::vector<float>& xyz) {
    const int64_t n = (int64_t)xyz.size() / 3;
    std::vector<float> out(n, 0.01f);
    if (n < 2) return out;
    float lo[3] = {1e30f, 1e30f, 1e30f}, hi[3] = {-1e30f, -1e30f, -1e30f};
    for (int64_t i = 0; i < n; ++i)
        for (int d = 0; d < 3; ++d) {
            lo[d] = std::min(lo[d], xyz[3 * i + d]);
            hi[d] = std::max(hi[d], xyz[3 * i + d]);
        }
    const double vol = std::max(1e-12, (double)(hi[0] - lo[0]) * (hi[1] - lo[1]) * (hi[2] - lo[2]));
    const float cell = (float)std::max(1e-6, std::cbrt(vol / std::max<int64_t>(1, n / 2)));
    auto key = [&](int cx, int cy, int cz) { return ((int64_t)cx * 73856093) ^ ((int64_t)cy * 19349663) ^ ((int64_t)cz * 83492791); };
    std::unordered_map<int64_t, std::vector<int64_t>> grid;
    grid.reserve((size_t)n);
    auto cell_of = [&](int64_t i, int* c) {
        for (int d = 0; d < 3; ++d) c[d] = (int)std::floor((xyz[3 * i + d] - lo[d]) / cell);
    };
    for (int64_t i = 0; i < n; ++i) {
        int c[3];
        cell_of(i, c);
        grid[key(c[0], c[1], c[2])].push_back(i);
    }
    for (int64_t i = 0; i < n; ++i) {
        int c[3];
        cell_of(i, c);
        float best[3] = {1e30f, 1e30f, 1e30f};
        for (int r = 1; r < 64; ++r) {
            for (int dx = -r; dx <= r; ++dx)
                for (int dy = -r; dy <= r; ++dy)
                    for (int dz = -r; dz <= r; ++dz) {
                        if (std::max({std::abs(dx), std::abs(dy), std::abs(dz)}) != r && r > 1) continue;
                        auto it = grid.find(key(c[0] + dx, c[1] + dy, c[2] + dz));
                        if (it == grid.end()) continue;
                        for (int64_t j : it->second) {
                            if (j == i) continue;
                            const float ex = xyz[3 * j] - xyz[3 * i], ey = xyz[3 * j + 1] - xyz[3 * i + 1],
                                        ez = xyz[3 * j + 2] - xyz[3 * i + 2];
                            const float d2 = ex * ex + ey * ey + ez * ez;
                            if (d2 < best[2]) {
                                best[2] = d2;
                                if (best[2] < best[1]) std::swap(best[1], best[2]);
                                if (best[1] < best[0]) std::swap(best[0], best[1]);
                            }
                        }
                    }
            // neighbours within r-1 cells are complete once the third best is closer than (r-1) cells
            if (best[2] < 1e29f && std::sqrt(best[2]) <= (r - 1) * cell) break;
        }
        float sum = 0.f;
        int k = 0;
        for (float b : best)
            if (b < 1e29f) {
                sum += std::sqrt(b);
                ++k;
            }
        out[i] = k ? sum / k : 0.01f;
    }
    return out;
}

struct Trainer {
    MsplatConfig cfg;
    Dataset* ds = nullptr;
    int n = 0, degree = 0, K = 0;
    DevArray<float> params[6], m[6], v[6], stats[3];
    int64_t counts[6] = {};
    float lr[6] = {0.00016f, 0.005f, 0.001f, 0.0025f, 0.000125f, 0.05f};  // model.cpp:142
    bool write_grads = false;  // msplat_trainer_set_write_gradients
    float means_lr_init = 0.00016f, means_lr_final = 0.0000016f;
    int adam_step = 0;
    int current_step = 0;
    int last_w = 0, last_h = 0;  // camera size of the last step (model.cpp:764)
    std::vector<size_t> cam_indices;
    size_t cam_pos = 0;
    std::mt19937 rng{42};
    DevArray<float> gt_full, gt_scaled, img, loss_dev;
    DevArray<uint8_t> rgba;
    float* loss_host = nullptr;  // pinned
    cudaStream_t stream = nullptr;
    // Full-resolution targets of training cameras, double-buffered: while a
    // step computes, the next camera's image is copied into the other buffer
    // on copy_stream (the reference reads images through unified memory and
    // needs no copy, msplat_api.mm / input_data.cpp:17-75).
    DevArray<float> tgt[2];
    long tgt_cam[2] = {-1, -1};
    int tgt_cur = 0;
    cudaEvent_t tgt_ready[2] = {nullptr, nullptr}, tgt_free[2] = {nullptr, nullptr};
    cudaStream_t copy_stream = nullptr;

    ~Trainer() {
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        if (stream) cudaStreamSynchronize(stream);
        for (int b = 0; b < 2; ++b) {
            if (tgt_ready[b]) cudaEventDestroy(tgt_ready[b]);
            if (tgt_free[b]) cudaEventDestroy(tgt_free[b]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
        if (loss_host) cudaFreeHost(loss_host);
        if (stream) cudaStreamDestroy(stream);
    }

    void init_common() {
        K = num_sh_bases(degree) - 1;
        const int64_t d[6] = {3, 2, 4, 3, 3LL * K, 1};
        for (int g = 0; g < 6; ++g) {
            counts[g] = d[g] * n;
            params[g].alloc((size_t)counts[g]);
            m[g].alloc((size_t)counts[g]);
            v[g].alloc((size_t)counts[g]);
        }
        for (auto& s : stats) s.alloc((size_t)n);
        loss_dev.alloc(1);
        CKT(cudaHostAlloc(reinterpret_cast<void**>(&loss_host), sizeof(float), cudaHostAllocDefault));
        CKT(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        CKT(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking));
        for (int b = 0; b < 2; ++b) {
            CKT(cudaEventCreateWithFlags(&tgt_ready[b], cudaEventDisableTiming));
            CKT(cudaEventCreateWithFlags(&tgt_free[b], cudaEventDisableTiming));
            CKT(cudaEventRecord(tgt_free[b], stream));
        }
        cam_indices.resize(ds->train.size());
        std::iota(cam_indices.begin(), cam_indices.end(), 0);
        shuffle();
    }

    void shuffle() {
        std::shuffle(cam_indices.begin(), cam_indices.end(), rng);
        cam_pos = 0;
    }
    size_t next_camera() {
        if (cam_pos >= cam_indices.size()) shuffle();
        return cam_indices[cam_pos++];
    }
    // The camera next_camera() will return (shuffling a little early does not
    // change the order).
    size_t peek_camera() {
        if (cam_pos >= cam_indices.size()) shuffle();
        return cam_indices[cam_pos];
    }

    // Full-resolution target of training camera ci on the device, ordered
    // before the work that `stream` receives next.
    const float* train_target(size_t ci) {
        const Camera& c = ds->train[ci];
        if (!c.image) throw ApiError("camera has no image");
        for (int b = 0; b < 2; ++b)
            if (tgt_cam[b] == (long)ci) {
                CKT(cudaStreamWaitEvent(stream, tgt_ready[b], 0));
                tgt_cur = b;
                return tgt[b].p;
            }
        const int b = 1 - tgt_cur;
        const size_t full = (size_t)c.width * c.height * 3;
        tgt[b].ensure(full);
        tgt_cam[b] = -1;
        CKT(cudaStreamWaitEvent(stream, tgt_free[b], 0));
        CKT(cudaMemcpyAsync(tgt[b].p, c.image, full * sizeof(float), cudaMemcpyHostToDevice, stream));
        tgt_cam[b] = (long)ci;
        tgt_cur = b;
        return tgt[b].p;
    }

    // After the step's work on buffer tgt_cur is enqueued: mark it, and start
    // copying camera ci's target into the other buffer on copy_stream.
    void prefetch_target(size_t ci) {
        CKT(cudaEventRecord(tgt_free[tgt_cur], stream));
        const int b = 1 - tgt_cur;
        if (tgt_cam[b] == (long)ci || tgt_cam[tgt_cur] == (long)ci) return;
        const Camera& c = ds->train[ci];
        if (!c.image) return;
        const size_t full = (size_t)c.width * c.height * 3;
        tgt[b].ensure(full);
        tgt_cam[b] = -1;
        CKT(cudaStreamWaitEvent(copy_stream, tgt_free[b], 0));
        CKT(cudaMemcpyAsync(tgt[b].p, c.image, full * sizeof(float), cudaMemcpyHostToDevice, copy_stream));
        CKT(cudaEventRecord(tgt_ready[b], copy_stream));
        tgt_cam[b] = (long)ci;
    }

    void upload(int g, const float* host) {
        if (counts[g]) CKT(cudaMemcpy(params[g].p, host, counts[g] * sizeof(float), cudaMemcpyHostToDevice));
    }

    MsplatGaussians gaussians() {
        MsplatGaussians G;
        G.num_points = n;
        G.sh_degree = degree;
        G.means = params[0].p;
        G.scales = params[1].p;
        G.quats = params[2].p;
        G.features_dc = params[3].p;
        G.features_rest = K ? params[4].p : nullptr;
        G.opacities = params[5].p;
        return G;
    }

    int downscale_factor(int step) const {  // model.cpp:235-238
        const int remaining = cfg.numDownscales - step / std::max(1, cfg.resolutionSchedule);
        return 1 << std::max(remaining, 0);
    }

    MsplatCamera prepare(const Camera& c, int sf) const {  // model.cpp:500-544
        const float f = (float)sf;
        MsplatCamera cam;
        check_rc(msplat_prepare_camera(c.c2w, c.fx / f, c.fy / f, c.cx / f, c.cy / f,
                                       static_cast<int>(c.width / f), static_cast<int>(c.height / f), &cam));
        return cam;
    }

    // Target image of a camera at downscale factor sf, on the device.
    const float* target(const Camera& c, int sf, const MsplatCamera& cam) {
        if (!c.image) throw ApiError("camera has no image");
        const size_t full = (size_t)c.width * c.height * 3;
        gt_full.ensure(full);
        CKT(cudaMemcpyAsync(gt_full.p, c.image, full * sizeof(float), cudaMemcpyHostToDevice, stream));
        if (sf == 1) return gt_full.p;
        gt_scaled.ensure((size_t)cam.width * cam.height * 3);
        launch_resize_area(gt_full.p, c.width, c.height, gt_scaled.p, cam.width, cam.height, stream);
        return gt_scaled.p;
    }

    MsplatStats step() {  // Trainer::step, msplat_api.mm:106-128
        if (ds->train.empty()) throw ApiError("dataset has no training cameras");
        current_step++;
        const size_t ci = next_camera();
        const Camera& c = ds->train[ci];
        const int sf = downscale_factor(current_step);
        const MsplatCamera cam = prepare(c, sf);
        const float* gt = train_target(ci);
        if (sf != 1) {
            gt_scaled.ensure((size_t)cam.width * cam.height * 3);
            launch_resize_area(gt, c.width, c.height, gt_scaled.p, cam.width, cam.height, stream);
            gt = gt_scaled.p;
        }
        last_w = cam.width;
        last_h = cam.height;
        auto t0 = std::chrono::high_resolution_clock::now();
        adam_step++;
        MsplatAdamState A;
        for (int g = 0; g < 6; ++g) {
            A.exp_avg[g] = m[g].p;
            A.exp_avg_sq[g] = v[g].p;
            A.lr[g] = lr[g];
        }
        A.step = adam_step;
        A.beta1 = 0.9f;
        A.beta2 = 0.999f;
        A.eps = 1e-8f;
        const int degrees_to_use = std::min(current_step / std::max(1, cfg.shDegreeInterval), degree);
        MsplatGaussians G = gaussians();
        check_rc(msplat_train_step_fused(&G, &cam, degrees_to_use, cfg.bgColor, gt, 1.0f - cfg.ssimWeight, 0.0f,
                                         cfg.ssimWeight, &A, stats[0].p, stats[1].p, stats[2].p, loss_dev.p,
                                         write_grads ? 1 : 0, stream));
        prefetch_target(peek_camera());
        // schedulersStep (model.cpp:183-186), then afterTrain (:240-306)
        lr[0] = msplat_means_lr(current_step, cfg.iterations, means_lr_init, means_lr_final);
        CKT(cudaMemcpyAsync(loss_host, loss_dev.p, sizeof(float), cudaMemcpyDeviceToHost, stream));
        after_train(current_step);
        CKT(cudaStreamSynchronize(stream));
        auto t1 = std::chrono::high_resolution_clock::now();
        MsplatStats st;
        st.iteration = current_step;
        st.splatCount = n;
        st.msPerStep = std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count() / 1000.0f;
        st.loss = *loss_host;
        return st;
    }

    int64_t width_of(int g) const {
        const int64_t d[6] = {3, 2, 4, 3, 3LL * K, 1};
        return d[g];
    }

    // Replaces all parameter and moment arrays by `np`/`nm`/`nv` of `count` rows.
    void adopt(int count, DevArray<float> (&np)[6], DevArray<float> (&nm)[6], DevArray<float> (&nv)[6]) {
        for (int g = 0; g < 6; ++g) {
            std::swap(params[g].p, np[g].p);
            std::swap(params[g].n, np[g].n);
            std::swap(m[g].p, nm[g].p);
            std::swap(m[g].n, nm[g].n);
            std::swap(v[g].p, nv[g].p);
            std::swap(v[g].n, nv[g].n);
            counts[g] = width_of(g) * count;
        }
        n = count;
    }

    // Model::afterTrain (model.cpp:240-306): every refineEvery steps after the
    // warm-up, densify (split / duplicate / cull) while below the 250k cap and
    // outside the opacity-reset window, reset opacities once per reset
    // interval, and restart the densification statistics.
    void after_train(int step) {
        const int every = cfg.refineEvery;
        if (every <= 0 || step % every != 0 || step <= cfg.warmupLength) return;
        const int reset_interval = cfg.resetAlphaEvery * every;
        const int stop_split_at = cfg.iterations - 500;
        constexpr int kMaxSplats = 250000;
        const int num_cameras = (int)ds->train.size();
        const bool do_densify = reset_interval > 0 && step < stop_split_at &&
                                step % reset_interval > num_cameras + every && n < kMaxSplats;
        if (do_densify) {
            MsplatDensifyArgs a;
            a.grad_thresh = cfg.densifyGradThresh;
            a.size_thresh = cfg.densifySizeThresh;
            a.screen_thresh = cfg.splitScreenSize;
            a.check_screen = step < cfg.stopScreenSizeAt ? 1 : 0;
            a.cull_alpha_thresh = 0.1f;
            a.cull_scale_thresh = 0.5f;
            a.cull_screen_size = 0.15f;
            a.check_huge = step > every * cfg.resetAlphaEvery ? 1 : 0;
            a.half_max_dim = 0.5f * static_cast<float>(std::max(last_w, last_h));
            a.log_size_fac = std::log(1.6f);
            a.xys_grad_norm = stats[0].p;
            a.vis_counts = stats[1].p;
            a.max_2d_size = stats[2].p;
            MsplatGaussians G = gaussians();
            MsplatDensifyPlan plan;
            check_rc(msplat_densify_plan(&G, &a, &plan, stream));
            DevArray<float> samples;
            if (plan.num_splits > 0) {
                std::vector<float> host(6 * (size_t)plan.num_splits);
                check_rc(msplat_normal_samples((uint32_t)step, (int64_t)host.size(), host.data()));
                samples.alloc(host.size());
                CKT(cudaMemcpy(samples.p, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice));
            }
            const int nn = plan.new_count;
            DevArray<float> np[6], nm[6], nv[6];
            for (int g = 0; g < 6; ++g) {
                np[g].alloc((size_t)(width_of(g) * nn));
                nm[g].alloc((size_t)(width_of(g) * nn));
                nv[g].alloc((size_t)(width_of(g) * nn));
            }
            MsplatGaussians O;
            O.num_points = nn;
            O.sh_degree = degree;
            O.means = np[0].p;
            O.scales = np[1].p;
            O.quats = np[2].p;
            O.features_dc = np[3].p;
            O.features_rest = K ? np[4].p : nullptr;
            O.opacities = np[5].p;
            MsplatAdamState Ain{}, Aout{};
            for (int g = 0; g < 6; ++g) {
                Ain.exp_avg[g] = m[g].p;
                Ain.exp_avg_sq[g] = v[g].p;
                Aout.exp_avg[g] = nm[g].p;
                Aout.exp_avg_sq[g] = nv[g].p;
            }
            check_rc(msplat_densify_apply(&G, &Ain, &a, samples.p, &O, &Aout, stream));
            CKT(cudaStreamSynchronize(stream));
            adopt(nn, np, nm, nv);
        }
        if (reset_interval > 0 && step < stop_split_at && step % reset_interval == every)
            check_rc(msplat_reset_opacity(params[5].p, m[5].p, v[5].p, n, -1.3862943611198906f, stream));
        // xysGradNorm / visCounts / max2DSize are released and re-created
        // zeroed with the current count at the next step (model.cpp:302-304, 771-775)
        CKT(cudaStreamSynchronize(stream));
        for (auto& st : stats) st.alloc((size_t)n);
    }

    // ---- checkpoints: "MSPL" version 1 (model.cpp:341-498) ----
    void write_tensor(std::ofstream& f, const float* dev, std::vector<int64_t> shape) {
        const uint32_t ndim = (uint32_t)shape.size();
        f.write(reinterpret_cast<const char*>(&ndim), sizeof(ndim));
        int64_t numel = 1;
        for (int64_t d : shape) {
            f.write(reinterpret_cast<const char*>(&d), sizeof(d));
            numel *= d;
        }
        const uint64_t bytes = (uint64_t)numel * sizeof(float);
        f.write(reinterpret_cast<const char*>(&bytes), sizeof(bytes));
        std::vector<float> host((size_t)numel);
        if (numel) CKT(cudaMemcpy(host.data(), dev, bytes, cudaMemcpyDeviceToHost));
        f.write(reinterpret_cast<const char*>(host.data()), (std::streamsize)bytes);
    }

    std::vector<std::vector<int64_t>> group_shapes(int count) const {
        return {{count, 3}, {count, 2}, {count, 4}, {count, 3}, {count, K, 3}, {count, 1}};
    }

    void save_checkpoint(const std::string& path) {
        CKT(cudaStreamSynchronize(stream));
        std::ofstream f(path, std::ios::binary);
        if (!f.is_open()) throw ApiError("Cannot open checkpoint file for writing: " + path);
        const uint32_t header[6] = {0x4C50534Du, 1u, (uint32_t)current_step, (uint32_t)n, (uint32_t)degree,
                                    (uint32_t)adam_step};
        f.write(reinterpret_cast<const char*>(header), sizeof(header));
        f.write(reinterpret_cast<const char*>(lr), sizeof(lr));
        f.write(reinterpret_cast<const char*>(&means_lr_init), sizeof(float));
        f.write(reinterpret_cast<const char*>(&means_lr_final), sizeof(float));
        const auto shapes = group_shapes(n);
        for (int g = 0; g < 6; ++g) write_tensor(f, params[g].p, shapes[g]);
        for (int g = 0; g < 6; ++g) write_tensor(f, m[g].p, shapes[g]);
        for (int g = 0; g < 6; ++g) write_tensor(f, v[g].p, shapes[g]);
        if (!f) throw ApiError("error writing checkpoint: " + path);
    }

    int load_checkpoint(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f.is_open()) throw ApiError("Cannot open checkpoint file: " + path);
        uint32_t magic = 0, version = 0;
        f.read(reinterpret_cast<char*>(&magic), 4);
        f.read(reinterpret_cast<char*>(&version), 4);
        if (!f || magic != 0x4C50534Du) throw ApiError("Not a valid msplat checkpoint file");
        if (version != 1) throw ApiError("Unsupported checkpoint version: " + std::to_string(version));
        uint32_t step = 0, num = 0, sh = 0, adam_steps = 0;
        f.read(reinterpret_cast<char*>(&step), 4);
        f.read(reinterpret_cast<char*>(&num), 4);
        f.read(reinterpret_cast<char*>(&sh), 4);
        f.read(reinterpret_cast<char*>(&adam_steps), 4);
        float file_lr[6], lr_init = 0.f, lr_final = 0.f;
        f.read(reinterpret_cast<char*>(file_lr), sizeof(file_lr));
        f.read(reinterpret_cast<char*>(&lr_init), 4);
        f.read(reinterpret_cast<char*>(&lr_final), 4);
        if (!f) throw ApiError("truncated checkpoint: " + path);
        if ((int)sh != degree)
            throw ApiError("checkpoint SH degree " + std::to_string(sh) + " does not match the trainer's " +
                           std::to_string(degree));
        const int count = (int)num;
        const auto shapes = group_shapes(count);
        std::vector<float> data[18];
        for (int k = 0; k < 18; ++k) {
            uint32_t ndim = 0;
            f.read(reinterpret_cast<char*>(&ndim), 4);
            if (!f || ndim > 8) throw ApiError("corrupt checkpoint tensor header: " + path);
            std::vector<int64_t> shape(ndim);
            for (uint32_t d = 0; d < ndim; ++d) f.read(reinterpret_cast<char*>(&shape[d]), 8);
            uint64_t bytes = 0;
            f.read(reinterpret_cast<char*>(&bytes), 8);
            if (!f || shape != shapes[k % 6])
                throw ApiError("checkpoint tensor " + std::to_string(k) + " has an unexpected shape");
            const uint64_t want = (uint64_t)(width_of(k % 6) * count) * sizeof(float);
            if (bytes != want) throw ApiError("checkpoint tensor " + std::to_string(k) + " has an unexpected size");
            data[k].resize(bytes / sizeof(float));
            f.read(reinterpret_cast<char*>(data[k].data()), (std::streamsize)bytes);
            if (!f) throw ApiError("truncated checkpoint: " + path);
        }
        CKT(cudaStreamSynchronize(stream));
        DevArray<float> np[6], nm[6], nv[6];
        DevArray<float>* dst[3] = {np, nm, nv};
        for (int k = 0; k < 18; ++k) {
            DevArray<float>& a = dst[k / 6][k % 6];
            a.alloc(data[k].size());
            if (!data[k].empty())
                CKT(cudaMemcpy(a.p, data[k].data(), data[k].size() * sizeof(float), cudaMemcpyHostToDevice));
        }
        adopt(count, np, nm, nv);
        std::memcpy(lr, file_lr, sizeof(lr));
        means_lr_init = lr_init;
        means_lr_final = lr_final;
        adam_step = (int)adam_steps;
        current_step = (int)step;
        for (auto& st : stats) st.alloc((size_t)n);
        shuffle();  // Trainer::loadCheckpoint re-shuffles (msplat_api.mm:260-265)
        return current_step;
    }

    // ---- exports (save_gaussians.cpp) ----
    std::vector<float> host_group(int g) {
        std::vector<float> h((size_t)counts[g]);
        if (counts[g]) CKT(cudaMemcpy(h.data(), params[g].p, h.size() * sizeof(float), cudaMemcpyDeviceToHost));
        return h;
    }

    // Position in the dataset's original frame when keepCrs is set (the
    // dataset normalised positions by translation and scale).
    float out_pos(const std::vector<float>& means, int64_t i, int axis) const {
        const float v = means[3 * i + axis];
        return cfg.keepCrs ? v / ds->scale + ds->translation[axis] : v;
    }

    // 2DGS PLY (the reference's saveGaussianPly format,
    // core/src/loaders/save_gaussians.cpp:11-58): binary little-endian
    // vertices with the property list below; f_rest is stored channel-major
    // ([3, bases]) and normals are zero. Built as a column table, written with
    // one call.
    void export_ply(const std::string& path) {
        CKT(cudaStreamSynchronize(stream));
        std::vector<std::string> props = {"x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"};
        for (int k = 0; k < 3 * K; ++k) props.push_back("f_rest_" + std::to_string(k));
        props.push_back("opacity");
        props.push_back("scale_0");
        props.push_back("scale_1");
        for (int k = 0; k < 4; ++k) props.push_back("rot_" + std::to_string(k));
        const size_t stride = props.size();
        const std::vector<float> means = host_group(0), log_scales = host_group(1), quats = host_group(2),
                                 dc = host_group(3), rest = host_group(4), opac = host_group(5);
        std::vector<float> table((size_t)n * stride, 0.0f);
        for (int64_t i = 0; i < n; ++i) {
            float* v = &table[(size_t)i * stride];
            for (int axis = 0; axis < 3; ++axis) v[axis] = out_pos(means, i, axis);  // normals (3..5) stay 0
            for (int ch = 0; ch < 3; ++ch) {
                v[6 + ch] = dc[3 * i + ch];
                for (int b = 0; b < K; ++b) v[9 + ch * K + b] = rest[((size_t)i * K + b) * 3 + ch];
            }
            float* tail = v + 9 + 3 * K;
            tail[0] = opac[i];
            for (int k = 0; k < 2; ++k) {
                const float ls = log_scales[2 * i + k];
                tail[1 + k] = cfg.keepCrs ? std::log(std::exp(ls) / ds->scale) : ls;
            }
            for (int k = 0; k < 4; ++k) tail[3 + k] = quats[4 * i + k];
        }
        std::string header = "ply\nformat binary_little_endian 1.0\ncomment msplat v" + std::to_string(current_step) +
                             "\nelement vertex " + std::to_string(n) + "\n";
        for (const std::string& name : props) header += "property float " + name + "\n";
        header += "end_header\n";
        std::ofstream o(path, std::ios::binary);
        if (!o.is_open()) throw ApiError("Cannot open PLY file for writing: " + path);
        o.write(header.data(), (std::streamsize)header.size());
        o.write(reinterpret_cast<const char*>(table.data()), (std::streamsize)(table.size() * sizeof(float)));
        if (!o) throw ApiError("error writing PLY: " + path);
    }

    // .splat (the 32-byte-per-splat web viewer format the reference writes,
    // core/src/loaders/save_gaussians.cpp:60-111): float position, float
    // scale (a flat disc: third axis 1e-5), RGBA8 colour (SH DC through
    // 0.5 + C0 dc, alpha = sigmoid(opacity)), quaternion quantised to q * 128 +
    // 128; splats ordered by (sum of scales) x opacity, largest first, as the
    // reference orders them.
    struct SplatRecord {
        float pos[3];
        float scale[3];
        uint8_t rgba[4];
        uint8_t rot[4];
    };
    static_assert(sizeof(SplatRecord) == 32, "splat records are 32 bytes");

    static uint8_t quantise_u8(double x) { return (uint8_t)std::min(255.0, std::max(0.0, x)); }

    void export_splat(const std::string& path) {
        CKT(cudaStreamSynchronize(stream));
        const std::vector<float> means = host_group(0), log_scales = host_group(1), quats = host_group(2),
                                 dc = host_group(3), opac = host_group(5);
        std::vector<SplatRecord> recs((size_t)n);
        std::vector<float> importance((size_t)n);
        for (int64_t i = 0; i < n; ++i) {
            SplatRecord& r = recs[(size_t)i];
            const float opacity = 1.0f / (1.0f + std::exp(-opac[i]));
            float size = 0.0f;
            for (int axis = 0; axis < 3; ++axis) r.pos[axis] = out_pos(means, i, axis);
            for (int k = 0; k < 2; ++k) {
                float e = std::exp(log_scales[2 * i + k]);
                size += e;
                r.scale[k] = cfg.keepCrs ? e / ds->scale : e;
            }
            r.scale[2] = 1e-5f;
            importance[(size_t)i] = (cfg.keepCrs ? size / ds->scale : size) / (1.0f + std::exp(-opac[i]));
            for (int ch = 0; ch < 3; ++ch) r.rgba[ch] = quantise_u8(((double)dc[3 * i + ch] * kC0 + 0.5) * 255.0);
            r.rgba[3] = quantise_u8((double)(opacity * 255.0f));
            for (int k = 0; k < 4; ++k) r.rot[k] = quantise_u8((double)(quats[4 * i + k] * 128.0f + 128.0f));
        }
        std::vector<int64_t> order((size_t)n);
        std::iota(order.begin(), order.end(), (int64_t)0);
        std::sort(order.begin(), order.end(),
                  [&](int64_t x, int64_t y) { return importance[(size_t)x] > importance[(size_t)y]; });
        std::vector<SplatRecord> sorted;
        sorted.reserve((size_t)n);
        for (int64_t i : order) sorted.push_back(recs[(size_t)i]);
        std::ofstream o(path, std::ios::binary);
        if (!o.is_open()) throw ApiError("Cannot open .splat file for writing: " + path);
        o.write(reinterpret_cast<const char*>(sorted.data()), (std::streamsize)(sorted.size() * sizeof(SplatRecord)));
        if (!o) throw ApiError("error writing .splat: " + path);
    }

    // Renders a camera; returns the device image and its camera.
    const float* render_cam(const Camera& c, int step, MsplatCamera* out_cam) {
        const int sf = downscale_factor(step);
        const MsplatCamera cam = prepare(c, sf);
        img.ensure((size_t)cam.width * cam.height * 3);
        const int degrees_to_use = std::min(step / std::max(1, cfg.shDegreeInterval), degree);
        MsplatGaussians G = gaussians();
        check_rc(msplat_render(&G, &cam, 1.0f, 0.01f, degrees_to_use, cfg.bgColor, img.p, stream));
        if (out_cam) *out_cam = cam;
        return img.p;
    }

    MsplatPixelBuffer to_host(const float* dev, const MsplatCamera& cam) {
        const size_t bytes = (size_t)cam.width * cam.height * 3 * sizeof(float);
        float* buf = static_cast<float*>(std::malloc(bytes));
        if (!buf) throw ApiError("out of host memory");
        CKT(cudaMemcpyAsync(buf, dev, bytes, cudaMemcpyDeviceToHost, stream));
        CKT(cudaStreamSynchronize(stream));
        return MsplatPixelBuffer{buf, cam.width, cam.height};
    }
};

// SSIM for evaluation (core/src/ssim.cpp:61-123): 11-tap sigma-1.5 window,
// clamp-to-edge padding (unlike the training loss, which zero-pads).
double ssim_eval(const std::vector<float>& r, const std::vector<float>& g, int H, int W) {
    float kern[11], ks = 0.f;
    for (int i = 0; i < 11; ++i) {
        const float x = (float)(i - 5);
        kern[i] = std::exp(-(x * x) / (2.0f * 1.5f * 1.5f));
        ks += kern[i];
    }
    for (float& k : kern) k /= ks;
    const int HW = H * W;
    std::vector<float> a(HW), b(HW), aa(HW), bb(HW), ab(HW), tmp(HW), m1(HW), m2(HW), s11(HW), s22(HW), s12(HW);
    auto blur = [&](const std::vector<float>& in, std::vector<float>& out) {
        for (int y = 0; y < H; ++y)
            for (int x = 0; x < W; ++x) {
                float s = 0;
                for (int k = 0; k < 11; ++k) s += in[y * W + std::min(std::max(x + k - 5, 0), W - 1)] * kern[k];
                tmp[y * W + x] = s;
            }
        for (int y = 0; y < H; ++y)
            for (int x = 0; x < W; ++x) {
                float s = 0;
                for (int k = 0; k < 11; ++k) s += tmp[std::min(std::max(y + k - 5, 0), H - 1) * W + x] * kern[k];
                out[y * W + x] = s;
            }
    };
    const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
    double sum = 0;
    for (int c = 0; c < 3; ++c) {
        for (int i = 0; i < HW; ++i) {
            a[i] = r[3 * i + c];
            b[i] = g[3 * i + c];
            aa[i] = a[i] * a[i];
            bb[i] = b[i] * b[i];
            ab[i] = a[i] * b[i];
        }
        blur(a, m1);
        blur(b, m2);
        blur(aa, s11);
        blur(bb, s22);
        blur(ab, s12);
        for (int i = 0; i < HW; ++i) {
            const float q11 = m1[i] * m1[i], q22 = m2[i] * m2[i], q12 = m1[i] * m2[i];
            const float num = (2.0f * q12 + C1) * (2.0f * (s12[i] - q12) + C2);
            const float den = (q11 + q22 + C1) * ((s11[i] - q11) + (s22[i] - q22) + C2);
            sum += num / den;
        }
    }
    return sum / (3.0 * HW);
}

template <typename R, typename F>
R api(R fallback, F&& f) {
    try {
        R r = f();
        set_last_error("");
        return r;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return fallback;
    }
}

Trainer* T(MsplatTrainer t) {
    if (!t) throw ApiError("null trainer");
    return static_cast<Trainer*>(t);
}
Dataset* D(MsplatDataset d) {
    if (!d) throw ApiError("null dataset");
    return static_cast<Dataset*>(d);
}

}  // namespace
}  // namespace msplat

using namespace msplat;

extern "C" {

MsplatDataset msplat_dataset_create(const char* path, float, bool, int) {
    set_last_error(
        (std::string("dataset loaders (COLMAP, Nerfstudio, Polycam) are not part of this build; cannot load '") +
         (path ? path : "") + "'; use msplat_dataset_create_from_memory")
            .c_str());
    return nullptr;
}

MsplatDataset msplat_dataset_create_from_memory(int numCameras, const float* camToWorld, const float* intrinsics,
                                                int width, int height, const float* images, int numPoints,
                                                const float* xyz, const uint8_t* rgb, bool evalMode,
                                                int testEvery) {
    return api<MsplatDataset>(nullptr, [&]() -> MsplatDataset {
        if (numCameras < 0 || (numCameras > 0 && (!camToWorld || !intrinsics)) || width <= 0 || height <= 0 ||
            numPoints < 0 || (numPoints > 0 && (!xyz || !rgb)))
            throw ApiError("bad dataset arguments");
        auto* ds = new Dataset();
        const size_t img = (size_t)width * height * 3;
        for (int i = 0; i < numCameras; ++i) {
            Camera c;
            std::memcpy(c.c2w, camToWorld + 16 * (size_t)i, sizeof(c.c2w));
            c.fx = intrinsics[4 * i];
            c.fy = intrinsics[4 * i + 1];
            c.cx = intrinsics[4 * i + 2];
            c.cy = intrinsics[4 * i + 3];
            c.width = width;
            c.height = height;
            if (images) {
                float* p = nullptr;
                cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&p), img * sizeof(float), cudaHostAllocDefault);
                if (e != cudaSuccess) {
                    delete ds;
                    throw ApiError(std::string("cudaHostAlloc: ") + cudaGetErrorString(e));
                }
                std::memcpy(p, images + img * i, img * sizeof(float));
                ds->pinned.push_back(p);
                c.image = p;
            }
            // InputData::splitTrainTest: every testEvery-th camera is a test camera
            if (evalMode && testEvery > 0 && i % testEvery == 0)
                ds->test.push_back(c);
            else
                ds->train.push_back(c);
        }
        ds->xyz.assign(xyz, xyz + 3 * (size_t)numPoints);
        ds->rgb.assign(rgb, rgb + 3 * (size_t)numPoints);
        return ds;
    });
}

void msplat_dataset_destroy(MsplatDataset ds) { delete static_cast<Dataset*>(ds); }
int msplat_dataset_num_train(MsplatDataset ds) { return api<int>(0, [&] { return (int)D(ds)->train.size(); }); }
int msplat_dataset_num_test(MsplatDataset ds) { return api<int>(0, [&] { return (int)D(ds)->test.size(); }); }
void msplat_dataset_camera_pose(MsplatDataset ds, int i, float camToWorld[16]) {
    api<int>(0, [&] {
        Dataset* d = D(ds);
        if (i >= 0 && i < (int)d->train.size()) std::memcpy(camToWorld, d->train[i].c2w, 16 * sizeof(float));
        return 0;
    });
}

MsplatTrainer msplat_trainer_create(MsplatDataset dsh, MsplatConfig config) {
    return api<MsplatTrainer>(nullptr, [&]() -> MsplatTrainer {
        Dataset* ds = D(dsh);
        if (config.shDegree < 0 || config.shDegree > 3) throw ApiError("shDegree must be 0..3");
        auto* t = new Trainer();
        try {
            t->cfg = config;
            t->ds = ds;
            t->n = (int)(ds->xyz.size() / 3);
            t->degree = config.shDegree;
            t->init_common();
            const int n = t->n, K = t->K;
            // Model::Model, model.cpp:61-113
            std::vector<float> scales(2 * (size_t)n), quats(4 * (size_t)n), dc(3 * (size_t)n),
                rest((size_t)3 * K * n, 0.f), opac(n, std::log(0.1f / 0.9f));
            const std::vector<float> knn = knn_mean_distance(ds->xyz);
            for (int i = 0; i < n; ++i) scales[2 * i] = scales[2 * i + 1] = std::log(knn[i]);
            std::mt19937 rng(42);
            std::uniform_real_distribution<float> U(0.0f, 1.0f);
            for (int i = 0; i < n; ++i) {
                const float u = U(rng), vv = U(rng), w = U(rng);
                quats[4 * i + 0] = std::sqrt(1 - u) * std::sin(2 * M_PI * vv);
                quats[4 * i + 1] = std::sqrt(1 - u) * std::cos(2 * M_PI * vv);
                quats[4 * i + 2] = std::sqrt(u) * std::sin(2 * M_PI * w);
                quats[4 * i + 3] = std::sqrt(u) * std::cos(2 * M_PI * w);
            }
            for (int i = 0; i < 3 * n; ++i) dc[i] = (float)((ds->rgb[i] / 255.0 - 0.5) / kC0);
            t->upload(0, ds->xyz.data());
            t->upload(1, scales.data());
            t->upload(2, quats.data());
            t->upload(3, dc.data());
            t->upload(4, rest.data());
            t->upload(5, opac.data());
        } catch (...) {
            delete t;
            throw;
        }
        return t;
    });
}

MsplatTrainer msplat_trainer_create_from_params(MsplatDataset dsh, MsplatConfig config, int numPoints,
                                                const float* means, const float* scales, const float* quats,
                                                const float* opacities, const float* featuresDc,
                                                const float* featuresRest) {
    return api<MsplatTrainer>(nullptr, [&]() -> MsplatTrainer {
        Dataset* ds = D(dsh);
        if (config.shDegree < 0 || config.shDegree > 3) throw ApiError("shDegree must be 0..3");
        if (numPoints < 0 || (numPoints > 0 && (!means || !scales || !quats || !opacities || !featuresDc)) ||
            (numPoints > 0 && config.shDegree > 0 && !featuresRest))
            throw ApiError("bad parameter arrays");
        auto* t = new Trainer();
        try {
            t->cfg = config;
            t->ds = ds;
            t->n = numPoints;
            t->degree = config.shDegree;
            t->init_common();
            t->upload(0, means);
            t->upload(1, scales);
            t->upload(2, quats);
            t->upload(3, featuresDc);
            if (t->K) t->upload(4, featuresRest);
            t->upload(5, opacities);
        } catch (...) {
            delete t;
            throw;
        }
        return t;
    });
}

void msplat_trainer_destroy(MsplatTrainer t) { delete static_cast<Trainer*>(t); }

MsplatStats msplat_trainer_step(MsplatTrainer t) {
    return api<MsplatStats>(MsplatStats{0, 0, 0.f, 0.f}, [&] { return T(t)->step(); });
}

void msplat_trainer_train(MsplatTrainer t) {
    api<int>(0, [&] {
        Trainer* tr = T(t);
        while (tr->current_step < tr->cfg.iterations) tr->step();
        return 0;
    });
}

MsplatEvalMetrics msplat_trainer_evaluate(MsplatTrainer t) {
    return api<MsplatEvalMetrics>(MsplatEvalMetrics{0, 0, 0, 0, 0}, [&] {
        Trainer* tr = T(t);
        MsplatEvalMetrics mtr{0, 0, 0, 0, tr->n};
        const auto& cams = tr->ds->test;
        if (cams.empty()) return mtr;
        double sp = 0, ss = 0, sl = 0;
        for (const Camera& c : cams) {
            MsplatCamera cam;
            const float* dev = tr->render_cam(c, tr->cfg.iterations, &cam);
            const size_t e = (size_t)cam.width * cam.height * 3;
            std::vector<float> r(e), g(e);
            CKT(cudaMemcpyAsync(r.data(), dev, e * 4, cudaMemcpyDeviceToHost, tr->stream));
            const float* gt = tr->target(c, tr->downscale_factor(tr->cfg.iterations), cam);
            CKT(cudaMemcpyAsync(g.data(), gt, e * 4, cudaMemcpyDeviceToHost, tr->stream));
            CKT(cudaStreamSynchronize(tr->stream));
            double mse = 0, l1 = 0;
            for (size_t i = 0; i < e; ++i) {
                const double d = (double)r[i] - g[i];
                mse += d * d;
                l1 += std::fabs(d);
            }
            sp += 10.0 * std::log10(1.0 / (mse / e));  // model.cpp:25-32
            sl += l1 / e;
            ss += ssim_eval(r, g, cam.height, cam.width);
        }
        mtr.psnr = (float)(sp / cams.size());
        mtr.ssim = (float)(ss / cams.size());
        mtr.l1 = (float)(sl / cams.size());
        mtr.numTest = (int)cams.size();
        return mtr;
    });
}

MsplatPixelBuffer msplat_trainer_render(MsplatTrainer t, int cameraIndex, bool useTest) {
    return api<MsplatPixelBuffer>(MsplatPixelBuffer{nullptr, 0, 0}, [&] {
        Trainer* tr = T(t);
        const auto& cams = useTest ? tr->ds->test : tr->ds->train;
        if (cameraIndex < 0 || cameraIndex >= (int)cams.size()) return MsplatPixelBuffer{nullptr, 0, 0};
        MsplatCamera cam;
        const float* dev = tr->render_cam(cams[cameraIndex], tr->current_step, &cam);
        return tr->to_host(dev, cam);
    });
}

MsplatPixelBuffer msplat_trainer_render_pose(MsplatTrainer t, const float camToWorld[16], int refCameraIndex) {
    return api<MsplatPixelBuffer>(MsplatPixelBuffer{nullptr, 0, 0}, [&] {
        Trainer* tr = T(t);
        const auto& cams = tr->ds->train;
        if (refCameraIndex < 0 || refCameraIndex >= (int)cams.size()) return MsplatPixelBuffer{nullptr, 0, 0};
        Camera c = cams[refCameraIndex];
        std::memcpy(c.c2w, camToWorld, sizeof(c.c2w));
        MsplatCamera cam;
        const float* dev = tr->render_cam(c, tr->current_step, &cam);
        return tr->to_host(dev, cam);
    });
}

void msplat_trainer_render_pose_to_buffer(MsplatTrainer t, const float camToWorld[16], int refCameraIndex,
                                          uint8_t* outRGBA, int* outWidth, int* outHeight) {
    api<int>(0, [&] {
        Trainer* tr = T(t);
        const auto& cams = tr->ds->train;
        if (refCameraIndex < 0 || refCameraIndex >= (int)cams.size()) {
            *outWidth = 0;
            *outHeight = 0;
            return 0;
        }
        Camera c = cams[refCameraIndex];
        std::memcpy(c.c2w, camToWorld, sizeof(c.c2w));
        const int sf = tr->downscale_factor(tr->current_step);
        *outWidth = static_cast<int>(c.width / (float)sf);
        *outHeight = static_cast<int>(c.height / (float)sf);
        if (!outRGBA) return 0;
        MsplatCamera cam;
        const float* dev = tr->render_cam(c, tr->current_step, &cam);
        const int64_t px = (int64_t)cam.width * cam.height;
        tr->rgba.ensure((size_t)px * 4);
        launch_rgba8(dev, tr->rgba.p, px, tr->stream);
        CKT(cudaMemcpyAsync(outRGBA, tr->rgba.p, (size_t)px * 4, cudaMemcpyDeviceToHost, tr->stream));
        CKT(cudaStreamSynchronize(tr->stream));
        return 0;
    });
}

static void not_in_build(const char* what) {
    set_last_error((std::string(what) + " is not part of this build").c_str());
}

void msplat_trainer_export_ply(MsplatTrainer t, const char* path) {
    api<int>(0, [&] {
        if (!path) throw ApiError("null path");
        T(t)->export_ply(path);
        return 0;
    });
}
void msplat_trainer_export_splat(MsplatTrainer t, const char* path) {
    api<int>(0, [&] {
        if (!path) throw ApiError("null path");
        T(t)->export_splat(path);
        return 0;
    });
}
int64_t msplat_trainer_extract_mesh(MsplatTrainer, const char*, float, float, float, float) {
    not_in_build("mesh extraction (TSDF + marching cubes)");
    return -1;
}
void msplat_trainer_save_checkpoint(MsplatTrainer t, const char* path) {
    api<int>(0, [&] {
        if (!path) throw ApiError("null path");
        T(t)->save_checkpoint(path);
        return 0;
    });
}
int msplat_trainer_load_checkpoint(MsplatTrainer t, const char* path) {
    return api<int>(-1, [&] {
        if (!path) throw ApiError("null path");
        return T(t)->load_checkpoint(path);
    });
}
int msplat_trainer_splat_count(MsplatTrainer t) { return api<int>(0, [&] { return T(t)->n; }); }
int msplat_trainer_iteration(MsplatTrainer t) { return api<int>(0, [&] { return T(t)->current_step; }); }

int msplat_trainer_set_write_gradients(MsplatTrainer t, int enable) {
    return api<int>(-1, [&] {
        T(t)->write_grads = enable != 0;
        return 0;
    });
}

int msplat_trainer_get_params(MsplatTrainer t, float* means, float* scales, float* quats, float* opacities,
                              float* featuresDc, float* featuresRest) {
    return api<int>(-1, [&] {
        Trainer* tr = T(t);
        float* outs[6] = {means, scales, quats, featuresDc, featuresRest, opacities};
        CKT(cudaStreamSynchronize(tr->stream));
        for (int g = 0; g < 6; ++g)
            if (outs[g] && tr->counts[g])
                CKT(cudaMemcpy(outs[g], tr->params[g].p, tr->counts[g] * sizeof(float), cudaMemcpyDeviceToHost));
        return 0;
    });
}

void msplat_set_metallib_path(const char*) {}
void msplat_sync(void) { cudaDeviceSynchronize(); }
void msplat_cleanup(void) { msplat_backend_cleanup(); }

}  // extern "C"
