// densify.cu — densification (split / duplicate / cull / compact) and the
// opacity reset of Model::afterTrain (core/src/model.cpp:240-306).
//
// The reference runs densify_classify_kernel, two block scans, the split and
// duplicate append kernels, densify_cull_classify_kernel, a scan of the keep
// flags and 18 scatter + copy-back passes over buffers sized for 3N
// (core/metal/msplat_metal.mm:1339-1594, msplat_metal.metal:3231-3491). Here
// every Gaussian's fate is known from its own data, so one kernel decides
// everything per original Gaussian (its own survival, its two children's and
// its duplicate's) and emits four counts; one scan turns them into output
// positions; after the host reads the totals, one kernel writes the survivors,
// the children and the duplicates, parameters and moments, straight into
// arrays of the final size. Compiled with -fmad=false: with det_exp and IEEE
// division/square root the results are bit-identical to the CPU restatement.
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>

#include "msplat_backend.h"
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

constexpr int kScanBlock = 1024;
constexpr uint8_t kSplit = 1, kDup = 2, kKeepOrig = 4, kKeepChild = 8, kKeepDup = 16;

__device__ __forceinline__ float sigmoid_det(float x) { return 1.0f / (1.0f + det_exp(-x)); }
__device__ __forceinline__ float max_exp2(float s0, float s1) { return fmaxf(det_exp(s0), det_exp(s1)); }

struct ClassifyArgs {
    int n;
    MsplatDensifyArgs a;
    const float* scales;     // [n, 2]
    const float* opacities;  // [n]
    uint8_t* flags;          // [n]
    int4* counts;            // [n] (kept original, kept children, kept duplicate, split)
    int* num_dups;           // [1] (+=)
};

// densify_classify_kernel (metal:3231-3263) and densify_cull_classify_kernel
// (metal:3408-3441) evaluated for an original Gaussian and for the children
// and duplicate it would produce.
__global__ void __launch_bounds__(256) k_densify_classify(ClassifyArgs c) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= c.n) return;
    const MsplatDensifyArgs& a = c.a;
    const float s0 = c.scales[2 * i], s1 = c.scales[2 * i + 1];
    const float max2d = a.max_2d_size[i];
    bool split = false, dup = false;
    const float vc = a.vis_counts[i];
    const float ms = max_exp2(s0, s1);
    if (vc > 0.0f) {
        const float avg_grad = (a.xys_grad_norm[i] / vc) * a.half_max_dim;
        const bool high_grad = avg_grad > a.grad_thresh;
        const bool is_large = ms > a.size_thresh;
        split = is_large;
        if (a.check_screen && max2d > a.screen_thresh) split = true;
        split = split && high_grad;
        dup = !is_large && high_grad;
    }
    // split parents shrink in place before duplicates copy them (metal:3330-3332)
    const float sc0 = s0 - a.log_size_fac, sc1 = s1 - a.log_size_fac;
    const float ms_child = max_exp2(sc0, sc1);
    const bool faint = sigmoid_det(c.opacities[i]) < a.cull_alpha_thresh;
    bool cull_orig = faint || split;
    if (a.check_huge) {
        if (ms > a.cull_scale_thresh) cull_orig = true;
        if (a.check_screen && max2d > a.cull_screen_size) cull_orig = true;
    }
    const bool cull_child = faint || (a.check_huge && ms_child > a.cull_scale_thresh);
    const float ms_dup = split ? ms_child : ms;
    const bool cull_dup = faint || (a.check_huge && ms_dup > a.cull_scale_thresh);
    uint8_t f = 0;
    if (split) f |= kSplit;
    if (dup) f |= kDup;
    if (!cull_orig) f |= kKeepOrig;
    if (!cull_child) f |= kKeepChild;
    if (!cull_dup) f |= kKeepDup;
    c.flags[i] = f;
    c.counts[i] = make_int4(cull_orig ? 0 : 1, (split && !cull_child) ? 2 : 0, (dup && !cull_dup) ? 1 : 0,
                            split ? 1 : 0);
    if (dup) atomicAdd(c.num_dups, 1);
}

__device__ __forceinline__ int4 add4(int4 a, int4 b) { return make_int4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

// Block-wide exclusive scan of int4 over kScanBlock threads; returns the
// block total through *total.
__device__ int4 block_exclusive_scan(int4 v, int4* total) {
    __shared__ int4 warp_tot[kScanBlock / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int4 inc = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        int4 o;
        o.x = __shfl_up_sync(0xffffffffu, inc.x, d);
        o.y = __shfl_up_sync(0xffffffffu, inc.y, d);
        o.z = __shfl_up_sync(0xffffffffu, inc.z, d);
        o.w = __shfl_up_sync(0xffffffffu, inc.w, d);
        if (lane >= d) inc = add4(inc, o);
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int4 t = warp_tot[lane];
        int4 ti = t;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            int4 o;
            o.x = __shfl_up_sync(0xffffffffu, ti.x, d);
            o.y = __shfl_up_sync(0xffffffffu, ti.y, d);
            o.z = __shfl_up_sync(0xffffffffu, ti.z, d);
            o.w = __shfl_up_sync(0xffffffffu, ti.w, d);
            if (lane >= d) ti = add4(ti, o);
        }
        warp_tot[lane] = make_int4(ti.x - t.x, ti.y - t.y, ti.z - t.z, ti.w - t.w);  // exclusive
        if (lane == 31) *total = ti;
    }
    __syncthreads();
    const int4 wbase = warp_tot[warp];
    return make_int4(wbase.x + inc.x - v.x, wbase.y + inc.y - v.y, wbase.z + inc.z - v.z, wbase.w + inc.w - v.w);
}

// Exclusive scan within blocks of kScanBlock elements, plus block totals.
__global__ void __launch_bounds__(kScanBlock) k_scan_blocks(const int4* counts, int n, int4* prefix, int4* btot) {
    __shared__ int4 total;
    const int i = blockIdx.x * kScanBlock + threadIdx.x;
    const int4 v = i < n ? counts[i] : make_int4(0, 0, 0, 0);
    const int4 ex = block_exclusive_scan(v, &total);
    if (i < n) prefix[i] = ex;
    __syncthreads();
    if (threadIdx.x == 0) btot[blockIdx.x] = total;
}

// Exclusive scan of the block totals (one CTA walks them in chunks) and the
// grand totals.
__global__ void __launch_bounds__(kScanBlock) k_scan_totals(int4* btot, int nb, int4* grand) {
    __shared__ int4 total;
    int4 carry = make_int4(0, 0, 0, 0);
    for (int base = 0; base < nb; base += kScanBlock) {
        const int b = base + threadIdx.x;
        const int4 v = b < nb ? btot[b] : make_int4(0, 0, 0, 0);
        const int4 ex = block_exclusive_scan(v, &total);
        __syncthreads();
        if (b < nb) btot[b] = add4(carry, ex);
        carry = add4(carry, total);
        __syncthreads();
    }
    if (threadIdx.x == 0) *grand = carry;
}

struct BuildArgs {
    int n, K3;
    MsplatDensifyArgs a;
    const float* src[6];
    const float* src_m[6];
    const float* src_v[6];
    float* dst[6];
    float* dst_m[6];
    float* dst_v[6];
    const uint8_t* flags;
    const int4* prefix;
    const int4* boff;
    const int4* grand;
    const float* random_samples;
};

__device__ __forceinline__ void copy_row(const float* src, float* dst, int w, int from, int to) {
    for (int j = 0; j < w; ++j) dst[(size_t)to * w + j] = src[(size_t)from * w + j];
}
__device__ __forceinline__ void zero_row(float* dst, int w, int to) {
    for (int j = 0; j < w; ++j) dst[(size_t)to * w + j] = 0.0f;
}

// densify_append_split_kernel (metal:3265-3340), densify_append_dup_kernel
// (:3342-3394) and the compaction (:3443-3478) in one pass: row i of the input
// goes to its survivor slot, its children and its duplicate to theirs.
__global__ void __launch_bounds__(256) k_densify_build(BuildArgs b) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= b.n) return;
    const int w[6] = {3, 2, 4, 3, b.K3, 1};
    const uint8_t f = b.flags[i];
    const int4 pre = add4(b.prefix[i], b.boff[i / kScanBlock]);
    const int4 tot = *b.grand;
    if (f & kKeepOrig) {
        for (int g = 0; g < 6; ++g) {
            if (w[g] == 0) continue;
            copy_row(b.src[g], b.dst[g], w[g], i, pre.x);
            copy_row(b.src_m[g], b.dst_m[g], w[g], i, pre.x);
            copy_row(b.src_v[g], b.dst_v[g], w[g], i, pre.x);
        }
    }
    const float lsf = b.a.log_size_fac;
    const float* sc = b.src[1] + 2 * (size_t)i;
    if ((f & kSplit) && (f & kKeepChild)) {
        const int ord = pre.w;
        const float* q = b.src[2] + 4 * (size_t)i;
        float qw = q[0], qx = q[1], qy = q[2], qz = q[3];
        const float qlen = sqrtf(qw * qw + qx * qx + qy * qy + qz * qz);
        qw /= qlen; qx /= qlen; qy /= qlen; qz /= qlen;
        const float sx = det_exp(sc[0]), sy = det_exp(sc[1]), sz = 0.0f;  // 2DGS: no third axis
        const float* mp = b.src[0] + 3 * (size_t)i;
        for (int k = 0; k < 2; ++k) {
            const int child = tot.x + pre.y + k;
            const float* rs = b.random_samples + (size_t)(ord * 2 + k) * 3;
            const float r0 = rs[0] * sx, r1 = rs[1] * sy, r2 = rs[2] * sz;
            const float v0 = (1 - 2 * (qy * qy + qz * qz)) * r0 + 2 * (qx * qy - qw * qz) * r1 + 2 * (qx * qz + qw * qy) * r2;
            const float v1 = 2 * (qx * qy + qw * qz) * r0 + (1 - 2 * (qx * qx + qz * qz)) * r1 + 2 * (qy * qz - qw * qx) * r2;
            const float v2 = 2 * (qx * qz - qw * qy) * r0 + 2 * (qy * qz + qw * qx) * r1 + (1 - 2 * (qx * qx + qy * qy)) * r2;
            float* md = b.dst[0] + 3 * (size_t)child;
            md[0] = mp[0] + v0;
            md[1] = mp[1] + v1;
            md[2] = mp[2] + v2;
            b.dst[1][2 * (size_t)child] = sc[0] - lsf;
            b.dst[1][2 * (size_t)child + 1] = sc[1] - lsf;
            for (int g = 2; g < 6; ++g)
                if (w[g]) copy_row(b.src[g], b.dst[g], w[g], i, child);
            for (int g = 0; g < 6; ++g) {
                if (w[g] == 0) continue;
                zero_row(b.dst_m[g], w[g], child);
                zero_row(b.dst_v[g], w[g], child);
            }
        }
    }
    if ((f & kDup) && (f & kKeepDup)) {
        const int d = tot.x + tot.y + pre.z;
        for (int g = 0; g < 6; ++g) {
            if (w[g] == 0) continue;
            if (g == 1 && (f & kSplit)) {
                b.dst[1][2 * (size_t)d] = sc[0] - lsf;
                b.dst[1][2 * (size_t)d + 1] = sc[1] - lsf;
            } else {
                copy_row(b.src[g], b.dst[g], w[g], i, d);
            }
            zero_row(b.dst_m[g], w[g], d);
            zero_row(b.dst_v[g], w[g], d);
        }
    }
}

__global__ void k_reset_opacity(float* op, float* m, float* v, int n, float max_logit) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (op[i] > max_logit) op[i] = max_logit;
    if (m) m[i] = 0.0f;
    if (v) v[i] = 0.0f;
}

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CKD(call)                                                                                   \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess)                                                                      \
            throw Error(MSPLAT_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));       \
    } while (0)

// Per-device decisions kept between plan and apply.
struct Plan {
    int n = 0, num_splits = 0, new_count = 0;
    void* mem = nullptr;
    size_t bytes = 0;
    uint8_t* flags = nullptr;
    int4 *counts = nullptr, *prefix = nullptr, *btot = nullptr, *grand = nullptr;
    int* num_dups = nullptr;
    int4* h_grand = nullptr;  // pinned
    int* h_dups = nullptr;    // pinned

    void ensure(int count) {
        const int nb = (count + kScanBlock - 1) / kScanBlock;
        const size_t need = 3 * sizeof(int4) * (size_t)count + sizeof(int4) * ((size_t)nb + 1) + 256 +
                            (size_t)count + 64;
        if (need > bytes) {
            if (mem) cudaFree(mem);
            mem = nullptr;
            bytes = 0;
            CKD(cudaMalloc(&mem, need));
            bytes = need;
        }
        char* p = static_cast<char*>(mem);
        counts = reinterpret_cast<int4*>(p); p += sizeof(int4) * (size_t)count;
        prefix = reinterpret_cast<int4*>(p); p += sizeof(int4) * (size_t)count;
        btot = reinterpret_cast<int4*>(p); p += sizeof(int4) * (size_t)count;  // >= nb entries
        grand = reinterpret_cast<int4*>(p); p += sizeof(int4) * ((size_t)nb + 1);
        num_dups = reinterpret_cast<int*>(p); p += 256;
        flags = reinterpret_cast<uint8_t*>(p);
        if (!h_grand) CKD(cudaHostAlloc(reinterpret_cast<void**>(&h_grand), sizeof(int4), cudaHostAllocDefault));
        if (!h_dups) CKD(cudaHostAlloc(reinterpret_cast<void**>(&h_dups), sizeof(int), cudaHostAllocDefault));
    }
};

constexpr int kMaxDevices = 64;
std::mutex g_plan_mu;
Plan g_plans[kMaxDevices];

Plan& plan_for_device() {
    int dev = 0;
    CKD(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) throw Error(MSPLAT_ERR_ARGUMENT, "device index out of range");
    return g_plans[dev];
}

void check_gaussians(const MsplatGaussians* g, const char* what) {
    if (!g) throw Error(MSPLAT_ERR_ARGUMENT, std::string("null ") + what);
    if (g->num_points < 0) throw Error(MSPLAT_ERR_ARGUMENT, std::string(what) + ": negative num_points");
    if (g->sh_degree < 0 || g->sh_degree > 3) throw Error(MSPLAT_ERR_ARGUMENT, std::string(what) + ": sh_degree must be 0..3");
    if (g->num_points > 0 && (!g->means || !g->scales || !g->quats || !g->opacities || !g->features_dc ||
                              (g->sh_degree > 0 && !g->features_rest)))
        throw Error(MSPLAT_ERR_ARGUMENT, std::string(what) + ": null parameter pointer");
}

template <typename F>
int guarded_d(F&& f) {
    try {
        f();
        set_last_error("");
        return MSPLAT_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return MSPLAT_ERR_CUDA;
    }
}

int rest_floats(int degree) { return 3 * ((degree + 1) * (degree + 1) - 1); }

}  // namespace
}  // namespace msplat

using namespace msplat;

extern "C" {

int msplat_densify_plan(const MsplatGaussians* g, const MsplatDensifyArgs* args, MsplatDensifyPlan* plan,
                        void* stream) {
    return guarded_d([&] {
        check_gaussians(g, "gaussians");
        if (!args || !plan) throw Error(MSPLAT_ERR_ARGUMENT, "null args or plan");
        const int n = g->num_points;
        if (n > 0 && (!args->xys_grad_norm || !args->vis_counts || !args->max_2d_size))
            throw Error(MSPLAT_ERR_ARGUMENT, "null densify statistics");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        std::lock_guard<std::mutex> lk(g_plan_mu);
        Plan& p = plan_for_device();
        p.ensure(n > 0 ? n : 1);
        p.n = n;
        CKD(cudaMemsetAsync(p.num_dups, 0, sizeof(int), s));
        if (n > 0) {
            ClassifyArgs c;
            c.n = n;
            c.a = *args;
            c.scales = g->scales;
            c.opacities = g->opacities;
            c.flags = p.flags;
            c.counts = p.counts;
            c.num_dups = p.num_dups;
            note_launches(3);
            k_densify_classify<<<(n + 255) / 256, 256, 0, s>>>(c);
            const int nb = (n + kScanBlock - 1) / kScanBlock;
            k_scan_blocks<<<nb, kScanBlock, 0, s>>>(p.counts, n, p.prefix, p.btot);
            k_scan_totals<<<1, kScanBlock, 0, s>>>(p.btot, nb, p.grand);
            CKD(cudaMemcpyAsync(p.h_grand, p.grand, sizeof(int4), cudaMemcpyDeviceToHost, s));
        } else {
            *p.h_grand = make_int4(0, 0, 0, 0);
        }
        CKD(cudaMemcpyAsync(p.h_dups, p.num_dups, sizeof(int), cudaMemcpyDeviceToHost, s));
        CKD(cudaStreamSynchronize(s));
        CKD(cudaGetLastError());
        const int4 t = *p.h_grand;
        const int64_t total = (int64_t)t.x + t.y + t.z;
        if (t.x < 0 || t.y < 0 || t.z < 0 || t.w < 0 || total > 3LL * n)
            throw Error(MSPLAT_ERR_CAPACITY, "corrupt densification counts");
        p.num_splits = t.w;
        p.new_count = (int)total;
        plan->num_splits = t.w;
        plan->num_dups = *p.h_dups;
        plan->new_count = p.new_count;
    });
}

int msplat_densify_apply(const MsplatGaussians* g, const MsplatAdamState* adam, const MsplatDensifyArgs* args,
                         const float* random_samples, const MsplatGaussians* out, const MsplatAdamState* out_adam,
                         void* stream) {
    return guarded_d([&] {
        check_gaussians(g, "gaussians");
        check_gaussians(out, "output gaussians");
        if (!adam || !out_adam || !args) throw Error(MSPLAT_ERR_ARGUMENT, "null adam state or args");
        std::lock_guard<std::mutex> lk(g_plan_mu);
        Plan& p = plan_for_device();
        if (p.n != g->num_points || p.mem == nullptr)
            throw Error(MSPLAT_ERR_ARGUMENT, "msplat_densify_apply without a matching msplat_densify_plan");
        if (out->num_points != p.new_count || out->sh_degree != g->sh_degree)
            throw Error(MSPLAT_ERR_ARGUMENT, "output arrays must have plan.new_count rows and the input's sh_degree");
        if (p.num_splits > 0 && !random_samples) throw Error(MSPLAT_ERR_ARGUMENT, "null random samples");
        const int n = g->num_points;
        const int K3 = rest_floats(g->sh_degree);
        const int w[6] = {3, 2, 4, 3, K3, 1};
        for (int k = 0; k < 6; ++k)
            if (w[k] > 0 && n > 0 && (!adam->exp_avg[k] || !adam->exp_avg_sq[k]))
                throw Error(MSPLAT_ERR_ARGUMENT, "null adam moment");
        for (int k = 0; k < 6; ++k)
            if (w[k] > 0 && p.new_count > 0 && (!out_adam->exp_avg[k] || !out_adam->exp_avg_sq[k]))
                throw Error(MSPLAT_ERR_ARGUMENT, "null output adam moment");
        if (n == 0 || p.new_count == 0) return;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        BuildArgs b;
        b.n = n;
        b.K3 = K3;
        b.a = *args;
        const float* srcp[6] = {g->means, g->scales, g->quats, g->features_dc, g->features_rest, g->opacities};
        float* dstp[6] = {out->means, out->scales, out->quats, out->features_dc, out->features_rest, out->opacities};
        for (int k = 0; k < 6; ++k) {
            b.src[k] = srcp[k];
            b.dst[k] = dstp[k];
            b.src_m[k] = adam->exp_avg[k];
            b.src_v[k] = adam->exp_avg_sq[k];
            b.dst_m[k] = out_adam->exp_avg[k];
            b.dst_v[k] = out_adam->exp_avg_sq[k];
        }
        b.flags = p.flags;
        b.prefix = p.prefix;
        b.boff = p.btot;
        b.grand = p.grand;
        b.random_samples = random_samples;
        note_launches(1);
        k_densify_build<<<(n + 255) / 256, 256, 0, s>>>(b);
        CKD(cudaGetLastError());
    });
}

int msplat_reset_opacity(float* opacities, float* exp_avg, float* exp_avg_sq, int32_t n, float max_logit,
                         void* stream) {
    return guarded_d([&] {
        if (n < 0) throw Error(MSPLAT_ERR_ARGUMENT, "negative count");
        if (n == 0) return;
        if (!opacities) throw Error(MSPLAT_ERR_ARGUMENT, "null opacities");
        note_launches(1);
        k_reset_opacity<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(opacities, exp_avg,
                                                                                          exp_avg_sq, n, max_logit);
        CKD(cudaGetLastError());
    });
}

int msplat_normal_samples(uint32_t seed, int64_t count, float* out) {
    return guarded_d([&] {
        if (count < 0 || (count > 0 && !out)) throw Error(MSPLAT_ERR_ARGUMENT, "bad sample buffer");
        std::mt19937 rng(seed);
        std::normal_distribution<float> dist(0.0f, 1.0f);
        for (int64_t i = 0; i < count; ++i) out[i] = dist(rng);
    });
}

}  // extern "C"
