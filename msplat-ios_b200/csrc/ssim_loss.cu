// ssim_loss.cu — fused L1 + DSSIM loss, forward and backward, in one pass.
//
// Replaces the reference's 21-dispatch chain (core/metal/msplat_metal.mm:
// 1077-1212): ssim_prep_products_kernel, 5 x (ssim_blur_horiz_kernel +
// ssim_blur_vert_kernel), ssim_compute_kernel, loss_l1_distortion_2dgs_kernel,
// ssim_backward_compute_kernel, 3 x re-blur and ssim_backward_accumulate_kernel
// (core/metal/msplat_metal.metal:2704-3085). Same mathematics: 11-tap
// sigma-1.5 separable window with zero padding, C1 = 1e-4, C2 = 9e-4,
// dL/dssim = -lambda_dssim / (3HW) uniform, dL/dimg = lambda_l1 * sign(r-g) /
// (3HW) + blur(g_mu1) + 2 img blur(g_sigma1^2) + gt blur(g_sigma12).
//
// One CTA walks down a strip of SW = 54 output columns over a segment of
// rows, for all three channels at once, one image row per step:
//   S1  load image and target row r (columns x0-10 .. x0+SW+10) into shared
//       memory (double-buffered);
//   S2  blur row r-1 horizontally: the five moments img, gt, img^2, gt^2,
//       img*gt for the 64 columns x0-5 .. x0+SW+5;
//   S3  blur vertically over the last 11 moment rows, evaluate SSIM and its
//       three per-pixel partials at row r-6 (zero outside the image, as the
//       adjoint of zero padding requires);
//   S4  blur the partials of row r-7 horizontally onto the SW output columns;
//   S5  blur them vertically over the last 11 rows and write dL/dimg of row
//       r-12, together with the L1 term.
// Each thread owns one (channel, column) item of S2/S3 and one of S4/S5; the
// 11-row windows of its moments and partials live in registers (the step loop
// is unrolled 11 times so that every ring index is a constant), so the only
// shared-memory traffic is the horizontal taps. Paired quantities ((image,
// target) moments, (g_mu1, g_sigma1^2) partials) use sm_100's packed FP32
// multiply-adds. The only recomputed halo is
// 10 columns per strip and 22 rows per segment. The image and target are read
// once and dL/dimg is written once; no [H,W,3] intermediate touches HBM. Loss
// partial sums are reduced per CTA in double and summed in a fixed order
// afterwards.
#include <algorithm>
#include <mutex>
#include <string>

#include "msplat_backend.h"
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

__constant__ float kW[11] = {0.001028380084f, 0.007598758135f, 0.036000772128f, 0.109360689510f,
                             0.213005537711f, 0.266011724862f, 0.213005537711f, 0.109360689510f,
                             0.036000772128f, 0.007598758135f, 0.001028380084f};

constexpr int R = 5;
constexpr int CW = 64;             // columns of moments and partials per strip
constexpr int SW = CW - 2 * R;     // output columns per strip
constexpr int IWID = SW + 4 * R;   // input columns per strip
constexpr int kThreads = 3 * CW;   // one thread per (channel, column) of S2/S3
constexpr int kRing = 2 * R + 1;   // rows in a vertical window
constexpr int kSlots = 2 * 148;  // resident CTAs: 2 per SM (__launch_bounds__ below) x 148 SMs
constexpr int kMaxSegs = 64;

struct LossGrid {
    int strips, segs, seg_rows;
};

// Strips x row segments. Every CTA of a segment length L costs about L + 22
// row steps; the segment count minimises waves x (L + 22), so the grid fills
// whole waves of resident CTAs with the least recomputed halo. max_blocks > 0
// caps strips x segments (one segment per strip at least).
LossGrid loss_grid(int width, int rows, int max_blocks = 0) {
    LossGrid g;
    g.strips = (width + SW - 1) / SW;
    const int max_segs = max_blocks > 0 ? std::max(1, max_blocks / std::max(g.strips, 1)) : kMaxSegs;
    int best_segs = 1;
    int64_t best_cost = -1;
    for (int segs = 1; segs <= kMaxSegs && segs <= max_segs && segs <= rows; ++segs) {
        const int64_t waves = ((int64_t)g.strips * segs + kSlots - 1) / kSlots;
        const int64_t cost = waves * ((rows + segs - 1) / segs + 4 * R + 2);
        if (best_cost < 0 || cost < best_cost) {
            best_cost = cost;
            best_segs = segs;
        }
    }
    g.seg_rows = (rows + best_segs - 1) / best_segs;
    g.segs = (rows + g.seg_rows - 1) / g.seg_rows;
    return g;
}

// (image, target) pairs and the partial pairs are processed with the packed
// FP32 instructions of sm_100 (__ffma2_rn / __fmul2_rn: each component is
// rounded exactly as the scalar fmaf / fmul), which halve the instructions of
// the paired blurs.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

__global__ void __launch_bounds__(kThreads, 2) k_loss_ssim(LossArgs a, int seg_rows) {
    __shared__ float2 sIn[2][3][IWID];    // [buffer][channel][column]: (image, target)
    __shared__ float2 sPa[2][3][CW];      // [buffer][channel][column]: (g_mu1, g_sigma1^2)
    __shared__ float sPb[2][3][CW];       // [buffer][channel][column]: g_sigma12
    __shared__ double red[3][kThreads];
    const int W = a.width, H = a.height;
    const int t = threadIdx.x;
    const int ch = t / CW, col = t - ch * CW;      // S2/S3 item
    // S4/S5 item: same channel, output column col (threads col >= SW idle),
    // so that no warp spans two channels
    const bool out_item = col < SW;
    const int och = ch, ocol = col;
    const int x0 = blockIdx.x * SW;
    const int Y0 = a.row_begin + blockIdx.y * seg_rows;
    const int Y1 = min(Y0 + seg_rows, a.row_end);
    const int ybase = Y0 - 2 * R;  // input row of step 0
    const int nsteps = (Y1 - Y0) + 4 * R + 2;
    const int xm = x0 - R + col;   // image column of the S2/S3 item
    const int xo = x0 + ocol;      // image column of the S4/S5 item
    const bool own_col = col >= R && col < R + SW && xm < W;
    const float C1 = 0.0001f, C2 = 0.0009f;
    const float g = -a.lambda_dssim * a.inv_num;
    double l1_sum = 0.0, ssim_sum = 0.0, dist_sum = 0.0;

    // register rings of the vertical windows: moments (img, gt), (img^2,
    // gt^2), img*gt; partials (g_mu1, g_sigma1^2), g_sigma12
    float2 hm01[kRing], hm23[kRing], hp01[kRing];
    float hm4[kRing], hp2[kRing];
#pragma unroll
    for (int k = 0; k < kRing; ++k) {
        hm01[k] = f2(0.f, 0.f); hm23[k] = f2(0.f, 0.f); hm4[k] = 0.f;
        hp01[k] = f2(0.f, 0.f); hp2[k] = 0.f;
    }
    // S1 of one row: each thread moves up to two (image, target) pairs of the
    // contiguous span [x0-10, x0+SW+10) x 3 channels
    constexpr int kSpan = 3 * IWID;
    static_assert(kSpan <= 2 * kThreads, "two loads per thread");
    auto fetch = [&](int y, float2 (&v)[2]) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int q = t + u * kThreads;
            const int xx = x0 - 2 * R + q / 3;
            v[u] = f2(0.f, 0.f);
            if (q < kSpan && y >= 0 && y < H && xx >= 0 && xx < W) {
                const size_t e = ((size_t)y * W + xx) * 3 + (q - (q / 3) * 3);
                v[u] = f2(__ldg(a.out_img + e), __ldg(a.gt + e));
            }
        }
    };
    auto stash = [&](int buf, const float2 (&v)[2]) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int q = t + u * kThreads;
            if (q < kSpan) sIn[buf][q % 3][q / 3] = v[u];
        }
    };
    {
        float2 v[2];
        fetch(ybase, v);
        stash(0, v);
    }
    __syncthreads();

    for (int t0 = 0; t0 < nsteps; t0 += kRing) {
#pragma unroll
        for (int k = 0; k < kRing; ++k) {
            const int step = t0 + k;  // sIn[step & 1] holds input row ybase + step
            // S1 (issued first, stored last): input row ybase + step + 1
            float2 nv[2];
            fetch(ybase + step + 1, nv);
            // S2: moments of input row ybase + step
            {
                const float2* pin = &sIn[step & 1][ch][col];
                float2 m01 = f2(0.f, 0.f), m23 = f2(0.f, 0.f);
                float m4 = 0.f;
#pragma unroll
                for (int j = 0; j < kRing; ++j) {
                    const float w = kW[j];
                    const float2 w2 = f2(w, w), xy = pin[j];
                    m01 = __ffma2_rn(w2, xy, m01);
                    m23 = __ffma2_rn(w2, __fmul2_rn(xy, xy), m23);
                    m4 = fmaf(w, xy.x * xy.y, m4);
                }
                hm01[k] = m01; hm23[k] = m23; hm4[k] = m4;
            }
            // S3: SSIM partials of row ybase + step - 5 from moment rows
            // ybase + step - 10 .. ybase + step (ring slots k+1 .. k+11)
            {
                const int cy = ybase + step - R;
                float2 a01 = f2(0.f, 0.f), a23 = f2(0.f, 0.f);
                float a4 = 0.f;
#pragma unroll
                for (int j = 0; j < kRing; ++j) {
                    const float w = kW[j];
                    const float2 w2 = f2(w, w);
                    const int sl = (k + 1 + j) % kRing;
                    a01 = __ffma2_rn(w2, hm01[sl], a01);
                    a23 = __ffma2_rn(w2, hm23[sl], a23);
                    a4 = fmaf(w, hm4[sl], a4);
                }
                float gm1 = 0.f, gs1 = 0.f, g12 = 0.f;
                if (cy >= 0 && cy < H && xm >= 0 && xm < W) {
                    const float mu1 = a01.x, mu2 = a01.y, b11 = a23.x, b22 = a23.y, b12 = a4;
                    // Separately rounded operations: sigma1^2, sigma2^2 and
                    // sigma12 must round identically where img == gt (flat
                    // background), where the reference's SSIM is exactly 1.
                    const float m1s = fmul(mu1, mu1), m2s = fmul(mu2, mu2), m1m2 = fmul(mu1, mu2);
                    const float v1 = fsub(b11, m1s), v2 = fsub(b22, m2s), v12 = fsub(b12, m1m2);
                    const float A = fadd(fmul(2.0f, m1m2), C1), B = fadd(fmul(2.0f, v12), C2);
                    const float Cd = fadd(fadd(m1s, m2s), C1), Dd = fadd(fadd(v1, v2), C2);
                    const float CD = fmul(Cd, Dd), AB = fmul(A, B);
                    if (own_col && cy >= Y0 && cy < Y1) ssim_sum += (double)(AB / CD);
                    // 1/Cd and 1/Dd from 1/CD: one approximate reciprocal
                    const float inv_CD = __fdividef(1.0f, CD);
                    const float inv_Cd = Dd * inv_CD, inv_Dd = Cd * inv_CD;
                    const float d_mu1 = 2.0f * inv_CD * (mu2 * B - mu1 * AB * inv_Cd);
                    const float d_s12 = 2.0f * A * inv_CD;
                    const float d_s1 = -AB * inv_CD * inv_Dd;
                    gs1 = g * d_s1;
                    g12 = g * d_s12;
                    gm1 = g * d_mu1 + gs1 * (-2.0f * mu1) + g12 * (-mu2);
                }
                sPa[step & 1][ch][col] = f2(gm1, gs1);
                sPb[step & 1][ch][col] = g12;
            }
            if (out_item) {
                // S4: horizontal blur of the partials of row ybase + step - 6
                // (written last step) into ring slot k
                const int pb = (step + 1) & 1;
                const float2* pa = &sPa[pb][och][ocol];
                const float* pbb = &sPb[pb][och][ocol];
                float2 acc01 = f2(0.f, 0.f);
                float acc2 = 0.f;
#pragma unroll
                for (int j = 0; j < kRing; ++j) {
                    const float w = kW[j];
                    acc01 = __ffma2_rn(f2(w, w), pa[j], acc01);
                    acc2 = fmaf(w, pbb[j], acc2);
                }
                hp01[k] = acc01;
                hp2[k] = acc2;
                // S5: dL/dimg of row ybase + step - 11 from partial rows
                // ybase + step - 16 .. ybase + step - 6 (slots k+1 .. k+11)
                const int oy = ybase + step - 2 * R - 1;
                if (oy >= Y0 && oy < Y1 && xo < W) {
                    float2 b01 = f2(0.f, 0.f);
                    float b12 = 0.f;
#pragma unroll
                    for (int j = 0; j < kRing; ++j) {
                        const float w = kW[j];
                        const int sl = (k + 1 + j) % kRing;
                        b01 = __ffma2_rn(f2(w, w), hp01[sl], b01);
                        b12 = fmaf(w, hp2[sl], b12);
                    }
                    const float bm1 = b01.x, bs1 = b01.y;
                    const size_t pix = (size_t)oy * W + xo;
                    const float va = __ldg(a.out_img + pix * 3 + och), vb = __ldg(a.gt + pix * 3 + och);
                    const float diff = va - vb;
                    l1_sum += (double)(a.lambda_l1 * fabsf(diff) * a.inv_num);
                    const float sg = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
                    const float l1g = a.lambda_l1 * sg * a.inv_num;
                    a.dL_dout_img[pix * 3 + och] = l1g + (bm1 + 2.0f * va * bs1 + vb * b12);
                    if (och == 0 && a.lambda_dist != 0.f)
                        dist_sum += (double)(a.lambda_dist * a.out_distortion[pix] * (a.inv_num * 3.0f));
                }
            }
            stash((step + 1) & 1, nv);
            __syncthreads();
        }
    }
    // Block reduction of the three partial sums in a fixed order.
    red[0][t] = l1_sum;
    red[1][t] = ssim_sum;
    red[2][t] = dist_sum;
    __syncthreads();
    if (t < 64) {
        for (int k = 0; k < 3; ++k) red[k][t] += red[k][t + 64] + red[k][t + 128];
    }
    __syncthreads();
    for (int off = 32; off > 0; off >>= 1) {
        if (t < off)
            for (int k = 0; k < 3; ++k) red[k][t] += red[k][t + off];
        __syncthreads();
    }
    if (t == 0) {
        const size_t b = (size_t)blockIdx.y * gridDim.x + blockIdx.x;
        a.partials[3 * b + 0] = red[0][0];
        a.partials[3 * b + 1] = red[1][0];
        a.partials[3 * b + 2] = red[2][0];
    }
}

__global__ void __launch_bounds__(1024) k_loss_finalize(const double* partials, int nb, float lambda_dssim,
                                                        float inv_num, double* out, float* loss_f, uint32_t* err) {
    __shared__ double red[3][1024];
    double s[3] = {0.0, 0.0, 0.0};
    for (int b = threadIdx.x; b < nb; b += blockDim.x)
        for (int k = 0; k < 3; ++k) s[k] += partials[3 * b + k];
    for (int k = 0; k < 3; ++k) red[k][threadIdx.x] = s[k];
    __syncthreads();
    for (int off = blockDim.x / 2; off > 0; off >>= 1) {
        if ((int)threadIdx.x < off)
            for (int k = 0; k < 3; ++k) red[k][threadIdx.x] += red[k][threadIdx.x + off];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double l1 = red[0][0], ss = red[1][0], dd = red[2][0];
        const double loss = l1 + dd + (double)lambda_dssim * (1.0 - ss * (double)inv_num);
        out[0] = loss;
        out[1] = ss;
        out[2] = l1;
        out[3] = dd;
        if (loss_f) *loss_f = (float)loss;
        if (err && (!(loss == loss) || loss > 1e300 || loss < -1e300)) atomicOr(err, kErrNonFinite);
    }
}

}  // namespace

int loss_num_blocks(int width, int row_begin, int row_end, int max_blocks) {
    if (row_end <= row_begin || width <= 0) return 0;
    const LossGrid g = loss_grid(width, row_end - row_begin, max_blocks);
    return g.strips * g.segs;
}

void launch_loss_ssim(const LossArgs& a, cudaStream_t s, int max_blocks) {
    const int rows = a.row_end - a.row_begin;
    if (rows <= 0 || a.width <= 0) return;
    const LossGrid g = loss_grid(a.width, rows, max_blocks);
    note_launches(1);
    k_loss_ssim<<<dim3(g.strips, g.segs), kThreads, 0, s>>>(a, g.seg_rows);
}

void launch_loss_finalize(const double* partials, int num_blocks, float lambda_dssim, float inv_num, double* out,
                          float* loss_f, uint32_t* err, cudaStream_t s) {
    note_launches(1);
    k_loss_finalize<<<1, 1024, 0, s>>>(partials, num_blocks, lambda_dssim, inv_num, out, loss_f, err);
}

// ---- allocation-free variant (msplat_loss_ssim_noalloc) --------------------
//
// The same two kernels, with their scratch (per-block partial sums and the
// four loss terms) in fixed arrays that belong to the library's device image
// instead of workspace buffers, so the entry point never allocates. Every GPU
// that loads the library holds these arrays (about 192 KiB) until the process
// exits. The grid is capped at kNoAllocMaxBlocks CTAs (fewer row segments per
// strip), so any image of up to 8192 strips of 54 columns fits at any height.
// Host code cannot use the array names as device addresses; the addresses are
// looked up once per device with cudaGetSymbolAddress. The finalize kernel
// gets no error word here: a non-finite loss shows only as NaN or Inf in
// loss_out.
constexpr int kNoAllocMaxBlocks = 8192;  // loss CTAs: widths up to 8192 x 54 = 442,368 pixels
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxBlocks * 3];
static __device__ __align__(256) double g_noalloc_terms[4];

namespace {
constexpr int kMaxDevices = 64;
struct NoAllocScratch {
    bool ready = false;
    double* partials = nullptr;
    double* terms = nullptr;
};
std::mutex g_noalloc_mu;
NoAllocScratch g_noalloc[kMaxDevices];

// Looks the scratch arrays up for the current device (first call per device).
int noalloc_scratch(NoAllocScratch* out, std::string* msg) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *msg = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
        return MSPLAT_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *msg = "device index out of range for the allocation-free loss";
        return MSPLAT_ERR_ARGUMENT;
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocScratch& s = g_noalloc[dev];
    if (!s.ready) {
        void* p = nullptr;
        if ((e = cudaGetSymbolAddress(&p, g_noalloc_partials)) != cudaSuccess) {
            *msg = std::string("cudaGetSymbolAddress(partials): ") + cudaGetErrorString(e);
            return MSPLAT_ERR_CUDA;
        }
        s.partials = static_cast<double*>(p);
        if ((e = cudaGetSymbolAddress(&p, g_noalloc_terms)) != cudaSuccess) {
            *msg = std::string("cudaGetSymbolAddress(terms): ") + cudaGetErrorString(e);
            return MSPLAT_ERR_CUDA;
        }
        s.terms = static_cast<double*>(p);
        s.ready = true;
    }
    *out = s;
    return MSPLAT_OK;
}
}  // namespace

int loss_ssim_noalloc(const float* out_img, const float* gt, const float* out_distortion, int width, int height,
                      float lambda_l1, float lambda_dist, float lambda_dssim, float* dL_dout_img, float* loss_out,
                      cudaStream_t s, std::string* msg) {
    if (!out_img || !gt || !dL_dout_img) {
        *msg = "out_img, gt and dL_dout_img must be device pointers";
        return MSPLAT_ERR_ARGUMENT;
    }
    if (width <= 0 || height <= 0) {
        *msg = "width and height must be positive";
        return MSPLAT_ERR_ARGUMENT;
    }
    if (lambda_dist != 0.0f && !out_distortion) {
        *msg = "out_distortion is required when lambda_dist != 0";
        return MSPLAT_ERR_ARGUMENT;
    }
    const int64_t strips = ((int64_t)width + SW - 1) / SW;
    if (strips > kNoAllocMaxBlocks) {
        *msg = "image too wide for the allocation-free loss: " + std::to_string(strips) + " strips of " +
               std::to_string(SW) + " columns, the fixed scratch holds " + std::to_string(kNoAllocMaxBlocks) +
               " (widths up to " + std::to_string((int64_t)kNoAllocMaxBlocks * SW) + ")";
        return MSPLAT_ERR_ARGUMENT;
    }
    const int64_t nb = loss_num_blocks(width, 0, height, kNoAllocMaxBlocks);
    if (nb <= 0 || nb > kNoAllocMaxBlocks) {  // cannot happen with the cap; kept as a guard of the array
        *msg = "allocation-free loss grid of " + std::to_string(nb) + " blocks exceeds its scratch";
        return MSPLAT_ERR_ARGUMENT;
    }
    NoAllocScratch sc;
    int rc = noalloc_scratch(&sc, msg);
    if (rc != MSPLAT_OK) return rc;
    LossArgs la{};
    la.width = width; la.height = height; la.row_begin = 0; la.row_end = height;
    la.out_img = out_img; la.gt = gt; la.out_distortion = out_distortion;
    la.lambda_l1 = lambda_l1; la.lambda_dist = lambda_dist; la.lambda_dssim = lambda_dssim;
    // 3HW in double: it can exceed the int range for the largest images
    la.inv_num = 1.0f / (float)((double)height * (double)width * 3.0);
    la.dL_dout_img = dL_dout_img;
    la.partials = sc.partials;
    launch_loss_ssim(la, s, kNoAllocMaxBlocks);
    launch_loss_finalize(sc.partials, (int)nb, lambda_dssim, la.inv_num, sc.terms, loss_out, nullptr, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("loss kernels: ") + cudaGetErrorString(e);
        return MSPLAT_ERR_CUDA;
    }
    return MSPLAT_OK;
}

}  // namespace msplat
