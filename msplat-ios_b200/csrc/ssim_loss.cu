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
// One CTA produces a 32x16 tile of dL/dimg for one channel at a time: it
// stages the rendered and target images with a 10-pixel halo in shared
// memory, blurs the five moment maps horizontally then vertically over a
// 5-pixel halo, evaluates SSIM and its per-pixel partials there (zero outside
// the image, as the adjoint of zero padding requires), and blurs the partials
// back to the tile. The image and target are read once (plus halo) and
// dL/dimg is written once; no [H,W,3] intermediate touches HBM. Loss partial
// sums are reduced per CTA in double and summed in a fixed order afterwards.
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

constexpr int OW = 32, OH = 16, R = 5;
constexpr int IW = OW + 4 * R, IH = OH + 4 * R;  // input region (halo 10)
constexpr int PW = OW + 2 * R, PH = OH + 2 * R;  // partial region (halo 5)
constexpr int kThreads = 256;
constexpr int kSmemFloats = 2 * IH * IW + 5 * IH * PW + 3 * PH * PW + 3 * PH * OW;

__global__ void __launch_bounds__(kThreads) k_loss_ssim(LossArgs a) {
    extern __shared__ float sm[];
    float* sI = sm;                     // [IH][IW]
    float* sG = sI + IH * IW;           // [IH][IW]
    float* hb = sG + IH * IW;           // [5][IH][PW]
    float* pmap = hb + 5 * IH * PW;     // [3][PH][PW]
    float* hp = pmap + 3 * PH * PW;     // [3][PH][OW]
    const int W = a.width, H = a.height;
    const int x0 = blockIdx.x * OW;
    const int y0 = a.row_begin + blockIdx.y * OH;
    const float C1 = 0.0001f, C2 = 0.0009f;
    const float g = -a.lambda_dssim * a.inv_num;
    double l1_sum = 0.0, ssim_sum = 0.0, dist_sum = 0.0;

    for (int c = 0; c < 3; ++c) {
        for (int q = threadIdx.x; q < IH * IW; q += kThreads) {
            const int r = q / IW, cc = q - r * IW;
            const int y = y0 - 2 * R + r, x = x0 - 2 * R + cc;
            float vi = 0.f, vg = 0.f;
            if (y >= 0 && y < H && x >= 0 && x < W) {
                const size_t e = ((size_t)y * W + x) * 3 + c;
                vi = a.out_img[e];
                vg = a.gt[e];
            }
            sI[q] = vi;
            sG[q] = vg;
        }
        __syncthreads();
        // Horizontal blur of img, gt, img^2, gt^2, img*gt; each work item is a
        // run of HR outputs of one row, so the 11 taps are loaded once per run.
        constexpr int HR = 6, HRUNS = PW / HR;  // 42 = 7 x 6
        static_assert(PW % HR == 0, "run length");
        for (int item = threadIdx.x; item < IH * HRUNS; item += kThreads) {
            const int r = item / HRUNS, c0 = (item - r * HRUNS) * HR;
            float xi[HR + 10], yi[HR + 10];
            const float* pi = sI + r * IW + c0;
            const float* pg = sG + r * IW + c0;
#pragma unroll
            for (int k = 0; k < HR + 10; ++k) {
                xi[k] = pi[k];
                yi[k] = pg[k];
            }
#pragma unroll
            for (int o = 0; o < HR; ++o) {
                float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f, m4 = 0.f;
#pragma unroll
                for (int k = 0; k < 11; ++k) {
                    const float w = kW[k], x = xi[o + k], y = yi[o + k];
                    m0 += w * x;
                    m1 += w * y;
                    m2 += w * (x * x);
                    m3 += w * (y * y);
                    m4 += w * (x * y);
                }
                const int q = r * PW + c0 + o;
                hb[0 * IH * PW + q] = m0;
                hb[1 * IH * PW + q] = m1;
                hb[2 * IH * PW + q] = m2;
                hb[3 * IH * PW + q] = m3;
                hb[4 * IH * PW + q] = m4;
            }
        }
        __syncthreads();
        // Vertical blur -> SSIM and its partials on the halo-5 region, runs of
        // VR outputs down one column.
        constexpr int VR = 4, VRUNS = (PH + VR - 1) / VR;  // 26 -> 7 runs (last one short)
        for (int item = threadIdx.x; item < PW * VRUNS; item += kThreads) {
            const int cc = item % PW, r0 = (item / PW) * VR;
            float acc[5][VR];
#pragma unroll
            for (int mm = 0; mm < 5; ++mm) {
                float col[VR + 10];
#pragma unroll
                for (int k = 0; k < VR + 10; ++k) {
                    const int rr = min(r0 + k, IH - 1);
                    col[k] = hb[mm * IH * PW + rr * PW + cc];
                }
#pragma unroll
                for (int o = 0; o < VR; ++o) {
                    float sacc = 0.f;
#pragma unroll
                    for (int k = 0; k < 11; ++k) sacc += kW[k] * col[o + k];
                    acc[mm][o] = sacc;
                }
            }
#pragma unroll
            for (int o = 0; o < VR; ++o) {
                const int r = r0 + o;
                if (r >= PH) break;
                const int y = y0 - R + r, x = x0 - R + cc;
                const float mu1 = acc[0][o], mu2 = acc[1][o], b11 = acc[2][o], b22 = acc[3][o], b12 = acc[4][o];
                float gm1 = 0.f, gs1 = 0.f, g12 = 0.f;
                if (y >= 0 && y < H && x >= 0 && x < W) {
                    // Separately rounded operations: sigma1^2, sigma2^2 and sigma12
                    // must round identically where img == gt (flat background),
                    // where the reference's SSIM is exactly 1.
                    const float m1s = fmul(mu1, mu1), m2s = fmul(mu2, mu2), m1m2 = fmul(mu1, mu2);
                    const float v1 = fsub(b11, m1s), v2 = fsub(b22, m2s), v12 = fsub(b12, m1m2);
                    const float A = fadd(fmul(2.0f, m1m2), C1), B = fadd(fmul(2.0f, v12), C2);
                    const float Cd = fadd(fadd(m1s, m2s), C1), Dd = fadd(fadd(v1, v2), C2);
                    const float CD = fmul(Cd, Dd), AB = fmul(A, B);
                    const bool own = r >= R && r < R + OH && cc >= R && cc < R + OW && y < a.row_end;
                    if (own) ssim_sum += (double)(AB / CD);
                    const float inv_CD = 1.0f / CD, inv_Cd = 1.0f / Cd, inv_Dd = 1.0f / Dd;
                    const float d_mu1 = 2.0f * inv_CD * (mu2 * B - mu1 * AB * inv_Cd);
                    const float d_s12 = 2.0f * A * inv_CD;
                    const float d_s1 = -AB * inv_CD * inv_Dd;
                    gs1 = g * d_s1;
                    g12 = g * d_s12;
                    gm1 = g * d_mu1 + gs1 * (-2.0f * mu1) + g12 * (-mu2);
                }
                const int q = r * PW + cc;
                pmap[0 * PH * PW + q] = gm1;
                pmap[1 * PH * PW + q] = gs1;
                pmap[2 * PH * PW + q] = g12;
            }
        }
        __syncthreads();
        // Horizontal blur of the partials, runs of PR outputs.
        constexpr int PR = 4, PRUNS = OW / PR;
        for (int item = threadIdx.x; item < PH * PRUNS; item += kThreads) {
            const int r = item / PRUNS, c0 = (item - r * PRUNS) * PR;
#pragma unroll
            for (int mm = 0; mm < 3; ++mm) {
                float row[PR + 10];
                const float* src = pmap + mm * PH * PW + r * PW + c0;
#pragma unroll
                for (int k = 0; k < PR + 10; ++k) row[k] = src[k];
#pragma unroll
                for (int o = 0; o < PR; ++o) {
                    float sacc = 0.f;
#pragma unroll
                    for (int k = 0; k < 11; ++k) sacc += kW[k] * row[o + k];
                    hp[mm * PH * OW + r * OW + c0 + o] = sacc;
                }
            }
        }
        __syncthreads();
        for (int q = threadIdx.x; q < OH * OW; q += kThreads) {
            const int r = q / OW, cc = q - r * OW;
            const int y = y0 + r, x = x0 + cc;
            if (y >= a.row_end || y >= H || x >= W) continue;
            float bm1 = 0.f, bs1 = 0.f, b12 = 0.f;
#pragma unroll
            for (int k = 0; k < 11; ++k) {
                const float w = kW[k];
                const int o = (r + k) * OW + cc;
                bm1 += w * hp[0 * PH * OW + o];
                bs1 += w * hp[1 * PH * OW + o];
                b12 += w * hp[2 * PH * OW + o];
            }
            const float va = sI[(r + 2 * R) * IW + cc + 2 * R];
            const float vb = sG[(r + 2 * R) * IW + cc + 2 * R];
            const float diff = va - vb;
            l1_sum += (double)(a.lambda_l1 * fabsf(diff) * a.inv_num);
            const float sg = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            const float l1g = a.lambda_l1 * sg * a.inv_num;
            const size_t pix = (size_t)y * W + x;
            a.dL_dout_img[pix * 3 + c] = l1g + (bm1 + 2.0f * va * bs1 + vb * b12);
            if (c == 0 && a.lambda_dist != 0.f) dist_sum += (double)(a.lambda_dist * a.out_distortion[pix] * (a.inv_num * 3.0f));
        }
        __syncthreads();
    }
    // Block reduction of the three partial sums in a fixed order.
    __shared__ double red[3][kThreads];
    red[0][threadIdx.x] = l1_sum;
    red[1][threadIdx.x] = ssim_sum;
    red[2][threadIdx.x] = dist_sum;
    __syncthreads();
    for (int off = kThreads / 2; off > 0; off >>= 1) {
        if ((int)threadIdx.x < off)
            for (int k = 0; k < 3; ++k) red[k][threadIdx.x] += red[k][threadIdx.x + off];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
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
        if (!(loss == loss) || loss > 1e300 || loss < -1e300) atomicOr(err, kErrNonFinite);
    }
}

}  // namespace

int loss_num_blocks(int width, int row_begin, int row_end) {
    return ((width + OW - 1) / OW) * ((row_end - row_begin + OH - 1) / OH);
}

void launch_loss_ssim(const LossArgs& a, cudaStream_t s) {
    const int rows = a.row_end - a.row_begin;
    if (rows <= 0) return;
    dim3 grid((a.width + OW - 1) / OW, (rows + OH - 1) / OH);
    const size_t smem = sizeof(float) * kSmemFloats;
    cudaFuncSetAttribute(k_loss_ssim, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    note_launches(1);
    k_loss_ssim<<<grid, kThreads, smem, s>>>(a);
}

void launch_loss_finalize(const double* partials, int num_blocks, float lambda_dssim, float inv_num, double* out,
                          float* loss_f, uint32_t* err, cudaStream_t s) {
    note_launches(1);
    k_loss_finalize<<<1, 1024, 0, s>>>(partials, num_blocks, lambda_dssim, inv_num, out, loss_f, err);
}

// ---- allocation-free variant (msplat_loss_ssim_noalloc) --------------------
//
// The same two kernels, with their scratch (per-block partial sums, the four
// loss terms and the error word) in fixed arrays that belong to the library's
// device image instead of workspace buffers, so the entry point never
// allocates. Every GPU that loads the library holds these arrays (about
// 1.5 MiB) until the process exits. Host code cannot use the array names as
// device addresses; the addresses are looked up once per device with
// cudaGetSymbolAddress.
constexpr int kNoAllocMaxBlocks = 65536;  // 32x16-pixel loss blocks: e.g. 8192 x 4096
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxBlocks * 3];
static __device__ __align__(256) double g_noalloc_terms[4];
static __device__ __align__(256) uint32_t g_noalloc_err[4];

namespace {
constexpr int kMaxDevices = 64;
struct NoAllocScratch {
    bool ready = false;
    double* partials = nullptr;
    double* terms = nullptr;
    uint32_t* err = nullptr;
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
        if ((e = cudaGetSymbolAddress(&p, g_noalloc_err)) != cudaSuccess) {
            *msg = std::string("cudaGetSymbolAddress(err): ") + cudaGetErrorString(e);
            return MSPLAT_ERR_CUDA;
        }
        s.err = static_cast<uint32_t*>(p);
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
    const int64_t nb = (int64_t)((width + OW - 1) / OW) * ((height + OH - 1) / OH);
    if (nb > kNoAllocMaxBlocks) {
        *msg = "image too large for the allocation-free loss: " + std::to_string(nb) +
               " blocks of 32x16 pixels, the fixed scratch holds " + std::to_string(kNoAllocMaxBlocks) +
               " (e.g. 8192 x 4096)";
        return MSPLAT_ERR_ARGUMENT;
    }
    NoAllocScratch sc;
    int rc = noalloc_scratch(&sc, msg);
    if (rc != MSPLAT_OK) return rc;
    cudaError_t e = cudaMemsetAsync(sc.err, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) {
        *msg = std::string("cudaMemsetAsync: ") + cudaGetErrorString(e);
        return MSPLAT_ERR_CUDA;
    }
    LossArgs la{};
    la.width = width; la.height = height; la.row_begin = 0; la.row_end = height;
    la.out_img = out_img; la.gt = gt; la.out_distortion = out_distortion;
    la.lambda_l1 = lambda_l1; la.lambda_dist = lambda_dist; la.lambda_dssim = lambda_dssim;
    la.inv_num = 1.0f / (float)(height * width * 3);
    la.dL_dout_img = dL_dout_img;
    la.partials = sc.partials;
    launch_loss_ssim(la, s);
    launch_loss_finalize(sc.partials, (int)nb, lambda_dssim, la.inv_num, sc.terms, loss_out, sc.err, s);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("loss kernels: ") + cudaGetErrorString(e);
        return MSPLAT_ERR_CUDA;
    }
    return MSPLAT_OK;
}

}  // namespace msplat
