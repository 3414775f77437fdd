// image_ops.cu — small image kernels of the trainer-level API: area
// downscaling of target images (resizeArea, core/src/loaders/image_io.cpp:
// 116-160, used by Camera::getImage for the resolution schedule) and float
// RGB -> RGBA8 conversion (Trainer::renderFromPoseToBuffer,
// core/src/msplat_api.mm:207-236, done on the device here instead of reading
// unified memory on the host).
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

__global__ void k_resize_area(const float* __restrict__ src, int sw, int sh, float* __restrict__ dst, int dw, int dh) {
    const int dx = blockIdx.x * blockDim.x + threadIdx.x, dy = blockIdx.y * blockDim.y + threadIdx.y;
    if (dx >= dw || dy >= dh) return;
    const float sx = (float)sw / dw, sy = (float)sh / dh;
    const float y0 = dy * sy, y1 = (dy + 1) * sy, x0 = dx * sx, x1 = (dx + 1) * sx;
    const int iy0 = (int)y0, iy1 = min((int)ceilf(y1), sh), ix0 = (int)x0, ix1 = min((int)ceilf(x1), sw);
    float acc[3] = {0.f, 0.f, 0.f}, total = 0.f;
    for (int iy = iy0; iy < iy1; ++iy) {
        const float wy = fminf((float)(iy + 1), y1) - fmaxf((float)iy, y0);
        for (int ix = ix0; ix < ix1; ++ix) {
            const float wx = fminf((float)(ix + 1), x1) - fmaxf((float)ix, x0);
            const float ar = wx * wy;
            const float* p = src + ((size_t)iy * sw + ix) * 3;
            acc[0] += p[0] * ar;
            acc[1] += p[1] * ar;
            acc[2] += p[2] * ar;
            total += ar;
        }
    }
    float* o = dst + ((size_t)dy * dw + dx) * 3;
    const float inv = total > 0.f ? 1.0f / total : 0.f;
    o[0] = acc[0] * inv;
    o[1] = acc[1] * inv;
    o[2] = acc[2] * inv;
}

__global__ void k_rgba8(const float* __restrict__ src, uint8_t* __restrict__ dst, int64_t n) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    uchar4 o;
    o.x = (uint8_t)(fminf(fmaxf(src[3 * i + 0], 0.f), 1.f) * 255.f);
    o.y = (uint8_t)(fminf(fmaxf(src[3 * i + 1], 0.f), 1.f) * 255.f);
    o.z = (uint8_t)(fminf(fmaxf(src[3 * i + 2], 0.f), 1.f) * 255.f);
    o.w = 255;
    reinterpret_cast<uchar4*>(dst)[i] = o;
}

}  // namespace

void launch_resize_area(const float* src, int sw, int sh, float* dst, int dw, int dh, cudaStream_t s) {
    if (dw <= 0 || dh <= 0) return;
    note_launches(1);
    k_resize_area<<<dim3((dw + 15) / 16, (dh + 15) / 16), dim3(16, 16), 0, s>>>(src, sw, sh, dst, dw, dh);
}

void launch_rgba8(const float* src, uint8_t* dst, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    note_launches(1);
    k_rgba8<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, dst, n);
}

}  // namespace msplat
