// adam.cu — stand-alone Adam for one parameter group, and the unpacking of the
// internal raster-gradient record into the reference's gradient tensors.
//
// launch_fused_adam follows fused_adam_kernel (core/metal/msplat_metal.metal:
// 1383-1406) as dispatched by msplat_fused_adam (core/metal/msplat_metal.mm:
// 884-906): m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2;
// p -= step_size * m / (sqrt(v) / bc2_sqrt + eps). It streams float4 when the
// four pointers are 16-byte aligned. The training step itself does not use it:
// there Adam runs inside the projection backward (project.cu).
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

__device__ __forceinline__ float adam1(float& p, float g, float& m_, float& v_, float st, float b1, float b2,
                                       float bc, float eps) {
    const float m = fmaf(b1, m_, (1.0f - b1) * g);
    const float v = fmaf(b2, v_, (1.0f - b2) * g * g);
    p -= st * m / (sqrtf(v) / bc + eps);
    m_ = m;
    v_ = v;
    return p;
}

__global__ void __launch_bounds__(256) k_adam_vec4(float4* __restrict__ p, const float4* __restrict__ g,
                                                   float4* __restrict__ m, float4* __restrict__ v, int64_t n4,
                                                   float st, float b1, float b2, float bc, float eps) {
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n4; t += (int64_t)gridDim.x * blockDim.x) {
        float4 pp = p[t], gg = g[t], mm = m[t], vv = v[t];
        adam1(pp.x, gg.x, mm.x, vv.x, st, b1, b2, bc, eps);
        adam1(pp.y, gg.y, mm.y, vv.y, st, b1, b2, bc, eps);
        adam1(pp.z, gg.z, mm.z, vv.z, st, b1, b2, bc, eps);
        adam1(pp.w, gg.w, mm.w, vv.w, st, b1, b2, bc, eps);
        p[t] = pp;
        m[t] = mm;
        v[t] = vv;
    }
}

__global__ void __launch_bounds__(256) k_adam_scalar(float* __restrict__ p, const float* __restrict__ g,
                                                     float* __restrict__ m, float* __restrict__ v, int64_t b,
                                                     int64_t n, float st, float b1, float b2, float bc, float eps) {
    for (int64_t t = b + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x)
        adam1(p[t], g[t], m[t], v[t], st, b1, b2, bc, eps);
}

__global__ void __launch_bounds__(256) k_unpack(int n, const float* __restrict__ rg, float* dT, float* dN, float* dC,
                                                float* dO) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = rg + (size_t)i * kGradStride;
    if (dT)
        for (int k = 0; k < 9; ++k) dT[9 * (size_t)i + k] = r[k];
    if (dO) dO[i] = r[9];
    if (dC)
        for (int k = 0; k < 3; ++k) dC[3 * (size_t)i + k] = r[10 + k];
    if (dN)
        for (int k = 0; k < 3; ++k) dN[3 * (size_t)i + k] = r[13 + k];
}

int grid_for(int64_t work) {
    int64_t b = (work + 255) / 256;
    const int64_t cap = 148 * 16;  // persistent-ish: 16 resident CTAs per SM
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

void launch_fused_adam(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, int64_t n,
                       float step_size, float beta1, float beta2, float bc2_sqrt, float eps, cudaStream_t s) {
    if (n <= 0) return;
    const bool aligned = ((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(grads) |
                           reinterpret_cast<uintptr_t>(exp_avg) | reinterpret_cast<uintptr_t>(exp_avg_sq)) & 15) == 0;
    int64_t done = 0;
    if (aligned && n >= 4) {
        const int64_t n4 = n / 4;
        note_launches(1);
        k_adam_vec4<<<grid_for(n4), 256, 0, s>>>(reinterpret_cast<float4*>(params),
                                                  reinterpret_cast<const float4*>(grads),
                                                  reinterpret_cast<float4*>(exp_avg),
                                                  reinterpret_cast<float4*>(exp_avg_sq), n4, step_size, beta1, beta2,
                                                  bc2_sqrt, eps);
        done = n4 * 4;
    }
    if (done < n) note_launches(1);
    if (done < n)
        k_adam_scalar<<<grid_for(n - done), 256, 0, s>>>(params, grads, exp_avg, exp_avg_sq, done, n, step_size,
                                                         beta1, beta2, bc2_sqrt, eps);
}

void launch_unpack_raster_grads(int n, const float* raster_grads, float* dL_dtransMat, float* dL_dnormal3D,
                                float* dL_dcolors, float* dL_dopacity, cudaStream_t s) {
    if (n <= 0) return;
    note_launches(1);
    k_unpack<<<(n + 255) / 256, 256, 0, s>>>(n, raster_grads, dL_dtransMat, dL_dnormal3D, dL_dcolors, dL_dopacity);
}

}  // namespace msplat
