// project_bwd.cu — the projection VJP fused with Adam.
//
// Follows project_and_sh_backward_2dgs_kernel (core/metal/msplat_metal.metal:
// 2003-2209) with quat_to_rotmat_vjp (:1252-1295), sh_coeffs_to_color_vjp
// (:825-912), sh_color_dL_ddir (:925-1013) and dnormvdv (:1017-1025), then
// applies fused_adam_kernel (:1383-1406) to all six parameter groups in the
// same launch, so the per-Gaussian gradients never round-trip through HBM.
// Gradients are checked against tolerances, so this file is compiled with
// fused multiply-adds and approximate sqrt/division.
#include "kernels.cuh"
#include "sh_math.cuh"

namespace msplat {
namespace {

constexpr int kBwdThreads = 128;  // Gaussians per CTA

// Coalesced copy of n floats between global and shared memory (float4 when
// both ends are 16-byte aligned).
// Copies n floats into shared memory: 16-byte cp.async copies when both
// pointers are 16-byte aligned (the caller waits with cp_async_wait_all
// before its barrier, so the copies of several groups are in flight
// together), plain loads for the rest.
__device__ __forceinline__ void copy_in(float* dst, const float* __restrict__ src, int n) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const int n4 = n >> 2;
        for (int q = threadIdx.x; q < n4; q += blockDim.x)
            cp_async16(reinterpret_cast<float4*>(dst) + q, reinterpret_cast<const float4*>(src) + q);
        for (int q = (n4 << 2) + threadIdx.x; q < n; q += blockDim.x) dst[q] = __ldg(src + q);
    } else {
        for (int q = threadIdx.x; q < n; q += blockDim.x) dst[q] = __ldg(src + q);
    }
}

// Adam over n contiguous elements of one group; old parameters and gradients
// come from shared memory, moments and new parameters stream through HBM.
// When every global pointer is 16-byte aligned, each thread handles four
// float4 chunks per iteration and issues all their moment loads before any
// arithmetic, so enough bytes are in flight to saturate HBM.
template <typename GradAt>
__device__ __forceinline__ void adam_stream(int n, const float* sparam, GradAt grad, float* __restrict__ p,
                                            float* __restrict__ m, float* __restrict__ v, float* __restrict__ gout,
                                            float st, float b1, float b2, float bc, float eps, bool do_adam) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(m) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(gout);
    int done = 0;
    if (do_adam && (al & 15) == 0) {
        constexpr int U = 4;
        const int n4 = n >> 2;
        const int step = blockDim.x * U;
        for (int base = threadIdx.x; base < n4; base += step) {
            float4 mm[U], vv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * blockDim.x;
                if (c < n4) {
                    mm[u] = reinterpret_cast<const float4*>(m)[c];
                    vv[u] = reinterpret_cast<const float4*>(v)[c];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * blockDim.x;
                if (c >= n4) break;
                const int e = c << 2;
                const float g0 = grad(e), g1 = grad(e + 1), g2 = grad(e + 2), g3 = grad(e + 3);
                float4 pp;
                pp.x = adam_update(sparam[e], g0, &mm[u].x, &vv[u].x, st, b1, b2, bc, eps);
                pp.y = adam_update(sparam[e + 1], g1, &mm[u].y, &vv[u].y, st, b1, b2, bc, eps);
                pp.z = adam_update(sparam[e + 2], g2, &mm[u].z, &vv[u].z, st, b1, b2, bc, eps);
                pp.w = adam_update(sparam[e + 3], g3, &mm[u].w, &vv[u].w, st, b1, b2, bc, eps);
                reinterpret_cast<float4*>(p)[c] = pp;
                reinterpret_cast<float4*>(m)[c] = mm[u];
                reinterpret_cast<float4*>(v)[c] = vv[u];
                if (gout) reinterpret_cast<float4*>(gout)[c] = make_float4(g0, g1, g2, g3);
            }
        }
        done = n4 << 2;
    }
    for (int q = done + threadIdx.x; q < n; q += blockDim.x) {
        const float g = grad(q);
        if (gout) gout[q] = g;
        if (do_adam) p[q] = adam_update(sparam[q], g, m + q, v + q, st, b1, b2, bc, eps);
    }
}

// adam_stream for a group whose old parameters are read from global memory
// (coalesced float4 with the moments) instead of shared memory.
template <typename GradAt>
__device__ __forceinline__ void adam_stream_global(int n, GradAt grad, float* __restrict__ p, float* __restrict__ m,
                                                   float* __restrict__ v, float* __restrict__ gout, float st,
                                                   float b1, float b2, float bc, float eps, bool do_adam) {
    const uintptr_t al = reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(m) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(gout);
    int done = 0;
    if (do_adam && (al & 15) == 0) {
        constexpr int U = 4;
        const int n4 = n >> 2;
        const int step = blockDim.x * U;
        for (int base = threadIdx.x; base < n4; base += step) {
            float4 pp[U], mm[U], vv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * blockDim.x;
                if (c < n4) {
                    pp[u] = reinterpret_cast<const float4*>(p)[c];
                    mm[u] = reinterpret_cast<const float4*>(m)[c];
                    vv[u] = reinterpret_cast<const float4*>(v)[c];
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * blockDim.x;
                if (c >= n4) break;
                const int e = c << 2;
                const float g0 = grad(e), g1 = grad(e + 1), g2 = grad(e + 2), g3 = grad(e + 3);
                float4 q;
                q.x = adam_update(pp[u].x, g0, &mm[u].x, &vv[u].x, st, b1, b2, bc, eps);
                q.y = adam_update(pp[u].y, g1, &mm[u].y, &vv[u].y, st, b1, b2, bc, eps);
                q.z = adam_update(pp[u].z, g2, &mm[u].z, &vv[u].z, st, b1, b2, bc, eps);
                q.w = adam_update(pp[u].w, g3, &mm[u].w, &vv[u].w, st, b1, b2, bc, eps);
                reinterpret_cast<float4*>(p)[c] = q;
                reinterpret_cast<float4*>(m)[c] = mm[u];
                reinterpret_cast<float4*>(v)[c] = vv[u];
                if (gout) reinterpret_cast<float4*>(gout)[c] = make_float4(g0, g1, g2, g3);
            }
        }
        done = n4 << 2;
    }
    for (int q = done + threadIdx.x; q < n; q += blockDim.x) {
        const float g = grad(q);
        if (gout) gout[q] = g;
        if (do_adam) p[q] = adam_update(p[q], g, m + q, v + q, st, b1, b2, bc, eps);
    }
}

// One CTA owns kBwdThreads consecutive Gaussians [b0, b0 + cnt).
//  phase 0: stage their parameters and SH-rest coefficients in shared memory
//           (contiguous, float4 loads);
//  phase 1: one thread per Gaussian computes the projection and SH VJPs
//           (project_and_sh_backward_2dgs_kernel) into shared memory;
//  phase 2: Adam on every group as contiguous streams (fused_adam_kernel),
//           so moments and parameters are read and written fully coalesced.
template <int K>
__global__ void __launch_bounds__(kBwdThreads, 6) k_project_backward(ProjBwdArgs a) {
    extern __shared__ float smem[];
    constexpr int K3 = 3 * K;
    const int b0 = a.g_begin + blockIdx.x * kBwdThreads;
    const int cnt = min(kBwdThreads, a.g_end - b0);
    if (cnt <= 0) return;
    constexpr int T = kBwdThreads;
    float* sMean = smem;            // [3T]
    float* sScale = sMean + 3 * T;  // [2T]
    float* sQuat = sScale + 2 * T;  // [4T]
    float* sDc = sQuat + 4 * T;     // [3T]
    float* sOp = sDc + 3 * T;       // [T]
    float* gMean = sOp + T;         // [3T] gradients
    float* gScale = gMean + 3 * T;  // [2T]
    float* gQuat = gScale + 2 * T;  // [4T]
    float* gDc = gQuat + 4 * T;     // [3T]
    float* gOp = gDc + 3 * T;       // [T]
    float* sB = gOp + T;            // [T][15] SH basis of the used bands
    float* sDC = sB + 15 * T;       // [T][3] dL/d colour
    copy_in(sMean, a.means + 3 * (size_t)b0, 3 * cnt);
    copy_in(sScale, a.scales + 2 * (size_t)b0, 2 * cnt);
    copy_in(sQuat, a.quats + 4 * (size_t)b0, 4 * cnt);
    copy_in(sDc, a.f_dc + 3 * (size_t)b0, 3 * cnt);
    copy_in(sOp, a.opacities + (size_t)b0, cnt);
    const int t = threadIdx.x;
    // this Gaussian's raster-gradient record, loaded while the copies run
    float4 q0 = make_float4(0.f, 0.f, 0.f, 0.f), q1 = q0, q2 = q0, q3 = q0;
    if (t < cnt) {
        const float4* gr4 = reinterpret_cast<const float4*>(a.raster_grads + (size_t)(b0 + t) * kGradStride);
        q0 = __ldg(gr4); q1 = __ldg(gr4 + 1); q2 = __ldg(gr4 + 2); q3 = __ldg(gr4 + 3);
    }
    cp_async_wait_all();
    __syncthreads();

    if (t < cnt) {
        const int i = b0 + t;
        const CameraDev& cam = a.cam;
        const float* pm = cam.projmat;
        const float dT[9] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w, q2.x};
        const float d_opac = q2.y;
        float dC[3] = {q2.z, q2.w, q3.x};
        const float dN[3] = {q3.y, q3.z, q3.w};
        float g_mean[3] = {0.f, 0.f, 0.f}, g_scale[2] = {0.f, 0.f}, g_quat[4] = {0.f, 0.f, 0.f, 0.f};
        float g_m2[2] = {0.f, 0.f};
        float basis[15];
        int nb = 0;
        const int rad = a.radii[i];
        // the SH-rest coefficients are read from global memory here and again,
        // coalesced, by the Adam stream below (an L2 hit)
        const float* myR = a.f_rest + (size_t)i * K3;
        auto rest_at = [&](int k) { return __ldg(myR + k); };
        if (rad > 0) {
            V3 p = v3(sMean[3 * t], sMean[3 * t + 1], sMean[3 * t + 2]);
            float ex = det_exp(sScale[2 * t]), ey = det_exp(sScale[2 * t + 1]);
            float q[4] = {sQuat[4 * t], sQuat[4 * t + 1], sQuat[4 * t + 2], sQuat[4 * t + 3]};
            V3 R[3];
            quat_to_rotmat(q, R);
            float sx = ex * a.glob_scale, sy = ey * a.glob_scale;
            float pcw = pm[12] * p.x + pm[13] * p.y + pm[14] * p.z + pm[15];
            float W = (float)cam.width, H = (float)cam.height;
            float halfW = 0.5f * W, halfH = 0.5f * H, bx = cam.cx - 0.5f, by = cam.cy - 0.5f;
            V3 dcu = v3(dT[0], dT[3], dT[6]), dcv = v3(dT[1], dT[4], dT[7]), dco = v3(dT[2], dT[5], dT[8]);
            float dtu[4] = {halfW * dcu.x, halfH * dcu.y, 0.0f, bx * dcu.x + by * dcu.y + dcu.z};
            float dtv[4] = {halfW * dcv.x, halfH * dcv.y, 0.0f, bx * dcv.x + by * dcv.y + dcv.z};
            float dpc[4] = {halfW * dco.x, halfH * dco.y, 0.0f, bx * dco.x + by * dco.y + dco.z};
            auto back = [&](const float* d) {
                return v3(pm[0] * d[0] + pm[4] * d[1] + pm[8] * d[2] + pm[12] * d[3],
                          pm[1] * d[0] + pm[5] * d[1] + pm[9] * d[2] + pm[13] * d[3],
                          pm[2] * d[0] + pm[6] * d[1] + pm[10] * d[2] + pm[14] * d[3]);
            };
            V3 dtuw = back(dtu), dtvw = back(dtv), dpo = back(dpc);
            float dsx = dot3(dtuw, R[0]), dsy = dot3(dtvw, R[1]);
            g_scale[0] = dsx * ex * a.glob_scale;
            g_scale[1] = dsy * ey * a.glob_scale;
            // quat_to_rotmat_vjp with v_R columns (dtuw*sx, dtvw*sy, dN).
            V3 c0 = scale3(dtuw, sx), c1 = scale3(dtvw, sy), c2 = v3(dN[0], dN[1], dN[2]);
            {
                float s_ = 1.0f / sqrtf(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
                float w = q[0] * s_, x = q[1] * s_, y = q[2] * s_, z = q[3] * s_;
                // R(c, r): column c, row r.
                float R00 = c0.x, R01 = c0.y, R02 = c0.z, R10 = c1.x, R11 = c1.y, R12 = c1.z;
                float R20 = c2.x, R21 = c2.y, R22 = c2.z;
                g_quat[0] = 2.f * (x * (R12 - R21) + y * (R20 - R02) + z * (R01 - R10));
                g_quat[1] = 2.f * (-2.f * x * (R11 + R22) + y * (R01 + R10) + z * (R02 + R20) + w * (R12 - R21));
                g_quat[2] = 2.f * (x * (R01 + R10) - 2.f * y * (R00 + R22) + z * (R12 + R21) + w * (R20 - R02));
                g_quat[3] = 2.f * (x * (R02 + R20) + y * (R12 + R21) - 2.f * z * (R00 + R11) + w * (R01 - R10));
            }
            V3 v = v3(p.x - cam.cam_pos[0], p.y - cam.cam_pos[1], p.z - cam.cam_pos[2]);
            float inv = 1.0f / sqrtf(dot3(v, v));
            V3 dir = scale3(v, inv);
            nb = sh_basis(a.degrees_to_use, dir, basis);
            if (a.degrees_to_use >= 1) {
                V3 dd = sh_color_dL_ddir(a.degrees_to_use, dir, rest_at, dC);
                // dnormvdv
                float sum2 = v.x * v.x + v.y * v.y + v.z * v.z;
                float invs = 1.0f / sqrtf(sum2 * sum2 * sum2);
                V3 dpv = v3(((sum2 - v.x * v.x) * dd.x - v.y * v.x * dd.y - v.z * v.x * dd.z) * invs,
                            (-v.x * v.y * dd.x + (sum2 - v.y * v.y) * dd.y - v.z * v.y * dd.z) * invs,
                            (-v.x * v.z * dd.x - v.y * v.z * dd.y + (sum2 - v.z * v.z) * dd.z) * invs);
                dpo = v3(dpo.x + dpv.x, dpo.y + dpv.y, dpo.z + dpv.z);
            }
            g_mean[0] = dpo.x; g_mean[1] = dpo.y; g_mean[2] = dpo.z;
            g_m2[0] = dT[6] * pcw * 0.5f * W;
            g_m2[1] = dT[7] * pcw * 0.5f * H;
            if (a.xys_grad_norm) {
                a.xys_grad_norm[i] += fabsf(g_m2[0]) + fabsf(g_m2[1]);
                a.vis_counts[i] += 1.0f;
                float r_norm = float(rad) * a.inv_max_dim;
                if (r_norm > a.max_2d_size[i]) a.max_2d_size[i] = r_norm;
            }
        } else {
            dC[0] = dC[1] = dC[2] = 0.f;
        }
        for (int k = 0; k < 15; ++k) sB[t * 15 + k] = (k < nb) ? basis[k] : 0.f;
        for (int c = 0; c < 3; ++c) {
            sDC[t * 3 + c] = dC[c];
            gMean[3 * t + c] = g_mean[c];
            gDc[3 * t + c] = SH_C0 * dC[c];
        }
        gScale[2 * t] = g_scale[0]; gScale[2 * t + 1] = g_scale[1];
        for (int c = 0; c < 4; ++c) gQuat[4 * t + c] = g_quat[c];
        gOp[t] = d_opac;
        if (a.dL_dmean2D) {
            a.dL_dmean2D[2 * i] = g_m2[0];
            a.dL_dmean2D[2 * i + 1] = g_m2[1];
        }
    }
    __syncthreads();
    const bool ad = a.do_adam != 0;
    const float b1 = a.beta1, b2 = a.beta2, bc = a.bc2_sqrt, eps = a.eps;
    float* const* M = a.exp_avg;
    float* const* Vv = a.exp_avg_sq;
    const size_t i0 = (size_t)b0;
    adam_stream(3 * cnt, sMean, [&](int q) { return gMean[q]; }, a.means + 3 * i0, ad ? M[0] + 3 * i0 : nullptr,
                ad ? Vv[0] + 3 * i0 : nullptr, a.dL_dmean3D ? a.dL_dmean3D + 3 * i0 : nullptr, a.step_size[0], b1, b2,
                bc, eps, ad);
    adam_stream(2 * cnt, sScale, [&](int q) { return gScale[q]; }, a.scales + 2 * i0, ad ? M[1] + 2 * i0 : nullptr,
                ad ? Vv[1] + 2 * i0 : nullptr, a.dL_dscale ? a.dL_dscale + 2 * i0 : nullptr, a.step_size[1], b1, b2,
                bc, eps, ad);
    adam_stream(4 * cnt, sQuat, [&](int q) { return gQuat[q]; }, a.quats + 4 * i0, ad ? M[2] + 4 * i0 : nullptr,
                ad ? Vv[2] + 4 * i0 : nullptr, a.dL_dquat ? a.dL_dquat + 4 * i0 : nullptr, a.step_size[2], b1, b2,
                bc, eps, ad);
    adam_stream(3 * cnt, sDc, [&](int q) { return gDc[q]; }, a.f_dc + 3 * i0, ad ? M[3] + 3 * i0 : nullptr,
                ad ? Vv[3] + 3 * i0 : nullptr, a.dL_dfeatures_dc ? a.dL_dfeatures_dc + 3 * i0 : nullptr,
                a.step_size[3], b1, b2, bc, eps, ad);
    adam_stream(cnt, sOp, [&](int q) { return gOp[q]; }, a.opacities + i0, ad ? M[5] + i0 : nullptr,
                ad ? Vv[5] + i0 : nullptr, a.dL_dopacity ? a.dL_dopacity + i0 : nullptr, a.step_size[5], b1, b2, bc,
                eps, ad);
    if constexpr (K3 > 0)
        adam_stream_global(cnt * K3,
                           [&](int q) {
                               const int gl = q / K3;
                               const int r = q - gl * K3;
                               const int k = r / 3;
                               return sB[gl * 15 + k] * sDC[gl * 3 + (r - k * 3)];
                           },
                           a.f_rest + i0 * K3, ad ? M[4] + i0 * K3 : nullptr, ad ? Vv[4] + i0 * K3 : nullptr,
                           a.dL_dfeatures_rest ? a.dL_dfeatures_rest + i0 * K3 : nullptr, a.step_size[4], b1, b2, bc,
                           eps, ad);
}

}  // namespace

template <int K>
void launch_k(const ProjBwdArgs& a, int grid, size_t smem, cudaStream_t s) {
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(k_project_backward<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_project_backward<K><<<grid, kBwdThreads, smem, s>>>(a);
}

void launch_project_backward(const ProjBwdArgs& a, cudaStream_t s) {
    int cnt = a.g_end - a.g_begin;
    if (cnt <= 0) return;
    const size_t smem = sizeof(float) * (size_t)kBwdThreads * (26 + 15 + 3);
    if (a.rest_bases == 0 || a.rest_bases == 3 || a.rest_bases == 8 || a.rest_bases == 15) note_launches(1);
    const int grid = (cnt + kBwdThreads - 1) / kBwdThreads;
    switch (a.rest_bases) {
        case 0: launch_k<0>(a, grid, smem, s); break;
        case 3: launch_k<3>(a, grid, smem, s); break;
        case 8: launch_k<8>(a, grid, smem, s); break;
        case 15: launch_k<15>(a, grid, smem, s); break;
        default: set_last_error("project_backward: SH-rest bases must be 0, 3, 8 or 15"); break;
    }
}

}  // namespace msplat
