// project.cu — per-Gaussian projection (forward) and its VJP fused with Adam.
//
// Forward follows project_and_sh_forward_2dgs_kernel
// (core/metal/msplat_metal.metal:1413-1521) and its helpers
// compute_transmat_2dgs (:226-295), compute_aabb_2dgs (:302-330),
// get_tile_bbox (:77-92), quat_to_rotmat (:116-136), sh_coeffs_to_color
// (:756-823). Backward follows project_and_sh_backward_2dgs_kernel
// (:2003-2209) with quat_to_rotmat_vjp (:1252-1295), sh_coeffs_to_color_vjp
// (:825-912), sh_color_dL_ddir (:925-1013), dnormvdv (:1017-1025), and then
// applies fused_adam_kernel (:1383-1406) to all six parameter groups in the
// same launch, so the per-Gaussian gradients never round-trip through HBM.
//
// This translation unit is compiled with -fmad=false: every multiply and add
// below is rounded separately, in source order, which is what makes the
// forward outputs (and therefore tile binning) bit-reproducible.
#include "common.cuh"
#include "kernels.cuh"

namespace msplat {
namespace {

__constant__ float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                               -1.0925484305920792f, 0.5462742152960396f};
__constant__ float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                               0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                               -0.5900435899266435f};
constexpr float SH_C0 = 0.28209479177387814f;
constexpr float SH_C1 = 0.4886025119029199f;

struct V3 { float x, y, z; };
__device__ __forceinline__ V3 v3(float x, float y, float z) { return V3{x, y, z}; }
__device__ __forceinline__ float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
__device__ __forceinline__ V3 mul3(V3 a, V3 b) { return v3(a.x * b.x, a.y * b.y, a.z * b.z); }
__device__ __forceinline__ V3 scale3(V3 a, float s) { return v3(a.x * s, a.y * s, a.z * s); }
// std::max / std::min semantics (first argument wins ties and NaN compares).
__device__ __forceinline__ float smax(float a, float b) { return (a < b) ? b : a; }

__device__ __forceinline__ void quat_to_rotmat(const float q[4], V3 R[3]) {
    float s = 1.0f / sqrtf(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
    float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0] = v3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y));
    R[1] = v3(2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x));
    R[2] = v3(2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));
}

// SH basis values b[0..nb) of bands 1..degree for a unit direction (the
// factors sh_coeffs_to_color_vjp multiplies into dL/dRGB).
__device__ __forceinline__ int sh_basis(int degree, V3 d, float b[15]) {
    if (degree < 1) return 0;
    float x = d.x, y = d.y, z = d.z;
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
    b[0] = -SH_C1 * y; b[1] = SH_C1 * z; b[2] = -SH_C1 * x;
    if (degree < 2) return 3;
    b[3] = SH_C2[0] * xy; b[4] = SH_C2[1] * yz; b[5] = SH_C2[2] * (2.f * zz - xx - yy);
    b[6] = SH_C2[3] * xz; b[7] = SH_C2[4] * (xx - yy);
    if (degree < 3) return 8;
    b[8] = SH_C3[0] * y * (3.f * xx - yy); b[9] = SH_C3[1] * xy * z;
    b[10] = SH_C3[2] * y * (4.f * zz - xx - yy);
    b[11] = SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy);
    b[12] = SH_C3[4] * x * (4.f * zz - xx - yy); b[13] = SH_C3[5] * z * (xx - yy);
    b[14] = SH_C3[6] * x * (xx - 3.f * yy);
    return 15;
}

// sh_coeffs_to_color with the reference's exact per-band association.
template <typename RestAt>
__device__ __forceinline__ void sh_to_color(int degree, V3 d, const float* dc, RestAt rest, float out[3]) {
    for (int c = 0; c < 3; ++c) out[c] = SH_C0 * dc[c];
    if (degree < 1) return;
    float x = d.x, y = d.y, z = d.z;
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        out[c] += SH_C1 * (-y * rest(0 * 3 + c) + z * rest(1 * 3 + c) - x * rest(2 * 3 + c));
        if (degree < 2) continue;
        out[c] += (SH_C2[0] * xy * rest(3 * 3 + c) + SH_C2[1] * yz * rest(4 * 3 + c) +
                   SH_C2[2] * (2.f * zz - xx - yy) * rest(5 * 3 + c) + SH_C2[3] * xz * rest(6 * 3 + c) +
                   SH_C2[4] * (xx - yy) * rest(7 * 3 + c));
        if (degree < 3) continue;
        out[c] += (SH_C3[0] * y * (3.f * xx - yy) * rest(8 * 3 + c) + SH_C3[1] * xy * z * rest(9 * 3 + c) +
                   SH_C3[2] * y * (4.f * zz - xx - yy) * rest(10 * 3 + c) +
                   SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy) * rest(11 * 3 + c) +
                   SH_C3[4] * x * (4.f * zz - xx - yy) * rest(12 * 3 + c) +
                   SH_C3[5] * z * (xx - yy) * rest(13 * 3 + c) + SH_C3[6] * x * (xx - 3.f * yy) * rest(14 * 3 + c));
    }
}

template <typename RestAt>
__device__ __forceinline__ V3 sh_color_dL_ddir(int degree, V3 d, RestAt rest, const float v[3]) {
    if (degree < 1) return v3(0.f, 0.f, 0.f);
    float x = d.x, y = d.y, z = d.z;
    float dx[3], dy[3], dz[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        dx[c] = -SH_C1 * rest(2 * 3 + c);
        dy[c] = -SH_C1 * rest(0 * 3 + c);
        dz[c] = SH_C1 * rest(1 * 3 + c);
    }
    if (degree >= 2) {
        float xx = x * x, yy = y * y, zz = z * z;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float s4 = rest(3 * 3 + c), s5 = rest(4 * 3 + c), s6 = rest(5 * 3 + c);
            float s7 = rest(6 * 3 + c), s8 = rest(7 * 3 + c);
            dx[c] += SH_C2[0] * y * s4 + SH_C2[2] * (-2.f * x) * s6 + SH_C2[3] * z * s7 + SH_C2[4] * (2.f * x) * s8;
            dy[c] += SH_C2[0] * x * s4 + SH_C2[1] * z * s5 + SH_C2[2] * (-2.f * y) * s6 + SH_C2[4] * (-2.f * y) * s8;
            dz[c] += SH_C2[1] * y * s5 + SH_C2[2] * (4.f * z) * s6 + SH_C2[3] * x * s7;
        }
        if (degree >= 3) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                float s9 = rest(8 * 3 + c), s10 = rest(9 * 3 + c), s11 = rest(10 * 3 + c);
                float s12 = rest(11 * 3 + c), s13 = rest(12 * 3 + c), s14 = rest(13 * 3 + c);
                float s15 = rest(14 * 3 + c);
                dx[c] += SH_C3[0] * s9 * (6.f * x * y) + SH_C3[1] * s10 * (y * z) + SH_C3[2] * s11 * (-2.f * x * y) +
                         SH_C3[3] * s12 * (-6.f * x * z) + SH_C3[4] * s13 * (-3.f * xx + 4.f * zz - yy) +
                         SH_C3[5] * s14 * (2.f * x * z) + SH_C3[6] * s15 * (3.f * (xx - yy));
                dy[c] += SH_C3[0] * s9 * (3.f * (xx - yy)) + SH_C3[1] * s10 * (x * z) +
                         SH_C3[2] * s11 * (-3.f * yy + 4.f * zz - xx) + SH_C3[3] * s12 * (-6.f * y * z) +
                         SH_C3[4] * s13 * (-2.f * x * y) + SH_C3[5] * s14 * (-2.f * y * z) +
                         SH_C3[6] * s15 * (-6.f * x * y);
                dz[c] += SH_C3[1] * s10 * (x * y) + SH_C3[2] * s11 * (8.f * y * z) +
                         SH_C3[3] * s12 * (3.f * (2.f * zz - xx - yy)) + SH_C3[4] * s13 * (8.f * x * z) +
                         SH_C3[5] * s14 * (xx - yy);
            }
        }
    }
    V3 r = v3(0.f, 0.f, 0.f);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        r.x += dx[c] * v[c];
        r.y += dy[c] * v[c];
        r.z += dz[c] * v[c];
    }
    return r;
}

__device__ __forceinline__ float adam_update(float p, float g, float* m_, float* v_, float step_size, float b1,
                                             float b2, float bc2_sqrt, float eps) {
    float m = fmaf(b1, *m_, (1.0f - b1) * g);
    float v = fmaf(b2, *v_, (1.0f - b2) * g * g);
    *m_ = m;
    *v_ = v;
    return p - step_size * m / (sqrtf(v) / bc2_sqrt + eps);
}

__global__ void __launch_bounds__(256) k_project_forward(ProjFwdArgs a) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    const CameraDev& cam = a.cam;
    const float* vm = cam.viewmat;
    const float* pm = cam.projmat;
    float4* rec = a.records + (size_t)i * kRecordF4;
    a.radii[i] = 0;
    a.rects[i] = make_uint2(0u, 0u);
    a.depths[i] = 0.f;
    if (a.num_tiles_hit) {
        a.num_tiles_hit[i] = 0;
        a.xys[2 * i] = 0.f; a.xys[2 * i + 1] = 0.f;
        for (int k = 0; k < 9; ++k) a.transmats[9 * i + k] = 0.f;
        for (int k = 0; k < 4; ++k) a.normal_opacity[4 * i + k] = 0.f;
        for (int k = 0; k < 3; ++k) a.colors[3 * i + k] = 0.f;
        a.aabb[2 * i] = 0.f; a.aabb[2 * i + 1] = 0.f;
    }
    V3 p = v3(a.means[3 * i], a.means[3 * i + 1], a.means[3 * i + 2]);
    float pvz = vm[8] * p.x + vm[9] * p.y + vm[10] * p.z + vm[11];
    if (pvz <= a.clip_thresh) return;
    float sx = det_exp(a.scales[2 * i]) * a.glob_scale;
    float sy = det_exp(a.scales[2 * i + 1]) * a.glob_scale;
    float q[4] = {a.quats[4 * i], a.quats[4 * i + 1], a.quats[4 * i + 2], a.quats[4 * i + 3]};
    V3 R[3];
    quat_to_rotmat(q, R);
    V3 tu = scale3(R[0], sx), tv = scale3(R[1], sy);
    float tuc0 = pm[0] * tu.x + pm[1] * tu.y + pm[2] * tu.z, tuc1 = pm[4] * tu.x + pm[5] * tu.y + pm[6] * tu.z;
    float tuc3 = pm[12] * tu.x + pm[13] * tu.y + pm[14] * tu.z;
    float tvc0 = pm[0] * tv.x + pm[1] * tv.y + pm[2] * tv.z, tvc1 = pm[4] * tv.x + pm[5] * tv.y + pm[6] * tv.z;
    float tvc3 = pm[12] * tv.x + pm[13] * tv.y + pm[14] * tv.z;
    float pc0 = pm[0] * p.x + pm[1] * p.y + pm[2] * p.z + pm[3];
    float pc1 = pm[4] * p.x + pm[5] * p.y + pm[6] * p.z + pm[7];
    float pc3 = pm[12] * p.x + pm[13] * p.y + pm[14] * p.z + pm[15];
    float halfW = 0.5f * (float)cam.width, halfH = 0.5f * (float)cam.height;
    float bx = cam.cx - 0.5f, by = cam.cy - 0.5f;
    V3 cu = v3(halfW * tuc0 + bx * tuc3, halfH * tuc1 + by * tuc3, tuc3);
    V3 cv = v3(halfW * tvc0 + bx * tvc3, halfH * tvc1 + by * tvc3, tvc3);
    V3 co = v3(halfW * pc0 + bx * pc3, halfH * pc1 + by * pc3, pc3);
    V3 T0 = v3(cu.x, cv.x, co.x), T1 = v3(cu.y, cv.y, co.y), T2 = v3(cu.z, cv.z, co.z);
    const float cutoff = 3.0f;
    V3 tt = v3(cutoff * cutoff, cutoff * cutoff, -1.0f);
    float dd = dot3(tt, mul3(T2, T2));
    if (dd == 0.0f) return;
    V3 f = scale3(tt, 1.0f / dd);
    float cxp = dot3(f, mul3(T0, T2)), cyp = dot3(f, mul3(T1, T2));
    float h0x = cxp * cxp - dot3(f, mul3(T0, T0));
    float h0y = cyp * cyp - dot3(f, mul3(T1, T1));
    float hx = sqrtf(smax(1e-4f, h0x)), hy = sqrtf(smax(1e-4f, h0y));
    float radius = ceilf(smax(smax(hx, hy), cutoff * kFilterSize));
    // get_tile_bbox
    float tcx = cxp / (float)kTile, tcy = cyp / (float)kTile, tr = radius / (float)kTile;
    int x0 = min(max(0, (int)(tcx - tr)), cam.tiles_x);
    int x1 = min(max(0, (int)(tcx + tr + 1)), cam.tiles_x);
    int y0 = min(max(0, (int)(tcy - tr)), cam.tiles_y);
    int y1 = min(max(0, (int)(tcy + tr + 1)), cam.tiles_y);
    int area = (x1 - x0) * (y1 - y0);
    if (area <= 0) return;
    a.radii[i] = (int)radius;
    a.depths[i] = pvz;
    a.rects[i] = make_uint2((uint32_t)x0 | ((uint32_t)y0 << 16), (uint32_t)x1 | ((uint32_t)y1 << 16));
    const int dw = cam.tiles_x + 1;
    atomicAdd(&a.tile_diff[y0 * dw + x0], 1);
    atomicAdd(&a.tile_diff[y0 * dw + x1], -1);
    atomicAdd(&a.tile_diff[y1 * dw + x0], -1);
    atomicAdd(&a.tile_diff[y1 * dw + x1], 1);

    V3 v = v3(p.x - cam.cam_pos[0], p.y - cam.cam_pos[1], p.z - cam.cam_pos[2]);
    float inv = 1.0f / sqrtf(dot3(v, v));
    V3 dir = scale3(v, inv);
    const int K = a.rest_bases;
    const float* rest = a.f_rest + (size_t)K * 3 * i;
    float col[3];
    sh_to_color(a.degrees_to_use, dir, a.f_dc + 3 * i, [&](int k) { return __ldg(rest + k); }, col);
    float opac_raw = a.opacities[i];
    float opac = 1.f / (1.f + det_exp(-opac_raw));
    float rgb[3];
    for (int c = 0; c < 3; ++c) rgb[c] = smax(col[c] + 0.5f, 0.0f);
    V3 nrm = R[2];
    rec[0] = make_float4(T0.x, T0.y, T0.z, T1.x);
    rec[1] = make_float4(T1.y, T1.z, T2.x, T2.y);
    rec[2] = make_float4(T2.z, cxp, cyp, opac);
    rec[3] = make_float4(rgb[0], rgb[1], rgb[2], nrm.x);
    rec[4] = make_float4(nrm.y, nrm.z, 0.f, 0.f);
    if (a.num_tiles_hit) {
        a.num_tiles_hit[i] = area;
        a.xys[2 * i] = cxp; a.xys[2 * i + 1] = cyp;
        float tm[9] = {T0.x, T0.y, T0.z, T1.x, T1.y, T1.z, T2.x, T2.y, T2.z};
        for (int k = 0; k < 9; ++k) a.transmats[9 * i + k] = tm[k];
        a.normal_opacity[4 * i + 0] = nrm.x; a.normal_opacity[4 * i + 1] = nrm.y;
        a.normal_opacity[4 * i + 2] = nrm.z; a.normal_opacity[4 * i + 3] = opac_raw;
        for (int c = 0; c < 3; ++c) a.colors[3 * i + c] = col[c];
        a.aabb[2 * i] = radius; a.aabb[2 * i + 1] = radius;
    }
}

constexpr int kBwdThreads = 128;  // Gaussians per CTA

// Coalesced copy of n floats between global and shared memory (float4 when
// both ends are 16-byte aligned).
__device__ __forceinline__ void copy_in(float* dst, const float* __restrict__ src, int n) {
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        const int n4 = n >> 2;
#pragma unroll 4
        for (int q = threadIdx.x; q < n4; q += blockDim.x)
            reinterpret_cast<float4*>(dst)[q] = __ldg(reinterpret_cast<const float4*>(src) + q);
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

// One CTA owns kBwdThreads consecutive Gaussians [b0, b0 + cnt).
//  phase 0: stage their parameters and SH-rest coefficients in shared memory
//           (contiguous, float4 loads);
//  phase 1: one thread per Gaussian computes the projection and SH VJPs
//           (project_and_sh_backward_2dgs_kernel) into shared memory;
//  phase 2: Adam on every group as contiguous streams (fused_adam_kernel),
//           so moments and parameters are read and written fully coalesced.
__global__ void __launch_bounds__(kBwdThreads) k_project_backward(ProjBwdArgs a) {
    extern __shared__ float smem[];
    const int K = a.rest_bases;
    const int K3 = 3 * K;
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
    float* sR = sDC + 3 * T;        // [T * K3] SH-rest coefficients
    copy_in(sMean, a.means + 3 * (size_t)b0, 3 * cnt);
    copy_in(sScale, a.scales + 2 * (size_t)b0, 2 * cnt);
    copy_in(sQuat, a.quats + 4 * (size_t)b0, 4 * cnt);
    copy_in(sDc, a.f_dc + 3 * (size_t)b0, 3 * cnt);
    copy_in(sOp, a.opacities + (size_t)b0, cnt);
    if (K3) copy_in(sR, a.f_rest + (size_t)b0 * K3, cnt * K3);
    __syncthreads();

    const int t = threadIdx.x;
    if (t < cnt) {
        const int i = b0 + t;
        const CameraDev& cam = a.cam;
        const float* pm = cam.projmat;
        const float4* gr4 = reinterpret_cast<const float4*>(a.raster_grads + (size_t)i * kGradStride);
        const float4 q0 = __ldg(gr4), q1 = __ldg(gr4 + 1), q2 = __ldg(gr4 + 2), q3 = __ldg(gr4 + 3);
        const float dT[9] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w, q2.x};
        const float d_opac = q2.y;
        float dC[3] = {q2.z, q2.w, q3.x};
        const float dN[3] = {q3.y, q3.z, q3.w};
        float g_mean[3] = {0.f, 0.f, 0.f}, g_scale[2] = {0.f, 0.f}, g_quat[4] = {0.f, 0.f, 0.f, 0.f};
        float g_m2[2] = {0.f, 0.f};
        float basis[15];
        int nb = 0;
        const int rad = a.radii[i];
        const float* myR = sR + t * K3;
        auto rest_at = [&](int k) { return myR[k]; };
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
    if (K3)
        adam_stream(cnt * K3, sR,
                    [&](int q) {
                        const int gl = q / K3;
                        const int r = q - gl * K3;
                        const int k = r / 3;
                        return sB[gl * 15 + k] * sDC[gl * 3 + (r - k * 3)];
                    },
                    a.f_rest + i0 * K3, ad ? M[4] + i0 * K3 : nullptr, ad ? Vv[4] + i0 * K3 : nullptr,
                    a.dL_dfeatures_rest ? a.dL_dfeatures_rest + i0 * K3 : nullptr, a.step_size[4], b1, b2, bc, eps,
                    ad);
}

}  // namespace

void launch_project_forward(const ProjFwdArgs& a, cudaStream_t s) {
    if (a.n <= 0) return;
    note_launches(1);
    k_project_forward<<<(a.n + 255) / 256, 256, 0, s>>>(a);
}

void launch_project_backward(const ProjBwdArgs& a, cudaStream_t s) {
    int cnt = a.g_end - a.g_begin;
    if (cnt <= 0) return;
    const size_t smem = sizeof(float) * (size_t)kBwdThreads * (26 + 15 + 3 + 3 * a.rest_bases);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(k_project_backward, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    note_launches(1);
    k_project_backward<<<(cnt + kBwdThreads - 1) / kBwdThreads, kBwdThreads, smem, s>>>(a);
}

}  // namespace msplat
