// sh_math.cuh — per-Gaussian math shared by the projection forward
// (project.cu, compiled with -fmad=false for a fixed rounding sequence) and its
// VJP (project_bwd.cu, compiled with contraction and approximate sqrt/div):
// quat_to_rotmat (core/metal/msplat_metal.metal:116-136), the SH basis and
// colour (:756-823), the colour VJP with respect to the view direction
// (:925-1013) and the Adam update (:1383-1406).
#pragma once
#include "common.cuh"

namespace msplat {
namespace {

static __constant__ float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                               -1.0925484305920792f, 0.5462742152960396f};
static __constant__ float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
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

}  // namespace
}  // namespace msplat
