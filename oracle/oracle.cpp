// oracle.cpp — TEST INFRASTRUCTURE ONLY (see oracle.h for the contract).
//
// Scalar CPU restatement of the reference's 2DGS training step. Every function
// cites the reference file:line it follows. Floating-point expressions are
// written with an explicit evaluation order (left to right, explicit fmaf where
// the CUDA build uses a fused multiply-add) and the file is compiled with
// -ffp-contract=off, so the forward path (projection, binning, rasterisation)
// is bit-reproducible by an IEEE-conforming GPU implementation that evaluates
// the same sequence.
#include "oracle.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr int kTile = 16;                       // BLOCK_X/BLOCK_Y, metal:5-6
constexpr int kMaxTileElems = ORC_MAX_TILE_ELEMS;  // metal:1553
constexpr float kFilterSize = 0.707106f;        // FILTER_SIZE_2DGS, metal:210
constexpr float kFilterInvSq = 2.0f;            // FILTER_INV_SQ_2DGS, metal:212
constexpr float kNearN = 0.2f;                  // NEAR_N_2DGS, metal:216
constexpr float kFarN = 100.0f;                 // FAR_N_2DGS, metal:217

// SH constants, metal:19-44.
constexpr float SH_C0 = 0.28209479177387814f;
constexpr float SH_C1 = 0.4886025119029199f;
constexpr float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f,
                            0.31539156525252005f, -1.0925484305920792f,
                            0.5462742152960396f};
constexpr float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f,
                            -0.4570457994644658f, 0.3731763325901154f,
                            -0.4570457994644658f, 1.445305721320277f,
                            -0.5900435899266435f};

// SSIM 1-D window, metal:2804-2816.
constexpr float kSsimW[11] = {0.001028380084f, 0.007598758135f, 0.036000772128f,
                              0.109360689510f, 0.213005537711f, 0.266011724862f,
                              0.213005537711f, 0.109360689510f, 0.036000772128f,
                              0.007598758135f, 0.001028380084f};

struct F3 { float x, y, z; };
inline F3 f3(float x, float y, float z) { return F3{x, y, z}; }
inline float dot3(F3 a, F3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline F3 mul3(F3 a, F3 b) { return f3(a.x * b.x, a.y * b.y, a.z * b.z); }
inline F3 scale3(F3 a, float s) { return f3(a.x * s, a.y * s, a.z * s); }

int num_sh_bases(int degree) {  // metal:46-57
    if (degree == 0) return 1;
    if (degree == 1) return 4;
    if (degree == 2) return 9;
    if (degree == 3) return 16;
    return 25;
}

// quat_to_rotmat, metal:116-136. Returns the three COLUMNS of R (Metal's
// float3x3 is column-major: R[0] is the first column).
void quat_to_rotmat(const float* q, F3 R[3]) {
    // float4 quat = (q0, q1, q2, q3) as (.x .y .z .w); the sum starts with .w.
    float s = 1.0f / std::sqrt(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
    float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    R[0] = f3(1.f - 2.f * (y * y + z * z), 2.f * (x * y + w * z), 2.f * (x * z - w * y));
    R[1] = f3(2.f * (x * y - w * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z + w * x));
    R[2] = f3(2.f * (x * z + w * y), 2.f * (y * z - w * x), 1.f - 2.f * (x * x + y * y));
}

// sh_coeffs_to_color, metal:756-823 (degrees <= 3 are all this path uses).
void sh_to_color(int degree, F3 d, const float* dc, const float* rest, float* out) {
    for (int c = 0; c < 3; ++c) out[c] = SH_C0 * dc[c];
    if (degree < 1) return;
    float x = d.x, y = d.y, z = d.z;
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
    for (int c = 0; c < 3; ++c) {
        out[c] += SH_C1 * (-y * rest[0 * 3 + c] + z * rest[1 * 3 + c] - x * rest[2 * 3 + c]);
        if (degree < 2) continue;
        out[c] += (SH_C2[0] * xy * rest[3 * 3 + c] + SH_C2[1] * yz * rest[4 * 3 + c] +
                   SH_C2[2] * (2.f * zz - xx - yy) * rest[5 * 3 + c] +
                   SH_C2[3] * xz * rest[6 * 3 + c] + SH_C2[4] * (xx - yy) * rest[7 * 3 + c]);
        if (degree < 3) continue;
        out[c] += (SH_C3[0] * y * (3.f * xx - yy) * rest[8 * 3 + c] +
                   SH_C3[1] * xy * z * rest[9 * 3 + c] +
                   SH_C3[2] * y * (4.f * zz - xx - yy) * rest[10 * 3 + c] +
                   SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy) * rest[11 * 3 + c] +
                   SH_C3[4] * x * (4.f * zz - xx - yy) * rest[12 * 3 + c] +
                   SH_C3[5] * z * (xx - yy) * rest[13 * 3 + c] +
                   SH_C3[6] * x * (xx - 3.f * yy) * rest[14 * 3 + c]);
    }
}

// sh_coeffs_to_color_vjp, metal:825-912.
void sh_to_color_vjp(int degree, F3 d, const float* v_col, float* v_dc, float* v_rest) {
    for (int c = 0; c < 3; ++c) v_dc[c] = SH_C0 * v_col[c];
    if (degree < 1) return;
    float x = d.x, y = d.y, z = d.z;
    float xx = x * x, xy = x * y, xz = x * z, yy = y * y, yz = y * z, zz = z * z;
    for (int c = 0; c < 3; ++c) {
        float b[15];
        b[0] = -SH_C1 * y; b[1] = SH_C1 * z; b[2] = -SH_C1 * x;
        int nb = 3;
        if (degree >= 2) {
            b[3] = SH_C2[0] * xy; b[4] = SH_C2[1] * yz; b[5] = SH_C2[2] * (2.f * zz - xx - yy);
            b[6] = SH_C2[3] * xz; b[7] = SH_C2[4] * (xx - yy);
            nb = 8;
        }
        if (degree >= 3) {
            b[8] = SH_C3[0] * y * (3.f * xx - yy); b[9] = SH_C3[1] * xy * z;
            b[10] = SH_C3[2] * y * (4.f * zz - xx - yy);
            b[11] = SH_C3[3] * z * (2.f * zz - 3.f * xx - 3.f * yy);
            b[12] = SH_C3[4] * x * (4.f * zz - xx - yy); b[13] = SH_C3[5] * z * (xx - yy);
            b[14] = SH_C3[6] * x * (xx - 3.f * yy);
            nb = 15;
        }
        for (int k = 0; k < nb; ++k) v_rest[k * 3 + c] = b[k] * v_col[c];
    }
}

// sh_color_dL_ddir, metal:925-1013.
F3 sh_color_dL_ddir(int degree, F3 d, const float* rest, const float* v_col) {
    if (degree < 1) return f3(0, 0, 0);
    float x = d.x, y = d.y, z = d.z;
    float dx[3], dy[3], dz[3];
    for (int c = 0; c < 3; ++c) {
        dx[c] = -SH_C1 * rest[2 * 3 + c];
        dy[c] = -SH_C1 * rest[0 * 3 + c];
        dz[c] = SH_C1 * rest[1 * 3 + c];
    }
    if (degree >= 2) {
        float xx = x * x, yy = y * y, zz = z * z;
        for (int c = 0; c < 3; ++c) {
            float s4 = rest[3 * 3 + c], s5 = rest[4 * 3 + c], s6 = rest[5 * 3 + c];
            float s7 = rest[6 * 3 + c], s8 = rest[7 * 3 + c];
            dx[c] += SH_C2[0] * y * s4 + SH_C2[2] * (-2.f * x) * s6 + SH_C2[3] * z * s7 +
                     SH_C2[4] * (2.f * x) * s8;
            dy[c] += SH_C2[0] * x * s4 + SH_C2[1] * z * s5 + SH_C2[2] * (-2.f * y) * s6 +
                     SH_C2[4] * (-2.f * y) * s8;
            dz[c] += SH_C2[1] * y * s5 + SH_C2[2] * (4.f * z) * s6 + SH_C2[3] * x * s7;
        }
        if (degree >= 3) {
            for (int c = 0; c < 3; ++c) {
                float s9 = rest[8 * 3 + c], s10 = rest[9 * 3 + c], s11 = rest[10 * 3 + c];
                float s12 = rest[11 * 3 + c], s13 = rest[12 * 3 + c];
                float s14 = rest[13 * 3 + c], s15 = rest[14 * 3 + c];
                dx[c] += SH_C3[0] * s9 * (6.f * x * y) + SH_C3[1] * s10 * (y * z) +
                         SH_C3[2] * s11 * (-2.f * x * y) + SH_C3[3] * s12 * (-6.f * x * z) +
                         SH_C3[4] * s13 * (-3.f * xx + 4.f * zz - yy) +
                         SH_C3[5] * s14 * (2.f * x * z) + SH_C3[6] * s15 * (3.f * (xx - yy));
                dy[c] += SH_C3[0] * s9 * (3.f * (xx - yy)) + SH_C3[1] * s10 * (x * z) +
                         SH_C3[2] * s11 * (-3.f * yy + 4.f * zz - xx) +
                         SH_C3[3] * s12 * (-6.f * y * z) + SH_C3[4] * s13 * (-2.f * x * y) +
                         SH_C3[5] * s14 * (-2.f * y * z) + SH_C3[6] * s15 * (-6.f * x * y);
                dz[c] += SH_C3[1] * s10 * (x * y) + SH_C3[2] * s11 * (8.f * y * z) +
                         SH_C3[3] * s12 * (3.f * (2.f * zz - xx - yy)) +
                         SH_C3[4] * s13 * (8.f * x * z) + SH_C3[5] * s14 * (xx - yy);
            }
        }
    }
    F3 r = f3(0, 0, 0);
    for (int c = 0; c < 3; ++c) {
        r.x += dx[c] * v_col[c];
        r.y += dy[c] * v_col[c];
        r.z += dz[c] * v_col[c];
    }
    return r;
}

// dnormvdv, metal:1017-1025.
F3 dnormvdv(F3 v, F3 dv) {
    float sum2 = v.x * v.x + v.y * v.y + v.z * v.z;
    float inv = 1.0f / std::sqrt(sum2 * sum2 * sum2);
    return f3(((sum2 - v.x * v.x) * dv.x - v.y * v.x * dv.y - v.z * v.x * dv.z) * inv,
              (-v.x * v.y * dv.x + (sum2 - v.y * v.y) * dv.y - v.z * v.y * dv.z) * inv,
              (-v.x * v.z * dv.x - v.y * v.z * dv.y + (sum2 - v.z * v.z) * dv.z) * inv);
}

// quat_to_rotmat_vjp, metal:1252-1295. vR[i] is the gradient on column i.
void quat_to_rotmat_vjp(const float* q, const F3 vR[3], float* v_quat) {
    float s = 1.0f / std::sqrt(q[3] * q[3] + q[0] * q[0] + q[1] * q[1] + q[2] * q[2]);
    float w = q[0] * s, x = q[1] * s, y = q[2] * s, z = q[3] * s;
    // v_R[c][r] = column c, row r.
    auto R = [&](int c, int r) -> float {
        const F3& col = vR[c];
        return r == 0 ? col.x : (r == 1 ? col.y : col.z);
    };
    v_quat[0] = 2.f * (x * (R(1, 2) - R(2, 1)) + y * (R(2, 0) - R(0, 2)) + z * (R(0, 1) - R(1, 0)));
    v_quat[1] = 2.f * (-2.f * x * (R(1, 1) + R(2, 2)) + y * (R(0, 1) + R(1, 0)) +
                       z * (R(0, 2) + R(2, 0)) + w * (R(1, 2) - R(2, 1)));
    v_quat[2] = 2.f * (x * (R(0, 1) + R(1, 0)) - 2.f * y * (R(0, 0) + R(2, 2)) +
                       z * (R(1, 2) + R(2, 1)) + w * (R(2, 0) - R(0, 2)));
    v_quat[3] = 2.f * (x * (R(0, 2) + R(2, 0)) + y * (R(1, 2) + R(2, 1)) -
                       2.f * z * (R(0, 0) + R(1, 1)) + w * (R(0, 1) - R(1, 0)));
}

// Homogeneous-pixel columns of the 2DGS homography (compute_transmat_2dgs,
// metal:226-295): col_u, col_v, col_o; T row r = (col_u[r], col_v[r], col_o[r]).
struct Transmat { F3 col_u, col_v, col_o, normal; float p_clip_w; };

Transmat compute_transmat(F3 p, float sx, float sy, const float* q, const float* pm,
                          float W, float H, float cx, float cy) {
    F3 R[3];
    quat_to_rotmat(q, R);
    F3 tu = scale3(R[0], sx);
    F3 tv = scale3(R[1], sy);
    float tuc[4] = {pm[0] * tu.x + pm[1] * tu.y + pm[2] * tu.z, pm[4] * tu.x + pm[5] * tu.y + pm[6] * tu.z,
                    pm[8] * tu.x + pm[9] * tu.y + pm[10] * tu.z, pm[12] * tu.x + pm[13] * tu.y + pm[14] * tu.z};
    float tvc[4] = {pm[0] * tv.x + pm[1] * tv.y + pm[2] * tv.z, pm[4] * tv.x + pm[5] * tv.y + pm[6] * tv.z,
                    pm[8] * tv.x + pm[9] * tv.y + pm[10] * tv.z, pm[12] * tv.x + pm[13] * tv.y + pm[14] * tv.z};
    float pc[4] = {pm[0] * p.x + pm[1] * p.y + pm[2] * p.z + pm[3], pm[4] * p.x + pm[5] * p.y + pm[6] * p.z + pm[7],
                   pm[8] * p.x + pm[9] * p.y + pm[10] * p.z + pm[11],
                   pm[12] * p.x + pm[13] * p.y + pm[14] * p.z + pm[15]};
    float halfW = 0.5f * W, halfH = 0.5f * H, bx = cx - 0.5f, by = cy - 0.5f;
    Transmat t;
    t.col_u = f3(halfW * tuc[0] + bx * tuc[3], halfH * tuc[1] + by * tuc[3], tuc[3]);
    t.col_v = f3(halfW * tvc[0] + bx * tvc[3], halfH * tvc[1] + by * tvc[3], tvc[3]);
    t.col_o = f3(halfW * pc[0] + bx * pc[3], halfH * pc[1] + by * pc[3], pc[3]);
    t.normal = R[2];
    t.p_clip_w = pc[3];
    return t;
}

// get_bbox / get_tile_bbox, metal:62-92.
void tile_bbox(float cx, float cy, float r, int tx, int ty, int* x0, int* y0, int* x1, int* y1) {
    float tcx = cx / (float)kTile, tcy = cy / (float)kTile;
    float trx = r / (float)kTile, try_ = r / (float)kTile;
    *x0 = std::min(std::max(0, (int)(tcx - trx)), tx);
    *x1 = std::min(std::max(0, (int)(tcx + trx + 1)), tx);
    *y0 = std::min(std::max(0, (int)(tcy - try_)), ty);
    *y1 = std::min(std::max(0, (int)(tcy + try_ + 1)), ty);
}

inline float sigmoid(float x) { return 1.f / (1.f + orc_exp(-x)); }

}  // namespace

extern "C" {

int orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

// Deterministic exponential. The reference calls Metal's exp(); this build
// fixes one evaluation so that CPU and GPU agree bit for bit: Cody-Waite
// reduction x = k*ln2 + r (ln2 split into a 16-bit head and a tail), a degree-7
// Taylor polynomial for exp(r) on |r| <= ln2/2 (truncation error < 6e-9
// relative) evaluated by Horner with fmaf, and an exact scaling by 2^k.
// Results are flushed to 0 below x = -86 and to +inf above x = 88.
float orc_exp(float x) {
    if (x != x) return x;
    if (x > 88.0f) return INFINITY;
    if (x < -86.0f) return 0.0f;
    float kf = std::nearbyint(x * 1.44269502f);
    float r = std::fma(-kf, 0.693145751953125f, x);
    r = std::fma(-kf, 1.42860677e-06f, r);
    float p = 1.98412698e-04f;
    p = std::fma(p, r, 1.38888889e-03f);
    p = std::fma(p, r, 8.33333377e-03f);
    p = std::fma(p, r, 4.16666679e-02f);
    p = std::fma(p, r, 1.66666672e-01f);
    p = std::fma(p, r, 0.5f);
    p = std::fma(p, r, 1.0f);
    p = std::fma(p, r, 1.0f);
    int k = (int)kf;
    uint32_t bits = (uint32_t)(k + 127) << 23;
    float scale;
    std::memcpy(&scale, &bits, 4);
    return p * scale;
}

void orc_prepare_cam(const float camToWorld[16], float fx, float fy, float cx, float cy,
                     int width, int height, OrcCamera* out) {
    // Model::prepareCam, model.cpp:500-544 (downscale factor 1).
    float fovX = 2.0f * std::atan(width / (2.0f * fx));
    float fovY = 2.0f * std::atan(height / (2.0f * fy));
    const float* d = camToWorld;
    float R[3][3], Rinv[3][3], T[3], Tinv[3];
    for (int i = 0; i < 3; i++) {
        R[i][0] = d[i * 4 + 0]; R[i][1] = -d[i * 4 + 1]; R[i][2] = -d[i * 4 + 2]; T[i] = d[i * 4 + 3];
    }
    for (int i = 0; i < 3; i++)
        for (int j = 0; j < 3; j++) Rinv[i][j] = R[j][i];
    for (int i = 0; i < 3; i++) Tinv[i] = -(Rinv[i][0] * T[0] + Rinv[i][1] * T[1] + Rinv[i][2] * T[2]);
    float vm[16] = {Rinv[0][0], Rinv[0][1], Rinv[0][2], Tinv[0], Rinv[1][0], Rinv[1][1], Rinv[1][2], Tinv[1],
                    Rinv[2][0], Rinv[2][1], Rinv[2][2], Tinv[2], 0, 0, 0, 1};
    float t_p = 0.001f * std::tan(0.5f * fovY), r_p = 0.001f * std::tan(0.5f * fovX);
    float pm[16] = {0.001f / r_p, 0, 0, 0, 0, 0.001f / t_p, 0, 0, 0, 0,
                    (1000.0f + 0.001f) / (1000.0f - 0.001f), -1000.0f * 0.001f / (1000.0f - 0.001f),
                    0, 0, 1, 0};
    float pvm[16] = {};
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++)
            for (int k = 0; k < 4; k++) pvm[i * 4 + j] += pm[i * 4 + k] * vm[k * 4 + j];
    std::memcpy(out->viewmat, vm, sizeof(vm));
    std::memcpy(out->projmat, pvm, sizeof(pvm));
    out->fx = fx; out->fy = fy; out->cx = cx; out->cy = cy;
    out->width = width; out->height = height;
    out->cam_pos[0] = T[0]; out->cam_pos[1] = T[1]; out->cam_pos[2] = T[2];
}

void orc_project_forward(int n, const float* means, const float* scales, float glob_scale,
                         const float* quats, const float* opacities, const float* f_dc,
                         const float* f_rest, int degree, int degrees_to_use,
                         const OrcCamera* cam, float clip_thresh, float* xys, float* depths,
                         int32_t* radii, float* transmats, int32_t* num_tiles_hit,
                         float* normal_opacity, float* colors, float* aabb) {
    const int tx = (cam->width + kTile - 1) / kTile, ty = (cam->height + kTile - 1) / kTile;
    const int K = num_sh_bases(degree) - 1;
    const float* vm = cam->viewmat;
    const float* pm = cam->projmat;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        radii[i] = 0; num_tiles_hit[i] = 0;
        xys[2 * i] = xys[2 * i + 1] = 0.f; depths[i] = 0.f;
        for (int k = 0; k < 9; ++k) transmats[9 * i + k] = 0.f;
        for (int k = 0; k < 4; ++k) normal_opacity[4 * i + k] = 0.f;
        for (int k = 0; k < 3; ++k) colors[3 * i + k] = 0.f;
        aabb[2 * i] = aabb[2 * i + 1] = 0.f;

        F3 p = f3(means[3 * i], means[3 * i + 1], means[3 * i + 2]);
        // clip_near_plane / transform_4x3, metal:100-107, 139-150.
        float pvz = vm[8] * p.x + vm[9] * p.y + vm[10] * p.z + vm[11];
        if (pvz <= clip_thresh) continue;
        float sx = orc_exp(scales[2 * i]) * glob_scale;
        float sy = orc_exp(scales[2 * i + 1]) * glob_scale;
        Transmat t = compute_transmat(p, sx, sy, quats + 4 * i, pm, (float)cam->width,
                                      (float)cam->height, cam->cx, cam->cy);
        F3 T0 = f3(t.col_u.x, t.col_v.x, t.col_o.x);
        F3 T1 = f3(t.col_u.y, t.col_v.y, t.col_o.y);
        F3 T2 = f3(t.col_u.z, t.col_v.z, t.col_o.z);
        // compute_aabb_2dgs, metal:302-330 (cutoff 3).
        const float cutoff = 3.0f;
        F3 tt = f3(cutoff * cutoff, cutoff * cutoff, -1.0f);
        float dd = dot3(tt, mul3(T2, T2));
        if (dd == 0.0f) continue;
        F3 f = scale3(tt, 1.0f / dd);
        // (1/d) * t in Metal multiplies the scalar into each lane: (1/d)*t.x ...
        float px_ = dot3(f, mul3(T0, T2)), py_ = dot3(f, mul3(T1, T2));
        float h0x = px_ * px_ - dot3(f, mul3(T0, T0));
        float h0y = py_ * py_ - dot3(f, mul3(T1, T1));
        float hx = std::sqrt(std::max(1e-4f, h0x)), hy = std::sqrt(std::max(1e-4f, h0y));
        float radius = std::ceil(std::max(std::max(hx, hy), cutoff * kFilterSize));
        int x0, y0, x1, y1;
        tile_bbox(px_, py_, radius, tx, ty, &x0, &y0, &x1, &y1);
        int area = (x1 - x0) * (y1 - y0);
        if (area <= 0) continue;
        num_tiles_hit[i] = area;
        depths[i] = pvz;
        radii[i] = (int)radius;
        xys[2 * i] = px_; xys[2 * i + 1] = py_;
        aabb[2 * i] = radius; aabb[2 * i + 1] = radius;
        float tm[9] = {T0.x, T0.y, T0.z, T1.x, T1.y, T1.z, T2.x, T2.y, T2.z};
        std::memcpy(transmats + 9 * i, tm, sizeof(tm));
        normal_opacity[4 * i + 0] = t.normal.x;
        normal_opacity[4 * i + 1] = t.normal.y;
        normal_opacity[4 * i + 2] = t.normal.z;
        normal_opacity[4 * i + 3] = opacities[i];
        // normalize(p_world - cam_pos) = v * rsqrt(dot(v, v)).
        F3 v = f3(p.x - cam->cam_pos[0], p.y - cam->cam_pos[1], p.z - cam->cam_pos[2]);
        float inv = 1.0f / std::sqrt(dot3(v, v));
        F3 dir = scale3(v, inv);
        sh_to_color(degrees_to_use, dir, f_dc + 3 * i, f_rest + (int64_t)K * 3 * i, colors + 3 * i);
    }
}

int64_t orc_bin_and_sort(int n, const float* xys, const float* depths, const int32_t* radii,
                         const float* aabb, int tiles_x, int tiles_y, int64_t* raw_counts,
                         int32_t* tile_bins, int32_t* gaussian_ids, int64_t capacity) {
    const int T = tiles_x * tiles_y;
    // Per-tile candidate lists (the scatter of metal:1557-1591). Filled in
    // parallel; each list is then put into id order, so the result does not
    // depend on the fill order.
    std::vector<int64_t> cnt(T, 0);
    std::vector<int> rect(4 * (size_t)n, 0);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        if (radii[i] <= 0) continue;
        int* r = &rect[4 * (size_t)i];
        tile_bbox(xys[2 * i], xys[2 * i + 1], aabb[2 * i], tiles_x, tiles_y, &r[0], &r[1], &r[2], &r[3]);
        for (int y = r[1]; y < r[3]; ++y)
            for (int x = r[0]; x < r[2]; ++x) {
#pragma omp atomic
                cnt[y * tiles_x + x] += 1;
            }
    }
    std::vector<int64_t> off(T + 1, 0);
    for (int t = 0; t < T; ++t) off[t + 1] = off[t] + cnt[t];
    std::vector<uint64_t> keys((size_t)off[T] + 1);
    std::vector<int64_t> fill(T, 0);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        if (radii[i] <= 0) continue;
        const int* r = &rect[4 * (size_t)i];
        uint32_t db;
        std::memcpy(&db, &depths[i], 4);
        const uint64_t key = ((uint64_t)db << 32) | (uint64_t)(uint32_t)i;
        for (int y = r[1]; y < r[3]; ++y)
            for (int x = r[0]; x < r[2]; ++x) {
                const int t = y * tiles_x + x;
                int64_t slot;
#pragma omp atomic capture
                slot = fill[t]++;
                keys[off[t] + slot] = key;
            }
    }
    // prefix_sum_kernel over min(count, 2048) (metal:3093-3145); tile_bins
    // (start, end) as written by the sort kernel (metal:1628-1635).
    int64_t running = 0;
    for (int t = 0; t < T; ++t) {
        raw_counts[t] = cnt[t];
        int64_t kept = std::min<int64_t>(cnt[t], kMaxTileElems);
        tile_bins[2 * t] = (int32_t)running;
        running += kept;
        tile_bins[2 * t + 1] = (int32_t)running;
    }
    if (running > capacity) return -1;
#pragma omp parallel for schedule(dynamic, 16)
    for (int t = 0; t < T; ++t) {
        uint64_t* L = keys.data() + off[t];
        int64_t c = cnt[t];
        if (c > kMaxTileElems) {
            // Overflow policy: keep the 2048 lowest Gaussian ids.
            std::nth_element(L, L + kMaxTileElems, L + c, [](uint64_t a, uint64_t b) {
                return (uint32_t)a < (uint32_t)b;
            });
            c = kMaxTileElems;
        }
        std::sort(L, L + c);  // ascending (depth_bits, id), metal:1649-1664
        int32_t start = tile_bins[2 * t];
        for (int64_t k = 0; k < c; ++k) gaussian_ids[start + k] = (int32_t)(L[k] & 0xFFFFFFFFu);
    }
    return running;
}

// Raw counts only (the scatter's per-tile counters before the clamp,
// metal:1557-1591), from per-thread 2-D difference arrays of the tile
// rectangles; no key buffer, so it scales to billions of intersections.
void orc_tile_counts(int n, const float* xys, const int32_t* radii, const float* aabb, int tiles_x,
                     int tiles_y, int64_t* raw_counts) {
    const int DX = tiles_x + 1, DY = tiles_y + 1;
    std::vector<int64_t> total((size_t)DX * DY, 0);
#pragma omp parallel
    {
        std::vector<int64_t> d((size_t)DX * DY, 0);
#pragma omp for schedule(static)
        for (int i = 0; i < n; ++i) {
            if (radii[i] <= 0) continue;
            int x0, y0, x1, y1;
            tile_bbox(xys[2 * i], xys[2 * i + 1], aabb[2 * i], tiles_x, tiles_y, &x0, &y0, &x1, &y1);
            if (x1 <= x0 || y1 <= y0) continue;
            d[(size_t)y0 * DX + x0] += 1;
            d[(size_t)y0 * DX + x1] -= 1;
            d[(size_t)y1 * DX + x0] -= 1;
            d[(size_t)y1 * DX + x1] += 1;
        }
#pragma omp critical
        for (size_t k = 0; k < d.size(); ++k) total[k] += d[k];
    }
    // 2-D inclusive prefix sum of the difference array
    std::vector<int64_t> acc((size_t)DX * DY, 0);
    for (int y = 0; y < tiles_y; ++y)
        for (int x = 0; x < tiles_x; ++x) {
            int64_t v = total[(size_t)y * DX + x];
            if (x > 0) v += acc[(size_t)y * DX + x - 1];
            if (y > 0) v += acc[(size_t)(y - 1) * DX + x];
            if (x > 0 && y > 0) v -= acc[(size_t)(y - 1) * DX + x - 1];
            acc[(size_t)y * DX + x] = v;
            raw_counts[(size_t)y * tiles_x + x] = v;
        }
}

// Kept ids of the listed tiles under the overflow policy of orc_bin_and_sort
// (the 2048 lowest Gaussian ids of an overfull tile), sorted by the key
// (depth_bits << 32) | id. Each tile scans the Gaussians in id order, so the
// first 2048 it meets are its lowest ids. ids_out holds 2048 ids per listed
// tile; counts_out the kept count of each.
void orc_tile_kept_ids(int n, const float* xys, const float* depths, const int32_t* radii, const float* aabb,
                       int tiles_x, int tiles_y, int num_tiles, const int32_t* tiles, int32_t* ids_out,
                       int32_t* counts_out) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int k = 0; k < num_tiles; ++k) {
        const int t = tiles[k];
        const int tx = t % tiles_x, ty = t / tiles_x;
        std::vector<uint64_t> keys;
        keys.reserve(kMaxTileElems);
        for (int i = 0; i < n && (int64_t)keys.size() < kMaxTileElems; ++i) {
            if (radii[i] <= 0) continue;
            int x0, y0, x1, y1;
            tile_bbox(xys[2 * i], xys[2 * i + 1], aabb[2 * i], tiles_x, tiles_y, &x0, &y0, &x1, &y1);
            if (tx < x0 || tx >= x1 || ty < y0 || ty >= y1) continue;
            uint32_t db;
            std::memcpy(&db, &depths[i], 4);
            keys.push_back(((uint64_t)db << 32) | (uint64_t)(uint32_t)i);
        }
        std::sort(keys.begin(), keys.end());
        counts_out[k] = (int32_t)keys.size();
        for (size_t q = 0; q < keys.size(); ++q) ids_out[(size_t)k * kMaxTileElems + q] = (int32_t)(keys[q] & 0xFFFFFFFFu);
    }
}

void orc_pack(int64_t kept, const int32_t* ids, const float* xys, const float* transmats,
              const float* normal_opacity, const float* colors, float* packed_xy,
              float* packed_transmat, float* packed_normal_opac, float* packed_rgb) {
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < kept; ++k) {
        int g = ids[k];
        packed_xy[2 * k] = xys[2 * g];
        packed_xy[2 * k + 1] = xys[2 * g + 1];
        for (int j = 0; j < 9; ++j) packed_transmat[9 * k + j] = transmats[9 * g + j];
        packed_normal_opac[4 * k + 0] = normal_opacity[4 * g + 0];
        packed_normal_opac[4 * k + 1] = normal_opacity[4 * g + 1];
        packed_normal_opac[4 * k + 2] = normal_opacity[4 * g + 2];
        packed_normal_opac[4 * k + 3] = sigmoid(normal_opacity[4 * g + 3]);
        for (int j = 0; j < 3; ++j) packed_rgb[3 * k + j] = colors[3 * g + j];
    }
}

namespace {
// Per-(pixel, surfel) evaluation shared by the forward and the backward replay
// (metal:630-667 and 1819-1852). Returns false when the surfel is skipped.
struct PairEval { float u, v, pz, rho3d, rho2d, depth, G, alpha, dx, dy; F3 k, l, p; };

inline bool eval_pair(float px, float py, const float* xy, const float* tm, float opac, PairEval* e) {
    F3 Tu = f3(tm[0], tm[1], tm[2]), Tv = f3(tm[3], tm[4], tm[5]), Tw = f3(tm[6], tm[7], tm[8]);
    F3 k = f3(std::fma(px, Tw.x, -Tu.x), std::fma(px, Tw.y, -Tu.y), std::fma(px, Tw.z, -Tu.z));
    F3 l = f3(std::fma(py, Tw.x, -Tv.x), std::fma(py, Tw.y, -Tv.y), std::fma(py, Tw.z, -Tv.z));
    F3 p = f3(std::fma(k.y, l.z, -(k.z * l.y)), std::fma(k.z, l.x, -(k.x * l.z)),
              std::fma(k.x, l.y, -(k.y * l.x)));
    if (p.z == 0.0f) return false;
    float inv_z = 1.0f / p.z;
    float u = p.x * inv_z, v = p.y * inv_z;
    float rho3d = std::fma(u, u, v * v);
    float dx = xy[0] - px, dy = xy[1] - py;
    float rho2d = kFilterInvSq * std::fma(dx, dx, dy * dy);
    float rho = std::min(rho3d, rho2d);
    float depth = std::fma(u, Tw.x, std::fma(v, Tw.y, Tw.z));
    if (depth < kNearN) return false;
    float power = -0.5f * rho;
    if (power > 0.0f) return false;
    float G = orc_exp(power);
    float alpha = std::min(0.99f, opac * G);
    if (alpha < 1.0f / 255.0f) return false;
    *e = PairEval{u, v, p.z, rho3d, rho2d, depth, G, alpha, dx, dy, k, l, p};
    return true;
}
}  // namespace

namespace {
// Tile-row sampling used only by orc_time_step_sample: rows of tiles whose
// index is not a multiple of g_row_stride are skipped.
thread_local int g_row_stride = 1;
// Pixel rows at or below this limit are skipped by the forward (render of a
// band, for the reference arm's sampled target). Read on the calling thread.
thread_local int g_row_limit = 1 << 30;
}  // namespace

void orc_rasterize_forward(int width, int height, int tiles_x, const int32_t* tile_bins,
                           const float* packed_xy, const float* packed_normal_opac,
                           const float* packed_transmat, const float* packed_rgb,
                           const float* background, float* final_Ts, int32_t* final_idx,
                           float* out_img, float* out_depth, float* out_normal, float* out_alpha,
                           float* out_median_depth, float* out_distortion) {
    const float mscale = kFarN / (kFarN - kNearN);
    const int row_stride = g_row_stride;
    const int row_limit = g_row_limit;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t pix = 0; pix < (int64_t)width * height; ++pix) {
        int i = (int)(pix / width), j = (int)(pix % width);
        if ((i / kTile) % row_stride != 0 || i >= row_limit) continue;
        int tile = (i / kTile) * tiles_x + (j / kTile);
        float px = (float)j, py = (float)i;
        int start = tile_bins[2 * tile], end = tile_bins[2 * tile + 1];
        float T = 1.f, col[3] = {0, 0, 0}, nrm[3] = {0, 0, 0}, pdepth = 0.f;
        float M1 = 0.f, M2 = 0.f, dist = 0.f, median_depth = 0.f;
        int median_c = -1, contributor = 0, last_c = 0;
        for (int s = start; s < end; ++s) {
            contributor++;
            PairEval e;
            const float* no = packed_normal_opac + 4 * s;
            if (!eval_pair(px, py, packed_xy + 2 * s, packed_transmat + 9 * s, no[3], &e)) continue;
            float next_T = T * (1.0f - e.alpha);
            if (next_T <= 1e-4f) break;
            float w = e.alpha * T;
            float A = 1.f - T;
            float m = mscale * (1.f - kNearN / e.depth);
            dist = std::fma((m * m) * A + M2 - (2.f * m) * M1, w, dist);
            M1 = std::fma(m, w, M1);
            M2 = std::fma(m * m, w, M2);
            if (T > 0.5f) { median_depth = e.depth; median_c = contributor; }
            const float* rgb = packed_rgb + 3 * s;
            for (int c = 0; c < 3; ++c) col[c] = std::fma(std::max(rgb[c] + 0.5f, 0.0f), w, col[c]);
            pdepth = std::fma(e.depth, w, pdepth);
            for (int c = 0; c < 3; ++c) nrm[c] = std::fma(no[c], w, nrm[c]);
            T = next_T;
            last_c = contributor;
        }
        final_Ts[3 * pix + 0] = T; final_Ts[3 * pix + 1] = M1; final_Ts[3 * pix + 2] = M2;
        final_idx[2 * pix + 0] = last_c; final_idx[2 * pix + 1] = median_c;
        for (int c = 0; c < 3; ++c) out_img[3 * pix + c] = std::fma(background[c], T, col[c]);
        out_depth[pix] = pdepth;
        for (int c = 0; c < 3; ++c) out_normal[3 * pix + c] = nrm[c];
        out_alpha[pix] = 1.f - T;
        out_median_depth[pix] = median_depth;
        out_distortion[pix] = dist;
    }
}

namespace {
// ssim_blur_horiz_kernel / ssim_blur_vert_kernel (metal:2847-2903): 11-tap
// window, zero padding, taps summed from k = -5 to +5.
void blur(int W, int H, const float* in, float* out, bool horiz) {
#pragma omp parallel for schedule(static)
    for (int y = 0; y < H; ++y)
        for (int x = 0; x < W; ++x) {
            float acc[3] = {0, 0, 0};
            for (int k = -5; k <= 5; ++k) {
                int xs = horiz ? x + k : x, ys = horiz ? y : y + k;
                if (xs < 0 || xs >= W || ys < 0 || ys >= H) continue;
                float w = kSsimW[k + 5];
                const float* s = in + ((int64_t)ys * W + xs) * 3;
                acc[0] += w * s[0]; acc[1] += w * s[1]; acc[2] += w * s[2];
            }
            float* o = out + ((int64_t)y * W + x) * 3;
            o[0] = acc[0]; o[1] = acc[1]; o[2] = acc[2];
        }
}
void blur2d(int W, int H, const float* in, float* out, float* tmp) {
    blur(W, H, in, tmp, true);
    blur(W, H, tmp, out, false);
}
}  // namespace

void orc_loss_ssim(int width, int height, const float* out_img, const float* gt,
                   const float* out_distortion, float lambda_l1, float lambda_dist,
                   float lambda_dssim, float* dL_dout_img, float* dL_dout_distortion,
                   double* loss, double* ssim_sum) {
    const int64_t P = (int64_t)width * height, E = P * 3;
    std::vector<float> s1(E), s2(E), s12(E), mu1(E), mu2(E), b1(E), b2(E), b12(E), tmp(E);
    // ssim_prep_products_kernel, metal:2823-2843.
    for (int64_t e = 0; e < E; ++e) {
        s1[e] = out_img[e] * out_img[e];
        s2[e] = gt[e] * gt[e];
        s12[e] = out_img[e] * gt[e];
    }
    blur2d(width, height, out_img, mu1.data(), tmp.data());
    blur2d(width, height, gt, mu2.data(), tmp.data());
    blur2d(width, height, s1.data(), b1.data(), tmp.data());
    blur2d(width, height, s2.data(), b2.data(), tmp.data());
    blur2d(width, height, s12.data(), b12.data(), tmp.data());
    const float C1 = 0.0001f, C2 = 0.0009f;
    // ssim_compute_kernel, metal:2910-2952.
    double ssum = 0.0;
    for (int64_t e = 0; e < E; ++e) {
        float m1 = mu1[e], m2 = mu2[e];
        float m1s = m1 * m1, m2s = m2 * m2, m1m2 = m1 * m2;
        float v1 = b1[e] - m1s, v2 = b2[e] - m2s, v12 = b12[e] - m1m2;
        float A = 2.0f * m1m2 + C1, B = 2.0f * v12 + C2;
        float Cd = m1s + m2s + C1, Dd = v1 + v2 + C2;
        ssum += (double)((A * B) / (Cd * Dd));
    }
    *ssim_sum = ssum;
    // loss_l1_distortion_2dgs_kernel, metal:2704-2762.
    const float inv_num = 1.0f / (float)(height * width * 3);
    const float inv_HW = inv_num * 3.0f;
    double l = 0.0;
    for (int64_t pix = 0; pix < P; ++pix) {
        for (int c = 0; c < 3; ++c) {
            float diff = out_img[3 * pix + c] - gt[3 * pix + c];
            l += (double)(lambda_l1 * std::fabs(diff) * inv_num);
            float sg = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            dL_dout_img[3 * pix + c] = lambda_l1 * sg * inv_num;
        }
        l += (double)(lambda_dist * out_distortion[pix] * inv_HW);
        dL_dout_distortion[pix] = lambda_dist * inv_HW;
    }
    l += (double)lambda_dssim * (1.0 - ssum * (double)inv_num);
    *loss = l;
    // ssim_backward_compute_kernel, metal:2965-3047.
    const float g = -lambda_dssim * inv_num;
    std::vector<float> gm1(E), gs1(E), g12(E);
    for (int64_t e = 0; e < E; ++e) {
        float m1 = mu1[e], m2 = mu2[e];
        float m1s = m1 * m1, m2s = m2 * m2, m1m2 = m1 * m2;
        float v1 = b1[e] - m1s, v2 = b2[e] - m2s, v12 = b12[e] - m1m2;
        float A = 2.0f * m1m2 + C1, B = 2.0f * v12 + C2;
        float Cd = m1s + m2s + C1, Dd = v1 + v2 + C2;
        float CD = Cd * Dd, AB = A * B;
        float inv_CD = 1.0f / CD, inv_Cd = 1.0f / Cd, inv_Dd = 1.0f / Dd;
        float d_mu1 = 2.0f * inv_CD * (m2 * B - m1 * AB * inv_Cd);
        float d_s12 = 2.0f * A * inv_CD;
        float d_s1 = -AB * inv_CD * inv_Dd;
        float a_mu1 = g * d_mu1, a_s12 = g * d_s12, a_s1 = g * d_s1;
        a_mu1 += a_s1 * (-2.0f * m1);
        a_mu1 += a_s12 * (-m2);
        gm1[e] = a_mu1; gs1[e] = a_s1; g12[e] = a_s12;
    }
    // Re-blur (metal:3059-3085 inputs) and accumulate.
    std::vector<float> bgm1(E), bgs1(E), bg12(E);
    blur2d(width, height, gm1.data(), bgm1.data(), tmp.data());
    blur2d(width, height, gs1.data(), bgs1.data(), tmp.data());
    blur2d(width, height, g12.data(), bg12.data(), tmp.data());
    for (int64_t e = 0; e < E; ++e) {
        float a = out_img[e], b = gt[e];
        dL_dout_img[e] += bgm1[e] + 2.0f * a * bgs1[e] + b * bg12[e];
    }
}

void orc_rasterize_backward(int n, int width, int height, int tiles_x, const int32_t* tile_bins,
                            const int32_t* gaussian_ids, const float* packed_xy,
                            const float* packed_normal_opac, const float* packed_transmat,
                            const float* packed_rgb, const float* final_Ts,
                            const int32_t* final_idx, const float* background,
                            const float* dL_dout_img, const float* dL_dout_depth,
                            const float* dL_dout_alpha, const float* dL_dout_normal,
                            const float* dL_dout_median_depth, const float* dL_dout_distortion,
                            float* dL_dtransMat, float* dL_dmean2D, float* dL_dnormal3D,
                            float* dL_dopacity, float* dL_dcolors) {
    std::vector<double> gT((size_t)n * 9, 0.0), gM((size_t)n * 2, 0.0), gN((size_t)n * 3, 0.0),
        gO((size_t)n, 0.0), gC((size_t)n * 3, 0.0);
    const float mscale = kFarN / (kFarN - kNearN);
    const int64_t P = (int64_t)width * height;
    const int row_stride = g_row_stride;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t pix = 0; pix < P; ++pix) {
        int i = (int)(pix / width), j = (int)(pix % width);
        if ((i / kTile) % row_stride != 0) continue;
        int tile = (i / kTile) * tiles_x + (j / kTile);
        float px = (float)j, py = (float)i;
        int start = tile_bins[2 * tile], end = tile_bins[2 * tile + 1];
        const float T_final = final_Ts[3 * pix], final_D = final_Ts[3 * pix + 1],
                    final_D2 = final_Ts[3 * pix + 2];
        const float final_A = 1.0f - T_final;
        const int last_c = final_idx[2 * pix], median_c = final_idx[2 * pix + 1];
        float dpix[3] = {dL_dout_img[3 * pix], dL_dout_img[3 * pix + 1], dL_dout_img[3 * pix + 2]};
        float dL_ddepth = dL_dout_depth ? dL_dout_depth[pix] : 0.f;
        float dL_daccum = dL_dout_alpha ? dL_dout_alpha[pix] : 0.f;
        float dnorm2[3] = {0, 0, 0};
        if (dL_dout_normal)
            for (int c = 0; c < 3; ++c) dnorm2[c] = dL_dout_normal[3 * pix + c];
        float dL_dmed = dL_dout_median_depth ? dL_dout_median_depth[pix] : 0.f;
        float dL_dreg = dL_dout_distortion ? dL_dout_distortion[pix] : 0.f;
        float T = T_final;
        float accum_rec[3] = {0, 0, 0}, last_color[3] = {0, 0, 0};
        float last_alpha = 0.f, accum_depth_rec = 0.f, last_depth = 0.f, accum_alpha_rec = 0.f;
        float accum_normal_rec[3] = {0, 0, 0}, last_normal[3] = {0, 0, 0}, last_dL_dT = 0.f;
        const float bg_dot = background[0] * dpix[0] + background[1] * dpix[1] + background[2] * dpix[2];
        int contributor = end - start;
        for (int s = end - 1; s >= start; --s) {
            contributor--;
            if (contributor >= last_c) continue;
            const float* no = packed_normal_opac + 4 * s;
            PairEval e;
            if (!eval_pair(px, py, packed_xy + 2 * s, packed_transmat + 9 * s, no[3], &e)) continue;
            const float* tm = packed_transmat + 9 * s;
            F3 Tw = f3(tm[6], tm[7], tm[8]);
            const float alpha = e.alpha, G = e.G, opa = no[3];
            T = T / (1.0f - alpha);
            const float w = alpha * T;
            float dL_dalpha = 0.0f;
            const int gid = gaussian_ids[s];
            double gc[3];
            for (int c = 0; c < 3; ++c) {
                const float c_raw = packed_rgb[3 * s + c];
                const float c_used = std::max(c_raw + 0.5f, 0.0f);
                const float mask = (c_raw + 0.5f > 0.0f) ? 1.0f : 0.0f;
                accum_rec[c] = last_alpha * last_color[c] + (1.f - last_alpha) * accum_rec[c];
                last_color[c] = c_used;
                dL_dalpha += (c_used - accum_rec[c]) * dpix[c];
                gc[c] = (double)(w * dpix[c] * mask);
            }
            float dL_dz = 0.0f, dL_dweight = 0.0f;
            const float m_d = mscale * (1.0f - kNearN / e.depth);
            const float dmd_dd = (kFarN * kNearN) / ((kFarN - kNearN) * e.depth * e.depth);
            if (contributor == median_c - 1) dL_dz += dL_dmed;
            dL_dweight += (final_D2 + m_d * m_d * final_A - 2.0f * m_d * final_D) * dL_dreg;
            dL_dalpha += dL_dweight - last_dL_dT;
            last_dL_dT = dL_dweight * alpha + (1.0f - alpha) * last_dL_dT;
            const float dL_dmd = 2.0f * (T * alpha) * (m_d * final_A - final_D) * dL_dreg;
            dL_dz += dL_dmd * dmd_dd;
            accum_depth_rec = last_alpha * last_depth + (1.f - last_alpha) * accum_depth_rec;
            last_depth = e.depth;
            dL_dalpha += (e.depth - accum_depth_rec) * dL_ddepth;
            accum_alpha_rec = last_alpha * 1.0f + (1.f - last_alpha) * accum_alpha_rec;
            dL_dalpha += (1.0f - accum_alpha_rec) * dL_daccum;
            double gn[3];
            for (int c = 0; c < 3; ++c) {
                accum_normal_rec[c] = last_alpha * last_normal[c] + (1.f - last_alpha) * accum_normal_rec[c];
                last_normal[c] = no[c];
                dL_dalpha += (no[c] - accum_normal_rec[c]) * dnorm2[c];
                gn[c] = (double)(alpha * T * dnorm2[c]);
            }
            dL_dalpha *= T;
            last_alpha = alpha;
            dL_dalpha += (-T_final / (1.f - alpha)) * bg_dot;
            const float dL_dG = opa * dL_dalpha;
            dL_dz += alpha * T * dL_ddepth;
            double gt9[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0}, gm2[2] = {0, 0};
            if (e.rho3d <= e.rho2d) {
                const float dsx = dL_dG * -G * e.u + dL_dz * Tw.x;
                const float dsy = dL_dG * -G * e.v + dL_dz * Tw.y;
                const float dsx_pz = dsx / e.pz, dsy_pz = dsy / e.pz;
                F3 dp = f3(dsx_pz, dsy_pz, -(dsx_pz * e.u + dsy_pz * e.v));
                // cross(l, dp) and cross(dp, k).
                F3 dk = f3(e.l.y * dp.z - e.l.z * dp.y, e.l.z * dp.x - e.l.x * dp.z, e.l.x * dp.y - e.l.y * dp.x);
                F3 dl = f3(dp.y * e.k.z - dp.z * e.k.y, dp.z * e.k.x - dp.x * e.k.z, dp.x * e.k.y - dp.y * e.k.x);
                gt9[0] = -dk.x; gt9[1] = -dk.y; gt9[2] = -dk.z;
                gt9[3] = -dl.x; gt9[4] = -dl.y; gt9[5] = -dl.z;
                gt9[6] = px * dk.x + py * dl.x + dL_dz * e.u;
                gt9[7] = px * dk.y + py * dl.y + dL_dz * e.v;
                gt9[8] = px * dk.z + py * dl.z + dL_dz * 1.0f;
            } else {
                const float dGdx = -G * kFilterInvSq * e.dx;
                const float dGdy = -G * kFilterInvSq * e.dy;
                gm2[0] = dL_dG * dGdx;
                gm2[1] = dL_dG * dGdy;
                gt9[6] = e.u * dL_dz; gt9[7] = e.v * dL_dz; gt9[8] = dL_dz;
            }
            const float dsig = opa * (1.0f - opa);
            const double go = (double)(G * dL_dalpha * dsig);
            for (int c = 0; c < 3; ++c) {
#pragma omp atomic
                gC[3 * (size_t)gid + c] += gc[c];
#pragma omp atomic
                gN[3 * (size_t)gid + c] += gn[c];
            }
            for (int c = 0; c < 9; ++c) {
#pragma omp atomic
                gT[9 * (size_t)gid + c] += gt9[c];
            }
            for (int c = 0; c < 2; ++c) {
#pragma omp atomic
                gM[2 * (size_t)gid + c] += gm2[c];
            }
#pragma omp atomic
            gO[gid] += go;
        }
    }
    for (int64_t q = 0; q < (int64_t)n * 9; ++q) dL_dtransMat[q] = (float)gT[q];
    for (int64_t q = 0; q < (int64_t)n * 2; ++q) dL_dmean2D[q] = (float)gM[q];
    for (int64_t q = 0; q < (int64_t)n * 3; ++q) dL_dnormal3D[q] = (float)gN[q];
    for (int64_t q = 0; q < (int64_t)n; ++q) dL_dopacity[q] = (float)gO[q];
    for (int64_t q = 0; q < (int64_t)n * 3; ++q) dL_dcolors[q] = (float)gC[q];
}

void orc_project_backward(int n, const float* means, const float* scales, float glob_scale,
                          const float* quats, const OrcCamera* cam, const int32_t* radii,
                          const float* dT, const float* dN, const float* dC, int degree,
                          int degrees_to_use, const float* f_rest, float* dL_dmean3D,
                          float* dL_dscale, float* dL_dquat, float* dL_dmean2D,
                          float* dL_dfeatures_dc, float* dL_dfeatures_rest, float* xys_grad_norm,
                          float* vis_counts, float* max_2d_size, float inv_max_dim) {
    const int K = num_sh_bases(degree) - 1;
    const float* pm = cam->projmat;
    const float W = (float)cam->width, H = (float)cam->height;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        float* drest = dL_dfeatures_rest + (int64_t)K * 3 * i;
        for (int k = 0; k < K * 3; ++k) drest[k] = 0.f;  // blit-zeroed, mm:1304
        if (radii[i] <= 0) {
            for (int k = 0; k < 3; k++) dL_dmean3D[3 * i + k] = 0.f;
            for (int k = 0; k < 2; k++) dL_dscale[2 * i + k] = 0.f;
            for (int k = 0; k < 4; k++) dL_dquat[4 * i + k] = 0.f;
            for (int k = 0; k < 2; k++) dL_dmean2D[2 * i + k] = 0.f;
            for (int k = 0; k < 3; k++) dL_dfeatures_dc[3 * i + k] = 0.f;
            continue;
        }
        F3 p = f3(means[3 * i], means[3 * i + 1], means[3 * i + 2]);
        float ex = orc_exp(scales[2 * i]), ey = orc_exp(scales[2 * i + 1]);
        const float* q = quats + 4 * i;
        F3 R[3];
        quat_to_rotmat(q, R);
        float sx = ex * glob_scale, sy = ey * glob_scale;
        float pcw = pm[12] * p.x + pm[13] * p.y + pm[14] * p.z + pm[15];
        float halfW = 0.5f * W, halfH = 0.5f * H, bx = cam->cx - 0.5f, by = cam->cy - 0.5f;
        const float* g = dT + 9 * i;
        F3 dcu = f3(g[0], g[3], g[6]), dcv = f3(g[1], g[4], g[7]), dco = f3(g[2], g[5], g[8]);
        float dtu[4] = {halfW * dcu.x, halfH * dcu.y, 0.0f, bx * dcu.x + by * dcu.y + dcu.z};
        float dtv[4] = {halfW * dcv.x, halfH * dcv.y, 0.0f, bx * dcv.x + by * dcv.y + dcv.z};
        float dpc[4] = {halfW * dco.x, halfH * dco.y, 0.0f, bx * dco.x + by * dco.y + dco.z};
        auto back = [&](const float* d) {
            return f3(pm[0] * d[0] + pm[4] * d[1] + pm[8] * d[2] + pm[12] * d[3],
                      pm[1] * d[0] + pm[5] * d[1] + pm[9] * d[2] + pm[13] * d[3],
                      pm[2] * d[0] + pm[6] * d[1] + pm[10] * d[2] + pm[14] * d[3]);
        };
        F3 dtuw = back(dtu), dtvw = back(dtv), dpo = back(dpc);
        float dsx = dot3(dtuw, R[0]), dsy = dot3(dtvw, R[1]);
        dL_dscale[2 * i] = dsx * ex * glob_scale;
        dL_dscale[2 * i + 1] = dsy * ey * glob_scale;
        F3 vR[3] = {scale3(dtuw, sx), scale3(dtvw, sy), f3(dN[3 * i], dN[3 * i + 1], dN[3 * i + 2])};
        quat_to_rotmat_vjp(q, vR, dL_dquat + 4 * i);
        F3 v = f3(p.x - cam->cam_pos[0], p.y - cam->cam_pos[1], p.z - cam->cam_pos[2]);
        float inv = 1.0f / std::sqrt(dot3(v, v));
        F3 dir = scale3(v, inv);
        const float* rest = f_rest + (int64_t)K * 3 * i;
        sh_to_color_vjp(degrees_to_use, dir, dC + 3 * i, dL_dfeatures_dc + 3 * i, drest);
        if (degrees_to_use >= 1) {
            F3 ddir = sh_color_dL_ddir(degrees_to_use, dir, rest, dC + 3 * i);
            F3 dpv = dnormvdv(v, ddir);
            dpo = f3(dpo.x + dpv.x, dpo.y + dpv.y, dpo.z + dpv.z);
        }
        dL_dmean3D[3 * i] = dpo.x; dL_dmean3D[3 * i + 1] = dpo.y; dL_dmean3D[3 * i + 2] = dpo.z;
        float dmx = g[6] * pcw * 0.5f * W;
        float dmy = g[7] * pcw * 0.5f * H;
        dL_dmean2D[2 * i] = dmx; dL_dmean2D[2 * i + 1] = dmy;
        xys_grad_norm[i] += std::fabs(dmx) + std::fabs(dmy);
        vis_counts[i] += 1.0f;
        float r_norm = float(radii[i]) * inv_max_dim;
        if (r_norm > max_2d_size[i]) max_2d_size[i] = r_norm;
    }
}

void orc_fused_adam(float* params, const float* grads, float* m_, float* v_, int64_t n,
                    float step_size, float beta1, float beta2, float bc2_sqrt, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < n; ++t) {
        float gr = grads[t];
        float m = std::fma(beta1, m_[t], (1.0f - beta1) * gr);
        float v = std::fma(beta2, v_[t], (1.0f - beta2) * gr * gr);
        params[t] -= step_size * m / (std::sqrt(v) / bc2_sqrt + eps);
        m_[t] = m;
        v_[t] = v;
    }
}

namespace {
struct Forward {
    std::vector<float> xys, depths, transmats, normal_opacity, colors, aabb;
    std::vector<int32_t> radii, tiles_hit, tile_bins, ids;
    std::vector<int64_t> raw;
    std::vector<float> pxy, ptm, pno, prgb;
    std::vector<float> final_Ts, out_img, out_depth, out_normal, out_alpha, out_median, out_dist;
    std::vector<int32_t> final_idx;
    int64_t kept = 0;
};

void run_forward(int n, const float* means, const float* scales, const float* quats,
                 const float* opac, const float* f_dc, const float* f_rest, int degree,
                 int degrees_to_use, const float* bg, const OrcCamera* cam, Forward& F) {
    const int tx = (cam->width + kTile - 1) / kTile, ty = (cam->height + kTile - 1) / kTile;
    const int64_t P = (int64_t)cam->width * cam->height;
    F.xys.resize(2 * (size_t)n); F.depths.resize(n); F.radii.resize(n);
    F.transmats.resize(9 * (size_t)n); F.tiles_hit.resize(n); F.normal_opacity.resize(4 * (size_t)n);
    F.colors.resize(3 * (size_t)n); F.aabb.resize(2 * (size_t)n);
    orc_project_forward(n, means, scales, 1.0f, quats, opac, f_dc, f_rest, degree, degrees_to_use, cam,
                        0.01f, F.xys.data(), F.depths.data(), F.radii.data(), F.transmats.data(),
                        F.tiles_hit.data(), F.normal_opacity.data(), F.colors.data(), F.aabb.data());
    int64_t cap = (int64_t)tx * ty * kMaxTileElems;
    int64_t total = 0;
    for (int i = 0; i < n; ++i) total += F.tiles_hit[i];
    cap = std::min<int64_t>(cap, total);
    F.raw.resize((size_t)tx * ty); F.tile_bins.resize(2 * (size_t)tx * ty); F.ids.resize(std::max<int64_t>(cap, 1));
    F.kept = orc_bin_and_sort(n, F.xys.data(), F.depths.data(), F.radii.data(), F.aabb.data(), tx, ty,
                              F.raw.data(), F.tile_bins.data(), F.ids.data(), cap);
    int64_t k = std::max<int64_t>(F.kept, 1);
    F.pxy.resize(2 * k); F.ptm.resize(9 * k); F.pno.resize(4 * k); F.prgb.resize(3 * k);
    orc_pack(F.kept, F.ids.data(), F.xys.data(), F.transmats.data(), F.normal_opacity.data(),
             F.colors.data(), F.pxy.data(), F.ptm.data(), F.pno.data(), F.prgb.data());
    F.final_Ts.resize(3 * P); F.final_idx.resize(2 * P); F.out_img.resize(3 * P); F.out_depth.resize(P);
    F.out_normal.resize(3 * P); F.out_alpha.resize(P); F.out_median.resize(P); F.out_dist.resize(P);
    orc_rasterize_forward(cam->width, cam->height, tx, F.tile_bins.data(), F.pxy.data(), F.pno.data(),
                          F.ptm.data(), F.prgb.data(), bg, F.final_Ts.data(), F.final_idx.data(),
                          F.out_img.data(), F.out_depth.data(), F.out_normal.data(), F.out_alpha.data(),
                          F.out_median.data(), F.out_dist.data());
}
}  // namespace

void orc_render(int n, const float* means, const float* scales, const float* quats,
                const float* opacities, const float* f_dc, const float* f_rest, int degree,
                int degrees_to_use, const float* background, const OrcCamera* cam, float* out_img) {
    Forward F;
    run_forward(n, means, scales, quats, opacities, f_dc, f_rest, degree, degrees_to_use, background, cam, F);
    std::memcpy(out_img, F.out_img.data(), F.out_img.size() * sizeof(float));
}

void orc_render_rows(int n, const float* means, const float* scales, const float* quats, const float* opacities,
                     const float* f_dc, const float* f_rest, int degree, int degrees_to_use,
                     const float* background, const OrcCamera* cam, int pixel_rows, float* out_img) {
    g_row_limit = pixel_rows;
    Forward F;
    run_forward(n, means, scales, quats, opacities, f_dc, f_rest, degree, degrees_to_use, background, cam, F);
    g_row_limit = 1 << 30;
    std::memcpy(out_img, F.out_img.data(), F.out_img.size() * sizeof(float));
}

float orc_train_step(const OrcStepArgs* a, const OrcCamera* cam, float* grads_out, float* out_img_out,
                     int64_t* kept_out) {
    const int n = a->n;
    const int K = num_sh_bases(a->degree) - 1;
    const int W = cam->width, H = cam->height, tx = (W + kTile - 1) / kTile;
    const int64_t P = (int64_t)W * H;
    Forward F;
    run_forward(n, a->means, a->scales, a->quats, a->opacities, a->f_dc, a->f_rest, a->degree,
                a->degrees_to_use, a->background, cam, F);
    if (kept_out) *kept_out = F.kept;
    if (out_img_out) std::memcpy(out_img_out, F.out_img.data(), 3 * P * sizeof(float));
    std::vector<float> dimg(3 * P), ddist(P), zeros1(P, 0.f), zeros3(3 * P, 0.f);
    double loss = 0, ssum = 0;
    orc_loss_ssim(W, H, F.out_img.data(), a->gt, F.out_dist.data(), a->lambda_l1, a->lambda_dist,
                  a->lambda_dssim, dimg.data(), ddist.data(), &loss, &ssum);
    std::vector<float> dT(9 * (size_t)n), dM2(2 * (size_t)n), dN(3 * (size_t)n), dO(n), dC(3 * (size_t)n);
    orc_rasterize_backward(n, W, H, tx, F.tile_bins.data(), F.ids.data(), F.pxy.data(), F.pno.data(),
                           F.ptm.data(), F.prgb.data(), F.final_Ts.data(), F.final_idx.data(),
                           a->background, dimg.data(), zeros1.data(), zeros1.data(), zeros3.data(),
                           zeros1.data(), ddist.data(), dT.data(), dM2.data(), dN.data(), dO.data(),
                           dC.data());
    std::vector<float> gmean(3 * (size_t)n), gscale(2 * (size_t)n), gquat(4 * (size_t)n),
        gdc(3 * (size_t)n), grest((size_t)3 * K * n + 1);
    float inv_max_dim = 1.0f / (float)std::max(W, H);
    orc_project_backward(n, a->means, a->scales, 1.0f, a->quats, cam, F.radii.data(), dT.data(), dN.data(),
                         dC.data(), a->degree, a->degrees_to_use, a->f_rest, gmean.data(), gscale.data(),
                         gquat.data(), dM2.data(), gdc.data(), grest.data(), a->xys_grad_norm,
                         a->vis_counts, a->max_2d_size, inv_max_dim);
    // Model::fullIteration Adam loop, model.cpp:766-826.
    const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    // std::pow(float, int) promotes to double, as in model.cpp:768-769.
    float bc1 = 1.0f - std::pow(b1, a->adam_step);
    float bc2 = 1.0f - std::pow(b2, a->adam_step);
    float bc2_sqrt = std::sqrt(bc2);
    float* params[6] = {a->means, a->scales, a->quats, a->f_dc, a->f_rest, a->opacities};
    const float* grads[6] = {gmean.data(), gscale.data(), gquat.data(), gdc.data(), grest.data(), dO.data()};
    int64_t counts[6] = {3LL * n, 2LL * n, 4LL * n, 3LL * n, 3LL * K * n, (int64_t)n};
    int64_t off = 0;
    for (int gi = 0; gi < 6; ++gi) {
        if (grads_out) std::memcpy(grads_out + off, grads[gi], counts[gi] * sizeof(float));
        off += counts[gi];
        if (counts[gi] == 0) continue;
        orc_fused_adam(params[gi], grads[gi], a->exp_avg[gi], a->exp_avg_sq[gi], counts[gi],
                       a->lr[gi] / bc1, b1, b2, bc2_sqrt, eps);
    }
    return (float)loss;
}

double orc_time_step_sample(const OrcStepArgs* a, const OrcCamera* cam, int tile_row_stride,
                            double* stage_seconds) {
    // Bounded CPU sample of one training step (see oracle.h).
    using clk = std::chrono::steady_clock;
    auto secs = [](clk::time_point t0) { return std::chrono::duration<double>(clk::now() - t0).count(); };
    const int S = tile_row_stride < 1 ? 1 : tile_row_stride;
    const int n = a->n;
    const int K = num_sh_bases(a->degree) - 1;
    const int W = cam->width, H = cam->height, tx = (W + kTile - 1) / kTile, ty = (H + kTile - 1) / kTile;
    const int64_t P = (int64_t)W * H;
    double st[7] = {0, 0, 0, 0, 0, 0, 0};
    Forward F;
    auto t0 = clk::now();
    F.xys.resize(2 * (size_t)n); F.depths.resize(n); F.radii.resize(n); F.transmats.resize(9 * (size_t)n);
    F.tiles_hit.resize(n); F.normal_opacity.resize(4 * (size_t)n); F.colors.resize(3 * (size_t)n);
    F.aabb.resize(2 * (size_t)n);
    orc_project_forward(n, a->means, a->scales, 1.0f, a->quats, a->opacities, a->f_dc, a->f_rest, a->degree,
                        a->degrees_to_use, cam, 0.01f, F.xys.data(), F.depths.data(), F.radii.data(),
                        F.transmats.data(), F.tiles_hit.data(), F.normal_opacity.data(), F.colors.data(),
                        F.aabb.data());
    st[0] = secs(t0);
    t0 = clk::now();
    int64_t cap = (int64_t)tx * ty * kMaxTileElems;
    F.raw.resize((size_t)tx * ty); F.tile_bins.resize(2 * (size_t)tx * ty); F.ids.resize(cap);
    F.kept = orc_bin_and_sort(n, F.xys.data(), F.depths.data(), F.radii.data(), F.aabb.data(), tx, ty,
                              F.raw.data(), F.tile_bins.data(), F.ids.data(), cap);
    int64_t k = std::max<int64_t>(F.kept, 1);
    F.pxy.resize(2 * k); F.ptm.resize(9 * k); F.pno.resize(4 * k); F.prgb.resize(3 * k);
    orc_pack(F.kept, F.ids.data(), F.xys.data(), F.transmats.data(), F.normal_opacity.data(), F.colors.data(),
             F.pxy.data(), F.ptm.data(), F.pno.data(), F.prgb.data());
    st[1] = secs(t0);
    F.final_Ts.resize(3 * P); F.final_idx.resize(2 * P); F.out_img.resize(3 * P); F.out_depth.resize(P);
    F.out_normal.resize(3 * P); F.out_alpha.resize(P); F.out_median.resize(P); F.out_dist.resize(P);
    g_row_stride = S;
    t0 = clk::now();
    orc_rasterize_forward(W, H, tx, F.tile_bins.data(), F.pxy.data(), F.pno.data(), F.ptm.data(), F.prgb.data(),
                          a->background, F.final_Ts.data(), F.final_idx.data(), F.out_img.data(), F.out_depth.data(),
                          F.out_normal.data(), F.out_alpha.data(), F.out_median.data(), F.out_dist.data());
    st[2] = secs(t0) * S;
    // loss on a band of H/S rows (same per-pixel work), scaled by S
    const int hb = std::max(1, H / S);
    std::vector<float> dimg(3 * P, 0.f), ddist(P, 0.f);
    double loss = 0, ssum = 0;
    t0 = clk::now();
    orc_loss_ssim(W, hb, F.out_img.data(), a->gt, F.out_dist.data(), a->lambda_l1, a->lambda_dist, a->lambda_dssim,
                  dimg.data(), ddist.data(), &loss, &ssum);
    st[3] = secs(t0) * ((double)H / hb);
    std::vector<float> zeros1(P, 0.f), zeros3(3 * P, 0.f);
    std::vector<float> dT(9 * (size_t)n), dM2(2 * (size_t)n), dN(3 * (size_t)n), dO(n), dC(3 * (size_t)n);
    t0 = clk::now();
    orc_rasterize_backward(n, W, H, tx, F.tile_bins.data(), F.ids.data(), F.pxy.data(), F.pno.data(), F.ptm.data(),
                           F.prgb.data(), F.final_Ts.data(), F.final_idx.data(), a->background, dimg.data(),
                           zeros1.data(), zeros1.data(), zeros3.data(), zeros1.data(), ddist.data(), dT.data(),
                           dM2.data(), dN.data(), dO.data(), dC.data());
    st[4] = secs(t0) * S;
    g_row_stride = 1;
    std::vector<float> gmean(3 * (size_t)n), gscale(2 * (size_t)n), gquat(4 * (size_t)n), gdc(3 * (size_t)n),
        grest((size_t)3 * K * n + 1);
    t0 = clk::now();
    orc_project_backward(n, a->means, a->scales, 1.0f, a->quats, cam, F.radii.data(), dT.data(), dN.data(), dC.data(),
                         a->degree, a->degrees_to_use, a->f_rest, gmean.data(), gscale.data(), gquat.data(),
                         dM2.data(), gdc.data(), grest.data(), a->xys_grad_norm, a->vis_counts, a->max_2d_size,
                         1.0f / (float)std::max(W, H));
    st[5] = secs(t0);
    t0 = clk::now();
    float* params[6] = {a->means, a->scales, a->quats, a->f_dc, a->f_rest, a->opacities};
    const float* grads[6] = {gmean.data(), gscale.data(), gquat.data(), gdc.data(), grest.data(), dO.data()};
    int64_t counts[6] = {3LL * n, 2LL * n, 4LL * n, 3LL * n, 3LL * K * n, (int64_t)n};
    for (int gi = 0; gi < 6; ++gi)
        if (counts[gi])
            orc_fused_adam(params[gi], grads[gi], a->exp_avg[gi], a->exp_avg_sq[gi], counts[gi], a->lr[gi] / 0.1f,
                           0.9f, 0.999f, 0.0447f, 1e-8f);
    st[6] = secs(t0);
    double total = 0;
    for (int q = 0; q < 7; ++q) {
        total += st[q];
        if (stage_seconds) stage_seconds[q] = st[q];
    }
    return total;
}


void orc_normal_samples(uint32_t seed, int64_t count, float* out) {
    // model.cpp:254-259
    std::mt19937 rng(seed);
    std::normal_distribution<float> dist(0.0f, 1.0f);
    for (int64_t i = 0; i < count; ++i) out[i] = dist(rng);
}

int orc_densify(int n, int cap, int rest_bases, const OrcDensifyArgs* a, const float* xys_grad_norm,
                const float* vis_counts, const float* max_2d_size, float* const params[6], float* const m[6],
                float* const v[6], const float* random_samples, int* num_splits, int* num_dups) {
    const int K3 = 3 * rest_bases;
    const int w[6] = {3, 2, 4, 3, K3, 1};
    float* means = params[0];
    float* scales = params[1];
    float* quats = params[2];
    float* opac = params[5];
    // Stage 1: densify_classify_kernel (metal:3231-3263)
    std::vector<int> split(n, 0), dup(n, 0);
    for (int i = 0; i < n; ++i) {
        const float vc = vis_counts[i];
        if (vc <= 0.0f) continue;
        const float avg_grad = (xys_grad_norm[i] / vc) * a->half_max_dim;
        const bool high_grad = avg_grad > a->grad_thresh;
        float max_scale = orc_exp(scales[2 * i]);
        max_scale = std::fmax(max_scale, orc_exp(scales[2 * i + 1]));
        const bool is_large = max_scale > a->size_thresh;
        bool do_split = is_large;
        if (a->check_screen && max_2d_size[i] > a->screen_thresh) do_split = true;
        do_split = do_split && high_grad;
        split[i] = do_split ? 1 : 0;
        dup[i] = (!is_large && high_grad) ? 1 : 0;
    }
    // Stages 2-3: inclusive prefix sums of the flags
    std::vector<int> split_prefix(n), dup_prefix(n);
    int acc_s = 0, acc_d = 0;
    for (int i = 0; i < n; ++i) {
        acc_s += split[i];
        acc_d += dup[i];
        split_prefix[i] = acc_s;
        dup_prefix[i] = acc_d;
    }
    const int S = acc_s, D = acc_d;
    if (num_splits) *num_splits = S;
    if (num_dups) *num_dups = D;
    const int n_new = n + 2 * S + D;
    if (n_new > cap) return -1;
    // Stage 4: densify_append_split_kernel (metal:3265-3340)
    for (int i = 0; i < n; ++i) {
        if (!split[i]) continue;
        const int ord = split_prefix[i] - 1;
        const int c0 = n + 2 * ord;
        float qw = quats[i * 4], qx = quats[i * 4 + 1], qy = quats[i * 4 + 2], qz = quats[i * 4 + 3];
        const float qlen = std::sqrt(qw * qw + qx * qx + qy * qy + qz * qz);
        qw /= qlen; qx /= qlen; qy /= qlen; qz /= qlen;
        const float sx = orc_exp(scales[i * 2]);
        const float sy = orc_exp(scales[i * 2 + 1]);
        const float sz = 0.0f;  // 2DGS: no third axis
        for (int k = 0; k < 2; ++k) {
            const int child = c0 + k;
            const int ri = ord * 2 + k;
            const float r0 = random_samples[ri * 3] * sx;
            const float r1 = random_samples[ri * 3 + 1] * sy;
            const float r2 = random_samples[ri * 3 + 2] * sz;
            const float v0 = (1 - 2 * (qy * qy + qz * qz)) * r0 + 2 * (qx * qy - qw * qz) * r1 + 2 * (qx * qz + qw * qy) * r2;
            const float v1 = 2 * (qx * qy + qw * qz) * r0 + (1 - 2 * (qx * qx + qz * qz)) * r1 + 2 * (qy * qz - qw * qx) * r2;
            const float v2 = 2 * (qx * qz - qw * qy) * r0 + 2 * (qy * qz + qw * qx) * r1 + (1 - 2 * (qx * qx + qy * qy)) * r2;
            means[child * 3] = means[i * 3] + v0;
            means[child * 3 + 1] = means[i * 3 + 1] + v1;
            means[child * 3 + 2] = means[i * 3 + 2] + v2;
            for (int j = 0; j < 2; ++j) scales[child * 2 + j] = scales[i * 2 + j] - a->log_size_fac;
            for (int gi = 2; gi < 6; ++gi)
                for (int j = 0; j < w[gi]; ++j) params[gi][(size_t)child * w[gi] + j] = params[gi][(size_t)i * w[gi] + j];
            for (int gi = 0; gi < 6; ++gi)
                for (int j = 0; j < w[gi]; ++j) {
                    m[gi][(size_t)child * w[gi] + j] = 0.0f;
                    v[gi][(size_t)child * w[gi] + j] = 0.0f;
                }
        }
        for (int j = 0; j < 2; ++j) scales[i * 2 + j] -= a->log_size_fac;
    }
    // Stage 5: densify_append_dup_kernel (metal:3342-3394)
    for (int i = 0; i < n; ++i) {
        if (!dup[i]) continue;
        const int dst = n + 2 * S + dup_prefix[i] - 1;
        for (int gi = 0; gi < 6; ++gi)
            for (int j = 0; j < w[gi]; ++j) {
                params[gi][(size_t)dst * w[gi] + j] = params[gi][(size_t)i * w[gi] + j];
                m[gi][(size_t)dst * w[gi] + j] = 0.0f;
                v[gi][(size_t)dst * w[gi] + j] = 0.0f;
            }
    }
    // Stage 6: densify_cull_classify_kernel (metal:3408-3441)
    std::vector<int> keep(n_new, 0);
    for (int idx = 0; idx < n_new; ++idx) {
        const float opacity_sigmoid = 1.0f / (1.0f + orc_exp(-opac[idx]));
        bool cull = opacity_sigmoid < a->cull_alpha_thresh;
        if (idx < n && split[idx]) cull = true;
        if (a->check_huge) {
            float max_s = orc_exp(scales[idx * 2]);
            max_s = std::fmax(max_s, orc_exp(scales[idx * 2 + 1]));
            if (max_s > a->cull_scale_thresh) cull = true;
            if (a->check_screen && idx < n && max_2d_size[idx] > a->cull_screen_size) cull = true;
        }
        keep[idx] = cull ? 0 : 1;
    }
    // Stages 7-8: keep prefix and compaction, every group with its own row size
    int out = 0;
    std::vector<int> dst_of(n_new, -1);
    for (int idx = 0; idx < n_new; ++idx)
        if (keep[idx]) dst_of[idx] = out++;
    float* const* groups[3] = {params, m, v};
    for (int t = 0; t < 3; ++t)
        for (int gi = 0; gi < 6; ++gi) {
            float* buf = groups[t][gi];
            if (w[gi] == 0) continue;
            for (int idx = 0; idx < n_new; ++idx) {
                const int d = dst_of[idx];
                if (d < 0 || d == idx) continue;
                std::memmove(buf + (size_t)d * w[gi], buf + (size_t)idx * w[gi], sizeof(float) * w[gi]);
            }
        }
    return out;
}

}  // extern "C"
