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

#include "sh_math.cuh"

namespace msplat {
namespace {

// Parameter pointers for Gaussian i: the local arrays, or with peers the
// arrays of the owner rank (indexed by the global id either way).
struct ParamPtrs {
    const float *means, *scales, *quats, *f_dc, *f_rest, *opacities;
};
__device__ __forceinline__ ParamPtrs param_ptrs(const ProjFwdArgs& a, int i) {
    if (a.peer_world > 1) {
        const int q = i / a.peer_chunk;
        return ParamPtrs{a.means, a.scales, a.quats, a.peer_dc[q], a.peer_rest[q], a.opacities};
    }
    return ParamPtrs{a.means, a.scales, a.quats, a.f_dc, a.f_rest, a.opacities};
}

// SH colour of Gaussian i for the camera position: raw colour (reference
// output) and the clamped colour max(raw + 0.5, 0) the rasteriser blends.
// rest_smem: the Gaussian's 3K rest coefficients already in shared memory
// (null: read them from global memory).
__device__ __forceinline__ void gaussian_color(const ProjFwdArgs& a, const ParamPtrs& pp, int i, V3 p, float col[3],
                                               float rgb[3], const float* rest_smem = nullptr) {
    const CameraDev& cam = a.cam;
    V3 v = v3(p.x - cam.cam_pos[0], p.y - cam.cam_pos[1], p.z - cam.cam_pos[2]);
    float inv = 1.0f / sqrtf(dot3(v, v));
    V3 dir = scale3(v, inv);
    const int K = a.rest_bases;
    if (rest_smem) {
        sh_to_color(a.degrees_to_use, dir, pp.f_dc + 3 * i, [&](int k) { return rest_smem[k]; }, col);
    } else {
        const float* rest = pp.f_rest + (size_t)K * 3 * i;
        sh_to_color(a.degrees_to_use, dir, pp.f_dc + 3 * i, [&](int k) { return __ldg(rest + k); }, col);
    }
    for (int c = 0; c < 3; ++c) rgb[c] = smax(col[c] + 0.5f, 0.0f);
}

// Whether a launch stages the rest coefficients through shared memory: the
// full projection (pass 0) with local coefficients on a 16-byte boundary.
__host__ __device__ __forceinline__ bool stage_rest(const ProjFwdArgs& a) {
    return a.pass == 0 && a.peer_world <= 1 && a.rest_bases > 0 &&
           (reinterpret_cast<uintptr_t>(a.f_rest) & 15) == 0;
}

// Cull record of one surfel (layout in common.cuh). With k = x Tw - Tu and
// l = y Tw - Tv, the ray/plane intersection before the division is
// p = k x l = M (x, y, 1) with columns m0 = Tv x Tw, m1 = Tw x Tu,
// m2 = Tu x Tv, so rho3d = (p.x^2 + p.y^2) / p.z^2 <= r is the conic
// Q(x, y) = p.x^2 + p.y^2 - r p.z^2 <= 0 with 2x2 part A (entries m_i^T W m_j,
// W = diag(1, 1, -r)). Since T M = det(T) I for T = (Tu; Tv; Tw), its centre
// (the pole of the line at infinity) is (Tu . w, Tv . w) / dd with
// w = (r Tw.x, r Tw.y, -Tw.z) and dd = Tw . w, det A = det(T)^2 (-dd), and its
// minimum Q(centre) = det(Q) / det(A) = r det(T)^2 / dd. These closed forms
// avoid the cancellation of evaluating Q at a rounded centre. It is an
// ellipse when dd < 0; the record stores the factors of E = A / -Q(centre):
// s1 = sqrt(E.xx), t1 = E.xy / s1, s2 = sqrt(det E / E.xx). Computed in double
// from the float rows (products of two floats are exact in double);
// (tr A)^2 / det A bounds the squared axis ratio.
__device__ void cull_record(V3 tu, V3 tv, V3 tw, float rmax, float4* out) {
    if (!(rmax > 0.f)) {
        out[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        out[1] = make_float4(0.f, 0.f, 0.f, -1.f);
        return;
    }
    const double r = (double)rmax * (double)kCullRhoScale;
    const double ux = tu.x, uy = tu.y, uz = tu.z, vx = tv.x, vy = tv.y, vz = tv.z, wx = tw.x, wy = tw.y, wz = tw.z;
    const double m0x = vy * wz - vz * wy, m0y = vz * wx - vx * wz, m0z = vx * wy - vy * wx;
    const double m1x = wy * uz - wz * uy, m1y = wz * ux - wx * uz, m1z = wx * uy - wy * ux;
    const double qa = m0x * m0x + m0y * m0y - r * m0z * m0z;
    const double qb = m0x * m1x + m0y * m1y - r * m0z * m1z;
    const double qc = m1x * m1x + m1y * m1y - r * m1z * m1z;
    const double det_t = ux * m0x + uy * m0y + uz * m0z;
    const double dd = r * (wx * wx + wy * wy) - wz * wz;
    const double det_a = det_t * det_t * -dd;
    const float rd = sqrtf(0.5f * rmax * kCullRhoScale) + kCullMargin;
    float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = make_float4(0.f, 0.f, 0.f, rd * rd);
    if (dd < 0.0 && det_t != 0.0 && qa > 0.0 && (qa + qc) * (qa + qc) <= kCullMaxAspect * kCullMaxAspect * det_a) {
        const double cx = (r * (ux * wx + uy * wy) - uz * wz) / dd;
        const double cy = (r * (vx * wx + vy * wy) - vz * wz) / dd;
        const double sc = -dd / (r * det_t * det_t);   // -1 / Q(centre)
        const double s1 = sqrt(qa * sc);
        c0 = make_float4((float)cx, (float)cy, (float)s1, (float)(qb * sc / s1));
        c1.x = (float)sqrt(det_a * sc / qa);
        c1.y = (float)(-qb / qc);
        c1.z = (float)(-qb / qa);
    }
    out[0] = c0;
    out[1] = c1;
}

__global__ void __launch_bounds__(256, 4) k_project_forward(ProjFwdArgs a) {
    // pass 0: each full warp copies its 32 Gaussians' rest coefficients (one
    // contiguous run of 32 x 3K floats, 16-byte aligned) into shared memory
    // with coalesced 16-byte cp.async copies before any lane leaves; lane l's
    // coefficients then sit at an odd stride (3K) of floats
    extern __shared__ float4 srest4[];
    const float* rest_smem = nullptr;
    {
        const int warp_first = blockIdx.x * blockDim.x + (threadIdx.x & ~31);
        const int K3 = 3 * a.rest_bases;
        if (stage_rest(a) && warp_first + 32 <= a.n) {
            float4* dst = srest4 + (size_t)(threadIdx.x >> 5) * (8 * K3);  // 32 x 3K floats = 8 x 3K float4
            const float4* src = reinterpret_cast<const float4*>(a.f_rest + (size_t)warp_first * K3);
            for (int k = threadIdx.x & 31; k < 8 * K3; k += 32) cp_async16(dst + k, src + k);
            cp_async_wait_all();
            __syncwarp();
            rest_smem = reinterpret_cast<const float*>(dst) + (threadIdx.x & 31) * K3;
        }
    }
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    const CameraDev& cam = a.cam;
    const float* vm = cam.viewmat;
    const float* pm = cam.projmat;
    float4* rec = a.records + (size_t)i * kRecordF4;
    const ParamPtrs pp = param_ptrs(a, i);
    if (a.pass == 2) {
        if (a.radii[i] <= 0) return;
        if (a.color_row1 > a.color_row0) {
            const uint2 rc = a.rects[i];
            if ((int)(rc.y >> 16) <= a.color_row0 || (int)(rc.x >> 16) >= a.color_row1) return;
        }
        if (a.rgb_in) {
            float* r3 = reinterpret_cast<float*>(rec + 3);
            r3[0] = a.rgb_in[3 * i]; r3[1] = a.rgb_in[3 * i + 1]; r3[2] = a.rgb_in[3 * i + 2];
            return;
        }
        float col[3], rgb[3];
        gaussian_color(a, pp, i, v3(pp.means[3 * i], pp.means[3 * i + 1], pp.means[3 * i + 2]), col, rgb);
        float* r3 = reinterpret_cast<float*>(rec + 3);
        r3[0] = rgb[0]; r3[1] = rgb[1]; r3[2] = rgb[2];
        if (a.colors)
            for (int c = 0; c < 3; ++c) a.colors[3 * i + c] = col[c];
        return;
    }
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
    // every parameter load is issued before the first dependent arithmetic
    V3 p = v3(__ldg(pp.means + 3 * i), __ldg(pp.means + 3 * i + 1), __ldg(pp.means + 3 * i + 2));
    const float s0 = __ldg(pp.scales + 2 * i), s1 = __ldg(pp.scales + 2 * i + 1);
    float q[4];
    if ((reinterpret_cast<uintptr_t>(pp.quats) & 15) == 0) {
        const float4 qv = __ldg(reinterpret_cast<const float4*>(pp.quats) + i);
        q[0] = qv.x; q[1] = qv.y; q[2] = qv.z; q[3] = qv.w;
    } else {
        for (int k = 0; k < 4; ++k) q[k] = __ldg(pp.quats + 4 * i + k);
    }
    const float opac_raw = __ldg(pp.opacities + i);
    float pvz = vm[8] * p.x + vm[9] * p.y + vm[10] * p.z + vm[11];
    if (pvz <= a.clip_thresh) return;
    float sx = det_exp(s0) * a.glob_scale;
    float sy = det_exp(s1) * a.glob_scale;
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
    int32_t* diff = a.tile_diff + (size_t)(i / a.id_chunk) * dw * (cam.tiles_y + 1);
    atomicAdd(&diff[y0 * dw + x0], 1);
    atomicAdd(&diff[y0 * dw + x1], -1);
    atomicAdd(&diff[y1 * dw + x0], -1);
    atomicAdd(&diff[y1 * dw + x1], 1);

    float col[3] = {0.f, 0.f, 0.f}, rgb[3] = {0.f, 0.f, 0.f};
    if (a.pass == 0) gaussian_color(a, pp, i, p, col, rgb, rest_smem);
    float opac = 1.f / (1.f + det_exp(-opac_raw));
    V3 nrm = R[2];
    rec[0] = make_float4(T0.x, T0.y, T0.z, T1.x);
    rec[1] = make_float4(T1.y, T1.z, T2.x, T2.y);
    rec[2] = make_float4(T2.z, cxp, cyp, opac);
    rec[3] = make_float4(rgb[0], rgb[1], rgb[2], nrm.x);
    const float rmax = reject_rho(opac);
    rec[4] = make_float4(nrm.y, nrm.z, rmax, 0.f);
    cull_record(T0, T1, T2, rmax, a.cull + (size_t)i * kCullF4);
    if (a.num_tiles_hit) {
        a.num_tiles_hit[i] = area;
        a.xys[2 * i] = cxp; a.xys[2 * i + 1] = cyp;
        float tm[9] = {T0.x, T0.y, T0.z, T1.x, T1.y, T1.z, T2.x, T2.y, T2.z};
        for (int k = 0; k < 9; ++k) a.transmats[9 * i + k] = tm[k];
        a.normal_opacity[4 * i + 0] = nrm.x; a.normal_opacity[4 * i + 1] = nrm.y;
        a.normal_opacity[4 * i + 2] = nrm.z; a.normal_opacity[4 * i + 3] = opac_raw;
        if (a.pass == 0)
            for (int c = 0; c < 3; ++c) a.colors[3 * i + c] = col[c];
        a.aabb[2 * i] = radius; a.aabb[2 * i + 1] = radius;
    }
}

// Colour pass for ranks that read colour coefficients from their owners
// (pass 2 with peers): each warp selects, among its 32 Gaussians, those kept
// by the geometry pass whose tile rectangle meets the band, copies their
// 3 + 3K coefficients from the owner rank with coalesced loads (all issued
// before any is used) into shared memory, and each lane then evaluates its
// own colour with the same SH code as k_project_forward.
constexpr int kColorCoefs = 48;  // 3 DC + 45 rest for SH degree 3
__global__ void __launch_bounds__(256) k_project_color_peers(ProjFwdArgs a) {
    __shared__ float scoef[8][32][kColorCoefs];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int wbase = i - lane;
    bool need = false;
    if (i < a.n && a.radii[i] > 0) {
        const uint2 rc = a.rects[i];
        need = a.color_row1 <= a.color_row0 ||
               ((int)(rc.y >> 16) > a.color_row0 && (int)(rc.x >> 16) < a.color_row1);
    }
    const unsigned sel = __ballot_sync(0xffffffffu, need);
    if (sel == 0) return;
    const int K3 = 3 * a.rest_bases;
    const int ncoef = 3 + K3;
    for (unsigned bits = sel; bits; bits &= bits - 1) {
        const int j = __ffs(bits) - 1;
        const int g = wbase + j;
        const int q = g / a.peer_chunk;
        const float* dc = a.peer_dc[q] + 3 * (size_t)g;
        const float* rest = a.peer_rest[q] + (size_t)K3 * g;
        for (int k = lane; k < ncoef; k += 32) scoef[warp][j][k] = k < 3 ? dc[k] : rest[k - 3];
    }
    __syncwarp();
    if (!need) return;
    const float* mine = scoef[warp][lane];
    const CameraDev& cam = a.cam;
    V3 p = v3(a.means[3 * i], a.means[3 * i + 1], a.means[3 * i + 2]);
    V3 v = v3(p.x - cam.cam_pos[0], p.y - cam.cam_pos[1], p.z - cam.cam_pos[2]);
    float inv = 1.0f / sqrtf(dot3(v, v));
    V3 dir = scale3(v, inv);
    float col[3];
    sh_to_color(a.degrees_to_use, dir, mine, [&](int k) { return mine[3 + k]; }, col);
    float* r3 = reinterpret_cast<float*>(a.records + (size_t)i * kRecordF4 + 3);
    for (int c = 0; c < 3; ++c) r3[c] = smax(col[c] + 0.5f, 0.0f);
    if (a.colors)
        for (int c = 0; c < 3; ++c) a.colors[3 * i + c] = col[c];
}

// Colours of an owner's slice for the next step's camera (multi-GPU): the
// same evaluation as the forward's colour pass, for every Gaussian of the
// slice (culled ones included; the forward copies only what it needs).
__global__ void __launch_bounds__(256) k_shard_colors(ProjFwdArgs a, int g0, int g1, float* __restrict__ rgb_out) {
    const int i = g0 + blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= g1) return;
    const ParamPtrs pp = param_ptrs(a, i);
    float col[3], rgb[3];
    gaussian_color(a, pp, i, v3(pp.means[3 * i], pp.means[3 * i + 1], pp.means[3 * i + 2]), col, rgb);
    rgb_out[3 * i] = rgb[0];
    rgb_out[3 * i + 1] = rgb[1];
    rgb_out[3 * i + 2] = rgb[2];
}

}  // namespace

void launch_shard_colors(const ProjFwdArgs& a, int g0, int g1, float* rgb_out, cudaStream_t s) {
    if (g1 <= g0) return;
    note_launches(1);
    k_shard_colors<<<(g1 - g0 + 255) / 256, 256, 0, s>>>(a, g0, g1, rgb_out);
}

void launch_project_forward(const ProjFwdArgs& a, cudaStream_t s) {
    if (a.n <= 0) return;
    note_launches(1);
    if (a.pass == 2 && a.peer_world > 1)
        k_project_color_peers<<<(a.n + 255) / 256, 256, 0, s>>>(a);
    else {
        const size_t smem = stage_rest(a) ? (size_t)256 * 3 * a.rest_bases * sizeof(float) : 0;
        if (smem > 48 * 1024)
            (void)cudaFuncSetAttribute(k_project_forward, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k_project_forward<<<(a.n + 255) / 256, 256, smem, s>>>(a);
    }
}

}  // namespace msplat
