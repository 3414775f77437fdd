// common.cuh — device helpers shared by the msplat B200 kernels.
//
// The forward path (projection, binning keys, rasterisation) is evaluated with
// a fixed sequence of IEEE-rounded operations so that tile counts, per-tile
// order and the rendered image are reproducible bit for bit on any IEEE
// implementation that follows the same sequence. The helpers below pin that
// sequence: __fmul_rn/__fadd_rn/__fsub_rn are never contracted into an FMA by
// the compiler, __fmaf_rn is always one fused operation.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace msplat {

constexpr int kTile = 16;               // 16x16 pixel tiles (BLOCK_X/BLOCK_Y)
constexpr int kTilePixels = kTile * kTile;
constexpr int kMaxTileElems = 2048;     // per-tile intersection cap
constexpr float kFilterSize = 0.707106f;
constexpr float kFilterInvSq = 2.0f;
constexpr float kNearN = 0.2f;
constexpr float kFarN = 100.0f;

// Per-Gaussian raster record written by the projection and gathered by the
// rasterisers: 5 x float4 = 80 bytes.
//   r0 = (Tu.x, Tu.y, Tu.z, Tv.x)
//   r1 = (Tv.y, Tv.z, Tw.x, Tw.y)
//   r2 = (Tw.z, xy.x, xy.y, sigmoid(opacity))
//   r3 = (rgb.r, rgb.g, rgb.b, normal.x)   rgb = max(raw SH colour + 0.5, 0)
//   r4 = (normal.y, normal.z, rmax, 0)   rmax = reject_rho(sigmoid(opacity))
constexpr int kRecordF4 = 5;

// Per-Gaussian cull record written by the projection and read by the forward
// rasteriser to skip pixel blocks a surfel cannot reach: 2 x float4 = 32 bytes.
//   c0 = (centre.x, centre.y, s1, t1)
//   c1 = (s2, -E.xy / E.yy, -E.xy / E.xx, rd2)
// The pixels where rho3d <= rmax * kCullRhoScale form a conic; when it is an
// ellipse, d^T E d <= 1 inside it (d = pixel - centre), with E factored as
// d^T E d = (s1 d.x + t1 d.y)^2 + (s2 d.y)^2, a sum of squares that float
// arithmetic evaluates without cancellation however thin the ellipse.
// Otherwise (not an ellipse, or thinner than kCullMaxAspect) s1 = t1 = s2 = 0
// and every block passes. rd2 is the squared radius of the 2-D filter disc
// 2 d^2 <= rmax around xy, grown by the margin; -1 when the surfel never
// reaches alpha 1/255.
constexpr int kCullF4 = 2;
constexpr float kCullRhoScale = 1.002f;  // rmax growth covering float rounding of rho
constexpr float kCullMargin = 0.25f;     // pixel margin around each tested block
// Screen ellipses with an axis ratio above this come from surfels seen almost
// edge-on, where the rasteriser's own float rho3d loses relative accuracy;
// they are never culled.
constexpr double kCullMaxAspect = 1.0e4;

// Rho above which a surfel of opacity o is certainly skipped by the 1/255
// alpha cut: o * exp(-rho/2) < 1/255 for rho > 2 ln(255 o); the +0.01 margin
// covers the rounding of det_exp and of this bound. Negative for o < 1/255.
__device__ __forceinline__ float reject_rho(float opac) {
    return opac > 0.f ? 2.0f * logf(255.0f * opac) + 0.01f : -1.0f;
}

// Per-Gaussian raster-space gradient record accumulated by the backward
// rasteriser: 16 floats = 4 x float4.
//   [0..8]  dL/dT (rows Tu, Tv, Tw)   [9] dL/d(raw opacity)
//   [10..12] dL/d(raw SH colour)      [13..15] dL/d(world normal)
constexpr int kGradStride = 16;

// Work estimate of a tile row for band balancing across GPUs: kept
// intersections plus a per-tile cost in the same unit. Fitted to per-rank
// rasteriser + loss times of 8 ranks on the 4946x3286 benchmark scene
// (time ~ 0.33 ns per kept intersection + 144 ns per tile): per-pixel outputs
// and the loss cost the same for every tile, and sparse regions carry larger
// surfels that blend over more pixels per intersection.
constexpr int kRowWorkPerTile = 430;

// First row of band r of `world` contiguous bands of about equal work
// (rows are added while less than half of the next row's work overshoots).
__device__ inline int band_cut(const int64_t* work, int ty, double total, int r, int world) {
    if (r <= 0) return 0;
    if (r >= world) return ty;
    const double target = total * r / world;
    double run = 0;
    int y = 0;
    while (y < ty && run + (double)work[y] / 2 < target) run += (double)work[y++];
    return y;
}

// 16-byte asynchronous copy global -> shared (cp.async, cached in L1 and L2:
// the CTAs of neighbouring tiles on one SM share many records) and the wait
// for every copy the thread issued (commit + wait for the group). Both
// addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float ffma(float a, float b, float c) { return __fmaf_rn(a, b, c); }

// Deterministic exponential: Cody-Waite reduction x = k*ln2 + r with ln2 split
// into a 16-bit head (0.693145751953125) and a tail, degree-7 Taylor
// polynomial for exp(r) on |r| <= ln2/2 evaluated by Horner with fused
// multiply-adds, exact scaling by 2^k. Flushes to 0 below -86 and to +inf
// above 88. Relative error is a few ulp; what matters here is that the CPU
// checker evaluates the identical sequence.
__device__ __forceinline__ float det_exp(float x) {
    if (x != x) return x;
    if (x > 88.0f) return __int_as_float(0x7f800000);
    if (x < -86.0f) return 0.0f;
    // k = nearest integer (ties to even) of x log2(e): adding 1.5 * 2^23 puts
    // the value where the float spacing is 1, so the addition itself rounds
    // (|x log2 e| <= 127 here); k is read from the bits of the sum.
    const float shifted = __fadd_rn(__fmul_rn(x, 1.44269502f), 12582912.0f);
    const float kf = __fsub_rn(shifted, 12582912.0f);
    float r = __fmaf_rn(-kf, 0.693145751953125f, x);
    r = __fmaf_rn(-kf, 1.42860677e-06f, r);
    float p = 1.98412698e-04f;
    p = __fmaf_rn(p, r, 1.38888889e-03f);
    p = __fmaf_rn(p, r, 8.33333377e-03f);
    p = __fmaf_rn(p, r, 4.16666679e-02f);
    p = __fmaf_rn(p, r, 1.66666672e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int k = __float_as_int(shifted) - 0x4B400000;
    return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

// det_exp for arguments known to lie in [-86, 0] (or NaN): the same sequence
// without the range tests, so the results are identical there (a NaN
// propagates through the polynomial). The rasteriser's falloff exp(-rho/2)
// is used only for rho within the surfel's rejection bound (at most
// 2 ln 255 + 0.01 plus rounding), i.e. for arguments in [-5.6, 0]; lanes whose
// result is discarded may pass anything, so the exponent is assembled in
// unsigned arithmetic, defined for every input.
__device__ __forceinline__ float det_exp_nonpos(float x) {
    const float shifted = __fadd_rn(__fmul_rn(x, 1.44269502f), 12582912.0f);
    const float kf = __fsub_rn(shifted, 12582912.0f);
    float r = __fmaf_rn(-kf, 0.693145751953125f, x);
    r = __fmaf_rn(-kf, 1.42860677e-06f, r);
    float p = 1.98412698e-04f;
    p = __fmaf_rn(p, r, 1.38888889e-03f);
    p = __fmaf_rn(p, r, 8.33333377e-03f);
    p = __fmaf_rn(p, r, 4.16666679e-02f);
    p = __fmaf_rn(p, r, 1.66666672e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const unsigned k = __float_as_uint(shifted) - 0x4B400000u;
    return __fmul_rn(p, __uint_as_float((k + 127u) << 23));
}

// Device-side error word: kernels OR bits into it instead of trapping; the
// host reads it after the step.
enum : uint32_t {
    kErrTileOverflow = 1u << 0,   // a tile had more than 2048 intersections (informational)
    kErrCapacity = 1u << 1,       // an intersection buffer was too small: step invalid
    kErrNonFinite = 1u << 2,      // non-finite loss
};

}  // namespace msplat
