// Fused AngMF propagate for sm_100a.
//
// Replaces the reference's angmf_kernel (src/dsine_ops.cu:76-155, one thread
// per pixel, fp64 math, 25 uncached gathers of the neighbour normals) with:
//
//  * a CTA tile of 16 x 32 output pixels whose replicate-padded halo of source
//    normals ((16+2R) x (32+2R), R = (ps/2)*dil) is staged once in shared
//    memory, already unit-length (and, for the first iteration of the fused
//    refine, already RayReLU'd: the initial ray_relu of
//    src/dsine_refine.cpp:241-242 costs no extra pass);
//  * per-neighbour streams (prob, xy pair, angle) read exactly once, in
//    coalesced pixel pairs, evict-first;
//  * fp32 arithmetic carried two pixels at a time in packed f32x2 form, using
//    a closed form of the reference's per-neighbour geometry (below) that
//    needs no division, no fp64 and no transcendental beyond three rsqrt;
//  * an exact fp64 fix-up, identical in arithmetic to the reference
//    (src/dsine_ops.cpp:110-162), for the rare neighbours whose fp32
//    evaluation would be ill-conditioned or out of range.
//
// Closed form. With source ray P = (tu0, tv0, 1), tu0 = (sx+0.5-cu)/fu,
// tv0 = (sy+0.5-cv)/fv, unit xy offset (xs, ys), d = (xs/fu, ys/fv, 0), and
// unit source normal n, the reference builds
//     dd = (P + d).n,  dz = -(d.n)/dd,  a = d + dz (P + d),
// so a.n = 0 and dd a = n x (d x P) (vector triple product). Writing
// g = d x P and g_perp = g - n (n.g), the rotation about unit(a) by theta is
//     R n = cos(theta) n + sign(dd) sin(theta) g_perp / |g_perp|
// (Rodrigues with the axis orthogonal to n). g is scale-free here, so the raw
// xy pair can be used for it: g ~ (ys/fv, -xs/fu, xs tv0/fu - ys tu0/fv);
// only dd needs the normalised pair (one rsqrt). The quaternion route of
// axis_angle_to_matrix (src/dsine_ops.cpp:31-51) computes the same rotation.
// sin and cos come from the half-angle Taylor series (6 terms each, error
// < 1e-8 on |theta| <= pi), not from library code.
//
// Fix-up criteria (per pixel, per neighbour), each a place where the fp32
// evaluation can leave the reference's fp64 result by more than ~1e-6:
//  * |dd| < 1e-5: the sign of dd (which flips the rotation) may be wrong in
//    fp32, and the reference clamps |dd| < 1e-8;
//  * w |sin(theta)| |g| > 10 |g_perp|: g nearly parallel to n, so the rotation
//    direction comes from a cancellation; its fp32 error (~2e-7 |g|/|g_perp|)
//    is only tolerable while the neighbour's weighted sine is small;
//  * |m|^2 < 1e-2 after the RayReLU: the rotated normal points almost straight
//    away from the camera and the clamped vector is a cancellation too;
//  * |xy|^2 outside [1e-10, 1e30] (the reference's 1e-12 clamp on |xy|, or
//    fp32 overflow), |theta| > 3.2 (outside the series' range), or any NaN.
// Such neighbours are dropped from the fast sum, recorded in a bit mask and
// recomputed after the loop in fp64 exactly as the reference does. On
// camera-facing inputs this is about 1 neighbour evaluation in 10^5.
#include "bvml_common.cuh"
#include "bvml_internal.h"

#include <type_traits>

namespace bvml {
namespace {

constexpr int kTW = 32;         // tile width (16 pixel pairs)
constexpr int kTH = 16;         // tile height
constexpr int kThreads = 256;   // one pixel pair per thread

struct AngmfArgs {
    int B, H, W, dil, R, tiles_x, tiles_y;
    long HW;
    float ifu, ifv, tu_c, tv_c;   // 1/fu, 1/fv, (0.5-cu)/fu, (0.5-cv)/fv
    double fu, cu, fv, cv;        // exact values for the fp64 fix-up
};

// RayReLU of one normal in fp32 (src/dsine_ops.cpp:55-76 semantics).
__device__ __forceinline__ void ray_relu_f32(float& nx, float& ny, float& nz, float rx, float ry,
                                             float rz) {
    const float nn2 = fmaf(nx, nx, fmaf(ny, ny, nz * nz));
    const float rr2 = fmaf(rx, rx, fmaf(ry, ry, rz * rz));
    const float c = fmaf(nx, rx, fmaf(ny, ry, nz * rz)) * rsqrtf(fmaxf(nn2 * rr2, 1e-16f));
    const float dc = fmaxf(kRayEps - c, 0.0f);
    nx = fmaf(rx, dc, nx);
    ny = fmaf(ry, dc, ny);
    nz = fmaf(rz, dc, nz);
    const float inv = rsqrtf(fmaxf(fmaf(nx, nx, fmaf(ny, ny, nz * nz)), 1e-24f));
    nx *= inv;
    ny *= inv;
    nz *= inv;
}

__device__ __forceinline__ double dmax(double a, double b) { return (a < b) ? b : a; }

// Products and sums in the fp64 code below go through __dmul_rn / __dadd_rn so
// that no contracted fused multiply-add changes their rounding relative to the
// CPU twin (which is compiled without contraction).
__device__ __forceinline__ double dot3(double a0, double a1, double a2, double b0, double b1,
                                       double b2) {
    return __dadd_rn(__dadd_rn(__dmul_rn(a0, b0), __dmul_rn(a1, b1)), __dmul_rn(a2, b2));
}

// RayReLU in fp64 with the CPU twin's arithmetic (src/dsine_ops.cpp:59-75),
// rounded to float like the reference's stored pred_norm.
__device__ void ray_relu_exact(double& nx, double& ny, double& nz, double rx, double ry,
                               double rz) {
    const double nn = sqrt(dot3(nx, ny, nz, nx, ny, nz));
    const double rr = sqrt(dot3(rx, ry, rz, rx, ry, rz));
    const double denom = dmax(__dmul_rn(nn, rr), 1e-8);
    const double cs = dot3(nx, ny, nz, rx, ry, rz) / denom;
    const double eps = (double)kRayEps;
    const double dcoef = (dmax(cs - eps, 0.0) + eps) - cs;
    const double m0 = __dadd_rn(nx, __dmul_rn(rx, dcoef));
    const double m1 = __dadd_rn(ny, __dmul_rn(ry, dcoef));
    const double m2 = __dadd_rn(nz, __dmul_rn(rz, dcoef));
    const double inv = 1.0 / dmax(sqrt(dot3(m0, m1, m2, m0, m1, m2)), 1e-12);
    nx = (double)(float)__dmul_rn(m0, inv);
    ny = (double)(float)__dmul_rn(m1, inv);
    nz = (double)(float)__dmul_rn(m2, inv);
}

// One neighbour's weighted contribution in fp64, operation for operation as
// src/dsine_ops.cpp:104-162 (the fix-up path; see the file header).
__device__ __noinline__ double3 angmf_neighbor_exact(double nx, double ny, double nz, int sx,
                                                     int sy, double xs, double ys, double theta,
                                                     double w, double rx, double ry, double rz,
                                                     double fu, double cu, double fv,
                                                     double cv) {
    const double pix_x = sx + 0.5, pix_y = sy + 0.5;
    const double xyinv = 1.0 / dmax(sqrt(__dadd_rn(__dmul_rn(xs, xs), __dmul_rn(ys, ys))), 1e-12);
    xs = __dmul_rn(xs, xyinv);
    ys = __dmul_rn(ys, xyinv);
    const double du = xs / fu;
    const double dv = ys / fv;
    const double tu = (pix_x + xs - cu) / fu;
    const double tv = (pix_y + ys - cv) / fv;
    const double num = -__dadd_rn(__dmul_rn(du, nx), __dmul_rn(dv, ny));
    double dd = __dadd_rn(__dadd_rn(__dmul_rn(tu, nx), __dmul_rn(tv, ny)), nz);
    if (fabs(dd) < 1e-8) {
        const double sgn = (dd > 0.0) ? 1.0 : (dd < 0.0 ? -1.0 : 0.0);
        dd = 1e-8 * sgn;
    }
    const double dz = num / dd;
    double ax = __dadd_rn(du, __dmul_rn(dz, tu));
    double ay = __dadd_rn(dv, __dmul_rn(dz, tv));
    double az = dz;
    const double an =
        sqrt(__dadd_rn(__dadd_rn(__dmul_rn(ax, ax), __dmul_rn(ay, ay)), __dmul_rn(az, az)));
    const double ainv = 1.0 / dmax(an, 1e-12);
    ax = __dmul_rn(ax, ainv);
    ay = __dmul_rn(ay, ainv);
    az = __dmul_rn(az, ainv);
    if (!isfinite(ax) || !isfinite(ay) || !isfinite(az)) ax = ay = az = 0.0;
    // axis_angle_to_matrix on axis * theta (quaternion route).
    const double vx = __dmul_rn(ax, theta), vy = __dmul_rn(ay, theta), vz = __dmul_rn(az, theta);
    const double ang =
        sqrt(__dadd_rn(__dadd_rn(__dmul_rn(vx, vx), __dmul_rn(vy, vy)), __dmul_rn(vz, vz)));
    const double half = ang * 0.5;
    double s;
    if (ang < 1e-6)
        s = 0.5 - __dmul_rn(ang, ang) / 48.0;
    else
        s = sin(half) / ang;
    const double qr = cos(half);
    const double qi = __dmul_rn(vx, s), qj = __dmul_rn(vy, s), qk = __dmul_rn(vz, s);
    const double two_s =
        2.0 / __dadd_rn(__dadd_rn(__dadd_rn(__dmul_rn(qr, qr), __dmul_rn(qi, qi)),
                                  __dmul_rn(qj, qj)),
                        __dmul_rn(qk, qk));
    const double ii = __dmul_rn(qi, qi), jj = __dmul_rn(qj, qj), kk = __dmul_rn(qk, qk);
    const double ij = __dmul_rn(qi, qj), ik = __dmul_rn(qi, qk), jk = __dmul_rn(qj, qk);
    const double ir = __dmul_rn(qi, qr), jr = __dmul_rn(qj, qr), kr = __dmul_rn(qk, qr);
    const double R0 = 1.0 - __dmul_rn(two_s, __dadd_rn(jj, kk));
    const double R1 = __dmul_rn(two_s, ij - kr);
    const double R2 = __dmul_rn(two_s, __dadd_rn(ik, jr));
    const double R3 = __dmul_rn(two_s, __dadd_rn(ij, kr));
    const double R4 = 1.0 - __dmul_rn(two_s, __dadd_rn(ii, kk));
    const double R5 = __dmul_rn(two_s, jk - ir);
    const double R6 = __dmul_rn(two_s, ik - jr);
    const double R7 = __dmul_rn(two_s, __dadd_rn(jk, ir));
    const double R8 = 1.0 - __dmul_rn(two_s, __dadd_rn(ii, jj));
    double qx = __dadd_rn(__dadd_rn(__dmul_rn(R0, nx), __dmul_rn(R1, ny)), __dmul_rn(R2, nz));
    double qy = __dadd_rn(__dadd_rn(__dmul_rn(R3, nx), __dmul_rn(R4, ny)), __dmul_rn(R5, nz));
    double qz = __dadd_rn(__dadd_rn(__dmul_rn(R6, nx), __dmul_rn(R7, ny)), __dmul_rn(R8, nz));
    const double rinv = 1.0 / dmax(sqrt(__dadd_rn(__dadd_rn(__dmul_rn(qx, qx), __dmul_rn(qy, qy)),
                                                  __dmul_rn(qz, qz))),
                                   1e-12);
    qx = __dmul_rn(qx, rinv);
    qy = __dmul_rn(qy, rinv);
    qz = __dmul_rn(qz, rinv);
    const double nn =
        sqrt(__dadd_rn(__dadd_rn(__dmul_rn(qx, qx), __dmul_rn(qy, qy)), __dmul_rn(qz, qz)));
    const double rr =
        sqrt(__dadd_rn(__dadd_rn(__dmul_rn(rx, rx), __dmul_rn(ry, ry)), __dmul_rn(rz, rz)));
    const double denom = dmax(__dmul_rn(nn, rr), 1e-8);
    const double cs =
        __dadd_rn(__dadd_rn(__dmul_rn(qx, rx), __dmul_rn(qy, ry)), __dmul_rn(qz, rz)) / denom;
    const double eps = (double)kRayEps;
    const double dcoef = (dmax(cs - eps, 0.0) + eps) - cs;
    double m0 = __dadd_rn(qx, __dmul_rn(rx, dcoef));
    double m1 = __dadd_rn(qy, __dmul_rn(ry, dcoef));
    double m2 = __dadd_rn(qz, __dmul_rn(rz, dcoef));
    const double minv = 1.0 / dmax(sqrt(__dadd_rn(__dadd_rn(__dmul_rn(m0, m0), __dmul_rn(m1, m1)),
                                                  __dmul_rn(m2, m2))),
                                   1e-12);
    return make_double3(__dmul_rn(w, __dmul_rn(m0, minv)), __dmul_rn(w, __dmul_rn(m1, minv)),
                        __dmul_rn(w, __dmul_rn(m2, minv)));
}

// Half-angle Taylor coefficients: 2 sin(t/2) = t * sum_k (-1)^k t^2k / (4^k (2k+1)!),
// cos(t/2) = sum_k (-1)^k t^2k / (4^k (2k)!).
constexpr float kS1 = -1.0f / 24.0f, kS2 = 1.0f / 1920.0f, kS3 = -1.0f / 322560.0f,
                kS4 = 1.0f / 92897280.0f, kS5 = -1.0f / 40874803200.0f,
                kS6 = 1.0f / 25505877196800.0f;
constexpr float kC1 = -1.0f / 8.0f, kC2 = 1.0f / 384.0f, kC3 = -1.0f / 46080.0f,
                kC4 = 1.0f / 10321920.0f, kC5 = -1.0f / 3715891200.0f,
                kC6 = 1.0f / 1961990553600.0f;

constexpr float kTau = 1e-5f;     // |dd| fix-up threshold
constexpr float kGCond = 0.1f;    // 1 / (largest tolerated w |sin| |g| / |g_perp|)
constexpr float kMMin = 1e-2f;    // smallest tolerated |m|^2 after the RayReLU
constexpr float kQMin = 1e-10f, kQMax = 1e30f;  // |xy|^2 range of the fast path
constexpr float kThMax = 3.2f;    // |theta| range of the series

template <int PS, typename TS, typename TNI, typename TNO, bool FUSE_RR>
__global__ void __launch_bounds__(kThreads, 2)
angmf_kernel(const TNI* __restrict__ pn, const TS* __restrict__ prob, const TS* __restrict__ xy,
             const TS* __restrict__ ang, const float* __restrict__ ray, TNO* __restrict__ out,
             const AngmfArgs a) {
    constexpr int P = PS * PS;
    using Mask = typename std::conditional<(P <= 32), uint32_t, unsigned long long>::type;
    extern __shared__ float4 smem4[];
    const int R = a.R;
    const int SW = kTW + 2 * R;
    const int SH = kTH + 2 * R;
    float2* snx = reinterpret_cast<float2*>(smem4);   // [SH][SW] pair-duplicated planes:
    float2* sny = snx + SH * SW;                      // element (i,j) = (v[i][j], v[i][j+1])
    float2* snz = sny + SH * SW;
    float2* stu = snz + SH * SW;                      // [SW] pairs of tu0
    float* stv = reinterpret_cast<float*>(stu + SW);  // [SH] tv0

    int t = blockIdx.x;
    const int tix = t % a.tiles_x;
    t /= a.tiles_x;
    const int tiy = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int x0 = tix * kTW, y0 = tiy * kTH;
    const long HW = a.HW;
    const TNI* pnb = pn + (long)b * 3 * HW;

    // ---- stage the replicate-padded halo of unit source normals
    for (int idx = threadIdx.x; idx < SH * SW; idx += kThreads) {
        const int i = idx / SW, j = idx - i * SW;
        const int sy = clampi(y0 - R + i, 0, a.H - 1);
        const int sx = clampi(x0 - R + j, 0, a.W - 1);
        const long sp = (long)sy * a.W + sx;
        float nx = St<TNI>::ld(pnb + sp), ny = St<TNI>::ld(pnb + HW + sp),
              nz = St<TNI>::ld(pnb + 2 * HW + sp);
        if (FUSE_RR) ray_relu_f32(nx, ny, nz, __ldg(ray + sp), __ldg(ray + HW + sp),
                                  __ldg(ray + 2 * HW + sp));
        const float inv = rsqrtf(fmaxf(fmaf(nx, nx, fmaf(ny, ny, nz * nz)), 1e-24f));
        float* fx = reinterpret_cast<float*>(snx);
        float* fy = reinterpret_cast<float*>(sny);
        float* fz = reinterpret_cast<float*>(snz);
        const int e = 2 * (i * SW + j);
        fx[e] = nx * inv;
        fy[e] = ny * inv;
        fz[e] = nz * inv;
        if (j > 0) {
            fx[e - 1] = nx * inv;
            fy[e - 1] = ny * inv;
            fz[e - 1] = nz * inv;
        }
    }
    for (int j = threadIdx.x; j < SW; j += kThreads) {
        const int s0 = clampi(x0 - R + j, 0, a.W - 1);
        const int s1 = clampi(x0 - R + j + 1, 0, a.W - 1);
        stu[j] = make_float2(fmaf((float)s0, a.ifu, a.tu_c), fmaf((float)s1, a.ifu, a.tu_c));
    }
    for (int i = threadIdx.x; i < SH; i += kThreads) {
        const int s0 = clampi(y0 - R + i, 0, a.H - 1);
        stv[i] = fmaf((float)s0, a.ifv, a.tv_c);
    }
    __syncthreads();

    // ---- one pixel pair per thread
    const int lx = 2 * (threadIdx.x % (kTW / 2));
    const int ly = threadIdx.x / (kTW / 2);
    const int x = x0 + lx, y = y0 + ly;
    if (y >= a.H || x >= a.W) return;
    const bool two = x + 1 < a.W;
    const bool vec = (a.W & 1) == 0;  // pairs start at even offsets -> 8/4-byte aligned
    const long p0 = (long)y * a.W + x;
    const long p1 = two ? p0 + 1 : p0;

    float2 rx = f2(__ldg(ray + p0), __ldg(ray + p1));
    float2 ry = f2(__ldg(ray + HW + p0), __ldg(ray + HW + p1));
    float2 rz = f2(__ldg(ray + 2 * HW + p0), __ldg(ray + 2 * HW + p1));
    {
        const float2 ri = rsqrt2(max2(fma2(rx, rx, fma2(ry, ry, mul2(rz, rz))), f2(1e-16f)));
        rx = mul2(rx, ri);
        ry = mul2(ry, ri);
        rz = mul2(rz, ri);
    }

    const TS* xyb = xy + (long)b * 2 * P * HW;
    const TS* prb = prob + (long)b * P * HW;
    const TS* anb = ang + (long)b * P * HW;
    auto ld = [&](const TS* base) -> float2 {
        return vec ? St<TS>::ld2s(base + p0) : f2(St<TS>::lds1(base + p0), St<TS>::lds1(base + p1));
    };

    const float2 ifu2 = f2(a.ifu), ifv2 = f2(a.ifv);
    float2 accx = f2(0.f), accy = f2(0.f), accz = f2(0.f);
    Mask bad0 = 0, bad1 = 0;

#pragma unroll 1
    for (int ky = 0; ky < PS; ++ky) {
        const int i = ly + ky * a.dil;
        const float2 tv = f2(stv[i]);
        const float2* rnx = snx + i * SW + lx;
        const float2* rny = sny + i * SW + lx;
        const float2* rnz = snz + i * SW + lx;
        const float2* rtu = stu + lx;
#pragma unroll
        for (int kx = 0; kx < PS; ++kx) {
            const int n = ky * PS + kx;
            const int j = kx * a.dil;
            const float2 nx = rnx[j], ny = rny[j], nz = rnz[j], tu = rtu[j];
            const float2 xs = ld(xyb + (long)n * HW);
            const float2 ys = ld(xyb + (long)(P + n) * HW);
            const float2 th = ld(anb + (long)n * HW);
            float2 wt = ld(prb + (long)n * HW);

            const float2 q = fma2(xs, xs, mul2(ys, ys));
            const float2 iq = rsqrt2(q);
            const float2 xsf = mul2(xs, ifu2);
            const float2 ysf = mul2(ys, ifv2);
            const float2 e = fma2(xsf, nx, mul2(ysf, ny));
            const float2 as = fma2(tu, nx, fma2(tv, ny, nz));
            const float2 dd = fma2(iq, e, as);
            // g = (ysf, -xsf, gz); carry gy' = -g_perp.y to avoid negations
            const float2 gz = fnma2(ysf, tu, mul2(xsf, tv));
            const float2 ng = fma2(gz, nz, fnma2(xsf, ny, mul2(ysf, nx)));
            const float2 gpx = fnma2(nx, ng, ysf);
            const float2 gpyn = fma2(ny, ng, xsf);
            const float2 gpz = fnma2(nz, ng, gz);
            const float2 gp2 = fma2(gpx, gpx, fma2(gpyn, gpyn, mul2(gpz, gpz)));
            const float2 gg2 = fma2(ysf, ysf, fma2(xsf, xsf, mul2(gz, gz)));
            const float2 gi = rsqrt2(max2(gp2, f2(1e-30f)));
            // sin / cos of theta via the half angle
            const float2 t2 = mul2(th, th);
            float2 ps2 = fma2(t2, f2(kS6), f2(kS5));
            ps2 = fma2(t2, ps2, f2(kS4));
            ps2 = fma2(t2, ps2, f2(kS3));
            ps2 = fma2(t2, ps2, f2(kS2));
            ps2 = fma2(t2, ps2, f2(kS1));
            ps2 = fma2(t2, ps2, f2(1.0f));
            const float2 s2 = mul2(th, ps2);  // 2 sin(theta/2)
            float2 ch = fma2(t2, f2(kC6), f2(kC5));
            ch = fma2(t2, ch, f2(kC4));
            ch = fma2(t2, ch, f2(kC3));
            ch = fma2(t2, ch, f2(kC2));
            ch = fma2(t2, ch, f2(kC1));
            ch = fma2(t2, ch, f2(1.0f));      // cos(theta/2)
            const float2 sn = mul2(s2, ch);   // sin(theta)
            const float2 cs = fnma2(mul2(s2, f2(0.5f)), s2, f2(1.0f));  // cos(theta)
            float2 kk = mul2(sn, gi);
            kk.x = __uint_as_float(__float_as_uint(kk.x) ^ (__float_as_uint(dd.x) & 0x80000000u));
            kk.y = __uint_as_float(__float_as_uint(kk.y) ^ (__float_as_uint(dd.y) & 0x80000000u));
            const float2 qx = fma2(kk, gpx, mul2(cs, nx));
            const float2 qy = fnma2(kk, gpyn, mul2(cs, ny));
            const float2 qz = fma2(kk, gpz, mul2(cs, nz));
            // RayReLU against this pixel's ray, then the weighted sum
            const float2 c = fma2(qx, rx, fma2(qy, ry, mul2(qz, rz)));
            const float2 dc = max2(fnma2(c, f2(1.0f), f2(kRayEps)), f2(0.0f));
            const float2 mx = fma2(rx, dc, qx);
            const float2 my = fma2(ry, dc, qy);
            const float2 mz = fma2(rz, dc, qz);
            const float2 l2 = fma2(mx, mx, fma2(my, my, mul2(mz, mz)));
            const float2 wsg = mul2(mul2(wt, f2(kGCond)), sn);
            const float2 gcond = mul2(mul2(wsg, wsg), gg2);
            const bool b0 = !(fabsf(dd.x) >= kTau) || !(gp2.x >= gcond.x) || !(l2.x >= kMMin) ||
                            !(q.x >= kQMin) || !(q.x <= kQMax) || !(fabsf(th.x) <= kThMax);
            const bool b1 = !(fabsf(dd.y) >= kTau) || !(gp2.y >= gcond.y) || !(l2.y >= kMMin) ||
                            !(q.y >= kQMin) || !(q.y <= kQMax) || !(fabsf(th.y) <= kThMax);
            if (b0) { wt.x = 0.0f; bad0 |= Mask(1) << n; }
            if (b1) { wt.y = 0.0f; bad1 |= Mask(1) << n; }
            const float2 wm = mul2(wt, rsqrt2(l2));
            accx = fma2(wm, mx, accx);
            accy = fma2(wm, my, accy);
            accz = fma2(wm, mz, accz);
        }
    }

    // ---- rare exact fix-ups
    if ((bad0 | bad1) != 0) {
        const TNI* pnx = pnb;
#pragma unroll 1
        for (int e = 0; e < 2; ++e) {
            Mask m = e == 0 ? bad0 : bad1;
            if (e == 1 && !two) m = 0;
            const long pp = e == 0 ? p0 : p1;
            const int xx = x + e;
            const double orx = __ldg(ray + pp), ory = __ldg(ray + HW + pp),
                         orz = __ldg(ray + 2 * HW + pp);
            double ax = 0.0, ay = 0.0, az = 0.0;
            while (m != 0) {
                int n;
                if constexpr (sizeof(Mask) == 4) n = __ffs(m) - 1;
                else n = __ffsll((long long)m) - 1;
                m &= m - 1;
                const int ky = n / PS, kx = n - (n / PS) * PS;
                const int sy = clampi(y - R + ky * a.dil, 0, a.H - 1);
                const int sx = clampi(xx - R + kx * a.dil, 0, a.W - 1);
                const long sp = (long)sy * a.W + sx;
                double nx = St<TNI>::ld(pnx + sp), ny = St<TNI>::ld(pnx + HW + sp),
                       nz = St<TNI>::ld(pnx + 2 * HW + sp);
                if (FUSE_RR)
                    ray_relu_exact(nx, ny, nz, __ldg(ray + sp), __ldg(ray + HW + sp),
                                   __ldg(ray + 2 * HW + sp));
                const double3 c3 = angmf_neighbor_exact(
                    nx, ny, nz, sx, sy, St<TS>::ld(xyb + (long)n * HW + pp),
                    St<TS>::ld(xyb + (long)(P + n) * HW + pp), St<TS>::ld(anb + (long)n * HW + pp),
                    St<TS>::ld(prb + (long)n * HW + pp), orx, ory, orz, a.fu, a.cu, a.fv, a.cv);
                ax += c3.x;
                ay += c3.y;
                az += c3.z;
            }
            if (e == 0) {
                accx.x += (float)ax;
                accy.x += (float)ay;
                accz.x += (float)az;
            } else {
                accx.y += (float)ax;
                accy.y += (float)ay;
                accz.y += (float)az;
            }
        }
    }

    // ---- normalise and store
    const float2 l = fma2(accx, accx, fma2(accy, accy, mul2(accz, accz)));
    const float2 inv = rsqrt2(max2(l, f2(1e-24f)));
    const float2 ox = mul2(accx, inv), oy = mul2(accy, inv), oz = mul2(accz, inv);
    TNO* ob = out + (long)b * 3 * HW;
    if (vec) {
        St<TNO>::st2(ob + p0, ox);
        St<TNO>::st2(ob + HW + p0, oy);
        St<TNO>::st2(ob + 2 * HW + p0, oz);
    } else {
        St<TNO>::st(ob + p0, ox.x);
        St<TNO>::st(ob + HW + p0, oy.x);
        St<TNO>::st(ob + 2 * HW + p0, oz.x);
        if (two) {
            St<TNO>::st(ob + p1, ox.y);
            St<TNO>::st(ob + HW + p1, oy.y);
            St<TNO>::st(ob + 2 * HW + p1, oz.y);
        }
    }
}

template <int PS, typename TS, typename TNI, typename TNO, bool FUSE_RR>
cudaError_t launch_t(const AngmfLaunch& L, cudaStream_t s) {
    AngmfArgs a;
    a.B = L.B;
    a.H = L.H;
    a.W = L.W;
    a.dil = L.dil;
    a.R = (PS / 2) * L.dil;
    a.tiles_x = (L.W + kTW - 1) / kTW;
    a.tiles_y = (L.H + kTH - 1) / kTH;
    a.HW = (long)L.H * L.W;
    a.ifu = (float)(1.0 / L.fu);
    a.ifv = (float)(1.0 / L.fv);
    a.tu_c = (float)((0.5 - L.cu) / L.fu);
    a.tv_c = (float)((0.5 - L.cv) / L.fv);
    a.fu = L.fu;
    a.cu = L.cu;
    a.fv = L.fv;
    a.cv = L.cv;
    const int SW = kTW + 2 * a.R, SH = kTH + 2 * a.R;
    const size_t smem = sizeof(float2) * (3 * (size_t)SH * SW + SW) + sizeof(float) * SH;
    auto kern = angmf_kernel<PS, TS, TNI, TNO, FUSE_RR>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    const long blocks = (long)a.tiles_x * a.tiles_y * L.B;
    if (blocks > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    kern<<<(unsigned)blocks, kThreads, smem, s>>>(
        static_cast<const TNI*>(L.pn), static_cast<const TS*>(L.prob),
        static_cast<const TS*>(L.xy), static_cast<const TS*>(L.angle), L.ray,
        static_cast<TNO*>(L.out), a);
    return cudaGetLastError();
}

template <int PS, typename TS>
cudaError_t launch_ps(const AngmfLaunch& L, cudaStream_t s) {
    const bool in_f32 = L.pn_t == SType::F32, out_f32 = L.out_t == SType::F32;
    using TO = TS;
    if (L.fuse_ray_relu) {
        // fused refine, first iteration: storage-typed decoder normals in, fp32 out
        if (!out_f32) return cudaErrorInvalidValue;
        if (in_f32) return launch_t<PS, TS, float, float, true>(L, s);
        return launch_t<PS, TS, TO, float, true>(L, s);
    }
    // fused refine, later iterations (fp32 intermediates) or the fp32 single op
    if (in_f32 && out_f32) return launch_t<PS, TS, float, float, false>(L, s);
    // single op on storage-typed normals
    if (!in_f32 && !out_f32) return launch_t<PS, TS, TO, TO, false>(L, s);
    return cudaErrorInvalidValue;
}

template <typename TS>
cudaError_t launch_st(const AngmfLaunch& L, cudaStream_t s) {
    switch (L.ps) {
        case 3: return launch_ps<3, TS>(L, s);
        case 5: return launch_ps<5, TS>(L, s);
        case 7: return launch_ps<7, TS>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_angmf(const AngmfLaunch& L, cudaStream_t s) {
    if (L.B == 0 || L.H == 0 || L.W == 0) return cudaSuccess;
    if (L.st == SType::F32) {
        if (L.pn_t != SType::F32 && !L.fuse_ray_relu) return cudaErrorInvalidValue;
        return launch_st<float>(L, s);
    }
    return launch_st<__half>(L, s);
}

}  // namespace bvml
