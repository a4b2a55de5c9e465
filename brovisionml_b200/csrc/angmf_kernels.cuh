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
//    needs no division and no fp64: three rsqrt and one sin / cos pair;
//  * an exact fp64 fix-up, identical in arithmetic to the reference
//    (src/dsine_ops.cpp:110-162), for the rare neighbours whose fp32
//    evaluation would be ill-conditioned or out of range;
//  * optionally (ACT) the prediction heads' activations applied on load, so
//    the caller can pass raw head outputs and skip the separate sigmoid /
//    scale passes of src/dsine_refine.cpp:262-267.
//
// The kernels are templates included by angmf.cu (activated inputs) and
// angmf_logits.cu (raw head outputs), two translation units built in parallel.
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
// sin and cos come from the hardware approximations (sin.approx / cos.approx,
// absolute error ~5e-7 on |theta| <= pi).
//
// Fix-up criteria (per pixel, per neighbour), each a place where the fp32
// evaluation can leave the reference's fp64 result by more than ~1e-6:
//  * |dd| < 1e-5: the sign of dd (which flips the rotation) may be wrong in
//    fp32, and the reference clamps |dd| < 1e-8;
//  * w |sin(theta)| |n.g| > 19.97 |g_perp|: g nearly parallel to n, so the
//    rotation direction comes from the cancellation g - n (n.g); its fp32
//    error (~2e-7 |n.g| / |g_perp|) is only tolerable while the neighbour's
//    weighted sine is small;
//  * |m|^2 < 0.04 after the RayReLU: the rotated normal points almost straight
//    away from the camera and the clamped vector is a cancellation too;
//  * |xy|^2 outside [1e-10, 1e30] (the reference's 1e-12 clamp on |xy|, or
//    fp32 overflow), |theta| > pi (outside the approximations' range), or any
//    NaN.
// The tests of one neighbour form a single predicate chain (unordered
// comparisons, so NaN flags); a flagged neighbour's weight is zeroed and its
// bit set in the pixel's mask, without a branch. After the loop, the flagged
// neighbours are recomputed in fp64 exactly as the reference does; a pixel
// whose fast sum came out non-finite (a flagged neighbour with an infinite or
// NaN vector) or vanishing is recomputed over its whole window. On
// camera-facing inputs about 1 neighbour evaluation in 10^5 is flagged.
#pragma once

#include "bvml_common.cuh"
#include "bvml_internal.h"

#include <type_traits>

namespace bvml {
namespace {

constexpr int kTW = 32;         // tile width (16 pixel pairs)
constexpr int kTH = 16;         // tile height
// (angmf_iters_sync_bytes in bvml_internal.h counts tiles of this size)
static_assert(kTW == 32 && kTH == 16, "sync-word count assumes 32 x 16 tiles");
constexpr int kThreads = 256;   // one pixel pair per thread

struct AngmfArgs {
    int B, H, W, dil, R, tiles_x, tiles_y;
    long HW;
    float2 ifu2, ifv2;            // (1/fu, 1/fu), (1/fv, 1/fv): packed operands read from
                                  // the kernel's parameter bank, not held in registers
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

// Head activations of Refiner::forward (src/dsine_refine.cpp:262-267),
// applied on load when the kernel is given the heads' raw outputs (ACT):
// prob = sigmoid(prob_logit), angle = kPi * sigmoid(angle_logit), with kPi
// the reference's float constant (src/dsine_refine.cpp:26). Fast path:
// sigmoid(v) = 1 / (1 + 2^(-v log2 e)) with the hardware ex2 / rcp
// approximations (relative error a few 1e-7). The weight is handed on as
// its denominator d = 1 + e^-v (w = 1/d): angmf_pair folds 1/d into the
// rsqrt it takes anyway, so only the angle needs a reciprocal.
constexpr float kPiF = 3.14159265358979323846f;
__device__ __forceinline__ float2 sigmoid2_den(float2 v) {
    return add2(ex2_ftz2(mul2(v, f2(-1.4426950408889634f))), f2(1.0f));
}
__device__ __forceinline__ void head_activation(float2& wden, float2& th) {
    wden = sigmoid2_den(wden);
    th = mul2(rcp2_ftz(sigmoid2_den(th)), f2(kPiF));
}
// The same for the fix-up path: sigmoid in fp64 rounded to float (the fp32
// tensors the reference's activations produce), then the fp32 product by kPi.
__device__ __forceinline__ void head_activation_exact(double& w, double& th) {
    w = (double)(float)(1.0 / (1.0 + exp(-w)));
    th = (double)((float)(1.0 / (1.0 + exp(-th))) * kPiF);
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

constexpr float kTau = 1e-5f;     // |dd| fix-up threshold
constexpr float kTMax = 19.97f;   // largest tolerated w |sin| |n.g| / |g_perp|
constexpr float kMMin = 0.04f;    // smallest tolerated |m|^2 after the RayReLU
constexpr float kQMin = 1e-10f, kQMax = 1e30f;  // |xy|^2 range of the fast path
constexpr float kThMax = 3.1416f; // |theta| range of the sin / cos approximations

template <int PS> struct P_OF { static constexpr int value = PS * PS; };

template <typename Mask>
struct PairAcc {
    float2 x, y, z;   // prob-weighted sums of the rotated neighbours (before the RayReLU)
    float2 d;         // prob-weighted sum of the RayReLU coefficients dc
    Mask bad0, bad1;  // neighbours left to the exact fix-up, per pixel of the pair
};

// The RayReLU of neighbour k adds dc_k r to its rotated normal q_k, and r is
// the output pixel's own ray, the same for every neighbour, so
// sum_k w_k (q_k + dc_k r) = sum_k w_k q_k + (sum_k w_k dc_k) r: the loop
// accumulates the two sums and this adds the second once per pixel.
template <typename Mask>
__device__ __forceinline__ void fold_ray(PairAcc<Mask>& A, float2 rx, float2 ry, float2 rz) {
    A.x = fma2(A.d, rx, A.x);
    A.y = fma2(A.d, ry, A.y);
    A.z = fma2(A.d, rz, A.z);
}

// Flag one pixel's evaluation of neighbour slot `bit` for the exact fix-up:
// when |dd| < kTau, |t| > tlim, l2 < kMMin or |th| > kThMax (unordered: any
// NaN flags), plus |xy|^2 = q outside [kQMin, kQMax] (QRANGE) and lw > 3.4e38
// (WDEN), zero the weight wm and OR `bit` into the mask. One predicate chain
// of comparisons and two predicated moves; the immediates are kTau, kMMin,
// kThMax, kQMin, kQMax and 3.4e38 as fp32 bit patterns.
#define BVML_FLAG_CORE                                                      \
    "setp.ltu.f32 p, %2, 0f3727C5AC;\n\t"       /* |dd| < 1e-5   */          \
    "setp.gtu.or.f32 p, %3, %4, p;\n\t"         /* |t| > tlim    */          \
    "setp.ltu.or.f32 p, %5, 0f3D23D70A, p;\n\t" /* l2 < 0.04     */          \
    "setp.gtu.or.f32 p, %6, 0f40490FF9, p;\n\t" /* |th| > 3.1416 */
#define BVML_FLAG_Q(i)                                                      \
    "setp.ltu.or.f32 p, %" #i ", 0f2EDBE6FF, p;\n\t" /* q < 1e-10 */         \
    "setp.gtu.or.f32 p, %" #i ", 0f7149F2CA, p;\n\t" /* q > 1e30  */
#define BVML_FLAG_W(i) "setp.gtu.or.f32 p, %" #i ", 0f7F7FC99E, p;\n\t" /* lw > 3.4e38 */
#define BVML_FLAG_TAIL(op) "@p mov.f32 %0, 0f00000000;\n\t@p " op " %1, %1, %7;\n\t}"

template <bool QRANGE, bool WDEN>
__device__ __forceinline__ void flag_eval(float add, float at, float tlim, float l2, float ath,
                                          float q, float lw, float& wm, uint32_t& m,
                                          uint32_t bit) {
    if constexpr (QRANGE && WDEN)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_Q(8) BVML_FLAG_W(9)
            BVML_FLAG_TAIL("or.b32")
            : "+f"(wm), "+r"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "r"(bit),
              "f"(q), "f"(lw));
    else if constexpr (QRANGE)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_Q(8) BVML_FLAG_TAIL("or.b32")
            : "+f"(wm), "+r"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "r"(bit),
              "f"(q));
    else if constexpr (WDEN)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_W(8) BVML_FLAG_TAIL("or.b32")
            : "+f"(wm), "+r"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "r"(bit),
              "f"(lw));
    else
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_TAIL("or.b32")
            : "+f"(wm), "+r"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "r"(bit));
}
template <bool QRANGE, bool WDEN>
__device__ __forceinline__ void flag_eval(float add, float at, float tlim, float l2, float ath,
                                          float q, float lw, float& wm,
                                          unsigned long long& m, unsigned long long bit) {
    if constexpr (QRANGE && WDEN)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_Q(8) BVML_FLAG_W(9)
            BVML_FLAG_TAIL("or.b64")
            : "+f"(wm), "+l"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "l"(bit),
              "f"(q), "f"(lw));
    else if constexpr (QRANGE)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_Q(8) BVML_FLAG_TAIL("or.b64")
            : "+f"(wm), "+l"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "l"(bit),
              "f"(q));
    else if constexpr (WDEN)
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_W(8) BVML_FLAG_TAIL("or.b64")
            : "+f"(wm), "+l"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "l"(bit),
              "f"(lw));
    else
        asm("{\n\t.reg .pred p;\n\t" BVML_FLAG_CORE BVML_FLAG_TAIL("or.b64")
            : "+f"(wm), "+l"(m) : "f"(add), "f"(at), "f"(tlim), "f"(l2), "f"(ath), "l"(bit));
}

// One neighbour slot n for a pixel pair: rotate the (unit) source normals,
// RayReLU them against the pixels' (unit) rays, accumulate with weight w.
// tun = -tu is supplied by the caller (from the staged table).
// QRANGE: test |xy|^2 against [kQMin, kQMax]. fp16 inputs cannot leave that
// range except for an all-zero pair (|xy|^2 lies in {0} u [3.6e-15, 8.6e9]),
// and a zero pair makes dd = inf * 0 = NaN, which the |dd| test flags.
// WDEN: wt holds the weight's denominator d (w = 1/d), see head_activation.
// A flagged evaluation keeps its (possibly non-finite) vector but gets weight
// zero; a non-finite fast sum sends the pixel to a whole-window recompute.
template <typename Mask, bool QRANGE, bool WDEN>
__device__ __forceinline__ void angmf_pair(int n, float2 xs, float2 ys, float2 th, float2 wt,
                                           float2 nx, float2 ny, float2 nz, float2 as,
                                           float2 tun, float2 tv, float2 ifu2, float2 ifv2,
                                           float2 rx, float2 ry, float2 rz, PairAcc<Mask>& A) {
    const float2 q = fma2(xs, xs, mul2(ys, ys));
    const float2 iq = rsqrt2_ftz(q);
    const float2 X = mul2(xs, ifu2), Y = mul2(ys, ifv2);     // d (unnormalised)
    const float2 e = fma2(X, nx, mul2(Y, ny));               // d.n
    const float2 dd = fma2(iq, e, as);                       // (P + d).n, d normalised
    // g = d x P = (Y, -X, gz); g_perp = g - n (g.n) = (gpx, -gpyn, gpz)
    const float2 gz = fma2(X, tv, mul2(Y, tun));
    const float2 ng = fma2(Y, nx, fnma2(X, ny, mul2(gz, nz)));
    const float2 gpx = fnma2(nx, ng, Y);
    const float2 gpyn = fma2(ny, ng, X);
    const float2 gpz = fnma2(nz, ng, gz);
    const float2 gp2 = fma2(gpx, gpx, fma2(gpyn, gpyn, mul2(gpz, gpz)));
    // |g_perp| = 0 gives an infinite or NaN kk below, which the fix-up tests catch
    const float2 gi = rsqrt2_ftz(gp2);
    // sin / cos of theta with the hardware approximations (abs. error ~5e-7
    // on |theta| <= pi; larger angles are left to the fix-up)
    const float2 sn = sin2_approx(th);
    const float2 cs = cos2_approx(th);
    float2 kk = mul2(sn, gi);
    // cancellation guard: t = w sin (n.g) / |g_perp| against kTMax (with w =
    // 1/d: sin (n.g) / |g_perp| against d kTMax)
    float2 t, tlim;
    if constexpr (WDEN) {
        t = mul2(kk, ng);
        tlim = mul2(wt, f2(kTMax));
    } else {
        t = mul2(mul2(wt, kk), ng);
        tlim = f2(kTMax);
    }
    kk.x = __uint_as_float(__float_as_uint(kk.x) ^ (__float_as_uint(dd.x) & 0x80000000u));
    kk.y = __uint_as_float(__float_as_uint(kk.y) ^ (__float_as_uint(dd.y) & 0x80000000u));
    const float2 qx = fma2(kk, gpx, mul2(cs, nx));
    const float2 qy = fnma2(kk, gpyn, mul2(cs, ny));
    const float2 qz = fma2(kk, gpz, mul2(cs, nz));
    // RayReLU against the pixels' rays: m = q + dc r. q and r are unit
    // vectors, so |m|^2 = 1 + 2 dc c + dc^2 = 1 + dc (2c + dc) (exactly 1 when
    // dc = 0); m itself is never formed (fold_ray).
    const float2 c = fma2(qx, rx, fma2(qy, ry, mul2(qz, rz)));
    const float2 dc = max2(fma2(c, f2(-1.0f), f2(kRayEps)), f2(0.0f));
    const float2 l2 = fma2(dc, fma2(c, f2(2.0f), dc), f2(1.0f));
    // w / |m|; with w = 1/d one rsqrt of |m|^2 d^2. d^2 overflows for weights
    // below ~5e-20: those go to the fix-up, whose fp64 weight keeps them
    // nonzero (they decide the direction where every weight is that small).
    float2 wm, lw = f2(0.0f);
    if constexpr (WDEN) {
        lw = mul2(l2, mul2(wt, wt));
        wm = rsqrt2_ftz(lw);
    } else {
        wm = mul2(wt, rsqrt2_ftz(l2));
    }
    flag_eval<QRANGE, WDEN>(fabsf(dd.x), fabsf(t.x), tlim.x, l2.x, fabsf(th.x), q.x, lw.x,
                            wm.x, A.bad0, Mask(1) << n);
    flag_eval<QRANGE, WDEN>(fabsf(dd.y), fabsf(t.y), tlim.y, l2.y, fabsf(th.y), q.y, lw.y,
                            wm.y, A.bad1, Mask(1) << n);
    A.x = fma2(wm, qx, A.x);
    A.y = fma2(wm, qy, A.y);
    A.z = fma2(wm, qz, A.z);
    A.d = fma2(wm, dc, A.d);
}

// The replicate-padded halo of unit source normals in shared memory. Per
// component v, an "even" and an "odd" pair of columns,
//   E[i][k] = (v[i][2k], v[i][2k+1]),  O[i][k] = (v[i][2k+1], v[i][2k+2]),
// so the pair starting at column j is (j even ? E : O)[i][j >> 1]. The four
// staged components -- nx, ny, nz and P.n = tu0 nx + tv0 ny + nz of each
// source pixel (independent of the output pixel, so formed once per tile
// instead of once per evaluation) -- sit two to a float4 plane, (nx pair,
// ny pair) and (nz pair, P.n pair): a neighbour step reads its four pairs
// with two 16-byte loads, and a warp's loads are consecutive float4,
// conflict-free. -tu0 of each pair of columns is tabulated the same way (as
// float2), tv0 per row.
struct NTile {
    float4* e01;  // (nx, ny) pairs starting at column 2k
    float4* e23;  // (nz, P.n) pairs ...
    float4* o01;  // ... starting at column 2k + 1
    float4* o23;
    float2* tune; // (-tu0, -tu1) of the pair starting at column 2k
    float2* tuno; // ... at column 2k + 1
    float* tv;
    int swh;      // pairs per plane row

    // A pair starts at a column j <= SW - 2 (the last output pair, x = 30, at
    // the window's far column, 2R), so SW / 2 pairs per row cover every read:
    // E holds k <= SW/2 - 1, O (j odd, j <= SW - 3) k <= SW/2 - 2. Keeping the
    // rows this short puts the fp16 5x5 CTA at 43.9 KB of shared memory, so
    // three CTAs fit a 132 KB carve-out and leave more L1 for spills.
    static constexpr __host__ __device__ int pairs_per_row(int SW) { return SW / 2; }
    static constexpr __host__ __device__ size_t bytes(int SW, int SH) {
        const int h = pairs_per_row(SW);
        return sizeof(float4) * 4 * (size_t)SH * h + sizeof(float2) * 2 * h + sizeof(float) * SH;
    }
    // base: 16-byte aligned
    __device__ void carve(void* base, int SW, int SH) {
        swh = pairs_per_row(SW);
        e01 = reinterpret_cast<float4*>(base);
        e23 = e01 + SH * swh;
        o01 = e23 + SH * swh;
        o23 = o01 + SH * swh;
        tune = reinterpret_cast<float2*>(o23 + SH * swh);
        tuno = tune + swh;
        tv = reinterpret_cast<float*>(tuno + swh);
    }
    // component c (0..3) of the pair slot (first = the pair's first column)
    // of plane entry q, as a float offset into the 01 or 23 plane
    static __device__ __forceinline__ int slot(int q, int c, bool first) {
        return 4 * q + 2 * (c & 1) + (first ? 0 : 1);
    }
    __device__ __forceinline__ float* eplane(int c) const {
        return reinterpret_cast<float*>(c < 2 ? e01 : e23);
    }
    __device__ __forceinline__ float* oplane(int c) const {
        return reinterpret_cast<float*>(c < 2 ? o01 : o23);
    }
};

// A source normal as the fast path needs it: unit length. The reference
// rotates the raw normal and then divides by max(|Rn|, 1e-12)
// (src/dsine_ops.cpp:143-149), so a normal of length >= 1e-12 acts as its
// direction: huge ones (|v|^2 above 1e30, where the square overflows) are
// rescaled by an exact power of two first. Shorter ones act as a vector of
// length |v| * 1e12 < 1, which the closed form does not cover; they, and zero,
// infinite or NaN normals, are staged as NaN, which sends every evaluation
// that uses them to the exact fix-up (that reads the raw normal).
__device__ __forceinline__ void stage_unit(float (&v)[3]) {
    float n2 = fmaf(v[0], v[0], fmaf(v[1], v[1], v[2] * v[2]));
    if (!(n2 >= 1e-24f && n2 <= 1e30f)) {  // rare
        if (n2 > 1e30f) {
            v[0] *= 0x1p-100f;
            v[1] *= 0x1p-100f;
            v[2] *= 0x1p-100f;
            n2 = fmaf(v[0], v[0], fmaf(v[1], v[1], v[2] * v[2]));
        }
        if (!(n2 >= 1e-24f && n2 <= 3.0e38f)) n2 = __int_as_float(0x7fffffff);  // NaN
    }
    const float inv = rsqrtf(n2);
    v[0] *= inv;
    v[1] *= inv;
    v[2] *= inv;
}

// Stage the tile's normal halo and tu0 / tv0 tables at (x0, y0).
template <typename TNI, bool FUSE_RR>
__device__ __forceinline__ void stage_normals(const TNI* __restrict__ pnb,
                                              const float* __restrict__ ray, const NTile& T,
                                              int x0, int y0, const AngmfArgs& a) {
    const int R = a.R;
    const int SW = kTW + 2 * R;
    const int SH = kTH + 2 * R;
    const long HW = a.HW;
    for (int idx = threadIdx.x; idx < SH * SW; idx += kThreads) {
        const int i = idx / SW, j = idx - i * SW;
        const int sy = clampi(y0 - R + i, 0, a.H - 1);
        const int sx = clampi(x0 - R + j, 0, a.W - 1);
        long sp = (long)sy * a.W + sx;
        if (!check_ok(sp >= 0 && sp < HW, kChkNormalLoad)) sp = 0;
        float v[3] = {St<TNI>::ld(pnb + sp), St<TNI>::ld(pnb + HW + sp),
                      St<TNI>::ld(pnb + 2 * HW + sp)};
        if (FUSE_RR) ray_relu_f32(v[0], v[1], v[2], __ldg(ray + sp), __ldg(ray + HW + sp),
                                  __ldg(ray + 2 * HW + sp));
        stage_unit(v);
        const float tu = fmaf((float)sx, a.ifu, a.tu_c), tv = fmaf((float)sy, a.ifv, a.tv_c);
        const float u4[4] = {v[0], v[1], v[2], fmaf(tu, v[0], fmaf(tv, v[1], v[2]))};  // P.n
        const int k = j >> 1;
        if (!check_ok(i < SH && k < T.swh, kChkHaloSmem)) continue;
        const int q = i * T.swh + k;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float u = u4[c];
            if (j & 1) {
                T.eplane(c)[NTile::slot(q, c, false)] = u;   // E[i][k].y
                T.oplane(c)[NTile::slot(q, c, true)] = u;    // O[i][k].x
            } else {
                T.eplane(c)[NTile::slot(q, c, true)] = u;    // E[i][k].x
                if (k > 0) T.oplane(c)[NTile::slot(q - 1, c, false)] = u;  // O[i][k-1].y
            }
        }
    }
    for (int k = threadIdx.x; k < T.swh; k += kThreads) {
        float t[3];
#pragma unroll
        for (int d = 0; d < 3; ++d)
            t[d] = fmaf((float)clampi(x0 - R + 2 * k + d, 0, a.W - 1), a.ifu, a.tu_c);
        T.tune[k] = make_float2(-t[0], -t[1]);
        T.tuno[k] = make_float2(-t[1], -t[2]);
    }
    for (int i = threadIdx.x; i < SH; i += kThreads) {
        const int s0 = clampi(y0 - R + i, 0, a.H - 1);
        T.tv[i] = fmaf((float)s0, a.ifv, a.tv_c);
    }
}

// Stage the same halo and tables with compile-time geometry (the staged
// kernel): one item per two source columns, so each channel of an item is
// one 8-byte store to the even plane and two 4-byte stores to the odd plane,
// and the item index splits with a constant divisor.
template <int R, typename TNI, bool FUSE_RR, bool COH = false>
__device__ __forceinline__ void stage_normals_ct(const TNI* __restrict__ pnb,
                                                 const float* __restrict__ ray, const NTile& T,
                                                 int x0, int y0, const AngmfArgs& a) {
    constexpr int SW = kTW + 2 * R, SH = kTH + 2 * R;
    constexpr int NP = SW / 2;  // column pairs per halo row (SW is even)
    constexpr int SWH = NTile::pairs_per_row(SW);
    static_assert(SW % 2 == 0, "halo width must be even");
    const long HW = a.HW;
    for (int it = threadIdx.x; it < SH * NP; it += kThreads) {
        const int i = it / NP, k = it - (it / NP) * NP;
        const long row = (long)clampi(y0 - R + i, 0, a.H - 1) * a.W;
        const int sx = x0 - R + 2 * k;
        long q0 = row + clampi(sx, 0, a.W - 1);
        long q1 = row + clampi(sx + 1, 0, a.W - 1);
        if (!check_ok(q0 >= 0 && q0 < HW && q1 >= 0 && q1 < HW, kChkNormalLoad)) q0 = q1 = 0;
        float v0[3], v1[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            v0[c] = ldn<TNI, COH>(pnb + c * HW + q0);
            v1[c] = ldn<TNI, COH>(pnb + c * HW + q1);
        }
        if (FUSE_RR) {
            ray_relu_f32(v0[0], v0[1], v0[2], __ldg(ray + q0), __ldg(ray + HW + q0),
                         __ldg(ray + 2 * HW + q0));
            ray_relu_f32(v1[0], v1[1], v1[2], __ldg(ray + q1), __ldg(ray + HW + q1),
                         __ldg(ray + 2 * HW + q1));
        }
        stage_unit(v0);
        stage_unit(v1);
        // P.n of both source pixels (the same tu0 / tv0 as the tables below)
        const float tv = fmaf((float)clampi(y0 - R + i, 0, a.H - 1), a.ifv, a.tv_c);
        const float tu0 = fmaf((float)clampi(sx, 0, a.W - 1), a.ifu, a.tu_c);
        const float tu1 = fmaf((float)clampi(sx + 1, 0, a.W - 1), a.ifu, a.tu_c);
        const float w0[4] = {v0[0], v0[1], v0[2], fmaf(tu0, v0[0], fmaf(tv, v0[1], v0[2]))};
        const float w1[4] = {v1[0], v1[1], v1[2], fmaf(tu1, v1[0], fmaf(tv, v1[1], v1[2]))};
        if (!check_ok(i < SH && k < SWH, kChkHaloSmem)) continue;
        const int q = i * SWH + k;
        T.e01[q] = make_float4(w0[0], w1[0], w0[1], w1[1]);   // E[i][k] of nx, ny
        T.e23[q] = make_float4(w0[2], w1[2], w0[3], w1[3]);   // ... of nz, P.n
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float* op = T.oplane(c);
            op[NTile::slot(q, c, true)] = w1[c];                   // O[i][k].x
            if (k > 0) op[NTile::slot(q - 1, c, false)] = w0[c];   // O[i][k-1].y
        }
    }
    for (int k = threadIdx.x; k < SWH; k += kThreads) {
        float t[3];
#pragma unroll
        for (int d = 0; d < 3; ++d)
            t[d] = fmaf((float)clampi(x0 - R + 2 * k + d, 0, a.W - 1), a.ifu, a.tu_c);
        T.tune[k] = make_float2(-t[0], -t[1]);
        T.tuno[k] = make_float2(-t[1], -t[2]);
    }
    for (int i = threadIdx.x; i < SH; i += kThreads)
        T.tv[i] = fmaf((float)clampi(y0 - R + i, 0, a.H - 1), a.ifv, a.tv_c);
}

// The staged operands of the pair starting at column j of halo row i.
struct NPair {
    float2 nx, ny, nz, as, tun, tv;  // as = P.n
};
__device__ __forceinline__ NPair npair(const NTile& T, int i, int j) {
    const int k = i * T.swh + (j >> 1);
    const float4 a = (j & 1) ? T.o01[k] : T.e01[k];
    const float4 c = (j & 1) ? T.o23[k] : T.e23[k];
    NPair r;
    r.nx = f2(a.x, a.y);
    r.ny = f2(a.z, a.w);
    r.nz = f2(c.x, c.y);
    r.as = f2(c.z, c.w);
    r.tun = (j & 1) ? T.tuno[j >> 1] : T.tune[j >> 1];
    r.tv = f2(T.tv[i]);
    return r;
}

// Exact fp64 fix-ups of the flagged neighbours of one pixel; returns the sum
// in fp64 (a pixel whose weights all vanish has a sum far below the float
// range, and the reference normalises it in fp64).
template <int PS, typename TS, typename TNI, bool FUSE_RR, bool ACT, bool COH, typename Mask>
__device__ __noinline__ double3 fixups(Mask m, int b, int x, int y, const TNI* __restrict__ pn,
                                      const TS* __restrict__ prob, const TS* __restrict__ xy,
                                      const TS* __restrict__ ang, const float* __restrict__ ray,
                                      const AngmfArgs a) {
    constexpr int P = PS * PS;
    const long HW = a.HW;
    const long pp = (long)y * a.W + x;
    const TNI* pnb = pn + (long)b * 3 * HW;
    const TS* xyb = xy + (long)b * 2 * P * HW;
    const TS* prb = prob + (long)b * P * HW;
    const TS* anb = ang + (long)b * P * HW;
    const double orx = __ldg(ray + pp), ory = __ldg(ray + HW + pp), orz = __ldg(ray + 2 * HW + pp);
    double ax = 0.0, ay = 0.0, az = 0.0;
    while (m != 0) {
        int n;
        if constexpr (sizeof(Mask) == 4) n = __ffs(m) - 1;
        else n = __ffsll((long long)m) - 1;
        m &= m - 1;
        const int ky = n / PS, kx = n - (n / PS) * PS;
        const int sy = clampi(y - a.R + ky * a.dil, 0, a.H - 1);
        const int sx = clampi(x - a.R + kx * a.dil, 0, a.W - 1);
        const long sp = (long)sy * a.W + sx;
        double nx = ldn<TNI, COH>(pnb + sp), ny = ldn<TNI, COH>(pnb + HW + sp),
               nz = ldn<TNI, COH>(pnb + 2 * HW + sp);
        if (FUSE_RR)
            ray_relu_exact(nx, ny, nz, __ldg(ray + sp), __ldg(ray + HW + sp),
                           __ldg(ray + 2 * HW + sp));
        double th = St<TS>::ld(anb + (long)n * HW + pp), w = St<TS>::ld(prb + (long)n * HW + pp);
        if (ACT) head_activation_exact(w, th);
        const double3 c3 = angmf_neighbor_exact(
            nx, ny, nz, sx, sy, St<TS>::ld(xyb + (long)n * HW + pp),
            St<TS>::ld(xyb + (long)(P + n) * HW + pp), th, w, orx, ory, orz, a.fu, a.cu, a.fv,
            a.cv);
        ax += c3.x;
        ay += c3.y;
        az += c3.z;
    }
    return make_double3(ax, ay, az);
}

// Where a tile's source normals come from. SrcFixed: one type and RayReLU
// choice fixed at compile time (the one-tile kernels). SrcDual: chosen per
// work item (the persistent kernel: iteration 0 stages the storage-typed
// decoder normals with the initial RayReLU fused, later iterations the
// previous iteration's fp32 normals), so that the kernel holds one copy of
// the neighbour loop rather than one per variant: two copies in one body
// raised its register spills and cost about 5 % per item.
template <typename TNI, bool FUSE_RR>
struct SrcFixed {
    const TNI* pn;
    template <int R, bool COH>
    __device__ __forceinline__ void stage(int b, const float* ray, const NTile& T, int x0,
                                          int y0, const AngmfArgs& a) const {
        stage_normals_ct<R, TNI, FUSE_RR, COH>(pn + (long)b * 3 * a.HW, ray, T, x0, y0, a);
    }
    template <int PS, typename TS, bool ACT, bool COH, typename Mask>
    __device__ __forceinline__ double3 fix(Mask m, int b, int x, int y, const TS* prob,
                                           const TS* xy, const TS* ang, const float* ray,
                                           const AngmfArgs& a) const {
        return fixups<PS, TS, TNI, FUSE_RR, ACT, COH>(m, b, x, y, pn, prob, xy, ang, ray, a);
    }
};
template <typename TS>
struct SrcDual {
    const TS* pn0;      // iteration 0: the decoder normals (storage type), RayReLU fused
    const float* prev;  // later iterations: the previous iteration's fp32 normals
    bool first;
    template <int R, bool COH>
    __device__ __forceinline__ void stage(int b, const float* ray, const NTile& T, int x0,
                                          int y0, const AngmfArgs& a) const {
        if (first)
            stage_normals_ct<R, TS, true, COH>(pn0 + (long)b * 3 * a.HW, ray, T, x0, y0, a);
        else
            stage_normals_ct<R, float, false, COH>(prev + (long)b * 3 * a.HW, ray, T, x0, y0,
                                                   a);
    }
    template <int PS, typename TSS, bool ACT, bool COH, typename Mask>
    __device__ __forceinline__ double3 fix(Mask m, int b, int x, int y, const TSS* prob,
                                           const TSS* xy, const TSS* ang, const float* ray,
                                           const AngmfArgs& a) const {
        if (first)
            return fixups<PS, TSS, TS, true, ACT, COH>(m, b, x, y, pn0, prob, xy, ang, ray, a);
        return fixups<PS, TSS, float, false, ACT, COH>(m, b, x, y, prev, prob, xy, ang, ray, a);
    }
};

// Normalise the pair's sums (after fix-ups) and store.
template <int PS, typename TS, typename Src, typename TNO, bool ACT, bool COH, typename Mask>
__device__ __forceinline__ void finish_pair(PairAcc<Mask>& A, int b, int x, int y, bool two,
                                            bool vec, const Src& src, const TS* prob,
                                            const TS* xy, const TS* ang, const float* ray,
                                            TNO* out, const AngmfArgs& a) {
    const float2 l = fma2(A.x, A.x, fma2(A.y, A.y, mul2(A.z, A.z)));
    const float2 inv = rsqrt2(max2(l, f2(1e-24f)));
    float2 ox = mul2(A.x, inv), oy = mul2(A.y, inv), oz = mul2(A.z, inv);
    // A pixel with fix-ups is finished in fp64 (fast sum + exact sum, then the
    // reference's normalise, src/dsine_ops.cpp:165-169). A fast sum below
    // 1e-30 means every weight (nearly) vanished: its direction needs more
    // range than fp32 has, so the whole window is recomputed exactly; so is a
    // non-finite fast sum.
    constexpr Mask kAll = (P_OF<PS>::value >= 8 * (int)sizeof(Mask))
                              ? ~Mask(0)
                              : ((Mask(1) << P_OF<PS>::value) - 1);
    // a fast sum that is non-finite (a flagged neighbour's vector was) or
    // vanishing: the whole window in fp64 (the unordered test also catches NaN)
    auto whole = [](float u, float v, float w) {
        const float a = fabsf(u) + fabsf(v) + fabsf(w);
        return !(a >= 1e-30f && a <= 3.0e38f);
    };
    auto exact = [&](Mask m, int px, float fx, float fy, float fz, float& o0, float& o1,
                     float& o2) {
        if (whole(fx, fy, fz)) {
            m = kAll;
            fx = fy = fz = 0.0f;
        }
        if (m == 0) return;
        const double3 f =
            src.template fix<PS, TS, ACT, COH>(m, b, px, y, prob, xy, ang, ray, a);
        const double sx = (double)fx + f.x, sy = (double)fy + f.y, sz = (double)fz + f.z;
        const double sinv = 1.0 / fmax(sqrt(sx * sx + sy * sy + sz * sz), 1e-12);
        o0 = (float)(sx * sinv);
        o1 = (float)(sy * sinv);
        o2 = (float)(sz * sinv);
    };
    exact(A.bad0, x, A.x.x, A.y.x, A.z.x, ox.x, oy.x, oz.x);
    if (two) exact(A.bad1, x + 1, A.x.y, A.y.y, A.z.y, ox.y, oy.y, oz.y);
    const long HW = a.HW;
    const long p0 = (long)y * a.W + x;
    TNO* ob = out + (long)b * 3 * HW;
    if (!check_ok(y >= 0 && y < a.H && x >= 0 && x < a.W && (!two || x + 1 < a.W), kChkStore))
        return;
    if (vec) {
        if constexpr (std::is_same<TNO, float>::value) {
            // fp32 normals are the fused unit's intermediates (or its last
            // iteration's output, which the upsample reads next): kept in L2
            const uint64_t keep = l2_evict_last();
            st2_hint(ob + p0, ox, keep);
            st2_hint(ob + HW + p0, oy, keep);
            st2_hint(ob + 2 * HW + p0, oz, keep);
        } else {
            St<TNO>::st2(ob + p0, ox);
            St<TNO>::st2(ob + HW + p0, oy);
            St<TNO>::st2(ob + 2 * HW + p0, oz);
        }
    } else {
        St<TNO>::st(ob + p0, ox.x);
        St<TNO>::st(ob + HW + p0, oy.x);
        St<TNO>::st(ob + 2 * HW + p0, oz.x);
        if (two) {
            St<TNO>::st(ob + p0 + 1, ox.y);
            St<TNO>::st(ob + HW + p0 + 1, oy.y);
            St<TNO>::st(ob + 2 * HW + p0 + 1, oz.y);
        }
    }
}

__device__ __forceinline__ void pair_ray(const float* __restrict__ ray, long HW, long p0, long p1,
                                         float2& rx, float2& ry, float2& rz) {
    rx = f2(__ldg(ray + p0), __ldg(ray + p1));
    ry = f2(__ldg(ray + HW + p0), __ldg(ray + HW + p1));
    rz = f2(__ldg(ray + 2 * HW + p0), __ldg(ray + 2 * HW + p1));
    const float2 ri = rsqrt2(max2(fma2(rx, rx, fma2(ry, ry, mul2(rz, rz))), f2(1e-16f)));
    rx = mul2(rx, ri);
    ry = mul2(ry, ri);
    rz = mul2(rz, ri);
}

__device__ __forceinline__ void tile_of(const AngmfArgs& a, int& b, int& x0, int& y0) {
    int t = blockIdx.x;
    const int tix = t % a.tiles_x;
    t /= a.tiles_x;
    const int tiy = t % a.tiles_y;
    b = t / a.tiles_y;
    x0 = tix * kTW;
    y0 = tiy * kTH;
}

// ---------------------------------------------------------------------------
// General kernel: per-neighbour channels read straight from global memory.
// Any shape; used when the width does not allow 16-byte staged copies.
template <int PS, typename TS, typename TNI, typename TNO, bool FUSE_RR, bool ACT>
__global__ void __launch_bounds__(kThreads, 2)
angmf_kernel(const TNI* __restrict__ pn, const TS* __restrict__ prob, const TS* __restrict__ xy,
             const TS* __restrict__ ang, const float* __restrict__ ray, TNO* __restrict__ out,
             const AngmfArgs a) {
    constexpr int P = PS * PS;
    using Mask = typename std::conditional<(P <= 32), uint32_t, unsigned long long>::type;
    pdl_trigger();
    pdl_wait();  // (launched as a dependent: the previous iteration's normals)
    extern __shared__ float4 smem4[];
    NTile T;
    T.carve(smem4, kTW + 2 * a.R, kTH + 2 * a.R);
    int b, x0, y0;
    tile_of(a, b, x0, y0);
    const long HW = a.HW;
    stage_normals<TNI, FUSE_RR>(pn + (long)b * 3 * HW, ray, T, x0, y0, a);
    __syncthreads();

    const int lx = 2 * (threadIdx.x % (kTW / 2));
    const int ly = threadIdx.x / (kTW / 2);
    const int x = x0 + lx, y = y0 + ly;
    if (y >= a.H || x >= a.W) return;
    const bool two = x + 1 < a.W;
    const bool vec = (a.W & 1) == 0;
    const long p0 = (long)y * a.W + x;
    const long p1 = two ? p0 + 1 : p0;
    float2 rx, ry, rz;
    pair_ray(ray, HW, p0, p1, rx, ry, rz);
    const TS* xyb = xy + (long)b * 2 * P * HW;
    const TS* prb = prob + (long)b * P * HW;
    const TS* anb = ang + (long)b * P * HW;
    auto ld = [&](const TS* base) -> float2 {
        return vec ? St<TS>::ld2s(base + p0) : f2(St<TS>::lds1(base + p0), St<TS>::lds1(base + p1));
    };
    const float2 ifu2 = a.ifu2, ifv2 = a.ifv2;
    PairAcc<Mask> A{f2(0.f), f2(0.f), f2(0.f), f2(0.f), 0, 0};
#pragma unroll 1
    for (int ky = 0; ky < PS; ++ky) {
        const int i = ly + ky * a.dil;
#pragma unroll
        for (int kx = 0; kx < PS; ++kx) {
            const int n = ky * PS + kx;
            const NPair q = npair(T, i, lx + kx * a.dil);
            float2 th = ld(anb + (long)n * HW), wt = ld(prb + (long)n * HW);
            if (ACT) head_activation(wt, th);
            angmf_pair<Mask, sizeof(TS) == 4, ACT>(
                n, ld(xyb + (long)n * HW), ld(xyb + (long)(P + n) * HW), th, wt, q.nx, q.ny,
                q.nz, q.as, q.tun, q.tv, ifu2, ifv2, rx, ry, rz, A);
        }
    }
    fold_ray(A, rx, ry, rz);
    finish_pair<PS, TS, SrcFixed<TNI, FUSE_RR>, TNO, ACT, false>(
        A, b, x, y, two, vec, SrcFixed<TNI, FUSE_RR>{pn}, prob, xy, ang, ray, out, a);
}

// ---------------------------------------------------------------------------
// Staged kernel (width a multiple of 16 bytes of storage, dilation 1 or 2).
// Each warp owns two rows of the tile; for every neighbour slot n it copies
// exactly the data its own lanes will consume -- the four channel strips
// (prob, x offset, y offset, angle; 2 rows x 32 pixels each) -- global ->
// shared with 16-byte cp.async into a warp-private ring of kN = kM * PS
// slots (slot of neighbour n: n mod kN), kD = kN - kSP slots ahead of the one
// being computed. Memory latency is covered by the copies in flight instead of
// registers, and publishing slots needs only a warp barrier: one per kSP
// neighbour slots (two for fp16 storage, so that two neighbours' dependency
// chains interleave between barriers). With the window size, the dilation and
// the window column compile-time constants, every shared-memory offset is an
// immediate.
// (evict-first in L2: every per-neighbour input is read exactly once)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;\n" ::"r"(s),
                 "l"(gmem), "r"(valid ? 16 : 0), "l"(l2_evict_first())
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename TS, int PS>
struct Stages {
    static constexpr int kEpc = 16 / (int)sizeof(TS);     // elements per 16-byte chunk
    static constexpr int kCpr = kTW / kEpc;                // chunks per strip row
    static constexpr int kRowsW = 2;                       // tile rows per warp
    static constexpr int kChunksW = 4 * kRowsW * kCpr;     // per warp per slot
    static constexpr int kPerLane = kChunksW / 32;         // 1 (fp16) or 2 (fp32)
    static constexpr int kElemsW = 4 * kRowsW * kTW;       // per warp per slot
    // window rows per ring: one. Two rows for fp16 (10 slots, 8 ahead) were
    // slower: the larger shared-memory carve-out left less L1 for the
    // kernel's register spills (0.2591 against 0.2550 ms per config-4 launch,
    // bit-identical)
    static constexpr int kM = 1;
    static constexpr int kN = kM * PS;                     // ring depth
    static constexpr int kSP = sizeof(TS) == 2 ? 2 : 1;    // slots per warp barrier
    static constexpr int kD = kN - kSP;                    // slots issued ahead
    static constexpr size_t kBytes = (size_t)(kThreads / 32) * kN * kElemsW * sizeof(TS);
};

// Shared memory of a staged variant and the CTAs per SM it is compiled for:
// three when three fit (more warps to hide the dependency chains; the
// register cap is then 80 and a few loop invariants spill to L1), else two.
template <int PS, int DIL, typename TS>
struct StagedCfg {
    static constexpr int R = (PS / 2) * DIL;
    static constexpr size_t kSmem =
        Stages<TS, PS>::kBytes + NTile::bytes(kTW + 2 * R, kTH + 2 * R);
    static constexpr int kMinBlocks = 3 * (kSmem + 1024) <= 228 * 1024 ? 3 : 2;
};

template <typename TS> __device__ __forceinline__ float2 lds2(const TS* p);
template <> __device__ __forceinline__ float2 lds2<float>(const float* p) {
    return *reinterpret_cast<const float2*>(p);
}
template <> __device__ __forceinline__ float2 lds2<__half>(const __half* p) {
    return __half22float2(*reinterpret_cast<const __half2*>(p));
}

// One tile of one iteration: frame b, tile origin (x0, y0). `pre` runs after
// the first ring slots are in flight and before the normal halo is staged
// (the persistent kernel waits there for the tiles it depends on). COH: read
// the normals with L2-coherent loads (they were written in the same launch).
template <int PS, int DIL, typename TS, typename Src, typename TNO, bool ACT, bool COH,
          typename Pre>
__device__ __forceinline__ void angmf_tile(const Src& nsrc, const TS* __restrict__ prob,
                                           const TS* __restrict__ xy, const TS* __restrict__ ang,
                                           const float* __restrict__ ray, TNO* __restrict__ out,
                                           const AngmfArgs& a, int b, int x0, int y0,
                                           Pre&& pre) {
    constexpr int P = PS * PS;
    constexpr int R = (PS / 2) * DIL;
    constexpr int SW = kTW + 2 * R, SH = kTH + 2 * R;
    constexpr int SWH = NTile::pairs_per_row(SW);
    using Mask = typename std::conditional<(P <= 32), uint32_t, unsigned long long>::type;
    using S = Stages<TS, PS>;
    extern __shared__ float4 smem4[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    TS* ring = reinterpret_cast<TS*>(smem4) + warp * S::kN * S::kElemsW;  // this warp's slots
    NTile T;
    T.carve(reinterpret_cast<char*>(smem4) + S::kBytes, SW, SH);
    const long HW = a.HW;
    const TS* xyb = xy + (long)b * 2 * P * HW;
    const TS* prb = prob + (long)b * P * HW;
    const TS* anb = ang + (long)b * P * HW;

    // this lane's chunks: source of the next slot to issue, slot offset, validity
    const TS* src[S::kPerLane];
    int dst[S::kPerLane];
    bool valid[S::kPerLane];
#pragma unroll
    for (int k = 0; k < S::kPerLane; ++k) {
        const int q = lane + 32 * k;
        const int c = q / (S::kRowsW * S::kCpr);
        const int r = (q / S::kCpr) % S::kRowsW;
        const int cc = q % S::kCpr;
        const TS* base = c == 0 ? prb : c == 1 ? xyb : c == 2 ? xyb + (long)P * HW : anb;
        const int gy = y0 + S::kRowsW * warp + r, gx = x0 + cc * S::kEpc;
        valid[k] = gy < a.H && gx < a.W;
        if (!check_ok(!valid[k] || gx + S::kEpc <= a.W, kChkRing)) valid[k] = false;
        src[k] = valid[k] ? base + (long)gy * a.W + gx : base;
        dst[k] = (c * S::kRowsW + r) * kTW + cc * S::kEpc;
    }
    auto issue = [&](int slot) {
        if (!check_ok(slot >= 0 && slot < S::kN, kChkRing)) return;
        TS* sl = ring + slot * S::kElemsW;
#pragma unroll
        for (int k = 0; k < S::kPerLane; ++k) {
            cp_async16(sl + dst[k], src[k], valid[k]);
            if (valid[k]) src[k] += HW;  // the same strip of the next neighbour slot
        }
    };

    // prologue: the first kD slots in flight while the normals are staged (the
    // warp's lanes are done with the ring of any earlier tile)
    __syncwarp();
#pragma unroll
    for (int sl = 0; sl < S::kD; ++sl) {
        if (sl < P) issue(sl);
        cp_async_commit();
    }
    pre();
    nsrc.template stage<R, COH>(b, ray, T, x0, y0, a);
    __syncthreads();  // the normal halo is shared by all warps

    const int lx = 2 * (lane & 15);
    const int ly = S::kRowsW * warp + (lane >> 4);
    const int x = x0 + lx, y = y0 + ly;
    const bool active = y < a.H && x < a.W;
    // A warp whose lanes all lie outside the frame has nothing to compute: its
    // ring is private and no CTA barrier follows, so it leaves now. Lanes of a
    // partly covered warp compute on the clamped, zero-filled data like the
    // others (no per-step branch) and drop their results at the end.
    if (__all_sync(0xffffffffu, !active)) {
        cp_async_wait<0>();
        return;
    }
    const bool two = x + 1 < a.W;
    const long p0 = (long)min(y, a.H - 1) * a.W + min(x, a.W - 1);
    const long p1 = two ? p0 + 1 : p0;
    float2 rx, ry, rz;
    pair_ray(ray, HW, p0, p1, rx, ry, rz);
    const float2 ifu2 = a.ifu2, ifv2 = a.ifv2;
    PairAcc<Mask> A{f2(0.f), f2(0.f), f2(0.f), f2(0.f), 0, 0};
    constexpr int kStrip = S::kRowsW * kTW;
    const TS* ring_lane = ring + (lane >> 4) * kTW + lx;   // this pair inside a slot
    const int pbase = ly * SWH + (lx >> 1);                // this pair's first window pair

    // Window rows: fully unrolled for activated inputs (every ring slot and
    // window offset an immediate), rolled for raw head outputs, whose larger
    // per-neighbour step spills less that way (0.097 against 0.107 ms per
    // 64-frame launch; unrolled is 5 % faster for activated inputs). With a
    // one-row ring the slots depend on the window column only.
    constexpr int kRowUnroll = ACT ? 1 : PS;
#pragma unroll kRowUnroll
    for (int ky = 0; ky < PS; ++ky) {
        const int grp = (ky % S::kM) * PS;                  // slot group of this window row
        const int prev_grp = ((ky + S::kM - 1) % S::kM) * PS;  // ... of the previous row
        const TS* st_row = ring_lane + grp * S::kElemsW;
        const int prow = pbase + ky * DIL * SWH;
        const float2 tv = f2(T.tv[ly + ky * DIL]);
#pragma unroll
        for (int kx = 0; kx < PS; ++kx) {
            const int n = ky * PS + kx;
            if (kx % S::kSP == 0) {
                // a group of gs slots (the last of a window row may be short);
                // one commit group per slot, so the wait depth is kD - gs
                const int gs = PS - kx < S::kSP ? PS - kx : S::kSP;
                static_assert(S::kSP <= 2, "wait depths below cover groups of 1 or 2");
                if (gs == 2) cp_async_wait<S::kD - 2>();
                else cp_async_wait<S::kD - 1>();
                __syncwarp();  // the group's slots visible; every lane done with earlier slots
                // refill the slots of the previous kSP neighbours with the ones kD ahead
#pragma unroll
                for (int e = 0; e < S::kSP; ++e) {
                    if (e < gs) {
                        const int j = kx + e - S::kSP;  // window column of neighbour n+e-kSP
                        if (n + e + S::kD < P) issue(j >= 0 ? grp + j : prev_grp + PS + j);
                        cp_async_commit();
                    }
                }
            }
            {
                const TS* st = st_row + kx * S::kElemsW;
                // window column offset: a constant once the kx loop is unrolled
                const int dj = kx * DIL;
                int pi = prow + (dj >> 1);
                if (!check_ok(pi >= 0 && pi < SH * SWH, kChkHaloSmem)) pi = 0;
                const float4 n01 = (dj & 1) ? T.o01[pi] : T.e01[pi];
                const float4 n23 = (dj & 1) ? T.o23[pi] : T.e23[pi];
                const float2 tun = (dj & 1) ? T.tuno[(lx >> 1) + (dj >> 1)]
                                            : T.tune[(lx >> 1) + (dj >> 1)];
                float2 th = lds2<TS>(st + 3 * kStrip), wt = lds2<TS>(st);
                if (ACT) head_activation(wt, th);
                angmf_pair<Mask, sizeof(TS) == 4, ACT>(
                    n, lds2<TS>(st + 1 * kStrip), lds2<TS>(st + 2 * kStrip), th, wt,
                    f2(n01.x, n01.y), f2(n01.z, n01.w), f2(n23.x, n23.y), f2(n23.z, n23.w), tun,
                    tv, ifu2, ifv2, rx, ry, rz, A);
            }
        }
    }
    cp_async_wait<0>();
    if (!active) return;
    fold_ray(A, rx, ry, rz);
    finish_pair<PS, TS, Src, TNO, ACT, COH>(A, b, x, y, two, true, nsrc, prob, xy, ang, ray,
                                            out, a);
}

template <int PS, int DIL, typename TS, typename TNI, typename TNO, bool FUSE_RR, bool ACT>
__global__ void __launch_bounds__(kThreads, (StagedCfg<PS, DIL, TS>::kMinBlocks))
angmf_staged_kernel(const TNI* __restrict__ pn, const TS* __restrict__ prob,
                    const TS* __restrict__ xy, const TS* __restrict__ ang,
                    const float* __restrict__ ray, TNO* __restrict__ out, const AngmfArgs a) {
    // The next iteration's launch may start its CTAs (ring prologue: its own
    // per-neighbour inputs, written before this launch began) during this
    // launch's last wave; a CTA launched that way waits before it stages the
    // normals this launch writes.
    pdl_trigger();
    // grid (tiles_x, tiles_y, frames)
    angmf_tile<PS, DIL, TS, SrcFixed<TNI, FUSE_RR>, TNO, ACT, false>(
        SrcFixed<TNI, FUSE_RR>{pn}, prob, xy, ang, ray, out, a, (int)blockIdx.z,
        (int)blockIdx.x * kTW, (int)blockIdx.y * kTH, [] { pdl_wait(); });
}

// ---------------------------------------------------------------------------
// Persistent kernel: all iterations of the fused refine in one launch.
//
// Work items are (iteration, frame, tile), numbered iteration-major, and CTAs
// take them in order from an atomic counter. The tile of iteration it reads
// iteration it-1's normals of its own and its 8 neighbouring tiles (the halo
// R <= 4 fits inside one tile on every side), so before staging them it waits
// until those tiles' completion counters reach it; one thread per neighbour
// polls with acquire loads while the tile's own first ring slots (inputs of
// iteration it, independent of the normals) are already in flight. A tile
// publishes its own counter (release, after a CTA barrier) once its outputs
// are stored. Every item a CTA waits on was taken earlier by a CTA that is
// running, so the order always makes progress whatever the residency; there
// is no barrier across the whole grid, and the tiles of iteration it+1 run
// while the last tiles of iteration it finish (the kernel boundary and its
// tail of partly idle SMs is paid once, not once per iteration). It is used
// for batches of at most kPersistentMaxWaves waves of tiles per iteration;
// larger batches launch the one-tile kernel once per iteration.
//
// Iteration it writes buf[it & 1] and reads buf[(it - 1) & 1] (iteration 0
// reads the decoder normals, RayReLU fused in the staging). Writing
// buf[it & 1] over what iteration it-1 of a neighbouring tile reads is safe
// because it waits for exactly those tiles. The waits are bounded
// (kDepWaitLimit polls): a wait that gives up sets the status word and the
// tile goes on (no hang); the host reads the word with bvml_refine_status.
constexpr int kMaxFusedIters = 64;
constexpr unsigned kDepWaitLimit = 1u << 22;
constexpr long kPersistentMaxWaves = 3;  // tiles per iteration, in waves of the GPU

struct AngmfIters {
    const void* pn0;                    // iteration 0 input normals (storage type)
    const void* prob[kMaxFusedIters];   // per iteration (storage type)
    const void* xy[kMaxFusedIters];
    const void* ang[kMaxFusedIters];
    float* buf[2];                      // fp32 normals, ping-pong
    int iters;
    int first;                          // first iteration this launch runs
    int* counter;                       // next work item (zero at launch)
    int* done;                          // per tile: iterations completed (zero at launch)
    int* status;                        // nonzero: a dependency wait gave up
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int PS, int DIL, typename TS, bool ACT>
__global__ void __launch_bounds__(kThreads, (StagedCfg<PS, DIL, TS>::kMinBlocks))
angmf_iters_kernel(const float* __restrict__ ray, const AngmfArgs a, const AngmfIters J) {
    // Three round trips per item are spread over three warps so that their
    // latencies overlap instead of adding up ahead of a CTA barrier: warp 2
    // claims the next item (its atomic issued at the start, its result stored
    // only at the end), warp 1 polls the dependencies, warp 7 publishes the
    // completion.
    constexpr int kClaim = 64, kPoll = 32, kSignal = kThreads - 32;
    pdl_trigger();  // the upsample's CTAs may take the slots of exiting CTAs
    __shared__ int s_item[2];
    const int tid = threadIdx.x;
    const int per_it = a.tiles_x * a.tiles_y * a.B;
    const int total = per_it * (J.iters - J.first);
    if (tid == kClaim) s_item[0] = atomicAdd(J.counter, 1);
    __syncthreads();
    int item = s_item[0];
    int par = 0;
    while (item < total) {
        const int it = J.first + item / per_it;
        int t = item % per_it;
        const int tx = t % a.tiles_x;
        t /= a.tiles_x;
        const int ty = t % a.tiles_y;
        const int b = t / a.tiles_y;
        int* mine = J.done + ((long)b * a.tiles_y + ty) * a.tiles_x + tx;
        if (!check_ok(b < a.B && ty < a.tiles_y && tx < a.tiles_x, kChkDep)) break;
        int next = 0;
        if (tid == kClaim) next = atomicAdd(J.counter, 1);
        auto pre = [&] {
            const int q = tid - kPoll;
            if (it > J.first && q >= 0 && q < 9) {
                const int nx = tx + q % 3 - 1, ny = ty + q / 3 - 1;
                if (nx >= 0 && nx < a.tiles_x && ny >= 0 && ny < a.tiles_y) {
                    const int* f = J.done + ((long)b * a.tiles_y + ny) * a.tiles_x + nx;
                    // bounded; once any wait has given up, the others stop too
                    unsigned k = 0;
                    while (ld_acquire_gpu(f) < it - J.first) {
                        if (++k == kDepWaitLimit) {
                            atomicOr(J.status, 1);
                            break;
                        }
                        if (ld_acquire_gpu(J.status) != 0) break;
                        __nanosleep(64);
                    }
                }
            }
            __syncthreads();  // the neighbours' normals are visible to every thread
        };
        float* o = J.buf[it & 1];
        // one tile body for every iteration: iteration 0 stages the decoder
        // normals with the initial RayReLU, later ones the previous fp32 result
        const SrcDual<TS> src{static_cast<const TS*>(J.pn0), J.buf[(it - 1) & 1], it == 0};
        angmf_tile<PS, DIL, TS, SrcDual<TS>, float, ACT, true>(
            src, static_cast<const TS*>(J.prob[it]), static_cast<const TS*>(J.xy[it]),
            static_cast<const TS*>(J.ang[it]), ray, o, a, b, tx * kTW, ty * kTH, pre);
        if (tid == kClaim) s_item[par ^ 1] = next;
        // every output of the tile stored (and the halo no longer read); the
        // release store is cumulative over the stores ordered before the barrier
        __syncthreads();
        if (tid == kSignal) st_release_gpu(mine, it - J.first + 1);
        item = s_item[par ^ 1];
        par ^= 1;
    }
}

template <int PS, typename LaunchT>
AngmfArgs make_args(const LaunchT& L) {
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
    a.ifu2 = make_float2(a.ifu, a.ifu);
    a.ifv2 = make_float2(a.ifv, a.ifv);
    a.tu_c = (float)((0.5 - L.cu) / L.fu);
    a.tv_c = (float)((0.5 - L.cv) / L.fv);
    a.fu = L.fu;
    a.cu = L.cu;
    a.fv = L.fv;
    a.cv = L.cv;
    return a;
}

// The persistent all-iterations kernel for one window / storage type:
// cudaErrorNotSupported when the shape does not take the staged path (the
// caller then launches iteration by iteration).
template <int PS, int DIL, typename TS, bool ACT>
cudaError_t launch_iters_t(const AngmfItersLaunch& L, cudaStream_t s) {
    AngmfArgs a = make_args<PS>(L);
    const long per_it = (long)a.tiles_x * a.tiles_y * L.B;
    const long total = per_it * (L.iters - L.first);
    if (total <= 0 || total > 0x7fffffffL - 0x100000L) return cudaErrorNotSupported;
    auto kern = angmf_iters_kernel<PS, DIL, TS, ACT>;
    const size_t smem = StagedCfg<PS, DIL, TS>::kSmem;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per_sm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem)) !=
        cudaSuccess)
        return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const long slots = (long)sms * per_sm;
    // Per tile, the persistent loop costs about 1.3 us more than a one-tile
    // CTA (claiming the item, the completion fence, the dependency poll): it
    // pays off only where an iteration is a few waves of tiles, so that the
    // per-launch tails it removes are a large share (32 frames of 720p: 2.2
    // waves, 5 % faster per unit; from 64 frames on, one launch per iteration
    // is faster).
    if (per_it > kPersistentMaxWaves * slots) return cudaErrorNotSupported;
    const unsigned grid = (unsigned)(total < slots ? total : slots);
    e = cudaMemsetAsync(L.sync, 0, angmf_iters_sync_bytes(L.B, L.H, L.W), s);
    if (e != cudaSuccess) return e;
    AngmfIters J{};
    J.pn0 = L.pn0;
    for (int i = 0; i < L.iters; ++i) {
        J.prob[i] = L.prob[i];
        J.xy[i] = L.xy[i];
        J.ang[i] = L.angle[i];
    }
    J.buf[0] = L.buf[0];
    J.buf[1] = L.buf[1];
    J.iters = L.iters;
    J.first = L.first;
    J.counter = L.sync;
    J.status = L.sync + 1;
    J.done = L.sync + kSyncHeaderWords;
    kern<<<grid, kThreads, smem, s>>>(L.ray, a, J);
    return cudaGetLastError();
}

template <typename TS, bool ACT>
cudaError_t launch_iters_st(const AngmfItersLaunch& L, cudaStream_t s) {
    if (L.iters < 1 || L.iters > kMaxFusedIters) return cudaErrorNotSupported;
    if ((L.W % Stages<TS, 5>::kEpc) != 0 || (L.dil != 1 && L.dil != 2))
        return cudaErrorNotSupported;
    switch (L.ps * 4 + L.dil) {
        case 3 * 4 + 1: return launch_iters_t<3, 1, TS, ACT>(L, s);
        case 3 * 4 + 2: return launch_iters_t<3, 2, TS, ACT>(L, s);
        case 5 * 4 + 1: return launch_iters_t<5, 1, TS, ACT>(L, s);
        case 5 * 4 + 2: return launch_iters_t<5, 2, TS, ACT>(L, s);
        case 7 * 4 + 1: return launch_iters_t<7, 1, TS, ACT>(L, s);
        case 7 * 4 + 2: return launch_iters_t<7, 2, TS, ACT>(L, s);
        default: return cudaErrorNotSupported;
    }
}

template <bool ACT>
cudaError_t launch_angmf_iters_act(const AngmfItersLaunch& L, cudaStream_t s) {
    if (L.st == SType::F32) return launch_iters_st<float, ACT>(L, s);
    return launch_iters_st<__half, ACT>(L, s);
}

template <int PS, typename TS, typename TNI, typename TNO, bool FUSE_RR, bool ACT>
cudaError_t launch_t(const AngmfLaunch& L, cudaStream_t s) {
    AngmfArgs a = make_args<PS>(L);
    const size_t nsmem = NTile::bytes(kTW + 2 * a.R, kTH + 2 * a.R);
    const long blocks = (long)a.tiles_x * a.tiles_y * L.B;
    if (blocks > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    // staged copies need every 16-byte chunk of a row to start on a 16-byte
    // boundary (W a multiple of 16 bytes of storage); dilations 1 and 2 (the
    // benchmark windows) have compile-time staged variants
    if ((L.W % Stages<TS, PS>::kEpc) == 0 && (L.dil == 1 || L.dil == 2) &&
        a.tiles_y <= 65535) {
        const size_t smem = Stages<TS, PS>::kBytes + nsmem;  // = StagedCfg<...>::kSmem
        auto kern = L.dil == 1 ? angmf_staged_kernel<PS, 1, TS, TNI, TNO, FUSE_RR, ACT>
                               : angmf_staged_kernel<PS, 2, TS, TNI, TNO, FUSE_RR, ACT>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        // grid (tiles_x, tiles_y, frames), frames in launches of at most 65535
        constexpr int P = PS * PS;
        constexpr long kMaxZ = 65535;
        for (long b0 = 0; b0 < L.B; b0 += kMaxZ) {
            const long nb = L.B - b0 < kMaxZ ? L.B - b0 : kMaxZ;
            a.B = (int)nb;
            const dim3 grid((unsigned)a.tiles_x, (unsigned)a.tiles_y, (unsigned)nb);
            e = launch_pdl(kern, grid, dim3(kThreads), smem, s, L.pdl && b0 == 0,
                           static_cast<const TNI*>(L.pn) + b0 * 3 * a.HW,
                           static_cast<const TS*>(L.prob) + b0 * P * a.HW,
                           static_cast<const TS*>(L.xy) + b0 * 2 * P * a.HW,
                           static_cast<const TS*>(L.angle) + b0 * P * a.HW, L.ray,
                           static_cast<TNO*>(L.out) + b0 * 3 * a.HW, a);
            if (e == cudaSuccess) e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    auto kern = angmf_kernel<PS, TS, TNI, TNO, FUSE_RR, ACT>;
    if (nsmem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)nsmem);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = launch_pdl(kern, dim3((unsigned)blocks), dim3(kThreads), nsmem, s, L.pdl,
                               static_cast<const TNI*>(L.pn), static_cast<const TS*>(L.prob),
                               static_cast<const TS*>(L.xy), static_cast<const TS*>(L.angle),
                               L.ray, static_cast<TNO*>(L.out), a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int PS, typename TS, bool ACT>
cudaError_t launch_ps(const AngmfLaunch& L, cudaStream_t s) {
    const bool in_f32 = L.pn_t == SType::F32, out_f32 = L.out_t == SType::F32;
    using TO = TS;
    if (L.fuse_ray_relu) {
        // fused refine, first iteration: storage-typed decoder normals in, fp32 out
        if (!out_f32) return cudaErrorInvalidValue;
        if (in_f32) return launch_t<PS, TS, float, float, true, ACT>(L, s);
        return launch_t<PS, TS, TO, float, true, ACT>(L, s);
    }
    // fused refine, later iterations (fp32 intermediates) or the fp32 single op
    if (in_f32 && out_f32) return launch_t<PS, TS, float, float, false, ACT>(L, s);
    // single op on storage-typed normals
    if (!in_f32 && !out_f32) return launch_t<PS, TS, TO, TO, false, ACT>(L, s);
    return cudaErrorInvalidValue;
}

template <typename TS, bool ACT>
cudaError_t launch_st(const AngmfLaunch& L, cudaStream_t s) {
    switch (L.ps) {
        case 3: return launch_ps<3, TS, ACT>(L, s);
        case 5: return launch_ps<5, TS, ACT>(L, s);
        case 7: return launch_ps<7, TS, ACT>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

// Every AngMF variant with head activations on (ACT) or off.
template <bool ACT>
cudaError_t launch_angmf_act(const AngmfLaunch& L, cudaStream_t s) {
    if (L.B == 0 || L.H == 0 || L.W == 0) return cudaSuccess;
    if (L.st == SType::F32) {
        if (L.pn_t != SType::F32 && !L.fuse_ray_relu) return cudaErrorInvalidValue;
        return launch_st<float, ACT>(L, s);
    }
    return launch_st<__half, ACT>(L, s);
}

}  // namespace
}  // namespace bvml
