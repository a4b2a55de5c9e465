/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the DSINE refine ops.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
 * its `--impl reference` arm) may load this library, and only as the checker
 * or as the timed CPU baseline. The product path (brovisionml_b200, the CUDA
 * kernels behind include/bvml_dsine.h) never calls into it.
 *
 * A plain-C, fp64-math restatement of the reference's algorithm for the path,
 * generalised past what the reference supports:
 *   - window size ps (odd) and dilation dil (the reference is fixed at 5x5,
 *     dilation 1: src/dsine_ops.cpp:24-27);
 *   - the convex 8x upsample + channel L2-normalise + crop that the reference
 *     delegates to the absent brotensor library (called at
 *     src/dsine_refine.cpp:277-292; semantics stated only in the comment at
 *     include/brovisionml/dsine_refine.h:91-97, so that part is UNPINNED);
 *   - get_ray_core / build_ray8 (src/dsine_decoder.cpp:242-290).
 *
 * At (ps=5, dil=1) bb_angmf() and bb_ray_relu() must be BIT-EXACT with the
 * reference CPU twin compiled from src/dsine_ops.cpp (oracle/Makefile builds
 * it into oracle/_ref/); tests/test_oracle.py enforces that. Bit-exactness is
 * why every arithmetic expression below keeps the reference's operation order
 * and its std::max tie/NaN semantics (a < b ? b : a), and why the Makefile
 * builds both with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* std::max(a, b) semantics: returns a unless a < b (so NaN in `a` survives). */
static inline double mx(double a, double b) { return (a < b) ? b : a; }
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static const double kRayEpsF = (double)1e-2f; /* src/dsine_ops.cpp:27 (float 1e-2f) */

/* Quaternion-route axis-angle -> 3x3, src/dsine_ops.cpp:31-51. */
static void aa_to_mat(double ax, double ay, double az, double R[9]) {
    const double angle = sqrt(ax * ax + ay * ay + az * az);
    const double half = angle * 0.5;
    double s;
    if (angle < 1e-6)
        s = 0.5 - (angle * angle) / 48.0;
    else
        s = sin(half) / angle;
    const double r = cos(half);
    const double i = ax * s, j = ay * s, k = az * s;
    const double two_s = 2.0 / (r * r + i * i + j * j + k * k);
    R[0] = 1.0 - two_s * (j * j + k * k);
    R[1] = two_s * (i * j - k * r);
    R[2] = two_s * (i * k + j * r);
    R[3] = two_s * (i * j + k * r);
    R[4] = 1.0 - two_s * (i * i + k * k);
    R[5] = two_s * (j * k - i * r);
    R[6] = two_s * (i * k - j * r);
    R[7] = two_s * (j * k + i * r);
    R[8] = 1.0 - two_s * (i * i + j * j);
}

/* RayReLU of one planar frame in place, src/dsine_ops.cpp:55-76. */
void bb_ray_relu(float* n, const float* r, long HW) {
    for (long p = 0; p < HW; ++p) {
        const double nx = n[p], ny = n[HW + p], nz = n[2 * HW + p];
        const double rx = r[p], ry = r[HW + p], rz = r[2 * HW + p];
        const double nn = sqrt(nx * nx + ny * ny + nz * nz);
        const double rr = sqrt(rx * rx + ry * ry + rz * rz);
        const double denom = mx(nn * rr, 1e-8);
        const double cs = (nx * rx + ny * ry + nz * rz) / denom;
        const double relu_cm = mx(cs - kRayEpsF, 0.0) + kRayEpsF;
        const double dcoef = relu_cm - cs;
        const double m0 = nx + rx * dcoef;
        const double m1 = ny + ry * dcoef;
        const double m2 = nz + rz * dcoef;
        const double inv = 1.0 / mx(sqrt(m0 * m0 + m1 * m1 + m2 * m2), 1e-12);
        n[p] = (float)(m0 * inv);
        n[HW + p] = (float)(m1 * inv);
        n[2 * HW + p] = (float)(m2 * inv);
    }
}

/*
 * One neighbour's contribution (already multiplied by its weight) for output
 * pixel p, following the per-neighbour body of src/dsine_ops.cpp:98-162.
 * Exposed so tests can probe single configurations.
 */
void bb_angmf_neighbor(double nx, double ny, double nz, int sx, int sy,
                       double xs, double ys, double theta, double w,
                       double rx, double ry, double rz,
                       double fu, double cu, double fv, double cv, double out3[3]) {
    const double pix_x = sx + 0.5, pix_y = sy + 0.5;
    const double xyinv = 1.0 / mx(sqrt(xs * xs + ys * ys), 1e-12);
    xs *= xyinv;
    ys *= xyinv;
    const double du_over_fu = xs / fu;
    const double dv_over_fv = ys / fv;
    const double term_u = (pix_x + xs - cu) / fu;
    const double term_v = (pix_y + ys - cv) / fv;
    const double num = -(du_over_fu * nx + dv_over_fv * ny);
    double dd = term_u * nx + term_v * ny + nz;
    if (fabs(dd) < 1e-8) {
        const double sgn = (dd > 0.0) ? 1.0 : (dd < 0.0 ? -1.0 : 0.0);
        dd = 1e-8 * sgn;
    }
    const double dz = num / dd;
    double axx = du_over_fu + dz * term_u;
    double axy = dv_over_fv + dz * term_v;
    double axz = dz;
    const double an = sqrt(axx * axx + axy * axy + axz * axz);
    const double ainv = 1.0 / mx(an, 1e-12);
    axx *= ainv;
    axy *= ainv;
    axz *= ainv;
    if (!isfinite(axx) || !isfinite(axy) || !isfinite(axz)) axx = axy = axz = 0.0;
    double R[9];
    aa_to_mat(axx * theta, axy * theta, axz * theta, R);
    double rnx = R[0] * nx + R[1] * ny + R[2] * nz;
    double rny = R[3] * nx + R[4] * ny + R[5] * nz;
    double rnz = R[6] * nx + R[7] * ny + R[8] * nz;
    const double rinv = 1.0 / mx(sqrt(rnx * rnx + rny * rny + rnz * rnz), 1e-12);
    rnx *= rinv;
    rny *= rinv;
    rnz *= rinv;
    const double nn = sqrt(rnx * rnx + rny * rny + rnz * rnz);
    const double rr = sqrt(rx * rx + ry * ry + rz * rz);
    const double denom = mx(nn * rr, 1e-8);
    const double cs = (rnx * rx + rny * ry + rnz * rz) / denom;
    const double relu_cm = mx(cs - kRayEpsF, 0.0) + kRayEpsF;
    const double dcoef = relu_cm - cs;
    double m0 = rnx + rx * dcoef, m1 = rny + ry * dcoef, m2 = rnz + rz * dcoef;
    const double minv = 1.0 / mx(sqrt(m0 * m0 + m1 * m1 + m2 * m2), 1e-12);
    m0 *= minv;
    m1 *= minv;
    m2 *= minv;
    out3[0] = w * m0;
    out3[1] = w * m1;
    out3[2] = w * m2;
}

/*
 * Fused AngMF propagate for one frame, src/dsine_ops.cpp:78-172, generalised to
 * a ps x ps window at dilation dil. Slot n = ky*ps + kx samples
 * (clamp(y - r*dil + ky*dil), clamp(x - r*dil + kx*dil)), replicate padding.
 * Layouts are planar: pn/rp/out (3,H,W); pr/ap (P,H,W); xy (2P,H,W) with the
 * x offsets in channels [0,P) and the y offsets in [P,2P).
 */
void bb_angmf(const float* pn, const float* pr, const float* xyp, const float* ap,
              const float* rp, double fu, double cu, double fv, double cv,
              int H, int W, int ps, int dil, float* op) {
    const long HW = (long)H * W;
    const int P = ps * ps;
    const int pad = (ps - 1) / 2 * dil;
    for (int y = 0; y < H; ++y) {
        for (int x = 0; x < W; ++x) {
            const long p = (long)y * W + x;
            const double rx = rp[p], ry = rp[HW + p], rz = rp[2 * HW + p];
            double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;
            for (int n = 0; n < P; ++n) {
                const int ky = n / ps, kx = n % ps;
                const int sy = clampi(y - pad + ky * dil, 0, H - 1);
                const int sx = clampi(x - pad + kx * dil, 0, W - 1);
                const long sp = (long)sy * W + sx;
                double c3[3];
                bb_angmf_neighbor(pn[sp], pn[HW + sp], pn[2 * HW + sp], sx, sy,
                                  xyp[(long)n * HW + p], xyp[(long)(P + n) * HW + p],
                                  ap[(long)n * HW + p], pr[(long)n * HW + p],
                                  rx, ry, rz, fu, cu, fv, cv, c3);
                acc0 += c3[0];
                acc1 += c3[1];
                acc2 += c3[2];
            }
            const double inv = 1.0 / mx(sqrt(acc0 * acc0 + acc1 * acc1 + acc2 * acc2), 1e-12);
            op[p] = (float)(acc0 * inv);
            op[HW + p] = (float)(acc1 * inv);
            op[2 * HW + p] = (float)(acc2 * inv);
        }
    }
}

/*
 * Convex upsample (restated from include/brovisionml/dsine_refine.h:91-97):
 * mask (9*s*s, H, W) viewed as (9, s, s, H, W), softmax over the 9 taps
 * (max-subtracted); tap t = ty*3 + tx reads x at (clamp(y+ty-1), clamp(x+tx-1))
 * (replicate pad 1); output (C, s*H, s*W) with row s*y+ky, col s*x+kx.
 */
void bb_convex_upsample(const float* x, const float* mask, int C, int H, int W, int s,
                        float* y) {
    const long HW = (long)H * W;
    const long Ws = (long)W * s;
    const long HWs = (long)H * s * Ws;
    for (int yy = 0; yy < H; ++yy) {
        for (int xx = 0; xx < W; ++xx) {
            const long p = (long)yy * W + xx;
            long sp[9];
            for (int t = 0; t < 9; ++t) {
                const int sy = clampi(yy + t / 3 - 1, 0, H - 1);
                const int sx = clampi(xx + t % 3 - 1, 0, W - 1);
                sp[t] = (long)sy * W + sx;
            }
            for (int ky = 0; ky < s; ++ky) {
                for (int kx = 0; kx < s; ++kx) {
                    double l[9], m = -INFINITY, S = 0.0;
                    for (int t = 0; t < 9; ++t) {
                        l[t] = mask[((long)t * s * s + (long)ky * s + kx) * HW + p];
                        if (l[t] > m) m = l[t];
                    }
                    for (int t = 0; t < 9; ++t) {
                        l[t] = exp(l[t] - m);
                        S += l[t];
                    }
                    for (int c = 0; c < C; ++c) {
                        double a = 0.0;
                        for (int t = 0; t < 9; ++t) a += (l[t] / S) * x[(long)c * HW + sp[t]];
                        y[(long)c * HWs + ((long)yy * s + ky) * Ws + (long)xx * s + kx] = (float)a;
                    }
                }
            }
        }
    }
}

/* Channel L2-normalise x / max(|x|, eps), planar (C, HW); y may alias x. */
void bb_l2_normalize(const float* x, int C, long HW, double eps, float* y) {
    for (long p = 0; p < HW; ++p) {
        double ss = 0.0;
        for (int c = 0; c < C; ++c) {
            const double v = x[(long)c * HW + p];
            ss += v * v;
        }
        const double inv = 1.0 / mx(sqrt(ss), eps);
        for (int c = 0; c < C; ++c) y[(long)c * HW + p] = (float)(x[(long)c * HW + p] * inv);
    }
}

/* Crop planar (C, H, W) at (h0, w0) to (C, Ho, Wo). */
void bb_crop(const float* x, int C, int H, int W, int h0, int w0, int Ho, int Wo, float* y) {
    for (int c = 0; c < C; ++c)
        for (int r = 0; r < Ho; ++r)
            memcpy(y + ((long)c * Ho + r) * Wo, x + ((long)c * H + h0 + r) * W + w0,
                   sizeof(float) * (size_t)Wo);
}

/*
 * get_ray_core + build_ray8 (src/dsine_decoder.cpp:242-290): the (3, Hf, Wf)
 * unit ray for a grid, from pre-"+0.5" intrinsics and the padded full dims.
 */
void bb_build_ray(double fx, double fy, double cx, double cy, int Hf, int Wf,
                  int origH, int origW, float* ray) {
    const double sw = (double)Wf / origW;
    const double sh = (double)Hf / origH;
    const double fu = fx * sw, cu = (cx + 0.5) * sw;
    const double fv = fy * sh, cv = (cy + 0.5) * sh;
    const long HW = (long)Hf * Wf;
    for (int y = 0; y < Hf; ++y) {
        for (int x = 0; x < Wf; ++x) {
            const long i = (long)y * Wf + x;
            const float rxf = (float)(((x + 0.5) - cu) / fu);
            const float ryf = (float)(((y + 0.5) - cv) / fv);
            const double X = rxf, Y = ryf, Z = 1.0;
            const double inv = 1.0 / mx(sqrt(X * X + Y * Y + Z * Z), 1e-12);
            ray[i] = (float)(X * inv);
            ray[HW + i] = (float)(Y * inv);
            ray[2 * HW + i] = (float)(Z * inv);
        }
    }
}

/*
 * The ray from already-scaled grid intrinsics (fu, cu, fv, cv) -- the form the
 * fused device path uses for its analytic ray. Same arithmetic as above with
 * the scaling done by the caller.
 */
void bb_build_ray_scaled(double fu, double cu, double fv, double cv, int Hf, int Wf,
                         float* ray) {
    const long HW = (long)Hf * Wf;
    for (int y = 0; y < Hf; ++y) {
        for (int x = 0; x < Wf; ++x) {
            const long i = (long)y * Wf + x;
            const float rxf = (float)(((x + 0.5) - cu) / fu);
            const float ryf = (float)(((y + 0.5) - cv) / fv);
            const double X = rxf, Y = ryf, Z = 1.0;
            const double inv = 1.0 / mx(sqrt(X * X + Y * Y + Z * Z), 1e-12);
            ray[i] = (float)(X * inv);
            ray[HW + i] = (float)(Y * inv);
            ray[2 * HW + i] = (float)(Z * inv);
        }
    }
}

/*
 * The whole refine-ops unit for ONE frame, in the reference's order
 * (src/dsine_refine.cpp:241-292): ray_relu(normal0, ray8); `iters` AngMF
 * updates; convex upsample x s; L2-normalise (eps 1e-12); optional full-res
 * RayReLU against the full-res ray (intrinsics x s); crop.
 *   normal0 (3,h,w)   ray8 (3,h,w)
 *   prob[i] (P,h,w)   xy[i] (2P,h,w)   angle[i] (P,h,w)  for i < iters
 *   mask (9 s s, h, w)   out (3, out_h, out_w)
 * Returns 0, or -1 on allocation failure.
 */
int bb_refine_unit(const float* normal0, const float* ray8, const float* const* prob,
                   const float* const* xy, const float* const* angle, const float* mask,
                   int h, int w, int iters, int ps, int dil, double fu, double cu,
                   double fv, double cv, int s, int full_res_ray_relu, int crop_t,
                   int crop_l, int out_h, int out_w, float* out) {
    const long HW = (long)h * w;
    const long HWs = HW * s * s;
    float* a = (float*)malloc(sizeof(float) * 3 * HW);
    float* b = (float*)malloc(sizeof(float) * 3 * HW);
    float* up = (float*)malloc(sizeof(float) * 3 * HWs);
    if (!a || !b || !up) {
        free(a); free(b); free(up);
        return -1;
    }
    memcpy(a, normal0, sizeof(float) * 3 * HW);
    bb_ray_relu(a, ray8, HW);
    for (int it = 0; it < iters; ++it) {
        bb_angmf(a, prob[it], xy[it], angle[it], ray8, fu, cu, fv, cv, h, w, ps, dil, b);
        float* t = a; a = b; b = t;
    }
    bb_convex_upsample(a, mask, 3, h, w, s, up);
    bb_l2_normalize(up, 3, HWs, 1e-12, up);
    if (full_res_ray_relu) {
        float* rf = (float*)malloc(sizeof(float) * 3 * HWs);
        if (!rf) {
            free(a); free(b); free(up);
            return -1;
        }
        bb_build_ray_scaled(fu * s, cu * s, fv * s, cv * s, h * s, w * s, rf);
        bb_ray_relu(up, rf, HWs);
        free(rf);
    }
    bb_crop(up, 3, h * s, w * s, crop_t, crop_l, out_h, out_w, out);
    free(a); free(b); free(up);
    return 0;
}
