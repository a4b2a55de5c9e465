/* Sanitizer run of the oracle's C restatement (oracle/dsine_oracle.c): the
 * whole refine unit and its pieces on odd and degenerate shapes, every window
 * and dilation, crops and the full-resolution RayReLU, with seeded inputs.
 * Built with -fsanitize=address,undefined by tests/test_oracle_sanitize.py;
 * any out-of-bounds access, leak or undefined behaviour fails the run.
 * Prints one checksum per case (so the work is not optimised away). */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

int bb_refine_unit(const float* normal0, const float* ray8, const float* const* prob,
                   const float* const* xy, const float* const* angle, const float* mask,
                   int h, int w, int iters, int ps, int dil, double fu, double cu, double fv,
                   double cv, int s, int full_res_ray_relu, int crop_t, int crop_l, int out_h,
                   int out_w, float* out);

static uint64_t g_state = 0x9E3779B97F4A7C15ull;
static double uni(void) { /* splitmix64 -> [0, 1) */
    uint64_t z = (g_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}
static float* alloc_fill(long n, double lo, double hi) {
    float* p = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (long i = 0; i < n; ++i) p[i] = (float)(lo + (hi - lo) * uni());
    return p;
}

static int run_case(int h, int w, int ps, int dil, int iters, int rr, int crop) {
    const long HW = (long)h * w;
    const int P = ps * ps, s = 8;
    float* n0 = alloc_fill(3 * HW, -1.0, 1.0);
    float* ray = alloc_fill(3 * HW, -0.5, 0.5);
    for (long i = 0; i < HW; ++i) ray[2 * HW + i] = 1.0f;
    float** prob = (float**)malloc(sizeof(float*) * (size_t)iters);
    float** xy = (float**)malloc(sizeof(float*) * (size_t)iters);
    float** ang = (float**)malloc(sizeof(float*) * (size_t)iters);
    for (int i = 0; i < iters; ++i) {
        prob[i] = alloc_fill(P * HW, 0.0, 1.0);
        xy[i] = alloc_fill(2 * P * HW, -2.0, 2.0);
        ang[i] = alloc_fill(P * HW, 0.0, 3.14);
        /* degenerate entries: zero offsets, zero weights, angle 0 */
        if (HW > 0) {
            xy[i][0] = 0.0f;
            xy[i][(long)P * HW] = 0.0f;
            prob[i][HW - 1] = 0.0f;
            ang[i][0] = 0.0f;
        }
    }
    float* mask = alloc_fill(576 * HW, -3.0, 3.0);
    const int ct = crop ? (8 * h) / 3 : 0, cl = crop ? (8 * w) / 4 : 0;
    const int oh = crop ? 8 * h - ct - 1 : 8 * h, ow = crop ? 8 * w - cl - 2 : 8 * w;
    float* out = (float*)malloc(sizeof(float) * (size_t)(3L * (oh > 0 ? oh : 1) * (ow > 0 ? ow : 1)));
    const int rc = bb_refine_unit(n0, ray, (const float* const*)prob, (const float* const*)xy,
                                  (const float* const*)ang, mask, h, w, iters, ps, dil,
                                  0.8 * w + 0.3, w / 2.0 + 0.06, 0.8 * h + 0.7, h / 2.0 + 0.06,
                                  s, rr, ct, cl, oh, ow, out);
    double sum = 0.0;
    for (long i = 0; i < 3L * oh * ow; ++i) sum += out[i];
    printf("case h=%d w=%d ps=%d dil=%d iters=%d rr=%d crop=%d rc=%d sum=%.6g\n", h, w, ps,
           dil, iters, rr, crop, rc, sum);
    for (int i = 0; i < iters; ++i) {
        free(prob[i]);
        free(xy[i]);
        free(ang[i]);
    }
    free(prob);
    free(xy);
    free(ang);
    free(n0);
    free(ray);
    free(mask);
    free(out);
    return rc;
}

int main(void) {
    static const int shapes[][2] = {{1, 1}, {1, 7}, {7, 1}, {5, 13}, {13, 5}, {9, 16}};
    static const int windows[][2] = {{3, 1}, {5, 1}, {5, 2}, {7, 1}, {7, 2}, {3, 4}};
    int bad = 0;
    for (size_t i = 0; i < sizeof(shapes) / sizeof(shapes[0]); ++i)
        for (size_t j = 0; j < sizeof(windows) / sizeof(windows[0]); ++j)
            bad |= run_case(shapes[i][0], shapes[i][1], windows[j][0], windows[j][1], 2,
                            (int)((i + j) & 1), (int)(j & 1)) != 0;
    return bad;
}
