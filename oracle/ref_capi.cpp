// TEST INFRASTRUCTURE ONLY -- extern "C" doors into the reference's own CPU
// twin of the DSINE ops.
//
// oracle/Makefile compiles the READ-ONLY reference source src/dsine_ops.cpp
// (wlejon/brovisionml) in place, together with this file and the host-only
// tensor stand-in under oracle/shim/, into oracle/_ref/libbvml_ref.so. Only
// tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
// `--impl reference` arm) load it.
//
// Entry points:
//   bvml_ref_ray_relu  -> brovisionml::dsine::ray_relu        (dsine_ops.cpp:178-192)
//   bvml_ref_angmf     -> brovisionml::dsine::angmf_propagate (dsine_ops.cpp:194-215)
//   bvml_ref_unit_mt   -> the refine-ops unit (dsine_refine.cpp:241-292) for a
//                         batch of frames, frames split over host threads. The
//                         convex upsample / L2 / crop steps are brotensor ops in
//                         the reference and brotensor is not available, so
//                         those steps use the oracle restatement
//                         (dsine_oracle.c), linked into the same library.
#include "brovisionml/dsine_ops.h"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

extern "C" {
void bb_convex_upsample(const float* x, const float* mask, int C, int H, int W, int s,
                        float* y);
void bb_l2_normalize(const float* x, int C, long HW, double eps, float* y);
void bb_crop(const float* x, int C, int H, int W, int h0, int w0, int Ho, int Wo, float* y);
void bb_build_ray_scaled(double fu, double cu, double fv, double cv, int Hf, int Wf,
                         float* ray);
void bb_ray_relu(float* n, const float* r, long HW);
}

using brotensor::Tensor;

extern "C" int bvml_ref_ray_relu(float* normal, const float* ray, int H, int W) {
    try {
        const int HW = H * W;
        Tensor n = Tensor::view(normal, 1, 3 * HW);
        Tensor r = Tensor::view(const_cast<float*>(ray), 1, 3 * HW);
        brovisionml::dsine::ray_relu(n, r, H, W);
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

extern "C" int bvml_ref_angmf(const float* pred_norm, const float* prob, const float* xy,
                              const float* angle, const float* ray, double fu, double cu,
                              double fv, double cv, int H, int W, float* out) {
    try {
        const int HW = H * W;
        Tensor pn = Tensor::view(const_cast<float*>(pred_norm), 1, 3 * HW);
        Tensor pr = Tensor::view(const_cast<float*>(prob), 1, 25 * HW);
        Tensor x = Tensor::view(const_cast<float*>(xy), 1, 50 * HW);
        Tensor a = Tensor::view(const_cast<float*>(angle), 1, 25 * HW);
        Tensor r = Tensor::view(const_cast<float*>(ray), 1, 3 * HW);
        Tensor o;
        brovisionml::dsine::angmf_propagate(pn, pr, x, a, r, fu, cu, fv, cv, H, W, o);
        std::memcpy(out, o.host_f32(), sizeof(float) * 3 * static_cast<std::size_t>(HW));
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// One frame of the unit through the reference twin (5x5, dilation 1 only).
static int ref_unit_frame(const float* normal0, const float* ray8, const float* const* prob,
                          const float* const* xy, const float* const* angle,
                          const float* mask, int h, int w, int iters, double fu, double cu,
                          double fv, double cv, int full_res_ray_relu, int crop_t,
                          int crop_l, int out_h, int out_w, float* out) {
    const int HW = h * w;
    const int s = 8;
    const long HWs = static_cast<long>(HW) * s * s;
    Tensor pn = Tensor::mat(1, 3 * HW);
    std::memcpy(pn.host_f32_mut(), normal0, sizeof(float) * 3 * static_cast<std::size_t>(HW));
    Tensor r = Tensor::view(const_cast<float*>(ray8), 1, 3 * HW);
    brovisionml::dsine::ray_relu(pn, r, h, w);
    for (int it = 0; it < iters; ++it) {
        Tensor pr = Tensor::view(const_cast<float*>(prob[it]), 1, 25 * HW);
        Tensor x = Tensor::view(const_cast<float*>(xy[it]), 1, 50 * HW);
        Tensor a = Tensor::view(const_cast<float*>(angle[it]), 1, 25 * HW);
        Tensor o;
        brovisionml::dsine::angmf_propagate(pn, pr, x, a, r, fu, cu, fv, cv, h, w, o);
        pn = o;
    }
    std::vector<float> up(static_cast<std::size_t>(3 * HWs));
    bb_convex_upsample(pn.host_f32(), mask, 3, h, w, s, up.data());
    bb_l2_normalize(up.data(), 3, HWs, 1e-12, up.data());
    if (full_res_ray_relu) {
        std::vector<float> rf(static_cast<std::size_t>(3 * HWs));
        bb_build_ray_scaled(fu * s, cu * s, fv * s, cv * s, h * s, w * s, rf.data());
        bb_ray_relu(up.data(), rf.data(), HWs);
    }
    bb_crop(up.data(), 3, h * s, w * s, crop_t, crop_l, out_h, out_w, out);
    return 0;
}

// The unit for `frames` frames, split over `threads` host threads
// (0 = hardware_concurrency). Inputs hold `src_frames` frames laid out
// (B, C, h, w) back to back and frame b reads input frame b % src_frames (a
// timing sample can repeat a few distinct frames); prob/xy/angle are arrays
// of `iters` pointers to whole-batch buffers; `out` holds `frames` frames.
// Returns the thread count used, or -1 on failure.
extern "C" int bvml_ref_unit_mt(const float* normal0, const float* ray8,
                                const float* const* prob, const float* const* xy,
                                const float* const* angle, const float* mask, int frames,
                                int src_frames, int h, int w, int iters, double fu, double cu,
                                double fv,
                                double cv, int full_res_ray_relu, int crop_t, int crop_l,
                                int out_h, int out_w, float* out, int threads) {
    if (iters > 16 || frames <= 0 || src_frames <= 0) return -1;
    int nt = threads > 0 ? threads : static_cast<int>(std::thread::hardware_concurrency());
    nt = std::max(1, std::min(nt, frames));
    const long HW = static_cast<long>(h) * w;
    std::atomic<int> next{0};
    std::atomic<int> failed{0};
    auto worker = [&]() {
        for (;;) {
            const int fb = next.fetch_add(1);
            if (fb >= frames) return;
            const int b = fb % src_frames;
            const float* pb[16];
            const float* xb[16];
            const float* ab[16];
            for (int i = 0; i < iters; ++i) {
                pb[i] = prob[i] + static_cast<long>(b) * 25 * HW;
                xb[i] = xy[i] + static_cast<long>(b) * 50 * HW;
                ab[i] = angle[i] + static_cast<long>(b) * 25 * HW;
            }
            try {
                ref_unit_frame(normal0 + static_cast<long>(b) * 3 * HW, ray8, pb, xb, ab,
                               mask + static_cast<long>(b) * 576 * HW, h, w, iters, fu, cu,
                               fv, cv, full_res_ray_relu, crop_t, crop_l, out_h, out_w,
                               out + static_cast<long>(fb) * 3 * out_h * out_w);
            } catch (const std::exception&) {
                failed.store(1);
                return;
            }
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < nt; ++t) pool.emplace_back(worker);
    worker();
    for (auto& t : pool) t.join();
    return failed.load() ? -1 : nt;
}
