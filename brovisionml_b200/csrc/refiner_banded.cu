// Large frames for C / C++ hosts: the whole learned refinement of ONE frame,
// from host memory, as exact-halo row bands dealt over one or more refiner
// handles (bvml_refiner_forward_banded), and the halo it needs
// (bvml_refine_halo_rows).
//
// The reference caps the resolution instead (src/dsine.cpp:117-141: a frame
// above the cap is downscaled, refined and upsampled back). Here band k owns
// grid rows [own0, own1) of the frame and computes rows [comp0, comp1), its
// owned rows plus H rows of halo on each side clipped to the frame. H is the
// receptive field of the whole refinement through `iters` iterations, so the
// owned output rows equal the whole-frame refinement: the convolutions' zero
// padding and AngMF's replicate padding act only at the true frame edges, and
// the rows a band edge contaminates are exactly its halo. A band is refined as
// an image of 8 * rows padded rows whose principal point sits 8 * comp0
// pixels higher (the grid intrinsics then follow src/dsine_refine.cpp:230-237
// as for a whole frame), and only its owned rows inside the caller's crop are
// produced and copied out. The same plan as the Python driver
// (brovisionml_b200.pipeline.refine_frame_banded_full).
//
// Each handle gets one host thread (a handle is not used by two threads at
// once) and its own stream; bands go to the handles in turn. A band that fails
// stops the other threads at their next band; every thread is joined and the
// first failure is reported with its band's rows and its device.
#include "bvml_dsine.h"
#include "bvml_internal.h"
#include "trace.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

int fail(int code, const std::string& msg) { return bvml::report_error(code, msg); }

// Grid rows of halo per side for an exact band of the whole refinement, with
// R = (ps / 2) * dil and n = 1 row for the upsample's 3x3: iteration i's
// normals are needed n + (I - i) R rows out, the heads' 3x3 reads the hidden
// state h_i one row further, h_i reads h_(i-1) four rows out (the 5x5 z / r
// convolutions over h, then the 5x5 q convolution over r * h), and the
// decoder's hidden state and feature (through the hoisted 5x5 GRU terms) are
// read need(h_1) + 4 rows out, its normals n + I R rows out.
int halo_rows(int iters, int ps, int dil) {
    const int n = 1, R = (ps / 2) * dil;
    if (iters <= 0) return n;
    int need = n + 1;
    for (int i = iters - 1; i >= 1; --i) need = std::max(n + (iters - i) * R + 1, need + 4);
    return std::max(need + 4, n + iters * R);
}

struct BandPlan {
    int own0, own1, comp0, comp1;   // grid rows
    int out0, out1;                 // rows of the caller's (cropped) output this band fills
};

struct Failure {
    int band = -1, device = -1, code = BVML_OK;
    std::string msg;
};

// Device buffers of one worker, grown to its largest band.
struct Slab {
    float* in = nullptr;   // normal (3), feature (64), hidden (64) planes of a band
    void* out = nullptr;   // the band's (3, rows, out_w) output in the storage type
    size_t in_n = 0, out_n = 0;
    cudaError_t ensure(size_t in_bytes, size_t out_bytes) {
        cudaError_t e = cudaSuccess;
        if (in_bytes > in_n) {
            cudaFree(in);
            in = nullptr;
            in_n = 0;
            if ((e = cudaMalloc(&in, in_bytes)) != cudaSuccess) return e;
            in_n = in_bytes;
        }
        if (out_bytes > out_n) {
            cudaFree(out);
            out = nullptr;
            out_n = 0;
            if ((e = cudaMalloc(&out, out_bytes)) != cudaSuccess) return e;
            out_n = out_bytes;
        }
        return e;
    }
    void release() {
        cudaFree(in);
        cudaFree(out);
        in = nullptr;
        out = nullptr;
    }
};

}  // namespace

extern "C" {

int bvml_refine_halo_rows(int iters, int ps, int dil) {
    if (iters < 0 || iters > 64 || (ps != 3 && ps != 5 && ps != 7) || dil < 1 || dil > 4)
        return fail(BVML_EINVAL, "dsine ops: refine_halo_rows: iters 0..64, window 3/5/7, "
                                 "dilation 1..4");
    return halo_rows(iters, ps, dil);
}

int bvml_refiner_forward_banded(bvml_refiner* const* refiners, int n_refiners,
                                const float* normal, const float* feature, const float* hidden,
                                int h, int w, const float* intrins, int origH, int origW,
                                int iters, int n_bands, int crop_t, int crop_l, int out_h,
                                int out_w, int dtype, void* out) {
    bvml::NvtxRange nvtx("bvml_refiner_forward_banded");
    if (!refiners || n_refiners <= 0 || !normal || !feature || !hidden || !intrins || !out)
        return fail(BVML_EINVAL, "dsine ops: refiner banded: null argument");
    for (int k = 0; k < n_refiners; ++k)
        if (!refiners[k]) return fail(BVML_EINVAL, "dsine ops: refiner banded: null handle");
    if (h <= 0 || w <= 0 || origH <= 0 || origW <= 0 || iters < 1 || iters > 64 || n_bands < 1)
        return fail(BVML_EINVAL, "dsine ops: refiner banded: bad shape, iteration or band count");
    if (dtype != BVML_F32 && dtype != BVML_F16)
        return fail(BVML_EINVAL, "dsine ops: refiner banded: dtype must be F32 or F16");
    if (crop_t < 0 || crop_l < 0 || out_h <= 0 || out_w <= 0 || crop_t + out_h > 8 * h ||
        crop_l + out_w > 8 * w)
        return fail(BVML_EINVAL, "dsine ops: refiner banded: crop window outside the 8x output");

    // balanced owned bands (as sharding.plan_bands), halo clipped to the frame
    const int halo = halo_rows(iters, 5, 1);
    const int nb = std::min(n_bands, h);
    std::vector<BandPlan> plan;
    for (int k = 0, s = 0; k < nb; ++k) {
        const int n = h / nb + (k < h % nb ? 1 : 0);
        BandPlan b;
        b.own0 = s;
        b.own1 = s + n;
        s += n;
        b.comp0 = std::max(0, b.own0 - halo);
        b.comp1 = std::min(h, b.own1 + halo);
        // the band's owned full-resolution rows inside the crop
        const int r0 = std::max(8 * b.own0, crop_t), r1 = std::min(8 * b.own1, crop_t + out_h);
        if (r1 <= r0) continue;  // nothing of this band reaches the output
        b.out0 = r0 - crop_t;
        b.out1 = r1 - crop_t;
        plan.push_back(b);
    }
    const size_t es = dtype == BVML_F16 ? 2 : 4;
    const size_t plane = (size_t)h * w;
    std::atomic<bool> stop{false};
    std::mutex mu;
    Failure first;

    auto work = [&](int d) {
        bvml_refiner* r = refiners[d];
        const int dev = bvml::refiner_device(r);
        Slab slab;
        cudaStream_t s = nullptr;
        auto record = [&](int band, int code, const std::string& msg) {
            std::lock_guard<std::mutex> lk(mu);
            if (first.code == BVML_OK) {
                first.band = band;
                first.device = dev;
                first.code = code;
                first.msg = msg;
            }
            stop = true;
        };
        cudaError_t e = cudaSetDevice(dev);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            record(-1, BVML_ECUDA, std::string("stream: ") + cudaGetErrorString(e));
            return;
        }
        for (size_t k = d; k < plan.size() && !stop; k += (size_t)n_refiners) {
            const BandPlan& b = plan[k];
            const int rows = b.comp1 - b.comp0, orows = b.out1 - b.out0;
            const size_t bplane = (size_t)rows * w;
            auto cuda_err = [&](const char* what) {
                (void)cudaGetLastError();
                record((int)k, BVML_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
            };
            if ((e = slab.ensure(sizeof(float) * bplane * (3 + 64 + 64),
                                 es * 3 * (size_t)orows * out_w)) != cudaSuccess) {
                cuda_err("band buffers");
                break;
            }
            // the band's rows of every plane: one strided copy per tensor
            const struct {
                const float* src;
                int c;
                size_t off;
            } parts[3] = {{normal, 3, 0}, {feature, 64, 3 * bplane}, {hidden, 64, 67 * bplane}};
            for (const auto& p : parts) {
                e = cudaMemcpy2DAsync(slab.in + p.off, sizeof(float) * bplane,
                                      p.src + (size_t)b.comp0 * w, sizeof(float) * plane,
                                      sizeof(float) * bplane, (size_t)p.c, cudaMemcpyHostToDevice,
                                      s);
                if (e != cudaSuccess) break;
            }
            if (e != cudaSuccess) {
                cuda_err("band upload");
                break;
            }
            const float intr_b[4] = {intrins[0], intrins[1], intrins[2],
                                     intrins[3] - 8.0f * (float)b.comp0};
            const int top = b.out0 + crop_t - 8 * b.comp0;  // first output row in the band image
            int rc = bvml_refiner_forward(r, slab.in, slab.in + 3 * bplane, slab.in + 67 * bplane,
                                          1, rows, w, intr_b, 8 * rows, origW, iters, top, crop_l,
                                          orows, out_w, dtype, slab.out, s);
            if (rc == BVML_OK) rc = bvml_refiner_status(r, s);
            if (rc != BVML_OK) {
                record((int)k, rc, bvml_last_error());
                break;
            }
            // the band's rows of each output plane into the caller's frame
            e = cudaMemcpy2DAsync(static_cast<char*>(out) + es * (size_t)b.out0 * out_w,
                                  es * (size_t)out_h * out_w, slab.out, es * (size_t)orows * out_w,
                                  es * (size_t)orows * out_w, 3, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                cuda_err("band download");
                break;
            }
        }
        if (s) cudaStreamSynchronize(s);
        slab.release();
        if (s) cudaStreamDestroy(s);
    };

    int caller_dev = 0;
    if (cudaGetDevice(&caller_dev) != cudaSuccess) caller_dev = -1;
    const int nw = std::min<int>(n_refiners, (int)plan.size());
    std::vector<std::thread> threads;
    try {
        for (int d = 1; d < nw; ++d) threads.emplace_back(work, d);
    } catch (const std::exception& ex) {  // no exception crosses the C ABI
        {
            std::lock_guard<std::mutex> lk(mu);
            if (first.code == BVML_OK) {
                first.code = BVML_EUNSUPPORTED;
                first.msg = std::string("host thread: ") + ex.what();
            }
            stop = true;
        }
    }
    if (nw > 0) work(0);
    for (auto& t : threads) t.join();
    if (caller_dev >= 0) cudaSetDevice(caller_dev);  // work(0) ran on this thread
    if (first.code != BVML_OK) {
        std::string where = first.band < 0 ? std::string("worker")
                                           : "band " + std::to_string(first.band) +
                                                 " (grid rows " +
                                                 std::to_string(plan[first.band].comp0) + ".." +
                                                 std::to_string(plan[first.band].comp1) + ")";
        return fail(first.code, "dsine ops: refiner banded: " + where + " on device " +
                                    std::to_string(first.device) + ": " + first.msg);
    }
    return bvml::report_error(BVML_OK, "");
}

}  // extern "C"
