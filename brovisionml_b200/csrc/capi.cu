// extern "C" entry points of libbvml_dsine.so (declared in include/bvml_dsine.h).
//
// Argument checking and error reporting mirror the reference: argument
// problems read "dsine ops: ..." (src/dsine_ops.cpp:18-22) and CUDA failures
// "dsine cuda: <what>: <cudaGetErrorString>" (src/dsine_ops.cu:25-29), but
// they are returned as status codes with the text in bvml_last_error(), since
// no exception may cross a C ABI.
#include "bvml_dsine.h"
#include "bvml_internal.h"
#include "trace.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdint>
#include <cstdlib>
#include <string>
#include <vector>

namespace {

thread_local std::string g_last_error;
thread_local std::vector<cudaEvent_t> g_probe;
thread_local int g_probe_recorded = 0;

cudaError_t probe(size_t k, cudaStream_t s) {
    if (k >= g_probe.size()) return cudaSuccess;
    g_probe_recorded = (int)k + 1;
    return cudaEventRecord(g_probe[k], s);
}

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}
int einval(const std::string& msg) { return fail(BVML_EINVAL, "dsine ops: " + msg); }
// A failed runtime call (an allocation that did not fit, a bad launch
// configuration) also sets the thread's last-error state; it is read and
// reset here so that the next call's launch checks do not report it again.
// Sticky errors (a lost context) stay, as they must.
int cuda_fail(cudaError_t e, const char* what) {
    (void)cudaGetLastError();
    return fail(BVML_ECUDA, std::string("dsine cuda: ") + what + ": " + cudaGetErrorString(e));
}
int finish(cudaError_t e, const char* what) {
    if (e == cudaErrorInvalidValue)
        return fail(BVML_EUNSUPPORTED, std::string("dsine ops: ") + what +
                                           ": unsupported type / option combination");
    if (e != cudaSuccess) return cuda_fail(e, what);
    g_last_error.clear();
    return BVML_OK;
}

bool dtype_ok(int dtype) { return dtype == BVML_F32 || dtype == BVML_F16; }
bvml::SType st_of(int dtype) { return dtype == BVML_F16 ? bvml::SType::F16 : bvml::SType::F32; }
bool window_ok(int ps, int dil) { return (ps == 3 || ps == 5 || ps == 7) && dil >= 1 && dil <= 4; }
bool dims_ok(int B, int H, int W) {
    if (B < 0 || H < 0 || W < 0) return false;
    // every per-frame plane offset must fit the kernels' index arithmetic
    return (int64_t)H * W * 2 * 49 < (int64_t)INT32_MAX;
}
bool intr_ok(double fu, double fv) { return fu != 0.0 && fv != 0.0 && fu == fu && fv == fv; }
size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// bvml_refine's workspace: the persistent AngMF's sync words, then two fp32
// normal buffers and the ray.
size_t sync_region(int B, int h, int w) { return align256(bvml::angmf_iters_sync_bytes(B, h, w)); }

}  // namespace

int bvml::report_error(int code, const std::string& msg) { return fail(code, msg); }

bool bvml::profile_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("BROVISIONML_PROFILE");
        return v != nullptr && v[0] != '\0' && v[0] != '0';
    }();
    return on;
}

void bvml::profile_mark(cudaStream_t s, const char* name) {
    if (!profile_enabled()) return;
    cudaStreamSynchronize(s);
    using clock = std::chrono::steady_clock;
    static thread_local clock::time_point last = clock::now();
    const clock::time_point now = clock::now();
    if (name)
        std::fprintf(stderr, "[brovisionml-prof] %-28s %9.2f ms\n", name,
                     std::chrono::duration<double, std::milli>(now - last).count());
    last = now;
}

namespace {

// bvml_angmf_propagate and bvml_angmf_propagate_logits (`act`: prob / angle
// are raw head outputs, activated on load).
int angmf_entry(const std::string& name, bool act, const void* pred_norm, const void* prob,
                const void* xy, const void* angle, const float* ray, double fu, double cu,
                double fv, double cv, int B, int H, int W, int ps, int dil, int dtype, void* out,
                void* stream) {
    if (!dtype_ok(dtype)) return einval(name + ": unknown dtype");
    if (!window_ok(ps, dil)) return einval(name + ": window must be 3/5/7, dilation 1..4");
    if (!dims_ok(B, H, W)) return einval(name + ": bad shape");
    if ((long)B * H * W == 0) return finish(cudaSuccess, name.c_str());
    if (!pred_norm || !prob || !xy || !angle || !ray || !out)
        return einval(name + ": null tensor");
    if (out == pred_norm) return einval(name + ": out must not alias pred_norm");
    if (!intr_ok(fu, fv)) return einval(name + ": focal lengths must be nonzero");
    bvml::AngmfLaunch L{};
    L.pn = pred_norm;
    L.prob = prob;
    L.xy = xy;
    L.angle = angle;
    L.ray = ray;
    L.out = out;
    L.st = L.pn_t = L.out_t = st_of(dtype);
    L.fuse_ray_relu = false;
    L.act = act;
    L.B = B;
    L.H = H;
    L.W = W;
    L.ps = ps;
    L.dil = dil;
    L.fu = fu;
    L.cu = cu;
    L.fv = fv;
    L.cv = cv;
    return finish(bvml::launch_angmf(L, static_cast<cudaStream_t>(stream)),
                  (name + " launch").c_str());
}

// bvml_refine and bvml_refine_logits (`act`: the per-iteration prob / angle
// are raw head outputs, activated on load).
int refine_entry(bool act, const void* normal0, const float* ray8, const void* const* prob,
                 const void* const* xy, const void* const* angle, int iters, const void* mask,
                 int B, int h, int w, int ps, int dil, double fu, double cu, double fv,
                 double cv, int full_res_ray_relu, int crop_t, int crop_l, int out_h, int out_w,
                 int dtype, void* workspace, size_t workspace_bytes, void* out, void* stream) {
    if (!dtype_ok(dtype)) return einval("refine: unknown dtype");
    if (!window_ok(ps, dil)) return einval("refine: window must be 3/5/7, dilation 1..4");
    if (!dims_ok(B, h, w)) return einval("refine: bad shape");
    if (iters < 0 || iters > 64) return einval("refine: iters must be in 0..64");
    if (crop_t < 0 || crop_l < 0 || out_h < 0 || out_w < 0 || crop_t + out_h > 8 * h ||
        crop_l + out_w > 8 * w)
        return einval("refine: crop window outside the 8x output");
    if ((long)B * h * w == 0 || (long)out_h * out_w == 0) return finish(cudaSuccess, "refine");
    if (!normal0 || !mask || !out || !workspace) return einval("refine: null tensor");
    if (iters > 0 && (!prob || !xy || !angle)) return einval("refine: null per-iteration arrays");
    for (int i = 0; i < iters; ++i)
        if (!prob[i] || !xy[i] || !angle[i]) return einval("refine: null per-iteration tensor");
    if (!intr_ok(fu, fv)) return einval("refine: focal lengths must be nonzero");
    if (workspace_bytes < bvml_refine_workspace_bytes(B, h, w))
        return einval("refine: workspace too small");
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return einval("refine: workspace must be 256-byte aligned");

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    size_t launch_no = 0;
    g_probe_recorded = 0;
    if (cudaError_t e = probe(launch_no++, s); e != cudaSuccess)
        return cuda_fail(e, "refine: probe event record");
    const size_t nbytes = align256(sizeof(float) * 3 * (size_t)h * w * (size_t)B);
    char* wsb = static_cast<char*>(workspace);
    int* sync = reinterpret_cast<int*>(wsb);
    const size_t s0 = sync_region(B, h, w);
    float* bufa = reinterpret_cast<float*>(wsb + s0);
    float* bufb = reinterpret_cast<float*>(wsb + s0 + nbytes);
    float* rayw = reinterpret_cast<float*>(wsb + s0 + 2 * nbytes);
    const float* ray = ray8;
    if (!ray) {
        cudaError_t e = bvml::launch_build_ray(rayw, h, w, fu, cu, fv, cv, s);
        if (e != cudaSuccess) return cuda_fail(e, "refine: ray launch");
        if ((e = probe(launch_no++, s)) != cudaSuccess)
            return cuda_fail(e, "refine: probe event record");
        ray = rayw;
    }
    const bvml::SType st = st_of(dtype);
    const float* cur = nullptr;
    if (iters == 0) {
        // only the initial RayReLU: copy to fp32 workspace then clamp in place
        if (cudaError_t e = cudaMemsetAsync(sync, 0, sizeof(int) * bvml::kSyncHeaderWords, s);
            e != cudaSuccess)
            return cuda_fail(e, "refine: status reset");
        if (st == bvml::SType::F32) {
            cudaError_t e = cudaMemcpyAsync(bufa, normal0, sizeof(float) * 3 * (size_t)h * w * B,
                                            cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "refine: copy");
        } else {
            return fail(BVML_EUNSUPPORTED, "dsine ops: refine: iters = 0 needs fp32 storage");
        }
        cudaError_t e = bvml::launch_ray_relu(bufa, bvml::SType::F32, ray, B, h, w, s);
        if (e != cudaSuccess) return cuda_fail(e, "refine: ray_relu launch");
        if ((e = probe(launch_no++, s)) != cudaSuccess)
            return cuda_fail(e, "refine: probe event record");
        cur = bufa;
    } else {
        // all iterations in one persistent launch where the shape allows it
        bvml::AngmfItersLaunch J{};
        J.pn0 = normal0;
        J.prob = prob;
        J.xy = xy;
        J.angle = angle;
        J.ray = ray;
        J.buf[0] = bufa;
        J.buf[1] = bufb;
        J.sync = sync;
        J.st = st;
        J.act = act;
        J.iters = iters;
        J.B = B;
        J.H = h;
        J.W = w;
        J.ps = ps;
        J.dil = dil;
        J.fu = fu;
        J.cu = cu;
        J.fv = fv;
        J.cv = cv;
        J.first = 0;
        cudaError_t e = bvml::launch_angmf_iters(J, s);
        if (e == cudaSuccess) {
            if ((e = probe(launch_no++, s)) != cudaSuccess)
                return cuda_fail(e, "refine: probe event record");
            cur = (iters - 1) % 2 == 0 ? bufa : bufb;
        } else if (e != cudaErrorNotSupported) {
            return finish(e, "refine: angmf launch");
        } else {
            // one launch per iteration: no dependency waits, status word zero
            e = cudaMemsetAsync(sync, 0, sizeof(int) * bvml::kSyncHeaderWords, s);
            if (e != cudaSuccess) return cuda_fail(e, "refine: status reset");
        }
    }
    if (iters > 0 && !cur) {
        float* dst = bufa;
        float* other = bufb;
        for (int it = 0; it < iters; ++it) {
            bvml::AngmfLaunch L{};
            L.pn = it == 0 ? normal0 : static_cast<const void*>(cur);
            L.prob = prob[it];
            L.xy = xy[it];
            L.angle = angle[it];
            L.ray = ray;
            L.out = dst;
            L.st = st;
            L.pn_t = it == 0 ? st : bvml::SType::F32;
            L.out_t = bvml::SType::F32;
            L.fuse_ray_relu = it == 0;
            L.act = act;
            // iterations after the first overlap the previous one's tail: their
            // per-neighbour inputs were written before the unit started
            L.pdl = it > 0;
            L.B = B;
            L.H = h;
            L.W = w;
            L.ps = ps;
            L.dil = dil;
            L.fu = fu;
            L.cu = cu;
            L.fv = fv;
            L.cv = cv;
            cudaError_t e = bvml::launch_angmf(L, s);
            if (e != cudaSuccess) return finish(e, "refine: angmf launch");
            if ((e = probe(launch_no++, s)) != cudaSuccess)
                return cuda_fail(e, "refine: probe event record");
            cur = dst;
            float* t = dst;
            dst = other;
            other = t;
        }
    }
    bvml::UpsampleLaunch U{};
    U.n = cur;
    U.mask = mask;
    U.out = out;
    U.st = st;
    U.n_t = bvml::SType::F32;
    U.normalize = true;
    U.ray_relu = full_res_ray_relu != 0;
    U.B = B;
    U.h = h;
    U.w = w;
    U.crop_t = crop_t;
    U.crop_l = crop_l;
    U.out_h = out_h;
    U.out_w = out_w;
    U.fu = fu;
    U.cu = cu;
    U.fv = fv;
    U.cv = cv;
    U.status = sync + 1;
    U.pdl = true;  // its mask was written before the unit started
    cudaError_t e = bvml::launch_upsample(U, s);
    if (e != cudaSuccess) return finish(e, "refine: upsample launch");
    if ((e = probe(launch_no++, s)) != cudaSuccess)
        return cuda_fail(e, "refine: probe event record");
    return finish(cudaSuccess, "refine");
}

}  // namespace

extern "C" {

const char* bvml_last_error(void) { return g_last_error.c_str(); }

int bvml_abi_version(void) { return BVML_ABI_VERSION; }

int bvml_probe_events(void* const* events, int n) {
    if (n < 0 || (n > 0 && !events)) return einval("probe_events: bad event list");
    g_probe.clear();
    for (int i = 0; i < n; ++i) {
        if (!events[i]) {
            g_probe.clear();
            return einval("probe_events: null event handle (create the events first)");
        }
        g_probe.push_back(static_cast<cudaEvent_t>(events[i]));
    }
    g_last_error.clear();
    return BVML_OK;
}

int bvml_ray_relu(void* normal, const float* ray, int B, int H, int W, int dtype, void* stream) {
    bvml::NvtxRange nvtx("bvml_ray_relu");
    if (!dtype_ok(dtype)) return einval("ray_relu: unknown dtype");
    if (!dims_ok(B, H, W)) return einval("ray_relu: bad shape");
    if ((long)B * H * W == 0) return finish(cudaSuccess, "ray_relu");
    if (!normal || !ray) return einval("ray_relu: null tensor");
    return finish(bvml::launch_ray_relu(normal, st_of(dtype), ray, B, H, W,
                                        static_cast<cudaStream_t>(stream)),
                  "ray_relu launch");
}

int bvml_angmf_propagate(const void* pred_norm, const void* prob, const void* xy,
                         const void* angle, const float* ray, double fu, double cu, double fv,
                         double cv, int B, int H, int W, int ps, int dil, int dtype, void* out,
                         void* stream) {
    bvml::NvtxRange nvtx("bvml_angmf_propagate");
    return angmf_entry("angmf_propagate", false, pred_norm, prob, xy, angle, ray, fu, cu, fv,
                       cv, B, H, W, ps, dil, dtype, out, stream);
}

int bvml_angmf_propagate_logits(const void* pred_norm, const void* prob_logits, const void* xy,
                                const void* angle_logits, const float* ray, double fu,
                                double cu, double fv, double cv, int B, int H, int W, int ps,
                                int dil, int dtype, void* out, void* stream) {
    bvml::NvtxRange nvtx("bvml_angmf_propagate_logits");
    return angmf_entry("angmf_propagate_logits", true, pred_norm, prob_logits, xy, angle_logits,
                       ray, fu, cu, fv, cv, B, H, W, ps, dil, dtype, out, stream);
}

int bvml_convex_upsample(const void* x, const void* mask, int N, int C, int H, int W, int scale,
                         int dtype, void* y, void* stream) {
    bvml::NvtxRange nvtx("bvml_convex_upsample");
    if (!dtype_ok(dtype)) return einval("convex_upsample: unknown dtype");
    if (C != 3 || scale != 8)
        return fail(BVML_EUNSUPPORTED, "dsine ops: convex_upsample: only C = 3, scale = 8");
    if (!dims_ok(N, H, W)) return einval("convex_upsample: bad shape");
    if ((long)N * H * W == 0) return finish(cudaSuccess, "convex_upsample");
    if (!x || !mask || !y) return einval("convex_upsample: null tensor");
    bvml::UpsampleLaunch L{};
    L.n = x;
    L.mask = mask;
    L.out = y;
    L.st = L.n_t = st_of(dtype);
    L.normalize = false;
    L.ray_relu = false;
    L.B = N;
    L.h = H;
    L.w = W;
    L.crop_t = 0;
    L.crop_l = 0;
    L.out_h = 8 * H;
    L.out_w = 8 * W;
    L.fu = L.fv = 1.0;
    return finish(bvml::launch_upsample(L, static_cast<cudaStream_t>(stream)),
                  "convex_upsample launch");
}

int bvml_l2_normalize_nchw(const void* x, int N, int C, int H, int W, float eps, int dtype,
                           void* y, void* stream) {
    bvml::NvtxRange nvtx("bvml_l2_normalize_nchw");
    if (!dtype_ok(dtype)) return einval("l2_normalize: unknown dtype");
    if (C < 0 || C > 16) return fail(BVML_EUNSUPPORTED, "dsine ops: l2_normalize: C must be <= 16");
    if (N < 0 || H < 0 || W < 0) return einval("l2_normalize: bad shape");
    if ((long)N * C * H * W == 0) return finish(cudaSuccess, "l2_normalize");
    if (!x || !y) return einval("l2_normalize: null tensor");
    return finish(bvml::launch_l2_normalize(x, y, st_of(dtype), N, C, H, W, eps,
                                            static_cast<cudaStream_t>(stream)),
                  "l2_normalize launch");
}

int bvml_slice2d(const void* x, int N, int C, int H, int W, int h0, int w0, int Ho, int Wo,
                 int dtype, void* y, void* stream) {
    bvml::NvtxRange nvtx("bvml_slice2d");
    if (!dtype_ok(dtype)) return einval("slice2d: unknown dtype");
    if (N < 0 || C < 0 || H < 0 || W < 0 || Ho < 0 || Wo < 0 || h0 < 0 || w0 < 0 ||
        h0 + Ho > H || w0 + Wo > W)
        return einval("slice2d: window outside the input");
    if ((long)N * C * Ho * Wo == 0) return finish(cudaSuccess, "slice2d");
    if (!x || !y) return einval("slice2d: null tensor");
    return finish(bvml::launch_slice2d(x, y, st_of(dtype), N, C, H, W, h0, w0, Ho, Wo,
                                       static_cast<cudaStream_t>(stream)),
                  "slice2d launch");
}

int bvml_conv2d_nhwc_f16(const void* x, const void* w, const float* bias, int B, int H, int W,
                          int cin_pad, int cout, int cout_pad, int ks, int act, void* y,
                          int* err, void* stream) {
    bvml::NvtxRange nvtx("bvml_conv2d_nhwc_f16");
    if (!(ks == 1 || ks == 3 || ks == 5)) return einval("conv2d: kernel size must be 1, 3 or 5");
    if (act < 0 || act > 3) return einval("conv2d: unknown activation");
    if (B < 0 || H < 0 || W < 0 || cin_pad <= 0 || cin_pad % 64 != 0 || cout_pad <= 0 ||
        cout_pad % 64 != 0 || cout <= 0 || cout > cout_pad)
        return einval("conv2d: channel counts must be positive, padded to multiples of 64");
    if ((int64_t)B * H * W > INT32_MAX / 2) return einval("conv2d: too many pixels");
    if ((long)B * H * W == 0) return finish(cudaSuccess, "conv2d");
    if (!x || !w || !bias || !y || !err) return einval("conv2d: null tensor");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) |
         reinterpret_cast<uintptr_t>(y)) & 15)
        return einval("conv2d: tensors must be 16-byte aligned");
    bvml::ConvLaunch L{};
    L.x = x;
    L.w = w;
    L.bias = bias;
    L.y = y;
    L.err = err;
    L.B = B;
    L.H = H;
    L.W = W;
    L.x_c = cin_pad;
    L.cin_off = 0;
    L.cin_pad = cin_pad;
    L.cout = cout;
    L.cout_pad = cout_pad;
    L.ks = ks;
    L.epi = bvml::ConvEpi::NHWC;
    L.act = act;
    L.out_c = cout_pad;
    L.out_off = 0;
    return finish(bvml::launch_conv_tc(L, static_cast<cudaStream_t>(stream)), "conv2d launch");
}

int bvml_conv2d_nhwc_f16_ex(const void* x, int x_c, int cin_off, int cin_pad, const void* w,
                             const float* bias, int B, int H, int W, int cout, int cout_pad,
                             int ks, const bvml_conv_epilogue* epi, int* err, void* stream) {
    bvml::NvtxRange nvtx("bvml_conv2d_nhwc_f16_ex");
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!(ks == 1 || ks == 3 || ks == 5)) return einval("conv2d: kernel size must be 1, 3 or 5");
    if (!epi || epi->mode < 0 || epi->mode > 6) return einval("conv2d: unknown epilogue");
    if (B < 0 || H < 0 || W < 0 || x_c <= 0 || x_c % 8 != 0 || cin_off < 0 ||
        cin_off % 64 != 0 || cin_pad <= 0 || cin_pad % 64 != 0 || cin_off + cin_pad > x_c + 63 ||
        cout <= 0 || cout_pad % 64 != 0 || cout > cout_pad)
        return einval("conv2d: bad channel layout");
    if ((int64_t)B * H * W > INT32_MAX / 2) return einval("conv2d: too many pixels");
    if ((long)B * H * W == 0) return finish(cudaSuccess, "conv2d");
    if (!x || !w || !bias || !err || !a16(x) || !a16(w))
        return einval("conv2d: null or unaligned tensor");
    bvml::ConvLaunch L{};
    L.x = x;
    L.w = w;
    L.bias = bias;
    L.err = err;
    L.B = B;
    L.H = H;
    L.W = W;
    L.x_c = x_c;
    L.cin_off = cin_off;
    L.cin_pad = cin_pad;
    L.cout = cout;
    L.cout_pad = cout_pad;
    L.ks = ks;
    L.epi = static_cast<bvml::ConvEpi>(epi->mode);
    L.act = epi->act;
    L.y = epi->out;
    L.out_c = epi->out_c;
    L.out_off = epi->out_off;
    L.h32 = epi->h32;
    L.z = epi->z;
    L.rh = epi->rh;
    L.rh_c = epi->rh_c;
    L.hx = epi->hx;
    L.hx_c = epi->hx_c;
    L.hin = epi->hin;
    L.hin_c = epi->hin_c;
    L.add = epi->add;
    L.add_c = epi->add_c;
    L.add_shared = epi->add_shared;
    if (epi->add && (!a16(epi->add) || epi->add_c % 4 || epi->add_c < cout))
        return einval("conv2d: addend must be 16-byte aligned, add_c a multiple of 4 and >= cout");
    if (epi->add && (epi->mode == BVML_EPI_GRU_ZR || epi->mode == BVML_EPI_GRU_Q))
        return einval("conv2d: the GRU epilogues take no addend (use the extra K block)");
    L.xin = epi->xin;
    L.xin_c = epi->xin_c;
    L.wx = epi->wx;
    L.xin_stride = epi->xin_stride;
    L.wait_limit = epi->wait_limit;
    if (epi->xin && (!epi->wx || !a16(epi->xin) || !a16(epi->wx) || epi->xin_c <= 0 ||
                     epi->xin_c % 64 || epi->xin_stride < 0 || epi->xin_stride % 8 ||
                     (epi->xin_stride && epi->xin_stride < epi->xin_c)))
        return einval("conv2d: extra K needs xin and wx, 16-byte aligned, xin_c a positive "
                      "multiple of 64, xin_stride 0 or a multiple of 8 >= xin_c");
    switch (epi->mode) {
        case BVML_EPI_NHWC:
            if (epi->act < 0 || epi->act > 3) return einval("conv2d: unknown activation");
            if (!epi->out || !a16(epi->out) || epi->out_c % 8 || epi->out_off % 8 ||
                epi->out_off + cout_pad > epi->out_c)
                return einval("conv2d: bad NHWC output");
            break;
        case BVML_EPI_SPLIT_F16:
            if (cout % 32 || !epi->out || !a16(epi->out) || epi->out_c % 8 ||
                epi->out_off % 8 || epi->out_off + 2 * cout_pad > epi->out_c)
                return einval("conv2d: split fp16 output needs cout a multiple of 32 and "
                              "out_c >= out_off + 2 cout_pad");
            break;
        case BVML_EPI_C4_F32:
            if (epi->act < 0 || epi->act > 1)
                return einval("conv2d: fp32 C4 output takes no activation or ReLU");
            if (!epi->out || !a16(epi->out) || epi->out_c % 4 || epi->out_off % 4 ||
                epi->out_off + cout_pad > epi->out_c)
                return einval("conv2d: bad C4 fp32 output");
            break;
        case BVML_EPI_PLANAR_F16:
        case BVML_EPI_PLANAR_F32:
            if (!epi->out || !a16(epi->out)) return einval("conv2d: null or unaligned planar output");
            break;
        case BVML_EPI_GRU_ZR:
            if (cout != 128 || !epi->h32 || !epi->z || !epi->rh || !a16(epi->h32) ||
                !a16(epi->z) || !a16(epi->rh) || epi->rh_c % 8 || epi->rh_c < 64)
                return einval("conv2d: GRU z/r epilogue needs cout 128, h32, z and rh");
            break;
        case BVML_EPI_GRU_Q:
            if (cout != 64 || !epi->h32 || !epi->z || !epi->hx || !a16(epi->h32) ||
                !a16(epi->z) || !a16(epi->hx) || epi->hx_c % 8 || epi->hx_c < 64 ||
                (epi->hin && (!a16(epi->hin) || epi->hin_c % 8 || epi->hin_c < 64)))
                return einval("conv2d: GRU q epilogue needs cout 64, h32, z and hx");
            break;
    }
    return finish(bvml::launch_conv_tc(L, static_cast<cudaStream_t>(stream)), "conv2d launch");
}

int bvml_head_tail_1x1(const void* x, int x_c, int cin_off, const void* w2, const float* b2,
                       const void* w4, const float* b4, int B, int H, int W, int cout,
                       int dtype, void* out, int* err, void* stream) {
    bvml::NvtxRange nvtx("bvml_head_tail_1x1");
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (B < 0 || H < 0 || W < 0 || cout <= 0 || cout > 64 || x_c % 8 || cin_off < 0 ||
        cin_off % 64 || cin_off + 128 > x_c)
        return einval("head tail: bad shape (cout 1..64, 128 input channels at a multiple of "
                      "64 within x_c)");
    if (dtype != BVML_F32 && dtype != BVML_F16) return einval("head tail: dtype must be F32 or F16");
    if ((long)B * H * W == 0) return finish(cudaSuccess, "head tail");
    if ((int64_t)B * H * W > INT32_MAX / 2) return einval("head tail: too many pixels");
    if (!x || !w2 || !b2 || !w4 || !b4 || !out || !err || !a16(x) || !a16(w2) || !a16(w4) ||
        !a16(out))
        return einval("head tail: null or unaligned tensor");
    bvml::HeadTailLaunch L{};
    L.x = x;
    L.x_c = x_c;
    L.cin_off = cin_off;
    L.w2 = w2;
    L.b2 = b2;
    L.w4 = w4;
    L.b4 = b4;
    L.B = B;
    L.H = H;
    L.W = W;
    L.cout = cout;
    L.f16 = dtype == BVML_F16;
    L.y = out;
    L.err = err;
    return finish(bvml::launch_head_tail(L, static_cast<cudaStream_t>(stream)), "head tail launch");
}

int bvml_stage_inputs(const float* h0, const float* feat, int B, int H, int W, float* h32,
                      void* hx, void* fx, void* stream) {
    bvml::NvtxRange nvtx("bvml_stage_inputs");
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (B < 0 || H < 0 || W < 0) return einval("stage inputs: negative size");
    if ((long)B * H * W == 0) return finish(cudaSuccess, "stage inputs");
    if (!h0 || !h32 || !hx || !a16(h32) || !a16(hx) || (!feat) != (!fx) || (fx && !a16(fx)))
        return einval("stage inputs: null or unaligned tensor (feat and fx go together)");
    return finish(bvml::launch_stage_inputs(h0, feat, B, H, W, h32, hx, fx,
                                            static_cast<cudaStream_t>(stream)),
                  "stage inputs");
}

size_t bvml_refine_workspace_bytes(int B, int h, int w) {
    if (B < 0 || h < 0 || w < 0) return 0;
    const size_t plane = (size_t)h * (size_t)w;
    return sync_region(B, h, w) + 2 * align256(sizeof(float) * 3 * plane * (size_t)B) +
           align256(sizeof(float) * 3 * plane);
}

int bvml_refine_status(const void* workspace, void* stream) {
    if (!workspace) return einval("refine_status: null workspace");
    int st = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&st, static_cast<const int*>(workspace) + 1, sizeof(int),
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "refine_status: copy");
    if (st != 0) {
        std::string what;
        if (st & 1) what += "a persistent AngMF dependency wait";
        if (st & 2) what += std::string(what.empty() ? "" : " and ") + "an upsample staging wait";
        if (what.empty()) what = "a device-side wait";
        return fail(BVML_ECUDA, "dsine cuda: refine: " + what + " gave up (status " +
                                    std::to_string(st) + "); results unspecified");
    }
    g_last_error.clear();
    return BVML_OK;
}

unsigned bvml_upsample_wait_limit(unsigned limit) {
    return bvml::set_upsample_wait_limit(limit);
}

int bvml_probe_recorded(void) { return g_probe_recorded; }

int bvml_check_word(int reset) {
#ifdef BVML_CHECKED
    const bool r = reset != 0;
    const unsigned v = bvml::check_word_angmf(r) | bvml::check_word_angmf_logits(r) |
                       bvml::check_word_upsample(r) | bvml::check_word_conv(r);
    return (int)(v & 0x7fffffffu) | (v >> 31 ? (int)0x40000000 : 0);
#else
    (void)reset;
    return -1;
#endif
}

int bvml_refine(const void* normal0, const float* ray8, const void* const* prob,
                const void* const* xy, const void* const* angle, int iters, const void* mask,
                int B, int h, int w, int ps, int dil, double fu, double cu, double fv, double cv,
                int full_res_ray_relu, int crop_t, int crop_l, int out_h, int out_w, int dtype,
                void* workspace, size_t workspace_bytes, void* out, void* stream) {
    bvml::NvtxRange nvtx("bvml_refine");
    return refine_entry(false, normal0, ray8, prob, xy, angle, iters, mask, B, h, w, ps, dil, fu,
                        cu, fv, cv, full_res_ray_relu, crop_t, crop_l, out_h, out_w, dtype,
                        workspace, workspace_bytes, out, stream);
}

int bvml_refine_logits(const void* normal0, const float* ray8, const void* const* prob_logits,
                       const void* const* xy, const void* const* angle_logits, int iters,
                       const void* mask, int B, int h, int w, int ps, int dil, double fu,
                       double cu, double fv, double cv, int full_res_ray_relu, int crop_t,
                       int crop_l, int out_h, int out_w, int dtype, void* workspace,
                       size_t workspace_bytes, void* out, void* stream) {
    bvml::NvtxRange nvtx("bvml_refine_logits");
    return refine_entry(true, normal0, ray8, prob_logits, xy, angle_logits, iters, mask, B, h, w,
                        ps, dil, fu, cu, fv, cv, full_res_ray_relu, crop_t, crop_l, out_h, out_w,
                        dtype, workspace, workspace_bytes, out, stream);
}

}  // extern "C"
