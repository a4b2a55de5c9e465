// bvml_refiner_*: the whole learned refinement of Refiner::forward
// (src/dsine_refine.cpp:212-294) behind a C ABI, for C and C++ hosts that run
// no Python: the ConvGRU and the four prediction heads on the tensor cores for
// `iters` iterations, then the fused refine ops on the heads' raw outputs.
//
// bvml_refiner_create packs the reference's fp32 OIHW weights once into the
// tensor-core layouts (fp16, [tap][C_out_pad][C_in_pad], the hidden-state
// part of each GRU / head convolution apart from its fixed feature / uv
// part); bvml_refiner_forward runs, on the caller's stream,
//   uv from the intrinsics (the reference's +0.5 convention, double math
//   rounded to float, src/dsine_decoder.cpp:242-275), the stage inputs,
//   the three hoisted convolutions of the fixed inputs, per iteration the
//   z/r and q convolutions with the GRU gates fused, the heads' shared 3x3
//   layer, the prob / xy / angle head tails and (last iteration only) the
//   up-mask head, then bvml_refine_logits,
// the same sequence, packing and launches as the Python RefineStage /
// Refiner (brovisionml_b200/refine_stage.py, refiner.py), so the two give
// bit-identical results. Buffers are allocated on the first forward of a
// shape and reused.
#include "bvml_dsine.h"
#include "bvml_internal.h"
#include "trace.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

namespace {

constexpr int kHidden = 64, kFeature = 64, kHeadHidden = 128;
constexpr int kHeadOut[4] = {25, 50, 25, 576};  // prob, xy, angle, up-mask heads
constexpr const char* kHeadName[4] = {"prob_head", "xy_head", "angle_head", "up_prob_head"};

int fail(int code, const std::string& msg) { return bvml::report_error(code, msg); }
// Resets the thread's last-error state like capi.cu's cuda_fail, so that a
// failed allocation does not resurface in the next forward's launch checks.
int cuda_fail(cudaError_t e, const char* what) {
    (void)cudaGetLastError();
    return fail(BVML_ECUDA, std::string("dsine cuda: refiner: ") + what + ": " +
                                cudaGetErrorString(e));
}
int pad64(int c) { return (c + 63) / 64 * 64; }

// uv of one frame written as channels 0 and 1 of the (h, w, 64) fp16 stage
// input (the other 62 channels zero): u = (x + 0.5 - cu) / fu, v likewise.
__global__ void uv_kernel(__half* ux, int h, int w, double fu, double cu, double fv, double cv) {
    const long n = (long)h * w * 64;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int c = (int)(i % 64);
        const long p = i / 64;
        const int x = (int)(p % w), y = (int)(p / w);
        float v = 0.0f;
        if (c == 0) v = (float)(((double)x + 0.5 - cu) / fu);
        if (c == 1) v = (float)(((double)y + 0.5 - cv) / fv);
        ux[i] = __float2half_rn(v);
    }
}

__global__ void to_half_kernel(const float* __restrict__ x, __half* __restrict__ y, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x)
        y[i] = __float2half_rn(x[i]);
}

struct DevBuf {
    void* p = nullptr;
    size_t n = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= n && p) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
        if (e == cudaSuccess) n = bytes;
        return e;
    }
    template <typename T> T* as() const { return static_cast<T*>(p); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

}  // namespace

struct bvml_refiner {
    int device = 0;
    // packed weights (fp16) and biases (fp32)
    DevBuf w_zr, b_zr, w_q, b_q, w_c0, b_c0, w_c0_3, w_gx, w_gxu, w_gu, iz, iq, zeros;
    DevBuf w_c2[4], b_c2[4], w_c4[4], b_c4[4];
    // per-shape buffers
    int B = 0, h = 0, w = 0, iters = 0, dtype = -1;
    DevBuf hx, rhx, z, h32, fx, ux, gx, gxu, gu, t1, t2, err, n16, ws;
    DevBuf prob, xy, angle, mask;
    ~bvml_refiner() {
        DevBuf* all[] = {&w_zr, &b_zr, &w_q, &b_q, &w_c0, &b_c0, &w_c0_3, &w_gx, &w_gxu, &w_gu,
                         &iz, &iq, &zeros, &hx, &rhx, &z, &h32, &fx, &ux, &gx, &gxu, &gu, &t1,
                         &t2, &err, &n16, &ws, &prob, &xy, &angle, &mask};
        for (DevBuf* b : all) b->release();
        for (int k = 0; k < 4; ++k) {
            w_c2[k].release();
            b_c2[k].release();
            w_c4[k].release();
            b_c4[k].release();
        }
    }
};

namespace {

// OIHW weights (co_total, ci_total, k, k), output channels [co0, co1) and input
// channels [ci0, ci1) -> (k*k, cout_pad, cin_pad) fp16, zero padded.
std::vector<__half> pack(const float* W, int ci_total, int k, int co0, int co1, int ci0, int ci1,
                         int cin_pad, int cout_pad) {
    std::vector<__half> out((size_t)k * k * cout_pad * cin_pad, __float2half_rn(0.0f));
    for (int o = co0; o < co1; ++o)
        for (int c = ci0; c < ci1; ++c)
            for (int t = 0; t < k * k; ++t)
                out[((size_t)t * cout_pad + (o - co0)) * cin_pad + (c - ci0)] =
                    __float2half_rn(W[(((size_t)o * ci_total + c) * k * k) + t]);
    return out;
}

template <typename T>
cudaError_t upload(DevBuf& b, const std::vector<T>& v) {
    cudaError_t e = b.ensure(sizeof(T) * v.size());
    if (e != cudaSuccess) return e;
    return cudaMemcpy(b.p, v.data(), sizeof(T) * v.size(), cudaMemcpyHostToDevice);
}

// weight i of the reference's names (bvml_refiner_weight_name)
struct Spec {
    std::string name;
    int shape[4];
};
std::vector<Spec> specs() {
    std::vector<Spec> s;
    for (const char* g : {"z", "r", "q"}) {
        s.push_back({std::string("gru.conv") + g + ".weight", {kHidden, kHidden + kFeature + 2, 5, 5}});
        s.push_back({std::string("gru.conv") + g + ".bias", {kHidden, 0, 0, 0}});
    }
    for (int k = 0; k < 4; ++k) {
        const std::string n = kHeadName[k];
        s.push_back({n + ".0.weight", {kHeadHidden, kHidden + 2, 3, 3}});
        s.push_back({n + ".0.bias", {kHeadHidden, 0, 0, 0}});
        s.push_back({n + ".2.weight", {kHeadHidden, kHeadHidden, 1, 1}});
        s.push_back({n + ".2.bias", {kHeadHidden, 0, 0, 0}});
        s.push_back({n + ".4.weight", {kHeadOut[k], kHeadHidden, 1, 1}});
        s.push_back({n + ".4.bias", {kHeadOut[k], 0, 0, 0}});
    }
    return s;
}

// One convolution through the library's C entry point; cin_pad input channels
// from cin_off (64 for the GRU and 3x3 layers, 128 for the 1x1 head layers).
int conv(bvml_refiner* r, const void* x, int x_c, int cin_off, const DevBuf& w, const float* b,
         int cout, int cout_pad, int ks, const bvml_conv_epilogue& e, cudaStream_t s,
         int cin_pad = 64) {
    return bvml_conv2d_nhwc_f16_ex(x, x_c, cin_off, cin_pad, w.p, b, r->B, r->h, r->w, cout,
                                   cout_pad, ks, &e, r->err.as<int>(), s);
}

}  // namespace

namespace {

// ConvGRU + heads: `iters` iterations from the decoder's hidden state and
// feature, raw head outputs into the handle's buffers.
int stage(bvml_refiner* r, const float* normal, const float* feature, const float* hidden, int B,
          int h, int w, int iters, int dtype, size_t px, size_t es, cudaStream_t s) {
    (void)normal;
    int rc;
    if ((rc = bvml_stage_inputs(hidden, feature, B, h, w, r->h32.as<float>(), r->hx.p, r->fx.p,
                                s)) != BVML_OK)
        return rc;
    // the fixed inputs, once: uv -> z|r|q (one frame, shared), feature (+ that)
    // -> z|r|q as fp16 hi / lo halves, uv -> the heads' 3x3 (shared)
    const int saved_B = r->B;
    {
        bvml_conv_epilogue ep{};
        ep.mode = BVML_EPI_C4_F32;
        ep.out = r->gxu.p;
        ep.out_c = 192;
        r->B = 1;
        rc = conv(r, r->ux.p, 64, 0, r->w_gxu, r->zeros.as<float>(), 192, 192, 5, ep, s);
        if (rc == BVML_OK) {
            ep = bvml_conv_epilogue{};
            ep.mode = BVML_EPI_C4_F32;
            ep.out = r->gu.p;
            ep.out_c = 512;
            rc = conv(r, r->ux.p, 64, 0, r->w_gu, r->zeros.as<float>(), 512, 512, 3, ep, s);
        }
        r->B = saved_B;
        if (rc != BVML_OK) return rc;
        ep = bvml_conv_epilogue{};
        ep.mode = BVML_EPI_SPLIT_F16;
        ep.out = r->gx.p;
        ep.out_c = 384;
        ep.add = r->gxu.as<float>();
        ep.add_c = 192;
        ep.add_shared = 1;
        if ((rc = conv(r, r->fx.p, 64, 0, r->w_gx, r->zeros.as<float>(), 192, 192, 5, ep, s)) !=
            BVML_OK)
            return rc;
    }
    char* prob = r->prob.as<char>();
    char* xy = r->xy.as<char>();
    char* angle = r->angle.as<char>();
    const int planar = dtype == BVML_F16 ? BVML_EPI_PLANAR_F16 : BVML_EPI_PLANAR_F32;
    for (int it = 0; it < iters; ++it) {
        const bool up = it == iters - 1;  // only the last upsample reaches the output
        bvml_conv_epilogue ep{};
        ep.mode = BVML_EPI_GRU_ZR;
        ep.h32 = r->h32.as<float>();
        ep.z = r->z.p;
        ep.rh = r->rhx.p;
        ep.rh_c = 64;
        ep.xin = r->gx.p;
        ep.xin_c = 256;
        ep.xin_stride = 384;
        ep.wx = r->iz.p;
        if ((rc = conv(r, r->hx.p, 64, 0, r->w_zr, r->b_zr.as<float>(), 128, 128, 5, ep, s)) !=
            BVML_OK)
            return rc;
        ep = bvml_conv_epilogue{};
        ep.mode = BVML_EPI_GRU_Q;
        ep.h32 = r->h32.as<float>();
        ep.z = r->z.p;
        ep.hx = r->hx.p;
        ep.hx_c = 64;
        ep.xin = r->gx.as<__half>() + 256;
        ep.xin_c = 128;
        ep.xin_stride = 384;
        ep.wx = r->iq.p;
        if ((rc = conv(r, r->rhx.p, 64, 0, r->w_q, r->b_q.as<float>(), 64, 64, 5, ep, s)) !=
            BVML_OK)
            return rc;
        ep = bvml_conv_epilogue{};
        ep.mode = BVML_EPI_NHWC;
        ep.act = 1;
        ep.out = r->t1.p;
        ep.out_c = 512;
        ep.add = r->gu.as<float>();
        ep.add_c = 512;
        ep.add_shared = 1;
        const int n3 = up ? 512 : 384;
        if ((rc = conv(r, r->hx.p, 64, 0, up ? r->w_c0 : r->w_c0_3, r->b_c0.as<float>(), n3, n3,
                       3, ep, s)) != BVML_OK)
            return rc;
        void* dst[3] = {prob + es * px * 25 * it, xy + es * px * 50 * it,
                        angle + es * px * 25 * it};
        for (int k = 0; k < 3; ++k)
            if ((rc = bvml_head_tail_1x1(r->t1.p, 512, k * kHeadHidden, r->w_c2[k].p,
                                         r->b_c2[k].as<float>(), r->w_c4[k].p,
                                         r->b_c4[k].as<float>(), B, h, w, kHeadOut[k], dtype,
                                         dst[k], r->err.as<int>(), s)) != BVML_OK)
                return rc;
        if (up) {
            ep = bvml_conv_epilogue{};
            ep.mode = BVML_EPI_NHWC;
            ep.act = 1;
            ep.out = r->t2.p;
            ep.out_c = 512;
            ep.out_off = 3 * kHeadHidden;
            if ((rc = conv(r, r->t1.p, 512, 3 * kHeadHidden, r->w_c2[3], r->b_c2[3].as<float>(),
                           128, 128, 1, ep, s, kHeadHidden)) != BVML_OK)
                return rc;
            ep = bvml_conv_epilogue{};
            ep.mode = planar;
            ep.out = r->mask.p;
            if ((rc = conv(r, r->t2.p, 512, 3 * kHeadHidden, r->w_c4[3], r->b_c4[3].as<float>(),
                           576, 576, 1, ep, s, kHeadHidden)) != BVML_OK)
                return rc;
        }
    }
    return BVML_OK;
}

// The refine ops on the raw head outputs (activations applied on load).
int ops(bvml_refiner* r, const float* normal, int B, int h, int w, int iters, double fu,
        double cu, double fv, double cv, int crop_t, int crop_l, int out_h, int out_w, int dtype,
        size_t px, size_t es, void* out, cudaStream_t s) {
    cudaError_t e;
    char* prob = r->prob.as<char>();
    char* xy = r->xy.as<char>();
    char* angle = r->angle.as<char>();
    const void* n0 = normal;
    if (dtype == BVML_F16) {
        to_half_kernel<<<(unsigned)((px * 3 + 255) / 256 < 4096 ? (px * 3 + 255) / 256 : 4096),
                         256, 0, s>>>(normal, r->n16.as<__half>(), (long)px * 3);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "normal conversion");
        n0 = r->n16.p;
    }
    std::vector<const void*> pp(iters), xp(iters), ap(iters);
    for (int it = 0; it < iters; ++it) {
        pp[it] = prob + es * px * 25 * it;
        xp[it] = xy + es * px * 50 * it;
        ap[it] = angle + es * px * 25 * it;
    }
    return bvml_refine_logits(n0, nullptr, pp.data(), xp.data(), ap.data(), iters, r->mask.p, B, h,
                              w, 5, 1, fu, cu, fv, cv, 0, crop_t, crop_l, out_h, out_w, dtype,
                              r->ws.p, r->ws.n, out, s);
}

}  // namespace

extern "C" {

const char* bvml_refiner_weight_name(int i) {
    static const std::vector<Spec> s = specs();
    return (i >= 0 && i < (int)s.size()) ? s[i].name.c_str() : nullptr;
}

int bvml_refiner_weight_shape(int i, int* shape4) {
    static const std::vector<Spec> s = specs();
    if (i < 0 || i >= (int)s.size() || !shape4) return fail(BVML_EINVAL, "dsine ops: refiner: no such weight");
    for (int d = 0; d < 4; ++d) shape4[d] = s[i].shape[d];
    return BVML_OK;
}

int bvml_refiner_create(const float* const* weights, int device, bvml_refiner** out) {
    if (!weights || !out) return fail(BVML_EINVAL, "dsine ops: refiner: null argument");
    const std::vector<Spec> s = specs();
    for (size_t i = 0; i < s.size(); ++i)
        if (!weights[i]) return fail(BVML_EINVAL, "dsine ops: refiner: null weight " + s[i].name);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "set device");
    auto* r = new bvml_refiner;
    r->device = device;
    auto W = [&](int i) { return weights[i]; };
    const int cin = kHidden + kFeature + 2;  // 130
    // z and r stacked (128 outputs), q (64); hidden part = input channels [0, 64)
    std::vector<__half> wzr = pack(W(0), cin, 5, 0, 64, 0, 64, 64, 128);
    {
        std::vector<__half> wr = pack(W(2), cin, 5, 0, 64, 0, 64, 64, 64);
        for (int t = 0; t < 25; ++t)
            for (int o = 0; o < 64; ++o)
                for (int c = 0; c < 64; ++c)
                    wzr[((size_t)t * 128 + 64 + o) * 64 + c] = wr[((size_t)t * 64 + o) * 64 + c];
    }
    std::vector<float> bzr(W(1), W(1) + 64);
    bzr.insert(bzr.end(), W(3), W(3) + 64);
    std::vector<__half> wq = pack(W(4), cin, 5, 0, 64, 0, 64, 64, 64);
    std::vector<float> bq(W(5), W(5) + 64);
    // the fixed inputs' parts of z, r, q stacked (192 outputs): feature [64,128), uv [128,130)
    std::vector<__half> wgx((size_t)25 * 192 * 64), wgxu((size_t)25 * 192 * 64);
    for (int g = 0; g < 3; ++g) {
        std::vector<__half> f = pack(W(2 * g), cin, 5, 0, 64, 64, 128, 64, 64);
        std::vector<__half> u = pack(W(2 * g), cin, 5, 0, 64, 128, 130, 64, 64);
        for (int t = 0; t < 25; ++t)
            for (int o = 0; o < 64; ++o)
                for (int c = 0; c < 64; ++c) {
                    wgx[((size_t)t * 192 + 64 * g + o) * 64 + c] = f[((size_t)t * 64 + o) * 64 + c];
                    wgxu[((size_t)t * 192 + 64 * g + o) * 64 + c] = u[((size_t)t * 64 + o) * 64 + c];
                }
    }
    // the four heads' 3x3 layers stacked (512 outputs): hidden part and uv part
    std::vector<__half> wc0((size_t)9 * 512 * 64), wgu((size_t)9 * 512 * 64);
    std::vector<float> bc0;
    for (int k = 0; k < 4; ++k) {
        const float* w0 = W(6 + 6 * k);
        std::vector<__half> hpart = pack(w0, kHidden + 2, 3, 0, 128, 0, 64, 64, 128);
        std::vector<__half> upart = pack(w0, kHidden + 2, 3, 0, 128, 64, 66, 64, 128);
        for (int t = 0; t < 9; ++t)
            for (int o = 0; o < 128; ++o)
                for (int c = 0; c < 64; ++c) {
                    wc0[((size_t)t * 512 + 128 * k + o) * 64 + c] = hpart[((size_t)t * 128 + o) * 64 + c];
                    wgu[((size_t)t * 512 + 128 * k + o) * 64 + c] = upart[((size_t)t * 128 + o) * 64 + c];
                }
        bc0.insert(bc0.end(), W(7 + 6 * k), W(7 + 6 * k) + 128);
    }
    std::vector<__half> wc0_3((size_t)9 * 384 * 64);
    for (int t = 0; t < 9; ++t)
        for (int o = 0; o < 384; ++o)
            for (int c = 0; c < 64; ++c)
                wc0_3[((size_t)t * 384 + o) * 64 + c] = wc0[((size_t)t * 512 + o) * 64 + c];
    // identity blocks of the extra K that adds the hoisted GRU terms' hi + lo
    std::vector<__half> iz((size_t)128 * 256, __float2half_rn(0.0f)),
        iq((size_t)64 * 128, __float2half_rn(0.0f));
    for (int n = 0; n < 128; ++n) {
        iz[(size_t)n * 256 + (n / 64) * 128 + n % 64] = __float2half_rn(1.0f);
        iz[(size_t)n * 256 + (n / 64) * 128 + 64 + n % 64] = __float2half_rn(1.0f);
    }
    for (int n = 0; n < 64; ++n) {
        iq[(size_t)n * 128 + n] = __float2half_rn(1.0f);
        iq[(size_t)n * 128 + 64 + n] = __float2half_rn(1.0f);
    }
    if ((e = upload(r->w_zr, wzr)) != cudaSuccess || (e = upload(r->b_zr, bzr)) != cudaSuccess ||
        (e = upload(r->w_q, wq)) != cudaSuccess || (e = upload(r->b_q, bq)) != cudaSuccess ||
        (e = upload(r->w_gx, wgx)) != cudaSuccess || (e = upload(r->w_gxu, wgxu)) != cudaSuccess ||
        (e = upload(r->w_c0, wc0)) != cudaSuccess || (e = upload(r->w_c0_3, wc0_3)) != cudaSuccess ||
        (e = upload(r->b_c0, bc0)) != cudaSuccess || (e = upload(r->w_gu, wgu)) != cudaSuccess ||
        (e = upload(r->iz, iz)) != cudaSuccess || (e = upload(r->iq, iq)) != cudaSuccess ||
        (e = upload(r->zeros, std::vector<float>(512, 0.0f))) != cudaSuccess) {
        delete r;
        return cuda_fail(e, "weight upload");
    }
    for (int k = 0; k < 4; ++k) {
        const int c = kHeadOut[k];
        if ((e = upload(r->w_c2[k], pack(W(8 + 6 * k), 128, 1, 0, 128, 0, 128, 128, 128))) !=
                cudaSuccess ||
            (e = upload(r->b_c2[k], std::vector<float>(W(9 + 6 * k), W(9 + 6 * k) + 128))) !=
                cudaSuccess ||
            (e = upload(r->w_c4[k], pack(W(10 + 6 * k), 128, 1, 0, c, 0, 128, 128, pad64(c)))) !=
                cudaSuccess ||
            (e = upload(r->b_c4[k], std::vector<float>(W(11 + 6 * k), W(11 + 6 * k) + c))) !=
                cudaSuccess) {
            delete r;
            return cuda_fail(e, "weight upload");
        }
    }
    *out = r;
    return BVML_OK;
}

}  // extern "C"

int bvml::refiner_device(const bvml_refiner* r) { return r->device; }

extern "C" {

void bvml_refiner_destroy(bvml_refiner* r) {
    if (!r) return;
    cudaSetDevice(r->device);
    delete r;
}

int bvml_refiner_forward(bvml_refiner* r, const float* normal, const float* feature,
                         const float* hidden, int B, int h, int w, const float* intrins,
                         int origH, int origW, int iters, int crop_t, int crop_l, int out_h,
                         int out_w, int dtype, void* out, void* stream) {
    if (!r || !normal || !feature || !hidden || !intrins || !out)
        return fail(BVML_EINVAL, "dsine ops: refiner: null argument");
    if (B <= 0 || h <= 0 || w <= 0 || origH <= 0 || origW <= 0 || iters < 1 || iters > 64)
        return fail(BVML_EINVAL, "dsine ops: refiner: bad shape or iteration count");
    if (dtype != BVML_F32 && dtype != BVML_F16)
        return fail(BVML_EINVAL, "dsine ops: refiner: dtype must be F32 or F16");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    bvml::NvtxRange nvtx("bvml_refiner_forward");
    bvml::profile_mark(s, nullptr);
    cudaError_t e = cudaSetDevice(r->device);
    if (e != cudaSuccess) return cuda_fail(e, "set device");
    const size_t px = (size_t)B * h * w, hw = (size_t)h * w;
    const size_t es = dtype == BVML_F16 ? 2 : 4;
    if (r->B != B || r->h != h || r->w != w || r->iters != iters || r->dtype != dtype) {
        struct {
            DevBuf* b;
            size_t bytes;
        } need[] = {
            {&r->hx, 2 * px * 64},       {&r->rhx, 2 * px * 64},      {&r->z, 2 * px * 64},
            {&r->h32, 4 * px * 64},      {&r->fx, 2 * px * 64},       {&r->ux, 2 * hw * 64},
            {&r->gx, 2 * px * 384},      {&r->gxu, 4 * hw * 192},     {&r->gu, 4 * hw * 512},
            {&r->t1, 2 * px * 512},      {&r->t2, 2 * px * 512},      {&r->err, 16},
            {&r->n16, 2 * px * 3},       {&r->ws, bvml_refine_workspace_bytes(B, h, w)},
            {&r->prob, es * px * 25 * iters}, {&r->xy, es * px * 50 * iters},
            {&r->angle, es * px * 25 * iters}, {&r->mask, es * px * 576},
        };
        for (auto& n : need)
            if ((e = n.b->ensure(n.bytes)) != cudaSuccess) return cuda_fail(e, "buffer allocation");
        r->B = B;
        r->h = h;
        r->w = w;
        r->iters = iters;
        r->dtype = dtype;
    }
    // grid intrinsics from the raw float intrinsics and the padded size
    // (src/dsine_refine.cpp:230-237)
    const double sw = (double)w / origW, sh = (double)h / origH;
    const double fu = (double)intrins[0] * sw, cu = ((double)intrins[2] + 0.5) * sw;
    const double fv = (double)intrins[1] * sh, cv = ((double)intrins[3] + 0.5) * sh;
    if ((e = cudaMemsetAsync(r->err.p, 0, sizeof(int), s)) != cudaSuccess)
        return cuda_fail(e, "error word reset");
    uv_kernel<<<(unsigned)((hw * 64 + 255) / 256 < 4096 ? (hw * 64 + 255) / 256 : 4096), 256, 0,
                s>>>(r->ux.as<__half>(), h, w, fu, cu, fv, cv);
    if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "uv launch");
    int rc;
    nvtxRangePushA("refine.stage");
    rc = stage(r, normal, feature, hidden, B, h, w, iters, dtype, px, es, s);
    nvtxRangePop();
    if (rc != BVML_OK) return rc;
    bvml::profile_mark(s, "refine.stage");
    nvtxRangePushA("refine.ops");
    rc = ops(r, normal, B, h, w, iters, fu, cu, fv, cv, crop_t, crop_l, out_h, out_w, dtype, px,
             es, out, s);
    nvtxRangePop();
    if (rc == BVML_OK) bvml::profile_mark(s, "refine.ops");
    return rc;
}

int bvml_refiner_status(bvml_refiner* r, void* stream) {
    if (!r) return fail(BVML_EINVAL, "dsine ops: refiner: null handle");
    int v = 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&v, r->err.p, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "status copy");
    if (v != 0)
        return fail(BVML_ECUDA, "dsine cuda: refiner: a tensor-core pipeline gave up (code " +
                                    std::to_string(v) + ")");
    if (r->ws.p) return bvml_refine_status(r->ws.p, stream);
    return BVML_OK;
}

}  // extern "C"
