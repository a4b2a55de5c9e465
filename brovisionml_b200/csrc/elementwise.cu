// The small per-pixel kernels of the path (sm_100a):
//  * RayReLU in place   (replaces ray_relu_kernel, src/dsine_ops.cu:58-74)
//  * the analytic ray   (replaces the host get_ray_core/build_ray8 + upload,
//                        src/dsine_decoder.cpp:242-290, src/dsine_refine.cpp:223-228)
//  * channel L2-normalise and the 2-D crop (the brotensor
//    l2_normalize_nchw_forward / slice2d_forward calls of
//    src/dsine_refine.cpp:280-292), for callers that drive the ops one by one;
//  * the refine stage's input layouts: the decoder's hidden state and feature
//    (planar fp32) into the GRU state (C4 fp32) and the convolutions' NHWC fp16
//    inputs, one pass (the concat of src/dsine_refine.cpp:245-248).
// All are HBM-bound streams with grid-stride loops sized to the SM count.
#include <cuda_fp16.h>

#include "bvml_common.cuh"
#include "bvml_internal.h"

namespace bvml {
namespace {

constexpr int kThreads = 256;

int grid_for(long work) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    const long want = (work + kThreads - 1) / kThreads;
    const long cap = (long)sms * 8;
    return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
ray_relu_kernel(T* __restrict__ n, const float* __restrict__ r, int B, long HW) {
    const long total = (long)B * HW;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total;
         i += (long)gridDim.x * kThreads) {
        const long b = i / HW, p = i - b * HW;
        T* nb = n + b * 3 * HW;
        float nx = St<T>::ld(nb + p), ny = St<T>::ld(nb + HW + p), nz = St<T>::ld(nb + 2 * HW + p);
        const float rx = __ldg(r + p), ry = __ldg(r + HW + p), rz = __ldg(r + 2 * HW + p);
        const float nn2 = fmaf(nx, nx, fmaf(ny, ny, nz * nz));
        const float rr2 = fmaf(rx, rx, fmaf(ry, ry, rz * rz));
        const float c = fmaf(nx, rx, fmaf(ny, ry, nz * rz)) * rsqrtf(fmaxf(nn2 * rr2, 1e-16f));
        const float dc = fmaxf(kRayEps - c, 0.0f);
        nx = fmaf(rx, dc, nx);
        ny = fmaf(ry, dc, ny);
        nz = fmaf(rz, dc, nz);
        const float inv = rsqrtf(fmaxf(fmaf(nx, nx, fmaf(ny, ny, nz * nz)), 1e-24f));
        St<T>::st(nb + p, nx * inv);
        St<T>::st(nb + HW + p, ny * inv);
        St<T>::st(nb + 2 * HW + p, nz * inv);
    }
}

__global__ void __launch_bounds__(kThreads)
build_ray_kernel(float* __restrict__ ray, int H, int W, float ifu, float tu_c, float ifv,
                 float tv_c) {
    const long HW = (long)H * W;
    for (long p = (long)blockIdx.x * kThreads + threadIdx.x; p < HW;
         p += (long)gridDim.x * kThreads) {
        const int y = (int)(p / W), x = (int)(p - (long)y * W);
        const float rx = fmaf((float)x, ifu, tu_c);
        const float ry = fmaf((float)y, ifv, tv_c);
        const float inv = rsqrtf(fmaf(rx, rx, fmaf(ry, ry, 1.0f)));
        ray[p] = rx * inv;
        ray[HW + p] = ry * inv;
        ray[2 * HW + p] = inv;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
l2norm_kernel(const T* x, T* y, int N, int C, long HW, float eps) {
    const long total = (long)N * HW;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total;
         i += (long)gridDim.x * kThreads) {
        const long b = i / HW, p = i - b * HW;
        const T* xb = x + b * C * HW + p;
        T* yb = y + b * C * HW + p;
        float v[16];
        float ss = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            if (c < C) {
                v[c] = St<T>::ld(xb + c * HW);
                ss = fmaf(v[c], v[c], ss);
            }
        }
        const float inv = rsqrtf(fmaxf(ss, eps * eps));
#pragma unroll
        for (int c = 0; c < 16; ++c)
            if (c < C) St<T>::st(yb + c * HW, v[c] * inv);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
slice_kernel(const T* __restrict__ x, T* __restrict__ y, int NC, int H, int W, int h0, int w0,
             int Ho, int Wo) {
    const long total = (long)NC * Ho * Wo;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total;
         i += (long)gridDim.x * kThreads) {
        const long plane = i / ((long)Ho * Wo);
        const long rem = i - plane * Ho * Wo;
        const int r = (int)(rem / Wo), c = (int)(rem - (long)r * Wo);
        y[i] = x[(plane * H + h0 + r) * W + w0 + c];
    }
}

// One thread per pixel of 64-channel planar fp32 inputs: h0 -> h32 (C4 fp32,
// [b][16][HW][4]) and hx (NHWC fp16), feat -> fx (NHWC fp16). The planar reads
// are coalesced across the warp's consecutive pixels; each thread writes its
// pixel's 128-byte NHWC rows whole.
__global__ void __launch_bounds__(kThreads)
stage_inputs_kernel(const float* __restrict__ h0, const float* __restrict__ feat, int B, long HW,
                    float* __restrict__ h32, __half* __restrict__ hx,
                    __half* __restrict__ fx) {
    const long total = (long)B * HW;
    for (long i = (long)blockIdx.x * kThreads + threadIdx.x; i < total;
         i += (long)gridDim.x * kThreads) {
        const long b = i / HW, p = i - b * HW;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __ldg(h0 + (b * 64 + g * 8 + j) * HW + p);
            float4* c4 = reinterpret_cast<float4*>(h32) + (b * 16 + 2 * g) * HW + p;
            c4[0] = make_float4(v[0], v[1], v[2], v[3]);
            c4[HW] = make_float4(v[4], v[5], v[6], v[7]);
            alignas(16) __half o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = __float2half_rn(v[j]);
            reinterpret_cast<uint4*>(hx)[i * 8 + g] = *reinterpret_cast<const uint4*>(o);
            if (feat) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    o[j] = __float2half_rn(__ldg(feat + (b * 64 + g * 8 + j) * HW + p));
                reinterpret_cast<uint4*>(fx)[i * 8 + g] = *reinterpret_cast<const uint4*>(o);
            }
        }
    }
}

}  // namespace

cudaError_t launch_stage_inputs(const float* h0, const float* feat, int B, int H, int W,
                                float* h32, void* hx, void* fx, cudaStream_t s) {
    const long HW = (long)H * W;
    if (B == 0 || HW == 0) return cudaSuccess;
    stage_inputs_kernel<<<grid_for((long)B * HW), kThreads, 0, s>>>(
        h0, feat, B, HW, h32, static_cast<__half*>(hx), static_cast<__half*>(fx));
    return cudaGetLastError();
}

cudaError_t launch_ray_relu(void* normal, SType t, const float* ray, int B, int H, int W,
                            cudaStream_t s) {
    const long HW = (long)H * W;
    if (B == 0 || HW == 0) return cudaSuccess;
    const int g = grid_for((long)B * HW);
    if (t == SType::F32)
        ray_relu_kernel<float><<<g, kThreads, 0, s>>>(static_cast<float*>(normal), ray, B, HW);
    else
        ray_relu_kernel<__half><<<g, kThreads, 0, s>>>(static_cast<__half*>(normal), ray, B, HW);
    return cudaGetLastError();
}

cudaError_t launch_build_ray(float* ray, int H, int W, double fu, double cu, double fv,
                             double cv, cudaStream_t s) {
    const long HW = (long)H * W;
    if (HW == 0) return cudaSuccess;
    build_ray_kernel<<<grid_for(HW), kThreads, 0, s>>>(
        ray, H, W, (float)(1.0 / fu), (float)((0.5 - cu) / fu), (float)(1.0 / fv),
        (float)((0.5 - cv) / fv));
    return cudaGetLastError();
}

cudaError_t launch_l2_normalize(const void* x, void* y, SType t, int N, int C, int H, int W,
                                float eps, cudaStream_t s) {
    const long HW = (long)H * W;
    if (N == 0 || C == 0 || HW == 0) return cudaSuccess;
    if (C > 16) return cudaErrorInvalidValue;
    const int g = grid_for((long)N * HW);
    if (t == SType::F32)
        l2norm_kernel<float><<<g, kThreads, 0, s>>>(static_cast<const float*>(x),
                                                    static_cast<float*>(y), N, C, HW, eps);
    else
        l2norm_kernel<__half><<<g, kThreads, 0, s>>>(static_cast<const __half*>(x),
                                                     static_cast<__half*>(y), N, C, HW, eps);
    return cudaGetLastError();
}

cudaError_t launch_slice2d(const void* x, void* y, SType t, int N, int C, int H, int W, int h0,
                           int w0, int Ho, int Wo, cudaStream_t s) {
    const long total = (long)N * C * Ho * Wo;
    if (total == 0) return cudaSuccess;
    const int g = grid_for(total);
    if (t == SType::F32)
        slice_kernel<float><<<g, kThreads, 0, s>>>(static_cast<const float*>(x),
                                                   static_cast<float*>(y), N * C, H, W, h0, w0,
                                                   Ho, Wo);
    else
        slice_kernel<__half><<<g, kThreads, 0, s>>>(static_cast<const __half*>(x),
                                                    static_cast<__half*>(y), N * C, H, W, h0,
                                                    w0, Ho, Wo);
    return cudaGetLastError();
}

}  // namespace bvml
