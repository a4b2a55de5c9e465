// TEST INFRASTRUCTURE ONLY -- an extern "C" door into the reference's own
// CUDA kernels (src/dsine_ops.cu of wlejon/brovisionml), compiled in place,
// unchanged, for sm_100a by oracle/Makefile against the CUDA tensor stand-in
// under oracle/shim_cuda/ into oracle/_ref/libbvml_refgpu.so. Only tests/
// load it: it times the reference's GPU path on the B200 beside the repo's
// kernels and checks its results.
//
// bvml_refgpu_unit runs, frame by frame as Refiner::forward does
// (src/dsine_refine.cpp:241-272), the reference's device ops on fp32 device
// buffers: ray_relu_cuda on a copy of the frame's normals, then `iters`
// angmf_propagate_cuda calls (each re-allocating its output tensor, as the
// reference does), and copies the final grid normals to out. Everything runs
// on the legacy default stream, the reference's stream. The convex upsample
// is a brotensor op in the reference and is not part of this path.
#include "dsine_ops_cuda.h"

#include <cuda_runtime.h>

#include <exception>

using brotensor::Device;
using brotensor::Tensor;

extern "C" int bvml_refgpu_unit(const float* normal0, const float* ray,
                                const float* const* prob, const float* const* xy,
                                const float* const* angle, int iters, int frames, int H, int W,
                                double fu, double cu, double fv, double cv, float* out) {
    try {
        const int HW = H * W;
        const size_t nbytes = sizeof(float) * 3 * static_cast<size_t>(HW);
        for (int b = 0; b < frames; ++b) {
            Tensor n = Tensor::zeros_on(Device::CUDA, 1, 3 * HW);
            if (cudaMemcpyAsync(n.data, normal0 + static_cast<long>(b) * 3 * HW, nbytes,
                                cudaMemcpyDeviceToDevice, 0) != cudaSuccess)
                return -1;
            Tensor r = Tensor::view(const_cast<float*>(ray), 1, 3 * HW);
            brovisionml::dsine::detail::ray_relu_cuda(n, r, H, W);
            for (int it = 0; it < iters; ++it) {
                const long f = static_cast<long>(b) * HW;
                Tensor pr = Tensor::view(const_cast<float*>(prob[it]) + 25 * f, 1, 25 * HW);
                Tensor x = Tensor::view(const_cast<float*>(xy[it]) + 50 * f, 1, 50 * HW);
                Tensor a = Tensor::view(const_cast<float*>(angle[it]) + 25 * f, 1, 25 * HW);
                Tensor o;
                brovisionml::dsine::detail::angmf_propagate_cuda(n, pr, x, a, r, fu, cu, fv, cv,
                                                                 H, W, o);
                n = o;
            }
            if (cudaMemcpyAsync(out + static_cast<long>(b) * 3 * HW, n.data, nbytes,
                                cudaMemcpyDeviceToDevice, 0) != cudaSuccess)
                return -1;
        }
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    } catch (const std::exception&) {
        return -1;
    }
}
