// C++ drop-in for the reference's CUDA op wrappers (src/dsine_ops_cuda.h).
//
// brovisionml's dispatch (src/dsine_ops.cpp:178-215) calls
//   brovisionml::dsine::detail::ray_relu_cuda(Tensor&, const Tensor&, int, int)
//   brovisionml::dsine::detail::angmf_propagate_cuda(..., Tensor& out)
// for CUDA-resident tensors. This file defines exactly those two functions on
// top of libbvml_dsine.so, so an integrator replaces src/dsine_ops.cu with
// this file (plus the library) and src/dsine_ops.cpp / src/dsine_refine.cpp
// compile unchanged. Contract kept from the reference:
//  * fp32 (1, 3HW) / (1, 25HW) / (1, 50HW) tensors, ps = 5, dilation 1;
//  * `out` is (re)allocated as a fresh zeroed (1, 3HW) CUDA tensor
//    (src/dsine_ops.cu:178);
//  * launches go to the legacy default stream, no synchronisation;
//  * failures throw std::runtime_error("dsine cuda: <what>: <error>") or
//    "dsine ops: ..." like the reference.
// It additionally exposes refine_ops_cuda(), the fused unit of
// Refiner::forward's op calls, for a Refiner that wants one call per forward,
// and angmf_propagate_logits_cuda(), which takes the prediction heads' raw
// prob / angle outputs and applies their activations on load.
#include "brotensor/tensor.h"
#include "bvml_dsine.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace brovisionml::dsine::detail {

namespace {

void check(int rc) {
    if (rc != BVML_OK) throw std::runtime_error(bvml_last_error());
}

}  // namespace

void ray_relu_cuda(brotensor::Tensor& normal, const brotensor::Tensor& ray, int H, int W) {
    if (static_cast<int64_t>(H) * W == 0) return;
    check(bvml_ray_relu(normal.data, static_cast<const float*>(ray.data), 1, H, W, BVML_F32,
                        nullptr));
}

void angmf_propagate_cuda(const brotensor::Tensor& pred_norm, const brotensor::Tensor& prob,
                          const brotensor::Tensor& xy, const brotensor::Tensor& angle,
                          const brotensor::Tensor& ray, double fu, double cu, double fv,
                          double cv, int H, int W, brotensor::Tensor& out) {
    const int HW = H * W;
    out = brotensor::Tensor::zeros_on(brotensor::Device::CUDA, 1, 3 * HW);
    if (HW == 0) return;
    check(bvml_angmf_propagate(pred_norm.data, prob.data, xy.data, angle.data,
                               static_cast<const float*>(ray.data), fu, cu, fv, cv, 1, H, W,
                               /*ps=*/5, /*dil=*/1, BVML_F32, out.data, nullptr));
}

// angmf_propagate_cuda on the heads' raw outputs: prob = sigmoid(prob_logits)
// and angle = kPi * sigmoid(angle_logits) are applied while the kernel loads
// them, so a Refiner can drop apply_sigmoid(prob), apply_sigmoid(angle) and
// scale_inplace(angle, kPi) (src/dsine_refine.cpp:262-267).
void angmf_propagate_logits_cuda(const brotensor::Tensor& pred_norm,
                                 const brotensor::Tensor& prob_logits,
                                 const brotensor::Tensor& xy,
                                 const brotensor::Tensor& angle_logits,
                                 const brotensor::Tensor& ray, double fu, double cu, double fv,
                                 double cv, int H, int W, brotensor::Tensor& out) {
    const int HW = H * W;
    out = brotensor::Tensor::zeros_on(brotensor::Device::CUDA, 1, 3 * HW);
    if (HW == 0) return;
    check(bvml_angmf_propagate_logits(pred_norm.data, prob_logits.data, xy.data,
                                      angle_logits.data, static_cast<const float*>(ray.data), fu,
                                      cu, fv, cv, 1, H, W, /*ps=*/5, /*dil=*/1, BVML_F32,
                                      out.data, nullptr));
}

// The op part of Refiner::forward (src/dsine_refine.cpp:241-292) in one call:
// ray_relu(normal), iterations of angmf_propagate over the per-iteration head
// outputs, one convex upsample + L2-normalise, crop to (out_h, out_w) at
// (crop_t, crop_l). Returns the (1, 3*out_h*out_w) CUDA tensor. With
// head_logits, prob / angle are the heads' raw outputs (activated on load).
brotensor::Tensor refine_ops_cuda(const brotensor::Tensor& normal, const brotensor::Tensor& ray8,
                                  const std::vector<const brotensor::Tensor*>& prob,
                                  const std::vector<const brotensor::Tensor*>& xy,
                                  const std::vector<const brotensor::Tensor*>& angle,
                                  const brotensor::Tensor& up_mask, double fu, double cu,
                                  double fv, double cv, int H, int W, int crop_t, int crop_l,
                                  int out_h, int out_w, bool head_logits) {
    if (prob.size() != xy.size() || prob.size() != angle.size())
        throw std::runtime_error("dsine ops: refine_ops: per-iteration lists differ in length");
    const int iters = static_cast<int>(prob.size());
    std::vector<const void*> pp(iters), xp(iters), ap(iters);
    for (int i = 0; i < iters; ++i) {
        pp[i] = prob[i]->data;
        xp[i] = xy[i]->data;
        ap[i] = angle[i]->data;
    }
    const size_t ws_bytes = bvml_refine_workspace_bytes(1, H, W);
    brotensor::Tensor ws = brotensor::Tensor::zeros_on(
        brotensor::Device::CUDA, 1, static_cast<int>((ws_bytes + sizeof(float) - 1) / sizeof(float)));
    brotensor::Tensor out =
        brotensor::Tensor::zeros_on(brotensor::Device::CUDA, 1, 3 * out_h * out_w);
    auto fn = head_logits ? bvml_refine_logits : bvml_refine;
    check(fn(normal.data, static_cast<const float*>(ray8.data), pp.data(), xp.data(), ap.data(),
             iters, up_mask.data, 1, H, W, 5, 1, fu, cu, fv, cv, /*full_res_ray_relu=*/0, crop_t,
             crop_l, out_h, out_w, BVML_F32, ws.data, ws_bytes, out.data, nullptr));
    return out;
}

}  // namespace brovisionml::dsine::detail
