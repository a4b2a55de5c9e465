// Test driver for the reference-facing C++ bridge (libbvml_dsine_bridge.so):
// calls brovisionml::dsine::detail::{ray_relu_cuda, angmf_propagate_cuda,
// angmf_propagate_logits_cuda, refine_ops_cuda} on brotensor-shaped (1, C*HW)
// fp32 CUDA tensors, the way brovisionml's dispatch (src/dsine_ops.cpp:178-215)
// and Refiner::forward (src/dsine_refine.cpp:241-292) call them.
//
//   bridge_driver <op> <dir> <H> <W> [iters]
//     op: ray_relu | angmf | angmf_logits | refine
//     reads <dir>/<name>.f32 (raw float32), writes <dir>/out.f32
// Built and run by tests/test_gpu_bridge.py.
#include <cuda_runtime.h>

#include <cstdio>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "brotensor/tensor.h"

namespace brovisionml::dsine::detail {
void ray_relu_cuda(brotensor::Tensor& normal, const brotensor::Tensor& ray, int H, int W);
void angmf_propagate_cuda(const brotensor::Tensor& pred_norm, const brotensor::Tensor& prob,
                          const brotensor::Tensor& xy, const brotensor::Tensor& angle,
                          const brotensor::Tensor& ray, double fu, double cu, double fv,
                          double cv, int H, int W, brotensor::Tensor& out);
void angmf_propagate_logits_cuda(const brotensor::Tensor& pred_norm,
                                 const brotensor::Tensor& prob_logits,
                                 const brotensor::Tensor& xy,
                                 const brotensor::Tensor& angle_logits,
                                 const brotensor::Tensor& ray, double fu, double cu, double fv,
                                 double cv, int H, int W, brotensor::Tensor& out);
brotensor::Tensor refine_ops_cuda(const brotensor::Tensor& normal, const brotensor::Tensor& ray8,
                                  const std::vector<const brotensor::Tensor*>& prob,
                                  const std::vector<const brotensor::Tensor*>& xy,
                                  const std::vector<const brotensor::Tensor*>& angle,
                                  const brotensor::Tensor& up_mask, double fu, double cu,
                                  double fv, double cv, int H, int W, int crop_t, int crop_l,
                                  int out_h, int out_w, bool head_logits);
}  // namespace brovisionml::dsine::detail

namespace {

using brotensor::Device;
using brotensor::Tensor;

std::string g_dir;

Tensor load(const std::string& name, int cols) {
    std::vector<float> h(static_cast<size_t>(cols));
    std::ifstream f(g_dir + "/" + name + ".f32", std::ios::binary);
    if (!f.read(reinterpret_cast<char*>(h.data()), sizeof(float) * h.size()))
        throw std::runtime_error("bridge_driver: cannot read " + name);
    Tensor t = Tensor::zeros_on(Device::CUDA, 1, cols);
    if (cudaMemcpy(t.data, h.data(), sizeof(float) * h.size(), cudaMemcpyHostToDevice) !=
        cudaSuccess)
        throw std::runtime_error("bridge_driver: upload failed");
    return t;
}

void save(const Tensor& t) {
    std::vector<float> h(static_cast<size_t>(t.rows) * t.cols);
    if (cudaMemcpy(h.data(), t.data, sizeof(float) * h.size(), cudaMemcpyDeviceToHost) !=
        cudaSuccess)
        throw std::runtime_error("bridge_driver: download failed");
    std::ofstream f(g_dir + "/out.f32", std::ios::binary);
    f.write(reinterpret_cast<const char*>(h.data()), sizeof(float) * h.size());
}

}  // namespace

int main(int argc, char** argv) {
    namespace d = brovisionml::dsine::detail;
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s op dir H W [iters]\n", argv[0]);
        return 2;
    }
    const std::string op = argv[1];
    g_dir = argv[2];
    const int H = std::stoi(argv[3]), W = std::stoi(argv[4]), HW = H * W;
    const int iters = argc > 5 ? std::stoi(argv[5]) : 1;
    try {
        std::ifstream f(g_dir + "/intr.f64", std::ios::binary);
        std::vector<double> k(4);
        if (!f.read(reinterpret_cast<char*>(k.data()), sizeof(double) * 4))
            throw std::runtime_error("bridge_driver: cannot read intrinsics");
        Tensor normal = load("normal", 3 * HW), ray = load("ray", 3 * HW);
        if (op == "ray_relu") {
            d::ray_relu_cuda(normal, ray, H, W);
            save(normal);
        } else if (op == "angmf" || op == "angmf_logits") {
            Tensor prob = load("prob0", 25 * HW), xy = load("xy0", 50 * HW),
                   angle = load("angle0", 25 * HW), out;
            (op == "angmf" ? d::angmf_propagate_cuda : d::angmf_propagate_logits_cuda)(
                normal, prob, xy, angle, ray, k[0], k[1], k[2], k[3], H, W, out);
            save(out);
        } else if (op == "refine") {
            std::vector<Tensor> p, x, a;
            for (int i = 0; i < iters; ++i) {
                p.push_back(load("prob" + std::to_string(i), 25 * HW));
                x.push_back(load("xy" + std::to_string(i), 50 * HW));
                a.push_back(load("angle" + std::to_string(i), 25 * HW));
            }
            std::vector<const Tensor*> pp, xp, ap;
            for (int i = 0; i < iters; ++i) {
                pp.push_back(&p[i]);
                xp.push_back(&x[i]);
                ap.push_back(&a[i]);
            }
            Tensor mask = load("mask", 576 * HW);
            save(d::refine_ops_cuda(normal, ray, pp, xp, ap, mask, k[0], k[1], k[2], k[3], H, W,
                                    0, 0, 8 * H, 8 * W, false));
        } else {
            throw std::runtime_error("bridge_driver: unknown op " + op);
        }
        if (cudaDeviceSynchronize() != cudaSuccess)
            throw std::runtime_error("bridge_driver: device error");
    } catch (const std::exception& e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 1;
    }
    return 0;
}
