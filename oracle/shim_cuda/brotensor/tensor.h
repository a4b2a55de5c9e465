#pragma once
// TEST INFRASTRUCTURE ONLY (oracle build). A CUDA-capable stand-in for the
// members of brotensor::Tensor that the reference's CUDA ops
// (src/dsine_ops.cu in wlejon/brovisionml) touch: `data`, `device`,
// `zeros_on(Device::CUDA, rows, cols)` and non-owning views. brotensor is a
// sibling repository that is not vendored with the reference, so the timing
// of the reference's own GPU kernels compiles them against this header.
//
// zeros_on keeps freed device buffers in a per-size cache (as a tensor
// library's caching allocator would) and zeroes them with cudaMemsetAsync on
// the legacy default stream, the stream the reference's kernels use: the
// timing then measures the reference's kernels and its per-call output
// re-allocation, not cudaMalloc.

#include <cuda_runtime.h>

#include <cstddef>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <vector>

namespace brotensor {

enum class Device { CPU, CUDA, Metal };

namespace shim_detail {
struct Cache {
    std::mutex m;
    std::multimap<std::size_t, void*> free;
};
inline Cache& cache() {
    static Cache* c = new Cache;  // never destroyed: buffers live until exit
    return *c;
}
inline void* acquire(std::size_t bytes) {
    Cache& c = cache();
    {
        std::lock_guard<std::mutex> g(c.m);
        auto it = c.free.find(bytes);
        if (it != c.free.end()) {
            void* p = it->second;
            c.free.erase(it);
            return p;
        }
    }
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess)
        throw std::runtime_error("brotensor shim: cudaMalloc failed");
    return p;
}
inline void release(std::size_t bytes, void* p) {
    Cache& c = cache();
    std::lock_guard<std::mutex> g(c.m);
    c.free.emplace(bytes, p);
}
}  // namespace shim_detail

struct Tensor {
    void* data = nullptr;
    Device device = Device::CPU;
    int rows = 0;
    int cols = 0;
    std::shared_ptr<void> owner;

    static Tensor zeros_on(Device dev, int r, int c) {
        if (dev != Device::CUDA) throw std::runtime_error("brotensor shim: CUDA tensors only");
        Tensor t;
        t.device = dev;
        t.rows = r;
        t.cols = c;
        const std::size_t bytes = sizeof(float) * static_cast<std::size_t>(r) * c;
        void* p = shim_detail::acquire(bytes);
        if (cudaMemsetAsync(p, 0, bytes, 0) != cudaSuccess)
            throw std::runtime_error("brotensor shim: cudaMemsetAsync failed");
        t.owner = std::shared_ptr<void>(p, [bytes](void* q) { shim_detail::release(bytes, q); });
        t.data = p;
        return t;
    }

    // Non-owning view over existing device memory.
    static Tensor view(void* p, int r, int c) {
        Tensor t;
        t.data = p;
        t.device = Device::CUDA;
        t.rows = r;
        t.cols = c;
        return t;
    }
};

}  // namespace brotensor
