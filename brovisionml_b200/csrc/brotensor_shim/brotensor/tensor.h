#pragma once
// Build stand-in for brotensor/tensor.h (the sibling library the reference
// builds against, not available here). It carries only the members that the
// DSINE op bridge (dsine_ops_b200.cpp) uses -- `data`, `device`, `rows`,
// `cols`, `zeros_on` -- so that the bridge can be compiled and exercised in
// this repository. An integrator compiles the bridge against the real
// brotensor header instead.

#include <cstddef>
#include <cstring>
#include <memory>
#include <stdexcept>

#if defined(BVML_SHIM_CUDA)
#include <cuda_runtime.h>
#endif

namespace brotensor {

enum class Device { CPU, CUDA, Metal };

struct Tensor {
    void* data = nullptr;
    Device device = Device::CPU;
    int rows = 0;
    int cols = 0;
    std::shared_ptr<void> owner;

    static Tensor zeros_on(Device dev, int r, int c) {
        Tensor t;
        t.device = dev;
        t.rows = r;
        t.cols = c;
        const std::size_t bytes = sizeof(float) * static_cast<std::size_t>(r) * c;
        if (dev == Device::CUDA) {
#if defined(BVML_SHIM_CUDA)
            void* p = nullptr;
            if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess)
                throw std::runtime_error("brotensor shim: cudaMalloc failed");
            cudaMemset(p, 0, bytes);
            t.owner = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
#else
            throw std::runtime_error("brotensor shim: built without CUDA");
#endif
        } else {
            t.owner = std::shared_ptr<void>(::operator new(bytes ? bytes : 1),
                                            [](void* q) { ::operator delete(q); });
            std::memset(t.owner.get(), 0, bytes);
        }
        t.data = t.owner.get();
        return t;
    }

    // Non-owning view over existing memory.
    static Tensor view(void* p, Device dev, int r, int c) {
        Tensor t;
        t.data = p;
        t.device = dev;
        t.rows = r;
        t.cols = c;
        return t;
    }
};

}  // namespace brotensor
