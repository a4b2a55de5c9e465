#pragma once
// TEST INFRASTRUCTURE ONLY (oracle build). A host-only stand-in for the few
// members of brotensor::Tensor that the reference CPU twin
// (src/dsine_ops.cpp in wlejon/brovisionml) touches: `device`, `mat()`,
// `host_f32()` and `host_f32_mut()`. brotensor itself is a sibling repository
// that is not vendored with the reference, so the oracle compiles the
// reference source against this header instead. Nothing here ever reaches a
// GPU; the CUDA device value exists only so the reference's dispatch compiles.

#include <cstddef>
#include <memory>
#include <vector>

namespace brotensor {

enum class Device { CPU, CUDA, Metal };

struct Tensor {
    void* data = nullptr;
    Device device = Device::CPU;
    int rows = 0;
    int cols = 0;
    std::shared_ptr<std::vector<float>> store;  // owned storage, if any

    // Zero-filled host (rows x cols) fp32 matrix.
    static Tensor mat(int r, int c) {
        Tensor t;
        t.store = std::make_shared<std::vector<float>>(
            static_cast<std::size_t>(r) * static_cast<std::size_t>(c), 0.0f);
        t.data = t.store->data();
        t.rows = r;
        t.cols = c;
        return t;
    }

    // Non-owning host view over caller memory.
    static Tensor view(float* p, int r, int c) {
        Tensor t;
        t.data = p;
        t.rows = r;
        t.cols = c;
        return t;
    }

    const float* host_f32() const { return static_cast<const float*>(data); }
    float* host_f32_mut() { return static_cast<float*>(data); }
};

}  // namespace brotensor
