// Test driver: the whole learned refinement from a C++ program through the C
// ABI only (bvml_refiner_*), as a C++ host without Python would run it.
//
//   refiner_driver <dir> <B> <h> <w> <origH> <origW> <dtype 0|1>
//     reads <dir>/w<i>.f32 (the BVML_REFINER_WEIGHTS weights in
//     bvml_refiner_weight_name order, OIHW fp32), <dir>/{normal,feature,
//     hidden}.f32 and <dir>/intrins.f32 (fx, fy, cx, cy); writes <dir>/out.f32
//     (the (B,3,8h,8w) refined normals as fp32).
// Built and run by tests/test_gpu_refiner_capi.py.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include "bvml_dsine.h"

static std::vector<float> load(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) {
        std::fprintf(stderr, "missing %s\n", path.c_str());
        std::exit(2);
    }
    const std::streamsize n = f.tellg();
    f.seekg(0);
    std::vector<float> v((size_t)n / sizeof(float));
    f.read(reinterpret_cast<char*>(v.data()), n);
    return v;
}

static float* upload(const std::vector<float>& v) {
    float* d = nullptr;
    if (cudaMalloc(&d, v.size() * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(d, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        std::exit(3);
    return d;
}

int main(int argc, char** argv) {
    if (argc != 8) {
        std::fprintf(stderr, "usage: refiner_driver dir B h w origH origW dtype\n");
        return 1;
    }
    const std::string dir = argv[1];
    const int B = std::atoi(argv[2]), h = std::atoi(argv[3]), w = std::atoi(argv[4]);
    const int origH = std::atoi(argv[5]), origW = std::atoi(argv[6]), dtype = std::atoi(argv[7]);
    std::vector<std::vector<float>> wv(BVML_REFINER_WEIGHTS);
    std::vector<const float*> wp(BVML_REFINER_WEIGHTS);
    for (int i = 0; i < BVML_REFINER_WEIGHTS; ++i) {
        wv[i] = load(dir + "/w" + std::to_string(i) + ".f32");
        wp[i] = wv[i].data();
    }
    bvml_refiner* r = nullptr;
    if (bvml_refiner_create(wp.data(), 0, &r) != BVML_OK) {
        std::fprintf(stderr, "create: %s\n", bvml_last_error());
        return 4;
    }
    float* normal = upload(load(dir + "/normal.f32"));
    float* feature = upload(load(dir + "/feature.f32"));
    float* hidden = upload(load(dir + "/hidden.f32"));
    const std::vector<float> intr = load(dir + "/intrins.f32");
    const size_t n_out = (size_t)B * 3 * 8 * h * 8 * w;
    const size_t es = dtype == BVML_F16 ? 2 : 4;
    void* out = nullptr;
    cudaMalloc(&out, n_out * es);
    if (bvml_refiner_forward(r, normal, feature, hidden, B, h, w, intr.data(), origH, origW, 5, 0,
                             0, 8 * h, 8 * w, dtype, out, nullptr) != BVML_OK ||
        bvml_refiner_status(r, nullptr) != BVML_OK) {
        std::fprintf(stderr, "forward: %s\n", bvml_last_error());
        return 5;
    }
    std::vector<float> host(n_out);
    if (dtype == BVML_F16) {
        std::vector<__half> hh(n_out);
        cudaMemcpy(hh.data(), out, n_out * 2, cudaMemcpyDeviceToHost);
        for (size_t i = 0; i < n_out; ++i) host[i] = __half2float(hh[i]);
    } else {
        cudaMemcpy(host.data(), out, n_out * 4, cudaMemcpyDeviceToHost);
    }
    std::ofstream(dir + "/out.f32", std::ios::binary)
        .write(reinterpret_cast<const char*>(host.data()), (std::streamsize)(n_out * 4));
    bvml_refiner_destroy(r);
    return 0;
}
