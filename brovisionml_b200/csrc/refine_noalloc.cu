// bvml_refine_noalloc: the fused refine unit for callers that must not
// allocate device memory.
//
// bvml_refine needs a scratch workspace (the intermediate normals between
// AngMF iterations, and the ray when none is given). Most callers pass a
// buffer they allocated once. Some cannot: a plugin running inside another
// application's inference or render loop, where that host owns the GPU memory
// budget and forbids allocations after start-up; or a latency-critical loop
// that cannot afford cudaMalloc's implicit device synchronisation stalling
// its other streams. For them this file keeps the scratch in a fixed
// file-scope device array that the CUDA runtime creates when it loads this
// library's device code on a GPU, and that stays there until the process
// exits.
//
// Set-up: every call looks the array's device address up
// (cudaGetSymbolAddress) with the caller's device current, and passes that
// pointer, never the array's host-side name, to the kernels. Nothing is
// cached between calls, so a device reset or another context made current
// through the driver API cannot leave a stale address behind. Under CUDA's
// default lazy module loading, the first call on a device is also the one
// that loads this library's device code there and so reserves the array;
// callers with a fixed memory budget should make one call at start-up, and
// before any stream capture.
//
// Limits and sharing: the array holds BVML_REFINE_NOALLOC_MAX_BYTES bytes;
// requests needing more scratch (bvml_refine_workspace_bytes(B, h, w)) are
// rejected with BVML_EINVAL. All calls on one device share the array, and
// it keeps whatever the last call left in it: two calls whose work overlaps
// on the GPU (different streams, or different host threads) race on it and
// corrupt each other's results, so callers must serialise them. Nothing in
// the scratch needs to start at zero: every intermediate is written before it
// is read, so no clearing is done.
#include "bvml_dsine.h"
#include "bvml_internal.h"

#include <cuda_runtime.h>

#include <string>

namespace {

// The scratch itself: BVML_REFINE_NOALLOC_MAX_BYTES bytes per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[BVML_REFINE_NOALLOC_MAX_BYTES];

}  // namespace

extern "C" int bvml_refine_noalloc(const void* normal0, const float* ray8,
                                   const void* const* prob, const void* const* xy,
                                   const void* const* angle, int iters, const void* mask, int B,
                                   int h, int w, int ps, int dil, double fu, double cu, double fv,
                                   double cv, int full_res_ray_relu, int crop_t, int crop_l,
                                   int out_h, int out_w, int dtype, void* out, void* stream) {
    if (B < 0 || h < 0 || w < 0)
        return bvml::report_error(BVML_EINVAL, "dsine ops: refine_noalloc: bad shape");
    const size_t need = bvml_refine_workspace_bytes(B, h, w);
    if (need > (size_t)BVML_REFINE_NOALLOC_MAX_BYTES)
        return bvml::report_error(
            BVML_EINVAL, "dsine ops: refine_noalloc: " + std::to_string(B) + " frames of " +
                             std::to_string(h) + "x" + std::to_string(w) + " need " +
                             std::to_string(need) + " bytes of scratch, more than the " +
                             std::to_string((size_t)BVML_REFINE_NOALLOC_MAX_BYTES) +
                             "-byte built-in buffer (use bvml_refine with a workspace)");
    // the device address of the array in the current device's context; the
    // runtime resolves this without allocating once the module is loaded
    void* scratch = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e != cudaSuccess || !scratch)
        return bvml::report_error(
            BVML_ECUDA, std::string("dsine cuda: refine_noalloc: scratch set-up "
                                    "(cudaGetSymbolAddress): ") +
                            cudaGetErrorString(e != cudaSuccess ? e : cudaErrorUnknown));
    return bvml_refine(normal0, ray8, prob, xy, angle, iters, mask, B, h, w, ps, dil, fu, cu, fv,
                       cv, full_res_ray_relu, crop_t, crop_l, out_h, out_w, dtype, scratch,
                       (size_t)BVML_REFINE_NOALLOC_MAX_BYTES, out, stream);
}
