// Shared device helpers for the DSINE refine-ops kernels (sm_100a only).
//
// Pixel pairs: the hot kernels give every thread two horizontally adjacent
// pixels and carry their arithmetic in float2, issued as Blackwell's packed
// f32x2 instructions (__ffma2_rn / __fadd2_rn / __fmul2_rn): one issue slot
// does the work of two, which matters because these kernels sit close to the
// issue-rate ridge.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "brovisionml_b200 kernels are written for sm_100a (B200) only"
#endif

namespace bvml {

// ----------------------------------------------------------- checked builds
// With -DBVML_CHECKED (brovisionml_b200/_lib/libbvml_dsine_checked.so, built
// beside the release library) the kernels test their index arithmetic,
// shared-memory offsets and TMA coordinates before each access: a failed test
// ORs its bit into this translation unit's check word and the access is
// skipped -- never a trap, so the context stays usable. The test suite runs
// the odd shapes and edge cases through that build and requires a zero word
// (compute-sanitizer is not available on the GPU pool this was built on).
// Release builds compile the tests away.
enum CheckBit : unsigned {
    kChkNormalLoad = 1u << 0,   // AngMF halo load outside the frame
    kChkHaloSmem = 1u << 1,     // AngMF halo plane offset outside the plane
    kChkRing = 1u << 2,         // AngMF ring slot or offset outside the warp's ring
    kChkStore = 1u << 3,        // AngMF store outside the frame
    kChkDep = 1u << 4,          // persistent AngMF counter outside the tile table
    kChkUpTma = 1u << 5,        // upsample TMA box misaligned or outside the mask
    kChkUpRing = 1u << 6,       // upsample ring slot outside the ring
    kChkUpStore = 1u << 7,      // upsample store outside the output
    kChkConvTma = 1u << 8,      // convolution TMA channel coordinate misaligned
    kChkConvStore = 1u << 9,    // convolution epilogue pixel outside the frame
};
#ifdef BVML_CHECKED
static __device__ unsigned g_check_word;
__device__ __forceinline__ bool check_ok(bool ok, unsigned bit) {
    if (!ok) atomicOr(&g_check_word, bit);
    return ok;
}
// Host reader of this translation unit's check word (optionally reset).
#define BVML_CHECK_READER(fn)                                                    \
    unsigned fn(bool reset) {                                                   \
        unsigned v = 0;                                                         \
        if (cudaMemcpyFromSymbol(&v, g_check_word, sizeof(v)) != cudaSuccess)   \
            return 0x80000000u;                                                 \
        if (reset) {                                                            \
            const unsigned z = 0;                                               \
            cudaMemcpyToSymbol(g_check_word, &z, sizeof(z));                    \
        }                                                                       \
        return v;                                                               \
    }
#else
__device__ __forceinline__ constexpr bool check_ok(bool, unsigned) { return true; }
#define BVML_CHECK_READER(fn) \
    unsigned fn(bool) { return 0; }
#endif

// ------------------------------------------------------------------ float2 ops
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
// a * b + c
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
// c - a * b
__device__ __forceinline__ float2 fnma2(float2 a, float2 b, float2 c) {
    return __ffma2_rn(make_float2(-a.x, -a.y), b, c);
}
__device__ __forceinline__ float2 max2(float2 a, float2 b) {
    return make_float2(fmaxf(a.x, b.x), fmaxf(a.y, b.y));
}
__device__ __forceinline__ float2 rsqrt2(float2 a) { return make_float2(rsqrtf(a.x), rsqrtf(a.y)); }
// 1/sqrt(x) with the hardware approximation (PTX rsqrt.approx.ftz.f32, ~2 ulp):
// for arguments known to be normal numbers (clamped or range-checked).
__device__ __forceinline__ float rsqrt_ftz(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 rsqrt2_ftz(float2 a) { return make_float2(rsqrt_ftz(a.x), rsqrt_ftz(a.y)); }
// sin / cos with the hardware approximations (PTX sin.approx.ftz.f32 /
// cos.approx.ftz.f32; absolute error about 5e-7 on [-pi, pi]).
__device__ __forceinline__ float2 sin2_approx(float2 a) {
    float x, y;
    asm("sin.approx.ftz.f32 %0, %1;" : "=f"(x) : "f"(a.x));
    asm("sin.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(a.y));
    return make_float2(x, y);
}
__device__ __forceinline__ float2 cos2_approx(float2 a) {
    float x, y;
    asm("cos.approx.ftz.f32 %0, %1;" : "=f"(x) : "f"(a.x));
    asm("cos.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(a.y));
    return make_float2(x, y);
}
__device__ __forceinline__ float2 ex2_2(float2 a) { return make_float2(exp2f(a.x), exp2f(a.y)); }
// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32): results below
// 2^-126 flush to zero, which is harmless where x <= 0 feeds a softmax.
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 ex2_ftz2(float2 a) { return make_float2(ex2_ftz(a.x), ex2_ftz(a.y)); }
// 1/x with the hardware approximation (PTX rcp.approx.ftz.f32, ~1 ulp);
// 1/inf = 0.
__device__ __forceinline__ float rcp_ftz(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float2 rcp2_ftz(float2 a) { return make_float2(rcp_ftz(a.x), rcp_ftz(a.y)); }
// Programmatic dependent launch. A kernel launched with the programmatic
// stream serialization attribute (launch_pdl) may be scheduled while the
// previous kernel in its stream is still running: only once every CTA of
// that kernel has started and executed pdl_trigger() (or exited), so a
// waiting CTA never holds resources the previous kernel still needs.
// pdl_wait() blocks until the previous kernel has completed and its memory
// is visible; before it, a kernel may only read what was written before the
// previous kernel started. Both are no-ops for a normally launched kernel.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 eviction priorities (PTX createpolicy, used as .L2::cache_hint operands):
// streams read exactly once are marked evict-first so that they do not push
// out of L2 the data that is read again soon (AngMF's intermediate normals,
// marked evict-last when stored).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Two floats to global memory (8-byte aligned) with an L2 policy.
__device__ __forceinline__ void st2_hint(float* p, float2 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(v.x),
                 "f"(v.y), "l"(pol)
                 : "memory");
}

// -------------------------------------------------------------- storage types
template <typename T> struct St;
template <> struct St<float> {
    __device__ __forceinline__ static float ld(const float* p) { return __ldg(p); }
    // L2-coherent load (no L1): data another CTA of the same launch wrote.
    __device__ __forceinline__ static float ldcg(const float* p) { return __ldcg(p); }
    // Two consecutive elements; p must be 8-byte aligned.
    __device__ __forceinline__ static float2 ld2(const float* p) {
        return __ldg(reinterpret_cast<const float2*>(p));
    }
    // Streaming (read-once) variant: evict-first in L1/L2.
    __device__ __forceinline__ static float2 ld2s(const float* p) {
        return __ldcs(reinterpret_cast<const float2*>(p));
    }
    __device__ __forceinline__ static float lds1(const float* p) { return __ldcs(p); }
    __device__ __forceinline__ static void st(float* p, float v) { *p = v; }
    __device__ __forceinline__ static void st2(float* p, float2 v) {
        *reinterpret_cast<float2*>(p) = v;
    }
};
template <> struct St<__half> {
    __device__ __forceinline__ static float ld(const __half* p) { return __half2float(__ldg(p)); }
    __device__ __forceinline__ static float ldcg(const __half* p) { return __half2float(__ldcg(p)); }
    __device__ __forceinline__ static float2 ld2(const __half* p) {
        return __half22float2(__ldg(reinterpret_cast<const __half2*>(p)));
    }
    __device__ __forceinline__ static float2 ld2s(const __half* p) {
        return __half22float2(__ldcs(reinterpret_cast<const __half2*>(p)));
    }
    __device__ __forceinline__ static float lds1(const __half* p) {
        return __half2float(__ldcs(p));
    }
    __device__ __forceinline__ static void st(__half* p, float v) { *p = __float2half_rn(v); }
    __device__ __forceinline__ static void st2(__half* p, float2 v) {
        *reinterpret_cast<__half2*>(p) = __float22half2_rn(v);
    }
};

// A normal component: read-only path, or L2-coherent (COH) where the normals
// were written earlier in the same launch by other CTAs.
template <typename T, bool COH>
__device__ __forceinline__ float ldn(const T* p) {
    if constexpr (COH) return St<T>::ldcg(p);
    else return St<T>::ld(p);
}

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// RayReLU eps: the CPU twin's float constant 1e-2f (src/dsine_ops.cpp:27).
constexpr float kRayEps = 1e-2f;

// Launch `kern` on `s`, as a programmatic dependent of the previous kernel in
// the stream when `pdl` (the kernel then calls pdl_wait() before it reads
// that kernel's results).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? at : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace bvml
