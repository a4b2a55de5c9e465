// Implicit-GEMM 2-D convolution on the 5th-generation tensor cores (sm_100a):
// the dense convolutions of the refine stage's ConvGRU and prediction heads
// (src/dsine_refine.cpp:95-158: 5x5 pad 2, 3x3 pad 1, 1x1), which the
// reference runs as brotensor conv2d_forward calls.
//
// Layout: activations NHWC bf16 with the channel count padded to a multiple
// of 64 (pad channels zero), weights [tap][C_out_pad][C_in_pad] bf16 (K-major
// rows), fp32 bias, fp32 accumulation in tensor memory.
//
// GEMM view: M = pixels, N = output channels, K = taps x input channels. A CTA
// owns a tile of 128 pixels (tw x th, chosen per width to waste the fewest
// rows) and N output channels (64, 128 or 256). For each filter tap and
// 64-channel chunk:
//  * warp 0 (one lane) loads the A tile -- the 128 pixels shifted by the tap,
//    64 channels -- with one 4-D TMA box from the NHWC tensor (coordinates
//    outside the frame read zeros: the convolution's zero padding), and the
//    B tile (N x 64 weights) with one 3-D box, both 128-byte swizzled, into a
//    ring of S stages;
//  * warp 1 (one lane) issues four tcgen05.mma (K = 16 each) per stage into
//    the TMEM accumulator (128 lanes x N fp32 columns) and releases the stage
//    with tcgen05.commit;
//  * warps 2-5 wait for the last commit, read the accumulator with
//    tcgen05.ld (one pixel per thread), add the bias, apply the activation
//    and store bf16 (pad channels as zeros, so the output can feed the next
//    convolution directly).
// All waits are bounded (tc_common.cuh); a wait that gives up sets *err and
// the CTA tears down after its copies and MMAs in flight have completed.
#include <cuda_bf16.h>

#include <mutex>

#include "bvml_common.cuh"
#include "bvml_internal.h"
#include "tc_common.cuh"

#include <cudaTypedefs.h>

namespace bvml {
namespace {

constexpr int kTM = 128;             // pixels per tile (MMA M)
constexpr int kKC = 64;              // channels per K chunk (one 128-byte swizzle row)
constexpr int kConvThreads = 192;    // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr uint32_t kWaitLimit = 1u << 22;

struct ConvArgs {
    int B, H, W;
    int cin_off, cin_pad, cout, cout_pad;  // input channel slice, output channels
    int ks, pad;
    int tw, th, tiles_x, tiles_y;
    const float* bias;
    int* err;
    // epilogue targets (see ConvEpi)
    void* out;
    int out_c, out_off;
    float* h32;
    __nv_bfloat16* z;
    __nv_bfloat16* rh;
    int rh_c;
    __nv_bfloat16* hx;
    int hx_c;
    __nv_bfloat16* hin;
    int hin_c;
};

template <int ACT>
__device__ __forceinline__ float activate(float v) {
    if constexpr (ACT == 1) return fmaxf(v, 0.0f);
    else if constexpr (ACT == 2) return 1.0f / (1.0f + __expf(-v));
    else if constexpr (ACT == 3) return tanhf(v);
    else return v;
}

// Epilogue of one thread's pixel for 32 consecutive output channels
// cb .. cb+31 (accumulators + bias in v). Modes (ConvEpi in bvml_internal.h):
//  NHWC      act(v) as bf16 at out[pix * out_c + out_off + c], zeros past cout;
//  PLANAR16/32  v as fp16 / fp32 at out[(b * cout + c) * H * W + y * W + x]
//            for c < cout (the NCHW planes the refine ops take);
//  GRU_ZR    c < 64: z = sigmoid(v) -> z[pix * 64 + c];
//            64 <= c < 128: r = sigmoid(v) -> rh[pix * rh_c + c - 64] = r * h32;
//  GRU_Q     c < 64: q = tanh(v), h = (1 - z) h + z q -> h32 (fp32 state) and
//            bf16 copies at hx[pix * hx_c + c] and, if set, hin[pix * hin_c + c]
//  (src/dsine_refine.cpp:140-158).
template <int EPI, int ACT>
__device__ __forceinline__ void epilogue32(const ConvArgs& a, long pix, int b, int px, int py,
                                           int cb, const uint32_t (&v)[32]) {
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        f[i] = cb + i < a.cout ? __uint_as_float(v[i]) + a.bias[cb + i] : 0.0f;
    if constexpr (EPI == (int)ConvEpi::NHWC) {
        alignas(16) __nv_bfloat16 o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
            o[i] = __float2bfloat16_rn(cb + i < a.cout ? activate<ACT>(f[i]) : 0.0f);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) +
                                              pix * a.out_c + a.out_off + cb);
        const uint4* src = reinterpret_cast<const uint4*>(o);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = src[q];
    } else if constexpr (EPI == (int)ConvEpi::PLANAR16 || EPI == (int)ConvEpi::PLANAR32) {
        const long hw = (long)a.H * a.W;
        const long p = (long)py * a.W + px;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int c = cb + i;
            if (c >= a.cout) break;
            const long o = ((long)b * a.cout + c) * hw + p;
            if constexpr (EPI == (int)ConvEpi::PLANAR16)
                static_cast<__half*>(a.out)[o] = __float2half_rn(f[i]);
            else
                static_cast<float*>(a.out)[o] = f[i];
        }
    } else if constexpr (EPI == (int)ConvEpi::GRU_ZR) {
        alignas(16) __nv_bfloat16 o[32];
        if (cb < 64) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float2bfloat16_rn(activate<2>(f[i]));
            uint4* dst = reinterpret_cast<uint4*>(a.z + pix * 64 + cb);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<const uint4*>(o)[q];
        } else if (cb < 128) {
            const float4* h4 = reinterpret_cast<const float4*>(a.h32 + pix * 64 + (cb - 64));
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 h = h4[q];
                o[4 * q + 0] = __float2bfloat16_rn(activate<2>(f[4 * q + 0]) * h.x);
                o[4 * q + 1] = __float2bfloat16_rn(activate<2>(f[4 * q + 1]) * h.y);
                o[4 * q + 2] = __float2bfloat16_rn(activate<2>(f[4 * q + 2]) * h.z);
                o[4 * q + 3] = __float2bfloat16_rn(activate<2>(f[4 * q + 3]) * h.w);
            }
            uint4* dst = reinterpret_cast<uint4*>(a.rh + pix * a.rh_c + (cb - 64));
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<const uint4*>(o)[q];
        }
    } else if constexpr (EPI == (int)ConvEpi::GRU_Q) {
        if (cb >= 64) return;
        float4* h4 = reinterpret_cast<float4*>(a.h32 + pix * 64 + cb);
        const uint4* z4 = reinterpret_cast<const uint4*>(a.z + pix * 64 + cb);
        alignas(16) __nv_bfloat16 zb[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(zb)[q] = z4[q];
        alignas(16) __nv_bfloat16 o[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 h = h4[q];
            float* hh = reinterpret_cast<float*>(&h);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * q + e;
                const float z = __bfloat162float(zb[i]);
                hh[e] = fmaf(z, tanhf(f[i]) - hh[e], hh[e]);  // (1 - z) h + z q
                o[i] = __float2bfloat16_rn(hh[e]);
            }
            h4[q] = h;
        }
        uint4* d1 = reinterpret_cast<uint4*>(a.hx + pix * a.hx_c + cb);
#pragma unroll
        for (int q = 0; q < 4; ++q) d1[q] = reinterpret_cast<const uint4*>(o)[q];
        if (a.hin) {
            uint4* d2 = reinterpret_cast<uint4*>(a.hin + pix * a.hin_c + cb);
#pragma unroll
            for (int q = 0; q < 4; ++q) d2[q] = reinterpret_cast<const uint4*>(o)[q];
        }
    }
}

template <int N, int S>
struct ConvCfg {
    static constexpr int kABytes = kTM * kKC * 2;
    static constexpr int kBBytes = N * kKC * 2;
    static constexpr int kStage = kABytes + kBBytes;
    static constexpr int kBarOff = S * kStage;                 // mbarriers after the ring
    static constexpr int kSmem = kBarOff + 256 + 1024;         // + barriers, alignment slack
};


template <int N, int S, int EPI, int ACT>
__global__ void __launch_bounds__(kConvThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const ConvArgs a) {
    using C = ConvCfg<N, S>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bar_full = sbase + C::kBarOff;        // S barriers
    const uint32_t bar_empty = bar_full + 8 * S;         // S barriers
    const uint32_t bar_done = bar_empty + 8 * S;         // 1 barrier
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + 16 * S + 8);
    int* abort_flag = reinterpret_cast<int*>(smem + C::kBarOff + 16 * S + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int t = blockIdx.x;
    const int tx = t % a.tiles_x;
    t /= a.tiles_x;
    const int ty = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int x0 = tx * a.tw, y0 = ty * a.th, n0 = blockIdx.y * N;
    const int chunks = a.cin_pad / kKC;
    const int k_iters = a.ks * a.ks * chunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(bar_full + 8 * s, 1);
            tc::mbar_init(bar_empty + 8 * s, 1);
        }
        tc::mbar_init(bar_done, 1);
        *abort_flag = 0;
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&map_a);
        tc::tma_prefetch_desc(&map_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), N);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&](int code) {
        atomicExch(a.err, code);
        *reinterpret_cast<volatile int*>(abort_flag) = 1;
    };
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(abort_flag) != 0; };

    if (warp == 0 && lane == 0) {
        // ---------------------------------------------------------- producer
        int issued = 0;
        for (int it = 0; it < k_iters && !aborted(); ++it) {
            const int s = it % S, j = it / S;
            if (j > 0 && !tc::mbar_wait(bar_empty + 8 * s, (j - 1) & 1, kWaitLimit)) {
                fail(1);
                break;
            }
            const int tap = it / chunks, ch = it - tap * chunks;
            const int ky = tap / a.ks, kx = tap - ky * a.ks;
            const uint32_t sa = sbase + s * C::kStage, sb = sa + C::kABytes;
            tc::mbar_expect_tx(bar_full + 8 * s, C::kABytes + C::kBBytes);
            tc::tma_load_4d(sa, &map_a, bar_full + 8 * s, a.cin_off + ch * kKC, x0 + kx - a.pad,
                            y0 + ky - a.pad, b);
            tc::tma_load_3d(sb, &map_b, bar_full + 8 * s, ch * kKC, n0, tap);
            issued = it + 1;
        }
        // no copy may still be landing when the CTA exits
        for (int it = issued - S > 0 ? issued - S : 0; it < issued; ++it)
            if (!tc::mbar_wait(bar_full + 8 * (it % S), (it / S) & 1, kWaitLimit)) fail(2);
    } else if (warp == 1 && lane == 0) {
        // --------------------------------------------------------------- MMA
        constexpr uint32_t idesc = tc::idesc_bf16_f32(kTM, N);
        int it = 0;
        for (; it < k_iters; ++it) {
            const int s = it % S, j = it / S;
            if (!tc::mbar_wait(bar_full + 8 * s, j & 1, kWaitLimit) || aborted()) {
                fail(3);
                break;
            }
            tc::tc_fence_after();
            const uint32_t sa = sbase + s * C::kStage, sb = sa + C::kABytes;
            const uint64_t da = tc::umma_desc_k_sw128(sa), db = tc::umma_desc_k_sw128(sb);
#pragma unroll
            for (int k = 0; k < kKC / 16; ++k)  // K = 16 per MMA: 32 bytes = 2 descriptor units
                tc::umma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, it > 0 || k > 0);
            tc::umma_commit(bar_empty + 8 * s);
        }
        tc::umma_commit(bar_done);  // also after an abort: every issued MMA has completed
        if (!tc::mbar_wait(bar_done, 0, kWaitLimit)) fail(4);
    } else if (warp >= 2) {
        // ---------------------------------------------------------- epilogue
        const int wq = warp & 3;              // the TMEM lane quarter this warp may read
        const int row = wq * 32 + lane;       // pixel index in the tile
        const bool ok = tc::mbar_wait(bar_done, 0, kWaitLimit);
        if (!ok) fail(5);
        tc::tc_fence_after();
        const int px = x0 + row % a.tw, py = y0 + row / a.tw;
        const bool in = ok && !aborted() && px < a.W && py < a.H;
        const long pix = ((long)b * a.H + py) * a.W + px;
#pragma unroll 1
        for (int c0 = 0; c0 < N; c0 += 32) {
            uint32_t v[32];
            tc::tmem_ld_32cols(tmem + ((uint32_t)(wq * 32) << 16) + c0, v);
            tc::tmem_ld_wait();
            const int cb = n0 + c0;
            if (!in || cb >= a.cout_pad) continue;
            epilogue32<EPI, ACT>(a, pix, b, px, py, cb, v);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, N);
    }
}

// ------------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
            const cuuint64_t* strides_bytes, const cuuint32_t* box) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
              strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int N, int S, int EPI, int ACT>
cudaError_t launch_n(const CUtensorMap& ma, const CUtensorMap& mb, const ConvArgs& a,
                     cudaStream_t s) {
    auto kern = conv_tc_kernel<N, S, EPI, ACT>;
    constexpr int smem = ConvCfg<N, S>::kSmem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)(a.tiles_x * a.tiles_y * a.B), (unsigned)((a.cout_pad + N - 1) / N));
    kern<<<grid, kConvThreads, smem, s>>>(ma, mb, a);
    return cudaGetLastError();
}

template <int EPI, int ACT>
cudaError_t launch_act(int n, const CUtensorMap& ma, const CUtensorMap& mb, const ConvArgs& a,
                       cudaStream_t s) {
    switch (n) {
        case 256: return launch_n<256, 4, EPI, ACT>(ma, mb, a, s);
        case 128: return launch_n<128, 5, EPI, ACT>(ma, mb, a, s);
        default: return launch_n<64, 6, EPI, ACT>(ma, mb, a, s);
    }
}

}  // namespace

cudaError_t launch_conv_tc(const ConvLaunch& L, cudaStream_t s) {
    if (L.B == 0 || L.H == 0 || L.W == 0 || L.cout_pad == 0) return cudaSuccess;
    ConvArgs a{};
    a.B = L.B;
    a.H = L.H;
    a.W = L.W;
    a.cin_off = L.cin_off;
    a.cin_pad = L.cin_pad;
    a.cout = L.cout;
    a.cout_pad = L.cout_pad;
    a.ks = L.ks;
    a.pad = L.ks / 2;
    a.bias = L.bias;
    a.err = L.err;
    a.out = L.y;
    a.out_c = L.out_c;
    a.out_off = L.out_off;
    a.h32 = L.h32;
    a.z = static_cast<__nv_bfloat16*>(L.z);
    a.rh = static_cast<__nv_bfloat16*>(L.rh);
    a.rh_c = L.rh_c;
    a.hx = static_cast<__nv_bfloat16*>(L.hx);
    a.hx_c = L.hx_c;
    a.hin = static_cast<__nv_bfloat16*>(L.hin);
    a.hin_c = L.hin_c;
    // pixel tile tw x th (= 128): the shape with the fewest out-of-frame rows
    static const int tws[4] = {128, 64, 32, 16};
    long best = -1;
    for (int tw : tws) {
        const int th = kTM / tw;
        const long tiles = (long)((L.W + tw - 1) / tw) * ((L.H + th - 1) / th);
        if (best < 0 || tiles < best) {
            best = tiles;
            a.tw = tw;
            a.th = th;
        }
    }
    a.tiles_x = (L.W + a.tw - 1) / a.tw;
    a.tiles_y = (L.H + a.th - 1) / a.th;
    if ((long)a.tiles_x * a.tiles_y * L.B > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    // GRU gates need every channel of a pixel in one CTA (z with r, q with z)
    int n = L.cout_pad >= 256 ? 256 : (L.cout_pad >= 128 ? 128 : 64);
    if (L.epi == ConvEpi::GRU_ZR) n = 128;
    if (L.epi == ConvEpi::GRU_Q) n = 64;

    CUtensorMap ma, mb;
    const cuuint64_t dims_a[4] = {(cuuint64_t)L.x_c, (cuuint64_t)L.W, (cuuint64_t)L.H,
                                  (cuuint64_t)L.B};
    const cuuint64_t str_a[3] = {(cuuint64_t)L.x_c * 2, (cuuint64_t)L.W * L.x_c * 2,
                                 (cuuint64_t)L.H * L.W * L.x_c * 2};
    const cuuint32_t box_a[4] = {(cuuint32_t)kKC, (cuuint32_t)a.tw, (cuuint32_t)a.th, 1};
    const cuuint64_t dims_b[3] = {(cuuint64_t)L.cin_pad, (cuuint64_t)L.cout_pad,
                                  (cuuint64_t)(L.ks * L.ks)};
    const cuuint64_t str_b[2] = {(cuuint64_t)L.cin_pad * 2,
                                 (cuuint64_t)L.cout_pad * L.cin_pad * 2};
    const cuuint32_t box_b[3] = {(cuuint32_t)kKC, (cuuint32_t)n, 1};
    if (!encode(&ma, L.x, 4, dims_a, str_a, box_a) || !encode(&mb, L.w, 3, dims_b, str_b, box_b))
        return cudaErrorInvalidValue;
    switch (L.epi) {
        case ConvEpi::NHWC:
            switch (L.act) {
                case 0: return launch_act<(int)ConvEpi::NHWC, 0>(n, ma, mb, a, s);
                case 1: return launch_act<(int)ConvEpi::NHWC, 1>(n, ma, mb, a, s);
                case 2: return launch_act<(int)ConvEpi::NHWC, 2>(n, ma, mb, a, s);
                case 3: return launch_act<(int)ConvEpi::NHWC, 3>(n, ma, mb, a, s);
                default: return cudaErrorInvalidValue;
            }
        case ConvEpi::PLANAR16: return launch_act<(int)ConvEpi::PLANAR16, 0>(n, ma, mb, a, s);
        case ConvEpi::PLANAR32: return launch_act<(int)ConvEpi::PLANAR32, 0>(n, ma, mb, a, s);
        case ConvEpi::GRU_ZR: return launch_act<(int)ConvEpi::GRU_ZR, 0>(n, ma, mb, a, s);
        case ConvEpi::GRU_Q: return launch_act<(int)ConvEpi::GRU_Q, 0>(n, ma, mb, a, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace bvml
