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
//  * warps 2-9 wait for the last commit, read the accumulator with
//    tcgen05.ld (one pixel per thread; two warps per TMEM lane quarter, each
//    half of the columns), add the bias, apply the epilogue and store (pad
//    channels as zeros, so the output can feed the next convolution).
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
constexpr int kConvThreads = 320;    // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 epilogue
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter, each half the columns
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
//  (PLANAR16/32: planar_chunk, through a shared-memory transpose)
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

// BRES (1x1 convolutions with at most kBResChunks input chunks): the CTA's
// weights stay resident in shared memory, loaded once, and the ring carries
// only pixel tiles; each CTA then keeps one output-channel tile.
constexpr int kBResChunks = 2;

template <int N, int S, int EPI, bool BRES = false>
struct ConvCfg {
    static constexpr int kABytes = kTM * kKC * 2;
    static constexpr int kBBytes = N * kKC * 2;
    static constexpr int kBRes = BRES ? kBResChunks * kBBytes : 0;  // resident weights first
    static constexpr int kStage = BRES ? kABytes : kABytes + kBBytes;
    static constexpr bool kPlanar = EPI == (int)ConvEpi::PLANAR16 || EPI == (int)ConvEpi::PLANAR32;
    static constexpr int kOutElem = EPI == (int)ConvEpi::PLANAR16 ? 2 : 4;
    // planar outputs: per epilogue warp two 32-channel x 32-pixel staging buffers
    static constexpr int kStageWarpBytes = 32 * 32 * kOutElem;
    static constexpr int kStageOutOff = kBRes + S * kStage;
    static constexpr int kStageOutBytes = kPlanar ? kEpiWarps * 2 * kStageWarpBytes : 0;
    static constexpr int kBarOff = kStageOutOff + kStageOutBytes;  // mbarriers last
    static constexpr int kSmem = kBarOff + 256 + 1024;         // + barriers, alignment slack
};

// Planar output of one 32-channel chunk (channels cb .. cb+31) of one
// epilogue warp's 32 pixels: every lane puts its pixel's values into the
// warp's staging buffer ([channel][pixel], the TMA box layout), and lane 0
// stores the box (pw x ph pixels x 32 channels at (px0, py0, cb, b)) into the
// planar tensor with one TMA store -- clipped at the frame and channel edges,
// asynchronous; the buffer is reused two chunks later, after the store has
// read it.
template <typename TO>
__device__ __forceinline__ void planar_chunk_tma(const ConvArgs& a, const CUtensorMap* map_o,
                                                 TO* stg, uint32_t stg_addr, int lane,
                                                 int px0, int py0, int b, int cb,
                                                 const uint32_t (&v)[32]) {
    if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's previous store has read it
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float f = cb + i < a.cout ? __uint_as_float(v[i]) + a.bias[cb + i] : 0.0f;
        if constexpr (sizeof(TO) == 2) stg[i * 32 + lane] = __float2half_rn(f);
        else stg[i * 32 + lane] = f;
    }
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tc::tma_store_4d(map_o, stg_addr, px0, py0, cb, b);
        tc::bulk_commit();
    }
}

// Persistent: CTA c computes tiles c, c + G, c + 2G, ... (G CTAs, one per
// SM). The TMA / MMA ring runs on across tiles; the accumulator is double
// buffered in TMEM (2 x N columns), so the epilogue warps drain tile i while
// the MMA lane accumulates tile i + 1.
template <int N, int S, int EPI, int ACT, bool BRES>
__global__ void __launch_bounds__(kConvThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_o, const ConvArgs a) {
    using C = ConvCfg<N, S, EPI, BRES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bar_full = sbase + C::kBarOff;        // S barriers: stage loaded
    const uint32_t bar_empty = bar_full + 8 * S;         // S barriers: stage consumed
    const uint32_t bar_acc_full = bar_empty + 8 * S;     // 2 barriers: accumulator ready
    const uint32_t bar_acc_empty = bar_acc_full + 16;    // 2 barriers: accumulator drained
    const uint32_t bar_end = bar_acc_empty + 16;         // 1 barrier: every MMA complete
    const uint32_t bar_bres = bar_end + 8;               // 1 barrier: resident weights loaded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOff + 16 * S + 48);
    int* abort_flag = reinterpret_cast<int*>(smem + C::kBarOff + 16 * S + 56);
    const uint32_t ring = sbase + C::kBRes;              // the A (and B) stages

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = a.cin_pad / kKC;
    const int k_iters = a.ks * a.ks * chunks;
    const int n_nt = (a.cout_pad + N - 1) / N;
    const int n_tiles = a.tiles_x * a.tiles_y * a.B * n_nt;
    // this CTA's tiles: t0, t0 + dt, ... (BRES: one output-channel tile per CTA)
    const int n_sp = a.tiles_x * a.tiles_y * a.B;
    const int g_per = BRES ? (int)gridDim.x / n_nt : 0;
    const int my_nt = BRES ? (int)blockIdx.x % n_nt : 0;
    const int t0 = BRES ? ((int)blockIdx.x / n_nt) * n_nt + my_nt : (int)blockIdx.x;
    const int dt = BRES ? g_per * n_nt : (int)gridDim.x;
    const int t_end = BRES ? ((int)blockIdx.x / n_nt < g_per ? n_sp * n_nt : 0) : n_tiles;
    // tile t -> output channels nt, frame b, pixel tile (tx, ty)
    auto tile_of = [&](int t, int& b, int& x0, int& y0, int& n0) {
        n0 = (t % n_nt) * N;
        int r = t / n_nt;
        const int tx = r % a.tiles_x;
        r /= a.tiles_x;
        const int ty = r % a.tiles_y;
        b = r / a.tiles_y;
        x0 = tx * a.tw;
        y0 = ty * a.th;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(bar_full + 8 * s, 1);
            tc::mbar_init(bar_empty + 8 * s, 1);
        }
        for (int q = 0; q < 2; ++q) {
            tc::mbar_init(bar_acc_full + 8 * q, 1);
            tc::mbar_init(bar_acc_empty + 8 * q, kEpiWarps);  // one arrive per epilogue warp
        }
        tc::mbar_init(bar_end, 1);
        tc::mbar_init(bar_bres, 1);
        *abort_flag = 0;
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&map_a);
        tc::tma_prefetch_desc(&map_b);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), 2 * N);
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
        int g = 0;  // stages issued by this CTA
        if constexpr (BRES) {  // the CTA's weights, once
            tc::mbar_expect_tx(bar_bres, chunks * C::kBBytes);
            for (int ch = 0; ch < chunks; ++ch)
                tc::tma_load_3d(sbase + ch * C::kBBytes, &map_b, bar_bres, ch * kKC, my_nt * N, 0);
        }
        for (int t = t0; t < t_end && !aborted(); t += dt) {
            int b, x0, y0, n0;
            tile_of(t, b, x0, y0, n0);
            for (int it = 0; it < k_iters; ++it, ++g) {
                const int s = g % S, j = g / S;
                if (j > 0 && !tc::mbar_wait(bar_empty + 8 * s, (j - 1) & 1, kWaitLimit)) {
                    fail(1);
                    break;
                }
                if (aborted()) break;
                const int tap = it / chunks, ch = it - tap * chunks;
                const int ky = tap / a.ks, kx = tap - ky * a.ks;
                const uint32_t sa = ring + s * C::kStage, sb = sa + C::kABytes;
                tc::mbar_expect_tx(bar_full + 8 * s, C::kStage);
                tc::tma_load_4d(sa, &map_a, bar_full + 8 * s, a.cin_off + ch * kKC,
                                x0 + kx - a.pad, y0 + ky - a.pad, b);
                if constexpr (!BRES) tc::tma_load_3d(sb, &map_b, bar_full + 8 * s, ch * kKC, n0, tap);
            }
        }
        // no copy may still be landing when the CTA exits
        for (int q = g - S > 0 ? g - S : 0; q < g; ++q)
            if (!tc::mbar_wait(bar_full + 8 * (q % S), (q / S) & 1, kWaitLimit)) fail(2);
        if (BRES && !tc::mbar_wait(bar_bres, 0, kWaitLimit)) fail(2);
    } else if (warp == 1 && lane == 0) {
        // --------------------------------------------------------------- MMA
        constexpr uint32_t idesc = tc::idesc_bf16_f32(kTM, N);
        int g = 0, tl = 0;
        if (BRES && t0 < t_end && !tc::mbar_wait(bar_bres, 0, kWaitLimit)) fail(7);
        for (int t = t0; t < t_end && !aborted(); t += dt, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            if (u > 0 && !tc::mbar_wait(bar_acc_empty + 8 * buf, (u - 1) & 1, kWaitLimit)) {
                fail(3);
                break;
            }
            tc::tc_fence_after();
            const uint32_t acc = tmem + buf * N;
            bool ok = true;
            for (int it = 0; it < k_iters; ++it, ++g) {
                const int s = g % S, j = g / S;
                if (!tc::mbar_wait(bar_full + 8 * s, j & 1, kWaitLimit) || aborted()) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint32_t sa = ring + s * C::kStage;
                const uint32_t sb = BRES ? sbase + it * C::kBBytes : sa + C::kABytes;
                const uint64_t da = tc::umma_desc_k_sw128(sa), db = tc::umma_desc_k_sw128(sb);
#pragma unroll
                for (int k = 0; k < kKC / 16; ++k)  // K = 16 per MMA: 32 B = 2 descriptor units
                    tc::umma_bf16(acc, da + 2 * k, db + 2 * k, idesc, it > 0 || k > 0);
                tc::umma_commit(bar_empty + 8 * s);
            }
            if (!ok) {
                fail(4);
                break;
            }
            tc::umma_commit(bar_acc_full + 8 * buf);
        }
        tc::umma_commit(bar_end);  // also after an abort: every issued MMA has completed
        if (!tc::mbar_wait(bar_end, 0, kWaitLimit)) fail(5);
    } else if (warp >= 2) {
        // ---------------------------------------------------------- epilogue
        const int wq = warp & 3;              // the TMEM lane quarter this warp may read
        const int row = wq * 32 + lane;       // pixel index in the tile
        const int half = (warp - 2) >> 2;     // which half of the N columns it drains
        int pcount = 0;                       // planar chunks stored by this warp
        int tl = 0;
        for (int t = t0; t < t_end; t += dt, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            const bool ok = tc::mbar_wait(bar_acc_full + 8 * buf, u & 1, kWaitLimit);
            if (!ok) fail(6);
            if (!ok || aborted()) break;
            tc::tc_fence_after();
            int b, x0, y0, n0;
            tile_of(t, b, x0, y0, n0);
            const int px = x0 + row % a.tw, py = y0 + row / a.tw;
            const bool in = px < a.W && py < a.H;
            const long pix = ((long)b * a.H + py) * a.W + px;
            const uint32_t acc = tmem + buf * N + ((uint32_t)(wq * 32) << 16);
#pragma unroll 1
            for (int c0 = half * (N / 2); c0 < (half + 1) * (N / 2); c0 += 32) {
                uint32_t v[32];
                tc::tmem_ld_32cols(acc + c0, v);
                tc::tmem_ld_wait();
                const int cb = n0 + c0;
                if constexpr (C::kPlanar) {
                    if (cb >= a.cout) continue;  // the same for the whole warp
                    // this warp's 32 pixels: tile rows [wq * 32, wq * 32 + 32) as a
                    // pw x ph box (pw = min(tw, 32))
                    const int px0 = x0 + (wq * 32) % a.tw, py0 = y0 + (wq * 32) / a.tw;
                    if (px0 >= a.W || py0 >= a.H) continue;  // the whole box is off the frame
                    const int slot = (warp - 2) * 2 + (pcount & 1);
                    uint8_t* stg = smem + C::kStageOutOff + slot * C::kStageWarpBytes;
                    const uint32_t stg_addr = sbase + C::kStageOutOff + slot * C::kStageWarpBytes;
                    if constexpr (EPI == (int)ConvEpi::PLANAR16)
                        planar_chunk_tma<__half>(a, &map_o, reinterpret_cast<__half*>(stg),
                                                 stg_addr, lane, px0, py0, b, cb, v);
                    else
                        planar_chunk_tma<float>(a, &map_o, reinterpret_cast<float*>(stg),
                                                stg_addr, lane, px0, py0, b, cb, v);
                    ++pcount;
                } else {
                    if (!in || cb >= a.cout_pad) continue;
                    epilogue32<EPI, ACT>(a, pix, b, px, py, cb, v);
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(bar_acc_empty + 8 * buf);
        }
        if (C::kPlanar && lane == 0) tc::bulk_wait_all();  // stores complete before exit
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 2 * N);
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
            const cuuint64_t* strides_bytes, const cuuint32_t* box,
            CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
            CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int N, int S, int EPI, int ACT, bool BRES>
cudaError_t launch_n(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                     const ConvArgs& a, cudaStream_t s) {
    auto kern = conv_tc_kernel<N, S, EPI, ACT, BRES>;
    constexpr int smem = ConvCfg<N, S, EPI, BRES>::kSmem;
    static_assert(smem <= 227 * 1024, "shared memory per CTA");
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const long tiles = (long)a.tiles_x * a.tiles_y * a.B * ((a.cout_pad + N - 1) / N);
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    const long n_nt = (a.cout_pad + N - 1) / N;
    unsigned grid = (unsigned)(tiles < sms ? tiles : sms);  // one CTA per SM
    if (BRES) grid = (unsigned)(n_nt * (sms / n_nt > 0 ? sms / n_nt : 1));  // whole groups
    kern<<<grid, kConvThreads, smem, s>>>(ma, mb, mo, a);
    return cudaGetLastError();
}

template <int EPI, int ACT>
cudaError_t launch_act(int n, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                       const ConvArgs& a, cudaStream_t s) {
    const bool bres = a.ks == 1 && a.cin_pad <= kBResChunks * kKC;
    if (bres) {
        switch (n) {
            case 256: return launch_n<256, 6, EPI, ACT, true>(ma, mb, mo, a, s);
            case 128: return launch_n<128, 8, EPI, ACT, true>(ma, mb, mo, a, s);
            default: return launch_n<64, 8, EPI, ACT, true>(ma, mb, mo, a, s);
        }
    }
    switch (n) {
        case 256: return launch_n<256, 3, EPI, ACT, false>(ma, mb, mo, a, s);
        case 128: return launch_n<128, 5, EPI, ACT, false>(ma, mb, mo, a, s);
        default: return launch_n<64, 6, EPI, ACT, false>(ma, mb, mo, a, s);
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
    // planar outputs: a 4-D map (W, H, cout, B) over the output, written by each
    // epilogue warp as pw x ph pixels x 32 channels boxes
    CUtensorMap mo = ma;  // unused by the other epilogues
    if (L.epi == ConvEpi::PLANAR16 || L.epi == ConvEpi::PLANAR32) {
        const int es = L.epi == ConvEpi::PLANAR16 ? 2 : 4;
        if ((L.W * es) % 16 != 0) return cudaErrorInvalidValue;
        const int pw = a.tw < 32 ? a.tw : 32;
        const cuuint64_t dims_o[4] = {(cuuint64_t)L.W, (cuuint64_t)L.H, (cuuint64_t)L.cout,
                                      (cuuint64_t)L.B};
        const cuuint64_t str_o[3] = {(cuuint64_t)L.W * es, (cuuint64_t)L.H * L.W * es,
                                     (cuuint64_t)L.cout * L.H * L.W * es};
        const cuuint32_t box_o[4] = {(cuuint32_t)pw, (cuuint32_t)(32 / pw), 32, 1};
        if (!encode(&mo, L.y, 4, dims_o, str_o, box_o,
                    es == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    }
    switch (L.epi) {
        case ConvEpi::NHWC:
            switch (L.act) {
                case 0: return launch_act<(int)ConvEpi::NHWC, 0>(n, ma, mb, mo, a, s);
                case 1: return launch_act<(int)ConvEpi::NHWC, 1>(n, ma, mb, mo, a, s);
                case 2: return launch_act<(int)ConvEpi::NHWC, 2>(n, ma, mb, mo, a, s);
                case 3: return launch_act<(int)ConvEpi::NHWC, 3>(n, ma, mb, mo, a, s);
                default: return cudaErrorInvalidValue;
            }
        case ConvEpi::PLANAR16: return launch_act<(int)ConvEpi::PLANAR16, 0>(n, ma, mb, mo, a, s);
        case ConvEpi::PLANAR32: return launch_act<(int)ConvEpi::PLANAR32, 0>(n, ma, mb, mo, a, s);
        case ConvEpi::GRU_ZR: return launch_act<(int)ConvEpi::GRU_ZR, 0>(n, ma, mb, mo, a, s);
        case ConvEpi::GRU_Q: return launch_act<(int)ConvEpi::GRU_Q, 0>(n, ma, mb, mo, a, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace bvml
