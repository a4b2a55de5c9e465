// Implicit-GEMM 2-D convolution on the 5th-generation tensor cores (sm_100a):
// the dense convolutions of the refine stage's ConvGRU and prediction heads
// (src/dsine_refine.cpp:95-158: 5x5 pad 2, 3x3 pad 1, 1x1), which the
// reference runs as brotensor conv2d_forward calls followed by separate
// activation, concat and elementwise passes.
//
// Layout: inputs NHWC fp16 with the channel count padded to a multiple of 64
// (pad channels zero), weights [tap][C_out_pad][C_in_pad] fp16 (K-major
// rows), fp32 bias, fp32 accumulation in tensor memory.
//
// GEMM view: M = pixels, N = output channels, K = taps x input channels. A
// persistent CTA (one per SM) walks tiles of MT sub-tiles of 128 pixels (tw x
// th each, stacked vertically) by N output channels (64, 128, 192 or 256):
//  * warp 0 (one lane) streams operands with TMA into two rings: halo tiles
//    (one 4-D box per 64-channel chunk and filter column; coordinates outside
//    the frame read zeros, the convolution's zero padding; every filter row
//    reuses the same copy at a whole-image-row offset) and per-tap weight
//    tiles, both 128-byte swizzled; 1x1 layers keep their weights resident;
//  * warp 1 allocates TMEM and one lane issues tcgen05.mma (M = 128, K = 16)
//    into two accumulator sets, committing each ring entry back to the
//    producer and each finished tile to the epilogue;
//  * warps 2-9 drain the other accumulator set with tcgen05.ld while the next
//    tile accumulates: bias, an optional per-pixel addend (the hoisted terms
//    of the refine stage), activation or the GRU gate arithmetic, and stores
//    (NHWC and planar outputs through per-warp shared-memory staging and TMA
//    stores; the GRU tensors in coalesced channel-group layouts).
// All waits are bounded (tc_common.cuh); a wait that gives up sets *err and
// the CTA tears down after its copies and MMAs in flight have completed. The
// pipeline waits' bound is a launch argument (ConvLaunch::wait_limit, default
// kWaitLimit); the teardown waits for work already in flight keep kWaitLimit.
#include <cuda_fp16.h>

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
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter (see the epilogue)
constexpr uint32_t kWaitLimit = 1u << 22;

struct ConvArgs {
    int B, H, W;
    int cin_off, cin_pad, cout, cout_pad;  // input channel slice, output channels
    int ks, pad;
    int tw, th, tiles_x, tiles_y;
    const float* bias;
    const float* bias1;  // head tail: the first layer's bias (128)
    int* err;
    uint32_t wait_limit;  // attempts of a pipeline wait before it gives up (mbar_wait_pipe)
    // epilogue targets (see ConvEpi)
    void* out;
    int out_c, out_off;
    float* h32;
    __half* z;
    __half* rh;
    int rh_c;
    __half* hx;
    int hx_c;
    __half* hin;
    int hin_c;
    int obox;     // NHWC outputs: channels per TMA store (64: two chunks, 128-byte rows)
    int xchunks;  // extra K: 64-channel chunks of a 1x1 term xin . wx^T (0: none)
    int x_bytes;  // bytes of one extra-K A box (the tile's pixels, no halo)
    int planar_direct;  // planar rows not a multiple of 16 bytes: plain stores, no TMA
    // optional per-pixel addend in channel groups of 4 (C4, see load_addend)
    const float* add;
    long add_fs;  // frame stride in floats (0: one frame shared by all)
    // shared-memory plan (see below)
    int a_bytes, b_bytes;  // one A entry (halo tile), one B entry (one tap's weights)
    int s_a, s_b;          // ring depths
    int off_b, off_out, off_bias, off_bar;
};

template <int ACT>
__device__ __forceinline__ float activate(float v) {
    if constexpr (ACT == 1) return fmaxf(v, 0.0f);
    else if constexpr (ACT == 2) return __fdividef(1.0f, 1.0f + __expf(-v));  // 0 as e^-v -> inf
    else if constexpr (ACT == 3) return tanhf(v);
    else return v;
}

// Channel-group layouts of the fp32 / fp16 per-pixel tensors the epilogues
// read and write (the addend, the GRU state h32 and gate z): C4 fp32 is
// [frame][C / 4][H][W][4], C8 fp16 is [frame][C / 8][H][W][8]. A thread owns
// one pixel and moves 16 bytes per access; the lanes of a warp hold
// consecutive pixels, so every access is one coalesced 512-byte segment.
__device__ __forceinline__ long c4_index(const ConvArgs& a, long frame_groups, int b, int g,
                                         int p) {
    return ((long)b * frame_groups + g) * ((long)a.H * a.W) + p;
}

// The addend of one thread's pixel p for channels cb .. cb+31 into t (zeros
// where there is none). Issued ahead of use: the epilogue loads chunk k + 1
// while it finishes chunk k, and a tile's first chunk before waiting for its
// accumulator, so the loads' latency overlaps other work.
__device__ __forceinline__ void load_addend(const ConvArgs& a, bool in, int b, int p, int cb,
                                            float (&t)[32]) {
    if (a.add && in && cb < a.cout) {
        const long hw = (long)a.H * a.W;
        const float4* ad = reinterpret_cast<const float4*>(a.add + b * a.add_fs) +
                           (long)(cb / 4) * hw + p;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = cb + 4 * q < a.cout ? __ldg(ad + q * hw) : make_float4(0, 0, 0, 0);
            t[4 * q + 0] = v.x;
            t[4 * q + 1] = v.y;
            t[4 * q + 2] = v.z;
            t[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = 0.0f;
    }
}

// The GRU state h (C4 fp32) a GRU epilogue chunk needs, into t: for GRU_ZR
// the r channels' h (cb in [64, 128): h channels cb - 64 ..), for GRU_Q the
// updated channels' h (cb < 64). Prefetched like the addend of the other
// modes, through the same buffers.
template <int EPI>
__device__ __forceinline__ void load_gru_state(const ConvArgs& a, bool in, int b, int p, int cb,
                                               float (&t)[32]) {
    const int hc = EPI == (int)ConvEpi::GRU_ZR ? cb - 64 : cb;
    if (in && hc >= 0 && hc < 64) {
        const long hw = (long)a.H * a.W;
        const float4* h4 = reinterpret_cast<const float4*>(a.h32) + c4_index(a, 16, b, hc / 4, p);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 v = h4[q * hw];
            t[4 * q + 0] = v.x;
            t[4 * q + 1] = v.y;
            t[4 * q + 2] = v.z;
            t[4 * q + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = 0.0f;
    }
}

// f[i] = accumulator + bias + addend t for channels cb + i < cout, else 0.
// sbias: the bias staged in shared memory, zero past cout (float4 broadcasts).
__device__ __forceinline__ void pre_activation(const ConvArgs& a, const float* sbias,
                                               const float (&t)[32], int cb,
                                               const uint32_t (&v)[32], float (&f)[32]) {
    const float4* b4 = reinterpret_cast<const float4*>(sbias + cb);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 bq = b4[q];
        f[4 * q + 0] = __uint_as_float(v[4 * q + 0]) + bq.x + t[4 * q + 0];
        f[4 * q + 1] = __uint_as_float(v[4 * q + 1]) + bq.y + t[4 * q + 1];
        f[4 * q + 2] = __uint_as_float(v[4 * q + 2]) + bq.z + t[4 * q + 2];
        f[4 * q + 3] = __uint_as_float(v[4 * q + 3]) + bq.w + t[4 * q + 3];
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (cb + i >= a.cout) f[i] = 0.0f;
}

// Epilogue of one thread's pixel p of frame b for 32 consecutive output
// channels cb .. cb+31 (accumulators in v, plus bias and the addend t).
// Modes (ConvEpi in bvml_internal.h):
//  (NHWC: act(v) as fp16 at out[pix * out_c + out_off + c], zeros past cout,
//  through shared memory and TMA stores: nhwc_chunk_tma, nhwc_pair_tma)
//  C4_32     act(v) as fp32 in C4 layout, out_c channels per frame, at
//            channel out_off + c;
//  (SPLIT16: v as two fp16 halves (hi, lo = v - hi), per 64-channel block
//  hi then lo, at NHWC channels out_off + 128 (c / 64) + c % 64 and 64
//  further, through shared memory and TMA stores; an operand for the extra K
//  of another convolution that keeps about 16 mantissa bits)
//  (PLANAR16/32: planar_chunk_tma, through a shared-memory transpose)
//  GRU_ZR    c < 64: z = sigmoid(v) -> z (C8 fp16, 64 channels);
//            64 <= c < 128: r = sigmoid(v) -> rh[pix * rh_c + c - 64] = r * h,
//            h from h32 (C4 fp32, 64 channels);
//  GRU_Q     c < 64: q = tanh(v), h = (1 - z) h + z q -> h32 and fp16 copies
//            at hx[pix * hx_c + c] and, if set, hin[pix * hin_c + c]
//  (src/dsine_refine.cpp:140-158).
template <int EPI, int ACT>
__device__ __forceinline__ void epilogue32(const ConvArgs& a, const float* sbias, int b, int p,
                                           int cb, const float (&t)[32],
                                           const uint32_t (&v)[32]) {
    // GRU modes: t holds the GRU state h of these channels (prefetched), not
    // an addend; the other modes: t is the addend
    constexpr bool kGru = EPI == (int)ConvEpi::GRU_ZR || EPI == (int)ConvEpi::GRU_Q;
    float f[32];
    if constexpr (kGru) {
        float zero[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) zero[i] = 0.0f;
        pre_activation(a, sbias, zero, cb, v, f);
    } else {
        pre_activation(a, sbias, t, cb, v, f);
    }
    const long hw = (long)a.H * a.W;
    const long pix = b * hw + p;
    if constexpr (EPI == (int)ConvEpi::C4_32) {
        float4* dst = reinterpret_cast<float4*>(a.out) +
                      c4_index(a, a.out_c / 4, b, (a.out_off + cb) / 4, p);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 o;
            o.x = cb + 4 * q + 0 < a.cout ? activate<ACT>(f[4 * q + 0]) : 0.0f;
            o.y = cb + 4 * q + 1 < a.cout ? activate<ACT>(f[4 * q + 1]) : 0.0f;
            o.z = cb + 4 * q + 2 < a.cout ? activate<ACT>(f[4 * q + 2]) : 0.0f;
            o.w = cb + 4 * q + 3 < a.cout ? activate<ACT>(f[4 * q + 3]) : 0.0f;
            dst[q * hw] = o;
        }
    } else if constexpr (EPI == (int)ConvEpi::GRU_ZR) {
        alignas(16) __half o[32];
        if (cb < 64) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float2half_rn(activate<2>(f[i]));
            uint4* dst = reinterpret_cast<uint4*>(a.z) + c4_index(a, 8, b, cb / 8, p);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q * hw] = reinterpret_cast<const uint4*>(o)[q];
        } else if (cb < 128) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 h = make_float4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
                o[4 * q + 0] = __float2half_rn(activate<2>(f[4 * q + 0]) * h.x);
                o[4 * q + 1] = __float2half_rn(activate<2>(f[4 * q + 1]) * h.y);
                o[4 * q + 2] = __float2half_rn(activate<2>(f[4 * q + 2]) * h.z);
                o[4 * q + 3] = __float2half_rn(activate<2>(f[4 * q + 3]) * h.w);
            }
            uint4* dst = reinterpret_cast<uint4*>(a.rh + pix * a.rh_c + (cb - 64));
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<const uint4*>(o)[q];
        }
    } else if constexpr (EPI == (int)ConvEpi::GRU_Q) {
        if (cb >= 64) return;
        float4* h4 = reinterpret_cast<float4*>(a.h32) + c4_index(a, 16, b, cb / 4, p);
        const uint4* z4 = reinterpret_cast<const uint4*>(a.z) + c4_index(a, 8, b, cb / 8, p);
        alignas(16) __half zb[32];
#pragma unroll
        for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(zb)[q] = z4[q * hw];
        alignas(16) __half o[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 h = make_float4(t[4 * q], t[4 * q + 1], t[4 * q + 2], t[4 * q + 3]);
            float* hh = reinterpret_cast<float*>(&h);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = 4 * q + e;
                const float z = __half2float(zb[i]);
                hh[e] = fmaf(z, tanhf(f[i]) - hh[e], hh[e]);  // (1 - z) h + z q
                o[i] = __float2half_rn(hh[e]);
            }
            h4[q * hw] = h;
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

// Shared-memory plan (byte offsets from the 1024-aligned base), decided on
// the host per launch:
//  * A ring, s_a entries of a_bytes: one halo tile each -- tw pixels x
//    (MT * th + ks - 1) image rows x 64 channels, 128-byte swizzled. Rows are
//    stored image row by image row, so the operand of sub-tile m and filter
//    row ky starts (m * th + ky) image rows in: tw * 128 bytes per image row,
//    a multiple of the 1024-byte swizzle atom (tw >= 8), and every filter
//    row reuses the same copy;
//  * B ring, s_b entries of N x 64 weights (one tap), or, for BRES, the
//    layer's whole 1x1 weights resident (chunks entries, loaded once);
//  * planar staging (PLANAR epilogues), then the barriers.
constexpr int kMaxStages = 8;
constexpr int kBarBytes = 512;
constexpr int kSmemLimit = 227 * 1024;

// BRES (1x1 convolutions with at most kBResChunks input chunks): the CTA's
// weights stay resident in shared memory, loaded once, and the ring carries
// only pixel tiles; each CTA then keeps one output-channel tile.
constexpr int kBResChunks = 2;

// planar outputs: per epilogue warp two 32-channel x 32-pixel staging buffers
__host__ __device__ constexpr int stage_warp_bytes(int epi) {
    return 32 * 32 * (epi == (int)ConvEpi::PLANAR32 ? 4 : 2);  // NHWC, PLANAR16: 2 bytes
}

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
                                                 const float* sbias, const float (&t)[32],
                                                 const uint32_t (&v)[32]) {
    float f[32];
    pre_activation(a, sbias, t, cb, v, f);
    if (a.planar_direct) {
        // rows the TMA cannot address (W x element size not a multiple of 16
        // bytes): each channel's 32 pixels as plain stores, coalesced across
        // the warp's consecutive pixels
        const int pw = a.tw < 32 ? a.tw : 32;
        const int px = px0 + lane % pw, py = py0 + lane / pw;
        if (px < a.W && py < a.H) {
            const long hw = (long)a.H * a.W;
            TO* o = static_cast<TO*>(a.out) + ((long)b * a.cout + cb) * hw + (long)py * a.W + px;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (cb + i < a.cout) {
                    if constexpr (sizeof(TO) == 2) o[i * hw] = __float2half_rn(f[i]);
                    else o[i * hw] = f[i];
                }
            }
        }
        return;
    }
    if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's previous store has read it
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if constexpr (sizeof(TO) == 2) stg[i * 32 + lane] = __float2half_rn(f[i]);
        else stg[i * 32 + lane] = f[i];
    }
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        // a TMA store's innermost coordinate must start on 16 bytes, and no
        // store may start at a negative coordinate
        if (check_ok((px0 * (int)sizeof(TO)) % 16 == 0 && px0 >= 0 && py0 >= 0, kChkConvTma))
            tc::tma_store_4d(map_o, stg_addr, px0, py0, cb, b);
        tc::bulk_commit();
    }
}

// NHWC fp16 output of one 32-channel chunk of one epilogue warp's 32 pixels
// through shared memory: lane r writes its pixel's 64 bytes as row r of the
// warp's staging buffer ([pixel][channel], the TMA box layout) in the
// 64-byte swizzle (16-byte unit u of row r at u ^ ((r >> 1) & 3), which
// spreads a warp's rows over all banks), and lane 0 stores the box (32
// channels at c0 x pw x ph pixels) with one TMA store, clipped at the frame
// edges. The buffer is reused two chunks later, after the store has read it.
__device__ __forceinline__ void stage_f16_box(const CUtensorMap* map_o, uint8_t* stg,
                                               uint32_t stg_addr, int lane, int c0, int px0,
                                               int py0, int b, const __half (&o)[32]) {
    if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's previous store has read it
    __syncwarp();
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(stg + lane * 64 + ((q ^ sw) << 4)) =
            reinterpret_cast<const uint4*>(o)[q];
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (check_ok(c0 % 8 == 0 && c0 >= 0 && px0 >= 0 && py0 >= 0, kChkConvTma))
            tc::tma_store_4d(map_o, stg_addr, c0, px0, py0, b);
        tc::bulk_commit();
    }
}

template <int ACT>
__device__ __forceinline__ void nhwc_chunk_tma(const ConvArgs& a, const CUtensorMap* map_o,
                                               uint8_t* stg, uint32_t stg_addr, int lane, int c0,
                                               int px0, int py0, int b, int cb,
                                               const float* sbias, const float (&t)[32],
                                               const uint32_t (&v)[32]) {
    float f[32];
    pre_activation(a, sbias, t, cb, v, f);
    alignas(16) __half o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        o[i] = __float2half_rn(cb + i < a.cout ? activate<ACT>(f[i]) : 0.0f);
    stage_f16_box(map_o, stg, stg_addr, lane, c0, px0, py0, b, o);
}

// NHWC fp16 output of two consecutive 32-channel chunks (half 0: channels
// cb .. cb+31, half 1: the next 32) of one epilogue warp's 32 pixels, stored
// as one box of 64 channels: 128-byte rows, half as many as 32-channel boxes
// (the TMA store engine's cost is per row). Lane r writes its half row into
// row r of one of the warp's two 4 KB staging buffers (alternating per
// pair) in the 128-byte swizzle (16-byte unit u at u ^ (r & 7)); lane 0
// stores after half 1, and waits before half 0 until the store that used
// this buffer two pairs ago has read it.
template <int ACT>
__device__ __forceinline__ void nhwc_pair_tma(const ConvArgs& a, const CUtensorMap* map_o,
                                              uint8_t* stg, uint32_t stg_addr, int lane, int half,
                                              int c0, int px0, int py0, int b, int cb,
                                              const float* sbias, const float (&t)[32],
                                              const uint32_t (&v)[32]) {
    float f[32];
    pre_activation(a, sbias, t, cb, v, f);
    alignas(16) __half o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        o[i] = __float2half_rn(cb + i < a.cout ? activate<ACT>(f[i]) : 0.0f);
    if (half == 0) {
        if (lane == 0) tc::bulk_wait_read<1>();  // this buffer's previous store has read it
        __syncwarp();
    }
    const int sw = lane & 7;
#pragma unroll
    for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(stg + lane * 128 + (((half * 4 + q) ^ sw) << 4)) =
            reinterpret_cast<const uint4*>(o)[q];
    if (half == 1) {
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (check_ok((c0 - 32) % 8 == 0 && c0 >= 32 && px0 >= 0 && py0 >= 0, kChkConvTma))
                tc::tma_store_4d(map_o, stg_addr, c0 - 32, px0, py0, b);
            tc::bulk_commit();
        }
    }
}

// Persistent: CTA c computes tiles c, c + G, c + 2G, ... (G CTAs, one per
// SM). A tile is MT sub-tiles of 128 pixels (tw x th, stacked vertically)
// by N output channels; each sub-tile has its own TMEM accumulator, so one
// weight tile feeds MT MMAs. The TMA / MMA rings run on across tiles; the
// accumulators are double buffered in TMEM (2 x MT x N columns), so the
// epilogue warps drain tile i while the MMA lane accumulates tile i + 1.
template <int N, int MT, int EPI, int ACT, bool BRES>
__global__ void __launch_bounds__(kConvThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_x,
               const __grid_constant__ CUtensorMap map_bx, const ConvArgs a) {
    constexpr bool kPlanar = EPI == (int)ConvEpi::PLANAR16 || EPI == (int)ConvEpi::PLANAR32;
    constexpr bool kStaged =  // TMA-store epilogues
        kPlanar || EPI == (int)ConvEpi::NHWC || EPI == (int)ConvEpi::SPLIT16;
    // TMEM columns: two accumulator sets, allocated as a power of two >= 32
    constexpr int kCols = 2 * MT * N <= 128 ? 128 : (2 * MT * N <= 256 ? 256 : 512);
    static_assert(2 * MT * N <= 512, "TMEM allocation");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bars = sbase + a.off_bar;
    const uint32_t bar_full_a = bars;                 // kMaxStages: A entry loaded
    const uint32_t bar_empty_a = bars + 64;           // kMaxStages: A entry consumed
    const uint32_t bar_full_b = bars + 128;           // kMaxStages: B entry loaded
    const uint32_t bar_empty_b = bars + 192;          // kMaxStages: B entry consumed
    const uint32_t bar_acc_full = bars + 256;         // 2: accumulator set ready
    const uint32_t bar_acc_empty = bars + 272;        // 2: accumulator set drained
    const uint32_t bar_end = bars + 288;              // every MMA complete
    const uint32_t bar_bres = bars + 296;             // resident weights loaded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_bar + 304);
    int* abort_flag = reinterpret_cast<int*>(smem + a.off_bar + 308);
    const uint32_t ring_b = sbase + a.off_b;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = a.cin_pad / kKC;
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
        y0 = ty * a.th * MT;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            tc::mbar_init(bar_full_a + 8 * s, 1);
            tc::mbar_init(bar_empty_a + 8 * s, 1);
            tc::mbar_init(bar_full_b + 8 * s, 1);
            tc::mbar_init(bar_empty_b + 8 * s, 1);
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
        tc::tmem_alloc(tc::smem_u32(tmem_slot), kCols);
        tc::tmem_relinquish();
    }
    float* sbias = reinterpret_cast<float*>(smem + a.off_bias);
    for (int c = threadIdx.x; c < a.cout_pad; c += blockDim.x)
        sbias[c] = c < a.cout ? a.bias[c] : 0.0f;
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
        int ga = 0, gb = 0;  // A and B entries issued by this CTA
        if (!check_ok(a.cin_off % 8 == 0, kChkConvTma)) fail(8);
        if constexpr (BRES) {  // the CTA's weights, once
            tc::mbar_expect_tx(bar_bres, chunks * a.b_bytes);
            for (int ch = 0; ch < chunks; ++ch)
                tc::tma_load_3d(ring_b + ch * a.b_bytes, &map_b, bar_bres, ch * kKC, my_nt * N, 0);
        }
        bool ok = true;
        for (int t = t0; ok && t < t_end && !aborted(); t += dt) {
            int b, x0, y0, n0;
            tile_of(t, b, x0, y0, n0);
            for (int ch = 0; ok && ch < chunks; ++ch) {
                for (int kx = 0; ok && kx < a.ks; ++kx) {
                    const int s = ga % a.s_a, j = ga / a.s_a;
                    if (j > 0 && !tc::mbar_wait_pipe(bar_empty_a + 8 * s, (j - 1) & 1, a.wait_limit)) {
                        fail(1);
                        ok = false;
                        break;
                    }
                    if (aborted()) {
                        ok = false;
                        break;
                    }
                    tc::mbar_expect_tx(bar_full_a + 8 * s, a.a_bytes);
                    tc::tma_load_4d(sbase + s * a.a_bytes, &map_a, bar_full_a + 8 * s,
                                    a.cin_off + ch * kKC, x0 + kx - a.pad, y0 - a.pad, b);
                    ++ga;
                    if constexpr (!BRES) {
                        for (int ky = 0; ky < a.ks; ++ky, ++gb) {
                            const int q = gb % a.s_b, jb = gb / a.s_b;
                            if (jb > 0 &&
                                !tc::mbar_wait_pipe(bar_empty_b + 8 * q, (jb - 1) & 1, a.wait_limit)) {
                                fail(1);
                                ok = false;
                                break;
                            }
                            tc::mbar_expect_tx(bar_full_b + 8 * q, a.b_bytes);
                            tc::tma_load_3d(ring_b + q * a.b_bytes, &map_b, bar_full_b + 8 * q,
                                            ch * kKC, n0, ky * a.ks + kx);
                        }
                    }
                }
            }
            if constexpr (!BRES) {
                // extra K: the tile's pixels of xin (no halo) and the weights wx,
                // through the same rings
                for (int xc = 0; ok && xc < a.xchunks; ++xc) {
                    const int s = ga % a.s_a, j = ga / a.s_a;
                    if (j > 0 && !tc::mbar_wait_pipe(bar_empty_a + 8 * s, (j - 1) & 1, a.wait_limit)) {
                        fail(1);
                        ok = false;
                        break;
                    }
                    if (aborted()) {
                        ok = false;
                        break;
                    }
                    tc::mbar_expect_tx(bar_full_a + 8 * s, a.x_bytes);
                    tc::tma_load_4d(sbase + s * a.a_bytes, &map_x, bar_full_a + 8 * s, xc * kKC, x0,
                                    y0, b);
                    ++ga;
                    const int q = gb % a.s_b, jb = gb / a.s_b;
                    if (jb > 0 && !tc::mbar_wait_pipe(bar_empty_b + 8 * q, (jb - 1) & 1, a.wait_limit)) {
                        fail(1);
                        ok = false;
                        break;
                    }
                    tc::mbar_expect_tx(bar_full_b + 8 * q, a.b_bytes);
                    tc::tma_load_3d(ring_b + q * a.b_bytes, &map_bx, bar_full_b + 8 * q, xc * kKC,
                                    n0, 0);
                    ++gb;
                }
            }
        }
        // no copy may still be landing when the CTA exits
        for (int q = ga - a.s_a > 0 ? ga - a.s_a : 0; q < ga; ++q)
            if (!tc::mbar_wait(bar_full_a + 8 * (q % a.s_a), (q / a.s_a) & 1, kWaitLimit)) fail(2);
        if constexpr (!BRES) {
            for (int q = gb - a.s_b > 0 ? gb - a.s_b : 0; q < gb; ++q)
                if (!tc::mbar_wait(bar_full_b + 8 * (q % a.s_b), (q / a.s_b) & 1, kWaitLimit))
                    fail(2);
        }
        if (BRES && !tc::mbar_wait(bar_bres, 0, kWaitLimit)) fail(2);
    } else if (warp == 1 && lane == 0) {
        // --------------------------------------------------------------- MMA
        constexpr uint32_t idesc = tc::idesc_f16_f32(kTM, N);
        const uint32_t row_bytes = (uint32_t)a.tw * 128;  // one image row of an A entry
        int ga = 0, gb = 0, tl = 0;
        bool ok = true;
        if (BRES && t0 < t_end && !tc::mbar_wait_pipe(bar_bres, 0, a.wait_limit)) {
            fail(7);
            ok = false;
        }
        for (int t = t0; ok && t < t_end && !aborted(); t += dt, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            if (u > 0 && !tc::mbar_wait_pipe(bar_acc_empty + 8 * buf, (u - 1) & 1, a.wait_limit)) {
                fail(3);
                break;
            }
            tc::tc_fence_after();
            const uint32_t acc = tmem + buf * (MT * N);
            bool first = true;
            for (int ch = 0; ok && ch < chunks; ++ch) {
                for (int kx = 0; ok && kx < a.ks; ++kx) {
                    const int s = ga % a.s_a, j = ga / a.s_a;
                    if (!tc::mbar_wait_pipe(bar_full_a + 8 * s, j & 1, a.wait_limit) || aborted()) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = sbase + s * a.a_bytes;
                    for (int ky = 0; ky < a.ks; ++ky) {
                        int q = 0;
                        uint32_t sb;
                        if constexpr (BRES) {
                            sb = ring_b + ch * a.b_bytes;  // ks == 1
                        } else {
                            q = gb % a.s_b;
                            if (!tc::mbar_wait_pipe(bar_full_b + 8 * q, (gb / a.s_b) & 1, a.wait_limit) ||
                                aborted()) {
                                ok = false;
                                break;
                            }
                            tc::tc_fence_after();
                            sb = ring_b + q * a.b_bytes;
                        }
                        const uint64_t db = tc::umma_desc_k_sw128(sb);
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            const uint64_t da =
                                tc::umma_desc_k_sw128(sa + (uint32_t)(m * a.th + ky) * row_bytes);
#pragma unroll
                            for (int k = 0; k < kKC / 16; ++k)  // K = 16 per MMA: 2 descriptor units
                                tc::umma_f16(acc + m * N, da + 2 * k, db + 2 * k, idesc,
                                              !first || k > 0);
                        }
                        first = false;
                        if constexpr (!BRES) {
                            tc::umma_commit(bar_empty_b + 8 * q);
                            ++gb;
                        }
                    }
                    if (!ok) break;
                    tc::umma_commit(bar_empty_a + 8 * s);
                    ++ga;
                }
            }
            if constexpr (!BRES) {
                for (int xc = 0; ok && xc < a.xchunks; ++xc) {  // extra K (no halo: ky = 0)
                    const int s = ga % a.s_a, j = ga / a.s_a;
                    if (!tc::mbar_wait_pipe(bar_full_a + 8 * s, j & 1, a.wait_limit) || aborted()) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = sbase + s * a.a_bytes;
                    const int q = gb % a.s_b;
                    if (!tc::mbar_wait_pipe(bar_full_b + 8 * q, (gb / a.s_b) & 1, a.wait_limit) ||
                        aborted()) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint64_t db = tc::umma_desc_k_sw128(ring_b + q * a.b_bytes);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint64_t da =
                            tc::umma_desc_k_sw128(sa + (uint32_t)(m * a.th) * row_bytes);
#pragma unroll
                        for (int k = 0; k < kKC / 16; ++k)
                            tc::umma_f16(acc + m * N, da + 2 * k, db + 2 * k, idesc,
                                          !first || k > 0);
                    }
                    first = false;
                    tc::umma_commit(bar_empty_b + 8 * q);
                    ++gb;
                    tc::umma_commit(bar_empty_a + 8 * s);
                    ++ga;
                }
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
        // MT = 1: two warps per TMEM lane quarter, each half of the columns;
        // MT >= 2: warp group g (warps 2-5, 6-9) drains sub-tiles g, g + 2, ...
        const int wq = warp & 3;              // the TMEM lane quarter this warp may read
        const int row = wq * 32 + lane;       // pixel index in the sub-tile
        const int grp = (warp - 2) >> 2;
        const int c_lo = MT == 1 ? grp * (N / 2) : 0;
        int pcount = 0;                       // TMA-stored chunks of this warp
        // this warp's chunks of a tile: sub-tiles m (MT >= 2: grp, grp + 2, ..)
        // x 32-column groups from c_lo (MT = 1: this warp's half of the columns)
        constexpr int kCPer = MT == 1 ? N / 64 : N / 32;  // column groups per sub-tile
        constexpr int kChunks = (MT == 1 ? 1 : MT / 2) * kCPer;
        int b = 0, x0 = 0, y0 = 0, n0 = 0;
        auto geo = [&](int k, int& ys, int& px, int& py, bool& in, int& c0) {
            const int m = MT == 1 ? 0 : grp + 2 * (k / kCPer);
            c0 = c_lo + 32 * (k % kCPer);
            ys = y0 + m * a.th;  // the sub-tile's first image row
            px = x0 + row % a.tw;
            py = ys + row / a.tw;
            in = px < a.W && py < a.H;
            return m;
        };
        auto prefetch = [&](int k, float (&tt)[32]) {
            int ys, px, py, c0;
            bool in;
            geo(k, ys, px, py, in, c0);
            if constexpr (EPI == (int)ConvEpi::GRU_ZR || EPI == (int)ConvEpi::GRU_Q)
                load_gru_state<EPI>(a, in, b, py * a.W + px, n0 + c0, tt);
            else
                load_addend(a, in, b, py * a.W + px, n0 + c0, tt);
        };
        auto process = [&](int k, int buf, const float (&tt)[32]) {
            int ys, px, py, c0;
            bool in;
            const int m = geo(k, ys, px, py, in, c0);
            const uint32_t acc = tmem + buf * (MT * N) + m * N + ((uint32_t)(wq * 32) << 16);
            uint32_t v[32];
            tc::tmem_ld_32cols(acc + c0, v);
            tc::tmem_ld_wait();
            const int cb = n0 + c0;
            if constexpr (kStaged) {
                if (cb >= (kPlanar ? a.cout : a.cout_pad)) return;  // the same for the whole warp
                // this warp's 32 pixels: sub-tile rows [wq * 32, wq * 32 + 32) as a
                // pw x ph box (pw = min(tw, 32))
                const int px0 = x0 + (wq * 32) % a.tw, py0 = ys + (wq * 32) / a.tw;
                if (px0 >= a.W || py0 >= a.H) return;  // the whole box is off the frame
                if constexpr (EPI == (int)ConvEpi::SPLIT16) {
                    if (cb >= a.cout) return;  // cout is a multiple of 32
                    float f[32];
                    pre_activation(a, sbias, tt, cb, v, f);
                    alignas(16) __half hi[32], lo[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        hi[i] = __float2half_rn(f[i]);
                        lo[i] = __float2half_rn(f[i] - __half2float(hi[i]));
                    }
                    const int cx = a.out_off + (cb / 64) * 128 + cb % 64;
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
                        const int slot = (warp - 2) * 2 + (pcount & 1);
                        stage_f16_box(&map_o, smem + a.off_out + slot * stage_warp_bytes(EPI),
                                       sbase + a.off_out + slot * stage_warp_bytes(EPI), lane,
                                       cx + 64 * part, px0, py0, b, part ? lo : hi);
                        ++pcount;
                    }
                    return;
                }
                if constexpr (EPI == (int)ConvEpi::NHWC) {
                    if (a.obox == 64) {  // chunk pairs share a 4 KB buffer and one store
                        const int wbase = ((warp - 2) * 2 + ((pcount >> 1) & 1)) * 4096;
                        nhwc_pair_tma<ACT>(a, &map_o, smem + a.off_out + wbase,
                                           sbase + a.off_out + wbase, lane, (c0 >> 5) & 1,
                                           a.out_off + cb, px0, py0, b, cb, sbias, tt, v);
                        ++pcount;
                        return;
                    }
                }
                const int slot = (warp - 2) * 2 + (pcount & 1);
                uint8_t* stg = smem + a.off_out + slot * stage_warp_bytes(EPI);
                const uint32_t stg_addr = sbase + a.off_out + slot * stage_warp_bytes(EPI);
                if constexpr (EPI == (int)ConvEpi::PLANAR16)
                    planar_chunk_tma<__half>(a, &map_o, reinterpret_cast<__half*>(stg), stg_addr,
                                             lane, px0, py0, b, cb, sbias, tt, v);
                else if constexpr (EPI == (int)ConvEpi::PLANAR32)
                    planar_chunk_tma<float>(a, &map_o, reinterpret_cast<float*>(stg), stg_addr,
                                            lane, px0, py0, b, cb, sbias, tt, v);
                else
                    nhwc_chunk_tma<ACT>(a, &map_o, stg, stg_addr, lane, a.out_off + cb, px0, py0,
                                        b, cb, sbias, tt, v);
                ++pcount;
            } else {
                if (!in || cb >= a.cout_pad) return;
                epilogue32<EPI, ACT>(a, sbias, b, py * a.W + px, cb, tt, v);
            }
        };
        int tl = 0;
        for (int t = t0; t < t_end; t += dt, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            tile_of(t, b, x0, y0, n0);
            float ta[32], tb[32];
            prefetch(0, ta);  // overlaps the wait for this tile's MMAs
            const bool ok = tc::mbar_wait_pipe(bar_acc_full + 8 * buf, u & 1, a.wait_limit);
            if (!ok) fail(6);
            if (!ok || aborted()) break;
            tc::tc_fence_after();
#pragma unroll 1
            for (int k = 0; k < kChunks; k += 2) {
                if (k + 1 < kChunks) prefetch(k + 1, tb);
                process(k, buf, ta);
                if (k + 1 < kChunks) {
                    if (k + 2 < kChunks) prefetch(k + 2, ta);
                    process(k + 1, buf, tb);
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(bar_acc_empty + 8 * buf);
        }
        if (kStaged && lane == 0) tc::bulk_wait_all();  // stores complete before exit
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kCols);
    }
}

// ------------------------------------------------------------ head tail
// The last two layers of a prediction head in one kernel (src/dsine_refine.cpp:
// 118-125: conv1x1 128 -> 128, ReLU, conv1x1 128 -> C with C <= 64): GEMM1 of
// a 128-pixel tile into TMEM, bias + ReLU + fp16 written by the epilogue warps
// straight into shared memory in the 128-byte-swizzled K-major layout the MMA
// reads (row r = pixel, 16-byte unit u at u ^ (r & 7)), GEMM2 from there, and
// the planar epilogue -- the 128-channel intermediate never reaches global
// memory. Both weight matrices stay resident. Everything after the operand
// loads is double buffered -- GEMM1 and GEMM2 accumulators, intermediate --
// and issued one tile apart: the MMA lane issues GEMM1 of tile i + 1 before
// GEMM2 of tile i, the epilogue warps convert tile i + 1's GEMM1 output
// before they store tile i's GEMM2 output, so neither waits on the other.
constexpr int kHTRing = 8;          // A ring entries (16 KB: 128 pixels x 64 channels)
constexpr int kHTW2 = 0;            // W2 resident: 2 chunks x 128 rows x 128 B
constexpr int kHTW4 = 32768;        // W4 resident: 2 chunks x 64 rows x 128 B
constexpr int kHTA2 = 49152;        // intermediates: 2 x (2 chunks x 128 rows x 128 B)
constexpr int kHTRingOff = 114688;  // the A ring

template <int EPI>
__global__ void __launch_bounds__(kConvThreads, 1)
head_tail_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w2,
                 const __grid_constant__ CUtensorMap map_w4, const __grid_constant__ CUtensorMap map_o,
                 const ConvArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bars = sbase + a.off_bar;
    const uint32_t bar_full_a = bars;            // kHTRing: A entry loaded
    const uint32_t bar_empty_a = bars + 64;      // kHTRing: A entry consumed
    const uint32_t bar_acc1_full = bars + 128;   // 2: GEMM1 accumulator ready
    const uint32_t bar_acc1_empty = bars + 144;  // 2: GEMM1 accumulator drained
    const uint32_t bar_a2_full = bars + 160;     // 2: intermediate written
    const uint32_t bar_acc2_full = bars + 176;   // 2: GEMM2 accumulator ready
    const uint32_t bar_acc2_empty = bars + 192;  // 2: GEMM2 accumulator drained
    const uint32_t bar_wres = bars + 208;        // resident weights loaded
    const uint32_t bar_end = bars + 216;         // every MMA complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_bar + 224);
    int* abort_flag = reinterpret_cast<int*>(smem + a.off_bar + 228);
    const int s_a = a.s_a;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = a.tiles_x * a.tiles_y * a.B;
    auto tile_of = [&](int t, int& b, int& x0, int& y0) {
        const int tx = t % a.tiles_x;
        const int r = t / a.tiles_x;
        x0 = tx * a.tw;
        y0 = (r % a.tiles_y) * a.th;
        b = r / a.tiles_y;
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kHTRing; ++s) {
            tc::mbar_init(bar_full_a + 8 * s, 1);
            tc::mbar_init(bar_empty_a + 8 * s, 1);
        }
        for (int q = 0; q < 2; ++q) {
            tc::mbar_init(bar_acc1_full + 8 * q, 1);
            tc::mbar_init(bar_acc1_empty + 8 * q, kEpiWarps);
            tc::mbar_init(bar_a2_full + 8 * q, kEpiWarps);
            tc::mbar_init(bar_acc2_full + 8 * q, 1);
            tc::mbar_init(bar_acc2_empty + 8 * q, kEpiWarps);
        }
        tc::mbar_init(bar_wres, 1);
        tc::mbar_init(bar_end, 1);
        *abort_flag = 0;
        tc::mbar_fence_init();
        tc::tma_prefetch_desc(&map_a);
    }
    if (warp == 1) {
        tc::tmem_alloc(tc::smem_u32(tmem_slot), 512);  // acc1 x 2 (256) + acc2 x 2 (128)
        tc::tmem_relinquish();
    }
    float* sbias1 = reinterpret_cast<float*>(smem + a.off_bias);
    float* sbias2 = sbias1 + 128;
    for (int c = threadIdx.x; c < 128 + 64; c += blockDim.x) {
        if (c < 128) sbias1[c] = a.bias1[c];
        else sbias2[c - 128] = c - 128 < a.cout ? a.bias[c - 128] : 0.0f;
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
        tc::mbar_expect_tx(bar_wres, 32768 + 16384);
        for (int ch = 0; ch < 2; ++ch) {
            tc::tma_load_3d(sbase + kHTW2 + ch * 16384, &map_w2, bar_wres, ch * kKC, 0, 0);
            tc::tma_load_3d(sbase + kHTW4 + ch * 8192, &map_w4, bar_wres, ch * kKC, 0, 0);
        }
        int ga = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < n_tiles && !aborted(); t += gridDim.x) {
            int b, x0, y0;
            tile_of(t, b, x0, y0);
            for (int ch = 0; ch < 2; ++ch, ++ga) {
                const int s = ga % s_a, j = ga / s_a;
                if (j > 0 && !tc::mbar_wait_pipe(bar_empty_a + 8 * s, (j - 1) & 1, a.wait_limit)) {
                    fail(1);
                    ok = false;
                    break;
                }
                tc::mbar_expect_tx(bar_full_a + 8 * s, 16384);
                tc::tma_load_4d(sbase + kHTRingOff + s * 16384, &map_a, bar_full_a + 8 * s,
                                a.cin_off + ch * kKC, x0, y0, b);
            }
        }
        for (int q = ga - s_a > 0 ? ga - s_a : 0; q < ga; ++q)  // nothing still landing
            if (!tc::mbar_wait(bar_full_a + 8 * (q % s_a), (q / s_a) & 1, kWaitLimit)) fail(2);
        if (!tc::mbar_wait(bar_wres, 0, kWaitLimit)) fail(2);
    } else if (warp == 1 && lane == 0) {
        // --------------------------------------------------------------- MMA
        constexpr uint32_t idesc1 = tc::idesc_f16_f32(kTM, 128);
        constexpr uint32_t idesc2 = tc::idesc_f16_f32(kTM, 64);
        bool ok = tc::mbar_wait_pipe(bar_wres, 0, a.wait_limit);
        if (!ok) fail(7);
        // GEMM2 of tile j: intermediate j & 1 (2 chunks) x W4^T into acc2 j & 1
        auto gemm2 = [&](int j) {
            const int q = j & 1, v = j >> 1;
            if (!tc::mbar_wait_pipe(bar_a2_full + 8 * q, v & 1, a.wait_limit) ||
                (v > 0 && !tc::mbar_wait_pipe(bar_acc2_empty + 8 * q, (v - 1) & 1, a.wait_limit)) ||
                aborted())
                return false;
            tc::tc_fence_after();
            const uint32_t acc2 = tmem + 256 + q * 64;
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                const uint64_t da =
                    tc::umma_desc_k_sw128(sbase + kHTA2 + q * 32768 + ch * 16384);
                const uint64_t db = tc::umma_desc_k_sw128(sbase + kHTW4 + ch * 8192);
#pragma unroll
                for (int k = 0; k < kKC / 16; ++k)
                    tc::umma_f16(acc2, da + 2 * k, db + 2 * k, idesc2, ch > 0 || k > 0);
            }
            tc::umma_commit(bar_acc2_full + 8 * q);
            return true;
        };
        int ga = 0, tl = 0;
        for (int t = blockIdx.x; ok && t < n_tiles && !aborted(); t += gridDim.x, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            if (u > 0 && !tc::mbar_wait_pipe(bar_acc1_empty + 8 * buf, (u - 1) & 1, a.wait_limit)) {
                fail(3);
                ok = false;
                break;
            }
            tc::tc_fence_after();
            const uint32_t acc1 = tmem + buf * 128;
            for (int ch = 0; ch < 2; ++ch, ++ga) {
                const int s = ga % s_a;
                if (!tc::mbar_wait_pipe(bar_full_a + 8 * s, (ga / s_a) & 1, a.wait_limit) || aborted()) {
                    ok = false;
                    break;
                }
                tc::tc_fence_after();
                const uint64_t da = tc::umma_desc_k_sw128(sbase + kHTRingOff + s * 16384);
                const uint64_t db = tc::umma_desc_k_sw128(sbase + kHTW2 + ch * 16384);
#pragma unroll
                for (int k = 0; k < kKC / 16; ++k)
                    tc::umma_f16(acc1, da + 2 * k, db + 2 * k, idesc1, ch > 0 || k > 0);
                tc::umma_commit(bar_empty_a + 8 * s);
            }
            if (!ok) {
                fail(4);
                break;
            }
            tc::umma_commit(bar_acc1_full + 8 * buf);
            if (tl > 0 && !gemm2(tl - 1)) {
                fail(4);
                ok = false;
                break;
            }
        }
        if (ok && tl > 0 && !gemm2(tl - 1)) fail(4);
        tc::umma_commit(bar_end);  // also after an abort: every issued MMA has completed
        if (!tc::mbar_wait(bar_end, 0, kWaitLimit)) fail(5);
    } else if (warp >= 2) {
        // ---------------------------------------------------------- epilogue
        const int wq = warp & 3, grp = (warp - 2) >> 2;
        const int row = wq * 32 + lane;  // pixel of the tile = row of the intermediate
        const float zero[32] = {};
        int pcount = 0;
        // E2 of tile j at (b, x0, y0): GEMM2 columns [32 grp, 32 grp + 32) +
        // bias, planar store
        auto e2 = [&](int j, int b, int x0, int y0) {
            const int q = j & 1;
            if (!tc::mbar_wait_pipe(bar_acc2_full + 8 * q, (j >> 1) & 1, a.wait_limit)) {
                fail(6);
                return false;
            }
            tc::tc_fence_after();
            uint32_t v[32];
            tc::tmem_ld_32cols(tmem + 256 + q * 64 + grp * 32 + ((uint32_t)(wq * 32) << 16), v);
            tc::tmem_ld_wait();
            const int cb = grp * 32;
            const int px0 = x0 + (wq * 32) % a.tw, py0 = y0 + (wq * 32) / a.tw;
            if (cb < a.cout && px0 < a.W && py0 < a.H) {
                const int slot = (warp - 2) * 2 + (pcount & 1);
                uint8_t* stg = smem + a.off_out + slot * stage_warp_bytes(EPI);
                const uint32_t stg_addr = sbase + a.off_out + slot * stage_warp_bytes(EPI);
                if constexpr (EPI == (int)ConvEpi::PLANAR16)
                    planar_chunk_tma<__half>(a, &map_o, reinterpret_cast<__half*>(stg), stg_addr,
                                             lane, px0, py0, b, cb, sbias2, zero, v);
                else
                    planar_chunk_tma<float>(a, &map_o, reinterpret_cast<float*>(stg), stg_addr,
                                            lane, px0, py0, b, cb, sbias2, zero, v);
                ++pcount;
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(bar_acc2_empty + 8 * q);
            return true;
        };
        int tl = 0, pb = 0, px = 0, py = 0;  // the previous tile's frame and origin
        bool ok = true;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tl) {
            const int buf = tl & 1, u = tl >> 1;
            if (!tc::mbar_wait_pipe(bar_acc1_full + 8 * buf, u & 1, a.wait_limit)) {
                fail(6);
                ok = false;
                break;
            }
            if (aborted()) {
                ok = false;
                break;
            }
            tc::tc_fence_after();
            int b, x0, y0;
            tile_of(t, b, x0, y0);
            // E1: GEMM1 columns [64 grp, 64 grp + 64) + bias, ReLU, fp16 ->
            // intermediate buf, chunk grp, row `row` (its previous reader, GEMM2
            // of tile tl - 2, completed before this warp's E2 of that tile)
            uint8_t* a2row = smem + kHTA2 + buf * 32768 + grp * 16384 + row * 128;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t v[32];
                tc::tmem_ld_32cols(tmem + buf * 128 + grp * 64 + c * 32 + ((uint32_t)(wq * 32) << 16),
                                   v);
                tc::tmem_ld_wait();
                alignas(16) __half o[32];
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    o[i] = __float2half_rn(
                        fmaxf(__uint_as_float(v[i]) + sbias1[grp * 64 + c * 32 + i], 0.0f));
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<uint4*>(a2row + (((c * 4 + q) ^ (row & 7)) << 4)) =
                        reinterpret_cast<const uint4*>(o)[q];
            }
            tc::fence_proxy_async_smem();  // the MMA reads the intermediate through the async proxy
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                tc::mbar_arrive(bar_a2_full + 8 * buf);
                tc::mbar_arrive(bar_acc1_empty + 8 * buf);
            }
            if (tl > 0 && !e2(tl - 1, pb, px, py)) {
                ok = false;
                break;
            }
            pb = b;
            px = x0;
            py = y0;
        }
        if (ok && tl > 0) e2(tl - 1, pb, px, py);
        if (lane == 0) tc::bulk_wait_all();  // stores complete before exit
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------- host side
bool encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
            const cuuint64_t* strides_bytes, const cuuint32_t* box,
            CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
            CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
    return tma_encode(m, base, rank, dims, strides_bytes, box, dt, sw);
}

template <int N, int MT, int EPI, int ACT, bool BRES>
cudaError_t launch_n(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo,
                     const CUtensorMap& mx, const CUtensorMap& mbx, const ConvArgs& a, int smem,
                     cudaStream_t s) {
    auto kern = conv_tc_kernel<N, MT, EPI, ACT, BRES>;
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
    kern<<<grid, kConvThreads, smem, s>>>(ma, mb, mo, mx, mbx, a);
    return cudaGetLastError();
}

template <int EPI, int ACT>
cudaError_t launch_act(int n, int mt, bool bres, const CUtensorMap& ma, const CUtensorMap& mb,
                       const CUtensorMap& mo, const CUtensorMap& mx, const CUtensorMap& mbx,
                       const ConvArgs& a, int smem, cudaStream_t s) {
    if (bres) {
        switch (n) {
            case 256: return launch_n<256, 1, EPI, ACT, true>(ma, mb, mo, mx, mbx, a, smem, s);
            case 192: return launch_n<192, 1, EPI, ACT, true>(ma, mb, mo, mx, mbx, a, smem, s);
            case 128: return launch_n<128, 1, EPI, ACT, true>(ma, mb, mo, mx, mbx, a, smem, s);
            default: return launch_n<64, 1, EPI, ACT, true>(ma, mb, mo, mx, mbx, a, smem, s);
        }
    }
    if (n == 256) return launch_n<256, 1, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
    if (n == 192) return launch_n<192, 1, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
    if (n == 128) {
        if (mt == 2) return launch_n<128, 2, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
        return launch_n<128, 1, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
    }
    if (mt == 4) return launch_n<64, 4, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
    if (mt == 2) return launch_n<64, 2, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
    return launch_n<64, 1, EPI, ACT, false>(ma, mb, mo, mx, mbx, a, smem, s);
}

// Tile geometry and shared-memory plan for one launch: sub-tile tw x th
// (= 128 pixels), MT sub-tiles per CTA tile, ring depths. Returns the dynamic
// shared-memory size, or 0 if nothing fits.
int plan_conv(ConvArgs& a, int n, int& mt, bool bres, int out_bytes) {
    const int bias_bytes = (a.cout_pad * 4 + 127) / 128 * 128;
    const int budget = kSmemLimit - 1024 - kBarBytes - out_bytes - bias_bytes;  // 1024: alignment
    const int b_bytes = n * kKC * 2;
    for (; mt >= 1; mt /= 2) {
        // the tw with the fewest computed pixels; for ks > 1 tw = 128 is not
        // used (its halo) and ties go to 32 (128-byte rows for the epilogue's
        // planar reads and stores, a moderate halo)
        static const int tws1[4] = {128, 64, 32, 16};
        static const int tws3[3] = {32, 64, 16};
        const int* tws = a.ks > 1 ? tws3 : tws1;
        const int ntw = a.ks > 1 ? 3 : 4;
        long best = -1;
        for (int i = 0; i < ntw; ++i) {
            const int tw = tws[i];
            const int th = kTM / tw;
            const long tiles = (long)((a.W + tw - 1) / tw) * ((a.H + th * mt - 1) / (th * mt));
            if (best < 0 || tiles < best) {
                best = tiles;
                a.tw = tw;
                a.th = th;
            }
        }
        a.tiles_x = (a.W + a.tw - 1) / a.tw;
        a.tiles_y = (a.H + a.th * mt - 1) / (a.th * mt);
        a.a_bytes = a.tw * (mt * a.th + a.ks - 1) * kKC * 2;
        a.b_bytes = b_bytes;
        if (bres) {
            const int rest = budget - (a.cin_pad / kKC) * b_bytes;
            a.s_a = rest / a.a_bytes < kMaxStages ? rest / a.a_bytes : kMaxStages;
            a.s_b = 0;
            if (a.s_a < 2) continue;
            a.off_b = a.s_a * a.a_bytes;
            a.off_out = a.off_b + (a.cin_pad / kKC) * b_bytes;
        } else if (a.ks == 1) {
            const int st = budget / (a.a_bytes + b_bytes);
            a.s_a = a.s_b = st < kMaxStages ? st : kMaxStages;
            if (a.s_a < 2) continue;
            a.off_b = a.s_a * a.a_bytes;
            a.off_out = a.off_b + a.s_b * b_bytes;
        } else {
            // a few halo tiles, and as many weight taps as fit (up to 8)
            a.s_a = 3 * a.a_bytes + kMaxStages * b_bytes <= budget ? 3 : 2;
            const int sb = (budget - a.s_a * a.a_bytes) / b_bytes;
            a.s_b = sb < kMaxStages ? sb : kMaxStages;
            if (a.s_b < 2) continue;
            a.off_b = a.s_a * a.a_bytes;
            a.off_out = a.off_b + a.s_b * b_bytes;
        }
        a.off_bias = a.off_out + out_bytes;
        a.off_bar = a.off_bias + bias_bytes;
        return a.off_bar + kBarBytes + 1024;
    }
    return 0;
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda); false when the driver lacks it or refuses the map.
bool tma_encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapDataType dt,
                CUtensorMapSwizzle sw) {
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
    if (!fn) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return fn(m, dt, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
    a.wait_limit = L.wait_limit ? L.wait_limit : kWaitLimit;
    a.out = L.y;
    a.out_c = L.out_c;
    a.out_off = L.out_off;
    a.h32 = L.h32;
    a.z = static_cast<__half*>(L.z);
    a.rh = static_cast<__half*>(L.rh);
    a.rh_c = L.rh_c;
    a.hx = static_cast<__half*>(L.hx);
    a.hx_c = L.hx_c;
    a.hin = static_cast<__half*>(L.hin);
    a.hin_c = L.hin_c;
    a.add = L.add;
    a.add_fs = L.add_shared ? 0 : (long)L.H * L.W * L.add_c;
    // N: output channels per tile. GRU gates need every channel of a pixel in
    // one CTA (z with r, q with z). Filters wider than 1x1 with N < 256 use 2
    // or 4 sub-tiles per CTA tile, so one weight tile feeds 256 or 512 pixels
    // and the halo tile is shared by more filter rows.
    // Among 256, 192, 128, 64 (in that order of preference) the N that pads
    // cout_pad the least: 576 channels as 3 x 192, not 256 + 256 + 64.
    int n = 64;
    {
        long waste = -1;
        for (int cand : {256, 192, 128, 64}) {
            if (cand > 64 && cand > L.cout_pad) continue;
            const long w = (long)(L.cout_pad + cand - 1) / cand * cand - L.cout_pad;
            if (waste < 0 || w < waste) {
                waste = w;
                n = cand;
            }
        }
    }
    if (L.epi == ConvEpi::GRU_ZR) n = 128;
    if (L.epi == ConvEpi::GRU_Q) n = 64;
    int mt = L.ks == 1 || n >= 192 ? 1 : (n == 128 ? 2 : 4);
    // resident weights (1x1, few input chunks) unless an extra K block is given
    const bool bres = L.ks == 1 && L.cin_pad <= kBResChunks * kKC && !L.xin;
    const bool planar = L.epi == ConvEpi::PLANAR16 || L.epi == ConvEpi::PLANAR32;
    const int es = L.epi == ConvEpi::PLANAR16 ? 2 : 4;
    const bool obox64 = L.epi == ConvEpi::NHWC && bres && n != 64 && n != 192;
    const int out_bytes = obox64 ? kEpiWarps * 2 * 4096
                          : planar || L.epi == ConvEpi::NHWC || L.epi == ConvEpi::SPLIT16
                              ? kEpiWarps * 2 * stage_warp_bytes((int)L.epi) : 0;
    const int smem = plan_conv(a, n, mt, bres, out_bytes);
    if (smem == 0) return cudaErrorInvalidConfiguration;
    if ((long)a.tiles_x * a.tiles_y * L.B * ((L.cout_pad + n - 1) / n) > 0x7fffffffL)
        return cudaErrorInvalidConfiguration;

    CUtensorMap ma, mb;
    const cuuint64_t dims_a[4] = {(cuuint64_t)L.x_c, (cuuint64_t)L.W, (cuuint64_t)L.H,
                                  (cuuint64_t)L.B};
    const cuuint64_t str_a[3] = {(cuuint64_t)L.x_c * 2, (cuuint64_t)L.W * L.x_c * 2,
                                 (cuuint64_t)L.H * L.W * L.x_c * 2};
    // the halo tile: tw pixels x (mt * th + ks - 1) rows x 64 channels
    const cuuint32_t box_a[4] = {(cuuint32_t)kKC, (cuuint32_t)a.tw,
                                 (cuuint32_t)(mt * a.th + L.ks - 1), 1};
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
    a.planar_direct = planar && (L.W * es) % 16 != 0;
    if (planar && !a.planar_direct) {
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
    } else if (L.epi == ConvEpi::NHWC || L.epi == ConvEpi::SPLIT16) {
        // NHWC fp16: a 4-D map (out_c, W, H, B); each epilogue warp stores
        // obox channels x pw x ph pixels, 64- or 128-byte swizzled in shared
        // memory. 64-channel boxes (two 4 KB buffers per warp) for the 1x1
        // layers, whose shared memory has room; they need every warp's
        // column range to be whole chunk pairs (not so for N = 64 or 192).
        a.obox = L.epi == ConvEpi::NHWC && bres && n != 64 && n != 192 ? 64 : 32;
        const int pw = a.tw < 32 ? a.tw : 32;
        const cuuint64_t dims_o[4] = {(cuuint64_t)L.out_c, (cuuint64_t)L.W, (cuuint64_t)L.H,
                                      (cuuint64_t)L.B};
        const cuuint64_t str_o[3] = {(cuuint64_t)L.out_c * 2, (cuuint64_t)L.W * L.out_c * 2,
                                     (cuuint64_t)L.H * L.W * L.out_c * 2};
        const cuuint32_t box_o[4] = {(cuuint32_t)a.obox, (cuuint32_t)pw, (cuuint32_t)(32 / pw), 1};
        if (!encode(&mo, L.y, 4, dims_o, str_o, box_o, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    a.obox == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
    }
    // extra K: xin (B,H,W,xin_c) fp16 NHWC as boxes of the tile's pixels (no
    // halo), wx (xin_c-long rows for each of cout_pad outputs) as N x 64 boxes
    CUtensorMap mx = ma, mbx = mb;  // unused without an extra K block
    if (L.xin) {
        const cuuint64_t dims_x[4] = {(cuuint64_t)L.xin_c, (cuuint64_t)L.W, (cuuint64_t)L.H,
                                      (cuuint64_t)L.B};
        const long xs = L.xin_stride ? L.xin_stride : L.xin_c;  // channels per pixel
        const cuuint64_t str_x[3] = {(cuuint64_t)xs * 2, (cuuint64_t)L.W * xs * 2,
                                     (cuuint64_t)L.H * L.W * xs * 2};
        const cuuint32_t box_x[4] = {(cuuint32_t)kKC, (cuuint32_t)a.tw, (cuuint32_t)(mt * a.th), 1};
        const cuuint64_t dims_bx[3] = {(cuuint64_t)L.xin_c, (cuuint64_t)L.cout_pad, 1};
        const cuuint64_t str_bx[2] = {(cuuint64_t)L.xin_c * 2,
                                      (cuuint64_t)L.cout_pad * L.xin_c * 2};
        const cuuint32_t box_bx[3] = {(cuuint32_t)kKC, (cuuint32_t)n, 1};
        if (!encode(&mx, L.xin, 4, dims_x, str_x, box_x) ||
            !encode(&mbx, L.wx, 3, dims_bx, str_bx, box_bx))
            return cudaErrorInvalidValue;
        a.xchunks = L.xin_c / kKC;
        a.x_bytes = kKC * 2 * a.tw * mt * a.th;
    }
    switch (L.epi) {
        case ConvEpi::SPLIT16: return launch_act<(int)ConvEpi::SPLIT16, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
        case ConvEpi::NHWC:
            switch (L.act) {
                case 0: return launch_act<(int)ConvEpi::NHWC, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                case 1: return launch_act<(int)ConvEpi::NHWC, 1>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                case 2: return launch_act<(int)ConvEpi::NHWC, 2>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                case 3: return launch_act<(int)ConvEpi::NHWC, 3>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                default: return cudaErrorInvalidValue;
            }
        case ConvEpi::C4_32:
            switch (L.act) {
                case 0: return launch_act<(int)ConvEpi::C4_32, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                case 1: return launch_act<(int)ConvEpi::C4_32, 1>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
                default: return cudaErrorInvalidValue;
            }
        case ConvEpi::PLANAR16: return launch_act<(int)ConvEpi::PLANAR16, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
        case ConvEpi::PLANAR32: return launch_act<(int)ConvEpi::PLANAR32, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
        case ConvEpi::GRU_ZR: return launch_act<(int)ConvEpi::GRU_ZR, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
        case ConvEpi::GRU_Q: return launch_act<(int)ConvEpi::GRU_Q, 0>(n, mt, bres, ma, mb, mo, mx, mbx, a, smem, s);
    }
    return cudaErrorInvalidValue;
}


cudaError_t launch_head_tail(const HeadTailLaunch& L, cudaStream_t s) {
    if (L.B == 0 || L.H == 0 || L.W == 0) return cudaSuccess;
    ConvArgs a{};
    a.B = L.B;
    a.H = L.H;
    a.W = L.W;
    a.cin_off = L.cin_off;
    a.cout = L.cout;
    a.cout_pad = 64;
    a.bias = L.b4;
    a.bias1 = L.b2;
    a.err = L.err;
    a.wait_limit = L.wait_limit ? L.wait_limit : kWaitLimit;
    a.out = L.y;
    // pixel tile: the tw with the fewest tiles (ties to the wider one)
    long best = -1;
    for (int tw : {128, 64, 32, 16}) {
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
    const int es = L.f16 ? 2 : 4;
    a.planar_direct = (L.W * es) % 16 != 0;
    // shared memory: weights, intermediate, ring, planar staging, biases, barriers
    const int stage = kEpiWarps * 2 * 32 * 32 * es;
    const int fixed = kHTRingOff + stage + 1024 + kBarBytes + 1024;  // bias 768 B, rounded
    const int ring = (kSmemLimit - fixed) / 16384;
    a.s_a = ring < kHTRing ? ring : kHTRing;
    if (a.s_a < 2) return cudaErrorInvalidConfiguration;
    a.off_out = kHTRingOff + a.s_a * 16384;
    a.off_bias = a.off_out + stage;
    a.off_bar = a.off_bias + 1024;
    const int smem = a.off_bar + kBarBytes + 1024;

    CUtensorMap ma, mw2, mw4, mo;
    const cuuint64_t dims_a[4] = {(cuuint64_t)L.x_c, (cuuint64_t)L.W, (cuuint64_t)L.H,
                                  (cuuint64_t)L.B};
    const cuuint64_t str_a[3] = {(cuuint64_t)L.x_c * 2, (cuuint64_t)L.W * L.x_c * 2,
                                 (cuuint64_t)L.H * L.W * L.x_c * 2};
    const cuuint32_t box_a[4] = {(cuuint32_t)kKC, (cuuint32_t)a.tw, (cuuint32_t)a.th, 1};
    const cuuint64_t dims_w2[3] = {128, 128, 1};
    const cuuint64_t str_w2[2] = {256, 128 * 256};
    const cuuint32_t box_w2[3] = {(cuuint32_t)kKC, 128, 1};
    const cuuint64_t dims_w4[3] = {128, 64, 1};
    const cuuint64_t str_w4[2] = {256, 64 * 256};
    const cuuint32_t box_w4[3] = {(cuuint32_t)kKC, 64, 1};
    if (!encode(&ma, L.x, 4, dims_a, str_a, box_a) || !encode(&mw2, L.w2, 3, dims_w2, str_w2, box_w2) ||
        !encode(&mw4, L.w4, 3, dims_w4, str_w4, box_w4))
        return cudaErrorInvalidValue;
    mo = ma;  // unused when the rows take plain stores
    if (!a.planar_direct) {
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
    int dev = 0, sms = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    const long tiles = (long)a.tiles_x * a.tiles_y * L.B;
    const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);
    if (L.f16) {
        auto kern = head_tail_kernel<(int)ConvEpi::PLANAR16>;
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
            cudaSuccess)
            return e;
        kern<<<grid, kConvThreads, smem, s>>>(ma, mw2, mw4, mo, a);
    } else {
        auto kern = head_tail_kernel<(int)ConvEpi::PLANAR32>;
        if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) !=
            cudaSuccess)
            return e;
        kern<<<grid, kConvThreads, smem, s>>>(ma, mw2, mw4, mo, a);
    }
    return cudaGetLastError();
}

BVML_CHECK_READER(check_word_conv)

}  // namespace bvml
