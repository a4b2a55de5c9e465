// Fused convex 8x upsample for sm_100a: softmax over the 9 taps, 3x3
// replicate-padded combine, channel L2-normalise, optional full-resolution
// RayReLU and crop, in one pass.
//
// In the reference this is three brotensor passes per iteration
// (convex_upsample_forward, l2_normalize_nchw_forward at
// src/dsine_refine.cpp:277-282, then slice2d_forward at :288-292), run in all
// five iterations although only the last result is used. Here it runs once,
// after the last AngMF iteration.
//
// Work split: a CTA owns an 8 x 64 tile of grid pixels; each warp one grid
// row of it, each lane one grid-pixel pair (x, x+1). A thread walks the 8
// sub-rows ky and, inside each, the 8 sub-columns kx: for every (ky, kx) it
// takes the pair's 9 mask logits (planes t*64 + ky*8 + kx), so after the 8
// sub-columns it holds output row 8y+ky, columns 8x .. 8x+15, contiguous, and
// writes them with 16-byte stores. The pair's 3x3 source normals (27 float2)
// stay in registers for all 64 sub-pixels.
//
// Logit staging (grid width a multiple of 16 bytes of storage): the 9 logit
// strips of a warp's row for one (ky, kx) -- planes t*64 + ky*8 + kx, t < 9,
// 64 columns -- are one box of a 4-D tensor map (columns, rows, sub-pixel
// plane, frame * 9 + tap), copied by one TMA load into a warp-private ring
// slot and counted on that slot's mbarrier. kN stages per ring (kN divides
// 8, so every slot index is a compile-time constant); one lane keeps kN - kSP
// stages in flight and refills a group's slots once the warp has read them.
// Stages are consumed in groups of kSP so that the sub-pixels of a group,
// independent dependency chains, interleave. The mbarrier waits are bounded;
// one that gives up records it in the status word (when one is given) and the
// kernel carries on without hanging. Other widths read the logits straight
// from global memory.
//
// The softmax denominator is folded into the normalise: with e_t = exp(l_t -
// max l), normalise(sum_t (e_t/S) n_t) = a / max(|a|, 1e-12 S) for
// a = sum_t e_t n_t, which is the reference's x / max(|x|, eps) exactly in
// real arithmetic. Since 1 <= S <= 9, the clamp can only act when
// |a|^2 < 8.1e-23; a sub-pixel that close is flagged, and a run with a
// flagged sub-pixel is recomputed with S summed before it is stored (one
// warp vote per 16-byte run instead of a branch per sub-pixel).
#include "bvml_common.cuh"
#include "bvml_internal.h"
#include "tc_common.cuh"

#include <atomic>

namespace bvml {
namespace {

constexpr int kUTW = 64;        // grid columns per tile (32 pairs = one warp)
constexpr int kUTH = 8;         // grid rows per tile (one per warp)
constexpr int kUThreads = 256;
constexpr uint32_t kUpWaitLimit = 1u << 22;
// Attempts per staging wait for launches that follow (bvml_upsample_wait_limit).
std::atomic<uint32_t> g_up_wait_limit{kUpWaitLimit};

// The TMA ring of one warp: kN stages of 9 x 64 logits.
template <typename TS>
struct UpRing {
    static constexpr int kN = sizeof(TS) == 2 ? 8 : 4;          // stages (divides 8)
    static constexpr int kSP = sizeof(TS) == 2 ? 4 : 1;         // stages per group
    static constexpr int kElems = 9 * kUTW;                     // elements per stage
    static constexpr uint32_t kBytes = kElems * sizeof(TS);     // a multiple of 128
    static constexpr size_t kWarpBytes = (size_t)kN * kBytes;
    static constexpr size_t kSmem = (kUThreads / 32) * (kWarpBytes + 8 * kN);
    static_assert(8 % kN == 0 && kN % kSP == 0, "slots must tile a sub-row");
    // at least one group of stages in flight: with kN == kSP the prologue
    // issues nothing and every wait targets a phase that was never started
    static_assert(kN > kSP, "the ring must keep stages in flight");
    static_assert(kBytes % 128 == 0, "stage size keeps every slot 128-byte aligned");
};

// Logits of a pixel pair in storage form: half2 for fp16 storage (their max is
// taken packed, exactly, before any conversion), float2 for fp32.
template <typename TS> struct Logit;
template <> struct Logit<float> {
    using T = float2;
    __device__ __forceinline__ static T lds(const float* p) { return *reinterpret_cast<const float2*>(p); }
    __device__ __forceinline__ static T ldg(const float* p, long d1, bool vec) {
        return vec ? St<float>::ld2s(p) : f2(St<float>::lds1(p), St<float>::lds1(p + d1));
    }
    __device__ __forceinline__ static T mx(T a, T b) { return max2(a, b); }
    __device__ __forceinline__ static float2 f(T v) { return v; }
};
template <> struct Logit<__half> {
    using T = __half2;
    __device__ __forceinline__ static T lds(const __half* p) { return *reinterpret_cast<const __half2*>(p); }
    __device__ __forceinline__ static T ldg(const __half* p, long d1, bool vec) {
        return vec ? __ldcs(reinterpret_cast<const __half2*>(p)) : __halves2half2(__ldcs(p), __ldcs(p + d1));
    }
    __device__ __forceinline__ static T mx(T a, T b) { return __hmax2(a, b); }
    __device__ __forceinline__ static float2 f(T v) { return __half22float2(v); }
};

struct UpArgs {
    int B, h, w, tiles_x, tiles_y;
    long hw;
    int crop_t, crop_l, out_h, out_w;
    bool vec_out;                   // 16-byte aligned output runs
    float ifu8, ifv8, tu8_c, tv8_c; // full-res ray: ((X+0.5)-8cu)/(8fu) = X*ifu8 + tu8_c
    int* status;                    // nonzero after a staging wait gave up (may be null)
    uint32_t wait_limit;            // attempts per staging wait; 0: give up at once
                                    // (failure injection, bvml_upsample_wait_limit)
};

// Packs two fp32 results into one 32-bit storage word for TS = half; for
// float the results are kept as they are.
template <typename TS> struct OutRun;
template <> struct OutRun<float> {
    // 4 sub-columns x 2 pixels per channel, stored after every 4 sub-columns
    float v[3][2][4];
};
template <> struct OutRun<__half> {
    __half2 v[3][2][4];  // 8 sub-columns x 2 pixels per channel, as half pairs
    float ev[3][2];      // the even sub-column's results, until the odd one packs them
};

constexpr float kL2E = 1.4426950408889634f;

// One sub-pixel of a pixel pair from its 9 logits: softmax-weighted combine of
// the 3x3 normals N, then (NORM) the L2 normalise, (RR) the full-res RayReLU.
// EXACT sums S and applies the 1e-12 S clamp; otherwise the result is a / |a|
// and `tiny` is raised where the clamp could act.
template <typename TS, bool NORM, bool RR, bool EXACT>
__device__ __forceinline__ void subpixel(const typename Logit<TS>::T (&l)[9],
                                         const float2 (&N)[9][3], const UpArgs& a, int x,
                                         int y, int ky, int kx, float2& ox, float2& oy,
                                         float2& oz, bool& tiny) {
    using L = Logit<TS>;
    const float2 m = L::f(L::mx(L::mx(L::mx(l[0], l[1]), L::mx(l[2], l[3])),
                                L::mx(L::mx(l[4], l[5]), L::mx(L::mx(l[6], l[7]), l[8]))));
    const float2 mo = mul2(m, f2(-kL2E));
    float2 ax = f2(0.f), ay = f2(0.f), az = f2(0.f);
    // softmax weights up to the factor 1/S (e_t = exp(l_t - max l))
    auto ew = [&](int tp) { return ex2_ftz2(fma2(L::f(l[tp]), f2(kL2E), mo)); };
#pragma unroll
    for (int tp = 0; tp < 9; ++tp) {
        const float2 e = ew(tp);
        ax = fma2(e, N[tp][0], ax);
        ay = fma2(e, N[tp][1], ay);
        az = fma2(e, N[tp][2], az);
    }
    if (NORM) {
        // x / max(|x|, 1e-12) for x = a / S; with 1 <= S <= 9 the clamp can
        // only act when |a| < 9e-12
        float2 l2 = fma2(ax, ax, fma2(ay, ay, mul2(az, az)));
        if constexpr (EXACT) {
            float2 S = ew(0);
#pragma unroll
            for (int tp = 1; tp < 9; ++tp) S = add2(S, ew(tp));
            const float2 se = mul2(S, f2(1e-12f));
            l2 = max2(l2, mul2(se, se));
        } else {
            tiny |= (l2.x < 8.1e-23f) | (l2.y < 8.1e-23f);
        }
        const float2 inv = rsqrt2(l2);
        ox = mul2(ax, inv);
        oy = mul2(ay, inv);
        oz = mul2(az, inv);
    } else {
        float2 S = ew(0);
#pragma unroll
        for (int tp = 1; tp < 9; ++tp) S = add2(S, ew(tp));
        const float2 inv = f2(__frcp_rn(S.x), __frcp_rn(S.y));
        ox = mul2(ax, inv);
        oy = mul2(ay, inv);
        oz = mul2(az, inv);
    }
    if (RR) {
        // full-res ray at (8y+ky, 8x+kx) and (8y+ky, 8x+8+kx)
        const float X0 = (float)(8 * x + kx);
        float2 rx = f2(fmaf(X0, a.ifu8, a.tu8_c), fmaf(X0 + 8.0f, a.ifu8, a.tu8_c));
        float2 ry = f2(fmaf((float)(8 * y + ky), a.ifv8, a.tv8_c));
        const float2 ri = rsqrt2(fma2(rx, rx, fma2(ry, ry, f2(1.0f))));
        rx = mul2(rx, ri);
        ry = mul2(ry, ri);
        const float2 rz = ri;
        const float2 nn2 = fma2(ox, ox, fma2(oy, oy, mul2(oz, oz)));
        const float2 c = mul2(fma2(ox, rx, fma2(oy, ry, mul2(oz, rz))),
                              rsqrt2(max2(nn2, f2(1e-16f))));
        const float2 dc = max2(fma2(c, f2(-1.0f), f2(kRayEps)), f2(0.0f));
        ox = fma2(rx, dc, ox);
        oy = fma2(ry, dc, oy);
        oz = fma2(rz, dc, oz);
        const float2 inv = rsqrt2(max2(fma2(ox, ox, fma2(oy, oy, mul2(oz, oz))), f2(1e-24f)));
        ox = mul2(ox, inv);
        oy = mul2(oy, inv);
        oz = mul2(oz, inv);
    }
}

// Collect sub-column kx of a sub-row into the pixels' 16-byte runs.
template <typename TS>
__device__ __forceinline__ void collect(OutRun<TS>& run, int kx, float2 ox, float2 oy, float2 oz) {
    const float o[3][2] = {{ox.x, ox.y}, {oy.x, oy.y}, {oz.x, oz.y}};
    if constexpr (sizeof(TS) == 2) {
        // half pairs (kx even, kx odd) per pixel, one packed conversion each
        // once the odd sub-column is done
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                if ((kx & 1) == 0)
                    run.ev[c][e] = o[c][e];
                else
                    run.v[c][e][kx >> 1] = __floats2half2_rn(run.ev[c][e], o[c][e]);
            }
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int e = 0; e < 2; ++e) run.v[c][e][kx & 3] = o[c][e];
    }
}

// Store the pair's completed runs of output row Yo (kx: the run's last
// sub-column), cropped.
template <typename TS>
__device__ __forceinline__ void store_run(const OutRun<TS>& run, int kx, TS* __restrict__ out,
                                          const UpArgs& a, int b, int x, int Yo) {
    if (!check_ok(Yo >= 0 && Yo < a.out_h && b >= 0 && b < a.B, kChkUpStore)) return;
    TS* orow = out + (long)b * 3 * a.out_h * a.out_w + (long)Yo * a.out_w;
    if constexpr (sizeof(TS) == 2) {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int X = 8 * (x + e) - a.crop_l;  // first column of the run
                TS* dst = orow + (long)c * a.out_h * a.out_w + X;
                if (e == 1 && x + 1 >= a.w) continue;
                if (a.vec_out && X >= 0 && X + 8 <= a.out_w) {
                    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(&run.v[c][e][0]);
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const __half hv = (k & 1) ? run.v[c][e][k >> 1].y : run.v[c][e][k >> 1].x;
                        if (X + k >= 0 && X + k < a.out_w) dst[k] = hv;
                    }
                }
            }
    } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int X = 8 * (x + e) + (kx & 4) - a.crop_l;
                TS* dst = orow + (long)c * a.out_h * a.out_w + X;
                if (e == 1 && x + 1 >= a.w) continue;
                if (a.vec_out && X >= 0 && X + 4 <= a.out_w) {
                    *reinterpret_cast<float4*>(dst) = make_float4(run.v[c][e][0], run.v[c][e][1],
                                                                  run.v[c][e][2], run.v[c][e][3]);
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (X + k >= 0 && X + k < a.out_w) dst[k] = run.v[c][e][k];
                }
            }
    }
}

template <typename TNI, typename TS, bool NORM, bool RR, bool TMA>
__global__ void __launch_bounds__(kUThreads, 2)
upsample_kernel(const TNI* __restrict__ nrm, const TS* __restrict__ mask, TS* __restrict__ out,
                const UpArgs a, const __grid_constant__ CUtensorMap mmap) {
    using U = UpRing<TS>;
    using L = Logit<TS>;
    constexpr int kRun = sizeof(TS) == 2 ? 8 : 4;  // sub-columns per 16-byte run
    extern __shared__ __align__(128) unsigned char up_smem[];
    int t = blockIdx.x;
    const int tix = t % a.tiles_x;
    t /= a.tiles_x;
    const int tiy = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int x0 = tix * kUTW, y0 = tiy * kUTH;
    const int y = y0 + warp;
    const int x = x0 + 2 * lane;
    const bool active = x < a.w;
    // only warp barriers and warp votes below: a warp past the last row can
    // leave now; every lane of a row computes (lanes past the last column on
    // clamped, zero-filled data) and stores only its own columns
    if (y >= a.h) return;
    const long hw = a.hw;

    TS* ring = reinterpret_cast<TS*>(up_smem + warp * U::kWarpBytes);
    const uint32_t bar0 =
        tc::smem_u32(up_smem + (kUThreads / 32) * U::kWarpBytes) + 8 * U::kN * warp;
    bool failed = false;
    auto issue = [&](int k) {  // lane 0: stage k (= ky * 8 + kx) into slot k % kN
        const int s = k % U::kN;
        // the box's innermost coordinate must start on 16 bytes
        if (!check_ok((x0 * (int)sizeof(TS)) % 16 == 0 && x0 < a.w && y < a.h && k < 64 &&
                          b < a.B,
                      kChkUpTma)) {
            tc::mbar_arrive(bar0 + 8 * s);  // completes the phase with no bytes
            return;
        }
        tc::mbar_expect_tx(bar0 + 8 * s, U::kBytes);
        tc::tma_load_4d(tc::smem_u32(ring + s * U::kElems), &mmap, bar0 + 8 * s, x0, y, k, b * 9);
    };
    if constexpr (TMA) {
        if (lane == 0) {
#pragma unroll
            for (int s = 0; s < U::kN; ++s) tc::mbar_init(bar0 + 8 * s, 1);
            tc::mbar_fence_init();
#pragma unroll
            for (int k = 0; k < U::kN - U::kSP; ++k) issue(k);
        }
        __syncwarp();
    }
    int issued_hi = U::kN - U::kSP - 1;  // last stage issued (lane 0 issues)
    const bool vec = (a.w & 1) == 0;   // pairs start at even offsets: 8/4-byte aligned
    const int xc = vec ? min(x, a.w - 2) : min(x, a.w - 1);
    const int x1 = min(xc + 1, a.w - 1);

    // (launched as a dependent of the last AngMF launch: its mask stages are
    // in flight above; the normals are that launch's output)
    pdl_wait();
    // 3x3 replicate-padded neighbourhood of the pair, per channel
    const TNI* nb = nrm + (long)b * 3 * hw;
    float2 N[9][3];
#pragma unroll
    for (int ty = 0; ty < 3; ++ty) {
        const long row = (long)clampi(y + ty - 1, 0, a.h - 1) * a.w;
#pragma unroll
        for (int tx = 0; tx < 3; ++tx) {
            const long c0 = row + clampi(xc + tx - 1, 0, a.w - 1);
            const long c1 = row + clampi(x1 + tx - 1, 0, a.w - 1);
#pragma unroll
            for (int c = 0; c < 3; ++c)
                N[ty * 3 + tx][c] = f2(St<TNI>::ld(nb + c * hw + c0), St<TNI>::ld(nb + c * hw + c1));
        }
    }

    const TS* mb = mask + (long)b * 576 * hw + (long)y * a.w + xc;
    const long d1 = x1 - xc;
    const int so = 2 * lane;  // pair offset in a staged strip

#pragma unroll 1
    for (int ky = 0; ky < 8; ++ky) {
        const int Yo = 8 * y + ky - a.crop_t;
        const bool row_in = Yo >= 0 && Yo < a.out_h;
        OutRun<TS> run;
        bool tiny = false;
#pragma unroll
        for (int kg = 0; kg < 8 / U::kSP; ++kg) {
            typename L::T lg[U::kSP][9];
            if constexpr (TMA) {
                const int k = ky * 8 + kg * U::kSP;  // first stage of the group
#pragma unroll
                for (int e = 0; e < U::kSP; ++e) {
                    const int s = (kg * U::kSP + e) % U::kN;
                    const uint32_t parity = ((k + e) / U::kN) & 1;
                    if (!failed && !(a.wait_limit != 0 &&
                                     tc::mbar_wait_pipe(bar0 + 8 * s, parity, a.wait_limit))) {
                        failed = true;
                        if (lane == 0 && a.status) atomicOr(a.status, 2);
                    }
                }
                __syncwarp();  // every lane done with the previous group's slots
                if (lane == 0 && !failed) {
                    // the previous group's slots get the stages kN - kSP ahead
                    // (every lane's loads from them were consumed by the
                    // previous group's arithmetic, so they have completed).
                    // After a wait gave up nothing more is issued: a slot
                    // whose copy may still be in flight is never refilled.
#pragma unroll
                    for (int e = 0; e < U::kSP; ++e)
                        if (k + e + U::kN - U::kSP < 64) {
                            issue(k + e + U::kN - U::kSP);
                            issued_hi = k + e + U::kN - U::kSP;
                        }
                }
#pragma unroll
                for (int e = 0; e < U::kSP; ++e) {
                    const TS* st = ring + ((kg * U::kSP + e) % U::kN) * U::kElems + so;
#pragma unroll
                    for (int tp = 0; tp < 9; ++tp) lg[e][tp] = L::lds(st + tp * kUTW);
                }
            } else {
#pragma unroll
                for (int e = 0; e < U::kSP; ++e)
#pragma unroll
                    for (int tp = 0; tp < 9; ++tp)
                        lg[e][tp] = L::ldg(mb + (long)(tp * 64 + ky * 8 + kg * U::kSP + e) * hw,
                                           d1, vec);
            }
#pragma unroll
            for (int sg = 0; sg < U::kSP; ++sg) {
                const int kx = kg * U::kSP + sg;
                float2 ox, oy, oz;
                subpixel<TS, NORM, RR, false>(lg[sg], N, a, x, y, ky, kx, ox, oy, oz, tiny);
                collect<TS>(run, kx, ox, oy, oz);
                if (kx % kRun == kRun - 1) {
                    if (NORM && __any_sync(0xffffffffu, tiny)) {
                        // rare: a sub-pixel of this run came within the clamp's
                        // reach; recompute the run with S summed
#pragma unroll
                        for (int k2 = kx + 1 - kRun; k2 <= kx; ++k2) {
                            typename L::T l2[9];
#pragma unroll
                            for (int tp = 0; tp < 9; ++tp)
                                l2[tp] = L::ldg(mb + (long)(tp * 64 + ky * 8 + k2) * hw, d1, vec);
                            bool unused = false;
                            subpixel<TS, NORM, RR, true>(l2, N, a, x, y, ky, k2, ox, oy, oz,
                                                         unused);
                            collect<TS>(run, k2, ox, oy, oz);
                        }
                        tiny = false;
                    }
                    if (row_in && active) store_run<TS>(run, kx, out, a, b, x, Yo);
                }
            }
        }
    }
    if constexpr (TMA) {
        // After a wait that gave up, the later waits were skipped and nothing
        // more was issued: before the warp's shared memory can be reused,
        // wait (bounded) for the last copy issued into each slot -- the
        // largest stage j <= issued_hi with j = s mod kN, one copy per slot at
        // most in flight -- so that no copy lands after the CTA has exited.
        // (Without a failure every copy was waited on already.)
        if (failed && lane == 0) {
#pragma unroll
            for (int s = 0; s < U::kN; ++s)
                if (issued_hi >= s) {
                    const int j = issued_hi - (issued_hi - s) % U::kN;
                    tc::mbar_wait(bar0 + 8 * s, (j / U::kN) & 1, kUpWaitLimit);
                }
        }
        __syncwarp();
    }
}

template <typename TNI, typename TS, bool NORM, bool RR>
cudaError_t launch_t(const UpsampleLaunch& L, const UpArgs& a, cudaStream_t s) {
    const long blocks = (long)a.tiles_x * a.tiles_y * a.B;
    if (blocks > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    CUtensorMap m{};
    // staged: the mask as a 4-D tensor (w, h, 64 sub-pixel planes, B * 9
    // taps; the frame stride is 9 tap strides); rows a multiple of 16 bytes
    if ((a.w * (int)sizeof(TS)) % 16 == 0 && (long)L.B * 9 < 0x7fffffffL) {
        const cuuint64_t dims[4] = {(cuuint64_t)a.w, (cuuint64_t)a.h, 64, (cuuint64_t)L.B * 9};
        const cuuint64_t str[3] = {(cuuint64_t)a.w * sizeof(TS), (cuuint64_t)a.hw * sizeof(TS),
                                   (cuuint64_t)a.hw * 64 * sizeof(TS)};
        const cuuint32_t box[4] = {kUTW, 1, 1, 9};
        if (tma_encode(&m, L.mask, 4, dims, str, box,
                       sizeof(TS) == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                       CU_TENSOR_MAP_SWIZZLE_NONE)) {
            auto kern = upsample_kernel<TNI, TS, NORM, RR, true>;
            const size_t smem = UpRing<TS>::kSmem;
            cudaError_t e =
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            e = launch_pdl(kern, dim3((unsigned)blocks), dim3(kUThreads), smem, s, L.pdl,
                           static_cast<const TNI*>(L.n), static_cast<const TS*>(L.mask),
                           static_cast<TS*>(L.out), a, m);
            return e != cudaSuccess ? e : cudaGetLastError();
        }
    }
    cudaError_t e = launch_pdl(upsample_kernel<TNI, TS, NORM, RR, false>,
                               dim3((unsigned)blocks), dim3(kUThreads), 0, s, L.pdl,
                               static_cast<const TNI*>(L.n), static_cast<const TS*>(L.mask),
                               static_cast<TS*>(L.out), a, m);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename TNI, typename TS>
cudaError_t launch_flags(const UpsampleLaunch& L, const UpArgs& a, cudaStream_t s) {
    if (L.normalize && L.ray_relu) return launch_t<TNI, TS, true, true>(L, a, s);
    if (L.normalize) return launch_t<TNI, TS, true, false>(L, a, s);
    if (!L.ray_relu) return launch_t<TNI, TS, false, false>(L, a, s);
    return cudaErrorInvalidValue;
}

}  // namespace

uint32_t set_upsample_wait_limit(uint32_t limit) { return g_up_wait_limit.exchange(limit); }

cudaError_t launch_upsample(const UpsampleLaunch& L, cudaStream_t s) {
    if (L.B == 0 || L.h == 0 || L.w == 0 || L.out_h == 0 || L.out_w == 0) return cudaSuccess;
    UpArgs a;
    a.B = L.B;
    a.h = L.h;
    a.w = L.w;
    a.tiles_x = (L.w + kUTW - 1) / kUTW;
    a.tiles_y = (L.h + kUTH - 1) / kUTH;
    a.hw = (long)L.h * L.w;
    a.crop_t = L.crop_t;
    a.crop_l = L.crop_l;
    a.out_h = L.out_h;
    a.out_w = L.out_w;
    // 16-byte runs: 8 halves or 4 floats, every run start aligned
    const int run = L.st == SType::F16 ? 8 : 4;
    a.vec_out = (L.out_w % run == 0) && (L.crop_l % run == 0);
    // full-res intrinsics are 8x the grid ones (the /8 grid of a padded frame)
    a.ifu8 = (float)(1.0 / (8.0 * L.fu));
    a.ifv8 = (float)(1.0 / (8.0 * L.fv));
    a.tu8_c = (float)((0.5 - 8.0 * L.cu) / (8.0 * L.fu));
    a.tv8_c = (float)((0.5 - 8.0 * L.cv) / (8.0 * L.fv));
    a.status = L.status;
    a.wait_limit = g_up_wait_limit.load(std::memory_order_relaxed);
    if (L.st == SType::F32) {
        if (L.n_t != SType::F32) return cudaErrorInvalidValue;
        return launch_flags<float, float>(L, a, s);
    }
    if (L.n_t == SType::F32) return launch_flags<float, __half>(L, a, s);
    return launch_flags<__half, __half>(L, a, s);
}

BVML_CHECK_READER(check_word_upsample)

}  // namespace bvml
