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
// Logit staging: when the grid width is a multiple of 16 bytes of storage,
// each warp copies, for every (ky, kx), the 9 logit strips of its own row
// (9 planes x 64 columns) global -> shared with 16-byte cp.async into a
// warp-private ring kN stages deep. Stages go in groups of kSP: one warp
// barrier publishes a group, and the kSP sub-pixels of a group are computed
// together so that their independent dependency chains interleave (the kernel
// is otherwise bound by fixed-latency waits at 4 warps per scheduler). The
// bytes in flight do not cost registers. Other widths read the logits
// straight from global memory.
//
// The softmax denominator is folded into the normalise: with e_t = exp(l_t -
// max l), normalise(sum_t (e_t/S) n_t) = a / max(|a|, 1e-12 S) for
// a = sum_t e_t n_t, which is the reference's x / max(|x|, eps) exactly in
// real arithmetic.
#include "bvml_common.cuh"
#include "bvml_internal.h"

namespace bvml {
namespace {

constexpr int kUTW = 64;        // grid columns per tile (32 pairs = one warp)
constexpr int kUTH = 8;         // grid rows per tile (one per warp)
constexpr int kUThreads = 256;

template <typename TS>
struct UpStages {
    static constexpr int kEpc = 16 / (int)sizeof(TS);             // elements per chunk
    static constexpr int kCpr = kUTW / kEpc;                      // chunks per strip
    static constexpr int kChunksW = 9 * kCpr;                     // per warp per stage
    static constexpr int kElemsW = 9 * kUTW;                      // per warp per stage
    static constexpr int kSP = sizeof(TS) == 2 ? 2 : 1;           // stages per group
    static constexpr int kN = sizeof(TS) == 2 ? 6 : 4;            // ring depth
    static constexpr int kG = kN / kSP;                           // groups in the ring
    static_assert(kN % kSP == 0 && 8 % kSP == 0, "stage groups must tile the ring and a row");
    static constexpr size_t kBytes = (size_t)(kUThreads / 32) * kN * kElemsW * sizeof(TS);
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

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

// A lane's share of one stage: chunks q = lane + 32 m (m < kPerLane) of the
// 9 x kCpr chunk grid. Because 32 is a multiple of kCpr, a lane keeps one
// column cc for all its chunks and its plane advances by 32 / kCpr per m, so
// only a base offset, a column validity flag and a plane stride are kept.
template <typename TS>
struct LaneChunks {
    using U = UpStages<TS>;
    static constexpr int kPerLane = (U::kChunksW + 31) / 32;
    static constexpr int kTStep = 32 / U::kCpr;   // planes between a lane's chunks
    int off0;       // element offset of chunk m = 0 from the stage's plane-0 row
    int doff0;      // its offset inside a warp slot
    int tstep_hw;   // 64 * kTStep * hw: source distance between consecutive m
    int nlast;      // chunks this lane has (kPerLane or kPerLane - 1)
    bool col_ok;    // the lane's column lies inside the frame
    __device__ void init(int lane, int ncols, long hw) {
        const int t0 = lane / U::kCpr, cc = lane % U::kCpr;
        off0 = t0 * 64 * (int)hw + cc * U::kEpc;
        doff0 = t0 * kUTW + cc * U::kEpc;
        tstep_hw = 64 * kTStep * (int)hw;
        nlast = (lane + 32 * (kPerLane - 1) < U::kChunksW) ? kPerLane : kPerLane - 1;
        col_ok = cc * U::kEpc < ncols;
    }
    // copy the lane's chunks of the stage whose plane-0 row starts at `src`
    __device__ __forceinline__ void issue(TS* slot, const TS* src) const {
        const TS* p = src + off0;
#pragma unroll
        for (int m = 0; m < kPerLane; ++m) {
            if (m < nlast)
                cp_async16(slot + doff0 + m * kTStep * kUTW, col_ok ? p : src, col_ok);
            p += tstep_hw;
        }
    }
};

struct UpArgs {
    int B, h, w, tiles_x, tiles_y;
    long hw;
    int crop_t, crop_l, out_h, out_w;
    bool vec_out;                   // 16-byte aligned output runs
    float ifu8, ifv8, tu8_c, tv8_c; // full-res ray: ((X+0.5)-8cu)/(8fu) = X*ifu8 + tu8_c
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

template <typename TNI, typename TS, bool NORM, bool RR, bool STAGED>
__global__ void __launch_bounds__(kUThreads, 2)
upsample_kernel(const TNI* __restrict__ nrm, const TS* __restrict__ mask, TS* __restrict__ out,
                const UpArgs a) {
    using U = UpStages<TS>;
    extern __shared__ float4 up_smem[];
    TS* ring = reinterpret_cast<TS*>(up_smem) + (threadIdx.x >> 5) * U::kN * U::kElemsW;
    int t = blockIdx.x;
    const int tix = t % a.tiles_x;
    t /= a.tiles_x;
    const int tiy = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int lane = threadIdx.x & 31;
    const int x0 = tix * kUTW, y0 = tiy * kUTH;
    const int y = y0 + (threadIdx.x >> 5);
    const int x = x0 + 2 * lane;
    const bool active = y < a.h && x < a.w;
    // only warp barriers below: a warp past the last row, or (unstaged) a
    // lane past the last column, can leave now
    if (y >= a.h || (!STAGED && !active)) return;
    const long hw = a.hw;
    const TS* mframe = mask + (long)b * 576 * hw;
    const TS* mrow = mframe + (long)y * a.w + x0;  // plane 0 of this warp's row
    LaneChunks<TS> lc;
    const TS* mnext = mrow;                         // plane-0 row of the next stage to copy
    if (STAGED) {
        lc.init(lane, a.w - x0, hw);
#pragma unroll
        for (int s = 0; s < U::kN - U::kSP; ++s) {  // the first kG-1 groups
            lc.issue(ring + s * U::kElemsW, mnext);
            mnext += hw;
            if (s % U::kSP == U::kSP - 1) cp_async_commit();
        }
    }
    const bool vec = (a.w & 1) == 0;   // pairs start at even offsets: 8/4-byte aligned
    const int yc = min(y, a.h - 1);
    const int xc = vec ? min(x, a.w - 2) : min(x, a.w - 1);
    const int x1 = min(xc + 1, a.w - 1);

    // 3x3 replicate-padded neighbourhood of the pair, per channel
    const TNI* nb = nrm + (long)b * 3 * hw;
    float2 N[9][3];
#pragma unroll
    for (int ty = 0; ty < 3; ++ty) {
        const long row = (long)clampi(yc + ty - 1, 0, a.h - 1) * a.w;
#pragma unroll
        for (int tx = 0; tx < 3; ++tx) {
            const long c0 = row + clampi(xc + tx - 1, 0, a.w - 1);
            const long c1 = row + clampi(x1 + tx - 1, 0, a.w - 1);
#pragma unroll
            for (int c = 0; c < 3; ++c)
                N[ty * 3 + tx][c] = f2(St<TNI>::ld(nb + c * hw + c0), St<TNI>::ld(nb + c * hw + c1));
        }
    }

    const TS* mb = mframe + (long)yc * a.w + xc;
    const long d1 = x1 - xc;
    constexpr float kL2E = 1.4426950408889634f;
    using L = Logit<TS>;
    const int so = 2 * lane;  // pair offset in a staged strip
    int rslot = 0;            // ring slot of the first stage of the group being computed

#pragma unroll 1
    for (int ky = 0; ky < 8; ++ky) {
        const int Yo = 8 * y + ky - a.crop_t;
        const bool row_in = Yo >= 0 && Yo < a.out_h;
        OutRun<TS> run;
#pragma unroll
        for (int kg = 0; kg < 8 / U::kSP; ++kg) {
            typename L::T lg[U::kSP][9];
            if (STAGED) {
                const int k = ky * 8 + kg * U::kSP;  // first stage of the group
                cp_async_wait<U::kG - 2>();
                __syncwarp();  // group visible to the warp; every lane done with the previous one
                // the group kG-1 ahead goes to the slots of the previous group
                // (slot counters wrap instead of taking k % kN)
                const int islot = rslot == 0 ? U::kN - U::kSP : rslot - U::kSP;
                if (k + U::kN - U::kSP < 64) {
#pragma unroll
                    for (int e = 0; e < U::kSP; ++e) {
                        lc.issue(ring + (islot + e) * U::kElemsW, mnext);
                        mnext += hw;
                    }
                }
                cp_async_commit();
                const TS* st = ring + rslot * U::kElemsW + so;
                rslot = rslot == U::kN - U::kSP ? 0 : rslot + U::kSP;
#pragma unroll
                for (int e = 0; e < U::kSP; ++e)
#pragma unroll
                    for (int tp = 0; tp < 9; ++tp)
                        lg[e][tp] = L::lds(st + e * U::kElemsW + tp * kUTW);
            } else {
#pragma unroll
                for (int e = 0; e < U::kSP; ++e)
#pragma unroll
                    for (int tp = 0; tp < 9; ++tp)
                        lg[e][tp] = L::ldg(mb + (long)(tp * 64 + ky * 8 + kg * U::kSP + e) * hw,
                                           d1, vec);
            }
            if (!active) continue;  // staged mode: idle lanes only keep the warp barriers
#pragma unroll
            for (int sg = 0; sg < U::kSP; ++sg) {
                const int kx = kg * U::kSP + sg;
                const typename L::T* l = lg[sg];
                const float2 m =
                    L::f(L::mx(L::mx(L::mx(l[0], l[1]), L::mx(l[2], l[3])),
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
                float2 ox, oy, oz;
                if (NORM) {
                    // x / max(|x|, 1e-12) for x = a / S; with 1 <= S <= 9 the clamp can
                    // only act when |a| < 9e-12, so S is summed only then.
                    float2 l2 = fma2(ax, ax, fma2(ay, ay, mul2(az, az)));
                    if ((l2.x < 8.1e-23f) | (l2.y < 8.1e-23f)) {
                        float2 S = ew(0);
                        for (int tp = 1; tp < 9; ++tp) S = add2(S, ew(tp));
                        const float2 se = mul2(S, f2(1e-12f));
                        l2 = max2(l2, mul2(se, se));
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
                    const float2 inv =
                        rsqrt2(max2(fma2(ox, ox, fma2(oy, oy, mul2(oz, oz))), f2(1e-24f)));
                    ox = mul2(ox, inv);
                    oy = mul2(oy, inv);
                    oz = mul2(oz, inv);
                }
                // collect; flush a 16-byte run per channel and pixel when complete
                if constexpr (sizeof(TS) == 2) {
                    // half pairs (kx even, kx odd) per pixel, one packed
                    // conversion each once the odd sub-column is done
                    const float o[3][2] = {{ox.x, ox.y}, {oy.x, oy.y}, {oz.x, oz.y}};
#pragma unroll
                    for (int c = 0; c < 3; ++c)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            if ((kx & 1) == 0)
                                run.ev[c][e] = o[c][e];
                            else
                                run.v[c][e][kx >> 1] = __floats2half2_rn(run.ev[c][e], o[c][e]);
                        }
                    if (kx == 7 && row_in && active) {
                        TS* orow = out + (long)b * 3 * a.out_h * a.out_w + (long)Yo * a.out_w;
#pragma unroll
                        for (int c = 0; c < 3; ++c)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int X = 8 * (x + e) - a.crop_l;  // first column of the run
                                TS* dst = orow + (long)c * a.out_h * a.out_w + X;
                                if (e == 1 && x + 1 >= a.w) continue;
                                if (a.vec_out && X >= 0 && X + 8 <= a.out_w) {
                                    *reinterpret_cast<uint4*>(dst) =
                                        *reinterpret_cast<const uint4*>(&run.v[c][e][0]);
                                } else {
#pragma unroll
                                    for (int k = 0; k < 8; ++k) {
                                        const __half hv = (k & 1) ? run.v[c][e][k >> 1].y
                                                                  : run.v[c][e][k >> 1].x;
                                        if (X + k >= 0 && X + k < a.out_w) dst[k] = hv;
                                    }
                                }
                            }
                    }
                } else {
                    const float o[3][2] = {{ox.x, ox.y}, {oy.x, oy.y}, {oz.x, oz.y}};
#pragma unroll
                    for (int c = 0; c < 3; ++c)
#pragma unroll
                        for (int e = 0; e < 2; ++e) run.v[c][e][kx & 3] = o[c][e];
                    if ((kx & 3) == 3 && row_in && active) {
                        TS* orow = out + (long)b * 3 * a.out_h * a.out_w + (long)Yo * a.out_w;
#pragma unroll
                        for (int c = 0; c < 3; ++c)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int X = 8 * (x + e) + (kx & 4) - a.crop_l;
                                TS* dst = orow + (long)c * a.out_h * a.out_w + X;
                                if (e == 1 && x + 1 >= a.w) continue;
                                if (a.vec_out && X >= 0 && X + 4 <= a.out_w) {
                                    *reinterpret_cast<float4*>(dst) =
                                        make_float4(run.v[c][e][0], run.v[c][e][1], run.v[c][e][2],
                                                    run.v[c][e][3]);
                                } else {
#pragma unroll
                                    for (int k = 0; k < 4; ++k)
                                        if (X + k >= 0 && X + k < a.out_w) dst[k] = run.v[c][e][k];
                                }
                            }
                    }
                }
            }
        }
    }
    if (STAGED) cp_async_wait<0>();
}

template <typename TNI, typename TS, bool NORM, bool RR>
cudaError_t launch_t(const UpsampleLaunch& L, const UpArgs& a, cudaStream_t s) {
    const long blocks = (long)a.tiles_x * a.tiles_y * a.B;
    if (blocks > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    if (a.w % UpStages<TS>::kEpc == 0) {
        auto kern = upsample_kernel<TNI, TS, NORM, RR, true>;
        const size_t smem = UpStages<TS>::kBytes;
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<(unsigned)blocks, kUThreads, smem, s>>>(static_cast<const TNI*>(L.n),
                                                      static_cast<const TS*>(L.mask),
                                                      static_cast<TS*>(L.out), a);
    } else {
        upsample_kernel<TNI, TS, NORM, RR, false><<<(unsigned)blocks, kUThreads, 0, s>>>(
            static_cast<const TNI*>(L.n), static_cast<const TS*>(L.mask),
            static_cast<TS*>(L.out), a);
    }
    return cudaGetLastError();
}

template <typename TNI, typename TS>
cudaError_t launch_flags(const UpsampleLaunch& L, const UpArgs& a, cudaStream_t s) {
    if (L.normalize && L.ray_relu) return launch_t<TNI, TS, true, true>(L, a, s);
    if (L.normalize) return launch_t<TNI, TS, true, false>(L, a, s);
    if (!L.ray_relu) return launch_t<TNI, TS, false, false>(L, a, s);
    return cudaErrorInvalidValue;
}

}  // namespace

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
    if (L.st == SType::F32) {
        if (L.n_t != SType::F32) return cudaErrorInvalidValue;
        return launch_flags<float, float>(L, a, s);
    }
    if (L.n_t == SType::F32) return launch_flags<float, __half>(L, a, s);
    return launch_flags<__half, __half>(L, a, s);
}

}  // namespace bvml
