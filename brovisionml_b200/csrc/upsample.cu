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
// Work split: a CTA owns a 2 x 32 grid-pixel tile; warp k (of 8) owns
// sub-column kx = k of every 8x8 output cell, and each lane one grid pixel
// pair of the tile. So every mask plane (tap t, sub-row ky, sub-column kx) is
// read as 32-pixel coalesced rows, exactly once. The pair's 3x3 source
// normals (27 float2) stay in registers for all 64 sub-pixels. Each sub-row
// ky of results goes through a padded shared-memory row buffer (double
// buffered) and leaves as coalesced row segments of the output.
//
// The softmax denominator is folded into the normalise: with e_t = exp(l_t -
// max l), normalise(sum_t (e_t/S) n_t) = a / max(|a|, 1e-12 S) for
// a = sum_t e_t n_t, which is the reference's x / max(|x|, eps) exactly in
// real arithmetic.
#include "bvml_common.cuh"
#include "bvml_internal.h"

namespace bvml {
namespace {

constexpr int kUTW = 32;               // grid columns per tile (16 pairs)
constexpr int kUTH = 2;                // grid rows per tile
constexpr int kUThreads = 256;         // 8 warps (kx) x 32 lanes (2 rows x 16 pairs)
constexpr int kRowCols = 8 * kUTW;     // output columns per tile row
constexpr int kRowPad = kRowCols + kRowCols / 16;  // one pad word per 16 columns

struct UpArgs {
    int B, h, w, tiles_x, tiles_y;
    long hw;
    int crop_t, crop_l, out_h, out_w;
    float ifu8, ifv8, tu8_c, tv8_c;    // full-res ray: ((X+0.5)-8cu)/(8fu) = X*ifu8 + tu8_c
};

__device__ __forceinline__ int rb_index(int col) { return col + (col >> 4); }

template <typename TNI, typename TS, bool NORM, bool RR>
__global__ void __launch_bounds__(kUThreads, 2)
upsample_kernel(const TNI* __restrict__ nrm, const TS* __restrict__ mask, TS* __restrict__ out,
                const UpArgs a) {
    __shared__ float rowbuf[2][kUTH][3][kRowPad];

    int t = blockIdx.x;
    const int tix = t % a.tiles_x;
    t /= a.tiles_x;
    const int tiy = t % a.tiles_y;
    const int b = t / a.tiles_y;
    const int x0 = tix * kUTW, y0 = tiy * kUTH;

    const int lane = threadIdx.x & 31;
    const int kx = threadIdx.x >> 5;
    const int lr = lane >> 4;            // tile row
    const int lp = lane & 15;            // pair index
    const int y = y0 + lr, x = x0 + 2 * lp;
    const bool active = (y < a.h) && (x < a.w);
    const long hw = a.hw;
    const bool vec = (a.w & 1) == 0;
    // Lanes past the frame edge compute on clamped (valid) pixels and are not
    // stored. With even w the clamp keeps the pair start even, so the paired
    // loads below stay 8/4-byte aligned.
    const int yc = min(y, a.h - 1);
    const int xc0 = vec ? min(x, a.w - 2) : min(x, a.w - 1);
    const int xc1 = min(xc0 + 1, a.w - 1);

    // 3x3 replicate-padded neighbourhood of the pair, per channel.
    const TNI* nb = nrm + (long)b * 3 * hw;
    float2 N[9][3];
#pragma unroll
    for (int ty = 0; ty < 3; ++ty) {
        const long row = (long)clampi(yc + ty - 1, 0, a.h - 1) * a.w;
#pragma unroll
        for (int tx = 0; tx < 3; ++tx) {
            const long c0 = row + clampi(xc0 + tx - 1, 0, a.w - 1);
            const long c1 = row + clampi(xc1 + tx - 1, 0, a.w - 1);
#pragma unroll
            for (int c = 0; c < 3; ++c)
                N[ty * 3 + tx][c] = f2(St<TNI>::ld(nb + c * hw + c0), St<TNI>::ld(nb + c * hw + c1));
        }
    }

    const TS* mb = mask + (long)b * 576 * hw + (long)yc * a.w + xc0;
    const long pofs1 = xc1 - xc0;
    constexpr float kL2E = 1.4426950408889634f;

#pragma unroll 1
    for (int ky = 0; ky < 8; ++ky) {
        float2 l[9];
#pragma unroll
        for (int tp = 0; tp < 9; ++tp) {
            const TS* pch = mb + (long)(tp * 64 + ky * 8 + kx) * hw;
            l[tp] = vec ? St<TS>::ld2s(pch) : f2(St<TS>::lds1(pch), St<TS>::lds1(pch + pofs1));
        }
        float2 m = l[0];
#pragma unroll
        for (int tp = 1; tp < 9; ++tp) m = max2(m, l[tp]);
        const float2 mo = mul2(m, f2(-kL2E));
        float2 S = f2(0.f), ax = f2(0.f), ay = f2(0.f), az = f2(0.f);
#pragma unroll
        for (int tp = 0; tp < 9; ++tp) {
            const float2 e = ex2_2(fma2(l[tp], f2(kL2E), mo));
            S = add2(S, e);
            ax = fma2(e, N[tp][0], ax);
            ay = fma2(e, N[tp][1], ay);
            az = fma2(e, N[tp][2], az);
        }
        float2 ox, oy, oz;
        if (NORM) {
            const float2 l2 = fma2(ax, ax, fma2(ay, ay, mul2(az, az)));
            const float2 se = mul2(S, f2(1e-12f));
            const float2 inv = rsqrt2(max2(l2, mul2(se, se)));
            ox = mul2(ax, inv);
            oy = mul2(ay, inv);
            oz = mul2(az, inv);
        } else {
            const float2 inv = f2(1.0f / S.x, 1.0f / S.y);
            ox = mul2(ax, inv);
            oy = mul2(ay, inv);
            oz = mul2(az, inv);
        }
        if (RR) {
            // full-res ray at (8y+ky, 8x+kx) and (8y+ky, 8x+8+kx)
            const float Yf = (float)(8 * y + ky);
            const float X0 = (float)(8 * x + kx);
            float2 rx = f2(fmaf(X0, a.ifu8, a.tu8_c), fmaf(X0 + 8.0f, a.ifu8, a.tu8_c));
            float2 ry = f2(fmaf(Yf, a.ifv8, a.tv8_c));
            const float2 ri = rsqrt2(fma2(rx, rx, fma2(ry, ry, f2(1.0f))));
            rx = mul2(rx, ri);
            ry = mul2(ry, ri);
            const float2 rz = ri;
            const float2 nn2 = fma2(ox, ox, fma2(oy, oy, mul2(oz, oz)));
            const float2 c = mul2(fma2(ox, rx, fma2(oy, ry, mul2(oz, rz))),
                                  rsqrt2(max2(nn2, f2(1e-16f))));
            const float2 dc = max2(fnma2(c, f2(1.0f), f2(kRayEps)), f2(0.0f));
            ox = fma2(rx, dc, ox);
            oy = fma2(ry, dc, oy);
            oz = fma2(rz, dc, oz);
            const float2 inv = rsqrt2(max2(fma2(ox, ox, fma2(oy, oy, mul2(oz, oz))), f2(1e-24f)));
            ox = mul2(ox, inv);
            oy = mul2(oy, inv);
            oz = mul2(oz, inv);
        }
        float(*rb)[3][kRowPad] = rowbuf[ky & 1];
        const int c0 = rb_index(16 * lp + kx), c1 = rb_index(16 * lp + 8 + kx);
        rb[lr][0][c0] = ox.x;
        rb[lr][1][c0] = oy.x;
        rb[lr][2][c0] = oz.x;
        rb[lr][0][c1] = ox.y;
        rb[lr][1][c1] = oy.y;
        rb[lr][2][c1] = oz.y;
        __syncthreads();

        // write-out: kUTH rows x 3 channels x kRowCols columns, in column pairs
        const int X0 = 8 * x0 - a.crop_l;
        const bool vout = ((a.out_w & 1) == 0) && ((a.crop_l & 1) == 0);
        constexpr int kChunks = kUTH * 3 * kRowCols / 2;
#pragma unroll 1
        for (int ch = threadIdx.x; ch < kChunks; ch += kUThreads) {
            const int cp = ch % (kRowCols / 2);
            const int rc = ch / (kRowCols / 2);
            const int c = rc % 3;
            const int r = rc / 3;
            const int gy = y0 + r;
            if (gy >= a.h) continue;
            const int Yo = 8 * gy + ky - a.crop_t;
            if (Yo < 0 || Yo >= a.out_h) continue;
            const int col = 2 * cp;
            const int Xo = X0 + col;
            if (8 * (x0 + (col >> 3)) >= 8 * a.w) continue;  // beyond the grid's last column
            const float v0 = rb[r][c][rb_index(col)], v1 = rb[r][c][rb_index(col + 1)];
            TS* orow = out + (((long)b * 3 + c) * a.out_h + Yo) * (long)a.out_w;
            if (vout && Xo >= 0 && Xo + 1 < a.out_w) {
                St<TS>::st2(orow + Xo, f2(v0, v1));
            } else {
                if (Xo >= 0 && Xo < a.out_w) St<TS>::st(orow + Xo, v0);
                if (Xo + 1 >= 0 && Xo + 1 < a.out_w) St<TS>::st(orow + Xo + 1, v1);
            }
        }
    }
    (void)active;
}

template <typename TNI, typename TS, bool NORM, bool RR>
cudaError_t launch_t(const UpsampleLaunch& L, const UpArgs& a, cudaStream_t s) {
    const long blocks = (long)a.tiles_x * a.tiles_y * a.B;
    if (blocks > 0x7fffffffL) return cudaErrorInvalidConfiguration;
    upsample_kernel<TNI, TS, NORM, RR><<<(unsigned)blocks, kUThreads, 0, s>>>(
        static_cast<const TNI*>(L.n), static_cast<const TS*>(L.mask), static_cast<TS*>(L.out), a);
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
