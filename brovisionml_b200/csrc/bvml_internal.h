// Internal launcher interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

namespace bvml {

// Record `msg` as the calling thread's bvml_last_error() text; returns `code`.
int report_error(int code, const std::string& msg);

}  // namespace bvml
struct bvml_refiner;
namespace bvml {
// The device a refiner handle (bvml_refiner_create) was created on.
int refiner_device(const bvml_refiner* r);

enum class SType { F32 = 0, F16 = 1 };

struct AngmfLaunch {
    const void* pn;      // source normals (B,3,H,W); type pn_t
    const void* prob;    // (B,P,H,W) storage type st
    const void* xy;      // (B,2P,H,W)
    const void* angle;   // (B,P,H,W)
    const float* ray;    // (3,H,W)
    void* out;           // (B,3,H,W); type out_t
    SType st, pn_t, out_t;
    bool fuse_ray_relu;  // apply RayReLU to the source normals while staging them
    bool act;            // prob / angle are raw head outputs: activate them on load
    int B, H, W, ps, dil;
    double fu, cu, fv, cv;
    bool pdl;            // launch as a programmatic dependent of the previous kernel
                         // (which must not write prob / xy / angle)
};
cudaError_t launch_angmf(const AngmfLaunch& L, cudaStream_t s);
cudaError_t launch_angmf_logits(const AngmfLaunch& L, cudaStream_t s);  // L.act variants

// All iterations of the fused refine's AngMF in one persistent launch (tiles
// taken in iteration-major order, each waiting for its neighbour tiles of the
// previous iteration). Returns cudaErrorNotSupported for shapes that do not
// take the staged path; the caller then launches iteration by iteration.
struct AngmfItersLaunch {
    const void* pn0;              // (B,3,H,W) decoder normals, storage type st
    const void* const* prob;      // iters x (B,P,H,W)
    const void* const* xy;        // iters x (B,2P,H,W)
    const void* const* angle;     // iters x (B,P,H,W)
    const float* ray;             // (3,H,W)
    float* buf[2];                // (B,3,H,W) fp32 each; iteration i writes buf[i & 1]
    int* sync;                    // angmf_iters_sync_bytes(B,H,W), zeroed by the launch
    SType st;
    bool act;
    int iters, B, H, W, ps, dil;
    int first;                    // first iteration of this launch (earlier ones done)
    double fu, cu, fv, cv;
};
// sync words: [0] work counter, [1] status, [kSyncHeaderWords ..) one per tile
constexpr int kSyncHeaderWords = 64;
inline size_t angmf_iters_sync_bytes(int B, int H, int W) {
    const size_t tiles = (size_t)((W + 31) / 32) * (size_t)((H + 15) / 16) * (size_t)B;
    return sizeof(int) * (kSyncHeaderWords + tiles);
}
cudaError_t launch_angmf_iters(const AngmfItersLaunch& L, cudaStream_t s);
cudaError_t launch_angmf_iters_logits(const AngmfItersLaunch& L, cudaStream_t s);

struct UpsampleLaunch {
    const void* n;       // (B,3,h,w); type n_t
    const void* mask;    // (B,576,h,w) storage type st
    void* out;           // (B,3,out_h,out_w) storage type st
    SType st, n_t;
    bool normalize;      // channel L2-normalise (eps 1e-12) after the combine
    bool ray_relu;       // full-resolution RayReLU after the normalise
    int B, h, w;
    int crop_t, crop_l, out_h, out_w;
    double fu, cu, fv, cv;  // GRID intrinsics; the full-res ray uses 8x these
    int* status;         // optional: bit 2 set if a staging wait gave up
    bool pdl;            // launch as a programmatic dependent of the previous kernel
                         // (which must not write the mask)
};
cudaError_t launch_upsample(const UpsampleLaunch& L, cudaStream_t s);
// Attempts the upsample makes at each TMA staging wait, for launches that
// follow (0: every wait gives up at once); returns the previous value.
uint32_t set_upsample_wait_limit(uint32_t limit);

enum class ConvEpi : int {
    NHWC = 0, PLANAR16 = 1, PLANAR32 = 2, GRU_ZR = 3, GRU_Q = 4, C4_32 = 5, SPLIT16 = 6
};

struct ConvLaunch {
    const void* x;       // (B,H,W,x_c) fp16; channels [cin_off, cin_off + cin_pad) are read
    const void* w;       // (ks*ks, cout_pad, cin_pad) fp16
    const float* bias;   // (cout) fp32
    int* err;            // device int: nonzero if a pipeline wait gave up
    uint32_t wait_limit; // attempts of a pipeline wait before it gives up (0: 1 << 22)
    int B, H, W, x_c, cin_off, cin_pad, cout, cout_pad, ks;
    ConvEpi epi;
    int act;             // NHWC: 0 none, 1 ReLU, 2 sigmoid, 3 tanh; C4_32: 0, 1
    void* y;             // NHWC: (B,H,W,out_c) fp16 at out_off; C4_32: (B,out_c/4,H,W,4) fp32
                         // at channel out_off; PLANAR: (B,cout,H,W)
    int out_c, out_off;
    float* h32;          // GRU: fp32 hidden state, C4 (B,16,H,W,4)
    void* z;             // GRU: gate z, C8 fp16 (B,8,H,W,8)
    void* rh;            // GRU_ZR: r * h at channels [0,64) of (B,H,W,rh_c)
    int rh_c;
    void* hx;            // GRU_Q: new h (fp16) at channels [0,64) of (B,H,W,hx_c)
    int hx_c;
    void* hin;           // GRU_Q: ... and of (B,H,W,hin_c) when not null
    int hin_c;
    const float* add;    // optional per-pixel addend, C4 fp32 (B or 1,add_c/4,H,W,4)
    int add_c;
    int add_shared;      // nonzero: one frame of addends shared by all B frames
    const void* xin;     // optional extra K: conv += xin[.., 0:xin_c] . wx^T per pixel, fp16
    int xin_c;           // a multiple of 64
    int xin_stride;      // channels per pixel of xin (0: xin_c)
    const void* wx;      // (cout_pad, xin_c) fp16
};
cudaError_t launch_conv_tc(const ConvLaunch& L, cudaStream_t s);

// The last two 1x1 layers of a prediction head in one kernel: x channels
// [cin_off, cin_off + 128) (B,H,W,x_c) fp16 -> ReLU(. W2^T + b2) -> . W4^T + b4
// -> planar (B,cout,H,W) fp16 / fp32, cout <= 64. w2 (128,128), w4 (64,128) fp16.
struct HeadTailLaunch {
    const void* x;
    int x_c, cin_off;
    const void* w2;
    const float* b2;
    const void* w4;
    const float* b4;
    int B, H, W, cout;
    int f16;
    void* y;
    int* err;
    uint32_t wait_limit;  // as ConvLaunch::wait_limit
};
cudaError_t launch_head_tail(const HeadTailLaunch& L, cudaStream_t s);

// Checked builds: each kernel translation unit's check word (see
// bvml_common.cuh), optionally reset; release builds return 0.
unsigned check_word_angmf(bool reset);
unsigned check_word_angmf_logits(bool reset);
unsigned check_word_upsample(bool reset);
unsigned check_word_conv(bool reset);

// Encode a tiled TMA tensor map (defined in conv_tc.cu).
bool tma_encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapDataType dt,
                CUtensorMapSwizzle sw);

cudaError_t launch_ray_relu(void* normal, SType t, const float* ray, int B, int H, int W,
                            cudaStream_t s);
cudaError_t launch_stage_inputs(const float* h0, const float* feat, int B, int H, int W,
                                float* h32, void* hx, void* fx, cudaStream_t s);
cudaError_t launch_build_ray(float* ray, int H, int W, double fu, double cu, double fv,
                             double cv, cudaStream_t s);
cudaError_t launch_l2_normalize(const void* x, void* y, SType t, int N, int C, int H, int W,
                                float eps, cudaStream_t s);
cudaError_t launch_slice2d(const void* x, void* y, SType t, int N, int C, int H, int W, int h0,
                           int w0, int Ho, int Wo, cudaStream_t s);

}  // namespace bvml
