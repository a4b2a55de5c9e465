/*
 * bvml_dsine.h -- C ABI of the B200 (sm_100a) DSINE refine-ops library
 * (libbvml_dsine.so, built from brovisionml_b200/csrc/).
 *
 * It replaces the GPU half of wlejon/brovisionml's only repo-owned GPU path:
 * the DSINE surface-normal refinement ops driven by Refiner::forward
 * (src/dsine_refine.cpp:212-294). Each entry point names the reference
 * interface it replaces.
 *
 * Conventions
 *  - All pointers are DEVICE pointers of the current CUDA device, except the
 *    pointer ARRAYS of bvml_refine (host arrays of device pointers) and the
 *    frame buffers of bvml_refiner_forward_banded (host memory).
 *  - Tensors are planar NCHW and contiguous: (B, C, H, W), W fastest. B frames
 *    of one camera share the intrinsics and the (3, H, W) fp32 ray map.
 *  - `dtype` selects the storage type of the big tensors: BVML_F32 (float) or
 *    BVML_F16 (IEEE binary16, fp32 arithmetic). Ray maps are always fp32.
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream, which is
 *    where the reference launches). Calls are asynchronous; like the
 *    reference, device faults surface at the caller's next synchronisation.
 *  - Every call returns BVML_OK (0) or a BVML_E* code and never throws; the
 *    text of the last failure on the calling thread is bvml_last_error(),
 *    worded like the reference's exceptions: "dsine ops: ..." for argument
 *    errors (src/dsine_ops.cpp:18-22) and "dsine cuda: <what>: <cuda error>"
 *    for CUDA failures (src/dsine_ops.cu:25-29).
 *  - Intrinsics fu, cu, fv, cv are the ones scaled to the (H, W) grid from
 *    the "+0.5" principal point (src/dsine_refine.cpp:232-237).
 */
#ifndef BVML_DSINE_H
#define BVML_DSINE_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BVML_ABI_VERSION 9

enum bvml_dtype { BVML_F32 = 0, BVML_F16 = 1 };

enum bvml_status {
    BVML_OK = 0,
    BVML_EINVAL = 1,      /* bad argument (null pointer, bad size, bad window) */
    BVML_ECUDA = 2,       /* a CUDA call or kernel launch failed              */
    BVML_EUNSUPPORTED = 3 /* valid request outside what this build implements  */
};

/* Text of the last failure on this thread ("" if none). */
const char* bvml_last_error(void);

/* BVML_ABI_VERSION of the loaded library. */
int bvml_abi_version(void);

/*
 * RayReLU in place on B frames of (3, H, W) normals against one (3, H, W)
 * ray: c = n.r / max(|n||r|, 1e-8); n <- normalise(n + r (max(c - eps, 0) + eps - c)),
 * eps = 1e-2.
 * Replaces brovisionml::dsine::detail::ray_relu_cuda
 * (src/dsine_ops_cuda.h:13-14, src/dsine_ops.cu:159-168; CPU twin
 * src/dsine_ops.cpp:55-76). B = 1 is the reference's call.
 */
int bvml_ray_relu(void* normal, const float* ray, int B, int H, int W, int dtype,
                  void* stream);

/*
 * Fused AngMF propagate: for every pixel, rotate each of the ps*ps window
 * neighbours' normals (dilation dil, replicate padding) by its predicted
 * axis-angle, RayReLU it against the pixel's ray, take the prob-weighted sum
 * and L2-normalise.
 *   pred_norm (B,3,H,W)  prob (B,P,H,W)  xy (B,2P,H,W)  angle (B,P,H,W)
 *   ray (3,H,W) fp32     out (B,3,H,W), caller-allocated, must not alias inputs
 * with P = ps*ps, slot n = ky*ps + kx, xy channels [0,P) = x, [P,2P) = y.
 * ps in {3, 5, 7}, dil in 1..4.
 * Replaces brovisionml::dsine::detail::angmf_propagate_cuda
 * (src/dsine_ops_cuda.h:16-23, src/dsine_ops.cu:170-191; CPU twin
 * src/dsine_ops.cpp:78-172). The reference is ps = 5, dil = 1, B = 1, fp32
 * and allocates `out` itself; the C++ bridge (brovisionml_b200/csrc/
 * dsine_ops_b200.cpp) keeps that allocation contract.
 */
int bvml_angmf_propagate(const void* pred_norm, const void* prob, const void* xy,
                         const void* angle, const float* ray, double fu, double cu,
                         double fv, double cv, int B, int H, int W, int ps, int dil,
                         int dtype, void* out, void* stream);

/*
 * bvml_angmf_propagate on the prediction heads' raw outputs: prob_logits and
 * angle_logits (shapes and dtype as prob / angle) are activated while they
 * are loaded, prob = sigmoid(prob_logit), angle = pi * sigmoid(angle_logit)
 * with pi the float 3.14159265f. Replaces the separate passes
 * apply_sigmoid(prob); apply_sigmoid(angle); brotensor::scale_inplace(angle,
 * kPi) of Refiner::forward (src/dsine_refine.cpp:262-267, kPi at :26) and the
 * angmf_propagate call after them (:271-272). xy is raw in both entry points.
 */
int bvml_angmf_propagate_logits(const void* pred_norm, const void* prob_logits, const void* xy,
                                const void* angle_logits, const float* ray, double fu,
                                double cu, double fv, double cv, int B, int H, int W, int ps,
                                int dil, int dtype, void* out, void* stream);

/*
 * Convex upsample: mask (N, 9*s*s, H, W) viewed (9, s, s), softmax over the 9
 * taps, 3x3 replicate-padded unfold of x (N, C, H, W), output y (N, C, s*H, s*W)
 * with row s*y+ky, col s*x+kx. This build implements C = 3, s = 8 (the path's
 * only call); other shapes return BVML_EUNSUPPORTED.
 * Replaces brotensor::convex_upsample_forward(X, mask, N, C, H, W, scale, Y)
 * as called at src/dsine_refine.cpp:277-279 (semantics:
 * include/brovisionml/dsine_refine.h:91-97).
 */
int bvml_convex_upsample(const void* x, const void* mask, int N, int C, int H, int W,
                         int scale, int dtype, void* y, void* stream);

/*
 * Per-pixel channel L2-normalise y = x / max(|x|, eps), (N, C, H, W), C <= 16;
 * y may alias x.
 * Replaces brotensor::l2_normalize_nchw_forward(X, N, C, H, W, eps, Y)
 * (src/dsine_refine.cpp:280-281).
 */
int bvml_l2_normalize_nchw(const void* x, int N, int C, int H, int W, float eps, int dtype,
                           void* y, void* stream);

/*
 * Crop (N, C, H, W) at (h0, w0) to (N, C, Ho, Wo).
 * Replaces brotensor::slice2d_forward(X, N, C, H, W, h0, w0, Ho, Wo, Y)
 * (src/dsine_refine.cpp:288-292).
 */
int bvml_slice2d(const void* x, int N, int C, int H, int W, int h0, int w0, int Ho, int Wo,
                 int dtype, void* y, void* stream);

/* Bytes of device workspace bvml_refine needs for B frames of an (h, w) grid. */
size_t bvml_refine_workspace_bytes(int B, int h, int w);

/*
 * Status of the last bvml_refine / bvml_refine_logits call that used
 * `workspace` (no reference counterpart: the reference's per-iteration
 * launches have no device-side waits). The persistent AngMF launch lets a
 * tile wait for its neighbour tiles of the previous iteration, and the
 * upsample waits for its TMA-staged mask logits; every such wait is bounded,
 * and one that gives up (the GPU stopped making progress) records it in the
 * workspace (bit 1: an AngMF dependency wait, bit 2: an upsample staging
 * wait) instead of hanging. Synchronises `stream`; returns BVML_OK, or
 * BVML_ECUDA with the reason in bvml_last_error().
 */
int bvml_refine_status(const void* workspace, void* stream);

/*
 * Failure injection for tests (no counterpart in the reference): how many
 * attempts the fused upsample makes at each of its TMA staging waits, for the
 * launches that follow, process-wide; returns the previous value. The default
 * is BVML_UPSAMPLE_WAIT_DEFAULT; 0 makes every staging wait give up at once,
 * as if a copy were stuck. A wait that gives up sets bit 2 of the unit's
 * status word (bvml_refine_status reports it), stops the warp's staging,
 * waits (bounded) for the copies the warp already issued and leaves that
 * call's output unspecified; the GPU context stays usable and later calls
 * with the default are normal.
 */
#define BVML_UPSAMPLE_WAIT_DEFAULT 4194304u
unsigned bvml_upsample_wait_limit(unsigned limit);

/*
 * The whole refine-ops unit of Refiner::forward (src/dsine_refine.cpp:241-292)
 * for B frames, fused into two kernel launches (one persistent launch for all
 * AngMF iterations, one for the upsample; iters + 1 launches for shapes the
 * persistent kernel does not take: grid widths that are not a multiple of 16
 * bytes of storage, or dilations above 2):
 *   n = RayReLU(normal0, ray8)                      (fused into iteration 0)
 *   repeat iters times: n = AngMF(n, prob[i], xy[i], angle[i], ray8)
 *   up = L2normalise(ConvexUpsample8(n, mask))      (upsampled once: the
 *        reference recomputes it every iteration but only keeps the last)
 *   if full_res_ray_relu: up = RayReLU(up, full-res ray from 8x the intrinsics)
 *   out = crop(up, crop_t, crop_l, out_h, out_w)
 *   normal0 (B,3,h,w)  ray8 (3,h,w) fp32 or NULL (then computed from the
 *   intrinsics exactly as get_ray_core, src/dsine_decoder.cpp:242-261)
 *   prob/xy/angle: HOST arrays of `iters` device pointers, shapes as in
 *   bvml_angmf_propagate   mask (B,576,h,w)   out (B,3,out_h,out_w)
 * Intermediate normals stay fp32 in `workspace` (>= bvml_refine_workspace_bytes,
 * 256-byte aligned); storage-typed tensors follow `dtype`.
 */
int bvml_refine(const void* normal0, const float* ray8, const void* const* prob,
                const void* const* xy, const void* const* angle, int iters, const void* mask,
                int B, int h, int w, int ps, int dil, double fu, double cu, double fv,
                double cv, int full_res_ray_relu, int crop_t, int crop_l, int out_h,
                int out_w, int dtype, void* workspace, size_t workspace_bytes, void* out,
                void* stream);

/*
 * bvml_refine with every iteration's prob / angle given as the heads' raw
 * outputs (activated on load, as bvml_angmf_propagate_logits): the unit of
 * src/dsine_refine.cpp:241-292 including the activations at :262-267.
 */
int bvml_refine_logits(const void* normal0, const float* ray8, const void* const* prob_logits,
                       const void* const* xy, const void* const* angle_logits, int iters,
                       const void* mask, int B, int h, int w, int ps, int dil, double fu,
                       double cu, double fv, double cv, int full_res_ray_relu, int crop_t,
                       int crop_l, int out_h, int out_w, int dtype, void* workspace,
                       size_t workspace_bytes, void* out, void* stream);

/* Scratch bytes built into the library per device for bvml_refine_noalloc. */
#define BVML_REFINE_NOALLOC_MAX_BYTES (32u * 1024u * 1024u)

/*
 * bvml_refine for callers that cannot allocate device memory (no counterpart
 * in the reference, which allocates freely). Same arguments and results as
 * bvml_refine, minus the workspace: the scratch is a fixed 32 MiB array built
 * into this library, present on every GPU that loads it until the process
 * exits. For hosts that own the GPU memory budget and forbid allocations after
 * start-up (a plugin in another application's inference or render loop), or
 * loops that cannot take cudaMalloc's implicit device synchronisation.
 *  - Every call looks the array's device address up (cudaGetSymbolAddress)
 *    in the current device's context; no address is cached, so a device
 *    reset between calls is harmless. Under CUDA's default lazy module
 *    loading the first call on a device loads this library's device code
 *    there, which is when the 32 MiB are reserved: a caller with a fixed
 *    memory budget should make one call at start-up, before any stream
 *    capture.
 *  - Work needing more than BVML_REFINE_NOALLOC_MAX_BYTES of scratch
 *    (bvml_refine_workspace_bytes(B, h, w); about 1.39 M grid pixels, e.g. 96
 *    frames of 90x160) is rejected with BVML_EINVAL.
 *  - All calls on a device share the array: calls that overlap on the GPU
 *    (other streams or host threads) race and must be serialised by the
 *    caller. Nothing in it needs clearing between calls.
 *  - Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 */
int bvml_refine_noalloc(const void* normal0, const float* ray8, const void* const* prob,
                        const void* const* xy, const void* const* angle, int iters,
                        const void* mask, int B, int h, int w, int ps, int dil, double fu,
                        double cu, double fv, double cv, int full_res_ray_relu, int crop_t,
                        int crop_l, int out_h, int out_w, int dtype, void* out, void* stream);

/*
 * 2-D convolution, stride 1, zero padding ks/2 ("same"), on fp16 NHWC tensors
 * with fp32 accumulation on the tensor cores (tcgen05), plus bias and an
 * activation (0 none, 1 ReLU, 2 sigmoid, 3 tanh): the conv2d_forward calls of
 * the refine stage's ConvGRU (5x5, src/dsine_refine.cpp:140-158) and
 * prediction heads (3x3, 1x1, :118-125), which the reference runs through
 * brotensor on NCHW fp32 tensors.
 *   x    (B,H,W,cin_pad) fp16, cin_pad a multiple of 64, pad channels zero
 *   w    (ks*ks, cout_pad, cin_pad) fp16, w[ky*ks+kx][o][c] = weight[o][c][ky][kx]
 *   bias (cout) fp32
 *   y    (B,H,W,cout_pad) fp16, cout_pad a multiple of 64; channels >= cout
 *        are written as zeros, so y can be the next convolution's x
 *   ks in {1, 3, 5}; err: a device int the kernel sets nonzero if its
 *   pipeline had to give up (read it after synchronising; 0 = fine).
 */
int bvml_conv2d_nhwc_f16(const void* x, const void* w, const float* bias, int B, int H, int W,
                          int cin_pad, int cout, int cout_pad, int ks, int act, void* y,
                          int* err, void* stream);

/* Epilogue modes of bvml_conv2d_nhwc_f16_ex. */
#define BVML_EPI_NHWC 0        /* act(conv) as fp16 at out[pixel * out_c + out_off + o] */
#define BVML_EPI_PLANAR_F16 1  /* conv as fp16 at out[(b * cout + o) * H * W + y * W + x]
                                  (TMA stores when W * 2 is a multiple of 16 bytes,
                                  plain stores otherwise) */
#define BVML_EPI_PLANAR_F32 2  /* the same in fp32 */
#define BVML_EPI_GRU_ZR 3      /* ConvGRU gates z, r (cout = 128: z then r) */
#define BVML_EPI_GRU_Q 4       /* ConvGRU candidate and update (cout = 64) */
#define BVML_EPI_C4_F32 5      /* act(conv) as fp32 in channel groups of 4 (C4, below),
                                  out_c channels per frame, at channel out_off + o
                                  (act 0 or 1; out_c, out_off multiples of 4) */
#define BVML_EPI_SPLIT_F16 6   /* conv as two fp16 halves per 64-channel block:
                                  hi = fp16(v) at NHWC channel out_off + 128 (o / 64) +
                                  o % 64, lo = fp16(v - hi) 64 channels further (cout a
                                  multiple of 32, out_c >= out_off + 2 cout_pad): an
                                  extra-K operand (xin below) keeping ~16 bits of v */

/*
 * Where and how bvml_conv2d_nhwc_f16_ex writes its result. Channel strides
 * and offsets in elements, multiples of 8; tensors 16-byte aligned.
 * Channel-group layouts: C4 fp32 = [frame][C / 4][H][W][4] (channel c of
 * pixel (y, x) at ((f * C / 4 + c / 4) * H * W + y * W + x) * 4 + c % 4), C8
 * fp16 the same with groups of 8 -- 16 bytes per pixel and group, so the
 * epilogue's per-pixel reads and writes are coalesced.
 * GRU_ZR (src/dsine_refine.cpp:144-147): z = sigmoid(conv[0:64]) -> z
 *   (C8 fp16, 64 channels); r = sigmoid(conv[64:128]) -> rh[pixel * rh_c +
 *   o] = r * h, h the fp32 hidden state h32 (C4, 64 channels).
 * GRU_Q (:148-156): q = tanh(conv) -> h32 = (1 - z) h32 + z q, with fp16
 *   copies at hx[pixel * hx_c + o] and, when hin is not null, hin[...].
 * add (optional, every mode but the GRU ones): a per-pixel fp32 addend in C4 layout with
 *   add_c channels per frame (a multiple of 4, >= cout); channel o of frame f
 *   (f = 0 for every frame when add_shared is nonzero) joins conv[o] +
 *   bias[o] before the epilogue. It carries the part of a
 *   convolution whose input does not change between calls: the ConvGRU's
 *   feature and uv channels, the heads' uv channels, which the refine stage
 *   convolves once per refinement instead of once per iteration.
 * xin (optional, every mode): an extra K block, conv[o] += sum_k xin[pixel *
 *   xin_stride + k] * wx[o * xin_c + k] for k < xin_c, xin fp16 with
 *   xin_stride channels per pixel (0: xin_c; a multiple of 8), wx (cout_pad,
 *   xin_c) fp16, xin_c a multiple of 64 -- a 1x1 term the tensor cores add
 *   before the epilogue (the refine stage adds its hoisted terms this way, as
 *   BVML_EPI_SPLIT_F16 halves times identity blocks).
 */
typedef struct {
    int mode;
    int act;             /* NHWC: 0 none, 1 ReLU, 2 sigmoid, 3 tanh; C4_F32: 0, 1 */
    void* out;
    int out_c, out_off;
    float* h32;
    void* z;
    void* rh;
    int rh_c;
    void* hx;
    int hx_c;
    void* hin;
    int hin_c;
    const float* add;
    int add_c;
    int add_shared;
    const void* xin;     /* optional extra K, below */
    int xin_c;
    const void* wx;
    int xin_stride;
    unsigned wait_limit; /* attempts of each pipeline wait (between the TMA,
                            MMA and epilogue warps) before the kernel gives
                            up, sets *err and ends; 0: the default, 1 << 22.
                            The first attempt does not block, so 1 gives up
                            at the first wait that is not already satisfied.
                            The kernel still waits (with the default bound)
                            for its copies and MMAs in flight before it ends. */
} bvml_conv_epilogue;

/*
 * bvml_conv2d_nhwc_f16 reading input channels [cin_off, cin_off + cin_pad)
 * of x (B,H,W,x_c) fp16 (cin_off and cin_pad multiples of 64; x_c a multiple
 * of 8) and writing through `epi`: the fused ConvGRU gates and the
 * prediction heads' planar outputs, so that the refine stage runs on NHWC
 * buffers with no separate elementwise or layout passes.
 */
int bvml_conv2d_nhwc_f16_ex(const void* x, int x_c, int cin_off, int cin_pad, const void* w,
                             const float* bias, int B, int H, int W, int cout, int cout_pad,
                             int ks, const bvml_conv_epilogue* epi, int* err, void* stream);

/*
 * The last two layers of a prediction head in one kernel: conv1x1 (128 ->
 * 128) + ReLU + conv1x1 (128 -> cout), src/dsine_refine.cpp:118-125, which
 * the reference runs as two brotensor conv2d_forward calls and a relu_forward
 * with the 128-channel intermediate in memory; here it stays on the chip.
 *   x     (B,H,W,x_c) fp16 NHWC; input channels [cin_off, cin_off + 128)
 *         (cin_off a multiple of 64)
 *   w2    (1,128,128) fp16, b2 (128) fp32: the first 1x1 layer
 *   w4    (1,64,128) fp16 (rows >= cout zero), b4 (cout) fp32: the second
 *   out   (B,cout,H,W) planar, dtype BVML_F16 or BVML_F32; cout <= 64
 *   err   as bvml_conv2d_nhwc_f16
 * The results equal the two separate convolutions'
 * (bvml_conv2d_nhwc_f16_ex with NHWC + ReLU, then planar), bit for bit.
 */
int bvml_head_tail_1x1(const void* x, int x_c, int cin_off, const void* w2, const float* b2,
                       const void* w4, const float* b4, int B, int H, int W, int cout,
                       int dtype, void* out, int* err, void* stream);

/*
 * The refine stage's inputs in its layouts, one pass: the decoder's hidden
 * state h0 and feature (B,64,H,W) fp32 planar -> the GRU state h32 (C4 fp32,
 * (B,16,H,W,4)) and its fp16 NHWC copy hx (B,H,W,64), and the feature as
 * NHWC fp16 fx (B,H,W,64); feat and fx may both be null. Replaces the
 * concat / layout work at the start of Refiner::forward
 * (src/dsine_refine.cpp:245-248) for the tensor-core stage.
 */
int bvml_stage_inputs(const float* h0, const float* feat, int B, int H, int W, float* h32,
                      void* hx, void* fx, void* stream);

/*
 * The whole learned refinement of Refiner::forward (src/dsine_refine.cpp:
 * 212-294) for C / C++ hosts that run no Python: an opaque handle holding the
 * refine stage's weights packed once for the tensor cores, and a forward that
 * runs `iters` iterations of the ConvGRU + the four prediction heads
 * (src/dsine_refine.cpp:95-158, 245-276) on the tensor cores and then the
 * fused refine ops on the heads' raw outputs (as bvml_refine_logits), on the
 * caller's stream. The same sequence and packing as the Python
 * brovisionml_b200.refiner.Refiner, with bit-identical results.
 *   weights: host fp32 arrays in the reference's OIHW layout, in the order of
 *     bvml_refiner_weight_name(0 .. BVML_REFINER_WEIGHTS - 1) (the reference's
 *     safetensors names, gru.convz.weight ... up_prob_head.4.bias) with the
 *     shapes bvml_refiner_weight_shape gives (biases: shape[1..3] = 0).
 *   normal (B,3,h,w), feature and hidden (B,64,h,w): the decoder's outputs,
 *     fp32 on the handle's device; intrins = raw (fx, fy, cx, cy) of the
 *     padded origH x origW image (src/dsine_refine.cpp:230-237);
 *     crop (crop_t, crop_l, out_h, out_w) in the 8x output (the
 *     DsineTransform's pad_t, pad_l, orig_h, orig_w); out (B,3,out_h,out_w)
 *     in dtype (the storage of the head outputs and of the result).
 * Buffers for a shape are allocated (cudaMalloc) on its first forward and
 * reused; bvml_refiner_status synchronises the stream and reports whether a
 * tensor-core pipeline or a persistent AngMF wait gave up.
 */
#define BVML_REFINER_WEIGHTS 30
typedef struct bvml_refiner bvml_refiner;
const char* bvml_refiner_weight_name(int i);
int bvml_refiner_weight_shape(int i, int* shape4);
int bvml_refiner_create(const float* const* weights, int device, bvml_refiner** out);
int bvml_refiner_forward(bvml_refiner* r, const float* normal, const float* feature,
                         const float* hidden, int B, int h, int w, const float* intrins,
                         int origH, int origW, int iters, int crop_t, int crop_l, int out_h,
                         int out_w, int dtype, void* out, void* stream);
int bvml_refiner_status(bvml_refiner* r, void* stream);
void bvml_refiner_destroy(bvml_refiner* r);

/*
 * Large frames without the reference's resolution cap (src/dsine.cpp:117-141:
 * downscale, refine, upsample back), for C / C++ hosts.
 *
 * bvml_refine_halo_rows: the grid rows of halo per side that make a row band
 * of the whole learned refinement (`iters` iterations of the ConvGRU + heads,
 * AngMF with a ps x ps window at dilation dil, then the upsample) equal the
 * whole-frame result; -1 (BVML_EINVAL) for arguments outside iters 0..64,
 * window 3/5/7, dilation 1..4. 22 for 5 iterations of 5x5 at dilation 1.
 *
 * bvml_refiner_forward_banded: the whole learned refinement of ONE frame from
 * HOST memory as exact-halo row bands (bvml_refine_halo_rows(iters, 5, 1)
 * rows of halo, clipped to the frame), dealt in turn over n_refiners handles
 * -- one per GPU, or several on one -- each driven by its own host thread and
 * stream. normal (3,h,w), feature and hidden (64,h,w): the decoder's fp32
 * outputs in host memory; intrins, origH, origW, iters, the crop and dtype as
 * for bvml_refiner_forward; out: HOST memory, (3, out_h, out_w) in dtype. Only
 * the bands whose owned rows reach the crop run. Synchronous: returns when the
 * frame is written. A failing band stops the others at their next band; the
 * error names the band's grid rows and its device. The result equals
 * bvml_refiner_forward on the whole frame up to the rounding of each band's
 * shifted principal point (max-abs below 1e-6 in the tests).
 */
int bvml_refine_halo_rows(int iters, int ps, int dil);
int bvml_refiner_forward_banded(bvml_refiner* const* refiners, int n_refiners,
                                const float* normal, const float* feature, const float* hidden,
                                int h, int w, const float* intrins, int origH, int origW,
                                int iters, int n_bands, int crop_t, int crop_l, int out_h,
                                int out_w, int dtype, void* out);

/*
 * Profiling aid (no reference counterpart): arm `n` caller-created CUDA events
 * (cudaEvent_t, cast to void*) for the calling thread. While armed,
 * bvml_refine records events[0] on its stream before its first kernel and
 * events[k] after its k-th kernel (k = 1 .. n-1), so the caller can time
 * every launch of the fused unit on the stream it runs on. n = 0 disarms.
 */
int bvml_probe_events(void* const* events, int n);

/* How many probe events the calling thread's last bvml_refine call recorded
 * (its kernel launches + 1). */
int bvml_probe_recorded(void);

/*
 * Checked builds only (libbvml_dsine_checked.so, compiled with BVML_CHECKED;
 * no reference counterpart): the kernels test their indices, shared-memory
 * offsets and TMA coordinates before each access, skip an access that fails
 * and record it. Returns the OR of the recorded check bits since the last
 * reset (0: every access was in bounds; bit 30: a word could not be read)
 * and resets them when `reset` is nonzero. The release library returns -1.
 * Synchronous: call after the work has completed.
 */
int bvml_check_word(int reset);

#ifdef __cplusplus
}
#endif

#endif /* BVML_DSINE_H */
