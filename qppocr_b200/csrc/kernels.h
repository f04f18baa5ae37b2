// Launchers for the sm_100a kernels of the qppocr B200 backend.  All tensors
// are fp32 device pointers; 4-D activations are NHWC.  Every launcher returns
// a cudaError_t from the launch itself (asynchronous faults surface at the
// next synchronisation).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "runtime.h"

namespace qpc {

// Convolution geometry (ONNX Conv attributes after pad resolution;
// qppocr-kernels conv.rs:124-143 ConvParams).
struct ConvGeom {
  int n, h, w, c;        // input NHWC
  int oh, ow, m;         // output spatial and channels
  int kh, kw, sh, sw;
  int ph, pw;            // begin pads (end pads are implied by oh/ow)
};

// Tiled fp32 tensor map through the driver's cuTensorMapEncodeTiled (looked
// up once via the runtime).  dims / box innermost first, strides in bytes for
// dims 1..rank-1; out-of-bounds elements load as zero.  swizzle128: 128-byte
// swizzle (tensor-core operands) instead of the plain row layout.
bool make_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides, const uint32_t* box, bool swizzle128);

// Failure-path self-test: one CTA initialises an mbarrier that nothing ever
// arrives on and waits for it with the bounded wait every pipelined kernel
// uses (mbar_wait_for), here with a limit of limit_ns.  The wait runs out,
// raises KERR_MBAR_TIMEOUT in `err` and the kernel returns: the context stays
// usable and the host reads the flag like any kernel fault.
cudaError_t launch_wait_selftest(unsigned int* err, uint64_t limit_ns, cudaStream_t st);

// Depthwise conv (group == C, one filter per channel), NHWC in/out.
// wt is tap-major [kh*kw][C].  out = act(sum_taps + bias) (+ residual).
// Restates conv.rs:45-71 (fma from 0, ky outer / kx inner, bias after) with
// the fused activation and residual of conv.rs:673-713.
// `err`: device error word for the tiled kernel's bounded waits (null: the
// untiled kernel, which has no waits).
cudaError_t launch_dwconv_nhwc(const float* x, const float* wt, const float* bias,
                               const float* residual, float* y, const ConvGeom& g,
                               const ActParams& act, cudaStream_t st, unsigned int* err = nullptr);

// GEMM epilogue: out[r, col] = act(acc + bias[col]) + residual[r', col]
// where r' = r, or, for a nearest-upsample residual (FPN top-down add fused
// into the lateral 1x1 conv), the row of the coarser map that the nearest
// resize of resize.rs:8-57 reads.
struct GemmEpilogue {
  const float* bias = nullptr;      // [N]
  const float* residual = nullptr;  // [Mres, ldr]
  float* out = nullptr;             // [M, ldo]
  int ldo = 0, ldr = 0;
  int col_off = 0;                  // column offset of this GEMM inside `out`
  ActParams act{};
  // nearest-upsample residual: output rows are pixels of an (n, oh, ow) map;
  // the residual is an (n, rh, rw) map. rh == 0 disables the remap.
  int oh = 0, ow = 0, rh = 0, rw = 0;
  // Per-image channel gate on A (SE block: the 1x1 conv reads x * g with g
  // [images, K] broadcast over each image's a_gate_rows pixels), applied as A
  // is rounded on chip, so x * g is never written.  Rows-mode GEMM only.
  const float* a_gate = nullptr;
  int a_gate_rows = 0;
  // Row-argmax epilogue (CTC head): instead of storing D, each CTA (a
  // contiguous run of tiles) has each epilogue group write, per row of each
  // row block it covers, (max, argmax bits, sum exp(l - max)) over the
  // group's columns there to partials[slot * M + row] (float4), slot = the
  // group's first column tile in that block; nothing is written to `out`.
  // Buffer: n_tiles * M float4, of which launch_argmax_combine reads only the
  // slots written.
  float4* partials = nullptr;
  // A already rounded to tf32 by its producer (a depthwise conv with
  // ActParams::round_tf32, or an epilogue / resize storing rounded values):
  // TF32 rows-mode GEMMs and the tap-folded conv skip their rounding pass.
  int a_rounded = 0;
  // Store the outputs rounded to tf32 (nearest), after bias, activation and
  // residual: set when every consumer reads them only as a TF32 A operand,
  // which would round them to the same values.
  int round_out = 0;
  // ConvT pair epilogue (two 2x2 stride-2 ConvTranspose layers, the second
  // to one channel; launch_convt_pair): set by that launcher only.
  int pair_h = 0, pair_w = 0;  // input map of the first ConvT
  ActParams pair_act{};        // activation after the second ConvT
};

enum MathMode : int { MATH_TF32 = 0, MATH_3XTF32 = 1 };

// Row-major GEMM on tcgen05 tensor cores: D[M,N] = A[M,K] * B[N,K]^T with the
// fused epilogue.  A rows are NHWC pixels (or tokens); B is the weight matrix
// in the ONNX Conv layout [Cout, Cin] (K-major).  For MATH_3XTF32, b_lo holds
// B - tf32(B) (prepared at load time) and A is split on chip.
// K % 4 == 0 (16-byte TMA row pitch); pointers 16-byte aligned.  `err` is the
// device error word that a timed-out pipeline wait sets.
cudaError_t launch_gemm_tc(const float* a, int64_t M, int K, int lda, const float* b,
                           const float* b_lo, int N, const GemmEpilogue& epi, int math,
                           unsigned int* err, cudaStream_t st);

// Number of output-column tiles launch_gemm_tc uses for N with the
// row-argmax epilogue (sizes the partials buffer: n_tiles * M float4).
int gemm_tc_col_tiles(int N, int math);

// Combines row-argmax partials into (value, index-bits) pairs: the first
// strict maximum over all columns (ties -> lowest column) and its softmax
// probability 1 / sum_j exp(l_j - max).  `math` must be the head GEMM's
// (it fixes the number of epilogue workers, hence the slots written).
cudaError_t launch_argmax_combine(const float4* partials, int n_tiles, int64_t M, int math, float* pairs,
                                  cudaStream_t st);
// CTAs of the CTC head GEMM over M rows and n_tiles column tiles on the
// current device; each owns a contiguous tile range, and each of its epilogue
// groups leaves one partial per row of every row block it touches.
int head_workers(int64_t M, int n_tiles, int math);

// kxk stride-1 dense conv as implicit GEMM on tcgen05: A tiles are 4-D TMA
// boxes of the NHWC input shifted per tap (out-of-bounds rows/cols read as
// the zero padding).  wk is tap-major [kh*kw][M][C] (and wk_lo its 3xTF32
// residue).  Epilogue as launch_gemm_tc with out rows = output pixels.
// wk_fold (optional, TF32 only): the kx-folded filter [kh][roundup16(kw*M)][C]
// (tf32-rounded) for the tap-folded kernel, used when conv_fold_ok(g).
cudaError_t launch_conv_tc(const float* x, const ConvGeom& g, const float* wk, const float* wk_lo,
                           const GemmEpilogue& epi, int math, unsigned int* err,
                           cudaStream_t st, const float* wk_fold = nullptr);

// Two 2x2 stride-2 ConvTranspose layers back to back, the second to one
// channel (DB head: ConvT -> BN -> act1 -> ConvT -> act2; executor.rs:654-731,
// conv.rs:730-838), as one tcgen05 GEMM of the first layer whose epilogue
// finishes the second, so the 2x-upsampled intermediate is never written.
//   x     n x h x w x c NHWC, c % 4 == 0; m1 (<= 32) channels between the layers
//   b1    [128][c]: row 32 (2 dy + dx) + m = W1[c][m][dy][dx] * scale[m] for
//         m < m1 (the first layer's BN scale folded in; other rows zero),
//         tf32-rounded (b1_lo: 3xTF32 residue)
//   consts  shift[128] (BN shift of the first layer per column, zero on
//         padding columns), w2[32][4] = W2[m][0][ey][ex] (zero rows past m1);
//         256 floats in HOST memory, passed to the kernel by value
//   out   n x 4h x 4w (one channel): out[4y + 2dy + ey][4x + 2dx + ex] =
//         act2(sum_m act1(acc[32 s + m] + shift) * w2[m][2 ey + ex])
cudaError_t launch_convt_pair(const float* x, int n, int h, int w, int c, int m1, const float* b1,
                              const float* b1_lo, const float* consts, const ActParams& act1,
                              const ActParams& act2, float* out, int math, unsigned int* err,
                              cudaStream_t st);

// Fused depthwise-separable block (dwpw.cu): a depthwise conv `g` (group ==
// C, k = 3 or 5, equal strides 1 or 2, C == 16 or C % 32 == 0) whose output
// feeds only a TF32 pointwise conv to n_out (<= 256) channels, in one tcgen05
// kernel: y = epi(pw_w * round_tf32(act(dw(x) + dw_bias))).  dw_w is
// tap-major [k*k][C]; pw_w is [n_out][C], tf32-rounded; epi supplies the
// pointwise bias, activation and output (no residual).  The depthwise part
// is bit-identical to launch_dwconv_nhwc and the pointwise part to
// launch_gemm_tc on its (rounded) output.
bool dwpw_ok(const ConvGeom& g, int n_out);
cudaError_t launch_dwpw(const float* x, const ConvGeom& g, const float* dw_w, const float* dw_bias,
                        const ActParams& dw_act, const float* pw_w, int n_out, const GemmEpilogue& epi,
                        unsigned int* err, cudaStream_t st);

// Whether the tap-folded TF32 kernel takes this conv (kw <= 3, M <= 32,
// output rows >= 48 wide, stride 1, filter within the shared-memory budget).
bool conv_fold_ok(const ConvGeom& g);

// Direct (SIMT) dense conv for shapes the tensor-core path does not take
// (C % 4 != 0 stems, strided kxk).  Input is NCHW when x_nchw != 0 (graph
// input), NHWC otherwise.  w is the ONNX layout [M][C/group][kh][kw].
// Accumulation order: ch -> ky -> kx ascending, fma from 0, bias after
// (gemm.rs:75-128 implicit-GEMM k order).  w_host / bias_host: host copies
// of w and bias (the 3 -> 8/16/32 stride-2 stem specialisation takes its
// filter by value from them; without them the generic kernel runs).
cudaError_t launch_conv_direct(const float* x, int x_nchw, const float* w, const float* bias,
                               const float* residual, float* y, const ConvGeom& g, int group,
                               const ActParams& act, cudaStream_t st, unsigned int* err = nullptr,
                               const float* w_host = nullptr, const float* bias_host = nullptr);

// ---- det / rec pre and post (prepost.cu), bit-exact with the reference's
// host code.  Images are n x h x w x 3 uint8 (HWC), masks n x h x w uint8.
// Bilinear RGB u8 resize (qppocr-kernels resize.rs:158-210).
cudaError_t launch_resize_bilinear_rgb_u8(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh,
                                          int dw, cudaStream_t st);
// Det input (engine.rs:930-982): resize to dh x dw (skipped when equal), then
// (u8 / 255 - 0.5) * 2 into planar n x 3 x dh x dw f32.
cudaError_t launch_det_preprocess(const uint8_t* src, int n, int sh, int sw, float* dst, int dh, int dw,
                                  cudaStream_t st);
// Rec line pack (crop.rs:153-185 into engine.rs:1425-1440's zeroed batch): n
// uint8 crops (h x w x 3 at byte offsets off) -> n x 3 x img_h x img_w f32,
// line k resized to rws[k] x img_h (or centred unresized when pads[k]).
// All arrays on the device.
cudaError_t launch_rec_pack(const uint8_t* crops, const int64_t* off, const int* hs, const int* ws,
                            const int* rws, const int* pads, int n, int img_h, int img_w, float* out,
                            cudaStream_t st);
// DB mask (geometry.rs:286-296): pred > thresh (or an existing u8 mask when
// pred is null), then the 2x2 dilation when `dilate`.
cudaError_t launch_db_mask(const float* pred, const uint8_t* mask_in, uint8_t* out, int n, int h, int w,
                           float thresh, int dilate, cudaStream_t st);

// ---- text boxes and line preparation (crop.cu), bit-exact with the
// reference's host code.
// box_score_fast (geometry.rs:221-269) per box: pred is n x h x w, boxes
// [n_boxes][4][2] (x, y) in pred coordinates, img[k] the box's image.
cudaError_t launch_box_score(const float* pred, int h, int w, const float* boxes, const int* img, int n,
                             float* out, cudaStream_t st);
// crop_text_box (crop.rs:8-127) per box from n images of h x w x 3 uint8:
// box k (corners pts[8k..8k+7]) of image img[k] -> cw[k] x ch[k] x 3 bytes at
// out + off[k] (rotated clockwise, ch x cw, when ch / cw >= 1.5); max_pixels
// is the largest cw * ch (sizes the grid).
cudaError_t launch_crop_boxes(const uint8_t* imgs, int h, int w, const float* pts, const int* img, const int* cw,
                              const int* ch, const int64_t* off, int n, int max_pixels, uint8_t* out,
                              cudaStream_t st);
// Per-line views for launch_line_pack (device arrays, one entry per line).
struct LinePack {
  const int64_t* off;  // byte offset of the line's crop
  const int* stride;   // pixels per crop row
  const int* x0;       // first column of the view in the crop
  const int* h;        // view rows
  const int* w;        // view columns
  const int* rw;       // resized width (ignored when pad)
  const int* pad;      // 1: unresized, centred vertically (pack_crop's pad_only)
  const int* flip;     // 1: view rotated 180 degrees; null: none
};
// pack_crop (crop.rs:153-185) of each line's view into a zeroed
// [3, img_h, img_w] slot of out (n slots): the rec batch and, with cls_view
// windows (crop.rs:193-218), the cls batch.
cudaError_t launch_line_pack(const uint8_t* crops, const LinePack& lp, int n, int img_h, int img_w, float* out,
                             cudaStream_t st);

}  // namespace qpc
