// SIMT operator kernels around the tensor-core path (see misc.cu).
#pragma once
#include "kernels.h"

namespace qpc {

constexpr int kMaxDims = 6;

// A contiguous output of `rank` dims with per-dim element strides of up to
// two strided (possibly broadcast, stride 0) inputs.
struct StridedDims {
  int rank = 0;
  int64_t total = 0;
  int64_t dims[kMaxDims] = {};
  int64_t sa[kMaxDims] = {};
  int64_t sb[kMaxDims] = {};
};

// Batched small matmul with a two-level batch and arbitrary element strides.
struct BmmDims {
  int nb0 = 1, nb1 = 1, m = 0, n = 0, k = 0;
  int64_t sa0 = 0, sa1 = 0, sam = 0, sak = 0;
  int64_t sb0 = 0, sb1 = 0, sbk = 0, sbn = 0;
};

cudaError_t launch_convt2x2(const float* x, const float* wt, const float* bn_a, const float* bn_b,
                            float* y, int n, int h, int w, int c, int m, const ActParams& act,
                            cudaStream_t st, unsigned int* err = nullptr);
cudaError_t launch_gap_nhwc(const float* x, float* y, int n, int hw, int c, cudaStream_t st);
cudaError_t launch_pool2d_nhwc(const float* x, float* y, int n, int h, int w, int c, int oh, int ow,
                               int kh, int kw, int sh, int sw, int ph, int pw, int is_max,
                               cudaStream_t st);
// Nearest-neighbour resize sources written by one launch (FPN concat slices).
constexpr int RESIZE_MAX_SRC = 4;
struct ResizeSrcs {
  const float* x[RESIZE_MAX_SRC];  // NHWC [n, h, w, 4 * c4]
  int h[RESIZE_MAX_SRC], w[RESIZE_MAX_SRC], c4[RESIZE_MAX_SRC];
  int c_off[RESIZE_MAX_SRC];       // first output channel of each source's slice
  int n;                           // sources used
  int quads;                       // sum of c4
  int round_tf32;                  // store tf32-rounded (nearest) values
};
cudaError_t launch_resize_nearest_multi_nhwc(const ResizeSrcs& s, float* y, int n, int oh, int ow, int ldc,
                                             cudaStream_t st);
cudaError_t launch_resize_nearest_nhwc(const float* x, float* y, int n, int h, int w, int c, int oh,
                                       int ow, int ldc, int c_off, cudaStream_t st);
cudaError_t launch_binary(const float* a, const float* b, float* y, const StridedDims& sd, int op,
                          const ActParams& post, cudaStream_t st);
cudaError_t launch_unary(const float* a, float* y, const StridedDims& sd, const ActParams& act,
                         cudaStream_t st);
cudaError_t launch_mul_add_scale_nhwc(const float* f, const float* g, const float* r, float* y,
                                      int64_t total, int hw, int c, int gate_per_n, cudaStream_t st);
cudaError_t launch_copy_strided(const float* a, float* y, const StridedDims& sd, cudaStream_t st);
cudaError_t launch_copy_channels(const float* x, float* y, int64_t pix, int c, int ldc, int c_off,
                                 cudaStream_t st);
cudaError_t launch_reduce_mean(const float* x, float* y, int64_t outer, int64_t mid, int64_t inner,
                               cudaStream_t st);
cudaError_t launch_softmax_rows(const float* x, float* y, int64_t rows, int inner, cudaStream_t st);
cudaError_t launch_bmm_small(const float* a, const float* b, float* c, const BmmDims& d,
                             cudaStream_t st);
cudaError_t launch_argmax_pairs(const float* x, float* pairs, int64_t rows, int cols,
                                cudaStream_t st);
cudaError_t launch_affine_nhwc(const float* x, const float* a, const float* b, float* y,
                               int64_t total, int c, const ActParams& act, cudaStream_t st);

cudaError_t launch_copy_view(const float* a, float* y, const StridedDims& sd, cudaStream_t st);
// round: store tf32-rounded (nearest, ties away) outputs, for a value that
// is read only as a TF32 A operand.
cudaError_t launch_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                             int64_t rows, int c, float eps, int round, cudaStream_t st);
// Fused SVTR multi-head attention: qkv [B, T, 3*H*D] -> out [B, T, H*D]
// (q scaled, softmax(q k^T) v per head), bit-identical to the reference's
// Mul / MatMul / Softmax / MatMul ops.  D <= 32.
cudaError_t launch_attention(const float* qkv, int64_t B, int T, int H, int D, float scale, float* out,
                             cudaStream_t st);
cudaError_t launch_softmax_argmax(const float* x, float* pairs, int64_t rows, int cols,
                                  cudaStream_t st);

}  // namespace qpc
