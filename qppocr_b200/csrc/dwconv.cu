// Depthwise convolution, NHWC, fp32 — the bandwidth-bound half of every
// depthwise-separable block (qppocr-kernels conv.rs:461-505, 912-1051).
//
// Each thread produces 4 consecutive channels (one float4) of RUN consecutive
// output pixels along a row.  Per channel the accumulation is exactly the
// reference's scalar plane kernel (conv.rs:45-71): acc = 0, then
// acc = fma(w, x, acc) over taps ky-major / kx-minor, padding taps reading 0,
// then + bias, then the fused activation, then + residual.  The result is
// bit-identical to the reference CPU path for the same inputs.
#include "kernels.h"

namespace qpc {

template <int KH, int KW, int SW, int RUN>
__global__ void __launch_bounds__(256) dwconv_nhwc_kernel(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bias,
    const float* __restrict__ residual, float* __restrict__ y, int N, int H, int W, int C, int OH,
    int OW, int SH, int PH, int PW, ActParams act) {
  const int C4 = C >> 2;
  const int runs = (OW + RUN - 1) / RUN;
  const int64_t total = (int64_t)N * OH * runs * C4;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int c4 = (int)(t % C4);
    int64_t r = t / C4;
    const int run = (int)(r % runs);
    r /= runs;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    const int ox0 = run * RUN;
    float4 acc[RUN];
#pragma unroll
    for (int i = 0; i < RUN; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* wt4 = reinterpret_cast<const float4*>(wt) + c4;
#pragma unroll
    for (int ky = 0; ky < KH; ++ky) {
      const int iy = oy * SH - PH + ky;
      const bool row_ok = iy >= 0 && iy < H;
      const float4* xrow = reinterpret_cast<const float4*>(x) + ((int64_t)(n * H + iy) * W) * C4 + c4;
#pragma unroll
      for (int kx = 0; kx < KW; ++kx) {
        const float4 w4 = __ldg(wt4 + (ky * KW + kx) * C4);
#pragma unroll
        for (int i = 0; i < RUN; ++i) {
          const int ix = (ox0 + i) * SW - PW + kx;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (row_ok && ix >= 0 && ix < W) v = __ldg(xrow + (int64_t)ix * C4);
          acc[i].x = __fmaf_rn(w4.x, v.x, acc[i].x);
          acc[i].y = __fmaf_rn(w4.y, v.y, acc[i].y);
          acc[i].z = __fmaf_rn(w4.z, v.z, acc[i].z);
          acc[i].w = __fmaf_rn(w4.w, v.w, acc[i].w);
        }
      }
    }
    const float4 b4 = bias ? __ldg(reinterpret_cast<const float4*>(bias) + c4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    float vals[4 * RUN];
#pragma unroll
    for (int i = 0; i < RUN; ++i) {
      vals[4 * i] = __fadd_rn(acc[i].x, b4.x);
      vals[4 * i + 1] = __fadd_rn(acc[i].y, b4.y);
      vals[4 * i + 2] = __fadd_rn(acc[i].z, b4.z);
      vals[4 * i + 3] = __fadd_rn(acc[i].w, b4.w);
    }
    apply_act_n(vals, act);
#pragma unroll
    for (int i = 0; i < RUN; ++i) {
      const int ox = ox0 + i;
      if (ox >= OW) break;
      float4 o = make_float4(vals[4 * i], vals[4 * i + 1], vals[4 * i + 2], vals[4 * i + 3]);
      const int64_t oidx = ((int64_t)(n * OH + oy) * OW + ox) * C4 + c4;
      if (residual) {
        const float4 rr = __ldg(reinterpret_cast<const float4*>(residual) + oidx);
        o.x = __fadd_rn(o.x, rr.x);
        o.y = __fadd_rn(o.y, rr.y);
        o.z = __fadd_rn(o.z, rr.z);
        o.w = __fadd_rn(o.w, rr.w);
      }
      reinterpret_cast<float4*>(y)[oidx] = o;
    }
  }
}

// Generic-kernel-size fallback (one pixel per thread).
__global__ void __launch_bounds__(256) dwconv_nhwc_generic(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bias,
    const float* __restrict__ residual, float* __restrict__ y, int N, int H, int W, int C, int OH,
    int OW, int KH, int KW, int SH, int SW, int PH, int PW, ActParams act) {
  const int64_t total = (int64_t)N * OH * OW * C;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(t % C);
    int64_t r = t / C;
    const int ox = (int)(r % OW);
    r /= OW;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    float acc = 0.f;
    for (int ky = 0; ky < KH; ++ky)
      for (int kx = 0; kx < KW; ++kx) {
        const int iy = oy * SH - PH + ky, ix = ox * SW - PW + kx;
        const float v = (iy >= 0 && iy < H && ix >= 0 && ix < W)
                            ? __ldg(x + ((int64_t)(n * H + iy) * W + ix) * C + c)
                            : 0.f;
        acc = __fmaf_rn(__ldg(wt + (ky * KW + kx) * C + c), v, acc);
      }
    float o = apply_act(__fadd_rn(acc, bias ? __ldg(bias + c) : 0.f), act);
    if (residual) o = __fadd_rn(o, __ldg(residual + t));
    y[t] = o;
  }
}

static int grid_for(int64_t threads) {
  int64_t blocks = (threads + 255) / 256;
  const int64_t cap = 148 * 16;  // persistent-style cap: 16 resident 256-thread CTAs per SM
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

cudaError_t launch_dwconv_nhwc(const float* x, const float* wt, const float* bias,
                               const float* residual, float* y, const ConvGeom& g,
                               const ActParams& act, cudaStream_t st) {
  constexpr int RUN = 4;
  const bool vec = (g.c % 4) == 0;
  const int runs = (g.ow + RUN - 1) / RUN;
  const int64_t vthreads = (int64_t)g.n * g.oh * runs * (g.c / 4);
#define QPC_DW(KH_, KW_, SW_)                                                                  \
  if (vec && g.kh == KH_ && g.kw == KW_ && g.sw == SW_) {                                      \
    dwconv_nhwc_kernel<KH_, KW_, SW_, RUN><<<grid_for(vthreads), 256, 0, st>>>(               \
        x, wt, bias, residual, y, g.n, g.h, g.w, g.c, g.oh, g.ow, g.sh, g.ph, g.pw, act);      \
    return cudaGetLastError();                                                                 \
  }
  QPC_DW(3, 3, 1)
  QPC_DW(3, 3, 2)
  QPC_DW(5, 5, 1)
  QPC_DW(5, 5, 2)
  QPC_DW(7, 7, 1)
  QPC_DW(7, 7, 2)
#undef QPC_DW
  dwconv_nhwc_generic<<<grid_for((int64_t)g.n * g.oh * g.ow * g.c), 256, 0, st>>>(
      x, wt, bias, residual, y, g.n, g.h, g.w, g.c, g.oh, g.ow, g.kh, g.kw, g.sh, g.sw, g.ph, g.pw,
      act);
  return cudaGetLastError();
}

}  // namespace qpc
