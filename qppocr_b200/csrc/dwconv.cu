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
      if (act.round_tf32) o = make_float4(tf32_rna(o.x), tf32_rna(o.y), tf32_rna(o.z), tf32_rna(o.w));
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
    y[t] = act.round_tf32 ? tf32_rna(o) : o;
  }
}

// Shared-memory tiled variant (C % 16 == 0, square kernels, equal strides).
// A persistent block walks tiles (channel chunk of CC, image, TH x TW output
// pixels), chunk-major so a block keeps its filter registers across tiles.
// The tile's input window, ((TH-1)*S + K) x ((TW-1)*S + K) pixels x CC
// channels, arrives by one 4-D TMA load (zeros outside the image, which the
// padding taps multiply exactly as the reference's zero padding does) into
// one of two shared-memory buffers, the next tile's load overlapping this
// tile's arithmetic.  Thread (group g, quad q) makes channels 4q..4q+3 of a
// run of R pixels along a row: per kernel row it reads the (R-1)*S + K input
// quads once and applies all K taps to the run.  Per element the chain is the
// scalar kernel's: fma from 0 over ky outer / kx inner, + bias, act,
// + residual (bit-identical).
template <int K, int S, int CC, int TW, int TH, int MINB>
struct DwTile {
  static constexpr int Q = CC / 4;                 // channel quads per pixel
  static constexpr int G = 256 / Q;                // pixel groups
  static constexpr int R = TW * TH / G;            // pixels per group (one row run)
  static constexpr int IW = (TW - 1) * S + K, IH = (TH - 1) * S + K;
  static constexpr int NC = (R - 1) * S + K;       // input quads per kernel row of a run
  static constexpr int BUF = ((IW * IH * CC * 4 + 1023) / 1024) * 1024;
  // MINB == 1: one block per SM, filter slice in registers, up to 4 windows
  // in flight; MINB == 2: two blocks per SM (registers capped), filter slice
  // in shared memory, 2 windows each.
  static constexpr int STAGES = MINB == 1 ? ((220 * 1024) / BUF > 4 ? 4 : (220 * 1024) / BUF) : 2;
  static constexpr int WBYTES = MINB == 1 ? 0 : K * K * CC * 4;
  static constexpr int SMEM = STAGES * BUF + WBYTES + 1024;
  static_assert(TW % R == 0 && R >= 1, "runs must not cross rows");
  static_assert(STAGES >= 2 && SMEM <= (MINB == 1 ? 224 : 112) * 1024, "windows do not fit");
};

template <int K, int S, int CC, int TW, int TH, int MINB>
__global__ void __launch_bounds__(256, MINB) dwconv_tile_kernel(
    const __grid_constant__ CUtensorMap tmX, const float* __restrict__ wt, const float* __restrict__ bias,
    const float* __restrict__ residual, float* __restrict__ y, int N, int C, int OH, int OW, int PH, int PW,
    ActParams act, unsigned int* err) {
  using T = DwTile<K, S, CC, TW, TH, MINB>;
  extern __shared__ __align__(1024) uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int NS = T::STAGES;
  __shared__ __align__(8) uint64_t full[NS];
  const int tid = threadIdx.x;
  const int q = tid % T::Q, g = tid / T::Q;
  const int run0 = g * T::R;                     // first pixel of this thread's run
  const int ty = run0 / TW, tx0 = run0 % TW;
  const int tiles_x = (OW + TW - 1) / TW, tiles_y = (OH + TH - 1) / TH;
  const int per_chunk = N * tiles_y * tiles_x;
  const int total = (C / CC) * per_chunk;
  const uint32_t bytes = (uint32_t)(T::IW * T::IH * CC * 4);
  if (tid == 0) {
    for (int b = 0; b < NS; ++b) mbar_init(&full[b], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmX);
  }
  __syncthreads();
  auto issue = [&](int tile, int buf) {
    const int chunk = tile / per_chunk;
    int r = tile % per_chunk;
    const int bx = r % tiles_x;
    r /= tiles_x;
    const int by = r % tiles_y, n = r / tiles_y;
    fence_proxy_async_smem();  // earlier generic reads of this buffer before the async write
    mbar_arrive_expect_tx(&full[buf], bytes);
    tma_load_4d(dsm + buf * T::BUF, &tmX, &full[buf], chunk * CC, bx * TW * S - PW, by * TH * S - PH, n);
  };
  if (tid == 0)
    for (int j = 0; j < NS - 1; ++j)
      if ((int)blockIdx.x + j * (int)gridDim.x < total) issue(blockIdx.x + j * gridDim.x, j);
  int cur_chunk = -1;
  float4* wsm = reinterpret_cast<float4*>(dsm + NS * T::BUF);  // [K*K][Q] (MINB == 2)
  float4 wr[MINB == 1 ? K * K : 1];                             // (MINB == 1)
  float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
    const int buf = it % NS;
    // the buffer of iteration it + NS - 1 was last read in iteration it - 1
    const int ahead = tile + (NS - 1) * (int)gridDim.x;
    if (tid == 0 && ahead < total) issue(ahead, (it + NS - 1) % NS);
    const int chunk = tile / per_chunk;
    int r = tile % per_chunk;
    const int bx = r % tiles_x;
    r /= tiles_x;
    const int by = r % tiles_y, n = r / tiles_y;
    const int c = chunk * CC + 4 * q;
    if (chunk != cur_chunk) {  // uniform: every thread sees the same tile
      cur_chunk = chunk;
      if (MINB == 1) {
#pragma unroll
        for (int k = 0; k < K * K; ++k)
          wr[k % (MINB == 1 ? K * K : 1)] = __ldg(reinterpret_cast<const float4*>(wt + (int64_t)k * C + c));
      } else {
        for (int i = tid; i < K * K * T::Q; i += 256)
          wsm[i] = __ldg(reinterpret_cast<const float4*>(wt + (int64_t)(i / T::Q) * C + chunk * CC) + i % T::Q);
        __syncthreads();
      }
      if (bias) b4 = __ldg(reinterpret_cast<const float4*>(bias + c));
    }
    const bool ok = mbar_wait(&full[buf], (it / NS) & 1u, err);
    if (ok) {
      const float4* xs = reinterpret_cast<const float4*>(dsm + buf * T::BUF);
      float4 acc[T::R];
#pragma unroll
      for (int i = 0; i < T::R; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int ky = 0; ky < K; ++ky) {
        const float4* row = xs + ((ty * S + ky) * T::IW + tx0 * S) * T::Q + q;
        float4 xr[T::NC];
#pragma unroll
        for (int j = 0; j < T::NC; ++j) xr[j] = row[j * T::Q];
#pragma unroll
        for (int kx = 0; kx < K; ++kx) {
          const float4 wv = MINB == 1 ? wr[(ky * K + kx) % (MINB == 1 ? K * K : 1)] : wsm[(ky * K + kx) * T::Q + q];
#pragma unroll
          for (int i = 0; i < T::R; ++i) {
            const float4 v = xr[i * S + kx];
            acc[i].x = __fmaf_rn(wv.x, v.x, acc[i].x);
            acc[i].y = __fmaf_rn(wv.y, v.y, acc[i].y);
            acc[i].z = __fmaf_rn(wv.z, v.z, acc[i].z);
            acc[i].w = __fmaf_rn(wv.w, v.w, acc[i].w);
          }
        }
      }
      const int oy = by * TH + ty;
#pragma unroll
      for (int i = 0; i < T::R; ++i) {
        const int ox = bx * TW + tx0 + i;
        float o[4] = {__fadd_rn(acc[i].x, b4.x), __fadd_rn(acc[i].y, b4.y), __fadd_rn(acc[i].z, b4.z),
                      __fadd_rn(acc[i].w, b4.w)};
        apply_act_n(o, act);
        if (oy < OH && ox < OW) {
          const int64_t oidx = (((int64_t)n * OH + oy) * OW + ox) * C + c;
          float4 v = make_float4(o[0], o[1], o[2], o[3]);
          if (residual) {
            const float4 rr = __ldg(reinterpret_cast<const float4*>(residual + oidx));
            v.x = __fadd_rn(v.x, rr.x);
            v.y = __fadd_rn(v.y, rr.y);
            v.z = __fadd_rn(v.z, rr.z);
            v.w = __fadd_rn(v.w, rr.w);
          }
          if (act.round_tf32) v = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
          *reinterpret_cast<float4*>(y + oidx) = v;
        }
      }
    }
    // buffer `buf` is refilled by the issue at the top of the next iteration;
    // a timed-out wait anywhere stops the whole block, after its loads land
    if (__syncthreads_or(!ok)) {
      if (tid == 0)
        for (int j = 0; j < NS; ++j)
          if (tile + j * (int)gridDim.x < total) mbar_wait(&full[(it + j) % NS], ((it + j) / NS) & 1u, nullptr);
      __syncthreads();
      break;
    }
  }
}

// Launch the tiled kernel if the geometry has an instantiation; returns
// cudaErrorNotSupported otherwise (the caller falls back).
template <int K, int S, int CC, int TW, int TH, int MINB>
cudaError_t run_dw_tile(const float* x, const float* wt, const float* bias, const float* residual,
                        float* y, const ConvGeom& g, const ActParams& act, unsigned int* err,
                        cudaStream_t st) {
  using T = DwTile<K, S, CC, TW, TH, MINB>;
  CUtensorMap map;
  const uint64_t dims[4] = {(uint64_t)g.c, (uint64_t)g.w, (uint64_t)g.h, (uint64_t)g.n};
  const uint64_t strides[3] = {(uint64_t)g.c * 4, (uint64_t)g.c * g.w * 4, (uint64_t)g.c * g.w * g.h * 4};
  const uint32_t box[4] = {CC, T::IW, T::IH, 1};
  if (!make_tensor_map(&map, x, 4, dims, strides, box, false)) return cudaErrorNotSupported;
  const int smem = T::SMEM;
  auto kern = dwconv_tile_kernel<K, S, CC, TW, TH, MINB>;
  cudaError_t ae = ensure_dyn_smem((const void*)kern, smem);
  if (ae != cudaSuccess) return ae;
  const int64_t tiles = (int64_t)(g.c / CC) * g.n * ((g.oh + TH - 1) / TH) * ((g.ow + TW - 1) / TW);
  const int per_sm = blocks_per_sm((const void*)kern, 256, smem);
  const int64_t cap = (int64_t)current_sm_count() * per_sm;
  const int grid = (int)(tiles < cap ? tiles : cap);
  kern<<<grid, 256, smem, st>>>(map, wt, bias, residual, y, g.n, g.c, g.oh, g.ow, g.ph, g.pw, act, err);
  return cudaGetLastError();
}

static int grid_for(int64_t threads) {
  int64_t blocks = (threads + 255) / 256;
  const int64_t cap = 148 * 16;  // persistent-style cap: 16 resident 256-thread CTAs per SM
  return (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

cudaError_t launch_dwconv_nhwc(const float* x, const float* wt, const float* bias,
                               const float* residual, float* y, const ConvGeom& g,
                               const ActParams& act, cudaStream_t st, unsigned int* err) {
  // Tiled TMA path: C % 16 == 0, 16-byte aligned pointers, square 3x3 / 5x5,
  // equal strides 1 or 2, the input window within the TMA box limits.
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(wt) |
                    reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(bias) |
                    reinterpret_cast<uintptr_t>(residual)) & 15) == 0;
  if (err && al && (g.c % 16) == 0 && g.kh == g.kw && g.sh == g.sw && g.ph < g.kh && g.pw < g.kw) {
    const bool c32 = (g.c % 32) == 0;
    cudaError_t e = cudaErrorNotSupported;
    // per geometry, the configuration measured fastest on the det backbone
    if (g.kh == 3 && g.sh == 1)
      e = c32 ? run_dw_tile<3, 1, 32, 32, 8, 2>(x, wt, bias, residual, y, g, act, err, st)
              : run_dw_tile<3, 1, 16, 32, 16, 2>(x, wt, bias, residual, y, g, act, err, st);
    else if (g.kh == 3 && g.sh == 2)
      e = c32 ? run_dw_tile<3, 2, 32, 16, 8, 1>(x, wt, bias, residual, y, g, act, err, st)
              : run_dw_tile<3, 2, 16, 16, 8, 1>(x, wt, bias, residual, y, g, act, err, st);
    else if (g.kh == 5 && g.sh == 1 && c32)
      // maps at most 4 rows tall (the rec lines' 3 x 40): a 40 x 4 tile, so
      // an 8-row tile does not compute 5 rows of nothing
      e = g.oh <= 4   ? run_dw_tile<5, 1, 32, 40, 4, 2>(x, wt, bias, residual, y, g, act, err, st)
          : g.ow <= 32 ? run_dw_tile<5, 1, 32, 10, 16, 2>(x, wt, bias, residual, y, g, act, err, st)
                       : run_dw_tile<5, 1, 32, 20, 8, 2>(x, wt, bias, residual, y, g, act, err, st);
    else if (g.kh == 5 && g.sh == 1)
      e = run_dw_tile<5, 1, 16, 32, 8, 1>(x, wt, bias, residual, y, g, act, err, st);
    else if (g.kh == 5 && g.sh == 2)
      e = c32 ? run_dw_tile<5, 2, 32, 16, 8, 1>(x, wt, bias, residual, y, g, act, err, st)
              : run_dw_tile<5, 2, 16, 16, 8, 1>(x, wt, bias, residual, y, g, act, err, st);
    if (e != cudaErrorNotSupported) return e;
  }
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
