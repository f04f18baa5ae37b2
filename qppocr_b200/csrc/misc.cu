// SIMT kernels for the operators around the tensor-core path.  Each restates
// one qppocr-kernels CPU routine element by element (cited per kernel), so
// that, given identical inputs, their outputs match the reference bit for bit
// (reductions in f64 match to the final f32 rounding).
#include "misc.h"

namespace qpc {

static int grid_for(int64_t threads, int block = 256) {
  int64_t blocks = (threads + block - 1) / block;
  const int64_t cap = 148 * 16;
  if (blocks < 1) blocks = 1;
  return (int)(blocks < cap ? blocks : cap);
}
#define GRID_LOOP(i, total) \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (total); i += (int64_t)gridDim.x * blockDim.x)

// ------------------------------------------------------------ self-test
__global__ void wait_selftest_kernel(unsigned int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    // nothing arrives: phase 0 never completes, so the bounded wait runs out
    mbar_wait_for(&bar, 0, err, limit_ns);
  }
}

cudaError_t launch_wait_selftest(unsigned int* err, uint64_t limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(err, limit_ns);
  return cudaGetLastError();
}

// ------------------------------------------------------------ direct conv
// Implicit-GEMM per-element semantics of conv.rs:553-637 / gemm.rs:75-128 and
// 523-589: k order ch -> ky -> kx; acc from 0 then + bias, except M%4 tail rows
// of a partial 32-wide output-column panel, which seed the chain with bias.
// Each thread computes MB output channels of one output pixel.
template <int MB>
__global__ void __launch_bounds__(256) conv_direct_kernel(
    const float* __restrict__ x, int x_nchw, const float* __restrict__ w,
    const float* __restrict__ bias, const float* __restrict__ residual, float* __restrict__ y,
    int N, int C, int H, int W, int M, int OH, int OW, int KH, int KW, int SH, int SW, int PH,
    int PW, int group, ActParams act) {
  const int cg = C / group, mg = M / group;
  const int mblocks = (M + MB - 1) / MB;
  const int64_t total = (int64_t)N * OH * OW * mblocks;
  const int m4 = mg - (mg % 4);
  const int full_cols = (OW / 32) * 32;
  GRID_LOOP(t, total) {
    const int mb = (int)(t % mblocks);
    int64_t r = t / mblocks;
    const int ox = (int)(r % OW);
    r /= OW;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    const int m0 = mb * MB;
    float acc[MB];
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      const int m = m0 + i;
      float seed = 0.f;
      if (m < M && bias) {
        const int mo = m % mg;
        if (mo >= m4 && ox >= full_cols) seed = __ldg(bias + m);
      }
      acc[i] = seed;
    }
    const int g = (m0 / mg);  // MB never straddles a group (MB divides mg or group == 1)
    for (int ch = 0; ch < cg; ++ch) {
      const int ci = g * cg + ch;
      for (int ky = 0; ky < KH; ++ky) {
        const int iy = oy * SH - PH + ky;
        for (int kx = 0; kx < KW; ++kx) {
          const int ix = ox * SW - PW + kx;
          float v = 0.f;
          if (iy >= 0 && iy < H && ix >= 0 && ix < W)
            v = x_nchw ? __ldg(x + (((int64_t)n * C + ci) * H + iy) * W + ix)
                       : __ldg(x + (((int64_t)n * H + iy) * W + ix) * C + ci);
          const int kidx = (ch * KH + ky) * KW + kx;
#pragma unroll
          for (int i = 0; i < MB; ++i)
            if (m0 + i < M) acc[i] = __fmaf_rn(__ldg(w + (int64_t)(m0 + i) * cg * KH * KW + kidx), v, acc[i]);
        }
      }
    }
    const int64_t obase = (((int64_t)n * OH + oy) * OW + ox) * M;
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      const int m = m0 + i;
      if (m >= M) break;
      float o = acc[i];
      if (bias) {
        const int mo = m % mg;
        if (!(mo >= m4 && ox >= full_cols)) o = __fadd_rn(o, __ldg(bias + m));
      }
      o = apply_act(o, act);
      if (residual) o = __fadd_rn(o, __ldg(residual + obase + m));
      y[obase + m] = o;
    }
  }
}

// Small-C dense conv (stems: C <= 4): one thread per output pixel computes
// all M channels; weights live in shared memory as [k][M] so every thread
// reads the same word (broadcast).  Same per-element chain as above; for
// M % 4 == 0 there are no bias-seeded tail rows.
template <int M>
__global__ void __launch_bounds__(256) conv_small_c_kernel(
    const float* __restrict__ x, int x_nchw, const float* __restrict__ w,
    const float* __restrict__ bias, const float* __restrict__ residual, float* __restrict__ y,
    int N, int C, int H, int W, int OH, int OW, int KH, int KW, int SH, int SW, int PH, int PW,
    ActParams act) {
  extern __shared__ float wsm[];
  const int K = C * KH * KW;
  for (int i = threadIdx.x; i < K * M; i += blockDim.x) {
    const int k = i / M, m = i % M;
    wsm[i] = w[m * K + k];
  }
  __syncthreads();
  const int64_t total = (int64_t)N * OH * OW;
  GRID_LOOP(t, total) {
    const int ox = (int)(t % OW);
    int64_t r = t / OW;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) acc[i] = 0.f;
    int k = 0;
    for (int ch = 0; ch < C; ++ch)
      for (int ky = 0; ky < KH; ++ky) {
        const int iy = oy * SH - PH + ky;
        for (int kx = 0; kx < KW; ++kx, ++k) {
          const int ix = ox * SW - PW + kx;
          float v = 0.f;
          if (iy >= 0 && iy < H && ix >= 0 && ix < W)
            v = x_nchw ? __ldg(x + (((int64_t)n * C + ch) * H + iy) * W + ix)
                       : __ldg(x + (((int64_t)n * H + iy) * W + ix) * C + ch);
          const float* wk = wsm + k * M;
#pragma unroll
          for (int i = 0; i < M; ++i) acc[i] = __fmaf_rn(wk[i], v, acc[i]);
        }
      }
    float* yo = y + t * M;
    const float* ro = residual ? residual + t * M : nullptr;
#pragma unroll
    for (int i = 0; i < M; i += 4) {
      float4 o;
      float* op = reinterpret_cast<float*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = acc[i + j];
        if (bias) v = __fadd_rn(v, __ldg(bias + i + j));
        v = apply_act(v, act);
        if (ro) v = __fadd_rn(v, __ldg(ro + i + j));
        op[j] = v;
      }
      *reinterpret_cast<float4*>(yo + i) = o;
    }
  }
}

// Stem specialisation (C = 3, 3x3, stride 2, NCHW input, NHWC output).  A
// persistent block walks 8 x 64 output tiles.  Each tile's input window
// (3 planes x 17 rows x 129 columns, its first column rounded down to a
// 16-byte boundary, hence 132) arrives by one 4-D TMA load (zeros outside
// the image = the zero padding) into one of two shared-memory buffers, the
// next tile's load overlapping this tile's arithmetic.  Thread (row tr, lane
// tc) makes pixels tc and tc + 32 of its row: each broadcast weight read
// feeds 2 FMAs and a warp writes 32 consecutive pixels.  Per element the
// chain is the generic kernel's: acc = 0, fma over k = (ch, ky, kx)
// ascending, then + bias, act, + residual.
constexpr int STEM_TH = 8, STEM_TW = 64, STEM_IR = 2 * STEM_TH + 1, STEM_IC = 132;
constexpr int STEM_BOX_BYTES = 3 * STEM_IR * STEM_IC * 4;           // 26,928 bytes per load
constexpr int STEM_BUF = ((STEM_BOX_BYTES + 1023) / 1024) * 1024;   // buffer stride, 1024-aligned

// Filter and bias by value in the kernel parameters: the unrolled FMA chain
// reads them as constant-bank operands (no shared-memory weight loads).
template <int M>
struct StemConsts {
  float w[27][M];  // [(ch * 3 + ky) * 3 + kx][m]
  float b[M];      // zeros when the conv has no bias
};

template <int M>
__global__ void __launch_bounds__(256) conv_stem3s2_kernel(
    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ StemConsts<M> sc, int has_bias,
    const float* __restrict__ residual, float* __restrict__ y, int N, int OH, int OW, int PH, int PW,
    ActParams act, unsigned int* err) {
  extern __shared__ __align__(1024) uint8_t stem_raw[];
  float* xs0 = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(stem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[2];
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmX);
  }
  __syncthreads();
  const int tiles_x = (OW + STEM_TW - 1) / STEM_TW, tiles_y = (OH + STEM_TH - 1) / STEM_TH;
  const int total = N * tiles_y * tiles_x;
  auto coords = [&](int tile, int& n, int& oy0, int& ox0) {
    const int bx = tile % tiles_x;
    const int r = tile / tiles_x;
    oy0 = (r % tiles_y) * STEM_TH;
    n = r / tiles_y;
    ox0 = bx * STEM_TW;
  };
  auto issue = [&](int tile, int buf) {
    int n, oy0, ox0;
    coords(tile, n, oy0, ox0);
    const int ix0 = 2 * ox0 - PW;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&full[buf], STEM_BOX_BYTES);
    tma_load_4d(reinterpret_cast<uint8_t*>(xs0) + buf * STEM_BUF, &tmX, &full[buf], ix0 & ~3, 2 * oy0 - PH, 0, n);
  };
  if (tid == 0 && (int)blockIdx.x < total) issue(blockIdx.x, 0);
  const int tr = tid >> 5, tc = tid & 31;
  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
    const int buf = it & 1;
    if (tid == 0 && tile + (int)gridDim.x < total) issue(tile + gridDim.x, buf ^ 1);
    int n, oy0, ox0;
    coords(tile, n, oy0, ox0);
    const int d = (2 * ox0 - PW) - ((2 * ox0 - PW) & ~3);  // column offset of the window in the box
    const bool ok = mbar_wait(&full[buf], (it >> 1) & 1u, err);
    if (ok) {
      const float* xs = xs0 + buf * (STEM_BUF / 4);
      float a0[M], a1[M];
#pragma unroll
      for (int i = 0; i < M; ++i) a0[i] = a1[i] = 0.f;
#pragma unroll
      for (int ch = 0; ch < 3; ++ch)
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const int k = (ch * 3 + ky) * 3 + kx;
            const float* row = xs + (ch * STEM_IR + 2 * tr + ky) * STEM_IC + d + kx;
            const float v0 = row[2 * tc], v1 = row[2 * tc + 64];
#pragma unroll
            for (int i = 0; i < M; ++i) {
              a0[i] = __fmaf_rn(sc.w[k][i], v0, a0[i]);
              a1[i] = __fmaf_rn(sc.w[k][i], v1, a1[i]);
            }
          }
      const int oy = oy0 + tr;
#pragma unroll
      for (int px = 0; px < 2; ++px) {
        const int ox = ox0 + tc + 32 * px;
        if (oy >= OH || ox >= OW) continue;
        const int64_t t = ((int64_t)n * OH + oy) * OW + ox;
        float o[M];
#pragma unroll
        for (int i = 0; i < M; ++i) o[i] = px ? a1[i] : a0[i];
        if (has_bias)
#pragma unroll
          for (int i = 0; i < M; ++i) o[i] = __fadd_rn(o[i], sc.b[i]);
        apply_act_n(o, act);
        if (residual)
#pragma unroll
          for (int i = 0; i < M; ++i) o[i] = __fadd_rn(o[i], __ldg(residual + t * M + i));
        float4* yo = reinterpret_cast<float4*>(y + t * M);
#pragma unroll
        for (int i4 = 0; i4 < M / 4; ++i4)
          yo[i4] = make_float4(o[4 * i4], o[4 * i4 + 1], o[4 * i4 + 2], o[4 * i4 + 3]);
      }
    }
    // buffer `buf` is refilled by the issue at the top of the next iteration;
    // a timed-out wait anywhere stops the whole block, after its loads land
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        mbar_wait(&full[buf], (it >> 1) & 1u, nullptr);
        if (tile + (int)gridDim.x < total) mbar_wait(&full[buf ^ 1], ((it + 1) >> 1) & 1u, nullptr);
      }
      __syncthreads();
      break;
    }
  }
}

cudaError_t launch_conv_direct(const float* x, int x_nchw, const float* w, const float* bias,
                               const float* residual, float* y, const ConvGeom& g, int group,
                               const ActParams& act, cudaStream_t st, unsigned int* err, const float* w_host,
                               const float* bias_host) {
  const int mg = g.m / group;
  const int64_t pix = (int64_t)g.n * g.oh * g.ow;
  if (group == 1 && x_nchw && err && w_host && (!bias || bias_host) && g.c == 3 && g.kh == 3 && g.kw == 3 &&
      g.sh == 2 && g.sw == 2 &&
      (g.m == 8 || g.m == 16 || g.m == 32) && (g.w % 4) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    CUtensorMap map;
    const uint64_t dims[4] = {(uint64_t)g.w, (uint64_t)g.h, 3, (uint64_t)g.n};
    const uint64_t strides[3] = {(uint64_t)g.w * 4, (uint64_t)g.w * g.h * 4, (uint64_t)g.w * g.h * 3 * 4};
    const uint32_t box[4] = {STEM_IC, STEM_IR, 3, 1};
    if (make_tensor_map(&map, x, 4, dims, strides, box, false)) {
      const int smem = 2 * STEM_BUF + 1024;
      const int64_t tiles = (int64_t)g.n * ((g.oh + STEM_TH - 1) / STEM_TH) * ((g.ow + STEM_TW - 1) / STEM_TW);
#define QPC_STEM(M_)                                                                                    \
  if (g.m == M_) {                                                                                      \
    StemConsts<M_> sc;                                                                                  \
    for (int k = 0; k < 27; ++k)                                                                        \
      for (int m = 0; m < M_; ++m) sc.w[k][m] = w_host[m * 27 + k];                                     \
    for (int m = 0; m < M_; ++m) sc.b[m] = bias ? bias_host[m] : 0.0f;                                  \
    auto kern = conv_stem3s2_kernel<M_>;                                                                \
    if (cudaError_t ae = ensure_dyn_smem((const void*)kern, smem); ae != cudaSuccess) return ae;        \
    const int per_sm = blocks_per_sm((const void*)kern, 256, smem);                                     \
    const int64_t cap = (int64_t)current_sm_count() * per_sm;                                           \
    kern<<<(int)(tiles < cap ? tiles : cap), 256, smem, st>>>(map, sc, bias ? 1 : 0, residual, y, g.n,  \
                                                              g.oh, g.ow, g.ph, g.pw, act, err);        \
    return cudaGetLastError();                                                                          \
  }
      QPC_STEM(8)
      QPC_STEM(16)
      QPC_STEM(32)
#undef QPC_STEM
    }
  }
  if (group == 1 && g.c <= 4 && (g.m == 8 || g.m == 16 || g.m == 32)) {
    const size_t smem = (size_t)g.c * g.kh * g.kw * g.m * sizeof(float);
#define QPC_SMALLC(M_)                                                                            \
  if (g.m == M_) {                                                                                \
    conv_small_c_kernel<M_><<<grid_for(pix), 256, smem, st>>>(x, x_nchw, w, bias, residual, y,    \
                                                             g.n, g.c, g.h, g.w, g.oh, g.ow,      \
                                                             g.kh, g.kw, g.sh, g.sw, g.ph, g.pw,  \
                                                             act);                                \
    return cudaGetLastError();                                                                    \
  }
    QPC_SMALLC(8)
    QPC_SMALLC(16)
    QPC_SMALLC(32)
#undef QPC_SMALLC
  }
  if (group == 1 || mg % 8 == 0) {
    const int mblocks = (g.m + 7) / 8;
    conv_direct_kernel<8><<<grid_for(pix * mblocks), 256, 0, st>>>(
        x, x_nchw, w, bias, residual, y, g.n, g.c, g.h, g.w, g.m, g.oh, g.ow, g.kh, g.kw, g.sh,
        g.sw, g.ph, g.pw, group, act);
  } else {
    conv_direct_kernel<1><<<grid_for(pix * g.m), 256, 0, st>>>(
        x, x_nchw, w, bias, residual, y, g.n, g.c, g.h, g.w, g.m, g.oh, g.ow, g.kh, g.kw, g.sh,
        g.sw, g.ph, g.pw, group, act);
  }
  return cudaGetLastError();
}

// --------------------------------------------------- ConvTranspose 2x2 s2
// conv.rs:730-838: each output pixel is one tap of one input pixel; the sum
// over input channels is a c-ascending fma chain from 0.  The following
// BatchNormalization (shape.rs:700-733: y = fma(x, a, b)) and activation are
// fused when present.  wt: [C][M][2][2] (ONNX ConvTranspose layout).
__global__ void __launch_bounds__(256) convt2x2_kernel(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bn_a,
    const float* __restrict__ bn_b, float* __restrict__ y, int N, int H, int W, int C, int M,
    ActParams act) {
  const int OH = 2 * H, OW = 2 * W;
  const int64_t total = (int64_t)N * OH * OW * M;
  GRID_LOOP(t, total) {
    const int co = (int)(t % M);
    int64_t r = t / M;
    const int ox = (int)(r % OW);
    r /= OW;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    const int ky = oy & 1, kx = ox & 1;
    const float* xp = x + (((int64_t)n * H + (oy >> 1)) * W + (ox >> 1)) * C;
    float acc = 0.f;
    for (int ch = 0; ch < C; ++ch)
      acc = __fmaf_rn(__ldg(xp + ch), __ldg(wt + ((ch * M + co) * 4) + ky * 2 + kx), acc);
    if (bn_a) acc = __fmaf_rn(acc, __ldg(bn_a + co), __ldg(bn_b + co));
    y[t] = apply_act(acc, act);
  }
}

// Same arithmetic, one thread per INPUT pixel: its C channels are read once
// and all 4 taps x M outputs are produced (each a c-ascending chain from 0).
template <int C, int M>
__global__ void __launch_bounds__(256) convt2x2_pix_kernel(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bn_a,
    const float* __restrict__ bn_b, float* __restrict__ y, int N, int H, int W, ActParams act) {
  __shared__ float wsm[C * M * 4];
  for (int i = threadIdx.x; i < C * M * 4; i += blockDim.x) wsm[i] = wt[i];
  __syncthreads();
  const int OW = 2 * W;
  const int64_t total = (int64_t)N * H * W;
  GRID_LOOP(p, total) {
    const int ix = (int)(p % W);
    int64_t r = p / W;
    const int iy = (int)(r % H);
    const int n = (int)(r / H);
    float xv[C];
    const float4* xp = reinterpret_cast<const float4*>(x + p * C);
#pragma unroll
    for (int c4 = 0; c4 < C / 4; ++c4) {
      const float4 v = __ldg(xp + c4);
      xv[4 * c4] = v.x;
      xv[4 * c4 + 1] = v.y;
      xv[4 * c4 + 2] = v.z;
      xv[4 * c4 + 3] = v.w;
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int oy = 2 * iy + (t >> 1), ox = 2 * ix + (t & 1);
      float* yo = y + (((int64_t)n * 2 * H + oy) * OW + ox) * M;
      float out[M];
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float acc = 0.f;
#pragma unroll
        for (int ch = 0; ch < C; ++ch) acc = __fmaf_rn(xv[ch], wsm[(ch * M + m) * 4 + t], acc);
        if (bn_a) acc = __fmaf_rn(acc, __ldg(bn_a + m), __ldg(bn_b + m));
        out[m] = apply_act(acc, act);
      }
      if (M % 4 == 0) {
#pragma unroll
        for (int m = 0; m < M; m += 4)
          *reinterpret_cast<float4*>(yo + m) = make_float4(out[m], out[m + 1], out[m + 2], out[m + 3]);
      } else {
#pragma unroll
        for (int m = 0; m < M; ++m) yo[m] = out[m];
      }
    }
  }
}

// Same arithmetic again, organised for wide outputs (M % 4 == 0): thread j of
// a pixel slot owns tap t = j / (M/4) and output channels 4*(j % (M/4)) ..+3,
// and keeps those C x 4 weights in registers.  A block stages PIX input pixels
// in shared memory (coalesced float4 loads) and its SLOTS pixel slots walk
// them; per pixel a thread reads the C inputs as broadcast float4s and makes
// 4 outputs (each the c-ascending chain from 0, then BN fma, then act).  The
// M threads of one pixel write its 4 output pixels as 2 runs of 2*M floats.
template <int C, int M, int SLOTS, int PIX>
__global__ void __launch_bounds__(SLOTS * M) convt2x2_wide_kernel(
    const float* __restrict__ x, const float* __restrict__ wt, const float* __restrict__ bn_a,
    const float* __restrict__ bn_b, float* __restrict__ y, int N, int H, int W, ActParams act) {
  static_assert(C % 4 == 0 && M % 4 == 0, "vector widths");
  constexpr int G = M / 4;  // float4 groups per tap
  __shared__ __align__(16) float xs[PIX * C];
  const int j = threadIdx.x % M, slot = threadIdx.x / M;
  const int t = j / G, m0 = 4 * (j % G);
  float w[C][4];
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) w[c][i] = __ldg(wt + (c * M + m0 + i) * 4 + t);
  float4 ba = make_float4(1.f, 1.f, 1.f, 1.f), bb = make_float4(0.f, 0.f, 0.f, 0.f);
  if (bn_a) {
    ba = __ldg(reinterpret_cast<const float4*>(bn_a + m0));
    bb = __ldg(reinterpret_cast<const float4*>(bn_b + m0));
  }
  const int OW = 2 * W;
  const int64_t total = (int64_t)N * H * W;
  for (int64_t p0 = (int64_t)blockIdx.x * PIX; p0 < total; p0 += (int64_t)gridDim.x * PIX) {
    const int np = (int)(total - p0 < PIX ? total - p0 : PIX);
    __syncthreads();  // previous chunk fully consumed
    const float4* src = reinterpret_cast<const float4*>(x + p0 * C);
    for (int i = threadIdx.x; i < np * (C / 4); i += SLOTS * M)
      reinterpret_cast<float4*>(xs)[i] = __ldg(src + i);
    __syncthreads();
    for (int k = slot; k < np; k += SLOTS) {
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      const float4* xp = reinterpret_cast<const float4*>(xs + k * C);
#pragma unroll
      for (int c4 = 0; c4 < C / 4; ++c4) {
        const float4 v = xp[c4];
        const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = 4 * c4 + q;
          a0 = __fmaf_rn(xv[q], w[c][0], a0);
          a1 = __fmaf_rn(xv[q], w[c][1], a1);
          a2 = __fmaf_rn(xv[q], w[c][2], a2);
          a3 = __fmaf_rn(xv[q], w[c][3], a3);
        }
      }
      if (bn_a) {
        a0 = __fmaf_rn(a0, ba.x, bb.x);
        a1 = __fmaf_rn(a1, ba.y, bb.y);
        a2 = __fmaf_rn(a2, ba.z, bb.z);
        a3 = __fmaf_rn(a3, ba.w, bb.w);
      }
      float o[4] = {a0, a1, a2, a3};
      apply_act_n(o, act);
      const int64_t p = p0 + k;
      const int ix = (int)(p % W);
      const int64_t r = p / W;
      const int iy = (int)(r % H);
      const int n = (int)(r / H);
      const int oy = 2 * iy + (t >> 1), ox = 2 * ix + (t & 1);
      *reinterpret_cast<float4*>(y + (((int64_t)n * 2 * H + oy) * OW + ox) * M + m0) =
          make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

// The same arithmetic with the input chunks arriving by TMA (the input as a
// [pixels, C] matrix, PIX rows per load) into a 2-stage shared-memory ring,
// so the next chunk's load overlaps this chunk's FMAs, and two pixels per
// iteration for more independent chains.  Waits are bounded (error word).
template <int C, int M, int SLOTS, int PIX>
__global__ void __launch_bounds__(SLOTS * M) convt2x2_tma_kernel(
    const __grid_constant__ CUtensorMap tmX, const float* __restrict__ wt, const float* __restrict__ bn_a,
    const float* __restrict__ bn_b, float* __restrict__ y, int N, int H, int W, ActParams act,
    unsigned int* err) {
  static_assert(C % 4 == 0 && M % 4 == 0 && (PIX * C * 4) % 1024 == 0, "vector widths / buffer alignment");
  constexpr int G = M / 4;  // float4 groups per tap
  constexpr uint32_t BYTES = PIX * C * 4;
  extern __shared__ __align__(1024) uint8_t ct_raw[];
  float* xs0 = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ct_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[2];
  const int tid = threadIdx.x;
  const int j = tid % M, slot = tid / M;
  const int t = j / G, m0 = 4 * (j % G);
  float w[C][4];
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) w[c][i] = __ldg(wt + (c * M + m0 + i) * 4 + t);
  float4 ba = make_float4(1.f, 1.f, 1.f, 1.f), bb = make_float4(0.f, 0.f, 0.f, 0.f);
  if (bn_a) {
    ba = __ldg(reinterpret_cast<const float4*>(bn_a + m0));
    bb = __ldg(reinterpret_cast<const float4*>(bn_b + m0));
  }
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmX);
  }
  __syncthreads();
  const int OW = 2 * W;
  const int64_t total = (int64_t)N * H * W;
  const int chunks = (int)((total + PIX - 1) / PIX);
  auto issue = [&](int chunk, int buf) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&full[buf], BYTES);
    tma_load_2d(reinterpret_cast<uint8_t*>(xs0) + buf * BYTES, &tmX, &full[buf], 0, chunk * PIX);
  };
  if (tid == 0 && (int)blockIdx.x < chunks) issue(blockIdx.x, 0);
  uint32_t it = 0;
  for (int chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x, ++it) {
    const int buf = it & 1;
    if (tid == 0 && chunk + (int)gridDim.x < chunks) issue(chunk + gridDim.x, buf ^ 1);
    const bool ok = mbar_wait(&full[buf], (it >> 1) & 1u, err);
    if (ok) {
      const float* xs = xs0 + buf * (PIX * C);
      const int64_t p0 = (int64_t)chunk * PIX;
      const int np = (int)(total - p0 < PIX ? total - p0 : PIX);
      // slot `slot` takes the contiguous run [slot * RUN, slot * RUN + RUN) of
      // the chunk, two adjacent pixels per step; its coordinates are found
      // once per run and then stepped
      constexpr int RUN = PIX / SLOTS;
      const int kb = slot * RUN;
      const uint32_t pp = (uint32_t)(p0 + kb);
      const uint32_t rr = pp / (uint32_t)W;
      int ix = (int)(pp - rr * (uint32_t)W);
      const uint32_t nn = rr / (uint32_t)H;
      int iy = (int)(rr - nn * (uint32_t)H);
      int n = (int)nn;
      for (int k = kb; k < kb + RUN && k < np; k += 2) {
        const bool two = k + 1 < np;
        float a[2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < 4; ++i) a[u][i] = 0.f;
        const float4* xp0 = reinterpret_cast<const float4*>(xs + k * C);
        const float4* xp1 = reinterpret_cast<const float4*>(xs + (two ? k + 1 : k) * C);
#pragma unroll
        for (int c4 = 0; c4 < C / 4; ++c4) {
          const float4 v0 = xp0[c4], v1 = xp1[c4];
          const float x0[4] = {v0.x, v0.y, v0.z, v0.w}, x1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int c = 4 * c4 + qq;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              a[0][i] = __fmaf_rn(x0[qq], w[c][i], a[0][i]);
              a[1][i] = __fmaf_rn(x1[qq], w[c][i], a[1][i]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          if (u == 1 && !two) break;
          float o[4] = {a[u][0], a[u][1], a[u][2], a[u][3]};
          if (bn_a) {
            o[0] = __fmaf_rn(o[0], ba.x, bb.x);
            o[1] = __fmaf_rn(o[1], ba.y, bb.y);
            o[2] = __fmaf_rn(o[2], ba.z, bb.z);
            o[3] = __fmaf_rn(o[3], ba.w, bb.w);
          }
          apply_act_n(o, act);
          const int oy = 2 * iy + (t >> 1), ox = 2 * ix + (t & 1);
          *reinterpret_cast<float4*>(y + (((int64_t)n * 2 * H + oy) * OW + ox) * M + m0) =
              make_float4(o[0], o[1], o[2], o[3]);
          // next input pixel
          if (++ix == W) {
            ix = 0;
            if (++iy == H) {
              iy = 0;
              ++n;
            }
          }
        }
      }
    }
    // buffer `buf` is refilled by the issue at the top of the next iteration;
    // a timed-out wait stops the whole block after its loads have landed
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        mbar_wait(&full[buf], (it >> 1) & 1u, nullptr);
        if (chunk + (int)gridDim.x < chunks) mbar_wait(&full[buf ^ 1], ((it + 1) >> 1) & 1u, nullptr);
      }
      __syncthreads();
      break;
    }
  }
}

cudaError_t launch_convt2x2(const float* x, const float* wt, const float* bn_a, const float* bn_b,
                            float* y, int n, int h, int w, int c, int m, const ActParams& act,
                            cudaStream_t st, unsigned int* err) {
  if (c == 24 && m == 24 && err && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0 && (!bn_a || (reinterpret_cast<uintptr_t>(bn_a) & 15) == 0) &&
      (!bn_b || (reinterpret_cast<uintptr_t>(bn_b) & 15) == 0)) {
    constexpr int SLOTS = 8, PIX = 256;
    CUtensorMap map;
    const int64_t pixels = (int64_t)n * h * w;
    const uint64_t dims[2] = {24, (uint64_t)pixels};
    const uint64_t strides[1] = {24 * 4};
    const uint32_t box[2] = {24, PIX};
    if (make_tensor_map(&map, x, 2, dims, strides, box, false)) {
      auto kern = convt2x2_tma_kernel<24, 24, SLOTS, PIX>;
      const int smem = 2 * PIX * 24 * 4 + 1024;
      if (cudaError_t ae = ensure_dyn_smem((const void*)kern, smem); ae != cudaSuccess) return ae;
      const int per_sm = blocks_per_sm((const void*)kern, SLOTS * 24, smem);
      const int64_t chunks = (pixels + PIX - 1) / PIX;
      const int64_t cap = (int64_t)current_sm_count() * per_sm;
      kern<<<(int)(chunks < cap ? chunks : cap), SLOTS * 24, smem, st>>>(map, wt, bn_a, bn_b, y, n, h, w, act,
                                                                         err);
      return cudaGetLastError();
    }
  }
  if (c == 24 && m == 24) {
    constexpr int SLOTS = 8, PIX = 256;
    const int64_t chunks = ((int64_t)n * h * w + PIX - 1) / PIX;
    const int grid = (int)(chunks < 148 * 8 ? chunks : 148 * 8);
    convt2x2_wide_kernel<24, 24, SLOTS, PIX><<<grid > 0 ? grid : 1, SLOTS * 24, 0, st>>>(
        x, wt, bn_a, bn_b, y, n, h, w, act);
    return cudaGetLastError();
  }
  if (c == 24 && m == 1) {
    convt2x2_pix_kernel<24, 1><<<grid_for((int64_t)n * h * w, 256), 256, 0, st>>>(x, wt, bn_a, bn_b, y, n, h, w, act);
    return cudaGetLastError();
  }
  convt2x2_kernel<<<grid_for((int64_t)n * 4 * h * w * m), 256, 0, st>>>(x, wt, bn_a, bn_b, y, n, h,
                                                                         w, c, m, act);
  return cudaGetLastError();
}

// ------------------------------------------------------------ pooling
// pool2d.rs:10-30 global_avg_pool (f64 sum / plane) on NHWC.  A block owns
// (n, 32 channels); its 8 warps sum strided slices of the plane in f64 and the
// 8 partial f64 sums are added in a fixed order.  f64 partial sums of f32
// values are exact far beyond the f32 result's precision, so the rounded mean
// equals the sequential sum's except at ties ~1e-16 apart.
__global__ void __launch_bounds__(256) gap_nhwc_kernel(const float* __restrict__ x,
                                                       float* __restrict__ y, int N, int HW, int C) {
  __shared__ double part[8][32];
  const int cblocks = (C + 31) / 32;
  const int n = blockIdx.x / cblocks, c = (blockIdx.x % cblocks) * 32 + (threadIdx.x & 31);
  const int w = threadIdx.x >> 5;
  double s = 0.0;
  if (c < C) {
    const float* p = x + (int64_t)n * HW * C + c;
    for (int i = w; i < HW; i += 8) s += (double)__ldg(p + (int64_t)i * C);
  }
  part[w][threadIdx.x & 31] = s;
  __syncthreads();
  if (w == 0 && c < C) {
    double t = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k][threadIdx.x];
    y[(int64_t)n * C + c] = (float)(t / (double)HW);
  }
}

cudaError_t launch_gap_nhwc(const float* x, float* y, int n, int hw, int c, cudaStream_t st) {
  gap_nhwc_kernel<<<n * ((c + 31) / 32), 256, 0, st>>>(x, y, n, hw, c);
  return cudaGetLastError();
}

// pool2d.rs:51-260 (max / avg over the kernel window, avg divides by kh*kw).
__global__ void pool2d_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int N, int H,
                                   int W, int C, int OH, int OW, int KH, int KW, int SH, int SW,
                                   int PH, int PW, int is_max) {
  GRID_LOOP(t, (int64_t)N * OH * OW * C) {
    const int c = (int)(t % C);
    int64_t r = t / C;
    const int ox = (int)(r % OW);
    r /= OW;
    const int oy = (int)(r % OH);
    const int n = (int)(r / OH);
    float acc = is_max ? -INFINITY : 0.f;
    for (int ky = 0; ky < KH; ++ky)
      for (int kx = 0; kx < KW; ++kx) {
        const int iy = oy * SH - PH + ky, ix = ox * SW - PW + kx;
        if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
        const float v = __ldg(x + (((int64_t)n * H + iy) * W + ix) * C + c);
        if (is_max) acc = v > acc ? v : acc;
        else acc = __fadd_rn(acc, v);
      }
    y[t] = is_max ? acc : __fdiv_rn(acc, (float)(KH * KW));
  }
}

// C % 4 == 0 and fewer than 2^31 input elements: a thread makes 4 adjacent
// channels of one output pixel (float4 loads and stores, 32-bit index math),
// each channel with the generic kernel's operations in its order.
__global__ void __launch_bounds__(256) pool2d_nhwc4_kernel(const float4* __restrict__ x, float4* __restrict__ y,
                                                           int N, int H, int W, int C4, int OH, int OW, int KH,
                                                           int KW, int SH, int SW, int PH, int PW, int is_max) {
  const int total = N * OH * OW * C4;
  const float inv_n = (float)(KH * KW);
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
    const int c4 = t % C4;
    int r = t / C4;
    const int ox = r % OW;
    r /= OW;
    const int oy = r % OH;
    const int n = r / OH;
    float4 acc = is_max ? make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ky = 0; ky < KH; ++ky) {
      const int iy = oy * SH - PH + ky;
      if (iy < 0 || iy >= H) continue;
      for (int kx = 0; kx < KW; ++kx) {
        const int ix = ox * SW - PW + kx;
        if (ix < 0 || ix >= W) continue;
        const float4 v = __ldg(x + ((n * H + iy) * W + ix) * C4 + c4);
        if (is_max) {
          acc.x = v.x > acc.x ? v.x : acc.x;
          acc.y = v.y > acc.y ? v.y : acc.y;
          acc.z = v.z > acc.z ? v.z : acc.z;
          acc.w = v.w > acc.w ? v.w : acc.w;
        } else {
          acc.x = __fadd_rn(acc.x, v.x);
          acc.y = __fadd_rn(acc.y, v.y);
          acc.z = __fadd_rn(acc.z, v.z);
          acc.w = __fadd_rn(acc.w, v.w);
        }
      }
    }
    if (!is_max)
      acc = make_float4(__fdiv_rn(acc.x, inv_n), __fdiv_rn(acc.y, inv_n), __fdiv_rn(acc.z, inv_n),
                        __fdiv_rn(acc.w, inv_n));
    y[t] = acc;
  }
}

cudaError_t launch_pool2d_nhwc(const float* x, float* y, int n, int h, int w, int c, int oh, int ow,
                               int kh, int kw, int sh, int sw, int ph, int pw, int is_max,
                               cudaStream_t st) {
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if ((c & 3) == 0 && aligned && (int64_t)n * h * w * c < ((int64_t)1 << 31) &&
      (int64_t)n * oh * ow * c < ((int64_t)1 << 31)) {
    const int64_t total = (int64_t)n * oh * ow * (c / 4);
    pool2d_nhwc4_kernel<<<grid_for(total), 256, 0, st>>>(reinterpret_cast<const float4*>(x),
                                                         reinterpret_cast<float4*>(y), n, h, w, c / 4, oh, ow, kh,
                                                         kw, sh, sw, ph, pw, is_max);
    return cudaGetLastError();
  }
  pool2d_nhwc_kernel<<<grid_for((int64_t)n * oh * ow * c), 256, 0, st>>>(x, y, n, h, w, c, oh, ow, kh,
                                                                        kw, sh, sw, ph, pw, is_max);
  return cudaGetLastError();
}

// resize.rs:8-57 nearest: iy = min((int)((float)oy * H / oh), H - 1), the
// source index (int)((float)o * in / out) clamped (resize.rs:43-50), in
// 32-bit arithmetic.  Up to RESIZE_MAX_SRC sources of one output size are
// written in one launch, each into its channel slice [c_off, c_off + C) of an
// output with ldc channels: the FPN's upsampled maps land in their concat
// slices side by side, so each output pixel's slices are written together.
// Threads take one (ox, channel quad) column of the output (quads enumerated
// source after source), its source and source column found once; blockIdx.y
// takes RESIZE_ROWS consecutive output rows (n * OH + oy), whose loads are all
// issued before their stores so several are in flight per thread.
constexpr int RESIZE_ROWS = 8;
__global__ void __launch_bounds__(256) resize_nearest_nhwc_kernel(const ResizeSrcs s, float* __restrict__ y,
                                                                  int N, int OH, int OW, int ldc) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= OW * s.quads) return;
  const int ox = i / s.quads;
  int q = i - ox * s.quads, k = 0;
#pragma unroll
  for (int j = 0; j < RESIZE_MAX_SRC - 1; ++j)
    if (k + 1 < s.n && q >= s.c4[k]) {
      q -= s.c4[k];
      ++k;
    }
  const int H = s.h[k], W = s.w[k], C = 4 * s.c4[k];
  const float* __restrict__ x = s.x[k];
  int ix = (int)__fdiv_rn(__fmul_rn((float)ox, (float)W), (float)OW);
  ix = ix < W - 1 ? ix : W - 1;
  const int col = s.c_off[k] + 4 * q;
  const int rows = N * OH;
  for (int row0 = blockIdx.y * RESIZE_ROWS; row0 < rows; row0 += gridDim.y * RESIZE_ROWS) {
    float4 v[RESIZE_ROWS];
#pragma unroll
    for (int r = 0; r < RESIZE_ROWS; ++r) {
      const int row = row0 + r;
      if (row < rows) {
        const int n = row / OH, oy = row - n * OH;
        int iy = (int)__fdiv_rn(__fmul_rn((float)oy, (float)H), (float)OH);
        iy = iy < H - 1 ? iy : H - 1;
        v[r] = __ldg(reinterpret_cast<const float4*>(x + (((int64_t)n * H + iy) * W + ix) * C) + q);
      }
    }
    if (s.round_tf32)
#pragma unroll
      for (int r = 0; r < RESIZE_ROWS; ++r)
        v[r] = make_float4(tf32_rna(v[r].x), tf32_rna(v[r].y), tf32_rna(v[r].z), tf32_rna(v[r].w));
#pragma unroll
    for (int r = 0; r < RESIZE_ROWS; ++r) {
      const int row = row0 + r;
      if (row < rows) *reinterpret_cast<float4*>(y + ((int64_t)row * OW + ox) * ldc + col) = v[r];
    }
  }
}

cudaError_t launch_resize_nearest_multi_nhwc(const ResizeSrcs& s, float* y, int n, int oh, int ow, int ldc,
                                             cudaStream_t st) {
  if (s.n < 1 || s.n > RESIZE_MAX_SRC || (ldc & 3)) return cudaErrorInvalidValue;
  int quads = 0;
  for (int k = 0; k < s.n; ++k) {
    if (s.c4[k] <= 0 || (s.c_off[k] & 3) || s.c_off[k] + 4 * s.c4[k] > ldc || s.h[k] <= 0 || s.w[k] <= 0)
      return cudaErrorInvalidValue;
    quads += s.c4[k];
  }
  if (quads != s.quads) return cudaErrorInvalidValue;
  if ((int64_t)n * oh + RESIZE_ROWS >= (1LL << 31) || (int64_t)ow * quads >= (1LL << 31))
    return cudaErrorInvalidValue;
  if (n <= 0 || oh <= 0 || ow <= 0) return cudaSuccess;
  const int per_row = ow * quads;
  const int row_groups = (n * oh + RESIZE_ROWS - 1) / RESIZE_ROWS;
  dim3 grid((per_row + 255) / 256, row_groups < 65535 ? row_groups : 65535);
  resize_nearest_nhwc_kernel<<<grid, 256, 0, st>>>(s, y, n, oh, ow, ldc);
  return cudaGetLastError();
}

cudaError_t launch_resize_nearest_nhwc(const float* x, float* y, int n, int h, int w, int c, int oh,
                                       int ow, int ldc, int c_off, cudaStream_t st) {
  if ((c & 3) || (ldc & 3) || (c_off & 3)) return cudaErrorInvalidValue;
  if (n <= 0 || oh <= 0 || ow <= 0 || c <= 0) return cudaSuccess;
  ResizeSrcs s{};
  s.n = 1;
  s.x[0] = x;
  s.h[0] = h;
  s.w[0] = w;
  s.c4[0] = c / 4;
  s.c_off[0] = c_off;
  s.quads = c / 4;
  return launch_resize_nearest_multi_nhwc(s, y, n, oh, ow, ldc, st);
}

// ------------------------------------------------------------ elementwise
// elementwise.rs:185-420 broadcast binary op over a strided view.  The
// output is contiguous in `out_dims` order; a_str / b_str are element
// strides per output dim (0 where broadcast).  op: 0 add 1 sub 2 mul 3 div
// 4 pow.  `post` applies an activation to the result.
__global__ void binary_kernel(const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ y, StridedDims sd, int op, ActParams post) {
  GRID_LOOP(t, sd.total) {
    int64_t rem = t, ia = 0, ib = 0;
    for (int d = sd.rank - 1; d >= 0; --d) {
      const int64_t idx = rem % sd.dims[d];
      rem /= sd.dims[d];
      ia += idx * sd.sa[d];
      ib += idx * sd.sb[d];
    }
    const float va = __ldg(a + ia), vb = __ldg(b + ib);
    float r;
    switch (op) {
      case 0: r = __fadd_rn(va, vb); break;
      case 1: r = __fsub_rn(va, vb); break;
      case 2: r = __fmul_rn(va, vb); break;
      case 3: r = __fdiv_rn(va, vb); break;
      default: r = (vb == 2.0f) ? __fmul_rn(va, va) : powf(va, vb); break;
    }
    y[t] = apply_act(r, post);
  }
}

cudaError_t launch_binary(const float* a, const float* b, float* y, const StridedDims& sd, int op,
                          const ActParams& post, cudaStream_t st) {
  binary_kernel<<<grid_for(sd.total), 256, 0, st>>>(a, b, y, sd, op, post);
  return cudaGetLastError();
}

// Unary ops on a strided view (sa = input strides): activation kinds plus
// sqrt (kind 100), clip (kind 101, lo = alpha, hi = beta) and erf (kind 102).
__global__ void unary_kernel(const float* __restrict__ a, float* __restrict__ y, StridedDims sd,
                             ActParams act) {
  GRID_LOOP(t, sd.total) {
    int64_t rem = t, ia = 0;
    for (int d = sd.rank - 1; d >= 0; --d) {
      const int64_t idx = rem % sd.dims[d];
      rem /= sd.dims[d];
      ia += idx * sd.sa[d];
    }
    const float v = __ldg(a + ia);
    float r;
    if (act.kind == 100) r = __fsqrt_rn(v);
    else if (act.kind == 102) r = erf1(v);
    else if (act.kind == 101) {
      const float m = v < act.alpha ? act.alpha : v;
      r = act.beta < m ? act.beta : m;
    } else r = apply_act(v, act);
    y[t] = r;
  }
}

cudaError_t launch_unary(const float* a, float* y, const StridedDims& sd, const ActParams& act,
                         cudaStream_t st) {
  unary_kernel<<<grid_for(sd.total), 256, 0, st>>>(a, y, sd, act);
  return cudaGetLastError();
}

// elementwise.rs:134-165 mul_add_scale on NHWC with a per-channel gate:
// out = f * g[n, c] + r  (two roundings).  gate_per_n: gate is [N, C].
__global__ void mul_add_scale_nhwc_kernel(const float* __restrict__ f, const float* __restrict__ g,
                                          const float* __restrict__ r, float* __restrict__ y,
                                          int64_t total, int HW, int C, int gate_per_n) {
  GRID_LOOP(t, total) {
    const int c = (int)(t % C);
    const int64_t n = t / ((int64_t)HW * C);
    const float gv = __ldg(g + (gate_per_n ? n * C : 0) + c);
    y[t] = __fadd_rn(__fmul_rn(__ldg(f + t), gv), r ? __ldg(r + t) : 0.0f);
  }
}

cudaError_t launch_mul_add_scale_nhwc(const float* f, const float* g, const float* r, float* y,
                                      int64_t total, int hw, int c, int gate_per_n, cudaStream_t st) {
  mul_add_scale_nhwc_kernel<<<grid_for(total), 256, 0, st>>>(f, g, r, y, total, hw, c, gate_per_n);
  return cudaGetLastError();
}

// Strided view -> contiguous copy (Transpose / Slice / Reshape materialise),
// optionally into a channel slice of a wider buffer (out row = ldo, c_off).
__global__ void copy_strided_kernel(const float* __restrict__ a, float* __restrict__ y,
                                    StridedDims sd) {
  GRID_LOOP(t, sd.total) {
    int64_t rem = t, ia = 0;
    for (int d = sd.rank - 1; d >= 0; --d) {
      const int64_t idx = rem % sd.dims[d];
      rem /= sd.dims[d];
      ia += idx * sd.sa[d];
    }
    y[t] = __ldg(a + ia);
  }
}

cudaError_t launch_copy_strided(const float* a, float* y, const StridedDims& sd, cudaStream_t st) {
  copy_strided_kernel<<<grid_for(sd.total), 256, 0, st>>>(a, y, sd);
  return cudaGetLastError();
}

// Channel-slice copy for Concat(axis=1) on NHWC: y[p, c_off + c] = x[p, c].
__global__ void copy_channels_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t pix,
                                     int C, int ldc, int c_off) {
  GRID_LOOP(t, pix * C) {
    const int c = (int)(t % C);
    const int64_t p = t / C;
    y[p * ldc + c_off + c] = __ldg(x + t);
  }
}

__global__ void copy_channels4_kernel(const float4* __restrict__ x, float* __restrict__ y, int64_t pix,
                                      int C4, int ldc, int c_off) {
  GRID_LOOP(t, pix * C4) {
    const int c4 = (int)(t % C4);
    const int64_t p = t / C4;
    *reinterpret_cast<float4*>(y + p * ldc + c_off + 4 * c4) = __ldg(x + t);
  }
}

cudaError_t launch_copy_channels(const float* x, float* y, int64_t pix, int c, int ldc, int c_off,
                                 cudaStream_t st) {
  if ((c & 3) == 0 && (ldc & 3) == 0 && (c_off & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0) {
    copy_channels4_kernel<<<grid_for(pix * (c / 4)), 256, 0, st>>>(reinterpret_cast<const float4*>(x), y,
                                                                  pix, c / 4, ldc, c_off);
    return cudaGetLastError();
  }
  copy_channels_kernel<<<grid_for(pix * c), 256, 0, st>>>(x, y, pix, c, ldc, c_off);
  return cudaGetLastError();
}

// ------------------------------------------------------------ reductions
// shape.rs:510-566 reduce_mean over [outer, mid, inner] with f64 sums.
__global__ void reduce_mean_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t outer,
                                   int64_t mid, int64_t inner) {
  GRID_LOOP(t, outer * inner) {
    const int64_t o = t / inner, i = t % inner;
    const float* p = x + o * mid * inner + i;
    double s = 0.0;
    for (int64_t m = 0; m < mid; ++m) s += (double)__ldg(p + m * inner);
    y[t] = (float)(s / (double)mid);
  }
}

cudaError_t launch_reduce_mean(const float* x, float* y, int64_t outer, int64_t mid, int64_t inner,
                               cudaStream_t st) {
  reduce_mean_kernel<<<grid_for(outer * inner), 256, 0, st>>>(x, y, outer, mid, inner);
  return cudaGetLastError();
}

// activation.rs:321-403 softmax_last_dim on one row: 8-lane max, exp1(x -
// max), per-lane partial sums combined by the hsum8 tree, scalar tail,
// y = e * (1 / sum).  Bit-identical to the reference row kernel.  `row` and
// `out` may alias.
__device__ __forceinline__ void softmax_row(const float* row, float* out, int inner) {
  int i = 0;
  float mx;
  if (inner >= 8) {
    float vmax[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) vmax[j] = row[0];
    for (; i + 8 <= inner; i += 8)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = row[i + j];
        if (v > vmax[j]) vmax[j] = v;
      }
    mx = vmax[0];
#pragma unroll
    for (int j = 1; j < 8; ++j)
      if (vmax[j] > mx) mx = vmax[j];
  } else {
    i = 1;
    mx = row[0];
  }
  for (; i < inner; ++i)
    if (row[i] > mx) mx = row[i];
  float sum = 0.f;
  int i2 = 0;
  if (inner >= 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (; i2 + 8 <= inner; i2 += 8)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float e = exp1(__fsub_rn(row[i2 + j], mx));
        out[i2 + j] = e;
        acc[j] = __fadd_rn(acc[j], e);
      }
    const float t0 = __fadd_rn(acc[0], acc[4]), t1 = __fadd_rn(acc[1], acc[5]);
    const float t2 = __fadd_rn(acc[2], acc[6]), t3 = __fadd_rn(acc[3], acc[7]);
    sum = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
  }
  for (; i2 < inner; ++i2) {
    const float e = exp1(__fsub_rn(row[i2], mx));
    out[i2] = e;
    sum = __fadd_rn(sum, e);
  }
  const float inv = __fdiv_rn(1.0f, sum);
  for (int j = 0; j < inner; ++j) out[j] = __fmul_rn(out[j], inv);
}

// One thread per row.
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t rows,
                                    int inner) {
  GRID_LOOP(r, rows) softmax_row(x + r * inner, y + r * inner, inner);
}

cudaError_t launch_softmax_rows(const float* x, float* y, int64_t rows, int inner, cudaStream_t st) {
  softmax_rows_kernel<<<grid_for(rows, 128), 128, 0, st>>>(x, y, rows, inner);
  return cudaGetLastError();
}

// shape.rs:669-697 small batched matmul (attention): per output row, zeroed
// accumulators, then c[j] = fma(a[k], b[k][j], c[j]) for k ascending.  Fully
// strided operands (batch index decomposed as b0 * nb1 + b1).
__global__ void bmm_small_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                 float* __restrict__ c, BmmDims d) {
  const int64_t total = (int64_t)d.nb0 * d.nb1 * d.m * d.n;
  GRID_LOOP(t, total) {
    const int j = (int)(t % d.n);
    int64_t r = t / d.n;
    const int i = (int)(r % d.m);
    r /= d.m;
    const int b1 = (int)(r % d.nb1), b0 = (int)(r / d.nb1);
    const float* ap = a + b0 * d.sa0 + b1 * d.sa1 + (int64_t)i * d.sam;
    const float* bp = b + b0 * d.sb0 + b1 * d.sb1 + (int64_t)j * d.sbn;
    float acc = 0.f;
    for (int k = 0; k < d.k; ++k) acc = __fmaf_rn(__ldg(ap + (int64_t)k * d.sak), __ldg(bp + (int64_t)k * d.sbk), acc);
    c[t] = acc;
  }
}

cudaError_t launch_bmm_small(const float* a, const float* b, float* c, const BmmDims& d,
                             cudaStream_t st) {
  bmm_small_kernel<<<grid_for((int64_t)d.nb0 * d.nb1 * d.m * d.n), 256, 0, st>>>(a, b, c, d);
  return cudaGetLastError();
}

// n_exit3_argmax.comp / rec.rs:34-79: first strict maximum per row, ties to
// the lowest index; pairs[2r] = value, pairs[2r+1] = index bit pattern.
// One warp per row.
__global__ void argmax_pairs_kernel(const float* __restrict__ x, float* __restrict__ pairs,
                                    int64_t rows, int cols) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = x + row * cols;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = lane; c < cols; c += 32) {
    const float v = __ldg(p + c);
    if (v > bv) { bv = v; bi = c; }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) {
    pairs[2 * row] = bv;
    pairs[2 * row + 1] = __uint_as_float((unsigned)bi);
  }
}

cudaError_t launch_argmax_pairs(const float* x, float* pairs, int64_t rows, int cols,
                                cudaStream_t st) {
  const int64_t blocks = (rows + 7) / 8;
  argmax_pairs_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, pairs, rows, cols);
  return cudaGetLastError();
}

// BatchNormalization on NHWC (unfused fallback): y = fma(x, a[c], b[c]).
__global__ void affine_nhwc_kernel(const float* __restrict__ x, const float* __restrict__ a,
                                   const float* __restrict__ b, float* __restrict__ y,
                                   int64_t total, int C, ActParams act) {
  GRID_LOOP(t, total) {
    const int c = (int)(t % C);
    y[t] = apply_act(__fmaf_rn(__ldg(x + t), __ldg(a + c), __ldg(b + c)), act);
  }
}

cudaError_t launch_affine_nhwc(const float* x, const float* a, const float* b, float* y,
                               int64_t total, int c, const ActParams& act, cudaStream_t st) {
  affine_nhwc_kernel<<<grid_for(total), 256, 0, st>>>(x, a, b, y, total, c, act);
  return cudaGetLastError();
}

// Strided view -> strided view copy (sa = source strides, sb = destination
// strides, both in the same logical dim order).
__global__ void copy_view_kernel(const float* __restrict__ a, float* __restrict__ y, StridedDims sd) {
  GRID_LOOP(t, sd.total) {
    int64_t rem = t, ia = 0, ib = 0;
    for (int d = sd.rank - 1; d >= 0; --d) {
      const int64_t idx = rem % sd.dims[d];
      rem /= sd.dims[d];
      ia += idx * sd.sa[d];
      ib += idx * sd.sb[d];
    }
    y[ib] = __ldg(a + ia);
  }
}

cudaError_t launch_copy_view(const float* a, float* y, const StridedDims& sd, cudaStream_t st) {
  copy_view_kernel<<<grid_for(sd.total), 256, 0, st>>>(a, y, sd);
  return cudaGetLastError();
}

// LayerNorm over the last axis, fused from the reference's decomposed chain
// (executor ReduceMean -> Sub -> Pow 2 -> ReduceMean -> Add eps -> Sqrt ->
// Div -> Mul gamma -> Add beta; shape.rs:510-566 f64 means, elementwise.rs
// single roundings).  Per row, the two sums are sequential f64 sums in index
// order, so every intermediate equals the reference's.  `round` stores the
// result tf32-rounded (nearest, ties away), for a value read only as a TF32
// A operand.
__device__ __forceinline__ float layernorm_elem(float x, float mean, float sd, const float* __restrict__ gamma,
                                                const float* __restrict__ beta, int i, int round) {
  float v = __fdiv_rn(__fsub_rn(x, mean), sd);
  if (gamma) v = __fmul_rn(v, __ldg(gamma + i));
  if (beta) v = __fadd_rn(v, __ldg(beta + i));
  return round ? tf32_rna(v) : v;
}
__device__ __forceinline__ void layernorm_stats(const float* p, int C, float eps, float* mean_out, float* sd_out) {
  double s = 0.0;
  for (int i = 0; i < C; ++i) s += (double)p[i];
  const float mean = (float)(s / (double)C);
  double s2 = 0.0;
  for (int i = 0; i < C; ++i) {
    const float d = __fsub_rn(p[i], mean);
    s2 += (double)__fmul_rn(d, d);
  }
  const float var = (float)(s2 / (double)C);
  *mean_out = mean;
  *sd_out = __fsqrt_rn(__fadd_rn(var, eps));
}

// One thread per row (rows wider than the staged kernel takes).
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, float* __restrict__ y,
                                 int64_t rows, int C, float eps, int round) {
  GRID_LOOP(r, rows) {
    const float* p = x + r * C;
    float mean, sd;
    layernorm_stats(p, C, eps, &mean, &sd);
    for (int i = 0; i < C; ++i) y[r * C + i] = layernorm_elem(p[i], mean, sd, gamma, beta, i, round);
  }
}

// Rows of at most LN_STAGED_MAX_C channels, C % 4 == 0: each warp takes 8
// consecutive rows (one contiguous block of 8 C floats), copies them into
// shared memory with 16-byte coalesced loads, lane 4 r computes row r's
// mean and sd (the sequential sums), then the row's 4 lanes normalise its
// columns sub, sub + 4, ... in place, and the block leaves with 16-byte
// coalesced stores.  Row pitch = 4 (mod 32) floats: the 8 summing lanes read
// 8 distinct banks, and the 32 lanes of the elementwise pass 32.  (One
// thread per row over global memory touched 32 lines per warp access and
// left the elementwise pass to one lane per row.)
constexpr int LN_STAGED_MAX_C = 352;  // 4 warps x 8 rows x pitch floats within 48 KB
constexpr int LN_WARPS = 4;
__host__ __device__ __forceinline__ int ln_pitch(int C) { return C + ((4 - C) % 32 + 32) % 32; }
__global__ void __launch_bounds__(32 * LN_WARPS) layernorm_staged_kernel(
    const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
    float* __restrict__ y, int64_t rows, int C, float eps, int round) {
  extern __shared__ __align__(16) float ln_rows[];
  const int pitch = ln_pitch(C);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t r0 = ((int64_t)blockIdx.x * LN_WARPS + wid) * 8;
  if (r0 >= rows) return;
  const int nr = rows - r0 < 8 ? (int)(rows - r0) : 8;
  float* buf = ln_rows + wid * 8 * pitch;
  const int n4 = nr * C / 4;
  const float4* s4 = reinterpret_cast<const float4*>(x + r0 * C);
  float4* d4 = reinterpret_cast<float4*>(y + r0 * C);
  const int c4 = C / 4;
#pragma unroll 4
  for (int q = lane; q < n4; q += 32) {
    const int row = q / c4;
    *reinterpret_cast<float4*>(buf + row * pitch + 4 * (q - row * c4)) = __ldg(s4 + q);
  }
  __syncwarp();
  const int rr = lane >> 2, sub = lane & 3;
  float mean = 0.f, sd = 1.f;
  if (sub == 0 && rr < nr) layernorm_stats(buf + rr * pitch, C, eps, &mean, &sd);
  mean = __shfl_sync(0xffffffffu, mean, lane & ~3);
  sd = __shfl_sync(0xffffffffu, sd, lane & ~3);
  if (rr < nr) {
    float* p = buf + rr * pitch;
    for (int i = sub; i < C; i += 4) p[i] = layernorm_elem(p[i], mean, sd, gamma, beta, i, round);
  }
  __syncwarp();
#pragma unroll 4
  for (int q = lane; q < n4; q += 32) {
    const int row = q / c4;
    d4[q] = *reinterpret_cast<const float4*>(buf + row * pitch + 4 * (q - row * c4));
  }
}

cudaError_t launch_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                             int64_t rows, int c, float eps, int round, cudaStream_t st) {
  if (rows <= 0 || c <= 0) return cudaSuccess;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  if (c <= LN_STAGED_MAX_C && (c & 3) == 0 && aligned) {
    const int64_t blocks = (rows + 8 * LN_WARPS - 1) / (8 * LN_WARPS);
    const size_t smem = (size_t)LN_WARPS * 8 * ln_pitch(c) * sizeof(float);
    layernorm_staged_kernel<<<(unsigned)blocks, 32 * LN_WARPS, smem, st>>>(x, gamma, beta, y, rows, c, eps, round);
  } else {
    layernorm_kernel<<<grid_for(rows, 128), 128, 0, st>>>(x, gamma, beta, y, rows, c, eps, round);
  }
  return cudaGetLastError();
}

// CTC-head exit on logits: per row the first strict maximum (ties -> lowest
// index) and its softmax probability 1 / sum_j exp1(l_j - max) (the max's own
// term is exp1(0) == 1).  One warp per row.  Replaces Softmax + argmax exit
// (activation.rs:321-403 + n_exit3_argmax.comp) without writing the
// probabilities.
__global__ void softmax_argmax_kernel(const float* __restrict__ x, float* __restrict__ pairs,
                                      int64_t rows, int cols) {
  const int warps_per_block = blockDim.x >> 5;
  const int64_t row = (int64_t)blockIdx.x * warps_per_block + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = x + row * cols;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = lane; c < cols; c += 32) {
    const float v = __ldg(p + c);
    if (v > bv) { bv = v; bi = c; }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  float s = 0.f;
  for (int c = lane; c < cols; c += 32) s = __fadd_rn(s, exp1(__fsub_rn(__ldg(p + c), bv)));
#pragma unroll
  for (int off = 16; off; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  if (lane == 0) {
    pairs[2 * row] = __fdiv_rn(1.0f, s);
    pairs[2 * row + 1] = __uint_as_float((unsigned)bi);
  }
}

cudaError_t launch_softmax_argmax(const float* x, float* pairs, int64_t rows, int cols,
                                  cudaStream_t st) {
  const int64_t blocks = (rows + 7) / 8;
  softmax_argmax_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, pairs, rows, cols);
  return cudaGetLastError();
}

}  // namespace qpc

namespace qpc {

// softmax_row on a shared-memory row, by one 8-lane group of the warp
// (lanes 8 g .. 8 g + 7; j = lane & 7): the group's lanes keep the
// reference's eight lane accumulators (element i goes to lane i % 8, in
// ascending order), the max and the hsum8 tree are combined from them in the
// reference's order, the scalar tail follows sequentially, and the group
// scales.  Bit-identical to softmax_row.  Every lane of the warp calls it
// (the groups' shuffles are warp-wide); `valid` = false marks a group without
// a row (its scratch row is processed and nothing reads it).
__device__ __forceinline__ void softmax_row_group8(float* row, int inner, int j, bool valid) {
  const unsigned full = 0xffffffffu;
  const int base = (threadIdx.x & 31) & ~7;
  if (inner < 8) {
    if (j == 0 && valid) softmax_row(row, row, inner);
    __syncwarp();
    return;
  }
  const int n8 = inner & ~7;
  float vmax = row[0];
  for (int i = 0; i < n8; i += 8) {
    const float v = row[i + j];
    if (v > vmax) vmax = v;
  }
  float mx = __shfl_sync(full, vmax, base);
#pragma unroll
  for (int k = 1; k < 8; ++k) {
    const float vk = __shfl_sync(full, vmax, base + k);
    if (vk > mx) mx = vk;
  }
  for (int i = n8; i < inner; ++i)
    if (row[i] > mx) mx = row[i];
  float acc = 0.f;
  for (int i = 0; i < n8; i += 8) {
    const float e = exp1(__fsub_rn(row[i + j], mx));
    row[i + j] = e;
    acc = __fadd_rn(acc, e);
  }
  float a[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = __shfl_sync(full, acc, base + k);
  const float t0 = __fadd_rn(a[0], a[4]), t1 = __fadd_rn(a[1], a[5]);
  const float t2 = __fadd_rn(a[2], a[6]), t3 = __fadd_rn(a[3], a[7]);
  float sum = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
  __syncwarp();
  for (int i = n8; i < inner; ++i) {
    const float e = exp1(__fsub_rn(row[i], mx));
    sum = __fadd_rn(sum, e);
    __syncwarp();
    if (j == 0) row[i] = e;
  }
  const float inv = __fdiv_rn(1.0f, sum);
  __syncwarp();
  for (int i = j; i < inner; i += 8) row[i] = __fmul_rn(row[i], inv);
  __syncwarp();
}

// Fused multi-head attention of the SVTR rec block, one CTA per (line,
// head), bit-identical to the reference's separate ops: q' = q * scale
// (Mul), s[t][u] = fma chain over d ascending of q'[t][d] k[u][d] from 0
// (the dynamic MatMul's per-row outer product, shape.rs:669-697), the row
// softmax (activation.rs:321-403), o[t][d] = fma chain over u ascending of
// p[t][u] v[u][d] from 0, written at column h*D + d of the line's [T, H*D]
// rows (the Transpose + Reshape).  q, k, v of the head are staged in shared
// memory; each warp takes 4 query rows at a time (the rec net's 40 rows: one
// quad per warp): all 32 lanes make the 4 x T scores, each 8-lane group one
// row's softmax (softmax_row_group8, in the reference's order), and all lanes
// the 4 x D outputs.  (One row per warp at a time left 24 lanes idle in the
// softmax and 17 in P V.)
// TT, DD > 0: T and D known at compile time (the rec net's 40 x 15), so the
// dot-product and P V loops unroll and their shared-memory loads are issued
// ahead of the FMA chains, whose order is unchanged; 0: runtime sizes.
constexpr int ATT_WARPS = 10;
template <int TT, int DD>
__global__ void __launch_bounds__(32 * ATT_WARPS) attention_kernel(const float* __restrict__ qkv,
                                                                  float* __restrict__ out, int T_rt, int H,
                                                                  int D_rt, float scale) {
  const int T = TT > 0 ? TT : T_rt, D = DD > 0 ? DD : D_rt;
  extern __shared__ float sm[];
  const int b = blockIdx.x / H, h = blockIdx.x % H;
  const int C = H * D, C3 = 3 * C;
  float* qs = sm;            // [T][D], scaled
  float* ks = qs + T * D;    // [T][D]
  float* vs = ks + T * D;    // [T][D]
  float* pr = vs + T * D;    // [ATT_WARPS][4][T] score / probability rows
  const float* base = qkv + (int64_t)b * T * C3 + h * D;
  for (int i = threadIdx.x; i < T * D; i += blockDim.x) {
    const int t = i / D, d = i - t * D;
    const float* r = base + (int64_t)t * C3 + d;
    qs[i] = __fmul_rn(__ldg(r), scale);
    ks[i] = __ldg(r + C);
    vs[i] = __ldg(r + 2 * C);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 3, j = lane & 7;  // 8-lane group g: query row 4 quad + g
  float* p4 = pr + warp * 4 * T;
  for (int t0 = 4 * warp; t0 < T; t0 += 4 * ATT_WARPS) {
    const int nq = min(4, T - t0);
    // scores: (row, key) pairs over all lanes, each a D-long fma chain
    for (int idx = lane; idx < nq * T; idx += 32) {
      const int r = idx / T, u = idx - r * T;
      const float* q = qs + (t0 + r) * D;
      const float* k = ks + u * D;
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) acc = __fmaf_rn(q[d], k[d], acc);
      p4[r * T + u] = acc;
    }
    __syncwarp();
    softmax_row_group8(p4 + g * T, T, j, g < nq);
    // P V: (row, dim) pairs over all lanes, each a T-long fma chain
    for (int idx = lane; idx < nq * D; idx += 32) {
      const int r = idx / D, d = idx - r * D;
      const float* pp = p4 + r * T;
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < T; ++u) acc = __fmaf_rn(pp[u], vs[u * D + d], acc);
      out[((int64_t)b * T + t0 + r) * C + h * D + d] = acc;
    }
    __syncwarp();
  }
}

cudaError_t launch_attention(const float* qkv, int64_t B, int T, int H, int D, float scale, float* out,
                             cudaStream_t st) {
  if (B < 0 || T <= 0 || H <= 0 || D <= 0 || D > 32) return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  const int64_t blocks = B * H;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  const size_t smem = ((size_t)3 * T * D + (size_t)ATT_WARPS * 4 * T) * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  auto kern = (T == 40 && D == 15) ? attention_kernel<40, 15> : attention_kernel<0, 0>;
  if (cudaError_t e = ensure_dyn_smem((const void*)kern, (int)smem); e != cudaSuccess) return e;
  kern<<<(unsigned)blocks, 32 * ATT_WARPS, smem, st>>>(qkv, out, T, H, D, scale);
  return cudaGetLastError();
}

}  // namespace qpc
