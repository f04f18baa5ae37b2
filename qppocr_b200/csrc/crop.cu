// Text-box post-processing and line preparation on the device, bit-exact
// with the reference's host code:
//
//  * box_score_fast (crates/qppocr-core/src/pipeline/geometry.rs:221-269):
//    mean DB probability inside a quadrilateral by scan-line even-odd fill.
//    The sum is f64 in the reference's order (rows ascending, spans left to
//    right), so one warp scores one box: the lanes load each 32-pixel piece
//    of a span (coalesced) into shared memory and lane 0 adds them in order.
//  * crop_text_box (crates/qppocr-core/src/pipeline/crop.rs:8-127): the
//    perspective crop of a box.  Thread 0 of the box's block solves the 8 x 9
//    homography system in f64 exactly as the reference does (Gauss-Jordan,
//    partial pivoting by strict |a| >, rows scaled by the pivot captured
//    before the loop); every thread then maps its output pixels back in f64
//    and samples bilinearly with the edge replicated (first term two
//    multiplies, then three fused multiply-adds, as the reference's
//    mul_add).  Tall crops (ch / cw >= 1.5) are written rotated clockwise.
//  * line pack (crop.rs:153-185 pack_crop, crop.rs:193-218 cls_view): a view
//    of a crop (column offset and width inside the crop's rows, optionally
//    rotated 180 degrees as the engine does for lines the classifier flags,
//    engine.rs:1402-1407) resized to rw x img_h and normalised (v/255 - 0.5)
//    / 0.5 into a zeroed [3, img_h, img_w] slot, or placed unresized and
//    centred vertically (pad_only).
// All arithmetic uses the round-to-nearest intrinsics (nothing contracts).
#include "kernels.h"

namespace qpc {

namespace {

// Rust `as i32` on f32 / f64: truncation toward zero, saturating, NaN -> 0
// (the PTX float-to-int conversions saturate and map NaN to 0 as well).
__device__ __forceinline__ int to_i32(double v) { return __double2int_rz(v); }
__device__ __forceinline__ int to_i32f(float v) { return __float2int_rz(v); }

// One warp per box; every lane follows the scan (uniform control flow) and
// lane 0 holds the sum.
__device__ float box_score_warp(const float* __restrict__ pred, int hh, int ww, const float* __restrict__ bp,
                                int lane, float* __restrict__ stage) {
  float fxmin = 3.40282347e38f, fxmax = -3.40282347e38f, fymin = 3.40282347e38f, fymax = -3.40282347e38f;
  float px[4], py[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    px[i] = bp[2 * i];
    py[i] = bp[2 * i + 1];
    fxmin = fminf(fxmin, px[i]);
    fxmax = fmaxf(fxmax, px[i]);
    fymin = fminf(fymin, py[i]);
    fymax = fmaxf(fymax, py[i]);
  }
  const int xmin = min(max(to_i32f(floorf(fxmin)), 0), ww - 1);
  const int xmax = min(max(to_i32f(ceilf(fxmax)), 0), ww - 1);
  const int ymin = min(max(to_i32f(floorf(fymin)), 0), hh - 1);
  const int ymax = min(max(to_i32f(ceilf(fymax)), 0), hh - 1);
  double sum = 0.0;
  long long count = 0;
  for (int y = ymin; y <= ymax; ++y) {
    const float sy = __fadd_rn((float)y, 0.5f);
    float xs[4];
    int nx = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = (i + 1) & 3;
      if ((py[i] <= sy && py[j] > sy) || (py[j] <= sy && py[i] > sy)) {
        const float t = __fdiv_rn(__fsub_rn(sy, py[i]), __fsub_rn(py[j], py[i]));
        xs[nx++] = __fadd_rn(px[i], __fmul_rn(t, __fsub_rn(px[j], px[i])));
      }
    }
    // ascending insertion sort (equal values are interchangeable)
    for (int i = 1; i < nx; ++i) {
      const float v = xs[i];
      int j = i - 1;
      while (j >= 0 && xs[j] > v) {
        xs[j + 1] = xs[j];
        --j;
      }
      xs[j + 1] = v;
    }
    for (int i = 0; i + 1 < nx; i += 2) {
      const int xa = max(to_i32f(ceilf(__fsub_rn(xs[i], 0.5f))), xmin);
      const int xb = min(to_i32f(floorf(__fsub_rn(xs[i + 1], 0.5f))), xmax);
      const float* row = pred + (int64_t)y * ww;
      for (int x0 = xa; x0 <= xb; x0 += 32) {
        const int cnt = min(32, xb - x0 + 1);
        stage[lane] = lane < cnt ? __ldg(row + x0 + lane) : 0.0f;
        __syncwarp();
        if (lane == 0) {
#pragma unroll 8
          for (int j = 0; j < cnt; ++j) sum = __dadd_rn(sum, (double)stage[j]);
        }
        __syncwarp();  // lane 0 has read the piece before it is overwritten
        count += cnt;
      }
    }
  }
  if (count == 0) return 0.0f;
  return __double2float_rn(__ddiv_rn(sum, (double)count));
}

__global__ void __launch_bounds__(256) box_score_kernel(const float* __restrict__ pred, int hh, int ww,
                                                        const float* __restrict__ boxes,
                                                        const int* __restrict__ img, int n,
                                                        float* __restrict__ out) {
  __shared__ float stage[8][32];  // one 32-value piece per warp
  const int k = (int)((blockIdx.x * (unsigned)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (k >= n) return;  // whole warps
  const float r = box_score_warp(pred + (int64_t)img[k] * hh * ww, hh, ww, boxes + 8 * (int64_t)k, lane,
                                 stage[threadIdx.x >> 5]);
  if (lane == 0) out[k] = r;
}

// Pixels of one crop per block: 4 per thread, so the homography (thread 0's
// serial f64 solve) is repeated once per 1024 pixels.
constexpr int CROP_PIX_PER_BLOCK = 1024;

// Blocks (x, k): crop k, pixels [x * 1024, (x + 1) * 1024); thread 0 of each
// active block solves the homography into shared memory.
__global__ void __launch_bounds__(256) crop_boxes_kernel(const uint8_t* __restrict__ imgs, int h, int w,
                                                         const float* __restrict__ pts, const int* __restrict__ img,
                                                         const int* __restrict__ cws, const int* __restrict__ chs,
                                                         const int64_t* __restrict__ off, uint8_t* __restrict__ out) {
  const int k = blockIdx.y;
  const int cw = cws[k], ch = chs[k];
  // blocks past this crop's pixels (the grid is sized for the largest crop)
  // leave before solving
  if ((int64_t)blockIdx.x * CROP_PIX_PER_BLOCK >= (int64_t)cw * ch) return;
  __shared__ double hm[9];
  if (threadIdx.x == 0) {
    const float* p = pts + 8 * (int64_t)k;
    double a[8][9];
    for (int i = 0; i < 4; ++i) {
      const double dx = (i == 1 || i == 2) ? (double)cw : 0.0;
      const double dy = i >= 2 ? (double)ch : 0.0;
      const double sx = (double)p[2 * i], sy = (double)p[2 * i + 1];
      a[2 * i][0] = dx;
      a[2 * i][1] = dy;
      a[2 * i][2] = 1.0;
      a[2 * i][3] = 0.0;
      a[2 * i][4] = 0.0;
      a[2 * i][5] = 0.0;
      a[2 * i][6] = __dmul_rn(-dx, sx);
      a[2 * i][7] = __dmul_rn(-dy, sx);
      a[2 * i][8] = sx;
      a[2 * i + 1][0] = 0.0;
      a[2 * i + 1][1] = 0.0;
      a[2 * i + 1][2] = 0.0;
      a[2 * i + 1][3] = dx;
      a[2 * i + 1][4] = dy;
      a[2 * i + 1][5] = 1.0;
      a[2 * i + 1][6] = __dmul_rn(-dx, sy);
      a[2 * i + 1][7] = __dmul_rn(-dy, sy);
      a[2 * i + 1][8] = sy;
    }
    for (int col = 0; col < 8; ++col) {
      int piv = col;
      for (int r = col + 1; r < 8; ++r)
        if (fabs(a[r][col]) > fabs(a[piv][col])) piv = r;
      if (piv != col)
        for (int c = 0; c < 9; ++c) {
          const double t = a[col][c];
          a[col][c] = a[piv][c];
          a[piv][c] = t;
        }
      const double d = a[col][col];
      if (fabs(d) < 1e-12) continue;
      for (int c = col; c < 9; ++c) a[col][c] = __ddiv_rn(a[col][c], d);
      for (int r = 0; r < 8; ++r) {
        if (r == col) continue;
        const double f = a[r][col];
        if (f == 0.0) continue;
        for (int c = col; c < 9; ++c) a[r][c] = __dsub_rn(a[r][c], __dmul_rn(f, a[col][c]));
      }
    }
    for (int i = 0; i < 8; ++i) hm[i] = a[i][8];
    hm[8] = 1.0;
  }
  __syncthreads();
  const bool rot = __fdiv_rn((float)ch, (float)cw) >= 1.5f;
  const uint8_t* src = imgs + (int64_t)img[k] * h * w * 3;
  uint8_t* dst = out + off[k];
  const int i_end = min(cw * ch, (int)((blockIdx.x + 1) * CROP_PIX_PER_BLOCK));
  for (int i = blockIdx.x * CROP_PIX_PER_BLOCK + threadIdx.x; i < i_end; i += blockDim.x) {
    const int y = i / cw, x = i - y * cw;
    const double xf = (double)x, yf = (double)y;
    const double den = __dadd_rn(__dadd_rn(__dmul_rn(hm[6], xf), __dmul_rn(hm[7], yf)), hm[8]);
    const double sx = __ddiv_rn(__dadd_rn(__dadd_rn(__dmul_rn(hm[0], xf), __dmul_rn(hm[1], yf)), hm[2]), den);
    const double sy = __ddiv_rn(__dadd_rn(__dadd_rn(__dmul_rn(hm[3], xf), __dmul_rn(hm[4], yf)), hm[5]), den);
    int ix = to_i32(floor(sx));
    int iy = to_i32(floor(sy));
    const float fx = __double2float_rn(__dsub_rn(sx, (double)ix));
    const float fy = __double2float_rn(__dsub_rn(sy, (double)iy));
    ix = min(max(ix, 0), w - 1);
    iy = min(max(iy, 0), h - 1);
    const int ix1 = min(ix + 1, w - 1), iy1 = min(iy + 1, h - 1);
    const uint8_t* r0 = src + (int64_t)iy * w * 3;
    const uint8_t* r1 = src + (int64_t)iy1 * w * 3;
    const int64_t o = rot ? ((int64_t)x * ch + (ch - 1 - y)) * 3 : (int64_t)i * 3;
    const float ifx = __fsub_rn(1.0f, fx), ify = __fsub_rn(1.0f, fy);
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float v00 = r0[ix * 3 + c], v01 = r0[ix1 * 3 + c], v10 = r1[ix * 3 + c], v11 = r1[ix1 * 3 + c];
      float t = __fmul_rn(__fmul_rn(v00, ifx), ify);
      t = __fmaf_rn(__fmul_rn(v01, fx), ify, t);
      t = __fmaf_rn(__fmul_rn(v10, ifx), fy, t);
      const float v = __fmaf_rn(__fmul_rn(v11, fx), fy, t);
      dst[o + c] = (uint8_t)fminf(fmaxf(__fadd_rn(v, 0.5f), 0.0f), 255.0f);
    }
  }
}

// Bilinear taps of one output coordinate (resize.rs:158-210).
__device__ __forceinline__ void tap(int o, float s, int size, int& i0, int& i1, float& f) {
  float v = __fsub_rn(__fmul_rn(__fadd_rn((float)o, 0.5f), s), 0.5f);
  v = fmaxf(v, 0.0f);
  i0 = min((int)v, size - 1);
  i1 = min(i0 + 1, size - 1);
  f = __fsub_rn(v, (float)i0);
}

__device__ __forceinline__ uint8_t lerp_u8(float p00, float p01, float p10, float p11, float lx, float fy) {
  const float ilx = __fsub_rn(1.0f, lx), ify = __fsub_rn(1.0f, fy);
  float t = __fmul_rn(__fmul_rn(p00, ilx), ify);
  t = __fmaf_rn(__fmul_rn(p01, lx), ify, t);
  t = __fmaf_rn(__fmul_rn(p10, ilx), fy, t);
  const float val = __fmaf_rn(__fmul_rn(p11, lx), fy, t);
  return (uint8_t)fminf(fmaxf(__fadd_rn(val, 0.5f), 0.0f), 255.0f);
}

// One block row (blockIdx.y) per line.  View of line k: rows of `stride`
// pixels at byte offset off[k], columns x0[k] .. x0[k] + w[k] - 1, h[k] rows;
// flip[k]: the view rotated 180 degrees.
__global__ void __launch_bounds__(256) line_pack_kernel(const uint8_t* __restrict__ crops, const LinePack lp,
                                                        float* __restrict__ out, int img_h, int img_w) {
  const int k = blockIdx.y;
  const int h = lp.h[k], w = lp.w[k], rw = lp.rw[k], pad = lp.pad[k], x0 = lp.x0[k], stride = lp.stride[k];
  const int flip = lp.flip ? lp.flip[k] : 0;
  const uint8_t* src = crops + lp.off[k];
  auto pix = [&](int x, int y) -> const uint8_t* {  // pixel (x, y) of the (possibly flipped) view
    if (flip) {
      x = w - 1 - x;
      y = h - 1 - y;
    }
    return src + ((int64_t)y * stride + x0 + x) * 3;
  };
  const int64_t plane = (int64_t)img_h * img_w;
  float* dst = out + (int64_t)k * 3 * plane;
  const float sx = __fdiv_rn((float)w, (float)rw), sy = __fdiv_rn((float)h, (float)img_h);
  const int y0 = (img_h - h) / 2, cols = min(w, img_w);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < img_h * img_w; i += gridDim.x * blockDim.x) {
    const int y = i / img_w, x = i - y * img_w;
    float o[3] = {0.f, 0.f, 0.f};
    bool have = false;
    uint8_t px[3];
    if (pad) {
      if (y >= y0 && y < y0 + h && x < cols) {
        const uint8_t* p = pix(x, y - y0);
        px[0] = p[0];
        px[1] = p[1];
        px[2] = p[2];
        have = true;
      }
    } else if (x < rw) {
      int i0, i1, j0, j1;
      float lx, fy;
      tap(x, sx, w, i0, i1, lx);
      tap(y, sy, h, j0, j1, fy);
      const uint8_t *p00 = pix(i0, j0), *p01 = pix(i1, j0), *p10 = pix(i0, j1), *p11 = pix(i1, j1);
#pragma unroll
      for (int c = 0; c < 3; ++c)
        px[c] = lerp_u8((float)p00[c], (float)p01[c], (float)p10[c], (float)p11[c], lx, fy);
      have = true;
    }
    if (have)
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float v = __fdiv_rn((float)px[c], 255.0f);
        o[c] = __fdiv_rn(__fsub_rn(v, 0.5f), 0.5f);
      }
#pragma unroll
    for (int c = 0; c < 3; ++c) dst[c * plane + i] = o[c];
  }
}

}  // namespace

cudaError_t launch_box_score(const float* pred, int h, int w, const float* boxes, const int* img, int n,
                             float* out, cudaStream_t st) {
  if (n < 0 || h <= 0 || w <= 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  box_score_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(pred, h, w, boxes, img, n, out);  // a warp per box
  return cudaGetLastError();
}

cudaError_t launch_crop_boxes(const uint8_t* imgs, int h, int w, const float* pts, const int* img, const int* cw,
                              const int* ch, const int64_t* off, int n, int max_pixels, uint8_t* out,
                              cudaStream_t st) {
  if (n < 0 || h <= 0 || w <= 0 || n > 65535 || max_pixels <= 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int bx = (max_pixels + CROP_PIX_PER_BLOCK - 1) / CROP_PIX_PER_BLOCK;
  if (bx > 65535) return cudaErrorInvalidValue;
  dim3 grid(bx, n);
  crop_boxes_kernel<<<grid, 256, 0, st>>>(imgs, h, w, pts, img, cw, ch, off, out);
  return cudaGetLastError();
}

cudaError_t launch_line_pack(const uint8_t* crops, const LinePack& lp, int n, int img_h, int img_w, float* out,
                             cudaStream_t st) {
  if (n < 0 || img_h <= 0 || img_w <= 0 || n > 65535) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int per = img_h * img_w;
  dim3 grid((per + 255) / 256, n);
  line_pack_kernel<<<grid, 256, 0, st>>>(crops, lp, out, img_h, img_w);
  return cudaGetLastError();
}

}  // namespace qpc
