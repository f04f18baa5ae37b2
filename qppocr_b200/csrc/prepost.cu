// Det / rec pre- and post-processing around the network, on the device:
// the byte and f32 arithmetic of the reference's host code, bit for bit.
//
//  * resize_bilinear_rgb_u8 (qppocr-kernels resize.rs:158-210): the det input
//    resize and the rec line resize.  Source coordinate (x + 0.5) * sx - 0.5
//    clamped at 0, truncated to the left tap, right tap clamped to the edge;
//    value = p00 (1-lx)(1-fy) with two multiplies, then three fused
//    multiply-adds (p01 lx, 1-fy), (p10 (1-lx), fy), (p11 lx, fy); stored as
//    u8 (val + 0.5) clamped to [0, 255] and truncated.
//  * det normalisation (engine.rs:963-982): v = u8 * (1/255), (v - 0.5) * 2,
//    HWC -> planar CHW.  Fused with the resize: the u8 value of the resized
//    pixel is produced and normalised in registers.
//  * DB mask (geometry.rs:286-296 binarize, resize.rs:213-245 dilate2x2_max):
//    pred > thresh -> 1, then the 2x2 dilation (cv2.dilate 2x2 kernel,
//    anchor (1,1), out-of-bounds samples ignored).
// All intrinsics are the IEEE round-to-nearest forms, so nothing contracts.
#include "kernels.h"

namespace qpc {

namespace {

struct ResizeMap {
  int sw, sh, dw, dh;
  float sx, sy;  // sw / dw, sh / dh (f32 division, computed on the host)
};

// Left tap, right tap and weight of one output coordinate.
__device__ __forceinline__ void bilinear_tap(int o, float s, int size, int& i0, int& i1, float& f) {
  float v = __fsub_rn(__fmul_rn(__fadd_rn((float)o, 0.5f), s), 0.5f);
  v = fmaxf(v, 0.0f);
  i0 = min((int)v, size - 1);
  i1 = min(i0 + 1, size - 1);
  f = __fsub_rn(v, (float)i0);
}

__device__ __forceinline__ uint8_t bilinear_u8(float p00, float p01, float p10, float p11, float lx,
                                               float fy) {
  const float ilx = __fsub_rn(1.0f, lx), ify = __fsub_rn(1.0f, fy);
  float t = __fmul_rn(__fmul_rn(p00, ilx), ify);
  t = __fmaf_rn(__fmul_rn(p01, lx), ify, t);
  t = __fmaf_rn(__fmul_rn(p10, ilx), fy, t);
  const float val = __fmaf_rn(__fmul_rn(p11, lx), fy, t);
  return (uint8_t)fminf(fmaxf(__fadd_rn(val, 0.5f), 0.0f), 255.0f);
}

// The three channels of resized pixel (x, y) of image `img`.
__device__ __forceinline__ void resized_rgb(const uint8_t* __restrict__ src, const ResizeMap& m, int img, int x,
                                            int y, uint8_t (&out)[3]) {
  int i0, i1, j0, j1;
  float lx, fy;
  bilinear_tap(x, m.sx, m.sw, i0, i1, lx);
  bilinear_tap(y, m.sy, m.sh, j0, j1, fy);
  const uint8_t* r0 = src + ((int64_t)img * m.sh + j0) * m.sw * 3;
  const uint8_t* r1 = src + ((int64_t)img * m.sh + j1) * m.sw * 3;
#pragma unroll
  for (int c = 0; c < 3; ++c)
    out[c] = bilinear_u8((float)r0[i0 * 3 + c], (float)r0[i1 * 3 + c], (float)r1[i0 * 3 + c],
                         (float)r1[i1 * 3 + c], lx, fy);
}

__global__ void __launch_bounds__(256) resize_bilinear_rgb_u8_kernel(const uint8_t* __restrict__ src,
                                                                     uint8_t* __restrict__ dst, int n,
                                                                     ResizeMap m) {
  const int64_t total = (int64_t)n * m.dh * m.dw;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int x = (int)(t % m.dw);
    const int64_t r = t / m.dw;
    const int y = (int)(r % m.dh), img = (int)(r / m.dh);
    uint8_t px[3];
    resized_rgb(src, m, img, x, y, px);
    uint8_t* o = dst + t * 3;
    o[0] = px[0];
    o[1] = px[1];
    o[2] = px[2];
  }
}

// resize (skipped when the sizes match, as the reference does) + normalise.
__global__ void __launch_bounds__(256) det_preprocess_kernel(const uint8_t* __restrict__ src,
                                                             float* __restrict__ dst, int n, ResizeMap m,
                                                             int identity) {
  const int64_t plane = (int64_t)m.dh * m.dw;
  const int64_t total = (int64_t)n * plane;
  const float scale = 1.0f / 255.0f, mean = 0.5f, istd = 1.0f / 0.5f;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int x = (int)(t % m.dw);
    const int64_t r = t / m.dw;
    const int y = (int)(r % m.dh), img = (int)(r / m.dh);
    uint8_t px[3];
    if (identity) {
      const uint8_t* p = src + t * 3;
      px[0] = p[0];
      px[1] = p[1];
      px[2] = p[2];
    } else {
      resized_rgb(src, m, img, x, y, px);
    }
    float* d = dst + (int64_t)img * 3 * plane + (int64_t)y * m.dw + x;
#pragma unroll
    for (int c = 0; c < 3; ++c) d[c * plane] = __fmul_rn(__fsub_rn(__fmul_rn((float)px[c], scale), mean), istd);
  }
}

// 4 horizontally adjacent mask bytes per thread (one u32 store).
__global__ void __launch_bounds__(256) db_mask_kernel(const float* __restrict__ pred, const uint8_t* __restrict__ m_in,
                                                      uint8_t* __restrict__ out, int n, int h, int w, float thresh,
                                                      int dilate, int vec4) {
  const int wq = (w + 3) / 4;
  const int64_t total = (int64_t)n * h * wq;
  auto bit = [&](int img, int y, int x) -> uint8_t {
    const int64_t i = ((int64_t)img * h + y) * w + x;
    return pred ? (uint8_t)(__ldg(pred + i) > thresh ? 1 : 0) : __ldg(m_in + i);
  };
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int xq = (int)(t % wq);
    const int64_t r = t / wq;
    const int y = (int)(r % h), img = (int)(r / h);
    uint8_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int x = xq * 4 + k;
      uint8_t v = 0;
      if (x < w) {
        v = bit(img, y, x);
        if (dilate) {
          if (x > 0) v = max(v, bit(img, y, x - 1));
          if (y > 0) {
            v = max(v, bit(img, y - 1, x));
            if (x > 0) v = max(v, bit(img, y - 1, x - 1));
          }
        }
      }
      o[k] = v;
    }
    uint8_t* dp = out + ((int64_t)img * h + y) * w + xq * 4;
    if (vec4) {
      *reinterpret_cast<uint32_t*>(dp) = (uint32_t)o[0] | ((uint32_t)o[1] << 8) | ((uint32_t)o[2] << 16) |
                                         ((uint32_t)o[3] << 24);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (xq * 4 + k < w) dp[k] = o[k];
    }
  }
}

// Rec line pack (crop.rs:153-185 pack_crop into the zeroed batch tensor of
// engine.rs:1425-1440): line k (an h x w x 3 uint8 crop at byte offset
// off[k]) becomes rows 0..img_h-1, columns 0..rw-1 of batch item k: bilinear
// resize to rw x img_h, then v = u8 / 255, (v - 0.5) / 0.5; or, pad_only, the
// crop itself centred vertically (columns < min(w, img_w)).  Everything else
// is 0.  One block row (blockIdx.y) per line.
__global__ void __launch_bounds__(256) rec_pack_kernel(const uint8_t* __restrict__ crops,
                                                       const int64_t* __restrict__ off, const int* __restrict__ hs,
                                                       const int* __restrict__ ws, const int* __restrict__ rws,
                                                       const int* __restrict__ pads, float* __restrict__ out,
                                                       int img_h, int img_w) {
  const int k = blockIdx.y;
  const int h = hs[k], w = ws[k], rw = rws[k], pad = pads[k];
  const uint8_t* src = crops + off[k];
  const int64_t plane = (int64_t)img_h * img_w;
  float* dst = out + (int64_t)k * 3 * plane;
  ResizeMap m;
  m.sw = w;
  m.sh = h;
  m.dw = rw;
  m.dh = img_h;
  m.sx = __fdiv_rn((float)w, (float)rw);
  m.sy = __fdiv_rn((float)h, (float)img_h);
  const int y0 = (img_h - h) / 2, cols = min(w, img_w);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < img_h * img_w; i += gridDim.x * blockDim.x) {
    const int y = i / img_w, x = i - y * img_w;
    float o[3] = {0.f, 0.f, 0.f};
    bool have = false;
    uint8_t px[3];
    if (pad) {
      if (y >= y0 && y < y0 + h && x < cols) {
        const uint8_t* p = src + ((int64_t)(y - y0) * w + x) * 3;
        px[0] = p[0];
        px[1] = p[1];
        px[2] = p[2];
        have = true;
      }
    } else if (x < rw) {
      resized_rgb(src, m, 0, x, y, px);
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

int grid_of(int64_t items) {
  const int64_t blocks = (items + 255) / 256;
  const int64_t cap = 148LL * 16;
  return (int)(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

ResizeMap make_map(int sh, int sw, int dh, int dw) {
  ResizeMap m;
  m.sw = sw;
  m.sh = sh;
  m.dw = dw;
  m.dh = dh;
  m.sx = (float)sw / (float)dw;
  m.sy = (float)sh / (float)dh;
  return m;
}

}  // namespace

cudaError_t launch_resize_bilinear_rgb_u8(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh,
                                          int dw, cudaStream_t st) {
  if (n < 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  resize_bilinear_rgb_u8_kernel<<<grid_of((int64_t)n * dh * dw), 256, 0, st>>>(src, dst, n,
                                                                               make_map(sh, sw, dh, dw));
  return cudaGetLastError();
}

cudaError_t launch_det_preprocess(const uint8_t* src, int n, int sh, int sw, float* dst, int dh, int dw,
                                  cudaStream_t st) {
  if (n < 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  det_preprocess_kernel<<<grid_of((int64_t)n * dh * dw), 256, 0, st>>>(
      src, dst, n, make_map(sh, sw, dh, dw), (sh == dh && sw == dw) ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_rec_pack(const uint8_t* crops, const int64_t* off, const int* hs, const int* ws,
                            const int* rws, const int* pads, int n, int img_h, int img_w, float* out,
                            cudaStream_t st) {
  if (n < 0 || img_h <= 0 || img_w <= 0 || n > 65535) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int per = img_h * img_w;
  dim3 grid((per + 255) / 256, n);
  rec_pack_kernel<<<grid, 256, 0, st>>>(crops, off, hs, ws, rws, pads, out, img_h, img_w);
  return cudaGetLastError();
}

cudaError_t launch_db_mask(const float* pred, const uint8_t* mask_in, uint8_t* out, int n, int h, int w,
                           float thresh, int dilate, cudaStream_t st) {
  if (n < 0 || h <= 0 || w <= 0 || (!pred && !mask_in)) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  const int vec4 = (w & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0;
  db_mask_kernel<<<grid_of((int64_t)n * h * ((w + 3) / 4)), 256, 0, st>>>(pred, mask_in, out, n, h, w, thresh,
                                                                          dilate, vec4);
  return cudaGetLastError();
}

}  // namespace qpc
