// TEST INFRASTRUCTURE ONLY — CPU oracle for the qppocr conv/GEMM hot path.
//
// This file restates, in C++, the scalar semantics of the reference's CPU
// kernels (crate `qppocr-kernels`, Rust).  It is the checker the CUDA backend
// is compared against and the timed CPU baseline ("port") in bench.py.  Only
// tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
// may load it.  The product library (libqppocr_cuda.so) never links or calls
// anything here.
//
// Parity pin: the op-level known-answer vectors the reference's own tests hold
// (erf table and exp tolerance, activation.rs:472-513; the naive f64 conv /
// gemm / pool references of tests/kernels.rs:51-1467 with max|d|/max|ref| <
// 1e-5; the xorshift64* test RNG, tests/kernels.rs:30-48) are checked against
// this oracle in tests/test_oracle_pins.py.  Whole-network outputs on the
// synthetic random-init nets have no reference-side fixture (the reference's
// model tests need ONNX files that are not published with it), so at network
// level this oracle is the pin.
//
// Numerics rules restated from the reference:
//  * FTZ|DAZ on in every thread (par.rs:229-243).
//  * No floating-point contraction except where the reference writes
//    `mul_add` (Rust never contracts); this file is compiled with
//    -ffp-contract=off and uses std::fma exactly where the reference does.
//  * Per-output accumulation orders follow the scalar "判据" paths
//    (gemm.rs:523-589 panel_body, conv.rs:45-71 depthwise_plane_scalar,
//    conv.rs:816-838 convt_row_scalar, activation.rs:346-403 softmax).
//    Independent outputs are computed in SIMD-friendly loops; that never
//    changes any single element's operation sequence.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>
#include <xmmintrin.h>

namespace {

// ----------------------------------------------------------------- threads
// A persistent fork-join pool over all host cores (the reference's own pool,
// par.rs, also spans every core).  FTZ/DAZ is set in each worker.
void set_ftz_daz() { _mm_setcsr(_mm_getcsr() | 0x8040u); }

class Pool {
 public:
  Pool() {
    int n = (int)std::thread::hardware_concurrency();
    if (const char* e = std::getenv("ORC_THREADS")) n = std::max(1, atoi(e));
    nthreads_ = std::max(1, n);
    for (int i = 1; i < nthreads_; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int threads() const { return nthreads_; }
  // fn(begin, end) over [0, units) in chunks; the calling thread helps.
  void run(int64_t units, int64_t chunk, const std::function<void(int64_t, int64_t)>& fn) {
    set_ftz_daz();
    if (units <= 0) return;
    if (nthreads_ == 1 || units <= chunk) {
      fn(0, units);
      return;
    }
    std::unique_lock<std::mutex> big(run_mu_);  // one parallel region at a time
    {
      std::lock_guard<std::mutex> g(mu_);
      fn_ = &fn;
      units_ = units;
      chunk_ = chunk;
      next_.store(0);
      active_ = (int)workers_.size();
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> g(mu_);
    done_cv_.wait(g, [this] { return active_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      int64_t b = next_.fetch_add(chunk_);
      if (b >= units_) break;
      (*fn_)(b, std::min(units_, b + chunk_));
    }
  }
  void loop() {
    set_ftz_daz();
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> g(mu_);
        cv_.wait(g, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
      }
      work();
      std::lock_guard<std::mutex> g(mu_);
      if (--active_ == 0) done_cv_.notify_all();
    }
  }
  int nthreads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex mu_, run_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t, int64_t)>* fn_ = nullptr;
  int64_t units_ = 0, chunk_ = 1;
  std::atomic<int64_t> next_{0};
  int active_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

void parallel_for(int64_t units, const std::function<void(int64_t, int64_t)>& fn,
                  int64_t min_chunk = 1) {
  int64_t per = std::max<int64_t>(min_chunk, units / (pool().threads() * 4) + 1);
  pool().run(units, per, fn);
}

inline float f_from_bits(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint32_t f_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

// ------------------------------------------------------------ activations
// activation.rs:28-47 exp1 (scalar mirror of exp256_ps).
inline float exp1(float x) {
  const float LN2_HI = 0.6931472f;
  const float LN2_LO = -2.9802322e-8f;
  const float INV_LN2 = 1.442695f;
  x = std::max(std::min(x, 88.0f), -88.0f);
  float kf = std::nearbyint(x * INV_LN2);  // round-ties-even (default mode)
  float r = std::fma(-kf, LN2_HI, x);
  r = std::fma(-kf, LN2_LO, r);
  float p = 1.0f / 720.0f;
  p = std::fma(p, r, 1.0f / 120.0f);
  p = std::fma(p, r, 1.0f / 24.0f);
  p = std::fma(p, r, 1.0f / 6.0f);
  p = std::fma(p, r, 0.5f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  int32_t ki = (int32_t)kf + 127;
  return f_from_bits((uint32_t)ki << 23) * p;
}

// activation.rs:53-66 erf1 (A&S 7.1.26).
inline float erf1(float x) {
  float ax = f_from_bits(f_bits(x) & 0x7fffffffu);
  float t = 1.0f / std::fma(0.3275911f, ax, 1.0f);
  float p = 1.0614054f;
  p = std::fma(p, t, -1.453152027f);
  p = std::fma(p, t, 1.421413741f);
  p = std::fma(p, t, -0.284496736f);
  p = std::fma(p, t, 0.2548296f);
  p *= t;
  float e = exp1(ax * (0.0f - ax));
  float r = std::fma(-p, e, 1.0f);
  return f_from_bits(f_bits(r) | (f_bits(x) & 0x80000000u));
}

// Fused-activation codes carried by an optimized Conv node's `act` attribute
// (executor.rs:459-475): 0 none, 1 GELU(c1,c2,c3), 2 ReLU.
struct Act {
  int kind = 0;
  float c1 = 1.4142135f, c2 = 1.0f, c3 = 0.5f;
};

// activation.rs:136-145 apply_act on an already-written output segment.
void apply_act(float* p, int64_t n, const Act& a) {
  if (a.kind == 1) {
    float inv_c1 = 1.0f / a.c1;  // activation.rs:214
    for (int64_t i = 0; i < n; ++i) {
      float v = p[i];
      p[i] = a.c3 * v * (erf1(v * inv_c1) + a.c2);
    }
  } else if (a.kind == 2) {
    for (int64_t i = 0; i < n; ++i) p[i] = p[i] > 0.0f ? p[i] : 0.0f;
  }
}

// -------------------------------------------------------------- sgemm core
// Per-element semantics of gemm.rs:523-589 (panel_body, the scalar reference
// of the serial panel path):
//   * rows in a full 4-row block, and every row of a full 32-column panel:
//     acc = 0; acc = fma(a[k], b[k], acc) for k ascending; acc += bias.
//   * M%4 tail rows of a partial (<32) panel: s = bias (or 0); s = fma chain.
// This routine computes the sub-block rows [r0, r1) x columns [c0, c1) of the
// full m x n product; r0 must be a multiple of 4 and c0 a multiple of 32 so
// every element keeps the classification it has in the full matrix.
// A is [m][k] row-major, B is [k][ldb], C has row stride ldc.
void gemm_block(const float* a, int64_t m, int64_t k, const float* b, int64_t ldb, int64_t n,
                const float* bias, float* c, int64_t ldc, int64_t r0, int64_t r1, int64_t c0,
                int64_t c1) {
  const int64_t m4 = m - (m % 4);
  for (int64_t n0 = c0; n0 < c1; n0 += 32) {
    const int64_t nn = std::min<int64_t>(32, n - n0);
    const bool full = nn == 32;
    for (int64_t rb = r0; rb < r1; rb += 4) {
      const int64_t rows = std::min<int64_t>(4, r1 - rb);
      alignas(64) float acc[4][32];
      bool seeded[4];
      for (int64_t i = 0; i < rows; ++i) {
        const int64_t row = rb + i;
        seeded[i] = !(row < m4 || full);
        const float seed = (seeded[i] && bias) ? bias[row] : 0.0f;
        for (int j = 0; j < 32; ++j) acc[i][j] = seed;
      }
      if (full && rows == 4) {
        const float* a0 = a + rb * k;
        for (int64_t kk = 0; kk < k; ++kk) {
          const float* brow = b + kk * ldb + n0;
          const float av0 = a0[kk], av1 = a0[k + kk], av2 = a0[2 * k + kk], av3 = a0[3 * k + kk];
          for (int j = 0; j < 32; ++j) {
            const float bv = brow[j];
            acc[0][j] = std::fma(av0, bv, acc[0][j]);
            acc[1][j] = std::fma(av1, bv, acc[1][j]);
            acc[2][j] = std::fma(av2, bv, acc[2][j]);
            acc[3][j] = std::fma(av3, bv, acc[3][j]);
          }
        }
      } else {
        for (int64_t kk = 0; kk < k; ++kk) {
          const float* brow = b + kk * ldb + n0;
          float bv[32];
          for (int j = 0; j < 32; ++j) bv[j] = j < nn ? brow[j] : 0.0f;
          for (int64_t i = 0; i < rows; ++i) {
            const float av = a[(rb + i) * k + kk];
            for (int j = 0; j < 32; ++j) acc[i][j] = std::fma(av, bv[j], acc[i][j]);
          }
        }
      }
      for (int64_t i = 0; i < rows; ++i) {
        const int64_t row = rb + i;
        float* crow = c + row * ldc + n0;
        if (!seeded[i] && bias) {
          const float bb = bias[row];
          for (int64_t j = 0; j < nn; ++j) crow[j] = acc[i][j] + bb;
        } else {
          for (int64_t j = 0; j < nn; ++j) crow[j] = acc[i][j];
        }
      }
    }
  }
}

void gemm_panels(const float* a, int64_t m, int64_t k, const float* b, int64_t ldb, int64_t n,
                 const float* bias, float* c, int64_t ldc) {
  gemm_block(a, m, k, b, ldb, n, bias, c, ldc, 0, m, 0, n);
}

}  // namespace

extern "C" {

int orc_threads() { return pool().threads(); }

// tests/kernels.rs:30-48 — xorshift64* test RNG mapped to [-1, 1).
void orc_xorshift_fill(uint64_t* state, float* out, int64_t n) {
  uint64_t s = *state;
  for (int64_t i = 0; i < n; ++i) {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    uint64_t v = s * 0x2545F4914F6CDD1DULL;
    out[i] = (float)((double)((int64_t)(v >> 40) - (1LL << 23)) / (double)(1LL << 23));
  }
  *state = s;
}

void orc_exp1(const float* x, float* y, int64_t n) {
  set_ftz_daz();
  for (int64_t i = 0; i < n; ++i) y[i] = exp1(x[i]);
}
void orc_erf1(const float* x, float* y, int64_t n) {
  set_ftz_daz();
  for (int64_t i = 0; i < n; ++i) y[i] = erf1(x[i]);
}

// activation.rs:170-189 hardsigmoid_seg_scalar: clamp(fma(x, alpha, beta), 0, 1).
void orc_hardsigmoid(const float* x, float* y, int64_t n, float alpha, float beta) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      float v = std::fma(x[i], alpha, beta);
      y[i] = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
    }
  }, 4096);
}
// activation.rs:197-201 sigmoid_seg_scalar.
void orc_sigmoid(const float* x, float* y, int64_t n) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) y[i] = 1.0f / (1.0f + exp1(-x[i]));
  }, 4096);
}
// activation.rs:157-162 relu (v > 0 ? v : 0; NaN -> 0).
void orc_relu(float* t, int64_t n) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) t[i] = t[i] > 0.0f ? t[i] : 0.0f;
  }, 4096);
}
// activation.rs:208-217 gelu_seg_scalar.
void orc_gelu(float* t, int64_t n, float c1, float c2, float c3) {
  Act a;
  a.kind = 1; a.c1 = c1; a.c2 = c2; a.c3 = c3;
  parallel_for(n, [&](int64_t b, int64_t e) { apply_act(t + b, e - b, a); }, 4096);
}
// activation.rs:224-230 clip_seg_scalar.
void orc_clip(float* t, int64_t n, float lo, float hi) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      float v = t[i];
      float m = v < lo ? lo : v;
      t[i] = hi < m ? hi : m;
    }
  }, 4096);
}
// activation.rs:449-459 sqrt_inplace.
void orc_sqrt(float* t, int64_t n) {
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) t[i] = std::sqrt(t[i]);
  }, 4096);
}

// activation.rs:321-403 softmax_last_dim / softmax_row_scalar: 8-lane max,
// exp1(x - max) with 8 per-lane partial sums reduced by the hsum8 tree
// ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)), scalar tail, then x * (1/sum).
void orc_softmax_last_dim(float* t, int64_t outer, int64_t inner) {
  parallel_for(outer, [&](int64_t b, int64_t e) {
    for (int64_t o = b; o < e; ++o) {
      float* row = t + o * inner;
      int64_t i = 0;
      float mx;
      if (inner >= 8) {
        float vmax[8];
        for (int j = 0; j < 8; ++j) vmax[j] = row[0];
        while (i + 8 <= inner) {
          for (int j = 0; j < 8; ++j)
            if (row[i + j] > vmax[j]) vmax[j] = row[i + j];
          i += 8;
        }
        mx = vmax[0];
        for (int j = 1; j < 8; ++j)
          if (vmax[j] > mx) mx = vmax[j];
      } else {
        i = 1;
        mx = row[0];
      }
      for (; i < inner; ++i)
        if (row[i] > mx) mx = row[i];
      float sum = 0.0f;
      int64_t i2 = 0;
      if (inner >= 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        while (i2 + 8 <= inner) {
          for (int j = 0; j < 8; ++j) {
            float ev = exp1(row[i2 + j] - mx);
            row[i2 + j] = ev;
            acc[j] += ev;
          }
          i2 += 8;
        }
        float t4[4] = {acc[0] + acc[4], acc[1] + acc[5], acc[2] + acc[6], acc[3] + acc[7]};
        sum = (t4[0] + t4[1]) + (t4[2] + t4[3]);
      }
      for (; i2 < inner; ++i2) {
        row[i2] = exp1(row[i2] - mx);
        sum += row[i2];
      }
      float inv = 1.0f / sum;
      for (int64_t j = 0; j < inner; ++j) row[j] *= inv;
    }
  });
}

// gemm.rs:37-49 / 154-167: C[M,N] = A[M,K] * B[K,N] (+bias per row), then
// finish_res (act, residual).  Serial-panel semantics per element; the work is
// split into 2-D tiles (64 rows x 512 columns) that never cut a 4-row block or
// a 32-column panel.
void orc_sgemm(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
               const float* bias, int act, const float* act_c, const float* residual) {
  Act ac;
  ac.kind = act;
  if (act_c) { ac.c1 = act_c[0]; ac.c2 = act_c[1]; ac.c3 = act_c[2]; }
  const int64_t TR = 64, TC = 512;
  const int64_t tr = (m + TR - 1) / TR, tc = (n + TC - 1) / TC;
  parallel_for(tr * tc, [&](int64_t u0, int64_t u1) {
    for (int64_t u = u0; u < u1; ++u) {
      const int64_t ti = u / tc, tj = u % tc;
      const int64_t r0 = ti * TR, r1 = std::min(m, r0 + TR);
      const int64_t c0 = tj * TC, c1 = std::min(n, c0 + TC);
      gemm_block(a, m, k, b, n, n, bias, c, n, r0, r1, c0, c1);
      if (ac.kind || residual)
        for (int64_t r = r0; r < r1; ++r) {
          if (ac.kind) apply_act(c + r * n + c0, c1 - c0, ac);
          if (residual)
            for (int64_t j = c0; j < c1; ++j) c[r * n + j] += residual[r * n + j];
        }
    }
  });
}

// conv.rs:146-156 output shape and conv.rs:222-715 conv2d_res_into (NCHW).
// params: sh, sw, ph, pw, peh, pew, group.  act / act_c as orc_sgemm.
// Returns 0 on success, -1 on an unsupported configuration.
int orc_conv2d(const float* x, const int64_t* xs, const float* w, const int64_t* ws,
               const float* bias, const int32_t* prm, int act, const float* act_c,
               const float* residual, float* y) {
  const int64_t n = xs[0], c = xs[1], h = xs[2], wd = xs[3];
  const int64_t m = ws[0], cg = ws[1], kh = ws[2], kw = ws[3];
  const int64_t sh = prm[0], sw = prm[1], ph = prm[2], pw = prm[3], peh = prm[4], pew = prm[5];
  const int64_t group = prm[6];
  if (group * cg != c || m % group) return -1;
  const int64_t oh = (h + ph + peh - kh) / sh + 1, ow = (wd + pw + pew - kw) / sw + 1;
  if (oh <= 0 || ow <= 0) return -1;
  const int64_t ohw = oh * ow;
  Act ac;
  ac.kind = act;
  if (act_c) { ac.c1 = act_c[0]; ac.c2 = act_c[1]; ac.c3 = act_c[2]; }
  const bool depthwise = group > 1 && cg == 1;
  const bool pw1 = group == 1 && kh == 1 && kw == 1 && sh == 1 && sw == 1 && ph == 0 && pw == 0;
  if (pw1) {
    // 1x1 path: per batch C[m, ohw] = W[m, c] * X[c, ohw] (+bias) -> act -> +res
    for (int64_t bn = 0; bn < n; ++bn)
      orc_sgemm(w, x + bn * c * h * wd, y + bn * m * ohw, m, ohw, c, bias, act, act_c,
                residual ? residual + bn * m * ohw : nullptr);
    return 0;
  }
  if (depthwise) {
    // conv.rs:45-71: per (n, ch) plane, zero-padded input, acc from 0 with
    // ky outer / kx inner fma, then + bias.  Then act (conv.rs:673-677) and
    // residual (conv.rs:702-713).
    const int64_t mult = m / c;  // channel multiplier (1 for PP-OCR)
    parallel_for(n * m, [&](int64_t u0, int64_t u1) {
      std::vector<float> pad((h + ph + peh) * (wd + pw + pew) + 64, 0.0f);
      const int64_t pwidth = wd + pw + pew;
      int64_t last_plane = -1;
      std::vector<float> accrow(ow);
      for (int64_t u = u0; u < u1; ++u) {
        const int64_t bn = u / m, mo = u % m, ch = mo / mult;
        const int64_t plane_id = bn * c + ch;
        if (plane_id != last_plane) {
          std::fill(pad.begin(), pad.end(), 0.0f);
          const float* xc = x + plane_id * h * wd;
          for (int64_t yy = 0; yy < h; ++yy)
            std::memcpy(&pad[(ph + yy) * pwidth + pw], xc + yy * wd, sizeof(float) * wd);
          last_plane = plane_id;
        }
        const float* wc = w + mo * kh * kw;
        const float bv = bias ? bias[mo] : 0.0f;
        float* yc = y + u * ohw;
        for (int64_t oy = 0; oy < oh; ++oy) {
          for (int64_t ox = 0; ox < ow; ++ox) accrow[ox] = 0.0f;
          for (int64_t ky = 0; ky < kh; ++ky) {
            const float* row = &pad[(oy * sh + ky) * pwidth];
            for (int64_t kx = 0; kx < kw; ++kx) {
              const float wv = wc[ky * kw + kx];
              for (int64_t ox = 0; ox < ow; ++ox) accrow[ox] = std::fma(wv, row[ox * sw + kx], accrow[ox]);
            }
          }
          for (int64_t ox = 0; ox < ow; ++ox) yc[oy * ow + ox] = accrow[ox] + bv;
        }
        if (ac.kind) apply_act(yc, ohw, ac);
        if (residual)
          for (int64_t i = 0; i < ohw; ++i) yc[i] += residual[u * ohw + i];
      }
    });
    return 0;
  }
  // General grouped conv: implicit GEMM per output row (conv.rs:553-637 via
  // gemm.rs:75-128): C[mg, ow] = Wg[mg, kk] * B[kk, ow], kk order ch->ky->kx,
  // 32-column panels along the output row, bias by panel class, act per row
  // GEMM, residual added at the tail.
  const int64_t mg = m / group, kk = cg * kh * kw;
  parallel_for(n * group * oh, [&](int64_t u0, int64_t u1) {
    std::vector<float> bmat(kk * ow);
    std::vector<float> crow(mg * ow);
    for (int64_t u = u0; u < u1; ++u) {
      const int64_t oy = u % oh, g = (u / oh) % group, bn = u / (oh * group);
      const float* xg = x + (bn * c + g * cg) * h * wd;
      for (int64_t ch = 0; ch < cg; ++ch)
        for (int64_t ky = 0; ky < kh; ++ky) {
          const int64_t iy = oy * sh - ph + ky;
          for (int64_t kx = 0; kx < kw; ++kx) {
            float* dst = &bmat[((ch * kh + ky) * kw + kx) * ow];
            for (int64_t ox = 0; ox < ow; ++ox) {
              const int64_t ix = ox * sw - pw + kx;
              dst[ox] = (iy < 0 || iy >= h || ix < 0 || ix >= wd) ? 0.0f : xg[(ch * h + iy) * wd + ix];
            }
          }
        }
      gemm_panels(w + g * mg * kk, mg, kk, bmat.data(), ow, ow, bias ? bias + g * mg : nullptr,
                  crow.data(), ow);
      for (int64_t mo = 0; mo < mg; ++mo) {
        float* dst = y + ((bn * m + g * mg + mo) * oh + oy) * ow;
        std::memcpy(dst, &crow[mo * ow], sizeof(float) * ow);
        if (ac.kind) apply_act(dst, ow, ac);
      }
    }
  });
  if (residual) {
    const int64_t total = n * m * ohw;
    parallel_for(total, [&](int64_t b, int64_t e) {
      for (int64_t i = b; i < e; ++i) y[i] += residual[i];
    }, 4096);
  }
  return 0;
}

// conv.rs:730-838 convtranspose2d, 2x2 s2 p0 only: each output element is one
// tap; c-ascending fma chain from 0.  Weight layout [C_in, C_out, 2, 2].
int orc_convtranspose2d(const float* x, const int64_t* xs, const float* w, const int64_t* ws,
                        float* y) {
  const int64_t n = xs[0], c = xs[1], h = xs[2], wd = xs[3];
  const int64_t cin = ws[0], m = ws[1];
  if (cin != c || ws[2] != 2 || ws[3] != 2) return -1;
  const int64_t oh = 2 * h, ow = 2 * wd;
  parallel_for(n * m * 2, [&](int64_t u0, int64_t u1) {
    std::vector<float> w0(c), w1(c), a(wd), bb(wd);
    for (int64_t u = u0; u < u1; ++u) {
      const int64_t ky = u % 2, co = (u / 2) % m, bn = u / (2 * m);
      for (int64_t ch = 0; ch < c; ++ch) {
        w0[ch] = w[((ch * m + co) * 4) + ky * 2 + 0];
        w1[ch] = w[((ch * m + co) * 4) + ky * 2 + 1];
      }
      const float* xn = x + bn * c * h * wd;
      float* yo = y + (bn * m + co) * oh * ow;
      for (int64_t iy = 0; iy < h; ++iy) {
        std::fill(a.begin(), a.end(), 0.0f);
        std::fill(bb.begin(), bb.end(), 0.0f);
        for (int64_t ch = 0; ch < c; ++ch) {
          const float* xr = xn + (ch * h + iy) * wd;
          const float wa = w0[ch], wb = w1[ch];
          for (int64_t j = 0; j < wd; ++j) {
            a[j] = std::fma(xr[j], wa, a[j]);
            bb[j] = std::fma(xr[j], wb, bb[j]);
          }
        }
        float* orow = yo + (iy * 2 + ky) * ow;
        for (int64_t j = 0; j < wd; ++j) {
          orow[2 * j] = a[j];
          orow[2 * j + 1] = bb[j];
        }
      }
    }
  });
  return 0;
}

// conv.rs:912-1051 depthwise_nhwc_packed: x [n,h,w,c], wt tap-major [kh*kw, c];
// first tap y = w*x, later taps fma, then + bias; act; + residual.
// params: sh, sw, ph, pw, peh, pew.
void orc_depthwise_nhwc(const float* x, int64_t n, int64_t h, int64_t wd, int64_t c,
                        const float* wt, int64_t kh, int64_t kw, const int32_t* prm,
                        const float* bias, int act, const float* act_c, const float* residual,
                        float* y) {
  const int64_t sh = prm[0], sw = prm[1], ph = prm[2], pw = prm[3], peh = prm[4], pew = prm[5];
  const int64_t oh = (h + ph + peh - kh) / sh + 1, ow = (wd + pw + pew - kw) / sw + 1;
  Act ac;
  ac.kind = act;
  if (act_c) { ac.c1 = act_c[0]; ac.c2 = act_c[1]; ac.c3 = act_c[2]; }
  parallel_for(n * oh, [&](int64_t u0, int64_t u1) {
    for (int64_t u = u0; u < u1; ++u) {
      const int64_t bn = u / oh, oy = u % oh;
      for (int64_t ox = 0; ox < ow; ++ox) {
        float* dst = y + ((bn * oh + oy) * ow + ox) * c;
        for (int64_t t = 0; t < kh * kw; ++t) {
          const int64_t ky = t / kw, kx = t % kw;
          const int64_t iy = oy * sh + ky - ph, ix = ox * sw + kx - pw;
          const bool in = iy >= 0 && iy < h && ix >= 0 && ix < wd;
          const float* src = x + ((bn * h + iy) * wd + ix) * c;
          const float* wtp = wt + t * c;
          for (int64_t ci = 0; ci < c; ++ci) {
            const float xv = in ? src[ci] : 0.0f;
            dst[ci] = (t == 0) ? wtp[ci] * xv : std::fma(wtp[ci], xv, dst[ci]);
          }
        }
        if (bias)
          for (int64_t ci = 0; ci < c; ++ci) dst[ci] += bias[ci];
        if (ac.kind) apply_act(dst, c, ac);
        if (residual) {
          const float* rs = residual + ((bn * oh + oy) * ow + ox) * c;
          for (int64_t ci = 0; ci < c; ++ci) dst[ci] += rs[ci];
        }
      }
    }
  });
}

// conv.rs:856-901 conv1x1_nhwc: Y[R,M] = X[R,K] * Wt[K,M] (no bias in the
// chain), then per row: += bias, act, += residual.
void orc_conv1x1_nhwc(const float* x, const float* wt, int64_t r, int64_t k, int64_t m,
                      const float* bias, int act, const float* act_c, const float* residual,
                      float* y) {
  Act ac;
  ac.kind = act;
  if (act_c) { ac.c1 = act_c[0]; ac.c2 = act_c[1]; ac.c3 = act_c[2]; }
  parallel_for((r + 3) / 4, [&](int64_t g0, int64_t g1) {
    const int64_t r0 = g0 * 4, r1 = std::min(r, g1 * 4);
    gemm_block(x, r, k, wt, m, m, nullptr, y, m, r0, r1, 0, m);
    for (int64_t row = r0; row < r1; ++row) {
      float* s = y + row * m;
      if (bias)
        for (int64_t j = 0; j < m; ++j) s[j] += bias[j];
      if (ac.kind) apply_act(s, m, ac);
      if (residual)
        for (int64_t j = 0; j < m; ++j) s[j] += residual[row * m + j];
    }
  });
}

// shape.rs:700-733 batchnorm (inference): a = scale/sqrt(var+eps);
// b = fma(-mean, a, bias); y = fma(x, a, b).  NCHW, plane = H*W.
void orc_batchnorm(const float* x, int64_t n, int64_t c, int64_t plane, const float* scale,
                   const float* bias, const float* mean, const float* var, float eps, float* y) {
  parallel_for(n * c, [&](int64_t b0, int64_t e0) {
    for (int64_t nc = b0; nc < e0; ++nc) {
      const int64_t ch = nc % c;
      const float a = scale[ch] / std::sqrt(var[ch] + eps);
      const float b = std::fma(-mean[ch], a, bias[ch]);
      for (int64_t i = 0; i < plane; ++i) y[nc * plane + i] = std::fma(x[nc * plane + i], a, b);
    }
  });
}

// shape.rs:510-566 reduce_mean over a contiguous [outer, mid, inner] split,
// f64 accumulation, (s / mid) rounded to f32.
void orc_reduce_mean(const float* x, int64_t outer, int64_t mid, int64_t inner, float* out) {
  parallel_for(outer * inner, [&](int64_t b, int64_t e) {
    for (int64_t lin = b; lin < e; ++lin) {
      const int64_t o = lin / inner, i = lin % inner;
      const int64_t base = o * mid * inner + i;
      double s = 0.0;
      for (int64_t mm = 0; mm < mid; ++mm) s += (double)x[base + mm * inner];
      out[lin] = (float)(s / (double)mid);
    }
  }, 64);
}

// pool2d.rs:10-30 global_avg_pool, f64 accumulation.
void orc_global_avg_pool(const float* x, int64_t nc, int64_t plane, float* out) {
  orc_reduce_mean(x, nc, plane, 1, out);
}

// pool2d.rs:51-260 pool2d (max or avg), NCHW.  Average divides by the full
// kernel area (count_include_pad semantics of the reference's generic path).
void orc_pool2d(const float* x, int64_t n, int64_t c, int64_t h, int64_t wd, int64_t kh,
                int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t peh,
                int64_t pew, int max_pool, float* out) {
  const int64_t oh = (h + ph + peh - kh) / sh + 1, ow = (wd + pw + pew - kw) / sw + 1;
  parallel_for(n * c, [&](int64_t b, int64_t e) {
    for (int64_t nc = b; nc < e; ++nc) {
      const float* xp = x + nc * h * wd;
      float* op = out + nc * oh * ow;
      for (int64_t oy = 0; oy < oh; ++oy)
        for (int64_t ox = 0; ox < ow; ++ox) {
          float acc = max_pool ? -INFINITY : 0.0f;
          for (int64_t ky = 0; ky < kh; ++ky)
            for (int64_t kx = 0; kx < kw; ++kx) {
              const int64_t iy = oy * sh - ph + ky, ix = ox * sw - pw + kx;
              if (iy < 0 || iy >= h || ix < 0 || ix >= wd) continue;
              const float v = xp[iy * wd + ix];
              if (max_pool) acc = v > acc ? v : acc;
              else acc += v;
            }
          op[oy * ow + ox] = max_pool ? acc : acc / (float)(kh * kw);
        }
    }
  });
}

// resize.rs:8-57 resize_nearest: iy = (int)((float)oy * H / oh), clamped.
void orc_resize_nearest(const float* x, int64_t nc, int64_t h, int64_t wd, int64_t oh,
                        int64_t ow, float* out) {
  parallel_for(nc, [&](int64_t b, int64_t e) {
    for (int64_t p = b; p < e; ++p)
      for (int64_t oy = 0; oy < oh; ++oy) {
        int64_t iy = std::min<int64_t>((int64_t)((float)oy * (float)h / (float)oh), h - 1);
        for (int64_t ox = 0; ox < ow; ++ox) {
          int64_t ix = std::min<int64_t>((int64_t)((float)ox * (float)wd / (float)ow), wd - 1);
          out[(p * oh + oy) * ow + ox] = x[(p * h + iy) * wd + ix];
        }
      }
  });
}

// elementwise.rs:134-165 mul_add_scale: out = f * g[plane % c] + r (two roundings).
void orc_mul_add_scale(const float* f, const float* g, const float* r, float* out, int64_t planes,
                       int64_t c, int64_t hw) {
  parallel_for(planes, [&](int64_t b, int64_t e) {
    for (int64_t p = b; p < e; ++p) {
      const float gv = g[p % c];
      for (int64_t i = 0; i < hw; ++i) {
        const float prod = f[p * hw + i] * gv;
        out[p * hw + i] = prod + r[p * hw + i];
      }
    }
  });
}

// elementwise.rs:185-420 numpy-broadcast binary op.  Shapes are given
// right-aligned as rank-r arrays of the output rank (1 where broadcast).
// op: 0 add, 1 sub, 2 mul, 3 div, 4 pow.
void orc_binary(const float* a, const int64_t* as, const float* b, const int64_t* bs, int rank,
                int op, float* out) {
  std::vector<int64_t> os(rank), sa(rank), sb(rank);
  int64_t total = 1;
  for (int i = 0; i < rank; ++i) {
    os[i] = std::max(as[i], bs[i]);
    total *= os[i];
  }
  int64_t acc_a = 1, acc_b = 1;
  for (int i = rank - 1; i >= 0; --i) {
    sa[i] = as[i] == 1 ? 0 : acc_a;
    sb[i] = bs[i] == 1 ? 0 : acc_b;
    acc_a *= as[i];
    acc_b *= bs[i];
  }
  parallel_for(total, [&](int64_t s, int64_t e) {
    for (int64_t lin = s; lin < e; ++lin) {
      int64_t rem = lin, ia = 0, ib = 0;
      for (int i = rank - 1; i >= 0; --i) {
        const int64_t idx = rem % os[i];
        rem /= os[i];
        ia += idx * sa[i];
        ib += idx * sb[i];
      }
      const float va = a[ia], vb = b[ib];
      float r;
      switch (op) {
        case 0: r = va + vb; break;
        case 1: r = va - vb; break;
        case 2: r = va * vb; break;
        case 3: r = va / vb; break;
        default: r = std::pow(va, vb); break;
      }
      out[lin] = r;
    }
  }, 4096);
}

// shape.rs:568-698 matmul.  A: nbatch x [m,k] (abatch==1 means shared),
// B: nbatch x [k,n] (bbatch==1 means shared).  Large products use the sgemm
// semantics (batch folded into M when B is shared, shape.rs:628-653); small
// ones (attention) the per-row fma outer product from a zeroed row
// (shape.rs:669-697).  `large` selects the branch the reference would take
// (m*n*k >= its gemm_par_min threshold) and is decided by the caller.
void orc_matmul(const float* a, int64_t abatch, const float* b, int64_t bbatch, int64_t nbatch,
                int64_t m, int64_t k, int64_t n, int large, float* out) {
  if (nbatch == 1 || large) {
    if (nbatch > 1 && abatch == nbatch && bbatch == 1) {
      orc_sgemm(a, b, out, nbatch * m, n, k, nullptr, 0, nullptr, nullptr);
      return;
    }
    for (int64_t bi = 0; bi < nbatch; ++bi)
      orc_sgemm(a + (abatch == 1 ? 0 : (bi % abatch) * m * k), k == 0 ? b : b + (bbatch == 1 ? 0 : (bi % bbatch) * k * n),
                out + bi * m * n, m, n, k, nullptr, 0, nullptr, nullptr);
    return;
  }
  parallel_for(nbatch * m, [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t bi = t / m, mm = t % m;
      const float* arow = a + (abatch == 1 ? 0 : (bi % abatch) * m * k) + mm * k;
      const float* bp = b + (bbatch == 1 ? 0 : (bi % bbatch) * k * n);
      float* crow = out + t * n;
      for (int64_t j = 0; j < n; ++j) crow[j] = 0.0f;
      for (int64_t kk = 0; kk < k; ++kk) {
        const float av = arow[kk];
        const float* br = bp + kk * n;
        for (int64_t j = 0; j < n; ++j) crow[j] = std::fma(av, br[j], crow[j]);
      }
    }
  });
}

// rec.rs:34-79 / n_exit3_argmax.comp: per row the first strict maximum
// (ties keep the lowest index); writes (val, idx-as-f32-bit-pattern) pairs.
void orc_argmax_pairs(const float* p, int64_t rows, int64_t cols, float* pairs) {
  parallel_for(rows, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      const float* row = p + r * cols;
      int64_t best = 0;
      float bv = row[0];
      for (int64_t c = 1; c < cols; ++c)
        if (row[c] > bv) { bv = row[c]; best = c; }
      pairs[2 * r] = bv;
      const uint32_t bi = (uint32_t)best;
      std::memcpy(&pairs[2 * r + 1], &bi, 4);
    }
  });
}

// Generic copy-permute for Transpose nodes (shape.rs transpose): out[perm]
// of a row-major tensor.
void orc_transpose(const float* x, const int64_t* shape, const int32_t* perm, int rank, float* out) {
  std::vector<int64_t> in_stride(rank), out_shape(rank);
  int64_t acc = 1, total = 1;
  for (int i = rank - 1; i >= 0; --i) { in_stride[i] = acc; acc *= shape[i]; }
  for (int i = 0; i < rank; ++i) { out_shape[i] = shape[perm[i]]; total *= out_shape[i]; }
  parallel_for(total, [&](int64_t s, int64_t e) {
    for (int64_t lin = s; lin < e; ++lin) {
      int64_t rem = lin, src = 0;
      for (int i = rank - 1; i >= 0; --i) {
        const int64_t idx = rem % out_shape[i];
        rem /= out_shape[i];
        src += idx * in_stride[perm[i]];
      }
      out[lin] = x[src];
    }
  }, 4096);
}

// ------------------------------------------------ det / rec pre and post
// qppocr-kernels resize.rs:158-210 resize_bilinear_rgb_u8 (and its scalar
// reference, tests/rsz_par.rs:5-36): half-pixel source coordinates clamped at
// 0, first term two multiplies, the other three fused multiply-adds, then
// (val + 0.5) clamped to [0, 255] and truncated.  n images of sh x sw x 3.
void orc_resize_bilinear_rgb_u8(const uint8_t* src, int64_t n, int64_t sh, int64_t sw, uint8_t* dst,
                                int64_t dh, int64_t dw) {
  const float sx = (float)sw / (float)dw, sy = (float)sh / (float)dh;
  std::vector<int64_t> x0(dw), x1(dw);
  std::vector<float> fx(dw);
  for (int64_t x = 0; x < dw; ++x) {
    const float v = std::max(((float)x + 0.5f) * sx - 0.5f, 0.0f);
    const int64_t i0 = std::min((int64_t)v, sw - 1);
    x0[x] = i0;
    x1[x] = std::min(i0 + 1, sw - 1);
    fx[x] = v - (float)i0;
  }
  parallel_for(n * dh, [&](int64_t b, int64_t e) {
    for (int64_t ry = b; ry < e; ++ry) {
      const int64_t img = ry / dh, y = ry % dh;
      const float v = std::max(((float)y + 0.5f) * sy - 0.5f, 0.0f);
      const int64_t j0 = std::min((int64_t)v, sh - 1), j1 = std::min(j0 + 1, sh - 1);
      const float fy = v - (float)j0;
      const uint8_t* r0 = src + (img * sh + j0) * sw * 3;
      const uint8_t* r1 = src + (img * sh + j1) * sw * 3;
      uint8_t* out = dst + (img * dh + y) * dw * 3;
      for (int64_t x = 0; x < dw; ++x) {
        const int64_t a = x0[x] * 3, bb = x1[x] * 3;
        const float lx = fx[x];
        for (int ch = 0; ch < 3; ++ch) {
          const float p00 = r0[a + ch], p01 = r0[bb + ch], p10 = r1[a + ch], p11 = r1[bb + ch];
          float t = p00 * (1.0f - lx) * (1.0f - fy);
          t = std::fma(p01 * lx, 1.0f - fy, t);
          t = std::fma(p10 * (1.0f - lx), fy, t);
          const float val = std::fma(p11 * lx, fy, t);
          out[x * 3 + ch] = (uint8_t)std::min(std::max(val + 0.5f, 0.0f), 255.0f);
        }
      }
    }
  }, 16);
}

// crop.rs:153-185 pack_crop into a zeroed [3, img_h, img_w] slot: resize to
// rw x img_h (resize_bilinear_rgb_u8), v = u8 / 255, (v - 0.5) / 0.5 for
// columns < rw; or, pad_only, the crop centred vertically, columns <
// min(w, img_w).
void orc_rec_pack_line(const uint8_t* crop, int64_t h, int64_t w, int64_t rw, int pad, int64_t img_h,
                       int64_t img_w, float* dst) {
  const int64_t plane = img_h * img_w;
  std::fill(dst, dst + 3 * plane, 0.0f);
  auto put = [&](int64_t y, int64_t x, const uint8_t* px) {
    for (int c = 0; c < 3; ++c) {
      const float v = (float)px[c] / 255.0f;
      dst[c * plane + y * img_w + x] = (v - 0.5f) / 0.5f;
    }
  };
  if (pad) {
    const int64_t y0 = (img_h - h) / 2, cols = std::min(w, img_w);
    for (int64_t y = 0; y < h; ++y)
      for (int64_t x = 0; x < cols; ++x) put(y + y0, x, crop + (y * w + x) * 3);
    return;
  }
  std::vector<uint8_t> r((size_t)(img_h * rw * 3));
  orc_resize_bilinear_rgb_u8(crop, 1, h, w, r.data(), img_h, rw);
  for (int64_t y = 0; y < img_h; ++y)
    for (int64_t x = 0; x < rw; ++x) put(y, x, r.data() + (y * rw + x) * 3);
}

// engine.rs:963-982 det input: v = u8 * (1/255), (v - 0.5) * (1/0.5), HWC ->
// planar CHW.  n images of h x w x 3.
void orc_det_normalize(const uint8_t* src, int64_t n, int64_t h, int64_t w, float* dst) {
  const float scale = 1.0f / 255.0f, mean = 0.5f, istd = 1.0f / 0.5f;
  parallel_for(n * 3 * h, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      const int64_t img = r / (3 * h), c = (r / h) % 3, y = r % h;
      const uint8_t* row = src + (img * h + y) * w * 3;
      float* d = dst + ((img * 3 + c) * h + y) * w;
      for (int64_t x = 0; x < w; ++x) {
        const float v = (float)row[x * 3 + c] * scale;
        d[x] = (v - mean) * istd;
      }
    }
  }, 64);
}

// resize.rs:213-245 dilate2x2_max (cv2.dilate 2x2, anchor (1,1)): out[y][x] =
// max of the in-bounds samples of [y-1, y] x [x-1, x].  n masks of h x w.
void orc_dilate2x2(const uint8_t* m, int64_t n, int64_t h, int64_t w, uint8_t* out) {
  parallel_for(n * h, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      const int64_t img = r / h, y = r % h;
      const uint8_t* cur = m + (img * h + y) * w;
      const uint8_t* up = y > 0 ? cur - w : nullptr;
      uint8_t* o = out + (img * h + y) * w;
      for (int64_t x = 0; x < w; ++x) {
        uint8_t v = cur[x];
        if (x > 0) v = std::max(v, cur[x - 1]);
        if (up) {
          v = std::max(v, up[x]);
          if (x > 0) v = std::max(v, up[x - 1]);
        }
        o[x] = v;
      }
    }
  }, 64);
}

// geometry.rs:286-296 db_postprocess binarize (pred > thresh -> 1), then the
// 2x2 dilation when use_dilation.
void orc_db_mask(const float* pred, int64_t n, int64_t h, int64_t w, float thresh, int dilate,
                 uint8_t* out) {
  std::vector<uint8_t> m((size_t)(n * h * w));
  for (int64_t i = 0; i < n * h * w; ++i) m[i] = pred[i] > thresh ? 1 : 0;
  if (dilate) orc_dilate2x2(m.data(), n, h, w, out);
  else std::memcpy(out, m.data(), m.size());
}

// geometry.rs:221-269 box_score_fast: mean of pred over the quadrilateral
// bpts (x, y pairs) by scan-line even-odd fill (sample at y + 0.5, columns
// ceil(xa - 0.5) .. floor(xb - 0.5)), clipped to the box's integer bounds,
// summed in f64 in row order, left to right.
float orc_box_score_one(const float* pred, int hh, int ww, const float* bpts) {
  float fxmin = 3.40282347e38f, fxmax = -3.40282347e38f, fymin = 3.40282347e38f, fymax = -3.40282347e38f;
  for (int i = 0; i < 4; ++i) {
    fxmin = std::fmin(fxmin, bpts[2 * i]);
    fxmax = std::fmax(fxmax, bpts[2 * i]);
    fymin = std::fmin(fymin, bpts[2 * i + 1]);
    fymax = std::fmax(fymax, bpts[2 * i + 1]);
  }
  auto to_i32 = [](float v) -> int {  // Rust `as i32`: saturating, NaN -> 0
    if (v != v) return 0;
    if (v >= 2147483647.0f) return 2147483647;
    if (v <= -2147483648.0f) return (int)-2147483648LL;
    return (int)v;
  };
  auto clampi = [](int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); };
  const int xmin = clampi(to_i32(std::floor(fxmin)), 0, ww - 1);
  const int xmax = clampi(to_i32(std::ceil(fxmax)), 0, ww - 1);
  const int ymin = clampi(to_i32(std::floor(fymin)), 0, hh - 1);
  const int ymax = clampi(to_i32(std::ceil(fymax)), 0, hh - 1);
  double sum = 0.0;
  int64_t count = 0;
  for (int y = ymin; y <= ymax; ++y) {
    const float sy = (float)y + 0.5f;
    float xs[8];
    int nx = 0;
    for (int i = 0; i < 4; ++i) {
      const float ax = bpts[2 * i], ay = bpts[2 * i + 1];
      const float bx = bpts[2 * ((i + 1) % 4)], by = bpts[2 * ((i + 1) % 4) + 1];
      if ((ay <= sy && by > sy) || (by <= sy && ay > sy)) {
        const float t = (sy - ay) / (by - ay);
        xs[nx++] = ax + t * (bx - ax);
      }
    }
    std::sort(xs, xs + nx);
    for (int i = 0; i + 1 < nx; i += 2) {
      const int xa = to_i32(std::ceil(xs[i] - 0.5f));
      const int xb = to_i32(std::floor(xs[i + 1] - 0.5f));
      for (int x = xa; x <= xb; ++x) {
        if (x < xmin || x > xmax) continue;
        sum += (double)pred[(int64_t)y * ww + x];
        ++count;
      }
    }
  }
  if (count == 0) return 0.0f;
  return (float)(sum / (double)count);
}

void orc_box_scores(const float* pred, int64_t hh, int64_t ww, const float* boxes, const int* img, int64_t n,
                    float* out) {
  for (int64_t k = 0; k < n; ++k)
    out[k] = orc_box_score_one(pred + (int64_t)img[k] * hh * ww, (int)hh, (int)ww, boxes + 8 * k);
}

// crop.rs:8-127 crop_text_box size: cw = max(1, max(|p0 p1|, |p2 p3|) as i32),
// ch = max(1, max(|p0 p3|, |p1 p2|) as i32) with f32 hypot; rotated when
// ch / cw >= 1.5 (the output is then ch wide and cw high).
void orc_crop_size(const float* pts, int* cw, int* ch, int* rotated) {
  auto d = [&](int a, int b) { return std::hypot(pts[2 * a] - pts[2 * b], pts[2 * a + 1] - pts[2 * b + 1]); };
  const float w1 = d(0, 1), w2 = d(2, 3), h1 = d(0, 3), h2 = d(1, 2);
  const float mw = std::fmax(w1, w2), mh = std::fmax(h1, h2);
  *cw = std::max(1, (int)mw);
  *ch = std::max(1, (int)mh);
  *rotated = ((float)*ch / (float)*cw >= 1.5f) ? 1 : 0;
}

// crop.rs:8-127 crop_text_box: homography dst corners (0,0),(cw,0),(cw,ch),
// (0,ch) -> pts by f64 Gauss-Jordan with partial pivoting on the 8 x 9
// system; per output pixel the source point in f64, bilinear with the edge
// replicated (first term two multiplies, then fused multiply-adds), u8 by
// (v + 0.5) clamped and truncated; tall crops rotated clockwise.
// src: h x w x 3 uint8; out: cw * ch * 3 bytes.
void orc_crop_text_box(const uint8_t* src, int h, int w, const float* pts, uint8_t* out) {
  int cw, ch, rot;
  orc_crop_size(pts, &cw, &ch, &rot);
  double a[8][9];
  for (int i = 0; i < 4; ++i) {
    const double dx = (i == 1 || i == 2) ? (double)cw : 0.0;
    const double dy = i >= 2 ? (double)ch : 0.0;
    const double sx = (double)pts[2 * i], sy = (double)pts[2 * i + 1];
    const double r0[9] = {dx, dy, 1.0, 0.0, 0.0, 0.0, -dx * sx, -dy * sx, sx};
    const double r1[9] = {0.0, 0.0, 0.0, dx, dy, 1.0, -dx * sy, -dy * sy, sy};
    for (int c = 0; c < 9; ++c) {
      a[2 * i][c] = r0[c];
      a[2 * i + 1][c] = r1[c];
    }
  }
  for (int col = 0; col < 8; ++col) {
    int piv = col;
    for (int r = col + 1; r < 8; ++r)
      if (std::fabs(a[r][col]) > std::fabs(a[piv][col])) piv = r;
    if (piv != col)
      for (int c = 0; c < 9; ++c) std::swap(a[col][c], a[piv][c]);
    const double dd = a[col][col];
    if (std::fabs(dd) < 1e-12) continue;
    for (int c = col; c < 9; ++c) a[col][c] /= dd;
    for (int r = 0; r < 8; ++r) {
      if (r == col) continue;
      const double f = a[r][col];
      if (f == 0.0) continue;
      for (int c = col; c < 9; ++c) a[r][c] -= f * a[col][c];
    }
  }
  double hm[9];
  for (int i = 0; i < 8; ++i) hm[i] = a[i][8];
  hm[8] = 1.0;
  auto to_i32 = [](double v) -> int {
    if (v != v) return 0;
    if (v >= 2147483647.0) return 2147483647;
    if (v <= -2147483648.0) return (int)-2147483648LL;
    return (int)v;
  };
  for (int y = 0; y < ch; ++y)
    for (int x = 0; x < cw; ++x) {
      const double xf = (double)x, yf = (double)y;
      const double den = hm[6] * xf + hm[7] * yf + hm[8];
      const double sx = (hm[0] * xf + hm[1] * yf + hm[2]) / den;
      const double sy = (hm[3] * xf + hm[4] * yf + hm[5]) / den;
      int ix = to_i32(std::floor(sx));
      int iy = to_i32(std::floor(sy));
      const float fx = (float)(sx - (double)ix);
      const float fy = (float)(sy - (double)iy);
      ix = std::min(std::max(ix, 0), w - 1);
      iy = std::min(std::max(iy, 0), h - 1);
      const int ix1 = std::min(ix + 1, w - 1), iy1 = std::min(iy + 1, h - 1);
      const uint8_t* r0 = src + (int64_t)iy * w * 3;
      const uint8_t* r1 = src + (int64_t)iy1 * w * 3;
      const int64_t o = rot ? ((int64_t)x * ch + (ch - 1 - y)) * 3 : ((int64_t)y * cw + x) * 3;
      for (int c = 0; c < 3; ++c) {
        const float v00 = r0[ix * 3 + c], v01 = r0[ix1 * 3 + c], v10 = r1[ix * 3 + c], v11 = r1[ix1 * 3 + c];
        float t = v00 * (1.0f - fx) * (1.0f - fy);
        t = std::fma(v01 * fx, 1.0f - fy, t);
        t = std::fma(v10 * (1.0f - fx), fy, t);
        const float v = std::fma(v11 * fx, fy, t);
        out[o + c] = (uint8_t)std::min(std::max(v + 0.5f, 0.0f), 255.0f);
      }
    }
}

// crop.rs:193-218 cls_view then crop.rs:153-185 pack_crop (resize, never
// pad_only) into a zeroed [3, cls_h, cls_w] slot: crops wider than
// h * cls_w / cls_h (i64) are cut to that many centred columns first.
void orc_cls_pack_line(const uint8_t* crop, int64_t h, int64_t w, int64_t cls_h, int64_t cls_w, float* dst) {
  int64_t x0 = 0, ww = w;
  if (h > 0 && w > 0) {
    const int64_t max_w = h * cls_w / cls_h;
    if (w > max_w) {
      ww = std::max<int64_t>(1, max_w);
      x0 = (w - ww) / 2;
    }
  }
  std::vector<uint8_t> view((size_t)(h * ww * 3));
  for (int64_t y = 0; y < h; ++y) std::memcpy(&view[y * ww * 3], crop + (y * w + x0) * 3, ww * 3);
  const float ratio = (float)ww / (float)h;
  int64_t rw = (int64_t)std::ceil((float)cls_h * ratio);
  rw = std::max<int64_t>(std::min(rw, cls_w), 1);
  orc_rec_pack_line(view.data(), h, ww, rw, 0, cls_h, cls_w, dst);
}

}  // extern "C"
