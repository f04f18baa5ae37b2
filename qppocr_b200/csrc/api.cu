// extern "C" entry points of libqppocr_cuda.so (declared in
// include/qppocr_cuda.h).  Each converts exceptions into a status code plus
// a thread-local message.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>

#include "kernels.h"
#include "session.h"
#include "host_copy.h"

using namespace qpc;

namespace {

template <class F>
int guarded(F&& f) {
  try {
    set_error("");
    return f();
  } catch (GraphError& e) {
    set_error("graph: " + e.msg);
    return E_GRAPH;
  } catch (DeviceError& e) {
    set_error("device: " + e.msg);
    return E_DEVICE;
  } catch (OomError& e) {
    set_error("out of memory: " + e.msg);
    return E_OOM;
  } catch (std::bad_alloc&) {
    set_error("host allocation failed");
    return E_OOM;
  } catch (std::exception& e) {
    set_error(std::string("internal: ") + e.what());
    return E_DEVICE;
  }
}

ActParams act_from(int act, const float* p) {
  ActParams a{};
  a.kind = act;
  a.alpha = p ? p[0] : 1.0f / 6.0f;
  a.beta = p ? p[1] : 0.5f;
  a.c1 = p ? p[2] : 1.4142135f;
  a.c2 = p ? p[3] : 1.0f;
  a.c3 = p ? p[4] : 0.5f;
  return a;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

__global__ void split_tf32_kernel(const float* v, int64_t n, float* hi, float* lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = v[i];
    const float h = tf32_rna(x);
    hi[i] = h;
    lo[i] = tf32_rna(__fsub_rn(x, h));
  }
}

}  // namespace

extern "C" {

const char* qpc_last_error(void) { return last_error().c_str(); }

int qpc_device_count(int* count) {
  if (!count) return E_INVALID;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    *count = 0;
    return OK;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(std::string("device: cudaGetDeviceCount: ") + cudaGetErrorString(e));
    *count = 0;
    return E_DEVICE;
  }
  *count = n;
  return OK;
}

int qpc_device_info(int device, char* name, int name_len, int* driver_version, int* cc_major,
                    int* cc_minor) {
  return guarded([&] {
    int n = 0;
    if (qpc_device_count(&n) != OK) return (int)E_DEVICE;
    if (device < 0 || device >= n)
      throw DeviceError{"cuda:" + std::to_string(device) + " out of range (" + std::to_string(n) +
                        " CUDA devices)"};
    cudaDeviceProp p;
    QPC_CUDA_OR_THROW(cudaGetDeviceProperties(&p, device));
    if (name && name_len > 0) {
      std::strncpy(name, p.name, name_len - 1);
      name[name_len - 1] = 0;
    }
    if (driver_version) QPC_CUDA_OR_THROW(cudaDriverGetVersion(driver_version));
    if (cc_major) *cc_major = p.major;
    if (cc_minor) *cc_minor = p.minor;
    if (p.major != 10)
      throw DeviceError{std::string(p.name) + " is sm_" + std::to_string(p.major) +
                        std::to_string(p.minor) + "; this library carries sm_100a code only"};
    return (int)OK;
  });
}

int qpc_session_create(int device, const qpc_graph* graph, const qpc_tensor* weights,
                       int n_weights, int role, const qpc_session_options* opts,
                       qpc_session** out) {
  if (!graph || !out || (n_weights && !weights)) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    auto s = new qpc_session;
    try {
      s->impl = std::make_unique<Session>(device, graph, weights, n_weights, role, opts);
    } catch (...) {
      delete s;
      throw;
    }
    *out = s;
    return (int)OK;
  });
}

int qpc_session_caps(const qpc_session* s, qpc_caps* caps) {
  if (!s || !caps) return E_INVALID;
  *caps = s->impl->caps();
  return OK;
}

int qpc_run_async(qpc_session* s, const qpc_tensor* inputs, int n_inputs, qpc_ticket** ticket) {
  if (!s || !ticket || (n_inputs && !inputs)) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    PlanInstance* p = s->impl->launch(inputs, n_inputs);
    auto t = new qpc_ticket;
    t->session = s->impl.get();
    t->plan = p;
    *ticket = t;
    return (int)OK;
  });
}

int qpc_complete(qpc_ticket* t, int timeout_ms) {
  if (!t || !t->plan) return E_INVALID;
  if (t->completed) return OK;
  return guarded([&] {
    QPC_CUDA_OR_THROW(cudaSetDevice(t->session->device()));
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
      cudaError_t e = cudaEventQuery(t->plan->ev[3]);
      if (e == cudaSuccess) break;
      if (e != cudaErrorNotReady) throw DeviceError{std::string("run failed: ") + cudaGetErrorString(e)};
      if (timeout_ms >= 0 && std::chrono::steady_clock::now() > deadline) {
        set_error("device: run not complete after " + std::to_string(timeout_ms) + " ms");
        return (int)E_TIMEOUT;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    if (unsigned kerr = take_kernel_error(t->session->device()))
      throw DeviceError{"kernel pipeline wait timed out (flags " + std::to_string(kerr) + ")"};
    float ms = 0.f;
    cudaEventElapsedTime(&ms, t->plan->ev[1], t->plan->ev[2]);
    t->device_ms = ms;
    t->completed = true;
    return (int)OK;
  });
}

int qpc_ticket_output_count(const qpc_ticket* t, int* count) {
  if (!t || !t->plan || !count) return E_INVALID;
  *count = (int)t->plan->outs.size();
  return OK;
}

int qpc_ticket_output(const qpc_ticket* t, int index, const float** data, const int64_t** shape,
                      int* rank) {
  if (!t || !t->plan || index < 0 || index >= (int)t->plan->outs.size()) return E_INVALID;
  if (!t->completed) {
    set_error("ticket not completed");
    return E_INVALID;
  }
  const auto& io = t->plan->outs[index];
  if (data) *data = io.host;
  if (shape) *shape = io.shape.data();
  if (rank) *rank = (int)io.shape.size();
  return OK;
}

int qpc_ticket_output_copy(const qpc_ticket* t, int index, float* dst, int64_t count) {
  if (!t || !t->plan || !dst || index < 0 || index >= (int)t->plan->outs.size()) return E_INVALID;
  if (!t->completed) {
    set_error("ticket not completed");
    return E_INVALID;
  }
  const auto& io = t->plan->outs[index];
  if (io.device_only) {
    set_error("output " + std::to_string(index) + " stays in device memory (qpc_ticket_output_info)");
    return E_INVALID;
  }
  if (count != io.count) {
    set_error("output " + std::to_string(index) + " has " + std::to_string(io.count) + " elements, not " +
              std::to_string(count));
    return E_INVALID;
  }
  qpc::parallel_copy(dst, io.host, io.bytes);
  return OK;
}

int qpc_ticket_output_info(const qpc_ticket* t, int index, int* dtype, int* device_only,
                           const void** device_data) {
  if (!t || !t->plan || index < 0 || index >= (int)t->plan->outs.size()) return E_INVALID;
  if (!t->completed) {
    set_error("ticket not completed");
    return E_INVALID;
  }
  const auto& io = t->plan->outs[index];
  if (dtype) *dtype = io.dtype;
  if (device_only) *device_only = io.device_only ? 1 : 0;
  if (device_data) *device_data = io.dev;
  return OK;
}

int qpc_ticket_device_ms(const qpc_ticket* t, float* ms) {
  if (!t || !ms || !t->completed) return E_INVALID;
  *ms = t->device_ms;
  return OK;
}

int qpc_host_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes < 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  void* p = pinned_alloc((size_t)bytes);
  if (!p) {
    set_error("pinned host allocation of " + std::to_string(bytes) + " bytes failed");
    return E_OOM;
  }
  *ptr = p;
  return OK;
}

int qpc_host_free(void* ptr) {
  if (!ptr) return OK;
  if (!pinned_free(ptr)) {
    set_error("not a qpc_host_alloc block");
    return E_INVALID;
  }
  return OK;
}

int qpc_ticket_release(qpc_ticket* t) {
  if (!t) return E_INVALID;
  if (t->plan && !t->completed) {
    // never hand a plan back while its run may still be writing
    cudaSetDevice(t->session->device());
    cudaEventSynchronize(t->plan->ev[3]);
  }
  if (t->session) t->session->release(t->plan);
  delete t;
  return OK;
}

int qpc_run(qpc_session* s, const qpc_tensor* inputs, int n_inputs, qpc_ticket** ticket) {
  int st = qpc_run_async(s, inputs, n_inputs, ticket);
  if (st != OK) return st;
  st = qpc_complete(*ticket, -1);
  if (st != OK) {
    std::string msg = last_error();
    qpc_ticket_release(*ticket);
    *ticket = nullptr;
    set_error(msg);
  }
  return st;
}

int qpc_session_destroy(qpc_session* s) {
  if (!s) return E_INVALID;
  return guarded([&] {
    delete s;
    return (int)OK;
  });
}

// ---- diagnostics (QPPOCR_GPU_PROF analogue, vulkan/session.rs:828-835, 2073-2139)
int qpc_session_profile(qpc_session* s, const qpc_tensor* inputs, int n_inputs, int iters,
                        int* n_steps) {
  if (!s || !n_steps) return E_INVALID;
  return guarded([&] {
    s->impl->profile(inputs, n_inputs, iters);
    *n_steps = (int)s->impl->profile_steps().size();
    return (int)OK;
  });
}

int qpc_session_profile_step(const qpc_session* s, int idx, const char** kernel, const char** node,
                             double* bytes, double* flops, float* ms) {
  if (!s) return E_INVALID;
  const auto& v = s->impl->profile_steps();
  if (idx < 0 || idx >= (int)v.size()) return E_INVALID;
  if (kernel) *kernel = v[idx].kernel.c_str();
  if (node) *node = v[idx].node.c_str();
  if (bytes) *bytes = v[idx].bytes;
  if (flops) *flops = v[idx].flops;
  if (ms) *ms = v[idx].ms;
  return OK;
}

int qpc_session_replay(qpc_session* s, const qpc_tensor* inputs, int n_inputs, int iters,
                       float* ms_per_replay) {
  if (!s || !ms_per_replay) return E_INVALID;
  return guarded([&] {
    *ms_per_replay = s->impl->replay(inputs, n_inputs, iters);
    return (int)OK;
  });
}

// Fused plan nodes (after load-time fusion), for per-node dump-compare
// (QPPOCR_GPU_DUMP_CMP analogue, vulkan/session.rs:542-600).
int qpc_session_node_count(const qpc_session* s, int* n) {
  if (!s || !n) return E_INVALID;
  *n = (int)s->impl->nodes().size();
  return OK;
}

int qpc_session_node(const qpc_session* s, int idx, const char** op, const char** name,
                     const char** output) {
  if (!s) return E_INVALID;
  const auto& v = s->impl->nodes();
  if (idx < 0 || idx >= (int)v.size()) return E_INVALID;
  if (op) *op = v[idx].op.c_str();
  if (name) *name = v[idx].name.c_str();
  if (output) *output = v[idx].out.empty() ? "" : v[idx].out[0].c_str();
  return OK;
}

// ---- operator entry points
int qpc_op_dwconv_nhwc(const float* x, int n, int h, int w, int c, const float* w_tap_major,
                       int kh, int kw, const int* strides, const int* pads, const float* bias,
                       int act, const float* act_p, const float* residual, float* y,
                       void* stream) {
  if (!x || !w_tap_major || !y || !strides || !pads || n <= 0 || c <= 0 || kh <= 0 || kw <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    ConvGeom g{};
    g.n = n; g.h = h; g.w = w; g.c = c; g.m = c;
    g.kh = kh; g.kw = kw; g.sh = strides[0]; g.sw = strides[1];
    g.ph = pads[0]; g.pw = pads[1];
    g.oh = (h + pads[0] + pads[2] - kh) / g.sh + 1;
    g.ow = (w + pads[1] + pads[3] - kw) / g.sw + 1;
    if (g.oh <= 0 || g.ow <= 0) throw GraphError{"dwconv: empty output"};
    unsigned int* err = device_state(current_device()).err_word;
    QPC_CUDA_OR_THROW(launch_dwconv_nhwc(x, w_tap_major, bias, residual, y, g, act_from(act, act_p),
                                         (cudaStream_t)stream, err));
    return (int)OK;
  });
}

int qpc_op_gemm(const float* x, int64_t m, int k, const float* w, const float* w_lo, int n,
                const float* bias, int act, const float* act_p, const float* residual, float* y,
                int math, void* stream) {
  if (!x || !w || !y || m < 0 || k <= 0 || n <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    if (k % 4) throw GraphError{"gemm: K must be a multiple of 4 (16-byte TMA row pitch)"};
    if (math == QPC_MATH_3XTF32 && !w_lo) throw GraphError{"gemm: 3xTF32 needs w_lo"};
    GemmEpilogue e;
    e.bias = bias;
    e.residual = residual;
    e.out = y;
    e.ldo = n;
    e.ldr = n;
    e.act = act_from(act, act_p);
    unsigned int* err = device_state(current_device()).err_word;
    QPC_CUDA_OR_THROW(launch_gemm_tc(x, m, k, k, w, w_lo, n, e, math, err, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_ctc_head(const float* x, int64_t rows, int k, const float* w, const float* w_lo, int n,
                    const float* bias, int math, float* pairs, void* stream) {
  if (!x || !w || !pairs || rows < 0 || k <= 0 || n <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    if (k % 4) throw GraphError{"ctc head: K must be a multiple of 4 (16-byte TMA row pitch)"};
    if (math == QPC_MATH_3XTF32 && !w_lo) throw GraphError{"ctc head: 3xTF32 needs w_lo"};
    if (rows == 0) return (int)OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int ntiles = gemm_tc_col_tiles(n, math);
    void* part = nullptr;
    if (alloc_failure_due()) throw OomError{"cudaMallocAsync(ctc head partials): out of memory (injected)"};
    cudaError_t ae = cudaMallocAsync(&part, (size_t)ntiles * rows * sizeof(float4), st);
    if (ae == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      throw OomError{"cudaMallocAsync(ctc head partials): out of memory"};
    }
    QPC_CUDA_OR_THROW(ae);
    GemmEpilogue e;
    e.bias = bias;
    e.partials = static_cast<float4*>(part);
    e.ldo = n;
    unsigned int* err = device_state(current_device()).err_word;
    cudaError_t le = launch_gemm_tc(x, rows, k, k, w, w_lo, n, e, math, err, st);
    if (le == cudaSuccess) le = launch_argmax_combine(static_cast<float4*>(part), ntiles, rows, math, pairs, st);
    cudaFreeAsync(part, st);
    QPC_CUDA_OR_THROW(le);
    return (int)OK;
  });
}

int qpc_op_split_tf32(const float* v, int64_t count, float* hi, float* lo, void* stream) {
  if (!v || !hi || !lo || count < 0) return E_INVALID;
  return guarded([&] {
    int64_t blocks = (count + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    split_tf32_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(v, count, hi, lo);
    QPC_CUDA_OR_THROW(cudaGetLastError());
    return (int)OK;
  });
}

int qpc_op_resize_bilinear_rgb_u8(const uint8_t* src, int n, int sh, int sw, uint8_t* dst, int dh, int dw,
                                  void* stream) {
  if (!src || !dst || n < 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_resize_bilinear_rgb_u8(src, n, sh, sw, dst, dh, dw, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_det_preprocess(const uint8_t* src, int n, int sh, int sw, float* dst, int dh, int dw, void* stream) {
  if (!src || !dst || n < 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_det_preprocess(src, n, sh, sw, dst, dh, dw, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_rec_pack(const uint8_t* crops, const int64_t* off, const int* h, const int* w, const int* rw,
                    const int* pad, int n, int img_h, int img_w, float* out, void* stream) {
  if (!crops || !off || !h || !w || !rw || !pad || !out || n < 0 || n > 65535 || img_h <= 0 || img_w <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_rec_pack(crops, off, h, w, rw, pad, n, img_h, img_w, out, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_db_mask(const float* pred, const uint8_t* mask_in, uint8_t* mask, int n, int h, int w, float thresh,
                   int dilate, void* stream) {
  if ((!pred && !mask_in) || !mask || n < 0 || h <= 0 || w <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_db_mask(pred, mask_in, mask, n, h, w, thresh, dilate, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_box_score(const float* pred, int h, int w, const float* boxes, const int* img, int n_boxes,
                     float* scores, void* stream) {
  if (!pred || (n_boxes && (!boxes || !img || !scores)) || n_boxes < 0 || h <= 0 || w <= 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_box_score(pred, h, w, boxes, img, n_boxes, scores, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_crop_size(const float* pts, int n, int* cw, int* ch, int* rotated) {
  if ((n && (!pts || !cw || !ch || !rotated)) || n < 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  for (int k = 0; k < n; ++k) {
    const float* p = pts + 8 * (int64_t)k;
    auto d = [&](int a, int b) { return std::hypot(p[2 * a] - p[2 * b], p[2 * a + 1] - p[2 * b + 1]); };
    const float mw = std::fmax(d(0, 1), d(2, 3)), mh = std::fmax(d(0, 3), d(1, 2));
    if (!(mw < 2147483647.0f) || !(mh < 2147483647.0f)) {
      set_error("box " + std::to_string(k) + ": corners are not finite or too far apart");
      return E_INVALID;
    }
    cw[k] = std::max(1, (int)mw);
    ch[k] = std::max(1, (int)mh);
    rotated[k] = ((float)ch[k] / (float)cw[k] >= 1.5f) ? 1 : 0;
  }
  return OK;
}

int qpc_op_crop_text_boxes(const uint8_t* images, int n_images, int h, int w, const float* pts, const int* img,
                           const int* cw, const int* ch, const int64_t* off, int n_boxes, int max_pixels,
                           uint8_t* out, void* stream) {
  if (!images || n_images <= 0 || h <= 0 || w <= 0 || n_boxes < 0 || n_boxes > 65535 ||
      (n_boxes && (!pts || !img || !cw || !ch || !off || !out || max_pixels <= 0))) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    QPC_CUDA_OR_THROW(launch_crop_boxes(images, h, w, pts, img, cw, ch, off, n_boxes, max_pixels, out,
                                        (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_op_line_pack(const uint8_t* crops, const int64_t* off, const int* stride, const int* x0, const int* h,
                     const int* w, const int* rw, const int* pad, const int* flip, int n, int img_h, int img_w,
                     float* out, void* stream) {
  if (n < 0 || n > 65535 || img_h <= 0 || img_w <= 0 ||
      (n && (!crops || !off || !stride || !x0 || !h || !w || !rw || !pad || !out))) {
    set_error("invalid argument");
    return E_INVALID;
  }
  return guarded([&] {
    LinePack lp{off, stride, x0, h, w, rw, pad, flip};
    QPC_CUDA_OR_THROW(launch_line_pack(crops, lp, n, img_h, img_w, out, (cudaStream_t)stream));
    return (int)OK;
  });
}

int qpc_selftest_wait_timeout(int device, int path, int limit_us) {
  if (path < 0 || path > 1 || limit_us < 1 || limit_us > 1000000) {
    set_error("invalid argument (path 0 or 1, limit_us in [1, 1e6])");
    return E_INVALID;
  }
  return guarded([&] {
    DeviceState& ds = device_state(device);
    cudaStream_t st = nullptr;
    QPC_CUDA_OR_THROW(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    const uint64_t ns = (uint64_t)limit_us * 1000ull;
    cudaError_t e = path == 0 ? launch_wait_selftest(ds.err_word, ns, st) : noalloc_head_selftest(ns, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaStreamDestroy(st);
    QPC_CUDA_OR_THROW(e);
    return (int)OK;
  });
}

int qpc_inject_alloc_failure(int nth) {
  if (nth < 0) {
    set_error("invalid argument");
    return E_INVALID;
  }
  inject_alloc_failure(nth);
  return OK;
}

int qpc_kernel_error(int device, unsigned int* flags) {
  if (!flags) return E_INVALID;
  return guarded([&] {
    *flags = take_kernel_error(device);
    return (int)OK;
  });
}

}  // extern "C"
