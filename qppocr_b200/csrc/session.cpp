// Session runtime: graph import, load-time fusion, per-shape planning over
// strided device views, liveness-based arena reuse, CUDA-graph capture and
// deferred runs.
//
// Reference behaviour this follows:
//  * DeviceContext::create_session / DeviceSession::run / run_deferred
//    (crates/qppocr-core/src/device.rs:83-176): weights resident for the
//    session's lifetime, unsupported ops rejected at create time naming the
//    node, outputs in graph-output order, two same-shape runs in flight never
//    share buffers (the Vulkan backend's shadow plans,
//    crates/qppocr-gpu/src/vulkan/session.rs:291-352).
//  * Per-shape plan cache with a byte budget and oldest-first eviction
//    (vulkan/session.rs:369-395); here each plan is one captured CUDA graph.
//  * Op semantics: crates/qppocr-core/src/executor.rs:433-1580 (cited per op
//    below); fused epilogue order bias -> act -> residual
//    (crates/qppocr-core/src/graph/optimize.rs:337-770).
#include "session.h"
#include "host_copy.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <set>
#include <sstream>
#include <thread>
#include <tuple>

#include "kernels.h"
#include "misc.h"

namespace qpc {

// The plan-level type of a run input: device-resident f32 / u8 images use
// the same plans as their host forms (only the upload differs).
static int base_dtype(int d) {
  return d == QPC_F32_DEVICE ? QPC_F32 : (d == QPC_U8_IMAGE_DEVICE ? QPC_U8_IMAGE : d);
}

// ================================================================ runtime
static thread_local std::string g_err;
void set_error(const std::string& m) { g_err = m; }
const std::string& last_error() { return g_err; }

static std::atomic<int> g_alloc_fail_countdown{0};
void inject_alloc_failure(int nth) { g_alloc_fail_countdown.store(nth > 0 ? nth : 0); }
bool alloc_failure_due() {
  int v = g_alloc_fail_countdown.load();
  while (v > 0) {
    if (g_alloc_fail_countdown.compare_exchange_weak(v, v - 1)) return v == 1;
  }
  return false;
}

DevBuf::DevBuf(size_t n) : bytes(n) {
  if (n) {
    if (alloc_failure_due())
      throw OomError{"cudaMalloc(" + std::to_string(n) + " bytes): out of memory (injected)"};
    cudaError_t e = cudaMalloc(&ptr, n);
    if (e != cudaSuccess) {
      ptr = nullptr;
      cudaGetLastError();
      const std::string m = "cudaMalloc(" + std::to_string(n) + " bytes): " + cudaGetErrorString(e);
      if (e == cudaErrorMemoryAllocation) throw OomError{m};
      throw DeviceError{m};
    }
  }
}
DevBuf::~DevBuf() {
  if (ptr) cudaFree(ptr);
}

static std::mutex g_dev_mu;
static std::map<int, DeviceState> g_devs;

DeviceState& device_state(int d) {
  QPC_CUDA_OR_THROW(cudaSetDevice(d));
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& s = g_devs[d];
  if (!s.err_word) {
    s.device = d;
    QPC_CUDA_OR_THROW(cudaMalloc(&s.err_word, sizeof(unsigned int)));
    QPC_CUDA_OR_THROW(cudaMemset(s.err_word, 0, sizeof(unsigned int)));
  }
  return s;
}

unsigned int take_kernel_error(int d) {
  DeviceState& s = device_state(d);
  unsigned int v = 0;
  QPC_CUDA_OR_THROW(cudaMemcpy(&v, s.err_word, sizeof(v), cudaMemcpyDeviceToHost));
  if (v) QPC_CUDA_OR_THROW(cudaMemset(s.err_word, 0, sizeof(v)));
  return v | take_noalloc_head_error(d);
}

// ---- per-device launch configuration
namespace {
std::mutex g_launch_mu;
std::map<std::pair<int, const void*>, int> g_dyn_smem;           // (device, kernel) -> bytes set
std::map<std::tuple<int, const void*, int, int>, int> g_occupancy;  // (device, kernel, threads, smem)
std::map<int, int> g_sms;
int current_dev() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
}  // namespace

cudaError_t ensure_dyn_smem(const void* func, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  const int d = current_dev();
  std::lock_guard<std::mutex> lk(g_launch_mu);
  int& set = g_dyn_smem[{d, func}];
  if (bytes > set) {
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    set = bytes;
  }
  return cudaSuccess;
}

int current_sm_count() {
  const int d = current_dev();
  std::lock_guard<std::mutex> lk(g_launch_mu);
  auto it = g_sms.find(d);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148;
  }
  g_sms[d] = n;
  return n;
}

int blocks_per_sm(const void* func, int threads, int smem) {
  const int d = current_dev();
  std::lock_guard<std::mutex> lk(g_launch_mu);
  auto key = std::make_tuple(d, func, threads, smem);
  auto it = g_occupancy.find(key);
  if (it != g_occupancy.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, func, threads, smem) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  g_occupancy[key] = per_sm;
  return per_sm;
}

// ================================================================ IR
const Attr* Node::attr(const std::string& n) const {
  for (auto& a : attrs)
    if (a.name == n) return &a;
  return nullptr;
}
int64_t Node::geti(const std::string& n, int64_t d) const {
  const Attr* a = attr(n);
  return (a && a->kind == QPC_ATTR_INT) ? a->i : d;
}
float Node::getf(const std::string& n, float d) const {
  const Attr* a = attr(n);
  return (a && a->kind == QPC_ATTR_FLOAT) ? a->f : d;
}
std::string Node::gets(const std::string& n, const std::string& d) const {
  const Attr* a = attr(n);
  return (a && a->kind == QPC_ATTR_STRING) ? a->s : d;
}
std::vector<int64_t> Node::getints(const std::string& n) const {
  const Attr* a = attr(n);
  return (a && a->kind == QPC_ATTR_INTS) ? a->ints : std::vector<int64_t>{};
}
void Node::seti(const std::string& n, int64_t v) {
  for (auto& a : attrs)
    if (a.name == n) { a.kind = QPC_ATTR_INT; a.i = v; return; }
  Attr a;
  a.name = n;
  a.kind = QPC_ATTR_INT;
  a.i = v;
  attrs.push_back(a);
}
void Node::setf(const std::string& n, float v) {
  for (auto& a : attrs)
    if (a.name == n) { a.kind = QPC_ATTR_FLOAT; a.f = v; return; }
  Attr a;
  a.name = n;
  a.kind = QPC_ATTR_FLOAT;
  a.f = v;
  attrs.push_back(a);
}

static std::string shape_str(const std::vector<int64_t>& s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? "," : "") << s[i];
  o << "]";
  return o.str();
}

PlanInstance::~PlanInstance() {
  if (exec) cudaGraphExecDestroy(exec);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  if (stream) cudaStreamDestroy(stream);
  for (auto& io : ins)
    if (io.host) cudaFreeHost(io.host);
  for (auto& io : outs)
    if (io.host) cudaFreeHost(io.host);
}

// ================================================================ session
static const std::set<std::string>& supported_ops() {
  static const std::set<std::string> ops = {
      "Conv", "ConvTranspose", "BatchNormalization", "Relu", "Sigmoid", "HardSigmoid",
      "FusedGelu", "Erf", "Sqrt", "Clip", "MulAddScale", "Add", "Sub", "Mul", "Div", "Pow",
      "Softmax", "GlobalAveragePool", "AveragePool", "MaxPool", "Resize", "Concat", "Slice",
      "Transpose", "Reshape", "Squeeze", "Unsqueeze", "Flatten", "ReduceMean", "MatMul",
      "Identity", "Dropout", "Gather", "Shape", "Cast",
      // internal (produced by Session::fuse)
      "QpcLinear", "QpcConvT", "QpcConvTPair", "QpcLayerNorm", "QpcCtcHead", "QpcAttention"};
  return ops;
}

Session::Session(int device, const qpc_graph* g, const qpc_tensor* w, int nw, int role,
                 const qpc_session_options* opts)
    : device_(device), role_(role) {
  opts_.math = QPC_MATH_TF32;
  opts_.argmax_exit = -1;
  opts_.plan_budget_bytes = 0;
  opts_.use_cuda_graph = 1;
  opts_.det_mask_exit = 0;
  opts_.mask_thresh = 0.3f;
  opts_.mask_dilate = 1;
  if (opts) opts_ = *opts;
  if (opts_.det_mask_exit && role != QPC_ROLE_DET) throw GraphError{"det_mask_exit needs the det role"};
  if (opts_.plan_budget_bytes <= 0) {
    // a quarter of the device's memory: room for two in-flight instances of
    // a large shape (a 960 x 960 det plan at batch 64 holds ~4.5 GB) plus
    // the other shapes, without evicting the instance the next run needs
    size_t free_b = 0, total_b = 0;
    QPC_CUDA_OR_THROW(cudaSetDevice(device));
    QPC_CUDA_OR_THROW(cudaMemGetInfo(&free_b, &total_b));
    opts_.plan_budget_bytes = std::max<int64_t>((int64_t)8 << 30, (int64_t)(total_b / 4));
  }
  argmax_exit_ = opts_.argmax_exit < 0 ? (role == QPC_ROLE_REC) : (opts_.argmax_exit != 0);
  device_state(device_);
  for (int k = 0; k < g->n_nodes; ++k) {
    const qpc_node& qn = g->nodes[k];
    Node n;
    n.op = qn.op_type ? qn.op_type : "";
    n.name = qn.name ? qn.name : ("node" + std::to_string(k));
    for (int j = 0; j < qn.n_inputs; ++j) n.in.push_back(qn.inputs[j] ? qn.inputs[j] : "");
    for (int j = 0; j < qn.n_outputs; ++j) n.out.push_back(qn.outputs[j] ? qn.outputs[j] : "");
    for (int j = 0; j < qn.n_attrs; ++j) {
      const qpc_attr& qa = qn.attrs[j];
      Attr a;
      a.name = qa.name ? qa.name : "";
      a.kind = qa.kind;
      a.f = qa.f;
      a.i = qa.i;
      if (qa.s) a.s = qa.s;
      if (qa.kind == QPC_ATTR_FLOATS && qa.floats) a.floats.assign(qa.floats, qa.floats + qa.n);
      if (qa.kind == QPC_ATTR_INTS && qa.ints) a.ints.assign(qa.ints, qa.ints + qa.n);
      n.attrs.push_back(std::move(a));
    }
    nodes_.push_back(std::move(n));
  }
  for (int k = 0; k < g->n_inputs; ++k) inputs_.push_back(g->inputs[k]);
  for (int k = 0; k < g->n_outputs; ++k) outputs_.push_back(g->outputs[k]);
  for (int k = 0; k < nw; ++k) {
    const qpc_tensor& t = w[k];
    HostTensor h;
    h.shape.assign(t.shape, t.shape + t.rank);
    h.dtype = t.dtype;
    const int64_t n = h.numel();
    if (t.dtype == QPC_F32) {
      h.f.resize(n);
      if (n) std::memcpy(h.f.data(), t.data, n * sizeof(float));
    } else if (t.dtype == QPC_I64) {
      h.i.resize(n);
      if (n) std::memcpy(h.i.data(), t.data, n * sizeof(int64_t));
    } else {
      throw GraphError{std::string("weight ") + t.name + ": unsupported dtype"};
    }
    weights_[t.name] = std::move(h);
  }
  validate_ops();
  fuse();
}

Session::~Session() {
  cudaSetDevice(device_);
  for (auto& kv : plans_)
    for (auto& p : kv.second)
      if (p->stream) cudaStreamSynchronize(p->stream);
  if (compute_done_) cudaEventDestroy(compute_done_);
}

void Session::validate_ops() const {
  for (const Node& n : nodes_) {
    if (!supported_ops().count(n.op))
      throw GraphError{"unsupported op " + n.op + " (node " + n.name + ")"};
    if (n.op == "Conv") {
      if (!n.has_in(1) || !weights_.count(n.in[1]))
        throw GraphError{"Conv " + n.name + ": weight must be an initializer"};
      for (auto d : n.getints("dilations"))
        if (d != 1) throw GraphError{"Conv " + n.name + ": dilation != 1 unsupported"};
    }
    if (n.op == "ConvTranspose") {
      const HostTensor* w = weight(n.in[1]);
      if (!w || w->shape.size() != 4 || w->shape[2] != 2 || w->shape[3] != 2)
        throw GraphError{"ConvTranspose " + n.name + ": only 2x2 s2 p0 (conv.rs:754-757)"};
    }
    if (n.op == "Resize") {
      const std::string mode = n.gets("mode", "nearest");
      if (mode != "nearest") throw GraphError{"Resize " + n.name + ": mode " + mode + " unsupported"};
    }
  }
}

const HostTensor* Session::weight(const std::string& name) const {
  auto it = weights_.find(name);
  return it == weights_.end() ? nullptr : &it->second;
}

qpc_caps Session::caps() const {
  qpc_caps c;
  c.prefers_host_parallelism = 0;  // GPU executes in parallel internally (device.rs:134)
  c.bucket_grain = 64;             // width buckets collapse rec shapes (device.rs:139-141)
  c.batch_grain = 1;               // batch rows are not padded (device.rs:148-157)
  c.rec_chunk = 256;               // real lines merged per forward
  c.argmax_pairs = argmax_exit_ ? 1 : 0;
  return c;
}

// Device copies of weights, in the layout a kernel wants (built once).
//   raw        as given
//   dw         depthwise [C,1,kh,kw] -> tap-major [kh*kw][C]
//   kxk        dense [M,C,kh,kw] -> tap-major [kh*kw][M][C]
//   kxf        dense [M,C,kh,kw] -> kx-folded [kh][roundup16(kw*M)][C]
//   nk         MatMul B [K,N] -> [N,K]
//   X.rn       variant X rounded to tf32, nearest (TF32-mode B operand)
//   X.hi/X.lo  3xTF32 split of variant X: hi = rn(v), lo = rn(v - hi)
static float tf32_rn_host(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  u = (u + 0x1000u) & 0xFFFFE000u;  // round to nearest, ties away (cvt.rna.tf32.f32)
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

const float* Session::dweight(const std::string& name, const std::string& variant) {
  const std::string key = name + "#" + variant;
  auto it = dev_cache_.find(key);
  if (it != dev_cache_.end()) return it->second->f();
  const HostTensor* h = weight(name);
  if (!h) throw GraphError{"missing initializer " + name};
  std::vector<float> v;
  auto base_variant = variant;
  bool hi = false, lo = false, rn = false;
  if (variant.size() > 3 && variant.compare(variant.size() - 3, 3, ".hi") == 0) {
    hi = true;
    base_variant = variant.substr(0, variant.size() - 3);
  } else if (variant.size() > 3 && variant.compare(variant.size() - 3, 3, ".lo") == 0) {
    lo = true;
    base_variant = variant.substr(0, variant.size() - 3);
  } else if (variant.size() > 3 && variant.compare(variant.size() - 3, 3, ".rn") == 0) {
    rn = true;
    base_variant = variant.substr(0, variant.size() - 3);
  }
  std::vector<float> src;
  if (h->dtype == QPC_F32) src = h->f;
  else {
    src.resize(h->i.size());
    for (size_t k = 0; k < src.size(); ++k) src[k] = (float)h->i[k];
  }
  if (base_variant == "raw") {
    v = src;
  } else if (base_variant == "dw") {
    const int64_t c = h->shape[0], taps = h->shape[2] * h->shape[3];
    v.resize(c * taps);
    for (int64_t ch = 0; ch < c; ++ch)
      for (int64_t t = 0; t < taps; ++t) v[t * c + ch] = src[ch * taps + t];
  } else if (base_variant == "kxk") {
    const int64_t m = h->shape[0], c = h->shape[1], taps = h->shape[2] * h->shape[3];
    v.resize(m * c * taps);
    for (int64_t mo = 0; mo < m; ++mo)
      for (int64_t ch = 0; ch < c; ++ch)
        for (int64_t t = 0; t < taps; ++t) v[(t * m + mo) * c + ch] = src[(mo * c + ch) * taps + t];
  } else if (base_variant == "kxf") {
    // kx-folded rows of one kernel row: [kh][NF][C], row kx*M + m of kernel
    // row ky = W[m][c][ky][kx]; NF = kw*M rounded up to 16, zero rows after.
    const int64_t m = h->shape[0], c = h->shape[1], kh = h->shape[2], kw = h->shape[3];
    const int64_t nf = ((kw * m + 15) / 16) * 16;
    v.assign(kh * nf * c, 0.f);
    for (int64_t ky = 0; ky < kh; ++ky)
      for (int64_t kx = 0; kx < kw; ++kx)
        for (int64_t mo = 0; mo < m; ++mo)
          for (int64_t ch = 0; ch < c; ++ch)
            v[(ky * nf + kx * m + mo) * c + ch] = src[((mo * c + ch) * kh + ky) * kw + kx];
  } else if (base_variant.size() == 3 && base_variant.compare(0, 2, "pk") == 0) {
    // pkP: 1x1 conv [M, C] as the block diagonal of P copies, [P*M][P*C]:
    // P consecutive pixels share one row of P*C inputs and P*M outputs.
    const int64_t pk = base_variant[2] - '0';
    const int64_t m = h->shape[0], c = h->shape[1];
    v.assign(pk * m * pk * c, 0.f);
    for (int64_t q = 0; q < pk; ++q)
      for (int64_t mo = 0; mo < m; ++mo)
        for (int64_t ch = 0; ch < c; ++ch) v[(q * m + mo) * (pk * c) + q * c + ch] = src[mo * c + ch];
  } else if (base_variant.size() == 4 && base_variant.compare(0, 3, "dup") == 0) {
    // dupP: a vector repeated P times (bias of a pkP GEMM)
    const int64_t pk = base_variant[3] - '0';
    v.reserve(src.size() * pk);
    for (int64_t q = 0; q < pk; ++q) v.insert(v.end(), src.begin(), src.end());
  } else if (base_variant == "nk") {
    const int64_t k = h->shape[0], n = h->shape[1];
    v.resize(k * n);
    for (int64_t a = 0; a < k; ++a)
      for (int64_t b = 0; b < n; ++b) v[b * k + a] = src[a * n + b];
  } else {
    throw GraphError{"internal: unknown weight variant " + variant};
  }
  if (hi || lo || rn) {
    for (auto& x : v) {
      const float h = tf32_rn_host(x);
      x = lo ? tf32_rn_host(x - h) : h;
    }
  }
  // 16 zero floats of padding: vector loads of a trailing partial chunk
  // (bias of a 32-column tile) stay inside the allocation.
  const size_t real = v.size();
  v.resize(real + 16, 0.f);
  auto buf = std::make_unique<DevBuf>(v.size() * sizeof(float));
  QPC_CUDA_OR_THROW(cudaMemcpy(buf->ptr, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
  const float* p = buf->f();
  dev_cache_[key] = std::move(buf);
  return p;
}

// ================================================================ fusion
// Load-time graph rewrites into internal ops, each placed where the last
// absorbed node stood (all of its inputs exist there).  Only single-consumer
// intermediates are absorbed, so no other node can observe the change.
void Session::fuse() {
  std::vector<Node>& N = nodes_;
  std::vector<bool> alive(N.size(), true);
  std::set<std::string> gouts(outputs_.begin(), outputs_.end());
  auto consumers = [&](const std::string& t) {
    std::vector<int> r;
    for (size_t i = 0; i < N.size(); ++i)
      if (alive[i])
        for (auto& x : N[i].in)
          if (x == t) r.push_back((int)i);
    return r;
  };
  auto is_const = [&](const std::string& t) { return !t.empty() && weights_.count(t) > 0; };
  auto const_scalar = [&](const std::string& t, double* v) {
    const HostTensor* h = weight(t);
    if (!h || h->numel() != 1) return false;
    *v = h->scalar();
    return true;
  };

  // Conv fused-activation attribute from the reference optimizer
  // (optimize.rs:337-427: act 1 = GELU(c1..c3), 2 = ReLU) -> internal codes.
  for (auto& n : N) {
    if (n.op != "Conv") continue;
    const int64_t a = n.geti("act", 0);
    if (a == 1) {
      n.seti("qpc_act", ACT_GELU);
      n.setf("qpc_c1", n.getf("act_c1", 1.4142135f));
      n.setf("qpc_c2", n.getf("act_c2", 1.0f));
      n.setf("qpc_c3", n.getf("act_c3", 0.5f));
    } else if (a == 2) {
      n.seti("qpc_act", ACT_RELU);
    }
  }

  // MatMul(x, W[K,N]) (+ Add(b[N])) -> QpcLinear.  shape.rs:568-653 constant-B path.
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i] || N[i].op != "MatMul" || N[i].in.size() != 2) continue;
    const HostTensor* w = weight(N[i].in[1]);
    if (!w || w->shape.size() != 2 || (w->shape[0] % 4) != 0) continue;
    Node lin = N[i];
    lin.op = "QpcLinear";
    size_t pos = i;
    auto cs = consumers(N[i].out[0]);
    if (!gouts.count(N[i].out[0]) && cs.size() == 1 && N[cs[0]].op == "Add") {
      Node& ad = N[cs[0]];
      const std::string other = ad.in[0] == N[i].out[0] ? ad.in[1] : ad.in[0];
      const HostTensor* b = weight(other);
      if (b && b->numel() == w->shape[1] && ad.in[0] != ad.in[1]) {
        lin.in.push_back(other);
        lin.out = ad.out;
        alive[i] = false;
        pos = cs[0];
      }
    }
    N[pos] = lin;
    alive[pos] = true;
  }

  // ConvTranspose -> BatchNormalization -> QpcConvT (executor.rs:654-731).
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i] || N[i].op != "ConvTranspose") continue;
    Node ct = N[i];
    ct.op = "QpcConvT";
    ct.in.resize(2);
    size_t pos = i;
    auto cs = consumers(N[i].out[0]);
    if (!gouts.count(N[i].out[0]) && cs.size() == 1 && N[cs[0]].op == "BatchNormalization") {
      Node& bn = N[cs[0]];
      if (bn.in.size() == 5 && is_const(bn.in[1]) && is_const(bn.in[2]) && is_const(bn.in[3]) &&
          is_const(bn.in[4])) {
        for (int k = 1; k < 5; ++k) ct.in.push_back(bn.in[k]);
        ct.setf("qpc_eps", bn.getf("epsilon", 1e-5f));
        ct.out = bn.out;
        alive[i] = false;
        pos = cs[0];
      }
    }
    N[pos] = ct;
    alive[pos] = true;
  }

  // Activation absorption into producers with a fused epilogue.
  auto producer_ok = [&](const Node& n) {
    if (n.geti("qpc_act", 0) != 0 || n.geti("qpc_has_res", 0) != 0) return false;
    if (n.op == "QpcConvT") return true;  // inputs 2..5 are BN parameters, not a residual
    return (n.op == "Conv" || n.op == "QpcLinear") && !n.has_in(3);
  };
  bool changed = true;
  while (changed) {
    changed = false;
    for (size_t i = 0; i < N.size(); ++i) {
      if (!alive[i] || !producer_ok(N[i])) continue;
      const std::string o = N[i].out[0];
      if (gouts.count(o)) continue;
      auto cs = consumers(o);
      if (cs.size() == 2 && cs[0] != cs[1]) {
        // x * HardSigmoid(x) (hardswish) / x * Sigmoid(x) (swish)
        for (int pick = 0; pick < 2 && !changed; ++pick) {
          Node& h = N[cs[pick]];
          Node& m = N[cs[1 - pick]];
          if ((h.op != "HardSigmoid" && h.op != "Sigmoid") || h.in[0] != o || m.op != "Mul") continue;
          if (!((m.in[0] == o && m.in[1] == h.out[0]) || (m.in[1] == o && m.in[0] == h.out[0])))
            continue;
          auto hc = consumers(h.out[0]);
          if (hc.size() != 1 || gouts.count(h.out[0])) continue;
          if (h.op == "HardSigmoid") {
            N[i].seti("qpc_act", ACT_HARDSWISH);
            N[i].setf("qpc_alpha", h.getf("alpha", 0.2f));
            N[i].setf("qpc_beta", h.getf("beta", 0.5f));
          } else {
            N[i].seti("qpc_act", ACT_SWISH);
          }
          N[i].out = m.out;
          alive[cs[0]] = alive[cs[1]] = false;
          changed = true;
        }
      } else if (cs.size() == 1) {
        Node& a = N[cs[0]];
        int kind = 0;
        if (a.op == "Relu") kind = ACT_RELU;
        else if (a.op == "Sigmoid") kind = ACT_SIGMOID;
        else if (a.op == "HardSigmoid") kind = ACT_HARDSIGMOID;
        else if (a.op == "FusedGelu") kind = ACT_GELU;
        if (kind && a.in[0] == o) {
          N[i].seti("qpc_act", kind);
          if (kind == ACT_HARDSIGMOID) {
            N[i].setf("qpc_alpha", a.getf("alpha", 0.2f));
            N[i].setf("qpc_beta", a.getf("beta", 0.5f));
          }
          if (kind == ACT_GELU) {
            N[i].setf("qpc_c1", a.getf("c1", 1.4142135f));
            N[i].setf("qpc_c2", a.getf("c2", 1.0f));
            N[i].setf("qpc_c3", a.getf("c3", 0.5f));
          }
          N[i].out = a.out;
          alive[cs[0]] = false;
          changed = true;
        }
      }
    }
  }

  // ConvT pair: a QpcConvT to M <= 32 channels whose only consumer is a
  // QpcConvT to one channel (the DB head's two upsampling steps) becomes one
  // QpcConvTPair (in = x, w1, BN scale / bias / mean / var or "", w2; the
  // second layer's activation as qpc_act2...), planned as one tensor-core
  // GEMM whose epilogue applies the second layer.
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i] || N[i].op != "QpcConvT") continue;
    const std::string o = N[i].out[0];
    if (gouts.count(o)) continue;
    auto cs = consumers(o);
    if (cs.size() != 1 || N[cs[0]].op != "QpcConvT" || N[cs[0]].in.size() != 2 || N[cs[0]].in[0] != o)
      continue;
    const Node& second = N[cs[0]];
    const HostTensor* w1 = weight(N[i].in[1]);
    const HostTensor* w2 = weight(second.in[1]);
    if (!w1 || !w2 || w1->shape.size() != 4 || w2->shape.size() != 4 || w1->dtype != QPC_F32 ||
        w2->dtype != QPC_F32)
      continue;
    if (w1->shape[1] > 32 || w1->shape[0] % 4 != 0 || w2->shape[0] != w1->shape[1] || w2->shape[1] != 1 ||
        w2->shape[2] != 2 || w2->shape[3] != 2)
      continue;
    auto s2 = second.getints("strides");
    if (!(s2.empty() || (s2.size() == 2 && s2[0] == 2 && s2[1] == 2))) continue;
    bool padded = false;
    for (auto pd : second.getints("pads")) padded = padded || pd != 0;
    if (padded) continue;
    Node p = N[i];
    p.op = "QpcConvTPair";
    p.in.resize(6, "");
    p.in.push_back(second.in[1]);
    p.seti("qpc_act2", second.geti("qpc_act", 0));
    p.setf("qpc_alpha2", second.getf("qpc_alpha", 1.0f / 6.0f));
    p.setf("qpc_beta2", second.getf("qpc_beta", 0.5f));
    p.setf("qpc_c12", second.getf("qpc_c1", 1.4142135f));
    p.setf("qpc_c22", second.getf("qpc_c2", 1.0f));
    p.setf("qpc_c32", second.getf("qpc_c3", 0.5f));
    p.out = second.out;
    alive[i] = false;
    N[cs[0]] = p;
  }

  // Residual absorption: P -> Add(P.out, R) (fuse_conv_residual semantics,
  // optimize.rs:662-770: residual added after the activation).
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i]) continue;
    Node& p = N[i];
    if (!(p.op == "Conv" || p.op == "QpcLinear")) continue;
    if (p.has_in(3) || p.geti("qpc_has_res", 0)) continue;
    const std::string o = p.out[0];
    if (gouts.count(o)) continue;
    auto cs = consumers(o);
    if (cs.size() != 1 || N[cs[0]].op != "Add") continue;
    Node& ad = N[cs[0]];
    if (ad.in[0] == ad.in[1]) continue;
    const std::string r = ad.in[0] == o ? ad.in[1] : ad.in[0];
    if (is_const(r)) continue;
    Node f = p;
    if (f.op == "Conv") {
      f.in.resize(3);  // x, w, bias ("" if none)
      f.in.push_back(r);
    } else {
      if (f.in.size() < 3) f.in.push_back("");
      f.in.push_back(r);
    }
    f.seti("qpc_has_res", 1);
    f.out = ad.out;
    alive[i] = false;
    N[cs[0]] = f;
  }

  // Upsampled residual: a Conv's residual that is the output of a nearest
  // Resize used only there is read from the Resize's input through the
  // epilogue's nearest-source row remap (resize.rs:43-50), so the upsampled
  // map is never written (DBFPN: out_k = in_k + up(out_{k+1})).
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i] || N[i].op != "Conv" || !N[i].has_in(3)) continue;  // in[3]: residual
    const std::string r = N[i].in[3];
    if (gouts.count(r)) continue;
    auto rc = consumers(r);
    if (rc.size() != 1) continue;
    for (size_t k = 0; k < N.size(); ++k) {
      if (!alive[k] || N[k].op != "Resize" || N[k].out.empty() || N[k].out[0] != r) continue;
      if (N[k].gets("mode", "nearest") != "nearest" || N[k].in.empty() || is_const(N[k].in[0])) break;
      Node& c = N[i];
      c.in[3] = N[k].in[0];
      c.seti("qpc_res_up", 1);  // the upsampled size is the conv's output size
      alive[k] = false;
      break;
    }
  }

  // LayerNorm decomposition (executor ReduceMean/Sub/Pow/ReduceMean/Add/Sqrt/
  // Div then Mul/Add or MulAddScale; shape.rs:510-566 f64 means) -> QpcLayerNorm.
  for (size_t i = 0; i < N.size(); ++i) {
    if (!alive[i] || N[i].op != "ReduceMean") continue;
    const Node& rm1 = N[i];
    auto ax = rm1.getints("axes");
    if (!(ax.size() == 1 && ax[0] == -1) || rm1.geti("keepdims", 1) != 1) continue;
    const std::string x = rm1.in[0], mean = rm1.out[0];
    auto c1 = consumers(mean);
    if (c1.size() != 1 || N[c1[0]].op != "Sub" || N[c1[0]].in[0] != x || N[c1[0]].in[1] != mean)
      continue;
    const int isub = c1[0];
    const std::string d = N[isub].out[0];
    auto cd = consumers(d);
    if (cd.size() != 2) continue;
    int ipow = -1, idiv = -1;
    for (int k : cd) {
      if (N[k].op == "Pow" && N[k].in[0] == d) ipow = k;
      if (N[k].op == "Div" && N[k].in[0] == d) idiv = k;
    }
    double e2 = 0;
    if (ipow < 0 || idiv < 0 || !const_scalar(N[ipow].in[1], &e2) || e2 != 2.0) continue;
    auto cp = consumers(N[ipow].out[0]);
    if (cp.size() != 1 || N[cp[0]].op != "ReduceMean") continue;
    const int irm2 = cp[0];
    auto ax2 = N[irm2].getints("axes");
    if (!(ax2.size() == 1 && ax2[0] == -1)) continue;
    auto cv = consumers(N[irm2].out[0]);
    if (cv.size() != 1 || N[cv[0]].op != "Add") continue;
    const int iadd = cv[0];
    double eps = 0;
    const std::string eps_name = N[iadd].in[0] == N[irm2].out[0] ? N[iadd].in[1] : N[iadd].in[0];
    if (!const_scalar(eps_name, &eps)) continue;
    auto cs2 = consumers(N[iadd].out[0]);
    if (cs2.size() != 1 || N[cs2[0]].op != "Sqrt") continue;
    const int isq = cs2[0];
    if (N[idiv].in[1] != N[isq].out[0]) continue;
    auto cq = consumers(N[isq].out[0]);
    if (cq.size() != 1) continue;
    // affine tail
    Node ln;
    ln.op = "QpcLayerNorm";
    ln.name = rm1.name;
    ln.in = {x, "", ""};
    ln.setf("qpc_eps", (float)eps);
    std::vector<int> absorbed = {(int)i, isub, ipow, irm2, iadd, isq, idiv};
    int last = idiv;
    std::string out = N[idiv].out[0];
    auto cn = consumers(out);
    if (!gouts.count(out) && cn.size() == 1) {
      Node& t = N[cn[0]];
      if (t.op == "MulAddScale" && t.in[0] == out && is_const(t.in[1]) && is_const(t.in[2])) {
        ln.in[1] = t.in[1];
        ln.in[2] = t.in[2];
        absorbed.push_back(cn[0]);
        last = cn[0];
        out = t.out[0];
      } else if (t.op == "Mul" && is_const(t.in[1]) && t.in[0] == out) {
        auto cm = consumers(t.out[0]);
        if (!gouts.count(t.out[0]) && cm.size() == 1 && N[cm[0]].op == "Add" &&
            N[cm[0]].in[0] == t.out[0] && is_const(N[cm[0]].in[1])) {
          ln.in[1] = t.in[1];
          ln.in[2] = N[cm[0]].in[1];
          absorbed.push_back(cn[0]);
          absorbed.push_back(cm[0]);
          last = cm[0];
          out = N[cm[0]].out[0];
        }
      }
    }
    ln.out = {out};
    for (int k : absorbed) alive[k] = false;
    N[last] = ln;
    alive[last] = true;
  }

  // SVTR multi-head attention (the rec transformer block; the reference
  // runs it as separate Mul / MatMul / Softmax / MatMul passes, its GPU plan
  // as n_attn_mm + n_softmax, plan.rs:1882-1908, 2026-2055):
  //   qkv [B,T,3*H*D] -Reshape[0,0,3,H,D]-> -Transpose[2,0,3,1,4]-> Slice j,
  //   Squeeze -> q, k, v;  Mul(q, scale) -> MatMul(., Transpose(k)[0,1,3,2])
  //   -> Softmax(-1) -> MatMul(., v) -> Transpose[0,2,1,3] -> Reshape[0,0,H*D]
  // becomes QpcAttention(qkv, scale) -> [B,T,H*D] (launch_attention), when
  // every intermediate has exactly the consumers of this pattern.
  {
    auto producer = [&](const std::string& t) -> int {
      for (size_t j = 0; j < N.size(); ++j)
        if (alive[j] && !N[j].out.empty() && N[j].out[0] == t) return (int)j;
      return -1;
    };
    auto ints = [&](const Node& n, size_t k, const char* attr) -> std::vector<int64_t> {
      if (n.has_in(k)) {
        const HostTensor* h = weight(n.in[k]);
        if (!h) return {};
        if (h->dtype == QPC_I64) return h->i;
        std::vector<int64_t> v;
        for (float f : h->f) v.push_back((int64_t)f);
        return v;
      }
      return n.getints(attr);
    };
    auto sole = [&](const std::string& t, int who) {
      if (gouts.count(t)) return false;
      auto cs = consumers(t);
      return cs.size() == 1 && cs[0] == who;
    };
    // Squeeze(Slice(tq, [j], [j+1], [0]), [0]) -> (tq, j); -1 on mismatch
    auto slice_of = [&](const std::string& t, int who, std::string* tq) -> int {
      const int sq = producer(t);
      if (sq < 0 || N[sq].op != "Squeeze" || !sole(t, who) || ints(N[sq], 1, "axes") != std::vector<int64_t>{0})
        return -1;
      const int sl = producer(N[sq].in[0]);
      if (sl < 0 || N[sl].op != "Slice" || !sole(N[sl].out[0], sq)) return -1;
      const auto st = ints(N[sl], 1, "starts"), en = ints(N[sl], 2, "ends"), ax = ints(N[sl], 3, "axes");
      if (st.size() != 1 || en.size() != 1 || ax != std::vector<int64_t>{0} || en[0] != st[0] + 1) return -1;
      if (N[sl].has_in(4) && ints(N[sl], 4, "steps") != std::vector<int64_t>{1}) return -1;
      *tq = N[sl].in[0];
      return (int)st[0];
    };
    for (size_t i = 0; i < N.size(); ++i) {
      if (!alive[i] || N[i].op != "Softmax" || N[i].geti("axis", -1) != -1) continue;
      const int m1 = producer(N[i].in[0]);
      if (m1 < 0 || N[m1].op != "MatMul" || !sole(N[i].in[0], (int)i)) continue;
      const auto cs = consumers(N[i].out[0]);
      if (gouts.count(N[i].out[0]) || cs.size() != 1 || N[cs[0]].op != "MatMul" || N[cs[0]].in[0] != N[i].out[0])
        continue;
      const int m2 = cs[0];
      const int mu = producer(N[m1].in[0]), tk = producer(N[m1].in[1]);
      if (mu < 0 || tk < 0 || N[mu].op != "Mul" || N[tk].op != "Transpose") continue;
      if (!sole(N[m1].in[0], m1) || !sole(N[m1].in[1], m1) || N[tk].getints("perm") != std::vector<int64_t>{0, 1, 3, 2})
        continue;
      const bool q_first = !is_const(N[mu].in[0]);
      const std::string qn = q_first ? N[mu].in[0] : N[mu].in[1], sn = q_first ? N[mu].in[1] : N[mu].in[0];
      double scale = 0;
      if (!const_scalar(sn, &scale)) continue;
      std::string tq0, tq1, tq2;
      if (slice_of(qn, mu, &tq0) != 0 || slice_of(N[tk].in[0], tk, &tq1) != 1 ||
          slice_of(N[m2].in[1], m2, &tq2) != 2 || tq0 != tq1 || tq0 != tq2)
        continue;
      if (gouts.count(tq0) || consumers(tq0).size() != 3) continue;
      const int tr = producer(tq0);
      if (tr < 0 || N[tr].op != "Transpose" || N[tr].getints("perm") != std::vector<int64_t>{2, 0, 3, 1, 4}) continue;
      const int rs = producer(N[tr].in[0]);
      if (rs < 0 || N[rs].op != "Reshape" || !sole(N[tr].in[0], tr)) continue;
      const auto rshape = ints(N[rs], 1, "shape");
      if (rshape.size() != 5 || rshape[0] != 0 || rshape[1] != 0 || rshape[2] != 3 || rshape[3] <= 0 || rshape[4] <= 0)
        continue;
      const int64_t H = rshape[3], D = rshape[4];
      const auto c2 = consumers(N[m2].out[0]);
      if (gouts.count(N[m2].out[0]) || c2.size() != 1 || N[c2[0]].op != "Transpose" ||
          N[c2[0]].getints("perm") != std::vector<int64_t>{0, 2, 1, 3})
        continue;
      const int ot = c2[0];
      const auto c3 = consumers(N[ot].out[0]);
      if (gouts.count(N[ot].out[0]) || c3.size() != 1 || N[c3[0]].op != "Reshape") continue;
      const int orr = c3[0];
      if (ints(N[orr], 1, "shape") != std::vector<int64_t>{0, 0, H * D}) continue;
      Node at;
      at.op = "QpcAttention";
      at.name = N[m1].name + "+attention";
      at.in = {N[rs].in[0]};
      at.out = N[orr].out;
      at.seti("heads", H);
      at.seti("head_dim", D);
      at.setf("scale", (float)scale);
      for (int k : {rs, tr, mu, tk, m1, (int)i, m2, ot})
        alive[k] = false;
      for (const std::string& t : {qn, N[tk].in[0], N[m2].in[1]}) {
        const int sq = producer(t);
        alive[producer(N[sq].in[0])] = false;
        alive[sq] = false;
      }
      N[orr] = at;
      alive[orr] = true;
    }
  }

  // Rec CTC head: QpcLinear -> Softmax(last axis) -> graph output, with the
  // argmax exit on: one fused op emitting (val, idx) pairs
  // (DeviceSession::rec_argmax_pairs, device.rs:159-163; n_exit3_argmax.comp).
  if (argmax_exit_) {
    for (size_t i = 0; i < N.size(); ++i) {
      if (!alive[i] || N[i].op != "Softmax" || !gouts.count(N[i].out[0])) continue;
      const int64_t axis = N[i].geti("axis", -1);
      if (axis != -1) continue;
      int ip = -1;
      for (size_t j = 0; j < i; ++j)
        if (alive[j] && N[j].out.size() && N[j].out[0] == N[i].in[0]) ip = (int)j;
      if (ip < 0 || N[ip].op != "QpcLinear" || N[ip].has_in(3) || N[ip].geti("qpc_act", 0)) continue;
      if (consumers(N[ip].out[0]).size() != 1) continue;
      Node h = N[ip];
      h.op = "QpcCtcHead";
      h.out = N[i].out;
      alive[ip] = false;
      N[i] = h;
    }
  }

  std::vector<Node> kept;
  for (size_t i = 0; i < N.size(); ++i)
    if (alive[i]) kept.push_back(std::move(N[i]));
  nodes_ = std::move(kept);
}

// ================================================================ planner
namespace {

struct Val {
  bool is_const = false;
  const HostTensor* ct = nullptr;     // host constant (initializer or folded)
  std::shared_ptr<HostTensor> owned;  // folded constant storage
  std::vector<int64_t> shape, strides;
  int buf = -1;                       // arena buffer
  const float* cptr = nullptr;        // device constant (weights)
  int64_t off = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

std::vector<int64_t> rowmajor_strides(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size());
  int64_t acc = 1;
  for (int i = (int)s.size() - 1; i >= 0; --i) {
    st[i] = acc;
    acc *= s[i];
  }
  return st;
}
std::vector<int64_t> nhwc_strides(const std::vector<int64_t>& s) {
  const int64_t C = s[1], H = s[2], W = s[3];
  return {H * W * C, 1, W * C, C};
}
bool same_layout(const Val& v, const std::vector<int64_t>& want) {
  for (size_t i = 0; i < v.shape.size(); ++i)
    if (v.shape[i] != 1 && v.strides[i] != want[i]) return false;
  return true;
}
bool is_rowmajor(const Val& v) { return same_layout(v, rowmajor_strides(v.shape)); }
bool is_nhwc(const Val& v) { return v.shape.size() == 4 && same_layout(v, nhwc_strides(v.shape)); }

struct Arena {
  struct B {
    std::unique_ptr<DevBuf> mem;
    int64_t cap = 0;
    int refs = 0;
    bool pinned = false;  // graph I/O: never reused
  };
  std::vector<B> bufs;
  int alloc(int64_t elems, bool pinned = false) {
    elems = std::max<int64_t>(elems, 1);
    int best = -1;
    if (!pinned)
      for (size_t i = 0; i < bufs.size(); ++i)
        if (bufs[i].refs == 0 && !bufs[i].pinned && bufs[i].cap >= elems &&
            (best < 0 || bufs[i].cap < bufs[best].cap))
          best = (int)i;
    if (best >= 0 && bufs[best].cap <= 2 * elems + (1 << 20)) {
      bufs[best].refs = 1;
      return best;
    }
    B b;
    b.mem = std::make_unique<DevBuf>((size_t)(elems + 64) * sizeof(float));
    b.cap = elems + 64;
    b.refs = 1;
    b.pinned = pinned;
    bufs.push_back(std::move(b));
    return (int)bufs.size() - 1;
  }
  void retain(int b) {
    if (b >= 0) ++bufs[b].refs;
  }
  void release(int b) {
    if (b >= 0 && bufs[b].refs > 0) --bufs[b].refs;
  }
  float* ptr(int b) { return bufs[b].mem->f(); }
};

ActParams act_of(const Node& n) {
  ActParams a{};
  a.kind = (int)n.geti("qpc_act", 0);
  a.alpha = n.getf("qpc_alpha", 1.0f / 6.0f);
  a.beta = n.getf("qpc_beta", 0.5f);
  a.c1 = n.getf("qpc_c1", 1.4142135f);
  a.c2 = n.getf("qpc_c2", 1.0f);
  a.c3 = n.getf("qpc_c3", 0.5f);
  return a;
}

// ONNX pads / auto_pad -> (ph, pw, peh, pew); executor.rs resolve_pads.
void resolve_pads(const Node& n, int64_t h, int64_t w, int64_t kh, int64_t kw, int64_t sh,
                  int64_t sw, int64_t* ph, int64_t* pw, int64_t* peh, int64_t* pew) {
  const std::string ap = n.gets("auto_pad", "NOTSET");
  if (ap == "SAME_UPPER" || ap == "SAME_LOWER") {
    auto one = [&](int64_t in, int64_t k, int64_t s, int64_t* b, int64_t* e) {
      const int64_t out = (in + s - 1) / s;
      const int64_t tot = std::max<int64_t>(0, (out - 1) * s + k - in);
      *b = ap == "SAME_UPPER" ? tot / 2 : tot - tot / 2;
      *e = tot - *b;
    };
    one(h, kh, sh, ph, peh);
    one(w, kw, sw, pw, pew);
    return;
  }
  auto p = n.getints("pads");
  if (p.size() == 4) {
    *ph = p[0];
    *pw = p[1];
    *peh = p[2];
    *pew = p[3];
  } else {
    *ph = *pw = *peh = *pew = 0;
  }
}

// The pointwise tensor-core path of plan_conv: a 1x1, stride-1, unpadded,
// ungrouped conv over a C % 4 == 0 input (rows = pixels, one tcgen05 GEMM),
// given the conv's input height and width.
bool takes_pointwise_gemm(const Node& n, const HostTensor& w, int64_t H, int64_t W) {
  if (w.shape.size() != 4) return false;
  const int64_t cg = w.shape[1], kh = w.shape[2], kw = w.shape[3];
  const int64_t group = n.geti("group", 1);
  auto st = n.getints("strides");
  const int64_t sh = st.size() == 2 ? st[0] : 1, sw = st.size() == 2 ? st[1] : 1;
  int64_t ph, pw, peh, pew;
  resolve_pads(n, H, W, kh, kw, sh, sw, &ph, &pw, &peh, &pew);
  return group == 1 && kh == 1 && kw == 1 && sh == 1 && sw == 1 && ph == 0 && pw == 0 && peh == 0 &&
         pew == 0 && (cg % 4) == 0;
}

// The tap-folded tensor-core path of plan_conv (TF32 only): a k x k,
// stride-1, ungrouped conv over a C % 4 == 0 input of N x C x H x W that
// conv_fold_ok accepts (the geometry launch_conv_tc checks).
bool takes_fold_conv(const Node& n, const HostTensor& w, int64_t N, int64_t C, int64_t H, int64_t W) {
  if (w.shape.size() != 4 || takes_pointwise_gemm(n, w, H, W)) return false;
  const int64_t M = w.shape[0], cg = w.shape[1], kh = w.shape[2], kw = w.shape[3];
  auto st = n.getints("strides");
  const int64_t sh = st.size() == 2 ? st[0] : 1, sw = st.size() == 2 ? st[1] : 1;
  if (n.geti("group", 1) != 1 || cg != C || sh != 1 || sw != 1 || (C % 4) != 0 || kh * kw <= 1) return false;
  int64_t ph, pw, peh, pew;
  resolve_pads(n, H, W, kh, kw, sh, sw, &ph, &pw, &peh, &pew);
  const int64_t oh = H + ph + peh - kh + 1, ow = W + pw + pew - kw + 1;
  if (oh <= 0 || ow <= 0) return false;
  ConvGeom g{(int)N, (int)H, (int)W, (int)C, (int)oh, (int)ow, (int)M, (int)kh, (int)kw, 1, 1, (int)ph, (int)pw};
  return conv_fold_ok(g);
}

}  // namespace

class Planner {
 public:
  Planner(Session& s, PlanInstance& p) : S(s), P(p) {}

  void run(const qpc_tensor* inputs, int n_inputs) {
    // Remaining uses of each tensor (consumers + graph outputs).
    for (size_t i = 0; i < S.nodes().size(); ++i) {
      const Node& n = S.nodes()[i];
      for (auto& x : n.in)
        if (!x.empty()) {
          uses_[x]++;
          consumers_[x].push_back((int)i);
        }
      for (auto& o : n.out) producer_[o] = (int)i;
    }
    for (auto& o : S.graph_outputs()) uses_[o]++;

    // Graph inputs: contiguous row-major device buffers (logical NCHW).
    for (const std::string& gi : S.graph_inputs()) {
      const qpc_tensor* t = nullptr;
      for (int k = 0; k < n_inputs; ++k)
        if (gi == inputs[k].name) t = &inputs[k];
      if (!t) throw GraphError{"missing graph input " + gi};
      if (t->dtype != QPC_F32 && t->dtype != QPC_F32_DEVICE && t->dtype != QPC_U8_IMAGE &&
          t->dtype != QPC_U8_IMAGE_DEVICE)
        throw GraphError{"graph input " + gi + " must be f32 (or a u8 image batch)"};
      Val v;
      PlanInstance::IO io;
      io.name = gi;
      io.dtype = base_dtype(t->dtype);  // host or device data: same plan
      if (io.dtype == QPC_U8_IMAGE) {
        // n x h x w x 3 u8 images for an [n, 3, h, w] f32 input: staged as
        // bytes, normalised on the device as the reference engine does
        if (t->rank != 4 || t->shape[3] != 3) throw GraphError{"u8 image input " + gi + " must be n x h x w x 3"};
        const int64_t n = t->shape[0], h = t->shape[1], w = t->shape[2];
        v.shape = {n, 3, h, w};
        v.strides = rowmajor_strides(v.shape);
        v.buf = A.alloc(v.numel(), true);
        io.shape.assign(t->shape, t->shape + t->rank);
        io.bytes = (size_t)(n * h * w * 3);
        io.count = (int64_t)((io.bytes + 3) / 4);
        const int u8buf = A.alloc(io.count, true);
        io.dev = A.ptr(u8buf);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(io.dev);
        float* dst = A.ptr(v.buf);
        step("det_preprocess", gi, (double)io.bytes + 4.0 * v.numel(), 0, [=](cudaStream_t s) {
          return launch_det_preprocess(src, (int)n, (int)h, (int)w, dst, (int)h, (int)w, s);
        });
      } else {
        v.shape.assign(t->shape, t->shape + t->rank);
        v.strides = rowmajor_strides(v.shape);
        v.buf = A.alloc(v.numel(), true);
        io.shape = v.shape;
        io.count = v.numel();
        io.bytes = (size_t)io.count * sizeof(float);
        io.dev = A.ptr(v.buf);
      }
      P.ins.push_back(io);
      vals_[gi] = v;
    }
    for (size_t i = 0; i < S.nodes().size(); ++i) {
      const Node& n = S.nodes()[i];
      try {
        plan_node(n);
      } catch (GraphError& e) {
        throw GraphError{n.op + " " + n.name + ": " + e.msg};
      }
      for (auto& x : n.in)
        if (!x.empty()) use_done(x);
      for (auto& o : n.out)
        if (!uses_.count(o) || uses_[o] == 0) drop(o);
    }
    if (!pending_resize_.empty()) throw GraphError{"internal: resize into a concat that was never planned"};
    // Graph outputs: contiguous row-major, dedicated buffers.
    for (const std::string& go : S.graph_outputs()) {
      auto it = vals_.find(go);
      if (it == vals_.end()) throw GraphError{"graph output " + go + " not produced"};
      Val v = it->second;
      if (v.is_const) throw GraphError{"graph output " + go + " is a constant"};
      Val o;
      o.shape = v.shape;
      o.strides = rowmajor_strides(v.shape);
      if (is_rowmajor(v) && (v.off % 4) == 0) {
        o.buf = v.buf;  // already in host order: read it back directly
        o.off = v.off;
        A.bufs[v.buf].pinned = true;
      } else {
        o.buf = A.alloc(o.numel(), true);
        copy_into(v, o, "output " + go);
      }
      PlanInstance::IO io;
      io.name = go;
      io.shape = o.shape;
      io.count = o.numel();
      io.bytes = (size_t)io.count * sizeof(float);
      io.dtype = QPC_F32;
      io.dev = A.ptr(o.buf) + o.off;
      P.outs.push_back(io);
    }
    if (S.det_mask_exit()) {
      // DB mask exit (geometry.rs:286-296): the host receives the binarized,
      // 2x2-dilated u8 mask its connected components run on (a quarter of
      // the probability map's bytes); the map itself stays on the device
      // (output 1, device only) for box scoring (qpc_op_box_score).
      if (P.outs.size() != 1 || P.outs[0].shape.size() != 4 || P.outs[0].shape[1] != 1)
        throw GraphError{"det mask exit needs one [n, 1, h, w] output"};
      PlanInstance::IO& pred = P.outs[0];
      const int64_t n = pred.shape[0], h = pred.shape[2], w = pred.shape[3];
      PlanInstance::IO m;
      m.name = pred.name + ".mask";
      m.shape = {n, h, w};
      m.count = n * h * w;
      m.bytes = (size_t)m.count;
      m.dtype = QPC_U8;
      const int mb = A.alloc((m.count + 3) / 4, true);
      m.dev = A.ptr(mb);
      const float* pp = pred.dev;
      uint8_t* mp = reinterpret_cast<uint8_t*>(m.dev);
      const float th = S.mask_thresh();
      const int dil = S.mask_dilate() ? 1 : 0;
      step("db_mask", m.name, 4.0 * m.count + (double)m.count, 0, [=](cudaStream_t st) {
        return launch_db_mask(pp, nullptr, mp, (int)n, (int)h, (int)w, th, dil, st);
      });
      pred.device_only = true;
      pred.bytes = 0;
      P.outs.insert(P.outs.begin(), m);
    }
    for (auto& b : A.bufs) {
      P.bytes += b.mem->bytes;
      P.bufs.push_back(std::move(b.mem));
    }
  }

 private:
  Session& S;
  PlanInstance& P;
  Arena A;
  std::unordered_map<std::string, Val> vals_;
  std::unordered_map<std::string, int> uses_;
  std::unordered_map<std::string, std::vector<int>> consumers_;
  std::unordered_map<std::string, int> producer_;
  std::unordered_map<std::string, Val> concat_bufs_;  // Concat output -> buffer allocated early
  // Nearest resizes writing a slice of a Concat, held until the Concat is
  // planned and then launched together (one output pixel's slices written
  // by one kernel).  Each keeps its source alive (src) until then.
  struct PendingResize {
    Val src, dst;
    int h, w, c;
    bool round;  // store tf32-rounded
    std::string name;
  };
  std::unordered_map<std::string, std::vector<PendingResize>> pending_resize_;

  // Channel count of a 4-D tensor from its producer chain (before it exists).
  int64_t channels_of(const std::string& name, int depth = 0) {
    auto v = vals_.find(name);
    if (v != vals_.end() && v->second.shape.size() == 4) return v->second.shape[1];
    auto p = producer_.find(name);
    if (p == producer_.end() || depth > 64) return -1;
    const Node& n = S.nodes()[p->second];
    if (n.op == "Conv") return S.weight(n.in[1])->shape[0];
    if (n.op == "QpcConvT" || n.op == "ConvTranspose") return S.weight(n.in[1])->shape[1];
    if (n.op == "QpcConvTPair") return S.weight(n.in[6])->shape[1];
    if (n.op == "Concat") {
      int64_t t = 0;
      for (auto& x : n.in) {
        const int64_t c = channels_of(x, depth + 1);
        if (c < 0) return -1;
        t += c;
      }
      return t;
    }
    static const std::set<std::string> same = {"Resize", "Relu", "Sigmoid", "HardSigmoid", "Add", "Sub",
                                               "Mul", "Div", "MulAddScale", "BatchNormalization",
                                               "AveragePool", "MaxPool", "Identity", "Clip"};
    if (same.count(n.op)) return channels_of(n.in[0], depth + 1);
    return -1;
  }

  // A depthwise conv planned together with its pointwise consumer
  // (launch_dwpw): the consumer's input name -> the depthwise conv's operands.
  struct FusedDw {
    Val x;  // NHWC input, held until the consumer is planned
    ConvGeom g;
    const float* w = nullptr;
    const float* bias = nullptr;
    ActParams act{};
    std::string name;
  };
  std::map<std::string, FusedDw> fused_dw_;

  // Whether depthwise conv `n` (geometry g) runs fused into its consumer: TF32
  // math (the fused A operand is the tf32-rounded depthwise output), its
  // output is no graph output and feeds exactly one Conv, as input 0 only,
  // which takes the pointwise GEMM path without residual or channel gate,
  // and launch_dwpw supports the shapes.  QPPOCR_CUDA_FUSE_DWPW=0 turns the
  // fusion off (both paths give identical results).
  bool dw_fusable(const Node& n, const ConvGeom& g) {
    if (S.math() != QPC_MATH_TF32) return false;
    static const bool enabled = [] {
      const char* v = std::getenv("QPPOCR_CUDA_FUSE_DWPW");
      return !(v && std::string(v) == "0");
    }();
    if (!enabled) return false;
    const std::string& o = n.out[0];
    for (auto& go : S.graph_outputs())
      if (go == o) return false;
    auto cit = consumers_.find(o);
    if (cit == consumers_.end() || cit->second.size() != 1) return false;
    const Node& c = S.nodes()[cit->second[0]];
    if (c.op != "Conv" || c.in.size() < 2 || c.in[0] != o || c.has_in(3) || c.geti("qpc_res_up", 0)) return false;
    for (size_t k = 1; k < c.in.size(); ++k)
      if (c.in[k] == o) return false;
    const HostTensor* w = S.weight(c.in[1]);
    if (!w || !takes_pointwise_gemm(c, *w, g.oh, g.ow)) return false;
    if (c.has_in(2) && !S.weight(c.in[2])) return false;
    return dwpw_ok(g, (int)w->shape[0]);
  }

  // The pointwise conv `n` whose input is the fused depthwise conv `f`.
  void plan_dwpw(const Node& n, const FusedDw& f) {
    const HostTensor* w = S.weight(n.in[1]);
    const int64_t M = w->shape[0];
    const ConvGeom g = f.g;
    const std::vector<int64_t> oshape = {g.n, M, g.oh, g.ow};
    Val y = new_val(oshape, true);
    float* yp = out_ptr(y);
    const float* xp = out_ptr(f.x);
    const float* wb = S.dweight(n.in[1], "raw.rn");
    GemmEpilogue e;
    e.bias = n.has_in(2) ? S.dweight(n.in[2], "raw") : nullptr;
    e.out = yp;
    e.ldo = (int)M;
    e.ldr = (int)M;
    e.act = act_of(n);
    unsigned int* err = device_state(S.device()).err_word;
    const double pix = (double)g.n * g.oh * g.ow;
    const double bytes = 4.0 * g.n * g.h * g.w * g.c + 4.0 * pix * M + 4.0 * g.c * (M + g.kh * g.kw);
    const double flops = 2.0 * pix * g.c * (g.kh * g.kw + M);
    const float* dww = f.w;
    const float* dwb = f.bias;
    const ActParams dwa = f.act;
    step("dwpw", f.name + "+" + n.name, bytes, flops, [=](cudaStream_t s) {
      return launch_dwpw(xp, g, dww, dwb, dwa, wb, (int)M, e, err, s);
    });
    define(n.out[0], y);
  }

  // Whether every consumer of `o` (an N x C x H x W value) reads it only as
  // the A operand (input 0) of a TF32 conv on a tensor-core path that rounds
  // A to tf32 (nearest) - the pointwise GEMM or the tap-folded k x k conv,
  // the predicates plan_conv routes by - possibly through a channel Concat
  // whose output does the same, or of a linear / CTC head (plan_linear: the
  // rows-mode GEMM, which always rounds A).  Then `o` may be stored
  // tf32-rounded: each consumer would round it to the same values.  plan_conv
  // checks, when it plans each such consumer, that it took one of those paths.
  std::set<std::string> tf32_rounded_;
  bool feeds_only_tf32_a(const std::string& o, int64_t N, int64_t C, int64_t H, int64_t W, int depth = 0) {
    if (S.math() != QPC_MATH_TF32 || depth > 4) return false;
    for (auto& go : S.graph_outputs())
      if (go == o) return false;
    auto cit = consumers_.find(o);
    if (cit == consumers_.end() || cit->second.empty()) return false;
    for (int ci : cit->second) {
      const Node& c = S.nodes()[ci];
      if (c.op == "Concat") {
        int64_t axis = c.geti("axis", 0);
        if (axis < 0) axis += 4;
        if (axis != 1 || cit->second.size() != 1) return false;
        int64_t total = 0, seen = 0;
        for (auto& x : c.in) {
          const int64_t ch = channels_of(x);
          if (ch < 0) return false;
          total += ch;
          seen += x == o;
        }
        if (seen != 1 || !feeds_only_tf32_a(c.out[0], N, total, H, W, depth + 1)) return false;
        continue;
      }
      if (c.op == "QpcLinear" || c.op == "QpcCtcHead") {
        if (c.in.empty() || c.in[0] != o) return false;
        for (size_t k = 1; k < c.in.size(); ++k)
          if (c.in[k] == o) return false;
        continue;
      }
      if (c.op != "Conv" || c.in.size() < 2 || c.in[0] != o) return false;
      for (size_t k = 1; k < c.in.size(); ++k)
        if (c.in[k] == o) return false;
      const HostTensor* w = S.weight(c.in[1]);
      if (!w || !(takes_pointwise_gemm(c, *w, H, W) || takes_fold_conv(c, *w, N, C, H, W))) return false;
    }
    return true;
  }

  // If `o` (4-D, NHWC-produced) feeds only a channel Concat, return the view of
  // its slice in the Concat's buffer (allocated now, at the first part, so no
  // buffer that is live in between can alias it).
  bool concat_slot(const std::string& o, const std::vector<int64_t>& oshape, Val* dst,
                   std::string* concat_out = nullptr) {
    auto cit = consumers_.find(o);
    if (cit == consumers_.end() || cit->second.size() != 1) return false;
    const Node& c = S.nodes()[cit->second[0]];
    if (c.op != "Concat" || oshape.size() != 4) return false;
    for (auto& go : S.graph_outputs())
      if (go == o) return false;
    int64_t axis = c.geti("axis", 0);
    if (axis < 0) axis += 4;
    if (axis != 1) return false;
    int64_t off = -1, total = 0;
    for (auto& x : c.in) {
      if (x == o) {
        if (off >= 0) return false;  // same tensor twice
        off = total;
      }
      const int64_t ch = channels_of(x);
      if (ch < 0) return false;
      total += ch;
    }
    if (off < 0 || (off % 4) || (total % 4)) return false;
    auto it = concat_bufs_.find(c.out[0]);
    if (it == concat_bufs_.end()) {
      std::vector<int64_t> full = {oshape[0], total, oshape[2], oshape[3]};
      it = concat_bufs_.emplace(c.out[0], new_val(full, true)).first;
    }
    const Val& f = it->second;
    if (f.shape[0] != oshape[0] || f.shape[2] != oshape[2] || f.shape[3] != oshape[3]) return false;
    *dst = view_of(f, oshape, f.strides, f.off + off);
    if (concat_out) *concat_out = c.out[0];
    return true;
  }

  // Launch the resizes held for Concat `co`, up to RESIZE_MAX_SRC per kernel.
  void flush_resizes(const std::string& co) {
    auto it = pending_resize_.find(co);
    if (it == pending_resize_.end()) return;
    std::vector<PendingResize> parts = std::move(it->second);
    pending_resize_.erase(it);
    const Val& f = concat_bufs_.at(co);
    float* yp = out_ptr(f);
    const int64_t N = f.shape[0], oh = f.shape[2], ow = f.shape[3], ldc = f.strides[3];
    for (size_t b = 0; b < parts.size(); b += RESIZE_MAX_SRC) {
      ResizeSrcs rs{};
      rs.round_tf32 = parts[b].round ? 1 : 0;
      double bytes = 0;
      std::string nm;
      for (size_t k = b; k < parts.size() && k < b + RESIZE_MAX_SRC; ++k) {
        const PendingResize& r = parts[k];
        if (r.round != parts[b].round) throw GraphError{"internal: concat resizes disagree on rounding"};
        const int j = rs.n++;
        rs.x[j] = out_ptr(r.src);
        rs.h[j] = r.h;
        rs.w[j] = r.w;
        rs.c4[j] = r.c / 4;
        rs.c_off[j] = (int)(r.dst.off - f.off);
        rs.quads += r.c / 4;
        bytes += 4.0 * ((double)N * r.c * r.h * r.w + (double)N * r.c * oh * ow);
        nm += (nm.empty() ? "" : "+") + r.name;
      }
      step("resize", nm, bytes, 0, [=](cudaStream_t st) {
        return launch_resize_nearest_multi_nhwc(rs, yp, (int)N, (int)oh, (int)ow, (int)ldc, st);
      });
    }
    for (auto& r : parts) unref(r.src);
  }

  // ------------------------------------------------------------ bookkeeping
  void use_done(const std::string& x) {
    auto it = uses_.find(x);
    if (it == uses_.end()) return;
    if (--it->second == 0) drop(x);
  }
  void drop(const std::string& x) {
    auto it = vals_.find(x);
    if (it == vals_.end()) return;
    A.release(it->second.buf);
    vals_.erase(it);
  }
  void define(const std::string& name, Val v) {
    if (vals_.count(name)) A.release(vals_[name].buf);
    vals_[name] = std::move(v);
  }
  const Val& get(const std::string& name) {
    auto it = vals_.find(name);
    if (it != vals_.end()) return it->second;
    const HostTensor* h = S.weight(name);
    if (!h) throw GraphError{"missing tensor " + name};
    Val v;
    v.is_const = true;
    v.ct = h;
    v.shape = h->shape;
    v.strides = rowmajor_strides(v.shape);
    vals_[name] = v;
    uses_[name] += 0;
    return vals_[name];
  }
  const float* dptr(const Val& v, const std::string& name) {
    if (v.is_const) return S.dweight(name, "raw");
    return A.ptr(v.buf) + v.off;
  }
  float* out_ptr(const Val& v) { return A.ptr(v.buf) + v.off; }
  Val new_val(const std::vector<int64_t>& shape, bool nhwc) {
    Val v;
    v.shape = shape;
    v.strides = nhwc ? nhwc_strides(shape) : rowmajor_strides(shape);
    v.buf = A.alloc(v.numel());
    return v;
  }
  Val view_of(const Val& src, std::vector<int64_t> shape, std::vector<int64_t> strides, int64_t off) {
    Val v;
    v.shape = std::move(shape);
    v.strides = std::move(strides);
    v.buf = src.buf;
    v.cptr = src.cptr;
    v.off = off;
    A.retain(src.buf);
    return v;
  }
  void step(const std::string& kernel, const std::string& node, double bytes, double flops,
            std::function<cudaError_t(cudaStream_t)> fn) {
    StepInfo si;
    si.kernel = kernel;
    si.node = node;
    si.bytes = bytes;
    si.flops = flops;
    P.info.push_back(si);
    P.steps.push_back(std::move(fn));
  }

  // Copy a strided view into another view of the same shape.
  void copy_into(const Val& src, const Val& dst, const std::string& why) {
    if (src.is_const) {
      // constants used as outputs / concat parts: upload then copy
      throw GraphError{"constant operand not supported in " + why};
    }
    StridedDims sd;
    sd.rank = (int)src.shape.size();
    if (sd.rank > kMaxDims) throw GraphError{"rank > 6 in " + why};
    sd.total = src.numel();
    const bool dst_rm = is_rowmajor(dst);
    for (int d = 0; d < sd.rank; ++d) {
      sd.dims[d] = src.shape[d];
      sd.sa[d] = src.strides[d];
      sd.sb[d] = dst.strides[d];
    }
    const float* a = A.ptr(src.buf) + src.off;
    float* y = A.ptr(dst.buf) + dst.off;
    if (dst_rm) {
      step("copy", why, 8.0 * sd.total, 0, [=](cudaStream_t st) { return launch_copy_strided(a, y, sd, st); });
    } else {
      // dst strided: write through a second strided map (sb)
      step("copy", why, 8.0 * sd.total, 0, [=](cudaStream_t st) { return launch_copy_view(a, y, sd, st); });
    }
  }
  // Ensure a value is laid out as NHWC (4-D) or row-major; returns the value
  // to use (possibly a fresh copy).
  Val as_nhwc(const Val& v, const std::string& why) {
    if (v.is_const) throw GraphError{"constant activation in " + why};
    if (is_nhwc(v) && (v.off % 4) == 0) {
      Val r = v;
      A.retain(r.buf);
      return r;
    }
    Val o = new_val(v.shape, true);
    copy_into(v, o, why + " (to NHWC)");
    return o;
  }
  Val as_rowmajor(const Val& v, const std::string& why) {
    if (v.is_const) throw GraphError{"constant activation in " + why};
    if (is_rowmajor(v) && (v.off % 4) == 0) {
      Val r = v;
      A.retain(r.buf);
      return r;
    }
    Val o = new_val(v.shape, false);
    copy_into(v, o, why + " (to row-major)");
    return o;
  }
  void unref(const Val& v) { A.release(v.buf); }

  // ------------------------------------------------------------ node dispatch
  void plan_node(const Node& n) {
    const std::string& op = n.op;
    if (op == "Conv") return plan_conv(n);
    if (op == "QpcConvT" || op == "ConvTranspose") return plan_convt(n);
    if (op == "QpcConvTPair") return plan_convt_pair(n);
    if (op == "QpcLinear") return plan_linear(n, false);
    if (op == "QpcCtcHead") return plan_linear(n, true);
    if (op == "QpcLayerNorm") return plan_layernorm(n);
    if (op == "QpcAttention") return plan_attention(n);
    if (op == "BatchNormalization") return plan_bn(n);
    if (op == "Relu" || op == "Sigmoid" || op == "HardSigmoid" || op == "FusedGelu" ||
        op == "Erf" || op == "Sqrt" || op == "Clip")
      return plan_unary(n);
    if (op == "Add" || op == "Sub" || op == "Mul" || op == "Div" || op == "Pow") return plan_binary(n);
    if (op == "MulAddScale") return plan_mul_add_scale(n);
    if (op == "Softmax") return plan_softmax(n);
    if (op == "GlobalAveragePool") return plan_gap(n);
    if (op == "AveragePool" || op == "MaxPool") return plan_pool(n);
    if (op == "Resize") return plan_resize(n);
    if (op == "Concat") return plan_concat(n);
    if (op == "Slice") return plan_slice(n);
    if (op == "Transpose") return plan_transpose(n);
    if (op == "Reshape" || op == "Squeeze" || op == "Unsqueeze" || op == "Flatten")
      return plan_reshape(n);
    if (op == "ReduceMean") return plan_reduce_mean(n);
    if (op == "MatMul") return plan_matmul(n);
    if (op == "Identity" || op == "Dropout") {
      const Val& x = get(n.in[0]);
      define(n.out[0], view_of(x, x.shape, x.strides, x.off));
      return;
    }
    if (op == "Gather") return plan_gather(n);
    if (op == "Shape") {
      const Val& x = get(n.in[0]);
      auto h = std::make_shared<HostTensor>();
      h->dtype = QPC_I64;
      h->shape = {(int64_t)x.shape.size()};
      h->i = x.shape;
      Val v;
      v.is_const = true;
      v.owned = h;
      v.ct = h.get();
      v.shape = h->shape;
      v.strides = rowmajor_strides(v.shape);
      define(n.out[0], v);
      return;
    }
    if (op == "Cast") {
      const Val& x = get(n.in[0]);
      if (!x.is_const) {
        Val v = view_of(x, x.shape, x.strides, x.off);  // f32 -> f32 at run time
        define(n.out[0], v);
        return;
      }
      Val v = x;
      define(n.out[0], v);
      return;
    }
    throw GraphError{"no planner for op " + op};
  }

  std::vector<int64_t> const_ints(const std::string& name) {
    const Val& v = get(name);
    if (!v.is_const) throw GraphError{"expected a constant for " + name};
    std::vector<int64_t> r(v.ct->numel());
    for (int64_t k = 0; k < (int64_t)r.size(); ++k) r[k] = (int64_t)v.ct->scalar(k);
    return r;
  }

  // ------------------------------------------------------------ Conv
  // executor.rs:433-652 / conv.rs:222-715.  Routing:
  //   depthwise (group == C == M)        -> dwconv (SIMT, bandwidth bound)
  //   1x1 s1 p0 g1, C % 4 == 0           -> tcgen05 GEMM, rows = pixels
  //   kxk s1 g1, C % 4 == 0              -> tcgen05 implicit GEMM (4-D TMA)
  //   anything else                      -> direct SIMT conv
  void plan_conv(const Node& n) {
    auto fit = fused_dw_.find(n.in[0]);
    if (fit != fused_dw_.end()) {
      plan_dwpw(n, fit->second);
      unref(fit->second.x);
      fused_dw_.erase(fit);
      return;
    }
    const Val& x0 = get(n.in[0]);
    const HostTensor* w = S.weight(n.in[1]);
    if (x0.shape.size() != 4 || w->shape.size() != 4) throw GraphError{"only 2-D convolutions"};
    const int64_t N = x0.shape[0], C = x0.shape[1], H = x0.shape[2], W = x0.shape[3];
    const int64_t M = w->shape[0], cg = w->shape[1], kh = w->shape[2], kw = w->shape[3];
    const int64_t group = n.geti("group", 1);
    auto st = n.getints("strides");
    const int64_t sh = st.size() == 2 ? st[0] : 1, sw = st.size() == 2 ? st[1] : 1;
    int64_t ph, pw, peh, pew;
    resolve_pads(n, H, W, kh, kw, sh, sw, &ph, &pw, &peh, &pew);
    if (group * cg != C || M % group) throw GraphError{"group mismatch"};
    const int64_t oh = (H + ph + peh - kh) / sh + 1, ow = (W + pw + pew - kw) / sw + 1;
    if (oh <= 0 || ow <= 0) throw GraphError{"empty conv output"};
    const std::vector<int64_t> oshape = {N, M, oh, ow};
    const bool has_bias = n.has_in(2);
    const float* bias = has_bias ? S.dweight(n.in[2], "raw") : nullptr;
    const ActParams act = act_of(n);
    ConvGeom g{(int)N, (int)H, (int)W, (int)C, (int)oh, (int)ow, (int)M, (int)kh, (int)kw,
               (int)sh, (int)sw, (int)ph, (int)pw};
    const bool dw = group > 1 && cg == 1 && M == C;
    const bool pw1 = takes_pointwise_gemm(n, *w, H, W);
    const bool kxk_tc = group == 1 && sh == 1 && sw == 1 && (C % 4) == 0 && !pw1 && kh * kw > 1;
    const int math = S.math();
    const bool fold = kxk_tc && math == QPC_MATH_TF32 && takes_fold_conv(n, *w, N, C, H, W);
    if (tf32_rounded_.count(n.in[0]) && !pw1 && !fold)
      throw GraphError{"internal: " + n.name + " reads a tf32-rounded value but is not a TF32 tensor-core conv"};
    const double flops = 2.0 * N * oh * ow * M * cg * kh * kw;
    const double out_bytes = 4.0 * N * oh * ow * M;
    if (dw && !n.has_in(3) && dw_fusable(n, g)) {
      // planned with its pointwise consumer as one kernel (plan_dwpw); the
      // depthwise output is never materialised
      FusedDw f;
      f.x = as_nhwc(x0, n.name);
      f.g = g;
      f.w = S.dweight(n.in[1], "dw");
      f.bias = bias;
      f.act = act;
      f.name = n.name;
      fused_dw_[n.out[0]] = f;
      return;
    }

    // Residual: plain tensor, or (qpc_res_up) the pre-upsample map of a
    // nearest resize to the output size, read through the epilogue's remap
    // on the tensor-core paths and upsampled by a resize step elsewhere.
    const bool has_res = n.has_in(3);
    const bool res_up = has_res && n.geti("qpc_res_up", 0) != 0;
    const bool epi_path = (pw1 || kxk_tc) && !dw;
    Val res;
    int res_h = 0, res_w = 0;  // > 0: remap from a res_h x res_w map
    if (has_res) {
      const Val& r0 = get(n.in[3]);
      if (res_up) {
        if (r0.shape.size() != 4 || r0.shape[0] != N || r0.shape[1] != M)
          throw GraphError{"upsampled residual shape " + shape_str(r0.shape) + " vs " + shape_str(oshape)};
        res = as_nhwc(r0, n.name + " residual");
        if (epi_path) {
          res_h = (int)r0.shape[2];
          res_w = (int)r0.shape[3];
        } else {
          if (M % 4) throw GraphError{"upsampled residual: M % 4 != 0 unsupported"};
          Val up = new_val(oshape, true);
          const float* sp = out_ptr(res);
          float* dp = out_ptr(up);
          const int rh = (int)r0.shape[2], rw = (int)r0.shape[3];
          step("resize", n.name + " residual", 4.0 * (N * M * rh * rw + N * M * oh * ow), 0,
               [=](cudaStream_t s) {
                 return launch_resize_nearest_nhwc(sp, dp, (int)N, rh, rw, (int)M, (int)oh, (int)ow,
                                                   (int)M, 0, s);
               });
          unref(res);
          res = up;
        }
      } else {
        if (r0.shape != oshape) throw GraphError{"residual shape " + shape_str(r0.shape) + " != " + shape_str(oshape)};
        res = as_nhwc(r0, n.name + " residual");
      }
    }
    const double res_bytes = has_res ? (res_h > 0 ? 4.0 * N * M * res_h * res_w : out_bytes) : 0.0;
    Val y;
    int64_t ldo = M;
    if (epi_path && concat_slot(n.out[0], oshape, &y)) ldo = y.strides[3];
    else y = new_val(oshape, true);
    float* yp = out_ptr(y);
    const float* rp = has_res ? out_ptr(res) : nullptr;
    unsigned int* err = device_state(S.device()).err_word;
    const std::string nm = n.name;
    if (dw) {
      Val x = as_nhwc(x0, nm);
      const float* xp = out_ptr(x);
      const float* wt = S.dweight(n.in[1], "dw");
      const double bytes = 4.0 * N * H * W * C + out_bytes + (has_res ? out_bytes : 0);
      ActParams dact = act;
      if (feeds_only_tf32_a(n.out[0], N, M, oh, ow)) {
        dact.round_tf32 = 1;
        tf32_rounded_.insert(n.out[0]);
      }
      step("dwconv", nm, bytes, flops,
           [=](cudaStream_t s) { return launch_dwconv_nhwc(xp, wt, bias, rp, yp, g, dact, s, err); });
      unref(x);
    } else if (pw1) {
      Val x = as_nhwc(x0, nm);
      const float* xp = out_ptr(x);
      auto gi = gated_.find(n.in[0]);
      const float* gate = gi != gated_.end() ? optr(gi->second.g) : nullptr;
      const bool split = math == QPC_MATH_3XTF32;
      const float* wb = S.dweight(n.in[1], split ? "raw.hi" : "raw.rn");
      const float* wl = split ? S.dweight(n.in[1], "raw.lo") : nullptr;
      GemmEpilogue e;
      e.bias = bias;
      e.residual = rp;
      e.out = yp;
      e.ldo = (int)ldo;
      e.ldr = (int)M;
      e.act = act;
      if (res_h > 0) {
        e.rh = res_h;
        e.rw = res_w;
        e.oh = (int)oh;
        e.ow = (int)ow;
      }
      if (gate) {
        e.a_gate = gate;
        e.a_gate_rows = (int)(H * W);
      } else if (tf32_rounded_.count(n.in[0])) {
        e.a_rounded = 1;
      }
      if (feeds_only_tf32_a(n.out[0], N, M, oh, ow)) {
        e.round_out = 1;
        tf32_rounded_.insert(n.out[0]);
      }
      const int64_t rows = N * H * W;
      const double bytes = 4.0 * rows * C + out_bytes + 4.0 * M * C + res_bytes;
      // Narrow K (8 or 16 channels, a quarter / half of the 32-float k-block):
      // P = 32 / C consecutive pixels share one GEMM row against the block
      // diagonal of P filter copies, so no k-block is half padding and each
      // tile carries P times the pixels.  Rows are contiguous, so the input,
      // output and a plain residual are the same memory viewed [rows/P, P*C].
      const int64_t pk = (C == 8 || C == 16) ? 32 / C : 1;
      if (pk > 1 && !gate && (rows % pk) == 0 && M * pk <= 128 && ldo == M && res_h == 0 && (M % 4) == 0) {
        const std::string pv = "pk" + std::to_string(pk);
        const float* pwb = S.dweight(n.in[1], pv + (split ? ".hi" : ".rn"));
        const float* pwl = split ? S.dweight(n.in[1], pv + ".lo") : nullptr;
        GemmEpilogue ep = e;
        ep.bias = has_bias ? S.dweight(n.in[2], "dup" + std::to_string(pk)) : nullptr;
        ep.ldo = (int)(M * pk);
        ep.ldr = (int)(M * pk);
        const int64_t prow = rows / pk;
        const int pc = (int)(C * pk), pm = (int)(M * pk);
        step("gemm_tc", nm, bytes, flops, [=](cudaStream_t s) {
          return launch_gemm_tc(xp, prow, pc, pc, pwb, pwl, pm, ep, math, err, s);
        });
      } else {
        step("gemm_tc", nm, bytes, flops, [=](cudaStream_t s) {
          return launch_gemm_tc(xp, rows, (int)C, (int)C, wb, wl, (int)M, e, math, err, s);
        });
      }
      if (gate) {
        unref(gi->second.x);
        unref(gi->second.g);
        gated_.erase(gi);
      }
      unref(x);
    } else if (kxk_tc) {
      Val x = as_nhwc(x0, nm);
      const float* xp = out_ptr(x);
      const bool split = math == QPC_MATH_3XTF32;
      const float* wb = S.dweight(n.in[1], split ? "kxk.hi" : "kxk.rn");
      const float* wl = split ? S.dweight(n.in[1], "kxk.lo") : nullptr;
      const float* wf = (!split && conv_fold_ok(g)) ? S.dweight(n.in[1], "kxf.rn") : nullptr;
      GemmEpilogue e;
      e.bias = bias;
      e.residual = rp;
      e.out = yp;
      e.ldo = (int)ldo;
      e.ldr = (int)M;
      e.act = act;
      e.a_rounded = (fold && tf32_rounded_.count(n.in[0])) ? 1 : 0;
      if (feeds_only_tf32_a(n.out[0], N, M, oh, ow)) {
        e.round_out = 1;
        tf32_rounded_.insert(n.out[0]);
      }
      if (res_h > 0) {
        e.rh = res_h;
        e.rw = res_w;
        e.oh = (int)oh;
        e.ow = (int)ow;
      }
      const double bytes = 4.0 * N * H * W * C + out_bytes + 4.0 * M * C * kh * kw + res_bytes;
      step("conv_tc", nm, bytes, flops,
           [=](cudaStream_t s) { return launch_conv_tc(xp, g, wb, wl, e, math, err, s, wf); });
      unref(x);
    } else {
      const bool nchw_in = is_rowmajor(x0) && !x0.is_const && (x0.off % 4) == 0;
      Val x = nchw_in ? view_of(x0, x0.shape, x0.strides, x0.off) : as_nhwc(x0, nm);
      const float* xp = out_ptr(x);
      const float* wr = S.dweight(n.in[1], "raw");
      const double bytes = 4.0 * N * H * W * C + out_bytes + (has_res ? out_bytes : 0);
      const int grp = (int)group;
      // host copies (kernel-parameter filters); the session owns the weights
      const HostTensor* wh = S.weight(n.in[1]);
      const HostTensor* bh = has_bias ? S.weight(n.in[2]) : nullptr;
      const float* w_host = (wh && wh->dtype == QPC_F32) ? wh->f.data() : nullptr;
      const float* b_host = (bh && bh->dtype == QPC_F32) ? bh->f.data() : nullptr;
      step("conv_direct", nm, bytes, flops, [=](cudaStream_t s) {
        return launch_conv_direct(xp, nchw_in ? 1 : 0, wr, bias, rp, yp, g, grp, act, s, err, w_host, b_host);
      });
      unref(x);
    }
    if (has_res) unref(res);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ ConvTranspose
  void plan_convt(const Node& n) {
    const Val& x0 = get(n.in[0]);
    const HostTensor* w = S.weight(n.in[1]);
    if (!w || w->shape.size() != 4 || w->shape[2] != 2 || w->shape[3] != 2)
      throw GraphError{"ConvTranspose: only 2x2 s2 p0"};
    auto st = n.getints("strides");
    if (!(st.empty() || (st.size() == 2 && st[0] == 2 && st[1] == 2)))
      throw GraphError{"ConvTranspose: stride must be 2"};
    for (auto p : n.getints("pads"))
      if (p) throw GraphError{"ConvTranspose: pads must be 0"};
    const int64_t N = x0.shape[0], C = x0.shape[1], H = x0.shape[2], W = x0.shape[3];
    if (w->shape[0] != C) throw GraphError{"ConvTranspose: weight C_in mismatch"};
    const int64_t M = w->shape[1];
    const float* bn_a = nullptr;
    const float* bn_b = nullptr;
    if (n.op == "QpcConvT" && n.in.size() >= 6) {
      // BatchNormalization folded into the epilogue, shape.rs:700-733:
      // a = scale / sqrt(var + eps); b = fma(-mean, a, bias); y = fma(x, a, b).
      const HostTensor* sc = S.weight(n.in[2]);
      const HostTensor* bi = S.weight(n.in[3]);
      const HostTensor* me = S.weight(n.in[4]);
      const HostTensor* va = S.weight(n.in[5]);
      const float eps = n.getf("qpc_eps", 1e-5f);
      std::vector<float> a(M), b(M);
      for (int64_t c = 0; c < M; ++c) {
        a[c] = sc->f[c] / std::sqrt(va->f[c] + eps);
        b[c] = std::fma(-me->f[c], a[c], bi->f[c]);
      }
      bn_a = upload_temp(a);
      bn_b = upload_temp(b);
    }
    Val x = as_nhwc(x0, n.name);
    Val y = new_val({N, M, 2 * H, 2 * W}, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    const float* wp = S.dweight(n.in[1], "raw");
    const ActParams act = act_of(n);
    const double bytes = 4.0 * (N * H * W * C + N * 4 * H * W * M);
    unsigned int* err = device_state(S.device()).err_word;
    step("convt2x2", n.name, bytes, 2.0 * N * 4 * H * W * M * C, [=](cudaStream_t s) {
      return launch_convt2x2(xp, wp, bn_a, bn_b, yp, (int)N, (int)H, (int)W, (int)C, (int)M, act, s, err);
    });
    unref(x);
    define(n.out[0], y);
  }

  // ConvT pair (QpcConvTPair, fused at load): the first layer's 2x2 taps as
  // the [128][C] B operand of one GEMM (row 32 (2 dy + dx) + m), its BN as
  // per-column scale / shift, and the second layer's [m][ey][ex] filter; see
  // launch_convt_pair.
  void plan_convt_pair(const Node& n) {
    const Val& x0 = get(n.in[0]);
    const HostTensor* w1 = S.weight(n.in[1]);
    const HostTensor* w2 = S.weight(n.in[6]);
    if (!w1 || w1->shape.size() != 4 || w1->shape[2] != 2 || w1->shape[3] != 2)
      throw GraphError{"ConvTranspose: only 2x2 s2 p0"};
    auto st = n.getints("strides");
    if (!(st.empty() || (st.size() == 2 && st[0] == 2 && st[1] == 2)))
      throw GraphError{"ConvTranspose: stride must be 2"};
    for (auto p : n.getints("pads"))
      if (p) throw GraphError{"ConvTranspose: pads must be 0"};
    const int64_t N = x0.shape[0], C = x0.shape[1], H = x0.shape[2], W = x0.shape[3];
    if (w1->shape[0] != C) throw GraphError{"ConvTranspose: weight C_in mismatch"};
    const int64_t M = w1->shape[1];
    // BN of the first layer as plan_convt computes it (shape.rs:700-733):
    // y = acc * a + b; the scale a goes into the filter, the shift b into
    // the epilogue.
    std::vector<float> bn_a(M, 1.f), bn_b(M, 0.f);
    if (n.has_in(2)) {
      const float eps = n.getf("qpc_eps", 1e-5f);
      const HostTensor* sc = S.weight(n.in[2]);
      const HostTensor* bi = S.weight(n.in[3]);
      const HostTensor* me = S.weight(n.in[4]);
      const HostTensor* va = S.weight(n.in[5]);
      for (int64_t m = 0; m < M; ++m) {
        bn_a[m] = sc->f[m] / std::sqrt(va->f[m] + eps);
        bn_b[m] = std::fma(-me->f[m], bn_a[m], bi->f[m]);
      }
    }
    // B operand [128][C]: column block s = 2 dy + dx, row m < M
    std::vector<float> b1(128 * C, 0.f);
    for (int64_t s = 0; s < 4; ++s)
      for (int64_t m = 0; m < M; ++m)
        for (int64_t c = 0; c < C; ++c)
          b1[(32 * s + m) * C + c] = w1->f[((c * M + m) * 2 + s / 2) * 2 + s % 2] * bn_a[m];
    const bool split = S.math() == MATH_3XTF32;
    std::vector<float> hi(b1.size()), lo(b1.size());
    for (size_t k = 0; k < b1.size(); ++k) {
      hi[k] = tf32_rn_host(b1[k]);
      lo[k] = tf32_rn_host(b1[k] - hi[k]);
    }
    // shift[128], w2[32][4]
    std::vector<float> cs(256, 0.f);
    for (int64_t m = 0; m < M; ++m) {
      for (int64_t s = 0; s < 4; ++s) cs[32 * s + m] = bn_b[m];
      for (int e = 0; e < 4; ++e) cs[128 + 4 * m + e] = w2->f[m * 4 + e];
    }
    const float* b1p = upload_temp(hi);
    const float* b1lo = split ? upload_temp(lo) : nullptr;
    Val x = as_nhwc(x0, n.name);
    Val y = new_val({N, 1, 4 * H, 4 * W}, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    if ((reinterpret_cast<uintptr_t>(xp) | reinterpret_cast<uintptr_t>(yp)) & 15)
      throw GraphError{"internal: unaligned ConvT pair buffers"};
    const ActParams act1 = act_of(n);
    ActParams act2{};
    act2.kind = (int)n.geti("qpc_act2", 0);
    act2.alpha = n.getf("qpc_alpha2", 1.0f / 6.0f);
    act2.beta = n.getf("qpc_beta2", 0.5f);
    act2.c1 = n.getf("qpc_c12", 1.4142135f);
    act2.c2 = n.getf("qpc_c22", 1.0f);
    act2.c3 = n.getf("qpc_c32", 0.5f);
    const double bytes = 4.0 * (N * H * W * C + N * 16 * H * W);
    const double flops = 2.0 * N * H * W * (4 * M * C + 16 * M);
    unsigned int* err = device_state(S.device()).err_word;
    const int math = S.math();
    step("convt_pair", n.name, bytes, flops, [=](cudaStream_t s) {
      return launch_convt_pair(xp, (int)N, (int)H, (int)W, (int)C, (int)M, b1p, b1lo, cs.data(), act1, act2, yp,
                               math, err, s);
    });
    unref(x);
    define(n.out[0], y);
  }

  std::vector<std::unique_ptr<DevBuf>> temps_;
  const float* upload_temp(const std::vector<float>& v) {
    auto b = std::make_unique<DevBuf>(std::max<size_t>(v.size(), 1) * sizeof(float));
    QPC_CUDA_OR_THROW(cudaMemcpy(b->ptr, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice));
    const float* p = b->f();
    P.bufs.push_back(std::move(b));
    return p;
  }

  // ------------------------------------------------------------ BN (unfused)
  void plan_bn(const Node& n) {
    const Val& x0 = get(n.in[0]);
    if (x0.shape.size() != 4) throw GraphError{"BatchNormalization: 4-D input expected"};
    const int64_t C = x0.shape[1];
    const HostTensor* sc = S.weight(n.in[1]);
    const HostTensor* bi = S.weight(n.in[2]);
    const HostTensor* me = S.weight(n.in[3]);
    const HostTensor* va = S.weight(n.in[4]);
    if (!sc || !bi || !me || !va) throw GraphError{"BatchNormalization: parameters must be initializers"};
    const float eps = n.getf("epsilon", 1e-5f);
    std::vector<float> a(C), b(C);
    for (int64_t c = 0; c < C; ++c) {
      a[c] = sc->f[c] / std::sqrt(va->f[c] + eps);
      b[c] = std::fma(-me->f[c], a[c], bi->f[c]);
    }
    const float* ap = upload_temp(a);
    const float* bp = upload_temp(b);
    Val x = as_nhwc(x0, n.name);
    Val y = new_val(x0.shape, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    const int64_t total = x0.numel();
    ActParams act{};
    step("affine", n.name, 8.0 * total, 2.0 * total,
         [=](cudaStream_t s) { return launch_affine_nhwc(xp, ap, bp, yp, total, (int)C, act, s); });
    unref(x);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ elementwise
  // Output layout: NHWC when a runtime operand of the output's 4-D shape is
  // NHWC, else row-major.  Strides are given in the output's physical order.
  StridedDims make_sd(const std::vector<int64_t>& oshape, bool nhwc, const Val* a, const Val* b) {
    StridedDims sd;
    const int r = (int)oshape.size();
    if (r > kMaxDims) throw GraphError{"rank > 6"};
    sd.rank = r;
    sd.total = 1;
    for (auto d : oshape) sd.total *= d;
    auto ext = [&](const Val* v, std::vector<int64_t>& s) {
      s.assign(r, 0);
      if (!v) return;
      const int rv = (int)v->shape.size();
      for (int i = 0; i < r; ++i) {
        const int j = i - (r - rv);
        if (j < 0) continue;
        s[i] = (v->shape[j] == 1 && oshape[i] != 1) ? 0 : v->strides[j];
        if (v->shape[j] == 1) s[i] = 0;
      }
    };
    std::vector<int64_t> s1, s2;
    ext(a, s1);
    ext(b, s2);
    std::vector<int> perm(r);
    std::iota(perm.begin(), perm.end(), 0);
    if (nhwc) perm = {0, 2, 3, 1};
    for (int d = 0; d < r; ++d) {
      sd.dims[d] = oshape[perm[d]];
      sd.sa[d] = s1[perm[d]];
      sd.sb[d] = s2[perm[d]];
    }
    return sd;
  }
  std::vector<int64_t> bcast(const std::vector<int64_t>& a, const std::vector<int64_t>& b) {
    const size_t r = std::max(a.size(), b.size());
    std::vector<int64_t> o(r);
    for (size_t i = 0; i < r; ++i) {
      const int64_t da = i + a.size() >= r ? a[i + a.size() - r] : 1;
      const int64_t db = i + b.size() >= r ? b[i + b.size() - r] : 1;
      if (da != db && da != 1 && db != 1) throw GraphError{"broadcast mismatch " + shape_str(a) + " vs " + shape_str(b)};
      o[i] = std::max(da, db);
    }
    return o;
  }
  bool pick_nhwc(const std::vector<int64_t>& oshape, const Val& a, const Val* b) {
    if (oshape.size() != 4) return false;
    if (!a.is_const && a.shape == oshape && is_nhwc(a)) return true;
    if (b && !b->is_const && b->shape == oshape && is_nhwc(*b)) return true;
    return false;
  }
  // A device pointer + view for any operand (constants are uploaded raw).
  Val operand(const std::string& name) {
    const Val& v = get(name);
    if (!v.is_const) return v;
    Val c = v;
    c.cptr = S.dweight(name, "raw");
    return c;
  }
  const float* optr(const Val& v) { return v.cptr ? v.cptr + v.off : A.ptr(v.buf) + v.off; }

  void plan_unary(const Node& n) {
    Val x = operand(n.in[0]);
    ActParams act{};
    const std::string& op = n.op;
    if (op == "Relu") act.kind = ACT_RELU;
    else if (op == "Sigmoid") act.kind = ACT_SIGMOID;
    else if (op == "HardSigmoid") {
      act.kind = ACT_HARDSIGMOID;
      act.alpha = n.getf("alpha", 0.2f);
      act.beta = n.getf("beta", 0.5f);
    } else if (op == "FusedGelu") {
      act.kind = ACT_GELU;
      act.c1 = n.getf("c1", 1.4142135f);
      act.c2 = n.getf("c2", 1.0f);
      act.c3 = n.getf("c3", 0.5f);
    } else if (op == "Sqrt") act.kind = 100;
    else if (op == "Erf") act.kind = 102;
    else if (op == "Clip") {
      act.kind = 101;
      act.alpha = n.getf("min", -3.4e38f);
      act.beta = n.getf("max", 3.4e38f);
      if (n.has_in(1)) act.alpha = (float)get(n.in[1]).ct->scalar();
      if (n.has_in(2)) act.beta = (float)get(n.in[2]).ct->scalar();
    }
    const bool nhwc = pick_nhwc(x.shape, x, nullptr);
    Val y = new_val(x.shape, nhwc);
    StridedDims sd = make_sd(x.shape, nhwc, &x, nullptr);
    const float* xp = optr(x);
    float* yp = out_ptr(y);
    step("unary", n.name, 8.0 * sd.total, sd.total, [=](cudaStream_t s) { return launch_unary(xp, yp, sd, act, s); });
    define(n.out[0], y);
  }

  // SE gate: Mul(x [N,C,H,W], g [N,C,1,1]) whose only consumer is a 1x1
  // stride-1 unpadded Conv reading it as its input is not materialised; the
  // conv's GEMM multiplies A by g as it rounds A on chip (same f32 products).
  struct Gated {
    Val x, g;
  };
  std::map<std::string, Gated> gated_;

  bool try_gate(const Node& n) {
    const std::string& out = n.out[0];
    for (auto& go : S.graph_outputs())
      if (go == out) return false;
    auto cit = consumers_.find(out);
    if (cit == consumers_.end() || cit->second.size() != 1) return false;
    const Node& c = S.nodes()[cit->second[0]];
    if (c.op != "Conv" || c.in.empty() || c.in[0] != out || c.has_in(4)) return false;
    for (size_t k = 1; k < c.in.size(); ++k)
      if (c.in[k] == out) return false;
    Val a = operand(n.in[0]), b = operand(n.in[1]);
    if (a.is_const || b.is_const || a.shape.size() != 4 || b.shape.size() != 4) return false;
    const bool a_is_x = b.shape[2] == 1 && b.shape[3] == 1;
    const Val& x = a_is_x ? a : b;
    const Val& g = a_is_x ? b : a;
    const int64_t N = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
    if (g.shape != std::vector<int64_t>{N, C, 1, 1} || !is_rowmajor(g) || (g.off % 4) || (C % 4) || C == 8 ||
        C == 16 || H * W < 2)
      return false;
    const HostTensor* w = S.weight(c.in[1]);
    if (!w || w->shape.size() != 4 || w->shape[1] != C || w->shape[2] != 1 || w->shape[3] != 1 ||
        c.geti("group", 1) != 1)
      return false;
    auto st = c.getints("strides");
    if (st.size() == 2 && (st[0] != 1 || st[1] != 1)) return false;
    int64_t ph, pw, peh, pew;
    resolve_pads(c, H, W, 1, 1, 1, 1, &ph, &pw, &peh, &pew);
    if (ph || pw || peh || pew) return false;
    Gated gt;
    gt.x = as_nhwc(x, n.name);
    gt.g = g;
    A.retain(g.buf);
    Val y = gt.x;  // what the conv reads as its input; the gate rides along
    A.retain(y.buf);
    define(out, y);
    gated_[out] = gt;
    return true;
  }

  void plan_binary(const Node& n) {
    if (n.op == "Mul" && try_gate(n)) return;
    Val a = operand(n.in[0]);
    Val b = operand(n.in[1]);
    int op = 0;
    if (n.op == "Sub") op = 1;
    else if (n.op == "Mul") op = 2;
    else if (n.op == "Div") op = 3;
    else if (n.op == "Pow") op = 4;
    const auto oshape = bcast(a.shape, b.shape);
    const bool nhwc = pick_nhwc(oshape, a, &b);
    Val y = new_val(oshape, nhwc);
    StridedDims sd = make_sd(oshape, nhwc, &a, &b);
    const float* ap = optr(a);
    const float* bp = optr(b);
    float* yp = out_ptr(y);
    ActParams post{};
    step("binary", n.name, 12.0 * sd.total, sd.total,
         [=](cudaStream_t s) { return launch_binary(ap, bp, yp, sd, op, post, s); });
    define(n.out[0], y);
  }

  // executor.rs:808-884 MulAddScale: per-channel gate fast path, else Mul then Add.
  void plan_mul_add_scale(const Node& n) {
    Val f = operand(n.in[0]);
    Val g = operand(n.in[1]);
    Val r = operand(n.in[2]);
    if (f.shape.size() == 4 && r.shape == f.shape && !f.is_const && !r.is_const && !g.is_const &&
        (g.numel() == f.shape[1] || g.numel() == f.shape[0] * f.shape[1]) && is_rowmajor(g)) {
      Val fx = as_nhwc(f, n.name);
      Val rx = as_nhwc(r, n.name);
      Val y = new_val(f.shape, true);
      const float* fp = out_ptr(fx);
      const float* gp = optr(g);
      const float* rp = out_ptr(rx);
      float* yp = out_ptr(y);
      const int64_t total = f.numel();
      const int hw = (int)(f.shape[2] * f.shape[3]), c = (int)f.shape[1];
      const int per_n = g.numel() != f.shape[1] ? 1 : 0;
      step("mul_add_scale", n.name, 12.0 * total, 2.0 * total,
           [=](cudaStream_t s) { return launch_mul_add_scale_nhwc(fp, gp, rp, yp, total, hw, c, per_n, s); });
      unref(fx);
      unref(rx);
      define(n.out[0], y);
      return;
    }
    // generic: t = f * g ; y = t + r (two roundings, elementwise.rs:134-181)
    const auto s1 = bcast(f.shape, g.shape);
    const bool nh1 = pick_nhwc(s1, f, &g);
    Val t = new_val(s1, nh1);
    {
      StridedDims sd = make_sd(s1, nh1, &f, &g);
      const float* fp = optr(f);
      const float* gp = optr(g);
      float* tp = out_ptr(t);
      ActParams post{};
      step("binary", n.name + "/mul", 12.0 * sd.total, sd.total,
           [=](cudaStream_t s) { return launch_binary(fp, gp, tp, sd, 2, post, s); });
    }
    const auto s2 = bcast(s1, r.shape);
    const bool nh2 = pick_nhwc(s2, t, &r);
    Val y = new_val(s2, nh2);
    {
      StridedDims sd = make_sd(s2, nh2, &t, &r);
      const float* tp = out_ptr(t);
      const float* rp = optr(r);
      float* yp = out_ptr(y);
      ActParams post{};
      step("binary", n.name + "/add", 12.0 * sd.total, sd.total,
           [=](cudaStream_t s) { return launch_binary(tp, rp, yp, sd, 0, post, s); });
    }
    unref(t);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ LayerNorm
  // QpcAttention: [B, T, 3*H*D] qkv (row-major) -> [B, T, H*D].
  void plan_attention(const Node& n) {
    const Val& x0 = get(n.in[0]);
    const int64_t H = n.geti("heads", 0), D = n.geti("head_dim", 0);
    if (x0.shape.size() != 3 || x0.shape[2] != 3 * H * D) throw GraphError{"attention input " + shape_str(x0.shape)};
    const int64_t B = x0.shape[0], T = x0.shape[1];
    Val x = as_rowmajor(x0, n.name);
    Val y = new_val({B, T, H * D}, false);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    const float scale = n.getf("scale", 1.0f);
    const double bytes = 4.0 * B * T * 4 * H * D;
    const double flops = 4.0 * B * H * T * T * D;
    step("attention", n.name, bytes, flops, [=](cudaStream_t st) {
      return launch_attention(xp, B, (int)T, (int)H, (int)D, scale, yp, st);
    });
    unref(x);
    define(n.out[0], y);
  }

  void plan_layernorm(const Node& n) {
    const Val& x0 = get(n.in[0]);
    Val x = as_rowmajor(x0, n.name);
    const int64_t C = x.shape.back();
    const int64_t rows = x.numel() / C;
    Val y = new_val(x.shape, false);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    const float* gp = n.has_in(1) ? S.dweight(n.in[1], "raw") : nullptr;
    const float* bp = n.has_in(2) ? S.dweight(n.in[2], "raw") : nullptr;
    const float eps = n.getf("qpc_eps", 1e-5f);
    const int rnd = feeds_only_tf32_a(n.out[0], 0, C, 0, 0) ? 1 : 0;
    if (rnd) tf32_rounded_.insert(n.out[0]);
    step("layernorm", n.name, 8.0 * x.numel(), 8.0 * x.numel(),
         [=](cudaStream_t s) { return launch_layernorm(xp, gp, bp, yp, rows, (int)C, eps, rnd, s); });
    unref(x);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ Linear / head
  // QpcLinear(x[..., K], W[K, N], b?, residual?) on the tensor-core GEMM.
  // QpcCtcHead: the same GEMM followed by the row argmax exit.
  void plan_linear(const Node& n, bool head) {
    const Val& x0 = get(n.in[0]);
    const HostTensor* w = S.weight(n.in[1]);
    const int64_t K = w->shape[0], Nn = w->shape[1];
    if (x0.shape.empty() || x0.shape.back() != K) throw GraphError{"MatMul inner dim mismatch"};
    Val x = as_rowmajor(x0, n.name);
    const int64_t rows = x.numel() / K;
    std::vector<int64_t> oshape = x.shape;
    oshape.back() = Nn;
    const int math = S.math();
    const bool split = math == QPC_MATH_3XTF32;
    const float* wb = S.dweight(n.in[1], split ? "nk.hi" : "nk.rn");
    const float* wl = split ? S.dweight(n.in[1], "nk.lo") : nullptr;
    const float* bias = n.has_in(2) ? S.dweight(n.in[2], "raw") : nullptr;
    Val res;
    const bool has_res = n.has_in(3);
    if (has_res) {
      const Val& r0 = get(n.in[3]);
      if (r0.shape != oshape) throw GraphError{"residual shape mismatch"};
      res = as_rowmajor(r0, n.name + " residual");
    }
    unsigned int* err = device_state(S.device()).err_word;
    const double flops = 2.0 * rows * K * Nn;
    const float* xp = out_ptr(x);
    // A stored tf32-rounded by its producer (the GEMM skips its rounding pass)
    const int a_rounded = (!split && tf32_rounded_.count(n.in[0])) ? 1 : 0;
    if (!head) {
      Val y = new_val(oshape, false);
      GemmEpilogue e;
      e.bias = bias;
      e.residual = has_res ? out_ptr(res) : nullptr;
      e.out = out_ptr(y);
      e.ldo = (int)Nn;
      e.ldr = (int)Nn;
      e.act = act_of(n);
      e.a_rounded = a_rounded;
      if (feeds_only_tf32_a(n.out[0], 0, Nn, 0, 0)) {
        e.round_out = 1;
        tf32_rounded_.insert(n.out[0]);
      }
      step("gemm_tc", n.name, 4.0 * (rows * K + rows * Nn + K * Nn), flops, [=](cudaStream_t s) {
        return launch_gemm_tc(xp, rows, (int)K, (int)K, wb, wl, (int)Nn, e, math, err, s);
      });
      unref(x);
      if (has_res) unref(res);
      define(n.out[0], y);
      return;
    }
    // CTC head with the argmax exit: the GEMM epilogue reduces each row of
    // logits per column tile to (max, argmax, sum exp) partials (scratch), the
    // combine step emits (val = softmax prob of the first strict max, idx bits).
    if (has_res) throw GraphError{"CTC head with a residual"};
    const int ntiles = gemm_tc_col_tiles((int)Nn, math);
    Val part = new_val({(int64_t)ntiles * rows * 4}, false);
    // partials written and read: one per (CTA, epilogue group, row block)
    const int64_t mblk = (rows + 127) / 128;
    const double part_bytes =
        16.0 * 128 * (double)std::min<int64_t>(mblk * ntiles, 2 * (mblk + head_workers(rows, ntiles, math)));
    float4* pp4 = reinterpret_cast<float4*>(out_ptr(part));
    GemmEpilogue e;
    e.bias = bias;
    e.partials = pp4;
    e.out = nullptr;
    e.ldo = (int)Nn;
    e.act = act_of(n);
    e.a_rounded = a_rounded;
    step("head_gemm", n.name, 4.0 * (rows * K + K * Nn) + part_bytes, flops,
         [=](cudaStream_t s) { return launch_gemm_tc(xp, rows, (int)K, (int)K, wb, wl, (int)Nn, e, math, err, s); });
    unref(x);
    std::vector<int64_t> pshape = oshape;
    pshape.back() = 2;
    Val pr = new_val(pshape, false);
    float* prp = out_ptr(pr);
    step("head_combine", n.name, part_bytes + 8.0 * rows, 0,
         [=](cudaStream_t s) { return launch_argmax_combine(pp4, ntiles, rows, math, prp, s); });
    unref(part);
    define(n.out[0], pr);
  }

  // ------------------------------------------------------------ Softmax
  void plan_softmax(const Node& n) {
    const Val& x0 = get(n.in[0]);
    int64_t axis = n.geti("axis", -1);
    if (axis < 0) axis += (int64_t)x0.shape.size();
    if (axis != (int64_t)x0.shape.size() - 1) throw GraphError{"Softmax: only the last axis"};
    Val x = as_rowmajor(x0, n.name);
    const int64_t inner = x.shape.back(), rows = x.numel() / inner;
    const bool exit_here = S.argmax_exit() &&
        std::find(S.graph_outputs().begin(), S.graph_outputs().end(), n.out[0]) != S.graph_outputs().end();
    const float* xp = out_ptr(x);
    if (exit_here) {
      std::vector<int64_t> pshape = x.shape;
      pshape.back() = 2;
      Val pr = new_val(pshape, false);
      float* pp = out_ptr(pr);
      step("head_argmax", n.name, 4.0 * rows * inner, 3.0 * rows * inner,
           [=](cudaStream_t s) { return launch_softmax_argmax(xp, pp, rows, (int)inner, s); });
      unref(x);
      define(n.out[0], pr);
      return;
    }
    Val y = new_val(x.shape, false);
    float* yp = out_ptr(y);
    step("softmax", n.name, 8.0 * x.numel(), 4.0 * x.numel(),
         [=](cudaStream_t s) { return launch_softmax_rows(xp, yp, rows, (int)inner, s); });
    unref(x);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ pooling
  void plan_gap(const Node& n) {
    const Val& x0 = get(n.in[0]);
    Val x = as_nhwc(x0, n.name);
    const int64_t N = x.shape[0], C = x.shape[1], HW = x.shape[2] * x.shape[3];
    Val y = new_val({N, C, 1, 1}, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    step("gap", n.name, 4.0 * (N * C * HW + N * C), N * C * HW,
         [=](cudaStream_t s) { return launch_gap_nhwc(xp, yp, (int)N, (int)HW, (int)C, s); });
    unref(x);
    define(n.out[0], y);
  }

  void plan_pool(const Node& n) {
    const Val& x0 = get(n.in[0]);
    auto ks = n.getints("kernel_shape");
    if (ks.size() != 2) throw GraphError{"kernel_shape required"};
    auto st = n.getints("strides");
    const int64_t sh = st.size() == 2 ? st[0] : 1, sw = st.size() == 2 ? st[1] : 1;
    const int64_t N = x0.shape[0], C = x0.shape[1], H = x0.shape[2], W = x0.shape[3];
    int64_t ph, pw, peh, pew;
    resolve_pads(n, H, W, ks[0], ks[1], sh, sw, &ph, &pw, &peh, &pew);
    const int64_t oh = (H + ph + peh - ks[0]) / sh + 1, ow = (W + pw + pew - ks[1]) / sw + 1;
    Val x = as_nhwc(x0, n.name);
    Val y = new_val({N, C, oh, ow}, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    const int is_max = n.op == "MaxPool";
    step("pool2d", n.name, 4.0 * (N * C * H * W + N * C * oh * ow), N * C * oh * ow * ks[0] * ks[1],
         [=](cudaStream_t s) {
           return launch_pool2d_nhwc(xp, yp, (int)N, (int)H, (int)W, (int)C, (int)oh, (int)ow,
                                     (int)ks[0], (int)ks[1], (int)sh, (int)sw, (int)ph, (int)pw,
                                     is_max, s);
         });
    unref(x);
    define(n.out[0], y);
  }

  // executor.rs:1070-1183 Resize (nearest): sizes (inputs[3]) or scales (inputs[2]).
  void plan_resize(const Node& n) {
    const Val& x0 = get(n.in[0]);
    int64_t oh, ow;
    if (n.has_in(3)) {
      auto sz = const_ints(n.in[3]);
      oh = sz[sz.size() - 2];
      ow = sz[sz.size() - 1];
    } else if (n.has_in(2)) {
      const Val& sc = get(n.in[2]);
      const float s_h = (float)sc.ct->scalar(sc.ct->numel() - 2);
      const float s_w = (float)sc.ct->scalar(sc.ct->numel() - 1);
      oh = (int64_t)((float)x0.shape[2] * s_h);
      ow = (int64_t)((float)x0.shape[3] * s_w);
    } else {
      throw GraphError{"Resize: no scales/sizes"};
    }
    const int64_t N = x0.shape[0], C = x0.shape[1], H = x0.shape[2], W = x0.shape[3];
    Val x = as_nhwc(x0, n.name);
    const std::vector<int64_t> oshape = {N, C, oh, ow};
    if (C % 4) throw GraphError{"Resize: C % 4 != 0 unsupported"};
    Val y;
    int64_t ldc = C;
    std::string co;
    if (concat_slot(n.out[0], oshape, &y, &co)) {
      const bool rnd = feeds_only_tf32_a(n.out[0], N, C, oh, ow);
      if (rnd) tf32_rounded_.insert(n.out[0]);
      pending_resize_[co].push_back({x, y, (int)H, (int)W, (int)C, rnd, n.name});
      define(n.out[0], y);
      return;
    }
    y = new_val(oshape, true);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    step("resize", n.name, 4.0 * (N * C * H * W + N * C * oh * ow), 0, [=](cudaStream_t s) {
      return launch_resize_nearest_nhwc(xp, yp, (int)N, (int)H, (int)W, (int)C, (int)oh, (int)ow,
                                        (int)ldc, 0, s);
    });
    unref(x);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ Concat
  void plan_concat(const Node& n) {
    flush_resizes(n.out[0]);
    std::vector<Val> parts;
    for (auto& nm : n.in) parts.push_back(operand(nm));
    const int64_t r = (int64_t)parts[0].shape.size();
    int64_t axis = n.geti("axis", 0);
    if (axis < 0) axis += r;
    std::vector<int64_t> oshape = parts[0].shape;
    oshape[axis] = 0;
    for (auto& p : parts) {
      if ((int64_t)p.shape.size() != r) throw GraphError{"Concat rank mismatch"};
      oshape[axis] += p.shape[axis];
    }
    const bool nhwc = r == 4 && axis == 1;
    Val y;
    auto pre = concat_bufs_.find(n.out[0]);
    if (pre != concat_bufs_.end()) {
      y = pre->second;  // takes over the early allocation's reference
      concat_bufs_.erase(pre);
      if (y.shape != oshape) throw GraphError{"internal: concat buffer shape"};
    } else {
      y = new_val(oshape, nhwc);
    }
    int64_t off = 0;
    for (size_t k = 0; k < parts.size(); ++k) {
      const Val& p = parts[k];
      if (p.is_const) throw GraphError{"Concat of a constant"};
      Val dst;
      dst.shape = p.shape;
      dst.strides = y.strides;
      dst.buf = y.buf;
      dst.off = y.off + off * y.strides[axis];
      const bool in_place = p.buf == dst.buf && p.off == dst.off && p.strides == dst.strides;
      if (!in_place) {
        if (nhwc && is_nhwc(p) && (p.off % 4) == 0 && (p.shape[1] % 4) == 0 && (oshape[1] % 4) == 0 &&
            (off % 4) == 0) {
          const float* src = out_ptr(p);
          float* dp = A.ptr(y.buf) + y.off;
          const int64_t pix = p.shape[0] * p.shape[2] * p.shape[3];
          const int pc = (int)p.shape[1], ldc = (int)oshape[1], coff = (int)off;
          step("copy", n.name + "/part" + std::to_string(k), 8.0 * p.numel(), 0, [=](cudaStream_t st) {
            return launch_copy_channels(src, dp, pix, pc, ldc, coff, st);
          });
        } else {
          copy_into(p, dst, n.name + "/part" + std::to_string(k));
        }
      }
      off += p.shape[axis];
    }
    bool all_rounded = true;
    for (auto& nm : n.in) all_rounded = all_rounded && tf32_rounded_.count(nm) > 0;
    if (all_rounded) tf32_rounded_.insert(n.out[0]);
    define(n.out[0], y);
  }

  // ------------------------------------------------------------ views
  void plan_transpose(const Node& n) {
    const Val& x = get(n.in[0]);
    auto perm = n.getints("perm");
    const size_t r = x.shape.size();
    if (perm.empty()) {
      perm.resize(r);
      for (size_t i = 0; i < r; ++i) perm[i] = (int64_t)(r - 1 - i);
    }
    std::vector<int64_t> s(r), st(r);
    for (size_t i = 0; i < r; ++i) {
      s[i] = x.shape[perm[i]];
      st[i] = x.strides[perm[i]];
    }
    if (x.is_const) throw GraphError{"Transpose of a constant"};
    define(n.out[0], view_of(x, s, st, x.off));
  }

  // Try to express `shape` as a strided view of `x` without copying
  // (merging / splitting dims whose strides are compatible).
  bool reshape_view(const Val& x, const std::vector<int64_t>& shape, std::vector<int64_t>* out) {
    // drop size-1 dims of the source
    std::vector<int64_t> os, ost;
    for (size_t i = 0; i < x.shape.size(); ++i)
      if (x.shape[i] != 1) {
        os.push_back(x.shape[i]);
        ost.push_back(x.strides[i]);
      }
    out->assign(shape.size(), 0);
    size_t oi = 0, ni = 0;
    const size_t on = os.size(), nn = shape.size();
    while (ni < nn && shape[ni] == 1) (*out)[ni++] = 0;
    while (oi < on && ni < nn) {
      // group source dims [oi, oj) and target dims [ni, nj) with equal products
      int64_t np = shape[ni], op = os[oi];
      size_t oj = oi + 1, nj = ni + 1;
      while (np != op) {
        if (np < op) {
          if (nj >= nn) return false;
          np *= shape[nj++];
        } else {
          if (oj >= on) return false;
          op *= os[oj++];
        }
      }
      for (size_t k = oi; k + 1 < oj; ++k)
        if (ost[k] != ost[k + 1] * os[k + 1]) return false;  // source group must be contiguous
      (*out)[nj - 1] = ost[oj - 1];
      for (size_t k = nj - 1; k > ni; --k) (*out)[k - 1] = (*out)[k] * shape[k];
      oi = oj;
      ni = nj;
      while (ni < nn && shape[ni] == 1) (*out)[ni++] = 0;
    }
    return oi == on && ni == nn;
  }

  void plan_reshape(const Node& n) {
    const Val& x = get(n.in[0]);
    std::vector<int64_t> shape;
    const int64_t total = x.numel();
    if (n.op == "Reshape") {
      auto req = const_ints(n.in[1]);
      int64_t known = 1, infer = -1;
      for (size_t i = 0; i < req.size(); ++i) {
        int64_t d = req[i];
        if (d == 0 && n.geti("allowzero", 0) == 0) d = x.shape[i];
        if (d == -1) {
          infer = (int64_t)i;
          shape.push_back(1);
        } else {
          shape.push_back(d);
          known *= d;
        }
      }
      if (infer >= 0) shape[infer] = known ? total / known : 0;
    } else if (n.op == "Flatten") {
      int64_t axis = n.geti("axis", 1);
      if (axis < 0) axis += (int64_t)x.shape.size();
      int64_t a = 1, b = 1;
      for (int64_t i = 0; i < (int64_t)x.shape.size(); ++i) (i < axis ? a : b) *= x.shape[i];
      shape = {a, b};
    } else if (n.op == "Squeeze") {
      auto axes = n.getints("axes");
      if (axes.empty() && n.has_in(1)) axes = const_ints(n.in[1]);
      const int64_t r = (int64_t)x.shape.size();
      for (auto& a : axes)
        if (a < 0) a += r;
      for (int64_t i = 0; i < r; ++i) {
        const bool sq = axes.empty() ? x.shape[i] == 1 : std::count(axes.begin(), axes.end(), i) > 0;
        if (!sq) shape.push_back(x.shape[i]);
      }
    } else {  // Unsqueeze
      auto axes = n.getints("axes");
      if (axes.empty() && n.has_in(1)) axes = const_ints(n.in[1]);
      const int64_t r = (int64_t)x.shape.size() + (int64_t)axes.size();
      for (auto& a : axes)
        if (a < 0) a += r;
      size_t k = 0;
      for (int64_t i = 0; i < r; ++i) {
        if (std::count(axes.begin(), axes.end(), i)) shape.push_back(1);
        else shape.push_back(x.shape[k++]);
      }
    }
    int64_t chk = 1;
    for (auto d : shape) chk *= d;
    if (chk != total) throw GraphError{"reshape numel mismatch " + shape_str(x.shape) + " -> " + shape_str(shape)};
    if (x.is_const) {
      Val v = x;
      auto h = std::make_shared<HostTensor>(*x.ct);
      h->shape = shape;
      v.owned = h;
      v.ct = h.get();
      v.shape = shape;
      v.strides = rowmajor_strides(shape);
      define(n.out[0], v);
      return;
    }
    std::vector<int64_t> st;
    if (reshape_view(x, shape, &st)) {
      define(n.out[0], view_of(x, shape, st, x.off));
      return;
    }
    Val c = as_rowmajor(x, n.name);
    Val v = view_of(c, shape, rowmajor_strides(shape), c.off);
    unref(c);
    define(n.out[0], v);
  }

  void plan_slice(const Node& n) {
    const Val& x = get(n.in[0]);
    const int64_t r = (int64_t)x.shape.size();
    std::vector<int64_t> starts, ends, axes, steps;
    if (n.has_in(1)) {
      starts = const_ints(n.in[1]);
      ends = const_ints(n.in[2]);
      if (n.has_in(3)) axes = const_ints(n.in[3]);
      if (n.has_in(4)) steps = const_ints(n.in[4]);
    } else {
      starts = n.getints("starts");
      ends = n.getints("ends");
      axes = n.getints("axes");
    }
    if (axes.empty())
      for (size_t i = 0; i < starts.size(); ++i) axes.push_back((int64_t)i);
    if (steps.empty()) steps.assign(starts.size(), 1);
    std::vector<int64_t> shape = x.shape, st = x.strides;
    int64_t off = x.off;
    for (size_t k = 0; k < starts.size(); ++k) {
      int64_t a = axes[k] < 0 ? axes[k] + r : axes[k];
      const int64_t dim = x.shape[a], step_ = steps[k];
      if (step_ <= 0) throw GraphError{"Slice: only positive steps"};
      int64_t s0 = starts[k] < 0 ? starts[k] + dim : starts[k];
      int64_t e0 = ends[k] < 0 ? ends[k] + dim : ends[k];
      s0 = std::clamp<int64_t>(s0, 0, dim);
      e0 = std::clamp<int64_t>(e0, 0, dim);
      const int64_t cnt = e0 > s0 ? (e0 - s0 + step_ - 1) / step_ : 0;
      off += s0 * x.strides[a];
      shape[a] = cnt;
      st[a] = x.strides[a] * step_;
    }
    if (x.is_const) throw GraphError{"Slice of a constant"};
    define(n.out[0], view_of(x, shape, st, off));
  }

  void plan_gather(const Node& n) {
    const Val& x = get(n.in[0]);
    const Val& idx = get(n.in[1]);
    if (!idx.is_const || idx.ct->numel() != 1 || !idx.shape.empty())
      throw GraphError{"Gather: only a scalar constant index"};
    const int64_t r = (int64_t)x.shape.size();
    int64_t axis = n.geti("axis", 0);
    if (axis < 0) axis += r;
    int64_t k = (int64_t)idx.ct->scalar();
    if (k < 0) k += x.shape[axis];
    std::vector<int64_t> shape, st;
    for (int64_t i = 0; i < r; ++i)
      if (i != axis) {
        shape.push_back(x.shape[i]);
        st.push_back(x.strides[i]);
      }
    if (x.is_const) throw GraphError{"Gather of a constant"};
    define(n.out[0], view_of(x, shape, st, x.off + k * x.strides[axis]));
  }

  // shape.rs:510-566 (contiguous reduced axes, f64 sums).
  void plan_reduce_mean(const Node& n) {
    const Val& x0 = get(n.in[0]);
    std::vector<int64_t> axes = n.getints("axes");
    if (axes.empty() && n.has_in(1)) axes = const_ints(n.in[1]);
    const int64_t r = (int64_t)x0.shape.size();
    std::vector<bool> red(r, axes.empty());
    for (auto a : axes) red[a < 0 ? a + r : a] = true;
    int64_t outer = 1, mid = 1, inner = 1;
    int state = 0;
    for (int64_t i = 0; i < r; ++i) {
      if (red[i]) {
        if (state == 2) throw GraphError{"ReduceMean: non-contiguous axes"};
        mid *= x0.shape[i];
        state = 1;
      } else if (state == 0) outer *= x0.shape[i];
      else {
        inner *= x0.shape[i];
        state = 2;
      }
    }
    const bool keep = n.geti("keepdims", 1) != 0;
    std::vector<int64_t> shape;
    for (int64_t i = 0; i < r; ++i) {
      if (!red[i]) shape.push_back(x0.shape[i]);
      else if (keep) shape.push_back(1);
    }
    Val x = as_rowmajor(x0, n.name);
    Val y = new_val(shape, false);
    const float* xp = out_ptr(x);
    float* yp = out_ptr(y);
    step("reduce_mean", n.name, 4.0 * (x.numel() + y.numel()), x.numel(),
         [=](cudaStream_t s) { return launch_reduce_mean(xp, yp, outer, mid, inner, s); });
    unref(x);
    define(n.out[0], y);
  }

  // MatMul with a runtime B (attention) or a constant B the GEMM cannot take:
  // shape.rs:669-697 row outer product, strided operands, up to 2 batch dims.
  void plan_matmul(const Node& n) {
    Val a = operand(n.in[0]);
    Val b = operand(n.in[1]);
    if (a.shape.size() < 2 || b.shape.size() < 2) throw GraphError{"MatMul rank < 2"};
    const int ra = (int)a.shape.size(), rb = (int)b.shape.size();
    const int64_t M = a.shape[ra - 2], K = a.shape[ra - 1], K2 = b.shape[rb - 2], Nn = b.shape[rb - 1];
    if (K != K2) throw GraphError{"MatMul inner dim mismatch"};
    std::vector<int64_t> ba(a.shape.begin(), a.shape.end() - 2), bb(b.shape.begin(), b.shape.end() - 2);
    auto bs = bcast(ba, bb);
    if (bs.size() > 2) throw GraphError{"MatMul: more than 2 batch dims"};
    while (bs.size() < 2) bs.insert(bs.begin(), 1);
    auto bstride = [&](const Val& v, int rv, int which) -> int64_t {
      // stride of batch dim `which` (0/1 of the 2-dim padded batch) in v
      const int nb = rv - 2;
      const int j = which - (2 - nb);
      if (j < 0) return 0;
      return v.shape[j] == 1 ? 0 : v.strides[j];
    };
    BmmDims d;
    d.nb0 = (int)bs[0];
    d.nb1 = (int)bs[1];
    d.m = (int)M;
    d.n = (int)Nn;
    d.k = (int)K;
    d.sa0 = bstride(a, ra, 0);
    d.sa1 = bstride(a, ra, 1);
    d.sam = a.strides[ra - 2];
    d.sak = a.strides[ra - 1];
    d.sb0 = bstride(b, rb, 0);
    d.sb1 = bstride(b, rb, 1);
    d.sbk = b.strides[rb - 2];
    d.sbn = b.strides[rb - 1];
    std::vector<int64_t> oshape;
    for (size_t i = 0; i < std::max(ba.size(), bb.size()); ++i) oshape.push_back(bs[2 - std::max(ba.size(), bb.size()) + i]);
    oshape.push_back(M);
    oshape.push_back(Nn);
    Val y = new_val(oshape, false);
    const float* ap = optr(a);
    const float* bp = optr(b);
    float* yp = out_ptr(y);
    const double flops = 2.0 * d.nb0 * d.nb1 * M * Nn * K;
    step("bmm_small", n.name, 4.0 * (a.numel() + b.numel() + y.numel()), flops,
         [=](cudaStream_t s) { return launch_bmm_small(ap, bp, yp, d, s); });
    define(n.out[0], y);
  }
};

// ================================================================ plans / runs
static std::string shape_key(const qpc_tensor* in, int n) {
  std::ostringstream o;
  for (int k = 0; k < n; ++k) {
    o << (in[k].name ? in[k].name : "") << ":d" << base_dtype(in[k].dtype) << ":";
    for (int d = 0; d < in[k].rank; ++d) o << in[k].shape[d] << "x";
    o << ";";
  }
  return o.str();
}

std::unique_ptr<PlanInstance> Session::build(const qpc_tensor* inputs, int n, const std::string& key) {
  device_state(device_);
  auto p = std::make_unique<PlanInstance>();
  p->key = key;
  QPC_CUDA_OR_THROW(cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking));
  for (auto& e : p->ev) QPC_CUDA_OR_THROW(cudaEventCreate(&e));
  {
    Planner pl(*this, *p);
    pl.run(inputs, n);
  }
  for (auto& io : p->ins)
    QPC_CUDA_OR_THROW(cudaHostAlloc((void**)&io.host, std::max<size_t>(io.bytes, 4), cudaHostAllocDefault));
  for (auto& io : p->outs)
    if (!io.device_only)
      QPC_CUDA_OR_THROW(cudaHostAlloc((void**)&io.host, std::max<size_t>(io.bytes, 4), cudaHostAllocDefault));
  // Eager validation pass (sets kernel attributes, surfaces launch errors).
  for (size_t k = 0; k < p->steps.size(); ++k) {
    cudaError_t e = p->steps[k](p->stream);
    if (e != cudaSuccess)
      throw DeviceError{"launch of step " + std::to_string(k) + " (" + p->info[k].kernel + " " +
                        p->info[k].node + "): " + cudaGetErrorString(e)};
  }
  QPC_CUDA_OR_THROW(cudaStreamSynchronize(p->stream));
  if (unsigned kerr = take_kernel_error(device_))
    throw DeviceError{"kernel wait timeout during plan validation (flags " + std::to_string(kerr) + ")"};
  if (opts_.use_cuda_graph) {
    cudaGraph_t graph = nullptr;
    QPC_CUDA_OR_THROW(cudaStreamBeginCapture(p->stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t cap_err = cudaSuccess;
    for (size_t k = 0; k < p->steps.size() && cap_err == cudaSuccess; ++k) cap_err = p->steps[k](p->stream);
    cudaError_t end_err = cudaStreamEndCapture(p->stream, &graph);
    if (cap_err != cudaSuccess || end_err != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      throw DeviceError{std::string("CUDA graph capture failed: ") +
                        cudaGetErrorString(cap_err != cudaSuccess ? cap_err : end_err)};
    }
    cudaError_t ie = cudaGraphInstantiate(&p->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) throw DeviceError{std::string("cudaGraphInstantiate: ") + cudaGetErrorString(ie)};
  }
  return p;
}

PlanInstance* Session::acquire(const qpc_tensor* inputs, int n) {
  const std::string key = shape_key(inputs, n);
  std::lock_guard<std::mutex> lk(mu_);
  auto& vec = plans_[key];
  for (auto& p : vec) {
    bool expect = false;
    if (p->busy.compare_exchange_strong(expect, true)) {
      p->last_used = ++tick_;
      return p.get();
    }
  }
  // Evict idle plans oldest-first while over budget (vulkan/session.rs:369-395).
  auto total = [&] {
    size_t t = 0;
    for (auto& kv : plans_)
      for (auto& p : kv.second) t += p->bytes;
    return t;
  };
  while (total() > (size_t)opts_.plan_budget_bytes) {
    PlanInstance* oldest = nullptr;
    std::string okey;
    for (auto& kv : plans_)
      for (auto& p : kv.second)
        if (!p->busy && (!oldest || p->last_used < oldest->last_used)) {
          oldest = p.get();
          okey = kv.first;
        }
    if (!oldest) break;
    auto& v = plans_[okey];
    v.erase(std::remove_if(v.begin(), v.end(), [&](auto& q) { return q.get() == oldest; }), v.end());
  }
  auto p = build(inputs, n, key);
  p->busy = true;
  p->last_used = ++tick_;
  PlanInstance* raw = p.get();
  plans_[key].push_back(std::move(p));
  return raw;
}

void Session::release(PlanInstance* p) {
  if (p) p->busy = false;
}

PlanInstance* Session::launch(const qpc_tensor* inputs, int n) {
  device_state(device_);
  PlanInstance* p = acquire(inputs, n);
  try {
    QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[0], p->stream));
    for (auto& io : p->ins) {
      const qpc_tensor* t = nullptr;
      for (int k = 0; k < n; ++k)
        if (io.name == inputs[k].name) t = &inputs[k];
      const int dt = base_dtype(t->dtype);
      if (dt != io.dtype) throw GraphError{"input " + io.name + ": dtype differs from the plan's"};
      if (t->dtype == QPC_F32_DEVICE || t->dtype == QPC_U8_IMAGE_DEVICE)
        QPC_CUDA_OR_THROW(cudaMemcpyAsync(io.dev, t->data, io.bytes, cudaMemcpyDeviceToDevice, p->stream));
      else if (pinned_contains(t->data, io.bytes))  // caller's pinned buffer: DMA, no staging
        QPC_CUDA_OR_THROW(cudaMemcpyAsync(io.dev, t->data, io.bytes, cudaMemcpyHostToDevice, p->stream));
      else
        QPC_CUDA_OR_THROW(staged_h2d(io.dev, io.host, t->data, io.bytes, p->stream));
    }
    {
      std::lock_guard<std::mutex> lk(launch_mu_);
      if (!compute_done_) QPC_CUDA_OR_THROW(cudaEventCreateWithFlags(&compute_done_, cudaEventDisableTiming));
      QPC_CUDA_OR_THROW(cudaStreamWaitEvent(p->stream, compute_done_, 0));  // the previous run's graph first
      QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[1], p->stream));
      if (p->exec) {
        QPC_CUDA_OR_THROW(cudaGraphLaunch(p->exec, p->stream));
      } else {
        for (size_t k = 0; k < p->steps.size(); ++k) QPC_CUDA_OR_THROW(p->steps[k](p->stream));
      }
      QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[2], p->stream));
      QPC_CUDA_OR_THROW(cudaEventRecord(compute_done_, p->stream));
    }
    for (auto& io : p->outs)
      if (!io.device_only)
        QPC_CUDA_OR_THROW(cudaMemcpyAsync(io.host, io.dev, io.bytes, cudaMemcpyDeviceToHost, p->stream));
    QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[3], p->stream));
  } catch (...) {
    release(p);
    throw;
  }
  return p;
}

// Stage inputs once, then replay the compute graph `iters` times back to back;
// returns device ms per replay (CUDA events on the plan's stream).
float Session::replay(const qpc_tensor* inputs, int n, int iters) {
  PlanInstance* p = launch(inputs, n);
  float ms = 0.f;
  try {
    QPC_CUDA_OR_THROW(cudaStreamSynchronize(p->stream));
    QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[1], p->stream));
    for (int it = 0; it < iters; ++it) {
      if (p->exec) QPC_CUDA_OR_THROW(cudaGraphLaunch(p->exec, p->stream));
      else
        for (auto& s : p->steps) QPC_CUDA_OR_THROW(s(p->stream));
    }
    QPC_CUDA_OR_THROW(cudaEventRecord(p->ev[2], p->stream));
    QPC_CUDA_OR_THROW(cudaEventSynchronize(p->ev[2]));
    QPC_CUDA_OR_THROW(cudaEventElapsedTime(&ms, p->ev[1], p->ev[2]));
    if (unsigned kerr = take_kernel_error(device_))
      throw DeviceError{"kernel wait timeout (flags " + std::to_string(kerr) + ")"};
  } catch (...) {
    release(p);
    throw;
  }
  release(p);
  return iters > 0 ? ms / iters : 0.f;
}

// Per-step device times: each step run eagerly between two events, averaged
// over `iters` passes (QPPOCR_GPU_PROF analogue, vulkan/session.rs:2073-2139).
void Session::profile(const qpc_tensor* inputs, int n, int iters) {
  PlanInstance* p = launch(inputs, n);
  try {
    QPC_CUDA_OR_THROW(cudaStreamSynchronize(p->stream));
    const size_t ns = p->steps.size();
    std::vector<cudaEvent_t> evs(ns + 1);
    for (auto& e : evs) QPC_CUDA_OR_THROW(cudaEventCreate(&e));
    std::vector<double> acc(ns, 0.0);
    for (int it = 0; it < iters; ++it) {
      QPC_CUDA_OR_THROW(cudaEventRecord(evs[0], p->stream));
      for (size_t k = 0; k < ns; ++k) {
        QPC_CUDA_OR_THROW(p->steps[k](p->stream));
        QPC_CUDA_OR_THROW(cudaEventRecord(evs[k + 1], p->stream));
      }
      QPC_CUDA_OR_THROW(cudaEventSynchronize(evs[ns]));
      for (size_t k = 0; k < ns; ++k) {
        float ms = 0;
        QPC_CUDA_OR_THROW(cudaEventElapsedTime(&ms, evs[k], evs[k + 1]));
        acc[k] += ms;
      }
    }
    for (auto& e : evs) cudaEventDestroy(e);
    prof_ = p->info;
    for (size_t k = 0; k < ns; ++k) prof_[k].ms = (float)(acc[k] / std::max(iters, 1));
  } catch (...) {
    release(p);
    throw;
  }
  release(p);
}

}  // namespace qpc
