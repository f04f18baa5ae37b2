// Session = one loaded model on one device: graph IR, device-resident
// weights, and a cache of per-input-shape plans (each a captured CUDA graph).
#pragma once
#include <atomic>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qppocr_cuda.h"
#include "runtime.h"

namespace qpc {

struct Attr {
  std::string name;
  int kind = 0;  // qpc_attr_kind
  float f = 0.f;
  int64_t i = 0;
  std::string s;
  std::vector<float> floats;
  std::vector<int64_t> ints;
};

struct Node {
  std::string op, name;
  std::vector<std::string> in, out;
  std::vector<Attr> attrs;
  const Attr* attr(const std::string& n) const;
  int64_t geti(const std::string& n, int64_t d) const;
  float getf(const std::string& n, float d) const;
  std::string gets(const std::string& n, const std::string& d) const;
  std::vector<int64_t> getints(const std::string& n) const;
  void seti(const std::string& n, int64_t v);
  void setf(const std::string& n, float v);
  bool has_in(size_t k) const { return in.size() > k && !in[k].empty(); }
};

struct HostTensor {
  std::vector<int64_t> shape;
  int dtype = QPC_F32;
  std::vector<float> f;
  std::vector<int64_t> i;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  double scalar(int64_t k = 0) const { return dtype == QPC_F32 ? (double)f[k] : (double)i[k]; }
};

// One timed step of a plan (for profiling and roofline accounting).
struct StepInfo {
  std::string kernel;  // kernel family, e.g. "dwconv", "gemm_tc", "conv_tc"
  std::string node;    // graph node (or fused group) it implements
  double bytes = 0;    // algorithmic DRAM bytes (inputs read once + outputs written)
  double flops = 0;    // algorithmic flops
  float ms = 0;        // measured by qpc_session_profile
};

struct PlanInstance {
  std::string key;
  std::vector<std::unique_ptr<DevBuf>> bufs;
  std::vector<std::function<cudaError_t(cudaStream_t)>> steps;
  std::vector<StepInfo> info;
  cudaStream_t stream = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  struct IO {
    std::string name;
    std::vector<int64_t> shape;
    float* dev = nullptr;
    int64_t count = 0;
    float* host = nullptr;  // pinned
    size_t bytes = 0;       // bytes moved per run (inputs: u8 images are 1 byte per value; outputs: D2H bytes)
    int dtype = 0;          // qpc_dtype of the run tensor
    bool device_only = false;  // output kept in device memory (no D2H, host == nullptr)
  };
  std::vector<IO> ins, outs;
  std::atomic<bool> busy{false};
  size_t bytes = 0;
  uint64_t last_used = 0;
  ~PlanInstance();
};

class Session {
 public:
  Session(int device, const qpc_graph* g, const qpc_tensor* w, int nw, int role,
          const qpc_session_options* opts);
  ~Session();
  qpc_caps caps() const;
  // Stages inputs and launches; returns the plan instance now owned by the run.
  PlanInstance* launch(const qpc_tensor* inputs, int n);
  void profile(const qpc_tensor* inputs, int n, int iters);
  float replay(const qpc_tensor* inputs, int n, int iters);
  const std::vector<StepInfo>& profile_steps() const { return prof_; }
  void release(PlanInstance* p);
  int device() const { return device_; }
  bool use_graph() const { return opts_.use_cuda_graph != 0; }

  // --- used by the planner
  const float* dweight(const std::string& name, const std::string& variant);
  const HostTensor* weight(const std::string& name) const;
  int role() const { return role_; }
  int math() const { return opts_.math; }
  bool argmax_exit() const { return argmax_exit_; }
  bool det_mask_exit() const { return opts_.det_mask_exit != 0; }
  float mask_thresh() const { return opts_.mask_thresh; }
  bool mask_dilate() const { return opts_.mask_dilate != 0; }
  const std::vector<Node>& nodes() const { return nodes_; }
  const std::vector<std::string>& graph_inputs() const { return inputs_; }
  const std::vector<std::string>& graph_outputs() const { return outputs_; }

 private:
  PlanInstance* acquire(const qpc_tensor* inputs, int n);
  std::unique_ptr<PlanInstance> build(const qpc_tensor* inputs, int n, const std::string& key);
  void fuse();
  void validate_ops() const;

  int device_;
  int role_;
  qpc_session_options opts_;
  bool argmax_exit_ = false;
  std::vector<Node> nodes_;
  std::vector<std::string> inputs_, outputs_;
  std::unordered_map<std::string, HostTensor> weights_;
  std::unordered_map<std::string, std::unique_ptr<DevBuf>> dev_cache_;
  std::mutex mu_;
  // Runs of this session execute their graphs one after another: each
  // graph waits for the previous run's graph (compute_done_), so two runs in
  // flight overlap one's copies with the other's compute instead of sharing
  // the SMs and finishing together.
  std::mutex launch_mu_;
  cudaEvent_t compute_done_ = nullptr;
  std::map<std::string, std::vector<std::unique_ptr<PlanInstance>>> plans_;
  uint64_t tick_ = 0;
  std::vector<StepInfo> prof_;
};

}  // namespace qpc

struct qpc_session {
  std::unique_ptr<qpc::Session> impl;
};

struct qpc_ticket {
  qpc::Session* session = nullptr;
  qpc::PlanInstance* plan = nullptr;
  bool completed = false;
  float device_ms = 0.f;
};
