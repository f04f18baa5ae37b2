// Host runtime of the qppocr B200 backend: error reporting, per-device state,
// device buffers.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace qpc {

// Thread-local last-error message behind qpc_last_error().
void set_error(const std::string& msg);
const std::string& last_error();

// Status codes (mirror include/qppocr_cuda.h).
enum Status : int { OK = 0, E_INVALID = 1, E_GRAPH = 2, E_DEVICE = 3, E_TIMEOUT = 4, E_OOM = 5 };

struct GraphError {
  std::string msg;
};
struct DeviceError {
  std::string msg;
};
// A device allocation that failed for lack of memory (QPC_ERR_OOM).
struct OomError {
  std::string msg;
};

#define QPC_CUDA_OR_THROW(expr)                                                           \
  do {                                                                                    \
    cudaError_t e__ = (expr);                                                             \
    if (e__ != cudaSuccess)                                                               \
      throw ::qpc::DeviceError{std::string(#expr) + ": " + cudaGetErrorString(e__)};      \
  } while (0)

// Per-device state: the error word kernels with bounded waits report into.
struct DeviceState {
  int device = -1;
  unsigned int* err_word = nullptr;  // device memory, 1 word
};
DeviceState& device_state(int device);  // sets the device current; throws DeviceError

// Reads and clears the device error word (after the caller synchronised),
// ORed with the word of the allocation-free CTC head on that device.
unsigned int take_kernel_error(int device);

// Reads and clears the error word of the allocation-free CTC head on the
// current device (head_noalloc.cu); 0 when it was never called there.
unsigned int take_noalloc_head_error(int device);
// Runs the bounded-wait self-test into the allocation-free head's own fault
// word and keeps the fault there, as a timed-out call would (current device).
cudaError_t noalloc_head_selftest(uint64_t limit_ns, cudaStream_t st);

// Launch configuration, per device.  cudaFuncSetAttribute applies to the
// current device only, so the dynamic shared-memory opt-in of a kernel is
// recorded per (device, kernel) - the largest size set so far - under a
// mutex; a process with sessions on several GPUs sets it on each.
cudaError_t ensure_dyn_smem(const void* func, int bytes);
// SM count of the current device.
int current_sm_count();
// Resident blocks per SM of `func` at (threads, smem) on the current device
// (at least 1), after ensure_dyn_smem(func, smem).
int blocks_per_sm(const void* func, int threads, int smem);

// Test hook: when > 0, the n-th device allocation made by the library from
// now on (DevBuf, plan arenas, the stream-ordered scratch of the operator
// entry points) fails as if the device were out of memory, once.
void inject_alloc_failure(int nth);
// True when an injected failure is due for this allocation (consumes it).
bool alloc_failure_due();

// Owning device allocation.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  explicit DevBuf(size_t n);
  ~DevBuf();
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  float* f() const { return static_cast<float*>(ptr); }
};

}  // namespace qpc
