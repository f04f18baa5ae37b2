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

// Reads and clears the device error word (after the caller synchronised).
unsigned int take_kernel_error(int device);

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
