// CTC head entry point that allocates no device memory.
//
// Some callers cannot let a library allocate on the GPU: an engine that
// reserves all device memory for its own pool at start-up, or a latency-bound
// serving loop that must not call the CUDA allocator once it is running
// (cudaMalloc can block, synchronise the device, or fail under memory
// pressure).  qpc_op_ctc_head allocates its per-tile partials with
// cudaMallocAsync; qpc_op_ctc_head_noalloc runs the same kernels but keeps the
// partials in a fixed array compiled into this library.
//
// Properties a caller must know:
//  * The array holds at most kMaxPartials float4 (32 MiB) per device.  Every
//    GPU that loads the library holds it until the process exits.  A call
//    needs rows x (column tiles of n) entries, and is rejected with
//    QPC_ERR_INVALID above kMaxPartials.  A column tile is 32 to 256 classes
//    wide, never narrower than min(n, 128) classes, so
//    rows * ceil(n / 128) <= kMaxPartials is a sufficient (not the exact)
//    condition for acceptance.
//  * A bounded wait that runs out inside the kernels is kept in a second
//    fixed word per device until qpc_kernel_error (or the next session run on
//    that device) reads and clears it, so the calls report faults like every
//    other entry point; a call itself returns as soon as it is queued.
//  * All calls share the one array (per device) and it keeps the last call's
//    contents.  Two calls whose kernels overlap on the GPU (different streams,
//    or different host threads) race on it: serialise them.
//  * The first call on a device looks the array's device address up with
//    cudaGetSymbolAddress (once per device, with that device current).  Make
//    that first call before any stream capture on the device.
#include <mutex>

#include "../../include/qppocr_cuda.h"
#include "kernels.h"
#include "runtime.h"

namespace {

constexpr int64_t kMaxPartials = int64_t(1) << 21;  // float4 entries = 32 MiB

// Device-side storage.  In host code these names are host-side stand-ins, not
// device addresses: only the pointers from cudaGetSymbolAddress go to kernels.
static __device__ __align__(256) float4 g_head_partials[kMaxPartials];
// err[0]: the word this call's kernels report into (cleared at the start of
// each call, since the kernels stop early while it is set); err[1]: the
// faults of every call since the last read, kept until the host reads them.
static __device__ __align__(256) unsigned int g_head_err[2];

struct DevicePtrs {
  float4* partials = nullptr;
  unsigned int* err = nullptr;
};

// Folds this call's fault word into the kept one and clears it.
__global__ void keep_fault_kernel(unsigned int* err) {
  const unsigned v = err[0];
  if (v) atomicOr(&err[1], v);
  err[0] = 0;
}

std::mutex g_mu;
constexpr int kMaxDevices = 64;
DevicePtrs g_ptrs[kMaxDevices];

// Device addresses of the static arrays for the current device (set-up on the
// first call per device).
bool device_ptrs(int dev, DevicePtrs* out) {
  std::lock_guard<std::mutex> lk(g_mu);
  DevicePtrs& p = g_ptrs[dev];
  if (!p.partials) {
    void* a = nullptr;
    void* b = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&a, g_head_partials);
    if (e != cudaSuccess) {
      qpc::set_error(std::string("device: cudaGetSymbolAddress(partials): ") + cudaGetErrorString(e));
      return false;
    }
    e = cudaGetSymbolAddress(&b, g_head_err);
    if (e != cudaSuccess) {
      qpc::set_error(std::string("device: cudaGetSymbolAddress(error word): ") + cudaGetErrorString(e));
      return false;
    }
    p.partials = static_cast<float4*>(a);
    p.err = static_cast<unsigned int*>(b);
  }
  *out = p;
  return true;
}

}  // namespace

extern "C" int qpc_op_ctc_head_noalloc(const float* x, int64_t rows, int k, const float* w,
                                       const float* w_lo, int n, const float* bias, int math,
                                       float* pairs, void* stream) {
  qpc::set_error("");
  if (!x || !w || !pairs || rows < 0 || k <= 0 || n <= 0 || (k % 4) ||
      (math == QPC_MATH_3XTF32 && !w_lo)) {
    qpc::set_error("invalid argument (K % 4 == 0 required; 3xTF32 needs w_lo)");
    return QPC_ERR_INVALID;
  }
  if (rows == 0) return QPC_OK;
  const int ntiles = qpc::gemm_tc_col_tiles(n, math);
  if ((int64_t)ntiles * rows > kMaxPartials) {
    qpc::set_error("ctc head (no-alloc): rows * column tiles = " + std::to_string(rows) + " * " +
                   std::to_string(ntiles) + " = " + std::to_string((int64_t)ntiles * rows) +
                   " exceeds the fixed scratch of " + std::to_string(kMaxPartials) + " entries");
    return QPC_ERR_INVALID;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    qpc::set_error("device: no usable current device");
    return QPC_ERR_DEVICE;
  }
  DevicePtrs p;
  if (!device_ptrs(dev, &p)) return QPC_ERR_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The call's own fault word must start at zero (its kernels stop early
  // while it is set); every partial the combine reads is rewritten by the
  // GEMM first.  The fold afterwards keeps any fault for the host.
  e = cudaMemsetAsync(p.err, 0, sizeof(unsigned int), st);
  qpc::GemmEpilogue epi;
  epi.bias = bias;
  epi.partials = p.partials;
  epi.ldo = n;
  if (e == cudaSuccess) e = qpc::launch_gemm_tc(x, rows, k, k, w, w_lo, n, epi, math, p.err, st);
  if (e == cudaSuccess) e = qpc::launch_argmax_combine(p.partials, ntiles, rows, math, pairs, st);
  if (e == cudaSuccess) {
    keep_fault_kernel<<<1, 1, 0, st>>>(p.err);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    qpc::set_error(std::string("device: ctc head (no-alloc) launch: ") + cudaGetErrorString(e));
    return QPC_ERR_DEVICE;
  }
  return QPC_OK;
}

namespace qpc {

// Faults kept by the allocation-free CTC head on `dev` since the last read
// (0 if it never ran there); reads and clears them.  The device is current
// (take_kernel_error sets it).
// The failure path of a call whose bounded wait runs out, without the GEMM:
// the self-test wait kernel reports into this call's word, then the fold
// keeps it, as after a real timeout.
cudaError_t noalloc_head_selftest(uint64_t limit_ns, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  DevicePtrs p;
  if (!device_ptrs(dev, &p)) return cudaErrorInvalidSymbol;
  e = cudaMemsetAsync(p.err, 0, sizeof(unsigned int), st);
  if (e == cudaSuccess) e = launch_wait_selftest(p.err, limit_ns, st);
  if (e == cudaSuccess) {
    keep_fault_kernel<<<1, 1, 0, st>>>(p.err);
    e = cudaGetLastError();
  }
  return e;
}

unsigned int take_noalloc_head_error(int dev) {
  unsigned int* err = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (dev >= 0 && dev < kMaxDevices) err = g_ptrs[dev].err;
  }
  if (!err) return 0;
  unsigned int v = 0;
  QPC_CUDA_OR_THROW(cudaMemcpy(&v, err + 1, sizeof(v), cudaMemcpyDeviceToHost));
  if (v) QPC_CUDA_OR_THROW(cudaMemset(err + 1, 0, sizeof(v)));
  return v;
}

}  // namespace qpc
