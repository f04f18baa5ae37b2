// Parallel host copies for session I/O (see host_copy.h).
#include "host_copy.h"

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

namespace qpc {
namespace {

constexpr size_t kChunk = size_t(8) << 20;        // 8 MiB per chunk
constexpr size_t kSerialBelow = size_t(4) << 20;  // small copies stay on the caller

// One batch of chunk copies.  Workers and the caller claim chunks through
// `next`; `done[k]` is set once chunk k is in place.
struct Batch {
  char* dst = nullptr;
  const char* src = nullptr;
  size_t bytes = 0;
  size_t nchunks = 0;
  std::atomic<size_t> next{0};
  std::unique_ptr<std::atomic<int>[]> done;
  std::atomic<size_t> finished{0};
  std::mutex mu;
  std::condition_variable cv;

  // Copy chunks until none are left unclaimed.
  void work() {
    for (;;) {
      const size_t k = next.fetch_add(1);
      if (k >= nchunks) return;
      const size_t off = k * kChunk;
      const size_t n = std::min(kChunk, bytes - off);
      std::memcpy(dst + off, src + off, n);
      done[k].store(1, std::memory_order_release);
      finished.fetch_add(1);
      // taking the lock orders this wake-up after a waiter's predicate check
      { std::lock_guard<std::mutex> lk(mu); }
      cv.notify_all();
    }
  }
  void wait_chunk(size_t k) {
    if (done[k].load(std::memory_order_acquire)) return;
    std::unique_lock<std::mutex> lk(mu);
    cv.wait(lk, [&] { return done[k].load(std::memory_order_acquire) != 0; });
  }
};

class Pool {
 public:
  static Pool& get() {
    static Pool p;
    return p;
  }
  int threads() const { return (int)workers_.size(); }

  // Hand `b` to every worker; each returns when no chunk is left.
  void post(const std::shared_ptr<Batch>& b) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      for (size_t i = 0; i < workers_.size(); ++i) q_.push_back(b);
    }
    cv_.notify_all();
  }

  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }

 private:
  Pool() {
    // the host's cores shared by the processes of this node (one per GPU)
    int n = (int)std::thread::hardware_concurrency();
    if (const char* lw = std::getenv("LOCAL_WORLD_SIZE")) n /= std::max(1, std::atoi(lw));
    if (const char* env = std::getenv("QPPOCR_CUDA_COPY_THREADS")) n = std::atoi(env) + 1;
    n = std::max(1, std::min(n, 16)) - 1;  // the caller is the n-th copier
    for (int i = 0; i < n; ++i) workers_.emplace_back([this] { loop(); });
  }
  void loop() {
    for (;;) {
      std::shared_ptr<Batch> b;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !q_.empty(); });
        if (stop_ && q_.empty()) return;
        b = std::move(q_.front());
        q_.pop_front();
      }
      b->work();
    }
  }
  std::vector<std::thread> workers_;
  std::deque<std::shared_ptr<Batch>> q_;
  std::mutex mu_;
  std::condition_variable cv_;
  bool stop_ = false;
};

std::shared_ptr<Batch> make_batch(void* dst, const void* src, size_t bytes) {
  auto b = std::make_shared<Batch>();
  b->dst = static_cast<char*>(dst);
  b->src = static_cast<const char*>(src);
  b->bytes = bytes;
  b->nchunks = (bytes + kChunk - 1) / kChunk;
  b->done.reset(new std::atomic<int>[b->nchunks]);
  for (size_t k = 0; k < b->nchunks; ++k) b->done[k].store(0);
  return b;
}

}  // namespace

int host_copy_threads() { return Pool::get().threads(); }

namespace {
std::mutex g_pin_mu;
std::map<uintptr_t, size_t>& pinned_blocks() {  // base -> bytes
  static std::map<uintptr_t, size_t> m;
  return m;
}
}  // namespace

void* pinned_alloc(size_t bytes) {
  void* p = nullptr;
  if (cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocPortable) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_pin_mu);
  pinned_blocks()[reinterpret_cast<uintptr_t>(p)] = bytes;
  return p;
}

bool pinned_free(void* p) {
  {
    std::lock_guard<std::mutex> lk(g_pin_mu);
    auto& m = pinned_blocks();
    auto it = m.find(reinterpret_cast<uintptr_t>(p));
    if (it == m.end()) return false;
    m.erase(it);
  }
  cudaFreeHost(p);
  return true;
}

bool pinned_contains(const void* p, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  std::lock_guard<std::mutex> lk(g_pin_mu);
  auto& m = pinned_blocks();
  auto it = m.upper_bound(a);  // first block starting after a
  if (it == m.begin()) return false;
  --it;
  return a >= it->first && a - it->first <= it->second && bytes <= it->second - (a - it->first);
}

void parallel_copy(void* dst, const void* src, size_t bytes) {
  if (bytes < kSerialBelow || Pool::get().threads() == 0) {
    if (bytes) std::memcpy(dst, src, bytes);
    return;
  }
  auto b = make_batch(dst, src, bytes);
  Pool::get().post(b);
  b->work();
  for (size_t k = 0; k < b->nchunks; ++k) b->wait_chunk(k);
}

cudaError_t staged_h2d(void* dev, void* pinned, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes < kSerialBelow || Pool::get().threads() == 0) {
    if (bytes) std::memcpy(pinned, src, bytes);
    return bytes ? cudaMemcpyAsync(dev, pinned, bytes, cudaMemcpyHostToDevice, stream) : cudaSuccess;
  }
  auto b = make_batch(pinned, src, bytes);
  Pool::get().post(b);
  // The caller enqueues DMAs in chunk order as chunks land; it copies
  // chunks itself only once every staged chunk has been enqueued.
  char* d = static_cast<char*>(dev);
  const char* p = static_cast<const char*>(pinned);
  cudaError_t err = cudaSuccess;
  size_t k = 0;
  while (k < b->nchunks) {
    if (!b->done[k].load(std::memory_order_acquire)) {
      // nothing ready in order: help copy, or wait for the chunk in flight
      if (b->next.load() < b->nchunks) {
        const size_t mine = b->next.fetch_add(1);
        if (mine < b->nchunks) {
          const size_t off = mine * kChunk;
          std::memcpy(b->dst + off, b->src + off, std::min(kChunk, bytes - off));
          b->done[mine].store(1, std::memory_order_release);
          b->finished.fetch_add(1);
          continue;
        }
      }
      b->wait_chunk(k);
    }
    const size_t off = k * kChunk;
    const size_t n = std::min(kChunk, bytes - off);
    if (err == cudaSuccess) err = cudaMemcpyAsync(d + off, p + off, n, cudaMemcpyHostToDevice, stream);
    ++k;
  }
  return err;
}

}  // namespace qpc
