// Host-side copies around a run: caller tensors -> pinned staging -> device,
// and pinned results -> caller buffers.
//
// The reference hands a session its inputs as host tensors and takes fresh
// host tensors back (qppocr-core device.rs:105-176), so every run moves the
// whole batch through host memory twice.  One thread copying a 708 MB det
// batch runs at host-memcpy speed (~10 GB/s), several times slower than the
// GPU step it feeds.  These helpers split each copy into chunks that a pool of
// worker threads copies in parallel; the staged copy also queues each
// chunk's host->device DMA as soon as that chunk has landed in pinned memory,
// so the DMA overlaps the remaining host copies.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace qpc {

// Copy `bytes` from `src` (pageable) to `dst`, in parallel chunks.  Blocks
// until done.
void parallel_copy(void* dst, const void* src, size_t bytes);

// Copy `bytes` from `src` (pageable) into the pinned buffer `pinned` in
// parallel chunks and enqueue on `stream` one cudaMemcpyAsync per chunk into
// `dev`, each as soon as its chunk is staged.  Returns after every chunk is
// staged and enqueued (the DMA may still be running).
cudaError_t staged_h2d(void* dev, void* pinned, const void* src, size_t bytes, cudaStream_t stream);

// Worker threads used (excluding the calling thread).
int host_copy_threads();

// Pinned host allocations made through the library (qpc_host_alloc).  A run
// input that lies wholly inside one is copied to the device by DMA straight
// from the caller's memory, with no staging copy.
void* pinned_alloc(size_t bytes);
bool pinned_free(void* p);
bool pinned_contains(const void* p, size_t bytes);

}  // namespace qpc
