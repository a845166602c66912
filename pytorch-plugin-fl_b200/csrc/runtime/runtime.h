// Device runtime of the flagos PrivateUse1 device on B200.
//
// flagos tensors are plain CUDA device memory of the same GPU: device index i
// of flagos is CUDA device i, and flagos streams ARE CUDA streams (the ids of
// c10::cuda's stream pool).  Replaces the reference's csrc/runtime/
// (device_allocator.h:18-50, guard.h:16-140, hooks.h:25-121,
// functions.cc:43-80), whose allocator is a bare cudaMalloc/cudaFree per
// tensor (accelerator/cuda/memory.cc:45,74) and whose guard reports every
// stream as id 0 and synchronises the whole device (guard.h:58-88).
#pragma once

#include <c10/core/Allocator.h>
#include <c10/core/Device.h>
#include <c10/core/Stream.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace flb200::runtime {

// ---- devices -----------------------------------------------------------------
c10::DeviceIndex device_count() noexcept;
c10::DeviceIndex current_device();
void set_device(c10::DeviceIndex d);
c10::DeviceIndex exchange_device(c10::DeviceIndex d);  // returns the previous one

// ---- streams: a flagos c10::Stream carries the id of a c10::cuda stream ------
c10::Stream to_flagos(const c10::cuda::CUDAStream& s);
c10::cuda::CUDAStream to_cuda(const c10::Stream& s);
// The current CUDA stream of flagos device `d` (the stream every b200 kernel
// is launched on).
cudaStream_t current_stream(c10::DeviceIndex d);

// ---- allocator ---------------------------------------------------------------
// Stream-ordered caching allocator: blocks come from a per-device CUDA memory
// pool (cudaMallocFromPoolAsync on the current stream) whose release
// threshold keeps freed memory cached; frees are stream-ordered on the
// allocation stream after every stream the block was recorded on.
c10::Allocator* device_allocator();
// Makes the block behind `ptr` (allocated here) wait for `stream` before it is
// reused (Tensor.record_stream).  Returns false if the block is not ours.
bool record_stream(const c10::DataPtr& ptr, cudaStream_t stream);

struct AllocatorStats {
  uint64_t allocations;      // blocks handed out
  uint64_t frees;            // blocks returned
  uint64_t bytes_in_use;     // bytes currently held by live tensors
  uint64_t peak_bytes_in_use;
  uint64_t pool_reserved;    // bytes the pools hold from the driver
  uint64_t pending_frees;    // freed blocks waiting for other streams to pass their events
  uint64_t stream_uses;      // record_stream calls that added a stream to a block
};
AllocatorStats allocator_stats();
// Returns cached, unused memory of every pool to the driver.
void empty_cache();

// Installs the allocator, the guard and the hooks for PrivateUse1 (idempotent).
void init();

}  // namespace flb200::runtime
