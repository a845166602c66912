// Device runtime of the flagos PrivateUse1 device: devices, streams, the
// stream-ordered caching allocator, the device guard and the hooks.
#include "runtime.h"

#include <ATen/Context.h>
#include <ATen/core/CachingHostAllocator.h>
#include <ATen/cuda/CUDAGeneratorImpl.h>
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/util/Exception.h>

#include <atomic>
#include <limits>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace flb200::runtime {

// ============================================================== devices ====

c10::DeviceIndex device_count() noexcept {
  static const c10::DeviceIndex n = [] {
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) {
      (void)cudaGetLastError();
      c = 0;
    }
    return static_cast<c10::DeviceIndex>(c);
  }();
  return n;
}

c10::DeviceIndex current_device() {
  int d = 0;
  C10_CUDA_CHECK(cudaGetDevice(&d));
  return static_cast<c10::DeviceIndex>(d);
}

void set_device(c10::DeviceIndex d) {
  TORCH_CHECK(d >= 0 && d < device_count(), "flagos: invalid device index ", int(d),
              " (", int(device_count()), " devices)");
  int cur = -1;
  C10_CUDA_CHECK(cudaGetDevice(&cur));
  if (cur != d) C10_CUDA_CHECK(cudaSetDevice(d));
}

c10::DeviceIndex exchange_device(c10::DeviceIndex d) {
  const c10::DeviceIndex prev = current_device();
  if (d >= 0 && d != prev) set_device(d);
  return prev;
}

// ============================================================== streams ====

c10::Stream to_flagos(const c10::cuda::CUDAStream& s) {
  return c10::Stream(c10::Stream::UNSAFE,
                     c10::Device(c10::DeviceType::PrivateUse1, s.device_index()), s.id());
}

c10::cuda::CUDAStream to_cuda(const c10::Stream& s) {
  return c10::cuda::CUDAStream::unpack3(s.id(), s.device_index(), c10::DeviceType::CUDA);
}

cudaStream_t current_stream(c10::DeviceIndex d) {
  return c10::cuda::getCurrentCUDAStream(d).stream();
}

namespace {

// Switches the CUDA device for a scope (no-op when already current).
class DeviceScope {
 public:
  explicit DeviceScope(int d) {
    if (cudaGetDevice(&prev_) == cudaSuccess && prev_ != d && d >= 0) {
      if (cudaSetDevice(d) == cudaSuccess) changed_ = true;
    }
  }
  ~DeviceScope() {
    if (changed_) (void)cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1;
  bool changed_ = false;
};

// ============================================================ allocator ====

struct Block {
  size_t size;
  c10::DeviceIndex device;
  cudaStream_t stream;              // allocation stream: frees are ordered here
  std::vector<cudaStream_t> uses;   // other streams recorded through record_stream
};

constexpr int kMaxDevices = 64;

class PoolAllocator final : public c10::Allocator {
 public:
  c10::DataPtr allocate(size_t nbytes) override {
    const c10::DeviceIndex d = current_device();
    const c10::Device dev(c10::DeviceType::PrivateUse1, d);
    if (nbytes == 0) return {nullptr, nullptr, &raw_delete, dev};
    const cudaStream_t s = current_stream(d);
    cudaMemPool_t pool = pool_for(d);
    release_pending();
    void* p = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&p, nbytes, pool, s);
    if (e == cudaErrorMemoryAllocation) {
      // Give cached memory back (ours and torch's CUDA cache) and retry once.
      (void)cudaGetLastError();
      C10_CUDA_CHECK(cudaDeviceSynchronize());
      release_pending();  // this device's pending blocks are idle now
      C10_CUDA_CHECK(cudaMemPoolTrimTo(pool, 0));
      c10::cuda::CUDACachingAllocator::emptyCache();
      e = cudaMallocFromPoolAsync(&p, nbytes, pool, s);
    }
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      TORCH_CHECK(false, "flagos: out of device memory allocating ", nbytes,
                  " bytes on device ", int(d), ": ", cudaGetErrorString(e));
    }
    {
      std::lock_guard<std::mutex> lock(mu_);
      blocks_.emplace(p, Block{nbytes, d, s, {}});
    }
    allocations_.fetch_add(1, std::memory_order_relaxed);
    const uint64_t now = in_use_.fetch_add(nbytes, std::memory_order_relaxed) + nbytes;
    uint64_t peak = peak_.load(std::memory_order_relaxed);
    while (now > peak && !peak_.compare_exchange_weak(peak, now)) {
    }
    return {p, p, &raw_delete, dev};
  }

  c10::DeleterFnPtr raw_deleter() const override { return &raw_delete; }

  void copy_data(void* dest, const void* src, std::size_t count) const final {
    C10_CUDA_CHECK(cudaMemcpy(dest, src, count, cudaMemcpyDeviceToDevice));
  }

  static PoolAllocator& get() {
    static PoolAllocator* a = new PoolAllocator();  // lives until exit
    return *a;
  }

  bool record(void* p, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(mu_);
    auto it = blocks_.find(p);
    if (it == blocks_.end()) return false;
    Block& b = it->second;
    if (s == b.stream) return true;
    for (auto u : b.uses)
      if (u == s) return true;
    b.uses.push_back(s);
    stream_uses_.fetch_add(1, std::memory_order_relaxed);
    return true;
  }

  AllocatorStats stats() {
    AllocatorStats st{};
    st.allocations = allocations_.load();
    st.frees = frees_.load();
    st.bytes_in_use = in_use_.load();
    st.peak_bytes_in_use = peak_.load();
    st.stream_uses = stream_uses_.load();
    {
      std::lock_guard<std::mutex> lock(mu_);
      st.pending_frees = pending_.size();
    }
    for (int d = 0; d < kMaxDevices; ++d) {
      cudaMemPool_t pool = pools_[d].load();
      if (!pool) continue;
      uint64_t r = 0;
      if (cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &r) == cudaSuccess)
        st.pool_reserved += r;
      else
        (void)cudaGetLastError();
    }
    return st;
  }

  void trim() {
    for (int d = 0; d < kMaxDevices; ++d) {
      cudaMemPool_t pool = pools_[d].load();
      if (!pool) continue;
      DeviceScope scope(d);
      C10_CUDA_CHECK(cudaDeviceSynchronize());
      release_pending();
      C10_CUDA_CHECK(cudaMemPoolTrimTo(pool, 0));
    }
  }

 private:
  static void raw_delete(void* p) {
    if (p) get().free(p);
  }

  void free(void* p) {
    Block b;
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto it = blocks_.find(p);
      if (it == blocks_.end()) return;  // not ours (cannot happen through DataPtr)
      b = std::move(it->second);
      blocks_.erase(it);
    }
    frees_.fetch_add(1, std::memory_order_relaxed);
    in_use_.fetch_sub(b.size, std::memory_order_relaxed);
    DeviceScope scope(b.device);
    if (b.uses.empty()) {
      // Stream-ordered: later work on the allocation stream may reuse it.
      if (cudaFreeAsync(p, b.stream) != cudaSuccess) (void)cudaGetLastError();
    } else {
      // Other streams used the block: it goes back to the pool only once
      // each of them has passed this point (an event per stream).  No
      // stream waits for another here, so a copy stream can run ahead of
      // the compute stream that reads its buffers.
      Pending pend{p, b.device, b.stream, {}};
      for (cudaStream_t u : b.uses) {
        cudaEvent_t ev = nullptr;
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
          (void)cudaGetLastError();
          // No event: fall back to ordering the allocation stream after u.
          C10_CUDA_CHECK(cudaStreamSynchronize(u));
          continue;
        }
        C10_CUDA_CHECK(cudaEventRecord(ev, u));
        pend.events.push_back(ev);
      }
      std::lock_guard<std::mutex> lock(mu_);
      pending_.push_back(std::move(pend));
    }
    release_pending();
  }

  // Frees the pending blocks whose streams have all passed their events.
  void release_pending() {
    std::vector<Pending> ready;
    {
      std::lock_guard<std::mutex> lock(mu_);
      if (pending_.empty()) return;
      size_t keep = 0;
      for (size_t i = 0; i < pending_.size(); ++i) {
        bool done = true;
        for (cudaEvent_t ev : pending_[i].events) {
          if (cudaEventQuery(ev) == cudaErrorNotReady) {
            (void)cudaGetLastError();  // not an error: the stream is still busy
            done = false;
            break;
          }
        }
        if (done) {
          ready.push_back(std::move(pending_[i]));
        } else {
          // Never move an entry onto itself: a self-moved vector may come out
          // empty, and an entry without events would be freed at once.
          if (keep != i) pending_[keep] = std::move(pending_[i]);
          ++keep;
        }
      }
      pending_.resize(keep);
    }
    for (Pending& r : ready) {
      DeviceScope scope(r.device);
      for (cudaEvent_t ev : r.events) (void)cudaEventDestroy(ev);
      if (cudaFreeAsync(r.ptr, r.stream) != cudaSuccess) (void)cudaGetLastError();
    }
  }

  cudaMemPool_t pool_for(c10::DeviceIndex d) {
    TORCH_CHECK(d >= 0 && d < kMaxDevices, "flagos: device index out of range");
    cudaMemPool_t pool = pools_[d].load(std::memory_order_acquire);
    if (pool) return pool;
    std::lock_guard<std::mutex> lock(pool_mu_);
    pool = pools_[d].load(std::memory_order_relaxed);
    if (pool) return pool;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = d;
    C10_CUDA_CHECK(cudaMemPoolCreate(&pool, &props));
    // Keep freed blocks cached in the pool instead of returning them to the
    // driver at every synchronisation.
    uint64_t keep = std::numeric_limits<uint64_t>::max();
    C10_CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    // A freed block is reused only by allocations on the stream that freed
    // it (stream order makes that safe); cross-stream use is handled by
    // record_stream and the deferred frees above.  The pool's own
    // cross-stream reuse would also add waits between streams (a copy stream
    // held back behind the compute stream) that nothing asked for.
    int off = 0;
    C10_CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolReuseFollowEventDependencies, &off));
    C10_CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolReuseAllowOpportunistic, &off));
    C10_CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolReuseAllowInternalDependencies, &off));
    pools_[d].store(pool, std::memory_order_release);
    return pool;
  }

  // A freed block still in use by other streams, with an event per stream.
  struct Pending {
    void* ptr;
    c10::DeviceIndex device;
    cudaStream_t stream;
    std::vector<cudaEvent_t> events;
  };

  std::mutex mu_;
  std::unordered_map<void*, Block> blocks_;
  std::vector<Pending> pending_;
  std::mutex pool_mu_;
  std::atomic<cudaMemPool_t> pools_[kMaxDevices] = {};
  std::atomic<uint64_t> allocations_{0}, frees_{0}, in_use_{0}, peak_{0}, stream_uses_{0};
};

// ================================================================ guard ====

struct GuardImpl final : public c10::impl::DeviceGuardImplInterface {
  static constexpr c10::DeviceType static_type = c10::DeviceType::PrivateUse1;

  c10::DeviceType type() const override { return c10::DeviceType::PrivateUse1; }

  c10::Device exchangeDevice(c10::Device d) const override {
    TORCH_INTERNAL_ASSERT(d.is_privateuseone());
    return c10::Device(c10::DeviceType::PrivateUse1, exchange_device(d.index()));
  }
  c10::Device getDevice() const override {
    return c10::Device(c10::DeviceType::PrivateUse1, current_device());
  }
  void setDevice(c10::Device d) const override {
    TORCH_INTERNAL_ASSERT(d.is_privateuseone());
    set_device(d.index());
  }
  void uncheckedSetDevice(c10::Device d) const noexcept override {
    (void)cudaSetDevice(d.index());
  }

  c10::Stream getStream(c10::Device d) const override {
    return to_flagos(c10::cuda::getCurrentCUDAStream(d.index()));
  }
  c10::Stream getDefaultStream(c10::Device d) const override {
    return to_flagos(c10::cuda::getDefaultCUDAStream(d.index()));
  }
  c10::Stream getStreamFromGlobalPool(c10::Device d, bool high) const override {
    return to_flagos(c10::cuda::getStreamFromPool(high, d.index()));
  }
  c10::Stream getNewStream(c10::Device d, int priority) const override {
    return to_flagos(c10::cuda::getStreamFromPool(priority, d.index()));
  }
  c10::Stream exchangeStream(c10::Stream s) const override {
    auto cs = to_cuda(s);
    auto old = c10::cuda::getCurrentCUDAStream(s.device_index());
    c10::cuda::setCurrentCUDAStream(cs);
    return to_flagos(old);
  }
  void* getStreamNativeHandle(const c10::Stream s) const override {
    return to_cuda(s).stream();
  }
  c10::DeviceIndex deviceCount() const noexcept override { return device_count(); }

  void record(void** event, const c10::Stream& stream, const c10::DeviceIndex device_index,
              const c10::EventFlag flag) const override {
    TORCH_CHECK(device_index == -1 || device_index == stream.device_index(),
                "flagos: event device ", int(device_index), " does not match stream device ",
                int(stream.device_index()));
    DeviceScope scope(stream.device_index());
    auto ev = static_cast<cudaEvent_t>(*event);
    if (!ev) {
      const unsigned flags =
          flag == c10::EventFlag::BACKEND_DEFAULT ? cudaEventDefault : cudaEventDisableTiming;
      C10_CUDA_CHECK(cudaEventCreateWithFlags(&ev, flags));
    }
    C10_CUDA_CHECK(cudaEventRecord(ev, to_cuda(stream).stream()));
    *event = ev;
  }
  void block(void* event, const c10::Stream& stream) const override {
    if (!event) return;
    DeviceScope scope(stream.device_index());
    C10_CUDA_CHECK(cudaStreamWaitEvent(to_cuda(stream).stream(), static_cast<cudaEvent_t>(event), 0));
  }
  bool queryEvent(void* event) const override {
    if (!event) return true;
    const cudaError_t e = cudaEventQuery(static_cast<cudaEvent_t>(event));
    if (e == cudaErrorNotReady) {
      (void)cudaGetLastError();
      return false;
    }
    C10_CUDA_CHECK(e);
    return true;
  }
  void destroyEvent(void* event, const c10::DeviceIndex device_index) const noexcept override {
    if (!event) return;
    DeviceScope scope(device_index);
    (void)cudaEventDestroy(static_cast<cudaEvent_t>(event));
  }
  bool queryStream(const c10::Stream& s) const override { return to_cuda(s).query(); }
  void synchronizeStream(const c10::Stream& s) const override { to_cuda(s).synchronize(); }
  void synchronizeEvent(void* event) const override {
    if (event) C10_CUDA_CHECK(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
  }
  void synchronizeDevice(const c10::DeviceIndex d) const override {
    DeviceScope scope(d);
    C10_CUDA_CHECK(cudaDeviceSynchronize());
  }
  void recordDataPtrOnStream(const c10::DataPtr& p, const c10::Stream& s) const override {
    record_stream(p, to_cuda(s).stream());
  }
  double elapsedTime(void* e1, void* e2, const c10::DeviceIndex d) const override {
    TORCH_CHECK(e1 && e2, "flagos: both events must be recorded before elapsed_time");
    DeviceScope scope(d);
    float ms = 0.f;
    C10_CUDA_CHECK(cudaEventElapsedTime(&ms, static_cast<cudaEvent_t>(e1),
                                        static_cast<cudaEvent_t>(e2)));
    return ms;
  }
};

// ================================================================ hooks ====

struct Hooks final : public at::PrivateUse1HooksInterface {
  bool isBuilt() const override { return true; }
  bool isAvailable() const override { return device_count() > 0; }
  bool hasPrimaryContext(c10::DeviceIndex d) const override {
    return c10::cuda::hasPrimaryContext(d);
  }
  const at::Generator& getDefaultGenerator(c10::DeviceIndex d) const override {
    return at::cuda::detail::getDefaultCUDAGenerator(d);
  }
  at::Generator getNewGenerator(c10::DeviceIndex d) const override {
    return at::cuda::detail::createCUDAGenerator(d);
  }
  at::Device getDeviceFromPtr(void* data) const override {
    cudaPointerAttributes a{};
    C10_CUDA_CHECK(cudaPointerGetAttributes(&a, data));
    return at::Device(c10::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(a.device));
  }
  bool isPinnedPtr(const void* data) const override {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, data) != cudaSuccess) {
      (void)cudaGetLastError();
      return false;
    }
    return a.type == cudaMemoryTypeHost;
  }
  at::Allocator* getPinnedMemoryAllocator() const override {
    return at::getHostAllocator(at::kCUDA);
  }
  c10::DeviceIndex deviceCount() const override { return device_count(); }
  void setCurrentDevice(c10::DeviceIndex d) const override { set_device(d); }
  c10::DeviceIndex getCurrentDevice() const override { return current_device(); }
  c10::DeviceIndex exchangeDevice(c10::DeviceIndex d) const override { return exchange_device(d); }
  c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex d) const override {
    return exchange_device(d);
  }
  // Storage resize (FSDP frees and re-materialises parameter storage this way).
  void resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const override {
    auto* impl = storage.unsafeGetStorageImpl();
    const size_t old = impl->nbytes();
    if (newsize == old) return;
    auto* alloc = impl->allocator();
    TORCH_CHECK(alloc != nullptr, "flagos: storage has no allocator to resize with");
    if (newsize == 0) {
      impl->set_data_ptr_noswap(at::DataPtr(nullptr, impl->device()));
      impl->set_nbytes(0);
      return;
    }
    at::DataPtr fresh = alloc->allocate(newsize);
    const size_t keep = std::min(old, newsize);
    if (keep > 0 && impl->data()) {
      DeviceScope scope(impl->device().index());
      C10_CUDA_CHECK(cudaMemcpyAsync(fresh.get(), impl->data(), keep, cudaMemcpyDeviceToDevice,
                                     current_stream(impl->device().index())));
    }
    impl->set_data_ptr_noswap(std::move(fresh));
    impl->set_nbytes(newsize);
  }
};

}  // namespace

c10::Allocator* device_allocator() { return &PoolAllocator::get(); }

bool record_stream(const c10::DataPtr& ptr, cudaStream_t stream) {
  if (ptr.get_deleter() != PoolAllocator::get().raw_deleter() || ptr.get() == nullptr)
    return false;
  return PoolAllocator::get().record(ptr.get(), stream);
}

AllocatorStats allocator_stats() { return PoolAllocator::get().stats(); }

void empty_cache() { PoolAllocator::get().trim(); }

void init() {
  static std::once_flag once;
  std::call_once(once, [] {
    c10::SetAllocator(c10::DeviceType::PrivateUse1, device_allocator());
    at::RegisterPrivateUse1HooksInterface(new Hooks());
    // PyTorch answers is_pinned() through the current accelerator (flagos,
    // once registered) and only for one it has marked initialised; pinned
    // memory itself comes from the CUDA hooks, which mark CUDA, not flagos.
    // Mark flagos too (its init is a no-op), so pinned host tensors report
    // pinned.
    at::globalContext().lazyInitDevice(c10::DeviceType::PrivateUse1);
  });
}

// The guard is registered at load time, like every c10 device guard.
C10_REGISTER_GUARD_IMPL(PrivateUse1, GuardImpl);

}  // namespace flb200::runtime
