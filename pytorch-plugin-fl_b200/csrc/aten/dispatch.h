// Per-op backend routing of the flagos device.
//
// Same contract as the reference (csrc/aten/common.h:20, common.cc:44-133,
// dispatcher.h:38-133): every routed aten op has a Dispatcher holding one
// kernel pointer per backend; the backend an op runs on comes from
// backends.conf ("op = backend", file from $FLAGOS_BACKEND_CONFIG or next to
// the package), may be overridden per op with FLAGOS_OP_<op> (dots written as
// "__"), and FLAGOS_LOG_DISPATCH=1 prints "[flagos dispatch] <op> -> <backend>".
// Differences: a `b200` backend (this library's kernels); an op that the
// config does not name runs on b200 when it has a b200 kernel, else on cuda
// (PyTorch's CUDA kernels on the same memory); FLAGOS_OP_* overrides apply to
// every op, listed or not; and the route is resolved once per op, not hashed
// on every call.
#pragma once

#include <c10/util/Exception.h>

#include <atomic>
#include <string>
#include <utility>

namespace flb200::aten {

enum class Backend : int { kCuda = 0, kFlagOs, kFlagOsPython, kAscend, kMusa, kB200, kCount };

const char* BackendName(Backend b);
// Backend configured for `op` (config file + env override), or kCount when
// neither names it.
Backend ConfiguredBackend(const std::string& op);
bool LogDispatchEnabled();
void LogDispatch(const char* op, Backend b);
// Path of the config file that was loaded ("" if none).
std::string ConfigPath();

template <typename FnPtr>
class Dispatcher {
 public:
  constexpr explicit Dispatcher(const char* op) : op_(op) {}

  void Register(Backend b, FnPtr fn) { fns_[static_cast<int>(b)] = fn; }

  Backend Resolve() const {
    int r = resolved_.load(std::memory_order_acquire);
    if (r < 0) {
      Backend b = ConfiguredBackend(op_);
      if (b == Backend::kCount) b = fns_[static_cast<int>(Backend::kB200)] ? Backend::kB200
                                                                              : Backend::kCuda;
      r = static_cast<int>(b);
      resolved_.store(r, std::memory_order_release);
    }
    return static_cast<Backend>(r);
  }

  template <typename... Args>
  auto operator()(Args&&... args) const {
    const Backend b = Resolve();
    if (LogDispatchEnabled()) LogDispatch(op_, b);
    FnPtr fn = fns_[static_cast<int>(b)];
    TORCH_CHECK(fn, op_, ": backend '", BackendName(b), "' is not registered on this build");
    return fn(std::forward<Args>(args)...);
  }

  const char* name() const { return op_; }

 private:
  const char* op_;
  FnPtr fns_[static_cast<int>(Backend::kCount)] = {};
  mutable std::atomic<int> resolved_{-1};
};

namespace detail {
template <typename FnPtr>
struct Registrar {
  Registrar(Dispatcher<FnPtr>& d, Backend b, FnPtr fn) { d.Register(b, fn); }
};
}  // namespace detail

}  // namespace flb200::aten

#define FLB_DECLARE_DISPATCHER(fn_type, name) \
  extern ::flb200::aten::Dispatcher<fn_type> name;
#define FLB_DEFINE_DISPATCHER(fn_type, name, op) \
  ::flb200::aten::Dispatcher<fn_type> name(op);
#define FLB_REGISTER_CAT2(a, b) a##b
#define FLB_REGISTER_CAT(a, b) FLB_REGISTER_CAT2(a, b)
#define FLB_REGISTER_KERNEL(fn_type, name, backend, fn)                                    \
  __attribute__((used)) static ::flb200::aten::detail::Registrar<fn_type> FLB_REGISTER_CAT( \
      name##_reg_, __COUNTER__)(name, backend, fn);
