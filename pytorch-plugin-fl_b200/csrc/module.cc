// torch_fl._C: the Python face of the flagos device runtime.
//
// Same entry points as the reference's torch_fl/csrc/module.cc:261-271
// (_init, _get_device, _set_device, _exchangeDevice, _get_device_count,
// _synchronize, _get_default_generator, _flagos_to_cuda_view,
// _cuda_to_flagos_view) plus routing and allocator introspection.
#include <ATen/cuda/CUDAGeneratorImpl.h>
#include <c10/cuda/CUDAException.h>
#include <torch/csrc/Generator.h>
#include <torch/extension.h>

#include "aten/dispatch.h"
#include "aten/ops.h"
#include "aten/tensor_utils.h"
#include "runtime/runtime.h"

namespace {

using flb200::aten::Backend;

// Effective route of every routed aten op: {op: backend}.
std::map<std::string, std::string> Routes() {
  namespace A = flb200::aten;
  std::map<std::string, std::string> r;
  auto add = [&](const auto& d) { r[d.name()] = A::BackendName(d.Resolve()); };
  add(A::add_tensor_dispatcher);
  add(A::add_scalar_dispatcher);
  add(A::mul_tensor_dispatcher);
  add(A::mul_scalar_dispatcher);
  add(A::softmax_dispatcher);
  add(A::sum_dim_dispatcher);
  add(A::mean_dim_dispatcher);
  add(A::amax_dispatcher);
  add(A::argmax_dispatcher);
  add(A::silu_dispatcher);
  add(A::rsqrt_dispatcher);
  add(A::neg_dispatcher);
  add(A::cos_dispatcher);
  add(A::sin_dispatcher);
  add(A::pow_tensor_scalar_dispatcher);
  add(A::cat_dispatcher);
  add(A::softmax_backward_dispatcher);
  add(A::silu_backward_dispatcher);
  return r;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace R = flb200::runtime;
  R::init();  // allocator + hooks for PrivateUse1 (the guard registers at load)

  m.def("_init", [] { R::init(); });
  m.def("_get_device_count", [] { return static_cast<int>(R::device_count()); });
  m.def("_get_device", [] { return static_cast<int>(R::current_device()); });
  m.def("_set_device", [](int d) {
    if (d >= 0) R::set_device(static_cast<c10::DeviceIndex>(d));
  });
  m.def("_exchangeDevice", [](int d) {
    if (d < 0) return static_cast<int>(R::current_device());
    return static_cast<int>(R::exchange_device(static_cast<c10::DeviceIndex>(d)));
  });
  m.def("_synchronize", [](int d) {
    const int prev = static_cast<int>(R::current_device());
    if (d >= 0 && d != prev) R::set_device(static_cast<c10::DeviceIndex>(d));
    const cudaError_t e = cudaDeviceSynchronize();
    if (d >= 0 && d != prev) R::set_device(static_cast<c10::DeviceIndex>(prev));
    C10_CUDA_CHECK(e);
  }, py::arg("device") = -1);
  m.def("_get_default_generator", [](int d) {
    return THPGenerator_initDefaultGenerator(at::cuda::detail::getDefaultCUDAGenerator(d));
  });
  // Zero-copy views between the two device types (same GPU memory); the
  // result keeps the source's storage alive.
  m.def("_flagos_to_cuda_view", [](const at::Tensor& t) {
    TORCH_CHECK(t.is_privateuseone(), "_flagos_to_cuda_view: expected a flagos tensor");
    return flb200::aten::CudaAlias(t);
  });
  m.def("_cuda_to_flagos_view", [](const at::Tensor& t) {
    TORCH_CHECK(t.is_cuda(), "_cuda_to_flagos_view: expected a cuda tensor");
    return flb200::aten::ToFlagos(t);
  });
  m.def("_routes", &Routes, "effective backend of every routed aten op");
  m.def("_configured_backend", [](const std::string& op) {
    const Backend b = flb200::aten::ConfiguredBackend(op);
    return std::string(b == Backend::kCount ? "" : flb200::aten::BackendName(b));
  });
  m.def("_config_path", &flb200::aten::ConfigPath);
  m.def("_allocator_stats", [] {
    const auto s = R::allocator_stats();
    py::dict d;
    d["allocations"] = s.allocations;
    d["frees"] = s.frees;
    d["bytes_in_use"] = s.bytes_in_use;
    d["peak_bytes_in_use"] = s.peak_bytes_in_use;
    d["pool_reserved"] = s.pool_reserved;
    d["pending_frees"] = s.pending_frees;
    d["stream_uses"] = s.stream_uses;
    return d;
  });
  m.def("_empty_cache", &R::empty_cache);
}
