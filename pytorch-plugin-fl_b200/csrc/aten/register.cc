// aten registrations of the flagos (PrivateUse1) device.
//
// Mirrors the reference's csrc/aten/register.cc:382-448: tensor plumbing
// (empty, views, resize, copies, set_, record_stream), the routed hot ops
// (each through its Dispatcher, so backends.conf picks b200 or cuda), and a
// boxed fallback for every other aten op.  The reference's fallback runs the
// op on the CPU after copying every operand to the host
// (register.cc:439-442 -> fallback.cc:12-14); this one runs PyTorch's CUDA
// kernel for the op on CUDA aliases of the same device memory.
// _to_copy, contiguous and clone are not registered: aten's composite
// kernels build them from empty + copy_, and copy_ lands in _copy_from
// below, which casts on the device (the reference's flagos->flagos
// _to_copy round-trips through the host, copy_ops.cc:225-240).
#include <ATen/EmptyTensor.h>
#include <ATen/native/Resize.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAException.h>
#include <torch/library.h>

#include "../runtime/runtime.h"
#include "ops.h"
#include "tensor_utils.h"

namespace flb200::aten {
namespace {

constexpr c10::DispatchKeySet kFlagosKeys(c10::DispatchKey::PrivateUse1);

// ------------------------------------------------------------- creation ---
at::Tensor EmptyMemoryFormat(c10::IntArrayRef size, std::optional<c10::ScalarType> dtype,
                             std::optional<c10::Layout> layout, std::optional<c10::Device> device,
                             std::optional<bool> pin_memory,
                             std::optional<c10::MemoryFormat> memory_format) {
  const c10::Device dev = c10::device_or_default(device);
  TORCH_CHECK(dev.is_privateuseone(), "flagos empty: expected a flagos device, got ", dev);
  TORCH_CHECK(c10::layout_or_default(layout) == c10::Layout::Strided,
              "flagos: only strided tensors are supported");
  TORCH_CHECK(!c10::pinned_memory_or_default(pin_memory), "flagos: pin_memory is for CPU tensors");
  const c10::DeviceGuard guard(dev);
  return at::detail::empty_generic(size, runtime::device_allocator(), kFlagosKeys,
                                   c10::dtype_or_default(dtype), memory_format);
}

at::Tensor EmptyStrided(c10::IntArrayRef size, c10::IntArrayRef stride,
                        std::optional<c10::ScalarType> dtype, std::optional<c10::Layout> layout,
                        std::optional<c10::Device> device, std::optional<bool> pin_memory) {
  const c10::Device dev = c10::device_or_default(device);
  TORCH_CHECK(dev.is_privateuseone(), "flagos empty_strided: expected a flagos device, got ", dev);
  TORCH_CHECK(c10::layout_or_default(layout) == c10::Layout::Strided,
              "flagos: only strided tensors are supported");
  TORCH_CHECK(!c10::pinned_memory_or_default(pin_memory), "flagos: pin_memory is for CPU tensors");
  const c10::DeviceGuard guard(dev);
  return at::detail::empty_strided_generic(size, stride, runtime::device_allocator(), kFlagosKeys,
                                           c10::dtype_or_default(dtype));
}

// ---------------------------------------------------------------- views ---
at::Tensor AsStrided(const at::Tensor& self, c10::SymIntArrayRef size, c10::SymIntArrayRef stride,
                     std::optional<c10::SymInt> storage_offset) {
  std::optional<int64_t> off;
  if (storage_offset) off = storage_offset->expect_int();
  return at::native::as_strided_tensorimpl(self, C10_AS_INTARRAYREF_SLOW(size),
                                           C10_AS_INTARRAYREF_SLOW(stride), off);
}
at::Tensor View(const at::Tensor& self, c10::SymIntArrayRef size) {
  return at::native::view(self, C10_AS_INTARRAYREF_SLOW(size));
}
at::Tensor ReshapeAlias(const at::Tensor& self, c10::SymIntArrayRef size,
                        c10::SymIntArrayRef stride) {
  return at::native::_reshape_alias(self, C10_AS_INTARRAYREF_SLOW(size),
                                    C10_AS_INTARRAYREF_SLOW(stride));
}

// --------------------------------------------------------------- resize ---
void GrowStorage(const at::Tensor& self, size_t nbytes) {
  c10::StorageImpl* st = self.storage().unsafeGetStorageImpl();
  TORCH_CHECK(st->resizable() && st->allocator(),
              "flagos: trying to resize a storage that is not resizable");
  at::DataPtr fresh = st->allocator()->allocate(nbytes);
  const size_t keep = std::min(st->nbytes(), nbytes);
  if (keep && st->data()) {
    GpuGuard g(self);
    C10_CUDA_CHECK(cudaMemcpyAsync(fresh.get(), st->data(), keep, cudaMemcpyDeviceToDevice,
                                   StreamOf(self)));
  }
  st->set_data_ptr_noswap(std::move(fresh));
  st->set_nbytes(nbytes);
}

const at::Tensor& Resize(const at::Tensor& self, c10::SymIntArrayRef size,
                         std::optional<at::MemoryFormat> memory_format) {
  auto* impl = self.unsafeGetTensorImpl();
  at::native::resize_impl_cpu_(impl, C10_AS_INTARRAYREF_SLOW(size), std::nullopt,
                               /*resize_storage=*/false);
  const auto mf = memory_format.value_or(at::MemoryFormat::Contiguous);
  if (mf != at::MemoryFormat::Contiguous && mf != at::MemoryFormat::Preserve)
    impl->empty_tensor_restride(mf);
  const size_t need = at::detail::computeStorageNbytes(self.sizes(), self.strides(),
                                                       self.dtype().itemsize(),
                                                       self.storage_offset());
  if (need > self.storage().nbytes()) GrowStorage(self, need);
  return self;
}

// ----------------------------------------------------------------- copy ---
at::Tensor CopyFrom(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
  TORCH_CHECK(self.defined() && dst.defined(), "flagos _copy_from: undefined tensor");
  if (self.numel() == 0) return dst;
  if (self.is_privateuseone() && dst.is_privateuseone() && self.device() == dst.device() &&
      self.sizes() == dst.sizes() && self.is_contiguous() && dst.is_contiguous()) {
    GpuGuard g(dst);
    if (self.scalar_type() == dst.scalar_type()) {
      C10_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr(), self.data_ptr(),
                                     self.numel() * self.element_size(),
                                     cudaMemcpyDeviceToDevice, StreamOf(dst)));
      return dst;
    }
    const int cs = B200Dtype(self.scalar_type()), cd = B200Dtype(dst.scalar_type());
    if (cs >= 0 && cd >= 0) {  // dtype cast on the device (b200 kernel)
      CheckB200(fl_b200_cast(self.data_ptr(), cs, dst.data_ptr(), cd, self.numel(),
                             StreamOf(dst)),
                "_copy_from");
      return dst;
    }
  }
  // Strided, broadcast, cross-device and host copies: PyTorch's CUDA copy on aliases.
  at::Tensor d = CudaAlias(dst);
  d.copy_(CudaAlias(self), non_blocking);
  return dst;
}

at::Tensor CopyFromAndResize(const at::Tensor& self, const at::Tensor& dst) {
  Resize(dst, c10::fromIntArrayRefSlow(self.sizes()), std::nullopt);
  return CopyFrom(self, dst, false);
}

at::Scalar LocalScalarDense(const at::Tensor& self) {
  return CudaAlias(self).item();
}

// ----------------------------------------------------------------- set_ ---
at::Tensor& SetStorageOffset(at::Tensor& self, c10::Storage source, int64_t offset,
                             c10::IntArrayRef size, c10::IntArrayRef stride) {
  at::native::checkSetStorage(self, std::move(source), offset, size, stride);
  self.unsafeGetTensorImpl()->set_storage_offset(offset);
  at::OptionalIntArrayRef st;
  if (stride.data()) st = stride;
  at::native::resize_impl_cpu_(self.unsafeGetTensorImpl(), size, st, /*resize_storage=*/false);
  return self;
}
at::Tensor& SetStorage(at::Tensor& self, c10::Storage source) {
  const int64_t n = static_cast<int64_t>(source.nbytes() / self.dtype().itemsize());
  return SetStorageOffset(self, std::move(source), 0, {n}, {});
}
at::Tensor& SetTensor(at::Tensor& self, const at::Tensor& src) {
  return SetStorageOffset(self, src.storage(), src.storage_offset(), src.sizes(), src.strides());
}

void RecordStream(at::Tensor& self, at::Stream s) {
  runtime::record_stream(self.storage().data_ptr(), runtime::to_cuda(s).stream());
}

// ------------------------------------------------------------ routed ops ---
at::Tensor AddTensor(const at::Tensor& a, const at::Tensor& b, const at::Scalar& alpha) {
  return add_tensor_dispatcher(a, b, alpha);
}
at::Tensor AddScalar(const at::Tensor& a, const at::Scalar& b, const at::Scalar& alpha) {
  return add_scalar_dispatcher(a, b, alpha);
}
at::Tensor MulTensor(const at::Tensor& a, const at::Tensor& b) { return mul_tensor_dispatcher(a, b); }
at::Tensor MulScalar(const at::Tensor& a, const at::Scalar& b) { return mul_scalar_dispatcher(a, b); }
at::Tensor Softmax(const at::Tensor& x, int64_t dim, bool half_to_float) {
  return softmax_dispatcher(x, dim, half_to_float);
}
at::Tensor SumDim(const at::Tensor& x, at::OptionalIntArrayRef dim, bool keepdim,
                  std::optional<at::ScalarType> dtype) {
  return sum_dim_dispatcher(x, dim, keepdim, dtype);
}
at::Tensor MeanDim(const at::Tensor& x, at::OptionalIntArrayRef dim, bool keepdim,
                   std::optional<at::ScalarType> dtype) {
  return mean_dim_dispatcher(x, dim, keepdim, dtype);
}
at::Tensor Amax(const at::Tensor& x, at::IntArrayRef dim, bool keepdim) {
  return amax_dispatcher(x, dim, keepdim);
}
at::Tensor Argmax(const at::Tensor& x, std::optional<int64_t> dim, bool keepdim) {
  return argmax_dispatcher(x, dim, keepdim);
}
at::Tensor Silu(const at::Tensor& x) { return silu_dispatcher(x); }
at::Tensor Rsqrt(const at::Tensor& x) { return rsqrt_dispatcher(x); }
at::Tensor Neg(const at::Tensor& x) { return neg_dispatcher(x); }
at::Tensor Cos(const at::Tensor& x) { return cos_dispatcher(x); }
at::Tensor Sin(const at::Tensor& x) { return sin_dispatcher(x); }
at::Tensor PowTensorScalar(const at::Tensor& x, const at::Scalar& e) {
  return pow_tensor_scalar_dispatcher(x, e);
}
at::Tensor Cat(const at::ITensorListRef& ts, int64_t dim) { return cat_dispatcher(ts, dim); }
at::Tensor SoftmaxBackwardData(const at::Tensor& g, const at::Tensor& y, int64_t dim,
                               at::ScalarType input_dtype) {
  return softmax_backward_dispatcher(g, y, dim, input_dtype);
}
at::Tensor SiluBackward(const at::Tensor& g, const at::Tensor& x) {
  return silu_backward_dispatcher(g, x);
}

// ------------------------------------------------------------- fallback ---
// A CUDA alias whose storage may be resized by an out= kernel: the resized
// result is copied back into the flagos tensor afterwards.
at::Tensor ResizableAlias(const at::Tensor& t) {
  at::Tensor a = CudaAlias(t);
  auto* st = a.storage().unsafeGetStorageImpl();
  st->set_allocator(c10::cuda::CUDACachingAllocator::get());  // before: resizable needs one
  st->set_resizable(true);
  return a;
}

void CudaFallback(const c10::OperatorHandle& op, torch::jit::Stack* stack) {
  const auto& schema = op.schema();
  const size_t nargs = schema.arguments().size();
  const size_t first = stack->size() - nargs;
  struct Swap {
    c10::TensorImpl* alias;
    at::Tensor orig;
    at::Tensor alias_t;
  };
  std::vector<Swap> swaps;
  std::optional<c10::cuda::CUDAGuard> guard;
  auto to_alias = [&](const at::Tensor& t) -> at::Tensor {
    if (!t.defined() || !t.is_privateuseone()) return t;
    if (!guard) guard.emplace(t.device().index());
    at::Tensor a = ResizableAlias(t);
    swaps.push_back({a.unsafeGetTensorImpl(), t, a});
    return a;
  };
  for (size_t i = first; i < stack->size(); ++i) {
    c10::IValue& iv = (*stack)[i];
    if (iv.isTensor()) {
      iv = to_alias(iv.toTensor());
    } else if (iv.isTensorList()) {
      c10::List<at::Tensor> l;
      for (const at::Tensor& t : iv.toTensorList()) l.push_back(to_alias(t));
      iv = l;
    } else if (iv.isOptionalTensorList()) {
      c10::List<std::optional<at::Tensor>> l;
      for (const std::optional<at::Tensor>& t : iv.toOptionalTensorList())
        l.push_back(t ? std::optional<at::Tensor>(to_alias(*t)) : std::nullopt);
      iv = l;
    }
  }
  op.redispatchBoxed(c10::DispatchKeySet(c10::DispatchKey::CUDA), stack);
  // A mutated argument whose alias was resized or re-pointed: copy back.
  for (auto& s : swaps) {
    if (s.alias_t.storage().data() != s.orig.storage().data() ||
        s.alias_t.sizes() != s.orig.sizes() || s.alias_t.strides() != s.orig.strides()) {
      at::Tensor o = s.orig;
      Resize(o, c10::fromIntArrayRefSlow(s.alias_t.sizes()), std::nullopt);
      CudaAlias(o).copy_(s.alias_t);
    }
  }
  auto back = [&](const at::Tensor& t) -> at::Tensor {
    if (!t.defined() || !t.is_cuda()) return t;
    for (auto& s : swaps)
      if (s.alias == t.unsafeGetTensorImpl()) return s.orig;
    return ToFlagos(t);
  };
  const size_t nret = schema.returns().size();
  for (size_t i = stack->size() - nret; i < stack->size(); ++i) {
    c10::IValue& iv = (*stack)[i];
    if (iv.isTensor()) {
      iv = back(iv.toTensor());
    } else if (iv.isTensorList()) {
      c10::List<at::Tensor> l;
      for (const at::Tensor& t : iv.toTensorList()) l.push_back(back(t));
      iv = l;
    }
  }
}

}  // namespace

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
  m.impl("empty.memory_format", EmptyMemoryFormat);
  m.impl("empty_strided", EmptyStrided);
  m.impl("as_strided", AsStrided);
  m.impl("view", View);
  m.impl("_reshape_alias", ReshapeAlias);
  m.impl("resize_", Resize);
  m.impl("_copy_from", CopyFrom);
  m.impl("_copy_from_and_resize", CopyFromAndResize);
  m.impl("_local_scalar_dense", LocalScalarDense);
  m.impl("set_.source_Storage", SetStorage);
  m.impl("set_.source_Storage_storage_offset", SetStorageOffset);
  m.impl("set_.source_Tensor", SetTensor);
  m.impl("record_stream", RecordStream);
  // routed ops (backends.conf: b200 | cuda)
  m.impl("add.Tensor", AddTensor);
  m.impl("add.Scalar", AddScalar);
  m.impl("mul.Tensor", MulTensor);
  m.impl("mul.Scalar", MulScalar);
  m.impl("_softmax", Softmax);
  m.impl("sum.dim_IntList", SumDim);
  m.impl("mean.dim", MeanDim);
  m.impl("amax", Amax);
  m.impl("argmax", Argmax);
  m.impl("silu", Silu);
  m.impl("rsqrt", Rsqrt);
  m.impl("neg", Neg);
  m.impl("cos", Cos);
  m.impl("sin", Sin);
  m.impl("pow.Tensor_Scalar", PowTensorScalar);
  m.impl("cat", Cat);
  m.impl("_softmax_backward_data", SoftmaxBackwardData);
  m.impl("silu_backward", SiluBackward);
}

TORCH_LIBRARY_IMPL(_, PrivateUse1, m) {
  m.fallback(torch::CppFunction::makeFromBoxedFunction<&CudaFallback>());
}

}  // namespace flb200::aten
