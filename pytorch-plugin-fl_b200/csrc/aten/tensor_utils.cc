#include "tensor_utils.h"

#include <ATen/Context.h>
#include <c10/core/TensorImpl.h>

namespace flb200::aten {

at::Tensor Rewrap(const at::Tensor& t, c10::DeviceType target) {
  if (!t.defined() || t.device().type() == target || t.device().is_cpu()) return t;
  TORCH_CHECK(t.layout() == c10::kStrided, "flagos: only strided tensors are supported");
  // A CUDA alias is about to meet PyTorch's CUDA kernels, which allocate
  // through CUDA's caching allocator: make sure PyTorch's lazy CUDA set-up has
  // run (a process whose first op on flagos has no flagos kernel has not
  // touched CUDA through PyTorch yet).  A no-op after the first call.
  if (target == c10::DeviceType::CUDA) at::globalContext().lazyInitDevice(c10::DeviceType::CUDA);
  const c10::Storage& src = t.storage();
  const c10::Device dev(target, t.device().index());
  // The new storage points at the same bytes; its context owns a reference
  // to the original storage, so the memory lives as long as either tensor.
  auto* keep = new c10::Storage(src);
  c10::DataPtr dp(const_cast<void*>(src.data()), keep,
                  [](void* ctx) { delete static_cast<c10::Storage*>(ctx); }, dev);
  c10::Storage alias(c10::Storage::use_byte_size_t(), src.nbytes(), std::move(dp),
                     /*allocator=*/nullptr, /*resizable=*/false);
  auto out = at::detail::make_tensor<c10::TensorImpl>(
      std::move(alias),
      c10::DispatchKeySet(target == c10::DeviceType::CUDA ? c10::DispatchKey::CUDA
                                                          : c10::DispatchKey::PrivateUse1),
      t.dtype());
  out.unsafeGetTensorImpl()->set_sizes_and_strides(t.sizes(), t.strides(), t.storage_offset());
  return out;
}

int B200Dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return FL_B200_F32;
    case at::kBFloat16: return FL_B200_BF16;
    case at::kHalf: return FL_B200_F16;
    case at::kInt: return FL_B200_I32;
    case at::kLong: return FL_B200_I64;
    default: return -1;
  }
}

void CheckB200(int status, const char* op) {
  if (status == FL_B200_OK) return;
  TORCH_CHECK(false, op, " (b200 route): ", fl_b200_status_string(status), " [status ", status,
              ", cuda error ", fl_b200_last_cuda_error(), "]");
}

std::optional<RowsView> AsRows(const at::Tensor& x) {
  if (x.dim() == 0) return RowsView{1, 1, 1};
  const int64_t cols = x.size(-1);
  int64_t rows = 1;
  for (int64_t d = 0; d + 1 < x.dim(); ++d) rows *= x.size(d);
  if (cols > 1 && x.stride(-1) != 1) return std::nullopt;
  if (x.dim() == 1 || rows <= 1) return RowsView{rows, cols, std::max<int64_t>(cols, 1)};
  const int64_t ld = x.stride(-2);
  int64_t expect = ld;
  for (int64_t d = x.dim() - 2; d >= 0; --d) {
    if (x.size(d) != 1 && x.stride(d) != expect) return std::nullopt;
    expect *= x.size(d);
  }
  if (ld < cols) return std::nullopt;  // overlapping rows
  return RowsView{rows, cols, ld};
}

}  // namespace flb200::aten
