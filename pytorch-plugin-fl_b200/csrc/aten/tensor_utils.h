// Helpers shared by the flagos aten kernels.
#pragma once

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "../../../include/fl_b200.h"

namespace flb200::aten {

// A tensor of device type `target` over the same memory, sizes, strides and
// storage offset as `t` (flagos <-> cuda: same GPU, same bytes).  The alias
// keeps t's storage alive.  Tensors already of type `target` (and CPU
// tensors) are returned unchanged.
at::Tensor Rewrap(const at::Tensor& t, c10::DeviceType target);
inline at::Tensor CudaAlias(const at::Tensor& t) {
  return t.defined() && t.is_privateuseone() ? Rewrap(t, c10::DeviceType::CUDA) : t;
}
inline at::Tensor ToFlagos(const at::Tensor& t) {
  return t.defined() && t.is_cuda() ? Rewrap(t, c10::DeviceType::PrivateUse1) : t;
}

// fl_b200_dtype of a scalar type, or -1 when the b200 kernels do not take it.
int B200Dtype(at::ScalarType t);
// Raises with the op name and the library's status string.
void CheckB200(int status, const char* op);

// Current CUDA stream of the tensor's GPU (flagos streams are CUDA streams).
inline cudaStream_t StreamOf(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

// True for a 0-dim CPU tensor that aten treats as a scalar operand.
inline bool IsCpuScalar(const at::Tensor& t) {
  return t.defined() && t.device().is_cpu() && t.dim() == 0;
}

// Rows view of x over its last dim: (rows, cols, leading stride) when x's
// rows are evenly spaced with a unit last-dim stride, else nullopt.
struct RowsView {
  int64_t rows, cols, ld;
};
std::optional<RowsView> AsRows(const at::Tensor& x);

// Device guard for a flagos (or cuda) tensor's GPU.
class GpuGuard {
 public:
  explicit GpuGuard(const at::Tensor& t) : g_(t.device().index()) {}

 private:
  c10::cuda::CUDAGuard g_;
};

}  // namespace flb200::aten
