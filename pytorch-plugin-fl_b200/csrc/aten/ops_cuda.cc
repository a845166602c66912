// The `cuda` route: PyTorch's own CUDA kernels run on CUDA aliases of the
// flagos tensors (same memory, same GPU).  This is what the reference's cuda
// backend runs (csrc/aten/backends/cuda/*.cu wrap ATen's CUDALoops.cuh /
// Reduce.cuh / SoftMax), here without the device-type flipping of
// csrc/aten/device_boxing.h: an alias is a separate tensor over the bytes.
#include "ops.h"
#include "tensor_utils.h"

namespace flb200::aten {

FLB_DEFINE_DISPATCHER(AddTensorFn, add_tensor_dispatcher, "add.Tensor")
FLB_DEFINE_DISPATCHER(AddScalarFn, add_scalar_dispatcher, "add.Scalar")
FLB_DEFINE_DISPATCHER(MulTensorFn, mul_tensor_dispatcher, "mul.Tensor")
FLB_DEFINE_DISPATCHER(MulScalarFn, mul_scalar_dispatcher, "mul.Scalar")
FLB_DEFINE_DISPATCHER(SoftmaxFn, softmax_dispatcher, "_softmax")
FLB_DEFINE_DISPATCHER(ReduceDimFn, sum_dim_dispatcher, "sum.dim_IntList")
FLB_DEFINE_DISPATCHER(ReduceDimFn, mean_dim_dispatcher, "mean.dim")
FLB_DEFINE_DISPATCHER(AmaxFn, amax_dispatcher, "amax")
FLB_DEFINE_DISPATCHER(ArgmaxFn, argmax_dispatcher, "argmax")
FLB_DEFINE_DISPATCHER(UnaryFn, silu_dispatcher, "silu")
FLB_DEFINE_DISPATCHER(UnaryFn, rsqrt_dispatcher, "rsqrt")
FLB_DEFINE_DISPATCHER(UnaryFn, neg_dispatcher, "neg")
FLB_DEFINE_DISPATCHER(UnaryFn, cos_dispatcher, "cos")
FLB_DEFINE_DISPATCHER(UnaryFn, sin_dispatcher, "sin")
FLB_DEFINE_DISPATCHER(PowScalarFn, pow_tensor_scalar_dispatcher, "pow.Tensor_Scalar")
FLB_DEFINE_DISPATCHER(CatFn, cat_dispatcher, "cat")
FLB_DEFINE_DISPATCHER(SoftmaxBackwardFn, softmax_backward_dispatcher, "_softmax_backward_data")
FLB_DEFINE_DISPATCHER(SiluBackwardFn, silu_backward_dispatcher, "silu_backward")

namespace {

at::Tensor AddTensorCuda(const at::Tensor& a, const at::Tensor& b, const at::Scalar& alpha) {
  return ToFlagos(at::add(CudaAlias(a), CudaAlias(b), alpha));
}
at::Tensor AddScalarCuda(const at::Tensor& a, const at::Scalar& b, const at::Scalar& alpha) {
  return ToFlagos(at::add(CudaAlias(a), b, alpha));
}
at::Tensor MulTensorCuda(const at::Tensor& a, const at::Tensor& b) {
  return ToFlagos(at::mul(CudaAlias(a), CudaAlias(b)));
}
at::Tensor MulScalarCuda(const at::Tensor& a, const at::Scalar& b) {
  return ToFlagos(at::mul(CudaAlias(a), b));
}
at::Tensor SoftmaxCuda(const at::Tensor& x, int64_t dim, bool half_to_float) {
  return ToFlagos(at::_softmax(CudaAlias(x), dim, half_to_float));
}
at::Tensor SumDimCuda(const at::Tensor& x, at::OptionalIntArrayRef dim, bool keepdim,
                      std::optional<at::ScalarType> dtype) {
  return ToFlagos(at::sum(CudaAlias(x), dim, keepdim, dtype));
}
at::Tensor MeanDimCuda(const at::Tensor& x, at::OptionalIntArrayRef dim, bool keepdim,
                       std::optional<at::ScalarType> dtype) {
  return ToFlagos(at::mean(CudaAlias(x), dim, keepdim, dtype));
}
at::Tensor AmaxCuda(const at::Tensor& x, at::IntArrayRef dim, bool keepdim) {
  return ToFlagos(at::amax(CudaAlias(x), dim, keepdim));
}
at::Tensor ArgmaxCuda(const at::Tensor& x, std::optional<int64_t> dim, bool keepdim) {
  return ToFlagos(at::argmax(CudaAlias(x), dim, keepdim));
}
at::Tensor SiluCuda(const at::Tensor& x) { return ToFlagos(at::silu(CudaAlias(x))); }
at::Tensor RsqrtCuda(const at::Tensor& x) { return ToFlagos(at::rsqrt(CudaAlias(x))); }
at::Tensor NegCuda(const at::Tensor& x) { return ToFlagos(at::neg(CudaAlias(x))); }
at::Tensor CosCuda(const at::Tensor& x) { return ToFlagos(at::cos(CudaAlias(x))); }
at::Tensor SinCuda(const at::Tensor& x) { return ToFlagos(at::sin(CudaAlias(x))); }
at::Tensor PowScalarCuda(const at::Tensor& x, const at::Scalar& e) {
  return ToFlagos(at::pow(CudaAlias(x), e));
}
at::Tensor CatCuda(const at::ITensorListRef& ts, int64_t dim) {
  std::vector<at::Tensor> v;
  for (const at::Tensor& t : ts) v.push_back(CudaAlias(t));
  return ToFlagos(at::cat(v, dim));
}

at::Tensor SoftmaxBackwardCuda(const at::Tensor& g, const at::Tensor& y, int64_t dim,
                               at::ScalarType input_dtype) {
  return ToFlagos(at::_softmax_backward_data(CudaAlias(g), CudaAlias(y), dim, input_dtype));
}
at::Tensor SiluBackwardCuda(const at::Tensor& g, const at::Tensor& x) {
  return ToFlagos(at::silu_backward(CudaAlias(g), CudaAlias(x)));
}

}  // namespace

FLB_REGISTER_KERNEL(AddTensorFn, add_tensor_dispatcher, Backend::kCuda, AddTensorCuda)
FLB_REGISTER_KERNEL(AddScalarFn, add_scalar_dispatcher, Backend::kCuda, AddScalarCuda)
FLB_REGISTER_KERNEL(MulTensorFn, mul_tensor_dispatcher, Backend::kCuda, MulTensorCuda)
FLB_REGISTER_KERNEL(MulScalarFn, mul_scalar_dispatcher, Backend::kCuda, MulScalarCuda)
FLB_REGISTER_KERNEL(SoftmaxFn, softmax_dispatcher, Backend::kCuda, SoftmaxCuda)
FLB_REGISTER_KERNEL(ReduceDimFn, sum_dim_dispatcher, Backend::kCuda, SumDimCuda)
FLB_REGISTER_KERNEL(ReduceDimFn, mean_dim_dispatcher, Backend::kCuda, MeanDimCuda)
FLB_REGISTER_KERNEL(AmaxFn, amax_dispatcher, Backend::kCuda, AmaxCuda)
FLB_REGISTER_KERNEL(ArgmaxFn, argmax_dispatcher, Backend::kCuda, ArgmaxCuda)
FLB_REGISTER_KERNEL(UnaryFn, silu_dispatcher, Backend::kCuda, SiluCuda)
FLB_REGISTER_KERNEL(UnaryFn, rsqrt_dispatcher, Backend::kCuda, RsqrtCuda)
FLB_REGISTER_KERNEL(UnaryFn, neg_dispatcher, Backend::kCuda, NegCuda)
FLB_REGISTER_KERNEL(UnaryFn, cos_dispatcher, Backend::kCuda, CosCuda)
FLB_REGISTER_KERNEL(UnaryFn, sin_dispatcher, Backend::kCuda, SinCuda)
FLB_REGISTER_KERNEL(PowScalarFn, pow_tensor_scalar_dispatcher, Backend::kCuda, PowScalarCuda)
FLB_REGISTER_KERNEL(CatFn, cat_dispatcher, Backend::kCuda, CatCuda)
FLB_REGISTER_KERNEL(SoftmaxBackwardFn, softmax_backward_dispatcher, Backend::kCuda,
                    SoftmaxBackwardCuda)
FLB_REGISTER_KERNEL(SiluBackwardFn, silu_backward_dispatcher, Backend::kCuda, SiluBackwardCuda)

}  // namespace flb200::aten
