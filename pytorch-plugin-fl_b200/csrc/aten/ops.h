// Routed aten ops of the flagos device: one kernel type and one Dispatcher
// per op, with the signatures of the reference's stubs (csrc/aten/<op>.h,
// e.g. softmax.h:10, sum.h:10-11, mean.h:10-11, add.h:10, mul.h:10,
// silu_backward.h) plus the ops the reference leaves to its CPU fallback
// (amax, argmax, _softmax_backward_data).
#pragma once

#include <ATen/ATen.h>

#include "dispatch.h"

namespace flb200::aten {

using AddTensorFn = at::Tensor (*)(const at::Tensor&, const at::Tensor&, const at::Scalar&);
using AddScalarFn = at::Tensor (*)(const at::Tensor&, const at::Scalar&, const at::Scalar&);
using MulTensorFn = at::Tensor (*)(const at::Tensor&, const at::Tensor&);
using MulScalarFn = at::Tensor (*)(const at::Tensor&, const at::Scalar&);
using SoftmaxFn = at::Tensor (*)(const at::Tensor&, int64_t, bool);
using ReduceDimFn = at::Tensor (*)(const at::Tensor&, at::OptionalIntArrayRef, bool,
                                   std::optional<at::ScalarType>);
using AmaxFn = at::Tensor (*)(const at::Tensor&, at::IntArrayRef, bool);
using ArgmaxFn = at::Tensor (*)(const at::Tensor&, std::optional<int64_t>, bool);
using UnaryFn = at::Tensor (*)(const at::Tensor&);
using PowScalarFn = at::Tensor (*)(const at::Tensor&, const at::Scalar&);
using CatFn = at::Tensor (*)(const at::ITensorListRef&, int64_t);
using SoftmaxBackwardFn = at::Tensor (*)(const at::Tensor&, const at::Tensor&, int64_t,
                                         at::ScalarType);
using SiluBackwardFn = at::Tensor (*)(const at::Tensor&, const at::Tensor&);

FLB_DECLARE_DISPATCHER(AddTensorFn, add_tensor_dispatcher)
FLB_DECLARE_DISPATCHER(AddScalarFn, add_scalar_dispatcher)
FLB_DECLARE_DISPATCHER(MulTensorFn, mul_tensor_dispatcher)
FLB_DECLARE_DISPATCHER(MulScalarFn, mul_scalar_dispatcher)
FLB_DECLARE_DISPATCHER(SoftmaxFn, softmax_dispatcher)
FLB_DECLARE_DISPATCHER(ReduceDimFn, sum_dim_dispatcher)
FLB_DECLARE_DISPATCHER(ReduceDimFn, mean_dim_dispatcher)
FLB_DECLARE_DISPATCHER(AmaxFn, amax_dispatcher)
FLB_DECLARE_DISPATCHER(ArgmaxFn, argmax_dispatcher)
FLB_DECLARE_DISPATCHER(UnaryFn, silu_dispatcher)
FLB_DECLARE_DISPATCHER(UnaryFn, rsqrt_dispatcher)
FLB_DECLARE_DISPATCHER(UnaryFn, neg_dispatcher)
FLB_DECLARE_DISPATCHER(UnaryFn, cos_dispatcher)
FLB_DECLARE_DISPATCHER(UnaryFn, sin_dispatcher)
FLB_DECLARE_DISPATCHER(PowScalarFn, pow_tensor_scalar_dispatcher)
FLB_DECLARE_DISPATCHER(CatFn, cat_dispatcher)
FLB_DECLARE_DISPATCHER(SoftmaxBackwardFn, softmax_backward_dispatcher)
FLB_DECLARE_DISPATCHER(SiluBackwardFn, silu_backward_dispatcher)

}  // namespace flb200::aten
