// The `b200` route: the routed aten ops on this library's sm_100a kernels
// (libfl_b200.so, include/fl_b200.h).  Each kernel validates, allocates its
// output through the flagos allocator, launches on the current stream of the
// tensor's GPU and turns a non-zero status into a TORCH_CHECK.  There is no
// CPU fallback: a dtype the kernels do not take is an error naming the op.
#include <ATen/WrapDimUtils.h>
#include <ATen/ExpandUtils.h>

#include <algorithm>
#include <numeric>

#include "ops.h"
#include "tensor_utils.h"

namespace flb200::aten {
namespace {

constexpr int kAdd = 0, kMul = 1;

int RequireDtype(at::ScalarType t, const char* op) {
  const int c = B200Dtype(t);
  TORCH_CHECK(c >= 0, op, " (b200 route): dtype ", t, " is not supported "
              "(float32, bfloat16, float16, int32, int64)");
  return c;
}

bool IsFloat(at::ScalarType t) {
  return t == at::kFloat || t == at::kBFloat16 || t == at::kHalf;
}

at::Tensor AsType(const at::Tensor& t, at::ScalarType st) {
  return t.scalar_type() == st ? t : t.to(st);
}

// ------------------------------------------------------------- add / mul --
at::Tensor BinaryScalar(const at::Tensor& a, double s, int op, double alpha, at::ScalarType rt,
                        const char* name) {
  const int code = RequireDtype(rt, name);
  at::Tensor x = AsType(a, rt).contiguous();
  at::Tensor out = at::empty(x.sizes(), x.options());
  GpuGuard g(x);
  CheckB200(fl_b200_binary_scalar(x.data_ptr(), s, out.data_ptr(), x.numel(), op, alpha, code,
                                  StreamOf(x)),
            name);
  return out;
}

at::Tensor Binary(const at::Tensor& a, const at::Tensor& b, double alpha, int op,
                  const char* name) {
  const at::ScalarType rt = at::result_type(a, b);
  // aten keeps a 0-dim CPU operand in opmath (add.cu:67-76 in the reference)
  if (IsCpuScalar(b) && !IsCpuScalar(a))
    return BinaryScalar(a, b.item<double>(), op, alpha, rt, name);
  if (IsCpuScalar(a) && !IsCpuScalar(b) && (op == kMul || alpha == 1.0))
    return BinaryScalar(b, a.item<double>(), op, 1.0, rt, name);
  TORCH_CHECK(a.device() == b.device() || IsCpuScalar(a),
              name, ": expected both operands on the same device, got ", a.device(), " and ",
              b.device());
  const int code = RequireDtype(rt, name);
  at::Tensor x = AsType(IsCpuScalar(a) ? a.to(b.device()) : a, rt);
  at::Tensor y = AsType(b, rt);
  const std::vector<int64_t> shape = at::infer_size(x.sizes(), y.sizes());
  TORCH_CHECK(shape.size() <= 8, name, " (b200 route): at most 8 dims");
  at::Tensor xe = x.expand(shape), ye = y.expand(shape);
  at::Tensor out = at::empty(shape, x.options());
  if (out.numel() == 0) return out;
  const std::vector<int64_t> sa(xe.strides().begin(), xe.strides().end());
  const std::vector<int64_t> sb(ye.strides().begin(), ye.strides().end());
  GpuGuard g(out);
  const int st = op == kAdd
      ? fl_b200_add(xe.data_ptr(), sa.data(), ye.data_ptr(), sb.data(), out.data_ptr(),
                    shape.data(), (int)shape.size(), alpha, code, StreamOf(out))
      : fl_b200_mul(xe.data_ptr(), sa.data(), ye.data_ptr(), sb.data(), out.data_ptr(),
                    shape.data(), (int)shape.size(), code, StreamOf(out));
  CheckB200(st, name);
  return out;
}

at::Tensor AddTensorB200(const at::Tensor& a, const at::Tensor& b, const at::Scalar& alpha) {
  return Binary(a, b, alpha.toDouble(), kAdd, "add.Tensor");
}
at::Tensor AddScalarB200(const at::Tensor& a, const at::Scalar& s, const at::Scalar& alpha) {
  const at::ScalarType rt = at::result_type(a, s);
  return BinaryScalar(a, s.toDouble(), kAdd, alpha.toDouble(), rt, "add.Scalar");
}
at::Tensor MulTensorB200(const at::Tensor& a, const at::Tensor& b) {
  return Binary(a, b, 1.0, kMul, "mul.Tensor");
}
at::Tensor MulScalarB200(const at::Tensor& a, const at::Scalar& s) {
  const at::ScalarType rt = at::result_type(a, s);
  return BinaryScalar(a, s.toDouble(), kMul, 1.0, rt, "mul.Scalar");
}

// ---------------------------------------------------------------- softmax --
at::Tensor SoftmaxB200(const at::Tensor& self, int64_t dim, bool half_to_float) {
  const char* name = "_softmax";
  const at::ScalarType in = self.scalar_type();
  TORCH_CHECK(IsFloat(in), name, " (b200 route): floating point input expected, got ", in);
  TORCH_CHECK(!half_to_float || in != at::kFloat,
              name, ": half_to_float is only for float16/bfloat16 input");
  const at::ScalarType ot = half_to_float ? at::kFloat : in;
  if (self.dim() == 0) return at::ones({}, self.options().dtype(ot));
  dim = at::maybe_wrap_dim(dim, self.dim());
  at::Tensor x = self.contiguous();
  at::Tensor out = at::empty(x.sizes(), x.options().dtype(ot));
  if (x.numel() == 0) return out;
  GpuGuard g(x);
  const int64_t n = x.size(dim);
  if (dim == x.dim() - 1) {
    const int64_t rows = x.numel() / n;
    CheckB200(fl_b200_softmax_lastdim(x.data_ptr(), n, out.data_ptr(), n, rows, n,
                                      B200Dtype(in), B200Dtype(ot), 0, 1, 0, StreamOf(x)),
              name);
  } else {
    int64_t outer = 1, inner = 1;
    for (int64_t d = 0; d < dim; ++d) outer *= x.size(d);
    for (int64_t d = dim + 1; d < x.dim(); ++d) inner *= x.size(d);
    CheckB200(fl_b200_softmax_middim(x.data_ptr(), out.data_ptr(), outer, n, inner,
                                     B200Dtype(in), B200Dtype(ot), StreamOf(x)),
              name);
  }
  return out;
}

// ------------------------------------------------------------- backward --
// _softmax_backward_data: dx = y * (dy - sum(dy * y)) along dim, in
// input_dtype.  Last dim on the b200 kernel; another dim moves to the last
// place (a copy each way) so the same kernel runs.
at::Tensor SoftmaxBackwardB200(const at::Tensor& grad, const at::Tensor& output, int64_t dim,
                               at::ScalarType input_dtype) {
  const char* name = "_softmax_backward_data";
  const at::ScalarType t = output.scalar_type();
  TORCH_CHECK(IsFloat(t) && grad.scalar_type() == t, name,
              " (b200 route): grad and output must share a floating dtype");
  TORCH_CHECK(grad.sizes() == output.sizes(), name, ": grad and output shapes differ");
  TORCH_CHECK(IsFloat(input_dtype) && (input_dtype == t || t == at::kFloat), name,
              ": input_dtype must be the output's dtype, or 16-bit with float32 grads");
  if (output.dim() == 0) return at::zeros({}, output.options().dtype(input_dtype));
  dim = at::maybe_wrap_dim(dim, output.dim());
  const bool last = dim == output.dim() - 1;
  at::Tensor g = (last ? grad : grad.movedim(dim, -1)).contiguous();
  at::Tensor y = (last ? output : output.movedim(dim, -1)).contiguous();
  at::Tensor dx = at::empty(y.sizes(), y.options().dtype(input_dtype));
  if (y.numel() > 0) {
    GpuGuard gd(y);
    const int64_t n = y.size(-1), rows = y.numel() / n;
    CheckB200(fl_b200_softmax_bwd(g.data_ptr(), n, y.data_ptr(), n, dx.data_ptr(), n, rows, n,
                                  B200Dtype(t), B200Dtype(input_dtype), StreamOf(y)),
              name);
  }
  return last ? dx : dx.movedim(-1, dim).contiguous();
}

// silu_backward: dx = grad * s * (1 + x (1 - s)), s = sigmoid(x).
at::Tensor SiluBackwardB200(const at::Tensor& grad, const at::Tensor& self) {
  const char* name = "silu_backward";
  const at::ScalarType t = self.scalar_type();
  TORCH_CHECK(IsFloat(t) && grad.scalar_type() == t, name,
              " (b200 route): grad and input must share a floating dtype");
  TORCH_CHECK(grad.sizes() == self.sizes(), name, ": grad and input shapes differ");
  at::Tensor g = grad.contiguous(), x = self.contiguous();
  at::Tensor dx = at::empty(x.sizes(), x.options());
  if (x.numel() > 0) {
    GpuGuard gd(x);
    CheckB200(fl_b200_silu_bwd(g.data_ptr(), x.data_ptr(), dx.data_ptr(), x.numel(),
                               B200Dtype(t), StreamOf(x)),
              name);
  }
  return dx;
}

// ------------------------------------------------ the other HF formula ops --
// silu / rsqrt / neg / cos / sin / pow.Tensor_Scalar / cat on this library's
// kernels (unary.cu), in the arithmetic of the reference's cuda route
// (csrc/aten/register.cc:405-417).  A dtype the kernels do not take (integer
// tensors, except neg on int32/int64) runs PyTorch's CUDA kernel on the same
// memory, which is what the op's cuda route runs.

// Sizes and strides of the dims before `split`, when the dims from `split`
// on are contiguous in x: the rows of fl_b200_unary / fl_b200_cat.
bool OuterDims(const at::Tensor& x, int64_t split, std::vector<int64_t>& sizes,
               std::vector<int64_t>& strides) {
  int64_t expect = 1;
  for (int64_t d = x.dim() - 1; d >= split; --d) {
    if (x.size(d) != 1 && x.stride(d) != expect) return false;
    expect *= x.size(d);
  }
  sizes.assign(x.sizes().begin(), x.sizes().begin() + split);
  strides.assign(x.strides().begin(), x.strides().begin() + split);
  return true;
}

using AtenUnary = at::Tensor (*)(const at::Tensor&);

at::Tensor UnaryB200(const at::Tensor& self, int op, double p, const char* name,
                     AtenUnary cuda_op) {
  const at::ScalarType t = self.scalar_type();
  const int code = B200Dtype(t);
  const bool takes = IsFloat(t) || (op == FL_B200_UNARY_NEG && code >= 0);
  if (!takes) return ToFlagos(cuda_op(CudaAlias(self)));
  GpuGuard g(self);
  at::Tensor x = self;
  if (x.dim() > 0 && !x.is_non_overlapping_and_dense()) {
    std::vector<int64_t> sz, st;
    if (x.stride(-1) == 1 && OuterDims(x, x.dim() - 1, sz, st)) {
      // rows of the last dim, placed by the outer dims; the output dense
      at::Tensor out = at::empty(x.sizes(), x.options());
      if (x.numel() == 0) return out;
      CheckB200(fl_b200_unary(x.data_ptr(), sz.data(), st.data(), (int)sz.size(), x.size(-1),
                              out.data_ptr(), op, p, code, StreamOf(x)),
                name);
      return out;
    }
    x = x.contiguous();
  }
  // a dense layout in any dim order: one flat pass, the output keeps the strides
  at::Tensor out = at::empty_strided(x.sizes(), x.strides(), x.options());
  if (x.numel() == 0) return out;
  CheckB200(fl_b200_unary(x.data_ptr(), nullptr, nullptr, 0, x.numel(), out.data_ptr(), op, p,
                          code, StreamOf(x)),
            name);
  return out;
}

at::Tensor SiluB200(const at::Tensor& x) {
  return UnaryB200(x, FL_B200_UNARY_SILU, 0.0, "silu", [](const at::Tensor& t) {
    return at::silu(t);
  });
}
at::Tensor RsqrtB200(const at::Tensor& x) {
  return UnaryB200(x, FL_B200_UNARY_RSQRT, 0.0, "rsqrt", [](const at::Tensor& t) {
    return at::rsqrt(t);
  });
}
at::Tensor NegB200(const at::Tensor& x) {
  return UnaryB200(x, FL_B200_UNARY_NEG, 0.0, "neg", [](const at::Tensor& t) {
    return at::neg(t);
  });
}
at::Tensor CosB200(const at::Tensor& x) {
  return UnaryB200(x, FL_B200_UNARY_COS, 0.0, "cos", [](const at::Tensor& t) {
    return at::cos(t);
  });
}
at::Tensor SinB200(const at::Tensor& x) {
  return UnaryB200(x, FL_B200_UNARY_SIN, 0.0, "sin", [](const at::Tensor& t) {
    return at::sin(t);
  });
}

// pow(tensor, scalar): the exponent converted to the tensor's dtype first,
// then 2 -> x*x, 3 -> x*x*x, else pow (pow.cu:15-46).
at::Tensor PowScalarB200(const at::Tensor& self, const at::Scalar& e) {
  const at::ScalarType t = self.scalar_type();
  if (!IsFloat(t) || e.isComplex()) return ToFlagos(at::pow(CudaAlias(self), e));
  double ed;
  if (t == at::kBFloat16) ed = static_cast<float>(e.to<at::BFloat16>());
  else if (t == at::kHalf) ed = static_cast<float>(e.to<at::Half>());
  else ed = e.to<float>();
  const int op = ed == 2.0 ? FL_B200_UNARY_SQUARE
                           : (ed == 3.0 ? FL_B200_UNARY_CUBE : FL_B200_UNARY_POW);
  return UnaryB200(self, op, ed, "pow.Tensor_Scalar", nullptr);
}

// cat: inputs of one dtype on one flagos device as row blocks (fl_b200_cat);
// anything else (dtype promotion, a mismatch to report) goes to PyTorch's cat.
at::Tensor CatB200(const at::ITensorListRef& tensors, int64_t dim) {
  const char* name = "cat";
  std::vector<at::Tensor> all;
  for (const at::Tensor& t : tensors) all.push_back(t);
  auto cuda_cat = [&]() {
    std::vector<at::Tensor> v;
    for (const at::Tensor& t : all) v.push_back(CudaAlias(t));
    return ToFlagos(at::cat(v, dim));
  };
  // legacy empty tensors (1-D, size 0) take no part, as in PyTorch
  std::vector<at::Tensor> ts;
  for (const at::Tensor& t : all)
    if (!(t.dim() == 1 && t.size(0) == 0)) ts.push_back(t);
  if (ts.empty() || all.empty()) return cuda_cat();
  const at::Tensor& t0 = ts[0];
  const int64_t nd = t0.dim();
  if (nd == 0) return cuda_cat();
  const int64_t d = at::maybe_wrap_dim(dim, nd);
  // a byte copy: any dtype of 1, 2, 4 or 8 bytes
  if (!t0.is_privateuseone() || t0.element_size() > 8) return cuda_cat();
  int64_t cat_size = 0;
  for (const at::Tensor& t : ts) {
    if (t.dim() != nd || t.scalar_type() != t0.scalar_type() || t.device() != t0.device())
      return cuda_cat();
    for (int64_t i = 0; i < nd; ++i)
      if (i != d && t.size(i) != t0.size(i)) return cuda_cat();  // its error message
    cat_size += t.size(d);
  }
  std::vector<int64_t> shape(t0.sizes().begin(), t0.sizes().end());
  shape[d] = cat_size;
  at::Tensor out = at::empty(shape, t0.options());
  if (out.numel() == 0) return out;
  std::vector<at::Tensor> keep;  // contiguous copies of inputs the kernel cannot read
  std::vector<const void*> srcs;
  std::vector<int64_t> widths, strides;
  std::vector<int64_t> row_sizes(t0.sizes().begin(), t0.sizes().begin() + d);
  for (const at::Tensor& t0k : ts) {
    at::Tensor t = t0k;
    std::vector<int64_t> sz, st;
    if (!OuterDims(t, d, sz, st)) {
      keep.push_back(t.contiguous());
      t = keep.back();
      OuterDims(t, d, sz, st);
    }
    srcs.push_back(t.data_ptr());
    strides.insert(strides.end(), st.begin(), st.end());
    int64_t w = 1;  // the input's elements per row: its sizes from d on
    for (int64_t i = d; i < nd; ++i) w *= t.size(i);
    widths.push_back(w);
  }
  GpuGuard g(out);
  CheckB200(fl_b200_cat(srcs.data(), strides.data(), widths.data(), (int)srcs.size(),
                        row_sizes.data(), (int)row_sizes.size(), out.data_ptr(),
                        (int)t0.element_size(), StreamOf(out)),
            name);
  return out;
}

// ------------------------------------------------------------- reductions --
enum class Red { kSum, kMean, kAmax, kArgmax };

struct Workspace {
  at::Tensor buf;
  void* ptr = nullptr;
  size_t bytes = 0;
  Workspace(const at::Tensor& like, int64_t rows, int64_t cols) {
    bytes = fl_b200_reduce_workspace_size(rows, cols);
    if (bytes) {
      buf = at::empty({(int64_t)bytes}, like.options().dtype(at::kByte));
      ptr = buf.data_ptr();
    }
  }
};

// Sorted, unique, wrapped reduction dims; all dims when `dims` is empty.
std::vector<int64_t> NormDims(const at::Tensor& x, at::IntArrayRef dims) {
  std::vector<int64_t> d;
  if (dims.empty()) {
    d.resize(x.dim());
    std::iota(d.begin(), d.end(), 0);
    return d;
  }
  for (int64_t v : dims) d.push_back(at::maybe_wrap_dim(v, x.dim()));
  std::sort(d.begin(), d.end());
  d.erase(std::unique(d.begin(), d.end()), d.end());
  return d;
}

std::vector<int64_t> OutShape(const at::Tensor& x, const std::vector<int64_t>& red, bool keepdim) {
  std::vector<int64_t> s;
  for (int64_t d = 0; d < x.dim(); ++d) {
    const bool r = std::binary_search(red.begin(), red.end(), d);
    if (!r) s.push_back(x.size(d));
    else if (keepdim) s.push_back(1);
  }
  return s;
}

// One launch of the row reduction `kind` over x viewed as [rows, cols].
void LaunchRows(Red kind, const at::Tensor& x, int64_t rows, int64_t cols, int64_t ld,
                at::Tensor& out, int in_code, int out_code, const char* name) {
  Workspace ws(x, rows, cols);
  const auto s = StreamOf(x);
  int st = FL_B200_OK;
  switch (kind) {
    case Red::kSum:
      st = fl_b200_reduce_sum_lastdim(x.data_ptr(), ld, rows, cols, out.data_ptr(), in_code,
                                      out_code, ws.ptr, ws.bytes, s);
      break;
    case Red::kMean:
      st = fl_b200_reduce_mean_lastdim(x.data_ptr(), ld, rows, cols, out.data_ptr(), in_code,
                                       out_code, ws.ptr, ws.bytes, s);
      break;
    case Red::kAmax:
      st = fl_b200_reduce_amax_lastdim(x.data_ptr(), ld, rows, cols, out.data_ptr(), in_code,
                                       ws.ptr, ws.bytes, s);
      break;
    case Red::kArgmax:
      st = fl_b200_argmax_lastdim(x.data_ptr(), ld, rows, cols,
                                  static_cast<int64_t*>(out.data_ptr()), in_code, ws.ptr,
                                  ws.bytes, s);
      break;
  }
  CheckB200(st, name);
}

// Reduces x over `red` (sorted dims) into a fresh tensor of `out_t`.
at::Tensor Reduce(Red kind, const at::Tensor& self, const std::vector<int64_t>& red, bool keepdim,
                  at::ScalarType out_t, const char* name) {
  const int in_code = RequireDtype(self.scalar_type(), name);
  const int out_code = RequireDtype(out_t, name);
  at::Tensor out = at::empty(OutShape(self, red, keepdim), self.options().dtype(out_t));
  GpuGuard g(self);
  if (self.dim() == 0) {  // reducing a scalar is the identity
    out.copy_(kind == Red::kArgmax ? at::zeros({}, out.options()) : self.to(out_t).reshape({}));
    return out;
  }
  if (out.numel() == 0) return out;
  const int64_t nd = self.dim();
  // Trailing dims [k, nd) reduced on a contiguous tensor: one rows view.
  const bool trailing = red.back() == nd - 1 && (int64_t)red.size() == nd - red.front() &&
                        red.front() == nd - (int64_t)red.size();
  if (trailing) {
    at::Tensor x = self.contiguous();
    int64_t cols = 1;
    for (int64_t d : red) cols *= x.size(d);
    const int64_t rows = cols ? x.numel() / cols : out.numel();
    LaunchRows(kind, x, rows, cols, std::max<int64_t>(cols, 1), out, in_code, out_code, name);
    return out;
  }
  // One middle dim of a float tensor: reduce in place over [outer, n, inner].
  if (red.size() == 1 && kind != Red::kArgmax && IsFloat(self.scalar_type()) &&
      IsFloat(out_t)) {
    at::Tensor x = self.contiguous();
    const int64_t d = red[0];
    int64_t outer = 1, inner = 1;
    for (int64_t i = 0; i < d; ++i) outer *= x.size(i);
    for (int64_t i = d + 1; i < nd; ++i) inner *= x.size(i);
    const int op = kind == Red::kSum ? 0 : (kind == Red::kMean ? 1 : 2);
    CheckB200(fl_b200_reduce_middim(x.data_ptr(), outer, x.size(d), inner, out.data_ptr(), op,
                                    in_code, out_code, StreamOf(x)),
              name);
    return out;
  }
  // Anything else: move the reduced dims last, then one rows reduction.
  std::vector<int64_t> perm;
  for (int64_t d = 0; d < nd; ++d)
    if (!std::binary_search(red.begin(), red.end(), d)) perm.push_back(d);
  for (int64_t d : red) perm.push_back(d);
  at::Tensor x = self.permute(perm).contiguous();
  int64_t cols = 1;
  for (int64_t d : red) cols *= self.size(d);
  const int64_t rows = out.numel();
  LaunchRows(kind, x, rows, cols, std::max<int64_t>(cols, 1), out, in_code, out_code, name);
  return out;
}

at::Tensor SumDimB200(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim,
                      std::optional<at::ScalarType> dtype) {
  const char* name = "sum.dim_IntList";
  at::ScalarType in = self.scalar_type();
  const bool integral = at::isIntegralType(in, /*includeBool=*/true);
  const at::ScalarType out_t = dtype ? *dtype : (integral ? at::kLong : in);
  at::Tensor x = self;
  if (integral) {
    TORCH_CHECK(out_t == at::kLong, name, " (b200 route): integer sums produce int64");
    if (in != at::kInt && in != at::kLong) x = self.to(at::kInt);  // bool/int8/int16: exact
  } else {
    TORCH_CHECK(IsFloat(in) && IsFloat(out_t), name, " (b200 route): dtype ", in, " -> ", out_t,
                " is not supported");
  }
  const auto red = NormDims(x, dim.value_or(at::IntArrayRef{}));
  return Reduce(Red::kSum, x, red, keepdim, out_t, name);
}

at::Tensor MeanDimB200(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim,
                       std::optional<at::ScalarType> dtype) {
  const char* name = "mean.dim";
  const at::ScalarType out_t = dtype ? *dtype : self.scalar_type();
  TORCH_CHECK(IsFloat(self.scalar_type()) && IsFloat(out_t),
              "mean(): could not infer output dtype. Input dtype must be either a floating "
              "point or complex dtype. Got: ", self.scalar_type());
  const auto red = NormDims(self, dim.value_or(at::IntArrayRef{}));
  return Reduce(Red::kMean, self, red, keepdim, out_t, name);
}

at::Tensor AmaxB200(const at::Tensor& self, at::IntArrayRef dim, bool keepdim) {
  const char* name = "amax";
  TORCH_CHECK(IsFloat(self.scalar_type()), name, " (b200 route): dtype ", self.scalar_type(),
              " is not supported (float32, bfloat16, float16)");
  const auto red = NormDims(self, dim);
  for (int64_t d : red)
    TORCH_CHECK(self.size(d) > 0, "amax(): Expected reduction dim ", d, " to have non-zero size.");
  return Reduce(Red::kAmax, self, red, keepdim, self.scalar_type(), name);
}

at::Tensor ArgmaxB200(const at::Tensor& self, std::optional<int64_t> dim, bool keepdim) {
  const char* name = "argmax";
  TORCH_CHECK(IsFloat(self.scalar_type()), name, " (b200 route): dtype ", self.scalar_type(),
              " is not supported (float32, bfloat16, float16)");
  if (!dim) {
    TORCH_CHECK(self.numel() > 0, "argmax(): Expected reduction dim to be specified for "
                "input.numel() == 0.");
    at::Tensor flat = self.reshape({-1});
    at::Tensor r = Reduce(Red::kArgmax, flat, {0}, false, at::kLong, name);
    return keepdim ? r.reshape(std::vector<int64_t>(self.dim(), 1)) : r;
  }
  const int64_t d = at::maybe_wrap_dim(*dim, std::max<int64_t>(self.dim(), 1));
  if (self.dim() > 0)
    TORCH_CHECK(self.size(d) > 0, "argmax(): Expected reduction dim ", d,
                " to have non-zero size.");
  return Reduce(Red::kArgmax, self, {d}, keepdim, at::kLong, name);
}

}  // namespace

FLB_REGISTER_KERNEL(AddTensorFn, add_tensor_dispatcher, Backend::kB200, AddTensorB200)
FLB_REGISTER_KERNEL(AddScalarFn, add_scalar_dispatcher, Backend::kB200, AddScalarB200)
FLB_REGISTER_KERNEL(MulTensorFn, mul_tensor_dispatcher, Backend::kB200, MulTensorB200)
FLB_REGISTER_KERNEL(MulScalarFn, mul_scalar_dispatcher, Backend::kB200, MulScalarB200)
FLB_REGISTER_KERNEL(SoftmaxFn, softmax_dispatcher, Backend::kB200, SoftmaxB200)
FLB_REGISTER_KERNEL(ReduceDimFn, sum_dim_dispatcher, Backend::kB200, SumDimB200)
FLB_REGISTER_KERNEL(ReduceDimFn, mean_dim_dispatcher, Backend::kB200, MeanDimB200)
FLB_REGISTER_KERNEL(AmaxFn, amax_dispatcher, Backend::kB200, AmaxB200)
FLB_REGISTER_KERNEL(ArgmaxFn, argmax_dispatcher, Backend::kB200, ArgmaxB200)
FLB_REGISTER_KERNEL(SoftmaxBackwardFn, softmax_backward_dispatcher, Backend::kB200,
                    SoftmaxBackwardB200)
FLB_REGISTER_KERNEL(SiluBackwardFn, silu_backward_dispatcher, Backend::kB200, SiluBackwardB200)
FLB_REGISTER_KERNEL(UnaryFn, silu_dispatcher, Backend::kB200, SiluB200)
FLB_REGISTER_KERNEL(UnaryFn, rsqrt_dispatcher, Backend::kB200, RsqrtB200)
FLB_REGISTER_KERNEL(UnaryFn, neg_dispatcher, Backend::kB200, NegB200)
FLB_REGISTER_KERNEL(UnaryFn, cos_dispatcher, Backend::kB200, CosB200)
FLB_REGISTER_KERNEL(UnaryFn, sin_dispatcher, Backend::kB200, SinB200)
FLB_REGISTER_KERNEL(PowScalarFn, pow_tensor_scalar_dispatcher, Backend::kB200, PowScalarB200)
FLB_REGISTER_KERNEL(CatFn, cat_dispatcher, Backend::kB200, CatB200)

}  // namespace flb200::aten
