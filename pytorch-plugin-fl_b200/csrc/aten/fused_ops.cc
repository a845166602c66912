// flagos:: fused ops -- the kernels the HF hooks call in place of the
// HuggingFace formulas (transformers models/qwen3/modeling_qwen3.py:59-64,
// 81-82, 138-181, 209-213, 248-268).  Registered for the flagos device and for plain
// CUDA tensors (the memory is the same kind); each op allocates its outputs
// on the input's device and launches on that device's current stream.
#include <torch/library.h>

#include "tensor_utils.h"

namespace flb200::aten {
namespace {

int Rounding(c10::string_view r) {
  if (r == "fused") return FL_B200_ROUND_FUSED;
  if (r == "chain") return FL_B200_ROUND_CHAIN;
  TORCH_CHECK(false, "flagos: rounding must be 'fused' or 'chain', got '", std::string(r), "'");
}

int FloatCode(const at::Tensor& t, const char* op) {
  const int c = B200Dtype(t.scalar_type());
  TORCH_CHECK(c == FL_B200_F32 || c == FL_B200_BF16 || c == FL_B200_F16, op,
              ": float32, bfloat16 or float16 expected, got ", t.scalar_type());
  return c;
}

void SameDevice(const at::Tensor& a, const at::Tensor& b, const char* op) {
  TORCH_CHECK(a.device() == b.device(), op, ": tensors on ", a.device(), " and ", b.device());
}

RowsView Rows(const at::Tensor& x, at::Tensor& keep) {
  auto r = AsRows(x);
  if (r) {
    keep = x;
    return *r;
  }
  keep = x.contiguous();
  return *AsRows(keep);
}

// ---------------------------------------------------------------- RMSNorm --
at::Tensor RmsNorm(const at::Tensor& x_in, const at::Tensor& weight, double eps,
                   c10::string_view rounding) {
  const char* op = "flagos::rms_norm";
  const int code = FloatCode(x_in, op);
  SameDevice(x_in, weight, op);
  TORCH_CHECK(weight.scalar_type() == x_in.scalar_type() && weight.dim() == 1 &&
                  weight.numel() == x_in.size(-1),
              op, ": weight must be a [hidden] tensor of x's dtype");
  at::Tensor x;
  const RowsView r = Rows(x_in, x);
  at::Tensor w = weight.contiguous();
  at::Tensor out = at::empty(x.sizes(), x.options());
  GpuGuard g(x);
  CheckB200(fl_b200_rms_norm_fwd(x.data_ptr(), r.ld, w.data_ptr(), out.data_ptr(), r.cols,
                                 r.rows, r.cols, (float)eps, code, Rounding(rounding),
                                 StreamOf(x)),
            op);
  return out;
}

std::tuple<at::Tensor, at::Tensor> AddRmsNorm(const at::Tensor& x_in, const at::Tensor& res_in,
                                              const at::Tensor& weight, double eps,
                                              c10::string_view rounding) {
  const char* op = "flagos::add_rms_norm";
  const int code = FloatCode(x_in, op);
  SameDevice(x_in, res_in, op);
  SameDevice(x_in, weight, op);
  TORCH_CHECK(x_in.sizes() == res_in.sizes() && x_in.scalar_type() == res_in.scalar_type(),
              op, ": x and residual must match");
  TORCH_CHECK(weight.scalar_type() == x_in.scalar_type() && weight.numel() == x_in.size(-1),
              op, ": weight must be a [hidden] tensor of x's dtype");
  at::Tensor x = x_in.contiguous(), y = res_in.contiguous(), w = weight.contiguous();
  at::Tensor h = at::empty(x.sizes(), x.options());
  at::Tensor out = at::empty(x.sizes(), x.options());
  const int64_t cols = x.size(-1), rows = cols ? x.numel() / cols : 0;
  GpuGuard g(x);
  CheckB200(fl_b200_add_rms_norm_fwd(x.data_ptr(), y.data_ptr(), h.data_ptr(), w.data_ptr(),
                                     out.data_ptr(), rows, cols, (float)eps, code,
                                     Rounding(rounding), StreamOf(x)),
            op);
  return {out, h};
}

// ------------------------------------------------------------------- RoPE --
struct Bhsd {
  int64_t B, H, S, D, sb, sh, ss;
};
Bhsd Layout(const at::Tensor& t, int64_t unsqueeze_dim, const char* op) {
  TORCH_CHECK(t.dim() == 4, op, ": q/k must be 4-D");
  TORCH_CHECK(t.stride(3) == 1, op, ": the head dim must be contiguous");
  if (unsqueeze_dim == 1)  // [B, H, S, D]
    return {t.size(0), t.size(1), t.size(2), t.size(3), t.stride(0), t.stride(1), t.stride(2)};
  TORCH_CHECK(unsqueeze_dim == 2, op, ": unsqueeze_dim must be 1 ([B,H,S,D]) or 2 ([B,S,H,D])");
  return {t.size(0), t.size(2), t.size(1), t.size(3), t.stride(0), t.stride(2), t.stride(1)};
}

// cos/sin as [S, D], [B, S, D] or [B, 1, S, D]: strides over (b, s).
std::pair<int64_t, int64_t> TableStrides(const at::Tensor& c, int64_t B, int64_t S, int64_t D,
                                         const char* op) {
  at::Tensor t = c.dim() == 4 ? c.squeeze(1) : c;
  TORCH_CHECK(t.stride(-1) == 1 || D == 1, op, ": cos/sin last dim must be contiguous");
  if (t.dim() == 2) {
    TORCH_CHECK(t.size(0) == S && t.size(1) == D, op, ": cos/sin shape mismatch");
    return {0, t.stride(0)};
  }
  TORCH_CHECK(t.dim() == 3 && t.size(1) == S && t.size(2) == D && (t.size(0) == B || t.size(0) == 1),
              op, ": cos/sin must be [S, D], [B, S, D] or [B, 1, S, D]");
  return {t.size(0) == 1 ? 0 : t.stride(0), t.stride(1)};
}

std::tuple<at::Tensor, at::Tensor> RopeImpl(const at::Tensor& q, const at::Tensor& k,
                                            const at::Tensor* wq, const at::Tensor* wk,
                                            const at::Tensor& cos, const at::Tensor& sin,
                                            double eps, int64_t unsqueeze_dim,
                                            c10::string_view rounding, const char* op) {
  const int code = FloatCode(q, op);
  SameDevice(q, k, op);
  SameDevice(q, cos, op);
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && cos.scalar_type() == q.scalar_type() &&
                  sin.scalar_type() == q.scalar_type(),
              op, ": q, k, cos and sin must share a dtype");
  const Bhsd lq = Layout(q, unsqueeze_dim, op), lk = Layout(k, unsqueeze_dim, op);
  TORCH_CHECK(lq.B == lk.B && lq.S == lk.S && lq.D == lk.D, op, ": q and k disagree");
  const auto cs = TableStrides(cos, lq.B, lq.S, lq.D, op);
  TORCH_CHECK(TableStrides(sin, lq.B, lq.S, lq.D, op) == cs, op,
              ": cos and sin must share a layout");
  at::Tensor qo = at::empty_like(q), ko = at::empty_like(k);
  const Bhsd oq = Layout(qo, unsqueeze_dim, op), ok = Layout(ko, unsqueeze_dim, op);
  GpuGuard g(q);
  int st;
  if (wq) {
    TORCH_CHECK(wq->numel() == lq.D && wk->numel() == lq.D &&
                    wq->scalar_type() == q.scalar_type() && wk->scalar_type() == q.scalar_type(),
                op, ": q/k norm weights must be [head_dim] tensors of q's dtype");
    at::Tensor wqc = wq->contiguous(), wkc = wk->contiguous();
    st = fl_b200_rms_norm_rope(q.data_ptr(), qo.data_ptr(), lq.H, lq.sb, lq.sh, lq.ss, oq.sb,
                               oq.sh, oq.ss, wqc.data_ptr(), k.data_ptr(), ko.data_ptr(), lk.H,
                               lk.sb, lk.sh, lk.ss, ok.sb, ok.sh, ok.ss, wkc.data_ptr(),
                               cos.data_ptr(), sin.data_ptr(), cs.first, cs.second, lq.B, lq.S,
                               lq.D, (float)eps, code, Rounding(rounding), StreamOf(q));
  } else {
    st = fl_b200_rope_qk(q.data_ptr(), qo.data_ptr(), lq.H, lq.sb, lq.sh, lq.ss, oq.sb, oq.sh,
                         oq.ss, k.data_ptr(), ko.data_ptr(), lk.H, lk.sb, lk.sh, lk.ss, ok.sb,
                         ok.sh, ok.ss, cos.data_ptr(), sin.data_ptr(), cs.first, cs.second,
                         lq.B, lq.S, lq.D, code, Rounding(rounding), StreamOf(q));
  }
  CheckB200(st, op);
  return {qo, ko};
}

std::tuple<at::Tensor, at::Tensor> RopeQk(const at::Tensor& q, const at::Tensor& k,
                                          const at::Tensor& cos, const at::Tensor& sin,
                                          int64_t unsqueeze_dim, c10::string_view rounding) {
  return RopeImpl(q, k, nullptr, nullptr, cos, sin, 0.0, unsqueeze_dim, rounding,
                  "flagos::rope_qk");
}

std::tuple<at::Tensor, at::Tensor> RmsNormRope(const at::Tensor& q, const at::Tensor& k,
                                               const at::Tensor& q_weight,
                                               const at::Tensor& k_weight,
                                               const at::Tensor& cos, const at::Tensor& sin,
                                               double eps, int64_t unsqueeze_dim,
                                               c10::string_view rounding) {
  return RopeImpl(q, k, &q_weight, &k_weight, cos, sin, eps, unsqueeze_dim, rounding,
                  "flagos::rms_norm_rope");
}

// ----------------------------------------------------------------- SwiGLU --
at::Tensor Swiglu(const at::Tensor& gate_in, const at::Tensor& up_in, c10::string_view rounding) {
  const char* op = "flagos::swiglu";
  const int code = FloatCode(gate_in, op);
  SameDevice(gate_in, up_in, op);
  TORCH_CHECK(gate_in.sizes() == up_in.sizes() && gate_in.scalar_type() == up_in.scalar_type(),
              op, ": gate and up must match");
  at::Tensor g, u;
  const RowsView rg = Rows(gate_in, g), ru = Rows(up_in, u);
  at::Tensor out = at::empty(g.sizes(), g.options());
  GpuGuard guard(g);
  CheckB200(fl_b200_swiglu(g.data_ptr(), rg.ld, u.data_ptr(), ru.ld, out.data_ptr(), rg.cols,
                           rg.rows, rg.cols, code, Rounding(rounding), StreamOf(g)),
            op);
  return out;
}

std::tuple<at::Tensor, at::Tensor> SwigluResidual(const at::Tensor& gate, const at::Tensor& up,
                                                  const at::Tensor& x, const at::Tensor& y,
                                                  c10::string_view rounding) {
  const char* op = "flagos::swiglu_residual";
  const int code = FloatCode(gate, op);
  TORCH_CHECK(gate.sizes() == up.sizes() && x.sizes() == y.sizes() &&
                  gate.scalar_type() == up.scalar_type() && x.scalar_type() == gate.scalar_type() &&
                  y.scalar_type() == gate.scalar_type(),
              op, ": gate/up and x/y must match pairwise and share a dtype");
  TORCH_CHECK(gate.dim() >= 1 && x.dim() >= 1 && gate.numel() / std::max<int64_t>(gate.size(-1), 1) ==
                  x.numel() / std::max<int64_t>(x.size(-1), 1),
              op, ": gate and x must have the same number of rows");
  at::Tensor g = gate.contiguous(), u = up.contiguous(), xc = x.contiguous(), yc = y.contiguous();
  at::Tensor act = at::empty(g.sizes(), g.options()), h = at::empty(xc.sizes(), xc.options());
  const int64_t rows = g.size(-1) ? g.numel() / g.size(-1) : 0;
  GpuGuard guard(g);
  CheckB200(fl_b200_swiglu_residual(g.data_ptr(), u.data_ptr(), act.data_ptr(), g.size(-1),
                                    xc.data_ptr(), yc.data_ptr(), h.data_ptr(), xc.size(-1), rows,
                                    code, Rounding(rounding), StreamOf(g)),
            op);
  return {act, h};
}

// ---------------------------------------------------------- causal softmax --
at::Tensor CausalSoftmax(const at::Tensor& x_in, int64_t offset, std::optional<at::ScalarType> dtype) {
  const char* op = "flagos::causal_softmax";
  const int ci = FloatCode(x_in, op);
  const at::ScalarType ot = dtype.value_or(x_in.scalar_type());
  const int co = B200Dtype(ot);
  TORCH_CHECK(co == ci || co == FL_B200_F32, op, ": output dtype must be the input's or float32");
  TORCH_CHECK(x_in.dim() >= 2, op, ": x must be [..., q_len, k_len]");
  at::Tensor x;
  const RowsView r = Rows(x_in, x);
  at::Tensor out = at::empty(x.sizes(), x.options().dtype(ot));
  GpuGuard g(x);
  CheckB200(fl_b200_softmax_lastdim(x.data_ptr(), r.ld, out.data_ptr(), r.cols, r.rows, r.cols,
                                    ci, co, 1, x.size(-2), offset, StreamOf(x)),
            op);
  return out;
}

// ---------------------------------------------------- masked softmax --
// HF eager attention's `softmax(w * scaling + mask, dtype=float32)
// .to(query.dtype)` (modeling_qwen3.py eager_attention_forward) in one
// launch.  x is [B, H, Q, K] (or fewer leading dims); the mask has x's dtype
// and broadcasts to x (HF's is [B, 1, Q, K]).
at::Tensor MaskedSoftmax(const at::Tensor& x_in, const std::optional<at::Tensor>& mask_in,
                         double scale, std::optional<at::ScalarType> dtype,
                         c10::string_view rounding) {
  const char* op = "flagos::masked_softmax";
  const int ci = FloatCode(x_in, op);
  const at::ScalarType ot = dtype.value_or(x_in.scalar_type());
  const int co = B200Dtype(ot);
  TORCH_CHECK(co == ci || co == FL_B200_F32, op, ": output dtype must be the input's or float32");
  TORCH_CHECK(x_in.dim() >= 2 && x_in.dim() <= 4, op,
              ": x must be [Q, K], [H, Q, K] or [B, H, Q, K]");
  at::Tensor x4 = x_in;
  while (x4.dim() < 4) x4 = x4.unsqueeze(0);
  const int64_t H = x4.size(1), Q = x4.size(2), K = x4.size(3);
  at::Tensor x;
  const RowsView r = Rows(x4, x);
  at::Tensor mask;
  int64_t sb = 0, sh = 0, sq = 0;
  if (mask_in.has_value() && mask_in->defined()) {
    SameDevice(x_in, *mask_in, op);
    TORCH_CHECK(mask_in->scalar_type() == x_in.scalar_type(), op, ": mask must have x's dtype, got ",
                mask_in->scalar_type());
    mask = mask_in->expand(x4.sizes());
    if (K > 1 && mask.stride(3) != 1) mask = mask.contiguous();
    sb = mask.stride(0);
    sh = mask.stride(1);
    sq = mask.stride(2);
  }
  at::Tensor out = at::empty(x4.sizes(), x.options().dtype(ot));
  if (out.numel() == 0) return out.view(x_in.sizes());
  GpuGuard g(x);
  CheckB200(fl_b200_softmax_masked(x.data_ptr(), r.ld, mask.defined() ? mask.data_ptr() : nullptr,
                                   sb, sh, sq, out.data_ptr(), K, r.rows, K, H, Q, (float)scale,
                                   ci, co, Rounding(rounding), StreamOf(x)),
            op);
  return out.view(x_in.sizes());
}

// -------------------------------------------------------------- backward --
// The backward ops the autograd formulas of the fused ops call
// (torch_fl/autograd.py).  fp32 math, one rounding to the output dtype.
std::tuple<at::Tensor, at::Tensor> RmsNormBackward(const at::Tensor& dy_in,
                                                   const at::Tensor& x_in,
                                                   const at::Tensor& weight, double eps) {
  const char* op = "flagos::rms_norm_backward";
  const int code = FloatCode(x_in, op);
  SameDevice(x_in, dy_in, op);
  SameDevice(x_in, weight, op);
  TORCH_CHECK(dy_in.sizes() == x_in.sizes() && dy_in.scalar_type() == x_in.scalar_type(), op,
              ": dy and x must match");
  TORCH_CHECK(weight.scalar_type() == x_in.scalar_type() && weight.dim() == 1 &&
                  weight.numel() == x_in.size(-1),
              op, ": weight must be a [hidden] tensor of x's dtype");
  at::Tensor x, dy;
  const RowsView r = Rows(x_in, x), rd = Rows(dy_in, dy);
  at::Tensor w = weight.contiguous();
  at::Tensor dx = at::empty(x.sizes(), x.options());
  at::Tensor dw = at::empty({r.cols}, w.options());
  GpuGuard g(x);
  const size_t nws = fl_b200_rms_norm_bwd_workspace_size(r.rows, r.cols);
  at::Tensor ws = at::empty({(int64_t)std::max<size_t>(nws, 16)}, x.options().dtype(at::kByte));
  CheckB200(fl_b200_rms_norm_bwd(dy.data_ptr(), rd.ld, x.data_ptr(), r.ld, w.data_ptr(),
                                 dx.data_ptr(), r.cols, dw.data_ptr(), r.rows, r.cols, (float)eps,
                                 code, ws.data_ptr(), nws, StreamOf(x)),
            op);
  return {dx, dw};
}

std::tuple<at::Tensor, at::Tensor> SwigluBackward(const at::Tensor& dout, const at::Tensor& gate,
                                                  const at::Tensor& up) {
  const char* op = "flagos::swiglu_backward";
  const int code = FloatCode(gate, op);
  SameDevice(gate, up, op);
  SameDevice(gate, dout, op);
  TORCH_CHECK(gate.sizes() == up.sizes() && gate.sizes() == dout.sizes() &&
                  up.scalar_type() == gate.scalar_type() &&
                  dout.scalar_type() == gate.scalar_type(),
              op, ": dout, gate and up must match");
  at::Tensor d = dout.contiguous(), g = gate.contiguous(), u = up.contiguous();
  at::Tensor dg = at::empty(g.sizes(), g.options()), du = at::empty(u.sizes(), u.options());
  GpuGuard guard(g);
  CheckB200(fl_b200_swiglu_bwd(d.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(),
                               du.data_ptr(), g.numel(), code, StreamOf(g)),
            op);
  return {dg, du};
}

at::Tensor SoftmaxBackward(const at::Tensor& dy_in, const at::Tensor& y_in,
                           std::optional<at::ScalarType> dtype, double scale) {
  const char* op = "flagos::softmax_backward";
  const int ci = FloatCode(y_in, op);
  SameDevice(y_in, dy_in, op);
  TORCH_CHECK(dy_in.sizes() == y_in.sizes() && dy_in.scalar_type() == y_in.scalar_type(), op,
              ": dy and y must match");
  const at::ScalarType ot = dtype.value_or(y_in.scalar_type());
  const int co = B200Dtype(ot);
  TORCH_CHECK(co == ci || (ci == FL_B200_F32 && (co == FL_B200_BF16 || co == FL_B200_F16)), op,
              ": output dtype must be y's, or 16-bit with float32 y");
  at::Tensor y, dy;
  const RowsView r = Rows(y_in, y), rd = Rows(dy_in, dy);
  at::Tensor dx = at::empty(y.sizes(), y.options().dtype(ot));
  GpuGuard g(y);
  CheckB200(fl_b200_softmax_bwd_scaled(dy.data_ptr(), rd.ld, y.data_ptr(), r.ld, dx.data_ptr(),
                                       r.cols, r.rows, r.cols, (float)scale, ci, co, StreamOf(y)),
            op);
  return dx;
}

}  // namespace

TORCH_LIBRARY(flagos, m) {
  m.def("rms_norm(Tensor x, Tensor weight, float eps, str rounding='fused') -> Tensor");
  m.def("add_rms_norm(Tensor x, Tensor residual, Tensor weight, float eps, "
        "str rounding='fused') -> (Tensor, Tensor)");
  m.def("rope_qk(Tensor q, Tensor k, Tensor cos, Tensor sin, int unsqueeze_dim=1, "
        "str rounding='fused') -> (Tensor, Tensor)");
  m.def("rms_norm_rope(Tensor q, Tensor k, Tensor q_weight, Tensor k_weight, Tensor cos, "
        "Tensor sin, float eps, int unsqueeze_dim=1, str rounding='fused') -> (Tensor, Tensor)");
  m.def("swiglu(Tensor gate, Tensor up, str rounding='fused') -> Tensor");
  m.def("swiglu_residual(Tensor gate, Tensor up, Tensor x, Tensor y, str rounding='fused') "
        "-> (Tensor, Tensor)");
  m.def("causal_softmax(Tensor x, int offset=0, ScalarType? dtype=None) -> Tensor");
  m.def("rms_norm_backward(Tensor dy, Tensor x, Tensor weight, float eps) -> (Tensor, Tensor)");
  m.def("swiglu_backward(Tensor dout, Tensor gate, Tensor up) -> (Tensor, Tensor)");
  m.def("softmax_backward(Tensor dy, Tensor y, ScalarType? dtype=None, float scale=1.0) -> Tensor");
  m.def("masked_softmax(Tensor x, Tensor? mask=None, float scale=1.0, ScalarType? dtype=None, "
        "str rounding='fused') -> Tensor");
}

#define FLB_FUSED_IMPLS(m)                          \
  m.impl("rms_norm", RmsNorm);                      \
  m.impl("add_rms_norm", AddRmsNorm);               \
  m.impl("rope_qk", RopeQk);                        \
  m.impl("rms_norm_rope", RmsNormRope);             \
  m.impl("swiglu", Swiglu);                         \
  m.impl("swiglu_residual", SwigluResidual);        \
  m.impl("causal_softmax", CausalSoftmax);          \
  m.impl("rms_norm_backward", RmsNormBackward);     \
  m.impl("swiglu_backward", SwigluBackward);        \
  m.impl("softmax_backward", SoftmaxBackward);      \
  m.impl("masked_softmax", MaskedSoftmax);

TORCH_LIBRARY_IMPL(flagos, PrivateUse1, m) { FLB_FUSED_IMPLS(m) }
TORCH_LIBRARY_IMPL(flagos, CUDA, m) { FLB_FUSED_IMPLS(m) }

}  // namespace flb200::aten
