// The remaining ops of the HF formulas on the b200 route: silu, rsqrt, neg,
// cos, sin, pow(tensor, scalar), and cat.
//
// Reference behaviour (its cuda route, csrc/aten/backends/cuda/): each op is
// one TensorIterator pass computing in the op's own arithmetic --
//   silu.cu:15-35   x / (1 + exp(-x)) in fp32 opmath, rounded to the dtype
//   rsqrt.cu:14-32  ::rsqrt(a) (fp32 rsqrtf for 16-bit dtypes), rounded
//   neg.cu:14-32    -a (every dtype)
//   cos.cu, sin.cu  ::cos / ::sin in fp32 for 16-bit dtypes, rounded
//   pow.cu:15-46    exponent first converted to the tensor's dtype; 2 -> b*b,
//                   3 -> b*b*b, both in the dtype (so a 16-bit cube rounds
//                   after the square and after the product), else ::pow
//   cat.cc:13-39    PyTorch's structured cat_out_cuda
// HF's RMSNorm and RoPE reach these when the fused hooks are off
// (`hidden.pow(2)`, `torch.rsqrt`, `rotate_half` = cat(-x2, x1)).
//
// Layout: the input is a set of rows of `cols` contiguous elements whose
// starts follow up to 4 outer dims (sizes, element strides): HF's
// q[..., D/2:] of a transposed q is such a set, with no uniform row stride.
// The output is dense.  Contiguous rows take a flat loop; others give each
// CTA whole rows, so the outer index is decomposed once per row, never per
// element.  16-byte packs when every row start is 16-byte aligned, else one
// element at a time.
#include "common.cuh"

#include <algorithm>

namespace flb200 {
namespace {

constexpr int kBlock = 256;

// Row r of a set of rows -> element offset of its first element: r is split
// over the outer sizes (last fastest) and the parts multiplied by the
// strides.  `nd` <= 4.
struct RowMap {
  int64_t size[4], stride[4];
  int nd;
  __device__ __forceinline__ int64_t offset(int64_t r) const {
    int64_t off = 0;
#pragma unroll
    for (int d = 3; d >= 0; --d) {
      if (d >= nd) continue;
      const int64_t q = r / size[d];
      off += (r - q * size[d]) * stride[d];
      r = q;
    }
    return off;
  }
};

// Builds a RowMap from the caller's outer dims, dropping size-1 dims and
// merging neighbours that step evenly; false when more than 4 remain or a
// size is negative.  *rows = the product of the sizes; *dense = the rows are
// back to back (row r at r * cols).
bool make_rowmap(const int64_t* sizes, const int64_t* strides, int ndim, int64_t cols,
                 RowMap* m, int64_t* rows, bool* dense) {
  int64_t sz[8], st[8];
  int n = 0;
  *rows = 1;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] < 0) return false;
    *rows *= sizes[d];
    if (sizes[d] == 1) continue;
    if (n > 0 && st[n - 1] == strides[d] * sizes[d]) {  // merge with the outer one
      sz[n - 1] *= sizes[d];
      st[n - 1] = strides[d];
      continue;
    }
    if (n == 8) return false;
    sz[n] = sizes[d];
    st[n] = strides[d];
    ++n;
  }
  if (n > 4) return false;
  m->nd = n;
  for (int d = 0; d < 4; ++d) {
    m->size[d] = d < n ? sz[d] : 1;
    m->stride[d] = d < n ? st[d] : 0;
  }
  *dense = n == 0 || (n == 1 && st[0] == cols);
  return true;
}

template <typename T, int OP>
__device__ __forceinline__ float unary_op(float x, float p) {
  if constexpr (OP == FL_B200_UNARY_SILU) {
    return x / (1.0f + expf(-x));
  } else if constexpr (OP == FL_B200_UNARY_RSQRT) {
    return rsqrtf(x);
  } else if constexpr (OP == FL_B200_UNARY_NEG) {
    return -x;
  } else if constexpr (OP == FL_B200_UNARY_COS) {
    return cosf(x);
  } else if constexpr (OP == FL_B200_UNARY_SIN) {
    return sinf(x);
  } else if constexpr (OP == FL_B200_UNARY_SQUARE) {
    return x * x;
  } else if constexpr (OP == FL_B200_UNARY_CUBE) {
    return round_to<T>(x * x) * x;  // b*b rounds to T before the second product
  } else {
    return powf(x, p);
  }
}

template <typename T, int OP>
__device__ __forceinline__ uint4 unary_pack(const uint4& v, float p) {
  constexpr int VW = Elem<T>::kVec;
  float f[VW];
  unpack<T>(v, f);
#pragma unroll
  for (int e = 0; e < VW; ++e) f[e] = unary_op<T, OP>(f[e], p);
  return pack<T>(f);
}

// Dense: 4 packs per thread per step.
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
unary_dense_kernel(const T* __restrict__ x, T* __restrict__ o, int64_t npk, float p) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  const int64_t nth = (int64_t)gridDim.x * kBlock;
  int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  for (; i + 3 * nth < npk; i += 4 * nth) {
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = ld_stream(x + (i + k * nth) * VW);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      st_stream(o + (i + k * nth) * VW, unary_pack<T, OP>(v[k], p));
  }
  for (; i < npk; i += nth)
    st_stream(o + i * VW, unary_pack<T, OP>(ld_stream(x + i * VW), p));
}

// Dense, one element at a time (sizes or addresses that 16-byte packs do
// not fit).
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
unary_dense_scalar_kernel(const T* __restrict__ x, T* __restrict__ o, int64_t n, float p) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock)
    o[i] = Elem<T>::from_f(unary_op<T, OP>(Elem<T>::to_f(x[i]), p));
}

// Rows placed by a RowMap: TPR = min(units per row, 256) threads per row,
// 256 / TPR rows per CTA step.  PACK: 16-byte packs, else single elements.
template <typename T, int OP, bool PACK>
__global__ void __launch_bounds__(kBlock)
unary_rows_kernel(const T* __restrict__ x, RowMap rm, T* __restrict__ o, int64_t rows,
                  int units, int tpr, float p) {
  pdl_prologue();
  constexpr int U = PACK ? Elem<T>::kVec : 1;
  const int rpc = kBlock / tpr;
  const int slot = threadIdx.x / tpr;
  const int lane = threadIdx.x - slot * tpr;
  if (slot >= rpc) return;
  for (int64_t r = (int64_t)blockIdx.x * rpc + slot; r < rows; r += (int64_t)gridDim.x * rpc) {
    const T* xr = x + rm.offset(r);
    T* orow = o + r * (int64_t)units * U;
    for (int c = lane; c < units; c += tpr) {
      if constexpr (PACK) {
        const uint4 v = ld_stream(xr + (int64_t)c * U);
        st_stream(orow + (int64_t)c * U, unary_pack<T, OP>(v, p));
      } else {
        orow[c] = Elem<T>::from_f(unary_op<T, OP>(Elem<T>::to_f(xr[c]), p));
      }
    }
  }
}

// Integer negation (two's complement, the lowest value maps to itself).
template <typename I>
__global__ void __launch_bounds__(kBlock)
neg_int_rows_kernel(const I* __restrict__ x, RowMap rm, I* __restrict__ o, int64_t rows,
                    int cols, int tpr) {
  pdl_prologue();
  using UI = typename std::make_unsigned<I>::type;
  const int rpc = kBlock / tpr;
  const int slot = threadIdx.x / tpr;
  const int lane = threadIdx.x - slot * tpr;
  if (slot >= rpc) return;
  for (int64_t r = (int64_t)blockIdx.x * rpc + slot; r < rows; r += (int64_t)gridDim.x * rpc) {
    const I* xr = x + rm.offset(r);
    for (int c = lane; c < cols; c += tpr) o[r * cols + c] = (I)(UI(0) - (UI)xr[c]);
  }
}

int rows_grid(int64_t rows, int tpr) {
  return full_grid(ceil_div(rows, (int64_t)(kBlock / tpr)));
}

// Whether every row start of `m` (and x itself) is 16-byte aligned.
template <typename T>
bool rows_aligned16(const T* x, const RowMap& m) {
  if (!aligned16(x)) return false;
  for (int d = 0; d < m.nd; ++d)
    if ((m.stride[d] * (int64_t)sizeof(T)) % 16 != 0) return false;
  return true;
}

template <typename T, int OP>
int launch_unary(const T* x, const RowMap& rm, bool dense, T* o, int64_t rows, int64_t cols,
                 float p, cudaStream_t stream) {
  constexpr int VW = Elem<T>::kVec;
  const bool packs = cols % VW == 0 && rows_aligned16(x, rm) && aligned16(o);
  if (packs && dense) {
    const int64_t npk = rows * cols / VW;
    launch_k(unary_dense_kernel<T, OP>, full_grid(ceil_div(npk, (int64_t)kBlock * 4)), kBlock,
             0, stream, x, o, npk, p);
    return launch_status();
  }
  if (dense) {
    const int64_t n = rows * cols;
    launch_k(unary_dense_scalar_kernel<T, OP>, full_grid(ceil_div(n, (int64_t)kBlock * 4)),
             kBlock, 0, stream, x, o, n, p);
    return launch_status();
  }
  const int64_t units = packs ? cols / VW : cols;
  if (units >= (int64_t(1) << 31)) return FL_B200_ERR_INVALID_ARGUMENT;
  const int tpr = (int)std::min<int64_t>(units, kBlock);
  if (packs) {
    launch_k(unary_rows_kernel<T, OP, true>, rows_grid(rows, tpr), kBlock, 0, stream, x, rm,
             o, rows, (int)units, tpr, p);
  } else {
    launch_k(unary_rows_kernel<T, OP, false>, rows_grid(rows, tpr), kBlock, 0, stream, x, rm,
             o, rows, (int)units, tpr, p);
  }
  return launch_status();
}

template <typename T>
int unary_float(int op, const void* x, const RowMap& rm, bool dense, void* o, int64_t rows,
                int64_t cols, float p, cudaStream_t s) {
  auto xp = static_cast<const T*>(x);
  auto op_ = static_cast<T*>(o);
  switch (op) {
#define FLB_UNARY_CASE(OPC) \
    case OPC: return launch_unary<T, OPC>(xp, rm, dense, op_, rows, cols, p, s);
    FLB_UNARY_CASE(FL_B200_UNARY_SILU)
    FLB_UNARY_CASE(FL_B200_UNARY_RSQRT)
    FLB_UNARY_CASE(FL_B200_UNARY_NEG)
    FLB_UNARY_CASE(FL_B200_UNARY_COS)
    FLB_UNARY_CASE(FL_B200_UNARY_SIN)
    FLB_UNARY_CASE(FL_B200_UNARY_SQUARE)
    FLB_UNARY_CASE(FL_B200_UNARY_CUBE)
    FLB_UNARY_CASE(FL_B200_UNARY_POW)
#undef FLB_UNARY_CASE
    default: return FL_B200_ERR_INVALID_ARGUMENT;
  }
}

// ------------------------------------------------------------------- cat --
// out[r, off_k + j] = src_k[rowmap_k(r) + j] for j < width_k, in units of U
// bytes; blockIdx.y picks the input.
constexpr int kCatMax = 4;
struct CatArgs {
  const void* src[kCatMax];
  RowMap map[kCatMax];
  int64_t width[kCatMax], off[kCatMax];
  void* out;
  int64_t rows, out_ld;
};

template <typename U>
__global__ void __launch_bounds__(kBlock) cat_rows_kernel(CatArgs a) {
  pdl_prologue();
  const int k = blockIdx.y;
  const int64_t w = a.width[k];
  if (w == 0) return;
  const int tpr = w < kBlock ? (int)w : kBlock;
  const int rpc = kBlock / tpr;
  const int slot = threadIdx.x / tpr;
  const int lane = threadIdx.x - slot * tpr;
  if (slot >= rpc) return;
  const U* src = static_cast<const U*>(a.src[k]);
  U* out = static_cast<U*>(a.out) + a.off[k];
  for (int64_t r = (int64_t)blockIdx.x * rpc + slot; r < a.rows;
       r += (int64_t)gridDim.x * rpc) {
    const U* sr = src + a.map[k].offset(r);
    U* orow = out + r * a.out_ld;
    for (int64_t c = lane; c < w; c += tpr) orow[c] = sr[c];
  }
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_unary(const void* x, const int64_t* row_sizes,
                              const int64_t* row_strides, int row_ndim, int64_t cols, void* out,
                              int op, double p, int dtype, fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(row_ndim >= 0 && row_ndim <= 8 && cols >= 0);
  FLB_CHECK_ARG(row_ndim == 0 || (row_sizes && row_strides));
  FLB_CHECK_ARG(op >= FL_B200_UNARY_SILU && op <= FL_B200_UNARY_POW);
  RowMap rm;
  int64_t rows = 1;
  bool dense = true;
  FLB_CHECK_ARG(make_rowmap(row_sizes, row_strides, row_ndim, cols, &rm, &rows, &dense));
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && out);
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == FL_B200_I32 || dtype == FL_B200_I64) {
    if (op != FL_B200_UNARY_NEG) return FL_B200_ERR_UNSUPPORTED_DTYPE;
    if (cols >= (int64_t(1) << 31)) return FL_B200_ERR_INVALID_ARGUMENT;
    const int tpr = (int)std::min<int64_t>(cols, kBlock);
    if (dtype == FL_B200_I32) {
      launch_k(neg_int_rows_kernel<int32_t>, rows_grid(rows, tpr), kBlock, 0, s,
               static_cast<const int32_t*>(x), rm, static_cast<int32_t*>(out), rows, (int)cols,
               tpr);
    } else {
      launch_k(neg_int_rows_kernel<int64_t>, rows_grid(rows, tpr), kBlock, 0, s,
               static_cast<const int64_t*>(x), rm, static_cast<int64_t*>(out), rows, (int)cols,
               tpr);
    }
    return launch_status();
  }
  const float pf = (float)p;
  switch (dtype) {
    case FL_B200_F32: return unary_float<float>(op, x, rm, dense, out, rows, cols, pf, s);
    case FL_B200_BF16:
      return unary_float<__nv_bfloat16>(op, x, rm, dense, out, rows, cols, pf, s);
    case FL_B200_F16: return unary_float<__half>(op, x, rm, dense, out, rows, cols, pf, s);
    default: return FL_B200_ERR_UNSUPPORTED_DTYPE;
  }
}

FL_B200_API int fl_b200_cat(const void* const* srcs, const int64_t* src_row_strides,
                            const int64_t* widths, int n_inputs, const int64_t* row_sizes,
                            int row_ndim, void* out, int elem_size, fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n_inputs >= 0 && row_ndim >= 0 && row_ndim <= 8);
  FLB_CHECK_ARG(elem_size == 1 || elem_size == 2 || elem_size == 4 || elem_size == 8);
  if (n_inputs == 0) return FL_B200_OK;
  FLB_CHECK_ARG(srcs && widths && out && (row_ndim == 0 || (row_sizes && src_row_strides)));
  int64_t total = 0, rows = 1;
  for (int d = 0; d < row_ndim; ++d) {
    FLB_CHECK_ARG(row_sizes[d] >= 0);
    rows *= row_sizes[d];
  }
  for (int k = 0; k < n_inputs; ++k) {
    FLB_CHECK_ARG(widths[k] >= 0 && (widths[k] == 0 || srcs[k]));
    total += widths[k];
  }
  if (total == 0 || rows == 0) return FL_B200_OK;
  // The widest unit (16, 8, 4, 2 or 1 bytes) that divides every width,
  // offset and outer stride in bytes and every base address.
  auto fits = [&](int u) {
    if ((reinterpret_cast<uintptr_t>(out) % u) != 0 || (total * elem_size) % u != 0) return false;
    int64_t off = 0;
    for (int k = 0; k < n_inputs; ++k) {
      if (widths[k] == 0) continue;
      if ((widths[k] * elem_size) % u || (off * elem_size) % u ||
          (reinterpret_cast<uintptr_t>(srcs[k]) % u))
        return false;
      for (int d = 0; d < row_ndim; ++d)
        if (row_sizes[d] > 1 && (src_row_strides[k * row_ndim + d] * elem_size) % u) return false;
      off += widths[k];
    }
    return true;
  };
  int unit = 16;
  while (unit > elem_size && !fits(unit)) unit /= 2;
  if (unit < elem_size) unit = elem_size;
  const int per = unit / elem_size;  // elements per unit
  auto s = static_cast<cudaStream_t>(stream);
  int64_t off = 0;
  for (int k0 = 0; k0 < n_inputs; k0 += kCatMax) {
    CatArgs a{};
    const int n = std::min(kCatMax, n_inputs - k0);
    int64_t wmax = 0;
    for (int j = 0; j < n; ++j) {
      const int k = k0 + j;
      int64_t st[8], rr = 1;
      bool dense = true;
      for (int d = 0; d < row_ndim; ++d) st[d] = src_row_strides[k * row_ndim + d] / per;
      // the input's outer strides in units (widths in units are widths / per)
      FLB_CHECK_ARG(make_rowmap(row_sizes, st, row_ndim, widths[k] / per, &a.map[j], &rr,
                                &dense));
      a.src[j] = srcs[k];
      a.width[j] = widths[k] / per;
      a.off[j] = off / per;
      off += widths[k];
      wmax = std::max(wmax, a.width[j]);
    }
    a.out = out;
    a.rows = rows;
    a.out_ld = total / per;
    const int tpr = (int)std::min<int64_t>(std::max<int64_t>(wmax, 1), kBlock);
    const dim3 grid((unsigned)full_grid(ceil_div(rows, (int64_t)(kBlock / tpr))), (unsigned)n);
    switch (unit) {
      case 16: launch_k(cat_rows_kernel<uint4>, grid, kBlock, 0, s, a); break;
      case 8: launch_k(cat_rows_kernel<uint2>, grid, kBlock, 0, s, a); break;
      case 4: launch_k(cat_rows_kernel<uint32_t>, grid, kBlock, 0, s, a); break;
      case 2: launch_k(cat_rows_kernel<uint16_t>, grid, kBlock, 0, s, a); break;
      default: launch_k(cat_rows_kernel<uint8_t>, grid, kBlock, 0, s, a); break;
    }
    const int st = launch_status();
    if (st != FL_B200_OK) return st;
  }
  return FL_B200_OK;
}

}  // extern "C"
