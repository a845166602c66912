// Broadcast add / mul, tensor-scalar ops and dense dtype casts.
//
// Reference behaviour: add.Tensor `self + alpha*other` (csrc/aten/backends/
// cuda/add.cu:48-84) and mul.Tensor (mul.cu:28-52), both TensorIterator
// kernels with fp32 opmath for 16-bit floats; wrapped CPU scalars stay in
// opmath (add.cu:67-76); flagos->flagos dtype casts (copy_ops.cc:225-240).
//
// Paths, fastest first: dense same-shape operands (32-byte, else 16-byte
// packs); one operand a row vector broadcast over the rows of the other
// (the RMSNorm weight multiply, bias adds) or one value per row ([T, 1]
// scales); anything else through N-d index arithmetic.
#include "common.cuh"

#include <algorithm>

namespace flb200 {
namespace {

constexpr int kBlock = 256;
constexpr int kUnroll = 4;
constexpr int kMaxDims = 8;

enum BinOp { kAdd = 0, kMul = 1 };

template <int OP>
__device__ __forceinline__ float apply_f(float a, float b, float alpha) {
  if (OP == kAdd) return fmaf(alpha, b, a);
  return a * b;
}
template <int OP, typename I>
__device__ __forceinline__ I apply_i(I a, I b, I alpha) {
  // Unsigned arithmetic gives the two's-complement wrap of torch's integer ops.
  using U = typename std::make_unsigned<I>::type;
  if (OP == kAdd) return (I)((U)a + (U)alpha * (U)b);
  return (I)((U)a * (U)b);
}

// ---- dense same-shape, 16-byte packs ---------------------------------------
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
binary_dense_kernel(const T* a, const T* b, T* o, int64_t npk, float alpha) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  const int64_t nth = (int64_t)gridDim.x * kBlock;
  int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  for (; i + (kUnroll - 1) * nth < npk; i += kUnroll * nth) {
    uint4 av[kUnroll], bv[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      av[k] = ld_stream(a + (i + k * nth) * VW);
      bv[k] = ld_stream(b + (i + k * nth) * VW);
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      float x[VW], y[VW];
      unpack<T>(av[k], x);
      unpack<T>(bv[k], y);
#pragma unroll
      for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], y[e], alpha);
      st_stream(o + (i + k * nth) * VW, pack<T>(x));
    }
  }
  for (; i < npk; i += nth) {
    float x[VW], y[VW];
    unpack<T>(ld_stream(a + i * VW), x);
    unpack<T>(ld_stream(b + i * VW), y);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], y[e], alpha);
    st_stream(o + i * VW, pack<T>(x));
  }
}

// ---- dense same-shape, 32-byte packs ---------------------------------------
// Two 32-byte packs per thread (packs i and i + 512 of the CTA's 1024),
// 512-thread CTAs, one CTA per 1024 packs: for 32-byte aligned operands.
// Measured on B200, bf16 [131072, 4096] + [131072, 4096]: 7.0 TB/s against
// 6.3 with one 16-byte pack per thread (PyTorch's own add: 7.1).
constexpr int kBlock32 = 512;
constexpr int kPacks32 = 2;

template <typename T, int OP>
__global__ void __launch_bounds__(kBlock32)
binary_dense32_kernel(const T* a, const T* b, T* o, int64_t npk32, float alpha) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  const int64_t i0 = (int64_t)blockIdx.x * (kBlock32 * kPacks32) + threadIdx.x;
  Pack32 av[kPacks32], bv[kPacks32];
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i < npk32) {
      av[k] = ld_stream32(a + i * 2 * VW);
      bv[k] = ld_stream32(b + i * 2 * VW);
    }
  }
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i >= npk32) continue;
    float x[VW], y[VW];
    Pack32 r;
    unpack<T>(av[k].lo, x);
    unpack<T>(bv[k].lo, y);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], y[e], alpha);
    r.lo = pack<T>(x);
    unpack<T>(av[k].hi, x);
    unpack<T>(bv[k].hi, y);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], y[e], alpha);
    r.hi = pack<T>(x);
    st_stream32(o + i * 2 * VW, r);
  }
}

// ---- one operand broadcast over the rows of the other -----------------------
// full is a dense [rows, cols] operand; the other is a row vector v[c]
// (MODE kRowVec) or one value per row s[r] at s + r * s_stride (MODE
// kColVec).  A CTA takes kTileRows rows; each thread walks its column packs
// (c = threadIdx.x, + kBlock, ...), loads the vector pack once per column or
// the rows' values once (the same addresses for the whole CTA), and streams
// the rows' packs with kTileRows loads in flight.  VEC_FIRST: the broadcast
// operand is `a` (v op full), else `b` (full op v): the order matters for
// add's alpha.  Measured on B200, bf16 [131072, 4096] times a [4096] row
// vector: 6.6 TB/s (5.7 with a per-pack index modulo), times a [131072, 1]
// column: 6.6 TB/s (0.7 through the N-d path; PyTorch: 1.8 for both).
constexpr int kTileRows = 8;
enum { kRowVec = 0, kColVec = 1 };

template <typename T, int OP, int MODE, bool VEC_FIRST>
__global__ void __launch_bounds__(kBlock)
binary_bcast_rows_kernel(const T* full, const T* vec, int64_t s_stride, T* o, int64_t rows,
                         int64_t cpk, float alpha) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  const int64_t r0 = (int64_t)blockIdx.x * kTileRows;
  float sv[kTileRows];
  if constexpr (MODE == kColVec) {
#pragma unroll
    for (int k = 0; k < kTileRows; ++k)
      sv[k] = r0 + k < rows ? Elem<T>::to_f(vec[(r0 + k) * s_stride]) : 0.f;
  }
  for (int64_t c = threadIdx.x; c < cpk; c += kBlock) {
    float v[VW];
    if constexpr (MODE == kRowVec) unpack<T>(ld_cached(vec + c * VW), v);
    uint4 fv[kTileRows];
#pragma unroll
    for (int k = 0; k < kTileRows; ++k)
      fv[k] = r0 + k < rows ? ld_stream(full + ((r0 + k) * cpk + c) * VW) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < kTileRows; ++k) {
      if (r0 + k >= rows) continue;
      float x[VW];
      unpack<T>(fv[k], x);
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const float w = MODE == kRowVec ? v[e] : sv[k];
        x[e] = VEC_FIRST ? apply_f<OP>(w, x[e], alpha) : apply_f<OP>(x[e], w, alpha);
      }
      st_stream(o + ((r0 + k) * cpk + c) * VW, pack<T>(x));
    }
  }
}

// ---- general N-d broadcast --------------------------------------------------
struct NdArgs {
  int64_t sizes[kMaxDims];
  int64_t sa[kMaxDims];
  int64_t sb[kMaxDims];
  int ndim;
};

__device__ __forceinline__ void nd_offsets(const NdArgs& g, int64_t i, int64_t& oa,
                                           int64_t& ob) {
  oa = 0;
  ob = 0;
#pragma unroll
  for (int d = kMaxDims - 1; d >= 0; --d) {
    if (d < g.ndim) {
      const int64_t c = i % g.sizes[d];
      i /= g.sizes[d];
      oa += c * g.sa[d];
      ob += c * g.sb[d];
    }
  }
}

template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
binary_nd_float_kernel(const T* a, const T* b, T* o, int64_t n, NdArgs g, float alpha) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock) {
    int64_t oa, ob;
    nd_offsets(g, i, oa, ob);
    o[i] = Elem<T>::from_f(apply_f<OP>(Elem<T>::to_f(a[oa]), Elem<T>::to_f(b[ob]), alpha));
  }
}

template <typename I, int OP>
__global__ void __launch_bounds__(kBlock)
binary_nd_int_kernel(const I* a, const I* b, I* o, int64_t n, NdArgs g, I alpha) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock) {
    int64_t oa, ob;
    nd_offsets(g, i, oa, ob);
    o[i] = apply_i<OP, I>(a[oa], b[ob], alpha);
  }
}

// ---- tensor op scalar -------------------------------------------------------
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
scalar_float_kernel(const T* a, T* o, int64_t n, float s, float alpha) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock)
    o[i] = Elem<T>::from_f(apply_f<OP>(Elem<T>::to_f(a[i]), s, alpha));
}
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
scalar_float_vec_kernel(const T* a, T* o, int64_t npk, float s, float alpha) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < npk;
       i += (int64_t)gridDim.x * kBlock) {
    float x[VW];
    unpack<T>(ld_stream(a + i * VW), x);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], s, alpha);
    st_stream(o + i * VW, pack<T>(x));
  }
}
// Two 32-byte packs per thread, 512-thread CTAs (as binary_dense32_kernel),
// for 32-byte aligned tensors.
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock32)
scalar_float_vec32_kernel(const T* a, T* o, int64_t npk32, float s, float alpha) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  const int64_t i0 = (int64_t)blockIdx.x * (kBlock32 * kPacks32) + threadIdx.x;
  Pack32 av[kPacks32];
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i < npk32) av[k] = ld_stream32(a + i * 2 * VW);
  }
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i >= npk32) continue;
    float x[VW];
    Pack32 r;
    unpack<T>(av[k].lo, x);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], s, alpha);
    r.lo = pack<T>(x);
    unpack<T>(av[k].hi, x);
#pragma unroll
    for (int e = 0; e < VW; ++e) x[e] = apply_f<OP>(x[e], s, alpha);
    r.hi = pack<T>(x);
    st_stream32(o + i * 2 * VW, r);
  }
}
template <typename I, int OP>
__global__ void __launch_bounds__(kBlock)
scalar_int_kernel(const I* a, I* o, int64_t n, I s, I alpha) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock)
    o[i] = apply_i<OP, I>(a[i], s, alpha);
}

// ---- casts ------------------------------------------------------------------
template <typename S>
struct Load;
template <>
struct Load<float> {
  __device__ static float f(float v) { return v; }
};
template <>
struct Load<__nv_bfloat16> {
  __device__ static float f(__nv_bfloat16 v) { return __bfloat162float(v); }
};
template <>
struct Load<__half> {
  __device__ static float f(__half v) { return __half2float(v); }
};

template <typename S, typename D>
__device__ __forceinline__ D convert(S v) {
  constexpr bool s_int = std::is_integral<S>::value;
  constexpr bool d_int = std::is_integral<D>::value;
  if constexpr (s_int && d_int) {
    return (D)v;
  } else if constexpr (s_int) {  // int -> float: via fp32 (torch's cast path)
    if constexpr (std::is_same<D, float>::value) return (float)v;
    else return Elem<D>::from_f((float)v);
  } else if constexpr (d_int) {  // float -> int: truncate
    return (D)Load<S>::f(v);
  } else {
    if constexpr (std::is_same<D, float>::value) return Load<S>::f(v);
    else return Elem<D>::from_f(Load<S>::f(v));
  }
}

template <typename S, typename D>
__global__ void __launch_bounds__(kBlock) cast_kernel(const S* src, D* dst, int64_t n) {
  pdl_prologue();
  const int64_t nth = (int64_t)gridDim.x * kBlock;
  int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  // 4 independent elements per iteration for memory-level parallelism.
  for (; i + 3 * nth < n; i += 4 * nth) {
    S v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = src[i + k * nth];
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[i + k * nth] = convert<S, D>(v[k]);
  }
  for (; i < n; i += nth) dst[i] = convert<S, D>(src[i]);
}



// 8 elements per thread per step through 16-byte accesses (both sides
// aligned and n % 8 == 0).
template <typename S, typename D>
__global__ void __launch_bounds__(kBlock)
cast_vec8_kernel(const S* src, D* dst, int64_t n8) {
  pdl_prologue();
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * kBlock) {
    union {
      uint4 u[sizeof(S) * 8 / 16];
      S v[8];
    } in;
    union {
      uint4 u[sizeof(D) * 8 / 16];
      D v[8];
    } out;
    const uint4* sp = reinterpret_cast<const uint4*>(src + i * 8);
#pragma unroll
    for (int k = 0; k < (int)(sizeof(S) * 8 / 16); ++k) in.u[k] = ld_stream(sp + k);
#pragma unroll
    for (int e = 0; e < 8; ++e) out.v[e] = convert<S, D>(in.v[e]);
    uint4* dp = reinterpret_cast<uint4*>(dst + i * 8);
#pragma unroll
    for (int k = 0; k < (int)(sizeof(D) * 8 / 16); ++k) st_stream(dp + k, out.u[k]);
  }
}

template <typename K>
int grid_for(K, int64_t work, const DeviceInfo&, int = 1) {
  return full_grid(ceil_div(work, kBlock));  // one unit of work per thread
}

template <typename F>
int dispatch_any(int dtype, F&& f) {
  switch (dtype) {
    case FL_B200_F32: return f(float{});
    case FL_B200_BF16: return f(__nv_bfloat16{});
    case FL_B200_F16: return f(__half{});
    case FL_B200_I32: return f(int32_t{});
    case FL_B200_I64: return f(int64_t{});
    default: return FL_B200_ERR_UNSUPPORTED_DTYPE;
  }
}

bool dense_strides(const int64_t* sizes, const int64_t* st, int ndim) {
  int64_t expect = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (sizes[d] != 1 && st[d] != expect) return false;
    expect *= sizes[d];
  }
  return true;
}

// True if `st` addresses a row vector over the last dim: stride 1 on the
// last dim (or size 1) and 0 on every other dim of size > 1.
bool rowvec_strides(const int64_t* sizes, const int64_t* st, int ndim) {
  if (ndim < 1) return false;
  if (sizes[ndim - 1] != 1 && st[ndim - 1] != 1) return false;
  for (int d = 0; d < ndim - 1; ++d)
    if (sizes[d] != 1 && st[d] != 0) return false;
  return true;
}

// True if `st` addresses one value per row (stride 0 on the last dim) whose
// leading dims collapse to a single row stride, returned in *row_stride:
// e.g. a [T, 1] or [B, S, 1] tensor broadcast over the last dim.
bool colvec_strides(const int64_t* sizes, const int64_t* st, int ndim, int64_t* row_stride) {
  if (ndim < 2) return false;
  if (sizes[ndim - 1] != 1 && st[ndim - 1] != 0) return false;
  int64_t expect = -1;
  for (int d = ndim - 2; d >= 0; --d) {
    if (sizes[d] == 1) continue;
    if (expect < 0) {
      expect = st[d];
      *row_stride = st[d];
    } else if (st[d] != expect) {
      return false;
    }
    expect *= sizes[d];
  }
  if (expect < 0) *row_stride = 0;  // a single row
  return true;
}

template <int OP>
int binary_entry(const void* a, const int64_t* sa, const void* b, const int64_t* sb,
                 void* out, const int64_t* sizes, int ndim, double alpha, int dtype,
                 cudaStream_t stream) {
  FLB_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims);
  FLB_CHECK_ARG(ndim == 0 || (sizes && sa && sb));
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) {
    FLB_CHECK_ARG(sizes[d] >= 0);
    n *= sizes[d];
  }
  if (n == 0) return FL_B200_OK;
  FLB_CHECK_ARG(a && b && out);
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  static const int64_t kZero[kMaxDims] = {0};
  const int64_t* sz = ndim ? sizes : kZero;
  const int64_t* sa_ = ndim ? sa : kZero;
  const int64_t* sb_ = ndim ? sb : kZero;
  NdArgs g{};
  g.ndim = ndim;
  for (int d = 0; d < ndim; ++d) {
    g.sizes[d] = sz[d];
    g.sa[d] = sa_[d];
    g.sb[d] = sb_[d];
  }
  return dispatch_any(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const T* ap = static_cast<const T*>(a);
    const T* bp = static_cast<const T*>(b);
    T* op = static_cast<T*>(out);
    if constexpr (std::is_integral<T>::value) {
      auto kern = binary_nd_int_kernel<T, OP>;
      launch_k(kern, grid_for(kern, n, dev, 4), kBlock, 0, stream, ap, bp, op, n, g,
               (T)(int64_t)alpha);
      return launch_status();
    } else {
      constexpr int VW = Elem<T>::kVec;
      const float al = (float)alpha;
      const bool all_aligned = aligned16(ap) && aligned16(bp) && aligned16(op);
      const bool a_dense = dense_strides(sz, sa_, ndim);
      const bool b_dense = dense_strides(sz, sb_, ndim);
      if (a_dense && b_dense && n % (2 * VW) == 0 && aligned32(ap) && aligned32(bp) &&
          aligned32(op)) {
        const int64_t npk32 = n / (2 * VW);
        launch_k((binary_dense32_kernel<T, OP>),
                 full_grid(ceil_div(npk32, (int64_t)kBlock32 * kPacks32)), kBlock32, 0,
                 stream, ap, bp, op, npk32, al);
        return launch_status();
      }
      if (a_dense && b_dense && n % VW == 0 && all_aligned) {
        auto kern = binary_dense_kernel<T, OP>;
        const int64_t npk = n / VW;
        const int grid = full_grid(ceil_div(npk, kBlock));
        launch_k(kern, grid, kBlock, 0, stream, ap, bp, op, npk, al);
        return launch_status();
      }
      const int64_t cols = ndim ? sz[ndim - 1] : 1;
      if (ndim >= 1 && cols % VW == 0 && aligned16(op)) {
        const int64_t rows = n / cols, cpk = cols / VW;
        const int grid = full_grid(ceil_div(rows, kTileRows));
        int64_t rs = 0;
        // full op v[c] / v[c] op full (v 16-byte aligned)
        if (a_dense && aligned16(ap) && aligned16(bp) && rowvec_strides(sz, sb_, ndim)) {
          launch_k((binary_bcast_rows_kernel<T, OP, kRowVec, false>), grid, kBlock, 0, stream,
                   ap, bp, 0, op, rows, cpk, al);
          return launch_status();
        }
        if (b_dense && aligned16(ap) && aligned16(bp) && rowvec_strides(sz, sa_, ndim)) {
          launch_k((binary_bcast_rows_kernel<T, OP, kRowVec, true>), grid, kBlock, 0, stream,
                   bp, ap, 0, op, rows, cpk, al);
          return launch_status();
        }
        // full op s[r] / s[r] op full (one value per row, any alignment)
        if (a_dense && aligned16(ap) && colvec_strides(sz, sb_, ndim, &rs)) {
          launch_k((binary_bcast_rows_kernel<T, OP, kColVec, false>), grid, kBlock, 0, stream,
                   ap, bp, rs, op, rows, cpk, al);
          return launch_status();
        }
        if (b_dense && aligned16(bp) && colvec_strides(sz, sa_, ndim, &rs)) {
          launch_k((binary_bcast_rows_kernel<T, OP, kColVec, true>), grid, kBlock, 0, stream,
                   bp, ap, rs, op, rows, cpk, al);
          return launch_status();
        }
      }
      auto kern = binary_nd_float_kernel<T, OP>;
      launch_k(kern, grid_for(kern, n, dev, 4), kBlock, 0, stream, ap, bp, op, n, g, al);
      return launch_status();
    }
  });
}

template <typename S>
int cast_from(const S* src, void* dst, int dst_dtype, int64_t n, const DeviceInfo& dev,
              cudaStream_t stream) {
  return dispatch_any(dst_dtype, [&](auto tag) -> int {
    using D = decltype(tag);
    D* dp = static_cast<D*>(dst);
    if (n % 8 == 0 && aligned16(src) && aligned16(dp)) {
      auto kern = cast_vec8_kernel<S, D>;
      launch_k(kern, grid_for(kern, n / 8, dev), kBlock, 0, stream, src, dp, n / 8);
    } else {
      auto kern = cast_kernel<S, D>;
      launch_k(kern, grid_for(kern, ceil_div(n, 4), dev), kBlock, 0, stream, src, dp, n);
    }
    return launch_status();
  });
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_add(const void* a, const int64_t* a_strides, const void* b,
                            const int64_t* b_strides, void* out, const int64_t* sizes,
                            int ndim, double alpha, int dtype, fl_b200_stream_t stream) {
  return flb200::binary_entry<flb200::kAdd>(a, a_strides, b, b_strides, out, sizes, ndim,
                                            alpha, dtype,
                                            static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_mul(const void* a, const int64_t* a_strides, const void* b,
                            const int64_t* b_strides, void* out, const int64_t* sizes,
                            int ndim, int dtype, fl_b200_stream_t stream) {
  return flb200::binary_entry<flb200::kMul>(a, a_strides, b, b_strides, out, sizes, ndim,
                                            1.0, dtype, static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_binary_scalar(const void* a, double s, void* out, int64_t n,
                                      int op, double alpha, int dtype,
                                      fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n >= 0 && (op == kAdd || op == kMul));
  if (n == 0) return FL_B200_OK;
  FLB_CHECK_ARG(a && out);
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  auto cs = static_cast<cudaStream_t>(stream);
  return dispatch_any(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const T* ap = static_cast<const T*>(a);
    T* outp = static_cast<T*>(out);
    auto run = [&](auto opc) -> int {
      constexpr int OP = decltype(opc)::value;
      if constexpr (std::is_integral<T>::value) {
        auto kern = scalar_int_kernel<T, OP>;
        launch_k(kern, grid_for(kern, n, dev, 4), kBlock, 0, cs, ap, outp, n, (T)(int64_t)s,
                 (T)(int64_t)alpha);
      } else {
        constexpr int VW = Elem<T>::kVec;
        if (n % (2 * VW) == 0 && aligned32(ap) && aligned32(outp)) {
          const int64_t npk32 = n / (2 * VW);
          launch_k((scalar_float_vec32_kernel<T, OP>),
                   full_grid(ceil_div(npk32, (int64_t)kBlock32 * kPacks32)), kBlock32, 0, cs,
                   ap, outp, npk32, (float)s, (float)alpha);
        } else if (n % VW == 0 && aligned16(ap) && aligned16(outp)) {
          auto kern = scalar_float_vec_kernel<T, OP>;
          launch_k(kern, grid_for(kern, n / VW, dev), kBlock, 0, cs, ap, outp, n / VW,
                   (float)s, (float)alpha);
        } else {
          auto kern = scalar_float_kernel<T, OP>;
          launch_k(kern, grid_for(kern, n, dev, 4), kBlock, 0, cs, ap, outp, n, (float)s,
                   (float)alpha);
        }
      }
      return launch_status();
    };
    if (op == kAdd) return run(std::integral_constant<int, kAdd>{});
    return run(std::integral_constant<int, kMul>{});
  });
}

FL_B200_API int fl_b200_cast(const void* src, int src_dtype, void* dst, int dst_dtype,
                             int64_t n, fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n >= 0);
  if (n == 0) return FL_B200_OK;
  FLB_CHECK_ARG(src && dst);
  if (dtype_size(src_dtype) == 0 || dtype_size(dst_dtype) == 0)
    return FL_B200_ERR_UNSUPPORTED_DTYPE;
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  auto cs = static_cast<cudaStream_t>(stream);
  return dispatch_any(src_dtype, [&](auto tag) -> int {
    using S = decltype(tag);
    return cast_from<S>(static_cast<const S*>(src), dst, dst_dtype, n, dev, cs);
  });
}

}  // extern "C"
