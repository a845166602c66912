// SwiGLU (silu(gate) * up) and SwiGLU + residual add in one launch.
//
// Reference behaviour: HF Qwen3MLP act_fn(gate) * up (transformers
// models/qwen3/modeling_qwen3.py:81-82), run on flagos as silu
// (csrc/aten/backends/cuda/silu.cu:15-35: x / (1 + exp(-x)) in fp32 opmath,
// rounded to the tensor dtype) followed by mul (mul.cu:28-52).  The residual
// add is add.Tensor (add.cu:48-84).  Pure streaming, launched as a full grid.
// The hot kernel (swiglu32_kernel) runs 512-thread CTAs, each thread loading
// two 32-byte packs (v8 accesses) of gate and up, one CTA per 1024 packs; the
// residual rows, when present, are extra CTAs of the same launch.  Operands
// not 32-byte aligned take the 16-byte kernels (one pack per thread, 256-thread
// CTAs; common.cuh full_grid).
#include "common.cuh"

#include <algorithm>

namespace flb200 {
namespace {

constexpr int kBlock = 256;
constexpr int kUnroll = 4;

template <typename T, bool CHAIN>
__device__ __forceinline__ float swiglu_one(float g, float u) {
  if (CHAIN) {
    // silu is its own aten op (fp32 opmath with the accurate exp, rounded to
    // T); the mul rounds again.
    const float s = round_to<T>(g / (1.0f + expf(-g)));
    return s * u;
  }
  return __fdividef(g * u, 1.0f + __expf(-g));
}

template <typename T, bool CHAIN>
__device__ __forceinline__ uint4 swiglu_pack(const uint4& gv, const uint4& uv) {
  constexpr int VW = Elem<T>::kVec;
  float g[VW], u[VW], o[VW];
  unpack<T>(gv, g);
  unpack<T>(uv, u);
#pragma unroll
  for (int e = 0; e < VW; ++e) o[e] = swiglu_one<T, CHAIN>(g[e], u[e]);
  return pack<T>(o);
}

template <typename T>
__device__ __forceinline__ uint4 add_pack(const uint4& xv, const uint4& yv) {
  constexpr int VW = Elem<T>::kVec;
  float a[VW], b[VW];
  unpack<T>(xv, a);
  unpack<T>(yv, b);
#pragma unroll
  for (int e = 0; e < VW; ++e) a[e] = a[e] + b[e];
  return pack<T>(a);
}

// Grid-stride over n packs of dense gate/up/out.
template <typename T, bool CHAIN>
__device__ __forceinline__ void swiglu_dense(const T* g, const T* u, T* o, int64_t n,
                                             int64_t tid, int64_t nthreads) {
  constexpr int VW = Elem<T>::kVec;
  int64_t i = tid;
  for (; i + (kUnroll - 1) * nthreads < n; i += kUnroll * nthreads) {
    uint4 gv[kUnroll], uv[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      gv[k] = ld_stream(g + (i + k * nthreads) * VW);
      uv[k] = ld_stream(u + (i + k * nthreads) * VW);
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
      st_stream(o + (i + k * nthreads) * VW, swiglu_pack<T, CHAIN>(gv[k], uv[k]));
  }
  for (; i < n; i += nthreads)
    st_stream(o + i * VW, swiglu_pack<T, CHAIN>(ld_stream(g + i * VW), ld_stream(u + i * VW)));
}

template <typename T>
__device__ __forceinline__ void add_dense(const T* x, const T* y, T* h, int64_t n,
                                          int64_t tid, int64_t nthreads) {
  constexpr int VW = Elem<T>::kVec;
  int64_t i = tid;
  for (; i + (kUnroll - 1) * nthreads < n; i += kUnroll * nthreads) {
    uint4 xv[kUnroll], yv[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      xv[k] = ld_stream(x + (i + k * nthreads) * VW);
      yv[k] = ld_stream(y + (i + k * nthreads) * VW);
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k)
      st_stream(h + (i + k * nthreads) * VW, add_pack<T>(xv[k], yv[k]));
  }
  for (; i < n; i += nthreads)
    st_stream(h + i * VW, add_pack<T>(ld_stream(x + i * VW), ld_stream(y + i * VW)));
}

template <typename T, bool CHAIN>
__global__ void __launch_bounds__(kBlock)
swiglu_vec_kernel(const T* g, const T* u, T* o, int64_t n) {
  pdl_prologue();
  swiglu_dense<T, CHAIN>(g, u, o, n, (int64_t)blockIdx.x * kBlock + threadIdx.x,
                         (int64_t)gridDim.x * kBlock);
}

// Both passes in one grid: every thread does its share of the SwiGLU packs,
// then its share of the residual-add packs.
template <typename T, bool CHAIN>
__global__ void __launch_bounds__(kBlock)
swiglu_residual_kernel(const T* g, const T* u, T* act, int64_t n_act, const T* x,
                       const T* y, T* h, int64_t n_res) {
  pdl_prologue();
  const int64_t tid = (int64_t)blockIdx.x * kBlock + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * kBlock;
  swiglu_dense<T, CHAIN>(g, u, act, n_act, tid, nth);
  add_dense<T>(x, y, h, n_res, tid, nth);
}

// 32-byte packs (two 16-byte halves per access), two per thread (packs i
// and i + 512 of the CTA's 1024), 512-thread CTAs: the path for 32-byte
// aligned dense tensors.  Measured on B200, bf16 131072 x 14336 alone: 7.20
// TB/s against 7.04 with one pack per thread in 256-thread CTAs.  The CTAs
// of the grid's first `act_blocks` do SwiGLU packs, the rest residual-add
// packs (n_res may be 0).
constexpr int kBlock32 = 512;
constexpr int kPacks32 = 2;

template <typename T, bool CHAIN>
__global__ void __launch_bounds__(kBlock32)
swiglu32_kernel(const T* g, const T* u, T* act, int64_t n_act, int64_t act_blocks,
                const T* x, const T* y, T* h, int64_t n_res) {
  pdl_prologue();
  constexpr int VW2 = 2 * Elem<T>::kVec;  // elements per 32-byte pack
  const bool is_act = (int64_t)blockIdx.x < act_blocks;
  const int64_t blk = is_act ? (int64_t)blockIdx.x : (int64_t)blockIdx.x - act_blocks;
  const int64_t i0 = blk * (kBlock32 * kPacks32) + threadIdx.x;
  const T* a = is_act ? g : x;
  const T* b = is_act ? u : y;
  T* o = is_act ? act : h;
  const int64_t n = is_act ? n_act : n_res;
  Pack32 av[kPacks32], bv[kPacks32];
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i < n) {
      av[k] = ld_stream32(a + i * VW2);
      bv[k] = ld_stream32(b + i * VW2);
    }
  }
#pragma unroll
  for (int k = 0; k < kPacks32; ++k) {
    const int64_t i = i0 + (int64_t)k * kBlock32;
    if (i >= n) continue;
    Pack32 r;
    if (is_act) {
      r.lo = swiglu_pack<T, CHAIN>(av[k].lo, bv[k].lo);
      r.hi = swiglu_pack<T, CHAIN>(av[k].hi, bv[k].hi);
    } else {
      r.lo = add_pack<T>(av[k].lo, bv[k].lo);
      r.hi = add_pack<T>(av[k].hi, bv[k].hi);
    }
    st_stream32(o + i * VW2, r);
  }
}

template <typename T, bool CHAIN>
int launch_swiglu32(const T* g, const T* u, T* act, int64_t n_act, const T* x, const T* y,
                    T* h, int64_t n_res, cudaStream_t stream) {
  constexpr int VW2 = 2 * Elem<T>::kVec;
  const int64_t pa = n_act / VW2, pr = n_res / VW2;
  constexpr int64_t kChunk = (int64_t)kBlock32 * kPacks32;
  const int64_t ba = ceil_div(pa, kChunk), br = ceil_div(pr, kChunk);
  if (ba + br > 0x7fffffff) return FL_B200_ERR_TOO_LARGE;
  launch_k((swiglu32_kernel<T, CHAIN>), (int)std::max<int64_t>(ba + br, 1), kBlock32, 0,
           stream, g, u, act, pa, ba, x, y, h, pr);
  return launch_status();
}

// Strided / unaligned rows: scalar element access.
template <typename T, bool CHAIN>
__global__ void __launch_bounds__(kBlock)
swiglu_strided_kernel(const T* g, int64_t ldg, const T* u, int64_t ldu, T* o,
                      int64_t ldo, int64_t rows, int64_t cols) {
  pdl_prologue();
  const int64_t n = rows * cols;
  for (int64_t i = (int64_t)blockIdx.x * kBlock + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * kBlock) {
    const int64_t r = i / cols, c = i - r * cols;
    const float gv = Elem<T>::to_f(g[r * ldg + c]);
    const float uv = Elem<T>::to_f(u[r * ldu + c]);
    o[r * ldo + c] = Elem<T>::from_f(swiglu_one<T, CHAIN>(gv, uv));
  }
}

template <typename T, bool CHAIN>
int launch_swiglu(const T* g, int64_t ldg, const T* u, int64_t ldu, T* o, int64_t ldo,
                  int64_t rows, int64_t cols, cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<T>::kVec;
  const bool dense = ldg == cols && ldu == cols && ldo == cols;
  const int64_t n = rows * cols;
  if (dense && n % (2 * VW) == 0 && aligned32(g) && aligned32(u) && aligned32(o))
    return launch_swiglu32<T, CHAIN>(g, u, o, n, nullptr, nullptr, nullptr, 0, stream);
  if (dense && n % VW == 0 && aligned16(g) && aligned16(u) && aligned16(o)) {
    auto kern = swiglu_vec_kernel<T, CHAIN>;
    const int64_t npk = n / VW;
    const int grid = full_grid(ceil_div(npk, kBlock));  // one pack per thread
    launch_k(kern, grid, kBlock, 0, stream, g, u, o, npk);
    return launch_status();
  }
  auto kern = swiglu_strided_kernel<T, CHAIN>;
  const int grid = full_grid(ceil_div(n, kBlock));
  launch_k(kern, grid, kBlock, 0, stream, g, ldg, u, ldu, o, ldo, rows, cols);
  return launch_status();
}

template <typename T, bool CHAIN>
int launch_swiglu_residual(const T* g, const T* u, T* act, int64_t inter, const T* x,
                           const T* y, T* h, int64_t hidden, int64_t rows,
                           cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<T>::kVec;
  const int64_t n1 = rows * inter, n2 = rows * hidden;
  if (n1 % (2 * VW) == 0 && n2 % (2 * VW) == 0 && aligned32(g) && aligned32(u) &&
      aligned32(act) && aligned32(x) && aligned32(y) && aligned32(h))
    return launch_swiglu32<T, CHAIN>(g, u, act, n1, x, y, h, n2, stream);
  const bool vec_ok = n1 % VW == 0 && n2 % VW == 0 && aligned16(g) && aligned16(u) &&
                      aligned16(act) && aligned16(x) && aligned16(y) && aligned16(h);
  if (!vec_ok) return FL_B200_ERR_MISALIGNED;
  auto kern = swiglu_residual_kernel<T, CHAIN>;
  const int64_t npk = std::max(n1, n2) / VW;
  const int grid = full_grid(ceil_div(npk, kBlock));  // one pack of each part per thread
  launch_k(kern, grid, kBlock, 0, stream, g, u, act, n1 / VW, x, y, h, n2 / VW);
  return launch_status();
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_swiglu(const void* gate, int64_t ld_g, const void* up,
                               int64_t ld_u, void* out, int64_t ld_out, int64_t rows,
                               int64_t cols, int dtype, int rounding,
                               fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(gate && up && out && ld_g >= cols && ld_u >= cols && ld_out >= cols);
  FLB_CHECK_ARG(rounding == FL_B200_ROUND_FUSED || rounding == FL_B200_ROUND_CHAIN);
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto g = static_cast<const T*>(gate);
    auto u = static_cast<const T*>(up);
    auto o = static_cast<T*>(out);
    if (rounding == FL_B200_ROUND_CHAIN)
      return launch_swiglu<T, true>(g, ld_g, u, ld_u, o, ld_out, rows, cols, s);
    return launch_swiglu<T, false>(g, ld_g, u, ld_u, o, ld_out, rows, cols, s);
  });
}

FL_B200_API int fl_b200_swiglu_residual(const void* gate, const void* up, void* act,
                                        int64_t inter, const void* x, const void* y,
                                        void* h, int64_t hidden, int64_t rows,
                                        int dtype, int rounding,
                                        fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && inter >= 0 && hidden >= 0);
  if (rows == 0 || (inter == 0 && hidden == 0)) return FL_B200_OK;
  FLB_CHECK_ARG(inter == 0 || (gate && up && act));
  FLB_CHECK_ARG(hidden == 0 || (x && y && h));
  FLB_CHECK_ARG(rounding == FL_B200_ROUND_FUSED || rounding == FL_B200_ROUND_CHAIN);
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto g = static_cast<const T*>(gate);
    auto u = static_cast<const T*>(up);
    auto a = static_cast<T*>(act);
    auto xp = static_cast<const T*>(x);
    auto yp = static_cast<const T*>(y);
    auto hp = static_cast<T*>(h);
    if (rounding == FL_B200_ROUND_CHAIN)
      return launch_swiglu_residual<T, true>(g, u, a, inter, xp, yp, hp, hidden, rows, s);
    return launch_swiglu_residual<T, false>(g, u, a, inter, xp, yp, hp, hidden, rows, s);
  });
}

}  // extern "C"
