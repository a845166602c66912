// RMSNorm forward and fused residual-add + RMSNorm.
//
// Reference behaviour: the HF formula (transformers
// models/qwen3/modeling_qwen3.py:59-64) run op by op on the flagos device:
//   h32 = x.to(f32); var = h32.pow(2).mean(-1, keepdim); h = h32*rsqrt(var+eps)
//   out = w * h.to(x.dtype)
// i.e. csrc/aten/backends/cuda/{pow.cu:29-32, mean.cu:30-63, add.cu:72-76,
// rsqrt.cu:14-32, mul.cu:28-52} plus two _to_copy casts
// (csrc/aten/copy_ops.cc:225-240).  Here it is one pass: each row is read
// once into registers, reduced in fp32, scaled and written once.
#include "row_ladder.cuh"

namespace flb200 {
namespace {

// out = w * (x * r) with r = 1/sqrt(mean(x^2) + eps).  In chain mode the
// product x*r is rounded to T before the weight multiply, as the HF
// `.to(input_dtype)` does.
template <typename T, bool CHAIN>
__device__ __forceinline__ void rms_scale_store(const uint4& xv, const T* w, T* o,
                                                float r) {
  constexpr int VW = Elem<T>::kVec;
  float f[VW], wf[VW], y[VW];
  unpack<T>(xv, f);
  unpack<T>(ld_cached(w), wf);
#pragma unroll
  for (int e = 0; e < VW; ++e) {
    float t = f[e] * r;
    if (CHAIN) t = round_to<T>(t);
    y[e] = wf[e] * t;
  }
  st_stream(o, pack<T>(y));
}

// Row-in-registers kernel: TPR threads own a row, VPT packs each.
// If ADD, the row is h = x + y (rounded to T, stored to h) and the norm is
// taken over h.
template <typename T, int TPR, int VPT, int BLOCK, bool CHAIN, bool ADD>
__global__ void __launch_bounds__(BLOCK, ladder_min_blocks<BLOCK>())
rms_norm_vec_kernel(const T* x, int64_t ldx, const T* y, T* h, const T* w, T* out,
                    int64_t ldo, int64_t rows, int nvec, float eps, float cols_f) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  constexpr int RPB = BLOCK / TPR;
  __shared__ float smem[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows;
       base += (int64_t)gridDim.x * RPB) {
    const int64_t row = base + slot;
    const bool ok = row < rows;
    const T* xr = x + row * ldx;
    uint4 v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      v[i] = (ok && vi < nvec) ? ld_stream(xr + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
    }
    if constexpr (ADD) {
      const T* yr = y + row * ldx;
      T* hr = h + row * ldx;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lane + i * TPR;
        if (ok && vi < nvec) {
          float a[VW], b[VW];
          unpack<T>(v[i], a);
          unpack<T>(ld_stream(yr + (int64_t)vi * VW), b);
#pragma unroll
          for (int e = 0; e < VW; ++e) a[e] = a[e] + b[e];
          v[i] = pack<T>(a);  // the residual stream is stored in T
          st_stream(hr + (int64_t)vi * VW, v[i]);
        }
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[VW];
      unpack<T>(v[i], f);
#pragma unroll
      for (int e = 0; e < VW; ++e) ss = fmaf(f[e], f[e], ss);
    }
    ss = row_reduce<SumOp, TPR, BLOCK>(ss, smem);
    const float r = 1.0f / sqrtf(ss / cols_f + eps);
    T* orow = out + row * ldo;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (ok && vi < nvec)
        rms_scale_store<T, CHAIN>(opaque(v[i]), w + (int64_t)vi * VW, orow + (int64_t)vi * VW, r);
    }
  }
}

// Residual add + RMSNorm with 32-byte accesses and fp32 pairs: h = x + y
// (pair add, one conversion per pair gives both the stored h and its fp32
// value), the sum of squares by pair FMA, out = w * (h * r) by pair
// multiplies.  Same roundings as rms_norm_vec_kernel<ADD> per element; the
// sum of squares runs as two interleaved partial sums per thread.  Half the
// memory instructions and about 20 % fewer arithmetic ones, for the launch
// that runs right after SwiGLU in every decoder layer, under the power cap.
template <typename T>
__device__ __forceinline__ void unpack32(const Pack32& p, float (&f)[2 * Elem<T>::kVec]) {
  constexpr int VW = Elem<T>::kVec;
  float a[VW], b[VW];
  unpack<T>(p.lo, a);
  unpack<T>(p.hi, b);
#pragma unroll
  for (int e = 0; e < VW; ++e) {
    f[e] = a[e];
    f[VW + e] = b[e];
  }
}

// Encodes NP fp32 pairs as the 32 bytes of 2*NP values of T (rounded to
// nearest even for 16-bit T).
template <typename T, int NP>
__device__ __forceinline__ Pack32 pairs_to_pack32(const uint64_t (&pr)[NP]) {
  uint32_t wd[8];
  if constexpr (std::is_same<T, float>::value) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      wd[2 * p] = __float_as_uint(f2_lo(pr[p]));
      wd[2 * p + 1] = __float_as_uint(f2_hi(pr[p]));
    }
  } else {
#pragma unroll
    for (int p = 0; p < NP; ++p) wd[p] = pair_to_bits<T>(pr[p]);
  }
  return Pack32{make_uint4(wd[0], wd[1], wd[2], wd[3]), make_uint4(wd[4], wd[5], wd[6], wd[7])};
}

template <typename T, int TPR, int VPT, int BLOCK, bool CHAIN>
__global__ void __launch_bounds__(BLOCK, ladder_min_blocks<BLOCK>())
add_rms_norm_w32_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ y,
                        T* __restrict__ h, const T* __restrict__ w, T* __restrict__ out,
                        int64_t ldo, int64_t rows, int nvec32, float eps, float cols_f) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  constexpr int E = 2 * VW;  // elements per 32-byte pack
  constexpr int NP = E / 2;  // fp32 pairs per 32-byte pack
  constexpr int RPB = BLOCK / TPR;
  __shared__ float smem[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const Pack32 zero{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows;
       base += (int64_t)gridDim.x * RPB) {
    const int64_t row = base + slot;
    const bool ok = row < rows;
    const T* xr = x + row * ldx;
    const T* yr = y + row * ldx;
    Pack32 xa[VPT], ya[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      const bool in = ok && vi < nvec32;
      xa[i] = in ? ld_stream32(xr + (int64_t)vi * E) : zero;
      ya[i] = in ? ld_stream32(yr + (int64_t)vi * E) : zero;
    }
    // h between the two passes: fp32 pairs for fp32 rows, else its 16-bit
    // encodings (half the registers; re-expanded for the output pass)
    uint64_t hp[VPT][NP];
    uint32_t hb[VPT][NP];
    uint64_t ss2 = f2_make(0.f, 0.f);
    T* hr = h + row * ldx;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      float a[E], b[E];
      unpack32<T>(xa[i], a);
      unpack32<T>(ya[i], b);
      // the residual stream is stored in T: the sum rounded to T is both the
      // stored h and the value normalised (one conversion per pair)
      Pack32 hv;
      if constexpr (std::is_same<T, float>::value) {
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          hp[i][p] = f2_add(f2_make(a[2 * p], a[2 * p + 1]), f2_make(b[2 * p], b[2 * p + 1]));
          ss2 = f2_fma(hp[i][p], hp[i][p], ss2);
        }
        hv = pairs_to_pack32<T, NP>(hp[i]);
      } else {
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          hb[i][p] = pair_to_bits<T>(
              f2_add(f2_make(a[2 * p], a[2 * p + 1]), f2_make(b[2 * p], b[2 * p + 1])));
          const uint64_t t = pair_from_bits<T>(hb[i][p]);
          ss2 = f2_fma(t, t, ss2);
        }
        hv = Pack32{make_uint4(hb[i][0], hb[i][1], hb[i][2], hb[i][3]),
                    make_uint4(hb[i][4], hb[i][5], hb[i][6], hb[i][7])};
      }
      if (ok && vi < nvec32) st_stream32(hr + (int64_t)vi * E, hv);
    }
    float ss = f2_lo(ss2) + f2_hi(ss2);
    ss = row_reduce<SumOp, TPR, BLOCK>(ss, smem);
    const float r = 1.0f / sqrtf(ss / cols_f + eps);
    const uint64_t r2 = f2_make(r, r);
    T* orow = out + row * ldo;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (!ok || vi >= nvec32) continue;
      float wf[E];
      unpack32<T>(Pack32{ld_cached(w + (int64_t)vi * E), ld_cached(w + (int64_t)vi * E + VW)},
                  wf);
      uint64_t o[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        uint64_t hv;
        if constexpr (std::is_same<T, float>::value) hv = hp[i][p];
        else hv = pair_from_bits<T>(hb[i][p]);
        uint64_t t = f2_mul(hv, r2);
        if (CHAIN) t = round_pair<T>(t);
        o[p] = f2_mul(f2_make(wf[2 * p], wf[2 * p + 1]), t);
      }
      st_stream32(orow + (int64_t)vi * E, pairs_to_pack32<T, NP>(o));
    }
  }
}

// Looped kernel for any row length and alignment: one CTA per row, scalar
// element loads; the row is read twice (the second read mostly hits L2).
template <typename T, bool CHAIN, bool ADD>
__global__ void __launch_bounds__(256)
rms_norm_loop_kernel(const T* x, int64_t ldx, const T* y, T* h, const T* w, T* out,
                     int64_t ldo, int64_t rows, int64_t cols, float eps) {
  pdl_prologue();
  __shared__ float smem[256 / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * ldx;
    float ss = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      float f = Elem<T>::to_f(xr[c]);
      if constexpr (ADD) {
        f = round_to<T>(f + Elem<T>::to_f(y[row * ldx + c]));
        h[row * ldx + c] = Elem<T>::from_f(f);
      }
      ss = fmaf(f, f, ss);
    }
    ss = block_reduce<SumOp, 256>(ss, smem);
    const float r = 1.0f / sqrtf(ss / (float)cols + eps);
    const T* src = ADD ? h + row * ldx : xr;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      float t = Elem<T>::to_f(src[c]) * r;
      if (CHAIN) t = round_to<T>(t);
      out[row * ldo + c] = Elem<T>::from_f(Elem<T>::to_f(w[c]) * t);
    }
  }
}

template <typename T, bool CHAIN, bool ADD>
int launch_rms_norm(const T* x, int64_t ldx, const T* y, T* h, const T* w, T* out,
                    int64_t ldo, int64_t rows, int64_t cols, float eps,
                    cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<T>::kVec;
  const bool vec_ok = aligned16(x) && aligned16(w) && aligned16(out) &&
                      (!ADD || (aligned16(y) && aligned16(h))) && cols % VW == 0 &&
                      ldx % VW == 0 && ldo % VW == 0;
  if constexpr (ADD) {
    constexpr int E = 2 * VW;
    if (aligned32(x) && aligned32(y) && aligned32(h) && aligned32(w) && aligned32(out) &&
        cols % E == 0 && ldx % E == 0 && ldo % E == 0) {
      auto go = [&](auto tpr, auto vpt) -> int {
        constexpr int TPR = decltype(tpr)::value;
        constexpr int VPT = decltype(vpt)::value;
        constexpr int BLOCK = ladder_block<TPR>();
        launch_k((add_rms_norm_w32_kernel<T, TPR, VPT, BLOCK, CHAIN>),
                 full_grid(ceil_div(rows, BLOCK / TPR)), BLOCK, 0, stream, x, ldx, y, h, w,
                 out, ldo, rows, (int)(cols / E), eps, (float)cols);
        return launch_status();
      };
      // one 32-byte pack per thread from 129 to 1024 packs (4096-wide bf16
      // rows: 256 threads), the two-pack ladder elsewhere
      using std::integral_constant;
      using V1 = integral_constant<int, 1>;
      const int64_t n32 = cols / E;
      int r;
      if (n32 > 128 && n32 <= 256) r = go(integral_constant<int, 256>{}, V1{});
      else if (n32 > 256 && n32 <= 512) r = go(integral_constant<int, 512>{}, V1{});
      else if (n32 > 512 && n32 <= 1024) r = go(integral_constant<int, 1024>{}, V1{});
      else r = row_ladder<2>(n32, go);
      if (r >= 0) return r;
    }
  }
  if (vec_ok) {
    const int64_t nvec = cols / VW;
    // One CTA per group of rows (full grid); two input streams (ADD) want
    // fewer packs per thread and more threads per row.
    int r = row_ladder<ADD ? 2 : 8>(nvec, [&](auto tpr, auto vpt) -> int {
      constexpr int TPR = decltype(tpr)::value;
      constexpr int VPT = decltype(vpt)::value;
      constexpr int BLOCK = ladder_block<TPR>();
      auto kern = rms_norm_vec_kernel<T, TPR, VPT, BLOCK, CHAIN, ADD>;
      const int64_t units = ceil_div(rows, BLOCK / TPR);
      const int grid = full_grid(units);
      launch_k(kern, grid, BLOCK, 0, stream, x, ldx, y, h, w, out, ldo, rows, (int)nvec, eps,
               (float)cols);
      return launch_status();
    });
    if (r >= 0) return r;
  }
  auto kern = rms_norm_loop_kernel<T, CHAIN, ADD>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * dev.sm_count);
  launch_k(kern, grid, 256, 0, stream, x, ldx, y, h, w, out, ldo, rows, cols, eps);
  return launch_status();
}

template <bool ADD>
int rms_norm_entry(const void* x, int64_t ldx, const void* y, void* h, const void* w,
                   void* out, int64_t ldo, int64_t rows, int64_t cols, float eps,
                   int dtype, int rounding, cudaStream_t stream) {
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && w && out && ldx >= cols && ldo >= cols);
  FLB_CHECK_ARG(!ADD || (y && h));
  FLB_CHECK_ARG(rounding == FL_B200_ROUND_FUSED || rounding == FL_B200_ROUND_CHAIN);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto* xp = static_cast<const T*>(x);
    auto* yp = static_cast<const T*>(y);
    auto* hp = static_cast<T*>(h);
    auto* wp = static_cast<const T*>(w);
    auto* op = static_cast<T*>(out);
    if (rounding == FL_B200_ROUND_CHAIN)
      return launch_rms_norm<T, true, ADD>(xp, ldx, yp, hp, wp, op, ldo, rows, cols, eps,
                                           stream);
    return launch_rms_norm<T, false, ADD>(xp, ldx, yp, hp, wp, op, ldo, rows, cols, eps,
                                          stream);
  });
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_rms_norm_fwd(const void* x, int64_t ld_x, const void* w,
                                     void* out, int64_t ld_out, int64_t rows,
                                     int64_t cols, float eps, int dtype, int rounding,
                                     fl_b200_stream_t stream) {
  return flb200::rms_norm_entry<false>(x, ld_x, nullptr, nullptr, w, out, ld_out, rows,
                                       cols, eps, dtype, rounding,
                                       static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_add_rms_norm_fwd(const void* x, const void* y, void* h,
                                         const void* w, void* out, int64_t rows,
                                         int64_t cols, float eps, int dtype,
                                         int rounding, fl_b200_stream_t stream) {
  return flb200::rms_norm_entry<true>(x, cols, y, h, w, out, cols, rows, cols, eps,
                                      dtype, rounding, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
