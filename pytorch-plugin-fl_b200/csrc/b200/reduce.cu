// Reductions: sum / mean / amax / argmax over the last dim or the whole
// tensor, exact int32 -> int64 sums, and reductions over a middle dim.
//
// Reference behaviour: sum.dim_IntList (register.cc:333-337 -> csrc/aten/
// backends/cuda/sum.cu:32-66, fp32 accumulation for 16-bit inputs), mean.dim
// (register.cc:248-252 -> mean.cu:30-63) and amax / argmax, which the
// reference leaves unregistered so they run in the CPU fallback
// (register.cc:439-442 -> fallback.cc:12-14).  argmax returns the first
// index of the maximum; NaN counts as the maximum (torch semantics).
//
// One kernel family covers every row shape.  A row is cut into `splits`
// chunks (1 when there are enough rows to fill the GPU); each CTA reduces one
// chunk with 16-byte loads.  With splits > 1 the CTA writes its partial to
// the workspace and the last CTA of the row (atomic ticket) merges the
// partials in chunk order, so the result does not depend on CTA timing.
#include "common.cuh"

#include <atomic>
#include <mutex>

namespace flb200 {
namespace {

constexpr int kBlock = 256;
constexpr int kUnroll = 4;
// CTAs a split reduction aims for: 27 per SM of a 148-SM B200, so a long
// row's chunks fill every SM to the same depth and the last wave is short
// (2048 CTAs of 1 MB left a 0.3-wave tail: 5.4 vs 6.8 TB/s row-wise).  The
// parts of one row then fit the 64 KB scratch of the no-allocation sum.
constexpr int64_t kTargetCtas = 148 * 27;
constexpr int64_t kMinChunk = 16384;    // elements per CTA before splitting pays
constexpr int64_t kSplitRowsBelow = 1024;

// ---- accumulation policies --------------------------------------------------
// Each policy: Acc (per thread / per CTA), Part (cross-CTA partial), and the
// operations to fold an element, merge two Accs (lower indices first), widen
// an Acc to a Part and merge Parts.

struct SumPolicy {
  using Acc = float;
  using Part = double;
  __device__ static Acc init() { return 0.f; }
  __device__ static void fold(Acc& a, float v, int64_t) { a += v; }
  __device__ static Acc merge(Acc a, Acc b) { return a + b; }
  __device__ static Acc shfl(Acc a, int off) { return __shfl_xor_sync(0xffffffffu, a, off); }
  __device__ static Part part(Acc a) { return (double)a; }
  __device__ static Part pinit() { return 0.0; }
  __device__ static Part pmerge(Part a, Part b) { return a + b; }
};

struct MaxPolicy {
  using Acc = float;
  using Part = float;
  __device__ static Acc init() { return -INFINITY; }
  __device__ static void fold(Acc& a, float v, int64_t) { a = MaxOp::combine(a, v); }
  __device__ static Acc merge(Acc a, Acc b) { return MaxOp::combine(a, b); }
  __device__ static Acc shfl(Acc a, int off) { return __shfl_xor_sync(0xffffffffu, a, off); }
  __device__ static Part part(Acc a) { return a; }
  __device__ static Part pinit() { return -INFINITY; }
  __device__ static Part pmerge(Part a, Part b) { return MaxOp::combine(a, b); }
};

struct IntSumPolicy {
  using Acc = long long;
  using Part = long long;
  __device__ static Acc init() { return 0; }
  __device__ static void fold(Acc& a, long long v, int64_t) { a += v; }
  __device__ static Acc merge(Acc a, Acc b) { return a + b; }
  __device__ static Acc shfl(Acc a, int off) { return __shfl_xor_sync(0xffffffffu, a, off); }
  __device__ static Part part(Acc a) { return a; }
  __device__ static Part pinit() { return 0; }
  __device__ static Part pmerge(Part a, Part b) { return a + b; }
};

struct ArgMaxAcc {
  float v;
  long long i;
};
// True if candidate a wins over b: NaN beats numbers, larger beats smaller,
// ties go to the smaller index.
__device__ __forceinline__ bool argmax_better(const ArgMaxAcc& a, const ArgMaxAcc& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an || bn) return an && bn ? a.i < b.i : an;
  if (a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}
struct ArgMaxPolicy {
  using Acc = ArgMaxAcc;
  using Part = ArgMaxAcc;
  __device__ static Acc init() { return {-INFINITY, 0x7fffffffffffffffLL}; }
  __device__ static void fold(Acc& a, float v, int64_t j) {
    const Acc c{v, (long long)j};
    if (argmax_better(c, a)) a = c;
  }
  __device__ static Acc merge(Acc a, Acc b) { return argmax_better(b, a) ? b : a; }
  __device__ static Acc shfl(Acc a, int off) {
    Acc r;
    r.v = __shfl_xor_sync(0xffffffffu, a.v, off);
    r.i = __shfl_xor_sync(0xffffffffu, a.i, off);
    return r;
  }
  __device__ static Part part(Acc a) { return a; }
  __device__ static Part pinit() { return init(); }
  __device__ static Part pmerge(Part a, Part b) { return merge(a, b); }
};

// ---- element access ---------------------------------------------------------
template <typename T>
__device__ __forceinline__ float elem_value(T v) {
  return Elem<T>::to_f(v);
}

// NaN-propagating max of a 16-byte pack (PTX max.NaN on packed pairs: one
// instruction per two 16-bit elements), as fp32.  NaN if any element is NaN.
__device__ __forceinline__ float max_nan_f32(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_nan_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_nan_f16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <typename T>
__device__ __forceinline__ float pack_max_nan(const uint4& u) {
  if constexpr (std::is_same<T, float>::value) {
    return max_nan_f32(max_nan_f32(__uint_as_float(u.x), __uint_as_float(u.y)),
                       max_nan_f32(__uint_as_float(u.z), __uint_as_float(u.w)));
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const uint32_t m = max_nan_bf16x2(max_nan_bf16x2(u.x, u.y), max_nan_bf16x2(u.z, u.w));
    return max_nan_f32(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
  } else {
    const uint32_t m = max_nan_f16x2(max_nan_f16x2(u.x, u.y), max_nan_f16x2(u.z, u.w));
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&m));
    return max_nan_f32(v.x, v.y);
  }
}

// argmax of one thread's packs of a row chunk: packs p0 + t, p0 + t + kBlock,
// ... below p1.  The loop keeps only the running max (fp32, NaN-propagating)
// and the ordinal of the pack where it last rose: it rises where a pack's
// max is larger, or NaN while the running max is a number; an equal value
// never moves it (packs arrive in increasing index order, so the first stays).
// The winning pack stays in registers (copied on the rare rise), and is
// searched at the end for its first element equal to the max (or first
// NaN).  Same result as folding element by element with first-index ties
// and NaN as the maximum.
template <typename T, int U>
__device__ __forceinline__ ArgMaxAcc argmax_packs(const T* xr, int64_t p0, int64_t p1) {
  constexpr int VW = Elem<T>::kVec;
  const int64_t first = p0 + threadIdx.x;
  if (first >= p1) return ArgMaxPolicy::init();
  const int n = (int)ceil_div(p1 - first, kBlock);   // this thread's packs
  const T* base = xr + first * VW;
  float best = -INFINITY;
  int bestk = 0;  // a thread whose packs are all -inf keeps its first pack
  uint4 w = make_uint4(0, 0, 0, 0);
  for (int k0 = 0; k0 < n; k0 += U) {
    const T* pk = base + (int64_t)k0 * kBlock * VW;
    uint4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k)
      if (k0 + k < n) v[k] = ld_stream(pk + k * kBlock * VW);
    if (k0 == 0) w = v[0];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      if (k0 + k < n) {
        const float nb = max_nan_f32(best, pack_max_nan<T>(v[k]));
        const bool rose = (nb != best) && (best == best);
        if (rose) {
          bestk = k0 + k;
          w = v[k];
        }
        best = nb;
      }
    }
  }
  float f[VW];
  unpack<T>(w, f);
  const bool nan = best != best;
  int e = VW - 1;
#pragma unroll
  for (int k = VW - 1; k >= 0; --k)
    if (nan ? f[k] != f[k] : f[k] == best) e = k;
  return ArgMaxAcc{best, (long long)((first + (int64_t)bestk * kBlock) * VW + e)};
}

template <typename T, typename P>
__device__ __forceinline__ void fold_pack(typename P::Acc& acc, const uint4& u, int64_t j0) {
  if constexpr (std::is_same<T, int32_t>::value) {
    const int32_t w[4] = {(int32_t)u.x, (int32_t)u.y, (int32_t)u.z, (int32_t)u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) P::fold(acc, (long long)w[e], j0 + e);
  } else if constexpr (std::is_same<T, int64_t>::value) {
    P::fold(acc, (long long)(((uint64_t)u.y << 32) | u.x), j0);
    P::fold(acc, (long long)(((uint64_t)u.w << 32) | u.z), j0 + 1);
  } else {
    constexpr int VW = Elem<T>::kVec;
    float f[VW];
    unpack<T>(u, f);
#pragma unroll
    for (int e = 0; e < VW; ++e) P::fold(acc, f[e], j0 + e);
  }
}

template <typename T, typename P>
__device__ __forceinline__ void fold_scalar(typename P::Acc& acc, const T* p, int64_t j) {
  if constexpr (std::is_integral<T>::value) P::fold(acc, (long long)*p, j);
  else P::fold(acc, elem_value<T>(*p), j);
}

template <typename T>
__host__ __device__ constexpr int pack_width() {
  if constexpr (std::is_same<T, int32_t>::value) return 4;
  else if constexpr (std::is_same<T, int64_t>::value) return 2;
  else return Elem<T>::kVec;
}

// CTA-wide merge in a fixed tree (deterministic); result valid in thread 0.
template <typename P>
__device__ __forceinline__ typename P::Acc block_merge(typename P::Acc a) {
  using Acc = typename P::Acc;
  __shared__ Acc sm[kBlock / 32];
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    // Lane l merges with lane l^off; keep the lower-index side first.
    const Acc o = P::shfl(a, off);
    a = (threadIdx.x & off) ? P::merge(o, a) : P::merge(a, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sm[warp] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    a = sm[0];
#pragma unroll
    for (int w = 1; w < kBlock / 32; ++w) a = P::merge(a, sm[w]);
  }
  return a;
}

// The cross-CTA partials of a policy seen as a policy of their own, so the
// last CTA of a split row merges them with block_merge.
template <typename T>
__device__ __forceinline__ T shfl_part(T a, int off) {
  return __shfl_xor_sync(0xffffffffu, a, off);
}
template <>
__device__ __forceinline__ ArgMaxAcc shfl_part<ArgMaxAcc>(ArgMaxAcc a, int off) {
  return ArgMaxPolicy::shfl(a, off);
}
template <typename P>
struct PartOps {
  using Acc = typename P::Part;
  __device__ static Acc shfl(Acc a, int off) { return shfl_part(a, off); }
  __device__ static Acc merge(Acc a, Acc b) { return P::pmerge(a, b); }
};

// A partial written by another CTA of the grid (read past L1).
template <typename Part>
__device__ __forceinline__ Part load_part(const Part* p) {
  const volatile Part* v = p;
  if constexpr (std::is_same<Part, ArgMaxAcc>::value) {
    Part r;
    r.v = v->v;
    r.i = v->i;
    return r;
  } else {
    return *v;
  }
}

// ---- final stores -----------------------------------------------------------
enum Final { kFinalSum = 0, kFinalMean = 1, kFinalMax = 2, kFinalIdx = 3, kFinalI64 = 4 };

__device__ __forceinline__ void store_float(void* out, int64_t r, int out_dtype, float v) {
  switch (out_dtype) {
    case FL_B200_F32: static_cast<float*>(out)[r] = v; break;
    case FL_B200_BF16: static_cast<__nv_bfloat16*>(out)[r] = __float2bfloat16_rn(v); break;
    case FL_B200_F16: static_cast<__half*>(out)[r] = __float2half_rn(v); break;
    default: break;
  }
}

template <typename P, int FINAL>
__device__ __forceinline__ void store_final_acc(void* out, int64_t r, int out_dtype,
                                                typename P::Acc a, int64_t count) {
  if constexpr (FINAL == kFinalSum || FINAL == kFinalMax) store_float(out, r, out_dtype, a);
  else if constexpr (FINAL == kFinalMean) store_float(out, r, out_dtype, a / (float)count);
  else if constexpr (FINAL == kFinalIdx) static_cast<int64_t*>(out)[r] = a.i;
  else static_cast<int64_t*>(out)[r] = a;
}

template <typename P, int FINAL>
__device__ __forceinline__ void store_final_part(void* out, int64_t r, int out_dtype,
                                                 typename P::Part p, int64_t count) {
  if constexpr (FINAL == kFinalSum) store_float(out, r, out_dtype, (float)p);
  else if constexpr (FINAL == kFinalMean) store_float(out, r, out_dtype, (float)(p / (double)count));
  else if constexpr (FINAL == kFinalMax) store_float(out, r, out_dtype, p);
  else if constexpr (FINAL == kFinalIdx) static_cast<int64_t*>(out)[r] = p.i;
  else static_cast<int64_t*>(out)[r] = p;
}

// ---- the split-row kernel ---------------------------------------------------
// Work unit u = row * splits + split covers columns [split*chunk, +chunk).
template <typename T, typename P, int FINAL, bool VEC>
__global__ void __launch_bounds__(kBlock)
reduce_rows_kernel(const T* x, int64_t ld, int64_t rows, int64_t cols, int64_t splits,
                   int64_t chunk, void* out, int out_dtype, typename P::Part* parts,
                   unsigned int* tickets) {
  using Acc = typename P::Acc;
  using Part = typename P::Part;
  constexpr int VW = pack_width<T>();
  __shared__ bool last;
  const int64_t units = rows * splits;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int64_t r = u / splits, sp = u - r * splits;
    const int64_t c0 = sp * chunk;
    const int64_t c1 = min(cols, c0 + chunk);
    const T* xr = x + r * ld;
    Acc acc = P::init();
    if (VEC) {
      // chunk and ld are multiples of VW, so every pack is whole.  Loads go
      // out in batches of kUnroll packs per thread, the row's ragged end
      // included (a predicated batch), so a thread waits for HBM once per
      // batch.
      const int64_t p0 = c0 / VW, p1 = c1 / VW;
      if constexpr (std::is_same<P, ArgMaxPolicy>::value && !std::is_integral<T>::value) {
        acc = argmax_packs<T, 8>(xr, p0, p1);
      } else {
        for (int64_t p = p0 + threadIdx.x; p < p1; p += kUnroll * kBlock) {
          uint4 v[kUnroll];
#pragma unroll
          for (int k = 0; k < kUnroll; ++k)
            if (p + k * kBlock < p1) v[k] = ld_stream(xr + (p + k * kBlock) * VW);
#pragma unroll
          for (int k = 0; k < kUnroll; ++k)
            if (p + k * kBlock < p1) fold_pack<T, P>(acc, v[k], (p + k * kBlock) * VW);
        }
      }
    } else {
      for (int64_t c = c0 + threadIdx.x; c < c1; c += kBlock) fold_scalar<T, P>(acc, xr + c, c);
    }
    acc = block_merge<P>(acc);
    if (splits == 1) {
      if (threadIdx.x == 0) store_final_acc<P, FINAL>(out, r, out_dtype, acc, cols);
      continue;
    }
    if (threadIdx.x == 0) {
      parts[u] = P::part(acc);
      __threadfence();  // publish the partial before taking a ticket
      const unsigned int t = atomicAdd(&tickets[r], 1u);
      last = (t == (unsigned int)(splits - 1));
    }
    __syncthreads();
    if (last) {
      // Every other CTA of this row has published its partial.  Thread t
      // merges partials t, t + kBlock, ... in order, then the CTA merges the
      // threads in a fixed tree: the result does not depend on CTA timing.
      __threadfence();
      const Part* pr = parts + r * splits;
      Part acc2 = P::pinit();
      for (int64_t k = threadIdx.x; k < splits; k += kBlock)
        acc2 = P::pmerge(acc2, load_part(pr + k));
      acc2 = block_merge<PartOps<P>>(acc2);
      if (threadIdx.x == 0) {
        store_final_part<P, FINAL>(out, r, out_dtype, acc2, cols);
        tickets[r] = 0u;  // leave the workspace ready for the next call
      }
    }
    __syncthreads();  // `last` is rewritten by the next unit
  }
}

// ---- planning ---------------------------------------------------------------
struct Plan {
  int64_t splits;
  int64_t chunk;
  size_t parts_bytes;
  size_t ws_bytes;
};

constexpr size_t kPartBytes = 16;  // largest Part (ArgMaxAcc)

Plan make_plan(int64_t rows, int64_t cols) {
  Plan p{1, cols, 0, 0};
  if (rows > 0 && rows < kSplitRowsBelow && cols >= 2 * kMinChunk) {
    int64_t s = std::min<int64_t>(ceil_div(kTargetCtas, rows), cols / kMinChunk);
    if (s > 1) {
      // Chunks are whole multiples of kBlock*8 elements: pack-aligned for every
      // dtype and a whole number of CTA-wide steps.
      const int64_t quantum = kBlock * 8;
      const int64_t chunk = ceil_div(ceil_div(cols, s), quantum) * quantum;
      s = ceil_div(cols, chunk);
      if (s > 1) {
        p.splits = s;
        p.chunk = chunk;
        p.parts_bytes = (size_t)(rows * s) * kPartBytes;
        p.ws_bytes = p.parts_bytes + (size_t)rows * sizeof(unsigned int);
      }
    }
  }
  return p;
}

template <typename T, typename P, int FINAL>
int launch_reduce(const T* x, int64_t ld, int64_t rows, int64_t cols, void* out,
                  int out_dtype, void* ws, size_t ws_bytes, cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  const Plan plan = make_plan(rows, cols);
  using Part = typename P::Part;
  Part* parts = nullptr;
  unsigned int* tickets = nullptr;
  if (plan.splits > 1) {
    if (ws == nullptr || ws_bytes < plan.ws_bytes || !aligned16(ws))
      return FL_B200_ERR_WORKSPACE;
    parts = static_cast<Part*>(ws);
    tickets = reinterpret_cast<unsigned int*>(static_cast<char*>(ws) + plan.parts_bytes);
    cudaError_t e = cudaMemsetAsync(tickets, 0, (size_t)rows * sizeof(unsigned int), stream);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return FL_B200_ERR_LAUNCH;
    }
  }
  constexpr int VW = pack_width<T>();
  const bool vec = aligned16(x) && ld % VW == 0 && cols % VW == 0 && plan.chunk % VW == 0;
  const int64_t units = rows * plan.splits;
  auto go = [&](auto kern) -> int {
    const int grid = full_grid(units);  // one CTA per row chunk
    kern<<<grid, kBlock, 0, stream>>>(x, ld, rows, cols, plan.splits, plan.chunk, out,
                                      out_dtype, parts, tickets);
    return launch_status();
  };
  if (vec) return go(reduce_rows_kernel<T, P, FINAL, true>);
  return go(reduce_rows_kernel<T, P, FINAL, false>);
}

bool float_out_ok(int out_dtype) { return is_float_dtype(out_dtype); }

template <int FINAL>
int float_reduce_entry(const void* x, int64_t ld, int64_t rows, int64_t cols, void* out,
                       int in_dtype, int out_dtype, void* ws, size_t ws_bytes,
                       cudaStream_t stream) {
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x || cols == 0);
  FLB_CHECK_ARG(out && ld >= cols);
  if ((in_dtype == FL_B200_I32 || in_dtype == FL_B200_I64) && FINAL == kFinalSum &&
      out_dtype == FL_B200_I64) {
    if (cols == 0) return cudaMemsetAsync(out, 0, rows * 8, stream) == cudaSuccess
                              ? FL_B200_OK : FL_B200_ERR_LAUNCH;
    if (in_dtype == FL_B200_I64)
      return launch_reduce<int64_t, IntSumPolicy, kFinalI64>(
          static_cast<const int64_t*>(x), ld, rows, cols, out, out_dtype, ws, ws_bytes, stream);
    return launch_reduce<int32_t, IntSumPolicy, kFinalI64>(
        static_cast<const int32_t*>(x), ld, rows, cols, out, out_dtype, ws, ws_bytes, stream);
  }
  if (!is_float_dtype(in_dtype) || !float_out_ok(out_dtype)) return FL_B200_ERR_UNSUPPORTED_DTYPE;
  FLB_CHECK_ARG(cols > 0 || FINAL != kFinalMax);  // amax of an empty row is an error
  return dispatch_float(in_dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto xp = static_cast<const T*>(x);
    if constexpr (FINAL == kFinalMax)
      return launch_reduce<T, MaxPolicy, FINAL>(xp, ld, rows, cols, out, out_dtype, ws,
                                                ws_bytes, stream);
    else
      return launch_reduce<T, SumPolicy, FINAL>(xp, ld, rows, cols, out, out_dtype, ws,
                                                ws_bytes, stream);
  });
}

// ---- reduction over a middle dim -------------------------------------------
// x dense [outer, n, inner].  A CTA covers 32 consecutive inner positions of
// one outer index; its 8 warps split n and merge in a fixed order.
template <typename T, int OP>
__global__ void __launch_bounds__(kBlock)
reduce_middim_kernel(const T* x, int64_t outer, int64_t n, int64_t inner, void* out,
                     int out_dtype) {
  __shared__ float sm[8][33];
  const int64_t tiles = ceil_div(inner, 32);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t u = blockIdx.x; u < outer * tiles; u += gridDim.x) {
    const int64_t o = u / tiles;
    const int64_t i = (u - o * tiles) * 32 + lane;
    float acc = OP == 2 ? -INFINITY : 0.f;
    if (i < inner) {
      const T* xc = x + o * n * inner + i;
      for (int64_t k = warp; k < n; k += 8) {
        const float v = Elem<T>::to_f(xc[k * inner]);
        acc = OP == 2 ? MaxOp::combine(acc, v) : acc + v;
      }
    }
    sm[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && i < inner) {
      float r = sm[0][lane];
      for (int w = 1; w < 8; ++w) r = OP == 2 ? MaxOp::combine(r, sm[w][lane]) : r + sm[w][lane];
      if (OP == 1) r = r / (float)n;
      store_float(out, o * inner + i, out_dtype, r);
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace flb200

extern "C" {

using namespace flb200;

FL_B200_API size_t fl_b200_reduce_workspace_size(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return make_plan(rows, cols).ws_bytes;
}

FL_B200_API int fl_b200_reduce_sum_lastdim(const void* x, int64_t ld, int64_t rows,
                                           int64_t cols, void* out, int in_dtype,
                                           int out_dtype, void* workspace,
                                           size_t workspace_bytes, fl_b200_stream_t stream) {
  return float_reduce_entry<kFinalSum>(x, ld, rows, cols, out, in_dtype, out_dtype,
                                       workspace, workspace_bytes,
                                       static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_mean_lastdim(const void* x, int64_t ld, int64_t rows,
                                            int64_t cols, void* out, int in_dtype,
                                            int out_dtype, void* workspace,
                                            size_t workspace_bytes,
                                            fl_b200_stream_t stream) {
  if (in_dtype == FL_B200_I32) return FL_B200_ERR_UNSUPPORTED_DTYPE;  // torch: mean of int errors
  return float_reduce_entry<kFinalMean>(x, ld, rows, cols, out, in_dtype, out_dtype,
                                        workspace, workspace_bytes,
                                        static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_amax_lastdim(const void* x, int64_t ld, int64_t rows,
                                            int64_t cols, void* out, int dtype,
                                            void* workspace, size_t workspace_bytes,
                                            fl_b200_stream_t stream) {
  return float_reduce_entry<kFinalMax>(x, ld, rows, cols, out, dtype, dtype, workspace,
                                       workspace_bytes, static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_sum_all(const void* x, int64_t n, void* out, int in_dtype,
                                       int out_dtype, void* workspace,
                                       size_t workspace_bytes, fl_b200_stream_t stream) {
  FLB_CHECK_ARG(n >= 0);
  return float_reduce_entry<kFinalSum>(x, n, 1, n, out, in_dtype, out_dtype, workspace,
                                       workspace_bytes, static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_mean_all(const void* x, int64_t n, void* out, int in_dtype,
                                        int out_dtype, void* workspace,
                                        size_t workspace_bytes, fl_b200_stream_t stream) {
  FLB_CHECK_ARG(n >= 0);
  if (in_dtype == FL_B200_I32) return FL_B200_ERR_UNSUPPORTED_DTYPE;
  return float_reduce_entry<kFinalMean>(x, n, 1, n, out, in_dtype, out_dtype, workspace,
                                        workspace_bytes, static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_amax_all(const void* x, int64_t n, void* out, int dtype,
                                        void* workspace, size_t workspace_bytes,
                                        fl_b200_stream_t stream) {
  FLB_CHECK_ARG(n >= 0);
  return float_reduce_entry<kFinalMax>(x, n, 1, n, out, dtype, dtype, workspace,
                                       workspace_bytes, static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_reduce_middim(const void* x, int64_t outer, int64_t n,
                                      int64_t inner, void* out, int op, int in_dtype,
                                      int out_dtype, fl_b200_stream_t stream) {
  FLB_CHECK_ARG(outer >= 0 && n >= 0 && inner >= 0 && op >= 0 && op <= 2);
  if (outer == 0 || inner == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && out);
  FLB_CHECK_ARG(n > 0 || op != 2);
  if (!is_float_dtype(out_dtype)) return FL_B200_ERR_UNSUPPORTED_DTYPE;
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_float(in_dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    auto run = [&](auto kern) -> int {
      const int grid = full_grid(outer * ceil_div(inner, 32));
      kern<<<grid, kBlock, 0, s>>>(static_cast<const T*>(x), outer, n, inner, out,
                                   out_dtype);
      return launch_status();
    };
    if (op == 0) return run(reduce_middim_kernel<T, 0>);
    if (op == 1) return run(reduce_middim_kernel<T, 1>);
    return run(reduce_middim_kernel<T, 2>);
  });
}

FL_B200_API int fl_b200_argmax_lastdim(const void* x, int64_t ld, int64_t rows,
                                       int64_t cols, int64_t* out, int dtype,
                                       void* workspace, size_t workspace_bytes,
                                       fl_b200_stream_t stream) {
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0) return FL_B200_OK;
  FLB_CHECK_ARG(cols > 0 && x && out && ld >= cols);
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return launch_reduce<T, ArgMaxPolicy, kFinalIdx>(static_cast<const T*>(x), ld, rows,
                                                     cols, out, FL_B200_I64, workspace,
                                                     workspace_bytes, s);
  });
}

FL_B200_API int fl_b200_sum_i32_i64(const int32_t* x, int64_t ld, int64_t rows,
                                    int64_t cols, int64_t* out, int full, void* workspace,
                                    size_t workspace_bytes, fl_b200_stream_t stream) {
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  auto s = static_cast<cudaStream_t>(stream);
  if (full) {
    FLB_CHECK_ARG(out);
    if (rows == 0 || cols == 0)
      return cudaMemsetAsync(out, 0, 8, s) == cudaSuccess ? FL_B200_OK : FL_B200_ERR_LAUNCH;
    // The whole block is one row only when it is dense.
    FLB_CHECK_ARG(ld == cols || rows == 1);
    return float_reduce_entry<kFinalSum>(x, rows * cols, 1, rows * cols, out, FL_B200_I32,
                                         FL_B200_I64, workspace, workspace_bytes, s);
  }
  return float_reduce_entry<kFinalSum>(x, ld, rows, cols, out, FL_B200_I32, FL_B200_I64,
                                       workspace, workspace_bytes, s);
}

}  // extern "C"

// ---- full-tensor sum without any allocation ---------------------------------
// The partials of fl_b200_reduce_sum_all_noalloc live here.  In host code the
// name g_noalloc_scratch is only a host-side stand-in for the symbol, never a
// device address: the device address is looked up per device with
// cudaGetSymbolAddress and passed to the kernel like a caller's workspace.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FL_B200_NOALLOC_SCRATCH_BYTES];

namespace flb200 {
namespace {

constexpr int kNoallocMaxDevices = 64;
std::atomic<void*> g_noalloc_addr[kNoallocMaxDevices];
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device (looked up on
// the first call per device, with that device current, then cached).
int noalloc_scratch(void** addr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) {
    if (e != cudaSuccess) set_last_cuda_error(e);
    (void)cudaGetLastError();
    return FL_B200_ERR_NO_DEVICE;
  }
  void* p = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    p = g_noalloc_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr) {
        set_last_cuda_error(e);
        (void)cudaGetLastError();
        return FL_B200_ERR_LAUNCH;
      }
      g_noalloc_addr[dev].store(p, std::memory_order_release);
    }
  }
  *addr = p;
  return FL_B200_OK;
}

}  // namespace
}  // namespace flb200

extern "C" FL_B200_API int fl_b200_reduce_sum_all_noalloc(const void* x, int64_t n,
                                                          void* out, int in_dtype,
                                                          int out_dtype,
                                                          fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n >= 0);
  // The split this sum will use must fit the fixed scratch.
  const Plan plan = make_plan(1, n);
  if (plan.ws_bytes > (size_t)FL_B200_NOALLOC_SCRATCH_BYTES) return FL_B200_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if (plan.ws_bytes > 0) {
    const int st = noalloc_scratch(&scratch);
    if (st != FL_B200_OK) return st;
  }
  // Same kernel and split as fl_b200_reduce_sum_all; the scratch stands in for
  // the caller's workspace (its ticket counters are zeroed on the stream).
  return float_reduce_entry<kFinalSum>(x, n, 1, n, out, in_dtype, out_dtype, scratch,
                                       FL_B200_NOALLOC_SCRATCH_BYTES,
                                       static_cast<cudaStream_t>(stream));
}
