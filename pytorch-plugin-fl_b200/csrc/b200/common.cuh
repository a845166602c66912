// Shared device-side helpers of libfl_b200.so (sm_100a).
//
// Every kernel in this library is a memory-bound row-wise pass: the helpers
// here are the 128-bit packed loads/stores, the bf16/f16 <-> fp32 unpacking,
// the warp / CTA reductions and the per-device launch geometry cache.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>
#include <utility>

#include "../../../include/fl_b200.h"

namespace flb200 {

// ---------------------------------------------------------------- status --

// Records the CUDA error of the last failed call on this thread.
void set_last_cuda_error(cudaError_t e);

// Checks the launch that was just issued; converts a CUDA error to a status.
int launch_status();

// Per-device geometry, cached on first use (thread-safe).
struct DeviceInfo {
  int sm_count;
  int max_smem_optin;
};
// Fills *info for the current device; returns FL_B200_OK or an error.
int current_device_info(DeviceInfo* info);

#define FLB_CHECK_ARG(cond) \
  do {                      \
    if (!(cond)) return FL_B200_ERR_INVALID_ARGUMENT; \
  } while (0)

// ------------------------------------------------------------ dtype traits --

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte pack
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) {
    return __bfloat162float(v);
  }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) {
    return __float2bfloat16_rn(v);
  }
};
template <>
struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) {
    return __float2half_rn(v);
  }
};

// Rounds an fp32 value to T and back (the effect of storing an intermediate
// result in a T tensor, as an op-by-op chain does).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}
template <>
__device__ __forceinline__ float round_to<float>(float v) {
  return v;
}

// ------------------------------------------------------- packed 16-byte I/O --

// Streaming load: data read exactly once, keep it out of L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}
// Cached read-only load: small operands re-read by many rows (weights, tables).
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
// Plain coherent load (used where the same kernel may write the location).
__device__ __forceinline__ uint4 ld_plain(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
// Streaming store: written once, not re-read by this kernel.
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// 32-byte accesses (ld/st.global .v8.b32, sm_100): half the memory
// instructions of two 16-byte ones.  Both need 32-byte aligned addresses.
// Measured on B200 inside the 32-layer stack under the 1 kW power cap, the
// SwiGLU pass streams at 7.07 TB/s with these against 6.71 TB/s with 16-byte
// accesses.
struct Pack32 {
  uint4 lo, hi;
};
__device__ __forceinline__ Pack32 ld_stream32(const void* p) {
  Pack32 r;
  asm("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r.lo.x), "=r"(r.lo.y), "=r"(r.lo.z), "=r"(r.lo.w), "=r"(r.hi.x), "=r"(r.hi.y),
        "=r"(r.hi.z), "=r"(r.hi.w)
      : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream32(void* p, const Pack32& v) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p),
               "r"(v.lo.x), "r"(v.lo.y), "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y),
               "r"(v.hi.z), "r"(v.hi.w)
               : "memory");
}
inline bool aligned32(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 31u) == 0;
}

// 16-byte asynchronous copy global -> shared (cp.async, bypassing L1) and
// its group commit / wait (the wait returns once this thread's committed
// copies have landed: a hardware wait on the thread's own copies).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
// Returns once at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_pending() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Makes a pack opaque to the optimizer: after this the compiler cannot reuse
// fp32 values it unpacked from `v` earlier, so a kernel that walks a row held
// in registers twice keeps it packed (4 registers per 16 bytes) instead of
// holding every unpacked fp32 value live between the passes.
__device__ __forceinline__ uint4 opaque(uint4 v) {
  asm volatile("" : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w));
  return v;
}

// Unpack a 16-byte pack of T into fp32 values.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float (&f)[Elem<T>::kVec]);

template <>
__device__ __forceinline__ void unpack<float>(const uint4& u, float (&f)[4]) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
  // bf16 -> fp32 is exact: the 16 bits become the high half of the fp32 word.
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack<__half>(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 v = __half22float2(h);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// Pack fp32 values into a 16-byte pack of T (round to nearest even).
template <typename T>
__device__ __forceinline__ uint4 pack(const float (&f)[Elem<T>::kVec]);

template <>
__device__ __forceinline__ uint4 pack<float>(const float (&f)[4]) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                    __float_as_uint(f[2]), __float_as_uint(f[3]));
}
template <>
__device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 pack<__half>(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------ fp32 pairs ---------
// sm_100 runs fma / add / mul on two fp32 values held in a 64-bit register
// pair with one instruction (PTX .f32x2); each lane is rounded exactly like
// the scalar instruction (.rn, no contraction across the explicit ops), so
// results equal fmaf / __fadd_rn / __fmul_rn lane by lane.
__device__ __forceinline__ uint64_t f2_make(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t r) {
  float lo;
  asm("{ .reg .f32 t; mov.b64 {%0, t}, %1; }" : "=f"(lo) : "l"(r));
  return lo;
}
__device__ __forceinline__ float f2_hi(uint64_t r) {
  float hi;
  asm("{ .reg .f32 t; mov.b64 {t, %0}, %1; }" : "=f"(hi) : "l"(r));
  return hi;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// A pair as the 32-bit word of two 16-bit T values (round to nearest even,
// one cvt.rn.{bf16x2,f16x2}.f32; lo in the low half, as in memory) and back.
template <typename T>
__device__ __forceinline__ uint32_t pair_to_bits(uint64_t p) {
  static_assert(!std::is_same<T, float>::value, "16-bit types only");
  const float lo = f2_lo(p), hi = f2_hi(p);
  uint32_t h;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
  }
  return h;
}
template <typename T>
__device__ __forceinline__ uint64_t pair_from_bits(uint32_t h) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return f2_make(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u));
  } else {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&h));
    return f2_make(v.x, v.y);
  }
}
// Rounds both lanes of a pair to T and back (round_to<T> on each lane), two
// values per conversion instruction.
template <typename T>
__device__ __forceinline__ uint64_t round_pair(uint64_t p) {
  if constexpr (std::is_same<T, float>::value) {
    return p;
  } else {
    return pair_from_bits<T>(pair_to_bits<T>(p));
  }
}
// Max of three fp32 values in one instruction (sm_100); NaN inputs are
// ignored unless all are NaN, as with fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---------------------------------------------------------- reductions ------

struct SumOp {
  __device__ __forceinline__ static float identity() { return 0.f; }
  __device__ __forceinline__ static float combine(float a, float b) { return a + b; }
};
// NaN-propagating max (torch max/amax semantics): NaN wins over everything.
struct MaxOp {
  __device__ __forceinline__ static float identity() { return -INFINITY; }
  __device__ __forceinline__ static float combine(float a, float b) {
    return (a != a || a > b) ? a : b;  // a NaN -> a; b NaN -> b (a > NaN false)
  }
};
// Plain max that ignores the order of NaN (used where NaN cannot change the
// final result, e.g. the softmax row max: a NaN anywhere makes the sum NaN).
struct FastMaxOp {
  __device__ __forceinline__ static float identity() { return -INFINITY; }
  __device__ __forceinline__ static float combine(float a, float b) {
    return fmaxf(a, b);
  }
};

// Butterfly reduction among the GROUP consecutive lanes that own one row
// (GROUP a power of two <= 32); every lane of the group gets the result.
template <typename Op, int GROUP>
__device__ __forceinline__ float group_reduce_warp(float v) {
#pragma unroll
  for (int off = GROUP / 2; off > 0; off >>= 1)
    v = Op::combine(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Reduction among the TPR threads [row_slot*TPR, (row_slot+1)*TPR) of a CTA.
// For TPR <= 32 it is a warp butterfly; for TPR > 32 the per-warp results go
// through shared memory `smem` (>= BLOCK/32 floats) and EVERY thread of the
// CTA must call this (it contains __syncthreads).
template <typename Op, int TPR, int BLOCK>
__device__ __forceinline__ float row_reduce(float v, float* smem) {
  if constexpr (TPR <= 32) {
    return group_reduce_warp<Op, TPR>(v);
  } else {
    constexpr int kWarpsPerRow = TPR / 32;
    v = group_reduce_warp<Op, 32>(v);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    __syncthreads();  // smem may still be read by a previous reduction
    if (lane == 0) smem[warp] = v;
    __syncthreads();
    const int first = (warp / kWarpsPerRow) * kWarpsPerRow;
    float r = smem[first];
#pragma unroll
    for (int i = 1; i < kWarpsPerRow; ++i) r = Op::combine(r, smem[first + i]);
    return r;
  }
}

// Sums of a and b over the TPR threads of a row (TPR a multiple of 32, the
// row's warps consecutive, BLOCK / TPR <= 15 rows per CTA) with one barrier
// of the row's own warps instead of CTA-wide ones: each warp's pair of sums
// goes to its slot of `buf` (float2[2 * BLOCK / 32], two halves used by
// alternate rows through `parity`), the row's warps meet at named barrier
// 1 + row slot, and every thread adds the row's partials in warp order (so
// all of them get the same sums).  The halves alternate so that a warp's
// write for its next row cannot overwrite values its partners still read:
// they have passed the barrier of the row in between.
template <int TPR, int BLOCK>
__device__ __forceinline__ void row_sum2_named(float& a, float& b, float2* buf, int parity) {
  static_assert(TPR % 32 == 0 && BLOCK / TPR <= 15, "row_sum2_named geometry");
  constexpr int W = TPR / 32;
  a = group_reduce_warp<SumOp, 32>(a);
  b = group_reduce_warp<SumOp, 32>(b);
  const int warp = threadIdx.x >> 5;
  const int slot = threadIdx.x / TPR;
  float2* half = buf + parity * (BLOCK / 32);
  if ((threadIdx.x & 31) == 0) half[warp] = make_float2(a, b);
  asm volatile("bar.sync %0, %1;" ::"r"(1 + slot), "r"(TPR) : "memory");
  const float2* row = half + slot * W;
  float2 t = row[0];
#pragma unroll
  for (int i = 1; i < W; ++i) {
    t.x += row[i].x;
    t.y += row[i].y;
  }
  a = t.x;
  b = t.y;
}

// Whole-CTA reduction; the result is valid in every thread.
template <typename Op, int BLOCK>
__device__ __forceinline__ float block_reduce(float v, float* smem) {
  return row_reduce<Op, BLOCK, BLOCK>(v, smem);
}

// ----------------------------------------------------------- misc helpers ---

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

inline int dtype_size(int dtype) {
  switch (dtype) {
    case FL_B200_F32: return 4;
    case FL_B200_BF16: return 2;
    case FL_B200_F16: return 2;
    case FL_B200_I32: return 4;
    case FL_B200_I64: return 8;
    default: return 0;
  }
}

inline bool is_float_dtype(int dtype) {
  return dtype == FL_B200_F32 || dtype == FL_B200_BF16 || dtype == FL_B200_F16;
}

// Calls f(T{}) with T the C++ element type of a float dtype; returns
// FL_B200_ERR_UNSUPPORTED_DTYPE for anything else.
template <typename F>
int dispatch_float(int dtype, F&& f) {
  switch (dtype) {
    case FL_B200_F32: return f(float{});
    case FL_B200_BF16: return f(__nv_bfloat16{});
    case FL_B200_F16: return f(__half{});
    default: return FL_B200_ERR_UNSUPPORTED_DTYPE;
  }
}

// Number of CTAs of `kernel` (launched with `block` threads and `smem` bytes
// of dynamic shared memory) that fit on one SM.  Cached per kernel by the
// caller through a function-local static.
template <typename K>
int blocks_per_sm(K kernel, int block, size_t smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, block, smem) !=
          cudaSuccess ||
      n < 1) {
    (void)cudaGetLastError();
    n = 1;
  }
  return n;
}

// ------------------------------------------- programmatic dependent launch --
// Kernels of this library may be launched with programmatic stream
// serialization (PDL): such a launch can begin while the previous kernel in
// the stream is still running, as soon as every CTA of that kernel has
// started.  Its CTAs then become resident as the previous kernel's CTAs
// retire and wait in griddepcontrol.wait, which returns once the previous
// grid has completed and its memory operations are visible; so a kernel's
// launch latency and CTA rasterisation overlap the previous kernel's tail.
// Every kernel calls pdl_prologue() before its first global memory access
// (read or write), which makes the overlap safe for any producer/consumer
// order.  Launched without the attribute, both instructions return at once.
__device__ __forceinline__ void pdl_prologue() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Dependents may launch as soon as every CTA of this grid has passed here.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// True when launches use programmatic stream serialization (fl_b200_set_pdl;
// FL_B200_PDL=0 in the environment turns it off at load).
bool pdl_enabled();

// Launches `kern` on `stream`, with programmatic stream serialization when
// pdl_enabled().  A launch error is left for launch_status() to report.
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// One CTA per work unit ("full grid").  Measured on B200 for every streaming
// kernel here, a full grid of short-lived CTAs streams HBM faster than a
// persistent grid-stride loop (SwiGLU 7.1 vs 5.9 TB/s at 131072 x 14336
// bf16).  The kernels keep their grid-stride loops, so the cap at the
// largest grid dimension only lengthens the loop.
inline int full_grid(int64_t units) {
  return (int)std::min<int64_t>(std::max<int64_t>(units, 1), 0x7fffffff);
}

// Grid size for a grid-stride kernel over `units` work units: enough CTAs to
// fill every SM at the kernel's occupancy, never more than there are units.
template <typename K>
int persistent_grid(K kernel, int block, size_t smem, int64_t units,
                    const DeviceInfo& dev) {
  const int per_sm = blocks_per_sm(kernel, block, smem);
  int64_t g = (int64_t)per_sm * dev.sm_count;
  if (g > units) g = units;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace flb200
