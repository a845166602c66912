// Softmax with fp32 accumulation; last-dim (optionally causal) and middle-dim.
//
// Reference behaviour: _softmax(self, dim, half_to_float) (register.cc:
// 270-272 -> csrc/aten/backends/cuda/softmax.cc:14-40, PyTorch's host_softmax)
// on logits that HF has already masked (modeling_qwen3.py:209-213).  The
// causal variant applies the mask itself: masked keys are never read and are
// written as exact zeros, so a causal row of L keys costs (i+1)/L of a read.
//
// exp(x - m) is evaluated as exp2f(x*log2e - m*log2e) with one FMA (rows
// whose max is too far below zero for that are shifted by it first, exactly,
// wide_max); the row stays in registers (row_ladder), so HBM sees one read
// and one write.
//
// softmax_masked is HF's eager-attention tail in one pass
// (modeling_qwen3.py eager_attention_forward: `w * scaling + mask`,
// softmax(dtype=float32), `.to(query.dtype)`): scale, additive mask
// broadcast over heads, softmax, and the cast of the result.
#include "row_ladder.cuh"

namespace flb200 {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// 2^t with the PTX instruction ex2.approx.ftz.f32 (relative error about
// 2^-22 over the fp32 normal range; results below it flush to +0, inputs
// -inf -> +0, NaN -> NaN).
__device__ __forceinline__ float ex2_approx(float t) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(t));
  return r;
}

// exp(x - m) as 2^(x*log2e - m*log2e), one FMA and one ex2.
__device__ __forceinline__ float exp_shifted(float x, float mlog2e) {
  return ex2_approx(fmaf(x, kLog2e, -mlog2e));
}

// Pair k of a 16-byte pack as fp32 (elements 2k and 2k+1).
template <typename T>
__device__ __forceinline__ uint64_t pack_pair(const uint4& v, int k) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (std::is_same<T, float>::value) {
    return f2_make(__uint_as_float(w[2 * k]), __uint_as_float(w[2 * k + 1]));
  } else {
    return pair_from_bits<T>(w[k]);
  }
}

// A row max too far below zero for the one-FMA exp: m*log2e overflows to
// -inf for a finite m below -2.36e38, e.g. a row whose every key is masked
// with the lowest finite value (HF's additive attention mask for a padding
// query).  Every key x of such a row lies in [-3.41e38, m], within a factor
// of 2 of m, so x - m is exact in the row's own format (Sterbenz's lemma):
// the register-resident kernels subtract m from their packs once (a
// row-uniform branch that ordinary rows never take) and continue with m = 0,
// so the row comes out uniform over its keys as in the reference, not NaN.
__device__ __forceinline__ bool wide_max(float m) {
  return m * kLog2e == -INFINITY && m != -INFINITY;
}
template <typename T>
__device__ __forceinline__ uint4 shift_pack(const uint4& v, float m) {
  constexpr int VW = Elem<T>::kVec;
  float f[VW];
  unpack<T>(v, f);
#pragma unroll
  for (int e = 0; e < VW; ++e) f[e] -= m;
  return pack<T>(f);
}

// The same for the middle-dim kernel, which reads its column again instead
// of keeping it: exp(x - m) in the one-FMA form, or x - m first for a wide
// row.  Its sum and its outputs take the same form, so the factor
// 2^(rounding error of m*log2e) common to a row's exps cancels.
struct RowShift {
  float m, ml;
  bool wide;
  __device__ __forceinline__ explicit RowShift(float row_max)
      : m(row_max), ml(row_max * kLog2e), wide(wide_max(row_max)) {}
  __device__ __forceinline__ float exp(float x) const {
    return wide ? ex2_approx((x - m) * kLog2e) : exp_shifted(x, ml);
  }
};

// Max of a 16-byte pack as fp32, NaN ignored like fmaxf (a NaN anywhere in
// the row still makes every output NaN through its exp).  16-bit packs use
// the packed max.bf16x2 / max.f16x2 instructions: 3 for 8 elements.
template <typename T>
__device__ __forceinline__ float pack_max(const uint4& u) {
  if constexpr (std::is_same<T, float>::value) {
    return fmaxf(fmaxf(__uint_as_float(u.x), __uint_as_float(u.y)),
                 fmaxf(__uint_as_float(u.z), __uint_as_float(u.w)));
  } else {
    uint32_t a, b, m;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      asm("max.bf16x2 %0, %1, %2;" : "=r"(a) : "r"(u.x), "r"(u.y));
      asm("max.bf16x2 %0, %1, %2;" : "=r"(b) : "r"(u.z), "r"(u.w));
      asm("max.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(a), "r"(b));
      return fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
    } else {
      asm("max.f16x2 %0, %1, %2;" : "=r"(a) : "r"(u.x), "r"(u.y));
      asm("max.f16x2 %0, %1, %2;" : "=r"(b) : "r"(u.z), "r"(u.w));
      asm("max.f16x2 %0, %1, %2;" : "=r"(m) : "r"(a), "r"(b));
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&m));
      return fmaxf(v.x, v.y);
    }
  }
}

// Calls f(integral_constant<int, k>) for the runtime count k, a multiple of
// STEP in [N, MAX]: a chain of compares on a value uniform over a row's
// threads, so a causal row runs code for its visible pack iterations only,
// with every register array still indexed by constants.  Only multiples of
// STEP are instantiated (fewer code paths for the instruction cache).
template <int N, int MAX, int STEP, typename F>
__device__ __forceinline__ void with_count(int k, F& f) {
  if constexpr (N <= MAX) {
    if (k == N) {
      f(std::integral_constant<int, N>{});
      return;
    }
    with_count<N + STEP, MAX, STEP>(k, f);
  }
}

// Stores VW fp32 values (one input pack's worth) as TO at `o`.  W32: eight
// fp32 outputs of a 16-bit pack go out as one 32-byte store (o 32-byte
// aligned), half the store instructions of two 16-byte stores; measured on
// B200 for fp32-output softmax: 6.65-6.92 vs 5.36-5.61 TB/s.
template <typename TO, int VW, bool W32 = false>
__device__ __forceinline__ void store_vals(TO* o, const float (&v)[VW]) {
  if constexpr (W32) {
    static_assert(std::is_same<TO, float>::value && VW == 8, "32-byte stores: 8 fp32 values");
    Pack32 p;
    p.lo = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                      __float_as_uint(v[3]));
    p.hi = make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]),
                      __float_as_uint(v[7]));
    st_stream32(o, p);
    return;
  }
  constexpr int OW = Elem<TO>::kVec;
  static_assert(VW % OW == 0, "input pack must cover whole output packs");
#pragma unroll
  for (int c = 0; c < VW / OW; ++c) {
    float t[OW];
#pragma unroll
    for (int e = 0; e < OW; ++e) t[e] = v[c * OW + e];
    st_stream(o + c * OW, pack<TO>(t));
  }
}

// Sets elements [keep, VW) of a pack to -inf (the masked tail of a causal row).
template <typename T>
__device__ __forceinline__ uint4 mask_tail(uint4 v, int keep);
template <>
__device__ __forceinline__ uint4 mask_tail<float>(uint4 v, int keep) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (e >= keep) w[e] = 0xff800000u;
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <uint16_t NEG_INF>
__device__ __forceinline__ uint4 mask_tail16(uint4 v, int keep) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (2 * i >= keep) w[i] = (w[i] & 0xffff0000u) | NEG_INF;
    if (2 * i + 1 >= keep) w[i] = (w[i] & 0x0000ffffu) | ((uint32_t)NEG_INF << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ uint4 mask_tail<__nv_bfloat16>(uint4 v, int keep) {
  return mask_tail16<0xff80>(v, keep);
}
template <>
__device__ __forceinline__ uint4 mask_tail<__half>(uint4 v, int keep) {
  return mask_tail16<0xfc00>(v, keep);
}

// Resident CTAs per SM the register budget is set for.  A causal row reads
// only its visible keys, so each row has fewer bytes in flight than a plain
// one; causal rows therefore keep no fp32 exps in registers (they evaluate
// exp again when storing: one ex2 per element on average, since about half
// the keys are masked) and run twice as many rows per SM (<= 64 registers at
// 256 threads).
template <int BLOCK, bool CAUSAL, int VPT>
constexpr int softmax_min_blocks() {
  return CAUSAL ? (BLOCK <= 256 ? 4 : 1024 / BLOCK) : ladder_min_blocks<BLOCK>();
}

// Plain rows keep their fp32 exps in registers for the store pass (one ex2
// per element) up to 8 packs per thread.  The 16-pack rung (one warp per row
// of 257..512 packs, e.g. 4096 f16 keys) evaluates exp again when storing
// instead: no cross-warp reduction, twice the bytes in flight per warp;
// measured on B200, f16 [8x32x4096, 4096] 6.97 vs 5.96 TB/s.
template <bool CAUSAL, int VPT>
__host__ __device__ constexpr bool keeps_exps() {
  return !CAUSAL && VPT <= 8;
}

// Masked keys are loaded as -inf, so the max ignores them, their exp is an
// exact 0 and a row with no visible key comes out NaN (-inf - -inf), with no
// per-element masks in the arithmetic.
template <typename TI, typename TO, int TPR, int VPT, int BLOCK, bool CAUSAL, bool W32>
__global__ void __launch_bounds__(BLOCK, (softmax_min_blocks<BLOCK, CAUSAL, VPT>()))
softmax_vec_kernel(const TI* x, int64_t ldx, TO* y, int64_t ldy, int64_t rows,
                   int64_t cols, int64_t q_len, int64_t offset) {
  constexpr int VW = Elem<TI>::kVec;
  constexpr int RPB = BLOCK / TPR;
  __shared__ float smem[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const int nvec = (int)(cols / VW);
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows;
       base += (int64_t)gridDim.x * RPB) {
    const int64_t row = base + slot;
    const bool ok = row < rows;
    // Visible keys of this row, clamped to [0, cols].
    int nvalid = (int)cols;
    if (CAUSAL) nvalid = (int)max((int64_t)0, min(cols, (row % q_len) + offset + 1));
    const TI* xr = x + row * ldx;
    // Pack iterations i >= `iters` lie wholly past a causal row's last
    // visible key for every thread of the row: they are neither loaded nor
    // computed, and store zeros.  Inside the visible iterations a thread
    // whose pack is masked holds -inf (exp 0).  The phases run through
    // with_count, so this costs no predicated-off work; the reductions stay
    // outside it, where every thread of the CTA reaches them.
    // Rows of up to one warp with the input's dtype out dispatch only even
    // counts (one extra iteration over -inf packs at most, which read
    // nothing from HBM and add exact zeros): measured on B200, bf16 causal
    // rows of 2048 keys 6.26 vs 5.82 TB/s; wider rows and fp32 outputs are
    // faster with every count.
    constexpr int STEP = (TPR <= 32 && VPT % 2 == 0 && std::is_same<TI, TO>::value) ? 2 : 1;
    int iters = VPT;
    if constexpr (CAUSAL) {
      iters = (int)min((int64_t)VPT, ceil_div(ceil_div((int64_t)nvalid, VW), TPR));
      if constexpr (STEP == 2) iters = (iters + 1) & ~1;
    }
    uint4 v[VPT];
    float ex[VPT][VW];
    float m = -INFINITY, s = 0.f;
    auto load_max = [&](auto kc) {
      constexpr int K = decltype(kc)::value;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const int j0 = (lane + i * TPR) * VW;
        if (ok && j0 < nvalid) {
          v[i] = ld_stream(xr + j0);
          if (CAUSAL && j0 + VW > nvalid) v[i] = mask_tail<TI>(v[i], nvalid - j0);
        } else {
          v[i] = mask_tail<TI>(make_uint4(0, 0, 0, 0), 0);
        }
      }
#pragma unroll
      for (int i = 0; i < K; ++i) m = fmaxf(m, pack_max<TI>(v[i]));
    };
    // exp(x - m) per element, each pack summed as a tree; plain rows keep the
    // exps in fp32 registers for the store pass (one ex2 per element).
    const auto exp_sum = [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      const float ml = m * kLog2e;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float f[VW], t[VW];
        unpack<TI>(opaque(v[i]), f);
#pragma unroll
        for (int e = 0; e < VW; ++e) t[e] = exp_shifted(f[e], ml);
        if constexpr (keeps_exps<CAUSAL, VPT>()) {
#pragma unroll
          for (int e = 0; e < VW; ++e) ex[i][e] = t[e];
        }
#pragma unroll
        for (int w = VW / 2; w >= 1; w /= 2)
#pragma unroll
          for (int e = 0; e < w; ++e) t[e] += t[e + w];
        s += t[0];
      }
    };
    TO* yr = y + row * ldy;
    const auto store = [&](auto kc) {
      constexpr int K = decltype(kc)::value;
      const float inv = 1.0f / s;
      const float ml = m * kLog2e;
#pragma unroll
      for (int i = 0; i < K; ++i) {
        const int vi = lane + i * TPR;
        if (!ok || vi >= nvec) continue;
        float o[VW];
        if constexpr (!keeps_exps<CAUSAL, VPT>()) {
          unpack<TI>(opaque(v[i]), o);
#pragma unroll
          for (int e = 0; e < VW; ++e) o[e] = exp_shifted(o[e], ml) * inv;
        } else {
#pragma unroll
          for (int e = 0; e < VW; ++e) o[e] = ex[i][e] * inv;
        }
        store_vals<TO, VW, W32>(yr + (int64_t)vi * VW, o);
      }
      // Masked keys: exp = 0, so 0 * inv (NaN for a row with no visible key).
      float z[VW];
#pragma unroll
      for (int e = 0; e < VW; ++e) z[e] = 0.f * inv;
#pragma unroll
      for (int i = K; i < VPT; ++i) {
        const int vi = lane + i * TPR;
        if (ok && vi < nvec) store_vals<TO, VW, W32>(yr + (int64_t)vi * VW, z);
      }
    };
    using Full = std::integral_constant<int, VPT>;
    if constexpr (CAUSAL) with_count<0, VPT, STEP>(iters, load_max);
    else load_max(Full{});
    m = row_reduce<FastMaxOp, TPR, BLOCK>(m, smem);
    if (wide_max(m)) {
      const auto shift = [&](auto kc) {
#pragma unroll
        for (int i = 0; i < decltype(kc)::value; ++i) v[i] = shift_pack<TI>(v[i], m);
      };
      if constexpr (CAUSAL) with_count<0, VPT, STEP>(iters, shift);
      else shift(Full{});
      m = 0.f;
    }
    if constexpr (CAUSAL) with_count<0, VPT, STEP>(iters, exp_sum);
    else exp_sum(Full{});
    s = row_reduce<SumOp, TPR, BLOCK>(s, smem);
    if constexpr (CAUSAL) with_count<0, VPT, STEP>(iters, store);
    else store(Full{});
  }
}

// Any row length / alignment: one CTA per row; per-thread online max/sum,
// then a CTA combine; the row is read twice (the second read mostly from L2).
template <typename TI, typename TO, bool CAUSAL>
__global__ void __launch_bounds__(256)
softmax_loop_kernel(const TI* x, int64_t ldx, TO* y, int64_t ldy, int64_t rows,
                    int64_t cols, int64_t q_len, int64_t offset) {
  __shared__ float smem[256 / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    int64_t nvalid = cols;
    if (CAUSAL) nvalid = min(cols, (row % q_len) + offset + 1);
    const TI* xr = x + row * ldx;
    float m = -INFINITY, s = 0.f;
    for (int64_t c = threadIdx.x; c < nvalid; c += 256) {
      const float f = Elem<TI>::to_f(xr[c]);
      if (f > m) {
        s = s * exp2f((m - f) * kLog2e) + 1.0f;  // rescale the running sum
        m = f;
      } else if (f != -INFINITY) {  // exp(-inf) adds nothing (and -inf - -inf is NaN)
        s += exp2f((f - m) * kLog2e);
      }
    }
    const float mrow = block_reduce<FastMaxOp, 256>(m, smem);
    // Rescale each thread's partial sum to the row max (empty partials add 0).
    const float part = (m == -INFINITY) ? 0.f : s * exp2f((m - mrow) * kLog2e);
    const float srow = block_reduce<SumOp, 256>(part, smem);
    const float inv = nvalid > 0 ? 1.0f / srow : __int_as_float(0x7fc00000);
    TO* yr = y + row * ldy;
    // the argument the sum was taken of, (x - m) * log2e (see the two-pass
    // kernel below for why not the one-FMA form)
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      float o;
      if (c < nvalid) o = ex2_approx((Elem<TI>::to_f(xr[c]) - mrow) * kLog2e) * inv;
      else o = nvalid > 0 ? 0.f : inv;
      if constexpr (std::is_same<TO, float>::value) yr[c] = o;
      else yr[c] = Elem<TO>::from_f(o);
    }
  }
}

// Rows longer than the register ladder (more than 4096 packs, e.g. a
// vocabulary of 128256 logits), 16-byte aligned: one CTA per row,
// grid-stride over rows; BLOCK threads per row (1024 with one CTA per SM for
// rows over 12288 packs, else 512 with two CTAs per SM when the rows in
// flight fit in 64 MB of L2: measured on B200, bf16 128256-wide rows 3.4 vs
// 2.7 TB/s, bf16 40000-wide rows 3.3 vs 2.8 TB/s the other way round).  Pass 1 reads the row once with 16-byte loads
// (kLongUnroll packs per thread in flight), keeping a running max and a sum
// rescaled when the max rises (x - m first, so a row at the lowest finite
// value needs no special case there); the CTA combines the threads' (max,
// sum); pass 2 reads the row again, from L2 when the rows in flight fit
// there, and writes the probabilities.  Causal rows read their visible keys
// only and store zeros past them.
constexpr int kLongUnroll = 4;

template <typename TI, typename TO, bool CAUSAL, int kLongBlock>
__global__ void __launch_bounds__(kLongBlock, 1024 / kLongBlock)
softmax_long_kernel(const TI* x, int64_t ldx, TO* y, int64_t ldy, int64_t rows, int64_t cols,
                    int64_t q_len, int64_t offset) {
  constexpr int VW = Elem<TI>::kVec;
  constexpr int U = kLongUnroll;
  __shared__ float smem[kLongBlock / 32];
  const int64_t nvec = cols / VW;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    int64_t nvalid = cols;
    if (CAUSAL) nvalid = max((int64_t)0, min(cols, (row % q_len) + offset + 1));
    const int64_t nv = CAUSAL ? ceil_div(nvalid, (int64_t)VW) : nvec;  // packs with a key
    const TI* xr = x + row * ldx;
    const auto masked = [&](uint4 v, int64_t p) {
      if (CAUSAL && p * VW + VW > nvalid) v = mask_tail<TI>(v, (int)(nvalid - p * VW));
      return v;
    };
    constexpr int NP = VW / 2;  // fp32 pairs per pack
    const uint64_t log2e2 = f2_make(kLog2e, kLog2e);
    float m = -INFINITY;
    uint64_t s2 = f2_make(0.f, 0.f);  // the thread's running sum, in two lanes
    const auto consume = [&](uint4 v) {
      const float pm = pack_max<TI>(v);
      if (pm > m) {
        const float r = (m == -INFINITY) ? 0.f : ex2_approx((m - pm) * kLog2e);
        s2 = f2_mul(s2, f2_make(r, r));
        m = pm;
      }
      if (m != -INFINITY) {
        const uint64_t nm2 = f2_make(-m, -m);
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const uint64_t t = f2_mul(f2_add(pack_pair<TI>(v, k), nm2), log2e2);
          s2 = f2_add(s2, f2_make(ex2_approx(f2_lo(t)), ex2_approx(f2_hi(t))));
        }
      }
    };
    int64_t p = threadIdx.x;
    for (; p + (U - 1) * kLongBlock < nv; p += U * kLongBlock) {
      uint4 v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) v[k] = ld_stream(xr + (p + k * kLongBlock) * VW);
#pragma unroll
      for (int k = 0; k < U; ++k) consume(masked(v[k], p + k * kLongBlock));
    }
    for (; p < nv; p += kLongBlock) consume(masked(ld_stream(xr + p * VW), p));
    const float mrow = block_reduce<FastMaxOp, kLongBlock>(m, smem);
    // each thread's sum rescaled to the row max (empty partials add 0)
    const float s = f2_lo(s2) + f2_hi(s2);
    const float part = (m == -INFINITY) ? 0.f : s * ex2_approx((m - mrow) * kLog2e);
    const float srow = block_reduce<SumOp, kLongBlock>(part, smem);
    const float inv = nvalid > 0 ? 1.0f / srow : __int_as_float(0x7fc00000);
    const uint64_t nmrow2 = f2_make(-mrow, -mrow), inv2 = f2_make(inv, inv);
    TO* yr = y + row * ldy;
    // Pass 2: every output from ex2.approx (exact zeros below its range) of
    // (x - m) * log2e.  Pass 1 summed exp2((x - m_thread) * log2e) and rescaled
    // by exp2((m_thread - m) * log2e), so the two agree up to the rounding of
    // that per-thread rescale (a few fp32 ulp of the sum).  The one-FMA form
    // x*log2e - round(m*log2e) would scale every output by 2^(rounding error
    // of m*log2e), up to 2^(|m| * 2^-24), which the sum of pass 1 does not
    // share (0.15 % for a row at the fp16 lowest value).  x - m is exact near
    // the max, also for a max below -2.36e38, so no row needs a shift first.
    // Adds and multiplies in pairs, rounded lane by lane as the scalar ones.
    const auto emit = [&](uint4 v, int64_t q) {
      float o[VW];
      if (!CAUSAL || q < nv) {
        const uint4 u = masked(v, q);
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const uint64_t t = f2_mul(f2_add(pack_pair<TI>(u, k), nmrow2), log2e2);
          const uint64_t r = f2_mul(f2_make(ex2_approx(f2_lo(t)), ex2_approx(f2_hi(t))), inv2);
          o[2 * k] = f2_lo(r);
          o[2 * k + 1] = f2_hi(r);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VW; ++e) o[e] = 0.f * inv;
      }
      store_vals<TO, VW, false>(yr + q * VW, o);
    };
    int64_t q = threadIdx.x;
    for (; q + (U - 1) * kLongBlock < nvec; q += U * kLongBlock) {
      uint4 v[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int64_t qk = q + k * kLongBlock;
        v[k] = (!CAUSAL || qk < nv) ? ld_stream(xr + qk * VW) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) emit(v[k], q + k * kLongBlock);
    }
    for (; q < nvec; q += kLongBlock)
      emit((!CAUSAL || q < nv) ? ld_stream(xr + q * VW) : make_uint4(0, 0, 0, 0), q);
  }
}

// Softmax over the middle dim of a dense [outer, n, inner] view: one thread
// per (outer, inner) column, three passes over n (coalesced across inner).
template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
softmax_middim_kernel(const TI* x, TO* y, int64_t outer, int64_t n, int64_t inner) {
  const int64_t cols = outer * inner;
  for (int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x; t < cols;
       t += (int64_t)gridDim.x * 256) {
    const int64_t o = t / inner, in = t - o * inner;
    const TI* xc = x + o * n * inner + in;
    TO* yc = y + o * n * inner + in;
    float m = -INFINITY;
    for (int64_t k = 0; k < n; ++k) m = fmaxf(m, Elem<TI>::to_f(xc[k * inner]));
    const RowShift sh(m);
    float s = 0.f;
    for (int64_t k = 0; k < n; ++k) s += sh.exp(Elem<TI>::to_f(xc[k * inner]));
    const float inv = 1.0f / s;
    for (int64_t k = 0; k < n; ++k) {
      const float v = sh.exp(Elem<TI>::to_f(xc[k * inner])) * inv;
      if constexpr (std::is_same<TO, float>::value) yc[k * inner] = v;
      else yc[k * inner] = Elem<TO>::from_f(v);
    }
  }
}

// ---- rows split across a thread-block cluster ----------------------------
// Rows of 4097..16384 packs (e.g. a 128256-entry vocabulary of bf16 logits),
// too long for one CTA's registers: a cluster of C = 3..8 CTAs per row
// (cluster size chosen at launch), each CTA holding 512 threads x 4 packs of
// the row.  Each warp takes its max m_w and keeps its exponentials
// exp(x - m_w) in registers (fp32) with their sum s_w; one CTA barrier later
// warp 0 folds the warps' pairs into the CTA's (m_c, s_c) and publishes it
// in shared memory; after one cluster barrier (barrier.cluster) lane r of
// every warp reads CTA r's pair through distributed shared memory (mapa +
// ld.shared::cluster) and the warp combines them, so that every CTA gets the
// same M and S = sum_c s_c 2^((m_c - M) log2e).  The store pass scales the
// held exponentials by exp(m_w - M) / S: one ex2 per key, the row read once.
//
// Persistent clusters walk rows; each CTA keeps kClusterDepth rows of its
// slice in flight (cp.async into shared memory, one commit group per row),
// refilling a row's slots as soon as they are in registers.  The published
// CTA pair alternates between two slots by row parity: a partner cannot
// overwrite slot p (two rows later) before passing the cluster barrier of the
// row in between, which this CTA reaches only after reading slot p.
constexpr int kClusterBlock = 512;
constexpr int kClusterVPT = 4;
constexpr int kClusterPacks = kClusterBlock * kClusterVPT;  // packs per CTA
constexpr int kClusterDepth = 1;  // rows of the slice in flight ahead of use (2 measured slower)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// The float2 at `local` (this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ float2 ld_cluster_f2(const float2* local, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(ra)
               : "memory");
  return v;
}

template <typename TI, typename TO, bool W32>
__global__ void __launch_bounds__(kClusterBlock, 2)
softmax_cluster_kernel(const TI* __restrict__ x, int64_t ldx, TO* __restrict__ y, int64_t ldy,
                       int64_t rows, int nvec) {
  constexpr int VW = Elem<TI>::kVec;
  __shared__ float2 wpart[kClusterBlock / 32];
  __shared__ float2 part[2];
  extern __shared__ uint4 stage[];  // [kClusterDepth][pack][thread], 32 KB a row
  const uint32_t rank = cluster_rank(), C = cluster_size();
  const int64_t first = cluster_id_x(), step = cluster_count_x();
  const int p0 = (int)rank * kClusterPacks + threadIdx.x;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // one commit group per row, empty past the last row, so that the group of
  // the row in hand is always the oldest but kClusterDepth - 1
  const auto issue = [&](int64_t row, int buf) {
    if (row < rows) {
      const TI* xr = x + row * ldx;
      uint4* st = stage + buf * kClusterPacks + threadIdx.x;
#pragma unroll
      for (int i = 0; i < kClusterVPT; ++i) {
        const int p = p0 + i * kClusterBlock;
        if (p < nvec) cp_async16(st + i * kClusterBlock, xr + (int64_t)p * VW);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int d = 0; d < kClusterDepth; ++d) issue(first + d * step, d);
  int parity = 0, buf = 0;
  for (int64_t row = first; row < rows; row += step, parity ^= 1) {
    uint4 v[kClusterVPT];
    cp_async_wait_pending<kClusterDepth - 1>();  // (this thread's own copies)
    const uint4* st = stage + buf * kClusterPacks + threadIdx.x;
#pragma unroll
    for (int i = 0; i < kClusterVPT; ++i) {
      const int p = p0 + i * kClusterBlock;
      v[i] = p < nvec ? st[i * kClusterBlock] : mask_tail<TI>(make_uint4(0, 0, 0, 0), 0);
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kClusterVPT; ++i) m = fmaxf(m, pack_max<TI>(v[i]));
    // this thread's slots of `buf` are in registers now: refill them
    issue(row + kClusterDepth * step, buf);
    buf = buf + 1 == kClusterDepth ? 0 : buf + 1;
    // the warp's max, and its exponentials against it kept in registers (an
    // all -inf warp slice holds zeros and adds nothing)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float e[kClusterVPT][VW];
    float s = 0.f;
    const bool live = m != -INFINITY;
#pragma unroll
    for (int i = 0; i < kClusterVPT; ++i) {
      unpack<TI>(v[i], e[i]);
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        e[i][k] = live ? ex2_approx((e[i][k] - m) * kLog2e) : 0.f;
        s += e[i][k];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) wpart[warp] = make_float2(m, s);
    __syncthreads();
    // warp 0 folds the warps' pairs into this CTA's and publishes it; it
    // reads wpart before its cluster arrive, which every warp's next write to
    // wpart waits behind
    if (warp == 0) {
      const float2 q = lane < kClusterBlock / 32 ? wpart[lane] : make_float2(-INFINITY, 0.f);
      float mc = q.x;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
      float sc = q.x != -INFINITY ? q.y * ex2_approx((q.x - mc) * kLog2e) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
      if (lane == 0) part[parity] = make_float2(mc, sc);
    }
    cluster_arrive();
    cluster_wait();  // every CTA's pair for this row is published
    // lane r of every warp reads CTA r's pair (C remote loads in flight at
    // once, not in a row), then the warp combines lanes 0..7
    const float2 q = lane < C ? ld_cluster_f2(&part[parity], lane)
                              : make_float2(-INFINITY, 0.f);
    float M = q.x;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float S = q.x != -INFINITY ? q.y * ex2_approx((q.x - M) * kLog2e) : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    M = __shfl_sync(0xffffffffu, M, 0);
    S = __shfl_sync(0xffffffffu, S, 0);
    // exp(x - M) / S = exp(x - m_w) * exp(m_w - M) / S
    const float scale = ex2_approx((m - M) * kLog2e) * (1.0f / S);
    TO* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < kClusterVPT; ++i) {
      const int p = p0 + i * kClusterBlock;
      if (p >= nvec) continue;
#pragma unroll
      for (int k = 0; k < VW; ++k) e[i][k] *= scale;
      store_vals<TO, VW, W32>(yr + (int64_t)p * VW, e[i]);
    }
  }
  cp_async_wait_all();
  // no CTA leaves while a partner may still read its pairs
  cluster_arrive();
  cluster_wait();
}

// Launches the cluster kernel for rows of `nvec` packs, or returns -1 when the
// row needs more than 8 CTAs or the device cannot place the cluster.
template <typename TI, typename TO>
int launch_softmax_cluster(const TI* x, int64_t ldx, TO* y, int64_t ldy, int64_t rows,
                           int64_t nvec, cudaStream_t stream) {
  const int C = (int)ceil_div(nvec, kClusterPacks);
  if (C < 2 || C > 8 || rows * C > 0x7fffffff) return -1;
  const auto run = [&](auto w32) -> int {
    constexpr bool W = decltype(w32)::value;
    auto kern = softmax_cluster_kernel<TI, TO, W>;
    const size_t smem = (size_t)kClusterDepth * kClusterPacks * sizeof(uint4);
    // (per launch: the attribute is held per device)
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return -1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * C));
    cfg.blockDim = dim3(kClusterBlock);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
      (void)cudaGetLastError();
      return -1;
    }
    // persistent: as many clusters as are resident at once, each walking rows
    cfg.gridDim = dim3((unsigned)(std::min<int64_t>(rows, clusters) * C));
    (void)cudaLaunchKernelEx(&cfg, kern, x, ldx, y, ldy, rows, (int)nvec);
    return launch_status();
  };
  if constexpr (std::is_same<TO, float>::value && Elem<TI>::kVec == 8) {
    if (aligned32(y) && ldy % 8 == 0) return run(std::true_type{});
  }
  return run(std::false_type{});
}

template <typename TI, typename TO, bool CAUSAL>
int launch_softmax(const TI* x, int64_t ldx, TO* y, int64_t ldy, int64_t rows,
                   int64_t cols, int64_t q_len, int64_t offset, cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<TI>::kVec;
  const bool vec_ok = aligned16(x) && aligned16(y) && cols % VW == 0 && ldx % VW == 0 &&
                      ldy % VW == 0;
  if (vec_ok) {
    auto go = [&](auto tpr, auto vpt) -> int {
      constexpr int TPR = decltype(tpr)::value;
      constexpr int VPT = decltype(vpt)::value;
      constexpr int BLOCK = ladder_block<TPR>();
      const int grid = full_grid(ceil_div(rows, BLOCK / TPR));
      if constexpr (std::is_same<TO, float>::value && VW == 8) {
        if (aligned32(y) && ldy % 8 == 0) {
          softmax_vec_kernel<TI, TO, TPR, VPT, BLOCK, CAUSAL, true>
              <<<grid, BLOCK, 0, stream>>>(x, ldx, y, ldy, rows, cols, q_len, offset);
          return launch_status();
        }
      }
      softmax_vec_kernel<TI, TO, TPR, VPT, BLOCK, CAUSAL, false>
          <<<grid, BLOCK, 0, stream>>>(x, ldx, y, ldy, rows, cols, q_len, offset);
      return launch_status();
    };
    const int64_t nvec = cols / VW;
    int r = -1;
    if constexpr (!CAUSAL) {
      if (nvec > 256 && nvec <= 512)
        r = go(std::integral_constant<int, 32>{}, std::integral_constant<int, 16>{});
    }
    if (r < 0) r = row_ladder<8>(nvec, go);
    if (r >= 0) return r;
    // rows too long for one CTA: a cluster of CTAs per row, one pass
    if constexpr (!CAUSAL) {
      const int rc = launch_softmax_cluster<TI, TO>(x, ldx, y, ldy, rows, nvec, stream);
      if (rc >= 0) return rc;
    }
    // longer rows, causal rows: the two-pass kernel
    if (nvec > 12288) {
      const int grid = (int)std::min<int64_t>(rows, (int64_t)dev.sm_count);
      softmax_long_kernel<TI, TO, CAUSAL, 1024>
          <<<grid, 1024, 0, stream>>>(x, ldx, y, ldy, rows, cols, q_len, offset);
    } else {
      const int64_t row_bytes = cols * (int64_t)sizeof(TI);
      const int per_sm = row_bytes * 2 * dev.sm_count <= (int64_t)64 << 20 ? 2 : 1;
      const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * dev.sm_count);
      softmax_long_kernel<TI, TO, CAUSAL, 512>
          <<<grid, 512, 0, stream>>>(x, ldx, y, ldy, rows, cols, q_len, offset);
    }
    return launch_status();
  }
  auto kern = softmax_loop_kernel<TI, TO, CAUSAL>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * dev.sm_count);
  kern<<<grid, 256, 0, stream>>>(x, ldx, y, ldy, rows, cols, q_len, offset);
  return launch_status();
}

// ------------------------------------------------------- masked softmax ---
// Row r of x (viewed [B, H, Q, K]) is query i = r % Q of head h = (r / Q) % H
// in batch b = r / (Q*H); its mask row starts at b*sb + h*sh + i*sq elements
// (a stride of 0 broadcasts, e.g. HF's [B, 1, Q, K] mask over the heads).
//
// Visit order (head_inner, used by softmax_masked_pair_kernel): with the
// mask broadcast over the heads (sh == 0, HF's [B, 1, Q, K] mask) rows are
// walked query by query with the heads of one query next to each other
// (visit index v = (b*Q + i)*H + h), so the H rows that share a mask row run
// together and the mask row is reused from L2 within a few rows rather than
// a whole head (~96 MB of other traffic at [8, 32, 4096, 4096] f16) later.
// (For the four-warp kernel this order measured the same as row order.)
struct MaskRows {
  int64_t heads, q_len, sb, sh, sq;
  bool head_inner;
  __device__ __forceinline__ int64_t offset(int64_t row) const {
    const int64_t i = row % q_len, t = row / q_len;
    return (t / heads) * sb + (t % heads) * sh + i * sq;
  }
  // Row of x / y visited at position v.
  __device__ __forceinline__ int64_t row_of(int64_t v) const {
    if (!head_inner) return v;
    const int64_t h = v % heads, t = v / heads;  // t = b*Q + i
    return ((t / q_len) * heads + h) * q_len + (t % q_len);
  }
};

// The logit the softmax sees: x*scale + mask.  FUSED: one fp32 FMA.  CHAIN:
// rounded to T after the scale and after the mask add, as HF's two aten ops
// (mul by the scalar, add of the mask) leave it; no FMA contraction.
template <typename T, bool MASK, bool CHAIN>
__device__ __forceinline__ float masked_logit(float x, float scale, float mk) {
  if constexpr (CHAIN) {
    const float t = round_to<T>(__fmul_rn(x, scale));
    return MASK ? round_to<T>(__fadd_rn(t, mk)) : t;
  } else {
    return MASK ? fmaf(x, scale, mk) : x * scale;
  }
}

// A pack of -inf in T's encoding.
template <typename T>
__device__ __forceinline__ uint4 neg_inf_pack() {
  if constexpr (std::is_same<T, float>::value) {
    return make_uint4(0xff800000u, 0xff800000u, 0xff800000u, 0xff800000u);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
  } else {
    return make_uint4(0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u, 0xfc00fc00u);
  }
}

// Rows in registers as fp32 logits in pairs: x and mask packs are loaded
// together, turned into logits (fma.f32x2), max (3-input max), exps in
// place, sum and scaling in pairs, one store pass.  Lanes past the row load
// x = 0 and mask = -inf, so their logit is -inf for any finite scale with no
// per-element select (without a mask, in-range lanes add a zero pack).  The
// mask is read through L2: the rows of one batch's heads are scheduled
// together, so a [B, 1, Q, K] mask comes from DRAM about once per batch.
//
// Row geometry (measured on B200, HF-masked [8, 32, L, L] logits): rows of up
// to 256 packs run one warp per row with 8 packs per thread, 2 CTAs per SM
// (bf16 L = 2048: 6.14 TB/s); longer rows 4 packs per thread at 4 CTAs of
// 256 threads per SM (f16 L = 4096: 5.22 TB/s against 4.89 with 8 packs at 2
// CTAs).  Same-dtype outputs use a persistent grid: with no CTA-wide barrier
// between a warp's rows, the warps of a resident CTA never wait for its
// slowest row (6.14 vs 5.57 TB/s for one CTA per row group).
template <int BLOCK, int VPT>
constexpr int masked_min_blocks() {
  return (BLOCK <= 256 && VPT <= 4) ? 4 : ladder_min_blocks<BLOCK>();
}

template <typename TI, typename TO, int TPR, int VPT, int BLOCK, bool MASK, bool CHAIN, bool W32>
__global__ void __launch_bounds__(BLOCK, (masked_min_blocks<BLOCK, VPT>()))
softmax_masked_kernel(const TI* __restrict__ x, int64_t ldx, const TI* __restrict__ mask,
                      MaskRows mg, TO* __restrict__ y, int64_t ldy, int64_t rows, int nvec,
                      float scale) {
  constexpr int VW = Elem<TI>::kVec;
  constexpr int NP = VW / 2;  // fp32 pairs per pack
  constexpr int RPB = BLOCK / TPR;
  __shared__ float smem[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  const uint64_t scale2 = f2_make(scale, scale);
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows;
       base += (int64_t)gridDim.x * RPB) {
    const bool ok = base + slot < rows;
    const int64_t row = ok ? mg.row_of(base + slot) : 0;
    const TI* xr = x + row * ldx;
    const TI* mr = MASK ? mask + mg.offset(row) : nullptr;
    uint4 xv[VPT], mv[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      const bool in = ok && vi < nvec;
      xv[i] = in ? ld_stream(xr + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
      if constexpr (MASK) mv[i] = in ? ld_stream(mr + (int64_t)vi * VW) : neg_inf_pack<TI>();
      else mv[i] = in ? make_uint4(0, 0, 0, 0) : neg_inf_pack<TI>();
    }
    uint64_t v[VPT][NP];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[VW], mk[VW];
      unpack<TI>(xv[i], f);
      unpack<TI>(mv[i], mk);
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint64_t xp = f2_make(f[2 * p], f[2 * p + 1]);
        const uint64_t mp = f2_make(mk[2 * p], mk[2 * p + 1]);
        if constexpr (CHAIN) {  // masked_logit's chain rounding, a pair at a time
          v[i][p] = round_pair<TI>(f2_add(round_pair<TI>(f2_mul(xp, scale2)), mp));
        } else {
          v[i][p] = f2_fma(xp, scale2, mp);
        }
        m = fmax3(m, f2_lo(v[i][p]), f2_hi(v[i][p]));
      }
    }
    m = row_reduce<FastMaxOp, TPR, BLOCK>(m, smem);
    if (wide_max(m)) {
      const uint64_t nm = f2_make(-m, -m);
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int p = 0; p < NP; ++p) v[i][p] = f2_add(v[i][p], nm);
      m = 0.f;
    }
    const float ml = m * kLog2e;
    const uint64_t log2e2 = f2_make(kLog2e, kLog2e), nml2 = f2_make(-ml, -ml);
    uint64_t acc = f2_make(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint64_t t = f2_fma(v[i][p], log2e2, nml2);
        v[i][p] = f2_make(ex2_approx(f2_lo(t)), ex2_approx(f2_hi(t)));
      }
      // the pack's pairs as a tree, then into the running pair sum
      uint64_t t[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) t[p] = v[i][p];
#pragma unroll
      for (int w = NP / 2; w >= 1; w /= 2)
#pragma unroll
        for (int p = 0; p < w; ++p) t[p] = f2_add(t[p], t[p + w]);
      acc = f2_add(acc, t[0]);
    }
    float s = f2_lo(acc) + f2_hi(acc);
    s = row_reduce<SumOp, TPR, BLOCK>(s, smem);
    const float inv = 1.0f / s;
    const uint64_t inv2 = f2_make(inv, inv);
    TO* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (!ok || vi >= nvec) continue;
      float o[VW];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint64_t t = f2_mul(v[i][p], inv2);
        o[2 * p] = f2_lo(t);
        o[2 * p + 1] = f2_hi(t);
      }
      store_vals<TO, VW, W32>(yr + (int64_t)vi * VW, o);
    }
  }
}

// Rows of 257..512 packs (e.g. 4096 f16 keys): two warps per row, 8 packs
// of x and 8 of the mask per lane, turned into fp32 logits in registers as
// in softmax_masked_kernel.  Each warp takes its half's max m_w and the sum
// s_w of exp(logit - m_w) over its own exps; the pair then exchanges (m_w,
// s_w) once through shared memory, behind a named barrier for those two
// warps only (bar.sync 1 + slot, 64), and combines
//   M = max(m_a, m_b),  S = sum_w s_w * 2^((m_w - M) log2e),
// each warp storing its exps times c_w = 2^((m_w - M) log2e) / S.  So a row
// costs one barrier of two warps, and the four rows of a CTA never wait for
// each other (a persistent grid: each pair walks its own rows).  The
// per-warp factor changes a result by a few fp32 ulp against the one-max
// form.  A half whose keys are all -inf has s_w = 0 and c_w = 0; a row with
// no visible key gets S = 0 and comes out NaN, as in the reference.
//
// The packs come through shared memory one row ahead: as soon as a thread
// has its row in registers it issues cp.async copies of its next row's x and
// mask packs into the same slots (its own slots only, so no barrier), and
// the copies stream in while the row is reduced, exponentiated and stored.
// Registers hold one row; shared memory (64 KB a CTA) holds the next.
// Measured on B200, f16 [8, 32, 4096, 4096] with the [8, 1, 4096, 4096] HF
// mask: 2.95 ms (5.91 TB/s); the same kernel loading from global memory
// directly 3.19 ms (3.10 ms at 3 CTAs per SM, which spills); the four-warp
// rows it replaces (4 packs of x and mask per thread, two CTA-wide barriers
// per row) 3.47 ms; one warp per row holding only x and reading the mask
// again per pass spilled at 128 registers, and staging x in shared memory
// for that geometry was issue-bound at 12 warps per SM (5.9 ms).
constexpr int kPairVPT = 8;  // packs per lane: rows of up to 2 * 32 * 8 = 512 packs

template <typename TI, typename TO, bool MASK, bool CHAIN, bool W32>
__global__ void __launch_bounds__(256, 2)
softmax_masked_pair_kernel(const TI* __restrict__ x, int64_t ldx, const TI* __restrict__ mask,
                           MaskRows mg, TO* __restrict__ y, int64_t ldy, int64_t rows, int nvec,
                           float scale) {
  constexpr int VW = Elem<TI>::kVec;
  constexpr int NP = VW / 2;
  constexpr int RPB = 4;  // rows (warp pairs) per CTA
  __shared__ float2 part[RPB][2][2];  // [slot][row parity][warp of the pair] = (m_w, s_w)
  // each thread's x and mask packs of its next row, [pack][thread] so that a
  // warp's 16-byte accesses are consecutive (no bank conflicts)
  extern __shared__ uint4 stage[];
  const int slot = threadIdx.x >> 6;
  const int half = (threadIdx.x >> 5) & 1;
  const int lane = threadIdx.x & 63;  // lane within the row's 64 threads
  const uint64_t scale2 = f2_make(scale, scale);
  const uint64_t log2e2 = f2_make(kLog2e, kLog2e);
  const int64_t stride = (int64_t)gridDim.x * RPB;
  const auto issue = [&](int64_t vrow) {
    const int64_t r = mg.row_of(vrow);
    const TI* xr = x + r * ldx;
    const TI* mr = MASK ? mask + mg.offset(r) : nullptr;
#pragma unroll
    for (int i = 0; i < kPairVPT; ++i) {
      const int vi = lane + i * 64;
      if (vi < nvec) {
        cp_async16(&stage[i * 256 + threadIdx.x], xr + (int64_t)vi * VW);
        if constexpr (MASK)
          cp_async16(&stage[(kPairVPT + i) * 256 + threadIdx.x], mr + (int64_t)vi * VW);
      }
    }
    cp_async_commit();
  };
  if ((int64_t)blockIdx.x * RPB + slot < rows) issue((int64_t)blockIdx.x * RPB + slot);
  int parity = 0;
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows; base += stride, parity ^= 1) {
    if (base + slot >= rows) break;  // uniform over the pair
    const int64_t row = mg.row_of(base + slot);
    uint4 xv[kPairVPT], mv[kPairVPT];
    cp_async_wait_all();  // this row's copies (issued one row ahead) landed
#pragma unroll
    for (int i = 0; i < kPairVPT; ++i) {
      const bool in = lane + i * 64 < nvec;
      xv[i] = in ? stage[i * 256 + threadIdx.x] : make_uint4(0, 0, 0, 0);
      if constexpr (MASK) mv[i] = in ? stage[(kPairVPT + i) * 256 + threadIdx.x]
                                     : neg_inf_pack<TI>();
      else mv[i] = in ? make_uint4(0, 0, 0, 0) : neg_inf_pack<TI>();
    }
    uint64_t v[kPairVPT][NP];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPairVPT; ++i) {
      float f[VW], mk[VW];
      unpack<TI>(xv[i], f);
      unpack<TI>(mv[i], mk);
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint64_t xp = f2_make(f[2 * p], f[2 * p + 1]);
        const uint64_t mp = f2_make(mk[2 * p], mk[2 * p + 1]);
        if constexpr (CHAIN) {
          v[i][p] = round_pair<TI>(f2_add(round_pair<TI>(f2_mul(xp, scale2)), mp));
        } else {
          v[i][p] = f2_fma(xp, scale2, mp);
        }
        m = fmax3(m, f2_lo(v[i][p]), f2_hi(v[i][p]));
      }
    }
    // the next row's packs go into the slots just read (each thread reuses
    // only its own slots, after its values are in registers)
    if (base + stride + slot < rows) issue(base + stride + slot);
    m = group_reduce_warp<FastMaxOp, 32>(m);
    // exps against this warp's max: the one-FMA form, (logit - m) first for
    // a max below -2.36e38 (wide_max), and a zero shift for an all -inf half
    // (its exps are then exact zeros, not NaN)
    const float mw = (m == -INFINITY) ? 0.f : m;
    if (wide_max(mw)) {
      const uint64_t nm2 = f2_make(-mw, -mw);
#pragma unroll
      for (int i = 0; i < kPairVPT; ++i)
#pragma unroll
        for (int p = 0; p < NP; ++p) v[i][p] = f2_mul(f2_add(v[i][p], nm2), log2e2);
    } else {
      const uint64_t nml2 = f2_make(-mw * kLog2e, -mw * kLog2e);
#pragma unroll
      for (int i = 0; i < kPairVPT; ++i)
#pragma unroll
        for (int p = 0; p < NP; ++p) v[i][p] = f2_fma(v[i][p], log2e2, nml2);
    }
    uint64_t acc = f2_make(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kPairVPT; ++i) {
#pragma unroll
      for (int p = 0; p < NP; ++p)
        v[i][p] = f2_make(ex2_approx(f2_lo(v[i][p])), ex2_approx(f2_hi(v[i][p])));
      uint64_t t[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) t[p] = v[i][p];
#pragma unroll
      for (int w = NP / 2; w >= 1; w /= 2)
#pragma unroll
        for (int p = 0; p < w; ++p) t[p] = f2_add(t[p], t[p + w]);
      acc = f2_add(acc, t[0]);
    }
    float sw = f2_lo(acc) + f2_hi(acc);
    sw = group_reduce_warp<SumOp, 32>(sw);
    // the pair's exchange (double-buffered by row parity: the partner has
    // read this buffer's previous values before it reached the barrier of
    // the row in between)
    if ((threadIdx.x & 31) == 0) part[slot][parity][half] = make_float2(m, sw);
    asm volatile("bar.sync %0, 64;" ::"r"(1 + slot) : "memory");
    const float2 o = part[slot][parity][half ^ 1];
    const float M = fmaxf(m, o.x);
    // the scale of each half's exps against the row max (0 for an all -inf
    // half; for a wide row m - M is exact, Sterbenz)
    const float fw = (m == -INFINITY) ? 0.f : ex2_approx((m - M) * kLog2e);
    const float fo = (o.x == -INFINITY) ? 0.f : ex2_approx((o.x - M) * kLog2e);
    const float S = sw * fw + o.y * fo;
    const float c = fw / S;
    const uint64_t c2 = f2_make(c, c);
    TO* yr = y + row * ldy;
#pragma unroll
    for (int i = 0; i < kPairVPT; ++i) {
      const int vi = lane + i * 64;
      if (vi >= nvec) continue;
      float out[VW];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const uint64_t t = f2_mul(v[i][p], c2);
        out[2 * p] = f2_lo(t);
        out[2 * p + 1] = f2_hi(t);
      }
      store_vals<TO, VW, W32>(yr + (int64_t)vi * VW, out);
    }
  }
  cp_async_wait_all();
}

// Any row length / alignment: one CTA per row, three passes over the row
// (the second and third mostly from L2).
template <typename TI, typename TO, bool MASK, bool CHAIN>
__global__ void __launch_bounds__(256)
softmax_masked_loop_kernel(const TI* x, int64_t ldx, const TI* mask, MaskRows mg, TO* y,
                           int64_t ldy, int64_t rows, int64_t cols, float scale) {
  __shared__ float smem[256 / 32];
  for (int64_t v = blockIdx.x; v < rows; v += gridDim.x) {
    const int64_t row = mg.row_of(v);
    const TI* xr = x + row * ldx;
    const TI* mr = MASK ? mask + mg.offset(row) : nullptr;
    const auto logit = [&](int64_t c) {
      return masked_logit<TI, MASK, CHAIN>(Elem<TI>::to_f(xr[c]), scale,
                                           MASK ? Elem<TI>::to_f(mr[c]) : 0.f);
    };
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < cols; c += 256) m = fmaxf(m, logit(c));
    m = block_reduce<FastMaxOp, 256>(m, smem);
    const RowShift sh(m);
    float s = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256) s += sh.exp(logit(c));
    s = block_reduce<SumOp, 256>(s, smem);
    const float inv = 1.0f / s;
    TO* yr = y + row * ldy;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float o = sh.exp(logit(c)) * inv;
      if constexpr (std::is_same<TO, float>::value) yr[c] = o;
      else yr[c] = Elem<TO>::from_f(o);
    }
  }
}

template <typename TI, typename TO, bool MASK, bool CHAIN>
int launch_softmax_masked(const TI* x, int64_t ldx, const TI* mask, const MaskRows& mg, TO* y,
                          int64_t ldy, int64_t rows, int64_t cols, float scale,
                          cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<TI>::kVec;
  const bool mask_ok = !MASK || (aligned16(mask) && mg.sb % VW == 0 && mg.sh % VW == 0 &&
                                 mg.sq % VW == 0);
  const bool vec_ok = mask_ok && aligned16(x) && aligned16(y) && cols % VW == 0 &&
                      ldx % VW == 0 && ldy % VW == 0;
  if (vec_ok) {
    const int64_t nvec = cols / VW;
    auto go = [&](auto tpr, auto vpt) -> int {
      constexpr int TPR = decltype(tpr)::value;
      constexpr int VPT = decltype(vpt)::value;
      constexpr int BLOCK = ladder_block<TPR>();
      const int64_t groups = ceil_div(rows, BLOCK / TPR);
      if constexpr (std::is_same<TO, float>::value && VW == 8) {
        // fp32 outputs of 16-bit logits: one CTA per row group (bf16 L = 2048:
        // 5.28 vs 4.86 TB/s persistent; the wider stores keep more in flight)
        const int grid = full_grid(groups);
        if (aligned32(y) && ldy % 8 == 0) {
          softmax_masked_kernel<TI, TO, TPR, VPT, BLOCK, MASK, CHAIN, true>
              <<<grid, BLOCK, 0, stream>>>(x, ldx, mask, mg, y, ldy, rows, (int)nvec, scale);
        } else {
          softmax_masked_kernel<TI, TO, TPR, VPT, BLOCK, MASK, CHAIN, false>
              <<<grid, BLOCK, 0, stream>>>(x, ldx, mask, mg, y, ldy, rows, (int)nvec, scale);
        }
        return launch_status();
      } else {
        // resident CTAs per SM of this instantiation
        static const int per_sm = blocks_per_sm(
            softmax_masked_kernel<TI, TO, TPR, VPT, BLOCK, MASK, CHAIN, false>, BLOCK, 0);
        const int grid = (int)std::max<int64_t>(
            1, std::min<int64_t>(groups, (int64_t)per_sm * dev.sm_count));
        softmax_masked_kernel<TI, TO, TPR, VPT, BLOCK, MASK, CHAIN, false>
            <<<grid, BLOCK, 0, stream>>>(x, ldx, mask, mg, y, ldy, rows, (int)nvec, scale);
        return launch_status();
      }
    };
    if (nvec > 256 && nvec <= 512) {
      // two warps per row, one pair exchange (softmax_masked_pair_kernel)
      const auto pairs = [&](auto w32) -> int {
        constexpr bool W = decltype(w32)::value;
        auto kern = softmax_masked_pair_kernel<TI, TO, MASK, CHAIN, W>;
        const size_t smem = (size_t)2 * kPairVPT * 256 * 16;  // 64 KB: x and mask packs
        // (per device: a function attribute belongs to the current context)
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
          return launch_status();
        static const int per_sm = blocks_per_sm(kern, 256, smem);
        const int grid = (int)std::max<int64_t>(
            1, std::min<int64_t>(ceil_div(rows, 4), (int64_t)per_sm * dev.sm_count));
        MaskRows mgh = mg;
        mgh.head_inner = MASK && mg.sh == 0 && mg.heads > 1;
        kern<<<grid, 256, smem, stream>>>(x, ldx, mask, mgh, y, ldy, rows, (int)nvec, scale);
        return launch_status();
      };
      if constexpr (std::is_same<TO, float>::value && VW == 8) {
        if (aligned32(y) && ldy % 8 == 0) return pairs(std::true_type{});
      }
      return pairs(std::false_type{});
    }
    int r = -1;
    if constexpr (std::is_same<TO, float>::value && VW == 8) {
      r = row_ladder<8>(nvec, go);
    } else if (nvec <= 256) {
      r = row_ladder<8>(nvec, go);
    } else {  // 4 packs per thread, 4 CTAs of 256 threads per SM
      using std::integral_constant;
      using V4 = integral_constant<int, 4>;
      if (nvec <= 512) r = go(integral_constant<int, 128>{}, V4{});
      else if (nvec <= 1024) r = go(integral_constant<int, 256>{}, V4{});
      else if (nvec <= 2048) r = go(integral_constant<int, 512>{}, V4{});
      else if (nvec <= 4096) r = go(integral_constant<int, 1024>{}, V4{});
    }
    if (r >= 0) return r;
  }
  auto kern = softmax_masked_loop_kernel<TI, TO, MASK, CHAIN>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * dev.sm_count);
  kern<<<grid, 256, 0, stream>>>(x, ldx, mask, mg, y, ldy, rows, cols, scale);
  return launch_status();
}

// Calls f(TI{}, TO{}) for the supported (in, out) pairs: out == in, or
// 16-bit in with fp32 out (half_to_float).
template <typename F>
int dispatch_in_out(int in_dtype, int out_dtype, F&& f) {
  if (in_dtype == out_dtype) {
    return dispatch_float(in_dtype, [&](auto t) { return f(t, t); });
  }
  if (out_dtype == FL_B200_F32) {
    if (in_dtype == FL_B200_BF16) return f(__nv_bfloat16{}, float{});
    if (in_dtype == FL_B200_F16) return f(__half{}, float{});
  }
  return FL_B200_ERR_UNSUPPORTED_DTYPE;
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_softmax_lastdim(const void* x, int64_t ld_x, void* out,
                                        int64_t ld_out, int64_t rows, int64_t cols,
                                        int in_dtype, int out_dtype, int causal,
                                        int64_t q_len, int64_t causal_offset,
                                        fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && out && ld_x >= cols && ld_out >= cols);
  if (causal) FLB_CHECK_ARG(q_len > 0);
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_in_out(in_dtype, out_dtype, [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    auto xp = static_cast<const TI*>(x);
    auto yp = static_cast<TO*>(out);
    if (causal)
      return launch_softmax<TI, TO, true>(xp, ld_x, yp, ld_out, rows, cols, q_len,
                                          causal_offset, s);
    return launch_softmax<TI, TO, false>(xp, ld_x, yp, ld_out, rows, cols, 1, 0, s);
  });
}

FL_B200_API int fl_b200_softmax_masked(const void* x, int64_t ld_x, const void* mask,
                                       int64_t mask_stride_b, int64_t mask_stride_h,
                                       int64_t mask_stride_q, void* out, int64_t ld_out,
                                       int64_t rows, int64_t cols, int64_t heads,
                                       int64_t q_len, float scale, int in_dtype,
                                       int out_dtype, int rounding,
                                       fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && cols >= 0 && heads > 0 && q_len > 0);
  FLB_CHECK_ARG(rows % (heads * q_len) == 0);
  FLB_CHECK_ARG(rounding == FL_B200_ROUND_FUSED || rounding == FL_B200_ROUND_CHAIN);
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && out && ld_x >= cols && ld_out >= cols);
  const MaskRows mg{heads, q_len, mask_stride_b, mask_stride_h, mask_stride_q, false};
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_in_out(in_dtype, out_dtype, [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    auto xp = static_cast<const TI*>(x);
    auto mp = static_cast<const TI*>(mask);
    auto yp = static_cast<TO*>(out);
    const bool chain = rounding == FL_B200_ROUND_CHAIN;
    if (mask) {
      return chain ? launch_softmax_masked<TI, TO, true, true>(xp, ld_x, mp, mg, yp, ld_out, rows,
                                                                cols, scale, s)
                   : launch_softmax_masked<TI, TO, true, false>(xp, ld_x, mp, mg, yp, ld_out,
                                                                 rows, cols, scale, s);
    }
    return chain ? launch_softmax_masked<TI, TO, false, true>(xp, ld_x, mp, mg, yp, ld_out, rows,
                                                               cols, scale, s)
                 : launch_softmax_masked<TI, TO, false, false>(xp, ld_x, mp, mg, yp, ld_out,
                                                                rows, cols, scale, s);
  });
}

FL_B200_API int fl_b200_softmax_middim(const void* x, void* out, int64_t outer,
                                       int64_t n, int64_t inner, int in_dtype,
                                       int out_dtype, fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(outer >= 0 && n >= 0 && inner >= 0);
  if (outer == 0 || n == 0 || inner == 0) return FL_B200_OK;
  FLB_CHECK_ARG(x && out);
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  return dispatch_in_out(in_dtype, out_dtype, [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    auto kern = softmax_middim_kernel<TI, TO>;
    const int per_sm = blocks_per_sm(kern, 256, 0);
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(outer * inner, 256), (int64_t)per_sm * dev.sm_count));
    kern<<<grid, 256, 0, s>>>(static_cast<const TI*>(x), static_cast<TO*>(out), outer, n,
                              inner);
    return launch_status();
  });
}

}  // extern "C"
