// RoPE on q/k, and Qwen3's per-head RMSNorm immediately followed by RoPE.
//
// Reference behaviour: HF apply_rotary_pos_emb (transformers
// models/qwen3/modeling_qwen3.py:138-169):
//   q_embed = q*cos + rotate_half(q)*sin,  rotate_half(x) = cat(-x2, x1)
// which the reference runs on flagos as neg (csrc/aten/backends/cuda/
// neg.cu:14-32), cat (cat.cc:13-39), two mul (mul.cu:28-52) and an add
// (add.cu:48-84) per tensor; and Qwen3's q_norm/k_norm RMSNorm over the
// head dim right before it (modeling_qwen3.py:248-249,263-268).
//
// A head row of D elements is owned by G = D/(2*VW) threads; thread j holds
// pack j of the low half AND pack j of the high half, so rotate_half needs no
// data exchange, and the per-head norm needs one G-lane butterfly.
#include "common.cuh"

#include <algorithm>

namespace flb200 {
namespace {

struct RopeArgs {
  const void* q;
  void* qo;
  const void* k;
  void* ko;
  const void* wq;
  const void* wk;
  const void* cos;
  const void* sin;
  int64_t sq[3], soq[3], sk[3], sok[3];  // strides over (b, h, s)
  int64_t scb, scs;                      // cos/sin strides over (b, s)
  uint32_t Hq, Hk, S, D;
  float eps;
};

template <typename T, bool CHAIN>
__device__ __forceinline__ void rope_pair(float xl, float xh, float cl, float sl,
                                          float ch, float sh, float& ol, float& oh) {
  if (CHAIN) {
    // q*cos -> T;  rotate_half(q)*sin -> T;  sum -> T  (one aten op each)
    ol = round_to<T>(round_to<T>(xl * cl) + round_to<T>(-xh * sl));
    oh = round_to<T>(round_to<T>(xh * ch) + round_to<T>(xl * sh));
  } else {
    ol = fmaf(xl, cl, -xh * sl);
    oh = fmaf(xh, ch, xl * sh);
  }
}

template <typename T, int G, bool NORM, bool CHAIN>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeArgs a, uint32_t units) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  constexpr int UPB = 256 / G;  // head rows per CTA iteration
  const int j = threadIdx.x % G;
  const uint32_t htot = a.Hq + a.Hk;
  const uint32_t half = a.D / 2;
  for (uint32_t ub = blockIdx.x * UPB; ub < units; ub += gridDim.x * UPB) {
    const uint32_t u = ub + threadIdx.x / G;
    const bool valid = u < units;
    const uint32_t uu = valid ? u : 0;
    const uint32_t token = uu / htot;
    const uint32_t head = uu - token * htot;
    const uint32_t b = token / a.S;
    const uint32_t s = token - b * a.S;
    const bool isq = head < a.Hq;
    const uint32_t hh = isq ? head : head - a.Hq;
    const T* src;
    T* dst;
    const T* w;
    if (isq) {
      src = static_cast<const T*>(a.q) + b * a.sq[0] + hh * a.sq[1] + s * a.sq[2];
      dst = static_cast<T*>(a.qo) + b * a.soq[0] + hh * a.soq[1] + s * a.soq[2];
      w = static_cast<const T*>(a.wq);
    } else {
      src = static_cast<const T*>(a.k) + b * a.sk[0] + hh * a.sk[1] + s * a.sk[2];
      dst = static_cast<T*>(a.ko) + b * a.sok[0] + hh * a.sok[1] + s * a.sok[2];
      w = static_cast<const T*>(a.wk);
    }
    const uint32_t dl = j * VW;
    float xl[VW], xh[VW];
    {
      uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
      if (valid) {
        lo = ld_stream(src + dl);
        hi = ld_stream(src + half + dl);
      }
      unpack<T>(lo, xl);
      unpack<T>(hi, xh);
    }
    if constexpr (NORM) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < VW; ++e) ss = fmaf(xl[e], xl[e], fmaf(xh[e], xh[e], ss));
      ss = group_reduce_warp<SumOp, G>(ss);
      const float r = 1.0f / sqrtf(ss / (float)a.D + a.eps);
      if (valid) {
        float wl[VW], wh[VW];
        unpack<T>(ld_cached(w + dl), wl);
        unpack<T>(ld_cached(w + half + dl), wh);
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          if (CHAIN) {
            xl[e] = round_to<T>(wl[e] * round_to<T>(xl[e] * r));
            xh[e] = round_to<T>(wh[e] * round_to<T>(xh[e] * r));
          } else {
            xl[e] = wl[e] * (xl[e] * r);
            xh[e] = wh[e] * (xh[e] * r);
          }
        }
      }
    }
    if (!valid) continue;
    const T* cb = static_cast<const T*>(a.cos) + b * a.scb + s * a.scs;
    const T* sb = static_cast<const T*>(a.sin) + b * a.scb + s * a.scs;
    float cl[VW], ch[VW], sl[VW], sh[VW];
    unpack<T>(ld_cached(cb + dl), cl);
    unpack<T>(ld_cached(cb + half + dl), ch);
    unpack<T>(ld_cached(sb + dl), sl);
    unpack<T>(ld_cached(sb + half + dl), sh);
    float ol[VW], oh[VW];
#pragma unroll
    for (int e = 0; e < VW; ++e)
      rope_pair<T, CHAIN>(xl[e], xh[e], cl[e], sl[e], ch[e], sh[e], ol[e], oh[e]);
    st_stream(dst + dl, pack<T>(ol));
    st_stream(dst + half + dl, pack<T>(oh));
  }
}

// One warp per token.  Lane l owns pack j = l % G of every head row it
// visits (so it loads its cos/sin packs once per token) and head slot
// l / G; the warp walks the token's Hq + Hk head rows SLOTS = 32 / G at a
// time, U head steps per batch so 2*U packs per lane are in flight.  No
// per-row index division, table loads amortised over all heads of the token.
// The packs reach registers through shared memory: the next batch is copied
// (cp.async) while this one is rotated and stored, so a warp's second batch
// no longer waits a full memory round trip after its first (B200, bf16
// 40 heads x 128: 5.78 vs 5.60 TB/s at 16384 tokens, 6.61 vs 6.40 at 131072).
template <typename T, int G, bool NORM, bool CHAIN, int U>
__global__ void __launch_bounds__(256) rope_token_kernel(RopeArgs a, uint32_t tokens) {
  pdl_prologue();
  constexpr int VW = Elem<T>::kVec;
  constexpr int SLOTS = 32 / G;
  const int lane = threadIdx.x & 31;
  const int j = lane % G;
  const int slot = lane / G;
  const uint32_t htot = a.Hq + a.Hk;
  const uint32_t half = a.D / 2;
  const uint32_t dl = j * VW;
  const uint32_t warps = blockDim.x / 32;
  // The norm weights are the same for every token: each lane keeps its packs
  // of both halves of w_q and w_k as loaded (16-bit encodings for bf16/f16),
  // so a head step needs no weight load.
  uint4 wql = make_uint4(0, 0, 0, 0), wqh = wql, wkl = wql, wkh = wql;
  if constexpr (NORM) {
    if (a.Hq > 0) {
      wql = ld_cached(static_cast<const T*>(a.wq) + dl);
      wqh = ld_cached(static_cast<const T*>(a.wq) + half + dl);
    }
    if (a.Hk > 0) {
      wkl = ld_cached(static_cast<const T*>(a.wk) + dl);
      wkh = ld_cached(static_cast<const T*>(a.wk) + half + dl);
    }
  }
  // Staging: each lane's packs of the warp's next batch of head rows (the
  // next batch of this token, else the first of the warp's next token),
  // copied by cp.async while this batch is computed and stored; a lane reads
  // back only the slots it copied.
  constexpr uint32_t kStep = SLOTS * U;
  __shared__ uint4 stage[8][U][2][32];  // [warp][head step][half][lane], U * 8 KB
  uint4 (*my)[2][32] = stage[threadIdx.x / 32];
  const uint32_t stride = gridDim.x * warps;
  const auto issue = [&](uint32_t token, uint32_t h0) {
    if (token < tokens) {
      const uint32_t b = token / a.S;
      const uint32_t s = token - b * a.S;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t h = h0 + u * SLOTS + slot;
        if (h < htot) {
          const T* src = h < a.Hq
              ? static_cast<const T*>(a.q) + b * a.sq[0] + h * a.sq[1] + s * a.sq[2]
              : static_cast<const T*>(a.k) + b * a.sk[0] + (h - a.Hq) * a.sk[1] + s * a.sk[2];
          cp_async16(&my[u][0][lane], src + dl);
          cp_async16(&my[u][1][lane], src + half + dl);
        }
      }
    }
    cp_async_commit();
  };
  issue(blockIdx.x * warps + threadIdx.x / 32, 0);
  for (uint32_t token = blockIdx.x * warps + threadIdx.x / 32; token < tokens;
       token += stride) {  // warp-uniform
    const uint32_t b = token / a.S;
    const uint32_t s = token - b * a.S;
    const T* cb = static_cast<const T*>(a.cos) + b * a.scb + s * a.scs;
    const T* sb = static_cast<const T*>(a.sin) + b * a.scb + s * a.scs;
    float cl[VW], ch[VW], sl[VW], sh[VW];
    unpack<T>(ld_cached(cb + dl), cl);
    unpack<T>(ld_cached(cb + half + dl), ch);
    unpack<T>(ld_cached(sb + dl), sl);
    unpack<T>(ld_cached(sb + half + dl), sh);
    // fused rounding: the rotation in fp32 pairs, sin of the low half negated
    // once per token (x*(-s) is exactly -(x*s), so the results equal the
    // scalar fmaf(xl, cl, -xh*sl), fmaf(xh, ch, xl*sh) bit for bit)
    uint64_t cl2[VW / 2], ch2[VW / 2], nsl2[VW / 2], sh2[VW / 2];
    if constexpr (!CHAIN) {
#pragma unroll
      for (int p = 0; p < VW / 2; ++p) {
        cl2[p] = f2_make(cl[2 * p], cl[2 * p + 1]);
        ch2[p] = f2_make(ch[2 * p], ch[2 * p + 1]);
        nsl2[p] = f2_make(-sl[2 * p], -sl[2 * p + 1]);
        sh2[p] = f2_make(sh[2 * p], sh[2 * p + 1]);
      }
    }
    for (uint32_t h0 = 0; h0 < htot; h0 += kStep) {  // warp-uniform
      uint4 lo[U], hi[U];
      T* dst[U];
      bool valid[U], isq_[U];
      cp_async_wait_all();
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t h = h0 + u * SLOTS + slot;
        valid[u] = h < htot;
        const bool isq = h < a.Hq;
        isq_[u] = isq;
        const uint32_t hh = isq ? h : h - a.Hq;
        dst[u] = isq ? static_cast<T*>(a.qo) + b * a.soq[0] + hh * a.soq[1] + s * a.soq[2]
                     : static_cast<T*>(a.ko) + b * a.sok[0] + hh * a.sok[1] + s * a.sok[2];
        lo[u] = make_uint4(0, 0, 0, 0);
        hi[u] = make_uint4(0, 0, 0, 0);
        if (valid[u]) {
          lo[u] = my[u][0][lane];
          hi[u] = my[u][1][lane];
        }
      }
      // this lane's slots are in registers: stage the warp's next batch
      if (h0 + kStep < htot) issue(token, h0 + kStep);
      else issue(token + stride, 0);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float xl[VW], xh[VW];
        unpack<T>(lo[u], xl);
        unpack<T>(hi[u], xh);
        if constexpr (NORM) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < VW; ++e) ss = fmaf(xl[e], xl[e], fmaf(xh[e], xh[e], ss));
          ss = group_reduce_warp<SumOp, G>(ss);
          const float r = 1.0f / sqrtf(ss / (float)a.D + a.eps);
          if (valid[u]) {
            float wl[VW], wh[VW];
            unpack<T>(isq_[u] ? wql : wkl, wl);
            unpack<T>(isq_[u] ? wqh : wkh, wh);
#pragma unroll
            for (int e = 0; e < VW; ++e) {
              if (CHAIN) {
                xl[e] = round_to<T>(wl[e] * round_to<T>(xl[e] * r));
                xh[e] = round_to<T>(wh[e] * round_to<T>(xh[e] * r));
              } else {
                xl[e] = wl[e] * (xl[e] * r);
                xh[e] = wh[e] * (xh[e] * r);
              }
            }
          }
        }
        if (!valid[u]) continue;
        float ol[VW], oh[VW];
        if constexpr (CHAIN) {
#pragma unroll
          for (int e = 0; e < VW; ++e)
            rope_pair<T, CHAIN>(xl[e], xh[e], cl[e], sl[e], ch[e], sh[e], ol[e], oh[e]);
        } else {
#pragma unroll
          for (int p = 0; p < VW / 2; ++p) {
            const uint64_t xl2 = f2_make(xl[2 * p], xl[2 * p + 1]);
            const uint64_t xh2 = f2_make(xh[2 * p], xh[2 * p + 1]);
            const uint64_t o1 = f2_fma(xl2, cl2[p], f2_mul(xh2, nsl2[p]));
            const uint64_t o2 = f2_fma(xh2, ch2[p], f2_mul(xl2, sh2[p]));
            ol[2 * p] = f2_lo(o1);
            ol[2 * p + 1] = f2_hi(o1);
            oh[2 * p] = f2_lo(o2);
            oh[2 * p + 1] = f2_hi(o2);
          }
        }
        st_stream(dst[u] + dl, pack<T>(ol));
        st_stream(dst[u] + half + dl, pack<T>(oh));
      }
    }
  }
  cp_async_wait_all();
}

// Any alignment / head dim: one warp per head row, scalar element access.
template <typename T, bool NORM, bool CHAIN>
__global__ void __launch_bounds__(256) rope_scalar_kernel(RopeArgs a, uint32_t units) {
  pdl_prologue();
  constexpr int UPB = 256 / 32;
  const int lane = threadIdx.x & 31;
  const uint32_t htot = a.Hq + a.Hk;
  const uint32_t half = a.D / 2;
  for (uint32_t ub = blockIdx.x * UPB; ub < units; ub += gridDim.x * UPB) {
    const uint32_t u = ub + threadIdx.x / 32;
    if (u >= units) continue;  // whole warp leaves together
    const uint32_t token = u / htot;
    const uint32_t head = u - token * htot;
    const uint32_t b = token / a.S;
    const uint32_t s = token - b * a.S;
    const bool isq = head < a.Hq;
    const uint32_t hh = isq ? head : head - a.Hq;
    const T* src;
    T* dst;
    const T* w;
    if (isq) {
      src = static_cast<const T*>(a.q) + b * a.sq[0] + hh * a.sq[1] + s * a.sq[2];
      dst = static_cast<T*>(a.qo) + b * a.soq[0] + hh * a.soq[1] + s * a.soq[2];
      w = static_cast<const T*>(a.wq);
    } else {
      src = static_cast<const T*>(a.k) + b * a.sk[0] + hh * a.sk[1] + s * a.sk[2];
      dst = static_cast<T*>(a.ko) + b * a.sok[0] + hh * a.sok[1] + s * a.sok[2];
      w = static_cast<const T*>(a.wk);
    }
    float r = 1.f;
    if constexpr (NORM) {
      float ss = 0.f;
      for (uint32_t d = lane; d < a.D; d += 32) {
        const float v = Elem<T>::to_f(src[d]);
        ss = fmaf(v, v, ss);
      }
      ss = group_reduce_warp<SumOp, 32>(ss);
      r = 1.0f / sqrtf(ss / (float)a.D + a.eps);
    }
    const T* cb = static_cast<const T*>(a.cos) + b * a.scb + s * a.scs;
    const T* sb = static_cast<const T*>(a.sin) + b * a.scb + s * a.scs;
    // Read every element this lane needs before writing (in place allowed).
    for (uint32_t d = lane; d < half; d += 32) {
      float xl = Elem<T>::to_f(src[d]);
      float xh = Elem<T>::to_f(src[d + half]);
      if constexpr (NORM) {
        const float wl = Elem<T>::to_f(w[d]), wh = Elem<T>::to_f(w[d + half]);
        if (CHAIN) {
          xl = round_to<T>(wl * round_to<T>(xl * r));
          xh = round_to<T>(wh * round_to<T>(xh * r));
        } else {
          xl = wl * (xl * r);
          xh = wh * (xh * r);
        }
      }
      float ol, oh;
      rope_pair<T, CHAIN>(xl, xh, Elem<T>::to_f(cb[d]), Elem<T>::to_f(sb[d]),
                          Elem<T>::to_f(cb[d + half]), Elem<T>::to_f(sb[d + half]), ol,
                          oh);
      dst[d] = Elem<T>::from_f(ol);
      dst[d + half] = Elem<T>::from_f(oh);
    }
  }
}

template <typename T, int G, bool NORM, bool CHAIN>
int launch_vec(const RopeArgs& a, uint32_t units, const DeviceInfo& dev,
               cudaStream_t stream) {
  auto kern = rope_vec_kernel<T, G, NORM, CHAIN>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int64_t blocks = ceil_div(units, 256 / G);
  const int grid = (int)std::min<int64_t>(blocks, (int64_t)per_sm * dev.sm_count);
  launch_k(kern, grid, 256, 0, stream, a, units);
  return launch_status();
}

// Token-per-warp kernel, full grid (8 tokens per 256-thread CTA; the staging
// is laid out for 8 warps).  Measured on B200 at 131072 tokens x (32 + 8)
// heads x 128: 6.46 TB/s before the staging, against 5.42 TB/s for one head
// row per G threads; a persistent grid of the staged kernel (warps prefetch
// their next token) measured 5.90 and 5.37 TB/s at 131072 and 16384 tokens.
template <typename T, int G, bool NORM, bool CHAIN>
int launch_token(const RopeArgs& a, uint32_t tokens, cudaStream_t stream) {
  constexpr uint32_t kSlots = 32 / G;
  const uint32_t steps = (a.Hq + a.Hk + kSlots - 1) / kSlots;  // head steps per token
  const int grid = full_grid(ceil_div(tokens, 8));
  if (steps % 5 == 0) {
    launch_k((rope_token_kernel<T, G, NORM, CHAIN, 5>), grid, 256, 0, stream, a, tokens);
  } else {
    launch_k((rope_token_kernel<T, G, NORM, CHAIN, 4>), grid, 256, 0, stream, a, tokens);
  }
  return launch_status();
}

template <typename T, bool NORM, bool CHAIN>
int launch_rope(const RopeArgs& a, uint32_t units, cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<T>::kVec;
  const int64_t half = a.D / 2;
  auto strides_ok = [&](const int64_t* s) {
    return s[0] % VW == 0 && s[1] % VW == 0 && s[2] % VW == 0;
  };
  bool vec_ok = half % VW == 0 && aligned16(a.q) && aligned16(a.qo) &&
                aligned16(a.cos) && aligned16(a.sin) && strides_ok(a.sq) &&
                strides_ok(a.soq) && a.scb % VW == 0 && a.scs % VW == 0;
  if (a.Hk > 0)
    vec_ok = vec_ok && aligned16(a.k) && aligned16(a.ko) && strides_ok(a.sk) &&
             strides_ok(a.sok);
  if (NORM) vec_ok = vec_ok && aligned16(a.wq) && (a.Hk == 0 || aligned16(a.wk));
  if (vec_ok) {
    const int64_t g = half / VW;
    switch (g) {
      case 1: return launch_vec<T, 1, NORM, CHAIN>(a, units, dev, stream);
      case 2: return launch_vec<T, 2, NORM, CHAIN>(a, units, dev, stream);
      case 4: return launch_token<T, 4, NORM, CHAIN>(a, units / (a.Hq + a.Hk), stream);
      case 8: return launch_token<T, 8, NORM, CHAIN>(a, units / (a.Hq + a.Hk), stream);
      case 16: return launch_token<T, 16, NORM, CHAIN>(a, units / (a.Hq + a.Hk), stream);
      case 32: return launch_vec<T, 32, NORM, CHAIN>(a, units, dev, stream);
      default: break;
    }
  }
  auto kern = rope_scalar_kernel<T, NORM, CHAIN>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int64_t blocks = ceil_div(units, 8);
  const int grid = (int)std::min<int64_t>(blocks, (int64_t)per_sm * dev.sm_count);
  launch_k(kern, grid, 256, 0, stream, a, units);
  return launch_status();
}

template <bool NORM>
int rope_entry(RopeArgs& a, int64_t Hq, int64_t Hk, int64_t B, int64_t S, int64_t D,
               int dtype, int rounding, cudaStream_t stream) {
  FLB_CHECK_ARG(Hq >= 0 && Hk >= 0 && B >= 0 && S >= 0 && D >= 0);
  FLB_CHECK_ARG(rounding == FL_B200_ROUND_FUSED || rounding == FL_B200_ROUND_CHAIN);
  if (a.k == nullptr) Hk = 0;
  const int64_t units = B * S * (Hq + Hk);
  if (units == 0 || D == 0) return FL_B200_OK;
  FLB_CHECK_ARG(D % 2 == 0);
  FLB_CHECK_ARG(units < (int64_t(1) << 31) && B * S < (int64_t(1) << 31) && D < (1 << 30));
  FLB_CHECK_ARG(a.cos && a.sin);
  FLB_CHECK_ARG(Hq == 0 || (a.q && a.qo));
  FLB_CHECK_ARG(Hk == 0 || (a.k && a.ko));
  FLB_CHECK_ARG(!NORM || ((Hq == 0 || a.wq) && (Hk == 0 || a.wk)));
  a.Hq = (uint32_t)Hq;
  a.Hk = (uint32_t)Hk;
  a.S = (uint32_t)S;
  a.D = (uint32_t)D;
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    if (rounding == FL_B200_ROUND_CHAIN)
      return launch_rope<T, NORM, true>(a, (uint32_t)units, stream);
    return launch_rope<T, NORM, false>(a, (uint32_t)units, stream);
  });
}

RopeArgs make_args(const void* q, void* q_out, int64_t sqb, int64_t sqh, int64_t sqs,
                   int64_t soqb, int64_t soqh, int64_t soqs, const void* wq,
                   const void* k, void* k_out, int64_t skb, int64_t skh, int64_t sks,
                   int64_t sokb, int64_t sokh, int64_t soks, const void* wk,
                   const void* cos, const void* sin, int64_t scb, int64_t scs,
                   float eps) {
  RopeArgs a{};
  a.q = q;
  a.qo = q_out;
  a.k = k;
  a.ko = k_out;
  a.wq = wq;
  a.wk = wk;
  a.cos = cos;
  a.sin = sin;
  a.sq[0] = sqb, a.sq[1] = sqh, a.sq[2] = sqs;
  a.soq[0] = soqb, a.soq[1] = soqh, a.soq[2] = soqs;
  a.sk[0] = skb, a.sk[1] = skh, a.sk[2] = sks;
  a.sok[0] = sokb, a.sok[1] = sokh, a.sok[2] = soks;
  a.scb = scb;
  a.scs = scs;
  a.eps = eps;
  return a;
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API int fl_b200_rope_qk(const void* q, void* q_out, int64_t Hq, int64_t sqb,
                                int64_t sqh, int64_t sqs, int64_t soqb, int64_t soqh,
                                int64_t soqs, const void* k, void* k_out, int64_t Hk,
                                int64_t skb, int64_t skh, int64_t sks, int64_t sokb,
                                int64_t sokh, int64_t soks, const void* cos,
                                const void* sin, int64_t scb, int64_t scs, int64_t B,
                                int64_t S, int64_t D, int dtype, int rounding,
                                fl_b200_stream_t stream) {
  auto a = flb200::make_args(q, q_out, sqb, sqh, sqs, soqb, soqh, soqs, nullptr, k,
                             k_out, skb, skh, sks, sokb, sokh, soks, nullptr, cos, sin,
                             scb, scs, 0.f);
  return flb200::rope_entry<false>(a, Hq, Hk, B, S, D, dtype, rounding,
                                   static_cast<cudaStream_t>(stream));
}

FL_B200_API int fl_b200_rms_norm_rope(
    const void* q, void* q_out, int64_t Hq, int64_t sqb, int64_t sqh, int64_t sqs,
    int64_t soqb, int64_t soqh, int64_t soqs, const void* wq, const void* k,
    void* k_out, int64_t Hk, int64_t skb, int64_t skh, int64_t sks, int64_t sokb,
    int64_t sokh, int64_t soks, const void* wk, const void* cos, const void* sin,
    int64_t scb, int64_t scs, int64_t B, int64_t S, int64_t D, float eps, int dtype,
    int rounding, fl_b200_stream_t stream) {
  auto a = flb200::make_args(q, q_out, sqb, sqh, sqs, soqb, soqh, soqs, wq, k, k_out,
                             skb, skh, sks, sokb, sokh, soks, wk, cos, sin, scb, scs,
                             eps);
  return flb200::rope_entry<true>(a, Hq, Hk, B, S, D, dtype, rounding,
                                  static_cast<cudaStream_t>(stream));
}

}  // extern "C"
