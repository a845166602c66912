// Backward kernels for training through the fused ops: RMSNorm, SwiGLU,
// SiLU and last-dim softmax.
//
// Reference behaviour: the reference registers one backward kernel on this
// path, silu_backward (csrc/aten/register.cc:329-331, 427 ->
// csrc/aten/backends/cuda/silu_backward.cu:15-35: grad * s * (1 + x(1-s)),
// s = sigmoid(x), in the op-math type).  _softmax_backward_data is not
// registered and runs in the CPU fallback (register.cc:439-442 ->
// fallback.cc:12-14); RMSNorm's backward is autograd over the HF chain
// (modeling_qwen3.py:59-64: pow, mean, add, rsqrt, mul, casts), each op a
// separate launch.  Here each backward is one pass over its rows.
//
// RMSNorm, out = w * x * r with r = 1/sqrt(mean(x^2) + eps) and n = x * r:
//   dx_j = r * (w_j dy_j - n_j * (1/H) * sum_i w_i dy_i n_i)
//   dw_j = sum over rows of dy_j n_j
// SwiGLU, out = silu(g) * u:  du = dout * silu(g),
//   dg = dout * u * s * (1 + g (1 - s)),  s = sigmoid(g)
// Softmax, y = softmax(x):  dx_j = y_j (dy_j - sum_i dy_i y_i)
// All in fp32, rounded once to the output dtype.
#include "row_ladder.cuh"

namespace flb200 {
namespace {

// ---- RMSNorm backward -------------------------------------------------------
// A persistent CTA owns row groups blockIdx.x, blockIdx.x + gridDim.x, ...
// (a fixed assignment), writes dx for each row and keeps the running dw
// partial of its columns in registers; at the end the row slots of the CTA
// are added in slot order and the CTA's partial row goes to the workspace.
// A second kernel adds the partial rows in CTA order.  Both orders are
// fixed, so dw does not depend on timing.  The next row's x and dy are
// loaded while the current row is reduced and stored (two row buffers in
// registers, 3 CTAs per SM; for 4096-wide 16-bit rows the next row goes to
// shared memory instead, STAGE): measured on B200, bf16 [65536, 4096] 5.73
// vs 5.44 TB/s with one buffer at 4 CTAs per SM.  Rows of 257..512 packs run
// 128 threads x 4 packs (two rows per CTA) at 2 CTAs per SM: 6.12 vs 5.92
// TB/s for 256 x 2 at 3 CTAs (bf16 4096-wide rows, kernel alone).
constexpr int kBwdCtasPerSm = 3;

template <int BLOCK, int VPT>
constexpr int rms_bwd_min_blocks() {
  return BLOCK <= 256 ? (VPT >= 4 ? 2 : kBwdCtasPerSm) : 1;
}
// A CTA writes one dw partial row per row slot (one-slot CTAs, and the two
// slots of the 2-CTA rung: at most 4 partial rows per SM), else one row with
// its slots added in slot order.
template <int RPB, int VPT>
__host__ __device__ constexpr bool rms_bwd_slot_rows() {
  return RPB == 1 || (RPB == 2 && VPT >= 4);
}

template <typename T, int TPR, int VPT, int BLOCK, bool STAGE, int MINB>
__global__ void __launch_bounds__(BLOCK, MINB)
rms_norm_bwd_kernel(const T* __restrict__ dy, int64_t lddy, const T* __restrict__ x,
                    int64_t ldx, const T* __restrict__ w, T* __restrict__ dx, int64_t lddx,
                    float* __restrict__ partial, int64_t rows, int nvec, float eps,
                    float cols_f) {
  constexpr int VW = Elem<T>::kVec;
  constexpr int RPB = BLOCK / TPR;
  __shared__ float red[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  float acc[VPT][VW];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int e = 0; e < VW; ++e) acc[i][e] = 0.f;
  auto load = [&](int64_t row, uint4 (&xv)[VPT], uint4 (&gv)[VPT]) {
    const bool ok = row < rows;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      const bool in = ok && vi < nvec;
      xv[i] = in ? ld_stream(x + row * ldx + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
      gv[i] = in ? ld_stream(dy + row * lddy + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
    }
  };
  // STAGE: the next row's x and dy packs copied into shared memory
  // ([pack][thread]) by cp.async instead of held in a second set of registers
  extern __shared__ uint4 stage[];
  auto issue = [&](int64_t row) {
    if (row < rows) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lane + i * TPR;
        if (vi < nvec) {
          cp_async16(&stage[i * BLOCK + threadIdx.x], x + row * ldx + (int64_t)vi * VW);
          cp_async16(&stage[(VPT + i) * BLOCK + threadIdx.x], dy + row * lddy + (int64_t)vi * VW);
        }
      }
    }
    cp_async_commit();
  };
  auto take = [&](int64_t row, uint4 (&xv)[VPT], uint4 (&gv)[VPT]) {
    cp_async_wait_all();
    const bool ok = row < rows;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const bool in = ok && lane + i * TPR < nvec;
      xv[i] = in ? stage[i * BLOCK + threadIdx.x] : make_uint4(0, 0, 0, 0);
      gv[i] = in ? stage[(VPT + i) * BLOCK + threadIdx.x] : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 xv[VPT], gv[VPT];
  int64_t base = (int64_t)blockIdx.x * RPB;
  if constexpr (STAGE) issue(base + slot);
  else load(base + slot, xv, gv);
  __shared__ float2 sums[TPR > 32 ? 2 * BLOCK / 32 : 1];
  int parity = 0;
  for (; base < rows; base += (int64_t)gridDim.x * RPB, parity ^= 1) {
    const int64_t row = base + slot;
    const bool ok = row < rows;
    uint4 xn[VPT], gn[VPT];
    if constexpr (STAGE) {
      take(row, xv, gv);
      issue(base + (int64_t)gridDim.x * RPB + slot);  // the next row, in flight meanwhile
    } else {
      load(base + (int64_t)gridDim.x * RPB + slot, xn, gn);  // the next row, in flight meanwhile
    }
    float ss = 0.f, tx = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      float xf[VW], gf[VW], wf[VW];
      unpack<T>(xv[i], xf);
      unpack<T>(gv[i], gf);
      unpack<T>(vi < nvec ? ld_cached(w + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0), wf);
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        ss = fmaf(xf[e], xf[e], ss);
        tx = fmaf(wf[e] * gf[e], xf[e], tx);
      }
    }
    if constexpr (TPR > 32) {
      // both sums in one exchange among the row's warps (named barrier)
      row_sum2_named<TPR, BLOCK>(ss, tx, sums, parity);
    } else {
      ss = row_reduce<SumOp, TPR, BLOCK>(ss, red);
      tx = row_reduce<SumOp, TPR, BLOCK>(tx, red);
    }
    const float r = 1.0f / sqrtf(ss / cols_f + eps);
    const float m = tx * r / cols_f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (!ok || vi >= nvec) continue;
      float xf[VW], gf[VW], wf[VW], o[VW];
      unpack<T>(opaque(xv[i]), xf);
      unpack<T>(opaque(gv[i]), gf);
      unpack<T>(ld_cached(w + (int64_t)vi * VW), wf);
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const float n = xf[e] * r;
        o[e] = r * (wf[e] * gf[e] - n * m);
        acc[i][e] = fmaf(gf[e], n, acc[i][e]);
      }
      st_stream(dx + row * lddx + (int64_t)vi * VW, pack<T>(o));
    }
    if constexpr (!STAGE) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        xv[i] = xn[i];
        gv[i] = gn[i];
      }
    }
  }
  if constexpr (STAGE) cp_async_wait_all();
  if (partial == nullptr) return;
  if constexpr (rms_bwd_slot_rows<RPB, VPT>()) {
    // one partial row per row slot, in (CTA, slot) order
    float* out = partial + ((int64_t)blockIdx.x * RPB + slot) * nvec * VW;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (vi < nvec)
#pragma unroll
        for (int e = 0; e < VW; ++e) out[(int64_t)vi * VW + e] = acc[i][e];
    }
  } else {
    // the CTA's row slots added in slot order into one partial row
    float* out = partial + (int64_t)blockIdx.x * nvec * VW;
    __shared__ float part[BLOCK * VPT * VW];
#pragma unroll
    for (int i = 0; i < VPT; ++i)
#pragma unroll
      for (int e = 0; e < VW; ++e) part[(i * VW + e) * BLOCK + threadIdx.x] = acc[i][e];
    __syncthreads();
    if (slot == 0) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lane + i * TPR;
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          float s = 0.f;
          for (int k = 0; k < RPB; ++k) s += part[(i * VW + e) * BLOCK + k * TPR + lane];
          if (vi < nvec) out[(int64_t)vi * VW + e] = s;
        }
      }
    }
  }
}

// Any row length and alignment: one thread per column block of a row, the
// CTA's dw partial row accumulated in place in the workspace (each column
// is read-modify-written by one thread only).  The row is read twice.
template <typename T>
__global__ void __launch_bounds__(256)
rms_norm_bwd_loop_kernel(const T* dy, int64_t lddy, const T* x, int64_t ldx, const T* w,
                         T* dx, int64_t lddx, float* partial, int64_t rows, int64_t cols,
                         float eps) {
  __shared__ float red[256 / 32];
  float* part = partial ? partial + (int64_t)blockIdx.x * cols : nullptr;
  if (part)
    for (int64_t c = threadIdx.x; c < cols; c += 256) part[c] = 0.f;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * ldx;
    const T* gr = dy + row * lddy;
    float ss = 0.f, tx = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float xf = Elem<T>::to_f(xr[c]);
      ss = fmaf(xf, xf, ss);
      tx = fmaf(Elem<T>::to_f(w[c]) * Elem<T>::to_f(gr[c]), xf, tx);
    }
    ss = block_reduce<SumOp, 256>(ss, red);
    tx = block_reduce<SumOp, 256>(tx, red);
    const float r = 1.0f / sqrtf(ss / (float)cols + eps);
    const float m = tx * r / (float)cols;
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float g = Elem<T>::to_f(gr[c]);
      const float n = Elem<T>::to_f(xr[c]) * r;
      dx[row * lddx + c] = Elem<T>::from_f(r * (Elem<T>::to_f(w[c]) * g - n * m));
      if (part) part[c] = fmaf(g, n, part[c]);
    }
  }
}

// dw[c] = sum over p < P of partial[p][c] in a fixed order.  A CTA covers 32
// columns as 8 float4 lanes x 32 chunks of the partial rows; each thread
// keeps 4 independent running sums per column over its chunk (the loads of
// a chunk in flight together: the partials come from L2, so the time is
// latency, not bytes), then the 32 chunks are added in chunk order through
// shared memory.  Measured on B200 (296 partial rows x 4096 columns, fp32):
// the previous one-load-at-a-time form took 15.7 us.
template <typename T>
__global__ void __launch_bounds__(256)
rms_norm_dw_reduce_kernel(const float* __restrict__ partial, int64_t P, int64_t cols,
                          T* __restrict__ dw) {
  __shared__ float4 s[32][9];
  const int q = threadIdx.x & 7, ch = threadIdx.x >> 3;  // float4 lane, chunk
  const int64_t c = (int64_t)blockIdx.x * 32 + q * 4;     // first of 4 columns
  const int64_t per = ceil_div(P, 32);
  const int64_t p0 = ch * per, p1 = min(P, p0 + per);
  float4 acc[4] = {};
  if (c < cols) {  // cols % 4 == 0 (the vector path), so c + 3 < cols too
    int64_t p = p0;
    for (; p + 3 < p1; p += 4) {
      float4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        v[k] = *reinterpret_cast<const float4*>(partial + (p + k) * cols + c);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[k].x += v[k].x;
        acc[k].y += v[k].y;
        acc[k].z += v[k].z;
        acc[k].w += v[k].w;
      }
    }
    for (; p < p1; ++p) {
      const float4 v = *reinterpret_cast<const float4*>(partial + p * cols + c);
      acc[0].x += v.x;
      acc[0].y += v.y;
      acc[0].z += v.z;
      acc[0].w += v.w;
    }
  }
  float4 t = acc[0];
#pragma unroll
  for (int k = 1; k < 4; ++k) {
    t.x += acc[k].x;
    t.y += acc[k].y;
    t.z += acc[k].z;
    t.w += acc[k].w;
  }
  s[ch][q] = t;
  __syncthreads();
  if (ch == 0 && c < cols) {
    float4 r = s[0][q];
    for (int k = 1; k < 32; ++k) {
      r.x += s[k][q].x;
      r.y += s[k][q].y;
      r.z += s[k][q].z;
      r.w += s[k][q].w;
    }
    dw[c] = Elem<T>::from_f(r.x);
    dw[c + 1] = Elem<T>::from_f(r.y);
    dw[c + 2] = Elem<T>::from_f(r.z);
    dw[c + 3] = Elem<T>::from_f(r.w);
  }
}

// The same for any column count (the scalar backward's partial rows): one
// column per thread, 8 chunks of the partial rows added in chunk order.
template <typename T>
__global__ void __launch_bounds__(256)
rms_norm_dw_reduce_scalar_kernel(const float* __restrict__ partial, int64_t P, int64_t cols,
                                 T* __restrict__ dw) {
  __shared__ float s[8][33];
  const int cl = threadIdx.x & 31, ch = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + cl;
  const int64_t per = ceil_div(P, 8);
  const int64_t p0 = ch * per, p1 = min(P, p0 + per);
  float acc = 0.f;
  if (c < cols)
    for (int64_t p = p0; p < p1; ++p) acc += partial[p * cols + c];
  s[ch][cl] = acc;
  __syncthreads();
  if (ch == 0 && c < cols) {
    float t = s[0][cl];
#pragma unroll
    for (int k = 1; k < 8; ++k) t += s[k][cl];
    dw[c] = Elem<T>::from_f(t);
  }
}

// Rows of partials the backward uses on this device (an upper bound: the
// workspace is sized from it, a launch may use fewer): 3 CTAs of one row
// slot, or 2 CTAs of two slots, per SM.
int64_t rms_bwd_max_partials(const DeviceInfo& dev) { return (int64_t)dev.sm_count * 4; }

template <typename T>
int launch_rms_norm_bwd(const T* dy, int64_t lddy, const T* x, int64_t ldx, const T* w,
                        T* dx, int64_t lddx, T* dw, int64_t rows, int64_t cols, float eps,
                        float* partial, const DeviceInfo& dev, cudaStream_t stream) {
  constexpr int VW = Elem<T>::kVec;
  int64_t used = 0;  // partial rows written
  const bool vec_ok = aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx) &&
                      cols % VW == 0 && lddy % VW == 0 && ldx % VW == 0 && lddx % VW == 0;
  int st = -1;
  if (vec_ok) {
    auto go = [&](auto tpr, auto vpt) -> int {
      constexpr int TPR = decltype(tpr)::value;
      constexpr int VPT = decltype(vpt)::value;
      constexpr int BLOCK = ladder_block<TPR>();
      constexpr int RPB = BLOCK / TPR;
      const int64_t groups = ceil_div(rows, RPB);
      const int64_t ctas =
          std::min<int64_t>(groups, (int64_t)dev.sm_count * rms_bwd_min_blocks<BLOCK, VPT>());
      used = ctas * (rms_bwd_slot_rows<RPB, VPT>() ? RPB : 1);
      rms_norm_bwd_kernel<T, TPR, VPT, BLOCK, false, rms_bwd_min_blocks<BLOCK, VPT>()>
          <<<(int)ctas, BLOCK, 0, stream>>>(dy, lddy, x, ldx, w, dx, lddx, partial, rows,
                                            (int)(cols / VW), eps, (float)cols);
      return launch_status();
    };
    const int64_t nvec = cols / VW;
    if (nvec > 256 && nvec <= 512) {
      // 128 threads x 4 packs, two rows per CTA, 2 CTAs per SM, the next row's
      // x and dy staged in shared memory (32 KB a CTA) by cp.async.  Measured on
      // B200, bf16 [65536, 4096]: 0.257 ms against 0.263 with the next row in
      // registers; 3 CTAs per SM (80 registers) spills and takes 0.278 ms.
      constexpr int MINB = 2;
      auto kern = rms_norm_bwd_kernel<T, 128, 4, 256, true, MINB>;
      const size_t smem = (size_t)2 * 4 * 256 * 16;
      const int64_t ctas = std::min<int64_t>(ceil_div(rows, 2), (int64_t)dev.sm_count * MINB);
      used = ctas * 2;
      kern<<<(int)ctas, 256, smem, stream>>>(dy, lddy, x, ldx, w, dx, lddx, partial, rows,
                                             (int)nvec, eps, (float)cols);
      st = launch_status();
    } else {
      st = row_ladder<2>(nvec, go);
    }
  }
  if (st < 0) {
    used = std::min<int64_t>(rows, (int64_t)dev.sm_count * kBwdCtasPerSm);
    rms_norm_bwd_loop_kernel<T><<<(int)used, 256, 0, stream>>>(dy, lddy, x, ldx, w, dx, lddx,
                                                              partial, rows, cols, eps);
    st = launch_status();
  }
  if (st != FL_B200_OK || dw == nullptr) return st;
  if (cols % 4 == 0 && aligned16(partial)) {
    rms_norm_dw_reduce_kernel<T><<<(int)ceil_div(cols, 32), 256, 0, stream>>>(partial, used,
                                                                              cols, dw);
  } else {
    rms_norm_dw_reduce_scalar_kernel<T><<<(int)ceil_div(cols, 32), 256, 0, stream>>>(
        partial, used, cols, dw);
  }
  return launch_status();
}

// ---- SwiGLU / SiLU backward -------------------------------------------------
__device__ __forceinline__ float sigmoid_f(float g) { return 1.0f / (1.0f + __expf(-g)); }

// MODE 0: SwiGLU (a = dout, b = gate, c = up -> o1 = dgate, o2 = dup);
// MODE 1: SiLU   (a = dout, b = x -> o1 = dx).
template <int MODE>
__device__ __forceinline__ void silu_bwd_elem(float d, float g, float u, float& o1,
                                              float& o2) {
  const float s = sigmoid_f(g);
  const float ds = s * (1.0f + g * (1.0f - s));  // d silu / d g
  if (MODE == 0) {
    o1 = d * u * ds;
    o2 = d * g * s;
  } else {
    o1 = d * ds;
  }
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256)
silu_bwd_vec_kernel(const T* __restrict__ a, const T* __restrict__ b, const T* __restrict__ c,
                    T* __restrict__ o1, T* __restrict__ o2, int64_t npacks) {
  constexpr int VW = Elem<T>::kVec;
  const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (p >= npacks) return;
  float fa[VW], fb[VW], fc[VW], r1[VW], r2[VW];
  unpack<T>(ld_stream(a + p * VW), fa);
  unpack<T>(ld_stream(b + p * VW), fb);
  if (MODE == 0) unpack<T>(ld_stream(c + p * VW), fc);
#pragma unroll
  for (int e = 0; e < VW; ++e)
    silu_bwd_elem<MODE>(fa[e], fb[e], MODE == 0 ? fc[e] : 0.f, r1[e], r2[e]);
  st_stream(o1 + p * VW, pack<T>(r1));
  if (MODE == 0) st_stream(o2 + p * VW, pack<T>(r2));
}

template <typename T, int MODE>
__global__ void __launch_bounds__(256)
silu_bwd_scalar_kernel(const T* a, const T* b, const T* c, T* o1, T* o2, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * 256) {
    float r1, r2;
    silu_bwd_elem<MODE>(Elem<T>::to_f(a[i]), Elem<T>::to_f(b[i]),
                        MODE == 0 ? Elem<T>::to_f(c[i]) : 0.f, r1, r2);
    o1[i] = Elem<T>::from_f(r1);
    if (MODE == 0) o2[i] = Elem<T>::from_f(r2);
  }
}

template <typename T, int MODE>
int launch_silu_bwd(const T* a, const T* b, const T* c, T* o1, T* o2, int64_t n,
                    cudaStream_t stream) {
  constexpr int VW = Elem<T>::kVec;
  const bool vec = n % VW == 0 && aligned16(a) && aligned16(b) && aligned16(o1) &&
                   (MODE == 1 || (aligned16(c) && aligned16(o2)));
  if (vec) {
    const int64_t npacks = n / VW;
    silu_bwd_vec_kernel<T, MODE><<<full_grid(ceil_div(npacks, 256)), 256, 0, stream>>>(
        a, b, c, o1, o2, npacks);
  } else {
    DeviceInfo dev;
    int st = current_device_info(&dev);
    if (st != FL_B200_OK) return st;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(n, 256), (int64_t)dev.sm_count * 8));
    silu_bwd_scalar_kernel<T, MODE><<<grid, 256, 0, stream>>>(a, b, c, o1, o2, n);
  }
  return launch_status();
}

// ---- softmax backward -------------------------------------------------------
template <typename TO, int VW>
__device__ __forceinline__ void store_vals_bwd(TO* o, const float (&v)[VW]) {
  constexpr int OW = Elem<TO>::kVec;
  if constexpr (OW >= VW) {
    // a narrower output: VW values fill part of one output pack
    static_assert(OW % VW == 0, "pack widths");
  }
#pragma unroll
  for (int k = 0; k < VW / OW; ++k) {
    float t[OW];
#pragma unroll
    for (int e = 0; e < OW; ++e) t[e] = v[k * OW + e];
    st_stream(o + k * OW, pack<TO>(t));
  }
}

// Rows in registers: dy and y packs, one dot product, one store pass.  The
// output may be narrower than the inputs (fp32 grads of a half_to_float
// softmax back to 16 bits); then each thread handles two input packs per
// output pack.
template <typename TI, typename TO, int TPR, int VPT, int BLOCK>
__global__ void __launch_bounds__(BLOCK, ladder_min_blocks<BLOCK>())
softmax_bwd_vec_kernel(const TI* __restrict__ dy, int64_t lddy, const TI* __restrict__ y,
                       int64_t ldy, TO* __restrict__ dx, int64_t lddx, int64_t rows,
                       int nvec, float scale) {
  constexpr int VW = Elem<TI>::kVec;
  constexpr int RPB = BLOCK / TPR;
  __shared__ float red[BLOCK / 32];
  const int slot = threadIdx.x / TPR;
  const int lane = threadIdx.x % TPR;
  for (int64_t base = (int64_t)blockIdx.x * RPB; base < rows;
       base += (int64_t)gridDim.x * RPB) {
    const int64_t row = base + slot;
    const bool ok = row < rows;
    uint4 gv[VPT], yv[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      const bool in = ok && vi < nvec;
      gv[i] = in ? ld_stream(dy + row * lddy + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
      yv[i] = in ? ld_stream(y + row * ldy + (int64_t)vi * VW) : make_uint4(0, 0, 0, 0);
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float gf[VW], yf[VW];
      unpack<TI>(gv[i], gf);
      unpack<TI>(yv[i], yf);
#pragma unroll
      for (int e = 0; e < VW; ++e) dot = fmaf(gf[e], yf[e], dot);
    }
    dot = row_reduce<SumOp, TPR, BLOCK>(dot, red);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lane + i * TPR;
      if (!ok || vi >= nvec) continue;
      float gf[VW], yf[VW], o[VW];
      unpack<TI>(opaque(gv[i]), gf);
      unpack<TI>(opaque(yv[i]), yf);
#pragma unroll
      for (int e = 0; e < VW; ++e) o[e] = yf[e] * (gf[e] - dot) * scale;
      TO* dst = dx + row * lddx + (int64_t)vi * VW;
      if constexpr (Elem<TO>::kVec <= VW) {
        store_vals_bwd<TO, VW>(dst, o);
      } else {
        // TI = f32 (4 per pack), TO 16-bit (8 per pack): half a pack each
        float t[Elem<TO>::kVec];
#pragma unroll
        for (int e = 0; e < Elem<TO>::kVec; ++e) t[e] = e < VW ? o[e] : 0.f;
        const uint4 pk = pack<TO>(t);
        *reinterpret_cast<uint2*>(dst) = make_uint2(pk.x, pk.y);
      }
    }
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
softmax_bwd_loop_kernel(const TI* dy, int64_t lddy, const TI* y, int64_t ldy, TO* dx,
                        int64_t lddx, int64_t rows, int64_t cols, float scale) {
  __shared__ float red[256 / 32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const TI* gr = dy + row * lddy;
    const TI* yr = y + row * ldy;
    float dot = 0.f;
    for (int64_t c = threadIdx.x; c < cols; c += 256)
      dot = fmaf(Elem<TI>::to_f(gr[c]), Elem<TI>::to_f(yr[c]), dot);
    dot = block_reduce<SumOp, 256>(dot, red);
    for (int64_t c = threadIdx.x; c < cols; c += 256) {
      const float v = Elem<TI>::to_f(yr[c]) * (Elem<TI>::to_f(gr[c]) - dot) * scale;
      if constexpr (std::is_same<TO, float>::value) dx[row * lddx + c] = v;
      else dx[row * lddx + c] = Elem<TO>::from_f(v);
    }
  }
}

template <typename TI, typename TO>
int launch_softmax_bwd(const TI* dy, int64_t lddy, const TI* y, int64_t ldy, TO* dx,
                       int64_t lddx, int64_t rows, int64_t cols, float scale,
                       cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  constexpr int VW = Elem<TI>::kVec;
  // a store of VW outputs must start on a 16-byte boundary (8 bytes when a
  // 4-wide fp32 pack becomes half a 16-bit pack)
  constexpr int64_t kOutAlign = (int64_t)VW * sizeof(TO) >= 16 ? 16 : (int64_t)VW * sizeof(TO);
  const bool vec_ok = aligned16(dy) && aligned16(y) &&
                      (reinterpret_cast<uintptr_t>(dx) % kOutAlign) == 0 && cols % VW == 0 &&
                      lddy % VW == 0 && ldy % VW == 0 && lddx % VW == 0;
  if (vec_ok) {
    const int r = row_ladder<2>(cols / VW, [&](auto tpr, auto vpt) -> int {
      constexpr int TPR = decltype(tpr)::value;
      constexpr int VPT = decltype(vpt)::value;
      constexpr int BLOCK = ladder_block<TPR>();
      softmax_bwd_vec_kernel<TI, TO, TPR, VPT, BLOCK>
          <<<full_grid(ceil_div(rows, BLOCK / TPR)), BLOCK, 0, stream>>>(
              dy, lddy, y, ldy, dx, lddx, rows, (int)(cols / VW), scale);
      return launch_status();
    });
    if (r >= 0) return r;
  }
  auto kern = softmax_bwd_loop_kernel<TI, TO>;
  static const int per_sm = blocks_per_sm(kern, 256, 0);
  const int grid = (int)std::min<int64_t>(rows, (int64_t)per_sm * dev.sm_count);
  kern<<<grid, 256, 0, stream>>>(dy, lddy, y, ldy, dx, lddx, rows, cols, scale);
  return launch_status();
}

}  // namespace
}  // namespace flb200

extern "C" {

FL_B200_API size_t fl_b200_rms_norm_bwd_workspace_size(int64_t rows, int64_t cols) {
  using namespace flb200;
  if (rows <= 0 || cols <= 0) return 0;
  DeviceInfo dev;
  if (current_device_info(&dev) != FL_B200_OK) return 0;
  return (size_t)rms_bwd_max_partials(dev) * (size_t)cols * sizeof(float);
}

FL_B200_API int fl_b200_rms_norm_bwd(const void* dy, int64_t ld_dy, const void* x,
                                     int64_t ld_x, const void* w, void* dx, int64_t ld_dx,
                                     void* dw, int64_t rows, int64_t cols, float eps,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (cols == 0) return FL_B200_OK;
  auto s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (dw == nullptr) return FL_B200_OK;  // no rows: dw = 0
    const int sz = dtype_size(dtype);
    FLB_CHECK_ARG(sz > 0);
    return cudaMemsetAsync(dw, 0, (size_t)cols * sz, s) == cudaSuccess ? FL_B200_OK
                                                                       : FL_B200_ERR_LAUNCH;
  }
  FLB_CHECK_ARG(dy && x && w && dx && ld_dy >= cols && ld_x >= cols && ld_dx >= cols);
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != FL_B200_OK) return st;
  float* partial = nullptr;
  if (dw != nullptr) {
    const size_t need = (size_t)rms_bwd_max_partials(dev) * (size_t)cols * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
      return FL_B200_ERR_WORKSPACE;
    partial = static_cast<float*>(workspace);
  }
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return launch_rms_norm_bwd<T>(static_cast<const T*>(dy), ld_dy, static_cast<const T*>(x),
                                  ld_x, static_cast<const T*>(w), static_cast<T*>(dx), ld_dx,
                                  static_cast<T*>(dw), rows, cols, eps, partial, dev, s);
  });
}

FL_B200_API int fl_b200_swiglu_bwd(const void* dout, const void* gate, const void* up,
                                   void* dgate, void* dup, int64_t n, int dtype,
                                   fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n >= 0);
  if (n == 0) return FL_B200_OK;
  FLB_CHECK_ARG(dout && gate && up && dgate && dup);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return launch_silu_bwd<T, 0>(static_cast<const T*>(dout), static_cast<const T*>(gate),
                                 static_cast<const T*>(up), static_cast<T*>(dgate),
                                 static_cast<T*>(dup), n, static_cast<cudaStream_t>(stream));
  });
}

FL_B200_API int fl_b200_silu_bwd(const void* dout, const void* x, void* dx, int64_t n,
                                 int dtype, fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(n >= 0);
  if (n == 0) return FL_B200_OK;
  FLB_CHECK_ARG(dout && x && dx);
  return dispatch_float(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    return launch_silu_bwd<T, 1>(static_cast<const T*>(dout), static_cast<const T*>(x),
                                 nullptr, static_cast<T*>(dx), nullptr, n,
                                 static_cast<cudaStream_t>(stream));
  });
}

FL_B200_API int fl_b200_softmax_bwd_scaled(const void* dy, int64_t ld_dy, const void* y,
                                           int64_t ld_y, void* dx, int64_t ld_dx,
                                           int64_t rows, int64_t cols, float scale,
                                           int in_dtype, int out_dtype,
                                           fl_b200_stream_t stream) {
  using namespace flb200;
  FLB_CHECK_ARG(rows >= 0 && cols >= 0);
  if (rows == 0 || cols == 0) return FL_B200_OK;
  FLB_CHECK_ARG(dy && y && dx && ld_dy >= cols && ld_y >= cols && ld_dx >= cols);
  auto s = static_cast<cudaStream_t>(stream);
  auto go = [&](auto ti, auto to) -> int {
    using TI = decltype(ti);
    using TO = decltype(to);
    return launch_softmax_bwd<TI, TO>(static_cast<const TI*>(dy), ld_dy,
                                      static_cast<const TI*>(y), ld_y, static_cast<TO*>(dx),
                                      ld_dx, rows, cols, scale, s);
  };
  if (in_dtype == out_dtype) return dispatch_float(in_dtype, [&](auto t) { return go(t, t); });
  if (in_dtype == FL_B200_F32 && out_dtype == FL_B200_BF16) return go(float{}, __nv_bfloat16{});
  if (in_dtype == FL_B200_F32 && out_dtype == FL_B200_F16) return go(float{}, __half{});
  return FL_B200_ERR_UNSUPPORTED_DTYPE;
}

FL_B200_API int fl_b200_softmax_bwd(const void* dy, int64_t ld_dy, const void* y,
                                    int64_t ld_y, void* dx, int64_t ld_dx, int64_t rows,
                                    int64_t cols, int in_dtype, int out_dtype,
                                    fl_b200_stream_t stream) {
  return fl_b200_softmax_bwd_scaled(dy, ld_dy, y, ld_y, dx, ld_dx, rows, cols, 1.0f, in_dtype,
                                    out_dtype, stream);
}

}  // extern "C"
