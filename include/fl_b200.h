/*
 * fl_b200.h -- C ABI of libfl_b200.so, the B200 (sm_100a) kernel library behind
 * the `b200` route of the flagos PrivateUse1 device.
 *
 * Every entry point takes plain device pointers, element counts, leading
 * strides (in ELEMENTS), a dtype enum, scalar parameters and the CUDA stream
 * to launch on (passed as an opaque pointer; a cudaStream_t).  Nothing here
 * allocates device memory except where a function says so; nothing here
 * throws.  Each function returns an fl_b200_status code (0 = success).
 *
 * Launches go to the device that is current on the calling thread; the stream
 * must belong to that device.  All launches are asynchronous with respect to
 * the host.  Output buffers may alias their matching input buffer where a
 * function says "in place allowed".
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   the per-op C++ dispatcher function types in csrc/aten/<op>.h (e.g.
 *   csrc/aten/softmax.h:10) whose `cuda` implementations live in
 *   csrc/aten/backends/cuda/*.cu; the C error convention of
 *   include/flagos.h:17-23 (Error_t) is mirrored by fl_b200_status.
 */
#ifndef FL_B200_H_
#define FL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef FL_B200_API
#define FL_B200_API __attribute__((visibility("default")))
#endif

typedef void* fl_b200_stream_t; /* a cudaStream_t; NULL = legacy default stream */

typedef enum fl_b200_dtype {
  FL_B200_F32 = 0,
  FL_B200_BF16 = 1,
  FL_B200_F16 = 2,
  FL_B200_I32 = 3,
  FL_B200_I64 = 4
} fl_b200_dtype;

typedef enum fl_b200_status {
  FL_B200_OK = 0,
  FL_B200_ERR_INVALID_ARGUMENT = 1, /* bad shape / stride / null pointer      */
  FL_B200_ERR_UNSUPPORTED_DTYPE = 2,/* dtype (combination) not implemented    */
  FL_B200_ERR_MISALIGNED = 3,       /* pointer alignment a kernel requires    */
  FL_B200_ERR_LAUNCH = 4,           /* kernel launch failed (see cuda error)  */
  FL_B200_ERR_WORKSPACE = 5,        /* workspace missing or too small         */
  FL_B200_ERR_NO_DEVICE = 6,        /* no current CUDA device                 */
  FL_B200_ERR_TOO_LARGE = 7         /* size above a documented fixed maximum  */
} fl_b200_status;

/* Rounding policy for bf16/f16 results of the fused ops.
 *  FL_B200_ROUND_FUSED: compute in fp32, round once at the store (the default;
 *    within 1 ulp of the fp32-accumulated result).
 *  FL_B200_ROUND_CHAIN: round to the storage dtype after every step of the
 *    HuggingFace formula, exactly where the reference's op-by-op chain on the
 *    flagos device rounds (each aten op returns a bf16/f16 tensor).          */
typedef enum fl_b200_rounding {
  FL_B200_ROUND_FUSED = 0,
  FL_B200_ROUND_CHAIN = 1
} fl_b200_rounding;

/* Library identity and diagnostics. */
FL_B200_API int fl_b200_version(void);
FL_B200_API const char* fl_b200_status_string(int status);
/* Last CUDA error seen by a failed call on this thread (cudaError_t value). */
FL_B200_API int fl_b200_last_cuda_error(void);
/* Launch option, no counterpart in the reference (its cuda route launches    *
 * PyTorch's kernels with <<<>>>).  With enable != 0 (the default; the        *
 * environment variable FL_B200_PDL=0 turns it off at load) every kernel of   *
 * this library is launched with programmatic stream serialization: it may    *
 * begin while the previous kernel in the stream finishes, and waits on the   *
 * device (griddepcontrol.wait) before its first memory access, so results    *
 * are the same either way.  Process-wide; returns the previous setting.      */
FL_B200_API int fl_b200_set_pdl(int enable);

/* ------------------------------------------------------------------------ *
 * RMSNorm forward over the last dim:                                        *
 *   out[r, :] = w * (x[r, :] * rsqrt(mean(x[r, :]^2) + eps))               *
 * fp32 accumulation; x, w, out share `dtype` (F32/BF16/F16).                *
 * Replaces the HF formula (transformers models/qwen3/modeling_qwen3.py:     *
 * 59-64) as the reference runs it op by op on flagos: pow.Tensor_Scalar     *
 * (csrc/aten/backends/cuda/pow.cu:29-32), mean.dim (mean.cu:30-63),         *
 * add.Tensor (add.cu:72-76), rsqrt (rsqrt.cu:14-32), mul.Tensor             *
 * (mul.cu:28-52) and two _to_copy casts (csrc/aten/copy_ops.cc:225-240).    *
 * In place (out == x) allowed.                                              */
FL_B200_API int fl_b200_rms_norm_fwd(const void* x, int64_t ld_x, const void* w,
                                     void* out, int64_t ld_out, int64_t rows,
                                     int64_t cols, float eps, int dtype,
                                     int rounding, fl_b200_stream_t stream);

/* Fused residual add + RMSNorm (the decoder-layer prologue):                *
 *   h = x + y;  out = rmsnorm(h) * w.  h may alias x.  Replaces add.Tensor  *
 * (csrc/aten/backends/cuda/add.cu:48-84) followed by the RMSNorm chain.     */
FL_B200_API int fl_b200_add_rms_norm_fwd(const void* x, const void* y, void* h,
                                         const void* w, void* out, int64_t rows,
                                         int64_t cols, float eps, int dtype,
                                         int rounding, fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * RoPE on q and k (HF apply_rotary_pos_emb, modeling_qwen3.py:138-169):     *
 *   out = x * cos + rotate_half(x) * sin,                                   *
 *   rotate_half(x) = cat(-x[..., D/2:], x[..., :D/2]).                      *
 * q is addressed as q[b, h, s, d] = q + b*sqb + h*sqh + s*sqs + d           *
 * (element strides; d is contiguous), likewise k (Hk heads) and the         *
 * outputs; cos/sin as c[b, s, d] = cos + b*scb + s*scs + d (scb may be 0).  *
 * Replaces neg.cu:14-32, cat.cc:13-39, 2x mul.cu, add.cu per tensor.        *
 * In place (q_out == q, k_out == k) allowed.  k may be NULL (Hk ignored).   */
FL_B200_API int fl_b200_rope_qk(
    const void* q, void* q_out, int64_t Hq, int64_t sqb, int64_t sqh,
    int64_t sqs, int64_t soqb, int64_t soqh, int64_t soqs,
    const void* k, void* k_out, int64_t Hk, int64_t skb, int64_t skh,
    int64_t sks, int64_t sokb, int64_t sokh, int64_t soks,
    const void* cos, const void* sin, int64_t scb, int64_t scs,
    int64_t B, int64_t S, int64_t D, int dtype, int rounding,
    fl_b200_stream_t stream);

/* Per-head RMSNorm (Qwen3 q_norm / k_norm, modeling_qwen3.py:248-249,      *
 * 263-268) immediately followed by RoPE, in one pass.  Same addressing as  *
 * fl_b200_rope_qk; wq / wk are the [D] norm weights.  In place allowed.    */
FL_B200_API int fl_b200_rms_norm_rope(
    const void* q, void* q_out, int64_t Hq, int64_t sqb, int64_t sqh,
    int64_t sqs, int64_t soqb, int64_t soqh, int64_t soqs, const void* wq,
    const void* k, void* k_out, int64_t Hk, int64_t skb, int64_t skh,
    int64_t sks, int64_t sokb, int64_t sokh, int64_t soks, const void* wk,
    const void* cos, const void* sin, int64_t scb, int64_t scs,
    int64_t B, int64_t S, int64_t D, float eps, int dtype, int rounding,
    fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * SwiGLU: out = silu(gate) * up, silu(g) = g / (1 + exp(-g)).               *
 * Replaces silu.cu:15-35 followed by mul.cu:28-52 (HF Qwen3MLP,            *
 * modeling_qwen3.py:81-82).  Rows of `cols` elements with leading strides. *
 * In place (out == gate or out == up) allowed.                             */
FL_B200_API int fl_b200_swiglu(const void* gate, int64_t ld_g, const void* up,
                               int64_t ld_u, void* out, int64_t ld_out,
                               int64_t rows, int64_t cols, int dtype,
                               int rounding, fl_b200_stream_t stream);

/* SwiGLU over [rows, inter] and the residual add h = x + y over             *
 * [rows, hidden] in ONE launch (contiguous rows).  h may alias x.           */
FL_B200_API int fl_b200_swiglu_residual(const void* gate, const void* up,
                                        void* act, int64_t inter,
                                        const void* x, const void* y, void* h,
                                        int64_t hidden, int64_t rows, int dtype,
                                        int rounding, fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Broadcast binary ops, replacing add.cu:48-84 (a + alpha*b) and          *
 * mul.cu:28-52 (a*b) reached through register.cc:190-193 / 239-242.        *
 * Shapes are given already broadcast: `ndim` <= 8 dims of `sizes`, and     *
 * per-operand element strides (0 on a broadcast dim).  `out` is dense       *
 * row-major over `sizes`.  a, b, out share `dtype` (F32/BF16/F16/I32/I64);  *
 * float dtypes compute in fp32, integer dtypes in int64.  For I32/I64 the  *
 * alpha is truncated to an integer.                                        */
FL_B200_API int fl_b200_add(const void* a, const int64_t* a_strides,
                            const void* b, const int64_t* b_strides,
                            void* out, const int64_t* sizes, int ndim,
                            double alpha, int dtype, fl_b200_stream_t stream);
FL_B200_API int fl_b200_mul(const void* a, const int64_t* a_strides,
                            const void* b, const int64_t* b_strides,
                            void* out, const int64_t* sizes, int ndim,
                            int dtype, fl_b200_stream_t stream);
/* out = a op s for a scalar operand s (a CPU "wrapped number" in aten),     *
 * kept in fp32/int64 opmath and never rounded to `dtype` first            *
 * (add.cu:67-76).  a and out dense with n elements.  op: 0 = add           *
 * (a + alpha*s), 1 = mul (a*s).                                            */
FL_B200_API int fl_b200_binary_scalar(const void* a, double s, void* out,
                                      int64_t n, int op, double alpha,
                                      int dtype, fl_b200_stream_t stream);

/* Dense dtype conversion (replaces the host round trip of flagos->flagos   *
 * _to_copy, csrc/aten/copy_ops.cc:225-240).  Float->float rounds to        *
 * nearest-even; int->float rounds to nearest; float->int truncates toward *
 * zero (NaN/out-of-range give an unspecified value, as in C).              */
FL_B200_API int fl_b200_cast(const void* src, int src_dtype, void* dst,
                             int dst_dtype, int64_t n, fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * The other ops of the HF formulas, reached when the fused hooks are off:  *
 * one pass each, in the arithmetic of the reference's cuda route.          */
typedef enum {
  FL_B200_UNARY_SILU = 0,   /* x / (1 + exp(-x)) in fp32 (silu.cu:15-35)             */
  FL_B200_UNARY_RSQRT = 1,  /* rsqrtf (rsqrt.cu:14-32)                               */
  FL_B200_UNARY_NEG = 2,    /* -x; also int32/int64, two's complement (neg.cu:14-32) */
  FL_B200_UNARY_COS = 3,    /* cosf (cos.cu:14-32)                                   */
  FL_B200_UNARY_SIN = 4,    /* sinf (sin.cu:14-32)                                   */
  FL_B200_UNARY_SQUARE = 5, /* pow(x, 2) = x*x (pow.cu:29-32)                        */
  FL_B200_UNARY_CUBE = 6,   /* pow(x, 3) = x*x*x, the square rounded to the dtype    */
  FL_B200_UNARY_POW = 7     /* powf(x, p), p already rounded to the dtype (pow.cu:25) */
} fl_b200_unary_op;
/* Rows of `cols` contiguous elements, row r starting at x + offset(r):     *
 * r is split over row_sizes[0..row_ndim) (last fastest) and offset(r) is     *
 * the sum of the parts times row_strides (elements; up to 4 dims once size-1 *
 * dims are dropped and evenly stepping neighbours merged; HF's q[..., D/2:] *
 * of a transposed q fits).  out[r, j] = op(x[offset(r) + j]), out dense.     *
 * Replaces silu / rsqrt / neg / cos / sin / pow.Tensor_Scalar              *
 * (csrc/aten/register.cc:405-417 -> csrc/aten/backends/cuda/silu.cu,       *
 * rsqrt.cu, neg.cu, cos.cu, sin.cu, pow.cu).  Float dtypes; NEG also takes *
 * I32/I64.                                                                  */
FL_B200_API int fl_b200_unary(const void* x, const int64_t* row_sizes,
                              const int64_t* row_strides, int row_ndim, int64_t cols, void* out,
                              int op, double p, int dtype, fl_b200_stream_t stream);
/* Concatenation as row blocks: out[r, off_k + j] = srcs[k][offset_k(r) + j] *
 * for j < widths[k], off_k = widths[0] + ... + widths[k-1]; offset_k as in *
 * fl_b200_unary with the shared row_sizes and input k's strides            *
 * src_row_strides[k*row_ndim ..].  out dense: prod(row_sizes) rows of      *
 * sum(widths) elements of elem_size bytes.  A cat along dim d is this with *
 * row_sizes = the sizes before d and widths[k] = the product of input k's  *
 * sizes from d on (contiguous within each input).  Replaces cat            *
 * (csrc/aten/cat.cc:13-39 -> PyTorch's cat_out_cuda).                      */
FL_B200_API int fl_b200_cat(const void* const* srcs, const int64_t* src_row_strides,
                            const int64_t* widths, int n_inputs, const int64_t* row_sizes,
                            int row_ndim, void* out, int elem_size, fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Softmax over the last dim with fp32 accumulation, replacing _softmax      *
 * (register.cc:270-272 -> csrc/aten/backends/cuda/softmax.cc:14-40).       *
 * in_dtype F32/BF16/F16; out_dtype = in_dtype, or F32 (half_to_float).     *
 * causal != 0 applies the causal mask in the kernel: row r is query        *
 * i = r % q_len and sees keys j <= i + causal_offset; masked entries are   *
 * written as exact zeros and never read.  A row with no visible key is     *
 * all NaN, as softmax of an all -inf row is.                               */
FL_B200_API int fl_b200_softmax_lastdim(const void* x, int64_t ld_x, void* out,
                                        int64_t ld_out, int64_t rows,
                                        int64_t cols, int in_dtype,
                                        int out_dtype, int causal,
                                        int64_t q_len, int64_t causal_offset,
                                        fl_b200_stream_t stream);
/* Scaled, additively masked softmax over the last dim: the tail of HF's     *
 * eager attention (transformers models/qwen3/modeling_qwen3.py             *
 * eager_attention_forward: `attn_weights * scaling + attention_mask`,      *
 * softmax(dtype=float32), `.to(query.dtype)`; the reference runs it as     *
 * mul.cu:28-52, add.cu:48-84, _to_copy copy_ops.cc:225-240 and _softmax    *
 * register.cc:270-272 -> softmax.cc:14-40, one launch and one full-size    *
 * temporary each).  x holds rows = B*heads*q_len rows of `cols` keys, row  *
 * r = (b*heads + h)*q_len + i at x + r*ld_x.  mask (NULL: none) has x's     *
 * dtype; its row for (b, h, i) starts at mask + b*mask_stride_b +          *
 * h*mask_stride_h + i*mask_stride_q elements and is contiguous (stride 0   *
 * broadcasts: HF's [B, 1, Q, K] mask has mask_stride_h = 0).  FUSED        *
 * computes x*scale + mask in fp32; CHAIN rounds to in_dtype after the      *
 * scale and after the add, as the two aten ops do.  out_dtype = in_dtype   *
 * (the cast back fused) or F32.  A row whose keys are all masked with the  *
 * lowest finite value comes out uniform, as in the reference.              */
FL_B200_API int fl_b200_softmax_masked(const void* x, int64_t ld_x, const void* mask,
                                       int64_t mask_stride_b, int64_t mask_stride_h,
                                       int64_t mask_stride_q, void* out, int64_t ld_out,
                                       int64_t rows, int64_t cols, int64_t heads,
                                       int64_t q_len, float scale, int in_dtype,
                                       int out_dtype, int rounding,
                                       fl_b200_stream_t stream);
/* Softmax along a middle dim: x viewed dense as [outer, n, inner], softmax  *
 * over n for every (outer, inner).  Used for _softmax with dim != -1.      */
FL_B200_API int fl_b200_softmax_middim(const void* x, void* out, int64_t outer,
                                       int64_t n, int64_t inner, int in_dtype,
                                       int out_dtype, fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Reductions.  Replace sum.dim_IntList (register.cc:333-337 -> sum.cu:     *
 * 32-66), mean.dim (register.cc:248-252 -> mean.cu:30-63) and the          *
 * unregistered amax / argmax that the reference sends to the CPU fallback  *
 * (register.cc:439-442 -> fallback.cc:12-14).                              *
 * in_dtype F32/BF16/F16; sum also I32/I64 -> out I64 (exact); float sums   *
 * accumulate in fp32 inside a CTA and in fp64 across CTAs, so results are  *
 * deterministic run to run.  amax propagates NaN.                          *
 *                                                                           *
 * _lastdim: x is [rows, cols] with leading stride ld; out has rows          *
 * elements.  _all: x is dense with n elements; out has one element.        *
 * The workspace is device memory of at least fl_b200_reduce_workspace_size *
 * bytes (it may be NULL when that size is 0); calls that share one         *
 * workspace must be ordered on the GPU.                                    */
FL_B200_API size_t fl_b200_reduce_workspace_size(int64_t rows, int64_t cols);

FL_B200_API int fl_b200_reduce_sum_lastdim(const void* x, int64_t ld, int64_t rows,
                                           int64_t cols, void* out, int in_dtype,
                                           int out_dtype, void* workspace,
                                           size_t workspace_bytes,
                                           fl_b200_stream_t stream);
FL_B200_API int fl_b200_reduce_mean_lastdim(const void* x, int64_t ld, int64_t rows,
                                            int64_t cols, void* out, int in_dtype,
                                            int out_dtype, void* workspace,
                                            size_t workspace_bytes,
                                            fl_b200_stream_t stream);
FL_B200_API int fl_b200_reduce_amax_lastdim(const void* x, int64_t ld, int64_t rows,
                                            int64_t cols, void* out, int dtype,
                                            void* workspace, size_t workspace_bytes,
                                            fl_b200_stream_t stream);
FL_B200_API int fl_b200_reduce_sum_all(const void* x, int64_t n, void* out,
                                       int in_dtype, int out_dtype, void* workspace,
                                       size_t workspace_bytes,
                                       fl_b200_stream_t stream);
FL_B200_API int fl_b200_reduce_mean_all(const void* x, int64_t n, void* out,
                                        int in_dtype, int out_dtype, void* workspace,
                                        size_t workspace_bytes,
                                        fl_b200_stream_t stream);
FL_B200_API int fl_b200_reduce_amax_all(const void* x, int64_t n, void* out,
                                        int dtype, void* workspace,
                                        size_t workspace_bytes,
                                        fl_b200_stream_t stream);
/* Reduction over the middle dim of a dense [outer, n, inner] view (sum.dim / *
 * mean.dim / amax over a dim that is not the last).  op: 0 sum, 1 mean,     *
 * 2 amax.  out is dense [outer, inner].                                     */
FL_B200_API int fl_b200_reduce_middim(const void* x, int64_t outer, int64_t n,
                                      int64_t inner, void* out, int op,
                                      int in_dtype, int out_dtype,
                                      fl_b200_stream_t stream);
/* Index of the first maximum of each row (NaN counts as the maximum, the    *
 * first NaN wins), int64 output.  x: F32/BF16/F16 [rows, cols], stride ld. */
FL_B200_API int fl_b200_argmax_lastdim(const void* x, int64_t ld, int64_t rows,
                                       int64_t cols, int64_t* out, int dtype,
                                       void* workspace, size_t workspace_bytes,
                                       fl_b200_stream_t stream);
/* Exact int64 sum of int32 input.  full != 0: one int64 for the whole       *
 * [rows, cols] block; otherwise one int64 per row.  Replaces sum.cu's      *
 * int32 path, which promotes through self.to(int64) and so through the     *
 * host round trip of copy_ops.cc:225-240.                                  */
FL_B200_API int fl_b200_sum_i32_i64(const int32_t* x, int64_t ld, int64_t rows,
                                    int64_t cols, int64_t* out, int full,
                                    void* workspace, size_t workspace_bytes,
                                    fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Full-tensor sum that allocates nothing.  No counterpart in the reference: *
 * it exists for callers that cannot allocate device memory themselves --   *
 * code bound through a C FFI that only receives tensors from its host      *
 * framework and has no handle on that framework's allocator, or code that  *
 * runs where a cudaMalloc would synchronise the device or is not allowed.  *
 * Same result as fl_b200_reduce_sum_all (same kernel and split), but the   *
 * cross-CTA partials live in a fixed scratch array of                      *
 * FL_B200_NOALLOC_SCRATCH_BYTES inside this library: every GPU that loads  *
 * the library holds that array until the process exits.  A full-tensor    *
 * sum splits into at most 148*27 = 3996 partials of 16 bytes plus a 4-byte *
 * ticket (63,940 bytes); a request whose split would not fit the scratch   *
 * is rejected with FL_B200_ERR_TOO_LARGE before anything is launched.      *
 * The first call on a device looks up the scratch's device address        *
 * (cudaGetSymbolAddress) and caches it; make that first call before any    *
 * stream capture.  Every call shares the one scratch array, which keeps    *
 * the previous call's contents (the call zeroes what must start at zero):  *
 * calls that can overlap on the GPU -- on different streams, or from       *
 * different host threads -- race on it and must be serialised by the      *
 * caller.                                                                  */
#define FL_B200_NOALLOC_SCRATCH_BYTES 65536
FL_B200_API int fl_b200_reduce_sum_all_noalloc(const void* x, int64_t n, void* out,
                                               int in_dtype, int out_dtype,
                                               fl_b200_stream_t stream);

/* ------------------------------------------------------------------------ *
 * Backward kernels (training through the fused ops).  fp32 math, one       *
 * rounding to the output dtype.                                            *
 *                                                                           *
 * RMSNorm backward for out = w * x * r, r = 1/sqrt(mean(x^2) + eps):       *
 *   dx = r * (w*dy - n * mean(w*dy*n)), n = x*r;  dw = sum over rows dy*n.  *
 * Replaces autograd over the HF chain (modeling_qwen3.py:59-64), which the *
 * reference runs as the backward of pow (pow.cu), mean, add, rsqrt, mul    *
 * and the casts, op by op.  dw may be NULL (no weight gradient); else the  *
 * call needs a device workspace of fl_b200_rms_norm_bwd_workspace_size     *
 * bytes (per-CTA fp32 partials of dw, added in a fixed order: the result   *
 * is deterministic).  The size depends on the current device's SM count.  */
FL_B200_API size_t fl_b200_rms_norm_bwd_workspace_size(int64_t rows, int64_t cols);
FL_B200_API int fl_b200_rms_norm_bwd(const void* dy, int64_t ld_dy, const void* x,
                                     int64_t ld_x, const void* w, void* dx, int64_t ld_dx,
                                     void* dw, int64_t rows, int64_t cols, float eps,
                                     int dtype, void* workspace, size_t workspace_bytes,
                                     fl_b200_stream_t stream);

/* SwiGLU backward for out = silu(gate) * up over n dense elements:         *
 *   dup = dout * silu(gate),  dgate = dout * up * s * (1 + gate*(1 - s)),   *
 *   s = sigmoid(gate).                                                      *
 * Replaces silu_backward (csrc/aten/register.cc:329-331 -> csrc/aten/      *
 * backends/cuda/silu_backward.cu:15-35) plus the two mul.Tensor backward   *
 * products (mul.cu:28-52).                                                 */
FL_B200_API int fl_b200_swiglu_bwd(const void* dout, const void* gate, const void* up,
                                   void* dgate, void* dup, int64_t n, int dtype,
                                   fl_b200_stream_t stream);
/* silu_backward over n dense elements: dx = dout * s * (1 + x*(1 - s)).     *
 * Replaces silu_backward.cu:15-35 (same formula, fp32 op math).            */
FL_B200_API int fl_b200_silu_bwd(const void* dout, const void* x, void* dx, int64_t n,
                                 int dtype, fl_b200_stream_t stream);

/* Softmax backward over the last dim: dx = y * (dy - sum(dy * y)).          *
 * dy and y share in_dtype; out_dtype = in_dtype, or BF16/F16 with F32       *
 * inputs (the backward of a half_to_float softmax).  Replaces              *
 * _softmax_backward_data, which the reference leaves unregistered (CPU      *
 * fallback, csrc/aten/register.cc:439-442 -> fallback.cc:12-14).           */
FL_B200_API int fl_b200_softmax_bwd(const void* dy, int64_t ld_dy, const void* y,
                                    int64_t ld_y, void* dx, int64_t ld_dx, int64_t rows,
                                    int64_t cols, int in_dtype, int out_dtype,
                                    fl_b200_stream_t stream);
/* The same times `scale`: the backward of fl_b200_softmax_masked with      *
 * respect to x (dx = scale * y * (dy - sum(dy * y))); the mask's gradient  *
 * is the unscaled product summed over the dims it broadcasts.  Replaces    *
 * the chain's _softmax_backward_data followed by mul.cu:28-52.             */
FL_B200_API int fl_b200_softmax_bwd_scaled(const void* dy, int64_t ld_dy, const void* y,
                                           int64_t ld_y, void* dx, int64_t ld_dx,
                                           int64_t rows, int64_t cols, float scale,
                                           int in_dtype, int out_dtype,
                                           fl_b200_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* FL_B200_H_ */
