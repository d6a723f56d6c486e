/*
 * tileops_c.h -- C ABI of the B200 (sm_100a) TileOPs forward-operator library.
 *
 * Every entry point takes plain device pointers, element counts / shapes and
 * a CUDA stream handle passed as `void*` (a `cudaStream_t`; NULL selects the
 * legacy default stream of the current context).  No entry point allocates
 * device memory: the caller owns every input, output and workspace buffer.
 * Kernels are enqueued on `stream` and the call returns without
 * synchronising; a non-zero status is returned for invalid arguments (checked
 * on the host before anything is enqueued) and for launch failures.
 *
 * Each entry point replaces one TileLang `@tilelang.jit(target="npuir")`
 * factory of the reference (Yihuace/tile-ascendnpu-ops, package
 * examples/TileOPs/tileops); the factory a function stands in for is named in
 * its comment as file:line inside that package.
 *
 * Layout conventions: all tensors are dense and row-major (C-contiguous) in
 * the shapes given.  Pointers passed to the vectorised paths should be
 * 16-byte aligned; misaligned pointers take a scalar path (same results).
 */
#ifndef TILEOPS_C_H_
#define TILEOPS_C_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define TILEOPS_OK 0
#define TILEOPS_EBADDTYPE (-1) /* dtype code not supported by this entry   */
#define TILEOPS_EBADSHAPE (-2) /* a size / shape argument is out of range   */
#define TILEOPS_EALIGN (-3)    /* a pointer violates a hard alignment rule  */
#define TILEOPS_ELAUNCH (-4)   /* the CUDA launch (or a CUDA call) failed   */
#define TILEOPS_ETIMEOUT (-5)  /* a bounded device-side wait ran out        */
#define TILEOPS_EINVAL (-6)    /* any other invalid argument (NULL pointer) */

/* ---- dtype codes (torch dtype in parentheses) --------------------------- */
#define TILEOPS_DT_F32 0  /* torch.float32  */
#define TILEOPS_DT_F16 1  /* torch.float16  */
#define TILEOPS_DT_BF16 2 /* torch.bfloat16 */
#define TILEOPS_DT_BOOL 3 /* torch.bool (one byte, 0 or 1) */
#define TILEOPS_DT_U8 4   /* torch.uint8    */
#define TILEOPS_DT_I8 5   /* torch.int8     */
#define TILEOPS_DT_I16 6  /* torch.int16    */
#define TILEOPS_DT_I32 7  /* torch.int32    */
#define TILEOPS_DT_I64 8  /* torch.int64    */

/* ABI version of this header; bumped when a signature changes. */
#define TILEOPS_ABI_VERSION 1

int tileops_abi_version(void);
/* Static, human-readable text for a status code. */
const char* tileops_status_string(int status);
/* Device-side error word, read back by the host after the stream is
 * synchronised: 0 = none; 1 = a bounded mbarrier wait timed out (attention,
 * gated delta net); 2 = a malformed cu_seqlens was passed to
 * tileops_gdn_prefill_varlen_fwd.  The first code set is kept until cleared. */
int tileops_device_error_flag(void* stream, int clear);

/* Self-test of the give-up path the tensor-core kernels take when a wait
 * runs out: one warp allocates 32 TMEM columns, starts a bulk copy of `bytes`
 * (16..4096, a multiple of 16) from `src` (16-byte aligned device memory),
 * waits (polling, so the wait always ends) on an mbarrier nothing arrives on
 * for `limit_ns` (1e3..1e9) and then, as every kernel here does on a
 * timeout, sets device error 1, waits for its
 * copy to land, frees TMEM and returns.  `out` (6 device ints) receives:
 * [0] 1 if the wait gave up, [1] 1 if the copy landed, [2] the sum of the
 * copied bytes, [3] 1 once TMEM was freed, [4] / [5] the low / high 32 bits
 * of the nanoseconds the wait took before giving up.  A diagnostic of this
 * library with no counterpart in the reference (its kernels have no bounded
 * waits). */
int tileops_selftest_wait_timeout(const void* src, int64_t bytes, int64_t limit_ns, int* out,
                                  void* stream);

/* ---- elementwise unary (flat, n elements; y may not alias x) ----------- */

/* y = x * clamp(x + 3, 0, 6) / 6 in fp32, rounded once.  dtype f32/f16/bf16.
 * Replaces hardswish_fwd_kernel,
 * kernels/elementwise/hardswish/hardswish_kernel/hardswish_fwd_kernel.py:70. */
int tileops_hardswish_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);

/* y = clamp(x + 3, 0, 6) / 6 in fp32 (NaN propagates).  dtype f32/f16/bf16.
 * Replaces hardsigmoid_fwd_kernel,
 * kernels/elementwise/hardsigmoid/hardsigmoid_kernel/perf_opt/hardsigmoid_fwd_kernel.py. */
int tileops_hardsigmoid_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);

/* y = clamp(x, min, max) in fp32 with NaN propagation; a bound is applied
 * only when its has_* flag is non-zero (at least one must be).  The bounds
 * are rounded to fp32 first, as torch.clamp does for a float tensor.
 * Replaces clamp_scalar_fwd_kernel,
 * kernels/elementwise/clamp_scalar/clamp_scalar_kernel/perf_opt/clamp_scalar_fwd_kernel.py. */
int tileops_clamp_scalar_fwd(const void* x, void* y, int64_t n, int dtype, int has_min,
                             double min_val, int has_max, double max_val, void* stream);

/* IEEE predicates, y is torch.bool (one byte per element, 0/1); x f32/f16/bf16.
 * Replace isnan_fwd_kernel (kernels/elementwise/isnan/isnan_kernel/isnan_fwd_kernel.py),
 * isinf_fwd_kernel (…/isinf/isinf_kernel/isinf_fwd_kernel.py) and
 * isfinite_fwd_kernel (…/isfinite/isfinite_kernel/isfinite_fwd_kernel.py). */
int tileops_isnan_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);
int tileops_isinf_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);
int tileops_isfinite_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);

/* y = ~x for u8/i8/i16/i32/i64, logical not for bool.
 * Replaces bitwise_not_fwd_kernel,
 * kernels/elementwise/bitwise_not/bitwise_not_kernel/bitwise_not_fwd_kernel.py. */
int tileops_bitwise_not_fwd(const void* x, void* y, int64_t n, int dtype, void* stream);

/* ---- gated activations: x is (M, 2N), y is (M, N) ---------------------- */

/* y = 0.5*g*(1 + erf(g/sqrt(2))) * v, g = x[:, :N], v = x[:, N:], fp32 math.
 * Replaces gelu_and_mul_fwd_kernel,
 * kernels/elementwise/gelu_and_mul/gelu_and_mul_kernel/perf_opt/gelu_and_mul_fwd_kernel.py:143. */
int tileops_gelu_and_mul_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                             void* stream);

/* y = 0.5*g*(1 + tanh(sqrt(2/pi)*(g + 0.044715 g^3))) * v, fp32 math.
 * Replaces gelu_tanh_and_mul_fwd_kernel,
 * kernels/elementwise/gelu_tanh_and_mul/gelu_tanh_and_mul_kernel/perf_opt/gelu_tanh_and_mul_fwd_kernel.py. */
int tileops_gelu_tanh_and_mul_fwd(const void* x, void* y, int64_t M, int64_t N, int dtype,
                                  void* stream);

/* ---- fused residual add + LayerNorm ------------------------------------ */

/* s = round_dtype(x + residual);  y = round_dtype((s - mean) * rstd * w + b)
 * per row of N, statistics in fp32 (biased variance), rstd = 1/sqrt(var+eps).
 * x, residual, y, residual_out: (M, N) of `dtype` (f32/f16/bf16).
 * weight, bias: (N,) of `affine_dtype` (either `dtype` or f32).
 * Replaces _fused_add_layer_norm_kernel,
 * kernels/norm/fused_add_layer_norm/fused_add_layer_norm_kernel/_fused_add_layer_norm_kernel.py:144. */
int tileops_fused_add_layer_norm_fwd(const void* x, const void* residual, const void* weight,
                                     const void* bias, void* y, void* residual_out, int64_t M,
                                     int64_t N, double eps, int dtype, int affine_dtype,
                                     void* stream);

/* ---- 1-D convolution (NCL) ---------------------------------------------- */

#define TILEOPS_ACT_NONE 0
#define TILEOPS_ACT_SILU 1

/* Depthwise conv1d: out[n,c,l] = act(b[c] + sum_k w[c,k] * x[n,c,l*stride + k*dil - pad_left])
 * with zero padding outside [0, l_in).  x (n, c, l_in), w (c, k) contiguous
 * (the (c, 1, k) torch layout is the same memory), bias (c,) or NULL,
 * y (n, c, l_out).  x/y `dtype` f16/bf16/f32; w/bias `w_dtype` (= dtype or f32).
 * fp32 accumulation, one rounding.  Causal (Mamba-style) form: pad_left = k-1,
 * l_out = l_in.
 * Replaces _conv1d_direct_kernel,
 * kernels/convolution/conv1d/conv1d_kernel/_conv1d_direct_kernel.py:163 (depthwise path
 * selected by ops/convolution.py:143-145). */
int tileops_conv1d_depthwise_fwd(const void* x, const void* w, const void* bias, void* y,
                                 int64_t n, int64_t c, int64_t l_in, int64_t l_out,
                                 int64_t k, int64_t stride, int64_t pad_left,
                                 int64_t dilation, int dtype, int w_dtype, int activation,
                                 void* stream);

/* General grouped conv1d (any groups, stride, dilation, padding) with fp32
 * accumulation: the dense/grouped conv1d kernels of the reference
 * (kernels/convolution/conv1d/conv1d.py:152-516: pointwise, generic,
 * unit-stride and group kernels).  f16 / bf16 run as an implicit GEMM on
 * tcgen05 tensor cores (bias added in fp32, one rounding); f32 on CUDA cores.
 * x (n, c_in, l_in), w (c_out, c_in/groups, k) and bias (c_out,) or NULL in
 * `dtype`, y (n, c_out, l_out).  A bounded device-side wait that times out is
 * reported through tileops_device_error_flag. */
int tileops_conv1d_direct_fwd(const void* x, const void* w, const void* bias, void* y,
                              int64_t n, int64_t c_in, int64_t l_in, int64_t c_out,
                              int64_t l_out, int64_t k, int64_t stride, int64_t pad_left,
                              int64_t dilation, int64_t groups, int dtype, void* stream);

/* ---- attention ----------------------------------------------------------- */

/* Flash-style multi-head / grouped-query attention forward on tcgen05 tensor
 * cores, BSHD layout.  q (B, Sq, H, D), k / v (B, Skv, Hkv, D) of dtype
 * f16/bf16 (D = 64 or 128, H % Hkv == 0), o like q, lse (B, H, Sq) fp32 in the
 * log2 domain: lse = logsumexp(scale * q k^T) / ln 2.  Causal masking is
 * right-aligned (query i sees keys j <= i + Skv - Sq; needs Sq <= Skv).
 * q, k, v, o must be 16-byte aligned (TMA).  A bounded device-side wait that
 * times out is reported through tileops_device_error_flag.
 * Replaces _gqa_prefill_fwd_kernel,
 * kernels/attention/multi_head_attention/multi_head_attention_kernel/perf_opt/_gqa_prefill_fwd_kernel.py:199. */
int tileops_mha_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                    int64_t batch, int64_t heads, int64_t heads_kv, int64_t seq_q,
                    int64_t seq_kv, int64_t dim, int is_causal, double sm_scale, int dtype,
                    void* stream);

/* ---- gated linear attention decode ------------------------------------- */

/* One recurrent step per (b, h): new_state[i, j] = exp(gk[i]) state[i, j] +
 * k[i] v[j];  o[j] = scale * sum_i q[i] new_state[i, j], fp32 math, o from the
 * fp32 new state, both outputs rounded to `dtype` (f32/f16/bf16).  Layout BHD:
 * q, k, gk (B, H, DK); v, o (B, H, DV); state, new_state (B, H, DK, DV).
 * scale <= 0 means DK^-0.5.  new_state may not alias state.
 * Replaces _gla_decode_kernel,
 * kernels/linear_attention/gla_decode/gla_decode_kernel/_gla_decode_kernel.py:57. */
int tileops_gla_decode_fwd(const void* q, const void* k, const void* v, const void* gk,
                           const void* state, void* o, void* new_state, int64_t batch,
                           int64_t heads, int64_t dim_k, int64_t dim_v, double scale, int dtype,
                           void* stream);

/* ---- Mamba-2 SSD chunk scan --------------------------------------------- */

/* out[l, p] = exp(dA[l]) * sum_n C[l, n] prev[p, n]
 *           + sum_{s <= l} cb[l, s] exp(dA[l] - dA[s]) dt[s] x[s, p]
 * per batch, chunk and head (group g = h / (H / G)), fp32 accumulation on
 * tcgen05 tensor cores.  x (B, NC*Q, H, P), C (B, NC*Q, G, N), cb (B, NC, G,
 * Q, Q) and dt (B, H, NC, Q) in `dtype` (f16/bf16); dA_cumsum (B, H, NC, Q)
 * and prev_states (B, NC, H, P, N) fp32; out (B, NC*Q, H, P) fp32.  P a
 * multiple of 16 up to 128, N a multiple of 8 up to 256, Q up to 1024; x, C,
 * cb, prev_states, out 16-byte aligned.  prev_states enter the MMA rounded to
 * `dtype`.  Replaces _ssd_chunk_scan_fwd_kernel,
 * kernels/mamba/ssd_chunk_scan/ssd_chunk_scan_kernel/perf_opt/_ssd_chunk_scan_fwd_kernel.py:181. */
int tileops_ssd_chunk_scan_fwd(const void* x, const void* cb, const float* dA_cumsum,
                               const void* C, const float* prev_states, const void* dt,
                               float* out, int64_t batch, int64_t num_chunks, int64_t chunk_len,
                               int64_t n_heads, int64_t d_head, int64_t d_state,
                               int64_t n_groups, int dtype, void* stream);

/* ---- gated delta net (linear attention) -------------------------------- */

/* Bytes of scratch workspace tileops_gdn_prefill_fwd needs for this shape
 * (per 64-token chunk of every (batch, head): the WY factors Wk (64 x dk),
 * U (64 x dv) and the decayed causal q k^T (64 x 64) in bf16, plus 132 fp32),
 * or -1 for an unsupported shape. */
int64_t tileops_gdn_workspace_bytes(int64_t batch, int64_t seq_len, int64_t heads,
                                    int64_t dim_k, int64_t dim_v);

/* Gated delta rule, chunked prefill.  Per (b, h) and token t, with state S
 * (dk x dv, fp32):  S <- exp(g_t) S;  S <- S + k_t (x) beta_t (v_t - k_t^T S);
 * o_t = scale * q_t^T S.  Layout BTHD: q, k (B, T, H, dk) and v, o (B, T, H, dv)
 * bf16; g (log decay), beta (B, T, H) fp32; initial_state (NULL = zeros) and
 * final_state (NULL = not written) (B, H, dk, dv) fp32.  dk, dv in {64, 128};
 * chunk_size must be 64; dtype must be TILEOPS_DT_BF16.  `workspace` holds
 * tileops_gdn_workspace_bytes() bytes, 16-byte aligned, owned by the caller.
 * The reference defines no op for this path (GatedDeltaNetPrefillFwdOp was not
 * delivered); this entry replaces its probe kernel
 * examples/gdn_prefill/probe/gdn_prefill_probe.py:83 and follows the
 * sequential golden at :60-77. */
int tileops_gdn_prefill_fwd(const void* q, const void* k, const void* v, const float* g,
                            const float* beta, const float* initial_state, void* o,
                            float* final_state, void* workspace, int64_t batch, int64_t seq_len,
                            int64_t heads, int64_t dim_k, int64_t dim_v, int64_t chunk_size,
                            double scale, int dtype, void* stream);

/* Bytes of scratch workspace tileops_gdn_prefill_varlen_fwd needs: the WY
 * factors of (total_len / 64 + num_seqs) chunk slots per head plus a
 * chunk -> sequence table of as many int32, or -1 for an unsupported shape. */
int64_t tileops_gdn_varlen_workspace_bytes(int64_t total_len, int64_t num_seqs, int64_t heads,
                                           int64_t dim_k, int64_t dim_v);

/* Flags of tileops_gdn_prefill_varlen_fwd. */
#define TILEOPS_GDN_QK_L2NORM 1 /* use q / sqrt(|q|^2 + 1e-6), k likewise (fla's
                                   use_qk_l2norm_in_kernel), fused: no extra pass */

/* Variable-length form of tileops_gdn_prefill_fwd (the fla `cu_seqlens`
 * convention, batch 1): num_seqs sequences packed along one token axis,
 * sequence n being rows [cu_seqlens[n], cu_seqlens[n+1]) of q, k (total_len,
 * H, dk), v, o (total_len, H, dv), g, beta (total_len, H).  cu_seqlens is an
 * int32 DEVICE array of num_seqs + 1 offsets with cu_seqlens[0] = 0,
 * non-decreasing, cu_seqlens[num_seqs] = total_len (empty sequences allowed);
 * it is never copied to the host, so the call does not synchronise.  A
 * cu_seqlens that breaks these rules cannot make the kernels access memory
 * out of range (offsets are clamped) but gives meaningless results, and the
 * device error flag reads 2 (tileops_device_error_flag).  cu_seqlens = NULL
 * means num_seqs sequences of total_len / num_seqs rows each (a uniform batch,
 * the layout of tileops_gdn_prefill_fwd; total_len must divide evenly).
 * initial_state (NULL = zeros) and final_state (NULL = not written) are
 * (num_seqs, H, dk, dv) fp32; each sequence starts from its own initial
 * state.  flags: 0 or TILEOPS_GDN_QK_L2NORM.  `workspace` holds
 * tileops_gdn_varlen_workspace_bytes() bytes, 16-byte aligned.  Same sizes,
 * dtype and chunk rules as tileops_gdn_prefill_fwd; no reference counterpart
 * (the arguments follow fla chunk_gated_delta_rule). */
int tileops_gdn_prefill_varlen_fwd(const void* q, const void* k, const void* v, const float* g,
                                   const float* beta, const int32_t* cu_seqlens,
                                   int64_t num_seqs, const float* initial_state, void* o,
                                   float* final_state, void* workspace, int64_t total_len,
                                   int64_t heads, int64_t dim_k, int64_t dim_v,
                                   int64_t chunk_size, double scale, int flags, int dtype,
                                   void* stream);

/* Same as tileops_gdn_prefill_fwd, but allocates nothing and takes no
 * workspace: for callers that cannot allocate device memory when they call
 * (inside a captured CUDA graph, or a host runtime / plugin without a device
 * allocator).  The scratch is a fixed 16 MiB array in this library's device
 * memory, held on every GPU that loads the library until exit; shapes needing
 * more than that (tileops_gdn_workspace_bytes() > 16 MiB, i.e. more than 404
 * chunks of 64 tokens summed over batch * heads at dk = dv = 128) return
 * TILEOPS_EBADSHAPE before anything is enqueued.  All calls share the array,
 * so calls whose kernels overlap on the GPU race.  The first call on a device
 * looks up the device addresses of the array and of the device error word
 * (cudaGetSymbolAddress, which may load the module); make that first call
 * outside any stream capture.
 * This entry point has no counterpart in the reference. */
int tileops_gdn_prefill_fwd_noalloc(const void* q, const void* k, const void* v, const float* g,
                                    const float* beta, const float* initial_state, void* o,
                                    float* final_state, int64_t batch, int64_t seq_len,
                                    int64_t heads, int64_t dim_k, int64_t dim_v,
                                    int64_t chunk_size, double scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TILEOPS_C_H_ */
