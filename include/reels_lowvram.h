/*
 * reels_lowvram.h -- C ABI of the B200 (sm_100a) Int8-weight LoRA linear.
 *
 * Drop-in native backend for Reels.jl's quantised frozen-weight path
 * (`low_vram.frozen_weight_quantization = "int8"`).  Every entry point:
 *   - takes plain device pointers and sizes, and a cudaStream_t as `void *`;
 *   - is asynchronous on that stream unless documented otherwise;
 *   - returns 0 on success, REELS_EINVAL (-1) for bad arguments (nothing is
 *     launched) and REELS_EDEVICE (-2) for CUDA launch / device errors, with a
 *     message in reels_lowvram_last_error() (thread-local, like
 *     deps/sentencepiece_bridge.cpp:10-17 of the reference);
 *   - allocates no device memory: scratch space is caller-provided
 *     (`workspace`, sized by reels_q8lora_workspace_bytes);
 *   - may be called from several host threads and on several streams at
 *     once.  The per-thread state is the error message, the last path and
 *     the profiling counters; calls that share a workspace or a `saved`
 *     buffer must be ordered on one stream;
 *   - runs on the device that owns its buffers and leaves the calling
 *     thread's current device (CUDA context) as it found it: a call with
 *     device-1 buffers while device 0 is current returns with device 0
 *     current, and a thread with no current context is left with none.
 *
 * Array layouts are those of the reference's column-major, feature-first
 * Julia arrays, written as row-major C arrays:
 *   x, dx      [M][K]   (Julia (in, tokens))
 *   y, dy      [M][N]   (Julia (out, tokens))
 *   q          [K][N]   REELS_W_OUT_CONTIGUOUS (Julia QuantizedMatrix.values, (out, in))
 *              [N][K]   REELS_W_IN_CONTIGUOUS  (PyTorch nn.Linear.weight)
 *   scales     [N]      fp32, one per output row of the weight
 *   A, dA      [K][r]   (Julia LoRALinear.A, (rank, in))
 *   B, dB      [r][N]   (Julia LoRALinear.B, (out, rank))
 *   bias       [N]
 * Activations, A, B and bias share one element type `act_dtype`
 * (REELS_BF16, REELS_F16 or REELS_F32); dA and dB are fp32 accumulators.
 *
 * Numerics: weights are dequantised exactly (int8 -> 16-bit is exact, the
 * per-row scale is applied in fp32), products accumulate in fp32 on the
 * tensor cores.  bf16/fp16 with K % 16 == 0 and N % 16 == 0 and 16-byte
 * aligned pointers run on the tcgen05 path; every other case (fp32
 * activations, ragged feature sizes) runs on CUDA-core kernels.  Both are GPU
 * code; there is no CPU fallback.
 */
#ifndef REELS_LOWVRAM_H
#define REELS_LOWVRAM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define REELS_LOWVRAM_ABI_VERSION 1

#define REELS_OK 0
#define REELS_EINVAL (-1)
#define REELS_EDEVICE (-2)

/* element types */
#define REELS_F32 0
#define REELS_F16 1
#define REELS_BF16 2

/* frozen-weight layouts */
#define REELS_W_OUT_CONTIGUOUS 0 /* Julia (out, in) column-major == row-major [K][N] */
#define REELS_W_IN_CONTIGUOUS 1  /* row-major [N][K] */

/* which pass a workspace query is for */
#define REELS_PASS_FORWARD 0
#define REELS_PASS_BACKWARD 1
#define REELS_PASS_DROPOUT 2 /* or-ed into the pass: room for the dropped-out input */

/* Activation fused into a linear's output (forward) or its input's gradient
 * (backward). */
#define REELS_ACT_NONE 0
#define REELS_ACT_GELU_TANH 1 /* gelu_tanh, src/layers/linear.jl:61-68 */

/* Empty inputs: every call that takes a token count M (or a length n)
 * accepts 0.  Then nothing is read, the buffers sized by M may be NULL, and
 * gradients of parameters (dA, dB, dscale, dshift, dgate) are zero-filled,
 * or left unchanged when accumulating -- a sum over no tokens. */

/* execution paths reported by reels_lowvram_last_path() */
#define REELS_PATH_NONE 0
#define REELS_PATH_TENSORCORE 1
#define REELS_PATH_CUDACORE 2

/* Message for the last failing call on this thread ("" if none).
 * Mirrors reels_sp_last_error, deps/sentencepiece_bridge.cpp:85-87. */
const char *reels_lowvram_last_error(void);

int reels_lowvram_abi_version(void);

/* The plan the q8 GEMM takes for D[M][Nout] over a reduction of Kred, for
 * diagnostics and tests; no device work.  info (7 entries):
 *   [0] kernel: 1 weight-in-TMEM, 2 weight-in-TMEM on CTA pairs (tiles of
 *       256 output columns on two SMs), 0 both operands in shared memory
 *   [1] tokens per tile  [2] reduction elements per pipeline stage
 *   [3] reduction splits [4] pipeline stages per split
 *   [5] output-column tiles  [6] token tiles
 * act: REELS_ACT_NONE or REELS_ACT_GELU_TANH (the epilogue weighs the plans).
 * sms <= 0: the current device's SM count (148 without a device). */
int reels_q8_plan(int64_t M, int64_t Nout, int64_t Kred, int act, int sms, int64_t *info);

/* The skinny rank-r GEMM's reduction split for `rows` rows over `red`:
 * info[0] splits, info[1] 64-element blocks per split. */
int reels_sk_plan(int64_t rows, int64_t red, int64_t r, int sms, int64_t *info);

/* Plan of the backward's one pass over dy, which computes G = s*B'*dy and dB
 * together (no reference counterpart; the reference computes them as two
 * products, lora.jl:112-114).  info[0] 1 when the backward uses it (else G
 * and dB are separate passes), info[1] token ranges, info[2] feature
 * ranges, info[3] TMEM columns per CTA, info[4] and info[5] bytes of fp32
 * partials for G and dB. */
int reels_sk_dual_plan(int64_t M, int64_t N, int64_t r, int sms, int64_t *info);

/* Path taken by the last successful compute call on this thread. */
int reels_lowvram_last_path(void);

/* Synchronises `stream`, then reads and clears the device status word that
 * kernels set when a bounded pipeline wait gives up.  Returns 0, or
 * REELS_EDEVICE with the status in the message.  Not needed in normal use;
 * tests and debug builds call it after a step. */
int reels_lowvram_check_device_status(void *stream);

/* Profiling (off by default; no reference counterpart -- the reference only
 * times whole phases with time_ns, src/training/metrics.jl:4-10).  While
 * enabled, every q8 GEMM launch made by this thread is bracketed by two CUDA
 * events recorded on its own stream.  Every kernel launch is counted
 * whether or not profiling is on.  Enabling resets the counters. */
int reels_lowvram_profile_enable(int enable);

/* Synchronises the recorded events and returns, since the last enable/read:
 * the summed q8 GEMM kernel time (ms), the number of q8 launches, their
 * algorithmic FLOPs (2*M*Nout*(Kred + r) each) and the number of kernels this
 * thread launched; then resets them.  Any pointer may be NULL. */
int reels_lowvram_profile_read(double *q8_ms, int64_t *q8_launches, double *q8_flops, int64_t *kernel_launches);

/* Per-output-row symmetric Int8 quantiser, bit-exact to
 * quantize_frozen_matrix (src/layers/quantization.jl:35-44):
 * scale = max|w_row| / 127 (1 for an all-zero row),
 * q = round_to_even(clamp(w / scale, -127, 127)).
 * `w` (w_dtype REELS_F32/F16/BF16, widened to fp32 exactly like
 * `Float32.(Array(weight))`) and `q` share `layout`.
 * Synchronises `stream` to report the inputs the reference rejects with
 * InexactError, returning REELS_EINVAL: non-finite weights, and a row whose
 * max|w| / 127 underflows to 0 (max|w| <= 63 * 2^-149) while it holds a zero
 * element (0 / 0 = NaN, which Int8 cannot represent).  Such a row without
 * zeros quantises to +-127 with scale 0, as in the reference. */
int reels_q8_quantize(const void *w, int w_dtype, int layout, int64_t N, int64_t K, int8_t *q, float *scales,
                      void *stream);

/* _materialize_weight / _dequantize_for_compute (quantization.jl:54-64):
 * out (same layout as q) = Float16(q)*Float16(s) rounded to fp16 for
 * REELS_F16, Float32(q)*s for REELS_F32, and that fp32 product rounded once
 * to bf16 for REELS_BF16. */
int reels_q8_materialize(const int8_t *q, const float *scales, int layout, int64_t N, int64_t K, int out_dtype,
                         void *out, void *stream);

/* Bytes of scratch a forward or backward call needs (pass =
 * REELS_PASS_FORWARD / REELS_PASS_BACKWARD; r = 0 for the plain linears). */
size_t reels_q8lora_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r, int act_dtype, int pass);

/* Bytes of the `saved` buffer (A*x kept from the forward for the backward). */
size_t reels_q8lora_saved_bytes(int64_t M, int64_t r, int act_dtype);

/* Size of the library-owned scratch used by reels_q8lora_forward_static_ws. */
#define REELS_STATIC_WS_BYTES (32u << 20)

/* reels_q8lora_forward without a caller-supplied workspace.  No counterpart
 * in the reference: it exists for callers that cannot allocate device memory
 * themselves -- a foreign-function binding that is only handed raw device
 * pointers and has no device allocator of its own, or a loop that must run
 * inside a fixed device-memory budget where a per-call allocation could fail
 * or fragment the pool.  Its scratch is a file-scope device array of
 * REELS_STATIC_WS_BYTES (32 MiB) inside the library; every GPU that loads the
 * library holds that array until the process exits.  Arguments and results
 * are those of reels_q8lora_forward; a shape whose forward workspace
 * (reels_q8lora_workspace_bytes, REELS_PASS_FORWARD) exceeds the array is
 * rejected with REELS_EINVAL and nothing runs.
 *  - The first call on a device looks the array's device address up with that
 *    device current; make that first call before any stream capture.
 *  - All calls share the one array and it keeps the last call's contents.
 *    Nothing in it needs to start at zero (every byte a call reads it wrote
 *    earlier in the same call), but calls that overlap on the GPU (other
 *    streams, other host threads) race on it: serialise them.
 *  - Allocates nothing: no cudaMalloc, cudaFree or allocating library call. */
int reels_q8lora_forward_static_ws(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                                   const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                                   float alpha, int act_dtype, void *y, void *saved, void *stream);

/* _weight_mul (quantization.jl:73-74) for a QuantizedMatrix, optional bias
 * (linear, src/layers/linear.jl:38-46): y = dequant(q) * x (+ bias). */
int reels_q8_weight_mul(const void *x, const int8_t *q, const float *scales, int layout, const void *bias, int64_t M,
                        int64_t K, int64_t N, int act_dtype, void *y, void *workspace, size_t ws_bytes,
                        void *stream);

/* _weight_transpose_mul (quantization.jl:75-76), the frozen-weight pullback
 * of ad_rules.jl:55-80: dx = dequant(q)' * dy. */
int reels_q8_weight_transpose_mul(const void *dy, const int8_t *q, const float *scales, int layout, int64_t M,
                                  int64_t K, int64_t N, int act_dtype, void *dx, void *workspace, size_t ws_bytes,
                                  void *stream);

/* lora_forward (src/layers/lora.jl:56-95; training=false or dropout 0):
 *   y = dequant(q) * x (+ bias) + (alpha / r) * B * (A * x)
 * `saved` (nullable, reels_q8lora_saved_bytes) receives A*x for the backward.
 * alpha/r is formed in fp32 as in lora.jl:89. */
int reels_q8lora_forward(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                         const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                         int act_dtype, void *y, void *saved, void *workspace, size_t ws_bytes, void *stream);

/* lora_backward (lora.jl:106-118), equal to Zygote's pullback of
 * lora_forward through the _weight_mul rrule (ad_rules.jl:70-80):
 *   s  = alpha / r,  ax = A*x,  g = B'*dy
 *   dx = dequant(q)' * dy + s * A' * g          (dx nullable: skipped)
 *   dA = s * g * x'          dB = s * dy * ax'
 * dA/dB are fp32; with accumulate = 0 they are overwritten with
 * grad_scale * grad, with accumulate = 1 that is added (the fp32 gradient
 * accumulators of src/training/wan_runner.jl:143,201-203; grad_scale is the
 * 1/loss_scale of src/training/precision.jl:8-12).
 * `saved` is the forward's A*x, or NULL to recompute it. */
int reels_q8lora_backward(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                          const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N, int64_t r,
                          float alpha, float grad_scale, int act_dtype, void *dx, float *dA, float *dB,
                          int accumulate, void *workspace, size_t ws_bytes, void *stream);

/* A LoRA linear followed by an activation, the feed-forward input projection
 * and its gelu_tanh of src/models/wan21/transformer.jl:289-291 (likewise
 * ltx23/transformer.jl:308-310):
 *   pre = round(lora_forward(x))         the linear's output ("hidden")
 *   y   = round(act(float(pre)))         gelu_tanh, src/layers/linear.jl:61-68
 * computed in one pass over the output tile.  `pre` (nullable, [M][N], the
 * same element type) receives the linear's output, which the backward of
 * the next linear needs (reels_q8lora_backward_act); inference passes NULL.
 * act == REELS_ACT_NONE is reels_q8lora_forward.  Other arguments, results
 * and the workspace are those of reels_q8lora_forward. */
int reels_q8lora_forward_act(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                             const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                             float alpha, int act_dtype, int act, void *y, void *pre, void *saved, void *workspace,
                             size_t ws_bytes, void *stream);

/* reels_q8lora_backward for a linear whose input is an activation's output,
 * x = act(pre_x) (the feed-forward output projection applied to
 * gelu_tanh(hidden), transformer.jl:291): `dx` receives the gradient with
 * respect to pre_x, the chain rule through the activation fused into the dx
 * epilogue:
 *   dx = round(round(dequant(q)' * dy + s * A' * g) * act'(float(pre_x)))
 * which is Zygote's pullback of gelu_tanh (its derivative formed in fp32 and
 * the gradient cast back to the element type).  dA and dB use `x` (the
 * activation's output) as in reels_q8lora_backward.  pre_x [M][K] is required
 * when dx is given. */
int reels_q8lora_backward_act(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                              const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N,
                              int64_t r, float alpha, float grad_scale, int act_dtype, int act, const void *pre_x,
                              void *dx, float *dA, float *dB, int accumulate, void *workspace, size_t ws_bytes,
                              void *stream);

/* lora_forward with LoRA dropout (lora.jl:71-85, training with dropout > 0):
 * the adapter's input is z = x * keep / (1 - dropout) (rounded to act_dtype),
 * the frozen weight still multiplies x:
 *   y = dequant(q) * x (+ bias) + (alpha / r) * B * (A * z)
 * keep = (u >= dropout) with u a uniform Float32 per element of x drawn from
 * a counter-based generator keyed by seed xor (stream_id * 0x9e3779b97f4a7c15)
 * (the reference's _dropout_seed, lora.jl:41-43) and indexed by the element's
 * linear position; see reels_dropout_mask.  The workspace comes from
 * reels_q8lora_workspace_bytes(..., REELS_PASS_FORWARD | REELS_PASS_DROPOUT).
 * `saved` receives A * z. */
int reels_q8lora_forward_dropout(const void *x, const int8_t *q, const float *scales, int layout, const void *A,
                                 const void *B, const void *bias, int64_t M, int64_t K, int64_t N, int64_t r,
                                 float alpha, int act_dtype, float dropout, uint64_t seed, uint64_t stream_id, void *y,
                                 void *saved, void *workspace, size_t ws_bytes, void *stream);

/* The gradients of reels_q8lora_forward_dropout with the same seed and
 * stream_id (the mask is recomputed, not stored):
 *   dx = dequant(q)' * dy + keep * (s * A' * (B' * dy)) / (1 - dropout)
 *   dA = s * (B' * dy) * z'      dB = s * dy * (A * z)'
 * Workspace: REELS_PASS_BACKWARD | REELS_PASS_DROPOUT. */
int reels_q8lora_backward_dropout(const void *x, const void *dy, const int8_t *q, const float *scales, int layout,
                                  const void *A, const void *B, const void *saved, int64_t M, int64_t K, int64_t N,
                                  int64_t r, float alpha, float grad_scale, int act_dtype, float dropout, uint64_t seed,
                                  uint64_t stream_id, void *dx, float *dA, float *dB, int accumulate, void *workspace,
                                  size_t ws_bytes, void *stream);

/* The dropout mask itself: keep[i] = 1 where element i of the adapter input
 * is kept, 0 where dropped, for i < n (n = M * K, i = token * K + feature). */
int reels_dropout_mask(int64_t n, float dropout, uint64_t seed, uint64_t stream_id, uint8_t *keep, void *stream);

/* The linears' input producer of the Wan block,
 *   out = mixed_affine(layernorm(x; epsilon, ln_weight, ln_bias), scale, shift)
 * (src/layers/linear.jl:26-36,49-59, called at
 * src/models/wan21/transformer.jl:287-289), one pass per row of x [M][K]:
 * mean and variance in fp32, y = (x - mean) / sqrt(var + epsilon)
 * (* ln_weight) (+ ln_bias) rounded to act_dtype, then
 * round(y * (1 + scale[b]) + shift[b]) with b = token / tokens_per_sample.
 * scale and shift are [batch][K] (the per-sample modulation, AdaLN); any of
 * scale, shift, ln_weight, ln_bias may be NULL.  K <= 16384. */
int reels_layernorm_modulate(const void *x, int64_t M, int64_t K, int64_t tokens_per_sample, const void *scale,
                             const void *shift, const void *ln_weight, const void *ln_bias, float epsilon,
                             int act_dtype, void *out, void *stream);

/* Workspace of reels_layernorm_modulate_backward when the parameter
 * gradients are requested. */
size_t reels_layernorm_modulate_workspace_bytes(int64_t M, int64_t K, int64_t tokens_per_sample);

/* Its pullback for dout [M][K]: dx (required), and optionally the modulation's
 * parameter gradients (modulation.jl:13-22) as fp32 [batch][K]:
 *   dscale[b] = sum over the sample's tokens of dout * ln,  dshift[b] = sum dout
 * (overwritten, or added with accumulate = 1), in a fixed summation order.
 * The LayerNorm's own weight and bias receive no gradient (frozen). */
int reels_layernorm_modulate_backward(const void *x, const void *dout, int64_t M, int64_t K,
                                      int64_t tokens_per_sample, const void *scale, const void *ln_weight,
                                      const void *ln_bias, float epsilon, int act_dtype, void *dx, float *dscale,
                                      float *dshift, int accumulate, void *workspace, size_t ws_bytes, void *stream);

/* The gated residual after a block's output projection (transformer.jl:272,
 * 293): out = mixed_add(x, mixed_mul(y, gate[b])) = round(x + round(y * gate[b]))
 * per element of [M][N], b = token / tokens_per_sample, gate [batch][N].
 * out may be x (the residual stream updated in place). */
int reels_gated_residual(const void *x, const void *y, const void *gate, int64_t M, int64_t N,
                         int64_t tokens_per_sample, int act_dtype, void *out, void *stream);

/* Workspace of reels_gated_residual_backward when dgate is requested. */
size_t reels_gated_residual_workspace_bytes(int64_t M, int64_t N, int64_t tokens_per_sample);

/* Its pullback for dout: the residual's gradient is dout itself; dy (nullable)
 * = round(dout * gate[b]); dgate (nullable, fp32 [batch][N], overwritten or
 * with accumulate = 1 added) = the sample's sum of dout * y, in a fixed
 * order. */
int reels_gated_residual_backward(const void *dout, const void *y, const void *gate, int64_t M, int64_t N,
                                  int64_t tokens_per_sample, int act_dtype, void *dy, float *dgate, int accumulate,
                                  void *workspace, size_t ws_bytes, void *stream);

/* ---------------------------------------------------------------------
 * The optimizer step after the gradient all-reduce (src/training/
 * wan_runner.jl:213-227 and AdamW update!, src/training/optimizer.jl:48-73),
 * over all adapter tensors in two launches and without a host round trip:
 *   reels_grad_norm_sq   sum of g^2 over every tensor (the clip's norm^2)
 *   reels_adamw_update   clip by max_norm / norm when norm > max_norm, then
 *                        AdamW with fp32 master weights; the model's copy
 *                        of each parameter is rewritten from its master.
 * One descriptor per parameter tensor; the tensors may differ in length
 * and element type. */
typedef struct reels_opt_tensor {
    void *param;         /* [n] the model's copy, element type param_dtype   */
    const float *grad;   /* [n] fp32 gradient (all-reduced)                  */
    float *m;            /* [n] fp32 first moment                            */
    float *v;            /* [n] fp32 second moment                           */
    float *master;       /* [n] fp32 master weight                           */
    int64_t n;
    int param_dtype;     /* REELS_F32, REELS_F16 or REELS_BF16               */
    int decay;           /* 0: excluded from weight decay (weight_decay_mask) */
} reels_opt_tensor;

/* Bytes of the optimizer workspace for `count` descriptors: the descriptor
 * table (kept between steps) and the norm's partial sums. */
size_t reels_opt_workspace_bytes(int count);

/* Validate the descriptors and store them in `workspace` (device memory,
 * 256-byte aligned, reels_opt_workspace_bytes(count) bytes), which then
 * stands for this set of tensors in the calls below until it is prepared
 * again.  Done once per set of tensors, not per step: it synchronises
 * `stream` after the copy so `tensors` may be released on return. */
int reels_opt_prepare(const reels_opt_tensor *tensors, int count, void *workspace, size_t ws_bytes, void *stream);

/* *sumsq (device fp32) = sum over the prepared tensors of (grad_scale*g)^2,
 * the norm_squared of wan_runner.jl:215 (grad_scale: a factor applied first,
 * e.g. the 1/gradient_accumulation of wan_runner.jl:212).  Accumulated in
 * fp64 in a fixed order, then rounded: the same inputs give the same bits. */
int reels_grad_norm_sq(void *workspace, float grad_scale, float *sumsq, void *stream);

/* AdamW step `update!` (optimizer.jl:48-73) for every prepared tensor:
 *   g  = grad_scale * grad; if sumsq is given: norm = sqrt(*sumsq), and when
 *        norm > max_norm, g = g * (max_norm / norm)   (wan_runner.jl:218-221)
 *   m  = beta1 m + (1 - beta1) g ;  v = beta2 v + (1 - beta2) g^2
 *   master -= lr ((m / correction1) / (sqrt(v / correction2) + eps)
 *                 + decay * weight_decay * master)
 *   param  = master rounded to param_dtype
 * correction1/2 are 1 - beta1^step and 1 - beta2^step of the step being
 * taken (the caller counts steps).  Each operation is rounded once in fp32,
 * with no fused multiply-add, as the reference's broadcasts evaluate it. */
int reels_adamw_update(void *workspace, float lr, float beta1, float beta2, float eps, float weight_decay,
                       float correction1, float correction2, float grad_scale, const float *sumsq, float max_norm,
                       void *stream);

#ifdef __cplusplus
}
#endif

#endif /* REELS_LOWVRAM_H */
