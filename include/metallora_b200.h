/*
 * metallora_b200 -- C ABI of the B200 (sm_100a) LoRA-linear kernels.
 *
 * Drop-in boundary for the LoRA-linear hot path of Wilbatronic/MetalLora.  The
 * reference exposes this path as Python functions over MLX arrays
 * (python/metal_lora/ops.py, kernels.py and the .metal files under kernels/); every entry point
 * below names the reference interface it replaces.
 *
 * Conventions
 *   - All tensor arguments are DEVICE pointers of the current CUDA device,
 *     row-major and contiguous unless a leading dimension says otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call only enqueues work on that stream; none synchronises.
 *   - Return value: MLORA_OK (0) or a negative MLORA_ERR_* code; the detail is
 *     in mlora_last_error_message() (thread-local).  Arguments are validated
 *     before anything is launched.
 *   - The library never allocates device memory during a call.  Calls that
 *     need scratch take a caller-owned `workspace` whose size comes from the
 *     matching *_workspace_bytes query.
 *   - Kernels bound every internal wait.  A wait that runs out records a code
 *     in a per-device status word (mlora_device_status) instead of hanging.
 *   - Shapes: M tokens, K in_features, N out_features, r LoRA rank (1..256).
 *     The tensor-core paths need K % 8 == 0 and r % 8 == 0 (16-byte TMA row
 *     alignment), and N % 8 == 0 for the backward (rows of dy); the Python
 *     layer zero-pads the rank to a multiple of 8, which leaves every result
 *     unchanged.
 */
#ifndef METALLORA_B200_H_
#define METALLORA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MLORA_API __attribute__((visibility("default")))
#else
#define MLORA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MLORA_OK 0
#define MLORA_ERR_INVALID_ARG -1   /* bad pointer, shape, stride or alignment */
#define MLORA_ERR_UNSUPPORTED -2   /* valid request this build does not handle */
#define MLORA_ERR_CUDA -3          /* CUDA runtime/driver error */
#define MLORA_ERR_WORKSPACE -4     /* workspace too small or misaligned */
#define MLORA_ERR_DEVICE -5        /* device is not sm_100 */

/* ---- element types ----------------------------------------------------- */
#define MLORA_DTYPE_BF16 0
#define MLORA_DTYPE_F16 1
#define MLORA_DTYPE_F32 2

/* ---- library / device -------------------------------------------------- */

/* Version of this ABI (major*10000 + minor*100 + patch). */
MLORA_API int mlora_version(void);

/* Human-readable name of a status code. */
MLORA_API const char* mlora_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
MLORA_API const char* mlora_last_error_message(void);

/* 1 if `device` is an sm_100 GPU these kernels run on, else 0.
 * Replaces kernels.is_metal_available() (python/metal_lora/kernels.py:502). */
MLORA_API int mlora_device_supported(int device);

/* Reads (and with reset != 0 clears) the status word of the current device.
 * *out = 0 when no kernel has recorded a fault: 0x101-0x106 a bounded wait
 * timed out (the kernel gave up instead of hanging); 0x107 a gathered row
 * index was outside its table; 0x108 a peer GPU missed a barrier.  Synchronous. */
MLORA_API int mlora_device_status(uint32_t* out, int reset);

/* ---- measurement ------------------------------------------------------- */

/* Number of kernels this library has launched in this process (all devices). */
MLORA_API long long mlora_launch_count(void);

/* Enables (on != 0) or disables timing of every launch with a pair of CUDA
 * events recorded on the launch stream.  Off by default; costs two event
 * records per launch while on. */
MLORA_API int mlora_profile_enable(int on);

/* Sums the recorded launch times per kernel kind (0 GEMM, 1 rank projection,
 * 2 weight gradient, 3 elementwise, 4 quantisation, 5 GEMV, 6 optimizer) into
 * total_ms[0..nkinds) and counts into launches[0..nkinds); waits for the
 * recorded events.  reset != 0 clears the records. */
MLORA_API int mlora_profile_read(double* total_ms, long long* launches, int nkinds, int reset);

/* ---- fused LoRA linear ------------------------------------------------- */

/* Bytes of workspace mlora_lora_forward needs for this shape and dtype. */
MLORA_API size_t mlora_lora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                    int dtype);

/* y[M,N] = x[M,K].w0[N,K]^T + (alpha/r) (x.a[r,K]^T).b[N,r]^T
 * Replaces ops.lora_forward (python/metal_lora/ops.py:32-103, pure-MLX path
 * :91-94) and kernels.lora_forward_metal (kernels.py:507-566).  dtype is
 * BF16 or F16 for x, w0, a, b and y (fp32 accumulation), or F32: every
 * operand is split into bf16 hi/lo parts and the three significant partial
 * products are accumulated in fp32 on the tensor cores (about 2^-16 relative
 * error per product; saved_xa must then be NULL).
 * saved_xa (optional, may be NULL): receives (alpha/r).(x.a^T)^T as [r_pad, ldm]
 * of the same dtype, r_pad = the smallest power of two >= max(r, 16) and
 * ldm = M rounded up to a multiple of 8 -- the input mlora_lora_backward takes
 * to skip recomputing it (the Ax cache of kernels/lora_train.metal:66). */
MLORA_API int mlora_lora_forward(const void* x, const void* w0, const void* a, const void* b, void* y,
                       void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                       int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace mlora_lora_backward needs for this shape and dtype. */
MLORA_API size_t mlora_lora_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                     int dtype);

/* Gradients of y = x.w0^T + s (x.a^T).b^T, s = alpha/r:
 *   dx = dy.w0 + s (dy.b).a                      (optional: w0/dx may be NULL)
 *   da = s (dy.b)^T . x      -> fp32 [r, K]
 *   db = s dy^T . (x.a^T)    -> fp32 [N, r]
 * clipped elementwise to [-clip_value, clip_value] when clip_value > 0.
 * Replaces ops.lora_backward (python/metal_lora/ops.py:117-155, which clips the
 * summed gradients, default 1.0) and kernels.lora_backward_metal
 * (kernels.py:569-612); dx is the autodiff gradient of ops.py:91-94.
 * saved_xa: the [r_pad, ldm] output of mlora_lora_forward, or NULL to recompute
 * (always recomputed for F32).  dy, x, w0, a, b, dx share `dtype`. */
MLORA_API int mlora_lora_backward(const void* dy, const void* x, const void* w0, const void* a,
                        const void* b, const void* saved_xa, void* dx, float* da, float* db,
                        int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                        float clip_value, int dtype, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Flags of mlora_lora_backward_ex. */
#define MLORA_BWD_ACCUMULATE 1 /* da += result, db += result (after the clip) */
#define MLORA_BWD_DEFER_DX 2   /* everything but the dx GEMM; s.dy.B stays in the workspace */
#define MLORA_BWD_DX_ONLY 4    /* only the dx GEMM, from a MLORA_BWD_DEFER_DX call's workspace */
#define MLORA_BWD_GRADS_16BIT 8 /* da, db point to `dtype` (bf16/f16) buffers, not fp32 */

/* mlora_lora_backward with flags; with MLORA_BWD_ACCUMULATE the weight
 * gradients are added into da/db (gradient accumulation across micro-batches,
 * the reference trainer's gradient_accumulation_steps, trainer.py:82).
 * MLORA_BWD_DEFER_DX then MLORA_BWD_DX_ONLY split one backward in two calls
 * (same arguments, same workspace, same stream; 16-bit dtypes, dx set): the
 * caller can start work that needs only da/db -- a data-parallel gradient
 * exchange on another stream -- while the dx GEMM runs.  MLORA_BWD_GRADS_16BIT
 * stores da/db rounded to `dtype` (sums still accumulate in fp32), for
 * callers whose A/B parameters are 16-bit (the reference keeps gradients in the
 * parameters' dtype, ops.py:144-155). */
MLORA_API int mlora_lora_backward_ex(const void* dy, const void* x, const void* w0, const void* a,
                                     const void* b, const void* saved_xa, void* dx, float* da,
                                     float* db, int64_t M, int64_t K, int64_t N, int64_t r,
                                     float alpha, float clip_value, int dtype, int flags,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* ---- merged weights ------------------------------------------------------ */

/* Bytes of workspace mlora_linear needs (0 except for F32). */
MLORA_API size_t mlora_linear_workspace_bytes(int64_t M, int64_t K, int64_t N, int dtype);

/* y[M,N] = x[M,K] . w[N,K]^T -- the forward after the adapter is merged.
 * Replaces ops.lora_forward_inference (python/metal_lora/ops.py:106-114) and the
 * merged-mode call of LoRALinear (layers.py:112-117 then :92). */
MLORA_API int mlora_linear(const void* x, const void* w, void* y, int64_t M, int64_t K, int64_t N,
                           int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace mlora_merge needs (0 except for F32). */
MLORA_API size_t mlora_merge_workspace_bytes(int64_t N, int64_t K, int64_t r, int dtype);

/* w_out[N,K] = w0 + (alpha/r) . b[N,r] . a[r,K]; w_out may alias w0 (in place).
 * K and r must be multiples of 8; N is free.
 * Replaces ops.merge_lora_weights (python/metal_lora/ops.py:162-172), used by
 * LoRALinear.merge_weights / to_inference_mode (layers.py:108-117).  Runs as a
 * tensor-core GEMM over the rank with w0 added in the epilogue, so w0 is read
 * once and w_out written once. */
MLORA_API int mlora_merge(const void* w0, const void* a, const void* b, void* w_out, int64_t N,
                          int64_t K, int64_t r, float alpha, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ---- quantised base weights ---------------------------------------------
 * Layouts (the reference shaders' conventions, kernels/lora_quantized.metal):
 *   NF4 : codes uint8 [N, K/2], low nibble = even k, high nibble = odd k
 *         (:70-74); scales = absmax fp32 [N, ceil(K/group)] (:122,:135);
 *         w = NF4_LEVELS[code] * absmax with the 4-decimal levels (:10-15).
 *   INT4: codes as NF4; scales and zeros fp16 [N, ceil(K/group)];
 *         w = (q - zero) * scale (:17-20; the reference uses one fp32 scale and
 *         zero per row, which is group = K here).
 *   INT8: codes uint8 [N, K]; scales/zeros as INT4.  (The reference promises
 *         int8 but has no kernel for it.) */
#define MLORA_QUANT_NF4 1
#define MLORA_QUANT_INT4 2
#define MLORA_QUANT_INT8 3

/* Quantises w [N,K] (BF16/F16/F32) into codes/scales/zeros (zeros unused for
 * NF4).  NF4: per (row, block of `group`) absmax, nearest level (first on
 * ties).  INT4/INT8: asymmetric per (row, group): scale = (max-min)/(2^b-1)
 * rounded up to fp16, zero = rint(-min/scale), q = rint(w/scale) + zero, both
 * clamped to [0, 2^b-1].  The reference has no quantiser; this is the format's
 * producer for the kernels below. */
MLORA_API int mlora_quantize(const void* w, int w_dtype, int64_t N, int64_t K, int scheme,
                             int64_t group, void* codes, void* scales, void* zeros, void* stream);

/* out [N,K] = dequantised weights in out_dtype.  F32 output is bit-identical to
 * the reference's dequant_nf4 / dequant_int4 (lora_quantized.metal:17-25);
 * BF16/F16 output is that value rounded to nearest even -- exactly the operand
 * the quantised GEMMs feed the tensor cores. */
MLORA_API int mlora_dequantize(int scheme, const void* codes, const void* scales,
                               const void* zeros, int64_t N, int64_t K, int64_t group, void* out,
                               int out_dtype, void* stream);

/* Bytes of workspace mlora_qlora_forward / mlora_qlora_backward need for the
 * staged path (the fastest): it includes a bf16 [N, K] copy of the
 * dequantised weight, made by one HBM-bound pass at the start of each call. */
MLORA_API size_t mlora_qlora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                     int scheme, int64_t group);
MLORA_API size_t mlora_qlora_backward_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                      int scheme, int64_t group);
/* The smallest workspace the quantised paths accept (backward != 0: for
 * mlora_qlora_backward).  With less than the staged size and at least this
 * much, the fused kernel runs instead: it dequantises inside the tensor-core
 * main loop and keeps no dense copy of the weight.  Results are identical. */
MLORA_API size_t mlora_qlora_lean_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t r,
                                                  int scheme, int64_t group, int backward);

/* The prepared scale table of a quantised weight: its per-row scales re-laid
 * as [ceil(K/group), N rounded up to 4] -- fp32 absmax for NF4, (scale, zero)
 * fp16 pairs for INT4/INT8 -- so that one TMA box holds a block of rows'
 * scales.  The decode kernel and the fused kernel read scales only from it;
 * without one, each call builds it in its workspace.  No reference
 * counterpart (the reference reads its per-row scales directly,
 * kernels/lora_quantized.metal:122, :64-65). */
MLORA_API size_t mlora_qlora_prepared_scales_bytes(int scheme, int64_t N, int64_t K, int64_t group);
MLORA_API int mlora_qlora_prepare_scales(int scheme, const void* scales, const void* zeros,
                                         int64_t N, int64_t K, int64_t group, void* out,
                                         void* stream);

/* y[M,N] = x . deq(W)^T + (alpha/r)(x . a^T) . b^T over a quantised base weight
 * (codes/scales/zeros as above; x, a, b, y BF16).  Replaces qlora_forward_nf4
 * (kernels/lora_quantized.metal:97-164) and qlora_forward_int4 (:29-93).  The
 * GEMM operand is bf16(dequant(W)) -- staged in the workspace, or formed in
 * the fused kernel's main loop (lean workspace); up to 16 tokens without
 * saved_xa, a GEMV dequantises in registers.  group (NF4 block size / INT
 * group) must be 64, 128 or 256; K a multiple of 32 (4-bit) or 16 (INT8).
 * saved_xa as for mlora_lora_forward. */
MLORA_API int mlora_qlora_forward(const void* x, int scheme, const void* codes, const void* scales,
                                  const void* zeros, int64_t group, const void* a, const void* b,
                                  void* y, void* saved_xa, int64_t M, int64_t K, int64_t N,
                                  int64_t r, float alpha, int dtype, void* workspace,
                                  size_t workspace_bytes, void* stream);
/* Same, with the weight's prepared scale table (may be NULL). */
MLORA_API int mlora_qlora_forward_ex(const void* x, int scheme, const void* codes,
                                     const void* scales, const void* zeros, const void* prepared,
                                     int64_t group, const void* a, const void* b, void* y,
                                     void* saved_xa, int64_t M, int64_t K, int64_t N, int64_t r,
                                     float alpha, int dtype, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Gradients through the quantised base (frozen, as in QLoRA): dx = dy . deq(W)
 * + s (dy . b) . a (staged or lean as for the forward; dx may be NULL, then
 * the codes are not read), da, db as mlora_lora_backward_ex (flags:
 * MLORA_BWD_ACCUMULATE). */
MLORA_API int mlora_qlora_backward(const void* dy, const void* x, int scheme, const void* codes,
                                   const void* scales, const void* zeros, int64_t group,
                                   const void* a, const void* b, const void* saved_xa, void* dx,
                                   float* da, float* db, int64_t M, int64_t K, int64_t N,
                                   int64_t r, float alpha, float clip_value, int dtype, int flags,
                                   void* workspace, size_t workspace_bytes, void* stream);
/* Same, with the weight's prepared scale table (may be NULL). */
MLORA_API int mlora_qlora_backward_ex(const void* dy, const void* x, int scheme, const void* codes,
                                      const void* scales, const void* zeros, const void* prepared,
                                      int64_t group, const void* a, const void* b,
                                      const void* saved_xa, void* dx, float* da, float* db,
                                      int64_t M, int64_t K, int64_t N, int64_t r, float alpha,
                                      float clip_value, int dtype, int flags, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* ---- multiple adapters in one batch ------------------------------------ */

/* Token m uses adapter ids[m] of n adapters stacked in one pair of tensors:
 *   y[m,:] = (w0 ? x[m] . w0^T : 0) + (alpha/r) (x[m] . A_g^T) . B_g^T,  g = ids[m]
 * a_stack [n*r, K]: adapter g's A in rows g*r .. g*r+r-1; b_stack [N, n*r]:
 * adapter g's B in columns g*r .. g*r+r-1; ids [M] int32 on the device (an id
 * outside [0, n) adds no LoRA term).  n*r <= 256, r a multiple of 8, BF16 or
 * F16.  One pass over x projects onto all n adapters (the rank kernel keeps
 * each row's own adapter block), then the tcgen05 GEMM adds the stacked
 * up-projection as extra k-blocks.  Replaces
 * MultiAdapterManager.forward_batched (python/metal_lora/optimizations.py:193-217;
 * w0 = NULL, alpha = r) and the lora_multi_adapter kernel
 * (kernels/lora_kernels.metal:440-508). */
MLORA_API size_t mlora_multi_lora_forward_workspace_bytes(int64_t M, int64_t K, int64_t N,
                                                          int64_t r, int64_t n, int dtype);
MLORA_API int mlora_multi_lora_forward(const void* x, const void* w0, const void* a_stack,
                                       const void* b_stack, const int32_t* ids, void* y,
                                       int64_t M, int64_t K, int64_t N, int64_t r, int64_t n,
                                       float alpha, int dtype, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ---- KV-cache update (incremental decoding) ----------------------------- */

/* One new token per sequence: for b < batch,
 *   k_cache[b, cur_pos, :] = x[b] . wk^T + (alpha/r) (x[b] . ak^T) . bk^T
 *   v_cache[b, cur_pos, :] = x[b] . wv^T + (alpha/r) (x[b] . av^T) . bv^T
 * x [batch, D_in]; wk, wv [D_kv, D_in]; ak, av [r, D_in]; bk, bv [D_kv, r];
 * caches [batch, max_seq, D_kv] (D_kv = heads * head_dim), BF16/F16.  Each
 * projection writes its rows straight into the cache slot (decode kernel for
 * up to 16 sequences, tcgen05 GEMM above).  Replaces lora_kv_cache_update
 * (kernels/lora_kernels.metal:514-586; max_seq is a parameter here, not 8192)
 * with LoRAKVCache.update (python/metal_lora/optimizations.py:327-336). */
MLORA_API size_t mlora_lora_kv_cache_workspace_bytes(int64_t batch, int64_t D_in, int64_t D_kv,
                                                     int64_t r, int dtype);
MLORA_API int mlora_lora_kv_cache_update(const void* x, const void* wk, const void* wv,
                                         const void* ak, const void* bk, const void* av,
                                         const void* bv, void* k_cache, void* v_cache,
                                         int64_t batch, int64_t cur_pos, int64_t max_seq,
                                         int64_t D_in, int64_t D_kv, int64_t r, float alpha,
                                         int dtype, void* workspace, size_t workspace_bytes,
                                         void* stream);

/* ---- data-parallel gradient exchange ----------------------------------- */

/* out = scale * sum over ranks of their fp32 buffers [n], in rank order (the
 * same bits on every rank), in one kernel over NVLink peer memory.  bufs and
 * flags are DEVICE arrays of `world` pointers: each rank's buffer and its
 * `world`-word flag array, both in memory every rank can address (e.g.
 * symmetric memory); flags start at 0; seq counts calls from 1; counter is an
 * array of 4 device words on this GPU, owned by the caller and zeroed before
 * the first call.  `out` must not alias this rank's buffer (peers read the
 * buffer while `out` is written).  Every rank calls it once per step on its
 * own GPU; when it completes no peer reads this rank's buffer any more.  A
 * peer that does not arrive within 2 s sets status 0x108 (no hang); the
 * go/abort decision is taken once for the whole grid, so on a timeout `out`
 * is left untouched (never partly written).
 * Replaces the NCCL all-reduce of the LoRA gradients for small buffers (the
 * reference has no multi-device path: python/metal_lora/trainer.py:228-249 is
 * single-device). */
MLORA_API int mlora_peer_allreduce(const void* bufs, const void* flags, int rank, int world,
                                   uint32_t seq, float* out, int64_t n, float scale,
                                   uint32_t* counter, void* stream);

/* ---- LoRA embedding ----------------------------------------------------- */

/* out[t, :] = table[idx[t], :] + (alpha/r) * b[idx[t], :] . a  (LoRAEmbedding.__call__,
 * python/metal_lora/layers.py:220-225).  table [V, D], a [r, D], b [V, r],
 * idx [T] int32 on the device; BF16/F16 run on the tensor cores (D, r
 * multiples of 8), F32 on CUDA cores.  An index outside [0, V) gives a zero
 * row and sets the device status word. */
MLORA_API size_t mlora_lora_embedding_workspace_bytes(int64_t T, int64_t D, int64_t r, int dtype,
                                                      int backward);
MLORA_API int mlora_lora_embedding_forward(const int32_t* idx, const void* table, const void* a,
                                           const void* b, void* out, int64_t T, int64_t V,
                                           int64_t D, int64_t r, float alpha, int dtype,
                                           void* workspace, size_t workspace_bytes, void* stream);
/* Gradients of a and b (the table is frozen, layers.py:217-218), fp32:
 *   da[j, :] = (alpha/r) sum_t b[idx[t], j] dy[t, :]
 *   db[v, :] = (alpha/r) sum_{t: idx[t] = v} dy[t, :] . a^T
 * sorted_idx / order: idx sorted stably and the token positions in that order
 * (db rows are summed in that order: deterministic).  flags:
 * MLORA_BWD_ACCUMULATE adds into da/db; otherwise db rows no token uses are
 * zeroed. */
MLORA_API int mlora_lora_embedding_backward(const void* dy, const int32_t* idx,
                                            const int32_t* sorted_idx, const int32_t* order,
                                            const void* a, const void* b, float* da, float* db,
                                            int64_t T, int64_t V, int64_t D, int64_t r, float alpha,
                                            int dtype, int flags, void* workspace,
                                            size_t workspace_bytes, void* stream);

/* ---- optimizer --------------------------------------------------------- */

/* One AdamW step over a flat buffer of n parameters (reference:
 * kernels.lora_adamw_step_metal, python/metal_lora/kernels.py:615-643, kernel
 * :314-344, same operation order, bit-identical in fp32):
 *   g = grad * (*grad_scale or 1);  grad := 0
 *   m = b1 m + (1-b1) g;  v = b2 v + ((1-b2) g) g
 *   p -= lr (m/(1-b1^t) / (sqrt(v/(1-b2^t)) + eps) + wd p)
 * state is the device array [t, b1^t, b2^t] (kernels.py:471-481).  param may be
 * BF16, F16 or F32; grad, m, v are F32.  weight_decay 0 gives Adam. */
MLORA_API int mlora_adamw_step(void* param, float* grad, float* m, float* v, const float* state,
                               int64_t n, float lr, float beta1, float beta2, float eps,
                               float weight_decay, int param_dtype, const float* grad_scale,
                               void* stream);

/* p -= lr * g * (*grad_scale or 1); grad := 0 (the trainer's "sgd" optimizer,
 * python/metal_lora/trainer.py:213-214). */
MLORA_API int mlora_sgd_step(void* param, float* grad, int64_t n, float lr, int param_dtype,
                             const float* grad_scale, void* stream);

/* state := [t+1, b1^(t+1), b2^(t+1)] on the device (reference:
 * kernels.persistent_gpu_state_step, kernels.py:484-499, kernel :351-362). */
MLORA_API int mlora_adam_state_step(float* state, float beta1, float beta2, void* stream);

/* Bytes of workspace mlora_grad_norm_clip needs. */
MLORA_API size_t mlora_grad_norm_workspace_bytes(void);

/* Global-norm clip factor of a flat gradient buffer (trainer.py:237-240):
 * out[1] = ||grad||_2, out[0] = min(1, max_norm / (out[1] + 1e-6)), or 1 when
 * max_norm <= 0.  out is a device float[2]; pass out as grad_scale to the
 * optimizer step.  Deterministic (fixed reduction order). */
MLORA_API int mlora_grad_norm_clip(const float* grad, int64_t n, float max_norm, float* out,
                                   void* workspace, size_t workspace_bytes, void* stream);

/* ---- allocation-free weight gradients -------------------------------------
 * No counterpart in the reference: an addition of this library for callers
 * that cannot allocate device memory when the backward runs (a process whose
 * device memory is all owned by its own pool, or a loop that must not call
 * cudaMalloc because it can wait on the whole device).  It computes what
 * mlora_lora_backward computes with w0 = dx = saved_xa = NULL (da, db, the
 * same clip), taking its scratch from a 32 MiB array built into the library
 * instead of a caller workspace; every GPU that loads the library holds that
 * array until the process exits.
 *   - Shapes whose scratch exceeds the array (see
 *     mlora_lora_grads_static_scratch_bytes) return MLORA_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address (once
 *     per device context, with that device current); make that first call
 *     before any stream capture.  A failed lookup is not remembered (the next
 *     call tries again), and a context that is torn down and re-created
 *     (cudaDeviceReset) gets a fresh lookup on its first call.
 *   - A device index of 64 or more returns MLORA_ERR_UNSUPPORTED.
 *   - All calls on a device share the array: calls whose work overlaps on the
 *     GPU (different streams, no ordering between them) race and corrupt each
 *     other's results.  Each call clears the parts that must start at zero.
 *   - BF16 or F16 only. */
MLORA_API size_t mlora_lora_grads_static_scratch_bytes(void);
MLORA_API int mlora_lora_grads_static(const void* dy, const void* x, const void* a, const void* b,
                                      float* da, float* db, int64_t M, int64_t K, int64_t N,
                                      int64_t r, float alpha, float clip_value, int dtype,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* METALLORA_B200_H_ */
