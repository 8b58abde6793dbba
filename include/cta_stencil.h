/*
 * cta_stencil.h -- C ABI of the B200 (sm_100a) diffusion-stencil library
 * (libcta_stencil.so).
 *
 * The library computes the multi-step diffusion refinement of Continuous-Time
 * Attention,
 *     x[i] <- x[i] + alpha * ((x[i+1] - 2 x[i]) + x[i-1])      (fp32 math)
 * applied `steps` times along the sequence axis with the copy boundary (first
 * and last row unchanged), its causal variant, attention-mask handling, packed
 * variable-length sequences, and the adjoint (backward) with d(alpha).
 *
 * Conventions
 *   - All tensors are device pointers owned by the caller; the library never
 *     allocates device memory.  Strides are in ELEMENTS.
 *   - dtype: CTA_F32 / CTA_BF16 / CTA_F16; the output dtype equals the input
 *     dtype, arithmetic is fp32, results are rounded once at the end.
 *   - Work is enqueued on `stream` (a cudaStream_t, NULL = legacy default);
 *     no call synchronizes or reads device data on the host.
 *   - Return value: CTA_OK, or an error code with a message available from
 *     cta_last_error() (thread-local).  CTA_EINVAL corresponds to the
 *     reference's ValueError, the others to RuntimeError.
 *   - steps: 1..8 (every count has its own fused kernel).  Calls with
 *     steps == 0 or a sequence shorter than 3 rows are the identity and are
 *     handled by the caller (the Python layer mirrors the reference's
 *     aliasing rules for them).
 */
#ifndef CTA_STENCIL_H_
#define CTA_STENCIL_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CTA_ABI_VERSION 1

enum { CTA_F32 = 0, CTA_BF16 = 1, CTA_F16 = 2 };
enum { CTA_MASK_U8 = 0, CTA_MASK_I32 = 1, CTA_MASK_I64 = 2, CTA_MASK_F32 = 3, CTA_MASK_BF16 = 4, CTA_MASK_F16 = 5 };
enum { CTA_OK = 0, CTA_EINVAL = 1, CTA_EUNSUPPORTED = 2, CTA_ECUDA = 3 };
enum { CTA_SHARD_INTERIOR = 0, CTA_SHARD_LO_EDGE = 1, CTA_SHARD_HI_EDGE = 2 };
enum { CTA_PDE_ADVECTION = 0, CTA_PDE_REACTION = 1 };

/* ABI version of the loaded library (CTA_ABI_VERSION). */
int cta_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* cta_last_error(void);

/* Reads (and optionally clears) the device-side error word of every kernel
 * family: 0 = ok, 1 = a bounded wait inside a kernel timed out.  This call
 * synchronizes with the device. */
int cta_device_error(int clear);

/* Benchmark and test hook: key 1 = forced tile rows (0 = automatic), key 2 =
 * target CTAs per SM of the [B, L, D] march kernels (default 16), key 3 = launch
 * the [B, L, D] march kernels with programmatic dependent launch (default 0),
 * key 4 = plain vector stores instead of staged TMA stores in the forward
 * (default 0), key 5 = test of the timeout path: the first CTA of every
 * forward march waits this many microseconds (at most 100000) on an mbarrier
 * phase nothing completes, then reports the timeout in the device error word
 * and exits (default 0 = off).  Returns the previous value.  Process-wide, not
 * thread-safe against concurrent launches. */
int cta_set_tuning(int key, int value);

/* Arithmetic of the forward update c + alpha * lap for 16-bit (bf16 / fp16)
 * tensors; fp32 tensors always use CTA_ARITH_EXACT.
 *   CTA_ARITH_EXACT      : the product rounded to fp32, then the sum rounded --
 *                          the reference's PyTorch path (src/cta/ops/diffusion.py:
 *                          52-53, src/models/pde_layers.py:141-175), bit for bit;
 *   CTA_ARITH_CONTRACTED : product and sum as one fused multiply-add -- the op
 *                          order the reference's Triton kernels compile to
 *                          (kernels/diffusion_triton.py:89-90, :252-259); within
 *                          one bf16 / fp16 rounding of the exact result.
 * Applies to the forward kernels (cta_diffusion_fwd_bdl / _bdl_ex forward,
 * _fwd_bld, _fwd_bld_residual, _fwd_varlen[_residual], _shard_bld) and to the
 * [B, L, D] backward kernels (cta_diffusion_bwd_bld, its _noalloc form,
 * _shard_bld backward, _shard_bld_dalpha), where the adjoint level becomes
 * g + alpha * lap(a) in one fma and the forward recomputation follows the
 * forward's order; the [B, D, L] adjoint, the pooled forward and the
 * advection / reaction steps are always exact.  (The reference has no
 * bit-exact backward to match: its gradients come from autograd or from the
 * Triton adjoint kernel, kernels/diffusion_triton.py:96-133, each with its own
 * order.)  cta_set_arithmetic sets the process default (initially
 * CTA_ARITH_CONTRACTED) and returns the previous one (-1: unknown mode).
 * cta_set_thread_arithmetic overrides it for the calling thread (mode -1 =
 * follow the process default) and returns the thread's previous override. */
#define CTA_ARITH_EXACT 0
#define CTA_ARITH_CONTRACTED 1
int cta_set_arithmetic(int mode);
int cta_set_thread_arithmetic(int mode);

/* ---------------------------------------------------------------------------
 * [B, D, L] layout, L contiguous
 * ------------------------------------------------------------------------- */

/* y = A^steps x.  Replaces kernels/diffusion_triton.py:829-868
 * (_diffusion_fused_triton_forward, steps in {1,2,4,8} there, 1..8 here)
 * and :732-762 (_diffusion_step_triton_forward, steps = 1).
 * x, y: [B, D, L] with row stride `row_stride` (>= L) for both. */
int cta_diffusion_fwd_bdl(const void* x, void* y, int64_t B, int64_t D, int64_t L, int64_t row_stride, int dtype,
                          int steps, float alpha, void* stream);

/* grad_in = (A^T)^steps grad_out.  Replaces kernels/diffusion_triton.py:765-794
 * (diffusion_step_triton_backward, steps = 1) and the host loop of
 * _DiffusionFusedTriton.backward :880-888 (fused into one launch here). */
int cta_diffusion_bwd_bdl(const void* grad_out, void* grad_in, int64_t B, int64_t D, int64_t L, int64_t row_stride,
                          int dtype, int steps, float alpha, void* stream);

/* General [B, D, L] form used by the `layout="bdl"` PDE layers
 * (src/models/pde_layers.py:113-188): causal stencil, attention mask
 * ([B, L], any listed dtype, non-zero = valid, strides mask_sB/mask_sL),
 * one alpha per step given either as host floats (`alpha`, steps entries) or
 * as device scalars (`alpha_dev[k]`, dtype alpha_dev_dtype; entry k used when
 * non-NULL).  backward != 0 applies the adjoint instead. */
int cta_diffusion_bdl_ex(const void* in, void* out, int64_t B, int64_t D, int64_t L, int64_t in_row_stride,
                         int64_t out_row_stride, int dtype, int steps, int causal, int backward, const float* alpha,
                         const void* const* alpha_dev, int alpha_dev_dtype, const void* mask, int mask_dtype,
                         int64_t mask_sB, int64_t mask_sL, void* stream);

/* ---------------------------------------------------------------------------
 * [B, L, D] layout, D contiguous (TMA-fed kernels)
 * ------------------------------------------------------------------------- */

/* Fused forward over `steps` steps.  Replaces, with one launch per call:
 *   - src/cta/serving_vllm.py:29-46 (_diffusion_steps_bld) and the
 *     transpose + Triton + transpose path of CtaPostAttnMixer.forward :234-266;
 *   - a chain of `steps` DiffusionPDELayer(layout="bld") calls,
 *     src/models/pde_layers.py:113-188 with :218-219 (causal, mask, per-layer
 *     alpha), keeping fp32 between the steps. */
int cta_diffusion_fwd_bld(const void* x, void* y, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                          int64_t y_sB, int64_t y_sL, int dtype, int steps, int causal, const float* alpha,
                          const void* const* alpha_dev, int alpha_dev_dtype, const void* mask, int mask_dtype,
                          int64_t mask_sB, int64_t mask_sL, void* stream);

/* Bytes of caller scratch needed by cta_diffusion_bwd_bld when dalpha != NULL
 * (per-CTA partial sums and a completion counter).  The scratch must be
 * zero-filled before its first use; the kernel leaves it reusable. */
int64_t cta_diffusion_bwd_bld_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype, int steps, int causal);

/* Fused backward: grad_in = A_1^T ... A_steps^T grad_out, and when dalpha is
 * non-NULL also dalpha[k] = dLoss/dalpha_k (fp32, steps entries, deterministic)
 * which needs x (the forward input) and `workspace`.  Replaces the autograd
 * backward of the reference PDE layer chain (src/models/pde_layers.py:113-188,
 * per-layer alpha :216-219) and kernels/diffusion_triton.py:765-794,880-888. */
int cta_diffusion_bwd_bld(const void* grad_out, void* grad_in, const void* x, float* dalpha, void* workspace,
                          int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t g_sB, int64_t g_sL,
                          int64_t x_sB, int64_t x_sL, int64_t d_sB, int64_t d_sL, int dtype, int steps, int causal,
                          const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype, const void* mask,
                          int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* Allocation-free form of cta_diffusion_bwd_bld (no counterpart in the
 * reference).  For callers that cannot provide fresh device memory -- an engine
 * that has reserved almost the whole GPU for its own pool, or a latency-critical
 * path that must not pay cudaMalloc's implicit synchronisation -- the d(alpha)
 * scratch comes from a fixed array inside the library (270336 bytes per device,
 * held until the process exits).  Same arguments as cta_diffusion_bwd_bld minus
 * the workspace.  Shapes whose reduction needs more scratch than that (more than
 * 65536 CTA x step partial sums) are rejected with CTA_EINVAL.  The first call on
 * a device looks up the array's device address; make that first call before
 * any stream capture.  The array is shared by every call on a device and keeps
 * the previous call's contents (the completion counters are cleared at the start
 * of each call), so calls whose work overlaps on the GPU race and must be
 * serialised by the caller.  Calls no cudaMalloc, cudaFree or allocating
 * library routine. */
int cta_diffusion_bwd_bld_noalloc(const void* grad_out, void* grad_in, const void* x, float* dalpha, int64_t B,
                                  int64_t L, int64_t D, int64_t g_sB, int64_t g_sL, int64_t x_sB, int64_t x_sL,
                                  int64_t d_sB, int64_t d_sL, int dtype, int steps, int causal, const float* alpha,
                                  const void* const* alpha_dev, int alpha_dev_dtype, const void* mask,
                                  int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* Packed variable-length prefill: x, y are [total_rows, D] (row strides
 * x_sL / y_sL), cu_seqlens is a DEVICE int32 array of nseq+1 offsets.
 *   pad_to_max = 0: every sequence has its own copy boundary and no stencil
 *                   reads across sequences;
 *   pad_to_max = 1: the reference rule of src/cta/serving_vllm.py:72-111,
 *                   275-303 -- each sequence behaves as if zero-padded to
 *                   max_len rows (boundary rows 0 and max_len-1), results
 *                   identical to the reference's packed path.
 * max_len must be >= the longest sequence.  The host never reads cu_seqlens. */
int cta_diffusion_fwd_varlen(const void* x, void* y, int64_t total_rows, int64_t D, int64_t x_sL, int64_t y_sL,
                             const int32_t* cu_seqlens, int64_t nseq, int64_t max_len, int pad_to_max, int dtype,
                             int steps, float alpha, void* stream);

/* Fused residual add of the vLLM decoder layer (no counterpart in the
 * reference, whose patch computes `hidden_states = residual + mixer(x)` in two
 * passes, serving/vllm/patches/vllm_0_13_0_cta_post_attn.patch:66-68):
 * y = residual + stencil(x), the stencil result rounded to the tensor dtype
 * first and the add done as the elementwise add of two tensors of that dtype,
 * so the output equals the two-pass result bit for bit.  One pass: reads x and
 * residual once, writes y once.  residual has y's shape; its own row stride.
 * Non-causal forward only. */
int cta_diffusion_fwd_varlen_residual(const void* x, const void* residual, void* y, int64_t total_rows, int64_t D,
                                      int64_t x_sL, int64_t r_sL, int64_t y_sL, const int32_t* cu_seqlens,
                                      int64_t nseq, int64_t max_len, int pad_to_max, int dtype, int steps,
                                      float alpha, void* stream);

/* The classifier's last refinement and its masked mean pool in one pass
 * (src/models/transformers.py:120-139; no single counterpart in the
 * reference): pooled[b, :] = sum_l mask[b, l] * y[b, l, :] / max(sum_l mask, 1)
 * with y = `steps` fused non-causal steps of x under the same mask, y rounded to
 * the tensor dtype as the stored tensor would hold it, and the sum and the
 * division rounded to that dtype as the reference's half-precision ops do.  y
 * is never written.  pooled: [B, D] contiguous, x's dtype.  workspace: fp32
 * scratch of cta_diffusion_fwd_bld_pool_workspace_bytes(B, L, D) bytes (16-byte
 * aligned, no zeroing).  Two launches. */
int64_t cta_diffusion_fwd_bld_pool_workspace_bytes(int64_t B, int64_t L, int64_t D);
int cta_diffusion_fwd_bld_pool(const void* x, void* pooled, void* workspace, int64_t workspace_bytes, int64_t B,
                               int64_t L, int64_t D, int64_t x_sB, int64_t x_sL, int dtype, int steps,
                               const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype,
                               const void* mask, int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* The dense [B, L, D] form of cta_diffusion_fwd_varlen_residual (mask allowed,
 * host alphas, non-causal). */
int cta_diffusion_fwd_bld_residual(const void* x, const void* residual, void* y, int64_t B, int64_t L, int64_t D,
                                   int64_t x_sB, int64_t x_sL, int64_t r_sB, int64_t r_sL, int64_t y_sB,
                                   int64_t y_sL, int dtype, int steps, const float* alpha, const void* mask,
                                   int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* One step of the reaction-diffusion or advection-diffusion PDE layer on
 * [B, L, D] (src/models/pde_layers.py:249-318 with the forward of :113-188):
 *   y = x + (alpha * lap(x) + beta-term) on updated rows, x on fixed rows;
 *   kind CTA_PDE_ADVECTION: beta * (x[i+1] - x[i-1]) / 2 (causal: beta * (x[i] - x[i-1]));
 *   kind CTA_PDE_REACTION: (beta * x[i]) * (1 - sigmoid(x[i])).
 * alpha_dev / beta_dev are device scalars (the layer parameters, coef_dtype).
 * backward = 0: x -> y (grad_out, dcoef, workspace unused).
 * backward = 1: y = dx for grad_out and the forward input x, dcoef = fp32
 * [d(alpha), d(beta)] (reduced deterministically in the same launch);
 * workspace of cta_pde_step_workspace_bytes(B, L, D) bytes, 256-byte aligned,
 * zeroed once before its first use (the kernel leaves its counters at zero;
 * the d(alpha) workspace layout of cta_diffusion_bwd_bld). */
int64_t cta_pde_step_workspace_bytes(int64_t B, int64_t L, int64_t D);
int cta_pde_step_bld(const void* x, const void* grad_out, void* y, float* dcoef, void* workspace,
                     int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                     int64_t g_sB, int64_t g_sL, int64_t y_sB, int64_t y_sL, int dtype, int kind, int causal,
                     int backward, const void* alpha_dev, const void* beta_dev, int coef_dtype, const void* mask,
                     int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* One shard of an L-sharded sequence ([B, L_local, D], contiguous): rows
 * [pos_offset, pos_offset + L_local) of a sequence of global_len rows.
 * lo_halo: [B, lo_rows, D] contiguous copy of the lo_rows rows just before the
 * shard, hi_halo: [B, hi_rows, D] the hi_rows rows just after it (NULL at a
 * global end).  Rows needed: steps on each side for the non-causal stencil,
 * 2*steps before the shard for the causal forward, 2*steps after it for the
 * causal adjoint.  Edge parts need every halo that exists.
 *   part = CTA_SHARD_INTERIOR : output rows that need no halo (launch while
 *                               the halos are still in flight);
 *   part = CTA_SHARD_LO_EDGE / CTA_SHARD_HI_EDGE : the rows next to the shard
 *                               ends, reading the halos.
 * backward != 0 applies the adjoint to a gradient instead.  No reference
 * counterpart: the reference runs on one device only. */
int cta_diffusion_shard_bld(const void* in, void* out, int64_t B, int64_t L_local, int64_t D, int64_t pos_offset,
                            int64_t global_len, const void* lo_halo, int64_t lo_rows, const void* hi_halo,
                            int64_t hi_rows, int part, int dtype, int steps, int causal, int backward, float alpha,
                            void* stream);

/* The forward of `steps` (1..4) consecutive advection- or reaction-diffusion
 * layers of one kind (src/models/pde_layers.py:249-318, each with the base
 * forward of :113-188) in ONE launch, fp32 kept between the layers (a chain of
 * layer calls rounds to the tensor dtype after each; identical in fp32).
 * alpha_dev[k], beta_dev[k]: layer k's [1] parameters on the device (dtype
 * coef_dtype).  Same layout, mask and causality rules as cta_pde_step_bld; no
 * backward (gradients take one cta_pde_step_bld per layer). */
int cta_pde_stack_bld(const void* x, void* y, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                      int64_t y_sB, int64_t y_sL, int dtype, int kind, int steps, int causal,
                      const void* const* alpha_dev, const void* const* beta_dev, int coef_dtype, const void* mask,
                      int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream);

/* One part of an L-shard's fused backward WITH d(alpha), steps 1..8 (no
 * counterpart in the reference, which is single-device; together with an
 * all-reduce of the per-rank sums it is the sharded form of
 * cta_diffusion_bwd_bld with dalpha).  grad_out, x and grad_in are the local
 * contiguous [B, L_local, D] shards.  Halos are [B, rows, D] contiguous: g_lo /
 * x_lo are the rows just before the shard, g_hi / x_hi just after.  Needed rows:
 * non-causal steps of each halo; causal 2*steps of g_hi and x_lo (g_lo, x_hi
 * unused).  Halos are read only by the edge parts.  The part's d(alpha) sum is
 * ADDED to dalpha (fp32 [steps], zeroed by the caller before the first part);
 * run the parts in one stream so the sum order is fixed.  `workspace` as for
 * cta_diffusion_bwd_bld with L = L_local. */
int cta_diffusion_shard_bld_dalpha(const void* grad_out, const void* x, void* grad_in, float* dalpha,
                                   void* workspace, int64_t workspace_bytes, int64_t B, int64_t L_local, int64_t D,
                                   int64_t pos_offset, int64_t global_len, const void* g_lo_halo, int64_t g_lo_rows,
                                   const void* g_hi_halo, int64_t g_hi_rows, const void* x_lo_halo,
                                   int64_t x_lo_rows, const void* x_hi_halo, int64_t x_hi_rows, int part, int dtype,
                                   int steps, int causal, const float* alpha, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CTA_STENCIL_H_ */
