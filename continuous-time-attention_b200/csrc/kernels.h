// Internal launch descriptors shared by the C ABI (capi.cu) and the kernel
// translation units.  Host-only code sees plain structs; nothing here is part
// of the public ABI (that is include/cta_stencil.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cta {

constexpr int kMaxSteps = 8;

// ---------------------------------------------------------------------------
// [B, L, D] layout (feature axis contiguous): TMA-fed march along L
// ---------------------------------------------------------------------------
constexpr int kBldRC = 16;                    // row granularity of the tile sizes
constexpr int kBldMaxTL = 2048;               // max output rows per CTA tile
// forward kernel: one warp per CTA running its own pipeline; 4 columns per
// lane (two packed pairs) -> 128-column tiles, one TMA box per 8-row chunk
constexpr int kFwdThreads = 32;
constexpr int kFwdVec = 4;  // columns per lane (two packed pairs)
constexpr int kFwdDT = 32 * kFwdVec;
constexpr int kFwdRC = 8;
#ifndef CTA_FWD_STAGES
#define CTA_FWD_STAGES 3
#endif
#ifndef CTA_FWD_PRELOAD
#define CTA_FWD_PRELOAD 1
#endif
#ifndef CTA_FWD_MIN_CTAS
#define CTA_FWD_MIN_CTAS 16
#endif
constexpr int kFwdStages = CTA_FWD_STAGES;     // input chunks in flight
constexpr int kFwdMinCtas = CTA_FWD_MIN_CTAS;  // register budget (one-warp CTAs per SM) of the shallow variants
#ifndef CTA_FWD_OUT_SLOTS
#define CTA_FWD_OUT_SLOTS 2
#endif
#ifndef CTA_FWD_DIAG
#define CTA_FWD_DIAG 1
#endif
// forward march: lane 0's per-chunk TMA issue as predicated instructions of the
// whole warp (1) or inside a lane-0 branch (0)
#ifndef CTA_FWD_PRED
#define CTA_FWD_PRED 1
#endif
#ifndef CTA_FWD_EARLY_REFILL
#define CTA_FWD_EARLY_REFILL 0
#endif
// output staging chunks for the TMA stores (0: plain vector stores, no staging)
constexpr int kFwdOutSlots = CTA_FWD_OUT_SLOTS;
// d(alpha) workspace: a fixed header of completion counters (so that no shape's
// partial sums can land where another shape's counters live), then partials
constexpr int64_t kWsHeaderBytes = 8192;
constexpr int kWsMaxGroups = static_cast<int>(kWsHeaderBytes / 4) - 1;
constexpr int kDaMaxSteps = 8;  // steps handled by the march d(alpha) kernel
constexpr int kPdeMaxSteps = 4;  // advection / reaction layers fused per forward launch
// march d(alpha) kernel: full chunks whose pairings all lie inside the tile
// skip the per-row range test (1) or keep it (0)
#ifndef CTA_DA_INNER
#define CTA_DA_INNER 1
#endif
// march d(alpha) kernel: packed column pairs per lane (1: 64-column tiles, half
// the per-lane state of two pairs, twice the resident warps)
#ifndef CTA_DA_PAIRS
#define CTA_DA_PAIRS 1
#endif
constexpr int kDaPairs = CTA_DA_PAIRS;
constexpr int kDaDT = 64 * kDaPairs;  // columns per CTA (TMA box inner extent)
constexpr int kBldMaxWords = (kBldMaxTL + 2 * 2 * kMaxSteps + kBldRC + 31) / 32 + 1;
constexpr int kPoolThreads = 1024;  // masked-pool finish: 32 columns x 32 tile strides

struct BldArgs {
  // streams (element pointers); columns are contiguous
  const void* x;  // forward: input u_0.  backward: x for d(alpha) (nullable)
  const void* g;  // backward: grad of the output (level S)
  void* y;        // forward: output.  backward: grad of the input
  int64_t xsB, xsL, gsB, gsL, ysB, ysL;  // element strides (batch, row)
  int64_t L;      // rows of the addressed tensor (dense: rows per batch; varlen: packed rows)
  int D;          // columns
  int nbatch;     // dense: B.  varlen: number of sequences
  // varlen segmentation (cu_seqlens on the device, int32, nbatch+1 entries)
  const int32_t* cu_seqlens;
  int pad_to_max;   // emulate zero padding up to max_len (reference packed-prefill rule)
  int64_t max_len;
  // global row position of local row 0 and the global sequence length
  // (L-sharding: rows outside [0, L) come from the neighbour halos below)
  int64_t pos_offset, global_len;
  const void* lo_ext;  // [nbatch, hext_lo, D] rows just before local row 0 (nullable)
  const void* hi_ext;  // [nbatch, hext_hi, D] rows just after local row L-1 (nullable)
  int hext_lo, hext_hi;
  // attention mask [B, L] (nullable): a row updates only if its 3 stencil rows are valid
  const void* mask;
  int mask_dtype;
  int64_t msB, msL;
  // tiling: output rows [out_begin, out_end) in tiles of TL rows
  int TL;
  int64_t out_begin, out_end;
  int use_tma;
  int y_quad_ok;  // output rows allow aligned 4-column vector stores
  int use_tma_store;  // the output tensor map is valid: full chunks leave through TMA stores
  float neg_zero;  // -0.0f: run-time additive identity (see pmul_sep)
  // per-step coefficients: host values, or device scalars when alpha_dev[k] != nullptr
  float alpha[kMaxSteps];
  const void* alpha_dev[kMaxSteps];
  int alpha_dev_dtype;
  // backward with d(alpha): per-CTA partial sums + completion counter (caller scratch)
  float* dalpha_partial;   // [num_ctas * steps]
  unsigned int* counter;   // zero on entry, left zero on exit
  float* dalpha;           // [steps] fp32 result
  int num_ctas;
  int dalpha_group;        // CTAs per reduction group (march d(alpha) kernel)
  int dalpha_accumulate;   // add the result to dalpha[] instead of overwriting it
  // forward only: y = residual + stencil(x), the residual [B, L, D] / [T, D]
  // with element strides (rsB, rsL), added as an elementwise add of type T
  const void* residual;
  int64_t rsB, rsL;
  // 0: diffusion.  1 / 2: advection- / reaction-diffusion layer steps.  The
  // forward reads level k's beta from beta_dev[k] (device scalar of
  // alpha_dev_dtype) or beta[k]; the backward (steps 1) from coefficient slot 1
  int pde_kind;
  const void* beta_dev[kMaxSteps];
  float beta[kMaxSteps];
  // forward only: masked mean pool of the output instead of storing it,
  // per-CTA column sums [nbatch][row tiles][D] (fp32, caller scratch)
  float* pool_partial;
  // L-shard halos of the gradient stream for the d(alpha) kernel (lo_ext/hi_ext
  // above hold the x stream's): [nbatch, g_hext_lo|hi, D]
  const void* g_lo_ext;
  const void* g_hi_ext;
  int g_hext_lo, g_hext_hi;
  // diffusion with 16-bit I/O: the contracted update (one fma for c + alpha *
  // lap, the reference's Triton op order; g + alpha * lap(a) in the adjoint)
  // instead of the exact one
  int contract;
  // test hook (forward march only, 0 = off): CTA (0, 0, 0) waits this many
  // microseconds on an mbarrier phase that nothing completes, then takes the
  // timeout path (error word, drain of its issued loads, early exit)
  int debug_stall_us;
};

// ---------------------------------------------------------------------------
// [B, D, L] layout (sequence axis contiguous): warp windows with shuffles
// ---------------------------------------------------------------------------
constexpr int kBdlThreads = 256;  // 8 warps, each owns two 256-wide windows
constexpr int kBdlElems = 8;      // positions per lane
constexpr int kBdlOut = 240;      // output positions per window (30 lanes)
constexpr int kBdlWin = 256;      // loaded positions per window (32 lanes x 8)
#ifndef CTA_BDL_ROWS
#define CTA_BDL_ROWS 2
#endif
constexpr int kBdlRows = CTA_BDL_ROWS;  // rows per one-warp CTA of the TMA form (pairs of pair halves)
constexpr int kBdlStages = 4;     // input windows in flight per CTA (TMA form)
// staging slot of the TMA form: kBdlRows x kBdlOut elements, rounded up to 128 bytes
template <typename T>
constexpr int bdl_out_slot_elems() {
  return ((kBdlRows * kBdlOut * static_cast<int>(sizeof(T)) + 127) / 128) * 128 / static_cast<int>(sizeof(T));
}

struct BdlArgs {
  const void* in;   // forward: x.  backward: grad_out
  void* out;
  int64_t rows;     // B * D
  int64_t D;        // to map row -> batch for the mask
  int64_t L;
  int64_t in_rs, out_rs;  // row strides (elements)
  int vec_ok;             // 16-byte vector access is legal for every row
  float neg_zero;         // -0.0f: run-time additive identity (see pmul_sep)
  const void* mask;
  int mask_dtype;
  int64_t msB, msL;
  float alpha[kMaxSteps];
  const void* alpha_dev[kMaxSteps];
  int alpha_dev_dtype;
  // TMA form: windows per CTA and CTAs per row pair
  int tw, nseg;
  // forward with 16-bit I/O: the contracted update (see BldArgs::contract)
  int contract;
};

// launch march kernels with programmatic dependent launch (tuning key 3)
int pdl_enabled();

// launchers (return cudaError_t of the launch)
// resident one-warp CTAs per SM of a march kernel variant on the current device
// (occupancy query, cached), or -1
int bld_march_ctas_per_sm(int dtype, int steps, int causal, int adjoint, int residual = 0, int contract = 0);
// reduces the pooled partials of a POOL march launch with `ntl` row tiles into
// pooled [nbatch, D] of the tensor dtype
cudaError_t launch_pool_finish(const BldArgs& a, int dtype, int64_t ntl, void* pooled, cudaStream_t st);
// march kernel: forward (adjoint = 0) or the adjoint without d(alpha) (adjoint = 1)
// rmap: residual map (box as ymap), read only when a.residual is set (non-causal forward)
cudaError_t launch_bld_fwd(const BldArgs& a, const CUtensorMap* xmap, const CUtensorMap* ymap,
                           const CUtensorMap* rmap, int dtype, int steps, int causal, int adjoint, dim3 grid,
                           size_t smem, cudaStream_t st);
cudaError_t launch_bdl(const BdlArgs& a, int dtype, int steps, int causal, int backward, cudaStream_t st);
// [B, D, L] TMA form: in map box {kBdlWin, kBdlRows}, out map box {kBdlOut, kBdlRows}
cudaError_t launch_bdl_march(const BdlArgs& a, const CUtensorMap* imap, const CUtensorMap* omap, int dtype,
                             int steps, int causal, int backward, unsigned grid, cudaStream_t st);
int bdl_march_ctas_per_sm(int dtype, int steps, int causal, int backward, int contract = 0);
size_t bdl_march_smem_bytes(int dtype);

// march kernel with d(alpha), steps 1..kDaMaxSteps
cudaError_t launch_bld_dalpha(const BldArgs& a, const CUtensorMap* gmap, const CUtensorMap* xmap,
                              const CUtensorMap* ymap, int dtype, int steps, int causal, dim3 grid, cudaStream_t st);
int bld_dalpha_ctas_per_sm(int dtype, int steps, int causal, int contract = 0);
size_t dalpha_smem_bytes(int dtype, int steps, int causal);
int read_device_error_bld_dalpha(int clear);

// sets the thread-local message returned by cta_last_error()
void set_last_error(const char* fmt, ...) __attribute__((format(printf, 1, 2)));

size_t fwd_smem_bytes(int dtype);
int read_device_error_bld_fwd(int clear);
int read_device_error_bdl(int clear);

}  // namespace cta
