// C ABI of libcta_stencil.so: argument validation, tile sizing, TMA tensor-map
// encoding and kernel dispatch.  Declarations and contracts live in
// include/cta_stencil.h.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "cta_stencil.h"
#include "kernels.h"

using namespace cta;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CTA_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

int ok() {
  return CTA_OK;
}

size_t dtype_size(int dtype) { return dtype == CTA_F32 ? 4 : 2; }

bool valid_dtype(int dtype) { return dtype == CTA_F32 || dtype == CTA_BF16 || dtype == CTA_F16; }

bool valid_mask_dtype(int d) { return d >= CTA_MASK_U8 && d <= CTA_MASK_F16; }

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

// ---------------------------------------------------------------------------
// TMA tensor maps
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D map over a [nb, rows, D] tensor with element strides (sB, sL, 1); box is
// box_rows rows x box_cols columns.  Returns false when TMA cannot address it.
bool encode_map(CUtensorMap* m, const void* base, int dtype, int64_t nb, int64_t rows, int64_t D, int64_t sB,
                int64_t sL, int box_rows, int box_cols);

// Encoded maps are pure host data; the last few are kept per thread so that
// repeated calls on the same buffers skip the encode.
bool make_map(CUtensorMap* m, const void* base, int dtype, int64_t nb, int64_t rows, int64_t D, int64_t sB,
              int64_t sL, int box_rows, int box_cols) {
  struct Slot {
    const void* base;
    int dtype;
    int box_rows, box_cols;
    int64_t nb, rows, D, sB, sL;
    bool ok;
    CUtensorMap map;
  };
  constexpr int kSlots = 16;
  thread_local Slot cache[kSlots];
  thread_local int next = 0;
  for (int i = 0; i < kSlots; ++i) {
    const Slot& c = cache[i];
    if (c.base == base && base != nullptr && c.dtype == dtype && c.box_rows == box_rows && c.box_cols == box_cols &&
        c.nb == nb &&
        c.rows == rows && c.D == D && c.sB == sB && c.sL == sL) {
      if (c.ok) *m = c.map;
      return c.ok;
    }
  }
  Slot& c = cache[next];
  next = (next + 1) % kSlots;
  c.ok = encode_map(&c.map, base, dtype, nb, rows, D, sB, sL, box_rows, box_cols);
  c.base = base;
  c.dtype = dtype;
  c.box_rows = box_rows;
  c.box_cols = box_cols;
  c.nb = nb;
  c.rows = rows;
  c.D = D;
  c.sB = sB;
  c.sL = sL;
  if (c.ok) *m = c.map;
  return c.ok;
}

bool encode_map(CUtensorMap* m, const void* base, int dtype, int64_t nb, int64_t rows, int64_t D, int64_t sB,
                int64_t sL, int box_rows, int box_cols) {
  auto fn = encode_fn();
  if (fn == nullptr || base == nullptr) return false;
  const int64_t es = static_cast<int64_t>(dtype_size(dtype));
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
  if ((sL * es) % 16 != 0 || sL < D) return false;
  if (rows >= (1LL << 31) - 4096 || D >= (1LL << 31) || nb >= (1LL << 31)) return false;
  int64_t bstride = sB * es;
  if (nb == 1) bstride = ((rows * sL * es + 15) / 16) * 16;
  if (bstride % 16 != 0 || bstride <= 0) return false;
  if (sL * es >= (1LL << 40) || bstride >= (1LL << 40)) return false;
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(nb)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(sL * es), static_cast<cuuint64_t>(bstride)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt = dtype == CTA_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == CTA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(m, dt, 3, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// tile sizing: enough CTAs for ~kCtasPerSm resident per SM, tiles long enough
// that the 2*steps halo rows stay a small overhead
// ---------------------------------------------------------------------------
struct Tuning {
  int tl_override = 0;
  int fwd_ctas_per_sm = 16;  // forward kernels (one-warp CTAs): one full wave
  int pdl = 0;               // march kernels launched with programmatic dependent launch
  int no_tma_store = 0;      // forward march: plain vector stores instead of staged TMA stores
  int debug_stall_us = 0;    // test hook of the forward march's timeout path (microseconds, 0 = off)
};
Tuning g_tuning;

// Arithmetic of the forward update with 16-bit I/O: process default (set by
// cta_set_arithmetic) and a per-thread override (cta_set_thread_arithmetic, -1
// = follow the process default).  fp32 I/O always uses the exact update.
std::atomic<int> g_arith{CTA_ARITH_CONTRACTED};
thread_local int t_arith = -1;

int contract_for(int dtype) {
  const int mode = t_arith >= 0 ? t_arith : g_arith.load(std::memory_order_relaxed);
  return (mode == CTA_ARITH_CONTRACTED && dtype != CTA_F32) ? 1 : 0;
}

// Tile rows of a march grid: the fewest full waves of `per_sm` CTAs per SM whose
// tiles fit kBldMaxTL, and tiles sized so that the grid fills those waves
// evenly (a grid a little over a whole number of waves would run one short
// extra wave, its duration set by a full tile).
int pick_tl(int64_t rows, int64_t parallel_ctas, int steps, int per_sm) {
  if (g_tuning.tl_override > 0) return std::min(kBldMaxTL, ((g_tuning.tl_override + kBldRC - 1) / kBldRC) * kBldRC);
  const int64_t target = static_cast<int64_t>(num_sms()) * per_sm;
  const int64_t work = rows * std::max<int64_t>(parallel_ctas, 1);  // tile rows over all column tiles
  const int64_t waves = std::max<int64_t>(1, (work + target * kBldMaxTL - 1) / (target * kBldMaxTL));
  int64_t tl = (work + waves * target - 1) / (waves * target);
  tl = ((tl + kBldRC - 1) / kBldRC) * kBldRC;
  const int64_t min_tl = steps >= 6 ? 64 : 32;
  tl = std::max(tl, min_tl);
  tl = std::min<int64_t>(tl, kBldMaxTL);
  return static_cast<int>(tl);
}

// target resident CTAs per SM of a march kernel: the tuning value, capped by
// the occupancy the variant gets (deep variants hold more registers)
int march_per_sm(int dtype, int steps, int causal, int adjoint, int residual = 0, int contract = 0) {
  const int occ = bld_march_ctas_per_sm(dtype, steps, causal, adjoint, residual, contract);
  return occ > 0 ? std::min(g_tuning.fwd_ctas_per_sm, occ) : g_tuning.fwd_ctas_per_sm;
}

void fill_alpha(BldArgs& a, int steps, const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype) {
  for (int k = 0; k < kMaxSteps; ++k) {
    a.alpha[k] = (alpha != nullptr && k < steps) ? alpha[k] : 0.f;
    a.alpha_dev[k] = (alpha_dev != nullptr && k < steps) ? alpha_dev[k] : nullptr;
  }
  a.alpha_dev_dtype = alpha_dev_dtype;
}

int check_alpha(int steps, const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype) {
  if (alpha == nullptr && alpha_dev == nullptr) return fail(CTA_EINVAL, "alpha: need host or device coefficients");
  if (alpha == nullptr) {
    for (int k = 0; k < steps; ++k)
      if (alpha_dev[k] == nullptr) return fail(CTA_EINVAL, "alpha_dev[%d] is NULL and no host alpha given", k);
  }
  if (alpha_dev != nullptr && !valid_dtype(alpha_dev_dtype))
    return fail(CTA_EINVAL, "alpha_dev_dtype %d is not a float dtype", alpha_dev_dtype);
  return CTA_OK;
}

int check_common(int dtype, int steps) {
  if (!valid_dtype(dtype)) return fail(CTA_EINVAL, "unsupported dtype code %d", dtype);
  if (steps < 1 || steps > kMaxSteps)
    return fail(CTA_EINVAL, "steps must be in 1..%d for a fused launch, got %d", kMaxSteps, steps);
  return CTA_OK;
}

BldArgs blank_bld() {
  BldArgs a;
  std::memset(&a, 0, sizeof(a));
  a.neg_zero = -0.0f;
  a.debug_stall_us = g_tuning.debug_stall_us;
  return a;
}

// rows of y allow aligned stores of v consecutive elements per lane
bool vec_ok(const void* y, int dtype, int64_t nb, int64_t D, int64_t sB, int64_t sL, int64_t v) {
  const int64_t es = static_cast<int64_t>(dtype_size(dtype));
  return reinterpret_cast<uintptr_t>(y) % (v * es) == 0 && D % v == 0 && sL % v == 0 && (nb == 1 || sB % v == 0);
}
bool quad_ok(const void* y, int dtype, int64_t nb, int64_t D, int64_t sB, int64_t sL) {
  return vec_ok(y, dtype, nb, D, sB, sL, kFwdVec);
}

int launch_fwd(BldArgs& a, int dtype, int steps, int causal, int64_t nbatch, int64_t tile_rows, cudaStream_t st,
               const CUtensorMap& xmap, const CUtensorMap& ymap, int adjoint = 0,
               const CUtensorMap* rmap = nullptr) {
  static const CUtensorMap kNoMap = {};
  const int64_t ntl = (tile_rows + a.TL - 1) / a.TL;
  const int64_t ndt = (a.D + kFwdDT - 1) / kFwdDT;
  if (ntl <= 0 || nbatch <= 0) return ok();
  if (ntl * ndt > 0x7fffffffLL || nbatch > 65535)
    return fail(CTA_EUNSUPPORTED, "grid too large (tiles %lld, D tiles %lld, batch %lld)", (long long)ntl,
                (long long)ndt, (long long)nbatch);
  // x = row tile * column tiles + column tile (column tile fastest)
  dim3 grid(static_cast<unsigned>(ntl * ndt), 1u, static_cast<unsigned>(nbatch));
  const cudaError_t e =
      launch_bld_fwd(a, &xmap, &ymap, rmap != nullptr ? rmap : &kNoMap, dtype, steps, causal, adjoint, grid,
                     fwd_smem_bytes(dtype), st);
  if (e != cudaSuccess) return cuda_fail(e, "bld forward launch");
  return ok();
}

// Grid, workspace layout, tensor maps and launch of the march d(alpha) kernel
// over output rows [m.out_begin, m.out_end) of m's streams (g, x -> y); `tiled`
// = TMA may address the three tensors (dense, whole-tensor rows).
int launch_dalpha_march(BldArgs& m, int dtype, int steps, int causal, int64_t B, int64_t L, int64_t D,
                        void* workspace, float* dalpha, bool accumulate, bool tiled, cudaStream_t st) {
  const int64_t ndt = (D + kDaDT - 1) / kDaDT;
  const int64_t rows = m.out_end - m.out_begin;
  if (rows <= 0) return ok();
  m.contract = m.pde_kind == 0 ? contract_for(dtype) : 0;
  const int occ = bld_dalpha_ctas_per_sm(dtype, steps, causal, m.contract);
  // one wave at the occupancy the variant gets (up to 24 one-warp CTAs per SM)
  m.TL = pick_tl(rows, ndt * B, steps, occ > 0 ? occ : 8);
  const int64_t ntl = (rows + m.TL - 1) / m.TL;
  if (ntl * ndt > 0x7fffffffLL || B > 65535 || ntl * ndt * B > 0x7fffffffLL)
    return fail(CTA_EUNSUPPORTED, "grid too large (tiles %lld, D tiles %lld, batch %lld)", (long long)ntl,
                (long long)ndt, (long long)B);
  m.num_ctas = static_cast<int>(ntl * ndt * B);
  m.dalpha_group = static_cast<int>(32 * ((m.num_ctas + 32LL * kWsMaxGroups - 1) / (32LL * kWsMaxGroups)));
  m.dalpha_accumulate = accumulate ? 1 : 0;
  m.counter = static_cast<unsigned int*>(workspace);
  m.dalpha_partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kWsHeaderBytes);
  m.dalpha = dalpha;
  m.y_quad_ok = vec_ok(m.y, dtype, B, D, m.ysB, m.ysL, 2 * kDaPairs) ? 1 : 0;
  CUtensorMap gm, xm, dm;
  std::memset(&gm, 0, sizeof(gm));
  std::memset(&xm, 0, sizeof(xm));
  std::memset(&dm, 0, sizeof(dm));
  const bool tg = tiled && make_map(&gm, m.g, dtype, B, L, D, m.gsB, m.gsL, kFwdRC, kDaDT);
  const bool tx = tiled && make_map(&xm, m.x, dtype, B, L, D, m.xsB, m.xsL, kFwdRC, kDaDT);
  m.use_tma = (tg && tx) ? 1 : 0;
  m.use_tma_store = make_map(&dm, m.y, dtype, B, L, D, m.ysB, m.ysL, kFwdRC, kDaDT) ? 1 : 0;
  dim3 grid(static_cast<unsigned>(ntl * ndt), 1u, static_cast<unsigned>(B));
  const cudaError_t e = launch_bld_dalpha(m, &gm, &xm, &dm, dtype, steps, causal, grid, st);
  if (e != cudaSuccess) return cuda_fail(e, "bld backward (d(alpha)) launch");
  return ok();
}

}  // namespace

namespace {

// The forward of `steps` advection- / reaction-diffusion layer steps (m.pde_kind,
// coefficients already in m) on the march kernel.
int pde_forward_launch(BldArgs& m, int dtype, int steps, int causal, int64_t B, int64_t L, int64_t D, int64_t y_sB,
                       int64_t y_sL, cudaStream_t st) {
  const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
  m.TL = pick_tl(L, ndt * B, steps, march_per_sm(dtype, steps, causal ? 1 : 0, 0));
  m.y_quad_ok = quad_ok(m.y, dtype, B, D, y_sB, y_sL) ? 1 : 0;
  CUtensorMap xmap, ymap;
  std::memset(&xmap, 0, sizeof(xmap));
  std::memset(&ymap, 0, sizeof(ymap));
  m.use_tma = make_map(&xmap, m.x, dtype, B, L, D, m.xsB, m.xsL, kFwdRC, kFwdDT) ? 1 : 0;
  m.use_tma_store = make_map(&ymap, m.y, dtype, B, L, D, y_sB, y_sL, kFwdRC, kFwdDT) ? 1 : 0;
  return launch_fwd(m, dtype, steps, causal ? 1 : 0, B, L, st, xmap, ymap);
}

}  // namespace

int cta::pdl_enabled() { return g_tuning.pdl; }

void cta::set_last_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

extern "C" {

int cta_abi_version(void) { return CTA_ABI_VERSION; }

const char* cta_last_error(void) { return t_last_error.c_str(); }

int cta_device_error(int clear) {
  const int a = read_device_error_bld_fwd(clear);
  const int c = read_device_error_bdl(clear);
  const int d = read_device_error_bld_dalpha(clear);
  if (a < 0 || c < 0 || d < 0) return -1;
  return a != 0 ? a : (c != 0 ? c : d);
}

int cta_set_arithmetic(int mode) {
  if (mode != CTA_ARITH_EXACT && mode != CTA_ARITH_CONTRACTED) return fail(-1, "unknown arithmetic mode %d", mode);
  return g_arith.exchange(mode);
}

int cta_set_thread_arithmetic(int mode) {
  if (mode != -1 && mode != CTA_ARITH_EXACT && mode != CTA_ARITH_CONTRACTED)
    return fail(-2, "unknown arithmetic mode %d", mode);
  const int prev = t_arith;
  t_arith = mode;
  return prev;
}

// Benchmark and test hook; the keys are listed with the declaration in
// include/cta_stencil.h.  Returns the previous value.
int cta_set_tuning(int key, int value) {
  int prev = 0;
  if (key == 1) {
    prev = g_tuning.tl_override;
    g_tuning.tl_override = value > 0 ? value : 0;
  } else if (key == 2) {
    prev = g_tuning.fwd_ctas_per_sm;
    g_tuning.fwd_ctas_per_sm = value > 0 ? value : 16;
  } else if (key == 3) {
    prev = g_tuning.pdl;
    g_tuning.pdl = value != 0 ? 1 : 0;
  } else if (key == 4) {
    prev = g_tuning.no_tma_store;
    g_tuning.no_tma_store = value != 0 ? 1 : 0;
  } else if (key == 5) {
    prev = g_tuning.debug_stall_us;
    g_tuning.debug_stall_us = value > 0 ? std::min(value, 100000) : 0;
  }
  return prev;
}

// ---------------------------------------------------------------------------
// [B, D, L]
// ---------------------------------------------------------------------------
int cta_diffusion_bdl_ex(const void* in, void* out, int64_t B, int64_t D, int64_t L, int64_t in_row_stride,
                         int64_t out_row_stride, int dtype, int steps, int causal, int backward, const float* alpha,
                         const void* const* alpha_dev, int alpha_dev_dtype, const void* mask, int mask_dtype,
                         int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  rc = check_alpha(steps, alpha, alpha_dev, alpha_dev_dtype);
  if (rc) return rc;
  if (B < 0 || D < 0 || L < 0) return fail(CTA_EINVAL, "negative shape");
  if (B == 0 || D == 0 || L == 0) return ok();
  if (in == nullptr || out == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (in_row_stride < L || out_row_stride < L) return fail(CTA_EINVAL, "row stride smaller than L");
  if (mask != nullptr && !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "bad mask dtype %d", mask_dtype);
  if (L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  BdlArgs a;
  std::memset(&a, 0, sizeof(a));
  a.neg_zero = -0.0f;
  a.in = in;
  a.out = out;
  a.rows = B * D;
  a.D = D;
  a.L = L;
  a.in_rs = in_row_stride;
  a.out_rs = out_row_stride;
  const size_t es = dtype_size(dtype);
  a.vec_ok = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
             ((in_row_stride * static_cast<int64_t>(es)) % 16 == 0) &&
             ((out_row_stride * static_cast<int64_t>(es)) % 16 == 0);
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  a.msB = mask_sB;
  a.msL = mask_sL;
  for (int k = 0; k < kMaxSteps; ++k) {
    a.alpha[k] = (alpha != nullptr && k < steps) ? alpha[k] : 0.f;
    a.alpha_dev[k] = (alpha_dev != nullptr && k < steps) ? alpha_dev[k] : nullptr;
  }
  a.alpha_dev_dtype = alpha_dev_dtype;
  a.contract = backward ? 0 : contract_for(dtype);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // TMA form when both tensors are addressable: [B*D rows, L] maps, boxes of two
  // rows x 256 positions (loads) and two rows x 240 positions (stores)
  CUtensorMap imap, omap;
  std::memset(&imap, 0, sizeof(imap));
  std::memset(&omap, 0, sizeof(omap));
  const int64_t rows = B * D;
  if (make_map(&imap, in, dtype, 1, rows, L, rows * in_row_stride, in_row_stride, kBdlRows, kBdlWin) &&
      make_map(&omap, out, dtype, 1, rows, L, rows * out_row_stride, out_row_stride, kBdlRows, kBdlOut)) {
    const int64_t nwin = (L + kBdlOut - 1) / kBdlOut;
    const int64_t pairs = (rows + kBdlRows - 1) / kBdlRows;
    const int occ = bdl_march_ctas_per_sm(dtype, steps, causal ? 1 : 0, backward ? 1 : 0, a.contract);
    const int per_sm = occ > 0 ? std::min(g_tuning.fwd_ctas_per_sm, occ) : g_tuning.fwd_ctas_per_sm;
    const int64_t target = static_cast<int64_t>(num_sms()) * per_sm;
    const int64_t tw = std::max<int64_t>(1, (pairs * nwin + target - 1) / target);
    const int64_t nseg = (nwin + tw - 1) / tw;
    if (pairs * nseg <= 0x7fffffffLL) {
      a.tw = static_cast<int>(tw);
      a.nseg = static_cast<int>(nseg);
      const cudaError_t e = launch_bdl_march(a, &imap, &omap, dtype, steps, causal ? 1 : 0, backward ? 1 : 0,
                                             static_cast<unsigned>(pairs * nseg), st);
      if (e != cudaSuccess) return cuda_fail(e, "bdl launch");
      return ok();
    }
  }
  const cudaError_t e = launch_bdl(a, dtype, steps, causal ? 1 : 0, backward ? 1 : 0, st);
  if (e != cudaSuccess) return cuda_fail(e, "bdl launch");
  return ok();
}

int cta_diffusion_fwd_bdl(const void* x, void* y, int64_t B, int64_t D, int64_t L, int64_t row_stride, int dtype,
                          int steps, float alpha, void* stream) {
  float al[kMaxSteps];
  for (int k = 0; k < kMaxSteps; ++k) al[k] = alpha;
  return cta_diffusion_bdl_ex(x, y, B, D, L, row_stride, row_stride, dtype, steps, 0, 0, al, nullptr, CTA_F32,
                              nullptr, 0, 0, 0, stream);
}

int cta_diffusion_bwd_bdl(const void* grad_out, void* grad_in, int64_t B, int64_t D, int64_t L, int64_t row_stride,
                          int dtype, int steps, float alpha, void* stream) {
  float al[kMaxSteps];
  for (int k = 0; k < kMaxSteps; ++k) al[k] = alpha;
  return cta_diffusion_bdl_ex(grad_out, grad_in, B, D, L, row_stride, row_stride, dtype, steps, 0, 1, al, nullptr,
                              CTA_F32, nullptr, 0, 0, 0, stream);
}

// ---------------------------------------------------------------------------
// [B, L, D]
// ---------------------------------------------------------------------------
static int fwd_bld_impl(const void* x, const void* residual, void* y, int64_t B, int64_t L, int64_t D, int64_t x_sB,
                        int64_t x_sL, int64_t r_sB, int64_t r_sL, int64_t y_sB, int64_t y_sL, int dtype, int steps,
                        int causal, const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype,
                        const void* mask, int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  rc = check_alpha(steps, alpha, alpha_dev, alpha_dev_dtype);
  if (rc) return rc;
  if (B < 0 || L < 0 || D < 0) return fail(CTA_EINVAL, "negative shape");
  if (B == 0 || L == 0 || D == 0) return ok();
  if (L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  if (x == nullptr || y == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (x_sL < D || y_sL < D) return fail(CTA_EINVAL, "row stride smaller than D");
  if (mask != nullptr && !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "bad mask dtype %d", mask_dtype);
  BldArgs a = blank_bld();
  a.x = x;
  a.y = y;
  a.xsB = x_sB;
  a.xsL = x_sL;
  a.ysB = y_sB;
  a.ysL = y_sL;
  a.L = L;
  a.D = static_cast<int>(D);
  a.nbatch = static_cast<int>(B);
  a.pos_offset = 0;
  a.global_len = L;
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  a.msB = mask_sB;
  a.msL = mask_sL;
  fill_alpha(a, steps, alpha, alpha_dev, alpha_dev_dtype);
  const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
  a.contract = contract_for(dtype);
  a.TL = pick_tl(L, ndt * B, steps,
                 march_per_sm(dtype, steps, causal ? 1 : 0, 0, residual != nullptr ? 1 : 0, a.contract));
  a.out_begin = 0;
  a.out_end = L;
  a.y_quad_ok = quad_ok(y, dtype, B, D, y_sB, y_sL) ? 1 : 0;
  CUtensorMap xmap, ymap;
  std::memset(&xmap, 0, sizeof(xmap));
  std::memset(&ymap, 0, sizeof(ymap));
  a.use_tma = make_map(&xmap, x, dtype, B, L, D, x_sB, x_sL, kFwdRC, kFwdDT) ? 1 : 0;
  a.use_tma_store = !g_tuning.no_tma_store && make_map(&ymap, y, dtype, B, L, D, y_sB, y_sL, kFwdRC, kFwdDT) ? 1 : 0;
  CUtensorMap rmap;
  std::memset(&rmap, 0, sizeof(rmap));
  if (residual != nullptr) {
    if (causal) return fail(CTA_EUNSUPPORTED, "the fused residual add is the non-causal forward");
    if (r_sL < D) return fail(CTA_EINVAL, "residual row stride smaller than D");
    a.residual = residual;
    a.rsB = r_sB;
    a.rsL = r_sL;
    if (!quad_ok(residual, dtype, B, D, r_sB, r_sL)) a.y_quad_ok = 0;
    // full chunks take the residual through the staging buffer: it needs a map
    if (!make_map(&rmap, residual, dtype, B, L, D, r_sB, r_sL, kFwdRC, kFwdDT)) a.use_tma_store = 0;
  }
  return launch_fwd(a, dtype, steps, causal ? 1 : 0, B, L, static_cast<cudaStream_t>(stream), xmap, ymap, 0, &rmap);
}

int cta_diffusion_fwd_bld(const void* x, void* y, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                          int64_t y_sB, int64_t y_sL, int dtype, int steps, int causal, const float* alpha,
                          const void* const* alpha_dev, int alpha_dev_dtype, const void* mask, int mask_dtype,
                          int64_t mask_sB, int64_t mask_sL, void* stream) {
  return fwd_bld_impl(x, nullptr, y, B, L, D, x_sB, x_sL, 0, 0, y_sB, y_sL, dtype, steps, causal, alpha, alpha_dev,
                      alpha_dev_dtype, mask, mask_dtype, mask_sB, mask_sL, stream);
}

int64_t cta_diffusion_fwd_bld_pool_workspace_bytes(int64_t B, int64_t L, int64_t D) {
  if (B <= 0 || L <= 0 || D <= 0) return 256;
  // per row tile (at least 32 rows): D column sums and one valid-row count
  return std::max<int64_t>(256, ((L + 31) / 32) * B * (D + 1) * static_cast<int64_t>(sizeof(float)));
}

int cta_diffusion_fwd_bld_pool(const void* x, void* pooled, void* workspace, int64_t workspace_bytes, int64_t B,
                               int64_t L, int64_t D, int64_t x_sB, int64_t x_sL, int dtype, int steps,
                               const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype,
                               const void* mask, int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  rc = check_alpha(steps, alpha, alpha_dev, alpha_dev_dtype);
  if (rc) return rc;
  if (B < 0 || L < 0 || D < 0) return fail(CTA_EINVAL, "negative shape");
  if (B == 0 || D == 0) return ok();
  if (L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  if (B > 65535) return fail(CTA_EUNSUPPORTED, "at most 65535 batch rows");
  if (x == nullptr || pooled == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (x_sL < D) return fail(CTA_EINVAL, "row stride smaller than D");
  if (mask == nullptr || !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "the masked pool needs a mask");
  if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
    return fail(CTA_EINVAL, "the masked pool needs a 16-byte aligned workspace");
  const int64_t need = cta_diffusion_fwd_bld_pool_workspace_bytes(B, L, D);
  if (workspace_bytes < need)
    return fail(CTA_EINVAL, "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
  BldArgs a = blank_bld();
  a.x = x;
  a.y = workspace;  // never written: the pooled form stores no rows
  a.xsB = x_sB;
  a.xsL = x_sL;
  a.L = L;
  a.D = static_cast<int>(D);
  a.nbatch = static_cast<int>(B);
  a.global_len = L;
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  a.msB = mask_sB;
  a.msL = mask_sL;
  a.pool_partial = static_cast<float*>(workspace);
  fill_alpha(a, steps, alpha, alpha_dev, alpha_dev_dtype);
  const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
  a.TL = pick_tl(L, ndt * B, steps, march_per_sm(dtype, steps, 0, 0));
  // a row-tile override below 32 rows needs more partials than the size query reports
  const int64_t ntl = (L + a.TL - 1) / a.TL;
  if (ntl * B * (D + 1) * static_cast<int64_t>(sizeof(float)) > workspace_bytes)
    return fail(CTA_EINVAL, "workspace too small for %lld row tiles", (long long)ntl);
  a.out_begin = 0;
  a.out_end = L;
  CUtensorMap xmap, ymap;
  std::memset(&xmap, 0, sizeof(xmap));
  std::memset(&ymap, 0, sizeof(ymap));
  a.use_tma = make_map(&xmap, x, dtype, B, L, D, x_sB, x_sL, kFwdRC, kFwdDT) ? 1 : 0;
  a.use_tma_store = 0;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = launch_fwd(a, dtype, steps, 0, B, L, st, xmap, ymap);
  if (rc) return rc;
  const cudaError_t e = launch_pool_finish(a, dtype, ntl, pooled, st);
  if (e != cudaSuccess) return cuda_fail(e, "masked pool reduction launch");
  return ok();
}

int cta_diffusion_fwd_bld_residual(const void* x, const void* residual, void* y, int64_t B, int64_t L, int64_t D,
                                   int64_t x_sB, int64_t x_sL, int64_t r_sB, int64_t r_sL, int64_t y_sB,
                                   int64_t y_sL, int dtype, int steps, const float* alpha, const void* mask,
                                   int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  if (residual == nullptr) return fail(CTA_EINVAL, "null residual pointer");
  return fwd_bld_impl(x, residual, y, B, L, D, x_sB, x_sL, r_sB, r_sL, y_sB, y_sL, dtype, steps, 0, alpha, nullptr,
                      0, mask, mask_dtype, mask_sB, mask_sL, stream);
}

int64_t cta_diffusion_bwd_bld_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype, int steps, int causal) {
  (void)dtype;
  (void)causal;
  if (B <= 0 || L <= 0 || D <= 0 || steps < 1 || steps > kMaxSteps) return kWsHeaderBytes;
  if (steps <= kDaMaxSteps) {
    // march kernel: partials of up to ceil(L/32) x ceil(D/kDaDT) x B CTAs, then the
    // group sums (f64, 8-byte aligned)
    const int64_t ctas = ((L + 31) / 32) * ((D + kDaDT - 1) / kDaDT) * B;
    const int64_t ngroups = std::min<int64_t>(kWsMaxGroups, (ctas + 31) / 32);
    return kWsHeaderBytes + ctas * steps * 4 + 4 + ngroups * steps * 8;
  }
  return kWsHeaderBytes;
}

int cta_diffusion_bwd_bld(const void* grad_out, void* grad_in, const void* x, float* dalpha, void* workspace,
                          int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t g_sB, int64_t g_sL,
                          int64_t x_sB, int64_t x_sL, int64_t d_sB, int64_t d_sL, int dtype, int steps, int causal,
                          const float* alpha, const void* const* alpha_dev, int alpha_dev_dtype, const void* mask,
                          int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  rc = check_alpha(steps, alpha, alpha_dev, alpha_dev_dtype);
  if (rc) return rc;
  if (B < 0 || L < 0 || D < 0) return fail(CTA_EINVAL, "negative shape");
  if (L > 0 && L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  if (grad_out == nullptr || grad_in == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (g_sL < D || d_sL < D) return fail(CTA_EINVAL, "row stride smaller than D");
  if (mask != nullptr && !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "bad mask dtype %d", mask_dtype);
  const bool da = dalpha != nullptr;
  if (da) {
    if (x == nullptr) return fail(CTA_EINVAL, "dalpha requested without the forward input x");
    if (x_sL < D) return fail(CTA_EINVAL, "x row stride smaller than D");
    if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
      return fail(CTA_EINVAL, "dalpha needs a 256-byte aligned workspace");
    if (workspace_bytes < cta_diffusion_bwd_bld_workspace_bytes(B, L, D, dtype, steps, causal))
      return fail(CTA_EINVAL, "workspace too small: %lld < %lld bytes", (long long)workspace_bytes,
                  (long long)cta_diffusion_bwd_bld_workspace_bytes(B, L, D, dtype, steps, causal));
  }
  if (B == 0 || L == 0 || D == 0) {
    if (da) {
      const cudaError_t e = cudaMemsetAsync(dalpha, 0, sizeof(float) * steps, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "dalpha clear");
    }
    return ok();
  }
  if (!da) {
    // adjoint only: the one-warp TMA march kernel (same pipeline as the forward)
    BldArgs m = blank_bld();
    m.x = grad_out;
    m.y = grad_in;
    m.xsB = g_sB;
    m.xsL = g_sL;
    m.ysB = d_sB;
    m.ysL = d_sL;
    m.L = L;
    m.D = static_cast<int>(D);
    m.nbatch = static_cast<int>(B);
    m.global_len = L;
    m.mask = mask;
    m.mask_dtype = mask_dtype;
    m.msB = mask_sB;
    m.msL = mask_sL;
    fill_alpha(m, steps, alpha, alpha_dev, alpha_dev_dtype);
    m.contract = contract_for(dtype);
    const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
    m.TL = pick_tl(L, ndt * B, steps, march_per_sm(dtype, steps, causal ? 1 : 0, 1, 0, m.contract));
    m.out_begin = 0;
    m.out_end = L;
    m.y_quad_ok = quad_ok(grad_in, dtype, B, D, d_sB, d_sL) ? 1 : 0;
    CUtensorMap gm, dm;
    std::memset(&gm, 0, sizeof(gm));
    std::memset(&dm, 0, sizeof(dm));
    m.use_tma = make_map(&gm, grad_out, dtype, B, L, D, g_sB, g_sL, kFwdRC, kFwdDT) ? 1 : 0;
    m.use_tma_store = make_map(&dm, grad_in, dtype, B, L, D, d_sB, d_sL, kFwdRC, kFwdDT) ? 1 : 0;
    return launch_fwd(m, dtype, steps, causal ? 1 : 0, B, L, static_cast<cudaStream_t>(stream), gm, dm, 1);
  }
  // d(alpha), steps 1..8: the one-warp march carrying both wavefronts
  BldArgs m = blank_bld();
  m.g = grad_out;
  m.x = x;
  m.y = grad_in;
  m.gsB = g_sB;
  m.gsL = g_sL;
  m.xsB = x_sB;
  m.xsL = x_sL;
  m.ysB = d_sB;
  m.ysL = d_sL;
  m.L = L;
  m.D = static_cast<int>(D);
  m.nbatch = static_cast<int>(B);
  m.global_len = L;
  m.mask = mask;
  m.mask_dtype = mask_dtype;
  m.msB = mask_sB;
  m.msL = mask_sL;
  fill_alpha(m, steps, alpha, alpha_dev, alpha_dev_dtype);
  m.out_begin = 0;
  m.out_end = L;
  return launch_dalpha_march(m, dtype, steps, causal ? 1 : 0, B, L, D, workspace, dalpha, false, true,
                             static_cast<cudaStream_t>(stream));
}

static int fwd_varlen_impl(const void* x, const void* residual, void* y, int64_t total_rows, int64_t D,
                           int64_t x_sL, int64_t r_sL, int64_t y_sL, const int32_t* cu_seqlens, int64_t nseq,
                           int64_t max_len, int pad_to_max, int dtype, int steps, float alpha, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  if (total_rows < 0 || D < 0 || nseq < 0 || max_len < 0) return fail(CTA_EINVAL, "negative shape");
  if (total_rows == 0 || D == 0 || nseq == 0 || max_len == 0) return ok();
  if (x == nullptr || y == nullptr || cu_seqlens == nullptr) return fail(CTA_EINVAL, "null pointer");
  if (x_sL < D || y_sL < D) return fail(CTA_EINVAL, "row stride smaller than D");
  if (nseq > 65535) return fail(CTA_EUNSUPPORTED, "at most 65535 sequences per call, got %lld", (long long)nseq);
  BldArgs a = blank_bld();
  a.x = x;
  a.y = y;
  a.xsL = x_sL;
  a.ysL = y_sL;
  a.xsB = 0;
  a.ysB = 0;
  a.L = total_rows;
  a.D = static_cast<int>(D);
  a.nbatch = static_cast<int>(nseq);
  a.cu_seqlens = cu_seqlens;
  a.pad_to_max = pad_to_max ? 1 : 0;
  a.max_len = max_len;
  for (int k = 0; k < kMaxSteps; ++k) a.alpha[k] = alpha;
  a.contract = contract_for(dtype);
  const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
  // tiles are cut per sequence: about eight tiles per average sequence keeps
  // the waves balanced across unequal lengths (halo overhead 2*steps/TL)
  const int64_t avg = std::max<int64_t>(1, total_rows / nseq);
  a.TL = g_tuning.tl_override > 0
             ? pick_tl(avg, ndt * nseq, steps,
                       march_per_sm(dtype, steps, 0, 0, residual != nullptr ? 1 : 0, a.contract))
             : static_cast<int>(std::min<int64_t>(512, std::max<int64_t>(64, ((avg / 8 + 15) / 16) * 16)));
  a.out_begin = 0;
  a.out_end = max_len;
  a.y_quad_ok = quad_ok(y, dtype, 1, D, 0, y_sL) ? 1 : 0;
  CUtensorMap xmap, ymap;
  std::memset(&xmap, 0, sizeof(xmap));
  std::memset(&ymap, 0, sizeof(ymap));
  a.use_tma = make_map(&xmap, x, dtype, 1, total_rows, D, 0, x_sL, kFwdRC, kFwdDT) ? 1 : 0;
  a.use_tma_store = make_map(&ymap, y, dtype, 1, total_rows, D, 0, y_sL, kFwdRC, kFwdDT) ? 1 : 0;
  CUtensorMap rmap;
  std::memset(&rmap, 0, sizeof(rmap));
  if (residual != nullptr) {
    if (r_sL < D) return fail(CTA_EINVAL, "residual row stride smaller than D");
    a.residual = residual;
    a.rsB = 0;
    a.rsL = r_sL;
    if (!quad_ok(residual, dtype, 1, D, 0, r_sL)) a.y_quad_ok = 0;
    if (!make_map(&rmap, residual, dtype, 1, total_rows, D, 0, r_sL, kFwdRC, kFwdDT)) a.use_tma_store = 0;
  }
  return launch_fwd(a, dtype, steps, 0, nseq, max_len, static_cast<cudaStream_t>(stream), xmap, ymap, 0, &rmap);
}

int cta_diffusion_fwd_varlen(const void* x, void* y, int64_t total_rows, int64_t D, int64_t x_sL, int64_t y_sL,
                             const int32_t* cu_seqlens, int64_t nseq, int64_t max_len, int pad_to_max, int dtype,
                             int steps, float alpha, void* stream) {
  return fwd_varlen_impl(x, nullptr, y, total_rows, D, x_sL, 0, y_sL, cu_seqlens, nseq, max_len, pad_to_max, dtype,
                         steps, alpha, stream);
}

int cta_diffusion_fwd_varlen_residual(const void* x, const void* residual, void* y, int64_t total_rows, int64_t D,
                                      int64_t x_sL, int64_t r_sL, int64_t y_sL, const int32_t* cu_seqlens,
                                      int64_t nseq, int64_t max_len, int pad_to_max, int dtype, int steps,
                                      float alpha, void* stream) {
  if (residual == nullptr) return fail(CTA_EINVAL, "null residual pointer");
  return fwd_varlen_impl(x, residual, y, total_rows, D, x_sL, r_sL, y_sL, cu_seqlens, nseq, max_len, pad_to_max,
                         dtype, steps, alpha, stream);
}

int cta_diffusion_shard_bld(const void* in, void* out, int64_t B, int64_t L_local, int64_t D, int64_t pos_offset,
                            int64_t global_len, const void* lo_halo, int64_t lo_rows, const void* hi_halo,
                            int64_t hi_rows, int part, int dtype, int steps, int causal, int backward, float alpha,
                            void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  if (B < 0 || L_local < 0 || D < 0 || pos_offset < 0) return fail(CTA_EINVAL, "negative shape");
  if (B == 0 || L_local == 0 || D == 0) return ok();
  if (in == nullptr || out == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (pos_offset + L_local > global_len) return fail(CTA_EINVAL, "shard exceeds the global sequence");
  if (global_len < 3) return fail(CTA_EINVAL, "global length < 3 is the identity; handled by the caller");
  const int hl = causal ? (backward ? 0 : 2 * steps) : steps;
  const int hr = causal ? (backward ? 2 * steps : 0) : steps;
  const bool has_lo = pos_offset > 0;
  const bool has_hi = pos_offset + L_local < global_len;
  const int64_t ib = has_lo ? std::min<int64_t>(hl, L_local) : 0;
  const int64_t ie = has_hi ? std::max<int64_t>(L_local - hr, ib) : L_local;
  int64_t ob = 0, oe = 0;
  if (part == CTA_SHARD_INTERIOR) {
    ob = ib;
    oe = ie;
  } else if (part == CTA_SHARD_LO_EDGE) {
    ob = 0;
    oe = ib;
  } else if (part == CTA_SHARD_HI_EDGE) {
    ob = ie;
    oe = L_local;
  } else {
    return fail(CTA_EINVAL, "bad shard part %d", part);
  }
  if (oe <= ob) return ok();
  const bool edge = part != CTA_SHARD_INTERIOR;
  if (edge) {
    // an edge tile may reach past both shard ends when the shard is short: both halos must be present
    if (has_lo && hl > 0 && (lo_halo == nullptr || lo_rows < hl))
      return fail(CTA_EINVAL, "lo halo missing or shorter than %d rows", hl);
    if (has_hi && hr > 0 && (hi_halo == nullptr || hi_rows < hr))
      return fail(CTA_EINVAL, "hi halo missing or shorter than %d rows", hr);
    if (lo_rows < 0 || hi_rows < 0 || lo_rows > (1 << 20) || hi_rows > (1 << 20))
      return fail(CTA_EINVAL, "bad halo row counts");
  }
  BldArgs a = blank_bld();
  a.x = in;  // the march kernel's input stream (x forward, the gradient for the adjoint)
  a.y = out;
  a.xsB = a.gsB = a.ysB = L_local * D;
  a.xsL = a.gsL = a.ysL = D;
  a.L = L_local;
  a.D = static_cast<int>(D);
  a.nbatch = static_cast<int>(B);
  a.pos_offset = pos_offset;
  a.global_len = global_len;
  if (edge) {
    a.lo_ext = has_lo ? lo_halo : nullptr;
    a.hi_ext = has_hi ? hi_halo : nullptr;
    a.hext_lo = a.lo_ext ? static_cast<int>(lo_rows) : 0;
    a.hext_hi = a.hi_ext ? static_cast<int>(hi_rows) : 0;
  }
  for (int k = 0; k < kMaxSteps; ++k) a.alpha[k] = alpha;
  a.contract = contract_for(dtype);
  const int64_t ndt = (D + kFwdDT - 1) / kFwdDT;
  a.TL = edge ? static_cast<int>(std::min<int64_t>(kBldMaxTL, ((oe - ob + kBldRC - 1) / kBldRC) * kBldRC))
              : pick_tl(oe - ob, ndt * B, steps,
                        march_per_sm(dtype, steps, causal ? 1 : 0, backward ? 1 : 0, 0, a.contract));
  a.out_begin = ob;
  a.out_end = oe;
  a.y_quad_ok = quad_ok(out, dtype, B, D, L_local * D, D) ? 1 : 0;
  CUtensorMap map, omap;
  std::memset(&map, 0, sizeof(map));
  std::memset(&omap, 0, sizeof(omap));
  a.use_tma = (!edge && make_map(&map, in, dtype, B, L_local, D, L_local * D, D, kFwdRC, kFwdDT)) ? 1 : 0;
  a.use_tma_store = make_map(&omap, out, dtype, B, L_local, D, L_local * D, D, kFwdRC, kFwdDT) ? 1 : 0;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_fwd(a, dtype, steps, causal ? 1 : 0, B, oe - ob, st, map, omap, backward ? 1 : 0);
}

int64_t cta_pde_step_workspace_bytes(int64_t B, int64_t L, int64_t D) {
  // the d(alpha) march layout with two reduced values (d(alpha), d(beta))
  return cta_diffusion_bwd_bld_workspace_bytes(B, L, D, CTA_F32, 2, 0);
}

int cta_pde_step_bld(const void* x, const void* grad_out, void* y, float* dcoef, void* workspace,
                     int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                     int64_t g_sB, int64_t g_sL, int64_t y_sB, int64_t y_sL, int dtype, int kind, int causal,
                     int backward, const void* alpha_dev, const void* beta_dev, int coef_dtype, const void* mask,
                     int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, 1);
  if (rc) return rc;
  if (kind != CTA_PDE_ADVECTION && kind != CTA_PDE_REACTION) return fail(CTA_EINVAL, "bad PDE kind %d", kind);
  if (alpha_dev == nullptr || beta_dev == nullptr) return fail(CTA_EINVAL, "alpha / beta device scalars missing");
  if (coef_dtype != CTA_F32 && coef_dtype != CTA_BF16 && coef_dtype != CTA_F16)
    return fail(CTA_EINVAL, "bad coefficient dtype %d", coef_dtype);
  if (B < 0 || L < 0 || D < 0) return fail(CTA_EINVAL, "negative shape");
  if (B > 65535) return fail(CTA_EUNSUPPORTED, "at most 65535 batch rows");
  if (L > 0 && L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  if (x == nullptr || y == nullptr || (backward && grad_out == nullptr))
    return fail(CTA_EINVAL, "null tensor pointer");
  if (x_sL < D || y_sL < D || (backward && g_sL < D)) return fail(CTA_EINVAL, "row stride smaller than D");
  if (mask != nullptr && !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "bad mask dtype %d", mask_dtype);
  if (backward) {
    if (dcoef == nullptr) return fail(CTA_EINVAL, "backward needs dcoef (fp32 [2])");
    if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
      return fail(CTA_EINVAL, "backward needs a 256-byte aligned workspace");
    const int64_t need = cta_pde_step_workspace_bytes(B, L, D);
    if (workspace_bytes < need)
      return fail(CTA_EINVAL, "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
  }
  if (B == 0 || L == 0 || D == 0) {
    if (backward) {
      const cudaError_t e = cudaMemsetAsync(dcoef, 0, 2 * sizeof(float), static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "dcoef clear");
    }
    return ok();
  }
  // both directions run on the one-warp TMA march kernels at steps 1 with the
  // layer's update: the forward march, and the d(alpha) march (backward, which
  // also reduces d(beta))
  BldArgs m = blank_bld();
  m.x = x;
  m.y = y;
  m.xsB = x_sB;
  m.xsL = x_sL;
  m.ysB = y_sB;
  m.ysL = y_sL;
  m.L = L;
  m.D = static_cast<int>(D);
  m.nbatch = static_cast<int>(B);
  m.global_len = L;
  m.mask = mask;
  m.mask_dtype = mask_dtype;
  m.msB = mask_sB;
  m.msL = mask_sL;
  m.alpha_dev[0] = alpha_dev;
  m.alpha_dev[1] = beta_dev;
  m.alpha_dev_dtype = coef_dtype;
  m.pde_kind = kind == CTA_PDE_ADVECTION ? 1 : 2;
  m.out_begin = 0;
  m.out_end = L;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (backward) {
    m.g = grad_out;
    m.gsB = g_sB;
    m.gsL = g_sL;
    return launch_dalpha_march(m, dtype, 1, causal ? 1 : 0, B, L, D, workspace, dcoef, false, true, st);
  }
  m.beta_dev[0] = beta_dev;
  return pde_forward_launch(m, dtype, 1, causal, B, L, D, y_sB, y_sL, st);
}

int cta_pde_stack_bld(const void* x, void* y, int64_t B, int64_t L, int64_t D, int64_t x_sB, int64_t x_sL,
                      int64_t y_sB, int64_t y_sL, int dtype, int kind, int steps, int causal,
                      const void* const* alpha_dev, const void* const* beta_dev, int coef_dtype, const void* mask,
                      int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  if (steps > kPdeMaxSteps)
    return fail(CTA_EINVAL, "a fused advection / reaction stack takes at most %d steps, got %d", kPdeMaxSteps, steps);
  if (kind != CTA_PDE_ADVECTION && kind != CTA_PDE_REACTION) return fail(CTA_EINVAL, "bad PDE kind %d", kind);
  if (alpha_dev == nullptr || beta_dev == nullptr) return fail(CTA_EINVAL, "alpha / beta device scalars missing");
  for (int k = 0; k < steps; ++k)
    if (alpha_dev[k] == nullptr || beta_dev[k] == nullptr)
      return fail(CTA_EINVAL, "alpha_dev[%d] / beta_dev[%d] is NULL", k, k);
  if (coef_dtype != CTA_F32 && coef_dtype != CTA_BF16 && coef_dtype != CTA_F16)
    return fail(CTA_EINVAL, "bad coefficient dtype %d", coef_dtype);
  if (B < 0 || L < 0 || D < 0) return fail(CTA_EINVAL, "negative shape");
  if (B > 65535) return fail(CTA_EUNSUPPORTED, "at most 65535 batch rows");
  if (L > 0 && L < 3) return fail(CTA_EINVAL, "L < 3 is the identity; handled by the caller");
  if (x == nullptr || y == nullptr) return fail(CTA_EINVAL, "null tensor pointer");
  if (x_sL < D || y_sL < D) return fail(CTA_EINVAL, "row stride smaller than D");
  if (mask != nullptr && !valid_mask_dtype(mask_dtype)) return fail(CTA_EINVAL, "bad mask dtype %d", mask_dtype);
  if (B == 0 || L == 0 || D == 0) return ok();
  BldArgs m = blank_bld();
  m.x = x;
  m.y = y;
  m.xsB = x_sB;
  m.xsL = x_sL;
  m.ysB = y_sB;
  m.ysL = y_sL;
  m.L = L;
  m.D = static_cast<int>(D);
  m.nbatch = static_cast<int>(B);
  m.global_len = L;
  m.mask = mask;
  m.mask_dtype = mask_dtype;
  m.msB = mask_sB;
  m.msL = mask_sL;
  for (int k = 0; k < steps; ++k) {
    m.alpha_dev[k] = alpha_dev[k];
    m.beta_dev[k] = beta_dev[k];
  }
  m.alpha_dev_dtype = coef_dtype;
  m.pde_kind = kind == CTA_PDE_ADVECTION ? 1 : 2;
  m.out_begin = 0;
  m.out_end = L;
  return pde_forward_launch(m, dtype, steps, causal, B, L, D, y_sB, y_sL, static_cast<cudaStream_t>(stream));
}

int cta_diffusion_shard_bld_dalpha(const void* grad_out, const void* x, void* grad_in, float* dalpha,
                                   void* workspace, int64_t workspace_bytes, int64_t B, int64_t L_local, int64_t D,
                                   int64_t pos_offset, int64_t global_len, const void* g_lo_halo, int64_t g_lo_rows,
                                   const void* g_hi_halo, int64_t g_hi_rows, const void* x_lo_halo,
                                   int64_t x_lo_rows, const void* x_hi_halo, int64_t x_hi_rows, int part, int dtype,
                                   int steps, int causal, const float* alpha, void* stream) {
  int rc = check_common(dtype, steps);
  if (rc) return rc;
  if (steps > kDaMaxSteps)
    return fail(CTA_EUNSUPPORTED, "sharded d(alpha) supports steps 1..%d, got %d", kDaMaxSteps, steps);
  if (alpha == nullptr) return fail(CTA_EINVAL, "alpha: need host coefficients");
  if (B < 0 || L_local < 0 || D < 0 || pos_offset < 0) return fail(CTA_EINVAL, "negative shape");
  if (B == 0 || L_local == 0 || D == 0) return ok();
  if (grad_out == nullptr || x == nullptr || grad_in == nullptr || dalpha == nullptr)
    return fail(CTA_EINVAL, "null tensor pointer");
  if (pos_offset + L_local > global_len) return fail(CTA_EINVAL, "shard exceeds the global sequence");
  if (global_len < 3) return fail(CTA_EINVAL, "global length < 3 is the identity; handled by the caller");
  if (workspace == nullptr || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(CTA_EINVAL, "dalpha needs a 256-byte aligned workspace");
  const int64_t need = cta_diffusion_bwd_bld_workspace_bytes(B, L_local, D, dtype, steps, causal);
  if (workspace_bytes < need)
    return fail(CTA_EINVAL, "workspace too small: %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
  // rows each stream needs beyond an output row: g below (and above when
  // non-causal), x above (and below when non-causal)
  const int glo = causal ? 0 : steps, ghi = causal ? 2 * steps : steps;
  const int xlo = causal ? 2 * steps : steps, xhi = causal ? 0 : steps;
  const int hl = std::max(glo, xlo), hr = std::max(ghi, xhi);
  const bool has_lo = pos_offset > 0;
  const bool has_hi = pos_offset + L_local < global_len;
  const int64_t ib = has_lo ? std::min<int64_t>(hl, L_local) : 0;
  const int64_t ie = has_hi ? std::max<int64_t>(L_local - hr, ib) : L_local;
  int64_t ob = 0, oe = 0;
  if (part == CTA_SHARD_INTERIOR) {
    ob = ib;
    oe = ie;
  } else if (part == CTA_SHARD_LO_EDGE) {
    ob = 0;
    oe = ib;
  } else if (part == CTA_SHARD_HI_EDGE) {
    ob = ie;
    oe = L_local;
  } else {
    return fail(CTA_EINVAL, "bad shard part %d", part);
  }
  if (oe <= ob) return ok();
  const bool edge = part != CTA_SHARD_INTERIOR;
  if (edge) {
    if (has_lo && ((glo > 0 && (g_lo_halo == nullptr || g_lo_rows < glo)) ||
                   (xlo > 0 && (x_lo_halo == nullptr || x_lo_rows < xlo))))
      return fail(CTA_EINVAL, "lo halos missing or shorter than %d (g) / %d (x) rows", glo, xlo);
    if (has_hi && ((ghi > 0 && (g_hi_halo == nullptr || g_hi_rows < ghi)) ||
                   (xhi > 0 && (x_hi_halo == nullptr || x_hi_rows < xhi))))
      return fail(CTA_EINVAL, "hi halos missing or shorter than %d (g) / %d (x) rows", ghi, xhi);
    for (int64_t r : {g_lo_rows, g_hi_rows, x_lo_rows, x_hi_rows})
      if (r < 0 || r > (1 << 20)) return fail(CTA_EINVAL, "bad halo row counts");
  }
  BldArgs m = blank_bld();
  m.g = grad_out;
  m.x = x;
  m.y = grad_in;
  m.gsB = m.xsB = m.ysB = L_local * D;
  m.gsL = m.xsL = m.ysL = D;
  m.L = L_local;
  m.D = static_cast<int>(D);
  m.nbatch = static_cast<int>(B);
  m.pos_offset = pos_offset;
  m.global_len = global_len;
  if (edge) {
    m.g_lo_ext = (has_lo && g_lo_rows > 0) ? g_lo_halo : nullptr;
    m.g_hi_ext = (has_hi && g_hi_rows > 0) ? g_hi_halo : nullptr;
    m.g_hext_lo = m.g_lo_ext ? static_cast<int>(g_lo_rows) : 0;
    m.g_hext_hi = m.g_hi_ext ? static_cast<int>(g_hi_rows) : 0;
    m.lo_ext = (has_lo && x_lo_rows > 0) ? x_lo_halo : nullptr;
    m.hi_ext = (has_hi && x_hi_rows > 0) ? x_hi_halo : nullptr;
    m.hext_lo = m.lo_ext ? static_cast<int>(x_lo_rows) : 0;
    m.hext_hi = m.hi_ext ? static_cast<int>(x_hi_rows) : 0;
  }
  fill_alpha(m, steps, alpha, nullptr, 0);
  m.out_begin = ob;
  m.out_end = oe;
  return launch_dalpha_march(m, dtype, steps, causal ? 1 : 0, B, L_local, D, workspace, dalpha, true, !edge,
                             static_cast<cudaStream_t>(stream));
}

}  // extern "C"
