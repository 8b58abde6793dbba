// Host side of the [B, L, D] forward / adjoint march (bld_fwd_kernel.cuh):
// kernel selection across the per-dtype units, launches, occupancy and the
// device error words.
#include "bld_common.cuh"

namespace cta {

// bld_fwd_<dtype>[_fm].cu
const void* bld_fwd_kernel_f32(int steps, int causal, int adj, int res, int kind, int pool);
const void* bld_fwd_kernel_bf16(int steps, int causal, int adj, int res, int kind, int pool);
const void* bld_fwd_kernel_bf16_fm(int steps, int causal, int adj, int res, int kind, int pool);
const void* bld_fwd_kernel_f16(int steps, int causal, int adj, int res, int kind, int pool);
const void* bld_fwd_kernel_f16_fm(int steps, int causal, int adj, int res, int kind, int pool);
const void* bld_pool_finish_f32();
const void* bld_pool_finish_bf16();
const void* bld_pool_finish_f16();
int read_device_error_bld_fwd_f32(int clear);
int read_device_error_bld_fwd_bf16(int clear);
int read_device_error_bld_fwd_bf16_fm(int clear);
int read_device_error_bld_fwd_f16(int clear);
int read_device_error_bld_fwd_f16_fm(int clear);

size_t fwd_smem_bytes(int dtype) {
  const size_t es = dtype == kF32 ? 4 : 2;
  return static_cast<size_t>(kFwdStages + kFwdOutSlots) * kFwdRC * kFwdDT * es;
}

namespace {

// fm: the contracted arithmetic, built for 16-bit tensors only
const void* march_kernel(int dtype, int steps, int causal, int adj, int res, int kind = 0, int pool = 0, int fm = 0) {
  switch (dtype) {
    case kF32: return fm ? nullptr : bld_fwd_kernel_f32(steps, causal, adj, res, kind, pool);
    case kBF16:
      return fm ? bld_fwd_kernel_bf16_fm(steps, causal, adj, res, kind, pool)
                : bld_fwd_kernel_bf16(steps, causal, adj, res, kind, pool);
    case kF16:
      return fm ? bld_fwd_kernel_f16_fm(steps, causal, adj, res, kind, pool)
                : bld_fwd_kernel_f16(steps, causal, adj, res, kind, pool);
    default: return nullptr;
  }
}

}  // namespace

cudaError_t launch_bld_fwd(const BldArgs& a, const CUtensorMap* xmap, const CUtensorMap* ymap,
                           const CUtensorMap* rmap, int dtype, int steps, int causal, int adjoint, dim3 grid,
                           size_t smem, cudaStream_t st) {
  const void* kern = march_kernel(dtype, steps, causal, adjoint, a.residual != nullptr ? 1 : 0, a.pde_kind,
                                  a.pool_partial != nullptr ? 1 : 0, a.contract);
  if (kern == nullptr) return cudaErrorInvalidValue;
  cudaError_t e = ensure_smem_attr(kern, smem);
  if (e != cudaSuccess) return e;
  BldArgs la = a;
  if (kFwdOutSlots == 0) la.use_tma_store = 0;  // no staging slots: plain stores
  void* args[] = {const_cast<CUtensorMap*>(xmap), const_cast<CUtensorMap*>(ymap), const_cast<CUtensorMap*>(rmap),
                  &la};
  if (!pdl_enabled()) return cudaLaunchKernel(kern, grid, dim3(kFwdThreads), args, smem, st);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kFwdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

cudaError_t launch_pool_finish(const BldArgs& a, int dtype, int64_t ntl, void* pooled, cudaStream_t st) {
  const void* kern = dtype == kF32    ? bld_pool_finish_f32()
                     : dtype == kBF16 ? bld_pool_finish_bf16()
                     : dtype == kF16  ? bld_pool_finish_f16()
                                      : nullptr;
  if (kern == nullptr) return cudaErrorInvalidValue;
  // programmatic dependent launch: the launch overlaps the march's tail and the
  // kernel's griddepcontrol.wait holds it until the march's partials are visible
  void* args[] = {const_cast<BldArgs*>(&a), &ntl, &pooled};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((a.D + 31) / 32), static_cast<unsigned>(a.nbatch));
  cfg.blockDim = dim3(kPoolThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

int bld_march_ctas_per_sm(int dtype, int steps, int causal, int adjoint, int residual, int contract) {
  struct Entry {
    const void* kern;
    int dev;
    int n;
  };
  static Entry table[256];
  static int used = 0;
  static std::mutex mu;
  const void* kern = march_kernel(dtype, steps, causal, adjoint, residual, 0, 0, contract);
  if (kern == nullptr) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].kern == kern && table[i].dev == dev) return table[i].n;
  const size_t smem = fwd_smem_bytes(dtype);
  if (ensure_smem_attr(kern, smem) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kFwdThreads, smem) != cudaSuccess || n <= 0) return -1;
  if (used < 256) table[used++] = Entry{kern, dev, n};
  return n;
}

int read_device_error_bld_fwd(int clear) {
  // the first non-zero word of the units (each unit keeps its own)
  int (*const readers[])(int) = {read_device_error_bld_fwd_f32, read_device_error_bld_fwd_bf16,
                                 read_device_error_bld_fwd_bf16_fm, read_device_error_bld_fwd_f16,
                                 read_device_error_bld_fwd_f16_fm};
  int v = 0;
  for (auto* r : readers) {
    const int e = r(clear);
    if (e < 0) return -1;
    if (v == 0) v = e;
  }
  return v;
}

}  // namespace cta
