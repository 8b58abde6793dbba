// Host side of the backward with d(alpha) (bld_dalpha_kernel.cuh): kernel
// selection across the per-dtype units, launch, occupancy, shared-memory size
// and the device error words.
#include "bld_dalpha_kernel.cuh"

namespace cta {

// bld_dalpha_<dtype>[_fm].cu
const void* bld_dalpha_kernel_f32(int steps, int causal, int kind);
const void* bld_dalpha_kernel_bf16(int steps, int causal, int kind);
const void* bld_dalpha_kernel_bf16_fm(int steps, int causal, int kind);
const void* bld_dalpha_kernel_f16(int steps, int causal, int kind);
const void* bld_dalpha_kernel_f16_fm(int steps, int causal, int kind);
int read_device_error_bld_dalpha_f32(int clear);
int read_device_error_bld_dalpha_bf16(int clear);
int read_device_error_bld_dalpha_bf16_fm(int clear);
int read_device_error_bld_dalpha_f16(int clear);
int read_device_error_bld_dalpha_f16_fm(int clear);

size_t dalpha_smem_bytes(int dtype, int steps, int causal) {
  if (dtype == kF32) return causal ? da_smem_s<float, true>(steps) : da_smem_s<float, false>(steps);
  return causal ? da_smem_s<__nv_bfloat16, true>(steps) : da_smem_s<__nv_bfloat16, false>(steps);
}


namespace {

// fm: the contracted arithmetic, built for 16-bit tensors only
const void* da_kernel(int dtype, int steps, int causal, int kind = 0, int fm = 0) {
  switch (dtype) {
    case kF32: return fm ? nullptr : bld_dalpha_kernel_f32(steps, causal, kind);
    case kBF16: return fm ? bld_dalpha_kernel_bf16_fm(steps, causal, kind) : bld_dalpha_kernel_bf16(steps, causal, kind);
    case kF16: return fm ? bld_dalpha_kernel_f16_fm(steps, causal, kind) : bld_dalpha_kernel_f16(steps, causal, kind);
    default: return nullptr;
  }
}

}  // namespace

cudaError_t launch_bld_dalpha(const BldArgs& a, const CUtensorMap* gmap, const CUtensorMap* xmap,
                              const CUtensorMap* ymap, int dtype, int steps, int causal, dim3 grid, cudaStream_t st) {
  const void* kern = da_kernel(dtype, steps, causal, a.pde_kind, a.contract);
  if (kern == nullptr) return cudaErrorInvalidValue;
  const size_t smem = dalpha_smem_bytes(dtype, steps, causal);
  cudaError_t e = ensure_smem_attr(kern, smem);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<CUtensorMap*>(gmap), const_cast<CUtensorMap*>(xmap), const_cast<CUtensorMap*>(ymap),
                  const_cast<BldArgs*>(&a)};
  return cudaLaunchKernel(kern, grid, dim3(kFwdThreads), args, smem, st);
}

int bld_dalpha_ctas_per_sm(int dtype, int steps, int causal, int contract) {
  struct Entry {
    const void* kern;
    int dev;
    int n;
  };
  static Entry table[256];
  static int used = 0;
  static std::mutex mu;
  const void* kern = da_kernel(dtype, steps, causal, 0, contract);
  if (kern == nullptr) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].kern == kern && table[i].dev == dev) return table[i].n;
  const size_t smem = dalpha_smem_bytes(dtype, steps, causal);
  if (ensure_smem_attr(kern, smem) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kFwdThreads, smem) != cudaSuccess || n <= 0) return -1;
  if (used < 256) table[used++] = Entry{kern, dev, n};
  return n;
}

int read_device_error_bld_dalpha(int clear) {
  // the first non-zero word of the units (each unit keeps its own)
  int (*const readers[])(int) = {read_device_error_bld_dalpha_f32, read_device_error_bld_dalpha_bf16,
                                 read_device_error_bld_dalpha_bf16_fm, read_device_error_bld_dalpha_f16,
                                 read_device_error_bld_dalpha_f16_fm};
  int v = 0;
  for (auto* r : readers) {
    const int e = r(clear);
    if (e < 0) return -1;
    if (v == 0) v = e;
  }
  return v;
}

}  // namespace cta
