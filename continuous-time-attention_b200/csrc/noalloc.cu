// Allocation-free variant of the [B, L, D] fused backward with d(alpha).
//
// cta_diffusion_bwd_bld needs a small caller-provided scratch buffer for its
// d(alpha) reduction (one partial sum per CTA and step, plus a completion
// counter).  Some callers cannot hand out fresh device memory: an engine that
// has already reserved nearly all of the GPU for its own pool (a serving
// process that sizes its KV cache to fill the card), or a latency-critical
// path where cudaMalloc's implicit device synchronisation is not acceptable.
// For them this file keeps the scratch in a fixed, file-scope device array that
// is created with the library and lives until the process exits; the entry
// point below never calls cudaMalloc, cudaFree or any allocating routine.
//
// The array is one per device and shared by every call on that device: calls
// whose work overlaps on the GPU (different streams, or different host threads)
// race on it and must be serialised by the caller.
#include <mutex>

#include "cta_stencil.h"
#include "kernels.h"

namespace {

// Counter header (kWsHeaderBytes = 8 KiB) + 65536 fp32 partial sums = 270336 B per device.
constexpr int64_t kScratchHeader = cta::kWsHeaderBytes;
constexpr int64_t kScratchPartials = 65536;
constexpr int64_t kScratchBytes = kScratchHeader + kScratchPartials * static_cast<int64_t>(sizeof(float));

static __device__ __align__(256) unsigned char g_dalpha_scratch[kScratchBytes];

// Device address of g_dalpha_scratch for the current device.  On the host the
// symbol's name only stands for the array; the address a kernel may use has to
// be queried from the runtime, once per device, with that device current.
int scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CTA_ECUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dalpha_scratch) != cudaSuccess || p == nullptr) return CTA_ECUDA;
    addr[dev] = p;
  }
  *out = addr[dev];
  return CTA_OK;
}

}  // namespace

extern "C" int cta_diffusion_bwd_bld_noalloc(const void* grad_out, void* grad_in, const void* x, float* dalpha,
                                             int64_t B, int64_t L, int64_t D, int64_t g_sB, int64_t g_sL,
                                             int64_t x_sB, int64_t x_sL, int64_t d_sB, int64_t d_sL, int dtype,
                                             int steps, int causal, const float* alpha,
                                             const void* const* alpha_dev, int alpha_dev_dtype, const void* mask,
                                             int mask_dtype, int64_t mask_sB, int64_t mask_sL, void* stream) {
  void* scratch = nullptr;
  int64_t scratch_bytes = 0;
  if (dalpha != nullptr) {
    const int64_t need = cta_diffusion_bwd_bld_workspace_bytes(B, L, D, dtype, steps, causal);
    if (need > kScratchBytes) {
      cta::set_last_error(
          "cta_diffusion_bwd_bld_noalloc: this shape needs %lld bytes of d(alpha) scratch, the built-in "
          "scratch holds %lld bytes; use cta_diffusion_bwd_bld with a caller-provided workspace",
          static_cast<long long>(need), static_cast<long long>(kScratchBytes));
      return CTA_EINVAL;
    }
    const int rc = scratch_address(&scratch);
    if (rc != CTA_OK) {
      cta::set_last_error("cta_diffusion_bwd_bld_noalloc: could not look up the device address of the scratch");
      return rc;
    }
    // the completion counters must start at zero; the partials are rewritten by every call
    const cudaError_t e = cudaMemsetAsync(scratch, 0, kScratchHeader, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
      cta::set_last_error("cta_diffusion_bwd_bld_noalloc: clearing the scratch counters failed: %s",
                          cudaGetErrorString(e));
      return CTA_ECUDA;
    }
    scratch_bytes = kScratchBytes;
  }
  return cta_diffusion_bwd_bld(grad_out, grad_in, x, dalpha, scratch, scratch_bytes, B, L, D, g_sB, g_sL, x_sB,
                               x_sL, d_sB, d_sL, dtype, steps, causal, alpha, alpha_dev, alpha_dev_dtype, mask,
                               mask_dtype, mask_sB, mask_sL, stream);
}
