// Backward-with-d(alpha) kernels of bld_dalpha_kernel.cuh: fp16 tensors, contracted arithmetic.
// One translation unit per (dtype, arithmetic) so that they compile in parallel.
#include "bld_dalpha_kernel.cuh"

namespace cta {

const void* bld_dalpha_kernel_f16_fm(int steps, int causal, int kind) {
  return da_select<__half, true>(steps, causal, kind);
}

int read_device_error_bld_dalpha_f16_fm(int clear) { return read_da_error_word(clear); }

}  // namespace cta
