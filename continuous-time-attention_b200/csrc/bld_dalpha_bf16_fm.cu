// Backward-with-d(alpha) kernels of bld_dalpha_kernel.cuh: bf16 tensors, contracted arithmetic.
// One translation unit per (dtype, arithmetic) so that they compile in parallel.
#include "bld_dalpha_kernel.cuh"

namespace cta {

const void* bld_dalpha_kernel_bf16_fm(int steps, int causal, int kind) {
  return da_select<__nv_bfloat16, true>(steps, causal, kind);
}

int read_device_error_bld_dalpha_bf16_fm(int clear) { return read_da_error_word(clear); }

}  // namespace cta
