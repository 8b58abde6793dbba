// Forward / adjoint march kernels of bld_fwd_kernel.cuh: fp16 tensors, contracted arithmetic (forward and adjoint diffusion).
// One translation unit per (dtype, arithmetic) so that they compile in parallel.
#include "bld_fwd_kernel.cuh"

namespace cta {

const void* bld_fwd_kernel_f16_fm(int steps, int causal, int adj, int res, int kind, int pool) {
  return march_select<__half, true>(steps, causal, adj, res, kind, pool);
}

int read_device_error_bld_fwd_f16_fm(int clear) { return read_fwd_error_word(clear); }

}  // namespace cta
