// Forward / adjoint march kernels of bld_fwd_kernel.cuh: fp32 tensors (always the exact arithmetic), with the PDE kinds and the pooled form.
// One translation unit per (dtype, arithmetic) so that they compile in parallel.
#include "bld_fwd_kernel.cuh"

namespace cta {

const void* bld_fwd_kernel_f32(int steps, int causal, int adj, int res, int kind, int pool) {
  return march_select<float, false>(steps, causal, adj, res, kind, pool);
}

const void* bld_pool_finish_f32() { return reinterpret_cast<const void*>(&pool_finish_kernel<float>); }

int read_device_error_bld_fwd_f32(int clear) { return read_fwd_error_word(clear); }

}  // namespace cta
