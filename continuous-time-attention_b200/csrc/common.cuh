// Shared device helpers for the diffusion-stencil kernels (sm_100a only).
//
// Arithmetic contract.  The reference evaluates one diffusion step as a chain of
// separately rounded fp32 element-wise ops (src/cta/ops/diffusion.py:52-53,
// src/models/pde_layers.py:141,147/162,219):
//     lap = (right - 2*mid) + left ;  y = mid + alpha * lap
// `2*mid` is exact, so `right - 2*mid` rounded once equals fma(mid, -2, right).
// Every other op is issued as its own round-to-nearest instruction
// (__fadd2_rn / __fmul2_rn), never contracted, so the fp32 forward result is
// bit-identical to the reference's CPU result.
//
// Two adjacent feature columns are processed together as one float2 with the
// Blackwell packed-fp32 instructions (FADD2/FMUL2/FFMA2); each lane of a
// packed op rounds exactly like the scalar op.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "cta_stencil kernels target sm_100a only"
#endif

namespace cta {

// dtype codes shared with the C ABI (include/cta_stencil.h)
enum : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

// device-side error codes written to the per-TU error word
enum : int { kDevOk = 0, kDevTimeout = 1 };

// ---------------------------------------------------------------------------
// element traits: load/store pairs of columns as float2
// ---------------------------------------------------------------------------
template <typename T> struct Elem;

template <> struct Elem<float> {
  using Pair = float2;
  static constexpr int kCode = kF32;
  __device__ __forceinline__ static float2 unpack(float2 v) { return v; }
  __device__ __forceinline__ static float2 pack(float2 v) { return v; }
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};

template <> struct Elem<__nv_bfloat16> {
  using Pair = __nv_bfloat162;
  static constexpr int kCode = kBF16;
  __device__ __forceinline__ static float2 unpack(__nv_bfloat162 v) { return __bfloat1622float2(v); }
  __device__ __forceinline__ static __nv_bfloat162 pack(float2 v) { return __float22bfloat162_rn(v); }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <> struct Elem<__half> {
  using Pair = __half2;
  static constexpr int kCode = kF16;
  __device__ __forceinline__ static float2 unpack(__half2 v) { return __half22float2(v); }
  __device__ __forceinline__ static __half2 pack(float2 v) { return __float22half2_rn(v); }
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};

// ---------------------------------------------------------------------------
// packed fp32 stencil arithmetic
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Non-causal update of the centre row c from rows l (i-1) and r (i+1).
__device__ __forceinline__ float2 stencil_nc(float2 l, float2 c, float2 r, float2 al) {
  float2 t = __ffma2_rn(c, f2(-2.f), r);  // r - 2c, one rounding (2c is exact)
  t = __fadd2_rn(t, l);
  t = __fmul2_rn(al, t);
  return __fadd2_rn(c, t);
}

// Causal update of row i (value c) from rows i-1 (p1) and i-2 (p2):
// lap = (x[i] - 2 x[i-1]) + x[i-2] (src/models/pde_layers.py:141,145-147).
__device__ __forceinline__ float2 stencil_c(float2 p2, float2 p1, float2 c, float2 al) {
  float2 t = __ffma2_rn(p1, f2(-2.f), c);
  t = __fadd2_rn(t, p2);
  t = __fmul2_rn(al, t);
  return __fadd2_rn(c, t);
}

// Laplacian only, same rounding sequence as above.
__device__ __forceinline__ float2 lap3(float2 lo, float2 mid, float2 hi) {
  float2 t = __ffma2_rn(mid, f2(-2.f), hi);
  return __fadd2_rn(t, lo);
}

__device__ __forceinline__ float2 sel2(bool p, float2 a, float2 b) {
  return make_float2(p ? a.x : b.x, p ? a.y : b.y);
}

// ---------------------------------------------------------------------------
// shared-memory / mbarrier / TMA PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after ~1 s of wall time and
// reports false, so a lost transaction turns into an error status instead of
// a hung GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > 1000000000ull) return false;
  }
}

// 3-D tiled TMA load (no multicast): coordinates are (column, row, batch).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// mask helpers: any dtype, "valid" means non-zero (src/models/pde_layers.py:33,57-59)
// ---------------------------------------------------------------------------
enum : int { kMaskU8 = 0, kMaskI32 = 1, kMaskI64 = 2, kMaskF32 = 3, kMaskBF16 = 4, kMaskF16 = 5 };

__device__ __forceinline__ bool mask_valid(const void* m, int dtype, int64_t idx) {
  switch (dtype) {
    case kMaskU8: return static_cast<const uint8_t*>(m)[idx] != 0;
    case kMaskI32: return static_cast<const int32_t*>(m)[idx] != 0;
    case kMaskI64: return static_cast<const int64_t*>(m)[idx] != 0;
    case kMaskF32: return static_cast<const float*>(m)[idx] != 0.f;
    case kMaskBF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(m)[idx]) != 0.f;
    default: return __half2float(static_cast<const __half*>(m)[idx]) != 0.f;
  }
}

// alpha may live on the device (a learnable parameter) in fp32/bf16/fp16
__device__ __forceinline__ float load_scalar(const void* p, int dtype) {
  switch (dtype) {
    case kBF16: return __bfloat162float(*static_cast<const __nv_bfloat16*>(p));
    case kF16: return __half2float(*static_cast<const __half*>(p));
    default: return *static_cast<const float*>(p);
  }
}

}  // namespace cta
