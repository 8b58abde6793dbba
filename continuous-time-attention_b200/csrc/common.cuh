// Shared device helpers for the diffusion-stencil kernels (sm_100a only).
//
// Arithmetic contract.  The reference evaluates one diffusion step as a chain of
// separately rounded fp32 element-wise ops (src/cta/ops/diffusion.py:52-53,
// src/models/pde_layers.py:141,147/162,219):
//     lap = (right - 2*mid) + left ;  y = mid + alpha * lap
// `2*mid` is exact, so `right - 2*mid` rounded once equals fma(mid, -2, right).
// Every other op is issued as its own round-to-nearest instruction (add2 /
// mul2 below), never contracted, so the fp32 forward result is bit-identical
// to the reference's CPU result.
//
// Two adjacent feature columns are processed together as one float2 with the
// Blackwell packed-fp32 instructions (add/mul/fma .f32x2); each half of a
// packed op rounds exactly like the scalar op.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "cta_stencil kernels target sm_100a only"
#endif

// Force-inline a device lambda.  The march kernels are built from lambdas
// (row step, chunk, pipeline step) called from several places; one that the
// inliner leaves as a call takes the kernel's register state through local
// memory (a stack frame of a kilobyte or more) and runs an order of magnitude
// slower.
#define CTA_INLINE __attribute__((always_inline))

namespace cta {

// Calls f(std::integral_constant<int, I>{}) for I = 0 .. N-1 (compile-time unrolled loop).
template <typename F, int... I>
__device__ __forceinline__ void static_for_impl(F&& f, std::integer_sequence<int, I...>) {
  (f(std::integral_constant<int, I>{}), ...);
}
template <int N, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  static_for_impl(static_cast<F&&>(f), std::make_integer_sequence<int, N>{});
}

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
// packed fp32 arithmetic.  Issued as PTX with an explicit .rn rounding
// modifier: ptxas never contracts such instructions into a fused multiply-add,
// which the reference's separately rounded ops require for bit-identical fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// a * b + c with a single rounding
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Non-causal update of the centre row c from rows l (i-1) and r (i+1).
__device__ __forceinline__ float2 stencil_nc(float2 l, float2 c, float2 r, float2 al) {
  float2 t = fma2(c, f2(-2.f), r);  // r - 2c, one rounding (2c is exact)
  t = add2(t, l);
  t = mul2(al, t);
  return add2(c, t);
}

// Causal update of row i (value c) from rows i-1 (p1) and i-2 (p2):
// lap = (x[i] - 2 x[i-1]) + x[i-2] (src/models/pde_layers.py:141,145-147).
__device__ __forceinline__ float2 stencil_c(float2 p2, float2 p1, float2 c, float2 al) {
  float2 t = fma2(p1, f2(-2.f), c);
  t = add2(t, p2);
  t = mul2(al, t);
  return add2(c, t);
}

// Laplacian only, same rounding sequence as above.
__device__ __forceinline__ float2 lap3(float2 lo, float2 mid, float2 hi) {
  float2 t = fma2(mid, f2(-2.f), hi);
  return add2(t, lo);
}

__device__ __forceinline__ float2 sel2(bool p, float2 a, float2 b) {
  return make_float2(p ? a.x : b.x, p ? a.y : b.y);
}

// ---------------------------------------------------------------------------
// the same arithmetic on a pair held in ONE 64-bit register (pf2), so the
// packed instructions never need pair-forming moves.
// ---------------------------------------------------------------------------
typedef unsigned long long pf2;

__device__ __forceinline__ pf2 pk(float lo, float hi) {
  pf2 d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void upk(pf2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ pf2 pbc(float a) { return pk(a, a); }
__device__ __forceinline__ pf2 padd(pf2 a, pf2 b) {
  pf2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ pf2 pmul(pf2 a, pf2 b) {
  pf2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ pf2 pfma(pf2 a, pf2 b, pf2 c) {
  pf2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// Rounded product a*b computed as fma(a, b, zn) with zn = -0.0 supplied at
// run time.  -0 is the exact additive identity, so the result is round(a*b)
// for every sign; because ptxas cannot see that zn is zero it can neither turn
// this into a plain multiply nor contract it with the add that consumes it.
// (ptxas fuses packed mul.rn.f32x2 -> add.rn.f32x2 pairs into one fma even
// with -fmad=false; measured on B200, 148461 of 1M stencils differed.)
__device__ __forceinline__ pf2 pmul_sep(pf2 a, pf2 b, pf2 zn) { return pfma(a, b, zn); }

// non-causal update of centre c from l (row i-1) and r (row i+1); m2 = {-2,-2}.
// FM = false: c + round(alpha * lap), the reference's PyTorch ops (product and
// sum rounded separately).  FM = true: the product and the sum as ONE fma, the
// op order the reference's Triton kernels compile to (Triton contracts a
// multiply feeding an add by default; kernels/diffusion_triton.py:89-90).
template <bool FM = false>
__device__ __forceinline__ pf2 pst_nc(pf2 l, pf2 c, pf2 r, pf2 al, pf2 m2, pf2 zn) {
  pf2 t = pfma(c, m2, r);  // r - 2c, one rounding (2c is exact)
  t = padd(t, l);
  if constexpr (FM) {
    return pfma(al, t, c);
  } else {
    t = pmul_sep(al, t, zn);
    return padd(c, t);
  }
}
// causal update of c (row i) from p1 (row i-1) and p2 (row i-2)
template <bool FM = false>
__device__ __forceinline__ pf2 pst_c(pf2 p2, pf2 p1, pf2 c, pf2 al, pf2 m2, pf2 zn) {
  pf2 t = pfma(p1, m2, c);
  t = padd(t, p2);
  if constexpr (FM) {
    return pfma(al, t, c);
  } else {
    t = pmul_sep(al, t, zn);
    return padd(c, t);
  }
}
// (hi - 2 mid) + lo
__device__ __forceinline__ pf2 plap(pf2 lo, pf2 mid, pf2 hi, pf2 m2) { return padd(pfma(mid, m2, hi), lo); }
__device__ __forceinline__ pf2 psel(bool p, pf2 a, pf2 b) { return p ? a : b; }

// VEC (2 or 4) consecutive columns of one lane <-> one or two pairs
template <typename T, int VEC> struct ColVec;
template <typename T> struct Quad;
template <> struct Quad<__nv_bfloat16> {
  using V = uint2;
  __device__ __forceinline__ static pf2 w2p(uint32_t w) {
    return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t p2w(pf2 p) {
    float lo, hi;
    upk(p, lo, hi);
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ __forceinline__ static void split(V v, pf2& a, pf2& b) { a = w2p(v.x); b = w2p(v.y); }
  __device__ __forceinline__ static V join(pf2 a, pf2 b) { return make_uint2(p2w(a), p2w(b)); }
};
template <> struct Quad<__half> {
  using V = uint2;
  __device__ __forceinline__ static pf2 w2p(uint32_t w) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return pk(f.x, f.y);
  }
  __device__ __forceinline__ static uint32_t p2w(pf2 p) {
    float lo, hi;
    upk(p, lo, hi);
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  __device__ __forceinline__ static void split(V v, pf2& a, pf2& b) { a = w2p(v.x); b = w2p(v.y); }
  __device__ __forceinline__ static V join(pf2 a, pf2 b) { return make_uint2(p2w(a), p2w(b)); }
};
template <> struct Quad<float> {
  using V = float4;
  __device__ __forceinline__ static void split(V v, pf2& a, pf2& b) { a = pk(v.x, v.y); b = pk(v.z, v.w); }
  __device__ __forceinline__ static V join(pf2 a, pf2 b) {
    float4 r;
    upk(a, r.x, r.y);
    upk(b, r.z, r.w);
    return r;
  }
};
template <typename T> struct ColVec<T, 4> : Quad<T> {};

// y + r for two element vectors of T (y as stored, i.e. already rounded to T),
// added in fp32 and rounded once: an elementwise add of two tensors of type T
template <typename Q>
__device__ __forceinline__ typename Q::V vec_add_round(typename Q::V y, typename Q::V r) {
  pf2 ya, yb, ra, rb;
  Q::split(y, ya, yb);
  Q::split(r, ra, rb);
  return Q::join(padd(ya, ra), padd(yb, rb));
}
template <typename T> struct ColVec<T, 2> {
  // one pair; the second pair of the interface is unused and stays zero
  using V = typename std::conditional<sizeof(T) == 4, float2, uint32_t>::type;
  __device__ __forceinline__ static void split(V v, pf2& a, pf2& b) {
    if constexpr (sizeof(T) == 4) a = pk(v.x, v.y);
    else a = Quad<T>::w2p(v);
    b = 0ull;
  }
  __device__ __forceinline__ static V join(pf2 a, pf2) {
    if constexpr (sizeof(T) == 4) {
      float2 r;
      upk(a, r.x, r.y);
      return r;
    } else {
      return Quad<T>::p2w(a);
    }
  }
};

// ---------------------------------------------------------------------------
// shared-memory / mbarrier / TMA PTX wrappers
// ---------------------------------------------------------------------------
// Programmatic dependent launch.  launch_dependents lets the next kernel of the
// stream be scheduled as this grid's CTAs retire; wait blocks until every
// prerequisite grid has completed and its memory operations are visible.  Both
// are no-ops for a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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
__device__ __forceinline__ bool mbar_wait_bounded_ns(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  return mbar_wait_bounded_ns(bar, parity, 1000000000ull);
}

// 3-D tiled TMA load into this CTA's own shared memory: coordinates are (column, row, batch).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled TMA store from shared memory (plain store, no reduction); the
// coordinates must be non-negative, elements past the tensor end are dropped.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Predicated forms for one-warp CTAs: every lane executes the instruction and
// only a lane whose `p` is true issues it, so a lane-0 TMA section costs no
// divergent branch and no reconvergence.
__device__ __forceinline__ void mbar_arrive_expect_tx_if(bool p, uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t"
      "@q mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
      "r"(bytes), "r"(static_cast<uint32_t>(p))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_if(bool p, void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                               int c1, int c2) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %6, 0;\n\t"
      "@q cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(static_cast<uint32_t>(p))
      : "memory");
}
__device__ __forceinline__ void tma_store_3d_if(bool p, const CUtensorMap* map, const void* src, int c0, int c1,
                                                int c2) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %5, 0;\n\t"
      "@q cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];\n\t}" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(static_cast<uint32_t>(p))
      : "memory");
}
__device__ __forceinline__ void bulk_commit_if(bool p) {
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %0, 0;\n\t@q cp.async.bulk.commit_group;\n\t}" ::"r"(
                   static_cast<uint32_t>(p))
               : "memory");
}
// all committed bulk stores have finished READING their shared-memory source
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// all committed bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the async (TMA) proxy
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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
