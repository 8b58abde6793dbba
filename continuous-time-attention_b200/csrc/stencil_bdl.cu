// Fused multi-step diffusion stencil on [B, D, L] tensors (sequence axis
// contiguous) -- the layout of the reference's kernel entry points
// (kernels/diffusion_triton.py:732-910) and of the `layout="bdl"` PDE layers
// (src/models/pde_layers.py:113-188).
//
// Work decomposition.  Every (b, d) row is cut into windows of 256 positions
// (32 lanes x 8 consecutive positions, one 16-byte vector per lane for
// 16-bit types).  The outer lane(s) of a window are halo: all `steps` time
// levels are iterated in registers, each level exchanging one (or two, for the
// one-sided causal stencil) boundary values with the neighbouring lanes by
// warp shuffles, and the inner 30 lanes write 240 finished positions.  Two
// windows are processed together, packed into the two halves of a float2, so
// the arithmetic runs on the packed fp32 pipe.  Inputs are read once (the 16
// halo positions per window are L1/L2 hits) and outputs written once.
//
// Backward applies the adjoint of each step (kernels/diffusion_triton.py:96-133,
// generalised to masks and the causal stencil): with a = alpha * g on updated
// positions and 0 on fixed ones, g <- g + (a[i+1] - 2 a[i]) + a[i-1]
// (non-causal) or g <- g + (a[i] - 2 a[i+1]) + a[i+2] (causal).
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace cta {

__device__ int g_bdl_error;

namespace {

constexpr int E8 = kBdlElems;

template <typename T>
__device__ __forceinline__ void load_window(const BdlArgs& a, int64_t row, int64_t p0, float* v) {
  // positions p0 .. p0+7 of `row`; zero outside [0, L)
  using E = Elem<T>;
  const T* rp = static_cast<const T*>(a.in) + row * a.in_rs;
  if (a.vec_ok && p0 >= 0 && p0 + E8 <= a.L) {
    if (sizeof(T) == 2) {
      const uint4 q = *reinterpret_cast<const uint4*>(rp + p0);
      const typename E::Pair* pp = reinterpret_cast<const typename E::Pair*>(&q);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = E::unpack(pp[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const float4 q0 = *reinterpret_cast<const float4*>(rp + p0);
      const float4 q1 = *reinterpret_cast<const float4*>(rp + p0 + 4);
      v[0] = q0.x; v[1] = q0.y; v[2] = q0.z; v[3] = q0.w;
      v[4] = q1.x; v[5] = q1.y; v[6] = q1.z; v[7] = q1.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < E8; ++i) {
      const int64_t p = p0 + i;
      v[i] = (p >= 0 && p < a.L) ? E::to_f(rp[p]) : 0.f;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_window(const BdlArgs& a, int64_t row, int64_t p0, const float* v) {
  using E = Elem<T>;
  T* rp = static_cast<T*>(a.out) + row * a.out_rs;
  if (a.vec_ok && p0 >= 0 && p0 + E8 <= a.L) {
    if (sizeof(T) == 2) {
      uint4 q;
      typename E::Pair* pp = reinterpret_cast<typename E::Pair*>(&q);
#pragma unroll
      for (int i = 0; i < 4; ++i) pp[i] = E::pack(make_float2(v[2 * i], v[2 * i + 1]));
      *reinterpret_cast<uint4*>(rp + p0) = q;
    } else {
      *reinterpret_cast<float4*>(rp + p0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(rp + p0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < E8; ++i) {
      const int64_t p = p0 + i;
      if (p >= 0 && p < a.L) rp[p] = E::from_f(v[i]);
    }
  }
}

// fixed-position bits (bit i = position p0+i) for one lane of one window
template <bool CAUSAL>
__device__ __forceinline__ uint32_t fixed_bits(const BdlArgs& a, int64_t row, int64_t p0, bool valid_row) {
  uint32_t bits = 0;
  const int64_t lo = CAUSAL ? 1 : 0;
  const int64_t hi = CAUSAL ? a.L : a.L - 1;
#pragma unroll
  for (int i = 0; i < E8; ++i) {
    const int64_t p = p0 + i;
    bool fx = !valid_row || p <= lo || p >= hi;
    if (!fx && a.mask != nullptr) {
      const int64_t base = (row / a.D) * a.msB;
      const bool v0 = mask_valid(a.mask, a.mask_dtype, base + p * a.msL);
      const bool v1 = mask_valid(a.mask, a.mask_dtype, base + (p - 1) * a.msL);
      const bool v2 = mask_valid(a.mask, a.mask_dtype, base + (CAUSAL ? p - 2 : p + 1) * a.msL);
      fx = !(v0 && v1 && v2);
    }
    bits |= static_cast<uint32_t>(fx) << i;
  }
  return bits;
}

__device__ __forceinline__ pf2 shfl_up_p(pf2 v, int d) { return __shfl_up_sync(0xffffffffu, v, d); }
__device__ __forceinline__ pf2 shfl_down_p(pf2 v, int d) { return __shfl_down_sync(0xffffffffu, v, d); }

// select per packed half: keep `keep` where the fixed bit of that window is set
__device__ __forceinline__ pf2 sel_fixed(uint32_t fa, uint32_t fb, int i, pf2 keep, pf2 upd) {
  float k0, k1, u0, u1;
  upk(keep, k0, k1);
  upk(upd, u0, u1);
  return pk(((fa >> i) & 1u) ? k0 : u0, ((fb >> i) & 1u) ? k1 : u1);
}

}  // namespace

template <typename T, int S, bool CAUSAL, bool BWD>
__global__ void __launch_bounds__(kBdlThreads) bdl_kernel(const BdlArgs a) {
  // halo lanes: the one-sided causal stencil reaches 2*S <= 16 positions to
  // the left (forward) or right (adjoint); the centred one S <= 8 each side.
  constexpr int HLN = CAUSAL ? (BWD ? 0 : 2) : 1;
  constexpr int HRN = CAUSAL ? (BWD ? 2 : 0) : 1;
  const int lane = threadIdx.x & 31;
  const int64_t nwin = (a.L + kBdlOut - 1) / kBdlOut;
  const int64_t total = a.rows * nwin;
  const int64_t pair = (static_cast<int64_t>(blockIdx.x) * kBdlThreads + threadIdx.x) >> 5;
  const int64_t wa = 2 * pair, wb = 2 * pair + 1;
  if (wa >= total) return;  // warp-uniform
  const bool vb = wb < total;
  const int64_t ra = wa / nwin, rbw = vb ? wb / nwin : ra;
  const int64_t pa = (wa - ra * nwin) * kBdlOut - HLN * E8 + lane * E8;
  const int64_t pb = vb ? (wb - rbw * nwin) * kBdlOut - HLN * E8 + lane * E8 : pa;

  float va[E8], vbv[E8];
  load_window<T>(a, ra, pa, va);
  if (vb) load_window<T>(a, rbw, pb, vbv);
  else {
#pragma unroll
    for (int i = 0; i < E8; ++i) vbv[i] = 0.f;
  }
  // window A in the low half, window B in the high half of every pair
  pf2 e[E8];
#pragma unroll
  for (int i = 0; i < E8; ++i) e[i] = pk(va[i], vbv[i]);

  // Windows that lie strictly inside the domain (and calls without a mask) have
  // no fixed position: skip the per-position bookkeeping there (warp-uniform).
  const int64_t lo_fixed = CAUSAL ? 1 : 0, hi_fixed = CAUSAL ? a.L : a.L - 1;
  const int64_t wa0 = (wa - ra * nwin) * kBdlOut - HLN * E8;
  const int64_t wb0 = vb ? (wb - rbw * nwin) * kBdlOut - HLN * E8 : wa0;
  const bool interior = a.mask == nullptr && vb && wa0 > lo_fixed && wa0 + 32 * E8 - 1 < hi_fixed &&
                        wb0 > lo_fixed && wb0 + 32 * E8 - 1 < hi_fixed;
  uint32_t fa = 0u, fb = 0u;
  if (!interior) {
    fa = fixed_bits<CAUSAL>(a, ra, pa, true);
    fb = fixed_bits<CAUSAL>(a, rbw, pb, vb);
  }
  const bool slow = !interior && __any_sync(0xffffffffu, (fa | fb) != 0u);

  float al[kMaxSteps];
#pragma unroll
  for (int k = 0; k < kMaxSteps; ++k)
    if (k < S) al[k] = a.alpha_dev[k] != nullptr ? load_scalar(a.alpha_dev[k], a.alpha_dev_dtype) : a.alpha[k];
  const pf2 m2 = pbc(-2.f);
  const pf2 zn = pbc(a.neg_zero);

  auto run = [&](auto slow_tag) {
    constexpr bool SLOW = decltype(slow_tag)::value;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      if (!BWD) {
        const pf2 alv = pbc(al[s]);
        pf2 n[E8];
        if (CAUSAL) {
          const pf2 m2n = shfl_up_p(e[E8 - 2], 1), m1n = shfl_up_p(e[E8 - 1], 1);
#pragma unroll
          for (int i = 0; i < E8; ++i) {
            const pf2 p2 = i >= 2 ? e[i - 2] : (i == 1 ? m1n : m2n);
            const pf2 p1 = i >= 1 ? e[i - 1] : m1n;
            n[i] = pst_c(p2, p1, e[i], alv, m2, zn);
          }
        } else {
          const pf2 lft = shfl_up_p(e[E8 - 1], 1), rgt = shfl_down_p(e[0], 1);
#pragma unroll
          for (int i = 0; i < E8; ++i) {
            const pf2 l = i > 0 ? e[i - 1] : lft;
            const pf2 r = i < E8 - 1 ? e[i + 1] : rgt;
            n[i] = pst_nc(l, e[i], r, alv, m2, zn);
          }
        }
#pragma unroll
        for (int i = 0; i < E8; ++i) e[i] = SLOW ? sel_fixed(fa, fb, i, e[i], n[i]) : n[i];
      } else {
        // adjoint of forward step S-1-s: a = alpha * g on updated positions
        const pf2 alv = pbc(al[S - 1 - s]);
        pf2 av[E8];
#pragma unroll
        for (int i = 0; i < E8; ++i) {
          av[i] = pmul_sep(alv, e[i], zn);
          if (SLOW) av[i] = sel_fixed(fa, fb, i, 0ull, av[i]);
        }
        if (CAUSAL) {
          const pf2 q1 = shfl_down_p(av[0], 1), q2 = shfl_down_p(av[1], 1);
#pragma unroll
          for (int i = 0; i < E8; ++i) {
            const pf2 a1 = i + 1 < E8 ? av[i + 1] : (i + 1 == E8 ? q1 : q2);
            const pf2 a2 = i + 2 < E8 ? av[i + 2] : (i + 2 == E8 ? q1 : q2);
            e[i] = padd(e[i], plap(a2, a1, av[i], m2));  // (a[i] - 2a[i+1]) + a[i+2]
          }
        } else {
          const pf2 lft = shfl_up_p(av[E8 - 1], 1), rgt = shfl_down_p(av[0], 1);
          pf2 n[E8];
#pragma unroll
          for (int i = 0; i < E8; ++i) {
            const pf2 l = i > 0 ? av[i - 1] : lft;
            const pf2 r = i < E8 - 1 ? av[i + 1] : rgt;
            n[i] = padd(e[i], plap(l, av[i], r, m2));
          }
#pragma unroll
          for (int i = 0; i < E8; ++i) e[i] = n[i];
        }
      }
    }
  };
  if (slow) run(std::true_type{});
  else run(std::false_type{});

  if (lane >= HLN && lane < 32 - HRN) {
#pragma unroll
    for (int i = 0; i < E8; ++i) upk(e[i], va[i], vbv[i]);
    store_window<T>(a, ra, pa, va);
    if (vb) store_window<T>(a, rbw, pb, vbv);
  }
}

namespace {

template <typename T, int S, bool C, bool B>
cudaError_t launch_t(const BdlArgs& a, cudaStream_t st) {
  const int64_t nwin = (a.L + kBdlOut - 1) / kBdlOut;
  const int64_t pairs = (a.rows * nwin + 1) / 2;
  const int64_t blocks = (pairs * 32 + kBdlThreads - 1) / kBdlThreads;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  bdl_kernel<T, S, C, B><<<static_cast<unsigned>(blocks), kBdlThreads, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T, bool C, bool B>
cudaError_t by_steps(const BdlArgs& a, int steps, cudaStream_t st) {
  switch (steps) {
    case 1: return launch_t<T, 1, C, B>(a, st);
    case 2: return launch_t<T, 2, C, B>(a, st);
    case 3: return launch_t<T, 3, C, B>(a, st);
    case 4: return launch_t<T, 4, C, B>(a, st);
    case 5: return launch_t<T, 5, C, B>(a, st);
    case 6: return launch_t<T, 6, C, B>(a, st);
    case 7: return launch_t<T, 7, C, B>(a, st);
    case 8: return launch_t<T, 8, C, B>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t by_mode(const BdlArgs& a, int steps, int causal, int bwd, cudaStream_t st) {
  if (causal) return bwd ? by_steps<T, true, true>(a, steps, st) : by_steps<T, true, false>(a, steps, st);
  return bwd ? by_steps<T, false, true>(a, steps, st) : by_steps<T, false, false>(a, steps, st);
}

}  // namespace

cudaError_t launch_bdl(const BdlArgs& a, int dtype, int steps, int causal, int backward, cudaStream_t st) {
  switch (dtype) {
    case kF32: return by_mode<float>(a, steps, causal, backward, st);
    case kBF16: return by_mode<__nv_bfloat16>(a, steps, causal, backward, st);
    case kF16: return by_mode<__half>(a, steps, causal, backward, st);
    default: return cudaErrorInvalidValue;
  }
}

int read_device_error_bdl(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bdl_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bdl_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace cta
