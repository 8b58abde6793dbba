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

// 8 positions of two rows from shared memory, packed: row A in the low half,
// row B in the high half of each pair
template <typename T>
__device__ __forceinline__ void bdl_smem_pairs(const T* ra, const T* rb, pf2 (&e)[E8]) {
  using E = Elem<T>;
  if constexpr (sizeof(T) == 2) {
    const uint4 qa = *reinterpret_cast<const uint4*>(ra);
    const uint4 qb = *reinterpret_cast<const uint4*>(rb);
    const typename E::Pair* pa = reinterpret_cast<const typename E::Pair*>(&qa);
    const typename E::Pair* pb = reinterpret_cast<const typename E::Pair*>(&qb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = E::unpack(pa[i]), fb = E::unpack(pb[i]);
      e[2 * i] = pk(fa.x, fb.x);
      e[2 * i + 1] = pk(fa.y, fb.y);
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 qa = *reinterpret_cast<const float4*>(ra + 4 * h);
      const float4 qb = *reinterpret_cast<const float4*>(rb + 4 * h);
      e[4 * h] = pk(qa.x, qb.x);
      e[4 * h + 1] = pk(qa.y, qb.y);
      e[4 * h + 2] = pk(qa.z, qb.z);
      e[4 * h + 3] = pk(qa.w, qb.w);
    }
  }
}

template <typename T>
__device__ __forceinline__ void bdl_smem_store_pairs(T* ra, T* rb, const pf2 (&e)[E8]) {
  using E = Elem<T>;
  float va[E8], vb[E8];
#pragma unroll
  for (int i = 0; i < E8; ++i) upk(e[i], va[i], vb[i]);
  if constexpr (sizeof(T) == 2) {
    uint4 qa, qb;
    typename E::Pair* pa = reinterpret_cast<typename E::Pair*>(&qa);
    typename E::Pair* pb = reinterpret_cast<typename E::Pair*>(&qb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pa[i] = E::pack(make_float2(va[2 * i], va[2 * i + 1]));
      pb[i] = E::pack(make_float2(vb[2 * i], vb[2 * i + 1]));
    }
    *reinterpret_cast<uint4*>(ra) = qa;
    *reinterpret_cast<uint4*>(rb) = qb;
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      *reinterpret_cast<float4*>(ra + 4 * h) = make_float4(va[4 * h], va[4 * h + 1], va[4 * h + 2], va[4 * h + 3]);
      *reinterpret_cast<float4*>(rb + 4 * h) = make_float4(vb[4 * h], vb[4 * h + 1], vb[4 * h + 2], vb[4 * h + 3]);
    }
  }
}

// All `steps` levels of one 256-position window (8 positions per lane, two
// independent windows packed in the halves of each pair), in registers; the
// neighbours of a lane's first and last position come from the adjacent lanes.
// fa / fb: fixed-position bits of the two windows (SLOW only).
// MODE 0: forward; 1: adjoint; 2: forward with the contracted update (pst_nc).
template <int S, bool CAUSAL, int MODE, bool SLOW>
__device__ __forceinline__ void window_levels(pf2 (&e)[E8], uint32_t fa, uint32_t fb, const float (&al)[kMaxSteps],
                                              pf2 m2, pf2 zn) {
  constexpr bool BWD = MODE == 1;
  constexpr bool FM = MODE == 2;
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
          n[i] = pst_c<FM>(p2, p1, e[i], alv, m2, zn);
        }
      } else {
        const pf2 lft = shfl_up_p(e[E8 - 1], 1), rgt = shfl_down_p(e[0], 1);
#pragma unroll
        for (int i = 0; i < E8; ++i) {
          const pf2 l = i > 0 ? e[i - 1] : lft;
          const pf2 r = i < E8 - 1 ? e[i + 1] : rgt;
          n[i] = pst_nc<FM>(l, e[i], r, alv, m2, zn);
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
}

}  // namespace

template <typename T, int S, bool CAUSAL, int MODE>
__global__ void __launch_bounds__(kBdlThreads) bdl_kernel(const BdlArgs a) {
  constexpr bool BWD = MODE == 1;
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

  if (slow) window_levels<S, CAUSAL, MODE, true>(e, fa, fb, al, m2, zn);
  else window_levels<S, CAUSAL, MODE, false>(e, fa, fb, al, m2, zn);

  if (lane >= HLN && lane < 32 - HRN) {
#pragma unroll
    for (int i = 0; i < E8; ++i) upk(e[i], va[i], vbv[i]);
    store_window<T>(a, ra, pa, va);
    if (vb) store_window<T>(a, rbw, pb, vbv);
  }
}

// ---------------------------------------------------------------------------
// TMA pipeline form (dense rows that TMA can address).  A CTA is one warp
// owning two rows (packed in the halves of every pair) and a run of
// consecutive windows along L.  Each window's 256 x 2 input box arrives
// through a ring of TMA loads (kBdlStages deep, one mbarrier per slot), the
// levels run in registers as above, and the 240 x 2 finished positions leave
// through a staged TMA store, so loads, arithmetic and stores of successive
// windows overlap inside the warp.
// ---------------------------------------------------------------------------
template <typename T, int S, bool CAUSAL, int MODE>
__global__ void __launch_bounds__(32, 16)
    bdl_march_kernel(const __grid_constant__ CUtensorMap imap, const __grid_constant__ CUtensorMap omap,
                     const BdlArgs a) {
  constexpr bool BWD = MODE == 1;
  constexpr int HLN = CAUSAL ? (BWD ? 0 : 2) : 1;
  constexpr int HRN = CAUSAL ? (BWD ? 2 : 0) : 1;
  constexpr int NST = kBdlStages;
  constexpr int IN_CHUNK = kBdlRows * kBdlWin;                    // elements per input slot
  constexpr int OUT_SLOT = bdl_out_slot_elems<T>();               // elements per staging slot (128-B multiple)
  constexpr int NP = kBdlRows / 2;                                // row pairs (register pair sets) per CTA
  static_assert(kBdlRows % 2 == 0, "rows come in pairs");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  T* stage = ring + NST * IN_CHUNK;
  __shared__ __align__(8) uint64_t full_bar[NST];

  const int lane = threadIdx.x;
  const int64_t nwin = (a.L + kBdlOut - 1) / kBdlOut;
  const int64_t rp = blockIdx.x / a.nseg;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x % a.nseg) * a.tw;
  const int64_t w1 = w0 + a.tw < nwin ? w0 + a.tw : nwin;
  if (w0 >= w1) return;
  const int nw = static_cast<int>(w1 - w0);
  const int64_t r0 = static_cast<int64_t>(kBdlRows) * rp;

  if (lane == 0) {
    prefetch_tmap(&imap);
    prefetch_tmap(&omap);
#pragma unroll
    for (int s = 0; s < NST; ++s) mbar_init(&full_bar[s], 1);
    fence_mbar_init();
  }
  auto issue = [&](int i) {
    const int slot = i % NST;
    mbar_arrive_expect_tx(&full_bar[slot], IN_CHUNK * sizeof(T));
    tma_load_3d(ring + slot * IN_CHUNK, &imap, &full_bar[slot], static_cast<int>((w0 + i) * kBdlOut - HLN * E8),
                static_cast<int>(r0), 0);
  };
  if (lane == 0) {
    for (int i = 0; i < nw && i < NST; ++i) issue(i);
  }
  float al[kMaxSteps];
#pragma unroll
  for (int k = 0; k < kMaxSteps; ++k)
    if (k < S) al[k] = a.alpha_dev[k] != nullptr ? load_scalar(a.alpha_dev[k], a.alpha_dev_dtype) : a.alpha[k];
  const pf2 m2 = pbc(-2.f);
  const pf2 zn = pbc(a.neg_zero);
  const int64_t lo_fixed = CAUSAL ? 1 : 0, hi_fixed = CAUSAL ? a.L : a.L - 1;

  for (int i = 0; i < nw; ++i) {
    const int slot = i % NST;
    int err = mbar_wait_bounded(&full_bar[slot], (i / NST) & 1) ? 0 : 1;
    const int64_t ws = (w0 + i) * kBdlOut - HLN * E8;  // first loaded position of the window
    const int64_t p = ws + lane * E8;
    if (!err) {
      const T* buf = ring + slot * IN_CHUNK + lane * E8;
      const bool interior = a.mask == nullptr && ws > lo_fixed && ws + kBdlWin - 1 < hi_fixed;
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        pf2 e[E8];
        bdl_smem_pairs<T>(buf + (2 * q) * kBdlWin, buf + (2 * q + 1) * kBdlWin, e);
        uint32_t fa = 0u, fb = 0u;
        if (!interior) {
          fa = fixed_bits<CAUSAL>(a, r0 + 2 * q, p, r0 + 2 * q < a.rows);
          fb = fixed_bits<CAUSAL>(a, r0 + 2 * q + 1, p, r0 + 2 * q + 1 < a.rows);
        }
        if (!interior && __any_sync(0xffffffffu, (fa | fb) != 0u))
          window_levels<S, CAUSAL, MODE, true>(e, fa, fb, al, m2, zn);
        else
          window_levels<S, CAUSAL, MODE, false>(e, fa, fb, al, m2, zn);
        if (lane >= HLN && lane < 32 - HRN) {
          T* st = stage + (i & 1) * OUT_SLOT + (2 * q) * kBdlOut + (lane - HLN) * E8;
          bdl_smem_store_pairs<T>(st, st + kBdlOut, e);
        }
      }
      fence_proxy_async_smem();
    }
    // the store issued after the previous window must have finished reading the
    // staging slot that the next window overwrites
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    if (__any_sync(0xffffffffu, err)) {
      if (lane == 0) {
        atomicExch(&g_bdl_error, kDevTimeout);
        for (int j = i; j < nw && j < i + NST; ++j) mbar_wait_bounded(&full_bar[j % NST], (j / NST) & 1);
        bulk_wait_all();
      }
      __syncwarp();
      return;
    }
    if (lane == 0) {
      tma_store_3d(&omap, stage + (i & 1) * OUT_SLOT, static_cast<int>((w0 + i) * kBdlOut), static_cast<int>(r0), 0);
      bulk_commit();
      if (i + NST < nw) issue(i + NST);
    }
  }
  if (lane == 0) bulk_wait_all();
}

namespace {

template <typename T, int S, bool C, int M>
cudaError_t launch_t(const BdlArgs& a, cudaStream_t st) {
  const int64_t nwin = (a.L + kBdlOut - 1) / kBdlOut;
  const int64_t pairs = (a.rows * nwin + 1) / 2;
  const int64_t blocks = (pairs * 32 + kBdlThreads - 1) / kBdlThreads;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  bdl_kernel<T, S, C, M><<<static_cast<unsigned>(blocks), kBdlThreads, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T, bool C, int M>
cudaError_t by_steps(const BdlArgs& a, int steps, cudaStream_t st) {
  switch (steps) {
    case 1: return launch_t<T, 1, C, M>(a, st);
    case 2: return launch_t<T, 2, C, M>(a, st);
    case 3: return launch_t<T, 3, C, M>(a, st);
    case 4: return launch_t<T, 4, C, M>(a, st);
    case 5: return launch_t<T, 5, C, M>(a, st);
    case 6: return launch_t<T, 6, C, M>(a, st);
    case 7: return launch_t<T, 7, C, M>(a, st);
    case 8: return launch_t<T, 8, C, M>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int S, bool C, int M>
const void* march_ptr_s() {
  return reinterpret_cast<const void*>(bdl_march_kernel<T, S, C, M>);
}

template <typename T, bool C, int M>
const void* march_ptr(int steps) {
  switch (steps) {
    case 1: return march_ptr_s<T, 1, C, M>();
    case 2: return march_ptr_s<T, 2, C, M>();
    case 3: return march_ptr_s<T, 3, C, M>();
    case 4: return march_ptr_s<T, 4, C, M>();
    case 5: return march_ptr_s<T, 5, C, M>();
    case 6: return march_ptr_s<T, 6, C, M>();
    case 7: return march_ptr_s<T, 7, C, M>();
    case 8: return march_ptr_s<T, 8, C, M>();
    default: return nullptr;
  }
}

// mode: 0 forward, 1 adjoint, 2 forward with the contracted update (16-bit I/O only)
template <typename T>
const void* march_ptr_t(int steps, int causal, int mode) {
  if (mode == 2) {
    if constexpr (sizeof(T) == 2) return causal ? march_ptr<T, true, 2>(steps) : march_ptr<T, false, 2>(steps);
    return nullptr;
  }
  if (causal) return mode ? march_ptr<T, true, 1>(steps) : march_ptr<T, true, 0>(steps);
  return mode ? march_ptr<T, false, 1>(steps) : march_ptr<T, false, 0>(steps);
}

const void* bdl_march_ptr(int dtype, int steps, int causal, int mode) {
  switch (dtype) {
    case kF32: return march_ptr_t<float>(steps, causal, mode);
    case kBF16: return march_ptr_t<__nv_bfloat16>(steps, causal, mode);
    case kF16: return march_ptr_t<__half>(steps, causal, mode);
    default: return nullptr;
  }
}

template <typename T>
cudaError_t by_mode(const BdlArgs& a, int steps, int causal, int mode, cudaStream_t st) {
  if (mode == 2) {
    if constexpr (sizeof(T) == 2)
      return causal ? by_steps<T, true, 2>(a, steps, st) : by_steps<T, false, 2>(a, steps, st);
    return cudaErrorInvalidValue;
  }
  if (causal) return mode ? by_steps<T, true, 1>(a, steps, st) : by_steps<T, true, 0>(a, steps, st);
  return mode ? by_steps<T, false, 1>(a, steps, st) : by_steps<T, false, 0>(a, steps, st);
}

// kernel mode of a call: the adjoint, or the forward in the call's arithmetic
int bdl_mode(const BdlArgs& a, int backward) { return backward ? 1 : (a.contract ? 2 : 0); }

}  // namespace

cudaError_t launch_bdl(const BdlArgs& a, int dtype, int steps, int causal, int backward, cudaStream_t st) {
  const int mode = bdl_mode(a, backward);
  switch (dtype) {
    case kF32: return by_mode<float>(a, steps, causal, mode, st);
    case kBF16: return by_mode<__nv_bfloat16>(a, steps, causal, mode, st);
    case kF16: return by_mode<__half>(a, steps, causal, mode, st);
    default: return cudaErrorInvalidValue;
  }
}

size_t bdl_march_smem_bytes(int dtype) {
  return dtype == kF32 ? (kBdlStages * kBdlRows * kBdlWin + 2 * bdl_out_slot_elems<float>()) * sizeof(float)
                       : (kBdlStages * kBdlRows * kBdlWin + 2 * bdl_out_slot_elems<__half>()) * 2;
}

cudaError_t launch_bdl_march(const BdlArgs& a, const CUtensorMap* imap, const CUtensorMap* omap, int dtype,
                             int steps, int causal, int backward, unsigned grid, cudaStream_t st) {
  const void* kern = bdl_march_ptr(dtype, steps, causal, bdl_mode(a, backward));
  if (kern == nullptr) return cudaErrorInvalidValue;
  const size_t smem = bdl_march_smem_bytes(dtype);
  void* args[] = {const_cast<CUtensorMap*>(imap), const_cast<CUtensorMap*>(omap), const_cast<BdlArgs*>(&a)};
  return cudaLaunchKernel(kern, dim3(grid), dim3(32), args, smem, st);
}

int bdl_march_ctas_per_sm(int dtype, int steps, int causal, int backward, int contract) {
  const void* kern = bdl_march_ptr(dtype, steps, causal, backward ? 1 : (contract ? 2 : 0));
  if (kern == nullptr) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 32, bdl_march_smem_bytes(dtype)) != cudaSuccess)
    return -1;
  return n;
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
