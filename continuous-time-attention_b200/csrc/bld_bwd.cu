// Fused backward of the multi-step diffusion stencil on [B, L, D] hidden
// states; see bld_fwd.cu for the work decomposition shared with the forward.
#include "bld_common.cuh"

namespace cta {

__device__ int g_bld_bwd_error;

// ===========================================================================
// backward: grad_in = (A_1^T ... A_S^T) grad_out, optionally d(alpha_k)
//
// One step maps u -> u' with u'[i] = u[i] + alpha * lap(u)[i] on updated rows.
// Its adjoint, with a[i] = alpha * g'[i] on updated rows and 0 on fixed rows:
//   non-causal:  g[j] = g'[j] + (a[j+1] - 2 a[j]) + a[j-1]
//   causal:      g[j] = g'[j] + (a[j] - 2 a[j+1]) + a[j+2]      (anti-causal)
// which is kernels/diffusion_triton.py:116-131 generalised to masks/causality.
// d(alpha_k) = sum over updated rows of g_k[j] * lap(u_{k-1})[j]; the forward
// levels u_{k-1} are recomputed from x in the same march, and the two
// wavefronts (which reach a given row at different march steps) are paired
// through short register delay lines.
// ===========================================================================
template <int S, bool CAUSAL, bool DALPHA>
struct BwdGeom {
  // rows of the g stream above the output tile
  static constexpr int HLG = CAUSAL ? (DALPHA ? S + 1 : 0) : S;
  // rows of the x stream above the output tile
  static constexpr int HLX = CAUSAL ? 2 * S : S;
  // march rows before the first output row
  static constexpr int LAG = CAUSAL ? (DALPHA ? 3 * S + 1 : 2 * S) : 2 * S;
  // for d(alpha_k) (k = 1..S): delay of the early stream and pairing offset
  __host__ __device__ static constexpr int delay(int k) {
    return CAUSAL ? (2 * k - S - 1 >= 0 ? 2 * k - S - 1 : S + 1 - 2 * k) : (2 * k - S >= 0 ? 2 * k - S : S - 2 * k);
  }
  // true when g_k arrives before lap(u_{k-1}) and must be delayed
  __host__ __device__ static constexpr bool delay_g(int k) { return CAUSAL ? (2 * k > S + 1) : (2 * k > S); }
  // paired row = l0 + t - pair_off(k)
  __host__ __device__ static constexpr int pair_off(int k) {
    return CAUSAL ? (2 * S > 3 * S + 1 - 2 * k ? 2 * S : 3 * S + 1 - 2 * k) : (S + (k > S - k ? k : S - k));
  }
};

template <typename T, int S, bool CAUSAL, bool DALPHA>
__global__ void __launch_bounds__(kBldThreads) bld_bwd_kernel(const __grid_constant__ CUtensorMap gmap,
                                                              const __grid_constant__ CUtensorMap xmap,
                                                              const BldArgs a) {
  using E = Elem<T>;
  using P = typename E::Pair;
  using G = BwdGeom<S, CAUSAL, DALPHA>;
  constexpr int PAIRS = kBldDT / 2;
  constexpr int NST = (DALPHA && sizeof(T) == 4) ? 2 : kBldStages;
  constexpr int CHUNK = kBldRC * kBldDT;
  constexpr int DMAX = S + 1;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* gring = reinterpret_cast<T*>(smem_raw);
  T* xring = gring + NST * CHUNK;
  __shared__ __align__(8) uint64_t full_bar[kBldStages];
  __shared__ uint32_t fbits[kBldMaxWords + 2];
  __shared__ uint32_t zbits[kBldMaxWords + 2];
  __shared__ float red[kBldThreads / 32][kMaxSteps];
  __shared__ bool s_last;

  const Seg sg = resolve_seg(a, blockIdx.z);
  const int64_t l0 = a.out_begin + static_cast<int64_t>(blockIdx.x) * a.TL;
  const int64_t oend = a.out_end < sg.n ? a.out_end : sg.n;
  const int tid = threadIdx.x;
  const int cta_id = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const bool active = l0 < oend;
  // inactive CTAs still take part in the d(alpha) completion count
  if (!active && !DALPHA) return;

  const int d0 = blockIdx.y * kBldDT;
  const int64_t jbg = l0 - G::HLG;
  const int64_t jbx = l0 - G::HLX;
  const int nout = active ? static_cast<int>(oend - l0 < a.TL ? oend - l0 : a.TL) : 0;
  const int nrows = nout + G::LAG;
  const int nch = active ? (nrows + kBldRC - 1) / kBldRC : 0;
  const bool use_tma = a.use_tma != 0;

  float2 acc[S];
#pragma unroll
  for (int k = 0; k < S; ++k) acc[k] = f2(0.f);

  if (active) {
    if (tid == 0) {
      if (use_tma) {
        prefetch_tmap(&gmap);
        if (DALPHA) prefetch_tmap(&xmap);
      }
#pragma unroll
      for (int s = 0; s < kBldStages; ++s) mbar_init(&full_bar[s], 1);
      fence_mbar_init();
    }
    // bitmap covers rows of both streams
    const int64_t jbits = (jbg < jbx ? jbg : jbx);
    const int64_t span = (jbg > jbx ? jbg - jbx : jbx - jbg) + nch * kBldRC;
    RowBits rb{fbits, zbits, jbits};
    const bool slow = build_row_bits<CAUSAL>(a, sg, rb, static_cast<int>((span + 31) / 32));

    auto issue = [&](int c) {
      const int slot = c % NST;
      mbar_arrive_expect_tx(&full_bar[slot], (DALPHA ? 2 : 1) * CHUNK * sizeof(T));
      tma_load_3d(gring + slot * CHUNK, &gmap, &full_bar[slot], d0, static_cast<int>(sg.row0 + jbg + c * kBldRC),
                  sg.bcoord);
      if (DALPHA)
        tma_load_3d(xring + slot * CHUNK, &xmap, &full_bar[slot], d0, static_cast<int>(sg.row0 + jbx + c * kBldRC),
                    sg.bcoord);
    };
    if (use_tma && tid == 0) {
      for (int c = 0; c < nch && c < NST; ++c) issue(c);
    }

    float alf[kMaxSteps];
    load_alphas(a, alf, S);
    float2 al[S];
#pragma unroll
    for (int k = 0; k < S; ++k) al[k] = f2(alf[k]);
    // rounded products as fma with a run-time -0 addend: exactly the forward's rounding
    const float2 zn2 = f2(a.neg_zero);

    // adjoint state per level m (step k = S - m)
    float2 A1[S], A2[S], G1[S], G2[S];
    // forward state (d(alpha) only): levels q = 0..S-1
    float2 F1[S], F2[S];
    // delay lines for d(alpha): DL[k-1][0..delay(k)-1]
    float2 DL[S][DMAX];
#pragma unroll
    for (int k = 0; k < S; ++k) {
      A1[k] = A2[k] = G1[k] = G2[k] = F1[k] = F2[k] = f2(0.f);
#pragma unroll
      for (int d = 0; d < DMAX; ++d) DL[k][d] = f2(0.f);
    }

    const int col = d0 + 2 * tid;
    const bool col_ok = col < a.D;
    const bool pair_ok = (col + 1 < a.D) && ((a.ysB | a.ysL) % 2 == 0) &&
                         (reinterpret_cast<uintptr_t>(a.y) % sizeof(P) == 0);
    T* ybase = static_cast<T*>(a.y) + static_cast<int64_t>(sg.bcoord) * a.ysB;

    int err = 0;
    for (int c = 0; c < nch; ++c) {
      const int slot = c % NST;
      T* gbuf = gring + slot * CHUNK;
      T* xbuf = xring + slot * CHUNK;
      if (use_tma) {
        if (!mbar_wait_bounded(&full_bar[slot], (c / NST) & 1)) err = 1;
      } else {
        fill_chunk_generic<T>(a, a.g, a.gsB, a.gsL, sg, jbg + c * kBldRC, d0, gbuf);
        if (DALPHA) fill_chunk_generic<T>(a, a.x, a.xsB, a.xsL, sg, jbx + c * kBldRC, d0, xbuf);
        __syncthreads();
      }
      if (!err) {
        const P* gp = reinterpret_cast<const P*>(gbuf) + tid;
        const P* xp = reinterpret_cast<const P*>(xbuf) + tid;
        auto march = [&](auto slow_tag) {
          constexpr bool SLOW = decltype(slow_tag)::value;
#pragma unroll
          for (int i = 0; i < kBldRC; ++i) {
            const int t = c * kBldRC + i;
            const int64_t jg = jbg + t;  // row of the g value entering level 0
            // ---------------- forward recomputation (d(alpha) only) -------------
            float2 lapv[S];
            if (DALPHA) {
              const int64_t jx = jbx + t;
              float2 xc = E::unpack(xp[i * PAIRS]);
              if (SLOW) {
                if (rb.zero(jx)) xc = f2(0.f);
              }
              if (CAUSAL) {
                const bool fx = SLOW && rb.fixed(jx);
#pragma unroll
                for (int q = 0; q < S; ++q) {
                  const float2 lp = lap3(F2[q], F1[q], xc);  // lap_c(u_q)[jx]
                  lapv[q] = lp;
                  float2 un = add2(xc, fma2(al[q], lp, zn2));
                  if (SLOW) un = sel2(fx, xc, un);
                  F2[q] = F1[q];
                  F1[q] = xc;
                  xc = un;
                }
              } else {
                const uint32_t fw = SLOW ? rb.window8_fixed(jx - S) : 0u;
#pragma unroll
                for (int q = 0; q < S; ++q) {
                  const float2 lp = lap3(F2[q], F1[q], xc);  // lap(u_q)[jx - q - 1]
                  lapv[q] = lp;
                  float2 un = add2(F1[q], fma2(al[q], lp, zn2));
                  if (SLOW) un = sel2((fw >> (S - 1 - q)) & 1u, F1[q], un);
                  F2[q] = F1[q];
                  F1[q] = xc;
                  xc = un;
                }
              }
            }
            // ---------------- adjoint march ----------------
            float2 cur_g = E::unpack(gp[i * PAIRS]);
            if (SLOW) {
              if (rb.zero(jg)) cur_g = f2(0.f);
            }
            float2 cur_a = mul2(al[S - 1], cur_g);
            if (SLOW) cur_a = sel2(rb.fixed(jg), f2(0.f), cur_a);
            uint32_t fwg = 0u;
            if (SLOW && !CAUSAL) fwg = rb.window8_fixed(jg - S);
#pragma unroll
            for (int m = 0; m < S; ++m) {
              const int k = S - m;  // step whose adjoint this level applies
              // d(alpha_k): pair g_k with lap(u_{k-1})
              if (DALPHA) {
                const int dl = G::delay(k);
                float2 gk = cur_g, lk = lapv[k - 1];
                if (dl > 0) {
                  if (G::delay_g(k)) {
                    const float2 old = DL[k - 1][dl - 1];
#pragma unroll
                    for (int d = DMAX - 1; d > 0; --d)
                      if (d < dl) DL[k - 1][d] = DL[k - 1][d - 1];
                    DL[k - 1][0] = gk;
                    gk = old;
                  } else {
                    const float2 old = DL[k - 1][dl - 1];
#pragma unroll
                    for (int d = DMAX - 1; d > 0; --d)
                      if (d < dl) DL[k - 1][d] = DL[k - 1][d - 1];
                    DL[k - 1][0] = lk;
                    lk = old;
                  }
                }
                const int rel = t - G::pair_off(k);  // paired row - l0
                bool take = rel >= 0 && rel < nout;
                if (SLOW) take = take && !rb.fixed(l0 + rel);
                if (take) acc[k - 1] = fma2(gk, lk, acc[k - 1]);
              }
              float2 gn;
              if (CAUSAL) {
                gn = add2(G2[m], lap3(cur_a, A1[m], A2[m]));
                A2[m] = A1[m];
                A1[m] = cur_a;
                G2[m] = G1[m];
                G1[m] = cur_g;
              } else {
                gn = add2(G1[m], lap3(A2[m], A1[m], cur_a));
                A2[m] = A1[m];
                A1[m] = cur_a;
                G1[m] = cur_g;
              }
              cur_g = gn;
              if (m < S - 1) {
                cur_a = mul2(al[S - 2 - m], gn);
                if (SLOW) {
                  const bool fx = CAUSAL ? rb.fixed(jg - 2 * m - 2) : ((fwg >> (S - 1 - m)) & 1u);
                  cur_a = sel2(fx, f2(0.f), cur_a);
                }
              }
            }
            const int64_t orow = l0 + t - G::LAG;
            if (t >= G::LAG && orow < oend && col_ok) {
              const int64_t tr = sg.row0 + orow;
              if (tr >= 0 && tr < a.L) store_pair<T>(ybase + tr * a.ysL, col, a, cur_g, pair_ok);
            }
          }
        };
        if (slow) march(std::true_type{});
        else march(std::false_type{});
      }
      if (__syncthreads_or(err)) {
        if (tid == 0) {
          atomicExch(&g_bld_bwd_error, kDevTimeout);
          // drain (bounded) every load still in flight before leaving the pipeline
          if (use_tma)
            for (int cc = c; cc < nch && cc < c + NST; ++cc) mbar_wait_bounded(&full_bar[cc % NST], (cc / NST) & 1);
        }
        __syncthreads();
        if (!DALPHA) return;
        // keep the d(alpha) completion protocol consistent: contribute zeros
#pragma unroll
        for (int k = 0; k < S; ++k) acc[k] = f2(0.f);
        break;
      }
      if (use_tma && tid == 0 && c + NST < nch) issue(c + NST);
    }
    if (!col_ok) {
#pragma unroll
      for (int k = 0; k < S; ++k) acc[k] = f2(0.f);
    }
  }

  if (DALPHA) {
    // deterministic reduction: thread -> warp (shuffle tree) -> CTA (fixed
    // order) -> partial[cta]; the last CTA to finish sums the partials in
    // CTA order in double precision.
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int k = 0; k < S; ++k) {
      float v = acc[k].x + acc[k].y;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp][k] = v;
    }
    __syncthreads();
    if (tid < S) {
      float v = 0.f;
      for (int w = 0; w < kBldThreads / 32; ++w) v += red[w][tid];
      a.dalpha_partial[static_cast<int64_t>(cta_id) * S + tid] = v;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned int done = atomicAdd(a.counter, 1u);
      s_last = (done == static_cast<unsigned int>(a.num_ctas) - 1u);
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      if (tid < S) {
        double s = 0.0;
        for (int b = 0; b < a.num_ctas; ++b)
          s += static_cast<double>(__ldcg(a.dalpha_partial + static_cast<int64_t>(b) * S + tid));
        a.dalpha[tid] = static_cast<float>(s);
      }
      if (tid == 0) *a.counter = 0u;
    }
  }
}

// ===========================================================================
// host-side dispatch
// ===========================================================================
size_t bld_smem_bytes(int dtype, int with_x_stream) {
  const size_t es = dtype == kF32 ? 4 : 2;
  const int nst = (with_x_stream && es == 4) ? 2 : kBldStages;
  return static_cast<size_t>(with_x_stream ? 2 : 1) * nst * kBldRC * kBldDT * es;
}


namespace {

template <typename T, int S, bool CAUSAL, bool DA>
cudaError_t launch_bwd_t(const BldArgs& a, const CUtensorMap* gmap, const CUtensorMap* xmap, dim3 grid, size_t smem,
                         cudaStream_t st) {
  auto kern = bld_bwd_kernel<T, S, CAUSAL, DA>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kBldThreads, smem, st>>>(*gmap, *xmap, a);
  return cudaGetLastError();
}


template <typename T, bool CAUSAL, bool DA>
cudaError_t bwd_steps(const BldArgs& a, const CUtensorMap* gm, const CUtensorMap* xm, int steps, dim3 g, size_t sm,
                      cudaStream_t st) {
  switch (steps) {
    case 1: return launch_bwd_t<T, 1, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 2: return launch_bwd_t<T, 2, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 3: return launch_bwd_t<T, 3, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 4: return launch_bwd_t<T, 4, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 5: return launch_bwd_t<T, 5, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 6: return launch_bwd_t<T, 6, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 7: return launch_bwd_t<T, 7, CAUSAL, DA>(a, gm, xm, g, sm, st);
    case 8: return launch_bwd_t<T, 8, CAUSAL, DA>(a, gm, xm, g, sm, st);
    default: return cudaErrorInvalidValue;
  }
}


template <typename T>
cudaError_t bwd_dtype(const BldArgs& a, const CUtensorMap* gm, const CUtensorMap* xm, int steps, int causal, int da,
                      dim3 g, size_t sm, cudaStream_t st) {
  if (causal)
    return da ? bwd_steps<T, true, true>(a, gm, xm, steps, g, sm, st)
              : bwd_steps<T, true, false>(a, gm, xm, steps, g, sm, st);
  return da ? bwd_steps<T, false, true>(a, gm, xm, steps, g, sm, st)
            : bwd_steps<T, false, false>(a, gm, xm, steps, g, sm, st);
}


}  // namespace

cudaError_t launch_bld_bwd(const BldArgs& a, const CUtensorMap* gmap, const CUtensorMap* xmap, int dtype, int steps,
                           int causal, int with_dalpha, dim3 grid, size_t smem, cudaStream_t st) {
  switch (dtype) {
    case kF32: return bwd_dtype<float>(a, gmap, xmap, steps, causal, with_dalpha, grid, smem, st);
    case kBF16: return bwd_dtype<__nv_bfloat16>(a, gmap, xmap, steps, causal, with_dalpha, grid, smem, st);
    case kF16: return bwd_dtype<__half>(a, gmap, xmap, steps, causal, with_dalpha, grid, smem, st);
    default: return cudaErrorInvalidValue;
  }
}


int read_device_error_bld_bwd(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bld_bwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bld_bwd_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace cta
