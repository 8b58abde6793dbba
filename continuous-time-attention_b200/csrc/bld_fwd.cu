// Fused multi-step diffusion stencil on [B, L, D] hidden states (feature axis
// contiguous) -- forward, backward (A^T applied `steps` times) and backward
// with the per-step d(alpha) reduction, all in one launch per call.
//
// Reference semantics followed here:
//   * one step, copy boundary:      src/cta/ops/diffusion.py:17-56
//   * steps fused, fp32 in between: src/cta/ops/diffusion.py:59-77,
//                                   src/cta/serving_vllm.py:29-46 ([B,L,D])
//   * causal stencil, attention mask, per-layer alpha:
//                                   src/models/pde_layers.py:39-64,113-188,218-219
//   * adjoint of one step:          kernels/diffusion_triton.py:96-133
//   * zero-padded packed prefill:   src/cta/serving_vllm.py:72-111,275-303
//
// Work decomposition.  A CTA owns an output tile of TL rows x 256 columns.
// Its 128 threads each own two adjacent columns (one float2) and *march* down
// the rows of the tile plus a halo: every arriving input row advances all
// `steps` time levels by one row (a wavefront, level k lags k rows, or 0 rows
// for the causal stencil), so each thread keeps only two rows of state per
// level in registers and every intermediate level stays on chip.  Input rows
// arrive in shared memory through a ring of TMA tile loads (16 rows x 256
// columns per chunk, 4 chunks in flight, one mbarrier per slot); the output is
// written once, straight from registers.  HBM traffic is therefore one read of
// the input (the halo rows are re-read from L2 by the neighbouring tile) and
// one write of the output.
//
// Rows that must not change -- the copy boundary, rows whose 3-row stencil
// touches a masked position, per-sequence boundaries of packed prefill -- are
// "fixed" rows.  They are collected per tile into a bitmap; tiles without any
// fixed row run a branch-free march, the others test the bitmap per level.
#include "bld_common.cuh"

namespace cta {

__device__ int g_bld_fwd_error;

// ===========================================================================
// forward
// ===========================================================================
template <typename T, int S, bool CAUSAL>
__global__ void __launch_bounds__(kBldThreads) bld_fwd_kernel(const __grid_constant__ CUtensorMap xmap,
                                                              const BldArgs a) {
  using E = Elem<T>;
  using P = typename E::Pair;
  constexpr int HL = CAUSAL ? 2 * S : S;  // halo rows above the tile
  constexpr int LAG = 2 * S;              // march rows before the first output row
  constexpr int PAIRS = kBldDT / 2;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  __shared__ __align__(8) uint64_t full_bar[kBldStages];
  __shared__ uint32_t fbits[kBldMaxWords + 2];
  __shared__ uint32_t zbits[kBldMaxWords + 2];

  const Seg sg = resolve_seg(a, blockIdx.z);
  const int64_t l0 = a.out_begin + static_cast<int64_t>(blockIdx.x) * a.TL;
  const int64_t oend = a.out_end < sg.n ? a.out_end : sg.n;
  if (l0 >= oend) return;
  const int d0 = blockIdx.y * kBldDT;
  const int64_t jb = l0 - HL;
  const int nout = static_cast<int>(oend - l0 < a.TL ? oend - l0 : a.TL);
  const int nrows = nout + LAG;
  const int nch = (nrows + kBldRC - 1) / kBldRC;
  const int tid = threadIdx.x;
  const bool use_tma = a.use_tma != 0;

  if (tid == 0) {
    if (use_tma) prefetch_tmap(&xmap);
#pragma unroll
    for (int s = 0; s < kBldStages; ++s) mbar_init(&full_bar[s], 1);
    fence_mbar_init();
  }
  RowBits rb{fbits, zbits, jb};
  const bool slow = build_row_bits<CAUSAL>(a, sg, rb, (nch * kBldRC + 31) / 32);

  auto issue = [&](int c) {
    const int slot = c % kBldStages;
    mbar_arrive_expect_tx(&full_bar[slot], kBldRC * kBldDT * sizeof(T));
    tma_load_3d(ring + slot * kBldRC * kBldDT, &xmap, &full_bar[slot], d0,
                static_cast<int>(sg.row0 + jb + c * kBldRC), sg.bcoord);
  };
  if (use_tma && tid == 0) {
    for (int c = 0; c < nch && c < kBldStages; ++c) issue(c);
  }

  float alf[kMaxSteps];
  load_alphas(a, alf, S);
  float2 al[S];
#pragma unroll
  for (int k = 0; k < S; ++k) al[k] = f2(alf[k]);

  float2 P1[S], P2[S];
#pragma unroll
  for (int k = 0; k < S; ++k) P1[k] = P2[k] = f2(0.f);

  const int col = d0 + 2 * tid;
  const bool col_ok = col < a.D;
  const bool pair_ok = a.y != nullptr && (col + 1 < a.D) && ((a.ysB | a.ysL) % 2 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.y) % sizeof(P) == 0);
  T* ybase = static_cast<T*>(a.y) + static_cast<int64_t>(sg.bcoord) * a.ysB;

  int err = 0;
  for (int c = 0; c < nch; ++c) {
    const int slot = c % kBldStages;
    T* buf = ring + slot * kBldRC * kBldDT;
    if (use_tma) {
      if (!mbar_wait_bounded(&full_bar[slot], (c / kBldStages) & 1)) err = 1;
    } else {
      fill_chunk_generic<T>(a, a.x, a.xsB, a.xsL, sg, jb + c * kBldRC, d0, buf);
      __syncthreads();
    }
    if (!err) {
      const P* rp = reinterpret_cast<const P*>(buf) + tid;
      auto march = [&](auto slow_tag) {
        constexpr bool SLOW = decltype(slow_tag)::value;
#pragma unroll
        for (int i = 0; i < kBldRC; ++i) {
          const int t = c * kBldRC + i;
          const int64_t j = jb + t;
          float2 cur = E::unpack(rp[i * PAIRS]);
          if (SLOW) {
            if (rb.zero(j)) cur = f2(0.f);
          }
          if (CAUSAL) {
            const bool fx = SLOW && rb.fixed(j);
#pragma unroll
            for (int k = 0; k < S; ++k) {
              float2 nx = stencil_c(P2[k], P1[k], cur, al[k]);
              if (SLOW) nx = sel2(fx, cur, nx);
              P2[k] = P1[k];
              P1[k] = cur;
              cur = nx;
            }
          } else {
            // level k updates row j-1-k; bit (S-1-k) of the window of rows j-S .. j-1
            const uint32_t fw = SLOW ? rb.window8_fixed(j - S) : 0u;
#pragma unroll
            for (int k = 0; k < S; ++k) {
              float2 nx = stencil_nc(P2[k], P1[k], cur, al[k]);
              if (SLOW) nx = sel2((fw >> (S - 1 - k)) & 1u, P1[k], nx);
              P2[k] = P1[k];
              P1[k] = cur;
              cur = nx;
            }
          }
          const int64_t orow = l0 + t - LAG;
          if (t >= LAG && orow < oend && col_ok) {
            const int64_t tr = sg.row0 + orow;
            if (tr >= 0 && tr < a.L) store_pair<T>(ybase + tr * a.ysL, col, a, cur, pair_ok);
          }
        }
      };
      if (slow) march(std::true_type{});
      else march(std::false_type{});
    }
    if (__syncthreads_or(err)) {
      if (tid == 0) {
        atomicExch(&g_bld_fwd_error, kDevTimeout);
        // drain (bounded) every load still in flight before the CTA exits
        if (use_tma)
          for (int cc = c; cc < nch && cc < c + kBldStages; ++cc)
            mbar_wait_bounded(&full_bar[cc % kBldStages], (cc / kBldStages) & 1);
      }
      __syncthreads();
      return;
    }
    if (use_tma && tid == 0 && c + kBldStages < nch) issue(c + kBldStages);
  }
}


namespace {

template <typename T, int S, bool CAUSAL>
cudaError_t launch_fwd_t(const BldArgs& a, const CUtensorMap* xmap, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = bld_fwd_kernel<T, S, CAUSAL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  kern<<<grid, kBldThreads, smem, st>>>(*xmap, a);
  return cudaGetLastError();
}


template <typename T, bool CAUSAL>
cudaError_t fwd_steps(const BldArgs& a, const CUtensorMap* m, int steps, dim3 g, size_t sm, cudaStream_t st) {
  switch (steps) {
    case 1: return launch_fwd_t<T, 1, CAUSAL>(a, m, g, sm, st);
    case 2: return launch_fwd_t<T, 2, CAUSAL>(a, m, g, sm, st);
    case 3: return launch_fwd_t<T, 3, CAUSAL>(a, m, g, sm, st);
    case 4: return launch_fwd_t<T, 4, CAUSAL>(a, m, g, sm, st);
    case 5: return launch_fwd_t<T, 5, CAUSAL>(a, m, g, sm, st);
    case 6: return launch_fwd_t<T, 6, CAUSAL>(a, m, g, sm, st);
    case 7: return launch_fwd_t<T, 7, CAUSAL>(a, m, g, sm, st);
    case 8: return launch_fwd_t<T, 8, CAUSAL>(a, m, g, sm, st);
    default: return cudaErrorInvalidValue;
  }
}


template <typename T>
cudaError_t fwd_dtype(const BldArgs& a, const CUtensorMap* m, int steps, int causal, dim3 g, size_t sm,
                      cudaStream_t st) {
  return causal ? fwd_steps<T, true>(a, m, steps, g, sm, st) : fwd_steps<T, false>(a, m, steps, g, sm, st);
}


}  // namespace

cudaError_t launch_bld_fwd(const BldArgs& a, const CUtensorMap* xmap, int dtype, int steps, int causal, dim3 grid,
                           size_t smem, cudaStream_t st) {
  switch (dtype) {
    case kF32: return fwd_dtype<float>(a, xmap, steps, causal, grid, smem, st);
    case kBF16: return fwd_dtype<__nv_bfloat16>(a, xmap, steps, causal, grid, smem, st);
    case kF16: return fwd_dtype<__half>(a, xmap, steps, causal, grid, smem, st);
    default: return cudaErrorInvalidValue;
  }
}


int read_device_error_bld_fwd(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bld_fwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bld_fwd_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace cta
