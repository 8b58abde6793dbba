// Fused multi-step diffusion stencil on [B, L, D] hidden states (feature axis
// contiguous) -- forward, all `steps` steps in one launch.  The kernel
// templates; bld_fwd_<dtype>[_fm].cu instantiate them per dtype and
// arithmetic, bld_fwd.cu holds the host side.
//
// Reference semantics followed here:
//   * one step, copy boundary:      src/cta/ops/diffusion.py:17-56
//   * steps fused, fp32 in between: src/cta/ops/diffusion.py:59-77,
//                                   src/cta/serving_vllm.py:29-46 ([B,L,D])
//   * causal stencil, attention mask, per-layer alpha:
//                                   src/models/pde_layers.py:39-64,113-188,218-219
//   * zero-padded packed prefill:   src/cta/serving_vllm.py:72-111,275-303
//
// Work decomposition.  A CTA is ONE warp with its own pipeline, owning an
// output tile of TL rows x 128 columns; no CTA-wide barrier exists.  Each
// lane owns four adjacent columns (two packed fp32 pairs) and *marches* down
// the rows of the tile plus a halo: every arriving input row advances all
// `steps` time levels by one row (a wavefront: level k lags k rows, or 0 rows
// for the causal stencil), so a lane keeps two rows of state per level in
// registers and every intermediate level stays on chip.  Input rows arrive in
// shared memory through a ring of TMA tile loads (8 rows x 128 columns per
// chunk, 3 chunks in flight, one mbarrier per slot); finished rows are staged
// in shared memory and leave through TMA tile stores, 8 rows at a time.  HBM
// traffic is one read of the input (halo rows are re-read from L2 by the
// neighbouring tile) and one write of the output.
//
// Rows that must not change -- the copy boundary, rows whose 3-row stencil
// touches a masked position, per-sequence boundaries of packed prefill -- are
// "fixed" rows.  They are collected per tile into a bitmap; tiles without any
// fixed row run a branch-free march.  In the others each full chunk takes one
// of three forms from the bits its rows test: branch-free (none set), per-row
// tests, or all-fixed (every tested row fixed: the tests fold to constants).
#pragma once

#include "bld_common.cuh"

namespace cta {

// Each translation unit that instantiates these kernels has its own error word
// (no relocatable device code); the host reads every unit's word.
static __device__ int g_bld_fwd_error;

namespace {

// Plain-load fill of one forward chunk ([RC][128]), for tensors TMA cannot
// address and for shard edges that read neighbour halos.
template <typename T>
__device__ void fill_fwd_chunk(const BldArgs& a, const Seg& s, int64_t jrow0, int d0, T* dst) {
  const T zero = Elem<T>::from_f(0.f);
  for (int idx = threadIdx.x; idx < kFwdRC * kFwdDT; idx += kFwdThreads) {
    const int i = idx / kFwdDT;
    const int cc = idx - i * kFwdDT;
    const int64_t tr = s.row0 + jrow0 + i;
    const int col = d0 + cc;
    const T* rowp = nullptr;
    if (tr >= 0 && tr < a.L) {
      rowp = static_cast<const T*>(a.x) + static_cast<int64_t>(s.bcoord) * a.xsB + tr * a.xsL;
    } else if (tr < 0 && a.lo_ext != nullptr && tr >= -a.hext_lo) {
      rowp = static_cast<const T*>(a.lo_ext) + (static_cast<int64_t>(s.bcoord) * a.hext_lo + (a.hext_lo + tr)) * a.D;
    } else if (tr >= a.L && a.hi_ext != nullptr && tr - a.L < a.hext_hi) {
      rowp = static_cast<const T*>(a.hi_ext) + (static_cast<int64_t>(s.bcoord) * a.hext_hi + (tr - a.L)) * a.D;
    }
    dst[i * kFwdDT + cc] = (rowp != nullptr && col < a.D) ? rowp[col] : zero;
  }
}

}  // namespace

// ADJ = false: forward, x -> y.  ADJ = true: the adjoint of the same `steps`
// steps applied to a gradient, g -> dx (without d(alpha)); it shares the whole
// pipeline, only the per-row update and the halo side differ.
//
// Register budget.  A variant keeps, per lane and level, two rows of state for
// each of its two column pairs (the adjoint also one or two rows of g), so its
// register need grows with `steps`, and fastest for the causal adjoint.  The
// minimum resident CTAs per SM handed to __launch_bounds__ is the largest of
// 16/12/8 (4/3/2 warps per SM sub-partition, whose register file holds 16384
// registers) at which ptxas compiles the variant without spilling, checked with
// -Xptxas -v for every variant (only the 16-bit steps-8 forward and causal
// adjoint keep a few bytes of spill at 168 and 255 registers); the host sizes
// the grid from the occupancy the variant really gets (bld_march_ctas_per_sm).
template <typename T, int S, bool CAUSAL, bool ADJ, bool RES = false>
constexpr int march_min_ctas() {
  constexpr bool F32 = sizeof(T) == 4;
  if (!ADJ) return S <= 4 ? kFwdMinCtas : (S == 5 || (S == 6 && F32 && !RES)) ? 16 : 12;
  if (!CAUSAL) return S <= 3 ? kFwdMinCtas : S <= 5 ? 16 : (S == 8 && F32) ? 8 : 12;
  return S <= 3 ? (kFwdMinCtas < 16 ? kFwdMinCtas : 16) : S <= 5 ? 12 : 8;
}

// The per-pair update of one level.  KIND 0: the diffusion step (pst_c /
// pst_nc).  KIND 1 / 2 (steps 1 only): the advection- / reaction-diffusion
// layer step of src/models/pde_layers.py:276-281, :309-318 in the reference's
// op order: c + (alpha*lap + beta-term), beta-term = beta * (x[i+1] - x[i-1]) / 2
// (causal beta * (x[i] - x[i-1])) or (beta * c) * (1 - sigmoid(c)).
// (p2, p1, x) = rows (i-1, i, i+1) non-causal, (i-2, i-1, i) causal.
__device__ __forceinline__ float fast_sigmoid(float v) { return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-v))); }

template <int KIND, bool CAUSAL, bool FM = false>
__device__ __forceinline__ pf2 level_update(pf2 p2, pf2 p1, pf2 x, pf2 al, pf2 be, float be_s, pf2 m2, pf2 zn) {
  if constexpr (KIND == 0) {
    return CAUSAL ? pst_c<FM>(p2, p1, x, al, m2, zn) : pst_nc<FM>(p2, p1, x, al, m2, zn);
  } else {
    const pf2 lap = plap(p2, p1, x, m2);
    const pf2 c = CAUSAL ? x : p1;
    pf2 bterm;
    if constexpr (KIND == 1) {
      const pf2 n1 = pbc(-1.f), half = pbc(0.5f);
      const pf2 h = CAUSAL ? pfma(p1, n1, x) : pmul(pfma(p2, n1, x), half);  // x[i]-x[i-1] | (x[i+1]-x[i-1])/2
      bterm = pmul_sep(be, h, zn);
    } else {
      float c0, c1;
      upk(c, c0, c1);
      const float t0 = __fmul_rn(__fmul_rn(be_s, c0), __fsub_rn(1.0f, fast_sigmoid(c0)));
      const float t1 = __fmul_rn(__fmul_rn(be_s, c1), __fsub_rn(1.0f, fast_sigmoid(c1)));
      bterm = pk(t0, t1);
    }
    return padd(c, padd(pmul_sep(al, lap, zn), bterm));
  }
}

// RES (non-causal forward only): y = residual + stencil(x) in the same pass.
// The residual rows of each full output chunk are brought by a TMA load into
// the staging slot that chunk is about to use, issued one chunk ahead; the
// lanes add them in place and the TMA store sends the sum out.
// POOL (non-causal forward, masked): the classifier's masked mean pool
// (src/models/transformers.py:135-139) fused into the last refinement: the
// output rows are not stored; each lane sums mask[row] * y[row] (y rounded to
// T, as the stored tensor would hold it) over its rows, and the CTA writes its
// column sums to a.pool_partial[(batch * row tiles + row tile) * D + col], for
// pool_finish_kernel to reduce in a fixed order.
// FM: the contracted update (pst_nc / pst_c), forward diffusion only.
template <typename T, int S, bool CAUSAL, bool ADJ, bool RES, int KIND = 0, bool POOL = false, bool FM = false>
__global__ void __launch_bounds__(kFwdThreads, (march_min_ctas<T, S, CAUSAL, ADJ, RES>()))
    bld_march_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const __grid_constant__ CUtensorMap rmap, const BldArgs a) {
  static_assert(!FM || (KIND == 0 && !POOL), "the contracted update is the diffusion forward / adjoint");
  static_assert(!POOL || (!ADJ && !RES && KIND == 0 && !CAUSAL), "the pooled form is the non-causal forward");
  static_assert(!RES || (!ADJ && !CAUSAL), "the residual form is the non-causal forward");
  static_assert(KIND == 0 || (S <= kPdeMaxSteps && !ADJ && !RES), "the other PDE kinds: forward stacks of up to 4 steps");
  constexpr int PKIND = KIND;  // the update kind, as named inside the chunk lambdas
  // every global read (cu_seqlens, mask, alphas, the streams) comes after the wait
  pdl_launch_dependents();
  pdl_wait();
  using Q = ColVec<T, kFwdVec>;
  using V = typename Q::V;
  // halo rows above the tile: the causal forward reads 2S rows back, its
  // adjoint (anti-causal) only reads forward
  constexpr int HL = ADJ ? (CAUSAL ? 0 : S) : (CAUSAL ? 2 * S : S);
  constexpr int LAG = 2 * S;              // wavefront depth: march rows before the first finished row
  // extra leading rows so that output rows start on a chunk boundary
  constexpr int PAD = (kFwdRC - LAG % kFwdRC) % kFwdRC;
  constexpr int PRO = PAD + LAG;  // prologue rows (no output), a multiple of kFwdRC
  constexpr int NPRO = PRO / kFwdRC;
  constexpr int CHUNK = kFwdRC * kFwdDT;  // elements per pipeline slot (one TMA box)
  static_assert(NPRO >= 1 && NPRO <= 2, "prologue spans one or two chunks");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  T* stage = ring + kFwdStages * CHUNK;  // output staging for the TMA stores
  __shared__ __align__(8) uint64_t full_bar[kFwdStages];
  __shared__ __align__(8) uint64_t res_bar[RES ? 2 : 1];
  __shared__ __align__(8) uint64_t stall_bar;  // test hook: a phase nothing completes
  __shared__ uint32_t pbits[POOL ? kBldMaxWords + 2 : 1];  // POOL: mask bits of the march rows
  __shared__ uint32_t fbits[kBldMaxWords + 2];
  __shared__ uint32_t zbits[kBldMaxWords + 2];

  const Seg sg = resolve_seg(a, blockIdx.z);
  // column tile fastest: the CTAs launched together cover whole rows of the same
  // row tile, so each DRAM page is read (and written) by neighbouring CTAs at once
  const int ndt = (a.D + kFwdDT - 1) / kFwdDT;
  const int dtile = static_cast<int>(blockIdx.x % ndt);
  const int64_t l0 = a.out_begin + static_cast<int64_t>(blockIdx.x / ndt) * a.TL;
  const int64_t oend = a.out_end < sg.n ? a.out_end : sg.n;
  if (l0 >= oend) return;
  const int d0 = dtile * kFwdDT;
  const int64_t jb = l0 - HL - PAD;  // first march row
  const int nout = static_cast<int>(oend - l0 < a.TL ? oend - l0 : a.TL);
  const int nrows = PRO + nout;
  const int nch = (nrows + kFwdRC - 1) / kFwdRC;
  const int nfull_end = nrows / kFwdRC;  // chunks [NPRO, nfull_end) are full
  const int tid = threadIdx.x;
  const bool use_tma = a.use_tma != 0;
  const bool tstore = a.use_tma_store != 0;

  if (tid == 0) {
    if (use_tma) prefetch_tmap(&xmap);
    if (tstore) prefetch_tmap(&ymap);
#pragma unroll
    for (int s = 0; s < kFwdStages; ++s) mbar_init(&full_bar[s], 1);
    if constexpr (RES) {
      prefetch_tmap(&rmap);
      mbar_init(&res_bar[0], 1);
      mbar_init(&res_bar[1], 1);
    }
    if (a.debug_stall_us > 0) mbar_init(&stall_bar, 1);
    fence_mbar_init();
  }
  // full output chunk c's residual rows into its staging slot
  auto issue_res = [&](int c) {
    const int slot = (c - NPRO) & 1;
    mbar_arrive_expect_tx(&res_bar[slot], CHUNK * sizeof(T));
    tma_load_3d(stage + slot * CHUNK, &rmap, &res_bar[slot], d0, static_cast<int>(sg.row0 + l0 + c * kFwdRC - PRO),
                sg.bcoord);
  };
  auto issue = [&](int c) {
    const int slot = c % kFwdStages;
    mbar_arrive_expect_tx(&full_bar[slot], CHUNK * sizeof(T));
    tma_load_3d(ring + slot * CHUNK, &xmap, &full_bar[slot], d0, static_cast<int>(sg.row0 + jb + c * kFwdRC),
                sg.bcoord);
  };
  // the same, executed by the whole warp and issued by lane 0 only
  auto issue_lane0 = [&](int c) {
    const int slot = c % kFwdStages;
    const bool lead = tid == 0;
    mbar_arrive_expect_tx_if(lead, &full_bar[slot], CHUNK * sizeof(T));
    tma_load_3d_if(lead, ring + slot * CHUNK, &xmap, &full_bar[slot], d0,
                   static_cast<int>(sg.row0 + jb + c * kFwdRC), sg.bcoord);
  };
  // the first loads fly while the fixed-row bitmap is built
  if (use_tma && tid == 0) {
    for (int c = 0; c < nch && c < kFwdStages; ++c) issue(c);
  }
  RowBits rb{fbits, zbits, jb};
  const bool slow = build_row_bits<CAUSAL, 1>(a, sg, rb, (nch * kFwdRC + 31) / 32, POOL ? pbits : nullptr);
  if (a.debug_stall_us > 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
    // the timeout path of every pipeline wait, on demand: a bounded wait that
    // runs out, the error word, a bounded drain of the loads in flight, exit
    __syncwarp();
    if (!mbar_wait_bounded_ns(&stall_bar, 0, static_cast<uint64_t>(a.debug_stall_us) * 1000ull)) {
      if (tid == 0) {
        atomicExch(&g_bld_fwd_error, kDevTimeout);
        if (use_tma)
          for (int c = 0; c < nch && c < kFwdStages; ++c) mbar_wait_bounded(&full_bar[c], 0);
      }
      __syncwarp();
      return;
    }
  }
  if constexpr (POOL) {
    // a tile whose output rows are all masked out adds nothing to the pool:
    // zero partials and count, drain the loads already issued, and leave
    uint32_t anyv = 0u;
    for (int r0 = 0; r0 < nout; r0 += 32) {
      const int64_t p = l0 + r0 + tid - jb + 32;
      anyv |= __ballot_sync(0xffffffffu, r0 + tid < nout && ((pbits[p >> 5] >> (p & 31)) & 1u));
    }
    if (anyv == 0u) {
      if (use_tma && tid == 0)
        for (int c = 0; c < nch && c < kFwdStages; ++c)
          if (!mbar_wait_bounded(&full_bar[c], 0)) atomicExch(&g_bld_fwd_error, kDevTimeout);
      const int64_t ntl = gridDim.x / ndt;
      float* pp = a.pool_partial + ((static_cast<int64_t>(sg.bcoord) * ntl + blockIdx.x / ndt) * a.D);
      const int col0 = d0 + tid * kFwdVec;
#pragma unroll
      for (int j = 0; j < kFwdVec; ++j)
        if (col0 + j < a.D) pp[col0 + j] = 0.f;
      if (dtile == 0 && tid == 0)
        a.pool_partial[(static_cast<int64_t>(a.nbatch) * ntl) * a.D + static_cast<int64_t>(sg.bcoord) * ntl +
                       blockIdx.x / ndt] = 0.f;
      __syncwarp();
      return;
    }
  }

  float alf[kMaxSteps];
  load_alphas(a, alf, S);
  pf2 al[S];
#pragma unroll
  for (int k = 0; k < S; ++k) al[k] = pbc(alf[k]);
  const pf2 m2 = pbc(-2.f);
  const pf2 zn = pbc(a.neg_zero);
  // KIND 1/2: beta in coefficient slot 1
  // KIND 1/2: the per-level beta of each layer of the stack (device scalars or host values)
  float bes[S];
  pf2 bev[S];
#pragma unroll
  for (int k = 0; k < S; ++k) {
    bes[k] = KIND == 0 ? 0.f
                       : (a.beta_dev[k] != nullptr ? load_scalar(a.beta_dev[k], a.alpha_dev_dtype) : a.beta[k]);
    bev[k] = pbc(bes[k]);
  }

  // per-level state, for both pairs.  Forward: the level's input on the two
  // previous march rows (P1, P2).  Adjoint: a = alpha*g on the two previous
  // rows (P1, P2) and g on the one (non-causal) or two (causal) previous rows (G1, G2).
  pf2 P1a[S], P2a[S], P1b[S], P2b[S], G1a[S], G1b[S], G2a[S], G2b[S];
#pragma unroll
  for (int k = 0; k < S; ++k) P1a[k] = P2a[k] = P1b[k] = P2b[k] = G1a[k] = G1b[k] = G2a[k] = G2b[k] = 0ull;

  // column group of this lane
  const int cb = tid * kFwdVec;
  const int col = d0 + cb;
  const bool col_ok = col < a.D;
  const bool quad_ok = a.y_quad_ok != 0 && col + kFwdVec - 1 < a.D;
  T* const ybase = static_cast<T*>(a.y) + static_cast<int64_t>(sg.bcoord) * a.ysB + sg.row0 * a.ysL + col;
  const T* const rbase =
      RES ? static_cast<const T*>(a.residual) + static_cast<int64_t>(sg.bcoord) * a.rsB + sg.row0 * a.rsL + col
          : nullptr;
  const int soff = cb;  // element offset of this lane in a slot row

  pf2 pool_a = 0ull, pool_b = 0ull;  // POOL: masked column sums of this lane
  // allv_tag true: the row is known to be a valid row of the sequence (a chunk
  // with no fixed row near it), so the pooled form skips its mask bit
  auto store_row = [&](int64_t orow, pf2 pa, pf2 pb, auto allv_tag) CTA_INLINE {
    if constexpr (POOL) {
      const int64_t p = orow - jb + 32;  // fbits layout: word 0 is the guard word
      if (col_ok && (decltype(allv_tag)::value || ((pbits[p >> 5] >> (p & 31)) & 1u))) {
        pf2 ra, rb2;
        Q::split(Q::join(pa, pb), ra, rb2);  // the values the stored tensor would hold
        pool_a = padd(pool_a, ra);
        pool_b = padd(pool_b, rb2);
      }
      return;
    }
    T* yp = ybase + orow * a.ysL;
    if (quad_ok) {
      V y = Q::join(pa, pb);
      if constexpr (RES) y = vec_add_round<Q>(y, *reinterpret_cast<const V*>(rbase + orow * a.rsL));
      *reinterpret_cast<V*>(yp) = y;
    } else if (col_ok) {
      float v[4];
      upk(pa, v[0], v[1]);
      upk(pb, v[2], v[3]);
#pragma unroll
      for (int j = 0; j < kFwdVec; ++j) {
        if (col + j < a.D) {
          T t = Elem<T>::from_f(v[j]);
          if constexpr (RES) t = Elem<T>::from_f(Elem<T>::to_f(t) + Elem<T>::to_f(rbase[orow * a.rsL + j]));
          yp[j] = t;
        }
      }
    }
  };

  // One march row.  TCT >= 0 is the compile-time march row of a prologue row:
  // level k there is only computed once its inputs are valid (TCT >= 2k + 2),
  // so the start-up triangle of the wavefront costs nothing.
  // slow_tag: 0 = no fixed or zero row near the rows marched, 1 = per-row
  // tests, 2 = every tested row fixed and none zero (the tests are constants),
  // 3 = form 0 inside a tile that has fixed rows (a separate instantiation, so
  // that every chunk form has a single call site and is inlined)
  auto step_row = [&](auto slow_tag, auto tct_tag, int64_t j, pf2& xa, pf2& xb) CTA_INLINE {
    constexpr bool SLOW = decltype(slow_tag)::value == 1 || decltype(slow_tag)::value == 2;
    constexpr bool ALLF = decltype(slow_tag)::value == 2;
    constexpr int TCT = decltype(tct_tag)::value;
    if (SLOW && !ALLF) {
      if (rb.zero(j)) xa = xb = 0ull;
    }
    if constexpr (ADJ) {
      // g enters as level S; level m applies the adjoint of forward step S-m:
      //   non-causal  g_new[i] = g[i] + (a[i+1] - 2 a[i]) + a[i-1],  i = j-1-m
      //   causal      g_new[i] = g[i] + (a[i] - 2 a[i+1]) + a[i+2],  i = j-2-2m
      // with a = alpha * g on updated rows and 0 on fixed rows.
      // FM (contracted): a = g on updated rows, and the level applies
      // g + alpha * lap(a) as one fma instead of g + lap(alpha * g)
      const bool f0 = SLOW && (ALLF || rb.fixed(j));
      const uint32_t fw =
          !SLOW ? 0u : ALLF ? 0xffffffffu : (CAUSAL ? rb.window16_fixed(j - 2 * S) : rb.window8_fixed(j - S));
      pf2 ca = FM ? xa : pmul_sep(al[S - 1], xa, zn), cb = FM ? xb : pmul_sep(al[S - 1], xb, zn);
      if (SLOW && f0) ca = cb = 0ull;
#pragma unroll
      for (int m = 0; m < S; ++m) {
        pf2 na = xa, nb = xb;
        if (TCT < 0 || TCT >= 2 * m + 2) {
          if constexpr (FM) {
            if (CAUSAL) {
              na = pfma(al[S - 1 - m], plap(ca, P1a[m], P2a[m], m2), G2a[m]);
              nb = pfma(al[S - 1 - m], plap(cb, P1b[m], P2b[m], m2), G2b[m]);
            } else {
              na = pfma(al[S - 1 - m], plap(P2a[m], P1a[m], ca, m2), G1a[m]);
              nb = pfma(al[S - 1 - m], plap(P2b[m], P1b[m], cb, m2), G1b[m]);
            }
          } else if (CAUSAL) {
            na = padd(G2a[m], plap(ca, P1a[m], P2a[m], m2));
            nb = padd(G2b[m], plap(cb, P1b[m], P2b[m], m2));
          } else {
            na = padd(G1a[m], plap(P2a[m], P1a[m], ca, m2));
            nb = padd(G1b[m], plap(P2b[m], P1b[m], cb, m2));
          }
        }
        P2a[m] = P1a[m];
        P1a[m] = ca;
        P2b[m] = P1b[m];
        P1b[m] = cb;
        if (CAUSAL) {
          G2a[m] = G1a[m];
          G2b[m] = G1b[m];
        }
        G1a[m] = xa;
        G1b[m] = xb;
        xa = na;
        xb = nb;
        if (m < S - 1) {
          ca = FM ? xa : pmul_sep(al[S - 2 - m], xa, zn);
          cb = FM ? xb : pmul_sep(al[S - 2 - m], xb, zn);
          if (SLOW) {
            const bool f = CAUSAL ? ((fw >> (2 * S - 2 * m - 2)) & 1u) : ((fw >> (S - 1 - m)) & 1u);
            if (f) ca = cb = 0ull;
          }
        }
      }
    } else if (CAUSAL) {
      const bool fx = SLOW && (ALLF || rb.fixed(j));
#pragma unroll
      for (int k = 0; k < S; ++k) {
        pf2 na = xa, nb = xb;
        if (TCT < 0 || TCT >= 2 * k + 2) {
          na = level_update<KIND, true, FM>(P2a[k], P1a[k], xa, al[k], bev[k], bes[k], m2, zn);
          nb = level_update<KIND, true, FM>(P2b[k], P1b[k], xb, al[k], bev[k], bes[k], m2, zn);
          if (SLOW) {
            na = psel(fx, xa, na);
            nb = psel(fx, xb, nb);
          }
        }
        P2a[k] = P1a[k];
        P1a[k] = xa;
        xa = na;
        P2b[k] = P1b[k];
        P1b[k] = xb;
        xb = nb;
      }
    } else {
      // level k updates row j-1-k: bit (S-1-k) of the window of rows j-S .. j-1
      const uint32_t fw = !SLOW ? 0u : ALLF ? 0xffu : rb.window8_fixed(j - S);
#pragma unroll
      for (int k = 0; k < S; ++k) {
        pf2 na = xa, nb = xb;
        if (TCT < 0 || TCT >= 2 * k + 2) {
          na = level_update<KIND, false, FM>(P2a[k], P1a[k], xa, al[k], bev[k], bes[k], m2, zn);
          nb = level_update<KIND, false, FM>(P2b[k], P1b[k], xb, al[k], bev[k], bes[k], m2, zn);
          if (SLOW) {
            const bool fx = (fw >> (S - 1 - k)) & 1u;
            na = psel(fx, P1a[k], na);
            nb = psel(fx, P1b[k], nb);
          }
        }
        P2a[k] = P1a[k];
        P1a[k] = xa;
        xa = na;
        P2b[k] = P1b[k];
        P1b[k] = xb;
        xb = nb;
      }
    }
  };

  // kind: 0..NPRO-1 = prologue chunk, NPRO = full output chunk, NPRO+1 = partial last chunk
  auto march_chunk = [&](auto slow_tag, auto kind_tag, int c, const T* buf) CTA_INLINE {
    constexpr int CK = decltype(kind_tag)::value;
    const int t0 = c * kFwdRC;
    T* st = stage + ((c - NPRO) & 1) * CHUNK + soff;
    // the chunk's rows are read from shared memory up front (CTA_FWD_PRELOAD=1)
    // or as each row is reached
    V in[kFwdRC];
    if constexpr (CTA_FWD_PRELOAD) {
#pragma unroll
      for (int i = 0; i < kFwdRC; ++i) in[i] = *reinterpret_cast<const V*>(buf + soff + i * kFwdDT);
      if constexpr (CTA_FWD_EARLY_REFILL) {
        // the whole chunk is in registers: refill its slot before marching it.
        // Folding every loaded word into `dep` and handing it to the (volatile)
        // issue below orders the shared-memory reads before the TMA overwrite.
        uint32_t dep = 0;
#pragma unroll
        for (int i = 0; i < kFwdRC; ++i) {
          if constexpr (sizeof(V) == 16) {
            const uint4 w = *reinterpret_cast<const uint4*>(&in[i]);
            dep ^= w.x ^ w.y ^ w.z ^ w.w;
          } else if constexpr (sizeof(V) == 8) {
            const uint2 w = *reinterpret_cast<const uint2*>(&in[i]);
            dep ^= w.x ^ w.y;
          } else {
            dep ^= *reinterpret_cast<const uint32_t*>(&in[i]);
          }
        }
        asm volatile("" ::"r"(dep) : "memory");
        __syncwarp();
        if (use_tma && tid == 0 && c + kFwdStages < nch) issue(c + kFwdStages);
      }
    }
    // Full chunks of tiles without fixed rows: the S levels of the chunk's 8
    // rows in anti-diagonal order (row i of level k on diagonal i + k).  Every
    // level still sees its rows in order, so the arithmetic is unchanged, but
    // consecutive instructions come from up to min(S, 8) independent
    // (row, level) cells, which hides the FP32 latency of the dependent chain
    // of one row.
    constexpr bool FAST = decltype(slow_tag)::value == 0 || decltype(slow_tag)::value == 3;
    if constexpr (CTA_FWD_DIAG && CK == NPRO && FAST && CTA_FWD_PRELOAD) {
      pf2 ua[kFwdRC], ub[kFwdRC];
#pragma unroll
      for (int i = 0; i < kFwdRC; ++i) Q::split(in[i], ua[i], ub[i]);
      static_for<kFwdRC + S - 1>([&](auto Dg) {
        constexpr int dg = decltype(Dg)::value;
        static_for<S>([&](auto M) {
          constexpr int m = decltype(M)::value;
          constexpr int i = dg - m;
          if constexpr (i >= 0 && i < kFwdRC) {
            if constexpr (ADJ) {
              // adjoint level m (forward step S-m) at march row i; see step_row
              const pf2 ca = FM ? ua[i] : pmul_sep(al[S - 1 - m], ua[i], zn);
              const pf2 cb = FM ? ub[i] : pmul_sep(al[S - 1 - m], ub[i], zn);
              pf2 na, nb;
              if (CAUSAL) {
                if constexpr (FM) {
                  na = pfma(al[S - 1 - m], plap(ca, P1a[m], P2a[m], m2), G2a[m]);
                  nb = pfma(al[S - 1 - m], plap(cb, P1b[m], P2b[m], m2), G2b[m]);
                } else {
                  na = padd(G2a[m], plap(ca, P1a[m], P2a[m], m2));
                  nb = padd(G2b[m], plap(cb, P1b[m], P2b[m], m2));
                }
                G2a[m] = G1a[m];
                G2b[m] = G1b[m];
              } else if constexpr (FM) {
                na = pfma(al[S - 1 - m], plap(P2a[m], P1a[m], ca, m2), G1a[m]);
                nb = pfma(al[S - 1 - m], plap(P2b[m], P1b[m], cb, m2), G1b[m]);
              } else {
                na = padd(G1a[m], plap(P2a[m], P1a[m], ca, m2));
                nb = padd(G1b[m], plap(P2b[m], P1b[m], cb, m2));
              }
              P2a[m] = P1a[m];
              P1a[m] = ca;
              P2b[m] = P1b[m];
              P1b[m] = cb;
              G1a[m] = ua[i];
              G1b[m] = ub[i];
              ua[i] = na;
              ub[i] = nb;
            } else {
              const pf2 na = level_update<PKIND, CAUSAL, FM>(P2a[m], P1a[m], ua[i], al[m], bev[m], bes[m], m2, zn);
              const pf2 nb = level_update<PKIND, CAUSAL, FM>(P2b[m], P1b[m], ub[i], al[m], bev[m], bes[m], m2, zn);
              P2a[m] = P1a[m];
              P1a[m] = ua[i];
              ua[i] = na;
              P2b[m] = P1b[m];
              P1b[m] = ub[i];
              ub[i] = nb;
            }
          }
        });
      });
#pragma unroll
      for (int i = 0; i < kFwdRC; ++i) {
        if (tstore) {
          V y = Q::join(ua[i], ub[i]);
          if constexpr (RES) y = vec_add_round<Q>(y, *reinterpret_cast<const V*>(st + i * kFwdDT));
          *reinterpret_cast<V*>(st + i * kFwdDT) = y;
        } else {
          store_row(l0 + t0 + i - PRO, ua[i], ub[i], std::true_type{});
        }
      }
      return;
    }
    static_for<kFwdRC>([&](auto I) {
      constexpr int i = decltype(I)::value;
      pf2 xa, xb;
      Q::split(CTA_FWD_PRELOAD ? in[i] : *reinterpret_cast<const V*>(buf + soff + i * kFwdDT), xa, xb);
      if constexpr (CK < NPRO) {
        step_row(slow_tag, std::integral_constant<int, CK * kFwdRC + i>{}, jb + t0 + i, xa, xb);
      } else {
        step_row(slow_tag, std::integral_constant<int, -1>{}, jb + t0 + i, xa, xb);
        const int64_t orow = l0 + t0 + i - PRO;
        if constexpr (CK == NPRO) {
          if (tstore) {
            V y = Q::join(xa, xb);
            // RES: the slot row holds the residual (TMA-loaded for this chunk)
            if constexpr (RES) y = vec_add_round<Q>(y, *reinterpret_cast<const V*>(st + i * kFwdDT));
            *reinterpret_cast<V*>(st + i * kFwdDT) = y;
          } else {
            store_row(orow, xa, xb, std::false_type{});
          }
        } else {
          if (t0 + i < nrows) store_row(orow, xa, xb, std::false_type{});
        }
      }
    });
  };

  // One pipeline step: wait for chunk c, march it, hand full output chunks to
  // the TMA store, refill the slot.  Returns false after a timed-out wait.
  auto do_chunk = [&](auto slow_tag, auto kind_tag, int c) CTA_INLINE -> bool {
    constexpr int CK = decltype(kind_tag)::value;
    constexpr bool FULL = CK == NPRO;
    const int slot = c % kFwdStages;
    const T* buf = ring + slot * CHUNK;
    int err = 0;
    if (use_tma) {
      if (!mbar_wait_bounded(&full_bar[slot], (c / kFwdStages) & 1)) err = 1;
    } else {
      fill_fwd_chunk<T>(a, sg, jb + c * kFwdRC, d0, ring + slot * CHUNK);
      __syncwarp();
    }
    if constexpr (RES && FULL) {
      if (tstore && !err && !mbar_wait_bounded(&res_bar[(c - NPRO) & 1], ((c - NPRO) >> 1) & 1)) err = 1;
    }
    if (!err) march_chunk(slow_tag, kind_tag, c, buf);
    if (FULL && tstore) fence_proxy_async_smem();
    // the store issued after the previous chunk must have finished reading the
    // staging slot that the next chunk overwrites (lanes without bulk groups
    // pass at once)
    if (tstore && (CTA_FWD_PRED || tid == 0)) bulk_wait_read_all();
    __syncwarp();
    if (__any_sync(0xffffffffu, err)) {
      if (tid == 0) {
        atomicExch(&g_bld_fwd_error, kDevTimeout);
        // drain (bounded) every load still in flight, and the stores, before the CTA exits
        if (use_tma)
          for (int cc = c; cc < nch && cc < c + kFwdStages; ++cc)
            mbar_wait_bounded(&full_bar[cc % kFwdStages], (cc / kFwdStages) & 1);
        // the residual load of this chunk, if one was issued (a completed phase passes at once)
        if (RES && tstore && c >= NPRO && c < nfull_end)
          mbar_wait_bounded(&res_bar[(c - NPRO) & 1], ((c - NPRO) >> 1) & 1);
        if (tstore) bulk_wait_all();
      }
      __syncwarp();
      return false;
    }
    if constexpr (CTA_FWD_PRED && !RES) {
      // warp-uniform conditions, lane-0 predicated instructions: no divergence
      if (FULL && tstore) {
        const int orow0 = static_cast<int>(sg.row0 + l0 + c * kFwdRC - PRO);
        tma_store_3d_if(tid == 0, &ymap, stage + ((c - NPRO) & 1) * CHUNK, d0, orow0, sg.bcoord);
        bulk_commit_if(tid == 0);
      }
      if (!(CTA_FWD_PRELOAD && CTA_FWD_EARLY_REFILL) && use_tma && c + kFwdStages < nch) issue_lane0(c + kFwdStages);
    } else if (tid == 0) {
      if (FULL && tstore) {
        const int orow0 = static_cast<int>(sg.row0 + l0 + c * kFwdRC - PRO);
        tma_store_3d(&ymap, stage + ((c - NPRO) & 1) * CHUNK, d0, orow0, sg.bcoord);
        bulk_commit();
      }
      // the next full chunk's staging slot was last read by the store of chunk
      // c-1, which bulk_wait_read_all above has seen complete
      if (RES && tstore && c + 1 >= NPRO && c + 1 < nfull_end) issue_res(c + 1);
      if (!(CTA_FWD_PRELOAD && CTA_FWD_EARLY_REFILL) && use_tma && c + kFwdStages < nch) issue(c + kFwdStages);
    }
    return true;
  };

  // prologue chunks, then a single-body loop over full chunks, then the
  // partial last chunk; the fast/slow choice is made once per tile
  auto run = [&](auto slow_tag) CTA_INLINE -> bool {
    if (!do_chunk(slow_tag, std::integral_constant<int, 0>{}, 0)) return false;
    if constexpr (NPRO > 1) {
      if (!do_chunk(slow_tag, std::integral_constant<int, 1>{}, 1)) return false;
    }
    for (int c = NPRO; c < nfull_end; ++c) {
      if constexpr (decltype(slow_tag)::value != 0) {
        // a tile with fixed or zero rows picks the form of each full chunk from
        // the rows its tests read, [t0 - 2S, t0 + 8) of the march
        const int cls = rb.chunk_class(jb + c * kFwdRC - 2 * S, kFwdRC + 2 * S);
        bool ok = true;
        if (cls == 0) ok = do_chunk(std::integral_constant<int, 3>{}, std::integral_constant<int, NPRO>{}, c);
        else if (cls == 2) ok = do_chunk(std::integral_constant<int, 2>{}, std::integral_constant<int, NPRO>{}, c);
        else ok = do_chunk(slow_tag, std::integral_constant<int, NPRO>{}, c);
        if (!ok) return false;
      } else if (!do_chunk(slow_tag, std::integral_constant<int, NPRO>{}, c)) {
        return false;
      }
    }
    if (nfull_end < nch)
      if (!do_chunk(slow_tag, std::integral_constant<int, NPRO + 1>{}, nfull_end)) return false;
    return true;
  };
  const bool ok = slow ? run(std::integral_constant<int, 1>{}) : run(std::integral_constant<int, 0>{});
  if (ok && tstore && tid == 0) bulk_wait_all();
  if constexpr (POOL) {
    const int64_t ntl = gridDim.x / ndt;
    float* pp = a.pool_partial + ((static_cast<int64_t>(sg.bcoord) * ntl + blockIdx.x / ndt) * a.D);
    float v[4];
    upk(pool_a, v[0], v[1]);
    upk(pool_b, v[2], v[3]);
#pragma unroll
    for (int j = 0; j < kFwdVec; ++j)
      if (col + j < a.D) pp[col + j] = ok ? v[j] : 0.f;
    if (dtile == 0) {
      // valid rows of this tile, after the nbatch * ntl * D partials (exact in fp32)
      int n = 0;
      for (int r0 = 0; r0 < nout; r0 += 32) {
        const int64_t p = l0 + r0 + tid - jb + 32;
        const bool v = r0 + tid < nout && ((pbits[p >> 5] >> (p & 31)) & 1u);
        n += __popc(__ballot_sync(0xffffffffu, v));
      }
      if (tid == 0)
        a.pool_partial[(static_cast<int64_t>(a.nbatch) * ntl) * a.D + static_cast<int64_t>(sg.bcoord) * ntl +
                       blockIdx.x / ndt] = static_cast<float>(n);
    }
  }
}

// pooled[b, d] = round_T(round_T(sum_t partial[b][t][d]) / max(sum_t count[b][t], 1)):
// the reference's half-precision sum and division (transformers.py:135-139).
// A CTA owns 32 columns of one batch row; warp w sums tiles w, w + 32, ... of
// its lane's column with four interleaved accumulators, the per-tile valid-row
// counts are summed by a fixed tree, and warp 0 adds the 32 warp sums in order.
// Every order depends on the shape alone, so the result is deterministic.
template <typename T>
__global__ void __launch_bounds__(kPoolThreads) pool_finish_kernel(const BldArgs a, int64_t ntl, void* pooled) {
  // launched as a programmatic dependent of the march: wait for its partials
  pdl_wait();
  constexpr int NW = kPoolThreads / 32;
  __shared__ double part[NW][33];
  __shared__ double cnt[NW];
  const int b = blockIdx.y;
  const int cl = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float* counts = a.pool_partial + static_cast<int64_t>(a.nbatch) * ntl * a.D + static_cast<int64_t>(b) * ntl;
  double c = 0.0;
  for (int64_t t = threadIdx.x; t < ntl; t += kPoolThreads) c += static_cast<double>(counts[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if (cl == 0) cnt[w] = c;
  const int d = blockIdx.x * 32 + cl;
  double s[4] = {0.0, 0.0, 0.0, 0.0};
  if (d < a.D) {
    const float* col = a.pool_partial + static_cast<int64_t>(b) * ntl * a.D + d;
    int64_t t = w;
    for (; t + 3 * NW < ntl; t += 4 * NW) {
#pragma unroll
      for (int k = 0; k < 4; ++k) s[k] += static_cast<double>(col[(t + k * NW) * a.D]);
    }
    for (int k = 0; t < ntl; t += NW, ++k) s[k] += static_cast<double>(col[t * a.D]);
  }
  part[w][cl] = (s[0] + s[1]) + (s[2] + s[3]);
  __syncthreads();
  if (w == 0 && d < a.D) {
    double sum = 0.0, n = 0.0;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      sum += part[k][cl];
      n += cnt[k];
    }
    const float count = n < 1.0 ? 1.f : static_cast<float>(n);
    const float s_t = Elem<T>::to_f(Elem<T>::from_f(static_cast<float>(sum)));
    static_cast<T*>(pooled)[static_cast<int64_t>(b) * a.D + d] = Elem<T>::from_f(__fdiv_rn(s_t, count));
  }
}

namespace {

template <typename T, bool CAUSAL, bool ADJ, bool RES, bool FM = false>
const void* march_ptr(int steps) {
  switch (steps) {
    case 1: return reinterpret_cast<const void*>(bld_march_kernel<T, 1, CAUSAL, ADJ, RES, 0, false, FM>);
    case 2: return reinterpret_cast<const void*>(bld_march_kernel<T, 2, CAUSAL, ADJ, RES, 0, false, FM>);
    case 3: return reinterpret_cast<const void*>(bld_march_kernel<T, 3, CAUSAL, ADJ, RES, 0, false, FM>);
    case 4: return reinterpret_cast<const void*>(bld_march_kernel<T, 4, CAUSAL, ADJ, RES, 0, false, FM>);
    case 5: return reinterpret_cast<const void*>(bld_march_kernel<T, 5, CAUSAL, ADJ, RES, 0, false, FM>);
    case 6: return reinterpret_cast<const void*>(bld_march_kernel<T, 6, CAUSAL, ADJ, RES, 0, false, FM>);
    case 7: return reinterpret_cast<const void*>(bld_march_kernel<T, 7, CAUSAL, ADJ, RES, 0, false, FM>);
    case 8: return reinterpret_cast<const void*>(bld_march_kernel<T, 8, CAUSAL, ADJ, RES, 0, false, FM>);
    default: return nullptr;
  }
}

template <typename T, int KIND, bool CAUSAL>
const void* march_ptr_kind_c(int steps) {
  switch (steps) {
    case 1: return reinterpret_cast<const void*>(bld_march_kernel<T, 1, CAUSAL, false, false, KIND>);
    case 2: return reinterpret_cast<const void*>(bld_march_kernel<T, 2, CAUSAL, false, false, KIND>);
    case 3: return reinterpret_cast<const void*>(bld_march_kernel<T, 3, CAUSAL, false, false, KIND>);
    case 4: return reinterpret_cast<const void*>(bld_march_kernel<T, 4, CAUSAL, false, false, KIND>);
    default: return nullptr;
  }
}

template <typename T, int KIND>
const void* march_ptr_kind(int steps, int causal) {
  return causal ? march_ptr_kind_c<T, KIND, true>(steps) : march_ptr_kind_c<T, KIND, false>(steps);
}

// FM: the contracted diffusion kernels (16-bit I/O only); otherwise the exact
// ones and the PDE kinds
template <typename T, bool FM>
const void* march_ptr_t(int steps, int causal, int adj, int res, int kind) {
  if constexpr (FM) {
    if constexpr (sizeof(T) == 2) {
      if (kind != 0) return nullptr;
      if (adj) return causal ? march_ptr<T, true, true, false, true>(steps) : march_ptr<T, false, true, false, true>(steps);
      if (res) return causal ? nullptr : march_ptr<T, false, false, true, true>(steps);
      return causal ? march_ptr<T, true, false, false, true>(steps) : march_ptr<T, false, false, false, true>(steps);
    }
    return nullptr;
  } else {
    if (kind != 0) {
      if (adj || res) return nullptr;
      return kind == 1 ? march_ptr_kind<T, 1>(steps, causal) : kind == 2 ? march_ptr_kind<T, 2>(steps, causal) : nullptr;
    }
    if (res) return (causal || adj) ? nullptr : march_ptr<T, false, false, true>(steps);
    if (adj) return causal ? march_ptr<T, true, true, false>(steps) : march_ptr<T, false, true, false>(steps);
    return causal ? march_ptr<T, true, false, false>(steps) : march_ptr<T, false, false, false>(steps);
  }
}

template <typename T>
const void* march_ptr_pool(int steps) {
  switch (steps) {
    case 1: return reinterpret_cast<const void*>(bld_march_kernel<T, 1, false, false, false, 0, true>);
    case 2: return reinterpret_cast<const void*>(bld_march_kernel<T, 2, false, false, false, 0, true>);
    case 3: return reinterpret_cast<const void*>(bld_march_kernel<T, 3, false, false, false, 0, true>);
    case 4: return reinterpret_cast<const void*>(bld_march_kernel<T, 4, false, false, false, 0, true>);
    case 5: return reinterpret_cast<const void*>(bld_march_kernel<T, 5, false, false, false, 0, true>);
    case 6: return reinterpret_cast<const void*>(bld_march_kernel<T, 6, false, false, false, 0, true>);
    case 7: return reinterpret_cast<const void*>(bld_march_kernel<T, 7, false, false, false, 0, true>);
    case 8: return reinterpret_cast<const void*>(bld_march_kernel<T, 8, false, false, false, 0, true>);
    default: return nullptr;
  }
}

// every kernel of one (dtype, arithmetic) pair; FM: the contracted forward /
// adjoint diffusion kernels only, otherwise the exact ones, the PDE kinds and
// the pooled form
template <typename T, bool FM>
const void* march_select(int steps, int causal, int adj, int res, int kind, int pool) {
  if constexpr (FM) {
    if (pool) return nullptr;
  } else {
    if (pool) return (causal || adj || res || kind) ? nullptr : march_ptr_pool<T>(steps);
  }
  return march_ptr_t<T, FM>(steps, causal, adj, res, kind);
}

// this unit's error word
inline int read_fwd_error_word(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bld_fwd_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bld_fwd_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace

}  // namespace cta
