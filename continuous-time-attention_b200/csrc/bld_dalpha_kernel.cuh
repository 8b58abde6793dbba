// Fused backward WITH d(alpha) on [B, L, D] hidden states, steps 1..8: the
// one-warp march of bld_fwd_kernel.cuh carrying two wavefronts at once.  The
// kernel template; bld_dalpha_<dtype>[_fm].cu instantiate it per dtype and
// arithmetic, bld_dalpha.cu holds the host side.
//
// Gradient of one step u_k = A_k u_{k-1} (copy boundary, mask, per-step
// alpha_k), kernels/diffusion_triton.py:96-133 generalised to masks and the
// causal stencil, as autograd differentiates src/models/pde_layers.py:113-188:
//   g_{k-1} = A_k^T g_k        a = alpha_k * g_k on updated rows, 0 on fixed rows
//     non-causal  g_{k-1}[i] = g_k[i] + (a[i+1] - 2 a[i]) + a[i-1]
//     causal      g_{k-1}[i] = g_k[i] + (a[i] - 2 a[i+1]) + a[i+2]
//   d(alpha_k) = sum over updated rows i of g_k[i] * lap(u_{k-1})[i]
//
// Work decomposition.  A CTA is one warp owning TL output rows x kDaDT columns;
// each lane owns kDaPairs packed fp32 column pairs (one by default: 64-column
// tiles, so that the two wavefronts of a lane fit in half the registers of two
// pairs and twice as many warps stay resident).  Two input streams arrive
// through their own TMA rings, 8 rows per chunk: the gradient g (entering the
// adjoint wavefront as level S) and the forward input x (entering a
// recomputation of the forward levels u_0 .. u_{S-1}).  One march step
// advances both wavefronts by one row.  The adjoint of level k meets
// lap(u_{k-1}) of the same row a fixed number of march steps earlier or later
// (the forward wavefront lags one row per level, the adjoint one leads), so
// the earlier factor waits in a delay line.  The x stream starts DX rows after
// the g stream, which keeps every delay within 8 march steps.  A delay of 1, 2
// or 4 is a register ring whose slot is the row's position in the 8-row chunk,
// known at compile time, so it costs no moves; the other delays (3, 5, 6, 7 or
// 8, at steps 6..8) use an 8-slot ring per lane in shared memory, written at
// slot I and read at slot (I - delay) mod 8, again known at compile time.
//
// d(alpha) is reduced deterministically: lane sums -> warp shuffle tree (fixed
// order) -> one partial per CTA -> the last CTA of each group (32 CTAs, or a
// multiple of 32 so that there are at most kWsMaxGroups groups) sums its group
// in a fixed order (double) -> the last group to finish sums the group sums in
// order.  Every counter is left at zero.
#pragma once

#include "bld_common.cuh"

namespace cta {

// Each translation unit that instantiates the kernel has its own error word
// (no relocatable device code); the host reads every unit's word.
static __device__ int g_bld_da_error;

namespace {

template <int S, bool CAUSAL>
struct DaGeom {
  // row offset of the x stream from the g stream
  static constexpr int DX = CAUSAL ? -2 * (S / 2) : (S % 2);
  // g rows above the output tile (causal: enough that x starts 2S rows above)
  static constexpr int HLG = CAUSAL ? 2 * S + DX : S;
  // march rows from the first halo row of g to the first finished dx row
  static constexpr int LAG = CAUSAL ? HLG + 2 * S : 2 * S;
  static constexpr int PAD = (kFwdRC - LAG % kFwdRC) % kFwdRC;
  static constexpr int PRO = PAD + LAG;
  static constexpr int NPRO = PRO / kFwdRC;
  // march steps by which lap(u_{k-1}) of a row arrives before g_k of that row
  // (negative: g_k arrives first)
  static constexpr int delay(int k) { return CAUSAL ? DX + 2 * (S - k) : DX + S - 2 * k; }
  static constexpr int adelay(int k) { return delay(k) < 0 ? -delay(k) : delay(k); }
  // the pair (g_k, lap(u_{k-1})) completed at march step t belongs to output row
  // l0 + t - PRO + e(k)
  static constexpr int e(int k) {
    return CAUSAL ? (2 * k < 2 * S + DX ? 2 * k : 2 * S + DX) : (k < S + DX - k ? k : S + DX - k);
  }
  // delays of 1, 2 or 4 march steps divide the 8-row chunk: the delay line is a
  // register ring indexed by the row's place in the chunk (no moves).  Longer
  // or odd delays (3..8) use an 8-slot ring in shared memory, written at slot I
  // and read at slot (I - delay) mod 8, both known at compile time.
  static constexpr bool reg_ring(int k) { return adelay(k) == 1 || adelay(k) == 2 || adelay(k) == 4; }
  static constexpr bool smem_ring(int k) { return adelay(k) != 0 && !reg_ring(k); }
  static constexpr int smem_index(int k) {
    int n = 0;
    for (int j = 1; j < k; ++j) n += smem_ring(j) ? 1 : 0;
    return n;
  }
  static constexpr int n_smem_rings() { return smem_index(S + 1); }
  static constexpr int emax() {
    int m = 0;
    for (int k = 1; k <= S; ++k) m = e(k) > m ? e(k) : m;
    return m;
  }
  static constexpr bool delays_ok() {
    for (int k = 1; k <= S; ++k) {
      if (adelay(k) > kFwdRC) return false;
      if (e(k) < 0) return false;
    }
    return true;
  }
};

template <typename T>
constexpr int da_stages() {
  return sizeof(T) == 4 ? 3 : 4;
}

constexpr int kDaChunk = kFwdRC * kDaDT;  // elements per stream and pipeline slot
constexpr int kDaRingBytes = kFwdRC * kDaPairs * 32 * 8;  // one 8-slot shared-memory delay ring

template <typename T, int S, bool CAUSAL>
constexpr size_t da_smem() {
  return static_cast<size_t>(2 * da_stages<T>() + kFwdOutSlots) * kDaChunk * sizeof(T) +
         static_cast<size_t>(DaGeom<S, CAUSAL>::n_smem_rings()) * kDaRingBytes;
}

// Plain-load fill of one chunk ([8][kDaDT]) of a [B, L, D] stream, for tensors
// TMA cannot address and for L-shard edges: rows before / after the local
// shard come from the halo buffers lo / hi ([nbatch, nlo|nhi, D]), if given.
template <typename T>
__device__ void fill_da_chunk(const BldArgs& a, const void* src, int64_t sB, int64_t sL, const void* lo, int nlo,
                              const void* hi, int nhi, const Seg& s, int64_t jrow0, int d0, T* dst) {
  const T zero = Elem<T>::from_f(0.f);
  for (int idx = threadIdx.x; idx < kDaChunk; idx += kFwdThreads) {
    const int i = idx / kDaDT;
    const int cc = idx - i * kDaDT;
    const int64_t tr = s.row0 + jrow0 + i;
    const int col = d0 + cc;
    const T* rowp = nullptr;
    if (tr >= 0 && tr < a.L) {
      rowp = static_cast<const T*>(src) + static_cast<int64_t>(s.bcoord) * sB + tr * sL;
    } else if (tr < 0 && lo != nullptr && tr >= -nlo) {
      rowp = static_cast<const T*>(lo) + (static_cast<int64_t>(s.bcoord) * nlo + (nlo + tr)) * a.D;
    } else if (tr >= a.L && hi != nullptr && tr - a.L < nhi) {
      rowp = static_cast<const T*>(hi) + (static_cast<int64_t>(s.bcoord) * nhi + (tr - a.L)) * a.D;
    }
    dst[i * kDaDT + cc] = (rowp != nullptr && col < a.D) ? rowp[col] : zero;
  }
}

}  // namespace

// Register budget (one packed pair per lane): forward and adjoint state of S
// levels, the register delay rings and the S laps of a row in flight.  The
// minimum resident one-warp CTAs per SM handed to __launch_bounds__ is the
// largest at which ptxas -v shows no spills for every dtype and direction.
template <typename T, int S, bool CAUSAL>
#ifndef CTA_DA_MIN34
#define CTA_DA_MIN34 16
#endif
constexpr int da_min_ctas() {
  // ptxas budgets registers per SM sub-partition (16384 each, warps spread over
  // 4), so 10 or 12 CTAs both cap a lane at 168 registers and 8 at 255
  return S <= 2 ? 24 : S == 3 ? CTA_DA_MIN34 : S == 4 ? (CAUSAL ? 12 : CTA_DA_MIN34) : S == 5 ? 12
         : (S == 6 && !CAUSAL) ? 12 : 8;
}

// KIND 1 / 2 (steps 1 only): the backward of one advection- / reaction-
// diffusion layer step (src/models/pde_layers.py:276-281, :309-318), with q the
// output gradient on updated rows (0 on fixed rows) and h the layer's beta term:
//   dx[i] += beta * (q[i-1] - q[i+1]) / 2  (causal beta * (q[i] - q[i+1]))      advection
//   dx[i] += beta * q[i] * (1 - s) * (1 - x[i] s), s = sigmoid(x[i])             reaction
//   d(beta) = sum over updated rows of g[i] * h(x)[i], next to d(alpha)
// At steps 1 the adjoint and the recomputed stencil of a row meet in the same
// march step (delay 0), so no delay line is needed.
__device__ __forceinline__ float da_sigmoid(float v) { return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-v))); }

// per element of a pair: s = sigmoid(v); f(v) = v * (1 - s); f'(v) = (1 - s) * (1 - v s)
__device__ __forceinline__ pf2 psigmoid(pf2 v) {
  float v0, v1;
  upk(v, v0, v1);
  return pk(da_sigmoid(v0), da_sigmoid(v1));
}
__device__ __forceinline__ pf2 reaction_f(pf2 v, pf2 s) {
  float v0, v1, s0, s1;
  upk(v, v0, v1);
  upk(s, s0, s1);
  return pk(__fmul_rn(v0, __fsub_rn(1.0f, s0)), __fmul_rn(v1, __fsub_rn(1.0f, s1)));
}
__device__ __forceinline__ pf2 reaction_df(pf2 v, pf2 s) {
  float v0, v1, s0, s1;
  upk(v, v0, v1);
  upk(s, s0, s1);
  return pk(__fmul_rn(__fsub_rn(1.0f, s0), __fsub_rn(1.0f, __fmul_rn(v0, s0))),
            __fmul_rn(__fsub_rn(1.0f, s1), __fsub_rn(1.0f, __fmul_rn(v1, s1))));
}

// FM: the contracted arithmetic for 16-bit I/O -- the forward recomputation as
// u + alpha * lap in one fma (the contracted forward's op order) and the
// adjoint level as g + alpha * lap(a) in one fma with a = g on updated rows.
template <typename T, int S, bool CAUSAL, int KIND = 0, bool FM = false>
__global__ void __launch_bounds__(kFwdThreads, (da_min_ctas<T, S, CAUSAL>()))
    bld_dalpha_kernel(const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap ymap, const BldArgs a) {
  static_assert(KIND == 0 || S == 1, "the other PDE kinds are single steps");
  static_assert(!FM || KIND == 0, "the contracted arithmetic is the diffusion step's");
  constexpr int NV = S + (KIND != 0 ? 1 : 0);  // reduced values: d(alpha_k) [, d(beta)]
  constexpr int NP = kDaPairs;                 // packed column pairs per lane
  using Q = ColVec<T, 2 * NP>;
  using V = typename Q::V;
  using G = DaGeom<S, CAUSAL>;
  constexpr int NST = da_stages<T>();
  constexpr int CHUNK = kDaChunk;
  constexpr int PRO = G::PRO;
  constexpr int NPRO = G::NPRO;
  constexpr int NSR = G::n_smem_rings();
  static_assert(NP == 1 || NP == 2, "one or two packed pairs per lane");
  static_assert(NPRO >= 1 && NPRO <= 3, "prologue spans one to three chunks");
  static_assert(G::delays_ok(), "delays must fit an 8-slot ring");
  static_assert(CAUSAL || G::DX <= G::PAD, "x stream must start S rows above the tile");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* gring = reinterpret_cast<T*>(smem_raw);
  T* xring = gring + NST * CHUNK;
  T* stage = xring + NST * CHUNK;
  pf2* dring = reinterpret_cast<pf2*>(stage + kFwdOutSlots * CHUNK);  // [NSR][8][NP][32]
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ uint32_t fbits[kBldMaxWords + 2];
  __shared__ uint32_t zbits[kBldMaxWords + 2];

  const Seg sg = resolve_seg(a, blockIdx.z);
  const int ndt = (a.D + kDaDT - 1) / kDaDT;
  const int dtile = static_cast<int>(blockIdx.x % ndt);
  const int64_t l0 = a.out_begin + static_cast<int64_t>(blockIdx.x / ndt) * a.TL;
  const int64_t oend = a.out_end < sg.n ? a.out_end : sg.n;
  const int cta_id = blockIdx.x + gridDim.x * blockIdx.z;
  const int tid = threadIdx.x;
  const bool active = l0 < oend;
  const int d0 = dtile * kDaDT;
  const int64_t jbg = l0 - G::HLG - G::PAD;  // first g row of the march
  const int64_t jbx = jbg + G::DX;           // first x row of the march
  const int nout = active ? static_cast<int>(oend - l0 < a.TL ? oend - l0 : a.TL) : 0;
  const int nrows = PRO + nout;
  const int nch = active ? (nrows + kFwdRC - 1) / kFwdRC : 0;
  const bool use_tma = a.use_tma != 0;
  const bool tstore = a.use_tma_store != 0 && kFwdOutSlots > 0;

  pf2 acc[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) acc[k] = 0ull;
  int err = 0;

  if (active) {
    if (tid == 0) {
      if (use_tma) {
        prefetch_tmap(&gmap);
        prefetch_tmap(&xmap);
      }
      if (tstore) prefetch_tmap(&ymap);
#pragma unroll
      for (int s = 0; s < NST; ++s) mbar_init(&full_bar[s], 1);
      fence_mbar_init();
    }
    auto issue = [&](int c) {
      const int slot = c % NST;
      mbar_arrive_expect_tx(&full_bar[slot], 2 * CHUNK * sizeof(T));
      tma_load_3d(gring + slot * CHUNK, &gmap, &full_bar[slot], d0, static_cast<int>(sg.row0 + jbg + c * kFwdRC),
                  sg.bcoord);
      tma_load_3d(xring + slot * CHUNK, &xmap, &full_bar[slot], d0, static_cast<int>(sg.row0 + jbx + c * kFwdRC),
                  sg.bcoord);
    };
    if (use_tma && tid == 0) {
      for (int c = 0; c < nch && c < NST; ++c) issue(c);
    }
    // the shared-memory delay rings start at zero, as the register ones do
    for (int i = tid; i < NSR * kFwdRC * NP * 32; i += 32) dring[i] = 0ull;
    const int64_t jbits = jbg < jbx ? jbg : jbx;
    const int span = (G::DX < 0 ? -G::DX : G::DX) + nch * kFwdRC;
    RowBits rb{fbits, zbits, jbits};
    const bool slow = build_row_bits<CAUSAL, 1>(a, sg, rb, (span + 31) / 32);

    float alf[kMaxSteps];
    load_alphas(a, alf, S);
    pf2 al[S];
#pragma unroll
    for (int k = 0; k < S; ++k) al[k] = pbc(alf[k]);
    const pf2 m2 = pbc(-2.f);
    const pf2 zn = pbc(a.neg_zero);
    const pf2 n1 = pbc(-1.f), half = pbc(0.5f);
    // KIND 1/2: beta in coefficient slot 1; q history (output gradient on updated rows)
    const pf2 be = pbc(KIND == 0 ? 0.f
                                 : (a.alpha_dev[1] != nullptr ? load_scalar(a.alpha_dev[1], a.alpha_dev_dtype)
                                                              : a.alpha[1]));
    pf2 Q1[NP], Q2[NP];
    // reaction: sigmoid of the paired row, kept for the rows the adjoint finishes later
    pf2 S1[NP], S2[NP];
    // adjoint state per level m (forward step k = S - m): a = alpha*g on the two
    // previous rows (P1, P2), g on the one or two previous rows (G1, G2)
    pf2 P1[S][NP], P2[S][NP], G1[S][NP], G2[S][NP];
    // forward recomputation, level q: u_q on the two previous rows
    pf2 F1[S][NP], F2[S][NP];
    // register delay rings, one per step k whose delay is 1, 2 or 4 (the earlier of its two factors)
    pf2 DL[S][4][NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      Q1[p] = Q2[p] = S1[p] = S2[p] = 0ull;
#pragma unroll
      for (int k = 0; k < S; ++k) {
        P1[k][p] = P2[k][p] = G1[k][p] = G2[k][p] = F1[k][p] = F2[k][p] = 0ull;
#pragma unroll
        for (int d = 0; d < 4; ++d) DL[k][d][p] = 0ull;
      }
    }

    const int cb = tid * 2 * NP;
    const int col = d0 + cb;
    const bool col_ok = col < a.D;
    const bool vec_ok = a.y_quad_ok != 0 && col + 2 * NP - 1 < a.D;
    T* const ybase = static_cast<T*>(a.y) + static_cast<int64_t>(sg.bcoord) * a.ysB + sg.row0 * a.ysL + col;

    auto store_row = [&](int64_t orow, const pf2* v) CTA_INLINE {
      T* yp = ybase + orow * a.ysL;
      if (vec_ok) {
        *reinterpret_cast<V*>(yp) = Q::join(v[0], NP > 1 ? v[NP - 1] : 0ull);
      } else if (col_ok) {
        float f[4];
        upk(v[0], f[0], f[1]);
        if (NP > 1) upk(v[NP - 1], f[2], f[3]);
#pragma unroll
        for (int j = 0; j < 2 * NP; ++j)
          if (col + j < a.D) yp[j] = Elem<T>::from_f(f[j]);
      }
    };

    // The forward recomputation of one march row: lap(u_q) of the row for every
    // level q into la, the levels advanced (state F1, F2).
    auto fwd_levels = [&](auto slow_tag, auto tct_tag, int64_t jx, pf2* x, pf2 (&la)[S][NP]) CTA_INLINE {
      constexpr bool SLOW = decltype(slow_tag)::value == 1 || decltype(slow_tag)::value == 2;
      constexpr bool ALLF = decltype(slow_tag)::value == 2;
      constexpr int TCT = decltype(tct_tag)::value;
      {
        const bool fxc = SLOW && CAUSAL && (ALLF || rb.fixed(jx));
        const uint32_t fwx = (SLOW && !CAUSAL) ? (ALLF ? 0xffu : rb.window8_fixed(jx - S)) : 0u;
#pragma unroll
        for (int q = 0; q < S; ++q) {
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            la[q][p] = 0ull;
            pf2 n = x[p];
            if (TCT < 0 || TCT >= 2 * q + 2) {
              la[q][p] = plap(F2[q][p], F1[q][p], x[p], m2);
              if (CAUSAL) {
                n = FM ? pfma(al[q], la[q][p], x[p]) : padd(x[p], pmul_sep(al[q], la[q][p], zn));
                if (SLOW && fxc) n = x[p];
              } else {
                n = FM ? pfma(al[q], la[q][p], F1[q][p]) : padd(F1[q][p], pmul_sep(al[q], la[q][p], zn));
                if (SLOW && ((fwx >> (S - 1 - q)) & 1u)) n = F1[q][p];
              }
            }
            F2[q][p] = F1[q][p];
            F1[q][p] = x[p];
            x[p] = n;
          }
        }
      }
    };

    // The adjoint of one march row: g_k paired with lap(u_{k-1}) through the
    // delay rings into d(alpha), the adjoint levels advanced (state P, G).
    auto adj_levels = [&](auto slow_tag, auto tct_tag, auto i_tag, int t, int lim, int64_t jg, pf2* g,
                          const pf2 (&la)[S][NP], const pf2* h, const pf2* fp) CTA_INLINE {
      constexpr bool SLOW = decltype(slow_tag)::value == 1 || decltype(slow_tag)::value == 2;
      constexpr bool ALLF = decltype(slow_tag)::value == 2;
      constexpr int TCT = decltype(tct_tag)::value;
      constexpr int I = decltype(i_tag)::value;
      const bool f0 = SLOW && (ALLF || rb.fixed(jg));
      const uint32_t fw =
          !SLOW ? 0u : ALLF ? 0xffffffffu : (CAUSAL ? rb.window16_fixed(jg - 2 * S) : rb.window8_fixed(jg - S));
      pf2 c[NP], q[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        c[p] = FM ? g[p] : pmul_sep(al[S - 1], g[p], zn);
        if (SLOW && f0) c[p] = 0ull;
        q[p] = (SLOW && f0) ? 0ull : g[p];  // q at row jg
      }
      static_for<S>([&](auto M) {
        constexpr int m = decltype(M)::value;
        constexpr int k = S - m;
        constexpr int d = G::delay(k);
        constexpr int e = G::e(k);
        // d(alpha_k): g_k is g, lap(u_{k-1}) is la[k-1]
        // paired row - l0 = t - PRO + e, in [0, nout); only updated rows count
        bool take = (TCT < 0 || TCT + e >= PRO) && (TCT == -2 || I + e < lim);
        if (SLOW) take = take && !ALLF && !rb.fixed(l0 + t - PRO + e);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          pf2 pg = g[p], pl = la[k - 1][p];
          if constexpr (G::reg_ring(k)) {
            constexpr int slot = I % G::adelay(k);
            pf2& cell = DL[k - 1][slot][p];
            const pf2 old = cell;
            if constexpr (d > 0) {
              cell = pl;
              pl = old;
            } else {
              cell = pg;
              pg = old;
            }
          } else if constexpr (G::smem_ring(k)) {
            constexpr int r = G::smem_index(k);
            pf2* ring = dring + (r * kFwdRC * NP + p) * 32 + tid;
            constexpr int rd = (I - G::adelay(k) + kFwdRC) % kFwdRC;
            const pf2 old = ring[rd * NP * 32];
            ring[I * NP * 32] = d > 0 ? pl : pg;
            if constexpr (d > 0) pl = old;
            else pg = old;
          }
          if (take) {
            acc[k - 1] = pfma(pg, pl, acc[k - 1]);
            if constexpr (KIND != 0) acc[S] = pfma(pg, h[p], acc[S]);
          }
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          pf2 n = g[p];
          if (TCT < 0 || TCT >= 2 * m + 2) {
            if constexpr (FM) {
              if (CAUSAL) n = pfma(al[S - 1 - m], plap(c[p], P1[m][p], P2[m][p], m2), G2[m][p]);
              else n = pfma(al[S - 1 - m], plap(P2[m][p], P1[m][p], c[p], m2), G1[m][p]);
            } else if (CAUSAL) {
              n = padd(G2[m][p], plap(c[p], P1[m][p], P2[m][p], m2));
            } else {
              n = padd(G1[m][p], plap(P2[m][p], P1[m][p], c[p], m2));
            }
            if constexpr (KIND != 0) {
              // finished row i = jg-1 (causal jg-2): q[i-1], q[i], q[i+1] are
              // (Q2, Q1, q) non-causal, q[i], q[i+1] are (Q2, Q1) causal
              pf2 ht;
              if constexpr (KIND == 1) {
                ht = CAUSAL ? pfma(Q1[p], n1, Q2[p]) : pmul(pfma(q[p], n1, Q2[p]), half);
              } else {
                ht = pmul(fp[p], CAUSAL ? Q2[p] : Q1[p]);
              }
              n = padd(n, pmul_sep(be, ht, zn));
            }
          }
          if constexpr (KIND != 0) {
            Q2[p] = Q1[p];
            Q1[p] = q[p];
          }
          P2[m][p] = P1[m][p];
          P1[m][p] = c[p];
          if (CAUSAL) G2[m][p] = G1[m][p];
          G1[m][p] = g[p];
          g[p] = n;
        }
        if constexpr (m < S - 1) {
          bool f = false;
          if (SLOW) f = CAUSAL ? ((fw >> (2 * S - 2 * m - 2)) & 1u) : ((fw >> (S - 1 - m)) & 1u);
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            c[p] = FM ? g[p] : pmul_sep(al[S - 2 - m], g[p], zn);
            if (SLOW && f) c[p] = 0ull;
          }
        }
      });
    };

    // slow_tag: 0 = no fixed or zero row near the rows marched, 1 = per-row
    // tests, 2 = every tested row fixed and none zero (the tests are constants),
    // 3 = form 0 inside a tile that has fixed rows (its own instantiation).
    // One march row: TCT >= 0 is the compile-time march row of a prologue row
    // (start-up triangles of both wavefronts skipped); I the row in its chunk;
    // lim = nout + PRO - (first march row of the chunk).
    auto step_row = [&](auto slow_tag, auto tct_tag, auto i_tag, int t, int lim, pf2* g, pf2* x) CTA_INLINE {
      constexpr bool SLOW = decltype(slow_tag)::value == 1 || decltype(slow_tag)::value == 2;
      constexpr bool ALLF = decltype(slow_tag)::value == 2;
      constexpr int TCT = decltype(tct_tag)::value;
      constexpr int I = decltype(i_tag)::value;
      const int64_t jg = jbg + t, jx = jbx + t;
      if (SLOW && !ALLF) {
        if (rb.zero(jg))
#pragma unroll
          for (int p = 0; p < NP; ++p) g[p] = 0ull;
        if (rb.zero(jx))
#pragma unroll
          for (int p = 0; p < NP; ++p) x[p] = 0ull;
      }
      // ---- KIND 1/2: the beta term h(x) of the paired row and, for reaction,
      // f'(x) of the row the adjoint finishes (from the window before its shift) ----
      pf2 h[NP], fp[NP];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        h[p] = fp[p] = 0ull;
        if constexpr (KIND == 1) {
          h[p] = CAUSAL ? pfma(F1[0][p], n1, x[p]) : pmul(pfma(F2[0][p], n1, x[p]), half);
        } else if constexpr (KIND == 2) {
          // the paired row is jg; the finished row jg-1 (causal jg-2), whose x is
          // F2 and whose sigmoid was taken one (two) march steps ago
          const pf2 c_ = CAUSAL ? x[p] : F1[0][p];
          const pf2 sv = psigmoid(c_);
          h[p] = reaction_f(c_, sv);
          fp[p] = reaction_df(F2[0][p], CAUSAL ? S2[p] : S1[p]);
          S2[p] = S1[p];
          S1[p] = sv;
        }
      }
      pf2 la[S][NP];
      fwd_levels(slow_tag, tct_tag, jx, x, la);
      adj_levels(slow_tag, tct_tag, i_tag, t, lim, jg, g, la, h, fp);
    };

    // kind: 0..NPRO-1 = prologue chunk, NPRO = full output chunk, NPRO+1 = partial
    // last chunk, NPRO+2 = full chunk whose every pairing lies inside the tile
    // (its row-range test is a compile-time true: march row -2)
    auto march_chunk = [&](auto slow_tag, auto kind_tag, int c, const T* gbuf, const T* xbuf) CTA_INLINE {
      constexpr int CK = decltype(kind_tag)::value;
      constexpr bool FULLK = CK == NPRO || CK == NPRO + 2;
      const int t0 = c * kFwdRC;
      const int lim = nrows - t0;
      T* st = stage + ((c - NPRO) & 1) * CHUNK + cb;
      static_for<kFwdRC>([&](auto II) {
        constexpr int i = decltype(II)::value;
        pf2 g[NP], x[NP], hi_;
        Q::split(*reinterpret_cast<const V*>(gbuf + cb + i * kDaDT), g[0], NP > 1 ? g[NP - 1] : hi_);
        Q::split(*reinterpret_cast<const V*>(xbuf + cb + i * kDaDT), x[0], NP > 1 ? x[NP - 1] : hi_);
        if constexpr (CK < NPRO) {
          step_row(slow_tag, std::integral_constant<int, CK * kFwdRC + i>{}, II, t0 + i, lim, g, x);
        } else {
          step_row(slow_tag, std::integral_constant<int, CK == NPRO + 2 ? -2 : -1>{}, II, t0 + i, lim, g, x);
          const int64_t orow = l0 + t0 + i - PRO;
          if constexpr (FULLK) {
            if (tstore) *reinterpret_cast<V*>(st + i * kDaDT) = Q::join(g[0], NP > 1 ? g[NP - 1] : 0ull);
            else store_row(orow, g);
          } else {
            if (t0 + i < nrows) store_row(orow, g);
          }
        }
      });
    };

    auto do_chunk = [&](auto slow_tag, auto kind_tag, int c) CTA_INLINE -> bool {
      constexpr int CK = decltype(kind_tag)::value;
      constexpr bool FULL = CK == NPRO || CK == NPRO + 2;
      const int slot = c % NST;
      T* gbuf = gring + slot * CHUNK;
      T* xbuf = xring + slot * CHUNK;
      int e = 0;
      if (use_tma) {
        if (!mbar_wait_bounded(&full_bar[slot], (c / NST) & 1)) e = 1;
      } else {
        fill_da_chunk<T>(a, a.g, a.gsB, a.gsL, a.g_lo_ext, a.g_hext_lo, a.g_hi_ext, a.g_hext_hi, sg,
                         jbg + c * kFwdRC, d0, gbuf);
        fill_da_chunk<T>(a, a.x, a.xsB, a.xsL, a.lo_ext, a.hext_lo, a.hi_ext, a.hext_hi, sg, jbx + c * kFwdRC, d0,
                         xbuf);
        __syncwarp();
      }
      if (!e) march_chunk(slow_tag, kind_tag, c, gbuf, xbuf);
      if (FULL && tstore) fence_proxy_async_smem();
      if (tstore && tid == 0) bulk_wait_read_all();
      __syncwarp();
      if (__any_sync(0xffffffffu, e)) {
        if (tid == 0) {
          atomicExch(&g_bld_da_error, kDevTimeout);
          if (use_tma)
            for (int cc = c; cc < nch && cc < c + NST; ++cc) mbar_wait_bounded(&full_bar[cc % NST], (cc / NST) & 1);
          if (tstore) bulk_wait_all();
        }
        __syncwarp();
        return false;
      }
      if (tid == 0) {
        if (FULL && tstore) {
          const int orow0 = static_cast<int>(sg.row0 + l0 + c * kFwdRC - PRO);
          tma_store_3d(&ymap, stage + ((c - NPRO) & 1) * CHUNK, d0, orow0, sg.bcoord);
          bulk_commit();
        }
        if (use_tma && c + NST < nch) issue(c + NST);
      }
      return true;
    };

    const int nfull_end = nrows / kFwdRC;
    // chunks c with 8c + 8 + max e(k) <= nrows pair only rows of the tile
    const int ninner_end =
        !CTA_DA_INNER ? NPRO
                      : (nrows - G::emax() - kFwdRC < 0
                             ? NPRO
                             : max(NPRO, min(nfull_end, (nrows - G::emax() - kFwdRC) / kFwdRC + 1)));
    auto run = [&](auto slow_tag) CTA_INLINE -> bool {
      if (!do_chunk(slow_tag, std::integral_constant<int, 0>{}, 0)) return false;
      if constexpr (NPRO > 1) {
        if (!do_chunk(slow_tag, std::integral_constant<int, 1>{}, 1)) return false;
      }
      if constexpr (NPRO > 2) {
        if (!do_chunk(slow_tag, std::integral_constant<int, 2>{}, 2)) return false;
      }
      int c = NPRO;
      for (; c < ninner_end; ++c) {
        if constexpr (decltype(slow_tag)::value) {
          // a tile with fixed or zero rows picks the form of each inner chunk
          // from the rows its tests read (the g rows [t0 - 2S - 2, t0 + 10) of
          // the march cover the x rows and the pairing rows too)
          const int cls = rb.chunk_class(jbg + c * kFwdRC - 2 * S - 2, kFwdRC + 2 * S + 4);
          bool ok = true;
          if (cls == 0) ok = do_chunk(std::integral_constant<int, 3>{}, std::integral_constant<int, NPRO + 2>{}, c);
          else if (cls == 2) ok = do_chunk(std::integral_constant<int, 2>{}, std::integral_constant<int, NPRO + 2>{}, c);
          else ok = do_chunk(slow_tag, std::integral_constant<int, NPRO + 2>{}, c);
          if (!ok) return false;
        } else if (!do_chunk(slow_tag, std::integral_constant<int, NPRO + 2>{}, c)) {
          return false;
        }
      }
      for (; c < nfull_end; ++c)
        if (!do_chunk(slow_tag, std::integral_constant<int, NPRO>{}, c)) return false;
      if (nfull_end < nch)
        if (!do_chunk(slow_tag, std::integral_constant<int, NPRO + 1>{}, nfull_end)) return false;
      return true;
    };
    const bool ok = slow ? run(std::true_type{}) : run(std::false_type{});
    if (ok && tstore && tid == 0) bulk_wait_all();
    err = ok ? 0 : 1;
  }

  // ---------------- deterministic d(alpha) reduction ----------------
  // a CTA that gave up after a timed-out wait contributes zeros, so the
  // completion protocol (and the counters) stay consistent
  float part[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float lo, hi;
    upk(acc[k], lo, hi);
    float v = err ? 0.f : lo + hi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    part[k] = v;
  }
  // workspace (cta_diffusion_bwd_bld_workspace_bytes): counters at [0, kWsHeaderBytes)
  // -- [0] the group count, [1 + g] group g -- then the CTA partials
  // [num_ctas][S] (f32), then the group sums [ngroups][S] (f64, 8-byte aligned)
  const int gsz = a.dalpha_group;  // CTAs per group, a multiple of 32
  const int ngroups = (a.num_ctas + gsz - 1) / gsz;
  unsigned int* gcount = a.counter + 1;
  double* gsum = reinterpret_cast<double*>(a.dalpha_partial + static_cast<int64_t>(a.num_ctas) * NV +
                                           ((static_cast<int64_t>(a.num_ctas) * NV) & 1));
  if (tid == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) a.dalpha_partial[static_cast<int64_t>(cta_id) * NV + k] = part[k];
  }
  __threadfence();
  __syncwarp();
  const int grp = cta_id / gsz;
  const int gsize = (grp == ngroups - 1) ? a.num_ctas - grp * gsz : gsz;
  unsigned int done = 0;
  if (tid == 0) done = atomicAdd(gcount + grp, 1u);
  done = __shfl_sync(0xffffffffu, done, 0);
  if (done != static_cast<unsigned int>(gsize) - 1u) return;
  // last CTA of the group: lane l sums CTAs grp*gsz + l, + 32, ... in order,
  // then a fixed shuffle tree over the lanes
  __threadfence();
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    double v = 0.0;
    for (int j = tid; j < gsize; j += 32)
      v += static_cast<double>(__ldcg(a.dalpha_partial + static_cast<int64_t>(grp * gsz + j) * NV + k));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (tid == 0) gsum[static_cast<int64_t>(grp) * NV + k] = v;
  }
  if (tid == 0) gcount[grp] = 0u;
  __threadfence();
  __syncwarp();
  if (tid == 0) done = atomicAdd(a.counter, 1u);
  done = __shfl_sync(0xffffffffu, done, 0);
  if (done != static_cast<unsigned int>(ngroups) - 1u) return;
  // last group: lanes stride over the group sums in order, then the same tree
  __threadfence();
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    double v = 0.0;
    for (int g = tid; g < ngroups; g += 32) v += __ldcg(gsum + static_cast<int64_t>(g) * NV + k);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (tid == 0) a.dalpha[k] = static_cast<float>(a.dalpha_accumulate ? static_cast<double>(a.dalpha[k]) + v : v);
  }
  if (tid == 0) *a.counter = 0u;
}

namespace {

template <typename T, bool CAUSAL>
size_t da_smem_s(int steps) {
  switch (steps) {
    case 1: return da_smem<T, 1, CAUSAL>();
    case 2: return da_smem<T, 2, CAUSAL>();
    case 3: return da_smem<T, 3, CAUSAL>();
    case 4: return da_smem<T, 4, CAUSAL>();
    case 5: return da_smem<T, 5, CAUSAL>();
    case 6: return da_smem<T, 6, CAUSAL>();
    case 7: return da_smem<T, 7, CAUSAL>();
    default: return da_smem<T, 8, CAUSAL>();
  }
}

}  // namespace

namespace {

template <typename T, int KIND>
const void* da_ptr_kind(int steps, int causal) {
  if (steps != 1) return nullptr;
  return causal ? reinterpret_cast<const void*>(bld_dalpha_kernel<T, 1, true, KIND>)
                : reinterpret_cast<const void*>(bld_dalpha_kernel<T, 1, false, KIND>);
}

template <typename T>
const void* da_ptr_any(int steps, int causal, int kind) {
  if (kind == 1) return da_ptr_kind<T, 1>(steps, causal);
  if (kind == 2) return da_ptr_kind<T, 2>(steps, causal);
  return nullptr;
}

template <typename T, bool CAUSAL, bool FM = false>
const void* da_ptr(int steps) {
  switch (steps) {
    case 1: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 1, CAUSAL, 0, FM>);
    case 2: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 2, CAUSAL, 0, FM>);
    case 3: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 3, CAUSAL, 0, FM>);
    case 4: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 4, CAUSAL, 0, FM>);
    case 5: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 5, CAUSAL, 0, FM>);
    case 6: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 6, CAUSAL, 0, FM>);
    case 7: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 7, CAUSAL, 0, FM>);
    case 8: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 8, CAUSAL, 0, FM>);
    default: return nullptr;
  }
}

// every kernel of one (dtype, arithmetic) pair: FM the contracted diffusion
// kernels (16-bit I/O), otherwise the exact ones and the PDE kinds
template <typename T, bool FM>
const void* da_select(int steps, int causal, int kind) {
  if constexpr (FM) {
    if (kind != 0) return nullptr;
    return causal ? da_ptr<T, true, true>(steps) : da_ptr<T, false, true>(steps);
  } else {
    if (kind != 0) return da_ptr_any<T>(steps, causal, kind);
    return causal ? da_ptr<T, true>(steps) : da_ptr<T, false>(steps);
  }
}

// this unit's error word
inline int read_da_error_word(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bld_da_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bld_da_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace

}  // namespace cta
