// Fused backward WITH d(alpha) on [B, L, D] hidden states, steps 1..4: the
// one-warp march of bld_fwd.cu carrying two wavefronts at once.
//
// Gradient of one step u_k = A_k u_{k-1} (copy boundary, mask, per-step
// alpha_k), kernels/diffusion_triton.py:96-133 generalised to masks and the
// causal stencil, as autograd differentiates src/models/pde_layers.py:113-188:
//   g_{k-1} = A_k^T g_k        a = alpha_k * g_k on updated rows, 0 on fixed rows
//     non-causal  g_{k-1}[i] = g_k[i] + (a[i+1] - 2 a[i]) + a[i-1]
//     causal      g_{k-1}[i] = g_k[i] + (a[i] - 2 a[i+1]) + a[i+2]
//   d(alpha_k) = sum over updated rows i of g_k[i] * lap(u_{k-1})[i]
//
// Work decomposition.  A CTA is one warp owning TL output rows x 128 columns;
// each lane owns 4 columns (two packed fp32 pairs).  Two input streams arrive
// through their own TMA rings, 8 rows per chunk: the gradient g (entering the
// adjoint wavefront as level S) and the forward input x (entering a
// recomputation of the forward levels u_0 .. u_{S-1}).  One march step
// advances both wavefronts by one row.  The adjoint of level k meets
// lap(u_{k-1}) of the same row a fixed number of march steps earlier or later
// (the forward wavefront lags one row per level, the adjoint one leads), so
// the earlier factor waits in a register delay line.  The x stream starts
// DX rows after the g stream, with DX chosen so that every delay length is 0,
// 1, 2 or 4: a delay line is then a circular buffer whose slot is the row's
// position in the 8-row chunk, known at compile time, and costs no moves.
//
// d(alpha) is reduced deterministically: lane sums -> warp shuffle tree (fixed
// order) -> one partial per CTA -> the last CTA of each group (32 CTAs, or a
// multiple of 32 so that there are at most kWsMaxGroups groups) sums its group
// in a fixed order (double) -> the last group to finish sums the group sums in
// order.  Every counter is left at zero.
#include "bld_common.cuh"

namespace cta {

__device__ int g_bld_da_error;

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
  // the pair (g_k, lap(u_{k-1})) completed at march step t belongs to output row
  // l0 + t - PRO + e(k)
  static constexpr int e(int k) {
    return CAUSAL ? (2 * k < 2 * S + DX ? 2 * k : 2 * S + DX) : (k < S + DX - k ? k : S + DX - k);
  }
  static constexpr bool delays_ok() {
    for (int k = 1; k <= S; ++k) {
      const int d = delay(k) < 0 ? -delay(k) : delay(k);
      if (!(d == 0 || d == 1 || d == 2 || d == 4)) return false;
      if (e(k) < 0) return false;
    }
    return true;
  }
};

template <typename T>
constexpr int da_stages() {
  return sizeof(T) == 4 ? 2 : 3;
}

template <typename T>
constexpr size_t da_smem() {
  return static_cast<size_t>(2 * da_stages<T>() + kFwdOutSlots) * kFwdRC * kFwdDT * sizeof(T);
}

// Plain-load fill of one chunk ([8][128]) of a [B, L, D] stream, for tensors
// TMA cannot address and for L-shard edges: rows before / after the local
// shard come from the halo buffers lo / hi ([nbatch, nlo|nhi, D]), if given.
template <typename T>
__device__ void fill_da_chunk(const BldArgs& a, const void* src, int64_t sB, int64_t sL, const void* lo, int nlo,
                              const void* hi, int nhi, const Seg& s, int64_t jrow0, int d0, T* dst) {
  const T zero = Elem<T>::from_f(0.f);
  for (int idx = threadIdx.x; idx < kFwdRC * kFwdDT; idx += kFwdThreads) {
    const int i = idx / kFwdDT;
    const int cc = idx - i * kFwdDT;
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
    dst[i * kFwdDT + cc] = (rowp != nullptr && col < a.D) ? rowp[col] : zero;
  }
}

}  // namespace

// Register budget: two wavefronts, the delay lines and the S laps of a row in
// flight need up to ~200 registers at steps 4 (resident CTAs per SM from
// ptxas -v without spills: 16 up to steps 2, 12 at steps 3, 8 beyond)
template <typename T, int S, bool CAUSAL>
constexpr int da_min_ctas() {
  return S <= 2 ? 16 : (S == 3 && !(CAUSAL && sizeof(T) == 4)) ? 12 : 8;
}

// KIND 1 / 2 (steps 1 only): the backward of one advection- / reaction-
// diffusion layer step (src/models/pde_layers.py:276-281, :309-318), with q the
// output gradient on updated rows (0 on fixed rows) and h the layer's beta term:
//   dx[i] += beta * (q[i-1] - q[i+1]) / 2  (causal beta * (q[i] - q[i+1]))      advection
//   dx[i] += beta * q[i] * (1 - s) * (1 - x[i] s), s = sigmoid(x[i])             reaction
//   d(beta) = sum over updated rows of g[i] * h(x)[i], next to d(alpha)
// At steps 1 the adjoint and the recomputed stencil of a row meet in the same
// march step (delay 0), so no delay line is needed.
__device__ __forceinline__ float da_sigmoid(float v) { return __frcp_rn(__fadd_rn(1.0f, __expf(-v))); }

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

template <typename T, int S, bool CAUSAL, int KIND = 0>
__global__ void __launch_bounds__(kFwdThreads, (da_min_ctas<T, S, CAUSAL>()))
    bld_dalpha_kernel(const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap ymap, const BldArgs a) {
  static_assert(KIND == 0 || S == 1, "the other PDE kinds are single steps");
  constexpr int NV = S + (KIND != 0 ? 1 : 0);  // reduced values: d(alpha_k) [, d(beta)]
  using Q = ColVec<T, kFwdVec>;
  using V = typename Q::V;
  using G = DaGeom<S, CAUSAL>;
  constexpr int NST = da_stages<T>();
  constexpr int CHUNK = kFwdRC * kFwdDT;
  constexpr int PRO = G::PRO;
  constexpr int NPRO = G::NPRO;
  static_assert(kFwdVec == 4, "two packed pairs per lane");
  static_assert(NPRO >= 1 && NPRO <= 2, "prologue spans one or two chunks");
  static_assert(G::delays_ok(), "delay lines must divide the chunk");
  static_assert(CAUSAL || G::DX <= G::PAD, "x stream must start S rows above the tile");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  T* gring = reinterpret_cast<T*>(smem_raw);
  T* xring = gring + NST * CHUNK;
  T* stage = xring + NST * CHUNK;
  __shared__ __align__(8) uint64_t full_bar[NST];
  __shared__ uint32_t fbits[kBldMaxWords + 2];
  __shared__ uint32_t zbits[kBldMaxWords + 2];

  const Seg sg = resolve_seg(a, blockIdx.z);
  const int ndt = (a.D + kFwdDT - 1) / kFwdDT;
  const int dtile = static_cast<int>(blockIdx.x % ndt);
  const int64_t l0 = a.out_begin + static_cast<int64_t>(blockIdx.x / ndt) * a.TL;
  const int64_t oend = a.out_end < sg.n ? a.out_end : sg.n;
  const int cta_id = blockIdx.x + gridDim.x * blockIdx.z;
  const int tid = threadIdx.x;
  const bool active = l0 < oend;
  const int d0 = dtile * kFwdDT;
  const int64_t jbg = l0 - G::HLG - G::PAD;  // first g row of the march
  const int64_t jbx = jbg + G::DX;           // first x row of the march
  const int nout = active ? static_cast<int>(oend - l0 < a.TL ? oend - l0 : a.TL) : 0;
  const int nrows = PRO + nout;
  const int nch = active ? (nrows + kFwdRC - 1) / kFwdRC : 0;
  const bool use_tma = a.use_tma != 0;
  const bool tstore = a.use_tma_store != 0;

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
    pf2 Q1a = 0ull, Q1b = 0ull, Q2a = 0ull, Q2b = 0ull;
    // reaction: sigmoid of the paired row, kept for the rows the adjoint finishes later
    pf2 S1a = 0ull, S1b = 0ull, S2a = 0ull, S2b = 0ull;

    // adjoint state per level m (forward step k = S - m): a = alpha*g on the two
    // previous rows (P1, P2), g on the one or two previous rows (G1, G2)
    pf2 P1a[S], P2a[S], P1b[S], P2b[S], G1a[S], G1b[S], G2a[S], G2b[S];
    // forward recomputation, level q: u_q on the two previous rows
    pf2 F1a[S], F2a[S], F1b[S], F2b[S];
    // delay lines, one per step k (the earlier of its two factors)
    pf2 DLa[S][4], DLb[S][4];
#pragma unroll
    for (int k = 0; k < S; ++k) {
      P1a[k] = P2a[k] = P1b[k] = P2b[k] = G1a[k] = G1b[k] = G2a[k] = G2b[k] = 0ull;
      F1a[k] = F2a[k] = F1b[k] = F2b[k] = 0ull;
#pragma unroll
      for (int d = 0; d < 4; ++d) DLa[k][d] = DLb[k][d] = 0ull;
    }

    const int cb = tid * kFwdVec;
    const int col = d0 + cb;
    const bool col_ok = col < a.D;
    const bool quad_ok = a.y_quad_ok != 0 && col + kFwdVec - 1 < a.D;
    T* const ybase = static_cast<T*>(a.y) + static_cast<int64_t>(sg.bcoord) * a.ysB + sg.row0 * a.ysL + col;

    auto store_row = [&](int64_t orow, pf2 pa, pf2 pb) {
      T* yp = ybase + orow * a.ysL;
      if (quad_ok) {
        *reinterpret_cast<V*>(yp) = Q::join(pa, pb);
      } else if (col_ok) {
        float v[4];
        upk(pa, v[0], v[1]);
        upk(pb, v[2], v[3]);
#pragma unroll
        for (int j = 0; j < kFwdVec; ++j)
          if (col + j < a.D) yp[j] = Elem<T>::from_f(v[j]);
      }
    };

    // One march row: TCT >= 0 is the compile-time march row of a prologue row
    // (start-up triangles of both wavefronts skipped); I the row in its chunk;
    // lim = nout + PRO - (first march row of the chunk).
    auto step_row = [&](auto slow_tag, auto tct_tag, auto i_tag, int t, int lim, pf2& ga, pf2& gb, pf2 xa,
                        pf2 xb) {
      constexpr bool SLOW = decltype(slow_tag)::value;
      constexpr int TCT = decltype(tct_tag)::value;
      constexpr int I = decltype(i_tag)::value;
      const int64_t jg = jbg + t, jx = jbx + t;
      if (SLOW) {
        if (rb.zero(jg)) ga = gb = 0ull;
        if (rb.zero(jx)) xa = xb = 0ull;
      }
      // ---- KIND 1/2: the beta term h(x) of the paired row and, for reaction,
      // f'(x) of the row the adjoint finishes (from the window before its shift) ----
      pf2 ha = 0ull, hb = 0ull, fpa = 0ull, fpb = 0ull;
      if constexpr (KIND == 1) {
        ha = CAUSAL ? pfma(F1a[0], n1, xa) : pmul(pfma(F2a[0], n1, xa), half);
        hb = CAUSAL ? pfma(F1b[0], n1, xb) : pmul(pfma(F2b[0], n1, xb), half);
      } else if constexpr (KIND == 2) {
        // the paired row is jg; the finished row jg-1 (causal jg-2), whose x is
        // F2 and whose sigmoid was taken one (two) march steps ago
        const pf2 ca_ = CAUSAL ? xa : F1a[0], cb_ = CAUSAL ? xb : F1b[0];
        const pf2 sa = psigmoid(ca_), sb = psigmoid(cb_);
        ha = reaction_f(ca_, sa);
        hb = reaction_f(cb_, sb);
        fpa = reaction_df(F2a[0], CAUSAL ? S2a : S1a);
        fpb = reaction_df(F2b[0], CAUSAL ? S2b : S1b);
        S2a = S1a;
        S2b = S1b;
        S1a = sa;
        S1b = sb;
      }
      // ---- forward recomputation: lap(u_q) of this march row, q = 0..S-1 ----
      pf2 la[S], lb[S];
      {
        const bool fxc = SLOW && CAUSAL && rb.fixed(jx);
        const uint32_t fwx = (SLOW && !CAUSAL) ? rb.window8_fixed(jx - S) : 0u;
#pragma unroll
        for (int q = 0; q < S; ++q) {
          la[q] = lb[q] = 0ull;
          pf2 na = xa, nb = xb;
          if (TCT < 0 || TCT >= 2 * q + 2) {
            la[q] = plap(F2a[q], F1a[q], xa, m2);
            lb[q] = plap(F2b[q], F1b[q], xb, m2);
            if (CAUSAL) {
              na = padd(xa, pmul_sep(al[q], la[q], zn));
              nb = padd(xb, pmul_sep(al[q], lb[q], zn));
              if (SLOW && fxc) {
                na = xa;
                nb = xb;
              }
            } else {
              na = padd(F1a[q], pmul_sep(al[q], la[q], zn));
              nb = padd(F1b[q], pmul_sep(al[q], lb[q], zn));
              if (SLOW && ((fwx >> (S - 1 - q)) & 1u)) {
                na = F1a[q];
                nb = F1b[q];
              }
            }
          }
          F2a[q] = F1a[q];
          F1a[q] = xa;
          F2b[q] = F1b[q];
          F1b[q] = xb;
          xa = na;
          xb = nb;
        }
      }
      // ---- adjoint march, pairing g_k with lap(u_{k-1}) ----
      const bool f0 = SLOW && rb.fixed(jg);
      const uint32_t fw = SLOW ? (CAUSAL ? rb.window16_fixed(jg - 2 * S) : rb.window8_fixed(jg - S)) : 0u;
      pf2 ca = pmul_sep(al[S - 1], ga, zn), cb2 = pmul_sep(al[S - 1], gb, zn);
      if (SLOW && f0) ca = cb2 = 0ull;
      const pf2 qa = (SLOW && f0) ? 0ull : ga, qb = (SLOW && f0) ? 0ull : gb;  // q at row jg
      static_for<S>([&](auto M) {
        constexpr int m = decltype(M)::value;
        constexpr int k = S - m;
        constexpr int d = G::delay(k);
        constexpr int e = G::e(k);
        // d(alpha_k): g_k is (ga, gb), lap(u_{k-1}) is (la[k-1], lb[k-1])
        {
          pf2 pga = ga, pgb = gb, pla = la[k - 1], plb = lb[k - 1];
          if constexpr (d > 0) {
            constexpr int slot = I % d;
            const pf2 oa = DLa[k - 1][slot], ob = DLb[k - 1][slot];
            DLa[k - 1][slot] = pla;
            DLb[k - 1][slot] = plb;
            pla = oa;
            plb = ob;
          } else if constexpr (d < 0) {
            constexpr int slot = I % (-d);
            const pf2 oa = DLa[k - 1][slot], ob = DLb[k - 1][slot];
            DLa[k - 1][slot] = pga;
            DLb[k - 1][slot] = pgb;
            pga = oa;
            pgb = ob;
          }
          // paired row - l0 = t - PRO + e, in [0, nout); only updated rows count
          bool take = (TCT < 0 || TCT + e >= PRO) && (I + e < lim);
          if (SLOW) take = take && !rb.fixed(l0 + t - PRO + e);
          if (take) {
            acc[k - 1] = pfma(pga, pla, acc[k - 1]);
            acc[k - 1] = pfma(pgb, plb, acc[k - 1]);
            if constexpr (KIND != 0) {
              acc[S] = pfma(pga, ha, acc[S]);
              acc[S] = pfma(pgb, hb, acc[S]);
            }
          }
        }
        pf2 na = ga, nb = gb;
        if (TCT < 0 || TCT >= 2 * m + 2) {
          if (CAUSAL) {
            na = padd(G2a[m], plap(ca, P1a[m], P2a[m], m2));
            nb = padd(G2b[m], plap(cb2, P1b[m], P2b[m], m2));
          } else {
            na = padd(G1a[m], plap(P2a[m], P1a[m], ca, m2));
            nb = padd(G1b[m], plap(P2b[m], P1b[m], cb2, m2));
          }
          if constexpr (KIND != 0) {
            // finished row i = jg-1 (causal jg-2): q[i-1], q[i], q[i+1] are
            // (Q2, Q1, q) non-causal, q[i], q[i+1] are (Q2, Q1) causal
            pf2 hta, htb;
            if constexpr (KIND == 1) {
              hta = CAUSAL ? pfma(Q1a, n1, Q2a) : pmul(pfma(qa, n1, Q2a), half);
              htb = CAUSAL ? pfma(Q1b, n1, Q2b) : pmul(pfma(qb, n1, Q2b), half);
            } else {
              hta = pmul(fpa, CAUSAL ? Q2a : Q1a);
              htb = pmul(fpb, CAUSAL ? Q2b : Q1b);
            }
            na = padd(na, pmul_sep(be, hta, zn));
            nb = padd(nb, pmul_sep(be, htb, zn));
          }
        }
        if constexpr (KIND != 0) {
          Q2a = Q1a;
          Q2b = Q1b;
          Q1a = qa;
          Q1b = qb;
        }
        P2a[m] = P1a[m];
        P1a[m] = ca;
        P2b[m] = P1b[m];
        P1b[m] = cb2;
        if (CAUSAL) {
          G2a[m] = G1a[m];
          G2b[m] = G1b[m];
        }
        G1a[m] = ga;
        G1b[m] = gb;
        ga = na;
        gb = nb;
        if constexpr (m < S - 1) {
          ca = pmul_sep(al[S - 2 - m], ga, zn);
          cb2 = pmul_sep(al[S - 2 - m], gb, zn);
          if (SLOW) {
            const bool f = CAUSAL ? ((fw >> (2 * S - 2 * m - 2)) & 1u) : ((fw >> (S - 1 - m)) & 1u);
            if (f) ca = cb2 = 0ull;
          }
        }
      });
    };

    // kind: 0..NPRO-1 = prologue chunk, NPRO = full output chunk, NPRO+1 = partial last chunk
    auto march_chunk = [&](auto slow_tag, auto kind_tag, int c, const T* gbuf, const T* xbuf) {
      constexpr int KIND = decltype(kind_tag)::value;
      const int t0 = c * kFwdRC;
      const int lim = nrows - t0;
      T* st = stage + ((c - NPRO) & 1) * CHUNK + cb;
      static_for<kFwdRC>([&](auto II) {
        constexpr int i = decltype(II)::value;
        pf2 ga, gb, xa, xb;
        Q::split(*reinterpret_cast<const V*>(gbuf + cb + i * kFwdDT), ga, gb);
        Q::split(*reinterpret_cast<const V*>(xbuf + cb + i * kFwdDT), xa, xb);
        if constexpr (KIND < NPRO) {
          step_row(slow_tag, std::integral_constant<int, KIND * kFwdRC + i>{}, II, t0 + i, lim, ga, gb, xa, xb);
        } else {
          step_row(slow_tag, std::integral_constant<int, -1>{}, II, t0 + i, lim, ga, gb, xa, xb);
          const int64_t orow = l0 + t0 + i - PRO;
          if constexpr (KIND == NPRO) {
            if (tstore) *reinterpret_cast<V*>(st + i * kFwdDT) = Q::join(ga, gb);
            else store_row(orow, ga, gb);
          } else {
            if (t0 + i < nrows) store_row(orow, ga, gb);
          }
        }
      });
    };

    auto do_chunk = [&](auto slow_tag, auto kind_tag, int c) -> bool {
      constexpr int KIND = decltype(kind_tag)::value;
      constexpr bool FULL = KIND == NPRO;
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
    auto run = [&](auto slow_tag) -> bool {
      if (!do_chunk(slow_tag, std::integral_constant<int, 0>{}, 0)) return false;
      if constexpr (NPRO > 1) {
        if (!do_chunk(slow_tag, std::integral_constant<int, 1>{}, 1)) return false;
      }
      for (int c = NPRO; c < nfull_end; ++c)
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

size_t dalpha_smem_bytes(int dtype) { return dtype == kF32 ? da_smem<float>() : da_smem<__nv_bfloat16>(); }

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

template <typename T, bool CAUSAL>
const void* da_ptr(int steps) {
  switch (steps) {
    case 1: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 1, CAUSAL>);
    case 2: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 2, CAUSAL>);
    case 3: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 3, CAUSAL>);
    case 4: return reinterpret_cast<const void*>(bld_dalpha_kernel<T, 4, CAUSAL>);
    default: return nullptr;
  }
}

const void* da_kernel(int dtype, int steps, int causal, int kind = 0) {
  if (kind != 0) {
    switch (dtype) {
      case kF32: return da_ptr_any<float>(steps, causal, kind);
      case kBF16: return da_ptr_any<__nv_bfloat16>(steps, causal, kind);
      case kF16: return da_ptr_any<__half>(steps, causal, kind);
      default: return nullptr;
    }
  }
  switch (dtype) {
    case kF32: return causal ? da_ptr<float, true>(steps) : da_ptr<float, false>(steps);
    case kBF16: return causal ? da_ptr<__nv_bfloat16, true>(steps) : da_ptr<__nv_bfloat16, false>(steps);
    case kF16: return causal ? da_ptr<__half, true>(steps) : da_ptr<__half, false>(steps);
    default: return nullptr;
  }
}

}  // namespace

cudaError_t launch_bld_dalpha(const BldArgs& a, const CUtensorMap* gmap, const CUtensorMap* xmap,
                              const CUtensorMap* ymap, int dtype, int steps, int causal, dim3 grid, cudaStream_t st) {
  const void* kern = da_kernel(dtype, steps, causal, a.pde_kind);
  if (kern == nullptr) return cudaErrorInvalidValue;
  const size_t smem = dalpha_smem_bytes(dtype);
  cudaError_t e = ensure_smem_attr(kern, smem);
  if (e != cudaSuccess) return e;
  void* args[] = {const_cast<CUtensorMap*>(gmap), const_cast<CUtensorMap*>(xmap), const_cast<CUtensorMap*>(ymap),
                  const_cast<BldArgs*>(&a)};
  return cudaLaunchKernel(kern, grid, dim3(kFwdThreads), args, smem, st);
}

int bld_dalpha_ctas_per_sm(int dtype, int steps, int causal) {
  struct Entry {
    const void* kern;
    int dev;
    int n;
  };
  static Entry table[64];
  static int used = 0;
  static std::mutex mu;
  const void* kern = da_kernel(dtype, steps, causal);
  if (kern == nullptr) return -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].kern == kern && table[i].dev == dev) return table[i].n;
  const size_t smem = dalpha_smem_bytes(dtype);
  if (ensure_smem_attr(kern, smem) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kFwdThreads, smem) != cudaSuccess || n <= 0) return -1;
  if (used < 64) table[used++] = Entry{kern, dev, n};
  return n;
}

int read_device_error_bld_dalpha(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bld_da_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int z = 0;
    cudaMemcpyToSymbol(g_bld_da_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace cta
