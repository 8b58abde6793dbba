// One step of the non-diffusion PDE layers on [B, L, D] hidden states
// (src/models/pde_layers.py:249-318).  The forward runs on the march kernel
// (bld_fwd.cu, level_update KIND 1/2); this file holds the backward:
//
//   y[i] = x[i] + (alpha * lap[i] + beta * h[i])    on updated rows, x[i] on fixed rows
//   lap[i] = (x[i+1] - 2 x[i]) + x[i-1]              (causal: (x[i] - 2 x[i-1]) + x[i-2])
//   advection-diffusion (:309-318):  h[i] = (x[i+1] - x[i-1]) / 2   (causal: x[i] - x[i-1])
//   reaction-diffusion  (:276-281):  h[i] = x[i] * (1 - sigmoid(x[i]))
//
// with the reference's evaluation order (alpha*lap and beta*h rounded
// separately, then added, then added to x) and its fixed rows (copy boundary,
// rows whose 3-row stencil touches padding).  Reaction-diffusion is nonlinear,
// so its backward needs x: every step runs as its own launch, as the
// reference's layer loop does (src/models/transformers.py:127-133).
//
// Backward, with a = g on updated rows and 0 on fixed rows:
//   dx[j] = g[j] + alpha * (L^T a)[j] + beta * (H^T a)[j]
//     L^T a: (a[j+1] - 2 a[j]) + a[j-1]           (causal: (a[j] - 2 a[j+1]) + a[j+2])
//     H^T a: (a[j-1] - a[j+1]) / 2                (causal: a[j] - a[j+1])     advection
//            a[j] * (1 - s) * (1 - x[j] s), s = sigmoid(x[j])                  reaction
//   d(alpha) = sum_i a[i] lap[i],  d(beta) = sum_i a[i] h[i]
// reduced deterministically (per-CTA partials in a fixed order, then one CTA
// sums them in CTA order in double).
//
// Work decomposition: a thread owns 4 adjacent columns of a run of kPdeRows
// rows and marches down them, keeping the rows its stencil needs in
// registers; loads of the following rows are issued a few rows ahead.
#include "bld_common.cuh"

namespace cta {

namespace {

constexpr int kPdeThreads = 128;  // 4 warps, 512 columns per CTA
constexpr int kPdeVec = 4;        // columns per thread
constexpr int kPdeRows = 32;      // output rows per thread

struct F4 {
  float v[4];
};

template <typename T>
__device__ __forceinline__ F4 load4(const PdeArgs& a, const T* base, int64_t sB, int64_t sL, int b, int64_t row,
                                    int col, bool vec) {
  F4 r;
  if (row < 0 || row >= a.L) {
#pragma unroll
    for (int j = 0; j < 4; ++j) r.v[j] = 0.f;
    return r;
  }
  const T* p = base + static_cast<int64_t>(b) * sB + row * sL + col;
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      const float4 q = *reinterpret_cast<const float4*>(p);
      r.v[0] = q.x;
      r.v[1] = q.y;
      r.v[2] = q.z;
      r.v[3] = q.w;
    } else {
      const uint2 q = *reinterpret_cast<const uint2*>(p);
      const typename Elem<T>::Pair* pp = reinterpret_cast<const typename Elem<T>::Pair*>(&q);
      const float2 f0 = Elem<T>::unpack(pp[0]), f1 = Elem<T>::unpack(pp[1]);
      r.v[0] = f0.x;
      r.v[1] = f0.y;
      r.v[2] = f1.x;
      r.v[3] = f1.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) r.v[j] = (col + j < a.D) ? Elem<T>::to_f(p[j]) : 0.f;
  }
  return r;
}

template <typename T>
__device__ __forceinline__ void store4(const PdeArgs& a, T* base, int64_t sB, int64_t sL, int b, int64_t row, int col,
                                       bool vec, const F4& r) {
  T* p = base + static_cast<int64_t>(b) * sB + row * sL + col;
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
    } else {
      uint2 q;
      typename Elem<T>::Pair* pp = reinterpret_cast<typename Elem<T>::Pair*>(&q);
      pp[0] = Elem<T>::pack(make_float2(r.v[0], r.v[1]));
      pp[1] = Elem<T>::pack(make_float2(r.v[2], r.v[3]));
      *reinterpret_cast<uint2*>(p) = q;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < a.D) p[j] = Elem<T>::from_f(r.v[j]);
  }
}

// rows that keep their value: the copy boundary and rows whose stencil touches
// padding (src/models/pde_layers.py:39-64, :143-182)
template <bool CAUSAL>
__device__ __forceinline__ bool pde_row_fixed(const PdeArgs& a, int b, int64_t i) {
  if (i < 0 || i >= a.L) return true;
  if (CAUSAL ? (i <= 1) : (i <= 0 || i >= a.L - 1)) return true;
  if (a.mask != nullptr) {
    const int64_t base = static_cast<int64_t>(b) * a.msB;
    const bool v0 = mask_valid(a.mask, a.mask_dtype, base + i * a.msL);
    const bool v1 = mask_valid(a.mask, a.mask_dtype, base + (i - 1) * a.msL);
    const bool v2 = mask_valid(a.mask, a.mask_dtype, base + (CAUSAL ? i - 2 : i + 1) * a.msL);
    return !(v0 && v1 && v2);
  }
  return false;
}

// 1 / (1 + e^-v) with the fast exponential and a correctly rounded reciprocal
__device__ __forceinline__ float sigmoid_f(float v) { return __frcp_rn(__fadd_rn(1.0f, __expf(-v))); }

// the stencil terms of row i from its three rows: (lo, mid, hi) = (x[i-1], x[i], x[i+1])
// non-causal or (x[i-2], x[i-1], x[i]) causal.  lap, h as in the file comment,
// and the update alpha*lap + beta-term in the reference's order: advection
// beta*h; reaction (beta*x[i]) * (1 - sigmoid(x[i])), left to right as
// pde_layers.py:278-280 writes it.
template <int KIND, bool CAUSAL>
__device__ __forceinline__ void terms(float lo, float mid, float hi, float al, float be, float& lap, float& h,
                                      float& upd) {
  lap = __fadd_rn(__fmaf_rn(mid, -2.0f, hi), lo);  // (hi - 2 mid) + lo; 2*mid is exact
  const float c = CAUSAL ? hi : mid;
  float bterm;
  if (KIND == kPdeAdvection) {
    h = CAUSAL ? __fsub_rn(hi, mid) : __fmul_rn(__fsub_rn(hi, lo), 0.5f);  // /2 is exact
    bterm = __fmul_rn(be, h);
  } else {
    const float oms = __fsub_rn(1.0f, sigmoid_f(c));
    h = __fmul_rn(c, oms);
    bterm = __fmul_rn(__fmul_rn(be, c), oms);
  }
  upd = __fadd_rn(__fmul_rn(al, lap), bterm);
}

}  // namespace

template <typename T, int KIND, bool CAUSAL>
__global__ void __launch_bounds__(kPdeThreads) pde_step_bwd_kernel(const PdeArgs a) {
  __shared__ float red[kPdeThreads / 32][2];
  const int b = blockIdx.z;
  const int col = (blockIdx.y * kPdeThreads + threadIdx.x) * kPdeVec;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kPdeRows;
  const int64_t r1 = r0 + kPdeRows < a.L ? r0 + kPdeRows : a.L;
  float sa = 0.f, sb = 0.f;  // d(alpha), d(beta) partials of this thread
  if (col < a.D) {
    const bool vx = a.x_vec && col + kPdeVec <= a.D;
    const bool vg = a.g_vec && col + kPdeVec <= a.D;
    const bool vy = a.y_vec && col + kPdeVec <= a.D;
    const float al = load_scalar(a.alpha_dev, a.coef_dtype);
    const float be = load_scalar(a.beta_dev, a.coef_dtype);
    const T* X = static_cast<const T*>(a.x);
    const T* G = static_cast<const T*>(a.g);
    T* Y = static_cast<T*>(a.y);
    // a = g on updated rows: rows j-1, j, j+1 (non-causal) or j, j+1, j+2 (causal)
    auto arow = [&](int64_t i) {
      F4 r = load4<T>(a, G, a.gsB, a.gsL, b, i, col, vg);
      if (pde_row_fixed<CAUSAL>(a, b, i)) {
#pragma unroll
        for (int j = 0; j < 4; ++j) r.v[j] = 0.f;
      }
      return r;
    };
    F4 a0 = arow(CAUSAL ? r0 : r0 - 1);
    F4 a1 = arow(CAUSAL ? r0 + 1 : r0);
    // x rows of the forward stencil of row j: j-1..j+1 (non-causal), j-2..j (causal)
    F4 x0 = load4<T>(a, X, a.xsB, a.xsL, b, CAUSAL ? r0 - 2 : r0 - 1, col, vx);
    F4 x1 = load4<T>(a, X, a.xsB, a.xsL, b, CAUSAL ? r0 - 1 : r0, col, vx);
#pragma unroll 2
    for (int64_t i = r0; i < r1; ++i) {
      const F4 a2 = arow(CAUSAL ? i + 2 : i + 1);
      const F4 x2 = load4<T>(a, X, a.xsB, a.xsL, b, CAUSAL ? i : i + 1, col, vx);
      const F4 gi = load4<T>(a, G, a.gsB, a.gsL, b, i, col, vg);
      const F4& ai = CAUSAL ? a0 : a1;  // a at row i
      F4 out;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // row i's own terms, for d(alpha), d(beta) (a[i] = 0 on fixed rows)
        float lap, h, unused;
        terms<KIND, CAUSAL>(x0.v[j], x1.v[j], x2.v[j], al, be, lap, h, unused);
        sa = fmaf(ai.v[j], lap, sa);
        sb = fmaf(ai.v[j], h, sb);
        // transposed stencils at column row i
        const float am = a0.v[j];                     // non-causal: a[i-1]
        const float ac = CAUSAL ? a0.v[j] : a1.v[j];  // a[i]
        const float ap = CAUSAL ? a1.v[j] : a2.v[j];  // a[i+1]
        const float lt = CAUSAL ? __fadd_rn(__fmaf_rn(a1.v[j], -2.0f, a0.v[j]), a2.v[j])  // (a[i] - 2a[i+1]) + a[i+2]
                                : __fadd_rn(__fmaf_rn(ac, -2.0f, ap), am);              // (a[i+1] - 2a[i]) + a[i-1]
        float ht;
        if (KIND == kPdeAdvection) {
          ht = CAUSAL ? __fsub_rn(ac, ap) : __fmul_rn(__fsub_rn(am, ap), 0.5f);
        } else {
          const float xc = CAUSAL ? x2.v[j] : x1.v[j];  // x[i]
          const float s = sigmoid_f(xc);
          ht = __fmul_rn(ac, __fmul_rn(__fsub_rn(1.0f, s), __fsub_rn(1.0f, __fmul_rn(xc, s))));
        }
        out.v[j] = __fadd_rn(gi.v[j], __fadd_rn(__fmul_rn(al, lt), __fmul_rn(be, ht)));
      }
      store4<T>(a, Y, a.ysB, a.ysL, b, i, col, vy, out);
      a0 = a1;
      a1 = a2;
      x0 = x1;
      x1 = x2;
    }
  }
  // deterministic reduction: warp tree -> CTA (fixed order) -> partial[cta]
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sa += __shfl_xor_sync(0xffffffffu, sa, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[warp][0] = sa;
    red[warp][1] = sb;
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    float v = 0.f;
    for (int w = 0; w < kPdeThreads / 32; ++w) v += red[w][threadIdx.x];
    const int64_t cta = blockIdx.x + static_cast<int64_t>(gridDim.x) * (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z);
    a.partial[cta * 2 + threadIdx.x] = v;
  }
}

// sums the per-CTA partials in CTA order (each thread a strided subsequence,
// then a fixed tree) into dcoef[0..1]
__global__ void __launch_bounds__(256) pde_step_reduce_kernel(const float* partial, int64_t n, float* dcoef) {
  __shared__ double red[256][2];
  double s0 = 0.0, s1 = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 256) {
    s0 += static_cast<double>(partial[2 * i]);
    s1 += static_cast<double>(partial[2 * i + 1]);
  }
  red[threadIdx.x][0] = s0;
  red[threadIdx.x][1] = s1;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      red[threadIdx.x][0] += red[threadIdx.x + w][0];
      red[threadIdx.x][1] += red[threadIdx.x + w][1];
    }
    __syncthreads();
  }
  if (threadIdx.x < 2) dcoef[threadIdx.x] = static_cast<float>(red[0][threadIdx.x]);
}

namespace {

dim3 pde_grid(const PdeArgs& a) {
  return dim3(static_cast<unsigned>((a.L + kPdeRows - 1) / kPdeRows),
              static_cast<unsigned>((a.D + kPdeThreads * kPdeVec - 1) / (kPdeThreads * kPdeVec)),
              static_cast<unsigned>(a.nbatch));
}

template <typename T, int KIND>
cudaError_t launch_t(const PdeArgs& a, int causal, int backward, cudaStream_t st) {
  const dim3 grid = pde_grid(a);
  if (!backward) return cudaErrorInvalidValue;  // the forward runs on the march kernel
  if (causal) pde_step_bwd_kernel<T, KIND, true><<<grid, kPdeThreads, 0, st>>>(a);
  else pde_step_bwd_kernel<T, KIND, false><<<grid, kPdeThreads, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t n = static_cast<int64_t>(grid.x) * grid.y * grid.z;
  pde_step_reduce_kernel<<<1, 256, 0, st>>>(a.partial, n, a.dcoef);
  return cudaGetLastError();
}

template <typename T>
cudaError_t by_kind(const PdeArgs& a, int kind, int causal, int backward, cudaStream_t st) {
  if (kind == kPdeAdvection) return launch_t<T, kPdeAdvection>(a, causal, backward, st);
  if (kind == kPdeReaction) return launch_t<T, kPdeReaction>(a, causal, backward, st);
  return cudaErrorInvalidValue;
}

}  // namespace

int64_t pde_step_num_ctas(const PdeArgs& a) {
  const dim3 g = pde_grid(a);
  return static_cast<int64_t>(g.x) * g.y * g.z;
}

cudaError_t launch_pde_step(const PdeArgs& a, int dtype, int kind, int causal, int backward, cudaStream_t st) {
  switch (dtype) {
    case kF32: return by_kind<float>(a, kind, causal, backward, st);
    case kBF16: return by_kind<__nv_bfloat16>(a, kind, causal, backward, st);
    case kF16: return by_kind<__half>(a, kind, causal, backward, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cta
