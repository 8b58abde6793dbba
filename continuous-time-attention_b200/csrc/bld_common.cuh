// Device helpers shared by the [B, L, D] forward and backward kernels.
#pragma once

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace cta {

namespace {

struct Seg {
  int64_t row0;  // tensor row of local row 0
  int bcoord;    // batch coordinate in the tensor
  int64_t n;     // rows of this sequence present in the tensor
  int64_t gdom;  // length of the domain the copy-boundary rule applies to
  int64_t pos;   // global position of local row 0
};

__device__ __forceinline__ Seg resolve_seg(const BldArgs& a, int z) {
  Seg s;
  if (a.cu_seqlens != nullptr) {
    const int64_t b0 = a.cu_seqlens[z];
    const int64_t b1 = a.cu_seqlens[z + 1];
    s.row0 = b0;
    s.bcoord = 0;
    // offsets outside the packed tensor (malformed input) leave the sequence untouched
    s.n = (b1 > b0 && b0 >= 0 && b1 <= a.L) ? b1 - b0 : 0;
    s.gdom = a.pad_to_max ? a.max_len : s.n;
    s.pos = 0;
  } else {
    s.row0 = 0;
    s.bcoord = z;
    s.n = a.L;
    s.gdom = a.global_len;
    s.pos = a.pos_offset;
  }
  return s;
}

// Row j (local index) keeps its value in every step.
template <bool CAUSAL>
__device__ __forceinline__ bool row_fixed(const BldArgs& a, const Seg& s, int64_t j) {
  const int64_t gp = s.pos + j;
  if (CAUSAL) {
    if (gp <= 1 || gp >= s.gdom) return true;
  } else {
    if (gp <= 0 || gp >= s.gdom - 1) return true;
  }
  if (a.mask != nullptr) {
    const int64_t base = static_cast<int64_t>(s.bcoord) * a.msB;
    const bool v0 = mask_valid(a.mask, a.mask_dtype, base + j * a.msL);
    const bool v1 = mask_valid(a.mask, a.mask_dtype, base + (j - 1) * a.msL);
    const bool v2 = mask_valid(a.mask, a.mask_dtype, base + (CAUSAL ? j - 2 : j + 1) * a.msL);
    return !(v0 && v1 && v2);
  }
  return false;
}

// Row j reads as zero (virtual padding row of the zero-padded prefill rule).
__device__ __forceinline__ bool row_zero(const BldArgs& a, const Seg& s, int64_t j) {
  return a.pad_to_max && j >= s.n && j < s.gdom;
}

// Bitmap of fixed / zero rows for rows [jbits, jbits + 32*nwords).  Word 0 is
// a guard word of ones so that "row - 1 .. row - 8" never indexes below it.
struct RowBits {
  uint32_t* fbits;
  uint32_t* zbits;
  int64_t jbits;
  __device__ __forceinline__ uint32_t window8_fixed(int64_t row_lo) const {
    // bits for rows row_lo .. row_lo+7 (bit m = row_lo + m)
    const int64_t p = row_lo - jbits + 32;
    const int w = static_cast<int>(p >> 5), sh = static_cast<int>(p & 31);
    const uint64_t v = static_cast<uint64_t>(fbits[w]) | (static_cast<uint64_t>(fbits[w + 1]) << 32);
    return static_cast<uint32_t>(v >> sh) & 0xffu;
  }
  __device__ __forceinline__ uint32_t window16_fixed(int64_t row_lo) const {
    // bits for rows row_lo .. row_lo+15 (bit m = row_lo + m)
    const int64_t p = row_lo - jbits + 32;
    const int w = static_cast<int>(p >> 5), sh = static_cast<int>(p & 31);
    const uint64_t v = static_cast<uint64_t>(fbits[w]) | (static_cast<uint64_t>(fbits[w + 1]) << 32);
    return static_cast<uint32_t>(v >> sh) & 0xffffu;
  }
  // Rows row_lo .. row_lo+n-1 (n <= 32): 0 if none is fixed or zero, 2 if all
  // are fixed and none is zero, 1 otherwise.
  __device__ __forceinline__ int chunk_class(int64_t row_lo, int n) const {
    const int64_t p = row_lo - jbits + 32;
    const int w = static_cast<int>(p >> 5), sh = static_cast<int>(p & 31);
    const uint32_t m = n >= 32 ? 0xffffffffu : (1u << n) - 1u;
    const uint64_t f = static_cast<uint64_t>(fbits[w]) | (static_cast<uint64_t>(fbits[w + 1]) << 32);
    const uint64_t z = static_cast<uint64_t>(zbits[w]) | (static_cast<uint64_t>(zbits[w + 1]) << 32);
    const uint32_t fw = static_cast<uint32_t>(f >> sh) & m, zw = static_cast<uint32_t>(z >> sh) & m;
    return (fw | zw) == 0u ? 0 : (fw == m && zw == 0u) ? 2 : 1;
  }
  __device__ __forceinline__ bool fixed(int64_t row) const {
    const int64_t p = row - jbits + 32;
    return (fbits[p >> 5] >> (p & 31)) & 1u;
  }
  __device__ __forceinline__ bool zero(int64_t row) const {
    const int64_t p = row - jbits + 32;
    return (zbits[p >> 5] >> (p & 31)) & 1u;
  }
};

// pool_bits (optional, same word layout as fbits): bit set where row j is inside
// the segment and its mask entry is valid
template <bool CAUSAL, int NWARPS = 1>
__device__ __forceinline__ bool build_row_bits(const BldArgs& a, const Seg& sg, RowBits rb, int nwords,
                                               uint32_t* pool_bits = nullptr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t any = 0;
  if (threadIdx.x == 0) {
    rb.fbits[0] = 0xffffffffu;
    rb.zbits[0] = 0u;
  }
  for (int w = warp; w < nwords; w += NWARPS) {
    const int64_t j = rb.jbits + w * 32 + lane;
    const uint32_t fm = __ballot_sync(0xffffffffu, row_fixed<CAUSAL>(a, sg, j));
    const uint32_t zm = __ballot_sync(0xffffffffu, row_zero(a, sg, j));
    if (lane == 0) {
      rb.fbits[w + 1] = fm;
      rb.zbits[w + 1] = zm;
    }
    if (pool_bits != nullptr) {
      const bool pv = j >= 0 && j < sg.n &&
                      mask_valid(a.mask, a.mask_dtype, static_cast<int64_t>(sg.bcoord) * a.msB + j * a.msL);
      const uint32_t pm = __ballot_sync(0xffffffffu, pv);
      if (lane == 0) pool_bits[w + 1] = pm;
    }
    any |= fm | zm;
  }
  if (threadIdx.x == 0) {
    rb.fbits[nwords + 1] = 0xffffffffu;
    rb.zbits[nwords + 1] = 0u;
  }
  if (NWARPS == 1) {
    __syncwarp();
    return any != 0u;  // ballots made `any` warp-uniform
  }
  return __syncthreads_or(any != 0u) != 0;
}

template <typename T>
__device__ __forceinline__ void store_pair(T* rowp, int col, const BldArgs& a, float2 v, bool pair_ok) {
  using E = Elem<T>;
  if (pair_ok) {
    *reinterpret_cast<typename E::Pair*>(rowp + col) = E::pack(v);
  } else {
    rowp[col] = E::from_f(v.x);
    if (col + 1 < a.D) rowp[col + 1] = E::from_f(v.y);
  }
}

__device__ __forceinline__ void load_alphas(const BldArgs& a, float* out, int steps) {
#pragma unroll
  for (int k = 0; k < kMaxSteps; ++k) {
    if (k < steps) out[k] = a.alpha_dev[k] != nullptr ? load_scalar(a.alpha_dev[k], a.alpha_dev_dtype) : a.alpha[k];
  }
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device); the
// attribute lives in the device context, so it is tracked per device.
inline cudaError_t ensure_smem_attr(const void* kern, size_t smem) {
  struct Entry {
    const void* kern;
    unsigned long long devmask;
    size_t smem;
  };
  static Entry table[512];
  static int n = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  for (int i = 0; i < n; ++i) {
    if (table[i].kern == kern) {
      if (bit && (table[i].devmask & bit) && table[i].smem >= smem) return cudaSuccess;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e == cudaSuccess) {
        table[i].devmask |= bit;
        if (smem > table[i].smem) table[i].smem = smem;
      }
      return e;
    }
  }
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess && n < 512) table[n++] = Entry{kern, bit, smem};
  return e;
}

}  // namespace

}  // namespace cta
