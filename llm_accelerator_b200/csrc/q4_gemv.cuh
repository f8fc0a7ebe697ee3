// Batch-1 Q4 GEMV building blocks (exact integer, CUDA cores).
//
// Work split: a warp owns R consecutive rows for one 1024-column slice of K.
// Lane j of that warp reads 16 bytes (32 nibbles = half a 64-group) of each
// row with one coalesced 128-bit load, so a row slice is one 512-byte
// transaction per warp.  Activation byte limbs are staged once per CTA in
// shared memory and reused across the R rows.
#pragma once
#include "q4_common.cuh"

namespace q4 {

// Shared-memory limb table: per half-group (32 activations) 24 limb words,
// padded to 28 so a quarter-warp of 128-bit reads hits distinct banks.
constexpr int kLimbStride = 28;

__host__ __device__ constexpr int limb_words(int K) { return (K / 32) * kLimbStride; }

// Build limbs + 8*sum(a) for K activations held in shared memory.
// Must be followed by __syncthreads() before use.
__device__ __forceinline__ void stage_limbs(const int32_t* act, int K, uint32_t* limbs, int64_t* bias8) {
  for (int hg = threadIdx.x; hg < K / 32; hg += blockDim.x) {
    const int32_t* a = act + hg * 32;
    uint32_t* l = limbs + hg * kLimbStride;
    int64_t s = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      make_limbs8(a + 8 * c, l + 6 * c);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += a[8 * c + e];
    }
    bias8[hg] = 8 * s;
  }
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// sum(w*a) over this lane's 32 elements of one row, times the group scale.
__device__ __forceinline__ int64_t lane_span(const uint4& w, const uint32_t* l24, int64_t bias8, uint32_t scale) {
  uint32_t p0 = 0, p1 = 0;
  int32_t p2 = 0;
  dot8(w.x, l24 + 0, p0, p1, p2);
  dot8(w.y, l24 + 6, p0, p1, p2);
  dot8(w.z, l24 + 12, p0, p1, p2);
  dot8(w.w, l24 + 18, p0, p1, p2);
  return combine_limbs(p0, p1, p2, bias8) * (int64_t)scale;
}

// Per-lane partial row sums for rows [row0, row0+R) over K-slice `ks`
// (columns [1024*ks, 1024*ks+1024)).  Rows >= nrows contribute 0.
// The caller reduces across the warp.
template <int K, int R>
__device__ __forceinline__ void gemv_slice(const uint8_t* __restrict__ W, const uint16_t* __restrict__ S, int row0,
                                           int nrows, int ks, const uint32_t* limbs, const int64_t* bias8,
                                           int64_t (&acc)[R]) {
  const int lane = threadIdx.x & 31;
  const int hg = ks * 32 + lane;
  uint4 w[R];
  uint32_t sc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row < nrows) {
      w[r] = ldg_stream(W + (size_t)row * (K / 2) + (size_t)hg * 16);
      sc[r] = __ldg(S + (size_t)row * (K / 64) + (hg >> 1));
    } else {
      w[r] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // all-zero weights
      sc[r] = 0;
    }
  }
  uint32_t l24[24];
  const uint4* lp = reinterpret_cast<const uint4*>(limbs + hg * kLimbStride);
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint4 t = lp[i];
    l24[4 * i + 0] = t.x;
    l24[4 * i + 1] = t.y;
    l24[4 * i + 2] = t.z;
    l24[4 * i + 3] = t.w;
  }
  const int64_t b8 = bias8[hg];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] += lane_span(w[r], l24, b8, sc[r]);
}

// Reduce R per-lane values across the warp; every lane ends with all R sums.
template <int R>
__device__ __forceinline__ void warp_reduce_rows(int64_t (&acc)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = warp_sum_i64(acc[r]);
}

}  // namespace q4
