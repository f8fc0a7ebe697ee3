// Shared device helpers for the Q4 fixed-point decode kernels (sm_100a).
//
// Number formats (all exact integers):
//   hidden / residual    signed 24-bit Q14.10 held in int32
//   norm / projection    signed 24-bit Q12.12 held in int32
//   weights              signed int4, two per byte, even column in the low nibble
//   group scales         unsigned 16-bit Q2.14, one per (row, 64 columns)
//   row sums             int64 Q26 (Q12.12 x Q2.14)
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace q4 {

constexpr int kHidden = 1024;
constexpr int kQHeads = 16;
constexpr int kKvHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kQRows = kQHeads * kHeadDim;    // 2048
constexpr int kKvRows = kKvHeads * kHeadDim;  // 1024
constexpr int kInter = 3072;
constexpr int kGroup = 64;
constexpr int kExpLut = 257;
constexpr int kSigLut = 1025;
constexpr int kKvPage = 64;  // positions per KV page

// RMSNorm modes: hidden-size norm (input / post-attention / final) and the
// per-head q/k norm.  Constants follow the reference's fixed-point contract.
struct NormConsts {
  int mean_shift, eps, div_shift, out_shift;
};
constexpr NormConsts kHiddenNorm{10, 1, 26, 21};
constexpr NormConsts kHeadNorm{7, 17, 28, 23};

__device__ __forceinline__ int32_t sat24(int64_t v) {
  return (int32_t)(v < -(1LL << 23) ? -(1LL << 23) : (v > (1LL << 23) - 1 ? (1LL << 23) - 1 : v));
}

// sat24 that also counts saturations into *cnt (when cnt is non-null).
__device__ __forceinline__ int32_t sat24c(int64_t v, int32_t* cnt) {
  if (cnt && (v < -(1LL << 23) || v > (1LL << 23) - 1)) atomicAdd(cnt, 1);
  return sat24(v);
}

// floor(sqrt(n)) for 0 <= n < 2^62.  The double estimate is refined until exact.
__device__ __forceinline__ uint64_t isqrt_u64(uint64_t n) {
  uint64_t r = (uint64_t)sqrt((double)n);
  while (r > 0 && r * r > n) --r;
  while ((r + 1) * (r + 1) <= n) ++r;
  return r;
}

// inv_rms from a sum of squares (the scalar part of the fixed-point RMSNorm).
__device__ __forceinline__ int64_t inv_rms_from_ss(int64_t ss, NormConsts c) {
  const uint64_t rad = (uint64_t)(ss >> c.mean_shift) + (uint64_t)c.eps;
  const uint64_t rms = isqrt_u64(rad);
  if (rms == 0) return (1LL << 24) - 1;
  // rad < 2^47 (sums of at most 1024 squares of 24-bit values, shifted), so
  // rms < 2^24 and both operands fit 32 bits: a 32-bit division, same quotient
  const uint32_t q = (1u << c.div_shift) / (uint32_t)rms;
  return (int64_t)(q < (1u << 24) - 1 ? q : (1u << 24) - 1);
}

__device__ __forceinline__ int32_t norm_apply(int32_t x, int64_t inv, int32_t gamma, NormConsts c) {
  return sat24(((int64_t)x * inv * (int64_t)gamma) >> c.out_shift);
}

// (raw * scale) >> 31 with unbounded-integer semantics: raw = hi*2^32 + lo,
// hi*2^32*scale is a multiple of 2^31, so the floor splits exactly.
__device__ __forceinline__ int64_t scale_score(int64_t raw, int64_t scale_q0_31) {
  const int64_t hi = raw >> 32;
  const uint64_t lo = (uint64_t)raw & 0xFFFFFFFFULL;
  return 2 * hi * scale_q0_31 + (int64_t)((lo * (uint64_t)scale_q0_31) >> 31);
}

// Exp-LUT index of a score: min((max - s + 2^19) >> 20, 256), 0 when max <= s.
__device__ __forceinline__ int lut_index(int64_t max_score, int64_t score) {
  const int64_t d = max_score - score;
  if (d <= 0) return 0;
  const int64_t ix = (d + ((int64_t)1 << 19)) >> 20;
  return ix > kExpLut - 1 ? kExpLut - 1 : (int)ix;
}

// ---- byte-limb dot products --------------------------------------------------
// A Q4 weight w in [-8, 7] is used biased, u = w + 8 = nibble ^ 8 in [0, 15].
// An activation a (signed 24-bit) is split into bytes a = b0 + 256 b1 + 65536 b2
// with b0, b1 unsigned and b2 signed.  Then
//   sum w*a = P0 + 256 P1 + 65536 P2 - 8 sum a,   Pj = sum u * bj
// where each Pj over 64 terms fits comfortably in 32 bits.
__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
  int32_t d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Biased nibbles of one packed word: bytes of `lo` hold u[0], u[2], u[4], u[6]
// and bytes of `hi` hold u[1], u[3], u[5], u[7] (element i in nibble i).
__device__ __forceinline__ void unpack_biased(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = (w ^ 0x08080808u) & 0x0F0F0F0Fu;
  hi = ((w >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
}

// Activation limb words for one 8-element chunk, in the order the unpacked
// weight words expect: {b0 even, b0 odd, b1 even, b1 odd, b2 even, b2 odd}.
struct Limbs8 {
  uint32_t w[6];
};

__device__ __forceinline__ uint32_t byte_of(int32_t v, int k) { return ((uint32_t)v >> (8 * k)) & 0xFFu; }

__device__ __forceinline__ void make_limbs8(const int32_t* a, uint32_t* out6) {
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    out6[2 * k] = byte_of(a[0], k) | (byte_of(a[2], k) << 8) | (byte_of(a[4], k) << 16) | (byte_of(a[6], k) << 24);
    out6[2 * k + 1] = byte_of(a[1], k) | (byte_of(a[3], k) << 8) | (byte_of(a[5], k) << 16) | (byte_of(a[7], k) << 24);
  }
}

// Partial sums over one packed word (8 weights) against its limb words.
__device__ __forceinline__ void dot8(uint32_t word, const uint32_t* l6, uint32_t& p0, uint32_t& p1, int32_t& p2) {
  uint32_t lo, hi;
  unpack_biased(word, lo, hi);
  p0 = dp4a_uu(lo, l6[0], p0);
  p0 = dp4a_uu(hi, l6[1], p0);
  p1 = dp4a_uu(lo, l6[2], p1);
  p1 = dp4a_uu(hi, l6[3], p1);
  p2 = dp4a_us(lo, l6[4], p2);
  p2 = dp4a_us(hi, l6[5], p2);
}

// Combine limb partial sums of a span into sum(w * a) given bias8 = 8 * sum(a).
__device__ __forceinline__ int64_t combine_limbs(uint32_t p0, uint32_t p1, int32_t p2, int64_t bias8) {
  return ((int64_t)p2 << 16) + (int64_t)(p0 + (p1 << 8)) - bias8;
}

// acc + (int64)a * b as one widening multiply-add
__device__ __forceinline__ int64_t mad_wide(int32_t a, int32_t b, int64_t acc) {
  int64_t d;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(acc));
  return d;
}

// floor(n / d) for n, d < 2^53, d > 0: the IEEE double quotient of the exact
// operands is within one of the true quotient, fixed up with integer products.
__device__ __forceinline__ uint64_t udiv_exact(uint64_t n, uint64_t d) {
  uint64_t q = (uint64_t)((double)n / (double)d);
  if (q * d > n)
    --q;
  else if ((q + 1) * d <= n)
    ++q;
  return q;
}

// floor(n / d) (a quotient below 2^32) with a precomputed Barrett reciprocal
// rcp = floor((2^64 - 1) / d), d > 0 (Barrett, 1986): rcp >= (2^64 - d) / d, so
// n rcp / 2^64 > n / d - n / 2^64 > n / d - 1 and q = mulhi(n, rcp) is the
// quotient or one below it; one remainder test makes it exact.
__device__ __forceinline__ uint32_t barrett_div(uint64_t n, uint64_t d, uint64_t rcp) {
  uint64_t q = __umul64hi(n, rcp);
  if (n - q * d >= d) ++q;
  return (uint32_t)q;
}

__device__ __forceinline__ int64_t shfl_xor_i64(int64_t v, int m) {
  return (int64_t)__shfl_xor_sync(0xFFFFFFFFu, (unsigned long long)v, m);
}

__device__ __forceinline__ int64_t warp_sum_i64(int64_t v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += shfl_xor_i64(v, m);
  return v;
}

__device__ __forceinline__ int64_t warp_max_i64(int64_t v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const int64_t o = shfl_xor_i64(v, m);
    v = o > v ? o : v;
  }
  return v;
}

// Block-wide int64 sum; `red` needs blockDim/32 slots.  All threads get it:
// every warp combines the per-warp partials with shuffles (no serial chain of
// shared-memory reads).
__device__ __forceinline__ int64_t block_sum_i64(int64_t v, int64_t* red) {
  v = warp_sum_i64(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_sum_i64(lane < nw ? red[lane] : 0);
}

__device__ __forceinline__ int64_t block_max_i64(int64_t v, int64_t* red) {
  v = warp_max_i64(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_max_i64(lane < nw ? red[lane] : INT64_MIN);
}

// Programmatic dependent launch: wait for the producing grid's memory, and
// let the next grid in the stream start its own prologue early.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

}  // namespace q4
