// Per-module kernels: one CUDA kernel (or fused pair) per stage of the
// reference's fixed-point decode path, exposed through the C ABI in
// include/q4gpu.h so each stage can be checked bit-exactly on its own.
// The decode-step kernels (q4_decode.cu) fuse these same stages.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <utility>
#include <vector>

#include "q4_gemv.cuh"
#include "q4gpu_internal.h"

namespace q4 {

// ---------------------------------------------------------------------------
// Seeded synthetic values: fl32(C) * fl32(std * 2^-16) where C is the sum of
// twelve 16-bit fields of three splitmix64 hashes minus 6*65535.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ULL;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t tensor_id) {
  return mix64(seed * 0x9E3779B97F4A7C15ULL + tensor_id * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL);
}

__device__ __forceinline__ int32_t synth_centered(uint64_t key, uint64_t i) {
  int32_t s = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + (3 * i + j) * 0x9E3779B97F4A7C15ULL);
    s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
         (int32_t)((h >> 48) & 0xFFFF);
  }
  return s - 6 * 65535;
}

__device__ __forceinline__ float bf16_round(float x) {
  uint32_t b = __float_as_uint(x);
  b = (b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u;
  return __uint_as_float(b);
}

__global__ void synth_f32_kernel(uint64_t key, int64_t start, int64_t n, float k, int bf16, float* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = __fmul_rn(__int2float_rn(synth_centered(key, (uint64_t)(start + i))), k);
    out[i] = bf16 ? bf16_round(v) : v;
  }
}

// ---------------------------------------------------------------------------
// Q4 quantiser: per (row, 64-group) absmax / 7 -> rint(* 2^14) as unsigned
// Q2.14 (forced to 1 when absmax > 0 rounds to 0), q = clip(rint(w / scale)).
// Every float step is one correctly rounded IEEE float32 operation, so the
// result equals the reference's numpy float32 arithmetic bit for bit.
// ---------------------------------------------------------------------------
__global__ void quantize_q4_kernel(const float* __restrict__ w, int64_t rows, int cols, uint8_t* __restrict__ packed,
                                   uint16_t* __restrict__ scale, int* __restrict__ err) {
  const int groups = cols / kGroup;
  const int64_t total = rows * groups;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / groups;
    const int g = (int)(t % groups);
    const float4* src = reinterpret_cast<const float4*>(w + row * cols + g * kGroup);
    float v[kGroup];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < kGroup / 4; ++i) {
      const float4 f = src[i];
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
#pragma unroll
    for (int i = 0; i < kGroup; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float raw = __fdiv_rn(amax, 7.0f);
    float sqf = rintf(__fmul_rn(raw, 16384.0f));
    if (amax > 0.f && sqf == 0.f) sqf = 1.0f;
    if (!(sqf >= 0.f && sqf <= 65535.f)) {
      atomicExch(err, 1);
      sqf = 0.f;
    }
    scale[row * groups + g] = (uint16_t)sqf;
    const float used = __fmul_rn(sqf, 1.0f / 16384.0f);
    const float safe = used > 0.f ? used : 1.0f;
    uint8_t* dst = packed + row * (cols / 2) + g * (kGroup / 2);
#pragma unroll
    for (int i = 0; i < kGroup / 2; ++i) {
      float q0 = fminf(fmaxf(rintf(__fdiv_rn(v[2 * i], safe)), -8.f), 7.f);
      float q1 = fminf(fmaxf(rintf(__fdiv_rn(v[2 * i + 1], safe)), -8.f), 7.f);
      dst[i] = (uint8_t)(((int)q0 & 0xF) | (((int)q1 & 0xF) << 4));
    }
  }
}

// ---------------------------------------------------------------------------
// RMSNorm over `rows` vectors of length n (hidden norm or per-head norm).
// stats (optional) receives per row: sum_squares, mean_square, radicand, rms, inv_rms.
// ---------------------------------------------------------------------------
__global__ void rmsnorm_kernel(const int32_t* __restrict__ x, const int32_t* __restrict__ gamma, int n, int mode,
                               int32_t* __restrict__ out, int64_t* __restrict__ stats) {
  __shared__ int32_t nsat;
  if (threadIdx.x == 0) nsat = 0;
  __shared__ int64_t red[32];
  const NormConsts c = mode == 0 ? kHiddenNorm : kHeadNorm;
  const int32_t* xr = x + (size_t)blockIdx.x * n;
  int64_t ss = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (int64_t)xr[i] * xr[i];
  ss = block_sum_i64(ss, red);
  const int64_t inv = inv_rms_from_ss(ss, c);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[(size_t)blockIdx.x * n + i] = sat24c(((int64_t)xr[i] * inv * (int64_t)gamma[i]) >> c.out_shift, &nsat);
  __syncthreads();
  if (stats && threadIdx.x == 0) {
    const uint64_t rad = (uint64_t)(ss >> c.mean_shift) + c.eps;
    int64_t* st = stats + blockIdx.x * 6;
    st[0] = ss;
    st[1] = ss >> c.mean_shift;
    st[2] = (int64_t)rad;
    st[3] = (int64_t)isqrt_u64(rad);
    st[4] = inv;
    st[5] = nsat;
  }
}

// RoPE rotate-half over `heads` x 128, cos/sin Q1.15 of one position.
__global__ void rope_kernel(const int32_t* __restrict__ x, int heads, const int32_t* __restrict__ cosv,
                            const int32_t* __restrict__ sinv, int32_t* __restrict__ out, int32_t* __restrict__ sat) {
  const int h = blockIdx.x, d = threadIdx.x;
  if (h >= heads || d >= kHeadDim) return;
  const int32_t* xr = x + h * kHeadDim;
  const int64_t rot = d < 64 ? -(int64_t)xr[d + 64] : (int64_t)xr[d - 64];
  out[h * kHeadDim + d] = sat24c(((int64_t)xr[d] * cosv[d] + rot * sinv[d]) >> 15, sat);
}

// Scores raw/scaled for q [qh,128] against k [ctx, kvh, 128] (GQA: kv = q / (qh/kvh)).
__global__ void attn_scores_kernel(const int32_t* __restrict__ q, const int32_t* __restrict__ k, int ctx, int qh,
                                   int kvh, int64_t scale, int64_t* __restrict__ raw, int64_t* __restrict__ scaled) {
  const int h = blockIdx.y;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= ctx) return;
  const int kv = h / (qh / kvh);
  const int32_t* qr = q + h * kHeadDim;
  const int32_t* kr = k + ((size_t)p * kvh + kv) * kHeadDim;
  int64_t s = 0;
  for (int d = 0; d < kHeadDim; ++d) s += (int64_t)qr[d] * kr[d];
  raw[(size_t)h * ctx + p] = s;
  scaled[(size_t)h * ctx + p] = scale_score(s, scale);
}

// Exact LUT softmax of one row (block per row):  idx = min((max - s + 2^19) >> 20, 256),
// prob = (lut[idx] << 16) // sum(lut[idx]).
__global__ void softmax_kernel(const int64_t* __restrict__ scores, int ctx, const int32_t* __restrict__ lut,
                               int32_t* __restrict__ probs, int32_t* __restrict__ idx_out) {
  __shared__ int64_t red[32];
  __shared__ uint64_t probtab[kExpLut];
  const int64_t* s = scores + (size_t)blockIdx.x * ctx;
  int64_t mx = INT64_MIN;
  for (int p = threadIdx.x; p < ctx; p += blockDim.x) mx = s[p] > mx ? s[p] : mx;
  mx = block_max_i64(mx, red);
  int64_t sum = 0;
  for (int p = threadIdx.x; p < ctx; p += blockDim.x) sum += lut[lut_index(mx, s[p])];
  sum = block_sum_i64(sum, red);
  for (int i = threadIdx.x; i < kExpLut; i += blockDim.x) probtab[i] = ((uint64_t)lut[i] << 16) / (uint64_t)sum;
  __syncthreads();
  for (int p = threadIdx.x; p < ctx; p += blockDim.x) {
    const int ix = lut_index(mx, s[p]);
    probs[(size_t)blockIdx.x * ctx + p] = (int32_t)probtab[ix];
    if (idx_out) idx_out[(size_t)blockIdx.x * ctx + p] = ix;
  }
}

// out[h, d] = sat24((sum_p probs[h, p] * v[p, kv, d]) >> 16)
__global__ void value_accum_kernel(const int32_t* __restrict__ probs, const int32_t* __restrict__ v, int ctx, int qh,
                                   int kvh, int32_t* __restrict__ out, int32_t* __restrict__ sat) {
  const int h = blockIdx.x, d = threadIdx.x;
  const int kv = h / (qh / kvh);
  int64_t acc = 0;
  for (int p = 0; p < ctx; ++p) acc += (int64_t)probs[(size_t)h * ctx + p] * v[((size_t)p * kvh + kv) * kHeadDim + d];
  out[h * kHeadDim + d] = sat24c(acc >> 16, sat);
}

// SwiGLU: idx = (clip(g, -32768, 32768) + 32768 + 32) >> 6, silu = sat24(g*sig >> 16),
// h = sat24(silu*up >> 12).
__device__ __forceinline__ int32_t swiglu(int32_t g, int32_t u, const int32_t* sig_lut, int* idx_o, int32_t* silu_o,
                                          int32_t* sat) {
  const int32_t gc = g < -32768 ? -32768 : (g > 32768 ? 32768 : g);
  int ix = (gc + 32768 + 32) >> 6;
  ix = ix > kSigLut - 1 ? kSigLut - 1 : ix;
  const int32_t silu = sat24c(((int64_t)g * sig_lut[ix]) >> 16, sat);
  if (idx_o) *idx_o = ix;
  if (silu_o) *silu_o = silu;
  return sat24c(((int64_t)silu * u) >> 12, sat ? sat + 1 : nullptr);
}

__global__ void silu_mul_kernel(const int32_t* __restrict__ g, const int32_t* __restrict__ u, int n,
                                const int32_t* __restrict__ lut, int32_t* __restrict__ h, int32_t* __restrict__ silu,
                                int32_t* __restrict__ idx, int32_t* __restrict__ sat) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int ix;
  int32_t s;
  h[i] = swiglu(g[i], u[i], lut, &ix, &s, sat);
  if (silu) silu[i] = s;
  if (idx) idx[i] = ix;
}

// out = sat24(a + (b >> shift))
__global__ void residual_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ b, int n, int shift,
                                int32_t* __restrict__ out, int32_t* __restrict__ sat) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = sat24c((int64_t)a[i] + ((int64_t)b[i] >> shift), sat);
}

// Q26 row sums -> Q12.12 words: sat24(q26 >> 14)
__global__ void q26_to_q12_kernel(const int64_t* __restrict__ in, int n, int32_t* __restrict__ out,
                                  int32_t* __restrict__ sat) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = sat24c(in[i] >> 14, sat);
}

// Tied embedding: hidden = (q * scale) >> 4 for each requested token row.
__global__ void embedding_kernel(const int32_t* __restrict__ tokens, const uint8_t* __restrict__ W,
                                 const uint16_t* __restrict__ S, int32_t* __restrict__ out) {
  const int t = tokens[blockIdx.x];
  const uint8_t* row = W + (size_t)t * (kHidden / 2);
  const uint16_t* sc = S + (size_t)t * (kHidden / kGroup);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    const uint8_t b = row[i >> 1];
    const int q = (int)((i & 1) ? (b >> 4) : (b & 0xF));
    const int qs = q >= 8 ? q - 16 : q;
    out[(size_t)blockIdx.x * kHidden + i] = (qs * (int32_t)sc[i / kGroup]) >> 4;
  }
}

// ---------------------------------------------------------------------------
// LM head: Q26 logits over `rows` tied rows + exact argmax (strict > in
// ascending row order: lowest index wins ties).  Per-block bests go to the
// workspace; the last block to finish reduces them.
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Streaming Q4 GEMV (batch 1): rows stream from HBM through a 4-slot shared-
// memory ring by bulk copies (stages of SR consecutive rows, ~16 KB, one
// cp.async.bulk each), so every CTA keeps up to 64 KB of weights in flight.
// A warp owns RW = SR / 8 rows of a stage; lane j covers half-group j of
// each 1024-column slice (16 bytes, 32 nibbles) against the activation byte
// limbs staged once per CTA.  The RW per-lane partial sums meet in a
// transposing butterfly (each exchange halves the values a lane holds).
// Work units are (matrix, stage) over `count` matrices of the same shape at
// fixed strides; each CTA takes a contiguous range of units.
// MODE 0 writes Q26 row sums (and Q12.12); MODE 1 reduces a greedy argmax
// (strict '>' in ascending row order, lowest index on ties).
// ---------------------------------------------------------------------------
struct ArgBest {
  int64_t score;
  int32_t idx;
  int32_t pad;
};

__device__ __forceinline__ bool better(int64_t s, int32_t i, int64_t bs, int32_t bi) {
  return s > bs || (s == bs && i < bi);
}

struct GemvArgs {
  const int32_t* act;
  int64_t act_stride;  // elements between the activations of consecutive matrices (0: shared)
  const uint8_t* W;
  int64_t w_stride;    // bytes between matrices
  const uint16_t* S;
  int64_t s_stride;    // elements between matrices
  int rows;            // rows per matrix
  int count;           // matrices
  int64_t* out;        // [count, rows] Q26 (MODE 0), or logits (MODE 1, optional)
  int64_t out_stride;
  int32_t* out12;      // [count, rows] Q12.12 (optional)
  int32_t* sat;        // saturation counter (optional)
  ArgBest* partial;    // MODE 1: [gridDim.x]
  unsigned int* counter;
  int32_t* out_tok;
  int64_t* out_score;
};

constexpr int kGvConsumers = 8;                    // consumer warps; one more warp issues the copies
constexpr int kGvThreads = (kGvConsumers + 1) * 32;

template <int K>
struct GvCfg {
  static constexpr int SR = K == 1024 ? 32 : 16;  // rows per stage (a multiple of 8)
  static constexpr int RW = SR / kGvConsumers;    // rows per consumer warp per stage
  static constexpr int KS = K / 1024;
  static constexpr int ROWB = K / 2;   // packed bytes per row
  static constexpr int SROWB = K / 32;  // scale bytes per row
  static constexpr int STAGE = SR * ROWB + SR * SROWB;
  static constexpr int NS = K == 1024 ? 4 : (K == 2048 ? 6 : (K == 3072 ? 3 : 2));  // ring slots
  static constexpr size_t SMEM =
      128 + (size_t)NS * STAGE + (size_t)limb_words(K) * 4 + (size_t)(K / 32) * 4 + 2 * NS * 8 + 64;
};

__device__ __forceinline__ void gv_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes), "r"((uint32_t)__cvta_generic_to_shared(bar))
               : "memory");
}
__device__ __forceinline__ void gv_bar_init(uint64_t* b) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)) : "memory");
}
__device__ __forceinline__ void gv_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool gv_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"((uint32_t)__cvta_generic_to_shared(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait (about 0.2 s), false when it ran out
__device__ __forceinline__ bool gv_wait(uint64_t* b, unsigned parity) {
  if (gv_try(b, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 1;; ++it) {
    if (gv_try(b, parity)) return true;
    if ((it & 255u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 200000000ull) return false;
    }
  }
}

// Limb words of K activations (read from global) and, per half-group of 32,
// bias = 8 * sum(a) as int32 (|sum| <= 32 * 2^23, so 8 * sum fits).  One
// thread per 8-element chunk; the four chunks of a half-group sit in
// consecutive lanes.  Follow with __syncthreads().
__device__ __forceinline__ void gv_stage_limbs(const int32_t* __restrict__ act, int K, uint32_t* limbs, int32_t* bias,
                                               int nthreads) {
  for (int c = threadIdx.x; c < K / 8; c += nthreads) {
    const int4 x0 = *reinterpret_cast<const int4*>(act + 8 * c);
    const int4 x1 = *reinterpret_cast<const int4*>(act + 8 * c + 4);
    const int32_t v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    make_limbs8(v, limbs + (c >> 2) * kLimbStride + 6 * (c & 3));
    int32_t sum = v[0] + v[1] + v[2] + v[3] + v[4] + v[5] + v[6] + v[7];  // |sum| < 2^26
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
    if ((c & 3) == 0) bias[c >> 2] = 8 * sum;
  }
}

// sum(w * a) * s over one lane's 32 elements as three widening multiply-adds:
// (P0 + 256 P1) s + 2 P2 (s << 15) - bias s, with Pj the limb partial sums.
__device__ __forceinline__ int64_t gv_span(const uint4& w, const uint32_t* l24, int32_t bias, int32_t s, int64_t acc) {
  uint32_t p0 = 0, p1 = 0;
  int32_t p2 = 0;
  dot8(w.x, l24 + 0, p0, p1, p2);
  dot8(w.y, l24 + 6, p0, p1, p2);
  dot8(w.z, l24 + 12, p0, p1, p2);
  dot8(w.w, l24 + 18, p0, p1, p2);
  acc = mad_wide((int32_t)(p0 + (p1 << 8)), s, acc);
  acc = mad_wide(2 * p2, s << 15, acc);
  return mad_wide(bias, -s, acc);
}

// Butterfly over the warp: the RW lane-partial row sums become full sums;
// every lane ends with the sum of row gv_lane_row<RW>(lane).
template <int RW>
__device__ __forceinline__ int gv_lane_row(int lane) {
  if constexpr (RW == 4) return 2 * ((lane >> 4) & 1) + ((lane >> 3) & 1);
  if constexpr (RW == 2) return (lane >> 4) & 1;
  return 0;
}
template <int RW>
__device__ __forceinline__ int64_t gv_reduce(const int64_t (&acc)[RW], int lane) {
  int64_t v;
  if constexpr (RW == 4) {
    const bool h4 = lane & 16;
    int64_t k0 = h4 ? acc[2] : acc[0], k1 = h4 ? acc[3] : acc[1];
    k0 += shfl_xor_i64(h4 ? acc[0] : acc[2], 16);
    k1 += shfl_xor_i64(h4 ? acc[1] : acc[3], 16);
    const bool h3 = lane & 8;
    v = (h3 ? k1 : k0) + shfl_xor_i64(h3 ? k0 : k1, 8);
    v += shfl_xor_i64(v, 4);
    v += shfl_xor_i64(v, 2);
    v += shfl_xor_i64(v, 1);
  } else if constexpr (RW == 2) {
    const bool h4 = lane & 16;
    v = (h4 ? acc[1] : acc[0]) + shfl_xor_i64(h4 ? acc[0] : acc[1], 16);
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) v += shfl_xor_i64(v, m);
  } else {
    v = warp_sum_i64(acc[0]);
  }
  return v;
}

// SBULK: scales travel with the weights by bulk copy (16-byte aligned scale
// rows); otherwise each lane loads its scales from global memory.
__device__ __forceinline__ void gv_bar_init_n(uint64_t* b, unsigned n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)), "r"(n)
               : "memory");
}
__device__ __forceinline__ void gv_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"((uint32_t)__cvta_generic_to_shared(b)) : "memory");
}
__device__ __forceinline__ void gv_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");
}

template <int K, int MODE, bool SBULK>
__global__ void __launch_bounds__(kGvThreads) gemv_stream_kernel(GemvArgs g) {
  using C = GvCfg<K>;
  extern __shared__ __align__(128) unsigned char gv_smem[];
  uint8_t* ring = gv_smem;
  uint32_t* limbs = reinterpret_cast<uint32_t*>(gv_smem + C::NS * C::STAGE);
  int32_t* bias = reinterpret_cast<int32_t*>(limbs + limb_words(K));
  uint64_t* full = reinterpret_cast<uint64_t*>(bias + K / 32);
  uint64_t* empty = full + C::NS;
  __shared__ ArgBest wbest[kGvConsumers];
  __shared__ bool last;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int spm = (g.rows + C::SR - 1) / C::SR;  // stages per matrix
  const int64_t total = (int64_t)spm * g.count;
  const int64_t u0 = total * blockIdx.x / gridDim.x, u1 = total * (blockIdx.x + 1) / gridDim.x;
  const int n = (int)(u1 - u0);
  if (t == 0) {
    for (int s = 0; s < C::NS; ++s) {
      gv_bar_init(full + s);
      gv_bar_init_n(empty + s, kGvConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int64_t best_s = INT64_MIN;
  int32_t best_i = INT32_MAX;
  if (warp == kGvConsumers) {
    // producer: one lane streams the CTA's stages through the ring
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        const int s = i % C::NS;
        if (i >= C::NS && !gv_wait(empty + s, ((i / C::NS) - 1) & 1)) break;
        const int64_t u = u0 + i;
        const int m = (int)(u / spm), j = (int)(u % spm);
        const int nr = min(C::SR, g.rows - j * C::SR);
        uint8_t* dst = ring + s * C::STAGE;
        gv_expect(full + s, (uint32_t)nr * (C::ROWB + (SBULK ? C::SROWB : 0)));
        gv_bulk(dst, g.W + m * g.w_stride + (int64_t)j * C::SR * C::ROWB, (uint32_t)nr * C::ROWB, full + s);
        if constexpr (SBULK)
          gv_bulk(dst + C::SR * C::ROWB, g.S + m * g.s_stride + (int64_t)j * C::SR * (K / 64), (uint32_t)nr * C::SROWB,
                  full + s);
      }
    }
  } else {
    int cur_m = -1;
    uint32_t l24[24];  // this lane's limbs when K is one slice
    int32_t b32 = 0;
    for (int i = 0; i < n; ++i) {
      const int64_t u = u0 + i;
      const int m = (int)(u / spm), j = (int)(u % spm);
      if (m != cur_m && (cur_m < 0 || g.act_stride != 0)) {
        gv_consumer_sync();
        gv_stage_limbs(g.act + m * g.act_stride, K, limbs, bias, kGvConsumers * 32);
        gv_consumer_sync();
        if constexpr (C::KS == 1) {
          const uint4* lp = reinterpret_cast<const uint4*>(limbs + lane * kLimbStride);
#pragma unroll
          for (int q = 0; q < 6; ++q) {
            const uint4 v = lp[q];
            l24[4 * q] = v.x;
            l24[4 * q + 1] = v.y;
            l24[4 * q + 2] = v.z;
            l24[4 * q + 3] = v.w;
          }
          b32 = bias[lane];
        }
      }
      cur_m = m;
      const int row0 = j * C::SR;
      const int s = i % C::NS;
      uint32_t sc[C::RW][C::KS];
      if constexpr (!SBULK) {
#pragma unroll
        for (int r = 0; r < C::RW; ++r) {
          const int row = row0 + warp * C::RW + r;
          const uint16_t* srow = g.S + m * g.s_stride + (int64_t)min(row, g.rows - 1) * (K / 64);
#pragma unroll
          for (int ks = 0; ks < C::KS; ++ks) sc[r][ks] = __ldg(srow + ((ks * 32 + lane) >> 1));
        }
      }
      const bool ok = gv_wait(full + s, (i / C::NS) & 1);
      const uint8_t* st = ring + s * C::STAGE;
      if constexpr (SBULK) {
        const uint16_t* ss = reinterpret_cast<const uint16_t*>(st + C::SR * C::ROWB);
#pragma unroll
        for (int r = 0; r < C::RW; ++r)
#pragma unroll
          for (int ks = 0; ks < C::KS; ++ks) sc[r][ks] = ss[(warp * C::RW + r) * (K / 64) + ((ks * 32 + lane) >> 1)];
      }
      int64_t acc[C::RW];
#pragma unroll
      for (int r = 0; r < C::RW; ++r) acc[r] = 0;
#pragma unroll
      for (int ks = 0; ks < C::KS; ++ks) {
        if constexpr (C::KS > 1) {
          const int hg = ks * 32 + lane;
          const uint4* lp = reinterpret_cast<const uint4*>(limbs + hg * kLimbStride);
#pragma unroll
          for (int q = 0; q < 6; ++q) {
            const uint4 v = lp[q];
            l24[4 * q] = v.x;
            l24[4 * q + 1] = v.y;
            l24[4 * q + 2] = v.z;
            l24[4 * q + 3] = v.w;
          }
          b32 = bias[hg];
        }
#pragma unroll
        for (int r = 0; r < C::RW; ++r) {
          const int lr = warp * C::RW + r;
          if (row0 + lr < g.rows && ok) {
            const uint4 w = *reinterpret_cast<const uint4*>(st + lr * C::ROWB + ks * 512 + lane * 16);
            acc[r] = gv_span(w, l24, b32, (int32_t)sc[r][ks], acc[r]);
          }
        }
      }
      // the stage's bytes are in registers: hand the slot back
      __syncwarp();
      if (lane == 0) gv_arrive(empty + s);
      const int64_t v = gv_reduce<C::RW>(acc, lane);
      const int row = row0 + warp * C::RW + gv_lane_row<C::RW>(lane);
      if ((lane & (32 / C::RW - 1)) == 0 && row < g.rows) {
        if constexpr (MODE == 0) {
          g.out[m * g.out_stride + row] = v;
          if (g.out12) g.out12[m * g.out_stride + row] = sat24c(v >> 14, g.sat);
        } else {
          if (g.out) g.out[row] = v;
          if (better(v, row, best_s, best_i)) {
            best_s = v;
            best_i = row;
          }
        }
      }
    }
  }
  if constexpr (MODE == 1) {
    auto warp_best = [&](int64_t& bs, int32_t& bi) {
#pragma unroll
      for (int msk = 1; msk < 32; msk <<= 1) {
        const int64_t os = shfl_xor_i64(bs, msk);
        const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, msk);
        if (better(os, oi, bs, bi)) {
          bs = os;
          bi = oi;
        }
      }
    };
    __syncwarp();
    warp_best(best_s, best_i);
    if (lane == 0 && warp < kGvConsumers) wbest[warp] = ArgBest{best_s, best_i, 0};
    __syncthreads();
    if (t == 0) {
      ArgBest b = wbest[0];
      for (int w = 1; w < kGvConsumers; ++w)
        if (better(wbest[w].score, wbest[w].idx, b.score, b.idx)) b = wbest[w];
      g.partial[blockIdx.x] = b;
      __threadfence();
      const unsigned int done = atomicAdd(g.counter, 1u);
      last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (last) {  // the last CTA reduces all partials, every thread a strided share
      __threadfence();
      int64_t bs = INT64_MIN;
      int32_t bi = INT32_MAX;
      for (int i = t; i < (int)gridDim.x; i += kGvThreads) {
        const int64_t cs = *((volatile int64_t*)&g.partial[i].score);
        const int32_t ci = *((volatile int32_t*)&g.partial[i].idx);
        if (better(cs, ci, bs, bi)) {
          bs = cs;
          bi = ci;
        }
      }
      warp_best(bs, bi);
      __syncthreads();
      if (lane == 0 && warp < kGvConsumers) wbest[warp] = ArgBest{bs, bi, 0};
      // the producer warp's share (partials kGvConsumers*32 ..) joins through warp 0's slot
      __syncthreads();
      if (lane == 0 && warp == kGvConsumers && better(bs, bi, wbest[0].score, wbest[0].idx))
        wbest[0] = ArgBest{bs, bi, 0};
      __syncthreads();
      if (t == 0) {
        ArgBest b = wbest[0];
        for (int w = 1; w < kGvConsumers; ++w)
          if (better(wbest[w].score, wbest[w].idx, b.score, b.idx)) b = wbest[w];
        *g.out_tok = b.idx;
        *g.out_score = b.score;
        *g.counter = 0;  // ready for the next launch
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core Q4 GEMV (batch 1).  Weight rows stream into a ring of shared-
// memory slots by TMA (producer warp); consumer warps take the row sums from
// mma.sync m16n8k32 (u8 x u8 -> s32).
//
// A slot holds one unit: a block of up to 64 rows (four 16-row tiles) x 1024
// columns as four 128-byte-wide boxes with the 128-byte swizzle (16-byte
// chunk index XOR row % 8, so the eight rows one load instruction touches
// sit in different banks), and the block's scales for those columns.  A
// consumer warp claims one 16-row tile at a time from a shared counter (its
// K / 1024 units), so faster warps take more tiles.
//
// MMA operands: A = 16 rows of biased nibbles u = w + 8; B = the six 4-bit
// limbs n_j of c = a + 2^23 (columns 0..5) and a column of ones (column 6).
// Thread t of a row holds packed words t and t + 4 of each 64-column group.
// The group's first MMA takes their low nibbles as u with B = 16 n_j, the
// second their high nibbles in place (16 u) with B = n_j, so both add 16 u n_j
// and no shift is needed.  Per row and group the accumulator columns are
// D_j = 16 P_j (P_j = sum u n_j) and D_6 = 16 U (U = sum u), and
//   16 sum w * a = sum_j 16^j D_j - 2^23 D_6 - 128 sum(a).
// Lane t holds columns 2t, 2t + 1 and forms x_t = D_2t + 16 D_2t+1, started
// from the bias split -128 sum(a) = r - 2^23 Q' (0 <= r < 2^23): the MMA
// accumulator starts at r in column 0 (lane 0) and at Q' in column 6 (lane 3).
// Lane t accumulates x_t times the scale (exact int32 x exact int64) and the
// tile's row sum is (acc_0 + 2^8 acc_1 + 2^16 acc_2 - 2^23 acc_3) / 16, an
// exact division.
constexpr int kMvWarps = 15;  // consumer warps; one more issues the copies (16 warps: 128 registers each)
constexpr int kMvThreads = (kMvWarps + 1) * 32;
constexpr int kMvBox = 64 * 128;                     // one 64-row x 128-byte box
constexpr int kMvSlot = 4 * kMvBox + 64 * 32;        // 1024 columns of 64 rows + their scales

template <int K>
struct MvCfg {
  static constexpr int KS = K / 1024;                // units per block
  static constexpr int NS = K <= 2048 ? 6 : 5;       // ring slots
  static constexpr size_t SMEM =
      1024 + (size_t)NS * kMvSlot + (size_t)K * 8 + (size_t)(K / 16) * 4 + 2 * NS * 8 + NS * 4;  // ring, bf, bq, bars
};

// W and S as 3-D u8 tensors [count][rows][bytes]: 64- and 16-row boxes
struct MvMaps {
  CUtensorMap w64, w16, s64, s16;
};

__device__ __forceinline__ void mma_u8(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// first MMA of a group: the accumulator starts at {ci, 0, ci, 0}
__device__ __forceinline__ void mma_u8_init(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1, int32_t ci) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(ci), "r"(0));
}

// Nibble masks and biases held in registers: a three-register LOP3 then
// unpacks a word in one instruction (an immediate takes only one operand slot).
struct MvMasks {
  uint32_t mlo, blo, mhi, bhi;
  __device__ __forceinline__ MvMasks() {
    asm volatile("mov.b32 %0, 0x0F0F0F0F;" : "=r"(mlo));
    asm volatile("mov.b32 %0, 0x08080808;" : "=r"(blo));
    asm volatile("mov.b32 %0, 0xF0F0F0F0;" : "=r"(mhi));
    asm volatile("mov.b32 %0, 0x80808080;" : "=r"(bhi));
  }
  __device__ __forceinline__ uint32_t lo(uint32_t v) const { return (v & mlo) ^ blo; }  // u
  __device__ __forceinline__ uint32_t hi(uint32_t v) const { return (v & mhi) ^ bhi; }  // 16 u
};

__device__ __forceinline__ void mv_tma3(void* dst, const CUtensorMap* m, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"((uint32_t)__cvta_generic_to_shared(bar))
      : "memory");
}

__device__ __forceinline__ void mv_arrive_n(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(b)), "r"(n)
               : "memory");
}

// bounded wait (about 0.2 s) until the producer has issued unit u into the slot
__device__ __forceinline__ bool mv_wait_tag(volatile int* tag, int u) {
  if (*tag == u) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 1;; ++it) {
    __nanosleep(200);  // the unit is at least one slot turn away: leave the issue slots to working warps
    if (*tag == u) return true;
    if ((it & 255u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 200000000ull) return false;
    }
  }
}

// bounded wait (about 0.2 s) on an mbarrier phase; each try suspends the
// thread in hardware (up to 0.1 ms) until the phase completes, so waiting
// warps take no issue slots
__device__ __forceinline__ bool mv_wait(uint64_t* b, unsigned parity) {
  const uint32_t addr = (uint32_t)__cvta_generic_to_shared(b);
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "r"(100000u)
        : "memory");
    if (ok) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 200000000ull) return false;
  }
}

__device__ __forceinline__ void mv_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kMvWarps * 32) : "memory");
}

// B fragments and accumulator starts of K activations.  bf[G][lane] (g =
// lane / 4, t = lane % 4) = {lo b0, lo b1, hi b0, hi b1}: lo b0 holds
// 16 n_g(c) at columns 64 G + 8 t + {0, 2, 4, 6}, lo b1 the same + 32, hi b0
// and b1 n_g(c) at those columns + 1 (g = 6: ones, 16 for lo; g = 7: zeros).
// bq[G / 4][t][G % 4] = r (t = 0), Q' (t = 3), 0 otherwise, with
// -128 sum(a) = r - 2^23 Q'.
__device__ __forceinline__ uint32_t mv_limbs4(const int32_t (&v)[8], int h, int g, uint32_t mul) {
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t c = (uint32_t)(v[2 * i + h] + (1 << 23));
    const uint32_t n = g < 6 ? (c >> (4 * g)) & 15u : (g == 6 ? 1u : 0u);
    r |= (n * mul) << (8 * i);
  }
  return r;
}

// One warp per group G and pass: lane (g, t) reads the 16 activations of its
// fragment (two 8-column runs), and the quad g = 0 sums the group for bq.
// nthreads is a multiple of 32, so each warp's lanes share one G.
__device__ __forceinline__ void mv_stage_b(const int32_t* __restrict__ act, int K, uint4* bf, int32_t* bq, int tid,
                                           int nthreads) {
  for (int e = tid; e < K / 2; e += nthreads) {
    const int G = e >> 5, gq = (e & 31) >> 2, t = e & 3;
    const int4* a = reinterpret_cast<const int4*>(act + 64 * G + 8 * t);
    const int4 p0 = a[0], p1 = a[1], p2 = a[8], p3 = a[9];
    const int32_t lo[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
    const int32_t hi[8] = {p2.x, p2.y, p2.z, p2.w, p3.x, p3.y, p3.z, p3.w};
    bf[e] = make_uint4(mv_limbs4(lo, 0, gq, 16), mv_limbs4(hi, 0, gq, 16), mv_limbs4(lo, 1, gq, 1),
                       mv_limbs4(hi, 1, gq, 1));
    int64_t sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += (int64_t)lo[i] + hi[i];
    sum += shfl_xor_i64(sum, 1);
    sum += shfl_xor_i64(sum, 2);
    if (gq == 0) {
      const int64_t nb = -128 * sum;  // |nb| <= 2^36
      bq[((G >> 2) * 4 + t) * 4 + (G & 3)] =
          t == 0 ? (int32_t)(nb & ((1 << 23) - 1)) : (t == 3 ? (int32_t)(-(nb >> 23)) : 0);
    }
  }
}

// The CTA's tiles [t0, t1) form blocks of up to four consecutive tiles of one
// matrix: in matrix m they start at max(t0, m * tpm) + 4 k.
struct MvBlocks {
  int t0, t1, tpm, m0, nb0, bpm;
  __device__ MvBlocks(int a, int b, int tiles_per_matrix, int count) : t0(a), t1(b), tpm(tiles_per_matrix) {
    m0 = count == 1 ? 0 : t0 / tpm;
    const int e0 = (m0 + 1) * tpm;
    nb0 = ((t1 < e0 ? t1 : e0) - t0 + 3) / 4;
    bpm = (tpm + 3) / 4;
  }
  // matrix, block ordinal and index inside the block of tile t
  __device__ void locate(int t, int count, int& m, int& ord, int& j) const {
    m = count == 1 ? 0 : t / tpm;
    const int sm = m == m0 ? t0 : m * tpm;
    const int k = (t - sm) >> 2;
    j = t - sm - 4 * k;
    ord = m == m0 ? k : nb0 + (m - m0 - 1) * bpm + k;
  }
};

template <int K, int MODE>
__global__ void __launch_bounds__(kMvThreads, 1) gemv_mma_kernel(const __grid_constant__ MvMaps maps, GemvArgs g) {
  using C = MvCfg<K>;
  constexpr int KS = C::KS, NS = C::NS;
  extern __shared__ __align__(1024) unsigned char mv_smem_raw[];
  // the 128-byte swizzle repeats every 1024 bytes: slots start on that boundary
  uint8_t* slots = reinterpret_cast<uint8_t*>(((uintptr_t)mv_smem_raw + 1023) & ~(uintptr_t)1023);
  uint4* bf = reinterpret_cast<uint4*>(slots + NS * kMvSlot);
  int32_t* bq = reinterpret_cast<int32_t*>(bf + K / 2);
  uint64_t* full = reinterpret_cast<uint64_t*>(bq + K / 16);
  uint64_t* empty = full + NS;
  // tag[s]: the unit last issued into slot s.  A consumer that claimed a tile
  // far ahead waits for its unit's tag before the parity wait, so the parity
  // it waits on is never two phases away.
  volatile int* tag = reinterpret_cast<volatile int*>(empty + NS);
  __shared__ ArgBest wbest[kMvWarps + 1];
  __shared__ bool last;
  __shared__ int next_tile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tg = lane & 3;
  const int tpm = (g.rows + 15) >> 4;  // 16-row tiles per matrix (count * tpm < 2^31)
  const int64_t total = (int64_t)tpm * g.count;
  const int t0 = (int)(total * blockIdx.x / gridDim.x), t1 = (int)(total * (blockIdx.x + 1) / gridDim.x);
  const int ntile = t1 - t0;
  const MvBlocks blocks(t0, t1, tpm, g.count);
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      gv_bar_init(full + s);
      gv_bar_init_n(empty + s, 4);
      tag[s] = -1;
    }
    next_tile = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // the weights do not depend on earlier kernels: the next launch may start
  // its own weight loads now, and this one waits only before reading the
  // activation (programmatic dependent launch)
  grid_dep_launch();
  int64_t best_s = INT64_MIN;
  int32_t best_i = INT32_MAX;
  if (warp == kMvWarps) {
    // producer: the blocks in order, one unit (1024 columns) at a time
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.w64)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.s64)) : "memory");
      int ord = 0;
      bool ok = true;
      for (int tb = t0; ok && tb < t1; ++ord) {
        const int m = g.count == 1 ? 0 : tb / tpm;
        const int me = (m + 1) * tpm;
        const int n = min(4, (t1 < me ? t1 : me) - tb);
        const int row0 = (tb - m * tpm) * 16;
        for (int c = 0; c < KS; ++c) {
          const int u = ord * KS + c, s = u % NS;
          if (u >= NS && !mv_wait(empty + s, ((u / NS) - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t* dst = slots + s * kMvSlot;
          tag[s] = u;
          if (n == 4) {
            gv_expect(full + s, kMvSlot);
#pragma unroll
            for (int b = 0; b < 4; ++b) mv_tma3(dst + b * kMvBox, &maps.w64, c * 512 + b * 128, row0, m, full + s);
            mv_tma3(dst + 4 * kMvBox, &maps.s64, c * 32, row0, m, full + s);
          } else {
            gv_expect(full + s, (uint32_t)n * (4 * 2048 + 512));
            for (int j = 0; j < n; ++j) {
#pragma unroll
              for (int b = 0; b < 4; ++b)
                mv_tma3(dst + b * kMvBox + j * 2048, &maps.w16, c * 512 + b * 128, row0 + 16 * j, m, full + s);
              mv_tma3(dst + 4 * kMvBox + j * 512, &maps.s16, c * 32, row0 + 16 * j, m, full + s);
            }
            mv_arrive_n(empty + s, 4 - n);  // the block's missing tiles
          }
        }
        tb += n;
      }
    }
  } else {
    grid_dep_wait();
    mv_stage_b(g.act, K, bf, bq, tid, kMvWarps * 32);
    mv_consumer_sync();
    const MvMasks mk;
    // swizzled byte offsets of words t (ox0) and t + 4 (ox1) of group G, G % 4 = G4, in row gid of a box
    uint32_t ox0[4], ox1[4];
#pragma unroll
    for (int G4 = 0; G4 < 4; ++G4) {
      ox0[G4] = (uint32_t)(gid * 128 + (((2 * G4) ^ gid) << 4) + 4 * tg);
      ox1[G4] = (uint32_t)(gid * 128 + (((2 * G4 + 1) ^ gid) << 4) + 4 * tg);
    }
    for (;;) {
      int ti = 0;
      if (lane == 0) ti = atomicAdd(&next_tile, 1);
      ti = __shfl_sync(0xFFFFFFFFu, ti, 0);
      if (ti >= ntile) break;
      const int tile = t0 + ti;
      int m, ord, j;
      blocks.locate(tile, g.count, m, ord, j);
      const int row0 = (tile - m * tpm) * 16;
      int64_t acc0 = 0, acc1 = 0;  // rows row0 + gid, row0 + gid + 8
#pragma unroll 1
      for (int c = 0; c < KS; ++c) {
        const int u = ord * KS + c, s = u % NS;
        const bool ok = mv_wait_tag(tag + s, u) && mv_wait(full + s, (u / NS) & 1);
        // this tile's words and scales into registers, then the slot goes back
        const uint8_t* st = slots + s * kMvSlot + j * 2048;
        const uint8_t* sc = slots + s * kMvSlot + 4 * kMvBox + (16 * j + gid) * 32;
        uint32_t xw[16][4];
        uint4 sv[4];
#pragma unroll
        for (int GG = 0; GG < 16; ++GG) {
          const uint8_t* bx = st + (GG >> 2) * kMvBox;
          xw[GG][0] = *reinterpret_cast<const uint32_t*>(bx + ox0[GG & 3]);
          xw[GG][1] = *reinterpret_cast<const uint32_t*>(bx + ox1[GG & 3]);
          xw[GG][2] = *reinterpret_cast<const uint32_t*>(bx + 1024 + ox0[GG & 3]);
          xw[GG][3] = *reinterpret_cast<const uint32_t*>(bx + 1024 + ox1[GG & 3]);
        }
        sv[0] = *reinterpret_cast<const uint4*>(sc);
        sv[1] = *reinterpret_cast<const uint4*>(sc + 16);
        sv[2] = *reinterpret_cast<const uint4*>(sc + 8 * 32);
        sv[3] = *reinterpret_cast<const uint4*>(sc + 8 * 32 + 16);
        __syncwarp();
        if (lane == 0) gv_arrive(empty + s);
        if (!ok) continue;
        const uint4* bsm = bf + c * 512 + lane;
        const int4* bqs = reinterpret_cast<const int4*>(bq + c * 64) + tg;
#pragma unroll
        for (int GG = 0; GG < 16; ++GG) {
          const uint4 b = bsm[GG * 32];
          const int4 q4 = bqs[(GG >> 2) * 4];
          const int32_t q = (GG & 3) == 0 ? q4.x : (GG & 3) == 1 ? q4.y : (GG & 3) == 2 ? q4.z : q4.w;
          int32_t d[4];
          mma_u8_init(d, mk.lo(xw[GG][0]), mk.lo(xw[GG][2]), mk.lo(xw[GG][1]), mk.lo(xw[GG][3]), b.x, b.y, q);
          mma_u8(d, mk.hi(xw[GG][0]), mk.hi(xw[GG][2]), mk.hi(xw[GG][1]), mk.hi(xw[GG][3]), b.z, b.w);
          const uint32_t w0 = reinterpret_cast<const uint32_t*>(&sv[GG >> 3])[(GG >> 1) & 3];
          const uint32_t w1 = reinterpret_cast<const uint32_t*>(&sv[2 + (GG >> 3)])[(GG >> 1) & 3];
          const int32_t sa = (int32_t)((GG & 1) ? (w0 >> 16) : (w0 & 0xFFFFu));
          const int32_t sb = (int32_t)((GG & 1) ? (w1 >> 16) : (w1 & 0xFFFFu));
          acc0 = mad_wide(d[0] + 16 * d[1], sa, acc0);
          acc1 = mad_wide(d[2] + 16 * d[3], sb, acc1);
        }
      }
      // lane weights 1, 2^8, 2^16, -2^23; the sum over the quad is 16 x the row sum
      acc0 <<= 8 * tg - (tg == 3);
      acc1 <<= 8 * tg - (tg == 3);
      if (tg == 3) {
        acc0 = -acc0;
        acc1 = -acc1;
      }
      acc0 += shfl_xor_i64(acc0, 1);
      acc1 += shfl_xor_i64(acc1, 1);
      acc0 += shfl_xor_i64(acc0, 2);
      acc1 += shfl_xor_i64(acc1, 2);
      if (tg == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = row0 + gid + 8 * r;
          const int64_t v = (r ? acc1 : acc0) >> 4;
          if (row < g.rows) {
            if constexpr (MODE == 0) {
              g.out[m * g.out_stride + row] = v;
              if (g.out12) g.out12[m * g.out_stride + row] = sat24c(v >> 14, g.sat);
            } else {
              if (g.out) g.out[row] = v;
              if (better(v, row, best_s, best_i)) {
                best_s = v;
                best_i = row;
              }
            }
          }
        }
      }
    }
  }
  if constexpr (MODE == 1) {
    auto warp_best = [&](int64_t& bs, int32_t& bi) {
#pragma unroll
      for (int msk = 1; msk < 32; msk <<= 1) {
        const int64_t os = shfl_xor_i64(bs, msk);
        const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, msk);
        if (better(os, oi, bs, bi)) {
          bs = os;
          bi = oi;
        }
      }
    };
    __syncwarp();
    warp_best(best_s, best_i);
    if (lane == 0) wbest[warp] = ArgBest{best_s, best_i, 0};
    __syncthreads();
    if (tid == 0) {
      ArgBest b = wbest[0];
      for (int w = 1; w <= kMvWarps; ++w)
        if (better(wbest[w].score, wbest[w].idx, b.score, b.idx)) b = wbest[w];
      g.partial[blockIdx.x] = b;
      __threadfence();
      const unsigned int done = atomicAdd(g.counter, 1u);
      last = (done == gridDim.x - 1);
    }
    __syncthreads();
    if (last) {  // the last CTA reduces all partials, every thread a strided share
      __threadfence();
      int64_t bs = INT64_MIN;
      int32_t bi = INT32_MAX;
      for (int i = tid; i < (int)gridDim.x; i += kMvThreads) {
        const int64_t cs = *((volatile int64_t*)&g.partial[i].score);
        const int32_t ci = *((volatile int32_t*)&g.partial[i].idx);
        if (better(cs, ci, bs, bi)) {
          bs = cs;
          bi = ci;
        }
      }
      warp_best(bs, bi);
      __syncthreads();
      if (lane == 0) wbest[warp] = ArgBest{bs, bi, 0};
      __syncthreads();
      if (tid == 0) {
        ArgBest b = wbest[0];
        for (int w = 1; w <= kMvWarps; ++w)
          if (better(wbest[w].score, wbest[w].idx, b.score, b.idx)) b = wbest[w];
        *g.out_tok = b.idx;
        *g.out_score = b.score;
        *g.counter = 0;  // ready for the next launch
      }
    }
  }
}

// Scratch of q4gpu_lm_head_argmax_noalloc: the per-CTA best (score, row) of
// the LM-head grid and its completion counter, 444 * 16 + 16 = 7120 bytes,
// resident on every device that loads this library.
struct LmHeadStaticScratch {
  ArgBest partial[Q4GPU_LM_HEAD_BLOCKS];
  unsigned int counter;
  unsigned int pad[3];
};
static __device__ __align__(256) LmHeadStaticScratch g_lm_head_static_scratch;

}  // namespace q4

// ===========================================================================
// C ABI: per-module entry points
// ===========================================================================
using namespace q4;

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int q4gpu_synth_f32(uint64_t seed, uint64_t tensor_id, int64_t start, int64_t n, float std_dev, int bf16,
                    float* out, void* stream) {
  if (!out || n < 0) return Q4GPU_ERR_ARG;
  if (n == 0) return Q4GPU_OK;
  const float k = std_dev * (1.0f / 65536.0f);
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  synth_f32_kernel<<<blocks, 256, 0, as_stream(stream)>>>(stream_key(seed, tensor_id), start, n, k, bf16, out);
  return q4gpu_check_launch();
}

int q4gpu_quantize_q4(const float* w, int64_t rows, int32_t cols, uint8_t* packed, uint16_t* scale, int32_t* err_flag,
                      void* stream) {
  if (!w || !packed || !scale || !err_flag || rows <= 0 || cols <= 0 || cols % kGroup) return Q4GPU_ERR_ARG;
  if (((uintptr_t)w) & 15) return Q4GPU_ERR_ALIGN;
  const int64_t total = rows * (cols / kGroup);
  const int blocks = (int)std::min<int64_t>((total + 127) / 128, 148 * 32);
  quantize_q4_kernel<<<blocks, 128, 0, as_stream(stream)>>>(w, rows, cols, packed, scale, err_flag);
  return q4gpu_check_launch();
}

}  // extern "C"

namespace {

// 3-D u8 tensor map [count][rows][inner bytes] with a box of box_inner x box_rows x 1
int mv_encode(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t count, uint64_t row_stride,
              uint64_t mat_stride, uint32_t box_inner, uint32_t box_rows, bool swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !encode)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  }
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)count};
  const cuuint64_t strides[2] = {(cuuint64_t)row_stride, (cuuint64_t)mat_stride};
  const cuuint32_t box[3] = {box_inner, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE,
                            swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q4GPU_OK;
}

// Tensor maps of one GEMV operand set, cached by its pointers and shape (a
// model's GEMVs repeat every token).
int mv_maps(const GemvArgs& g, int K, MvMaps* out) {
  struct Entry {
    const void* W;
    const void* S;
    int K, rows, count;
    int64_t ws, ss;
    MvMaps maps;
  };
  static Entry cache[32];
  static int n_used = 0, next = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_used; ++i) {
    const Entry& e = cache[i];
    if (e.W == g.W && e.S == g.S && e.K == K && e.rows == g.rows && e.count == g.count && e.ws == g.w_stride &&
        e.ss == g.s_stride) {
      *out = e.maps;
      return Q4GPU_OK;
    }
  }
  Entry e{g.W, g.S, K, g.rows, g.count, g.w_stride, g.s_stride, {}};
  const uint64_t wrow = (uint64_t)K / 2, srow = (uint64_t)K / 32;
  const uint64_t wmat = g.count > 1 ? (uint64_t)g.w_stride : wrow * g.rows;
  const uint64_t smat = g.count > 1 ? (uint64_t)g.s_stride * 2 : srow * g.rows;
  int rc = mv_encode(&e.maps.w64, g.W, wrow, g.rows, g.count, wrow, wmat, 128, 64, true);
  if (rc == Q4GPU_OK) rc = mv_encode(&e.maps.w16, g.W, wrow, g.rows, g.count, wrow, wmat, 128, 16, true);
  if (rc == Q4GPU_OK) rc = mv_encode(&e.maps.s64, g.S, srow, g.rows, g.count, srow, smat, 32, 64, false);
  if (rc == Q4GPU_OK) rc = mv_encode(&e.maps.s16, g.S, srow, g.rows, g.count, srow, smat, 32, 16, false);
  if (rc != Q4GPU_OK) return rc;
  cache[next] = e;
  next = (next + 1) % 32;
  if (n_used < 32) ++n_used;
  *out = e.maps;
  return Q4GPU_OK;
}

template <int K, int MODE>
int mv_launch(const GemvArgs& g, int grid_cap, cudaStream_t s) {
  using C = MvCfg<K>;
  static_assert(C::SMEM <= 227 * 1024 - 512, "GEMV slot ring too large");
  MvMaps maps;
  const int rc = mv_maps(g, K, &maps);
  if (rc != Q4GPU_OK) return rc;
  const cudaError_t e =
      cudaFuncSetAttribute(gemv_mma_kernel<K, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "GEMV shared memory: %s", cudaGetErrorString(e));
  const int64_t tiles = (int64_t)((g.rows + 15) / 16) * g.count;
  // at least two 16-row tiles per CTA: a small matrix leaves SMs free for the
  // next launch, whose weight loads then overlap this one (PDL)
  const int grid = (int)std::min<int64_t>((tiles + 1) / 2, std::min(grid_cap, 148));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMvThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, gemv_mma_kernel<K, MODE>, maps, g);
  if (le != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "GEMV launch: %s", cudaGetErrorString(le));
  return q4gpu_check_launch();
}

template <int K, int MODE>
int gv_launch(const GemvArgs& g, int grid_cap, cudaStream_t s) {
  // tensor-core path when the scale rows can travel by bulk copy (16-byte aligned)
  if (((uintptr_t)g.S & 15) == 0 && ((g.s_stride * 2) & 15) == 0 && (g.act_stride == 0 || g.count == 1))
    return mv_launch<K, MODE>(g, grid_cap, s);
  using C = GvCfg<K>;
  static_assert(C::SMEM < 227 * 1024, "GEMV stage ring too large");
  // scales ride with the weights when every stage's scale rows start 16-byte aligned
  const bool sbulk = ((uintptr_t)g.S & 15) == 0 && ((g.s_stride * 2) & 15) == 0;
  auto kern = sbulk ? gemv_stream_kernel<K, MODE, true> : gemv_stream_kernel<K, MODE, false>;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "GEMV shared memory: %s", cudaGetErrorString(e));
  const int64_t units = (int64_t)((g.rows + C::SR - 1) / C::SR) * g.count;
  const int grid = (int)std::min<int64_t>(units, grid_cap);
  kern<<<grid, kGvThreads, C::SMEM, s>>>(g);
  return q4gpu_check_launch();
}

// CTAs per SM that fit the stage ring (x148 SMs), capped by the LM-head partial array
int gv_grid_cap(int K) { return (K == 1024 ? 3 : 2) * 148; }

template <int MODE>
int gv_dispatch(int K, const GemvArgs& g, int grid_cap, cudaStream_t s) {
  switch (K) {
    case 1024: return gv_launch<1024, MODE>(g, grid_cap, s);
    case 2048: return gv_launch<2048, MODE>(g, grid_cap, s);
    case 3072: return gv_launch<3072, MODE>(g, grid_cap, s);
    case 4096: return gv_launch<4096, MODE>(g, grid_cap, s);
    default: return q4gpu_fail(Q4GPU_ERR_SHAPE, "GEMV K must be 1024, 2048, 3072 or 4096 (got %d)", K);
  }
}

}  // namespace

extern "C" {

int q4gpu_gemv_q26(const int32_t* act, int32_t k, const uint8_t* packed, const uint16_t* scale, int32_t rows,
                   int64_t* out_q26, int32_t* out_q12_12, int32_t* sat_count, void* stream) {
  if (!act || !packed || !scale || !out_q26 || rows <= 0) return Q4GPU_ERR_ARG;
  if ((((uintptr_t)packed) & 15) || (((uintptr_t)scale) & 1) || (((uintptr_t)act) & 15)) return Q4GPU_ERR_ALIGN;
  if (k != 1024 && k != 2048 && k != 3072 && k != 4096) return Q4GPU_ERR_SHAPE;
  GemvArgs g{};
  g.act = act;
  g.W = packed;
  g.S = scale;
  g.rows = rows;
  g.count = 1;
  g.out = out_q26;
  g.out12 = out_q12_12;
  g.sat = sat_count;
  return gv_dispatch<0>(k, g, gv_grid_cap(k), as_stream(stream)) == Q4GPU_OK ? Q4GPU_OK : Q4GPU_ERR_CUDA;
}

int q4gpu_gemv_q26_strided(const int32_t* act, int64_t act_stride, int32_t k, const uint8_t* packed,
                           int64_t packed_stride, const uint16_t* scale, int64_t scale_stride, int32_t rows,
                           int32_t count, int64_t* out_q26, int32_t* out_q12_12, int64_t out_stride,
                           int32_t* sat_count, void* stream) {
  if (!act || !packed || !scale || !out_q26 || rows <= 0 || count <= 0 || act_stride < 0 ||
      out_stride < (count > 1 ? rows : 0))
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad strided GEMV arguments");
  if ((((uintptr_t)packed) & 15) || (packed_stride & 15) || (((uintptr_t)scale) & 1) || (((uintptr_t)act) & 15) ||
      (act_stride & 3))
    return q4gpu_fail(Q4GPU_ERR_ALIGN, "activations, packed weights and their strides must be 16-byte aligned");
  if (k != 1024 && k != 2048 && k != 3072 && k != 4096)
    return q4gpu_fail(Q4GPU_ERR_SHAPE, "GEMV K must be 1024, 2048, 3072 or 4096 (got %d)", k);
  if (count > 1 && (packed_stride < (int64_t)rows * k / 2 || scale_stride < (int64_t)rows * k / 64))
    return q4gpu_fail(Q4GPU_ERR_ARG, "matrix strides overlap");
  GemvArgs g{};
  g.act = act;
  g.act_stride = act_stride;
  g.W = packed;
  g.w_stride = packed_stride;
  g.S = scale;
  g.s_stride = scale_stride;
  g.rows = rows;
  g.count = count;
  g.out = out_q26;
  g.out_stride = out_stride;
  g.out12 = out_q12_12;
  g.sat = sat_count;
  return gv_dispatch<0>(k, g, gv_grid_cap(k), as_stream(stream));
}

int q4gpu_rmsnorm(const int32_t* x, const int32_t* gamma, int32_t rows, int32_t n, int32_t mode, int32_t* out,
                  int64_t* stats, void* stream) {
  if (!x || !gamma || !out || rows <= 0 || n <= 0 || (mode != 0 && mode != 1)) return Q4GPU_ERR_ARG;
  rmsnorm_kernel<<<rows, 256, 0, as_stream(stream)>>>(x, gamma, n, mode, out, stats);
  return q4gpu_check_launch();
}

int q4gpu_rope(const int32_t* x, int32_t heads, const int32_t* cos_q1_15, const int32_t* sin_q1_15, int32_t* out,
               int32_t* sat_count, void* stream) {
  if (!x || !cos_q1_15 || !sin_q1_15 || !out || heads <= 0) return Q4GPU_ERR_ARG;
  rope_kernel<<<heads, kHeadDim, 0, as_stream(stream)>>>(x, heads, cos_q1_15, sin_q1_15, out, sat_count);
  return q4gpu_check_launch();
}

int q4gpu_attention_scores(const int32_t* q, const int32_t* k_cache, int32_t ctx, int32_t q_heads, int32_t kv_heads,
                           int64_t scale_q0_31, int64_t* raw, int64_t* scaled, void* stream) {
  if (!q || !k_cache || !raw || !scaled || ctx <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return Q4GPU_ERR_ARG;
  dim3 grid((ctx + 127) / 128, q_heads);
  attn_scores_kernel<<<grid, 128, 0, as_stream(stream)>>>(q, k_cache, ctx, q_heads, kv_heads, scale_q0_31, raw,
                                                          scaled);
  return q4gpu_check_launch();
}

int q4gpu_softmax_probs(const int64_t* scores, int32_t rows, int32_t ctx, const int32_t* exp_lut, int32_t* probs,
                        int32_t* lut_index, void* stream) {
  if (!scores || !exp_lut || !probs || rows <= 0 || ctx <= 0) return Q4GPU_ERR_ARG;
  softmax_kernel<<<rows, 256, 0, as_stream(stream)>>>(scores, ctx, exp_lut, probs, lut_index);
  return q4gpu_check_launch();
}

int q4gpu_value_accum(const int32_t* probs, const int32_t* v_cache, int32_t ctx, int32_t q_heads, int32_t kv_heads,
                      int32_t* out, int32_t* sat_count, void* stream) {
  if (!probs || !v_cache || !out || ctx <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
    return Q4GPU_ERR_ARG;
  value_accum_kernel<<<q_heads, kHeadDim, 0, as_stream(stream)>>>(probs, v_cache, ctx, q_heads, kv_heads, out,
                                                                  sat_count);
  return q4gpu_check_launch();
}

int q4gpu_silu_mul(const int32_t* gate, const int32_t* up, int32_t n, const int32_t* sigmoid_lut, int32_t* hidden,
                   int32_t* silu, int32_t* lut_index, int32_t* sat_counts, void* stream) {
  if (!gate || !up || !sigmoid_lut || !hidden || n <= 0) return Q4GPU_ERR_ARG;
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(gate, up, n, sigmoid_lut, hidden, silu, lut_index,
                                                                  sat_counts);
  return q4gpu_check_launch();
}

int q4gpu_residual_add(const int32_t* a, const int32_t* b, int32_t n, int32_t shift, int32_t* out, int32_t* sat_count,
                       void* stream) {
  if (!a || !b || !out || n <= 0 || shift < 0 || shift > 31) return Q4GPU_ERR_ARG;
  residual_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(a, b, n, shift, out, sat_count);
  return q4gpu_check_launch();
}

int q4gpu_q26_to_q12_12(const int64_t* in_q26, int32_t n, int32_t* out_q12_12, int32_t* sat_count, void* stream) {
  if (!in_q26 || !out_q12_12 || n <= 0) return Q4GPU_ERR_ARG;
  q26_to_q12_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(in_q26, n, out_q12_12, sat_count);
  return q4gpu_check_launch();
}

int q4gpu_embedding(const int32_t* tokens, int32_t n_tokens, const uint8_t* packed, const uint16_t* scale,
                    int32_t* out, void* stream) {
  if (!tokens || !packed || !scale || !out || n_tokens <= 0) return Q4GPU_ERR_ARG;
  embedding_kernel<<<n_tokens, 256, 0, as_stream(stream)>>>(tokens, packed, scale, out);
  return q4gpu_check_launch();
}

size_t q4gpu_lm_head_workspace_bytes(int32_t rows) {
  (void)rows;
  return (size_t)Q4GPU_LM_HEAD_BLOCKS * sizeof(ArgBest) + 256;
}

int q4gpu_lm_head_argmax(const int32_t* act, const uint8_t* packed, const uint16_t* scale, int32_t rows,
                         int64_t* logits, void* workspace, size_t workspace_bytes, int32_t* out_token,
                         int64_t* out_score, void* stream) {
  if (!act || !packed || !scale || !workspace || !out_token || !out_score)
    return q4gpu_fail(Q4GPU_ERR_ARG, "null argument");
  if (rows <= 0) return q4gpu_fail(Q4GPU_ERR_ARG, "rows %d must be positive", rows);
  if (workspace_bytes < q4gpu_lm_head_workspace_bytes(rows))
    return q4gpu_fail(Q4GPU_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", workspace_bytes,
                      q4gpu_lm_head_workspace_bytes(rows));
  if ((((uintptr_t)packed) & 15) || (((uintptr_t)workspace) & 15) || (((uintptr_t)act) & 15))
    return q4gpu_fail(Q4GPU_ERR_ALIGN, "activation, packed weights and workspace must be 16-byte aligned");
  if (((uintptr_t)scale) & 1) return q4gpu_fail(Q4GPU_ERR_ALIGN, "scales must be 2-byte aligned");
  ArgBest* partial = reinterpret_cast<ArgBest*>(workspace);
  unsigned int* counter =
      reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(workspace) + Q4GPU_LM_HEAD_BLOCKS * sizeof(ArgBest));
  const cudaError_t ce = cudaMemsetAsync(counter, 0, sizeof(unsigned int), as_stream(stream));
  if (ce != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "workspace clear: %s", cudaGetErrorString(ce));
  GemvArgs g{};
  g.act = act;
  g.W = packed;
  g.S = scale;
  g.rows = rows;
  g.count = 1;
  g.out = logits;
  g.partial = partial;
  g.counter = counter;
  g.out_tok = out_token;
  g.out_score = out_score;
  return gv_dispatch<1>(kHidden, g, gv_grid_cap(kHidden), as_stream(stream));
}

// Device address of g_lm_head_static_scratch in the calling thread's current
// CUDA context.  A __device__ symbol exists once per context (the primary
// context of a device, or a caller's own driver-API context), so the address
// is looked up with cudaGetSymbolAddress, with that context current, the first
// time each context calls, and cached under the context's unique id
// (cuCtxGetId: ids are never reused, so a reset device or a destroyed and
// re-created context gets a fresh lookup).  In host code the symbol itself is
// only a host-side stand-in; kernels get this address.
static int lm_head_static_scratch(q4::LmHeadStaticScratch** out) {
  static std::mutex mu;
  static std::vector<std::pair<unsigned long long, void*>> by_ctx;
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!get_current || !get_id) {
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", reinterpret_cast<void**>(&get_current), cudaEnableDefault, &q1) !=
            cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", reinterpret_cast<void**>(&get_id), cudaEnableDefault, &q2) !=
            cudaSuccess ||
        q2 != cudaDriverEntryPointSuccess) {
      get_current = nullptr;
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId unavailable");
    }
  }
  void* p = nullptr;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuCtxGetCurrent failed");
  if (!ctx) {
    // no context current yet on this thread: the runtime call makes the
    // device's primary context current
    const cudaError_t e = cudaGetSymbolAddress(&p, q4::g_lm_head_static_scratch);
    if (e != cudaSuccess)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cudaGetSymbolAddress(lm-head scratch): %s", cudaGetErrorString(e));
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return q4gpu_fail(Q4GPU_ERR_CUDA, "no current CUDA context");
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuCtxGetId failed");
  for (const auto& e : by_ctx)
    if (e.first == id) {
      *out = static_cast<q4::LmHeadStaticScratch*>(e.second);
      return Q4GPU_OK;
    }
  if (!p) {
    const cudaError_t e = cudaGetSymbolAddress(&p, q4::g_lm_head_static_scratch);
    if (e != cudaSuccess)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cudaGetSymbolAddress(lm-head scratch): %s", cudaGetErrorString(e));
  }
  by_ctx.emplace_back(id, p);
  *out = static_cast<q4::LmHeadStaticScratch*>(p);
  return Q4GPU_OK;
}

int q4gpu_lm_head_argmax_noalloc(const int32_t* act, const uint8_t* packed, const uint16_t* scale, int32_t rows,
                                 int64_t* logits, int32_t* out_token, int64_t* out_score, void* stream) {
  if (!act || !packed || !scale || !out_token || !out_score) return q4gpu_fail(Q4GPU_ERR_ARG, "null argument");
  if (rows <= 0 || rows > Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS)
    return q4gpu_fail(Q4GPU_ERR_ARG, "rows %d outside 1..%d supported by the static LM-head scratch", rows,
                      Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS);
  if ((((uintptr_t)packed) & 15) || (((uintptr_t)act) & 15))
    return q4gpu_fail(Q4GPU_ERR_ALIGN, "activation and packed weights must be 16-byte aligned");
  if (((uintptr_t)scale) & 1) return q4gpu_fail(Q4GPU_ERR_ALIGN, "scales must be 2-byte aligned");
  q4::LmHeadStaticScratch* sc = nullptr;
  int rc = lm_head_static_scratch(&sc);
  if (rc) return rc;
  // the completion counter must start at zero (the kernel leaves it at zero,
  // but an earlier call may have been cut short)
  const cudaError_t e = cudaMemsetAsync(&sc->counter, 0, sizeof(unsigned int), as_stream(stream));
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "scratch clear: %s", cudaGetErrorString(e));
  GemvArgs g{};
  g.act = act;
  g.W = packed;
  g.S = scale;
  g.rows = rows;
  g.count = 1;
  g.out = logits;
  g.partial = sc->partial;
  g.counter = &sc->counter;
  g.out_tok = out_token;
  g.out_score = out_score;
  return gv_dispatch<1>(kHidden, g, gv_grid_cap(kHidden), as_stream(stream));
}

}  // extern "C"
