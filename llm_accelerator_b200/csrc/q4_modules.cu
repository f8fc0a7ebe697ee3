// Per-module kernels: one CUDA kernel (or fused pair) per stage of the
// reference's fixed-point decode path, exposed through the C ABI in
// include/q4gpu.h so each stage can be checked bit-exactly on its own.
// The decode-step kernels (q4_decode.cu) fuse these same stages.
#include <mutex>

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
// GEMV -> Q26 row sums (+ optional Q12.12 words).  One warp per R rows per
// 1024-column slice; K slices of a row are combined in shared memory.
// ---------------------------------------------------------------------------
template <int K, int R>
__global__ void __launch_bounds__(256) gemv_q26_kernel(const int32_t* __restrict__ act, const uint8_t* __restrict__ W,
                                                       const uint16_t* __restrict__ S, int rows,
                                                       int64_t* __restrict__ out_q26, int32_t* __restrict__ out_q12,
                                                       int32_t* __restrict__ sat) {
  constexpr int KS = K / 1024;
  constexpr int NW = 8;
  constexpr int ROW_GROUPS = NW / KS > 0 ? NW / KS : 1;  // warps per K-slice
  extern __shared__ __align__(16) unsigned char smem[];
  int32_t* a = reinterpret_cast<int32_t*>(smem);
  uint32_t* limbs = reinterpret_cast<uint32_t*>(a + K);
  int64_t* bias8 = reinterpret_cast<int64_t*>(limbs + limb_words(K));
  int64_t* part = bias8 + K / 32;  // [KS][ROW_GROUPS*R]
  for (int i = threadIdx.x; i < K; i += blockDim.x) a[i] = act[i];
  __syncthreads();
  stage_limbs(a, K, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = warp % KS;
  const int rg = warp / KS;
  const int rows_per_block = ROW_GROUPS * R;
  for (int base = blockIdx.x * rows_per_block; base < rows; base += gridDim.x * rows_per_block) {
    int64_t acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0;
    if (rg < ROW_GROUPS) {
      gemv_slice<K, R>(W, S, base + rg * R, rows, ks, limbs, bias8, acc);
      warp_reduce_rows<R>(acc);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; ++r) part[ks * rows_per_block + rg * R + r] = acc[r];
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rows_per_block; i += blockDim.x) {
      const int row = base + i;
      if (row < rows) {
        int64_t s = 0;
#pragma unroll
        for (int k = 0; k < KS; ++k) s += part[k * rows_per_block + i];
        out_q26[row] = s;
        if (out_q12) out_q12[row] = sat24c(s >> 14, sat);
      }
    }
    __syncthreads();
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
struct ArgBest {
  int64_t score;
  int32_t idx;
  int32_t pad;
};

__device__ __forceinline__ bool better(int64_t s, int32_t i, int64_t bs, int32_t bi) {
  return s > bs || (s == bs && i < bi);
}

template <int R>
__global__ void __launch_bounds__(256) lm_head_kernel(const int32_t* __restrict__ act, const uint8_t* __restrict__ W,
                                                      const uint16_t* __restrict__ S, int rows,
                                                      int64_t* __restrict__ logits, ArgBest* __restrict__ partial,
                                                      unsigned int* __restrict__ counter, int32_t* __restrict__ out_tok,
                                                      int64_t* __restrict__ out_score) {
  constexpr int K = kHidden;
  __shared__ __align__(16) int32_t a[K];
  __shared__ __align__(16) uint32_t limbs[limb_words(K)];
  __shared__ int64_t bias8[K / 32];
  __shared__ ArgBest wbest[8];
  __shared__ bool last;
  for (int i = threadIdx.x; i < K; i += blockDim.x) a[i] = act[i];
  __syncthreads();
  stage_limbs(a, K, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  int64_t best_s = INT64_MIN;
  int32_t best_i = INT32_MAX;
  for (int base = (blockIdx.x * nw + warp) * R; base < rows; base += gridDim.x * nw * R) {
    int64_t acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0;
    gemv_slice<K, R>(W, S, base, rows, 0, limbs, bias8, acc);
    warp_reduce_rows<R>(acc);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = base + r;
      if (row < rows) {
        if (logits && lane == r) logits[row] = acc[r];
        if (acc[r] > best_s) {  // rows visited in ascending order within a warp
          best_s = acc[r];
          best_i = row;
        }
      }
    }
  }
  if (lane == 0) wbest[warp] = ArgBest{best_s, best_i, 0};
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgBest b = wbest[0];
    for (int w = 1; w < nw; ++w)
      if (better(wbest[w].score, wbest[w].idx, b.score, b.idx)) b = wbest[w];
    partial[blockIdx.x] = b;
    __threadfence();
    const unsigned int done = atomicAdd(counter, 1u);
    last = (done == gridDim.x - 1);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    ArgBest b = partial[0];
    for (int i = 1; i < (int)gridDim.x; ++i) {
      const ArgBest c{*((volatile int64_t*)&partial[i].score), *((volatile int32_t*)&partial[i].idx), 0};
      if (better(c.score, c.idx, b.score, b.idx)) b = c;
    }
    *out_tok = b.idx;
    *out_score = b.score;
    *counter = 0;  // ready for the next launch
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

int q4gpu_gemv_q26(const int32_t* act, int32_t k, const uint8_t* packed, const uint16_t* scale, int32_t rows,
                   int64_t* out_q26, int32_t* out_q12_12, int32_t* sat_count, void* stream) {
  if (!act || !packed || !scale || !out_q26 || rows <= 0) return Q4GPU_ERR_ARG;
  if ((((uintptr_t)packed) & 15) || (((uintptr_t)scale) & 1)) return Q4GPU_ERR_ALIGN;
  constexpr int R = 4;
  auto launch = [&](auto kern, int K) {
    const int KS = K / 1024;
    const int rows_per_block = (8 / KS) * R;
    const size_t smem = K * 4 + limb_words(K) * 4 + (K / 32) * 8 + KS * rows_per_block * 8;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int blocks = std::min((rows + rows_per_block - 1) / rows_per_block, 148 * 8);
    kern<<<blocks, 256, smem, as_stream(stream)>>>(act, packed, scale, rows, out_q26, out_q12_12, sat_count);
  };
  switch (k) {
    case 1024: launch(gemv_q26_kernel<1024, R>, 1024); break;
    case 2048: launch(gemv_q26_kernel<2048, R>, 2048); break;
    case 3072: launch(gemv_q26_kernel<3072, R>, 3072); break;
    case 4096: launch(gemv_q26_kernel<4096, R>, 4096); break;
    default: return Q4GPU_ERR_SHAPE;
  }
  return q4gpu_check_launch();
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
  if (!act || !packed || !scale || rows <= 0 || !workspace || !out_token || !out_score) return Q4GPU_ERR_ARG;
  if (workspace_bytes < q4gpu_lm_head_workspace_bytes(rows)) return Q4GPU_ERR_WORKSPACE;
  if ((((uintptr_t)packed) & 15) || (((uintptr_t)workspace) & 15)) return Q4GPU_ERR_ALIGN;
  ArgBest* partial = reinterpret_cast<ArgBest*>(workspace);
  unsigned int* counter =
      reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(workspace) + Q4GPU_LM_HEAD_BLOCKS * sizeof(ArgBest));
  cudaMemsetAsync(counter, 0, sizeof(unsigned int), as_stream(stream));
  lm_head_kernel<4><<<Q4GPU_LM_HEAD_BLOCKS, 256, 0, as_stream(stream)>>>(act, packed, scale, rows, logits, partial,
                                                                          counter, out_token, out_score);
  return q4gpu_check_launch();
}

// Device address of g_lm_head_static_scratch, looked up once per device (with
// that device current) on the first no-alloc call there.  In host code the
// symbol itself is only a host-side stand-in; kernels get this address.
static int lm_head_static_scratch(q4::LmHeadStaticScratch** out) {
  static std::mutex mu;
  static q4::LmHeadStaticScratch* addr[Q4GPU_MAX_DEVICES] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= Q4GPU_MAX_DEVICES) return q4gpu_fail(Q4GPU_ERR_ARG, "device ordinal %d too large", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, q4::g_lm_head_static_scratch);
    if (e != cudaSuccess)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cudaGetSymbolAddress(lm-head scratch): %s", cudaGetErrorString(e));
    addr[dev] = static_cast<q4::LmHeadStaticScratch*>(p);
  }
  *out = addr[dev];
  return Q4GPU_OK;
}

int q4gpu_lm_head_argmax_noalloc(const int32_t* act, const uint8_t* packed, const uint16_t* scale, int32_t rows,
                                 int64_t* logits, int32_t* out_token, int64_t* out_score, void* stream) {
  if (!act || !packed || !scale || !out_token || !out_score) return q4gpu_fail(Q4GPU_ERR_ARG, "null argument");
  if (rows <= 0 || rows > Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS)
    return q4gpu_fail(Q4GPU_ERR_ARG, "rows %d outside 1..%d supported by the static LM-head scratch", rows,
                      Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS);
  if (((uintptr_t)packed) & 15) return q4gpu_fail(Q4GPU_ERR_ALIGN, "packed weights must be 16-byte aligned");
  q4::LmHeadStaticScratch* sc = nullptr;
  int rc = lm_head_static_scratch(&sc);
  if (rc) return rc;
  // the completion counter must start at zero (the kernel leaves it at zero,
  // but an earlier call may have been cut short)
  const cudaError_t e = cudaMemsetAsync(&sc->counter, 0, sizeof(unsigned int), as_stream(stream));
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "scratch clear: %s", cudaGetErrorString(e));
  lm_head_kernel<4><<<Q4GPU_LM_HEAD_BLOCKS, 256, 0, as_stream(stream)>>>(act, packed, scale, rows, logits,
                                                                          sc->partial, &sc->counter, out_token,
                                                                          out_score);
  return q4gpu_check_launch();
}

}  // extern "C"
