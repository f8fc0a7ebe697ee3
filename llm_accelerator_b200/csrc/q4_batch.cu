// Batched greedy decode: up to 64 independent sequences advance one position
// per step together, sharing every weight read.
//
// GEMMs run on the tensor cores with exact integer arithmetic.  Weights are
// expanded once to int8 (row-major [rows, K]).  Each sequence's activation a
// (signed 24-bit) is fed as the three unsigned byte limbs of a + 2^23, and
// eight B rows of ones yield sum(w) per row and 64-group.  Per group,
// mma.sync m16n8k32 (s8 x u8 -> s32) accumulates P0, P1, P2 and W1 exactly
// (|P| < 2^17), and
//     sum(w * a) = P0 + 256 P1 + 65536 P2 - 2^23 W1
// is formed in int64 and multiplied by the group's Q2.14 scale.  The B tile
// columns are ordered [limb][sequence], so the three limbs of one (row,
// sequence) land in the same thread's accumulator fragment.
//
// B ("limb") matrices are stored transposed, Bt[n][k] u8 with n = limb * SP + m
// (SP = padded sequence count) and n = 3 SP .. 3 SP + 7 the ones rows.
// Producers write them directly: a norm kernel for the norm-fed GEMMs, the
// attention epilogue for o_proj, the SwiGLU epilogue for down.  Both GEMM
// operands stream through a 4-stage cp.async pipeline per 64-column group.
#include <algorithm>

#include "q4_batch.h"
#include "q4_gemv.cuh"
#include "q4gpu_internal.h"

namespace q4 {

constexpr int kBStride = 80;  // bytes per row of a 64-byte k-chunk in shared memory (bank-conflict free)
constexpr int kNStage = 4;

struct BatchCtx {
  const SlotState* slots;  // [S]
  int S, SP;
  int32_t* qkv_raw;        // [S, 4096] raw Q12.12 q/k/v of the current layer
  uint8_t* bt1;            // [N, 1024]
  uint8_t* bt2;            // [N, 2048]
  uint8_t* bt3;            // [N, 3072]
  const int32_t* lm_from;  // [S]
};

__device__ __forceinline__ void mma_s8u8(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// limbs of the unsigned offset value a + 2^23
__device__ __forceinline__ void write_limbs(uint8_t* bt, int SP, int K, int m, int k, int32_t a) {
  const uint32_t u = (uint32_t)(a + (1 << 23));
  bt[(size_t)(0 * SP + m) * K + k] = (uint8_t)(u & 0xFF);
  bt[(size_t)(1 * SP + m) * K + k] = (uint8_t)((u >> 8) & 0xFF);
  bt[(size_t)(2 * SP + m) * K + k] = (uint8_t)((u >> 16) & 0xFF);
}

template <int J>
struct WarpAcc {
  int64_t v[2][2 * J];  // [row half][2j + c]
};

// Exact batched GEMV of one CTA: rows [row0, row0 + 16 RT) of A (int8
// [rows, K], scales [rows, K/64]) against all SP sequences of bt.  Warps:
// RT row tiles x SH sequence blocks of 8 J sequences (SH * 8 J == SP).
// acc.v[h][2j+c]: row row0 + 16 rt + lane/4 + 8h, sequence 8 J sb + 8j + 2(lane%4) + c.
template <int K, int J, int SH, int RT>
__device__ __forceinline__ void bgemm_cta(const int8_t* __restrict__ A, const uint16_t* __restrict__ Sc, int row0,
                                          const uint8_t* __restrict__ bt, uint8_t* smem, WarpAcc<J>& acc) {
  constexpr int G = K / 64;
  constexpr int SP = SH * 8 * J;
  constexpr int N = 3 * SP + 8;
  constexpr int ROWS = 16 * RT;
  constexpr int A_BYTES = ROWS * kBStride, B_BYTES = N * kBStride;
  constexpr int STAGE = A_BYTES + B_BYTES;
  constexpr int NT = 32 * RT * SH;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
  const int rt = warp % RT, sb = warp / RT;
  auto issue = [&](int g) {
    if (g < G) {
      uint8_t* st = smem + (g % kNStage) * STAGE;
      for (int i = threadIdx.x; i < (ROWS + N) * 4; i += NT) {
        const int r = i >> 2, part = i & 3;
        if (r < ROWS)
          cp_async16(st + r * kBStride + part * 16, A + (size_t)(row0 + r) * K + g * 64 + part * 16);
        else
          cp_async16(st + A_BYTES + (r - ROWS) * kBStride + part * 16,
                     bt + (size_t)(r - ROWS) * K + g * 64 + part * 16);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int q = 0; q < 2 * J; ++q) acc.v[h][q] = 0;
#pragma unroll
  for (int s = 0; s < kNStage - 1; ++s) issue(s);
  const int arow = (rt * 16 + gid) * kBStride + tig * 4;
  for (int g = 0; g < G; ++g) {
    cp_async_wait<kNStage - 2>();
    __syncthreads();
    issue(g + kNStage - 1);
    const uint8_t* st = smem + (g % kNStage) * STAGE;
    int32_t d[3 * J + 1][4];
#pragma unroll
    for (int t = 0; t < 3 * J + 1; ++t) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t a[4];
      a[0] = *reinterpret_cast<const uint32_t*>(st + arow + ks * 32);
      a[1] = *reinterpret_cast<const uint32_t*>(st + arow + 8 * kBStride + ks * 32);
      a[2] = *reinterpret_cast<const uint32_t*>(st + arow + ks * 32 + 16);
      a[3] = *reinterpret_cast<const uint32_t*>(st + arow + 8 * kBStride + ks * 32 + 16);
#pragma unroll
      for (int t = 0; t < 3 * J + 1; ++t) {
        const int n0 = t < 3 * J ? (t / J) * SP + sb * 8 * J + 8 * (t % J) : 3 * SP;
        const uint8_t* bp = st + A_BYTES + (n0 + gid) * kBStride + ks * 32 + tig * 4;
        mma_s8u8(d[t], a, *reinterpret_cast<const uint32_t*>(bp), *reinterpret_cast<const uint32_t*>(bp + 16));
      }
    }
    const int r0 = row0 + rt * 16 + gid;
    const int64_t s0 = __ldg(Sc + (size_t)r0 * G + g), s1 = __ldg(Sc + (size_t)(r0 + 8) * G + g);
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 2 * h + c;
          const int64_t gsum = ((int64_t)d[2 * J + j][r] << 16) + ((int64_t)d[J + j][r] << 8) + (int64_t)d[j][r] -
                               ((int64_t)d[3 * J][r] << 23);
          acc.v[h][2 * j + c] += gsum * (h ? s1 : s0);
        }
  }
  cp_async_wait<0>();
}

template <int J, int SH, int RT>
__host__ __device__ constexpr size_t bgemm_smem() {
  return (size_t)kNStage * (16 * RT + 3 * SH * 8 * J + 8) * kBStride;
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
__global__ void expand_int4_kernel(const uint8_t* __restrict__ packed, int64_t n_bytes, int8_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_bytes; i += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t b = packed[i];
    const int lo = b & 0xF, hi = b >> 4;
    out[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
    out[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
  }
}

// gate [3072, 1024] and up [3072, 1024] (packed, with scales) -> int8 [6144,
// 1024] in 32-row blocks: out rows 64 b .. 64 b + 31 = gate rows 32 b .., out
// rows 64 b + 32 .. 64 b + 63 = up rows 32 b ..
__global__ void expand_gu_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up,
                                 const uint16_t* __restrict__ sg, const uint16_t* __restrict__ su,
                                 int8_t* __restrict__ out, uint16_t* __restrict__ sout) {
  constexpr int64_t kBytes = (int64_t)2 * kInter * (kHidden / 2);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < kBytes; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / (kHidden / 2)), col = (int)(i % (kHidden / 2));
    const int src = 32 * (r / 64) + (r & 31);
    const uint8_t b = ((r & 32) ? up : gate)[(size_t)src * (kHidden / 2) + col];
    const int lo = b & 0xF, hi = b >> 4;
    out[2 * i] = (int8_t)(lo >= 8 ? lo - 16 : lo);
    out[2 * i + 1] = (int8_t)(hi >= 8 ? hi - 16 : hi);
    if (col < kHidden / kGroup) sout[(size_t)r * (kHidden / kGroup) + col] = ((r & 32) ? su : sg)[(size_t)src * 16 + col];
  }
}

// Per-sequence step inputs [S][2] = (token, position): store the token at its
// position, set the position, and make the argmax land for every position.
__global__ void batch_load_kernel(const SlotState* __restrict__ slots, int S, const int32_t* __restrict__ in,
                                  int32_t* __restrict__ lm_from) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S) return;
  const int pos = in[2 * m + 1];
  slots[m].tokens[pos] = in[2 * m];
  *slots[m].pos = pos;
  lm_from[m] = 0;
}

// out[m] = (token, pad, score lo, score hi) written at position in[2 m + 1] + 1
__global__ void batch_gather_kernel(const SlotState* __restrict__ slots, int S, const int32_t* __restrict__ in,
                                    int32_t* __restrict__ out) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S) return;
  const int p = in[2 * m + 1] + 1;
  out[4 * m] = slots[m].tokens[p];
  out[4 * m + 1] = 0;
  *reinterpret_cast<int64_t*>(out + 4 * m + 2) = slots[m].scores[p];
}

// Same position for every sequence, and the argmax threshold lm_from.
__global__ void batch_set_pos_kernel(const SlotState* __restrict__ slots, int S, int pos, int32_t* __restrict__ lm_from,
                                     int lm_value) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= S) return;
  *slots[m].pos = pos;
  if (lm_value >= 0) lm_from[m] = lm_value;
}

__global__ void batch_embed_kernel(BatchCtx c, const uint8_t* __restrict__ W, const uint16_t* __restrict__ S) {
  grid_dep_wait();
  grid_dep_launch();
  const SlotState& st = c.slots[blockIdx.x];
  const int pos = *st.pos;
  if (pos >= st.max_ctx) return;
  const int t = st.tokens[pos];
  const uint8_t* row = W + (size_t)t * (kHidden / 2);
  const uint16_t* sc = S + (size_t)t * (kHidden / kGroup);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    const uint8_t b = row[i >> 1];
    const int q = (int)((i & 1) ? (b >> 4) : (b & 0xF));
    st.hidden[i] = ((q >= 8 ? q - 16 : q) * (int32_t)sc[i / kGroup]) >> 4;
  }
}

// RMSNorm of one sequence's hidden (which 0) or post (which 1) vector -> limbs in bt1
__global__ void batch_norm_limbs_kernel(BatchCtx c, int which, const int32_t* __restrict__ gamma) {
  __shared__ int64_t red[32];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const SlotState& st = c.slots[m];
  const int32_t* x = which == 0 ? st.hidden : st.post;
  int64_t ss = 0;
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) ss += (int64_t)x[i] * x[i];
  ss = block_sum_i64(ss, red);
  const int64_t inv = inv_rms_from_ss(ss, kHiddenNorm);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x)
    write_limbs(c.bt1, c.SP, kHidden, m, i, norm_apply(x[i], inv, gamma[i], kHiddenNorm));
}

template <int J>
__device__ __forceinline__ int acc_seq(int sb, int q, int lane) {
  return sb * 8 * J + 8 * (q >> 1) + 2 * (lane & 3) + (q & 1);
}

// QKV projection: raw Q12.12 rows into qkv_raw (64 rows per CTA).
template <int J, int SH>
__global__ void __launch_bounds__(128 * SH) batch_qkv_kernel(BatchCtx c, const int8_t* __restrict__ W,
                                                             const uint16_t* __restrict__ Sc) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RT = 4;
  grid_dep_wait();
  grid_dep_launch();
  const int row0 = blockIdx.x * 16 * RT;
  WarpAcc<J> acc;
  bgemm_cta<kHidden, J, SH, RT>(W, Sc, row0, c.bt1, smem, acc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp % RT, sb = warp / RT;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int q = 0; q < 2 * J; ++q) {
      const int m = acc_seq<J>(sb, q, lane);
      if (m < c.S) c.qkv_raw[(size_t)m * 4096 + row0 + rt * 16 + (lane >> 2) + 8 * h] = sat24(acc.v[h][q] >> 14);
    }
}

// Attention for one (KV head, sequence): q/k head RMSNorm + RoPE, KV append,
// exact two-pass LUT softmax for the two query heads of the group; writes the
// output and its limbs (the o_proj B matrix).  256 threads.
__global__ void __launch_bounds__(256) batch_attn_kernel(BatchCtx c, int layer, const int32_t* __restrict__ g_q,
                                                         const int32_t* __restrict__ g_k,
                                                         const int32_t* __restrict__ cos_tab,
                                                         const int32_t* __restrict__ sin_tab,
                                                         const int32_t* __restrict__ exp_lut) {
  extern __shared__ int64_t sc[];  // [2][ctx] scaled scores, then LUT indices
  __shared__ __align__(16) int32_t hv[2][kHeadDim];  // roped q of the two heads
  __shared__ uint64_t probtab[2][kExpLut];
  __shared__ int64_t red[32];
  __shared__ int64_t part[8][2][kHeadDim];
  const int kv = blockIdx.x, m = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  grid_dep_wait();
  grid_dep_launch();
  const SlotState& st = c.slots[m];
  const int pos = *st.pos;
  if (pos >= st.max_ctx) return;
  const int ctx = pos + 1;
  const int32_t* raw = c.qkv_raw + (size_t)m * 4096;
  // warp 0: q head 2kv, warp 1: q head 2kv+1, warp 2: k (normed, roped);
  // warp 3: v.  A lane owns dims 4 lane .. 4 lane + 3; the RoPE partner
  // d +- 64 sits 16 lanes away.
  if (warp < 3) {
    const int row = warp < 2 ? (2 * kv + warp) * kHeadDim : kQRows + kv * kHeadDim;
    const int4 x = *reinterpret_cast<const int4*>(raw + row + 4 * lane);
    const int32_t xs[4] = {x.x, x.y, x.z, x.w};
    int64_t ss = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += (int64_t)xs[e] * xs[e];
    ss = warp_sum_i64(ss);
    const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
    const int32_t* g = warp < 2 ? g_q : g_k;
    int32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 4 * lane + e;
      const int32_t n = norm_apply(xs[e], inv, g[d], kHeadNorm);
      const int32_t partner = __shfl_xor_sync(0xFFFFFFFFu, n, 16);
      const int64_t rot = lane < 16 ? -(int64_t)partner : (int64_t)partner;
      o[e] = sat24(((int64_t)n * cos_tab[pos * kHeadDim + d] + rot * sin_tab[pos * kHeadDim + d]) >> 15);
    }
    const int4 o4 = make_int4(o[0], o[1], o[2], o[3]);
    if (warp < 2)
      *reinterpret_cast<int4*>(&hv[warp][4 * lane]) = o4;
    else
      reinterpret_cast<int4*>(st.kv.at(layer, 0, kv, pos))[lane] = o4;
  } else if (warp == 3) {
    reinterpret_cast<int4*>(st.kv.at(layer, 1, kv, pos))[lane] =
        *reinterpret_cast<const int4*>(raw + kQRows + kKvRows + kv * kHeadDim + 4 * lane);
  }
  // block barrier: makes this position's K/V (global) and q (shared) visible
  __syncthreads();
  // scores: 8 lanes per position, 4 positions per warp, 32 per pass; lane
  // `sub` holds dims 4 (sub + 8 j) .. +3, j = 0..3 (128-byte coalesced rows)
  {
    const int sub = lane & 7, quad = lane >> 3;
    int32_t q0[16], q1[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int4 a = *reinterpret_cast<const int4*>(&hv[0][4 * (sub + 8 * j)]);
      const int4 b = *reinterpret_cast<const int4*>(&hv[1][4 * (sub + 8 * j)]);
      q0[4 * j] = a.x; q0[4 * j + 1] = a.y; q0[4 * j + 2] = a.z; q0[4 * j + 3] = a.w;
      q1[4 * j] = b.x; q1[4 * j + 1] = b.y; q1[4 * j + 2] = b.z; q1[4 * j + 3] = b.w;
    }
    // the trip count is uniform across the warp (the shuffles need all lanes)
    for (int base = warp * 4; base < ctx; base += 64) {
      int4 k4[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int p = base + quad + 32 * u;
        if (p < ctx) {
          const int4* kr = reinterpret_cast<const int4*>(st.kv.at(layer, 0, kv, p));
#pragma unroll
          for (int j = 0; j < 4; ++j) k4[u][j] = kr[sub + 8 * j];
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) k4[u][j] = make_int4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int p = base + quad + 32 * u;
        int64_t s0 = 0, s1 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t kk[4] = {k4[u][j].x, k4[u][j].y, k4[u][j].z, k4[u][j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            s0 += (int64_t)q0[4 * j + e] * kk[e];
            s1 += (int64_t)q1[4 * j + e] * kk[e];
          }
        }
#pragma unroll
        for (int msk = 1; msk < 8; msk <<= 1) {
          s0 += shfl_xor_i64(s0, msk);
          s1 += shfl_xor_i64(s1, msk);
        }
        if (sub == 0 && p < ctx) {
          sc[p] = scale_score(s0, kScoreScale);
          sc[ctx + p] = scale_score(s1, kScoreScale);
        }
      }
    }
  }
  __syncthreads();
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    int64_t* s = sc + h * ctx;
    int64_t mx = INT64_MIN;
    for (int p = t; p < ctx; p += blockDim.x) mx = s[p] > mx ? s[p] : mx;
    mx = block_max_i64(mx, red);
    int64_t sum = 0;
    for (int p = t; p < ctx; p += blockDim.x) {
      const int ix = lut_index(mx, s[p]);
      s[p] = ix;
      sum += exp_lut[ix];
    }
    sum = block_sum_i64(sum, red);
    for (int i = t; i < kExpLut; i += blockDim.x) probtab[h][i] = ((uint64_t)exp_lut[i] << 16) / (uint64_t)sum;
  }
  __syncthreads();
  // values: thread (pg = warp, lane) accumulates dims 4 lane .. +3 of
  // positions p = pg (mod 8), two heads
  {
    int64_t a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
    for (int p0 = warp; p0 < ctx; p0 += 32) {
      int4 v4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + 8 * u;
        if (p < ctx) v4[u] = reinterpret_cast<const int4*>(st.kv.at(layer, 1, kv, p))[lane];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + 8 * u;
        if (p < ctx) {
          const int64_t pr0 = (int64_t)probtab[0][sc[p]], pr1 = (int64_t)probtab[1][sc[ctx + p]];
          const int32_t vv[4] = {v4[u].x, v4[u].y, v4[u].z, v4[u].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            a0[e] += pr0 * vv[e];
            a1[e] += pr1 * vv[e];
          }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      part[warp][0][4 * lane + e] = a0[e];
      part[warp][1][4 * lane + e] = a1[e];
    }
  }
  __syncthreads();
  {
    const int h = t >> 7, d = t & (kHeadDim - 1);
    int64_t acc = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc += part[w][h][d];
    const int32_t o = sat24(acc >> 16);
    const int k = (2 * kv + h) * kHeadDim + d;
    st.attn[k] = o;
    write_limbs(c.bt2, c.SP, 2 * kHidden, m, k, o);
  }
}

// o_proj (mode 0: post = sat24(hidden + (o >> 2))) or down (mode 1: hidden =
// sat24(post + (d >> 2))); 64 rows per CTA x all sequences.
template <int K, int J, int SH>
__global__ void __launch_bounds__(128 * SH) batch_resid_kernel(BatchCtx c, const int8_t* __restrict__ W,
                                                               const uint16_t* __restrict__ Sc, int mode) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RT = 4;
  grid_dep_wait();
  grid_dep_launch();
  const int row0 = blockIdx.x * 16 * RT;
  WarpAcc<J> acc;
  bgemm_cta<K, J, SH, RT>(W, Sc, row0, mode == 0 ? c.bt2 : c.bt3, smem, acc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp % RT, sb = warp / RT;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int q = 0; q < 2 * J; ++q) {
      const int m = acc_seq<J>(sb, q, lane);
      if (m >= c.S) continue;
      const SlotState& st = c.slots[m];
      if (*st.pos >= st.max_ctx) continue;
      const int r = row0 + rt * 16 + (lane >> 2) + 8 * h;
      const int32_t o = sat24(acc.v[h][q] >> 14);
      if (mode == 0)
        st.post[r] = sat24((int64_t)st.hidden[r] + (o >> 2));
      else
        st.hidden[r] = sat24((int64_t)st.post[r] + (o >> 2));
    }
}

// gate/up + SwiGLU: CTA = 32 gate rows and the same 32 up rows (row tiles
// 0-1 gate, 2-3 up) x all sequences; writes mlp and its limbs (down's B).
template <int J, int SH>
__global__ void __launch_bounds__(128 * SH) batch_gateup_kernel(BatchCtx c, const int8_t* __restrict__ Wgu,
                                                                const uint16_t* __restrict__ Sgu,
                                                                const int32_t* __restrict__ sig_lut) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RT = 4;
  constexpr int SP = SH * 8 * J;
  int32_t* gsm = reinterpret_cast<int32_t*>(smem + bgemm_smem<J, SH, RT>());  // [32][SP]
  grid_dep_wait();
  grid_dep_launch();
  // Wgu interleaves 32-row blocks: block b = gate rows [32b, 32b+32), then up rows
  const int row0 = blockIdx.x * 64;
  WarpAcc<J> acc;
  bgemm_cta<kHidden, J, SH, RT>(Wgu, Sgu, row0, c.bt1, smem, acc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp % RT, sb = warp / RT;
  const bool up = rt >= 2;
  if (!up) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 2 * J; ++q) {
        const int r = rt * 16 + (lane >> 2) + 8 * h;
        gsm[r * SP + acc_seq<J>(sb, q, lane)] = sat24(acc.v[h][q] >> 14);
      }
  }
  __syncthreads();
  if (up) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int q = 0; q < 2 * J; ++q) {
        const int m = acc_seq<J>(sb, q, lane);
        if (m >= c.S) continue;
        const SlotState& st = c.slots[m];
        if (*st.pos >= st.max_ctx) continue;
        const int r = (rt - 2) * 16 + (lane >> 2) + 8 * h;
        const int32_t g = gsm[r * SP + m], u = sat24(acc.v[h][q] >> 14);
        const int32_t gc = g < -32768 ? -32768 : (g > 32768 ? 32768 : g);
        int ix = (gc + 32768 + 32) >> 6;
        ix = ix > kSigLut - 1 ? kSigLut - 1 : ix;
        const int32_t silu = sat24(((int64_t)g * sig_lut[ix]) >> 16);
        const int32_t hv = sat24(((int64_t)silu * u) >> 12);
        const int i = blockIdx.x * 32 + r;
        st.mlp[i] = hv;
        write_limbs(c.bt3, SP, kInter, m, i, hv);
      }
  }
}

// LM head: 256 rows per CTA x all sequences -> per-CTA best (score, row) per sequence.
template <int J, int SH>
__global__ void __launch_bounds__(128 * SH) batch_lmhead_kernel(BatchCtx c, const int8_t* __restrict__ W,
                                                                const uint16_t* __restrict__ Sc, int rows,
                                                                ArgBestD* __restrict__ partial) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RT = 4;
  constexpr int SP = SH * 8 * J;
  ArgBestD* best = reinterpret_cast<ArgBestD*>(smem + bgemm_smem<J, SH, RT>());  // [RT][SP]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rt = warp % RT, sb = warp / RT;
  grid_dep_wait();
  grid_dep_launch();
  int64_t bs[2 * J];
  int32_t bi[2 * J];
#pragma unroll
  for (int q = 0; q < 2 * J; ++q) {
    bs[q] = INT64_MIN;
    bi[q] = INT32_MAX;
  }
  for (int sub = 0; sub < 4; ++sub) {  // 4 x 64 rows
    const int row0 = blockIdx.x * 256 + sub * 64;
    if (row0 >= rows) break;  // uniform per CTA
    // the last, partial tile reads a clamped (valid) window and drops the extra rows
    const int row_eff = row0 + 64 <= rows ? row0 : rows - 64;
    WarpAcc<J> acc;
    bgemm_cta<kHidden, J, SH, RT>(W, Sc, row_eff, c.bt1, smem, acc);
#pragma unroll
    for (int q = 0; q < 2 * J; ++q)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = row_eff + rt * 16 + (lane >> 2) + 8 * h;
        if (r >= row0 && (acc.v[h][q] > bs[q] || (acc.v[h][q] == bs[q] && r < bi[q]))) {
          bs[q] = acc.v[h][q];
          bi[q] = r;
        }
      }
    __syncthreads();
  }
#pragma unroll
  for (int q = 0; q < 2 * J; ++q) {
#pragma unroll
    for (int msk = 4; msk < 32; msk <<= 1) {  // across lanes with the same lane & 3
      const int64_t os = shfl_xor_i64(bs[q], msk);
      const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi[q], msk);
      if (os > bs[q] || (os == bs[q] && oi < bi[q])) {
        bs[q] = os;
        bi[q] = oi;
      }
    }
    if (lane < 4) best[rt * SP + acc_seq<J>(sb, q, lane)] = ArgBestD{bs[q], bi[q], 0};
  }
  __syncthreads();
  for (int m = threadIdx.x; m < c.S; m += blockDim.x) {
    ArgBestD b = best[m];
    for (int r = 1; r < RT; ++r) {
      const ArgBestD o = best[r * SP + m];
      if (o.score > b.score || (o.score == b.score && o.idx < b.idx)) b = o;
    }
    partial[(size_t)blockIdx.x * kBatchSeqMax + m] = b;
  }
}

// Reduce the LM-head partials of sequence blockIdx.x; write the argmax where
// the sequence has left its prompt, and advance its position.
__global__ void batch_argmax_kernel(BatchCtx c, const ArgBestD* __restrict__ partial, int n_parts) {
  __shared__ int64_t ss[32];
  __shared__ int32_t si[32];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const SlotState& st = c.slots[m];
  int64_t bs = INT64_MIN;
  int32_t bi = INT32_MAX;
  for (int i = threadIdx.x; i < n_parts; i += blockDim.x) {
    const ArgBestD o = partial[(size_t)i * kBatchSeqMax + m];
    if (o.score > bs || (o.score == bs && o.idx < bi)) {
      bs = o.score;
      bi = o.idx;
    }
  }
#pragma unroll
  for (int msk = 16; msk > 0; msk >>= 1) {
    const int64_t os = shfl_xor_i64(bs, msk);
    const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, msk);
    if (os > bs || (os == bs && oi < bi)) {
      bs = os;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    ss[warp] = bs;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (ss[w] > bs || (ss[w] == bs && si[w] < bi)) {
        bs = ss[w];
        bi = si[w];
      }
    const int pos = *st.pos;
    if (pos < st.max_ctx) {
      if (pos + 1 >= c.lm_from[m]) {
        st.tokens[pos + 1] = bi;
        st.scores[pos + 1] = bs;
      }
      *st.pos = pos + 1;
    }
  }
}

}  // namespace q4

// ===========================================================================
// Host side
// ===========================================================================
using namespace q4;

namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

#define BQ(call)                                                                                        \
  do {                                                                                                  \
    const cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

template <int J, int SH>
int enqueue_t(const BatchPlan& p, cudaStream_t s) {
  const BatchCtx c{p.slots, p.S, p.SP, p.qkv_raw, p.bt1, p.bt2, p.bt3, p.lm_from};
  constexpr size_t sm = bgemm_smem<J, SH, 4>();
  constexpr int SP = SH * 8 * J;
  const dim3 blk(128 * SH);
  BQ(launch_pdl(batch_embed_kernel, dim3(p.S), dim3(256), 0, s, c, p.emb, p.semb));
  for (int l = 0; l < p.n_layers; ++l) {
    const BatchLayerW& w = p.layers[l];
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 0, w.g_in));
    BQ(launch_pdl(batch_qkv_kernel<J, SH>, dim3(4096 / 64), blk, sm, s, c, w.wqkv, w.sqkv));
    BQ(launch_pdl(batch_attn_kernel, dim3(kKvHeads, p.S), dim3(256), (size_t)2 * p.max_ctx * 8, s, c, l, w.g_q, w.g_k,
                  p.cos_tab, p.sin_tab, p.exp_lut));
    BQ(launch_pdl(batch_resid_kernel<2 * kHidden, J, SH>, dim3(kHidden / 64), blk, sm, s, c, w.wo, w.so, 0));
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 1, w.g_post));
    BQ(launch_pdl(batch_gateup_kernel<J, SH>, dim3(kInter / 32), blk, sm + (size_t)32 * SP * 4, s, c, w.wgu, w.sgu,
                  p.sig_lut));
    BQ(launch_pdl(batch_resid_kernel<kInter, J, SH>, dim3(kHidden / 64), blk, sm, s, c, w.wdown, w.sdown, 1));
  }
  BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 0, p.g_final));
  const int lm_ctas = (p.vocab + 255) / 256;
  BQ(launch_pdl(batch_lmhead_kernel<J, SH>, dim3(lm_ctas), blk, sm + (size_t)4 * SP * sizeof(ArgBestD), s, c, p.emb8,
                p.semb, p.vocab, p.lm_partial));
  BQ(launch_pdl(batch_argmax_kernel, dim3(p.S), dim3(256), 0, s, c, (const ArgBestD*)p.lm_partial, lm_ctas));
  return Q4GPU_OK;
}

template <int J, int SH>
int setup_t(const BatchPlan& p) {
  constexpr size_t sm = bgemm_smem<J, SH, 4>();
  constexpr int SP = SH * 8 * J;
  BQ(cudaFuncSetAttribute(batch_qkv_kernel<J, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  BQ(cudaFuncSetAttribute(batch_resid_kernel<2 * kHidden, J, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)sm));
  BQ(cudaFuncSetAttribute(batch_resid_kernel<kInter, J, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  BQ(cudaFuncSetAttribute(batch_gateup_kernel<J, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)(sm + (size_t)32 * SP * 4)));
  BQ(cudaFuncSetAttribute(batch_lmhead_kernel<J, SH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)(sm + (size_t)4 * SP * sizeof(ArgBestD))));
  BQ(cudaFuncSetAttribute(batch_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)((size_t)2 * p.max_ctx * 8)));
  return Q4GPU_OK;
}

}  // namespace

int q4gpu_batch_padded(int S) { return S <= 8 ? 8 : S <= 16 ? 16 : S <= 24 ? 24 : S <= 32 ? 32 : 64; }

// SP <= 32: one warp block of J = SP / 8 sequence groups; SP == 64: two blocks of 4.
int q4gpu_batch_setup(const BatchPlan& p) {
  switch (p.SP) {
    case 8: return setup_t<1, 1>(p);
    case 16: return setup_t<2, 1>(p);
    case 24: return setup_t<3, 1>(p);
    case 32: return setup_t<4, 1>(p);
    case 64: return setup_t<4, 2>(p);
    default: return q4gpu_fail(Q4GPU_ERR_SHAPE, "padded batch %d", p.SP);
  }
}

int q4gpu_enqueue_batch_step(const BatchPlan& p, cudaStream_t s) {
  switch (p.SP) {
    case 8: return enqueue_t<1, 1>(p, s);
    case 16: return enqueue_t<2, 1>(p, s);
    case 24: return enqueue_t<3, 1>(p, s);
    case 32: return enqueue_t<4, 1>(p, s);
    case 64: return enqueue_t<4, 2>(p, s);
    default: return q4gpu_fail(Q4GPU_ERR_SHAPE, "padded batch %d", p.SP);
  }
}

int q4gpu_expand_int4(const uint8_t* packed, int64_t n_bytes, int8_t* out, cudaStream_t s) {
  const int blocks = (int)std::min<int64_t>((n_bytes + 255) / 256, 148 * 32);
  expand_int4_kernel<<<blocks, 256, 0, s>>>(packed, n_bytes, out);
  return q4gpu_check_launch();
}

int q4gpu_expand_gu(const uint8_t* gate, const uint8_t* up, const uint16_t* sg, const uint16_t* su, int8_t* out,
                    uint16_t* sout, cudaStream_t s) {
  expand_gu_kernel<<<148 * 8, 256, 0, s>>>(gate, up, sg, su, out, sout);
  return q4gpu_check_launch();
}

int q4gpu_batch_load(const SlotState* slots, int S, const int32_t* in, int32_t* lm_from, cudaStream_t s) {
  batch_load_kernel<<<1, 64, 0, s>>>(slots, S, in, lm_from);
  return q4gpu_check_launch();
}

int q4gpu_batch_gather(const SlotState* slots, int S, const int32_t* in, int32_t* out, cudaStream_t s) {
  batch_gather_kernel<<<1, 64, 0, s>>>(slots, S, in, out);
  return q4gpu_check_launch();
}

int q4gpu_batch_set_positions(const SlotState* slots, int S, int pos, int32_t* lm_from, int lm_value,
                              cudaStream_t s) {
  batch_set_pos_kernel<<<(S + 63) / 64, 64, 0, s>>>(slots, S, pos, lm_from, lm_value);
  return q4gpu_check_launch();
}
