// Batched greedy decode: up to 64 independent sequences advance one position
// per step together, sharing every weight read.
//
// GEMMs run on the tensor cores (tcgen05.mma, kind::i8) with exact integer
// arithmetic, reading the Q4 weights as the model stores them: the group
// scales are split into 4-bit digits and each digit's weight plane (w * s_j,
// a signed byte) is built in shared memory next to the MMA (see the GEMM
// section below).  Each sequence's activation a (signed 24-bit) is fed as the
// three unsigned byte limbs of a + 2^23.
//
// B ("limb") matrices are stored as Bt[n][k] u8 with n = limb * SP + m
// (SP = padded sequence count) and n = 3 SP .. 3 SP + 7 zero rows (the MMA's
// N is 3 SP rounded up to 16).  Producers write them directly: a norm kernel
// for the norm-fed GEMMs, the attention epilogue for o_proj, the SwiGLU
// epilogue for down.
#include <cudaTypedefs.h>

#include <algorithm>

#include "q4_batch.h"
#include "q4_gemv.cuh"
#include "q4_umma.cuh"
#include "q4gpu_internal.h"

namespace q4 {

struct BatchCtx {
  const SlotState* slots;  // [S]
  int S, SP;
  int32_t* qkv_raw;        // [S, 4096] raw Q12.12 q/k/v of the current layer
  uint8_t* bt1;            // [N, 1024]
  uint8_t* bt2;            // [N, 2048]
  uint8_t* bt3;            // [N, 3072]
  const int32_t* lm_from;  // [S]
  int* err;                // set when a pipeline wait runs out
  // the range's slots are consecutive in the model's state arrays
  const int32_t* pos0;     // position of sequence m at pos0[4 m]
  int32_t* hidden0;        // [S, 1024]
  int32_t* post0;          // [S, 1024]
  int max_ctx;
  // optional timeline (nullptr = off): attention CTA (m, kv) of layer l writes
  // %globaltimer stamps at its phase boundaries to trace[((l * S + m) * 8 + kv) * 8 + k]
  unsigned long long* trace;
  // Columns beyond SP (prefill): column m belongs to sub-batch m / SP, whose
  // limb matrices start bt_sub1 / bt_sub3 bytes after the previous one's in
  // bt1 / bt3 (0 when S <= SP).
  size_t bt_sub1;
  size_t bt_sub3;
};

__device__ __forceinline__ void attn_stamp(const BatchCtx& c, int layer, int m, int kv, int k) {
  if (c.trace && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    c.trace[(((size_t)layer * c.S + m) * kKvHeads + kv) * 8 + k] = t;
  }
}

// limbs of the unsigned offset value a + 2^23
__device__ __forceinline__ void write_limbs(uint8_t* bt, int SP, int K, int m, int k, int32_t a) {
  const uint32_t u = (uint32_t)(a + (1 << 23));
  bt[(size_t)(0 * SP + m) * K + k] = (uint8_t)(u & 0xFF);
  bt[(size_t)(1 * SP + m) * K + k] = (uint8_t)((u >> 8) & 0xFF);
  bt[(size_t)(2 * SP + m) * K + k] = (uint8_t)((u >> 16) & 0xFF);
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
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
  // released only after the wait: kernels later in the step read the
  // positions (advanced by the previous step's argmax) before their own waits
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x;
  const int pos = c.pos0[4 * m];
  if (pos >= c.max_ctx) return;
  const int t = c.slots[m].tokens[pos];
  const uint8_t* row = W + (size_t)t * (kHidden / 2);
  const uint16_t* sc = S + (size_t)t * (kHidden / kGroup);
  int32_t* h = c.hidden0 + (size_t)m * kHidden;
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    const uint8_t b = row[i >> 1];
    const int q = (int)((i & 1) ? (b >> 4) : (b & 0xF));
    h[i] = ((q >= 8 ? q - 16 : q) * (int32_t)sc[i / kGroup]) >> 4;
  }
}

// RMSNorm of one sequence's hidden (which 0) or post (which 1) vector -> limbs
// in bt1.  256 threads x 4 consecutive elements.
__global__ void __launch_bounds__(256) batch_norm_limbs_kernel(BatchCtx c, int which,
                                                               const int32_t* __restrict__ gamma,
                                                               int32_t* __restrict__ out_act) {
  __shared__ int64_t red[32];
  const int m = blockIdx.x, k = 4 * threadIdx.x;
  // the norm weights do not depend on earlier kernels: load them before the wait
  const int4 gm = *reinterpret_cast<const int4*>(gamma + k);
  // the next GEMM may start its weight-only set-up now (it waits for this
  // kernel before reading its output).  Safe here, inside a step: the first
  // norm of a step starts only after the embedding's wait, so nothing that
  // reads the positions before its own wait can start before the previous
  // step's argmax has completed.
  grid_dep_launch();
  grid_dep_wait();
  const int sub = m / c.SP, ms = m - sub * c.SP;
  uint8_t* bt = c.bt1 + (size_t)sub * c.bt_sub1;
  const int4 x = *reinterpret_cast<const int4*>((which == 0 ? c.hidden0 : c.post0) + (size_t)m * kHidden + k);
  int64_t ss = (int64_t)x.x * x.x + (int64_t)x.y * x.y + (int64_t)x.z * x.z + (int64_t)x.w * x.w;
  ss = block_sum_i64(ss, red);
  const int64_t inv = inv_rms_from_ss(ss, kHiddenNorm);
  const int4 nv = make_int4(norm_apply(x.x, inv, gm.x, kHiddenNorm), norm_apply(x.y, inv, gm.y, kHiddenNorm),
                            norm_apply(x.z, inv, gm.z, kHiddenNorm), norm_apply(x.w, inv, gm.w, kHiddenNorm));
  if (out_act) *reinterpret_cast<int4*>(out_act + (size_t)m * kHidden + k) = nv;
  const uint32_t u0 = (uint32_t)(nv.x + (1 << 23));
  const uint32_t u1 = (uint32_t)(nv.y + (1 << 23));
  const uint32_t u2 = (uint32_t)(nv.z + (1 << 23));
  const uint32_t u3 = (uint32_t)(nv.w + (1 << 23));
#pragma unroll
  for (int limb = 0; limb < 3; ++limb) {
    const int sh = 8 * limb;
    const uint32_t word = ((u0 >> sh) & 0xFF) | (((u1 >> sh) & 0xFF) << 8) | (((u2 >> sh) & 0xFF) << 16) |
                          (((u3 >> sh) & 0xFF) << 24);
    *reinterpret_cast<uint32_t*>(bt + (size_t)(limb * c.SP + ms) * kHidden + k) = word;
  }
}

// ---------------------------------------------------------------------------
// Split-KV attention: one CTA per (sequence m, KV head h, page c of 64
// positions), so the work spreads evenly over the GPU whatever the batch and
// context.  The exact two-pass LUT softmax is resolved across the pages of a
// (m, h) pair by the CTA that finishes last:
//   scores kernel: q head norm + RoPE (both query heads of the group), the new
//     position's k (norm + RoPE) and v appended to the cache, scaled scores
//     of the page to S, page maxima folded into M by atomicMax; the last page
//     turns S into probabilities P (LUT index, sum, one division per LUT entry)
//     and re-arms M.
//   values kernel: sum over the page of P * V into O by 64-bit atomic adds;
//     the last page writes sat24(O >> 16) as limbs of the o_proj input and
//     re-arms O.
// Integer sums are order independent, so the result equals the serial one.
// ---------------------------------------------------------------------------
constexpr int kPage = kKvPage;  // 64 positions per unit

struct AttnScratch {
  int64_t* S;         // [64 seqs][16 heads][max_ctx] scaled scores
  uint32_t* P;        // [64][16][max_ctx] probabilities (UQ0.16, <= 65536)
  int64_t* M;         // [64][16] running maxima, INT64_MIN when armed
  int64_t* O;         // [64][16][128] value sums, 0 when armed
  unsigned* cnt_s;    // [64][8] pages done, scores kernel
  unsigned* cnt_v;    // [64][8] pages done, values kernel
  int max_ctx;
};

// Bulk copy global -> shared of K/V rows.  The cache streams through L2 once
// per step (GBs against a 126 MB L2), so its lines are marked evict-first:
// the weights the GEMMs prefetch into L2 stay there.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          umma::smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(umma::smem_addr(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(umma::smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(umma::smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ int64_t ld_cg64(const int64_t* p) {
  return (int64_t)__ldcg(reinterpret_cast<const long long*>(p));
}

__global__ void __launch_bounds__(256) batch_attn_scores_kernel(BatchCtx c, AttnScratch a, int layer,
                                                                const int32_t* __restrict__ g_q,
                                                                const int32_t* __restrict__ g_k,
                                                                const int32_t* __restrict__ cos_tab,
                                                                const int32_t* __restrict__ sin_tab,
                                                                const int32_t* __restrict__ exp_lut) {
  __shared__ __align__(128) int32_t kpage[kPage * kHeadDim];  // 32 KB
  __shared__ __align__(16) int32_t hv[3][kHeadDim];           // roped q0, q1, k of the new position
  __shared__ int64_t red[32];
  __shared__ int64_t wmax[8][2];
  __shared__ uint32_t probtab[2][kExpLut];
  __shared__ uint64_t bar;
  __shared__ bool last;
  const int pg = blockIdx.x, h = blockIdx.y, m = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  grid_dep_wait();
  grid_dep_launch();
  const int pos = c.pos0[4 * m];
  if (pos >= c.max_ctx || pg * kPage > pos) return;
  const int ctx = pos + 1, nch = (ctx + kPage - 1) / kPage;
  const KvView kvv = c.slots[m].kv;
  const int p0 = pg * kPage;
  const int nold = min(kPage, pos - p0);  // rows of this page written by earlier steps
  if (t == 0) {
    umma::bar_init(&bar, 1);
    umma::bar_init_fence();
    umma::bar_expect_tx(&bar, nold > 0 ? (uint32_t)nold * kHeadDim * 4 : 0u);
    if (nold > 0) bulk_load(kpage, kvv.at(layer, 0, h, p0), (uint32_t)nold * kHeadDim * 4, &bar);
  }
  const int32_t* raw = c.qkv_raw + (size_t)m * (kQRows + 2 * kKvRows);
  const bool has_new = pos < p0 + kPage;
  // warps 0/1: q heads 2h, 2h+1; warp 2: k of the new position; warp 3: its v
  if (warp < 3 && (warp < 2 || has_new)) {
    const int row = warp < 2 ? (2 * h + warp) * kHeadDim : kQRows + h * kHeadDim;
    const int4 x = *reinterpret_cast<const int4*>(raw + row + 4 * lane);
    const int32_t xs[4] = {x.x, x.y, x.z, x.w};
    int64_t ss = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss += (int64_t)xs[e] * xs[e];
    ss = warp_sum_i64(ss);
    const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
    const int32_t* gm = warp < 2 ? g_q : g_k;
    int32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = 4 * lane + e;
      const int32_t n = norm_apply(xs[e], inv, gm[d], kHeadNorm);
      const int32_t partner = __shfl_xor_sync(0xFFFFFFFFu, n, 16);
      const int64_t rot = lane < 16 ? -(int64_t)partner : (int64_t)partner;
      o[e] = sat24(((int64_t)n * cos_tab[pos * kHeadDim + d] + rot * sin_tab[pos * kHeadDim + d]) >> 15);
    }
    const int4 o4 = make_int4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<int4*>(&hv[warp][4 * lane]) = o4;
    if (warp == 2) {
      reinterpret_cast<int4*>(kvv.at(layer, 0, h, pos))[lane] = o4;
      kpl_put4(kvv, layer, h, pos, 4 * lane, o4);
      asm volatile("fence.proxy.async.global;" ::: "memory");  // later bulk copies read this row
    }
  } else if (warp == 3 && has_new) {
    const int4 v4 = *reinterpret_cast<const int4*>(raw + kQRows + kKvRows + h * kHeadDim + 4 * lane);
    reinterpret_cast<int4*>(kvv.at(layer, 1, h, pos))[lane] = v4;
    vpl_put4(kvv, layer, h, pos, 4 * lane, v4);
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  __syncthreads();
  if (!umma::bar_wait(&bar, 0)) atomicExch(c.err, 4);
  // 64 positions: warp w takes 8, four at a time (8 lanes per position; lane
  // `sub` holds dims 4 (sub + 8 j) .. +3)
  const int sub = lane & 7, quad = lane >> 3;
  int32_t q0[16], q1[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int4 u = *reinterpret_cast<const int4*>(&hv[0][4 * (sub + 8 * j)]);
    const int4 v = *reinterpret_cast<const int4*>(&hv[1][4 * (sub + 8 * j)]);
    q0[4 * j] = u.x; q0[4 * j + 1] = u.y; q0[4 * j + 2] = u.z; q0[4 * j + 3] = u.w;
    q1[4 * j] = v.x; q1[4 * j + 1] = v.y; q1[4 * j + 2] = v.z; q1[4 * j + 3] = v.w;
  }
  int64_t mx0 = INT64_MIN, mx1 = INT64_MIN;
  int64_t* S0 = a.S + ((size_t)m * kQHeads + 2 * h) * a.max_ctx;
  int64_t* S1 = S0 + a.max_ctx;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int lp = warp * 8 + r * 4 + quad;
    const int p = p0 + lp;
    const int32_t* krow = p == pos ? hv[2] : kpage + lp * kHeadDim;
    int64_t s0 = 0, s1 = 0;
    if (p < ctx) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int4 k4 = *reinterpret_cast<const int4*>(krow + 4 * (sub + 8 * j));
        const int32_t kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          s0 = mad_wide(q0[4 * j + e], kk[e], s0);
          s1 = mad_wide(q1[4 * j + e], kk[e], s1);
        }
      }
    }
#pragma unroll
    for (int msk = 1; msk < 8; msk <<= 1) {
      s0 += shfl_xor_i64(s0, msk);
      s1 += shfl_xor_i64(s1, msk);
    }
    if (p < ctx) {
      const int64_t v0 = scale_score(s0, kScoreScale), v1 = scale_score(s1, kScoreScale);
      if (sub == 0) {
        S0[p] = v0;
        S1[p] = v1;
      }
      mx0 = v0 > mx0 ? v0 : mx0;
      mx1 = v1 > mx1 ? v1 : mx1;
    }
  }
#pragma unroll
  for (int msk = 8; msk < 32; msk <<= 1) {
    const int64_t o0 = shfl_xor_i64(mx0, msk), o1 = shfl_xor_i64(mx1, msk);
    mx0 = o0 > mx0 ? o0 : mx0;
    mx1 = o1 > mx1 ? o1 : mx1;
  }
  if (lane == 0) {
    wmax[warp][0] = mx0;
    wmax[warp][1] = mx1;
  }
  __syncthreads();
  int64_t* Mh = a.M + (size_t)m * kQHeads + 2 * h;
  if (t < 2) {
    int64_t b = wmax[0][t];
    for (int w = 1; w < 8; ++w) b = wmax[w][t] > b ? wmax[w][t] : b;
    atomicMax(reinterpret_cast<long long*>(Mh + t), (long long)b);
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    unsigned* cnt = a.cnt_s + m * kKvHeads + h;
    last = atomicAdd(cnt, 1u) == (unsigned)nch - 1;
    if (last) *cnt = 0;
  }
  __syncthreads();
  if (!last) return;
  // last page of (m, h): scores -> probabilities for both heads
  __threadfence();
  uint32_t* P0 = a.P + ((size_t)m * kQHeads + 2 * h) * a.max_ctx;
#pragma unroll 1
  for (int hh = 0; hh < 2; ++hh) {
    const int64_t mx = ld_cg64(Mh + hh);
    const int64_t* Sh = hh ? S1 : S0;
    int64_t sum = 0;
    for (int p = t; p < ctx; p += blockDim.x) sum += exp_lut[lut_index(mx, ld_cg64(Sh + p))];
    sum = block_sum_i64(sum, red);
    for (int i = t; i < kExpLut; i += blockDim.x)
      probtab[hh][i] = (uint32_t)udiv_exact((uint64_t)exp_lut[i] << 16, (uint64_t)sum);
    __syncthreads();
    uint32_t* Ph = P0 + (size_t)hh * a.max_ctx;
    for (int p = t; p < ctx; p += blockDim.x) Ph[p] = probtab[hh][lut_index(mx, ld_cg64(Sh + p))];
  }
  if (t < 2) Mh[t] = INT64_MIN;
}

__global__ void __launch_bounds__(256) batch_attn_values_kernel(BatchCtx c, AttnScratch a, int layer) {
  __shared__ __align__(128) int32_t vpage[kPage * kHeadDim];  // 32 KB
  __shared__ int2 pr[kPage];
  __shared__ uint64_t bar;
  __shared__ bool last;
  const int pg = blockIdx.x, h = blockIdx.y, m = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  grid_dep_wait();
  grid_dep_launch();
  const int pos = c.pos0[4 * m];
  if (pos >= c.max_ctx || pg * kPage > pos) return;
  const int ctx = pos + 1, nch = (ctx + kPage - 1) / kPage;
  const int p0 = pg * kPage;
  const int n = min(kPage, ctx - p0);
  if (t == 0) {
    umma::bar_init(&bar, 1);
    umma::bar_init_fence();
    umma::bar_expect_tx(&bar, (uint32_t)n * kHeadDim * 4);
    bulk_load(vpage, c.slots[m].kv.at(layer, 1, h, p0), (uint32_t)n * kHeadDim * 4, &bar);
  }
  const uint32_t* P0 = a.P + ((size_t)m * kQHeads + 2 * h) * a.max_ctx;
  if (t < kPage) pr[t] = t < n ? make_int2((int)P0[p0 + t], (int)P0[a.max_ctx + p0 + t]) : make_int2(0, 0);
  __syncthreads();
  if (!umma::bar_wait(&bar, 0)) atomicExch(c.err, 4);
  int64_t a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
#pragma unroll 4
  for (int u = 0; u < 8; ++u) {
    const int lp = warp + 8 * u;
    if (lp < n) {
      const int4 v4 = *reinterpret_cast<const int4*>(vpage + lp * kHeadDim + 4 * lane);
      const int2 p = pr[lp];
      const int32_t vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a0[e] = mad_wide(p.x, vv[e], a0[e]);
        a1[e] = mad_wide(p.y, vv[e], a1[e]);
      }
    }
  }
  // the page is consumed: its buffer takes the cross-warp sums [8][2][128]
  __syncthreads();
  int64_t* part = reinterpret_cast<int64_t*>(vpage);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    part[(warp * 2 + 0) * kHeadDim + 4 * lane + e] = a0[e];
    part[(warp * 2 + 1) * kHeadDim + 4 * lane + e] = a1[e];
  }
  __syncthreads();
  const int hh = t >> 7, d = t & (kHeadDim - 1);
  int64_t acc = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) acc += part[(w * 2 + hh) * kHeadDim + d];
  int64_t* Oh = a.O + ((size_t)m * kQHeads + 2 * h + hh) * kHeadDim;
  atomicAdd(reinterpret_cast<unsigned long long*>(Oh + d), (unsigned long long)acc);
  __threadfence();
  __syncthreads();
  if (t == 0) {
    unsigned* cnt = a.cnt_v + m * kKvHeads + h;
    last = atomicAdd(cnt, 1u) == (unsigned)nch - 1;
    if (last) *cnt = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int64_t sum = ld_cg64(Oh + d);
  Oh[d] = 0;
  write_limbs(c.bt2, c.SP, 2 * kHidden, m, (2 * h + hh) * kHeadDim + d, sat24(sum >> 16));
}

// Attention for one (KV head, sequence): q/k head RMSNorm + RoPE, KV append,
// exact two-pass LUT softmax for the two query heads of the group; writes the
// output and its limbs (the o_proj B matrix).  256 threads.  Used when the
// batch has enough (KV head, sequence) pairs to fill the GPU and contexts up
// to 1024; smaller batches and longer contexts use the cluster kernels
// (batch_attn_cl_tc_kernel with byte planes, batch_attn_cl_kernel without),
// the longest ones the split-KV kernels above.
//
// Scores on the tensor cores.  With the query split into the unsigned byte
// limbs c_b of c = q + 2^23 and the cached key into its byte planes k_a
// (k = sum_a 2^(8 a) k_a, k_2 signed; KvView::kpl),
//   q . k = sum_a 2^(8 a) (sum_b 2^(8 b) D_a[b] - 2^23 D_a[ones]),
//   D_a[x] = sum_d k_a[d] x[d]  (|D_a| < 2^23, exact in int32),
// so a 128-key chunk takes one M128 x N16 x K128 kind::i8 product per plane:
// A = the plane's 128 key rows as copied from the cache (two pages), B = 16
// rows of query bytes (c_b of both heads, a row of ones, zero rows), D in
// TMEM, read back by warps 0-3 (lane = key) and combined in int64.  The
// current position's key comes from this kernel's own q/k/v row and is
// scored on the CUDA cores.  Values the same way round: with the
// probability p <= 2^16 split into bytes p_b and the values into the
// transposed byte planes v_a (dims x positions; KvView::vpl),
//   sum_p p v[d] = sum_a 2^(8 a) sum_b 2^(8 b) E_a[d][b],
//   E_a[d][b] = sum_p v_a[d][p] p_b[p]  (|E_a| < 2^26 for 1024 positions),
// one M128 (dims) x N16 x K128 (positions) product per plane and chunk, A
// = two 64-byte-swizzled page planes, B = 16 rows of probability bytes, E
// accumulated in TMEM over the chunks; the current position's value is
// added on the CUDA cores.  One ring of two 16 KB slots carries the chunks'
// key planes (loads i = 0 .. 3 nch - 1, plane i % 3 of chunk i / 3), then
// their value planes, each slot released by the MMA's commit; the first
// loads start before the dependency wait.
constexpr int kAttnChunk = 32;
constexpr int kAttnChunkBytes = kAttnChunk * kHeadDim * 4;
constexpr int kAttnRing = 2;
constexpr int kStageAttnRing = 4;
constexpr int kTcKeys = 128;                  // keys per score chunk (the MMA's M)
constexpr int kTcSlot = 16384;                // ring slot: one key or value plane of a 128-position chunk
constexpr int kTcSmemFixed = 1024 + 2 * kTcSlot + 16 * 128;  // alignment slack, ring, query bytes
constexpr uint32_t kTcCols = 128;             // TMEM columns: D (scores) at 0, E (values) at 64, 3 planes x 16
constexpr uint32_t kTcVal = 64;

// Shared-memory descriptor of a K-major tile with 64-byte rows, 64-byte
// swizzled (8-row atoms of 512 bytes).
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

__global__ void __launch_bounds__(256, 4) batch_attn_kernel(BatchCtx c, int layer, const int32_t* __restrict__ g_q,
                                                            const int32_t* __restrict__ g_k,
                                                            const int32_t* __restrict__ cos_tab,
                                                            const int32_t* __restrict__ sin_tab,
                                                            const int32_t* __restrict__ exp_lut) {
  extern __shared__ uint8_t attn_raw[];
  // 128-byte-swizzled operand tiles need 1024-byte alignment
  const uint32_t raw_addr = umma::smem_addr(attn_raw);
  uint8_t* sbase = attn_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* slots = sbase;                                   // [2][16 KB]
  uint8_t* qb = sbase + 2 * kTcSlot;                        // [16][128] query bytes
  int64_t* sc = reinterpret_cast<int64_t*>(qb + 16 * 128);  // [2][ctx]; later the probability bytes
  uint8_t* pb = reinterpret_cast<uint8_t*>(sc);              // [nch][16][128] probability bytes
  __shared__ __align__(16) int32_t hv[4][kHeadDim];  // roped q0, q1, k; raw v
  __shared__ uint32_t probtab[2][kExpLut];
  __shared__ int64_t red[2][8];
  __shared__ uint64_t full[2], empty[2], dfull, dempty, vdone;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t ppos[2];  // the current position's probability per head
  const int kv = blockIdx.x, m = blockIdx.y;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  attn_stamp(c, layer, m, kv, 0);
  // The cached K/V rows (positions < pos, written by earlier steps) and the
  // position itself (advanced at the end of the previous step) do not depend
  // on the kernels of this step: the first loads start before the wait for
  // the q/k/v projections.
  const int pos = c.pos0[4 * m];
  if (pos >= c.max_ctx) return;
  const int ctx = pos + 1;
  const KvView kvv = c.slots[m].kv;
  if (!kvv.kpl || !kvv.vpl) {  // the model holds no byte planes (it allocates them where this kernel runs)
    if (t == 0) atomicExch(c.err, 4);
    return;
  }
  const int nch = (pos + kTcKeys - 1) / kTcKeys;  // chunks of the cached positions [0, pos)
  const int nkp = 3 * nch;                        // key-plane loads, then as many value-plane loads
  const int total = 2 * nkp;
  auto issue = [&](int i) {
    uint64_t* b = full + (i & 1);
    uint8_t* dst = slots + (i & 1) * kTcSlot;
    if (i < nkp) {
      const int ch = i / 3, a = i - 3 * ch, k0 = ch * kTcKeys;
      const int n0 = pos - k0 < kKvPage ? pos - k0 : kKvPage;  // >= 1
      int n1 = pos - k0 - kKvPage;
      n1 = n1 < 0 ? 0 : (n1 > kKvPage ? kKvPage : n1);
      umma::bar_expect_tx(b, (uint32_t)(n0 + n1) * 128u);
      bulk_load(dst, kvv.kplane(layer, kv, k0) + a * kKplPlane, (uint32_t)n0 * 128u, b);
      if (n1 > 0)
        bulk_load(dst + kKplPlane, kvv.kplane(layer, kv, k0 + kKvPage) + a * kKplPlane, (uint32_t)n1 * 128u, b);
    } else {
      // whole page planes (positions past pos get probability 0)
      const int j = i - nkp, ch = j / 3, a = j - 3 * ch, k0 = ch * kTcKeys;
      const bool two = k0 + kKvPage < pos;
      umma::bar_expect_tx(b, (two ? 2u : 1u) * kKplPlane);
      bulk_load(dst, kvv.vplane(layer, kv, k0) + a * kKplPlane, kKplPlane, b);
      if (two) bulk_load(dst + kKplPlane, kvv.vplane(layer, kv, k0 + kKvPage) + a * kKplPlane, kKplPlane, b);
    }
  };
  if (t == 0) {
    umma::bar_init(full, 1);
    umma::bar_init(full + 1, 1);
    umma::bar_init(empty, 1);
    umma::bar_init(empty + 1, 1);
    umma::bar_init(&dfull, 1);
    umma::bar_init(&dempty, 4);
    umma::bar_init(&vdone, 1);
    umma::bar_init_fence();
    for (int i = 0; i < total && i < 2; ++i) issue(i);
  }
  if (warp == 1) umma::tmem_alloc(&tmem_slot, kTcCols);
  // the exp LUT into probtab[0] now, off the critical path: the softmax of
  // every CTA would otherwise fetch the same few L2 lines at about the same time
  for (int e = t; e < kExpLut; e += blockDim.x) probtab[0][e] = (uint32_t)exp_lut[e];
  grid_dep_wait();
  grid_dep_launch();
  const int32_t* raw = c.qkv_raw + (size_t)m * (kQRows + 2 * kKvRows);
  // warp 0: q head 2kv, warp 1: q head 2kv+1, warp 2: k (normed, roped);
  // warp 3: v.  A lane owns dims 4 lane .. 4 lane + 3; the RoPE partner
  // d +- 64 sits 16 lanes away.
  if (warp < 3) {
    const int row = warp < 2 ? (2 * kv + warp) * kHeadDim : kQRows + kv * kHeadDim;
    const int4 x = *reinterpret_cast<const int4*>(raw + row + 4 * lane);
    const int4 cs = *reinterpret_cast<const int4*>(cos_tab + pos * kHeadDim + 4 * lane);
    const int4 sn = *reinterpret_cast<const int4*>(sin_tab + pos * kHeadDim + 4 * lane);
    const int4 gm = *reinterpret_cast<const int4*>((warp < 2 ? g_q : g_k) + 4 * lane);
    const int32_t xs[4] = {x.x, x.y, x.z, x.w}, cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
    const int32_t gv[4] = {gm.x, gm.y, gm.z, gm.w};
    int64_t ss = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = mad_wide(xs[e], xs[e], ss);
    ss = warp_sum_i64(ss);
    const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
    int32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int32_t n = norm_apply(xs[e], inv, gv[e], kHeadNorm);
      const int32_t partner = __shfl_xor_sync(0xFFFFFFFFu, n, 16);
      const int64_t rot = lane < 16 ? -(int64_t)partner : (int64_t)partner;
      o[e] = sat24(((int64_t)n * cv[e] + rot * sv[e]) >> 15);
    }
    const int4 o4 = make_int4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<int4*>(&hv[warp][4 * lane]) = o4;
    if (warp == 2) {
      reinterpret_cast<int4*>(kvv.at(layer, 0, kv, pos))[lane] = o4;
      kpl_put4(kvv, layer, kv, pos, 4 * lane, o4);
    }
  } else if (warp == 3) {
    const int4 v4 = *reinterpret_cast<const int4*>(raw + kQRows + kKvRows + kv * kHeadDim + 4 * lane);
    *reinterpret_cast<int4*>(&hv[3][4 * lane]) = v4;
    reinterpret_cast<int4*>(kvv.at(layer, 1, kv, pos))[lane] = v4;
    vpl_put4(kvv, layer, kv, pos, 4 * lane, v4);
  }
  __syncthreads();
  // query bytes, 128-byte-swizzled K-major: thread (row r = t / 16, dims
  // 8 (t % 16) .. +7); rows 3 h + b: byte b of q_h + 2^23, row 6: ones
  {
    const int r = t >> 4, d0 = 8 * (t & 15);
    uint32_t w0 = 0, w1 = 0;
    if (r < 6) {
      const int h = r >= 3, b = r - 3 * h;
      const int4 lo = *reinterpret_cast<const int4*>(&hv[h][d0]);
      const int4 hi = *reinterpret_cast<const int4*>(&hv[h][d0 + 4]);
      const int4 bl = make_int4(lo.x + (1 << 23), lo.y + (1 << 23), lo.z + (1 << 23), lo.w + (1 << 23));
      const int4 bh = make_int4(hi.x + (1 << 23), hi.y + (1 << 23), hi.z + (1 << 23), hi.w + (1 << 23));
      w0 = byte_plane_word(bl, b);
      w1 = byte_plane_word(bh, b);
    } else if (r == 6) {
      w0 = w1 = 0x01010101u;
    }
    *reinterpret_cast<uint2*>(qb + kpl_off(r, d0)) = make_uint2(w0, w1);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // read by the tensor cores
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  attn_stamp(c, layer, m, kv, 1);
  bool ok = true;
  int64_t mx0 = INT64_MIN, mx1 = INT64_MIN;
  // the current position's scores (warp 5)
  if (warp == 5) {
    const int4 k4 = *reinterpret_cast<const int4*>(&hv[2][4 * lane]);
    const int4 qa = *reinterpret_cast<const int4*>(&hv[0][4 * lane]);
    const int4 qc = *reinterpret_cast<const int4*>(&hv[1][4 * lane]);
    int64_t s0 = 0, s1 = 0;
    s0 = mad_wide(qa.x, k4.x, s0);
    s0 = mad_wide(qa.y, k4.y, s0);
    s0 = mad_wide(qa.z, k4.z, s0);
    s0 = mad_wide(qa.w, k4.w, s0);
    s1 = mad_wide(qc.x, k4.x, s1);
    s1 = mad_wide(qc.y, k4.y, s1);
    s1 = mad_wide(qc.z, k4.z, s1);
    s1 = mad_wide(qc.w, k4.w, s1);
    s0 = warp_sum_i64(s0);
    s1 = warp_sum_i64(s1);
    if (lane == 0) {
      mx0 = scale_score(s0, kScoreScale);
      mx1 = scale_score(s1, kScoreScale);
      sc[pos] = mx0;
      sc[ctx + pos] = mx1;
    }
  }
  if (t == 128) {
    // MMA issuer (warp 4): key plane i into D_(i % 3); chunk ch waits until
    // the previous chunk's D is read
    const uint64_t qdesc = umma::sw128_desc(umma::smem_addr(qb));
    for (int i = 0; i < nkp && ok; ++i) {
      const int ch = i / 3, a = i - 3 * ch;
      if (a == 0 && ch > 0 && !umma::bar_wait(&dempty, (ch - 1) & 1)) ok = false;
      if (ok && !umma::bar_wait(full + (i & 1), (i >> 1) & 1)) ok = false;
      if (!ok) break;
      umma::fence_after_sync();
      const uint64_t kdesc = umma::sw128_desc(umma::smem_addr(slots + (i & 1) * kTcSlot));
      const uint32_t idesc = umma::i8_idesc_ab(kTcKeys, 16, a == 2, false);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma::mma_i8(tmem + 16u * a, kdesc + (uint64_t)(2 * kk), qdesc + (uint64_t)(2 * kk), idesc, kk > 0);
      umma::mma_commit(empty + (i & 1));
      if (a == 2) umma::mma_commit(&dfull);
      if (i + 2 < total) {
        // the slot's MMAs have read it: reload
        if (!umma::bar_wait(empty + (i & 1), (i >> 1) & 1)) {
          ok = false;
          break;
        }
        issue(i + 2);
      }
    }
  }
  // scores of each chunk: warp w < 4 reads D of the three planes for TMEM
  // lanes (keys) 32 w .. 32 w + 31, both heads
  for (int ch = 0; ch < nch && warp < 4; ++ch) {
    // the warp agrees on the outcome: the TMEM loads below are warp-wide
    if (!__all_sync(0xFFFFFFFFu, umma::bar_wait(&dfull, ch & 1))) {
      ok = false;
      break;
    }
    umma::fence_after_sync();
    int32_t d[3][8];
    const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll
    for (int a = 0; a < 3; ++a) umma::tmem_ld<8>(lb + 16u * a, d[a]);
    umma::tmem_ld_wait();
    umma::fence_before_sync();
    __syncwarp();
    if (lane == 0) umma::bar_arrive(&dempty);
    const int key = ch * kTcKeys + 32 * warp + lane;
    if (key < pos) {
      int64_t s0 = 0, s1 = 0;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const int64_t bias = (int64_t)d[a][6] << 23;
        const int64_t t0 = (int64_t)d[a][0] + ((int64_t)d[a][1] << 8) + ((int64_t)d[a][2] << 16) - bias;
        const int64_t t1 = (int64_t)d[a][3] + ((int64_t)d[a][4] << 8) + ((int64_t)d[a][5] << 16) - bias;
        s0 += t0 << (8 * a);
        s1 += t1 << (8 * a);
      }
      const int64_t v0 = scale_score(s0, kScoreScale), v1 = scale_score(s1, kScoreScale);
      sc[key] = v0;
      sc[ctx + key] = v1;
      mx0 = v0 > mx0 ? v0 : mx0;
      mx1 = v1 > mx1 ? v1 : mx1;
    }
  }
  attn_stamp(c, layer, m, kv, 2);
  // maxima of both heads (one block reduction)
#pragma unroll
  for (int msk = 1; msk < 32; msk <<= 1) {
    const int64_t o0 = shfl_xor_i64(mx0, msk), o1 = shfl_xor_i64(mx1, msk);
    mx0 = o0 > mx0 ? o0 : mx0;
    mx1 = o1 > mx1 ? o1 : mx1;
  }
  if (lane == 0) {
    red[0][warp] = mx0;
    red[1][warp] = mx1;
  }
  __syncthreads();
  mx0 = red[0][0];
  mx1 = red[1][0];
#pragma unroll
  for (int w = 1; w < 8; ++w) {
    mx0 = red[0][w] > mx0 ? red[0][w] : mx0;
    mx1 = red[1][w] > mx1 ? red[1][w] : mx1;
  }
  // LUT indices and exp sums of both heads (one block reduction)
  int64_t sum0 = 0, sum1 = 0;
  for (int p = t; p < ctx; p += blockDim.x) {
    const int i0 = lut_index(mx0, sc[p]), i1 = lut_index(mx1, sc[ctx + p]);
    sc[p] = i0;
    sc[ctx + p] = i1;
    sum0 += probtab[0][i0];
    sum1 += probtab[0][i1];
  }
  sum0 = warp_sum_i64(sum0);
  sum1 = warp_sum_i64(sum1);
  __syncthreads();  // red reused
  if (lane == 0) {
    red[0][warp] = sum0;
    red[1][warp] = sum1;
  }
  __syncthreads();
  sum0 = 0;
  sum1 = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    sum0 += red[0][w];
    sum1 += red[1][w];
  }
  {
    // warps 4-7 build head 1's table from the LUT in probtab[0]; warps 0-3
    // compute head 0's in registers and overwrite the LUT once every read of
    // it is done: one reciprocal per thread
    const int h = t >> 7, e0 = t & 127;
    const uint64_t dd = (uint64_t)(h ? sum1 : sum0), rc = ~0ULL / dd;
    uint32_t p0[3] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int e = e0 + 128 * k;
      if (e < kExpLut) {
        const uint32_t v = barrett_div((uint64_t)probtab[0][e] << 16, dd, rc);
        if (h)
          probtab[1][e] = v;
        else
          p0[k] = v;
      }
    }
    __syncthreads();
    if (h == 0) {
#pragma unroll
      for (int k = 0; k < 3; ++k)
        if (e0 + 128 * k < kExpLut) probtab[0][e0 + 128 * k] = p0[k];
    }
  }
  __syncthreads();
  // probabilities of this thread's positions t + 256 j (ctx <= 1024) into
  // registers, then the index array becomes the probability bytes: chunk c,
  // row 3 h + b = byte b of head h's probability, 128-byte swizzled, zero for
  // the current position (added below) and past it
  uint32_t pr[4][2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int p = t + 256 * j;
    pr[j][0] = pr[j][1] = 0;
    if (p < ctx) {
      pr[j][0] = probtab[0][(int)sc[p]];
      pr[j][1] = probtab[1][(int)sc[ctx + p]];
      if (p == pos) {
        ppos[0] = pr[j][0];
        ppos[1] = pr[j][1];
      }
    }
  }
  __syncthreads();
  for (int i = t; i < nch * 128; i += blockDim.x) reinterpret_cast<uint4*>(pb)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int p = t + 256 * j;
    if (p < pos) {
      uint8_t* tile = pb + (p >> 7) * 2048;
      const int k = p & 127;
#pragma unroll
      for (int r = 0; r < 6; ++r) {
        const uint32_t v = pr[j][r >= 3] >> (8 * (r % 3));
        if (v & 0xFFu) tile[r * 128 + (((k >> 4) ^ (r & 7)) << 4) + (k & 15)] = (uint8_t)v;
      }
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // read by the tensor cores
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  attn_stamp(c, layer, m, kv, 3);
  if (t == 128) {
    // value products: plane a of chunk ch into E_a, accumulated over the chunks
    const uint64_t pdesc = umma::sw128_desc(umma::smem_addr(pb));
    for (int j = 0; j < nkp && ok; ++j) {
      const int i = nkp + j, ch = j / 3, a = j - 3 * ch;
      if (!umma::bar_wait(full + (i & 1), (i >> 1) & 1)) {
        ok = false;
        break;
      }
      umma::fence_after_sync();
      const uint32_t sa = umma::smem_addr(slots + (i & 1) * kTcSlot);
      const uint32_t idesc = umma::i8_idesc_ab(kTcKeys, 16, a == 2, false);
      const bool two = ch * kTcKeys + kKvPage < pos;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (kk >= 2 && !two) break;  // the second page holds no cached position
        const uint64_t vdesc = sw64_desc(sa + (kk >> 1) * kKplPlane) + (uint64_t)(2 * (kk & 1));
        const uint64_t bdesc = pdesc + (uint64_t)((ch * 2048 + 32 * kk) >> 4);
        umma::mma_i8(tmem + kTcVal + 16u * a, vdesc, bdesc, idesc, (ch | kk) != 0);
      }
      umma::mma_commit(empty + (i & 1));
      if (i + 2 < total) {
        if (!umma::bar_wait(empty + (i & 1), (i >> 1) & 1)) {
          ok = false;
          break;
        }
        issue(i + 2);
      }
    }
    umma::mma_commit(&vdone);  // every MMA of this CTA is done when it arrives
  }
  // outputs: warp w < 4 reads E for dims 32 w .. 32 w + 31 (TMEM lanes)
  if (warp < 4) {
    const int d = 32 * warp + lane;
    int64_t o0 = 0, o1 = 0;
    const bool got = __all_sync(0xFFFFFFFFu, umma::bar_wait(&vdone, 0));
    if (!got) ok = false;
    umma::fence_after_sync();
    if (nch > 0 && got) {
      int32_t e[3][8];
      const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16) + kTcVal;
#pragma unroll
      for (int a = 0; a < 3; ++a) umma::tmem_ld<8>(lb + 16u * a, e[a]);
      umma::tmem_ld_wait();
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        o0 += ((int64_t)e[a][0] + ((int64_t)e[a][1] << 8) + ((int64_t)e[a][2] << 16)) << (8 * a);
        o1 += ((int64_t)e[a][3] + ((int64_t)e[a][4] << 8) + ((int64_t)e[a][5] << 16)) << (8 * a);
      }
    }
    o0 += (int64_t)ppos[0] * hv[3][d];
    o1 += (int64_t)ppos[1] * hv[3][d];
    write_limbs(c.bt2, c.SP, 2 * kHidden, m, (2 * kv) * kHeadDim + d, sat24(o0 >> 16));
    write_limbs(c.bt2, c.SP, 2 * kHidden, m, (2 * kv + 1) * kHeadDim + d, sat24(o1 >> 16));
  }
  attn_stamp(c, layer, m, kv, 4);
  if (!ok) atomicExch(c.err, 4);
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, kTcCols);
  }
  attn_stamp(c, layer, m, kv, 5);
}

// ---------------------------------------------------------------------------
// Exact batched GEMM on the 5th-generation tensor cores, reading the Q4
// weights as stored (packed nibbles + u16 Q2.14 group scales).
//
//   out[r][m] = sum_k w[r][k] s[r][k / 64] a[m][k]     (exact, int64)
//
// with w the int4 weight, s its group scale and a the signed 24-bit
// activation of sequence m.  The scale is split into 4-bit digits
// s = sum_j 16^j s_j, so every w s_j lies in [-120, 105] and fits a signed
// byte: "plane" j of the A operand holds w s_j for every weight.  The
// activation enters as the three unsigned byte limbs c_i of c = a + 2^23
// (the B limb matrix, rows limb * SP + m).  Then
//   sum_k w s a = sum_{j,i} 16^j 256^i T[j][i] - 2^23 sum_k w s,
//   T[j][i][r][m] = sum_k (w s_j)[r][k] c_i[m][k],
// and each T is one int32 tensor-core accumulator over the CTA's whole K
// range (|T| < 120 * 255 * K): TMEM is read once per tile, not once per
// 64-column scale group.
//
// CTA tile: 128 weight rows x SN sequences (SN = SP columns of the limb
// matrix in decode: MMA N = 3 SN rounded up to 16, zero rows past 3 SN), K in
// 128-wide tiles.  An M128 x K32 kind::i8 MMA costs about 46 clocks at
// N <= 48 and 96 at N = 192, so chunks of fewer sequences buy nothing: a CTA
// takes all of them and K is split over the CTAs of a cluster instead where
// a matrix has few row tiles (q/k/v 4, gate/up 2, o_proj and down 8, the LM
// head 1).  Warp 0 issues the
// TMA loads (packed weights into a 4-slot ring, the three limb boxes of the
// chunk into a limb ring), warp 1 owns TMEM and issues tcgen05.mma (kind::i8,
// s8 x u8 -> s32), and warps 2-17 first build the planes of each K tile in
// shared memory, then read the accumulators and run the epilogue.
// Building a plane: u = w + 8 (nibble ^ 8) times s_j plus 128 - 8 s_j in
// each byte stays within [8, 233] (one IMAD per four weights, no carry
// between bytes), and XOR 0x80 turns it into the signed byte w s_j; the bytes
// go to the 128-byte-swizzled K-major layout the MMA descriptor expects.
// One pass covers two digits (2p, 2p + 1, accumulators T[2p..2p+1] at TMEM
// columns [0, N) and [N, 2N)); tiles whose scales all fit in 8 bits (the
// usual case) need one pass, others a second with the loads repeated and the
// accumulators read out in between.  The weight tiles and planes do not
// depend on earlier kernels, so the first ones are loaded and built before
// griddepcontrol.wait.
// K may be split over the CTAs of a cluster (gridDim.y = splits <= 8); the
// partial sums then meet in the owning CTA's shared memory over DSMEM.
// ---------------------------------------------------------------------------
enum GemmKind { kGemmQkv = 0, kGemmO = 1, kGemmGu = 2, kGemmDown = 3, kGemmLm = 4 };

constexpr int kUThreads = 576;  // 18 warps
constexpr int kUMaxKt = 8;      // K tiles per CTA (K / splits <= 1024)

template <int SN, int KIND>
struct UCfg {
  static constexpr int NM = (3 * SN + 15) / 16 * 16;  // MMA N: three limb blocks of SN columns
  static constexpr int Q = SN / 4;                    // sequences per epilogue thread
  static constexpr int A_PK = 128 * 128;              // packed weights of two 128-wide K tiles (one A stage)
  static constexpr int PLANE = 128 * 128;             // one plane of a K tile
  static constexpr int B_BYTES = NM * 128;            // limb tile (3 boxes of SN rows + zero rows)
  static constexpr int SA = 2;                        // packed-weight stages in flight (four K tiles)
  static constexpr int SB = KIND == kGemmLm && SN == 64 ? 4 : SN == 64 ? 2 : 3;  // limb tiles in flight
  static constexpr int SPL = 2;                       // plane pairs in flight
  static constexpr int TCOLS = 2 * NM <= 32 ? 32 : 2 * NM <= 64 ? 64 : 2 * NM <= 128 ? 128 : 2 * NM <= 256 ? 256 : 512;
  // per-row partial sums [splits][SN][rows]; the LM head never splits K and
  // keeps them in the plane slots, free once its MMAs are done
  static constexpr bool RED_IN_PLANES = KIND == kGemmLm;
  static constexpr int RED_BYTES = 128 * SN * 8;
  // operands of the final epilogue staged during the K loop: the residual
  // rows a CTA owns (O / down, splits >= 2: at most 64 rows x SN) or the
  // sigmoid table (gate/up)
  static constexpr int STG_BYTES = KIND == kGemmO || KIND == kGemmDown ? 64 * SN * 4
                                   : KIND == kGemmGu                   ? (4 * kSigLut + 15) / 16 * 16
                                                                       : 0;
  static constexpr size_t OFF_B = (size_t)SPL * 2 * PLANE;
  static constexpr size_t OFF_A = OFF_B + (size_t)SB * B_BYTES;
  static constexpr size_t OFF_RED = RED_IN_PLANES ? 0 : OFF_A + (size_t)SA * A_PK;
  static constexpr size_t OFF_RB = (RED_IN_PLANES ? OFF_A + (size_t)SA * A_PK : OFF_RED + RED_BYTES);
  static constexpr size_t OFF_BAR = OFF_RB + 1024;  // barriers, TMEM slot, flags, live[64]
  static constexpr size_t OFF_STG = OFF_BAR + 512;
  static constexpr size_t SMEM = 1024 + OFF_STG + STG_BYTES;
  static constexpr uint32_t IDESC = umma::i8_idesc(128, NM);
  static_assert(2 * NM <= 512, "two accumulator sets must fit TMEM");
  static_assert(B_BYTES % 1024 == 0 && SN % 8 == 0, "limb boxes stay on 1024-byte swizzle atoms");
  static_assert(!RED_IN_PLANES || RED_BYTES <= OFF_B, "row sums fit the plane slots");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Up to four byte ranges (16-byte aligned, sizes multiples of 16) that the
// CTAs of a launch prefetch into L2 between them, marked evict-last.
struct L2Prefetch {
  const void* p[4];
  uint32_t bytes[4];
};

__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  const uint32_t n = gridDim.x * gridDim.y * gridDim.z;
  const uint32_t i = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    if (!pf.p[r]) continue;
    const uint32_t chunk = ((pf.bytes[r] + n - 1) / n + 15u) & ~15u, off = i * chunk;
    if (off < pf.bytes[r]) {
      const uint32_t end = pf.bytes[r] - off < chunk ? pf.bytes[r] : off + chunk;
      for (uint32_t o = off; o < end; o += 65536u) {  // pieces of at most 64 KB
        const uint32_t len = end - o < 65536u ? end - o : 65536u;
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(
                         reinterpret_cast<const char*>(pf.p[r]) + o),
                     "r"(len), "l"(pol)
                     : "memory");
      }
    }
  }
}

struct UGemm {
  BatchCtx c;
  const uint16_t* scales;   // [rows, K / 64]; gate/up: the gate rows' scales
  const uint16_t* scales2;  // gate/up: the up rows' scales ([3072, 16])
  int rows;                 // rows of A (the LM head's may end inside the last tile)
  int K;
  int kt_per_split;         // 128-wide K tiles each CTA of a cluster covers (<= kUMaxKt)
  int SP;                   // padded sequences of the limb matrix (its rows are limb * SP + m)
  int chunks;               // sequence chunks of SN per sub-batch (SP / SN)
  int b_sub_rows;           // limb-matrix rows between consecutive sub-batches (prefill)
  const int32_t* sig_lut;
  ArgBestD* partial;        // LM head: [tiles, 64]
  unsigned long long* trace;  // optional: [CTA][8] %globaltimer stamps of this launch (nullptr = off)
  L2Prefetch pf;            // the next GEMM's weights, pulled into L2 while this one runs
};

// GEMM timeline points: 0 entry, 1 set-up done, 2 dependency released (TMA
// warp), 3 accumulators ready, 4 accumulators read, 5 partial sums exchanged,
// 6 epilogue done, 7 last K tile issued (epilogue warp 2 records 3-4, the MMA
// thread 7, thread 0 the rest)
__device__ __forceinline__ void gemm_stamp(const UGemm& g, int k) {
  if (g.trace) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g.trace[(((size_t)blockIdx.y * gridDim.z + blockIdx.z) * gridDim.x + blockIdx.x) * 8 + k] = t;
  }
}

// 16 packed weights (8 bytes, k order) -> four words of biased weights
// u = w + 8 in [0, 15], one per byte, U[t] holding k = 4t .. 4t + 3.
__device__ __forceinline__ void unpack16_biased(uint2 x, uint32_t* U) {
  const uint32_t l0 = (x.x ^ 0x88888888u) & 0x0F0F0F0Fu;         // k 0, 2, 4, 6
  const uint32_t h0 = ((x.x >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;  // k 1, 3, 5, 7
  const uint32_t l1 = (x.y ^ 0x88888888u) & 0x0F0F0F0Fu;
  const uint32_t h1 = ((x.y >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
  U[0] = __byte_perm(l0, h0, 0x5140);
  U[1] = __byte_perm(l0, h0, 0x7362);
  U[2] = __byte_perm(l1, h1, 0x5140);
  U[3] = __byte_perm(l1, h1, 0x7362);
}

// Signed bytes w * d (d a 4-bit scale digit) of four biased weights.
__device__ __forceinline__ uint32_t plane_word(uint32_t u4, uint32_t d, uint32_t bias) {
  return (u4 * d + bias) ^ 0x80808080u;
}

template <int SN, int KIND>
__global__ void __launch_bounds__(kUThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap amap2,
                     const __grid_constant__ CUtensorMap bmap, UGemm g) {
  using C = UCfg<SN, KIND>;
  constexpr int SA = C::SA, SB = C::SB, SPL = C::SPL;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = umma::smem_addr(smem_raw);
  uint8_t* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* planes = sm;
  uint8_t* bstage = sm + C::OFF_B;
  uint8_t* astage = sm + C::OFF_A;
  int64_t* red = reinterpret_cast<int64_t*>(sm + C::OFF_RED);
  int64_t* rbs = reinterpret_cast<int64_t*>(sm + C::OFF_RB);
  uint64_t* full_a = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* empty_a = full_a + SA;
  uint64_t* full_b = empty_a + SA;
  uint64_t* empty_b = full_b + SB;
  uint64_t* full_p = empty_b + SB;
  uint64_t* empty_p = full_p + SPL;
  uint64_t* tfull = empty_p + SPL;
  uint64_t* tempty = tfull + 1;
  uint64_t* scales_in = tempty + 1;  // the builders know whether a second pass is needed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(scales_in + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* wide_any = reinterpret_cast<int*>(tmem_slot + 2);
  int* live = reinterpret_cast<int*>(tmem_slot + 4);  // [64]: sequence m of the chunk takes part in this step
  int32_t* stg = reinterpret_cast<int32_t*>(sm + C::OFF_STG);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (sub-batch x sequence chunk, K splits, row tiles): the CTAs of one
  // weight tile are adjacent in launch order and share its reads through L2
  const int tile = blockIdx.z, split = blockIdx.y, splits = gridDim.y;
  const int nkt = g.kt_per_split, kt0 = split * nkt;
  const int row0 = tile * 128;
  const int G = g.K / 64;
  const int SP = g.SP;
  const int z = blockIdx.x / g.chunks, n0 = (blockIdx.x - z * g.chunks) * SN;
  // this CTA's sequences: columns SP z + n0 .. + SN - 1 of the batch
  BatchCtx c = g.c;
  {
    const size_t m0 = (size_t)SP * z + n0;
    c.qkv_raw += m0 * (kQRows + 2 * kKvRows);
    c.pos0 += 4 * m0;
    c.hidden0 += m0 * kHidden;
    c.post0 += m0 * kHidden;
    c.bt3 += z * c.bt_sub3;
    const int rem = c.S - SP * z - n0;
    c.S = rem < 0 ? 0 : (rem < SN ? rem : SN);
  }
  // weight rows of this tile: 128 consecutive rows, or for gate/up 64 gate
  // rows then the matching 64 up rows (amap2)
  const int arow0 = KIND == kGemmGu ? tile * 64 : row0;
  const int arow1 = KIND == kGemmGu ? tile * 64 : row0 + 64;

  if (threadIdx.x == 0) gemm_stamp(g, 0);
  // A stage u holds K tiles 2 (u % upp), + 1 of pass u / upp: one 128-row x
  // 128-byte box (gate/up: a 64-row box of each matrix), 128-byte swizzled
  const int upp = (nkt + 1) >> 1;
  const int pre_a = upp < SA ? upp : SA;
  auto issue_a = [&](int u) {
    const int sa = u % SA, x = (kt0 + 2 * (u % upp)) * 64;
    umma::bar_expect_tx(full_a + sa, C::A_PK);
    umma::tma_load(astage + sa * C::A_PK, &amap, x, arow0, full_a + sa);
    if (KIND == kGemmGu) umma::tma_load(astage + sa * C::A_PK + C::A_PK / 2, &amap2, x, arow1, full_a + sa);
  };
  // barrier set-up spread over warp 0 (one barrier per lane): thread 0 issues
  // the first weight loads right after
  if (warp == 0) {
    constexpr int kBars = 2 * SA + 2 * SB + 2 * SPL + 3;
    static_assert(kBars <= 32, "one barrier per lane of warp 0");
    if (lane < kBars) {
      const int b = lane;
      const unsigned count = b < SA                            ? 1u
                             : b < 2 * SA                      ? 16u
                             : b < 2 * SA + 2 * SB             ? 1u
                             : b < 2 * SA + 2 * SB + SPL       ? 16u
                             : b < 2 * SA + 2 * SB + 2 * SPL   ? 1u
                             : b == 2 * SA + 2 * SB + 2 * SPL  ? 1u  // tfull
                                                               : 16u;  // tempty, scales_in
      umma::bar_init(full_a + b, count);
      umma::bar_init_fence();
    }
    if (lane == 0) {
      *abort_flag = 0;
      *wide_any = 0;
    }
    __syncwarp();
  }
  if (threadIdx.x == 0) {
    umma::prefetch_map(&amap);
    umma::prefetch_map(&bmap);
    if (KIND == kGemmGu) umma::prefetch_map(&amap2);
    // the weights do not depend on earlier kernels: their first tiles
    // stream in while those finish
    for (int u = 0; u < pre_a; ++u) issue_a(u);
  }
  if (warp == 1) umma::tmem_alloc(tmem_slot, C::TCOLS);
  // plane builders (warps 2-17): builder et takes chunk cc (16 K values) of
  // rows r0 and r0 + 64 in every K tile; their group scales, all K tiles, load
  // into registers now (they do not depend on earlier kernels)
  const int et = threadIdx.x - 64;
  // warp w covers rows {b, b + 4, b + 1, b + 5} (b = 8 (w / 2) + 2 (w % 2)):
  // their swizzled 64-byte halves of an A stage fall in both bank halves
  const int wl = et >> 5, gq = (et >> 3) & 3;
  const int r0 = 8 * (wl >> 1) + 2 * (wl & 1) + 4 * (gq & 1) + (gq >> 1), cc = et & 7;
  uint32_t sc2[kUMaxKt];  // scale of row r0 (low half) and r0 + 64 (high half) per K tile
  bool wide = false;      // a scale of this tile needs more than 8 bits
  if (warp >= 2) {
    const uint16_t* s_lo;
    const uint16_t* s_hi;
    if constexpr (KIND == kGemmGu) {
      s_lo = g.scales + (size_t)(tile * 64 + r0) * G;
      s_hi = g.scales2 + (size_t)(tile * 64 + r0) * G;
    } else {
      const int ga = row0 + r0 < g.rows ? row0 + r0 : g.rows - 1;
      const int gb = row0 + r0 + 64 < g.rows ? row0 + r0 + 64 : g.rows - 1;
      s_lo = g.scales + (size_t)ga * G;
      s_hi = g.scales + (size_t)gb * G;
    }
    const int gq = 2 * kt0 + (cc >> 2);
#pragma unroll
    for (int kt = 0; kt < kUMaxKt; ++kt) {
      const uint32_t a = kt < nkt ? s_lo[gq + 2 * kt] : 0u, b = kt < nkt ? s_hi[gq + 2 * kt] : 0u;
      sc2[kt] = a | (b << 16);
      wide |= (a | b) > 255u;
    }
  }
  if constexpr (C::NM > 3 * SN) {
    // limb-tile rows past the chunk's 3 SN are read by the MMA: zeros
    constexpr int pad = (C::NM - 3 * SN) * 128 / 16;
    for (int i = threadIdx.x; i < SB * pad; i += kUThreads)
      *reinterpret_cast<uint4*>(bstage + (i / pad) * C::B_BYTES + 3 * SN * 128 + (i % pad) * 16) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) gemm_stamp(g, 1);
  // every CTA is resident now: the next kernel may launch and run its
  // prologue; it waits (griddepcontrol.wait) for this grid to complete
  grid_dep_launch();
  auto fail = [&]() {
    *abort_flag = 1;
    atomicExch(c.err, 3);
  };
  // a second pass (scale digits 2 and 3) once the builders have seen every scale
  auto passes = [&]() -> int {
    if (!umma::bar_wait(scales_in, 0)) {
      fail();
      return 1;
    }
    return *reinterpret_cast<volatile int*>(wide_any) ? 2 : 1;
  };

  if (warp == 0) {
    if (lane == 0) {
      grid_dep_wait();
      gemm_stamp(g, 2);
      int nv = nkt;
      for (int v = 0; v < nv && !*abort_flag; ++v) {
        const int pass = v / nkt, kt = v - pass * nkt;
        const int u = pass * upp + (kt >> 1);
        if ((kt & 1) == 0 && u >= pre_a) {
          if (!umma::bar_wait(empty_a + u % SA, ((u / SA) & 1) ^ 1)) {
            fail();
            break;
          }
          issue_a(u);
        }
        const int sb = v % SB;
        if (!umma::bar_wait(empty_b + sb, ((v / SB) & 1) ^ 1)) {
          fail();
          break;
        }
        // the chunk's three limb blocks are consecutive rows (SN = SP): one box
        umma::bar_expect_tx(full_b + sb, 3 * SN * 128);
        umma::tma_load(bstage + sb * C::B_BYTES, &bmap, (kt0 + kt) * 128, g.b_sub_rows * z + n0, full_b + sb);
        // the first pass's loads are all issued: does the tile need a second?
        if (v == nkt - 1) nv = passes() * nkt;
      }
    } else {
      grid_dep_wait();
    }
  } else if (warp == 1) {
    grid_dep_wait();
    if (lane == 0) {
      int nv = nkt;
      for (int v = 0; v < nv && !*abort_flag; ++v) {
        const int pass = v / nkt, kt = v - pass * nkt;
        if (pass == 1 && kt == 0 && !umma::bar_wait(tempty, 0)) {  // the first pass's accumulators are read
          fail();
          break;
        }
        const int sb = v % SB, sp = v % SPL;
        if (!umma::bar_wait(full_b + sb, (v / SB) & 1) || !umma::bar_wait(full_p + sp, (v / SPL) & 1)) {
          fail();
          break;
        }
        umma::fence_after_sync();
        const uint32_t a0 = umma::smem_addr(planes + sp * 2 * C::PLANE), b0 = umma::smem_addr(bstage + sb * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t acc = (kt | kk) != 0;
          umma::mma_i8(tmem, umma::sw128_desc(a0 + 32 * kk), umma::sw128_desc(b0 + 32 * kk), C::IDESC, acc);
          umma::mma_i8(tmem + C::NM, umma::sw128_desc(a0 + C::PLANE + 32 * kk), umma::sw128_desc(b0 + 32 * kk),
                       C::IDESC, acc);
        }
        umma::mma_commit(empty_p + sp);
        umma::mma_commit(empty_b + sb);
        if (kt == nkt - 1) {
          umma::mma_commit(tfull);
          if (pass == 0) nv = passes() * nkt;
          if (v == nv - 1) gemm_stamp(g, 7);
        }
      }
      // all MMAs issued: this thread is free to pull the next GEMM's weights into L2
      l2_prefetch_share(g.pf);
    }
  } else {
    // ---- plane builders (warps 2-17), then the epilogue ---------------------
    {
      if (__any_sync(0xFFFFFFFFu, wide) && lane == 0) atomicOr(wide_any, 1);
      __syncwarp();
      if (lane == 0) umma::bar_arrive(scales_in);
    }
    int64_t rbp0 = 0, rbp1 = 0;  // sum_k w s of rows r0, r0 + 64 over this thread's chunks
    const int sp_e = warp & 3, q = (warp - 2) >> 2;
    const int r = 32 * sp_e + lane;  // the tile row (TMEM lane) this thread reads back
    const uint32_t lane_base = tmem + ((uint32_t)(32 * sp_e) << 16);
    int64_t acc[C::Q];
#pragma unroll
    for (int j = 0; j < C::Q; ++j) acc[j] = 0;
    int pos_m = INT_MAX;
    bool dep_done = false;
    // After the dependency wait: stage what the final epilogue reads from
    // global memory (written by kernels this one waited for) by cp.async, the
    // residual of each owned (row, sequence) item (O / down) or the sigmoid
    // table (gate/up), and fetch the positions that say which sequences take
    // part in this step.
    auto dependent_loads = [&]() {
      grid_dep_wait();
      dep_done = true;
      if constexpr (KIND == kGemmO || KIND == kGemmDown || KIND == kGemmGu)
        if (et < c.S) pos_m = c.pos0[4 * et];
      if constexpr (KIND == kGemmO || KIND == kGemmDown) {
        // items i .. i + 3 (i a multiple of 4) are 4 consecutive rows of one
        // sequence: rows_per = 64 / splits >= 8
        const int32_t* res = KIND == kGemmO ? c.hidden0 : c.post0;
        const int lsp = __ffs(splits) - 1, lrp = 6 - lsp, rows_per = 64 >> lsp, lnl = 7 - lsp, nl = 128 >> lsp;
        for (int i = 4 * et; i < nl * SN; i += 4 * (kUThreads - 64)) {
          const int local = i & (nl - 1), m = i >> lnl;
          const int row = ((local >> lrp) << 6) + split * rows_per + (local & (rows_per - 1));
          if (m < c.S) cp_async16(stg + i, res + (size_t)m * kHidden + row0 + row);
        }
      } else if constexpr (KIND == kGemmGu) {
        if ((reinterpret_cast<uintptr_t>(g.sig_lut) & 15) == 0) {
          for (int e4 = et; e4 < kSigLut / 4; e4 += kUThreads - 64) cp_async16(stg + 4 * e4, g.sig_lut + 4 * e4);
          for (int e = kSigLut / 4 * 4 + et; e < kSigLut; e += kUThreads - 64) cp_async4(stg + e, g.sig_lut + e);
        } else {
          for (int e = et; e < kSigLut; e += kUThreads - 64) cp_async4(stg + e, g.sig_lut + e);
        }
      }
      cp_async_commit();
    };
    // planes of (pass, K tile) step v into plane slot v % SPL
    auto build = [&](int v) -> bool {
      const int pass = v / nkt, kt = v - pass * nkt;
      const int u = pass * upp + (kt >> 1), sa = u % SA;
      if (!umma::bar_wait(full_a + sa, (u / SA) & 1) || !umma::bar_wait(empty_p + v % SPL, ((v / SPL) & 1) ^ 1))
        return false;
      uint32_t s2 = sc2[0];
#pragma unroll
      for (int i = 1; i < kUMaxKt; ++i) s2 = kt == i ? sc2[i] : s2;
      const uint8_t* pk = astage + sa * C::A_PK;
      const int c16 = ((kt & 1) << 2) | (cc >> 1);  // 16-byte chunk of the row's 128-byte stage line
      uint8_t* pl = planes + (v % SPL) * 2 * C::PLANE;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = r0 + 64 * h;
        const uint32_t s = h ? (s2 >> 16) : (s2 & 0xFFFFu);
        const uint2 x = *reinterpret_cast<const uint2*>(pk + row * 128 + ((c16 ^ (row & 7)) << 4) + ((cc & 1) << 3));
        uint32_t U[4];
        unpack16_biased(x, U);
        if (pass == 0) {
          const uint32_t su = U[0] + U[1] + U[2] + U[3];                  // byte sums <= 60: no carries
          const int32_t sw = (int32_t)dp4a_uu(su, 0x01010101u, 0u) - 128;  // sum of the 16 weights
          if (h)
            rbp1 += (int64_t)sw * (int32_t)s;
          else
            rbp0 += (int64_t)sw * (int32_t)s;
        }
        // chunk cc of the row: 16-byte unit cc ^ (row % 8) of its 128-byte line
        const uint32_t off = (uint32_t)row * 128u + ((uint32_t)(cc ^ (row & 7)) << 4);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint32_t d = (s >> (8 * pass + 4 * j)) & 15u;
          const uint32_t bias = (128u - 8u * d) * 0x01010101u;
          uint4 o;
          o.x = plane_word(U[0], d, bias);
          o.y = plane_word(U[1], d, bias);
          o.z = plane_word(U[2], d, bias);
          o.w = plane_word(U[3], d, bias);
          *reinterpret_cast<uint4*>(pl + j * C::PLANE + off) = o;
        }
      }
      // plane bytes written by these threads are read by the tensor cores
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        umma::bar_arrive(full_p + v % SPL);
        if ((kt & 1) || kt == nkt - 1) umma::bar_arrive(empty_a + sa);  // both tiles of the stage are built
      }
      return true;
    };
    // the accumulators of one pass: wait for its last MMAs, add T[j][i] << (8 pass + 4 j + 8 i)
    // sum_k w s of each row (the 2^23 offset of the activation limbs): the
    // eight builders of a row add their chunks (every pass-0 plane is built
    // when the last pass is read out), the read-out subtracts it.  Every
    // builder thread reaches the named barrier exactly once.
    bool rb_done = false;
    auto row_bias = [&]() -> int64_t {
      rb_done = true;
#pragma unroll
      for (int msk = 1; msk < 8; msk <<= 1) {
        rbp0 += shfl_xor_i64(rbp0, msk);
        rbp1 += shfl_xor_i64(rbp1, msk);
      }
      if (cc == 0) {
        rbs[r0] = rbp0;
        rbs[r0 + 64] = rbp1;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kUThreads - 64) : "memory");
      return rbs[r];
    };
    // partial sums to the owning CTA: owner of row r is (r % 64) / rows_per,
    // so each owner holds matching rows of both 64-row halves (gate and up);
    // splits is a power of two (1, 2, 4 or 8), so these are shifts and masks
    const int lsp = __ffs(splits) - 1;
    const int rows_per = 64 >> lsp;
    const int owner = (r & 63) >> (6 - lsp);
    const int local = (r >> 6) * rows_per + (r & (rows_per - 1));
    const int nl = 128 >> lsp;
    // red[src][m][local]: a warp's 32 rows land contiguously (conflict-free)
    int64_t* dst = red + ((size_t)split * SN + q * C::Q) * nl + local;
    const uint32_t ca = splits > 1 ? umma::cluster_map(umma::smem_addr(dst), (uint32_t)owner) : 0u;
    // the accumulators of one pass: wait for its last MMAs, add T[j][i] << (8 pass + 4 j + 8 i).
    // The last pass sends each piece of sequences to its owner as soon as it
    // is read, so the DSMEM stores (bound by the SM-to-SM network) overlap the
    // remaining TMEM reads.
    auto read_pass = [&](int pass, int npass) -> bool {
      if (!umma::bar_wait(tfull, pass)) return false;
      umma::fence_after_sync();
      if (pass == 0 && warp == 2 && lane == 0) gemm_stamp(g, 3);
      const bool last = pass + 1 == npass;
      const int64_t bias = last ? row_bias() * (1LL << 23) : 0;
      // |T| < 120 * 255 * 1024 < 2^25 (K <= 1024 per CTA), so the two digits
      // of a limb combine in int32, X_i = T[0][i] + 16 T[1][i] (< 2^30), and
      // each limb adds X_i * 2^(8 i + 8 pass) with one widening multiply-add
      // pieces of kP sequences (a divisor of Q: 2, 3 or 4)
      constexpr int kP = C::Q % 4 == 0 ? 4 : C::Q % 3 == 0 ? 3 : C::Q;
#pragma unroll
      for (int j0 = 0; j0 < C::Q; j0 += kP) {
        int32_t d[3][2][kP];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          const uint32_t ta = lane_base + (uint32_t)(i * SN + q * C::Q + j0);
          umma::tmem_ld_any<kP>(ta, d[i][0]);
          umma::tmem_ld_any<kP>(ta + C::NM, d[i][1]);
        }
        umma::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < kP; ++j) {
          int64_t a = acc[j0 + j];
#pragma unroll
          for (int i = 0; i < 3; ++i) a = mad_wide(d[i][0][j] + 16 * d[i][1][j], 1 << (8 * i + 8 * pass), a);
          acc[j0 + j] = a;
        }
        if (last) {
#pragma unroll
          for (int j = 0; j < kP; ++j) {
            const int64_t v = acc[j0 + j] - bias;
            // (the LM head's row sums overwrite plane slots: every builder
            // finished them before its MMAs, whose completion was waited for)
            if (splits == 1)
              dst[(size_t)(j0 + j) * nl] = v;
            else
              umma::cluster_st64(ca + 8 * (j0 + j) * nl, v);
          }
        }
      }
      if (!last) {
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) umma::bar_arrive(tempty);
      }
      return true;
    };
    // the first plane slots fill before the dependency wait (weights only)
    const int early = nkt < SPL ? nkt : SPL;
    int nv = nkt;
    bool ok = true;
    for (int v = 0; v < nv && ok; ++v) {
      if (v == early && !dep_done) dependent_loads();
      ok = build(v);
      const int pass = v / nkt;
      if (ok && v - pass * nkt == nkt - 1) {
        if (!dep_done) dependent_loads();
        const int npass = passes();
        nv = npass * nkt;
        ok = read_pass(pass, npass);
      }
    }
    if (!ok) fail();
    if (!dep_done) dependent_loads();
    if (!rb_done) row_bias();
    if (warp == 2 && lane == 0) gemm_stamp(g, 4);
    cp_async_wait0();
    if constexpr (KIND == kGemmO || KIND == kGemmDown || KIND == kGemmGu)
      if (et < SN) live[et] = pos_m < c.max_ctx;
  }
  __syncwarp();
  if (splits > 1)
    umma::cluster_sync();
  else
    __syncthreads();
  if (threadIdx.x == 0) gemm_stamp(g, 5);

  // final epilogue over the rows this CTA owns: work item (four consecutive
  // local rows 4 lq .. 4 lq + 3, sequence m), which are four consecutive
  // weight rows (rows_per >= 8): the split-K partial sums of each source CTA
  // are two 16-byte shared loads, outputs one 16-byte global store
  const int lsp = __ffs(splits) - 1;
  const int lrp = 6 - lsp, rows_per = 64 >> lsp, lnl = 7 - lsp, nl = 128 >> lsp;
  const int lq_bits = lnl - 2, nq = nl >> 2;  // row quads of the owned rows
  const int ft = threadIdx.x;
  auto row_of = [&](int local) {
    return ((local >> lrp) << 6) + split * rows_per + (local & (rows_per - 1));
  };
  auto sums4 = [&](int local, int m, int64_t* v) {
    v[0] = v[1] = v[2] = v[3] = 0;
    for (int src = 0; src < splits; ++src) {
      const longlong2* p = reinterpret_cast<const longlong2*>(red + ((size_t)src * SN + m) * nl + local);
      const longlong2 a = p[0], b = p[1];
      v[0] += a.x;
      v[1] += a.y;
      v[2] += b.x;
      v[3] += b.y;
    }
  };
  if (!*abort_flag) {
    if constexpr (KIND == kGemmQkv) {
      for (int i = ft; i < nq * SN; i += kUThreads) {
        const int local = 4 * (i & (nq - 1)), m = i >> lq_bits;
        if (m >= c.S) continue;
        int64_t v[4];
        sums4(local, m, v);
        *reinterpret_cast<int4*>(c.qkv_raw + (size_t)m * (kQRows + 2 * kKvRows) + row0 + row_of(local)) =
            make_int4(sat24(v[0] >> 14), sat24(v[1] >> 14), sat24(v[2] >> 14), sat24(v[3] >> 14));
      }
    } else if constexpr (KIND == kGemmO || KIND == kGemmDown) {
      // residual (staged in stg: item local + nl m) + o_proj / down output >> 2
      int32_t* __restrict__ out = KIND == kGemmO ? c.post0 : c.hidden0;
      for (int i = ft; i < nq * SN; i += kUThreads) {
        const int local = 4 * (i & (nq - 1)), m = i >> lq_bits;
        if (m >= c.S || !live[m]) continue;
        int64_t v[4];
        sums4(local, m, v);
        const int4 r = *reinterpret_cast<const int4*>(stg + m * nl + local);
        *reinterpret_cast<int4*>(out + (size_t)m * kHidden + row0 + row_of(local)) =
            make_int4(sat24((int64_t)r.x + (sat24(v[0] >> 14) >> 2)), sat24((int64_t)r.y + (sat24(v[1] >> 14) >> 2)),
                      sat24((int64_t)r.z + (sat24(v[2] >> 14) >> 2)), sat24((int64_t)r.w + (sat24(v[3] >> 14) >> 2)));
      }
    } else if constexpr (KIND == kGemmGu) {
      // local rows 0 .. rows_per - 1 are gate rows, rows_per .. are the matching up rows
      const int jq_bits = lrp - 2, njq = rows_per >> 2;
      for (int i = ft; i < njq * SN; i += kUThreads) {
        const int j = 4 * (i & (njq - 1)), m = i >> jq_bits;
        if (m >= c.S || !live[m]) continue;
        int64_t gs[4], us[4];
        sums4(j, m, gs);
        sums4(rows_per + j, m, us);
        int32_t hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int32_t gv = sat24(gs[e] >> 14), uv = sat24(us[e] >> 14);
          const int32_t gc = gv < -32768 ? -32768 : (gv > 32768 ? 32768 : gv);
          int ix = (gc + 32768 + 32) >> 6;
          ix = ix > kSigLut - 1 ? kSigLut - 1 : ix;
          const int32_t silu = sat24(((int64_t)gv * stg[ix]) >> 16);
          hv[e] = sat24(((int64_t)silu * uv) >> 12);
        }
        // four consecutive intermediate columns: one 4-byte store per limb
        const int col = tile * 64 + split * rows_per + j;
        const uint32_t u[4] = {(uint32_t)(hv[0] + (1 << 23)), (uint32_t)(hv[1] + (1 << 23)),
                               (uint32_t)(hv[2] + (1 << 23)), (uint32_t)(hv[3] + (1 << 23))};
#pragma unroll
        for (int limb = 0; limb < 3; ++limb) {
          const int sh = 8 * limb;
          *reinterpret_cast<uint32_t*>(c.bt3 + (size_t)(limb * SP + n0 + m) * kInter + col) =
              ((u[0] >> sh) & 0xFF) | (((u[1] >> sh) & 0xFF) << 8) | (((u[2] >> sh) & 0xFF) << 16) |
              (((u[3] >> sh) & 0xFF) << 24);
        }
      }
    } else {
      // LM head (no split): best (score, row) of each sequence over the tile
      ArgBestD* cand = reinterpret_cast<ArgBestD*>(bstage);  // the limb ring is free now
      constexpr int kParts = kUThreads / SN;
      for (int i = ft; i < kParts * SN; i += kUThreads) {
        const int part = i % kParts, m = i / kParts;
        int64_t bs = INT64_MIN;
        int32_t bi = INT32_MAX;
        for (int lr = part; lr < 128; lr += kParts) {
          const int row = row0 + lr;
          if (row >= g.rows) break;
          const int64_t v = red[(size_t)m * 128 + lr];
          if (v > bs) {  // rows ascend within a part: strict '>' keeps the lowest index
            bs = v;
            bi = row;
          }
        }
        cand[part * SN + m] = ArgBestD{bs, bi, 0};
      }
      __syncthreads();
      for (int m = ft; m < SN; m += kUThreads) {
        ArgBestD b = cand[m];
        for (int part = 1; part < kParts; ++part) {
          const ArgBestD o = cand[part * SN + m];
          if (o.score > b.score || (o.score == b.score && o.idx < b.idx)) b = o;
        }
        g.partial[(size_t)tile * kBatchSeqMax + n0 + m] = b;
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) gemm_stamp(g, 6);
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, C::TCOLS);
  }
}

// Limb matrix of already-normed Q12.12 vectors (the input of a vocab-shard LM
// head): acts [n][1024] -> bt rows limb * SP + m.
__global__ void __launch_bounds__(256) act_limbs_kernel(const int32_t* __restrict__ acts, uint8_t* __restrict__ bt,
                                                        int SP) {
  const int m = blockIdx.x, k = 4 * threadIdx.x;
  const int4 v = *reinterpret_cast<const int4*>(acts + (size_t)m * kHidden + k);
  const uint32_t u[4] = {(uint32_t)(v.x + (1 << 23)), (uint32_t)(v.y + (1 << 23)), (uint32_t)(v.z + (1 << 23)),
                         (uint32_t)(v.w + (1 << 23))};
#pragma unroll
  for (int limb = 0; limb < 3; ++limb) {
    const int sh = 8 * limb;
    const uint32_t word = ((u[0] >> sh) & 0xFF) | (((u[1] >> sh) & 0xFF) << 8) | (((u[2] >> sh) & 0xFF) << 16) |
                          (((u[3] >> sh) & 0xFF) << 24);
    *reinterpret_cast<uint32_t*>(bt + (size_t)(limb * SP + m) * kHidden + k) = word;
  }
}

// Best (score, row) of vector blockIdx.x over the LM-head tile partials of a
// vocabulary shard starting at row_offset; the reference's rule (highest
// score, lowest row on ties).
__global__ void shard_argmax_kernel(const ArgBestD* __restrict__ partial, int n_parts, int row_offset,
                                    int64_t* __restrict__ best_score, int64_t* __restrict__ best_row) {
  __shared__ int64_t ss[32];
  __shared__ int32_t si[32];
  const int m = blockIdx.x;
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
    best_score[m] = bs;
    best_row[m] = (int64_t)bi + row_offset;
  }
}

// Chosen next tokens of sequences 0..S-1: stored at position + 1 (from
// lm_from on) with their scores; positions advance.
__global__ void batch_commit_kernel(BatchCtx c, const int64_t* __restrict__ tokens,
                                    const int64_t* __restrict__ scores) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= c.S) return;
  const SlotState& st = c.slots[m];
  const int pos = *st.pos;
  if (pos >= st.max_ctx) return;
  if (pos + 1 >= c.lm_from[m]) {
    st.tokens[pos + 1] = (int32_t)tokens[m];
    st.scores[pos + 1] = scores[m];
  }
  *st.pos = pos + 1;
}

// Vocabulary-sharded LM head: every shard's (score, row) winner of sequence
// m sits at win[(k * 2 + 0) * stride + col0 + m] / win[(k * 2 + 1) * stride +
// col0 + m] (shards k = 0 .. n_shards - 1, as an all_gather of [2][stride]
// per rank lays them out).  The global winner follows the reference's rule
// (highest score, lowest row on ties; the order shards are visited does not
// matter), is stored at position + 1 from lm_from on, and positions advance.
__global__ void batch_commit_shards_kernel(BatchCtx c, const int64_t* __restrict__ win, int n_shards, int stride,
                                           int col0) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= c.S) return;
  int64_t bs = INT64_MIN, br = INT64_MAX;
  for (int k = 0; k < n_shards; ++k) {
    const int64_t sc = win[(size_t)(2 * k) * stride + col0 + m], row = win[(size_t)(2 * k + 1) * stride + col0 + m];
    if (sc > bs || (sc == bs && row < br)) {
      bs = sc;
      br = row;
    }
  }
  const SlotState& st = c.slots[m];
  const int pos = *st.pos;
  if (pos >= st.max_ctx) return;
  if (pos + 1 >= c.lm_from[m]) {
    st.tokens[pos + 1] = (int32_t)br;
    st.scores[pos + 1] = bs;
  }
  *st.pos = pos + 1;
}

// Reduce the LM-head partials of sequence blockIdx.x; write the argmax where
// the sequence has left its prompt, and advance its position.
__global__ void batch_argmax_kernel(BatchCtx c, const ArgBestD* __restrict__ partial, int n_parts) {
  __shared__ int64_t ss[32];
  __shared__ int32_t si[32];
  // released only after the wait (see batch_embed_kernel)
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


// ---------------------------------------------------------------------------
// Batched exact prefill.  The prompt positions of the sequences become the
// columns of batched passes, column = (sequence, position) in sequence-major
// order: 64 columns per GEMM (the batched-step GEMMs, unchanged), a block of
// up to kPfBlock columns per attention launch.  Blocks run through all layers
// in column order, so the keys and values a column attends to are in the
// cache when its attention runs: earlier positions of the same sequence were
// written by earlier blocks (every layer) or, in this block, by the q/k
// kernel that runs before the attention.  Each column computes exactly what
// a decode step at its position computes, so the K/V cache it leaves equals
// the serial one bit for bit.
//
// Attention (prefill_attn_kernel): one CTA per (KV head, query tile of up to
// 64 consecutive positions of one sequence), 128 query rows (the two heads of
// the group).  The exact LUT softmax is done in three passes over 64-key
// chunks of the cache (cp.async into a staging buffer, then re-laid out):
//   1. scores -> row maxima;
//   2. scores again -> LUT indices (kept in a u16 scratch) and exp sums;
//   3. values in 128-key chunks: sum over keys of prob * v with
//      prob = (lut[idx] << 16) / sum by the row's Barrett reciprocal, then
//      sat24(>> 16) as limbs of the o_proj input.
// q and k are signed 24-bit, split into byte limbs x = x0 + 2^8 x1 + 2^16 x2
// (x0, x1 unsigned, x2 signed), and
//   q k = sum_{a,b} 2^(8 (a + b)) qa kb.
// Both products run on the 5th-generation tensor cores (tcgen05.mma kind::i8,
// u8 / s8 per operand in the instruction descriptor, one issuing thread, the
// operands in shared memory as 128-byte-swizzled K-major tiles written by the
// threads, accumulators in TMEM read back by all 16 warps with tcgen05.ld):
//   scores: A = q limbs (M = 128 rows), B = key limbs (N = 64 keys), nine
//     limb products into five accumulators, one per shift (each below
//     3 * 128 * 255^2 in magnitude), combined in int64;
//   values: A = probability limbs (128 rows x 128 keys), B = value limbs
//     (dims x 128 keys), p (0 .. 2^16) = p0 + 2^8 p1 + 2^16 p2 with p2 in
//     {0, 1} (its three products are skipped for chunks where no p reaches
//     2^16), two N = 64 halves of the dims per chunk, folded into int64
//     after every 128-key chunk.
// The results are the integers the int64 decode kernels compute.
// ---------------------------------------------------------------------------
constexpr int kPfStride = kHeadDim + 4;   // staged int32 key row (words): 16-byte aligned rows
constexpr int kPfRows = 2 * kPfTileQ;     // query rows of a CTA: the UMMA M of the score products
constexpr int kPfThreads = 512;           // 16 warps: 4 row tiles x 4 dim quarters in the value pass
constexpr size_t kPfQlBytes = (size_t)3 * kPfRows * 128;   // q limbs: three 128-byte-swizzled K-major planes
constexpr size_t kPfKlBytes = (size_t)3 * kPfKeys * 128;   // key limbs of a chunk, same layout
constexpr size_t kPfPvBytes = (size_t)3 * kPfRows * 128 + (size_t)3 * kHeadDim * 128;  // probability + value limbs
constexpr size_t kPfOperands = kPfQlBytes + kPfKlBytes > kPfPvBytes ? kPfQlBytes + kPfKlBytes : kPfPvBytes;
constexpr size_t kPfStageBytes = (size_t)kPfKeys * kPfStride * 4;   // one chunk as staged int32
constexpr size_t kPfSmem = 1024 + kPfOperands + kPfStageBytes;       // + alignment slack
static_assert(kPfRows == 128 && kPfKeys == 64, "score MMAs are M = 128, N = 64");

// byte `l` of each of four words, packed (the limb l of four elements)
__device__ __forceinline__ uint32_t limb_word(int4 v, int l) {
  const uint32_t sel = (uint32_t)l | ((uint32_t)(l + 4) << 4);
  const uint32_t lo = __byte_perm((uint32_t)v.x, (uint32_t)v.y, sel);
  const uint32_t hi = __byte_perm((uint32_t)v.z, (uint32_t)v.w, sel);
  return __byte_perm(lo, hi, 0x5410);
}


// q (kind 0) or k (kind 1) head row -> RMSNorm (head constants) -> RoPE at
// `pos`, by one warp: lane owns elements 4 lane .. 4 lane + 3, the rotation
// partner d +- 64 sits 16 lanes away.  Same arithmetic as the decode kernels.
__device__ __forceinline__ int4 head_norm_rope(const int32_t* row, const int32_t* gamma, const int32_t* cos_tab,
                                               const int32_t* sin_tab, int pos, int lane) {
  const int4 x = *reinterpret_cast<const int4*>(row + 4 * lane);
  const int4 cs = *reinterpret_cast<const int4*>(cos_tab + (size_t)pos * kHeadDim + 4 * lane);
  const int4 sn = *reinterpret_cast<const int4*>(sin_tab + (size_t)pos * kHeadDim + 4 * lane);
  const int4 gm = *reinterpret_cast<const int4*>(gamma + 4 * lane);
  const int32_t xs[4] = {x.x, x.y, x.z, x.w}, cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
  const int32_t gv[4] = {gm.x, gm.y, gm.z, gm.w};
  int64_t ss = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = mad_wide(xs[e], xs[e], ss);
  ss = warp_sum_i64(ss);
  const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
  int32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int32_t n = norm_apply(xs[e], inv, gv[e], kHeadNorm);
    const int32_t partner = __shfl_xor_sync(0xFFFFFFFFu, n, 16);
    const int64_t rot = lane < 16 ? -(int64_t)partner : (int64_t)partner;
    o[e] = sat24(((int64_t)n * cv[e] + rot * sv[e]) >> 15);
  }
  return make_int4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------
// Cluster attention for small batches and long contexts: the R CTAs of a
// thread-block cluster (R = gridDim.x: 8, or 16 for batches of up to four
// sequences) share one (KV head, sequence) pair, each streaming 1/R of the
// context through a ring of 32-key chunks (K, then V).
// The exact two-pass LUT softmax is resolved over DSMEM: every rank
// publishes its row maxima, then its exp sums, and reads the others' after a
// cluster barrier; the probability table uses a Barrett reciprocal of the
// total (R = floor((2^64 - 1) / sum), q = mulhi(n, R) is at most one below
// floor(n / sum) for n < 2^37 and a remainder test makes it exact); rank 0
// adds the ranks' int64 value sums and writes the o_proj limbs.  No
// global scratch, no atomics, no single-CTA tail over the whole context.
// ---------------------------------------------------------------------------
constexpr int kClKprMax = 4096;  // keys per rank the score buffer holds

// STAGE = false: the batched decode step (sequence m = blockIdx.z of c; q/k/v
// raw from the q/k/v GEMM, normed, roped and appended here; output the o_proj
// limbs).  STAGE = true: one slot of the per-stage batch-1 path (q heads
// already normed and roped in st.qrope, the new K/V row already in the cache;
// output st.attn).
template <bool STAGE, int RING>
__device__ __forceinline__ void attn_cl_body(const BatchCtx& c, const SlotState& st, int* err, int layer,
                                             const int32_t* __restrict__ g_q, const int32_t* __restrict__ g_k,
                                             const int32_t* __restrict__ cos_tab, const int32_t* __restrict__ sin_tab,
                                             const int32_t* __restrict__ exp_lut, int kpr_cap) {
  extern __shared__ __align__(128) uint8_t cl_smem[];
  int32_t* ring = reinterpret_cast<int32_t*>(cl_smem);                            // [2][32][128]
  int64_t* sc = reinterpret_cast<int64_t*>(cl_smem + RING * kAttnChunkBytes);  // [2][kpr_cap]
  __shared__ __align__(16) int32_t hv[4][kHeadDim];  // roped q0, q1, k; raw v of the new position
  __shared__ uint32_t probtab[2][kExpLut];
  __shared__ int64_t red[2][8];
  __shared__ int64_t xmax[2], xsum[2];       // published to the cluster
  __shared__ int64_t part[2][kHeadDim];      // this rank's value sums, published to the cluster
  __shared__ uint64_t bars[RING];
  const int rank = blockIdx.x, nranks = gridDim.x, kv = blockIdx.y, m = STAGE ? 0 : blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  // every rank reaches every cluster barrier below: no early return.  The
  // cached K/V rows and the position come from earlier steps, so the first
  // chunks load before the wait for this step's q/k/v projections.
  const int pos = STAGE ? *st.pos : c.pos0[4 * m];
  const bool live = pos < (STAGE ? st.max_ctx : c.max_ctx);
  const int ctx = live ? pos + 1 : 0;
  const int kpr = ((ctx + nranks - 1) / nranks + kAttnChunk - 1) / kAttnChunk * kAttnChunk;
  const int k0 = rank * kpr;
  const int k1 = k0 + kpr < ctx ? k0 + kpr : ctx;  // this rank's keys [k0, k1)
  const int nloc = k1 > k0 ? k1 - k0 : 0;
  const KvView kvv = STAGE ? st.kv : c.slots[m].kv;
  const int nk = (nloc + kAttnChunk - 1) / kAttnChunk, total = 2 * nk;
  const int kend = k1 < pos ? k1 : pos;  // cached keys of the range (the new position comes from shared memory)
  auto issue = [&](int i) {
    const int kind = i < nk ? 0 : 1, j = i < nk ? i : i - nk;
    const int p0 = k0 + j * kAttnChunk;
    int n = kend - p0;
    n = n < 0 ? 0 : (n > kAttnChunk ? kAttnChunk : n);
    uint64_t* b = bars + i % RING;
    umma::bar_expect_tx(b, (uint32_t)n * kHeadDim * 4);
    if (n > 0)
      bulk_load(ring + (i % RING) * kAttnChunk * kHeadDim, kvv.at(layer, kind, kv, p0), (uint32_t)n * kHeadDim * 4,
                b);
  };
  if (t == 0) {
    for (int s = 0; s < RING; ++s) umma::bar_init(bars + s, 1);
    umma::bar_init_fence();
    for (int i = 0; i < total && i < RING; ++i) issue(i);
  }
  grid_dep_wait();
  grid_dep_launch();
  if (STAGE && live) {
    // q heads 2 kv, 2 kv + 1 as roped by the q/k/v stage, the new K/V row from the cache
    if (warp < 2)
      reinterpret_cast<int4*>(hv[warp])[lane] = reinterpret_cast<const int4*>(st.qrope + (2 * kv + warp) * kHeadDim)[lane];
    else if (warp < 4)
      reinterpret_cast<int4*>(hv[warp])[lane] = reinterpret_cast<const int4*>(kvv.at(layer, warp - 2, kv, pos))[lane];
  } else if (live) {
    const int32_t* raw = c.qkv_raw + (size_t)m * (kQRows + 2 * kKvRows);
    const bool owner = pos >= k0 && pos < k1;  // the rank whose range holds the new position appends it
    if (warp < 2) {
      reinterpret_cast<int4*>(hv[warp])[lane] =
          head_norm_rope(raw + (2 * kv + warp) * kHeadDim, g_q, cos_tab, sin_tab, pos, lane);
    } else if (warp == 2) {
      const int4 k4 = head_norm_rope(raw + kQRows + kv * kHeadDim, g_k, cos_tab, sin_tab, pos, lane);
      reinterpret_cast<int4*>(hv[2])[lane] = k4;
      if (owner) {
        reinterpret_cast<int4*>(kvv.at(layer, 0, kv, pos))[lane] = k4;
        kpl_put4(kvv, layer, kv, pos, 4 * lane, k4);
      }
    } else if (warp == 3) {
      const int4 v4 = reinterpret_cast<const int4*>(raw + kQRows + kKvRows + kv * kHeadDim)[lane];
      reinterpret_cast<int4*>(hv[3])[lane] = v4;
      if (owner) {
        reinterpret_cast<int4*>(kvv.at(layer, 1, kv, pos))[lane] = v4;
        vpl_put4(kvv, layer, kv, pos, 4 * lane, v4);
      }
    }
  }
  __syncthreads();
  bool ok = true;
  // scores of the range: 32 keys per chunk, 4 per warp, 8 lanes per key
  int64_t mx0 = INT64_MIN, mx1 = INT64_MIN;
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
    for (int i = 0; i < nk; ++i) {
      if (!umma::bar_wait(bars + i % RING, (i / RING) & 1)) ok = false;
      const int lp = i * kAttnChunk + warp * 4 + quad, p = k0 + lp;
      const int32_t* krow = p == pos ? hv[2] : ring + ((i % RING) * kAttnChunk + warp * 4 + quad) * kHeadDim;
      int64_t s0 = 0, s1 = 0;
      if (p < k1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 k4 = *reinterpret_cast<const int4*>(krow + 4 * (sub + 8 * j));
          const int32_t kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            s0 = mad_wide(q0[4 * j + e], kk[e], s0);
            s1 = mad_wide(q1[4 * j + e], kk[e], s1);
          }
        }
      }
#pragma unroll
      for (int msk = 1; msk < 8; msk <<= 1) {
        s0 += shfl_xor_i64(s0, msk);
        s1 += shfl_xor_i64(s1, msk);
      }
      if (p < k1) {
        const int64_t v0 = scale_score(s0, kScoreScale), v1 = scale_score(s1, kScoreScale);
        if (sub == 0) {
          sc[lp] = v0;
          sc[kpr_cap + lp] = v1;
        }
        mx0 = v0 > mx0 ? v0 : mx0;
        mx1 = v1 > mx1 ? v1 : mx1;
      }
      __syncthreads();  // slot i % 2 is free again
      if (t == 0 && i + RING < total) issue(i + RING);
    }
  }
#pragma unroll
  for (int msk = 8; msk < 32; msk <<= 1) {
    const int64_t o0 = shfl_xor_i64(mx0, msk), o1 = shfl_xor_i64(mx1, msk);
    mx0 = o0 > mx0 ? o0 : mx0;
    mx1 = o1 > mx1 ? o1 : mx1;
  }
  if (lane == 0) {
    red[0][warp] = mx0;
    red[1][warp] = mx1;
  }
  __syncthreads();
  if (t < 2) {
    int64_t b = red[t][0];
    for (int w = 1; w < 8; ++w) b = red[t][w] > b ? red[t][w] : b;
    xmax[t] = b;
  }
  umma::cluster_sync();  // every rank's maxima are published
  // lane r of warp 0 reads rank r's (one round trip for all ranks), a warp
  // reduction combines them
  if (warp == 0) {
    int64_t o0 = INT64_MIN, o1 = INT64_MIN;
    if (lane < nranks) {
      o0 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xmax[0]), (uint32_t)lane));
      o1 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xmax[1]), (uint32_t)lane));
    }
#pragma unroll
    for (int msk = 1; msk < 32; msk <<= 1) {
      const int64_t a = shfl_xor_i64(o0, msk), b = shfl_xor_i64(o1, msk);
      o0 = a > o0 ? a : o0;
      o1 = b > o1 ? b : o1;
    }
    if (lane == 0) {
      red[0][0] = o0;
      red[1][0] = o1;
    }
  }
  __syncthreads();
  mx0 = red[0][0];
  mx1 = red[1][0];
  // LUT indices and exp sums of the range
  int64_t sum0 = 0, sum1 = 0;
  for (int lp = t; lp < nloc; lp += blockDim.x) {
    const int i0 = lut_index(mx0, sc[lp]), i1 = lut_index(mx1, sc[kpr_cap + lp]);
    sc[lp] = i0;
    sc[kpr_cap + lp] = i1;
    sum0 += exp_lut[i0];
    sum1 += exp_lut[i1];
  }
  sum0 = warp_sum_i64(sum0);
  sum1 = warp_sum_i64(sum1);
  __syncthreads();  // red reused
  if (lane == 0) {
    red[0][warp] = sum0;
    red[1][warp] = sum1;
  }
  __syncthreads();
  if (t < 2) {
    int64_t b = 0;
    for (int w = 0; w < 8; ++w) b += red[t][w];
    xsum[t] = b;
  }
  umma::cluster_sync();  // every rank's sums are published
  if (warp == 0) {
    int64_t o0 = 0, o1 = 0;
    if (lane < nranks) {
      o0 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xsum[0]), (uint32_t)lane));
      o1 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xsum[1]), (uint32_t)lane));
    }
    o0 = warp_sum_i64(o0);
    o1 = warp_sum_i64(o1);
    if (lane == 0) {
      red[0][1] = o0;
      red[1][1] = o1;
    }
  }
  __syncthreads();
  sum0 = red[0][1];
  sum1 = red[1][1];
  if (live) {
    const uint64_t d0 = (uint64_t)sum0, d1 = (uint64_t)sum1, r0 = ~0ULL / d0, r1 = ~0ULL / d1;
    for (int i = t; i < 2 * kExpLut; i += blockDim.x) {
      const int h = i >= kExpLut, e = i - h * kExpLut;
      probtab[h][e] = barrett_div((uint64_t)exp_lut[e] << 16, h ? d1 : d0, h ? r1 : r0);
    }
  }
  __syncthreads();
  for (int lp = t; lp < nloc; lp += blockDim.x) {
    sc[lp] = probtab[0][(int)sc[lp]];
    sc[kpr_cap + lp] = probtab[1][(int)sc[kpr_cap + lp]];
  }
  __syncthreads();
  // values of the range: thread (warp, lane) accumulates dims 4 lane .. +3 of
  // the chunk's keys warp, warp + 8, warp + 16, warp + 24 for both heads
  int64_t a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
  for (int i = nk; i < total; ++i) {
    if (!umma::bar_wait(bars + i % RING, (i / RING) & 1)) ok = false;
    const int base = (i - nk) * kAttnChunk;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int lp = base + warp + 8 * u, p = k0 + lp;
      if (p < k1) {
        const int32_t* vrow = p == pos ? hv[3] : ring + ((i % RING) * kAttnChunk + warp + 8 * u) * kHeadDim;
        const int4 v4 = *reinterpret_cast<const int4*>(vrow + 4 * lane);
        const int32_t p0 = (int32_t)sc[lp], p1 = (int32_t)sc[kpr_cap + lp];
        const int32_t vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a0[e] = mad_wide(p0, vv[e], a0[e]);
          a1[e] = mad_wide(p1, vv[e], a1[e]);
        }
      }
    }
    __syncthreads();
    if (t == 0 && i + RING < total) issue(i + RING);
  }
  if (!ok) atomicExch(err, 4);
  // cross-warp sums through the idle ring [8][2][128], then published
  int64_t* wpart = reinterpret_cast<int64_t*>(cl_smem);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wpart[(warp * 2 + 0) * kHeadDim + 4 * lane + e] = a0[e];
    wpart[(warp * 2 + 1) * kHeadDim + 4 * lane + e] = a1[e];
  }
  __syncthreads();
  {
    const int h = t >> 7, d = t & (kHeadDim - 1);
    int64_t acc = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc += wpart[(w * 2 + h) * kHeadDim + d];
    part[h][d] = acc;
  }
  umma::cluster_sync();  // every rank's value sums are published
  {
    // rank r finishes outputs [r per, (r + 1) per) of the 2 x 128: thread
    // (source rank src, output j) fetches one partial sum (one round trip),
    // the sums over the sources meet in the idle ring
    const int per = 2 * kHeadDim / nranks, j = t % per, src = t / per, o = rank * per + j;
    int64_t* gsum = wpart;  // [nranks][per]
    gsum[src * per + j] =
        umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&part[o >> 7][o & (kHeadDim - 1)]), (uint32_t)src));
    __syncthreads();
    if (t < per && live) {
      int64_t acc = 0;
      for (int r = 0; r < nranks; ++r) acc += gsum[r * per + t];
      const int oo = rank * per + t, h = oo >> 7, d = oo & (kHeadDim - 1);
      if constexpr (STAGE)
        st.attn[(2 * kv + h) * kHeadDim + d] = sat24(acc >> 16);
      else
        write_limbs(c.bt2, c.SP, 2 * kHidden, m, (2 * kv + h) * kHeadDim + d, sat24(acc >> 16));
    }
  }
  umma::cluster_sync();  // no rank leaves while another still reads its shared memory
}

__global__ void __launch_bounds__(256) batch_attn_cl_kernel(BatchCtx c, int layer, const int32_t* __restrict__ g_q,
                                                            const int32_t* __restrict__ g_k,
                                                            const int32_t* __restrict__ cos_tab,
                                                            const int32_t* __restrict__ sin_tab,
                                                            const int32_t* __restrict__ exp_lut, int kpr_cap) {
  attn_cl_body<false, kAttnRing>(c, SlotState{}, c.err, layer, g_q, g_k, cos_tab, sin_tab, exp_lut, kpr_cap);
}

// Cluster attention with tensor-core products (batched decode, models that
// hold the K/V byte planes): the R CTAs of a cluster share one (KV head,
// sequence) pair; rank r takes positions [r kpr, (r + 1) kpr) with kpr a
// multiple of 128, scores and values them as batch_attn_kernel does (key and
// value planes through a two-slot ring into M128 x N16 x K128 kind::i8
// products, D and E in TMEM), and the exact softmax crosses the cluster as in
// attn_cl_body: row maxima, then exp sums, then the int64 value sums of each
// rank meet over DSMEM.  The rank whose range holds the current position
// appends its K/V and scores it (and adds its value) on the CUDA cores.
// Ranks take at most kClTcKprMax positions.
constexpr int kClTcKprMax = 2048;
__global__ void __launch_bounds__(256) batch_attn_cl_tc_kernel(BatchCtx c, int layer, const int32_t* __restrict__ g_q,
                                                               const int32_t* __restrict__ g_k,
                                                               const int32_t* __restrict__ cos_tab,
                                                               const int32_t* __restrict__ sin_tab,
                                                               const int32_t* __restrict__ exp_lut, int kpr_cap) {
  extern __shared__ uint8_t cl_raw[];
  const uint32_t raw_addr = umma::smem_addr(cl_raw);
  uint8_t* sbase = cl_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* slots = sbase;                                   // [2][16 KB]
  uint8_t* qb = sbase + 2 * kTcSlot;                        // [16][128] query bytes
  int64_t* sc = reinterpret_cast<int64_t*>(qb + 16 * 128);  // [2][kpr_cap]; later the probability bytes
  uint8_t* pb = reinterpret_cast<uint8_t*>(sc);
  __shared__ __align__(16) int32_t hv[4][kHeadDim];
  __shared__ uint32_t probtab[2][kExpLut];
  __shared__ int64_t red[2][8];
  __shared__ int64_t xmax[2], xsum[2];   // published to the cluster
  __shared__ uint64_t full[2], empty[2], dfull, dempty, vdone;
  __shared__ uint32_t tmem_slot;
  __shared__ uint32_t ppos[2];
  const int rank = blockIdx.x, nranks = gridDim.x, kv = blockIdx.y, m = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  // every rank reaches every cluster barrier below: no early return
  const int pos = c.pos0[4 * m];
  const KvView kvv = c.slots[m].kv;
  const bool live = pos < c.max_ctx && kvv.kpl && kvv.vpl;
  if (pos < c.max_ctx && !live && t == 0 && rank == 0) atomicExch(c.err, 4);
  const int ctx = live ? pos + 1 : 0;
  const int kpr = ((ctx + nranks - 1) / nranks + kTcKeys - 1) / kTcKeys * kTcKeys;
  const int k0 = rank * kpr;
  const int k1 = k0 + kpr < ctx ? k0 + kpr : ctx;  // this rank's positions [k0, k1)
  const int nloc = k1 > k0 ? k1 - k0 : 0;
  const int kend = k1 < pos ? k1 : pos;             // cached positions of the range
  const int ncached = kend > k0 ? kend - k0 : 0;
  const bool owner = live && pos >= k0 && pos < k1;
  const int nch = (ncached + kTcKeys - 1) / kTcKeys;
  const int nkp = 3 * nch, total = 2 * nkp;
  auto issue = [&](int i) {
    uint64_t* b = full + (i & 1);
    uint8_t* dst = slots + (i & 1) * kTcSlot;
    const int j = i < nkp ? i : i - nkp, ch = j / 3, a = j - 3 * ch, p0 = k0 + ch * kTcKeys;
    if (i < nkp) {
      const int n0 = kend - p0 < kKvPage ? kend - p0 : kKvPage;  // >= 1
      int n1 = kend - p0 - kKvPage;
      n1 = n1 < 0 ? 0 : (n1 > kKvPage ? kKvPage : n1);
      umma::bar_expect_tx(b, (uint32_t)(n0 + n1) * 128u);
      bulk_load(dst, kvv.kplane(layer, kv, p0) + a * kKplPlane, (uint32_t)n0 * 128u, b);
      if (n1 > 0)
        bulk_load(dst + kKplPlane, kvv.kplane(layer, kv, p0 + kKvPage) + a * kKplPlane, (uint32_t)n1 * 128u, b);
    } else {
      const bool two = p0 + kKvPage < kend;
      umma::bar_expect_tx(b, (two ? 2u : 1u) * kKplPlane);
      bulk_load(dst, kvv.vplane(layer, kv, p0) + a * kKplPlane, kKplPlane, b);
      if (two) bulk_load(dst + kKplPlane, kvv.vplane(layer, kv, p0 + kKvPage) + a * kKplPlane, kKplPlane, b);
    }
  };
  if (t == 0) {
    umma::bar_init(full, 1);
    umma::bar_init(full + 1, 1);
    umma::bar_init(empty, 1);
    umma::bar_init(empty + 1, 1);
    umma::bar_init(&dfull, 1);
    umma::bar_init(&dempty, 4);
    umma::bar_init(&vdone, 1);
    umma::bar_init_fence();
    for (int i = 0; i < total && i < 2; ++i) issue(i);
  }
  if (warp == 1) umma::tmem_alloc(&tmem_slot, kTcCols);
  for (int e = t; e < kExpLut; e += blockDim.x) probtab[0][e] = (uint32_t)exp_lut[e];
  grid_dep_wait();
  grid_dep_launch();
  if (live) {
    const int32_t* raw = c.qkv_raw + (size_t)m * (kQRows + 2 * kKvRows);
    if (warp < 2) {
      reinterpret_cast<int4*>(hv[warp])[lane] =
          head_norm_rope(raw + (2 * kv + warp) * kHeadDim, g_q, cos_tab, sin_tab, pos, lane);
    } else if (warp == 2) {
      const int4 k4 = head_norm_rope(raw + kQRows + kv * kHeadDim, g_k, cos_tab, sin_tab, pos, lane);
      reinterpret_cast<int4*>(hv[2])[lane] = k4;
      if (owner) {
        reinterpret_cast<int4*>(kvv.at(layer, 0, kv, pos))[lane] = k4;
        kpl_put4(kvv, layer, kv, pos, 4 * lane, k4);
      }
    } else if (warp == 3) {
      const int4 v4 = reinterpret_cast<const int4*>(raw + kQRows + kKvRows + kv * kHeadDim)[lane];
      reinterpret_cast<int4*>(hv[3])[lane] = v4;
      if (owner) {
        reinterpret_cast<int4*>(kvv.at(layer, 1, kv, pos))[lane] = v4;
        vpl_put4(kvv, layer, kv, pos, 4 * lane, v4);
      }
    }
  }
  __syncthreads();
  {
    const int r = t >> 4, d0 = 8 * (t & 15);
    uint32_t w0 = 0, w1 = 0;
    if (r < 6) {
      const int h = r >= 3, b = r - 3 * h;
      const int4 lo = *reinterpret_cast<const int4*>(&hv[h][d0]);
      const int4 hi = *reinterpret_cast<const int4*>(&hv[h][d0 + 4]);
      const int4 bl = make_int4(lo.x + (1 << 23), lo.y + (1 << 23), lo.z + (1 << 23), lo.w + (1 << 23));
      const int4 bh = make_int4(hi.x + (1 << 23), hi.y + (1 << 23), hi.z + (1 << 23), hi.w + (1 << 23));
      w0 = byte_plane_word(bl, b);
      w1 = byte_plane_word(bh, b);
    } else if (r == 6) {
      w0 = w1 = 0x01010101u;
    }
    *reinterpret_cast<uint2*>(qb + kpl_off(r, d0)) = make_uint2(w0, w1);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  bool ok = true;
  int64_t mx0 = INT64_MIN, mx1 = INT64_MIN;
  // the current position's scores (warp 5 of the owner); sc is indexed by p - k0
  if (warp == 5 && owner) {
    const int4 k4 = *reinterpret_cast<const int4*>(&hv[2][4 * lane]);
    const int4 qa = *reinterpret_cast<const int4*>(&hv[0][4 * lane]);
    const int4 qc = *reinterpret_cast<const int4*>(&hv[1][4 * lane]);
    int64_t s0 = 0, s1 = 0;
    s0 = mad_wide(qa.x, k4.x, s0);
    s0 = mad_wide(qa.y, k4.y, s0);
    s0 = mad_wide(qa.z, k4.z, s0);
    s0 = mad_wide(qa.w, k4.w, s0);
    s1 = mad_wide(qc.x, k4.x, s1);
    s1 = mad_wide(qc.y, k4.y, s1);
    s1 = mad_wide(qc.z, k4.z, s1);
    s1 = mad_wide(qc.w, k4.w, s1);
    s0 = warp_sum_i64(s0);
    s1 = warp_sum_i64(s1);
    if (lane == 0) {
      mx0 = scale_score(s0, kScoreScale);
      mx1 = scale_score(s1, kScoreScale);
      sc[pos - k0] = mx0;
      sc[kpr_cap + pos - k0] = mx1;
    }
  }
  if (t == 128) {
    const uint64_t qdesc = umma::sw128_desc(umma::smem_addr(qb));
    for (int i = 0; i < nkp && ok; ++i) {
      const int ch = i / 3, a = i - 3 * ch;
      if (a == 0 && ch > 0 && !umma::bar_wait(&dempty, (ch - 1) & 1)) ok = false;
      if (ok && !umma::bar_wait(full + (i & 1), (i >> 1) & 1)) ok = false;
      if (!ok) break;
      umma::fence_after_sync();
      const uint64_t kdesc = umma::sw128_desc(umma::smem_addr(slots + (i & 1) * kTcSlot));
      const uint32_t idesc = umma::i8_idesc_ab(kTcKeys, 16, a == 2, false);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma::mma_i8(tmem + 16u * a, kdesc + (uint64_t)(2 * kk), qdesc + (uint64_t)(2 * kk), idesc, kk > 0);
      umma::mma_commit(empty + (i & 1));
      if (a == 2) umma::mma_commit(&dfull);
      if (i + 2 < total) {
        if (!umma::bar_wait(empty + (i & 1), (i >> 1) & 1)) {
          ok = false;
          break;
        }
        issue(i + 2);
      }
    }
  }
  for (int ch = 0; ch < nch && warp < 4; ++ch) {
    if (!__all_sync(0xFFFFFFFFu, umma::bar_wait(&dfull, ch & 1))) {
      ok = false;
      break;
    }
    umma::fence_after_sync();
    int32_t d[3][8];
    const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16);
#pragma unroll
    for (int a = 0; a < 3; ++a) umma::tmem_ld<8>(lb + 16u * a, d[a]);
    umma::tmem_ld_wait();
    umma::fence_before_sync();
    __syncwarp();
    if (lane == 0) umma::bar_arrive(&dempty);
    const int lk = ch * kTcKeys + 32 * warp + lane;  // local index
    if (lk < ncached) {
      int64_t s0 = 0, s1 = 0;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        const int64_t bias = (int64_t)d[a][6] << 23;
        const int64_t t0 = (int64_t)d[a][0] + ((int64_t)d[a][1] << 8) + ((int64_t)d[a][2] << 16) - bias;
        const int64_t t1 = (int64_t)d[a][3] + ((int64_t)d[a][4] << 8) + ((int64_t)d[a][5] << 16) - bias;
        s0 += t0 << (8 * a);
        s1 += t1 << (8 * a);
      }
      const int64_t v0 = scale_score(s0, kScoreScale), v1 = scale_score(s1, kScoreScale);
      sc[lk] = v0;
      sc[kpr_cap + lk] = v1;
      mx0 = v0 > mx0 ? v0 : mx0;
      mx1 = v1 > mx1 ? v1 : mx1;
    }
  }
  // maxima: block, then cluster
#pragma unroll
  for (int msk = 1; msk < 32; msk <<= 1) {
    const int64_t o0 = shfl_xor_i64(mx0, msk), o1 = shfl_xor_i64(mx1, msk);
    mx0 = o0 > mx0 ? o0 : mx0;
    mx1 = o1 > mx1 ? o1 : mx1;
  }
  if (lane == 0) {
    red[0][warp] = mx0;
    red[1][warp] = mx1;
  }
  __syncthreads();
  if (t < 2) {
    int64_t b = red[t][0];
    for (int w = 1; w < 8; ++w) b = red[t][w] > b ? red[t][w] : b;
    xmax[t] = b;
  }
  umma::cluster_sync();  // every rank's maxima are published
  if (warp == 0) {
    int64_t o0 = INT64_MIN, o1 = INT64_MIN;
    if (lane < nranks) {
      o0 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xmax[0]), (uint32_t)lane));
      o1 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xmax[1]), (uint32_t)lane));
    }
#pragma unroll
    for (int msk = 1; msk < 32; msk <<= 1) {
      const int64_t a = shfl_xor_i64(o0, msk), b = shfl_xor_i64(o1, msk);
      o0 = a > o0 ? a : o0;
      o1 = b > o1 ? b : o1;
    }
    if (lane == 0) {
      red[0][0] = o0;
      red[1][0] = o1;
    }
  }
  __syncthreads();
  mx0 = red[0][0];
  mx1 = red[1][0];
  // LUT indices and exp sums of the range
  int64_t sum0 = 0, sum1 = 0;
  for (int lp = t; lp < nloc; lp += blockDim.x) {
    const int i0 = lut_index(mx0, sc[lp]), i1 = lut_index(mx1, sc[kpr_cap + lp]);
    sc[lp] = i0;
    sc[kpr_cap + lp] = i1;
    sum0 += probtab[0][i0];
    sum1 += probtab[0][i1];
  }
  sum0 = warp_sum_i64(sum0);
  sum1 = warp_sum_i64(sum1);
  __syncthreads();  // red reused
  if (lane == 0) {
    red[0][warp] = sum0;
    red[1][warp] = sum1;
  }
  __syncthreads();
  if (t < 2) {
    int64_t b = 0;
    for (int w = 0; w < 8; ++w) b += red[t][w];
    xsum[t] = b;
  }
  umma::cluster_sync();  // every rank's sums are published
  if (warp == 0) {
    int64_t o0 = 0, o1 = 0;
    if (lane < nranks) {
      o0 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xsum[0]), (uint32_t)lane));
      o1 = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(&xsum[1]), (uint32_t)lane));
    }
    o0 = warp_sum_i64(o0);
    o1 = warp_sum_i64(o1);
    if (lane == 0) {
      red[0][1] = o0;
      red[1][1] = o1;
    }
  }
  __syncthreads();
  sum0 = red[0][1];
  sum1 = red[1][1];
  if (live) {
    // warps 4-7 build head 1's table from the LUT in probtab[0]; warps 0-3
    // compute head 0's in registers and overwrite the LUT after the barrier
    const int h = t >> 7, e0 = t & 127;
    const uint64_t dd = (uint64_t)(h ? sum1 : sum0), rc = ~0ULL / dd;
    uint32_t p0[3] = {0, 0, 0};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int e = e0 + 128 * k;
      if (e < kExpLut) {
        const uint32_t v = barrett_div((uint64_t)probtab[0][e] << 16, dd, rc);
        if (h)
          probtab[1][e] = v;
        else
          p0[k] = v;
      }
    }
    __syncthreads();
    if (h == 0) {
#pragma unroll
      for (int k = 0; k < 3; ++k)
        if (e0 + 128 * k < kExpLut) probtab[0][e0 + 128 * k] = p0[k];
    }
  } else {
    __syncthreads();
  }
  __syncthreads();
  // probabilities of the range into registers (nloc <= kClTcKprMax: 8 per
  // thread), then the index array becomes the probability bytes (as
  // batch_attn_kernel)
  uint32_t pr[kClTcKprMax / 256][2];
#pragma unroll
  for (int j = 0; j < kClTcKprMax / 256; ++j) {
    const int lp = t + 256 * j;
    pr[j][0] = pr[j][1] = 0;
    if (lp < nloc) {
      pr[j][0] = probtab[0][(int)sc[lp]];
      pr[j][1] = probtab[1][(int)sc[kpr_cap + lp]];
      if (owner && lp == pos - k0) {
        ppos[0] = pr[j][0];
        ppos[1] = pr[j][1];
      }
    }
  }
  __syncthreads();
  for (int i = t; i < nch * 128; i += blockDim.x) reinterpret_cast<uint4*>(pb)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kClTcKprMax / 256; ++j) {
    const int lp = t + 256 * j;
    if (lp < ncached) {
      uint8_t* tile = pb + (lp >> 7) * 2048;
      const int k = lp & 127;
#pragma unroll
      for (int r = 0; r < 6; ++r) {
        const uint32_t v = pr[j][r >= 3] >> (8 * (r % 3));
        if (v & 0xFFu) tile[r * 128 + (((k >> 4) ^ (r & 7)) << 4) + (k & 15)] = (uint8_t)v;
      }
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  if (t == 128) {
    const uint64_t pdesc = umma::sw128_desc(umma::smem_addr(pb));
    for (int j = 0; j < nkp && ok; ++j) {
      const int i = nkp + j, ch = j / 3, a = j - 3 * ch;
      if (!umma::bar_wait(full + (i & 1), (i >> 1) & 1)) {
        ok = false;
        break;
      }
      umma::fence_after_sync();
      const uint32_t sa = umma::smem_addr(slots + (i & 1) * kTcSlot);
      const uint32_t idesc = umma::i8_idesc_ab(kTcKeys, 16, a == 2, false);
      const bool two = k0 + ch * kTcKeys + kKvPage < kend;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (kk >= 2 && !two) break;
        const uint64_t vdesc = sw64_desc(sa + (kk >> 1) * kKplPlane) + (uint64_t)(2 * (kk & 1));
        const uint64_t bdesc = pdesc + (uint64_t)((ch * 2048 + 32 * kk) >> 4);
        umma::mma_i8(tmem + kTcVal + 16u * a, vdesc, bdesc, idesc, (ch | kk) != 0);
      }
      umma::mma_commit(empty + (i & 1));
      if (i + 2 < total) {
        if (!umma::bar_wait(empty + (i & 1), (i >> 1) & 1)) {
          ok = false;
          break;
        }
        issue(i + 2);
      }
    }
    umma::mma_commit(&vdone);
  }
  // this rank's value sums (warps 0-3: dims 32 w .. +31), published from
  // the ring, idle once the value MMAs are done
  int64_t* part = reinterpret_cast<int64_t*>(slots);         // [2][128]
  int64_t* gsum = reinterpret_cast<int64_t*>(slots) + 256;   // [nranks][per]
  if (warp < 4) {
    const int d = 32 * warp + lane;
    int64_t o0 = 0, o1 = 0;
    const bool got = __all_sync(0xFFFFFFFFu, umma::bar_wait(&vdone, 0));
    if (!got) ok = false;
    umma::fence_after_sync();
    if (nch > 0 && got) {
      int32_t e[3][8];
      const uint32_t lb = tmem + ((uint32_t)(32 * warp) << 16) + kTcVal;
#pragma unroll
      for (int a = 0; a < 3; ++a) umma::tmem_ld<8>(lb + 16u * a, e[a]);
      umma::tmem_ld_wait();
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        o0 += ((int64_t)e[a][0] + ((int64_t)e[a][1] << 8) + ((int64_t)e[a][2] << 16)) << (8 * a);
        o1 += ((int64_t)e[a][3] + ((int64_t)e[a][4] << 8) + ((int64_t)e[a][5] << 16)) << (8 * a);
      }
    }
    if (owner) {
      o0 += (int64_t)ppos[0] * hv[3][d];
      o1 += (int64_t)ppos[1] * hv[3][d];
    }
    part[d] = o0;
    part[kHeadDim + d] = o1;
  }
  if (!ok) atomicExch(c.err, 4);
  umma::fence_before_sync();
  umma::cluster_sync();  // every rank's value sums are published
  {
    // rank r finishes outputs [r per, (r + 1) per) of the 2 x 128 (any
    // cluster size): one DSMEM load per (source rank, output)
    const int per = (2 * kHeadDim + nranks - 1) / nranks;
    for (int i = t; i < nranks * per; i += blockDim.x) {
      const int src = i / per, o = rank * per + (i - src * per);
      if (o < 2 * kHeadDim) gsum[i] = umma::cluster_ld64(umma::cluster_map(umma::smem_addr(part + o), (uint32_t)src));
    }
    __syncthreads();
    for (int j = t; j < per && live; j += blockDim.x) {
      const int oo = rank * per + j;
      if (oo >= 2 * kHeadDim) break;
      int64_t acc = 0;
      for (int r = 0; r < nranks; ++r) acc += gsum[r * per + j];
      const int h = oo >> 7, d = oo & (kHeadDim - 1);
      write_limbs(c.bt2, c.SP, 2 * kHidden, m, (2 * kv + h) * kHeadDim + d, sat24(acc >> 16));
    }
  }
  if (warp == 1) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, kTcCols);
  }
  umma::cluster_sync();  // no rank leaves while another still reads its shared memory
}

// Attention of the per-stage batch-1 path (grid: ranks x 8 KV heads, one cluster per head).
// 128 CTAs leave room for a 4-slot ring: a rank's keys of a 513-position
// context (2 K + 2 V chunks) are all in flight at once.
__global__ void __launch_bounds__(256) stage_attn_cl_kernel(SlotState st, int* err, int layer,
                                                            const int32_t* __restrict__ exp_lut, int kpr_cap) {
  attn_cl_body<true, kStageAttnRing>(BatchCtx{}, st, err, layer, nullptr, nullptr, nullptr, nullptr, exp_lut, kpr_cap);
}

// Per (KV head, column): q heads 2 kv, 2 kv + 1 normed and roped in place in
// qkv, k normed and roped into the cache, v copied into the cache.
__global__ void __launch_bounds__(128) prefill_qk_kernel(const SlotState* __restrict__ col_slots,
                                                         const int32_t* __restrict__ col_pos4, int32_t* qkv,
                                                         int layer, const int32_t* __restrict__ g_q,
                                                         const int32_t* __restrict__ g_k,
                                                         const int32_t* __restrict__ cos_tab,
                                                         const int32_t* __restrict__ sin_tab) {
  grid_dep_wait();
  grid_dep_launch();
  const int kv = blockIdx.x, m = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = col_pos4[4 * m];
  const KvView kvv = col_slots[m].kv;
  int32_t* raw = qkv + (size_t)m * (kQRows + 2 * kKvRows);
  if (warp < 2) {
    int32_t* row = raw + (2 * kv + warp) * kHeadDim;
    const int4 o = head_norm_rope(row, g_q, cos_tab, sin_tab, pos, lane);
    reinterpret_cast<int4*>(row)[lane] = o;
  } else if (warp == 2) {
    const int4 o = head_norm_rope(raw + kQRows + kv * kHeadDim, g_k, cos_tab, sin_tab, pos, lane);
    reinterpret_cast<int4*>(kvv.at(layer, 0, kv, pos))[lane] = o;
    kpl_put4(kvv, layer, kv, pos, 4 * lane, o);
  } else {
    const int4 v = reinterpret_cast<const int4*>(raw + kQRows + kKvRows + kv * kHeadDim)[lane];
    reinterpret_cast<int4*>(kvv.at(layer, 1, kv, pos))[lane] = v;
    vpl_put4(kvv, layer, kv, pos, 4 * lane, v);
  }
}

__global__ void __launch_bounds__(kPfThreads, 1) prefill_attn_kernel(PfAttn a) {
  extern __shared__ uint8_t pf_raw[];
  const uint32_t raw_addr = umma::smem_addr(pf_raw);
  uint8_t* base = pf_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);  // 1024-byte aligned: swizzle atoms
  uint8_t* qL = base;                  // [3][128 rows][128 B] q limbs, UMMA A (passes 1-2)
  uint8_t* kL = base + kPfQlBytes;     // [3][64 keys][128 B] key limbs, UMMA B (passes 1-2)
  int32_t* stg = reinterpret_cast<int32_t*>(base + kPfOperands);  // [64][kPfStride] staged keys / values
  __shared__ int32_t elut[kExpLut];
  __shared__ int64_t rred[4][kPfRows];  // per column quarter: row maxima, then row sums
  __shared__ int64_t rmax[kPfRows];
  __shared__ uint64_t rsum[kPfRows], rrcp[kPfRows];  // row sums and floor((2^64 - 1) / sum)
  __shared__ uint64_t mbar;                           // the score MMAs of a chunk are done
  __shared__ uint32_t tmem_slot;
  grid_dep_wait();
  grid_dep_launch();
  const int kv = blockIdx.x;
  const PfTile tl = a.tiles[blockIdx.y];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const KvView kvv = a.col_slots[tl.col0].kv;
  const int kend = tl.pos0 + tl.nq;  // keys 0 .. kend - 1
  const int nch = (kend + kPfKeys - 1) / kPfKeys;
  auto keys_in = [&](int c) { return kend - c * kPfKeys < kPfKeys ? kend - c * kPfKeys : kPfKeys; };

  // chunk c of K (kind 0) or V (kind 1) into the staging buffer (one commit group)
  auto stage = [&](int kind, int c) {
    if (c < nch) {
      const int n = keys_in(c);
      const int32_t* src = kvv.at(a.layer, kind, kv, c * kPfKeys);  // a 64-aligned chunk is one page
      for (int i = t; i < n * (kHeadDim / 4); i += kPfThreads) {
        const int j = i >> 5, d4 = i & 31;
        cp_async16(stg + j * kPfStride + 4 * d4, src + (size_t)j * kHeadDim + 4 * d4);
      }
    }
    cp_async_commit();
  };
  // 4 limb bytes of dims 4 d4 .. +3 of row r in a 128-byte-swizzled K-major plane
  auto put_sw = [](uint8_t* plane, int r, int d4, uint32_t w) {
    *reinterpret_cast<uint32_t*>(plane + r * 128 + ((((d4 >> 2) ^ (r & 7))) << 4) + ((d4 & 3) << 2)) = w;
  };
  if (t == 0) {
    umma::bar_init(&mbar, 1);
    umma::bar_init_fence();
  }
  if (warp == 0) umma::tmem_alloc(&tmem_slot, 512);
  stage(0, 0);
  // q limbs: row r = hh * 64 + qi is head 2 kv + hh at position pos0 + qi
  for (int i = t; i < kPfRows * (kHeadDim / 4); i += kPfThreads) {
    const int r = i >> 5, d4 = i & 31, hh = r / kPfTileQ, qi = r % kPfTileQ;
    int4 v = make_int4(0, 0, 0, 0);
    if (qi < tl.nq)
      v = *reinterpret_cast<const int4*>(a.qkv + (size_t)(tl.col0 + qi) * (kQRows + 2 * kKvRows) +
                                         (2 * kv + hh) * kHeadDim + 4 * d4);
#pragma unroll
    for (int l = 0; l < 3; ++l) put_sw(qL + l * (kPfRows * 128), r, d4, limb_word(v, l));
  }
  for (int i = t; i < kExpLut; i += kPfThreads) elut[i] = a.exp_lut[i];
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // limbs written here, read by the tensor cores
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tmem_slot;

  // staged chunk -> key limbs
  auto key_limbs = [&](int c) {
    const int n = keys_in(c);
    for (int i = t; i < n * (kHeadDim / 4); i += kPfThreads) {
      const int j = i >> 5, d4 = i & 31;
      const int4 v = *reinterpret_cast<const int4*>(stg + j * kPfStride + 4 * d4);
#pragma unroll
      for (int l = 0; l < 3; ++l) put_sw(kL + l * (kPfKeys * 128), j, d4, limb_word(v, l));
    }
  };
  // Scores of a chunk on the tensor cores: D_g[128 rows][64 keys] (TMEM
  // columns 64 g) for the five shift groups g of the nine limb products,
  // 4 MMAs of K = 32 bytes each (one thread issues).
  const uint64_t qdesc = umma::sw128_desc(umma::smem_addr(qL)), kdesc = umma::sw128_desc(umma::smem_addr(kL));
  auto issue_scores = [&]() {
    constexpr int pa[9] = {0, 0, 1, 0, 1, 2, 1, 2, 2}, pb[9] = {0, 1, 0, 2, 1, 0, 2, 1, 2};
    constexpr int pg[9] = {0, 1, 1, 2, 2, 2, 3, 3, 4};
    constexpr bool first[9] = {true, true, false, true, false, false, true, false, true};
#pragma unroll
    for (int q = 0; q < 9; ++q) {
      const uint32_t idesc = umma::i8_idesc_ab(kPfRows, kPfKeys, pa[q] == 2, pb[q] == 2);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ad = qdesc + (uint64_t)((pa[q] * kPfRows * 128 + 32 * ks) >> 4);
        const uint64_t bd = kdesc + (uint64_t)((pb[q] * kPfKeys * 128 + 32 * ks) >> 4);
        const uint32_t d = tmem + (uint32_t)(pg[q] * kPfKeys);
        if (first[q] && ks == 0)
          umma::mma_i8_init(d, ad, bd, idesc);
        else
          umma::mma_i8_acc(d, ad, bd, idesc);
      }
    }
    umma::mma_commit(&mbar);
  };
  // TMEM read-out: warp (sp, cq) reads lanes 32 sp .. +31 (rows) and the
  // chunk's columns 16 cq .. +15 (keys); lane = row r = 32 sp + lane
  const int sp = warp & 3, cq = warp >> 2;
  const int er = 32 * sp + lane;
  const int eqi = er % kPfTileQ;
  const bool erow = eqi < tl.nq;
  bool ok = true;
  uint32_t phase = 0;
  auto scores_of = [&](int cb, int64_t (&raw)[8]) {
    int32_t v[5][8];
    const uint32_t lb = tmem + ((uint32_t)(32 * sp) << 16) + (uint32_t)cb;
#pragma unroll
    for (int g = 0; g < 5; ++g) umma::tmem_ld<8>(lb + (uint32_t)(g * kPfKeys), v[g]);
    umma::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 8; ++i)
      raw[i] = (int64_t)v[0][i] + (int64_t)v[1][i] * 256 + (int64_t)v[2][i] * 65536 + (int64_t)v[3][i] * 16777216 +
               (int64_t)v[4][i] * 4294967296LL;
  };
  // one pass over the K chunks; body(c, cb, raw) for every 8 keys of the warp's column quarter
  auto k_pass = [&](auto&& body) {
    for (int c = 0; c < nch; ++c) {
      cp_async_wait0();
      __syncthreads();  // chunk c staged; the previous chunk's TMEM reads are done
      key_limbs(c);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
      stage(0, c + 1);
      if (t == 0) issue_scores();
      if (!umma::bar_wait(&mbar, phase)) ok = false;
      umma::fence_after_sync();
#pragma unroll
      for (int cb = 16 * cq; cb < 16 * cq + 16; cb += 8) {
        int64_t raw[8];
        scores_of(cb, raw);
        body(c, cb, raw);
      }
      umma::fence_before_sync();
      phase ^= 1u;
    }
  };
  // pass 1: row maxima of the raw scores (the score scaling is monotonic, so
  // the maximum scaled score is the scaled maximum)
  int64_t mx = INT64_MIN;
  k_pass([&](int c, int cb, const int64_t (&raw)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = c * kPfKeys + cb + i;
      if (erow && j <= tl.pos0 + eqi) mx = raw[i] > mx ? raw[i] : mx;
    }
  });
  stage(0, 0);  // pass 2 streams K again
  rred[cq][er] = mx;
  __syncthreads();
  if (t < kPfRows) {
    int64_t m = rred[0][t];
#pragma unroll
    for (int q = 1; q < 4; ++q) m = rred[q][t] > m ? rred[q][t] : m;
    rmax[t] = m == INT64_MIN ? m : scale_score(m, kScoreScale);
  }
  __syncthreads();
  // pass 2: LUT indices (kept in the u16 scratch, one 16-byte store per 8 keys) and exp sums
  const int64_t rmx = rmax[er];
  uint16_t* erow_idx =
      a.lut_idx + ((size_t)(tl.col0 + (erow ? eqi : 0)) * kQHeads + 2 * kv + er / kPfTileQ) * a.idx_ld;
  int64_t esum = 0;
  k_pass([&](int c, int cb, const int64_t (&raw)[8]) {
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = c * kPfKeys + cb + i;
      if (erow && j <= tl.pos0 + eqi) {
        const int ix = lut_index(rmx, scale_score(raw[i], kScoreScale));
        esum += elut[ix];
        w[i >> 1] |= (uint32_t)ix << (16 * (i & 1));
      }
    }
    if (erow) *reinterpret_cast<uint4*>(erow_idx + c * kPfKeys + cb) = make_uint4(w[0], w[1], w[2], w[3]);
  });
  rred[cq][er] = esum;
  __syncthreads();
  if (t < kPfRows) {
    const uint64_t s = (uint64_t)(rred[0][t] + rred[1][t] + rred[2][t] + rred[3][t]);
    rsum[t] = s;
    rrcp[t] = s > 0 ? ~0ULL / s : 0;
  }
  if (!ok) atomicExch(a.err, 5);
  // pass 3: probability-weighted values on tcgen05, both heads at once, in
  // 128-key chunks (two 64-key stagings).  A = probability limbs [3][128 rows]
  // [128 keys], B = value limbs [3][128 dims][128 keys] (both 128-byte-swizzled
  // K-major, in the score operands' space), D = five TMEM accumulators per
  // 64-dim half (the halves run one after the other), folded into int64 after
  // every chunk, so no int32 sum spans more than 128 keys.  Probabilities come
  // from the row's Barrett reciprocal: prob = (lut[idx] << 16) / sum.
  uint8_t* pLt = base;                      // [3][128][128] probability limbs
  uint8_t* vTt = base + 3 * kPfRows * 128;  // [3][128][128] value limbs
  constexpr int kPvKeys = 2 * kPfKeys;
  const int nch2 = (kend + kPvKeys - 1) / kPvKeys;
  int64_t tot[2][16];  // dims 64 h + 16 cq + i of row er
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int i = 0; i < 16; ++i) tot[h][i] = 0;
  // the LUT-index scratch row of this thread's probability items
  auto idx_base = [&](int r) {
    const int qi = r % kPfTileQ;
    return a.lut_idx + ((size_t)(tl.col0 + (qi < tl.nq ? qi : 0)) * kQHeads + 2 * kv + r / kPfTileQ) * a.idx_ld;
  };
  // staged 64 keys -> value limbs at keys 64 half .. (lane (d % 8, j4) packs keys 4 j4 .. +3 of dim d)
  auto value_limbs = [&](int half) {
    for (int i = t; i < kHeadDim * (kPfKeys / 4); i += kPfThreads) {
      const int d = (i & 7) | ((i >> 5) << 3), j4 = (i >> 3) & 3;
      const int dd = d & (kHeadDim - 1), jg = j4 + 4 * (d >> 7);
      const int4 v = make_int4(stg[(4 * jg + 0) * kPfStride + dd], stg[(4 * jg + 1) * kPfStride + dd],
                               stg[(4 * jg + 2) * kPfStride + dd], stg[(4 * jg + 3) * kPfStride + dd]);
#pragma unroll
      for (int l = 0; l < 3; ++l) put_sw(vTt + l * (kHeadDim * 128), dd, 16 * half + jg, limb_word(v, l));
    }
  };
  const uint64_t pdesc = umma::sw128_desc(umma::smem_addr(pLt)), vdesc = umma::sw128_desc(umma::smem_addr(vTt));
  auto issue_values = [&](int h, bool any2) {
    constexpr int ppa[9] = {0, 0, 1, 0, 1, 1, 2, 2, 2}, ppb[9] = {0, 1, 0, 2, 1, 2, 0, 1, 2};
    constexpr int ppg[9] = {0, 1, 1, 2, 2, 3, 2, 3, 4};
    constexpr bool first[9] = {true, true, false, true, false, true, false, false, true};
#pragma unroll
    for (int q = 0; q < 9; ++q) {
      if (ppa[q] == 2 && !any2) continue;  // p2 = 0 in every row of the chunk: group 4 stays unused
      const uint32_t idesc = umma::i8_idesc_ab(kPfRows, 64, false, ppb[q] == 2);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t ad = pdesc + (uint64_t)((ppa[q] * kPfRows * 128 + 32 * ks) >> 4);
        const uint64_t bd = vdesc + (uint64_t)((ppb[q] * kHeadDim * 128 + h * 64 * 128 + 32 * ks) >> 4);
        const uint32_t d = tmem + (uint32_t)(ppg[q] * 64);
        if (first[q] && ks == 0)
          umma::mma_i8_init(d, ad, bd, idesc);
        else
          umma::mma_i8_acc(d, ad, bd, idesc);
      }
    }
    umma::mma_commit(&mbar);
  };
  stage(1, 0);  // the staging buffer is free: the last K chunk was converted
  constexpr int kPvItems = kPfRows * (kPvKeys / 4) / kPfThreads;  // (row, 4 keys) items per thread
  for (int c2 = 0; c2 < nch2; ++c2) {
    // this thread's LUT indices of the chunk, loaded first so that the loads
    // overlap the first value conversion
    uint2 ixw[kPvItems];
#pragma unroll
    for (int u = 0; u < kPvItems; ++u) {
      const int i = t + u * kPfThreads, r = i >> 5, k4 = i & 31, qi = r % kPfTileQ;
      const int j0 = c2 * kPvKeys + 4 * k4;
      ixw[u] = make_uint2(0, 0);
      if (qi < tl.nq && j0 <= tl.pos0 + qi) ixw[u] = *reinterpret_cast<const uint2*>(idx_base(r) + j0);
    }
    cp_async_wait0();
    __syncthreads();  // keys 128 c2 .. +63 staged; the previous chunk's TMEM reads are done
    value_limbs(0);
    __syncthreads();
    stage(1, 2 * c2 + 1);
    // probability limbs: item (row r, keys 4 k4 .. +3) -> one word per limb plane
    int big = 0;
#pragma unroll
    for (int u = 0; u < kPvItems; ++u) {
      const int i = t + u * kPfThreads, r = i >> 5, k4 = i & 31, qi = r % kPfTileQ;
      const int j0 = c2 * kPvKeys + 4 * k4;
      uint32_t pw[3] = {0, 0, 0};
      if (qi < tl.nq && j0 <= tl.pos0 + qi) {
        const uint2 ix = ixw[u];
        const uint32_t ixs[4] = {ix.x & 0xFFFFu, ix.x >> 16, ix.y & 0xFFFFu, ix.y >> 16};
        const uint64_t s = rsum[r], rc = rrcp[r];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (j0 + e <= tl.pos0 + qi) {
            const uint32_t p = barrett_div((uint64_t)elut[ixs[e]] << 16, s, rc);
            big |= (int)(p >> 16);
#pragma unroll
            for (int l = 0; l < 3; ++l) pw[l] |= ((p >> (8 * l)) & 0xFFu) << (8 * e);
          }
      }
#pragma unroll
      for (int l = 0; l < 3; ++l) put_sw(pLt + l * (kPfRows * 128), r, k4, pw[l]);
    }
    const bool any2 = __syncthreads_or(big) != 0;  // some p = 2^16 in this chunk: its limb-2 products count
    cp_async_wait0();
    __syncthreads();  // keys 128 c2 + 64 .. +63 staged
    value_limbs(1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    stage(1, 2 * c2 + 2);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (t == 0) issue_values(h, any2);
      if (!umma::bar_wait(&mbar, phase)) ok = false;
      phase ^= 1u;
      umma::fence_after_sync();
#pragma unroll
      for (int cb = 0; cb < 16; cb += 8) {
        int32_t v[5][8];
        const uint32_t lb = tmem + ((uint32_t)(32 * sp) << 16) + (uint32_t)(16 * cq + cb);
#pragma unroll
        for (int g5 = 0; g5 < 4; ++g5) umma::tmem_ld<8>(lb + (uint32_t)(g5 * 64), v[g5]);
        if (any2) umma::tmem_ld<8>(lb + 4u * 64u, v[4]);
        umma::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          tot[h][cb + i] += (int64_t)v[0][i] + (int64_t)v[1][i] * 256 + (int64_t)v[2][i] * 65536 +
                            (int64_t)v[3][i] * 16777216 + (any2 ? (int64_t)v[4][i] * 4294967296LL : 0);
      }
      umma::fence_before_sync();
      __syncthreads();  // TMEM read before the next MMAs overwrite it
      umma::fence_after_sync();
    }
  }
  if (!ok) atomicExch(a.err, 5);
  // outputs of row er (head 2 kv + er / 64, position pos0 + er % 64) as limbs of the o_proj input
  if (erow) {
    const int col = tl.col0 + eqi;
    uint8_t* bt = a.bt2 + (size_t)(col / kPfSub) * a.bt2_sub;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 16; ++i)
        write_limbs(bt, kPfSub, 2 * kHidden, col % kPfSub, (2 * kv + er / kPfTileQ) * kHeadDim + 64 * h + 16 * cq + i,
                    sat24(tot[h][i] >> 16));
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    umma::fence_after_sync();
    umma::tmem_dealloc(tmem, 512);
  }
}

}  // namespace q4

// ===========================================================================
// Host side
// ===========================================================================
using namespace q4;

namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, int cluster_y,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_y > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = (unsigned)cluster_y;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// PDL launch with thread-block clusters of `cluster_x` CTAs along x
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster_x(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, int cluster_x,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, Args... args) {
  return launch_ex(k, g, b, smem, s, 1, args...);
}

#define BQ(call)                                                                                        \
  do {                                                                                                  \
    const cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// K splits of each batched GEMM (a cluster of that many CTAs per row tile)
template <int SN, int KIND>
cudaError_t launch_gemm(const CUtensorMap& amap, const CUtensorMap& amap2, const CUtensorMap& bmap, const BatchCtx& c,
                        const uint16_t* scales, const uint16_t* scales2, int rows, int K, int splits, int SP,
                        const int32_t* sig_lut, ArgBestD* partial, cudaStream_t s, unsigned long long* trace,
                        int subs, int b_sub_rows, L2Prefetch pf = L2Prefetch{}) {
  // the epilogue's row bookkeeping uses shifts: splits must be 1, 2, 4 or 8;
  // a CTA holds the scales of at most kUMaxKt K tiles
  // the limb box of a K tile spans the three limb blocks: SN = SP
  if (splits < 1 || splits > 8 || (splits & (splits - 1)) || K % (128 * splits) || K / splits > 128 * kUMaxKt ||
      SN != SP || SP > kBatchSeqMax)
    return cudaErrorInvalidValue;
  // O / down stage their residual rows (128 / splits of them) in 64 rows' room
  if ((KIND == kGemmO || KIND == kGemmDown) && splits < 2) return cudaErrorInvalidValue;
  UGemm g{c, scales, scales2, rows, K, K / 128 / splits, SP, SP / SN, b_sub_rows, sig_lut, partial, trace, pf};
  const dim3 grid((unsigned)(subs * (SP / SN)), (unsigned)splits, (unsigned)((rows + 127) / 128));
  return launch_ex(umma_gemm_kernel<SN, KIND>, grid, dim3(kUThreads), UCfg<SN, KIND>::SMEM, s, splits, amap, amap2,
                   bmap, g);
}

// The same with the chunk width chosen at run time.
template <int KIND, typename... Args>
cudaError_t launch_gemm_sn(int sn, Args... args) {
  switch (sn) {
    case 8: return launch_gemm<8, KIND>(args...);
    case 16: return launch_gemm<16, KIND>(args...);
    case 24: return launch_gemm<24, KIND>(args...);
    case 32: return launch_gemm<32, KIND>(args...);
    case 64: return launch_gemm<64, KIND>(args...);
    default: return cudaErrorInvalidValue;
  }
}

// The weights of a layer's GEMMs, for the L2 prefetch issued one GEMM ahead:
// q/k/v prefetches o_proj (past the attention, whose K/V loads are
// evict-first), o_proj gate/up, gate/up down, down the next layer's q/k/v.
L2Prefetch pf_qkv(const BatchLayerW& w) {
  return L2Prefetch{{w.wqkv, w.sqkv, nullptr, nullptr},
                    {(uint32_t)(kQRows + 2 * kKvRows) * kHidden / 2, (uint32_t)(kQRows + 2 * kKvRows) * kHidden / 32, 0, 0}};
}
L2Prefetch pf_o(const BatchLayerW& w) {
  return L2Prefetch{{w.wo, w.so, nullptr, nullptr}, {(uint32_t)kHidden * kHidden, (uint32_t)kHidden * kHidden / 16, 0, 0}};
}
// the last layer's q/k/v GEMM also pulls the tied LM head (82.6 MB, fits L2
// beside the streamed evict-first K/V) in, about 60 us before the LM head runs
L2Prefetch pf_o_and_lm(const BatchLayerW& w, const uint8_t* emb, const uint16_t* semb, int vocab) {
  L2Prefetch pf = pf_o(w);
  pf.p[2] = emb;
  pf.bytes[2] = (uint32_t)vocab * (kHidden / 2);
  pf.p[3] = semb;
  pf.bytes[3] = (uint32_t)vocab * (kHidden / kGroup) * 2;
  return pf;
}
L2Prefetch pf_gu(const BatchLayerW& w) {
  return L2Prefetch{{w.wgate, w.wup, w.sgate, w.sup},
                    {(uint32_t)kInter * kHidden / 2, (uint32_t)kInter * kHidden / 2, (uint32_t)kInter * kHidden / 32,
                     (uint32_t)kInter * kHidden / 32}};
}
L2Prefetch pf_down(const BatchLayerW& w) {
  return L2Prefetch{{w.wdown, w.sdown, nullptr, nullptr}, {(uint32_t)kHidden * kInter / 2, (uint32_t)kHidden * kInter / 32, 0, 0}};
}

// K splits of each GEMM of a decode step (a cluster of that many CTAs per row
// tile); prefill launches cover up to 16 sub-batches of 64 columns each, so
// they need fewer splits to fill the GPU
int decode_splits(int kind, int SP) {
  (void)SP;
  return kind == kGemmQkv ? 4 : kind == kGemmGu ? 2 : kind == kGemmLm ? 1 : 8;
}
constexpr int kPfSplitQkv = 1, kPfSplitO = 2, kPfSplitGu = 1, kPfSplitDown = 4;

bool attn_one_cta_per_head(const BatchPlan& p) { return p.S * kKvHeads >= 148 && p.max_ctx <= 1024; }
// dynamic shared memory of batch_attn_kernel: alignment slack, ring, query
// bytes, scores [2][max_ctx]; with its 4.3 KB static and 1 KB reserved, four
// CTAs fit an SM up to max_ctx = 1024 (the occupancy calculator reports one
// for a kernel that allocates TMEM; 64 columns per CTA leave room for four)
size_t attn_tc_smem(const BatchPlan& p) {
  const size_t scores = (size_t)2 * p.max_ctx * 8, pbytes = (size_t)(p.max_ctx + kTcKeys - 1) / kTcKeys * 2048;
  return (size_t)kTcSmemFixed + (scores > pbytes ? scores : pbytes);
}
// cluster size of the cluster attention (16 CTAs for batches of up to 4 sequences), the keys per
// rank its score buffer must hold, and whether it covers max_ctx
int attn_cl_ranks(const BatchPlan& p) { return p.S <= 4 ? 16 : 8; }
int attn_cl_kpr(const BatchPlan& p) {
  const int r = attn_cl_ranks(p);
  return ((p.max_ctx + r - 1) / r + kAttnChunk - 1) / kAttnChunk * kAttnChunk;
}
bool attn_cluster(const BatchPlan& p) { return !attn_one_cta_per_head(p) && attn_cl_kpr(p) <= kClKprMax; }
// Tensor-core cluster attention (models with byte planes): positions per rank
// (a multiple of 128) and dynamic shared memory for R ranks, and the largest
// R <= 16 whose R x 8 x S CTAs fit the GPU at once (TMEM: 4 CTAs per SM;
// shared memory: the kernel's 4.3 KB static, 1 KB reserved), 0 if none.
int attn_cl_tc_kpr(const BatchPlan& p, int R) { return ((p.max_ctx + R - 1) / R + kTcKeys - 1) / kTcKeys * kTcKeys; }
size_t attn_cl_tc_smem(const BatchPlan& p, int R) { return (size_t)kTcSmemFixed + (size_t)16 * attn_cl_tc_kpr(p, R); }
int attn_cl_tc_ranks(const BatchPlan& p) {
  if (!p.kv_planes || attn_one_cta_per_head(p)) return 0;
  for (int R = 16; R >= 2; --R) {
    if (attn_cl_tc_kpr(p, R) > kClTcKprMax) break;
    const size_t per_cta = attn_cl_tc_smem(p, R) + 4608 + 1024;
    const int by_smem = (int)(233472 / per_cta), per_sm = by_smem < 4 ? by_smem : 4;
    if (R * kKvHeads * p.S <= 148 * per_sm) return R;
  }
  return 0;
}
size_t attn_cl_smem(const BatchPlan& p) {
  return (size_t)kAttnRing * kAttnChunkBytes + (size_t)2 * attn_cl_kpr(p) * 8;
}

template <int SP>
int enqueue_t(const BatchPlan& p, cudaStream_t s, BatchMarks* mk) {
  auto mark = [&](int kind) -> int {
    if (!mk) return Q4GPU_OK;
    cudaEvent_t e;
    BQ(cudaEventCreate(&e));
    mk->ev.push_back(e);
    mk->kind.push_back(kind);
    BQ(cudaEventRecord(e, s));
    return Q4GPU_OK;
  };
  int rc;
  // GEMM launch i records into its own slice of the trace (kGemmTraceCtas CTAs x 8 stamps)
  auto gtrace = [&](int i) -> unsigned long long* {
    return p.gemm_trace ? p.gemm_trace + (size_t)i * kGemmTraceCtas * 8 : nullptr;
  };
#define BMARK(k) \
  if ((rc = mark(k))) return rc
  const BatchCtx c{p.slots, p.S,    p.SP,      p.qkv_raw, p.bt1,   p.bt2,     p.bt3,
                   p.lm_from, p.err, p.pos0, p.hidden0, p.post0, p.max_ctx, p.trace};
  const AttnScratch as{p.att_S, p.att_P, p.att_M, p.att_O, p.att_cnt_s, p.att_cnt_v, p.max_ctx};
  const dim3 attn_grid((unsigned)((p.max_ctx + kPage - 1) / kPage), kKvHeads, (unsigned)p.S);
  // enough (KV head, sequence) pairs to fill the GPU in one wave: one CTA per
  // pair; otherwise split each pair's context over pages
  const bool one_cta_per_head = attn_one_cta_per_head(p);
  const size_t ring_smem = attn_tc_smem(p);
  BMARK(-1);
  BQ(launch_pdl(batch_embed_kernel, dim3(p.S), dim3(256), 0, s, c, p.emb, p.semb));
  BMARK(kBkEmbed);
  for (int l = 0; l < p.n_layers; ++l) {
    const BatchLayerW& w = p.layers[l];
    const bool last_layer = l + 1 == p.n_layers;
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 0, w.g_in, (int32_t*)nullptr));
    BMARK(kBkNorm);
    BQ(launch_gemm_sn<kGemmQkv>(q4gpu_batch_gemm_chunk(kGemmQkv, SP), w.mqkv, w.mqkv, p.mb_qkv, c, w.sqkv,
                                (const uint16_t*)nullptr, kQRows + 2 * kKvRows, kHidden, decode_splits(kGemmQkv, SP),
                                SP, (const int32_t*)nullptr, (ArgBestD*)nullptr, s, gtrace(4 * l + 0), 1, 0,
                                last_layer && !p.final_act ? pf_o_and_lm(w, p.emb, p.semb, p.vocab) : pf_o(w)));
    BMARK(kBkQkv);
    if (one_cta_per_head) {
      BQ(launch_pdl(batch_attn_kernel, dim3(kKvHeads, p.S), dim3(256), ring_smem, s, c, l, w.g_q, w.g_k, p.cos_tab,
                    p.sin_tab, p.exp_lut));
    } else if (attn_cl_tc_ranks(p) > 0) {
      const int R = attn_cl_tc_ranks(p);
      BQ(launch_cluster_x(batch_attn_cl_tc_kernel, dim3(R, kKvHeads, p.S), dim3(256), attn_cl_tc_smem(p, R), s, R, c,
                          l, w.g_q, w.g_k, p.cos_tab, p.sin_tab, p.exp_lut, attn_cl_tc_kpr(p, R)));
    } else if (attn_cluster(p)) {
      BQ(launch_cluster_x(batch_attn_cl_kernel, dim3(attn_cl_ranks(p), kKvHeads, p.S), dim3(256), attn_cl_smem(p),
                          s, attn_cl_ranks(p), c, l, w.g_q, w.g_k, p.cos_tab, p.sin_tab, p.exp_lut, attn_cl_kpr(p)));
    } else {
      BQ(launch_pdl(batch_attn_scores_kernel, attn_grid, dim3(256), 0, s, c, as, l, w.g_q, w.g_k, p.cos_tab,
                    p.sin_tab, p.exp_lut));
      BQ(launch_pdl(batch_attn_values_kernel, attn_grid, dim3(256), 0, s, c, as, l));
    }
    BMARK(kBkAttn);
    BQ(launch_gemm_sn<kGemmO>(q4gpu_batch_gemm_chunk(kGemmO, SP), w.mo, w.mo, p.mb_o, c, w.so,
                              (const uint16_t*)nullptr, kHidden, 2 * kHidden, decode_splits(kGemmO, SP), SP,
                              (const int32_t*)nullptr, (ArgBestD*)nullptr, s, gtrace(4 * l + 1), 1, 0, pf_gu(w)));
    BMARK(kBkO);
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 1, w.g_post, (int32_t*)nullptr));
    BMARK(kBkNorm);
    BQ(launch_gemm_sn<kGemmGu>(q4gpu_batch_gemm_chunk(kGemmGu, SP), w.mgate, w.mup, p.mb_gu, c, w.sgate, w.sup,
                               2 * kInter, kHidden, decode_splits(kGemmGu, SP), SP, p.sig_lut, (ArgBestD*)nullptr, s,
                               gtrace(4 * l + 2), 1, 0, pf_down(w)));
    BMARK(kBkGu);
    BQ(launch_gemm_sn<kGemmDown>(q4gpu_batch_gemm_chunk(kGemmDown, SP), w.mdown, w.mdown, p.mb_down, c, w.sdown,
                                 (const uint16_t*)nullptr, kHidden, kInter, decode_splits(kGemmDown, SP), SP,
                                 (const int32_t*)nullptr, (ArgBestD*)nullptr, s, gtrace(4 * l + 3), 1, 0,
                                 last_layer ? L2Prefetch{} : pf_qkv(p.layers[l + 1])));
    BMARK(kBkDown);
  }
  BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.S), dim3(256), 0, s, c, 0, p.g_final, p.final_act));
  BMARK(kBkNorm);
  if (p.final_act) return Q4GPU_OK;  // hidden-only step: the LM head runs per vocabulary shard
  BQ(launch_gemm_sn<kGemmLm>(q4gpu_batch_gemm_chunk(kGemmLm, SP), p.mlm, p.mlm, p.mb_lm, c, p.semb,
                             (const uint16_t*)nullptr, p.vocab, kHidden, 1, SP, (const int32_t*)nullptr, p.lm_partial,
                             s, gtrace(4 * p.n_layers), 1, 0));
  BMARK(kBkLm);
  BQ(launch_pdl(batch_argmax_kernel, dim3(p.S), dim3(256), 0, s, c, (const ArgBestD*)p.lm_partial,
                (p.vocab + 127) / 128));
  BMARK(kBkArgmax);
#undef BMARK
  return Q4GPU_OK;
}

template <int SN, int KIND>
int set_smem() {
  BQ(cudaFuncSetAttribute(umma_gemm_kernel<SN, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)UCfg<SN, KIND>::SMEM));
  return Q4GPU_OK;
}

template <int SN>
int set_smem_all_kinds() {
  int rc;
  if ((rc = set_smem<SN, kGemmQkv>()) || (rc = set_smem<SN, kGemmO>()) || (rc = set_smem<SN, kGemmGu>()) ||
      (rc = set_smem<SN, kGemmDown>()) || (rc = set_smem<SN, kGemmLm>()))
    return rc;
  return Q4GPU_OK;
}

// shared-memory attributes of every GEMM instantiation, once per process and device
int gemm_setup() {
  static bool done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return q4gpu_fail(Q4GPU_ERR_CUDA, "no device");
  if (done[dev]) return Q4GPU_OK;
  int rc;
  if ((rc = set_smem_all_kinds<8>()) || (rc = set_smem_all_kinds<16>()) || (rc = set_smem_all_kinds<24>()) ||
      (rc = set_smem_all_kinds<32>()) || (rc = set_smem_all_kinds<64>()))
    return rc;
  done[dev] = true;
  return Q4GPU_OK;
}

template <int SP>
int setup_t(const BatchPlan& p) {
  int rc;
  if ((rc = gemm_setup())) return rc;
  if (attn_cl_tc_ranks(p) > 0) {
    const int R = attn_cl_tc_ranks(p);
    BQ(cudaFuncSetAttribute(batch_attn_cl_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)attn_cl_tc_smem(p, R)));
    BQ(cudaFuncSetAttribute(batch_attn_cl_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  }
  if (attn_cluster(p)) {
    BQ(cudaFuncSetAttribute(batch_attn_cl_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_cl_smem(p)));
    BQ(cudaFuncSetAttribute(batch_attn_cl_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  }
  if (attn_one_cta_per_head(p))
    BQ(cudaFuncSetAttribute(batch_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_tc_smem(p)));
  return Q4GPU_OK;
}

}  // namespace

namespace {
int stage_attn_kpr(int max_ctx) {
  return ((max_ctx + kStageAttnRanks - 1) / kStageAttnRanks + kAttnChunk - 1) / kAttnChunk * kAttnChunk;
}
size_t stage_attn_smem(int max_ctx) {
  return (size_t)kStageAttnRing * kAttnChunkBytes + (size_t)2 * stage_attn_kpr(max_ctx) * 8;
}
}  // namespace

bool q4gpu_stage_attention_fits(int max_ctx) { return max_ctx > 0 && stage_attn_kpr(max_ctx) <= kClKprMax; }

int q4gpu_stage_attention_setup(int max_ctx) {
  if (!q4gpu_stage_attention_fits(max_ctx)) return q4gpu_fail(Q4GPU_ERR_SHAPE, "stage attention: max_ctx too large");
  BQ(cudaFuncSetAttribute(stage_attn_cl_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stage_attn_smem(max_ctx)));
  BQ(cudaFuncSetAttribute(stage_attn_cl_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return Q4GPU_OK;
}

int q4gpu_enqueue_stage_attention(const SlotState& st, int* err, int layer, const int32_t* exp_lut, int max_ctx,
                                  cudaStream_t s) {
  BQ(launch_cluster_x(stage_attn_cl_kernel, dim3(kStageAttnRanks, kKvHeads), dim3(256), stage_attn_smem(max_ctx), s,
                      kStageAttnRanks, st, err, layer, exp_lut, stage_attn_kpr(max_ctx)));
  return Q4GPU_OK;
}

int q4gpu_batch_padded(int S) { return S <= 8 ? 8 : S <= 16 ? 16 : S <= 24 ? 24 : S <= 32 ? 32 : 64; }

// One MMA costs about the same below N = 96 (M = 128, K = 32: ~46 cycles up
// to N = 64, ~96 at N = 192), and every sequence chunk of a tile repeats the
// tile's plane building, so decode GEMMs take all SP sequences per CTA and
// reach the GPU's width by splitting K.
int q4gpu_batch_gemm_chunk(int kind, int SP) {
  (void)kind;
  return SP;
}

int q4gpu_batch_setup(const BatchPlan& p) {
  switch (p.SP) {
    case 8: return setup_t<8>(p);
    case 16: return setup_t<16>(p);
    case 24: return setup_t<24>(p);
    case 32: return setup_t<32>(p);
    case 64: return setup_t<64>(p);
    default: return q4gpu_fail(Q4GPU_ERR_SHAPE, "padded batch %d", p.SP);
  }
}

int q4gpu_enqueue_batch_step(const BatchPlan& p, cudaStream_t s, BatchMarks* mk) {
  switch (p.SP) {
    case 8: return enqueue_t<8>(p, s, mk);
    case 16: return enqueue_t<16>(p, s, mk);
    case 24: return enqueue_t<24>(p, s, mk);
    case 32: return enqueue_t<32>(p, s, mk);
    case 64: return enqueue_t<64>(p, s, mk);
    default: return q4gpu_fail(Q4GPU_ERR_SHAPE, "padded batch %d", p.SP);
  }
}

int q4gpu_encode_u8_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !encode)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  }
  const cuuint64_t dims[2] = {(cuuint64_t)inner_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)inner_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q4GPU_OK;
}

int q4gpu_encode_q4_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !encode)
      return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner_bytes & 15))
    return q4gpu_fail(Q4GPU_ERR_ALIGN, "packed weights must start and have rows on 16-byte boundaries");
  const cuuint64_t dims[2] = {(cuuint64_t)inner_bytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)inner_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q4GPU_OK;
}

int q4gpu_batch_limb_rows(int SP) { return 3 * SP + kBatchPad; }

template <int SP>
int lm_shard_t(const LmShardPlan& q, cudaStream_t s) {
  BatchCtx c{};
  c.S = q.n_act;
  c.SP = SP;
  c.err = q.err;
  act_limbs_kernel<<<q.n_act, 256, 0, s>>>(q.acts, q.bt, SP);
  BQ(cudaGetLastError());
  int rc;
  if ((rc = gemm_setup())) return rc;
  const int rows = q.row_end - q.row_begin;
  BQ((launch_gemm<SP, kGemmLm>(q.amap, q.amap, q.bmap, c, q.scales, nullptr, rows, kHidden, 1, SP, nullptr, q.partial,
                               s, nullptr, 1, 0)));
  shard_argmax_kernel<<<q.n_act, 256, 0, s>>>(q.partial, (rows + 127) / 128, q.row_begin, q.best_score, q.best_row);
  BQ(cudaGetLastError());
  return Q4GPU_OK;
}

int q4gpu_prefill_setup() {
  int rc;
  if ((rc = gemm_setup())) return rc;
  BQ(cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem));
  return Q4GPU_OK;
}

int q4gpu_enqueue_prefill_block(const PrefillPlan& p, cudaStream_t s) {
  if (p.n_cols < 1 || p.n_cols > kPfBlock || p.n_tiles < 1 || p.n_tiles > kPfBlock)
    return q4gpu_fail(Q4GPU_ERR_SHAPE, "prefill block of %d columns / %d tiles", p.n_cols, p.n_tiles);
  constexpr int kRow = kQRows + 2 * kKvRows;
  constexpr size_t nb = (size_t)kPfSubRows;  // rows of one sub-batch's limb matrix
  const int nsub = (p.n_cols + kPfSub - 1) / kPfSub;
  // all columns of the block in one context: the GEMMs take sub-batch z from blockIdx.z
  const BatchCtx c{p.col_slots, p.n_cols, kPfSub, p.qkv,      p.bt1,         p.bt2,  p.bt3,
                   nullptr,     p.err,    p.col_pos4, p.hidden, p.post,        p.max_ctx, nullptr,
                   nb * kHidden, nb * kInter};
  BQ(launch_pdl(batch_embed_kernel, dim3(p.n_cols), dim3(256), 0, s, c, p.emb, p.semb));
  for (int l = 0; l < p.n_layers; ++l) {
    const BatchLayerW& w = p.layers[l];
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.n_cols), dim3(256), 0, s, c, 0, w.g_in, (int32_t*)nullptr));
    BQ((launch_gemm<kPfSub, kGemmQkv>(w.mqkv, w.mqkv, p.mb1, c, w.sqkv, nullptr, kRow, kHidden, kPfSplitQkv, kPfSub,
                                      nullptr, nullptr, s, nullptr, nsub, kPfSubRows, pf_o(w))));
    BQ(launch_pdl(prefill_qk_kernel, dim3(kKvHeads, p.n_cols), dim3(128), 0, s, p.col_slots, p.col_pos4, p.qkv, l,
                  w.g_q, w.g_k, p.cos_tab, p.sin_tab));
    const PfAttn a{p.tiles, p.col_slots, p.qkv, p.bt2, nb * 2 * kHidden, p.lut_idx, (p.max_ctx + 63) / 64 * 64, l,
                   p.exp_lut, p.err};
    BQ(launch_pdl(prefill_attn_kernel, dim3(kKvHeads, p.n_tiles), dim3(kPfThreads), kPfSmem, s, a));
    BQ((launch_gemm<kPfSub, kGemmO>(w.mo, w.mo, p.mb2, c, w.so, nullptr, kHidden, 2 * kHidden, kPfSplitO, kPfSub,
                                    nullptr, nullptr, s, nullptr, nsub, kPfSubRows, pf_gu(w))));
    BQ(launch_pdl(batch_norm_limbs_kernel, dim3(p.n_cols), dim3(256), 0, s, c, 1, w.g_post, (int32_t*)nullptr));
    BQ((launch_gemm<kPfSub, kGemmGu>(w.mgate, w.mup, p.mb1, c, w.sgate, w.sup, 2 * kInter, kHidden, kPfSplitGu,
                                     kPfSub, p.sig_lut, nullptr, s, nullptr, nsub, kPfSubRows, pf_down(w))));
    BQ((launch_gemm<kPfSub, kGemmDown>(w.mdown, w.mdown, p.mb3, c, w.sdown, nullptr, kHidden, kInter, kPfSplitDown,
                                       kPfSub, nullptr, nullptr, s, nullptr, nsub, kPfSubRows,
                                       l + 1 < p.n_layers ? pf_qkv(p.layers[l + 1]) : L2Prefetch{})));
  }
  return Q4GPU_OK;
}

int q4gpu_enqueue_lm_shard(const LmShardPlan& q, cudaStream_t s) {
  switch (q4gpu_batch_padded(q.n_act)) {
    case 8: return lm_shard_t<8>(q, s);
    case 16: return lm_shard_t<16>(q, s);
    case 24: return lm_shard_t<24>(q, s);
    case 32: return lm_shard_t<32>(q, s);
    default: return lm_shard_t<64>(q, s);
  }
}

int q4gpu_enqueue_batch_commit(const BatchPlan& p, const int64_t* tokens, const int64_t* scores, cudaStream_t s) {
  BatchCtx c{};
  c.slots = p.slots;
  c.S = p.S;
  c.lm_from = p.lm_from;
  batch_commit_kernel<<<(p.S + 63) / 64, 64, 0, s>>>(c, tokens, scores);
  return q4gpu_check_launch();
}

int q4gpu_enqueue_batch_commit_shards(const BatchPlan& p, const int64_t* win, int n_shards, int stride, int col0,
                                      cudaStream_t s) {
  BatchCtx c{};
  c.slots = p.slots;
  c.S = p.S;
  c.lm_from = p.lm_from;
  batch_commit_shards_kernel<<<(p.S + 63) / 64, 64, 0, s>>>(c, win, n_shards, stride, col0);
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
