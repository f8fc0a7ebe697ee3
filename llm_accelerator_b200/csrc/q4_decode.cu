// Decode-step kernels and the model runtime behind the runner seam.
//
// One decode step of one sequence slot is a chain of kernels launched with
// programmatic dependent launch (PDL) and captured once into a CUDA graph:
//   embed -> [qkv+head-norm+RoPE+KV append -> attention -> o_proj+residual
//             -> post-norm+gate/up+SwiGLU -> down+residual] x layers
//   -> final-norm+LM head+argmax (or a position advance during prefill)
// Each kernel prefetches its weight slice into L2 before it waits on the
// previous kernel, so weight traffic overlaps the dependency.  Position,
// token and score live in device memory, so successive replays feed the
// argmax back without a host round trip.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <climits>
#include <cmath>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "q4_batch.h"
#include "q4_gemv.cuh"
#include "q4_state.cuh"
#include "q4gpu_internal.h"

namespace q4 {

// Hidden-size RMSNorm of `src` (Q14.10) into `dst` (Q12.12), block-wide.
__device__ __forceinline__ void hidden_norm_to(const int32_t* __restrict__ src, const int32_t* __restrict__ gamma,
                                               int32_t* dst, int64_t* red) {
  int64_t ss = 0;
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    const int32_t v = src[i];
    dst[i] = v;
    ss += (int64_t)v * v;
  }
  ss = block_sum_i64(ss, red);
  const int64_t inv = inv_rms_from_ss(ss, kHiddenNorm);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) dst[i] = norm_apply(dst[i], inv, gamma[i], kHiddenNorm);
}

// ---------------------------------------------------------------------------
// Step kernels
// ---------------------------------------------------------------------------
__global__ void embed_step_kernel(SlotState st, const uint8_t* __restrict__ W, const uint16_t* __restrict__ S) {
  grid_dep_wait();
  grid_dep_launch();
  if (*st.pos >= st.max_ctx) return;  // stepping past the context does nothing
  const int t = st.tokens[*st.pos];
  const uint8_t* row = W + (size_t)t * (kHidden / 2);
  const uint16_t* sc = S + (size_t)t * (kHidden / kGroup);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    const uint8_t b = row[i >> 1];
    const int q = (int)((i & 1) ? (b >> 4) : (b & 0xF));
    st.hidden[i] = ((q >= 8 ? q - 16 : q) * (int32_t)sc[i / kGroup]) >> 4;
  }
}

// A cluster of four CTAs per head (16 q heads, 8 k heads, 8 v heads; 128
// rows each): CTA rank c computes dims [16 c, 16 c + 16) and their RoPE
// partners [64 + 16 c, 64 + 16 c + 16), 32 rows, so the rotation stays in the
// CTA; the per-head norm's sum of squares crosses the cluster over DSMEM.
constexpr int kQkvRanks = 4;
__global__ void __launch_bounds__(256) qkv_step_kernel(SlotState st, LayerW w, int layer,
                                                       const int32_t* __restrict__ cos_tab,
                                                       const int32_t* __restrict__ sin_tab) {
  __shared__ __align__(16) int32_t a[kHidden];
  __shared__ __align__(16) uint32_t limbs[limb_words(kHidden)];
  __shared__ int64_t bias8[kHidden / 32];
  __shared__ int64_t red[8];
  __shared__ int64_t part_ss;  // this CTA's sum of squares, read by the cluster
  __shared__ int32_t y[2 * 16];
  const int head = blockIdx.x / kQkvRanks, c = blockIdx.x % kQkvRanks;
  const int row0 = head * kHeadDim;
  const int lo = 16 * c, hi = 64 + 16 * c;  // this CTA's two 16-dim runs
  if (threadIdx.x == 0) {
    prefetch_l2(w.wqkv + (size_t)(row0 + lo) * 512, 16 * 512);
    prefetch_l2(w.wqkv + (size_t)(row0 + hi) * 512, 16 * 512);
    prefetch_l2(w.sqkv + (size_t)(row0 + lo) * 16, 16 * 32);
    prefetch_l2(w.sqkv + (size_t)(row0 + hi) * 16, 16 * 32);
  }
  grid_dep_wait();
  grid_dep_launch();
  // every CTA of the cluster reaches both cluster barriers below: no early return
  const bool live = *st.pos < st.max_ctx;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (live) {
    hidden_norm_to(st.hidden, w.g_in, a, red);
    __syncthreads();
    stage_limbs(a, kHidden, limbs, bias8);
    __syncthreads();
    // warps 0-3: rows lo + 4 w .. + 3; warps 4-7: rows hi + 4 (w - 4) .. + 3
    int64_t acc[4] = {0, 0, 0, 0};
    const int r0 = warp < 4 ? lo + 4 * warp : hi + 4 * (warp - 4);
    gemv_slice<kHidden, 4>(w.wqkv, w.sqkv, row0 + r0, kQRows + 2 * kKvRows, 0, limbs, bias8, acc);
    warp_reduce_rows<4>(acc);
    if (lane < 4) y[4 * warp + lane] = sat24(acc[lane] >> 14);  // y[j]: dim lo + j (j < 16), hi + j - 16
  }
  __syncthreads();
  const bool normed = head < kQHeads + kKvHeads;
  const int t = threadIdx.x;
  if (t < 32) {
    int64_t ss = normed && live ? (int64_t)y[t] * y[t] : 0;
    ss = warp_sum_i64(ss);
    if (t == 0) part_ss = ss;
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (live && t < 32) {
    const int pos = *st.pos;
    const int d = t < 16 ? lo + t : hi + (t - 16);
    if (normed) {
      int64_t ss = 0;
#pragma unroll
      for (int r = 0; r < kQkvRanks; ++r) {
        uint32_t addr;
        int64_t v;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"((uint32_t)__cvta_generic_to_shared(&part_ss)), "r"(r));
        asm volatile("ld.shared::cluster.b64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
        ss += v;
      }
      const int32_t* gamma = head < kQHeads ? w.g_q : w.g_k;
      const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
      // z of this dim and of its RoPE partner (the other run, same offset)
      const int tp = t < 16 ? t + 16 : t - 16, dp = t < 16 ? hi + t : lo + (t - 16);
      const int32_t z = norm_apply(y[t], inv, gamma[d], kHeadNorm);
      const int32_t zp = norm_apply(y[tp], inv, gamma[dp], kHeadNorm);
      const int64_t rot = d < 64 ? -(int64_t)zp : (int64_t)zp;
      const int32_t r = sat24(((int64_t)z * cos_tab[pos * kHeadDim + d] + rot * sin_tab[pos * kHeadDim + d]) >> 15);
      if (head < kQHeads)
        st.qrope[head * kHeadDim + d] = r;
      else {
        st.kv.at(layer, 0, head - kQHeads, pos)[d] = r;
        kpl_put1(st.kv, layer, head - kQHeads, pos, d, r);
      }
    } else {
      st.kv.at(layer, 1, head - kQHeads - kKvHeads, pos)[d] = y[t];
      vpl_put1(st.kv, layer, head - kQHeads - kKvHeads, pos, d, y[t]);
    }
  }
  // no CTA leaves while another may still read its part_ss
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One CTA per KV head (its two query heads) of one slot.  Exact two-pass
// softmax: scores of every position are kept in shared memory, then the
// row max, the LUT index, exp sum, per-index probabilities and sum(prob*v).
__global__ void __launch_bounds__(256) attn_step_kernel(SlotState st, int layer, const int32_t* __restrict__ exp_lut,
                                                        int64_t scale_q0_31) {
  extern __shared__ int64_t sc[];  // [2][ctx] scores, then LUT indices
  __shared__ int32_t q[2][kHeadDim];
  __shared__ uint64_t probtab[2][kExpLut];
  __shared__ int64_t red[8];
  __shared__ int64_t half_acc[2][kHeadDim];
  const int kv = blockIdx.x;
  grid_dep_wait();
  grid_dep_launch();
  if (*st.pos >= st.max_ctx) return;
  const int ctx = *st.pos + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < 2 * kHeadDim; i += blockDim.x) q[i / kHeadDim][i % kHeadDim] = st.qrope[2 * kv * kHeadDim + i];
  __syncthreads();
  for (int p = warp; p < ctx; p += nw) {
    const int4 k4 = reinterpret_cast<const int4*>(st.kv.at(layer, 0, kv, p))[lane];
    const int d = lane * 4;
    int64_t s0 = (int64_t)q[0][d] * k4.x + (int64_t)q[0][d + 1] * k4.y + (int64_t)q[0][d + 2] * k4.z +
                 (int64_t)q[0][d + 3] * k4.w;
    int64_t s1 = (int64_t)q[1][d] * k4.x + (int64_t)q[1][d + 1] * k4.y + (int64_t)q[1][d + 2] * k4.z +
                 (int64_t)q[1][d + 3] * k4.w;
    s0 = warp_sum_i64(s0);
    s1 = warp_sum_i64(s1);
    if (lane == 0) {
      sc[p] = scale_score(s0, scale_q0_31);
      sc[ctx + p] = scale_score(s1, scale_q0_31);
    }
  }
  __syncthreads();
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    int64_t* s = sc + h * ctx;
    int64_t mx = INT64_MIN;
    for (int p = threadIdx.x; p < ctx; p += blockDim.x) mx = s[p] > mx ? s[p] : mx;
    mx = block_max_i64(mx, red);
    int64_t sum = 0;
    for (int p = threadIdx.x; p < ctx; p += blockDim.x) {
      const int ix = lut_index(mx, s[p]);
      s[p] = ix;
      sum += exp_lut[ix];
    }
    sum = block_sum_i64(sum, red);
    for (int i = threadIdx.x; i < kExpLut; i += blockDim.x) probtab[h][i] = ((uint64_t)exp_lut[i] << 16) / (uint64_t)sum;
  }
  __syncthreads();
  const int d = threadIdx.x & (kHeadDim - 1);
  const int par = threadIdx.x >> 7;  // 0 or 1: even / odd positions
  int64_t acc0 = 0, acc1 = 0;
  for (int p = par; p < ctx; p += 2) {
    const int64_t v = st.kv.at(layer, 1, kv, p)[d];
    acc0 += (int64_t)probtab[0][sc[p]] * v;
    acc1 += (int64_t)probtab[1][sc[ctx + p]] * v;
  }
  if (par == 1) {
    half_acc[0][d] = acc0;
    half_acc[1][d] = acc1;
  }
  __syncthreads();
  if (par == 0) {
    acc0 += half_acc[0][d];
    acc1 += half_acc[1][d];
    st.attn[(2 * kv) * kHeadDim + d] = sat24(acc0 >> 16);
    st.attn[(2 * kv + 1) * kHeadDim + d] = sat24(acc1 >> 16);
  }
}

// o_proj (K = 2048) + residual: post = sat24(hidden + (sat24(q26 >> 14) >> 2)).
// 8 warps = 2 K-slices x 4 row groups of 2 rows -> 8 rows per CTA.
__global__ void __launch_bounds__(256) oproj_step_kernel(SlotState st, LayerW w) {
  constexpr int K = 2 * kHidden, R = 2, RPB = 8;
  __shared__ __align__(16) int32_t a[K];
  __shared__ __align__(16) uint32_t limbs[limb_words(K)];
  __shared__ int64_t bias8[K / 32];
  __shared__ int64_t part[2][RPB];
  const int row0 = blockIdx.x * RPB;
  if (threadIdx.x == 0) {
    prefetch_l2(w.wo + (size_t)row0 * (K / 2), RPB * (K / 2));
    prefetch_l2(w.so + (size_t)row0 * (K / 64), RPB * (K / 64) * 2);
  }
  grid_dep_wait();
  grid_dep_launch();
  for (int i = threadIdx.x; i < K; i += blockDim.x) a[i] = st.attn[i];
  __syncthreads();
  stage_limbs(a, K, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = warp & 1, rg = warp >> 1;
  int64_t acc[R] = {0, 0};
  gemv_slice<K, R>(w.wo, w.so, row0 + rg * R, kHidden, ks, limbs, bias8, acc);
  warp_reduce_rows<R>(acc);
  if (lane < R) part[ks][rg * R + lane] = acc[lane];
  __syncthreads();
  if (threadIdx.x < RPB) {
    const int r = row0 + threadIdx.x;
    const int32_t o = sat24((part[0][threadIdx.x] + part[1][threadIdx.x]) >> 14);
    st.post[r] = sat24((int64_t)st.hidden[r] + (o >> 2));
  }
}

// post-attention norm + gate/up + SwiGLU.  CTA: gate rows [r0, r0+16) by
// warps 0-3 and up rows [r0, r0+16) by warps 4-7.
__global__ void __launch_bounds__(256) gateup_step_kernel(SlotState st, LayerW w, const int32_t* __restrict__ sig_lut) {
  constexpr int R = 4, RPB = 16;
  __shared__ __align__(16) int32_t a[kHidden];
  __shared__ __align__(16) uint32_t limbs[limb_words(kHidden)];
  __shared__ int64_t bias8[kHidden / 32];
  __shared__ int64_t red[8];
  __shared__ int32_t gu[2][RPB];
  const int row0 = blockIdx.x * RPB;
  if (threadIdx.x == 0) {
    prefetch_l2(w.wgate + (size_t)row0 * 512, RPB * 512);
    prefetch_l2(w.wup + (size_t)row0 * 512, RPB * 512);
    prefetch_l2(w.sgate + (size_t)row0 * 16, RPB * 32);
    prefetch_l2(w.sup + (size_t)row0 * 16, RPB * 32);
  }
  grid_dep_wait();
  grid_dep_launch();
  hidden_norm_to(st.post, w.g_post, a, red);
  __syncthreads();
  stage_limbs(a, kHidden, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int which = warp >> 2;
  int64_t acc[R] = {0, 0, 0, 0};
  gemv_slice<kHidden, R>(which ? w.wup : w.wgate, which ? w.sup : w.sgate, row0 + (warp & 3) * R, kInter, 0, limbs,
                         bias8, acc);
  warp_reduce_rows<R>(acc);
  if (lane < R) gu[which][(warp & 3) * R + lane] = sat24(acc[lane] >> 14);
  __syncthreads();
  if (threadIdx.x < RPB) {
    const int32_t g = gu[0][threadIdx.x], u = gu[1][threadIdx.x];
    const int32_t gc = g < -32768 ? -32768 : (g > 32768 ? 32768 : g);
    int ix = (gc + 32768 + 32) >> 6;
    ix = ix > kSigLut - 1 ? kSigLut - 1 : ix;
    const int32_t silu = sat24(((int64_t)g * sig_lut[ix]) >> 16);
    st.mlp[row0 + threadIdx.x] = sat24(((int64_t)silu * u) >> 12);
  }
}

// down (K = 3072) + residual: hidden = sat24(post + (sat24(q26 >> 14) >> 2)).
// 6 warps = 3 K-slices x 2 row groups of 4 rows -> 8 rows per CTA.
__global__ void __launch_bounds__(192) down_step_kernel(SlotState st, LayerW w) {
  constexpr int K = kInter, R = 4, RPB = 8;
  __shared__ __align__(16) int32_t a[K];
  __shared__ __align__(16) uint32_t limbs[limb_words(K)];
  __shared__ int64_t bias8[K / 32];
  __shared__ int64_t part[3][RPB];
  const int row0 = blockIdx.x * RPB;
  if (threadIdx.x == 0) {
    prefetch_l2(w.wdown + (size_t)row0 * (K / 2), RPB * (K / 2));
    prefetch_l2(w.sdown + (size_t)row0 * (K / 64), RPB * (K / 64) * 2);
  }
  grid_dep_wait();
  grid_dep_launch();
  for (int i = threadIdx.x; i < K; i += blockDim.x) a[i] = st.mlp[i];
  __syncthreads();
  stage_limbs(a, K, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = warp % 3, rg = warp / 3;
  int64_t acc[R] = {0, 0, 0, 0};
  gemv_slice<K, R>(w.wdown, w.sdown, row0 + rg * R, kHidden, ks, limbs, bias8, acc);
  warp_reduce_rows<R>(acc);
  if (lane < R) part[ks][rg * R + lane] = acc[lane];
  __syncthreads();
  if (threadIdx.x < RPB) {
    const int r = row0 + threadIdx.x;
    const int32_t dn = sat24((part[0][threadIdx.x] + part[1][threadIdx.x] + part[2][threadIdx.x]) >> 14);
    st.hidden[r] = sat24((int64_t)st.post[r] + (dn >> 2));
  }
}

__device__ __forceinline__ bool better_d(int64_t s, int32_t i, int64_t bs, int32_t bi) {
  return s > bs || (s == bs && i < bi);
}

// Final norm + tied LM head + exact argmax; writes tokens[pos+1],
// scores[pos+1] and advances pos.  Persistent grid over row blocks.
__global__ void __launch_bounds__(256) lmhead_step_kernel(SlotState st, const uint8_t* __restrict__ W,
                                                          const uint16_t* __restrict__ S, int rows,
                                                          const int32_t* __restrict__ g_final) {
  constexpr int R = 4;
  __shared__ __align__(16) int32_t a[kHidden];
  __shared__ __align__(16) uint32_t limbs[limb_words(kHidden)];
  __shared__ int64_t bias8[kHidden / 32];
  __shared__ int64_t red[8];
  __shared__ ArgBestD wbest[8];
  __shared__ bool last;
  grid_dep_wait();
  grid_dep_launch();
  const int pos = *st.pos;
  if (pos >= st.max_ctx) return;
  hidden_norm_to(st.hidden, g_final, a, red);
  __syncthreads();
  stage_limbs(a, kHidden, limbs, bias8);
  __syncthreads();
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int64_t best_s = INT64_MIN;
  int32_t best_i = INT32_MAX;
  for (int base = (blockIdx.x * nw + warp) * R; base < rows; base += gridDim.x * nw * R) {
    int64_t acc[R] = {0, 0, 0, 0};
    gemv_slice<kHidden, R>(W, S, base, rows, 0, limbs, bias8, acc);
    warp_reduce_rows<R>(acc);
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (base + r < rows && acc[r] > best_s) {
        best_s = acc[r];
        best_i = base + r;
      }
  }
  if ((threadIdx.x & 31) == 0) wbest[warp] = ArgBestD{best_s, best_i, 0};
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgBestD b = wbest[0];
    for (int i = 1; i < nw; ++i)
      if (better_d(wbest[i].score, wbest[i].idx, b.score, b.idx)) b = wbest[i];
    st.lm_partial[blockIdx.x] = b;
    __threadfence();
    last = atomicAdd(st.lm_counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    ArgBestD b = st.lm_partial[0];
    for (int i = 1; i < (int)gridDim.x; ++i) {
      const ArgBestD c{*((volatile int64_t*)&st.lm_partial[i].score), *((volatile int32_t*)&st.lm_partial[i].idx), 0};
      if (better_d(c.score, c.idx, b.score, b.idx)) b = c;
    }
    st.tokens[pos + 1] = b.idx;
    st.scores[pos + 1] = b.score;
    *st.pos = pos + 1;
    *st.lm_counter = 0;
  }
}

__global__ void advance_step_kernel(SlotState st) {
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x == 0 && *st.pos < st.max_ctx) *st.pos += 1;
}

__global__ void set_pos_kernel(SlotState st, int position) {
  grid_dep_wait();
  grid_dep_launch();
  if (threadIdx.x == 0) *st.pos = position;
}

// Scatter a KV pool page range to/from the reference order [pos][head][128].
__global__ void kv_copy_kernel(KvView kv, int layer, int kind, int positions, int32_t* flat, int to_pool) {
  const int p = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  if (p >= positions) return;
  int32_t* slot = kv.at(layer, kind, h, p) + d;
  int32_t* f = flat + ((size_t)p * kKvHeads + h) * kHeadDim + d;
  if (to_pool) {
    *slot = *f;
    if (kind == 0)
      kpl_put1(kv, layer, h, p, d, *f);
    else
      vpl_put1(kv, layer, h, p, d, *f);
  } else {
    *f = *slot;
  }
}

}  // namespace q4

// ===========================================================================
// Host runtime
// ===========================================================================
using namespace q4;

namespace {
thread_local std::string g_last_error = "no error";
}

int q4gpu_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  // the failing runtime call is reported here: consume the runtime's record of
  // it, so a later launch check does not report it again
  if (code == Q4GPU_ERR_CUDA) (void)cudaGetLastError();
  return code;
}

int q4gpu_check_launch() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "CUDA launch failed: %s", cudaGetErrorString(e));
  return Q4GPU_OK;
}

#define Q4_CUDA(call)                                                                                  \
  do {                                                                                                 \
    const cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

struct q4gpu_model;
// A host <-> device copy that the model stream's kernels depend on: ordered on
// that stream and finished before returning.  (A plain cudaMemcpy runs on the
// legacy stream, which does not order against the non-blocking model stream,
// and a pageable host-to-device cudaMemcpy may return before its DMA lands.)
int stream_copy(q4gpu_model* m, void* dst, const void* src, size_t n, cudaMemcpyKind kind);

namespace {

constexpr int kMaxLayers = 28;

struct GraphKey {
  int slot, layer_start, layer_count, embed, tail;
  bool operator<(const GraphKey& o) const {
    return std::tie(slot, layer_start, layer_count, embed, tail) <
           std::tie(o.slot, o.layer_start, o.layer_count, o.embed, o.tail);
  }
};

struct HostResult {
  int32_t token;
  int32_t pos;
  int64_t score;
};

}  // namespace

struct q4gpu_model {
  q4gpu_model_config cfg{};
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  // weights
  LayerW layers[kMaxLayers]{};
  uint8_t* w_layers = nullptr;  // per layer: qkv, o, gate, up, down (packed)
  uint16_t* s_layers = nullptr;
  int32_t* gammas = nullptr;  // per layer: in[1024], post[1024], q[128], k[128]
  uint8_t* emb = nullptr;
  uint16_t* semb = nullptr;
  int32_t* g_final = nullptr;
  int32_t* cos_tab = nullptr;
  int32_t* sin_tab = nullptr;
  int32_t* exp_lut = nullptr;
  int32_t* sig_lut = nullptr;
  // KV pool
  int32_t* kv_pool = nullptr;
  int64_t page_elems = 0;
  uint8_t* kv_planes = nullptr;  // the keys as byte planes (KvView::kpl)
  uint8_t* v_planes = nullptr;   // the values as transposed byte planes (KvView::vpl)
  int64_t kpl_page_bytes = 0;
  int pages_per_seq = 0;
  int32_t* page_tables = nullptr;
  // slots
  std::vector<SlotState> slots;
  HostResult* h_res = nullptr;  // pinned, one per slot
  int32_t* h_in = nullptr;      // pinned staging: [token, pos] per slot
  std::vector<cudaEvent_t> done;
  std::vector<int> busy;
  std::map<GraphKey, cudaGraphExec_t> graphs;
  // persistent decode kernel (mode 1)
  int mode = 0;
  int p_grid = 0;
  size_t p_smem = 0;
  LayerW* layers_dev = nullptr;
  int32_t* p_qkv = nullptr;
  int64_t* p_acc = nullptr;
  ArgBestD* p_lm_part = nullptr;
  unsigned int* p_bar = nullptr;
  int* p_err = nullptr;      // set by the persistent kernel or the stage path's cluster attention
  bool stage_attn_cl = false;  // the per-stage path runs its attention on clusters (stage_attn_cl_kernel)
  CUtensorMap vmap{};
  // batched decode (q4_batch.cu), set up on first use
  bool b_ready = false;       // batched buffers and the TMA maps of the packed weights set up
  int32_t* b_qkv = nullptr;
  uint8_t* b_bt1 = nullptr;
  uint8_t* b_bt2 = nullptr;
  uint8_t* b_bt3 = nullptr;
  SlotState* b_slots = nullptr;  // device copy of slots
  int32_t* b_lm_from = nullptr;  // [max_seqs]
  ArgBestD* b_lm_part = nullptr;
  int32_t* b_io = nullptr;   // device [64][2] inputs, then [64][4] outputs
  int32_t* h_bio = nullptr;  // pinned mirror of b_io
  int* b_err = nullptr;      // set by a batched kernel whose pipeline wait ran out
  int64_t* b_att_S = nullptr;  // split-KV attention scratch
  uint32_t* b_att_P = nullptr;
  int64_t* b_att_M = nullptr;
  int64_t* b_att_O = nullptr;
  unsigned* b_att_cnt = nullptr;  // [2][64][8]
  CUtensorMap b_mlm{};       // TMA map of the packed embedding (the tied LM head)
  BatchLayerW b_layers[kMaxLayers]{};
  bool p_stale = true;  // the persistent kernel's o_proj slices out of date
  uint8_t* p_wo_sl = nullptr;
  uint16_t* p_so_sl = nullptr;
  int b_pad_sp = 0;     // SP whose zero padding rows the B matrices hold
  std::map<std::tuple<int, int, int>, cudaGraphExec_t> b_graphs;  // (first slot, S, hidden-only)
  int32_t* b_final_act = nullptr;   // [64, 1024] final-norm vectors of a hidden-only step
  uint8_t* b_lm_bt = nullptr;       // limb matrix of a vocabulary-shard LM head
  ArgBestD* b_lm_shard_part = nullptr;
  int b_lm_pad_sp = 0;
  // batched exact prefill (q4gpu_batch_prefill)
  int prefill_mode = 1;          // 1: batched prefill in q4gpu_decode_batch; 0: serial, position by position
  PrefillPlan* pf = nullptr;     // buffers and TMA maps; per-block fields set per launch
  SlotState* pf_cols = nullptr;  // [pf_cap] column -> its sequence's state
  int32_t* pf_pos4 = nullptr;    // [pf_cap][4]
  PfTile* pf_tiles = nullptr;    // [pf_tile_cap]
  size_t pf_cap = 0, pf_tile_cap = 0;

  template <class T>
  int alloc(T** p, size_t count) {
    void* v = nullptr;
    Q4_CUDA(cudaMalloc(&v, count * sizeof(T) + 256));
    // zeroed on the model stream (a plain cudaMemset runs on the legacy
    // stream, which does not order against the non-blocking model stream)
    Q4_CUDA(cudaMemsetAsync(v, 0, count * sizeof(T) + 256, stream));
    Q4_CUDA(cudaStreamSynchronize(stream));
    allocs.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return Q4GPU_OK;
  }
};

int stream_copy(q4gpu_model* m, void* dst, const void* src, size_t n, cudaMemcpyKind kind) {
  Q4_CUDA(cudaMemcpyAsync(dst, src, n, kind, m->stream));
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  return Q4GPU_OK;
}

namespace {

constexpr size_t kQkvBytes = (size_t)(kQRows + 2 * kKvRows) * 512;
constexpr size_t kOBytes = (size_t)kHidden * 1024;
constexpr size_t kGateBytes = (size_t)kInter * 512;
constexpr size_t kDownBytes = (size_t)kHidden * 1536;
constexpr size_t kLayerWBytes = kQkvBytes + kOBytes + 2 * kGateBytes + kDownBytes;
constexpr size_t kQkvScales = (size_t)(kQRows + 2 * kKvRows) * 16;
constexpr size_t kOScales = (size_t)kHidden * 32;
constexpr size_t kGateScales = (size_t)kInter * 16;
constexpr size_t kDownScales = (size_t)kHidden * 48;
constexpr size_t kLayerScales = kQkvScales + kOScales + 2 * kGateScales + kDownScales;
constexpr size_t kLayerGammas = 2 * kHidden + 2 * kHeadDim;

// (packed pointer, scale pointer, rows, cols) of one weight tensor
struct TensorRef {
  uint8_t* w;
  uint16_t* s;
  int64_t rows;
  int cols;
};

TensorRef layer_tensor(q4gpu_model* m, int layer, int which) {
  uint8_t* w = m->w_layers + (size_t)layer * kLayerWBytes;
  uint16_t* s = m->s_layers + (size_t)layer * kLayerScales;
  switch (which) {
    case Q4GPU_T_Q: return {w, s, kQRows, kHidden};
    case Q4GPU_T_K: return {w + (size_t)kQRows * 512, s + (size_t)kQRows * 16, kKvRows, kHidden};
    case Q4GPU_T_V:
      return {w + (size_t)(kQRows + kKvRows) * 512, s + (size_t)(kQRows + kKvRows) * 16, kKvRows, kHidden};
    case Q4GPU_T_O: return {w + kQkvBytes, s + kQkvScales, kHidden, 2 * kHidden};
    case Q4GPU_T_GATE: return {w + kQkvBytes + kOBytes, s + kQkvScales + kOScales, kInter, kHidden};
    case Q4GPU_T_UP:
      return {w + kQkvBytes + kOBytes + kGateBytes, s + kQkvScales + kOScales + kGateScales, kInter, kHidden};
    case Q4GPU_T_DOWN:
      return {w + kQkvBytes + kOBytes + 2 * kGateBytes, s + kQkvScales + kOScales + 2 * kGateScales, kHidden, kInter};
    default: return {nullptr, nullptr, 0, 0};
  }
}

int32_t* layer_gamma(q4gpu_model* m, int layer, int which, int* n) {
  int32_t* g = m->gammas + (size_t)layer * kLayerGammas;
  switch (which) {
    case Q4GPU_T_INPUT_GAMMA: *n = kHidden; return g;
    case Q4GPU_T_POST_GAMMA: *n = kHidden; return g + kHidden;
    case Q4GPU_T_Q_GAMMA: *n = kHeadDim; return g + 2 * kHidden;
    case Q4GPU_T_K_GAMMA: *n = kHeadDim; return g + 2 * kHidden + kHeadDim;
    default: *n = 0; return nullptr;
  }
}

// exp LUT (257 x UQ0.20) and sigmoid LUT (1025 x UQ0.16); round-half-even on
// the double value as Python's round() does.
void build_luts(int32_t* exp_lut, int32_t* sig_lut) {
  for (int i = 0; i < kExpLut; ++i) exp_lut[i] = (int32_t)std::nearbyint(std::exp(-(double)i / 16.0) * 1048576.0);
  for (int i = 0; i < kSigLut; ++i) {
    const double x = -8.0 + (double)i / 64.0;
    double y = std::nearbyint(1.0 / (1.0 + std::exp(-x)) * 65536.0);
    y = y < 0 ? 0 : (y > 65535 ? 65535 : y);
    sig_lut[i] = (int32_t)y;
  }
}

// HF default RoPE inverse frequencies for head_dim 128, theta 1e6, as the
// float32 values 1 / (1e6 ** (2i / 128)) that torch produces (torch's float32
// pow differs from libm powf in the last bit for some i, so the values are
// data here, not recomputed).
constexpr float kInvFreq[64] = {
    0x1.0000000000000p+0f, 0x1.9c975a0000000p-1f, 0x1.4c7bc00000000p-1f, 0x1.0bedde0000000p-1f,
    0x1.afd1360000000p-2f, 0x1.5bf9fe0000000p-2f, 0x1.186a080000000p-2f, 0x1.c3f06a0000000p-3f,
    0x1.6c310e0000000p-3f, 0x1.257b220000000p-3f, 0x1.d8ffac0000000p-4f, 0x1.7d298c0000000p-4f,
    0x1.33281a0000000p-4f, 0x1.ef0a260000000p-5f, 0x1.8eec7e0000000p-5f, 0x1.41783a0000000p-5f,
    0x1.030dc60000000p-5f, 0x1.a183500000000p-6f, 0x1.5073160000000p-6f, 0x1.0f20100000000p-6f,
    0x1.b4f7e40000000p-7f, 0x1.6020a40000000p-7f, 0x1.1bc25a0000000p-7f, 0x1.c9548c0000000p-8f,
    0x1.7089380000000p-8f, 0x1.28fb5c0000000p-8f, 0x1.dea41c0000000p-9f, 0x1.81b58a0000000p-9f,
    0x1.36d21a0000000p-9f, 0x1.f4f1e00000000p-10f, 0x1.93aeb80000000p-10f, 0x1.454dee0000000p-10f,
    0x1.0624de0000000p-10f, 0x1.a67e500000000p-11f, 0x1.5476880000000p-11f, 0x1.125c040000000p-11f,
    0x1.ba2e4a0000000p-12f, 0x1.6453f60000000p-12f, 0x1.1f24e40000000p-12f, 0x1.cec9240000000p-13f,
    0x1.74eea60000000p-13f, 0x1.2c86480000000p-13f, 0x1.e459c40000000p-14f, 0x1.864f6a0000000p-14f,
    0x1.3a87480000000p-14f, 0x1.faeba80000000p-15f, 0x1.987f7c0000000p-15f, 0x1.492f560000000p-15f,
    0x1.0945640000000p-15f, 0x1.ab88820000000p-16f, 0x1.58863a0000000p-16f, 0x1.15a1da0000000p-16f,
    0x1.bf749e0000000p-17f, 0x1.68941c0000000p-17f, 0x1.2291c60000000p-17f, 0x1.d44e640000000p-18f,
    0x1.7961820000000p-18f, 0x1.301c040000000p-18f, 0x1.ea20e00000000p-19f, 0x1.8af7560000000p-19f,
    0x1.3e47c80000000p-19f, 0x1.007bd80000000p-19f, 0x1.9d5ef20000000p-20f, 0x1.4d1c980000000p-20f};

// Q1.15 RoPE table: freqs and cos/sin in float32, rint(x * 2^15) clipped.
void build_rope(int positions, int32_t* cos_t, int32_t* sin_t) {
  const float* inv = kInvFreq;
  for (int p = 0; p < positions; ++p)
    for (int d = 0; d < kHeadDim; ++d) {
      const float f = inv[d & 63] * (float)p;
      double c = std::nearbyint((double)std::cos(f) * 32768.0), s = std::nearbyint((double)std::sin(f) * 32768.0);
      c = c > 32767 ? 32767 : (c < -32768 ? -32768 : c);
      s = s > 32767 ? 32767 : (s < -32768 ? -32768 : s);
      cos_t[p * kHeadDim + d] = (int32_t)c;
      sin_t[p * kHeadDim + d] = (int32_t)s;
    }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, Args... args) {
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

// The same with thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_kc(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t s, int cluster_x, Args... args) {
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

size_t attn_smem(int max_ctx) { return (size_t)2 * max_ctx * sizeof(int64_t); }

// Per-kernel event marks for q4gpu_model_time_kernels (kinds as in q4gpu.h).
struct KernelMarks {
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  int mark(cudaStream_t s, int k) {
    cudaEvent_t e;
    Q4_CUDA(cudaEventCreate(&e));
    ev.push_back(e);
    kind.push_back(k);
    Q4_CUDA(cudaEventRecord(e, s));
    return Q4GPU_OK;
  }
  ~KernelMarks() {
    for (auto e : ev) cudaEventDestroy(e);
  }
};

// Enqueue one step of `slot` (no capture logic here).  With `marks`, an
// event is recorded before every kernel and after the last one.
int enqueue_step(q4gpu_model* m, int slot, int layer_start, int layer_count, int embed, int tail,
                 KernelMarks* marks = nullptr) {
  const SlotState& st = m->slots[slot];
  cudaStream_t s = m->stream;
  auto mark = [&](int k) { return marks ? marks->mark(s, k) : Q4GPU_OK; };
  int rc;
  if (embed) {
    if ((rc = mark(Q4GPU_K_EMBED))) return rc;
    Q4_CUDA(launch_k(embed_step_kernel, dim3(1), dim3(256), 0, s, st, (const uint8_t*)m->emb,
                     (const uint16_t*)m->semb));
  }
  const int64_t scale = 189812531LL;  // round(128^-0.5 * 2^31)
  for (int l = layer_start; l < layer_start + layer_count; ++l) {
    const LayerW& w = m->layers[l];
    if ((rc = mark(Q4GPU_K_QKV))) return rc;
    Q4_CUDA(launch_kc(qkv_step_kernel, dim3((kQHeads + 2 * kKvHeads) * kQkvRanks), dim3(256), 0, s, kQkvRanks, st, w,
                      l, (const int32_t*)m->cos_tab, (const int32_t*)m->sin_tab));
    if ((rc = mark(Q4GPU_K_ATTN))) return rc;
    if (m->stage_attn_cl) {
      if ((rc = q4gpu_enqueue_stage_attention(st, m->p_err, l, (const int32_t*)m->exp_lut, m->cfg.max_context, s)))
        return rc;
    } else {
      Q4_CUDA(launch_k(attn_step_kernel, dim3(kKvHeads), dim3(256), attn_smem(m->cfg.max_context), s, st, l,
                       (const int32_t*)m->exp_lut, scale));
    }
    if ((rc = mark(Q4GPU_K_OPROJ))) return rc;
    Q4_CUDA(launch_k(oproj_step_kernel, dim3(kHidden / 8), dim3(256), 0, s, st, w));
    if ((rc = mark(Q4GPU_K_GATEUP))) return rc;
    Q4_CUDA(launch_k(gateup_step_kernel, dim3(kInter / 16), dim3(256), 0, s, st, w, (const int32_t*)m->sig_lut));
    if ((rc = mark(Q4GPU_K_DOWN))) return rc;
    Q4_CUDA(launch_k(down_step_kernel, dim3(kHidden / 8), dim3(192), 0, s, st, w));
  }
  if (tail) {
    if ((rc = mark(Q4GPU_K_LMHEAD))) return rc;
    Q4_CUDA(launch_k(lmhead_step_kernel, dim3(Q4GPU_LM_HEAD_BLOCKS), dim3(256), 0, s, st, (const uint8_t*)m->emb,
                     (const uint16_t*)m->semb, m->cfg.vocab, (const int32_t*)m->g_final));
  } else {
    if ((rc = mark(Q4GPU_K_ADVANCE))) return rc;
    Q4_CUDA(launch_k(advance_step_kernel, dim3(1), dim3(32), 0, s, st));
  }
  return mark(-1);
}

// 2-D tensor map over the KV pool for the persistent kernel's V-slice loads:
// rows of 128 int32 (one position of one (page, layer, kind, head)), box of
// 64 positions x 16 dims.
int encode_kv_map(q4gpu_model* m, int64_t n_pages) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !encode)
    return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t rows = (cuuint64_t)n_pages * m->cfg.n_layers * 2 * kKvHeads * kKvPage;
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 4};
  const cuuint32_t box[2] = {16, (cuuint32_t)kKvPage};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(&m->vmap, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, m->kv_pool, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return q4gpu_fail(Q4GPU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q4GPU_OK;
}

// n_steps decode steps of `slot` in one persistent launch, continuing from
// the slot's device position; the LM head runs where p + 1 >= lm_from.
int run_persistent(q4gpu_model* m, int slot, int n_steps, int lm_from, unsigned long long* trace = nullptr,
                   int trace_cap = 0) {
  if (n_steps <= 0) return Q4GPU_OK;
  if (m->p_stale) {
    const int rc = q4gpu_persistent_relayout(m->layers_dev, m->cfg.n_layers, m->stream);
    if (rc != Q4GPU_OK) return rc;
    m->p_stale = false;
  }
  PersistArgs a{};
  a.vmap = m->vmap;
  a.st = m->slots[slot];
  a.layers = m->layers_dev;
  a.n_layers = m->cfg.n_layers;
  a.emb = m->emb;
  a.semb = m->semb;
  a.vocab = m->cfg.vocab;
  a.g_final = m->g_final;
  a.cos_tab = m->cos_tab;
  a.sin_tab = m->sin_tab;
  a.exp_lut = m->exp_lut;
  a.sig_lut = m->sig_lut;
  a.qkv = m->p_qkv;
  a.acc = m->p_acc;
  a.lm_part = m->p_lm_part;
  a.bar = m->p_bar;
  a.err = m->p_err;
  a.n_steps = n_steps;
  a.lm_from = lm_from;
  a.score_cap = m->cfg.max_context;
  a.trace = trace;
  a.trace_cap = trace_cap;
  // the arrival counter of one launch counts (3 L + 1) G per step: split very
  // long runs so it stays below 2^32
  const int per_launch = (int)std::min<int64_t>(
      (int64_t)0xF0000000 / ((int64_t)m->p_grid * (3 * m->cfg.n_layers + 1)), 1 << 20);
  int rc = Q4GPU_OK;
  for (int done = 0; done < n_steps && rc == Q4GPU_OK; done += per_launch) {
    a.n_steps = std::min(per_launch, n_steps - done);
    Q4_CUDA(cudaMemsetAsync(m->p_bar, 0, 2 * sizeof(unsigned int), m->stream));
    Q4_CUDA(cudaMemsetAsync(m->p_acc, 0, 16 * kHidden * sizeof(int64_t), m->stream));
    rc = q4gpu_launch_persistent(a, m->p_grid, m->p_smem, m->stream);
    a.trace = nullptr;
  }
  return rc;
}

int check_persistent_error(q4gpu_model* m) {
  if (!m->p_err) return Q4GPU_OK;
  int e = 0;
  Q4_CUDA(cudaMemcpy(&e, m->p_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemsetAsync(m->p_err, 0, sizeof(int), m->stream);
    return q4gpu_fail(Q4GPU_ERR_CUDA, e == 2   ? "persistent decode kernel: stepped past max_context"
                                      : e == 4 ? "attention stage: a K/V copy wait ran out"
                                               : "persistent decode kernel: a grid barrier wait ran out");
  }
  return Q4GPU_OK;
}

int get_graph(q4gpu_model* m, const GraphKey& k, cudaGraphExec_t* out) {
  auto it = m->graphs.find(k);
  if (it != m->graphs.end()) {
    *out = it->second;
    return Q4GPU_OK;
  }
  cudaGraph_t g = nullptr;
  Q4_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  const int rc = enqueue_step(m, k.slot, k.layer_start, k.layer_count, k.embed, k.tail);
  const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
  if (rc != Q4GPU_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
  cudaGraphExec_t e = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
  m->graphs[k] = e;
  *out = e;
  return Q4GPU_OK;
}

int set_device(q4gpu_model* m) {
  Q4_CUDA(cudaSetDevice(m->cfg.device));
  return Q4GPU_OK;
}

// Wait for the slot's last work, polling at most max_polls times (0 = block).
int poll_slot(q4gpu_model* m, int slot, uint32_t max_polls) {
  if (max_polls == 0) {
    if (cudaEventSynchronize(m->done[slot]) != cudaSuccess) return QOT_ERR_STATUS;
    m->busy[slot] = 0;
    return QOT_OK;
  }
  for (uint32_t i = 0; i < max_polls; ++i) {
    const cudaError_t e = cudaEventQuery(m->done[slot]);
    if (e == cudaSuccess) {
      m->busy[slot] = 0;
      return QOT_OK;
    }
    if (e != cudaErrorNotReady) return QOT_ERR_STATUS;
  }
  return QOT_ERR_TIMEOUT;
}

bool slot_busy(q4gpu_model* m, int slot) {
  if (!m->busy[slot]) return false;
  if (cudaEventQuery(m->done[slot]) == cudaSuccess) m->busy[slot] = 0;
  return m->busy[slot] != 0;
}

uint64_t step_bytes(const q4gpu_model* m, int layers, int ctx, int tail) {
  const uint64_t per_layer = kLayerWBytes + 2 * kLayerScales + (uint64_t)2 * kKvRows * 4 * ctx;
  return per_layer * layers + (tail ? (uint64_t)m->cfg.vocab * (512 + 32) : 0);
}

// ---- batched decode (q4_batch.cu) ------------------------------------------
constexpr int kBtRows = 3 * kBatchSeqMax + kBatchPad;

int batch_lm_ctas(int vocab) { return (vocab + 127) / 128; }

// Allocate the batched-decode buffers and encode the TMA maps of the packed
// weights once (the maps address the model's own Q4 tensors, so later weight
// uploads need nothing here).
int batch_prepare(q4gpu_model* m) {
  if (m->cfg.vocab < 64) return q4gpu_fail(Q4GPU_ERR_SHAPE, "batched decode needs a vocabulary of at least 64");
  if (m->b_ready) return Q4GPU_OK;
  const int L = m->cfg.n_layers;
  int rc;
  if ((rc = m->alloc(&m->b_qkv, (size_t)kBatchSeqMax * (kQRows + 2 * kKvRows)))) return rc;
  if ((rc = m->alloc(&m->b_bt1, (size_t)kBtRows * kHidden))) return rc;
  if ((rc = m->alloc(&m->b_bt2, (size_t)kBtRows * 2 * kHidden))) return rc;
  if ((rc = m->alloc(&m->b_bt3, (size_t)kBtRows * kInter))) return rc;
  if ((rc = m->alloc(&m->b_slots, m->slots.size()))) return rc;
  if ((rc = stream_copy(m, m->b_slots, m->slots.data(), sizeof(SlotState) * m->slots.size(), cudaMemcpyHostToDevice)))
    return rc;
  if ((rc = m->alloc(&m->b_lm_from, (size_t)m->cfg.max_seqs))) return rc;
  if ((rc = m->alloc(&m->b_lm_part, (size_t)batch_lm_ctas(m->cfg.vocab) * kBatchSeqMax))) return rc;
  if ((rc = m->alloc(&m->b_io, (size_t)kBatchSeqMax * 6))) return rc;
  if ((rc = m->alloc(&m->b_err, 4))) return rc;
  if ((rc = m->alloc(&m->b_final_act, (size_t)kBatchSeqMax * kHidden))) return rc;
  if ((rc = m->alloc(&m->b_lm_bt, (size_t)kBtRows * kHidden))) return rc;
  if ((rc = m->alloc(&m->b_lm_shard_part, (size_t)batch_lm_ctas(m->cfg.vocab) * kBatchSeqMax))) return rc;
  const size_t sp = (size_t)kBatchSeqMax * kQHeads * m->cfg.max_context;
  if ((rc = m->alloc(&m->b_att_S, sp))) return rc;
  if ((rc = m->alloc(&m->b_att_P, sp))) return rc;
  if ((rc = m->alloc(&m->b_att_M, (size_t)kBatchSeqMax * kQHeads))) return rc;
  if ((rc = m->alloc(&m->b_att_O, (size_t)kBatchSeqMax * kQHeads * kHeadDim))) return rc;
  if ((rc = m->alloc(&m->b_att_cnt, (size_t)2 * kBatchSeqMax * kKvHeads))) return rc;
  {
    std::vector<int64_t> armed((size_t)kBatchSeqMax * kQHeads, INT64_MIN);
    if ((rc = stream_copy(m, m->b_att_M, armed.data(), armed.size() * 8, cudaMemcpyHostToDevice))) return rc;
  }
  Q4_CUDA(cudaMallocHost(&m->h_bio, (size_t)kBatchSeqMax * 6 * sizeof(int32_t)));
  for (int l = 0; l < L; ++l) {
    const LayerW& q = m->layers[l];
    BatchLayerW& b = m->b_layers[l];
    b.wqkv = q.wqkv;
    b.wo = q.wo;
    b.wgate = q.wgate;
    b.wup = q.wup;
    b.wdown = q.wdown;
    b.sqkv = q.sqkv;
    b.so = q.so;
    b.sgate = q.sgate;
    b.sup = q.sup;
    b.sdown = q.sdown;
    b.g_in = q.g_in;
    b.g_post = q.g_post;
    b.g_q = q.g_q;
    b.g_k = q.g_k;
    if ((rc = q4gpu_encode_q4_map(&b.mqkv, q.wqkv, kHidden / 2, kQRows + 2 * kKvRows, 128)) ||
        (rc = q4gpu_encode_q4_map(&b.mo, q.wo, kHidden, kHidden, 128)) ||
        (rc = q4gpu_encode_q4_map(&b.mgate, q.wgate, kHidden / 2, kInter, 64)) ||
        (rc = q4gpu_encode_q4_map(&b.mup, q.wup, kHidden / 2, kInter, 64)) ||
        (rc = q4gpu_encode_q4_map(&b.mdown, q.wdown, kInter / 2, kHidden, 128)))
      return rc;
  }
  if ((rc = q4gpu_encode_q4_map(&m->b_mlm, m->emb, kHidden / 2, (uint64_t)m->cfg.vocab, 128))) return rc;
  m->b_ready = true;
  return Q4GPU_OK;
}

int batch_plan(q4gpu_model* m, int first, int S, BatchPlan& p) {
  p = BatchPlan{};
  p.slots = m->b_slots + first;
  p.S = S;
  p.SP = q4gpu_batch_padded(S);
  p.qkv_raw = m->b_qkv;
  p.bt1 = m->b_bt1;
  p.bt2 = m->b_bt2;
  p.bt3 = m->b_bt3;
  p.lm_from = m->b_lm_from + first;
  p.emb = m->emb;
  p.semb = m->semb;
  p.layers = m->b_layers;
  p.n_layers = m->cfg.n_layers;
  p.max_ctx = m->cfg.max_context;
  p.kv_planes = m->kv_planes != nullptr;
  p.vocab = m->cfg.vocab;
  p.cos_tab = m->cos_tab;
  p.sin_tab = m->sin_tab;
  p.exp_lut = m->exp_lut;
  p.sig_lut = m->sig_lut;
  p.g_final = m->g_final;
  p.lm_partial = m->b_lm_part;
  p.err = m->b_err;
  p.pos0 = m->slots[first].pos;
  p.hidden0 = m->slots[first].hidden;
  p.post0 = m->slots[first].post;
  p.att_S = m->b_att_S;
  p.att_P = m->b_att_P;
  p.att_M = m->b_att_M;
  p.att_O = m->b_att_O;
  p.att_cnt_s = m->b_att_cnt;
  p.att_cnt_v = m->b_att_cnt + kBatchSeqMax * kKvHeads;
  p.mlm = m->b_mlm;
  // limb boxes of each GEMM's sequence chunk, its three limb blocks (kinds: 0 q/k/v, 1 o_proj, 2 gate/up, 3 down, 4 LM head)
  const uint64_t nrows = (uint64_t)q4gpu_batch_limb_rows(p.SP);
  auto box = [&](int kind) { return (uint32_t)(3 * q4gpu_batch_gemm_chunk(kind, p.SP)); };
  int rc;
  if ((rc = q4gpu_encode_u8_map(&p.mb_qkv, p.bt1, kHidden, nrows, box(0))) ||
      (rc = q4gpu_encode_u8_map(&p.mb_o, p.bt2, 2 * kHidden, nrows, box(1))) ||
      (rc = q4gpu_encode_u8_map(&p.mb_gu, p.bt1, kHidden, nrows, box(2))) ||
      (rc = q4gpu_encode_u8_map(&p.mb_down, p.bt3, kInter, nrows, box(3))) ||
      (rc = q4gpu_encode_u8_map(&p.mb_lm, p.bt1, kHidden, nrows, box(4))))
    return rc;
  return Q4GPU_OK;
}

// Prefill buffers and maps, once per model (64-column GEMMs, 192 limb rows per sub-batch).
int prefill_prepare(q4gpu_model* m) {
  if (m->pf) return Q4GPU_OK;
  int rc;
  static bool attrs = false;
  if (!attrs) {
    if ((rc = q4gpu_prefill_setup())) return rc;
    attrs = true;
  }
  auto p = std::make_unique<PrefillPlan>();
  const size_t rows = (size_t)kPfSubRows;  // 192 limb rows per 64-column sub-batch
  constexpr int nsub = kPfBlock / kPfSub;
  if ((rc = m->alloc(&p->hidden, (size_t)kPfBlock * kHidden)) || (rc = m->alloc(&p->post, (size_t)kPfBlock * kHidden)) ||
      (rc = m->alloc(&p->qkv, (size_t)kPfBlock * (kQRows + 2 * kKvRows))) ||
      (rc = m->alloc(&p->bt1, nsub * rows * kHidden)) || (rc = m->alloc(&p->bt2, nsub * rows * 2 * kHidden)) ||
      (rc = m->alloc(&p->bt3, nsub * rows * kInter)) ||
      (rc = m->alloc(&p->lut_idx, (size_t)kPfBlock * kQHeads * ((m->cfg.max_context + 63) / 64 * 64))))
    return rc;
  // boxes of the three limbs of one 64-column sub-batch
  if ((rc = q4gpu_encode_u8_map(&p->mb1, p->bt1, kHidden, nsub * rows, (uint32_t)(3 * kPfSub))) ||
      (rc = q4gpu_encode_u8_map(&p->mb2, p->bt2, 2 * kHidden, nsub * rows, (uint32_t)(3 * kPfSub))) ||
      (rc = q4gpu_encode_u8_map(&p->mb3, p->bt3, kInter, nsub * rows, (uint32_t)(3 * kPfSub))))
    return rc;
  p->emb = m->emb;
  p->semb = m->semb;
  p->layers = m->b_layers;
  p->n_layers = m->cfg.n_layers;
  p->max_ctx = m->cfg.max_context;
  p->cos_tab = m->cos_tab;
  p->sin_tab = m->sin_tab;
  p->exp_lut = m->exp_lut;
  p->sig_lut = m->sig_lut;
  p->err = m->b_err;
  m->pf = p.release();
  return Q4GPU_OK;
}

// Prefill of slots [first, first + S): the tokens at positions 0 .. len - 2 of
// each slot (already in the slot's token array) go through every layer as
// columns of batched passes, leaving the K/V cache exactly as serial decode
// steps over those positions would.  Positions are set to len - 1, so the next
// batched step runs the last prompt token.  Stream-ordered on the model stream.
int batch_prefill(q4gpu_model* m, int first, int S, const uint32_t* lens) {
  int rc;
  if ((rc = batch_prepare(m)) || (rc = prefill_prepare(m))) return rc;
  std::vector<SlotState> cols;
  std::vector<int32_t> pos4;
  for (int i = 0; i < S; ++i) {
    if (lens[i] < 1u || lens[i] > (uint32_t)m->cfg.max_context)
      return q4gpu_fail(Q4GPU_ERR_ARG, "prefill length %u of slot %d", lens[i], first + i);
    for (uint32_t q = 0; q + 1 < lens[i]; ++q) {
      cols.push_back(m->slots[first + i]);
      pos4.insert(pos4.end(), {(int32_t)q, 0, 0, 0});
    }
  }
  const size_t n = cols.size();
  // query tiles: runs of one sequence inside a block, at most kPfTileQ long
  std::vector<PfTile> tiles;
  std::vector<size_t> tile0;  // first tile of each block
  for (size_t b0 = 0; b0 < n; b0 += kPfBlock) {
    tile0.push_back(tiles.size());
    const size_t b1 = std::min(n, b0 + (size_t)kPfBlock);
    for (size_t c = b0; c < b1;) {
      size_t e = c + 1;
      while (e < b1 && e - c < (size_t)kPfTileQ && cols[e].tokens == cols[c].tokens) ++e;
      tiles.push_back(PfTile{(int32_t)(c - b0), (int32_t)(e - c), pos4[4 * c], 0});
      c = e;
    }
  }
  tile0.push_back(tiles.size());
  if (n > 0) {
    if (n > m->pf_cap) {
      size_t cap = std::max(n, (size_t)4096);
      if ((rc = m->alloc(&m->pf_cols, cap)) || (rc = m->alloc(&m->pf_pos4, 4 * cap))) return rc;
      m->pf_cap = cap;
    }
    if (tiles.size() > m->pf_tile_cap) {
      size_t cap = std::max(tiles.size(), (size_t)1024);
      if ((rc = m->alloc(&m->pf_tiles, cap))) return rc;
      m->pf_tile_cap = cap;
    }
    // pageable sources: each copy returns once its data is staged
    Q4_CUDA(cudaMemcpyAsync(m->pf_cols, cols.data(), n * sizeof(SlotState), cudaMemcpyHostToDevice, m->stream));
    Q4_CUDA(cudaMemcpyAsync(m->pf_pos4, pos4.data(), 4 * n * sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
    Q4_CUDA(cudaMemcpyAsync(m->pf_tiles, tiles.data(), tiles.size() * sizeof(PfTile), cudaMemcpyHostToDevice,
                            m->stream));
    PrefillPlan& p = *m->pf;
    for (size_t b = 0; b + 1 < tile0.size(); ++b) {
      const size_t c0 = b * kPfBlock;
      p.col_slots = m->pf_cols + c0;
      p.col_pos4 = m->pf_pos4 + 4 * c0;
      p.tiles = m->pf_tiles + tile0[b];
      p.n_cols = (int)std::min((size_t)kPfBlock, n - c0);
      p.n_tiles = (int)(tile0[b + 1] - tile0[b]);
      if ((rc = q4gpu_enqueue_prefill_block(p, m->stream))) return rc;
    }
  }
  for (int i = 0; i < S; ++i) {
    const int32_t pos = (int32_t)lens[i] - 1;
    Q4_CUDA(cudaMemcpyAsync(m->slots[first + i].pos, &pos, sizeof(int32_t), cudaMemcpyHostToDevice, m->stream));
  }
  return Q4GPU_OK;
}

int batch_check_error(q4gpu_model* m) {
  if (!m->b_err) return Q4GPU_OK;
  int e = 0;
  Q4_CUDA(cudaMemcpy(&e, m->b_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemsetAsync(m->b_err, 0, sizeof(int), m->stream);
    return q4gpu_fail(Q4GPU_ERR_CUDA, "batched GEMM: a pipeline wait ran out");
  }
  return Q4GPU_OK;
}

// Graph of one batched step over slots [first, first + S), with the B
// matrices' ones rows set for its padded size.
int batch_graph(q4gpu_model* m, int first, int S, cudaGraphExec_t* out, bool hidden_only = false) {
  int rc = batch_prepare(m);
  if (rc) return rc;
  auto pp = std::make_unique<BatchPlan>();
  BatchPlan& p = *pp;
  if ((rc = batch_plan(m, first, S, p))) return rc;
  if (m->b_pad_sp != p.SP) {
    // rows 3 SP .. 3 SP + 7 may hold limbs of a wider batch: the GEMMs read
    // them (N rounds 3 SP up to 16) and need zeros there
    Q4_CUDA(cudaMemsetAsync(m->b_bt1 + (size_t)3 * p.SP * kHidden, 0, (size_t)kBatchPad * kHidden, m->stream));
    Q4_CUDA(cudaMemsetAsync(m->b_bt2 + (size_t)3 * p.SP * 2 * kHidden, 0, (size_t)kBatchPad * 2 * kHidden, m->stream));
    Q4_CUDA(cudaMemsetAsync(m->b_bt3 + (size_t)3 * p.SP * kInter, 0, (size_t)kBatchPad * kInter, m->stream));
    m->b_pad_sp = p.SP;
  }
  if (hidden_only) p.final_act = m->b_final_act;
  const auto key = std::make_tuple(first, S, hidden_only ? 1 : 0);
  auto it = m->b_graphs.find(key);
  if (it != m->b_graphs.end()) {
    *out = it->second;
    return Q4GPU_OK;
  }
  if ((rc = q4gpu_batch_setup(p))) return rc;
  cudaGraph_t g = nullptr;
  Q4_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  rc = q4gpu_enqueue_batch_step(p, m->stream);
  const cudaError_t ce = cudaStreamEndCapture(m->stream, &g);
  if (rc != Q4GPU_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "batch graph capture: %s", cudaGetErrorString(ce));
  cudaGraphExec_t e = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "batch graph instantiate: %s", cudaGetErrorString(ie));
  m->b_graphs[key] = e;
  *out = e;
  return Q4GPU_OK;
}

int batch_range_ok(q4gpu_model* m, int first, int n_seq) {
  if (!m || first < 0 || n_seq < 1 || n_seq > kBatchSeqMax || first + n_seq > m->cfg.max_seqs)
    return q4gpu_fail(Q4GPU_ERR_ARG, "batch needs 1..%d slots inside max_seqs", kBatchSeqMax);
  for (int s = first; s < first + n_seq; ++s)
    if (slot_busy(m, s)) return q4gpu_fail(Q4GPU_ERR_ARG, "slot %d still has work queued", s);
  return set_device(m);
}

}  // namespace

extern "C" {

const char* q4gpu_last_error(void) { return g_last_error.c_str(); }
const char* q4gpu_version(void) { return "q4gpu 0.1 sm_100a"; }

int q4gpu_model_create(const q4gpu_model_config* cfg, q4gpu_model** out) {
  if (!cfg || !out) return q4gpu_fail(Q4GPU_ERR_ARG, "null config/out");
  *out = nullptr;
  if (cfg->n_layers < 1 || cfg->n_layers > kMaxLayers || cfg->vocab < 1 || cfg->max_context < 1 ||
      cfg->max_context > 16384 || cfg->max_seqs < 1 || cfg->max_seqs > 1024)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad model config");
  auto* m = new q4gpu_model();
  m->cfg = *cfg;
  int rc = Q4GPU_OK;
  auto fail = [&](int code) {
    q4gpu_model_destroy(m);
    return code;
  };
  if ((rc = set_device(m))) return fail(rc);
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
    return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "stream create"));
  const int L = cfg->n_layers;
  if ((rc = m->alloc(&m->w_layers, kLayerWBytes * L))) return fail(rc);
  if ((rc = m->alloc(&m->s_layers, kLayerScales * L))) return fail(rc);
  if ((rc = m->alloc(&m->gammas, kLayerGammas * L))) return fail(rc);
  if ((rc = m->alloc(&m->emb, (size_t)cfg->vocab * 512))) return fail(rc);
  if ((rc = m->alloc(&m->semb, (size_t)cfg->vocab * 16))) return fail(rc);
  if ((rc = m->alloc(&m->g_final, kHidden))) return fail(rc);
  if ((rc = m->alloc(&m->cos_tab, (size_t)cfg->max_context * kHeadDim))) return fail(rc);
  if ((rc = m->alloc(&m->sin_tab, (size_t)cfg->max_context * kHeadDim))) return fail(rc);
  if ((rc = m->alloc(&m->exp_lut, kExpLut))) return fail(rc);
  if ((rc = m->alloc(&m->sig_lut, kSigLut))) return fail(rc);
  if ((rc = m->alloc(&m->p_wo_sl, (size_t)L * 64 * kHidden * 16))) return fail(rc);
  if ((rc = m->alloc(&m->p_so_sl, (size_t)L * 64 * kHidden * 2))) return fail(rc);
  for (int l = 0; l < L; ++l) {
    LayerW& w = m->layers[l];
    w.wo_sl = m->p_wo_sl + (size_t)l * 64 * kHidden * 16;
    w.so_sl = m->p_so_sl + (size_t)l * 64 * kHidden * 2;
    const TensorRef q = layer_tensor(m, l, Q4GPU_T_Q), o = layer_tensor(m, l, Q4GPU_T_O),
                    g = layer_tensor(m, l, Q4GPU_T_GATE), u = layer_tensor(m, l, Q4GPU_T_UP),
                    d = layer_tensor(m, l, Q4GPU_T_DOWN);
    w.wqkv = q.w;
    w.sqkv = q.s;
    w.wo = o.w;
    w.so = o.s;
    w.wgate = g.w;
    w.sgate = g.s;
    w.wup = u.w;
    w.sup = u.s;
    w.wdown = d.w;
    w.sdown = d.s;
    int n;
    w.g_in = layer_gamma(m, l, Q4GPU_T_INPUT_GAMMA, &n);
    w.g_post = layer_gamma(m, l, Q4GPU_T_POST_GAMMA, &n);
    w.g_q = layer_gamma(m, l, Q4GPU_T_Q_GAMMA, &n);
    w.g_k = layer_gamma(m, l, Q4GPU_T_K_GAMMA, &n);
  }
  // default tables: gammas 1.0, LUTs, RoPE (float32 host build)
  {
    std::vector<int32_t> ones(kLayerGammas * L, 128), e(kExpLut), sg(kSigLut);
    if (stream_copy(m, m->gammas, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice) != Q4GPU_OK ||
        stream_copy(m, m->g_final, ones.data(), kHidden * 4, cudaMemcpyHostToDevice) != Q4GPU_OK)
      return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "gamma init"));
    build_luts(e.data(), sg.data());
    if (stream_copy(m, m->exp_lut, e.data(), kExpLut * 4, cudaMemcpyHostToDevice) != Q4GPU_OK ||
        stream_copy(m, m->sig_lut, sg.data(), kSigLut * 4, cudaMemcpyHostToDevice) != Q4GPU_OK)
      return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "lut init"));
    std::vector<int32_t> c((size_t)cfg->max_context * kHeadDim), s(c.size());
    build_rope(cfg->max_context, c.data(), s.data());
    if (stream_copy(m, m->cos_tab, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != Q4GPU_OK ||
        stream_copy(m, m->sin_tab, s.data(), s.size() * 4, cudaMemcpyHostToDevice) != Q4GPU_OK)
      return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "rope init"));
  }
  // paged KV pool: every slot owns ceil(max_context / 64) pages
  m->page_elems = (int64_t)L * 2 * kKvHeads * kKvPage * kHeadDim;
  m->pages_per_seq = (cfg->max_context + kKvPage - 1) / kKvPage;
  const int64_t n_pages = (int64_t)m->pages_per_seq * cfg->max_seqs;
  if ((rc = m->alloc(&m->kv_pool, (size_t)n_pages * m->page_elems))) return fail(rc);
  // the byte-plane copies of K and V, for the batched attention kernels that
  // read them (q4_batch.cu: batch_attn_kernel, batch_attn_cl_tc_kernel): in
  // multi-slot models and long contexts (the vocabulary-sharded long-context
  // decode runs one sequence per GPU through the batched path); a one-slot
  // model up to 1024 positions decodes on the batch-1 paths, which read none
  if (cfg->max_seqs >= 2 || cfg->max_context > 1024) {
    m->kpl_page_bytes = (int64_t)L * kKvHeads * kKplHead;
    if ((rc = m->alloc(&m->kv_planes, (size_t)n_pages * m->kpl_page_bytes))) return fail(rc);
    if ((rc = m->alloc(&m->v_planes, (size_t)n_pages * m->kpl_page_bytes))) return fail(rc);
  }
  if ((rc = m->alloc(&m->page_tables, (size_t)n_pages))) return fail(rc);
  {
    std::vector<int32_t> pt(n_pages);
    for (int64_t i = 0; i < n_pages; ++i) pt[i] = (int32_t)i;
    if (stream_copy(m, m->page_tables, pt.data(), n_pages * 4, cudaMemcpyHostToDevice) != Q4GPU_OK)
      return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "page table init"));
  }
  // per-slot state
  const int S = cfg->max_seqs;
  int32_t *pos, *tokens, *hidden, *qrope, *attn, *post, *mlp;
  int64_t* scores;
  ArgBestD* part;
  unsigned int* ctr;
  const int T = cfg->max_context + 2;
  if ((rc = m->alloc(&pos, (size_t)S * 4))) return fail(rc);
  if ((rc = m->alloc(&tokens, (size_t)S * T))) return fail(rc);
  if ((rc = m->alloc(&scores, (size_t)S * T))) return fail(rc);
  if ((rc = m->alloc(&hidden, (size_t)S * kHidden))) return fail(rc);
  if ((rc = m->alloc(&qrope, (size_t)S * kQRows))) return fail(rc);
  if ((rc = m->alloc(&attn, (size_t)S * kQRows))) return fail(rc);
  if ((rc = m->alloc(&post, (size_t)S * kHidden))) return fail(rc);
  if ((rc = m->alloc(&mlp, (size_t)S * kInter))) return fail(rc);
  if ((rc = m->alloc(&part, (size_t)S * Q4GPU_LM_HEAD_BLOCKS))) return fail(rc);
  if ((rc = m->alloc(&ctr, (size_t)S * 32))) return fail(rc);
  for (int i = 0; i < S; ++i) {
    SlotState st{};
    st.pos = pos + i * 4;
    st.tokens = tokens + (size_t)i * T;
    st.scores = scores + (size_t)i * T;
    st.hidden = hidden + (size_t)i * kHidden;
    st.qrope = qrope + (size_t)i * kQRows;
    st.attn = attn + (size_t)i * kQRows;
    st.post = post + (size_t)i * kHidden;
    st.mlp = mlp + (size_t)i * kInter;
    st.lm_partial = part + (size_t)i * Q4GPU_LM_HEAD_BLOCKS;
    st.lm_counter = ctr + (size_t)i * 32;
    st.kv = KvView{m->kv_pool, m->page_tables + (size_t)i * m->pages_per_seq, m->page_elems, m->kv_planes,
                   m->kpl_page_bytes, m->v_planes};
    st.max_ctx = cfg->max_context;
    m->slots.push_back(st);
  }
  if (cudaMallocHost(&m->h_res, sizeof(HostResult) * S) != cudaSuccess ||
      cudaMallocHost(&m->h_in, sizeof(int32_t) * 2 * S) != cudaSuccess)
    return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "pinned alloc"));
  m->done.resize(S);
  m->busy.assign(S, 0);
  for (int i = 0; i < S; ++i)
    if (cudaEventCreateWithFlags(&m->done[i], cudaEventDisableTiming) != cudaSuccess)
      return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "event create"));
  m->stage_attn_cl = q4gpu_stage_attention_fits(cfg->max_context) && q4gpu_stage_attention_setup(cfg->max_context) == Q4GPU_OK;
  if (!m->stage_attn_cl) {
    const size_t asmem = attn_smem(cfg->max_context);
    if (cudaFuncSetAttribute(attn_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)asmem) != cudaSuccess)
      return fail(q4gpu_fail(Q4GPU_ERR_SHAPE, "max_context %d needs %zu B of shared memory", cfg->max_context, asmem));
  }
  // persistent kernel: available when its shared memory fits (score buffer of max_context)
  if ((rc = m->alloc(&m->layers_dev, (size_t)L))) return fail(rc);
  if (stream_copy(m, m->layers_dev, m->layers, sizeof(LayerW) * L, cudaMemcpyHostToDevice) != Q4GPU_OK)
    return fail(q4gpu_fail(Q4GPU_ERR_CUDA, "layer table upload"));
  if ((rc = m->alloc(&m->p_qkv, (size_t)kQRows + 2 * kKvRows))) return fail(rc);
  if ((rc = m->alloc(&m->p_acc, (size_t)16 * kHidden))) return fail(rc);
  if ((rc = m->alloc(&m->p_lm_part, 1024))) return fail(rc);
  if ((rc = m->alloc(&m->p_bar, 16))) return fail(rc);
  if ((rc = m->alloc(&m->p_err, 16))) return fail(rc);
  if (q4gpu_persistent_setup(cfg->max_context, &m->p_smem, &m->p_grid) == Q4GPU_OK && m->p_grid <= 1024 &&
      encode_kv_map(m, n_pages) == Q4GPU_OK)
    m->mode = 1;
  else
    m->p_grid = 0;
  *out = m;
  return Q4GPU_OK;
}

void q4gpu_model_destroy(q4gpu_model* m) {
  if (!m) return;
  cudaSetDevice(m->cfg.device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : m->b_graphs) cudaGraphExecDestroy(kv.second);
  if (m->h_bio) cudaFreeHost(m->h_bio);
  for (auto e : m->done)
    if (e) cudaEventDestroy(e);
  for (void* p : m->allocs) cudaFree(p);
  delete m->pf;
  if (m->h_res) cudaFreeHost(m->h_res);
  if (m->h_in) cudaFreeHost(m->h_in);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

void* q4gpu_model_stream(q4gpu_model* m) { return m ? (void*)m->stream : nullptr; }

int q4gpu_model_init_synthetic(q4gpu_model* m, uint64_t seed, float std_dev, float gamma_std) {
  if (!m) return q4gpu_fail(Q4GPU_ERR_ARG, "null model");
  int rc = set_device(m);
  if (rc) return rc;
  const size_t max_elems = std::max<size_t>((size_t)m->cfg.vocab * kHidden, (size_t)kInter * kHidden);
  float* tmp = nullptr;
  int32_t* err = nullptr;
  Q4_CUDA(cudaMalloc(&tmp, max_elems * sizeof(float)));
  Q4_CUDA(cudaMalloc(&err, sizeof(int32_t)));
  Q4_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), m->stream));
  m->p_stale = true;
  auto gen_quant = [&](uint64_t tid, const TensorRef& t) -> int {
    int r = q4gpu_synth_f32(seed, tid, 0, t.rows * t.cols, std_dev, 1, tmp, m->stream);
    if (r) return r;
    return q4gpu_quantize_q4(tmp, t.rows, t.cols, t.w, t.s, err, m->stream);
  };
  // tensor ids: embedding 0, final norm 15, layer l tensor w -> 16 + 16 l + w
  rc = gen_quant(0, TensorRef{m->emb, m->semb, m->cfg.vocab, kHidden});
  for (int l = 0; l < m->cfg.n_layers && !rc; ++l)
    for (int wi = Q4GPU_T_Q; wi <= Q4GPU_T_DOWN && !rc; ++wi)
      rc = gen_quant(16 + 16 * (uint64_t)l + wi, layer_tensor(m, l, wi));
  if (!rc && gamma_std > 0.f) {
    std::vector<float> hv(kHidden);
    std::vector<int32_t> q(kHidden);
    auto gamma = [&](uint64_t tid, int32_t* dst, int n) -> int {
      int r = q4gpu_synth_f32(seed, tid, 0, n, gamma_std, 1, tmp, m->stream);
      if (r) return r;
      Q4_CUDA(cudaMemcpyAsync(hv.data(), tmp, n * 4, cudaMemcpyDeviceToHost, m->stream));
      Q4_CUDA(cudaStreamSynchronize(m->stream));
      for (int i = 0; i < n; ++i) {
        const float g = 1.0f + hv[i];
        double v = std::nearbyint((double)g * 128.0);
        v = v > 32767 ? 32767 : (v < -32768 ? -32768 : v);
        q[i] = (int32_t)v;
      }
      Q4_CUDA(cudaMemcpyAsync(dst, q.data(), n * 4, cudaMemcpyHostToDevice, m->stream));
      Q4_CUDA(cudaStreamSynchronize(m->stream));
      return Q4GPU_OK;
    };
    for (int l = 0; l < m->cfg.n_layers && !rc; ++l)
      for (int wi = Q4GPU_T_INPUT_GAMMA; wi <= Q4GPU_T_K_GAMMA && !rc; ++wi) {
        int n;
        int32_t* dst = layer_gamma(m, l, wi, &n);
        rc = gamma(16 + 16 * (uint64_t)l + wi, dst, n);
      }
    if (!rc) rc = gamma(15, m->g_final, kHidden);
  }
  int32_t herr = 0;
  if (!rc && cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess)
    rc = q4gpu_fail(Q4GPU_ERR_CUDA, "err readback");
  if (cudaStreamSynchronize(m->stream) != cudaSuccess && !rc) rc = q4gpu_fail(Q4GPU_ERR_CUDA, "init sync");
  cudaFree(tmp);
  cudaFree(err);
  if (!rc && herr) rc = q4gpu_fail(Q4GPU_ERR_QUANT, "a Q4 scale overflowed unsigned Q2.14");
  return rc;
}

static int tensor_io(q4gpu_model* m, int32_t layer, int32_t which, void* data, size_t data_bytes, uint16_t* scale,
                     size_t scale_bytes, bool to_device) {
  if (!m || !data) return q4gpu_fail(Q4GPU_ERR_ARG, "null model/data");
  int rc = set_device(m);
  if (rc) return rc;
  const cudaMemcpyKind kind = to_device ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
  if (to_device) m->p_stale = true;
  auto cp = [&](void* dev, void* host, size_t n) -> int {
    return to_device ? stream_copy(m, dev, host, n, kind) : stream_copy(m, host, dev, n, kind);
  };
  if (which >= Q4GPU_T_Q && which <= Q4GPU_T_DOWN) {
    if (layer < 0 || layer >= m->cfg.n_layers) return q4gpu_fail(Q4GPU_ERR_ARG, "bad layer");
    const TensorRef t = layer_tensor(m, layer, which);
    if (data_bytes != (size_t)t.rows * t.cols / 2 || !scale || scale_bytes != (size_t)t.rows * (t.cols / 64) * 2)
      return q4gpu_fail(Q4GPU_ERR_SHAPE, "tensor %d expects %lld x %d", which, (long long)t.rows, t.cols);
    if ((rc = cp(t.w, data, data_bytes))) return rc;
    return cp(t.s, scale, scale_bytes);
  }
  if (which >= Q4GPU_T_INPUT_GAMMA && which <= Q4GPU_T_K_GAMMA) {
    if (layer < 0 || layer >= m->cfg.n_layers) return q4gpu_fail(Q4GPU_ERR_ARG, "bad layer");
    int n;
    int32_t* g = layer_gamma(m, layer, which, &n);
    if (data_bytes != (size_t)n * 4) return q4gpu_fail(Q4GPU_ERR_SHAPE, "gamma expects %d int32", n);
    return cp(g, data, data_bytes);
  }
  switch (which) {
    case Q4GPU_T_EMBED:
      if (data_bytes != (size_t)m->cfg.vocab * 512 || !scale || scale_bytes != (size_t)m->cfg.vocab * 32)
        return q4gpu_fail(Q4GPU_ERR_SHAPE, "embedding expects %d x 1024", m->cfg.vocab);
      if ((rc = cp(m->emb, data, data_bytes))) return rc;
      return cp(m->semb, scale, scale_bytes);
    case Q4GPU_T_FINAL_GAMMA:
      if (data_bytes != kHidden * 4) return q4gpu_fail(Q4GPU_ERR_SHAPE, "final gamma expects 1024 int32");
      return cp(m->g_final, data, data_bytes);
    case Q4GPU_T_ROPE_COS:
    case Q4GPU_T_ROPE_SIN:
      if (data_bytes != (size_t)m->cfg.max_context * kHeadDim * 4)
        return q4gpu_fail(Q4GPU_ERR_SHAPE, "rope table expects [%d, 128] int32", m->cfg.max_context);
      return cp(which == Q4GPU_T_ROPE_COS ? m->cos_tab : m->sin_tab, data, data_bytes);
    case Q4GPU_T_EXP_LUT:
      if (data_bytes != kExpLut * 4) return q4gpu_fail(Q4GPU_ERR_SHAPE, "exp LUT expects 257 int32");
      return cp(m->exp_lut, data, data_bytes);
    case Q4GPU_T_SIGMOID_LUT:
      if (data_bytes != kSigLut * 4) return q4gpu_fail(Q4GPU_ERR_SHAPE, "sigmoid LUT expects 1025 int32");
      return cp(m->sig_lut, data, data_bytes);
    default: return q4gpu_fail(Q4GPU_ERR_ARG, "unknown tensor id %d", which);
  }
}

int q4gpu_model_get_config(q4gpu_model* m, q4gpu_model_config* cfg) {
  if (!m || !cfg) return q4gpu_fail(Q4GPU_ERR_ARG, "null model/config");
  *cfg = m->cfg;
  return Q4GPU_OK;
}

int q4gpu_model_set_tensor(q4gpu_model* m, int32_t layer, int32_t which, const void* data, size_t data_bytes,
                           const uint16_t* scale, size_t scale_bytes) {
  return tensor_io(m, layer, which, const_cast<void*>(data), data_bytes, const_cast<uint16_t*>(scale), scale_bytes,
                   true);
}

int q4gpu_model_get_tensor(q4gpu_model* m, int32_t layer, int32_t which, void* data, size_t data_bytes,
                           uint16_t* scale, size_t scale_bytes) {
  return tensor_io(m, layer, which, data, data_bytes, scale, scale_bytes, false);
}

// Validation shared by the runner and the decode API (reference order:
// qmap_one_token_runtime.h:249-283).
static int validate_run(q4gpu_model* m, uintptr_t base, const qot_run_config_t* c, uint32_t position) {
  if (!c) return QOT_ERR_NULL;
  if (c->layer_count == 0u || c->layer_start >= (uint32_t)m->cfg.n_layers) return QOT_ERR_BAD_LAYER;
  const uint32_t end = c->layer_start + c->layer_count;
  if (end > (uint32_t)m->cfg.n_layers || end < c->layer_start) return QOT_ERR_BAD_LAYER;
  if (position >= (uint32_t)m->cfg.max_context) return QOT_ERR_CONTEXT;
  if (base >= (uintptr_t)m->cfg.max_seqs) return QOT_ERR_BAD_ADDR;
  return QOT_OK;
}

int q4gpu_run_token(void* runner_context, uintptr_t base, const qot_run_config_t* config, uint32_t input_token_id,
                    uint32_t position, uint32_t max_polls, qot_result_t* result) {
  q4gpu_model* m = static_cast<q4gpu_model*>(runner_context);
  if (!m || !config || !result) return QOT_ERR_NULL;
  int rc = validate_run(m, base, config, position);
  if (rc != QOT_OK) return rc;
  if (config->embedding_enable && input_token_id >= (uint32_t)m->cfg.vocab) return QOT_ERR_BAD_TOKEN;
  if (set_device(m)) return QOT_ERR_STATUS;
  const int slot = (int)base;
  if (slot_busy(m, slot)) return QOT_ERR_BUSY;
  // a full-model call with the embedding runs as one step of the persistent
  // kernel (mode 1); layer ranges run the per-stage graph
  const bool persistent = m->mode == 1 && m->p_grid > 0 && config->layer_start == 0u &&
                          (int)config->layer_count == m->cfg.n_layers && config->embedding_enable;
  cudaGraphExec_t g = nullptr;
  if (!persistent && get_graph(m, GraphKey{slot, (int)config->layer_start, (int)config->layer_count,
                                           config->embedding_enable ? 1 : 0, 1},
                               &g) != Q4GPU_OK)
    return QOT_ERR_STATUS;
  const SlotState& st = m->slots[slot];
  int32_t* hin = m->h_in + 2 * slot;
  hin[0] = (int32_t)input_token_id;
  hin[1] = (int32_t)position;
  HostResult* hr = m->h_res + slot;
  if (cudaMemcpyAsync(st.tokens + position, &hin[0], 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess ||
      cudaMemcpyAsync(st.pos, &hin[1], 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess ||
      (persistent ? run_persistent(m, slot, 1, (int)position) != Q4GPU_OK
                  : cudaGraphLaunch(g, m->stream) != cudaSuccess) ||
      cudaMemcpyAsync(&hr->token, st.tokens + position + 1, 4, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess ||
      cudaMemcpyAsync(&hr->score, st.scores + position + 1, 8, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess ||
      cudaEventRecord(m->done[slot], m->stream) != cudaSuccess) {
    q4gpu_fail(Q4GPU_ERR_CUDA, "run_token enqueue: %s", cudaGetErrorString(cudaGetLastError()));
    return QOT_ERR_STATUS;
  }
  m->busy[slot] = 1;
  memset(result, 0, sizeof(*result));
  rc = poll_slot(m, slot, max_polls);
  if (rc != QOT_OK) return rc;
  if (check_persistent_error(m) != Q4GPU_OK) return QOT_ERR_TIMEOUT;
  result->status = 1u;  // done
  result->token_id = (uint32_t)hr->token;
  result->score_q26 = hr->score;
  result->layers_started = config->layer_count;
  result->layers_completed = config->layer_count;
  result->layer_done_mask =
      (uint32_t)((config->layer_count >= 32 ? 0xFFFFFFFFull : ((1ull << config->layer_count) - 1)) << config->layer_start);
  result->tail_tiles_started = result->tail_tiles_completed = (uint32_t)((m->cfg.vocab + 15) / 16);
  const uint64_t rd = step_bytes(m, config->layer_count, position + 1, 1) / 4;
  result->mem_read_words = (uint32_t)std::min<uint64_t>(rd, 0xFFFFFFFFull);
  result->mem_write_words = (uint32_t)(config->layer_count * 2 * kKvRows);
  return QOT_OK;
}

int q4gpu_decode_token_ids(q4gpu_model* m, uintptr_t base, const qot_run_config_t* cfg,
                           const uint32_t* prompt_token_ids, uint32_t prompt_token_count, uint32_t max_new_tokens,
                           uint32_t* generated_token_ids, uint32_t generated_token_capacity,
                           uint32_t max_polls_per_token, uint32_t* generated_token_count, qot_result_t* last_result) {
  if (generated_token_count) *generated_token_count = 0u;
  if (!m || !cfg || !prompt_token_ids || !generated_token_ids || !last_result) return QOT_ERR_NULL;
  if (prompt_token_count == 0u || max_new_tokens == 0u) return QOT_ERR_CAPACITY;
  if (generated_token_capacity < max_new_tokens) return QOT_ERR_CAPACITY;
  if (cfg->runtime_context_enable == 0u || cfg->embedding_enable == 0u) return QOT_ERR_CONTEXT;
  if (cfg->final_hidden_override_valid != 0u) return QOT_ERR_CONTEXT;
  for (uint32_t i = 0; i < prompt_token_count; ++i)
    if (prompt_token_ids[i] >= (uint32_t)m->cfg.vocab) return QOT_ERR_BAD_TOKEN;
  const uint32_t run_count = prompt_token_count + max_new_tokens - 1u;
  if (run_count < prompt_token_count || cfg->position >= (uint32_t)m->cfg.max_context ||
      run_count > (uint32_t)m->cfg.max_context - cfg->position)
    return QOT_ERR_CONTEXT;
  int rc = validate_run(m, base, cfg, cfg->position);
  if (rc != QOT_OK) return rc;
  if (set_device(m)) return QOT_ERR_STATUS;
  const int slot = (int)base;
  if (slot_busy(m, slot)) return QOT_ERR_BUSY;
  cudaGraphExec_t gpre, gstep;
  if (get_graph(m, GraphKey{slot, (int)cfg->layer_start, (int)cfg->layer_count, 1, 0}, &gpre) != Q4GPU_OK ||
      get_graph(m, GraphKey{slot, (int)cfg->layer_start, (int)cfg->layer_count, 1, 1}, &gstep) != Q4GPU_OK)
    return QOT_ERR_STATUS;
  const SlotState& st = m->slots[slot];
  std::vector<int32_t> toks(prompt_token_ids, prompt_token_ids + prompt_token_count);
  int32_t* hin = m->h_in + 2 * slot;
  hin[1] = (int32_t)cfg->position;
  std::vector<int32_t> gen(max_new_tokens);
  std::vector<int64_t> gsc(max_new_tokens);
  bool ok = cudaMemcpyAsync(st.tokens + cfg->position, toks.data(), toks.size() * 4, cudaMemcpyHostToDevice,
                            m->stream) == cudaSuccess &&
            cudaMemcpyAsync(st.pos, &hin[1], 4, cudaMemcpyHostToDevice, m->stream) == cudaSuccess;
  const bool full_model = cfg->layer_start == 0u && cfg->layer_count == (uint32_t)m->cfg.n_layers;
  if (m->prefill_mode == 1 && cfg->position == 0u && prompt_token_count >= 2u && full_model && m->cfg.vocab >= 64) {
    // prompt positions 0 .. len - 2 as batched prefill columns (the same K/V
    // cache as the serial runs), then max_new_tokens decode runs from the last
    // prompt token (persistent kernel or step graphs) instead of
    // len + max_new_tokens - 1
    const uint32_t len = prompt_token_count;
    ok = ok && batch_prefill(m, slot, 1, &len) == Q4GPU_OK;
    if (m->mode == 1)
      ok = ok && run_persistent(m, slot, (int)max_new_tokens, (int)len) == Q4GPU_OK;
    else
      for (uint32_t i = 0; ok && i < max_new_tokens; ++i) ok = cudaGraphLaunch(gstep, m->stream) == cudaSuccess;
  } else if (m->mode == 1) {
    ok = ok && run_persistent(m, slot, (int)run_count, (int)(cfg->position + prompt_token_count)) == Q4GPU_OK;
  } else {
    for (uint32_t i = 0; ok && i + 1 < prompt_token_count; ++i) ok = cudaGraphLaunch(gpre, m->stream) == cudaSuccess;
    for (uint32_t i = 0; ok && i < max_new_tokens; ++i) ok = cudaGraphLaunch(gstep, m->stream) == cudaSuccess;
  }
  const uint32_t first = cfg->position + prompt_token_count;
  ok = ok &&
       cudaMemcpyAsync(gen.data(), st.tokens + first, max_new_tokens * 4, cudaMemcpyDeviceToHost, m->stream) ==
           cudaSuccess &&
       cudaMemcpyAsync(gsc.data(), st.scores + first, max_new_tokens * 8, cudaMemcpyDeviceToHost, m->stream) ==
           cudaSuccess &&
       cudaEventRecord(m->done[slot], m->stream) == cudaSuccess;
  if (!ok) {
    q4gpu_fail(Q4GPU_ERR_CUDA, "decode enqueue: %s", cudaGetErrorString(cudaGetLastError()));
    return QOT_ERR_STATUS;
  }
  m->busy[slot] = 1;
  // The poll budget covers the whole run.
  const uint64_t polls = (uint64_t)max_polls_per_token * run_count;
  rc = poll_slot(m, slot, (uint32_t)std::min<uint64_t>(polls, 0xFFFFFFFFull));
  memset(last_result, 0, sizeof(*last_result));
  if (rc != QOT_OK) return rc;
  if (check_persistent_error(m) != Q4GPU_OK) return QOT_ERR_TIMEOUT;
  for (uint32_t i = 0; i < max_new_tokens; ++i) {
    if ((uint32_t)gen[i] >= (uint32_t)m->cfg.vocab) return QOT_ERR_BAD_TOKEN;
    generated_token_ids[i] = (uint32_t)gen[i];
  }
  if (generated_token_count) *generated_token_count = max_new_tokens;
  last_result->status = 1u;
  last_result->token_id = (uint32_t)gen[max_new_tokens - 1];
  last_result->score_q26 = gsc[max_new_tokens - 1];
  last_result->layers_started = last_result->layers_completed = cfg->layer_count;
  return QOT_OK;
}

int q4gpu_decode_batch(q4gpu_model* m, int32_t n_seq, const uint32_t* prompts, const uint32_t* prompt_lens,
                       uint32_t max_new_tokens, uint32_t* generated, int64_t* scores) {
  if (!m || !prompts || !prompt_lens || !generated) return QOT_ERR_NULL;
  if (n_seq <= 0 || n_seq > m->cfg.max_seqs || max_new_tokens == 0u) return QOT_ERR_CAPACITY;
  std::vector<size_t> off(n_seq + 1, 0);
  for (int s = 0; s < n_seq; ++s) {
    const uint32_t len = prompt_lens[s];
    if (len == 0u) return QOT_ERR_CAPACITY;
    if ((uint64_t)len + max_new_tokens - 1u > (uint64_t)m->cfg.max_context) return QOT_ERR_CONTEXT;
    off[s + 1] = off[s] + len;
    for (uint32_t i = 0; i < len; ++i)
      if (prompts[off[s] + i] >= (uint32_t)m->cfg.vocab) return QOT_ERR_BAD_TOKEN;
  }
  for (int first = 0; first < n_seq; first += kBatchSeqMax) {
    const int S = std::min(kBatchSeqMax, n_seq - first);
    if (batch_range_ok(m, first, S) != Q4GPU_OK) return QOT_ERR_BUSY;
    cudaGraphExec_t g;
    if (batch_graph(m, first, S, &g) != Q4GPU_OK) return QOT_ERR_STATUS;
    // prompts at positions 0.., every sequence from position 0; the argmax of
    // sequence s lands from position prompt_len[s] on
    std::vector<int32_t> lm(S);
    uint32_t longest = 0;
    bool ok = true;
    for (int i = 0; i < S && ok; ++i) {
      const int s = first + i;
      lm[i] = (int32_t)prompt_lens[s];
      longest = std::max(longest, prompt_lens[s]);
      ok = cudaMemcpyAsync(m->slots[s].tokens, prompts + off[s], (size_t)prompt_lens[s] * 4, cudaMemcpyHostToDevice,
                           m->stream) == cudaSuccess;
    }
    ok = ok &&
         cudaMemcpyAsync(m->b_lm_from + first, lm.data(), (size_t)S * 4, cudaMemcpyHostToDevice, m->stream) ==
             cudaSuccess;
    uint32_t steps;
    if (m->prefill_mode == 1) {
      // prompt positions 0 .. len - 2 as batched columns; then every sequence
      // steps from its last prompt token
      if (ok && batch_prefill(m, first, S, prompt_lens + first) != Q4GPU_OK) return QOT_ERR_STATUS;
      steps = max_new_tokens;
    } else {
      ok = ok && q4gpu_batch_set_positions(m->b_slots + first, S, 0, m->b_lm_from + first, -1, m->stream) == Q4GPU_OK;
      steps = longest + max_new_tokens - 1u;
    }
    for (uint32_t i = 0; ok && i < steps; ++i) ok = cudaGraphLaunch(g, m->stream) == cudaSuccess;
    for (int i = 0; ok && i < S; ++i) {
      const int s = first + i;
      ok = cudaMemcpyAsync(generated + (size_t)s * max_new_tokens, m->slots[s].tokens + prompt_lens[s],
                           (size_t)max_new_tokens * 4, cudaMemcpyDeviceToHost, m->stream) == cudaSuccess &&
           (!scores || cudaMemcpyAsync(scores + (size_t)s * max_new_tokens, m->slots[s].scores + prompt_lens[s],
                                       (size_t)max_new_tokens * 8, cudaMemcpyDeviceToHost, m->stream) == cudaSuccess);
    }
    ok = ok && cudaStreamSynchronize(m->stream) == cudaSuccess;
    if (!ok) {
      q4gpu_fail(Q4GPU_ERR_CUDA, "batched decode: %s", cudaGetErrorString(cudaGetLastError()));
      return QOT_ERR_STATUS;
    }
    if (batch_check_error(m) != Q4GPU_OK) return QOT_ERR_TIMEOUT;
  }
  for (size_t i = 0; i < (size_t)n_seq * max_new_tokens; ++i)
    if (generated[i] >= (uint32_t)m->cfg.vocab) return QOT_ERR_BAD_TOKEN;
  return QOT_OK;
}

int q4gpu_batch_steps(q4gpu_model* m, int32_t first_slot, int32_t n_seq, int32_t n_steps) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (n_steps < 0) return q4gpu_fail(Q4GPU_ERR_ARG, "negative step count");
  cudaGraphExec_t g;
  if ((rc = batch_graph(m, first_slot, n_seq, &g))) return rc;
  for (int i = 0; i < n_steps; ++i) Q4_CUDA(cudaGraphLaunch(g, m->stream));
  return Q4GPU_OK;
}

int q4gpu_batch_prefill(q4gpu_model* m, int32_t first_slot, int32_t n_seq, const uint32_t* prompts,
                        const uint32_t* prompt_lens) {
  if (!prompts || !prompt_lens) return q4gpu_fail(Q4GPU_ERR_ARG, "null prompts");
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  std::vector<int32_t> lm(n_seq);
  size_t off = 0;
  for (int i = 0; i < n_seq; ++i) {
    const uint32_t len = prompt_lens[i];
    if (len < 1u || len > (uint32_t)m->cfg.max_context)
      return q4gpu_fail(Q4GPU_ERR_ARG, "prompt %d: length %u outside 1..max_context", i, len);
    for (uint32_t j = 0; j < len; ++j)
      if (prompts[off + j] >= (uint32_t)m->cfg.vocab) return q4gpu_fail(Q4GPU_ERR_ARG, "prompt %d: bad token", i);
    Q4_CUDA(cudaMemcpyAsync(m->slots[first_slot + i].tokens, prompts + off, (size_t)len * 4, cudaMemcpyHostToDevice,
                            m->stream));
    lm[i] = (int32_t)len;
    off += len;
  }
  if ((rc = batch_prepare(m))) return rc;
  Q4_CUDA(cudaMemcpyAsync(m->b_lm_from + first_slot, lm.data(), (size_t)n_seq * 4, cudaMemcpyHostToDevice,
                          m->stream));
  return batch_prefill(m, first_slot, n_seq, prompt_lens);
}

int q4gpu_model_set_prefill(q4gpu_model* m, int32_t mode) {
  if (!m || mode < 0 || mode > 1) return q4gpu_fail(Q4GPU_ERR_ARG, "prefill mode must be 0 or 1");
  m->prefill_mode = mode;
  return Q4GPU_OK;
}

int q4gpu_batch_forward_hidden(q4gpu_model* m, int32_t first_slot, int32_t n_seq, int32_t* final_act) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (!final_act) return q4gpu_fail(Q4GPU_ERR_ARG, "null final_act");
  cudaGraphExec_t g;
  if ((rc = batch_graph(m, first_slot, n_seq, &g, true))) return rc;
  // inside a caller's stream capture (a whole sharded step recorded as one
  // graph) the kernels are enqueued directly: an executable graph cannot be
  // launched into a capturing stream
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  Q4_CUDA(cudaStreamIsCapturing(m->stream, &cs));
  if (cs == cudaStreamCaptureStatusActive) {
    auto pp = std::make_unique<BatchPlan>();
    if ((rc = batch_plan(m, first_slot, n_seq, *pp))) return rc;
    pp->final_act = m->b_final_act;
    if ((rc = q4gpu_enqueue_batch_step(*pp, m->stream))) return rc;
  } else {
    Q4_CUDA(cudaGraphLaunch(g, m->stream));
  }
  Q4_CUDA(cudaMemcpyAsync(final_act, m->b_final_act, (size_t)n_seq * kHidden * 4, cudaMemcpyDeviceToDevice,
                          m->stream));
  return Q4GPU_OK;
}

int q4gpu_lm_head_shard(q4gpu_model* m, const int32_t* acts, int32_t n_act, int32_t row_begin, int32_t row_end,
                        int64_t* best_score, int64_t* best_row) {
  if (!m || !acts || !best_score || !best_row) return q4gpu_fail(Q4GPU_ERR_ARG, "null argument");
  if (n_act < 1 || n_act > kBatchSeqMax || row_begin < 0 || row_end <= row_begin || row_end > m->cfg.vocab)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad LM-head shard: %d vectors, rows [%d, %d)", n_act, row_begin, row_end);
  if (((uintptr_t)acts) & 15) return q4gpu_fail(Q4GPU_ERR_ALIGN, "acts must be 16-byte aligned");
  int rc = set_device(m);
  if (rc) return rc;
  if ((rc = batch_prepare(m))) return rc;
  const int SP = q4gpu_batch_padded(n_act);
  if (m->b_lm_pad_sp != SP) {
    Q4_CUDA(cudaMemsetAsync(m->b_lm_bt + (size_t)3 * SP * kHidden, 0, (size_t)kBatchPad * kHidden, m->stream));
    m->b_lm_pad_sp = SP;
  }
  auto q = std::make_unique<LmShardPlan>();
  q->acts = acts;
  q->n_act = n_act;
  q->row_begin = row_begin;
  q->row_end = row_end;
  q->scales = m->semb + (size_t)row_begin * (kHidden / kGroup);
  q->bt = m->b_lm_bt;
  q->partial = m->b_lm_shard_part;
  q->best_score = best_score;
  q->best_row = best_row;
  q->err = m->b_err;
  if ((rc = q4gpu_encode_q4_map(&q->amap, m->emb + (size_t)row_begin * (kHidden / 2), kHidden / 2,
                                (uint64_t)(row_end - row_begin), 128)) ||
      (rc = q4gpu_encode_u8_map(&q->bmap, m->b_lm_bt, kHidden, (uint64_t)q4gpu_batch_limb_rows(SP), (uint32_t)(3 * SP))))
    return rc;
  return q4gpu_enqueue_lm_shard(*q, m->stream);
}

int q4gpu_batch_commit(q4gpu_model* m, int32_t first_slot, int32_t n_seq, const int64_t* tokens,
                       const int64_t* scores) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (!tokens || !scores) return q4gpu_fail(Q4GPU_ERR_ARG, "null tokens/scores");
  if ((rc = batch_prepare(m))) return rc;
  auto pp = std::make_unique<BatchPlan>();
  if ((rc = batch_plan(m, first_slot, n_seq, *pp))) return rc;
  return q4gpu_enqueue_batch_commit(*pp, tokens, scores, m->stream);
}

int q4gpu_batch_commit_shards(q4gpu_model* m, int32_t first_slot, int32_t n_seq, const int64_t* winners,
                              int32_t n_shards, int32_t stride, int32_t col0) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (!winners) return q4gpu_fail(Q4GPU_ERR_ARG, "null winners");
  if (n_shards < 1 || stride < 1 || col0 < 0 || col0 + n_seq > stride)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad winner layout: %d shards, stride %d, columns [%d, %d)", n_shards, stride, col0,
                      col0 + n_seq);
  if ((rc = batch_prepare(m))) return rc;
  auto pp = std::make_unique<BatchPlan>();
  if ((rc = batch_plan(m, first_slot, n_seq, *pp))) return rc;
  return q4gpu_enqueue_batch_commit_shards(*pp, winners, n_shards, stride, col0, m->stream);
}

int q4gpu_batch_set_position(q4gpu_model* m, int32_t first_slot, int32_t n_seq, int32_t position, int32_t lm_from) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (position < 0 || position >= m->cfg.max_context || lm_from < -1)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad batch position %d / lm_from %d", position, lm_from);
  if ((rc = batch_prepare(m))) return rc;
  return q4gpu_batch_set_positions(m->b_slots + first_slot, n_seq, position, m->b_lm_from + first_slot, lm_from,
                                   m->stream);
}

int q4gpu_batch_run_step(q4gpu_model* m, int32_t first_slot, int32_t n_seq, const uint32_t* token_ids,
                         const uint32_t* positions, uint32_t* out_tokens, int64_t* out_scores) {
  if (!m || !token_ids || !positions || !out_tokens) return q4gpu_fail(Q4GPU_ERR_ARG, "null argument");
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  for (int i = 0; i < n_seq; ++i)
    if (token_ids[i] >= (uint32_t)m->cfg.vocab || positions[i] >= (uint32_t)m->cfg.max_context)
      return q4gpu_fail(Q4GPU_ERR_ARG, "sequence %d: token %u / position %u out of range", i, token_ids[i],
                        positions[i]);
  cudaGraphExec_t g;
  if ((rc = batch_graph(m, first_slot, n_seq, &g))) return rc;
  int32_t* hin = m->h_bio;
  int32_t* hout = m->h_bio + 2 * kBatchSeqMax;
  for (int i = 0; i < n_seq; ++i) {
    hin[2 * i] = (int32_t)token_ids[i];
    hin[2 * i + 1] = (int32_t)positions[i];
  }
  const SlotState* slots = m->b_slots + first_slot;
  Q4_CUDA(cudaMemcpyAsync(m->b_io, hin, (size_t)n_seq * 8, cudaMemcpyHostToDevice, m->stream));
  if ((rc = q4gpu_batch_load(slots, n_seq, m->b_io, m->b_lm_from + first_slot, m->stream))) return rc;
  Q4_CUDA(cudaGraphLaunch(g, m->stream));
  if ((rc = q4gpu_batch_gather(slots, n_seq, m->b_io, m->b_io + 2 * kBatchSeqMax, m->stream))) return rc;
  Q4_CUDA(cudaMemcpyAsync(hout, m->b_io + 2 * kBatchSeqMax, (size_t)n_seq * 16, cudaMemcpyDeviceToHost, m->stream));
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  if ((rc = batch_check_error(m))) return rc;
  for (int i = 0; i < n_seq; ++i) {
    out_tokens[i] = (uint32_t)hout[4 * i];
    if (out_scores) memcpy(&out_scores[i], &hout[4 * i + 2], 8);
  }
  return Q4GPU_OK;
}

int q4gpu_decode_steps(q4gpu_model* m, uintptr_t base, int32_t n_steps) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || n_steps < 0) return q4gpu_fail(Q4GPU_ERR_ARG, "bad decode_steps");
  int rc = set_device(m);
  if (rc) return rc;
  if (m->mode == 1) return run_persistent(m, (int)base, n_steps, 0);
  cudaGraphExec_t g;
  if ((rc = get_graph(m, GraphKey{(int)base, 0, m->cfg.n_layers, 1, 1}, &g))) return rc;
  for (int i = 0; i < n_steps; ++i) Q4_CUDA(cudaGraphLaunch(g, m->stream));
  return Q4GPU_OK;
}

int q4gpu_model_trace_persistent(q4gpu_model* m, uintptr_t base, int32_t n_steps, int32_t lm_from,
                                 uint64_t* stamps, int32_t n_barriers) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || n_steps <= 0 || !stamps || n_barriers <= 0)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad trace request");
  if (m->p_grid == 0) return q4gpu_fail(Q4GPU_ERR_SHAPE, "persistent kernel unavailable");
  int rc = set_device(m);
  if (rc) return rc;
  unsigned long long* dev = nullptr;
  Q4_CUDA(cudaMalloc(&dev, (size_t)n_barriers * 2 * sizeof(unsigned long long)));
  bool ok = cudaMemsetAsync(dev, 0, (size_t)n_barriers * 16, m->stream) == cudaSuccess &&
            run_persistent(m, (int)base, n_steps, lm_from, dev, n_barriers) == Q4GPU_OK &&
            cudaStreamSynchronize(m->stream) == cudaSuccess &&
            cudaMemcpy(stamps, dev, (size_t)n_barriers * 16, cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(dev);
  if (!ok) return q4gpu_fail(Q4GPU_ERR_CUDA, "trace run failed");
  return check_persistent_error(m);
}

int q4gpu_model_set_mode(q4gpu_model* m, int32_t mode) {
  if (!m || (mode != 0 && mode != 1)) return q4gpu_fail(Q4GPU_ERR_ARG, "mode must be 0 or 1");
  if (mode == 1 && m->p_grid == 0) return q4gpu_fail(Q4GPU_ERR_SHAPE, "persistent kernel unavailable");
  m->mode = mode;
  return Q4GPU_OK;
}

int32_t q4gpu_model_get_mode(q4gpu_model* m) { return m ? m->mode : -1; }

int q4gpu_model_set_position(q4gpu_model* m, uintptr_t base, int32_t position) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || position < 0 || position >= m->cfg.max_context)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad set_position");
  int rc = set_device(m);
  if (rc) return rc;
  // a one-thread kernel keeps this stream-ordered without a host round trip
  Q4_CUDA(launch_k(set_pos_kernel, dim3(1), dim3(32), 0, m->stream, m->slots[base], (int)position));
  return Q4GPU_OK;
}

int q4gpu_model_sync(q4gpu_model* m) {
  if (!m) return q4gpu_fail(Q4GPU_ERR_ARG, "null model");
  int rc = set_device(m);
  if (rc) return rc;
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  for (size_t i = 0; i < m->busy.size(); ++i) m->busy[i] = 0;
  if ((rc = batch_check_error(m))) return rc;
  return check_persistent_error(m);
}

int q4gpu_model_read_tokens(q4gpu_model* m, uintptr_t base, int32_t start, int32_t n, int32_t* tokens,
                            int64_t* scores, int32_t* position) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || start < 0 || n < 0 || start + n > m->cfg.max_context + 2)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad read_tokens");
  int rc = set_device(m);
  if (rc) return rc;
  const SlotState& st = m->slots[base];
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  if (n && tokens) Q4_CUDA(cudaMemcpy(tokens, st.tokens + start, (size_t)n * 4, cudaMemcpyDeviceToHost));
  if (n && scores) Q4_CUDA(cudaMemcpy(scores, st.scores + start, (size_t)n * 8, cudaMemcpyDeviceToHost));
  if (position) Q4_CUDA(cudaMemcpy(position, st.pos, 4, cudaMemcpyDeviceToHost));
  return Q4GPU_OK;
}

int q4gpu_model_time_kernels(q4gpu_model* m, uintptr_t base, int32_t reps, double* ms_per_launch,
                             int32_t* launches_per_step) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || reps <= 0 || !ms_per_launch || !launches_per_step)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad time_kernels");
  int rc = set_device(m);
  if (rc) return rc;
  double tot[Q4GPU_K_COUNT] = {0};
  int cnt[Q4GPU_K_COUNT] = {0};
  for (int r = 0; r < reps; ++r) {
    KernelMarks mk;
    if ((rc = enqueue_step(m, (int)base, 0, m->cfg.n_layers, 1, 1, &mk))) return rc;
    Q4_CUDA(cudaStreamSynchronize(m->stream));
    for (size_t i = 0; i + 1 < mk.ev.size(); ++i) {
      float ms = 0.f;
      Q4_CUDA(cudaEventElapsedTime(&ms, mk.ev[i], mk.ev[i + 1]));
      tot[mk.kind[i]] += ms;
      cnt[mk.kind[i]] += 1;
    }
  }
  for (int k = 0; k < Q4GPU_K_COUNT; ++k) {
    ms_per_launch[k] = cnt[k] ? tot[k] / cnt[k] : 0.0;
    launches_per_step[k] = cnt[k] / reps;
  }
  return Q4GPU_OK;
}

int q4gpu_model_time_layers(q4gpu_model* m, uintptr_t base, int32_t layer_start, int32_t layer_count,
                            int32_t position, int32_t reps, double* ms) {
  if (!m || base >= (uintptr_t)m->cfg.max_seqs || layer_start < 0 || layer_count <= 0 ||
      layer_start + layer_count > m->cfg.n_layers || position < 0 || position >= m->cfg.max_context || reps <= 0 || !ms)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad time_layers");
  int rc = set_device(m);
  if (rc) return rc;
  std::vector<cudaGraphExec_t> g((size_t)layer_count);
  for (int i = 0; i < layer_count; ++i)
    if ((rc = get_graph(m, GraphKey{(int)base, layer_start + i, 1, 0, 0}, &g[(size_t)i]))) return rc;
  cudaEvent_t e0, e1;
  Q4_CUDA(cudaEventCreate(&e0));
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return q4gpu_fail(Q4GPU_ERR_CUDA, "event create");
  }
  double tot = 0.0;
  for (int r = 0; r < reps + 1 && rc == Q4GPU_OK; ++r)  // the first cycle warms up
    for (int i = 0; i < layer_count && rc == Q4GPU_OK; ++i) {
      float t = 0.f;
      const bool ok =
          launch_k(set_pos_kernel, dim3(1), dim3(32), 0, m->stream, m->slots[base], (int)position) == cudaSuccess &&
          cudaEventRecord(e0, m->stream) == cudaSuccess && cudaGraphLaunch(g[(size_t)i], m->stream) == cudaSuccess &&
          cudaEventRecord(e1, m->stream) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
          cudaEventElapsedTime(&t, e0, e1) == cudaSuccess;
      if (!ok) rc = q4gpu_fail(Q4GPU_ERR_CUDA, "time_layers: %s", cudaGetErrorString(cudaGetLastError()));
      if (r > 0) tot += t;
    }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  if ((rc = check_persistent_error(m))) return rc;
  *ms = tot / ((double)reps * layer_count);
  return Q4GPU_OK;
}

int q4gpu_batch_time_kernels(q4gpu_model* m, int32_t first_slot, int32_t n_seq, int32_t reps, double* ms_per_launch,
                             int32_t* launches_per_step) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  if (reps <= 0 || !ms_per_launch || !launches_per_step) return q4gpu_fail(Q4GPU_ERR_ARG, "bad batch_time_kernels");
  cudaGraphExec_t g;  // makes the buffers, maps and ones rows ready
  if ((rc = batch_graph(m, first_slot, n_seq, &g))) return rc;
  auto pp = std::make_unique<BatchPlan>();
  if ((rc = batch_plan(m, first_slot, n_seq, *pp))) return rc;
  double tot[kBkCount] = {0};
  int cnt[kBkCount] = {0};
  for (int r = 0; r < reps && rc == Q4GPU_OK; ++r) {
    BatchMarks mk;
    rc = q4gpu_enqueue_batch_step(*pp, m->stream, &mk);
    if (rc == Q4GPU_OK && cudaStreamSynchronize(m->stream) != cudaSuccess)
      rc = q4gpu_fail(Q4GPU_ERR_CUDA, "batch_time_kernels sync");
    for (size_t i = 0; rc == Q4GPU_OK && i + 1 < mk.ev.size(); ++i) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, mk.ev[i], mk.ev[i + 1]) != cudaSuccess) {
        rc = q4gpu_fail(Q4GPU_ERR_CUDA, "event timing");
        break;
      }
      tot[mk.kind[i + 1]] += ms;
      cnt[mk.kind[i + 1]] += 1;
    }
    for (cudaEvent_t e : mk.ev) cudaEventDestroy(e);
  }
  if (rc) return rc;
  for (int k = 0; k < kBkCount; ++k) {
    ms_per_launch[k] = cnt[k] ? tot[k] / cnt[k] : 0.0;
    launches_per_step[k] = cnt[k] / reps;
  }
  return batch_check_error(m);
}

int q4gpu_batch_trace(q4gpu_model* m, int32_t first_slot, int32_t n_seq, uint64_t* attn_stamps, int64_t n_attn,
                      uint64_t* gemm_stamps, int64_t n_gemm) {
  int rc = batch_range_ok(m, first_slot, n_seq);
  if (rc) return rc;
  const int64_t need_a = (int64_t)m->cfg.n_layers * n_seq * kKvHeads * 8;
  const int64_t need_g = (int64_t)(4 * m->cfg.n_layers + 1) * kGemmTraceCtas * 8;
  if ((attn_stamps && n_attn != need_a) || (gemm_stamps && n_gemm != need_g))
    return q4gpu_fail(Q4GPU_ERR_ARG, "trace needs %lld attention and %lld GEMM stamps", (long long)need_a,
                      (long long)need_g);
  cudaGraphExec_t g;  // makes the buffers, maps and ones rows ready
  if ((rc = batch_graph(m, first_slot, n_seq, &g))) return rc;
  auto pp = std::make_unique<BatchPlan>();
  if ((rc = batch_plan(m, first_slot, n_seq, *pp))) return rc;
  unsigned long long* dev = nullptr;
  Q4_CUDA(cudaMalloc(&dev, (size_t)(need_a + need_g) * 8));
  pp->trace = attn_stamps ? dev : nullptr;
  pp->gemm_trace = gemm_stamps ? dev + need_a : nullptr;
  bool ok = cudaMemsetAsync(dev, 0, (size_t)(need_a + need_g) * 8, m->stream) == cudaSuccess &&
            q4gpu_enqueue_batch_step(*pp, m->stream) == Q4GPU_OK && cudaStreamSynchronize(m->stream) == cudaSuccess &&
            (!attn_stamps || cudaMemcpy(attn_stamps, dev, (size_t)need_a * 8, cudaMemcpyDeviceToHost) == cudaSuccess) &&
            (!gemm_stamps ||
             cudaMemcpy(gemm_stamps, dev + need_a, (size_t)need_g * 8, cudaMemcpyDeviceToHost) == cudaSuccess);
  cudaFree(dev);
  if (!ok) return q4gpu_fail(Q4GPU_ERR_CUDA, "traced batch step failed");
  return batch_check_error(m);
}

int q4gpu_model_read_hidden(q4gpu_model* m, uintptr_t base, int32_t* hidden) {
  if (!m || !hidden || base >= (uintptr_t)m->cfg.max_seqs) return Q4GPU_ERR_ARG;
  int rc = set_device(m);
  if (rc) return rc;
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  Q4_CUDA(cudaMemcpy(hidden, m->slots[base].hidden, kHidden * 4, cudaMemcpyDeviceToHost));
  return Q4GPU_OK;
}

static int kv_io(q4gpu_model* m, uintptr_t base, int32_t layer, int32_t kind, int32_t positions, int32_t* data,
                 bool to_pool) {
  if (!m || !data || base >= (uintptr_t)m->cfg.max_seqs || layer < 0 || layer >= m->cfg.n_layers || kind < 0 ||
      kind > 1 || positions <= 0 || positions > m->cfg.max_context)
    return q4gpu_fail(Q4GPU_ERR_ARG, "bad kv request");
  int rc = set_device(m);
  if (rc) return rc;
  const size_t n = (size_t)positions * kKvRows;
  int32_t* dev = nullptr;
  Q4_CUDA(cudaMalloc(&dev, n * 4));
  bool ok = true;
  if (to_pool) ok = stream_copy(m, dev, data, n * 4, cudaMemcpyHostToDevice) == Q4GPU_OK;
  if (ok) {
    kv_copy_kernel<<<dim3(positions, kKvHeads), kHeadDim, 0, m->stream>>>(m->slots[base].kv, layer, kind, positions,
                                                                          dev, to_pool ? 1 : 0);
    ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(m->stream) == cudaSuccess;
  }
  if (ok && !to_pool) ok = cudaMemcpy(data, dev, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(dev);
  return ok ? Q4GPU_OK : q4gpu_fail(Q4GPU_ERR_CUDA, "kv copy failed");
}

int q4gpu_model_read_kv(q4gpu_model* m, uintptr_t base, int32_t layer, int32_t kind, int32_t positions,
                        int32_t* out) {
  return kv_io(m, base, layer, kind, positions, out, false);
}

int q4gpu_model_write_kv(q4gpu_model* m, uintptr_t base, int32_t layer, int32_t kind, int32_t positions,
                         const int32_t* data) {
  return kv_io(m, base, layer, kind, positions, const_cast<int32_t*>(data), true);
}

int q4gpu_model_write_hidden(q4gpu_model* m, uintptr_t base, const int32_t* hidden) {
  if (!m || !hidden || base >= (uintptr_t)m->cfg.max_seqs) return Q4GPU_ERR_ARG;
  int rc = set_device(m);
  if (rc) return rc;
  Q4_CUDA(cudaStreamSynchronize(m->stream));
  return stream_copy(m, m->slots[base].hidden, hidden, kHidden * 4, cudaMemcpyHostToDevice);
  return Q4GPU_OK;
}

void q4gpu_build_tables(int32_t* exp_lut, int32_t* sigmoid_lut) { build_luts(exp_lut, sigmoid_lut); }

void q4gpu_build_rope_table(int32_t positions, int32_t* cos_q1_15, int32_t* sin_q1_15) {
  build_rope(positions, cos_q1_15, sin_q1_15);
}

}  // extern "C"
