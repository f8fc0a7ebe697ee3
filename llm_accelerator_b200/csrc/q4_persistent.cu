// Persistent cooperative decode kernel: many batch-1 greedy decode steps of
// one sequence slot in a single launch.
//
// One CTA per SM (512 threads) walks every step through the stages
//   S1  input norm + QKV GEMV (rows split over the grid)      -> qkv (raw Q12.12)
//   S2  q/k head norm + RoPE, KV append, attention            -> attn
//   S3  o_proj + residual                                     -> post
//   S4  post-attention norm + gate/up + SwiGLU                -> mlp
//   S5  down + residual                                       -> hidden
//   ... x layers, then final norm + LM head + argmax           -> next token
// separated by grid-wide barriers.  Nothing that does not depend on this
// step's activations waits behind a barrier: every CTA prefetches into L2 its
// weight slices of the layer ahead, loads its weights of the next stage into
// registers before arriving at the barrier, and copies the K rows and V slice
// of its attention head into shared memory with TMA bulk copies (mbarrier
// completion) while the QKV stage runs.  Attention assigns each KV head to
// kAttnSplit CTAs, each owning a slice of head_dim: every CTA of a head
// recomputes the (cheap) scores, max and exp sum from its shared-memory copy
// of K, so no cross-CTA exchange is needed.
// The argmax is reduced redundantly by every CTA after a barrier, so the
// next step's embedding starts without another one.
//
// Inter-CTA data is read with ld.global.cg (L2) after acquire/release
// barriers; weights use the read-only path.  Every barrier wait is bounded:
// on timeout the kernel sets an error word and all CTAs leave.
#include "q4_gemv.cuh"
#include "q4_state.cuh"
#include "q4gpu_internal.h"

namespace q4 {

constexpr int kPThreads = 512;
constexpr int kPWarps = kPThreads / 32;
constexpr int kAttnSplit = 8;  // CTAs per KV head (head_dim slices of 16)
constexpr int kSliceDims = kHeadDim / kAttnSplit;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kKvWindow = 256;  // cached positions staged in shared memory
constexpr int kAttnCtas = kKvHeads * kAttnSplit;  // CTAs [0, 64): attention + o_proj partial sums
constexpr int kGuCtas = kInter / kGroup;          // CTAs [64, 112): 64 gate/up rows each + down partial sums

// ---- memory-model helpers ---------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int32_t ldcg(const int32_t* p) { return __ldcg(p); }
__device__ __forceinline__ int4 ldcg4(const int32_t* p) { return __ldcg(reinterpret_cast<const int4*>(p)); }

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier / bulk-copy helpers (shared memory of this CTA) --------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(b))
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(b))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bounded wait for phase `parity` of *b; false if it ran out (error word set,
// then one more bounded wait so no copy is still landing when the CTA exits).
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, int* err) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 1023) == 1023 && *((volatile int*)err) != 0) break;
  }
  atomicCAS(err, 0, 3);
  for (uint32_t it = 0; it < kSpinLimit && !mbar_try_wait(b, parity); ++it) {
  }
  return false;
}

// Grid-wide barrier on one monotonic arrival counter bar[0] (zeroed by the
// host before each launch): barrier i of a launch releases when the counter
// reaches (i + 1) x gridDim.x.  The arrival is one release add, the wait an
// acquire poll of the same word, so the release costs a single trip to L2.
struct Barrier {
  unsigned* bar;
  int* err;
  int* s_flag;
  unsigned long long* trace;
  int trace_cap;
  unsigned index;
};

struct NoHook {
  __device__ void operator()() const {}
};

template <class Hook = NoHook>
__device__ __forceinline__ bool grid_sync(Barrier& b, Hook hook = Hook()) {
  __syncthreads();
  const unsigned idx = b.index++;
  if (threadIdx.x == 0) {
    if (b.trace && (int)idx < b.trace_cap) atomicMax(&b.trace[2 * idx], globaltimer());
    const unsigned target = (idx + 1) * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(b.bar) : "memory");
    int ok = 1;
    uint32_t it = 0;
    while (ld_acquire_u32(b.bar) < target) {
      if (++it > kSpinLimit || ((it & 255) == 0 && *((volatile int*)b.err) != 0)) {
        atomicCAS(b.err, 0, 1);
        ok = 0;
        break;
      }
    }
    if (b.trace && blockIdx.x == 0 && (int)idx < b.trace_cap) b.trace[2 * idx + 1] = globaltimer();
    *b.s_flag = ok;
  } else if (threadIdx.x == 32) {
    hook();
  }
  __syncthreads();
  return *b.s_flag != 0;
}

__device__ __forceinline__ int part_of(int n, int i, int g) { return (int)(((int64_t)n * i) / g); }

// Limbs of K activations in shared memory, one 8-element chunk per thread.
__device__ __forceinline__ void stage_limbs_par(const int32_t* act, int K, uint32_t* limbs, int64_t* bias8) {
  const int c = threadIdx.x;
  int64_t s = 0;
  if (c < K / 8) {
    make_limbs8(act + 8 * c, limbs + (c >> 2) * kLimbStride + (c & 3) * 6);
#pragma unroll
    for (int e = 0; e < 8; ++e) s += act[8 * c + e];
  }
  s += shfl_xor_i64(s, 1);
  s += shfl_xor_i64(s, 2);
  if (c < K / 8 && (c & 3) == 0) bias8[c >> 2] = 8 * s;
}

// This thread's two hidden-size gamma values (elements t and t + 512), loaded
// at a stage's start so the read overlaps the stage's input read.
struct Gamma2 {
  int32_t v[2];
  __device__ __forceinline__ explicit Gamma2(const int32_t* __restrict__ g) {
    v[0] = __ldg(g + threadIdx.x);
    v[1] = __ldg(g + threadIdx.x + kPThreads);
  }
};
static_assert(2 * kPThreads == kHidden, "two hidden elements per thread");

// Hidden-size RMSNorm of act[] in place (Q14.10 -> Q12.12).
__device__ __forceinline__ void hidden_norm_inplace(int32_t* act, const Gamma2& gamma, int64_t* red) {
  const int i0 = threadIdx.x, i1 = threadIdx.x + kPThreads;
  const int32_t x0 = act[i0], x1 = act[i1];
  const int64_t ss = block_sum_i64((int64_t)x0 * x0 + (int64_t)x1 * x1, red);
  const int64_t inv = inv_rms_from_ss(ss, kHiddenNorm);
  act[i0] = norm_apply(x0, inv, gamma.v[0], kHiddenNorm);
  act[i1] = norm_apply(x1, inv, gamma.v[1], kHiddenNorm);
}

// Block-wide max (and sum) of two int64 values at once; red needs 32 slots.
// Every warp finishes the per-warp partials with shuffles.
__device__ __forceinline__ void block_max2(int64_t& x, int64_t& y, int64_t* red) {
  x = warp_max_i64(x);
  y = warp_max_i64(y);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[2 * warp] = x;
    red[2 * warp + 1] = y;
  }
  __syncthreads();
  x = warp_max_i64(lane < nw ? red[2 * lane] : INT64_MIN);
  y = warp_max_i64(lane < nw ? red[2 * lane + 1] : INT64_MIN);
}

__device__ __forceinline__ void block_sum2(int64_t& x, int64_t& y, int64_t* red) {
  x = warp_sum_i64(x);
  y = warp_sum_i64(y);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[2 * warp] = x;
    red[2 * warp + 1] = y;
  }
  __syncthreads();
  x = warp_sum_i64(lane < nw ? red[2 * lane] : 0);
  y = warp_sum_i64(lane < nw ? red[2 * lane + 1] : 0);
}

// ---- GEMV items with weights preloaded into registers -----------------------
// Item `it` is row row_of(it / KS) of a matrix at K-slice it % KS; warp w owns
// items w, w + 16, ..., (RMAX of them).  The preload runs before a barrier,
// the compute after it.
template <int K, int RMAX>
struct Pre {
  uint4 w[RMAX];
  uint32_t sc[RMAX];
};

template <int K, int RMAX, class RowFn>
__device__ __forceinline__ void preload_items(int n_items, RowFn row_of, Pre<K, RMAX>& pre) {
  constexpr int KS = K / 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < RMAX; ++j) {
    const int it = warp + j * kPWarps;
    if (it < n_items) {
      const uint8_t* W;
      const uint16_t* S;
      row_of(it / KS, W, S);
      const int hg = (it % KS) * 32 + lane;
      pre.w[j] = ldg_stream(W + (size_t)hg * 16);
      pre.sc[j] = __ldg(S + (hg >> 1));
    } else {
      pre.w[j] = make_uint4(0, 0, 0, 0);
      pre.sc[j] = 0;
    }
  }
}

// Sum over the warp of R per-lane values at once (R = 2, 8): halving exchanges
// leave lane l with the total of value (l >> 2) % R ... for R = 8, (l >> 4) % 2
// for R = 2; returns it.
template <int R>
__device__ __forceinline__ int64_t warp_sum_multi(int64_t (&v)[R], int lane) {
  if constexpr (R == 8) {
    const bool h = lane & 16, g = lane & 8, b = lane & 4;
    int64_t x[4], y[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = (h ? v[i + 4] : v[i]) + shfl_xor_i64(h ? v[i] : v[i + 4], 16);
#pragma unroll
    for (int i = 0; i < 2; ++i) y[i] = (g ? x[i + 2] : x[i]) + shfl_xor_i64(g ? x[i] : x[i + 2], 8);
    int64_t z = (b ? y[1] : y[0]) + shfl_xor_i64(b ? y[0] : y[1], 4);
    z += shfl_xor_i64(z, 2);
    z += shfl_xor_i64(z, 1);
    return z;
  } else {
    static_assert(R == 2, "R = 2 or 8");
    const bool h = lane & 16;
    int64_t z = (h ? v[1] : v[0]) + shfl_xor_i64(h ? v[0] : v[1], 16);
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) z += shfl_xor_i64(z, m);
    return z;
  }
}

template <int K, int RMAX>
__device__ __forceinline__ void compute_items(int n_items, const Pre<K, RMAX>& pre, const uint32_t* limbs,
                                              const int64_t* bias8, int64_t* part) {
  constexpr int KS = K / 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if constexpr (RMAX == 2 && KS == 1) {
    // one half-group of limbs serves both items; both sums leave one butterfly
    const uint32_t* l = limbs + lane * kLimbStride;
    uint32_t l24[24];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const uint4 t = reinterpret_cast<const uint4*>(l)[i];
      l24[4 * i] = t.x;
      l24[4 * i + 1] = t.y;
      l24[4 * i + 2] = t.z;
      l24[4 * i + 3] = t.w;
    }
    int64_t v[2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
      v[j] = warp + j * kPWarps < n_items ? lane_span(pre.w[j], l24, bias8[lane], pre.sc[j]) : 0;
    const int64_t tot = warp_sum_multi<2>(v, lane);
    const int it = warp + ((lane >> 4) & 1) * kPWarps;
    if ((lane & 15) == 0 && it < n_items) part[it] = tot;
  } else {
#pragma unroll
    for (int j = 0; j < RMAX; ++j) {
      const int it = warp + j * kPWarps;
      if (it < n_items) {
        const int hg = (it % KS) * 32 + lane;
        const uint32_t* l = limbs + hg * kLimbStride;
        uint32_t l24[24];
#pragma unroll
        for (int i = 0; i < 6; ++i) {
          const uint4 t = reinterpret_cast<const uint4*>(l)[i];
          l24[4 * i] = t.x;
          l24[4 * i + 1] = t.y;
          l24[4 * i + 2] = t.z;
          l24[4 * i + 3] = t.w;
        }
        const int64_t v = warp_sum_i64(lane_span(pre.w[j], l24, bias8[hg], pre.sc[j]));
        if (lane == 0) part[it] = v;
      }
    }
  }
}

struct PSmem {
  int32_t* act;       // [3072]
  uint32_t* limbs;    // [96 * 28]
  int64_t* bias8;     // [96]
  int64_t* part;      // [256]
  int64_t* red;       // [32]
  int64_t* sc;        // [2 * score_cap]
  uint64_t* probtab;  // [2 * 257]
  int32_t* hv;        // [4 * 128]: q0, q1, k, v of the attention head
  int64_t* vacc;      // [32 * kSliceDims * 2]
  int32_t* kwin;      // [kKvWindow * 128]: cached K rows of the attention head
  int32_t* vwin;      // [kKvWindow * kSliceDims]: cached V of this CTA's dims
  uint64_t* mbar;     // [5]: KV copy completion, then 4 LM-head ring slots
  int32_t* hid;       // [1024]: the layer's input hidden state (Q14.10), every CTA a full copy
  int32_t* post;      // [1024]: the post-attention hidden state (Q14.10), every CTA a full copy
  int* flag;
  int32_t* exp_lut;   // [257] softmax LUT
  int32_t* sig_lut;   // [1025] sigmoid LUT
  int32_t* rope;      // [256]: cos, sin rows of the step's position
};

constexpr int kLmChunkRows = 64;  // LM-head rows per ring slot (32 KB + 2 KB)
constexpr int kLmRing = 4;

// ---- prefetch of the weights this CTA reads later ---------------------------
// L2 prefetch of a byte range in pieces of at most 32 KB.
__device__ __forceinline__ void prefetch_range(const void* p, size_t bytes) {
  const char* c = static_cast<const char*>(p);
  for (size_t off = 0; off < bytes; off += 32768)
    prefetch_l2(c + off, (uint32_t)(bytes - off < 32768 ? bytes - off : 32768));
}

__device__ __forceinline__ void prefetch_rows(const uint8_t* W, const uint16_t* S, int K, int r0, int r1) {
  if (r1 > r0) {
    prefetch_range(W + (size_t)r0 * (K / 2), (size_t)(r1 - r0) * (K / 2));
    prefetch_range(S + (size_t)r0 * (K / 64), (size_t)(r1 - r0) * (K / 64) * 2);
  }
}

__device__ void prefetch_layer(const LayerW& w, int cta, int G) {
  prefetch_rows(w.wqkv, w.sqkv, kHidden, part_of(4096, cta, G), part_of(4096, cta + 1, G));
  prefetch_rows(w.wo, w.so, 2 * kHidden, part_of(kHidden, cta, G), part_of(kHidden, cta + 1, G));
  const int g0 = part_of(kInter, cta, G), g1 = part_of(kInter, cta + 1, G);
  prefetch_rows(w.wgate, w.sgate, kHidden, g0, g1);
  prefetch_rows(w.wup, w.sup, kHidden, g0, g1);
  prefetch_rows(w.wdown, w.sdown, kInter, part_of(kHidden, cta, G), part_of(kHidden, cta + 1, G));
}

// TMA copies of head h's cached K rows [0, n) (1-D bulk, one per page) and
// V dims [d0, d0+16) (2-D tensor map, one 64 x 16 box per page) of `layer`
// into shared memory; completion on sm.mbar[0] (one phase).
__device__ void issue_kv_copies(const PersistArgs& a, const PSmem& sm, int layer, int n) {
  const int h = blockIdx.x / kAttnSplit, d0 = (blockIdx.x % kAttnSplit) * kSliceDims;
  // order earlier generic reads of the windows and the (acquired) generic
  // writes of the KV rows by other CTAs before the async-proxy copies
  fence_proxy_async();
  asm volatile("fence.proxy.async.global;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    const int pages = (n + kKvPage - 1) / kKvPage;
    mbar_arrive_expect_tx(sm.mbar, (unsigned)n * kHeadDim * 4 + (unsigned)pages * kKvPage * kSliceDims * 4);
    for (int pg = 0; pg < pages; ++pg) {
      const int p0 = pg * kKvPage;
      bulk_g2s(sm.kwin + p0 * kHeadDim, a.st.kv.at(layer, 0, h, p0), (unsigned)min(kKvPage, n - p0) * kHeadDim * 4,
               sm.mbar);
      const int row = (int)((((int64_t)a.st.kv.pages[pg] * a.n_layers + layer) * 2 + 1) * kKvHeads + h) * kKvPage;
      tma_load_2d(sm.vwin + p0 * kSliceDims, &a.vmap, d0, row, sm.mbar);
    }
  }
}

// LM-head chunk `j` of this CTA's rows into ring slot j % kLmRing.
__device__ __forceinline__ void issue_lm_chunk(const PersistArgs& a, const PSmem& sm, int r0, int r1, int j) {
  const int c0 = r0 + j * kLmChunkRows;
  if (c0 >= r1) return;
  const int rows = min(kLmChunkRows, r1 - c0);
  const int slot = j % kLmRing;
  uint64_t* mb = sm.mbar + 1 + slot;
  mbar_arrive_expect_tx(mb, (unsigned)rows * (512 + 32));
  bulk_g2s(reinterpret_cast<uint8_t*>(sm.kwin) + (size_t)slot * kLmChunkRows * 512, a.emb + (size_t)c0 * 512,
           (unsigned)rows * 512, mb);
  bulk_g2s(reinterpret_cast<uint8_t*>(sm.vwin) + (size_t)slot * kLmChunkRows * 32, a.semb + (size_t)c0 * 16,
           (unsigned)rows * 32, mb);
}

// ---- stages -----------------------------------------------------------------
using PreQkv = Pre<kHidden, 2>;

__device__ __forceinline__ void preload_qkv(const LayerW& w, PreQkv& pre) {
  const int r0 = part_of(4096, blockIdx.x, gridDim.x), r1 = part_of(4096, blockIdx.x + 1, gridDim.x);
  preload_items(r1 - r0, [&](int r, const uint8_t*& W, const uint16_t*& S) {
    W = w.wqkv + (size_t)(r0 + r) * 512;
    S = w.sqkv + (size_t)(r0 + r) * 16;
  }, pre);
}

__device__ __forceinline__ int32_t nibble(uint32_t w, int k) { return (int32_t)(w << (28 - 4 * k)) >> 28; }
__device__ __forceinline__ void red_add_i64(int64_t* p, int64_t v) {
  atomicAdd(reinterpret_cast<unsigned long long*>(p), (unsigned long long)v);
}
__device__ __forceinline__ int64_t ldcg64(const int64_t* p) {
  return (int64_t)__ldcg(reinterpret_cast<const long long*>(p));
}
// split-K partial sums of the layer with parity `par`: o_proj in buffer par,
// down in buffer 2 + par; each row's sum owns a 32-byte sector (kAccStride
// int64) so the atomic adds of the contributing CTAs spread over more L2 lines
constexpr int kAccStride = 4;
__device__ __forceinline__ int64_t* acc_row(const PersistArgs& a, int buf, int row) {
  return a.acc + ((size_t)buf * kHidden + row) * kAccStride;
}

// o_proj columns fed by attention CTA (h, slice): for rows t and t + 512, the 16
// columns (8 bytes) of each of its two q heads and the scale of their group
// (16 columns starting at a multiple of 16 never straddle a 64-column group),
// read from the regrouped copy (LayerW::wo_sl) with coalesced 16-byte loads.
struct OSlice {
  uint2 w[2][2];
  uint32_t s[2][2];
};
__device__ __forceinline__ void preload_oslice(const LayerW& w, OSlice& o) {
  const uint4* src = reinterpret_cast<const uint4*>(w.wo_sl) + (size_t)blockIdx.x * kHidden;
  const uint32_t* ss = reinterpret_cast<const uint32_t*>(w.so_sl) + (size_t)blockIdx.x * kHidden;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = threadIdx.x + r * kPThreads;
    const uint4 v = __ldg(src + row);
    const uint32_t s2 = __ldg(ss + row);
    o.w[r][0] = make_uint2(v.x, v.y);
    o.w[r][1] = make_uint2(v.z, v.w);
    o.s[r][0] = s2 & 0xFFFFu;
    o.s[r][1] = s2 >> 16;
  }
}

// Regroup every layer's o_proj columns into the attention CTAs' slices (run
// whenever the weights change): grid (64 slices, layers).
__global__ void oslice_layout_kernel(const LayerW* __restrict__ layers) {
  const LayerW w = layers[blockIdx.y];
  const int c = blockIdx.x, h = c / kAttnSplit, d0 = (c % kAttnSplit) * kSliceDims;
  uint4* dst = reinterpret_cast<uint4*>(const_cast<uint8_t*>(w.wo_sl)) + (size_t)c * kHidden;
  uint32_t* ds = reinterpret_cast<uint32_t*>(const_cast<uint16_t*>(w.so_sl)) + (size_t)c * kHidden;
  for (int row = threadIdx.x; row < kHidden; row += blockDim.x) {
    uint2 v[2];
    uint32_t sc[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int col = (2 * h + hh) * kHeadDim + d0;
      v[hh] = *reinterpret_cast<const uint2*>(w.wo + (size_t)row * kHidden + col / 2);
      sc[hh] = w.so[(size_t)row * (2 * kHidden / kGroup) + col / kGroup];
    }
    dst[row] = make_uint4(v[0].x, v[0].y, v[1].x, v[1].y);
    ds[row] = sc[0] | (sc[1] << 16);
  }
}

// down columns [64 gc, 64 gc + 64) (this gate/up CTA's rows, one scale group)
// of every row and their scales, staged in the CTA's K-window buffer (gate/up
// CTAs run no attention): 32 bytes per row, then the 1024 scales.
__device__ __forceinline__ uint4* dslice_w(const PSmem& sm) { return reinterpret_cast<uint4*>(sm.kwin); }
__device__ __forceinline__ uint32_t* dslice_s(const PSmem& sm) {
  return reinterpret_cast<uint32_t*>(sm.kwin + 2 * kHidden * 4);
}
// gate/up CTA gc owns gate and up rows [64 gc, 64 gc + 64) (items 0..63 gate,
// 64..127 up); their packed rows sit in the K-window buffer after the down
// slice: item it, lane l -> 16 bytes at gu_w[32 it + l], its half-group scale at gu_s[32 it + l].
constexpr int kGuItems = 2 * kGroup;
constexpr int kGuWOffset = 2 * kHidden * 16 + kHidden * 4;
__device__ __forceinline__ uint4* gu_w(const PSmem& sm) {
  return reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.kwin) + kGuWOffset);
}
__device__ __forceinline__ uint32_t* gu_s(const PSmem& sm) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sm.kwin) + kGuWOffset + kGuItems * 32 * 16);
}
static_assert(kGuWOffset + kGuItems * 32 * 20 <= kKvWindow * kHeadDim * 4, "gate/up staging exceeds the K window");
__device__ __forceinline__ void preload_gateup(const LayerW& w, int gc, const PSmem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kGuItems / kPWarps; ++j) {
    const int it = warp + j * kPWarps;
    const bool up = it >= kGroup;
    const int row = gc * kGroup + (up ? it - kGroup : it);
    const uint8_t* W = (up ? w.wup : w.wgate) + (size_t)row * 512;
    const uint16_t* S = (up ? w.sup : w.sgate) + (size_t)row * 16;
    const uint4 v = ldg_stream(W + lane * 16);
    const uint32_t sc = __ldg(S + (lane >> 1));
    gu_w(sm)[it * 32 + lane] = v;
    gu_s(sm)[it * 32 + lane] = sc;
  }
}

__device__ __forceinline__ void preload_dslice(const LayerW& w, int gc, const PSmem& sm) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = threadIdx.x + r * kPThreads;
    const uint4* p = reinterpret_cast<const uint4*>(w.wdown + (size_t)row * (kInter / 2) + gc * (kGroup / 2));
    const uint4 w0 = __ldg(p), w1 = __ldg(p + 1);
    const uint32_t sc = __ldg(w.sdown + (size_t)row * (kInter / kGroup) + gc);
    dslice_w(sm)[2 * row] = w0;
    dslice_w(sm)[2 * row + 1] = w1;
    dslice_s(sm)[row] = sc;
  }
}

// Layer input hidden state, every CTA the whole vector: the embedding (layer 0,
// already in hid) or post + (down >> 2) of the previous layer from its partial sums.
// (two elements per thread, both partial sums requested before either is used)
__device__ __forceinline__ void build_hidden(const PersistArgs& a, const PSmem& sm, int par_prev) {
  const int i0 = threadIdx.x, i1 = threadIdx.x + kPThreads;
  const int64_t d0 = ldcg64(acc_row(a, 2 + par_prev, i0)), d1 = ldcg64(acc_row(a, 2 + par_prev, i1));
  sm.hid[i0] = sat24((int64_t)sm.post[i0] + (sat24(d0 >> 14) >> 2));
  sm.hid[i1] = sat24((int64_t)sm.post[i1] + (sat24(d1 >> 14) >> 2));
}

__device__ void stage_qkv(const PersistArgs& a, const LayerW& w, const PSmem& sm, bool first_layer, int par_prev,
                          const PreQkv& pre) {
  const int G = gridDim.x, cta = blockIdx.x;
  const Gamma2 gamma(w.g_in);
  if (!first_layer) build_hidden(a, sm, par_prev);
  __syncthreads();
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) sm.act[i] = sm.hid[i];
  __syncthreads();
  hidden_norm_inplace(sm.act, gamma, sm.red);
  __syncthreads();
  stage_limbs_par(sm.act, kHidden, sm.limbs, sm.bias8);
  __syncthreads();
  const int r0 = part_of(4096, cta, G), r1 = part_of(4096, cta + 1, G);
  compute_items(r1 - r0, pre, sm.limbs, sm.bias8, sm.part);
  __syncthreads();
  for (int i = threadIdx.x; i < r1 - r0; i += blockDim.x) a.qkv[r0 + i] = sat24(sm.part[i] >> 14);
}

// returns false on a copy timeout
__device__ bool stage_attention(const PersistArgs& a, const LayerW& w, const PSmem& sm, int layer, int pos, int par,
                                unsigned& mbar_phase, const OSlice& os) {
  const int cta = blockIdx.x;
  if (cta == (int)gridDim.x - 1) {
    // the other parity's partial sums are free now (last read before this
    // layer's first barrier, next written after this stage's barrier)
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
      __stcg(reinterpret_cast<long long*>(acc_row(a, par ^ 1, i)), 0ll);
      __stcg(reinterpret_cast<long long*>(acc_row(a, 2 + (par ^ 1), i)), 0ll);
    }
  }
  if (cta >= kAttnCtas) return true;
  const int h = cta / kAttnSplit, sl = cta % kAttnSplit, d0 = sl * kSliceDims;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int ctx = pos + 1;
  int32_t* q0 = sm.hv;
  int32_t* q1 = sm.hv + kHeadDim;
  int32_t* kc = sm.hv + 2 * kHeadDim;
  int32_t* vc = sm.hv + 3 * kHeadDim;
  // raw q (2 heads), k, v of this KV head; then per-head norm and RoPE
  int32_t raw = 0, gam = 0;
  if (t < 3 * kHeadDim) {
    const int which = t / kHeadDim, d = t % kHeadDim;
    const int row = which < 2 ? (2 * h + which) * kHeadDim + d : kQRows + h * kHeadDim + d;
    gam = __ldg((which < 2 ? w.g_q : w.g_k) + d);
    raw = ldcg(a.qkv + row);
  } else if (t < 4 * kHeadDim) {
    vc[t - 3 * kHeadDim] = ldcg(a.qkv + kQRows + kKvRows + h * kHeadDim + (t - 3 * kHeadDim));
  }
  int64_t sq = t < 3 * kHeadDim ? (int64_t)raw * raw : 0;
  sq = warp_sum_i64(sq);
  if (lane == 0) sm.red[warp] = sq;
  __syncthreads();
  if (t < 3 * kHeadDim) {
    const int which = t / kHeadDim, d = t % kHeadDim;
    const int64_t ss = sm.red[which * 4] + sm.red[which * 4 + 1] + sm.red[which * 4 + 2] + sm.red[which * 4 + 3];
    const int64_t inv = inv_rms_from_ss(ss, kHeadNorm);
    sm.hv[which * kHeadDim + d] = norm_apply(raw, inv, gam, kHeadNorm);
  }
  __syncthreads();
  int32_t rot_v = 0;
  if (t < 3 * kHeadDim) {
    const int which = t / kHeadDim, d = t % kHeadDim;
    const int32_t* x = sm.hv + which * kHeadDim;
    const int64_t rot = d < 64 ? -(int64_t)x[d + 64] : (int64_t)x[d - 64];
    rot_v = sat24(((int64_t)x[d] * sm.rope[d] + rot * sm.rope[kHeadDim + d]) >> 15);
  }
  __syncthreads();
  if (t < 3 * kHeadDim) sm.hv[t] = rot_v;
  if (sl == 0 && t >= 3 * kHeadDim && t < 4 * kHeadDim) {
    // this position's V goes to the cache (K below, after RoPE is in smem)
    a.st.kv.at(layer, 1, h, pos)[t - 3 * kHeadDim] = vc[t - 3 * kHeadDim];
    vpl_put1(a.st.kv, layer, h, pos, t - 3 * kHeadDim, vc[t - 3 * kHeadDim]);
  }
  __syncthreads();
  if (sl == 0 && t < kHeadDim) {
    a.st.kv.at(layer, 0, h, pos)[t] = kc[t];
    kpl_put1(a.st.kv, layer, h, pos, t, kc[t]);
  }
  // the cached K rows and V slice were copied into shared memory during QKV
  if (!mbar_wait(sm.mbar, mbar_phase, a.err)) return false;
  mbar_phase ^= 1u;
  // scores: 8 threads per position, thread c owns dims {4c + 32j + e}
  {
    const int pp = t >> 3, c = t & 7;
    int32_t qa[16], qb[16];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qa[4 * j + e] = q0[4 * c + 32 * j + e];
        qb[4 * j + e] = q1[4 * c + 32 * j + e];
      }
    const int64_t scale = 189812531LL;
    for (int p0 = 0; p0 < ctx; p0 += kPThreads / 8) {
      const int p = p0 + pp;
      int64_t s0 = 0, s1 = 0;
      if (p < ctx) {
        const int32_t* krow = p == pos ? kc : sm.kwin + p * kHeadDim;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 k4 = *reinterpret_cast<const int4*>(krow + 4 * c + 32 * j);
          s0 += (int64_t)qa[4 * j] * k4.x + (int64_t)qa[4 * j + 1] * k4.y + (int64_t)qa[4 * j + 2] * k4.z +
                (int64_t)qa[4 * j + 3] * k4.w;
          s1 += (int64_t)qb[4 * j] * k4.x + (int64_t)qb[4 * j + 1] * k4.y + (int64_t)qb[4 * j + 2] * k4.z +
                (int64_t)qb[4 * j + 3] * k4.w;
        }
      }
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        s0 += shfl_xor_i64(s0, m);
        s1 += shfl_xor_i64(s1, m);
      }
      if (c == 0 && p < ctx) {
        sm.sc[p] = scale_score(s0, scale);
        sm.sc[a.score_cap + p] = scale_score(s1, scale);
      }
    }
  }
  __syncthreads();
  {
    int64_t* s0 = sm.sc;
    int64_t* s1 = sm.sc + a.score_cap;
    int64_t m0 = INT64_MIN, m1 = INT64_MIN;
    for (int p = t; p < ctx; p += blockDim.x) {
      m0 = s0[p] > m0 ? s0[p] : m0;
      m1 = s1[p] > m1 ? s1[p] : m1;
    }
    block_max2(m0, m1, sm.red);
    int64_t e0 = 0, e1 = 0;
    for (int p = t; p < ctx; p += blockDim.x) {
      const int i0 = lut_index(m0, s0[p]), i1 = lut_index(m1, s1[p]);
      s0[p] = i0;
      s1[p] = i1;
      e0 += sm.exp_lut[i0];
      e1 += sm.exp_lut[i1];
    }
    block_sum2(e0, e1, sm.red);
    for (int i = t; i < 2 * kExpLut; i += blockDim.x) {
      const int hh = i / kExpLut, k = i % kExpLut;
      sm.probtab[i] = udiv_exact((uint64_t)sm.exp_lut[k] << 16, (uint64_t)(hh ? e1 : e0));  // operands < 2^53
    }
  }
  __syncthreads();
  // sum(prob * v) over this CTA's head_dim slice: thread = (dim, position lane)
  {
    const int dl = t % kSliceDims, pl = t / kSliceDims;  // pl in [0, 32)
    int64_t acc0 = 0, acc1 = 0;
    for (int p = pl; p < ctx; p += kPThreads / kSliceDims) {
      const int64_t v = p == pos ? (int64_t)vc[d0 + dl] : (int64_t)sm.vwin[p * kSliceDims + dl];
      acc0 += (int64_t)sm.probtab[sm.sc[p]] * v;
      acc1 += (int64_t)sm.probtab[kExpLut + sm.sc[a.score_cap + p]] * v;
    }
    sm.vacc[(pl * kSliceDims + dl) * 2] = acc0;
    sm.vacc[(pl * kSliceDims + dl) * 2 + 1] = acc1;
  }
  __syncthreads();
  {  // this CTA's 32 attention outputs (q heads 2h, 2h + 1; dims d0..d0+15): warp w
     // sums outputs 2w, 2w + 1 over the 32 position lanes (16 lanes each, 2 partials a lane)
    static_assert(kPThreads / kSliceDims == 32 && kPWarps * 2 == 2 * kSliceDims, "reduction layout");
    const int o = 2 * warp + (lane >> 4), dl = o % kSliceDims, hh = o / kSliceDims, pl = 2 * (lane & 15);
    int64_t acc = sm.vacc[(pl * kSliceDims + dl) * 2 + hh] + sm.vacc[((pl + 1) * kSliceDims + dl) * 2 + hh];
#pragma unroll
    for (int m = 8; m > 0; m >>= 1) acc += shfl_xor_i64(acc, m);
    if ((lane & 15) == 0) q0[hh * kSliceDims + dl] = sat24(acc >> 16);
  }
  __syncthreads();
  // o_proj partial sums of those 32 inputs for every output row
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int64_t v = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      int32_t dot = 0;  // 16 terms: |dot| < 2^30
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        dot += nibble(os.w[r][hh].x, k) * q0[hh * kSliceDims + k];
        dot += nibble(os.w[r][hh].y, k) * q0[hh * kSliceDims + 8 + k];
      }
      v += (int64_t)dot * os.s[r][hh];
    }
    red_add_i64(acc_row(a, par, t + r * kPThreads), v);
  }
  return true;
}

// post = hidden + (o_proj >> 2) from the o_proj partial sums (every CTA, whole
// vector); gate/up CTAs then run their 64 gate and 64 up rows, SwiGLU, and add
// their down partial sums (64 columns of K = one scale group) for every row.
__device__ void stage_gateup_down(const PersistArgs& a, const LayerW& w, const PSmem& sm, int par) {
  const int gc = (int)blockIdx.x - kAttnCtas;
  const bool gu = gc >= 0 && gc < kGuCtas;
  const Gamma2 gamma(w.g_post);
  {
    const int i0 = threadIdx.x, i1 = threadIdx.x + kPThreads;
    const int64_t s0 = ldcg64(acc_row(a, par, i0)), s1 = ldcg64(acc_row(a, par, i1));
    const int32_t p0 = sat24((int64_t)sm.hid[i0] + (sat24(s0 >> 14) >> 2));
    const int32_t p1 = sat24((int64_t)sm.hid[i1] + (sat24(s1 >> 14) >> 2));
    sm.post[i0] = p0;
    sm.act[i0] = p0;
    sm.post[i1] = p1;
    sm.act[i1] = p1;
  }
  if (!gu) return;
  __syncthreads();
  hidden_norm_inplace(sm.act, gamma, sm.red);
  __syncthreads();
  stage_limbs_par(sm.act, kHidden, sm.limbs, sm.bias8);
  __syncthreads();
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t l24[24];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const uint4 t = reinterpret_cast<const uint4*>(sm.limbs + lane * kLimbStride)[i];
      l24[4 * i] = t.x;
      l24[4 * i + 1] = t.y;
      l24[4 * i + 2] = t.z;
      l24[4 * i + 3] = t.w;
    }
    const int64_t b8 = sm.bias8[lane];
    constexpr int J = kGuItems / kPWarps;  // 8 items per warp
    int64_t v[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int it = warp + j * kPWarps;
      v[j] = lane_span(gu_w(sm)[it * 32 + lane], l24, b8, gu_s(sm)[it * 32 + lane]);
    }
    const int64_t tot = warp_sum_multi<J>(v, lane);
    if ((lane & 3) == 0) sm.part[warp + ((lane >> 2) & 7) * kPWarps] = tot;
  }
  __syncthreads();
  if (threadIdx.x < kGroup) {
    const int32_t g = sat24(sm.part[threadIdx.x] >> 14), u = sat24(sm.part[kGroup + threadIdx.x] >> 14);
    const int32_t gcl = g < -32768 ? -32768 : (g > 32768 ? 32768 : g);
    int ix = (gcl + 32768 + 32) >> 6;
    ix = ix > kSigLut - 1 ? kSigLut - 1 : ix;
    const int32_t silu = sat24(((int64_t)g * sm.sig_lut[ix]) >> 16);
    sm.hv[threadIdx.x] = sat24(((int64_t)silu * u) >> 12);
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = threadIdx.x + r * kPThreads;
    const uint4 w0 = dslice_w(sm)[2 * row], w1 = dslice_w(sm)[2 * row + 1];
    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    int64_t dot = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // 16 terms per int32 chunk: |sum| < 2^30
      int32_t part = 0;
#pragma unroll
      for (int k = 0; k < 16; ++k) part += nibble(wv[2 * q + k / 8], k % 8) * sm.hv[16 * q + k];
      dot += part;
    }
    red_add_i64(acc_row(a, 2 + par, row), dot * (int64_t)dslice_s(sm)[row]);
  }
}

// final norm + this CTA's LM-head rows (streamed through the shared-memory
// ring; chunks 0..kLmRing-1 were issued before the barrier) + local argmax
// -> lm_part[cta].  Bit s of `ring_phase` is the phase parity ring slot s waits
// on next (each slot alternates strictly between one issue and one use).
__device__ void stage_lmhead(const PersistArgs& a, const PSmem& sm, unsigned& ring_phase) {
  const int G = gridDim.x, cta = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Gamma2 gamma(a.g_final);
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) sm.act[i] = sm.hid[i];  // the final hidden state
  __syncthreads();
  hidden_norm_inplace(sm.act, gamma, sm.red);
  __syncthreads();
  stage_limbs_par(sm.act, kHidden, sm.limbs, sm.bias8);
  __syncthreads();
  const int r0 = part_of(a.vocab, cta, G), r1 = part_of(a.vocab, cta + 1, G);
  const int n_chunks = (r1 - r0 + kLmChunkRows - 1) / kLmChunkRows;
  int64_t best_s = INT64_MIN;
  int32_t best_i = INT32_MAX;
  // limbs of this lane's half-group stay in registers for every row
  uint32_t l24[24];
  {
    const uint4* lp = reinterpret_cast<const uint4*>(sm.limbs + lane * kLimbStride);
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const uint4 t = lp[i];
      l24[4 * i] = t.x;
      l24[4 * i + 1] = t.y;
      l24[4 * i + 2] = t.z;
      l24[4 * i + 3] = t.w;
    }
  }
  const int64_t b8 = sm.bias8[lane];
  for (int j = 0; j < n_chunks; ++j) {
    const int slot = j % kLmRing;
    if (!mbar_wait(sm.mbar + 1 + slot, (ring_phase >> slot) & 1u, a.err)) return;
    ring_phase ^= 1u << slot;
    const int c0 = r0 + j * kLmChunkRows;
    const int rows = min(kLmChunkRows, r1 - c0);
    const uint8_t* wbuf = reinterpret_cast<const uint8_t*>(sm.kwin) + (size_t)slot * kLmChunkRows * 512;
    const uint16_t* sbuf =
        reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(sm.vwin) + (size_t)slot * kLmChunkRows * 32);
    constexpr int RW = kLmChunkRows / kPWarps;  // rows per warp per chunk
    int64_t acc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int row = warp * RW + r;
      acc[r] = 0;
      if (row < rows) {
        const uint4 wv = *reinterpret_cast<const uint4*>(wbuf + (size_t)row * 512 + lane * 16);
        acc[r] = lane_span(wv, l24, b8, sbuf[row * 16 + (lane >> 1)]);
      }
    }
    warp_reduce_rows<RW>(acc);
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int row = warp * RW + r;
      if (row < rows && acc[r] > best_s) {  // ascending rows within a warp
        best_s = acc[r];
        best_i = c0 + row;
      }
    }
    __syncthreads();  // every warp is done with this slot
    if (threadIdx.x == 0 && j + kLmRing < n_chunks) issue_lm_chunk(a, sm, r0, r1, j + kLmRing);
  }
  if (lane == 0) {
    sm.part[2 * warp] = best_s;
    sm.part[2 * warp + 1] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t bs = sm.part[0];
    int32_t bi = (int32_t)sm.part[1];
    for (int i = 1; i < kPWarps; ++i) {
      const int64_t sv = sm.part[2 * i];
      const int32_t idx = (int32_t)sm.part[2 * i + 1];
      if (sv > bs || (sv == bs && idx < bi)) {
        bs = sv;
        bi = idx;
      }
    }
    __stcg(&a.lm_part[cta].score, bs);
    __stcg(&a.lm_part[cta].idx, bi);
  }
}

// Reduce the per-CTA bests with warp 0 (lowest row wins ties); result in sm.part[0..1].
__device__ void reduce_lm_parts(const PersistArgs& a, const PSmem& sm) {
  if (threadIdx.x < 32) {
    int64_t bs = INT64_MIN;
    int32_t bi = INT32_MAX;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += 32) {
      const int64_t s = __ldcg(&a.lm_part[i].score);
      const int32_t idx = __ldcg(&a.lm_part[i].idx);
      if (s > bs || (s == bs && idx < bi)) {
        bs = s;
        bi = idx;
      }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const int64_t os = shfl_xor_i64(bs, m);
      const int32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, m);
      if (os > bs || (os == bs && oi < bi)) {
        bs = os;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) {
      sm.part[0] = bi;
      sm.part[1] = bs;
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kPThreads, 1) decode_persistent_kernel(const __grid_constant__ PersistArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  PSmem sm;
  {
    unsigned char* p = smem_raw;
    auto take = [&](size_t bytes) {
      unsigned char* r = p;
      p += (bytes + 127) & ~(size_t)127;
      return r;
    };
    sm.kwin = reinterpret_cast<int32_t*>(take((size_t)kKvWindow * kHeadDim * 4));
    sm.vwin = reinterpret_cast<int32_t*>(take((size_t)kKvWindow * kSliceDims * 4));
    sm.act = reinterpret_cast<int32_t*>(take(kInter * 4));
    sm.limbs = reinterpret_cast<uint32_t*>(take(limb_words(kInter) * 4));
    sm.bias8 = reinterpret_cast<int64_t*>(take((kInter / 32) * 8));
    sm.part = reinterpret_cast<int64_t*>(take(256 * 8));
    sm.red = reinterpret_cast<int64_t*>(take(32 * 8));
    sm.probtab = reinterpret_cast<uint64_t*>(take(2 * kExpLut * 8));
    sm.hv = reinterpret_cast<int32_t*>(take(4 * kHeadDim * 4));
    sm.vacc = reinterpret_cast<int64_t*>(take((size_t)kPThreads * 2 * 8));
    sm.mbar = reinterpret_cast<uint64_t*>(take(8 * 8));
    sm.hid = reinterpret_cast<int32_t*>(take(kHidden * 4));
    sm.post = reinterpret_cast<int32_t*>(take(kHidden * 4));
    sm.flag = reinterpret_cast<int*>(take(16));
    sm.sc = reinterpret_cast<int64_t*>(take((size_t)2 * a.score_cap * 8));
    sm.exp_lut = reinterpret_cast<int32_t*>(take(kExpLut * 4));
    sm.sig_lut = reinterpret_cast<int32_t*>(take(kSigLut * 4));
    sm.rope = reinterpret_cast<int32_t*>(take(2 * kHeadDim * 4));
  }
  // the lookup tables stay in shared memory for the whole launch
  for (int i = threadIdx.x; i < kExpLut; i += blockDim.x) sm.exp_lut[i] = a.exp_lut[i];
  for (int i = threadIdx.x; i < kSigLut; i += blockDim.x) sm.sig_lut[i] = a.sig_lut[i];
  const int G = gridDim.x, cta = blockIdx.x;
  const bool attn_cta = cta < kAttnCtas;
  const int gc = cta - kAttnCtas;
  const bool gu_cta = gc >= 0 && gc < kGuCtas;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 1 + kLmRing; ++i) mbar_init(sm.mbar + i, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  Barrier bar{a.bar, a.err, sm.flag, a.trace, a.trace_cap, 0u};
  unsigned mbar_phase = 0;
  unsigned ring_phase = 0;
  int pos = ldcg(a.st.pos);
  int next_tok = -1;
  int par = 0;  // parity of the partial-sum buffers of the current layer (host zeroes parity 0)
  const int v0 = part_of(a.vocab, cta, G), v1 = part_of(a.vocab, cta + 1, G);
  PreQkv pq;
  OSlice os;
  for (int step = 0; step < a.n_steps; ++step) {
    if (pos >= a.st.max_ctx) {  // every CTA sees the same pos: all stop here
      if (cta == 0 && threadIdx.x == 0) atomicCAS(a.err, 0, 2);
      break;
    }
    const bool lm = pos + 1 >= a.lm_from;
    const int tok = next_tok >= 0 ? next_tok : ldcg(a.st.tokens + pos);
    // this position's RoPE rows, read by the attention stage of every layer
    if (attn_cta && threadIdx.x < 2 * kHeadDim)
      sm.rope[threadIdx.x] = threadIdx.x < kHeadDim ? a.cos_tab[pos * kHeadDim + threadIdx.x]
                                                    : a.sin_tab[pos * kHeadDim + threadIdx.x - kHeadDim];
    // tied embedding: layer 0's input hidden state, every CTA the whole vector
    {
      const uint8_t* row = a.emb + (size_t)tok * (kHidden / 2);
      const uint16_t* sc = a.semb + (size_t)tok * (kHidden / kGroup);
      for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
        const uint8_t b = row[i >> 1];
        const int q = (int)((i & 1) ? (b >> 4) : (b & 0xF));
        sm.hid[i] = ((q >= 8 ? q - 16 : q) * (int32_t)sc[i / kGroup]) >> 4;
      }
    }
    preload_qkv(a.layers[0], pq);
    for (int l = 0; l < a.n_layers; ++l) {
      const LayerW w = a.layers[l];
      const bool last = l + 1 == a.n_layers;
      // layer 0's K/V window streams in during its QKV stage; later layers'
      // windows were issued after the previous attention stage (the attention
      // CTAs have no gate/up work), so the copies overlap that stage instead
      if (attn_cta && l == 0) issue_kv_copies(a, sm, l, pos);
      stage_qkv(a, w, sm, l == 0, par ^ 1, pq);
      // issued here, not at the layer start: outstanding loads hold scoreboard
      // slots that the QKV stage would wait on; the barrier hides their latency
      if (attn_cta) preload_oslice(w, os);
      // L2 prefetch of the next layer's weight slices while waiting
      if (!grid_sync(bar, [&] {
            if (!last) prefetch_layer(a.layers[l + 1], cta, G);
          }))
        return;
      if (!stage_attention(a, w, sm, l, pos, par, mbar_phase, os)) return;
      if (gu_cta) {  // not attention CTAs: these loads overlap the barrier wait
        preload_gateup(w, gc, sm);
        preload_dslice(w, gc, sm);
      }
      if (!grid_sync(bar)) return;
      if (attn_cta && !last) issue_kv_copies(a, sm, l + 1, pos);
      stage_gateup_down(a, w, sm, par);
      if (!last) preload_qkv(a.layers[l + 1], pq);
      if (last && lm) {
        // the first LM-head chunks stream in while the layer barrier resolves
        fence_proxy_async();
        __syncthreads();
        if (threadIdx.x == 0)
          for (int j = 0; j < kLmRing; ++j) issue_lm_chunk(a, sm, v0, v1, j);
      }
      if (!grid_sync(bar)) return;
      par ^= 1;
    }
    // the final hidden state (every CTA; CTA 0 also keeps it in the slot state)
    build_hidden(a, sm, par ^ 1);
    __syncthreads();
    if (cta == 0)
      for (int i = threadIdx.x; i < kHidden; i += blockDim.x) a.st.hidden[i] = sm.hid[i];
    next_tok = -1;
    if (lm) {
      stage_lmhead(a, sm, ring_phase);
      if (!grid_sync(bar)) return;
      reduce_lm_parts(a, sm);
      if (cta == 0 && threadIdx.x == 0) {
        a.st.tokens[pos + 1] = (int32_t)sm.part[0];
        a.st.scores[pos + 1] = sm.part[1];
      }
      next_tok = (int)sm.part[0];
      __syncthreads();
      // lm_part is rewritten only after the next step's 3 x layers barriers
    }
    ++pos;
  }
  if (cta == 0 && threadIdx.x == 0) *a.st.pos = pos;
}

size_t persistent_smem_bytes(int score_cap) {
  auto r = [](size_t b) { return (b + 127) & ~(size_t)127; };
  return r((size_t)kKvWindow * kHeadDim * 4) + r((size_t)kKvWindow * kSliceDims * 4) + r(kInter * 4) +
         r(limb_words(kInter) * 4) + r((kInter / 32) * 8) + r(256 * 8) + r(32 * 8) + r(2 * kExpLut * 8) +
         r(4 * kHeadDim * 4) + r((size_t)kPThreads * 2 * 8) + r(64) + 2 * r(kHidden * 4) + r(16) +
         r((size_t)2 * score_cap * 8) +
         r(kExpLut * 4) + r(kSigLut * 4) + r(2 * kHeadDim * 4) + 128;
}

}  // namespace q4

// Host launcher, called by the runtime in q4_decode.cu.
int q4gpu_launch_persistent(const q4::PersistArgs& args, int grid, size_t smem, cudaStream_t stream) {
  void* params[] = {const_cast<q4::PersistArgs*>(&args)};
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)q4::decode_persistent_kernel, dim3(grid),
                                                    dim3(q4::kPThreads), params, smem, stream);
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "persistent launch: %s", cudaGetErrorString(e));
  return Q4GPU_OK;
}

int q4gpu_persistent_relayout(const q4::LayerW* layers_dev, int n_layers, cudaStream_t stream) {
  q4::oslice_layout_kernel<<<dim3(q4::kAttnCtas, n_layers), 256, 0, stream>>>(layers_dev);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "o_proj slice layout: %s", cudaGetErrorString(e));
  return Q4GPU_OK;
}

int q4gpu_persistent_setup(int score_cap, size_t* smem, int* grid) {
  // attention stages at most kKvWindow cached positions in shared memory
  if (score_cap > q4::kKvWindow + 1)
    return q4gpu_fail(Q4GPU_ERR_SHAPE, "persistent kernel supports max_context <= %d", q4::kKvWindow + 1);
  *smem = q4::persistent_smem_bytes(score_cap);
  cudaError_t e = cudaFuncSetAttribute(q4::decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)*smem);
  if (e != cudaSuccess) return q4gpu_fail(Q4GPU_ERR_CUDA, "persistent smem %zu: %s", *smem, cudaGetErrorString(e));
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, q4::decode_persistent_kernel, q4::kPThreads, *smem);
  if (e != cudaSuccess || per_sm < 1)
    return q4gpu_fail(Q4GPU_ERR_CUDA, "persistent kernel does not fit one CTA per SM");
  // one CTA per SM; the register preloads cover one pass when the grid has >= 128 CTAs
  *grid = sms;
  if (*grid < 128) return q4gpu_fail(Q4GPU_ERR_SHAPE, "persistent kernel needs >= 128 SMs (%d)", sms);
  return Q4GPU_OK;
}
