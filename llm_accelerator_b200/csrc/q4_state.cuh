// Device-side views shared by the decode-step kernels and the persistent
// decode kernel.
#pragma once
#include <cuda.h>

#include "q4_common.cuh"

namespace q4 {

// ---------------------------------------------------------------------------
// Device-side views
// ---------------------------------------------------------------------------
// One byte plane of a KV page's keys for one (layer, head): 64 rows of 128
// bytes; the three planes of a (layer, head) follow each other.
constexpr int kKplPlane = kKvPage * kHeadDim;  // 8192
constexpr int kKplHead = 3 * kKplPlane;        // 24576

struct KvView {
  int32_t* pool;         // [n_pages][layers][2][8][64][128] int32
  const int32_t* pages;  // this slot's page table: logical page -> physical page
  int64_t page_elems;    // layers * 2 * 8 * 64 * 128
  // The keys once more as byte planes, read by the tensor-core scores of the
  // batched attention: per physical page [layers][8 heads][3 planes][64][128]
  // bytes.  Plane a holds byte a of each 24-bit key element k = b0 + 2^8 b1 +
  // 2^16 b2 (b0, b1 unsigned, b2 the signed top byte); each 128-byte row (one
  // position) is swizzled like a 128-byte-swizzled K-major UMMA tile (16-byte
  // unit u of row r stored at unit u ^ (r % 8)), so a bulk copy of a plane's
  // rows is an operand as it lands.
  // Both byte-plane copies exist only in models with two or more sequence
  // slots or more than 1024 positions, where the batched attention reads
  // them (null otherwise, and the writers skip them).
  uint8_t* kpl;
  int64_t kpl_page_bytes;  // layers * 8 * kKplHead
  // The values as byte planes the other way round, read by the tensor-core
  // value products: per physical page [layers][8 heads][3 planes][128 dims]
  // [64 positions] bytes (same sizes as kpl); each 64-byte row (one dim) is
  // swizzled like a 64-byte-swizzled K-major UMMA tile (16-byte unit u of row
  // d stored at unit u ^ ((d / 2) % 4)).
  uint8_t* vpl;
  __device__ __forceinline__ int32_t* at(int layer, int kind, int head, int pos) const {
    return pool + (int64_t)pages[pos >> 6] * page_elems +
           ((((int64_t)layer * 2 + kind) * kKvHeads + head) * kKvPage + (pos & (kKvPage - 1))) * kHeadDim;
  }
  // plane 0 of the (layer, head) block of the page holding pos (row 0 of the page)
  __device__ __forceinline__ uint8_t* kplane(int layer, int head, int pos) const {
    return kpl + (int64_t)pages[pos >> 6] * kpl_page_bytes + ((int64_t)layer * kKvHeads + head) * kKplHead;
  }
  // plane 0 of the (layer, head) block of the V planes of the page holding pos
  __device__ __forceinline__ uint8_t* vplane(int layer, int head, int pos) const {
    return vpl + (int64_t)pages[pos >> 6] * kpl_page_bytes + ((int64_t)layer * kKvHeads + head) * kKplHead;
  }
};

// Byte offset of dims d .. d + 3 (d % 4 == 0) of row r in a swizzled plane.
__device__ __forceinline__ uint32_t kpl_off(int r, int d) {
  return (uint32_t)r * 128u + ((uint32_t)((d >> 4) ^ (r & 7)) << 4) + (uint32_t)(d & 15);
}
// Byte l of each of four 32-bit values, packed.
__device__ __forceinline__ uint32_t byte_plane_word(int4 v, int l) {
  const uint32_t sel = (uint32_t)l | ((uint32_t)(l + 4) << 4);
  const uint32_t lo = __byte_perm((uint32_t)v.x, (uint32_t)v.y, sel);
  const uint32_t hi = __byte_perm((uint32_t)v.z, (uint32_t)v.w, sel);
  return __byte_perm(lo, hi, 0x5410);
}
// Key elements d .. d + 3 (d % 4 == 0) of position pos into the byte planes.
__device__ __forceinline__ void kpl_put4(const KvView& kv, int layer, int head, int pos, int d, int4 v) {
  if (!kv.kpl) return;
  uint8_t* b = kv.kplane(layer, head, pos) + kpl_off(pos & (kKvPage - 1), d);
#pragma unroll
  for (int a = 0; a < 3; ++a) *reinterpret_cast<uint32_t*>(b + a * kKplPlane) = byte_plane_word(v, a);
}
// Byte offset of (dim d, position p % 64) in a swizzled V plane.
__device__ __forceinline__ uint32_t vpl_off(int d, int p) {
  return (uint32_t)d * 64u + ((uint32_t)(((p & 63) >> 4) ^ ((d >> 1) & 3)) << 4) + (uint32_t)(p & 15);
}
// One value element (dim d of position pos) into the V byte planes.
__device__ __forceinline__ void vpl_put1(const KvView& kv, int layer, int head, int pos, int d, int32_t x) {
  if (!kv.vpl) return;
  uint8_t* b = kv.vplane(layer, head, pos) + vpl_off(d, pos);
  b[0] = (uint8_t)x;
  b[kKplPlane] = (uint8_t)(x >> 8);
  b[2 * kKplPlane] = (uint8_t)(x >> 16);
}
// Value elements d .. d + 3 of position pos.
__device__ __forceinline__ void vpl_put4(const KvView& kv, int layer, int head, int pos, int d, int4 v) {
  if (!kv.vpl) return;
  vpl_put1(kv, layer, head, pos, d, v.x);
  vpl_put1(kv, layer, head, pos, d + 1, v.y);
  vpl_put1(kv, layer, head, pos, d + 2, v.z);
  vpl_put1(kv, layer, head, pos, d + 3, v.w);
}
// One key element.
__device__ __forceinline__ void kpl_put1(const KvView& kv, int layer, int head, int pos, int d, int32_t x) {
  if (!kv.kpl) return;
  uint8_t* b = kv.kplane(layer, head, pos) + kpl_off(pos & (kKvPage - 1), d & ~3) + (d & 3);
  b[0] = (uint8_t)x;
  b[kKplPlane] = (uint8_t)(x >> 8);
  b[2 * kKplPlane] = (uint8_t)(x >> 16);
}

struct ArgBestD {
  int64_t score;
  int32_t idx;
  int32_t pad;
};

struct SlotState {
  int32_t* pos;     // [1] position of the next step
  int32_t* tokens;  // [max_ctx + 1] input token per position; argmax written at pos+1
  int64_t* scores;  // [max_ctx + 1]
  int32_t* hidden;  // [1024] Q14.10 layer input / output
  int32_t* qrope;   // [2048] Q12.12
  int32_t* attn;    // [2048] Q12.12
  int32_t* post;    // [1024] Q14.10
  int32_t* mlp;     // [3072] Q12.12
  ArgBestD* lm_partial;
  unsigned int* lm_counter;
  KvView kv;
  int max_ctx;  // positions the KV pages, tables and token ring cover
};

struct LayerW {
  const uint8_t* wqkv;  // [4096, 512]: q rows 0..2047, k 2048..3071, v 3072..4095
  const uint16_t* sqkv;
  const uint8_t* wo;  // [1024, 1024]
  const uint16_t* so;
  const uint8_t* wgate;  // [3072, 512]
  const uint16_t* sgate;
  const uint8_t* wup;
  const uint16_t* sup;
  const uint8_t* wdown;  // [1024, 1536]
  const uint16_t* sdown;
  const int32_t* g_in;
  const int32_t* g_post;
  const int32_t* g_q;
  const int32_t* g_k;
  // o_proj columns regrouped for the persistent kernel's attention CTAs:
  // slice c (KV head c / 8, head dims 16 (c % 8) ..) holds, per output row, the
  // 16 columns of each of the head pair (16 B) and their two scales (u16 x 2)
  const uint8_t* wo_sl;   // [64][1024][16]
  const uint16_t* so_sl;  // [64][1024][2]
};

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}


// Arguments of the persistent decode kernel (q4_persistent.cu).
struct PersistArgs {
  // 2-D view of the KV pool: rows of 128 int32 (one position of one
  // (page, layer, kind, head)), box 64 rows x 16 dims, for the V slices
  alignas(64) CUtensorMap vmap;
  SlotState st;
  const LayerW* layers;  // device array [n_layers]
  int n_layers;
  const uint8_t* emb;
  const uint16_t* semb;
  int vocab;
  const int32_t* g_final;
  const int32_t* cos_tab;
  const int32_t* sin_tab;
  const int32_t* exp_lut;
  const int32_t* sig_lut;
  int32_t* qkv;        // [4096] raw projections of the current layer
  int64_t* acc;        // [4][1024][4]: o_proj partial sums (layer parity 0, 1), then down (0, 1); one 32-B sector per row
  ArgBestD* lm_part;   // [gridDim.x]
  unsigned int* bar;   // [2]: grid barrier arrival counter (monotonic within a launch), spare
  int* err;            // 0 = ok
  int n_steps;
  int lm_from;         // the LM head runs at positions p with p + 1 >= lm_from
  int score_cap;       // positions the shared score buffer holds
  // optional timeline (nullptr = off): per barrier b, trace[2b] = last CTA's
  // arrival time and trace[2b+1] = CTA 0's release time (%globaltimer, ns)
  unsigned long long* trace;
  int trace_cap;       // barriers the trace holds
};

}  // namespace q4

// Launch / set-up of the persistent kernel (q4_persistent.cu).
int q4gpu_persistent_relayout(const q4::LayerW* layers_dev, int n_layers, cudaStream_t stream);
int q4gpu_launch_persistent(const q4::PersistArgs& args, int grid, size_t smem, cudaStream_t stream);
int q4gpu_persistent_setup(int score_cap, size_t* smem, int* grid);
