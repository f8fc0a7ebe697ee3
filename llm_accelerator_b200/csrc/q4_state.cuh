// Device-side views shared by the decode-step kernels and the persistent
// decode kernel.
#pragma once
#include <cuda.h>

#include "q4_common.cuh"

namespace q4 {

// ---------------------------------------------------------------------------
// Device-side views
// ---------------------------------------------------------------------------
struct KvView {
  int32_t* pool;         // [n_pages][layers][2][8][64][128] int32
  const int32_t* pages;  // this slot's page table: logical page -> physical page
  int64_t page_elems;    // layers * 2 * 8 * 64 * 128
  __device__ __forceinline__ int32_t* at(int layer, int kind, int head, int pos) const {
    return pool + (int64_t)pages[pos >> 6] * page_elems +
           ((((int64_t)layer * 2 + kind) * kKvHeads + head) * kKvPage + (pos & (kKvPage - 1))) * kHeadDim;
  }
};

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
