// Batched decode (q4_batch.cu): device layout and launch interface.
#pragma once
#include <vector>

#include "q4_state.cuh"

namespace q4 {

constexpr int kBatchSeqMax = 64;  // sequences one batched step advances
constexpr int kBatchPad = 8;      // zero B rows after the 3 SP limb rows (the MMA's N rounds 3 SP up to 16)
constexpr int kScoreScale = 189812531;  // round(128^-0.5 * 2^31)

// TMA maps of one layer's Q4 matrices as the model stores them (packed
// nibbles [rows, K / 2], 64-byte x 64-row boxes), with their Q2.14 scales.
struct BatchLayerW {
  alignas(64) CUtensorMap mqkv;  // [4096, 512]: q, k, v rows
  CUtensorMap mo;                // [1024, 1024]
  CUtensorMap mgate;             // [3072, 512]
  CUtensorMap mup;               // [3072, 512]
  CUtensorMap mdown;             // [1024, 1536]
  const uint8_t* wqkv;           // the packed matrices the maps address
  const uint8_t* wo;
  const uint8_t* wgate;
  const uint8_t* wup;
  const uint8_t* wdown;
  const uint16_t* sqkv;          // [4096, 16]
  const uint16_t* so;            // [1024, 32]
  const uint16_t* sgate;         // [3072, 16]
  const uint16_t* sup;           // [3072, 16]
  const uint16_t* sdown;         // [1024, 48]
  const int32_t* g_in;
  const int32_t* g_post;
  const int32_t* g_q;
  const int32_t* g_k;
};

struct BatchPlan {
  // TMA maps of the limb matrices bt1 / bt2 / bt3 ([3 SP + 8] rows), one per
  // GEMM: boxes of the GEMM's sequence chunk (q4gpu_batch_gemm_chunk rows)
  alignas(64) CUtensorMap mb_qkv;  // bt1
  CUtensorMap mb_o;                // bt2
  CUtensorMap mb_gu;               // bt1
  CUtensorMap mb_down;             // bt3
  CUtensorMap mb_lm;               // bt1
  CUtensorMap mlm;  // packed Q4 embedding (the tied LM head)
  const SlotState* slots;  // device array [S]: sequence m is slot m
  int S;                   // live sequences (1..64)
  int SP;                  // padded sequence count: 8, 16, 24, 32 or 64
  int32_t* qkv_raw;        // [64, 4096]
  uint8_t* bt1;            // [3 SP + 8, 1024] limbs of the normed hidden / post vectors
  uint8_t* bt2;            // [3 SP + 8, 2048] limbs of the attention output
  uint8_t* bt3;            // [3 SP + 8, 3072] limbs of the SwiGLU output
  const int32_t* lm_from;  // [S] the argmax is stored at positions p with p + 1 >= lm_from
  const uint8_t* emb;      // packed Q4 embedding [vocab, 512]
  const uint16_t* semb;    // [vocab, 16]
  const BatchLayerW* layers;  // host array [n_layers]
  int n_layers;
  int max_ctx;
  int vocab;
  const int32_t* cos_tab;
  const int32_t* sin_tab;
  const int32_t* exp_lut;
  const int32_t* sig_lut;
  const int32_t* g_final;
  ArgBestD* lm_partial;  // [ceil(vocab / 128), 64]
  int* err;              // device flag: a pipeline wait ran out
  // slots [first, first + S) are consecutive in the model's state arrays
  const int32_t* pos0;   // position of sequence m at pos0[4 m]
  int32_t* hidden0;      // [S, 1024]
  int32_t* post0;        // [S, 1024]
  // split-KV attention scratch (re-armed by the kernels after each use)
  int64_t* att_S;        // [64, 16, max_ctx] scaled scores
  uint32_t* att_P;       // [64, 16, max_ctx] probabilities
  int64_t* att_M;        // [64, 16] maxima (INT64_MIN when armed)
  int64_t* att_O;        // [64, 16, 128] value sums (0 when armed)
  unsigned* att_cnt_s;   // [64, 8]
  unsigned* att_cnt_v;   // [64, 8]
  unsigned long long* trace;  // optional attention timeline, [layers, S, 8, 8] (nullptr = off)
  unsigned long long* gemm_trace;  // optional GEMM timeline, [4 layers + 1, kGemmTraceCtas, 8]
  int32_t* final_act;    // hidden-only step when set: final-norm Q12.12 [S, 1024], no LM head / argmax
  int kv_planes;         // the model holds K/V byte planes (KvView::kpl / vpl)
};

// LM head over one vocabulary shard [row_begin, row_end) for n_act vectors.
struct LmShardPlan {
  alignas(64) CUtensorMap amap;  // packed Q4 embedding rows of the shard
  CUtensorMap bmap;              // limbs of the vectors (boxes of SP rows)
  const int32_t* acts;           // [n_act, 1024] Q12.12
  int n_act;
  int row_begin, row_end;
  const uint16_t* scales;        // scales of the shard's first row
  uint8_t* bt;                   // [3 SP + 8, 1024] limb matrix
  ArgBestD* partial;             // [ceil(rows / 128), 64]
  int64_t* best_score;           // [n_act]
  int64_t* best_row;             // [n_act] global rows
  int* err;
};

// Batched exact prefill: prompt positions as columns (sequence-major).
constexpr int kPfSub = 64;     // columns per GEMM (padded batch 64)
constexpr int kPfBlock = 1024;  // columns per attention launch (and per enqueued block)
constexpr int kPfTileQ = 64;    // query positions per attention CTA (one sequence): 128 rows with both heads
constexpr int kPfKeys = 64;    // keys per staged attention chunk (one KV page)

// Query tile of an attention launch: block columns [col0, col0 + nq), all of
// one sequence, at positions pos0 .. pos0 + nq - 1.
struct PfTile {
  int32_t col0, nq, pos0, pad;
};

struct PfAttn {
  const PfTile* tiles;
  const SlotState* col_slots;  // [block columns] the column's sequence state
  const int32_t* qkv;          // [block columns][4096]; q rows normed and roped
  uint8_t* bt2;                // [block columns / 64][192][2048] limbs of the attention output
  size_t bt2_sub;              // bytes per 64-column sub-batch of bt2
  uint16_t* lut_idx;           // [block columns][16][idx_ld] exp-LUT indices (scratch)
  int idx_ld;                  // max_ctx rounded up to 64
  int layer;
  const int32_t* exp_lut;
  int* err;
};

// Limb matrices of the prefill hold kPfBlock / 64 sub-batches of kPfSubRows =
// 192 limb rows each; a GEMM's sub-batch z reads B rows 192 z .. 192 z + 191.
constexpr int kPfSubRows = 3 * kPfSub;
struct PrefillPlan {
  alignas(64) CUtensorMap mb1;  // TMA maps of bt1 / bt2 / bt3, 64-row boxes (one limb of a sub-batch)
  CUtensorMap mb2;
  CUtensorMap mb3;
  const SlotState* col_slots;  // [n_cols] this block's columns
  const int32_t* col_pos4;     // [n_cols][4], position at [4 c]
  const PfTile* tiles;         // [n_tiles], block-relative columns
  int n_cols, n_tiles;
  int32_t* hidden;  // [kPfBlock][1024]
  int32_t* post;    // [kPfBlock][1024]
  int32_t* qkv;     // [kPfBlock][4096]
  uint8_t* bt1;     // [kPfBlock / 64][192][1024]
  uint8_t* bt2;     // [kPfBlock / 64][192][2048]
  uint8_t* bt3;     // [kPfBlock / 64][192][3072]
  uint16_t* lut_idx;  // [kPfBlock][16][max_ctx rounded up to 64]
  const uint8_t* emb;
  const uint16_t* semb;
  const BatchLayerW* layers;
  int n_layers;
  int max_ctx;
  const int32_t* cos_tab;
  const int32_t* sin_tab;
  const int32_t* exp_lut;
  const int32_t* sig_lut;
  int* err;
};

constexpr int kGemmTraceCtas = 1200;  // CTAs one GEMM launch can record (the LM head has 1187)

}  // namespace q4

int q4gpu_batch_padded(int S);
int q4gpu_batch_limb_rows(int SP);  // rows of a limb matrix: 3 SP + 8 (the last 8 zero)
// Sequences per CTA (the limb-box rows) of a batched GEMM kind (q4_batch.cu
// GemmKind: 0 q/k/v, 1 o_proj, 2 gate/up, 3 down, 4 LM head) at SP padded sequences.
int q4gpu_batch_gemm_chunk(int kind, int SP);
// 2-D TMA map of a row-major u8 matrix [rows, inner_bytes], 128 x box_rows boxes, 128-byte swizzle
// (limb matrices: box_rows = 3 x the GEMM's sequence chunk, the three limb blocks of a K tile)
int q4gpu_encode_u8_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_rows);
// 2-D TMA map of packed Q4 weights [rows, inner_bytes]: 128-byte x box_rows boxes (two 128-wide
// K tiles), 128-byte swizzle; box_rows 128 (one weight tile) or 64 (a gate or up half tile)
int q4gpu_encode_q4_map(CUtensorMap* map, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_rows);
int q4gpu_batch_setup(const q4::BatchPlan& p);
// Kernel kinds of a batched step (q4gpu.h Q4GPU_BK_*), for per-kernel timing.
enum { kBkEmbed = 0, kBkNorm, kBkQkv, kBkAttn, kBkO, kBkGu, kBkDown, kBkLm, kBkArgmax, kBkCount };
struct BatchMarks {
  std::vector<cudaEvent_t> ev;  // an event after each launch (the first before the step)
  std::vector<int> kind;        // kind of the launch the event closes (-1: start)
};
// One decode position for all S sequences (embedding .. argmax), stream-ordered.
// With marks, an event is recorded after every launch (no overlap between kernels).
int q4gpu_enqueue_batch_step(const q4::BatchPlan& p, cudaStream_t s, BatchMarks* marks = nullptr);
// in: device [S][2] (token, position); lm_from[m] = 0
int q4gpu_batch_load(const q4::SlotState* slots, int S, const int32_t* in, int32_t* lm_from, cudaStream_t s);
// out: device [S][4] int32 = (token, 0, score as int64) at position in[m][1] + 1
int q4gpu_batch_gather(const q4::SlotState* slots, int S, const int32_t* in, int32_t* out, cudaStream_t s);
// every sequence to `pos`; lm_from[m] = lm_value unless lm_value < 0
int q4gpu_batch_set_positions(const q4::SlotState* slots, int S, int pos, int32_t* lm_from, int lm_value,
                              cudaStream_t s);
int q4gpu_enqueue_lm_shard(const q4::LmShardPlan& q, cudaStream_t s);
// kernel attributes of the prefill launches (once per process)
int q4gpu_prefill_setup();
// One block of prefill columns through every layer (embedding .. down_proj):
// K/V of every column written to its sequence's cache.
int q4gpu_enqueue_prefill_block(const q4::PrefillPlan& p, cudaStream_t s);

// tokens / scores: device int64 [S]; stores them at position + 1 and advances positions
int q4gpu_enqueue_batch_commit(const q4::BatchPlan& p, const int64_t* tokens, const int64_t* scores, cudaStream_t s);
// the same from per-shard (score, row) winners: win[(2 k) * stride + col0 + m] / win[(2 k + 1) * stride + col0 + m]
int q4gpu_enqueue_batch_commit_shards(const q4::BatchPlan& p, const int64_t* win, int n_shards, int stride, int col0,
                                      cudaStream_t s);

// Attention of the per-stage batch-1 path (one slot): a cluster of
// kStageAttnRanks CTAs per KV head splits the context (stage_attn_cl_kernel).
// Usable when max_ctx fits the ranks' score buffers.
constexpr int kStageAttnRanks = 16;
bool q4gpu_stage_attention_fits(int max_ctx);
int q4gpu_stage_attention_setup(int max_ctx);
// err: set to 4 when a K/V copy wait runs out
int q4gpu_enqueue_stage_attention(const q4::SlotState& st, int* err, int layer, const int32_t* exp_lut, int max_ctx,
                                  cudaStream_t s);
