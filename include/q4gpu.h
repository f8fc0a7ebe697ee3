/*
 * libq4gpu — B200 (sm_100a) implementation of the Qwen3-0.6B Q4 fixed-point
 * decode path of Tyler913/LLM_Accelerator.
 *
 * Plain C ABI: plain pointers and sizes, no framework types.  Per-module
 * functions take DEVICE pointers and a cudaStream_t passed as `void*`
 * (NULL = legacy default stream); they validate arguments, enqueue work and
 * return without synchronising.  Model/runner functions take HOST buffers.
 *
 * Every function returns Q4GPU_OK (0) or a negative Q4GPU_ERR_* code, except
 * the runner-seam functions, which return the reference's QOT_* codes.
 * Reference paths below are relative to the reference project root;
 * `H/` abbreviates `Qwen3-0.6B-Base/python_each_module/`.
 */
#ifndef Q4GPU_H
#define Q4GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- library status codes -------------------------------------------- */
enum {
    Q4GPU_OK = 0,
    Q4GPU_ERR_ARG = -1001,       /* null pointer or out-of-range argument   */
    Q4GPU_ERR_SHAPE = -1002,     /* unsupported K / rows / head count       */
    Q4GPU_ERR_ALIGN = -1003,     /* pointer misaligned for 128-bit loads    */
    Q4GPU_ERR_CUDA = -1004,      /* a CUDA call failed; see q4gpu_last_error */
    Q4GPU_ERR_WORKSPACE = -1005, /* workspace smaller than required          */
    Q4GPU_ERR_QUANT = -1006      /* a Q4 scale did not fit unsigned Q2.14    */
};

/* Text of the last error raised on this thread (static storage). */
const char *q4gpu_last_error(void);
/* Library build string, e.g. "q4gpu sm_100a". */
const char *q4gpu_version(void);

/* =========================================================================
 * Per-module entry points (device pointers).  Each replaces one reference
 * helper; the Python shim llm_accelerator_b200.reference_api keeps the
 * reference names and numpy signatures on top of these.
 * ======================================================================= */

/* Seeded synthetic values (not a reference function): for i in [start, start+n),
 * out[i-start] = fl32(C_i) * fl32(std_dev * 2^-16), optionally rounded to bf16
 * (ties to even), where C_i is the sum of the twelve 16-bit fields of
 * splitmix64(key + (3i+j) * 0x9E3779B97F4A7C15), j = 0..2, minus 6*65535, and
 * key = splitmix64(seed * 0x9E3779B97F4A7C15 + tensor_id * 0xD1B54A32D192ED03
 * + 0x632BE59BD9B4E019): an Irwin-Hall(12) approximation of N(0, std_dev). */
int q4gpu_synth_f32(uint64_t seed, uint64_t tensor_id, int64_t start, int64_t n, float std_dev,
                    int bf16, float *out, void *stream);

/* Q4 quantiser; replaces quantize_weight_q4 (H/13_export_q4_gemv_vectors.py:101-135,
 * same arithmetic at H/28_...:103-121, H/35_...:99-117, H/49_...:36-52).
 * w: float32 [rows, cols] (16-byte aligned), cols % 64 == 0.
 * packed: uint8 [rows, cols/2], even column in the low nibble (H/13_...:67-80).
 * scale: uint16 [rows, cols/64] unsigned Q2.14.
 * *err_flag (device int, caller zeroes it) is set to 1 if a scale overflowed. */
int q4gpu_quantize_q4(const float *w, int64_t rows, int32_t cols, uint8_t *packed, uint16_t *scale,
                      int32_t *err_flag, void *stream);

/* Saturation counters: every `sat_count` argument is an optional DEVICE int32
 * that the call increments once per saturated output (the caller zeroes it);
 * they reproduce the reference helpers' saturation counts and flags. */

/* Q4 GEMV; replaces compute_q4_gemv_q26 + q26_to_q12_12
 * (H/28_export_mlp_gate_up_vectors.py:124-138; H/26_...:147-161; H/30_...:124-138)
 * and compute_matrix_outputs (H/21_export_qmap_qkv_projection_image.py:163-219).
 * act: int32 [k] Q12.12; packed [rows, k/2] (16-byte aligned); scale [rows, k/64].
 * out_q26: int64 [rows]; out_q12_12 (optional): sat24(q26 >> 14).
 * k in {1024, 2048, 3072, 4096}. */
int q4gpu_gemv_q26(const int32_t *act, int32_t k, const uint8_t *packed, const uint16_t *scale,
                   int32_t rows, int64_t *out_q26, int32_t *out_q12_12, int32_t *sat_count,
                   void *stream);

/* `count` independent Q4 GEMVs of one shape [rows, k] whose operands sit at
 * fixed strides: matrix i uses act + i * act_stride (elements; 0 = one shared
 * activation), packed + i * packed_stride (bytes, a multiple of 16), scale +
 * i * scale_stride (elements) and writes out_q26 / out_q12_12 + i * out_stride.
 * One launch streams all matrices.  No reference counterpart: the reference
 * calls compute_q4_gemv_q26 once per matrix; results equal `count` such calls. */
int q4gpu_gemv_q26_strided(const int32_t *act, int64_t act_stride, int32_t k, const uint8_t *packed,
                           int64_t packed_stride, const uint16_t *scale, int64_t scale_stride,
                           int32_t rows, int32_t count, int64_t *out_q26, int32_t *out_q12_12,
                           int64_t out_stride, int32_t *sat_count, void *stream);

/* Q26 -> Q12.12 words, sat24(q26 >> 14); replaces q26_to_q12_12
 * (H/28_...:136-138) and q26_to_q12_12_words (H/21_...:157-160). */
int q4gpu_q26_to_q12_12(const int64_t *in_q26, int32_t n, int32_t *out_q12_12, int32_t *sat_count,
                        void *stream);

/* Fixed-point RMSNorm over `rows` vectors of length n.
 * mode 0: hidden norm Q14.10 -> Q12.12, replaces fixed_rmsnorm_reference
 *         (H/17_export_rmsnorm_fixed_vectors.py:107-147; H/27_...:110-149; H/32_...:101-140).
 * mode 1: per-head q/k norm Q12.12 -> Q12.12, replaces fixed_rmsnorm_vector /
 *         fixed_rmsnorm_heads (H/22_export_qk_norm_rope_fixed_vectors.py:153-205).
 * gamma: int32 [n] Q8.7.  stats (optional): int64 [rows, 6] =
 * {sum_squares, mean_square, sqrt_radicand, rms, inv_rms, saturation_count}. */
int q4gpu_rmsnorm(const int32_t *x, const int32_t *gamma, int32_t rows, int32_t n, int32_t mode,
                  int32_t *out, int64_t *stats, void *stream);

/* Rotate-half RoPE on [heads, 128] Q12.12 with one position's Q1.15 cos/sin [128];
 * replaces fixed_rope_reference (H/22_...:208-235). */
int q4gpu_rope(const int32_t *x, int32_t heads, const int32_t *cos_q1_15, const int32_t *sin_q1_15,
               int32_t *out, int32_t *sat_count, void *stream);

/* Attention scores; replaces the score loop of attention_score_value
 * (H/56_export_persistent_multitoken_layer_golden.py:359-385).
 * q: [q_heads,128]; k_cache: [ctx, kv_heads, 128]; raw/scaled: int64 [q_heads, ctx]. */
int q4gpu_attention_scores(const int32_t *q, const int32_t *k_cache, int32_t ctx, int32_t q_heads,
                           int32_t kv_heads, int64_t scale_q0_31, int64_t *raw, int64_t *scaled,
                           void *stream);

/* Exact LUT softmax; replaces fixed_softmax_probs
 * (H/46_export_chained_attention_score_value_vectors.py:109-125).
 * scores int64 [rows, ctx]; exp_lut int32 [257]; probs / lut_index int32 [rows, ctx]. */
int q4gpu_softmax_probs(const int64_t *scores, int32_t rows, int32_t ctx, const int32_t *exp_lut,
                        int32_t *probs, int32_t *lut_index, void *stream);

/* Value accumulation; replaces fixed_value_accum (H/46_...:128-141).
 * probs [q_heads, ctx]; v_cache [ctx, kv_heads, 128]; out [q_heads, 128]. */
int q4gpu_value_accum(const int32_t *probs, const int32_t *v_cache, int32_t ctx, int32_t q_heads,
                      int32_t kv_heads, int32_t *out, int32_t *sat_count, void *stream);

/* SwiGLU with the sigmoid LUT; replaces H/56_...:546-556 with
 * gate_to_lut_index (H/29_export_mlp_silu_mul_vectors.py:86-93).
 * silu and lut_index outputs are optional; sat_counts (optional) is int32[2]:
 * {silu saturations, hidden saturations}. */
int q4gpu_silu_mul(const int32_t *gate, const int32_t *up, int32_t n, const int32_t *sigmoid_lut,
                   int32_t *hidden, int32_t *silu, int32_t *lut_index, int32_t *sat_counts,
                   void *stream);

/* out = sat24(a + (b >> shift)); replaces the residual adds
 * (H/56_...:531-534, shift 2; H/56_...:561-564, shift 2). */
int q4gpu_residual_add(const int32_t *a, const int32_t *b, int32_t n, int32_t shift, int32_t *out,
                       int32_t *sat_count, void *stream);

/* Tied Q4 embedding rows -> Q14.10; replaces q4_embedding_hidden
 * (H/56_...:190-226).  tokens: int32 [n_tokens] (device); out [n_tokens, 1024]. */
int q4gpu_embedding(const int32_t *tokens, int32_t n_tokens, const uint8_t *packed,
                    const uint16_t *scale, int32_t *out, void *stream);

/* Full-vocabulary tied LM head + greedy argmax; replaces compute_q4_logits_q26
 * (H/35_export_lm_head_full_vocab_vectors.py:120-130) and the streamed argmax of
 * run_final_tail (H/56_...:773-798; RTL lm_head_argmax_stage.sv:110-117):
 * strict '>' in ascending row order, lowest index wins ties.
 * act: int32 [1024] Q12.12 (already final-normed).  logits (optional): int64 [rows].
 * workspace: device scratch of q4gpu_lm_head_workspace_bytes(rows) bytes.
 * out_token (int32) / out_score (int64) are device pointers.
 * Returns Q4GPU_OK, Q4GPU_ERR_ARG / _WORKSPACE / _ALIGN (activation, packed and
 * workspace 16-byte aligned, scales 2-byte aligned) before any device work, or
 * the launch's error; q4gpu_last_error() holds the message. */
size_t q4gpu_lm_head_workspace_bytes(int32_t rows);
int q4gpu_lm_head_argmax(const int32_t *act, const uint8_t *packed, const uint16_t *scale,
                         int32_t rows, int64_t *logits, void *workspace, size_t workspace_bytes,
                         int32_t *out_token, int64_t *out_score, void *stream);

/* The LM head + argmax above for callers that cannot allocate device memory.
 * No counterpart in the reference.  It allocates nothing: its scratch (the
 * per-CTA partial results and a completion counter, 7120 bytes) is a static
 * device array inside libq4gpu, present on every GPU that loads the library
 * until the process exits.  It serves callers whose device memory belongs to
 * someone else — a serving framework's pre-reserved pool, or a host ported
 * from the reference's bare-metal runtime that only owns the buffers it
 * passes in — and latency-critical loops that must not call cudaMalloc, which
 * synchronises the device.  The caller still passes inputs and outputs (all
 * device pointers, as above).
 * - rows must be 1..Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS; anything else returns
 *   Q4GPU_ERR_ARG before any device work.
 * - The scratch exists once per CUDA context.  The first call in a context
 *   (a device's primary context, or the caller's own driver-API context made
 *   current) looks up its address there (cudaGetSymbolAddress) and caches it
 *   under the context's unique id; make that first call before any stream
 *   capture.
 * - Errors are reported as by q4gpu_lm_head_argmax (same codes, message in
 *   q4gpu_last_error), so the two entry points can replace each other.
 * - Every call on a device shares the one scratch array and it keeps the last
 *   call's contents (the completion counter is cleared on each call): calls
 *   that overlap on the GPU race with each other and must be serialised by
 *   the caller, e.g. by issuing them on one stream. */
#define Q4GPU_LM_HEAD_NOALLOC_MAX_ROWS 16777216
int q4gpu_lm_head_argmax_noalloc(const int32_t *act, const uint8_t *packed, const uint16_t *scale,
                                 int32_t rows, int64_t *logits, int32_t *out_token, int64_t *out_score,
                                 void *stream);

/* =========================================================================
 * Runner seam: types of the reference's host runtime
 * (FPGA_Project/software/qmap_one_token_runtime/qmap_one_token_runtime.h:17-82),
 * declared here with the same names and layout unless that header is
 * already included.
 * ======================================================================= */
#ifndef QMAP_ONE_TOKEN_RUNTIME_H
enum {
    QOT_OK = 0,
    QOT_ERR_BUSY = -1,
    QOT_ERR_BAD_LAYER = -2,
    QOT_ERR_BAD_TABLE = -3,
    QOT_ERR_BAD_ADDR = -4,
    QOT_ERR_TIMEOUT = -5,
    QOT_ERR_STATUS = -6,
    QOT_ERR_NULL = -7,
    QOT_ERR_BAD_TOKEN = -8,
    QOT_ERR_CAPACITY = -9,
    QOT_ERR_CONTEXT = -10
};

typedef struct qot_layer_qmap_bases {
    uint64_t qkv;
    uint64_t input_norm;
    uint64_t attn_frontend;
    uint64_t attn_score_value;
    uint64_t o_proj;
    uint64_t post_attn_norm;
    uint64_t mlp_gate_up;
    uint64_t mlp_silu_mul;
    uint64_t mlp_down;
    uint64_t mlp_residual_add;
} qot_layer_qmap_bases_t;

typedef struct qot_run_config {
    uint32_t layer_start;
    uint32_t layer_count;
    uint32_t position;
    uint32_t runtime_context_enable;
    uint32_t input_token_id;
    uint32_t embedding_enable;
    uint64_t embedding_weight_base;
    uint64_t embedding_scale_base;
    uint64_t input_hidden_base;
    uint64_t output_hidden_base;
    uint64_t kv_cache_base;
    uint64_t final_tail_qmap_base;
    uint32_t final_hidden_override_valid;
    uint64_t final_hidden_override_base;
    const qot_layer_qmap_bases_t *layer_qmap_bases;
    uint32_t layer_qmap_base_count;
} qot_run_config_t;

typedef struct qot_result {
    uint32_t status;
    uint32_t token_id;
    int64_t score_q26;
    uint32_t layers_started;
    uint32_t layers_completed;
    uint32_t layer_done_mask;
    uint32_t layer_error_mask;
    uint64_t last_output_base;
    uint64_t tail_hidden_base;
    uint32_t tail_tiles_started;
    uint32_t tail_tiles_completed;
    uint32_t mem_read_reqs;
    uint32_t mem_read_words;
    uint32_t mem_write_reqs;
    uint32_t mem_write_words;
} qot_result_t;
#endif /* QMAP_ONE_TOKEN_RUNTIME_H */

/* =========================================================================
 * Model context (device-resident weights, paged KV cache, decode graphs)
 * ======================================================================= */
typedef struct q4gpu_model q4gpu_model;

typedef struct q4gpu_model_config {
    int32_t n_layers;     /* 1..28 */
    int32_t vocab;        /* tied embedding / LM-head rows (151936 for Qwen3-0.6B) */
    int32_t max_context;  /* positions per sequence (the reference caps at 256) */
    int32_t max_seqs;     /* sequence slots (independent KV caches) */
    int32_t device;       /* CUDA device ordinal */
    int32_t reserved[3];
} q4gpu_model_config;

/* Create a context: allocates weights, the paged KV pool, activations and
 * workspace on `device`.  Weights start zeroed; fill them with
 * q4gpu_model_init_synthetic or q4gpu_model_set_tensor.  With max_seqs >= 2
 * or max_context > 1024 the pool also holds K and V as byte planes for the batched attention's
 * tensor-core products: 0.75x the int32 cache's bytes more (28 layers, per 64
 * positions of a sequence slot: 14 MiB int32 + 10.5 MiB). */
int q4gpu_model_create(const q4gpu_model_config *cfg, q4gpu_model **out);
void q4gpu_model_destroy(q4gpu_model *m);

/* Fill every weight from the seeded generator (N(0, std) approximation,
 * rounded to bf16) and quantise it on the device with the reference's Q4
 * quantiser.  Gammas are 1.0 (Q8.7 = 128) unless gamma_std > 0. */
int q4gpu_model_init_synthetic(q4gpu_model *m, uint64_t seed, float std_dev, float gamma_std);

/* Tensor ids for q4gpu_model_set_tensor / q4gpu_model_get_tensor. */
enum {
    Q4GPU_T_Q = 0, Q4GPU_T_K, Q4GPU_T_V, Q4GPU_T_O, Q4GPU_T_GATE, Q4GPU_T_UP, Q4GPU_T_DOWN,
    Q4GPU_T_INPUT_GAMMA, Q4GPU_T_POST_GAMMA, Q4GPU_T_Q_GAMMA, Q4GPU_T_K_GAMMA,
    Q4GPU_T_EMBED = 100, Q4GPU_T_FINAL_GAMMA = 101, Q4GPU_T_ROPE_COS = 102, Q4GPU_T_ROPE_SIN = 103,
    Q4GPU_T_EXP_LUT = 104, Q4GPU_T_SIGMOID_LUT = 105
};

/* Copy one tensor between host memory and the context.  For weight tensors
 * `data` is the reference's packed Q4 layout ([rows, cols/2] bytes) and
 * `scale` its uint16 [rows, cols/64] scales; for gammas/tables `data` is
 * int32 and `scale` is NULL.  `layer` is ignored for model-wide tensors.
 * RoPE tables are int32 [max_context, 128] Q1.15. */
/* The configuration the context was created with. */
int q4gpu_model_get_config(q4gpu_model *m, q4gpu_model_config *cfg);

int q4gpu_model_set_tensor(q4gpu_model *m, int32_t layer, int32_t which, const void *data,
                           size_t data_bytes, const uint16_t *scale, size_t scale_bytes);
int q4gpu_model_get_tensor(q4gpu_model *m, int32_t layer, int32_t which, void *data,
                           size_t data_bytes, uint16_t *scale, size_t scale_bytes);

/* =======================================================================
 * QMAP v1 blob consumption (Source/QMAP_FORMAT.md).  The reference's
 * PL-DDR image (61 segments, init/q4_runtime_assets.json) is copied into one
 * host arena whose byte 0 sits at physical address arena_base
 * (0x4_0000_0000); the walker reads the per-layer runtime packets and binds
 * the tensors their descriptors point at.
 * ======================================================================= */

/* 256-byte QMAP header (QMAP_FORMAT.md:142-157), as stored (little-endian). */
typedef struct q4gpu_qmap_header {
    uint32_t magic, version, header_bytes, descriptor_bytes, descriptor_count, descriptor_capacity;
    uint64_t descriptor_table_addr, payload_base_addr, image_base_addr, image_bytes;
    uint32_t flags, checksum32;
} q4gpu_qmap_header;

/* 128-byte tensor descriptor (QMAP_FORMAT.md:193-214), as stored. */
typedef struct q4gpu_qmap_descriptor {
    uint32_t tensor_id, role, dtype, rank, flags, element_bits, group_size, scale_tensor_id;
    uint64_t base_addr, nbytes;
    uint32_t dims[4];
    uint64_t strides_bytes[4];
    uint32_t aux[4];
    uint32_t checksum32;
    uint32_t reserved[3];
} q4gpu_qmap_descriptor;

/* Where the packets are: per layer the ten bases of qot_layer_qmap_bases_t
 * (qmap_one_token_runtime.h:31-42: qkv, input_norm, attn_frontend,
 * attn_score_value, o_proj, post_attn_norm, mlp_gate_up, mlp_silu_mul,
 * mlp_down, mlp_residual_add) and the final-tail packet
 * (QOT_MODEL_FINAL_TAIL_QMAP_BASE).  The RoPE and embedding bases are
 * optional cross-checks (0 = take them from the descriptors). */
typedef struct q4gpu_qmap_layout {
    uint64_t arena_base;
    uint64_t final_tail_qmap_base;
    uint64_t rope_cos_base, rope_sin_base;
    uint64_t embed_weight_base, embed_scale_base;
    int32_t n_layers;
    int32_t reserved;
    const uint64_t *layer_bases; /* [n_layers][10] */
} q4gpu_qmap_layout;

/* One bound model tensor (Q4GPU_T_* `which`; layer -1 = model-wide) as arena
 * offsets.  Q4 weights: packed rows (rows x cols / 2 bytes) and their u16
 * scales.  Vectors: rows values of elem_stride bytes each. */
enum { Q4GPU_QMAP_PACKED_Q4 = 0, Q4GPU_QMAP_S16 = 1, Q4GPU_QMAP_U16 = 2, Q4GPU_QMAP_U32 = 3 };
typedef struct q4gpu_qmap_tensor {
    int32_t layer, which;
    uint64_t data_offset, data_bytes;
    uint64_t scale_offset, scale_bytes;
    int32_t rows, cols;
    int32_t elem_stride, elem_kind;
} q4gpu_qmap_tensor;

/* Decode and validate the packet at physical packet_addr (magic, version 1,
 * 256/128-byte header/descriptors, count <= capacity, image_base_addr =
 * packet_addr, table inside the arena).  Returns the descriptor count (up to
 * desc_cap copied) or a negative Q4GPU_ERR_*.  Host only. */
int q4gpu_qmap_read_packet(const uint8_t *arena, uint64_t arena_base, uint64_t arena_bytes, uint64_t packet_addr,
                           q4gpu_qmap_header *header, q4gpu_qmap_descriptor *desc, int32_t desc_cap);
/* Bind every model tensor of the image (11 per layer, then the RoPE planes,
 * exp / sigmoid LUTs, tied embedding and final gamma).  Weights are found by
 * role and matrix id (aux0), vectors by role, dtype and length; the LUTs must
 * agree across layers and the score scale must be 189812531.  With cap 0 only
 * *n_out is set.  Host only. */
int q4gpu_qmap_bind(const uint8_t *arena, uint64_t arena_bytes, const q4gpu_qmap_layout *layout,
                    q4gpu_qmap_tensor *out, int32_t cap, int32_t *n_out);
/* A bound vector as int32 values (16-bit values extended from their slots). */
int q4gpu_qmap_vector(const uint8_t *arena, const q4gpu_qmap_tensor *t, int32_t *out, int64_t count);
/* Bind and upload the whole image into the context (q4gpu_model_set_tensor). */
int q4gpu_model_load_qmap(q4gpu_model *m, const uint8_t *arena, uint64_t arena_bytes,
                          const q4gpu_qmap_layout *layout);

/* Runner with the exact signature of qot_session_runner_fn
 * (FPGA_Project/software/qmap_prompt_demo/qot_session.h:51-58; default runner
 * qot_run_token, qmap_one_token_runtime.h:369-392): one full-model token
 * invocation (tied embedding, layers [layer_start, layer_start+layer_count),
 * final norm, LM head, argmax) for sequence slot `base` at `position`.
 * runner_context is the q4gpu_model*.  Validation happens before any launch
 * (same QOT_ERR_* codes); max_polls bounds the completion poll (0 = wait),
 * QOT_ERR_TIMEOUT leaves the slot busy until the work drains. */
int q4gpu_run_token(void *runner_context, uintptr_t base, const qot_run_config_t *config,
                    uint32_t input_token_id, uint32_t position, uint32_t max_polls,
                    qot_result_t *result);

/* Greedy decode with the semantics of qot_decode_token_ids
 * (qmap_one_token_runtime.h:399-500): serial prefill, the first generated id
 * is the argmax after the last prompt token, later ids are fed back at the
 * next position.  All steps run on the device without host round trips. */
int q4gpu_decode_token_ids(q4gpu_model *m, uintptr_t base, const qot_run_config_t *config,
                           const uint32_t *prompt_token_ids, uint32_t prompt_token_count,
                           uint32_t max_new_tokens, uint32_t *generated_token_ids,
                           uint32_t generated_token_capacity, uint32_t max_polls_per_token,
                           uint32_t *generated_token_count, qot_result_t *last_result);

/* Batched greedy decode of independent sequences (slots 0..n_seq-1), each
 * with its own prompt (prompts concatenated; prompt_lens[n_seq]), every prompt
 * starting at position 0.  Up to 64 sequences advance together per step
 * (groups of 64 run one after another), sharing each weight read; results are
 * identical to decoding each sequence alone with q4gpu_decode_token_ids.
 * generated: uint32 [n_seq, max_new_tokens]; scores (optional) int64 same shape.
 * Returns QOT_* codes: QOT_ERR_CAPACITY (n_seq, an empty prompt, no tokens),
 * QOT_ERR_CONTEXT (prompt_len + max_new_tokens - 1 > max_context),
 * QOT_ERR_BAD_TOKEN, QOT_ERR_BUSY, QOT_ERR_STATUS. */
int q4gpu_decode_batch(q4gpu_model *m, int32_t n_seq, const uint32_t *prompts,
                       const uint32_t *prompt_lens, uint32_t max_new_tokens, uint32_t *generated,
                       int64_t *scores);

/* Batched decode, device-resident loop (no reference counterpart: the
 * reference decodes one sequence at a time).  Slots [first_slot, first_slot +
 * n_seq), 1 <= n_seq <= 64.  Each step feeds every sequence the token stored
 * at its position, runs all layers and the LM head for all of them at once,
 * stores the argmax at position + 1 (when position + 1 >= its lm_from) and
 * advances the position.  Asynchronous on the model stream. */
int q4gpu_batch_steps(q4gpu_model *m, int32_t first_slot, int32_t n_seq, int32_t n_steps);

/* Batched exact prefill (no reference counterpart: the reference runs a
 * prompt one position at a time).  Stores each prompt in its slot's token
 * array (prompts concatenated, prompt_lens[n_seq], 1 <= len <= max_context),
 * runs positions 0 .. len - 2 of all n_seq sequences (1 <= n_seq <= 64, slots
 * [first_slot, first_slot + n_seq)) through every layer as columns of batched
 * passes (64 columns per tcgen05 GEMM sub-batch, 1024 columns per block,
 * query tiles of up to 64 positions of one sequence per attention CTA), and leaves each slot at position len - 1 with lm_from = len: the K/V
 * cache equals the one serial decode steps leave, bit for bit, and
 * q4gpu_batch_steps continues from the last prompt token.  Asynchronous on
 * the model stream. */
int q4gpu_batch_prefill(q4gpu_model *m, int32_t first_slot, int32_t n_seq, const uint32_t *prompts,
                        const uint32_t *prompt_lens);
/* How prompts run: 1 = batched exact prefill (default): q4gpu_decode_batch uses
 * q4gpu_batch_prefill, and q4gpu_decode_token_ids (full model, from position 0,
 * persistent mode) prefills positions 0 .. len - 2 the same way before the
 * persistent kernel continues from the last prompt token; 0 = serial, one
 * step per prompt position (the reference's order).  Results are identical. */
int q4gpu_model_set_prefill(q4gpu_model *m, int32_t mode);

/* Vocabulary-sharded LM head (no reference counterpart; the reference scans the
 * whole vocabulary on one device).  A step becomes: q4gpu_batch_forward_hidden
 * on each rank's own sequences -> exchange of the final vectors -> each rank's
 * q4gpu_lm_head_shard over its rows for all vectors -> exchange of the
 * (score, row) winners, reduced with highest score / lowest row ->
 * q4gpu_batch_commit on each rank's sequences.  All asynchronous on the model
 * stream; pointers are device memory.
 *
 * forward_hidden: embedding, all layers and the final RMSNorm of one position
 * for slots [first_slot, first_slot + n_seq); final_act receives the normed
 * Q12.12 vectors (int32 [n_seq, 1024]).  Positions do not advance. */
int q4gpu_batch_forward_hidden(q4gpu_model *m, int32_t first_slot, int32_t n_seq, int32_t *final_act);

/* LM head over vocabulary rows [row_begin, row_end) for n_act (1..64) vectors
 * acts (int32 [n_act, 1024], 16-byte aligned): best_score / best_row (int64
 * [n_act]) get each vector's highest Q26 logit in the shard and its global row
 * (lowest row on ties). */
int q4gpu_lm_head_shard(q4gpu_model *m, const int32_t *acts, int32_t n_act, int32_t row_begin,
                        int32_t row_end, int64_t *best_score, int64_t *best_row);

/* The shard winners' reduction and the commit in one launch: winners is the
 * device int64 array an all_gather of every rank's [2][stride] (scores, rows)
 * buffer produces, [n_shards][2][stride]; sequence i of this rank reads column
 * col0 + i of every shard.  Highest score wins, the lowest row on ties (the
 * reference's rule, exact whatever the shard order); the winner is stored like
 * q4gpu_batch_commit stores tokens.  No reference counterpart. */
int q4gpu_batch_commit_shards(q4gpu_model *m, int32_t first_slot, int32_t n_seq, const int64_t *winners,
                              int32_t n_shards, int32_t stride, int32_t col0);

/* Store tokens[i] (with scores[i]; int64 [n_seq]) at position + 1 of slot
 * first_slot + i (from its lm_from on) and advance the positions. */
int q4gpu_batch_commit(q4gpu_model *m, int32_t first_slot, int32_t n_seq, const int64_t *tokens,
                       const int64_t *scores);

/* Every slot of the range to `position`; lm_from (>= 0) sets the position
 * from which argmax tokens are stored, -1 keeps it.  Stream-ordered. */
int q4gpu_batch_set_position(q4gpu_model *m, int32_t first_slot, int32_t n_seq, int32_t position,
                             int32_t lm_from);

/* Kernel kinds of a batched step (q4gpu_batch_time_kernels). */
#define Q4GPU_BK_EMBED 0
#define Q4GPU_BK_NORM 1
#define Q4GPU_BK_QKV_GEMM 2
#define Q4GPU_BK_ATTENTION 3
#define Q4GPU_BK_O_GEMM 4
#define Q4GPU_BK_GATE_UP_GEMM 5
#define Q4GPU_BK_DOWN_GEMM 6
#define Q4GPU_BK_LM_HEAD_GEMM 7
#define Q4GPU_BK_ARGMAX 8
#define Q4GPU_BK_COUNT 9

/* Runs `reps` batched steps (advancing the positions) with an event after
 * every kernel, so the kernels run back to back without overlap; returns the
 * mean device ms per launch and the launches per step of each kind
 * (arrays of Q4GPU_BK_COUNT). */
int q4gpu_batch_time_kernels(q4gpu_model *m, int32_t first_slot, int32_t n_seq, int32_t reps,
                             double *ms_per_launch, int32_t *launches_per_step);

/* Runs one batched step (advancing the positions) with timelines on
 * (%globaltimer ns; either array may be NULL):
 * attn_stamps[((layer * n_seq + m) * 8 + kv_head) * 8 + k] from the
 * one-CTA-per-head attention kernel, k = 0 start, 1 q/k ready, 2 scores done,
 * 3 probabilities ready, 4 values done, 5 end (zeros where the split-KV kernels
 * ran); n_attn = layers * n_seq * 64.
 * gemm_stamps[((4 * layer + g) * 1200 + cta) * 8 + k] for GEMM g = qkv, o_proj,
 * gate/up, down (the LM head at 4 * layers), cta = split * tiles + tile, k = 0
 * entry, 1 set-up done, 2 dependency released, 3 first accumulator ready,
 * 4 last scale group folded, 5 partial sums exchanged, 6 epilogue done;
 * n_gemm = (4 * layers + 1) * 1200 * 8. */
int q4gpu_batch_trace(q4gpu_model *m, int32_t first_slot, int32_t n_seq, uint64_t *attn_stamps,
                      int64_t n_attn, uint64_t *gemm_stamps, int64_t n_gemm);

/* One batched step with host buffers: sequence i of the range takes
 * token_ids[i] at positions[i] and returns the argmax (and its Q26 score,
 * optional) of the next position.  Blocks until the results are on the host. */
int q4gpu_batch_run_step(q4gpu_model *m, int32_t first_slot, int32_t n_seq,
                         const uint32_t *token_ids, const uint32_t *positions, uint32_t *out_tokens,
                         int64_t *out_scores);

/* Read back the Q14.10 hidden state after the last layer of slot `base`
 * (int32 [1024]) and the retained K or V entries of one layer in the
 * reference's [position][kv_head][128] order (int32 [positions, 8, 128]). */
int q4gpu_model_read_hidden(q4gpu_model *m, uintptr_t base, int32_t *hidden);
int q4gpu_model_read_kv(q4gpu_model *m, uintptr_t base, int32_t layer, int32_t kind,
                        int32_t positions, int32_t *out);

/* Write the Q14.10 layer input of slot `base` (used with embedding_enable = 0)
 * and write retained K or V entries in the reference order (e.g. to pre-fill
 * a context); same shapes as the readers above. */
int q4gpu_model_write_hidden(q4gpu_model *m, uintptr_t base, const int32_t *hidden);
int q4gpu_model_write_kv(q4gpu_model *m, uintptr_t base, int32_t layer, int32_t kind,
                         int32_t positions, const int32_t *data);

/* Host-side table builders (no device needed).  exp LUT: 257 x round(e^(-i/16) 2^20)
 * (H/46_...:92-97); sigmoid LUT: 1025 x UQ0.16 over [-8, 8] (H/29_...:77-83);
 * RoPE: Q1.15 cos/sin [positions, 128] from float32 HF default frequencies with
 * theta 1e6 (H/common.py:155-170 then H/56_...:942-956).  The Python host
 * builds the RoPE table with torch exactly as the reference does and installs
 * it with q4gpu_model_set_tensor.  This C builder (libm float32 cos/sin) is for
 * C-only callers and differs from the reference's table by 1 LSB in about
 * 0.02% of entries, where the two float32 cos/sin round differently; a C caller
 * that needs exact parity loads the table the Python host writes. */
void q4gpu_build_tables(int32_t *exp_lut, int32_t *sigmoid_lut);
void q4gpu_build_rope_table(int32_t positions, int32_t *cos_q1_15, int32_t *sin_q1_15);

/* Continue a greedy decode of slot `base` on the device: enqueue n_steps
 * replays of the full-model step graph (embedding of tokens[pos], all layers,
 * LM head writing tokens[pos+1] and advancing pos).  Returns without waiting;
 * q4gpu_model_sync waits.  The caller keeps pos + n_steps < max_context. */
int q4gpu_decode_steps(q4gpu_model *m, uintptr_t base, int32_t n_steps);
/* Execution mode of q4gpu_decode_steps / q4gpu_decode_token_ids / decode_batch:
 * 0 = one CUDA graph of per-stage kernels per step (PDL-chained);
 * 1 = the persistent cooperative kernel, many steps per launch (default when
 *     its shared memory fits; q4gpu_run_token uses it for full-model calls
 *     with the embedding, one step per call, and mode 0 for layer ranges).
 * A persistent launch whose grid barrier wait runs out reports through
 * q4gpu_model_sync (Q4GPU_ERR_CUDA) or QOT_ERR_TIMEOUT from the decode API. */
int q4gpu_model_set_mode(q4gpu_model *m, int32_t mode);
int32_t q4gpu_model_get_mode(q4gpu_model *m);

/* Diagnostics: run n_steps persistent decode steps of slot `base` (the LM head
 * where p + 1 >= lm_from) and return, for each of the first n_barriers grid
 * barriers, {last CTA's arrival, release} in %globaltimer ns (uint64 [n_barriers, 2]).
 * Per step there are 3 barriers per layer (after QKV, after attention + o_proj
 * partial sums, after gate/up + down partial sums), then one after the LM head. */
int q4gpu_model_trace_persistent(q4gpu_model *m, uintptr_t base, int32_t n_steps, int32_t lm_from,
                                 uint64_t *stamps, int32_t n_barriers);

/* Set slot's next position, stream-ordered after the slot's queued work. */
int q4gpu_model_set_position(q4gpu_model *m, uintptr_t base, int32_t position);
int q4gpu_model_sync(q4gpu_model *m);

/* Read tokens[start, start+n) and their argmax scores (scores[p] is the score
 * of the argmax that produced tokens[p]) and the slot's next position. */
int q4gpu_model_read_tokens(q4gpu_model *m, uintptr_t base, int32_t start, int32_t n, int32_t *tokens,
                            int64_t *scores, int32_t *position);

/* Kernel kinds of one decode step, for q4gpu_model_time_kernels. */
enum {
    Q4GPU_K_EMBED = 0, Q4GPU_K_QKV, Q4GPU_K_ATTN, Q4GPU_K_OPROJ, Q4GPU_K_GATEUP, Q4GPU_K_DOWN,
    Q4GPU_K_LMHEAD, Q4GPU_K_ADVANCE, Q4GPU_K_COUNT
};

/* Run `reps` decode steps of slot `base` (continuing its greedy decode) as
 * plain launches with a CUDA event between consecutive kernels, and return the
 * mean device time of one launch of each kernel kind (ms_per_launch[8]) and
 * the launches of each kind in one step (launches_per_step[8]). */
int q4gpu_model_time_kernels(q4gpu_model *m, uintptr_t base, int32_t reps, double *ms_per_launch,
                             int32_t *launches_per_step);

/* Mean device time of one decoder layer on the per-stage path at `position`
 * for slot `base`: each layer of [layer_start, layer_start + layer_count) runs
 * as its own CUDA graph (its five kernels PDL-chained, no embedding, no LM
 * head) and is timed with events, the layers in turn for `reps` cycles after
 * one warm-up cycle (so a layer's weights and K/V are not still in L2 from its
 * previous replay when the range is large); the position is reset before every
 * replay.  No reference counterpart (measurement). */
int q4gpu_model_time_layers(q4gpu_model *m, uintptr_t base, int32_t layer_start, int32_t layer_count,
                            int32_t position, int32_t reps, double *ms);

/* Stream the context launches on (a cudaStream_t), for timing. */
void *q4gpu_model_stream(q4gpu_model *m);

#ifdef __cplusplus
}
#endif

#endif /* Q4GPU_H */
