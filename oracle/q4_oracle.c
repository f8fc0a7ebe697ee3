/*
 * CPU oracle (C restatement) of the Qwen3-0.6B Q4 fixed-point decode path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
 * baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg load it; the product library never links it.
 *
 * It restates the same reference functions as oracle/q4_oracle.py (and is
 * tested against it): paths relative to Qwen3-0.6B-Base/python_each_module.
 *   quantize_weight_q4      13_export_q4_gemv_vectors.py:101-135
 *   compute_q4_gemv_q26     28_export_mlp_gate_up_vectors.py:124-138
 *   fixed_rmsnorm_reference 17_export_rmsnorm_fixed_vectors.py:107-147
 *   fixed_rmsnorm_heads     22_export_qk_norm_rope_fixed_vectors.py:153-205
 *   fixed_rope_reference    22_...:208-235
 *   attention_score_value   56_export_persistent_multitoken_layer_golden.py:359-395
 *   fixed_softmax_probs / fixed_value_accum  46_...:100-141
 *   SwiGLU, residuals       56_...:529-564, 29_...:86-93
 *   tied embedding          56_...:190-226
 *   final norm + LM head    56_...:702-798, 35_...:120-130
 * Integer arithmetic is exact (int64, __int128 for the scaled score).
 * OpenMP parallelises rows of each GEMV and the heads of attention.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define HID 1024
#define QH 16
#define KVH 8
#define HD 128
#define QROWS (QH * HD)
#define KVROWS (KVH * HD)
#define INTER 3072
#define GROUP 64
#define EXP_LUT 257
#define SIG_LUT 1025

static inline int64_t sat24(int64_t v) {
  const int64_t lo = -(1LL << 23), hi = (1LL << 23) - 1;
  return v < lo ? lo : (v > hi ? hi : v);
}

/* ---- seeded synthetic generator (same definition as the numpy oracle) ---- */
static inline uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ULL;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t tid) {
  return mix64(seed * 0x9E3779B97F4A7C15ULL + tid * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL);
}

static inline float bf16_round(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  b = (b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&x, &b, 4);
  return x;
}

void orc_synth_f32(uint64_t seed, uint64_t tid, int64_t start, int64_t n, float std_dev, int bf16, float *out) {
  const uint64_t key = stream_key(seed, tid);
  const float k = std_dev * (1.0f / 65536.0f);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t idx = (uint64_t)(start + i);
    int32_t s = 0;
    for (int j = 0; j < 3; ++j) {
      const uint64_t h = mix64(key + (3 * idx + j) * 0x9E3779B97F4A7C15ULL);
      s += (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
           (int32_t)((h >> 48) & 0xFFFF);
    }
    float v = (float)(s - 6 * 65535) * k;
    out[i] = bf16 ? bf16_round(v) : v;
  }
}

/* quantize_weight_q4 (13_...:101-135) in float32; q as int8 [rows, cols] */
int orc_quantize_q4(const float *w, int64_t rows, int cols, int8_t *q, uint16_t *scale) {
  const int groups = cols / GROUP;
  int err = 0;
#pragma omp parallel for schedule(static) reduction(| : err)
  for (int64_t t = 0; t < rows * groups; ++t) {
    const int64_t row = t / groups;
    const int g = (int)(t % groups);
    const float *src = w + row * cols + g * GROUP;
    float amax = 0.f;
    for (int i = 0; i < GROUP; ++i) amax = fmaxf(amax, fabsf(src[i]));
    const float raw = amax / 7.0f;
    float sq = rintf(raw * 16384.0f);
    if (amax > 0.f && sq == 0.f) sq = 1.f;
    if (!(sq >= 0.f && sq <= 65535.f)) {
      err |= 1;
      sq = 0.f;
    }
    scale[row * groups + g] = (uint16_t)sq;
    const float used = sq / 16384.0f;
    const float safe = used > 0.f ? used : 1.0f;
    for (int i = 0; i < GROUP; ++i) {
      float v = rintf(src[i] / safe);
      v = v < -8.f ? -8.f : (v > 7.f ? 7.f : v);
      q[row * cols + g * GROUP + i] = (int8_t)v;
    }
  }
  return err;
}

/* ---- GEMV: row_sum_q26 = sum_g (sum_64 a*w) * scale (28_...:124-133) ---- */
static inline int64_t row_dot(const int32_t *a, const int8_t *w, const uint16_t *s, int k) {
  int64_t acc = 0;
  for (int g = 0; g < k / GROUP; ++g) {
    int64_t grp = 0;
    for (int h = 0; h < GROUP; h += 16) {
      int32_t p = 0; /* 16 products of |a| < 2^23, |w| <= 8 fit in int32 */
      for (int i = 0; i < 16; ++i) p += a[g * GROUP + h + i] * (int32_t)w[g * GROUP + h + i];
      grp += p;
    }
    acc += grp * (int64_t)s[g];
  }
  return acc;
}

void orc_gemv_q26(const int32_t *a, int k, const int8_t *w, const uint16_t *s, int64_t rows, int64_t *out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) out[r] = row_dot(a, w + r * k, s + r * (k / GROUP), k);
}

static void proj(const int32_t *a, int k, const int8_t *w, const uint16_t *s, int rows, int32_t *out) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) out[r] = (int32_t)sat24(row_dot(a, w + (int64_t)r * k, s + (int64_t)r * (k / GROUP), k) >> 14);
}

/* ---- fixed-point RMSNorm (17_...:107-147 / 22_...:153-188) ---- */
static uint64_t isqrt_u64(uint64_t n) {
  uint64_t r = (uint64_t)sqrt((double)n);
  while (r > 0 && r * r > n) --r;
  while ((r + 1) * (r + 1) <= n) ++r;
  return r;
}

static void rmsnorm(const int32_t *x, const int32_t *gamma, int n, int mean_shift, int eps, int div_shift,
                    int out_shift, int32_t *out) {
  int64_t ss = 0;
  for (int i = 0; i < n; ++i) ss += (int64_t)x[i] * x[i];
  const uint64_t rms = isqrt_u64((uint64_t)(ss >> mean_shift) + (uint64_t)eps);
  int64_t inv = (1LL << 24) - 1;
  if (rms) {
    const uint64_t q = (1ULL << div_shift) / rms;
    inv = (int64_t)(q < (1ULL << 24) - 1 ? q : (1ULL << 24) - 1);
  }
  for (int i = 0; i < n; ++i) out[i] = (int32_t)sat24(((int64_t)x[i] * inv * gamma[i]) >> out_shift);
}

/* ---- model ---- */
typedef struct {
  int8_t *q_w, *k_w, *v_w, *o_w, *gate_w, *up_w, *down_w;
  uint16_t *q_s, *k_s, *v_s, *o_s, *gate_s, *up_s, *down_s;
  int32_t g_in[HID], g_post[HID], g_q[HD], g_k[HD];
} orc_layer;

typedef struct {
  int n_layers, vocab, max_ctx;
  orc_layer *layers;
  int8_t *emb_q;
  uint16_t *emb_s;
  int32_t g_final[HID];
  int32_t *cos_t, *sin_t;
  int32_t exp_lut[EXP_LUT], sig_lut[SIG_LUT];
  int32_t *k_cache, *v_cache; /* [layer][pos][8][128] */
  int32_t hidden[HID];
} orc_model;

static void *xalloc(size_t n) {
  void *p = NULL;
  if (posix_memalign(&p, 64, n ? n : 64)) return NULL;
  memset(p, 0, n);
  return p;
}

orc_model *orc_model_create(int n_layers, int vocab, int max_ctx) {
  orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
  if (!m) return NULL;
  m->n_layers = n_layers;
  m->vocab = vocab;
  m->max_ctx = max_ctx;
  m->layers = (orc_layer *)calloc((size_t)n_layers, sizeof(orc_layer));
  for (int l = 0; l < n_layers; ++l) {
    orc_layer *L = &m->layers[l];
    L->q_w = xalloc((size_t)QROWS * HID);
    L->k_w = xalloc((size_t)KVROWS * HID);
    L->v_w = xalloc((size_t)KVROWS * HID);
    L->o_w = xalloc((size_t)HID * QROWS);
    L->gate_w = xalloc((size_t)INTER * HID);
    L->up_w = xalloc((size_t)INTER * HID);
    L->down_w = xalloc((size_t)HID * INTER);
    L->q_s = xalloc((size_t)QROWS * 16 * 2);
    L->k_s = xalloc((size_t)KVROWS * 16 * 2);
    L->v_s = xalloc((size_t)KVROWS * 16 * 2);
    L->o_s = xalloc((size_t)HID * 32 * 2);
    L->gate_s = xalloc((size_t)INTER * 16 * 2);
    L->up_s = xalloc((size_t)INTER * 16 * 2);
    L->down_s = xalloc((size_t)HID * 48 * 2);
    for (int i = 0; i < HID; ++i) L->g_in[i] = L->g_post[i] = 128;
    for (int i = 0; i < HD; ++i) L->g_q[i] = L->g_k[i] = 128;
  }
  m->emb_q = xalloc((size_t)vocab * HID);
  m->emb_s = xalloc((size_t)vocab * 16 * 2);
  for (int i = 0; i < HID; ++i) m->g_final[i] = 128;
  m->cos_t = xalloc((size_t)max_ctx * HD * 4);
  m->sin_t = xalloc((size_t)max_ctx * HD * 4);
  m->k_cache = xalloc((size_t)n_layers * max_ctx * KVROWS * 4);
  m->v_cache = xalloc((size_t)n_layers * max_ctx * KVROWS * 4);
  if (!m->emb_q || !m->k_cache || !m->v_cache) return NULL;
  return m;
}

void orc_model_destroy(orc_model *m) {
  if (!m) return;
  for (int l = 0; l < m->n_layers; ++l) {
    orc_layer *L = &m->layers[l];
    free(L->q_w); free(L->k_w); free(L->v_w); free(L->o_w); free(L->gate_w); free(L->up_w); free(L->down_w);
    free(L->q_s); free(L->k_s); free(L->v_s); free(L->o_s); free(L->gate_s); free(L->up_s); free(L->down_s);
  }
  free(m->layers);
  free(m->emb_q); free(m->emb_s); free(m->cos_t); free(m->sin_t); free(m->k_cache); free(m->v_cache);
  free(m);
}

void orc_model_set_tables(orc_model *m, const int32_t *cos_t, const int32_t *sin_t, const int32_t *exp_lut,
                          const int32_t *sig_lut) {
  memcpy(m->cos_t, cos_t, (size_t)m->max_ctx * HD * 4);
  memcpy(m->sin_t, sin_t, (size_t)m->max_ctx * HD * 4);
  memcpy(m->exp_lut, exp_lut, sizeof(m->exp_lut));
  memcpy(m->sig_lut, sig_lut, sizeof(m->sig_lut));
}

static int gen_quant(uint64_t seed, uint64_t tid, int64_t rows, int cols, float std_dev, int8_t *q, uint16_t *s,
                     float *tmp) {
  orc_synth_f32(seed, tid, 0, rows * cols, std_dev, 1, tmp);
  return orc_quantize_q4(tmp, rows, cols, q, s);
}

static void gen_gamma(uint64_t seed, uint64_t tid, int n, float gstd, int32_t *dst, float *tmp) {
  orc_synth_f32(seed, tid, 0, n, gstd, 1, tmp);
  for (int i = 0; i < n; ++i) {
    const float g = 1.0f + tmp[i];
    double v = nearbyint((double)g * 128.0);
    dst[i] = (int32_t)(v > 32767 ? 32767 : (v < -32768 ? -32768 : v));
  }
}

/* Same tensor ids as the numpy oracle: embedding 0, final norm 15,
 * layer l tensor w -> 16 + 16 l + w. */
int orc_model_init_synthetic(orc_model *m, uint64_t seed, float std_dev, float gamma_std) {
  float *tmp = (float *)xalloc((size_t)m->vocab * HID * 4 > (size_t)INTER * HID * 4 ? (size_t)m->vocab * HID * 4
                                                                                    : (size_t)INTER * HID * 4);
  if (!tmp) return -1;
  int err = gen_quant(seed, 0, m->vocab, HID, std_dev, m->emb_q, m->emb_s, tmp);
  for (int l = 0; l < m->n_layers; ++l) {
    orc_layer *L = &m->layers[l];
    const uint64_t b = 16 + 16 * (uint64_t)l;
    err |= gen_quant(seed, b + 0, QROWS, HID, std_dev, L->q_w, L->q_s, tmp);
    err |= gen_quant(seed, b + 1, KVROWS, HID, std_dev, L->k_w, L->k_s, tmp);
    err |= gen_quant(seed, b + 2, KVROWS, HID, std_dev, L->v_w, L->v_s, tmp);
    err |= gen_quant(seed, b + 3, HID, QROWS, std_dev, L->o_w, L->o_s, tmp);
    err |= gen_quant(seed, b + 4, INTER, HID, std_dev, L->gate_w, L->gate_s, tmp);
    err |= gen_quant(seed, b + 5, INTER, HID, std_dev, L->up_w, L->up_s, tmp);
    err |= gen_quant(seed, b + 6, HID, INTER, std_dev, L->down_w, L->down_s, tmp);
    if (gamma_std > 0.f) {
      gen_gamma(seed, b + 7, HID, gamma_std, L->g_in, tmp);
      gen_gamma(seed, b + 8, HID, gamma_std, L->g_post, tmp);
      gen_gamma(seed, b + 9, HD, gamma_std, L->g_q, tmp);
      gen_gamma(seed, b + 10, HD, gamma_std, L->g_k, tmp);
    }
  }
  if (gamma_std > 0.f) gen_gamma(seed, 15, HID, gamma_std, m->g_final, tmp);
  free(tmp);
  return err;
}

/* (raw * scale) >> 31 with a 128-bit product, as Python's unbounded ints do */
static inline int64_t scale_score(int64_t raw, int64_t scale) {
  const __int128 p = (__int128)raw * scale;
  return (int64_t)(p >> 31);
}

static void attention(const orc_model *m, int layer, int pos, const int32_t *q, int32_t *out) {
  const int ctx = pos + 1;
  const int32_t *K = m->k_cache + (size_t)layer * m->max_ctx * KVROWS;
  const int32_t *V = m->v_cache + (size_t)layer * m->max_ctx * KVROWS;
#pragma omp parallel for schedule(static)
  for (int h = 0; h < QH; ++h) {
    const int kv = h / 2;
    int64_t *sc = (int64_t *)malloc(sizeof(int64_t) * ctx);
    int64_t mx = INT64_MIN;
    for (int p = 0; p < ctx; ++p) {
      int64_t d = 0;
      const int32_t *kr = K + ((size_t)p * KVH + kv) * HD;
      for (int i = 0; i < HD; ++i) d += (int64_t)q[h * HD + i] * kr[i];
      sc[p] = scale_score(d, 189812531LL);
      if (sc[p] > mx) mx = sc[p];
    }
    int64_t sum = 0;
    for (int p = 0; p < ctx; ++p) {
      const int64_t d = mx - sc[p];
      int64_t ix = d <= 0 ? 0 : (d + (1LL << 19)) >> 20;
      if (ix > EXP_LUT - 1) ix = EXP_LUT - 1;
      sc[p] = ix;
      sum += m->exp_lut[ix];
    }
    int64_t acc[HD];
    memset(acc, 0, sizeof(acc));
    for (int p = 0; p < ctx; ++p) {
      const int64_t prob = ((int64_t)m->exp_lut[sc[p]] << 16) / sum;
      const int32_t *vr = V + ((size_t)p * KVH + kv) * HD;
      for (int i = 0; i < HD; ++i) acc[i] += prob * vr[i];
    }
    for (int i = 0; i < HD; ++i) out[h * HD + i] = (int32_t)sat24(acc[i] >> 16);
    free(sc);
  }
}

static void head_norm_rope(const int32_t *x, const int32_t *gamma, const int32_t *cs, const int32_t *sn,
                           int32_t *out) {
  int32_t n[HD];
  rmsnorm(x, gamma, HD, 7, 17, 28, 23, n);
  for (int d = 0; d < HD; ++d) {
    const int64_t rot = d < 64 ? -(int64_t)n[d + 64] : (int64_t)n[d - 64];
    out[d] = (int32_t)sat24(((int64_t)n[d] * cs[d] + rot * sn[d]) >> 15);
  }
}

/* One layer at one position (56_...:468-564); hidden updated in place. */
void orc_layer_step(orc_model *m, int layer, int pos, int32_t *hidden) {
  const orc_layer *L = &m->layers[layer];
  int32_t norm[HID], q[QROWS], k[KVROWS], v[KVROWS], qr[QROWS], att[QROWS], o[HID], post[HID], pn[HID];
  static int32_t gate[INTER], up[INTER], h[INTER], dn[HID];
  rmsnorm(hidden, L->g_in, HID, 10, 1, 26, 21, norm);
  proj(norm, HID, L->q_w, L->q_s, QROWS, q);
  proj(norm, HID, L->k_w, L->k_s, KVROWS, k);
  proj(norm, HID, L->v_w, L->v_s, KVROWS, v);
  const int32_t *cs = m->cos_t + (size_t)pos * HD, *sn = m->sin_t + (size_t)pos * HD;
  int32_t *kc = m->k_cache + ((size_t)layer * m->max_ctx + pos) * KVROWS;
  int32_t *vc = m->v_cache + ((size_t)layer * m->max_ctx + pos) * KVROWS;
  for (int hh = 0; hh < QH; ++hh) head_norm_rope(q + hh * HD, L->g_q, cs, sn, qr + hh * HD);
  for (int hh = 0; hh < KVH; ++hh) head_norm_rope(k + hh * HD, L->g_k, cs, sn, kc + hh * HD);
  memcpy(vc, v, sizeof(v));
  attention(m, layer, pos, qr, att);
  proj(att, QROWS, L->o_w, L->o_s, HID, o);
  for (int i = 0; i < HID; ++i) post[i] = (int32_t)sat24((int64_t)hidden[i] + (o[i] >> 2));
  rmsnorm(post, L->g_post, HID, 10, 1, 26, 21, pn);
  proj(pn, HID, L->gate_w, L->gate_s, INTER, gate);
  proj(pn, HID, L->up_w, L->up_s, INTER, up);
  for (int i = 0; i < INTER; ++i) {
    const int32_t g = gate[i];
    const int32_t gc = g < -32768 ? -32768 : (g > 32768 ? 32768 : g);
    int ix = (gc + 32768 + 32) >> 6;
    if (ix > SIG_LUT - 1) ix = SIG_LUT - 1;
    const int64_t silu = sat24(((int64_t)g * m->sig_lut[ix]) >> 16);
    h[i] = (int32_t)sat24((silu * up[i]) >> 12);
  }
  proj(h, INTER, L->down_w, L->down_s, HID, dn);
  for (int i = 0; i < HID; ++i) hidden[i] = (int32_t)sat24((int64_t)post[i] + (dn[i] >> 2));
}

/* One full-model run: embedding, layers, final norm, LM head argmax. */
int orc_run_token(orc_model *m, int token, int pos, int want_logits, int32_t *out_token, int64_t *out_score) {
  if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->max_ctx) return -1;
  for (int i = 0; i < HID; ++i) m->hidden[i] = (m->emb_q[(size_t)token * HID + i] * (int32_t)m->emb_s[(size_t)token * 16 + i / 64]) >> 4;
  for (int l = 0; l < m->n_layers; ++l) orc_layer_step(m, l, pos, m->hidden);
  if (!want_logits) return 0;
  int32_t fn[HID];
  rmsnorm(m->hidden, m->g_final, HID, 10, 1, 26, 21, fn);
  int64_t best = INT64_MIN;
  int32_t best_i = -1;
#pragma omp parallel
  {
    int64_t lb = INT64_MIN;
    int32_t li = -1;
#pragma omp for schedule(static) nowait
    for (int r = 0; r < m->vocab; ++r) {
      const int64_t s = row_dot(fn, m->emb_q + (size_t)r * HID, m->emb_s + (size_t)r * 16, HID);
      if (s > lb) { lb = s; li = r; } /* ascending rows within a thread: lowest index wins ties */
    }
#pragma omp critical
    {
      if (li >= 0 && (lb > best || (lb == best && li < best_i))) { best = lb; best_i = li; }
    }
  }
  *out_token = best_i;
  *out_score = best;
  return 0;
}

/* Greedy decode like qot_decode_token_ids: prompt runs, then feedback. */
int orc_decode(orc_model *m, const int32_t *prompt, int n_prompt, int max_new, int32_t *gen, int64_t *scores) {
  int32_t tok = 0;
  int64_t sc = 0;
  int pos = 0;
  for (int i = 0; i < n_prompt; ++i, ++pos)
    if (orc_run_token(m, prompt[i], pos, i == n_prompt - 1, &tok, &sc)) return -1;
  gen[0] = tok;
  if (scores) scores[0] = sc;
  for (int i = 1; i < max_new; ++i, ++pos) {
    if (orc_run_token(m, tok, pos, 1, &tok, &sc)) return -1;
    gen[i] = tok;
    if (scores) scores[i] = sc;
  }
  return 0;
}

void orc_read_hidden(const orc_model *m, int32_t *out) { memcpy(out, m->hidden, sizeof(m->hidden)); }

/* K (kind 0) or V (kind 1) cache rows of one layer, positions [pos0, pos0 + n),
 * each [8 heads][128] Q12.12 as the decode path stores them.  Loading a
 * cache lets a check re-run single positions teacher-forced on top of a
 * cache some other implementation built (the long-prompt parity checks). */
int orc_set_kv(orc_model *m, int layer, int kind, int pos0, int n, const int32_t *rows) {
  if (layer < 0 || layer >= m->n_layers || kind < 0 || kind > 1 || pos0 < 0 || n < 0 || pos0 + n > m->max_ctx)
    return -1;
  int32_t *c = (kind ? m->v_cache : m->k_cache) + ((size_t)layer * m->max_ctx + pos0) * KVROWS;
  memcpy(c, rows, (size_t)n * KVROWS * sizeof(int32_t));
  return 0;
}

int orc_get_kv(const orc_model *m, int layer, int kind, int pos0, int n, int32_t *rows) {
  if (layer < 0 || layer >= m->n_layers || kind < 0 || kind > 1 || pos0 < 0 || n < 0 || pos0 + n > m->max_ctx)
    return -1;
  const int32_t *c = (kind ? m->v_cache : m->k_cache) + ((size_t)layer * m->max_ctx + pos0) * KVROWS;
  memcpy(rows, c, (size_t)n * KVROWS * sizeof(int32_t));
  return 0;
}

int orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}
