"""CPU oracle for the Qwen3-0.6B Q4 fixed-point decode path.

TEST INFRASTRUCTURE ONLY.  This module restates, in vectorised numpy, the
arithmetic of the reference's Python mirror of its RTL
(``Qwen3-0.6B-Base/python_each_module``).  It is the checker for the CUDA
path: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it.  The product package never imports it and has no
CPU fallback.

Every function cites the reference file:line it follows (paths relative to
``Qwen3-0.6B-Base/python_each_module`` unless stated).  The oracle is pinned
against the reference's golden vectors (``FPGA_Project/sim/vectors``) and
against outputs of the reference helpers themselves, both committed as
fixtures under ``tests/golden/``.

All arithmetic is exact integer arithmetic in int64.  The one place the
reference needs more than 64 bits (attention score x Q0.31 scale, done with
unbounded Python ints at ``56_...:374-385``) is split into a high and a low
32-bit half, which is exact (see ``scale_scores``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# ---------------------------------------------------------------------------
# Model shape and fixed-point constants
# (56_export_persistent_multitoken_layer_golden.py:25-34, config.json)
# ---------------------------------------------------------------------------
LAYERS = 28
HIDDEN = 1024
N_Q_HEADS = 16
N_KV_HEADS = 8
HEAD_DIM = 128
Q_ROWS = N_Q_HEADS * HEAD_DIM
KV_ROWS = N_KV_HEADS * HEAD_DIM
KV_REPEAT = N_Q_HEADS // N_KV_HEADS
INTER = 3072
VOCAB = 151936
REF_MAX_CONTEXT = 256  # 23_export_kv_cache_append_vectors.py:27

GROUP = 64  # 13_export_q4_gemv_vectors.py:14
Q4_MIN, Q4_MAX = -8, 7  # 13_...:16-17
SCALE_FRAC = 14  # 13_...:21 (unsigned Q2.14)

# input / post-attention / final RMSNorm (17_export_rmsnorm_fixed_vectors.py:31-46)
NORM_MEAN_SHIFT = 10
NORM_EPS_Q20 = 1
NORM_DIV_SHIFT = 10 + 16  # RMS_FRAC + INV_RMS_FRAC
NORM_OUT_SHIFT = 10 + 16 + 7 - 12  # = 21
INV_RMS_MAX = (1 << 24) - 1

# per-head q/k RMSNorm and RoPE (22_export_qk_norm_rope_fixed_vectors.py:39-58)
HEAD_MEAN_SHIFT = 7  # log2(HEAD_DIM)
HEAD_EPS_Q24 = 17
HEAD_DIV_SHIFT = 12 + 16
HEAD_OUT_SHIFT = 12 + 16 + 7 - 12  # = 23
ROPE_SHIFT = 15
GAMMA_WIDTH, GAMMA_FRAC = 16, 7
TRIG_WIDTH, TRIG_FRAC = 16, 15

# attention (46_export_chained_attention_score_value_vectors.py:24-37)
SCORE_SCALE_FRAC = 31
SCORE_FRAC = 24
EXP_FRAC = 20
EXP_LUT_STEP_FRAC = 4
EXP_LUT_SIZE = (16 << EXP_LUT_STEP_FRAC) + 1  # 257
PROB_FRAC = 16
# round(128 ** -0.5 * 2**31), computed at 56_...:455-460
SCORE_SCALE_Q0_31 = int(round((HEAD_DIM ** -0.5) * float(1 << SCORE_SCALE_FRAC)))

# SwiGLU (29_export_mlp_silu_mul_vectors.py:25-34)
SIG_FRAC = 16
SIG_WIDTH = 16
SIG_IDX_FRAC = 6
SIG_LUT_SIZE = int(16.0 * (1 << SIG_IDX_FRAC)) + 1  # 1025

# residual shifts (27_...:33-37, 31_...:34)
O_TO_RESIDUAL_SHIFT = 2
DOWN_TO_OUT_SHIFT = 2
EMBED_DEQUANT_SHIFT = 4  # 49_export_q4_embedding_vectors.py:22

I64 = np.int64


def signed_limits(width: int) -> tuple[int, int]:
    return -(1 << (width - 1)), (1 << (width - 1)) - 1


def saturate(values, width: int) -> tuple[np.ndarray, int]:
    """Clip to signed ``width`` bits; returns (clipped, count) like
    ``saturate_signed_array`` (26_export_o_proj_vectors.py:107-110)."""
    v = np.asarray(values, dtype=I64)
    lo, hi = signed_limits(width)
    count = int(np.count_nonzero((v < lo) | (v > hi)))
    return np.clip(v, lo, hi).astype(I64), count


def quantize_signed(values, width: int, frac: int) -> tuple[np.ndarray, int]:
    """float -> signed fixed point with round-half-even and clipping
    (22_export_qk_norm_rope_fixed_vectors.py:75-83; same as 17_...:86-89)."""
    lo, hi = signed_limits(width)
    scaled = np.rint(np.asarray(values).astype(np.float64) * float(1 << frac))
    count = int(np.count_nonzero((scaled < lo) | (scaled > hi)))
    return np.clip(scaled, lo, hi).astype(I64), count


# ---------------------------------------------------------------------------
# a1/a2: Q4 quantisation and nibble packing
# ---------------------------------------------------------------------------
def quantize_weight_q4(weight) -> tuple[np.ndarray, np.ndarray]:
    """Per (row, 64-group) absmax/7 scale in unsigned Q2.14, then
    q = clip(rint(w / scale), -8, 7).

    Restates 13_export_q4_gemv_vectors.py:101-135 (same formula at
    26_...:126-144, 28_...:103-121, 30_...:103-121, 35_...:99-117 and, per
    row, 49_...:36-52) for any [rows, cols] shape with cols % 64 == 0.
    All float steps are float32 exactly as numpy performs them there.
    Returns (q int8 [R, C], scale uint16 [R, C/64]).
    """
    w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
    if w.ndim != 2 or w.shape[1] % GROUP != 0:
        raise ValueError(f"expected [rows, cols] with cols % {GROUP} == 0, got {w.shape}")
    rows, cols = w.shape
    grouped = w.reshape(rows, cols // GROUP, GROUP)
    absmax = np.max(np.abs(grouped), axis=2)
    raw_scale = absmax / np.float32(Q4_MAX)
    scale_q = np.rint(raw_scale * np.float32(1 << SCALE_FRAC)).astype(I64)
    scale_q = np.where((absmax > 0.0) & (scale_q == 0), 1, scale_q)
    if np.any(scale_q < 0) or np.any(scale_q > 0xFFFF):
        raise ValueError("Q4 scale does not fit unsigned 16-bit Q2.14")
    scale_u16 = scale_q.astype(np.uint16)
    scale_used = scale_u16.astype(np.float32) / np.float32(1 << SCALE_FRAC)
    safe = np.where(scale_used > 0.0, scale_used, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(grouped / safe[:, :, None]), Q4_MIN, Q4_MAX).astype(np.int8)
    return q.reshape(rows, cols), scale_u16


def pack_int4(q) -> np.ndarray:
    """Even column -> low nibble, odd column -> high nibble, two's complement
    (13_export_q4_gemv_vectors.py:67-80)."""
    q = np.asarray(q)
    if q.ndim != 2 or q.shape[1] % 2:
        raise ValueError(f"expected [rows, even cols], got {q.shape}")
    if np.any(q < Q4_MIN) or np.any(q > Q4_MAX):
        raise ValueError("int4 values must be in [-8, 7]")
    nib = q.astype(np.int16) & 0xF
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed, cols: int) -> np.ndarray:
    """Inverse of ``pack_int4`` (13_...:83-98, 21_...:140-154)."""
    p = np.asarray(packed, dtype=np.uint8)
    if p.shape[1] * 2 != cols:
        raise ValueError(f"packed width {p.shape[1]} does not match {cols} int4 values")
    out = np.empty((p.shape[0], cols), dtype=np.int16)
    out[:, 0::2] = p & 0x0F
    out[:, 1::2] = (p >> 4) & 0x0F
    out[out >= 8] -= 16
    return out.astype(np.int8)


def pack_words32(q) -> np.ndarray:
    """Eight Q4 values per little-endian word32, lowest index in the low nibble
    (35_export_lm_head_full_vocab_vectors.py:80-89)."""
    flat = (np.asarray(q).reshape(-1).astype(np.int16) & 0xF).astype(np.uint32)
    g = flat.reshape(-1, 8)
    words = np.zeros(g.shape[0], dtype=np.uint32)
    for i in range(8):
        words |= g[:, i] << np.uint32(4 * i)
    return words


# ---------------------------------------------------------------------------
# a3: tied Q4 embedding
# ---------------------------------------------------------------------------
def embedding_hidden(q_row, scale_row) -> np.ndarray:
    """hidden_q14_10 = (q4 * scale) >> 4 (floor) for one tied row
    (56_export_persistent_multitoken_layer_golden.py:216-222)."""
    q = np.asarray(q_row, dtype=I64).reshape(-1)
    s = np.repeat(np.asarray(scale_row, dtype=I64).reshape(-1), GROUP)
    out = (q * s) >> EMBED_DEQUANT_SHIFT
    lo, hi = signed_limits(24)
    if np.any((out < lo) | (out > hi)):
        raise RuntimeError("embedding output exceeds signed 24-bit")
    return out


# ---------------------------------------------------------------------------
# a4/a6: integer RMSNorm
# ---------------------------------------------------------------------------
def _norm_core(x: np.ndarray, gamma: np.ndarray, mean_shift: int, eps: int,
               div_shift: int, out_shift: int) -> dict:
    """Shared body of 17_...:107-147 and 22_...:153-188: sum of squares,
    floor-shift to a mean, +eps, isqrt, inv = min(2^k // rms, 2^24-1),
    out = sat24((x * inv * gamma) >> shift).  Works on [..., n] batches."""
    x = np.asarray(x, dtype=I64)
    g = np.asarray(gamma, dtype=I64)
    ss = np.sum(x * x, axis=-1, dtype=I64)
    mean = ss >> mean_shift
    rad = mean + eps
    rms = np.vectorize(math.isqrt, otypes=[I64])(rad) if rad.ndim else I64(math.isqrt(int(rad)))
    rms = np.asarray(rms, dtype=I64)
    num = I64(1) << I64(div_shift)
    safe = np.where(rms == 0, 1, rms)
    inv = np.where(rms == 0, INV_RMS_MAX, np.minimum(num // safe, INV_RMS_MAX)).astype(I64)
    prod = x * inv[..., None] * g
    out, sat = saturate(prod >> out_shift, 24)
    return {"sum_squares": ss, "mean_square": mean, "sqrt_radicand": rad, "rms": rms,
            "inv_rms": inv, "output": out, "saturation_count": sat}


def rmsnorm(x_q14_10, gamma_q8_7) -> dict:
    """Hidden-size RMSNorm, Q14.10 in -> Q12.12 out.  One function serves the
    input norm (17_export_rmsnorm_fixed_vectors.py:107-147), the
    post-attention norm (27_...:110-149) and the final norm (32_...:101-140),
    which are the same arithmetic."""
    return _norm_core(x_q14_10, gamma_q8_7, NORM_MEAN_SHIFT, NORM_EPS_Q20,
                      NORM_DIV_SHIFT, NORM_OUT_SHIFT)


def rmsnorm_heads(x_q12_12, gamma) -> tuple[np.ndarray, dict, int]:
    """Per-head q/k RMSNorm over HEAD_DIM (22_...:153-205)."""
    r = _norm_core(x_q12_12, gamma, HEAD_MEAN_SHIFT, HEAD_EPS_Q24,
                   HEAD_DIV_SHIFT, HEAD_OUT_SHIFT)
    return r["output"], r, r["saturation_count"]


# ---------------------------------------------------------------------------
# a7: RoPE
# ---------------------------------------------------------------------------
def rope(x_q12_12, cos_q1_15, sin_q1_15) -> tuple[np.ndarray, int]:
    """rotate-half RoPE: (x[d]*cos[d] + (-x[d+64] | x[d-64])*sin[d]) >> 15,
    sat24 (22_...:208-235).  x is [heads, 128]; cos/sin are [128]."""
    x = np.asarray(x_q12_12, dtype=I64)
    half = HEAD_DIM // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    s = x * np.asarray(cos_q1_15, dtype=I64) + rot * np.asarray(sin_q1_15, dtype=I64)
    return saturate(s >> ROPE_SHIFT, 24)


def rope_inv_freq(theta: float = 1.0e6, dim: int = HEAD_DIM):
    """HF default RoPE inverse frequencies in float32, as the reference takes
    them from ``rotary_emb.inv_freq`` (common.py:159)."""
    import torch
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))


def rope_tables(n_positions: int, theta: float = 1.0e6) -> tuple[np.ndarray, np.ndarray]:
    """Q1.15 cos/sin tables [n, 128] built as common.py:155-170 (float32
    torch) followed by quantize_signed(., 16, 15) (56_...:942-956)."""
    import torch
    inv = rope_inv_freq(theta)
    pos = torch.arange(n_positions, dtype=torch.long).float()
    freqs = pos[:, None] * inv[None, :]  # the k=1 matmul's single float32 rounding
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos().numpy().astype(np.float32)  # attention_scaling is 1.0
    sin = emb.sin().numpy().astype(np.float32)
    c, _ = quantize_signed(cos, TRIG_WIDTH, TRIG_FRAC)
    s, _ = quantize_signed(sin, TRIG_WIDTH, TRIG_FRAC)
    return c, s


# ---------------------------------------------------------------------------
# a5/a12/a13/a14/a15: Q4 GEMV
# ---------------------------------------------------------------------------
def gemv_q26(act_q12_12, q_weight, scale_q2_14) -> np.ndarray:
    """row_sum_q26[r] = sum_g (sum_{64} act*w) * scale[r, g]
    (28_export_mlp_gate_up_vectors.py:124-133; identical at 26_...:147-156,
    30_...:124-133, 35_...:120-130, 21_...:163-219).  Any K % 64 == 0."""
    a = np.asarray(act_q12_12, dtype=I64).reshape(-1)
    w = np.asarray(q_weight)
    rows, k = w.shape
    if a.size != k:
        raise ValueError(f"activation length {a.size} != weight columns {k}")
    g = k // GROUP
    s = np.asarray(scale_q2_14, dtype=I64)
    ag = a.reshape(g, GROUP)
    out = np.empty(rows, dtype=I64)
    step = 4096  # chunk rows so the int64 temporaries stay small (LM head: 151936 rows)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        part = np.einsum("rgk,gk->rg", w[r0:r1].reshape(r1 - r0, g, GROUP).astype(I64), ag)
        out[r0:r1] = np.sum(part * s[r0:r1], axis=1, dtype=I64)
    return out


def gemv_q26_packed(act_q12_12, packed, scale_q2_14) -> np.ndarray:
    """GEMV on nibble-packed weights (21_...:163-219)."""
    p = np.asarray(packed, dtype=np.uint8)
    return gemv_q26(act_q12_12, unpack_int4(p, p.shape[1] * 2), scale_q2_14)


def q26_to_q12_12(row_sum_q26) -> tuple[np.ndarray, int]:
    """Arithmetic >> 14 then saturate to signed 24 bit (28_...:136-138)."""
    return saturate(np.asarray(row_sum_q26, dtype=I64) >> SCALE_FRAC, 24)


def lm_head_argmax(logits) -> tuple[int, int]:
    """Lowest index wins ties; strict '>' update in ascending row order
    (56_...:773-798; RTL lm_head_argmax_stage.sv:110-117)."""
    lg = np.asarray(logits, dtype=I64)
    i = int(np.argmax(lg))
    return i, int(lg[i])


# ---------------------------------------------------------------------------
# a8: KV address mapping
# ---------------------------------------------------------------------------
KV_CACHE_BASE_ADDR = 0x0000_0004_1410_0000  # 23_...:25, 56_...:35


def kv_addr(base_addr: int, layer: int, kind: int, head: int, position: int, dim: int,
            max_context: int = REF_MAX_CONTEXT) -> int:
    """Flat word32 address (23_export_kv_cache_append_vectors.py:64-84)."""
    pos_stride = HEAD_DIM * 4
    head_stride = max_context * pos_stride
    kind_stride = N_KV_HEADS * head_stride
    layer_stride = 2 * kind_stride
    return (base_addr + layer * layer_stride + kind * kind_stride + head * head_stride
            + position * pos_stride + dim * 4)


def sign_extend_to_word(value: int, width: int = 24) -> int:
    """23_...:55-61."""
    sign = 1 << (width - 1)
    v = int(value) & ((1 << width) - 1)
    return v | (((1 << (32 - width)) - 1) << width) if v & sign else v


def kv_write_trace(base_addr: int, layer: int, position: int, k_cur, v_cur,
                   max_context: int = REF_MAX_CONTEXT) -> dict:
    """All K heads/dims first, then all V (56_...:319-356)."""
    kinds, heads, dims = np.meshgrid(np.arange(2), np.arange(N_KV_HEADS), np.arange(HEAD_DIM),
                                     indexing="ij")
    kinds, heads, dims = kinds.reshape(-1), heads.reshape(-1), dims.reshape(-1)
    pos_stride = HEAD_DIM * 4
    head_stride = max_context * pos_stride
    kind_stride = N_KV_HEADS * head_stride
    addr = (base_addr + layer * 2 * kind_stride + kinds * kind_stride + heads * head_stride
            + position * pos_stride + dims * 4).astype(I64)
    data = np.concatenate([np.asarray(k_cur, dtype=I64).reshape(-1),
                           np.asarray(v_cur, dtype=I64).reshape(-1)]) & 0xFFFFFFFF
    return {"addr": addr, "data": data.astype(I64), "kind": kinds.astype(I64),
            "head": heads.astype(I64), "dim": dims.astype(I64)}


# ---------------------------------------------------------------------------
# a9-a11: attention
# ---------------------------------------------------------------------------
def scale_scores(raw, scale_q0_31: int = SCORE_SCALE_Q0_31) -> np.ndarray:
    """(raw * scale) >> 31 with unbounded-integer semantics (56_...:374-385).

    raw = hi * 2^32 + lo with lo in [0, 2^32); hi * 2^32 * s is a multiple of
    2^31, so floor((raw * s) / 2^31) = 2 * hi * s + ((lo * s) >> 31).  Both
    terms fit int64 for |raw| < 2^62 and s < 2^31.
    """
    r = np.asarray(raw, dtype=I64)
    s = I64(scale_q0_31)
    hi = r >> 32
    lo = r & I64(0xFFFFFFFF)
    return 2 * hi * s + ((lo * s) >> SCORE_SCALE_FRAC)


def attention_scores(q_rope, k_cache, scale_q0_31: int = SCORE_SCALE_Q0_31):
    """raw[h, p] = sum_d q[h, d] * k[p, h // 2, d]; scaled via scale_scores
    (56_...:359-385).  q is [16, 128], k_cache [ctx, 8, 128]."""
    q = np.asarray(q_rope, dtype=I64)
    k = np.asarray(k_cache, dtype=I64)
    kv = np.repeat(np.arange(N_KV_HEADS), KV_REPEAT)[: q.shape[0]]
    raw = np.einsum("hd,phd->hp", q, k[:, kv, :])
    return raw, scale_scores(raw, scale_q0_31)


def build_exp_lut() -> np.ndarray:
    """LUT[i] = round(e^(-i/16) * 2^20), 257 entries (46_...:92-97)."""
    return np.asarray([int(round(math.exp(-float(i) / float(1 << EXP_LUT_STEP_FRAC))
                                 * float(1 << EXP_FRAC))) for i in range(EXP_LUT_SIZE)], dtype=I64)


def score_lut_index(max_score, score):
    """min(((max - s) + 2^19) >> 20, 256); 0 when max - s <= 0
    (46_...:100-106)."""
    d = np.asarray(max_score, dtype=I64) - np.asarray(score, dtype=I64)
    shift = SCORE_FRAC - EXP_LUT_STEP_FRAC
    idx = np.minimum((d + (I64(1) << I64(shift - 1))) >> shift, EXP_LUT_SIZE - 1)
    return np.where(d <= 0, 0, idx).astype(I64)


def softmax_probs(scores_q24_24, exp_lut) -> tuple[np.ndarray, np.ndarray]:
    """Row max, LUT exp, prob = (e << 16) // sum(e) (46_...:109-125)."""
    s = np.asarray(scores_q24_24, dtype=I64)
    lut = np.asarray(exp_lut, dtype=I64)
    mx = np.max(s, axis=-1, keepdims=True)
    idx = score_lut_index(mx, s)
    e = lut[idx]
    tot = np.sum(e, axis=-1, keepdims=True, dtype=I64)
    if np.any(tot <= 0):
        raise RuntimeError("softmax exp_sum underflowed to zero")
    return (e << PROB_FRAC) // tot, idx


def value_accum(probs_q0_16, v_cache) -> tuple[np.ndarray, int]:
    """out[h, d] = sat24((sum_p prob[h, p] * v[p, h // 2, d]) >> 16)
    (46_...:128-141)."""
    p = np.asarray(probs_q0_16, dtype=I64)
    v = np.asarray(v_cache, dtype=I64)
    kv = np.repeat(np.arange(N_KV_HEADS), KV_REPEAT)[: p.shape[0]]
    acc = np.einsum("hp,phd->hd", p, v[:, kv, :])
    return saturate(acc >> PROB_FRAC, 24)


def attention(q_rope, k_cache, v_cache, exp_lut, scale_q0_31: int = SCORE_SCALE_Q0_31) -> dict:
    """Score, softmax and value stages for one position (56_...:359-395)."""
    raw, scaled = attention_scores(q_rope, k_cache, scale_q0_31)
    probs, idx = softmax_probs(scaled, exp_lut)
    out, sat = value_accum(probs, v_cache)
    return {"raw": raw, "scaled": scaled, "probs": probs, "lut_indices": idx,
            "output": out, "saturation_count": sat}


# ---------------------------------------------------------------------------
# a13: SwiGLU
# ---------------------------------------------------------------------------
def build_sigmoid_lut() -> np.ndarray:
    """1025 entries over [-8, 8] in steps of 1/64, UQ0.16 (29_...:77-83)."""
    vals = []
    for i in range(SIG_LUT_SIZE):
        x = -8.0 + float(i) / float(1 << SIG_IDX_FRAC)
        y = 1.0 / (1.0 + math.exp(-x))
        vals.append(int(np.clip(round(y * float(1 << SIG_FRAC)), 0, (1 << SIG_WIDTH) - 1)))
    return np.asarray(vals, dtype=I64)


def gate_lut_index(gate_q12_12) -> np.ndarray:
    """(clip(g, -32768, 32768) + 32768 + 32) >> 6 (29_...:86-93)."""
    g = np.clip(np.asarray(gate_q12_12, dtype=I64), -32768, 32768)
    return np.clip((g + 32768 + 32) >> 6, 0, SIG_LUT_SIZE - 1).astype(I64)


def silu_mul(gate_q12_12, up_q12_12, sigmoid_lut) -> dict:
    """silu = sat24((g * sigmoid) >> 16); h = sat24((silu * up) >> 12)
    (56_...:546-556)."""
    g = np.asarray(gate_q12_12, dtype=I64)
    u = np.asarray(up_q12_12, dtype=I64)
    idx = gate_lut_index(g)
    sig = np.asarray(sigmoid_lut, dtype=I64)[idx]
    silu, s1 = saturate((g * sig) >> SIG_FRAC, 24)
    h, s2 = saturate((silu * u) >> 12, 24)
    return {"lut_index": idx, "sigmoid": sig, "silu": silu, "hidden": h,
            "silu_saturation_count": s1, "hidden_saturation_count": s2}


# ---------------------------------------------------------------------------
# a16: one decoder layer at one position, a15: final tail
# ---------------------------------------------------------------------------
@dataclass
class LayerParams:
    """Quantised parameters of one layer (56_...:241-297).  Weights are int8
    unpacked Q4 [rows, cols]; scales uint16 [rows, cols/64]; gammas Q8.7."""
    q_w: np.ndarray
    q_s: np.ndarray
    k_w: np.ndarray
    k_s: np.ndarray
    v_w: np.ndarray
    v_s: np.ndarray
    o_w: np.ndarray
    o_s: np.ndarray
    gate_w: np.ndarray
    gate_s: np.ndarray
    up_w: np.ndarray
    up_s: np.ndarray
    down_w: np.ndarray
    down_s: np.ndarray
    input_gamma: np.ndarray
    post_gamma: np.ndarray
    q_gamma: np.ndarray
    k_gamma: np.ndarray


def _proj(act, w, s):
    out, _ = q26_to_q12_12(gemv_q26(act, w, s))
    return out


def layer_step(p: LayerParams, hidden_q14_10, position: int, k_cache: np.ndarray,
               v_cache: np.ndarray, cos_q1_15, sin_q1_15, exp_lut, sigmoid_lut,
               trace: dict | None = None) -> np.ndarray:
    """One layer at one position, following 56_...:468-564 step by step.
    ``k_cache``/``v_cache`` are [max_ctx, 8, 128] int64 and are appended at
    ``position``; attention reads positions [0, position]."""
    x = np.asarray(hidden_q14_10, dtype=I64)
    norm = rmsnorm(x, p.input_gamma)["output"]
    q = _proj(norm, p.q_w, p.q_s).reshape(N_Q_HEADS, HEAD_DIM)
    k = _proj(norm, p.k_w, p.k_s).reshape(N_KV_HEADS, HEAD_DIM)
    v = _proj(norm, p.v_w, p.v_s).reshape(N_KV_HEADS, HEAD_DIM)
    qn, _, _ = rmsnorm_heads(q, p.q_gamma)
    kn, _, _ = rmsnorm_heads(k, p.k_gamma)
    qr, _ = rope(qn, cos_q1_15[position], sin_q1_15[position])
    kr, _ = rope(kn, cos_q1_15[position], sin_q1_15[position])
    k_cache[position] = kr
    v_cache[position] = v
    att = attention(qr, k_cache[: position + 1], v_cache[: position + 1], exp_lut)
    attn_out = att["output"].reshape(-1)
    o, _ = q26_to_q12_12(gemv_q26(attn_out, p.o_w, p.o_s))
    post, _ = saturate(x + (o >> O_TO_RESIDUAL_SHIFT), 24)
    post_norm = rmsnorm(post, p.post_gamma)["output"]
    gate = _proj(post_norm, p.gate_w, p.gate_s)
    up = _proj(post_norm, p.up_w, p.up_s)
    h = silu_mul(gate, up, sigmoid_lut)["hidden"]
    d, _ = q26_to_q12_12(gemv_q26(h, p.down_w, p.down_s))
    out, _ = saturate(post + (d >> DOWN_TO_OUT_SHIFT), 24)
    if trace is not None:
        trace.update(input_norm=norm, q=q, k=k, v=v, q_norm=qn, k_norm=kn, q_rope=qr, k_rope=kr,
                     attn=att, attn_out=attn_out, o=o, post_hidden=post, post_norm=post_norm,
                     gate=gate, up=up, mlp_hidden=h, down=d, layer_out=out)
    return out


@dataclass
class Model:
    """A quantised model: per-layer params plus the tied Q4 embedding/LM head."""
    layers: list
    embed_q: np.ndarray  # int8 [vocab, 1024]
    embed_s: np.ndarray  # uint16 [vocab, 16]
    final_gamma: np.ndarray
    cos: np.ndarray = field(default=None)
    sin: np.ndarray = field(default=None)
    exp_lut: np.ndarray = field(default_factory=build_exp_lut)
    sigmoid_lut: np.ndarray = field(default_factory=build_sigmoid_lut)


class DecodeState:
    """Retained per-layer K/V caches of one sequence (56_...:456-457, 498-518)."""

    def __init__(self, n_layers: int, max_ctx: int):
        self.k = np.zeros((n_layers, max_ctx, N_KV_HEADS, HEAD_DIM), dtype=I64)
        self.v = np.zeros_like(self.k)


def run_token(m: Model, st: DecodeState, token: int, position: int,
              want_logits: bool = True) -> tuple[int, int, np.ndarray | None]:
    """One full-model run: tied embedding, every layer, final norm, full-vocab
    LM head and argmax (56_...:1008-1037 chained with 702-863)."""
    if not 0 <= token < m.embed_q.shape[0]:
        raise ValueError(f"token id {token} outside vocabulary")
    h = embedding_hidden(m.embed_q[token], m.embed_s[token])
    for li, p in enumerate(m.layers):
        h = layer_step(p, h, position, st.k[li], st.v[li], m.cos, m.sin, m.exp_lut, m.sigmoid_lut)
    if not want_logits:
        return -1, 0, h
    fn = rmsnorm(h, m.final_gamma)["output"]
    logits = gemv_q26(fn, m.embed_q, m.embed_s)
    tok, score = lm_head_argmax(logits)
    return tok, score, h


def greedy_decode(m: Model, prompt, max_new: int, max_ctx: int | None = None) -> tuple[list, list]:
    """Serial prefill then greedy feedback, as qot_decode_token_ids
    (FPGA_Project/software/qmap_one_token_runtime/qmap_one_token_runtime.h:399-500):
    the first generated id is the argmax after the last prompt token."""
    prompt = [int(t) for t in prompt]
    runs = len(prompt) + max_new - 1
    st = DecodeState(len(m.layers), max_ctx or runs)
    pos = 0
    tok = score = None
    for t in prompt:
        tok, score, _ = run_token(m, st, t, pos)
        pos += 1
    out, scores = [tok], [score]
    for _ in range(max_new - 1):
        tok, score, _ = run_token(m, st, tok, pos)
        out.append(tok)
        scores.append(score)
        pos += 1
    return out, scores


# ---------------------------------------------------------------------------
# Seeded synthetic inputs.  Not part of the reference: a counter-based
# generator that the CUDA initialiser and this oracle both implement, so the
# two sides build bit-identical float32 weights without moving them.
# value(i) = fl32(C_i) * fl32(std * 2^-16), C_i = (sum of twelve 16-bit
# fields of three splitmix64 hashes) - 6 * 65535, an Irwin-Hall(12)
# approximation of N(0, 1) * 65536; optionally rounded to bf16 (RNE).
# ---------------------------------------------------------------------------
_GOLD = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_KEYMUL = 0xD1B54A32D192ED03
_KEYADD = 0x632BE59BD9B4E019
MASK64 = (1 << 64) - 1


def _mix64_np(z: np.ndarray) -> np.ndarray:
    z = z ^ (z >> np.uint64(30))
    z = z * _M1
    z = z ^ (z >> np.uint64(27))
    z = z * _M2
    return z ^ (z >> np.uint64(31))


def _mix64_int(z: int) -> int:
    z &= MASK64
    z ^= z >> 30
    z = (z * 0xBF58476D1CE4E5B9) & MASK64
    z ^= z >> 27
    z = (z * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def stream_key(seed: int, tensor_id: int) -> int:
    return _mix64_int(seed * 0x9E3779B97F4A7C15 + tensor_id * _KEYMUL + _KEYADD)


def synth_centered(seed: int, tensor_id: int, n: int, start: int = 0) -> np.ndarray:
    """Integer C_i in [-393210, 393210] for i in [start, start + n)."""
    key = np.uint64(stream_key(seed, tensor_id))
    idx = np.arange(start, start + n, dtype=np.uint64)
    total = np.zeros(n, dtype=np.int64)
    with np.errstate(over="ignore"):
        for j in range(3):
            h = _mix64_np(key + (idx * np.uint64(3) + np.uint64(j)) * _GOLD)
            for f in range(4):
                total += ((h >> np.uint64(16 * f)) & np.uint64(0xFFFF)).astype(np.int64)
    return total - 6 * 65535


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
    return r.astype(np.uint32).view(np.float32)


def synth_f32(seed: int, tensor_id: int, shape, std: float, bf16: bool = True) -> np.ndarray:
    n = int(np.prod(shape))
    k = np.float32(std) * np.float32(2.0 ** -16)
    w = synth_centered(seed, tensor_id, n).astype(np.float32) * k
    if bf16:
        w = bf16_round(w)
    return w.reshape(shape)


# tensor ids of the synthetic model (also used by the CUDA initialiser)
TID_EMBED = 0
TID_FINAL_NORM = 15
TID_LAYER_BASE = 16
TID_PER_LAYER = 16
(T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_IN_NORM, T_POST_NORM, T_Q_NORM,
 T_K_NORM) = range(11)
LAYER_SHAPES = {T_Q: (Q_ROWS, HIDDEN), T_K: (KV_ROWS, HIDDEN), T_V: (KV_ROWS, HIDDEN),
                T_O: (HIDDEN, Q_ROWS), T_GATE: (INTER, HIDDEN), T_UP: (INTER, HIDDEN),
                T_DOWN: (HIDDEN, INTER)}


def layer_tid(layer: int, which: int) -> int:
    return TID_LAYER_BASE + layer * TID_PER_LAYER + which


def synth_layer(seed: int, layer: int, std: float = 0.02, gamma_std: float = 0.0) -> LayerParams:
    """Quantised synthetic layer.  Gammas are 1.0 (HF init) unless
    gamma_std > 0, in which case gamma = 1 + N(0, gamma_std)."""
    mats = {}
    for which, shape in LAYER_SHAPES.items():
        q, s = quantize_weight_q4(synth_f32(seed, layer_tid(layer, which), shape, std))
        mats[which] = (q, s)

    def gamma(which, n):
        g = np.ones(n, dtype=np.float32)
        if gamma_std > 0:
            g = g + synth_f32(seed, layer_tid(layer, which), (n,), gamma_std)
        return quantize_signed(g, GAMMA_WIDTH, GAMMA_FRAC)[0]

    return LayerParams(
        q_w=mats[T_Q][0], q_s=mats[T_Q][1], k_w=mats[T_K][0], k_s=mats[T_K][1],
        v_w=mats[T_V][0], v_s=mats[T_V][1], o_w=mats[T_O][0], o_s=mats[T_O][1],
        gate_w=mats[T_GATE][0], gate_s=mats[T_GATE][1], up_w=mats[T_UP][0], up_s=mats[T_UP][1],
        down_w=mats[T_DOWN][0], down_s=mats[T_DOWN][1],
        input_gamma=gamma(T_IN_NORM, HIDDEN), post_gamma=gamma(T_POST_NORM, HIDDEN),
        q_gamma=gamma(T_Q_NORM, HEAD_DIM), k_gamma=gamma(T_K_NORM, HEAD_DIM))
