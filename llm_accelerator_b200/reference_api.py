"""The reference's per-module Python entry points, executed on the B200.

Each function keeps the name, argument meaning, return shape and error
behaviour of the reference helper it replaces (paths relative to
``Qwen3-0.6B-Base/python_each_module``), takes and returns numpy integer
arrays, and runs the arithmetic in libq4gpu's CUDA kernels.  Inputs are
copied to the current CUDA device; there is no CPU fallback: without a GPU
or without the built library every call raises.

Weight arguments: the 26/28/30/35 helpers take *unpacked* int4 values as
int8 ``[rows, cols]``; the 21 helper takes the *packed* uint8 layout.  Both
are accepted and unpacked weights are packed once on the host
(``13_export_q4_gemv_vectors.py:67-80`` layout) before upload.
"""
from __future__ import annotations

import ctypes as C
from typing import Any, Optional

import numpy as np
import torch

from . import _native

GROUP = 64
SCORE_SCALE_Q0_31 = 189812531  # round(128 ** -0.5 * 2**31), 56_...:455-460


def _dev() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("llm_accelerator_b200 needs a CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _t(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=_dev(), dtype=dtype)


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _lib():
    return _native.load()


def _i32(a, name: str, width: int = 24) -> np.ndarray:
    v = np.asarray(a, dtype=np.int64)
    lim = 1 << (width - 1)
    if v.size and (v.min() < -lim or v.max() >= lim):
        raise ValueError(f"{name} exceeds signed {width}-bit range")
    return v.astype(np.int32)


def pack_int4(q) -> np.ndarray:
    """Even column -> low nibble (13_export_q4_gemv_vectors.py:67-80)."""
    q = np.asarray(q)
    if q.ndim != 2 or q.shape[1] % 2:
        raise ValueError(f"Expected a 2D int4 matrix with even width, got shape {q.shape}")
    if np.any(q < -8) or np.any(q > 7):
        raise ValueError("int4 values must be in [-8, 7]")
    nib = q.astype(np.int16) & 0xF
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def _gemv(act, packed: np.ndarray, scale, rows: int) -> tuple[np.ndarray, np.ndarray, int]:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    k = packed.shape[1] * 2
    a = _i32(act, "activation").reshape(-1)
    if a.size != k:
        raise ValueError(f"activation length {a.size} does not match weight width {k}")
    sc = np.ascontiguousarray(np.asarray(scale).reshape(packed.shape[0], k // GROUP)[:rows], dtype=np.uint16)
    if k not in (1024, 2048, 3072, 4096):
        raise ValueError(f"unsupported input size {k}")
    at, wt, st = _t(a, torch.int32), _t(packed[:rows], torch.uint8), _t(sc.view(np.int16), torch.int16)
    q26 = torch.empty(rows, dtype=torch.int64, device=at.device)
    q12 = torch.empty(rows, dtype=torch.int32, device=at.device)
    sat = torch.zeros(1, dtype=torch.int32, device=at.device)
    _native.check(_lib().q4gpu_gemv_q26(_p(at), k, _p(wt), _p(st), rows, _p(q26), _p(q12), _p(sat), _stream()),
                  "q4gpu_gemv_q26")
    return q26.cpu().numpy(), q12.cpu().numpy().astype(np.int64), int(sat.item())


# ---------------------------------------------------------------------------
# GEMV family
# ---------------------------------------------------------------------------
def compute_q4_gemv_q26(activation_q12_12, weight_q4, scale_q2_14) -> np.ndarray:
    """28_export_mlp_gate_up_vectors.py:124-133 (also 26_...:147-156, 30_...:124-133)."""
    w = np.asarray(weight_q4)
    return _gemv(activation_q12_12, pack_int4(w), scale_q2_14, w.shape[0])[0]


def compute_q4_logits_q26(activation_q12_12, weight_q4, scale_q2_14) -> np.ndarray:
    """35_export_lm_head_full_vocab_vectors.py:120-130."""
    return compute_q4_gemv_q26(activation_q12_12, weight_q4, scale_q2_14)


def q26_to_q12_12(row_sum_q26) -> tuple[np.ndarray, int]:
    """28_...:136-138: arithmetic >> 14 then saturate to signed 24 bit."""
    rs = np.ascontiguousarray(np.asarray(row_sum_q26, dtype=np.int64).reshape(-1))
    t = _t(rs, torch.int64)
    out = torch.empty(rs.size, dtype=torch.int32, device=t.device)
    sat = torch.zeros(1, dtype=torch.int32, device=t.device)
    _native.check(_lib().q4gpu_q26_to_q12_12(_p(t), rs.size, _p(out), _p(sat), _stream()), "q4gpu_q26_to_q12_12")
    return out.cpu().numpy().astype(np.int64), int(sat.item())


def compute_matrix_outputs(*, activation_q12_12, packed_weight, scale_q2_14, actual_q4_float: Optional[np.ndarray],
                           matrix_name: str, row_count: int) -> dict[str, Any]:
    """21_export_qmap_qkv_projection_image.py:163-219."""
    if row_count < 1:
        raise ValueError(f"{matrix_name} row_count must be positive")
    if row_count > packed_weight.shape[0]:
        raise ValueError(f"{matrix_name} row_count {row_count} exceeds available rows {packed_weight.shape[0]}")
    packed_rows = np.ascontiguousarray(packed_weight[:row_count])
    scale_rows = np.ascontiguousarray(scale_q2_14[:row_count])
    row_sum, q12, _ = _gemv(activation_q12_12, packed_rows, scale_rows, row_count)
    q12 = q12.astype(np.int32)
    recomputed = (row_sum.astype(np.float64) / float(1 << 26)).astype(np.float32)
    q12_float = (q12.astype(np.float64) / float(1 << 12)).astype(np.float32)
    if actual_q4_float is None:
        max_recompute_diff = max_q12_diff = None
    else:
        src = actual_q4_float[:row_count].astype(np.float32)
        max_recompute_diff = float(np.max(np.abs(recomputed - src)))
        if max_recompute_diff != 0.0:
            raise RuntimeError(f"{matrix_name} Q26 recompute mismatch against artifact: {max_recompute_diff}")
        max_q12_diff = float(np.max(np.abs(q12_float - src)))
    return {"packed_rows": packed_rows, "scale_rows": scale_rows, "row_sum_q26": row_sum, "q12_12": q12,
            "max_recompute_diff": max_recompute_diff, "max_q12_12_diff": max_q12_diff,
            "first_row_sum_q26": int(row_sum[0]), "first_q12_12_word": int(q12[0]),
            "first_q12_12_float": float(q12_float[0])}


# ---------------------------------------------------------------------------
# norms, RoPE
# ---------------------------------------------------------------------------
def _rmsnorm(x: np.ndarray, gamma, mode: int) -> tuple[np.ndarray, np.ndarray]:
    rows, n = x.shape
    xt, gt = _t(_i32(x, "input"), torch.int32), _t(_i32(gamma, "gamma", 16).reshape(-1), torch.int32)
    if gt.numel() != n:
        raise ValueError(f"gamma length {gt.numel()} does not match input length {n}")
    out = torch.empty(rows, n, dtype=torch.int32, device=xt.device)
    stats = torch.zeros(rows, 6, dtype=torch.int64, device=xt.device)
    _native.check(_lib().q4gpu_rmsnorm(_p(xt), _p(gt), rows, n, mode, _p(out), _p(stats), _stream()),
                  "q4gpu_rmsnorm")
    return out.cpu().numpy().astype(np.int64), stats.cpu().numpy()


def fixed_rmsnorm_reference(input_q14_10, gamma_q8_7) -> dict[str, Any]:
    """17_export_rmsnorm_fixed_vectors.py:107-147 (same arithmetic as
    27_...:110-149 and 32_...:101-140; 32 reports a saturation count)."""
    x = np.asarray(input_q14_10, dtype=np.int64).reshape(1, -1)
    out, st = _rmsnorm(x, gamma_q8_7, 0)
    ss, mean, rad, rms, inv, sat = (int(v) for v in st[0])
    rem = 0 if rms == 0 else (1 << 26) - inv * rms
    return {"sum_squares": ss, "mean_square": mean, "sqrt_radicand": rad, "rms_q14_10": rms,
            "inv_rms_uq8_16": inv, "div_remainder": rem, "output_q12_12": out[0], "saturation": sat > 0,
            "output_saturation_count": sat}


def fixed_rmsnorm_vector(input_q12_12, gamma_uq8_8) -> dict[str, Any]:
    """22_export_qk_norm_rope_fixed_vectors.py:153-188."""
    out, st = _rmsnorm(np.asarray(input_q12_12, dtype=np.int64).reshape(1, -1), gamma_uq8_8, 1)
    ss, mean, rad, rms, inv, sat = (int(v) for v in st[0])
    return {"sum_squares": ss, "mean_square": mean, "sqrt_radicand": rad, "rms_q12_12": rms,
            "inv_rms_uq8_16": inv, "output_q12_12": out[0], "saturation": sat > 0}


def fixed_rmsnorm_heads(input_heads_q12_12, gamma_uq8_8) -> tuple[np.ndarray, list, bool]:
    """22_...:191-205: one norm per head row."""
    x = np.asarray(input_heads_q12_12, dtype=np.int64)
    out, st = _rmsnorm(x, gamma_uq8_8, 1)
    debug = [{"sum_squares": int(r[0]), "mean_square": int(r[1]), "sqrt_radicand": int(r[2]),
              "rms_q12_12": int(r[3]), "inv_rms_uq8_16": int(r[4]), "output_q12_12": out[i],
              "saturation": bool(r[5] > 0)} for i, r in enumerate(st)]
    return out, debug, bool(np.any(st[:, 5] > 0))


def fixed_rope_reference(x_q12_12, cos_q1_15, sin_q1_15) -> tuple[np.ndarray, bool]:
    """22_...:208-235."""
    x = np.asarray(x_q12_12, dtype=np.int64)
    heads = x.shape[0]
    if x.shape[1] != 128:
        raise ValueError("RoPE expects [heads, 128]")
    xt = _t(_i32(x, "x"), torch.int32)
    ct, stt = _t(_i32(cos_q1_15, "cos", 17), torch.int32), _t(_i32(sin_q1_15, "sin", 17), torch.int32)
    out = torch.empty_like(xt)
    sat = torch.zeros(1, dtype=torch.int32, device=xt.device)
    _native.check(_lib().q4gpu_rope(_p(xt), heads, _p(ct), _p(stt), _p(out), _p(sat), _stream()), "q4gpu_rope")
    return out.cpu().numpy().astype(np.int64), bool(sat.item() > 0)


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def fixed_softmax_probs(scores_q24_24, exp_lut) -> tuple[np.ndarray, np.ndarray]:
    """46_export_chained_attention_score_value_vectors.py:109-125."""
    s = np.ascontiguousarray(np.asarray(scores_q24_24, dtype=np.int64))
    rows, ctx = s.shape
    st, lt = _t(s, torch.int64), _t(np.asarray(exp_lut, dtype=np.int32), torch.int32)
    probs = torch.empty(rows, ctx, dtype=torch.int32, device=st.device)
    idx = torch.empty_like(probs)
    _native.check(_lib().q4gpu_softmax_probs(_p(st), rows, ctx, _p(lt), _p(probs), _p(idx), _stream()),
                  "q4gpu_softmax_probs")
    return probs.cpu().numpy().astype(np.int64), idx.cpu().numpy().astype(np.int64)


def fixed_value_accum(probs_q0_16, v_cache_q12_12) -> tuple[np.ndarray, bool]:
    """46_...:128-141.  probs [q_heads, ctx]; v [ctx, kv_heads, 128]."""
    p = np.asarray(probs_q0_16, dtype=np.int64)
    v = np.asarray(v_cache_q12_12, dtype=np.int64)
    qh, ctx = p.shape
    kvh = v.shape[1]
    pt, vt = _t(p.astype(np.int32), torch.int32), _t(_i32(v, "v"), torch.int32)
    out = torch.empty(qh, 128, dtype=torch.int32, device=pt.device)
    sat = torch.zeros(1, dtype=torch.int32, device=pt.device)
    _native.check(_lib().q4gpu_value_accum(_p(pt), _p(vt), ctx, qh, kvh, _p(out), _p(sat), _stream()),
                  "q4gpu_value_accum")
    return out.cpu().numpy().astype(np.int64), bool(sat.item() > 0)


def attention_score_value(*, attention_helper: Any = None, q_current, k_cache, v_cache,
                          score_scale_q0_31: int = SCORE_SCALE_Q0_31, exp_lut) -> dict[str, Any]:
    """56_export_persistent_multitoken_layer_golden.py:359-395 (the
    ``attention_helper`` argument is accepted for signature compatibility)."""
    q = np.asarray(q_current, dtype=np.int64)
    k = np.asarray(k_cache, dtype=np.int64)
    qh, ctx, kvh = q.shape[0], k.shape[0], k.shape[1]
    qt, kt = _t(_i32(q, "q"), torch.int32), _t(_i32(k, "k"), torch.int32)
    raw = torch.empty(qh, ctx, dtype=torch.int64, device=qt.device)
    scaled = torch.empty_like(raw)
    _native.check(_lib().q4gpu_attention_scores(_p(qt), _p(kt), ctx, qh, kvh, int(score_scale_q0_31), _p(raw),
                                                _p(scaled), _stream()), "q4gpu_attention_scores")
    probs, idx = fixed_softmax_probs(scaled.cpu().numpy(), exp_lut)
    out, sat = fixed_value_accum(probs, v_cache)
    return {"raw": raw.cpu().numpy(), "scaled": scaled.cpu().numpy(), "probs": probs, "lut_indices": idx,
            "output": out, "saturated": sat}


# ---------------------------------------------------------------------------
# SwiGLU, residual, embedding, LM head
# ---------------------------------------------------------------------------
def silu_mul(gate_q12_12, up_q12_12, sigmoid_lut) -> dict[str, Any]:
    """56_...:546-556 with 29_export_mlp_silu_mul_vectors.py:86-93."""
    g, u = _i32(gate_q12_12, "gate").reshape(-1), _i32(up_q12_12, "up").reshape(-1)
    n = g.size
    gt, ut, lt = _t(g, torch.int32), _t(u, torch.int32), _t(np.asarray(sigmoid_lut, dtype=np.int32), torch.int32)
    h, s, ix = (torch.empty(n, dtype=torch.int32, device=gt.device) for _ in range(3))
    sat = torch.zeros(2, dtype=torch.int32, device=gt.device)
    _native.check(_lib().q4gpu_silu_mul(_p(gt), _p(ut), n, _p(lt), _p(h), _p(s), _p(ix), _p(sat), _stream()),
                  "q4gpu_silu_mul")
    sc = sat.cpu().numpy()
    return {"lut_index": ix.cpu().numpy().astype(np.int64), "silu": s.cpu().numpy().astype(np.int64),
            "hidden": h.cpu().numpy().astype(np.int64), "silu_saturation_count": int(sc[0]),
            "hidden_saturation_count": int(sc[1])}


def residual_add(a, b, shift: int = 2) -> tuple[np.ndarray, int]:
    """sat24(a + (b >> shift)) (56_...:531-534 and 561-564)."""
    av, bv = _i32(a, "a").reshape(-1), _i32(b, "b").reshape(-1)
    at, bt = _t(av, torch.int32), _t(bv, torch.int32)
    out = torch.empty_like(at)
    sat = torch.zeros(1, dtype=torch.int32, device=at.device)
    _native.check(_lib().q4gpu_residual_add(_p(at), _p(bt), av.size, shift, _p(out), _p(sat), _stream()),
                  "q4gpu_residual_add")
    return out.cpu().numpy().astype(np.int64), int(sat.item())


def embedding_hidden(token_ids, packed_rows, scale_rows) -> np.ndarray:
    """Tied Q4 embedding -> Q14.10 (56_...:190-226); ``packed_rows`` /
    ``scale_rows`` are the full packed tied matrix and its scales."""
    toks = np.asarray(token_ids, dtype=np.int64).reshape(-1)
    vocab = packed_rows.shape[0]
    if np.any(toks < 0) or np.any(toks >= vocab):
        raise ValueError(f"token id outside 0..{vocab - 1}")
    tt = _t(toks.astype(np.int32), torch.int32)
    wt = _t(np.asarray(packed_rows, dtype=np.uint8), torch.uint8)
    st = _t(np.asarray(scale_rows, dtype=np.uint16).view(np.int16), torch.int16)
    out = torch.empty(toks.size, 1024, dtype=torch.int32, device=tt.device)
    _native.check(_lib().q4gpu_embedding(_p(tt), toks.size, _p(wt), _p(st), _p(out), _stream()), "q4gpu_embedding")
    return out.cpu().numpy().astype(np.int64)


def lm_head_argmax(activation_q12_12, packed_rows, scale_rows, want_logits: bool = False):
    """Full-vocabulary tied LM head with the streamed strict-'>' argmax of
    run_final_tail (56_...:773-798).  Returns (token, score[, logits])."""
    a = _i32(activation_q12_12, "activation").reshape(-1)
    rows = packed_rows.shape[0]
    at = _t(a, torch.int32)
    wt = _t(np.asarray(packed_rows, dtype=np.uint8), torch.uint8)
    st = _t(np.asarray(scale_rows, dtype=np.uint16).view(np.int16), torch.int16)
    ws_bytes = _lib().q4gpu_lm_head_workspace_bytes(rows)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=at.device)
    logits = torch.empty(rows, dtype=torch.int64, device=at.device) if want_logits else None
    tok = torch.empty(1, dtype=torch.int32, device=at.device)
    score = torch.empty(1, dtype=torch.int64, device=at.device)
    _native.check(_lib().q4gpu_lm_head_argmax(_p(at), _p(wt), _p(st), rows, _p(logits), _p(ws), ws_bytes, _p(tok),
                                              _p(score), _stream()), "q4gpu_lm_head_argmax")
    r = (int(tok.item()), int(score.item()))
    return r + (logits.cpu().numpy(),) if want_logits else r


def quantize_weight_q4(weight) -> tuple[np.ndarray, np.ndarray]:
    """13_export_q4_gemv_vectors.py:101-135 on the GPU; returns (int8 q [R, C],
    uint16 scale [R, C/64])."""
    w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
    if w.ndim != 2 or w.shape[1] % GROUP:
        raise ValueError(f"Expected 2D weight matrix with width % 64 == 0, got shape {w.shape}")
    rows, cols = w.shape
    wt = _t(w, torch.float32)
    packed = torch.empty(rows, cols // 2, dtype=torch.uint8, device=wt.device)
    scale = torch.empty(rows, cols // GROUP, dtype=torch.int16, device=wt.device)
    err = torch.zeros(1, dtype=torch.int32, device=wt.device)
    _native.check(_lib().q4gpu_quantize_q4(_p(wt), rows, cols, _p(packed), _p(scale), _p(err), _stream()),
                  "q4gpu_quantize_q4")
    if int(err.item()):
        raise ValueError("Q4 scale does not fit unsigned 16-bit Q2.14 storage")
    p = packed.cpu().numpy()
    q = np.empty((rows, cols), dtype=np.int16)
    q[:, 0::2] = p & 0xF
    q[:, 1::2] = p >> 4
    q[q >= 8] -= 16
    return q.astype(np.int8), scale.cpu().numpy().view(np.uint16)
