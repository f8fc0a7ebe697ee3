"""Build the committed golden fixtures in this directory.

Run once in a container where the reference project tree is mounted
(read-only is enough):

    python tests/golden/make_golden.py --reference <reference project root>

It writes three kinds of fixture, and nothing at test time reads the
reference tree:

* ``kat_*.npz`` - compact copies of the reference's versioned RTL golden
  vectors (``FPGA_Project/sim/vectors``): real Qwen3 layer-0/1/2 data with
  the expected word of every stage.  Large weight matrices are cut to a row
  prefix (rows are independent in a GEMV), everything else is kept whole.
* ``ref_helpers.npz`` - outputs of the reference's own Python helpers
  (``Qwen3-0.6B-Base/python_each_module``), imported by path exactly as
  ``56_export_persistent_multitoken_layer_golden.py:37-45`` does, on seeded
  synthetic inputs including the edge cases (zero vectors, saturation,
  LUT clamps, ties, extreme activations).
* ``ref_model_seed0.npz`` - the reference's chained fixed-point layer and
  tail functions (``56_...:402-863``) run teacher-forced over a short
  token sequence on the seed-0 synthetic full-size model; its per-position
  argmax tokens and scores pin the whole-model greedy decode.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import sys
import tempfile
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
from oracle import q4_oracle as O  # noqa: E402

I64 = np.int64


def read_hex(path: Path, width: int, signed: bool) -> np.ndarray:
    vals = []
    mask = (1 << width) - 1
    sign = 1 << (width - 1)
    for line in path.read_text().split():
        v = int(line.replace("_", ""), 16) & mask
        if signed and (v & sign):
            v -= 1 << width
        vals.append(v)
    return np.asarray(vals, dtype=np.int64) if width <= 63 or signed else np.asarray(vals, dtype=np.uint64)


def words32_to_q4(words: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = words.astype(np.uint64)
    nib = np.stack([(w >> np.uint64(4 * i)) & np.uint64(0xF) for i in range(8)], axis=1).reshape(-1)
    q = nib.astype(np.int16)
    q[q >= 8] -= 16
    return q.astype(np.int8).reshape(rows, cols)


def words32_to_u16(words: np.ndarray, count: int) -> np.ndarray:
    w = words.astype(np.uint64)
    out = np.stack([w & np.uint64(0xFFFF), (w >> np.uint64(16)) & np.uint64(0xFFFF)], axis=1)
    return out.reshape(-1)[:count].astype(np.uint16)


# --------------------------------------------------------------------------
# 1. RTL golden vectors
# --------------------------------------------------------------------------
def kat_gemv_words(vec: Path, prefix: str, sub: str, rows: int, cols: int, acc_width: int,
                   keep_rows: int, act_name: str = "activation") -> dict:
    """GEMV stage KAT stored as packed words32 weights + scales."""
    w = read_hex(vec / f"{prefix}_{sub}weight_words32.hex", 32, False)
    s = read_hex(vec / f"{prefix}_{sub}scale_words32.hex", 32, False)
    q = words32_to_q4(w, rows, cols)[:keep_rows]
    sc = words32_to_u16(s, rows * cols // 64).reshape(rows, cols // 64)[:keep_rows]
    return {
        "activation": read_hex(vec / f"{prefix}_{act_name}.hex", 24, True),
        "packed": O.pack_int4(q),
        "scale": sc,
        "expected_q26": read_hex(vec / f"{prefix}_{sub}expected_q26.hex", acc_width, True)[:keep_rows],
        "expected_q12_12": read_hex(vec / f"{prefix}_{sub}expected_q12_12.hex", 24, True)[:keep_rows],
        "rows_total": np.int64(rows),
    }


def build_kats(vec: Path) -> dict[str, dict]:
    k: dict[str, dict] = {}
    # dot64/row GEMV on Q4.12 activations (15_export_q4_projection_vectors.py)
    for name, rows in (("q4_gemv_projection_1024_real", 16), ("q4_gemv_tile_1024", 4)):
        q = read_hex(vec / f"{name}_weight.hex", 4, True).astype(np.int8).reshape(rows, 1024)
        k[name] = {
            "activation": read_hex(vec / f"{name}_activation.hex", 16, True),
            "packed": O.pack_int4(q),
            "scale": read_hex(vec / f"{name}_scale.hex", 16, False).astype(np.uint16).reshape(rows, 16),
            "expected_q26": read_hex(vec / f"{name}_expected.hex", 48, True),
        }
    for pre, keep in (("", 256), ("layer1_chained_", 64), ("layer2_chained_", 64)):
        base = f"{pre}mlp_gate_up_proj_stage_real"
        for which in ("gate", "up"):
            k[f"{base}_{which}"] = kat_gemv_words(vec, base, f"{which}_", 3072, 1024, 56, keep)
        base = f"{pre}mlp_down_proj_stage_real"
        k[base] = kat_gemv_words(vec, base, "", 1024, 3072, 58, keep // 2)
        base = f"{pre}o_proj_stage_real"
        k[base] = kat_gemv_words(vec, base, "", 1024, 2048, 64, keep // 2)
    # LM head scan window: 1024 tied rows, logits and running argmax
    name = "lm_head_argmax_stage_real"
    w = read_hex(vec / f"{name}_weight_words32.hex", 32, False)
    s = read_hex(vec / f"{name}_scale_words32.hex", 32, False)
    k[name] = {
        "activation": read_hex(vec / f"{name}_activation.hex", 24, True),
        "packed": O.pack_int4(words32_to_q4(w, 1024, 1024)),
        "scale": words32_to_u16(s, 1024 * 16).reshape(1024, 16),
        "expected_logits_q26": read_hex(vec / f"{name}_expected_scan_logits_q26.hex", 56, True),
        "best_token": read_hex(vec / f"{name}_expected_best_token.hex", 32, False),
        "best_score_q26": read_hex(vec / f"{name}_expected_best_score_q26.hex", 56, True),
    }
    # hidden-size RMSNorms
    for name in ("rmsnorm_1024_real", "final_rmsnorm_stage_real",
                 "final_rmsnorm_layer2_chained_stage_real", "layer1_chained_input_rmsnorm_stage_real",
                 "layer2_chained_input_rmsnorm_stage_real"):
        if not (vec / f"{name}_input.hex").exists():
            continue
        k[name] = {
            "input": read_hex(vec / f"{name}_input.hex", 24, True),
            "gamma": read_hex(vec / f"{name}_gamma.hex", 16, True),
            "expected": read_hex(vec / f"{name}_expected.hex", 24, True),
            "sum_squares": read_hex(vec / f"{name}_sum_squares.hex", 64, True),
            "mean_square": read_hex(vec / f"{name}_mean_square.hex", 64, True),
            "sqrt_radicand": read_hex(vec / f"{name}_sqrt_radicand.hex", 64, True),
            "rms": read_hex(vec / f"{name}_rms.hex", 24, False),
            "inv_rms": read_hex(vec / f"{name}_inv_rms.hex", 24, False),
        }
    for pre in ("", "layer1_chained_", "layer2_chained_"):
        name = f"{pre}post_attention_residual_norm_stage_real"
        k[name] = {
            "residual_input": read_hex(vec / f"{name}_residual_input.hex", 24, True),
            "o_proj_input": read_hex(vec / f"{name}_o_proj_input.hex", 24, True),
            "expected_residual": read_hex(vec / f"{name}_expected_residual.hex", 24, True),
            "gamma": read_hex(vec / f"{name}_gamma.hex", 16, True),
            "expected_norm": read_hex(vec / f"{name}_expected_norm.hex", 24, True),
            "inv_rms": read_hex(vec / f"{name}_inv_rms.hex", 24, False),
        }
        name = f"{pre}qk_norm_rope_stage_128_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("q_input", 24, True), ("k_input", 24, True), ("q_gamma", 16, True), ("k_gamma", 16, True),
            ("cos", 16, True), ("sin", 16, True), ("q_norm_expected", 24, True),
            ("k_norm_expected", 24, True), ("q_rope_expected", 24, True),
            ("k_rope_expected", 24, True))}
        name = f"{pre}kv_cache_append_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("k_input", 24, True), ("v_input", 24, True), ("expected_addr", 63, False),
            ("expected_data", 32, False), ("expected_kind", 4, False), ("expected_head", 8, False),
            ("expected_dim", 8, False))}
        name = f"{pre}attention_score_stage_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("q_input", 24, True), ("k_cache", 24, True), ("score_scale_q0_31", 32, False),
            ("cache_length", 16, False), ("expected_raw", 64, True), ("expected_scaled", 64, True),
            ("expected_q_head", 8, False), ("expected_kv_head", 8, False),
            ("expected_position", 8, False))}
        name = f"{pre}attention_softmax_value_stage_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("score_input", 64, True), ("v_cache", 24, True), ("exp_lut", 24, False),
            ("cache_length", 16, False), ("expected_prob", 24, False),
            ("expected_lut_index", 16, False), ("expected_out", 24, True),
            ("score_q_head", 8, False), ("score_position", 8, False))}
        name = f"{pre}mlp_silu_mul_stage_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("gate_input", 24, True), ("up_input", 24, True), ("sigmoid_lut", 16, False),
            ("expected_lut_index", 16, False), ("expected_sigmoid_q0_16", 16, False),
            ("expected_silu_gate_q12_12", 24, True), ("expected_hidden_q12_12", 24, True))}
        name = f"{pre}mlp_residual_add_stage_real"
        k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
            ("post_attn_hidden", 24, True), ("down_out", 24, True),
            ("expected_layer_out", 24, True))}
    name = "rope_qk_layer_128_real"
    k[name] = {f: read_hex(vec / f"{name}_{f}.hex", w, sg) for f, w, sg in (
        ("q_input", 24, True), ("k_input", 24, True), ("cos", 16, True), ("sin", 16, True),
        ("q_expected", 24, True), ("k_expected", 24, True))}
    return k


# --------------------------------------------------------------------------
# 2. reference helpers on seeded synthetic inputs
# --------------------------------------------------------------------------
def load_helper(mod_dir: Path, filename: str, name: str):
    spec = importlib.util.spec_from_file_location(name, mod_dir / filename)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def helpers(mod_dir: Path) -> dict:
    sys.path.insert(0, str(mod_dir))
    names = {
        "q4": "13_export_q4_gemv_vectors.py", "rms": "17_export_rmsnorm_fixed_vectors.py",
        "qmap": "21_export_qmap_qkv_projection_image.py",
        "qk": "22_export_qk_norm_rope_fixed_vectors.py", "kv": "23_export_kv_cache_append_vectors.py",
        "chained": "46_export_chained_attention_score_value_vectors.py",
        "o_proj": "26_export_o_proj_vectors.py", "post": "27_export_post_attention_residual_norm_vectors.py",
        "gate_up": "28_export_mlp_gate_up_vectors.py", "silu": "29_export_mlp_silu_mul_vectors.py",
        "down": "30_export_mlp_down_vectors.py", "residual": "31_export_mlp_residual_add_vectors.py",
        "embedding": "49_export_q4_embedding_vectors.py",
        "final_norm": "32_export_final_rmsnorm_vectors.py",
        "lm_head": "35_export_lm_head_full_vocab_vectors.py",
    }
    h = {k: load_helper(mod_dir, f, f"golden_{k}") for k, f in names.items()}
    h["m56"] = load_helper(mod_dir, "56_export_persistent_multitoken_layer_golden.py", "golden_m56")
    return h


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def build_ref_helpers(h: dict, ref_root: Path) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(1234)

    # -- quantisers: synthetic rows plus edge rows (zero, tiny, large, ties)
    w = O.synth_f32(1, 1000, (64, 1024), 0.02)
    w[0] = 0.0
    w[1] = 1.0e-6
    w[2] = rng.normal(0.0, 1.0, 1024).astype(np.float32)
    w[3, :64] = np.float32(7.0 * 0.5)
    w[3, 1:64:2] = np.float32(0.25)  # w/scale lands on .5 -> round-half-even
    out["quant_w"] = w
    packed, scale, q = h["q4"].quantize_weight_q4(w)
    out["quant13_packed"], out["quant13_scale"], out["quant13_q"] = packed, scale, q
    q35, s35 = h["lm_head"].quantize_weight_q4_chunk(w[:48])
    out["quant35_q"], out["quant35_scale"] = q35, s35
    q49, s49 = h["embedding"].quantize_row(w[5])
    out["quant49_q"], out["quant49_scale"] = q49, s49

    # -- cfg 1: gate_proj shaped GEMV, W seed 0, x ~ N(0,1) -> Q12.12
    w_cfg1 = O.synth_f32(0, O.layer_tid(0, O.T_GATE), (3072, 1024), 0.02)
    x_cfg1 = O.synth_f32(0, 900, (1024,), 1.0, bf16=False)
    xq, _ = h["rms"].quantize_signed(x_cfg1, 24, 12), None
    xq = np.asarray(xq, dtype=I64)
    qg, sg = h["gate_up"].quantize_weight_q4(w_cfg1)
    out["cfg1_w_sha"] = np.frombuffer(sha(w_cfg1).encode(), dtype=np.uint8)
    out["cfg1_q_sha"] = np.frombuffer(sha(qg).encode(), dtype=np.uint8)
    out["cfg1_s_sha"] = np.frombuffer(sha(sg).encode(), dtype=np.uint8)
    out["cfg1_act_q12_12"] = xq
    rs = h["gate_up"].compute_q4_gemv_q26(xq, qg, sg)
    o12, sat = h["gate_up"].q26_to_q12_12(rs)
    out["cfg1_q26"], out["cfg1_q12_12"], out["cfg1_sat"] = rs, o12, np.int64(sat)
    pk, _, _ = h["q4"].quantize_weight_q4(w_cfg1)
    mo = h["qmap"].compute_matrix_outputs(activation_q12_12=xq, packed_weight=pk, scale_q2_14=sg,
                                          actual_q4_float=None, matrix_name="cfg1", row_count=3072)
    out["cfg1_matrix_q26"], out["cfg1_matrix_q12_12"] = mo["row_sum_q26"], mo["q12_12"].astype(I64)

    # -- extreme GEMV: activations at the signed 24-bit limits, weights -8/7,
    #    scales at 0xFFFF, for K = 1024 (28), 2048 (26), 3072 (30)
    for tag, mod, k, rows, keep in (("k1024", "gate_up", 1024, 3072, 192),
                                    ("k2048", "o_proj", 2048, 1024, 96), ("k3072", "down", 3072, 1024, 64)):
        act = rng.integers(-(1 << 23), 1 << 23, k).astype(I64)
        act[: k // 4] = -(1 << 23)
        act[k // 4: k // 2] = (1 << 23) - 1
        qw = rng.integers(-8, 8, (rows, k)).astype(np.int8)
        qw[0] = -8
        qw[1, : k // 4] = -8
        qw[1, k // 4:] = 7
        sc = rng.integers(0, 1 << 16, (rows, k // 64)).astype(np.uint16)
        sc[0] = 0xFFFF
        sc[1] = 0xFFFF
        # the reference helpers take full-height matrices; keep a row prefix
        rs = getattr(h[mod], "compute_q4_gemv_q26")(act, qw, sc)[:keep]
        qw, sc = qw[:keep], sc[:keep]
        o12, sat = h[mod].q26_to_q12_12(rs)
        out[f"xgemv_{tag}_act"], out[f"xgemv_{tag}_packed"] = act, O.pack_int4(qw)
        out[f"xgemv_{tag}_scale"], out[f"xgemv_{tag}_q26"] = sc, rs
        out[f"xgemv_{tag}_q12_12"], out[f"xgemv_{tag}_sat"] = o12, np.int64(sat)

    # -- hidden RMSNorm (17): random, zero, tiny, saturating
    cases = [rng.integers(-4000, 4000, 1024), np.zeros(1024, dtype=I64), rng.integers(-1, 2, 1024),
             rng.integers(-(1 << 23), 1 << 23, 1024)]
    gammas = [rng.integers(90, 170, 1024), np.full(1024, 128), rng.integers(-300, 300, 1024),
              np.full(1024, 32767)]
    for i, (x, g) in enumerate(zip(cases, gammas)):
        r = h["rms"].fixed_rmsnorm_reference(np.asarray(x, dtype=I64), np.asarray(g, dtype=I64))
        out[f"rms{i}_x"], out[f"rms{i}_g"] = np.asarray(x, dtype=I64), np.asarray(g, dtype=I64)
        out[f"rms{i}_out"] = r["output_q12_12"]
        out[f"rms{i}_inv"], out[f"rms{i}_rms"] = np.int64(r["inv_rms_uq8_16"]), np.int64(r["rms_q14_10"])
        out[f"rms{i}_sat"] = np.int64(r["saturation"])

    # -- per-head norm + RoPE (22)
    tab_pos = np.asarray(list(range(0, 260)) + [511, 512, 513, 1000, 4095, 8191, 8703])
    import torch
    from transformers import AutoConfig
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    cfg = AutoConfig.from_pretrained(ref_root / "Qwen3-0.6B-Base")
    remb = Qwen3RotaryEmbedding(cfg)
    common = sys.modules["common"]
    with torch.no_grad():
        cos, sin = common.manual_rope_cos_sin(remb, torch.zeros(1, len(tab_pos), 1024),
                                              torch.as_tensor(tab_pos)[None, :])
    cq = np.stack([h["qk"].quantize_signed(cos[0, i].numpy(), 16, 15)[0] for i in range(len(tab_pos))])
    sq = np.stack([h["qk"].quantize_signed(sin[0, i].numpy(), 16, 15)[0] for i in range(len(tab_pos))])
    out["rope_positions"], out["rope_cos"], out["rope_sin"] = tab_pos.astype(I64), cq, sq
    out["rope_inv_freq"] = remb.inv_freq.numpy().astype(np.float32)
    xh = rng.integers(-30000, 30000, (16, 128)).astype(I64)
    xh[3] = 0
    xh[4] = rng.integers(-(1 << 23), 1 << 23, 128)
    xh[5] = rng.integers(-2, 3, 128)
    gh = rng.integers(-200, 400, 128).astype(I64)
    nrm, _, nsat = h["qk"].fixed_rmsnorm_heads(xh, gh)
    out["heads_x"], out["heads_g"], out["heads_out"], out["heads_sat"] = xh, gh, nrm, np.int64(nsat)
    xr = rng.integers(-(1 << 23), 1 << 23, (24, 128)).astype(I64)
    xr[:4] = nrm[:4]
    for j, pi in enumerate((0, 7, 259, 265)):
        ro, rsat = h["qk"].fixed_rope_reference(xr, cq[pi], sq[pi])
        out[f"rope{j}_pos_index"], out[f"rope{j}_out"], out[f"rope{j}_sat"] = np.int64(pi), ro, np.int64(rsat)
    out["rope_x"] = xr

    # -- attention score scaling, softmax, value accumulation (46 / 56)
    ch = h["chained"]
    dots = np.concatenate([rng.integers(-(1 << 50), 1 << 50, 200), [0, -1, 1, (1 << 47), -(1 << 47),
                                                                    (1 << 53) - 1, -(1 << 53)]]).astype(I64)
    out["scale_dots"] = dots
    out["scale_out"] = np.asarray([ch.arithmetic_shift_right(int(d) * O.SCORE_SCALE_Q0_31, ch.SCALE_FRAC)
                                   for d in dots], dtype=I64)
    out["exp_lut"] = ch.build_exp_lut()
    for j, ctx in enumerate((1, 7, 96, 600)):
        s = rng.integers(-(1 << 28), 1 << 28, (16, ctx)).astype(I64)
        if ctx >= 7:
            s[0, :] = 5  # all equal
            s[1, 1] = s[1].max() + (1 << 34)  # one dominant, rest clamp to index 256
            s[2, : ctx // 2] = s[2, ctx // 2]  # many ties with the max
        probs, idx = ch.fixed_softmax_probs(s, out["exp_lut"])
        v = rng.integers(-(1 << 23), 1 << 23, (ctx, 8, 128)).astype(I64)
        if ctx > 128:
            v = rng.integers(-(1 << 23), 1 << 23, (ctx, 8, 1)).astype(I64) * np.ones(128, dtype=I64)
        if ctx >= 7:
            v[:, 0, :] = (1 << 23) - 1  # saturating accumulation for heads 0/1
        vo, vsat = ch.fixed_value_accum(probs, v)
        out[f"sm{j}_scores"], out[f"sm{j}_probs"], out[f"sm{j}_idx"] = s, probs, idx
        out[f"sm{j}_v"], out[f"sm{j}_out"], out[f"sm{j}_sat"] = v, vo, np.int64(vsat)
    # whole attention for one position (56_...:359-395)
    ctx = 9
    qa = rng.integers(-200000, 200000, (16, 128)).astype(I64)
    ka = rng.integers(-1500000, 1500000, (ctx, 8, 128)).astype(I64)
    va = rng.integers(-6000, 6000, (ctx, 8, 128)).astype(I64)
    att = h["m56"].attention_score_value(attention_helper=ch, q_current=qa, k_cache=ka, v_cache=va,
                                         score_scale_q0_31=O.SCORE_SCALE_Q0_31, exp_lut=out["exp_lut"])
    out["att_q"], out["att_k"], out["att_v"] = qa, ka, va
    for f in ("raw", "scaled", "probs", "lut_indices", "output"):
        out[f"att_{f}"] = np.asarray(att[f], dtype=I64)

    # -- SwiGLU LUT path (29 + 56_...:546-556)
    si = h["silu"]
    out["sigmoid_lut"] = si.build_sigmoid_lut()
    g = np.concatenate([np.arange(-40000, 40000, 37), [-(1 << 23), (1 << 23) - 1, -32768, 32768,
                                                       -32769, 32769, 0, 31, 32, 33, -31, -32, -33]])
    g = g.astype(I64)
    u = rng.integers(-(1 << 23), 1 << 23, g.size).astype(I64)
    idx = si.gate_to_lut_index(g)
    sg_ = out["sigmoid_lut"][idx]
    silu, s1 = si.saturate_signed_array((g * sg_) >> si.SIGMOID_FRAC, si.OUT_WIDTH)
    hid, s2 = si.saturate_signed_array((silu * u) >> si.IN_FRAC, si.OUT_WIDTH)
    out["silu_gate"], out["silu_up"], out["silu_idx"] = g, u, idx
    out["silu_silu"], out["silu_hidden"] = silu, hid

    # -- KV addresses (23) at the reference's 256 cap and an extended cap
    pts = rng.integers(0, [28, 2, 8, 256, 128], (64, 5))
    out["kv_points"] = pts.astype(I64)
    out["kv_addr"] = np.asarray([h["kv"].kv_addr(base_addr=O.KV_CACHE_BASE_ADDR, layer_id=int(a),
                                                 kv_kind=int(b), head=int(c), position=int(d), dim=int(e))
                                 for a, b, c, d, e in pts], dtype=I64)
    sv = rng.integers(-(1 << 23), 1 << 23, 64)
    out["kv_sext_in"] = sv.astype(I64)
    out["kv_sext_out"] = np.asarray([h["kv"].sign_extend_to_word(int(x)) for x in sv], dtype=I64)

    # -- tied embedding rows of the seed-0 model (56_...:190-226)
    toks = [0, 1, 374, 151935, 65536]
    rows = np.stack([O.synth_centered(0, O.TID_EMBED, 1024, start=t * 1024) for t in toks])
    erows = O.bf16_round(rows.astype(np.float32) * (np.float32(0.02) * np.float32(2.0 ** -16)))
    emb = np.zeros((151936, 1024), dtype=np.float32)
    emb[toks] = erows
    et = torch.from_numpy(emb)
    model = SimpleNamespace(lm_head=SimpleNamespace(weight=et), dtype=torch.float32)
    backbone = SimpleNamespace(embed_tokens=SimpleNamespace(weight=et))
    hid, _ = h["m56"].q4_embedding_hidden(token_ids=toks, model=model, backbone=backbone,
                                          embedding_helper=h["embedding"])
    out["embed_tokens"], out["embed_hidden"] = np.asarray(toks, dtype=I64), hid
    # 24-bit data is stored as int32 to keep the fixture small
    for key, val in out.items():
        if val.dtype == np.int64 and val.size > 64 and val.min() >= -(1 << 31) and val.max() < (1 << 31):
            out[key] = val.astype(np.int32)
    return out


# --------------------------------------------------------------------------
# 3. whole-model teacher-forced golden on the seed-0 synthetic model
# --------------------------------------------------------------------------
def synth_model_f32(seed: int) -> tuple[np.ndarray, list, np.ndarray]:
    emb = O.synth_f32(seed, O.TID_EMBED, (O.VOCAB, O.HIDDEN), 0.02)
    layers = []
    for li in range(O.LAYERS):
        layers.append({w: O.synth_f32(seed, O.layer_tid(li, w), shp, 0.02)
                       for w, shp in O.LAYER_SHAPES.items()})
    return emb, layers, np.ones(O.HIDDEN, dtype=np.float32)


def oracle_model(emb, layers) -> O.Model:
    ones_h = O.quantize_signed(np.ones(O.HIDDEN), 16, 7)[0]
    ones_d = O.quantize_signed(np.ones(O.HEAD_DIM), 16, 7)[0]
    lps = []
    for d in layers:
        qs = {w: O.quantize_weight_q4(d[w]) for w in O.LAYER_SHAPES}
        lps.append(O.LayerParams(
            q_w=qs[O.T_Q][0], q_s=qs[O.T_Q][1], k_w=qs[O.T_K][0], k_s=qs[O.T_K][1],
            v_w=qs[O.T_V][0], v_s=qs[O.T_V][1], o_w=qs[O.T_O][0], o_s=qs[O.T_O][1],
            gate_w=qs[O.T_GATE][0], gate_s=qs[O.T_GATE][1], up_w=qs[O.T_UP][0], up_s=qs[O.T_UP][1],
            down_w=qs[O.T_DOWN][0], down_s=qs[O.T_DOWN][1], input_gamma=ones_h, post_gamma=ones_h,
            q_gamma=ones_d, k_gamma=ones_d))
    eq, es = O.quantize_weight_q4(emb)
    return O.Model(layers=lps, embed_q=eq, embed_s=es, final_gamma=ones_h)


def build_ref_model(h: dict, ref_root: Path, prompt_len: int, new_tokens: int) -> dict[str, np.ndarray]:
    import torch
    from transformers import AutoConfig
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    t0 = time.time()
    emb, layers, _ = synth_model_f32(0)
    print(f"synthetic seed-0 model built in {time.time() - t0:.1f}s")
    prompt = np.random.default_rng(0).integers(0, O.VOCAB, 128)[:prompt_len].tolist()
    m = oracle_model(emb, layers)
    m.cos, m.sin = O.rope_tables(prompt_len + new_tokens)
    t0 = time.time()
    gen, gen_scores = O.greedy_decode(m, prompt, new_tokens)
    print(f"oracle greedy decode {gen} in {time.time() - t0:.1f}s")
    tokens = prompt + gen[:-1]

    # The reference's chained functions, driven as its main() does (56_...:866-1037)
    cfg = AutoConfig.from_pretrained(ref_root / "Qwen3-0.6B-Base")
    remb = Qwen3RotaryEmbedding(cfg)
    common = sys.modules["common"]
    with torch.no_grad():
        cos, sin = common.manual_rope_cos_sin(remb, torch.zeros(1, len(tokens), 1024),
                                              torch.arange(len(tokens))[None, :])
    cq = np.stack([h["qk"].quantize_signed(cos[0, p].numpy(), 16, 15)[0] for p in range(len(tokens))])
    sq = np.stack([h["qk"].quantize_signed(sin[0, p].numpy(), 16, 15)[0] for p in range(len(tokens))])

    def lin(wt):
        return SimpleNamespace(weight=torch.from_numpy(wt))

    ones = lambda n: SimpleNamespace(weight=torch.ones(n))  # noqa: E731
    et = torch.from_numpy(emb)
    model = SimpleNamespace(lm_head=SimpleNamespace(weight=et), dtype=torch.float32)
    backbone = SimpleNamespace(embed_tokens=SimpleNamespace(weight=et), norm=ones(1024))
    hidden, _ = h["m56"].q4_embedding_hidden(token_ids=tokens, model=model, backbone=backbone,
                                             embedding_helper=h["embedding"])
    helper_map = {k: h[k] for k in ("q4", "rms", "qmap", "qk", "kv", "chained", "o_proj", "post",
                                    "gate_up", "silu", "down", "residual")}
    tok_stub = SimpleNamespace(decode=lambda ids: "")
    exp_lut = h["chained"].build_exp_lut()
    sig_lut = h["silu"].build_sigmoid_lut()
    layer0_out = None
    with tempfile.TemporaryDirectory() as td:
        files: dict = {}
        cur = hidden
        t0 = time.time()
        for li, d in enumerate(layers):
            layer = SimpleNamespace(
                self_attn=SimpleNamespace(q_proj=lin(d[O.T_Q]), k_proj=lin(d[O.T_K]), v_proj=lin(d[O.T_V]),
                                          o_proj=lin(d[O.T_O]), q_norm=ones(128), k_norm=ones(128),
                                          scaling=128 ** -0.5),
                mlp=SimpleNamespace(gate_proj=lin(d[O.T_GATE]), up_proj=lin(d[O.T_UP]),
                                    down_proj=lin(d[O.T_DOWN])),
                input_layernorm=ones(1024), post_attention_layernorm=ones(1024))
            cur, _, _ = h["m56"].run_fixed_layer(
                layer_id=li, layer=layer, token_ids=tokens, hidden_inputs=cur, cos_q1_15=cq, sin_q1_15=sq,
                kv_cache_base=O.KV_CACHE_BASE_ADDR, tokenizer=tok_stub, helpers=helper_map,
                output_dir=Path(td), files=files, scope=f"layer_{li:02d}", exp_lut=exp_lut,
                sigmoid_lut=sig_lut)
            if li == 0:
                layer0_out = np.asarray(cur, dtype=I64).copy()
            print(f"reference layer {li} done ({time.time() - t0:.1f}s)")
        tail = h["m56"].run_final_tail(
            final_hidden=cur, token_ids=tokens, tokenizer=tok_stub, model=model, backbone=backbone,
            final_norm=h["final_norm"], lm_head=h["lm_head"], chained=h["chained"], output_dir=Path(td),
            files=files, chunk_rows=1024, full_model=True)
    argmax = np.asarray([r["argmax_token"] for r in tail["position_results"]], dtype=I64)
    scores = np.asarray([r["argmax_score_q26"] for r in tail["position_results"]], dtype=I64)
    expect = np.asarray(gen, dtype=I64)
    got = argmax[prompt_len - 1:]
    print("reference argmax from the last prompt position:", got.tolist(), "oracle:", expect.tolist())
    if not np.array_equal(got, expect):
        raise SystemExit("oracle greedy decode disagrees with the reference chain")
    return {"prompt": np.asarray(prompt, dtype=I64), "tokens": np.asarray(tokens, dtype=I64),
            "argmax": argmax, "scores": scores, "generated": expect,
            "generated_scores": np.asarray(gen_scores, dtype=I64), "final_hidden": np.asarray(cur, dtype=I64),
            "layer0_out": layer0_out, "embed_hidden": np.asarray(hidden, dtype=I64), "cos": cq, "sin": sq}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="reference project root")
    ap.add_argument("--skip-model", action="store_true", help="skip the whole-model golden")
    ap.add_argument("--prompt-len", type=int, default=5)
    ap.add_argument("--new-tokens", type=int, default=4)
    a = ap.parse_args()
    ref = a.reference.resolve()
    vec = ref / "FPGA_Project" / "sim" / "vectors"
    kats = build_kats(vec)
    np.savez_compressed(HERE / "kat_vectors.npz",
                        **{f"{n}/{f}": v for n, d in kats.items() for f, v in d.items()})
    print(f"wrote {len(kats)} KAT sets")
    h = helpers(ref / "Qwen3-0.6B-Base" / "python_each_module")
    np.savez_compressed(HERE / "ref_helpers.npz", **build_ref_helpers(h, ref))
    print("wrote reference helper goldens")
    if not a.skip_model:
        np.savez_compressed(HERE / "ref_model_seed0.npz",
                            **build_ref_model(h, ref, a.prompt_len, a.new_tokens))
        print("wrote whole-model golden")


if __name__ == "__main__":
    main()
