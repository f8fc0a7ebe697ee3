"""Pin the CPU oracle to the reference: its RTL golden vectors (real Qwen3
layer 0/1/2 data) and outputs of its own Python helpers.  CPU only."""
import numpy as np
import pytest

from oracle import q4_oracle as O

GEMV_KATS = [
    "mlp_gate_up_proj_stage_real_gate", "mlp_gate_up_proj_stage_real_up", "mlp_down_proj_stage_real",
    "o_proj_stage_real",
    "layer1_chained_mlp_gate_up_proj_stage_real_gate", "layer1_chained_mlp_gate_up_proj_stage_real_up",
    "layer1_chained_mlp_down_proj_stage_real", "layer1_chained_o_proj_stage_real",
    "layer2_chained_mlp_gate_up_proj_stage_real_gate", "layer2_chained_mlp_gate_up_proj_stage_real_up",
    "layer2_chained_mlp_down_proj_stage_real", "layer2_chained_o_proj_stage_real",
]
PREFIXES = ["", "layer1_chained_", "layer2_chained_"]


@pytest.mark.parametrize("name", ["q4_gemv_projection_1024_real", "q4_gemv_tile_1024"])
def test_dot_row_kat(kat, name):
    g = kat.group(name)
    rs = O.gemv_q26_packed(g["activation"], g["packed"], g["scale"])
    assert np.array_equal(rs, g["expected_q26"])


@pytest.mark.parametrize("name", GEMV_KATS)
def test_gemv_stage_kat(kat, name):
    g = kat.group(name)
    rs = O.gemv_q26_packed(g["activation"], g["packed"], g["scale"])
    assert np.array_equal(rs, g["expected_q26"])
    out, _ = O.q26_to_q12_12(rs)
    assert np.array_equal(out, g["expected_q12_12"])


def test_lm_head_kat(kat):
    g = kat.group("lm_head_argmax_stage_real")
    logits = O.gemv_q26_packed(g["activation"], g["packed"], g["scale"])
    assert np.array_equal(logits, g["expected_logits_q26"])
    tok, score = O.lm_head_argmax(logits)
    assert tok == int(g["best_token"][0]) == 264
    assert score == int(g["best_score_q26"][0]) == 1365150750


@pytest.mark.parametrize("name", ["rmsnorm_1024_real", "final_rmsnorm_stage_real",
                                  "final_rmsnorm_layer2_chained_stage_real",
                                  "layer1_chained_input_rmsnorm_stage_real",
                                  "layer2_chained_input_rmsnorm_stage_real"])
def test_rmsnorm_kat(kat, name):
    g = kat.group(name)
    if not g:
        pytest.skip("KAT not in this reference snapshot")
    r = O.rmsnorm(g["input"], g["gamma"])
    assert np.array_equal(r["output"], g["expected"])
    for f, k in (("sum_squares", "sum_squares"), ("mean_square", "mean_square"),
                 ("sqrt_radicand", "sqrt_radicand"), ("rms", "rms"), ("inv_rms", "inv_rms")):
        assert int(r[f]) == int(g[k][0]), f


def test_rmsnorm_known_scalars(kat):
    # Source/QMAP_FORMAT.md:599-603 quotes these for the layer-0 input norm
    r = O.rmsnorm(kat["rmsnorm_1024_real/input"], kat["rmsnorm_1024_real/gamma"])
    assert (int(r["sum_squares"]), int(r["mean_square"]), int(r["inv_rms"])) == (589959, 576, 2796202)


@pytest.mark.parametrize("pre", PREFIXES)
def test_post_attention_residual_norm_kat(kat, pre):
    g = kat.group(f"{pre}post_attention_residual_norm_stage_real")
    post, _ = O.saturate(g["residual_input"] + (g["o_proj_input"] >> O.O_TO_RESIDUAL_SHIFT), 24)
    assert np.array_equal(post, g["expected_residual"])
    r = O.rmsnorm(post, g["gamma"])
    assert np.array_equal(r["output"], g["expected_norm"])
    assert int(r["inv_rms"]) == int(g["inv_rms"][0])


@pytest.mark.parametrize("pre", PREFIXES)
def test_qk_norm_rope_kat(kat, pre):
    g = kat.group(f"{pre}qk_norm_rope_stage_128_real")
    qn, _, _ = O.rmsnorm_heads(g["q_input"].reshape(16, 128), g["q_gamma"])
    kn, _, _ = O.rmsnorm_heads(g["k_input"].reshape(8, 128), g["k_gamma"])
    assert np.array_equal(qn.reshape(-1), g["q_norm_expected"])
    assert np.array_equal(kn.reshape(-1), g["k_norm_expected"])
    qr, _ = O.rope(qn, g["cos"], g["sin"])
    kr, _ = O.rope(kn, g["cos"], g["sin"])
    assert np.array_equal(qr.reshape(-1), g["q_rope_expected"])
    assert np.array_equal(kr.reshape(-1), g["k_rope_expected"])


def test_rope_kat(kat):
    g = kat.group("rope_qk_layer_128_real")
    qr, _ = O.rope(g["q_input"].reshape(16, 128), g["cos"], g["sin"])
    kr, _ = O.rope(g["k_input"].reshape(8, 128), g["cos"], g["sin"])
    assert np.array_equal(qr.reshape(-1), g["q_expected"])
    assert np.array_equal(kr.reshape(-1), g["k_expected"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_kv_append_kat(kat, pre):
    g = kat.group(f"{pre}kv_cache_append_real")
    layer = {"": 0, "layer1_chained_": 1, "layer2_chained_": 2}[pre]
    tr = O.kv_write_trace(O.KV_CACHE_BASE_ADDR, layer, 4, g["k_input"], g["v_input"])
    for f in ("addr", "data", "kind", "head", "dim"):
        assert np.array_equal(tr[f], g[f"expected_{f}"].astype(np.int64)), f


@pytest.mark.parametrize("pre", PREFIXES)
def test_attention_score_kat(kat, pre):
    g = kat.group(f"{pre}attention_score_stage_real")
    ctx = int(g["cache_length"][0])
    assert int(g["score_scale_q0_31"][0]) == O.SCORE_SCALE_Q0_31 == 189812531
    raw, scaled = O.attention_scores(g["q_input"].reshape(16, 128), g["k_cache"].reshape(ctx, 8, 128))
    order = (g["expected_q_head"], g["expected_position"])
    assert np.array_equal(raw[order], g["expected_raw"])
    assert np.array_equal(scaled[order], g["expected_scaled"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_softmax_value_kat(kat, pre):
    g = kat.group(f"{pre}attention_softmax_value_stage_real")
    ctx = int(g["cache_length"][0])
    lut = O.build_exp_lut()
    assert np.array_equal(lut, g["exp_lut"])
    scores = np.zeros((16, ctx), dtype=np.int64)
    scores[g["score_q_head"], g["score_position"]] = g["score_input"]
    probs, idx = O.softmax_probs(scores, lut)
    order = (g["score_q_head"], g["score_position"])
    assert np.array_equal(probs[order], g["expected_prob"])
    assert np.array_equal(idx[order], g["expected_lut_index"])
    out, _ = O.value_accum(probs, g["v_cache"].reshape(ctx, 8, 128))
    assert np.array_equal(out.reshape(-1), g["expected_out"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_silu_mul_kat(kat, pre):
    g = kat.group(f"{pre}mlp_silu_mul_stage_real")
    lut = O.build_sigmoid_lut()
    assert np.array_equal(lut, g["sigmoid_lut"])
    r = O.silu_mul(g["gate_input"], g["up_input"], lut)
    assert np.array_equal(r["lut_index"], g["expected_lut_index"])
    assert np.array_equal(r["sigmoid"], g["expected_sigmoid_q0_16"])
    assert np.array_equal(r["silu"], g["expected_silu_gate_q12_12"])
    assert np.array_equal(r["hidden"], g["expected_hidden_q12_12"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_mlp_residual_kat(kat, pre):
    g = kat.group(f"{pre}mlp_residual_add_stage_real")
    out, _ = O.saturate(g["post_attn_hidden"] + (g["down_out"] >> O.DOWN_TO_OUT_SHIFT), 24)
    assert np.array_equal(out, g["expected_layer_out"])


# ---------------------------------------------------------------------------
# reference helpers on synthetic inputs
# ---------------------------------------------------------------------------
def test_quantizers_match_reference(refh):
    w = refh["quant_w"]
    q, s = O.quantize_weight_q4(w)
    assert np.array_equal(q, refh["quant13_q"]) and np.array_equal(s, refh["quant13_scale"])
    assert np.array_equal(O.pack_int4(q), refh["quant13_packed"])
    assert np.array_equal(O.unpack_int4(refh["quant13_packed"], 1024), q)
    q35, s35 = O.quantize_weight_q4(w[:48])
    assert np.array_equal(q35, refh["quant35_q"]) and np.array_equal(s35, refh["quant35_scale"])
    q49, s49 = O.quantize_weight_q4(w[5:6])
    assert np.array_equal(q49[0], refh["quant49_q"]) and np.array_equal(s49[0], refh["quant49_scale"])
    # edge rows: zero group -> scale 0 and q 0; tiny -> scale forced to 1
    assert np.all(s[0] == 0) and np.all(q[0] == 0)
    assert np.all(s[1] == 1)


def _sha(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_cfg1_gemv_matches_reference(refh):
    w = O.synth_f32(0, O.layer_tid(0, O.T_GATE), (3072, 1024), 0.02)
    assert _sha(w) == bytes(refh["cfg1_w_sha"]).decode()
    q, s = O.quantize_weight_q4(w)
    assert _sha(q) == bytes(refh["cfg1_q_sha"]).decode()
    assert _sha(s) == bytes(refh["cfg1_s_sha"]).decode()
    x = O.quantize_signed(O.synth_f32(0, 900, (1024,), 1.0, bf16=False), 24, 12)[0]
    assert np.array_equal(x, refh["cfg1_act_q12_12"])
    rs = O.gemv_q26(x, q, s)
    assert np.array_equal(rs, refh["cfg1_q26"])
    assert np.array_equal(rs, refh["cfg1_matrix_q26"])
    out, sat = O.q26_to_q12_12(rs)
    assert np.array_equal(out, refh["cfg1_q12_12"]) and sat == int(refh["cfg1_sat"])
    assert np.array_equal(out, refh["cfg1_matrix_q12_12"])


@pytest.mark.parametrize("tag", ["k1024", "k2048", "k3072"])
def test_extreme_gemv_matches_reference(refh, tag):
    rs = O.gemv_q26_packed(refh[f"xgemv_{tag}_act"], refh[f"xgemv_{tag}_packed"], refh[f"xgemv_{tag}_scale"])
    assert np.array_equal(rs, refh[f"xgemv_{tag}_q26"])
    out, sat = O.q26_to_q12_12(rs)
    assert np.array_equal(out, refh[f"xgemv_{tag}_q12_12"]) and sat == int(refh[f"xgemv_{tag}_sat"])


@pytest.mark.parametrize("i", range(4))
def test_rmsnorm_edge_cases(refh, i):
    r = O.rmsnorm(refh[f"rms{i}_x"], refh[f"rms{i}_g"])
    assert np.array_equal(r["output"], refh[f"rms{i}_out"])
    assert int(r["inv_rms"]) == int(refh[f"rms{i}_inv"]) and int(r["rms"]) == int(refh[f"rms{i}_rms"])
    assert (r["saturation_count"] > 0) == bool(refh[f"rms{i}_sat"])


def test_heads_norm_and_rope_match_reference(refh):
    out, _, sat = O.rmsnorm_heads(refh["heads_x"], refh["heads_g"])
    assert np.array_equal(out, refh["heads_out"]) and (sat > 0) == bool(refh["heads_sat"])
    for j in range(4):
        pi = int(refh[f"rope{j}_pos_index"])
        ro, rsat = O.rope(refh["rope_x"], refh["rope_cos"][pi], refh["rope_sin"][pi])
        assert np.array_equal(ro, refh[f"rope{j}_out"]) and (rsat > 0) == bool(refh[f"rope{j}_sat"])


def test_rope_tables_match_reference(refh):
    pos = refh["rope_positions"]
    assert np.array_equal(O.rope_inv_freq().numpy(), refh["rope_inv_freq"])
    c, s = O.rope_tables(int(pos.max()) + 1)
    assert np.array_equal(c[pos], refh["rope_cos"]) and np.array_equal(s[pos], refh["rope_sin"])


def test_score_scaling_is_exact(refh):
    assert np.array_equal(O.scale_scores(refh["scale_dots"]), refh["scale_out"])


@pytest.mark.parametrize("j", range(4))
def test_softmax_value_match_reference(refh, j):
    assert np.array_equal(O.build_exp_lut(), refh["exp_lut"])
    probs, idx = O.softmax_probs(refh[f"sm{j}_scores"], refh["exp_lut"])
    assert np.array_equal(probs, refh[f"sm{j}_probs"]) and np.array_equal(idx, refh[f"sm{j}_idx"])
    out, sat = O.value_accum(probs, refh[f"sm{j}_v"])
    assert np.array_equal(out, refh[f"sm{j}_out"]) and (sat > 0) == bool(refh[f"sm{j}_sat"])


def test_attention_matches_reference(refh):
    a = O.attention(refh["att_q"], refh["att_k"], refh["att_v"], refh["exp_lut"])
    for f in ("raw", "scaled", "probs", "lut_indices", "output"):
        assert np.array_equal(a[f], refh[f"att_{f}"]), f


def test_silu_matches_reference(refh):
    assert np.array_equal(O.build_sigmoid_lut(), refh["sigmoid_lut"])
    r = O.silu_mul(refh["silu_gate"], refh["silu_up"], refh["sigmoid_lut"])
    assert np.array_equal(r["lut_index"], refh["silu_idx"])
    assert np.array_equal(r["silu"], refh["silu_silu"]) and np.array_equal(r["hidden"], refh["silu_hidden"])


def test_kv_addr_matches_reference(refh):
    got = [O.kv_addr(O.KV_CACHE_BASE_ADDR, *map(int, p)) for p in refh["kv_points"]]
    assert np.array_equal(np.asarray(got, dtype=np.int64), refh["kv_addr"])
    ext = [O.sign_extend_to_word(int(x)) for x in refh["kv_sext_in"]]
    assert np.array_equal(np.asarray(ext, dtype=np.int64), refh["kv_sext_out"])


def test_embedding_matches_reference(refh):
    toks = refh["embed_tokens"]
    for i, t in enumerate(toks):
        c = O.synth_centered(0, O.TID_EMBED, 1024, start=int(t) * 1024)
        w = O.bf16_round(c.astype(np.float32) * (np.float32(0.02) * np.float32(2.0 ** -16)))
        q, s = O.quantize_weight_q4(w[None, :])
        assert np.array_equal(O.embedding_hidden(q[0], s[0]), refh["embed_hidden"][i])
