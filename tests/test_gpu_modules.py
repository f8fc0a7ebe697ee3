"""Per-module CUDA kernels vs the reference's golden vectors and the CPU
oracle: bit-exact for every stage."""
import numpy as np
import pytest

from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import reference_api as R  # noqa: E402

from test_oracle_golden import GEMV_KATS, PREFIXES  # noqa: E402


def _gemv_packed(act, packed, scale):
    return R.compute_matrix_outputs(activation_q12_12=act, packed_weight=packed, scale_q2_14=scale,
                                    actual_q4_float=None, matrix_name="kat", row_count=packed.shape[0])


@pytest.mark.parametrize("name", ["q4_gemv_projection_1024_real", "q4_gemv_tile_1024"])
def test_dot_row_kat(kat, name):
    g = kat.group(name)
    assert np.array_equal(_gemv_packed(g["activation"], g["packed"], g["scale"])["row_sum_q26"], g["expected_q26"])


@pytest.mark.parametrize("name", GEMV_KATS)
def test_gemv_stage_kat(kat, name):
    g = kat.group(name)
    r = _gemv_packed(g["activation"], g["packed"], g["scale"])
    assert np.array_equal(r["row_sum_q26"], g["expected_q26"])
    assert np.array_equal(r["q12_12"].astype(np.int64), g["expected_q12_12"])


def test_cfg1_gemv(refh):
    w = O.synth_f32(0, O.layer_tid(0, O.T_GATE), (3072, 1024), 0.02)
    q, s = R.quantize_weight_q4(w)  # device quantiser
    oq, os_ = O.quantize_weight_q4(w)
    assert np.array_equal(q, oq) and np.array_equal(s, os_)
    x = refh["cfg1_act_q12_12"].astype(np.int64)
    rs = R.compute_q4_gemv_q26(x, q, s)
    assert np.array_equal(rs, refh["cfg1_q26"])
    out, sat = R.q26_to_q12_12(rs)
    assert np.array_equal(out, refh["cfg1_q12_12"]) and sat == int(refh["cfg1_sat"])


@pytest.mark.parametrize("tag", ["k1024", "k2048", "k3072"])
def test_extreme_gemv(refh, tag):
    r = _gemv_packed(refh[f"xgemv_{tag}_act"], refh[f"xgemv_{tag}_packed"], refh[f"xgemv_{tag}_scale"])
    assert np.array_equal(r["row_sum_q26"], refh[f"xgemv_{tag}_q26"])
    assert np.array_equal(r["q12_12"].astype(np.int64), refh[f"xgemv_{tag}_q12_12"])


@pytest.mark.parametrize("k,rows", [(1024, 1), (1024, 3), (1024, 1000), (2048, 17), (3072, 33), (4096, 50)])
def test_gemv_random_shapes(k, rows):
    rng = np.random.default_rng(k + rows)
    q = rng.integers(-8, 8, (rows, k)).astype(np.int8)
    s = rng.integers(0, 1 << 16, (rows, k // 64)).astype(np.uint16)
    a = rng.integers(-(1 << 23), 1 << 23, k).astype(np.int64)
    assert np.array_equal(R.compute_q4_gemv_q26(a, q, s), O.gemv_q26(a, q, s))


def test_quantizer_edge_rows(refh):
    q, s = R.quantize_weight_q4(refh["quant_w"])
    assert np.array_equal(q, refh["quant13_q"]) and np.array_equal(s, refh["quant13_scale"])


def test_quantizer_overflow_raises():
    w = np.zeros((1, 64), dtype=np.float32)
    w[0, 0] = 100.0  # scale 100/7*2^14 > 65535
    with pytest.raises(ValueError):
        R.quantize_weight_q4(w)


def test_lm_head_kat(kat):
    g = kat.group("lm_head_argmax_stage_real")
    tok, score, logits = R.lm_head_argmax(g["activation"], g["packed"], g["scale"], want_logits=True)
    assert np.array_equal(logits, g["expected_logits_q26"])
    assert (tok, score) == (264, 1365150750)


def test_lm_head_ties_lowest_index():
    rng = np.random.default_rng(3)
    rows = 5000
    packed = np.zeros((rows, 512), dtype=np.uint8)
    scale = np.zeros((rows, 16), dtype=np.uint16)
    row = rng.integers(0, 256, 512).astype(np.uint8)
    sc = rng.integers(1, 100, 16).astype(np.uint16)
    for r in (17, 1234, 4999):  # identical best rows: the lowest index must win
        packed[r], scale[r] = row, sc
    act = rng.integers(-5000, 5000, 1024)
    tok, score = R.lm_head_argmax(act, packed, scale)
    logits = O.gemv_q26_packed(act, packed, scale)
    assert tok == int(np.argmax(logits)) and score == int(logits.max())
    assert tok == 17 or logits[17] < logits.max()


@pytest.mark.parametrize("name", ["rmsnorm_1024_real", "final_rmsnorm_stage_real",
                                  "final_rmsnorm_layer2_chained_stage_real",
                                  "layer1_chained_input_rmsnorm_stage_real"])
def test_rmsnorm_kat(kat, name):
    g = kat.group(name)
    r = R.fixed_rmsnorm_reference(g["input"], g["gamma"])
    assert np.array_equal(r["output_q12_12"], g["expected"])
    assert r["sum_squares"] == int(g["sum_squares"][0]) and r["inv_rms_uq8_16"] == int(g["inv_rms"][0])
    assert r["rms_q14_10"] == int(g["rms"][0])


@pytest.mark.parametrize("i", range(4))
def test_rmsnorm_edges(refh, i):
    r = R.fixed_rmsnorm_reference(refh[f"rms{i}_x"], refh[f"rms{i}_g"])
    assert np.array_equal(r["output_q12_12"], refh[f"rms{i}_out"])
    assert r["inv_rms_uq8_16"] == int(refh[f"rms{i}_inv"]) and r["saturation"] == bool(refh[f"rms{i}_sat"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_qk_norm_rope_kat(kat, pre):
    g = kat.group(f"{pre}qk_norm_rope_stage_128_real")
    qn, _, _ = R.fixed_rmsnorm_heads(g["q_input"].reshape(16, 128), g["q_gamma"])
    kn, _, _ = R.fixed_rmsnorm_heads(g["k_input"].reshape(8, 128), g["k_gamma"])
    assert np.array_equal(qn.reshape(-1), g["q_norm_expected"])
    assert np.array_equal(kn.reshape(-1), g["k_norm_expected"])
    qr, _ = R.fixed_rope_reference(qn, g["cos"], g["sin"])
    kr, _ = R.fixed_rope_reference(kn, g["cos"], g["sin"])
    assert np.array_equal(qr.reshape(-1), g["q_rope_expected"])
    assert np.array_equal(kr.reshape(-1), g["k_rope_expected"])


def test_heads_norm_rope_edges(refh):
    out, _, sat = R.fixed_rmsnorm_heads(refh["heads_x"], refh["heads_g"])
    assert np.array_equal(out, refh["heads_out"]) and sat == bool(refh["heads_sat"])
    for j in range(4):
        pi = int(refh[f"rope{j}_pos_index"])
        ro, rsat = R.fixed_rope_reference(refh["rope_x"], refh["rope_cos"][pi], refh["rope_sin"][pi])
        assert np.array_equal(ro, refh[f"rope{j}_out"]) and rsat == bool(refh[f"rope{j}_sat"])


@pytest.mark.parametrize("pre", PREFIXES)
def test_attention_kats(kat, pre):
    g = kat.group(f"{pre}attention_score_stage_real")
    ctx = int(g["cache_length"][0])
    a = R.attention_score_value(q_current=g["q_input"].reshape(16, 128), k_cache=g["k_cache"].reshape(ctx, 8, 128),
                                v_cache=np.zeros((ctx, 8, 128)), exp_lut=O.build_exp_lut())
    order = (g["expected_q_head"], g["expected_position"])
    assert np.array_equal(a["raw"][order], g["expected_raw"])
    assert np.array_equal(a["scaled"][order], g["expected_scaled"])
    g = kat.group(f"{pre}attention_softmax_value_stage_real")
    scores = np.zeros((16, ctx), dtype=np.int64)
    scores[g["score_q_head"], g["score_position"]] = g["score_input"]
    probs, idx = R.fixed_softmax_probs(scores, g["exp_lut"])
    order = (g["score_q_head"], g["score_position"])
    assert np.array_equal(probs[order], g["expected_prob"]) and np.array_equal(idx[order], g["expected_lut_index"])
    out, _ = R.fixed_value_accum(probs, g["v_cache"].reshape(ctx, 8, 128))
    assert np.array_equal(out.reshape(-1), g["expected_out"])


@pytest.mark.parametrize("j", range(4))
def test_softmax_value_edges(refh, j):
    probs, idx = R.fixed_softmax_probs(refh[f"sm{j}_scores"], refh["exp_lut"])
    assert np.array_equal(probs, refh[f"sm{j}_probs"]) and np.array_equal(idx, refh[f"sm{j}_idx"])
    out, sat = R.fixed_value_accum(probs, refh[f"sm{j}_v"])
    assert np.array_equal(out, refh[f"sm{j}_out"]) and sat == bool(refh[f"sm{j}_sat"])


def test_attention_whole(refh):
    a = R.attention_score_value(q_current=refh["att_q"], k_cache=refh["att_k"], v_cache=refh["att_v"],
                                exp_lut=refh["exp_lut"])
    for f in ("raw", "scaled", "probs", "lut_indices", "output"):
        assert np.array_equal(a[f], refh[f"att_{f}"]), f


@pytest.mark.parametrize("pre", PREFIXES)
def test_silu_and_residual_kats(kat, pre):
    g = kat.group(f"{pre}mlp_silu_mul_stage_real")
    r = R.silu_mul(g["gate_input"], g["up_input"], g["sigmoid_lut"])
    assert np.array_equal(r["lut_index"], g["expected_lut_index"])
    assert np.array_equal(r["silu"], g["expected_silu_gate_q12_12"])
    assert np.array_equal(r["hidden"], g["expected_hidden_q12_12"])
    g = kat.group(f"{pre}mlp_residual_add_stage_real")
    out, _ = R.residual_add(g["post_attn_hidden"], g["down_out"], 2)
    assert np.array_equal(out, g["expected_layer_out"])
    g = kat.group(f"{pre}post_attention_residual_norm_stage_real")
    post, _ = R.residual_add(g["residual_input"], g["o_proj_input"], 2)
    assert np.array_equal(post, g["expected_residual"])


def test_silu_sweep(refh):
    r = R.silu_mul(refh["silu_gate"], refh["silu_up"], refh["sigmoid_lut"])
    assert np.array_equal(r["lut_index"], refh["silu_idx"])
    assert np.array_equal(r["silu"], refh["silu_silu"]) and np.array_equal(r["hidden"], refh["silu_hidden"])


def test_embedding_rows():
    vocab = 2048
    w = O.synth_f32(5, O.TID_EMBED, (vocab, 1024), 0.02)
    q, s = O.quantize_weight_q4(w)
    toks = [0, 1, 77, 2047]
    got = R.embedding_hidden(toks, O.pack_int4(q), s)
    for i, t in enumerate(toks):
        assert np.array_equal(got[i], O.embedding_hidden(q[t], s[t]))


@pytest.mark.parametrize("k,rows,count,shared", [(1024, 3072, 4, False), (2048, 100, 5, True), (3072, 37, 3, False),
                                                 (4096, 9, 2, True)])
def test_gemv_strided_many(k, rows, count, shared):
    """q4gpu_gemv_q26_strided: `count` GEMVs in one launch equal `count`
    separate oracle GEMVs (distinct or one shared activation)."""
    from llm_accelerator_b200 import _native
    lib = _native.load()
    rng = np.random.default_rng(k * 7 + rows)
    q = rng.integers(-8, 8, (count, rows, k)).astype(np.int8)
    s = rng.integers(0, 1 << 16, (count, rows, k // 64)).astype(np.uint16)
    a = rng.integers(-(1 << 23), 1 << 23, (1 if shared else count, k)).astype(np.int32)
    packed = np.stack([O.pack_int4(q[i]) for i in range(count)])
    dev = torch.device("cuda")
    ta = torch.from_numpy(a).to(dev)
    tw = torch.from_numpy(packed).to(dev)
    ts = torch.from_numpy(s.view(np.int16)).to(dev)
    out = torch.zeros((count, rows), dtype=torch.int64, device=dev)
    o12 = torch.zeros((count, rows), dtype=torch.int32, device=dev)
    sat = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.q4gpu_gemv_q26_strided(ta.data_ptr(), 0 if shared else k, k, tw.data_ptr(), rows * k // 2, ts.data_ptr(),
                                    rows * k // 64, rows, count, out.data_ptr(), o12.data_ptr(), rows, sat.data_ptr(),
                                    None)
    assert rc == 0, lib.q4gpu_last_error()
    torch.cuda.synchronize()
    n_sat = 0
    for i in range(count):
        ref = O.gemv_q26(a[0 if shared else i].astype(np.int64), q[i], s[i])
        assert np.array_equal(out[i].cpu().numpy(), ref), i
        r12, ns = O.q26_to_q12_12(ref)
        assert np.array_equal(o12[i].cpu().numpy().astype(np.int64), r12), i
        n_sat += ns
    assert int(sat.item()) == n_sat
