"""The fused decode path (model context, paged KV, PDL-chained kernels in CUDA
graphs) vs the CPU oracle and vs the reference's own whole-model golden."""
import numpy as np
import pytest

from oracle import q4_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import _native  # noqa: E402
from llm_accelerator_b200.model import Q4Model, QotError  # noqa: E402


def oracle_small(seed, n_layers, vocab, max_ctx, gamma_std=0.0):
    m = O.Model(layers=[O.synth_layer(seed, li, gamma_std=gamma_std) for li in range(n_layers)],
                embed_q=None, embed_s=None, final_gamma=None)
    m.embed_q, m.embed_s = O.quantize_weight_q4(O.synth_f32(seed, O.TID_EMBED, (vocab, 1024), 0.02))
    fg = np.ones(1024, dtype=np.float32)
    if gamma_std > 0:
        fg = fg + O.synth_f32(seed, O.TID_FINAL_NORM, (1024,), gamma_std)
    m.final_gamma = O.quantize_signed(fg, 16, 7)[0]
    m.cos, m.sin = O.rope_tables(max_ctx)
    return m


@pytest.fixture(scope="module")
def small():
    seed, L, vocab, ctx = 11, 2, 8192, 128
    gm = Q4Model(n_layers=L, vocab=vocab, max_context=ctx, max_seqs=2)
    gm.init_synthetic(seed=seed, std=0.02, gamma_std=0.05)
    om = oracle_small(seed, L, vocab, ctx, gamma_std=0.05)
    yield gm, om
    gm.close()


def test_device_quantised_weights_match_oracle(small):
    gm, om = small
    for li, p in enumerate(om.layers):
        for which, (w, s) in {_native.T_Q: (p.q_w, p.q_s), _native.T_K: (p.k_w, p.k_s),
                              _native.T_O: (p.o_w, p.o_s), _native.T_DOWN: (p.down_w, p.down_s)}.items():
            gp, gs = gm.get_weight(li, which)
            assert np.array_equal(gp, O.pack_int4(w)) and np.array_equal(gs, s), (li, which)
        assert np.array_equal(gm.get_gamma(li, _native.T_INPUT_GAMMA), p.input_gamma)
        assert np.array_equal(gm.get_gamma(li, _native.T_Q_GAMMA), p.q_gamma)
    ep, es = gm.get_weight(0, _native.T_EMBED)
    assert np.array_equal(ep, O.pack_int4(om.embed_q)) and np.array_equal(es, om.embed_s)
    assert np.array_equal(gm.get_gamma(0, _native.T_FINAL_GAMMA), om.final_gamma)


def test_greedy_decode_matches_oracle(small):
    gm, om = small
    prompt = [3, 4096, 8191, 17, 5]
    toks, res = gm.decode(prompt, 6, slot=0)
    ref, scores = O.greedy_decode(om, prompt, 6, max_ctx=128)
    assert toks == ref
    assert res.token_id == ref[-1] and res.score_q26 == scores[-1]
    # retained K/V and the last hidden state, entry for entry
    st = O.DecodeState(2, 128)
    seq = prompt + ref[:-1]
    for pos, t in enumerate(seq):
        O.run_token(om, st, t, pos, want_logits=False)
    for li in range(2):
        assert np.array_equal(gm.read_kv(li, 0, len(seq), slot=0), st.k[li, :len(seq)])
        assert np.array_equal(gm.read_kv(li, 1, len(seq), slot=0), st.v[li, :len(seq)])


def test_runner_matches_oracle_per_position(small):
    gm, om = small
    seq = [100, 200, 300, 400]
    st = O.DecodeState(2, 128)
    for pos, t in enumerate(seq):
        r = gm.run_token(t, pos, slot=1)
        tok, score, h = O.run_token(om, st, t, pos)
        assert (r.token_id, r.score_q26) == (tok, score)
        assert np.array_equal(gm.read_hidden(slot=1), h)
        assert r.raw.layers_completed == 2 and r.raw.status == 1


def test_runner_error_codes(small):
    gm, _ = small
    with pytest.raises(QotError) as e:
        gm.run_token(8192, 0)  # vocab is 8192
    assert e.value.code == _native.QOT_ERR_BAD_TOKEN
    with pytest.raises(QotError) as e:
        gm.run_token(1, 128)
    assert e.value.code == _native.QOT_ERR_CONTEXT
    with pytest.raises(QotError) as e:
        gm.run_token(1, 0, layer_start=2, layer_count=1)
    assert e.value.code == _native.QOT_ERR_BAD_LAYER
    with pytest.raises(QotError) as e:
        gm.run_token(1, 0, slot=2)
    assert e.value.code == _native.QOT_ERR_BAD_ADDR
    with pytest.raises(QotError) as e:
        gm.decode([1, 2], 200)  # 201 runs > max_context 128
    assert e.value.code == _native.QOT_ERR_CONTEXT
    with pytest.raises(QotError) as e:
        gm.decode([1, 9000], 2)  # validated before any launch
    assert e.value.code == _native.QOT_ERR_BAD_TOKEN


def test_runner_timeout_then_busy(small):
    gm, _ = small
    timed_out = False
    try:
        gm.run_token(5, 0, slot=0, max_polls=1)
    except QotError as e:
        assert e.code == _native.QOT_ERR_TIMEOUT
        timed_out = True
    if timed_out:
        codes = set()
        for _ in range(100000):
            try:
                gm.run_token(5, 0, slot=0, max_polls=0)
                break
            except QotError as e:
                codes.add(e.code)
                assert e.code == _native.QOT_ERR_BUSY
        assert codes <= {_native.QOT_ERR_BUSY}


@pytest.mark.parametrize("ctx,pos", [(520, 512), (4104, 4100), (70, 33)])
def test_single_layer_long_context_matches_oracle(ctx, pos):
    """One layer at `pos` over a pre-filled context (512: the cfg-2 shape; 4100:
    every rank of the per-stage cluster attention holds several 32-key chunks;
    33: most ranks hold no key): K/V of positions 0..pos-1 are N(0,1) bf16
    values in Q12.12."""
    seed = 21
    gm = Q4Model(n_layers=1, vocab=256, max_context=ctx, max_seqs=1)
    try:
        gm.init_synthetic(seed=seed)
        gm.mode = 0  # the per-stage kernels (the persistent kernel covers only short contexts)
        om = oracle_small(seed, 1, 256, ctx)
        kpre = O.quantize_signed(O.synth_f32(seed, 901, (pos, 8, 128), 1.0), 24, 12)[0]
        vpre = O.quantize_signed(O.synth_f32(seed, 902, (pos, 8, 128), 1.0), 24, 12)[0]
        hidden = O.quantize_signed(O.synth_f32(seed, 903, (1024,), 1.0), 24, 10)[0]
        gm.write_kv(0, 0, kpre)
        gm.write_kv(0, 1, vpre)
        gm.write_hidden(hidden)
        r = gm.run_token(0, pos, embedding=False)
        st = O.DecodeState(1, ctx)
        st.k[0, :pos], st.v[0, :pos] = kpre, vpre
        tr = {}
        out = O.layer_step(om.layers[0], hidden, pos, st.k[0], st.v[0], om.cos, om.sin, om.exp_lut,
                           om.sigmoid_lut, trace=tr)
        assert np.array_equal(gm.read_hidden(), out)
        assert np.array_equal(gm.read_kv(0, 0, pos + 1)[pos], tr["k_rope"])
        fn = O.rmsnorm(out, om.final_gamma)["output"]
        tok, score = O.lm_head_argmax(O.gemv_q26(fn, om.embed_q, om.embed_s))
        assert (r.token_id, r.score_q26) == (tok, score)
    finally:
        gm.close()


def test_time_layers_replays_the_layer_graphs():
    """q4gpu_model_time_layers runs the one-layer graph of the per-stage path at
    a reset position: after its warm-up and one timed replay the hidden state
    is the oracle's layer applied twice at that position (zero cache before)."""
    seed, ctx, pos = 21, 300, 270
    with Q4Model(n_layers=1, vocab=256, max_context=ctx, max_seqs=1) as gm:
        gm.init_synthetic(seed=seed)
        gm.mode = 0
        om = oracle_small(seed, 1, 256, ctx)
        h = O.quantize_signed(O.synth_f32(seed, 903, (1024,), 1.0), 24, 10)[0]
        gm.write_hidden(h)
        assert gm.time_layers(0, 1, pos, reps=1) > 0
        st = O.DecodeState(1, ctx)
        x = h
        for _ in range(2):
            x = O.layer_step(om.layers[0], x, pos, st.k[0], st.v[0], om.cos, om.sin, om.exp_lut, om.sigmoid_lut)
        assert np.array_equal(gm.read_hidden(), x)


def test_full_model_matches_reference_golden(refmodel):
    """The 28-layer, 151936-vocabulary seed-0 model: every per-position argmax
    and score of the reference's own chained fixed-point functions, then the
    same ids from the greedy decode API."""
    tokens = refmodel["tokens"].tolist()
    prompt = refmodel["prompt"].tolist()
    with Q4Model(n_layers=28, vocab=151936, max_context=256, max_seqs=2) as gm:
        gm.init_synthetic(seed=0)
        c, s = O.rope_tables(256)
        assert np.array_equal(c[: len(tokens)], refmodel["cos"]) and np.array_equal(s[: len(tokens)], refmodel["sin"])
        for pos, t in enumerate(tokens):
            r = gm.run_token(t, pos, slot=0)
            assert r.token_id == int(refmodel["argmax"][pos]), pos
            assert r.score_q26 == int(refmodel["scores"][pos]), pos
        assert np.array_equal(gm.read_hidden(slot=0), refmodel["final_hidden"][-1])
        gen, res = gm.decode(prompt, len(refmodel["generated"]), slot=1)
        assert gen == refmodel["generated"].tolist()
        assert res.score_q26 == int(refmodel["generated_scores"][-1])


def test_device_decode_loop_matches_oracle(small):
    """decode_steps / set_position / read_tokens / time_kernels: the
    device-resident greedy loop used by bench.py, cycled back to a position."""
    gm, om = small
    prompt = [9, 8, 7]
    gen, _ = gm.decode(prompt, 1, slot=0)
    gm.decode_steps(5, slot=0)
    toks, scores, pos = gm.read_tokens(3, 6, slot=0)
    ref, ref_scores = O.greedy_decode(om, prompt, 6, max_ctx=128)
    assert toks.tolist() == ref and scores.tolist() == ref_scores and pos == 8
    gm.set_position(3, slot=0)  # replay the same five steps: identical tokens
    gm.decode_steps(5, slot=0)
    toks2, _, pos2 = gm.read_tokens(3, 6, slot=0)
    assert toks2.tolist() == ref and pos2 == 8
    gm.set_position(3, slot=0)
    kt = gm.time_kernels(reps=2, slot=0)
    assert kt["qkv_norm_rope_kv"][1] == 2 and kt["final_norm_lm_head_argmax"][1] == 1
    assert all(v[0] > 0 for v in kt.values())
    toks3, _, _ = gm.read_tokens(3, 3, slot=0)
    assert toks3.tolist() == ref[:3]


def test_persistent_and_graph_modes_agree(small):
    """Mode 1 (persistent cooperative kernel, the default) and mode 0
    (per-stage kernels in CUDA graphs) give the oracle's tokens and scores."""
    gm, om = small
    assert gm.mode == 1, "persistent kernel should be available for this shape"
    prompt = [11, 2222, 3333, 44, 5555, 6]
    ref, ref_scores = O.greedy_decode(om, prompt, 9, max_ctx=128)
    for mode in (1, 0, 1):
        gm.mode = mode
        toks, res = gm.decode(prompt, 9, slot=1)
        assert toks == ref, mode
        assert res.score_q26 == ref_scores[-1]
        _, scores, pos = gm.read_tokens(len(prompt), 9, slot=1)
        assert scores.tolist() == ref_scores and pos == len(prompt) + 8
    gm.mode = 1


def test_stepping_past_max_context_is_refused(small):
    gm, om = small
    prompt = [1, 2, 3]
    gm.decode(prompt, 1, slot=0)
    gm.set_position(126, slot=0)
    for mode in (1, 0):
        gm.mode = mode
        gm.set_position(126, slot=0)
        gm.decode_steps(4, slot=0)  # 126, 127 are valid; 128 and 129 are not
        if mode == 1:
            with pytest.raises(_native.Q4GpuError):
                gm.sync()
        else:
            gm.sync()
        _, _, pos = gm.read_tokens(0, 0, slot=0)
        assert pos == 128
    gm.mode = 1
    # the context is still usable afterwards
    toks, _ = gm.decode([5, 6], 3, slot=0)
    assert toks == O.greedy_decode(om, [5, 6], 3, max_ctx=128)[0]
