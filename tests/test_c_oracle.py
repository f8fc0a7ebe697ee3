"""The C restatement of the oracle agrees with the numpy oracle and with the
reference's whole-model golden (CPU only)."""
import numpy as np
import pytest

from oracle import c_oracle as CO
from oracle import q4_oracle as O


def test_synth_and_quantiser_match_numpy():
    w = CO.synth_f32(3, 77, 64 * 1024, 0.02).reshape(64, 1024)
    assert np.array_equal(w, O.synth_f32(3, 77, (64, 1024), 0.02))
    w[0] = 0
    w[1] = 1e-6
    q, s = CO.quantize_q4(w)
    oq, os_ = O.quantize_weight_q4(w)
    assert np.array_equal(q, oq) and np.array_equal(s, os_)


def test_gemv_matches_numpy(refh):
    for tag in ("k1024", "k2048", "k3072"):
        p = refh[f"xgemv_{tag}_packed"]
        q = O.unpack_int4(p, p.shape[1] * 2)
        assert np.array_equal(CO.gemv_q26(refh[f"xgemv_{tag}_act"], q, refh[f"xgemv_{tag}_scale"]),
                              refh[f"xgemv_{tag}_q26"])


def test_small_model_decode_matches_numpy():
    seed, L, vocab, ctx = 13, 2, 4096, 64
    cm = CO.CModel(L, vocab, ctx, seed=seed, gamma_std=0.05)
    om = O.Model(layers=[O.synth_layer(seed, li, gamma_std=0.05) for li in range(L)], embed_q=None,
                 embed_s=None, final_gamma=None)
    om.embed_q, om.embed_s = O.quantize_weight_q4(O.synth_f32(seed, O.TID_EMBED, (vocab, 1024), 0.02))
    om.final_gamma = O.quantize_signed(np.ones(1024, np.float32) + O.synth_f32(seed, O.TID_FINAL_NORM, (1024,), 0.05),
                                       16, 7)[0]
    om.cos, om.sin = O.rope_tables(ctx)
    prompt = [1, 2, 4000, 77]
    assert cm.decode(prompt, 5) == O.greedy_decode(om, prompt, 5, max_ctx=ctx)
    cm.close()


def test_full_model_matches_reference_golden(refmodel):
    cm = CO.CModel(28, 151936, 16, seed=0)
    toks = refmodel["tokens"].tolist()
    for pos, t in enumerate(toks):
        assert cm.run_token(t, pos) == (int(refmodel["argmax"][pos]), int(refmodel["scores"][pos])), pos
    assert np.array_equal(cm.hidden(), refmodel["final_hidden"][-1])
    cm.close()
    cm = CO.CModel(28, 151936, 16, seed=0)
    gen, scores = cm.decode(refmodel["prompt"].tolist(), len(refmodel["generated"]))
    assert gen == refmodel["generated"].tolist() and scores == refmodel["generated_scores"].tolist()
    cm.close()
