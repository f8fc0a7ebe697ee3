"""Batched decode (up to 64 sequences per step on the tensor cores) vs the CPU
oracle, vs the single-sequence GPU path and vs the reference's own
whole-model golden.  Token ids and Q26 scores are compared bit for bit."""
import numpy as np
import pytest

from oracle import q4_oracle as O
from oracle.c_oracle import CModel

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import _native  # noqa: E402
from llm_accelerator_b200.model import Q4Model, QotError  # noqa: E402

SEED, L, VOCAB, CTX, GAMMA = 11, 2, 8192, 128, 0.05


@pytest.fixture(scope="module")
def pair():
    gm = Q4Model(n_layers=L, vocab=VOCAB, max_context=CTX, max_seqs=72)
    gm.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
    cm = CModel(L, VOCAB, CTX, seed=SEED, std=0.02, gamma_std=GAMMA)
    yield gm, cm
    cm.close()
    gm.close()


def _prompts(rng, n, lo=1, hi=12):
    return [rng.integers(0, VOCAB, int(rng.integers(lo, hi + 1))).tolist() for _ in range(n)]


@pytest.mark.parametrize("n_seq", [1, 5, 8, 13, 24, 31, 33, 64, 70])
def test_batch_decode_matches_oracle(pair, n_seq):
    """Every padded batch width (8, 16, 24, 32, 64) and a second group of 64,
    ragged prompt lengths, tokens drawn over the whole vocabulary."""
    gm, cm = pair
    rng = np.random.default_rng(1000 + n_seq)
    prompts = _prompts(rng, n_seq)
    prompts[0] = [VOCAB - 1] + prompts[0]  # edge ids
    prompts[-1] = [0] + prompts[-1]
    gen, scores = gm.decode_batch(prompts, 5)
    for i, p in enumerate(prompts):
        ref, ref_scores = cm.decode(p, 5)
        assert gen[i].tolist() == ref, (n_seq, i)
        assert scores[i].tolist() == ref_scores, (n_seq, i)


def test_batch_decode_matches_numpy_oracle_and_single_path(pair):
    gm, _ = pair
    om = O.Model(layers=[O.synth_layer(SEED, li, gamma_std=GAMMA) for li in range(L)], embed_q=None, embed_s=None,
                 final_gamma=None)
    om.embed_q, om.embed_s = O.quantize_weight_q4(O.synth_f32(SEED, O.TID_EMBED, (VOCAB, 1024), 0.02))
    om.final_gamma = O.quantize_signed(1.0 + O.synth_f32(SEED, O.TID_FINAL_NORM, (1024,), GAMMA), 16, 7)[0]
    om.cos, om.sin = O.rope_tables(CTX)
    prompts = [[3, 4096, 8191, 17, 5], [42], [7, 7, 7, 7, 7, 7, 7, 7, 7]]
    gen, scores = gm.decode_batch(prompts, 6)
    for i, p in enumerate(prompts):
        ref, ref_scores = O.greedy_decode(om, p, 6, max_ctx=CTX)
        assert gen[i].tolist() == ref and scores[i].tolist() == ref_scores
        single, res = gm.decode(p, 6, slot=70)
        assert single == ref and res.score_q26 == ref_scores[-1]


def test_batch_run_step_host_buffers(pair):
    """q4gpu_batch_run_step: per-position argmax and score for each sequence,
    positions differing across the batch."""
    gm, cm = pair
    rng = np.random.default_rng(7)
    n = 12
    seqs = [rng.integers(0, VOCAB, 10).tolist() for _ in range(n)]
    start = [int(x) for x in rng.integers(0, 4, n)]
    # sequence i starts at position start[i]: feed its prefix one position at a time first
    ref = []
    for i, s in enumerate(seqs):
        out = []
        for pos in range(start[i] + len(s)):
            tok = s[pos - start[i]] if pos >= start[i] else s[0]
            out.append(cm.run_token(tok, pos))
        ref.append(out)
    for i, s in enumerate(seqs):
        for pos in range(start[i]):
            t, sc = gm.batch_run_step([s[0]], [pos], first_slot=i)
            assert (int(t[0]), int(sc[0])) == ref[i][pos]
    for k in range(len(seqs[0])):
        toks = [s[k] for s in seqs]
        pos = [start[i] + k for i in range(n)]
        t, sc = gm.batch_run_step(toks, pos)
        for i in range(n):
            assert (int(t[i]), int(sc[i])) == ref[i][pos[i]], (i, k)


def test_batch_device_loop_and_set_position(pair):
    """q4gpu_batch_steps / q4gpu_batch_set_position: the device-resident loop
    bench.py times, replayed from a rewound position."""
    gm, cm = pair
    rng = np.random.default_rng(3)
    n = 20
    prompts = [rng.integers(0, VOCAB, 4).tolist() for _ in range(n)]
    gm.decode_batch(prompts, 2)  # prompts at 0..3, argmax at 4, 5; positions end at 5
    gm.batch_steps(6, n)  # positions 5..10 -> tokens 6..11
    gm.sync()
    refs = [cm.decode(p, 8) for p in prompts]
    for i in range(n):
        toks, scores, pos = gm.read_tokens(4, 8, slot=i)
        assert toks.tolist() == refs[i][0] and scores.tolist() == refs[i][1] and pos == 11
    gm.batch_set_position(5, n)
    gm.batch_steps(6, n)
    for i in range(n):
        toks, _, pos = gm.read_tokens(4, 8, slot=i)
        assert toks.tolist() == refs[i][0] and pos == 11


def test_batch_errors(pair):
    gm, _ = pair
    with pytest.raises(QotError) as e:
        gm.decode_batch([[1, 2], [VOCAB]], 2)
    assert e.value.code == _native.QOT_ERR_BAD_TOKEN
    with pytest.raises(QotError) as e:
        gm.decode_batch([[1] * 120], 10)
    assert e.value.code == _native.QOT_ERR_CONTEXT
    with pytest.raises(QotError) as e:
        gm.decode_batch([[1], []], 2)
    assert e.value.code == _native.QOT_ERR_CAPACITY
    for n in (0, 65):
        with pytest.raises(_native.Q4GpuError):
            gm.batch_steps(1, n)
    with pytest.raises(_native.Q4GpuError):
        gm.batch_steps(1, 8, first_slot=70)
    with pytest.raises(_native.Q4GpuError):
        gm.batch_run_step([1, VOCAB], [0, 0])
    with pytest.raises(_native.Q4GpuError):
        gm.batch_set_position(CTX, 4)


def test_batch_stops_at_max_context(pair):
    """A sequence that reaches max_context stops advancing; the others in the
    same batch are unaffected."""
    gm, cm = pair
    prompts = [[5, 6, 7], [8, 9, 10]]
    gm.decode_batch(prompts, 2)
    gm.batch_set_position(CTX - 2, 1, first_slot=0)  # slot 0 near the end
    gm.batch_steps(4, 2)
    gm.sync()
    _, _, p0 = gm.read_tokens(0, 0, slot=0)
    toks, _, p1 = gm.read_tokens(3, 6, slot=1)
    assert p0 == CTX and p1 == 8
    assert toks.tolist() == cm.decode(prompts[1], 6)[0]


def test_batch_full_model_matches_reference_golden(refmodel):
    """28 layers, vocabulary 151936, seed 0: three copies of the reference's
    prompt inside a batch of other prompts give the reference's generated ids
    and scores."""
    prompt = refmodel["prompt"].tolist()
    n_gen = len(refmodel["generated"])
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 151936, int(rng.integers(1, 9))).tolist() for _ in range(9)]
    for i in (0, 4, 8):
        prompts[i] = prompt
    with Q4Model(n_layers=28, vocab=151936, max_context=64, max_seqs=9) as gm:
        gm.init_synthetic(seed=0)
        gen, scores = gm.decode_batch(prompts, n_gen)
        for i in (0, 4, 8):
            assert gen[i].tolist() == refmodel["generated"].tolist(), i
            assert scores[i].tolist() == refmodel["generated_scores"].tolist(), i
        # the other sequences agree with the single-sequence path
        for i in (1, 5):
            single, res = gm.decode(prompts[i], n_gen, slot=i)
            assert gen[i].tolist() == single and scores[i][-1] == res.score_q26


def test_batch_gemm_wide_scales_take_two_passes():
    """Group scales of 256 and above: the batched GEMMs split each scale into
    4-bit digits and need a second pass over the weights for digits 2 and 3.
    Layer 0's matrices get scales x 3 (up to ~700: three digits), layer 1's
    down_proj x 300 and the LM head's first rows x 150 (four digits).  Batched
    decode must equal the numpy oracle with the same widened scales, and the
    single-sequence GEMV path."""
    seed, n_layers, vocab, ctx = 5, 2, 4096, 64
    om = O.Model(layers=[O.synth_layer(seed, li) for li in range(n_layers)], embed_q=None, embed_s=None,
                 final_gamma=O.quantize_signed(np.ones(1024), 16, 7)[0])
    om.embed_q, om.embed_s = O.quantize_weight_q4(O.synth_f32(seed, O.TID_EMBED, (vocab, 1024), 0.02))
    om.cos, om.sin = O.rope_tables(ctx)
    names = {_native.T_Q: "q", _native.T_K: "k", _native.T_V: "v", _native.T_O: "o", _native.T_GATE: "gate",
             _native.T_UP: "up", _native.T_DOWN: "down"}
    widen = [(0, w, 3) for w in names] + [(1, _native.T_DOWN, 300)]
    with Q4Model(n_layers=n_layers, vocab=vocab, max_context=ctx, max_seqs=8) as gm:
        gm.init_synthetic(seed=seed)
        for layer, which, f in widen:
            packed, scale = gm.get_weight(layer, which)
            wide = np.minimum(scale.astype(np.int64) * f, 65535).astype(np.uint16)
            gm.set_weight(layer, which, packed, wide)
            setattr(om.layers[layer], names[which] + "_s", wide)
        packed, scale = gm.get_weight(0, _native.T_EMBED)
        scale = scale.astype(np.int64)
        scale[:300] = np.minimum(scale[:300] * 150, 65535)
        gm.set_weight(0, _native.T_EMBED, packed, scale.astype(np.uint16))
        om.embed_s = scale.astype(np.uint16)
        assert om.layers[1].down_s.max() >= 4096 and om.layers[0].q_s.max() >= 256
        prompts = [[1, 2, 3], [4000, 17], [250, 251, 7, 9]]
        gen, scores = gm.decode_batch(prompts, 4)
        for i, p in enumerate(prompts):
            ref, ref_scores = O.greedy_decode(om, p, 4, max_ctx=ctx)
            assert gen[i].tolist() == ref and scores[i].tolist() == ref_scores, i
            single, res = gm.decode(p, 4, slot=7)
            assert single == ref and res.score_q26 == ref_scores[-1], i
