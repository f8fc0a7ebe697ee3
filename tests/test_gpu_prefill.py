"""Batched exact prefill (q4gpu_batch_prefill): prompt positions as columns of
batched passes.  The K/V cache it leaves, and every token and Q26 score
decoded after it, equal the serial position-by-position path bit for bit and
the CPU oracle's."""
import numpy as np
import pytest

from oracle.c_oracle import CModel

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import _native  # noqa: E402
from llm_accelerator_b200.model import Q4Model  # noqa: E402

SEED, L, VOCAB, CTX, GAMMA = 23, 2, 8192, 1280, 0.05


@pytest.fixture(scope="module")
def gm():
    m = Q4Model(n_layers=L, vocab=VOCAB, max_context=CTX, max_seqs=16)
    m.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
    yield m
    m.close()


def _kv(m, n_seq, lens):
    return [[m.read_kv(layer, kind, lens[i], slot=i) for layer in range(L) for kind in (0, 1)] for i in range(n_seq)]


def _run(m, prompts, n_gen, mode):
    m.prefill_mode = mode
    gen, scores = m.decode_batch(prompts, n_gen)
    return gen, scores, _kv(m, len(prompts), [len(p) + n_gen - 1 for p in prompts])


def test_prefill_matches_serial_across_blocks_and_tiles(gm):
    """Ragged prompts (1 .. 700 tokens): 1227 prefill columns over two
    1024-column blocks (the 700-token prompt straddles the edge), query tiles
    cut at 64 positions, at sequence changes and at block edges; tokens, scores and the whole K/V cache of both layers equal
    the serial path's."""
    rng = np.random.default_rng(5)
    lens = [1, 2, 31, 32, 33, 64, 65, 300, 700, 9]
    prompts = [rng.integers(0, VOCAB, n).tolist() for n in lens]
    prompts[3][0], prompts[4][-1] = 0, VOCAB - 1
    g1, s1, kv1 = _run(gm, prompts, 6, 1)
    g0, s0, kv0 = _run(gm, prompts, 6, 0)
    gm.prefill_mode = 1
    assert g1.tolist() == g0.tolist()
    assert s1.tolist() == s0.tolist()
    for i in range(len(prompts)):
        for a, b in zip(kv1[i], kv0[i]):
            assert np.array_equal(a, b), i


def test_prefill_matches_c_oracle():
    """A 150-token prompt and two short ones against the C restatement of the
    reference's Python path (tokens and Q26 scores)."""
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, VOCAB, 150).tolist(), [7], rng.integers(0, VOCAB, 40).tolist()]
    with Q4Model(n_layers=L, vocab=VOCAB, max_context=256, max_seqs=3) as m:
        m.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
        gen, scores = m.decode_batch(prompts, 4)
    cm = CModel(L, VOCAB, 256, seed=SEED, std=0.02, gamma_std=GAMMA)
    try:
        for i, p in enumerate(prompts):
            ref, ref_scores = cm.decode(p, 4)
            assert gen[i].tolist() == ref and scores[i].tolist() == ref_scores, i
    finally:
        cm.close()


def test_prefill_api_then_device_steps(gm):
    """q4gpu_batch_prefill leaves slot i at position len - 1 with lm_from len;
    q4gpu_batch_steps then generates what q4gpu_decode_batch generates."""
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, VOCAB, n).tolist() for n in (17, 3, 96, 1)]
    gm.prefill_mode = 1
    ref, ref_scores = gm.decode_batch(prompts, 5)
    gm.batch_prefill(prompts)
    gm.sync()
    for i, p in enumerate(prompts):
        toks, _, pos = gm.read_tokens(0, len(p), slot=i)
        assert pos == len(p) - 1 and toks.tolist() == p
    gm.batch_steps(5, len(prompts))
    gm.sync()
    for i, p in enumerate(prompts):
        toks, scores, pos = gm.read_tokens(len(p), 5, slot=i)
        assert toks.tolist() == ref[i].tolist() and scores.tolist() == ref_scores[i].tolist()
        assert pos == len(p) + 4


def test_prefill_errors(gm):
    for prompts in ([[1, 2], []], [[1, VOCAB]], [[1] * (CTX + 1)]):
        with pytest.raises(_native.Q4GpuError):
            gm.batch_prefill(prompts)
    with pytest.raises(_native.Q4GpuError):
        gm.batch_prefill([[1]] * 4, first_slot=14)
    with pytest.raises(_native.Q4GpuError):
        gm.prefill_mode = 2


def test_prefill_sharp_attention_matches_serial():
    """q/k head-norm gammas of 8.0 make most attention rows put their whole
    probability (2^16) on one key, so the chunks that need the probabilities'
    third limb (p >> 16) run their extra products; the K/V cache, tokens and
    scores still equal the serial path's."""
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, VOCAB, n).tolist() for n in (130, 65, 3)]
    with Q4Model(n_layers=L, vocab=VOCAB, max_context=256, max_seqs=3) as m:
        m.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
        for layer in range(L):
            for which in (_native.T_Q_GAMMA, _native.T_K_GAMMA):
                m.set_table(which, np.full(128, 8 * 128, dtype=np.int32), layer=layer)
        g1, s1, kv1 = _run(m, prompts, 4, 1)
        g0, s0, kv0 = _run(m, prompts, 4, 0)
    assert g1.tolist() == g0.tolist() and s1.tolist() == s0.tolist()
    for i in range(len(prompts)):
        for a, b in zip(kv1[i], kv0[i]):
            assert np.array_equal(a, b), i


def test_long_prompt_matches_c_oracle():
    """A 2050-token prompt (one layer): prefill query tiles over 33 KV pages and
    batched decode steps through the 16-CTA cluster attention (160 keys per
    rank, several chunks each) give the C oracle's tokens and scores."""
    L1, V1, ctx, n_gen = 1, 256, 2064, 3
    prompt = np.random.default_rng(17).integers(0, V1, 2050).tolist()
    with Q4Model(n_layers=L1, vocab=V1, max_context=ctx, max_seqs=1) as m:
        m.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
        gen, scores = m.decode_batch([prompt], n_gen)
    cm = CModel(L1, V1, ctx, seed=SEED, std=0.02, gamma_std=GAMMA)
    try:
        ref, ref_scores = cm.decode(prompt, n_gen)
    finally:
        cm.close()
    assert gen[0].tolist() == ref and scores[0].tolist() == ref_scores
