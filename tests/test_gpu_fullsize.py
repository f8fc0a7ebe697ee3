"""Full-size parity: the 28-layer, 151936-vocabulary model at BASELINE's
configurations 3 and 5, bit for bit against the C oracle.

Configuration 3 (batch 1, 128-token prompt, 128 greedy tokens on the
persistent kernel) is checked end to end: every generated token id and Q26
score equals a serial oracle decode of the same seeded model.

Configuration 5 (8192-token prompts through the batched exact prefill, then
batched decode steps on the cluster attention) is checked by sampled
teacher-forced positions on top of the GPU's own K/V cache
(oracle.long_context): every K and V row the GPU wrote at a sampled position,
in all 28 layers, and every token and score from the last prompt position on,
equal the oracle's.  The samples sit on the prefill's 1024-column block, 64-
position query-tile and 64-position KV-page boundaries.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200.model import Q4Model  # noqa: E402
from oracle.c_oracle import CModel  # noqa: E402
from oracle.long_context import sampled_parity  # noqa: E402

LAYERS, VOCAB = 28, 151936


def test_cfg3_full_model_greedy_matches_oracle():
    prompt = np.random.default_rng(0).integers(0, VOCAB, 128).tolist()
    with Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=256, max_seqs=1) as m:
        m.init_synthetic(seed=0)
        assert m.mode == 1, "configuration 3 runs on the persistent decode kernel"
        gen, res = m.decode(prompt, 128)
        toks, scores, _ = m.read_tokens(128, 128)
    cm = CModel(LAYERS, VOCAB, 256, seed=0)
    want, want_scores = cm.decode(prompt, 128)
    cm.close()
    assert gen == want
    assert toks.tolist() == want and scores.tolist() == want_scores
    assert res.token_id == want[-1] and res.score_q26 == want_scores[-1]


def test_cfg5_long_prompts_sampled_parity():
    n_seq, prompt_len, new = 8, 8192, 5
    prompts = [np.random.default_rng(50_000 + i).integers(0, VOCAB, prompt_len).tolist() for i in range(n_seq)]
    max_ctx = prompt_len + 8
    boundaries = [0, 1, 63, 64, 65, 1023, 1024, 1025, 2047, 2048, 4095, 4096, 4097, 6000, 8127, 8128, 8190]
    decode = list(range(prompt_len - 1, prompt_len - 1 + new))  # last prompt position, then the decode steps
    with Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=max_ctx, max_seqs=n_seq) as m:
        m.init_synthetic(seed=0)
        gen, scores = m.decode_batch(prompts, new)
        cm = CModel(LAYERS, VOCAB, max_ctx, seed=0)
        # sequence 0 starts on a block boundary, sequence 5 does not (its columns
        # begin at 5 * 8191)
        for slot in (0, 5):
            bad = sampled_parity(cm, m, slot, boundaries + decode, n_cached=prompt_len - 1 + new,
                                 logits_from=prompt_len - 1)
            assert not bad, f"sequence {slot}: {bad[:8]}"
            toks, sc, _ = m.read_tokens(prompt_len, new, slot=slot)
            assert toks.tolist() == gen[slot].tolist() and sc.tolist() == scores[slot].tolist()
        cm.close()
