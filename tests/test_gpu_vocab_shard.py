"""Vocabulary-sharded LM head on one GPU: forward to the final norm, LM head
per shard (uneven shards, ties across shard edges), winners combined with the
reference's rule, tokens committed — identical ids and scores to the
unsharded batched decode and to the CPU oracle."""
import numpy as np
import pytest

from oracle.c_oracle import CModel

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import sharding as SH  # noqa: E402
from llm_accelerator_b200.model import Q4Model  # noqa: E402

SEED, L, VOCAB, CTX, GAMMA = 11, 2, 8192, 64, 0.05


def test_sharded_lm_head_matches_full_decode():
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, VOCAB, 4).tolist() for _ in range(5)]
    n_new = 5
    dev = torch.device("cuda")
    with Q4Model(n_layers=L, vocab=VOCAB, max_context=CTX, max_seqs=5) as gm:
        gm.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
        full, full_scores = gm.decode_batch(prompts, n_new)
        # prefill by the ordinary batched steps up to the last prompt position, then
        # every generated position through forward_hidden + shards + commit
        gm.decode_batch(prompts, 1)  # positions now 4, token 4 = first generated
        gm.batch_set_position(3, 5)  # replay the last prompt position through the shards
        acts = torch.empty((5, 1024), dtype=torch.int32, device=dev)
        shards = [(0, 3000), (3000, 5000), (5000, VOCAB)]
        stream = torch.cuda.ExternalStream(gm.stream)
        with torch.cuda.stream(stream):
            for _ in range(n_new):
                gm.batch_forward_hidden(5, acts)
                # shard winners as an all_gather lays them out: [shard][score | row][sequence]
                win = torch.empty((3, 2, 5), dtype=torch.int64, device=dev)
                for i, (a, b) in enumerate(shards):
                    gm.lm_head_shard(acts, a, b, win[i, 0], win[i, 1])
                host = SH.combine_argmax(win[:, 0].cpu().numpy(), win[:, 1].cpu().numpy())
                before = gm.read_tokens(0, CTX, slot=0)[2]
                gm.batch_commit_shards(win, 5, 0)
                gm.sync()
                for i in range(5):
                    t, sc, _ = gm.read_tokens(before + 1, 1, slot=i)
                    assert (int(t[0]), int(sc[0])) == (int(host[1][i]), int(host[0][i])), i
        gm.sync()
        for i in range(5):
            toks, scores, pos = gm.read_tokens(4, n_new, slot=i)
            assert toks.tolist() == full[i].tolist() and scores.tolist() == full_scores[i].tolist(), i
            assert pos == 3 + n_new
    cm = CModel(L, VOCAB, CTX, seed=SEED, std=0.02, gamma_std=GAMMA)
    for i, p in enumerate(prompts):
        assert full[i].tolist() == cm.decode(p, n_new)[0]
    cm.close()


def test_single_rank_decoder_equals_full_lm_head():
    rng = np.random.default_rng(22)
    prompts = [rng.integers(0, VOCAB, 3).tolist() for _ in range(4)]
    with Q4Model(n_layers=L, vocab=VOCAB, max_context=CTX, max_seqs=4) as gm:
        gm.init_synthetic(seed=SEED, std=0.02, gamma_std=GAMMA)
        full, _ = gm.decode_batch(prompts, 4)
        gm.decode_batch(prompts, 1)
        gm.batch_set_position(2, 4)
        dec = SH.VocabShardedDecoder(gm, 4)
        dec.step()  # eager
        gm.sync()
        captured = dec.capture()  # the same step as one CUDA graph (capture does not run it)
        for _ in range(3):
            dec.step()
        gm.sync()
        dec.release()
        for i in range(4):
            assert gm.read_tokens(3, 4, slot=i)[0].tolist() == full[i].tolist(), (i, captured)
        assert captured, "the sharded step should capture as a CUDA graph"


def test_lm_head_shard_rejects_bad_ranges():
    from llm_accelerator_b200 import _native
    with Q4Model(n_layers=1, vocab=1024, max_context=16, max_seqs=1) as gm:
        gm.init_synthetic(seed=1)
        acts = torch.zeros((1, 1024), dtype=torch.int32, device="cuda")
        s = torch.empty(1, dtype=torch.int64, device="cuda")
        for a, b in ((0, 0), (-1, 10), (10, 2000), (500, 400)):
            with pytest.raises(_native.Q4GpuError):
                gm.lm_head_shard(acts, a, b, s, s)
