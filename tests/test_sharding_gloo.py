"""Multi-rank host logic on CPU: two `gloo` ranks (127.0.0.1), no GPU.

Covers the sharding of sequences and of the LM-head vocabulary, the exact
(score, index) argmax exchange used by a vocab-sharded LM head, and the
max-over-ranks timing reduction bench.py applies."""
import os
import socket

import numpy as np
import pytest

from llm_accelerator_b200 import sharding as SH
from oracle import q4_oracle as O

torch = pytest.importorskip("torch")


def test_shard_ranges_cover_exactly():
    for n in (0, 1, 7, 64, 151936):
        for world in (1, 2, 3, 8):
            parts = [SH.shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        SH.shard_range(4, 2, 2)


def test_vocab_shards_on_tiles():
    for world in (1, 2, 4, 8):
        parts = [SH.vocab_shard(151936, world, r) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == 151936
        assert all(a % SH.LM_TILE == 0 for a, _ in parts)
    assert SH.vocab_shard(151936, 8, 3) == (3 * 18992, 4 * 18992)


def test_combine_argmax_matches_full_scan_with_ties():
    rng = np.random.default_rng(0)
    vocab, seqs = 1000, 5
    logits = rng.integers(-50, 50, (seqs, vocab)).astype(np.int64)
    logits[2, [10, 700]] = 10_000  # tie across shards: the lower index must win
    logits[4, [511, 512]] = 9_999  # tie at a shard boundary
    for world in (1, 2, 3, 4):
        sc, ix = [], []
        for r in range(world):
            a, b = SH.vocab_shard(vocab, world, r, tile=16)
            sub = logits[:, a:b]
            loc = np.array([O.lm_head_argmax(row)[0] if b > a else 0 for row in sub])
            sc.append(np.array([sub[s, loc[s]] if b > a else np.iinfo(np.int64).min for s in range(seqs)]))
            ix.append(loc + a)
        bs, bi = SH.combine_argmax(np.stack(sc), np.stack(ix))
        for s in range(seqs):
            t, score = O.lm_head_argmax(logits[s])
            assert (int(bi[s]), int(bs[s])) == (t, score), (world, s)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        vocab, seqs = 4096, 6
        rng = np.random.default_rng(42)
        logits = rng.integers(-(1 << 40), 1 << 40, (seqs, vocab)).astype(np.int64)
        logits[1, [5, 3000]] = 1 << 45  # tie across ranks
        a, b = SH.vocab_shard(vocab, world, rank)
        sub = logits[:, a:b]
        loc = np.array([O.lm_head_argmax(row)[0] for row in sub])
        score = torch.tensor([sub[s, loc[s]] for s in range(seqs)], dtype=torch.int64)
        index = torch.tensor(loc + a, dtype=torch.int64)
        bs, bi = SH.exchange_argmax(score, index)
        t_max = SH.max_over_ranks(1.0 + rank)
        prompts = SH.rank_prompts(rank, 3, 8, 151936)
        out.put((rank, bs.tolist(), bi.tolist(), t_max, prompts))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_exchange_argmax_and_timing():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    rng = np.random.default_rng(42)
    logits = rng.integers(-(1 << 40), 1 << 40, (6, 4096)).astype(np.int64)
    logits[1, [5, 3000]] = 1 << 45
    want = [O.lm_head_argmax(row) for row in logits]
    for rank, bs, bi, t_max, prompts in res:
        assert bi == [w[0] for w in want] and bs == [w[1] for w in want]
        assert bi[1] == 5
        assert t_max == 2.0
        assert prompts == SH.rank_prompts(rank, 3, 8, 151936)
    assert res[0][4] != res[1][4]  # ranks decode different sequences
