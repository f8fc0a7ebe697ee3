"""Host-side partitioning for multi-GPU runs (one process per GPU).

Independent sequences shard with no data-path collective: every rank owns a
contiguous block of sequences and a full weight replica.  The vocabulary of
the tied LM head can be split across ranks instead; the greedy argmax then
needs one exchange of each rank's (score, index) winner per sequence, reduced
with the reference's rule (highest score, lowest index on ties,
`Qwen3-0.6B-Base/python_each_module/56_…:773-798`), which is exact because the
winner does not depend on the order the shards are visited.
"""
from __future__ import annotations

import numpy as np

# rows of the LM head a shard boundary is aligned to (one 16-row tile of the reference's scan)
LM_TILE = 16


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) share of n items for `rank` of `world` (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def vocab_shard(vocab: int, world: int, rank: int, tile: int = LM_TILE) -> tuple[int, int]:
    """LM-head rows [start, end) of `rank`, boundaries on `tile`-row tiles."""
    tiles = -(-vocab // tile)
    t0, t1 = shard_range(tiles, world, rank)
    return min(t0 * tile, vocab), min(t1 * tile, vocab)


def rank_prompts(rank: int, n_seq: int, prompt_len: int, vocab: int, seed_stride: int = 1000) -> list[list[int]]:
    """Prompts of one rank's sequences: uniform ids, seed seed_stride * rank + i."""
    return [np.random.default_rng(seed_stride * rank + i).integers(0, vocab, prompt_len).tolist()
            for i in range(n_seq)]


def combine_argmax(scores: np.ndarray, indices: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Reduce per-shard winners [shards, seqs] to the global (score, index) per
    sequence: highest score, lowest global index among equal scores."""
    scores = np.asarray(scores, dtype=np.int64)
    indices = np.asarray(indices, dtype=np.int64)
    best_s = scores[0].copy()
    best_i = indices[0].copy()
    for k in range(1, scores.shape[0]):
        take = (scores[k] > best_s) | ((scores[k] == best_s) & (indices[k] < best_i))
        best_s = np.where(take, scores[k], best_s)
        best_i = np.where(take, indices[k], best_i)
    return best_s, best_i


def exchange_argmax(score, index, group=None):
    """All ranks' (score, index) per sequence via one all_gather, reduced with
    `combine_argmax`.  `score`/`index`: int64 tensors [seqs] on this rank's
    device (CUDA with NCCL, CPU with gloo).  Returns numpy arrays."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    packed = torch.stack([score.to(torch.int64), index.to(torch.int64)])  # [2, seqs]
    parts = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(parts, packed, group=group)
    allp = torch.stack(parts).cpu().numpy()  # [world, 2, seqs]
    return combine_argmax(allp[:, 0, :], allp[:, 1, :])


def max_over_ranks(x: float, device=None, group=None) -> float:
    """The maximum of a per-rank float over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return float(x)
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
