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


class VocabShardedDecoder:
    """Greedy decode steps with the tied LM head split over the ranks of a
    process group (one GPU each).  Every rank decodes `n_local` sequences of
    its own (slots 0..n_local-1 of `model`); per step the ranks exchange the
    final normed vectors (all_gather), each scores its vocabulary shard for all
    of them, the (score, row) winners are exchanged (all_gather) and one kernel
    (q4gpu_batch_commit_shards) reduces them with the reference's rule and
    commits this rank's tokens.  The result equals an unsharded LM head bit for
    bit.  `capture()` records the whole step (the batched forward graph, both
    collectives, the shard GEMM and the commit) as one CUDA graph."""

    def __init__(self, model, n_local: int, group=None):
        import torch
        import torch.distributed as dist

        self.m, self.n, self.group = model, n_local, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.v0, self.v1 = vocab_shard(model.vocab, self.world, self.rank)
        dev = torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.ExternalStream(model.stream)
        cols = self.world * n_local
        self.acts = torch.empty((n_local, 1024), dtype=torch.int32, device=dev)
        self.all_acts = torch.empty((cols, 1024), dtype=torch.int32, device=dev)
        # this rank's shard winners for every sequence of every rank: scores
        # then rows, one contiguous [2, cols] block as the all_gather sends it
        self.mine = torch.empty((2, cols), dtype=torch.int64, device=dev)
        self.win = torch.empty((self.world, 2, cols), dtype=torch.int64, device=dev)
        self.graph = None

    def _enqueue(self) -> None:
        import torch.distributed as dist

        self.m.batch_forward_hidden(self.n, self.acts)
        if self.world > 1:
            dist.all_gather_into_tensor(self.all_acts, self.acts, group=self.group)
        else:
            self.all_acts.copy_(self.acts)
        self.m.lm_head_shard(self.all_acts, self.v0, self.v1, self.mine[0], self.mine[1])
        if self.world > 1:
            dist.all_gather_into_tensor(self.win, self.mine, group=self.group)
        else:
            self.win[0].copy_(self.mine)
        self.m.batch_commit_shards(self.win, self.n, self.rank * self.n)

    def step(self) -> None:
        """One decode position for this rank's sequences (asynchronous on the model stream)."""
        import torch

        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()  # replays on the current stream: the model's
            else:
                self._enqueue()

    def capture(self) -> bool:
        """Record one step as a CUDA graph; later steps replay it.  Run one eager
        step first (buffers, communicators, the forward graph).  Returns False,
        leaving the eager path, if this CUDA / NCCL build cannot capture it."""
        import torch

        from ._native import Q4GpuError

        g = torch.cuda.CUDAGraph()
        try:
            # relaxed: the library's host-side set-up calls (device selection,
            # tensor-map encoding) run during the capture without being captured
            with torch.cuda.graph(g, stream=self.stream, capture_error_mode="relaxed"):
                self._enqueue()
        except (RuntimeError, Q4GpuError):
            torch.cuda.synchronize()
            return False
        self.graph = g
        return True

    def release(self) -> None:
        """Drop the captured graph (before the process group is destroyed)."""
        self.graph = None
