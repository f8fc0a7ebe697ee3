"""Sampled exact parity of a long-context decode against the C oracle.

TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's parity fields, never
by the product package.

A serial oracle run over an 8192-token prompt costs minutes, so the check is
inductive instead: the GPU's whole K/V cache of one sequence is loaded into
the C oracle (``CModel.set_kv``), and single positions are re-run there
teacher-forced (``orc_run_token`` follows the reference's per-position layer
step, ``Qwen3-0.6B-Base/python_each_module/56_export_persistent_multitoken_layer_golden.py:465-565``).
At every sampled position p the oracle reads only cache rows < p, so it
checks that the GPU computed position p's K and V rows in every layer, and,
from the last prompt position on, its argmax token and Q26 score, exactly
from the rows before it.  Positions at prefill block, query-tile and
KV-page boundaries are the ones worth sampling.
"""
from __future__ import annotations

import numpy as np

from .c_oracle import CModel


def load_cache(cm: CModel, model, slot: int, n_positions: int) -> None:
    """Copy slot's K/V rows [0, n_positions) of every layer from the GPU model into the oracle."""
    for layer in range(model.n_layers):
        for kind in (0, 1):
            cm.set_kv(layer, kind, 0, model.read_kv(layer, kind, n_positions, slot=slot, raw=True))


def sampled_parity(cm: CModel, model, slot: int, positions, n_cached: int, logits_from: int) -> list[str]:
    """Re-run `positions` (ascending, each < n_cached) in the oracle on top of the
    GPU's cache of `slot`; return the mismatches (empty when exact).

    The input token at p is the GPU's token ring entry p; where p >= logits_from
    the oracle's (token, score) must equal the ring's entry p + 1."""
    toks, scores, _ = model.read_tokens(0, n_cached + 1, slot=slot)
    load_cache(cm, model, slot, n_cached)
    bad = []
    for p in sorted(positions):
        if p < 0 or p >= n_cached:
            raise ValueError(f"position {p} outside the cached range [0, {n_cached})")
        gpu_kv = [(cm.get_kv(layer, 0, p, 1), cm.get_kv(layer, 1, p, 1)) for layer in range(model.n_layers)]
        want_logits = p >= logits_from
        tok, score = cm.run_token(int(toks[p]), p, want_logits=want_logits)
        for layer, (k, v) in enumerate(gpu_kv):
            if not np.array_equal(k, cm.get_kv(layer, 0, p, 1)):
                bad.append(f"K row of position {p}, layer {layer}")
            if not np.array_equal(v, cm.get_kv(layer, 1, p, 1)):
                bad.append(f"V row of position {p}, layer {layer}")
        if want_logits and (tok, score) != (int(toks[p + 1]), int(scores[p + 1])):
            bad.append(f"position {p}: gpu ({int(toks[p + 1])}, {int(scores[p + 1])}) oracle ({tok}, {score})")
    return bad
