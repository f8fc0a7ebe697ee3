"""Small, fixed GPU cases for profiling the kernels under ncu.

    python -m llm_accelerator_b200.profile_cases batch --seqs 64 --position 383 --steps 2
    python -m llm_accelerator_b200.profile_cases gemv --rows 151936 --k 1024 --reps 3
    python -m llm_accelerator_b200.profile_cases lmhead --rows 151936 --reps 3

`batch`: the 151936-vocabulary synthetic model (seed 0; 28 layers, or `--layers`
for a smaller capture: the per-layer launches do not depend on the layer count),
`seqs` sequences set to `position` and advanced `steps` batched decode steps
(4 + 7 L kernel launches per step: embed, L x [norm, qkv GEMM, attention,
o_proj GEMM, norm, gate/up GEMM, down GEMM], norm, LM-head GEMM, argmax).
`gemv` / `lmhead`: `reps` calls of q4gpu_gemv_q26 / q4gpu_lm_head_argmax on a
random packed matrix (a few hundred MB of device memory at most).
"""
from __future__ import annotations

import argparse


def batch_case(seqs: int, position: int, steps: int, max_context: int, layers: int = 28) -> None:
    from .model import Q4Model

    with Q4Model(n_layers=layers, vocab=151936, max_context=max_context, max_seqs=seqs) as m:
        m.init_synthetic(seed=0)
        m.batch_set_position(position, seqs, lm_from=0)
        m.batch_steps(steps, seqs)
        m.sync()


def gemv_case(rows: int, k: int, reps: int, lm_head: bool) -> None:
    import torch

    from . import _native

    lib = _native.load()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    act = torch.randint(-(1 << 23), 1 << 23, (k,), dtype=torch.int32, device=dev, generator=g)
    w = torch.randint(0, 256, (rows, k // 2), dtype=torch.uint8, device=dev, generator=g)
    s = torch.randint(0, 20000, (rows, k // 64), dtype=torch.int16, device=dev, generator=g)
    out = torch.empty(rows, dtype=torch.int64, device=dev)
    if lm_head:
        ws_bytes = lib.q4gpu_lm_head_workspace_bytes(rows)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        tok = torch.empty(1, dtype=torch.int32, device=dev)
        score = torch.empty(1, dtype=torch.int64, device=dev)
    for _ in range(reps):
        if lm_head:
            rc = lib.q4gpu_lm_head_argmax(act.data_ptr(), w.data_ptr(), s.data_ptr(), rows, None, ws.data_ptr(),
                                          ws_bytes, tok.data_ptr(), score.data_ptr(), None)
        else:
            rc = lib.q4gpu_gemv_q26(act.data_ptr(), k, w.data_ptr(), s.data_ptr(), rows, out.data_ptr(), None, None,
                                    None)
        _native.check(rc, "profile case")
    torch.cuda.synchronize()


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    b = sub.add_parser("batch")
    b.add_argument("--seqs", type=int, default=64)
    b.add_argument("--position", type=int, default=383)
    b.add_argument("--steps", type=int, default=2)
    b.add_argument("--max-context", type=int, default=512)
    b.add_argument("--layers", type=int, default=28)
    for name in ("gemv", "lmhead"):
        p = sub.add_parser(name)
        p.add_argument("--rows", type=int, default=151936)
        p.add_argument("--k", type=int, default=1024)
        p.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    if a.case == "batch":
        batch_case(a.seqs, a.position, a.steps, a.max_context, a.layers)
    else:
        gemv_case(a.rows, a.k if a.case == "gemv" else 1024, a.reps, a.case == "lmhead")
    print("ok")


if __name__ == "__main__":
    main()
