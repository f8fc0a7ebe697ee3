"""Decode benchmark: Qwen3-0.6B Q4 fixed-point greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: the 28-layer, 151936-vocabulary
Qwen3-0.6B with seeded synthetic Q4 weights (seed 0); 64 independent
sequences per GPU, each with its own 256-token prompt of uniform random ids,
greedy generation of 256 tokens, context up to 512.  The prompts are
prefilled as columns of batched passes (q4gpu_batch_prefill; the serial
position-by-position prefill, the reference's order, is timed beside it and
must give the same first tokens).  One timed step = one batched decode step: 64
tokens, one per sequence (embedding, 28 layers, final norm, LM head,
argmax), at decode positions in 256..510 (the generated half; a cycle replays
the same tokens).  The timed window of --steps steps is centred in that cycle,
so its mean context is the cycle's (384); the per-kernel roofline is taken at
the same mean context.  Per step the weights (317 MB of Q4) and the KV cache
of 64 sequences (~5.6 GB at context 384) stream from HBM: far larger than L2,
so no flush is needed.

Secondary (one GPU only): `batch1`: batch 1, prompt 128,
decode positions 128..255, on the persistent cooperative kernel; `cfg2` (one
decoder layer at batch 1, context 513); `gemv` (config 1); `cfg5` (config 5 on
one GPU: 8 x 8192-token prompts through the batched exact prefill, decode from
position 8192).  Each decode secondary carries a `parity` field from the C
oracle (config 3: every token and score of the timed run; config 5: sampled
positions re-run on top of the GPU's cache).  `--cfg5` runs config 5 alone,
on N GPUs with the vocabulary-sharded LM head.

N > 1 (torchrun, one rank per GPU): every rank decodes its own 64 sequences
(prompt seeds depend on the rank); no collective on the data path; value is
the total tokens/s over ranks with the max-over-ranks device time (weak
scaling).

`--impl reference` times the reference's arithmetic on the host CPU (the C
restatement of the reference's Python Q4 path, all host threads) on the
same workload, one sequence at a time as the reference runs; under torchrun
only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode tokens/sec (batch 64), Qwen3-0.6B Q4 greedy decode"
UNIT = "tokens/s"
VOCAB = 151936
LAYERS = 28
BATCH = 64
PROMPT = 256
GEN = 256
MAX_CTX = 512
CYCLE = GEN - 1  # decode steps of one generation: positions 256..510
WORKLOAD = ("cfg4: Qwen3-0.6B 28-layer Q4 (int4 + Q2.14 group scales) greedy decode, 64 sequences per GPU, "
            "prompt 256 uniform ids each, 256 generated tokens, context up to 512, timed window centred in decode "
            "positions 256..510")
B1_PROMPT, B1_CYCLE = 128, 128
CFG5_SEQS, CFG5_PROMPT, CFG5_GEN = 8, 8192, 512
HIDDEN, QKV_ROWS, INTER = 1024, 4096, 3072


# ---------------------------------------------------------------------------
# algorithmic bytes of one launch of each batched kernel (S sequences, the
# attention at context `ctx`): what the kernel must move at least
# ---------------------------------------------------------------------------
def batch_kernel_bytes(kind: str, S: int, ctx: int, planes: bool = False) -> int:
    """Algorithmic bytes of one launch: weights counted as Q4 (packed nibbles +
    u16 scales, the reference's storage), K/V at the reference's 4 B per element; with
    planes (the one-CTA-per-head attention of config 4) the cached keys and
    values are read as their three byte planes (3 B per element) and the new
    key and value rows are written both ways."""
    limbs = 3 * S  # limb rows of a B matrix (u8)

    def q4(rows: int, k: int) -> int:
        return rows * k // 2 + rows * k // 32

    if kind == "embed":
        return S * (512 + 32 + 4 * HIDDEN)
    if kind == "norm_limbs":
        return S * (4 * HIDDEN + limbs // S * HIDDEN) + 4 * HIDDEN
    if kind == "qkv_gemm":
        return q4(QKV_ROWS, HIDDEN) + limbs * HIDDEN + S * QKV_ROWS * 4
    if kind == "attention":
        elem_b = 3 if planes else 4
        kv_read = 8 * (ctx - 1) * 128 * 2 * elem_b
        new_rows = 8 * 128 * 2 * (4 + (3 if planes else 0))
        return S * (kv_read + new_rows + QKV_ROWS * 4 + 3 * 2 * HIDDEN)
    if kind == "o_proj_gemm":
        return q4(HIDDEN, 2 * HIDDEN) + limbs * 2 * HIDDEN + S * 3 * HIDDEN * 4
    if kind == "gate_up_gemm":
        return q4(2 * INTER, HIDDEN) + limbs * HIDDEN + limbs * INTER
    if kind == "down_gemm":
        return q4(HIDDEN, INTER) + limbs * INTER + S * 3 * HIDDEN * 4
    if kind == "lm_head_gemm":
        return q4(VOCAB, HIDDEN) + limbs * HIDDEN + (VOCAB + 127) // 128 * 64 * 16
    if kind == "argmax":
        return S * ((VOCAB + 127) // 128 * 16 + 16)
    return 0


def timed_window(steps: int) -> int:
    """First decode position of a timed window of `steps` steps: centred in the
    cycle 256..510 so that the window's mean context is the cycle's (384)."""
    return PROMPT if steps >= CYCLE else PROMPT + (CYCLE - steps) // 2


def window_positions(start: int, steps: int) -> list[int]:
    """Decode positions of `steps` steps from `start`, wrapping to 256 after 510."""
    out, p = [], start
    for _ in range(steps):
        if p >= PROMPT + CYCLE:
            p = PROMPT
        out.append(p)
        p += 1
    return out


def host_cpu() -> dict:
    """CPU model and logical core count of this host."""
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count()}


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        if kernel in d:
            return d[kernel]
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 50):
        self.gpu, self.period = gpu_index, period_ms
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.period)],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def prompts_for(rank: int) -> list[list[int]]:
    from llm_accelerator_b200.sharding import rank_prompts
    return rank_prompts(rank, BATCH, PROMPT, VOCAB)


# ---------------------------------------------------------------------------
# CPU arm: the C restatement of the reference path, one sequence at a time
# ---------------------------------------------------------------------------
def cpu_decode(n_steps: int, warmup: int, threads: int = 0, cm=None) -> dict:
    """Sequence 0 of rank 0 on the C oracle: serial prefill of its 256-token
    prompt, greedy decode up to the GPU's timed window (timed_window), then
    warm-up + n_steps steps (one token each) timed over that window's positions."""
    from oracle import c_oracle as CO
    cores = CO.set_threads(threads)
    own = cm is None
    if own:
        cm = CO.CModel(LAYERS, VOCAB, MAX_CTX, seed=0)
    prompt = prompts_for(0)[0]
    tok = 0
    for p, t in enumerate(prompt):
        tok, _ = cm.run_token(t, p, want_logits=(p == PROMPT - 1))
    ring = {PROMPT: tok}  # token at each decode position
    start = timed_window(n_steps)
    pos = PROMPT
    while pos < start:  # the tokens leading into the window (untimed)
        ring[pos + 1], _ = cm.run_token(ring[pos], pos)
        pos += 1
    positions = window_positions(start, warmup) + window_positions(start, n_steps)

    def step(p):
        ring[p + 1], _ = cm.run_token(ring[p], p)

    for p in positions[:warmup]:
        step(p)
    t0 = time.perf_counter()
    for p in positions[warmup:]:
        step(p)
    dt = time.perf_counter() - t0
    if own:
        cm.close()
    return {"value": n_steps / dt, "cores": cores, "seconds": dt, "start": start,
            "tokens": [ring[p] for p in range(PROMPT, PROMPT + 17) if p in ring]}


def cpu_sample_text(steps: int, warm: int, start: int) -> str:
    return (f"sequence 0 of the config-4 workload: {steps} decode steps (one token each) at positions "
            f"{start}..{start + steps - 1} (the GPU's timed window) after {warm} warm-up steps, its serial "
            "256-token prefill and the steps leading to the window; C restatement of the reference's Python Q4 "
            "path (oracle/q4_oracle.c), OpenMP over all host threads.  Extrapolated: the CPU decodes one sequence "
            "at a time, so its tokens/s on this sample stands for the 64-sequence workload")


def run_reference(args, ws, rank):
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    r = cpu_decode(steps, warm)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": round(1000.0 * r["seconds"] / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": BATCH, "prompt": PROMPT, "generate": GEN,
                   "timed_positions": [r["start"], r["start"] + steps - 1],
                   "parallelism": "host CPU, one sequence at a time"},
        "cpu_baseline": {"value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": cpu_sample_text(steps, warm, r["start"]), **host_cpu()},
        "e2e": {"value": round(r["value"], 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def batch1_secondary(device: int, steps: int, cm=None) -> dict:
    """Config 3 on the persistent kernel: batch 1, prompt 128, positions 128..255;
    with `cm` (a C-oracle model) every generated token and score of the run is
    compared with a serial oracle decode of the same prompt."""
    import torch

    from llm_accelerator_b200.model import Q4Model

    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=B1_PROMPT + B1_CYCLE, max_seqs=1, device=device)
    m.init_synthetic(seed=0)
    slot = 0
    prompt = np.random.default_rng(7).integers(0, VOCAB, B1_PROMPT).tolist()
    gen, _ = m.decode(prompt, 1, slot=slot)
    first = gen[0]
    stream = torch.cuda.ExternalStream(m.stream)
    m.decode_steps(8, slot=slot)
    m.set_position(B1_PROMPT, slot=slot)
    m.sync()
    steps = min(steps, B1_CYCLE)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    m.decode_steps(steps, slot=slot)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    toks, scores, _ = m.read_tokens(B1_PROMPT, steps + 1, slot=slot)
    n_e2e = 32
    tok, pos = first, B1_PROMPT
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        tok = m.run_token(tok, pos, slot=slot).token_id
        pos += 1
    e2e_s = time.perf_counter() - t0
    mode = m.mode
    m.close()
    out = {"workload": "cfg3: batch 1, prompt 128 uniform ids, decode positions 128..255",
           "value": round(steps / (ms / 1000.0), 2), "unit": UNIT, "ms_per_step": round(ms / steps, 4),
           "steps": steps, "mode": "persistent cooperative kernel" if mode == 1 else "per-stage CUDA graphs",
           "e2e": {"value": round(n_e2e / e2e_s, 2), "unit": UNIT, "h2d_bytes_per_step": 8,
                   "d2h_bytes_per_step": 12, "api": "q4gpu_run_token (qot_session_runner_fn)"}}
    if cm is not None:
        want, want_scores = cm.decode(prompt, steps + 1)
        same = toks.tolist() == want and scores.tolist() == want_scores
        out["parity"] = (f"identical: all {steps + 1} generated tokens and Q26 scores equal a serial C-oracle decode"
                         if same else f"MISMATCH gpu={toks.tolist()[:8]} oracle={want[:8]}")
    return out


def cfg2_secondary(device: int, peak_gbs: float) -> dict:
    """Config 2: one decoder layer at batch 1, single decode step at position 512
    (context 513) with the KV cache pre-filled with seeded N(0, 1) Q12.12 values.
    The model has 28 distinct layers, so every layer's 8.4 MB of Q4 weights and
    4.2 MB of K/V come from HBM (234 MB + 117 MB per step, above L2).  The layer
    time is one layer's graph (its five kernels PDL-chained, as the decode path
    runs them) timed per launch with the 28 layers in turn; the sum of the five
    kernels' serialised event times is reported beside it."""
    from llm_accelerator_b200.model import Q4Model

    ctx = 513
    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=ctx + 7, max_seqs=1, device=device)
    m.init_synthetic(seed=0)
    rng = np.random.default_rng(2)
    for layer in range(LAYERS):
        for kind in (0, 1):
            kv = np.clip(np.rint(rng.standard_normal((ctx - 1, 8, 128)) * 4096), -(1 << 23), (1 << 23) - 1)
            m.write_kv(layer, kind, kv.astype(np.int32))
    h = np.clip(np.rint(rng.standard_normal(1024) * 1024), -(1 << 23), (1 << 23) - 1).astype(np.int32)
    m.write_hidden(h)
    reps = 5
    tot = {}
    for _ in range(reps):
        m.set_position(ctx - 1)
        for k, (ms, n) in m.time_kernels(reps=1).items():
            tot.setdefault(k, []).append((ms, n))
    # the layer as the decode path runs it: its five kernels PDL-chained in one graph; the 28
    # layers in turn, so each layer's 12.6 MB are out of L2 again when it is next timed
    graph_us = 1000.0 * m.time_layers(0, LAYERS, ctx - 1, reps=3)
    m.close()
    layer_kinds = ("qkv_norm_rope_kv", "attention", "o_proj_residual", "post_norm_gate_up_swiglu", "down_residual")
    per = {k: float(np.median([x[0] for x in v])) for k, v in tot.items()}
    us_sum = 1000.0 * sum(per[k] for k in layer_kinds if k in per)
    us = graph_us
    layer_bytes = 8_355_840 + 4_194_304 + 24_576  # Q4 weights + K/V read + activations / K/V write
    gbs = layer_bytes / (us * 1e-6) / 1e9
    return {"workload": "cfg2: one Qwen3-0.6B layer, batch 1, decode step at position 512 (context 513), KV "
                        "pre-filled with seeded N(0,1) Q12.12, per-stage decode kernels",
            "us_per_layer": round(us, 2),
            "timing": "one layer's five kernels PDL-chained in one CUDA graph, CUDA events around each graph launch "
                      "(q4gpu_model_time_layers): the 28 layers in turn, 3 cycles after a warm-up, mean per layer",
            "us_per_layer_kernels_serialised": round(us_sum, 2),
            "kernels_us": {k: round(1000.0 * per[k], 2) for k in layer_kinds if k in per},
            "bytes_per_layer": layer_bytes, "gbs": round(gbs, 1), "frac": round(gbs / peak_gbs, 4),
            "peak": peak_gbs}


def cfg5_secondary(device: int, peak_gbs: float, steps: int = 16, check: bool = True) -> dict:
    """Config 5 on one GPU: 8 sequences with 8192-token prompts (batched exact
    prefill), greedy decode from position 8192; the attention kernel's K/V bytes
    against HBM at that context.  With `check`, sequence 0's cache is loaded into
    the C oracle and sampled positions (prompt positions, the last prompt
    position and the timed decode steps) are re-run there: K/V rows, tokens and
    scores must be identical."""
    import torch

    from llm_accelerator_b200.model import Q4Model

    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=CFG5_PROMPT + CFG5_GEN, max_seqs=CFG5_SEQS, device=device)
    m.init_synthetic(seed=0)
    prompts = [np.random.default_rng(50_000 + i).integers(0, VOCAB, CFG5_PROMPT).tolist() for i in range(CFG5_SEQS)]
    m.decode_batch([prompts[0][:2]], 1)  # batched-path buffers and prefill buffers
    t0 = time.perf_counter()
    m.decode_batch(prompts, 1)
    prefill_s = time.perf_counter() - t0
    stream = torch.cuda.ExternalStream(m.stream)
    m.batch_steps(3, CFG5_SEQS)
    m.batch_set_position(CFG5_PROMPT, CFG5_SEQS)
    m.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    m.batch_steps(steps, CFG5_SEQS)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    toks = m.read_tokens(CFG5_PROMPT, 4, slot=0)[0].tolist()
    kt = m.batch_time_kernels(CFG5_SEQS, reps=2)
    ctx = CFG5_PROMPT + steps + 2
    parity = None
    if check:
        from oracle.c_oracle import CModel
        from oracle.long_context import sampled_parity
        m.batch_set_position(CFG5_PROMPT, CFG5_SEQS)  # re-run the timed steps: the ring ends at 8192 + steps
        m.batch_steps(steps, CFG5_SEQS)
        m.sync()
        n_cached = CFG5_PROMPT + steps
        sample = [0, 1023, 1024, 4096, CFG5_PROMPT - 2, CFG5_PROMPT - 1, CFG5_PROMPT, CFG5_PROMPT + 1,
                  n_cached - 1]
        cm = CModel(LAYERS, VOCAB, CFG5_PROMPT + CFG5_GEN, seed=0)
        bad = sampled_parity(cm, m, 0, sample, n_cached=n_cached, logits_from=CFG5_PROMPT - 1)
        cm.close()
        parity = (f"identical: sequence 0 re-run by the C oracle on the GPU's cache at positions {sample}: K/V rows "
                  "of all 28 layers, and tokens and Q26 scores from the last prompt position on"
                  if not bad else f"MISMATCH {bad[:4]}")
    m.close()
    att_ms = kt["attention"][0]
    gbs = batch_kernel_bytes("attention", CFG5_SEQS, ctx, True) / (att_ms * 1e-3) / 1e9
    out = {"workload": "cfg5: 8 sequences x 8192-token uniform prompts (seeds 50000..), batched exact prefill, "
                       "greedy decode from position 8192, full vocabulary on one GPU",
           "value": round(CFG5_SEQS * steps / (ms / 1000.0), 2), "unit": UNIT, "ms_per_step": round(ms / steps, 4),
           "steps": steps, "prefill_s": round(prefill_s, 3),
           "prefill_prompt_tokens_per_s": round(CFG5_SEQS * CFG5_PROMPT / prefill_s, 1),
           "attention": {"kernel": "batch_attn_cl_tc_kernel (9-CTA clusters, tcgen05 products on the K/V byte "
                                   "planes)", "ms_per_launch": round(att_ms, 5),
                         "timing": "kernels serialised by events (q4gpu_batch_time_kernels)",
                         "context": ctx, "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak_gbs, 4)},
           "first_tokens_seq0": toks}
    if parity is not None:
        out["parity"] = parity
    return out


def gemv_secondary(device: int, peak_gbs: float) -> dict:
    """Config 1: the 3072 x 1024 Q4 GEMV over 160 distinct rotated weight copies
    (~267 MB, above L2), one q4gpu_gemv_q26_strided launch with the shared
    activation; plus the same 160 GEMVs as separate launches in one CUDA graph
    and one LM-head-sized (151936 x 1024) GEMV.  Packed bytes and scales are
    uniform random: the kernels' time does not depend on the values."""
    import torch

    from llm_accelerator_b200 import _native

    lib = _native.load()
    dev = torch.device("cuda", device)
    g = torch.Generator(device=dev).manual_seed(1)
    K, R, N, RB = 1024, 3072, 160, 151936
    act = torch.randint(-(1 << 23), 1 << 23, (K,), dtype=torch.int32, device=dev, generator=g)
    W = torch.randint(0, 256, (N, R, K // 2), dtype=torch.uint8, device=dev, generator=g)
    S = torch.randint(0, 1 << 15, (N, R, K // 64), dtype=torch.int16, device=dev, generator=g)
    out = torch.empty((N, R), dtype=torch.int64, device=dev)
    o12 = torch.empty((N, R), dtype=torch.int32, device=dev)
    per = R * K // 2 + R * K // 32 + K * 4 + R * 12  # packed + scales + activation + outputs (8 + 4 B)
    st = torch.cuda.Stream(device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn, reps):
        with torch.cuda.stream(st):
            for _ in range(3):
                fn()
            e0.record(st)
            for _ in range(reps):
                fn()
            e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    def strided():
        _native.check(lib.q4gpu_gemv_q26_strided(act.data_ptr(), 0, K, W.data_ptr(), R * K // 2, S.data_ptr(),
                                                 R * K // 64, R, N, out.data_ptr(), o12.data_ptr(), R, None,
                                                 st.cuda_stream), "q4gpu_gemv_q26_strided")

    def separate():
        for i in range(N):
            _native.check(lib.q4gpu_gemv_q26(act.data_ptr(), K, W[i].data_ptr(), S[i].data_ptr(), R,
                                             out[i].data_ptr(), o12[i].data_ptr(), None, st.cuda_stream),
                          "q4gpu_gemv_q26")

    ms_strided = timed(strided, 10)
    with torch.cuda.stream(st):
        separate()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            separate()
    ms_graph = timed(graph.replay, 5)
    del graph, W, S, out, o12
    # three copies used in turn (248 MB > L2): every launch reads its 82.6 MB from HBM
    NB = 3
    Wb = torch.randint(0, 256, (NB, RB, K // 2), dtype=torch.uint8, device=dev, generator=g)
    Sb = torch.randint(0, 1 << 15, (NB, RB, K // 64), dtype=torch.int16, device=dev, generator=g)
    ob = torch.empty(RB, dtype=torch.int64, device=dev)
    turn = [0]

    def big():
        i = turn[0] % NB
        turn[0] += 1
        _native.check(lib.q4gpu_gemv_q26(act.data_ptr(), K, Wb[i].data_ptr(), Sb[i].data_ptr(), RB, ob.data_ptr(),
                                         None, None, st.cuda_stream), "q4gpu_gemv_q26")

    ms_big = timed(big, 21)
    big_bytes = RB * (K // 2 + K // 32) + K * 4 + RB * 8
    gbs = N * per / ms_strided / 1e6
    return {"workload": "cfg1: 3072x1024 Q4 GEMV x 160 distinct weight copies (267 MB > L2), shared activation, "
                        "one q4gpu_gemv_q26_strided launch (tensor-core mma.sync u8 path)",
            "bytes_per_gemv": per, "us_per_gemv": round(ms_strided * 1000 / N, 3), "gbs": round(gbs, 1),
            "frac": round(gbs / peak_gbs, 4), "peak": peak_gbs,
            "separate_launches_in_graph": {"us_per_gemv": round(ms_graph * 1000 / N, 3),
                                           "gbs": round(N * per / ms_graph / 1e6, 1)},
            "lm_head_sized": {"rows": RB, "copies_in_turn": NB, "us": round(ms_big * 1000, 2),
                              "gbs": round(big_bytes / ms_big / 1e6, 1),
                              "frac": round(big_bytes / ms_big / 1e6 / peak_gbs, 4)}}


def run_ours(args, ws, rank, local):
    import torch

    from llm_accelerator_b200.model import Q4Model

    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    from llm_accelerator_b200.sharding import max_over_ranks as _max_over_ranks

    def max_over_ranks(x: float) -> float:
        return _max_over_ranks(x, device=torch.device("cuda", local))

    steps, warm = args.steps, args.warmup
    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=MAX_CTX, max_seqs=BATCH, device=local)
    m.init_synthetic(seed=0)
    prompts = prompts_for(rank)
    stream = torch.cuda.ExternalStream(m.stream)

    # prompts: warm the batched buffers (int8 weight copies, prefill buffers)
    # on a 2-token prompt, then run the 64 prompts twice, serially (one batched
    # step per position, the reference's order) and as batched prefill columns;
    # both leave the same K/V cache, and the argmax after position 255 is each
    # sequence's first generated token
    m.decode_batch([prompts[0][:2]], 1)
    prefill, firsts = {}, {}
    for mode, name in ((0, "serial"), (1, "batched")):
        m.prefill_mode = mode
        barrier()
        t0 = time.perf_counter()
        gen0, _ = m.decode_batch(prompts, 1)
        prefill[name] = max_over_ranks(time.perf_counter() - t0)
        firsts[name] = gen0[:, 0].copy()
    if not np.array_equal(firsts["serial"], firsts["batched"]):
        raise SystemExit("batched and serial prefill disagree")
    first = firsts["batched"]
    prefill_s = prefill["batched"]

    def enqueue(n: int, state: dict) -> int:
        """n batched decode steps cycling positions 256..510; returns launches of the resets."""
        resets = 0
        while n > 0:
            room = PROMPT + CYCLE - state["pos"]
            if room == 0:
                m.batch_set_position(PROMPT, BATCH)
                state["pos"] = PROMPT
                room = CYCLE
                resets += 1
            k = min(n, room)
            m.batch_steps(k, BATCH)
            state["pos"] += k
            n -= k
        return resets

    # one full pass over the cycle fills every sequence's token ring and cache
    # for positions 256..510; the timed window (centred in the cycle) and its
    # warm-up then replay positions whose tokens are known
    state = {"pos": PROMPT}
    enqueue(CYCLE, state)
    start = timed_window(steps)
    positions = window_positions(start, steps)
    ctx_mean = float(np.mean(positions)) + 1.0  # context of a step at position p is p + 1
    m.batch_set_position(start, BATCH)
    state["pos"] = start
    enqueue(warm, state)
    m.batch_set_position(start, BATCH)
    state["pos"] = start
    m.sync()

    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    resets = enqueue(steps, state)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    m.sync()
    ms_max = max_over_ranks(e0.elapsed_time(e1))
    value = ws * BATCH * steps / (ms_max / 1000.0)
    n_check = min(steps, CYCLE, 16)
    toks0 = m.read_tokens(PROMPT, n_check + 1, slot=0)[0].tolist()

    # end to end through the public C ABI with host buffers: per step the host
    # sends (token, position) of every sequence and reads back (token, score),
    # over the same window of positions
    e2e_steps = min(steps, PROMPT + CYCLE - start)
    tok = np.array([m.read_tokens(start, 1, slot=i)[0][0] for i in range(BATCH)], dtype=np.int64)
    pos = np.full(BATCH, start, dtype=np.int64)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok, _ = m.batch_run_step(tok, pos)
        pos += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = ws * BATCH * e2e_steps / e2e_s

    # per-kernel device times (kernels serialised by events) at the timed
    # window's mean context: `reps` steps from position mid run at contexts
    # mid + 1 .. mid + reps
    reps = 3
    mid = int(round(ctx_mean - (reps + 1) / 2.0))
    m.batch_set_position(mid, BATCH)
    m.sync()
    kt = m.batch_time_kernels(BATCH, reps=reps)
    kt_ctx = mid + (reps + 1) / 2.0
    share = {k: v[0] * v[1] for k, v in kt.items()}
    tot = sum(share.values())
    dom = max(share, key=share.get)
    peaks = measured_peaks()

    def gbs(kind: str) -> float:
        return batch_kernel_bytes(kind, BATCH, int(round(kt_ctx)), kind == "attention") / (kt[kind][0] * 1e-3) / 1e9

    launches_per_step = sum(v[1] for v in kt.values())

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms_max / steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH, "prompt": PROMPT, "generate": GEN,
                       "max_context": MAX_CTX, "timed_positions": [positions[0], positions[-1]],
                       "ctx_mean": round(ctx_mean, 2),
                       "parallelism": f"independent sequences, {BATCH} per GPU x{ws}" if ws > 1 else "single GPU",
                       "l2": "inputs larger than L2 (317 MB Q4 weights + ~5.6 GB KV cache per step)"},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": BATCH * 8,
                    "d2h_bytes_per_step": BATCH * 16,
                    "api": "q4gpu_batch_run_step: host (token, position) in, host (token, score) out, every step"},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(gbs(dom), 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs(dom) / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"], "traffic": profiled_traffic(dom),
                         "bytes_per_launch": batch_kernel_bytes(dom, BATCH, int(round(kt_ctx)), dom == "attention"),
                         "ms_per_launch": round(kt[dom][0], 5), "context": round(kt_ctx, 1)},
            "kernels": {k: {"ms_per_launch": round(v[0], 5), "launches_per_step": v[1],
                            "share": round(share[k] / tot, 4), "gbs": round(gbs(k), 1)} for k, v in kt.items()},
            "prefill_s": round(prefill_s, 3),
            "prefill": {"batched_s": round(prefill["batched"], 3), "serial_s": round(prefill["serial"], 3),
                        "prompt_tokens_per_s": round(ws * BATCH * PROMPT / prefill["batched"], 1),
                        "note": "q4gpu_decode_batch(prompts, 1) wall time, max over ranks: 64 x 255 prompt "
                                "positions as batched columns (or one batched step per position) plus the "
                                "step at the last prompt token; first tokens identical"},
            "gpu_launches": launches_per_step * steps + resets,
            "clocks": clocks,
        }
    m.close()
    if rank == 0:
        if ws == 1:
            from oracle import c_oracle as CO
            cm = None if args.no_cpu_baseline else CO.CModel(LAYERS, VOCAB, MAX_CTX, seed=0)
            line["batch1"] = batch1_secondary(local, 128, cm)
            line["cfg2"] = cfg2_secondary(local, peaks["hbm_gbs"])
            line["gemv"] = gemv_secondary(local, peaks["hbm_gbs"])
            line["cfg5"] = cfg5_secondary(local, peaks["hbm_gbs"], check=not args.no_cpu_baseline)
            if cm is not None:
                c = cpu_decode(args.cpu_steps, 2, cm=cm)
                cm.close()
                line["cpu_baseline"] = {
                    "value": round(c["value"], 3), "unit": UNIT, "cores": c["cores"], "kind": "port",
                    "sample": cpu_sample_text(args.cpu_steps, 2, c["start"]), **host_cpu()}
                n = min(len(c["tokens"]), len(toks0))
                line["parity"] = "sequence 0 tokens identical to the CPU oracle" if c["tokens"][:n] == toks0[:n] \
                    else f"MISMATCH gpu={toks0[:n]} cpu={c['tokens'][:n]}"
    if ws > 1:
        # config 5 across the same process group: the one collective on this
        # path (the vocabulary-sharded LM head's exchanges), measured per N
        c5 = cfg5_sharded(ws, rank, local, 16, 3)
        if rank == 0:
            line["cfg5"] = c5
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Config 5 (opt-in, --cfg5): 8 sequences with 8192-token prompts, decode at
# context 8192..; the 8 sequences are split over the ranks and, for N > 1, the
# LM head is vocabulary-sharded with an NCCL exchange of the (score, row)
# winners.  Prints its own JSON line (rank 0).
# ---------------------------------------------------------------------------


def cfg5_sharded(ws: int, rank: int, local: int, steps: int, warmup: int) -> dict:
    """Config 5 over the process group: the 8 sequences split over the ranks and,
    for N > 1, the tied LM head vocabulary-sharded (llm_accelerator_b200.sharding:
    NCCL all_gather of the final vectors and of the (score, row) winners, one
    reduce-and-commit kernel), the whole step replayed as one CUDA graph.  Steps
    are timed on the device, max over ranks; the two collectives alone are timed
    the same way on the same buffers (`exchange_us_per_step`)."""
    import torch
    import torch.distributed as dist

    from llm_accelerator_b200.model import Q4Model
    from llm_accelerator_b200.sharding import VocabShardedDecoder, max_over_ranks, shard_range

    dev = torch.device("cuda", local)
    if CFG5_SEQS % ws:
        raise SystemExit("config 5 needs a GPU count dividing 8")
    a, b = shard_range(CFG5_SEQS, ws, rank)
    n_local = b - a
    prompts = [np.random.default_rng(50_000 + i).integers(0, VOCAB, CFG5_PROMPT).tolist() for i in range(a, b)]
    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=CFG5_PROMPT + CFG5_GEN, max_seqs=n_local, device=local)
    m.init_synthetic(seed=0)
    stream = torch.cuda.ExternalStream(m.stream)
    if ws > 1:
        dist.barrier()
    t0 = time.perf_counter()
    m.decode_batch(prompts, 1)  # batched prefill; the first generated token of each sequence
    prefill_s = max_over_ranks(time.perf_counter() - t0, device=dev)
    steps = min(steps, CFG5_GEN - 1)
    dec = VocabShardedDecoder(m, n_local) if ws > 1 else None
    graphed = False
    if dec is not None:
        dec.step()  # eager: communicators, buffers, the forward graph
        m.sync()
        graphed = dec.capture()

    def run(n):
        for _ in range(n):
            if dec is not None:
                dec.step()
            else:
                m.batch_steps(1, n_local)

    run(max(warmup, 3))
    m.batch_set_position(CFG5_PROMPT, n_local)
    m.sync()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(steps)
    e1.record(stream)
    e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), device=dev)
    toks = m.read_tokens(CFG5_PROMPT, 4, slot=0)[0].tolist()
    exch_us = None
    if dec is not None:
        with torch.cuda.stream(stream):
            for _ in range(3):
                dist.all_gather_into_tensor(dec.all_acts, dec.acts)
                dist.all_gather_into_tensor(dec.win, dec.mine)
            x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            x0.record(stream)
            for _ in range(20):
                dist.all_gather_into_tensor(dec.all_acts, dec.acts)
                dist.all_gather_into_tensor(dec.win, dec.mine)
            x1.record(stream)
        x1.synchronize()
        exch_us = max_over_ranks(1000.0 * x0.elapsed_time(x1) / 20, device=dev)
        dec.release()
    m.close()
    out = {"workload": "cfg5: 8 sequences x 8192-token uniform prompts (seeds 50000..), batched exact prefill, "
                       "greedy decode from position 8192", "n_gpus": ws, "sequences_per_gpu": n_local,
           "value": round(CFG5_SEQS * steps / (ms / 1000), 2), "unit": UNIT, "ms_per_step": round(ms / steps, 4),
           "steps": steps, "scaling": "strong", "prefill_s": round(prefill_s, 3),
           "prefill_prompt_tokens_per_s": round(CFG5_SEQS * CFG5_PROMPT / prefill_s, 1),
           "lm_head": (f"vocabulary-sharded over {ws} GPUs: NCCL all_gather of the final vectors and of the (score, "
                       "row) winners, q4gpu_batch_commit_shards, step " + ("replayed as one CUDA graph" if graphed
                                                                          else "enqueued eagerly"))
           if ws > 1 else "full vocabulary on one GPU",
           "first_tokens_seq0": toks}
    if exch_us is not None:
        out["exchange_us_per_step"] = round(exch_us, 2)
    return out


def run_cfg5(args, ws, rank, local):
    import torch

    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    r = cfg5_sharded(ws, rank, local, args.steps, args.warmup)
    if rank == 0:
        line = {"metric": "decode tokens/sec (config 5: batch 8, context 8192..)", "higher_is_better": True,
                "dtype": "int64", "data": "synthetic", **r,
                "config": {"workload": r["workload"], "sequences_per_gpu": r["sequences_per_gpu"],
                           "lm_head": r["lm_head"]}}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=255)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cfg5", action="store_true", help="run config 5 (long context, sharded LM head) instead")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, ws, rank)
    elif args.cfg5:
        run_cfg5(args, ws, rank, local)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
