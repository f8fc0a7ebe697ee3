"""Decode benchmark: Qwen3-0.6B Q4 fixed-point greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the 28-layer, 151936-vocabulary Qwen3-0.6B with
seeded synthetic Q4 weights (seed 0), batch 1, a 128-token prompt of uniform
random ids, greedy decode.  One step = one generated token (embedding, 28
layers, final norm, LM head + argmax) with the decode positions cycling
through 128..255 (the generated half of config 3; every cycle repeats the
same tokens).  Weights are 316 MB per step, larger than L2.

N > 1 (torchrun, one rank per GPU): every rank decodes its own independent
sequence (prompt seed = rank); no collective on the data path; value is the
total tokens/s over ranks with the max-over-ranks device time (weak scaling).

`--impl reference` times the reference's arithmetic on the host CPU (the C
restatement of the reference's Python Q4 path, all host threads) on the
same workload; under torchrun only rank 0 runs it.
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

METRIC = "decode tokens/sec (batch 1), Qwen3-0.6B Q4 greedy decode"
UNIT = "tokens/s"
PROMPT_LEN = 128
CYCLE = 128  # decode positions 128..255
VOCAB = 151936
LAYERS = 28
WORKLOAD = ("cfg3: Qwen3-0.6B 28-layer Q4 (int4 + Q2.14 group scales) greedy decode, batch 1, tied "
            "151936-vocab LM head, prompt 128 uniform ids (seed = rank), decode positions 128..255 cycled")

# bytes one launch of each kernel kind reads/writes (algorithmic)
QKV_ROWS, O_ROWS, INTER = 4096, 1024, 3072


def kernel_bytes(kind: str, ctx: int) -> int:
    if kind == "embed":
        return 512 + 32 + 4096
    if kind == "qkv_norm_rope_kv":
        return QKV_ROWS * (512 + 32) + 4096 + 2 * 4096 + 2 * 128 * 4 * 2 + 8192
    if kind == "attention":
        return 2 * 8 * 128 * 4 * ctx + 8192 + 8192
    if kind == "o_proj_residual":
        return O_ROWS * (1024 + 64) + 8192 + 4096 + 4096
    if kind == "post_norm_gate_up_swiglu":
        return 2 * INTER * (512 + 32) + 4096 + INTER * 4
    if kind == "down_residual":
        return O_ROWS * (1536 + 96) + INTER * 4 + 4096 + 4096
    if kind == "final_norm_lm_head_argmax":
        return VOCAB * (512 + 32) + 4096 + 16
    return 0


def step_bytes(ctx: int) -> int:
    per_layer = sum(kernel_bytes(k, ctx) for k in ("qkv_norm_rope_kv", "attention", "o_proj_residual",
                                                   "post_norm_gate_up_swiglu", "down_residual"))
    return kernel_bytes("embed", ctx) + LAYERS * per_layer + kernel_bytes("final_norm_lm_head_argmax", ctx)


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


def stage_timeline(m, n_steps: int) -> dict:
    """Mean per-stage work and barrier latency (us) of persistent decode steps."""
    st = m.trace_persistent(n_steps).astype(np.int64)
    per_step = 5 * LAYERS + 1
    names = ["qkv", "attention", "o_proj", "gate_up", "down"]
    work = {k: [] for k in names + ["lm_head"]}
    wait = {k: [] for k in names + ["lm_head"]}
    for s in range(1, n_steps):
        base = s * per_step
        prev = st[base - 1, 1]
        for i in range(per_step):
            arr, rel = st[base + i]
            k = "lm_head" if i == per_step - 1 else names[i % 5]
            work[k].append(arr - prev)
            wait[k].append(rel - arr)
            prev = rel
    out = {k: {"work": round(float(np.mean(work[k])) / 1e3, 3), "barrier": round(float(np.mean(wait[k])) / 1e3, 3)}
           for k in work}
    out["step"] = round(float(st[n_steps * per_step - 1, 1] - st[per_step - 1, 1]) / (n_steps - 1) / 1e3, 2)
    return out


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def prompt_for(rank: int) -> list[int]:
    return np.random.default_rng(rank).integers(0, VOCAB, PROMPT_LEN).tolist()


# ---------------------------------------------------------------------------
# CPU arm: the C restatement of the reference path
# ---------------------------------------------------------------------------
def cpu_decode(n_steps: int, warmup: int, threads: int = 0) -> dict:
    from oracle import c_oracle as CO
    cores = CO.set_threads(threads)
    m = CO.CModel(LAYERS, VOCAB, PROMPT_LEN + CYCLE, seed=0)
    prompt = prompt_for(0)
    tok = 0
    for p, t in enumerate(prompt):
        tok, _ = m.run_token(t, p, want_logits=(p == PROMPT_LEN - 1))
    first = tok
    toks = []
    pos = PROMPT_LEN

    def step():
        nonlocal tok, pos
        if pos >= PROMPT_LEN + CYCLE:
            pos, tok = PROMPT_LEN, first
        tok, _ = m.run_token(tok, pos)
        toks.append(tok)
        pos += 1

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(n_steps):
        step()
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n_steps / dt, "cores": cores, "seconds": dt, "tokens": [first] + toks}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    r = cpu_decode(steps, warm)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "warmup": warm, "ms_per_step": round(1000.0 * r["seconds"] / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": 1, "prompt": PROMPT_LEN, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(r["value"], 3), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": f"{steps} decode steps after {warm} warm-up steps and the 128-token prefill, "
                                   "C restatement of the reference's Python Q4 path (oracle/q4_oracle.c), "
                                   "OpenMP over all host threads"},
        "e2e": {"value": round(r["value"], 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
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

    steps, warm = args.steps, args.warmup
    m = Q4Model(n_layers=LAYERS, vocab=VOCAB, max_context=PROMPT_LEN + CYCLE + 1, max_seqs=1, device=local)
    m.init_synthetic(seed=0)
    prompt = prompt_for(rank)
    gen, _ = m.decode(prompt, 1)  # serial prefill of the prompt; pos is now 128
    first = gen[0]
    stream = torch.cuda.ExternalStream(m.stream)

    def enqueue(n: int, state: dict):
        """n decode steps, cycling positions 128..255."""
        while n > 0:
            room = PROMPT_LEN + CYCLE - state["pos"]
            if room == 0:
                m.set_position(PROMPT_LEN)
                state["pos"] = PROMPT_LEN
                room = CYCLE
            k = min(n, room)
            m.decode_steps(k)
            state["pos"] += k
            n -= k

    state = {"pos": PROMPT_LEN}
    enqueue(warm, state)
    m.sync()
    # parity spot check of the cycle: the device must reproduce the first cycle's tokens
    toks = m.read_tokens(PROMPT_LEN, min(warm, CYCLE) + 1)[0].tolist()

    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    enqueue(steps, state)
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    value = ws * steps / (ms_max / 1000.0)

    # end to end through the runner seam (qot_session_runner_fn): per step the
    # host passes (token, position) from pinned memory and reads (token, score)
    e2e_steps = steps
    tok, pos = first, PROMPT_LEN
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if pos >= PROMPT_LEN + CYCLE:
            tok, pos = first, PROMPT_LEN
        tok = m.run_token(tok, pos).token_id
        pos += 1
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = ws * e2e_steps / e2e_s

    # timeline of the persistent kernel: per stage, work (previous release to
    # the last CTA's arrival) and barrier latency (last arrival to release)
    m.set_position(PROMPT_LEN)
    m.sync()
    tl = stage_timeline(m, 4) if m.mode == 1 else None
    # per-kernel device times of the per-stage kernels (mode 0, events between kernels)
    m.set_position(PROMPT_LEN)
    m.sync()
    kt = m.time_kernels(reps=3)
    peaks = measured_peaks()
    lm = "final_norm_lm_head_argmax"
    lm_gbs = kernel_bytes(lm, 0) / (kt[lm][0] * 1e-3) / 1e9
    step_b = step_bytes(PROMPT_LEN + CYCLE // 2)
    step_gb = step_b / 1e9
    if m.mode == 1:
        # one persistent launch per 128-step cycle: its bytes over its device time
        dom = "decode_persistent_kernel"
        dom_bytes = step_b * CYCLE
        dom_ms = ms_max / steps * CYCLE
        launches = -(-steps // CYCLE) * 2  # the persistent kernel + a position reset per cycle
    else:
        share = {k: v[0] * v[1] for k, v in kt.items()}
        dom = max(share, key=share.get)
        dom_bytes = kernel_bytes(dom, PROMPT_LEN + 2)
        dom_ms = kt[dom][0]
        launches = sum(v[1] for v in kt.values()) * steps
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    share = {k: v[0] * v[1] for k, v in kt.items()}
    tot = sum(share.values())

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms_max / steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": 1, "prompt": PROMPT_LEN, "seq_len": PROMPT_LEN + CYCLE,
                       "parallelism": f"independent sequences x{ws}" if ws > 1 else "single GPU",
                       "l2": "inputs larger than L2 (316 MB of Q4 weights per step)"},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 12,
                    "api": "q4gpu_run_token (qot_session_runner_fn signature), one host round trip per token"},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": peaks["source"], "traffic": profiled_traffic(dom),
                         "bytes_per_launch": dom_bytes, "ms_per_launch": round(dom_ms, 5)},
            "mode": "persistent cooperative kernel" if m.mode == 1 else "per-stage kernels in CUDA graphs",
            "stage_timeline_us": tl,
            "step_roofline": {"bytes_per_step": int(step_gb * 1e9),
                              "achieved_gbs": round(step_gb / (ms_max / steps / 1000.0), 1),
                              "frac": round(step_gb / (ms_max / steps / 1000.0) / peaks["hbm_gbs"], 4)},
            "gemv": {"kernel": "lm head 151936x1024 Q4 GEMV + argmax", "gbs": round(lm_gbs, 1),
                     "frac": round(lm_gbs / peaks["hbm_gbs"], 4)},
            "stage_kernels_mode0": {k: {"ms_per_launch": round(v[0], 5), "launches_per_step": v[1],
                                        "share": round(share[k] / tot, 4)} for k, v in kt.items()},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if ws == 1 and not args.no_cpu_baseline:
            c = cpu_decode(args.cpu_steps, 2)
            line["cpu_baseline"] = {
                "value": round(c["value"], 3), "unit": UNIT, "cores": c["cores"], "kind": "port",
                "sample": f"{args.cpu_steps} decode steps at positions 130.. after the same 128-token prefill, "
                          "C restatement of the reference's Python Q4 path (oracle/q4_oracle.c), all host threads"}
            n = min(len(c["tokens"]), len(toks))
            line["parity"] = "tokens identical to CPU oracle" if c["tokens"][:n] == toks[:n] else \
                f"MISMATCH gpu={toks[:n]} cpu={c['tokens'][:n]}"
        print(json.dumps(line), flush=True)
    m.close()
    if dist is not None:
        barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, ws, rank)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
