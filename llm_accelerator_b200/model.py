"""Host-side model context: device-resident Q4 weights, paged KV cache and
the decode graphs of libq4gpu, driven through the reference's runner seam.

``Q4Model.run_token`` is ``qot_run_token`` (one full-model invocation per
call, ``FPGA_Project/software/qmap_one_token_runtime/qmap_one_token_runtime.h:369-392``)
and ``Q4Model.decode`` is ``qot_decode_token_ids`` (``:399-500``); both return
the reference's ``QOT_*`` status codes through ``QotError``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native
from . import tables
from ._native import QotResult, QotRunConfig

HIDDEN = 1024
VOCAB = 151936
LAYERS = 28

QOT_NAMES = {0: "OK", -1: "BUSY", -2: "BAD_LAYER", -3: "BAD_TABLE", -4: "BAD_ADDR", -5: "TIMEOUT",
             -6: "STATUS", -7: "NULL", -8: "BAD_TOKEN", -9: "CAPACITY", -10: "CONTEXT"}

WEIGHT_SHAPES = {_native.T_Q: (2048, 1024), _native.T_K: (1024, 1024), _native.T_V: (1024, 1024),
                 _native.T_O: (1024, 2048), _native.T_GATE: (3072, 1024), _native.T_UP: (3072, 1024),
                 _native.T_DOWN: (1024, 3072)}
GAMMA_SIZES = {_native.T_INPUT_GAMMA: 1024, _native.T_POST_GAMMA: 1024, _native.T_Q_GAMMA: 128,
               _native.T_K_GAMMA: 128}


class QotError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: QOT_ERR_{QOT_NAMES.get(code, code)} ({code})")
        self.code = code


def _ptr(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


@dataclass
class RunResult:
    token_id: int
    score_q26: int
    raw: QotResult


class Q4Model:
    """One B200 model context (weights + KV for ``max_seqs`` sequence slots)."""

    def __init__(self, n_layers: int = LAYERS, vocab: int = VOCAB, max_context: int = 256, max_seqs: int = 1,
                 device: int = 0):
        self.lib = _native.load()
        cfg = _native.ModelConfig(n_layers=n_layers, vocab=vocab, max_context=max_context, max_seqs=max_seqs,
                                  device=device)
        h = C.c_void_p()
        _native.check(self.lib.q4gpu_model_create(C.byref(cfg), C.byref(h)), "q4gpu_model_create")
        self.handle = h
        self.n_layers, self.vocab, self.max_context, self.max_seqs = n_layers, vocab, max_context, max_seqs
        self._prefill_mode = 1
        self.install_rope_tables()

    # -- lifecycle ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.q4gpu_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def stream(self) -> int:
        return int(self.lib.q4gpu_model_stream(self.handle) or 0)

    # -- weights -----------------------------------------------------------
    def init_synthetic(self, seed: int = 0, std: float = 0.02, gamma_std: float = 0.0) -> None:
        """Seeded random-init weights quantised on the device."""
        _native.check(self.lib.q4gpu_model_init_synthetic(self.handle, seed, std, gamma_std),
                      "q4gpu_model_init_synthetic")

    def install_rope_tables(self) -> None:
        cos, sin = tables.rope_tables(self.max_context)
        self.set_table(_native.T_ROPE_COS, cos)
        self.set_table(_native.T_ROPE_SIN, sin)

    def set_table(self, which: int, values: np.ndarray, layer: int = 0) -> None:
        v = np.ascontiguousarray(values, dtype=np.int32)
        _native.check(self.lib.q4gpu_model_set_tensor(self.handle, layer, which, _ptr(v), v.nbytes, None, 0),
                      "q4gpu_model_set_tensor")

    def set_weight(self, layer: int, which: int, packed: np.ndarray, scale: np.ndarray) -> None:
        p = np.ascontiguousarray(packed, dtype=np.uint8)
        s = np.ascontiguousarray(scale, dtype=np.uint16)
        _native.check(self.lib.q4gpu_model_set_tensor(self.handle, layer, which, _ptr(p), p.nbytes, _ptr(s),
                                                      s.nbytes), "q4gpu_model_set_tensor")

    def get_weight(self, layer: int, which: int) -> tuple[np.ndarray, np.ndarray]:
        rows, cols = (self.vocab, HIDDEN) if which == _native.T_EMBED else WEIGHT_SHAPES[which]
        p = np.empty((rows, cols // 2), dtype=np.uint8)
        s = np.empty((rows, cols // 64), dtype=np.uint16)
        _native.check(self.lib.q4gpu_model_get_tensor(self.handle, layer, which, _ptr(p), p.nbytes, _ptr(s),
                                                      s.nbytes), "q4gpu_model_get_tensor")
        return p, s

    def get_gamma(self, layer: int, which: int) -> np.ndarray:
        n = HIDDEN if which == _native.T_FINAL_GAMMA else GAMMA_SIZES[which]
        g = np.empty(n, dtype=np.int32)
        _native.check(self.lib.q4gpu_model_get_tensor(self.handle, layer, which, _ptr(g), g.nbytes, None, 0),
                      "q4gpu_model_get_tensor")
        return g

    # -- runner seam -------------------------------------------------------
    def run_config(self, layer_start: int = 0, layer_count: int | None = None, embedding: bool = True,
                   position: int = 0) -> QotRunConfig:
        c = QotRunConfig()
        c.layer_start = layer_start
        c.layer_count = self.n_layers - layer_start if layer_count is None else layer_count
        c.position = position
        c.runtime_context_enable = 1
        c.embedding_enable = 1 if embedding else 0
        return c

    def run_token(self, token: int, position: int, slot: int = 0, layer_start: int = 0,
                  layer_count: int | None = None, embedding: bool = True, max_polls: int = 0) -> RunResult:
        cfg = self.run_config(layer_start, layer_count, embedding, position)
        res = QotResult()
        rc = self.lib.q4gpu_run_token(self.handle, slot, C.byref(cfg), token, position, max_polls, C.byref(res))
        if rc != 0:
            raise QotError(rc, "q4gpu_run_token")
        return RunResult(res.token_id, res.score_q26, res)

    def decode(self, prompt, max_new_tokens: int, slot: int = 0, position: int = 0,
               max_polls_per_token: int = 0) -> tuple[list[int], QotResult]:
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        out = np.zeros(max(max_new_tokens, 1), dtype=np.uint32)
        cnt = C.c_uint32(0)
        res = QotResult()
        cfg = self.run_config(position=position)
        rc = self.lib.q4gpu_decode_token_ids(self.handle, slot, C.byref(cfg), _ptr(p), p.size, max_new_tokens,
                                             _ptr(out), out.size, max_polls_per_token, C.byref(cnt), C.byref(res))
        if rc != 0:
            raise QotError(rc, "q4gpu_decode_token_ids")
        return out[: cnt.value].astype(np.int64).tolist(), res

    def decode_batch(self, prompts, max_new_tokens: int) -> tuple[np.ndarray, np.ndarray]:
        lens = np.asarray([len(p) for p in prompts], dtype=np.uint32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint32) for p in prompts]))
        gen = np.zeros((len(prompts), max_new_tokens), dtype=np.uint32)
        scores = np.zeros((len(prompts), max_new_tokens), dtype=np.int64)
        rc = self.lib.q4gpu_decode_batch(self.handle, len(prompts), _ptr(flat), _ptr(lens), max_new_tokens,
                                         _ptr(gen), _ptr(scores))
        if rc != 0:
            raise QotError(rc, "q4gpu_decode_batch: " + self.lib.q4gpu_last_error().decode(errors="replace"))
        return gen.astype(np.int64), scores

    # -- batched decode (up to 64 slots per step) ------------------------------
    def batch_steps(self, n_steps: int, n_seq: int, first_slot: int = 0) -> None:
        """Enqueue n batched steps for slots [first_slot, first_slot + n_seq) (async)."""
        _native.check(self.lib.q4gpu_batch_steps(self.handle, first_slot, n_seq, n_steps), "q4gpu_batch_steps")

    def batch_prefill(self, prompts, first_slot: int = 0) -> None:
        """Store the prompts in slots [first_slot, first_slot + len(prompts)) and prefill
        positions 0 .. len - 2 of each as batched columns; every slot is left at its last
        prompt token (position len - 1, lm_from len) for batch_steps (async)."""
        lens = np.asarray([len(p) for p in prompts], dtype=np.uint32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint32) for p in prompts]))
        _native.check(self.lib.q4gpu_batch_prefill(self.handle, first_slot, len(prompts), _ptr(flat), _ptr(lens)),
                      "q4gpu_batch_prefill")

    @property
    def prefill_mode(self) -> int:
        """How decode_batch runs prompts: 1 batched prefill (default), 0 serial steps."""
        return self._prefill_mode

    @prefill_mode.setter
    def prefill_mode(self, value: int) -> None:
        _native.check(self.lib.q4gpu_model_set_prefill(self.handle, value), "q4gpu_model_set_prefill")
        self._prefill_mode = int(value)

    def batch_set_position(self, position: int, n_seq: int, first_slot: int = 0, lm_from: int = -1) -> None:
        _native.check(self.lib.q4gpu_batch_set_position(self.handle, first_slot, n_seq, position, lm_from),
                      "q4gpu_batch_set_position")

    def batch_run_step(self, tokens, positions, first_slot: int = 0) -> tuple[np.ndarray, np.ndarray]:
        """One batched step with host buffers: (next tokens, Q26 scores) per sequence."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        out = np.zeros(t.size, dtype=np.uint32)
        sc = np.zeros(t.size, dtype=np.int64)
        _native.check(self.lib.q4gpu_batch_run_step(self.handle, first_slot, t.size, _ptr(t), _ptr(p), _ptr(out),
                                                    _ptr(sc)), "q4gpu_batch_run_step")
        return out.astype(np.int64), sc

    # -- vocabulary-sharded LM head -----------------------------------------
    def batch_forward_hidden(self, n_seq: int, out, first_slot: int = 0) -> None:
        """One position of slots [first_slot, first_slot + n_seq) up to the final RMSNorm;
        `out`: int32 CUDA tensor [n_seq, 1024] receiving the normed vectors (async)."""
        _native.check(self.lib.q4gpu_batch_forward_hidden(self.handle, first_slot, n_seq, out.data_ptr()),
                      "q4gpu_batch_forward_hidden")

    def lm_head_shard(self, acts, row_begin: int, row_end: int, best_score, best_row) -> None:
        """LM head over vocabulary rows [row_begin, row_end) for acts (int32 CUDA [n, 1024]);
        best_score / best_row: int64 CUDA [n] (async)."""
        _native.check(self.lib.q4gpu_lm_head_shard(self.handle, acts.data_ptr(), acts.shape[0], row_begin, row_end,
                                                   best_score.data_ptr(), best_row.data_ptr()),
                      "q4gpu_lm_head_shard")

    def batch_commit(self, tokens, scores, first_slot: int = 0) -> None:
        """Store tokens / scores (int64 CUDA [n]) at each slot's position + 1 and advance (async)."""
        _native.check(self.lib.q4gpu_batch_commit(self.handle, first_slot, tokens.shape[0], tokens.data_ptr(),
                                                  scores.data_ptr()), "q4gpu_batch_commit")

    def batch_commit_shards(self, winners, n_seq: int, col0: int, first_slot: int = 0) -> None:
        """Reduce per-shard (score, row) winners (int64 CUDA [shards, 2, stride]) for
        this model's sequences (columns col0 .. col0 + n_seq) and commit them (async)."""
        _native.check(self.lib.q4gpu_batch_commit_shards(self.handle, first_slot, n_seq, winners.data_ptr(),
                                                         winners.shape[0], winners.shape[2], col0),
                      "q4gpu_batch_commit_shards")

    def batch_time_kernels(self, n_seq: int, reps: int = 2, first_slot: int = 0) -> dict[str, tuple[float, int]]:
        """Mean device ms per launch and launches per step of each batched kernel
        (kernels serialised by events; advances the positions by `reps`)."""
        k = len(_native.BATCH_KERNEL_KINDS)
        ms = np.zeros(k, dtype=np.float64)
        cnt = np.zeros(k, dtype=np.int32)
        _native.check(self.lib.q4gpu_batch_time_kernels(self.handle, first_slot, n_seq, reps, _ptr(ms), _ptr(cnt)),
                      "q4gpu_batch_time_kernels")
        return {name: (float(ms[i]), int(cnt[i])) for i, name in enumerate(_native.BATCH_KERNEL_KINDS) if cnt[i]}

    def batch_trace(self, n_seq: int, first_slot: int = 0) -> tuple[np.ndarray, np.ndarray]:
        """One batched step with timelines on: attention stamps [layers, n_seq, 8, 8] and
        GEMM stamps [4 * layers + 1, 1200, 8] (ns; see q4gpu_batch_trace)."""
        at = np.zeros((self.n_layers, n_seq, 8, 8), dtype=np.uint64)
        gt = np.zeros((4 * self.n_layers + 1, 1200, 8), dtype=np.uint64)
        _native.check(self.lib.q4gpu_batch_trace(self.handle, first_slot, n_seq, _ptr(at), at.size, _ptr(gt), gt.size),
                      "q4gpu_batch_trace")
        return at, gt

    # -- device-resident decode loop ----------------------------------------
    def decode_steps(self, n_steps: int, slot: int = 0) -> None:
        """Enqueue n greedy steps continuing slot's decode on the device (async)."""
        _native.check(self.lib.q4gpu_decode_steps(self.handle, slot, n_steps), "q4gpu_decode_steps")

    @property
    def mode(self) -> int:
        """0: per-stage kernels in CUDA graphs; 1: persistent cooperative kernel."""
        return int(self.lib.q4gpu_model_get_mode(self.handle))

    @mode.setter
    def mode(self, value: int) -> None:
        _native.check(self.lib.q4gpu_model_set_mode(self.handle, value), "q4gpu_model_set_mode")

    def trace_persistent(self, n_steps: int, lm_from: int = 0, slot: int = 0) -> np.ndarray:
        """[barriers, 2] (last arrival, release) ns of a persistent run: per step
        3 grid barriers per layer (after QKV, after attention + o_proj, after
        gate/up + down) and one after the LM head."""
        n = n_steps * (3 * self.n_layers + 1)
        st = np.zeros((n, 2), dtype=np.uint64)
        _native.check(self.lib.q4gpu_model_trace_persistent(self.handle, slot, n_steps, lm_from, _ptr(st), n),
                      "q4gpu_model_trace_persistent")
        return st

    def persistent_stage_times(self, n_steps: int = 4, slot: int = 0) -> dict:
        """Mean µs per stage of the persistent decode kernel from its barrier
        timeline over steps 2..n_steps of a run from the slot's position:
        {stage: [work (previous release -> last arrival), barrier (last arrival
        -> release)]} for qkv, attn_o, gateup_down and lm, plus step_us."""
        st = self.trace_persistent(n_steps, slot=slot).astype(np.int64)
        per_step = 3 * self.n_layers + 1
        names = ["qkv", "attn_o", "gateup_down"]
        work = {k: [] for k in names + ["lm"]}
        bar = {k: [] for k in names + ["lm"]}
        for s in range(1, n_steps):
            base = s * per_step
            prev = st[base - 1, 1]
            for i in range(per_step):
                arr, rel = st[base + i]
                k = "lm" if i == per_step - 1 else names[i % 3]
                work[k].append(arr - prev)
                bar[k].append(rel - arr)
                prev = rel
        out = {"step_us": round(float(st[n_steps * per_step - 1, 1] - st[per_step - 1, 1]) / (n_steps - 1) / 1e3, 1)}
        for k in names + ["lm"]:
            out[k] = [round(float(np.mean(work[k])) / 1e3, 2), round(float(np.mean(bar[k])) / 1e3, 2)]
        return out

    def set_position(self, position: int, slot: int = 0) -> None:
        _native.check(self.lib.q4gpu_model_set_position(self.handle, slot, position), "q4gpu_model_set_position")

    def sync(self) -> None:
        _native.check(self.lib.q4gpu_model_sync(self.handle), "q4gpu_model_sync")

    def read_tokens(self, start: int, n: int, slot: int = 0) -> tuple[np.ndarray, np.ndarray, int]:
        t = np.zeros(max(n, 1), dtype=np.int32)
        s = np.zeros(max(n, 1), dtype=np.int64)
        pos = C.c_int32(0)
        _native.check(self.lib.q4gpu_model_read_tokens(self.handle, slot, start, n, _ptr(t), _ptr(s),
                                                       C.byref(pos)), "q4gpu_model_read_tokens")
        return t[:n].astype(np.int64), s[:n], pos.value

    def time_layers(self, layer_start: int, layer_count: int, position: int, reps: int = 3, slot: int = 0) -> float:
        """Mean device ms of one per-stage layer at `position`: each layer of
        [layer_start, +layer_count) as its own graph (PDL-chained kernels, no
        embedding, no LM head), the layers timed in turn for `reps` cycles."""
        ms = np.zeros(1, dtype=np.float64)
        _native.check(self.lib.q4gpu_model_time_layers(self.handle, slot, layer_start, layer_count, position, reps,
                                                       _ptr(ms)), "q4gpu_model_time_layers")
        return float(ms[0])

    def time_kernels(self, reps: int = 3, slot: int = 0) -> dict[str, tuple[float, int]]:
        """Mean device ms per launch and launches per step of each kernel kind."""
        ms = np.zeros(8, dtype=np.float64)
        cnt = np.zeros(8, dtype=np.int32)
        _native.check(self.lib.q4gpu_model_time_kernels(self.handle, slot, reps, _ptr(ms), _ptr(cnt)),
                      "q4gpu_model_time_kernels")
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(_native.KERNEL_KINDS) if cnt[i]}

    # -- state access ------------------------------------------------------
    def read_hidden(self, slot: int = 0) -> np.ndarray:
        h = np.empty(HIDDEN, dtype=np.int32)
        _native.check(self.lib.q4gpu_model_read_hidden(self.handle, slot, _ptr(h)), "q4gpu_model_read_hidden")
        return h.astype(np.int64)

    def write_hidden(self, hidden, slot: int = 0) -> None:
        h = np.ascontiguousarray(np.asarray(hidden, dtype=np.int32))
        _native.check(self.lib.q4gpu_model_write_hidden(self.handle, slot, _ptr(h)), "q4gpu_model_write_hidden")

    def read_kv(self, layer: int, kind: int, positions: int, slot: int = 0, raw: bool = False) -> np.ndarray:
        """K (kind 0) or V (kind 1) rows [positions, 8, 128] of a layer in the reference's
        order; int64 like the reference's arrays, or the stored int32 words with raw=True."""
        out = np.empty((positions, 8, 128), dtype=np.int32)
        _native.check(self.lib.q4gpu_model_read_kv(self.handle, slot, layer, kind, positions, _ptr(out)),
                      "q4gpu_model_read_kv")
        return out if raw else out.astype(np.int64)

    def write_kv(self, layer: int, kind: int, data, slot: int = 0) -> None:
        d = np.ascontiguousarray(np.asarray(data, dtype=np.int32))
        _native.check(self.lib.q4gpu_model_write_kv(self.handle, slot, layer, kind, d.shape[0], _ptr(d)),
                      "q4gpu_model_write_kv")
