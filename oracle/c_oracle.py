"""ctypes wrapper of the C oracle (oracle/q4_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import build_oracle
from . import q4_oracle as O

P = C.c_void_p
_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = build_oracle.build()
        L = C.CDLL(str(path))
        sig = {
            "orc_synth_f32": (None, [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, C.c_int, P]),
            "orc_quantize_q4": (C.c_int, [P, C.c_int64, C.c_int, P, P]),
            "orc_gemv_q26": (None, [P, C.c_int, P, P, C.c_int64, P]),
            "orc_model_create": (P, [C.c_int, C.c_int, C.c_int]),
            "orc_model_destroy": (None, [P]),
            "orc_model_set_tables": (None, [P, P, P, P, P]),
            "orc_model_init_synthetic": (C.c_int, [P, C.c_uint64, C.c_float, C.c_float]),
            "orc_layer_step": (None, [P, C.c_int, C.c_int, P]),
            "orc_run_token": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P]),
            "orc_decode": (C.c_int, [P, P, C.c_int, C.c_int, P, P]),
            "orc_read_hidden": (None, [P, P]),
            "orc_set_kv": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P]),
            "orc_get_kv": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P]),
            "orc_set_threads": (C.c_int, [C.c_int]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(P)


def set_threads(n: int = 0) -> int:
    return lib().orc_set_threads(n)


def synth_f32(seed, tid, n, std, bf16=True, start=0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_synth_f32(seed, tid, start, n, std, 1 if bf16 else 0, _p(out))
    return out


def quantize_q4(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    q = np.empty(w.shape, dtype=np.int8)
    s = np.empty((w.shape[0], w.shape[1] // 64), dtype=np.uint16)
    if lib().orc_quantize_q4(_p(w), w.shape[0], w.shape[1], _p(q), _p(s)):
        raise ValueError("Q4 scale does not fit unsigned 16-bit Q2.14")
    return q, s


def gemv_q26(act, q, s) -> np.ndarray:
    a = np.ascontiguousarray(act, dtype=np.int32)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    out = np.empty(q.shape[0], dtype=np.int64)
    lib().orc_gemv_q26(_p(a), q.shape[1], _p(q), _p(s), q.shape[0], _p(out))
    return out


class CModel:
    """Whole model in C: seeded synthetic weights, same tables as the GPU."""

    def __init__(self, n_layers: int, vocab: int, max_ctx: int, seed: int = 0, std: float = 0.02,
                 gamma_std: float = 0.0):
        self.L = lib()
        self.h = self.L.orc_model_create(n_layers, vocab, max_ctx)
        if not self.h:
            raise MemoryError("orc_model_create failed")
        cos, sin = O.rope_tables(max_ctx)
        self._tables = [np.ascontiguousarray(x, dtype=np.int32) for x in
                        (cos, sin, O.build_exp_lut(), O.build_sigmoid_lut())]
        self.L.orc_model_set_tables(self.h, *[_p(t) for t in self._tables])
        if self.L.orc_model_init_synthetic(self.h, seed, std, gamma_std):
            raise ValueError("Q4 scale overflow in synthetic init")
        self.max_ctx = max_ctx

    def close(self):
        if self.h:
            self.L.orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def run_token(self, token: int, pos: int, want_logits: bool = True) -> tuple[int, int]:
        t = np.zeros(1, dtype=np.int32)
        s = np.zeros(1, dtype=np.int64)
        if self.L.orc_run_token(self.h, token, pos, 1 if want_logits else 0, _p(t), _p(s)):
            raise ValueError("bad token or position")
        return int(t[0]), int(s[0])

    def hidden(self) -> np.ndarray:
        h = np.empty(1024, dtype=np.int32)
        self.L.orc_read_hidden(self.h, _p(h))
        return h.astype(np.int64)

    def layer_step(self, layer: int, pos: int, hidden) -> np.ndarray:
        h = np.ascontiguousarray(hidden, dtype=np.int32).copy()
        self.L.orc_layer_step(self.h, layer, pos, _p(h))
        return h.astype(np.int64)

    def set_kv(self, layer: int, kind: int, pos0: int, rows) -> None:
        """Load K (kind 0) or V (kind 1) rows [n, 8, 128] at positions pos0.. of a layer."""
        r = np.ascontiguousarray(rows, dtype=np.int32)
        if self.L.orc_set_kv(self.h, layer, kind, pos0, r.shape[0], _p(r)):
            raise ValueError("K/V rows out of range")

    def get_kv(self, layer: int, kind: int, pos0: int, n: int) -> np.ndarray:
        out = np.empty((n, 8, 128), dtype=np.int32)
        if self.L.orc_get_kv(self.h, layer, kind, pos0, n, _p(out)):
            raise ValueError("K/V rows out of range")
        return out

    def decode(self, prompt, max_new: int) -> tuple[list, list]:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        g = np.zeros(max_new, dtype=np.int32)
        s = np.zeros(max_new, dtype=np.int64)
        if self.L.orc_decode(self.h, _p(p), p.size, max_new, _p(g), _p(s)):
            raise ValueError("decode failed")
        return g.astype(np.int64).tolist(), s.tolist()
