"""Host-built tables of the fixed-point path: RoPE cos/sin in Q1.15, the
softmax exp LUT and the SwiGLU sigmoid LUT.

The RoPE table is built the way the reference builds it: HF's default
inverse frequencies (float32), ``freqs = inv_freq @ positions`` and
``cos/sin`` in float32 torch (``Qwen3-0.6B-Base/python_each_module/common.py:155-170``),
then ``rint(x * 2^15)`` clipped to signed 16 bit
(``22_export_qk_norm_rope_fixed_vectors.py:75-83`` as called at
``56_export_persistent_multitoken_layer_golden.py:942-956``).  The device
never evaluates trigonometry; both LUTs come from the library's host
builder (``q4gpu_build_tables``).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _native

ROPE_THETA = 1.0e6
HEAD_DIM = 128


def rope_inv_freq(theta: float = ROPE_THETA, dim: int = HEAD_DIM) -> torch.Tensor:
    """HF Qwen3 default-RoPE inverse frequencies (float32)."""
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))


def rope_tables(n_positions: int, theta: float = ROPE_THETA) -> tuple[np.ndarray, np.ndarray]:
    """int32 [n_positions, 128] cos and sin in Q1.15."""
    inv = rope_inv_freq(theta)
    pos = torch.arange(n_positions, dtype=torch.long).float()
    # the reference forms freqs with a k=1 float32 matmul (one rounding per
    # product); an elementwise float32 product is that same rounding without
    # depending on which BLAS path the matmul takes
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)

    def q115(t: torch.Tensor) -> np.ndarray:
        v = np.rint(t.numpy().astype(np.float64) * 32768.0)
        return np.clip(v, -32768, 32767).astype(np.int32)

    return q115(emb.cos()), q115(emb.sin())


def luts() -> tuple[np.ndarray, np.ndarray]:
    """(exp LUT int32[257], sigmoid LUT int32[1025])."""
    e = np.zeros(257, dtype=np.int32)
    s = np.zeros(1025, dtype=np.int32)
    _native.load().q4gpu_build_tables(e.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p))
    return e, s
