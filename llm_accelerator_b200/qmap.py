"""QMAP v1 PL-DDR images: write the reference's runtime layout from a model's
tensors, read a segment bundle back into one arena, and bind it into a device
context through the C walker (q4gpu_qmap_bind / q4gpu_model_load_qmap).

Format: Source/QMAP_FORMAT.md (header :142-157, descriptor :193-214, enums
:216-263, per-packet slot tables :546-1814).  Physical layout of the deployed
full28 image: Qwen3-0.6B-Base/python_each_module/53_export_embedding_full28_final_chain.py:21-75
(bases, persistent offsets, body-stage offsets and sizes),
FPGA_Project/software/qmap_one_token_runtime/qmap_model_config_generated.h
(per-layer packet bases), lmdeploy/qwen3-0p6b-q4-qweb-demo/model/pl_ddr_binary_segments.json
(61 segments and their entries) and init/q4_runtime_assets.json (aperture
0x4_0000_0000 .. 0x4_2000_0000).

The writer emits one packet per layer stage at the reference's addresses with
the documented descriptors (slot s holds tensor id s + 1); scratch and debug
payloads the GPU path does not read are left zero.  The reader accepts any
image with that layout, including the reference's own segments.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import _native

APERTURE_BASE = 0x4_0000_0000
APERTURE_END = 0x4_2000_0000
TIED_WEIGHT_BASE = 0x4_0010_0000
TIED_SCALE_BASE = 0x4_04B3_0000
LAYER_BLOCK_BASE = 0x4_0500_0000
LAYER_BLOCK_STRIDE = 0x84_0000
BODY_QMAP_BASE = 0x4_1790_0000
BODY_QMAP_STRIDE = 0x10_0000
KV_CACHE_BASE = 0x4_1410_0000
FINAL_TAIL_QMAP_BASE = 0x4_1950_0000
HIDDEN_A_BASE = 0x4_1960_0000
HIDDEN_B_BASE = 0x4_1960_1000
ROPE_TABLE_BASE = 0x4_1A10_0000
ROPE_POSITIONS = 256  # MAX_CONTEXT of the reference runtime
ROPE_PLANE_BYTES = ROPE_POSITIONS * 128 * 4
KV_BYTES_PER_LAYER = 2 * 8 * ROPE_POSITIONS * 128 * 4
QKV_IMAGE_BYTES = 0x22_B000
FINAL_TAIL_BYTES = 0x4000
PERSISTENT_OFFSETS = {  # inside a layer block, after the QKV packet
    "o_proj_weight": 0x23_0000, "o_proj_scale": 0x33_0000,
    "mlp_gate_weight": 0x34_0000, "mlp_gate_scale": 0x4C_0000,
    "mlp_up_weight": 0x4E_0000, "mlp_up_scale": 0x66_0000,
    "mlp_down_weight": 0x68_0000, "mlp_down_scale": 0x80_0000,
}
LAYER_BLOCK_BYTES = 0x80_0000 + 1024 * 96  # through the down scales
# body packets: (offset in the layer's body window, image bytes, descriptor capacity)
BODY_STAGES = {
    "attn_frontend": (0x2_0000, 0x7000, 16), "attn_score_value": (0x3_0000, 0x5000, 8),
    "o_proj": (0x4_0000, 0x5000, 8), "post_attn_norm": (0x5_0000, 0x8000, 8),
    "mlp_gate_up": (0x6_0000, 0xE000, 16), "mlp_silu_mul": (0x7_0000, 0xE000, 8),
    "mlp_down": (0x8_0000, 0x6000, 8), "mlp_residual_add": (0x9_0000, 0x5000, 8),
    "input_rmsnorm": (0xA_0000, 0x5000, 8),
}
# qot_layer_qmap_bases_t field order (qmap_one_token_runtime.h:31-42)
BASE_FIELDS = ("qkv", "input_rmsnorm", "attn_frontend", "attn_score_value", "o_proj", "post_attn_norm",
               "mlp_gate_up", "mlp_silu_mul", "mlp_down", "mlp_residual_add")

MAGIC = 0x50414D51
# roles, dtypes, flags, matrix ids (QMAP_FORMAT.md:216-297)
R_ACT, R_WEIGHT, R_SCALE, R_OUTPUT, R_EXPECTED, R_META, R_KV, R_ROPE, R_PARAM = range(1, 10)
DT_U32, DT_I32, DT_PACKED_Q4, DT_U16_Q2_14 = 5, 6, 16, 17
DT_I32_Q12_12, DT_I32_Q14_10, DT_I16_Q8_7, DT_I16_Q1_15, DT_U32_Q0_20, DT_U16_Q0_16 = 19, 20, 22, 23, 24, 25
F_ROW_MAJOR, F_PACKED_LOW_EVEN, F_READ_ONLY, F_WRITE_ONLY, F_DEBUG_ONLY = 1, 2, 4, 8, 16
M_Q, M_K, M_V, M_O, M_GATE, M_UP, M_DOWN, M_EMBED = range(1, 9)
NO_TENSOR = 0xFFFF_FFFF
SCORE_SCALE_Q0_31 = 189812531
RO = F_ROW_MAJOR | F_READ_ONLY
WO = F_ROW_MAJOR | F_WRITE_ONLY
Q4_FLAGS = F_ROW_MAJOR | F_PACKED_LOW_EVEN | F_READ_ONLY

_HEADER = struct.Struct("<IIIIIIQQQQII")
_DESC = struct.Struct("<8I2Q4I4Q8I")


def layer_bases(layer: int) -> tuple[int, ...]:
    """The ten qot_layer_qmap_bases_t addresses of `layer`."""
    body = BODY_QMAP_BASE + layer * BODY_QMAP_STRIDE
    return (LAYER_BLOCK_BASE + layer * LAYER_BLOCK_STRIDE,) + tuple(body + BODY_STAGES[n][0] for n in BASE_FIELDS[1:])


class _Packet:
    """One QMAP image: 256-byte header, descriptor table at +0x100, payloads."""

    def __init__(self, base: int, image_bytes: int, capacity: int):
        self.base, self.size, self.capacity = base, image_bytes, capacity
        self.payload_base = 0x100 + capacity * 128
        self.cursor = self.payload_base
        self.chunks: list[tuple[int, bytes]] = []
        self.descs: list[bytes] = []

    def payload(self, data: bytes | int, align: int = 64) -> int:
        """Place bytes (or reserve that many zero bytes); returns the address."""
        n = data if isinstance(data, int) else len(data)
        off = (self.cursor + align - 1) // align * align
        if off + n > self.size:
            raise ValueError(f"QMAP packet at {self.base:#x} overflows its {self.size:#x} bytes")
        if not isinstance(data, int):
            self.chunks.append((off, bytes(data)))
        self.cursor = off + n
        return self.base + off

    def add(self, role: int, dtype: int, dims, strides, base_addr: int, nbytes: int, element_bits: int, flags: int,
            aux=(0, 0, 0, 0), scale_tensor_id: int = NO_TENSOR) -> int:
        if len(self.descs) >= self.capacity:
            raise ValueError("QMAP descriptor capacity exceeded")
        tid = len(self.descs) + 1
        dims = tuple(dims) + (0,) * (4 - len(dims))
        strides = tuple(strides) + (0,) * (4 - len(strides))
        rank = sum(1 for d in dims if d)
        self.descs.append(_DESC.pack(tid, role, dtype, rank, flags, element_bits, 0 if role != R_WEIGHT else 64,
                                     scale_tensor_id, base_addr, nbytes, *dims, *strides, *aux, 0, 0, 0, 0))
        return tid

    def image(self) -> bytes:
        out = bytearray(self.size)
        hdr = _HEADER.pack(MAGIC, 1, 256, 128, len(self.descs), self.capacity, self.base + 0x100,
                           self.base + self.payload_base, self.base, self.size, 0, 0)
        out[0:len(hdr)] = hdr
        for i, d in enumerate(self.descs):
            out[0x100 + 128 * i:0x100 + 128 * (i + 1)] = d
        for off, data in self.chunks:
            out[off:off + len(data)] = data
        return bytes(out)


def _words(values, dtype="<i4") -> bytes:
    return np.ascontiguousarray(values).astype(dtype).tobytes()


def _vec(p: _Packet, n: int, dtype: int, role: int, flags: int, aux, addr: int | None = None) -> int:
    """A [n] 32-bit-word vector descriptor; reserves a zero payload unless
    `addr` points elsewhere.  Returns the vector's address."""
    a = p.payload(4 * n) if addr is None else addr
    bits = 24 if dtype in (DT_I32_Q12_12, DT_I32_Q14_10) else 32
    p.add(role, dtype, (n,), (4,), a, 4 * n, bits, flags, aux)
    return a


def _param(p: _Packet, dtype: int, values, word: str, bits: int, aux) -> int:
    """A read-only parameter vector stored one value per 32-bit word."""
    data = _words(values, word)
    return p.add(R_PARAM, dtype, (len(values),), (4,), p.payload(data), len(data), bits, RO, aux)


@dataclass
class ModelTensors:
    """Everything a QMAP image carries: Q4 weights as (packed uint8 [rows,
    cols/2], uint16 scales [rows, cols/64]) per layer and Q4GPU_T_* id, gammas
    int32 (Q8.7), the tied embedding, RoPE planes int32 [256, 128] (Q1.15), the
    exp LUT int32 [257] (UQ0.20) and the sigmoid LUT int32 [1025] (UQ0.16)."""
    n_layers: int
    weights: dict = field(default_factory=dict)   # (layer, which) -> (packed, scale)
    gammas: dict = field(default_factory=dict)    # (layer, which) -> int32
    embed: tuple | None = None
    final_gamma: np.ndarray | None = None
    rope_cos: np.ndarray | None = None
    rope_sin: np.ndarray | None = None
    exp_lut: np.ndarray | None = None
    sig_lut: np.ndarray | None = None

    @property
    def vocab(self) -> int:
        return int(self.embed[0].shape[0])


def tensors_from_model(m) -> ModelTensors:
    """Read every tensor of a device context (Q4Model) back to the host."""
    from . import tables

    t = ModelTensors(n_layers=m.n_layers)
    for layer in range(m.n_layers):
        for which in range(_native.T_Q, _native.T_DOWN + 1):
            t.weights[(layer, which)] = m.get_weight(layer, which)
        for which in range(_native.T_INPUT_GAMMA, _native.T_K_GAMMA + 1):
            t.gammas[(layer, which)] = m.get_gamma(layer, which)
    t.embed = m.get_weight(0, _native.T_EMBED)
    t.final_gamma = m.get_gamma(0, _native.T_FINAL_GAMMA)
    cos, sin = tables.rope_tables(max(ROPE_POSITIONS, m.max_context))
    t.rope_cos, t.rope_sin = cos[:ROPE_POSITIONS], sin[:ROPE_POSITIONS]
    t.exp_lut, t.sig_lut = tables.luts()
    return t


@dataclass
class Segment:
    index: int
    address: int
    nbytes: int
    data: bytes | None                     # None: a zero-initialised region (no file)
    entries: list = field(default_factory=list)  # (name, operation, address, nbytes)


def _layer_block(t: ModelTensors, layer: int, norm_out: int) -> tuple[bytes, list, tuple[int, int, int]]:
    """The layer's block: the self-contained QKV packet (QMAP_FORMAT.md:621-660;
    32 descriptor slots, payload at +0x1100) then the persistent o / gate / up /
    down weights and scales.  Returns (bytes, segment entries, q/k/v output
    addresses)."""
    base = LAYER_BLOCK_BASE + layer * LAYER_BLOCK_STRIDE
    p = _Packet(base, QKV_IMAGE_BYTES, 32)
    p.add(R_META, DT_U32, (16,), (4,), p.payload(64), 64, 32, RO, (0, layer, 0, 0))
    _vec(p, 1024, DT_I32_Q12_12, R_ACT, RO, (0, layer, 0, 0), norm_out)
    for mat, which, rows in ((M_Q, _native.T_Q, 2048), (M_K, _native.T_K, 1024), (M_V, _native.T_V, 1024)):
        w, s = t.weights[(layer, which)]
        wa, sa = p.payload(w.tobytes()), p.payload(s.astype("<u2").tobytes())
        sid = len(p.descs) + 2
        p.add(R_WEIGHT, DT_PACKED_Q4, (rows, 1024), (512, 0), wa, w.nbytes, 4, Q4_FLAGS, (mat, layer, 0, 0), sid)
        p.add(R_SCALE, DT_U16_Q2_14, (rows, 16), (32, 2), sa, s.nbytes, 16, RO, (mat, layer, 0, 0))
    outs = tuple(_vec(p, rows, DT_I32_Q12_12, R_OUTPUT, WO, (mat, layer, 0, 0))
                 for mat, rows in ((M_Q, 2048), (M_K, 1024), (M_V, 1024)))
    img = bytearray(LAYER_BLOCK_BYTES)
    img[0:QKV_IMAGE_BYTES] = p.image()
    entries = [(f"layer{layer}.qkv_qmap", "file", base, QKV_IMAGE_BYTES)]
    for name, which, in (("o_proj", _native.T_O), ("mlp_gate", _native.T_GATE), ("mlp_up", _native.T_UP),
                         ("mlp_down", _native.T_DOWN)):
        w, s = t.weights[(layer, which)]
        for kind, arr in (("weight", w), ("scale", s.astype("<u2"))):
            off = PERSISTENT_OFFSETS[f"{name}_{kind}"]
            img[off:off + arr.nbytes] = arr.tobytes()
            entries.append((f"layer{layer}.{name}_{kind}", "file", base + off, arr.nbytes))
    return bytes(img), entries, outs


def _body_packets(t: ModelTensors, layer: int) -> tuple[dict[str, bytes], int]:
    """The nine per-layer body packets, each at the reference's address with
    the documented descriptor slots, chained through their buffers; returns
    (images by stage, the input-norm output address the QKV packet reads)."""
    body = BODY_QMAP_BASE + layer * BODY_QMAP_STRIDE
    block = LAYER_BLOCK_BASE + layer * LAYER_BLOCK_STRIDE
    kv = KV_CACHE_BASE + layer * KV_BYTES_PER_LAYER
    g = t.gammas
    pk = {n: _Packet(body + off, size, cap) for n, (off, size, cap) in BODY_STAGES.items()}

    def meta(p, aux):
        p.add(R_META, DT_U32, (16,), (4,), p.payload(64), 64, 32, RO, aux)

    def q4(p, mat, which, rows, cols, key):
        w, s = t.weights[(layer, which)]
        sid = len(p.descs) + 2
        aux = (mat, layer, 0, rows)
        p.add(R_WEIGHT, DT_PACKED_Q4, (rows, cols), (cols // 2, 0), block + PERSISTENT_OFFSETS[key + "_weight"],
              w.nbytes, 4, Q4_FLAGS, aux, sid)
        p.add(R_SCALE, DT_U16_Q2_14, (rows, cols // 64), (cols // 32, 2), block + PERSISTENT_OFFSETS[key + "_scale"],
              s.nbytes, 16, RO, aux)

    def kv_desc(p, flags):
        p.add(R_KV, DT_I32_Q12_12, (2, 8, ROPE_POSITIONS, 128), (KV_BYTES_PER_LAYER // 2, ROPE_POSITIONS * 512, 512, 4),
              kv, KV_BYTES_PER_LAYER, 24, flags, (0, layer, 0, 0))

    # input RMSNorm (QMAP_FORMAT.md:546-575): hidden, gamma, norm out
    p = pk["input_rmsnorm"]
    meta(p, (6, layer, 1024, 0))
    _vec(p, 1024, DT_I32_Q14_10, R_ACT, RO, (6, layer, 1024, 0), HIDDEN_A_BASE)
    _param(p, DT_I16_Q8_7, g[(layer, _native.T_INPUT_GAMMA)], "<i4", 16, (6, layer, 1024, 0))
    norm_out = _vec(p, 1024, DT_I32_Q12_12, R_OUTPUT, WO, (6, layer, 1024, 0))
    # attention front-end (:748-800): q/k/v in, q_norm and k_norm gamma, the
    # runtime RoPE table, the layer's KV cache, q RoPE out
    p = pk["attn_frontend"]
    meta(p, (0, layer, 0, 0))
    qkv_in = [_vec(p, rows, DT_I32_Q12_12, R_ACT, RO, (mat, layer, 0, 0), 0)
              for mat, rows in ((M_Q, 2048), (M_K, 1024), (M_V, 1024))]
    del qkv_in  # patched once the QKV packet's output addresses are known
    for which in (_native.T_Q_GAMMA, _native.T_K_GAMMA):
        _param(p, DT_I16_Q8_7, g[(layer, which)], "<i4", 16, (0, layer, 0, 0))
    for plane in range(2):
        p.add(R_ROPE, DT_I16_Q1_15, (ROPE_POSITIONS, 128), (512, 4), ROPE_TABLE_BASE + plane * ROPE_PLANE_BYTES,
              ROPE_PLANE_BYTES, 16, RO, (0, layer, 0, 0))
    kv_desc(p, F_ROW_MAJOR)
    q_rope = _vec(p, 2048, DT_I32_Q12_12, R_OUTPUT, WO, (0, layer, 0, 0))
    # attention score/value (:811-845)
    p = pk["attn_score_value"]
    meta(p, (SCORE_SCALE_Q0_31, layer, 0, 0))
    _vec(p, 2048, DT_I32_Q12_12, R_ACT, RO, (0, layer, 0, 0), q_rope)
    kv_desc(p, RO)
    _param(p, DT_U32_Q0_20, t.exp_lut, "<u4", 20, (0, layer, 0, 0))
    attn_out = _vec(p, 2048, DT_I32_Q12_12, R_OUTPUT, WO, (0, layer, 0, 0))
    # o_proj (:866-880)
    p = pk["o_proj"]
    meta(p, (M_O, layer, 1024, 2048))
    _vec(p, 2048, DT_I32_Q12_12, R_ACT, RO, (M_O, layer, 0, 0), attn_out)
    q4(p, M_O, _native.T_O, 1024, 2048, "o_proj")
    o_out = _vec(p, 1024, DT_I32_Q12_12, R_OUTPUT, WO, (M_O, layer, 0, 1024))
    # post-attention residual / RMSNorm (:938-960)
    p = pk["post_attn_norm"]
    meta(p, (1, layer, 1024, 0))
    _vec(p, 1024, DT_I32_Q14_10, R_ACT, RO, (1, layer, 1024, 0), HIDDEN_A_BASE)
    _vec(p, 1024, DT_I32_Q12_12, R_ACT, RO, (M_O, layer, 0, 0), o_out)
    _param(p, DT_I16_Q8_7, g[(layer, _native.T_POST_GAMMA)], "<i4", 16, (1, layer, 1024, 0))
    post_hidden = _vec(p, 1024, DT_I32_Q14_10, R_OUTPUT, WO, (1, layer, 1024, 0))
    post_norm = _vec(p, 1024, DT_I32_Q12_12, R_OUTPUT, WO, (1, layer, 1024, 0))
    # MLP gate/up (:1001-1020)
    p = pk["mlp_gate_up"]
    meta(p, (2, layer, 3072, 1024))
    _vec(p, 1024, DT_I32_Q12_12, R_ACT, RO, (2, layer, 3072, 1024), post_norm)
    q4(p, M_GATE, _native.T_GATE, 3072, 1024, "mlp_gate")
    q4(p, M_UP, _native.T_UP, 3072, 1024, "mlp_up")
    gate_out = _vec(p, 3072, DT_I32_Q12_12, R_OUTPUT, WO, (M_GATE, layer, 0, 0))
    up_out = _vec(p, 3072, DT_I32_Q12_12, R_OUTPUT, WO, (M_UP, layer, 0, 0))
    # SiLU / multiply (:1087-1100)
    p = pk["mlp_silu_mul"]
    meta(p, (3, layer, 3072, 1025))
    _vec(p, 3072, DT_I32_Q12_12, R_ACT, RO, (3, layer, 3072, 1025), gate_out)
    _vec(p, 3072, DT_I32_Q12_12, R_ACT, RO, (3, layer, 3072, 1025), up_out)
    _param(p, DT_U16_Q0_16, t.sig_lut, "<u4", 16, (3, layer, 3072, 1025))
    mlp_hidden = _vec(p, 3072, DT_I32_Q12_12, R_OUTPUT, WO, (3, layer, 3072, 1025))
    # MLP down (:1147-1160)
    p = pk["mlp_down"]
    meta(p, (4, layer, 1024, 3072))
    _vec(p, 3072, DT_I32_Q12_12, R_ACT, RO, (4, layer, 1024, 3072), mlp_hidden)
    q4(p, M_DOWN, _native.T_DOWN, 1024, 3072, "mlp_down")
    down_out = _vec(p, 1024, DT_I32_Q12_12, R_OUTPUT, WO, (M_DOWN, layer, 0, 1024))
    # final MLP residual (:1219-1230)
    p = pk["mlp_residual_add"]
    meta(p, (5, layer, 1024, 0))
    _vec(p, 1024, DT_I32_Q14_10, R_ACT, RO, (5, layer, 1024, 0), post_hidden)
    _vec(p, 1024, DT_I32_Q12_12, R_ACT, RO, (M_DOWN, layer, 0, 0), down_out)
    _vec(p, 1024, DT_I32_Q14_10, R_OUTPUT, WO, (5, layer, 1024, 0), HIDDEN_B_BASE)
    return pk, norm_out


def _patch_frontend_inputs(p: _Packet, qkv_out: tuple[int, int, int]) -> None:
    """Point the front-end's q/k/v descriptors (slots 1..3) at the QKV outputs."""
    for slot, addr in zip((1, 2, 3), qkv_out):
        d = bytearray(p.descs[slot])
        struct.pack_into("<Q", d, 32, addr)
        p.descs[slot] = bytes(d)


def _final_tail(t: ModelTensors) -> bytes:
    vocab = t.vocab
    p = _Packet(FINAL_TAIL_QMAP_BASE, FINAL_TAIL_BYTES, 8)
    tiles = (vocab + 15) // 16
    aux = (M_EMBED, 0, 0, tiles)
    p.add(R_META, DT_U32, (16,), (4,), p.payload(64), 64, 32, RO, aux)
    _vec(p, 1024, DT_I32_Q12_12, R_ACT, F_ROW_MAJOR, (M_EMBED, 0, 0, 0))
    p.add(R_WEIGHT, DT_PACKED_Q4, (vocab, 1024), (512, 0), TIED_WEIGHT_BASE, vocab * 512, 4, Q4_FLAGS, aux, 4)
    p.add(R_SCALE, DT_U16_Q2_14, (vocab, 16), (32, 2), TIED_SCALE_BASE, vocab * 32, 16, RO, aux)
    p.add(R_OUTPUT, DT_U32, (3,), (4,), p.payload(12), 12, 32, WO, aux)
    _vec(p, 1024, DT_I32_Q14_10, R_ACT, RO, (0, 0, 0, 0), HIDDEN_B_BASE)
    _param(p, DT_I16_Q8_7, t.final_gamma, "<i4", 16, (0, 0, 0, 0))
    return p.image()


_BODY_ORDER = ("attn_frontend", "attn_score_value", "o_proj", "post_attn_norm", "mlp_gate_up", "mlp_silu_mul",
               "mlp_down", "mlp_residual_add", "input_rmsnorm")
_BODY_LO = min(BODY_STAGES[n][0] for n in _BODY_ORDER)
_BODY_HI = max(BODY_STAGES[n][0] + BODY_STAGES[n][1] for n in _BODY_ORDER)


def segment_plan(n_layers: int, vocab: int) -> list[Segment]:
    """Addresses, sizes and entries of the image's segments, without data:
    for 28 layers and the full vocabulary this is the reference's 61-segment
    plan (pl_ddr_binary_segments.json)."""
    if vocab * 512 > TIED_SCALE_BASE - TIED_WEIGHT_BASE:
        raise ValueError("vocabulary too large for the tied-embedding region")
    segs: list[Segment] = []

    def add(address, nbytes, zero, entries):
        segs.append(Segment(len(segs), address, nbytes, None if zero else b"", entries))

    add(TIED_WEIGHT_BASE, TIED_SCALE_BASE - TIED_WEIGHT_BASE + vocab * 32, False,
        [("tied_embedding_weight", "file", TIED_WEIGHT_BASE, vocab * 512),
         ("tied_embedding_scale", "file", TIED_SCALE_BASE, vocab * 32)])
    sizes = {"o_proj_weight": 1024 * 1024, "o_proj_scale": 1024 * 64, "mlp_gate_weight": 3072 * 512,
             "mlp_gate_scale": 3072 * 32, "mlp_up_weight": 3072 * 512, "mlp_up_scale": 3072 * 32,
             "mlp_down_weight": 1024 * 1536, "mlp_down_scale": 1024 * 96}
    for layer in range(n_layers):
        base = LAYER_BLOCK_BASE + layer * LAYER_BLOCK_STRIDE
        add(base, LAYER_BLOCK_BYTES, False, [(f"layer{layer}.qkv_qmap", "file", base, QKV_IMAGE_BYTES)] +
            [(f"layer{layer}.{k}", "file", base + PERSISTENT_OFFSETS[k], sizes[k]) for k in PERSISTENT_OFFSETS])
    add(KV_CACHE_BASE, n_layers * KV_BYTES_PER_LAYER, True,
        [("kv_cache", "zero", KV_CACHE_BASE, n_layers * KV_BYTES_PER_LAYER)])
    for layer in range(n_layers):
        body = BODY_QMAP_BASE + layer * BODY_QMAP_STRIDE
        add(body + _BODY_LO, _BODY_HI - _BODY_LO, False,
            [(f"layer{layer}.{n}_qmap", "file", body + BODY_STAGES[n][0], BODY_STAGES[n][1]) for n in _BODY_ORDER])
    add(FINAL_TAIL_QMAP_BASE, FINAL_TAIL_BYTES, False, [("final_tail_qmap", "file", FINAL_TAIL_QMAP_BASE,
                                                          FINAL_TAIL_BYTES)])
    add(HIDDEN_A_BASE, HIDDEN_B_BASE + 4096 - HIDDEN_A_BASE, True,
        [("runtime_hidden_a", "zero", HIDDEN_A_BASE, 4096), ("runtime_hidden_b", "zero", HIDDEN_B_BASE, 4096)])
    add(ROPE_TABLE_BASE, 2 * ROPE_PLANE_BYTES, False,
        [("runtime_rope_table", "file", ROPE_TABLE_BASE, 2 * ROPE_PLANE_BYTES)])
    return segs


def build_segments(t: ModelTensors) -> list[Segment]:
    """The image of `t` on segment_plan(t.n_layers, t.vocab): each file
    segment's bytes (packets, weights, tables; gaps zero)."""
    plan = segment_plan(t.n_layers, t.vocab)
    blobs: dict[int, bytes] = {}
    w, s = t.embed
    emb = bytearray(plan[0].nbytes)
    emb[0:w.nbytes] = w.tobytes()
    emb[TIED_SCALE_BASE - TIED_WEIGHT_BASE:] = s.astype("<u2").tobytes()
    blobs[0] = bytes(emb)
    bodies = []
    for layer in range(t.n_layers):
        packets, norm_out = _body_packets(t, layer)
        data, entries, qkv_out = _layer_block(t, layer, norm_out)
        _patch_frontend_inputs(packets["attn_frontend"], qkv_out)
        bodies.append(packets)
        blobs[1 + layer] = data
    for layer in range(t.n_layers):
        win = bytearray(_BODY_HI - _BODY_LO)
        for n in _BODY_ORDER:
            off, size, _ = BODY_STAGES[n]
            win[off - _BODY_LO:off - _BODY_LO + size] = bodies[layer][n].image()
        blobs[2 + t.n_layers + layer] = bytes(win)
    blobs[2 + 2 * t.n_layers] = _final_tail(t)
    rope = np.concatenate([np.asarray(t.rope_cos, np.int32)[:ROPE_POSITIONS].reshape(-1),
                           np.asarray(t.rope_sin, np.int32)[:ROPE_POSITIONS].reshape(-1)])
    blobs[4 + 2 * t.n_layers] = _words(rope)
    for sg in plan:
        if sg.data is not None:
            sg.data = blobs[sg.index]
            if len(sg.data) != sg.nbytes:
                raise AssertionError(f"segment {sg.index}: {len(sg.data)} bytes, plan {sg.nbytes}")
    return plan


def write_bundle(segs: list[Segment], out_dir: str | Path) -> Path:
    """Segment files qwen3_runtime_NN.bin plus pl_ddr_binary_segments.json in
    the reference's manifest schema; returns the manifest path."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    rows = []
    for sg in segs:
        fname = f"qwen3_runtime_{sg.index:02d}.bin"
        row = {"index": sg.index, "file": fname, "address": sg.address, "address_hex": f"0x{sg.address:016X}",
               "nbytes": sg.nbytes,
               "entries": [{"name": n, "operation": op, "address": a, "nbytes": b} for n, op, a, b in sg.entries]}
        if sg.data is not None:
            (out / fname).write_bytes(sg.data)
            row["sha256"] = hashlib.sha256(sg.data).hexdigest()
        else:
            row["file"] = None
        rows.append(row)
    manifest = {"format_version": 1, "name": "qwen3_0p6b_pl_ddr_binary_segments", "segment_count": len(rows),
                "total_segment_bytes": sum(r["nbytes"] for r in rows), "segments": rows}
    path = out / "pl_ddr_binary_segments.json"
    path.write_text(json.dumps(manifest, indent=2))
    return path


def load_bundle(manifest_path: str | Path, verify_sha256: bool = True) -> tuple[np.ndarray, int]:
    """Read a segment bundle into one zero-initialised arena spanning the
    aperture up to the highest segment end; returns (arena, arena_base).
    Checks aperture bounds, non-overlap, file sizes and (optionally) SHA-256;
    `zero` entries stay zero."""
    mpath = Path(manifest_path)
    man = json.loads(mpath.read_text())
    segs = man["segments"]
    if len(segs) != man.get("segment_count", len(segs)):
        raise ValueError("segment_count does not match the segment list")
    spans = sorted((int(s["address"]), int(s["address"]) + int(s["nbytes"])) for s in segs)
    for (a0, a1), (b0, _) in zip(spans, spans[1:]):
        if b0 < a1:
            raise ValueError(f"segments overlap at {b0:#x}")
    if spans[0][0] < APERTURE_BASE or spans[-1][1] > APERTURE_END:
        raise ValueError("a segment leaves the PL-DDR aperture")
    arena = np.zeros(spans[-1][1] - APERTURE_BASE, dtype=np.uint8)
    for s in segs:
        addr, n = int(s["address"]), int(s["nbytes"])
        file_ops = [e for e in s.get("entries", []) if e.get("operation") == "file"]
        if not s.get("file") or not file_ops:
            continue
        data = (mpath.parent / s["file"]).read_bytes()
        if len(data) != n:
            raise ValueError(f"{s['file']}: {len(data)} bytes, manifest says {n}")
        if verify_sha256 and s.get("sha256") and hashlib.sha256(data).hexdigest() != s["sha256"]:
            raise ValueError(f"{s['file']}: SHA-256 mismatch")
        arena[addr - APERTURE_BASE:addr - APERTURE_BASE + n] = np.frombuffer(data, dtype=np.uint8)
    return arena, APERTURE_BASE


class Layout:
    """q4gpu_qmap_layout of the reference's layout for n_layers layers."""

    def __init__(self, n_layers: int, arena_base: int = APERTURE_BASE, bases=None):
        rows = bases if bases is not None else [layer_bases(i) for i in range(n_layers)]
        self._bases = (C.c_uint64 * (10 * n_layers))(*[int(x) for r in rows for x in r])
        self.struct = _native.QmapLayout(arena_base, FINAL_TAIL_QMAP_BASE, ROPE_TABLE_BASE,
                                         ROPE_TABLE_BASE + ROPE_PLANE_BYTES, TIED_WEIGHT_BASE, TIED_SCALE_BASE,
                                         n_layers, 0, C.cast(self._bases, C.POINTER(C.c_uint64)))


def read_packet(arena: np.ndarray, arena_base: int, addr: int) -> tuple[dict, list[dict]]:
    """Header and descriptors of the packet at `addr` (decoded by the C walker)."""
    lib = _native.load()
    h = _native.QmapHeader()
    d = (_native.QmapDescriptor * 4096)()
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    n = lib.q4gpu_qmap_read_packet(arena.ctypes.data, arena_base, arena.nbytes, addr, C.byref(h), d, 4096)
    if n < 0:
        _native.check(n, "q4gpu_qmap_read_packet")
    hdr = {f: getattr(h, f) for f, _ in _native.QmapHeader._fields_}
    descs = []
    for i in range(n):
        x = d[i]
        descs.append({f: (list(getattr(x, f)) if f in ("dims", "strides_bytes", "aux", "reserved") else getattr(x, f))
                      for f, _ in _native.QmapDescriptor._fields_})
    return hdr, descs


def bind(arena: np.ndarray, layout: Layout) -> list:
    """The bound tensors (q4gpu_qmap_tensor) of an image."""
    lib = _native.load()
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    n = C.c_int32(0)
    _native.check(lib.q4gpu_qmap_bind(arena.ctypes.data, arena.nbytes, C.byref(layout.struct), None, 0, C.byref(n)),
                  "q4gpu_qmap_bind")
    out = (_native.QmapTensor * n.value)()
    _native.check(lib.q4gpu_qmap_bind(arena.ctypes.data, arena.nbytes, C.byref(layout.struct), out, n.value,
                                      C.byref(n)), "q4gpu_qmap_bind")
    return list(out)


def vector(arena: np.ndarray, t) -> np.ndarray:
    """A bound vector tensor as int32 values."""
    lib = _native.load()
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    count = t.data_bytes // t.elem_stride
    v = np.empty(count, dtype=np.int32)
    _native.check(lib.q4gpu_qmap_vector(arena.ctypes.data, C.byref(t), v.ctypes.data, count), "q4gpu_qmap_vector")
    return v


def load_into_model(m, arena: np.ndarray, layout: Layout | None = None) -> None:
    """Upload every tensor of the image into the context `m` (Q4Model)."""
    lay = layout or Layout(m.n_layers)
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    _native.check(m.lib.q4gpu_model_load_qmap(m.handle, arena.ctypes.data, arena.nbytes, C.byref(lay.struct)),
                  "q4gpu_model_load_qmap")
