"""Build tests/golden/qmap_ref.npz from the reference project tree.

    python tests/golden/make_qmap_golden.py --reference <reference project root>

Contents (nothing at test time reads the reference tree):

* ``pkt_<name>``: real QMAP v1 runtime packets exported by the reference
  (``FPGA_Project/sim/vectors/qmap_*_image_words32.hex``, little-endian 32-bit
  words) - Layer 1 chained body packets, the compact Layer 1 QKV packet and
  the compact final-token tail - as uint8 images;
* companions of those packets from the same vector set: the input and
  post-attention RMSNorm gammas, q/k norm gammas and RoPE cos/sin rows, the
  softmax exp LUT, the sigmoid LUT (``*_stage_real_*.hex``) and the final
  RMSNorm gamma;
* the deployed 61-segment PL-DDR plan of
  ``lmdeploy/qwen3-0p6b-q4-qweb-demo/model/pl_ddr_binary_segments.json``:
  per segment its address and size, per entry its segment, name, operation,
  address and size.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
VEC = "FPGA_Project/sim/vectors"
PACKETS = {
    "input_rmsnorm": "qmap_layer1_chained_input_rmsnorm_image_words32.hex",
    "attn_frontend": "qmap_layer1_chained_attention_frontend_image_words32.hex",
    "attn_score_value": "qmap_layer1_chained_attention_score_value_image_words32.hex",
    "o_proj": "qmap_layer1_chained_o_proj_image_words32.hex",
    "post_attn_norm": "qmap_layer1_chained_post_attention_residual_norm_image_words32.hex",
    "mlp_gate_up": "qmap_layer1_chained_mlp_gate_up_image_words32.hex",
    "mlp_silu_mul": "qmap_layer1_chained_mlp_silu_mul_image_words32.hex",
    "mlp_down": "qmap_layer1_chained_mlp_down_image_words32.hex",
    "mlp_residual_add": "qmap_layer1_chained_mlp_residual_add_image_words32.hex",
    "qkv": "qmap_layer1_qkv_projection_image_words32.hex",
    "final_tail": "qmap_final_token_tail_compact_image_words32.hex",
}
# (key, file, bits, signed)
COMPANIONS = [
    ("input_gamma", "layer1_chained_input_rmsnorm_stage_real_gamma.hex", 16, True),
    ("post_gamma", "layer1_chained_post_attention_residual_norm_stage_real_gamma.hex", 16, True),
    ("q_gamma", "layer1_chained_qk_norm_rope_stage_128_real_q_gamma.hex", 16, True),
    ("k_gamma", "layer1_chained_qk_norm_rope_stage_128_real_k_gamma.hex", 16, True),
    ("rope_cos", "layer1_chained_qk_norm_rope_stage_128_real_cos.hex", 16, True),
    ("rope_sin", "layer1_chained_qk_norm_rope_stage_128_real_sin.hex", 16, True),
    ("exp_lut", "layer1_chained_attention_softmax_value_stage_real_exp_lut.hex", 32, False),
    ("sigmoid_lut", "layer1_chained_mlp_silu_mul_stage_real_sigmoid_lut.hex", 16, False),
    ("final_gamma", "final_rmsnorm_stage_real_gamma.hex", 16, True),
]
OPS = {"file": 0, "zero": 1}


def words(path: Path) -> np.ndarray:
    return np.array([int(x, 16) for x in path.read_text().split()], dtype=np.uint32)


def values(path: Path, bits: int, signed: bool) -> np.ndarray:
    v = words(path).astype(np.int64) & ((1 << bits) - 1)
    if signed:
        v = np.where(v >= 1 << (bits - 1), v - (1 << bits), v)
    return v


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    a = ap.parse_args()
    ref = a.reference
    out = {}
    for key, name in PACKETS.items():
        out[f"pkt_{key}"] = words(ref / VEC / name).view(np.uint8)
    for key, name, bits, signed in COMPANIONS:
        out[f"ref_{key}"] = values(ref / VEC / name, bits, signed)
    man = json.loads((ref / "lmdeploy/qwen3-0p6b-q4-qweb-demo/model/pl_ddr_binary_segments.json").read_text())
    out["seg_address"] = np.array([s["address"] for s in man["segments"]], dtype=np.int64)
    out["seg_nbytes"] = np.array([s["nbytes"] for s in man["segments"]], dtype=np.int64)
    ent = [(s["index"], e) for s in man["segments"] for e in s["entries"]]
    out["ent_segment"] = np.array([i for i, _ in ent], dtype=np.int64)
    out["ent_name"] = np.array([e["name"] for _, e in ent])
    out["ent_op"] = np.array([OPS[e["operation"]] for _, e in ent], dtype=np.int64)
    out["ent_address"] = np.array([e["address"] for _, e in ent], dtype=np.int64)
    out["ent_nbytes"] = np.array([e["nbytes"] for _, e in ent], dtype=np.int64)
    np.savez_compressed(HERE / "qmap_ref.npz", **out)
    print("wrote", HERE / "qmap_ref.npz")


if __name__ == "__main__":
    main()
