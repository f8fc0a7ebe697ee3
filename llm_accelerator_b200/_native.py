"""ctypes binding of libq4gpu.so (the C ABI declared in include/q4gpu.h).

Importing this module loads the in-tree shared library and fails loudly if it
is missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libq4gpu.so"

Q4GPU_OK = 0
ERRORS = {-1001: "ARG", -1002: "SHAPE", -1003: "ALIGN", -1004: "CUDA", -1005: "WORKSPACE", -1006: "QUANT"}

# qot_* error codes (qmap_one_token_runtime.h:17-29)
QOT_OK, QOT_ERR_BUSY, QOT_ERR_BAD_LAYER, QOT_ERR_BAD_TABLE, QOT_ERR_BAD_ADDR = 0, -1, -2, -3, -4
QOT_ERR_TIMEOUT, QOT_ERR_STATUS, QOT_ERR_NULL, QOT_ERR_BAD_TOKEN = -5, -6, -7, -8
QOT_ERR_CAPACITY, QOT_ERR_CONTEXT = -9, -10

# tensor ids (q4gpu_model_set_tensor)
T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN = range(7)
T_INPUT_GAMMA, T_POST_GAMMA, T_Q_GAMMA, T_K_GAMMA = range(7, 11)
T_EMBED, T_FINAL_GAMMA, T_ROPE_COS, T_ROPE_SIN, T_EXP_LUT, T_SIGMOID_LUT = range(100, 106)

# kernel kinds of one decode step (q4gpu_model_time_kernels)
KERNEL_KINDS = ["embed", "qkv_norm_rope_kv", "attention", "o_proj_residual", "post_norm_gate_up_swiglu",
                "down_residual", "final_norm_lm_head_argmax", "advance"]
# kernels of a batched step (Q4GPU_BK_*)
BATCH_KERNEL_KINDS = ["embed", "norm_limbs", "qkv_gemm", "attention", "o_proj_gemm", "gate_up_gemm", "down_gemm",
                      "lm_head_gemm", "argmax"]


class QotLayerQmapBases(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("qkv", "input_norm", "attn_frontend", "attn_score_value", "o_proj",
                                           "post_attn_norm", "mlp_gate_up", "mlp_silu_mul", "mlp_down",
                                           "mlp_residual_add")]


class QotRunConfig(C.Structure):
    _fields_ = [("layer_start", C.c_uint32), ("layer_count", C.c_uint32), ("position", C.c_uint32),
                ("runtime_context_enable", C.c_uint32), ("input_token_id", C.c_uint32),
                ("embedding_enable", C.c_uint32), ("embedding_weight_base", C.c_uint64),
                ("embedding_scale_base", C.c_uint64), ("input_hidden_base", C.c_uint64),
                ("output_hidden_base", C.c_uint64), ("kv_cache_base", C.c_uint64),
                ("final_tail_qmap_base", C.c_uint64), ("final_hidden_override_valid", C.c_uint32),
                ("final_hidden_override_base", C.c_uint64), ("layer_qmap_bases", C.POINTER(QotLayerQmapBases)),
                ("layer_qmap_base_count", C.c_uint32)]


class QotResult(C.Structure):
    _fields_ = [("status", C.c_uint32), ("token_id", C.c_uint32), ("score_q26", C.c_int64),
                ("layers_started", C.c_uint32), ("layers_completed", C.c_uint32),
                ("layer_done_mask", C.c_uint32), ("layer_error_mask", C.c_uint32),
                ("last_output_base", C.c_uint64), ("tail_hidden_base", C.c_uint64),
                ("tail_tiles_started", C.c_uint32), ("tail_tiles_completed", C.c_uint32),
                ("mem_read_reqs", C.c_uint32), ("mem_read_words", C.c_uint32),
                ("mem_write_reqs", C.c_uint32), ("mem_write_words", C.c_uint32)]


class ModelConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("vocab", C.c_int32), ("max_context", C.c_int32),
                ("max_seqs", C.c_int32), ("device", C.c_int32), ("reserved", C.c_int32 * 3)]


class QmapHeader(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("magic", "version", "header_bytes", "descriptor_bytes",
                                           "descriptor_count", "descriptor_capacity")] + \
               [(n, C.c_uint64) for n in ("descriptor_table_addr", "payload_base_addr", "image_base_addr",
                                           "image_bytes")] + [("flags", C.c_uint32), ("checksum32", C.c_uint32)]


class QmapDescriptor(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("tensor_id", "role", "dtype", "rank", "flags", "element_bits",
                                           "group_size", "scale_tensor_id")] + \
               [("base_addr", C.c_uint64), ("nbytes", C.c_uint64), ("dims", C.c_uint32 * 4),
                ("strides_bytes", C.c_uint64 * 4), ("aux", C.c_uint32 * 4), ("checksum32", C.c_uint32),
                ("reserved", C.c_uint32 * 3)]


class QmapLayout(C.Structure):
    _fields_ = [("arena_base", C.c_uint64), ("final_tail_qmap_base", C.c_uint64), ("rope_cos_base", C.c_uint64),
                ("rope_sin_base", C.c_uint64), ("embed_weight_base", C.c_uint64), ("embed_scale_base", C.c_uint64),
                ("n_layers", C.c_int32), ("reserved", C.c_int32), ("layer_bases", C.POINTER(C.c_uint64))]


class QmapTensor(C.Structure):
    _fields_ = [("layer", C.c_int32), ("which", C.c_int32), ("data_offset", C.c_uint64),
                ("data_bytes", C.c_uint64), ("scale_offset", C.c_uint64), ("scale_bytes", C.c_uint64),
                ("rows", C.c_int32), ("cols", C.c_int32), ("elem_stride", C.c_int32), ("elem_kind", C.c_int32)]


QMAP_PACKED_Q4, QMAP_S16, QMAP_U16, QMAP_U32 = range(4)

P = C.c_void_p
I32, I64, U32, U64, SZ = C.c_int32, C.c_int64, C.c_uint32, C.c_uint64, C.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "q4gpu_last_error": (C.c_char_p, []),
    "q4gpu_version": (C.c_char_p, []),
    "q4gpu_synth_f32": (C.c_int, [U64, U64, I64, I64, C.c_float, C.c_int, P, P]),
    "q4gpu_quantize_q4": (C.c_int, [P, I64, I32, P, P, P, P]),
    "q4gpu_gemv_q26": (C.c_int, [P, I32, P, P, I32, P, P, P, P]),
    "q4gpu_gemv_q26_strided": (C.c_int, [P, C.c_int64, I32, P, C.c_int64, P, C.c_int64, I32, I32, P, P,
                                         C.c_int64, P, P]),
    "q4gpu_q26_to_q12_12": (C.c_int, [P, I32, P, P, P]),
    "q4gpu_rmsnorm": (C.c_int, [P, P, I32, I32, I32, P, P, P]),
    "q4gpu_rope": (C.c_int, [P, I32, P, P, P, P, P]),
    "q4gpu_attention_scores": (C.c_int, [P, P, I32, I32, I32, I64, P, P, P]),
    "q4gpu_softmax_probs": (C.c_int, [P, I32, I32, P, P, P, P]),
    "q4gpu_value_accum": (C.c_int, [P, P, I32, I32, I32, P, P, P]),
    "q4gpu_silu_mul": (C.c_int, [P, P, I32, P, P, P, P, P, P]),
    "q4gpu_residual_add": (C.c_int, [P, P, I32, I32, P, P, P]),
    "q4gpu_embedding": (C.c_int, [P, I32, P, P, P, P]),
    "q4gpu_lm_head_workspace_bytes": (SZ, [I32]),
    "q4gpu_lm_head_argmax": (C.c_int, [P, P, P, I32, P, P, SZ, P, P, P]),
    "q4gpu_lm_head_argmax_noalloc": (C.c_int, [P, P, P, I32, P, P, P, P]),
    "q4gpu_model_create": (C.c_int, [C.POINTER(ModelConfig), C.POINTER(P)]),
    "q4gpu_model_destroy": (None, [P]),
    "q4gpu_model_init_synthetic": (C.c_int, [P, U64, C.c_float, C.c_float]),
    "q4gpu_model_set_tensor": (C.c_int, [P, I32, I32, P, SZ, P, SZ]),
    "q4gpu_model_get_tensor": (C.c_int, [P, I32, I32, P, SZ, P, SZ]),
    "q4gpu_run_token": (C.c_int, [P, C.c_size_t, C.POINTER(QotRunConfig), U32, U32, U32, C.POINTER(QotResult)]),
    "q4gpu_decode_token_ids": (C.c_int, [P, C.c_size_t, C.POINTER(QotRunConfig), P, U32, U32, P, U32, U32,
                                         C.POINTER(U32), C.POINTER(QotResult)]),
    "q4gpu_decode_batch": (C.c_int, [P, I32, P, P, U32, P, P]),
    "q4gpu_batch_steps": (C.c_int, [P, I32, I32, I32]),
    "q4gpu_batch_prefill": (C.c_int, [P, I32, I32, P, P]),
    "q4gpu_model_set_prefill": (C.c_int, [P, I32]),
    "q4gpu_batch_forward_hidden": (C.c_int, [P, I32, I32, P]),
    "q4gpu_lm_head_shard": (C.c_int, [P, P, I32, I32, I32, P, P]),
    "q4gpu_batch_commit": (C.c_int, [P, I32, I32, P, P]),
    "q4gpu_batch_commit_shards": (C.c_int, [P, I32, I32, P, I32, I32, I32]),
    "q4gpu_batch_set_position": (C.c_int, [P, I32, I32, I32, I32]),
    "q4gpu_batch_run_step": (C.c_int, [P, I32, I32, P, P, P, P]),
    "q4gpu_batch_time_kernels": (C.c_int, [P, I32, I32, I32, P, P]),
    "q4gpu_batch_trace": (C.c_int, [P, I32, I32, P, C.c_int64, P, C.c_int64]),
    "q4gpu_model_read_hidden": (C.c_int, [P, C.c_size_t, P]),
    "q4gpu_model_read_kv": (C.c_int, [P, C.c_size_t, I32, I32, I32, P]),
    "q4gpu_model_write_hidden": (C.c_int, [P, C.c_size_t, P]),
    "q4gpu_model_write_kv": (C.c_int, [P, C.c_size_t, I32, I32, I32, P]),
    "q4gpu_build_tables": (None, [P, P]),
    "q4gpu_build_rope_table": (None, [I32, P, P]),
    "q4gpu_model_stream": (P, [P]),
    "q4gpu_decode_steps": (C.c_int, [P, C.c_size_t, I32]),
    "q4gpu_model_sync": (C.c_int, [P]),
    "q4gpu_model_set_mode": (C.c_int, [P, I32]),
    "q4gpu_model_get_mode": (I32, [P]),
    "q4gpu_model_trace_persistent": (C.c_int, [P, C.c_size_t, I32, I32, P, I32]),
    "q4gpu_model_set_position": (C.c_int, [P, C.c_size_t, I32]),
    "q4gpu_model_read_tokens": (C.c_int, [P, C.c_size_t, I32, I32, P, P, P]),
    "q4gpu_model_time_kernels": (C.c_int, [P, C.c_size_t, I32, P, P]),
    "q4gpu_model_time_layers": (C.c_int, [P, C.c_size_t, I32, I32, I32, I32, P]),
    "q4gpu_model_get_config": (C.c_int, [P, C.POINTER(ModelConfig)]),
    "q4gpu_qmap_read_packet": (C.c_int, [P, U64, U64, U64, C.POINTER(QmapHeader), C.POINTER(QmapDescriptor), I32]),
    "q4gpu_qmap_bind": (C.c_int, [P, U64, C.POINTER(QmapLayout), C.POINTER(QmapTensor), I32, C.POINTER(I32)]),
    "q4gpu_qmap_vector": (C.c_int, [P, C.POINTER(QmapTensor), P, I64]),
    "q4gpu_model_load_qmap": (C.c_int, [P, P, U64, C.POINTER(QmapLayout)]),
}

_lib = None


def load() -> C.CDLL:
    """Load libq4gpu.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m llm_accelerator_b200.build` "
                               "(there is no CPU fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class Q4GpuError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != Q4GPU_OK:
        msg = load().q4gpu_last_error().decode(errors="replace")
        raise Q4GpuError(f"{what} failed ({ERRORS.get(rc, rc)}): {msg}")
