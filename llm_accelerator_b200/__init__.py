"""B200-native Qwen3-0.6B Q4 fixed-point decode path.

A from-scratch sm_100a implementation of the hot path that
Tyler913/LLM_Accelerator implements in Verilog and mirrors in Python: exact
integer Q4 GEMVs, fixed-point RMSNorm / RoPE / LUT softmax / SwiGLU, paged KV
cache and a fused LM head + argmax, behind the reference's runner seam
(``qot_session_runner_fn``) and per-module helper names.

* ``llm_accelerator_b200.reference_api`` - the reference helper names on GPU.
* ``llm_accelerator_b200.model.Q4Model`` - model context and decode APIs.
* ``include/q4gpu.h`` / ``_lib/libq4gpu.so`` - the C ABI.
"""
from ._native import load as load_library  # noqa: F401

__all__ = ["load_library"]
