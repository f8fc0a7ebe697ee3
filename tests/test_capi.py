"""The C ABI library on CPU: it loads, exports every function the public
header declares, and its host-side table builders match the reference."""
import ctypes as C
import re

import numpy as np
import pytest

from conftest import REPO


def _header_functions():
    text = (REPO / "include" / "q4gpu.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q4gpu_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from llm_accelerator_b200 import _native
    return _native.load()


def test_library_exports_every_header_symbol(lib):
    names = _header_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"


def test_ctypes_signatures_cover_header():
    from llm_accelerator_b200 import _native
    assert set(_header_functions()) <= set(_native.SIGNATURES)


def test_struct_layouts_match_reference_abi():
    from llm_accelerator_b200 import _native
    # qot_run_config_t / qot_result_t of qmap_one_token_runtime.h:44-82 on LP64
    assert C.sizeof(_native.QotResult) == 72
    assert _native.QotResult.score_q26.offset == 8
    assert _native.QotRunConfig.layer_qmap_bases.offset == 88
    assert C.sizeof(_native.QotRunConfig) == 104


def test_luts_match_reference(lib, refh):
    e = np.zeros(257, dtype=np.int32)
    s = np.zeros(1025, dtype=np.int32)
    lib.q4gpu_build_tables(e.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p))
    assert np.array_equal(e, refh["exp_lut"])
    assert np.array_equal(s, refh["sigmoid_lut"])


def test_host_rope_tables_match_reference(refh):
    from llm_accelerator_b200 import tables
    pos = refh["rope_positions"]
    c, s = tables.rope_tables(int(pos.max()) + 1)
    assert np.array_equal(c[pos], refh["rope_cos"]) and np.array_equal(s[pos], refh["rope_sin"])


def test_c_rope_builder_within_one_lsb(lib, refh):
    """The C-only RoPE builder (libm float32 cos/sin) is an approximation:
    torch's float32 cos/sin differ from libm in the last bit for some
    arguments, which flips a Q1.15 rounding in a small fraction of entries.
    The Python host installs the torch-built table (exact, tested above)."""
    pos = refh["rope_positions"]
    n = int(pos.max()) + 1
    c = np.zeros((n, 128), dtype=np.int32)
    s = np.zeros((n, 128), dtype=np.int32)
    lib.q4gpu_build_rope_table(n, c.ctypes.data_as(C.c_void_p), s.ctypes.data_as(C.c_void_p))
    dc = np.abs(c[pos] - refh["rope_cos"])
    ds = np.abs(s[pos] - refh["rope_sin"])
    assert max(dc.max(), ds.max()) <= 1
    assert (np.count_nonzero(dc) + np.count_nonzero(ds)) / (2 * dc.size) < 1e-3


def test_error_codes_without_gpu_work(lib):
    from llm_accelerator_b200 import _native
    # argument validation happens before any device work
    assert lib.q4gpu_gemv_q26(None, 1024, None, None, 16, None, None, None, None) == -1001
    assert lib.q4gpu_rmsnorm(None, None, 1, 1024, 5, None, None, None) == -1001
    cfg = _native.ModelConfig(n_layers=0, vocab=10, max_context=8, max_seqs=1, device=0)
    h = C.c_void_p()
    assert lib.q4gpu_model_create(C.byref(cfg), C.byref(h)) == -1001
    assert b"bad model config" in lib.q4gpu_last_error()
