"""q4gpu_lm_head_argmax_noalloc: the LM head + argmax for callers that cannot
allocate device memory (their memory belongs to another allocator's pool, or
they are ported hosts that only own the buffers they pass in).  Its scratch is
a static device array inside the library instead of a caller workspace.

Checked through the C ABI against the workspace entry point
q4gpu_lm_head_argmax, bit for bit (the path is exact integer arithmetic), on
two calls in a row with different inputs.  Collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from llm_accelerator_b200 import _native  # noqa: E402

MAX_ROWS = 16777216


def _case_inputs(act, packed, scale):
    a = torch.from_numpy(np.ascontiguousarray(act, dtype=np.int32)).cuda()
    w = torch.from_numpy(np.ascontiguousarray(packed, dtype=np.uint8)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(scale, dtype=np.uint16).view(np.int16)).cuda()
    return a, w, s


def _with_workspace(lib, a, w, s, rows, stream, scale_ptr=None, want_logits=True):
    ws_bytes = lib.q4gpu_lm_head_workspace_bytes(rows)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    logits = torch.empty(rows, dtype=torch.int64, device="cuda") if want_logits else None
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    score = torch.empty(1, dtype=torch.int64, device="cuda")
    rc = lib.q4gpu_lm_head_argmax(a.data_ptr(), w.data_ptr(), s.data_ptr() if scale_ptr is None else scale_ptr, rows,
                                  logits.data_ptr() if want_logits else None, ws.data_ptr(), ws_bytes,
                                  tok.data_ptr(), score.data_ptr(), stream)
    assert rc == 0, lib.q4gpu_last_error()
    return logits, tok, score


def test_noalloc_matches_workspace_entry_two_calls(kat):
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    g = kat.group("lm_head_argmax_stage_real")
    rng = np.random.default_rng(2024)
    rows2 = 20011
    cases = [
        (g["activation"], g["packed"], g["scale"]),
        (rng.integers(-(1 << 23), 1 << 23, 1024), rng.integers(0, 256, (rows2, 512)).astype(np.uint8),
         rng.integers(0, 1 << 16, (rows2, 16)).astype(np.uint16)),
    ]
    inputs = [_case_inputs(*c) for c in cases]
    rows = [int(c[1].shape[0]) for c in cases]
    # two no-alloc calls back to back on one stream, outputs kept apart
    outs = []
    for (a, w, s), r in zip(inputs, rows):
        logits = torch.empty(r, dtype=torch.int64, device="cuda")
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        score = torch.empty(1, dtype=torch.int64, device="cuda")
        rc = lib.q4gpu_lm_head_argmax_noalloc(a.data_ptr(), w.data_ptr(), s.data_ptr(), r, logits.data_ptr(),
                                              tok.data_ptr(), score.data_ptr(), stream)
        assert rc == 0, lib.q4gpu_last_error()
        outs.append((logits, tok, score))
    torch.cuda.synchronize()
    for (a, w, s), r, (logits, tok, score) in zip(inputs, rows, outs):
        ref_logits, ref_tok, ref_score = _with_workspace(lib, a, w, s, r, stream)
        torch.cuda.synchronize()
        assert torch.equal(logits, ref_logits)
        assert int(tok.item()) == int(ref_tok.item()) and int(score.item()) == int(ref_score.item())
    # the reference's own scan window result for the first case
    assert (int(outs[0][1].item()), int(outs[0][2].item())) == (264, 1365150750)


def test_noalloc_unaligned_scales_without_logits():
    """Scales that start 2 bytes past a 16-byte boundary take the library's
    CUDA-core GEMV kernel instead of the tensor-core one; it writes the same
    static scratch.  No logits are requested.  Two calls in a row, each checked
    against the workspace entry point on the same pointers."""
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(77)
    for rows in (4099, 1536):
        act = rng.integers(-(1 << 23), 1 << 23, 1024)
        packed = rng.integers(0, 256, (rows, 512)).astype(np.uint8)
        scale = rng.integers(0, 1 << 16, rows * 16 + 1).astype(np.uint16)  # one spare u16 in front
        a, w, s = _case_inputs(act, packed, scale)
        sp = s.data_ptr() + 2
        assert sp % 16 == 2
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        score = torch.empty(1, dtype=torch.int64, device="cuda")
        rc = lib.q4gpu_lm_head_argmax_noalloc(a.data_ptr(), w.data_ptr(), sp, rows, None, tok.data_ptr(),
                                              score.data_ptr(), stream)
        assert rc == 0, lib.q4gpu_last_error()
        _, ref_tok, ref_score = _with_workspace(lib, a, w, s, rows, stream, scale_ptr=sp, want_logits=False)
        torch.cuda.synchronize()
        assert (int(tok.item()), int(score.item())) == (int(ref_tok.item()), int(ref_score.item()))
        # and the tensor-core path on the aligned copy of the same scales agrees
        s2 = torch.from_numpy(scale[1:].copy().view(np.int16)).cuda()
        _, al_tok, al_score = _with_workspace(lib, a, w, s2, rows, stream, want_logits=False)
        torch.cuda.synchronize()
        assert (int(al_tok.item()), int(al_score.item())) == (int(tok.item()), int(score.item()))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _native.load()
    dummy = torch.zeros(16, dtype=torch.int64, device="cuda")
    p = dummy.data_ptr()
    for rows in (0, -5, MAX_ROWS + 1):
        rc = lib.q4gpu_lm_head_argmax_noalloc(p, p, p, rows, None, p, p, None)
        assert rc == _native.Q4GPU_OK - 1001, rows
        assert b"outside 1.." in lib.q4gpu_last_error()
