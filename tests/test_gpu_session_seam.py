"""The reference's own prompt/session state machine (qot_session.c, compiled
from the reference sources into oracle/_ref/session_seam by oracle/build_ref.py)
drives q4gpu_run_token as its runner: the generated ids and scores must equal
the CPU oracle's greedy decode."""
import subprocess
from pathlib import Path

import pytest

from oracle.c_oracle import CModel

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

EXE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "session_seam"


@pytest.mark.skipif(not EXE.exists(), reason="oracle/_ref/session_seam not built (needs the reference sources)")
@pytest.mark.parametrize("prompt,max_new", [([3, 4096, 8191, 17, 5], 6), ([42], 4)])
def test_reference_session_drives_gpu_runner(prompt, max_new):
    seed, layers, vocab, gamma = 11, 2, 8192, 0.05
    out = subprocess.run([str(EXE), str(layers), str(vocab), str(seed), str(gamma), str(max_new)] +
                         [str(t) for t in prompt], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = out.stdout.strip().splitlines()
    toks = [(int(l.split()[1]), int(l.split()[3]), int(l.split()[5])) for l in lines if l.startswith("token")]
    assert lines[-1] == "state DONE stop MAX_NEW", lines[-1]
    cm = CModel(layers, vocab, 256, seed=seed, std=0.02, gamma_std=gamma)
    ref, ref_scores = cm.decode(prompt, max_new)
    cm.close()
    # the session emits one token event per generated id; the first comes from the last prompt position
    assert [t for t, _, _ in toks] == ref
    assert [s for _, s, _ in toks] == ref_scores
    assert [p for _, _, p in toks] == list(range(len(prompt) - 1, len(prompt) - 1 + max_new))
