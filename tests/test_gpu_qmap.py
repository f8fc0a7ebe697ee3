"""QMAP image -> device context on the GPU: a synthetic model written as the
reference's PL-DDR segment bundle and loaded into a fresh context through
q4gpu_model_load_qmap decodes exactly like the original."""
import numpy as np
import pytest

from llm_accelerator_b200 import _native, qmap
from llm_accelerator_b200.model import Q4Model

pytestmark = pytest.mark.gpu


def test_qmap_bundle_loads_into_a_context(tmp_path):
    layers, vocab = 2, 4096
    prompt = np.random.default_rng(5).integers(0, vocab, 12).tolist()
    with Q4Model(n_layers=layers, vocab=vocab, max_context=64, max_seqs=1) as src:
        src.init_synthetic(seed=3, gamma_std=0.2)
        t = qmap.tensors_from_model(src)
        want, want_scores = src.decode_batch([prompt], 8)
        want_b1, _ = src.decode(prompt, 8)
    man = qmap.write_bundle(qmap.build_segments(t), tmp_path)
    arena, base = qmap.load_bundle(man)
    with Q4Model(n_layers=layers, vocab=vocab, max_context=64, max_seqs=1) as dst:
        qmap.load_into_model(dst, arena)
        for layer in range(layers):
            for which in range(_native.T_Q, _native.T_DOWN + 1):
                w, s = dst.get_weight(layer, which)
                assert np.array_equal(w, t.weights[(layer, which)][0]) and np.array_equal(s, t.weights[(layer, which)][1])
            for which in range(_native.T_INPUT_GAMMA, _native.T_K_GAMMA + 1):
                assert np.array_equal(dst.get_gamma(layer, which), t.gammas[(layer, which)])
        got, got_scores = dst.decode_batch([prompt], 8)
        got_b1, _ = dst.decode(prompt, 8)
    assert np.array_equal(got, want) and np.array_equal(got_scores, want_scores)
    assert got_b1 == want_b1 == want[0].tolist()
