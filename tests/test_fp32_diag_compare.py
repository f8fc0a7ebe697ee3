"""Host part of the FP32 diagnostic: the comparison of two logit matrices."""
import numpy as np

from llm_accelerator_b200 import fp32_diag


def test_compare_identical_and_shifted():
    rng = np.random.default_rng(0)
    a = rng.normal(size=(3, 50))
    r = fp32_diag.compare(a, a.copy())
    assert r["top1_agreement"] == 1.0 and r["max_abs_diff"] == 0.0 and abs(r["pearson_min"] - 1) < 1e-12
    b = a.copy()
    b[0, np.argmax(a[0])] -= 10.0  # float32 demotes position 0's winner
    r = fp32_diag.compare(a, b)
    assert r["per_position"][0]["agree"] is False and r["per_position"][0]["fp32_rank_of_q4_top1"] > 0
    assert r["top1_agreement"] == 2 / 3
