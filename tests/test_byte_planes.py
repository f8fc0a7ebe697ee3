"""The integer identities behind the batched attention's tensor-core products
(q4_batch.cu: batch_attn_kernel, batch_attn_cl_tc_kernel), checked on the CPU.

Keys and values (signed 24-bit) are stored as three byte planes, the low two
unsigned and the top one signed; the query enters as the unsigned bytes of
q + 2^23 and the probability (0 .. 2^16) as its three bytes.  The kernels
form int32 partial products of those bytes on the tensor cores and combine
them in int64; these tests show the combination equals the direct int64 dot
product and that no int32 partial overflows, at the extremes the kernels
admit (128 dims; up to 2048 positions per CTA).
"""
import numpy as np
import pytest

LO, HI = -(1 << 23), (1 << 23) - 1


def planes(x: np.ndarray) -> list[np.ndarray]:
    """Byte planes of signed 24-bit values: b0, b1 unsigned, b2 signed."""
    x = x.astype(np.int64)
    return [x & 0xFF, (x >> 8) & 0xFF, x >> 16]


def score_by_planes(q: np.ndarray, k: np.ndarray) -> tuple[int, int]:
    """q . k from the products D_a[b] = sum_d k_a[d] c_b[d] and D_a[ones]."""
    c = q.astype(np.int64) + (1 << 23)
    cb = [(c >> (8 * b)) & 0xFF for b in range(3)]
    total, peak = 0, 0
    for a, ka in enumerate(planes(k)):
        d = [int(np.dot(ka, cb[b])) for b in range(3)]
        ones = int(ka.sum())
        peak = max(peak, *(abs(v) for v in d), abs(ones))
        total += (d[0] + (d[1] << 8) + (d[2] << 16) - (ones << 23)) << (8 * a)
    return total, peak


def values_by_planes(p: np.ndarray, v: np.ndarray) -> tuple[int, int]:
    """sum_pos p v from E_a[b] = sum_pos v_a p_b."""
    pb = [(p.astype(np.int64) >> (8 * b)) & 0xFF for b in range(3)]
    total, peak = 0, 0
    for a, va in enumerate(planes(v)):
        e = [int(np.dot(va, pb[b])) for b in range(3)]
        peak = max(peak, *(abs(x) for x in e))
        total += (e[0] + (e[1] << 8) + (e[2] << 16)) << (8 * a)
    return total, peak


@pytest.mark.parametrize("case", ["random", "min", "max", "mixed", "zero"])
def test_score_identity(case):
    rng = np.random.default_rng(7)
    q = {"random": rng.integers(LO, HI + 1, 128), "min": np.full(128, LO), "max": np.full(128, HI),
         "mixed": np.where(np.arange(128) % 2 == 0, LO, HI), "zero": np.zeros(128, dtype=np.int64)}[case]
    for k in (rng.integers(LO, HI + 1, 128), np.full(128, LO), np.full(128, HI), -q):
        got, peak = score_by_planes(q, k)
        assert got == int(np.dot(q.astype(object), k.astype(object)))
        assert peak < 2**31


@pytest.mark.parametrize("n", [1, 127, 128, 1024, 2048])
def test_value_identity(n):
    rng = np.random.default_rng(n)
    for p, v in ((rng.integers(0, (1 << 16) + 1, n), rng.integers(LO, HI + 1, n)),
                 (np.full(n, 1 << 16), np.full(n, LO)), (np.full(n, (1 << 16) - 1), np.full(n, HI)),
                 (np.full(n, 0xFFFF), np.full(n, LO))):
        got, peak = values_by_planes(p, v)
        assert got == int(np.dot(p.astype(object), v.astype(object)))
        assert peak < 2**31


def test_planes_reassemble():
    x = np.array([LO, LO + 1, -65536, -65537, -256, -1, 0, 1, 255, 256, 65535, 65536, HI - 1, HI])
    b0, b1, b2 = planes(x)
    assert ((b0 >= 0) & (b0 < 256) & (b1 >= 0) & (b1 < 256) & (b2 >= -128) & (b2 < 128)).all()
    assert (b0 + (b1 << 8) + (b2 << 16) == x).all()
