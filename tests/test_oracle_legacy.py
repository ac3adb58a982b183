"""CPU oracle for the four formats the reference has no kernel for (Q4_1, Q5_0, Q5_1, Q8_0),
pinned byte for byte to gguf-py's own quantizers (gguf.quants.quantize), the same pin the
reference uses for Q4_0 (tests/test_q4_0.py:113-117). Q4_0 is checked the same way."""

import numpy as np
import pytest
from gguf import GGMLQuantizationType as GT
from gguf.quants import quantize as gguf_quantize

import oracle
from conftest import golden_x

LEGACY = {"q4_0": GT.Q4_0, "q4_1": GT.Q4_1, "q5_0": GT.Q5_0, "q5_1": GT.Q5_1, "q8_0": GT.Q8_0}


def adversarial_rows(k: int = 256) -> np.ndarray:
    """Rows (k values, 32-blocks) that hit every branch of the 32-block formats."""
    rng = np.random.default_rng(7)
    rows = []
    rows.append(np.zeros(k))                                     # d == 0
    rows.append(np.full(k, 0.25))                                # max == min (Q4_1 / Q5_1 d == 0)
    rows.append(np.full(k, -0.0))                                # negative zeros
    r = rng.normal(0, 0.02, k); r[::32] = 0.5; r[5::32] = -0.5   # +a and -a in every block
    rows.append(r)
    r = rng.normal(0, 0.02, k); r[3::32] = -0.5; r[9::32] = 0.5  # -a first
    rows.append(r)
    rows.append(rng.normal(0, 1e-30, k))                         # tiny but normal scales
    rows.append(rng.normal(0, 1e-38, k))                         # subnormal scales: 1 / d overflows
    rows.append(rng.normal(0, 3e-39, k))
    rows.append(rng.normal(0, 1e30, k))                          # huge values
    r = np.zeros(k); r[::32] = 1.0                               # one value per block
    rows.append(r)
    r = np.zeros(k); r[7::32] = -1e-40                           # one subnormal value per block
    rows.append(r)
    r = rng.integers(-127, 128, k) / 127.0                       # exact halves after scaling
    rows.append(r)
    r = (rng.integers(0, 31, k) + 0.5) / 31.0                    # Q5_1 ties at .5
    rows.append(r)
    r = np.abs(rng.normal(0, 0.02, k)); r[::4] = 0.0; r[1::8] = -0.0   # zero min: +0 and -0 mixed
    rows.append(r)
    r = -np.abs(rng.normal(0, 0.02, k)); r[3::8] = -0.0; r[::16] = 0.0  # zero max: +0 and -0 mixed
    rows.append(r)
    r = np.zeros(k); r[31::32] = -0.0; r[5::32] = -0.0                  # all zeros, mixed signs
    rows.append(r)
    return np.array(rows, dtype=np.float32)


# f16 scale fields (byte offsets) of each format
HALF_FIELDS = {"q4_0": (0,), "q4_1": (0, 2), "q5_0": (0,), "q5_1": (0, 2), "q8_0": (0,)}
BLOCK_BYTES = {"q4_0": 18, "q4_1": 20, "q5_0": 22, "q5_1": 24, "q8_0": 34}


def zero_sign_canonical(qtype: str, rows: np.ndarray) -> np.ndarray:
    """Rows with every f16 scale field that is +0 or -0 set to +0. ggml's scalar min / max
    keep the first of tied zeros, numpy's vectorised reductions one that depends on its SIMD
    lane order; only the sign of a zero d / m of Q4_1 / Q5_1 can differ, nothing else."""
    b = rows.reshape(rows.shape[0], -1, BLOCK_BYTES[qtype]).copy()
    for off in HALF_FIELDS[qtype]:
        h = b[..., off].astype(np.uint16) | (b[..., off + 1].astype(np.uint16) << 8)
        z = (h & 0x7FFF) == 0
        b[..., off][z] = 0
        b[..., off + 1][z] = 0
    return b.reshape(rows.shape)


def inputs():
    from conftest import golden_inputs
    g = golden_inputs()
    rng = np.random.default_rng(3)
    bench = rng.normal(0, 0.02, (64, 2560)).astype(np.float32)
    m = rng.random(bench.shape) < 0.001
    bench[m] = rng.normal(0, 0.5, int(m.sum()))
    return {"A": golden_x(g, "A"), "B": golden_x(g, "B"), "C": golden_x(g, "C"),
            "adversarial": adversarial_rows(), "k2560": bench}


def subnormal_scale_rows(x: np.ndarray) -> np.ndarray:
    """Rows with a block whose Q4_0 scale |max| / 8 is below 2^-128 (1 / d overflows)."""
    b = np.abs(x.reshape(x.shape[0], -1, 32)).max(-1)
    return ((b > 0) & (b / 8 < 2.0 ** -128)).any(1)


@pytest.mark.parametrize("qtype", list(LEGACY))
def test_oracle_matches_gguf_py(qtype):
    for name, x in inputs().items():
        if qtype == "q4_0":
            # Q4_0's ground truth is the reference (torch: +inf levels clamp to 15, NaN -> 0),
            # which gguf-py (numpy: every non-finite level -> 0) differs from on blocks whose
            # 1 / d overflows; the golden fixtures pin those blocks to the reference.
            x = x[~subnormal_scale_rows(x)]
        want = zero_sign_canonical(qtype, gguf_quantize(x, LEGACY[qtype]))
        got = zero_sign_canonical(qtype, oracle.quantize(qtype, x, nthreads=2))
        bad = np.nonzero((got != want).any(1))[0]
        assert bad.size == 0, f"{qtype}/{name}: rows {bad[:8]} differ from gguf-py"


def test_zero_sign_follows_ggml_scalar_loop():
    """Q4_1: a block whose minimum is zero takes the sign of the first zero (ggml's
    `if (v < min) min = v`), whatever numpy's vectorised min returns."""
    x = np.zeros((2, 32), np.float32)
    x[0, 3] = 0.5
    x[0, 7] = -0.0   # first zero is +0 -> m = +0
    x[1, 0] = -0.0   # first zero is -0 -> m = -0
    x[1, 9] = 0.25
    out = oracle.quantize("q4_1", x, nthreads=1)
    assert out[0, 2:4].tolist() == [0, 0] and out[1, 2:4].tolist() == [0, 0x80]
