"""Parity with the reference on the benchmark configurations' own rows (tests/golden/
config_parity.json, written by tests/golden/gen_config_golden.py from the reference).

The bar, per (type, row subset):
  * bit-exact against the reference with a correctly rounded sqrt: the oracle (CPU) and
    libqsb200 (GPU) produce the same sha256 as that reference;
  * against the reference as shipped, whose torch CPU sqrt (MKL VML) returns about 0.6 % of
    its results 1 ulp low: the output differs only in the blocks the fixture lists (the
    as-shipped sha256 is rebuilt from ours plus those blocks), the identical-block fraction
    is at least the reference's own README figure against llama-quantize, and every
    differing block has an importance-weighted squared error no larger than the shipped
    block's (within 1e-6 relative), except the blocks named in SQRT_TIPPED below;
  * the summed importance-weighted error of each subset within 1e-4 of the shipped one.

SQRT_TIPPED names every block where the shipped reference's 1-ulp-low square roots moved a
near tie of a scale search to a candidate with lower error; with a correctly rounded sqrt the
reference itself returns our bytes there (the first check). Each is an expected failure with
its error ratio; any other worse block fails the suite, and so does a listed block that stops
failing (strict). The same effect goes the other way about as often (blocks where ours has the
lower error are not listed); a subset's summed error is at most 2e-5 above the shipped one
(and up to 5e-4 below it).
"""

import hashlib
import json

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN
from wmse import block_wmse

import sys
sys.path.insert(0, str(GOLDEN))
import config_rows  # noqa: E402

FIX = json.loads((GOLDEN / "config_parity.json").read_text())
CASES = FIX["cases"]

# identical-block % of the reference against llama-quantize, README.md:28-49 (the scheme
# named after the type; Q4_K: Q4_K_M, Q5_K: Q5_K_M, Q3_K: Q3_K_M)
README_IDENTICAL = {"q2_k": 0.9971, "q3_k": 0.9956, "q4_k": 0.9901, "q5_k": 0.9885, "q6_k": 1.0, "iq4_xs": 0.9963,
                    "iq2_xxs": 0.9950, "iq2_xs": 0.9867, "iq2_s": 0.9878, "iq3_xxs": 0.9915, "iq3_s": 0.9971,
                    "q4_0": 1.0}

# blocks (case#block) where the shipped reference has the lower importance-weighted error,
# with ours / shipped: every one is a sqrt-tipped tie (see the module docstring)
SQRT_TIPPED = {
    "q2_k/c2_a#410": 1.118525, "q4_k/c2_a#655": 1.059257, "q5_k/c2_a#791": 1.066816, "q5_k/c2_a#3605": 1.033054,
    "iq2_xs/c2_a#20": 1.032185, "iq2_xs/c2_a#123": 1.002646, "iq2_s/c2_a#739": 1.001282,
    "iq2_s/c2_a#2782": 1.001377, "iq3_xxs/c2_a#1438": 1.036814, "q2_k/c2_b#36": 1.118242,
    "q2_k/c2_b#2420": 1.014561, "q2_k/c2_b#3299": 1.010899, "q4_k/c2_b#3151": 1.010237,
    "q5_k/c2_b#3017": 1.128772, "iq2_xs/c2_b#1044": 1.020152, "iq2_s/c2_b#1533": 1.003111,
    "iq2_s/c2_b#1999": 1.039588, "iq2_s/c2_b#2406": 1.000107, "iq2_s/c2_b#3280": 1.011744,
    "iq2_s/c5_dn#2203": 1.216773, "q4_k/c5_dn#330": 1.053532, "q4_k/c5_dn#1425": 1.020557,
    "q4_k/c5_dn#1565": 1.001703, "q5_k/c5_dn#1161": 1.060045,
}


def case_inputs(case: str):
    if case == "edge":
        from test_oracle_legacy import adversarial_rows
        return torch.from_numpy(adversarial_rows(256)).to(torch.bfloat16)
    return config_rows.rows_bf16(case)


def oracle_output(key: str) -> np.ndarray:
    c = CASES[key]
    x = case_inputs(c["case"]).float().numpy()
    qw = config_rows.imatrix(x.shape[1]) if c["imatrix"] else None
    return oracle.quantize(c["type"], x, qw)


def shipped_from(key: str, ours: np.ndarray) -> np.ndarray:
    """The shipped reference's output rebuilt from ours and the fixture's differing blocks."""
    c = CASES[key]
    b = ours.reshape(c["blocks"], -1).copy()
    for d in c["diff"]:
        assert bytes(b[d["block"]]).hex() == d["ieee"], f"{key} block {d['block']}"
        b[d["block"]] = np.frombuffer(bytes.fromhex(d["shipped"]), np.uint8)
    return b


def test_inputs_regenerate_bit_for_bit():
    for case, digest in FIX["inputs"].items():
        assert config_rows.bf16_digest(case) == digest, case


@pytest.mark.parametrize("key", list(CASES))
def test_oracle_bit_exact_vs_ieee_sqrt_reference(key):
    got = oracle_output(key)
    assert hashlib.sha256(got.tobytes()).hexdigest() == CASES[key]["sha_ieee"]


@pytest.mark.parametrize("key", list(CASES))
def test_shipped_reference_differs_only_in_listed_blocks(key):
    c = CASES[key]
    shipped = shipped_from(key, oracle_output(key))
    assert hashlib.sha256(shipped.tobytes()).hexdigest() == c["sha_shipped"]
    identical = 1.0 - len(c["diff"]) / c["blocks"]
    assert identical >= README_IDENTICAL[c["type"]], f"{key}: {identical:.5f} identical"


def _block_errors(key: str, block: int):
    c = CASES[key]
    x = case_inputs(c["case"]).float().numpy()
    qk = 32 if c["type"] == "q4_0" else 256
    row, col = divmod(block, x.shape[1] // qk)
    xb = x[row, col * qk:(col + 1) * qk]
    wb = config_rows.imatrix(x.shape[1])[col * qk:(col + 1) * qk] if c["imatrix"] else None
    d = next(d for d in c["diff"] if d["block"] == block)
    ours = np.frombuffer(bytes.fromhex(d["ieee"]), np.uint8)
    ref = np.frombuffer(bytes.fromhex(d["shipped"]), np.uint8)
    return block_wmse(c["type"], ours, xb, wb), block_wmse(c["type"], ref, xb, wb)


DIFF_BLOCKS = [f"{k}#{d['block']}" for k, c in CASES.items() for d in c["diff"]]


@pytest.mark.parametrize("name", [
    pytest.param(n, marks=pytest.mark.xfail(strict=True, reason=(
        f"torch CPU sqrt 1 ulp low in the shipped reference's importance weights tipped a scale-search "
        f"tie; the reference with a correctly rounded sqrt returns our bytes; error ours/shipped "
        f"{SQRT_TIPPED[n]:.6f}"))) if n in SQRT_TIPPED else n
    for n in DIFF_BLOCKS])
def test_differing_block_error_no_worse_than_shipped(name):
    key, block = name.rsplit("#", 1)
    e_ours, e_ref = _block_errors(key, int(block))
    assert e_ours <= e_ref * (1 + 1e-6), f"{name}: {e_ours:.6g} > {e_ref:.6g} (x{e_ours / e_ref:.6f})"


def test_named_blocks_are_exactly_the_worse_ones():
    ratios = {}
    for n in DIFF_BLOCKS:
        key, block = n.rsplit("#", 1)
        e_ours, e_ref = _block_errors(key, int(block))
        ratios[n] = e_ours / e_ref
    assert {n for n, r in ratios.items() if r > 1 + 1e-6} == set(SQRT_TIPPED)
    for n, r in SQRT_TIPPED.items():
        assert abs(ratios[n] - r) < 1e-5, n


@pytest.mark.parametrize("key", [k for k, c in CASES.items() if c["agg_wmse_qw"][1] > 0])
def test_summed_error_matches_shipped(key):
    ours, ref = CASES[key]["agg_wmse_qw"]
    assert ours <= ref * (1 + 1e-4), f"{key}: summed weighted error x{ours / ref:.8f}"


@pytest.mark.gpu
@pytest.mark.parametrize("key", list(CASES))
def test_gpu_bit_exact_vs_ieee_sqrt_reference(key):
    from kernels import _native
    c = CASES[key]
    x = case_inputs(c["case"]).cuda()
    qw = torch.from_numpy(config_rows.imatrix(x.shape[1])).cuda() if c["imatrix"] else None
    got = _native.quantize(int(oracle.TYPE_IDS[c["type"]]), x, qw).cpu().numpy()
    assert hashlib.sha256(got.tobytes()).hexdigest() == c["sha_ieee"]
