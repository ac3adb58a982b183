"""The CPU oracle against the reference's own outputs (tests/golden, from gen_golden.py)."""

import numpy as np
import pytest

import oracle
from conftest import ALL_TYPES, golden_cases, golden_x
from wmse import block_wmse


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_oracle_bit_exact_vs_ieee_sqrt_reference(qtype, inputs):
    """Pin: the reference with only torch.sqrt made correctly rounded == oracle, bit for bit."""
    for key, src, qwk, _ref, ref_ieee in golden_cases(qtype):
        qw = None if qwk is None else inputs[qwk]
        got = oracle.quantize(qtype, golden_x(inputs, src), qw)
        assert got.shape == ref_ieee.shape, key
        bad = np.nonzero((got != ref_ieee).any(1))[0]
        assert bad.size == 0, f"{qtype} {key}: rows {bad[:8]} differ"


# Blocks of the fixtures where the reference as shipped has the lower importance-weighted
# error, with ours / shipped: each is a scale-search tie tipped by torch's CPU sqrt (1 ulp low
# on about 0.6 % of inputs); the reference with a correctly rounded sqrt returns our bytes
# there (test_oracle_bit_exact_vs_ieee_sqrt_reference).
SQRT_TIPPED = {"q5_k/A_qw#133": 1.002756, "q5_k/A_qw#204": 1.001886, "iq2_xs/A_qw#499": 1.000431,
               "iq2_s/A_qw#265": 1.022513, "iq2_s/A_qw#602": 1.000676}


def _differing_blocks(inputs):
    """[(name, ours_block, shipped_block, x, qw)] over every fixture case of every type."""
    out = []
    for qtype in ALL_TYPES:
        for key, src, qwk, ref, ref_ieee in golden_cases(qtype):
            qw = None if qwk is None else inputs[qwk]
            x = golden_x(inputs, src)
            qk = 32 if qtype == "q4_0" else 256
            nb = x.shape[0] * x.shape[1] // qk
            a, b = ref_ieee.reshape(nb, -1), ref.reshape(nb, -1)
            for blk in np.nonzero(~(a == b).all(1))[0]:
                row, c = divmod(int(blk), x.shape[1] // qk)
                out.append((f"{qtype}/{key}#{blk}", qtype, a[blk], b[blk], x[row, c * qk:(c + 1) * qk],
                            None if qw is None else qw[c * qk:(c + 1) * qk]))
    return out


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_oracle_vs_reference_as_shipped(qtype, inputs):
    """The reference as shipped uses torch's CPU sqrt: blocks differ only where the IEEE-sqrt
    reference differs from it (the oracle equals the latter), and >= 99.5 % are identical."""
    for key, src, qwk, ref, ref_ieee in golden_cases(qtype):
        qw = None if qwk is None else inputs[qwk]
        x = golden_x(inputs, src)
        got = oracle.quantize(qtype, x, qw)
        qk = 32 if qtype == "q4_0" else 256
        nb = x.shape[0] * x.shape[1] // qk
        same = (got.reshape(nb, -1) == ref.reshape(nb, -1)).all(1)
        assert same.mean() >= 0.995, f"{qtype} {key}: {same.mean():.4f} identical"


def test_sqrt_tipped_blocks_are_exactly_the_named_ones(inputs):
    """Every differing block has importance-weighted error <= the shipped block's (within 1e-6
    relative) except the named ones, whose ratios are as recorded."""
    ratios = {}
    for name, qtype, ours, shipped, xb, wb in _differing_blocks(inputs):
        ratios[name] = block_wmse(qtype, ours, xb, wb) / block_wmse(qtype, shipped, xb, wb)
    assert {n for n, r in ratios.items() if r > 1 + 1e-6} == set(SQRT_TIPPED)
    for n, r in SQRT_TIPPED.items():
        assert abs(ratios[n] - r) < 1e-5, n


@pytest.mark.parametrize("name", list(SQRT_TIPPED))
@pytest.mark.xfail(strict=True, reason="torch CPU sqrt 1 ulp low in the shipped reference's importance weights "
                                       "tipped a scale-search tie; the IEEE-sqrt reference returns our bytes")
def test_named_block_error_no_worse_than_shipped(name, inputs):
    blk = next(b for b in _differing_blocks(inputs) if b[0] == name)
    _, qtype, ours, shipped, xb, wb = blk
    assert block_wmse(qtype, ours, xb, wb) <= block_wmse(qtype, shipped, xb, wb) * (1 + 1e-6)
