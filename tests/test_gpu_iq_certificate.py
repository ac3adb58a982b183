"""The IQ lattice searches on inputs built to reach every branch of their certified runs (GPU).

The kernels solve a run of sweep steps that keep one off-grid code with one walk over the
neighbour list and a rounding-error certificate; runs that fail it are scored step by step,
and steps that fail again are searched exactly as the reference does. Benchmark-like data
certifies almost everything, so these rows force the other branches, and every byte must
still equal the oracle's:

* magnitudes far below and far above the certificate's guards (every run exact);
* groups of identical values and values on the lattice's points and midpoints (equal
  distances, which no certificate may decide);
* zeros, single outliers and mixed signs, with and without importance weights.
"""

import numpy as np
import pytest
import torch

import oracle
from kernels import _native

pytestmark = pytest.mark.gpu

IQ = ["iq2_xxs", "iq2_xs", "iq2_s", "iq3_xxs", "iq3_s"]
NEEDS_QW = {"iq2_xxs", "iq2_xs", "iq2_s"}  # the reference quantizes these only with an imatrix


def rows(k: int = 512) -> np.ndarray:
    rng = np.random.default_rng(20)
    base = rng.normal(0, 0.02, (8, k))
    # below and above the certificate's magnitude guards, every float staying finite
    out = [base * 1e-28, base * 1e-36, base * 1e7, base * 1e10]
    out.append(np.full((2, k), 0.0175))                                 # identical values
    out.append(np.tile([0.01, -0.01], (2, k // 2)))
    step = 0.004                                                        # lattice points, midpoints
    out.append(step * (2 * rng.integers(0, 8, (4, k)) + 1))
    out.append(step * (2 * rng.integers(0, 8, (4, k)) + 2))
    out.append(step * np.round(rng.normal(0, 4, (4, k))))
    z = rng.normal(0, 0.02, (4, k))
    z[:, ::3] = 0.0
    z[:, 5::64] = 0.9                                                   # one outlier per block
    out.append(z)
    signs = np.where(rng.random((4, k)) < 0.5, -1.0, 1.0)
    out.append(signs * np.abs(rng.normal(0, 0.02, (4, k))) + signs * 1e-4)
    return np.concatenate(out).astype(np.float32)


def run(qtype: str, x: torch.Tensor, qw):
    q = None if qw is None else torch.from_numpy(qw).cuda()
    out = _native.quantize(oracle.TYPE_IDS[qtype], x.cuda(), q)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("qtype", IQ)
@pytest.mark.parametrize("weights", ["imatrix", "none", "flat"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_certified_runs_and_fallbacks_match_the_oracle(qtype, weights, dtype):
    if weights == "none" and qtype in NEEDS_QW:
        pytest.skip("the reference quantizes this type only with importance weights")
    a = rows()
    x = torch.from_numpy(a).to(dtype)
    qw = {"imatrix": np.random.default_rng(3).lognormal(0, 1.5, a.shape[1]).astype(np.float32),
          "flat": np.ones(a.shape[1], np.float32), "none": None}[weights]
    got = run(qtype, x, qw)
    want = oracle.quantize(qtype, x.float().numpy(), qw)
    bad = np.nonzero((got != want).any(1))[0]
    assert bad.size == 0, f"{qtype} {weights} {dtype}: rows {bad[:8]} differ from the oracle"
