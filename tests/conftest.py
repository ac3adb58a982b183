import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "quant-studio_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden_inputs() -> dict:
    return dict(np.load(GOLDEN / "inputs.npz"))


def golden_x(inputs: dict, src: str) -> np.ndarray:
    """Input matrix of a fixture case as float32 (what the reference quantized)."""
    if src == "A":
        return (inputs["A_bf16"].astype(np.uint32) << 16).view(np.float32)
    if src == "B":
        return inputs["B_f32"]
    return inputs["C_f16"].astype(np.float32)


def golden_cases(qtype: str):
    """[(case_key, src, qw_key|None, ref_rows, ref_ieee_rows)] for one type."""
    ref = np.load(GOLDEN / f"{qtype}.npz")
    sparse = np.load(GOLDEN / f"{qtype}.ieee.npz")
    out = []
    for key in ref.files:
        src, qk = key.split("_")
        r = ref[key]
        ri = r.copy()
        ri[sparse[key + "_rows"]] = sparse[key + "_data"]
        out.append((key, src, None if qk == "none" else f"{src}_qw", r, ri))
    return out


ALL_TYPES = ["q4_0", "q2_k", "q3_k", "q4_k", "q5_k", "q6_k", "iq4_xs",
             "iq2_xxs", "iq2_xs", "iq2_s", "iq3_xxs", "iq3_s"]


@pytest.fixture(scope="session")
def inputs():
    return golden_inputs()
