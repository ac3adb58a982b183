"""Row subsets of the benchmark configurations, regenerated bit for bit from fixed seeds.

The configurations quantize synthetic bf16 weights drawn N(0, 0.02) with 0.1 % of the
entries replaced by N(0, 0.5) outliers, with a per-column importance matrix drawn
lognormal(0, 1.5) (weights seed 0, importance seed 1). Whole tensors are too large to run
through the reference's CPU path in a test, so each case is a fixed slice of such a tensor
with the row length of the configuration it stands for:

    c2_a   256 rows of a 4096 x 4096 tensor          (configs[1], attn_q-like)
    c2_b   256 rows of a 14336 x 4096 tensor         (configs[1], ffn_up-like)
    c5_dn  64 rows of an 8B-class ffn_down, k 14336  (configs[4])
    c4_dn  64 rows of a 4B-class ffn_down, k 9728    (configs[3])
    c3_emb 256 rows of the 151936 x 2560 token embedding, N(0, 0.02) without outliers
           (configs[2], quantized to Q4_0)

Used by gen_config_golden.py (which runs the reference on them) and by the tests (which
run the oracle and the GPU on the same rows).
"""

from __future__ import annotations

import numpy as np
import torch

CASES = {  # name: (rows, k, outliers, weight seed offset)
    "c2_a": (256, 4096, True, 0),
    "c2_b": (256, 4096, True, 1),
    "c5_dn": (64, 14336, True, 2),
    "c4_dn": (64, 9728, True, 3),
    "c3_emb": (256, 2560, False, 4),
}


def rows_bf16(case: str) -> torch.Tensor:
    """The case's rows as a bf16 tensor (round to nearest even of the f32 draw)."""
    n, k, outliers, off = CASES[case]
    rng = np.random.default_rng([0, off])
    a = rng.normal(0.0, 0.02, (n, k))
    if outliers:
        m = rng.random(a.shape) < 0.001
        a[m] = rng.normal(0.0, 0.5, int(m.sum()))
    return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)


def rows_f32(case: str) -> np.ndarray:
    """The bf16 rows widened to float32: what the reference's quantizers receive."""
    return rows_bf16(case).float().numpy()


def imatrix(k: int) -> np.ndarray:
    """Per-column importance weights of a tensor with k columns (seed 1)."""
    return np.random.default_rng(1).lognormal(0.0, 1.5, k).astype(np.float32)


def bf16_digest(case: str) -> str:
    import hashlib
    return hashlib.sha256(rows_bf16(case).view(torch.int16).numpy().tobytes()).hexdigest()
