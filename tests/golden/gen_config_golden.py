#!/usr/bin/env python3
"""Run the reference quantizers on row subsets of the benchmark configurations and record
what they return, as shipped and with a correctly rounded sqrt (config_parity.json).

    python tests/golden/gen_config_golden.py --reference /path/to/quant-studio

The reference (ngxson/quant-studio) is pure Python; its eager torch CPU path is the ground
truth. It runs only where the reference checkout exists. For every (type, case) the file
holds the sha256 of the packed output of the reference as shipped and of the reference with
torch.sqrt replaced by numpy's correctly rounded sqrt, plus every block where the two differ
(both byte strings). Blocks are identical everywhere else, so the tests can rebuild the
as-shipped output from any output that matches the IEEE-sqrt one. Each differing block also
carries its squared error, weighted by the importance matrix and by the search's own weight
(qw * sqrt(sigma2 + x^2), the quantity the reference's scale searches minimise), for both
versions, and every case the aggregate of both over all its blocks.

Why two sets: torch's float32 CPU sqrt (MKL VML on x86 builds) is not correctly rounded;
about 0.6 % of its results are 1 ulp low, and a near tie in a scale search can then tip to
a neighbouring candidate. Everything else the reference computes is IEEE-exact.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

import config_rows  # noqa: E402
from gen_golden import TYPES, _shim_gguf_enums  # noqa: E402

# (type, case) pairs: every configured type on the configs[1] rows (imatrix), the types of the
# configs[4] mixes on 8B ffn_down rows, Q4_K / Q6_K on 4B ffn_down rows, Q4_0 on the
# configs[2] embedding rows and on edge rows (no imatrix)
PAIRS = ([(t, c) for c in ("c2_a", "c2_b") for t in ("q2_k", "q3_k", "q4_k", "q5_k", "q6_k", "iq4_xs", "iq2_xxs",
                                                     "iq2_xs", "iq2_s", "iq3_xxs", "iq3_s")]
         + [(t, "c5_dn") for t in ("iq3_xxs", "iq3_s", "iq2_s", "iq2_xxs", "q4_k", "q5_k")]
         + [(t, "c4_dn") for t in ("q4_k", "q6_k")]
         + [("q4_0", "c3_emb"), ("q4_0", "edge")])

# sigma2 factor of the search weight qw * sqrt(f * sum(x^2) / 256 + x^2) per type
# (kernels/<type>.py of the reference); Q6_K's search weight is qw itself
SEARCH_SIGMA = {"q2_k": 1.0, "q3_k": 2.0, "q4_k": 2.0, "q5_k": 2.0, "iq4_xs": 2.0, "iq2_xxs": 1.0, "iq2_xs": 1.0,
                "iq2_s": 2.0, "iq3_xxs": 2.0, "iq3_s": 2.0}


def case_rows(case: str) -> np.ndarray:
    if case == "edge":
        from test_oracle_legacy import adversarial_rows
        import torch
        return torch.from_numpy(adversarial_rows(256)).to(torch.bfloat16).float().numpy()
    return config_rows.rows_f32(case)


def search_weight(qtype: str, x: np.ndarray, qw: np.ndarray | None) -> np.ndarray:
    """Per value: the weight the reference's search minimises (float64, IEEE sqrt)."""
    if qw is None:
        return np.ones_like(x, dtype=np.float64)
    q = np.broadcast_to(qw[None, :], x.shape).astype(np.float64)
    if qtype not in SEARCH_SIGMA:
        return q
    sb = x.astype(np.float64).reshape(x.shape[0], -1, 256)
    sigma2 = SEARCH_SIGMA[qtype] * (sb * sb).sum(-1, keepdims=True) / 256.0
    return q * np.sqrt(sigma2 + sb * sb).reshape(x.shape)


def block_errors(qtype: str, blocks: np.ndarray, x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """sum w * (deq - x)^2 per block, float64, blocks decoded with gguf-py."""
    from wmse import _GT
    from gguf.quants import dequantize
    deq = dequantize(blocks, _GT[qtype]).astype(np.float64).reshape(x.shape)
    qk = 32 if qtype == "q4_0" else 256
    return (w * (deq - x.astype(np.float64)) ** 2).reshape(x.shape[0], -1, qk).sum(-1).reshape(-1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="quant-studio checkout")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    _shim_gguf_enums()
    sys.path.insert(0, str(args.reference.resolve()))
    import importlib

    import torch

    torch_sqrt = torch.sqrt

    def ieee_sqrt(t, *a, **kw):
        assert t.dtype == torch.float32 and t.device.type == "cpu" and not a and not kw
        return torch.from_numpy(np.sqrt(t.contiguous().numpy()))

    out = {"meta": {"torch": torch.__version__, "cpu_capability": torch.backends.cpu.get_cpu_capability(),
                    "threads": torch.get_num_threads()},
           "inputs": {c: config_rows.bf16_digest(c) for c in config_rows.CASES}, "cases": {}}
    for qtype, case in PAIRS:
        mod_name, fn_name, _needs, _none = TYPES[qtype]
        fn = getattr(importlib.import_module(f"kernels.{mod_name}"), fn_name)
        x = case_rows(case)
        qw = None if qtype == "q4_0" else config_rows.imatrix(x.shape[1])

        def run():
            xt = torch.from_numpy(x.copy())
            return (fn(xt) if qtype == "q4_0" else fn(xt, torch.from_numpy(qw.copy()))).numpy()

        shipped = run()
        torch.sqrt = ieee_sqrt
        try:
            ieee = run()
        finally:
            torch.sqrt = torch_sqrt
        qk = 32 if qtype == "q4_0" else 256
        nb = x.size // qk
        a, b = ieee.reshape(nb, -1), shipped.reshape(nb, -1)
        diff = np.nonzero((a != b).any(1))[0]
        wq = search_weight(qtype, x, None) if qw is None else np.broadcast_to(qw[None, :], x.shape).astype(np.float64)
        ws = search_weight(qtype, x, qw)
        eq_i, eq_s = block_errors(qtype, ieee, x, wq), block_errors(qtype, shipped, x, wq)
        es_i, es_s = block_errors(qtype, ieee, x, ws), block_errors(qtype, shipped, x, ws)
        out["cases"][f"{qtype}/{case}"] = {
            "type": qtype, "case": case, "imatrix": qw is not None, "blocks": int(nb),
            "sha_ieee": hashlib.sha256(ieee.tobytes()).hexdigest(),
            "sha_shipped": hashlib.sha256(shipped.tobytes()).hexdigest(),
            "identical_fraction": round(1.0 - diff.size / nb, 6),
            "agg_wmse_qw": [float(eq_i.sum()), float(eq_s.sum())],
            "agg_wmse_search": [float(es_i.sum()), float(es_s.sum())],
            "diff": [{"block": int(i), "ieee": a[i].tobytes().hex(), "shipped": b[i].tobytes().hex(),
                      "wmse_qw": [float(eq_i[i]), float(eq_s[i])],
                      "wmse_search": [float(es_i[i]), float(es_s[i])]} for i in diff],
        }
        print(f"{qtype}/{case}: {nb} blocks, {diff.size} differ", flush=True)
    (HERE / "config_parity.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
