#!/usr/bin/env python3
"""Generate the golden fixtures in this folder by running the reference quantizers.

The reference (ngxson/quant-studio) is pure Python. Its eager torch CPU path is the
ground truth for every block format here, so this script imports it from a local
checkout, feeds it seeded synthetic matrices and stores the packed bytes it returns.
It runs only where the reference checkout exists; the fixtures it writes are what the
test suite reads, so nothing at test time needs the reference.

    python tests/golden/gen_golden.py --reference /path/to/quant-studio

Outputs (all small, npz-compressed):
    inputs.npz          the input matrices (bf16 bit patterns, f32, f16) and imatrix vectors
    <type>.npz          one array of packed output rows per (input, imatrix) case
    <type>.ieee.npz     the same cases with the reference's torch.sqrt swapped for a
                        correctly rounded sqrt, stored sparsely as the rows that differ
    MANIFEST.txt        per-fixture sha256 and shapes

Why two sets: torch's float32 CPU sqrt (MKL VML on x86 builds) is not correctly
rounded; about 0.6 % of its results are 1 ulp low. Every other op in the reference is
IEEE-exact, so the .ieee fixtures pin an IEEE restatement bit for bit, while the plain
fixtures hold the reference's own output as shipped.
"""

from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
f32 = np.float32

# reference module, function, needs qw?, accepts qw=None?
TYPES = {
    "q4_0":    ("q4_0", "quantize_q4_0", False, True),
    "q2_k":    ("q2_k", "quantize_q2_k", False, True),
    "q3_k":    ("q3_k", "quantize_q3_k", False, True),
    "q4_k":    ("q4_k", "quantize_q4_k", False, True),
    "q5_k":    ("q5_k", "quantize_q5_k", False, True),
    "q6_k":    ("q6_k", "quantize_q6_k", False, True),
    "iq4_xs":  ("iq4_xs", "quantize_iq4_xs", False, True),
    "iq2_xxs": ("iq2", "quantize_iq2_xxs", True, False),
    "iq2_xs":  ("iq2_xs", "quantize_iq2_xs", True, False),
    "iq2_s":   ("iq2_s", "quantize_iq2_s", True, False),
    "iq3_xxs": ("iq3_xxs", "quantize_iq3_xxs", False, True),
    "iq3_s":   ("iq3_s", "quantize_iq3_s", False, True),
}


def _shim_gguf_enums() -> None:
    """pip gguf 0.19 lacks Q2_0 / MOSTLY_Q2_0, which the reference's scheme module names."""
    from gguf import GGMLQuantizationType as GT
    from gguf.constants import LlamaFileType as FT

    def add(cls, name, value):
        m = int.__new__(cls, value)
        m._name_ = name
        m._value_ = value
        type.__setattr__(cls, name, m)
        cls._member_map_[name] = m
        cls._value2member_map_[value] = m
        cls._member_names_.append(name)

    if not hasattr(FT, "MOSTLY_Q2_0"):
        add(FT, "MOSTLY_Q2_0", 1000)
    if not hasattr(GT, "Q2_0"):
        add(GT, "Q2_0", 1000)


def adversarial_rows(a: np.ndarray, rng: np.random.Generator) -> None:
    """Edge-case rows: the reference's own adversarial set plus zero/denormal/tie cases."""
    k = a.shape[1]
    a[0, :] = 0.0
    a[1, :] = 0.5
    a[2, :] = -0.5
    a[3, :] = 1e-6
    a[3, 7] = 8.0
    a[4, :128] = 0.25
    a[5, :] = np.abs(a[5, :])
    a[6, :] = -np.abs(a[6, :])
    a[7, :] = rng.standard_normal(k) * 1e-30            # w = x*x underflows
    a[8, :] = rng.standard_normal(k) * 1e-19            # w near the f32 tiny
    a[9, :64] = 0.0                                      # dead groups inside a live block
    a[10, :] = rng.standard_normal(k) * np.repeat(10.0 ** rng.uniform(-8, 2, k // 32), 32)
    a[11, :] = 0.01 * np.where(np.arange(k) % 2 == 0, 1.0, -1.0)   # abs-max ties
    a[12, :] = rng.choice([-0.02, -0.01, 0.0, 0.01, 0.02], k)
    a[13, :] = rng.standard_normal(k) * 20.0
    a[14, :] = -0.0
    a[15, :] = 0.0
    a[15, ::32] = rng.standard_normal(k // 32)            # one value per 32-block
    a[16, :] = np.abs(rng.standard_normal(k)) * 1e-3 + 1.0  # positive, narrow range
    a[17, :] = rng.choice([-1.0, 1.0], k) * 0.125           # constant magnitude, random signs


def make_inputs() -> dict[str, np.ndarray]:
    import torch

    rng = np.random.default_rng(20261201)
    # A: the benchmark distribution, N(0, 0.02) with 0.1 % N(0, 0.5) outliers, stored as bf16
    a = rng.normal(0.0, 0.02, (256, 1024))
    m = rng.random(a.shape) < 0.001
    a[m] = rng.normal(0.0, 0.5, int(m.sum()))
    adversarial_rows(a, rng)
    a_bf16 = torch.from_numpy(a.astype(f32)).to(torch.bfloat16)
    qw_a = rng.lognormal(0.0, 1.5, 1024).astype(f32)
    qw_a[5] = 0.0
    qw_a[100:132] = 0.0                                  # a whole 32-group with zero weight

    # B: per-row magnitude spread like the reference's GPU check, plain f32 input
    b = rng.standard_normal((64, 512)) * 0.05 * (0.2 + rng.random((64, 1)) * 3.0)
    adversarial_rows(b, rng)
    qw_b = (rng.random(512) * 4.0 + 0.05).astype(f32)

    # C: f16 input with k not a multiple of 256 (Q4_0 only)
    c = (rng.standard_normal((40, 96)) * 0.1).astype(np.float16)

    return {
        "A_bf16": a_bf16.view(torch.int16).numpy().view(np.uint16),
        "A_qw": qw_a,
        "B_f32": b.astype(f32),
        "B_qw": qw_b,
        "C_f16": c,
    }


def as_f32(inputs: dict[str, np.ndarray], name: str) -> np.ndarray:
    if name == "A":
        return (inputs["A_bf16"].astype(np.uint32) << 16).view(f32)
    if name == "B":
        return inputs["B_f32"]
    return inputs["C_f16"].astype(f32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="quant-studio checkout")
    ap.add_argument("--types", default=",".join(TYPES))
    args = ap.parse_args()

    sys.dont_write_bytecode = True                      # the checkout may be read-only
    _shim_gguf_enums()
    sys.path.insert(0, str(args.reference.resolve()))
    import importlib

    import torch

    inputs = make_inputs()
    np.savez_compressed(HERE / "inputs.npz", **inputs)
    torch_sqrt = torch.sqrt

    def ieee_sqrt(t, *a, **kw):
        """Correctly rounded float32 sqrt (numpy's), in place of torch's CPU sqrt."""
        assert t.dtype == torch.float32 and t.device.type == "cpu" and not a and not kw
        return torch.from_numpy(np.sqrt(t.contiguous().numpy()))
    manifest = [f"torch {torch.__version__} cpu_capability {torch.backends.cpu.get_cpu_capability()} "
                f"threads {torch.get_num_threads()}"]

    for tname in args.types.split(","):
        mod_name, fn_name, needs_qw, accepts_none = TYPES[tname]
        fn = getattr(importlib.import_module(f"kernels.{mod_name}"), fn_name)
        cases = [("A", "A_qw"), ("B", "B_qw")]
        if tname == "q4_0":
            cases = [("A", None), ("B", None), ("C", None)]

        def run_all():
            outs = {}
            for src, qwk in cases:
                x = torch.from_numpy(as_f32(inputs, src).copy())
                if tname == "q4_0":
                    outs[f"{src}_none"] = fn(x).numpy()
                    continue
                if accepts_none:
                    outs[f"{src}_none"] = fn(x, None).numpy()
                qw = torch.from_numpy(inputs[qwk].copy())
                outs[f"{src}_qw"] = fn(x, qw).numpy()
            return outs

        outs = run_all()
        torch.sqrt = ieee_sqrt
        try:
            outs_ieee = run_all()
        finally:
            torch.sqrt = torch_sqrt
        sparse = {}
        for key, v in outs_ieee.items():
            rows = np.nonzero((v != outs[key]).any(1))[0].astype(np.int32)
            sparse[f"{key}_rows"] = rows
            sparse[f"{key}_data"] = v[rows]
        np.savez_compressed(HERE / f"{tname}.npz", **outs)
        np.savez_compressed(HERE / f"{tname}.ieee.npz", **sparse)
        for key, v in outs.items():
            manifest.append(f"{tname}.{key} shape={v.shape} sha256={hashlib.sha256(v.tobytes()).hexdigest()[:16]}")
        print(tname, {k: v.shape for k, v in outs.items()},
              {k: len(sparse[f"{k}_rows"]) for k in outs}, flush=True)

    (HERE / "MANIFEST.txt").write_text("\n".join(manifest) + "\n")


if __name__ == "__main__":
    main()
