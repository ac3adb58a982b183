"""CPU oracle for the GGML block quantizers: TEST INFRASTRUCTURE ONLY.

A plain-C restatement (qs_oracle.c) of the reference's eager torch path, loaded with
ctypes. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
it, and only as the checker or the timed CPU baseline; the product never calls it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

TYPE_IDS = {"q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8, "q2_k": 10, "q3_k": 11, "q4_k": 12, "q5_k": 13, "q6_k": 14,
            "iq2_xxs": 16, "iq2_xs": 17, "iq3_xxs": 18, "iq3_s": 21, "iq2_s": 22, "iq4_xs": 23}

_lib = None


def build() -> Path:
    """Compile liboracle.so with the Makefile beside this file (gcc, strict IEEE flags)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.oq_quantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.oq_quantize.restype = ctypes.c_int
        L.oq_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int64]
        L.oq_row_bytes.restype = ctypes.c_int64
        _lib = L
    return _lib


def row_bytes(qtype: str, k: int) -> int:
    return int(lib().oq_row_bytes(TYPE_IDS[qtype], k))


def quantize(qtype: str, x: np.ndarray, qw: np.ndarray | None = None, nthreads: int | None = None) -> np.ndarray:
    """x: (n, k) float32 rows; qw: (k,) float32 or None. Returns (n, row_bytes) uint8."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = x.shape
    rb = row_bytes(qtype, k)
    if rb < 0:
        raise ValueError(f"{qtype}: row length {k} is not a multiple of the block size")
    out = np.empty((n, rb), dtype=np.uint8)
    qwp = None
    if qw is not None:
        qw = np.ascontiguousarray(qw[:k], dtype=np.float32)
        qwp = qw.ctypes.data
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    rc = lib().oq_quantize(TYPE_IDS[qtype], x.ctypes.data, n, k, qwp, out.ctypes.data, nthreads)
    if rc != 0:
        raise ValueError(f"oracle rejected {qtype} (rc={rc})")
    return out
