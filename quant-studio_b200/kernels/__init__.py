"""qs-b200 kernel registry: the reference's `kernels` package API over libqsb200.

QUANT_TYPES maps a type name to its QuantSpec exactly like the reference
(kernels/__init__.py:18-27); every kernel runs on a CUDA device through the C ABI in
include/qsb200.h.
"""

import importlib

from .common import QuantSpec, TORCH_DTYPES

QUANT_TYPES: dict[str, QuantSpec] = {}
for _m in ("iq2", "iq2_s", "iq2_xs", "iq3_s", "iq3_xxs", "iq4_xs",
           "q2_k", "q3_k", "q4_0", "q4_k", "q5_k", "q6_k"):
    QUANT_TYPES.update(importlib.import_module(f".{_m}", __package__).SPECS)
