"""qs-b200 kernel registry: the reference's `kernels` package API over libqsb200.

QUANT_TYPES maps a type name to its QuantSpec exactly like the reference
(kernels/__init__.py:18-27); every kernel runs on a CUDA device through the C ABI in
include/qsb200.h.

The reference spreads its entry points over one module per type (kernels/q4_k.py
`quantize_q4_k`, kernels/iq2.py `quantize_iq2_xxs`, ...). Here every type is the same
call into the library, so those modules are not files: each is created below as a module
object holding `quantize_<type>` and `SPECS`, under the reference's module name, so that
`from kernels.q4_k import quantize_q4_k` keeps working.
"""

import sys
import types

from . import _specs
from .common import QuantSpec, TORCH_DTYPES

# reference module name -> the type names it provides
MODULES = {
    "q4_0": ("q4_0",), "q2_k": ("q2_k",), "q3_k": ("q3_k",), "q4_k": ("q4_k",), "q5_k": ("q5_k",),
    "q6_k": ("q6_k",), "iq4_xs": ("iq4_xs",), "iq2": ("iq2_xxs",), "iq2_xs": ("iq2_xs",),
    "iq2_s": ("iq2_s",), "iq3_xxs": ("iq3_xxs",), "iq3_s": ("iq3_s",),
    # formats the reference's policy selects but has no module for
    "q4_1": ("q4_1",), "q5_0": ("q5_0",), "q5_1": ("q5_1",), "q8_0": ("q8_0",),
}

QUANT_TYPES: dict[str, QuantSpec] = {}
for _mod, _names in MODULES.items():
    _m = types.ModuleType(f"{__name__}.{_mod}", f"{', '.join(n.upper() for n in _names)} through libqsb200")
    _m.SPECS = {}
    for _n in _names:
        setattr(_m, f"quantize_{_n}", _specs.quantizer(_n))
        _m.SPECS[_n] = _specs.spec(_n)
    sys.modules[_m.__name__] = _m
    globals()[_mod] = _m
    QUANT_TYPES.update(_m.SPECS)
