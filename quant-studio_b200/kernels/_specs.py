"""One table for the output types: GGML id, file type, imatrix flags (values of the
reference's per-module SPECS, e.g. kernels/q4_k.py:86-89, kernels/iq2.py:506-509)."""

from __future__ import annotations

from gguf import GGMLQuantizationType as GT
from gguf.constants import LlamaFileType as FT

from . import _native
from .common import QuantSpec

# device working set per source value: the source element (<= 4 B) plus the packed output
BYTES_PER_ELEM = 5

# name: (ggml type, file type, needs_imatrix, uses_imatrix)
TYPES = {
    "q4_0": (GT.Q4_0, FT.MOSTLY_Q4_0, False, False),
    "q2_k": (GT.Q2_K, FT.MOSTLY_Q2_K, False, True),
    "q3_k": (GT.Q3_K, FT.MOSTLY_Q3_K_M, False, True),
    "q4_k": (GT.Q4_K, FT.MOSTLY_Q4_K_M, False, True),
    "q5_k": (GT.Q5_K, FT.MOSTLY_Q5_K_M, False, True),
    "q6_k": (GT.Q6_K, FT.MOSTLY_Q6_K, False, True),
    "iq4_xs": (GT.IQ4_XS, FT.MOSTLY_IQ4_XS, False, True),
    "iq2_xxs": (GT.IQ2_XXS, FT.MOSTLY_IQ2_XXS, True, True),
    "iq2_xs": (GT.IQ2_XS, FT.MOSTLY_IQ2_XS, True, True),
    "iq2_s": (GT.IQ2_S, FT.MOSTLY_IQ2_S, True, True),
    "iq3_xxs": (GT.IQ3_XXS, FT.MOSTLY_IQ3_XXS, True, True),
    "iq3_s": (GT.IQ3_S, FT.MOSTLY_IQ3_S, False, True),
    # no kernel in the reference (its policy selects them: kernels/scheme.py:375, :521-523);
    # like its Q4_0 they ignore importance weights
    "q4_1": (GT.Q4_1, FT.MOSTLY_Q4_1, False, False),
    "q5_0": (GT.Q5_0, FT.MOSTLY_Q5_0, False, False),
    "q5_1": (GT.Q5_1, FT.MOSTLY_Q5_1, False, False),
    "q8_0": (GT.Q8_0, FT.MOSTLY_Q8_0, False, False),
}


def quantizer(name: str):
    """quantize_<name>(x, qw=None): x (n, k) f32/f16/bf16 on a CUDA device -> new uint8 rows.

    The reference's quantize_iq2_xxs also takes `T`, its host-side table cache
    (kernels/iq2.py:418); it is accepted and ignored here, since the lattice tables live on
    each device inside libqsb200."""
    gt = TYPES[name][0]

    def fn(x, qw=None, T=None):
        return _native.quantize(int(gt), x, qw)

    fn.__name__ = f"quantize_{name}"
    fn.__qualname__ = fn.__name__
    fn.__doc__ = (f"x: (n_rows, k) float32/float16/bfloat16 CUDA tensor; qw: (k,) float32 importance "
                  f"weights or None. Returns (n_rows, k // QK * block_bytes) uint8 on x's device.")
    return fn


def spec(name: str) -> QuantSpec:
    gt, ft, needs, uses = TYPES[name]
    fn = quantizer(name)

    def make_kernel(device, qw):
        return lambda x: fn(x, qw)

    return QuantSpec(gt, ft, BYTES_PER_ELEM, needs, make_kernel, uses_imatrix=uses)
