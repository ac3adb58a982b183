"""Q4_0 through libqsb200 (replaces the reference's kernels/q4_0.py entry point)."""

from ._specs import quantizer, spec

quantize_q4_0 = quantizer("q4_0")

SPECS = {"q4_0": spec("q4_0")}
