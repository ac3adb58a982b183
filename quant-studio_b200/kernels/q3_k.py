"""Q3_K through libqsb200 (replaces the reference's kernels/q3_k.py entry point)."""

from ._specs import quantizer, spec

quantize_q3_k = quantizer("q3_k")

SPECS = {"q3_k": spec("q3_k")}
