"""Q4_K through libqsb200 (replaces the reference's kernels/q4_k.py entry point)."""

from ._specs import quantizer, spec

quantize_q4_k = quantizer("q4_k")

SPECS = {"q4_k": spec("q4_k")}
