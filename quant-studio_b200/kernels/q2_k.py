"""Q2_K through libqsb200 (replaces the reference's kernels/q2_k.py entry point)."""

from ._specs import quantizer, spec

quantize_q2_k = quantizer("q2_k")

SPECS = {"q2_k": spec("q2_k")}
