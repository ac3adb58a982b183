"""Q6_K through libqsb200 (replaces the reference's kernels/q6_k.py entry point)."""

from ._specs import quantizer, spec

quantize_q6_k = quantizer("q6_k")

SPECS = {"q6_k": spec("q6_k")}
