"""Q5_K through libqsb200 (replaces the reference's kernels/q5_k.py entry point)."""

from ._specs import quantizer, spec

quantize_q5_k = quantizer("q5_k")

SPECS = {"q5_k": spec("q5_k")}
