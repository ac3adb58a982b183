"""IQ3_S through libqsb200 (replaces the reference's kernels/iq3_s.py entry point)."""

from ._specs import quantizer, spec

quantize_iq3_s = quantizer("iq3_s")

SPECS = {"iq3_s": spec("iq3_s")}
