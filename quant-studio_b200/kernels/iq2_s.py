"""IQ2_S through libqsb200 (replaces the reference's kernels/iq2_s.py entry point)."""

from ._specs import quantizer, spec

quantize_iq2_s = quantizer("iq2_s")

SPECS = {"iq2_s": spec("iq2_s")}
