"""IQ2_XS through libqsb200 (replaces the reference's kernels/iq2_xs.py entry point)."""

from ._specs import quantizer, spec

quantize_iq2_xs = quantizer("iq2_xs")

SPECS = {"iq2_xs": spec("iq2_xs")}
