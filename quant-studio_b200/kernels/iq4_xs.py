"""IQ4_XS through libqsb200 (replaces the reference's kernels/iq4_xs.py entry point)."""

from ._specs import quantizer, spec

quantize_iq4_xs = quantizer("iq4_xs")

SPECS = {"iq4_xs": spec("iq4_xs")}
