"""IQ3_XXS through libqsb200 (replaces the reference's kernels/iq3_xxs.py entry point)."""

from ._specs import quantizer, spec

quantize_iq3_xxs = quantizer("iq3_xxs")

SPECS = {"iq3_xxs": spec("iq3_xxs")}
