"""IQ2_XXS through libqsb200 (replaces the reference's kernels/iq2.py entry point)."""

from ._specs import quantizer, spec

_q = quantizer("iq2_xxs")


def quantize_iq2_xxs(x, qw, T=None):
    """Same signature as the reference; T (its host-side table cache) is accepted and ignored:
    the lattice tables live on each device inside libqsb200."""
    return _q(x, qw)


SPECS = {"iq2_xxs": spec("iq2_xxs")}
