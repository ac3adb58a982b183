"""The kernels registry mirrors the reference's QUANT_TYPES entries (kernels/*.py SPECS)."""

from gguf import GGMLQuantizationType as GT
from gguf.constants import LlamaFileType as FT

import kernels

# name: (ggml type, ftype, needs_imatrix, uses_imatrix) as in the reference's SPECS
EXPECTED = {
    "q4_0": (GT.Q4_0, FT.MOSTLY_Q4_0, False, False),
    "q2_k": (GT.Q2_K, FT.MOSTLY_Q2_K, False, True),
    "q3_k": (GT.Q3_K, FT.MOSTLY_Q3_K_M, False, True),
    "q4_k": (GT.Q4_K, FT.MOSTLY_Q4_K_M, False, True),
    "q5_k": (GT.Q5_K, FT.MOSTLY_Q5_K_M, False, True),
    "q6_k": (GT.Q6_K, FT.MOSTLY_Q6_K, False, True),
    "iq4_xs": (GT.IQ4_XS, FT.MOSTLY_IQ4_XS, False, True),
    "iq2_xxs": (GT.IQ2_XXS, FT.MOSTLY_IQ2_XXS, True, True),
    "iq2_xs": (GT.IQ2_XS, FT.MOSTLY_IQ2_XS, True, True),
    "iq2_s": (GT.IQ2_S, FT.MOSTLY_IQ2_S, True, True),
    "iq3_xxs": (GT.IQ3_XXS, FT.MOSTLY_IQ3_XXS, True, True),
    "iq3_s": (GT.IQ3_S, FT.MOSTLY_IQ3_S, False, True),
    # not in the reference's registry (no kernel there); the same flags as its Q4_0
    "q4_1": (GT.Q4_1, FT.MOSTLY_Q4_1, False, False),
    "q5_0": (GT.Q5_0, FT.MOSTLY_Q5_0, False, False),
    "q5_1": (GT.Q5_1, FT.MOSTLY_Q5_1, False, False),
    "q8_0": (GT.Q8_0, FT.MOSTLY_Q8_0, False, False),
}


def test_registry_matches_reference():
    assert set(kernels.QUANT_TYPES) == set(EXPECTED)
    for name, (gt, ft, needs, uses) in EXPECTED.items():
        s = kernels.QUANT_TYPES[name]
        assert (s.ggml_type, s.ftype, s.needs_imatrix, s.uses_imatrix) == (gt, ft, needs, uses), name
        assert callable(s.make_kernel)


def test_torch_dtypes():
    import torch
    assert kernels.TORCH_DTYPES == {GT.F32: torch.float32, GT.F16: torch.float16, GT.BF16: torch.bfloat16}


def test_entry_point_names():
    from kernels.iq2 import quantize_iq2_xxs
    from kernels.q4_0 import quantize_q4_0
    from kernels.q4_k import quantize_q4_k
    assert quantize_q4_0.__name__ == "quantize_q4_0" and callable(quantize_q4_k) and callable(quantize_iq2_xxs)
