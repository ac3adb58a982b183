"""Imatrix-weighted squared error of one packed block, decoded with gguf-py's dequantizer."""

import numpy as np
from gguf import GGMLQuantizationType as GT
from gguf.quants import dequantize

_GT = {"q4_0": GT.Q4_0, "q2_k": GT.Q2_K, "q3_k": GT.Q3_K, "q4_k": GT.Q4_K, "q5_k": GT.Q5_K,
       "q6_k": GT.Q6_K, "iq4_xs": GT.IQ4_XS, "iq2_xxs": GT.IQ2_XXS, "iq2_xs": GT.IQ2_XS,
       "iq2_s": GT.IQ2_S, "iq3_xxs": GT.IQ3_XXS, "iq3_s": GT.IQ3_S, "q4_1": GT.Q4_1, "q5_0": GT.Q5_0,
       "q5_1": GT.Q5_1, "q8_0": GT.Q8_0}


def block_wmse(qtype: str, blk: np.ndarray, x: np.ndarray, qw: np.ndarray | None) -> float:
    deq = dequantize(blk.reshape(1, -1), _GT[qtype]).reshape(-1).astype(np.float64)
    w = np.ones_like(deq) if qw is None else qw.astype(np.float64)
    return float((w * (deq - x.astype(np.float64)) ** 2).sum())
