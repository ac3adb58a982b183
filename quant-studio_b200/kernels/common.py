"""Shared pieces of the kernel registry (mirrors kernels/common.py of the reference)."""

from __future__ import annotations

import torch
from gguf import GGMLQuantizationType
from gguf.constants import LlamaFileType

F32_TINY = torch.finfo(torch.float32).tiny

# source tensor types the quantizers accept (reference: kernels/common.py:20-24)
TORCH_DTYPES = {
    GGMLQuantizationType.F32: torch.float32,
    GGMLQuantizationType.F16: torch.float16,
    GGMLQuantizationType.BF16: torch.bfloat16,
}


class QuantSpec:
    """One output type: same fields and meaning as the reference's QuantSpec
    (kernels/common.py:27-37). make_kernel(device, qw) returns fn(x) -> uint8 rows."""

    def __init__(self, ggml_type: GGMLQuantizationType, ftype: LlamaFileType,
                 bytes_per_elem: int, needs_imatrix: bool, make_kernel,
                 uses_imatrix: bool | None = None):
        self.ggml_type = ggml_type
        self.ftype = ftype
        self.bytes_per_elem = bytes_per_elem  # --mem chunk heuristic, bytes of working set per value
        self.needs_imatrix = needs_imatrix
        self.make_kernel = make_kernel
        self.uses_imatrix = needs_imatrix if uses_imatrix is None else uses_imatrix
