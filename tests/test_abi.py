"""The C ABI library: loads, exports what include/qsb200.h declares, argument checks.
None of these calls touch a GPU."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch
from gguf.constants import GGML_QUANT_SIZES

from conftest import ROOT
from kernels import _native

HEADER = ROOT / "include" / "qsb200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(qs_\w+)\s*\(", text, re.M)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for n in ("qs_quantize", "qs_init", "qs_row_bytes", "qs_block_info", "qs_last_error",
              "qs_type_supported", "qs_type_needs_qw", "qs_version", "qs_dequantize", "qs_block_error",
              "qs_tensor_error", "qs_tensor_error_noalloc", "qs_device_fault"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for n in declared_functions():
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (qs_\w+)", out))
    assert set(declared_functions()) <= exported


def test_version():
    assert _native.lib().qs_version() == 1


@pytest.mark.parametrize("name", ["Q4_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ4_XS",
                                  "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS", "IQ3_S", "Q4_1", "Q5_0", "Q5_1", "Q8_0"])
def test_block_geometry_matches_gguf(name):
    from gguf import GGMLQuantizationType as GT
    gt = GT[name]
    assert _native.lib().qs_type_supported(int(gt)) == 1
    assert _native.block_info(int(gt)) == GGML_QUANT_SIZES[gt]
    qk, nb = GGML_QUANT_SIZES[gt]
    assert _native.row_bytes(int(gt), 4096 if qk == 256 else 96) == (4096 if qk == 256 else 96) // qk * nb


def test_needs_qw_flags():
    L = _native.lib()
    assert [t for t in (2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 16, 17, 18, 21, 22, 23) if L.qs_type_needs_qw(t)] == [16, 17, 22]


def test_argument_errors():
    L = _native.lib()
    with pytest.raises(_native.QsError) as e:
        _native.row_bytes(20, 256)                     # IQ4_NL: not implemented
    assert e.value.code == _native.QS_ENOTSUP
    with pytest.raises(_native.QsError) as e:
        _native.row_bytes(12, 300)                     # not a multiple of 256
    assert e.value.code == _native.QS_EINVAL and "300" in str(e.value)
    # qs_quantize rejects before touching CUDA
    assert L.qs_quantize(12, None, 30, 4, 250, None, None, 0, None) == _native.QS_EINVAL
    assert L.qs_quantize(12, None, 5, 4, 256, None, None, 144, None) == _native.QS_EINVAL
    assert L.qs_quantize(16, None, 30, 4, 256, None, None, 66, None) == _native.QS_ENOIMAT
    assert L.qs_quantize(12, None, 30, 4, 256, None, None, 100, None) == _native.QS_EINVAL
    assert L.qs_quantize(12, None, 30, 0, 256, None, None, 144, None) == _native.QS_OK
    assert b"dst_row_bytes" in L.qs_last_error() or L.qs_last_error() == b""


def test_cpu_tensor_is_rejected_not_fallen_back():
    with pytest.raises(_native.QsError):
        _native.quantize(12, torch.zeros(2, 256), None)


def test_decode_argument_errors():
    """The decode entry points reject bad geometry before touching CUDA."""
    L = _native.lib()
    assert L.qs_dequantize(12, None, 144, 4, 250, None, 256, None) == _native.QS_EINVAL   # k % 256
    assert L.qs_dequantize(12, None, 100, 4, 256, None, 256, None) == _native.QS_EINVAL   # row stride
    assert L.qs_dequantize(12, None, 144, 4, 256, None, 255, None) == _native.QS_EINVAL   # dst stride
    assert L.qs_dequantize(20, None, 144, 4, 256, None, 256, None) == _native.QS_ENOTSUP
    assert L.qs_dequantize(12, None, 144, 0, 256, None, 256, None) == _native.QS_OK       # nothing to do
    assert L.qs_block_error(12, None, 144, None, 5, 4, 256, None, None, None) == _native.QS_EINVAL
    assert L.qs_block_error(12, None, 144, None, 30, 0, 256, None, None, None) == _native.QS_OK
    assert L.qs_tensor_error(12, None, 144, None, 30, 4, 256, None, None, None) == _native.QS_EINVAL  # null out


def test_cpu_blocks_are_rejected():
    with pytest.raises(_native.QsError):
        _native.dequantize(torch.zeros((2, 144), dtype=torch.uint8), 12)
