"""ctypes binding of libqsb200.so, the sm_100a kernels behind include/qsb200.h.

There is no CPU or Triton fallback: if the library is missing or no CUDA device is
present, every quantize call raises.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import torch

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("QSB200_LIB", PKG_ROOT / "lib" / "libqsb200.so"))

QS_OK, QS_EINVAL, QS_ECUDA, QS_ENOTSUP, QS_ENOIMAT = 0, -1, -2, -3, -4
SRC_IDS = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 30}

_lib = None
_lock = threading.Lock()


class QsError(RuntimeError):
    """A libqsb200 call failed; `code` is the QS_E* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"qsb200 error {code}: {msg}")
        self.code = code


def build(force: bool = False) -> Path:
    """Compile libqsb200.so in-tree with the Makefile in csrc/ (nvcc, sm_100a)."""
    cmd = ["make", "-s", "-j8", "-C", str(PKG_ROOT / "csrc")]
    if force:
        subprocess.run(cmd + ["clean"], check=True)
    subprocess.run(cmd, check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise QsError(QS_ECUDA, f"{LIB_PATH} is missing; build it with kernels._native.build()")
            L = ctypes.CDLL(str(LIB_PATH))
            c_i64, c_vp = ctypes.c_int64, ctypes.c_void_p
            L.qs_version.restype = ctypes.c_int
            L.qs_init.argtypes = [ctypes.c_int]
            L.qs_type_supported.argtypes = [ctypes.c_int]
            L.qs_type_needs_qw.argtypes = [ctypes.c_int]
            L.qs_block_info.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
            L.qs_row_bytes.argtypes = [ctypes.c_int, c_i64, ctypes.POINTER(c_i64)]
            L.qs_quantize.argtypes = [ctypes.c_int, c_vp, ctypes.c_int, c_i64, c_i64, c_vp, c_vp, c_i64, c_vp]
            L.qs_dequantize.argtypes = [ctypes.c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]
            L.qs_block_error.argtypes = [ctypes.c_int, c_vp, c_i64, c_vp, ctypes.c_int, c_i64, c_i64, c_vp, c_vp, c_vp]
            L.qs_tensor_error.argtypes = [ctypes.c_int, c_vp, c_i64, c_vp, ctypes.c_int, c_i64, c_i64, c_vp, c_vp, c_vp]
            L.qs_tensor_error_noalloc.argtypes = L.qs_tensor_error.argtypes
            L.qs_device_fault.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
            L.qs_last_error.restype = ctypes.c_char_p
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != QS_OK:
        raise QsError(rc, lib().qs_last_error().decode(errors="replace"))


def row_bytes(ggml_type: int, k: int) -> int:
    out = ctypes.c_int64()
    check(lib().qs_row_bytes(int(ggml_type), int(k), ctypes.byref(out)))
    return out.value


def block_info(ggml_type: int) -> tuple[int, int]:
    qk, nb = ctypes.c_int(), ctypes.c_int()
    check(lib().qs_block_info(int(ggml_type), ctypes.byref(qk), ctypes.byref(nb)))
    return qk.value, nb.value


def quantize_into(ggml_type: int, x: torch.Tensor, qw: torch.Tensor | None, out: torch.Tensor,
                  stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Enqueue the quantization of x (n, k) into out (n, >= row_bytes) uint8 on `stream`."""
    if x.device.type != "cuda":
        raise QsError(QS_EINVAL, f"input is on {x.device}; qsb200 runs on CUDA devices only")
    if x.dtype not in SRC_IDS:
        raise QsError(QS_EINVAL, f"unsupported input dtype {x.dtype}")
    if x.dim() != 2 or not x.is_contiguous():
        raise QsError(QS_EINVAL, "input must be a contiguous (n_rows, k) tensor")
    if out.dtype != torch.uint8 or out.device != x.device or out.dim() != 2 or out.stride(1) != 1:
        raise QsError(QS_EINVAL, "out must be a row-major (n_rows, bytes) uint8 tensor on the input's device")
    qptr = None
    if qw is not None:
        if qw.device != x.device or qw.dtype != torch.float32 or not qw.is_contiguous() or qw.numel() < x.shape[1]:
            raise QsError(QS_EINVAL, "qw must be a contiguous float32 tensor of >= k values on the input's device")
        qptr = qw.data_ptr()
    if stream is None:
        stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        check(lib().qs_quantize(int(ggml_type), x.data_ptr(), SRC_IDS[x.dtype], x.shape[0], x.shape[1],
                                qptr, out.data_ptr(), out.stride(0), stream.cuda_stream))
    return out


def quantize(ggml_type: int, x: torch.Tensor, qw: torch.Tensor | None) -> torch.Tensor:
    """New (n, row_bytes) uint8 tensor on x's device: the reference's quant_fn(x) contract."""
    x = x.contiguous()
    rb = row_bytes(ggml_type, x.shape[1])
    out = torch.empty((x.shape[0], rb), dtype=torch.uint8, device=x.device)
    if qw is not None:
        qw = qw.to(device=x.device, dtype=torch.float32).contiguous()
    return quantize_into(ggml_type, x, qw, out)


def _blocks_arg(blocks: torch.Tensor, ggml_type: int) -> tuple[int, int]:
    """(n_rows, k) of a (n_rows, row_bytes) uint8 block tensor (row stride may exceed row_bytes)."""
    if blocks.device.type != "cuda":
        raise QsError(QS_EINVAL, f"blocks are on {blocks.device}; qsb200 runs on CUDA devices only")
    if blocks.dtype != torch.uint8 or blocks.dim() != 2 or blocks.stride(1) != 1:
        raise QsError(QS_EINVAL, "blocks must be a row-major (n_rows, bytes) uint8 tensor")
    qk, nb = block_info(ggml_type)
    if blocks.shape[1] % nb:
        raise QsError(QS_EINVAL, f"row of {blocks.shape[1]} bytes is not a whole number of {nb}-byte blocks")
    return blocks.shape[0], blocks.shape[1] // nb * qk


def dequantize(blocks: torch.Tensor, ggml_type: int) -> torch.Tensor:
    """Decode (n_rows, row_bytes) packed blocks to a new (n_rows, k) float32 tensor on the
    same device: the values gguf.quants.dequantize returns for the same bytes."""
    n, k = _blocks_arg(blocks, ggml_type)
    out = torch.empty((n, k + (-k) % 4), dtype=torch.float32, device=blocks.device)
    stream = torch.cuda.current_stream(blocks.device)
    with torch.cuda.device(blocks.device):
        check(lib().qs_dequantize(int(ggml_type), blocks.data_ptr(), blocks.stride(0), n, k,
                                  out.data_ptr(), out.stride(0), stream.cuda_stream))
    return out[:, :k]


def _error_args(blocks: torch.Tensor, ggml_type: int, x: torch.Tensor, qw: torch.Tensor | None):
    n, k = _blocks_arg(blocks, ggml_type)
    if x.device != blocks.device or x.dtype not in SRC_IDS or not x.is_contiguous() or tuple(x.shape) != (n, k):
        raise QsError(QS_EINVAL, f"x must be a contiguous ({n}, {k}) f32/f16/bf16 tensor on the blocks' device")
    qptr = None
    if qw is not None:
        if qw.device != x.device or qw.dtype != torch.float32 or not qw.is_contiguous() or qw.numel() < k:
            raise QsError(QS_EINVAL, "qw must be a contiguous float32 tensor of >= k values on the blocks' device")
        qptr = qw.data_ptr()
    return n, k, qptr


def block_error(blocks: torch.Tensor, ggml_type: int, x: torch.Tensor, qw: torch.Tensor | None = None) -> torch.Tensor:
    """(n_rows, k // qk) float64 tensor: per block, sum of qw * (decoded - x)^2 (qw = 1 if None)."""
    n, k, qptr = _error_args(blocks, ggml_type, x, qw)
    qk, _ = block_info(ggml_type)
    err = torch.empty((n, k // qk), dtype=torch.float64, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        check(lib().qs_block_error(int(ggml_type), blocks.data_ptr(), blocks.stride(0), x.data_ptr(), SRC_IDS[x.dtype],
                                   n, k, qptr, err.data_ptr(), stream.cuda_stream))
    return err


def tensor_error(blocks: torch.Tensor, ggml_type: int, x: torch.Tensor, qw: torch.Tensor | None = None) -> torch.Tensor:
    """float64 device tensor [sum qw (decoded - x)^2, sum (decoded - x)^2] over the tensor,
    summed in a fixed order (bit-identical across calls)."""
    n, k, qptr = _error_args(blocks, ggml_type, x, qw)
    out = torch.empty(2, dtype=torch.float64, device=x.device)
    stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        check(lib().qs_tensor_error(int(ggml_type), blocks.data_ptr(), blocks.stride(0), x.data_ptr(), SRC_IDS[x.dtype],
                                    n, k, qptr, out.data_ptr(), stream.cuda_stream))
    return out
