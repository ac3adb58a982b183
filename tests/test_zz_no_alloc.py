"""qs_tensor_error_noalloc through the C ABI (GPU; this file is collected last).

The allocation-free entry point must give the same bits as qs_tensor_error on the same
inputs, on two calls in a row of each; it must work both as the first libqsb200 call of a
process (its set-up then runs here) and after every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import golden_cases

pytestmark = pytest.mark.gpu

TYPE_IDS = {"q4_0": 2, "q2_k": 10, "q4_k": 12, "q6_k": 14, "iq2_xxs": 16, "iq3_s": 21, "iq4_xs": 23}


def _lib():
    from kernels import _native
    L = _native.lib()
    c_i64, c_vp = ctypes.c_int64, ctypes.c_void_p
    for name in ("qs_tensor_error", "qs_tensor_error_noalloc"):
        getattr(L, name).argtypes = [ctypes.c_int, c_vp, c_i64, c_vp, ctypes.c_int, c_i64, c_i64, c_vp, c_vp, c_vp]
    return L, _native


def _both(gt: int, blocks: torch.Tensor, x: torch.Tensor, qw):
    """[existing, existing, noalloc, noalloc] results as float64 bit patterns."""
    L, nat = _lib()
    src = nat.SRC_IDS[x.dtype]
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for name in ("qs_tensor_error", "qs_tensor_error", "qs_tensor_error_noalloc", "qs_tensor_error_noalloc"):
        out = torch.full((2,), float("nan"), dtype=torch.float64, device=x.device)
        rc = getattr(L, name)(gt, blocks.data_ptr(), blocks.stride(0), x.data_ptr(), src, x.shape[0], x.shape[1],
                              None if qw is None else qw.data_ptr(), out.data_ptr(), stream)
        assert rc == 0, L.qs_last_error()
        outs.append(out.cpu().numpy().view(np.uint64).tolist())
    return outs


@pytest.mark.parametrize("qtype", list(TYPE_IDS))
def test_noalloc_matches_existing_on_golden(qtype, inputs):
    for key, src, qwk, ref, _ in golden_cases(qtype):
        if src == "A":
            x = torch.from_numpy(inputs["A_bf16"].view(np.int16)).view(torch.bfloat16).cuda()
        elif src == "B":
            x = torch.from_numpy(inputs["B_f32"]).cuda()
        else:
            x = torch.from_numpy(inputs["C_f16"]).cuda()
        qw = None if qwk is None else torch.from_numpy(inputs[qwk]).cuda()
        r = _both(TYPE_IDS[qtype], torch.from_numpy(ref).cuda(), x, qw)
        assert r[0] == r[1] == r[2] == r[3], f"{qtype}/{key}: {r}"


def test_noalloc_matches_existing_at_full_occupancy():
    """A tensor large enough that the launch uses its full grid (8 CTAs per SM)."""
    _, nat = _lib()
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    x = (torch.randn((4096, 4096), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    qw = torch.rand(4096, device="cuda", generator=g) + 0.05
    blocks = nat.quantize(12, x, qw)
    r = _both(12, blocks, x, qw)
    assert r[0] == r[1] == r[2] == r[3]
    assert np.isfinite(np.array(r[2], dtype=np.uint64).view(np.float64)).all()


def test_noalloc_argument_errors():
    L, nat = _lib()
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    assert L.qs_tensor_error_noalloc(12, None, 144, None, 30, 4, 250, None, out.data_ptr(), None) == nat.QS_EINVAL
    assert L.qs_tensor_error_noalloc(12, None, 144, None, 30, 4, 256, None, None, None) == nat.QS_EINVAL
    assert L.qs_tensor_error_noalloc(7, None, 144, None, 30, 4, 256, None, out.data_ptr(), None) == nat.QS_ENOTSUP
    # empty tensor: sums are zero
    assert L.qs_tensor_error_noalloc(12, None, 144, None, 30, 0, 256, None, out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [0.0, 0.0]
