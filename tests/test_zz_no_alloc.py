"""qs_tensor_error_noalloc through the C ABI (GPU; this file is collected last).

The allocation-free entry point must give the same bits as qs_tensor_error on the same
inputs, on two calls in a row of each; it must work both as the first libqsb200 call of a
process (test_noalloc_first_call_in_fresh_process runs that in a child process) and after
every other test.
"""

import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from conftest import golden_cases

pytestmark = pytest.mark.gpu

# every decode the entry point runs, including each of the five IQ codebooks in its static copy
TYPE_IDS = {"q4_0": 2, "q2_k": 10, "q3_k": 11, "q4_k": 12, "q5_k": 13, "q6_k": 14, "iq2_xxs": 16, "iq2_xs": 17,
            "iq3_xxs": 18, "iq3_s": 21, "iq2_s": 22, "iq4_xs": 23}


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
    assert L.qs_tensor_error_noalloc(20, None, 144, None, 30, 4, 256, None, out.data_ptr(), None) == nat.QS_ENOTSUP
    # empty tensor: sums are zero
    assert L.qs_tensor_error_noalloc(12, None, 144, None, 30, 0, 256, None, out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [0.0, 0.0]


def test_noalloc_first_call_in_fresh_process():
    """In a new process, the allocation-free entry point is the first libqsb200 call (its
    per-device set-up runs inside it), on the committed IQ3_XXS fixture blocks; then
    qs_tensor_error on the same inputs must give the same bits."""
    code = textwrap.dedent("""
        import ctypes, sys
        import numpy as np, torch
        from conftest import golden_cases, golden_inputs
        from kernels import _native
        L = _native.lib()
        c_i64, c_vp = ctypes.c_int64, ctypes.c_void_p
        for name in ("qs_tensor_error", "qs_tensor_error_noalloc"):
            getattr(L, name).argtypes = [ctypes.c_int, c_vp, c_i64, c_vp, ctypes.c_int, c_i64, c_i64, c_vp, c_vp, c_vp]
        inputs = golden_inputs()
        key, src, qwk, ref, _ = next(c for c in golden_cases("iq3_xxs") if c[1] == "A" and c[2] is not None)
        x = torch.from_numpy(inputs["A_bf16"].view(np.int16)).view(torch.bfloat16).cuda()
        qw = torch.from_numpy(inputs[qwk]).cuda()
        blocks = torch.from_numpy(ref).cuda()
        res = []
        for name in ("qs_tensor_error_noalloc", "qs_tensor_error_noalloc", "qs_tensor_error"):
            out = torch.full((2,), float("nan"), dtype=torch.float64, device="cuda")
            rc = getattr(L, name)(18, blocks.data_ptr(), blocks.stride(0), x.data_ptr(), 30, x.shape[0], x.shape[1],
                                  qw.data_ptr(), out.data_ptr(), None)
            assert rc == 0, L.qs_last_error()
            torch.cuda.synchronize()
            res.append(out.cpu().numpy().view(np.uint64).tolist())
        assert res[0] == res[1] == res[2], res
        print("ok", res[0])
    """)
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([here, os.path.join(here, "..", "quant-studio_b200"),
                                                      os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, env=env, cwd=here)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]


def test_noalloc_rejects_pointer_on_another_memory_space():
    """blocks in host memory: an argument error before anything is enqueued."""
    L, nat = _lib()
    out = torch.zeros(2, dtype=torch.float64, device="cuda")
    host_blocks = np.zeros((4, 144), dtype=np.uint8)
    x = torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda")
    rc = L.qs_tensor_error_noalloc(12, host_blocks.ctypes.data, 144, x.data_ptr(), 30, 4, 256, None,
                                   out.data_ptr(), None)
    assert rc == nat.QS_EINVAL and b"blocks" in L.qs_last_error()
    # out must be 8-byte aligned
    rc = L.qs_tensor_error_noalloc(12, None, 144, None, 30, 0, 256, None, out.data_ptr() + 4, None)
    assert rc == nat.QS_EINVAL
