"""Block decode and decode-error checkers on the GPU, through the C ABI.

Decode parity: every value bit-identical to gguf-py's gguf.quants.dequantize (the
decode of the reference's correctness harness, tools/dev_harness.py:108-109) on the
golden fixture blocks and on random blocks of every format. Error checkers: per-block
and whole-tensor sums of qw * (deq - x)^2 against the same definition restated in numpy
(float32 terms and runs of 8, double above; relative 1e-12 since only the association
of the double additions differs), and the tensor sums bit-identical from call to call.
"""

import numpy as np
import pytest
import torch

from conftest import ALL_TYPES, golden_cases, golden_x

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as GT  # noqa: E402
from gguf.quants import dequantize as gguf_dequantize  # noqa: E402

pytestmark = pytest.mark.gpu

GTYPE = {t: getattr(GT, t.upper()) for t in ALL_TYPES}
# byte offsets of the fp16 scale fields in each block (kept finite in random blocks)
F16_FIELDS = {"q4_0": (0,), "q2_k": (80, 82), "q3_k": (108,), "q4_k": (0, 2), "q5_k": (0, 2), "q6_k": (208,),
              "iq4_xs": (0,), "iq2_xxs": (0,), "iq2_xs": (0,), "iq2_s": (0,), "iq3_xxs": (0,), "iq3_s": (0,)}


def _native():
    from kernels import _native
    return _native


def _bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _random_blocks(qtype: str, n_rows: int, k: int, seed: int) -> np.ndarray:
    qk, bb = gguf.GGML_QUANT_SIZES[GTYPE[qtype]]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(n_rows, k // qk, bb), dtype=np.uint8)
    for off in F16_FIELDS[qtype]:
        d = (rng.standard_normal((n_rows, k // qk)) * 0.01).astype(np.float16)
        b[..., off:off + 2] = d.view(np.uint8).reshape(n_rows, k // qk, 2)
    return b.reshape(n_rows, -1)


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_decode_matches_gguf_on_golden_blocks(qtype):
    for key, src, _, ref, _ in golden_cases(qtype):
        got = _native().dequantize(torch.from_numpy(ref).cuda(), int(GTYPE[qtype])).cpu().numpy()
        want = gguf_dequantize(ref, GTYPE[qtype])
        assert got.shape == want.shape, key
        assert np.array_equal(_bits(got), _bits(want)), f"{qtype}/{key}"


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_decode_matches_gguf_on_random_blocks(qtype):
    qk = gguf.GGML_QUANT_SIZES[GTYPE[qtype]][0]
    k = qk * (5 if qk == 32 else 3)  # tiles span rows
    blocks = _random_blocks(qtype, 37, k, seed=hash(qtype) % 1000)
    got = _native().dequantize(torch.from_numpy(blocks).cuda(), int(GTYPE[qtype])).cpu().numpy()
    want = gguf_dequantize(blocks, GTYPE[qtype])
    assert np.array_equal(_bits(got), _bits(want)), qtype


@pytest.mark.parametrize("qtype", ["q4_0", "q4_k", "iq3_s"])
def test_decode_strided_rows(qtype):
    qk, bb = gguf.GGML_QUANT_SIZES[GTYPE[qtype]]
    k = qk * 4
    blocks = _random_blocks(qtype, 9, k, seed=3)
    wide = torch.zeros((9, blocks.shape[1] + 40), dtype=torch.uint8)
    wide[:, :blocks.shape[1]] = torch.from_numpy(blocks)
    got = _native().dequantize(wide.cuda()[:, :blocks.shape[1]], int(GTYPE[qtype])).cpu().numpy()
    want = gguf_dequantize(blocks, GTYPE[qtype])
    assert np.array_equal(_bits(got), _bits(want))


def test_decode_empty_and_errors():
    nat = _native()
    empty = torch.empty((0, 144), dtype=torch.uint8, device="cuda")
    assert nat.dequantize(empty, 12).shape == (0, 256)
    with pytest.raises(nat.QsError):
        nat.dequantize(torch.zeros((2, 145), dtype=torch.uint8, device="cuda"), 12)


def _runs8(t: np.ndarray) -> np.ndarray:
    """float32 sums of each run of 8 consecutive values, left to right, as float64."""
    t = t.reshape(t.shape[0], -1, 8)
    s = t[..., 0].copy()
    for j in range(1, 8):
        s = s + t[..., j]
    return s.astype(np.float64)


def _ref_errors(deq: np.ndarray, x: np.ndarray, qw, qk: int):
    """The checkers' definition: float32 terms, float32 runs of 8, double above."""
    e = deq.astype(np.float32) - x.astype(np.float32)
    ee = e * e
    we = ee if qw is None else qw.astype(np.float32)[None, :] * ee
    rw, r = _runs8(we), _runs8(ee)
    blk = rw.reshape(x.shape[0], -1, qk // 8).sum(-1)
    return blk, rw.sum(), r.sum()


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_block_and_tensor_error(qtype, inputs):
    nat = _native()
    qk = gguf.GGML_QUANT_SIZES[GTYPE[qtype]][0]
    for key, src, qwk, ref, _ in golden_cases(qtype):
        x = golden_x(inputs, src)
        qw = inputs[qwk] if qwk else None
        deq = gguf_dequantize(ref, GTYPE[qtype])
        want_blk, want_w, want = _ref_errors(deq, x, qw, qk)
        if src == "A":
            xt = torch.from_numpy(inputs["A_bf16"].view(np.int16)).view(torch.bfloat16).cuda()
        elif src == "B":
            xt = torch.from_numpy(x).cuda()
        else:
            xt = torch.from_numpy(inputs["C_f16"]).cuda()
        bt = torch.from_numpy(ref).cuda()
        qwt = None if qw is None else torch.from_numpy(qw).cuda()
        blk = nat.block_error(bt, int(GTYPE[qtype]), xt, qwt).cpu().numpy()
        np.testing.assert_allclose(blk, want_blk, rtol=1e-12, atol=0, err_msg=f"{qtype}/{key}")
        t1 = nat.tensor_error(bt, int(GTYPE[qtype]), xt, qwt).cpu().numpy()
        t2 = nat.tensor_error(bt, int(GTYPE[qtype]), xt, qwt).cpu().numpy()
        assert t1.view(np.uint64).tolist() == t2.view(np.uint64).tolist()
        np.testing.assert_allclose(t1, [want_w, want], rtol=1e-12, atol=0, err_msg=f"{qtype}/{key}")


def test_tensor_error_large_ragged():
    """More blocks than one wave of CTAs, a row count that leaves a partial tile."""
    nat = _native()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = (torch.randn((3001, 2048), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    qw = torch.rand(2048, device="cuda", generator=g) + 0.1
    blocks = nat.quantize(12, x, qw)
    deq = nat.dequantize(blocks, 12).cpu().numpy()
    _, want_w, want = _ref_errors(deq, x.float().cpu().numpy(), qw.cpu().numpy(), 256)
    got = nat.tensor_error(blocks, 12, x, qw).cpu().numpy()
    np.testing.assert_allclose(got, [want_w, want], rtol=1e-10, atol=0)
    blk = nat.block_error(blocks, 12, x, qw)
    np.testing.assert_allclose(blk.sum().item(), want_w, rtol=1e-10)
