"""The 32-value block formats on the GPU (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0), bit for bit.

Q4_0 against the oracle (pinned to the reference's fixtures); Q4_1 / Q5_0 / Q5_1 / Q8_0,
which the reference has no kernel for, against the oracle and directly against gguf-py's
quantizers. Every source dtype, the adversarial rows (including blocks whose 1 / d
overflows), ragged block counts (a CTA's range and a stage are multiples of 8 and 256
blocks), strided destinations, and the decode of the same blocks against gguf-py."""

import numpy as np
import pytest
import torch
from gguf import GGMLQuantizationType as GGT
from gguf.quants import dequantize as gguf_dequantize, quantize as gguf_quantize

import oracle
from kernels import _native
from test_oracle_legacy import adversarial_rows, subnormal_scale_rows, zero_sign_canonical

pytestmark = pytest.mark.gpu

TYPES = {"q4_0": GGT.Q4_0, "q4_1": GGT.Q4_1, "q5_0": GGT.Q5_0, "q5_1": GGT.Q5_1, "q8_0": GGT.Q8_0}
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def bench_rows(rows, k, seed):
    rng = np.random.default_rng(seed)
    a = rng.normal(0.0, 0.02, (rows, k))
    m = rng.random(a.shape) < 0.001
    a[m] = rng.normal(0.0, 0.5, int(m.sum()))
    return a.astype(np.float32)


def gpu(qtype, x: torch.Tensor) -> np.ndarray:
    out = _native.quantize(int(TYPES[qtype]), x.cuda(), None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def check(qtype, x_dev: torch.Tensor, what: str, gguf_pin: bool = True):
    xf = x_dev.float().cpu().numpy()
    got = gpu(qtype, x_dev)
    want = oracle.quantize(qtype, xf)
    bad = np.nonzero((got != want).any(1))[0]
    assert bad.size == 0, f"{qtype} {what}: rows {bad[:8]} differ from the oracle"
    if gguf_pin and qtype != "q4_0":
        ref = gguf_quantize(xf, TYPES[qtype]).reshape(got.shape)
        assert np.array_equal(zero_sign_canonical(qtype, got), zero_sign_canonical(qtype, ref)), \
            f"{qtype} {what}: differs from gguf-py"


@pytest.mark.parametrize("qtype", list(TYPES))
@pytest.mark.parametrize("dt", list(DTYPES))
def test_benchmark_distribution(qtype, dt):
    x = torch.from_numpy(bench_rows(512, 4096, 1)).to(DTYPES[dt])
    check(qtype, x, f"512x4096 {dt}")


@pytest.mark.parametrize("qtype", list(TYPES))
@pytest.mark.parametrize("dt", list(DTYPES))
def test_adversarial_rows(qtype, dt):
    a = adversarial_rows(256)
    if dt != "f32":  # keep the rows in range of the 16-bit type
        a = a[np.abs(a).max(1) < 6e4] if dt == "f16" else a
    x = torch.from_numpy(a).to(DTYPES[dt])
    xf = x.float().numpy()
    # gguf-py differs from the reference's Q4_0 only on blocks whose 1 / d overflows
    check(qtype, x, f"adversarial {dt}", gguf_pin=not subnormal_scale_rows(xf).any() or qtype != "q4_0")


@pytest.mark.parametrize("qtype", list(TYPES))
@pytest.mark.parametrize("shape", [(1, 32), (3, 96), (7, 2560), (1, 8192 + 32), (33, 4096 + 96), (1000, 352)])
def test_ragged_block_counts(qtype, shape):
    """Block counts that are not multiples of 8 (a CTA range) or of 256 (a stage)."""
    x = torch.from_numpy(bench_rows(*shape, seed=sum(shape))).to(torch.bfloat16)
    check(qtype, x, f"{shape}")


@pytest.mark.parametrize("qtype", list(TYPES))
def test_strided_destination_keeps_padding(qtype):
    x = torch.from_numpy(bench_rows(37, 2560, 5)).to(torch.bfloat16).cuda()
    rb = _native.row_bytes(int(TYPES[qtype]), 2560)
    out = torch.full((37, rb + 13), 0xA5, dtype=torch.uint8, device="cuda")
    _native.quantize_into(int(TYPES[qtype]), x, None, out[:, :rb])
    got = out.cpu().numpy()
    want = oracle.quantize(qtype, x.float().cpu().numpy())
    assert np.array_equal(got[:, :rb], want)
    assert (got[:, rb:] == 0xA5).all()


@pytest.mark.parametrize("qtype", list(TYPES))
def test_large_tensor(qtype):
    """The config-3 embedding row length (2560) over 20000 rows: several stages per CTA."""
    x = torch.from_numpy(bench_rows(20000, 2560, 9)).to(torch.bfloat16)
    check(qtype, x, "20000x2560", gguf_pin=False)


@pytest.mark.parametrize("qtype", list(TYPES))
def test_decode_matches_gguf_py(qtype):
    x = torch.from_numpy(np.concatenate([bench_rows(64, 256, 3), adversarial_rows(256)])).to(torch.bfloat16).cuda()
    blocks = _native.quantize(int(TYPES[qtype]), x, None)
    deq = _native.dequantize(blocks, int(TYPES[qtype])).cpu().numpy()
    want = gguf_dequantize(blocks.cpu().numpy(), TYPES[qtype])
    # the adversarial rows include blocks whose f16 scale overflows to inf (inf * 0 = NaN):
    # NaN at the same places, every other value bit for bit
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(deq), nan)
    assert np.array_equal(deq[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_no_kernel_gave_up_waiting():
    """Every bounded wait in the streaming kernels completed in the runs above."""
    import ctypes
    bits = ctypes.c_int(-1)
    _native.check(_native.lib().qs_device_fault(0, ctypes.byref(bits)))
    assert bits.value == 0


@pytest.mark.parametrize("qtype", list(TYPES))
def test_launch_waits_for_the_kernel_that_wrote_its_input(qtype):
    """Each launch may start while the previous kernel on its stream finishes (programmatic
    stream serialization); it must still read the rows that kernel wrote, and its blocks must
    land after those of an earlier launch into the same destination."""
    s = torch.cuda.Stream()
    base = torch.from_numpy(bench_rows(4096, 4096, 21)).to(torch.bfloat16).cuda()
    rb = _native.row_bytes(int(TYPES[qtype]), 4096)
    out = torch.empty((4096, rb), dtype=torch.uint8, device="cuda")
    with torch.cuda.stream(s):
        for scale in (0.5, 3.0, -1.25):
            y = base * scale  # a torch kernel on the same stream writes the source rows
            _native.quantize_into(int(TYPES[qtype]), y, None, out, s)
    s.synchronize()
    want = oracle.quantize(qtype, (base.float() * -1.25).to(torch.bfloat16).float().cpu().numpy())
    assert np.array_equal(out.cpu().numpy(), want)
