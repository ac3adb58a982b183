"""The host pipeline on a GPU: consecutive tensors with their own importance weights.

Regression test for a race: a job's device copy of its weights must stay alive until the
job's kernel has finished, even after the next job (on the other slot and stream) uploads
its own. The first tensor here is large and slow (IQ3_S), the next ones tiny with different
weights, so their uploads land while the first kernel still runs; every output byte is
compared with the oracle.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from kernels import _native
from kernels.pipeline import QuantJob, ShardedQuantizer

pytestmark = pytest.mark.gpu


def _bf16_rows(rng, rows, k):
    a = rng.normal(0.0, 0.02, (rows, k)).astype(np.float32)
    m = rng.random(a.shape) < 0.001
    a[m] = rng.normal(0.0, 0.5, int(m.sum())).astype(np.float32)
    b = torch.from_numpy(a).to(torch.bfloat16)
    return b.view(torch.uint8).numpy().reshape(rows, 2 * k), b.float().numpy()


@pytest.mark.parametrize("qtype", ["iq3_s", "iq2_xxs"])
def test_weights_stay_alive_across_jobs(qtype, tmp_path):
    rng = np.random.default_rng(7)
    gt = oracle.TYPE_IDS[qtype]
    k = 4096
    shapes = [16384, 64, 64, 32]
    jobs, want, pos = [], [], 0
    for i, rows in enumerate(shapes):
        raw, xf = _bf16_rows(rng, rows, k)
        qw = rng.lognormal(0.0, 1.5, k).astype(np.float32)
        rb = _native.row_bytes(gt, k)
        jobs.append(QuantJob(f"t{i}", raw, torch.bfloat16, k, gt, qw, pos, rb, 5))
        want.append(oracle.quantize(qtype, xf, qw))
        pos += rows * rb
    path = tmp_path / "out.bin"
    fd = os.open(path, os.O_RDWR | os.O_CREAT, 0o644)
    try:
        os.ftruncate(fd, pos)
        ShardedQuantizer([torch.device("cuda", 0)], fd, mem_bytes=4 << 30).run(jobs)
    finally:
        os.close(fd)
    data = np.fromfile(path, dtype=np.uint8)
    off = 0
    for j, w in zip(jobs, want):
        got = data[off:off + w.size].reshape(w.shape)
        bad = np.nonzero((got != w).any(1))[0]
        assert bad.size == 0, f"{j.name}: {bad.size} rows differ, first {bad[:8]}"
        off += w.size


def test_staged_buffers_taken_over_and_grown(tmp_path):
    """Staging allocated ahead of a run (as the CLI's start-up thread does) is taken over by
    the run, grown where the run's chunks are larger, and left staged for no later run."""
    from kernels import pipeline

    dev = torch.device("cuda", 0)
    pipeline.stage_buffers(dev, in_bytes=1 << 16, out_bytes=1 << 15, max_k=256)  # deliberately small
    assert 0 in pipeline._STAGED
    rng = np.random.default_rng(11)
    k, rows = 2048, 512
    raw, xf = _bf16_rows(rng, rows, k)
    qw = rng.lognormal(0.0, 1.5, k).astype(np.float32)
    gt = oracle.TYPE_IDS["q4_k"]
    rb = _native.row_bytes(gt, k)
    job = QuantJob("t", raw, torch.bfloat16, k, gt, qw, 0, rb, 5)
    path = tmp_path / "out.bin"
    fd = os.open(path, os.O_RDWR | os.O_CREAT, 0o644)
    try:
        os.ftruncate(fd, rows * rb)
        ShardedQuantizer([dev], fd, mem_bytes=4 << 30).run([job])
    finally:
        os.close(fd)
    assert 0 not in pipeline._STAGED
    got = np.fromfile(path, dtype=np.uint8).reshape(rows, rb)
    assert np.array_equal(got, oracle.quantize("q4_k", xf, qw))
