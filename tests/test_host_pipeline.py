"""Host logic of the multi-GPU pipeline and of bench.py's multi-rank timing, on CPU.

The pipeline's queue, chunking and pwrite-at-offset logic is driven with a stand-in for the
device steps (the oracle quantizes on the CPU); the real device steps are covered by the GPU
tests. bench.py's max-over-ranks runs as two gloo ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from kernels.pipeline import CopyJob, QuantJob, ShardedQuantizer  # noqa: F401

NAMES = {2: "q4_0", 12: "q4_k", 18: "iq3_xxs"}


class CpuStandIn(ShardedQuantizer):
    """Same queue / chunking / write path, device steps replaced by the CPU oracle."""

    def _open(self, device):
        return {}

    def _submit(self, ctx, job, r0, r1):
        x = job.rows[r0:r1].view(np.uint16).astype(np.uint32) << 16  # bf16 rows
        out = oracle.quantize(NAMES[job.ggml_type], x.view(np.float32), job.qw, nthreads=1)
        self._write(out, job.out_offset + r0 * job.row_bytes)

    def _drain(self, ctx):
        pass


def _bf16(a):
    return ((a.astype(np.float32).view(np.uint32) + 0x8000) >> 16).astype(np.uint16)


@pytest.mark.parametrize("workers", [1, 3])
def test_chunks_land_at_their_offsets(tmp_path, workers):
    rng = np.random.default_rng(0)
    path = tmp_path / "o.bin"
    jobs, expect, pos = [], [], 64
    for i, (n, k, t) in enumerate([(37, 256, 12), (5, 512, 18), (70, 96, 2)]):
        a = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        rows = _bf16(a).view(np.uint8).reshape(n, 2 * k)
        qw = rng.lognormal(0, 1.5, k).astype(np.float32) if t != 2 else None
        rb = oracle.row_bytes(NAMES[t], k)
        jobs.append(QuantJob(f"t{i}", rows, torch.bfloat16, k, t, qw, pos, rb, 5))
        expect.append((pos, oracle.quantize(NAMES[t], (rows.view(np.uint16).astype(np.uint32) << 16).view(np.float32), qw)))
        pos += (n * rb + 31) // 32 * 32
    raw = rng.integers(0, 255, 1000, dtype=np.uint8)
    copies = [CopyJob("p", raw, pos)]
    pos += 1024
    with open(path, "wb") as f:
        os.ftruncate(f.fileno(), pos)
        q = CpuStandIn([f"fake{i}" for i in range(workers)], f.fileno(), mem_bytes=3000)
        q.run(jobs, copies)
    data = np.fromfile(path, dtype=np.uint8)
    for off, e in expect:
        assert np.array_equal(data[off:off + e.size], e.reshape(-1))
    assert np.array_equal(data[pos - 1024:pos - 24], raw)
    assert sum(q.stats.values()) == 37 + 5 + 70


def test_worker_error_surfaces(tmp_path):
    class Boom(CpuStandIn):
        def _submit(self, ctx, job, r0, r1):
            raise RuntimeError("injected device failure")

    with open(tmp_path / "o.bin", "wb") as f:
        q = Boom(["a", "b"], f.fileno(), mem_bytes=1000)
        job = QuantJob("t", np.zeros((4, 512), np.uint8), torch.bfloat16, 256, 12, None, 0, 144, 5)
        with pytest.raises(RuntimeError, match="injected"):
            q.run([job])


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    got = bench.max_over_ranks(dist, float(10 + rank), torch.device("cpu"))
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, got))


def test_max_over_ranks_gloo():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: 11.0, 1: 11.0}


def test_host_copy_split_over_the_pool():
    """A chunk larger than one copy slice is copied in row slices on the pool, exactly."""
    from concurrent.futures import ThreadPoolExecutor

    from kernels.pipeline import ShardedQuantizer

    sq = ShardedQuantizer([], fd=-1, mem_bytes=1 << 30, copy_threads=4)
    src = np.random.default_rng(0).integers(0, 256, size=(3001, 8192), dtype=np.uint8)  # 24.6 MB, 4 slices
    dst = np.zeros_like(src)
    sq._pool = ThreadPoolExecutor(max_workers=4)
    try:
        sq._copy_rows(dst, src)
    finally:
        sq._pool.shutdown()
    assert np.array_equal(dst, src)


def test_rows_read_from_the_file(tmp_path):
    """The positioned-read path fills the staging buffer with exactly the file's bytes."""
    from concurrent.futures import ThreadPoolExecutor

    from kernels.pipeline import ShardedQuantizer

    data = np.random.default_rng(1).integers(0, 256, size=30_000_123, dtype=np.uint8)
    path = tmp_path / "src.bin"
    data.tofile(path)
    fd = os.open(path, os.O_RDONLY)
    sq = ShardedQuantizer([], fd=-1, mem_bytes=1 << 30, copy_threads=4)
    try:
        for pool in (None, ThreadPoolExecutor(max_workers=4)):
            sq._pool = pool
            dst = np.zeros(20_000_000, dtype=np.uint8)
            sq._read_rows(dst, fd, 5_000_007)
            assert np.array_equal(dst, data[5_000_007:25_000_007])
            if pool is not None:
                pool.shutdown()
    finally:
        os.close(fd)
