"""Host pipeline: GGUF rows -> one or more GPUs -> packed blocks at their file offsets.

Replaces the reference's CudaPipeline / OutputWriter (quant-studio.py:103-213). The
reference streams one tensor's row chunks through one GPU and appends the results in
order on a writer thread. Here the output layout is known up front (gguf-py assigns
every tensor an aligned offset), so any chunk can be written the moment it is ready:

  * every tensor is cut into row chunks of at most `mem` bytes of device working set
    (the reference's --mem rule, quant-studio.py:457);
  * one worker thread per GPU pulls chunks from a shared queue (dynamic balance: IQ
    searches cost more on some rows than others), stages the rows in pinned memory,
    copies them to the device, runs the libqsb200 kernel on the source dtype directly
    (no f32 upcast), copies the blocks back and writes them with os.pwrite;
  * two slots per GPU, each with its own stream, so the host copy and the file write of
    one chunk overlap the device work of the other;
  * the copy of a chunk from the mapped model into pinned memory is split over a shared
    pool of host threads (numpy releases the GIL for it): one thread moves only a few GB/s
    and takes the mapping's page faults alone, which made it the bottleneck of the CLI;
  * passthrough tensors are copied with pwrite from the source mmap.
No collective and no peer traffic: the GPUs share nothing but the queue.
"""

from __future__ import annotations

import os
import queue
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np
import torch

from . import _native


@dataclass
class QuantJob:
    name: str
    rows: np.ndarray          # (n_rows, in_row_bytes) uint8 view of the source (mmap)
    src_dtype: torch.dtype    # float32 / float16 / bfloat16
    k: int                    # values per row
    ggml_type: int            # destination GGML type id
    qw: np.ndarray | None     # (k,) float32 importance weights or None
    out_offset: int           # absolute file offset of the tensor's data
    row_bytes: int            # packed bytes per row
    bytes_per_elem: int       # working-set heuristic for the chunk size


@dataclass
class CopyJob:
    name: str
    data: np.ndarray          # raw bytes of the source tensor
    out_offset: int


class _Slot:
    def __init__(self, device: torch.device):
        self.stream = torch.cuda.Stream(device)
        self.event = torch.cuda.Event()
        self.h_in = self.h_out = None
        self.d_in = self.d_out = None
        self.pending = None       # (nbytes, file offset) of the chunk in flight
        self.qw = None            # the weights the chunk in flight reads: kept alive until it is retired

    @staticmethod
    def _grow_pinned(buf, nbytes):
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, pin_memory=True)
        return buf

    @staticmethod
    def _grow_dev(buf, nbytes, device):
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        return buf


class ShardedQuantizer:
    """Quantize a list of jobs across `devices`, writing into the open file `fd`."""

    COPY_SLICE = 8 << 20  # bytes per host-copy task

    def __init__(self, devices: list[torch.device], fd: int, mem_bytes: int, copy_threads: int | None = None):
        self.devices = devices
        self.fd = fd
        self.mem_bytes = mem_bytes
        self.error: BaseException | None = None
        self.stats: dict[str, float] = {}
        self.copy_threads = copy_threads or min(32, os.cpu_count() or 1)
        self._pool: ThreadPoolExecutor | None = None

    def _copy_rows(self, dst: np.ndarray, src: np.ndarray) -> None:
        """dst[:] = src for (n, row_bytes) arrays, in row slices on the copy pool."""
        n = src.shape[0]
        per = max(1, self.COPY_SLICE // max(1, src.shape[1]))
        if self._pool is None or n <= per:
            np.copyto(dst, src)
            return
        futs = [self._pool.submit(np.copyto, dst[r:r + per], src[r:r + per]) for r in range(0, n, per)]
        for f in futs:
            f.result()

    # -- work list ---------------------------------------------------------
    def _chunks(self, jobs: list[QuantJob]):
        for j in jobs:
            n = j.rows.shape[0]
            step = max(1, self.mem_bytes // max(1, j.k * j.bytes_per_elem))
            for r0 in range(0, n, step):
                yield j, r0, min(n, r0 + step)

    # -- one GPU -----------------------------------------------------------
    def _open(self, device: torch.device):
        torch.cuda.set_device(device)
        return {"device": device, "slots": [_Slot(device), _Slot(device)], "next": 0, "qw": {}}

    def _submit(self, ctx, job: QuantJob, r0: int, r1: int):
        """Stage rows r0:r1 of `job`, run the kernel, start the copy back (asynchronous)."""
        device = ctx["device"]
        slot = ctx["slots"][ctx["next"]]
        ctx["next"] ^= 1
        self._retire(slot)
        n = r1 - r0
        in_bytes = n * job.rows.shape[1]
        out_bytes = n * job.row_bytes
        slot.h_in = _Slot._grow_pinned(slot.h_in, in_bytes)
        slot.h_out = _Slot._grow_pinned(slot.h_out, out_bytes)
        slot.d_in = _Slot._grow_dev(slot.d_in, in_bytes, device)
        slot.d_out = _Slot._grow_dev(slot.d_out, out_bytes, device)
        self._copy_rows(slot.h_in[:in_bytes].numpy().reshape(n, -1), job.rows[r0:r1])
        qw = None
        if job.qw is not None:
            cache = ctx["qw"]
            if id(job) not in cache:
                cache.clear()
                cache[id(job)] = torch.from_numpy(np.ascontiguousarray(job.qw[:job.k], dtype=np.float32)).to(device)
            qw = cache[id(job)]
        # the other slot's kernel may still read the previous job's weights; holding them here
        # keeps the caching allocator from giving their memory to the next upload
        slot.qw = qw
        with torch.cuda.stream(slot.stream):
            if qw is not None:
                slot.stream.wait_stream(torch.cuda.current_stream(device))
            slot.d_in[:in_bytes].copy_(slot.h_in[:in_bytes], non_blocking=True)
            x = slot.d_in[:in_bytes].view(job.src_dtype).view(n, job.k)
            out = slot.d_out[:out_bytes].view(n, job.row_bytes)
            _native.quantize_into(job.ggml_type, x, qw, out, slot.stream)
            slot.h_out[:out_bytes].copy_(slot.d_out[:out_bytes], non_blocking=True)
            slot.event.record(slot.stream)
        slot.pending = (out_bytes, job.out_offset + r0 * job.row_bytes)

    def _drain(self, ctx):
        for slot in ctx["slots"]:
            self._retire(slot)

    def _retire(self, slot: _Slot):
        """Wait for the slot's chunk and write its blocks to the file."""
        if slot.pending is None:
            return
        nbytes, off = slot.pending
        slot.event.synchronize()
        slot.qw = None
        self._write(slot.h_out[:nbytes].numpy(), off)
        slot.pending = None

    def _write(self, buf: np.ndarray, off: int):
        mv = memoryview(buf.reshape(-1).view(np.uint8))
        done = 0
        while done < len(mv):
            done += os.pwrite(self.fd, mv[done:done + (64 << 20)], off + done)

    def _worker(self, device, work: queue.Queue, lock: threading.Lock):
        try:
            ctx = self._open(device)
            while self.error is None:
                item = work.get()
                if item is None:
                    break
                job, r0, r1 = item
                self._submit(ctx, job, r0, r1)
                with lock:
                    self.stats[job.name] = self.stats.get(job.name, 0) + (r1 - r0)
            self._drain(ctx)
        except BaseException as e:  # surfaced by run()
            self.error = e

    # -- driver ------------------------------------------------------------
    def run(self, jobs: list[QuantJob], copies: list[CopyJob] = ()) -> float:
        t0 = time.time()
        work: queue.Queue = queue.Queue()
        for c in self._chunks(jobs):
            work.put(c)
        for _ in self.devices:
            work.put(None)
        lock = threading.Lock()
        self._pool = ThreadPoolExecutor(max_workers=self.copy_threads) if self.copy_threads > 1 else None
        try:
            threads = [threading.Thread(target=self._worker, args=(d, work, lock), daemon=True) for d in self.devices]
            for t in threads:
                t.start()
            for c in copies:  # passthroughs on this thread while the GPUs work
                self._write(np.ascontiguousarray(c.data), c.out_offset)
            for t in threads:
                t.join()
        finally:
            if self._pool is not None:
                self._pool.shutdown(wait=True)
                self._pool = None
        if self.error is not None:
            raise self.error
        return time.time() - t0
