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
  * the rows of a chunk reach pinned memory by positioned reads of the model file (the CLI
    passes its descriptor), split over a shared pool of host threads (reading through the
    mapping costs a page fault per 4 KiB on first touch; one thread moves only a few GB/s);
  * a chunk's blocks go to the file on a writer thread while the worker reads the next
    chunk; the slot waits for that write only before its output staging is reused;
  * chunks are also capped at CHUNK_BYTES of source rows, so the pinned staging stays small
    (page-locking memory costs about 0.5 s per GB) and large tensors pipeline in pieces;
  * each slot owns its device copy of the importance weights, uploaded on the slot's own
    stream: a chunk's kernel can never see the weights of the chunk after it;
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
    src_fd: int = -1          # when >= 0: read the rows from this file at src_offset instead
    src_offset: int = 0       #   of copying them out of `rows` (the mapping), see _read_rows


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
        self.h_qw = self.d_qw = None  # this slot's importance weights: pinned staging, device copy
        self.wfut = None              # the write of the slot's last chunk (reads h_out)

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


# Staging slots allocated ahead of a run, per device index (stage_buffers); taken by _open.
_STAGED: dict[int, list[_Slot]] = {}
_STAGED_LOCK = threading.Lock()


def _fill_slot(sl: _Slot, device: torch.device, in_bytes: int, out_bytes: int, max_k: int) -> None:
    sl.h_in = _Slot._grow_pinned(sl.h_in, in_bytes)
    sl.h_out = _Slot._grow_pinned(sl.h_out, out_bytes)
    sl.d_in = _Slot._grow_dev(sl.d_in, in_bytes, device)
    sl.d_out = _Slot._grow_dev(sl.d_out, out_bytes, device)
    if sl.h_qw is None or sl.h_qw.numel() < max_k:
        sl.h_qw = torch.empty(max(max_k, 1), dtype=torch.float32, pin_memory=True)
        sl.d_qw = torch.empty(max(max_k, 1), dtype=torch.float32, device=device)


def stage_buffers(device: torch.device, in_bytes: int, out_bytes: int, max_k: int = 1 << 16) -> None:
    """Allocate one device's staging slots (pinned and device buffers, streams) ahead of a
    run, e.g. on a start-up thread while the model is read and planned. The next
    ShardedQuantizer that opens this device takes them and only grows what is too small."""
    torch.cuda.set_device(device)
    slots = [_Slot(device), _Slot(device)]
    for sl in slots:
        _fill_slot(sl, device, in_bytes, out_bytes, max_k)
    with _STAGED_LOCK:
        _STAGED[device.index] = slots


class ShardedQuantizer:
    """Quantize a list of jobs across `devices`, writing into the open file `fd`."""

    COPY_SLICE = 8 << 20     # bytes per host read / write task
    CHUNK_BYTES = 128 << 20  # source bytes per chunk at most

    def __init__(self, devices: list[torch.device], fd: int, mem_bytes: int, copy_threads: int | None = None):
        self.devices = devices
        self.fd = fd
        self.mem_bytes = mem_bytes
        self.error: BaseException | None = None
        self.stats: dict[str, float] = {}
        self.copy_threads = copy_threads or min(32, os.cpu_count() or 1)
        self._pool: ThreadPoolExecutor | None = None
        self._writer: ThreadPoolExecutor | None = None
        # seconds per phase, summed over the GPU workers (read / alloc / enqueue / wait / write)
        self.timing = dict.fromkeys(("read", "alloc", "enqueue", "wait", "write"), 0.0)
        self._tlock = threading.Lock()
        self._max_in = self._max_out = self._max_k = 0  # largest chunk / row, for sizing the staging once

    def _tick(self, key: str, t0: float) -> float:
        t = time.perf_counter()
        with self._tlock:
            self.timing[key] += t - t0
        return t

    def _read_rows(self, dst: np.ndarray, fd: int, offset: int) -> None:
        """Fill the 1-D uint8 array dst from file fd at offset, in slices on the copy pool."""
        mv = memoryview(dst)

        def read(a: int, b: int) -> None:
            while a < b:
                n = os.preadv(fd, [mv[a:b]], offset + a)
                if n <= 0:
                    raise OSError(f"short read at offset {offset + a}")
                a += n

        n = dst.size
        if self._pool is None or n <= self.COPY_SLICE:
            read(0, n)
            return
        futs = [self._pool.submit(read, a, min(n, a + self.COPY_SLICE)) for a in range(0, n, self.COPY_SLICE)]
        for f in futs:
            f.result()

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
            step = max(1, min(self.mem_bytes // max(1, j.k * j.bytes_per_elem),
                              self.CHUNK_BYTES // max(1, j.rows.shape[1])))
            for r0 in range(0, n, step):
                yield j, r0, min(n, r0 + step)

    # -- one GPU -----------------------------------------------------------
    def _open(self, device: torch.device):
        torch.cuda.set_device(device)
        t0 = time.perf_counter()
        with _STAGED_LOCK:
            slots = _STAGED.pop(device.index, None)
        if slots is None:
            slots = [_Slot(device), _Slot(device)]
        for sl in slots:  # sized once for the largest chunk of the run
            _fill_slot(sl, device, self._max_in, self._max_out, self._max_k)
        self._tick("alloc", t0)
        return {"device": device, "slots": slots, "next": 0}

    def _submit(self, ctx, job: QuantJob, r0: int, r1: int):
        """Stage rows r0:r1 of `job`, run the kernel, start the copy back (asynchronous)."""
        device = ctx["device"]
        slot = ctx["slots"][ctx["next"]]
        ctx["next"] ^= 1
        self._retire(slot)
        n = r1 - r0
        in_bytes = n * job.rows.shape[1]
        out_bytes = n * job.row_bytes
        t0 = time.perf_counter()
        slot.h_in = _Slot._grow_pinned(slot.h_in, in_bytes)
        slot.h_out = _Slot._grow_pinned(slot.h_out, out_bytes)
        slot.d_in = _Slot._grow_dev(slot.d_in, in_bytes, device)
        slot.d_out = _Slot._grow_dev(slot.d_out, out_bytes, device)
        t0 = self._tick("alloc", t0)
        if job.src_fd >= 0:
            self._read_rows(slot.h_in[:in_bytes].numpy(), job.src_fd, job.src_offset + r0 * job.rows.shape[1])
        else:
            self._copy_rows(slot.h_in[:in_bytes].numpy().reshape(n, -1), job.rows[r0:r1])
        t0 = self._tick("read", t0)
        if slot.wfut is not None:  # h_out is about to be overwritten by this chunk's blocks
            slot.wfut.result()
            slot.wfut = None
            t0 = self._tick("write", t0)
        qw = None
        if job.qw is not None:  # the slot is retired, so its staging is free
            np.copyto(slot.h_qw[:job.k].numpy(), np.asarray(job.qw[:job.k], dtype=np.float32))
            qw = slot.d_qw[:job.k]
        with torch.cuda.stream(slot.stream):
            if qw is not None:
                qw.copy_(slot.h_qw[:job.k], non_blocking=True)
            slot.d_in[:in_bytes].copy_(slot.h_in[:in_bytes], non_blocking=True)
            x = slot.d_in[:in_bytes].view(job.src_dtype).view(n, job.k)
            out = slot.d_out[:out_bytes].view(n, job.row_bytes)
            _native.quantize_into(job.ggml_type, x, qw, out, slot.stream)
            slot.h_out[:out_bytes].copy_(slot.d_out[:out_bytes], non_blocking=True)
            slot.event.record(slot.stream)
        slot.pending = (out_bytes, job.out_offset + r0 * job.row_bytes)
        self._tick("enqueue", t0)

    def _drain(self, ctx):
        for slot in ctx["slots"]:
            self._retire(slot)
        for slot in ctx["slots"]:
            if slot.wfut is not None:
                slot.wfut.result()
                slot.wfut = None

    def _retire(self, slot: _Slot):
        """Wait for the slot's chunk and write its blocks to the file."""
        if slot.pending is None:
            return
        nbytes, off = slot.pending
        t0 = time.perf_counter()
        slot.event.synchronize()
        self._tick("wait", t0)
        buf = slot.h_out[:nbytes].numpy()
        slot.wfut = self._writer.submit(self._write, buf, off) if self._writer else None
        if slot.wfut is None:
            self._write(buf, off)
        slot.pending = None

    def _write(self, buf: np.ndarray, off: int):
        """Write buf at file offset off (positioned writes to one file serialize in the
        kernel, so one thread per write)."""
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
        for j, r0, r1 in self._chunks(jobs):
            self._max_in = max(self._max_in, (r1 - r0) * j.rows.shape[1])
            self._max_out = max(self._max_out, (r1 - r0) * j.row_bytes)
            self._max_k = max(self._max_k, j.k)
            work.put((j, r0, r1))
        for _ in self.devices:
            work.put(None)
        lock = threading.Lock()
        self._pool = ThreadPoolExecutor(max_workers=self.copy_threads) if self.copy_threads > 1 else None
        self._writer = ThreadPoolExecutor(max_workers=2 * len(self.devices)) if self.devices else None
        try:
            threads = [threading.Thread(target=self._worker, args=(d, work, lock), daemon=True) for d in self.devices]
            for t in threads:
                t.start()
            for c in copies:  # passthroughs on this thread while the GPUs work
                self._write(np.ascontiguousarray(c.data), c.out_offset)
            for t in threads:
                t.join()
        finally:
            for ex in (self._pool, self._writer):
                if ex is not None:
                    ex.shutdown(wait=True)
            self._pool = self._writer = None
        if self.error is not None:
            raise self.error
        return time.time() - t0
