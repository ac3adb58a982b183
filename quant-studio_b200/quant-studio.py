#!/usr/bin/env python3
"""qs-b200: GGUF quantizer on B200 GPUs, a drop-in for quant-studio / llama-quantize.

Same command line as the reference (quant-studio.py:267-476):

    python quant-studio.py in.gguf out.gguf Q4_K_M --mem 4G --imatrix imatrix.gguf
    python quant-studio.py in.gguf out.gguf iq2_xxs --pure --imatrix im.gguf --token-embedding-type q4_0

plus --gpus N to shard the row chunks over N GPUs of this machine. The per-tensor type
plan is the llama.cpp mixture (kernels/scheme.py); the quantization runs in libqsb200
(sm_100a CUDA kernels) through kernels.pipeline. There is no CPU path: without a CUDA
device the tool stops with an error.
"""

from __future__ import annotations

import argparse
import os
import re
import sys
import threading
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np
import torch

import gguf
from gguf import GGMLQuantizationType, GGUFReader, GGUFValueType, GGUFWriter
from gguf.constants import GGML_QUANT_SIZES, GGML_QUANT_VERSION

from kernels import QUANT_TYPES, TORCH_DTYPES, _native, scheme
from kernels.pipeline import CopyJob, QuantJob, ShardedQuantizer, stage_buffers


_MEM_RE = re.compile(r"(\d+(?:\.\d*)?|\.\d+)\s*([KMG]?)(?:I?B)?", re.IGNORECASE)
_MEM_SHIFT = {"": 0, "K": 10, "M": 20, "G": 30}


def parse_mem(text: str) -> int:
    """--mem value in bytes: a number with an optional binary K / M / G suffix ("4G",
    "512m", "1.5G", "65536"); the reference's --mem accepts the same forms
    (quant-studio.py:41-48). A trailing "B" / "iB" is tolerated."""
    m = _MEM_RE.fullmatch(text.strip())
    if m is None:
        sys.exit(f"error: --mem {text!r} is not a size like 4G, 512M or 65536")
    return int(float(m.group(1)) * (1 << _MEM_SHIFT[m.group(2).upper()]))


_GGML_TYPE_BY_NAME = {t.name.lower(): t for t in GGMLQuantizationType}


def parse_ggml_type(text: str) -> GGMLQuantizationType:
    """A ggml type name in any case (q4_0, Q6_K, bf16) as --token-embedding-type,
    --output-tensor-type and --tensor-type take it."""
    t = _GGML_TYPE_BY_NAME.get(text.strip().lower())
    if t is None:
        sys.exit(f"error: unknown ggml type: {text}")
    return t


def load_imatrix(path: Path) -> dict[str, np.ndarray]:
    """Importance weights per tensor from a GGUF imatrix file: for every tensor name with
    both a `<name>.in_sum2` (summed squared activations per column, one row per expert)
    and a `<name>.counts` (tokens seen per expert), the per-column mean in_sum2 / count as
    float32, and 0 for an expert that saw no tokens. Flattened over experts; the caller
    takes the first k values (the reference's convention, quant-studio.py:454-455)."""
    parts: dict[str, dict[str, np.ndarray]] = {}
    for t in GGUFReader(path).tensors:
        base, dot, kind = t.name.rpartition(".")
        if dot and kind in ("in_sum2", "counts"):
            parts.setdefault(base, {})[kind] = np.asarray(t.data, dtype=np.float32).ravel()
    weights = {}
    for base, p in parts.items():
        if "in_sum2" not in p or "counts" not in p:
            continue
        n = p["counts"][:, None]                      # (experts, 1)
        sums = p["in_sum2"].reshape(n.shape[0], -1)   # (experts, columns)
        seen = n > 0
        weights[base] = np.where(seen, sums / np.where(seen, n, np.float32(1)), np.float32(0)).ravel()
    return weights


def fmt_size(n: float) -> str:
    for unit in ("B", "KiB", "MiB", "GiB"):
        if n < 1024 or unit == "GiB":
            return f"{n:8.1f} {unit}" if unit != "B" else f"{int(n):8d} B  "
        n /= 1024
    return f"{n} B"


def out_row_bytes_for(k: int, t: GGMLQuantizationType) -> int:
    block, size = GGML_QUANT_SIZES[t]
    return k // block * size


def copy_metadata(reader: GGUFReader, writer: GGUFWriter, ftype) -> None:
    """All KV pairs of the source, with file_type and quantization_version replaced."""
    overrides = {
        gguf.Keys.General.FILE_TYPE: (int(ftype), GGUFValueType.UINT32),
        gguf.Keys.General.QUANTIZATION_VERSION: (GGML_QUANT_VERSION, GGUFValueType.UINT32),
    }
    for f in reader.fields.values():
        if f.name == gguf.Keys.General.ARCHITECTURE or f.name.startswith("GGUF.") or f.name in overrides:
            continue
        vt = f.types[0]
        writer.add_key_value(f.name, f.contents(), vt, sub_type=f.types[-1] if vt == GGUFValueType.ARRAY else None)
    for key, (val, vt) in overrides.items():
        writer.add_key_value(key, val, vt)


def pick_devices(device: str, ngpus: int) -> list[torch.device]:
    if device in ("cpu", "mps"):
        sys.exit(f"error: --device {device}: qs-b200 quantizes on CUDA devices only")
    if not torch.cuda.is_available():
        sys.exit("error: no CUDA device is visible; qs-b200 has no CPU path")
    first = torch.device(device).index if device.startswith("cuda:") else 0
    n = torch.cuda.device_count() - first if ngpus <= 0 else ngpus
    if first + n > torch.cuda.device_count():
        sys.exit(f"error: asked for {n} GPUs from cuda:{first}, {torch.cuda.device_count()} visible")
    return [torch.device("cuda", first + i) for i in range(n)]


def start_device_warmup(args) -> tuple[threading.Thread, dict]:
    """Pick the devices, bring up their CUDA contexts and libqsb200 state and allocate the
    pipeline's staging buffers on a background thread (the devices in parallel, one thread
    each), while the main thread reads and plans the model."""
    box: dict = {}

    def run() -> None:
        try:
            devs = pick_devices(args.device, args.gpus)
            # a chunk holds at most CHUNK_BYTES of source rows; blocks are under half of that
            # from 16-bit sources (the pipeline grows the staging if a run needs more)
            in_bytes = min(ShardedQuantizer.CHUNK_BYTES, 16 * parse_mem(args.mem))
            errors: list[BaseException] = []

            def up(d: torch.device) -> None:  # one device: context, library state, staging
                try:
                    torch.cuda.set_device(d)
                    torch.empty(1, device=d)
                    _native.check(_native.lib().qs_init(d.index))
                    stage_buffers(d, in_bytes, in_bytes // 2)
                except BaseException as e:
                    errors.append(e)

            torch.cuda.init()  # once, before the devices come up in parallel
            ups = [threading.Thread(target=up, args=(d,), daemon=True) for d in devs]
            for t in ups:
                t.start()
            for t in ups:
                t.join()
            if errors:
                raise errors[0]
            box["devices"] = devs
        except BaseException as e:  # re-raised on the main thread
            box["error"] = e

    t = threading.Thread(target=run, daemon=True)
    t.start()
    return t, box


def main() -> None:
    ap = argparse.ArgumentParser(description="B200 GGUF quantizer, drop-in for llama-quantize",
                                 formatter_class=argparse.RawDescriptionHelpFormatter,
                                 epilog=scheme.format_scheme_table())
    ap.add_argument("input", type=Path, help="source GGUF (F32/F16/BF16)")
    ap.add_argument("output", nargs="?", default=None, help="output GGUF (default: ggml-model-<TYPE>.gguf next to the input)")
    ap.add_argument("qtype", nargs="?", default=None, metavar="type", help="quantization scheme, see the table below")
    ap.add_argument("nthreads", nargs="?", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--mem", default="4G", help="device working-set budget per row chunk, e.g. 4G / 512M")
    ap.add_argument("--device", default="auto", help="auto / cuda / cuda:N (first GPU to use)")
    ap.add_argument("--gpus", type=int, default=1, help="GPUs to shard the row chunks over (0 = all from --device on)")
    ap.add_argument("--imatrix", type=Path, default=None, help="GGUF importance matrix")
    ap.add_argument("--pure", action="store_true", help="disable k-quant mixtures and quantize all tensors to the same type")
    ap.add_argument("--leave-output-tensor", action="store_true", help="leave output.weight un(re)quantized")
    ap.add_argument("--output-tensor-type", default=None, metavar="ggml_type", help="use this ggml_type for the output.weight tensor")
    ap.add_argument("--token-embedding-type", default=None, metavar="ggml_type", help="use this ggml_type for the token embeddings tensor")
    ap.add_argument("--tensor-type", action="append", default=[], metavar="name=ggml_type",
                    help="quantize tensors matching this name regex to this type; repeatable")
    ap.add_argument("--tensor-type-file", type=Path, default=None, metavar="file",
                    help="file with name=ggml_type entries, separated by spaces or newlines")
    ap.add_argument("--dry-run", action="store_true", help="show the per-tensor plan and final size without quantizing")
    rej = ap.add_argument_group("rejected llama-quantize options")
    rej.add_argument("--allow-requantize", action="store_true", help=argparse.SUPPRESS)
    rej.add_argument("--include-weights", default=None, help=argparse.SUPPRESS)
    rej.add_argument("--exclude-weights", default=None, help=argparse.SUPPRESS)
    rej.add_argument("--prune-layers", default=None, help=argparse.SUPPRESS)
    rej.add_argument("--keep-split", action="store_true", help=argparse.SUPPRESS)
    rej.add_argument("--override-kv", action="append", default=[], help=argparse.SUPPRESS)
    args = ap.parse_args()
    warm = None if args.dry_run else start_device_warmup(args)

    for flag, val in (("--allow-requantize", args.allow_requantize), ("--include-weights", args.include_weights),
                      ("--exclude-weights", args.exclude_weights), ("--prune-layers", args.prune_layers),
                      ("--keep-split", args.keep_split), ("--override-kv", args.override_kv)):
        if val:
            sys.exit(f"error: {flag} is not supported by qs-b200")

    # llama-quantize positional style: the output name may be omitted
    if args.output is not None and scheme.parse_scheme(args.output) is not None and \
            (args.qtype is None or args.qtype.isdigit()):
        args.nthreads, args.qtype, args.output = args.qtype, args.output, None
    if args.qtype is None:
        ap.error("missing quantization type")
    if args.nthreads is not None:
        sys.exit("error: the nthreads argument is not supported by qs-b200 (GPU pipeline)")

    opt = scheme.parse_scheme(args.qtype)
    if opt is None:
        sys.exit(f"error: unknown quantization scheme {args.qtype!r}\n\n" + scheme.format_scheme_table())
    if not opt.supported:
        sys.exit(f"error: scheme {opt.name} is not supported by qs-b200\n\n" + scheme.format_scheme_table())
    out_path = Path(args.output) if args.output else args.input.parent / f"ggml-model-{opt.name}.gguf"

    entries = list(args.tensor_type)
    if args.tensor_type_file is not None:
        entries += args.tensor_type_file.read_text().split()
    overrides = []
    for ent in entries:
        pat, _, tname = ent.partition("=")
        if not tname:
            sys.exit(f"error: invalid --tensor-type {ent!r}, expected name=ggml_type")
        overrides.append((pat, parse_ggml_type(tname)))
    tet = parse_ggml_type(args.token_embedding_type) if args.token_embedding_type else None
    ott = parse_ggml_type(args.output_tensor_type) if args.output_tensor_type else None
    mem_bytes = parse_mem(args.mem)

    imatrix: dict[str, np.ndarray] = {}
    if args.imatrix is not None:
        imatrix = load_imatrix(args.imatrix)

    reader = GGUFReader(args.input, mode="r")
    arch_field = reader.get_field(gguf.Keys.General.ARCHITECTURE)
    if arch_field is None:
        sys.exit("error: input has no general.architecture key")
    arch = arch_field.contents()

    tensors = sorted(reader.tensors, key=lambda t: scheme.weight_name_key(t.name))
    model = scheme.ModelInfo.from_reader(reader)
    qs = scheme.init_state(model, [t.name for t in tensors], bool(imatrix), overrides)
    spec_by_type = {s.ggml_type: s for s in QUANT_TYPES.values()}

    plans, missing, need_imat = [], {}, []
    for t in tensors:
        src = t.tensor_type
        dst = src
        if src in TORCH_DTYPES:
            ne = tuple(int(d) for d in t.shape)
            try:
                dst = scheme.tensor_get_type(qs, model, t.name, ne, src, opt.ftype, pure=args.pure,
                                             quantize_output_tensor=not args.leave_output_tensor,
                                             token_embedding_type=tet, output_tensor_type=ott)
            except ValueError as e:
                print(f"warning: {t.name}: {e}; keeping {src.name}", file=sys.stderr)
        if dst == src:
            plans.append((t, None, None))
            continue
        spec = spec_by_type.get(dst)
        if spec is None:
            missing.setdefault(dst.name, []).append(t.name)
            plans.append((t, None, None))
            continue
        if (scheme.tensor_requires_imatrix(t.name, dst, opt.ftype) or spec.needs_imatrix) and t.name not in imatrix:
            need_imat.append(t.name)
        plans.append((t, dst, spec))

    if missing:
        detail = "; ".join(f"{k} for {len(v)} tensors (e.g. {v[0]})" for k, v in sorted(missing.items()))
        sys.exit(f"error: this scheme needs kernel types qs-b200 does not have yet: {detail}")
    if need_imat:
        uniq = sorted(set(need_imat))
        hint = "" if args.imatrix else " (pass --imatrix)"
        if "token_embd.weight" in uniq:
            hint += " (token_embd can be overridden with --token-embedding-type)"
        sys.exit(f"error: {len(uniq)} tensors require importance matrix data{hint}: "
                 + ", ".join(uniq[:4]) + ("..." if len(uniq) > 4 else ""))

    def out_nbytes(t, dst):
        k = int(t.shape[0])
        return t.n_bytes if dst is None else t.n_elements // k * out_row_bytes_for(k, dst)

    if args.dry_run:
        tin = tout = 0
        for t, dst, _ in plans:
            nb = out_nbytes(t, dst)
            tin += t.n_bytes
            tout += nb
            print(f"{t.name:48s} {t.tensor_type.name:>8s} -> {dst.name if dst else t.tensor_type.name:<8s} {fmt_size(nb)}")
        print(f"dry run: {fmt_size(tin)} -> {fmt_size(tout)} tensor data ({tout / max(tin, 1) * 100:.1f}%)")
        return

    t_wait = time.perf_counter()
    warm[0].join()
    t_wait = time.perf_counter() - t_wait
    if "error" in warm[1]:
        raise warm[1]["error"]
    devices = warm[1]["devices"]
    print(f"qs-b200: {args.input} -> {out_path} [{opt.name}] gpus={len(devices)} mem={args.mem} "
          f"(waited {t_wait:.3f}s for device start-up)")
    if args.imatrix is not None:
        print(f"imatrix: {len(imatrix)} entries from {args.imatrix}")

    writer = GGUFWriter(None, arch=arch)
    copy_metadata(reader, writer, opt.ftype)
    for t, dst, _ in plans:
        if dst is not None:
            k = int(t.shape[0])
            rb = out_row_bytes_for(k, dst)
            byte_shape = (*[int(d) for d in reversed(t.shape[1:])], rb)
            writer.add_tensor_info(t.name, byte_shape, np.uint8, out_nbytes(t, dst), raw_dtype=dst)
        else:
            writer.add_tensor_info(t.name, t.data.shape, t.data.dtype, t.data.nbytes, raw_dtype=t.tensor_type)
    writer.write_header_to_file(path=out_path)
    writer.write_kv_data_to_file()
    writer.write_ti_data_to_file()
    fout = writer.fout[0]
    fout.flush()
    align = writer.data_alignment
    pos = GGUFWriter.ggml_pad(fout.tell(), align)

    src_fd = os.open(args.input, os.O_RDONLY)  # rows are read with pread, not through the mapping
    jobs, copies, offsets = [], [], []
    for t, dst, spec in plans:
        offsets.append(pos)
        if dst is not None:
            k = int(t.shape[0])
            qw = imatrix[t.name][:k] if (spec.uses_imatrix and t.name in imatrix) else None
            rows = t.data.reshape(-1, t.data.shape[-1]).view(np.uint8)
            jobs.append(QuantJob(t.name, rows, TORCH_DTYPES[t.tensor_type], k, int(dst), qw, pos,
                                 out_row_bytes_for(k, dst), spec.bytes_per_elem, src_fd, int(t.data_offset)))
        else:
            copies.append(CopyJob(t.name, t.data, pos))
        pos += GGUFWriter.ggml_pad(out_nbytes(t, dst), align)
    fd = fout.fileno()
    os.ftruncate(fd, pos)  # zero padding between tensors, like the reference's pad_to_alignment

    sq = ShardedQuantizer(devices, fd, mem_bytes)
    try:
        dt = sq.run(jobs, copies)
    finally:
        os.close(src_fd)
    tin = tout = 0
    for i, (t, dst, _) in enumerate(plans):
        nb = out_nbytes(t, dst)
        tin += t.n_bytes
        tout += nb
        shape = "x".join(str(int(d)) for d in t.shape)
        print(f"[{i + 1:4d}/{len(plans)}] {t.name:48s} {shape:>16s}  {t.tensor_type.name:>5s} -> "
              f"{dst.name if dst else t.tensor_type.name:<8s} {fmt_size(t.n_bytes)} -> {fmt_size(nb)}")
    os.fsync(fd)
    writer.close()
    print(f"done in {dt:.3f}s: {fmt_size(tin)} -> {fmt_size(tout)} ({tout / max(tin, 1) * 100:.1f}%)")
    print("pipeline seconds (summed over GPU workers): " + ", ".join(f"{k} {v:.3f}" for k, v in sq.timing.items()))


if __name__ == "__main__":
    main()
