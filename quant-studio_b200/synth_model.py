#!/usr/bin/env python3
"""Synthetic bf16 GGUF models (and imatrix files) at the sizes of BASELINE's model configs.

The reference builds its small test model with tools/dev_make_synth.py: a llama GGUF in bf16
with the llama.* metadata the type-mix policy reads (block count, heads, kv heads, ...), and
a matching imatrix. This writes the same kind of file at full model size:

  4b  36 layers, hidden 2560, 32 q-heads / 8 kv-heads of 128, SwiGLU 9728, vocab 151936,
      tied embeddings (no output.weight)                            ~4.0 G parameters
  8b  32 layers, hidden 4096, 32 / 8 heads of 128, SwiGLU 14336, vocab 128256, untied
                                                                    ~8.0 G parameters

Weights: N(0, 0.02) with 0.1 % of the entries replaced by N(0, 0.5) outliers, stored bf16;
RMSNorm weights: float32 ones. imatrix: per quantizable tensor, lognormal(0, 1.5) per column
as `in_sum2` with `counts` = 1. Tensors are drawn one at a time (on the GPU when one is
present) and streamed to the file, so host memory stays at about one tensor.

    python synth_model.py 4b /tmp/m4b.gguf --imatrix /tmp/m4b.imatrix.gguf
"""

from __future__ import annotations

import argparse
import time
from pathlib import Path

import numpy as np
import torch
import gguf
from gguf import GGMLQuantizationType, GGUFWriter

MODELS = {
    "4b": dict(n_layer=36, hidden=2560, n_head=32, n_kv=8, head_dim=128, ff=9728, vocab=151936, tied=True),
    "8b": dict(n_layer=32, hidden=4096, n_head=32, n_kv=8, head_dim=128, ff=14336, vocab=128256, tied=False),
    "tiny": dict(n_layer=2, hidden=256, n_head=4, n_kv=2, head_dim=64, ff=512, vocab=1000, tied=False),  # tests
}


def tensor_list(cfg: dict) -> list[tuple[str, tuple[int, ...], bool]]:
    """(name, (rows, cols) or (n,), is_weight) in file order; rows = ne[1], cols = ne[0]."""
    h, q, kv, ff = cfg["hidden"], cfg["n_head"] * cfg["head_dim"], cfg["n_kv"] * cfg["head_dim"], cfg["ff"]
    out = [("token_embd.weight", (cfg["vocab"], h), True)]
    for i in range(cfg["n_layer"]):
        p = f"blk.{i}."
        out += [(p + "attn_norm.weight", (h,), False),
                (p + "attn_q.weight", (q, h), True), (p + "attn_k.weight", (kv, h), True),
                (p + "attn_v.weight", (kv, h), True), (p + "attn_output.weight", (h, q), True),
                (p + "ffn_norm.weight", (h,), False),
                (p + "ffn_gate.weight", (ff, h), True), (p + "ffn_up.weight", (ff, h), True),
                (p + "ffn_down.weight", (h, ff), True)]
    out.append(("output_norm.weight", (h,), False))
    if not cfg["tied"]:
        out.append(("output.weight", (cfg["vocab"], h), True))
    return out


def _weight_bf16(rows: int, cols: int, gen: torch.Generator, device: torch.device) -> np.ndarray:
    a = torch.empty((rows, cols), device=device).normal_(0.0, 0.02, generator=gen)
    m = torch.rand((rows, cols), device=device, generator=gen) < 0.001
    a[m] = torch.empty(int(m.sum()), device=device).normal_(0.0, 0.5, generator=gen)
    return a.to(torch.bfloat16).view(torch.uint8).cpu().numpy()


def write_model(path: Path, model: str, seed: int = 0) -> dict[str, int]:
    """Write the model; returns {quantizable tensor name: columns}."""
    cfg = MODELS[model]
    device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w = GGUFWriter(path, arch="llama")
    w.add_name(f"qs-b200 synthetic {model}")
    w.add_block_count(cfg["n_layer"])
    w.add_context_length(4096)
    w.add_embedding_length(cfg["hidden"])
    w.add_feed_forward_length(cfg["ff"])
    w.add_head_count(cfg["n_head"])
    w.add_head_count_kv(cfg["n_kv"])
    w.add_key_length(cfg["head_dim"])
    w.add_value_length(cfg["head_dim"])
    w.add_rope_dimension_count(cfg["head_dim"])
    w.add_layer_norm_rms_eps(1e-6)
    w.add_vocab_size(cfg["vocab"])
    w.add_file_type(gguf.LlamaFileType.MOSTLY_BF16)
    tensors = tensor_list(cfg)
    cols = {}
    for name, shape, is_w in tensors:
        if is_w:
            rows, k = shape
            w.add_tensor_info(name, (rows, 2 * k), np.dtype(np.uint8), rows * k * 2, raw_dtype=GGMLQuantizationType.BF16)
            cols[name] = k
        else:
            w.add_tensor_info(name, shape, np.dtype(np.float32), shape[0] * 4)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_ti_data_to_file()
    for name, shape, is_w in tensors:
        if is_w:
            w.write_tensor_data(_weight_bf16(shape[0], shape[1], gen, device))
        else:
            w.write_tensor_data(np.ones(shape, np.float32))
    w.close()
    return cols


def write_imatrix(path: Path, cols: dict[str, int], seed: int = 1) -> None:
    """lognormal(0, 1.5) per column for every quantizable tensor, stored as in_sum2 / counts 1."""
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path, arch="imatrix")
    w.add_string("general.type", "imatrix")
    for name, k in cols.items():
        w.add_tensor(name + ".in_sum2", rng.lognormal(0.0, 1.5, k).astype(np.float32))
        w.add_tensor(name + ".counts", np.array([1.0], dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("model", choices=sorted(MODELS))
    ap.add_argument("output", type=Path)
    ap.add_argument("--imatrix", type=Path, default=None, help="also write a matching imatrix GGUF here")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    t0 = time.time()
    cols = write_model(args.output, args.model, args.seed)
    if args.imatrix is not None:
        write_imatrix(args.imatrix, cols)
    n = sum(r * c for name, (r, c) in ((nm, s) for nm, s, w_ in tensor_list(MODELS[args.model]) if w_))
    print(f"{args.output}: {args.model}, {n / 1e9:.2f} G weight values, {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
