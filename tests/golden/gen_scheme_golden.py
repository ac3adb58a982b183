#!/usr/bin/env python3
"""Golden per-tensor type plans from the reference's policy module (kernels/scheme.py).

For a set of model layouts (tensor names + ggml shapes, no data) and every scheme,
record the type the reference picks for each tensor under several flag combinations.
Run where a reference checkout exists:

    python tests/golden/gen_scheme_golden.py --reference /path/to/quant-studio
"""

from __future__ import annotations

import argparse
import json
import sys
import zlib
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))


def llama_like(n_layer, hidden, n_head, n_kv, ff, vocab, tied, arch="llama", n_expert=0, head_dim=128, odd=False):
    """(name, ne, src) in file order plus the model facts the policy reads."""
    t = [("token_embd.weight", (hidden, vocab), "BF16")]
    if not tied:
        t.append(("output.weight", (hidden, vocab), "BF16"))
    t.append(("output_norm.weight", (hidden,), "F32"))
    for i in range(n_layer):
        p = f"blk.{i}."
        t.append((p + "attn_norm.weight", (hidden,), "F32"))
        if arch == "falcon":
            t.append((p + "attn_qkv.weight", (hidden, (n_head + 2 * n_kv) * head_dim), "BF16"))
        else:
            t.append((p + "attn_q.weight", (hidden, n_head * head_dim), "BF16"))
            t.append((p + "attn_k.weight", (hidden, n_kv * head_dim), "BF16"))
            t.append((p + "attn_v.weight", (hidden, n_kv * head_dim), "BF16"))
        t.append((p + "attn_output.weight", (n_head * head_dim, hidden), "BF16"))
        t.append((p + "ffn_norm.weight", (hidden,), "F32"))
        if n_expert:
            t.append((p + "ffn_gate_inp.weight", (hidden, n_expert), "F32"))
            t.append((p + "ffn_gate_exps.weight", (hidden, ff, n_expert), "BF16"))
            t.append((p + "ffn_up_exps.weight", (hidden, ff, n_expert), "BF16"))
            t.append((p + "ffn_down_exps.weight", (ff, hidden, n_expert), "BF16"))
        else:
            t.append((p + "ffn_gate.weight", (hidden, ff), "BF16"))
            t.append((p + "ffn_up.weight", (hidden, ff), "BF16"))
            t.append((p + "ffn_down.weight", (ff if not odd else ff + 40, hidden), "BF16"))
    t.append(("rope_freqs.weight", (64,), "F32"))
    facts = dict(arch=arch, n_layer=n_layer, n_expert=n_expert, n_head=n_head, n_head_kv=n_kv,
                 is_70b=arch == "llama" and n_layer == 80)
    return t, facts


MODELS = {
    "c4_4b_tied": llama_like(36, 2560, 32, 8, 9728, 151936, tied=True, arch="qwen3"),
    "c5_8b": llama_like(32, 4096, 32, 8, 14336, 128256, tied=False),
    "synth_2l": llama_like(2, 256, 8, 8, 512, 512, tied=False, head_dim=32),
    "llama_70b": llama_like(80, 8192, 64, 8, 28672, 32000, tied=False),
    "falcon": llama_like(12, 4544, 71, 1, 18176, 65024, tied=True, arch="falcon", head_dim=64),
    "moe8": llama_like(8, 4096, 32, 8, 14336, 32000, tied=False, n_expert=8),
    "odd_cols": llama_like(4, 1024, 8, 2, 2816, 32000, tied=True, odd=True),
}

FLAGS = [
    {},
    {"has_imatrix": True},
    {"pure": True},
    {"has_imatrix": True, "token_embedding_type": "Q4_0", "output_tensor_type": "Q8_0"},
    {"tt_overrides": [["attn_v", "Q6_K"], ["ffn_down", "Q5_K"]]},
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    from gen_golden import _shim_gguf_enums
    _shim_gguf_enums()
    sys.path.insert(0, str(args.reference.resolve()))
    from gguf import GGMLQuantizationType as GT

    from kernels import scheme

    out = {"models": {}, "plans": {}}
    for mname, (tensors, facts) in MODELS.items():
        out["models"][mname] = {"tensors": [[n, list(ne), s] for n, ne, s in tensors], "facts": facts}
        model = scheme.ModelInfo(**facts)
        order = sorted(tensors, key=lambda t: scheme.weight_name_key(t[0]))
        for opt in scheme.QUANT_OPTIONS:
            if opt.name in ("COPY", "Q2_0") or opt.default_type is None:  # Q2_0: an enum this gguf lacks
                continue
            for fi, fl in enumerate(FLAGS):
                kw = dict(fl)
                for key in ("token_embedding_type", "output_tensor_type"):
                    if key in kw:
                        kw[key] = GT[kw[key]]
                if "tt_overrides" in kw:
                    kw["tt_overrides"] = [(p, GT[t]) for p, t in kw["tt_overrides"]]
                try:
                    plan = scheme.decide_types(model, [(n, ne, GT[s]) for n, ne, s in order], opt.ftype, **kw)
                    res = [p.name for p in plan]
                except ValueError as e:
                    res = f"error: {e}"
                out["plans"][f"{mname}|{opt.name}|{fi}"] = res
    out["flags"] = FLAGS
    raw = json.dumps(out, sort_keys=True).encode()
    (HERE / "scheme_plans.json.z").write_bytes(zlib.compress(raw, 9))
    print(len(out["plans"]), "plans,", len(raw), "bytes raw")


if __name__ == "__main__":
    main()
