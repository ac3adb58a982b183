"""Small synthetic GGUF models and imatrix files for the CLI tests."""

from pathlib import Path

import numpy as np
import torch
import gguf
from gguf import GGMLQuantizationType, GGUFWriter


def bf16_bytes(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).view(torch.uint8).numpy()


def bf16_values(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).float().numpy()


def write_mixed(path: Path, seed: int = 42) -> dict[str, np.ndarray]:
    """The reference test's layout (tests/test_q4_0.py:28-70): f32/f16/bf16 2-D, a 3-D
    expert tensor and passthroughs. Returns the f32 values of tensors that get quantized."""
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path, arch="llama")
    w.add_context_length(2048)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_bool("test.flag", True)
    w.add_array("tokenizer.ggml.tokens", ["<s>", "</s>", "hello"])
    w.add_file_type(gguf.LlamaFileType.MOSTLY_BF16)
    expect = {}
    a = rng.standard_normal((200, 128)).astype(np.float32)
    w.add_tensor("blk.0.attn_q.weight", a)
    expect["blk.0.attn_q.weight"] = a
    b = rng.standard_normal((96, 64)).astype(np.float16)
    w.add_tensor("blk.0.ffn_up.weight", b)
    expect["blk.0.ffn_up.weight"] = b.astype(np.float32)
    c = rng.standard_normal((80, 96)).astype(np.float32)
    w.add_tensor("blk.0.attn_k.weight", bf16_bytes(c), raw_dtype=GGMLQuantizationType.BF16)
    expect["blk.0.attn_k.weight"] = bf16_values(c)
    d = rng.standard_normal((4, 16, 64)).astype(np.float16)
    w.add_tensor("blk.0.ffn_gate_exps.weight", d)
    expect["blk.0.ffn_gate_exps.weight"] = d.astype(np.float32)
    w.add_tensor("blk.0.attn_norm.weight", rng.standard_normal(128).astype(np.float32))
    w.add_tensor("blk.0.odd.weight", rng.standard_normal((10, 40)).astype(np.float32))
    w.add_tensor("rope_freqs.weight", rng.standard_normal(32).astype(np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return expect


def write_llama(path: Path, n_layer=2, hidden=256, ff=512, vocab=512, seed=1234, tied=False):
    """A small llama model in bf16 (the reference's dev_make_synth layout) plus the
    f32 values of every 2-D weight; ffn and attention weights use N(0, 0.02) + outliers."""
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path, arch="llama")
    w.add_block_count(n_layer)
    w.add_context_length(512)
    w.add_embedding_length(hidden)
    w.add_feed_forward_length(ff)
    w.add_head_count(8)
    w.add_head_count_kv(2)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_file_type(gguf.LlamaFileType.MOSTLY_BF16)
    vals = {}

    def weight(name, rows, cols):
        a = rng.normal(0.0, 0.02, (rows, cols))
        m = rng.random(a.shape) < 0.001
        a[m] = rng.normal(0.0, 0.5, int(m.sum()))
        w.add_tensor(name, bf16_bytes(a), raw_dtype=GGMLQuantizationType.BF16)
        vals[name] = bf16_values(a)

    weight("token_embd.weight", vocab, hidden)
    for i in range(n_layer):
        p = f"blk.{i}."
        weight(p + "attn_q.weight", hidden, hidden)
        weight(p + "attn_k.weight", hidden // 4, hidden)
        weight(p + "attn_v.weight", hidden // 4, hidden)
        weight(p + "attn_output.weight", hidden, hidden)
        weight(p + "ffn_gate.weight", ff, hidden)
        weight(p + "ffn_up.weight", ff, hidden)
        weight(p + "ffn_down.weight", hidden, ff)
        w.add_tensor(p + "attn_norm.weight", np.ones(hidden, np.float32))
        w.add_tensor(p + "ffn_norm.weight", np.ones(hidden, np.float32))
    w.add_tensor("output_norm.weight", np.ones(hidden, np.float32))
    if not tied:
        weight("output.weight", vocab, hidden)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return vals


def write_imatrix(path: Path, names_cols: dict[str, int], seed=1) -> dict[str, np.ndarray]:
    """lognormal(0, 1.5) per column, stored as in_sum2 with counts 1 (so qw = in_sum2)."""
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path, arch="imatrix")
    w.add_string("general.type", "imatrix")
    out = {}
    for name, k in names_cols.items():
        v = rng.lognormal(0.0, 1.5, k).astype(np.float32)
        w.add_tensor(name + ".in_sum2", v)
        w.add_tensor(name + ".counts", np.array([1.0], dtype=np.float32))
        out[name] = v
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return out
