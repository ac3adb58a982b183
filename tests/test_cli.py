"""quant-studio.py end to end (drop-in CLI): plans and errors on CPU, bytes on GPU."""

import subprocess
import sys

import numpy as np
import pytest
import torch
from gguf import GGMLQuantizationType as GT, GGUFReader
from gguf.quants import quantize as gguf_quantize

import gguf
import oracle
from conftest import PKG
from synth_gguf import write_imatrix, write_llama, write_mixed

CLI = str(PKG / "quant-studio.py")
ORACLE_NAMES = {GT.Q4_0: "q4_0", GT.Q2_K: "q2_k", GT.Q3_K: "q3_k", GT.Q4_K: "q4_k", GT.Q5_K: "q5_k",
                GT.Q6_K: "q6_k", GT.IQ4_XS: "iq4_xs", GT.IQ2_XXS: "iq2_xxs", GT.IQ2_XS: "iq2_xs",
                GT.IQ2_S: "iq2_s", GT.IQ3_XXS: "iq3_xxs", GT.IQ3_S: "iq3_s", GT.Q4_1: "q4_1", GT.Q5_0: "q5_0",
                GT.Q5_1: "q5_1", GT.Q8_0: "q8_0"}


def run(*args, check=True):
    return subprocess.run([sys.executable, CLI, *map(str, args)], capture_output=True, text=True, check=check)


def test_dry_run_plan(tmp_path):
    src = tmp_path / "m.gguf"
    write_llama(src)
    r = run(src, tmp_path / "o.gguf", "Q4_K_M", "--dry-run")
    lines = [l for l in r.stdout.splitlines() if " -> " in l and not l.startswith("dry run")]
    plan = {l.split()[0]: l.split()[3] for l in lines}
    assert plan["blk.0.attn_q.weight"] == "Q4_K"
    assert plan["blk.0.attn_v.weight"] == "Q4_K"
    assert plan["blk.1.attn_v.weight"] == "Q6_K"          # more bits on the last eighth of attn_v
    assert plan["blk.1.ffn_down.weight"] == "Q6_K"
    assert plan["output.weight"] == "Q6_K"
    assert plan["blk.0.attn_norm.weight"] == "F32"
    assert "dry run:" in r.stdout


def test_errors(tmp_path):
    src = tmp_path / "m.gguf"
    write_llama(src)
    r = run(src, tmp_path / "o.gguf", "IQ2_XXS", check=False)
    assert r.returncode != 0 and "importance matrix" in r.stderr
    r = run(src, tmp_path / "o.gguf", "IQ1_S", check=False)
    assert r.returncode != 0 and "not supported" in r.stderr
    r = run(src, tmp_path / "o.gguf", "NOPE", check=False)
    assert r.returncode != 0 and "unknown quantization scheme" in r.stderr
    r = run(src, tmp_path / "o.gguf", "Q4_0", "--keep-split", check=False)
    assert r.returncode != 0 and "--keep-split" in r.stderr
    r = run(src, "Q4_0", "4", check=False)               # llama-quantize positional nthreads
    assert r.returncode != 0 and "nthreads" in r.stderr


@pytest.mark.gpu
def test_q4_0_end_to_end_like_reference_test(tmp_path):
    """The reference's own end-to-end check (tests/test_q4_0.py), run through qs-b200."""
    src, dst = tmp_path / "in.gguf", tmp_path / "out.gguf"
    expect = write_mixed(src)
    run(src, dst, "q4_0", "--mem", "64K")
    r_in, r_out = GGUFReader(src), GGUFReader(dst)
    assert r_out.get_field("general.architecture").contents() == "llama"
    assert r_out.get_field("llama.context_length").contents() == 2048
    assert r_out.get_field("test.flag").contents() is True
    assert r_out.get_field("tokenizer.ggml.tokens").contents() == ["<s>", "</s>", "hello"]
    assert r_out.get_field("general.file_type").contents() == int(gguf.LlamaFileType.MOSTLY_Q4_0)
    assert r_out.get_field("general.quantization_version").contents() == gguf.GGML_QUANT_VERSION
    outs = {t.name: t for t in r_out.tensors}
    for t_in in r_in.tensors:
        t_out = outs[t_in.name]
        assert list(t_out.shape) == list(t_in.shape)
        if t_in.name in expect:
            assert t_out.tensor_type == GT.Q4_0
            ref = gguf_quantize(expect[t_in.name], GT.Q4_0)
            assert np.array_equal(t_out.data.reshape(-1), ref.reshape(-1)), t_in.name
        else:
            assert t_out.tensor_type == t_in.tensor_type
            assert np.array_equal(t_out.data.reshape(-1).view(np.uint8), t_in.data.reshape(-1).view(np.uint8))


def _check_against_oracle(dst, vals, imat):
    r = GGUFReader(dst)
    n = 0
    for t in r.tensors:
        if t.name not in vals or t.tensor_type not in ORACLE_NAMES:
            continue
        x = vals[t.name]
        qw = imat.get(t.name)
        name = ORACLE_NAMES[t.tensor_type]
        if qw is None and name in ("iq2_xxs", "iq2_xs", "iq2_s"):
            continue
        if name in ("q4_0", "q4_1", "q5_0", "q5_1", "q8_0"):  # these ignore importance weights
            qw = None
        ref = oracle.quantize(name, x, None if qw is None else qw[: x.shape[1]])
        assert np.array_equal(np.asarray(t.data).reshape(ref.shape), ref), f"{t.name} ({name})"
        n += 1
    return n


@pytest.mark.gpu
@pytest.mark.parametrize("scheme_name", ["Q4_K_M", "IQ3_XXS", "IQ2_M", "Q3_K_S", "IQ4_XS"])
def test_mixture_end_to_end_vs_oracle(tmp_path, scheme_name):
    src, dst, im = tmp_path / "in.gguf", tmp_path / "out.gguf", tmp_path / "im.gguf"
    vals = write_llama(src)
    imat = write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    run(src, dst, scheme_name, "--imatrix", im, "--mem", "256K")
    assert _check_against_oracle(dst, vals, imat) >= 10


def _plan(r):
    lines = [l for l in r.stdout.splitlines() if " -> " in l and not l.startswith("dry run")]
    return {l.split()[0]: l.split()[3] for l in lines}


def test_dry_run_plans_the_formats_the_reference_rejects(tmp_path):
    """The policy's Q5_0 / Q5_1 / Q8_0 shape fallbacks (scheme.py:375) and the Q4_1 ffn_down of
    Q4_0 with an imatrix (scheme.py:521-523) plan and run here; the reference stops on them
    (quant-studio.py:396-399)."""
    src, im = tmp_path / "m.gguf", tmp_path / "im.gguf"
    vals = write_llama(src, hidden=288)                  # rows of 288: not a multiple of 256
    write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    plan = _plan(run(src, tmp_path / "o.gguf", "Q4_K_M", "--dry-run"))
    assert plan["blk.0.attn_q.weight"] == "Q5_0" and plan["blk.1.attn_v.weight"] == "Q8_0"
    plan = _plan(run(src, tmp_path / "o.gguf", "Q5_K_M", "--dry-run"))
    assert plan["blk.0.attn_q.weight"] == "Q5_1"
    src8 = tmp_path / "m8.gguf"
    vals = write_llama(src8, n_layer=8)
    write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    plan = _plan(run(src8, tmp_path / "o.gguf", "Q4_0", "--imatrix", im, "--dry-run"))
    assert plan["blk.0.ffn_down.weight"] == "Q4_1" and plan["blk.1.ffn_down.weight"] == "Q4_0"


@pytest.mark.gpu
@pytest.mark.parametrize("scheme_name,hidden,n_layer", [("Q4_K_M", 288, 2), ("Q5_K_M", 288, 2), ("Q4_0", 256, 8),
                                                        ("Q5_0", 256, 8), ("Q8_0", 256, 2)])
def test_fallback_formats_end_to_end_vs_oracle(tmp_path, scheme_name, hidden, n_layer):
    src, dst, im = tmp_path / "in.gguf", tmp_path / "out.gguf", tmp_path / "im.gguf"
    vals = write_llama(src, hidden=hidden, n_layer=n_layer)
    imat = write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    run(src, dst, scheme_name, "--imatrix", im, "--mem", "256K")
    types = {t.tensor_type for t in GGUFReader(dst).tensors}
    want = {"Q4_K_M": GT.Q5_0, "Q5_K_M": GT.Q5_1, "Q4_0": GT.Q4_1, "Q5_0": GT.Q5_1, "Q8_0": GT.Q8_0}[scheme_name]
    assert want in types
    assert _check_against_oracle(dst, vals, imat) >= 8


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharding_over_gpus_gives_identical_bytes(tmp_path):
    src, im = tmp_path / "in.gguf", tmp_path / "im.gguf"
    vals = write_llama(src, n_layer=4)
    write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    run(src, tmp_path / "one.gguf", "IQ3_XXS", "--imatrix", im, "--mem", "128K", "--gpus", "1")
    run(src, tmp_path / "two.gguf", "IQ3_XXS", "--imatrix", im, "--mem", "128K", "--gpus", str(torch.cuda.device_count()))
    assert (tmp_path / "one.gguf").read_bytes() == (tmp_path / "two.gguf").read_bytes()
