"""The type-mix policy against the reference's plans (tests/golden/scheme_plans.json.z)."""

import json
import zlib
from pathlib import Path

import pytest
from gguf import GGMLQuantizationType as GT

from kernels import scheme

GOLD = json.loads(zlib.decompress((Path(__file__).parent / "golden" / "scheme_plans.json.z").read_bytes()))


def _kwargs(fl):
    kw = dict(fl)
    for key in ("token_embedding_type", "output_tensor_type"):
        if key in kw:
            kw[key] = GT[kw[key]]
    if "tt_overrides" in kw:
        kw["tt_overrides"] = [(p, GT[t]) for p, t in kw["tt_overrides"]]
    return kw


@pytest.mark.parametrize("mname", sorted(GOLD["models"]))
def test_plans_match_reference(mname):
    m = GOLD["models"][mname]
    model = scheme.ModelInfo(**m["facts"])
    tensors = [(n, tuple(ne), GT[s]) for n, ne, s in m["tensors"]]
    order = sorted(tensors, key=lambda t: scheme.weight_name_key(t[0]))
    checked = 0
    for key, want in GOLD["plans"].items():
        mk, sname, fi = key.split("|")
        if mk != mname:
            continue
        opt = scheme.parse_scheme(sname)
        if opt is None:  # scheme whose file type this gguf package lacks (Q2_0)
            continue
        try:
            got = [t.name for t in scheme.decide_types(model, order, opt.ftype, **_kwargs(GOLD["flags"][int(fi)]))]
        except ValueError as e:
            got = f"error: {e}"
        assert got == want, f"{key}"
        checked += 1
    assert checked > 100


def test_weight_name_key_orders_like_the_loader():
    names = ["blk.10.attn_q.weight", "output.weight", "blk.2.ffn_up.weight", "token_embd.weight", "blk.2.attn_k.weight"]
    assert sorted(names, key=scheme.weight_name_key) == [
        "output.weight", "token_embd.weight", "blk.2.attn_k.weight", "blk.2.ffn_up.weight", "blk.10.attn_q.weight"]


def test_requires_imatrix():
    FT = scheme.FT
    assert scheme.tensor_requires_imatrix("blk.0.attn_q.weight", GT.IQ2_XXS, FT.MOSTLY_IQ2_XXS)
    assert not scheme.tensor_requires_imatrix("token_embd.weight", GT.IQ2_XXS, FT.MOSTLY_IQ2_XXS)
    assert scheme.tensor_requires_imatrix("blk.0.ffn_down.weight", GT.Q2_K, FT.MOSTLY_Q2_K_S)
    assert not scheme.tensor_requires_imatrix("blk.0.ffn_down.weight", GT.Q2_K, FT.MOSTLY_Q2_K)


def test_scheme_table_marks_supported():
    table = scheme.format_scheme_table()
    for name in ("Q4_K_M", "IQ2_XXS", "Q6_K", "IQ3_XXS", "IQ2_M", "Q4_0", "IQ4_XS", "Q4_1", "Q5_0", "Q5_1", "Q8_0"):
        assert scheme.parse_scheme(name).supported, name
        assert f"[x] {name}" in table
    for name in ("IQ1_S", "TQ1_0", "IQ4_NL"):
        assert not scheme.parse_scheme(name).supported, name
