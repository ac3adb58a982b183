"""Per-tensor type-mix policy: which GGML type each tensor of a model gets.

Same decisions as the reference's kernels/scheme.py, itself a port of llama.cpp's
tools/quantize/quantize.cpp (QUANT_OPTIONS) and src/llama-quant.cpp at commit
9871d51fd7a6a4fb300100ed236f3962e72fd6ee (tensor_allows_quantization,
tensor_get_category, llama_tensor_get_type_impl, tensor_type_fallback,
llama_ftype_get_default_type, tensor_requires_imatrix). The rules are restated here
as per-category rule functions; every branch keeps the reference's order, because the
first matching rule wins and some rules advance layer counters.

The selection is stateful (QuantState counters), so tensors must be visited in
weight_name_key order, the llama model loader's order.
"""

from __future__ import annotations

import re
import sys
from dataclasses import dataclass, field
from enum import Enum

from gguf import GGMLQuantizationType as GT
from gguf.constants import GGML_QUANT_SIZES, LlamaFileType as FT

LLAMA_CPP_COMMIT = "9871d51fd7a6a4fb300100ed236f3962e72fd6ee"


def _ft(name: str):
    """File-type member by name, or None if this gguf package predates it."""
    return getattr(FT, name, None)


def _gt(name: str):
    return getattr(GT, name, None)


# ---------------------------------------------------------------------------
# schemes (quantize.cpp QUANT_OPTIONS): name, file type, description
# ---------------------------------------------------------------------------
_SCHEMES = (
    ("Q1_0", "MOSTLY_Q1_0", "1.125 bpw quantization"),
    ("Q2_0", "MOSTLY_Q2_0", "2.25 bpw quantization (group 64)"),
    ("Q4_0", "MOSTLY_Q4_0", "4.34G, +0.4685 ppl @ Llama-3-8B"),
    ("Q4_1", "MOSTLY_Q4_1", "4.78G, +0.4511 ppl @ Llama-3-8B"),
    ("MXFP4_MOE", "MOSTLY_MXFP4_MOE", "MXFP4 MoE"),
    ("Q5_0", "MOSTLY_Q5_0", "5.21G, +0.1316 ppl @ Llama-3-8B"),
    ("Q5_1", "MOSTLY_Q5_1", "5.65G, +0.1062 ppl @ Llama-3-8B"),
    ("IQ2_XXS", "MOSTLY_IQ2_XXS", "2.06 bpw quantization"),
    ("IQ2_XS", "MOSTLY_IQ2_XS", "2.31 bpw quantization"),
    ("IQ2_S", "MOSTLY_IQ2_S", "2.5  bpw quantization"),
    ("IQ2_M", "MOSTLY_IQ2_M", "2.7  bpw quantization"),
    ("IQ1_S", "MOSTLY_IQ1_S", "1.56 bpw quantization"),
    ("IQ1_M", "MOSTLY_IQ1_M", "1.75 bpw quantization"),
    ("TQ1_0", "MOSTLY_TQ1_0", "1.69 bpw ternarization"),
    ("TQ2_0", "MOSTLY_TQ2_0", "2.06 bpw ternarization"),
    ("Q2_K", "MOSTLY_Q2_K", "2.96G, +3.5199 ppl @ Llama-3-8B"),
    ("Q2_K_S", "MOSTLY_Q2_K_S", "2.96G, +3.1836 ppl @ Llama-3-8B"),
    ("IQ3_XXS", "MOSTLY_IQ3_XXS", "3.06 bpw quantization"),
    ("IQ3_S", "MOSTLY_IQ3_S", "3.44 bpw quantization"),
    ("IQ3_M", "MOSTLY_IQ3_M", "3.66 bpw quantization mix"),
    ("Q3_K", "MOSTLY_Q3_K_M", "alias for Q3_K_M"),
    ("IQ3_XS", "MOSTLY_IQ3_XS", "3.3 bpw quantization"),
    ("Q3_K_S", "MOSTLY_Q3_K_S", "3.41G, +1.6321 ppl @ Llama-3-8B"),
    ("Q3_K_M", "MOSTLY_Q3_K_M", "3.74G, +0.6569 ppl @ Llama-3-8B"),
    ("Q3_K_L", "MOSTLY_Q3_K_L", "4.03G, +0.5562 ppl @ Llama-3-8B"),
    ("IQ4_NL", "MOSTLY_IQ4_NL", "4.50 bpw non-linear quantization"),
    ("IQ4_XS", "MOSTLY_IQ4_XS", "4.25 bpw non-linear quantization"),
    ("Q4_K", "MOSTLY_Q4_K_M", "alias for Q4_K_M"),
    ("Q4_K_S", "MOSTLY_Q4_K_S", "4.37G, +0.2689 ppl @ Llama-3-8B"),
    ("Q4_K_M", "MOSTLY_Q4_K_M", "4.58G, +0.1754 ppl @ Llama-3-8B"),
    ("Q5_K", "MOSTLY_Q5_K_M", "alias for Q5_K_M"),
    ("Q5_K_S", "MOSTLY_Q5_K_S", "5.21G, +0.1049 ppl @ Llama-3-8B"),
    ("Q5_K_M", "MOSTLY_Q5_K_M", "5.33G, +0.0569 ppl @ Llama-3-8B"),
    ("Q6_K", "MOSTLY_Q6_K", "6.14G, +0.0217 ppl @ Llama-3-8B"),
    ("Q8_0", "MOSTLY_Q8_0", "7.96G, +0.0026 ppl @ Llama-3-8B"),
    ("F16", "MOSTLY_F16", "14.00G, +0.0020 ppl @ Mistral-7B"),
    ("BF16", "MOSTLY_BF16", "14.00G, -0.0050 ppl @ Mistral-7B"),
    ("F32", "ALL_F32", "26.00G              @ 7B"),
    ("COPY", "ALL_F32", "only copy tensors, no quantizing"),
)

# file type -> the tensor type most tensors get (llama_ftype_get_default_type)
_DEFAULT_TYPE = {
    "MOSTLY_Q4_0": "Q4_0", "MOSTLY_Q4_1": "Q4_1", "MOSTLY_Q5_0": "Q5_0", "MOSTLY_Q5_1": "Q5_1",
    "MOSTLY_Q8_0": "Q8_0", "MOSTLY_F16": "F16", "MOSTLY_BF16": "BF16", "ALL_F32": "F32",
    "MOSTLY_Q1_0": "Q1_0", "MOSTLY_Q2_0": "Q2_0", "MOSTLY_MXFP4_MOE": "MXFP4",
    "MOSTLY_Q2_K_S": "Q2_K", "MOSTLY_Q2_K": "Q2_K", "MOSTLY_IQ3_XS": "IQ3_S",
    "MOSTLY_Q3_K_S": "Q3_K", "MOSTLY_Q3_K_M": "Q3_K", "MOSTLY_Q3_K_L": "Q3_K",
    "MOSTLY_Q4_K_S": "Q4_K", "MOSTLY_Q4_K_M": "Q4_K", "MOSTLY_Q5_K_S": "Q5_K", "MOSTLY_Q5_K_M": "Q5_K",
    "MOSTLY_Q6_K": "Q6_K", "MOSTLY_TQ1_0": "TQ1_0", "MOSTLY_TQ2_0": "TQ2_0",
    "MOSTLY_IQ2_XXS": "IQ2_XXS", "MOSTLY_IQ2_XS": "IQ2_XS",
    "MOSTLY_IQ2_S": "IQ2_XS",  # the IQ2_S scheme keeps most tensors at IQ2_XS (upstream table)
    "MOSTLY_IQ2_M": "IQ2_S", "MOSTLY_IQ3_XXS": "IQ3_XXS", "MOSTLY_IQ1_S": "IQ1_S",
    "MOSTLY_IQ1_M": "IQ1_M", "MOSTLY_IQ4_NL": "IQ4_NL", "MOSTLY_IQ4_XS": "IQ4_XS",
    "MOSTLY_IQ3_S": "IQ3_S", "MOSTLY_IQ3_M": "IQ3_S",
}
_DEFAULT_BY_FT = {_ft(f): _gt(t) for f, t in _DEFAULT_TYPE.items() if _ft(f) is not None}


def ftype_default_type(ftype: FT) -> GT | None:
    """llama_ftype_get_default_type()."""
    return _DEFAULT_BY_FT.get(ftype)


def _studio_tensor_types() -> set[GT]:
    from . import QUANT_TYPES
    return {s.ggml_type for s in QUANT_TYPES.values()}


@dataclass(frozen=True)
class QuantOption:
    name: str
    ftype: FT
    desc: str

    @property
    def default_type(self) -> GT | None:
        return ftype_default_type(self.ftype)

    @property
    def supported(self) -> bool:
        """A scheme is runnable when its default tensor type has a kernel here."""
        return self.name != "COPY" and self.default_type in _studio_tensor_types()


QUANT_OPTIONS: list[QuantOption] = [QuantOption(n, _ft(f), d) for n, f, d in _SCHEMES if _ft(f) is not None]


def parse_scheme(name: str) -> QuantOption | None:
    key = name.upper()
    return next((o for o in QUANT_OPTIONS if o.name.upper() == key), None)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
_PLAIN = {GT.F32, GT.F16, GT.BF16, GT.F64, GT.I8, GT.I16, GT.I32, GT.I64}


def ggml_is_quantized(t: GT) -> bool:
    return t not in _PLAIN


def ggml_blck_size(t: GT) -> int:
    return GGML_QUANT_SIZES[t][0]


class Category(Enum):
    OUTPUT = 1
    TOKEN_EMBD = 2
    ATTENTION_QKV = 3
    ATTENTION_KV_B = 4
    ATTENTION_V = 5
    ATTENTION_K = 6
    ATTENTION_Q = 7
    ATTENTION_OUTPUT = 8
    FFN_UP = 9
    FFN_GATE = 10
    FFN_DOWN = 11
    OTHER = 12


_TOKEN_EMBD_NAMES = ("token_embd.weight", "per_layer_token_embd.weight")
# substring -> category, tried in this order (tensor_get_category)
_CATEGORY_BY_SUBSTR = (
    ("attn_qkv.weight", Category.ATTENTION_QKV),
    ("attn_kv_b.weight", Category.ATTENTION_KV_B),
    ("attn_v.weight", Category.ATTENTION_V),
    ("attn_k.weight", Category.ATTENTION_K),
    ("attn_q.weight", Category.ATTENTION_Q),
    ("attn_output.weight", Category.ATTENTION_OUTPUT),
    ("ffn_up", Category.FFN_UP),
    ("ffn_gate", Category.FFN_GATE),
    ("ffn_down", Category.FFN_DOWN),
)


def tensor_get_category(name: str) -> Category:
    if name == "output.weight":
        return Category.OUTPUT
    if name in _TOKEN_EMBD_NAMES:
        return Category.TOKEN_EMBD
    for frag, cat in _CATEGORY_BY_SUBSTR:
        if frag in name:
            return cat
    return Category.OTHER


_BLK = re.compile(r"blk\.(\d+)\.")


def weight_name_key(name: str) -> tuple[int, str]:
    """Loader order: layer number (non-layer tensors first), then name."""
    m = _BLK.match(name)
    return (int(m.group(1)) if m else -1, name)


def category_is_attn_v(cat: Category) -> bool:
    return cat in (Category.ATTENTION_V, Category.ATTENTION_QKV, Category.ATTENTION_KV_B)


# tensors that are never quantized, by name fragment (tensor_allows_quantization)
_KEEP_FRAGMENTS = (
    "_norm.weight", "ffn_gate_inp.weight", "ffn_gate_tid2eid.weight", "altup", "laurel",
    "per_layer_model_proj", "ssm_conv1d", "shortconv.conv.weight", "indexer.k_proj.weight",
    "indexer.q_proj.weight", "attn_rel_b.weight", ".position_embd", "sam.pos_embd", "sam.neck.",
    "sam.net_", ".rel_pos", ".patch_embd", ".patch_merger", "a.rvq.codebook", "mm.a.code_embd",
) + tuple(f"time_mix_{k}.weight" for k in
          ("first", "w0", "w1", "w2", "v0", "v1", "v2", "a0", "a1", "a2", "g1", "g2",
           "decay_w1", "decay_w2", "lerp_fused"))


def tensor_allows_quantization(name: str, n_dims: int, quantize_output_tensor: bool = True,
                               only_copy: bool = False) -> bool:
    if only_copy or n_dims < 2 or not name.endswith("weight"):
        return False
    if name == "output.weight" and not quantize_output_tensor:
        return False
    if name in ("position_embd.weight", "token_types.weight"):
        return False
    return all(frag not in name for frag in _KEEP_FRAGMENTS)


# ---------------------------------------------------------------------------
# model facts and selection state
# ---------------------------------------------------------------------------
@dataclass
class ModelInfo:
    arch: str = ""
    n_layer: int = 0
    n_expert: int = 0
    n_head: int = 0
    n_head_kv: int = 0
    is_70b: bool = False  # llama with 80 layers (llama.cpp reads the model type)

    @property
    def n_gqa(self) -> int:
        return self.n_head // self.n_head_kv if self.n_head_kv > 0 else 0

    @classmethod
    def from_reader(cls, reader) -> "ModelInfo":
        arch = reader.get_field("general.architecture").contents()

        def hparam(key: str, default: int = 0) -> int:
            f = reader.get_field(f"{arch}.{key}")
            if f is None:
                return default
            v = f.contents()
            return int(v[0]) if isinstance(v, list) else int(v)  # per-layer arrays: layer 0

        n_layer = hparam("block_count")
        n_head = hparam("attention.head_count")
        return cls(arch=arch, n_layer=n_layer, n_expert=hparam("expert_count"), n_head=n_head,
                   n_head_kv=hparam("attention.head_count_kv", n_head),
                   is_70b=arch == "llama" and n_layer == 80)


@dataclass
class QuantState:
    """Counters that make the choice depend on the tensor's position among its kind."""
    n_attention_wv: int = 0
    n_ffn_down: int = 0
    n_ffn_gate: int = 0
    n_ffn_up: int = 0
    i_attention_wv: int = 0
    i_ffn_down: int = 0
    i_ffn_gate: int = 0
    i_ffn_up: int = 0
    n_fallback: int = 0
    has_imatrix: bool = False
    has_tied_embeddings: bool = True
    tensor_type_patterns: list = field(default_factory=list)


def init_state(model: ModelInfo, tensor_names: list[str], has_imatrix: bool,
               tt_overrides: list[tuple[str, GT]] | None = None) -> QuantState:
    qs = QuantState(has_imatrix=has_imatrix)
    qs.n_attention_wv = sum(category_is_attn_v(tensor_get_category(n)) for n in tensor_names)
    qs.has_tied_embeddings = "output.weight" not in tensor_names
    qs.n_ffn_down = qs.n_ffn_gate = qs.n_ffn_up = model.n_layer
    qs.tensor_type_patterns = [(re.compile(p), t) for p, t in (tt_overrides or [])]
    return qs


def _use_more_bits(i: int, n: int) -> bool:
    """First and last eighth of the layers, and every third one in between."""
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


def _layer_of(counter: int, n_layer: int, name: str, n_expert: int) -> tuple[int, int]:
    """Layer index of a tensor: its counter, or for MoE models the blk.N in its name."""
    if n_expert <= 1:
        return counter, n_layer
    m = _BLK.match(name)
    if m is None:
        raise ValueError(f"failed to determine layer for tensor {name}")
    i = int(m.group(1))
    if not 0 <= i < n_layer:
        raise ValueError(f"bad layer {i} for tensor {name}")
    return i, n_layer


_FALLBACK = {"IQ1_S": "IQ4_NL", "IQ1_M": "IQ4_NL", "IQ2_XXS": "IQ4_NL", "IQ2_XS": "IQ4_NL",
             "IQ2_S": "IQ4_NL", "IQ3_XXS": "IQ4_NL", "IQ3_S": "IQ4_NL", "IQ4_XS": "IQ4_NL",
             "Q2_0": "Q4_0", "Q2_K": "Q4_0", "Q3_K": "Q4_0", "TQ1_0": "Q4_0", "TQ2_0": "Q4_0",
             "Q4_K": "Q5_0", "Q5_K": "Q5_1", "Q6_K": "Q8_0"}
_FALLBACK_BY_GT = {_gt(a): _gt(b) for a, b in _FALLBACK.items() if _gt(a) is not None}


def tensor_type_fallback(qs: QuantState, name: str, ncols: int, target: GT) -> GT:
    """Rows that do not split into the target's blocks drop to a smaller-block type."""
    if ncols % ggml_blck_size(target) == 0:
        return target
    qs.n_fallback += 1
    if target not in _FALLBACK_BY_GT:
        raise ValueError(f"no tensor type fallback is defined for type {target.name}")
    alt = _FALLBACK_BY_GT[target]
    if ncols % ggml_blck_size(alt) != 0:
        alt = GT.F16
    print(f"warning: {name}: ncols {ncols} not divisible by {ggml_blck_size(target)} "
          f"(required for {target.name}) -> falling back to {alt.name}", file=sys.stderr)
    return alt


# ---------------------------------------------------------------------------
# the mixture rules (llama_tensor_get_type_impl), one function per tensor kind
# ---------------------------------------------------------------------------
def _fts(*names: str) -> set:
    return {f for f in (_ft(n) for n in names) if f is not None}


_IQ_LOW = _fts("MOSTLY_IQ2_XXS", "MOSTLY_IQ2_XS", "MOSTLY_IQ1_S", "MOSTLY_IQ2_S", "MOSTLY_IQ2_M", "MOSTLY_IQ1_M")
_IQ2S_M = _fts("MOSTLY_IQ2_S", "MOSTLY_IQ2_M")
_IQ1 = _fts("MOSTLY_IQ1_S", "MOSTLY_IQ1_M")


@dataclass
class _Ctx:
    qs: QuantState
    model: ModelInfo
    ftype: FT
    name: str
    ne: tuple
    cat: Category
    tok_type: GT | None
    out_type: GT | None


def _rule_output_or_tied_embd(c: _Ctx, t: GT) -> GT:
    if c.out_type is not None:
        return c.out_type
    if c.ftype == _ft("MOSTLY_MXFP4_MOE") or c.model.arch == "falcon" or c.ne[0] % ggml_blck_size(t):
        return GT.Q8_0
    if c.ftype in _fts("MOSTLY_IQ2_XXS", "MOSTLY_IQ2_XS", "MOSTLY_IQ3_XXS", "MOSTLY_IQ1_S",
                       "MOSTLY_IQ2_S", "MOSTLY_IQ2_M", "MOSTLY_IQ1_M"):
        return GT.Q5_K
    return t if t == GT.Q8_0 else GT.Q6_K


def _rule_token_embd(c: _Ctx, t: GT) -> GT:
    if c.tok_type is not None:
        return c.tok_type
    if c.ftype in _fts("MOSTLY_IQ2_XXS", "MOSTLY_IQ2_XS", "MOSTLY_IQ1_S", "MOSTLY_IQ1_M"):
        return GT.Q2_K
    if c.ftype in _IQ2S_M or c.ftype == _ft("MOSTLY_IQ3_XXS"):
        return GT.IQ3_S
    if c.ftype in _fts("MOSTLY_TQ1_0", "MOSTLY_TQ2_0", "MOSTLY_Q2_0"):
        return GT.Q4_K
    return t


def _rule_low_bit_iq(c: _Ctx, t: GT) -> GT:
    """Every non-embedding tensor of the 1-2 bit IQ file types."""
    qs, m, cat = c.qs, c.model, c.cat
    cheap = GT.IQ3_S if c.ftype in _IQ2S_M else GT.Q2_K
    if category_is_attn_v(cat):
        t = GT.Q4_K if (m.n_gqa >= 4 or m.n_expert >= 4) else cheap
        qs.i_attention_wv += 1
    elif m.n_expert == 8 and cat == Category.ATTENTION_K:
        t = GT.Q4_K
    elif cat == Category.FFN_DOWN:
        if qs.i_ffn_down < qs.n_ffn_down // 8:
            t = cheap
        qs.i_ffn_down += 1
    elif cat == Category.ATTENTION_OUTPUT:
        if m.n_expert == 8:
            t = GT.Q5_K
        elif c.ftype in _IQ1:
            t = GT.IQ2_XXS
        elif c.ftype in _IQ2S_M:
            t = GT.IQ3_S
    return t


def _rule_attn_v(c: _Ctx, t: GT) -> GT:
    qs, m, f = c.qs, c.model, c.ftype
    gqa4 = m.n_gqa >= 4
    if f == _ft("MOSTLY_Q2_K"):
        t = GT.Q4_K if gqa4 else GT.Q3_K
    elif f == _ft("MOSTLY_Q2_K_S") and gqa4:
        t = GT.Q4_K
    elif f == _ft("MOSTLY_IQ3_XXS"):
        t = GT.Q4_K if gqa4 else (GT.IQ3_XXS if qs.has_imatrix else GT.IQ3_S)
    elif f in _fts("MOSTLY_IQ3_XS", "MOSTLY_IQ3_S") and gqa4:
        t = GT.Q4_K
    elif f == _ft("MOSTLY_IQ3_M"):
        t = GT.Q4_K
    elif f == _ft("MOSTLY_Q3_K_M"):
        t = GT.Q5_K if qs.i_attention_wv < 2 else GT.Q4_K
    elif f == _ft("MOSTLY_Q3_K_L"):
        t = GT.Q5_K
    elif f in _fts("MOSTLY_IQ4_NL", "MOSTLY_IQ4_XS") and gqa4:
        t = GT.Q5_K
    elif f in _fts("MOSTLY_Q4_K_M", "MOSTLY_Q5_K_M") and _use_more_bits(qs.i_attention_wv, qs.n_attention_wv):
        t = GT.Q6_K
    elif f == _ft("MOSTLY_Q4_K_S") and qs.i_attention_wv < 4:
        t = GT.Q5_K
    if m.is_70b and t in (GT.Q3_K, GT.Q4_K):
        t = GT.Q5_K  # 8 heads share attn_v: the tensor is small, bits are cheap
    if m.n_expert == 8:
        t = GT.Q8_0
    qs.i_attention_wv += 1
    return t


def _rule_attn_k(c: _Ctx, t: GT) -> GT:
    if c.model.n_expert == 8:
        return GT.Q8_0
    return _rule_attn_q(c, t)


def _rule_attn_q(c: _Ctx, t: GT) -> GT:
    if c.ftype == _ft("MOSTLY_IQ3_XS"):
        return GT.IQ3_XXS
    if c.ftype == _ft("MOSTLY_IQ3_XXS"):
        return GT.IQ2_S
    return t


def _rule_ffn_down(c: _Ctx, t: GT) -> GT:
    qs, m, f = c.qs, c.model, c.ftype
    i, n = _layer_of(qs.i_ffn_down, qs.n_ffn_down, c.name, max(1, m.n_expert))
    falcon = m.arch == "falcon"
    first8 = i < n // 8
    if f == _ft("MOSTLY_Q2_K"):
        t = GT.Q3_K
    elif f == _ft("MOSTLY_Q2_K_S"):
        if first8:
            t = GT.Q4_K
    elif f == _ft("MOSTLY_IQ3_XXS") and not qs.has_imatrix:
        t = GT.Q4_K if first8 else GT.Q3_K
    elif f == _ft("MOSTLY_Q3_K_M"):
        if i < n // 16:
            t = GT.Q5_K
        else:
            t = GT.Q4_K if (not falcon or _use_more_bits(i, n)) else GT.Q3_K
    elif f == _ft("MOSTLY_IQ3_M") and (first8 or (m.n_expert == 8 and _use_more_bits(i, n))):
        t = GT.Q4_K
    elif f == _ft("MOSTLY_Q3_K_L"):
        t = GT.Q4_K if falcon else GT.Q5_K
    elif f == _ft("MOSTLY_Q4_K_M"):
        if falcon:
            t = GT.Q6_K if i < n // 16 else (GT.Q5_K if _use_more_bits(i, n) else GT.Q4_K)
        elif _use_more_bits(i, n):
            t = GT.Q6_K
    elif first8 and f in _fts("MOSTLY_IQ4_NL", "MOSTLY_IQ4_XS") and not qs.has_imatrix:
        t = GT.Q5_K
    elif f == _ft("MOSTLY_Q5_K_M") and _use_more_bits(i, n):
        t = GT.Q6_K
    elif f == _ft("MOSTLY_Q4_K_S") and not falcon and first8:
        t = GT.Q5_K
    elif f in _fts("MOSTLY_Q4_0", "MOSTLY_Q5_0") and qs.has_imatrix and first8:
        t = GT.Q4_1 if f == _ft("MOSTLY_Q4_0") else GT.Q5_1  # first ffn_down layers are fragile
    qs.i_ffn_down += 1
    return t


def _rule_attn_output(c: _Ctx, t: GT) -> GT:
    f = c.ftype
    if c.model.arch == "falcon":
        return GT.Q4_K if f == _ft("MOSTLY_Q3_K_L") else t
    if c.model.n_expert == 8:
        if f in _fts("MOSTLY_Q2_K", "MOSTLY_IQ3_XS", "MOSTLY_IQ3_XXS", "MOSTLY_Q3_K_S", "MOSTLY_Q3_K_M",
                     "MOSTLY_IQ4_NL", "MOSTLY_Q4_K_S", "MOSTLY_Q4_K_M", "MOSTLY_IQ3_S", "MOSTLY_IQ3_M",
                     "MOSTLY_IQ4_XS"):
            return GT.Q5_K
        return t
    by_ft = {_ft("MOSTLY_Q2_K"): GT.Q3_K, _ft("MOSTLY_IQ3_XXS"): GT.IQ3_S, _ft("MOSTLY_Q3_K_M"): GT.Q4_K,
             _ft("MOSTLY_Q3_K_L"): GT.Q5_K, _ft("MOSTLY_IQ3_M"): GT.Q4_K}
    return by_ft.get(f, t)


def _rule_attn_qkv(c: _Ctx, t: GT) -> GT:
    f = c.ftype
    if f in _fts("MOSTLY_Q3_K_M", "MOSTLY_Q3_K_L", "MOSTLY_IQ3_M"):
        return GT.Q4_K
    if f == _ft("MOSTLY_Q4_K_M"):
        return GT.Q5_K
    if f == _ft("MOSTLY_Q5_K_M"):
        return GT.Q6_K
    return t


def _rule_ffn_gate_up(c: _Ctx, t: GT, counter: str, total: str) -> GT:
    qs = c.qs
    i, n = _layer_of(getattr(qs, counter), getattr(qs, total), c.name, max(1, c.model.n_expert))
    if c.ftype == _ft("MOSTLY_IQ3_XS") and n // 8 <= i < 7 * n // 8:
        t = GT.IQ3_XXS
    setattr(qs, counter, getattr(qs, counter) + 1)
    return t


def _mixture(c: _Ctx, t: GT) -> GT:
    """llama_tensor_get_type_impl: the first applicable rule decides."""
    cat, f = c.cat, c.ftype
    if cat == Category.OUTPUT or (c.qs.has_tied_embeddings and cat == Category.TOKEN_EMBD):
        return _rule_output_or_tied_embd(c, t)
    if f == _ft("MOSTLY_MXFP4_MOE"):  # MoE tensors -> MXFP4, the rest -> Q8_0
        return GT.MXFP4 if len(c.ne) > 2 and c.ne[2] > 1 else GT.Q8_0
    if cat == Category.TOKEN_EMBD:
        return _rule_token_embd(c, t)
    if f in _IQ_LOW:
        return _rule_low_bit_iq(c, t)
    if category_is_attn_v(cat):
        return _rule_attn_v(c, t)
    rules = {
        Category.ATTENTION_K: _rule_attn_k,
        Category.ATTENTION_Q: _rule_attn_q,
        Category.FFN_DOWN: _rule_ffn_down,
        Category.ATTENTION_OUTPUT: _rule_attn_output,
        Category.ATTENTION_QKV: _rule_attn_qkv,
        Category.FFN_GATE: lambda cc, tt: _rule_ffn_gate_up(cc, tt, "i_ffn_gate", "n_ffn_gate"),
        Category.FFN_UP: lambda cc, tt: _rule_ffn_gate_up(cc, tt, "i_ffn_up", "n_ffn_up"),
    }
    rule = rules.get(cat)
    return rule(c, t) if rule else t


def tensor_get_type(qs: QuantState, model: ModelInfo, name: str, ne: tuple[int, ...],
                    src_type: GT, ftype: FT, pure: bool = False,
                    quantize_output_tensor: bool = True, only_copy: bool = False,
                    token_embedding_type: GT | None = None,
                    output_tensor_type: GT | None = None) -> GT:
    """Target type of one tensor (ne = ggml shape, ne[0] = row length); src_type means
    passthrough. Call in weight_name_key order: the counters in qs advance."""
    n_dims = max([i + 1 for i, d in enumerate(ne) if d > 1], default=1)
    if not tensor_allows_quantization(name, n_dims, quantize_output_tensor, only_copy):
        return src_type
    cat = tensor_get_category(name)
    if token_embedding_type is not None and cat == Category.TOKEN_EMBD:
        return token_embedding_type
    if output_tensor_type is not None and cat == Category.OUTPUT:
        return output_tensor_type
    t = ftype_default_type(ftype)
    if t is None:
        raise ValueError(f"no default tensor type for ftype {ftype!r}")
    if not ggml_is_quantized(t):
        return t
    override = next((ot for pat, ot in qs.tensor_type_patterns if pat.search(name)), None)
    if override is not None:
        t = override
    elif not pure:
        t = _mixture(_Ctx(qs, model, ftype, name, tuple(ne), cat, token_embedding_type, output_tensor_type), t)
    return tensor_type_fallback(qs, name, ne[0], t)


_NEEDS_IMATRIX = {_gt(n) for n in ("IQ3_XXS", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ1_M", "IQ1_S")}


def tensor_requires_imatrix(name: str, dst_type: GT, ftype: FT) -> bool:
    if name in _TOKEN_EMBD_NAMES or name == "output.weight":
        return False
    if dst_type in _NEEDS_IMATRIX:
        return True
    return dst_type == GT.Q2_K and ftype == _ft("MOSTLY_Q2_K_S")


def decide_types(model: ModelInfo, tensors: list[tuple[str, tuple[int, ...], GT]], ftype: FT,
                 has_imatrix: bool = False, pure: bool = False,
                 token_embedding_type: GT | None = None,
                 output_tensor_type: GT | None = None,
                 tt_overrides: list[tuple[str, GT]] | None = None) -> list[GT]:
    """Plan a whole model: count over all names first, then choose per tensor in order."""
    qs = init_state(model, [t[0] for t in tensors], has_imatrix, tt_overrides)
    return [tensor_get_type(qs, model, n, ne, src, ftype, pure=pure,
                            token_embedding_type=token_embedding_type,
                            output_tensor_type=output_tensor_type) for n, ne, src in tensors]


def format_scheme_table() -> str:
    lines = [f"quantization schemes (llama.cpp {LLAMA_CPP_COMMIT[:10]}), [x] = has a qs-b200 kernel"]
    for o in QUANT_OPTIONS:
        dt = o.default_type
        lines.append(f"  [{'x' if o.supported else ' '}] {o.name:10s} default "
                     f"{dt.name if dt is not None else '-':8s} {o.desc}")
    return "\n".join(lines)


if __name__ == "__main__":
    print(format_scheme_table())
