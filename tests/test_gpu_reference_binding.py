"""The reference-side binding of INTEGRATION.md, run inside the reference's own CLI (GPU).

The ctypes stub that INTEGRATION.md shows a maintainer adding to quant-studio
(kernels/qsb200.py plus three lines in kernels/__init__.py) is taken from the document
itself, installed into a scratch copy of the unmodified reference (baseline/_ref), and the
reference's quant-studio.py then quantizes a small model on the GPU through its own
CudaPipeline (quant-studio.py:148-213) with libqsb200 underneath. Every tensor it writes must
hold the same type and bytes as the one qs-b200's own CLI writes for the same model.
Skipped when the reference copy is absent.
"""

import os
import re
import shutil
import subprocess
import sys

import numpy as np
import pytest
from gguf import GGUFReader

from conftest import PKG, ROOT
from synth_gguf import write_imatrix, write_llama

pytestmark = pytest.mark.gpu

REF = ROOT / "baseline" / "_ref" / "quant-studio"
LIB = PKG / "lib" / "libqsb200.so"

# pip gguf 0.19 lacks two enum members the reference's policy module names; added at start-up
SHIM = '''
from gguf import GGMLQuantizationType as GT
from gguf.constants import LlamaFileType as FT
def _add(cls, name, value):
    if hasattr(cls, name):
        return
    m = int.__new__(cls, value)
    m._name_, m._value_ = name, value
    type.__setattr__(cls, name, m)
    cls._member_map_[name] = m
    cls._value2member_map_[value] = m
    cls._member_names_.append(name)
_add(FT, "MOSTLY_Q2_0", 1000)
_add(GT, "Q2_0", 1000)
'''


def install_binding(dst) -> None:
    """Copy the reference and add INTEGRATION.md's stub to its kernels package, as written."""
    shutil.copytree(REF, dst)
    doc = (ROOT / "INTEGRATION.md").read_text()
    code = re.search(r"```python\n(# kernels/qsb200.py.*?)```", doc, re.S).group(1)
    code = code.replace("/path/to/quant-studio_b200/lib/libqsb200.so", str(LIB))
    (dst / "kernels" / "qsb200.py").write_text(code)
    wiring = [ln[4:].rstrip() for ln in code.splitlines() if ln.startswith("#   ")]
    assert wiring, "INTEGRATION.md lost its kernels/__init__.py lines"
    with open(dst / "kernels" / "__init__.py", "a") as f:
        f.write("\n" + "\n".join(wiring) + "\n")


def tensors(path):
    return {t.name: (t.tensor_type, np.asarray(t.data).reshape(-1).view(np.uint8)) for t in GGUFReader(path).tensors}


@pytest.mark.skipif(not REF.exists(), reason="no copy of the reference in baseline/_ref")
@pytest.mark.parametrize("scheme", ["Q4_K_M", "IQ3_XXS", "Q4_0"])
def test_reference_cli_with_the_binding_writes_our_bytes(tmp_path, scheme):
    ref = tmp_path / "ref"
    install_binding(ref)
    (tmp_path / "shim").mkdir()
    (tmp_path / "shim" / "sitecustomize.py").write_text(SHIM)
    src, im = tmp_path / "in.gguf", tmp_path / "im.gguf"
    vals = write_llama(src, n_layer=2)
    write_imatrix(im, {k: v.shape[1] for k, v in vals.items()})
    extra = [] if scheme == "Q4_0" else ["--imatrix", str(im)]
    env = dict(os.environ, PYTHONPATH=str(tmp_path / "shim"), PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, str(ref / "quant-studio.py"), str(src), str(tmp_path / "ref.gguf"), scheme,
                        "--device", "cuda", "--mem", "256K", *extra], capture_output=True, text=True, env=env, cwd=ref)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run([sys.executable, str(PKG / "quant-studio.py"), str(src), str(tmp_path / "ours.gguf"), scheme,
                        "--mem", "256K", *extra], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    a, b = tensors(tmp_path / "ref.gguf"), tensors(tmp_path / "ours.gguf")
    assert set(a) == set(b)
    quantized = 0
    for name, (ta, da) in a.items():
        tb, db = b[name]
        assert ta == tb, name
        assert np.array_equal(da, db), f"{name} ({ta.name})"
        quantized += ta.name not in ("F32", "F16", "BF16")
    assert quantized >= 10
