"""The synthetic-model writer (quant-studio_b200/synth_model.py), CPU only: layout, dtypes,
metadata and the imatrix, on the tiny configuration; the CLI plans it like a real model."""

import subprocess
import sys

import numpy as np
from gguf import GGMLQuantizationType as GT, GGUFReader

from conftest import PKG

sys.path.insert(0, str(PKG))
import synth_model  # noqa: E402


def test_tiny_model_layout_and_values(tmp_path):
    path, imat = tmp_path / "m.gguf", tmp_path / "m.imatrix.gguf"
    cols = synth_model.write_model(path, "tiny", seed=3)
    synth_model.write_imatrix(imat, cols)
    r = GGUFReader(path)
    names = [t.name for t in r.tensors]
    want = [n for n, _, _ in synth_model.tensor_list(synth_model.MODELS["tiny"])]
    assert names == want
    for t, (_, shape, is_w) in zip(r.tensors, synth_model.tensor_list(synth_model.MODELS["tiny"])):
        assert tuple(int(d) for d in reversed(t.shape)) == shape
        assert t.tensor_type == (GT.BF16 if is_w else GT.F32)
        if is_w:
            v = (np.asarray(t.data).reshape(-1).view(np.uint16).astype(np.uint32) << 16).view(np.float32)
            assert 0.015 < float(np.std(v[np.abs(v) < 0.1])) < 0.025
            assert 0.0003 < float(np.mean(np.abs(v) > 0.15)) < 0.003   # the outliers
        else:
            assert np.all(np.asarray(t.data) == 1.0)
    fields = {f.name: f for f in r.fields.values()}
    assert int(fields["llama.block_count"].parts[-1][0]) == 2
    assert int(fields["llama.attention.head_count_kv"].parts[-1][0]) == 2
    ri = {t.name: np.asarray(t.data) for t in GGUFReader(imat).tensors}
    assert set(ri) == {n + s for n in cols for s in (".in_sum2", ".counts")}
    assert all(ri[n + ".in_sum2"].size == k and np.all(ri[n + ".in_sum2"] > 0) for n, k in cols.items())


def test_cli_plans_the_tiny_model(tmp_path):
    path = tmp_path / "m.gguf"
    synth_model.write_model(path, "tiny", seed=3)
    out = subprocess.run([sys.executable, str(PKG / "quant-studio.py"), str(path), str(tmp_path / "o.gguf"),
                          "Q4_K_M", "--dry-run"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "blk.1.ffn_down.weight" in out.stdout and "Q6_K" in out.stdout and "dry run:" in out.stdout
