"""Pins of the constants the GPU block decode derives its IQ values from (CPU only).

qs_dequant.cu decodes an IQ grid index through the type's lattice codebook (the same
code list the quantizers search, quant-studio_b200/csrc/iq_grids.h) and a per-type
level -> value map, and rebuilds the ksigns table as i | parity(i) << 7. These tests
restate those maps and check them entry for entry against gguf-py's own tables
(gguf/quants.py IQ*.grid after init_grid, IQ2_XXS.ksigns), which define the formats.
"""

import re

import numpy as np
import pytest

from conftest import PKG

gguf = pytest.importorskip("gguf")
import gguf.quants as Q  # noqa: E402

GRIDS = PKG / "csrc" / "iq_grids.h"
# (gguf class, codebook, bits per level, positions, level -> value map of qs_dequant.cu)
CASES = [
    (Q.IQ2_XXS, "KGRID_2BIT_256", 2, 8, (8, 25, 43)),
    (Q.IQ2_XS, "KGRID_2BIT_512", 2, 8, (8, 25, 43)),
    (Q.IQ2_S, "KGRID_2BIT_1024", 2, 8, (8, 25, 43)),
    (Q.IQ3_XXS, "KGRID_3BIT_256", 3, 4, (4, 12, 20, 28, 36, 44, 52, 62)),
    (Q.IQ3_S, "KGRID_3BIT_512", 3, 4, (1, 3, 5, 7, 9, 11, 13, 15)),
]


def _codebook(name: str) -> np.ndarray:
    m = re.search(name + r"\[\d+\] = \{([^}]*)\}", GRIDS.read_text())
    return np.array([int(v, 0) for v in m.group(1).replace("\n", " ").split(",") if v.strip()])


@pytest.mark.parametrize("cls,name,bits,npos,vmap", CASES, ids=[c[1] for c in CASES])
def test_dequant_grid_from_codebook(cls, name, bits, npos, vmap):
    cls.init_grid()
    want = cls.grid.reshape(cls.grid_shape)
    codes = _codebook(name)
    levels = np.stack([(codes >> (bits * j)) & ((1 << bits) - 1) for j in range(npos)], 1)
    assert levels.max() < len(vmap)
    assert np.array_equal(np.asarray(vmap, dtype=np.float32)[levels], want)


def test_ksigns_is_parity_completed():
    want = np.frombuffer(Q.IQ2_XXS.ksigns, dtype=np.uint8)
    mine = np.array([i | ((bin(i).count("1") & 1) << 7) for i in range(128)], dtype=np.uint8)
    assert np.array_equal(mine, want)


def test_iq4_kvalues():
    src = (PKG / "csrc" / "qs_dequant.cu").read_text()
    m = re.search(r"c_kvalues\[16\] = \{([^}]*)\}", src)
    assert tuple(int(v) for v in m.group(1).split(",")) == Q.IQ4_NL.kvalues
