"""IQ4_XS's scale search with the GPU's lookup and packed sweep, checked against the reference (CPU).

The reference (kernels/iq4_xs.py:35-76, the oracle's iq4_search) projects every value onto the
16 non-linear levels with a bracket search and a float midpoint compare, then scores 15 scales
with left-to-right sums of (w q) x and (w q) q. The CUDA kernel (iq4xs_kernel in
quant-studio_b200/csrc/qs_kquant.cu) takes the bracket from a table indexed by the value's floor
and computes the sweep's products as fma(a, b, +0) on f32x2 pairs, so a zero product may come out
+0 where the reference's is -0. The argument: best >= 0 throughout (sumqx^2 / sumq2 with
sumq2 > 0, or a signed zero), so a step is accepted only with sumqx != 0 and sumq2 > 0, whose
values the sign of a zero term does not change.

This file restates both in float32 numpy and checks the returned scale bit for bit on
adversarial groups: the benchmark distribution, zeros, constants, ties on the level midpoints,
huge and tiny magnitudes, zero, negative and subnormal weights, NaN and inf entries.
"""

import numpy as np
import pytest

f32 = np.float32
KV = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)


def _seq(t):
    s = t[:, 0].copy()
    for i in range(1, t.shape[1]):
        s = (s + t[:, i]).astype(np.float32)
    return s


def level_search(al):
    """best_index_int8 -> level: count kv <= al, clamp to 1..15, the float midpoint compare."""
    mu = (KV[None, None, :] <= al[..., None]).sum(-1).clip(1, 15)
    lo, hi = KV[mu - 1], KV[mu]
    return np.where((al - lo) < (hi - al), lo, hi).astype(np.float32)


_T = np.arange(271, dtype=np.float32) - 136
_P = (KV[None, 1:15] <= _T[:, None]).sum(1)
_LO, _HI = KV[_P], KV[_P + 1]


def level_table(al):
    """iq4_tab_level: floor(clamp(al, -136, 134.5)) by the rounding-down add, then the compare."""
    y = np.minimum(np.maximum(al, f32(-136)), f32(134.5))
    y = np.where(np.isnan(al), f32(-136), y)
    e = (np.floor(y.astype(np.float64) + 12583048.0).astype(np.int64) - 12582912) & 0x1FF
    lo, hi = _LO[e], _HI[e]
    return np.where((al - lo) < (hi - al), lo, hi).astype(np.float32)


def _absmax_first(x):
    a, m = np.abs(x[:, 0]), x[:, 0].copy()
    for i in range(1, x.shape[1]):
        v = np.abs(x[:, i])
        c = v > a
        a, m = np.where(c, v, a), np.where(c, x[:, i], m)
    return m.astype(np.float32)


def iq4_search(x, w, gpu):
    mx = _absmax_first(x)
    live = np.abs(mx) >= f32(1e-15)
    mxs = np.where(live, mx, f32(1)).astype(np.float32)
    d0 = (-mxs / f32(-127)).astype(np.float32)
    id0 = (f32(1) / d0).astype(np.float32)
    lev = level_table if gpu else level_search
    q = lev((id0[:, None] * x).astype(np.float32))
    sumqx, sumq2 = _seq((w * q) * x), _seq((w * q) * q)     # the first guess is scalar in both
    d = np.where(sumq2 > 0, sumqx / np.where(sumq2 > 0, sumq2, f32(1)), f32(0)).astype(np.float32)
    best = (d * sumqx).astype(np.float32)
    r = (f32(1) / mxs).astype(np.float32)
    z = f32(0)
    for itry in range(-7, 8):
        idv = (r * f32(itry - 127)).astype(np.float32)
        if gpu:
            q = lev(((idv[:, None] * x) + z).astype(np.float32))
            wq = ((w * q) + z).astype(np.float32)
            sx, s2 = _seq(((wq * x) + z).astype(np.float32)), _seq(((wq * q) + z).astype(np.float32))
        else:
            q = lev((idv[:, None] * x).astype(np.float32))
            sx, s2 = _seq((w * q) * x), _seq((w * q) * q)
        acc = (s2 > 0) & (sx * sx > best * s2)
        nd = (sx / np.where(acc, s2, f32(1))).astype(np.float32)
        d = np.where(acc, nd, d)
        best = np.where(acc, nd * sx, best).astype(np.float32)
    return np.where(live, d, f32(0)).astype(np.float32)


def _groups(rng, g):
    x = rng.normal(0.0, 0.02, (g, 32))
    out = rng.random(x.shape) < 0.01
    x[out] = rng.normal(0.0, 0.5, int(out.sum()))
    w = (rng.lognormal(0.0, 1.5, (g, 32)) * np.sqrt(0.0008 + x * x))
    k = g // 12
    x[0 * k:1 * k][rng.random((k, 32)) < 0.5] = 0.0
    x[1 * k:2 * k] = 0.013
    # values on the level midpoints of the first guess's scale (mx = 1: al = 127 x)
    mids = ((KV[:-1] + KV[1:]) / 2 / 127.0).astype(np.float32)
    x[2 * k:3 * k] = rng.choice(mids, (k, 32))
    x[2 * k:3 * k, 0] = 1.0
    x[3 * k:4 * k] *= 1e30
    x[4 * k:5 * k] *= 1e-30
    w[5 * k:6 * k][rng.random((k, 32)) < 0.5] = 0.0
    w[6 * k:7 * k] *= np.where(rng.random((k, 32)) < 0.4, -1.0, 1.0)
    w[7 * k:8 * k][rng.random((k, 32)) < 0.5] = 1e-44
    x[8 * k:9 * k, 3] = np.nan
    x[9 * k:10 * k, 5] = np.inf
    x[10 * k:11 * k, 0] = np.nan                       # the first value NaN: the group is not live
    x[11 * k:12 * k, 7] = -np.inf
    return x.astype(np.float32), w.astype(np.float32)


def test_table_lookup_and_packed_sweep_equal_the_reference():
    rng = np.random.default_rng(23)
    x, w = _groups(rng, 4800)
    with np.errstate(all="ignore"):
        ref, gpu = iq4_search(x, w, False), iq4_search(x, w, True)
    same = (ref.view(np.uint32) == gpu.view(np.uint32)) | (np.isnan(ref) & np.isnan(gpu))
    assert same.all(), f"scale differs in groups {np.nonzero(~same)[0][:8]}"


@pytest.mark.parametrize("scale", [1.0, 1e-3, 1e20])
def test_lookup_matches_on_every_sweep_value(scale):
    """The lookup equals the search on every value the sweep forms, not only in the result."""
    rng = np.random.default_rng(5)
    x = (rng.normal(0, 0.02, (256, 32)) * scale).astype(np.float32)
    mx = _absmax_first(x)
    r = (f32(1) / mx).astype(np.float32)
    for itry in range(-7, 8):
        al = ((r * f32(itry - 127))[:, None] * x).astype(np.float32)
        assert np.array_equal(level_table(al), level_search(al))
