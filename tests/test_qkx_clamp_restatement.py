"""The k-quant group search with the GPU's level clamp, checked against the sequential search (CPU).

make_qkx_quants (kernels/kq_common.py:51-96) clamps every candidate level with
`clamp(round(isc * (x - min)), 0, nmax)`. In the CUDA search loop (`qkx_search` in
quant-studio_b200/csrc/qs_kquant.cuh) that clamp is a NaN-propagating max then min
(`clamp_nan`), which equals the compare-and-select clamp for every non-NaN level and gives
NaN for a NaN level, except that a -0 level may come out +0. The argument that this never
changes a block: a NaN level makes the step's sums NaN, so the step is rejected either way;
a -0 level only changes a level sum whose terms are all zero, and then D <= 0 rejects the
step. The final levels are rebuilt with the exact clamp.

This file restates the search in float32 numpy, vectorised over groups, with the GPU's clamp
and every -0 level forced to +0 (the worst case; about 1 % of the levels here are -0), and
checks scale, min and levels bit for bit against the oracle's sequential make_qkx on
adversarial groups: the benchmark distribution, all-negative and all-positive groups, zeros,
constants, a few distinct values, huge and tiny magnitudes, zero weights, and NaN / inf
entries. (In a group with a NaN or infinite entry the first guess's error is already NaN, so
no step is accepted with either clamp; those groups check that path, not the NaN argument.)
"""

import ctypes

import numpy as np
import pytest

import oracle

f32 = np.float32
TINY = f32(1.17549435e-38)


def _tree(v):  # adjacent-pair tree over the last axis (32 or 16 values)
    while v.shape[-1] > 1:
        v = v[..., 0::2] + v[..., 1::2]
    return v[..., 0]


def _clampf(v, hi):  # x < lo ? lo : (x > hi ? hi : x), lo = 0
    return np.where(v < 0, f32(0), np.where(v > hi, hi, v)).astype(np.float32)


def _clamp_gpu(v, hi):  # max.NaN then min.NaN, with -0 forced to +0
    r = np.minimum(np.maximum(v, f32(0)), hi)  # numpy max/min propagate NaN
    return (r + f32(0)).astype(np.float32)     # -0 + 0 = +0


def _seq_extreme(x, less):
    m = x[:, 0].copy()
    for i in range(1, x.shape[1]):
        c = x[:, i] < m if less else x[:, i] > m
        m = np.where(c, x[:, i], m)
    return m


def qkx_gpu(x, w, nmax, steps):
    """The GPU search on (G, n) float32 groups: returns (scale, the_min, levels)."""
    fmax = f32(nmax)
    mn = _seq_extreme(x, True)
    mn = np.where(mn > 0, f32(0), mn).astype(np.float32)
    mx = _seq_extreme(x, False)
    degen = mx == mn
    sum_w = _tree(w)
    sum_x = _tree(w * x)
    den = np.where(degen, f32(1), mx - mn).astype(np.float32)
    iscale = (fmax / den).astype(np.float32)
    scale = (f32(1) / iscale).astype(np.float32)
    la = _clamp_gpu(np.rint(iscale[:, None] * (x - mn[:, None])), fmax)
    d = (scale[:, None] * la + mn[:, None]) - x
    best = _tree(w * (d * d))
    win_isc, win_mn = iscale.copy(), mn.copy()
    for c in steps:
        den = np.where(degen, f32(1), mx - mn).astype(np.float32)
        isc = (f32(c) / den).astype(np.float32)
        la = _clamp_gpu(np.rint(isc[:, None] * (x - mn[:, None])), fmax)
        wl = w * la
        sum_l, sum_l2, sum_xl = _tree(wl), _tree(wl * la), _tree(wl * x)
        D = sum_w * sum_l2 - sum_l * sum_l
        Ds = np.where(D > 0, D, f32(1)).astype(np.float32)
        ts = ((sum_w * sum_xl - sum_x * sum_l) / Ds).astype(np.float32)
        tm = ((sum_l2 * sum_x - sum_l * sum_xl) / Ds).astype(np.float32)
        pos = tm > 0
        ts = np.where(pos, sum_xl / np.where(sum_l2 < TINY, TINY, sum_l2), ts).astype(np.float32)
        tm = np.where(pos, f32(0), tm).astype(np.float32)
        d = (ts[:, None] * la + tm[:, None]) - x
        cur = _tree(w * (d * d))
        acc = (D > 0) & (cur < best) & ~degen
        win_isc = np.where(acc, isc, win_isc)
        win_mn = np.where(acc, mn, win_mn)
        scale = np.where(acc, ts, scale)
        mn = np.where(acc, tm, mn)
        best = np.where(acc, cur, best)
    levels = _clampf(np.rint(win_isc[:, None] * (x - win_mn[:, None])), fmax)
    levels = np.where(degen[:, None], f32(0), levels)
    the_min = np.where(mn == 0, f32(0), -mn).astype(np.float32)
    return np.where(degen, f32(0), scale).astype(np.float32), the_min, levels.astype(np.float32)


def _groups(rng, g, n):
    x = rng.normal(0.0, 0.02, (g, n))
    out = rng.random(x.shape) < 0.01
    x[out] = rng.normal(0.0, 0.5, int(out.sum()))
    w = rng.lognormal(0.0, 1.5, (g, n)) * (0.02 + np.abs(x))
    k = g // 12
    x[0 * k:1 * k] = -np.abs(x[0 * k:1 * k])                      # all negative
    x[1 * k:2 * k] = np.abs(x[1 * k:2 * k])                       # all positive
    x[2 * k:3 * k][rng.random((k, n)) < 0.5] = 0.0                # zeros
    x[3 * k:4 * k] = 0.013                                        # constant
    x[4 * k:5 * k] = rng.integers(-2, 3, (k, n)) * 0.01           # few distinct values, ties
    x[5 * k:6 * k] *= 1e30                                        # huge
    x[6 * k:7 * k] *= 1e-30                                       # tiny
    w[7 * k:8 * k][rng.random((k, n)) < 0.5] = 0.0                # zero weights
    x[8 * k:9 * k, 3] = np.nan                                    # NaN entries
    x[9 * k:10 * k, 5] = np.inf                                   # inf entries
    x[10 * k:11 * k, 7] = -np.inf
    x[11 * k:12 * k, 0] = 0.0                                     # a single zero in front
    return x.astype(np.float32), w.astype(np.float32)


def _steps(nmax):  # imatrix candidate numerators, kernels/kq_common.py:21-24, folded in float32
    return [f32(f32(f32(-0.9) + f32(f32(0.05) * f32(s))) + f32(nmax)) for s in range(37)]


@pytest.mark.parametrize("n, nmax", [(32, 15), (32, 31), (16, 3)])
def test_gpu_clamp_search_equals_sequential(n, nmax):
    L = oracle.lib()
    L.oq_core_qkx.restype = ctypes.c_float
    L.oq_core_qkx.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    rng = np.random.default_rng(17 + n + nmax)
    x, w = _groups(rng, 1200, n)
    with np.errstate(all="ignore"):
        scale, the_min, levels = qkx_gpu(x, w, nmax, _steps(nmax))
    for gi in range(x.shape[0]):
        xg, wg = np.ascontiguousarray(x[gi]), np.ascontiguousarray(w[gi])
        lv = np.zeros(n, np.float32)
        mn = np.zeros(1, np.float32)
        s = np.float32(L.oq_core_qkx(xg.ctypes.data, wg.ctypes.data, n, nmax, 1, 0, mn.ctypes.data, lv.ctypes.data))
        assert np.array_equal(np.float32(scale[gi]).view(np.uint32), s.view(np.uint32)) or (np.isnan(s) and np.isnan(scale[gi])), gi
        assert np.array_equal(the_min[gi:gi + 1].view(np.uint32), mn.view(np.uint32)) or (np.isnan(mn[0]) and np.isnan(the_min[gi])), gi
        assert np.array_equal(levels[gi], lv, equal_nan=True), gi
