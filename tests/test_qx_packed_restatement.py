"""make_qx_quants with the GPU's packed candidate loop, checked against the sequential search (CPU).

make_qx_quants (kernels/qx_common.py:52-82; the oracle's make_qx in oracle/qs_oracle.c) scores
18 candidate scales per group with left-to-right sums of (w x) l and (w l) l. The CUDA loop
(`qx_search` in quant-studio_b200/csrc/qs_kquant.cuh) computes the levels with the rounding add
pair and a NaN-propagating clamp, and every product as fma(a, b, +0), so a zero level or a zero
product may come out +0 where the reference's is -0. The argument that this never changes a
result: sl2 <= 0 is rejected whatever its sign; a zero slx passes the accept test only when
best < 0, which takes negative weights, and then the reference's zero is +0 too (the kernel
keeps a re-sum there as a guard); the accepted levels are rebuilt from the winning scale.

This file restates both in float32 numpy, vectorised over groups, and checks the scale and the
levels bit for bit on adversarial groups: the benchmark distribution, all-negative and
all-positive groups, zeros, constants, few distinct values, huge and tiny magnitudes, zero,
negative and subnormal weights, NaN / inf entries, and groups built so that a zero slx meets
best < 0 (with the largest value positive and negative).
"""

import numpy as np
import pytest

f32 = np.float32
MAGIC = f32(12582912.0)


def _seq(t):  # t[:, 0] + t[:, 1] + ... left to right
    s = t[:, 0].copy()
    for i in range(1, t.shape[1]):
        s = (s + t[:, i]).astype(np.float32)
    return s


def _clampf(v, lo, hi):  # x < lo ? lo : (x > hi ? hi : x)
    return np.where(v < lo, lo, np.where(v > hi, hi, v)).astype(np.float32)


def _absmax_first(x):
    a, m = np.abs(x[:, 0]), x[:, 0].copy()
    for i in range(1, x.shape[1]):
        v = np.abs(x[:, i])
        c = v > a
        a, m = np.where(c, v, a), np.where(c, x[:, i], m)
    return a.astype(np.float32), m.astype(np.float32)


def qx_steps(nmax):  # c = nmax + 0.1 s (s = -9..9, s != 0), folded in float32
    return [f32(f32(nmax) + f32(f32(0.1) * f32(s))) for s in range(-9, 10) if s]


def _head(x, w, nmax):
    fmax = f32(nmax)
    amax, mx = _absmax_first(x)
    live = amax >= f32(1e-15)
    r = (f32(1) / np.where(live, mx, f32(1))).astype(np.float32)
    wx = (w * x).astype(np.float32)
    iscale = (r * -fmax).astype(np.float32)
    L = _clampf(np.rint(iscale[:, None] * x), -fmax, fmax - 1)
    sumlx = _seq(wx * L)
    suml2 = _seq((w * L) * L)
    scale = np.where(suml2 != 0, sumlx / np.where(suml2 != 0, suml2, f32(1)), f32(0)).astype(np.float32)
    best = (scale * sumlx).astype(np.float32)
    return fmax, live, r, wx, iscale, scale, best


def qx_reference(x, w, nmax):
    """The sequential search (oracle make_qx): exact levels, scalar products, levels copied on accept."""
    fmax, live, r, wx, iscale, scale, best = _head(x, w, nmax)
    L = _clampf(np.rint(iscale[:, None] * x), -fmax, fmax - 1)
    for c in qx_steps(nmax):
        isc = (r * -c).astype(np.float32)
        la = _clampf(np.rint(isc[:, None] * x), -fmax, fmax - 1)
        slx, sl2 = _seq(wx * la), _seq((w * la) * la)
        acc = (sl2 > 0) & (slx * slx > best * sl2)
        cand = (slx / np.where(acc, sl2, f32(1))).astype(np.float32)
        scale = np.where(acc, cand, scale)
        best = np.where(acc, cand * slx, best).astype(np.float32)
        L = np.where(acc[:, None], la, L)
    return np.where(live, scale, f32(0)).astype(np.float32), np.where(live[:, None], L + fmax, f32(0)).astype(np.float32)


def qx_gpu(x, w, nmax):
    """The CUDA loop: rounding-add levels, NaN-propagating clamp, products with -0 -> +0, pairs
    summed left to right, the re-sum branch for a zero slx, levels rebuilt from the winner."""
    fmax, live, r, wx, iscale, scale, best = _head(x, w, nmax)
    win = iscale.copy()
    z = f32(0)
    for c in qx_steps(nmax):
        isc = (r * -c).astype(np.float32)
        al = (isc[:, None] * x) + z                               # fma(isc, x, +0)
        lv = ((al + MAGIC).astype(np.float32) - MAGIC).astype(np.float32)
        la = np.minimum(np.maximum(lv, -fmax), fmax - 1).astype(np.float32)   # max.NaN, min.NaN
        a = (wx * la) + z
        b = (((w * la) + z) * la) + z
        slx, sl2 = _seq(a.astype(np.float32)), _seq(b.astype(np.float32))
        acc = (sl2 > 0) & (slx * slx > best * sl2)
        redo = acc & (slx == 0)
        if redo.any():
            exact = _seq(wx * _clampf(np.rint(isc[:, None] * x), -fmax, fmax - 1))
            slx = np.where(redo, exact, slx)
        cand = (slx / np.where(acc, sl2, f32(1))).astype(np.float32)
        scale = np.where(acc, cand, scale)
        best = np.where(acc, cand * slx, best).astype(np.float32)
        win = np.where(acc, isc, win)
    L = _clampf(np.rint(win[:, None] * x), -fmax, fmax - 1) + fmax
    return np.where(live, scale, f32(0)).astype(np.float32), np.where(live[:, None], L, f32(0)).astype(np.float32)


def _groups(rng, g, n):
    x = rng.normal(0.0, 0.02, (g, n))
    out = rng.random(x.shape) < 0.01
    x[out] = rng.normal(0.0, 0.5, int(out.sum()))
    w = rng.lognormal(0.0, 1.5, (g, n))
    k = g // 14
    x[0 * k:1 * k] = -np.abs(x[0 * k:1 * k])
    x[1 * k:2 * k] = np.abs(x[1 * k:2 * k])
    x[2 * k:3 * k][rng.random((k, n)) < 0.5] = 0.0
    x[3 * k:4 * k] = 0.013
    x[4 * k:5 * k] = rng.integers(-2, 3, (k, n)) * 0.01
    x[5 * k:6 * k] *= 1e30
    x[6 * k:7 * k] *= 1e-30
    w[7 * k:8 * k][rng.random((k, n)) < 0.5] = 0.0
    w[8 * k:9 * k] *= np.where(rng.random((k, n)) < 0.4, -1.0, 1.0)      # negative weights
    w[9 * k:10 * k][rng.random((k, n)) < 0.5] = 1e-44                     # subnormal weights
    x[10 * k:11 * k, 3] = np.nan
    x[11 * k:12 * k, 5] = np.inf
    x[12 * k:13 * k, 7] = -np.inf
    # a zero slx against best < 0: the largest value carries no weight, a small value with a
    # negative weight makes suml2 < 0 at the first guess, and a value whose w x underflows
    # while w l does not keeps sl2 > 0 at the steps where the small value's level drops to 0
    for j in range(13 * k, 14 * k):
        x[j] = 0.0
        w[j] = 0.0
        sg = 1.0 if j % 2 else -1.0
        x[j, 0], w[j, 0] = sg, 0.0
        x[j, 1], w[j, 1] = -sg * rng.uniform(0.0150, 0.0160), -1e6
        x[j, 2], w[j, 2] = rng.uniform(0.02, 0.05), 1e-44
        x[j, 3], w[j, 3] = rng.uniform(0.003, 0.01), rng.uniform(0.5, 2.0)
    return x.astype(np.float32), w.astype(np.float32)


@pytest.mark.parametrize("nmax", [32, 4])
def test_packed_qx_search_equals_sequential(nmax):
    rng = np.random.default_rng(41 + nmax)
    x, w = _groups(rng, 2800, 16)
    with np.errstate(all="ignore"):
        s_ref, l_ref = qx_reference(x, w, nmax)
        s_gpu, l_gpu = qx_gpu(x, w, nmax)
    same_s = (s_ref.view(np.uint32) == s_gpu.view(np.uint32)) | (np.isnan(s_ref) & np.isnan(s_gpu))
    assert same_s.all(), f"scale differs in groups {np.nonzero(~same_s)[0][:8]}"
    assert np.array_equal(l_ref, l_gpu, equal_nan=True)


def test_an_accepted_zero_slx_is_plus_zero_in_the_reference():
    """Where a zero slx passes the accept test (best < 0), the reference's sum is +0, so the
    packed loop's +0 already equals it: the kernel's re-sum is a guard, not a fix."""
    rng = np.random.default_rng(7)
    x, w = _groups(rng, 2800, 16)
    seen = 0
    with np.errstate(all="ignore"):
        for nmax in (32, 4):
            fmax, live, r, wx, iscale, scale, best = _head(x, w, nmax)
            for c in qx_steps(nmax):
                isc = (r * -c).astype(np.float32)
                la = _clampf(np.rint(isc[:, None] * x), -fmax, fmax - 1)
                slx, sl2 = _seq(wx * la), _seq((w * la) * la)
                acc = (sl2 > 0) & (slx * slx > best * sl2)
                z = acc & (slx == 0)
                seen += int(z.sum())
                assert not np.signbit(slx[z]).any()
                cand = (slx / np.where(acc, sl2, f32(1))).astype(np.float32)
                best = np.where(acc, cand * slx, best).astype(np.float32)
    assert seen > 0, "the constructed groups should reach an accepted zero slx"
