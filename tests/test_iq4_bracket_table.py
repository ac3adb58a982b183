"""The IQ4_XS scale search's level lookup, restated in float32 numpy (CPU).

The kernel (iq4_tab_level in csrc/qs_kquant.cu) replaces the reference's bracket search
(kernels/iq4_xs.py:35-39: searchsorted(right), clamp to 1..15, then the float midpoint
compare) by one load from a table indexed by floor(clamp(al, -136, 134.5)), the floor taken
as an add rounding toward -inf of 1.5 * 2^23 + 136. This checks that lookup against the
search on every float class: random values, the midpoints and levels with their
neighbouring floats, integers and half-integers, values beyond both clamps, +-inf and NaN.
"""

import numpy as np

KV = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], np.float32)
TAB_LO, TAB_N = -136, 271


def search_level(al: np.ndarray) -> np.ndarray:
    """_best_index as the oracle writes it: count kv <= al, clamp to 1..15, compare."""
    mu = (KV[None, :] <= al[:, None]).sum(1).clip(1, 15)
    lo, hi = KV[mu - 1], KV[mu]
    with np.errstate(invalid="ignore"):
        return np.where((al - lo) < (hi - al), lo, hi)


def table() -> np.ndarray:
    """Row e = floor - TAB_LO: the bracket {kv[p], kv[p + 1]}, p = #kv[1..14] <= floor."""
    f = np.arange(TAB_N, dtype=np.float32) + TAB_LO
    p = (KV[None, 1:15] <= f[:, None]).sum(1)
    return np.stack([KV[p], KV[p + 1]], 1)


def table_level(al: np.ndarray) -> np.ndarray:
    y = np.minimum(np.maximum(al, np.float32(TAB_LO)), np.float32(134.5))
    y = np.where(np.isnan(al), np.float32(TAB_LO), y)   # max.f32 returns the non-NaN operand
    # y + 1.5 * 2^23 + 136 is exact in float64; rounding it down to float32 in [2^23, 2^24),
    # where one ulp is 1, is the floor
    e = (np.floor(y.astype(np.float64) + 12583048.0).astype(np.int64) - 12582912) & 0x1FF
    assert e.max() < TAB_N
    t = table()
    lo, hi = t[e, 0], t[e, 1]
    with np.errstate(invalid="ignore"):
        return np.where((al - lo) < (hi - al), lo, hi)


def test_table_lookup_equals_the_bracket_search():
    rng = np.random.default_rng(7)
    mids = ((KV[:-1] + KV[1:]) / 2).astype(np.float32)
    up, dn = np.float32(np.inf), np.float32(-np.inf)
    ints = np.arange(-300, 300, dtype=np.float32)
    parts = [
        rng.uniform(-200, 200, 200_000).astype(np.float32),
        rng.normal(0, 1, 50_000).astype(np.float32),
        (rng.normal(0, 1, 50_000) * 1e-30).astype(np.float32),
        mids, np.nextafter(mids, up), np.nextafter(mids, dn),
        KV, np.nextafter(KV, up), np.nextafter(KV, dn),
        ints, ints + np.float32(0.5), np.nextafter(ints, dn),
        np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e30, -1e30, 134.4, 134.6, 135.0,
                  -136.5, -135.9, 3.4e38, -3.4e38], np.float32),
    ]
    al = np.concatenate(parts)
    got, want = table_level(al), search_level(al)
    same = (got == want) | (np.isnan(got) & np.isnan(want))
    assert same.all(), f"differs at {al[~same][:8]}"


def test_nan_takes_the_second_level():
    assert table_level(np.array([np.nan], np.float32))[0] == KV[1] == search_level(np.array([np.nan], np.float32))[0]
