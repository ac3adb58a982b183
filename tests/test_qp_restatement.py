"""The superblock scale/min fit as the GPU runs it, checked against the sequential fit (CPU).

make_qp_quants (kernels/kq_common.py:99-141) fits the 8 block scales (or mins) of a Q4_K /
Q5_K superblock, 16 for Q2_K: a first guess, 8 candidate steps with strict-< selection, then
5 greedy passes that re-fit one element at a time against running sums. The CUDA kernel
(`qp_pair` in quant-studio_b200/csrc/qs_kquant.cuh) runs it over the superblock's lanes in a
different order: the candidate fits are computed independently and the selection replayed in
the reference's order; in a greedy pass every element is tried against the current sums at
once and the first element at or after the pass position that commits is applied (the
elements before it saw the same sums and did not commit), then the rest are tried again; a
pass without a commit ends the search. This file restates that order in float32 numpy and
checks it against the oracle's sequential fit, bit for bit, on inputs that make the greedy
passes commit (including in the last pass), for n = 8 (nmax 63) and n = 16 (nmax 15).
The GPU parity tests check the kernel itself; this checks the reordering argument on many
more inputs than the parity fixtures hold.
"""

import ctypes

import numpy as np
import pytest

import oracle

f = np.float32
EPS15 = f(1e-15)
TINY = f(1.17549435e-38)


def _min_hi(v, hi):
    return hi if v > hi else v


def _torch_sum(t):  # torch CPU `.sum(-1)` for 8 (left to right from +0) or 16 (lane pairs)
    s = f(0)
    if len(t) == 8:
        for v in t:
            s = f(s + v)
    else:
        for l in range(8):
            s = f(s + f(t[l] + t[8 + l]))
    return s


def _steps(nmax):  # kernels/kq_common.py:27-30, folded in float32 like the kernel's table
    return [f(f(f(0.1) * f(s)) + f(nmax)) for s in range(-4, 5) if s]


def qp_parallel(x, w, nmax):
    """The GPU order of make_qp: returns (scale, levels, greedy commits made)."""
    n, nm, steps = len(x), f(nmax), _steps(nmax)
    mx = x[0]
    for v in x[1:]:
        mx = v if v > mx else mx
    dead = mx < EPS15
    r = f(f(1) / (f(1) if dead else mx))
    # the 9 candidate fits, each on its own (one per lane on the GPU)
    mse = []
    for c in range(9):
        isc = f(r * (nm if c == 0 else steps[c - 1]))
        ric = f(f(1) / isc)
        hi = f(np.inf) if c == 0 else nm  # the first guess is not clamped
        mse.append(_torch_sum([f(w[i] * f(f(x[i] - f(ric * _min_hi(np.rint(f(isc * x[i])), hi))) ** 2))
                               for i in range(n)]))
    # strict-< selection replayed in the reference's order
    isc, best = f(r * nm), mse[0]
    for s in range(8):
        if mse[1 + s] < best:
            best, isc = mse[1 + s], f(r * steps[s])
    L = [_min_hi(np.rint(f(isc * x[i])), nm) for i in range(n)]
    slx = _torch_sum([f(f(w[i] * x[i]) * L[i]) for i in range(n)])
    sl2 = _torch_sum([f(f(w[i] * L[i]) * L[i]) for i in range(n)])
    pos, npass, moved, commits = 0, 0, False, 0
    while True:
        # every element tried against the same sums
        tries = []
        for g in range(n):
            a = f(slx - f(f(w[g] * x[g]) * L[g]))
            b = f(sl2 - f(f(w[g] * L[g]) * L[g]))
            ok = a > 0 and b > 0
            newl = _min_hi(np.rint(f(f(x[g] * b) / (a if ok else f(1)))), nm)
            a2 = f(a + f(f(w[g] * x[g]) * newl))
            b2 = f(b + f(f(w[g] * newl) * newl))
            commit = g >= pos and ok and newl != L[g] and f(f(a2 * a2) * sl2) > f(f(slx * slx) * b2)
            tries.append((commit, a2, b2, newl))
        first = next((g for g in range(n) if tries[g][0]), None)
        if first is not None:
            _, slx, sl2, L[first] = tries[first]
            moved, pos, commits = True, first + 1, commits + 1
        else:
            pos = n
        if pos == n:  # end of a pass; a pass without a commit would repeat unchanged
            if not moved or npass == 4:
                break
            npass, pos, moved = npass + 1, 0, False
    d = f(slx / (TINY if sl2 < TINY else sl2)) if sl2 > 0 else f(0)
    if dead:
        d, L = f(0), [f(0)] * n
    return d, np.array(L, dtype=np.float32), commits


def _inputs(rng, n, kind):
    if kind == 0:    # block scales of the benchmark distribution's size
        x = rng.lognormal(-5.0, 0.5, n)
    elif kind == 1:  # wide spread: many greedy commits
        x = rng.lognormal(-5.0, 1.5, n)
    elif kind == 2:  # zeros mixed in
        x = np.abs(rng.normal(0.0, 1e-3, n))
        x[rng.random(n) < 0.3] = 0.0
    else:            # values on a coarse grid: ties between candidates
        x = rng.integers(0, 64, n) * 1e-4
    return x.astype(np.float32), rng.lognormal(0.0, 1.5, n).astype(np.float32)


@pytest.mark.parametrize("n, nmax", [(8, 63), (16, 15)])
def test_parallel_fit_equals_sequential(n, nmax):
    L = oracle.lib()
    L.oq_core_qp.restype = ctypes.c_float
    L.oq_core_qp.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    rng = np.random.default_rng(3 + n)
    np.seterr(all="ignore")
    commits = 0
    for it in range(600):
        x, w = _inputs(rng, n, it % 4)
        lv = np.zeros(n, np.float32)
        want = np.float32(L.oq_core_qp(x.ctypes.data, w.ctypes.data, n, nmax, lv.ctypes.data))
        got, got_l, c = qp_parallel(list(x), list(w), nmax)
        commits += c
        assert np.float32(got).view(np.uint32) == want.view(np.uint32), (it, got, want)
        assert np.array_equal(got_l, lv), (it, got_l, lv)
    assert commits > 100  # the greedy passes were exercised
