// Search cores of the k-quants, one thread per quantization group.
//
// Each function restates a reference site op for op (see the citations); the thread
// keeps the whole group in registers, so the reference's sequential and pairwise sum
// orders come out exactly.
#pragma once

#include "qs_common.cuh"

namespace qs {

// make_qkx_quants_eager (kernels/kq_common.py:51-96): weighted [scale, min] fit over
// the candidate numerators `steps`; L gets the levels 0..NMAX of the accepted step.
template <int N, int NMAX, bool MAD>
__device__ __forceinline__ float qkx_search(const float* x, const float* w, const float* steps, int nsteps,
                                            float& the_min, float* L) {
    const float fmax = (float)NMAX;
    float mn = min_of<N>(x);
    mn = mn > 0.0f ? 0.0f : mn;
    const float mx = max_of<N>(x);
    const bool degen = mx == mn;
    const float sum_w = tree_sum<N>(w);
    float t[N];
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = w[i] * x[i];
    const float sum_x = tree_sum<N>(t);

    float iscale = __fdiv_rn(fmax, degen ? 1.0f : mx - mn);
    float scale = rcp_rn(iscale);
#pragma unroll
    for (int i = 0; i < N; i++) {
        float l = clamp_nan(rintf(iscale * (x[i] - mn)), 0.0f, fmax);
        float d = (scale * l + mn) - x[i];
        t[i] = MAD ? w[i] * fabsf(d) : w[i] * (d * d);
    }
    float best = tree_sum<N>(t);
    // the accepted levels are rebuilt from (isc, mn) of the winning step at the end
    float win_isc = iscale, win_mn = mn;

    if constexpr (N == 32) {
        // the candidate steps on packed pairs (v[k], v[k + N/2]): every operation is the scalar
        // one, two values at a time, and the adjacent-pair trees stay lane-parallel (tree_sum2).
        // Products are f2_mul_z (a -0 product comes out +0) where that sign cannot reach a result:
        // isc (x - mn) feeds the rounding add; w l and w l l are -0 only for a -0 weight, and
        // their sums matter only when nonzero (D > 0); the residual products are squared or
        // taken absolute after + tm - x. w l x keeps scalar products: a zero weight on a negative
        // value makes a -0 term, and an all-zero sum_xl's sign reaches ts.
        constexpr int H = N / 2;
        f32x2 x2[H], w2[H];
#pragma unroll
        for (int k = 0; k < H; k++) {
            x2[k] = f2_pack(x[k], x[k + H]);
            w2[k] = f2_pack(w[k], w[k + H]);
        }
        const f32x2 magic = f2_splat(12582912.0f), nmagic = f2_splat(-12582912.0f);
#pragma unroll 1
        for (int s = 0; s < nsteps; s++) {
            const float isc = __fdiv_rn(steps[s], degen ? 1.0f : mx - mn);
            const f32x2 isc2 = f2_splat(isc), mn2 = f2_splat(mn);
            f32x2 la[H], wl[H], wl2[H], wlx[H];
#pragma unroll
            for (int k = 0; k < H; k++) {
                // clamp(rint_add(isc * (x - mn)), 0, fmax), the clamp per lane
                float l0, l1;
                f2_unpack(f2_add(f2_add(f2_mul_z(isc2, f2_sub(x2[k], mn2)), magic), nmagic), l0, l1);
                la[k] = f2_pack(clamp_nan(l0, 0.0f, fmax), clamp_nan(l1, 0.0f, fmax));
                wl[k] = f2_mul_z(w2[k], la[k]);
                wl2[k] = f2_mul_z(wl[k], la[k]);
                float a0, a1;
                f2_unpack(wl[k], a0, a1);
                wlx[k] = f2_pack(a0 * x[k], a1 * x[k + H]);
            }
            const float sum_l = tree_sum2<H>(wl);
            const float sum_l2 = tree_sum2<H>(wl2);
            const float sum_xl = tree_sum2<H>(wlx);
            const float D = sum_w * sum_l2 - sum_l * sum_l;
            const float Dsafe = D > 0.0f ? D : 1.0f;
            float ts = __fdiv_rn(sum_w * sum_xl - sum_x * sum_l, Dsafe);
            float tm = __fdiv_rn(sum_l2 * sum_x - sum_l * sum_xl, Dsafe);
            if (tm > 0.0f) {
                ts = __fdiv_rn(sum_xl, sum_l2 < F32_TINY ? F32_TINY : sum_l2);
                tm = 0.0f;
            }
            const f32x2 ts2 = f2_splat(ts), tm2 = f2_splat(tm);
            f32x2 t2[H];
#pragma unroll
            for (int k = 0; k < H; k++) {
                const f32x2 d = f2_sub(f2_add(f2_mul_z(ts2, la[k]), tm2), x2[k]);  // (ts * la + tm) - x
                t2[k] = MAD ? f2_mul_z(w2[k], f2_abs(d)) : f2_mul_z(w2[k], f2_mul_z(d, d));
            }
            const float cur = tree_sum2<H>(t2);
            if (D > 0.0f && cur < best && !degen) {
                win_isc = isc;
                win_mn = mn;
                scale = ts;
                mn = tm;
                best = cur;
            }
        }
    } else {  // 16-value groups: scalar (the packed form measured 6 % slower on Q2_K)
#pragma unroll 1
        for (int s = 0; s < nsteps; s++) {
            const float isc = __fdiv_rn(steps[s], degen ? 1.0f : mx - mn);
            float la[N], wl[N], wl2[N], wlx[N];
#pragma unroll
            for (int i = 0; i < N; i++) {
                la[i] = clamp_nan(rint_add(isc * (x[i] - mn)), 0.0f, fmax);
                wl[i] = w[i] * la[i];
                wl2[i] = wl[i] * la[i];
                wlx[i] = wl[i] * x[i];
            }
            const float sum_l = tree_sum<N>(wl);
            const float sum_l2 = tree_sum<N>(wl2);
            const float sum_xl = tree_sum<N>(wlx);
            const float D = sum_w * sum_l2 - sum_l * sum_l;
            const float Dsafe = D > 0.0f ? D : 1.0f;
            float ts = __fdiv_rn(sum_w * sum_xl - sum_x * sum_l, Dsafe);
            float tm = __fdiv_rn(sum_l2 * sum_x - sum_l * sum_xl, Dsafe);
            if (tm > 0.0f) {
                ts = __fdiv_rn(sum_xl, sum_l2 < F32_TINY ? F32_TINY : sum_l2);
                tm = 0.0f;
            }
#pragma unroll
            for (int i = 0; i < N; i++) {
                float d = (ts * la[i] + tm) - x[i];
                t[i] = MAD ? w[i] * fabsf(d) : w[i] * (d * d);
            }
            const float cur = tree_sum<N>(t);
            if (D > 0.0f && cur < best && !degen) {
                win_isc = isc;
                win_mn = mn;
                scale = ts;
                mn = tm;
                best = cur;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < N; i++) L[i] = degen ? 0.0f : clampf(rintf(win_isc * (x[i] - win_mn)), 0.0f, fmax);
    the_min = mn == 0.0f ? 0.0f : -mn;
    return degen ? 0.0f : scale;
}

// make_qp_quants_eager (kernels/kq_common.py:99-141) over N values; torch `.sum(-1)`
// orders for N = 8 / 16 / 32. steps: the 8 candidate numerators.
template <int N>
__device__ __forceinline__ float qp_search(const float* x, const float* w, float nmax, const float* steps, float* L) {
    float t[N];
    const float mx = max_of<N>(x);
    const bool dead = mx < EPS15;
    const float r = rcp_rn(dead ? 1.0f : mx);
    float iscale = r * nmax;
    {
        const float ri = rcp_rn(iscale);
#pragma unroll
        for (int i = 0; i < N; i++) {
            float d = x[i] - ri * rintf(iscale * x[i]);
            t[i] = w[i] * (d * d);
        }
    }
    float best_mse = torch_sum<N>(t);
#pragma unroll 1
    for (int s = 0; s < 8; s++) {
        const float isc = r * steps[s];
        const float ric = rcp_rn(isc);
#pragma unroll
        for (int i = 0; i < N; i++) {
            float d = x[i] - ric * min_hi(rintf(isc * x[i]), nmax);
            t[i] = w[i] * (d * d);
        }
        const float mse = torch_sum<N>(t);
        if (mse < best_mse) { best_mse = mse; iscale = isc; }
    }
#pragma unroll
    for (int i = 0; i < N; i++) L[i] = min_hi(rintf(iscale * x[i]), nmax);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = (w[i] * x[i]) * L[i];
    float sumlx = torch_sum<N>(t);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = (w[i] * L[i]) * L[i];
    float suml2 = torch_sum<N>(t);
#pragma unroll 1
    for (int p = 0; p < 5; p++) {
#pragma unroll
        for (int i = 0; i < N; i++) {
            const float xi = x[i], wi = w[i], Li = L[i];
            const float slx = sumlx - (wi * xi) * Li;
            const float sl2 = suml2 - (wi * Li) * Li;
            const bool ok = slx > 0.0f && sl2 > 0.0f;
            const float newl = min_hi(rintf(__fdiv_rn(xi * sl2, ok ? slx : 1.0f)), nmax);
            const float slx2 = slx + (wi * xi) * newl;
            const float sl22 = sl2 + (wi * newl) * newl;
            if (ok && newl != Li && (slx2 * slx2) * suml2 > (sumlx * sumlx) * sl22) {
                L[i] = newl;
                sumlx = slx2;
                suml2 = sl22;
            }
        }
    }
    float scale = suml2 > 0.0f ? __fdiv_rn(sumlx, suml2 < F32_TINY ? F32_TINY : suml2) : 0.0f;
    if (dead) {
        scale = 0.0f;
#pragma unroll
        for (int i = 0; i < N; i++) L[i] = 0.0f;
    }
    return scale;
}

// One element's greedy try of make_qp_quants_eager (kernels/kq_common.py:125-137) against the
// superblock's current sums, for qp_pair below. State is replicated on the superblock's
// lanes except L (the lane's own level). The first lane at or after the pass position whose
// element commits is applied: the elements before it were tried with the same sums and did
// not commit, exactly as in the sequential pass.
struct QpGreedy {
    float slx, sl2, L;
    int pos, pass;
    bool moved, done;
};

template <int N>
__device__ __forceinline__ void qp_greedy_try(QpGreedy& st, float xi, float wi, float nmax, int g, int base) {
    const float Li = st.L;
    const float slx = st.slx - (wi * xi) * Li;
    const float sl2 = st.sl2 - (wi * Li) * Li;
    const bool ok = slx > 0.0f && sl2 > 0.0f;
    const float newl = min_hi(rintf(__fdiv_rn(xi * sl2, ok ? slx : 1.0f)), nmax);
    const float slx2 = slx + (wi * xi) * newl;
    const float sl22 = sl2 + (wi * newl) * newl;
    const bool commit = !st.done && g >= st.pos && ok && newl != Li &&
                        (slx2 * slx2) * st.sl2 > (st.slx * st.slx) * sl22;
    const unsigned bits = (__ballot_sync(0xFFFFFFFFu, commit) >> base) & ((1u << N) - 1u);
    const int j = bits ? __ffs(bits) - 1 : g;
    const float nx = __shfl_sync(0xFFFFFFFFu, slx2, base + j);
    const float n2 = __shfl_sync(0xFFFFFFFFu, sl22, base + j);
    if (st.done) return;
    if (bits) {
        st.slx = nx;
        st.sl2 = n2;
        if (g == j) st.L = newl;
        st.moved = true;
        st.pos = j + 1;
    } else {
        st.pos = N;
    }
    if (st.pos == N) {  // end of the pass; a pass without a commit would repeat unchanged
        if (!st.moved || st.pass == 4) st.done = true;
        else { st.pass++; st.pos = 0; st.moved = false; }
    }
}

// make_qp_quants_eager (kernels/kq_common.py:99-141) for both vectors of one superblock (its
// N block scales xa and N block mins xb, weights w; all in shared memory), spread over the
// superblock's N lanes (N = 8 or 16, lanes aligned to N in the warp; every lane of the warp
// calls this). Lane g owns element g. The 18 candidate fits (first guess + 8 steps, per
// vector) are evaluated one per lane per pass into mse[18]; every lane replays the strict-<
// selection over them in the reference's order; the greedy passes run element-parallel
// (qp_greedy_try). Results: the lane's own levels La / Lb and the scales da / db, the same
// values qp_search gives for each vector.
template <int N>
__device__ __forceinline__ void qp_pair(const float* xa, const float* xb, const float* w, float nmax,
                                        const float* steps, float* mse, int g,
                                        float& La, float& Lb, float& da, float& db) {
    const int base = (threadIdx.x & 31) & ~(N - 1);
    float mxa = xa[0], mxb = xb[0];
#pragma unroll
    for (int i = 1; i < N; i++) {
        mxa = xa[i] > mxa ? xa[i] : mxa;
        mxb = xb[i] > mxb ? xb[i] : mxb;
    }
    const bool deada = mxa < EPS15, deadb = mxb < EPS15;
    const float ra = rcp_rn(deada ? 1.0f : mxa), rb = rcp_rn(deadb ? 1.0f : mxb);

#pragma unroll 1
    for (int j = g; j < 18; j += N) {
        const bool vb = j >= 9;
        const int c = vb ? j - 9 : j;
        const float* x = vb ? xb : xa;
        const float isc = (vb ? rb : ra) * (c == 0 ? nmax : steps[c - 1]);
        const float ric = rcp_rn(isc);
        const float hi = c == 0 ? __int_as_float(0x7F800000) : nmax;  // the first guess is not clamped
        float s = 0.0f;
        if (N == 8) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float d = x[i] - ric * min_hi(rintf(isc * x[i]), hi);
                s = __fadd_rn(s, w[i] * (d * d));
            }
        } else {
#pragma unroll
            for (int l = 0; l < 8; l++) {
                const float d0 = x[l] - ric * min_hi(rintf(isc * x[l]), hi);
                const float d1 = x[8 + l] - ric * min_hi(rintf(isc * x[8 + l]), hi);
                s = __fadd_rn(s, __fadd_rn(w[l] * (d0 * d0), w[8 + l] * (d1 * d1)));
            }
        }
        mse[j] = s;
    }
    __syncwarp();

    float isa = ra * nmax, isb = rb * nmax, ba = mse[0], bb = mse[9];
#pragma unroll
    for (int s = 0; s < 8; s++) {
        if (mse[1 + s] < ba) { ba = mse[1 + s]; isa = ra * steps[s]; }
        if (mse[10 + s] < bb) { bb = mse[10 + s]; isb = rb * steps[s]; }
    }
    QpGreedy A{0.0f, 0.0f, 0.0f, 0, 0, false, false}, B{0.0f, 0.0f, 0.0f, 0, 0, false, false};
    {
        float t[N], u[N];
#pragma unroll
        for (int i = 0; i < N; i++) {
            const float l = min_hi(rintf(isa * xa[i]), nmax);
            t[i] = (w[i] * xa[i]) * l;
            u[i] = (w[i] * l) * l;
        }
        A.slx = torch_sum<N>(t);
        A.sl2 = torch_sum<N>(u);
#pragma unroll
        for (int i = 0; i < N; i++) {
            const float l = min_hi(rintf(isb * xb[i]), nmax);
            t[i] = (w[i] * xb[i]) * l;
            u[i] = (w[i] * l) * l;
        }
        B.slx = torch_sum<N>(t);
        B.sl2 = torch_sum<N>(u);
    }
    const float xga = xa[g], xgb = xb[g], wg = w[g];
    A.L = min_hi(rintf(isa * xga), nmax);
    B.L = min_hi(rintf(isb * xgb), nmax);
#pragma unroll 1
    while (__any_sync(0xFFFFFFFFu, !(A.done && B.done))) {
        qp_greedy_try<N>(A, xga, wg, nmax, g, base);
        qp_greedy_try<N>(B, xgb, wg, nmax, g, base);
    }
    da = A.sl2 > 0.0f ? __fdiv_rn(A.slx, A.sl2 < F32_TINY ? F32_TINY : A.sl2) : 0.0f;
    db = B.sl2 > 0.0f ? __fdiv_rn(B.slx, B.sl2 < F32_TINY ? F32_TINY : B.sl2) : 0.0f;
    La = deada ? 0.0f : A.L;
    Lb = deadb ? 0.0f : B.L;
    if (deada) da = 0.0f;
    if (deadb) db = 0.0f;
}

// make_qx_quants_eager (kernels/qx_common.py:52-82), rmse_type 1; L gets level + NMAX.
// steps: the 18 candidate numerators.
template <int N>
__device__ __forceinline__ float qx_search(const float* x, const float* w, float fmax, const float* steps, float* L) {
    float amax, mx;
    absmax_first<N>(x, amax, mx);
    const bool live = amax >= EPS15;
    const float r = rcp_rn(live ? mx : 1.0f);
    float wx[N], t[N];
#pragma unroll
    for (int i = 0; i < N; i++) wx[i] = w[i] * x[i];
    float iscale = r * (-fmax);
#pragma unroll
    for (int i = 0; i < N; i++) L[i] = clampf(rintf(iscale * x[i]), -fmax, fmax - 1.0f);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = wx[i] * L[i];
    const float sumlx = seq_sum<N>(t);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = (w[i] * L[i]) * L[i];
    const float suml2 = seq_sum<N>(t);
    float scale = suml2 != 0.0f ? __fdiv_rn(sumlx, suml2) : 0.0f;
    float best = scale * sumlx;
    float win_isc = iscale;
#pragma unroll 1
    for (int s = 0; s < 18; s++) {
        const float isc = r * (-steps[s]);
        // adjacent pairs on f32x2, the sums still left to right. clamp(rint(.)) is the rounding add
        // pair and a NaN-propagating clamp (as in qkx_search), and every product is f2_mul_z: a
        // zero level or product may come out +0 where the reference's is -0. That changes only
        // an all-zero sum's sign. sl2 <= 0 is rejected whatever its sign, and the accepted levels
        // are rebuilt from the winning iscale below. slx == 0 passes the accept test only when
        // best < 0 (negative weights), and there the reference's zero is +0 as well: with isc > 0
        // the positively weighted nonzero level that sl2 > 0 needs gives a +0 or positive term,
        // with isc < 0 the negatively weighted one that made best < 0 does. The branch that sums
        // slx again as the reference does is a guard that gives the same value.
        float slx = 0.0f, sl2 = 0.0f;
        const f32x2 isc2 = f2_splat(isc), magic = f2_splat(12582912.0f), nmagic = f2_splat(-12582912.0f);
#pragma unroll
        for (int k = 0; k < N / 2; k++) {
            float l0, l1;
            f2_unpack(f2_add(f2_add(f2_mul_z(isc2, f2_pack(x[2 * k], x[2 * k + 1])), magic), nmagic), l0, l1);
            const f32x2 la = f2_pack(clamp_nan(l0, -fmax, fmax - 1.0f), clamp_nan(l1, -fmax, fmax - 1.0f));
            float a0, a1, b0, b1;
            f2_unpack(f2_mul_z(f2_pack(wx[2 * k], wx[2 * k + 1]), la), a0, a1);
            f2_unpack(f2_mul_z(f2_mul_z(f2_pack(w[2 * k], w[2 * k + 1]), la), la), b0, b1);
            slx = k == 0 ? __fadd_rn(a0, a1) : __fadd_rn(__fadd_rn(slx, a0), a1);
            sl2 = k == 0 ? __fadd_rn(b0, b1) : __fadd_rn(__fadd_rn(sl2, b0), b1);
        }
        if (sl2 > 0.0f && slx * slx > best * sl2) {
            if (slx == 0.0f) {
#pragma unroll
                for (int i = 0; i < N; i++) t[i] = wx[i] * clampf(rintf(isc * x[i]), -fmax, fmax - 1.0f);
                slx = seq_sum<N>(t);
            }
            const float cand = __fdiv_rn(slx, sl2);
            scale = cand;
            best = cand * slx;
            win_isc = isc;
        }
    }
#pragma unroll
    for (int i = 0; i < N; i++)
        L[i] = live ? clampf(rintf(win_isc * x[i]), -fmax, fmax - 1.0f) + fmax : 0.0f;
    return live ? scale : 0.0f;
}

// make_q3_quants_eager (kernels/qx_common.py:85-121), do_rmse; L gets level + NMAX.
template <int N>
__device__ __forceinline__ float q3_search(const float* x, float fmax, float* L) {
    float w[N], t[N], amax, mx;
#pragma unroll
    for (int i = 0; i < N; i++) w[i] = x[i] * x[i];
    absmax_first<N>(x, amax, mx);
    const bool live = amax >= EPS15;
    const float iscale = rcp_rn(live ? mx : 1.0f) * (-fmax);
#pragma unroll
    for (int i = 0; i < N; i++) L[i] = clampf(rintf(iscale * x[i]), -fmax, fmax - 1.0f);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = (w[i] * x[i]) * L[i];
    float sumlx = seq_sum<N>(t);
#pragma unroll
    for (int i = 0; i < N; i++) t[i] = (w[i] * L[i]) * L[i];
    float suml2 = seq_sum<N>(t);
#pragma unroll 1
    for (int p = 0; p < 5; p++) {
#pragma unroll
        for (int i = 0; i < N; i++) {
            const float xi = x[i], wi = w[i], Li = L[i];
            const float slx = sumlx - (wi * xi) * Li;
            const bool ok = slx > 0.0f;
            const float sl2 = suml2 - (wi * Li) * Li;
            const float newl = clampf(rintf(__fdiv_rn(xi * sl2, ok ? slx : 1.0f)), -fmax, fmax - 1.0f);
            const float slx2 = slx + (wi * xi) * newl;
            const float sl22 = sl2 + (wi * newl) * newl;
            if (ok && newl != Li && sl22 > 0.0f && (slx2 * slx2) * suml2 > (sumlx * sumlx) * sl22) {
                L[i] = newl;
                sumlx = slx2;
                suml2 = sl22;
            }
        }
    }
    const float scale = suml2 > 0.0f ? __fdiv_rn(sumlx, suml2) : 0.0f;
#pragma unroll
    for (int i = 0; i < N; i++) L[i] = live ? L[i] + fmax : 0.0f;
    return live ? scale : 0.0f;
}

}  // namespace qs
