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
        float l = clampf(rintf(iscale * (x[i] - mn)), 0.0f, fmax);
        float d = (scale * l + mn) - x[i];
        t[i] = MAD ? w[i] * fabsf(d) : w[i] * (d * d);
    }
    float best = tree_sum<N>(t);
    // the accepted levels are rebuilt from (isc, mn) of the winning step at the end
    float win_isc = iscale, win_mn = mn;

#pragma unroll 1
    for (int s = 0; s < nsteps; s++) {
        const float isc = __fdiv_rn(steps[s], degen ? 1.0f : mx - mn);
        float la[N], wl[N], wl2[N], wlx[N];
#pragma unroll
        for (int i = 0; i < N; i++) {
            la[i] = clampf(rintf(isc * (x[i] - mn)), 0.0f, fmax);
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
        float slx = 0.0f, sl2 = 0.0f;
#pragma unroll
        for (int i = 0; i < N; i++) {
            const float la = clampf(rintf(isc * x[i]), -fmax, fmax - 1.0f);
            const float a = wx[i] * la, b = (w[i] * la) * la;
            slx = i == 0 ? a : slx + a;
            sl2 = i == 0 ? b : sl2 + b;
        }
        if (sl2 > 0.0f && slx * slx > best * sl2) {
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
