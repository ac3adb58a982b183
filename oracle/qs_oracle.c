/*
 * CPU oracle for the bf16 -> GGML block quantizers (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the reference's eager torch path (ngxson/quant-studio,
 * kernels/<type>.py), which is the ground truth for every block format here. Only the
 * test suite, the smoke check and the bench's CPU-baseline leg may load this file's
 * library; the product path never does.
 *
 * Every function follows the eager torch code op by op, with the same rounding:
 *   - no FMA contraction (build with -ffp-contract=off);
 *   - `python_scalar / tensor` is torch's reciprocal-then-multiply (two roundings),
 *     `tensor / x` a true IEEE divide;
 *   - torch.round is round-half-even (nearbyintf);
 *   - `.sum(-1)` on a float32 CPU tensor follows torch's 8-lane cascade (tsum*),
 *     the reference's own seq_sum / tree_sum keep their explicit orders.
 * Pinned against the fixtures in tests/golden (outputs of the reference itself); the four
 * formats the reference has no kernel for (Q4_1, Q5_0, Q5_1, Q8_0) restate gguf-py's
 * quantizers and are pinned against gguf-py on the same inputs (tests/test_oracle_golden.py).
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "qs_oracle.h"

typedef float f32;

#define QK_K 256
#define EPS15 1e-15f
#define EPS8 1e-8f
static const f32 F32_TINY = 1.17549435e-38f; /* torch.finfo(float32).tiny */

/* ------------------------------------------------------------------ */
/* numeric helpers                                                      */
/* ------------------------------------------------------------------ */

static inline f32 rcp(f32 x) { return 1.0f / x; }
static inline f32 rnd(f32 x) { return nearbyintf(x); }
static inline f32 clampf(f32 x, f32 lo, f32 hi) { return x < lo ? lo : (x > hi ? hi : x); }
static inline f32 minf_(f32 x, f32 hi) { return x > hi ? hi : x; }

static inline uint16_t f16_bits(f32 v) {
    _Float16 h = (_Float16)v; /* round to nearest even */
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}
static inline f32 f16_val(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (f32)h;
}
static inline void put16(uint8_t *p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* torch CPU float32 .sum(-1) over a contiguous last dim (torch 2.11, 8-lane vectors):
 * n < 8 sequential; else lane partials then a sequential pass over the 8 lanes. */
static f32 tsum8(const f32 *x) {
    f32 s = 0.0f;
    for (int i = 0; i < 8; i++) s += x[i];
    return s;
}
static f32 tsum16(const f32 *x) {
    f32 s = 0.0f;
    for (int l = 0; l < 8; l++) s += (x[l] + x[8 + l]);
    return s;
}
static f32 tsum32(const f32 *x) {
    f32 s = 0.0f;
    for (int l = 0; l < 8; l++) s += ((x[l] + x[8 + l]) + x[16 + l]) + x[24 + l];
    return s;
}
static f32 tsum256(const f32 *x) {
    /* 32 vectors of 8; four accumulators take vectors 4i+k, i = 0..7 */
    f32 s = 0.0f;
    for (int l = 0; l < 8; l++) {
        f32 acc[4];
        for (int k = 0; k < 4; k++) {
            f32 a = 0.0f;
            for (int i = 0; i < 8; i++) a += x[8 * (4 * i + k) + l];
            acc[k] = a + 0.0f;
        }
        s += ((acc[0] + acc[1]) + acc[2]) + acc[3];
    }
    return s;
}
static f32 tsum_n(const f32 *x, int n) {
    switch (n) {
    case 8: return tsum8(x);
    case 16: return tsum16(x);
    case 32: return tsum32(x);
    default: return tsum256(x);
    }
}
/* reference seq_sum: parts[0] + parts[1] + ... (no zero seed) */
static f32 seq_sum(const f32 *x, int n) {
    f32 s = x[0];
    for (int i = 1; i < n; i++) s = s + x[i];
    return s;
}
/* reference tree_sum: adjacent pairs, n a power of two */
static f32 tree_sum(const f32 *x, int n) {
    f32 t[32];
    for (int i = 0; i < n; i++) t[i] = x[i];
    while (n > 1) {
        for (int i = 0; i < n / 2; i++) t[i] = t[2 * i] + t[2 * i + 1];
        n /= 2;
    }
    return t[0];
}
/* absmax_first (qx_common.py:26-34): max |x| and the signed value at its first index */
static void absmax_first(const f32 *x, int n, f32 *amax, f32 *mx) {
    f32 a = fabsf(x[0]);
    for (int i = 1; i < n; i++) if (fabsf(x[i]) > a) a = fabsf(x[i]);
    int first = n;
    for (int i = 0; i < n; i++) if (fabsf(x[i]) == a) { first = i; break; }
    *amax = a;
    *mx = x[first < n ? first : 0];
}
static f32 maxv(const f32 *x, int n) { f32 m = x[0]; for (int i = 1; i < n; i++) if (x[i] > m) m = x[i]; return m; }
static f32 minv(const f32 *x, int n) { f32 m = x[0]; for (int i = 1; i < n; i++) if (x[i] < m) m = x[i]; return m; }

/* ------------------------------------------------------------------ */
/* candidate tables, folded like the reference's numpy / python exprs   */
/* ------------------------------------------------------------------ */

static void qx_steps(int nmax, f32 *c) { /* qx_common.py:20-23 */
    int j = 0;
    for (int s = -9; s <= 9; s++) if (s) c[j++] = (f32)nmax + 0.1f * (f32)s;
}
static int qkx_steps(f32 rmin, f32 rdelta, int nstep, int nmax, f32 *c) { /* kq_common.py:21-24 */
    for (int s = 0; s <= nstep; s++) c[s] = (rmin + rdelta * (f32)s) + (f32)nmax;
    return nstep + 1;
}
static void qp_steps(int nmax, f32 *c) { /* kq_common.py:27-30 */
    int j = 0;
    for (int s = -4; s <= 4; s++) if (s) c[j++] = 0.1f * (f32)s + (f32)nmax;
}

/* ------------------------------------------------------------------ */
/* search cores                                                         */
/* ------------------------------------------------------------------ */

/* make_qx_quants_eager (qx_common.py:52-82); L returned with the +nmax offset */
static f32 make_qx(const f32 *x, const f32 *w, int n, int nmax, f32 *L) {
    const f32 fmax = (f32)nmax;
    f32 amax, mx, steps[18], La[16], t[16];
    absmax_first(x, n, &amax, &mx);
    int live = amax >= EPS15;
    f32 mxs = live ? mx : 1.0f;
    f32 r = rcp(mxs);
    f32 iscale = r * (-fmax);
    for (int i = 0; i < n; i++) L[i] = clampf(rnd(iscale * x[i]), -fmax, fmax - 1.0f);
    for (int i = 0; i < n; i++) t[i] = (w[i] * x[i]) * L[i];
    f32 sumlx = seq_sum(t, n);
    for (int i = 0; i < n; i++) t[i] = (w[i] * L[i]) * L[i];
    f32 suml2 = seq_sum(t, n);
    f32 scale = suml2 != 0.0f ? sumlx / suml2 : 0.0f;
    f32 best = scale * sumlx;
    qx_steps(nmax, steps);
    for (int s = 0; s < 18; s++) {
        f32 isc = r * (-steps[s]);
        for (int i = 0; i < n; i++) La[i] = clampf(rnd(isc * x[i]), -fmax, fmax - 1.0f);
        for (int i = 0; i < n; i++) t[i] = (w[i] * x[i]) * La[i];
        f32 slx = seq_sum(t, n);
        for (int i = 0; i < n; i++) t[i] = (w[i] * La[i]) * La[i];
        f32 sl2 = seq_sum(t, n);
        int acc = (sl2 > 0.0f) && (slx * slx > best * sl2);
        if (acc) {
            f32 cand = slx / sl2;
            scale = cand;
            best = cand * slx;
            memcpy(L, La, sizeof(f32) * n);
        }
    }
    for (int i = 0; i < n; i++) L[i] = live ? L[i] + fmax : 0.0f;
    return live ? scale : 0.0f;
}

/* make_q3_quants_eager (qx_common.py:85-121) */
static f32 make_q3(const f32 *x, int n, int nmax, f32 *L) {
    const f32 fmax = (f32)nmax;
    f32 w[16], t[16], amax, mx;
    for (int i = 0; i < n; i++) w[i] = x[i] * x[i];
    absmax_first(x, n, &amax, &mx);
    int live = amax >= EPS15;
    f32 mxs = live ? mx : 1.0f;
    f32 iscale = rcp(mxs) * (-fmax);
    for (int i = 0; i < n; i++) L[i] = clampf(rnd(iscale * x[i]), -fmax, fmax - 1.0f);
    for (int i = 0; i < n; i++) t[i] = (w[i] * x[i]) * L[i];
    f32 sumlx = seq_sum(t, n);
    for (int i = 0; i < n; i++) t[i] = (w[i] * L[i]) * L[i];
    f32 suml2 = seq_sum(t, n);
    for (int p = 0; p < 5; p++) {
        for (int i = 0; i < n; i++) {
            f32 xi = x[i], wi = w[i], Li = L[i];
            f32 slx = sumlx - (wi * xi) * Li;
            int ok = slx > 0.0f;
            f32 sl2 = suml2 - (wi * Li) * Li;
            f32 newl = clampf(rnd((xi * sl2) / (ok ? slx : 1.0f)), -fmax, fmax - 1.0f);
            f32 slx2 = slx + (wi * xi) * newl;
            f32 sl22 = sl2 + (wi * newl) * newl;
            int commit = ok && (newl != Li) && (sl22 > 0.0f) &&
                         ((slx2 * slx2) * suml2 > (sumlx * sumlx) * sl22);
            if (commit) { L[i] = newl; sumlx = slx2; suml2 = sl22; }
        }
    }
    f32 scale = suml2 > 0.0f ? sumlx / suml2 : 0.0f;
    for (int i = 0; i < n; i++) L[i] = live ? L[i] + fmax : 0.0f;
    return live ? scale : 0.0f;
}

/* make_qkx_quants_eager (kq_common.py:51-96); returns scale, *the_min, L in 0..nmax */
static f32 make_qkx(const f32 *x, const f32 *w, int n, const f32 *steps, int nsteps, int nmax,
                    int use_mad, f32 *the_min, f32 *L) {
    const f32 fmax = (f32)nmax;
    f32 t[32] = {0}, La[32];  /* zeroed: only t[0..n) is read, gcc cannot see that */
    f32 mn = minv(x, n);
    mn = mn > 0.0f ? 0.0f : mn;
    f32 mx = maxv(x, n);
    int degen = mx == mn;
    f32 sum_w = tree_sum(w, n);
    for (int i = 0; i < n; i++) t[i] = w[i] * x[i];
    f32 sum_x = tree_sum(t, n);
    f32 iscale = fmax / (degen ? 1.0f : mx - mn);
    f32 scale = rcp(iscale);
    for (int i = 0; i < n; i++) L[i] = clampf(rnd(iscale * (x[i] - mn)), 0.0f, fmax);
    for (int i = 0; i < n; i++) {
        f32 d = ((scale * L[i]) + mn) - x[i];
        t[i] = use_mad ? w[i] * fabsf(d) : w[i] * (d * d);
    }
    f32 best = tree_sum(t, n);
    for (int s = 0; s < nsteps; s++) {
        f32 isc = steps[s] / (degen ? 1.0f : mx - mn);
        for (int i = 0; i < n; i++) La[i] = clampf(rnd(isc * (x[i] - mn)), 0.0f, fmax);
        for (int i = 0; i < n; i++) t[i] = w[i] * La[i];
        f32 sum_l = tree_sum(t, n);
        for (int i = 0; i < n; i++) t[i] = (w[i] * La[i]) * La[i];
        f32 sum_l2 = tree_sum(t, n);
        for (int i = 0; i < n; i++) t[i] = (w[i] * La[i]) * x[i];
        f32 sum_xl = tree_sum(t, n);
        f32 D = sum_w * sum_l2 - sum_l * sum_l;
        f32 Dsafe = D > 0.0f ? D : 1.0f;
        f32 this_scale = (sum_w * sum_xl - sum_x * sum_l) / Dsafe;
        f32 this_min = (sum_l2 * sum_x - sum_l * sum_xl) / Dsafe;
        if (this_min > 0.0f) {
            this_scale = sum_xl / (sum_l2 < F32_TINY ? F32_TINY : sum_l2);
            this_min = 0.0f;
        }
        for (int i = 0; i < n; i++) {
            f32 d = ((this_scale * La[i]) + this_min) - x[i];
            t[i] = use_mad ? w[i] * fabsf(d) : w[i] * (d * d);
        }
        f32 cur = tree_sum(t, n);
        if ((D > 0.0f) && (cur < best) && !degen) {
            scale = this_scale;
            mn = this_min;
            best = cur;
            memcpy(L, La, sizeof(f32) * n);
        }
    }
    if (degen) { scale = 0.0f; for (int i = 0; i < n; i++) L[i] = 0.0f; }
    *the_min = mn == 0.0f ? 0.0f : -mn;
    return scale;
}

/* make_qp_quants_eager (kq_common.py:99-141), n = 8 or 16; also iq2.py:375-415 (n = 32) */
static f32 make_qp(const f32 *x, const f32 *w, int n, int nmax, const f32 *steps, f32 *L) {
    const f32 fmax = (f32)nmax;
    f32 t[32], l[32];
    f32 mx = maxv(x, n);
    int dead = mx < EPS15;
    f32 mxs = dead ? 1.0f : mx;
    f32 r = rcp(mxs);
    f32 iscale = r * fmax;
    f32 ri = rcp(iscale);
    for (int i = 0; i < n; i++) {
        f32 L0 = rnd(iscale * x[i]);
        f32 d = x[i] - ri * L0;
        t[i] = w[i] * (d * d);
    }
    f32 best_mse = tsum_n(t, n);
    for (int s = 0; s < 8; s++) {
        f32 isc = r * steps[s];
        f32 ric = rcp(isc);
        for (int i = 0; i < n; i++) {
            l[i] = minf_(rnd(isc * x[i]), fmax);
            f32 d = x[i] - ric * l[i];
            t[i] = w[i] * (d * d);
        }
        f32 mse = tsum_n(t, n);
        if (mse < best_mse) { best_mse = mse; iscale = isc; }
    }
    for (int i = 0; i < n; i++) L[i] = minf_(rnd(iscale * x[i]), fmax);
    for (int i = 0; i < n; i++) t[i] = (w[i] * x[i]) * L[i];
    f32 sumlx = tsum_n(t, n);
    for (int i = 0; i < n; i++) t[i] = (w[i] * L[i]) * L[i];
    f32 suml2 = tsum_n(t, n);
    for (int p = 0; p < 5; p++) {
        for (int i = 0; i < n; i++) {
            f32 xi = x[i], wi = w[i], Li = L[i];
            f32 slx = sumlx - (wi * xi) * Li;
            f32 sl2 = suml2 - (wi * Li) * Li;
            int ok = (slx > 0.0f) && (sl2 > 0.0f);
            f32 newl = minf_(rnd((xi * sl2) / (ok ? slx : 1.0f)), fmax);
            f32 slx2 = slx + (wi * xi) * newl;
            f32 sl22 = sl2 + (wi * newl) * newl;
            int commit = ok && (newl != Li) && ((slx2 * slx2) * suml2 > (sumlx * sumlx) * sl22);
            if (commit) { L[i] = newl; sumlx = slx2; suml2 = sl22; }
        }
    }
    f32 scale = suml2 > 0.0f ? sumlx / (suml2 < F32_TINY ? F32_TINY : suml2) : 0.0f;
    if (dead) { scale = 0.0f; for (int i = 0; i < n; i++) L[i] = 0.0f; }
    return scale;
}

/* imatrix weights qw * sqrt(sigma2 + x*x), sigma2 = fac * sum(x*x) / 256 */
static void imat_weights(const f32 *x, const f32 *qw, f32 fac, int seq, f32 *w) {
    f32 t[QK_K];
    for (int i = 0; i < QK_K; i++) t[i] = x[i] * x[i];
    f32 s = seq ? seq_sum(t, QK_K) : tsum256(t);
    f32 sigma2 = (fac * s) / 256.0f;
    for (int i = 0; i < QK_K; i++) w[i] = qw[i] * sqrtf(sigma2 + x[i] * x[i]);
}

/* ------------------------------------------------------------------ */
/* Q4_0 (q4_0.py:14-33), one 32-block                                   */
/* ------------------------------------------------------------------ */
static void q4_0_block(const f32 *x, uint8_t *out) {
    f32 amax, mx;
    absmax_first(x, 32, &amax, &mx);
    f32 d = mx / -8.0f;
    f32 id = d != 0.0f ? rcp(d) : 0.0f;
    put16(out, f16_bits(d));
    uint8_t q[32];
    for (int i = 0; i < 32; i++) q[i] = (uint8_t)clampf(floorf(x[i] * id + 8.5f), 0.0f, 15.0f);
    for (int i = 0; i < 16; i++) out[2 + i] = (uint8_t)(q[i] + q[16 + i] * 16);
}

/* ------------------------------------------------------------------ */
/* Q4_1 / Q5_0 / Q5_1 / Q8_0: no kernel in the reference; restated from  */
/* gguf-py 0.19.0 gguf/quants.py (Q4_1 :254-289, Q5_0 :291-331, Q5_1     */
/* :333-376, Q8_0 :378-395, np_roundf :43-47), the float32 numpy code of */
/* ggml-quants.c's quantize_row_*_ref. numpy casts float -> uint8/int8   */
/* through a 32-bit integer: non-finite or out-of-range values give 0.   */
/* ------------------------------------------------------------------ */
static inline int32_t np_i32(f32 v) {
    if (!isfinite(v) || v >= 2147483648.0f || v < -2147483648.0f) return 0;
    return (int32_t)v;
}
static inline f32 np_roundf1(f32 v) {
    f32 a = fabsf(v), f = floorf(a);
    f32 b = f + floorf(2.0f * (a - f));
    return v > 0.0f ? b : (v < 0.0f ? -b : (v == 0.0f ? 0.0f * b : v));
}
static inline f32 inv_or_zero(f32 d) { return d == 0.0f ? 0.0f : 1.0f / d; }

/* levels q[32] -> qs[16] nibble pairs (value j low, value j + 16 high) */
static void pack_nibbles(const int *q, uint8_t *qs) {
    for (int j = 0; j < 16; j++) qs[j] = (uint8_t)((q[j] & 0x0F) | ((q[16 + j] & 0x0F) << 4));
}
static void pack_high_bits(const int *q, uint8_t *qh) {
    for (int m = 0; m < 4; m++) {
        int v = 0;
        for (int j = 0; j < 8; j++) v |= ((q[8 * m + j] >> 4) != 0) << j;
        qh[m] = (uint8_t)v;
    }
}

static void q4_1_block(const f32 *x, uint8_t *out) {
    f32 mx = x[0], mn = x[0];
    for (int i = 1; i < 32; i++) { mx = x[i] > mx ? x[i] : mx; mn = x[i] < mn ? x[i] : mn; }
    f32 d = (mx - mn) / 15.0f, id = inv_or_zero(d);
    int q[32];
    for (int i = 0; i < 32; i++) {
        int v = np_i32(truncf((x[i] - mn) * id + 0.5f)) & 0xFF;
        q[i] = v > 15 ? 15 : v;
    }
    put16(out, f16_bits(d));
    put16(out + 2, f16_bits(mn));
    pack_nibbles(q, out + 4);
}

static void q5_0_block(const f32 *x, uint8_t *out) {
    f32 amax, mx;
    absmax_first(x, 32, &amax, &mx);
    f32 d = mx / -16.0f, id = inv_or_zero(d);
    int q[32];
    for (int i = 0; i < 32; i++) {
        int v = np_i32(truncf(x[i] * id + 16.5f)) & 0xFF;
        q[i] = v > 31 ? 31 : v;
    }
    put16(out, f16_bits(d));
    pack_high_bits(q, out + 2);
    pack_nibbles(q, out + 6);
}

static void q5_1_block(const f32 *x, uint8_t *out) {
    f32 mx = x[0], mn = x[0];
    for (int i = 1; i < 32; i++) { mx = x[i] > mx ? x[i] : mx; mn = x[i] < mn ? x[i] : mn; }
    f32 d = (mx - mn) / 31.0f, id = inv_or_zero(d);
    int q[32];
    for (int i = 0; i < 32; i++) {
        int v = np_i32(truncf((x[i] - mn) * id + 0.5f)) & 0xFF;
        q[i] = v > 31 ? 31 : v;
    }
    put16(out, f16_bits(d));
    put16(out + 2, f16_bits(mn));
    pack_high_bits(q, out + 4);
    pack_nibbles(q, out + 8);
}

static void q8_0_block(const f32 *x, uint8_t *out) {
    f32 amax = fabsf(x[0]);
    for (int i = 1; i < 32; i++) amax = fabsf(x[i]) > amax ? fabsf(x[i]) : amax;
    f32 d = amax / 127.0f, id = inv_or_zero(d);
    put16(out, f16_bits(d));
    for (int i = 0; i < 32; i++) out[2 + i] = (uint8_t)(np_i32(np_roundf1(x[i] * id)) & 0xFF);
}

/* ------------------------------------------------------------------ */
/* Q6_K (q6_k.py:22-65)                                                 */
/* ------------------------------------------------------------------ */
static void q6_k_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    f32 w[QK_K], L[QK_K], sc[16];
    for (int i = 0; i < QK_K; i++) w[i] = qw ? qw[i] : x[i] * x[i];
    for (int g = 0; g < 16; g++) sc[g] = make_qx(x + 16 * g, w + 16 * g, 16, 32, L + 16 * g);
    f32 amax, max_scale;
    absmax_first(sc, 16, &amax, &max_scale);
    int live = amax >= EPS15;
    f32 iscale = rcp(live ? max_scale : 1.0f) * -128.0f;
    uint16_t d16 = f16_bits(live ? rcp(iscale) : 0.0f);
    int sc8[16];
    for (int g = 0; g < 16; g++) {
        int64_t v = (int64_t)minf_(rnd(iscale * sc[g]), 127.0f);
        v = ((v & 0xFF) ^ 0x80) - 0x80;
        sc8[g] = live ? (int)v : 0;
    }
    int Lf[QK_K];
    f32 dd = f16_val(d16);
    for (int g = 0; g < 16; g++) {
        f32 dq = dd * (f32)sc8[g];
        for (int i = 0; i < 16; i++) {
            int e = 16 * g + i;
            f32 v = dq != 0.0f ? clampf(rnd(x[e] / dq), -32.0f, 31.0f) + 32.0f : L[e];
            Lf[e] = live ? (int)v : 0;
        }
    }
    uint8_t *ql = out, *qh = out + 128;
    for (int h = 0; h < 2; h++) {
        const int *q = Lf + 128 * h;
        for (int l = 0; l < 32; l++) {
            ql[64 * h + l] = (uint8_t)((q[l] & 0xF) | ((q[64 + l] & 0xF) << 4));
            ql[64 * h + 32 + l] = (uint8_t)((q[32 + l] & 0xF) | ((q[96 + l] & 0xF) << 4));
            qh[32 * h + l] = (uint8_t)((q[l] >> 4) | ((q[32 + l] >> 4) << 2) | ((q[64 + l] >> 4) << 4) |
                                       ((q[96 + l] >> 4) << 6));
        }
    }
    for (int g = 0; g < 16; g++) out[192 + g] = (uint8_t)(int8_t)sc8[g];
    put16(out + 208, d16);
}

/* ------------------------------------------------------------------ */
/* Q3_K (q3_k.py:23-78)                                                 */
/* ------------------------------------------------------------------ */
static void q3_k_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    f32 L[QK_K], sc[16];
    int ls6[16];
    uint16_t d16;
    if (!qw) {
        for (int g = 0; g < 16; g++) sc[g] = make_q3(x + 16 * g, 16, 4, L + 16 * g);
        f32 amax, max_scale;
        absmax_first(sc, 16, &amax, &max_scale);
        int has = max_scale != 0.0f;
        f32 iscale = rcp(has ? max_scale : 1.0f) * -32.0f;
        for (int g = 0; g < 16; g++) {
            int64_t l = (int64_t)rnd(iscale * sc[g]);
            l = ((l & 0xFF) ^ 0x80) - 0x80;
            l = l < -32 ? -32 : (l > 31 ? 31 : l);
            ls6[g] = has ? (int)(l + 32) : 0;
        }
        d16 = f16_bits(has ? rcp(iscale) : 0.0f);
    } else {
        f32 w[QK_K], sw[16], ls[16];
        imat_weights(x, qw, 2.0f, 1, w);
        for (int g = 0; g < 16; g++) sc[g] = make_qx(x + 16 * g, w + 16 * g, 16, 4, L + 16 * g);
        for (int g = 0; g < 16; g++) sw[g] = seq_sum(w + 16 * g, 16);
        f32 d_blk = make_qx(sc, sw, 16, 32, ls);
        for (int g = 0; g < 16; g++) ls6[g] = (int)ls[g];
        d16 = f16_bits(d_blk);
    }
    int Lf[QK_K];
    f32 dd = f16_val(d16);
    for (int g = 0; g < 16; g++) {
        f32 dq = dd * (f32)(ls6[g] - 32);
        for (int i = 0; i < 16; i++) {
            int e = 16 * g + i;
            Lf[e] = (int)(dq != 0.0f ? clampf(rnd(x[e] / dq), -4.0f, 3.0f) + 4.0f : L[e]);
        }
    }
    uint8_t *hmask = out, *qs = out + 32, *scb = out + 96;
    memset(hmask, 0, 32);
    for (int e = 0; e < QK_K; e++) if (Lf[e] > 3) hmask[e & 31] |= (uint8_t)(1 << (e >> 5));
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            int v = 0;
            for (int j = 0; j < 4; j++) {
                int q = Lf[128 * h + 32 * j + l];
                if (q > 3) q -= 4;
                v |= q << (2 * j);
            }
            qs[32 * h + l] = (uint8_t)v;
        }
    for (int j = 0; j < 8; j++) scb[j] = (uint8_t)((ls6[j] & 0xF) | ((ls6[j + 8] & 0xF) << 4));
    for (int j = 0; j < 4; j++)
        scb[8 + j] = (uint8_t)((ls6[j] >> 4) | ((ls6[4 + j] >> 4) << 2) | ((ls6[8 + j] >> 4) << 4) |
                               ((ls6[12 + j] >> 4) << 6));
    put16(out + 108, d16);
}

/* ------------------------------------------------------------------ */
/* Q4_K / Q5_K (q4_k.py:25-79, q5_k.py:25-82)                           */
/* ------------------------------------------------------------------ */
static void q45_k_sb(const f32 *x, const f32 *qw, int nmax, uint8_t *out) {
    f32 w[QK_K], L[QK_K], sc[8], mn[8], steps[37];
    int64_t ls[8], lm[8];
    uint16_t d16, m16;
    if (!qw) {
        int ns = nmax == 15 ? qkx_steps(-1.0f, 0.1f, 20, 15, steps) : qkx_steps(-0.5f, 0.1f, 15, 31, steps);
        for (int g = 0; g < 8; g++) {
            const f32 *xg = x + 32 * g;
            f32 t[32];
            for (int i = 0; i < 32; i++) t[i] = xg[i] * xg[i];
            f32 av_x = sqrtf(tsum32(t) / 32.0f);
            for (int i = 0; i < 32; i++) w[32 * g + i] = av_x + fabsf(xg[i]);
            sc[g] = make_qkx(xg, w + 32 * g, 32, steps, ns, nmax, 0, &mn[g], L + 32 * g);
        }
        f32 max_scale = maxv(sc, 8), max_min = maxv(mn, 8);
        f32 inv_scale = max_scale > 0.0f ? rcp(max_scale) * 63.0f : 0.0f;
        f32 inv_min = max_min > 0.0f ? rcp(max_min) * 63.0f : 0.0f;
        for (int g = 0; g < 8; g++) {
            int64_t a = (int64_t)rnd(inv_scale * sc[g]) & 0xFF;
            int64_t b = (int64_t)rnd(inv_min * mn[g]) & 0xFF;
            ls[g] = a > 63 ? 63 : a;
            lm[g] = b > 63 ? 63 : b;
        }
        d16 = f16_bits(max_scale / 63.0f);
        m16 = f16_bits(max_min / 63.0f);
    } else {
        int ns = qkx_steps(-0.9f, 0.05f, 36, nmax, steps);
        f32 sw[8], lsf[8], lmf[8], qps[8];
        imat_weights(x, qw, 2.0f, 0, w);
        for (int g = 0; g < 8; g++)
            sc[g] = make_qkx(x + 32 * g, w + 32 * g, 32, steps, ns, nmax, 0, &mn[g], L + 32 * g);
        for (int g = 0; g < 8; g++) sw[g] = tsum32(w + 32 * g);
        qp_steps(63, qps);
        f32 d_blk = make_qp(sc, sw, 8, 63, qps, lsf);
        f32 m_blk = make_qp(mn, sw, 8, 63, qps, lmf);
        for (int g = 0; g < 8; g++) { ls[g] = (int64_t)lsf[g] & 0xFF; lm[g] = (int64_t)lmf[g] & 0xFF; }
        d16 = f16_bits(d_blk);
        m16 = f16_bits(m_blk);
    }
    int Lf[QK_K];
    f32 dd = f16_val(d16), dm = f16_val(m16);
    for (int g = 0; g < 8; g++) {
        f32 dg = dd * (f32)(ls[g] & 63);
        f32 mg = dm * (f32)(lm[g] & 63);
        for (int i = 0; i < 32; i++) {
            int e = 32 * g + i;
            Lf[e] = (int)(dg != 0.0f ? clampf(rnd((x[e] + mg) / dg), 0.0f, (f32)nmax) : L[e]);
        }
    }
    put16(out, d16);
    put16(out + 2, m16);
    uint8_t *scb = out + 4;
    for (int j = 0; j < 4; j++) {
        scb[j] = (uint8_t)(ls[j] | ((ls[4 + j] >> 4) << 6));
        scb[4 + j] = (uint8_t)(lm[j] | ((lm[4 + j] >> 4) << 6));
        scb[8 + j] = (uint8_t)((ls[4 + j] & 0xF) | ((lm[4 + j] & 0xF) << 4));
    }
    uint8_t *qs = out + 16;
    if (nmax == 31) {
        uint8_t *qh = out + 16;
        qs = out + 48;
        for (int l = 0; l < 32; l++) {
            int v = 0;
            for (int s = 0; s < 8; s++) v += (Lf[32 * s + l] >> 4) << s;
            qh[l] = (uint8_t)v;
        }
    }
    for (int j = 0; j < 4; j++)
        for (int l = 0; l < 32; l++)
            qs[32 * j + l] = (uint8_t)((Lf[64 * j + l] & 0xF) | ((Lf[64 * j + 32 + l] & 0xF) << 4));
}

/* ------------------------------------------------------------------ */
/* Q2_K (q2_k.py:25-81)                                                 */
/* ------------------------------------------------------------------ */
static void q2_k_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    f32 w[QK_K], L[QK_K], sc[16], mn[16], steps[37];
    int64_t ls[16], lm[16];
    uint16_t d16, m16;
    if (!qw) {
        int ns = qkx_steps(-0.5f, 0.1f, 15, 3, steps);
        for (int i = 0; i < QK_K; i++) w[i] = fabsf(x[i]);
        for (int g = 0; g < 16; g++)
            sc[g] = make_qkx(x + 16 * g, w + 16 * g, 16, steps, ns, 3, 1, &mn[g], L + 16 * g);
        f32 max_scale = maxv(sc, 16), max_min = maxv(mn, 16);
        int pos_s = max_scale > 0.0f, pos_m = max_min > 0.0f;
        f32 inv_scale = pos_s ? 15.0f / max_scale : 0.0f;
        f32 inv_min = pos_m ? 15.0f / max_min : 0.0f;
        for (int g = 0; g < 16; g++) {
            ls[g] = (int64_t)rnd(inv_scale * sc[g]) & 0xFF;
            lm[g] = (int64_t)rnd(inv_min * mn[g]) & 0xFF;
        }
        d16 = f16_bits(pos_s ? max_scale / 15.0f : 0.0f);
        m16 = f16_bits(pos_m ? max_min / 15.0f : 0.0f);
    } else {
        int ns = qkx_steps(-0.9f, 0.05f, 36, 3, steps);
        f32 sw[16], lsf[16], lmf[16], qps[8];
        imat_weights(x, qw, 1.0f, 0, w);
        for (int g = 0; g < 16; g++)
            sc[g] = make_qkx(x + 16 * g, w + 16 * g, 16, steps, ns, 3, 0, &mn[g], L + 16 * g);
        for (int g = 0; g < 16; g++) sw[g] = tsum16(w + 16 * g);
        qp_steps(15, qps);
        f32 d_blk = make_qp(sc, sw, 16, 15, qps, lsf);
        f32 m_blk = make_qp(mn, sw, 16, 15, qps, lmf);
        for (int g = 0; g < 16; g++) { ls[g] = (int64_t)lsf[g] & 0xFF; lm[g] = (int64_t)lmf[g] & 0xFF; }
        d16 = f16_bits(d_blk);
        m16 = f16_bits(m_blk);
    }
    int scb[16], Lf[QK_K];
    f32 dd = f16_val(d16), dm = f16_val(m16);
    for (int g = 0; g < 16; g++) {
        scb[g] = (int)((ls[g] | (lm[g] << 4)) & 0xFF);
        f32 dg = dd * (f32)(scb[g] & 0xF);
        f32 mg = dm * (f32)(scb[g] >> 4);
        for (int i = 0; i < 16; i++) {
            int e = 16 * g + i;
            Lf[e] = (int)(dg != 0.0f ? clampf(rnd((x[e] + mg) / dg), 0.0f, 3.0f) : L[e]);
        }
    }
    for (int g = 0; g < 16; g++) out[g] = (uint8_t)scb[g];
    for (int h = 0; h < 2; h++)
        for (int l = 0; l < 32; l++) {
            const int *q = Lf + 128 * h;
            out[16 + 32 * h + l] = (uint8_t)(q[l] | (q[32 + l] << 2) | (q[64 + l] << 4) | (q[96 + l] << 6));
        }
    put16(out + 80, d16);
    put16(out + 82, m16);
}

/* ------------------------------------------------------------------ */
/* IQ4_XS (iq4_xs.py:35-188)                                            */
/* ------------------------------------------------------------------ */
static const f32 KV_IQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

static int best_index_iq4(f32 al) { /* _best_index: searchsorted(right) then midpoint compare */
    int mu = 0;
    while (mu < 16 && KV_IQ4NL[mu] <= al) mu++;
    mu = mu < 1 ? 1 : (mu > 15 ? 15 : mu);
    f32 lo = KV_IQ4NL[mu - 1], hi = KV_IQ4NL[mu];
    return (al - lo < hi - al) ? mu - 1 : mu;
}

static f32 iq4_search(const f32 *xb, const f32 *w) {
    f32 amax, mx, t[32], q[32];
    absmax_first(xb, 32, &amax, &mx); /* argmax |x| keeps the first hit */
    int live = fabsf(mx) >= EPS15;
    f32 mxs = live ? mx : 1.0f;
    f32 d0 = -mxs / -127.0f;
    f32 id0 = rcp(d0);
    for (int i = 0; i < 32; i++) q[i] = KV_IQ4NL[best_index_iq4(id0 * xb[i])];
    for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * xb[i];
    f32 sumqx = seq_sum(t, 32);
    for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
    f32 sumq2 = seq_sum(t, 32);
    f32 d = sumq2 > 0.0f ? sumqx / sumq2 : 0.0f;
    f32 best = d * sumqx;
    f32 r = rcp(mxs);
    for (int itry = -7; itry <= 7; itry++) {
        f32 idv = r * (f32)(itry - 127);
        for (int i = 0; i < 32; i++) q[i] = KV_IQ4NL[best_index_iq4(idv * xb[i])];
        for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * xb[i];
        sumqx = seq_sum(t, 32);
        for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
        sumq2 = seq_sum(t, 32);
        if ((sumq2 > 0.0f) && (sumqx * sumqx > best * sumq2)) {
            f32 nd = sumqx / sumq2;
            d = nd;
            best = nd * sumqx;
        }
    }
    return live ? d : 0.0f;
}

static void iq4_xs_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    f32 w[QK_K], sc[8];
    if (qw) imat_weights(x, qw, 2.0f, 0, w);
    else for (int i = 0; i < QK_K; i++) w[i] = x[i] * x[i];
    for (int b = 0; b < 8; b++) sc[b] = iq4_search(x + 32 * b, w + 32 * b);
    f32 amax, max_scale;
    absmax_first(sc, 8, &amax, &max_scale);
    f32 d = -max_scale / 32.0f;
    f32 idq = d != 0.0f ? rcp(d) : 0.0f;
    int lsq[8], L[QK_K];
    for (int b = 0; b < 8; b++) {
        f32 ls = clampf(rnd(idq * sc[b]), -32.0f, 31.0f);
        f32 dl = d * ls;
        f32 idl = dl != 0.0f ? rcp(dl) : 0.0f;
        for (int i = 0; i < 32; i++) L[32 * b + i] = best_index_iq4(idl * x[32 * b + i]);
        lsq[b] = (int)(ls + 32.0f);
    }
    put16(out, f16_bits(d));
    int hbits = 0;
    for (int b = 0; b < 8; b++) hbits += (lsq[b] >> 4) << (2 * b);
    out[2] = (uint8_t)(hbits & 0xFF);
    out[3] = (uint8_t)(hbits >> 8);
    for (int j = 0; j < 4; j++) out[4 + j] = (uint8_t)((lsq[2 * j] & 0xF) | ((lsq[2 * j + 1] & 0xF) << 4));
    for (int b = 0; b < 8; b++)
        for (int l = 0; l < 16; l++) out[8 + 16 * b + l] = (uint8_t)(L[32 * b + l] | (L[32 * b + 16 + l] << 4));
}

/* ------------------------------------------------------------------ */
/* IQ grids: kmap + neighbour lists (iq2.py:31-74, iq2xs_common.py:41-95, */
/* iq3_common.py:29-68)                                                 */
/* ------------------------------------------------------------------ */
typedef struct {
    int grid_size, bits, npos, kmap_size;
    const uint16_t *codes;
    int32_t *kmap;      /* code -> grid index or -1 */
    int32_t *off;       /* code -> first list entry */
    int32_t *len;       /* code -> list length (on-grid codes: 1, themselves) */
    int16_t *list;      /* grid indices ordered by (distance, index) */
    f32 *gv;            /* grid values 2l+1, grid_size x npos */
} grid_t;

static grid_t G_IQ2XXS, G_IQ2XS, G_IQ2S, G_IQ3XXS, G_IQ3S;

static int cmp_d2idx(const void *a, const void *b) {
    const int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return x < y ? -1 : x > y;
}

static void grid_build(grid_t *g, const uint16_t *codes, int grid_size, int bits, int npos, int nwant) {
    int mask = (1 << bits) - 1;
    g->grid_size = grid_size;
    g->bits = bits;
    g->npos = npos;
    g->codes = codes;
    g->kmap_size = bits == 2 ? 43692 : 4096;
    g->kmap = malloc(sizeof(int32_t) * g->kmap_size);
    g->off = calloc(g->kmap_size, sizeof(int32_t));
    g->len = calloc(g->kmap_size, sizeof(int32_t));
    g->gv = malloc(sizeof(f32) * grid_size * npos);
    for (int i = 0; i < g->kmap_size; i++) g->kmap[i] = -1;
    for (int i = 0; i < grid_size; i++) {
        g->kmap[codes[i]] = i;
        for (int j = 0; j < npos; j++) g->gv[i * npos + j] = (f32)(2 * ((codes[i] >> (bits * j)) & mask) + 1);
    }
    int64_t *keys = malloc(sizeof(int64_t) * grid_size);
    int cap = 1 << 20, used = 0;
    g->list = malloc(sizeof(int16_t) * cap);
    for (int c = 0; c < g->kmap_size; c++) {
        g->off[c] = used;
        if (g->kmap[c] >= 0) {
            g->list[used++] = (int16_t)g->kmap[c];
            g->len[c] = 1;
            continue;
        }
        /* 2-bit sweeps clamp levels to 0..2, so codes with a level 3 are never looked up */
        int reachable = 1;
        for (int j = 0; j < npos && bits == 2; j++) reachable &= ((c >> (2 * j)) & 3) != 3;
        if (!reachable) continue;
        for (int i = 0; i < grid_size; i++) {
            int d2 = 0;
            for (int j = 0; j < npos; j++) {
                int p = 2 * ((c >> (bits * j)) & mask) + 1;
                int dv = p - (int)g->gv[i * npos + j];
                d2 += dv * dv;
            }
            keys[i] = (int64_t)d2 * 65536 + i;
        }
        qsort(keys, grid_size, sizeof(int64_t), cmp_d2idx);
        int ndist = 0, n = 0;
        int64_t prev = -1;
        for (int i = 0; i < grid_size; i++) {
            int64_t d2 = keys[i] / 65536;
            if (d2 != prev) { ndist++; prev = d2; }
            if (ndist > nwant) break;
            n++;
        }
        for (int i = 0; i < n; i++) g->list[used++] = (int16_t)(keys[i] % 65536);
        g->len[c] = n;
    }
    free(keys);
}

#include "iq_grids.h"

static void init_steps(void);
static int g_tables_ready = 0;
void oq_init(void) {
    if (g_tables_ready) return;
    init_steps();
    grid_build(&G_IQ2XXS, KGRID_2BIT_256, 256, 2, 8, 2);
    grid_build(&G_IQ2XS, KGRID_2BIT_512, 512, 2, 8, 2);
    grid_build(&G_IQ2S, KGRID_2BIT_1024, 1024, 2, 8, 1);
    grid_build(&G_IQ3XXS, KGRID_3BIT_256, 256, 3, 4, 2);
    grid_build(&G_IQ3S, KGRID_3BIT_512, 512, 3, 4, 3);
    g_tables_ready = 1;
}

/* best grid index for one subgroup: kmap hit, else first minimum of the weighted
 * error over the neighbour list (iq2.py:347-372, iq3_common.py:209-234) */
static int grid_project(const grid_t *g, int code, const f32 *xv, const f32 *wv, f32 sc) {
    if (g->kmap[code] >= 0) return g->kmap[code];
    int o = g->off[code], n = g->len[code];
    f32 best = INFINITY;
    int bi = 0;
    for (int t = 0; t < n; t++) {
        int gi = g->list[o + t];
        const f32 *gv = g->gv + gi * g->npos;
        f32 d2;
        if (g->npos == 8) {
            f32 tt[8];
            for (int j = 0; j < 8; j++) { f32 df = sc * gv[j] - xv[j]; tt[j] = (wv[j] * df) * df; }
            d2 = tsum8(tt);
        } else {
            f32 tt[4];
            for (int j = 0; j < 4; j++) { f32 df = sc * gv[j] - xv[j]; tt[j] = (wv[j] * df) * df; }
            d2 = ((tt[0] + tt[1]) + tt[2]) + tt[3];
        }
        if (t == 0 || d2 < best) { best = d2; bi = gi; }
    }
    return bi;
}

/* tentative level code of one subgroup: clamp(round(0.5*(inv*x - 1)), 0, maxl) */
static int level_code(const f32 *xv, int npos, int bits, f32 inv, f32 maxl) {
    int u = 0;
    for (int j = 0; j < npos; j++) {
        int l = (int)clampf(rnd(0.5f * (inv * xv[j] - 1.0f)), 0.0f, maxl);
        u |= l << (bits * j);
    }
    return u;
}

/* sign-parity fold shared by IQ2_XXS/XS and IQ3_XXS (iq2.py:439-449) */
static int parity_fold(const f32 *x, const f32 *w, f32 *xval) {
    int s = 0, nneg = 0;
    for (int j = 0; j < 8; j++) {
        xval[j] = fabsf(x[j]);
        if (x[j] < 0.0f) { s |= 1 << j; nneg++; }
    }
    if (nneg & 1) {
        int imin = 0;
        f32 m = (w[0] * x[0]) * x[0];
        for (int j = 1; j < 8; j++) {
            f32 v = (w[j] * x[j]) * x[j];
            if (v < m) { m = v; imin = j; }
        }
        xval[imin] = -xval[imin];
        s ^= 1 << imin;
    }
    return s & 127;
}

/* ------------------------------------------------------------------ */
/* IQ2_XXS (iq2.py:418-498 + _finalize :87-108)                         */
/* ------------------------------------------------------------------ */
static void iq2_xxs_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    const grid_t *g = &G_IQ2XXS;
    f32 weight[QK_K];
    imat_weights(x, qw, 1.0f, 0, weight);
    uint32_t q2lo[8], q2hi[8];
    f32 scales[8];
    f32 qp4[8];
    { int j = 0; for (int s = -4; s <= 4; s++) if (s) qp4[j++] = (f32)(0.1 * s + 4.0); }
    for (int gr = 0; gr < 8; gr++) {
        const f32 *xb = x + 32 * gr, *w = weight + 32 * gr;
        f32 waux[32], xval[32], t[32], Lqp[32];
        int bs[4];
        for (int i = 0; i < 32; i++) waux[i] = sqrtf(w[i]);
        for (int s = 0; s < 4; s++) bs[s] = parity_fold(xb + 8 * s, w + 8 * s, xval + 8 * s);
        f32 gmax = maxv(xval, 32);
        int active = gmax >= EPS15;
        f32 scale0 = make_qp(xval, w, 32, 4, qp4, Lqp);
        f32 eff_max = scale0 * 3.0f;
        active = active && eff_max > 0.0f;
        f32 eff_safe = active ? eff_max : 1.0f;
        f32 scale = scale0, best = 0.0f;
        int L[32] = {0}, La[32];
        f32 re = rcp(eff_safe);
        for (int step = -6; step <= 6; step++) {
            f32 inv = re * (f32)(5.0 + 0.1 * step);
            f32 sc = rcp(inv);
            for (int s = 0; s < 4; s++) {
                int u = level_code(xval + 8 * s, 8, 2, inv, 2.0f);
                int gi = grid_project(g, u, xval + 8 * s, waux + 8 * s, sc);
                for (int j = 0; j < 8; j++) La[8 * s + j] = (g->codes[gi] >> (2 * j)) & 3;
            }
            f32 q[32];
            for (int i = 0; i < 32; i++) q[i] = (f32)(2 * La[i] + 1);
            for (int i = 0; i < 32; i++) t[i] = (w[i] * xval[i]) * q[i];
            f32 sumqx = tsum32(t);
            for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
            f32 sumq2 = tsum32(t);
            if (active && sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                f32 ns = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
                scale = ns;
                best = ns * sumqx;
                memcpy(L, La, sizeof(L));
            }
        }
        int proj = active && scale > 0.0f;
        f32 inv = rcp(proj ? scale : 1.0f);
        int Lp[32];
        for (int s = 0; s < 4; s++) {
            int u = level_code(xval + 8 * s, 8, 2, inv, 2.0f);
            int gi = grid_project(g, u, xval + 8 * s, waux + 8 * s, scale);
            for (int j = 0; j < 8; j++) Lp[8 * s + j] = (g->codes[gi] >> (2 * j)) & 3;
        }
        f32 q[32];
        for (int i = 0; i < 32; i++) q[i] = (f32)(2 * Lp[i] + 1);
        for (int i = 0; i < 32; i++) t[i] = (w[i] * xval[i]) * q[i];
        f32 sumqx = tsum32(t);
        for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
        f32 sumq2 = tsum32(t);
        if (proj && sumq2 > 0.0f) scale = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
        if (proj) memcpy(L, Lp, sizeof(L));
        if (active && scale < 0.0f) {
            scale = -scale;
            for (int s = 0; s < 4; s++) bs[s] = (~bs[s]) & 127;
        }
        uint32_t lo = 0, hi = 0;
        for (int s = 0; s < 4; s++) {
            int u = 0;
            for (int j = 0; j < 8; j++) u |= L[8 * s + j] << (2 * j);
            int gi = g->kmap[u] < 0 ? 0 : g->kmap[u];
            lo |= (uint32_t)gi << (8 * s);
            hi |= (uint32_t)bs[s] << (7 * s);
        }
        q2lo[gr] = active ? lo : 0;
        q2hi[gr] = active ? hi : 0;
        scales[gr] = active ? scale : 0.0f;
    }
    f32 max_scale = maxv(scales, 8);
    int has = max_scale > 0.0f;
    f32 d = max_scale / 31.0f;
    put16(out, f16_bits(has ? d : 0.0f));
    f32 inv_d = rcp(has ? d : 1.0f);
    for (int gr = 0; gr < 8; gr++) {
        uint32_t lnib = (uint32_t)clampf(rnd(0.5f * (inv_d * scales[gr] - 1.0f)), 0.0f, 15.0f);
        uint32_t lo = has ? q2lo[gr] : 0, hi = has ? (q2hi[gr] | (lnib << 28)) : 0;
        for (int b = 0; b < 4; b++) {
            out[2 + 8 * gr + b] = (uint8_t)(lo >> (8 * b));
            out[2 + 8 * gr + 4 + b] = (uint8_t)(hi >> (8 * b));
        }
    }
}

/* ------------------------------------------------------------------ */
/* IQ2_XS / IQ2_S shared per-16 search (iq2xs_common.py:280-355)        */
/* ------------------------------------------------------------------ */
static f32 SWEEP_CS_IQ2[19], STEPS_IQ3XXS[31], STEPS_IQ3S[19];

static void init_steps(void) {
    for (int s = -9; s <= 9; s++) SWEEP_CS_IQ2[s + 9] = 5.0f + (f32)s * 0.1f;   /* iq2xs_common.py:21 */
    for (int s = -15; s <= 15; s++) STEPS_IQ3XXS[s + 15] = 15.0f + (f32)s * 0.2f; /* iq3_xxs.py:22 */
    for (int s = -9; s <= 9; s++) STEPS_IQ3S[s + 9] = 15.0f + (f32)s * 0.2f;     /* iq3_s.py:22 */
}

/* returns the scale; win[2] grid indices */
static f32 iq2_scale_search(const grid_t *g, const f32 *xval, const f32 *w, const f32 *waux, int active, int *win) {
    const f32 *cs = SWEEP_CS_IQ2;
    f32 gmax = maxv(xval, 16);
    f32 gsafe = active ? gmax : 1.0f;
    f32 r = rcp(gsafe);
    f32 t[16], q[16];
    int code0 = g->kmap[0] >= 0 ? g->kmap[0] : 0;
    f32 scale = active ? gmax / 5.0f : 0.0f, best = 0.0f;
    win[0] = win[1] = code0;
    int og[2] = {1, 1};
    for (int st = 0; st < 19; st++) {
        f32 inv = r * cs[st];
        f32 sc = rcp(inv);
        int ws[2], os[2];
        for (int s = 0; s < 2; s++) {
            int u = level_code(xval + 8 * s, 8, 2, inv, 2.0f);
            os[s] = g->kmap[u] >= 0;
            ws[s] = grid_project(g, u, xval + 8 * s, waux + 8 * s, sc);
        }
        for (int i = 0; i < 16; i++) q[i] = g->gv[ws[i >> 3] * 8 + (i & 7)];
        for (int i = 0; i < 16; i++) t[i] = (w[i] * xval[i]) * q[i];
        f32 sumqx = tree_sum(t, 16);
        for (int i = 0; i < 16; i++) t[i] = (w[i] * q[i]) * q[i];
        f32 sumq2 = tree_sum(t, 16);
        if (active && sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
            f32 ns = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
            scale = ns;
            best = ns * sumqx;
            win[0] = ws[0]; win[1] = ws[1];
            og[0] = os[0]; og[1] = os[1];
        }
    }
    int need = active && scale > 0.0f && !(og[0] && og[1]);
    if (need) {
        f32 inv = rcp(scale > 0.0f ? scale : 1.0f);
        for (int s = 0; s < 2; s++) {
            if (og[s]) continue;
            int u = level_code(xval + 8 * s, 8, 2, inv, 2.0f);
            win[s] = grid_project(g, u, xval + 8 * s, waux + 8 * s, scale);
        }
        for (int i = 0; i < 16; i++) q[i] = g->gv[win[i >> 3] * 8 + (i & 7)];
        for (int i = 0; i < 16; i++) t[i] = (w[i] * xval[i]) * q[i];
        f32 sumqx = tree_sum(t, 16);
        for (int i = 0; i < 16; i++) t[i] = (w[i] * q[i]) * q[i];
        f32 sumq2 = tree_sum(t, 16);
        if (sumq2 > 0.0f) scale = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
    }
    return scale;
}

/* pack_scales (iq2xs_common.py:345-355) */
static int iq2_pack_scales(const f32 *sc16, f32 *d, uint8_t *sbytes) {
    f32 max_scale = maxv(sc16, 16);
    int has = max_scale > 0.0f;
    *d = max_scale / 31.0f;
    f32 inv_d = rcp(has ? *d : 1.0f);
    int l[16];
    for (int i = 0; i < 16; i++) l[i] = has ? (int)clampf(rnd(0.5f * (inv_d * sc16[i] - 1.0f)), 0.0f, 15.0f) : 0;
    for (int j = 0; j < 8; j++) sbytes[j] = (uint8_t)(l[2 * j] | (l[2 * j + 1] << 4));
    return has;
}

static void iq2_xs_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    const grid_t *g = &G_IQ2XS;
    f32 weight[QK_K], sc16[16];
    uint32_t q2[32];
    imat_weights(x, qw, 1.0f, 0, weight);
    for (int gr = 0; gr < 16; gr++) {
        const f32 *xb = x + 16 * gr, *w = weight + 16 * gr;
        f32 waux[16], xval[16];
        int signs[2], win[2];
        for (int i = 0; i < 16; i++) waux[i] = sqrtf(w[i]);
        for (int s = 0; s < 2; s++) signs[s] = parity_fold(xb + 8 * s, w + 8 * s, xval + 8 * s);
        int active = maxv(xval, 16) >= EPS15;
        f32 scale = iq2_scale_search(g, xval, w, waux, active, win);
        if (active && scale < 0.0f) {
            scale = -scale;
            signs[0] = (~signs[0]) & 127;
            signs[1] = (~signs[1]) & 127;
        }
        for (int s = 0; s < 2; s++) q2[2 * gr + s] = active ? (uint32_t)(win[s] | (signs[s] << 9)) : 0;
        sc16[gr] = active ? scale : 0.0f;
    }
    f32 d;
    int has = iq2_pack_scales(sc16, &d, out + 66);
    put16(out, f16_bits(has ? d : 0.0f));
    for (int j = 0; j < 32; j++) {
        uint32_t v = has ? q2[j] : 0;
        out[2 + 2 * j] = (uint8_t)v;
        out[3 + 2 * j] = (uint8_t)(v >> 8);
    }
}

static void iq2_s_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    const grid_t *g = &G_IQ2S;
    f32 weight[QK_K], sc16[16];
    int wins[32], sgn[32];
    imat_weights(x, qw, 2.0f, 0, weight);
    for (int gr = 0; gr < 16; gr++) {
        const f32 *xb = x + 16 * gr, *w = weight + 16 * gr;
        f32 waux[16], xval[16];
        int signs[2] = {0, 0}, win[2];
        for (int i = 0; i < 16; i++) {
            waux[i] = sqrtf(w[i]);
            xval[i] = fabsf(xb[i]);
            if (xb[i] < 0.0f) signs[i >> 3] |= 1 << (i & 7);
        }
        int active = maxv(xval, 16) >= EPS8;
        f32 scale = iq2_scale_search(g, xval, w, waux, active, win);
        if (active && scale < 0.0f) {
            scale = -scale;
            signs[0] = (~signs[0]) & 255;
            signs[1] = (~signs[1]) & 255;
        }
        for (int s = 0; s < 2; s++) {
            wins[2 * gr + s] = active ? win[s] : 0;
            sgn[2 * gr + s] = active ? signs[s] : 0;
        }
        sc16[gr] = active ? scale : 0.0f;
    }
    f32 d;
    int has = iq2_pack_scales(sc16, &d, out + 74);
    put16(out, f16_bits(has ? d * 0.9875f : 0.0f));
    for (int j = 0; j < 32; j++) {
        out[2 + j] = (uint8_t)(wins[j] & 255);
        out[34 + j] = (uint8_t)sgn[j];
    }
    for (int j = 0; j < 8; j++) {
        int v = 0;
        for (int t = 0; t < 4; t++) v += (wins[4 * j + t] >> 8) << (2 * t);
        out[66 + j] = (uint8_t)v;
    }
}

/* ------------------------------------------------------------------ */
/* IQ3_XXS / IQ3_S (iq3_xxs.py:31-134, iq3_s.py:31-140)                 */
/* ------------------------------------------------------------------ */
/* per-32 search; returns scale, Wg[8] grid indices */
static f32 iq3_group(const grid_t *g, const f32 *xval, const f32 *w, const f32 *waux, int active,
                     const f32 *steps, int nsteps, int og_init, int redo_all, int *Wg) {
    f32 gmax = maxv(xval, 32);
    f32 gsafe = active ? gmax : 1.0f;
    f32 r = rcp(gsafe);
    f32 t[32], q[32];
    f32 scale = gmax / 15.0f, best = 0.0f;
    int og[8];
    for (int s = 0; s < 8; s++) { Wg[s] = 0; og[s] = og_init; }
    for (int st = 0; st < nsteps; st++) {
        f32 inv = r * steps[st];
        f32 sc = rcp(inv);
        int ws[8], os[8];
        for (int s = 0; s < 8; s++) {
            int u = level_code(xval + 4 * s, 4, 3, inv, 7.0f);
            os[s] = g->kmap[u] >= 0;
            ws[s] = grid_project(g, u, xval + 4 * s, waux + 4 * s, sc);
        }
        for (int i = 0; i < 32; i++) q[i] = g->gv[ws[i >> 2] * 4 + (i & 3)];
        for (int i = 0; i < 32; i++) t[i] = (w[i] * xval[i]) * q[i];
        f32 sumqx = tree_sum(t, 32);
        for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
        f32 sumq2 = tree_sum(t, 32);
        if (active && sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
            f32 ns = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
            scale = ns;
            best = ns * sumqx;
            memcpy(Wg, ws, sizeof(ws));
            memcpy(og, os, sizeof(os));
        }
    }
    int anyoff = 0;
    for (int s = 0; s < 8; s++) anyoff |= !og[s];
    int redo = active && anyoff && scale > 0.0f;
    if (redo) {
        f32 inv2 = rcp(scale);
        for (int s = 0; s < 8; s++) {
            if (!redo_all && og[s]) continue;
            int u = level_code(xval + 4 * s, 4, 3, inv2, 7.0f);
            Wg[s] = grid_project(g, u, xval + 4 * s, waux + 4 * s, scale);
        }
        for (int i = 0; i < 32; i++) q[i] = g->gv[Wg[i >> 2] * 4 + (i & 3)];
        for (int i = 0; i < 32; i++) t[i] = (w[i] * xval[i]) * q[i];
        f32 sumqx = tree_sum(t, 32);
        for (int i = 0; i < 32; i++) t[i] = (w[i] * q[i]) * q[i];
        f32 sumq2 = tree_sum(t, 32);
        if (sumq2 > 0.0f) scale = sumqx / (sumq2 < F32_TINY ? F32_TINY : sumq2);
    }
    return scale;
}

static void iq3_weights(const f32 *x, const f32 *qw, f32 *w) {
    if (qw) imat_weights(x, qw, 2.0f, 0, w);
    else for (int i = 0; i < QK_K; i++) w[i] = x[i] * x[i];
}

static void iq3_xxs_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    const grid_t *g = &G_IQ3XXS;
    const f32 *steps = STEPS_IQ3XXS;
    f32 weight[QK_K], scales[8];
    int Wg[8][8];
    uint32_t sw[8];
    iq3_weights(x, qw, weight);
    for (int gr = 0; gr < 8; gr++) {
        const f32 *xb = x + 32 * gr, *w = weight + 32 * gr;
        f32 waux[32], xval[32];
        int bs[4];
        for (int i = 0; i < 32; i++) waux[i] = sqrtf(w[i]);
        for (int s = 0; s < 4; s++) bs[s] = parity_fold(xb + 8 * s, w + 8 * s, xval + 8 * s);
        int active = maxv(xval, 32) >= EPS8;
        f32 scale = iq3_group(g, xval, w, waux, active, steps, 31, 1, 0, Wg[gr]);
        if (active && scale < 0.0f) {
            scale = -scale;
            for (int s = 0; s < 4; s++) bs[s] = (~bs[s]) & 127;
        }
        uint32_t v = 0;
        for (int s = 0; s < 4; s++) v |= (uint32_t)bs[s] << (7 * s);
        sw[gr] = active ? v : 0;
        scales[gr] = active ? scale : 0.0f;
        if (!active) for (int s = 0; s < 8; s++) Wg[gr][s] = 0;
    }
    f32 max_scale = maxv(scales, 8);
    int has = max_scale > 0.0f;
    f32 d = max_scale / 31.0f;
    put16(out, f16_bits(has ? d * 1.0125f : 0.0f));
    f32 inv_d = rcp(has ? d : 1.0f);
    for (int gr = 0; gr < 8; gr++) {
        uint32_t lnib = (uint32_t)clampf(rnd(0.5f * (inv_d * scales[gr] - 1.0f)), 0.0f, 15.0f);
        uint32_t word = has ? (sw[gr] | (lnib << 28)) : 0;
        for (int s = 0; s < 8; s++) out[2 + 8 * gr + s] = has ? (uint8_t)Wg[gr][s] : 0;
        for (int b = 0; b < 4; b++) out[66 + 4 * gr + b] = (uint8_t)(word >> (8 * b));
    }
}

static void iq3_s_sb(const f32 *x, const f32 *qw, uint8_t *out) {
    const grid_t *g = &G_IQ3S;
    const f32 *steps = STEPS_IQ3S;
    f32 weight[QK_K], scales[8];
    int Wg[8][8], act[8], bs[8][4];
    iq3_weights(x, qw, weight);
    for (int gr = 0; gr < 8; gr++) {
        const f32 *xb = x + 32 * gr, *w = weight + 32 * gr;
        f32 waux[32], xval[32];
        for (int s = 0; s < 4; s++) bs[gr][s] = 0;
        for (int i = 0; i < 32; i++) {
            waux[i] = sqrtf(w[i]);
            xval[i] = fabsf(xb[i]);
            if (xb[i] < 0.0f) bs[gr][i >> 3] |= 1 << (i & 7);
        }
        int active = maxv(xval, 32) > 0.0f;
        f32 scale = iq3_group(g, xval, w, waux, active, steps, 19, 0, 1, Wg[gr]);
        if (active && scale < 0.0f) {
            scale = -scale;
            for (int s = 0; s < 4; s++) bs[gr][s] = (~bs[gr][s]) & 255;
        }
        act[gr] = active;
        scales[gr] = active ? scale : 0.0f;
    }
    uint8_t *qs = out + 2, *qh = out + 66, *sg = out + 74, *scb = out + 106;
    memset(qs, 0, 64);
    memset(sg, 0, 32);
    int slot = 0;
    for (int gr = 0; gr < 8; gr++) {
        int h = 0;
        for (int s = 0; s < 8; s++) h += (Wg[gr][s] >> 8) << s;
        qh[gr] = act[gr] ? (uint8_t)h : 0;
        if (!act[gr]) continue;
        for (int s = 0; s < 8; s++) qs[8 * slot + s] = (uint8_t)(Wg[gr][s] & 255);
        for (int s = 0; s < 4; s++) sg[4 * slot + s] = (uint8_t)bs[gr][s];
        slot++;
    }
    f32 max_scale = maxv(scales, 8);
    int has = max_scale > 0.0f;
    f32 d = max_scale / 31.0f;
    put16(out, f16_bits(has ? d * 1.033f : 0.0f));
    f32 inv_d = rcp(has ? d : 1.0f);
    int ln[8];
    for (int gr = 0; gr < 8; gr++) ln[gr] = has ? (int)clampf(rnd(0.5f * (inv_d * scales[gr] - 1.0f)), 0.0f, 15.0f) : 0;
    for (int j = 0; j < 4; j++) scb[j] = (uint8_t)(ln[2 * j] | (ln[2 * j + 1] << 4));
}

/* ------------------------------------------------------------------ */
/* dispatch                                                             */
/* ------------------------------------------------------------------ */
typedef void (*sb_fn)(const f32 *, const f32 *, uint8_t *);

static int type_info(int type, int *qk, int *bytes, sb_fn *fn, int *needs_qw) {
    *needs_qw = 0;
    switch (type) {
    case OQ_Q4_0: *qk = 32; *bytes = 18; *fn = NULL; return 0;
    case OQ_Q4_1: *qk = 32; *bytes = 20; *fn = NULL; return 0;
    case OQ_Q5_0: *qk = 32; *bytes = 22; *fn = NULL; return 0;
    case OQ_Q5_1: *qk = 32; *bytes = 24; *fn = NULL; return 0;
    case OQ_Q8_0: *qk = 32; *bytes = 34; *fn = NULL; return 0;
    case OQ_Q2_K: *qk = QK_K; *bytes = 84; *fn = q2_k_sb; return 0;
    case OQ_Q3_K: *qk = QK_K; *bytes = 110; *fn = q3_k_sb; return 0;
    case OQ_Q4_K: *qk = QK_K; *bytes = 144; *fn = NULL; return 0;
    case OQ_Q5_K: *qk = QK_K; *bytes = 176; *fn = NULL; return 0;
    case OQ_Q6_K: *qk = QK_K; *bytes = 210; *fn = q6_k_sb; return 0;
    case OQ_IQ2_XXS: *qk = QK_K; *bytes = 66; *fn = iq2_xxs_sb; *needs_qw = 1; return 0;
    case OQ_IQ2_XS: *qk = QK_K; *bytes = 74; *fn = iq2_xs_sb; *needs_qw = 1; return 0;
    case OQ_IQ3_XXS: *qk = QK_K; *bytes = 98; *fn = iq3_xxs_sb; return 0;
    case OQ_IQ3_S: *qk = QK_K; *bytes = 110; *fn = iq3_s_sb; return 0;
    case OQ_IQ2_S: *qk = QK_K; *bytes = 82; *fn = iq2_s_sb; *needs_qw = 1; return 0;
    case OQ_IQ4_XS: *qk = QK_K; *bytes = 136; *fn = iq4_xs_sb; return 0;
    default: return -1;
    }
}

int64_t oq_row_bytes(int type, int64_t k) {
    int qk, bytes, nq;
    sb_fn fn;
    if (type_info(type, &qk, &bytes, &fn, &nq) || k <= 0 || k % qk) return -1;
    return k / qk * bytes;
}

typedef struct {
    int type, qk, bytes;
    sb_fn fn;
    const f32 *x, *qw;
    uint8_t *out;
    int64_t nb_row, nb;
    atomic_llong next;
} job_t;

static void run_block(const job_t *j, int64_t b) {
    const f32 *xb = j->x + b * j->qk;
    const f32 *qb = j->qw ? j->qw + (b % j->nb_row) * j->qk : NULL;
    uint8_t *ob = j->out + b * j->bytes;
    if (j->type == OQ_Q4_0) q4_0_block(xb, ob);
    else if (j->type == OQ_Q4_1) q4_1_block(xb, ob);
    else if (j->type == OQ_Q5_0) q5_0_block(xb, ob);
    else if (j->type == OQ_Q5_1) q5_1_block(xb, ob);
    else if (j->type == OQ_Q8_0) q8_0_block(xb, ob);
    else if (j->type == OQ_Q4_K) q45_k_sb(xb, qb, 15, ob);
    else if (j->type == OQ_Q5_K) q45_k_sb(xb, qb, 31, ob);
    else j->fn(xb, qb, ob);
}

static void *worker(void *arg) {
    job_t *j = arg;
    for (;;) {
        int64_t b0 = atomic_fetch_add(&j->next, 64);
        if (b0 >= j->nb) break;
        int64_t b1 = b0 + 64 < j->nb ? b0 + 64 : j->nb;
        for (int64_t b = b0; b < b1; b++) run_block(j, b);
    }
    return NULL;
}

static pthread_once_t g_once = PTHREAD_ONCE_INIT;

int oq_quantize(int type, const float *x, int64_t n, int64_t k, const float *qw, uint8_t *out, int nthreads) {
    int qk, bytes, needs_qw;
    sb_fn fn;
    if (type_info(type, &qk, &bytes, &fn, &needs_qw) || k <= 0 || k % qk || n < 0) return -1;
    if (needs_qw && !qw) return -2;
    pthread_once(&g_once, oq_init);
    job_t j = {type, qk, bytes, fn, x, qw, out, k / qk, n * (k / qk), 0};
    if (nthreads <= 1) { worker(&j); return 0; }
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    int started = 0;
    for (int i = 0; i < nthreads; i++) if (pthread_create(&th[started], NULL, worker, &j) == 0) started++;
    worker(&j);
    for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
    return 0;
}

/* ------------------------------------------------------------------ */
/* search-core entry points for unit tests of the oracle itself         */
/* ------------------------------------------------------------------ */
float oq_core_qkx(const float *x, const float *w, int n, int nmax, int impl, int use_mad, float *the_min, float *L) {
    f32 steps[37];
    int ns;
    if (impl) ns = qkx_steps(-0.9f, 0.05f, 36, nmax, steps);
    else if (nmax == 15) ns = qkx_steps(-1.0f, 0.1f, 20, 15, steps);
    else ns = qkx_steps(-0.5f, 0.1f, 15, nmax, steps);
    return make_qkx(x, w, n, steps, ns, nmax, use_mad, the_min, L);
}
float oq_core_qp(const float *x, const float *w, int n, int nmax, float *L) {
    f32 steps[8];
    qp_steps(nmax, steps);
    return make_qp(x, w, n, nmax, steps, L);
}
