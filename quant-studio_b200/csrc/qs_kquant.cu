// K-quant (Q2_K..Q6_K) and IQ4_XS kernels for sm_100a.
//
// Layout: one thread per quantization group (16 or 32 values in registers), the
// threads of a superblock are consecutive lanes of one warp, a CTA of 128 or 256 threads
// works on a tile of 16 or 32 superblocks and stages the packed tile in shared
// memory before a coalesced store. Reference for every formula: the eager torch path
// of ngxson/quant-studio kernels/<type>.py (citations per kernel).
#include "qs_kquant.cuh"
#include "qs_kernels.h"

namespace qs {

// ---------------------------------------------------------------------------
// Q2_K / Q4_K / Q5_K (kernels/q2_k.py:25-81, q4_k.py:25-79, q5_k.py:25-82)
// ---------------------------------------------------------------------------
template <int T>
struct QkxTraits;
template <>
struct QkxTraits<QS_Q2_K> { static constexpr int GS = 16, NMAX = 3, BB = 84, QPMAX = 15, THREADS = 256, MIN_CTAS = 2; static constexpr float SIGFAC = 1.0f; };
template <>
struct QkxTraits<QS_Q4_K> { static constexpr int GS = 32, NMAX = 15, BB = 144, QPMAX = 63, THREADS = 128, MIN_CTAS = 3; static constexpr float SIGFAC = 2.0f; };
template <>
struct QkxTraits<QS_Q5_K> { static constexpr int GS = 32, NMAX = 31, BB = 176, QPMAX = 63, THREADS = 128, MIN_CTAS = 3; static constexpr float SIGFAC = 2.0f; };

template <int T, bool IMAT>
__device__ __forceinline__ void qkx_body(const QuantArgs& a, const KParams& p) {
    using Tr = QkxTraits<T>;
    constexpr int GS = Tr::GS, NG = QK_K / GS, SBT = Tr::THREADS / NG, BB = Tr::BB;
    constexpr bool MAD = (T == QS_Q2_K) && !IMAT;
    __shared__ float s_steps[40], s_qp[8];
    __shared__ __align__(16) float s_sq[SBT * QK_K];  // squares, then the SB's level bytes
    __shared__ float s_part[SBT][8];
    __shared__ float s_sc[SBT][NG], s_mn[SBT][NG], s_sw[SBT][NG], s_ls[SBT][NG], s_lm[SBT][NG];
    __shared__ float s_mse[SBT][18];
    __shared__ __align__(16) uint8_t s_out[SBT * BB];

    const int tid = threadIdx.x, sbl = tid / NG, g = tid % NG;
    if (tid < 40) s_steps[tid] = p.steps[tid];
    if (tid < 8) s_qp[tid] = p.qp[tid];
    __syncthreads();
    float* sq = s_sq + sbl * QK_K;
    uint8_t* lev = reinterpret_cast<uint8_t*>(sq);

    for (int64_t tile = blockIdx.x; tile * SBT < a.nblk; tile += gridDim.x) {
        const int64_t b = min(tile * SBT + sbl, a.nblk - 1);  // tail lanes redo the last block
        float x[GS], w[GS], L[GS];
        load_row<GS>(a.src, b * QK_K + g * GS, a.src_type, x);
        if (IMAT) {
            if constexpr (GS == 32) {
                sb_put_sq32(sq, g, x);
                __syncwarp();
                s_part[sbl][g] = sb_sum256_partial32(sq, g);
            } else {
                sb_put_sq16(sq, g, x);
                __syncwarp();
                if (g < 8) s_part[sbl][g] = sb_sum256_partial16(sq, g);
            }
            __syncwarp();
            const float sigma2 = __fdiv_rn(Tr::SIGFAC * sb_sum256_finish(s_part[sbl]), 256.0f);
            float q[GS];
            load_f32<GS>(a.qw + (b % a.nblk_row) * QK_K + g * GS, q);
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = q[i] * sqrtf(sigma2 + x[i] * x[i]);
        } else if (T == QS_Q2_K) {
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = fabsf(x[i]);
        } else {
            float t[GS];
#pragma unroll
            for (int i = 0; i < GS; i++) t[i] = x[i] * x[i];
            const float av_x = sqrtf(__fdiv_rn(torch_sum<GS>(t), 32.0f));
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = av_x + fabsf(x[i]);
        }
        float the_min;
        const float scale = qkx_search<GS, Tr::NMAX, MAD>(x, w, s_steps, p.nsteps, the_min, L);
        s_sc[sbl][g] = scale;
        s_mn[sbl][g] = the_min;
        if (IMAT) s_sw[sbl][g] = torch_sum<GS>(w);
        __syncwarp();

        // superblock scale/min quantization
        uint16_t d16, m16;
        int ls, lm;  // this group's 8-bit codes
        if (IMAT) {
            float La, Lb, da, db;
            qp_pair<NG>(s_sc[sbl], s_mn[sbl], s_sw[sbl], (float)Tr::QPMAX, s_qp, s_mse[sbl], g, La, Lb, da, db);
            s_ls[sbl][g] = La;
            s_lm[sbl][g] = Lb;
            d16 = f16_bits(da);
            m16 = f16_bits(db);
            ls = (int)((long long)La & 0xFF);
            lm = (int)((long long)Lb & 0xFF);
        } else {
            float max_scale = s_sc[sbl][0], max_min = s_mn[sbl][0];
#pragma unroll
            for (int j = 1; j < NG; j++) {
                max_scale = s_sc[sbl][j] > max_scale ? s_sc[sbl][j] : max_scale;
                max_min = s_mn[sbl][j] > max_min ? s_mn[sbl][j] : max_min;
            }
            if (T == QS_Q2_K) {
                const float inv_s = max_scale > 0.0f ? __fdiv_rn(15.0f, max_scale) : 0.0f;
                const float inv_m = max_min > 0.0f ? __fdiv_rn(15.0f, max_min) : 0.0f;
                ls = (int)((long long)rintf(inv_s * scale) & 0xFF);
                lm = (int)((long long)rintf(inv_m * the_min) & 0xFF);
                d16 = f16_bits(max_scale > 0.0f ? __fdiv_rn(max_scale, 15.0f) : 0.0f);
                m16 = f16_bits(max_min > 0.0f ? __fdiv_rn(max_min, 15.0f) : 0.0f);
            } else {
                const float inv_s = max_scale > 0.0f ? rcp_rn(max_scale) * 63.0f : 0.0f;
                const float inv_m = max_min > 0.0f ? rcp_rn(max_min) * 63.0f : 0.0f;
                ls = min((int)((long long)rintf(inv_s * scale) & 0xFF), 63);
                lm = min((int)((long long)rintf(inv_m * the_min) & 0xFF), 63);
                d16 = f16_bits(__fdiv_rn(max_scale, 63.0f));
                m16 = f16_bits(__fdiv_rn(max_min, 63.0f));
            }
            s_ls[sbl][g] = (float)ls;
            s_lm[sbl][g] = (float)lm;
        }

        // requantize with the stored block scales; d == 0 keeps the search levels
        int scb = 0;
        float dg, mg;
        if (T == QS_Q2_K) {
            scb = (ls | (lm << 4)) & 0xFF;
            dg = f16_val(d16) * (float)(scb & 0xF);
            mg = f16_val(m16) * (float)(scb >> 4);
        } else {
            dg = f16_val(d16) * (float)(ls & 63);
            mg = f16_val(m16) * (float)(lm & 63);
        }
        // the group's level bytes as 16-byte stores (GS / 16 per lane)
        uint32_t pk[GS / 4];
#pragma unroll
        for (int i = 0; i < GS / 4; i++) pk[i] = 0u;
#pragma unroll
        for (int i = 0; i < GS; i++) {
            const float q = dg != 0.0f ? clampf(rintf(__fdiv_rn(x[i] + mg, dg)), 0.0f, (float)Tr::NMAX) : L[i];
            pk[i >> 2] |= ((uint32_t)(int)q & 0xFFu) << (8 * (i & 3));
        }
#pragma unroll
        for (int h = 0; h < GS / 16; h++)
            *reinterpret_cast<uint4*>(lev + g * GS + 16 * h) = make_uint4(pk[4 * h], pk[4 * h + 1], pk[4 * h + 2], pk[4 * h + 3]);
        __syncwarp();

        uint8_t* o = s_out + sbl * BB;
        if (T == QS_Q2_K) {
            o[g] = (uint8_t)scb;
            {  // bytes 4g..4g+3: levels l, l + 32, l + 64, l + 96 of half h as 2-bit fields, a word at a time
                const int h = g >> 3, l = (4 * g) & 31;
                const uint32_t* q = reinterpret_cast<const uint32_t*>(lev + 128 * h + l);
                *reinterpret_cast<uint32_t*>(o + 16 + 4 * g) = q[0] | (q[8] << 2) | (q[16] << 4) | (q[24] << 6);
            }
            if (g == 0) {
                o[80] = (uint8_t)d16; o[81] = (uint8_t)(d16 >> 8);
                o[82] = (uint8_t)m16; o[83] = (uint8_t)(m16 >> 8);
            }
        } else {
            if (g == 0) {
                o[0] = (uint8_t)d16; o[1] = (uint8_t)(d16 >> 8);
                o[2] = (uint8_t)m16; o[3] = (uint8_t)(m16 >> 8);
            }
            if (g < 4) {
                const int l0 = (int)s_ls[sbl][g], l4 = (int)s_ls[sbl][4 + g];
                const int m0 = (int)s_lm[sbl][g], m4 = (int)s_lm[sbl][4 + g];
                o[4 + g] = (uint8_t)(l0 | ((l4 >> 4) << 6));
                o[8 + g] = (uint8_t)(m0 | ((m4 >> 4) << 6));
                o[12 + g] = (uint8_t)((l4 & 0xF) | ((m4 & 0xF) << 4));
            }
            int qs0 = 16;
            if (T == QS_Q5_K) {
                qs0 = 48;
                // qh bytes 4g..4g+3: bit s of byte l is bit 4 of level 32 s + l, a word at a time
                uint32_t v = 0u;
#pragma unroll
                for (int s = 0; s < 8; s++) v |= ((*reinterpret_cast<const uint32_t*>(lev + 32 * s + 4 * g) >> 4) & 0x01010101u) << s;
                *reinterpret_cast<uint32_t*>(o + 16 + 4 * g) = v;
            }
            {  // qs bytes 16g..16g+15: low nibbles of levels 64 j + l0 + i and 64 j + 32 + l0 + i
                const int j = g >> 1, l0 = 16 * (g & 1);
                const uint4 a4 = *reinterpret_cast<const uint4*>(lev + 64 * j + l0);
                const uint4 b4 = *reinterpret_cast<const uint4*>(lev + 64 * j + 32 + l0);
                auto nib = [](uint32_t a, uint32_t b) { return (a & 0x0F0F0F0Fu) | ((b & 0x0F0F0F0Fu) << 4); };
                *reinterpret_cast<uint4*>(o + qs0 + 16 * g) =
                    make_uint4(nib(a4.x, b4.x), nib(a4.y, b4.y), nib(a4.z, b4.z), nib(a4.w, b4.w));
            }
        }
        __syncthreads();
        store_tile(a, s_out, tile * SBT, (int)min((int64_t)SBT, a.nblk - tile * SBT), BB, tid, Tr::THREADS);
        __syncthreads();
    }
}

// Q2_K and Q4_K keep the launch bounds of their CTA shape. Q5_K is capped at 152 registers
// (147 used, no spills) instead of the 168 that three CTAs of 128 threads allow: the same
// body then measured 6 % faster (64.4 -> 68.2 GB/s); at 159 registers it executed 734 thread
// instructions per value against Q4_K's 673.
template <int T, bool IMAT>
__global__ void __launch_bounds__(QkxTraits<T>::THREADS, QkxTraits<T>::MIN_CTAS) qkx_kernel(QuantArgs a, KParams p) {
    qkx_body<T, IMAT>(a, p);
}
template <int T, bool IMAT>
__global__ void __maxnreg__(152) qkx_kernel_r152(QuantArgs a, KParams p) {
    qkx_body<T, IMAT>(a, p);
}

// ---------------------------------------------------------------------------
// Q6_K / Q3_K (kernels/q6_k.py:22-65, q3_k.py:23-78): one thread per 16-group
// ---------------------------------------------------------------------------
template <int T, bool IMAT>
__global__ void __launch_bounds__(256) qx_kernel(QuantArgs a, KParams p) {
    constexpr int GS = 16, NG = 16, SBT = 16;
    constexpr int BB = T == QS_Q6_K ? 210 : 110;
    __shared__ float s_qx[18], s_qx2[18];
    __shared__ __align__(16) float s_sq[SBT * QK_K];
    __shared__ float s_sc[SBT][NG], s_sw[SBT][NG], s_ls[SBT][NG];
    __shared__ float s_d[SBT], s_sig[SBT];
    __shared__ __align__(16) uint8_t s_out[SBT * BB];

    const int tid = threadIdx.x, sbl = tid / NG, g = tid % NG;
    if (tid < 18) { s_qx[tid] = p.qx[tid]; s_qx2[tid] = p.qx2[tid]; }
    __syncthreads();
    float* sq = s_sq + sbl * QK_K;
    uint8_t* lev = reinterpret_cast<uint8_t*>(sq);

    for (int64_t tile = blockIdx.x; tile * SBT < a.nblk; tile += gridDim.x) {
        const int64_t b = min(tile * SBT + sbl, a.nblk - 1);
        float x[GS], w[GS], L[GS];
        load_row<GS>(a.src, b * QK_K + g * GS, a.src_type, x);
        const float* qwp = IMAT ? a.qw + (b % a.nblk_row) * QK_K + g * GS : nullptr;
        float scale;
        if (T == QS_Q6_K) {
            if (IMAT) load_f32<GS>(qwp, w);
            else {
#pragma unroll
                for (int i = 0; i < GS; i++) w[i] = x[i] * x[i];
            }
            scale = qx_search<GS>(x, w, 32.0f, s_qx, L);
        } else if (!IMAT) {
            scale = q3_search<GS>(x, 4.0f, L);
        } else {
            // sigma2 = 2 * seq_sum(x*x over 256) / 256: one strict left-to-right chain
#pragma unroll
            for (int i = 0; i < GS; i++) sq[g * GS + i] = x[i] * x[i];
            __syncwarp();
            if (g == 0) {
                float s = sq[0];
                for (int i = 1; i < QK_K; i++) s = __fadd_rn(s, sq[i]);
                s_sig[sbl] = __fdiv_rn(2.0f * s, 256.0f);
            }
            __syncwarp();
            const float sigma2 = s_sig[sbl];
            float q[GS];
            load_f32<GS>(qwp, q);
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = q[i] * sqrtf(sigma2 + x[i] * x[i]);
            scale = qx_search<GS>(x, w, 4.0f, s_qx, L);
            s_sw[sbl][g] = seq_sum<GS>(w);
        }
        s_sc[sbl][g] = scale;
        __syncwarp();

        float sc16[NG];
#pragma unroll
        for (int j = 0; j < NG; j++) sc16[j] = s_sc[sbl][j];
        uint16_t d16;
        int myls;
        bool live = true;
        if (T == QS_Q6_K) {
            float amax, max_scale;
            absmax_first<NG>(sc16, amax, max_scale);
            live = amax >= EPS15;
            const float iscale = rcp_rn(live ? max_scale : 1.0f) * -128.0f;
            d16 = f16_bits(live ? rcp_rn(iscale) : 0.0f);
            long long v = (long long)min_hi(rintf(iscale * scale), 127.0f);
            v = ((v & 0xFF) ^ 0x80) - 0x80;
            myls = live ? (int)v : 0;
        } else if (!IMAT) {
            float amax, max_scale;
            absmax_first<NG>(sc16, amax, max_scale);
            const bool has = max_scale != 0.0f;
            const float iscale = rcp_rn(has ? max_scale : 1.0f) * -32.0f;
            long long l = (long long)rintf(iscale * scale);
            l = ((l & 0xFF) ^ 0x80) - 0x80;
            l = l < -32 ? -32 : (l > 31 ? 31 : l);
            myls = has ? (int)(l + 32) : 0;
            d16 = f16_bits(has ? rcp_rn(iscale) : 0.0f);
        } else {
            if (g == 0) {
                float sw[NG], lv[NG];
#pragma unroll
                for (int j = 0; j < NG; j++) sw[j] = s_sw[sbl][j];
                s_d[sbl] = qx_search<NG>(sc16, sw, 32.0f, s_qx2, lv);
#pragma unroll
                for (int j = 0; j < NG; j++) s_ls[sbl][j] = lv[j];
            }
            __syncwarp();
            d16 = f16_bits(s_d[sbl]);
            myls = (int)s_ls[sbl][g];
        }
        s_ls[sbl][g] = (float)myls;
        __syncwarp();

        // the group's 16 level bytes go to shared memory as one 16-byte store (lanes at a
        // 16-byte stride: no bank conflicts)
        const float dd = f16_val(d16);
        uint32_t pk[4] = {0u, 0u, 0u, 0u};
        if (T == QS_Q6_K) {
            const float dq = dd * (float)myls;
#pragma unroll
            for (int i = 0; i < GS; i++) {
                const float v = dq != 0.0f ? clampf(rintf(__fdiv_rn(x[i], dq)), -32.0f, 31.0f) + 32.0f : L[i];
                pk[i >> 2] |= (live ? (uint32_t)(int)v & 0xFFu : 0u) << (8 * (i & 3));
            }
        } else {
            const float dq = dd * (float)(myls - 32);
#pragma unroll
            for (int i = 0; i < GS; i++) {
                const float v = dq != 0.0f ? clampf(rintf(__fdiv_rn(x[i], dq)), -4.0f, 3.0f) + 4.0f : L[i];
                pk[i >> 2] |= ((uint32_t)(int)v & 0xFFu) << (8 * (i & 3));
            }
        }
        *reinterpret_cast<uint4*>(lev + g * GS) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        __syncwarp();

        // packing: a lane's output bytes come from runs of 4 or 8 consecutive level bytes, read
        // as words and combined four bytes at a time (no byte-wide shared-memory traffic)
        uint8_t* o = s_out + sbl * BB;
        auto put32 = [&](int off, uint32_t v) {  // o + off is 2-byte aligned (BB is even)
            reinterpret_cast<uint16_t*>(o + off)[0] = (uint16_t)v;
            reinterpret_cast<uint16_t*>(o + off)[1] = (uint16_t)(v >> 16);
        };
        auto lw = [&](int off) { return *reinterpret_cast<const uint32_t*>(lev + off); };
        if (T == QS_Q6_K) {
            {  // ql bytes 8g..8g+7: low nibbles of levels [A, A + 8) and [A + 64, A + 72)
                const int A = 128 * (g >> 3) + 32 * ((g >> 2) & 1) + 8 * (g & 3);
                const uint2 q0 = *reinterpret_cast<const uint2*>(lev + A), q1 = *reinterpret_cast<const uint2*>(lev + A + 64);
                put32(8 * g, (q0.x & 0x0F0F0F0Fu) | ((q1.x & 0x0F0F0F0Fu) << 4));
                put32(8 * g + 4, (q0.y & 0x0F0F0F0Fu) | ((q1.y & 0x0F0F0F0Fu) << 4));
            }
            {  // qh bytes 4g..4g+3: bits 4-5 of levels C, C + 32, C + 64, C + 96 (+ 0..3)
                const int C = 128 * (g >> 3) + 4 * (g & 7);
                put32(128 + 4 * g, ((lw(C) >> 4) & 0x03030303u) | (((lw(C + 32) >> 4) & 0x03030303u) << 2) |
                                       (((lw(C + 64) >> 4) & 0x03030303u) << 4) | (((lw(C + 96) >> 4) & 0x03030303u) << 6));
            }
            o[192 + g] = (uint8_t)(int8_t)myls;
            if (g == 0) { o[208] = (uint8_t)d16; o[209] = (uint8_t)(d16 >> 8); }
        } else {
            {  // hmask bytes 2g, 2g + 1: bit bb = level[32 bb + l] > 3 (its bit 2), for the four l of
               // one word, of which this lane keeps two
                const int W = 4 * (g >> 1);
                uint32_t acc = 0;
#pragma unroll
                for (int bb = 0; bb < 8; bb++) acc |= ((lw(32 * bb + W) >> 2) & 0x01010101u) << bb;
                reinterpret_cast<uint16_t*>(o + 2 * g)[0] = (uint16_t)(acc >> (16 * (g & 1)));
            }
            {  // qs bytes 4g..4g+3: the low 2 bits of levels D + 32 j (j = 0..3; q > 3 ? q - 4 : q)
                const int D = 128 * (g >> 3) + 4 * (g & 7);
                put32(32 + 4 * g, (lw(D) & 0x03030303u) | ((lw(D + 32) & 0x03030303u) << 2) |
                                      ((lw(D + 64) & 0x03030303u) << 4) | ((lw(D + 96) & 0x03030303u) << 6));
            }
            if (g < 8) {
                const int a0 = (int)s_ls[sbl][g], a8 = (int)s_ls[sbl][g + 8];
                o[96 + g] = (uint8_t)((a0 & 0xF) | ((a8 & 0xF) << 4));
            }
            if (g < 4) {
                int v = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) v |= ((int)s_ls[sbl][4 * j + g] >> 4) << (2 * j);
                o[104 + g] = (uint8_t)v;
            }
            if (g == 0) { o[108] = (uint8_t)d16; o[109] = (uint8_t)(d16 >> 8); }
        }
        __syncthreads();
        store_tile(a, s_out, tile * SBT, (int)min((int64_t)SBT, a.nblk - tile * SBT), BB, tid, 256);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// IQ4_XS (kernels/iq4_xs.py:35-188): one thread per 32-block
// ---------------------------------------------------------------------------
__constant__ float c_kv_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// _best_index (iq4_xs.py:35-39): bracket with searchsorted(right), midpoint compare
__device__ __forceinline__ int iq4nl_index(const float* kv, float al) {
    int p = 0;  // number of kv[1..14] <= al
#pragma unroll
    for (int step = 8; step >= 1; step >>= 1)
        if (p + step <= 14 && kv[p + step] <= al) p += step;
    const int mu = 1 + p;
    return (al - kv[mu - 1] < kv[mu] - al) ? mu - 1 : mu;
}

// The scale search's level lookup without a search. Because the table is integer,
// kv[j] <= al exactly when kv[j] <= floor(al), so the bracket kv[p] <= al < kv[p + 1] (p
// clamped to 0..14 as searchsorted + clamp does) is a function of floor(al). A floor in
// [-136, 134] indexes a table of brackets {kv[p], kv[p + 1]} held as two bf16 halves (the
// levels are 7-bit integers, exact in bf16). The table keeps one column per lane (word
// 32 e + lane), so a warp's 32 lookups hit 32 banks whatever the values. The midpoint
// compare then runs on al itself, in the reference's float arithmetic. Clamping before the
// floor keeps every value exact: below -136 the bracket is {kv[0], kv[1]} and above 134 it is
// {kv[14], kv[15]}, as for any al beyond kv[1] or kv[14]. A NaN clamps to -136, fails the
// compare and takes kv[1], as the search does.
constexpr int IQ4_TAB_LO = -136, IQ4_TAB_N = 271;                 // floors -136..134
constexpr float IQ4_TAB_FLOOR = 12582912.0f - (float)IQ4_TAB_LO;  // 1.5 * 2^23 + 136
constexpr size_t IQ4_TAB_BYTES = (size_t)IQ4_TAB_N * 32 * 4;

__device__ __forceinline__ uint32_t iq4_tab_row(float al) {  // floor(clamp(al)) - IQ4_TAB_LO
    const float y = fminf(fmaxf(al, (float)IQ4_TAB_LO), 134.5f);
    // y + 1.5 * 2^23 + 136 lies in [2^23, 2^24), where one ulp is 1: rounding down leaves
    // floor(y) + 136 in the low mantissa bits
    return __float_as_uint(__fadd_rd(y, IQ4_TAB_FLOOR)) & 0x1FFu;
}
__device__ __forceinline__ float iq4_tab_level(const uint32_t* tab, float al) {
    const uint32_t w = tab[iq4_tab_row(al) * 32];
    const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xFFFF0000u);
    return (al - lo < hi - al) ? lo : hi;
}
__device__ __forceinline__ f32x2 iq4_tab_level2(const uint32_t* tab, f32x2 al) {
    float a0, a1;
    f2_unpack(al, a0, a1);
    uint32_t b0, b1;
    f2_unpack_bits(f2_add_rm(f2_pack(fminf(fmaxf(a0, (float)IQ4_TAB_LO), 134.5f), fminf(fmaxf(a1, (float)IQ4_TAB_LO), 134.5f)),
                             f2_splat(IQ4_TAB_FLOOR)),
                   b0, b1);
    const uint32_t w0 = tab[(b0 & 0x1FFu) * 32], w1 = tab[(b1 & 0x1FFu) * 32];
    const f32x2 lo = f2_pack(__uint_as_float(w0 << 16), __uint_as_float(w1 << 16));
    const f32x2 hi = f2_pack(__uint_as_float(w0 & 0xFFFF0000u), __uint_as_float(w1 & 0xFFFF0000u));
    float d0, d1, e0, e1, l0, l1, h0, h1;
    f2_unpack(f2_sub(al, lo), d0, d1);
    f2_unpack(f2_sub(hi, al), e0, e1);
    f2_unpack(lo, l0, l1);
    f2_unpack(hi, h0, h1);
    return f2_pack(d0 < e0 ? l0 : h0, d1 < e1 ? l1 : h1);
}

// Fills the lane-column bracket table (IQ4_TAB_N rows of 32 words).
__device__ __forceinline__ void iq4_tab_fill(uint32_t* tab, int tid, int nthreads) {
    for (int i = tid; i < IQ4_TAB_N * 32; i += nthreads) {
        const float f = (float)(i / 32 + IQ4_TAB_LO);
        int p = 0;
        for (int j = 1; j <= 14; j++) p += c_kv_iq4nl[j] <= f;
        tab[i] = (__float_as_uint(c_kv_iq4nl[p]) >> 16) | (__float_as_uint(c_kv_iq4nl[p + 1]) & 0xFFFF0000u);
    }
}

// 4 CTAs of 4 warps per SM at <= 128 registers; each CTA holds 19 KB of static shared memory
// and the 34.7 KB bracket table
constexpr int IQ4XS_THREADS = 128, IQ4XS_MIN_CTAS = 4;

template <bool IMAT>
__global__ void __launch_bounds__(IQ4XS_THREADS, IQ4XS_MIN_CTAS) iq4xs_kernel(QuantArgs a) {
    constexpr int GS = 32, NG = 8, SBT = IQ4XS_THREADS / NG, BB = 136;
    __shared__ float s_kv[16];
    __shared__ __align__(16) float s_sq[SBT * QK_K];
    __shared__ float s_part[SBT][8], s_sc[SBT][NG];
    __shared__ __align__(16) uint8_t s_out[SBT * BB];
    extern __shared__ uint32_t s_l4[];  // IQ4_TAB_N x 32 lane columns
    const int tid = threadIdx.x, sbl = tid / NG, g = tid % NG;
    if (tid < 16) s_kv[tid] = c_kv_iq4nl[tid];
    iq4_tab_fill(s_l4, tid, IQ4XS_THREADS);
    __syncthreads();
    float* sq = s_sq + sbl * QK_K;
    const uint32_t* tab = s_l4 + (tid & 31);

    for (int64_t tile = blockIdx.x; tile * SBT < a.nblk; tile += gridDim.x) {
        const int64_t b = min(tile * SBT + sbl, a.nblk - 1);
        float x[GS], w[GS], t[GS];
        load_row<GS>(a.src, b * QK_K + g * GS, a.src_type, x);
        if (IMAT) {
            sb_put_sq32(sq, g, x);
            __syncwarp();
            s_part[sbl][g] = sb_sum256_partial32(sq, g);
            __syncwarp();
            const float sigma2 = __fdiv_rn(2.0f * sb_sum256_finish(s_part[sbl]), 256.0f);
            float q[GS];
            load_f32<GS>(a.qw + (b % a.nblk_row) * QK_K + g * GS, q);
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = q[i] * sqrtf(sigma2 + x[i] * x[i]);
        } else {
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = x[i] * x[i];
        }
        // _search_scales_eager (iq4_xs.py:52-76)
        float amax, mx;
        absmax_first<GS>(x, amax, mx);
        const bool live = fabsf(mx) >= EPS15;
        const float mxs = live ? mx : 1.0f;
        const float d0 = __fdiv_rn(-mxs, -127.0f);
        const float id0 = rcp_rn(d0);
        float sumqx, sumq2;
        {
            float u[GS];
#pragma unroll
            for (int i = 0; i < GS; i++) {
                const float q = iq4_tab_level(tab, id0 * x[i]);
                t[i] = (w[i] * q) * x[i];
                u[i] = (w[i] * q) * q;
            }
            sumqx = seq_sum<GS>(t);
            sumq2 = seq_sum<GS>(u);
        }
        float d = sumq2 > 0.0f ? __fdiv_rn(sumqx, sumq2) : 0.0f;
        float best = d * sumqx;
        const float r = rcp_rn(mxs);
        // Sweep products on f32x2 pairs. The sign of a zero product cannot reach the result:
        // best >= 0 throughout (sumqx^2 / sumq2 with sumq2 > 0, or a signed zero), so a step
        // is accepted only with sumqx != 0 and sumq2 > 0, whose values the sign of a zero
        // term does not change.
#pragma unroll 1
        for (int itry = -7; itry <= 7; itry++) {
            const f32x2 idv = f2_splat(r * (float)(itry - 127));
            float sx = 0.0f, s2 = 0.0f;
#pragma unroll
            for (int i = 0; i < GS; i += 2) {
                const f32x2 xx = f2_pack(x[i], x[i + 1]);
                const f32x2 q = iq4_tab_level2(tab, f2_mul_z(idv, xx));
                const f32x2 wq = f2_mul_z(f2_pack(w[i], w[i + 1]), q);
                float tx0, tx1, tq0, tq1;
                f2_unpack(f2_mul_z(wq, xx), tx0, tx1);
                f2_unpack(f2_mul_z(wq, q), tq0, tq1);
                sx = i == 0 ? __fadd_rn(tx0, tx1) : __fadd_rn(__fadd_rn(sx, tx0), tx1);
                s2 = i == 0 ? __fadd_rn(tq0, tq1) : __fadd_rn(__fadd_rn(s2, tq0), tq1);
            }
            if (s2 > 0.0f && sx * sx > best * s2) {
                const float nd = __fdiv_rn(sx, s2);
                d = nd;
                best = nd * sx;
            }
        }
        const float scale = live ? d : 0.0f;
        s_sc[sbl][g] = scale;
        __syncwarp();

        float sc8[NG], as, max_scale;
#pragma unroll
        for (int j = 0; j < NG; j++) sc8[j] = s_sc[sbl][j];
        absmax_first<NG>(sc8, as, max_scale);
        const float dsb = __fdiv_rn(-max_scale, 32.0f);
        const float idq = dsb != 0.0f ? rcp_rn(dsb) : 0.0f;
        uint8_t* o = s_out + sbl * BB;
        {
            const float ls = clampf(rintf(idq * scale), -32.0f, 31.0f);
            const float dl = dsb * ls;
            const float idl = dl != 0.0f ? rcp_rn(dl) : 0.0f;
#pragma unroll
            for (int l = 0; l < 16; l++) {
                const int lo = iq4nl_index(s_kv, idl * x[l]);
                const int hi = iq4nl_index(s_kv, idl * x[16 + l]);
                o[8 + 16 * g + l] = (uint8_t)(lo | (hi << 4));
            }
        }
        if (g == 0) {
            int lsq[NG], hb = 0;
#pragma unroll
            for (int j = 0; j < NG; j++) lsq[j] = (int)(clampf(rintf(idq * sc8[j]), -32.0f, 31.0f) + 32.0f);
#pragma unroll
            for (int j = 0; j < NG; j++) hb += (lsq[j] >> 4) << (2 * j);
            const uint16_t dh = f16_bits(dsb);
            o[0] = (uint8_t)dh; o[1] = (uint8_t)(dh >> 8);
            o[2] = (uint8_t)(hb & 0xFF); o[3] = (uint8_t)(hb >> 8);
#pragma unroll
            for (int j = 0; j < 4; j++) o[4 + j] = (uint8_t)((lsq[2 * j] & 0xF) | ((lsq[2 * j + 1] & 0xF) << 4));
        }
        __syncthreads();
        store_tile(a, s_out, tile * SBT, (int)min((int64_t)SBT, a.nblk - tile * SBT), BB, tid, IQ4XS_THREADS);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// host side: candidate tables folded exactly like the reference's numpy/python
// expressions (host code is built with -ffp-contract=off), grid sizing, launch
// ---------------------------------------------------------------------------
static void qkx_steps(float rmin, float rdelta, int nstep, int nmax, KParams& p) {  // kq_common.py:21-24
    for (int s = 0; s <= nstep; s++) p.steps[s] = (rmin + rdelta * (float)s) + (float)nmax;
    p.nsteps = nstep + 1;
}
static void qp_steps(int nmax, KParams& p) {  // kq_common.py:27-30
    int j = 0;
    for (int s = -4; s <= 4; s++) if (s) p.qp[j++] = 0.1f * (float)s + (float)nmax;
}
static void qx_steps(int nmax, float* c) {  // qx_common.py:20-23
    int j = 0;
    for (int s = -9; s <= 9; s++) if (s) c[j++] = (float)nmax + 0.1f * (float)s;
}

template <typename K>
static int grid_for(K kernel, int64_t tiles, const LaunchCtx& ctx, size_t smem = 0, int threads = 256) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1) per_sm = 1;
    int64_t g = (int64_t)per_sm * ctx.num_sms;
    return (int)(tiles < g ? (tiles > 0 ? tiles : 1) : g);
}

cudaError_t launch_kquant(int type, const QuantArgs& a, const LaunchCtx& ctx) {
    KParams p;
    memset(&p, 0, sizeof(p));
    const bool imat = a.qw != nullptr;
    cudaStream_t st = ctx.stream;
    switch (type) {
    case QS_Q4_K:
    case QS_Q5_K:
    case QS_Q2_K: {
        const int nmax = type == QS_Q4_K ? 15 : (type == QS_Q5_K ? 31 : 3);
        if (imat) qkx_steps(-0.9f, 0.05f, 36, nmax, p);
        else if (type == QS_Q4_K) qkx_steps(-1.0f, 0.1f, 20, 15, p);
        else qkx_steps(-0.5f, 0.1f, 15, nmax, p);
        qp_steps(type == QS_Q2_K ? 15 : 63, p);
#define QS_LAUNCH_QKX(K, T, I)                                         \
    {                                                                  \
        constexpr int NT = QkxTraits<T>::THREADS, SBT = NT / (QK_K / QkxTraits<T>::GS); \
        auto k = K<T, I>;                                              \
        const int64_t tiles = (a.nblk + SBT - 1) / SBT;                \
        k<<<grid_for(k, tiles, ctx, 0, NT), NT, 0, st>>>(a, p);        \
    }
        if (type == QS_Q4_K) { if (imat) QS_LAUNCH_QKX(qkx_kernel, QS_Q4_K, true) else QS_LAUNCH_QKX(qkx_kernel, QS_Q4_K, false) }
        else if (type == QS_Q5_K) { if (imat) QS_LAUNCH_QKX(qkx_kernel_r152, QS_Q5_K, true) else QS_LAUNCH_QKX(qkx_kernel_r152, QS_Q5_K, false) }
        else { if (imat) QS_LAUNCH_QKX(qkx_kernel, QS_Q2_K, true) else QS_LAUNCH_QKX(qkx_kernel, QS_Q2_K, false) }
#undef QS_LAUNCH_QKX
        break;
    }
    case QS_Q6_K:
    case QS_Q3_K: {
        qx_steps(type == QS_Q6_K ? 32 : 4, p.qx);
        qx_steps(32, p.qx2);
        const int64_t tiles = (a.nblk + 15) / 16;
#define QS_LAUNCH_QX(T, I)                                            \
    {                                                                 \
        auto k = qx_kernel<T, I>;                                     \
        qx_kernel<T, I><<<grid_for(k, tiles, ctx), 256, 0, st>>>(a, p); \
    }
        if (type == QS_Q6_K) { if (imat) QS_LAUNCH_QX(QS_Q6_K, true) else QS_LAUNCH_QX(QS_Q6_K, false) }
        else { if (imat) QS_LAUNCH_QX(QS_Q3_K, true) else QS_LAUNCH_QX(QS_Q3_K, false) }
#undef QS_LAUNCH_QX
        break;
    }
    case QS_IQ4_XS: {
        constexpr int SBT = IQ4XS_THREADS / 8;
        const int64_t tiles = (a.nblk + SBT - 1) / SBT;
        auto k = imat ? iq4xs_kernel<true> : iq4xs_kernel<false>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)IQ4_TAB_BYTES);
        if (e != cudaSuccess) return e;
        k<<<grid_for(k, tiles, ctx, IQ4_TAB_BYTES, IQ4XS_THREADS), IQ4XS_THREADS, IQ4_TAB_BYTES, st>>>(a);
        break;
    }
    default:
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace qs
