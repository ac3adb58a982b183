// Block decode (GGUF dequantization) and the decode-error checkers (sm_100a).
//
// The decode of every block format restates gguf-py's numpy dequantizers
// (gguf/quants.py, gguf 0.19.0: Q4_0 / Q4_1 / Q5_0 / Q5_1 / Q8_0 / Q2_K / Q3_K / Q4_K / Q5_K / Q6_K / IQ2_XXS /
// IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S / IQ4_XS .dequantize_blocks), which is what the
// reference's correctness harness decodes with (tools/dev_harness.py:108-109): the same
// float32 operations in the same order, so the values are bit-identical. The checkers
// measure what that harness measures next (tools/dev_harness.py:110-112), the squared
// error of the decoded values against the source rows, with optional importance
// weights: per value in float32 like the harness, (deq - x)^2 and w * (deq - x)^2;
// 8 consecutive values summed left to right in float32; everything above in double.
//
// Mapping: a CTA of 256 threads takes a tile of blocks (8 superblocks, or 64 Q4_0
// blocks), copies their bytes to shared memory with 16-byte loads, and each thread
// decodes 8 consecutive values of one block. HBM-bound: the decode writes 4 bytes per
// value, the checkers read the source rows (2 or 4 bytes per value).
#include <mutex>

#include "iq_grids.h"
#include "qs_kernels.h"

namespace qs {

namespace {

constexpr int DQ_THREADS = 256;

enum DqMode { DQ_DECODE, DQ_BLOCK_ERR, DQ_SUM_ERR };

__device__ __forceinline__ float f16_at(const uint8_t* p) { return f16_val((uint16_t)(p[0] | (p[1] << 8))); }
__device__ __forceinline__ uint32_t u32_at(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
// ksigns[i] of the IQ2/IQ3 formats: 7 sign bits plus their parity in bit 7
__device__ __forceinline__ uint32_t ksign(uint32_t i) { return i | ((__popc(i) & 1u) << 7); }
__device__ __forceinline__ float sgn(uint32_t bits, int j) { return (bits >> j) & 1u ? -1.0f : 1.0f; }

// Eight consecutive bytes as two little-endian words: one 8-byte load when aligned. Otherwise
// the decode, which reads its staged tile in shared memory, loads the (two or three) aligned
// words that hold them and joins them by funnel shifts (never past the word holding p[7]); the
// error passes, which read blocks straight from global memory (BY), load the eight bytes (for
// the unaligned 210-byte Q6_K blocks that measured faster than the word loads).
template <bool BY>
__device__ __forceinline__ uint2 ld8(const uint8_t* p) {
    const uintptr_t a = (uintptr_t)p;
    if ((a & 7) == 0) return *reinterpret_cast<const uint2*>(p);
    if (BY) {
        uint32_t w[2];
#pragma unroll
        for (int k = 0; k < 2; k++)
            w[k] = __byte_perm(__byte_perm(p[4 * k], p[4 * k + 1], 0x0040u), __byte_perm(p[4 * k + 2], p[4 * k + 3], 0x0040u), 0x5410u);
        return make_uint2(w[0], w[1]);
    }
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    if ((a & 3) == 0) return make_uint2(w[0], w[1]);
    const uint32_t sh = (uint32_t)(a & 3) * 8, w0 = w[0], w1 = w[1], w2 = w[2];
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}
// byte i of w as a float minus `bias` (an integer): 2^23 + byte, then one exact subtraction of
// 2^23 + bias, where (float)(byte - bias) needs an integer conversion
template <int BIAS>
__device__ __forceinline__ float byte_f(uint32_t w, int i) {
    return __fadd_rn(__int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)i)), -(8388608.0f + (float)BIAS));
}

// Level -> grid value maps of the IQ dequant grids (gguf IQ*.grid_map).
__device__ __forceinline__ float iq2_val(int l) { return l == 0 ? 8.0f : (l == 1 ? 25.0f : 43.0f); }
__device__ __forceinline__ float iq3xxs_val(int l) { return l == 7 ? 62.0f : (float)(4 + 8 * l); }
__device__ __forceinline__ float iq3s_val(int l) { return (float)(2 * l + 1); }

__constant__ int8_t c_kvalues[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

template <int T> struct Dq;

// Q4_0 (gguf Q4_0.dequantize_blocks): d * (q - 8); bytes hold values j (low) and j + 16 (high)
template <> struct Dq<QS_Q4_0> {
    static constexpr int QK = 32, BB = 18;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b);
        const int p = 8 * t;
        const uint2 q8 = ld8<BY>(b + 2 + (p & 15));
        const uint32_t sh = p < 16 ? 0 : 4, lo = (q8.x >> sh) & 0x0F0F0F0Fu, hi = (q8.y >> sh) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = d * byte_f<8>(lo, i);
            v[4 + i] = d * byte_f<8>(hi, i);
        }
    }
};

// Q4_1 (gguf Q4_1.dequantize_blocks): (d * q) + m, q as in Q4_0 without the offset
template <> struct Dq<QS_Q4_1> {
    static constexpr int QK = 32, BB = 20;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b), m = f16_at(b + 2);
        const int p = 8 * t;
        const uint2 q8 = ld8<BY>(b + 4 + (p & 15));
        const uint32_t sh = p < 16 ? 0 : 4, lo = (q8.x >> sh) & 0x0F0F0F0Fu, hi = (q8.y >> sh) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = d * byte_f<0>(lo, i) + m;
            v[4 + i] = d * byte_f<0>(hi, i) + m;
        }
    }
};

// Q5_0 (gguf Q5_0.dequantize_blocks): d * ((ql | qh << 4) - 16), bit j of qh for value j
template <> struct Dq<QS_Q5_0> {
    static constexpr int QK = 32, BB = 22;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b);
        const int p = 8 * t;
        const uint32_t hb = b[2 + t];  // qh bits of values p .. p + 7
        const uint8_t* ql = b + 6 + (p & 15);
        const int sh = p < 16 ? 0 : 4;
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = d * (float)((((ql[i] >> sh) & 0xF) | (int)(((hb >> i) & 1u) << 4)) - 16);
    }
};

// Q5_1 (gguf Q5_1.dequantize_blocks): (d * (ql | qh << 4)) + m
template <> struct Dq<QS_Q5_1> {
    static constexpr int QK = 32, BB = 24;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b), m = f16_at(b + 2);
        const int p = 8 * t;
        const uint32_t hb = b[4 + t];  // qh bits of values p .. p + 7
        const uint8_t* ql = b + 8 + (p & 15);
        const int sh = p < 16 ? 0 : 4;
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = d * (float)(((ql[i] >> sh) & 0xF) | (int)(((hb >> i) & 1u) << 4)) + m;
    }
};

// Q8_0 (gguf Q8_0.dequantize_blocks): x * d with x the int8 values
template <> struct Dq<QS_Q8_0> {
    static constexpr int QK = 32, BB = 34;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b);
        const uint2 q8 = ld8<BY>(b + 2 + 8 * t);
        const uint32_t lo = q8.x ^ 0x80808080u, hi = q8.y ^ 0x80808080u;  // int8 + 128
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = byte_f<128>(lo, i) * d;
            v[4 + i] = byte_f<128>(hi, i) * d;
        }
    }
};

// Q2_K: scales[16] qs[64] d dmin; value e: (d * (sc & 15)) * q - dmin * (sc >> 4)
template <> struct Dq<QS_Q2_K> {
    static constexpr int QK = 256, BB = 84;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b + 80), dmin = f16_at(b + 82);
        const int e0 = 8 * t, sc = b[e0 / 16];
        const float dl = d * (float)(sc & 0xF), ml = dmin * (float)(sc >> 4);
        const int h = e0 / 128, s = (e0 % 128) / 32, l0 = e0 % 32;
        const uint2 q8 = ld8<BY>(b + 16 + 32 * h + l0);
        const uint32_t lo = (q8.x >> (2 * s)) & 0x03030303u, hi = (q8.y >> (2 * s)) & 0x03030303u;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = dl * byte_f<0>(lo, i) - ml;
            v[4 + i] = dl * byte_f<0>(hi, i) - ml;
        }
    }
};

// Q3_K: hmask[32] qs[64] scales[12] d; value e: (d * (sc - 32)) * (ql - 4 * !hbit)
template <> struct Dq<QS_Q3_K> {
    static constexpr int QK = 256, BB = 110;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b + 108);
        const int e0 = 8 * t, g = e0 / 16;
        const uint8_t* sc = b + 96;
        const int ls = (sc[g % 8] >> (4 * (g / 8))) & 0xF, hs = (sc[8 + g % 4] >> (2 * (g / 4))) & 3;
        const float dl = d * (float)((int)(int8_t)(uint8_t)(ls | (hs << 4)) - 32);
        const int h = e0 / 128, s = (e0 % 128) / 32, s8 = e0 / 32, l0 = e0 % 32;
        // ql - 4 * !hbit = (ql | hbit << 2) - 4
        const uint2 l8 = ld8<BY>(b + 32 + 32 * h + l0), h8 = ld8<BY>(b + l0);
        const uint32_t lo = ((l8.x >> (2 * s)) & 0x03030303u) | (((h8.x >> s8) & 0x01010101u) << 2);
        const uint32_t hi = ((l8.y >> (2 * s)) & 0x03030303u) | (((h8.y >> s8) & 0x01010101u) << 2);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = dl * byte_f<4>(lo, i);
            v[4 + i] = dl * byte_f<4>(hi, i);
        }
    }
};

// 6-bit scale / min j of the Q4_K / Q5_K scale block (gguf Q4_K.get_scale_min)
__device__ __forceinline__ void k_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 0x3F;
        mn = s[4 + j] & 0x3F;
    } else {
        sc = (s[8 + j - 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
        mn = (s[8 + j - 4] >> 4) | ((s[4 + j - 4] >> 2) & 0x30);
    }
}

// Q4_K: d dmin scales[12] qs[128]; value e: (d * sc) * q - dmin * m
template <> struct Dq<QS_Q4_K> {
    static constexpr int QK = 256, BB = 144;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b), dmin = f16_at(b + 2);
        const int e0 = 8 * t, sub = e0 / 32, c = e0 / 64, s = (e0 % 64) / 32, l0 = e0 % 32;
        int sc, mn;
        k_scale_min(b + 4, sub, sc, mn);
        const float dl = d * (float)sc, ml = dmin * (float)mn;
        const uint2 q8 = ld8<BY>(b + 16 + 32 * c + l0);
        const uint32_t lo = (q8.x >> (4 * s)) & 0x0F0F0F0Fu, hi = (q8.y >> (4 * s)) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = dl * byte_f<0>(lo, i) - ml;
            v[4 + i] = dl * byte_f<0>(hi, i) - ml;
        }
    }
};

// Q5_K: d dmin scales[12] qh[32] qs[128]
template <> struct Dq<QS_Q5_K> {
    static constexpr int QK = 256, BB = 176;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b), dmin = f16_at(b + 2);
        const int e0 = 8 * t, sub = e0 / 32, c = e0 / 64, s = (e0 % 64) / 32, l0 = e0 % 32;
        int sc, mn;
        k_scale_min(b + 4, sub, sc, mn);
        const float dl = d * (float)sc, ml = dmin * (float)mn;
        const uint2 l8 = ld8<BY>(b + 48 + 32 * c + l0), h8 = ld8<BY>(b + 16 + l0);
        const uint32_t lo = ((l8.x >> (4 * s)) & 0x0F0F0F0Fu) | (((h8.x >> sub) & 0x01010101u) << 4);
        const uint32_t hi = ((l8.y >> (4 * s)) & 0x0F0F0F0Fu) | (((h8.y >> sub) & 0x01010101u) << 4);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = dl * byte_f<0>(lo, i) - ml;
            v[4 + i] = dl * byte_f<0>(hi, i) - ml;
        }
    }
};

// Q6_K: ql[128] qh[64] scales[16] (int8) d; value e: (d * sc) * (q - 32)
template <> struct Dq<QS_Q6_K> {
    static constexpr int QK = 256, BB = 210;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b + 208);
        const int e0 = 8 * t;
        const float dl = d * (float)(int8_t)b[192 + e0 / 16];
        const int c = e0 / 128, sl = (e0 % 128) / 64, ll = e0 % 64, sh = (e0 % 128) / 32, lh = e0 % 32;
        const uint2 l8 = ld8<BY>(b + 64 * c + ll), h8 = ld8<BY>(b + 128 + 32 * c + lh);
        const uint32_t lo = ((l8.x >> (4 * sl)) & 0x0F0F0F0Fu) | (((h8.x >> (2 * sh)) & 0x03030303u) << 4);
        const uint32_t hi = ((l8.y >> (4 * sl)) & 0x0F0F0F0Fu) | (((h8.y >> (2 * sh)) & 0x03030303u) << 4);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[i] = dl * byte_f<32>(lo, i);
            v[4 + i] = dl * byte_f<32>(hi, i);
        }
    }
};

// IQ2_XXS: d, 8 x (4 grid bytes, u32 of 4 x 7 sign bits | scale << 28)
template <> struct Dq<QS_IQ2_XXS> {
    static constexpr int QK = 256, BB = 66;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t* kgrid, float* v) {
        const float d = f16_at(b);
        const int g = t / 4, s = t % 4;
        const uint32_t w1 = u32_at(b + 2 + 8 * g + 4);
        const float db = (d * (0.5f + (float)(w1 >> 28))) * 0.25f;
        const uint32_t sg = ksign((w1 >> (7 * s)) & 127);
        const int code = __ldg(kgrid + b[2 + 8 * g + s]);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = (db * iq2_val((code >> (2 * j)) & 3)) * sgn(sg, j);
    }
};

// IQ2_XS: d, 32 x u16 (9-bit grid index | 7-bit sign index << 9), 8 bytes of 4-bit scales
template <> struct Dq<QS_IQ2_XS> {
    static constexpr int QK = 256, BB = 74;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t* kgrid, float* v) {
        const float d = f16_at(b);
        const int q16 = b[2 + 2 * t] | (b[3 + 2 * t] << 8);
        const int sc = (b[66 + t / 4] >> (4 * ((t / 2) & 1))) & 0xF;
        const float db = (d * (0.5f + (float)sc)) * 0.25f;
        const uint32_t sg = ksign((uint32_t)q16 >> 9);
        const int code = __ldg(kgrid + (q16 & 511));
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = (db * iq2_val((code >> (2 * j)) & 3)) * sgn(sg, j);
    }
};

// IQ2_S: d, qs[32], signs[32], qh[8] (2 high index bits each), scales[8]
template <> struct Dq<QS_IQ2_S> {
    static constexpr int QK = 256, BB = 82;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t* kgrid, float* v) {
        const float d = f16_at(b);
        const int sc = (b[74 + t / 4] >> (4 * ((t / 2) & 1))) & 0xF;
        const float db = (d * (0.5f + (float)sc)) * 0.25f;
        const int gi = b[2 + t] | (((b[66 + t / 4] >> (2 * (t % 4))) & 3) << 8);
        const uint32_t sg = b[34 + t];
        const int code = __ldg(kgrid + gi);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = (db * iq2_val((code >> (2 * j)) & 3)) * sgn(sg, j);
    }
};

// IQ3_XXS: d, qs[64] grid bytes (4 values each), 8 x u32 (4 x 7 sign bits | scale << 28)
template <> struct Dq<QS_IQ3_XXS> {
    static constexpr int QK = 256, BB = 98;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t* kgrid, float* v) {
        const float d = f16_at(b);
        const int g = t / 4, s = t % 4;
        const uint32_t w = u32_at(b + 66 + 4 * g);
        const float db = (d * (0.5f + (float)(w >> 28))) * 0.5f;
        const uint32_t sg = ksign((w >> (7 * s)) & 127);
        const int c0 = __ldg(kgrid + b[2 + 2 * t]), c1 = __ldg(kgrid + b[3 + 2 * t]);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            v[j] = (db * iq3xxs_val((c0 >> (3 * j)) & 7)) * sgn(sg, j);
            v[4 + j] = (db * iq3xxs_val((c1 >> (3 * j)) & 7)) * sgn(sg, 4 + j);
        }
    }
};

// IQ3_S: d, qs[64], qh[8] (high index bit), signs[32], scales[4]; db = d * (1 + 2 * sc)
template <> struct Dq<QS_IQ3_S> {
    static constexpr int QK = 256, BB = 110;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t* kgrid, float* v) {
        const float d = f16_at(b);
        const int g = t / 4;
        const int sc = (b[106 + g / 2] >> (4 * (g & 1))) & 0xF;
        const float db = d * (float)(1 + 2 * sc);
        const uint32_t sg = b[74 + t];
        const int k0 = 2 * t, k1 = 2 * t + 1;
        const int g0 = b[2 + k0] | (((b[66 + k0 / 8] >> (k0 % 8)) & 1) << 8);
        const int g1 = b[2 + k1] | (((b[66 + k1 / 8] >> (k1 % 8)) & 1) << 8);
        const int c0 = __ldg(kgrid + g0), c1 = __ldg(kgrid + g1);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            v[j] = (db * iq3s_val((c0 >> (3 * j)) & 7)) * sgn(sg, j);
            v[4 + j] = (db * iq3s_val((c1 >> (3 * j)) & 7)) * sgn(sg, 4 + j);
        }
    }
};

// IQ4_XS: d, scales_h (u16), scales_l[4], qs[128]; value: (d * (sc - 32)) * kvalues[q]
template <> struct Dq<QS_IQ4_XS> {
    static constexpr int QK = 256, BB = 136;
    template <bool BY>
    __device__ static void decode(const uint8_t* b, int t, const uint16_t*, float* v) {
        const float d = f16_at(b);
        const int i = t / 4, u = (t % 4) / 2, j0 = 8 * (t % 2);
        const int sh = b[2] | (b[3] << 8);
        const int ls = (b[4 + i / 2] >> (4 * (i & 1))) & 0xF, hs = (sh >> (2 * i)) & 3;
        const float dl = d * (float)((int)(int8_t)(uint8_t)(ls | (hs << 4)) - 32);
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = dl * (float)c_kvalues[(b[8 + 16 * i + j0 + j] >> (4 * u)) & 0xF];
    }
};

struct DqArgs {
    const uint8_t* src;       // packed rows
    int64_t src_row_bytes;
    int64_t n_rows, k, nblk_row, nblk;
    float* dst;               // DQ_DECODE
    int64_t dst_stride;       // elements
    const void* x;            // DQ_*_ERR: source rows, n_rows x k contiguous
    int x_type;
    const float* qw;          // k weights or null
    double* err;              // DQ_BLOCK_ERR: one per block
    double* partial;          // DQ_SUM_ERR: 2 per CTA (weighted, plain)
    const uint16_t* kgrid;    // IQ codebook of the type (grid index -> code)
};

__device__ __forceinline__ void load_x8(const void* base, int64_t e0, int src, float* v) { load_row<8>(base, e0, src, v); }

// resident CTAs per SM the register budget is sized for (64 registers): the checkers hold the
// prefetched source values and weights; the decode's word loads spilled at five
template <int MODE> struct DqOcc { static constexpr int CTAS = 4; };

template <int TYPE, int MODE>
__global__ void __launch_bounds__(DQ_THREADS, DqOcc<MODE>::CTAS) dq_kernel(DqArgs a) {
    using D = Dq<TYPE>;
    constexpr int TPB = D::QK / 8, BPT = DQ_THREADS / TPB;  // threads per block, blocks per tile
    __shared__ __align__(16) uint8_t s_blk[BPT * D::BB + 32];
    __shared__ double s_red[2][DQ_THREADS / 32];
    const int tid = threadIdx.x, lb = tid / TPB, t = tid % TPB;
    const bool packed = a.src_row_bytes == a.nblk_row * D::BB;
    // the error passes read packed blocks straight from global memory (L1): they also load
    // the source rows, and staging the blocks cost two CTA barriers a tile (their main stall,
    // +7-9 % without); decode keeps the coalesced 16-byte staging (5-12 % faster there)
    const bool direct = MODE != DQ_DECODE && packed;
    double acc_w = 0.0, acc = 0.0;

    // Packed rows: a tile is one contiguous span of nb * BB bytes, at most one 16-byte body
    // chunk plus a head and a tail byte per thread. The next tile's share is loaded into
    // registers before the current tile is decoded, so the load latency overlaps the decode
    // and the stores; the share lands in shared memory at s_blk + (address & 15), so the
    // 16-byte aligned body moves with 16-byte stores.
    static_assert((BPT * D::BB) / 16 + 1 <= DQ_THREADS, "one body chunk per thread");
    struct Share {
        uint4 v;
        uint8_t h, tl;
        int mis, head, body, nbytes;
    };
    auto fetch = [&](int64_t tile, Share& sh) {
        const int64_t b0 = tile * BPT;
        const uint8_t* g = a.src + b0 * D::BB;
        sh.nbytes = (int)min((int64_t)BPT, a.nblk - b0) * D::BB;
        sh.mis = (int)((uintptr_t)g & 15);
        sh.head = min((16 - sh.mis) & 15, sh.nbytes);
        sh.body = (sh.nbytes - sh.head) / 16;
        if (tid < sh.body) sh.v = __ldg(reinterpret_cast<const uint4*>(g + sh.head) + tid);
        if (tid < sh.head) sh.h = __ldg(g + tid);
        const int ti = sh.head + 16 * sh.body + tid;
        if (ti < sh.nbytes) sh.tl = __ldg(g + ti);
    };
    Share cur;
    if (packed && !direct && (int64_t)blockIdx.x * BPT < a.nblk) fetch(blockIdx.x, cur);

    for (int64_t tile = blockIdx.x; tile * BPT < a.nblk; tile += gridDim.x) {
        const int64_t b0 = tile * BPT;
        const int nb = (int)min((int64_t)BPT, a.nblk - b0);
        const bool live = lb < nb;
        const int64_t b = b0 + lb;
        // the source values and weights do not depend on the blocks: in flight with the staging
        float cx[8], cw[8];
        if (MODE != DQ_DECODE && live) {
            const int64_t row = b / a.nblk_row, col = (b - row * a.nblk_row) * D::QK + 8 * t;
            load_x8(a.x, row * a.k + col, a.x_type, cx);
            if (a.qw) load_f32<8>(a.qw + col, cw);
        }
        const uint8_t* tb;
        if (direct) {
            tb = a.src + b0 * D::BB;
        } else if (packed) {
            uint8_t* sp = s_blk + cur.mis;
            if (tid < cur.body) reinterpret_cast<uint4*>(sp + cur.head)[tid] = cur.v;
            if (tid < cur.head) sp[tid] = cur.h;
            const int ti = cur.head + 16 * cur.body + tid;
            if (ti < cur.nbytes) sp[ti] = cur.tl;
            tb = sp;
        } else {
            for (int i = tid; i < nb * D::BB; i += DQ_THREADS) {
                const int64_t bb = b0 + i / D::BB;
                const int64_t r = bb / a.nblk_row, c = bb - r * a.nblk_row;
                s_blk[i] = __ldg(a.src + r * a.src_row_bytes + c * D::BB + i % D::BB);
            }
            tb = s_blk;
        }
        if (!direct) {
            __syncthreads();
            if (packed && (tile + gridDim.x) * BPT < a.nblk) fetch(tile + gridDim.x, cur);  // the next tile
            __syncthreads();
        }
        if (live) {
            float v[8];
            D::template decode<MODE != DQ_DECODE>(tb + lb * D::BB, t, a.kgrid, v);
            if (MODE == DQ_DECODE) {
                const int64_t row = b / a.nblk_row, col = (b - row * a.nblk_row) * D::QK + 8 * t;
                float4* o = reinterpret_cast<float4*>(a.dst + row * a.dst_stride + col);
                o[0] = make_float4(v[0], v[1], v[2], v[3]);
                o[1] = make_float4(v[4], v[5], v[6], v[7]);
            } else {
                // per value in float32 as the reference harness computes it, (deq - x)^2
                // and w * that; the 8 values summed left to right in float32, then double
                float fw = 0.0f, f2 = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float e = v[i] - cx[i];
                    const float ee = e * e;
                    const float we = a.qw ? cw[i] * ee : ee;
                    f2 = i == 0 ? ee : f2 + ee;
                    fw = i == 0 ? we : fw + we;
                }
                double ew = (double)fw;
                const double e2 = (double)f2;
                if (MODE == DQ_BLOCK_ERR) {
                    // the TPB threads of the block are adjacent lanes; fixed xor tree
#pragma unroll
                    for (int o = TPB / 2; o > 0; o >>= 1) ew += __shfl_xor_sync(TPB == 32 ? 0xffffffffu : (0xFu << (tid & 28)), ew, o);
                    if (t == 0) a.err[b] = ew;
                } else {
                    acc_w += ew;
                    acc += e2;
                }
            }
        }
        if (!direct) __syncthreads();
    }
    if (MODE == DQ_SUM_ERR) {
        // CTA partial: xor tree within each warp, then warps in order
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            acc_w += __shfl_xor_sync(0xffffffffu, acc_w, o);
            acc += __shfl_xor_sync(0xffffffffu, acc, o);
        }
        if ((tid & 31) == 0) { s_red[0][tid >> 5] = acc_w; s_red[1][tid >> 5] = acc; }
        __syncthreads();
        if (tid == 0) {
            double sw = 0.0, s = 0.0;
            for (int i = 0; i < DQ_THREADS / 32; i++) { sw += s_red[0][i]; s += s_red[1][i]; }
            a.partial[2 * blockIdx.x] = sw;
            a.partial[2 * blockIdx.x + 1] = s;
        }
    }
}

// Sum the per-CTA partials in a fixed order: thread i adds partials i, i + 256, ...,
// then a tree over the 256 threads. out[0] weighted, out[1] plain.
__global__ void __launch_bounds__(DQ_THREADS) dq_finish_kernel(const double* partial, int n, double* out) {
    __shared__ double s[2][DQ_THREADS];
    const int tid = threadIdx.x;
    double sw = 0.0, sp = 0.0;
    for (int i = tid; i < n; i += DQ_THREADS) { sw += partial[2 * i]; sp += partial[2 * i + 1]; }
    s[0][tid] = sw;
    s[1][tid] = sp;
    __syncthreads();
    for (int h = DQ_THREADS / 2; h > 0; h >>= 1) {
        if (tid < h) { s[0][tid] += s[0][tid + h]; s[1][tid] += s[1][tid + h]; }
        __syncthreads();
    }
    if (tid == 0) { out[0] = s[0][0]; out[1] = s[1][0]; }
}

template <int TYPE, int MODE>
cudaError_t launch_dq_t(const DqArgs& a, const LaunchCtx& ctx, int grid) {
    dq_kernel<TYPE, MODE><<<grid, DQ_THREADS, 0, ctx.stream>>>(a);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t launch_dq_mode(int type, const DqArgs& a, const LaunchCtx& ctx, int grid) {
    switch (type) {
    case QS_Q4_0: return launch_dq_t<QS_Q4_0, MODE>(a, ctx, grid);
    case QS_Q4_1: return launch_dq_t<QS_Q4_1, MODE>(a, ctx, grid);
    case QS_Q5_0: return launch_dq_t<QS_Q5_0, MODE>(a, ctx, grid);
    case QS_Q5_1: return launch_dq_t<QS_Q5_1, MODE>(a, ctx, grid);
    case QS_Q8_0: return launch_dq_t<QS_Q8_0, MODE>(a, ctx, grid);
    case QS_Q2_K: return launch_dq_t<QS_Q2_K, MODE>(a, ctx, grid);
    case QS_Q3_K: return launch_dq_t<QS_Q3_K, MODE>(a, ctx, grid);
    case QS_Q4_K: return launch_dq_t<QS_Q4_K, MODE>(a, ctx, grid);
    case QS_Q5_K: return launch_dq_t<QS_Q5_K, MODE>(a, ctx, grid);
    case QS_Q6_K: return launch_dq_t<QS_Q6_K, MODE>(a, ctx, grid);
    case QS_IQ2_XXS: return launch_dq_t<QS_IQ2_XXS, MODE>(a, ctx, grid);
    case QS_IQ2_XS: return launch_dq_t<QS_IQ2_XS, MODE>(a, ctx, grid);
    case QS_IQ2_S: return launch_dq_t<QS_IQ2_S, MODE>(a, ctx, grid);
    case QS_IQ3_XXS: return launch_dq_t<QS_IQ3_XXS, MODE>(a, ctx, grid);
    case QS_IQ3_S: return launch_dq_t<QS_IQ3_S, MODE>(a, ctx, grid);
    case QS_IQ4_XS: return launch_dq_t<QS_IQ4_XS, MODE>(a, ctx, grid);
    default: return cudaErrorInvalidValue;
    }
}

int block_qk(int type) {
    return type == QS_Q4_0 || type == QS_Q4_1 || type == QS_Q5_0 || type == QS_Q5_1 || type == QS_Q8_0 ? 32 : 256;
}

DqArgs make_args(int type, const DqCall& c, const IqTables* t) {
    DqArgs a;
    a.src = static_cast<const uint8_t*>(c.blocks);
    a.src_row_bytes = c.blocks_row_bytes;
    a.n_rows = c.n_rows;
    a.k = c.k;
    a.nblk_row = c.k / block_qk(type);
    a.nblk = c.n_rows * a.nblk_row;
    a.dst = c.dst;
    a.dst_stride = c.dst_stride;
    a.x = c.x;
    a.x_type = c.x_type;
    a.qw = c.qw;
    a.err = c.err;
    a.partial = nullptr;
    a.kgrid = iq_kgrid(t, type);
    return a;
}

// CTAs for a pass over nblk blocks: tiles of 8 superblocks (64 Q4_0 blocks), capped at
// 8 resident CTAs per SM.
int dq_grid(int type, int64_t nblk, const LaunchCtx& ctx) {
    const int bpt = DQ_THREADS / (block_qk(type) / 8);
    const int64_t tiles = (nblk + bpt - 1) / bpt;
    const int64_t cap = (int64_t)ctx.num_sms * 8;
    return (int)(tiles < cap ? (tiles > 0 ? tiles : 1) : cap);
}

}  // namespace

int dq_partial_count(int type, int64_t n_rows, int64_t k, const LaunchCtx& ctx) {
    return dq_grid(type, n_rows * (k / block_qk(type)), ctx);
}

cudaError_t launch_dequant(int type, const DqCall& c, const LaunchCtx& ctx, const IqTables* t) {
    DqArgs a = make_args(type, c, t);
    if (a.nblk == 0) return cudaSuccess;
    return launch_dq_mode<DQ_DECODE>(type, a, ctx, dq_grid(type, a.nblk, ctx));
}

cudaError_t launch_block_error(int type, const DqCall& c, const LaunchCtx& ctx, const IqTables* t) {
    DqArgs a = make_args(type, c, t);
    if (a.nblk == 0) return cudaSuccess;
    return launch_dq_mode<DQ_BLOCK_ERR>(type, a, ctx, dq_grid(type, a.nblk, ctx));
}

cudaError_t launch_tensor_error(int type, const DqCall& c, double* partial, int npartial, double* out,
                                const LaunchCtx& ctx, const IqTables* t) {
    DqArgs a = make_args(type, c, t);
    a.partial = partial;
    const int grid = dq_grid(type, a.nblk, ctx);
    if (grid > npartial) return cudaErrorInvalidValue;
    cudaError_t e = a.nblk ? launch_dq_mode<DQ_SUM_ERR>(type, a, ctx, grid) : cudaSuccess;
    if (e != cudaSuccess) return e;
    dq_finish_kernel<<<1, DQ_THREADS, 0, ctx.stream>>>(partial, a.nblk ? grid : 0, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// qs_tensor_error_noalloc: the same launch with its scratch in static device memory
// ---------------------------------------------------------------------------
namespace {

// Per-CTA partial sums (weighted, plain) of one launch. Every CTA of the launch writes its
// own pair before the final pass reads the pairs, so nothing here needs to start at zero.
static __device__ __align__(256) double g_na_partial[2 * NA_MAX_PARTIALS];
// The five IQ codebooks (grid index -> code), copied in once per device at set-up.
constexpr int NA_KG_OFF[5] = {0, 256, 768, 1792, 2048};
static __device__ __align__(256) uint16_t g_na_kgrid[256 + 512 + 1024 + 256 + 512];

std::mutex g_na_mu;
NoAllocDevice g_na_dev[NA_MAX_DEVICES];

}  // namespace

cudaError_t noalloc_setup(int device, const NoAllocDevice** out) {
    if (device < 0 || device >= NA_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_na_mu);
    NoAllocDevice& d = g_na_dev[device];
    if (!d.ready) {
        cudaError_t e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) return e;
        void* p = nullptr;
        if ((e = cudaGetSymbolAddress(&p, g_na_partial)) != cudaSuccess) return e;
        d.partial = static_cast<double*>(p);
        if ((e = cudaGetSymbolAddress(&p, g_na_kgrid)) != cudaSuccess) return e;
        uint16_t* kg = static_cast<uint16_t*>(p);
        const uint16_t* src[5] = {KGRID_2BIT_256, KGRID_2BIT_512, KGRID_2BIT_1024, KGRID_3BIT_256, KGRID_3BIT_512};
        const int n[5] = {256, 512, 1024, 256, 512};
        for (int i = 0; i < 5; i++)
            if ((e = cudaMemcpy(kg + NA_KG_OFF[i], src[i], n[i] * sizeof(uint16_t), cudaMemcpyHostToDevice)) != cudaSuccess)
                return e;
        d.kgrid = kg;
        d.ready = true;
    }
    *out = &d;
    return cudaSuccess;
}

cudaError_t launch_tensor_error_noalloc(int type, const DqCall& c, double* out, const LaunchCtx& ctx,
                                        const NoAllocDevice& d) {
    DqArgs a;
    a.src = static_cast<const uint8_t*>(c.blocks);
    a.src_row_bytes = c.blocks_row_bytes;
    a.n_rows = c.n_rows;
    a.k = c.k;
    a.nblk_row = c.k / block_qk(type);
    a.nblk = c.n_rows * a.nblk_row;
    a.dst = nullptr;
    a.dst_stride = 0;
    a.x = c.x;
    a.x_type = c.x_type;
    a.qw = c.qw;
    a.err = nullptr;
    a.partial = d.partial;
    const int gi = type == QS_IQ2_XXS ? 0 : type == QS_IQ2_XS ? 1 : type == QS_IQ2_S ? 2 : type == QS_IQ3_XXS ? 3 : 4;
    a.kgrid = d.kgrid + NA_KG_OFF[gi];
    const int grid = dq_grid(type, a.nblk, ctx);
    if (grid > NA_MAX_PARTIALS) return cudaErrorInvalidValue;
    cudaError_t e = a.nblk ? launch_dq_mode<DQ_SUM_ERR>(type, a, ctx, grid) : cudaSuccess;
    if (e != cudaSuccess) return e;
    dq_finish_kernel<<<1, DQ_THREADS, 0, ctx.stream>>>(d.partial, a.nblk ? grid : 0, out);
    return cudaGetLastError();
}

}  // namespace qs
