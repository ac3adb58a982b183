// Shared device helpers for the qs-b200 block quantizers (sm_100a).
//
// Every kernel here reproduces the reference's eager torch arithmetic bit for bit, so:
//   - the library is built with -fmad=false: no mul+add contraction anywhere;
//   - divides and square roots are IEEE round-to-nearest (-prec-div / -prec-sqrt);
//   - torch.round is rintf (half to even);
//   - sums keep the association of the reference site they restate: seq (left to
//     right from the first term), tree (adjacent pairs), or torch's CPU cascade for
//     `.sum(-1)` (8 lane partials, then a left-to-right pass seeded with +0).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace qs {

constexpr int QK_K = 256;
constexpr float EPS15 = 1e-15f;
constexpr float EPS8 = 1e-8f;
constexpr float F32_TINY = 1.17549435e-38f;

// Source element types (GGML type ids).
enum SrcType : int { SRC_F32 = 0, SRC_F16 = 1, SRC_BF16 = 30 };

// ---------------------------------------------------------------------------
// loads: n consecutive source elements -> f32 registers (exact conversions)
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ void load_row(const void* base, int64_t elem0, int src, float* v) {
    if (src == SRC_F32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + elem0);
#pragma unroll
        for (int i = 0; i < N / 4; i++) {
            float4 t = __ldg(p + i);
            v[4 * i + 0] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
        }
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + elem0);
#pragma unroll
        for (int i = 0; i < N / 8; i++) {
            uint4 t = __ldg(p + i);
            uint32_t w4[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint32_t lo = w4[j] & 0xFFFFu, hi = w4[j] >> 16;
                if (src == SRC_BF16) {
                    v[8 * i + 2 * j] = __uint_as_float(lo << 16);
                    v[8 * i + 2 * j + 1] = __uint_as_float(hi << 16);
                } else {
                    v[8 * i + 2 * j] = __half2float(__ushort_as_half((unsigned short)lo));
                    v[8 * i + 2 * j + 1] = __half2float(__ushort_as_half((unsigned short)hi));
                }
            }
        }
    }
}

template <int N>
__device__ __forceinline__ void load_f32(const float* p, float* v) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < N / 4; i++) {
        float4 t = __ldg(q + i);
        v[4 * i + 0] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
}

// ---------------------------------------------------------------------------
// exact scalar helpers
// ---------------------------------------------------------------------------
// 1 / x correctly rounded (the reciprocal intrinsic: the same value as the IEEE division 1 / x)
__device__ __forceinline__ float rcp_rn(float x) { return __frcp_rn(x); }
__device__ __forceinline__ float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }
__device__ __forceinline__ float min_hi(float x, float hi) { return x > hi ? hi : x; }
// clampf for the search loops, two NaN-propagating min/max instructions: equal to clampf for
// every non-NaN x (a -0 may come out +0, which only reaches an all-zero level sum, where the
// candidate is rejected anyway) and NaN for NaN x, so every accept decision is the same.
__device__ __forceinline__ float clamp_nan(float x, float lo, float hi) {
    float r;
    asm("{.reg .f32 t; max.NaN.f32 t, %1, %2; min.NaN.f32 %0, t, %3;}" : "=f"(r) : "f"(x), "f"(lo), "f"(hi));
    return r;
}
// rintf(v) (ties to even) for the candidate loops, as two adds on the FMA pipe instead of a
// round instruction on the slower XU pipe: v + 1.5 * 2^23 lands in [2^23, 2^24), where the
// spacing is 1, so the add rounds v to an integer (ties to even, as 1.5 * 2^23 is even) and
// the subtraction is exact. Equal to rintf for |v| < 2^22 except that a zero result is +0;
// beyond that it stays beyond +-(2^22 - 1), so a following clamp to a small level range gives
// the same level for every finite v; inf and NaN pass through.
__device__ __forceinline__ float rint_add(float v) { return __fadd_rn(__fadd_rn(v, 12582912.0f), -12582912.0f); }
__device__ __forceinline__ uint16_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ float f16_val(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// ---------------------------------------------------------------------------
// reductions in the reference's association orders
// ---------------------------------------------------------------------------
template <int N>
__device__ __forceinline__ float seq_sum(const float* t) {  // parts[0] + parts[1] + ...
    float s = t[0];
#pragma unroll
    for (int i = 1; i < N; i++) s = __fadd_rn(s, t[i]);
    return s;
}

template <int N>
__device__ __forceinline__ float tree_sum(const float* t) {  // adjacent-pair tree
    float a[N];
#pragma unroll
    for (int i = 0; i < N; i++) a[i] = t[i];
#pragma unroll
    for (int n = N; n > 1; n >>= 1) {
#pragma unroll
        for (int i = 0; i < n / 2; i++) a[i] = __fadd_rn(a[2 * i], a[2 * i + 1]);
    }
    return a[0];
}

// torch CPU float32 `.sum(-1)` over a contiguous dim of 8, 16 or 32
template <int N>
__device__ __forceinline__ float torch_sum(const float* t) {
    float s = 0.0f;
    if (N == 8) {
#pragma unroll
        for (int i = 0; i < 8; i++) s = __fadd_rn(s, t[i]);
    } else if (N == 16) {
#pragma unroll
        for (int l = 0; l < 8; l++) s = __fadd_rn(s, __fadd_rn(t[l], t[8 + l]));
    } else {
#pragma unroll
        for (int l = 0; l < 8; l++)
            s = __fadd_rn(s, __fadd_rn(__fadd_rn(__fadd_rn(t[l], t[8 + l]), t[16 + l]), t[24 + l]));
    }
    return s;
}

// First index of the largest |x| and the signed value there (absmax_first / argmax).
template <int N>
__device__ __forceinline__ void absmax_first(const float* x, float& amax, float& mx) {
    float a = fabsf(x[0]);
    float m = x[0];
#pragma unroll
    for (int i = 1; i < N; i++) {
        float v = fabsf(x[i]);
        if (v > a) { a = v; m = x[i]; }
    }
    amax = a;
    mx = m;
}

template <int N>
__device__ __forceinline__ float max_of(const float* x) {
    float m = x[0];
#pragma unroll
    for (int i = 1; i < N; i++) m = x[i] > m ? x[i] : m;
    return m;
}
template <int N>
__device__ __forceinline__ float min_of(const float* x) {
    float m = x[0];
#pragma unroll
    for (int i = 1; i < N; i++) m = x[i] < m ? x[i] : m;
    return m;
}

// torch's `(x*x).sum(-1)` over a 256-element superblock: 32 vectors of 8 lanes, four
// accumulators over vectors 4i+k, then a left-to-right pass over the 8 lane partials. Partial
// `lane8` in [0, 8) sums elements 32 i + 8 k + lane8 over i for each k; the caller reduces the
// 8 partials with sb_sum256_finish. The squares go through shared memory in a layout without
// bank conflicts. For 32-value groups (8 per superblock, group g's values are elements
// 32 g + c), partial `lane8` reads the columns c = lane8 + 8 k (k = 0..3) of every group row, so
// row g keeps those four columns together as one 16-byte chunk, chunk j = c & 7 stored at
// position (j + g) & 7. The 8 lanes of a superblock then write (8 x 16 B per lane) and read
// (one 16 B load per row) distinct bank quads. sq: the superblock's 256 floats, 16-byte aligned.
__device__ __forceinline__ void sb_put_sq32(float* sq, int g, const float* x) {
#pragma unroll
    for (int j = 0; j < 8; j++)
        *reinterpret_cast<float4*>(sq + 32 * g + 4 * ((j + g) & 7)) =
            make_float4(x[j] * x[j], x[j + 8] * x[j + 8], x[j + 16] * x[j + 16], x[j + 24] * x[j + 24]);
}
__device__ __forceinline__ float sb_sum256_partial32(const float* sq, int lane8) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float4 v = *reinterpret_cast<const float4*>(sq + 32 * i + 4 * ((lane8 + i) & 7));
        a0 = __fadd_rn(a0, v.x);
        a1 = __fadd_rn(a1, v.y);
        a2 = __fadd_rn(a2, v.z);
        a3 = __fadd_rn(a3, v.w);
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
}
// 16-value groups (16 per superblock, elements 16 g + c): partial `lane8` reads columns
// lane8 and lane8 + 8 of every row, so row g keeps the pair (c, c + 8) together as one
// 8-byte slot, pair p = c & 7 stored at position (p + g / 2) & 7. A superblock's 16 lanes
// write, and its 8 partial lanes read, distinct bank pairs.
__device__ __forceinline__ void sb_put_sq16(float* sq, int g, const float* x) {
#pragma unroll
    for (int p = 0; p < 8; p++)
        *reinterpret_cast<float2*>(sq + 16 * g + 2 * ((p + (g >> 1)) & 7)) = make_float2(x[p] * x[p], x[p + 8] * x[p + 8]);
}
__device__ __forceinline__ float sb_sum256_partial16(const float* sq, int lane8) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int pos = 2 * ((lane8 + i) & 7);  // rows 2i and 2i + 1 both rotate by i
        const float2 v = *reinterpret_cast<const float2*>(sq + 32 * i + pos);
        const float2 u = *reinterpret_cast<const float2*>(sq + 32 * i + 16 + pos);
        a0 = __fadd_rn(a0, v.x);
        a1 = __fadd_rn(a1, v.y);
        a2 = __fadd_rn(a2, u.x);
        a3 = __fadd_rn(a3, u.y);
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
}
__device__ __forceinline__ float sb_sum256_finish(const float* part8) {
    float s = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; l++) s = __fadd_rn(s, part8[l]);
    return s;
}

// ---------------------------------------------------------------------------
// output staging: copy `nbytes` from shared memory to global with the widest
// stores the destination alignment allows (16 B body, byte head/tail)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_bytes(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                            int nbytes, int tid, int nthreads) {
    int head = (int)((16 - ((uintptr_t)dst & 15)) & 15);
    if (head > nbytes) head = nbytes;
    for (int i = tid; i < head; i += nthreads) dst[i] = src[i];
    int body = (nbytes - head) / 16;
    uint4* d4 = reinterpret_cast<uint4*>(dst + head);
    const uint8_t* s = src + head;
    if (((uintptr_t)s & 15) == 0) {
        const uint4* s16 = reinterpret_cast<const uint4*>(s);
        for (int i = tid; i < body; i += nthreads) d4[i] = s16[i];
    } else if (((uintptr_t)s & 3) == 0) {
        for (int i = tid; i < body; i += nthreads) {
            const uint32_t* s4 = reinterpret_cast<const uint32_t*>(s + 16 * i);
            d4[i] = make_uint4(s4[0], s4[1], s4[2], s4[3]);
        }
    } else {
        for (int i = tid; i < body; i += nthreads) {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                w[j] = (uint32_t)s[16 * i + 4 * j] | ((uint32_t)s[16 * i + 4 * j + 1] << 8) |
                       ((uint32_t)s[16 * i + 4 * j + 2] << 16) | ((uint32_t)s[16 * i + 4 * j + 3] << 24);
            d4[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    for (int i = head + 16 * body + tid; i < nbytes; i += nthreads) dst[i] = src[i];
}

// ---------------------------------------------------------------------------
// packed f32x2 arithmetic (sm_100): two floats in one 64-bit register pair, one rounding
// per lane as the scalar instruction. ptxas fuses a packed product into a packed add that
// uses it (one rounding instead of two) even with .rn, and treats a fused multiply-add with
// a -0 addend as that product; a +0 addend is kept apart, and gives the correctly rounded
// product except that a -0 product comes out +0. So f2_mul_z is exact wherever the sign of
// a zero product cannot reach a result; sites where it can keep scalar products (which
// ptxas does not fuse into packed adds).
// ---------------------------------------------------------------------------
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2_pack(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ f32x2 f2_splat(float v) { return f2_pack(v, v); }
__device__ __forceinline__ void f2_unpack(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_mul_z(f32x2 a, f32x2 b) {  // a * b as fma(a, b, +0): -0 -> +0
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(0ull));
    return d;
}
__device__ __forceinline__ f32x2 f2_add(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 f2_sub(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 f2_abs(f32x2 a) { return a & 0x7FFFFFFF7FFFFFFFull; }
__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f32x2 f2_add_rm(f32x2 a, f32x2 b) {  // rounding toward -infinity
    f32x2 d;
    asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ void f2_unpack_bits(f32x2 v, uint32_t& lo, uint32_t& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}

// The adjacent-pair tree of 2H values held as pairs (v[k], v[k + H]): both halves' trees
// run side by side, and the last level adds them, as the scalar tree does.
template <int H>
__device__ __forceinline__ float tree_sum2(const f32x2* t) {
    f32x2 a[H];
#pragma unroll
    for (int i = 0; i < H; i++) a[i] = t[i];
#pragma unroll
    for (int n = H; n > 1; n >>= 1) {
#pragma unroll
        for (int i = 0; i < n / 2; i++) a[i] = f2_add(a[2 * i], a[2 * i + 1]);
    }
    float lo, hi;
    f2_unpack(a[0], lo, hi);
    return __fadd_rn(lo, hi);
}

// Parameters shared by every quantize launch.
struct QuantArgs {
    const void* src;      // n_rows x k elements of src_type, row-major, contiguous
    int src_type;
    int64_t n_rows, k;
    const float* qw;      // k importance weights or nullptr
    uint8_t* dst;         // n_rows rows of dst_row_bytes
    int64_t dst_row_bytes;
    int64_t row_bytes;    // packed bytes per row
    int64_t nblk;         // total quant blocks (superblocks, or 32-blocks for Q4_0)
    int64_t nblk_row;     // blocks per row
};

// Copy the packed output of blocks [b0, b0 + nb) from shared memory to the rows
// they belong to; rows may be strided in the destination (then, and only then, the
// block index is split into row and column: a 64-bit division).
__device__ __forceinline__ void store_tile(const QuantArgs& a, const uint8_t* stage, int64_t b0, int nb,
                                           int block_bytes, int tid, int nthreads) {
    if (a.dst_row_bytes == a.row_bytes) {
        store_bytes(a.dst + b0 * block_bytes, stage, nb * block_bytes, tid, nthreads);
        return;
    }
    int64_t b = b0;
    int done = 0;
    while (done < nb) {
        const int64_t row = b / a.nblk_row, col = b - row * a.nblk_row;
        const int run = (int)min((int64_t)(nb - done), a.nblk_row - col);
        store_bytes(a.dst + row * a.dst_row_bytes + col * block_bytes, stage + (size_t)done * block_bytes,
                    run * block_bytes, tid, nthreads);
        done += run;
        b += run;
    }
}

}  // namespace qs
