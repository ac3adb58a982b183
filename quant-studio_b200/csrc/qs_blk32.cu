// 32-value block formats on sm_100a: Q4_0, Q4_1, Q5_0, Q5_1, Q8_0. HBM-bound.
//
// Q4_0 follows the reference's kernels/q4_0.py:14-33. The reference has no kernel for the
// other four; its type-mix policy still routes tensors to them (kernels/scheme.py:375:
// Q4_K / Q5_K / Q6_K fall back to Q5_0 / Q5_1 / Q8_0 when a row is not a multiple of 256;
// :521-523: Q4_0 / Q5_0 with an importance matrix send the first ffn_down layers to Q4_1 /
// Q5_1). Those follow ggml-quants.c's quantize_row_{q4_1,q5_0,q5_1,q8_0}_ref as gguf-py
// restates them in numpy (gguf/quants.py quantize_blocks); like the reference's Q4_0 they
// ignore importance weights. Where numpy's vectorised min / max and ggml's scalar loop
// disagree (the sign of a zero minimum or maximum in a block holding both +0 and -0) this
// follows ggml's loop: the first of the tied zeros.
//
// Streaming (warp-specialised, no CTA-wide barrier in the loop):
//   * the source is a 2-D tensor of blocks (one row of 32 values per block) under a TMA
//     tensor map with a 64-byte (16-bit sources) or 128-byte (f32) swizzle, so that the
//     16-byte chunk c of the block in stage row R lands at chunk c ^ ((R >> 1) & 3), resp.
//     c ^ (R & 7): lane R of a warp reads its block's chunks in block order and the 8
//     lanes of every quarter warp still hit 8 different bank groups;
//   * a persistent CTA owns one contiguous range of blocks; the ranges of all CTAs differ by
//     at most 8 blocks and start at multiples of 8 blocks, so every warp's packed output
//     starts on a 16-byte boundary;
//   * a producer warp streams the range through a ring of shared-memory stages
//     (cp.async.bulk.tensor, no multicast), each completing on its `full` mbarrier; 8
//     consumer warps quantize one block per lane, release the stage on its `empty`
//     mbarrier and store their 32 packed blocks from a per-warp staging with 16-byte
//     stores. Stages are G x 32 blocks shared by G warps: G = 8 (256-block stages that all
//     warps read) for long ranges, G = 1 (32-block stages, stage j for warp j % 8) when a
//     CTA has fewer than 8 of the large stages, where ramp and tail are a good part of the
//     launch: every warp starts after a 2 KB copy, and the CTA ends one small stage after
//     its last copy (measured: 4096 x 4096 Q4_0 12.0 -> 11.1 us, while 14336 x 4096 keeps
//     the 256-block stages, 31.9 us against 35.0 us with small ones);
//   * under programmatic stream serialization the next launch's CTAs set up while this
//     grid's last CTAs finish; the producer waits for the previous grid before its first
//     copy.
// Every mbarrier wait is bounded: a wait that runs out records bit 0 of g_qs_fault_bits
// (read by qs_device_fault) and the warp leaves instead of hanging the GPU.
#include <cuda.h>  // CUtensorMap; the encoder is resolved at run time through the runtime
#include <mutex>

#include "qs_kernels.h"

namespace qs {

__device__ unsigned int g_qs_fault_bits = 0;

namespace {

constexpr int B32_CW = 8;                         // consumer warps
constexpr int B32_THREADS = (B32_CW + 1) * 32;    // + one producer warp
constexpr int64_t B32_PIECE = int64_t(1) << 31;   // blocks per launch (tensor-map extent limit)

template <int QT> struct B32;
template <> struct B32<QS_Q4_0> { static constexpr int BB = 18; };
template <> struct B32<QS_Q4_1> { static constexpr int BB = 20; };
template <> struct B32<QS_Q5_0> { static constexpr int BB = 22; };
template <> struct B32<QS_Q5_1> { static constexpr int BB = 24; };
template <> struct B32<QS_Q8_0> { static constexpr int BB = 34; };

// Shared memory of one CTA: ring of 1024-byte aligned stages of G x 32 blocks, per-warp
// double-buffered output staging, mbarriers. 16-bit sources: about 64 KB of stages within
// 75 KB, three CTAs per SM (up to 192 KB of copies in flight per SM); f32: about 96 KB, two
// CTAs per SM. G = 1 keeps a multiple of 8 slots, the same number for each warp.
template <int QT, int ES, int G> struct B32Cfg {
    static constexpr int ROWS = 32 * G;  // blocks per stage
    static constexpr int STAGE = ROWS * 32 * ES;
    static constexpr int WST = (32 * B32<QT>::BB + 15) / 16 * 16;  // one warp's staging
    static constexpr int BUDGET = ES == 2 ? 75 * 1024 : 110 * 1024;
    static constexpr int N0 = (BUDGET - 2 * B32_CW * WST - 512) / STAGE;
    static constexpr int NSLOT = G == 1 ? (N0 / 8 < 2 ? 16 : N0 / 8 * 8) : (N0 < 2 ? 2 : N0);
    static constexpr int BYTES = NSLOT * STAGE + 2 * B32_CW * WST + 16 * NSLOT;
    static constexpr int MIN_CTAS = ES == 2 ? 3 : 2;
};

// --- mbarrier / TMA primitives ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
// The box of rows [y, ...) of the block tensor into `dst` (the whole box is always written:
// rows past the tensor's end are zero-filled), completing `bytes` on the barrier.
__device__ __forceinline__ void tensor_load(uint32_t dst, const CUtensorMap* map, int y, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%3], %2; }\n"
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%4, %5}], [%3];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bytes), "r"(bar), "r"(0), "r"(y) : "memory");
}
// Wait for the completion of phase `parity`; false after a bounded number of polls (each
// poll may suspend for a hardware-defined slice; with the back-off the bound is seconds).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (int it = 0; it < (1 << 20); it++) {
        uint32_t ok;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
        if (it > 64) __nanosleep(128);
    }
    return false;
}

// Byte offset of 16-byte chunk c of stage row R (the tensor map's swizzle).
template <int ES>
__device__ __forceinline__ int chunk_off(int R, int c) {
    if constexpr (ES == 2) return 64 * R + 16 * (c ^ ((R >> 1) & 3));
    else return 128 * R + 16 * (c ^ (R & 7));
}

// --- per-block arithmetic ----------------------------------------------------------------
// Low bytes of four words -> one word (a in byte 0).
__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}
// LSB of each byte of w -> 4 bits, byte j -> bit j.
__device__ __forceinline__ uint32_t byte_lsbs(uint32_t w) { return ((w & 0x01010101u) * 0x01020408u) >> 24; }

// Source element size of a GGML source type.
template <int SRC> __host__ __device__ constexpr int es_of() { return SRC == SRC_F32 ? 4 : 2; }

// One block of 32 values in block order: 16-bit sources keep the 16 packed words, f32 the
// floats. The source type is a template parameter, so each value costs one conversion.
template <int SRC> struct Blk {
    uint32_t w[16];
    __device__ __forceinline__ float at(int i) const {
        if constexpr (SRC == SRC_BF16) return __uint_as_float((i & 1) ? (w[i >> 1] & 0xFFFF0000u) : (w[i >> 1] << 16));
        else return __half2float(__ushort_as_half((unsigned short)((i & 1) ? (w[i >> 1] >> 16) : (w[i >> 1] & 0xFFFFu))));
    }
};
template <> struct Blk<SRC_F32> {
    float x[32];
    __device__ __forceinline__ float at(int i) const { return x[i]; }
};

template <int SRC>
__device__ __forceinline__ void load_block(const uint8_t* stage, int R, Blk<SRC>& B) {
    constexpr int ES = es_of<SRC>();
#pragma unroll
    for (int c = 0; c < 2 * ES; c++) {
        const uint4 t = *reinterpret_cast<const uint4*>(stage + chunk_off<ES>(R, c));
        if constexpr (ES == 2) {
            B.w[4 * c] = t.x; B.w[4 * c + 1] = t.y; B.w[4 * c + 2] = t.z; B.w[4 * c + 3] = t.w;
        } else {
            B.x[4 * c] = __uint_as_float(t.x); B.x[4 * c + 1] = __uint_as_float(t.y);
            B.x[4 * c + 2] = __uint_as_float(t.z); B.x[4 * c + 3] = __uint_as_float(t.w);
        }
    }
}

// Block max and min as trees (order-free; the sign of a tied zero is settled separately).
template <typename H>
__device__ __forceinline__ void max_min_16(const uint32_t* w, float& mx, float& mn) {
    H hx[8], hn[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const H a = *reinterpret_cast<const H*>(&w[i]), b = *reinterpret_cast<const H*>(&w[i + 8]);
        hx[i] = __hmax2(a, b);
        hn[i] = __hmin2(a, b);
    }
#pragma unroll
    for (int h = 4; h > 0; h >>= 1)
#pragma unroll
        for (int i = 0; i < h; i++) { hx[i] = __hmax2(hx[i], hx[i + h]); hn[i] = __hmin2(hn[i], hn[i + h]); }
    mx = fmaxf(__low2float(hx[0]), __high2float(hx[0]));
    mn = fminf(__low2float(hn[0]), __high2float(hn[0]));
}
template <int SRC>
__device__ __forceinline__ void max_min(const Blk<SRC>& B, float& mx, float& mn) {
    if constexpr (SRC == SRC_BF16) {
        max_min_16<__nv_bfloat162>(B.w, mx, mn);
    } else if constexpr (SRC == SRC_F16) {
        max_min_16<__half2>(B.w, mx, mn);
    } else {
        float a[16], b[16];
#pragma unroll
        for (int i = 0; i < 16; i++) { a[i] = fmaxf(B.x[i], B.x[i + 16]); b[i] = fminf(B.x[i], B.x[i + 16]); }
#pragma unroll
        for (int h = 8; h > 0; h >>= 1)
#pragma unroll
            for (int i = 0; i < h; i++) { a[i] = fmaxf(a[i], a[i + h]); b[i] = fminf(b[i], b[i + h]); }
        mx = a[0];
        mn = b[0];
    }
}

// v if v > a (resp. v < a) else a, as a compare and a select: the compiler may not turn
// these into max / min instructions, which order -0 below +0 instead of keeping `a`.
__device__ __forceinline__ float keep_gt(float v, float a) {
    float r;
    asm("{ .reg .pred p; setp.gt.f32 p, %1, %2; selp.f32 %0, %1, %2, p; }" : "=f"(r) : "f"(v), "f"(a));
    return r;
}
__device__ __forceinline__ float keep_lt(float v, float a) {
    float r;
    asm("{ .reg .pred p; setp.lt.f32 p, %1, %2; selp.f32 %0, %1, %2, p; }" : "=f"(r) : "f"(v), "f"(a));
    return r;
}

// Signed value of the first largest |x| (argmax of |x|, first index): max and min decide
// it unless both +a and -a occur, or the block is all zeros (the first zero's sign).
template <int SRC>
__device__ __forceinline__ float first_absmax(float mx, float mn, const Blk<SRC>& B) {
    if (mx != -mn) return mx > -mn ? mx : mn;
    float m = B.at(0), am = fabsf(m);
#pragma unroll
    for (int i = 1; i < 32; i++) {
        const float v = B.at(i);
        const bool gt = fabsf(v) > am;
        am = gt ? fabsf(v) : am;
        m = gt ? v : m;
    }
    return m;
}

// ggml's scalar max / min (`if (v > max) max = v`, the first of tied values kept): only the
// sign of a zero result can differ from the order-free trees, so the scalar loop runs only
// when a result is zero.
template <int SRC>
__device__ __forceinline__ void first_max_min(float& mx, float& mn, const Blk<SRC>& B) {
    if (mx != 0.0f && mn != 0.0f) return;
    float a = B.at(0), b = a;
#pragma unroll
    for (int i = 1; i < 32; i++) {
        const float v = B.at(i);
        a = keep_gt(v, a);
        b = keep_lt(v, b);
    }
    mx = a;
    mn = b;
}

// --- packing on the FMA pipe ----------------------------------------------------------------
// floor(v) for v in [0, 2^23): v + 2^23 added rounding toward -infinity is the float
// 2^23 + floor(v), whose bits are 0x4B000000 + floor(v) (the "floor bits" of v). Multiplying
// those by 2^8, 2^16 or 2^24 modulo 2^32 drops the 0x4B000000 term, so four levels pack into
// one word with integer multiply-adds (IMAD, FMA pipe) instead of byte permutes on the ALU pipe.
__device__ __forceinline__ uint32_t mad_lo(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t mul_hi(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// bytes n0 | n1 << 8 | n2 << 16 | n3 << 24 from the floor bits of four levels
__device__ __forceinline__ uint32_t pack_levels(uint32_t f0, uint32_t f1, uint32_t f2, uint32_t f3) {
    return mad_lo(f3, 1u << 24, mad_lo(f2, 1u << 16, mad_lo(f1, 1u << 8, f0 - 0x4B000000u)));
}
// qs words of the 4-bit formats from the low (values j) and high (values j + 16) level words
// whose bytes are <= 16: clamp each byte to 15 and combine, lo + 16 * hi with the 16s taken
// out: lo - ((lo & 0x10..) >> 4) + 16 * hi - (hi & 0x10..).
__device__ __forceinline__ uint32_t qs_clamp16(uint32_t lo, uint32_t hi) {
    const uint32_t t = lo & 0x10101010u, u = hi & 0x10101010u;
    return mad_lo(hi, 16u, lo) - mul_hi(t, 1u << 28) - u;
}

// Lane l's record to bytes [l * BB, (l + 1) * BB) of the warp's staging, with 32-bit stores
// (all 32 lanes call it). BB = 2 mod 4 (Q4_0, Q5_0, Q8_0): a lane pair's two records span
// whole words from the even lane's start; the even lane also writes its partner's first 2
// bytes (shuffled over), the odd lane the rest of its own record, shifted by 2 bytes.
template <int BB>
__device__ __forceinline__ void put_record(uint8_t* os, int lane, const uint32_t* rec) {
    if constexpr (BB % 4 == 0) {
#pragma unroll
        for (int i = 0; i < BB / 4; i++) reinterpret_cast<uint32_t*>(os + lane * BB)[i] = rec[i];
    } else {
        constexpr int H = (BB - 2) / 4;  // whole words before a record's last 2 bytes
        const uint32_t first = __shfl_down_sync(0xffffffffu, rec[0], 1);
        uint32_t* w = reinterpret_cast<uint32_t*>(os + (lane & ~1) * BB);  // the pair's first word
        if ((lane & 1) == 0) {
#pragma unroll
            for (int i = 0; i < H; i++) w[i] = rec[i];
            w[H] = (rec[H] & 0xFFFFu) | (first << 16);
        } else {
#pragma unroll
            for (int i = 0; i < H; i++) w[H + 1 + i] = __funnelshift_r(rec[i], rec[i + 1], 16);
        }
    }
}

// Levels of the 4- / 5-bit formats into [d][qh][qs] records: qs byte j = level j | level
// (j + 16) << 4, qh bit j = level j >> 4. W: levels, 4 per word, block order.
__device__ __forceinline__ void nibbles(const uint32_t* W, uint32_t* qs) {
#pragma unroll
    for (int m = 0; m < 4; m++) qs[m] = (W[m] & 0x0F0F0F0Fu) | ((W[m + 4] & 0x0F0F0F0Fu) << 4);
}
__device__ __forceinline__ uint32_t high_bits(const uint32_t* W) {
    uint32_t h = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) h |= byte_lsbs(W[k] >> 4) << (4 * k);
    return h;
}

// Quantize the block of stage row R into the record words rec (BB bytes, little-endian).
template <int QT, int SRC>
__device__ __forceinline__ void quantize_block(const uint8_t* stage, int R, uint32_t* rec) {
    Blk<SRC> B;
    load_block<SRC>(stage, R, B);
    float mx, mn;
    max_min<SRC>(B, mx, mn);
    uint32_t W[8];  // level bytes, 4 per word, block order
    if constexpr (QT == QS_Q4_0 || QT == QS_Q5_0) {
        // kernels/q4_0.py:20-28: d = max / -8 (max * -0.125, the same value), id = 1 / d,
        // q = clamp(floor(x * id + 8.5), 0, 15). Q5_0: d = max / -16, q = clip(trunc(x * id
        // + 16.5), 0, 31) (the argument is >= 0, so trunc == floor). |x * id| <= 8 (16) up to
        // rounding, so the floors lie in 0..16 (0..32) and only the top value is clamped,
        // by subtracting bit 4 (5) of each byte. An infinite id (|d| below 2^-128) makes every
        // x * id + off infinite or NaN: the levels then follow the casts of the two
        // references, torch's clamp + uint8 for Q4_0 (+inf -> 15, -inf / NaN -> 0) and ggml's
        // / numpy's int cast for Q5_0 (0).
        const float m = first_absmax<SRC>(mx, mn, B);
        const float d = QT == QS_Q4_0 ? m * -0.125f : m * -0.0625f;
        const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        constexpr float off = QT == QS_Q4_0 ? 8.5f : 16.5f;
        uint32_t qs[4];
        if (!isinf(id)) {
            // x * id, + off and the floor add, two values per packed f32x2 instruction (one
            // rounding each, as the scalar ones; the product as f2_mul_z, whose +0 for a -0
            // product the + off cannot tell apart)
            const f32x2 id2 = f2_splat(id), off2 = f2_splat(off), big2 = f2_splat(8388608.0f);
#pragma unroll
            for (int k = 0; k < 8; k++) {
                uint32_t fb[4];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const f32x2 y = f2_mul_z(f2_pack(B.at(4 * k + 2 * h), B.at(4 * k + 2 * h + 1)), id2);
                    f2_unpack_bits(f2_add_rm(f2_add(y, off2), big2), fb[2 * h], fb[2 * h + 1]);
                }
                W[k] = pack_levels(fb[0], fb[1], fb[2], fb[3]);
            }
            if constexpr (QT == QS_Q4_0) {
#pragma unroll
                for (int j = 0; j < 4; j++) qs[j] = qs_clamp16(W[j], W[j + 4]);
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) W[k] -= mul_hi(W[k] & 0x20202020u, 1u << 27);  // 32 -> 31
                nibbles(W, qs);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                uint32_t w = 0;
                if constexpr (QT == QS_Q4_0) {
#pragma unroll
                    for (int j = 0; j < 4; j++) w |= (B.at(4 * k + j) * id + off == INFINITY ? 15u : 0u) << (8 * j);
                }
                W[k] = w;
            }
            nibbles(W, qs);
        }
        const uint32_t dh = f16_bits(d);
        if constexpr (QT == QS_Q4_0) {  // [d][qs 16]
            rec[0] = dh | (qs[0] << 16);
#pragma unroll
            for (int i = 1; i < 4; i++) rec[i] = (qs[i - 1] >> 16) | (qs[i] << 16);
            rec[4] = qs[3] >> 16;
        } else {  // [d][qh 4][qs 16]
            const uint32_t qh = high_bits(W);
            rec[0] = dh | (qh << 16);
            rec[1] = (qh >> 16) | (qs[0] << 16);
#pragma unroll
            for (int i = 2; i < 5; i++) rec[i] = (qs[i - 2] >> 16) | (qs[i - 1] << 16);
            rec[5] = qs[3] >> 16;
        }
    } else if constexpr (QT == QS_Q4_1 || QT == QS_Q5_1) {
        // quantize_row_q4_1_ref / q5_1_ref: d = (max - min) / nmax, id = 1 / d (0 if d == 0),
        // q = min(trunc((x - min) * id + 0.5), nmax), m = min. (x - min) * id <= nmax up to a
        // few ulps, so the floors never exceed nmax; an infinite id (d below 2^-128) makes
        // every level inf / NaN, which the int cast of the references turns into 0: an id of
        // 0 gives those zeros through the same arithmetic.
        first_max_min<SRC>(mx, mn, B);
        const float d = __fdiv_rn(mx - mn, QT == QS_Q4_1 ? 15.0f : 31.0f);
        float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        id = isinf(id) ? 0.0f : id;
        // x - mn, * id, + 0.5 and the floor add on packed f32x2, two values per instruction
        // (x - mn >= +0 and id >= 0: the +0-addend product is the exact product here)
        const f32x2 mn2 = f2_splat(mn), id2 = f2_splat(id), half2 = f2_splat(0.5f), big2 = f2_splat(8388608.0f);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            uint32_t fb[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const f32x2 y = f2_mul_z(f2_sub(f2_pack(B.at(4 * k + 2 * h), B.at(4 * k + 2 * h + 1)), mn2), id2);
                f2_unpack_bits(f2_add_rm(f2_add(y, half2), big2), fb[2 * h], fb[2 * h + 1]);
            }
            W[k] = pack_levels(fb[0], fb[1], fb[2], fb[3]);
        }
        uint32_t qs[4];
        if constexpr (QT == QS_Q4_1) {
#pragma unroll
            for (int j = 0; j < 4; j++) qs[j] = mad_lo(W[j + 4], 16u, W[j]);  // levels <= 15
        } else {
            nibbles(W, qs);
        }
        rec[0] = f16_bits(d) | ((uint32_t)f16_bits(mn) << 16);
        if constexpr (QT == QS_Q4_1) {  // [d][m][qs 16]
#pragma unroll
            for (int i = 0; i < 4; i++) rec[1 + i] = qs[i];
        } else {  // [d][m][qh 4][qs 16]
            rec[1] = high_bits(W);
#pragma unroll
            for (int i = 0; i < 4; i++) rec[2 + i] = qs[i];
        }
    } else {
        // quantize_row_q8_0_ref: d = max|x| / 127, id = 1 / d (0 if d == 0), q = roundf(x * id)
        // (half away from zero) as int8; non-finite -> 0
        const float amax = fmaxf(fabsf(mx), fabsf(mn));
        const float d = __fdiv_rn(amax, 127.0f);
        float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
        id = isinf(id) ? 0.0f : id;  // every level inf / NaN -> 0 in the references' int cast
#pragma unroll
        for (int k = 0; k < 8; k++)
            W[k] = pack4((uint32_t)(int)roundf(B.at(4 * k) * id), (uint32_t)(int)roundf(B.at(4 * k + 1) * id),
                         (uint32_t)(int)roundf(B.at(4 * k + 2) * id), (uint32_t)(int)roundf(B.at(4 * k + 3) * id));
        rec[0] = f16_bits(d) | (W[0] << 16);
#pragma unroll
        for (int i = 1; i < 8; i++) rec[i] = (W[i - 1] >> 16) | (W[i] << 16);
        rec[8] = W[7] >> 16;
    }
}

// Blocks [base, base + a.nblk) of the tensor in one launch (the tensor map starts at `base`),
// in stages of G x 32 blocks.
template <int QT, int SRC, int G>
__global__ void __launch_bounds__(B32_THREADS, B32Cfg<QT, es_of<SRC>(), G>::MIN_CTAS)
    blk32_kernel(const __grid_constant__ CUtensorMap map, QuantArgs a, int64_t base) {
    constexpr int ES = es_of<SRC>();
    using C = B32Cfg<QT, ES, G>;
    constexpr int BB = B32<QT>::BB, NSLOT = C::NSLOT, STAGE = C::STAGE, ROWS = C::ROWS;
    extern __shared__ __align__(1024) uint8_t b32_smem_raw[];
    uint8_t* ring = b32_smem_raw;
    uint8_t* wstage = ring + NSLOT * STAGE;                                      // [CW][2][WST]
    uint64_t* full = reinterpret_cast<uint64_t*>(wstage + 2 * B32_CW * C::WST);  // [NSLOT]
    uint64_t* empty = full + NSLOT;                                              // [NSLOT]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the swizzle arithmetic needs 1024-byte aligned stages
    if (smem_u32(ring) & 1023) {
        if (threadIdx.x == 0) atomicOr(&g_qs_fault_bits, 2u);
        return;
    }

    // this CTA's blocks [b_begin, b_end) of the piece: groups of 8 spread evenly over the grid
    const int64_t ngroups = (a.nblk + 7) / 8;
    const int64_t g0 = (int64_t)blockIdx.x * ngroups / gridDim.x, g1 = (int64_t)(blockIdx.x + 1) * ngroups / gridDim.x;
    const int64_t b_begin = 8 * g0, b_end = min(8 * g1, a.nblk);
    const int nstage = (int)((b_end - b_begin + ROWS - 1) / ROWS);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), G);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // the next launch on the stream may start its CTAs (they take SM room only as this
        // grid's CTAs leave, and wait for its completion before reading their inputs)
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    __syncthreads();

    if (warp == B32_CW) {  // producer
        if (lane != 0) return;
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");
        // under programmatic launch, the previous grid on the stream (which may write this
        // launch's source, or its destination) completes and its writes become visible here;
        // the consumers read nothing global and write only after a stage arrives, so the
        // producer's wait orders the whole CTA (a no-op for an ordinary launch)
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int j = 0; j < nstage; j++) {
            const int slot = j % NSLOT;
            if (j >= NSLOT && !mbar_wait(smem_u32(&empty[slot]), (uint32_t)(j / NSLOT - 1) & 1u)) {
                atomicOr(&g_qs_fault_bits, 1u);
                return;
            }
            tensor_load(smem_u32(ring + slot * STAGE), &map, (int)(b_begin + (int64_t)j * ROWS), STAGE,
                        smem_u32(&full[slot]));
        }
        return;
    }

    // consumers: G = 8, every stage, warp w taking rows 32 w .. 32 w + 31; G = 1, stages
    // w, w + 8, ...; lane l quantizes the warp's row l
    const bool contiguous = a.dst_row_bytes == a.row_bytes;
    const int R = (G == 1 ? 0 : warp * 32) + lane;
    uint8_t* mystage = wstage + warp * 2 * C::WST;
    for (int i = G == 1 ? warp : 0, k = 0; i < nstage; i += G == 1 ? B32_CW : 1, k++) {
        const int slot = i % NSLOT;
        const int64_t b0 = b_begin + (int64_t)i * ROWS + (G == 1 ? 0 : warp * 32);
        const int nb = (int)max((int64_t)0, min((int64_t)32, b_end - b0));
        __syncwarp();  // every lane is done with the staging written two stages ago
        if (!mbar_wait(smem_u32(&full[slot]), (uint32_t)(i / NSLOT) & 1u)) {
            if (lane == 0) atomicOr(&g_qs_fault_bits, 1u);
            return;
        }
        uint8_t* os = mystage + (k & 1) * C::WST;
        uint32_t rec[(BB + 3) / 4];
        if (lane < nb) quantize_block<QT, SRC>(ring + slot * STAGE, R, rec);
        put_record<BB>(os, lane, rec);  // the whole warp: paired lanes share words
        __syncwarp();  // the warp's reads of the slot and writes of the staging are done
        if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
        uint8_t* d = a.dst + (base + b0) * BB;
        if (nb == 32 && contiguous && ((uintptr_t)d & 15) == 0) {
            // the usual case: 32 whole records, a 16-byte aligned span of 2 * BB chunks
            const uint4* s4 = reinterpret_cast<const uint4*>(os);
            uint4* d4 = reinterpret_cast<uint4*>(d);
#pragma unroll
            for (int c = lane; c < 2 * BB; c += 32) d4[c] = s4[c];
        } else if (nb > 0) {
            if (contiguous)
                store_bytes(d, os, nb * BB, lane, 32);
            else
                store_tile(a, os, base + b0, nb, BB, lane, 32);
        }
    }
}

// cuTensorMapEncodeTiled, looked up once through the runtime (no direct libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

template <int QT, int SRC, int G>
cudaError_t launch_g(const QuantArgs& p, int64_t base, int grid, const LaunchCtx& ctx) {
    constexpr int ES = es_of<SRC>();
    using C = B32Cfg<QT, ES, G>;
    EncodeTiledFn encode = encode_tiled();
    if (!encode) return cudaErrorNotSupported;
    auto k = blk32_kernel<QT, SRC, G>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
    if (e != cudaSuccess) return e;
    // the piece's blocks as a (p.nblk rows) x (32 values) tensor, one stage = ROWS rows
    CUtensorMap map;
    const cuuint64_t dims[2] = {32, (cuuint64_t)p.nblk};
    const cuuint64_t strides[1] = {32 * ES};
    const cuuint32_t box[2] = {32, (cuuint32_t)C::ROWS};
    const cuuint32_t estr[2] = {1, 1};
    void* gaddr = const_cast<uint8_t*>(static_cast<const uint8_t*>(p.src) + base * 32 * ES);
    if (encode(&map, ES == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, gaddr, dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, ES == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    // programmatic stream serialization: this launch's prologue (barrier set-up, tensor-map
    // prefetch) overlaps the tail of the previous kernel on the stream
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(B32_THREADS);
    cfg.dynamicSmemBytes = C::BYTES;
    cfg.stream = ctx.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, map, p, base);
}

template <int QT, int SRC>
cudaError_t launch_t(const QuantArgs& a, const LaunchCtx& ctx) {
    constexpr int ES = es_of<SRC>();
    using C = B32Cfg<QT, ES, 8>;
    static_assert(B32Cfg<QT, ES, 1>::BYTES <= C::BYTES + 1024, "both stage shapes fit the same CTAs per SM");
    auto k = blk32_kernel<QT, SRC, 8>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, B32_THREADS, C::BYTES) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    for (int64_t base = 0; base < a.nblk; base += B32_PIECE) {
        QuantArgs p = a;
        p.nblk = min(B32_PIECE, a.nblk - base);
        const int64_t want = (p.nblk + C::ROWS - 1) / C::ROWS;  // at least one large stage per CTA
        const int grid = (int)min((int64_t)per_sm * ctx.num_sms, max(want, (int64_t)1));
        // fewer than 8 large stages per CTA: the small stages
        e = p.nblk < (int64_t)grid * 8 * C::ROWS ? launch_g<QT, SRC, 1>(p, base, grid, ctx)
                                                  : launch_g<QT, SRC, 8>(p, base, grid, ctx);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
template <int QT>
cudaError_t launch_q(const QuantArgs& a, const LaunchCtx& ctx) {
    switch (a.src_type) {
    case SRC_F32: return launch_t<QT, SRC_F32>(a, ctx);
    case SRC_F16: return launch_t<QT, SRC_F16>(a, ctx);
    default: return launch_t<QT, SRC_BF16>(a, ctx);
    }
}

}  // namespace

bool is_blk32(int type) {
    return type == QS_Q4_0 || type == QS_Q4_1 || type == QS_Q5_0 || type == QS_Q5_1 || type == QS_Q8_0;
}

cudaError_t launch_blk32(int type, const QuantArgs& a, const LaunchCtx& ctx) {
    switch (type) {
    case QS_Q4_0: return launch_q<QS_Q4_0>(a, ctx);
    case QS_Q4_1: return launch_q<QS_Q4_1>(a, ctx);
    case QS_Q5_0: return launch_q<QS_Q5_0>(a, ctx);
    case QS_Q5_1: return launch_q<QS_Q5_1>(a, ctx);
    case QS_Q8_0: return launch_q<QS_Q8_0>(a, ctx);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t read_fault_bits(unsigned int* bits, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(bits, g_qs_fault_bits, sizeof(unsigned int));
    if (e != cudaSuccess || !clear || *bits == 0) return e;
    const unsigned int zero = 0;
    return cudaMemcpyToSymbol(g_qs_fault_bits, &zero, sizeof(unsigned int));
}

}  // namespace qs
