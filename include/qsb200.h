/*
 * qsb200: B200 (sm_100a) GGUF block quantizers behind a plain C ABI.
 *
 * Drop-in boundary for the per-type kernels of ngxson/quant-studio. In the reference a
 * kernel is obtained as `QuantSpec.make_kernel(device, qw)` (kernels/common.py:27-37)
 * and called as `quant_fn(x)` on an (n_rows, k) float32 device tensor, returning a
 * new (n_rows, k // QK * block_bytes) uint8 tensor (quant-studio.py:456, :198). The
 * entry points below replace that call: the caller owns every buffer, passes the
 * source rows in bf16 / f16 / f32 directly (the reference's f32 upcast at
 * quant-studio.py:197 is not needed) and a CUDA stream; work is enqueued on that
 * stream and the call returns without synchronizing.
 *
 * Type ids are gguf GGMLQuantizationType values; source types are GGML F32 (0),
 * F16 (1) and BF16 (30). Every function returns QS_OK (0) or a negative QS_E* code;
 * qs_last_error() gives the message of the calling thread's last failure.
 *
 * Devices: a call runs on the GPU that owns its first device pointer (src, or out for the
 * tensor error sums), whatever device the caller has current; every other pointer of the
 * call must be memory of that same GPU (or managed memory), else QS_EINVAL. The calling
 * thread's current CUDA context is the same on return as it was on entry.
 */
#ifndef QSB200_H
#define QSB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QSB200_VERSION 1

#define QS_OK 0
#define QS_EINVAL (-1)    /* bad argument: type, k, alignment, null pointer, stride */
#define QS_ECUDA (-2)     /* a CUDA call failed; see qs_last_error() */
#define QS_ENOTSUP (-3)   /* type id not implemented */
#define QS_ENOIMAT (-4)   /* the type needs importance weights and qw was NULL */

/* GGML type ids this library quantizes to (gguf GGMLQuantizationType). */
#define QS_TYPE_Q4_0 2
#define QS_TYPE_Q4_1 3   /* Q4_1 / Q5_0 / Q5_1 / Q8_0: no kernel in the reference (see qs_quantize) */
#define QS_TYPE_Q5_0 6
#define QS_TYPE_Q5_1 7
#define QS_TYPE_Q8_0 8
#define QS_TYPE_Q2_K 10
#define QS_TYPE_Q3_K 11
#define QS_TYPE_Q4_K 12
#define QS_TYPE_Q5_K 13
#define QS_TYPE_Q6_K 14
#define QS_TYPE_IQ2_XXS 16
#define QS_TYPE_IQ2_XS 17
#define QS_TYPE_IQ3_XXS 18
#define QS_TYPE_IQ3_S 21
#define QS_TYPE_IQ2_S 22
#define QS_TYPE_IQ4_XS 23

/* Source element types (GGML ids); the reference's TORCH_DTYPES (kernels/common.py:20-24). */
#define QS_SRC_F32 0
#define QS_SRC_F16 1
#define QS_SRC_BF16 30

/* Library version (QSB200_VERSION). */
int qs_version(void);

/* Prepare `device` (SM count, lattice tables). Idempotent and thread-safe; qs_quantize
 * calls it lazily for the current device. Replaces the per-device table caches of the
 * reference (kernels/iq2.py:77-84 tables_for, iq2xs_common.py:98-106, iq3_common.py:78-85). */
int qs_init(int device);

/* 1 if `ggml_type` is implemented, else 0 (the reference's QUANT_TYPES registry,
 * kernels/__init__.py:18-27). */
int qs_type_supported(int ggml_type);

/* 1 if the kernel cannot run without importance weights (IQ2_XXS, IQ2_XS, IQ2_S:
 * kernels/iq2.py:418, iq2_xs.py:20, iq2_s.py:21 take qw unconditionally). */
int qs_type_needs_qw(int ggml_type);

/* Block geometry: values per block (*qk) and packed bytes per block (*block_bytes);
 * the gguf GGML_QUANT_SIZES entry the reference uses (quant-studio.py:143-145). */
int qs_block_info(int ggml_type, int* qk, int* block_bytes);

/* Packed bytes of one row of k values: k / qk * block_bytes (quant-studio.py:143-145). */
int qs_row_bytes(int ggml_type, int64_t k, int64_t* out_bytes);

/*
 * Quantize n_rows x k source values into packed GGML blocks.
 * Replaces quant_fn(x) (the `quantize_<type>(x, qw)` functions, e.g.
 * kernels/q4_k.py:25-79, kernels/iq2.py:418-498) as called at quant-studio.py:198.
 *   src            device pointer, n_rows x k elements of src_type, rows contiguous,
 *                  16-byte aligned
 *   qw             device pointer to k float32 importance weights (16-byte aligned),
 *                  or NULL for the no-imatrix variant
 *   dst            device pointer; row r is written at dst + r * dst_row_bytes
 *   dst_row_bytes  >= qs_row_bytes(type, k)
 *   stream         cudaStream_t (NULL = legacy default stream)
 * Output bytes are identical to the reference's eager CPU path for the same values.
 * Q4_1, Q5_0, Q5_1 and Q8_0 have no kernel in the reference, whose type-mix policy still
 * selects them (kernels/scheme.py:375 shape fallbacks, :521-523 ffn_down under Q4_0 / Q5_0
 * with an importance matrix) and whose CLI then stops (quant-studio.py:396-399); here they
 * give the bytes of gguf-py's quantize_blocks for those types (the ggml-quants.c reference
 * rows) and, like the reference's Q4_0, ignore qw.
 */
int qs_quantize(int ggml_type, const void* src, int src_type, int64_t n_rows, int64_t k,
                const float* qw, void* dst, int64_t dst_row_bytes, void* stream);

/*
 * Decode n_rows rows of packed blocks to float32: the GGUF dequantization of every type
 * above, value for value what gguf-py's gguf.quants.dequantize returns (the decode the
 * reference's correctness harness compares with, tools/dev_harness.py:108-109).
 *   src             device pointer; row r starts at src + r * src_row_bytes
 *   src_row_bytes   >= qs_row_bytes(type, k)
 *   dst             device pointer, 16-byte aligned; row r at dst + r * dst_row_stride
 *   dst_row_stride  elements, a multiple of 4, >= k
 */
int qs_dequantize(int ggml_type, const void* src, int64_t src_row_bytes, int64_t n_rows, int64_t k,
                  float* dst, int64_t dst_row_stride, void* stream);

/*
 * Squared error of every decoded block against the source values:
 *   err[r * (k / qk) + j] = sum over the values of block j of row r of w * (deq - x)^2,
 *   w = qw[column], or 1 when qw is NULL. Each term is a float32 product as the harness
 *   computes it; each run of 8 consecutive values is summed left to right in float32,
 *   and those partial sums in double.
 * The per-block form of the harness's decoded-error check (tools/dev_harness.py:110-112).
 *   blocks, blocks_row_bytes   as src / src_row_bytes of qs_dequantize
 *   x, x_type                  n_rows x k source values (F32 / F16 / BF16), rows
 *                              contiguous, 16-byte aligned
 *   qw                         k float32 weights (16-byte aligned) or NULL
 *   err                        device pointer to n_rows * (k / qk) doubles
 */
int qs_block_error(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x, int x_type,
                   int64_t n_rows, int64_t k, const float* qw, double* err, void* stream);

/*
 * Error sums over the whole tensor (terms and 8-value runs as qs_block_error), the runs
 * added in double in a fixed order (the same bits on every call on the same GPU model):
 *   out[0] = sum w * (deq - x)^2, out[1] = sum (deq - x)^2   (out: 2 device doubles, 8-byte aligned)
 * out[1] / (n_rows * k) is the `((dq - xf) ** 2).mean()` of tools/dev_harness.py:110-111.
 * Arguments as qs_block_error. Scratch for the per-CTA partial sums comes from the
 * library's per-device memory pool, stream-ordered on `stream` (cudaMallocFromPoolAsync /
 * cudaFreeAsync); the pool keeps its memory between calls.
 */
int qs_tensor_error(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x, int x_type,
                    int64_t n_rows, int64_t k, const float* qw, double* out, void* stream);

/* Capacity of the static scratch of qs_tensor_error_noalloc, in per-CTA partial sums. */
#define QS_NOALLOC_MAX_PARTIALS 4096

/*
 * qs_tensor_error without any allocation. No counterpart in the reference (its harness
 * sums the decoded error on the host, tools/dev_harness.py:110-111); an addition of this
 * library for callers that may not allocate device memory.
 * Same arguments, same kernels and the same result bits as qs_tensor_error, but the
 * per-CTA partial sums live in a fixed static device array of QS_NOALLOC_MAX_PARTIALS
 * pairs of doubles (64 KiB per device) and the IQ codebooks in a 5 KiB static device
 * array: no cudaMalloc, no pool, no library allocator on any call. The launch uses one
 * partial sum per CTA, at most 8 CTAs per SM; a launch that would need more than
 * QS_NOALLOC_MAX_PARTIALS (a GPU with more than 512 SMs) is rejected with QS_EINVAL before
 * anything is enqueued. Nothing in the static scratch needs to start at zero: each CTA
 * writes its own pair before the final pass reads them.
 * Overlapping calls on one device (concurrent streams or host threads) share the static
 * scratch and race; callers must serialize them.
 * Set-up: the first call on each device, with that device current, resolves the static
 * arrays (cudaGetSymbolAddress) and copies the codebooks in (a synchronous copy); make
 * that first call outside any stream capture. Like every entry point here, the call
 * leaves the caller's current context as it found it.
 */
int qs_tensor_error_noalloc(int ggml_type, const void* blocks, int64_t blocks_row_bytes, const void* x,
                            int x_type, int64_t n_rows, int64_t k, const float* qw, double* out, void* stream);

/*
 * Fault word of `device`: bit 0 is set when a quantize kernel gave up waiting for one of its
 * own bulk copies (every wait in the kernels is bounded; on that path the kernel records
 * the fault and returns instead of hanging the GPU). Synchronous; clears the word.
 * No counterpart in the reference (its kernels have no waits).
 */
int qs_device_fault(int device, int* bits);

/* Message of the calling thread's last failure ("" if none). */
const char* qs_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QSB200_H */
