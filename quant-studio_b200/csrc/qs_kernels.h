// Internal interface between the C ABI (qs_api.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "qs_common.cuh"

namespace qs {

// GGML type ids (gguf GGMLQuantizationType)
enum QsType : int {
    QS_Q4_0 = 2, QS_Q4_1 = 3, QS_Q5_0 = 6, QS_Q5_1 = 7, QS_Q8_0 = 8, QS_Q2_K = 10, QS_Q3_K = 11, QS_Q4_K = 12, QS_Q5_K = 13, QS_Q6_K = 14,
    QS_IQ2_XXS = 16, QS_IQ2_XS = 17, QS_IQ3_XXS = 18, QS_IQ3_S = 21, QS_IQ2_S = 22, QS_IQ4_XS = 23,
};

// Candidate tables passed by value (kernel parameter space).
struct KParams {
    float steps[40];  // make_qkx candidate numerators
    int nsteps;
    float qp[8];      // make_qp candidate numerators
    float qx[18];     // make_qx candidates for the group fit
    float qx2[18];    // make_qx candidates for the Q3_K superblock scale fit (nmax 32)
};

struct LaunchCtx {
    cudaStream_t stream;
    int device;
    int num_sms;
};

struct IqTables;  // per-device lattice tables (qs_iq.cu)

cudaError_t launch_kquant(int type, const QuantArgs& a, const LaunchCtx& ctx);
// 32-value block formats (qs_blk32.cu): Q4_0, Q4_1, Q5_0, Q5_1, Q8_0
bool is_blk32(int type);
cudaError_t launch_blk32(int type, const QuantArgs& a, const LaunchCtx& ctx);
// Fault word of the current device: bit 0 = a kernel gave up waiting for a bulk copy.
// Synchronous; clears the word when `clear` and it is non-zero.
cudaError_t read_fault_bits(unsigned int* bits, bool clear);
cudaError_t launch_iq(int type, const QuantArgs& a, const LaunchCtx& ctx, const IqTables* t);
cudaError_t iq_tables_create(IqTables** out);  // uploads the codebooks to the current device
cudaError_t iq_tables_ensure(IqTables* t, int type);  // neighbour tables of type's grid, once
void iq_tables_destroy(IqTables* t);
const uint16_t* iq_kgrid(const IqTables* t, int type);  // IQ codebook (grid index -> code), else null

// One decode / decode-error pass (qs_dequant.cu).
struct DqCall {
    const void* blocks;        // packed rows, row r at blocks + r * blocks_row_bytes
    int64_t blocks_row_bytes;
    int64_t n_rows, k;
    float* dst;                // decode: row r at dst + r * dst_stride
    int64_t dst_stride;
    const void* x;             // error passes: n_rows x k source values of x_type
    int x_type;
    const float* qw;           // k weights or null
    double* err;               // block error: one double per block
};

cudaError_t launch_dequant(int type, const DqCall& c, const LaunchCtx& ctx, const IqTables* t);
cudaError_t launch_block_error(int type, const DqCall& c, const LaunchCtx& ctx, const IqTables* t);
// Number of per-CTA partials (2 doubles each) launch_tensor_error writes.
int dq_partial_count(int type, int64_t n_rows, int64_t k, const LaunchCtx& ctx);
// Error sums over the tensor: CTA partials into `partial` (room for npartial), then
// out[0] = sum w (deq - x)^2, out[1] = sum (deq - x)^2 in a fixed order.
cudaError_t launch_tensor_error(int type, const DqCall& c, double* partial, int npartial, double* out,
                                const LaunchCtx& ctx, const IqTables* t);

// qs_tensor_error_noalloc: static device scratch resolved once per device (qs_dequant.cu).
constexpr int NA_MAX_PARTIALS = 4096;  // pairs of doubles: 64 KiB per device
constexpr int NA_MAX_DEVICES = 64;
struct NoAllocDevice {
    bool ready = false;
    int num_sms = 0;
    double* partial = nullptr;        // device address of the static partial sums
    const uint16_t* kgrid = nullptr;  // device address of the static codebooks
};
// With `device` current: resolve the static arrays (cudaGetSymbolAddress) and fill the
// codebooks, once per device; thread-safe.
cudaError_t noalloc_setup(int device, const NoAllocDevice** out);
// qs_tensor_error's launch on the static scratch; cudaErrorInvalidValue if the launch
// needs more than NA_MAX_PARTIALS partial sums (nothing is launched then).
cudaError_t launch_tensor_error_noalloc(int type, const DqCall& c, double* out, const LaunchCtx& ctx,
                                        const NoAllocDevice& d);

}  // namespace qs
