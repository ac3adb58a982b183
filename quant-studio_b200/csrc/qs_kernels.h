// Internal interface between the C ABI (qs_api.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "qs_common.cuh"

namespace qs {

// GGML type ids (gguf GGMLQuantizationType)
enum QsType : int {
    QS_Q4_0 = 2, QS_Q2_K = 10, QS_Q3_K = 11, QS_Q4_K = 12, QS_Q5_K = 13, QS_Q6_K = 14,
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
cudaError_t launch_iq(int type, const QuantArgs& a, const LaunchCtx& ctx, const IqTables* t);
cudaError_t iq_tables_create(IqTables** out);  // uploads to the current device
void iq_tables_destroy(IqTables* t);

}  // namespace qs
