/* CPU oracle for the GGML block quantizers (test infrastructure only). */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids (gguf GGMLQuantizationType) */
enum {
    OQ_Q4_0 = 2, OQ_Q4_1 = 3, OQ_Q5_0 = 6, OQ_Q5_1 = 7, OQ_Q8_0 = 8, OQ_Q2_K = 10, OQ_Q3_K = 11, OQ_Q4_K = 12, OQ_Q5_K = 13, OQ_Q6_K = 14,
    OQ_IQ2_XXS = 16, OQ_IQ2_XS = 17, OQ_IQ3_XXS = 18, OQ_IQ3_S = 21, OQ_IQ2_S = 22, OQ_IQ4_XS = 23,
};

void oq_init(void);
int64_t oq_row_bytes(int type, int64_t k);
/* x: n x k f32 row-major; qw: k f32 or NULL; out: n x row_bytes. Returns 0, -1 (bad type/k), -2 (qw needed). */
int oq_quantize(int type, const float *x, int64_t n, int64_t k, const float *qw, uint8_t *out, int nthreads);

#ifdef __cplusplus
}
#endif
