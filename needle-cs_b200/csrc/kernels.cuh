// Internal launch helpers shared between translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ndl {

int launch_quantize_rows(const float *x, const float *weight, int rows, int cols, int8_t *q, float *scales,
                         cudaStream_t stream);

struct MatmulArgs {
    const int8_t *q;
    const float *sa;
    int m, k;
    const int8_t *w;
    const uint16_t *sw;
    int n;
    float *y;
    int ldy;
    const float *residual;
    int32_t *acc;
    long long w_stride, sw_stride, y_stride;
    int batch;
};

// Streaming int8 GEMV (mma.sync m16n8k32 per 32-column group), any m.
int launch_gemv_i8g32(const MatmulArgs &a, cudaStream_t stream);
// tcgen05 kind::i8 GEMM for m >= 64; returns NDL_ERR_UNSUPPORTED when the
// shape does not fit its tiling so the caller can fall back to the GEMV.
int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream);

}  // namespace ndl
