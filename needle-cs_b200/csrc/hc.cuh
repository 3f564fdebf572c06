// Hyper-connection steps shared by the Needle-3 decoder and the Whistle
// encoder kernels.
#pragma once

#include "common.cuh"

namespace ndl {

// Scalar.Sinkhorn4x4 (src/Needle/Scalar.cs:361-381) on 16 lanes of a warp,
// lane 4 * row + c (within its half-warp) holding logit (row, c): the row
// exponentials after the row peak, then 20 rounds of row and column
// normalisation.  Each row or column sum gathers its four entries by
// shuffles and adds them in index order, and every lane divides its own
// entry, so the steps and roundings are the scalar loop's with sixteen
// divisions in parallel.  All 32 lanes must call it (each half-warp holds
// one matrix); returns the lane's entry.
__device__ __forceinline__ float hc_sinkhorn16(float v, int lane) {
    const int base = lane & 16, e = lane & 15, row = e >> 2, c = e & 3;
    const int rl = base + 4 * row;
    const float peak = fmaxf(fmaxf(__shfl_sync(0xffffffffu, v, rl), __shfl_sync(0xffffffffu, v, rl + 1)),
                             fmaxf(__shfl_sync(0xffffffffu, v, rl + 2), __shfl_sync(0xffffffffu, v, rl + 3)));
    float r = exp_rn(__fsub_rn(v, peak));
    for (int it = 0; it < 20; it++) {
        const float a0 = __shfl_sync(0xffffffffu, r, rl), a1 = __shfl_sync(0xffffffffu, r, rl + 1);
        const float a2 = __shfl_sync(0xffffffffu, r, rl + 2), a3 = __shfl_sync(0xffffffffu, r, rl + 3);
        r = __fdiv_rn(r, __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3));
        const float b0 = __shfl_sync(0xffffffffu, r, base + c), b1 = __shfl_sync(0xffffffffu, r, base + 4 + c);
        const float b2 = __shfl_sync(0xffffffffu, r, base + 8 + c), b3 = __shfl_sync(0xffffffffu, r, base + 12 + c);
        const float sum = __fadd_rn(__fadd_rn(__fadd_rn(b0, b1), b2), b3);
        if (sum > 0.0f) r = __fdiv_rn(r, sum);
    }
    return r;
}

// Ops.Mix4's scalar form for one column: w0 s0 + w1 s1 + w2 s2 + w3 s3, left
// to right, s the four lanes of a row's stream ([4][dim]).
__device__ __forceinline__ float hc_mix4(const float *s, int dim, int c, float w0, float w1, float w2, float w3) {
    float acc = __fadd_rn(__fmul_rn(w0, s[c]), __fmul_rn(w1, s[dim + c]));
    acc = __fadd_rn(acc, __fmul_rn(w2, s[2 * dim + c]));
    return __fadd_rn(acc, __fmul_rn(w3, s[3 * dim + c]));
}

}  // namespace ndl
