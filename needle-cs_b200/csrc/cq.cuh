// CQ Prepare's per-group steps (Quant.PrepareRange scalar branch,
// src/Needle/Quant.cs:471-484; Scalar.Hadamard / QuantizeInt8 / Planes,
// src/Needle/Scalar.cs:66-111), shared by the Prepare kernel and the row
// kernels that end in a Prepare.
#pragma once

#include "common.cuh"

namespace ndl {

constexpr float kCqHadamardScale = 0.08838834764831845f;  // Scalar.cs:49 (Quant.cs:51)

__device__ __forceinline__ int8_t cq_quant1(float x, float inverse) {
    const float r = rintf(__fmul_rn(x, inverse));
    return (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
}

// Plane position of group element e: 2-bit [p*32 + j] = q[4j + p];
// 4-bit [h*64 + p*32 + j] = q[h*64 + 2j + p].
__device__ __forceinline__ int cq_plane_at(int e, int bits) {
    return bits == 2 ? (e & 3) * 32 + (e >> 2) : (e >> 6) * 64 + (e & 1) * 32 + ((e & 63) >> 1);
}

// One 128-column group held by a warp as elements 4l .. 4l + 3 on lane l:
// the Hadamard butterflies of strides 1, 2 (inside the lane), then 4 .. 64
// (lanes l ^ 1 .. l ^ 16), lower index a + b, upper a - b, in that order;
// the 1/sqrt(128) scale, the group's int8 quantization with one scale, the
// plane reorder into dst (the group's 128 bytes) and offset = 63 * sum(q).
// Lane 0 writes *scale and *offset.  All 32 lanes must call it together.
__device__ __forceinline__ void cq_prepare_group_lane4(float (&w)[4], int lane, int bits, int8_t *dst, float *scale,
                                                      float *offset) {
    {  // stride 1: elements (4l, 4l + 1), (4l + 2, 4l + 3)
        const float a0 = w[0], b0 = w[1], a1 = w[2], b1 = w[3];
        w[0] = __fadd_rn(a0, b0);
        w[1] = __fsub_rn(a0, b0);
        w[2] = __fadd_rn(a1, b1);
        w[3] = __fsub_rn(a1, b1);
    }
    {  // stride 2: elements (4l, 4l + 2), (4l + 1, 4l + 3)
        const float a0 = w[0], b0 = w[2], a1 = w[1], b1 = w[3];
        w[0] = __fadd_rn(a0, b0);
        w[2] = __fsub_rn(a0, b0);
        w[1] = __fadd_rn(a1, b1);
        w[3] = __fsub_rn(a1, b1);
    }
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {  // element strides 4 s
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float o = __shfl_xor_sync(0xffffffffu, w[k], s);
            w[k] = upper ? __fsub_rn(o, w[k]) : __fadd_rn(w[k], o);
        }
    }
    float peak = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        w[k] = __fmul_rn(w[k], kCqHadamardScale);
        peak = fmaxf(peak, fabsf(w[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    const float sc = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, sc);
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int8_t q = cq_quant1(w[k], inverse);
        dst[cq_plane_at(4 * lane + k, bits)] = q;
        sum += q;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        *scale = sc;
        *offset = __fmul_rn(63.0f, (float)sum);
    }
}

}  // namespace ndl
