// Row quantizers: the reference's per-row int8 activation quantizer and the
// fused RMSNorm -> quantize prologue of every synthetic-decoder linear.
//
// One warp per row.  The peak is an exact max (order-free); scale, inverse
// and every product use round-to-nearest intrinsics, so the int8 values and
// the fp32 scale are bit-identical to Scalar.QuantizeInt8
// (src/Needle/Scalar.cs:67-74).  The RMSNorm sum of squares is a warp tree
// (the reference sums left to right), so the normalised row can differ from
// the scalar one in the last ulp.
#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int8_t quantize_one(float x, float inverse) {
    float r = rintf(__fmul_rn(x, inverse));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    return (int8_t)(int)r;
}

__device__ __forceinline__ void scale_from_peak(float peak, float &scale, float &inverse) {
    scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    inverse = __fdiv_rn(1.0f, scale);
}

// Vector path: cols % 16 == 0, x 16-byte aligned, q 16-byte aligned.
// MODE 0: plain quantize.  MODE 1: RMSNorm (weight) then quantize.
template <int MODE>
__global__ void __launch_bounds__(256) quantize_rows_vec_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ weight, int rows,
                                                                int cols, int8_t *__restrict__ q,
                                                                float *__restrict__ scales) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *row = x + (size_t)warp * cols;
    int8_t *out = q + (size_t)warp * cols;
    float inv_rms = 1.0f;
    if (MODE == 1) {
        float ss = 0.0f;
        for (int c = lane * 4; c < cols; c += 128) {
            float4 v = *reinterpret_cast<const float4 *>(row + c);
            ss = __fadd_rn(ss, __fmul_rn(v.x, v.x));
            ss = __fadd_rn(ss, __fmul_rn(v.y, v.y));
            ss = __fadd_rn(ss, __fmul_rn(v.z, v.z));
            ss = __fadd_rn(ss, __fmul_rn(v.w, v.w));
        }
        ss = warp_sum(ss);
        inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), 1e-6f)));
    }
    float peak = 0.0f;
    for (int c = lane * 16; c < cols; c += 512) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            float4 v = *reinterpret_cast<const float4 *>(row + c + j);
            if (MODE == 1) {
                float4 w = *reinterpret_cast<const float4 *>(weight + c + j);
                v.x = __fmul_rn(__fmul_rn(w.x, v.x), inv_rms);
                v.y = __fmul_rn(__fmul_rn(w.y, v.y), inv_rms);
                v.z = __fmul_rn(__fmul_rn(w.z, v.z), inv_rms);
                v.w = __fmul_rn(__fmul_rn(w.w, v.w), inv_rms);
            }
            peak = fmaxf(peak, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    peak = warp_max(peak);
    float scale, inverse;
    scale_from_peak(peak, scale, inverse);
    for (int c = lane * 16; c < cols; c += 512) {
        uint32_t packed[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4 v = *reinterpret_cast<const float4 *>(row + c + 4 * j);
            if (MODE == 1) {
                float4 w = *reinterpret_cast<const float4 *>(weight + c + 4 * j);
                v.x = __fmul_rn(__fmul_rn(w.x, v.x), inv_rms);
                v.y = __fmul_rn(__fmul_rn(w.y, v.y), inv_rms);
                v.z = __fmul_rn(__fmul_rn(w.z, v.z), inv_rms);
                v.w = __fmul_rn(__fmul_rn(w.w, v.w), inv_rms);
            }
            uint32_t b0 = (uint8_t)quantize_one(v.x, inverse), b1 = (uint8_t)quantize_one(v.y, inverse);
            uint32_t b2 = (uint8_t)quantize_one(v.z, inverse), b3 = (uint8_t)quantize_one(v.w, inverse);
            packed[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        *reinterpret_cast<uint4 *>(out + c) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
    if (lane == 0) scales[warp] = scale;
}

// Scalar path for any cols / alignment.
template <int MODE>
__global__ void __launch_bounds__(256) quantize_rows_scalar_kernel(const float *__restrict__ x,
                                                                   const float *__restrict__ weight, int rows,
                                                                   int cols, int8_t *__restrict__ q,
                                                                   float *__restrict__ scales) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *row = x + (size_t)warp * cols;
    int8_t *out = q + (size_t)warp * cols;
    float inv_rms = 1.0f;
    if (MODE == 1) {
        float ss = 0.0f;
        for (int c = lane; c < cols; c += 32) ss = __fadd_rn(ss, __fmul_rn(row[c], row[c]));
        ss = warp_sum(ss);
        inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), 1e-6f)));
    }
    float peak = 0.0f;
    for (int c = lane; c < cols; c += 32) {
        float v = row[c];
        if (MODE == 1) v = __fmul_rn(__fmul_rn(weight[c], v), inv_rms);
        peak = fmaxf(peak, fabsf(v));
    }
    peak = warp_max(peak);
    float scale, inverse;
    scale_from_peak(peak, scale, inverse);
    for (int c = lane; c < cols; c += 32) {
        float v = row[c];
        if (MODE == 1) v = __fmul_rn(__fmul_rn(weight[c], v), inv_rms);
        out[c] = quantize_one(v, inverse);
    }
    if (lane == 0) scales[warp] = scale;
}

int launch_quantize_rows(const float *x, const float *weight, int rows, int cols, int8_t *q, float *scales,
                         cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    dim3 block(256);
    dim3 grid((rows + 7) / 8);
    bool vec = (cols % 16 == 0) && aligned(x, 16) && aligned(q, 16) && (!weight || aligned(weight, 16));
    if (weight) {
        if (vec) quantize_rows_vec_kernel<1><<<grid, block, 0, stream>>>(x, weight, rows, cols, q, scales);
        else quantize_rows_scalar_kernel<1><<<grid, block, 0, stream>>>(x, weight, rows, cols, q, scales);
    } else {
        if (vec) quantize_rows_vec_kernel<0><<<grid, block, 0, stream>>>(x, nullptr, rows, cols, q, scales);
        else quantize_rows_scalar_kernel<0><<<grid, block, 0, stream>>>(x, nullptr, rows, cols, q, scales);
    }
    return check_launch("quantize_rows");
}

}  // namespace ndl

using namespace ndl;

extern "C" NDL_API int ndl_quantize_rows(const float *x, int rows, int cols, int8_t *q, float *scales,
                                         void *stream) {
    NDL_REQUIRE(rows >= 0 && cols >= 1, "rows %d / cols %d out of range", rows, cols);
    NDL_REQUIRE(rows == 0 || (x && q && scales), "null pointer");
    return launch_quantize_rows(x, nullptr, rows, cols, q, scales, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_rmsnorm_quantize(const float *x, const float *weight, int rows, int cols, int8_t *q,
                                            float *scales, void *stream) {
    NDL_REQUIRE(rows >= 0 && cols >= 1, "rows %d / cols %d out of range", rows, cols);
    NDL_REQUIRE(rows == 0 || (x && weight && q && scales), "null pointer");
    return launch_quantize_rows(x, weight, rows, cols, q, scales, (cudaStream_t)stream);
}
