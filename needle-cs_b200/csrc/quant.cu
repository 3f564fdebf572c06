// Row quantizers: the reference's per-row int8 activation quantizer and the
// fused RMSNorm -> quantize prologue of every synthetic-decoder linear.
//
// The peak is an exact max (order-free); scale, inverse and every product
// use round-to-nearest intrinsics, so the int8 values and the fp32 scale are
// bit-identical to Scalar.QuantizeInt8 (src/Needle/Scalar.cs:67-74).  The
// RMSNorm sum of squares runs left to right on one lane, as
// Scalar.SumOfSquares does (src/Needle/Scalar.cs:206-211), from squares the
// other lanes compute, so the normalised row is the scalar one bit for bit.
// SiLU's sigmoid is the reference's vector one (Ops.Sigmoid with Ops.Exp).
#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Ops.InverseRms (src/Needle/Ops.cs:209, epsilon 1e-6): 1/sqrt(sum/n + eps)
// with the sum of squares taken left to right by lane 0 of the warp (the
// row is read from global memory; a fallback path for shapes the CTA
// kernel cannot hold).
__device__ __forceinline__ float inverse_rms_in_order(const float *row, int cols, int lane) {
    float ss = 0.0f;
    if (lane == 0)
        for (int c = 0; c < cols; c++) ss = __fadd_rn(ss, __fmul_rn(row[c], row[c]));
    ss = __shfl_sync(0xffffffffu, ss, 0);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), 1e-6f)));
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
    pdl_enter();
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *row = x + (size_t)warp * cols;
    int8_t *out = q + (size_t)warp * cols;
    float inv_rms = 1.0f;
    if (MODE == 1) inv_rms = inverse_rms_in_order(row, cols, lane);
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
    pdl_enter();
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *row = x + (size_t)warp * cols;
    int8_t *out = q + (size_t)warp * cols;
    float inv_rms = 1.0f;
    if (MODE == 1) inv_rms = inverse_rms_in_order(row, cols, lane);
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

// CTA-per-row variant: 128 threads, element float4 i handled by thread
// i % 128 (coalesced), values kept in registers between the passes.
// MODE 0 quantize, 1 RMSNorm + quantize, 2 SwiGLU (row = [gate | up]) + quantize.
constexpr int kRowThreads = 128;
constexpr int kRowMaxVec = 8;  // float4 per thread: cols <= 4096

template <int MODE>
__global__ void __launch_bounds__(kRowThreads) row_quantize_kernel(const float *__restrict__ x,
                                                                   const float *__restrict__ weight, int cols,
                                                                   int ld_in, int8_t *__restrict__ q,
                                                                   float *__restrict__ scales) {
    pdl_enter();
    __shared__ float red[kRowThreads / 32];
    __shared__ float4 squares[MODE == 1 ? kRowThreads * kRowMaxVec : 1];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float4 *in = reinterpret_cast<const float4 *>(x + (size_t)row * ld_in);
    const int nv = cols >> 2;
    float4 v[kRowMaxVec];
#pragma unroll
    for (int i = 0; i < kRowMaxVec; i++) {
        const int idx = tid + i * kRowThreads;
        v[i] = idx < nv ? in[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (MODE == 2) {
        const float4 *up = in + nv;
#pragma unroll
        for (int i = 0; i < kRowMaxVec; i++) {
            const int idx = tid + i * kRowThreads;
            if (idx < nv) {
                const float4 u = up[idx];
                float *g = reinterpret_cast<float *>(&v[i]);
                const float *uu = reinterpret_cast<const float *>(&u);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float sig = sigmoid_simd(g[e]);
                    g[e] = __fmul_rn(__fmul_rn(g[e], sig), uu[e]);
                }
            }
        }
    }
    if (MODE == 1) {
        // squares in element order through shared memory, summed left to
        // right by one thread (Scalar.SumOfSquares)
#pragma unroll
        for (int i = 0; i < kRowMaxVec; i++) {
            const int idx = tid + i * kRowThreads;
            if (idx < nv)
                squares[idx] = make_float4(__fmul_rn(v[i].x, v[i].x), __fmul_rn(v[i].y, v[i].y),
                                           __fmul_rn(v[i].z, v[i].z), __fmul_rn(v[i].w, v[i].w));
        }
        __syncthreads();
        if (tid == 0) {
            // the chain of adds is the kernel's critical path: the next four
            // float4 loads go out before the current sixteen adds
            float ss = 0.0f;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 nxt[4];
#pragma unroll
            for (int j = 0; j < 4; j++) nxt[j] = j < nv ? squares[j] : zero;
            for (int i = 0; i < nv; i += 4) {
                float4 cur[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    cur[j] = nxt[j];
                    nxt[j] = i + 4 + j < nv ? squares[i + 4 + j] : zero;
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (i + j < nv) {
                        ss = __fadd_rn(ss, cur[j].x);
                        ss = __fadd_rn(ss, cur[j].y);
                        ss = __fadd_rn(ss, cur[j].z);
                        ss = __fadd_rn(ss, cur[j].w);
                    }
                }
            }
            red[0] = ss;
        }
        __syncthreads();
        const float ss = red[0];
        __syncthreads();
        const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), 1e-6f)));
        const float4 *wv = reinterpret_cast<const float4 *>(weight);
#pragma unroll
        for (int i = 0; i < kRowMaxVec; i++) {
            const int idx = tid + i * kRowThreads;
            if (idx < nv) {
                const float4 w = wv[idx];
                v[i].x = __fmul_rn(__fmul_rn(w.x, v[i].x), inv_rms);
                v[i].y = __fmul_rn(__fmul_rn(w.y, v[i].y), inv_rms);
                v[i].z = __fmul_rn(__fmul_rn(w.z, v[i].z), inv_rms);
                v[i].w = __fmul_rn(__fmul_rn(w.w, v[i].w), inv_rms);
            }
        }
    }
    float peak = 0.0f;
#pragma unroll
    for (int i = 0; i < kRowMaxVec; i++)
        peak = fmaxf(peak, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    peak = warp_max(peak);
    if (lane == 0) red[warp] = peak;
    __syncthreads();
    peak = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float scale, inverse;
    scale_from_peak(peak, scale, inverse);
    uint32_t *out = reinterpret_cast<uint32_t *>(q + (size_t)row * cols);
#pragma unroll
    for (int i = 0; i < kRowMaxVec; i++) {
        const int idx = tid + i * kRowThreads;
        if (idx < nv) {
            const uint32_t b0 = (uint8_t)quantize_one(v[i].x, inverse), b1 = (uint8_t)quantize_one(v[i].y, inverse);
            const uint32_t b2 = (uint8_t)quantize_one(v[i].z, inverse), b3 = (uint8_t)quantize_one(v[i].w, inverse);
            out[idx] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    }
    if (tid == 0) scales[row] = scale;
}

int launch_quantize_rows(const float *x, const float *weight, int rows, int cols, int8_t *q, float *scales,
                         cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    const bool row_path = (cols % 4 == 0) && cols <= 4 * kRowThreads * kRowMaxVec && aligned(x, 16) &&
                          aligned(q, 4) && (!weight || aligned(weight, 16));
    if (row_path) {
        if (weight) launch_kernel(row_quantize_kernel<1>, dim3(rows), dim3(kRowThreads), 0, stream, x, weight, cols, cols, q, scales);
        else launch_kernel(row_quantize_kernel<0>, dim3(rows), dim3(kRowThreads), 0, stream, x, nullptr, cols, cols, q, scales);
        return check_launch("row_quantize");
    }
    dim3 block(256);
    dim3 grid((rows + 7) / 8);
    bool vec = (cols % 16 == 0) && aligned(x, 16) && aligned(q, 16) && (!weight || aligned(weight, 16));
    if (weight) {
        if (vec) launch_kernel(quantize_rows_vec_kernel<1>, dim3(grid), dim3(block), 0, stream, x, weight, rows, cols, q, scales);
        else launch_kernel(quantize_rows_scalar_kernel<1>, dim3(grid), dim3(block), 0, stream, x, weight, rows, cols, q, scales);
    } else {
        if (vec) launch_kernel(quantize_rows_vec_kernel<0>, dim3(grid), dim3(block), 0, stream, x, nullptr, rows, cols, q, scales);
        else launch_kernel(quantize_rows_scalar_kernel<0>, dim3(grid), dim3(block), 0, stream, x, nullptr, rows, cols, q, scales);
    }
    return check_launch("quantize_rows");
}

// SwiGLU of rows [gate (ffn) | up (ffn)] then quantize; falls back to the
// warp-per-row kernel in step_kernels.cu for shapes the row path cannot hold.
int launch_swiglu_quantize_rows(const float *gu, int rows, int ffn, int8_t *q, float *scales, cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    if (ffn % 4 != 0 || ffn > 4 * kRowThreads * kRowMaxVec || !aligned(gu, 16) || !aligned(q, 4))
        return NDL_ERR_UNSUPPORTED;
    launch_kernel(row_quantize_kernel<2>, dim3(rows), dim3(kRowThreads), 0, stream, gu, nullptr, ffn, 2 * ffn, q, scales);
    return check_launch("swiglu_quantize");
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
