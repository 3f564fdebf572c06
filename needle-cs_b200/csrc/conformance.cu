// KernelTable-signature conformance exports: the reference's own kernel
// slots (src/Needle/Kernels/KernelTable.cs:5-47, signatures fixed by
// Net10KernelExports.Fill, src/Needle/Kernels/Net10KernelExports.cs:118-150)
// computed on the GPU, host pointers in and out, synchronous.  Installed in a
// KernelTable they let the reference's conformance cases drive the device
// kernels.  Like the slots they replace they have no error channel: a CUDA
// failure returns NaN (scales, probabilities) or -2 (argmax) and leaves the
// reason in ndl_last_error.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

using namespace ndl;

namespace ndl {
int launch_argmax_masked(const float *x, long long ldx, const uint32_t *mask, int words, long long ldm,
                         const int32_t *mask_index, int length, int rows, int32_t *ids, float *probs,
                         cudaStream_t stream);
int launch_best_probability(const float *x, int count, float best, float *out, cudaStream_t stream);
}  // namespace ndl

namespace {

// One growing device buffer, shared by the exports and guarded by a mutex
// (the reference calls kernel slots from several pool threads).
std::mutex g_mu;
void *g_buf = nullptr;
size_t g_cap = 0;
int g_dev = -1;

int scratch(size_t bytes, void **out) {
    int dev = 0;
    NDL_CUDA(cudaGetDevice(&dev));
    if (g_buf && (g_cap < bytes || g_dev != dev)) {
        cudaFree(g_buf);
        g_buf = nullptr;
        g_cap = 0;
    }
    if (!g_buf) {
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        if (cudaMalloc(&g_buf, cap) != cudaSuccess) {
            cudaGetLastError();
            return set_error(NDL_ERR_OUT_OF_MEMORY, "conformance scratch (%zu bytes)", cap);
        }
        g_cap = cap;
        g_dev = dev;
    }
    *out = g_buf;
    return NDL_OK;
}

size_t align16(size_t n) { return (n + 15) & ~size_t(15); }

}  // namespace

extern "C" {

// float QuantizeInt8(float* x, int n, sbyte* destination)  (Quant.QuantizeInt8)
NDL_API float ndl_kt_quantize_int8(const float *x, int n, int8_t *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !destination || n < 1) {
        set_error(NDL_ERR_INVALID_ARG, "quantize_int8: bad arguments");
        return NAN;
    }
    void *buf = nullptr;
    if (scratch(align16((size_t)n * 4) + align16((size_t)n) + 16, &buf) != NDL_OK) return NAN;
    float *dx = static_cast<float *>(buf);
    int8_t *dq = reinterpret_cast<int8_t *>(static_cast<char *>(buf) + align16((size_t)n * 4));
    float *ds = reinterpret_cast<float *>(reinterpret_cast<char *>(dq) + align16((size_t)n));
    float scale = NAN;
    if (cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        ndl_quantize_rows(dx, 1, n, dq, ds, nullptr) != NDL_OK ||
        cudaMemcpy(destination, dq, (size_t)n, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&scale, ds, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "quantize_int8 failed");
        return NAN;
    }
    return scale;
}

// int ArgMaxMasked(float* x, uint* mask, int words, int length)  (Ops.ArgMaxMasked)
NDL_API int ndl_kt_argmax_masked(const float *x, const uint32_t *mask, int words, int length) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !mask || words < 0 || length < 0) {
        set_error(NDL_ERR_INVALID_ARG, "argmax_masked: bad arguments");
        return -2;
    }
    const int n = length < words * 32 ? length : words * 32;  // ids >= length or >= 32*words are never chosen
    if (n <= 0) return -1;
    void *buf = nullptr;
    if (scratch(align16((size_t)n * 4) + align16((size_t)words * 4) + 16, &buf) != NDL_OK) return -2;
    float *dx = static_cast<float *>(buf);
    uint32_t *dm = reinterpret_cast<uint32_t *>(static_cast<char *>(buf) + align16((size_t)n * 4));
    int32_t *did = reinterpret_cast<int32_t *>(reinterpret_cast<char *>(dm) + align16((size_t)words * 4));
    int id = -2;
    if (cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dm, mask, (size_t)words * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_argmax_masked(dx, n, dm, words, words, nullptr, n, 1, did, nullptr, nullptr) != NDL_OK ||
        cudaMemcpy(&id, did, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "argmax_masked failed");
        return -2;
    }
    return id;
}

// float BestProbability(float* values, int count, float best)  (Ops.BestProbability)
NDL_API float ndl_kt_best_probability(const float *values, int count, float best) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!values || count < 1) {
        set_error(NDL_ERR_INVALID_ARG, "best_probability: bad arguments");
        return NAN;
    }
    void *buf = nullptr;
    if (scratch(align16((size_t)count * 4) + 16, &buf) != NDL_OK) return NAN;
    float *dx = static_cast<float *>(buf);
    float *dp = reinterpret_cast<float *>(static_cast<char *>(buf) + align16((size_t)count * 4));
    float p = NAN;
    if (cudaMemcpy(dx, values, (size_t)count * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_best_probability(dx, count, best, dp, nullptr) != NDL_OK ||
        cudaMemcpy(&p, dp, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "best_probability failed");
        return NAN;
    }
    return p;
}

}  // extern "C"
