// Library identity, status strings, per-thread error messages and the
// synthetic-input generators (host and device).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace ndl {

static thread_local char g_last_error[512];

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return NDL_OK;
}

int device_sm_count() {
    static std::atomic<int> counts[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 1;
    int n = counts[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) return 1;
    counts[dev].store(n, std::memory_order_relaxed);
    return n;
}

// ------------------------------------------------------------ generators --
template <typename F>
__global__ void synth_fill_kernel(size_t count, F f) {
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) f(i);
}

template <typename F>
static int launch_fill(size_t count, F f, void *stream, const char *what) {
    if (count == 0) return NDL_OK;
    size_t blocks = (count + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    synth_fill_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(count, f);
    return check_launch(what);
}

struct NormalF32 {
    uint64_t key, first;
    float scale;
    float *out;
    __device__ void operator()(size_t i) const { out[i] = __fmul_rn(synth_normal(key, first + i), scale); }
};
struct NormalF16 {
    uint64_t key, first;
    float scale;
    uint16_t *out;
    __device__ void operator()(size_t i) const {
        out[i] = float_to_half_rne(__fmul_rn(synth_normal(key, first + i), scale));
    }
};
struct UniformF16 {
    uint64_t key, first;
    float lo, hi;
    uint16_t *out;
    __device__ void operator()(size_t i) const { out[i] = float_to_half_rne(synth_uniform(key, first + i, lo, hi)); }
};
struct Int8Fill {
    uint64_t key, first;
    int8_t *out;
    __device__ void operator()(size_t i) const { out[i] = synth_int8(key, first + i); }
};

}  // namespace ndl

using namespace ndl;

extern "C" {

NDL_API const char *ndl_version(void) { return "needle-b200 0.1.0 (sm_100a)"; }

NDL_API const char *ndl_status_string(int status) {
    switch (status) {
        case NDL_OK: return "ok";
        case NDL_FAIL_EMPTY_INPUT: return "EmptyInput";
        case NDL_FAIL_INPUT_TOO_LONG: return "InputTooLong";
        case NDL_FAIL_CONTEXT_EXHAUSTED: return "ContextExhausted";
        case NDL_FAIL_CALL_TOKEN_BUDGET: return "CallTokenBudgetExceeded";
        case NDL_FAIL_CALL_TEXT_TOO_LONG: return "CallTextTooLong";
        case NDL_FAIL_GRAMMAR_DEAD_END: return "GrammarDeadEnd";
        case NDL_FAIL_GRAMMAR_REJECTED: return "GrammarRejectedToken";
        case NDL_FAIL_CALLS_BUFFER: return "CallsBufferTooSmall";
        case NDL_FAIL_MALFORMED_CALLS: return "MalformedCalls";
        case NDL_FAIL_TOOL_CONTEXT: return "ToolContextFailed";
        case NDL_FAIL_FRAME_BUDGET: return "FrameBudgetExceeded";
        case NDL_ERR_INVALID_ARG: return "invalid argument";
        case NDL_ERR_CUDA: return "CUDA error";
        case NDL_ERR_BOUNDS: return "out of bounds";
        case NDL_ERR_TIMEOUT: return "timeout";
        case NDL_ERR_OUT_OF_MEMORY: return "out of memory";
        case NDL_ERR_UNSUPPORTED: return "unsupported";
        case NDL_ERR_NO_DEVICE: return "no device";
        case NDL_ERR_MALFORMED_MODEL: return "malformed model";
        case NDL_ERR_PAGES_EXHAUSTED: return "KV pages exhausted";
        case NDL_ERR_CANCELLED: return "cancelled";
        default: return "unknown status";
    }
}

NDL_API const char *ndl_last_error(void) { return g_last_error; }

NDL_API int ndl_device_count(int *count) {
    if (!count) return set_error(NDL_ERR_INVALID_ARG, "count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        cudaGetLastError();
        return set_error(NDL_ERR_NO_DEVICE, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = n;
    return NDL_OK;
}

NDL_API void ndl_synth_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                  float *out) {
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < count; i++) out[i] = synth_normal(key, first + i) * scale;
}

NDL_API void ndl_synth_normal_f16(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                  uint16_t *out) {
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < count; i++) out[i] = float_to_half_rne(synth_normal(key, first + i) * scale);
}

NDL_API void ndl_synth_uniform_f16(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo,
                                   float hi, uint16_t *out) {
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < count; i++) out[i] = float_to_half_rne(synth_uniform(key, first + i, lo, hi));
}

NDL_API void ndl_synth_int8(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out) {
    uint64_t key = synth_key(seed, stream);
    for (size_t i = 0; i < count; i++) out[i] = synth_int8(key, first + i);
}

NDL_API uint16_t ndl_f32_to_f16(float value) { return float_to_half_rne(value); }
NDL_API float ndl_f16_to_f32(uint16_t half) { return half_to_float_ref(half); }

NDL_API int ndl_synth_normal_f32_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                        float *out, void *cuda_stream) {
    NDL_REQUIRE(out || count == 0, "out is NULL");
    return launch_fill(count, NormalF32{synth_key(seed, stream), first, scale, out}, cuda_stream, "synth_normal_f32");
}

NDL_API int ndl_synth_normal_f16_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count,
                                        float scale, uint16_t *out, void *cuda_stream) {
    NDL_REQUIRE(out || count == 0, "out is NULL");
    return launch_fill(count, NormalF16{synth_key(seed, stream), first, scale, out}, cuda_stream, "synth_normal_f16");
}

NDL_API int ndl_synth_uniform_f16_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo,
                                         float hi, uint16_t *out, void *cuda_stream) {
    NDL_REQUIRE(out || count == 0, "out is NULL");
    return launch_fill(count, UniformF16{synth_key(seed, stream), first, lo, hi, out}, cuda_stream,
                       "synth_uniform_f16");
}

NDL_API int ndl_synth_int8_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out,
                                  void *cuda_stream) {
    NDL_REQUIRE(out || count == 0, "out is NULL");
    return launch_fill(count, Int8Fill{synth_key(seed, stream), first, out}, cuda_stream, "synth_int8");
}

}  // extern "C"
