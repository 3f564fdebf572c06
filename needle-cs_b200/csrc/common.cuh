// Shared helpers for the needle B200 library: status plumbing, the
// reference's fp16 decode, the counter-based synthetic generator, and small
// PTX wrappers.  Everything here is used by host and device code alike.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "../../include/needle_cuda.h"

namespace ndl {

// ---------------------------------------------------------------- status --
// Records a per-thread message for ndl_last_error() and returns `status`.
int set_error(int status, const char *fmt, ...);
// Converts the last CUDA error (launch or sticky) into a status.
int check_launch(const char *what);

#define NDL_REQUIRE(cond, ...)                                                   \
    do {                                                                         \
        if (!(cond)) return ::ndl::set_error(NDL_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

#define NDL_CUDA(call)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess)                                                                  \
            return ::ndl::set_error(NDL_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_));     \
    } while (0)

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ------------------------------------------------------- per-device set-up --
// A process may drive several GPUs (one engine per device, host threads per
// engine), and function attributes and SM counts belong to a device, so
// one-time set-up is keyed by the current device and guarded for threads.
constexpr int kMaxDevices = 64;

// SM count of the current device, queried once per device.
int device_sm_count();

// Runs a set-up step once per device: the first caller on each device runs
// it under a lock, later callers see the flag.  A failed set-up is retried
// on the next call.
class DeviceOnce {
  public:
    template <class F>
    int run(F &&setup) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        if (dev < 0 || dev >= kMaxDevices) return set_error(NDL_ERR_UNSUPPORTED, "device %d out of range", dev);
        if (done_[dev].load(std::memory_order_acquire)) return NDL_OK;
        std::lock_guard<std::mutex> lock(mutex_);
        if (done_[dev].load(std::memory_order_relaxed)) return NDL_OK;
        int st = setup();
        if (st == NDL_OK) done_[dev].store(true, std::memory_order_release);
        return st;
    }

  private:
    std::atomic<bool> done_[kMaxDevices] = {};
    std::mutex mutex_;
};

// ------------------------------------------------------------------ fp16 --
// Scalar.HalfToSingle (src/Needle/Scalar.cs:121-128): exact for finite
// halves, no Inf/NaN case (0x7C00 -> 65536).  Integer-only so host and
// device agree bit for bit.
__host__ __device__ __forceinline__ float half_to_float_ref(uint16_t half) {
    uint32_t magnitude = half & 0x7FFFu;
    if (magnitude == 0) return 0.0f;
    if (magnitude < 0x0400u) {
        float v = (float)magnitude * 5.9604645e-8f;
        return (half & 0x8000u) ? -v : v;
    }
    uint32_t bits = ((magnitude << 13) + 0x38000000u) | ((uint32_t)(half & 0x8000u) << 16);
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float f;
    __builtin_memcpy(&f, &bits, 4);
    return f;
#endif
}

#ifdef __CUDACC__
// Same values as half_to_float_ref with one hardware conversion: IEEE
// binary16 decode is identical for finite halves; the reference's Inf/NaN
// pattern (no special case) is patched in with a select.
__device__ __forceinline__ float half_to_float_ref_fast(uint16_t h) {
    float f = __half2float(__ushort_as_half(h));
    if ((h & 0x7C00u) == 0x7C00u)
        f = __uint_as_float(((((uint32_t)h & 0x7FFFu) << 13) + 0x38000000u) | ((uint32_t)(h & 0x8000u) << 16));
    return f;
}

// Packed pairs of fp32 (fma/add.rn.f32x2: each half is an IEEE fma/add with
// round-to-nearest, the same bits as the scalar forms).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Ops.Exp (src/Needle/Ops.cs:16-31), the reference's SIMD exponential, which
// its AVX2 attention softmax and vector sigmoid use: clamp to [-87.3, 88.7]
// (a NaN becomes -87.3, as maxps returns its second operand), n = nearest
// integer of x * log2(e), r = x - n*ln2 in two fused steps, a degree-5
// polynomial by fused multiply-adds, y = p*r^2 + (r + 1), times 2^n built in
// the exponent bits.  Each step is one IEEE operation (explicit fma, mul and
// add intrinsics), so the CPU oracle, which takes the same steps, gets the
// same bits.
__device__ __forceinline__ float exp_simd(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.7f);
    const float n = rintf(__fmul_rn(x, 1.44269504f));
    float r = __fmaf_rn(-n, 0.693359375f, x);
    r = __fmaf_rn(-n, -2.12194440e-4f, r);
    float p = 1.9875691500e-4f;
    p = __fmaf_rn(p, r, 1.3981999507e-3f);
    p = __fmaf_rn(p, r, 8.3334519073e-3f);
    p = __fmaf_rn(p, r, 4.1665795894e-2f);
    p = __fmaf_rn(p, r, 1.6666665459e-1f);
    p = __fmaf_rn(p, r, 5.0000001201e-1f);
    const float y = __fmaf_rn(p, __fmul_rn(r, r), __fadd_rn(r, 1.0f));
    return __fmul_rn(y, __int_as_float(((int)n + 127) << 23));
}
// Ops.Sigmoid (src/Needle/Ops.cs:36-40): 1 / (1 + Exp(0 - x)).
__device__ __forceinline__ float sigmoid_simd(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_simd(__fsub_rn(0.0f, x))));
}

// MathF.Exp where the reference's scalar tier calls it (Softmax, Sigmoid,
// Sinkhorn4x4, the Needle-3 gates, MLP and Engram): the float exponential
// rounded to nearest, computed in double precision from the mathematics
// (Cody and Waite's reduction with fdlibm's two-part ln 2, then the Taylor
// series to degree 13 in Estrin's form), which equals the correctly rounded exp except within
// about 1e-15 of a rounding midpoint.  Every double step is an explicit
// IEEE operation, so the CPU oracle, which evaluates the same steps, returns
// the same bits.
__device__ __forceinline__ float exp_rn(float x) {
    if (x != x) return x;
    if (x > 89.0f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    const double xd = (double)x;
    const double k = rint(__dmul_rn(xd, 1.4426950408889634));
    const double r =
        __dsub_rn(__dsub_rn(xd, __dmul_rn(k, 6.93147180369123816490e-01)), __dmul_rn(k, 1.90821492927058770002e-10));
    // the degree-13 Taylor polynomial by Estrin's scheme (pairs, then r^2, r^4,
    // r^8 levels): four dependent fused steps instead of thirteen
    const double r2 = __dmul_rn(r, r), r4 = __dmul_rn(r2, r2), r8 = __dmul_rn(r4, r4);
    const double q0 = __fma_rn(1.0, r, 1.0);
    const double q1 = __fma_rn(1.6666666666666666667e-01, r, 0.5);
    const double q2 = __fma_rn(8.3333333333333333333e-03, r, 4.1666666666666666667e-02);
    const double q3 = __fma_rn(1.9841269841269841270e-04, r, 1.3888888888888888889e-03);
    const double q4 = __fma_rn(2.7557319223985890653e-06, r, 2.4801587301587301587e-05);
    const double q5 = __fma_rn(2.5052108385441718775e-08, r, 2.7557319223985890653e-07);
    const double q6 = __fma_rn(1.6059043836821614599e-10, r, 2.0876756987868098979e-09);
    const double s0 = __fma_rn(q1, r2, q0), s1 = __fma_rn(q3, r2, q2), s2 = __fma_rn(q5, r2, q4);
    const double t0 = __fma_rn(s1, r4, s0), t1 = __fma_rn(q6, r4, s2);
    const double p = __fma_rn(t1, r8, t0);
    // times 2^k (|k| <= 151: exact in double), one rounding to float
    const double two_k = __longlong_as_double((long long)((int)k + 1023) << 52);
    return __double2float_rn(__dmul_rn(p, two_k));
}
// Ops.Sigmoid's scalar form (src/Needle/Ops.cs:88): 1 / (1 + MathF.Exp(-x)).
__device__ __forceinline__ float sigmoid_rn(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-x)));
}
#endif

// exp_rn's steps on the host (MathF.Exp in double, one rounding), for the
// sigmoids of stored gate logits that the host evaluates once per model.
inline float host_exp_rn(float x) {
    if (x != x) return x;
    if (x > 89.0f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const double xd = (double)x;
    const double k = rint(xd * 1.4426950408889634);
    const double r = (xd - k * 6.93147180369123816490e-01) - k * 1.90821492927058770002e-10;
    const double r2 = r * r, r4 = r2 * r2, r8 = r4 * r4;  // exp_rn's Estrin steps
    const double q0 = fma(1.0, r, 1.0);
    const double q1 = fma(1.6666666666666666667e-01, r, 0.5);
    const double q2 = fma(8.3333333333333333333e-03, r, 4.1666666666666666667e-02);
    const double q3 = fma(1.9841269841269841270e-04, r, 1.3888888888888888889e-03);
    const double q4 = fma(2.7557319223985890653e-06, r, 2.4801587301587301587e-05);
    const double q5 = fma(2.5052108385441718775e-08, r, 2.7557319223985890653e-07);
    const double q6 = fma(1.6059043836821614599e-10, r, 2.0876756987868098979e-09);
    const double s0 = fma(q1, r2, q0), s1 = fma(q3, r2, q2), s2 = fma(q5, r2, q4);
    const double t0 = fma(s1, r4, s0), t1 = fma(q6, r4, s2);
    return (float)scalbn(fma(t1, r8, t0), (int)k);
}
inline float host_sigmoid_rn(float x) { return 1.0f / (1.0f + host_exp_rn(-x)); }

// IEEE round-to-nearest-even float -> binary16 (integer-only).
__host__ __device__ __forceinline__ uint16_t float_to_half_rne(float f) {
#ifdef __CUDA_ARCH__
    uint32_t x = __float_as_uint(f);
#else
    uint32_t x;
    __builtin_memcpy(&x, &f, 4);
#endif
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t abs = x & 0x7FFFFFFFu;
    if (abs >= 0x7F800000u) return (uint16_t)(sign | (abs > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (abs >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    if (abs < 0x38800000u) {                                     // subnormal or zero in half
        if (abs < 0x33000000u) return (uint16_t)sign;            // < 2^-25 rounds to 0
        uint32_t mant = (abs & 0x007FFFFFu) | 0x00800000u;
        int shift = 126 - (int)(abs >> 23);                      // 14 + (113 - exp) ... >= 14
        // value = mant * 2^(exp-150); half subnormal unit = 2^-24 -> q = mant >> (126 - exp)
        uint32_t q = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t rebased = abs - 0x38000000u;  // exponent bias 127 -> 15
    uint32_t q = rebased >> 13;
    uint32_t rem = rebased & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

// ------------------------------------------------------ synthetic inputs --
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ (stream * 0x9E3779B97F4A7C15ull));
}
__host__ __device__ __forceinline__ uint64_t synth_hash(uint64_t key, uint64_t i) {
    return splitmix64(key + i * 0xD1B54A32D192ED03ull);
}
__host__ __device__ __forceinline__ int sum16x4(uint64_t h) {
    return (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
}
// Irwin-Hall(12) - 6 in exact arithmetic: identical on host and device.
__host__ __device__ __forceinline__ float synth_normal(uint64_t key, uint64_t i) {
    int s = sum16x4(synth_hash(key, 3 * i)) + sum16x4(synth_hash(key, 3 * i + 1)) +
            sum16x4(synth_hash(key, 3 * i + 2));
    return (float)(2 * s - 786420) * (1.0f / 131072.0f);
}
__host__ __device__ __forceinline__ float synth_uniform(uint64_t key, uint64_t i, float lo, float hi) {
    float u = (float)(synth_hash(key, i) >> 40) * (1.0f / 16777216.0f);
#ifdef __CUDA_ARCH__
    return __fadd_rn(lo, __fmul_rn(__fsub_rn(hi, lo), u));  // no contraction: matches the host
#else
    float span = hi - lo;
    float t = span * u;
    return lo + t;
#endif
}
__host__ __device__ __forceinline__ int8_t synth_int8(uint64_t key, uint64_t i) {
    return (int8_t)((int)(synth_hash(key, i) % 255u) - 127);
}

// ---- programmatic dependent launch (step kernels) ----
// A step kernel first waits for its predecessor grid to complete
// (griddepcontrol.wait: a no-op when launched without the attribute), then
// lets its own dependent launch (griddepcontrol.launch_dependents), so the
// next kernel's launch overlaps this one's work while memory order is kept.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
    pdl_wait();
    pdl_trigger();
}
#endif
// Host: launches made while the flag is set (the engine's step) carry the
// programmatic-stream-serialization attribute.
inline bool &pdl_flag() {
    static thread_local bool flag = false;
    return flag;
}
struct PdlScope {
    bool old;
    explicit PdlScope(bool on) : old(pdl_flag()) { pdl_flag() = on; }
    ~PdlScope() { pdl_flag() = old; }
};
#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    if (pdl_flag()) {
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
#endif

}  // namespace ndl
