// Failure detection without a GPU fault: every kernel wait in the library is
// bounded (a limited number of suspend-hinted mbarrier tests), after which
// the kernel records kStatusTimeout, stops waiting and returns, so the host
// reads NDL_ERR_TIMEOUT and the CUDA context stays usable.  This entry point
// runs that path on purpose: one thread waits for an mbarrier phase that
// nothing completes, gives up after `tests` tests and reports the status.
#include "common.cuh"
#include "kv.cuh"

using namespace ndl;

namespace {

__global__ void bounded_wait_kernel(uint32_t tests, int *status) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);  // expects one arrival; none comes
    fence_mbar_init();
    if (!mbar_wait_bounded(&bar, 0, tests)) atomicOr(status, kStatusTimeout);
    // complete the phase ourselves so the barrier is left in a finished state
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
}

__global__ void exp_kernel(const float *x, int n, float *y) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = exp_simd(x[i]);
}

}  // namespace

extern "C" {

// Runs the bounded wait on the current device; returns NDL_ERR_TIMEOUT when
// the wait gave up (the expected outcome) and NDL_OK if it did not.
NDL_API int ndl_selftest_bounded_wait(int tests) {
    NDL_REQUIRE(tests >= 1 && tests <= (1 << 20), "tests %d outside 1..2^20", tests);
    int *d_status = nullptr;
    NDL_CUDA(cudaMalloc(&d_status, sizeof(int)));
    int st = NDL_OK, h = 0;
    if (cudaMemset(d_status, 0, sizeof(int)) == cudaSuccess) {
        bounded_wait_kernel<<<1, 32>>>((uint32_t)tests, d_status);
        if (cudaGetLastError() != cudaSuccess || cudaMemcpy(&h, d_status, sizeof(int), cudaMemcpyDeviceToHost) !=
                                                     cudaSuccess)
            st = set_error(NDL_ERR_CUDA, "bounded wait self-test failed to run");
    } else {
        st = set_error(NDL_ERR_CUDA, "bounded wait self-test: memset failed");
    }
    cudaFree(d_status);
    if (st != NDL_OK) return st;
    if (h & kStatusTimeout) return set_error(NDL_ERR_TIMEOUT, "a kernel wait gave up after %d tests", tests);
    return NDL_OK;
}

// exp_simd, the library's float exponential (Ops.Exp, the one its softmax
// and SiLU use), over n device floats: lets a test pin it to the CPU
// oracle's.
NDL_API int ndl_selftest_exp(const float *x, int n, float *y, void *stream) {
    NDL_REQUIRE(n >= 0 && (n == 0 || (x && y)), "bad arguments");
    if (n == 0) return NDL_OK;
    exp_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(x, n, y);
    return check_launch("selftest_exp");
}

}  // extern "C"
