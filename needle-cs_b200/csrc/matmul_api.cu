// C-ABI entry points of the I8G32 quantized linear (MatMulRows / MatMulBatch
// replacements).  Validation happens here, on the host, before any launch.
#include "common.cuh"
#include "kernels.cuh"

using namespace ndl;

static int validate(const MatmulArgs &a) {
    NDL_REQUIRE(a.m >= 0 && a.n >= 1 && a.k >= 32, "m=%d n=%d k=%d out of range", a.m, a.n, a.k);
    NDL_REQUIRE(a.k % 32 == 0, "k=%d is not a multiple of the 32-column group", a.k);
    NDL_REQUIRE(a.ldy >= a.n, "ldy=%d < n=%d", a.ldy, a.n);
    NDL_REQUIRE(a.batch >= 1, "batch=%d", a.batch);
    if (a.m == 0) return NDL_OK;
    NDL_REQUIRE(a.q && a.sa && a.w && a.sw && a.y, "null pointer");
    NDL_REQUIRE(aligned(a.q, 16) && aligned(a.w, 16), "q and w must be 16-byte aligned");
    NDL_REQUIRE(aligned(a.sw, 2) && aligned(a.y, 4) && aligned(a.sa, 4), "misaligned scale/output pointer");
    NDL_REQUIRE(a.w_stride % 16 == 0 && a.sw_stride >= 0 && a.y_stride >= 0, "bad batch strides");
    return NDL_OK;
}

static int dispatch(const MatmulArgs &a, cudaStream_t stream) {
    if (a.m == 0) return NDL_OK;
    if (a.m >= 64) {
        int st = launch_gemm_i8g32_tc(a, stream);
        if (st != NDL_ERR_UNSUPPORTED) return st;
    }
    return launch_gemv_i8g32(a, stream);
}

extern "C" NDL_API int ndl_matmul_i8g32(const int8_t *q, const float *sa, int m, const int8_t *w, const uint16_t *sw,
                                        int n, int k, float *y, int ldy, const float *residual, int32_t *acc,
                                        void *stream) {
    MatmulArgs a{q, sa, m, k, w, sw, n, y, ldy, residual, acc, 0, 0, 0, 1};
    int st = validate(a);
    if (st != NDL_OK) return st;
    return dispatch(a, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_matmul_i8g32_batched(const int8_t *q, const float *sa, int m, const int8_t *w,
                                                const uint16_t *sw, int n, int k, int batch, long long w_stride,
                                                long long sw_stride, float *y, int ldy, long long y_stride,
                                                void *stream) {
    MatmulArgs a{q, sa, m, k, w, sw, n, y, ldy, nullptr, nullptr, w_stride, sw_stride, y_stride, batch};
    int st = validate(a);
    if (st != NDL_OK) return st;
    return dispatch(a, (cudaStream_t)stream);
}
