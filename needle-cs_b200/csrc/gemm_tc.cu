// tcgen05 kind::i8 GEMM for packed batches (m >= 64).
#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream) {
    (void)a;
    (void)stream;
    return NDL_ERR_UNSUPPORTED;
}

}  // namespace ndl
