// I8G32 GEMM on the 5th-generation tensor cores for packed batches (m >= 64).
//
// Same result as the streaming GEMV and the oracle (Scalar.MatMulRows
// skeleton, src/Needle/Scalar.cs:146-192, with raw int8 weights, 32-column
// groups and the per-row activation scale factored out), bit for bit:
//   y[t][n] = (residual) + sa[t] * (fma over g ascending of half(sw[n][g]) * D[t][n][g])
//
// One CTA computes a 128 x BN output tile (BN = 32, or 16 when 32 would
// leave fewer than two tiles per SM); two CTAs fit on an SM.
//  * warp 0 (one lane): TMA loads of the activation tile A [128 rows][128 B]
//    and the weight tile B [BN rows][128 B] per stage, 128-byte swizzle,
//    3- or 4-stage ring (no cluster multicast).
//  * warp 1: allocates 8*BN TMEM columns; one lane issues one
//    tcgen05.mma kind::i8 (M 128, N BN, K 32) per 32-column group, with
//    accumulate off, into its own BN-column accumulator: the four groups of
//    a stage fill one of two TMEM slots.  Each MMA's int32 result is
//    therefore exactly D of that group.
//  * warps 2..: epilogue, one per (TMEM lane quadrant, 16 columns).  Thread
//    (warp w, lane l) owns output row 32*(w%4)+l; per slot it reads the four
//    groups' D from TMEM, releases the slot, and for every group in
//    ascending order folds
//    acc = fma(sw, float(D), acc); the row's activation scale multiplies
//    the result once at the end.
// Every wait is bounded; on a timeout the CTA records kStatusTimeout,
// drains, frees TMEM and exits.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace ndl {

constexpr int kTcBlockM = 128;
constexpr int kTcBlockK = 128;  // bytes = 4 groups per stage
constexpr int kTcAccBufs = 4;
constexpr int kTcMaxGroups = 64;  // k <= 2048
constexpr int kTcATileBytes = kTcBlockM * kTcBlockK;  // 16 KB
constexpr uint32_t kTcWaitLimit = 1u << 26;

// BN = 16 or 32 output columns per CTA (two CTAs per SM fit); one epilogue
// warp per (TMEM lane quadrant, 16 columns).
template <int BN>
constexpr int tc_stages() {
    return 4;  // about 76 KB (BN 16) or 88 KB (BN 32): two CTAs per SM
}

template <int BN>
struct TcSmem {
    static constexpr int kStages = tc_stages<BN>();
    uint8_t a[kStages][kTcATileBytes];  // 1024-byte aligned (swizzle atoms)
    uint8_t b[kStages][BN * kTcBlockK];
    float swf[kTcMaxGroups][BN];  // decoded weight scales of the tile
    uint64_t full[kStages], empty[kStages], acc_full[kTcAccBufs], acc_empty[kTcAccBufs];
    uint32_t tmem_base;
    volatile int abort;
};

template <int BN>
__host__ __device__ constexpr int tc_threads() {
    return 64 + 8 * BN;  // 2 control warps + (BN / 16) * 4 epilogue warps
}

struct TcParams {
    int m, n, k, ldy, batch;
    const float *sa;
    const uint16_t *sw;
    long long sw_stride, y_stride;
    float *y;
    const float *residual;
    int32_t *acc;
    int *status;
};

template <int BN>
__device__ __forceinline__ bool tc_wait(TcSmem<BN> &s, uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity, kTcWaitLimit)) return true;
    s.abort = 1;
    return false;
}

template <int BN>
__global__ void __launch_bounds__(tc_threads<BN>(), 2)
    gemm_i8g32_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         TcParams p) {
    constexpr int kThreads = tc_threads<BN>();
    constexpr int kEpiWarps = 4 * (BN / 16);
    constexpr int kSlotCols = 4 * BN;                 // one smem stage = 4 groups = 4 accumulators
    constexpr uint32_t kTmemCols = kTcAccBufs / 2 * kSlotCols;  // two slots: 128 (BN 16) or 256 (BN 32)
    constexpr int kBTileBytes = BN * kTcBlockK;
    constexpr int kTcStages = TcSmem<BN>::kStages;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<BN> &s =
        *reinterpret_cast<TcSmem<BN> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kTcBlockM, n0 = blockIdx.y * BN, bz = blockIdx.z;
    const int G = p.k >> 5;
    const int n_stages = (G + 3) / 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTcStages; i++) mbar_init(&s.full[i], 1), mbar_init(&s.empty[i], 1);
        for (int i = 0; i < 2; i++) mbar_init(&s.acc_full[i], 1), mbar_init(&s.acc_empty[i], kEpiWarps);
        s.abort = 0;
        fence_mbar_init();
        prefetch_tmap(&map_a);
        prefetch_tmap(&map_b);
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            for (int st = 0; st < n_stages && !s.abort; st++) {
                const int slot = st % kTcStages;
                if (st >= kTcStages && !tc_wait(s, &s.empty[slot], ((st / kTcStages) - 1) & 1)) break;
                mbar_arrive_expect_tx(&s.full[slot], kTcATileBytes + kBTileBytes);
                tma_load_2d(s.a[slot], &map_a, st * kTcBlockK, m0, &s.full[slot]);
                tma_load_3d(s.b[slot], &map_b, st * kTcBlockK, n0, bz, &s.full[slot]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(kTcBlockM, BN);
            for (int st = 0; st < n_stages && !s.abort; st++) {
                const int slot = st % kTcStages, acc = st & 1;
                if (!tc_wait(s, &s.full[slot], (st / kTcStages) & 1)) break;
                if (st >= 2 && !tc_wait(s, &s.acc_empty[acc], ((st >> 1) - 1) & 1)) break;
                tc_fence_after();
                const uint64_t da0 = sw128_kmajor_desc(s.a[slot]), db0 = sw128_kmajor_desc(s.b[slot]);
                const int groups = min(4, G - 4 * st);
                for (int j = 0; j < groups; j++)
                    mma_i8(tmem + (uint32_t)(acc * kSlotCols + j * BN), da0 + (uint64_t)(j * 2),
                           db0 + (uint64_t)(j * 2), idesc, 0u);
                mma_commit(&s.acc_full[acc]);
                mma_commit(&s.empty[slot]);
            }
        }
    } else {
        // epilogue warp: lane quadrant (TMEM lanes 32*quad..), 16 columns at col0
        const int quad = warp & 3, col0 = ((warp - 2) >> 2) * 16;
        const int epi = threadIdx.x - 64;
        // decoded scales of this tile, swf[g][nl] = half(sw[n0+nl][g]), loaded
        // while the first TMA loads are in flight
        {
            const uint16_t *sw = p.sw + (long long)bz * p.sw_stride;
            for (int i = epi; i < BN * G; i += kThreads - 64) {
                const int nl = i / G, g = i - nl * G;
                const int n = n0 + nl;
                s.swf[g][nl] = n < p.n ? half_to_float_ref_fast(sw[(size_t)n * G + g]) : 0.0f;
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kThreads - 64) : "memory");
        }
        const int t = m0 + quad * 32 + lane;
        const bool tv = t < p.m;
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; j++) acc[j] = 0.0f;
        const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)col0;
        for (int st = 0; st < n_stages; st++) {
            const int a = st & 1;
            if (!tc_wait(s, &s.acc_full[a], (st >> 1) & 1)) break;
            tc_fence_after();
            const int groups = min(4, G - 4 * st);
            // two groups at a time (32 registers of D); the slot is released
            // once all four are in registers
#pragma unroll
            for (int h = 0; h < 2; h++) {
                uint32_t d[2][16];
#pragma unroll
                for (int jj = 0; jj < 2; jj++)
                    if (2 * h + jj < groups)
                        tmem_ld16(lane_addr + (uint32_t)(a * kSlotCols + (2 * h + jj) * BN), d[jj]);
                tmem_ld_wait();
                if (h == 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.acc_empty[a]);
                }
                // acc = fma(sw, float(D), acc) in ascending group order; float(D)
                // exact by the 1.5*2^23 trick
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    const int j = 2 * h + jj;
                    if (j >= groups) break;
                    const int g = 4 * st + j;
                    const float4 *sc = reinterpret_cast<const float4 *>(&s.swf[g][col0]);
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float4 w = sc[q];
                        acc[4 * q + 0] = __fmaf_rn(w.x, __int_as_float((int)d[jj][4 * q + 0] + 0x4B400000) - 12582912.0f, acc[4 * q + 0]);
                        acc[4 * q + 1] = __fmaf_rn(w.y, __int_as_float((int)d[jj][4 * q + 1] + 0x4B400000) - 12582912.0f, acc[4 * q + 1]);
                        acc[4 * q + 2] = __fmaf_rn(w.z, __int_as_float((int)d[jj][4 * q + 2] + 0x4B400000) - 12582912.0f, acc[4 * q + 2]);
                        acc[4 * q + 3] = __fmaf_rn(w.w, __int_as_float((int)d[jj][4 * q + 3] + 0x4B400000) - 12582912.0f, acc[4 * q + 3]);
                    }
                    if (p.acc && tv) {  // optional int32 accumulator output (parity checks)
                        int32_t *dst = p.acc + ((size_t)t * p.n + n0 + col0) * G + g;
                        const int cmax = min(16, p.n - (n0 + col0));
#pragma unroll
                        for (int c = 0; c < 16; c++)
                            if (c < cmax) dst[(size_t)c * G] = (int)d[jj][c];
                    }
                }
            }
        }
        if (tv && !s.abort) {
            const float sa = p.sa[t];
            float *y = p.y + (long long)bz * p.y_stride + (size_t)t * p.ldy;
            const float *res = p.residual ? p.residual + (size_t)t * p.ldy : nullptr;
            const int nb = n0 + col0;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int n = nb + j;
                if (n < p.n) {
                    const float v = __fmul_rn(acc[j], sa);
                    y[n] = res ? __fadd_rn(res[n], v) : v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (s.abort && threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusTimeout);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ------------------------------------------------------------- host side --
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *ptr = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// int8 [depth][rows][k] K-major, box 128 bytes x 128 rows, 128-byte swizzle.
static int make_map(CUtensorMap *map, const void *base, int k, int rows, int depth, long long depth_stride) {
    auto encode = get_encode();
    if (!encode) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)depth};
    cuuint64_t strides[2] = {(cuuint64_t)k, (cuuint64_t)(depth_stride > 0 ? depth_stride : (long long)k * rows)};
    cuuint32_t box[3] = {kTcBlockK, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, depth > 1 ? 3 : 2, const_cast<void *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NDL_OK;
}

template <int BN>
static int launch_bn(const CUtensorMap &map_a, const CUtensorMap &map_b, const TcParams &p, const MatmulArgs &a,
                     cudaStream_t stream) {
    const size_t smem = sizeof(TcSmem<BN>) + 1024;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i8g32_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
        configured = true;
    }
    dim3 grid((a.m + kTcBlockM - 1) / kTcBlockM, (a.n + BN - 1) / BN, a.batch);
    gemm_i8g32_tc_kernel<BN><<<grid, tc_threads<BN>(), smem, stream>>>(map_a, map_b, p);
    return check_launch("gemm_i8g32_tc");
}

// Weight tile rows per TMA box for a given BN.
static int make_weight_map(CUtensorMap *map, const MatmulArgs &a, int bn) {
    auto encode = get_encode();
    if (!encode) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)a.k, (cuuint64_t)a.n, (cuuint64_t)a.batch};
    cuuint64_t strides[2] = {(cuuint64_t)a.k, (cuuint64_t)(a.batch > 1 ? a.w_stride : (long long)a.k * a.n)};
    cuuint32_t box[3] = {kTcBlockK, (cuuint32_t)bn, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(a.w), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (%d)", (int)r);
    return NDL_OK;
}

int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream) {
    const int G = a.k >> 5;
    if (G > kTcMaxGroups || a.m < 64) return NDL_ERR_UNSUPPORTED;
    if (a.w_stride % 16 != 0) return NDL_ERR_UNSUPPORTED;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    // widest tile that still covers the SMs (two CTAs per SM fit for BN <= 64)
    const long long mt = (a.m + kTcBlockM - 1) / kTcBlockM * (long long)a.batch;
    // 32-column tiles when they still give two tiles per SM, else 16
    const int bn = mt * ((a.n + 31) / 32) >= 2 * sms ? 32 : 16;
    CUtensorMap map_a, map_b;
    int st = make_map(&map_a, a.q, a.k, a.m, 1, 0);
    if (st != NDL_OK) return st;
    st = make_weight_map(&map_b, a, bn);
    if (st != NDL_OK) return st;
    TcParams p{a.m, a.n, a.k, a.ldy, a.batch, a.sa, a.sw, a.sw_stride, a.y_stride, a.y, a.residual, a.acc, a.status};
    if (bn == 32) return launch_bn<32>(map_a, map_b, p, a, stream);
    return launch_bn<16>(map_a, map_b, p, a, stream);
}

}  // namespace ndl
