// I8G32 GEMM on the 5th-generation tensor cores for packed batches (m >= 64).
//
// Same result as the streaming GEMV and the scalar definition
// (Scalar.MatMulRows skeleton, src/Needle/Scalar.cs:146-192, with raw int8
// weights and 32-column groups), bit for bit:
//   y[t][n] = (residual) + sum_g (half(sw[n][g]) * sa[t]) * float(D[t][n][g])
//
// One CTA computes a 128 x BN output tile (BN = 64, or 32 when 64 would
// leave SMs without a tile); two CTAs fit on an SM.
//  * warp 0 (one lane): TMA loads of the activation tile A [128 rows][128 B]
//    and the weight tile B [BN rows][128 B] per stage, 128-byte swizzle,
//    3- or 4-stage ring (no cluster multicast).
//  * warp 1: allocates 4*BN TMEM columns; one lane issues one
//    tcgen05.mma kind::i8 (M 128, N BN, K 32) per 32-column group, with
//    accumulate off, into one of four BN-column TMEM buffers.  Each MMA's
//    int32 result is therefore exactly D of that group.
//  * warps 2..: epilogue, one per (TMEM lane quadrant, 32 columns).  Thread
//    (warp w, lane l) owns output row 32*(w%4)+l; for every group in
//    ascending order it reads
//    D from TMEM, releases the buffer, and folds
//    acc += (sw * sa) * float(D) with round-to-nearest multiplies and adds.
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

// BN = 32 or 64 output columns per CTA (two CTAs per SM fit); one epilogue
// warp per (TMEM lane quadrant, 32 columns).
template <int BN>
constexpr int tc_stages() {
    return BN == 64 ? 3 : 4;  // ~90 KB of shared memory either way: two CTAs per SM
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
    return 64 + 4 * BN;  // 2 control warps + (BN / 32) * 4 epilogue warps
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
    constexpr int kEpiWarps = 4 * (BN / 32);
    constexpr uint32_t kTmemCols = kTcAccBufs * BN;  // 128 or 256: a power of two
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
        for (int i = 0; i < kTcAccBufs; i++) mbar_init(&s.acc_full[i], 1), mbar_init(&s.acc_empty[i], kEpiWarps);
        s.abort = 0;
        fence_mbar_init();
        prefetch_tmap(&map_a);
        prefetch_tmap(&map_b);
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTmemCols);
        tmem_relinquish();
    }
    // decoded scales of this tile: swf[g][nl] = half(sw[n0+nl][g]) (coalesced rows)
    {
        const uint16_t *sw = p.sw + (long long)bz * p.sw_stride;
        for (int i = threadIdx.x; i < BN * G; i += kThreads) {
            const int nl = i / G, g = i - nl * G;
            const int n = n0 + nl;
            s.swf[g][nl] = n < p.n ? half_to_float_ref_fast(sw[(size_t)n * G + g]) : 0.0f;
        }
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
            for (int g = 0; g < G && !s.abort; g++) {
                const int st = g >> 2, j = g & 3, slot = st % kTcStages, buf = g % kTcAccBufs;
                if (j == 0 && !tc_wait(s, &s.full[slot], (st / kTcStages) & 1)) break;
                if (g >= kTcAccBufs && !tc_wait(s, &s.acc_empty[buf], ((g / kTcAccBufs) - 1) & 1)) break;
                tc_fence_after();
                const uint64_t da = sw128_kmajor_desc(s.a[slot]) + (uint64_t)(j * 2);
                const uint64_t db = sw128_kmajor_desc(s.b[slot]) + (uint64_t)(j * 2);
                mma_i8(tmem + (uint32_t)(buf * BN), da, db, idesc, 0u);
                mma_commit(&s.acc_full[buf]);
                if (j == 3 || g == G - 1) mma_commit(&s.empty[slot]);
            }
        }
    } else {
        // epilogue warp: lane quadrant (TMEM lanes 32*quad..), 32 columns at col0
        const int quad = warp & 3, col0 = ((warp - 2) >> 2) * 32;
        const int t = m0 + quad * 32 + lane;
        const bool tv = t < p.m;
        const float sa = tv ? p.sa[t] : 0.0f;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; j++) acc[j] = 0.0f;
        const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)col0;
        for (int g = 0; g < G; g++) {
            const int buf = g % kTcAccBufs;
            if (!tc_wait(s, &s.acc_full[buf], (g / kTcAccBufs) & 1)) break;
            tc_fence_after();
            uint32_t d[32];
            tmem_ld32(lane_addr + (uint32_t)(buf * BN), d);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.acc_empty[buf]);
            const float4 *sc = reinterpret_cast<const float4 *>(&s.swf[g][col0]);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const float4 w = sc[q];
                acc[4 * q + 0] = __fadd_rn(acc[4 * q + 0], __fmul_rn(__fmul_rn(w.x, sa), __int_as_float((int)d[4 * q + 0] + 0x4B400000) - 12582912.0f));
                acc[4 * q + 1] = __fadd_rn(acc[4 * q + 1], __fmul_rn(__fmul_rn(w.y, sa), __int_as_float((int)d[4 * q + 1] + 0x4B400000) - 12582912.0f));
                acc[4 * q + 2] = __fadd_rn(acc[4 * q + 2], __fmul_rn(__fmul_rn(w.z, sa), __int_as_float((int)d[4 * q + 2] + 0x4B400000) - 12582912.0f));
                acc[4 * q + 3] = __fadd_rn(acc[4 * q + 3], __fmul_rn(__fmul_rn(w.w, sa), __int_as_float((int)d[4 * q + 3] + 0x4B400000) - 12582912.0f));
            }
            if (p.acc && tv) {  // optional int32 accumulator output (parity checks)
                int32_t *dst = p.acc + ((size_t)t * p.n + n0 + col0) * G + g;
                const int jmax = min(32, p.n - (n0 + col0));
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (j < jmax) dst[(size_t)j * G] = (int)d[j];
            }
        }
        if (tv && !s.abort) {
            float *y = p.y + (long long)bz * p.y_stride + (size_t)t * p.ldy;
            const float *res = p.residual ? p.residual + (size_t)t * p.ldy : nullptr;
            const int nb = n0 + col0;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int n = nb + j;
                if (n < p.n) y[n] = res ? __fadd_rn(res[n], acc[j]) : acc[j];
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
    const int bn = mt * ((a.n + 63) / 64) >= sms ? 64 : 32;
    CUtensorMap map_a, map_b;
    int st = make_map(&map_a, a.q, a.k, a.m, 1, 0);
    if (st != NDL_OK) return st;
    st = make_weight_map(&map_b, a, bn);
    if (st != NDL_OK) return st;
    TcParams p{a.m, a.n, a.k, a.ldy, a.batch, a.sa, a.sw, a.sw_stride, a.y_stride, a.y, a.residual, a.acc, a.status};
    if (bn == 64) return launch_bn<64>(map_a, map_b, p, a, stream);
    return launch_bn<32>(map_a, map_b, p, a, stream);
}

}  // namespace ndl
