// I8G32 GEMM on the 5th-generation tensor cores for packed batches (m >= 64).
//
// Same result as the streaming GEMV and the oracle (Scalar.MatMulRows
// skeleton, src/Needle/Scalar.cs:146-192, with raw int8 weights, 32-column
// groups and the per-row activation scale factored out), bit for bit:
//   y[t][n] = (residual) + sa[t] * (fma over g ascending of half(sw[n][g]) * D[t][n][g])
//
// Persistent: one CTA per SM walks output tiles of 128 weight rows x BT
// tokens (BT = 32, or 16 when 32 would leave SMs idle), tokens fastest so
// concurrent CTAs share weight rows in L2.  The weights are the MMA's M
// operand, so TMEM lane = output feature n and each epilogue thread owns
// one n: its fp16 group scales are one contiguous row of sw and its stores
// are coalesced across the warp.
//  * warp 0: TMA loads of the weight tile [128 rows][128 B] and the
//    activation tile [BT rows][128 B] per stage (4 groups), 128-byte
//    swizzle, running ahead across tiles (no cluster multicast).  Copies
//    issued by one thread complete one after another, so every load in
//    flight is issued by its own lane.
//  * warp 1: allocates all 512 TMEM columns; elect.sync issues one
//    tcgen05.mma kind::i8 (M 128, N BT, K 32) per 32-column group with
//    accumulate off, so each accumulator holds exactly D of that group.  A
//    stage's four groups fill TMEM slot r of a 512 / (4 BT)-slot ring; one
//    commit per stage both fills the slot and frees shared-memory stage r.
//  * warps 2..17: epilogue, (TMEM lane quadrant) x (BT / 4 token columns).
//    Per slot a thread reads its four groups' D, releases the slot and folds
//    acc = fma(half(sw[n][g]), float(D), acc) in ascending group order, two
//    tokens per packed f32x2 instruction; the token's activation scale
//    multiplies once per tile.
// Every wait is bounded; on a timeout the CTA records kStatusTimeout, leaves
// its loops, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace ndl {

constexpr int kTcBlockN = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int kTcBlockK = 128;  // bytes per stage = 4 groups
constexpr int kTcEpiWarps = 16;
constexpr int kTcThreads = 64 + 32 * kTcEpiWarps;
constexpr uint32_t kTcTmemCols = 512;
constexpr int kTcWBytes = kTcBlockN * kTcBlockK;  // 16 KB
constexpr uint32_t kTcWaitLimit = 1u << 22;  // tests of about a microsecond each: a few seconds

// One stage of shared memory per TMEM slot (4 groups x BT columns), so the
// MMA commit that fills slot r also frees stage r: S = 512 / (4 BT).
template <int BT>
struct TcSmem {
    static constexpr int kStages = kTcTmemCols / (4 * BT);
    uint8_t w[kStages][kTcWBytes];      // 1024-byte aligned (swizzle atoms)
    uint8_t x[kStages][BT * kTcBlockK];  // 2 or 4 KB: stays 1024-aligned
    uint64_t full[kStages], acc_full[kStages], acc_empty[kStages];
    uint32_t tmem_base;
    volatile int abort;
};

struct TcParams {
    int m, n, k, ldy, batch;
    const float *sa;
    const uint16_t *sw;
    long long sw_stride, y_stride;
    float *y;
    const float *residual;
    int32_t *acc;
    int *status;
    int sw_vec;  // rows of sw are 16-byte aligned and G % 8 == 0
};

template <int BT>
__device__ __forceinline__ bool tc_wait(TcSmem<BT> &s, uint64_t *bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity, kTcWaitLimit)) return true;
    s.abort = 1;
    return false;
}

struct TcTile {
    int bz, n0, tb;  // batch, first weight row, token block
};
__device__ __forceinline__ TcTile tc_tile(int tile, int nblk, int tblk) {
    const int tb = tile % tblk, r = tile / tblk;
    return TcTile{r / nblk, (r % nblk) * kTcBlockN, tb};
}

// Eight consecutive fp16 group scales of one weight row (groups c8..c8+7).
__device__ __forceinline__ uint4 tc_scales8(const uint16_t *row, int c8, int G, bool vec) {
    if (vec) return __ldg(reinterpret_cast<const uint4 *>(row + c8));
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = c8 + i < G ? (uint32_t)__ldg(row + c8 + i) : 0u;
    return make_uint4(h[0] | h[1] << 16, h[2] | h[3] << 16, h[4] | h[5] << 16, h[6] | h[7] << 16);
}

template <int BT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_i8g32_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                         TcParams p) {
    pdl_enter();
    constexpr int EC = BT / 4;  // token columns per epilogue warp
    constexpr int kSlotCols = 4 * BT;
    constexpr int S = TcSmem<BT>::kStages;
    constexpr uint32_t kXBytes = BT * kTcBlockK;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<BT> &s =
        *reinterpret_cast<TcSmem<BT> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.k >> 5;
    const int n_stages = (G + 3) >> 2;
    const int nblk = (p.n + kTcBlockN - 1) / kTcBlockN, tblk = (p.m + BT - 1) / BT;
    const int tiles = p.batch * nblk * tblk;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++)
            mbar_init(&s.full[i], 1), mbar_init(&s.acc_full[i], 1), mbar_init(&s.acc_empty[i], kTcEpiWarps);
        s.abort = 0;
        fence_mbar_init();
        prefetch_tmap(&map_w);
        prefetch_tmap(&map_x);
    }
    if (warp == 1) {
        tmem_alloc(&s.tmem_base, kTcTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        // Producer, warp-converged.  Copies issued by one thread complete one
        // after another, so stage seq's weight and activation tiles are issued
        // by lanes 2(seq % S) and 2(seq % S) + 1: every load in flight has its
        // own thread.  Stage r is reused once the MMAs that read it committed
        // (acc_full[r]).
        uint32_t seq = 0;
        for (int tile = blockIdx.x; tile < tiles && !s.abort; tile += gridDim.x) {
            const TcTile tt = tc_tile(tile, nblk, tblk);
            for (int st = 0; st < n_stages; st++, seq++) {
                const int r = seq % S;
                if (seq >= (uint32_t)S && !tc_wait(s, &s.acc_full[r], ((seq / S) - 1) & 1)) break;
                const int lw = 2 * r;
                if (lane == lw) {
                    mbar_arrive_expect_tx(&s.full[r], kTcWBytes + kXBytes);
                    tma_load_3d(s.w[r], &map_w, st * kTcBlockK, tt.n0, tt.bz, &s.full[r]);
                } else if (lane == lw + 1) {
                    tma_load_2d(s.x[r], &map_x, st * kTcBlockK, tt.tb * BT, &s.full[r]);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issuer, warp-converged with elect.sync: one commit per stage
        const uint32_t idesc = idesc_i8(kTcBlockN, BT);
        uint32_t seq = 0;
        for (int tile = blockIdx.x; tile < tiles && !s.abort; tile += gridDim.x) {
            for (int st = 0; st < n_stages && !s.abort; st++, seq++) {
                const int r = seq % S;
                if (!tc_wait(s, &s.full[r], (seq / S) & 1)) break;
                if (seq >= (uint32_t)S && !tc_wait(s, &s.acc_empty[r], ((seq / S) - 1) & 1)) break;
                __syncwarp();
                tc_fence_after();
                const uint64_t dw = sw128_kmajor_desc(s.w[r]), dx = sw128_kmajor_desc(s.x[r]);
                const int groups = min(4, G - 4 * st);
                for (int j = 0; j < groups; j++)
                    mma_i8_elect(tmem + (uint32_t)(r * kSlotCols + j * BT), dw + (uint64_t)(j * 2),
                                 dx + (uint64_t)(j * 2), idesc);
                mma_commit_elect(&s.acc_full[r]);
            }
        }
    } else {
        const int quad = warp & 3, c0 = ((warp - 2) >> 2) * EC;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0;
        const bool vec = p.sw_vec != 0;
        const uint64_t neg_magic = f2_pack(-12582912.0f, -12582912.0f);
        uint32_t seq = 0;
        bool ok = true;
        // first scale chunk of the next tile, loaded one tile ahead
        uint4 sc_first = make_uint4(0u, 0u, 0u, 0u);
        if ((int)blockIdx.x < tiles) {
            const TcTile t0 = tc_tile(blockIdx.x, nblk, tblk);
            const int n = min(t0.n0 + quad * 32 + lane, p.n - 1);
            sc_first = tc_scales8(p.sw + (long long)t0.bz * p.sw_stride + (size_t)n * G, 0, G, vec);
        }
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const TcTile tt = tc_tile(tile, nblk, tblk);
            const int n = tt.n0 + quad * 32 + lane;
            const bool nv = n < p.n;
            const uint16_t *srow = p.sw + (long long)tt.bz * p.sw_stride + (size_t)(nv ? n : 0) * G;
            uint4 sc = sc_first;
            uint4 sc_next = G > 8 ? tc_scales8(srow, 8, G, vec) : make_uint4(0u, 0u, 0u, 0u);
            if (tile + (int)gridDim.x < tiles) {
                const TcTile tn = tc_tile(tile + gridDim.x, nblk, tblk);
                const int nn = min(tn.n0 + quad * 32 + lane, p.n - 1);
                sc_first = tc_scales8(p.sw + (long long)tn.bz * p.sw_stride + (size_t)nn * G, 0, G, vec);
            }
            // this tile's activation scales and residuals, needed at the end
            float sa[EC], res[EC];
#pragma unroll
            for (int c = 0; c < EC; c++) {
                const int t = tt.tb * BT + c0 + c;
                const bool ok_t = t < p.m && nv;
                sa[c] = ok_t ? __ldg(p.sa + t) : 0.0f;
                res[c] = ok_t && p.residual ? p.residual[(size_t)t * p.ldy + n] : 0.0f;
            }
            uint64_t acc[EC / 2];
#pragma unroll
            for (int c = 0; c < EC / 2; c++) acc[c] = 0ull;
            for (int st = 0; st < n_stages; st++, seq++) {
                const int r = seq % S;
                if (!tc_wait(s, &s.acc_full[r], (seq / S) & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int groups = min(4, G - 4 * st);
                // all four groups' D in registers with one wait, then the slot is released
                uint32_t d[4][EC];
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (j < groups) tmem_ld<EC>(lane_base + (uint32_t)(r * kSlotCols + j * BT), d[j]);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s.acc_empty[r]);
                // scales of groups 4st..4st+3: half (st & 1) of the current 8-group chunk
                const uint32_t w01 = (st & 1) ? sc.z : sc.x, w23 = (st & 1) ? sc.w : sc.y;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (j >= groups) break;
                    const uint32_t hw = j < 2 ? w01 : w23;
                    const float scale = half_to_float_ref_fast((uint16_t)((j & 1) ? hw >> 16 : hw & 0xFFFFu));
                    const uint64_t sc2 = f2_pack(scale, scale);
                    // acc = fma(sw, float(D), acc); float(D) exact by the 1.5*2^23 trick
#pragma unroll
                    for (int c = 0; c < EC / 2; c++) {
                        const uint64_t dv = f2_add(f2_pack(__int_as_float((int)d[j][2 * c] + 0x4B400000),
                                                           __int_as_float((int)d[j][2 * c + 1] + 0x4B400000)),
                                                   neg_magic);
                        acc[c] = f2_fma(sc2, dv, acc[c]);
                    }
                    if (p.acc && nv) {  // optional int32 accumulator output (parity checks)
                        const int g = 4 * st + j;
#pragma unroll
                        for (int c = 0; c < EC; c++) {
                            const int t = tt.tb * BT + c0 + c;
                            if (t < p.m) p.acc[((size_t)t * p.n + n) * G + g] = (int)d[j][c];
                        }
                    }
                }
                if (st & 1) {  // next 8-group chunk
                    sc = sc_next;
                    const int c8 = 8 * ((st >> 1) + 2);
                    if (c8 < G) sc_next = tc_scales8(srow, c8, G, vec);
                }
            }
            if (!ok || s.abort) break;
            if (nv) {
                float *y = p.y + (long long)tt.bz * p.y_stride;
#pragma unroll
                for (int c = 0; c < EC / 2; c++) {
                    float v[2];
                    f2_unpack(acc[c], v[0], v[1]);
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const int t = tt.tb * BT + c0 + 2 * c + e;
                        if (t < p.m) {
                            const float out = __fmul_rn(v[e], sa[2 * c + e]);
                            y[(size_t)t * p.ldy + n] = p.residual ? __fadd_rn(res[2 * c + e], out) : out;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (s.abort && threadIdx.x == 0 && p.status) atomicOr(p.status, kStatusTimeout);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTcTmemCols);
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

// int8 [depth][rows][k] K-major tensor map with a box of 128 bytes x box_rows,
// 128-byte swizzle.
static int make_map(CUtensorMap *map, const void *base, int k, int rows, int depth, long long depth_stride,
                    int box_rows, int rank) {
    auto encode = get_encode();
    if (!encode) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)depth};
    cuuint64_t strides[2] = {(cuuint64_t)k, (cuuint64_t)(depth_stride > 0 ? depth_stride : (long long)k * rows)};
    cuuint32_t box[3] = {kTcBlockK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void *>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(NDL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NDL_OK;
}

static int tc_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    return sms;
}

template <int BT>
static int launch_bt(const MatmulArgs &a, const TcParams &p, cudaStream_t stream) {
    const size_t smem = sizeof(TcSmem<BT>) + 1024;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_i8g32_tc_kernel<BT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
        configured = true;
    }
    CUtensorMap map_w, map_x;
    // weights [batch][n][k] (a 3-D map even for batch 1: the kernel issues
    // 3-D loads), activations [m][k] (2-D)
    int st = make_map(&map_w, a.w, a.k, a.n, a.batch, a.batch > 1 ? a.w_stride : 0, kTcBlockN, 3);
    if (st != NDL_OK) return st;
    st = make_map(&map_x, a.q, a.k, a.m, 1, 0, BT, 2);
    if (st != NDL_OK) return st;
    const long long tiles = (long long)a.batch * ((a.n + kTcBlockN - 1) / kTcBlockN) * ((a.m + BT - 1) / BT);
    if (tiles > 0x7fffffff) return NDL_ERR_UNSUPPORTED;
    const int grid = (int)std::min<long long>(tiles, tc_sms());
    launch_kernel(gemm_i8g32_tc_kernel<BT>, dim3(grid), dim3(kTcThreads), smem, stream, map_w, map_x, p);
    return check_launch("gemm_i8g32_tc");
}

int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream) {
    if (a.m < 64) return NDL_ERR_UNSUPPORTED;
    if (a.w_stride % 16 != 0) return NDL_ERR_UNSUPPORTED;
    const int G = a.k >> 5;
    const bool sw_vec = G % 8 == 0 && aligned(a.sw, 16) && (a.sw_stride * 2) % 16 == 0;
    TcParams p{a.m,     a.n, a.k,        a.ldy, a.batch,    a.sa, a.sw, a.sw_stride, a.y_stride, a.y, a.residual,
               a.acc, a.status, sw_vec ? 1 : 0};
    // 32-token tiles when they still give every SM a tile, else 16
    const long long nblk = (long long)a.batch * ((a.n + kTcBlockN - 1) / kTcBlockN);
    if (nblk * ((a.m + 31) / 32) >= tc_sms()) return launch_bt<32>(a, p, stream);
    return launch_bt<16>(a, p, stream);
}

}  // namespace ndl
