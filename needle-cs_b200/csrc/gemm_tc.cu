// I8G32 GEMM on the 5th-generation tensor cores for packed batches (m >= 64).
//
// Same result as the streaming GEMV and the oracle (Scalar.MatMulRows
// skeleton, src/Needle/Scalar.cs:146-192, with raw int8 weights, 32-column
// groups and the per-row activation scale factored out), bit for bit:
//   y[t][n] = (residual) + sa[t] * (fma over g ascending of half(sw[n][g]) * D[t][n][g])
//
// Persistent: one CTA per SM walks output tiles of 128 weight rows x BT
// tokens (BT = 16, 32 or 64, chosen on the host from the shape), tokens
// fastest so concurrently running CTAs share weight rows in L2.  The weights
// are the MMA's M operand, so TMEM lane = output feature n and each epilogue
// thread owns one n: its fp16 group scales are one contiguous row of sw and
// its stores are coalesced across the warp.
//  * warps 0..1 (loads, even / odd stages): per shared-memory stage (4
//    groups = 128 bytes of K) the weight tile [128 rows][128 B] and the
//    activation tile [BT rows][128 B], 128-byte swizzle, no cluster
//    multicast, 8 stages in flight.  Copies issued by one thread complete one
//    after another, so stage r's two loads come from lanes 2r and 2r + 1, in
//    one converged instruction; the first 8 stages go out together.  Weights
//    are constant: those stages' weight loads are issued before the wait on
//    the preceding kernel.
//  * warps 2..3 (MMA): one thread issues about one tcgen05.mma per 150
//    cycles, while lanes and warps issue in parallel, so the two warps take
//    alternate stages and lanes 0..3 each issue one group's MMA (kind::i8,
//    M 128, N BT, K 32, accumulate off: each accumulator holds exactly D of
//    one group), then commit it to the TMEM slot's full barrier and to the
//    stage's empty barrier.
//  * warps 4..11 (epilogue): (TMEM lane quadrant) x (BT / 2 token columns).
//    Three warps per scheduler leave the issuing warps their share of issue
//    slots and each epilogue thread up to 168 registers.
//    TMEM is a ring of slots of min(4, 128 / BT) groups.  A thread loads D
//    in batches of 4 / 2 / 1 groups (BT 16 / 32 / 64: 32 registers each),
//    one wait per batch, the next batch loading while it folds the current
//    one, acc = fma(half(sw[n][g]), float(D), acc), two tokens per packed
//    f32x2 instruction (a load round trip per group, not the fold, set the
//    pace before); a slot is released as soon as its last group is in
//    registers, and a finished tile (times the token's activation scale,
//    plus the residual) is written while the next tile's first batch loads.
// Every wait is bounded; on a timeout the CTA records kStatusTimeout, leaves
// its loops, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tc.cuh"

namespace ndl {

constexpr int kTcBlockN = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int kTcBlockK = 128;  // bytes of K per shared-memory stage = 4 groups
constexpr int kTcStages = 8;    // shared-memory ring depth
constexpr int kTcLoadWarps = 2;
constexpr int kTcMmaWarps = 2;
constexpr int kTcEpiWarps = 8;
constexpr int kTcEpiWarp0 = kTcLoadWarps + kTcMmaWarps;
constexpr int kTcThreads = 32 * (kTcEpiWarp0 + kTcEpiWarps);
constexpr uint32_t kTcTmemCols = 512;
constexpr int kTcWBytes = kTcBlockN * kTcBlockK;  // 16 KB
constexpr uint32_t kTcWaitLimit = 1u << 22;  // tests of about a microsecond each: a few seconds

template <int BT>
struct TcShape {
    static constexpr int kGroupsPerSlot = BT >= 64 ? 128 / BT : 4;
    static constexpr int kSlotCols = kGroupsPerSlot * BT;
    static constexpr int kSlots = kTcTmemCols / kSlotCols;  // 8 (BT 16) or 4
    static constexpr int kXBytes = BT * kTcBlockK;
    static constexpr int kCols = BT / 2;  // token columns per epilogue thread
    // groups per TMEM load batch (one wait per batch; two batches in flight):
    // 32 registers of accumulators per batch
    static constexpr int kBatch = kCols <= 8 ? 4 : kCols <= 16 ? 2 : 1;
    static_assert(kGroupsPerSlot % kBatch == 0 && 8 % (2 * kBatch) == 0, "batches tile slots and scale chunks");
};
// K groups per tile must fill whole batch pairs (and so whole TMEM slots).
__host__ __device__ constexpr int tc_group_multiple(int bt) { return bt <= 16 ? 8 : bt <= 32 ? 4 : 2; }

template <int BT>
struct TcSmem {
    uint8_t w[kTcStages][kTcWBytes];               // 1024-byte aligned (swizzle atoms)
    uint8_t x[kTcStages][TcShape<BT>::kXBytes];    // 2, 4 or 8 KB: stays 1024-aligned
    uint64_t full[kTcStages], empty[kTcStages];
    uint64_t acc_full[TcShape<BT>::kSlots], acc_empty[TcShape<BT>::kSlots];
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
// True when one of the eight halves is an infinity or a NaN (exponent 31):
// those take the exact slow conversion.
__device__ __forceinline__ bool tc_scales_special(uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    bool sp = false;
#pragma unroll
    for (int i = 0; i < 4; i++) sp |= (w[i] & 0x7C00u) == 0x7C00u || (w[i] & 0x7C000000u) == 0x7C000000u;
    return sp;
}

// acc = fma(s2, float(D), acc) for two tokens; the conversion is exact
// (|D| <= 2^19 < 2^24).
__device__ __forceinline__ void tc_fold2(uint64_t &acc, uint32_t d0, uint32_t d1, uint64_t s2) {
    acc = f2_fma(s2, f2_pack(__int2float_rn((int)d0), __int2float_rn((int)d1)), acc);
}

template <int BT, bool kAccOut, bool kResidual>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_i8g32_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                         TcParams p) {
    using Sh = TcShape<BT>;
    constexpr int EC = Sh::kCols, Q = Sh::kGroupsPerSlot, S = Sh::kSlots;
    constexpr uint32_t kStageBytes = kTcWBytes + Sh::kXBytes;
    extern __shared__ uint8_t smem_raw[];
    TcSmem<BT> &s =
        *reinterpret_cast<TcSmem<BT> *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.k >> 5;
    const int n_stages = (G + 3) >> 2;  // shared-memory stages per tile
    const int slots_per_tile = (G + Q - 1) / Q;
    const int nblk = (p.n + kTcBlockN - 1) / kTcBlockN, tblk = (p.m + BT - 1) / BT;
    const int tiles = p.batch * nblk * tblk;
    // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int my_tiles = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total_stages = my_tiles * n_stages;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kTcStages; i++) mbar_init(&s.full[i], 1), mbar_init(&s.empty[i], 4);
        for (int i = 0; i < S; i++) mbar_init(&s.acc_full[i], Q), mbar_init(&s.acc_empty[i], kTcEpiWarps);
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

    if (warp < kTcLoadWarps) {
        // Loads.  Stage i of this CTA = K block i % n_stages of its tile
        // number i / n_stages, ring position i % kTcStages; warp i % 2 issues
        // it.  The first kTcStages stages: lane 2r loads stage r's weights
        // (before the dependency wait), lane 2r + 1 its activations.
        {
            const int r = lane >> 1;
            const bool mine = r < min(kTcStages, total_stages) && r % kTcLoadWarps == warp;
            const int lt0 = r / n_stages, st0 = r - lt0 * n_stages;
            const TcTile t0 = tc_tile(blockIdx.x + lt0 * gridDim.x, nblk, tblk);
            if (mine && !(lane & 1)) {
                mbar_arrive_expect_tx(&s.full[r], kStageBytes);
                tma_load_3d(s.w[r], &map_w, st0 * kTcBlockK, t0.n0, t0.bz, &s.full[r]);
            }
            __syncwarp();
            pdl_wait();
            pdl_trigger();
            if (mine && (lane & 1)) tma_load_3d(s.x[r], &map_x, st0 * kTcBlockK, t0.tb * BT, 0, &s.full[r]);
            __syncwarp();
        }
        int i = kTcStages + warp, tile = blockIdx.x, st = i;
        while (st >= n_stages) st -= n_stages, tile += gridDim.x;
        TcTile tt = tc_tile(tile, nblk, tblk);
        for (; i < total_stages && !s.abort; i += kTcLoadWarps) {
            const int r = i % kTcStages;
            if (!tc_wait(s, &s.empty[r], ((i / kTcStages) - 1) & 1)) break;
            if (lane == 2 * r) mbar_arrive_expect_tx(&s.full[r], kStageBytes);
            __syncwarp();
            const bool wl = lane == 2 * r, xl = lane == 2 * r + 1;
            if (wl || xl)
                tma_load_3d(wl ? (void *)s.w[r] : (void *)s.x[r], wl ? &map_w : &map_x, st * kTcBlockK,
                            wl ? tt.n0 : tt.tb * BT, wl ? tt.bz : 0, &s.full[r]);
            __syncwarp();
            st += kTcLoadWarps;
            if (st >= n_stages) {
                while (st >= n_stages) st -= n_stages, tile += gridDim.x;
                tt = tc_tile(tile, nblk, tblk);
            }
        }
    } else if (warp < kTcEpiWarp0) {
        // MMA: warp kTcLoadWarps + w takes stages w, w + kTcMmaWarps, ...;
        // lane j < 4 issues group j of the stage and commits it.
        const uint32_t idesc = idesc_i8(kTcBlockN, BT);
        const int mw = warp - kTcLoadWarps;
        int lt = 0, st = mw;  // stage i = lt * n_stages + st
        while (st >= n_stages) st -= n_stages, lt++;
        for (int i = mw; i < total_stages && !s.abort; i += kTcMmaWarps) {
            const int r = i % kTcStages;
            if (!tc_wait(s, &s.full[r], (i / kTcStages) & 1)) break;
            const int groups = min(4, G - 4 * st);
            const int nsl = (groups + Q - 1) / Q;  // TMEM slots this stage fills
            const int sl0 = lt * slots_per_tile + (4 * st) / Q;
            bool ok = true;
            for (int k = 0; k < nsl && ok; k++) {
                const int sq = sl0 + k;
                if (sq >= S) ok = tc_wait(s, &s.acc_empty[sq % S], ((sq / S) - 1) & 1);
            }
            if (!ok) break;
            tc_fence_after();
            if (lane < 4) {
                const int sq = sl0 + lane / Q;
                if (lane < groups)
                    mma_i8(tmem + (uint32_t)((sq % S) * Sh::kSlotCols + (lane % Q) * BT),
                           sw128_kmajor_desc(s.w[r]) + (uint64_t)(lane * 2), sw128_kmajor_desc(s.x[r]) + (uint64_t)(lane * 2),
                           idesc, 0u);
                if (lane / Q < nsl) mma_commit(&s.acc_full[sq % S]);
                mma_commit(&s.empty[r]);
            }
            __syncwarp();
            st += kTcMmaWarps;
            while (st >= n_stages) st -= n_stages, lt++;
        }
    } else {
        // Epilogue.  TMEM loads go in batches of LG groups, one wait per
        // batch, the next batch loading while the current one folds: dA
        // holds batches 0, 2, ... and dB batches 1, 3, ... of each 8-group
        // scale chunk, so buffers, scale halves and slot positions are fixed
        // at compile time (LG divides Q and Q divides 8; G is a multiple of
        // 2 * LG, so every tile ends on a batch pair and a whole slot).
        constexpr int LG = Sh::kBatch;
        const int quad = warp & 3, c0 = ((warp - kTcEpiWarp0) >> 2) * EC;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0;
        const bool vec = p.sw_vec != 0;
        pdl_wait();
        pdl_trigger();
        uint32_t lsq = 0xFFFFFFFFu, slot_addr = 0;  // TMEM slot of the latest load
        auto next_slot = [&]() -> bool {  // wait for the next slot's MMAs
            lsq++;
            if (!tc_wait(s, &s.acc_full[lsq % S], (lsq / S) & 1)) return false;
            tc_fence_after();
            slot_addr = lane_base + (lsq % S) * Sh::kSlotCols;
            return true;
        };
        auto release_slot = [&]() {  // the latest slot is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.acc_empty[lsq % S]);
        };
        auto load_batch = [&](uint32_t (&d)[LG][EC], int pos) {  // groups at slot positions pos ..
#pragma unroll
            for (int i = 0; i < LG; i++) tmem_ld<EC>(slot_addr + (uint32_t)((pos + i) * BT), d[i]);
        };
        auto wait_batch = [&](uint32_t (&d)[LG][EC]) {
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < LG; i++)
#pragma unroll
                for (int c = 0; c < EC; c++) asm volatile("" : "+r"(d[i][c]));
        };
        auto scale_row = [&](int tile) {
            const TcTile tn = tc_tile(tile, nblk, tblk);
            const int nn = min(tn.n0 + quad * 32 + lane, p.n - 1);
            return p.sw + (long long)tn.bz * p.sw_stride + (size_t)nn * G;
        };
        uint32_t dA[LG][EC], dB[LG][EC];
        uint4 sc_nx = make_uint4(0u, 0u, 0u, 0u);
        bool ok = my_tiles > 0;
        if (ok) {
            sc_nx = tc_scales8(scale_row(blockIdx.x), 0, G, vec);
            ok = next_slot();
            if (ok) {
                load_batch(dA, 0);
                wait_batch(dA);
            }
        }
        for (int lt = 0; lt < my_tiles && ok; lt++) {
            const TcTile tt = tc_tile(blockIdx.x + lt * gridDim.x, nblk, tblk);
            const int n = tt.n0 + quad * 32 + lane, t0 = tt.tb * BT + c0;
            const bool nv = n < p.n, more_tiles = lt + 1 < my_tiles;
            const uint16_t *srow = p.sw + (long long)tt.bz * p.sw_stride + (size_t)min(n, p.n - 1) * G;
            // activation scales (lane c holds token t0 + c) and residuals: used at the end
            const float sa_l = lane < EC && t0 + lane < p.m ? __ldg(p.sa + t0 + lane) : 0.0f;
            float res[kResidual ? EC : 1];
            if constexpr (kResidual) {
#pragma unroll
                for (int c = 0; c < EC; c++)
                    res[c] = nv && t0 + c < p.m ? p.residual[(size_t)(t0 + c) * p.ldy + n] : 0.0f;
            }
            uint64_t acc[EC / 2];
#pragma unroll
            for (int c = 0; c < EC / 2; c++) acc[c] = 0ull;
            auto fold = [&](const uint32_t(&d)[EC], uint4 sc, int gi, bool special, int g) {
                const uint32_t hw = gi < 2 ? sc.x : gi < 4 ? sc.y : gi < 6 ? sc.z : sc.w;
                const uint16_t h = (uint16_t)((gi & 1) ? hw >> 16 : hw & 0xFFFFu);
                float scale = __half2float(__ushort_as_half(h));
                if (special) scale = half_to_float_ref_fast(h);
                const uint64_t s2 = f2_pack(scale, scale);
#pragma unroll
                for (int c = 0; c < EC / 2; c++) tc_fold2(acc[c], d[2 * c], d[2 * c + 1], s2);
                if constexpr (kAccOut) {  // int32 accumulators of every group (parity checks)
                    if (nv) {
#pragma unroll
                        for (int c = 0; c < EC; c++)
                            if (t0 + c < p.m) p.acc[((size_t)(t0 + c) * p.n + n) * G + g] = (int)d[c];
                    }
                }
            };
            for (int c8 = 0; c8 < G && ok; c8 += 8) {
                const uint4 sc = sc_nx;
                const bool special = tc_scales_special(sc);
                if (c8 + 8 < G) sc_nx = tc_scales8(srow, c8 + 8, G, vec);
                else if (more_tiles) sc_nx = tc_scales8(scale_row(blockIdx.x + (lt + 1) * gridDim.x), 0, G, vec);
#pragma unroll
                for (int bi = 0; bi < 8; bi += 2 * LG) {
                    const int g = c8 + bi;
                    if (g >= G) break;
                    // batch g .. g + LG - 1 is in dA; g + LG .. loads into dB (same tile)
                    const bool end_a = (bi + LG) % Q == 0;  // dA's batch ends its slot
                    if (end_a) {
                        release_slot();
                        ok = next_slot();
                    }
                    if (ok) load_batch(dB, (bi + LG) % Q);
#pragma unroll
                    for (int i = 0; i < LG; i++) fold(dA[i], sc, bi + i, special, g + i);
                    if (!ok) break;
                    wait_batch(dB);
                    // dB's batch ends its slot at a multiple of Q, always at the tile's end
                    const bool last = g + 2 * LG >= G;
                    const bool end_b = (bi + 2 * LG) % Q == 0;
                    if (end_b) release_slot();
                    // next into dA: g + 2 LG, or the next tile's first batch
                    const bool next = !last || more_tiles;
                    if (next) {
                        if (end_b) ok = next_slot();
                        if (ok) load_batch(dA, last ? 0 : (bi + 2 * LG) % Q);
                    }
#pragma unroll
                    for (int i = 0; i < LG; i++) fold(dB[i], sc, bi + LG + i, special, g + LG + i);
                    if (!ok) break;
                    if (next) wait_batch(dA);
                }
            }
            if (!ok) break;
            // tile done: y = (residual) + acc * sa
            float *y = p.y + (long long)tt.bz * p.y_stride;
#pragma unroll
            for (int c = 0; c < EC / 2; c++) {
                float v[2];
                f2_unpack(acc[c], v[0], v[1]);
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int cc = 2 * c + e;
                    const float sat = __shfl_sync(0xffffffffu, sa_l, cc);
                    if (nv && t0 + cc < p.m) {
                        const float out = __fmul_rn(v[e], sat);
                        float r = out;
                        if constexpr (kResidual) r = __fadd_rn(res[cc], out);
                        y[(size_t)(t0 + cc) * p.ldy + n] = r;
                    }
                }
            }
        }
        tmem_ld_wait();
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

static int tc_sms() { return device_sm_count(); }

template <int BT, bool kAccOut, bool kResidual>
static int launch_bt(const MatmulArgs &a, const TcParams &p, cudaStream_t stream) {
    auto kernel = gemm_i8g32_tc_kernel<BT, kAccOut, kResidual>;
    const size_t smem = sizeof(TcSmem<BT>) + 1024;
    static DeviceOnce smem_attribute;  // one per instantiation and device
    int st0 = smem_attribute.run([&] {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
        return (int)NDL_OK;
    });
    if (st0 != NDL_OK) return st0;
    CUtensorMap map_w, map_x;
    // weights [batch][n][k], activations [1][m][k]: both 3-D, so one load
    // instruction serves either
    int st = make_map(&map_w, a.w, a.k, a.n, a.batch, a.batch > 1 ? a.w_stride : 0, kTcBlockN, 3);
    if (st != NDL_OK) return st;
    st = make_map(&map_x, a.q, a.k, a.m, 1, 0, BT, 3);
    if (st != NDL_OK) return st;
    const long long tiles = (long long)a.batch * ((a.n + kTcBlockN - 1) / kTcBlockN) * ((a.m + BT - 1) / BT);
    if (tiles > 0x7fffffff) return NDL_ERR_UNSUPPORTED;
    const int grid = (int)std::min<long long>(tiles, tc_sms());
    launch_kernel(kernel, dim3(grid), dim3(kTcThreads), smem, stream, map_w, map_x, p);
    return check_launch("gemm_i8g32_tc");
}

template <int BT>
static int launch_bt(const MatmulArgs &a, const TcParams &p, cudaStream_t stream) {
    if constexpr (BT == 64) {  // no residual: its 32 registers do not fit beside 64-token tiles
        return a.acc ? launch_bt<64, true, false>(a, p, stream) : launch_bt<64, false, false>(a, p, stream);
    } else {
        if (a.acc) return a.residual ? launch_bt<BT, true, true>(a, p, stream) : launch_bt<BT, true, false>(a, p, stream);
        return a.residual ? launch_bt<BT, false, true>(a, p, stream) : launch_bt<BT, false, false>(a, p, stream);
    }
}

// Token tile: per 128-row x BT-token group an SM spends about the longer of
// the epilogue's fold (~28 / 36 / 46 elements per cycle at BT 16 / 32 / 64)
// and the MMA issue (~60 cycles), times the waves of tiles over the SMs;
// ties go to the larger tile (fewer weight re-reads from L2).
static int pick_bt(const MatmulArgs &a) {
    const int bts[3] = {16, 32, 64};
    const double rate[3] = {28.0, 36.0, 46.0};
    const long long nblk = (long long)a.batch * ((a.n + kTcBlockN - 1) / kTcBlockN);
    const int G = a.k >> 5;
    int best = 0;
    double best_t = 1e300;
    for (int i = 0; i < 3; i++) {
        if (G % tc_group_multiple(bts[i]) != 0) continue;
        if (bts[i] == 64 && a.residual) continue;  // 64-token tiles have no residual variant
        const long long tiles = nblk * ((a.m + bts[i] - 1) / bts[i]);
        const long long waves = (tiles + tc_sms() - 1) / tc_sms();
        const double t = (double)waves * std::max(60.0, 128.0 * bts[i] / rate[i]);
        if (t <= best_t) best_t = t, best = bts[i];
    }
    return best;
}

int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream) {
    if (a.m < 64) return NDL_ERR_UNSUPPORTED;
    if (a.w_stride % 16 != 0) return NDL_ERR_UNSUPPORTED;
    const int G = a.k >> 5;
    if (G % tc_group_multiple(64) != 0) return NDL_ERR_UNSUPPORTED;  // groups go in pairs
    const bool sw_vec = G % 8 == 0 && aligned(a.sw, 16) && (a.sw_stride * 2) % 16 == 0;
    TcParams p{a.m,     a.n, a.k,        a.ldy, a.batch,    a.sa, a.sw, a.sw_stride, a.y_stride, a.y, a.residual,
               a.acc, a.status, sw_vec ? 1 : 0};
    switch (pick_bt(a)) {
        case 64: return launch_bt<64>(a, p, stream);
        case 32: return launch_bt<32>(a, p, stream);
        case 16: return launch_bt<16>(a, p, stream);
        default: return NDL_ERR_UNSUPPORTED;  // no tile fits this K: the GEMV serves it
    }
}

}  // namespace ndl
