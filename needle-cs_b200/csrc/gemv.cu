// I8G32 streaming GEMV: y[t][n] = sa[t] * sum_g half(sw[n][g]) * D[t][n][g]
// with D the exact int32 dot over one 32-column group, the group sum a chain
// of fused multiply-adds in ascending group order.
//
// Replaces Quant.MatMulRows -> Gemv.Rows/Block/Tile4/Tile2
// (src/Needle/Quant.cs:615-633, src/Needle/Gemv.cs:117-333) for the M < 64
// decode shapes.  Design:
//  * One warp owns 8 weight rows and one 16-row tile of activations and
//    walks every 32-column group in ascending order.  Each group is one
//    mma.sync.m16n8k32 (K = 32 = one group), so the int32 accumulator of an
//    MMA is exactly D for that group; the lane then folds its four (t, n)
//    results into fp32 accumulators, acc = fma(sw, D, acc), in group order,
//    and multiplies by the row's activation scale at the end.  That is the
//    oracle's definition bit for bit, and a row's result does not depend on
//    the batch it is in.
//  * Weight bytes are read once with L1-bypassing 8-byte loads; the next
//    eight groups' loads are issued before the current eight are computed
//    (8-16 loads in flight per lane) together with their scales (eight groups
//    per 16-byte load); the activations come from L1 as they are needed, which
//    keeps the kernel within 102 registers at 20 warps per SM.  The MMA computes sum_k A[t][k] B[k][n] over a
//    32-wide k slice; any permutation of k applied to both operands leaves
//    that sum unchanged, so each lane loads 8 contiguous bytes of its weight
//    row (group bytes 8*tig .. 8*tig+7) and the same 8 bytes of its two
//    activation rows: b0 = bytes 0..3, b1 = bytes 4..7, a0/a2 (row gid),
//    a1/a3 (row gid+8) likewise.
//  * int32 -> fp32 is exact by the 1.5*2^23 trick (|D| <= 32*128*128 < 2^22).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

__device__ __forceinline__ uint2 ld_stream_u2(const void *p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

__device__ __forceinline__ void mma_s8_16x8x32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Exact int32 -> fp32 for |d| < 2^22.
__device__ __forceinline__ float exact_i2f(int d) { return __int_as_float(d + 0x4B400000) - 12582912.0f; }

constexpr int kGemvWarps = 4;
constexpr int kGemvUnroll = 8;  // groups per iteration; the next iteration's weights load meanwhile

// Eight consecutive fp16 scales (groups g..g+7) of one weight row: one
// 16-byte load when rows are 16-byte aligned and G % 8 == 0.
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 gemv_scales8(const uint16_t *row, int g, int G, bool vec) {
    if (vec) return ld_stream_u4(row + g);
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = g + i < G ? (uint32_t)__ldg(row + g + i) : 0u;
    return make_uint4(h[0] | h[1] << 16, h[2] | h[3] << 16, h[4] | h[5] << 16, h[6] | h[7] << 16);
}
__device__ __forceinline__ uint16_t half_of(const uint4 &v, int i) {
    const uint32_t w = i < 2 ? v.x : i < 4 ? v.y : i < 6 ? v.z : v.w;
    return (uint16_t)((i & 1) ? w >> 16 : w & 0xFFFFu);
}

// Any half of these eight with exponent bits 11111 (the reference decodes
// those patterns without an Inf/NaN case)?
__device__ __forceinline__ bool any_max_exponent(const uint4 &v) {
    const uint32_t m = 0x7C007C00u;
    return __vcmpeq2(v.x & m, m) | __vcmpeq2(v.y & m, m) | __vcmpeq2(v.z & m, m) | __vcmpeq2(v.w & m, m);
}
__device__ __forceinline__ float half_plain(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// kAcc: also write every group's int32 D to a.acc (the parity tests' view).
// kFull: G % 8 == 0, so every 8-group chunk is whole and needs no bounds tests.
//
// Persistent: warp w walks the 8-row weight tiles w, w + W, ... of every
// batch entry (blockIdx.y selects the 16-row activation tile) as one stream
// of 8-group chunks; chunk c + 1, possibly the first chunk of the next tile,
// is loaded while chunk c is computed, so a warp's loads stay in flight
// across tile boundaries.  Weight rows past n and activation rows past m are
// read from row 0 instead (always valid memory): they only feed outputs that
// are never stored.
// kSmemA: the CTA first copies its 16 activation rows into shared memory (row
// pitch k + 32 bytes: the 8-byte fragment reads of a half-warp then hit 32
// distinct banks), so they are not evicted by the streamed weights and scales.
template <bool kAcc, bool kFull, bool kSmemA>
__global__ void __launch_bounds__(kGemvWarps * 32, 5) gemv_i8g32_kernel(MatmulArgs a, int scales_vec) {
    pdl_enter();
    extern __shared__ __align__(16) int8_t s_act[];
    const int lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int W = gridDim.x * kGemvWarps;
    const int G = a.k >> 5;
    const int chunks = (G + kGemvUnroll - 1) / kGemvUnroll;
    const int tiles_per = (a.n + 7) / 8;
    const int tiles = tiles_per * a.batch;  // the host checks that this fits an int
    const bool svec = scales_vec != 0;
    const int t0 = blockIdx.y * 16;
    const int ta = t0 + gid, tb = ta + 8;
    const bool va = ta < a.m, vb = tb < a.m;
    const int pitch = a.k + 32;
    if (kSmemA) {  // rows t0..t0+15 (rows past m: zeros), 16-byte copies
        const int per_row = a.k / 16;
        for (int i = threadIdx.x; i < 16 * per_row; i += blockDim.x) {
            const int r = i / per_row, c16 = i - r * per_row;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (t0 + r < a.m) v = __ldg(reinterpret_cast<const uint4 *>(a.q + (size_t)(t0 + r) * a.k) + c16);
            *reinterpret_cast<uint4 *>(s_act + r * pitch + c16 * 16) = v;
        }
        __syncthreads();
    }
    const int8_t *qa = kSmemA ? s_act + gid * pitch + 8 * tig : a.q + (size_t)(va ? ta : 0) * a.k + 8 * tig;
    const int8_t *qb = kSmemA ? s_act + (gid + 8) * pitch + 8 * tig : a.q + (size_t)(vb ? tb : 0) * a.k + 8 * tig;
    const float sa_a = va ? a.sa[ta] : 0.0f, sa_b = vb ? a.sa[tb] : 0.0f;

    int tile = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (tile >= tiles) return;
    struct Tile {
        const int8_t *wl;
        const uint16_t *s0p, *s1p;
        float *y;
        int nc;
    };
    auto make_tile = [&](int t) {
        Tile r;
        const int bz = t / tiles_per, tw = t - bz * tiles_per;
        const int nl = tw * 8 + gid;
        r.wl = a.w + (long long)bz * a.w_stride + (size_t)(nl < a.n ? nl : 0) * a.k + 8 * tig;
        r.nc = tw * 8 + 2 * tig;
        const uint16_t *sw = a.sw + (long long)bz * a.sw_stride;
        r.s0p = sw + (size_t)(r.nc < a.n ? r.nc : 0) * G;
        r.s1p = sw + (size_t)(r.nc + 1 < a.n ? r.nc + 1 : 0) * G;
        r.y = a.y + (long long)bz * a.y_stride;
        return r;
    };
    auto load_chunk = [&](const int8_t *wc, int g0, uint2 (&B)[kGemvUnroll]) {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; u++)
            B[u] = (kFull || g0 + u < G) ? ld_stream_u2(wc + u * 32) : make_uint2(0u, 0u);
    };
    Tile cur = make_tile(tile);
    uint2 B[kGemvUnroll];
    load_chunk(cur.wl, 0, B);
    uint4 S0 = gemv_scales8(cur.s0p, 0, G, svec), S1 = gemv_scales8(cur.s1p, 0, G, svec);
    int c = 0;
    const uint64_t neg_magic = f2_pack(-12582912.0f, -12582912.0f);
    uint64_t acc_a = 0ull, acc_b = 0ull;  // (t=ta: nc, nc+1), (t=tb: nc, nc+1)
    while (true) {
        // the stream position after this chunk
        int nt = tile, ncnk = c + 1;
        Tile nxt = cur;
        if (ncnk == chunks) {
            nt = tile + W;
            ncnk = 0;
            if (nt < tiles) nxt = make_tile(nt);
        }
        // the next chunk's weights and scales load while this one is computed
        uint2 Bn[kGemvUnroll];
        uint4 S0n = make_uint4(0u, 0u, 0u, 0u), S1n = S0n;
        if (nt < tiles) {
            load_chunk(nxt.wl + ncnk * 256, ncnk * kGemvUnroll, Bn);
            S0n = gemv_scales8(nxt.s0p, ncnk * kGemvUnroll, G, svec);
            S1n = gemv_scales8(nxt.s1p, ncnk * kGemvUnroll, G, svec);
        }
        const int g0 = c * kGemvUnroll;
        const bool special = any_max_exponent(S0) || any_max_exponent(S1);
        const int8_t *qac = qa + g0 * 32, *qbc = qb + g0 * 32;
#pragma unroll
        for (int u = 0; u < kGemvUnroll; u++) {
            if (!kFull && g0 + u >= G) break;
            uint2 A0, A1;
            if (kSmemA) {
                A0 = *reinterpret_cast<const uint2 *>(qac + u * 32);
                A1 = *reinterpret_cast<const uint2 *>(qbc + u * 32);
            } else {
                A0 = __ldg(reinterpret_cast<const uint2 *>(qac + u * 32));
                A1 = __ldg(reinterpret_cast<const uint2 *>(qbc + u * 32));
            }
            int d[4];
            mma_s8_16x8x32(d, A0.x, A1.x, A0.y, A1.y, B[u].x, B[u].y);
            float s0, s1;
            if (!special) {
                s0 = half_plain(half_of(S0, u));
                s1 = half_plain(half_of(S1, u));
            } else {
                s0 = half_to_float_ref_fast(half_of(S0, u));
                s1 = half_to_float_ref_fast(half_of(S1, u));
            }
            // acc = fma(sw, float(D), acc) per (t, n); float(D) exact by the 1.5*2^23 trick
            const uint64_t sc = f2_pack(s0, s1);
            acc_a = f2_fma(sc, f2_add(f2_pack(__int_as_float(d[0] + 0x4B400000), __int_as_float(d[1] + 0x4B400000)),
                                      neg_magic), acc_a);
            acc_b = f2_fma(sc, f2_add(f2_pack(__int_as_float(d[2] + 0x4B400000), __int_as_float(d[3] + 0x4B400000)),
                                      neg_magic), acc_b);
            if (kAcc) {
                const int g = g0 + u, nc = cur.nc;
                if (va && nc < a.n) a.acc[((size_t)ta * a.n + nc) * G + g] = d[0];
                if (va && nc + 1 < a.n) a.acc[((size_t)ta * a.n + nc + 1) * G + g] = d[1];
                if (vb && nc < a.n) a.acc[((size_t)tb * a.n + nc) * G + g] = d[2];
                if (vb && nc + 1 < a.n) a.acc[((size_t)tb * a.n + nc + 1) * G + g] = d[3];
            }
        }
        if (c + 1 == chunks) {  // tile done: outputs, then the next tile
            float v[4];
            f2_unpack(acc_a, v[0], v[1]);
            f2_unpack(acc_b, v[2], v[3]);
            const int nc = cur.nc;
            auto store = [&](int t, int n, float x) {
                size_t o = (size_t)t * a.ldy + n;
                cur.y[o] = a.residual ? __fadd_rn(a.residual[o], x) : x;
            };
            if (va && nc < a.n) store(ta, nc, __fmul_rn(v[0], sa_a));
            if (va && nc + 1 < a.n) store(ta, nc + 1, __fmul_rn(v[1], sa_a));
            if (vb && nc < a.n) store(tb, nc, __fmul_rn(v[2], sa_b));
            if (vb && nc + 1 < a.n) store(tb, nc + 1, __fmul_rn(v[3], sa_b));
            acc_a = acc_b = 0ull;
        }
        if (nt >= tiles) break;
        tile = nt;
        c = ncnk;
        cur = nxt;
        S0 = S0n;
        S1 = S1n;
#pragma unroll
        for (int u = 0; u < kGemvUnroll; u++) B[u] = Bn[u];
    }
}

// K <= 512 (kChunks = G / 8 = 1 or 2), vector scales, no int32 output: the
// warp's whole activation operand (16 rows x K, 4 registers per group) stays
// in registers, so the only memory traffic is the weight and scale stream
// and the outputs (5 - kChunks CTAs per SM fit the registers).  Same tile
// stream, prefetch and arithmetic as above.
template <int kChunks>
__global__ void __launch_bounds__(kGemvWarps * 32, 5 - kChunks) gemv_i8g32_reg_kernel(MatmulArgs a) {
    pdl_enter();
    constexpr int G = kChunks * kGemvUnroll;
    const int lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int W = gridDim.x * kGemvWarps;
    const int tiles_per = (a.n + 7) / 8;
    const int tiles = tiles_per * a.batch;
    const int t0 = blockIdx.y * 16;
    const int ta = t0 + gid, tb = ta + 8;
    const bool va = ta < a.m, vb = tb < a.m;
    int tile = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (tile >= tiles) return;
    // activation fragments of every group: rows ta, tb (rows past m: zeros)
    uint2 A0[G], A1[G];
    {
        const int8_t *qa = a.q + (size_t)(va ? ta : 0) * a.k + 8 * tig;
        const int8_t *qb = a.q + (size_t)(vb ? tb : 0) * a.k + 8 * tig;
#pragma unroll
        for (int g = 0; g < G; g++) {
            A0[g] = va ? __ldg(reinterpret_cast<const uint2 *>(qa + g * 32)) : make_uint2(0u, 0u);
            A1[g] = vb ? __ldg(reinterpret_cast<const uint2 *>(qb + g * 32)) : make_uint2(0u, 0u);
        }
    }
    const float sa_a = va ? a.sa[ta] : 0.0f, sa_b = vb ? a.sa[tb] : 0.0f;
    const uint64_t neg_magic = f2_pack(-12582912.0f, -12582912.0f);
    struct Tile {
        const int8_t *wl;
        const uint16_t *s0p, *s1p;
        float *y;
        int nc;
    };
    auto make_tile = [&](int t) {
        Tile r;
        const int bz = t / tiles_per, tw = t - bz * tiles_per;
        const int nl = tw * 8 + gid;
        r.wl = a.w + (long long)bz * a.w_stride + (size_t)(nl < a.n ? nl : 0) * a.k + 8 * tig;
        r.nc = tw * 8 + 2 * tig;
        const uint16_t *sw = a.sw + (long long)bz * a.sw_stride;
        r.s0p = sw + (size_t)(r.nc < a.n ? r.nc : 0) * G;
        r.s1p = sw + (size_t)(r.nc + 1 < a.n ? r.nc + 1 : 0) * G;
        r.y = a.y + (long long)bz * a.y_stride;
        return r;
    };
    Tile cur = make_tile(tile);
    uint2 B[kGemvUnroll];
#pragma unroll
    for (int u = 0; u < kGemvUnroll; u++) B[u] = ld_stream_u2(cur.wl + u * 32);
    uint4 S0 = ld_stream_u4(cur.s0p), S1 = ld_stream_u4(cur.s1p);
    while (true) {
        uint64_t acc_a = 0ull, acc_b = 0ull;  // (t=ta: nc, nc+1), (t=tb: nc, nc+1)
        const int nt = tile + W;
        Tile nxt = cur;
        if (nt < tiles) nxt = make_tile(nt);
#pragma unroll
        for (int c = 0; c < kChunks; c++) {
            // the next chunk (this tile's, or the next tile's first) loads meanwhile
            uint2 Bn[kGemvUnroll];
            uint4 S0n = make_uint4(0u, 0u, 0u, 0u), S1n = S0n;
            const bool last = c + 1 == kChunks;
            if (!last || nt < tiles) {
                const int8_t *wn = last ? nxt.wl : cur.wl + (c + 1) * 256;
#pragma unroll
                for (int u = 0; u < kGemvUnroll; u++) Bn[u] = ld_stream_u2(wn + u * 32);
                S0n = ld_stream_u4(last ? nxt.s0p : cur.s0p + (c + 1) * kGemvUnroll);
                S1n = ld_stream_u4(last ? nxt.s1p : cur.s1p + (c + 1) * kGemvUnroll);
            }
            const bool special = any_max_exponent(S0) || any_max_exponent(S1);
#pragma unroll
            for (int u = 0; u < kGemvUnroll; u++) {
                const int g = c * kGemvUnroll + u;
                int d[4];
                mma_s8_16x8x32(d, A0[g].x, A1[g].x, A0[g].y, A1[g].y, B[u].x, B[u].y);
                float s0, s1;
                if (!special) {
                    s0 = half_plain(half_of(S0, u));
                    s1 = half_plain(half_of(S1, u));
                } else {
                    s0 = half_to_float_ref_fast(half_of(S0, u));
                    s1 = half_to_float_ref_fast(half_of(S1, u));
                }
                // acc = fma(sw, float(D), acc) per (t, n); float(D) exact by the 1.5*2^23 trick
                const uint64_t sc = f2_pack(s0, s1);
                acc_a = f2_fma(sc, f2_add(f2_pack(__int_as_float(d[0] + 0x4B400000), __int_as_float(d[1] + 0x4B400000)),
                                          neg_magic), acc_a);
                acc_b = f2_fma(sc, f2_add(f2_pack(__int_as_float(d[2] + 0x4B400000), __int_as_float(d[3] + 0x4B400000)),
                                          neg_magic), acc_b);
            }
            S0 = S0n;
            S1 = S1n;
#pragma unroll
            for (int u = 0; u < kGemvUnroll; u++) B[u] = Bn[u];
        }
        float v[4];
        f2_unpack(acc_a, v[0], v[1]);
        f2_unpack(acc_b, v[2], v[3]);
        const int nc = cur.nc;
        auto store = [&](int t, int n, float x) {
            size_t o = (size_t)t * a.ldy + n;
            cur.y[o] = a.residual ? __fadd_rn(a.residual[o], x) : x;
        };
        if (va && nc < a.n) store(ta, nc, __fmul_rn(v[0], sa_a));
        if (va && nc + 1 < a.n) store(ta, nc + 1, __fmul_rn(v[1], sa_a));
        if (vb && nc < a.n) store(tb, nc, __fmul_rn(v[2], sa_b));
        if (vb && nc + 1 < a.n) store(tb, nc + 1, __fmul_rn(v[3], sa_b));
        if (nt >= tiles) break;
        tile = nt;
        cur = nxt;
    }
}

int launch_gemv_i8g32(const MatmulArgs &a, cudaStream_t stream) {
    const int sms = device_sm_count();
    const long long tiles = (long long)((a.n + 7) / 8) * a.batch;
    const long long mtiles = (a.m + 15) / 16;
    if (mtiles > 65535 || tiles + (long long)sms * 5 * kGemvWarps > 0x7fffffffLL)
        return set_error(NDL_ERR_INVALID_ARG, "gemv work too large");
    // persistent: five 4-warp CTAs per SM share the 8-row tiles of each 16-row activation tile
    const long long want = std::max<long long>(1, (long long)sms * 5 / mtiles);
    const long long blocks = std::min<long long>((tiles + kGemvWarps - 1) / kGemvWarps, want);
    dim3 grid((unsigned)blocks, (unsigned)mtiles, 1);
    const int G = a.k >> 5;
    const bool scales_vec = G % 8 == 0 && aligned(a.sw, 16) && (a.sw_stride * 2) % 16 == 0;
    const int sv = scales_vec ? 1 : 0;
    const bool full = G % kGemvUnroll == 0;
    // activations staged in shared memory when 16 rows fit in 48 KB (k <= 3040)
    const int smem = 16 * (a.k + 32);
    const bool sm_a = smem <= 48 * 1024;
    const dim3 blk(kGemvWarps * 32);
    if (!a.acc && scales_vec && (G == 8 || G == 16)) {  // K = 256 or 512: activations in registers
        const long long want_r = std::max<long long>(1, (long long)sms * (G == 8 ? 4 : 3) / mtiles);  // resident CTAs
        const dim3 grid_r((unsigned)std::min<long long>((tiles + kGemvWarps - 1) / kGemvWarps, want_r), (unsigned)mtiles, 1);
        if (G == 8) launch_kernel(gemv_i8g32_reg_kernel<1>, grid_r, blk, 0, stream, a);
        else launch_kernel(gemv_i8g32_reg_kernel<2>, grid_r, blk, 0, stream, a);
        return check_launch("gemv_i8g32_reg");
    }
#define NDL_GEMV(ACC, FULL, SMA) launch_kernel(gemv_i8g32_kernel<ACC, FULL, SMA>, dim3(grid), dim3(blk), SMA ? smem : 0, stream, a, sv)
    if (a.acc) {
        if (full) { if (sm_a) NDL_GEMV(true, true, true); else NDL_GEMV(true, true, false); }
        else { if (sm_a) NDL_GEMV(true, false, true); else NDL_GEMV(true, false, false); }
    } else {
        if (full) { if (sm_a) NDL_GEMV(false, true, true); else NDL_GEMV(false, true, false); }
        else { if (sm_a) NDL_GEMV(false, false, true); else NDL_GEMV(false, false, false); }
    }
#undef NDL_GEMV
    return check_launch("gemv_i8g32");
}

}  // namespace ndl
