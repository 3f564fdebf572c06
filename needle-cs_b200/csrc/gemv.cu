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
//  * Weight bytes are read once with L1-bypassing 8-byte loads, eight groups
//    in flight per lane.  The MMA computes sum_k A[t][k] B[k][n] over a
//    32-wide k slice; any permutation of k applied to both operands leaves
//    that sum unchanged, so each lane loads 8 contiguous bytes of its weight
//    row (group bytes 8*tig .. 8*tig+7) and the same 8 bytes of its two
//    activation rows: b0 = bytes 0..3, b1 = bytes 4..7, a0/a2 (row gid),
//    a1/a3 (row gid+8) likewise.
//  * int32 -> fp32 is exact by the 1.5*2^23 trick (|D| <= 32*128*128 < 2^22).
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
constexpr int kGemvUnroll = 8;  // groups in flight per lane

__global__ void __launch_bounds__(kGemvWarps * 32) gemv_i8g32_kernel(MatmulArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int tile = blockIdx.x * kGemvWarps + warp;  // 8-row weight tile
    if (tile * 8 >= a.n) return;
    const int G = a.k >> 5;
    const int b = blockIdx.z;
    const int8_t *w = a.w + (long long)b * a.w_stride;
    const uint16_t *sw = a.sw + (long long)b * a.sw_stride;
    float *y = a.y + (long long)b * a.y_stride;

    const int nl = tile * 8 + gid;  // weight row this lane loads
    const int nc = tile * 8 + 2 * tig;  // output columns nc, nc+1
    const int t0 = blockIdx.y * 16;
    const int ta = t0 + gid, tb = ta + 8;
    const bool va = ta < a.m, vb = tb < a.m;
    const bool vl = nl < a.n, vc0 = nc < a.n, vc1 = nc + 1 < a.n;
    const int8_t *wl = w + (size_t)(vl ? nl : 0) * a.k + 8 * tig;
    const int8_t *qa = a.q + (size_t)(va ? ta : 0) * a.k + 8 * tig;
    const int8_t *qb = a.q + (size_t)(vb ? tb : 0) * a.k + 8 * tig;
    const uint16_t *s0p = sw + (size_t)(vc0 ? nc : 0) * G;
    const uint16_t *s1p = sw + (size_t)(vc1 ? nc + 1 : 0) * G;
    const float sa_a = va ? a.sa[ta] : 0.0f, sa_b = vb ? a.sa[tb] : 0.0f;

    float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
    for (int g0 = 0; g0 < G; g0 += kGemvUnroll) {
        uint2 B[kGemvUnroll], A0[kGemvUnroll], A1[kGemvUnroll];
        uint16_t h0[kGemvUnroll], h1[kGemvUnroll];
#pragma unroll
        for (int u = 0; u < kGemvUnroll; u++) {
            const int g = g0 + u;
            const bool in = g < G;
            B[u] = (in && vl) ? ld_stream_u2(wl + g * 32) : make_uint2(0u, 0u);
            A0[u] = (in && va) ? __ldg(reinterpret_cast<const uint2 *>(qa + g * 32)) : make_uint2(0u, 0u);
            A1[u] = (in && vb) ? __ldg(reinterpret_cast<const uint2 *>(qb + g * 32)) : make_uint2(0u, 0u);
            h0[u] = in ? __ldg(s0p + g) : (uint16_t)0;
            h1[u] = in ? __ldg(s1p + g) : (uint16_t)0;
        }
#pragma unroll
        for (int u = 0; u < kGemvUnroll; u++) {
            if (g0 + u >= G) break;
            int d[4];
            mma_s8_16x8x32(d, A0[u].x, A1[u].x, A0[u].y, A1[u].y, B[u].x, B[u].y);
            const float s0 = half_to_float_ref_fast(h0[u]), s1 = half_to_float_ref_fast(h1[u]);
            acc0 = __fmaf_rn(s0, exact_i2f(d[0]), acc0);
            acc1 = __fmaf_rn(s1, exact_i2f(d[1]), acc1);
            acc2 = __fmaf_rn(s0, exact_i2f(d[2]), acc2);
            acc3 = __fmaf_rn(s1, exact_i2f(d[3]), acc3);
            if (a.acc) {
                const int g = g0 + u;
                if (va && vc0) a.acc[((size_t)ta * a.n + nc) * G + g] = d[0];
                if (va && vc1) a.acc[((size_t)ta * a.n + nc + 1) * G + g] = d[1];
                if (vb && vc0) a.acc[((size_t)tb * a.n + nc) * G + g] = d[2];
                if (vb && vc1) a.acc[((size_t)tb * a.n + nc + 1) * G + g] = d[3];
            }
        }
    }
    auto store = [&](int t, int n, float v) {
        size_t o = (size_t)t * a.ldy + n;
        y[o] = a.residual ? __fadd_rn(a.residual[o], v) : v;
    };
    if (va && vc0) store(ta, nc, __fmul_rn(acc0, sa_a));
    if (va && vc1) store(ta, nc + 1, __fmul_rn(acc1, sa_a));
    if (vb && vc0) store(tb, nc, __fmul_rn(acc2, sa_b));
    if (vb && vc1) store(tb, nc + 1, __fmul_rn(acc3, sa_b));
}

int launch_gemv_i8g32(const MatmulArgs &a, cudaStream_t stream) {
    const int tiles = (a.n + 7) / 8;
    dim3 grid((tiles + kGemvWarps - 1) / kGemvWarps, (a.m + 15) / 16, a.batch);
    if (grid.y > 65535 || grid.z > 65535) return set_error(NDL_ERR_INVALID_ARG, "gemv grid too large");
    gemv_i8g32_kernel<<<grid, kGemvWarps * 32, 0, stream>>>(a);
    return check_launch("gemv_i8g32");
}

}  // namespace ndl
