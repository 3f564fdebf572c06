// I8G32 streaming GEMV: y[t][n] = sum_g (half(sw[n][g]) * sa[t]) * D[t][n][g]
// with D the exact int32 dot over one 32-column group.
//
// Replaces Quant.MatMulRows -> Gemv.Rows/Block/Tile4/Tile2
// (src/Needle/Quant.cs:615-633, src/Needle/Gemv.cs:117-333) for the M < 64
// decode shapes.  Design:
//  * A CTA owns 8*R weight rows and one 16-row tile of activations.  Its
//    warps split the K/32 groups; each group of 8 rows is one
//    mma.sync.m16n8k32 (K = 32 = one group), so the int32 accumulator of an
//    MMA is exactly D for that group.  Weight bytes are read once, 8 bytes
//    per lane per group, with L1-bypassing loads.
//  * D goes to shared memory.  An epilogue pass then sums the groups of
//    each (t, n) in ascending order with round-to-nearest multiplies and
//    adds (no FMA), which reproduces the scalar definition bit for bit and
//    makes a row's result independent of the batch it is in.
//  * The MMA computes sum_k A[t][k] B[k][n] over a 32-wide k slice.  Any
//    permutation of k applied to both operands leaves that sum unchanged,
//    so each lane loads 8 contiguous bytes of its weight row (group bytes
//    8*tig .. 8*tig+7) and the same 8 bytes of its two activation rows; the
//    fragment registers are then b0 = bytes 0..3, b1 = bytes 4..7 and
//    a0/a2 (row gid), a1/a3 (row gid+8) likewise.
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

constexpr int kGemvWarps = 4;

template <int R>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_i8g32_kernel(MatmulArgs a) {
    extern __shared__ int32_t smem_d[];  // [G][16][8R+1]
    constexpr int NT = 8 * R;            // rows per CTA
    constexpr int S = NT + 1;            // padded row stride
    const int G = a.k >> 5;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int b = blockIdx.z;
    const int8_t *w = a.w + (long long)b * a.w_stride;
    const uint16_t *sw = a.sw + (long long)b * a.sw_stride;
    float *y = a.y + (long long)b * a.y_stride;
    const int n0 = blockIdx.x * NT;
    const int t0 = blockIdx.y * 16;
    const int ta = t0 + gid, tb = ta + 8;
    const bool va = ta < a.m, vb = tb < a.m;
    const int8_t *qa = a.q + (size_t)(va ? ta : 0) * a.k + 8 * tig;
    const int8_t *qb = a.q + (size_t)(vb ? tb : 0) * a.k + 8 * tig;
    const int8_t *wrow[R];
    bool vrow[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        int n = n0 + 8 * r + gid;
        vrow[r] = n < a.n;
        wrow[r] = w + (size_t)(vrow[r] ? n : 0) * a.k + 8 * tig;
    }

#pragma unroll 2
    for (int g = warp; g < G; g += kGemvWarps) {
        uint2 bw[R];
#pragma unroll
        for (int r = 0; r < R; r++) bw[r] = vrow[r] ? ld_stream_u2(wrow[r] + g * 32) : make_uint2(0u, 0u);
        uint2 A0 = va ? *reinterpret_cast<const uint2 *>(qa + g * 32) : make_uint2(0u, 0u);
        uint2 A1 = vb ? *reinterpret_cast<const uint2 *>(qb + g * 32) : make_uint2(0u, 0u);
        int32_t *dg = smem_d + (size_t)g * 16 * S;
#pragma unroll
        for (int r = 0; r < R; r++) {
            int d[4];
            mma_s8_16x8x32(d, A0.x, A1.x, A0.y, A1.y, bw[r].x, bw[r].y);
            int col = 8 * r + 2 * tig;
            dg[gid * S + col] = d[0];
            dg[gid * S + col + 1] = d[1];
            dg[(gid + 8) * S + col] = d[2];
            dg[(gid + 8) * S + col + 1] = d[3];
        }
    }
    __syncthreads();

    for (int p = threadIdx.x; p < 16 * NT; p += kGemvWarps * 32) {
        int tl = p / NT, nl = p - tl * NT;
        int t = t0 + tl, n = n0 + nl;
        if (t >= a.m || n >= a.n) continue;
        float s_a = a.sa[t];
        const uint16_t *swr = sw + (size_t)n * G;
        float accum = 0.0f;
        for (int g = 0; g < G; g++) {
            int d = smem_d[((size_t)g * 16 + tl) * S + nl];
            float scaled = __fmul_rn(half_to_float_ref(swr[g]), s_a);
            accum = __fadd_rn(accum, __fmul_rn(scaled, __int2float_rn(d)));
            if (a.acc) a.acc[((size_t)t * a.n + n) * G + g] = d;
        }
        size_t o = (size_t)t * a.ldy + n;
        y[o] = a.residual ? __fadd_rn(a.residual[o], accum) : accum;
    }
}

template <int R>
static int launch_r(const MatmulArgs &a, cudaStream_t stream) {
    const int G = a.k >> 5;
    size_t smem = (size_t)G * 16 * (8 * R + 1) * sizeof(int32_t);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(gemv_i8g32_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "gemv smem attribute: %s", cudaGetErrorString(e));
    }
    dim3 grid((a.n + 8 * R - 1) / (8 * R), (a.m + 15) / 16, a.batch);
    gemv_i8g32_kernel<R><<<grid, kGemvWarps * 32, smem, stream>>>(a);
    return check_launch("gemv_i8g32");
}

int launch_gemv_i8g32(const MatmulArgs &a, cudaStream_t stream) {
    const int G = a.k >> 5;
    if (G > 256) return set_error(NDL_ERR_UNSUPPORTED, "gemv: k=%d exceeds 8192", a.k);
    // Enough CTAs to cover the SMs, and at most ~64 group-rows of D in smem.
    long long ctas4 = (long long)((a.n + 31) / 32) * ((a.m + 15) / 16) * a.batch;
    if (G <= 16 && ctas4 >= 2 * 148) return launch_r<4>(a, stream);
    if (G <= 32 && ctas4 >= 148) return launch_r<2>(a, stream);
    return launch_r<1>(a, stream);
}

}  // namespace ndl
