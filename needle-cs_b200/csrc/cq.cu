// CQ weights, the reference's own quantized format (Needle 3 `.cact`
// records): each weight row holds 2- or 4-bit codebook indices in groups of
// 128 columns with one fp16 norm per (row, group); a 16-entry codebook maps
// an index to a byte level (Codebook.Fill, src/Needle/Model.cs:36-52).
//
// Prepare (Quant.PrepareRange scalar branch, src/Needle/Quant.cs:471-484;
// Scalar.Hadamard / QuantizeInt8 / Planes, src/Needle/Scalar.cs:66-111):
// per (token, 128-group) a fast Walsh-Hadamard transform scaled by 1/sqrt(128),
// int8 quantization with one scale per group, the plane reorder that lines
// the activations up with the packed indices, and offset = 63 * sum(q).
//
// MatMulRows (Scalar.MatMulRows, src/Needle/Scalar.cs:146-192): per (token,
// row) and ascending group g, the exact int32 dot of the codebook bytes with
// the prepared activations, then in fp32 without contraction
//   scaled = (norm[g] * byte_scale) * scale[t][g]
//   acc += scaled * dot;  bias += scaled * offset[t][g];   y = acc - bias.
#include "common.cuh"
#include "cq.cuh"
#include "kernels.cuh"

namespace ndl {

constexpr int kCqMaxTokens = 16;                          // tokens per matmul launch (lane t folds token t)
constexpr int kCqWarps = 8;
constexpr int kCqMaxCols = 8192;
constexpr int kCqSplitMaxWarps = 8;   // warps per CTA of cq_matmul_split_kernel at most
constexpr int kCqSplitMaxBlocks = 8;  // 8-token blocks per CTA of cq_matmul_split_kernel at most
constexpr int kCqMaxJobs = 4;     // matrices per cq_matmul_split_kernel launch

// Scalar.Hadamard's butterflies (src/Needle/Scalar.cs:76-89) on a warp's
// 128 values, lane l holding elements l, l+32, l+64, l+96: strides 1, 2, ...,
// 64 in that order, lower index a + b, upper a - b; strides below 32 across
// lanes.  The 1/sqrt(128) scale is left to the caller.
__device__ __forceinline__ void cq_fwht128(float (&v)[4], int lane) {
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const bool upper = (lane & s) != 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[k], s);
            v[k] = upper ? __fsub_rn(o, v[k]) : __fadd_rn(v[k], o);
        }
    }
    {  // stride 32: elements (l, l+32) and (l+64, l+96)
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
    {  // stride 64: elements (l, l+64) and (l+32, l+96)
        const float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
}

// Warp per (token, group); lane l holds elements l, l+32, l+64, l+96.
__global__ void __launch_bounds__(256) cq_prepare_kernel(const float *__restrict__ x, int tokens, int cols, int bits,
                                                         int8_t *__restrict__ values, float *__restrict__ scales,
                                                         float *__restrict__ offsets, int stride) {
    pdl_enter();
    const int groups = cols / 128;
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (long long)tokens * groups) return;
    const int t = (int)(gw / groups), g = (int)(gw - (long long)t * groups);
    const float *src = x + (size_t)t * cols + (size_t)g * 128;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = src[lane + 32 * k];
    cq_fwht128(v, lane);
    float peak = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        v[k] = __fmul_rn(v[k], kCqHadamardScale);
        peak = fmaxf(peak, fabsf(v[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    int8_t *dst = values + ((size_t)t * groups + g) * 128;
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int8_t q = cq_quant1(v[k], inverse);
        const int e = lane + 32 * k;
        dst[cq_plane_at(e, bits)] = q;
        sum += q;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        scales[(size_t)t * stride + g] = scale;
        offsets[(size_t)t * stride + g] = __fmul_rn(63.0f, (float)sum);
    }
}

struct CqBook {
    uint32_t bytes[4];  // Codebook.Bytes[0..15], little-endian words
    float byte_scale;
};

__device__ __forceinline__ uint32_t cq_prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// 0xFF in every byte of w whose bit `bit` (0..7) is set: the bit moves to the
// byte's sign position and prmt's sign-replicate mode spreads it.
template <int kBit>
__device__ __forceinline__ uint32_t cq_bytemask(uint32_t w) {
    return cq_prmt(w << (7 - kBit), 0u, 0xBA98u);
}
// prmt selector with the low (kHigh = 0) or high nibble of w's byte k in
// nibble k.
template <int kHigh>
__device__ __forceinline__ uint32_t cq_nibble_sel(uint32_t w) {
    const uint32_t u = (kHigh ? w >> 4 : w) & 0x0F0F0F0Fu;  // nibble of byte k at bits 8k..8k+3
    return cq_prmt(u | (u >> 4), 0u, 0x0020u);            // bytes 0 and 2 hold nibbles (0, 1) and (2, 3)
}
// The codebook bytes of a word's sixteen 2-bit indices (index m at bits
// 2m..2m+1: byte m >> 2, plane m & 3) in four permutes, o[k] for MMA k:
// o[0] = indices 0, 2, 4, 6; o[1] = 1, 3, 5, 7; o[2] = 8, 10, 12, 14;
// o[3] = 9, 11, 13, 15.  A prmt selector nibble (bits 4n..4n+3 of the
// shifted word) holds two indices; with the top bit cleared its low three
// bits pick a byte of (t0, t0), the 4-entry book twice, so the nibble's
// second index drops out.  Eleven integer operations for 16 indices.
__device__ __forceinline__ void cq_decode2(uint32_t w, uint32_t t0, uint32_t (&o)[4]) {
    o[0] = cq_prmt(t0, t0, w & 0x7777u);
    o[1] = cq_prmt(t0, t0, (w >> 2) & 0x7777u);
    o[2] = cq_prmt(t0, t0, (w >> 16) & 0x7777u);
    o[3] = cq_prmt(t0, t0, (w >> 18) & 0x7777u);
}

// Codebook bytes for the four 4-bit indices in the low (kS = 0) or high
// (kS = 1) nibbles of w's bytes: the nibbles gathered into a prmt selector,
// two 8-entry permutes and a select on the index's top bit.
template <int kS>
__device__ __forceinline__ uint32_t cq_lut4(uint32_t w, const uint32_t (&t)[4]) {
    const uint32_t sel = cq_nibble_sel<kS>(w) & 0x7777u;  // index k in nibble k, top bit cleared
    const uint32_t lo = cq_prmt(t[0], t[1], sel), hi = cq_prmt(t[2], t[3], sel);
    const uint32_t m = cq_bytemask<kS ? 7 : 3>(w);  // bytes whose index is >= 8
    return (hi & m) | (lo & ~m);
}

__device__ __forceinline__ uint32_t cq_lut_plane4(uint32_t w, int s, const uint32_t (&t)[4]) {
    return s == 0 ? cq_lut4<0>(w, t) : cq_lut4<1>(w, t);
}

__device__ __forceinline__ void cq_mma(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Warp per tile of 16 weight rows (grid-stride), up to 16 tokens as two
// 8-token MMA columns.  Per 128-column group and 32-column chunk k of it, the
// codebook bytes of the chunk's indices become the A fragment of one
// mma.sync m16n8k32 s8 (byte permutes in registers), the prepared
// activations the B fragment (shared memory, rows padded by 16 bytes so the
// fragment loads hit 32 distinct banks); the four chunks chain in the
// accumulator to the exact group dot.  4-bit: chunk k of a group is nibble
// k&1 of bytes 32(k>>1)..+31, the plane order Prepare writes; 2-bit: the
// decode's own order (cq_decode2), the activations permuted to match when
// they are staged.  Each lane then folds
// its four (row, token) dots per column block into fp32 in ascending group
// order.
template <int kBits>
__global__ void __launch_bounds__(32 * kCqWarps, 2) cq_matmul_kernel(
    const uint32_t *__restrict__ indices, const uint16_t *__restrict__ norms, CqBook book, int cols,
    const int8_t *__restrict__ values, const float *__restrict__ scales, const float *__restrict__ offsets,
    int stride, int tokens, float *__restrict__ y, int ldy, int row_start, int row_end) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int groups = cols / 128, row_words = cols * kBits / 32, xstride = cols + 16;
    constexpr int kGroupWords = kBits == 2 ? 8 : 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    uint8_t *xs = smem;                                                              // [16][cols + 16]
    float *ss = reinterpret_cast<float *>(smem + (size_t)kCqMaxTokens * xstride);    // [16][groups]
    float *os = ss + kCqMaxTokens * groups;
    pdl_enter();
    if (kBits == 2) {
        // the activations in the order the 2-bit decode produces codes (see cq_decode2): slot s of MMA k in
        // a group holds plane p(k, i) of byte 16 * half + 4 * tig + b(k, i), with s = 16 * half + 4 * tig + i,
        // b = 2 (k >> 1) + (i >> 1), p = (k & 1) + 2 (i & 1); the group dot is an exact int32 sum in any order
        for (int i = threadIdx.x; i < kCqMaxTokens * (cols / 4); i += blockDim.x) {
            const int t = i / (cols / 4), ow = i - t * (cols / 4), g = ow >> 5, s0 = 4 * (ow & 31);
            const int k = s0 >> 5, half = (s0 >> 4) & 1, tg = (s0 >> 2) & 3;
            uint32_t out = 0u;
            if (t < tokens) {
                const int8_t *src = values + (size_t)t * cols + (size_t)g * 128 + half * 16 + tg * 4;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int b = 2 * (k >> 1) + (j >> 1), p = (k & 1) + 2 * (j & 1);
                    out |= (uint32_t)(uint8_t)src[p * 32 + b] << (8 * j);
                }
            }
            *reinterpret_cast<uint32_t *>(xs + (size_t)t * xstride + 4 * ow) = out;
        }
    } else {
        for (int i = threadIdx.x; i < kCqMaxTokens * (cols / 16); i += blockDim.x) {
            const int t = i / (cols / 16), c = i - t * (cols / 16);
            const uint4 v = t < tokens ? reinterpret_cast<const uint4 *>(values + (size_t)t * cols)[c]
                                       : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4 *>(xs + (size_t)t * xstride + 16 * c) = v;
        }
    }
    for (int i = threadIdx.x; i < kCqMaxTokens * groups; i += blockDim.x) {
        const int t = i / groups, g = i - t * groups;
        ss[i] = t < tokens ? scales[(size_t)t * stride + g] : 0.0f;
        os[i] = t < tokens ? offsets[(size_t)t * stride + g] : 0.0f;
    }
    __syncthreads();
    const int n_tiles = (row_end - row_start + 15) / 16;
    const int warps = gridDim.x * kCqWarps;
    // two tiles per warp pass, their index words loaded a chunk of groups at a
    // time before any is used, so each warp keeps 2 x kChunk group tiles of
    // loads in flight
    constexpr int kTiles = 2, kChunk = kBits == 2 ? 4 : 2, kBlocks = kBits == 2 ? 1 : 2;
    for (int pair = blockIdx.x * kCqWarps + warp; pair * kTiles < n_tiles; pair += warps) {
        int r0[kTiles], r1[kTiles];
        bool ok0[kTiles], ok1[kTiles];
        const uint32_t *w0[kTiles], *w1[kTiles];
#pragma unroll
        for (int tt = 0; tt < kTiles; tt++) {
            r0[tt] = row_start + (pair * kTiles + tt) * 16 + gid;
            r1[tt] = r0[tt] + 8;
            ok0[tt] = r0[tt] < row_end;
            ok1[tt] = r1[tt] < row_end;
            w0[tt] = indices + (size_t)(ok0[tt] ? r0[tt] : row_start) * row_words;
            w1[tt] = indices + (size_t)(ok1[tt] ? r1[tt] : row_start) * row_words;
        }
        float acc[kTiles][2][4], bias[kTiles][2][4];
#pragma unroll
        for (int tt = 0; tt < kTiles; tt++)
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[tt][nt][i] = 0.0f, bias[tt][nt][i] = 0.0f;
        for (int g0 = 0; g0 < groups; g0 += kChunk) {
            // this lane's index words: rows r0, r1; word tig and 4 + tig of each 32-byte block
            uint32_t c0[kTiles][kChunk][kBlocks][2], c1[kTiles][kChunk][kBlocks][2];
            uint16_t n0[kTiles][kChunk], n1[kTiles][kChunk];
#pragma unroll
            for (int tt = 0; tt < kTiles; tt++)
#pragma unroll
                for (int cg = 0; cg < kChunk; cg++) {
                    const int g = g0 + cg;
                    const bool in = g < groups;
#pragma unroll
                    for (int h = 0; h < kBlocks; h++) {
                        const int wi = g * kGroupWords + 8 * h + tig;
                        c0[tt][cg][h][0] = in && ok0[tt] ? __ldg(w0[tt] + wi) : 0u;
                        c0[tt][cg][h][1] = in && ok0[tt] ? __ldg(w0[tt] + wi + 4) : 0u;
                        c1[tt][cg][h][0] = in && ok1[tt] ? __ldg(w1[tt] + wi) : 0u;
                        c1[tt][cg][h][1] = in && ok1[tt] ? __ldg(w1[tt] + wi + 4) : 0u;
                    }
                    n0[tt][cg] = in && ok0[tt] ? norms[(size_t)r0[tt] * groups + g] : (uint16_t)0;
                    n1[tt][cg] = in && ok1[tt] ? norms[(size_t)r1[tt] * groups + g] : (uint16_t)0;
                }
#pragma unroll
            for (int cg = 0; cg < kChunk; cg++) {
                const int g = g0 + cg;
                if (g >= groups) break;
#pragma unroll
                for (int tt = 0; tt < kTiles; tt++) {
                    const float nf0 = __fmul_rn(half_to_float_ref(n0[tt][cg]), book.byte_scale);
                    const float nf1 = __fmul_rn(half_to_float_ref(n1[tt][cg]), book.byte_scale);
                    int d[2][4];
#pragma unroll
                    for (int nt = 0; nt < 2; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) d[nt][i] = 0;
                    // 2-bit: the codebook bytes of the four index words (a0..a3 order), four MMAs' worth each
                    uint32_t dec[4][4];
                    if (kBits == 2) {
                        const uint32_t wds[4] = {c0[tt][cg][0][0], c1[tt][cg][0][0], c0[tt][cg][0][1], c1[tt][cg][0][1]};
#pragma unroll
                        for (int j = 0; j < 4; j++) cq_decode2(wds[j], book.bytes[0], dec[j]);
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int h = kBits == 2 ? 0 : k >> 1;
                        uint32_t a[4];
                        if (kBits == 2) {
                            a[0] = dec[0][k];
                            a[1] = dec[1][k];
                            a[2] = dec[2][k];
                            a[3] = dec[3][k];
                        } else {
                            a[0] = cq_lut_plane4(c0[tt][cg][h][0], k & 1, book.bytes);
                            a[1] = cq_lut_plane4(c1[tt][cg][h][0], k & 1, book.bytes);
                            a[2] = cq_lut_plane4(c0[tt][cg][h][1], k & 1, book.bytes);
                            a[3] = cq_lut_plane4(c1[tt][cg][h][1], k & 1, book.bytes);
                        }
#pragma unroll
                        for (int nt = 0; nt < 2; nt++) {
                            if (nt == 1 && tokens <= 8) break;  // one 8-token column block suffices
                            const uint8_t *xb = xs + (size_t)(nt * 8 + gid) * xstride + g * 128 + 32 * k + 4 * tig;
                            cq_mma(d[nt], a, *reinterpret_cast<const uint32_t *>(xb),
                                   *reinterpret_cast<const uint32_t *>(xb + 16));
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < 2; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            if (nt == 1 && tokens <= 8) break;
                            const int t = nt * 8 + 2 * tig + (i & 1);
                            const float scaled = __fmul_rn(i < 2 ? nf0 : nf1, ss[t * groups + g]);
                            acc[tt][nt][i] = __fadd_rn(acc[tt][nt][i], __fmul_rn(scaled, (float)d[nt][i]));
                            bias[tt][nt][i] = __fadd_rn(bias[tt][nt][i], __fmul_rn(scaled, os[t * groups + g]));
                        }
                }
            }
        }
#pragma unroll
        for (int tt = 0; tt < kTiles; tt++)
#pragma unroll
            for (int nt = 0; nt < 2; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int t = nt * 8 + 2 * tig + (i & 1);
                    const bool ok = i < 2 ? ok0[tt] : ok1[tt];
                    if (ok && t < tokens)
                        y[(size_t)t * ldy + (i < 2 ? r0[tt] : r1[tt])] = __fsub_rn(acc[tt][nt][i], bias[tt][nt][i]);
                }
    }
}

// Up to kCqMaxJobs matrices over the same prepared activations in one launch
// (the projections of one layer); jobs in ascending tile_begin order.
struct CqJob {
    const uint32_t *indices;
    const uint16_t *norms;
    float *y;
    CqBook book;
    int ldy, row_start, row_end, tile_begin;
};
struct CqJobList {
    CqJob job[kCqMaxJobs];
    int n;
};

// The same MatMulRows for many tokens or few rows.  A CTA takes one 16-row
// tile of one job and up to eight 8-token blocks; its warps are `split`
// group phases times `wb` block phases: warp (p, q) takes groups p, p +
// split, ... and, for each, blocks q, q + wb, ...  Per group the codebook
// bytes are decoded into A fragments once (as in cq_matmul_kernel) and used
// for every block the warp takes; per block the B fragments are loaded
// straight from the prepared values (each lane's eight words g*128 + 4*tig +
// 16*j of its token; for 2-bit the plane permutation of cq_matmul_kernel's
// staging done with byte permutes), four mma.sync give the exact int32 dots,
// which go to shared memory with the rows' norm * byte_scale and the tokens'
// scales and offsets.  Then each (row, token) is folded over the groups in
// ascending order with the same fp32 steps as cq_matmul_kernel
// (Scalar.MatMulRows, src/Needle/Scalar.cs:146-192).
template <int kBits>
__global__ void __launch_bounds__(32 * kCqSplitMaxWarps) cq_matmul_split_kernel(
    CqJobList jobs, int cols, const int8_t *__restrict__ values, const float *__restrict__ scales,
    const float *__restrict__ offsets, int stride, int tokens, int split, int tbs) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int groups = cols / 128, row_words = cols * kBits / 32;
    constexpr int kGroupWords = kBits == 2 ? 8 : 16;
    constexpr int kBlocks = kBits == 2 ? 1 : 2;
    const int wb = (int)(blockDim.x >> 5) / split, token_blocks = (tokens + 7) >> 3;
    const int ctas_per_tile = (token_blocks + tbs - 1) / tbs;
    const int tile = blockIdx.x / ctas_per_tile, tb0 = (blockIdx.x - tile * ctas_per_tile) * tbs;
    CqJob job = jobs.job[0];
#pragma unroll
    for (int i = 1; i < kCqMaxJobs; i++)
        if (i < jobs.n && tile >= jobs.job[i].tile_begin) job = jobs.job[i];
    const int r_base = job.row_start + (tile - job.tile_begin) * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const int bq = warp / split, phase = warp - bq * split;
    int *dots = reinterpret_cast<int *>(smem);                         // [tbs][groups][16 rows][8 tokens]
    float *nf = reinterpret_cast<float *>(dots + tbs * groups * 128);  // [groups][16]
    float *ss = nf + groups * 16;                                      // [tbs][groups][8]
    float *os = ss + tbs * groups * 8;                                 // [tbs][groups][8]
    const int r0 = r_base + gid, r1 = r0 + 8;
    const bool ok0 = r0 < job.row_end, ok1 = r1 < job.row_end;
    const uint32_t *w0 = job.indices + (size_t)(ok0 ? r0 : job.row_start) * row_words;
    const uint32_t *w1 = job.indices + (size_t)(ok1 ? r1 : job.row_start) * row_words;
    // side values per lane: lanes 0..15 a row's norm * byte_scale (block phase 0
    // writes them), 16..23 a token's scale, 24..31 its offset
    const int side_row = r_base + (lane & 15);
    const float *side_src = lane < 24 ? scales : offsets;
    pdl_enter();
    for (int g = phase; g < groups; g += split) {
        uint32_t c0[kBlocks][2], c1[kBlocks][2];
#pragma unroll
        for (int h = 0; h < kBlocks; h++) {
            const int wi = g * kGroupWords + 8 * h + tig;
            c0[h][0] = ok0 ? __ldg(w0 + wi) : 0u;
            c0[h][1] = ok0 ? __ldg(w0 + wi + 4) : 0u;
            c1[h][0] = ok1 ? __ldg(w1 + wi) : 0u;
            c1[h][1] = ok1 ? __ldg(w1 + wi + 4) : 0u;
        }
        if (lane < 16 && bq == 0)
            nf[g * 16 + lane] = side_row < job.row_end
                                    ? __fmul_rn(half_to_float_ref_fast(job.norms[(size_t)side_row * groups + g]),
                                                job.book.byte_scale)
                                    : 0.0f;
        uint32_t a[4][4];  // A fragments of MMA k
        if (kBits == 2) {
            const uint32_t wds[4] = {c0[0][0], c1[0][0], c0[0][1], c1[0][1]};
            uint32_t dec[4][4];
#pragma unroll
            for (int j = 0; j < 4; j++) cq_decode2(wds[j], job.book.bytes[0], dec[j]);
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int j = 0; j < 4; j++) a[k][j] = dec[j][k];
        } else {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int h = k >> 1;
                a[k][0] = cq_lut_plane4(c0[h][0], k & 1, job.book.bytes);
                a[k][1] = cq_lut_plane4(c1[h][0], k & 1, job.book.bytes);
                a[k][2] = cq_lut_plane4(c0[h][1], k & 1, job.book.bytes);
                a[k][3] = cq_lut_plane4(c1[h][1], k & 1, job.book.bytes);
            }
        }
#pragma unroll 2
        for (int b = bq; b < tbs; b += wb) {
            const int t = (tb0 + b) * 8 + gid;
            const bool okt = t < tokens;
            const uint32_t *xw = reinterpret_cast<const uint32_t *>(values + (size_t)(okt ? t : 0) * cols) + g * 32 + tig;
            uint32_t x[8];
#pragma unroll
            for (int j = 0; j < 8; j++) x[j] = okt ? __ldg(xw + 4 * j) : 0u;
            if (lane >= 16) {
                const int side_tok = (tb0 + b) * 8 + (lane & 7);
                (lane < 24 ? ss : os)[((size_t)b * groups + g) * 8 + (lane & 7)] =
                    side_tok < tokens ? side_src[(size_t)side_tok * stride + g] : 0.0f;
            }
            int d[4] = {0, 0, 0, 0};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (kBits == 2) {
                    // byte i of half h of MMA k: plane (k & 1) + 2 (i & 1) of byte 2 (k >> 1) + (i >> 1), i.e.
                    // word h + 2 (k & 1) (even i) or h + 2 (k & 1) + 4 (odd i) of this lane's eight
                    const uint32_t sel = (k >> 1) ? 0x7362u : 0x5140u;
                    const int p = 2 * (k & 1);
                    cq_mma(d, a[k], cq_prmt(x[p], x[p + 4], sel), cq_prmt(x[p + 1], x[p + 5], sel));
                } else {
                    cq_mma(d, a[k], x[2 * k], x[2 * k + 1]);
                }
            }
            // rows gid, gid + 8; tokens 2 tig, 2 tig + 1
            int *bd = dots + ((size_t)b * groups + g) * 128;
            *reinterpret_cast<int2 *>(bd + gid * 8 + 2 * tig) = make_int2(d[0], d[1]);
            *reinterpret_cast<int2 *>(bd + (gid + 8) * 8 + 2 * tig) = make_int2(d[2], d[3]);
        }
    }
    __syncthreads();
    for (int q = threadIdx.x; q < tbs * 128; q += blockDim.x) {
        const int b = q >> 7, r = (q >> 3) & 15, tk = q & 7;
        const int *bd = dots + (size_t)b * groups * 128 + r * 8 + tk;
        const float *bs = ss + (size_t)b * groups * 8 + tk, *bo = os + (size_t)b * groups * 8 + tk;
        float acc = 0.0f, bias = 0.0f;
        for (int g = 0; g < groups; g++) {
            const float scaled = __fmul_rn(nf[g * 16 + r], bs[g * 8]);
            acc = __fadd_rn(acc, __fmul_rn(scaled, (float)bd[g * 128]));
            bias = __fadd_rn(bias, __fmul_rn(scaled, bo[g * 8]));
        }
        const int row = r_base + r, tok = (tb0 + b) * 8 + tk;
        if (row < job.row_end && tok < tokens) job.y[(size_t)tok * job.ldy + row] = __fsub_rn(acc, bias);
    }
}

// Quant.GatherRow (src/Needle/Quant.cs:566-576): a CQ row decoded to floats
// (Scalar.DecodeRow, src/Needle/Scalar.cs:130-144: levels[index] * norm in
// natural column order) and rotated back per 128-column group
// (Scalar.Hadamard).  Warp per (output row, group); out[r] = row rows[r].
struct CqLevels {
    float v[16];
};
__global__ void __launch_bounds__(256) cq_gather_kernel(const uint8_t *__restrict__ indices,
                                                        const uint16_t *__restrict__ norms, CqLevels levels, int rows,
                                                        int cols, int bits, const int32_t *__restrict__ row_ids, int n,
                                                        float *__restrict__ out, int *status) {
    pdl_enter();
    const int groups = cols / 128;
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (long long)n * groups) return;
    const int r = (int)(gw / groups), g = (int)(gw - (long long)r * groups);
    const int row = row_ids[r];
    float *dst = out + (size_t)r * cols + (size_t)g * 128;
    if (row < 0 || row >= rows) {  // checked on the host for the C entry points; zeros and a status bit here
        for (int k = 0; k < 4; k++) dst[lane + 32 * k] = 0.0f;
        if (lane == 0 && status) atomicOr(status, 2);
        return;
    }
    const size_t row_bytes = (size_t)cols * bits / 8;
    const uint8_t *packed = indices + (size_t)row * row_bytes + (size_t)g * (bits == 2 ? 32 : 64);
    const float norm = half_to_float_ref(norms[(size_t)row * groups + g]);
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int e = lane + 32 * k;
        const int code = bits == 2 ? (packed[e >> 2] >> ((e & 3) * 2)) & 3 : (packed[e >> 1] >> ((e & 1) * 4)) & 15;
        v[k] = __fmul_rn(levels.v[code], norm);
    }
    cq_fwht128(v, lane);
#pragma unroll
    for (int k = 0; k < 4; k++) dst[lane + 32 * k] = __fmul_rn(v[k], kCqHadamardScale);
}

int launch_cq_gather(const uint8_t *indices, const uint16_t *norms, const float *levels16, int rows, int cols, int bits,
                     const int32_t *row_ids, int n, float *out, int *status, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    CqLevels lv;
    memcpy(lv.v, levels16, sizeof(lv.v));
    const long long warps = (long long)n * (cols / 128);
    launch_kernel(cq_gather_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, stream, indices, norms, lv, rows,
                  cols, bits, row_ids, n, out, status);
    return check_launch("cq_gather");
}

int launch_cq_prepare(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales, float *offsets,
                      int stride, cudaStream_t stream) {
    if (tokens == 0) return NDL_OK;
    const long long warps = (long long)tokens * (cols / 128);
    launch_kernel(cq_prepare_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, stream, x, tokens, cols, bits,
                  values, scales, offsets, stride);
    return check_launch("cq_prepare");
}

int launch_cq_matmul_jobs(const CqMatmulJob *jobs, int n_jobs, int cols, int bits, const int8_t *values,
                          const float *scales, const float *offsets, int stride, int tokens, cudaStream_t stream) {
    if (tokens == 0) return NDL_OK;
    const int groups = cols / 128, token_blocks = (tokens + 7) / 8, sms = device_sm_count();
    // a warp per group phase (up to kCqSplitMaxWarps), the rest as block phases
    const int split = groups < kCqSplitMaxWarps ? groups : kCqSplitMaxWarps;
    // token blocks per CTA: within 48 KB of shared memory and kCqSplitMaxBlocks
    int cap = (12288 - 16 * groups) / (144 * groups);
    cap = cap < kCqSplitMaxBlocks ? cap : kCqSplitMaxBlocks;
    cap = cap < token_blocks ? cap : token_blocks;
    int next = 0;
    while (next < n_jobs) {
        CqJobList list{};
        long long tiles = 0;
        for (; next < n_jobs && list.n < kCqMaxJobs; next++) {
            const CqMatmulJob &s = jobs[next];
            if (s.row_end <= s.row_start) continue;
            CqJob &d = list.job[list.n++];
            d.indices = reinterpret_cast<const uint32_t *>(s.indices);
            d.norms = s.norms;
            d.y = s.y;
            memcpy(d.book.bytes, s.book_bytes, 16);
            d.book.byte_scale = s.byte_scale;
            d.ldy = s.ldy;
            d.row_start = s.row_start;
            d.row_end = s.row_end;
            d.tile_begin = (int)tiles;
            tiles += (s.row_end - s.row_start + 15) / 16;
        }
        if (list.n == 0) break;
        // fewer blocks per CTA (more CTAs, each block's decode repeated) while
        // the grid would not give every SM two CTAs
        int tbs = cap;
        while (tbs > 1 && tiles * ((token_blocks + tbs - 1) / tbs) < 2LL * sms) tbs--;
        const int wb = kCqSplitMaxWarps / split < tbs ? kCqSplitMaxWarps / split : tbs;
        const long long blocks = tiles * ((token_blocks + tbs - 1) / tbs);
        if (blocks > 0x7fffffffLL) return set_error(NDL_ERR_INVALID_ARG, "cq matmul: %lld CTAs", blocks);
        const size_t smem = ((size_t)tbs * groups * (128 + 16) + (size_t)groups * 16) * 4;  // dots, scales, offsets, norms
        if (bits == 2)
            launch_kernel(cq_matmul_split_kernel<2>, dim3((unsigned)blocks), dim3(32 * split * wb), smem, stream,
                          list, cols, values, scales, offsets, stride, tokens, split, tbs);
        else
            launch_kernel(cq_matmul_split_kernel<4>, dim3((unsigned)blocks), dim3(32 * split * wb), smem, stream,
                          list, cols, values, scales, offsets, stride, tokens, split, tbs);
        const int st = check_launch("cq_matmul_split");
        if (st != NDL_OK) return st;
    }
    return NDL_OK;
}

size_t cq_matmul_smem(int cols) {
    return (size_t)kCqMaxTokens * (cols + 16) + (size_t)2 * kCqMaxTokens * (cols / 128) * 4;
}

int launch_cq_matmul(const uint8_t *indices, const uint16_t *norms, const uint8_t *book_bytes, float byte_scale,
                     int cols, int bits, const int8_t *values, const float *scales, const float *offsets, int stride,
                     int tokens, float *y, int ldy, int row_start, int row_end, cudaStream_t stream) {
    if (tokens == 0 || row_end <= row_start) return NDL_OK;
    static DeviceOnce smem_attribute;
    int st0 = smem_attribute.run([] {
        const int max_smem = (int)cq_matmul_smem(kCqMaxCols);
        cudaError_t e = cudaFuncSetAttribute(cq_matmul_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(cq_matmul_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "cq matmul smem attribute: %s", cudaGetErrorString(e));
        return (int)NDL_OK;
    });
    if (st0 != NDL_OK) return st0;
    const int sms = device_sm_count();
    if (tokens > kCqMaxTokens || (row_end - row_start + 15) / 16 < 8 * sms) {
        // many tokens, or too few tiles for warp-per-tile: split the groups
        const CqMatmulJob job{indices, norms, book_bytes, byte_scale, y, ldy, row_start, row_end};
        return launch_cq_matmul_jobs(&job, 1, cols, bits, values, scales, offsets, stride, tokens, stream);
    }
    CqBook book;
    memcpy(book.bytes, book_bytes, 16);
    book.byte_scale = byte_scale;
    const int rows = row_end - row_start;
    for (int t0 = 0; t0 < tokens; t0 += kCqMaxTokens) {  // token chunks; each launch reads the rows once
        const int tk = tokens - t0 < kCqMaxTokens ? tokens - t0 : kCqMaxTokens;
        const size_t smem = cq_matmul_smem(cols);
        long long blocks = ((rows + 31) / 32 + kCqWarps - 1) / kCqWarps;  // two 16-row tiles per warp
        int per_sm = 1;  // resident CTAs per SM at this shared-memory size
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bits == 2 ? cq_matmul_kernel<2> : cq_matmul_kernel<4>,
                                                      32 * kCqWarps, smem);
        const long long cap = (long long)sms * (per_sm > 0 ? per_sm : 1);
        if (blocks > cap) blocks = cap;
        const int8_t *v = values + (size_t)t0 * cols;
        const float *sc = scales + (size_t)t0 * stride, *of = offsets + (size_t)t0 * stride;
        float *yt = y + (size_t)t0 * ldy;
        if (bits == 2)
            launch_kernel(cq_matmul_kernel<2>, dim3((unsigned)blocks), dim3(32 * kCqWarps), smem, stream,
                          reinterpret_cast<const uint32_t *>(indices), norms, book, cols, v, sc, of, stride, tk, yt,
                          ldy, row_start, row_end);
        else
            launch_kernel(cq_matmul_kernel<4>, dim3((unsigned)blocks), dim3(32 * kCqWarps), smem, stream,
                          reinterpret_cast<const uint32_t *>(indices), norms, book, cols, v, sc, of, stride, tk, yt,
                          ldy, row_start, row_end);
        const int st = check_launch("cq_matmul");
        if (st != NDL_OK) return st;
    }
    return NDL_OK;
}

}  // namespace ndl

using namespace ndl;

extern "C" NDL_API int ndl_cq_prepare(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales,
                                      float *offsets, int stride, void *stream) {
    NDL_REQUIRE(tokens >= 0 && cols >= 128 && cols % 128 == 0 && cols <= kCqMaxCols, "cols %d (a multiple of 128 up to %d)",
                cols, kCqMaxCols);
    NDL_REQUIRE(bits == 2 || bits == 4, "bits %d (2 or 4)", bits);
    NDL_REQUIRE(stride >= cols / 128, "stride %d below %d groups", stride, cols / 128);
    if (tokens == 0) return NDL_OK;
    NDL_REQUIRE(x && values && scales && offsets, "null pointer");
    return launch_cq_prepare(x, tokens, cols, bits, values, scales, offsets, stride, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_cq_matmul(const uint8_t *indices, const uint16_t *norms, const uint8_t *book_bytes,
                                     float byte_scale, int rows, int cols, int bits, const int8_t *values,
                                     const float *scales, const float *offsets, int stride, int tokens, float *y,
                                     int ldy, int row_start, int row_end, void *stream) {
    NDL_REQUIRE(cols >= 128 && cols % 128 == 0 && cols <= kCqMaxCols, "cols %d (a multiple of 128 up to %d)", cols,
                kCqMaxCols);
    NDL_REQUIRE(bits == 2 || bits == 4, "bits %d (2 or 4)", bits);
    NDL_REQUIRE(0 <= row_start && row_start <= row_end && row_end <= rows, "rows [%d, %d) outside 0..%d", row_start,
                row_end, rows);
    NDL_REQUIRE(tokens >= 0 && stride >= cols / 128 && ldy >= row_end, "tokens %d / stride %d / ldy %d", tokens,
                stride, ldy);
    if (tokens == 0 || row_start == row_end) return NDL_OK;
    NDL_REQUIRE(indices && norms && book_bytes && values && scales && offsets && y, "null pointer");
    NDL_REQUIRE(aligned(indices, 4) && aligned(values, 16), "indices need 4-byte, values 16-byte alignment");
    return launch_cq_matmul(indices, norms, book_bytes, byte_scale, cols, bits, values, scales, offsets, stride, tokens,
                            y, ldy, row_start, row_end, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_cq_gather_rows(const uint8_t *indices, const uint16_t *norms, const float *levels, int rows,
                                          int cols, int bits, const int32_t *row_ids, int n, float *out, void *stream) {
    NDL_REQUIRE(cols >= 128 && cols % 128 == 0 && rows >= 1 && n >= 0, "rows %d / cols %d / n %d", rows, cols, n);
    NDL_REQUIRE(bits == 2 || bits == 4, "bits %d (2 or 4)", bits);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(indices && norms && levels && row_ids && out, "null pointer");
    return launch_cq_gather(indices, norms, levels, rows, cols, bits, row_ids, n, out, nullptr, (cudaStream_t)stream);
}
