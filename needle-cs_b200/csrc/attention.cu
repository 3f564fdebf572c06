// Paged int8 KV cache: the KV-write epilogue and split-K decode attention.
//
// KV write (src/Needle/Engine.cs:2552-2569): RoPE at the row's absolute
// position (half-split rotation, Scalar.Rope src/Needle/Scalar.cs:233-248),
// then QuantizeInt8 of q per head and of k, v per (position, head) into the
// slot's page.  Bit-exact: round-to-nearest products, no FMA.
//
// Decode attention (Scalar.AttentionHead src/Needle/Scalar.cs:290-312,
// AttentionBatch.ExecuteChunk + MergePartials src/Needle/Blocks.cs:750-990):
// one warp per (row, head, chunk of pages).  Each page's 8704-byte (layer,
// head) record arrives in shared memory by one cp.async.bulk (3-stage ring,
// mbarrier completion, bounded waits).  Scores are exact int8 dots scaled by
// ks * (qs / sqrt(d)); softmax is online (running max, rescaled sum) in fp32
// with expf; V is accumulated in fp32.  A row split into several chunks
// writes (peak, sum, unnormalised output) partials and the last chunk to
// finish merges them with exp(peak - max) weights, like MergePartials.
#include "common.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int8_t quant1(float x, float inverse) {
    float r = rintf(__fmul_rn(x, inverse));
    return (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
}

// Quantizes the 64-vector held as (lo = v[lane], hi = v[lane+32]) across the
// warp; returns the scale.
__device__ __forceinline__ float warp_quantize64(float lo, float hi, int8_t &qlo, int8_t &qhi) {
    float peak = warp_max_f(fmaxf(fabsf(lo), fabsf(hi)));
    float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    float inverse = __fdiv_rn(1.0f, scale);
    qlo = quant1(lo, inverse);
    qhi = quant1(hi, inverse);
    return scale;
}

// ------------------------------------------------------------- KV write --
__global__ void __launch_bounds__(256) kv_write_kernel(KvWriteArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.rows * a.heads) return;
    const int row = warp / a.heads, head = warp - row * a.heads;
    const int pos = a.row_pos[row];
    const int slot = a.row_slot[row];
    const float *base = a.qkv + (size_t)row * a.ld_qkv + head * kHeadDim;
    const int width = a.heads * kHeadDim;
    const float c = a.rope_cos[(size_t)pos * (kHeadDim / 2) + lane];
    const float s = a.rope_sin[(size_t)pos * (kHeadDim / 2) + lane];
    int8_t lo8, hi8;
    // q: RoPE + per-head quantize
    {
        float x0 = base[lane], x1 = base[lane + 32];
        float lo = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float hi = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        float scale = warp_quantize64(lo, hi, lo8, hi8);
        int8_t *qo = a.q8 + ((size_t)row * a.heads + head) * kHeadDim;
        qo[lane] = lo8;
        qo[lane + 32] = hi8;
        if (lane == 0) a.qs[(size_t)row * a.heads + head] = scale;
    }
    const int pg = pos / kPagePositions, j = pos - pg * kPagePositions;
    int page = (pg < a.max_pages) ? a.page_table[(size_t)slot * a.max_pages + pg] : -1;
    bool ok = page >= 0 && page < a.num_pages;
    if (!ok && lane == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    uint8_t *blk = ok ? a.pool + (size_t)page * a.page_bytes + kv_block_offset(a.layer, head, a.heads) : nullptr;
    // k: RoPE + per-(position, head) quantize into the page
    {
        const float *kb = base + width;
        float x0 = kb[lane], x1 = kb[lane + 32];
        float lo = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float hi = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        float scale = warp_quantize64(lo, hi, lo8, hi8);
        if (ok) {
            blk[j * kHeadDim + lane] = (uint8_t)lo8;
            blk[j * kHeadDim + lane + 32] = (uint8_t)hi8;
            if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[j] = scale;
        }
    }
    // v: per-(position, head) quantize into the page
    {
        const float *vb = base + 2 * width;
        float scale = warp_quantize64(vb[lane], vb[lane + 32], lo8, hi8);
        if (ok) {
            blk[kVOffset + j * kHeadDim + lane] = (uint8_t)lo8;
            blk[kVOffset + j * kHeadDim + lane + 32] = (uint8_t)hi8;
            if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[j] = scale;
        }
    }
}

int launch_kv_write(const KvWriteArgs &a, cudaStream_t stream) {
    int warps = a.rows * a.heads;
    if (warps == 0) return NDL_OK;
    kv_write_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(a);
    return check_launch("kv_write");
}

// ------------------------------------------------------ decode attention --
constexpr int kAttnWarps = 4;
constexpr int kAttnStages = 3;
constexpr int kWarpSmem = kAttnStages * kKvBlockBytes + 64 + 64;  // ring + barriers + query
constexpr uint32_t kWaitLimit = 1u << 22;

// int8x4 -> 4 floats exactly: bias each byte by 128, splice it under the
// exponent of 2^23 and subtract 2^23 + 128.
__device__ __forceinline__ void i8x4_to_f32(uint32_t v, float (&f)[4]) {
    uint32_t u = v ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
}

__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * kAttnWarps + warp;
    const int chunk = (int)(item % a.max_chunks);
    const long long rh = item / a.max_chunks;
    const int head = (int)(rh % a.heads);
    const int ri = (int)(rh / a.heads);
    if (ri >= a.rows) return;
    const int row = a.row_order ? a.row_order[ri] : ri;
    const int len = a.row_pos[row] + 1;
    const int n_pages = (len + kPagePositions - 1) / kPagePositions;
    const int n_chunks = (n_pages + a.chunk_pages - 1) / a.chunk_pages;
    if (chunk >= n_chunks) return;
    const int first_page = chunk * a.chunk_pages;
    const int n_it = min(n_pages, first_page + a.chunk_pages) - first_page;
    const int slot = a.row_slot[row];

    uint8_t *ring = smem + warp * kWarpSmem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + kAttnStages * kKvBlockBytes);
    if (lane == 0) {
        for (int s = 0; s < kAttnStages; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    auto issue = [&](int it) {  // lane 0 only
        const int pg = first_page + it;
        const int page = a.page_table[(size_t)slot * a.max_pages + pg];
        uint64_t *bar = &bars[it % kAttnStages];
        if (page < 0 || page >= a.num_pages) {
            if (a.status) atomicOr(a.status, kStatusBadPage);
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
            return;
        }
        const uint8_t *src = a.pool + (size_t)page * a.page_bytes + kv_block_offset(a.layer, head, a.heads);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, kKvBlockBytes);
        bulk_g2s(ring + (it % kAttnStages) * kKvBlockBytes, src, kKvBlockBytes, bar);
    };
    if (lane == 0)
        for (int it = 0; it < min(kAttnStages, n_it); it++) issue(it);

    // the query row, staged in shared memory (lanes read rotated 16-byte chunks)
    uint4 *qsm = reinterpret_cast<uint4 *>(ring + kAttnStages * kKvBlockBytes + 64);
    if (lane < 4) qsm[lane] = reinterpret_cast<const uint4 *>(a.q + ((size_t)row * a.heads + head) * kHeadDim)[lane];
    __syncwarp();
    const float scale = __fmul_rn(a.qs[(size_t)row * a.heads + head], a.inv_sqrt_d);

    float m = -INFINITY, l = 0.0f;
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int par = lane >> 4;          // PV: even (0) or odd (1) positions
    const int dd = 4 * (lane & 15);     // PV: this lane's 4 dims
    int it = 0;
    bool timed_out = false;
    for (; it < n_it; it++) {
        const int stage = it % kAttnStages;
        if (!mbar_wait_bounded(&bars[stage], (it / kAttnStages) & 1, kWaitLimit)) {
            timed_out = true;
            break;
        }
        const uint8_t *blk = ring + stage * kKvBlockBytes;
        const int valid = min(kPagePositions, len - (first_page + it) * kPagePositions);
        // scores for positions lane and lane + 32 (16-byte chunks rotated per lane pair: no bank conflicts)
        float sc[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = lane + 32 * h;
            const uint4 *krow = reinterpret_cast<const uint4 *>(blk + j * kHeadDim);
            int dot = 0;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int cc = (c + (lane >> 1)) & 3;
                const uint4 kv = krow[cc];
                const uint4 qv = qsm[cc];
                dot = __dp4a((int)kv.x, (int)qv.x, dot);
                dot = __dp4a((int)kv.y, (int)qv.y, dot);
                dot = __dp4a((int)kv.z, (int)qv.z, dot);
                dot = __dp4a((int)kv.w, (int)qv.w, dot);
            }
            const float ks = reinterpret_cast<const float *>(blk + kKScaleOffset)[j];
            sc[h] = j < valid ? __fmul_rn(__fmul_rn(__int2float_rn(dot), ks), scale) : -INFINITY;
        }
        const float m_new = fmaxf(m, warp_max_f(fmaxf(sc[0], sc[1])));
        const float corr = expf(m - m_new);
        const float p0 = lane < valid ? expf(sc[0] - m_new) : 0.0f;
        const float p1 = lane + 32 < valid ? expf(sc[1] - m_new) : 0.0f;
        l = l * corr + warp_sum_f(p0 + p1);
        m = m_new;
        const float *vsc = reinterpret_cast<const float *>(blk + kVScaleOffset);
        const float w0 = lane < valid ? p0 * vsc[lane] : 0.0f;
        const float w1 = lane + 32 < valid ? p1 * vsc[lane + 32] : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) o[i] *= corr;
        const uint8_t *vbase = blk + kVOffset + dd;
#pragma unroll 8
        for (int jj = 0; jj < 32; jj++) {
            const int j = 2 * jj + par;
            const float w = jj < 16 ? __shfl_sync(0xffffffffu, w0, j & 31) : __shfl_sync(0xffffffffu, w1, j & 31);
            float f[4];
            i8x4_to_f32(*reinterpret_cast<const uint32_t *>(vbase + j * kHeadDim), f);
#pragma unroll
            for (int i = 0; i < 4; i++) o[i] = fmaf(w, f[i], o[i]);
        }
        __syncwarp();
        if (lane == 0 && it + kAttnStages < n_it) issue(it + kAttnStages);
    }
    if (timed_out) {
        // record, then wait (bounded) for the copies this warp still has in flight
        if (lane == 0 && a.status) atomicOr(a.status, kStatusTimeout);
        for (int k = it + 1; k < min(n_it, it + kAttnStages); k++)
            mbar_wait_bounded(&bars[k % kAttnStages], (k / kAttnStages) & 1, kWaitLimit);
        return;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) o[i] += __shfl_xor_sync(0xffffffffu, o[i], 16);

    const size_t rh_index = (size_t)row * a.heads + head;
    float *out = a.out + rh_index * kHeadDim;
    if (n_chunks == 1) {
        const float inv = 1.0f / l;
        if (lane < 16)
            *reinterpret_cast<float4 *>(out + dd) = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
        return;
    }
    // split: publish this chunk's partial, the last arrival merges
    float *part = a.partials + (rh_index * a.max_chunks + chunk) * kPartialFloats;
    if (lane < 16) *reinterpret_cast<float4 *>(part + dd) = make_float4(o[0], o[1], o[2], o[3]);
    if (lane == 0) {
        part[64] = m;
        part[65] = l;
    }
    __threadfence();
    int last = 0;
    if (lane == 0) last = atomicAdd(&a.arrivals[rh_index], 1) == n_chunks - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    const float *parts = a.partials + rh_index * a.max_chunks * kPartialFloats;
    float peak = -INFINITY;
    for (int c = 0; c < n_chunks; c++) peak = fmaxf(peak, __ldcg(parts + c * kPartialFloats + 64));
    float total = 0.0f;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = 0; c < n_chunks; c++) {
        const float *pc = parts + c * kPartialFloats;
        const float wgt = expf(__ldcg(pc + 64) - peak);
        total += wgt * __ldcg(pc + 65);
        if (lane < 16) {
            float4 v = __ldcg(reinterpret_cast<const float4 *>(pc + dd));
            acc[0] += wgt * v.x, acc[1] += wgt * v.y, acc[2] += wgt * v.z, acc[3] += wgt * v.w;
        }
    }
    const float inv = 1.0f / total;
    if (lane < 16)
        *reinterpret_cast<float4 *>(out + dd) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    if (lane == 0) a.arrivals[rh_index] = 0;  // leave the counter ready for the next launch
}

int launch_attn_decode(const AttnArgs &a, cudaStream_t stream) {
    if (a.rows == 0) return NDL_OK;
    static bool configured = false;  // per process; the attribute is per device function
    const int smem = kAttnWarps * kWarpSmem;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
        configured = true;
    }
    long long items = (long long)a.rows * a.heads * a.max_chunks;
    long long blocks = (items + kAttnWarps - 1) / kAttnWarps;
    if (blocks > 0x7FFFFFFF) return set_error(NDL_ERR_INVALID_ARG, "attention grid too large");
    attn_decode_kernel<<<(unsigned)blocks, kAttnWarps * 32, smem, stream>>>(a);
    return check_launch("attn_decode");
}

}  // namespace ndl
