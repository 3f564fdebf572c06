// Small kernels of the batched decode step: step preparation (page-table
// updates + embedding gather), SwiGLU + quantize, head-row gather, masked
// argmax with probability, top-k log-softmax, and the synthetic KV fill.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {

// ---------------------------------------------------------- preparation --
// Applies (slot, index, page) updates to the device page table (the count
// is read from device memory so one captured graph serves every step),
// then gathers fp16 embedding rows into the fp32 residual stream x.
__global__ void __launch_bounds__(256) step_prepare_kernel(const int32_t *__restrict__ updates,
                                                           int32_t *__restrict__ page_table, int max_pages,
                                                           const int32_t *__restrict__ tokens, int rows,
                                                           const uint16_t *__restrict__ embedding, int vocab,
                                                           int dim, float *__restrict__ x, int *status) {
    pdl_enter();
    // updates[0] = count, then (slot, index, page) triples
    if (blockIdx.x == 0) {
        const int n_updates = updates[0];
        for (int i = threadIdx.x; i < n_updates; i += blockDim.x)
            page_table[(size_t)updates[1 + 3 * i] * max_pages + updates[2 + 3 * i]] = updates[3 + 3 * i];
    }
    const int row = blockIdx.x;
    if (row >= rows) return;
    int tok = tokens[row];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && status) atomicOr(status, kStatusBadPage);
        tok = 0;
    }
    const uint16_t *e = embedding + (size_t)tok * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[(size_t)row * dim + i] = half_to_float_ref(e[i]);
}

int launch_step_prepare(const int32_t *updates, int32_t *page_table, int max_pages, const int32_t *tokens, int rows,
                        const uint16_t *embedding, int vocab, int dim, float *x, int *status, cudaStream_t stream) {
    int blocks = rows > 0 ? rows : 1;
    launch_kernel(step_prepare_kernel, dim3(blocks), dim3(256), 0, stream, updates, page_table, max_pages, tokens, rows, embedding, vocab,
                                                     dim, x, status);
    return check_launch("step_prepare");
}

// --------------------------------------------------------------- SwiGLU --
__device__ __forceinline__ float warp_max_s(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// a = (g * sigmoid(g)) * u per row (Scalar.Silu/Glu, src/Needle/Scalar.cs:194-204,280-283),
// then the row quantizer.  gu rows are [gate (ffn) | up (ffn)].
__global__ void __launch_bounds__(256) swiglu_quantize_kernel(const float *__restrict__ gu, int rows, int ffn,
                                                              float *__restrict__ act, int8_t *__restrict__ q,
                                                              float *__restrict__ scales) {
    pdl_enter();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *g = gu + (size_t)warp * 2 * ffn;
    const float *u = g + ffn;
    float *a = act + (size_t)warp * ffn;
    float peak = 0.0f;
    for (int i = lane; i < ffn; i += 32) {
        const float gv = g[i];
        const float sig = sigmoid_simd(gv);
        const float v = __fmul_rn(__fmul_rn(gv, sig), u[i]);
        a[i] = v;
        peak = fmaxf(peak, fabsf(v));
    }
    peak = warp_max_s(peak);
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    __syncwarp();
    int8_t *qr = q + (size_t)warp * ffn;
    for (int i = lane; i < ffn; i += 32) {
        float r = rintf(__fmul_rn(a[i], inverse));
        qr[i] = (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
    }
    if (lane == 0) scales[warp] = scale;
}

int launch_swiglu_quantize(const float *gu, int rows, int ffn, float *act, int8_t *q, float *scales,
                           cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    int st = launch_swiglu_quantize_rows(gu, rows, ffn, q, scales, stream);
    if (st != NDL_ERR_UNSUPPORTED) return st;
    launch_kernel(swiglu_quantize_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, gu, rows, ffn, act, q, scales);
    return check_launch("swiglu_quantize");
}

// ---------------------------------------------------------- head gather --
__global__ void gather_rows_kernel(const float *__restrict__ x, const int32_t *__restrict__ idx, int n, int dim,
                                   float *__restrict__ out) {
    pdl_enter();
    const int r = blockIdx.x;
    if (r >= n) return;
    const float *src = x + (size_t)idx[r] * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) out[(size_t)r * dim + i] = src[i];
}

int launch_gather_rows(const float *x, const int32_t *idx, int n, int dim, float *out, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    launch_kernel(gather_rows_kernel, dim3(n), dim3(128), 0, stream, x, idx, n, dim, out);
    return check_launch("gather_rows");
}

// ------------------------------------------------------- masked argmax --
// Ops.ArgMaxMasked (src/Needle/Ops.cs:1223-1299): strict '>' so the lowest
// id wins ties; ids >= length are ignored; -1 when nothing is allowed.
// With want_prob, also p = 1 / sum_allowed exp(x - max)
// (ArgMaxMaskedWithProbability / BestProbability, Ops.cs:1302-1330,1435-1470).
// One CTA per row; mask may be NULL (all allowed) and is indexed per row.
__global__ void __launch_bounds__(256) argmax_masked_kernel(const float *__restrict__ x, long long ldx,
                                                            const uint32_t *__restrict__ mask, int words,
                                                            long long ldm, const int32_t *__restrict__ mask_index,
                                                            int length, int rows, int32_t *__restrict__ ids,
                                                            float *__restrict__ probs) {
    __shared__ float s_val[256];
    __shared__ int s_idx[256];
    __shared__ float s_sum[256];
    const int row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + (size_t)row * ldx;
    // mask row: row itself, or mask_index[row] (negative: no mask)
    const long long mrow = mask_index ? (long long)mask_index[row] : (long long)row;
    const uint32_t *mr = mask && mrow >= 0 ? mask + mrow * ldm : nullptr;
    const int limit = mr ? min(length, words * 32) : length;
    float best = -INFINITY;
    int best_i = -1;
    // each thread scans four consecutive ids at a time (one 16-byte load, ids in increasing order, so the
    // first of equal values stays), four such loads in flight per pass
    const bool vec = (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
    const int quads = vec ? limit >> 2 : 0;
    for (int q0 = threadIdx.x; q0 < quads; q0 += 4 * blockDim.x) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = q0 + u * blockDim.x;
            v[u] = q < quads ? __ldg(reinterpret_cast<const float4 *>(xr) + q) : make_float4(-INFINITY, -INFINITY,
                                                                                              -INFINITY, -INFINITY);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = q0 + u * blockDim.x;
            if (q >= quads) break;
            const uint32_t bits = mr ? (mr[q >> 3] >> ((q & 7) * 4)) & 0xFu : 0xFu;
            const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (((bits >> j) & 1u) && e[j] > best) {
                    best = e[j];
                    best_i = 4 * q + j;
                }
        }
    }
    // the scalar remainder (and every id when the row cannot be read as float4)
    for (int i = 4 * quads + threadIdx.x; i < limit; i += blockDim.x) {
        if (mr && !((mr[i >> 5] >> (i & 31)) & 1u)) continue;
        const float v = xr[i];
        if (v > best) {
            best = v;
            best_i = i;
        }
    }
    s_val[threadIdx.x] = best;
    s_idx[threadIdx.x] = best_i;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = s_val[threadIdx.x + s];
            const int oi = s_idx[threadIdx.x + s];
            const float mv = s_val[threadIdx.x];
            const int mi = s_idx[threadIdx.x];
            // keep the larger value; on equal values the lower index
            if (oi >= 0 && (mi < 0 || ov > mv || (ov == mv && oi < mi))) {
                s_val[threadIdx.x] = ov;
                s_idx[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    const int arg = s_idx[0];
    const float peak = s_val[0];
    if (probs) {
        float sum = 0.0f;
        if (arg >= 0)
            for (int i = threadIdx.x; i < limit; i += blockDim.x) {
                if (mr && !((mr[i >> 5] >> (i & 31)) & 1u)) continue;
                sum += expf(xr[i] - peak);
            }
        __syncthreads();
        s_sum[threadIdx.x] = sum;
        __syncthreads();
        for (int s = blockDim.x / 2; s > 0; s >>= 1) {
            if (threadIdx.x < s) s_sum[threadIdx.x] += s_sum[threadIdx.x + s];
            __syncthreads();
        }
        if (threadIdx.x == 0) probs[row] = arg >= 0 ? 1.0f / s_sum[0] : 0.0f;
    }
    if (threadIdx.x == 0) ids[row] = arg;
}

int launch_argmax_masked(const float *x, long long ldx, const uint32_t *mask, int words, long long ldm,
                         const int32_t *mask_index, int length, int rows, int32_t *ids, float *probs,
                         cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    argmax_masked_kernel<<<rows, 256, 0, stream>>>(x, ldx, mask, words, ldm, mask_index, length, rows, ids, probs);
    return check_launch("argmax_masked");
}

// ------------------------------------------------- top-k log-softmax --
// Ops.TopKLogSoftmax (src/Needle/Ops.cs:1092-1221): top-k ordered by
// (value desc, index asc); log-probabilities x - (max + ln sum exp(x - max));
// mask_special_023 removes ids 0, 2 and 3.  One CTA per row, k <= 8.
constexpr int kTopKMax = 8;

__device__ __forceinline__ bool topk_better(float v, int i, float w, int j) {
    return v > w || (v == w && i < j);
}

__global__ void __launch_bounds__(256) topk_logsoftmax_kernel(const float *__restrict__ x, long long ldx, int n,
                                                              int k, int mask023, int rows, int32_t *__restrict__ idx,
                                                              float *__restrict__ logp, float *__restrict__ probs) {
    __shared__ float s_v[256 * kTopKMax];
    __shared__ int s_i[256 * kTopKMax];
    __shared__ double s_sum[256];
    const int row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + (size_t)row * ldx;
    float tv[kTopKMax];
    int ti[kTopKMax];
    for (int j = 0; j < kTopKMax; j++) tv[j] = -INFINITY, ti[j] = 0x7FFFFFFF;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        if (mask023 && (i == 0 || i == 2 || i == 3)) continue;
        const float v = xr[i];
        if (!topk_better(v, i, tv[k - 1], ti[k - 1])) continue;
        int p = k - 1;
        while (p > 0 && topk_better(v, i, tv[p - 1], ti[p - 1])) {
            tv[p] = tv[p - 1];
            ti[p] = ti[p - 1];
            p--;
        }
        tv[p] = v;
        ti[p] = i;
    }
    for (int j = 0; j < k; j++) s_v[threadIdx.x * kTopKMax + j] = tv[j], s_i[threadIdx.x * kTopKMax + j] = ti[j];
    __syncthreads();
    // pairwise merge of sorted lists
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float *av = s_v + threadIdx.x * kTopKMax;
            const int *ai = s_i + threadIdx.x * kTopKMax;
            const float *bv = s_v + (threadIdx.x + s) * kTopKMax;
            const int *bi = s_i + (threadIdx.x + s) * kTopKMax;
            float mv[kTopKMax];
            int mi[kTopKMax];
            int pa = 0, pb = 0;
            for (int j = 0; j < k; j++) {
                if (topk_better(av[pa], ai[pa], bv[pb], bi[pb])) mv[j] = av[pa], mi[j] = ai[pa], pa++;
                else mv[j] = bv[pb], mi[j] = bi[pb], pb++;
            }
            for (int j = 0; j < k; j++) s_v[threadIdx.x * kTopKMax + j] = mv[j], s_i[threadIdx.x * kTopKMax + j] = mi[j];
        }
        __syncthreads();
    }
    const float peak = s_v[0];
    double sum = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = (mask023 && (i == 0 || i == 2 || i == 3)) ? -1e30f : xr[i];
        sum += exp((double)(v - peak));
    }
    s_sum[threadIdx.x] = sum;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) s_sum[threadIdx.x] += s_sum[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const float shift = peak + (float)log(s_sum[0]);
        for (int j = 0; j < k; j++) {
            idx[(size_t)row * k + j] = s_i[j];
            const float lp = s_v[j] - shift;
            logp[(size_t)row * k + j] = lp;
            if (probs) probs[(size_t)row * k + j] = expf(lp);
        }
    }
}

int launch_topk_logsoftmax(const float *x, long long ldx, int n, int k, int mask023, int rows, int32_t *idx,
                           float *logp, float *probs, cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    if (k < 1 || k > kTopKMax) return set_error(NDL_ERR_INVALID_ARG, "top-k: k=%d outside 1..%d", k, kTopKMax);
    topk_logsoftmax_kernel<<<rows, 256, 0, stream>>>(x, ldx, n, k, mask023, rows, idx, logp, probs);
    return check_launch("topk_logsoftmax");
}

// ---------------------------------------------------- synthetic KV fill --
// Prefix K/V of one slot: value (layer, kind, pos, head, d) is the fp16 of
// normal(seed, session stream, index) with
//   index = ((((layer * 2 + kind) << 20) + pos) * heads + head) * 64 + d,
// quantized per (position, head) like the KV write (src/Needle/Engine.cs:2566-2567).
__global__ void __launch_bounds__(256) kv_fill_kernel(uint64_t key, int layers, int heads, int first, int count,
                                                      const int32_t *__restrict__ page_row, uint8_t *pool,
                                                      long long page_bytes) {
    const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long long total = (long long)layers * 2 * count * heads;
    if (warp >= total) return;
    const int head = (int)(warp % heads);
    long long r = warp / heads;
    const int pos = first + (int)(r % count);
    r /= count;
    const int kind = (int)(r % 2);
    const int layer = (int)(r / 2);
    const uint64_t base = ((((uint64_t)(layer * 2 + kind)) << 20) + (uint64_t)pos) * heads + head;
    const float lo = half_to_float_ref(float_to_half_rne(synth_normal(key, base * 64 + lane)));
    const float hi = half_to_float_ref(float_to_half_rne(synth_normal(key, base * 64 + lane + 32)));
    float peak = warp_max_s(fmaxf(fabsf(lo), fabsf(hi)));
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    const int8_t q0 = (int8_t)(int)fminf(fmaxf(rintf(__fmul_rn(lo, inverse)), -128.0f), 127.0f);
    const int8_t q1 = (int8_t)(int)fminf(fmaxf(rintf(__fmul_rn(hi, inverse)), -128.0f), 127.0f);
    const int page = page_row[pos / kPagePositions];
    const int j = pos % kPagePositions;
    uint8_t *blk = pool + (size_t)page * page_bytes + kv_block_offset(layer, head, heads);
    if (kind == 0) {
        blk[k_byte(j, lane)] = (uint8_t)q0;
        blk[k_byte(j, lane + 32)] = (uint8_t)q1;
        if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[k_scale_index(j)] = scale;
    } else {
        blk[v_byte(j, lane)] = (uint8_t)q0;
        blk[v_byte(j, lane + 32)] = (uint8_t)q1;
        if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[v_scale_index(j)] = scale;
    }
}

int launch_kv_fill(uint64_t seed, uint64_t session, int layers, int heads, int first, int count,
                   const int32_t *page_row, uint8_t *pool, long long page_bytes, cudaStream_t stream) {
    if (count <= 0) return NDL_OK;
    long long warps = (long long)layers * 2 * count * heads;
    kv_fill_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(synth_key(seed, session), layers, heads, first,
                                                                     count, page_row, pool, page_bytes);
    return check_launch("kv_fill");
}

// fp16 bits -> fp32 (the reference's HalfToSingle, exact), e.g. the encoder
// memory before its rows are quantized.
__global__ void half_to_float_kernel(const uint16_t *__restrict__ src, long long n, float *__restrict__ dst) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        dst[i] = half_to_float_ref(src[i]);
}

int launch_half_to_float(const uint16_t *src, long long n, float *dst, cudaStream_t stream) {
    if (n <= 0) return NDL_OK;
    const long long blocks = std::min<long long>((n + 255) / 256, 148 * 16);
    half_to_float_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, n, dst);
    return check_launch("half_to_float");
}

// BestProbability (src/Needle/Ops.cs:1435-1470): 1 / sum_i exp(x_i - best),
// one CTA (tree sum; the reference's vector sum order differs: tolerance).
__global__ void __launch_bounds__(256) best_probability_kernel(const float *__restrict__ x, int count, float best,
                                                               float *__restrict__ out) {
    __shared__ float s_sum[256];
    float acc = 0.0f;
    for (int i = threadIdx.x; i < count; i += blockDim.x) acc += expf(x[i] - best);
    s_sum[threadIdx.x] = acc;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) s_sum[threadIdx.x] += s_sum[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[0] = 1.0f / s_sum[0];
}

int launch_best_probability(const float *x, int count, float best, float *out, cudaStream_t stream) {
    best_probability_kernel<<<1, 256, 0, stream>>>(x, count, best, out);
    return check_launch("best_probability");
}

}  // namespace ndl
