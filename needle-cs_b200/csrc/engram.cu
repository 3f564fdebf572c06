// Engram, the Needle-3 n-gram memory (EngineCore.ApplyEngramBatch,
// src/Needle/Engine.cs:2405-2469, and EngramHashRowsBatch, :2652-2681),
// batched on the device.  The block's table gather, fake-A8, activation prep
// and key / value matmuls are the CQ kernels (cq.cu) and the fake-A8 row op
// (rowops.cu); this file holds the three steps that are Engram's own:
//  * the row hash: per (token, table) an FNV-style hash of the token's
//    n-gram (tokens of the same slot earlier in the batch, else the slot's
//    last two tokens) picks a table row, -1 while the n-gram does not fit;
//  * the causal conv: per token a window of the slot's last 9 values and its
//    own, out = sum_j taps[j] * window[9 - j*dilation] over 4 taps; a run's
//    last window becomes the slot's new history;
//  * the gate: residual += sigmoid(dot(RmsUnit(x), RmsUnit(key)) / sqrt(dim)) * v.
// Rows of consecutive tokens with the same slot form a run, as in the
// reference's batch.  Integer work is exact; the float sums run in the
// scalar code's order (the gate's exp aside).
#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

constexpr int kEngramHistory = 9;  // EngineCore.EngramHistory (Engine.cs:27)
constexpr int kEngramTaps = 4;     // EngineCore.EngramTaps (Engine.cs:28)
constexpr int kEngramMaxOrders = 4;

struct EngramOrders {
    int v[kEngramMaxOrders];
};

__device__ __forceinline__ int run_first(const int32_t *row_slots, int t) {
    int k = t;
    while (k > 0 && row_slots[k - 1] == row_slots[t]) k--;
    return k;
}
__device__ __forceinline__ int run_last(const int32_t *row_slots, int count, int t) {
    int k = t;
    while (k + 1 < count && row_slots[k + 1] == row_slots[t]) k++;
    return k;
}

// Thread per (token, table).
__global__ void __launch_bounds__(256) engram_hash_kernel(const int32_t *__restrict__ tokens,
                                                          const int32_t *__restrict__ row_slots, int count,
                                                          const int32_t *__restrict__ slot_length,
                                                          const int32_t *__restrict__ slot_prev, int slots,
                                                          EngramOrders orders, int order_count, int heads,
                                                          int engram_slots, int32_t *__restrict__ rows) {
    pdl_enter();
    const int tables = order_count * heads;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)count * tables) return;
    const int t = (int)(i / tables), table = (int)(i - (long long)t * tables);
    const int slot = row_slots[t];
    if (slot < 0 || slot >= slots) {
        rows[i] = -1;
        return;
    }
    const int rs = run_first(row_slots, t);
    const int position = slot_length[slot] + t - rs;
    const int order = orders.v[table / heads];
    if (position < order - 1) {
        rows[i] = -1;
        return;
    }
    uint32_t acc = 0x9E3779B9u * (uint32_t)(table + 1);
    for (int j = 0; j < order; j++) {
        const int back = t - rs - j;
        const int token = back >= 0 ? tokens[rs + back] : slot_prev[2 * slot + back + 2];
        acc = (acc ^ (uint32_t)token) * 0x01000193u;
    }
    acc ^= acc >> 15;
    rows[i] = table * engram_slots + (int)(acc % (uint32_t)engram_slots);
}

// Thread per (token, column).  The slot's value sequence is its 9 history
// entries followed by the run's values; token t's window is entries
// (t - run start) .. (t - run start) + 9 of it.
__global__ void __launch_bounds__(256) engram_conv_kernel(const float *__restrict__ history_in,
                                                          const float *__restrict__ values,
                                                          const int32_t *__restrict__ row_slots, int count,
                                                          int slots, const float *__restrict__ taps, int dilation,
                                                          int dim, float *__restrict__ out,
                                                          float *__restrict__ history_out) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)count * dim) return;
    const int t = (int)(i / dim), c = (int)(i - (long long)t * dim);
    const int slot = row_slots[t];
    if (slot < 0 || slot >= slots) {
        out[(size_t)t * dim + c] = 0.0f;
        return;
    }
    const int rs = run_first(row_slots, t), off = t - rs;
    const float *hist = history_in + (size_t)slot * kEngramHistory * dim;
    auto seq = [&](int p) { return p < kEngramHistory ? hist[(size_t)p * dim + c] : values[(size_t)(rs + p - kEngramHistory) * dim + c]; };
    float acc = 0.0f;
#pragma unroll
    for (int j = 0; j < kEngramTaps; j++)
        acc = __fadd_rn(acc, __fmul_rn(taps[(size_t)j * dim + c], seq(off + kEngramHistory - j * dilation)));
    out[(size_t)t * dim + c] = acc;
    if (t == run_last(row_slots, count, t)) {
        float *ho = history_out + (size_t)slot * kEngramHistory * dim;
        for (int k = 0; k < kEngramHistory; k++) ho[(size_t)k * dim + c] = seq(off + 1 + k);
    }
}

// Warp per token; the sums of squares and the dot run on lane 0 in order.
__global__ void __launch_bounds__(256) engram_gate_kernel(const float *__restrict__ x, const float *__restrict__ key,
                                                          const float *__restrict__ v, int count, int dim,
                                                          float *__restrict__ residual) {
    pdl_enter();
    const int t = (int)(((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (t >= count) return;
    const float *xt = x + (size_t)t * dim, *kt = key + (size_t)t * dim;
    float alpha = 0.0f;
    if (lane == 0) {
        float sa = 0.0f, sb = 0.0f;
        for (int i = 0; i < dim; i++) {
            sa = __fadd_rn(sa, __fmul_rn(xt[i], xt[i]));
            sb = __fadd_rn(sb, __fmul_rn(kt[i], kt[i]));
        }
        const float ia = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sa, (float)dim), 1e-6f)));
        const float ib = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sb, (float)dim), 1e-6f)));
        float dot = 0.0f;
        for (int i = 0; i < dim; i++) dot = __fadd_rn(dot, __fmul_rn(__fmul_rn(xt[i], ia), __fmul_rn(kt[i], ib)));
        const float z = __fmul_rn(dot, __fdiv_rn(1.0f, __fsqrt_rn((float)dim)));
        alpha = sigmoid_rn(z);
    }
    alpha = __shfl_sync(0xffffffffu, alpha, 0);
    float *rt = residual + (size_t)t * dim;
    const float *vt = v + (size_t)t * dim;
    for (int i = lane; i < dim; i += 32) rt[i] = __fadd_rn(rt[i], __fmul_rn(alpha, vt[i]));
}

// CTA-per-row form of engram_gate_kernel for dim % 4 == 0, dim <= 4096 and
// 16-byte aligned rows, the same arithmetic term for term: the rows stay in
// registers (float4 i on thread i % 128); the squares of x and key, then the
// products of the unit rows, go through shared memory, and thread 0 runs the
// ascending add chains (both sums of squares interleaved, then the dot)
// with its next float4 loads issued ahead of the current adds.
constexpr int kGateThreads = 128;
constexpr int kGateMaxVec = 8;

__global__ void __launch_bounds__(kGateThreads) engram_gate_row_kernel(const float *__restrict__ x,
                                                                       const float *__restrict__ key,
                                                                       const float *__restrict__ v, int dim,
                                                                       float *__restrict__ residual) {
    pdl_enter();
    __shared__ float4 sq_a[kGateThreads * kGateMaxVec], sq_b[kGateThreads * kGateMaxVec];
    __shared__ float shared_scalar[2];
    const int t = blockIdx.x, tid = threadIdx.x, nv = dim >> 2;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *xa = reinterpret_cast<const float4 *>(x + (size_t)t * dim);
    const float4 *ka = reinterpret_cast<const float4 *>(key + (size_t)t * dim);
    float4 xv[kGateMaxVec], kv[kGateMaxVec];
#pragma unroll
    for (int i = 0; i < kGateMaxVec; i++) {
        const int idx = tid + i * kGateThreads;
        xv[i] = idx < nv ? xa[idx] : zero;
        kv[i] = idx < nv ? ka[idx] : zero;
        if (idx < nv) {
            sq_a[idx] = make_float4(__fmul_rn(xv[i].x, xv[i].x), __fmul_rn(xv[i].y, xv[i].y),
                                    __fmul_rn(xv[i].z, xv[i].z), __fmul_rn(xv[i].w, xv[i].w));
            sq_b[idx] = make_float4(__fmul_rn(kv[i].x, kv[i].x), __fmul_rn(kv[i].y, kv[i].y),
                                    __fmul_rn(kv[i].z, kv[i].z), __fmul_rn(kv[i].w, kv[i].w));
        }
    }
    __syncthreads();
    if (tid == 0) {
        float sa = 0.0f, sb = 0.0f;
        float4 na[2], nb[2];
#pragma unroll
        for (int j = 0; j < 2; j++) na[j] = j < nv ? sq_a[j] : zero, nb[j] = j < nv ? sq_b[j] : zero;
        for (int i = 0; i < nv; i += 2) {
            float4 ca[2], cb[2];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                ca[j] = na[j], cb[j] = nb[j];
                na[j] = i + 2 + j < nv ? sq_a[i + 2 + j] : zero;
                nb[j] = i + 2 + j < nv ? sq_b[i + 2 + j] : zero;
            }
#pragma unroll
            for (int j = 0; j < 2; j++)
                if (i + j < nv) {
                    sa = __fadd_rn(sa, ca[j].x), sb = __fadd_rn(sb, cb[j].x);
                    sa = __fadd_rn(sa, ca[j].y), sb = __fadd_rn(sb, cb[j].y);
                    sa = __fadd_rn(sa, ca[j].z), sb = __fadd_rn(sb, cb[j].z);
                    sa = __fadd_rn(sa, ca[j].w), sb = __fadd_rn(sb, cb[j].w);
                }
        }
        shared_scalar[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sa, (float)dim), 1e-6f)));
        shared_scalar[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sb, (float)dim), 1e-6f)));
    }
    __syncthreads();
    const float ia = shared_scalar[0], ib = shared_scalar[1];
#pragma unroll
    for (int i = 0; i < kGateMaxVec; i++) {
        const int idx = tid + i * kGateThreads;
        if (idx < nv)
            sq_a[idx] = make_float4(__fmul_rn(__fmul_rn(xv[i].x, ia), __fmul_rn(kv[i].x, ib)),
                                    __fmul_rn(__fmul_rn(xv[i].y, ia), __fmul_rn(kv[i].y, ib)),
                                    __fmul_rn(__fmul_rn(xv[i].z, ia), __fmul_rn(kv[i].z, ib)),
                                    __fmul_rn(__fmul_rn(xv[i].w, ia), __fmul_rn(kv[i].w, ib)));
    }
    __syncthreads();
    if (tid == 0) {
        float dot = 0.0f;
        float4 nxt[4];
#pragma unroll
        for (int j = 0; j < 4; j++) nxt[j] = j < nv ? sq_a[j] : zero;
        for (int i = 0; i < nv; i += 4) {
            float4 cur[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                cur[j] = nxt[j];
                nxt[j] = i + 4 + j < nv ? sq_a[i + 4 + j] : zero;
            }
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (i + j < nv) {
                    dot = __fadd_rn(dot, cur[j].x);
                    dot = __fadd_rn(dot, cur[j].y);
                    dot = __fadd_rn(dot, cur[j].z);
                    dot = __fadd_rn(dot, cur[j].w);
                }
        }
        const float z = __fmul_rn(dot, __fdiv_rn(1.0f, __fsqrt_rn((float)dim)));
        shared_scalar[0] = sigmoid_rn(z);
    }
    __syncthreads();
    const float alpha = shared_scalar[0];
    float4 *rt = reinterpret_cast<float4 *>(residual + (size_t)t * dim);
    const float4 *vt = reinterpret_cast<const float4 *>(v + (size_t)t * dim);
#pragma unroll
    for (int i = 0; i < kGateMaxVec; i++) {
        const int idx = tid + i * kGateThreads;
        if (idx < nv) {
            const float4 w = vt[idx];
            float4 r = rt[idx];
            r.x = __fadd_rn(r.x, __fmul_rn(alpha, w.x));
            r.y = __fadd_rn(r.y, __fmul_rn(alpha, w.y));
            r.z = __fadd_rn(r.z, __fmul_rn(alpha, w.z));
            r.w = __fadd_rn(r.w, __fmul_rn(alpha, w.w));
            rt[idx] = r;
        }
    }
}

// Quant.FakeA8 (src/Needle/Quant.cs:69-80) per row, warp per row: the row's
// peak, then each value quantized with the reference's RoundEven (the
// 1.5 * 2^23 bias, which also turns -0 into +0) and scaled back.
__global__ void __launch_bounds__(256) engram_fake_a8_kernel(float *__restrict__ x, int rows, int n) {
    pdl_enter();
    const int r = (int)(((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    float *row = x + (size_t)r * n;
    float peak = 0.0f;
    for (int i = lane; i < n; i += 32) peak = fmaxf(peak, fabsf(row[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    for (int i = lane; i < n; i += 32) {
        const float q = __fsub_rn(__fadd_rn(__fmul_rn(row[i], inverse), 12582912.0f), 12582912.0f);
        row[i] = __fmul_rn(fminf(fmaxf(q, -128.0f), 127.0f), scale);
    }
}

// Workspace of ndl_engram_apply, 256-byte aligned pieces.
struct EngramWork {
    size_t rows, e, values, scales, offsets, key, value, conv, total;
    int stride;
};
EngramWork engram_work(int count, int tables, int dim) {
    EngramWork w{};
    size_t end = 0;
    auto place = [&](size_t bytes) {
        end = (end + 255) & ~(size_t)255;
        const size_t at = end;
        end += bytes;
        return at;
    };
    const size_t rd = (size_t)count * dim;
    w.stride = ((dim / 128) + 7) & ~7;
    w.rows = place((size_t)count * tables * 4);
    w.e = place(rd * 4);
    w.values = place(rd);
    w.scales = place((size_t)count * w.stride * 4);
    w.offsets = place((size_t)count * w.stride * 4);
    w.key = place(rd * 4);
    w.value = place(rd * 4);
    w.conv = place(rd * 4);
    w.total = (end + 255) & ~(size_t)255;
    return w;
}

}  // namespace ndl

using namespace ndl;

extern "C" NDL_API int ndl_engram_hash(const int32_t *tokens, const int32_t *row_slots, int count,
                                       const int32_t *slot_length, const int32_t *slot_prev, int slots,
                                       const int32_t *orders, int order_count, int heads, int engram_slots,
                                       int32_t *rows, void *stream) {
    NDL_REQUIRE(count >= 0 && slots >= 1 && heads >= 1 && engram_slots >= 1, "count %d / slots %d / heads %d / rows %d",
                count, slots, heads, engram_slots);
    NDL_REQUIRE(orders && order_count >= 1 && order_count <= kEngramMaxOrders, "%d orders (1..%d)", order_count,
                kEngramMaxOrders);
    EngramOrders ov{};
    for (int o = 0; o < order_count; o++) {
        NDL_REQUIRE(orders[o] >= 1 && orders[o] <= 3, "order %d (1..3: two earlier tokens are kept per slot)",
                    orders[o]);
        ov.v[o] = orders[o];
    }
    NDL_REQUIRE((long long)order_count * heads * engram_slots <= 0x7FFFFFFF, "table rows overflow int");
    if (count == 0) return NDL_OK;
    NDL_REQUIRE(tokens && row_slots && slot_length && slot_prev && rows, "null pointer");
    const long long n = (long long)count * order_count * heads;
    launch_kernel(engram_hash_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, tokens,
                  row_slots, count, slot_length, slot_prev, slots, ov, order_count, heads, engram_slots, rows);
    return check_launch("engram_hash");
}

extern "C" NDL_API int ndl_engram_conv(const float *history_in, const float *values, const int32_t *row_slots,
                                       int count, int slots, const float *taps, int dilation, int dim, float *out,
                                       float *history_out, void *stream) {
    NDL_REQUIRE(count >= 0 && slots >= 1 && dim >= 1, "count %d / slots %d / dim %d", count, slots, dim);
    NDL_REQUIRE(dilation >= 1 && (kEngramTaps - 1) * dilation <= kEngramHistory, "dilation %d (1..3)", dilation);
    if (count == 0) return NDL_OK;
    NDL_REQUIRE(history_in && values && row_slots && taps && out && history_out, "null pointer");
    NDL_REQUIRE(history_in != history_out, "history_out must not alias history_in");
    const long long n = (long long)count * dim;
    launch_kernel(engram_conv_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, (cudaStream_t)stream,
                  history_in, values, row_slots, count, slots, taps, dilation, dim, out, history_out);
    return check_launch("engram_conv");
}

extern "C" NDL_API int ndl_engram_gate(const float *x, const float *key, const float *v, int count, int dim,
                                       float *residual, void *stream) {
    NDL_REQUIRE(count >= 0 && dim >= 1, "count %d / dim %d", count, dim);
    if (count == 0) return NDL_OK;
    NDL_REQUIRE(x && key && v && residual, "null pointer");
    if (dim % 4 == 0 && dim <= 4 * kGateThreads * kGateMaxVec && aligned(x, 16) && aligned(key, 16) &&
        aligned(v, 16) && aligned(residual, 16)) {
        launch_kernel(engram_gate_row_kernel, dim3((unsigned)count), dim3(kGateThreads), 0, (cudaStream_t)stream, x,
                      key, v, dim, residual);
        return check_launch("engram_gate_row");
    }
    launch_kernel(engram_gate_kernel, dim3((unsigned)((count * 32LL + 255) / 256)), dim3(256), 0,
                  (cudaStream_t)stream, x, key, v, count, dim, residual);
    return check_launch("engram_gate");
}

// The Engram block of one site on a loaded model (ApplyEngramBatch,
// src/Needle/Engine.cs:2405-2469), chained on the stream:
//  row hash -> table rows gathered (GatherRow; -1 gives zeros) into
//  e[t] = [table 0 | table 1 | ...] -> FakeA8 per row -> 2-bit CQ prep ->
//  key and value CQ matmuls -> dilated conv over the slot history ->
//  residual += sigmoid(dot(RmsUnit(x), RmsUnit(key)) / sqrt(dim)) * conv.
static int engram_site_views(const ndl_model *m, int site, ndl_model_info *g, ndl_model_tensor *tables,
                             ndl_model_tensor *key, ndl_model_tensor *value, ndl_model_tensor *taps) {
    NDL_REQUIRE(m, "null model");
    if (ndl_model_get_info(m, g) != NDL_OK) return NDL_ERR_INVALID_ARG;
    NDL_REQUIRE(site >= 0 && site < g->site_count, "site %d of %d", site, g->site_count);
    NDL_REQUIRE(g->device >= 0, "the model is not on a device (load it with a device)");
    if (ndl_model_get_tensor(m, "site.tables", site, tables) != NDL_OK ||
        ndl_model_get_tensor(m, "site.key", site, key) != NDL_OK ||
        ndl_model_get_tensor(m, "site.value", site, value) != NDL_OK ||
        ndl_model_get_tensor(m, "site.taps", site, taps) != NDL_OK)
        return NDL_ERR_INVALID_ARG;
    const int dim = g->dim, heads = g->order_count > 0 ? g->engram_tables / g->order_count : 0;
    if (g->order_count < 1 || heads * g->order_count != g->engram_tables || g->engram_tables * g->engram_sub != dim ||
        tables->cols != g->engram_sub || tables->rows != g->engram_tables * g->engram_slots)
        return set_error(NDL_ERR_UNSUPPORTED,
                         "Engram site %d: %d tables of %d columns (%d x %d rows) do not tile the %d-wide input", site,
                         g->engram_tables, tables->cols, g->engram_tables, g->engram_slots, dim);
    if (key->bits != 2 || value->bits != 2 || key->rows != dim || key->cols != dim || value->rows != dim ||
        value->cols != dim || taps->count < 4LL * dim)
        return set_error(NDL_ERR_UNSUPPORTED, "Engram site %d: key / value must be 2-bit %d x %d, taps 4 x %d", site,
                         dim, dim, dim);
    return NDL_OK;
}

extern "C" NDL_API size_t ndl_engram_workspace(const ndl_model *m, int count) {
    ndl_model_info g;
    if (!m || count < 0 || ndl_model_get_info(m, &g) != NDL_OK) return 0;
    return engram_work(count, g.engram_tables, g.dim).total;
}

extern "C" NDL_API int ndl_engram_apply(const ndl_model *m, int site, const int32_t *tokens, const int32_t *row_slots,
                                        int count, const int32_t *slot_length, const int32_t *slot_prev, int slots,
                                        const float *history_in, float *history_out, const float *x, float *residual,
                                        void *workspace, size_t workspace_bytes, void *stream) {
    ndl_model_info g;
    ndl_model_tensor tables, key, value, taps;
    const int st = engram_site_views(m, site, &g, &tables, &key, &value, &taps);
    if (st != NDL_OK) return st;
    NDL_REQUIRE(count >= 0 && slots >= 1, "count %d / slots %d", count, slots);
    if (count == 0) return NDL_OK;
    const int dim = g.dim;
    const EngramWork w = engram_work(count, g.engram_tables, dim);
    NDL_REQUIRE(workspace && workspace_bytes >= w.total, "workspace of %zu bytes, %zu needed", workspace_bytes,
                w.total);
    NDL_REQUIRE(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int32_t *rows = reinterpret_cast<int32_t *>(ws + w.rows);
    float *e = reinterpret_cast<float *>(ws + w.e), *scales = reinterpret_cast<float *>(ws + w.scales);
    float *offsets = reinterpret_cast<float *>(ws + w.offsets), *k = reinterpret_cast<float *>(ws + w.key);
    float *v = reinterpret_cast<float *>(ws + w.value), *conv = reinterpret_cast<float *>(ws + w.conv);
    int8_t *values = reinterpret_cast<int8_t *>(ws + w.values);
    const int heads = g.engram_tables / g.order_count;
#define ENGRAM_TRY(x)                      \
    do {                                   \
        const int s_ = (x);                \
        if (s_ != NDL_OK) return s_;       \
    } while (0)
    ENGRAM_TRY(ndl_engram_hash(tokens, row_slots, count, slot_length, slot_prev, slots, g.orders, g.order_count, heads,
                               g.engram_slots, rows, stream));
    ENGRAM_TRY(ndl_cq_gather_rows(tables.indices, tables.norms, tables.book->levels, tables.rows, tables.cols,
                                  tables.bits, rows, count * g.engram_tables, e, stream));
    launch_kernel(engram_fake_a8_kernel, dim3((unsigned)((count * 32LL + 255) / 256)), dim3(256), 0,
                  (cudaStream_t)stream, e, count, dim);
    ENGRAM_TRY(check_launch("engram_fake_a8"));
    ENGRAM_TRY(ndl_cq_prepare(e, count, dim, 2, values, scales, offsets, w.stride, stream));
    ENGRAM_TRY(ndl_cq_matmul(key.indices, key.norms, key.book->bytes, key.book->byte_scale, dim, dim, 2, values,
                             scales, offsets, w.stride, count, k, dim, 0, dim, stream));
    ENGRAM_TRY(ndl_cq_matmul(value.indices, value.norms, value.book->bytes, value.book->byte_scale, dim, dim, 2,
                             values, scales, offsets, w.stride, count, v, dim, 0, dim, stream));
    ENGRAM_TRY(ndl_engram_conv(history_in, v, row_slots, count, slots, taps.values, g.engram_dilation, dim, conv,
                               history_out, stream));
    ENGRAM_TRY(ndl_engram_gate(x, k, conv, count, dim, residual, stream));
#undef ENGRAM_TRY
    return NDL_OK;
}
