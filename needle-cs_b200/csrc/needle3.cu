// Needle-3 batched decode on a loaded .cact model: EngineCore.ForwardBatch
// with RunLayerBatch (src/Needle/Engine.cs:2303-2596) on the device, the
// reference's scalar tier throughout (MathF.Exp as exp_rn, products and sums
// rounded one operation at a time), so every slot's logits equal the CPU
// restatement's bit for bit.
//
// Per forward of rows with distinct slots (a run of one slot is fed as
// consecutive forwards, which the reference's run semantics equal):
//   embedding  GatherRow (CQ), x += x * (sqrt(dim) - 1), copied to 4 streams
//   per layer  RmsFakeA8 of the 4-stream row, Prepare at 4 bits; the phi
//              pre / post / res CQ matmuls on the layer's row slices;
//              hyper-connection gates (sigmoids of the scaled phi outputs);
//              u = Mix4(streams, hpre); mix = Sinkhorn4x4; residual = u;
//              Engram at a site layer (ndl_engram_apply);
//              CenteredRmsFakeA8(residual, norm_in), Prepare at 2 bits; Q, K,
//              V, gate CQ matmuls; 3-tap convs over the slot's two previous
//              projections; per head ZeroCenteredRms and RoPE, QuantizeInt8
//              of q and of the new K / V position into the slot's cache;
//              attention (grouped heads, sliding window on local layers);
//              GateFakeA8, Prepare, out matmul, PostNormAdd; the Kronecker
//              MLP (ndl_mlp_apply); CombineDiff4x4 into the next streams
//   after      the slots' last two tokens and lengths advance
//   heads      Mix4 by 1/4, CenteredRmsFakeA8(final_norm), Prepare at 4 bits,
//              the embedding CQ matmul over the vocabulary.
// Per-slot state lives on the device: the convs' two previous projections
// per layer, an int8 K / V cache per layer with fp32 scales per (position,
// kv head), the Engram histories per site and the previous two tokens.
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "needle3.cuh"

namespace ndl {

namespace {

constexpr int kLanes = 4;
constexpr int kConvHist = 2;      // ConvTaps - 1 previous projections per layer
constexpr int kEngramHistory = 9;
constexpr int kN3Warps = 4;       // warps per CTA of the per-(row, head) kernels

struct CqView {
    const uint8_t *indices = nullptr;
    const uint16_t *norms = nullptr;
    const ndl_kt_codebook *book = nullptr;
    int rows = 0, cols = 0, bits = 0;
};

struct LayerView {
    CqView q, k, v, gate, out;
    const float *norm_in, *q_taps, *k_taps, *v_taps, *q_norm, *k_norm, *post_norm;
    float attn_gate;  // sigmoid of the stored logit
    int window;       // 0: global
    const float *mlp[13], *pre_hada;  // HadamardMlp factors (d1 .. cond_u) and pre-norm scale
};

}  // namespace

struct N3State {
    const ndl_model *model = nullptr;
    ndl_model_info info{};
    int slots = 0, capacity = 0, max_rows = 0, max_heads = 0;
    int dim = 0, heads = 0, kv = 0, qk = 0, vd = 0, qw = 0, kw = 0, vw = 0, ow = 0, layers = 0, sites = 0;
    std::vector<LayerView> layer;
    CqView embedding, phi_pre, phi_post, phi_res;
    const float *a_pre = nullptr, *b_pre = nullptr, *a_post = nullptr, *b_post = nullptr, *a_res = nullptr,
                *b_res = nullptr, *final_norm = nullptr;
    std::vector<int> site_of_layer;
    std::vector<void *> allocations;
    // per-slot device state
    int32_t *len = nullptr, *prev = nullptr;
    float *conv_hist = nullptr;  // [slots][layers][2][qw + kw + vw]
    int8_t *keys = nullptr, *values = nullptr;  // [slots][layers][capacity][kw | vw]
    float *kscale = nullptr, *vscale = nullptr;  // [slots][layers][capacity][kv]
    float *ehist[2] = {nullptr, nullptr};        // [sites][slots][9][dim], current / scratch
    float *rope_cos = nullptr, *rope_sin = nullptr;  // [capacity][qk / 2]
    // step buffers
    int32_t *d_rows = nullptr;  // tokens, slots, heads [max_rows] each
    int32_t *h_rows = nullptr;  // pinned staging
    cudaEvent_t rows_copied = nullptr;  // the last forward's staging copy (h_rows is free once it has run)
    float *gathered, *stream, *next, *u, *residual, *norm4, *pre, *post, *res, *hpre, *post_gate, *mix_logits, *mix;
    const int32_t *perm_a = nullptr, *perm_b = nullptr;  // the model's HadamardMlp permutations (device)
    int hada_rows = 0, hada_cols = 0;
    float *quarters, *gate_rows, *q, *k, *v, *gate, *qc, *kc, *vc, *attn_out, *proj, *mean, *headn;
    float *head_logits;  // [max_heads][vocab] of one wave
    int8_t *act_values = nullptr, *q8 = nullptr;
    float *act_scales = nullptr, *act_offsets = nullptr, *qs = nullptr;
    int act_stride = 0;
    void *engram_ws = nullptr;
    size_t engram_ws_bytes = 0;
    std::vector<int> host_len, host_mark;
    // each slot's state at its mark (MarkSlot / RewindSlot): conv and Engram histories, previous tokens
    float *snap_conv = nullptr, *snap_ehist = nullptr;
    int32_t *snap_prev = nullptr;
    int pool_rows = 0;  // the confidence head's pool rows the reference's state carries (this engine does not pool)
    // captured single-wave forwards (every row a distinct slot, head rows in order), keyed by (rows, heads)
    struct WaveGraph {
        int rows, heads;
        cudaGraphExec_t exec;
    };
    std::vector<WaveGraph> graphs;
};

namespace {

template <typename T>
int n3_alloc(N3State *s, T **p, size_t count) {
    void *raw = nullptr;
    cudaError_t e = cudaMalloc(&raw, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return set_error(NDL_ERR_OUT_OF_MEMORY, "Needle-3 state: %s", cudaGetErrorString(e));
    s->allocations.push_back(raw);
    *p = static_cast<T *>(raw);
    return NDL_OK;
}

int cq_view(const ndl_model *m, const char *role, int index, CqView *v) {
    ndl_model_tensor t;
    int st = ndl_model_get_tensor(m, role, index, &t);
    if (st != NDL_OK) return st;
    if (t.kind != NDL_TENSOR_CQ && t.kind != NDL_TENSOR_CQ_ROWS)
        return set_error(NDL_ERR_UNSUPPORTED, "%s %d is not a CQ matrix", role, index);
    *v = CqView{t.indices, t.norms, t.book, t.rows, t.cols, t.bits};
    return NDL_OK;
}

int dense_view(const ndl_model *m, const char *role, int index, int64_t need, const float **out) {
    ndl_model_tensor t;
    int st = ndl_model_get_tensor(m, role, index, &t);
    if (st != NDL_OK) return st;
    if (t.kind != NDL_TENSOR_DENSE || t.count < need)
        return set_error(NDL_ERR_UNSUPPORTED, "%s %d: %lld values, %lld needed", role, index, (long long)t.count,
                         (long long)need);
    *out = t.values;
    return NDL_OK;
}

// ---------------------------------------------------------------- kernels --

// x += x * (sqrt(dim) - 1) (AddScaled, src/Needle/Scalar.cs:275-278: a
// rounded product, then a rounded sum), copied to the row's four streams.
__global__ void n3_embed_kernel(const float *__restrict__ x, int rows, int dim, float scale,
                                float *__restrict__ stream) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * dim) return;
    const int r = (int)(i / dim), c = (int)(i - (long long)r * dim);
    const float v = __fadd_rn(x[i], __fmul_rn(scale, x[i]));
#pragma unroll
    for (int l = 0; l < kLanes; l++) stream[((size_t)r * kLanes + l) * dim + c] = v;
}

// The 3-tap convs of the projections (ChainTriple, src/Needle/Engine.cs:
// 2471-2478, and Scalar.Taps3, src/Needle/Scalar.cs:285-288): per row and
// column of q | k | v, the triple (x_{t-2}, x_{t-1}, x_t) from the slot's two
// previous projections, out = taps[c] x_t + taps[w + c] x_{t-1} + taps[2w + c]
// x_{t-2} in that order, and the history becomes (x_{t-1}, x_t).  Thread per
// (row, column).
__global__ void n3_conv_kernel(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                               const int32_t *__restrict__ row_slots, int rows, int layer, int layers, int qw, int kw,
                               int vw, const float *__restrict__ q_taps, const float *__restrict__ k_taps,
                               const float *__restrict__ v_taps, float *__restrict__ hist, float *__restrict__ qc,
                               float *__restrict__ kc, float *__restrict__ vc) {
    pdl_enter();
    const int width = qw + kw + vw;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * width) return;
    const int r = (int)(i / width), c = (int)(i - (long long)r * width);
    const int slot = row_slots[r];
    float *h = hist + ((size_t)slot * layers + layer) * kConvHist * width;
    float cur;
    int w, cc;
    const float *taps;
    float *dst;
    if (c < qw) {
        cc = c, cur = q[(size_t)r * qw + cc], w = qw, taps = q_taps, dst = qc + (size_t)r * qw;
    } else if (c < qw + kw) {
        cc = c - qw, cur = k[(size_t)r * kw + cc], w = kw, taps = k_taps, dst = kc + (size_t)r * kw;
    } else {
        cc = c - qw - kw, cur = v[(size_t)r * vw + cc], w = vw, taps = v_taps, dst = vc + (size_t)r * vw;
    }
    // history layout per slot and layer: [2][q | k | v] as QkvOf (q history both entries, then k, then v)
    float *hq = h + (c < qw ? 0 : c < qw + kw ? kConvHist * qw : kConvHist * (qw + kw));
    const float h0 = hq[cc], h1 = hq[w + cc];
    const float acc = __fadd_rn(__fmul_rn(taps[cc], cur), __fmul_rn(taps[w + cc], h1));
    dst[cc] = __fadd_rn(acc, __fmul_rn(taps[2 * w + cc], h0));
    hq[cc] = h1;
    hq[w + cc] = cur;
}

__device__ __forceinline__ float n3_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 1 / sqrt(SumOfSquares(x, n) / n + 1e-6) (Ops.InverseRms over
// Scalar.SumOfSquares): the sum left to right on lane 0.
__device__ float n3_inverse_rms(const float *x, int n, int lane) {
    float inv = 0.0f;
    if (lane == 0) {
        float sum = 0.0f;
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), 1e-6f)));
    }
    return __shfl_sync(0xffffffffu, inv, 0);
}

// Scalar.QuantizeInt8 of x[0..n) (n <= 64, lane holds i = lane, lane + 32)
// into dst; returns the scale.
__device__ float n3_quantize(const float *x, int n, int8_t *dst, int lane) {
    float peak = 0.0f;
    for (int i = lane; i < n; i += 32) peak = fmaxf(peak, fabsf(x[i]));
    peak = n3_warp_max(peak);
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    for (int i = lane; i < n; i += 32) dst[i] = (int8_t)fminf(fmaxf(rintf(__fmul_rn(x[i], inverse)), -128.0f), 127.0f);
    return scale;
}

// Per row and head (q heads, then kv heads) after the convs
// (RunAttentionBatch, src/Needle/Engine.cs:2569-2583): ZeroCenteredRms with
// q_norm / k_norm, RoPE at the row's position (half-split, Scalar.Rope), then
// QuantizeInt8 of q per head, and of k and v per kv head into the slot's cache
// at that position.  Warp per (row, head); the head's values pass through the
// warp's shared scratch.
__global__ void __launch_bounds__(32 * kN3Warps) n3_qkv_post_kernel(
    float *__restrict__ qc, float *__restrict__ kc, const float *__restrict__ vc, const int32_t *__restrict__ row_slots,
    const int32_t *__restrict__ len, int rows, int heads, int kv, int qk, int vd, const float *__restrict__ q_norm,
    const float *__restrict__ k_norm, const float *__restrict__ rope_cos, const float *__restrict__ rope_sin,
    int layer, int layers, int capacity, int8_t *__restrict__ q8, float *__restrict__ qs, int8_t *__restrict__ keys,
    float *__restrict__ kscale, int8_t *__restrict__ values, float *__restrict__ vscale) {
    pdl_enter();
    __shared__ float buf[kN3Warps][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * kN3Warps + warp;
    if (item >= rows * (heads + kv)) return;
    const int r = item / (heads + kv), h = item - r * (heads + kv);
    const int slot = row_slots[r], p = len[slot];
    const bool is_q = h < heads;
    const int hh = is_q ? h : h - heads;
    float *x = is_q ? qc + (size_t)r * heads * qk + hh * qk : kc + (size_t)r * kv * qk + hh * qk;
    const float *scale = is_q ? q_norm : k_norm;
    float *b = buf[warp];
    for (int i = lane; i < qk; i += 32) b[i] = x[i];
    __syncwarp();
    const float inv = n3_inverse_rms(b, qk, lane);
    __syncwarp();
    for (int i = lane; i < qk; i += 32) b[i] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, scale[i]), b[i]), inv);
    __syncwarp();
    const int half = qk / 2;
    const float *cs = rope_cos + (size_t)p * half, *sn = rope_sin + (size_t)p * half;
    float lo = 0.0f, hi = 0.0f;
    if (lane < half) {
        const float a = b[lane], bb = b[lane + half];
        lo = __fsub_rn(__fmul_rn(a, cs[lane]), __fmul_rn(bb, sn[lane]));
        hi = __fadd_rn(__fmul_rn(bb, cs[lane]), __fmul_rn(a, sn[lane]));
    }
    __syncwarp();
    if (lane < half) {
        b[lane] = lo;
        b[lane + half] = hi;
    }
    __syncwarp();
    if (is_q) {
        const float s = n3_quantize(b, qk, q8 + (size_t)r * heads * qk + hh * qk, lane);
        if (lane == 0) qs[(size_t)r * heads + hh] = s;
        return;
    }
    const size_t at = ((size_t)slot * layers + layer) * capacity + p;
    const float ks = n3_quantize(b, qk, keys + at * kv * qk + hh * qk, lane);
    if (lane == 0) kscale[at * kv + hh] = ks;
    __syncwarp();
    const float *vx = vc + (size_t)r * kv * vd + hh * vd;
    for (int i = lane; i < vd; i += 32) b[i] = vx[i];
    __syncwarp();
    const float vs = n3_quantize(b, vd, values + at * kv * vd + hh * vd, lane);
    if (lane == 0) vscale[at * kv + hh] = vs;
}

// Scalar.AttentionHead (src/Needle/Scalar.cs:290-312) for grouped heads:
// warp per (row, q head) over positions [first, p] of the slot's cache (kv
// head = head / (heads / kv)): s_j = (dot_j * ks_j) * (qs / sqrt(qk)); the
// softmax as Ops.Softmax's scalar form (maximum, e_j = MathF.Exp(s_j - max)
// summed in position order, p_j = e_j / total); out[d] += (p_j * vs_j) *
// v_j[d] in position order, two dims per lane.  Scores live in the warp's
// shared slice [capacity].
__global__ void __launch_bounds__(32 * kN3Warps) n3_attention_kernel(
    const int8_t *__restrict__ q8, const float *__restrict__ qs, const int32_t *__restrict__ row_slots,
    const int32_t *__restrict__ len, int rows, int heads, int kv, int qk, int vd, int layer, int layers, int capacity,
    int window, float inv_sqrt, const int8_t *__restrict__ keys, const float *__restrict__ kscale,
    const int8_t *__restrict__ values, const float *__restrict__ vscale, float *__restrict__ out) {
    pdl_enter();
    extern __shared__ float n3_scores[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * kN3Warps + warp;
    if (item >= rows * heads) return;
    float *sc = n3_scores + (size_t)warp * capacity;
    const int r = item / heads, h = item - r * heads;
    const int slot = row_slots[r], p = len[slot];
    const int first = window == 0 ? 0 : max(0, p - window + 1);
    const int group = heads / kv, kh = h / group;
    // the query as int32 words (qk % 4 == 0, rows on 4-byte boundaries): dp4a gives the exact int32 dot
    const int words = qk / 4;
    int qw[16];
    const int *qrow = reinterpret_cast<const int *>(q8 + (size_t)r * heads * qk + h * qk);
#pragma unroll
    for (int i = 0; i < 16; i++) qw[i] = i < words ? qrow[i] : 0;
    const float scale = __fmul_rn(qs[(size_t)r * heads + h], inv_sqrt);
    const size_t base = ((size_t)slot * layers + layer) * capacity;
    float peak = -INFINITY;
    for (int j = first + lane; j <= p; j += 32) {
        const int *kr = reinterpret_cast<const int *>(keys + (base + j) * kv * qk + kh * qk);
        int dot = 0;
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < words) dot = __dp4a(kr[i], qw[i], dot);
        const float s = __fmul_rn(__fmul_rn(__int2float_rn(dot), kscale[(base + j) * kv + kh]), scale);
        sc[j - first] = s;
        peak = fmaxf(peak, s);
    }
    peak = n3_warp_max(peak);
    const int count = p - first + 1;
    for (int j = lane; j < count; j += 32) sc[j] = exp_rn(__fsub_rn(sc[j], peak));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0)
        for (int j = 0; j < count; j++) total = __fadd_rn(total, sc[j]);
    total = __shfl_sync(0xffffffffu, total, 0);
    // p_j = e_j / total, then the PV weight p_j * vs_j, per position
    for (int j = lane; j < count; j += 32)
        sc[j] = __fmul_rn(__fdiv_rn(sc[j], total), vscale[(base + first + j) * kv + kh]);
    __syncwarp();
    const int8_t *vb = values + (base + first) * kv * vd + kh * vd;
    const size_t vstride = (size_t)kv * vd;
    for (int d0 = lane; d0 < vd; d0 += 64) {  // dims d0 and d0 + 32 side by side
        const int d1 = d0 + 32;
        const bool has1 = d1 < vd;
        float a0 = 0.0f, a1 = 0.0f;
        int j = 0;
        for (; j + 8 <= count; j += 8) {
            float w8[8], v0[8], v1[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                w8[u] = sc[j + u];
                v0[u] = (float)vb[(size_t)(j + u) * vstride + d0];
                v1[u] = has1 ? (float)vb[(size_t)(j + u) * vstride + d1] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                a0 = __fadd_rn(a0, __fmul_rn(w8[u], v0[u]));
                a1 = __fadd_rn(a1, __fmul_rn(w8[u], v1[u]));
            }
        }
        for (; j < count; j++) {
            a0 = __fadd_rn(a0, __fmul_rn(sc[j], (float)vb[(size_t)j * vstride + d0]));
            if (has1) a1 = __fadd_rn(a1, __fmul_rn(sc[j], (float)vb[(size_t)j * vstride + d1]));
        }
        float *o = out + (size_t)r * heads * vd + h * vd;
        o[d0] = a0;
        if (has1) o[d1] = a1;
    }
}

// The head rows' 4-stream rows: dst[h] = src[rows[h]] (width floats each).
__global__ void n3_pick_rows_kernel(const float *__restrict__ src, int width, const int32_t *__restrict__ rows,
                                    int n, float *__restrict__ dst) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * width) return;
    const int h = (int)(i / width), c = (int)(i - (long long)h * width);
    dst[i] = src[(size_t)rows[h] * width + c];
}

// The slots' previous two tokens and lengths after a forward (ForwardBatch,
// src/Needle/Engine.cs:2327-2340), one thread per row (distinct slots).
__global__ void n3_advance_kernel(const int32_t *__restrict__ tokens, const int32_t *__restrict__ row_slots, int rows,
                                  int32_t *__restrict__ prev, int32_t *__restrict__ len) {
    pdl_enter();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int s = row_slots[r];
    prev[2 * s] = prev[2 * s + 1];
    prev[2 * s + 1] = tokens[r];
    len[s] += 1;
}

// EngineCore.RopeFrequencies + BuildRopeTables (src/Needle/Engine.cs:336-356)
// on the host, as the synthetic decoder's tables.
void rope_tables(float theta, int qk, int positions, std::vector<float> &cs, std::vector<float> &sn) {
    const int half = qk / 2;
    std::vector<float> freq(half);
    for (int i = 0; i < half; i++) freq[i] = 1.0f / powf(theta, 2.0f * (float)i / (float)qk);
    cs.resize((size_t)positions * half);
    sn.resize((size_t)positions * half);
    for (int p = 0; p < positions; p++)
        for (int i = 0; i < half; i++) {
            const float angle = (float)p * freq[i];
            cs[(size_t)p * half + i] = cosf(angle);
            sn[(size_t)p * half + i] = sinf(angle);
        }
}

int cq_matmul(const CqView &w, const N3State *s, int tokens, int row_start, int row_end, float *y, int ldy,
              cudaStream_t st) {
    return ndl_cq_matmul(w.indices, w.norms, w.book->bytes, w.book->byte_scale, w.rows, w.cols, w.bits, s->act_values,
                         s->act_scales, s->act_offsets, s->act_stride, tokens, y, ldy, row_start, row_end, st);
}
int cq_prepare(N3State *s, const float *x, int tokens, int cols, int bits, cudaStream_t st);
// A fake-A8 row op (modes 0..2) and the CQ Prepare of its output: one
// launch where the width allows, else the two steps through `tmp`.
int fake_a8_prepare(N3State *s, int mode, const float *x, const float *aux, int rows, int n, int bits, float *tmp,
                    cudaStream_t st) {
    const int rc = launch_fake_a8_prepare(mode, x, aux, rows, n, bits, s->act_values, s->act_scales, s->act_offsets,
                                          s->act_stride, st);
    if (rc != NDL_ERR_UNSUPPORTED) return rc;
    const int rc2 = ndl_fake_a8_rows(mode, x, aux, nullptr, rows, n, tmp, st);
    return rc2 != NDL_OK ? rc2 : cq_prepare(s, tmp, rows, n, bits, st);
}
// Matrices of one width over the current Prepare in as few launches as
// their bits allow (the layer's projections share one activation Prepare).
int cq_matmuls(const N3State *s, int tokens, const CqView *const *views, const CqMatmulJob *jobs, int n,
               cudaStream_t st) {
    bool same = true;
    for (int i = 1; i < n; i++) same = same && views[i]->bits == views[0]->bits && views[i]->cols == views[0]->cols;
    for (int i = 0; i < n; i += same ? n : 1) {
        const int st_ = launch_cq_matmul_jobs(jobs + i, same ? n : 1, views[i]->cols, views[i]->bits, s->act_values,
                                              s->act_scales, s->act_offsets, s->act_stride, tokens, st);
        if (st_ != NDL_OK) return st_;
    }
    return NDL_OK;
}
CqMatmulJob cq_job(const CqView &w, int row_start, int row_end, float *y, int ldy) {
    return CqMatmulJob{w.indices, w.norms, w.book->bytes, w.book->byte_scale, y, ldy, row_start, row_end};
}
int cq_prepare(N3State *s, const float *x, int tokens, int cols, int bits, cudaStream_t st) {
    return ndl_cq_prepare(x, tokens, cols, bits, s->act_values, s->act_scales, s->act_offsets, s->act_stride, st);
}

#define N3_TRY(x)                     \
    do {                              \
        int st_ = (x);                \
        if (st_ != NDL_OK) return st_; \
    } while (0)

// One forward over `rows` rows of distinct slots (device arrays in s->d_rows:
// tokens, slots, head rows); logits [heads][vocab].
// One forward over `rows` rows of distinct slots (device arrays tokens,
// slots [rows] and head_rows [heads], rows of this forward); logits
// [heads][vocab].
int forward_wave(N3State *s, const int32_t *tokens, const int32_t *slots, const int32_t *head_rows, int rows,
                 int heads, float *logits, cudaStream_t st) {
    const int d = s->dim, R = rows;
    N3_TRY(ndl_cq_gather_rows(s->embedding.indices, s->embedding.norms, s->embedding.book->levels, s->embedding.rows,
                              s->embedding.cols, s->embedding.bits, tokens, R, s->gathered, st));
    {
        const float scale = sqrtf((float)d) - 1.0f;
        const long long n = (long long)R * d;
        launch_kernel(n3_embed_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, s->gathered, R, d, scale,
                      s->stream);
        N3_TRY(check_launch("n3_embed"));
    }
    const int sw = kLanes * d;
    for (int l = 0; l < s->layers; l++) {
        const LayerView &L = s->layer[l];
        // hyper-connection prepare, phi matmuls, gates, Mix4, Sinkhorn
        N3_TRY(fake_a8_prepare(s, 0, s->stream, nullptr, R, sw, s->phi_pre.bits, s->norm4, st));
        // the layer's row slices of the phi matrices, into columns [4l, 4l + 4) / [16l, 16l + 16)
        {
            const CqView *views[3] = {&s->phi_pre, &s->phi_post, &s->phi_res};
            const CqMatmulJob jobs[3] = {
                cq_job(s->phi_pre, l * kLanes, l * kLanes + kLanes, s->pre, s->phi_pre.rows),
                cq_job(s->phi_post, l * kLanes, l * kLanes + kLanes, s->post, s->phi_post.rows),
                cq_job(s->phi_res, l * 16, l * 16 + 16, s->res, s->phi_res.rows)};
            N3_TRY(cq_matmuls(s, R, views, jobs, 3, st));
        }
        N3_TRY(launch_hc_prepare(s->pre, s->phi_pre.rows, s->post, s->phi_post.rows, s->res, s->phi_res.rows, s->a_pre,
                                 s->b_pre, s->a_post, s->b_post, s->a_res, s->b_res, l, s->stream, d, R, s->u,
                                 s->residual, s->post_gate, s->mix, st));
        // Engram
        const int site = s->site_of_layer[l];
        if (site >= 0) {
            float *cur = s->ehist[0] + (size_t)site * s->slots * kEngramHistory * d;
            float *nxt = s->ehist[1] + (size_t)site * s->slots * kEngramHistory * d;
            NDL_CUDA(cudaMemcpyAsync(nxt, cur, (size_t)s->slots * kEngramHistory * d * 4, cudaMemcpyDeviceToDevice, st));
            N3_TRY(ndl_engram_apply(s->model, site, tokens, slots, R, s->len, s->prev, s->slots, cur, nxt, s->u,
                                    s->residual, s->engram_ws, s->engram_ws_bytes, st));
            NDL_CUDA(cudaMemcpyAsync(cur, nxt, (size_t)s->slots * kEngramHistory * d * 4, cudaMemcpyDeviceToDevice, st));
        }
        // attention: prepare, projections, convs, per-head norms / RoPE / quantize, attention, gate, out, post-norm
        N3_TRY(fake_a8_prepare(s, 1, s->residual, L.norm_in, R, d, L.q.bits, s->norm4, st));
        {
            const CqView *views[4] = {&L.q, &L.k, &L.v, &L.gate};
            const CqMatmulJob jobs[4] = {cq_job(L.q, 0, s->qw, s->q, s->qw), cq_job(L.k, 0, s->kw, s->k, s->kw),
                                         cq_job(L.v, 0, s->vw, s->v, s->vw), cq_job(L.gate, 0, s->ow, s->gate, s->ow)};
            N3_TRY(cq_matmuls(s, R, views, jobs, 4, st));
        }
        {
            const long long n = (long long)R * (s->qw + s->kw + s->vw);
            launch_kernel(n3_conv_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, s->q, s->k, s->v, slots,
                          R, l, s->layers, s->qw, s->kw, s->vw, L.q_taps, L.k_taps, L.v_taps, s->conv_hist, s->qc,
                          s->kc, s->vc);
            N3_TRY(check_launch("n3_conv"));
        }
        {
            const int items = R * (s->heads + s->kv);
            launch_kernel(n3_qkv_post_kernel, dim3((items + kN3Warps - 1) / kN3Warps), dim3(32 * kN3Warps), 0, st,
                          s->qc, s->kc, s->vc, slots, s->len, R, s->heads, s->kv, s->qk, s->vd, L.q_norm, L.k_norm,
                          s->rope_cos, s->rope_sin, l, s->layers, s->capacity, s->q8, s->qs, s->keys, s->kscale,
                          s->values, s->vscale);
            N3_TRY(check_launch("n3_qkv_post"));
        }
        {
            const int items = R * s->heads;
            const size_t smem = (size_t)kN3Warps * s->capacity * sizeof(float);
            static DeviceOnce smem_attribute;  // scores of up to 8192 positions per warp
            N3_TRY(smem_attribute.run([] {
                int dev = 0, optin = 0;
                cudaGetDevice(&dev);
                cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
                cudaError_t e = cudaFuncSetAttribute(n3_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     optin);
                if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "n3 attention smem: %s", cudaGetErrorString(e));
                return (int)NDL_OK;
            }));
            const float inv_sqrt = 1.0f / sqrtf((float)s->qk);
            launch_kernel(n3_attention_kernel, dim3((items + kN3Warps - 1) / kN3Warps), dim3(32 * kN3Warps), smem, st,
                          s->q8, s->qs, slots, s->len, R, s->heads, s->kv, s->qk, s->vd, l, s->layers, s->capacity,
                          L.window, inv_sqrt, s->keys, s->kscale, s->values, s->vscale, s->attn_out);
            N3_TRY(check_launch("n3_attention"));
        }
        N3_TRY(fake_a8_prepare(s, 2, s->attn_out, s->gate, R, s->ow, L.out.bits, s->norm4, st));
        N3_TRY(cq_matmul(L.out, s, R, 0, d, s->proj, d, st));
        // one kernel per row: PostNormAdd(residual, proj, post_norm, sigmoid(attn_gate)) (the layer's gate
        // for every row), the MLP, CombineDiff4x4 into the next streams
        {
            KtMlpArgs a{};
            for (int k = 0; k < 13; k++) a.w[k] = L.mlp[k];
            a.pre_norm = L.pre_hada;
            a.perm_a = s->perm_a;
            a.perm_b = s->perm_b;
            a.dim = d;
            a.rows = s->hada_rows;
            a.cols = s->hada_cols;
            a.scale = 1.0f;
            a.residual = s->residual;
            a.row_stride = d;
            a.pn_x = s->proj;
            a.pn_scale = L.post_norm;
            a.pn_gate = s->gate_rows + (size_t)l * s->max_rows;
            a.cb_stream = s->stream;
            a.cb_mix = s->mix;
            a.cb_u = s->u;
            a.cb_post = s->post_gate;
            a.cb_next = s->next;
            N3_TRY(launch_mlp_rows(a, R, st));
        }
        std::swap(s->stream, s->next);
    }
    launch_kernel(n3_advance_kernel, dim3((R + 127) / 128), dim3(128), 0, st, tokens, slots, R, s->prev, s->len);
    N3_TRY(check_launch("n3_advance"));
    if (heads > 0) {
        // PrepareHeadVectors (src/Needle/Engine.cs:921-929) for the head rows
        launch_kernel(n3_pick_rows_kernel, dim3((unsigned)(((long long)heads * kLanes * d + 255) / 256)), dim3(256), 0,
                      st, (const float *)s->stream, kLanes * d, head_rows, heads, s->headn);
        N3_TRY(check_launch("n3_pick_rows"));
        N3_TRY(ndl_hc_mix4(s->headn, d, s->quarters, heads, s->mean, st));
        N3_TRY(fake_a8_prepare(s, 1, s->mean, s->final_norm, heads, d, s->embedding.bits, s->headn, st));
        N3_TRY(cq_matmul(s->embedding, s, heads, 0, s->embedding.rows, logits, s->embedding.rows, st));
    }
    return NDL_OK;
}

}  // namespace

// A single-wave forward (rows of distinct slots, staged at d_rows) replayed
// from a CUDA graph per (rows, heads); the first call of a shape captures it.
static int launch_wave_graph(N3State *s, int rows, int heads, float *logits, cudaStream_t st) {
    for (auto &g : s->graphs)
        if (g.rows == rows && g.heads == heads) {
            NDL_CUDA(cudaGraphLaunch(g.exec, st));
            return NDL_OK;
        }
    cudaGraph_t graph = nullptr;
    NDL_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = forward_wave(s, s->d_rows, s->d_rows + rows, s->d_rows + 2 * rows, rows, heads, logits, st);
    cudaError_t end = cudaStreamEndCapture(st, &graph);
    if (rc != NDL_OK || end != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        if (rc != NDL_OK) return rc;
        return set_error(NDL_ERR_CUDA, "Needle-3 step capture: %s", cudaGetErrorString(end));
    }
    cudaGraphExec_t exec = nullptr;
    cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) return set_error(NDL_ERR_CUDA, "Needle-3 step graph: %s", cudaGetErrorString(inst));
    if (s->graphs.size() >= 16) {  // keep the 16 latest shapes
        cudaGraphExecDestroy(s->graphs.front().exec);
        s->graphs.erase(s->graphs.begin());
    }
    s->graphs.push_back({rows, heads, exec});
    NDL_CUDA(cudaGraphLaunch(exec, st));
    return NDL_OK;
}

// ForwardBatch over rows whose runs (consecutive rows of one slot) become
// waves: wave w holds the w-th row of every run, so each wave's rows are
// distinct slots and a run's rows go in order.  All waves' rows are staged
// in one copy; the head rows' logits land in `logits` [heads][vocab] in the
// caller's order.
int n3_forward(N3State *s, cudaStream_t st, const int *tokens, const int *row_slots, int rows, const int *head_rows,
               int heads, float *logits) {
    const int V = s->embedding.rows;
    std::vector<int> wave(rows), index(rows);
    int waves = 0;
    for (int r = 0; r < rows; r++) {
        const int slot = row_slots[r];
        if (slot < 0 || slot >= s->slots) return set_error(NDL_ERR_INVALID_ARG, "row %d: slot %d", r, slot);
        if (tokens[r] < 0 || tokens[r] >= V) return set_error(NDL_ERR_INVALID_ARG, "row %d: token %d", r, tokens[r]);
        const bool cont = r > 0 && row_slots[r - 1] == slot;
        if (!cont)
            for (int q = 0; q < r; q++)
                if (row_slots[q] == slot) return set_error(NDL_ERR_INVALID_ARG, "slot %d rows are not consecutive", slot);
        wave[r] = cont ? wave[r - 1] + 1 : 0;
        if (s->host_len[slot] + wave[r] >= s->capacity)
            return set_error(NDL_FAIL_CONTEXT_EXHAUSTED, "slot %d: context capacity %d exceeded", slot, s->capacity);
        waves = std::max(waves, wave[r] + 1);
    }
    for (int h = 0; h < heads; h++)
        if (head_rows[h] < 0 || head_rows[h] >= rows) return set_error(NDL_ERR_INVALID_ARG, "head row %d", head_rows[h]);
    // staging: per wave its tokens, then its slots, then its head rows (indices within the wave); the
    // previous forward's copy out of h_rows must have run before it is rewritten
    NDL_CUDA(cudaEventSynchronize(s->rows_copied));
    int32_t *h = s->h_rows;
    std::vector<int> start(waves + 1, 0), hstart(waves + 1, 0), head_dst;
    int at = 0;
    for (int w = 0; w < waves; w++) {
        start[w] = at;
        for (int r = 0; r < rows; r++)
            if (wave[r] == w) {
                h[at] = tokens[r];
                h[rows + at] = row_slots[r];
                index[r] = at - start[w];
                at++;
            }
    }
    start[waves] = at;
    int hat = 0;
    for (int w = 0; w < waves; w++) {
        hstart[w] = hat;
        for (int j = 0; j < heads; j++)
            if (wave[head_rows[j]] == w) {
                h[2 * rows + hat++] = index[head_rows[j]];
                head_dst.push_back(j);
            }
    }
    hstart[waves] = hat;
    NDL_CUDA(cudaMemcpyAsync(s->d_rows, h, (size_t)(2 * rows + heads) * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    NDL_CUDA(cudaEventRecord(s->rows_copied, st));
    bool in_order = waves == 1;
    for (int k = 0; k < heads && in_order; k++) in_order = head_dst[k] == k;
    if (in_order) {
        // a decode step: one wave, the logits straight into place, from a captured graph; the call returns
        // without waiting, so forwards of several engines run side by side
        N3_TRY(launch_wave_graph(s, rows, heads, logits, st));
        for (int r = 0; r < rows; r++) s->host_len[row_slots[r]]++;
        return NDL_OK;
    }
    for (int w = 0; w < waves; w++) {
        const int n = start[w + 1] - start[w], nh = hstart[w + 1] - hstart[w];
        N3_TRY(forward_wave(s, s->d_rows + start[w], s->d_rows + rows + start[w], s->d_rows + 2 * rows + hstart[w], n,
                            nh, s->head_logits, st));
        for (int k = 0; k < nh; k++)
            NDL_CUDA(cudaMemcpyAsync(logits + (size_t)head_dst[hstart[w] + k] * V, s->head_logits + (size_t)k * V,
                                     (size_t)V * 4, cudaMemcpyDeviceToDevice, st));
    }
    for (int r = 0; r < rows; r++) s->host_len[row_slots[r]]++;
    // the staging buffer is reused by the next call: its copy must have run
    NDL_CUDA(cudaStreamSynchronize(st));
    return NDL_OK;
}

int n3_reset_slot(N3State *s, int slot, cudaStream_t st) {
    if (slot < 0 || slot >= s->slots) return set_error(NDL_ERR_INVALID_ARG, "slot %d", slot);
    const int L = s->layers, width = s->qw + s->kw + s->vw, d = s->dim;
    NDL_CUDA(cudaMemsetAsync(s->len + slot, 0, 4, st));
    NDL_CUDA(cudaMemsetAsync(s->prev + 2 * slot, 0, 8, st));
    NDL_CUDA(cudaMemsetAsync(s->conv_hist + (size_t)slot * L * kConvHist * width, 0,
                             (size_t)L * kConvHist * width * 4, st));
    for (int site = 0; site < s->sites; site++)
        NDL_CUDA(cudaMemsetAsync(s->ehist[0] + ((size_t)site * s->slots + slot) * kEngramHistory * d, 0,
                                 (size_t)kEngramHistory * d * 4, st));
    s->host_len[slot] = 0;
    s->host_mark[slot] = 0;
    return n3_mark(s, slot, st);  // the reset state is also the mark's
}

int n3_slot_length(const N3State *s, int slot) { return s->host_len[slot]; }

// The slot's live (or snapshot) histories: conv [L][2][width], each site's
// Engram [9][dim], previous tokens [2], copied one way or the other.
static int copy_state(N3State *s, int slot, bool to_snapshot, cudaStream_t st) {
    const int L = s->layers, width = s->qw + s->kw + s->vw, d = s->dim;
    const size_t conv = (size_t)L * kConvHist * width;
    float *live_c = s->conv_hist + (size_t)slot * conv, *snap_c = s->snap_conv + (size_t)slot * conv;
    NDL_CUDA(cudaMemcpyAsync(to_snapshot ? snap_c : live_c, to_snapshot ? live_c : snap_c, conv * 4,
                             cudaMemcpyDeviceToDevice, st));
    for (int site = 0; site < s->sites; site++) {
        const size_t at = ((size_t)site * s->slots + slot) * kEngramHistory * d;
        NDL_CUDA(cudaMemcpyAsync(to_snapshot ? s->snap_ehist + at : s->ehist[0] + at,
                                 to_snapshot ? s->ehist[0] + at : s->snap_ehist + at, (size_t)kEngramHistory * d * 4,
                                 cudaMemcpyDeviceToDevice, st));
    }
    NDL_CUDA(cudaMemcpyAsync(to_snapshot ? s->snap_prev + 2 * slot : s->prev + 2 * slot,
                             to_snapshot ? s->prev + 2 * slot : s->snap_prev + 2 * slot, 8, cudaMemcpyDeviceToDevice,
                             st));
    return NDL_OK;
}

__global__ void n3_set_length_kernel(int32_t *len, int slot, int value) { len[slot] = value; }

// MarkView (src/Needle/Engine.cs:2235-2244): the histories and previous
// tokens as they are now, and the length.
int n3_mark(N3State *s, int slot, cudaStream_t st) {
    if (slot < 0 || slot >= s->slots) return set_error(NDL_ERR_INVALID_ARG, "slot %d", slot);
    N3_TRY(copy_state(s, slot, true, st));
    s->host_mark[slot] = s->host_len[slot];
    return NDL_OK;
}

// RewindView (:2246-2255): back to the mark's histories, previous tokens and
// length (cache positions past it are rewritten by later forwards).
int n3_rewind(N3State *s, int slot, cudaStream_t st) {
    if (slot < 0 || slot >= s->slots) return set_error(NDL_ERR_INVALID_ARG, "slot %d", slot);
    N3_TRY(copy_state(s, slot, false, st));
    s->host_len[slot] = s->host_mark[slot];
    n3_set_length_kernel<<<1, 1, 0, st>>>(s->len, slot, s->host_mark[slot]);
    return check_launch("n3_set_length");
}

int n3_slot_mark(const N3State *s, int slot) { return s->host_mark[slot]; }

// Engine.PrimedPrefixBytes (src/Needle/Engine.cs:398-400) for a marked length:
// int32 length, the state (stateBytes: conv histories, Engram histories,
// previous tokens, the confidence pools), then per layer the cache rows.
size_t n3_prefix_bytes(const N3State *s, int len) {
    const size_t width = (size_t)s->qw + s->kw + s->vw;
    const size_t state = ((size_t)s->layers * kConvHist * width + (size_t)s->sites * kEngramHistory * s->dim + 2 +
                          (size_t)s->pool_rows * (s->dim + 2)) * 4;
    return 4 + state + (size_t)s->layers * len * (s->kw + s->vw + 2 * (size_t)s->kv * 4);
}

// ExportPrimedPrefix / ImportPrimedPrefix (src/Needle/Engine.cs:402-464) on
// one slot: the state section is the slot's marked state (the pools at their
// reset values: this engine keeps no confidence pools), then for each layer
// the first `len` cache positions: keys [len][kw], values [len][vw], key and
// value scales [len][kv].  Each piece is one copy between host and device.
int n3_prefix_move(N3State *s, int slot, bool to_blob, uint8_t *blob, int len, cudaStream_t st) {
    const int L = s->layers, width = s->qw + s->kw + s->vw, d = s->dim;
    const cudaMemcpyKind kind = to_blob ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice;
    auto move = [&](void *dev, uint8_t *host, size_t bytes) -> int {
        if (bytes == 0) return NDL_OK;
        cudaError_t e = to_blob ? cudaMemcpyAsync(host, dev, bytes, kind, st) : cudaMemcpyAsync(dev, host, bytes, kind, st);
        return e == cudaSuccess ? NDL_OK : set_error(NDL_ERR_CUDA, "primed prefix copy: %s", cudaGetErrorString(e));
    };
    uint8_t *at = blob + 4;
    const size_t conv = (size_t)L * kConvHist * width;
    // state: the snapshot on export; on import both the live state and the snapshot
    N3_TRY(move(s->snap_conv + (size_t)slot * conv, at, conv * 4));
    at += conv * 4;
    for (int site = 0; site < s->sites; site++) {
        N3_TRY(move(s->snap_ehist + ((size_t)site * s->slots + slot) * kEngramHistory * d, at,
                    (size_t)kEngramHistory * d * 4));
        at += (size_t)kEngramHistory * d * 4;
    }
    N3_TRY(move(s->snap_prev + 2 * slot, at, 8));
    at += 8;
    if (to_blob) {
        float *pool = reinterpret_cast<float *>(at);
        for (int i = 0; i < s->pool_rows; i++) pool[i] = -1e30f;  // ResetView's pool maxima
        memset(pool + s->pool_rows, 0, (size_t)s->pool_rows * (d + 1) * 4);
    }
    at += (size_t)s->pool_rows * (d + 2) * 4;
    for (int l = 0; l < L; l++) {
        const size_t base = ((size_t)slot * L + l) * s->capacity;
        N3_TRY(move(s->keys + base * s->kw, at, (size_t)len * s->kw));
        at += (size_t)len * s->kw;
        N3_TRY(move(s->values + base * s->vw, at, (size_t)len * s->vw));
        at += (size_t)len * s->vw;
        N3_TRY(move(s->kscale + base * s->kv, at, (size_t)len * s->kv * 4));
        at += (size_t)len * s->kv * 4;
        N3_TRY(move(s->vscale + base * s->kv, at, (size_t)len * s->kv * 4));
        at += (size_t)len * s->kv * 4;
    }
    if (!to_blob) {
        N3_TRY(copy_state(s, slot, false, st));  // the live state starts as the blob's
        s->host_len[slot] = s->host_mark[slot] = len;
        n3_set_length_kernel<<<1, 1, 0, st>>>(s->len, slot, len);
        N3_TRY(check_launch("n3_set_length"));
    }
    NDL_CUDA(cudaStreamSynchronize(st));  // the host blob is complete (export) or consumed (import)
    return NDL_OK;
}

int n3_capacity(const N3State *s) { return s->capacity; }

int n3_create(const ndl_model *m, int slots, int capacity, int max_rows, int max_heads, cudaStream_t st,
              N3State **out) {
    *out = nullptr;
    ndl_model_info info;
    N3_TRY(ndl_model_get_info(m, &info));
    if (info.device < 0) return set_error(NDL_ERR_INVALID_ARG, "the model is not on a device");
    if (info.lanes != kLanes) return set_error(NDL_ERR_UNSUPPORTED, "%d hyper-connection lanes (4 supported)", info.lanes);
    if (info.conv_taps != 3) return set_error(NDL_ERR_UNSUPPORTED, "%d conv taps (3 supported)", info.conv_taps);
    if (info.qk_dim > 64 || info.v_dim > 64 || info.qk_dim % 4 != 0)
        return set_error(NDL_ERR_UNSUPPORTED, "head dims %d / %d (at most 64, qk a multiple of 4)", info.qk_dim,
                         info.v_dim);
    if (info.kv_heads < 1 || info.heads % info.kv_heads != 0)
        return set_error(NDL_ERR_UNSUPPORTED, "%d heads over %d kv heads", info.heads, info.kv_heads);
    if (capacity < 1 || capacity > 8192) return set_error(NDL_ERR_UNSUPPORTED, "capacity %d (1..8192)", capacity);
    N3State *s = new N3State();
    s->model = m;
    s->info = info;
    s->slots = slots, s->capacity = capacity, s->max_rows = max_rows, s->max_heads = max_heads;
    s->dim = info.dim, s->heads = info.heads, s->kv = info.kv_heads, s->qk = info.qk_dim, s->vd = info.v_dim;
    s->qw = s->heads * s->qk, s->kw = s->kv * s->qk, s->vw = s->kv * s->vd, s->ow = s->heads * s->vd;
    s->layers = info.layers, s->sites = info.site_count;
    auto fail = [&](int code) {
        n3_destroy(s);
        return code;
    };
    int rc;
    const int d = s->dim, L = s->layers;
    if ((rc = cq_view(m, "embedding", 0, &s->embedding)) != NDL_OK) return fail(rc);
    if ((rc = cq_view(m, "hyper.phi_pre", 0, &s->phi_pre)) != NDL_OK) return fail(rc);
    if ((rc = cq_view(m, "hyper.phi_post", 0, &s->phi_post)) != NDL_OK) return fail(rc);
    if ((rc = cq_view(m, "hyper.phi_res", 0, &s->phi_res)) != NDL_OK) return fail(rc);
    if (s->phi_pre.rows < L * kLanes || s->phi_post.rows < L * kLanes || s->phi_res.rows < L * 16 ||
        s->phi_pre.cols != kLanes * d)
        return fail(set_error(NDL_ERR_UNSUPPORTED, "phi matrices do not cover %d layers", L));
    if ((rc = dense_view(m, "hyper.a_pre", 0, L, &s->a_pre)) != NDL_OK ||
        (rc = dense_view(m, "hyper.b_pre", 0, (int64_t)L * kLanes, &s->b_pre)) != NDL_OK ||
        (rc = dense_view(m, "hyper.a_post", 0, L, &s->a_post)) != NDL_OK ||
        (rc = dense_view(m, "hyper.b_post", 0, (int64_t)L * kLanes, &s->b_post)) != NDL_OK ||
        (rc = dense_view(m, "hyper.a_res", 0, L, &s->a_res)) != NDL_OK ||
        (rc = dense_view(m, "hyper.b_res", 0, (int64_t)L * 16, &s->b_res)) != NDL_OK ||
        (rc = dense_view(m, "final_norm", 0, d, &s->final_norm)) != NDL_OK)
        return fail(rc);
    s->layer.resize(L);
    std::vector<float> gates(L);
    for (int l = 0; l < L; l++) {
        LayerView &v = s->layer[l];
        if ((rc = cq_view(m, "layer.q", l, &v.q)) != NDL_OK || (rc = cq_view(m, "layer.k", l, &v.k)) != NDL_OK ||
            (rc = cq_view(m, "layer.v", l, &v.v)) != NDL_OK || (rc = cq_view(m, "layer.gate", l, &v.gate)) != NDL_OK ||
            (rc = cq_view(m, "layer.out", l, &v.out)) != NDL_OK)
            return fail(rc);
        if (v.q.rows != s->qw || v.k.rows != s->kw || v.v.rows != s->vw || v.gate.rows != s->ow || v.out.rows != d ||
            v.q.cols != d || v.out.cols != s->ow)
            return fail(set_error(NDL_ERR_UNSUPPORTED, "layer %d projection shapes", l));
        if ((rc = dense_view(m, "layer.norm_in", l, d, &v.norm_in)) != NDL_OK ||
            (rc = dense_view(m, "layer.q_taps", l, 3 * (int64_t)s->qw, &v.q_taps)) != NDL_OK ||
            (rc = dense_view(m, "layer.k_taps", l, 3 * (int64_t)s->kw, &v.k_taps)) != NDL_OK ||
            (rc = dense_view(m, "layer.v_taps", l, 3 * (int64_t)s->vw, &v.v_taps)) != NDL_OK ||
            (rc = dense_view(m, "layer.q_norm", l, s->qk, &v.q_norm)) != NDL_OK ||
            (rc = dense_view(m, "layer.k_norm", l, s->qk, &v.k_norm)) != NDL_OK ||
            (rc = dense_view(m, "layer.post_norm", l, d, &v.post_norm)) != NDL_OK)
            return fail(rc);
        float logit = 0.0f;
        if ((rc = ndl_model_read_host(m, "layer.attn_gate", l, &logit, sizeof(float))) != NDL_OK) return fail(rc);
        v.attn_gate = 1.0f / (1.0f + host_exp_rn(-logit));  // Ops.Sigmoid's scalar form
        gates[l] = v.attn_gate;
        v.window = ((info.global_mask >> l) & 1) ? 0 : info.sliding_window;
        static const char *mlp_names[13] = {"layer.mlp.d1",  "layer.mlp.d2",  "layer.mlp.b2",     "layer.mlp.d3",
                                            "layer.mlp.d4",  "layer.mlp.w1a", "layer.mlp.w1b",    "layer.mlp.w2a",
                                            "layer.mlp.w2b", "layer.mlp.w3a", "layer.mlp.w3b",    "layer.mlp.cond_v",
                                            "layer.mlp.cond_u"};
        const int hr = info.hada_rows, hc = info.hada_cols, hw = info.hada_n, in_rows = hc > 0 ? (d + hc - 1) / hc : 0;
        const int64_t mlp_need[13] = {d, hw, hw, hw, d, (int64_t)in_rows * hr, (int64_t)hc * hc, (int64_t)hr * hr,
                                      (int64_t)hc * hc, (int64_t)hr * hr, (int64_t)hc * hc, (int64_t)d * 8, 8LL * hw};
        for (int k = 0; k < 13; k++)
            if ((rc = dense_view(m, mlp_names[k], l, mlp_need[k], &v.mlp[k])) != NDL_OK) return fail(rc);
        if ((rc = dense_view(m, "layer.pre_hada", l, d, &v.pre_hada)) != NDL_OK) return fail(rc);
    }
    {
        ndl_model_tensor t;
        if (ndl_model_get_tensor(m, "hyper.perm_a", 0, &t) != NDL_OK || t.count < info.hada_n) return fail(NDL_ERR_UNSUPPORTED);
        s->perm_a = t.permutation;
        if (ndl_model_get_tensor(m, "hyper.perm_b", 0, &t) != NDL_OK || t.count < info.hada_n) return fail(NDL_ERR_UNSUPPORTED);
        s->perm_b = t.permutation;
        s->hada_rows = info.hada_rows;
        s->hada_cols = info.hada_cols;
        if (info.hada_n <= 0 || (d + info.hada_cols - 1) / info.hada_cols > info.hada_rows)
            return fail(set_error(NDL_ERR_UNSUPPORTED, "HadaN %d cannot hold a %d-wide row", info.hada_n, d));
    }
    s->site_of_layer.assign(L, -1);
    for (int i = 0; i < info.site_count; i++)
        if (info.sites[i] >= 0 && info.sites[i] < L) s->site_of_layer[info.sites[i]] = i;
    const int R = max_rows, H = max_heads, width = s->qw + s->kw + s->vw;
    const int actcols = std::max(kLanes * d, std::max(d, s->ow));
    s->act_stride = ((actcols / 128) + 7) & ~7;
    // device state
    if ((rc = n3_alloc(s, &s->len, slots)) != NDL_OK || (rc = n3_alloc(s, &s->prev, (size_t)slots * 2)) != NDL_OK ||
        (rc = n3_alloc(s, &s->conv_hist, (size_t)slots * L * kConvHist * width)) != NDL_OK ||
        (rc = n3_alloc(s, &s->keys, (size_t)slots * L * capacity * s->kw)) != NDL_OK ||
        (rc = n3_alloc(s, &s->values, (size_t)slots * L * capacity * s->vw)) != NDL_OK ||
        (rc = n3_alloc(s, &s->kscale, (size_t)slots * L * capacity * s->kv)) != NDL_OK ||
        (rc = n3_alloc(s, &s->vscale, (size_t)slots * L * capacity * s->kv)) != NDL_OK ||
        (rc = n3_alloc(s, &s->ehist[0], (size_t)std::max(s->sites, 1) * slots * kEngramHistory * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->ehist[1], (size_t)std::max(s->sites, 1) * slots * kEngramHistory * d)) != NDL_OK)
        return fail(rc);
    {
        std::vector<float> cs, sn;
        rope_tables(info.rope_theta, s->qk, capacity, cs, sn);
        if ((rc = n3_alloc(s, &s->rope_cos, cs.size())) != NDL_OK || (rc = n3_alloc(s, &s->rope_sin, sn.size())) != NDL_OK)
            return fail(rc);
        cudaMemcpy(s->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    }
    // step buffers
    if ((rc = n3_alloc(s, &s->d_rows, (size_t)3 * R)) != NDL_OK ||
        (rc = n3_alloc(s, &s->gathered, (size_t)R * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->stream, (size_t)R * kLanes * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->next, (size_t)R * kLanes * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->u, (size_t)R * d)) != NDL_OK || (rc = n3_alloc(s, &s->residual, (size_t)R * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->norm4, (size_t)R * actcols)) != NDL_OK ||
        (rc = n3_alloc(s, &s->pre, (size_t)R * s->phi_pre.rows)) != NDL_OK ||
        (rc = n3_alloc(s, &s->post, (size_t)R * s->phi_post.rows)) != NDL_OK ||
        (rc = n3_alloc(s, &s->res, (size_t)R * s->phi_res.rows)) != NDL_OK ||
        (rc = n3_alloc(s, &s->hpre, (size_t)R * kLanes)) != NDL_OK ||
        (rc = n3_alloc(s, &s->post_gate, (size_t)R * kLanes)) != NDL_OK ||
        (rc = n3_alloc(s, &s->mix_logits, (size_t)R * 16)) != NDL_OK || (rc = n3_alloc(s, &s->mix, (size_t)R * 16)) != NDL_OK ||
        (rc = n3_alloc(s, &s->quarters, (size_t)R * kLanes)) != NDL_OK ||
        (rc = n3_alloc(s, &s->gate_rows, (size_t)R * L)) != NDL_OK ||
        (rc = n3_alloc(s, &s->head_logits, (size_t)H * info.vocab)) != NDL_OK ||
        (rc = n3_alloc(s, &s->q, (size_t)R * s->qw)) != NDL_OK || (rc = n3_alloc(s, &s->k, (size_t)R * s->kw)) != NDL_OK ||
        (rc = n3_alloc(s, &s->v, (size_t)R * s->vw)) != NDL_OK || (rc = n3_alloc(s, &s->gate, (size_t)R * s->ow)) != NDL_OK ||
        (rc = n3_alloc(s, &s->qc, (size_t)R * s->qw)) != NDL_OK || (rc = n3_alloc(s, &s->kc, (size_t)R * s->kw)) != NDL_OK ||
        (rc = n3_alloc(s, &s->vc, (size_t)R * s->vw)) != NDL_OK ||
        (rc = n3_alloc(s, &s->attn_out, (size_t)R * s->ow)) != NDL_OK ||
        (rc = n3_alloc(s, &s->proj, (size_t)R * d)) != NDL_OK || (rc = n3_alloc(s, &s->mean, (size_t)H * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->headn, (size_t)H * kLanes * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->act_values, (size_t)R * actcols)) != NDL_OK ||
        (rc = n3_alloc(s, &s->act_scales, (size_t)R * s->act_stride)) != NDL_OK ||
        (rc = n3_alloc(s, &s->act_offsets, (size_t)R * s->act_stride)) != NDL_OK ||
        (rc = n3_alloc(s, &s->q8, (size_t)R * s->qw)) != NDL_OK || (rc = n3_alloc(s, &s->qs, (size_t)R * s->heads)) != NDL_OK)
        return fail(rc);
    if ((rc = n3_alloc(s, &s->snap_conv, (size_t)slots * L * kConvHist * width)) != NDL_OK ||
        (rc = n3_alloc(s, &s->snap_ehist, (size_t)std::max(s->sites, 1) * slots * kEngramHistory * d)) != NDL_OK ||
        (rc = n3_alloc(s, &s->snap_prev, (size_t)slots * 2)) != NDL_OK)
        return fail(rc);
    if (info.confidence_head >= 0) {
        ndl_model_tensor pv;
        if (ndl_model_get_tensor(m, "probe.probe_vectors", info.confidence_head, &pv) == NDL_OK && L + 1 > 0)
            s->pool_rows = (pv.rows / (L + 1)) * (L + 1);
    }
    if (cudaEventCreateWithFlags(&s->rows_copied, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        return fail(set_error(NDL_ERR_CUDA, "n3 event"));
    }
    if (cudaMallocHost(&s->h_rows, (size_t)3 * R * sizeof(int32_t)) != cudaSuccess)
        return fail(set_error(NDL_ERR_OUT_OF_MEMORY, "Needle-3 staging"));
    s->engram_ws_bytes = s->sites > 0 ? ndl_engram_workspace(m, R) : 0;
    if (s->engram_ws_bytes > 0) {
        uint8_t *ws = nullptr;
        if ((rc = n3_alloc(s, &ws, s->engram_ws_bytes)) != NDL_OK) return fail(rc);
        s->engram_ws = ws;
    }
    {
        // quarters [R][4] = 0.25 (the head's Mix4); gate_rows [L][R]: each layer's post-norm gate per row
        std::vector<float> q4((size_t)R * kLanes, 0.25f), g((size_t)R * L);
        for (int l = 0; l < L; l++)
            for (int r = 0; r < R; r++) g[(size_t)l * R + r] = gates[l];
        cudaMemcpy(s->quarters, q4.data(), q4.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(s->gate_rows, g.data(), g.size() * 4, cudaMemcpyHostToDevice);
    }
    s->host_len.assign(slots, 0);
    s->host_mark.assign(slots, 0);
    NDL_CUDA(cudaMemsetAsync(s->snap_conv, 0, (size_t)slots * L * kConvHist * width * 4, st));
    NDL_CUDA(cudaMemsetAsync(s->snap_ehist, 0, (size_t)std::max(s->sites, 1) * slots * kEngramHistory * d * 4, st));
    NDL_CUDA(cudaMemsetAsync(s->snap_prev, 0, (size_t)slots * 8, st));
    NDL_CUDA(cudaMemsetAsync(s->len, 0, (size_t)slots * 4, st));
    NDL_CUDA(cudaMemsetAsync(s->prev, 0, (size_t)slots * 8, st));
    NDL_CUDA(cudaMemsetAsync(s->conv_hist, 0, (size_t)slots * L * kConvHist * width * 4, st));
    NDL_CUDA(cudaMemsetAsync(s->ehist[0], 0, (size_t)std::max(s->sites, 1) * slots * kEngramHistory * d * 4, st));
    NDL_CUDA(cudaStreamSynchronize(st));
    *out = s;
    return NDL_OK;
}

void n3_destroy(N3State *s) {
    if (!s) return;
    for (auto &g : s->graphs) cudaGraphExecDestroy(g.exec);
    for (void *p : s->allocations) cudaFree(p);
    if (s->h_rows) cudaFreeHost(s->h_rows);
    if (s->rows_copied) cudaEventDestroy(s->rows_copied);
    delete s;
}

int n3_vocab(const N3State *s) { return s->embedding.rows; }

}  // namespace ndl
