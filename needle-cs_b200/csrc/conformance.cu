// KernelTable-signature conformance exports: the reference's own kernel
// slots (src/Needle/Kernels/KernelTable.cs:5-47, signatures fixed by
// Net10KernelExports.Fill, src/Needle/Kernels/Net10KernelExports.cs:118-150)
// computed on the GPU, host pointers in and out, synchronous.  Installed in a
// KernelTable they let the reference's conformance cases drive the device
// kernels.  Like the slots they replace they have no error channel: a CUDA
// failure returns NaN (scales, probabilities) or -2 (argmax) and leaves the
// reason in ndl_last_error.
#include <initializer_list>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

using namespace ndl;

namespace ndl {
int launch_argmax_masked(const float *x, long long ldx, const uint32_t *mask, int words, long long ldm,
                         const int32_t *mask_index, int length, int rows, int32_t *ids, float *probs,
                         cudaStream_t stream);
int launch_best_probability(const float *x, int count, float best, float *out, cudaStream_t stream);
int launch_cq_prepare(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales, float *offsets,
                      int stride, cudaStream_t stream);
int launch_cq_matmul(const uint8_t *indices, const uint16_t *norms, const uint8_t *book_bytes, float byte_scale,
                     int cols, int bits, const int8_t *values, const float *scales, const float *offsets, int stride,
                     int tokens, float *y, int ldy, int row_start, int row_end, cudaStream_t stream);
int launch_cq_gather(const uint8_t *indices, const uint16_t *norms, const float *levels16, int rows, int cols, int bits,
                     const int32_t *row_ids, int n, float *out, int *status, cudaStream_t stream);
int launch_mix4(const float *s, int dim, const float *w, int n, float *dst, cudaStream_t stream);
int launch_combine4(bool diff, const float *s, int dim, const float *mix, const float *x, const float *u,
                    const float *post, int n, float *dst, cudaStream_t stream);
int launch_sinkhorn4x4(const float *logits, int n, float *out, cudaStream_t stream);
int launch_taps3(const float *taps, int width, const float *triples, int n, float *dst, cudaStream_t stream);
int launch_fake_a8(int mode, const float *x, const float *aux, const float *gate, int rows, int n, float *dst,
                   cudaStream_t stream);
int launch_slot_vec(int mode, float *x, const float *aux, float *dst, float s0, float s1, int n, float *out,
                    cudaStream_t stream);
int launch_slot_rope(float *x, int heads, int head_dim, const float *cs, const float *sn, cudaStream_t stream);
struct KtTileArgs {
    const int8_t *q;
    const float *qs;
    int heads;
    const int8_t *keys;
    const float *ks;
    const int8_t *values;
    const float *vs;
    int key_stride, value_stride, scale_stride, count;
    float *scores;
    float *output;
    float *probs;
    float *peaks, *sums;
};
int launch_slot_attention_tile(const KtTileArgs &a, cudaStream_t stream);
int launch_slot_merge_partials(const float *partials, int count, int heads, float *out, cudaStream_t stream);
}  // namespace ndl

namespace {

// One growing device buffer, shared by the exports and guarded by a mutex
// (the reference calls kernel slots from several pool threads).
std::mutex g_mu;
void *g_buf = nullptr;
size_t g_cap = 0;
int g_dev = -1;

int scratch(size_t bytes, void **out) {
    int dev = 0;
    NDL_CUDA(cudaGetDevice(&dev));
    if (g_buf && (g_cap < bytes || g_dev != dev)) {
        cudaFree(g_buf);
        g_buf = nullptr;
        g_cap = 0;
    }
    if (!g_buf) {
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        if (cudaMalloc(&g_buf, cap) != cudaSuccess) {
            cudaGetLastError();
            return set_error(NDL_ERR_OUT_OF_MEMORY, "conformance scratch (%zu bytes)", cap);
        }
        g_cap = cap;
        g_dev = dev;
    }
    *out = g_buf;
    return NDL_OK;
}

size_t align16(size_t n) { return (n + 15) & ~size_t(15); }

// Host float arrays in, one launch, host float arrays out, through the
// scratch buffer: in[k] (n_in[k] floats) go up, the launch gets their device
// copies (ins) and the outputs' (outs), outputs come back.
template <typename F>
bool run_floats(const char *what, std::initializer_list<std::pair<const float *, size_t>> in,
                std::initializer_list<std::pair<float *, size_t>> out, F launch) {
    size_t bytes = 0;
    for (auto &a : in) bytes += align16(a.second * 4);
    for (auto &a : out) bytes += align16(a.second * 4);
    void *buf = nullptr;
    if (scratch(bytes + 16, &buf) != NDL_OK) return false;
    char *p = static_cast<char *>(buf);
    std::vector<float *> ins, outs;
    bool ok = true;
    for (auto &a : in) {
        ins.push_back(reinterpret_cast<float *>(p));
        ok = ok && cudaMemcpy(p, a.first, a.second * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        p += align16(a.second * 4);
    }
    for (auto &a : out) {
        outs.push_back(reinterpret_cast<float *>(p));
        p += align16(a.second * 4);
    }
    ok = ok && launch(ins, outs) == NDL_OK;
    size_t k = 0;
    for (auto &a : out) ok = ok && cudaMemcpy(a.first, outs[k++], a.second * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "%s failed", what);
    }
    return ok;
}

}  // namespace

extern "C" {

// float QuantizeInt8(float* x, int n, sbyte* destination)  (Quant.QuantizeInt8)
NDL_API float ndl_kt_quantize_int8(const float *x, int n, int8_t *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !destination || n < 1) {
        set_error(NDL_ERR_INVALID_ARG, "quantize_int8: bad arguments");
        return NAN;
    }
    void *buf = nullptr;
    if (scratch(align16((size_t)n * 4) + align16((size_t)n) + 16, &buf) != NDL_OK) return NAN;
    float *dx = static_cast<float *>(buf);
    int8_t *dq = reinterpret_cast<int8_t *>(static_cast<char *>(buf) + align16((size_t)n * 4));
    float *ds = reinterpret_cast<float *>(reinterpret_cast<char *>(dq) + align16((size_t)n));
    float scale = NAN;
    if (cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        ndl_quantize_rows(dx, 1, n, dq, ds, nullptr) != NDL_OK ||
        cudaMemcpy(destination, dq, (size_t)n, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(&scale, ds, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "quantize_int8 failed");
        return NAN;
    }
    return scale;
}

// int ArgMaxMasked(float* x, uint* mask, int words, int length)  (Ops.ArgMaxMasked)
NDL_API int ndl_kt_argmax_masked(const float *x, const uint32_t *mask, int words, int length) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !mask || words < 0 || length < 0) {
        set_error(NDL_ERR_INVALID_ARG, "argmax_masked: bad arguments");
        return -2;
    }
    const int n = length < words * 32 ? length : words * 32;  // ids >= length or >= 32*words are never chosen
    if (n <= 0) return -1;
    void *buf = nullptr;
    if (scratch(align16((size_t)n * 4) + align16((size_t)words * 4) + 16, &buf) != NDL_OK) return -2;
    float *dx = static_cast<float *>(buf);
    uint32_t *dm = reinterpret_cast<uint32_t *>(static_cast<char *>(buf) + align16((size_t)n * 4));
    int32_t *did = reinterpret_cast<int32_t *>(reinterpret_cast<char *>(dm) + align16((size_t)words * 4));
    int id = -2;
    if (cudaMemcpy(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dm, mask, (size_t)words * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_argmax_masked(dx, n, dm, words, words, nullptr, n, 1, did, nullptr, nullptr) != NDL_OK ||
        cudaMemcpy(&id, did, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "argmax_masked failed");
        return -2;
    }
    return id;
}

// float BestProbability(float* values, int count, float best)  (Ops.BestProbability)
NDL_API float ndl_kt_best_probability(const float *values, int count, float best) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!values || count < 1) {
        set_error(NDL_ERR_INVALID_ARG, "best_probability: bad arguments");
        return NAN;
    }
    void *buf = nullptr;
    if (scratch(align16((size_t)count * 4) + 16, &buf) != NDL_OK) return NAN;
    float *dx = static_cast<float *>(buf);
    float *dp = reinterpret_cast<float *>(static_cast<char *>(buf) + align16((size_t)count * 4));
    float p = NAN;
    if (cudaMemcpy(dx, values, (size_t)count * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_best_probability(dx, count, best, dp, nullptr) != NDL_OK ||
        cudaMemcpy(&p, dp, 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "best_probability failed");
        return NAN;
    }
    return p;
}


// void MatMulRows(Cq* w, Activations* a, int tokens, float* y, int ldy, int rowStart, int rowEnd)
// (Quant.MatMulRows on CQ weights).  Writes y[t*ldy + n] for n in [rowStart, rowEnd) only.
NDL_API void ndl_kt_matmul_rows(const ndl_kt_cq *w, const ndl_kt_activations *a, int tokens, float *y, int ldy,
                                int row_start, int row_end) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!w || !a || !y || tokens < 0 || row_start < 0 || row_end > w->rows || row_start > row_end || !w->book ||
        (w->bits != 2 && w->bits != 4) || w->cols % 128 != 0 || a->cols != w->cols || a->stride < w->cols / 128 ||
        ldy < row_end) {
        set_error(NDL_ERR_INVALID_ARG, "matmul_rows: bad arguments");
        return;
    }
    if (tokens == 0 || row_start == row_end) return;
    const int rows = row_end - row_start, cols = w->cols, groups = cols / 128;
    const size_t row_bytes = (size_t)cols * w->bits / 8;
    const size_t b_idx = align16((size_t)rows * row_bytes), b_nrm = align16((size_t)rows * groups * 2),
                 b_val = align16((size_t)tokens * cols), b_sc = align16((size_t)tokens * a->stride * 4),
                 b_y = align16((size_t)tokens * rows * 4);
    void *buf = nullptr;
    if (scratch(b_idx + b_nrm + b_val + 2 * b_sc + b_y, &buf) != NDL_OK) return;
    char *p = static_cast<char *>(buf);
    uint8_t *d_idx = reinterpret_cast<uint8_t *>(p);
    uint16_t *d_nrm = reinterpret_cast<uint16_t *>(p + b_idx);
    int8_t *d_val = reinterpret_cast<int8_t *>(p + b_idx + b_nrm);
    float *d_sc = reinterpret_cast<float *>(p + b_idx + b_nrm + b_val);
    float *d_of = reinterpret_cast<float *>(p + b_idx + b_nrm + b_val + b_sc);
    float *d_y = reinterpret_cast<float *>(p + b_idx + b_nrm + b_val + 2 * b_sc);
    if (cudaMemcpy(d_idx, w->indices + (size_t)row_start * row_bytes, (size_t)rows * row_bytes,
                   cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_nrm, w->norms + (size_t)row_start * groups, (size_t)rows * groups * 2, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(d_val, a->values, (size_t)tokens * cols, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_sc, a->scales, (size_t)tokens * a->stride * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_of, a->offsets, (size_t)tokens * a->stride * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_cq_matmul(d_idx, d_nrm, w->book->bytes, w->book->byte_scale, cols, w->bits, d_val, d_sc, d_of,
                         a->stride, tokens, d_y, rows, 0, rows, nullptr) != NDL_OK ||
        cudaMemcpy2D(y + row_start, (size_t)ldy * 4, d_y, (size_t)rows * 4, (size_t)rows * 4, tokens,
                     cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "matmul_rows failed");
    }
}

// void Prepare(float* x, int tokens, int cols, int bits, Activations* a)  (Quant.Prepare)
NDL_API void ndl_kt_prepare(const float *x, int tokens, int cols, int bits, const ndl_kt_activations *a) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !a || tokens < 0 || cols % 128 != 0 || cols < 128 || (bits != 2 && bits != 4) || a->cols != cols ||
        a->stride < cols / 128) {
        set_error(NDL_ERR_INVALID_ARG, "prepare: bad arguments");
        return;
    }
    if (tokens == 0) return;
    const int groups = cols / 128;
    const size_t b_x = align16((size_t)tokens * cols * 4), b_val = align16((size_t)tokens * cols),
                 b_sc = align16((size_t)tokens * a->stride * 4);
    void *buf = nullptr;
    if (scratch(b_x + b_val + 2 * b_sc, &buf) != NDL_OK) return;
    char *p = static_cast<char *>(buf);
    float *d_x = reinterpret_cast<float *>(p);
    int8_t *d_val = reinterpret_cast<int8_t *>(p + b_x);
    float *d_sc = reinterpret_cast<float *>(p + b_x + b_val);
    float *d_of = reinterpret_cast<float *>(p + b_x + b_val + b_sc);
    if (cudaMemcpy(d_x, x, (size_t)tokens * cols * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_cq_prepare(d_x, tokens, cols, bits, d_val, d_sc, d_of, a->stride, nullptr) != NDL_OK ||
        cudaMemcpy(a->values, d_val, (size_t)tokens * cols, cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy2D(a->scales, (size_t)a->stride * 4, d_sc, (size_t)a->stride * 4, (size_t)groups * 4, tokens,
                     cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy2D(a->offsets, (size_t)a->stride * 4, d_of, (size_t)a->stride * 4, (size_t)groups * 4, tokens,
                     cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "prepare failed");
    }
}


// void GatherRow(Cq* w, int row, float* destination)  (Quant.GatherRow)
NDL_API void ndl_kt_gather_row(const ndl_kt_cq *w, int row, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!w || !destination || !w->book || row < 0 || row >= w->rows || (w->bits != 2 && w->bits != 4) ||
        w->cols % 128 != 0 || w->cols < 128) {
        set_error(NDL_ERR_INVALID_ARG, "gather_row: bad arguments");
        return;
    }
    const int cols = w->cols, groups = cols / 128;
    const size_t row_bytes = (size_t)cols * w->bits / 8;
    const size_t b_idx = align16(row_bytes), b_nrm = align16((size_t)groups * 2), b_out = align16((size_t)cols * 4);
    void *buf = nullptr;
    if (scratch(b_idx + b_nrm + b_out + 16, &buf) != NDL_OK) return;
    char *p = static_cast<char *>(buf);
    uint8_t *d_idx = reinterpret_cast<uint8_t *>(p);
    uint16_t *d_nrm = reinterpret_cast<uint16_t *>(p + b_idx);
    float *d_out = reinterpret_cast<float *>(p + b_idx + b_nrm);
    int32_t *d_row = reinterpret_cast<int32_t *>(p + b_idx + b_nrm + b_out);
    const int32_t zero = 0;  // the one uploaded row is row 0 of the slice
    if (cudaMemcpy(d_idx, w->indices + (size_t)row * row_bytes, row_bytes, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_nrm, w->norms + (size_t)row * groups, (size_t)groups * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_row, &zero, 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        launch_cq_gather(d_idx, d_nrm, w->book->levels, 1, cols, w->bits, d_row, 1, d_out, nullptr, nullptr) != NDL_OK ||
        cudaMemcpy(destination, d_out, (size_t)cols * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "gather_row failed");
    }
}


// The Needle-3 row slots (Scalar.cs:250-439): 6 RmsFakeA8, 7 CenteredRmsFakeA8,
// 8 GateFakeA8, 9 PostNormAdd, 10 CombineDiff4, 11 Mix4, 12 Combine4,
// 13 Taps3, 24 Sinkhorn4x4.
NDL_API void ndl_kt_rms_fake_a8(const float *x, int n, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !destination || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "rms_fake_a8: bad arguments");
    run_floats("rms_fake_a8", {{x, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) { return launch_fake_a8(0, i[0], nullptr, nullptr, 1, n, o[0], nullptr); });
}

NDL_API void ndl_kt_centered_rms_fake_a8(const float *x, const float *scale, int n, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !scale || !destination || n < 1)
        return (void)set_error(NDL_ERR_INVALID_ARG, "centered_rms_fake_a8: bad arguments");
    run_floats("centered_rms_fake_a8", {{x, (size_t)n}, {scale, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) { return launch_fake_a8(1, i[0], i[1], nullptr, 1, n, o[0], nullptr); });
}

NDL_API void ndl_kt_gate_fake_a8(float *x, const float *gate, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !gate || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "gate_fake_a8: bad arguments");
    run_floats("gate_fake_a8", {{x, (size_t)n}, {gate, (size_t)n}}, {{x, (size_t)n}},
               [&](auto &i, auto &o) { return launch_fake_a8(2, i[0], i[1], nullptr, 1, n, o[0], nullptr); });
}

NDL_API void ndl_kt_post_norm_add(float *residual, const float *x, const float *scale, float gate, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!residual || !x || !scale || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "post_norm_add: bad arguments");
    run_floats("post_norm_add", {{x, (size_t)n}, {scale, (size_t)n}, {&gate, 1}, {residual, (size_t)n}},
               {{residual, (size_t)n}}, [&](auto &i, auto &o) -> int {
                   if (cudaMemcpy(o[0], i[3], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
                       return (int)NDL_ERR_CUDA;
                   return launch_fake_a8(3, i[0], i[1], i[2], 1, n, o[0], nullptr);
               });
}

NDL_API void ndl_kt_combine_diff4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *x,
                                  const float *u, float post, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!s || !x || !u || !destination || dim < 1)
        return (void)set_error(NDL_ERR_INVALID_ARG, "combine_diff4: bad arguments");
    const float mix[16] = {w0, w1, w2, w3};  // stream 0 is the slot's; streams 1-3 are discarded
    const float gates[4] = {post, 0.0f, 0.0f, 0.0f};
    std::vector<float> all((size_t)4 * dim);
    if (run_floats("combine_diff4", {{s, (size_t)4 * dim}, {mix, 16}, {x, (size_t)dim}, {u, (size_t)dim}, {gates, 4}},
                   {{all.data(), all.size()}}, [&](auto &i, auto &o) {
                       return launch_combine4(true, i[0], dim, i[1], i[2], i[3], i[4], 1, o[0], nullptr);
                   }))
        memcpy(destination, all.data(), (size_t)dim * 4);
}

NDL_API void ndl_kt_mix4(const float *s, int dim, float w0, float w1, float w2, float w3, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!s || !destination || dim < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "mix4: bad arguments");
    const float w[4] = {w0, w1, w2, w3};
    run_floats("mix4", {{s, (size_t)4 * dim}, {w, 4}}, {{destination, (size_t)dim}},
               [&](auto &i, auto &o) { return launch_mix4(i[0], dim, i[1], 1, o[0], nullptr); });
}

NDL_API void ndl_kt_combine4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *y,
                             float post, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!s || !y || !destination || dim < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "combine4: bad arguments");
    const float w[4] = {w0, w1, w2, w3};
    run_floats("combine4", {{s, (size_t)4 * dim}, {w, 4}, {y, (size_t)dim}, {&post, 1}}, {{destination, (size_t)dim}},
               [&](auto &i, auto &o) { return launch_combine4(false, i[0], dim, i[1], i[2], nullptr, i[3], 1, o[0], nullptr); });
}

NDL_API void ndl_kt_taps3(const float *taps, int width, const float *current, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!taps || !current || !destination || width < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "taps3: bad arguments");
    run_floats("taps3", {{taps, (size_t)3 * width}, {current - 2 * (size_t)width, (size_t)3 * width}},
               {{destination, (size_t)width}},
               [&](auto &i, auto &o) { return launch_taps3(i[0], width, i[1], 1, o[0], nullptr); });
}

NDL_API void ndl_kt_sinkhorn4x4(const float *logits, float *result) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!logits || !result) return (void)set_error(NDL_ERR_INVALID_ARG, "sinkhorn4x4: bad arguments");
    run_floats("sinkhorn4x4", {{logits, 16}}, {{result, 16}},
               [&](auto &i, auto &o) { return launch_sinkhorn4x4(i[0], 1, o[0], nullptr); });
}


// The float helper slots: 14 Rope, 15 ZeroCenteredRms, 16 RmsUnit, 17 Softmax,
// 18 Dot, 19 AddScaled, 20 ScaleAdd, 21 MultiplyAccumulate, 23 FakeA8.
NDL_API void ndl_kt_rope(float *x, int heads, int head_dim, const float *cos_t, const float *sin_t) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !cos_t || !sin_t || heads < 0 || head_dim < 2 || head_dim % 2)
        return (void)set_error(NDL_ERR_INVALID_ARG, "rope: bad arguments");
    const size_t n = (size_t)heads * head_dim, half = head_dim / 2;
    run_floats("rope", {{x, n}, {cos_t, half}, {sin_t, half}}, {{x, n}}, [&](auto &i, auto &o) -> int {
        if (cudaMemcpy(o[0], i[0], n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess) return (int)NDL_ERR_CUDA;
        return launch_slot_rope(o[0], heads, head_dim, i[1], i[2], nullptr);
    });
}

NDL_API void ndl_kt_zero_centered_rms(const float *x, const float *scale, int n, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !scale || !destination || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "zero_centered_rms: bad arguments");
    run_floats("zero_centered_rms", {{x, (size_t)n}, {scale, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) { return launch_slot_vec(1, i[0], i[1], o[0], 0, 0, n, nullptr, nullptr); });
}

NDL_API void ndl_kt_rms_unit(const float *x, int n, float *destination) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || !destination || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "rms_unit: bad arguments");
    run_floats("rms_unit", {{x, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) { return launch_slot_vec(0, i[0], nullptr, o[0], 0, 0, n, nullptr, nullptr); });
}

NDL_API void ndl_kt_softmax(float *s, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!s || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "softmax: bad arguments");
    run_floats("softmax", {{s, (size_t)n}}, {{s, (size_t)n}}, [&](auto &i, auto &o) -> int {
        if (cudaMemcpy(o[0], i[0], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess) return (int)NDL_ERR_CUDA;
        return launch_slot_vec(6, o[0], nullptr, nullptr, 0, 0, n, nullptr, nullptr);
    });
}

NDL_API float ndl_kt_dot(const float *a, const float *b, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!a || !b || n < 0) {
        set_error(NDL_ERR_INVALID_ARG, "dot: bad arguments");
        return NAN;
    }
    if (n == 0) return 0.0f;
    float r = NAN;
    if (!run_floats("dot", {{a, (size_t)n}, {b, (size_t)n}}, {{&r, 1}}, [&](auto &i, auto &o) {
            return launch_slot_vec(5, i[0], i[1], nullptr, 0, 0, n, o[0], nullptr);
        }))
        return NAN;
    return r;
}

NDL_API void ndl_kt_add_scaled(float *destination, const float *x, float scale, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!destination || !x || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "add_scaled: bad arguments");
    run_floats("add_scaled", {{x, (size_t)n}, {destination, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) -> int {
                   if (cudaMemcpy(o[0], i[1], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
                       return (int)NDL_ERR_CUDA;
                   return launch_slot_vec(2, i[0], nullptr, o[0], scale, 0, n, nullptr, nullptr);
               });
}

NDL_API void ndl_kt_scale_add(float *destination, float scale, const float *x, float x_scale, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!destination || !x || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "scale_add: bad arguments");
    run_floats("scale_add", {{x, (size_t)n}, {destination, (size_t)n}}, {{destination, (size_t)n}},
               [&](auto &i, auto &o) -> int {
                   if (cudaMemcpy(o[0], i[1], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
                       return (int)NDL_ERR_CUDA;
                   return launch_slot_vec(3, i[0], nullptr, o[0], scale, x_scale, n, nullptr, nullptr);
               });
}

NDL_API void ndl_kt_multiply_accumulate(float *destination, const float *a, const float *b, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!destination || !a || !b || n < 1) return (void)set_error(NDL_ERR_INVALID_ARG, "multiply_accumulate: bad arguments");
    run_floats("multiply_accumulate", {{a, (size_t)n}, {b, (size_t)n}, {destination, (size_t)n}},
               {{destination, (size_t)n}}, [&](auto &i, auto &o) -> int {
                   if (cudaMemcpy(o[0], i[2], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess)
                       return (int)NDL_ERR_CUDA;
                   return launch_slot_vec(4, i[0], i[1], o[0], 0, 0, n, nullptr, nullptr);
               });
}

NDL_API float ndl_kt_fake_a8(float *x, int n) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!x || n < 1) {
        set_error(NDL_ERR_INVALID_ARG, "fake_a8: bad arguments");
        return NAN;
    }
    float scale = NAN;
    if (!run_floats("fake_a8", {{x, (size_t)n}}, {{x, (size_t)n}, {&scale, 1}}, [&](auto &i, auto &o) -> int {
            if (cudaMemcpy(o[0], i[0], (size_t)n * 4, cudaMemcpyDeviceToDevice) != cudaSuccess) return (int)NDL_ERR_CUDA;
            return launch_slot_vec(7, o[0], nullptr, nullptr, 0, 0, n, o[1], nullptr);
        }))
        return NAN;
    return scale;
}


// void AttentionTile(AttentionTile* tile)  slot 3: 48-dim keys, 64-dim values, up
// to 6 heads over one span (Attention.Run, src/Needle/Blocks.cs:65-84).
NDL_API void ndl_kt_attention_tile(const ndl_kt_tile *t) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!t || t->heads < 1 || t->heads > 6 || t->count < 1 || t->first < 0 || !t->queries || !t->query_scales ||
        !t->keys || !t->key_scales || !t->values || !t->value_scales || !t->output || !t->scores ||
        t->key_stride < 48 || t->value_stride < 64 || t->scale_stride < 1 || (!t->peaks) != (!t->sums) ||
        (t->probabilities && t->probability_stride < t->first + t->count)) {
        set_error(NDL_ERR_INVALID_ARG, "attention_tile: bad arguments");
        return;
    }
    const int H = t->heads, n = t->count;
    const size_t kb = (size_t)(n - 1) * t->key_stride + 48, vb = (size_t)(n - 1) * t->value_stride + 64;
    const size_t sf = (size_t)(n - 1) * t->scale_stride + 1;
    const size_t sizes[] = {align16((size_t)H * 48), align16((size_t)H * 4), align16(kb), align16(vb), align16(sf * 4),
                            align16(sf * 4), align16((size_t)H * n * 4), align16((size_t)H * 64 * 4),
                            align16((size_t)H * n * 4), align16((size_t)H * 4), align16((size_t)H * 4)};
    size_t total = 0;
    for (size_t z : sizes) total += z;
    void *buf = nullptr;
    if (scratch(total, &buf) != NDL_OK) return;
    char *p = static_cast<char *>(buf);
    char *ptrs[11];
    for (int i = 0; i < 11; i++) ptrs[i] = p, p += sizes[i];
    KtTileArgs a{reinterpret_cast<int8_t *>(ptrs[0]), reinterpret_cast<float *>(ptrs[1]), H,
                 reinterpret_cast<int8_t *>(ptrs[2]), reinterpret_cast<float *>(ptrs[4]),
                 reinterpret_cast<int8_t *>(ptrs[3]), reinterpret_cast<float *>(ptrs[5]), t->key_stride,
                 t->value_stride, t->scale_stride, n, reinterpret_cast<float *>(ptrs[6]),
                 reinterpret_cast<float *>(ptrs[7]), t->probabilities ? reinterpret_cast<float *>(ptrs[8]) : nullptr,
                 t->peaks ? reinterpret_cast<float *>(ptrs[9]) : nullptr,
                 t->sums ? reinterpret_cast<float *>(ptrs[10]) : nullptr};
    const size_t first = (size_t)t->first;
    bool ok = cudaMemcpy(ptrs[0], t->queries, (size_t)H * 48, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(ptrs[1], t->query_scales, (size_t)H * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(ptrs[2], t->keys + first * t->key_stride, kb, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(ptrs[3], t->values + first * t->value_stride, vb, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(ptrs[4], t->key_scales + first * t->scale_stride, sf * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(ptrs[5], t->value_scales + first * t->scale_stride, sf * 4, cudaMemcpyHostToDevice) ==
                  cudaSuccess &&
              launch_slot_attention_tile(a, nullptr) == NDL_OK &&
              cudaMemcpy(t->output, ptrs[7], (size_t)H * 64 * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
              cudaMemcpy(t->scores, ptrs[6] + (size_t)(H - 1) * n * 4, (size_t)n * 4, cudaMemcpyDeviceToHost) ==
                  cudaSuccess;  // the reference's scratch ends with the last head's scores
    if (ok && t->probabilities)
        ok = cudaMemcpy2D(t->probabilities + first, (size_t)t->probability_stride * 4, ptrs[8], (size_t)n * 4,
                          (size_t)n * 4, H, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (ok && t->peaks)
        ok = cudaMemcpy(t->peaks, ptrs[9], (size_t)H * 4, cudaMemcpyDeviceToHost) == cudaSuccess &&
             cudaMemcpy(t->sums, ptrs[10], (size_t)H * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "attention_tile failed");
    }
}

// void MergePartials(float* partials, int count, int heads, float* output)  slot 4
NDL_API void ndl_kt_merge_partials(const float *partials, int count, int heads, float *output) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!partials || !output || count < 1 || heads < 1 || heads > 6)
        return (void)set_error(NDL_ERR_INVALID_ARG, "merge_partials: bad arguments");
    run_floats("merge_partials", {{partials, (size_t)count * (6 * 64 + 16)}}, {{output, (size_t)heads * 64}},
               [&](auto &i, auto &o) { return launch_slot_merge_partials(i[0], count, heads, o[0], nullptr); });
}

// void HadamardMlpApply(MlpBatch* b, float* residual, float* scratch)  slot 5
// (HadamardMlp.Apply, src/Needle/Blocks.cs:1067-1093): the residual row is
// updated in place; the reference's scratch argument is not used.
NDL_API void ndl_kt_hadamard_mlp(const ndl_kt_mlp_batch *b, float *residual, float *work) {
    (void)work;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!b || !b->weights || !residual || !b->pre_norm || !b->perm_a || !b->perm_b || b->dim < 1 || b->rows < 1 ||
        b->cols < 1 || b->cols > 1024) {
        set_error(NDL_ERR_INVALID_ARG, "hadamard_mlp: bad arguments");
        return;
    }
    const int dim = b->dim, rows = b->rows, cols = b->cols, width = rows * cols, in_rows = (dim + cols - 1) / cols;
    if (in_rows > rows) return (void)set_error(NDL_ERR_INVALID_ARG, "hadamard_mlp: dim %d beyond %d x %d", dim, rows, cols);
    for (int n = 0; n < width; n++)
        if (b->perm_a[n] < 0 || b->perm_a[n] >= width || b->perm_b[n] < 0 || b->perm_b[n] >= width)
            return (void)set_error(NDL_ERR_INVALID_ARG, "hadamard_mlp: permutation entry out of range");
    const ndl_kt_mlp_weights &w = *b->weights;
    const float *src[13] = {w.d1, w.d2, w.b2, w.d3, w.d4, w.w1a, w.w1b, w.w2a, w.w2b, w.w3a, w.w3b, w.cond_v, w.cond_u};
    const size_t cnt[13] = {(size_t)dim, (size_t)width, (size_t)width, (size_t)width, (size_t)dim,
                            (size_t)in_rows * rows, (size_t)cols * cols, (size_t)rows * rows, (size_t)cols * cols,
                            (size_t)rows * rows, (size_t)cols * cols, (size_t)dim * 8, (size_t)8 * width};
    size_t total = align16((size_t)dim * 4) * 2 + align16((size_t)width * 4) * 2;
    for (int k = 0; k < 13; k++) {
        if (!src[k]) return (void)set_error(NDL_ERR_INVALID_ARG, "hadamard_mlp: null weight array %d", k);
        total += align16(cnt[k] * 4);
    }
    void *buf = nullptr;
    if (scratch(total, &buf) != NDL_OK) return;
    char *p = static_cast<char *>(buf);
    KtMlpArgs a{};
    bool ok = true;
    for (int k = 0; k < 13; k++) {
        a.w[k] = reinterpret_cast<const float *>(p);
        ok = ok && cudaMemcpy(p, src[k], cnt[k] * 4, cudaMemcpyHostToDevice) == cudaSuccess;
        p += align16(cnt[k] * 4);
    }
    float *d_pre = reinterpret_cast<float *>(p);
    p += align16((size_t)dim * 4);
    float *d_res = reinterpret_cast<float *>(p);
    p += align16((size_t)dim * 4);
    int32_t *d_pa = reinterpret_cast<int32_t *>(p);
    p += align16((size_t)width * 4);
    int32_t *d_pb = reinterpret_cast<int32_t *>(p);
    ok = ok && cudaMemcpy(d_pre, b->pre_norm, (size_t)dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(d_res, residual, (size_t)dim * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(d_pa, b->perm_a, (size_t)width * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(d_pb, b->perm_b, (size_t)width * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    a.pre_norm = d_pre;
    a.perm_a = d_pa;
    a.perm_b = d_pb;
    a.dim = dim;
    a.rows = rows;
    a.cols = cols;
    a.scale = b->scale;
    a.residual = d_res;
    ok = ok && launch_slot_hadamard_mlp(a, nullptr) == NDL_OK &&
         cudaMemcpy(residual, d_res, (size_t)dim * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(NDL_ERR_CUDA, "hadamard_mlp failed");
    }
}

}  // extern "C"
