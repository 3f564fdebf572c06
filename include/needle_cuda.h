/*
 * needle_cuda.h - C ABI of the B200 (sm_100a) batched quantized decode path
 * for needle-cs.
 *
 * Plain C: pointers, sizes and int status codes; no CUDA or torch types.
 * A `stream` argument is a cudaStream_t passed as void* (NULL = legacy
 * default stream).  Functions named ndl_kt_* take HOST pointers and are
 * synchronous: they have the exact signatures of the reference's
 * KernelTable slots (src/Needle/Kernels/KernelTable.cs:5-47, signatures
 * fixed by src/Needle/Kernels/Net10KernelExports.cs:118-150) so that the C#
 * engine can install them with Kernels.Install.  Every other compute entry
 * point takes DEVICE pointers and is stream-ordered (asynchronous).
 *
 * Errors never cross the ABI as exceptions.  Codes 1..11 mirror the
 * reference's FailureReason (src/Needle/Reply.cs:8-22); codes >= 100 are
 * library errors.  ndl_last_error() returns a per-thread message for the
 * last non-zero status.
 */
#ifndef NEEDLE_CUDA_H
#define NEEDLE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define NDL_API __declspec(dllexport)
#else
#define NDL_API __attribute__((visibility("default")))
#endif

/* ------------------------------------------------------------------ */
/* Status codes                                                        */
/* ------------------------------------------------------------------ */
enum {
    NDL_OK = 0,
    /* FailureReason mirror (src/Needle/Reply.cs:8-22) */
    NDL_FAIL_EMPTY_INPUT = 1,
    NDL_FAIL_INPUT_TOO_LONG = 2,
    NDL_FAIL_CONTEXT_EXHAUSTED = 3,
    NDL_FAIL_CALL_TOKEN_BUDGET = 4,
    NDL_FAIL_CALL_TEXT_TOO_LONG = 5,
    NDL_FAIL_GRAMMAR_DEAD_END = 6,
    NDL_FAIL_GRAMMAR_REJECTED = 7,
    NDL_FAIL_CALLS_BUFFER = 8,
    NDL_FAIL_MALFORMED_CALLS = 9,
    NDL_FAIL_TOOL_CONTEXT = 10,
    NDL_FAIL_FRAME_BUDGET = 11,
    /* library errors */
    NDL_ERR_INVALID_ARG = 100,
    NDL_ERR_CUDA = 101,
    NDL_ERR_BOUNDS = 102,
    NDL_ERR_TIMEOUT = 103,
    NDL_ERR_OUT_OF_MEMORY = 104,
    NDL_ERR_UNSUPPORTED = 105,
    NDL_ERR_NO_DEVICE = 106,
    NDL_ERR_MALFORMED_MODEL = 107,
    NDL_ERR_PAGES_EXHAUSTED = 108,
    NDL_ERR_CANCELLED = 109
};

/* Failure detection self-test (no reference counterpart): a kernel waits
 * for an mbarrier phase that never completes; its bounded wait gives up
 * after `tests` suspend-hinted tests (about a microsecond each), records the
 * timeout and returns.  Returns NDL_ERR_TIMEOUT, the status every kernel
 * reports after a wait that ran out; the context stays usable. */
NDL_API int ndl_selftest_bounded_wait(int tests);
/* The library's float exponential (the reference's Ops.Exp, which its
 * softmax and SiLU use) over n device floats, on `stream`: for pinning it to
 * a CPU restatement.  No counterpart in the reference. */
NDL_API int ndl_selftest_exp(const float *x, int n, float *y, void *stream);

/* Library identity and diagnostics (no reference counterpart). */
NDL_API const char *ndl_version(void);
NDL_API const char *ndl_status_string(int status);
NDL_API const char *ndl_last_error(void);
NDL_API int ndl_device_count(int *count);

/* ------------------------------------------------------------------ */
/* Synthetic inputs                                                    */
/* ------------------------------------------------------------------ */
/* Counter-based generator used for every synthetic workload.  Value i of
 * stream s under seed k is a pure function of (k, s, i), so host and device
 * produce identical bits:
 *   key     = splitmix64(k ^ (s * 0x9E3779B97F4A7C15))
 *   h(i)    = splitmix64(key + i * 0xD1B54A32D192ED03)
 *   normal  = (2*S - 786420) / 131072, S = sum of the twelve 16-bit fields
 *             of h(3i), h(3i+1), h(3i+2)     (Irwin-Hall(12) - 6, var 1)
 *   uniform = lo + (hi - lo) * float(h(i) >> 40) * 2^-24
 *   int8    = int(h(i) % 255) - 127            (U{-127..127})
 *   fp16    = round-to-nearest-even of a float
 * The reference's own test RNG (XorShift64, tests/Needle.Tests/Conformance/
 * Conformance.cs:10-38) drives only the conformance-case ports. */
NDL_API void ndl_synth_normal_f32(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                  float *out);
NDL_API void ndl_synth_normal_f16(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                  uint16_t *out);
NDL_API void ndl_synth_uniform_f16(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo,
                                   float hi, uint16_t *out);
NDL_API void ndl_synth_int8(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out);
NDL_API uint16_t ndl_f32_to_f16(float value);
NDL_API float ndl_f16_to_f32(uint16_t half);
/* Device-side fills (same bits as the host functions). */
NDL_API int ndl_synth_normal_f32_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale,
                                        float *out, void *cuda_stream);
NDL_API int ndl_synth_normal_f16_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count,
                                        float scale, uint16_t *out, void *cuda_stream);
NDL_API int ndl_synth_uniform_f16_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo,
                                         float hi, uint16_t *out, void *cuda_stream);
NDL_API int ndl_synth_int8_device(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out,
                                  void *cuda_stream);

/* ------------------------------------------------------------------ */
/* Device kernels (device pointers, stream-ordered)                    */
/* ------------------------------------------------------------------ */

/* Per-row int8 quantizer.  Replaces Quant.QuantizeInt8
 * (src/Needle/Quant.cs:103-132; scalar definition src/Needle/Scalar.cs:67-74)
 * applied to each row of x [rows][cols]: scale = max|x|/127 (1 if zero),
 * q = clamp(round_half_even(x * (1/scale)), -128, 127).  Bit-exact. */
NDL_API int ndl_quantize_rows(const float *x, int rows, int cols, int8_t *q, float *scales, void *stream);

/* Fused RMSNorm + quantizer for the synthetic decoder: h = (w*x)*inv_rms(x)
 * (eps 1e-6, src/Needle/Ops.cs:12,209,233-255), then ndl_quantize_rows(h). */
NDL_API int ndl_rmsnorm_quantize(const float *x, const float *weight, int rows, int cols, int8_t *q, float *scales,
                                 void *stream);

/* I8G32 quantized linear.  Replaces Quant.MatMulRows
 * (src/Needle/Quant.cs:615-633 -> src/Needle/Gemv.cs:117-333; scalar
 * skeleton src/Needle/Scalar.cs:146-192) for int8 weights with one fp16
 * scale per (row, 32-column group) and one activation scale per row:
 *   D[t][n][g] = sum_{k in g} w[n][k]*q[t][k]              (int32, exact)
 *   acc        = fma(half(sw[n][g]), float(D), acc)         (g ascending)
 *   y[t][n]    = (residual ? residual[t][n] : 0) + acc * sa[t]
 * The same operation order in every kernel, so y is bit-identical across
 * batch sizes and kernels.  acc (nullable) receives D as [m][n][k/32].
 * k must be a multiple of 32; w, q 16-byte aligned.  Small m runs the
 * streaming GEMV (mma.sync); packed batches the tcgen05 kind::i8 GEMM. */
NDL_API int ndl_matmul_i8g32(const int8_t *q, const float *sa, int m, const int8_t *w, const uint16_t *sw, int n,
                             int k, float *y, int ldy, const float *residual, int32_t *acc, void *stream);

/* The same linear over `batch` independent weight sets sharing one set of
 * activations (MatMulBatch, src/Needle/Quant.cs:679-816): set b uses
 * w + b*w_stride, sw + b*sw_stride and writes y + b*y_stride. */
NDL_API int ndl_matmul_i8g32_batched(const int8_t *q, const float *sa, int m, const int8_t *w,
                                     const uint16_t *sw, int n, int k, int batch, long long w_stride,
                                     long long sw_stride, float *y, int ldy, long long y_stride, void *stream);

/* Paged int8 decode attention: the device-pointer counterpart of the
 * AttentionTile / AttentionBatch kernel slots (Scalar.AttentionHead
 * src/Needle/Scalar.cs:290-312, AttentionBatch src/Needle/Blocks.cs:830-990).
 * For row r and head h it attends to positions 0..row_pos[r] of slot
 * row_slot[r], with every rounding of Scalar.AttentionHead in its order:
 *   s_j = ((q . k_j) * ks_j) * (qs[r][h] / 8);  e_j = exp(s_j - max s);
 *   total = e_0 + e_1 + ... (in position order);  p_j = e_j / total;
 *   out = 0;  out += (p_j * vs_j) * v_j  for j = 0, 1, ...
 * (exp is the correctly rounded single-precision exponential), so the
 * output equals the scalar routine's bit for bit.
 * Page layout: a page holds 64 positions of one slot for every layer; the
 * (layer, head) record at ((layer*heads + head) * 8704) is two halves,
 *   [K int8 64x64][K scale f32 x64] [V scale f32 x64][V int8 64x64]
 * K (row = position p, col = dim d) is stored in mma m16n8k32 A-fragment
 * order: element (row, col) at byte
 *   (row>>4)*1024 + (col>>5)*512 + ((row&7)*4 + (col>>2&3))*16
 *   + ((row>>3&1) + 2*(col>>4&1))*4 + (col&3)
 * and the K scale of p at index 2*((p&7)*4 + (p>>4&3)) + (p>>3&1).  The V
 * scales are in position order; V (p, d) sits at byte 4608 +
 * d*64 + ((((p>>4) ^ ((d>>1)&3)) << 4) | (p&15)) of the record.
 * The query's dims are in the order k_slot(d) = ((d&15)>>2)*16 + (d>>4)*4 + (d&3).
 * q: int8 [rows][heads][64] in k_slot order; qs [rows][heads]; out fp32
 * [rows][heads][64]; max_pages * 64 <= 8192.  The work list (one record per
 * row) lives in `workspace` (NULL: allocated and freed on `stream` by the
 * library).
 * status (nullable, device int) receives 2 for an out-of-range slot, page
 * or length and 1 for a timed-out wait.  A row with an out-of-range slot or
 * length, and a head whose pages include one outside the pool, is skipped
 * and its out values are NaN; after a timed-out wait out is undefined. */
NDL_API size_t ndl_attention_paged_workspace(int rows, int heads, int max_pages);
NDL_API int ndl_attention_paged(const int8_t *q, const float *qs, const int32_t *row_slot, const int32_t *row_pos,
                                int rows, int heads, const int32_t *page_table, int slots, int max_pages,
                                const uint8_t *pool, size_t page_bytes, int num_pages, int layer, float *out,
                                void *workspace, size_t workspace_bytes, int *status, void *stream);

/* ndl_attention_paged for callers that cannot allocate.  No counterpart in
 * the reference: it exists for hosts that must not allocate while serving
 * (frame-budgeted game or job threads, audio callbacks, zero-allocation
 * request loops), where cudaMalloc could block or synchronise the device.
 * Same arguments and results as ndl_attention_paged, without a workspace:
 * the work list lives in a 4 MiB device array owned by the library (held
 * on every GPU that loads it until exit).  Requests whose
 * ndl_attention_paged_workspace(rows, heads, max_pages) exceeds 4 MiB are
 * rejected with NDL_ERR_INVALID_ARG: each row takes 16 + 4 * max_pages
 * bytes (max_pages rounded up to a multiple of 4), so rows *
 * (16 + 4 * max_pages) + 16 may be at most 4 MiB; 512 rows fit at any
 * supported max_pages (<= 128).  The first call on a device looks the array up
 * (cudaGetSymbolAddress) and must come before any stream capture.  All
 * calls share the array: calls that overlap on the GPU race and must be
 * ordered by the caller (e.g. one stream).  Allocates nothing. */
NDL_API int ndl_attention_paged_noalloc(const int8_t *q, const float *qs, const int32_t *row_slot,
                                        const int32_t *row_pos, int rows, int heads, const int32_t *page_table,
                                        int slots, int max_pages, const uint8_t *pool, size_t page_bytes,
                                        int num_pages, int layer, float *out, int *status, void *stream);

/* ------------------------------------------------------------------ */
/* KernelTable conformance exports                                     */
/* ------------------------------------------------------------------ */
/* The reference's kernel slots with their exact Cdecl signatures
 * (src/Needle/Kernels/KernelTable.cs:5-47, Net10KernelExports.Fill
 * src/Needle/Kernels/Net10KernelExports.cs:118-150), computed on the current
 * CUDA device; host pointers, synchronous, safe to call from several
 * threads.  No error channel, like the slots: NaN / -2 on failure with the
 * reason in ndl_last_error.
 *   QuantizeInt8     float(float* x, int n, sbyte* destination)  slot 22
 *   ArgMaxMasked     int(float* x, uint* mask, int words, int length)  slot 25
 *   BestProbability  float(float* values, int count, float best)  slot 26 */
NDL_API float ndl_kt_quantize_int8(const float *x, int n, int8_t *destination);
NDL_API int ndl_kt_argmax_masked(const float *x, const uint32_t *mask, int words, int length);
NDL_API float ndl_kt_best_probability(const float *values, int count, float best);

/* CQ weights (the reference's `.cact` matrices): Codebook, Cq and
 * Activations with the reference's sequential layouts (src/Needle/Model.cs:8-52,
 * src/Needle/Quant.cs:11-42).
 *   MatMulRows  void(Cq* w, Activations* a, int tokens, float* y, int ldy,
 *               int rowStart, int rowEnd)  slot 0: y[t*ldy + n] for n in
 *               [rowStart, rowEnd) only, equal bit for bit to Scalar.MatMulRows
 *               (src/Needle/Scalar.cs:146-192).
 *   Prepare     void(float* x, int tokens, int cols, int bits, Activations* a)
 *               slot 1: Quant.PrepareRange's scalar branch
 *               (src/Needle/Quant.cs:471-484), bit for bit. */
typedef struct {
    float levels[16];
    uint8_t bytes[32];
    float byte_scale;
} ndl_kt_codebook;
typedef struct {
    const uint8_t *indices;  /* [rows][cols * bits / 8] */
    const uint16_t *norms;   /* [rows][cols / 128] fp16 */
    const ndl_kt_codebook *book;
    int rows, cols, bits;
} ndl_kt_cq;
typedef struct {
    int8_t *values;  /* [tokens][cols], plane order */
    float *scales;   /* [tokens][stride] */
    float *offsets;  /* [tokens][stride] */
    int cols, groups, stride;
} ndl_kt_activations;
NDL_API void ndl_kt_matmul_rows(const ndl_kt_cq *w, const ndl_kt_activations *a, int tokens, float *y, int ldy,
                                int row_start, int row_end);
NDL_API void ndl_kt_prepare(const float *x, int tokens, int cols, int bits, const ndl_kt_activations *a);
/* GatherRow  void(Cq* w, int row, float* destination)  slot 2: Quant.GatherRow
 * (src/Needle/Quant.cs:566-576), row decoded (Scalar.DecodeRow) and rotated
 * per 128-column group (Scalar.Hadamard), bit for bit. */
NDL_API void ndl_kt_gather_row(const ndl_kt_cq *w, int row, float *destination);

/* The Needle-3 row slots, same conventions (Scalar.cs:250-439, Ops.cs:800-812):
 *   RmsFakeA8          void(float* x, int n, float* destination)              slot 6
 *   CenteredRmsFakeA8  void(float* x, float* scale, int n, float* destination) slot 7
 *   GateFakeA8         void(float* x, float* gate, int n)                      slot 8 (x in place)
 *   PostNormAdd        void(float* residual, float* x, float* scale, float gate, int n)  slot 9
 *   CombineDiff4       void(float* s, int dim, float w0..w3, float* x, float* u, float post, float* destination) slot 10
 *   Mix4               void(float* s, int dim, float w0..w3, float* destination)  slot 11
 *   Combine4           void(float* s, int dim, float w0..w3, float* y, float post, float* destination) slot 12
 *   Taps3              void(float* taps, int width, float* current, float* destination) slot 13
 *                      (reads current[-2*width .. width))
 *   Sinkhorn4x4        void(float* logits, float* result)                      slot 24
 * Equal to the scalar code bit for bit (MathF.Exp in GateFakeA8 and
 * Sinkhorn4x4 is the correctly rounded exponential the CPU oracle computes
 * in the same double-precision steps). */
NDL_API void ndl_kt_rms_fake_a8(const float *x, int n, float *destination);
NDL_API void ndl_kt_centered_rms_fake_a8(const float *x, const float *scale, int n, float *destination);
NDL_API void ndl_kt_gate_fake_a8(float *x, const float *gate, int n);
NDL_API void ndl_kt_post_norm_add(float *residual, const float *x, const float *scale, float gate, int n);
NDL_API void ndl_kt_combine_diff4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *x,
                                  const float *u, float post, float *destination);
NDL_API void ndl_kt_mix4(const float *s, int dim, float w0, float w1, float w2, float w3, float *destination);
NDL_API void ndl_kt_combine4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *y,
                             float post, float *destination);
NDL_API void ndl_kt_taps3(const float *taps, int width, const float *current, float *destination);
NDL_API void ndl_kt_sinkhorn4x4(const float *logits, float *result);

/* The float helper slots, same conventions:
 *   Rope               void(float* x, int heads, int headDim, float* cos, float* sin)  slot 14 (x in place)
 *   ZeroCenteredRms    void(float* x, float* scale, int n, float* destination)  slot 15
 *   RmsUnit            void(float* x, int n, float* destination)                slot 16
 *   Softmax            void(float* s, int n)                                    slot 17 (in place)
 *   Dot                float(float* a, float* b, int n)                         slot 18
 *   AddScaled          void(float* destination, float* x, float scale, int n)   slot 19
 *   ScaleAdd           void(float* destination, float scale, float* x, float xScale, int n)  slot 20
 *   MultiplyAccumulate void(float* destination, float* a, float* b, int n)      slot 21
 *   FakeA8             float(float* x, int n)                                   slot 23 (x in place)
 * Bit-exact to the scalar code except Softmax's exp (tolerance). */
NDL_API void ndl_kt_rope(float *x, int heads, int head_dim, const float *cos_t, const float *sin_t);
NDL_API void ndl_kt_zero_centered_rms(const float *x, const float *scale, int n, float *destination);
NDL_API void ndl_kt_rms_unit(const float *x, int n, float *destination);
NDL_API void ndl_kt_softmax(float *s, int n);
NDL_API float ndl_kt_dot(const float *a, const float *b, int n);
NDL_API void ndl_kt_add_scaled(float *destination, const float *x, float scale, int n);
NDL_API void ndl_kt_scale_add(float *destination, float scale, const float *x, float x_scale, int n);
NDL_API void ndl_kt_multiply_accumulate(float *destination, const float *a, const float *b, int n);
NDL_API float ndl_kt_fake_a8(float *x, int n);

/* AttentionTile  void(AttentionTile* tile)  slot 3 and MergePartials
 * void(float* partials, int count, int heads, float* output)  slot 4 (the
 * reference's tile: 48-dim int8 keys, 64-dim values, up to 6 heads,
 * src/Needle/Blocks.cs:11-27,65-84,750-817).  With peaks and sums set the
 * tile's outputs are unnormalized and each head's peak and exp sum are
 * stored (the split-position mode); MergePartials combines `count` slots of
 * 6*64 + 16 floats.  fp32 throughout; tolerance-equal to the scalar code. */
typedef struct {
    const int8_t *queries;      /* [heads][48] */
    const float *query_scales;  /* [heads] */
    int heads;
    const int8_t *keys;         /* row p at keys + p * key_stride */
    const float *key_scales;    /* [p * scale_stride] */
    const int8_t *values;
    const float *value_scales;
    int key_stride, value_stride, scale_stride, first, count;
    float *scores;              /* scratch, >= count floats */
    float *output;              /* [heads][64] */
    float *probabilities;       /* nullable: head h at + h * probability_stride + first */
    int probability_stride;
    float *peaks;               /* nullable (with sums): [heads] */
    float *sums;
} ndl_kt_tile;
NDL_API void ndl_kt_attention_tile(const ndl_kt_tile *tile);
NDL_API void ndl_kt_merge_partials(const float *partials, int count, int heads, float *output);

/* HadamardMlpApply  void(MlpBatch* b, float* residual, float* scratch)  slot 5
 * (HadamardMlp.Apply, src/Needle/Blocks.cs:1067-1093): the Kronecker-factored
 * MLP on one token's residual row, updated in place; MlpWeights and MlpBatch
 * in the reference's sequential layouts (src/Needle/Audio.cs:5-27,
 * src/Needle/Blocks.cs:992-1004).  Inner sums in the scalar order; the
 * condition softmax and the SiLU take MathF.Exp as the correctly rounded
 * exponential, so the row equals the scalar code's bit for bit. */
typedef struct {
    const float *d1, *d2, *b2, *d3, *d4;
    const float *w1a, *w1b, *w2a, *w2b, *w3a, *w3b;
    const float *cond_v, *cond_u;
} ndl_kt_mlp_weights;
typedef struct {
    const ndl_kt_mlp_weights *weights;
    const float *pre_norm;
    const int32_t *perm_a, *perm_b;
    float *residual;  /* unused by the slot (the row comes as an argument) */
    int dim, rows, cols;
    float scale;
} ndl_kt_mlp_batch;
NDL_API void ndl_kt_hadamard_mlp(const ndl_kt_mlp_batch *b, float *residual, float *scratch);

/* The same two operations on device memory, stream-ordered: CQ activation
 * prep for `tokens` rows of x [tokens][cols] (values [tokens][cols], scales
 * and offsets [tokens][stride]) and the CQ matmul y[t*ldy + n] for n in
 * [row_start, row_end) of a [rows][cols] CQ matrix (book_bytes: the
 * codebook's 16 level bytes, host memory).  cols a multiple of 128 up to
 * 8192; bits 2 or 4. */
NDL_API int ndl_cq_prepare(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales,
                           float *offsets, int stride, void *stream);
NDL_API int ndl_cq_matmul(const uint8_t *indices, const uint16_t *norms, const uint8_t *book_bytes, float byte_scale,
                          int rows, int cols, int bits, const int8_t *values, const float *scales,
                          const float *offsets, int stride, int tokens, float *y, int ldy, int row_start, int row_end,
                          void *stream);
/* GatherRow for a batch on device memory (embedding lookups): out[r] =
 * row row_ids[r] of the CQ matrix (row_ids and out on the device, levels: the
 * codebook's 16 float levels, host memory).  An id outside [0, rows) gives a
 * row of zeros: ids are device data, so check them where they are made. */
NDL_API int ndl_cq_gather_rows(const uint8_t *indices, const uint16_t *norms, const float *levels, int rows, int cols,
                               int bits, const int32_t *row_ids, int n, float *out, void *stream);

/* The same row operations batched over n tokens on device memory (a Needle-3
 * layer, EngineCore.RunLayerBatch, src/Needle/Engine.cs:2352-2404):
 *   hc_mix4           dst[t] = sum_i w[t][i] * s[t][i]       s [n][4][dim], w [n][4]
 *   hc_combine4       dst[t] = post[t] * y[t] + sum_i w[t][i] * s[t][i]
 *   hc_combine_diff4x4  stream o of dst[t] = post_gate[t][o] * (x[t] - u[t])
 *                     + sum_i mix[t][4o + i] * s[t][i]          dst [n][4][dim]
 *   hc_sinkhorn4x4    out[t] = Sinkhorn4x4(logits[t])        [n][16]
 *   taps3             dst[t] = Taps3 over triples[t] = (x_{t-2}, x_{t-1}, x_t)  [n][3][width]
 *   fake_a8_rows      mode 0 RmsFakeA8, 1 CenteredRmsFakeA8 (aux = scale [n]),
 *                     2 GateFakeA8 (aux = gates [rows][n]), 3 PostNormAdd
 *                     (aux = scale [n], gate [rows], dst = residual, updated). */
NDL_API int ndl_hc_mix4(const float *s, int dim, const float *w, int n, float *dst, void *stream);
NDL_API int ndl_hc_combine4(const float *s, int dim, const float *w, const float *y, const float *post, int n,
                            float *dst, void *stream);
NDL_API int ndl_hc_combine_diff4x4(const float *s, int dim, const float *mix, const float *x, const float *u,
                                   const float *post_gate, int n, float *dst, void *stream);
NDL_API int ndl_hc_sinkhorn4x4(const float *logits, int n, float *out, void *stream);
NDL_API int ndl_taps3(const float *taps, int width, const float *triples, int n, float *dst, void *stream);
NDL_API int ndl_fake_a8_rows(int mode, const float *x, const float *aux, const float *gate, int rows, int n,
                             float *dst, void *stream);

/* Engram, the Needle-3 n-gram memory (EngineCore.ApplyEngramBatch,
 * src/Needle/Engine.cs:2405-2469; EngramHashRowsBatch, :2652-2681), its own
 * three steps on device memory (the table gather, fake-A8, prep and key /
 * value matmuls are ndl_cq_gather_rows, ndl_kt_fake_a8's kernel, ndl_cq_prepare
 * and ndl_cq_matmul).  Consecutive rows with the same slot form a run.
 *   engram_hash  rows[t][table] (table = order index * heads + head) = the
 *                table row of token t's n-gram, -1 while position < order - 1;
 *                position = slot_length[slot] + offset in the run; tokens
 *                before the run come from slot_prev[slot][0..1] (the slot's
 *                last two, oldest first); orders: host array, 1..3 each.
 *   engram_conv  out[t] = sum_j taps[j] * window[9 - j*dilation], j = 0..3,
 *                window = the slot's 9 history values (history_in [slots][9]
 *                [dim]) then the run's values; each run's slot gets its new
 *                history in history_out (must not alias history_in).
 *   engram_gate  residual[t] += sigmoid(dot(RmsUnit(x), RmsUnit(key)) /
 *                sqrt(dim)) * v[t]. */
NDL_API int ndl_engram_hash(const int32_t *tokens, const int32_t *row_slots, int count, const int32_t *slot_length,
                            const int32_t *slot_prev, int slots, const int32_t *orders, int order_count, int heads,
                            int engram_slots, int32_t *rows, void *stream);
NDL_API int ndl_engram_conv(const float *history_in, const float *values, const int32_t *row_slots, int count,
                            int slots, const float *taps, int dilation, int dim, float *out, float *history_out,
                            void *stream);
NDL_API int ndl_engram_gate(const float *x, const float *key, const float *v, int count, int dim, float *residual,
                            void *stream);

/* The Needle-3 confidence head (EngineCore.PoolTokensBatch,
 * src/Needle/Engine.cs:2598-2650; ConfidenceLogitForSlot, :2702-2738) on
 * caller-owned device state, pool_rows = (layers + 1) * probes per slot:
 *   conf_pool_update  for layer row `row`: per token of each run (consecutive
 *                     rows of one slot; a slot in at most one run per call),
 *                     cell = mean of its 4 streams (streams [count][4][dim];
 *                     stream 0 for a run's first token when initial), then per
 *                     probe the online softmax of score = dot(cell, probe) /
 *                     sqrt(dim) updates pool_max / pool_sum [slots][pool_rows]
 *                     and pool_acc [slots][pool_rows][dim]; cell [slots][dim]
 *                     keeps the run's last cell.  pending [slots] (nullable):
 *                     a set slot first restores the row's pools from the
 *                     snapshot arrays; the caller clears the flags.
 *   conf_logit        per listed slot: logits[r] = bias + dot(pooled,
 *                     projection) where pooled[q] = sum_i softmax_i(dot(k_i,
 *                     query_q) / sqrt(dim) + row_bias[q][i]) * k_i and k_i =
 *                     gain[i] * RmsUnit(pool_acc_i / pool_sum_i); pooled_out
 *                     [n][queries][dim] nullable. */
NDL_API int ndl_conf_pool_update(int row, const float *streams, const int32_t *row_slots, int count, int initial,
                                 const float *probe_vectors, int probes, int dim, int pool_rows, int slots, float *cell,
                                 float *pool_max, float *pool_sum, float *pool_acc, const float *snap_max,
                                 const float *snap_sum, const float *snap_acc, const uint8_t *pending, void *stream);
NDL_API int ndl_conf_logit(const int32_t *slot_list, int n, const float *pool_sum, const float *pool_acc,
                           int pool_rows, int dim, const float *gain, const float *query_vectors,
                           const float *row_bias, float bias, const float *projection, int queries, float *logits,
                           float *pooled_out, void *stream);

/* ------------------------------------------------------------------ */
/* Batched decode engine (replaces BatchedEngine + EngineCore slots)   */
/* ------------------------------------------------------------------ */
typedef struct ndl_engine ndl_engine;

/* Synthetic decoder (I8G32 weights generated on the device from `seed`):
 * RMSNorm -> int8 QKV -> RoPE -> paged int8 KV -> attention -> int8 O ->
 * residual; RMSNorm -> int8 gate|up -> SwiGLU -> int8 down -> residual;
 * final RMSNorm -> int8 head quantized from the fp16 embedding.  With
 * `cross`, each layer adds after its self-attention residual
 * x += W_co . Attn(W_cq . RMSNorm(x), memory) over the memory attached to
 * the row's slot (the reference's cross branch, src/Needle/Engine.cs:
 * 1098-1184, with the synthetic decoder's int8 linears). */
typedef struct {
    int layers, dim, heads, head_dim, ffn, vocab;
    float rope_theta; /* <= 0 selects 10000 */
    uint64_t seed;
    int cross; /* 1: every layer has a cross-attention block (Whistle-shaped decoder) */
} ndl_decoder_config;

typedef struct {
    int device;
    int slots;     /* resident sessions (BatchedEngine slots, src/Needle/BatchEngine.cs:9-14) */
    int capacity;  /* positions per slot, a multiple of 64 */
    int kv_pages;  /* page pool size, 0 = slots * capacity / 64 */
    int max_rows;  /* rows per forward_batch */
    int max_heads; /* logits rows per forward_batch */
} ndl_engine_config;

/* Creates an engine on `device` and generates the synthetic decoder there
 * (Model.Open + new BatchedEngine, src/Needle/Model.cs:400-425,
 * src/Needle/BatchEngine.cs:9-14). */
NDL_API int ndl_engine_create(const ndl_engine_config *engine, const ndl_decoder_config *model, ndl_engine **out);
NDL_API int ndl_engine_destroy(ndl_engine *e);
/* The engine's CUDA stream (cudaStream_t as void*). */
NDL_API int ndl_engine_stream(ndl_engine *e, void **stream);
/* Device view of a named tensor (layer >= 0 for per-layer tensors): weights
 * w_qkv s_qkv w_o s_o w_gu s_gu w_d s_d attn_norm ffn_norm; global
 * final_norm embedding w_head s_head rope_cos rope_sin kv_pool page_table
 * logits.  For export and tests; the pointer stays owned by the engine. */
NDL_API int ndl_engine_tensor(ndl_engine *e, const char *name, int layer, void **ptr, size_t *bytes);
/* Synchronous host copy of the first `bytes` bytes of a named tensor. */
NDL_API int ndl_engine_read_tensor(ndl_engine *e, const char *name, int layer, void *host, size_t bytes);
NDL_API int ndl_engine_page_bytes(ndl_engine *e, size_t *bytes);
/* Waits for the engine stream and reports kernel-side status (bounds,
 * timeouts) as NDL_ERR_BOUNDS / NDL_ERR_TIMEOUT. */
NDL_API int ndl_engine_sync(ndl_engine *e);

/* Per-kernel-class device timing (CUDA events on the engine stream), the
 * B200 counterpart of the reference's IStageClock laps
 * (src/Needle/StageClock.cs:5-48).  profile_read synchronizes, adds every
 * recorded interval to ms[class] / launches[class] (arrays of
 * NDL_PROF_CLASSES, nullable) and optionally resets the totals. */
enum {
    NDL_PROF_PREPARE = 0,
    NDL_PROF_NORM_QUANT,
    NDL_PROF_GEMM_QKV,
    NDL_PROF_KV_WRITE,
    NDL_PROF_ATTENTION,
    NDL_PROF_GEMM_O,
    NDL_PROF_GEMM_GATEUP,
    NDL_PROF_SWIGLU,
    NDL_PROF_GEMM_DOWN,
    NDL_PROF_HEAD,
    NDL_PROF_SAMPLE,
    NDL_PROF_CROSS, /* the cross-attention blocks */
    NDL_PROF_CLASSES
};
NDL_API int ndl_engine_profile(ndl_engine *e, int enable);
/* Steps are captured as one CUDA graph per (rows, heads) shape and replayed
 * (default on; profiling runs the kernels directly). */
NDL_API int ndl_engine_use_graphs(ndl_engine *e, int enable);
/* Step kernels are launched with programmatic dependent launch (default on):
 * each waits for its predecessor to complete before reading anything, so
 * results are identical either way; only launch latency overlaps. */
NDL_API int ndl_engine_use_pdl(ndl_engine *e, int enable);
NDL_API int ndl_engine_profile_read(ndl_engine *e, double *ms, long long *launches, int reset);

/* Slot state: BatchedEngine.SlotLength/ResetSlot/MarkSlot/RewindSlot
 * (src/Needle/BatchEngine.cs:23-30 -> src/Needle/Engine.cs:2261-2283). */
NDL_API int ndl_slot_length(ndl_engine *e, int slot, int *length);
NDL_API int ndl_slot_reset(ndl_engine *e, int slot);
NDL_API int ndl_slot_mark(ndl_engine *e, int slot);
NDL_API int ndl_slot_rewind(ndl_engine *e, int slot);
/* Page id backing positions [64*index, 64*index+64) of a slot (-1 = none). */
NDL_API int ndl_slot_page(ndl_engine *e, int slot, int index, int *page);
/* Appends `count` synthetic prefix positions to a slot: K/V fp16 N(0,1)
 * from (seed, session) quantized per (position, head) on load. */
NDL_API int ndl_slot_fill_synthetic(ndl_engine *e, int slot, int count, uint64_t seed, uint64_t session);

/* Cross memory (Whistle-shaped decoders).  A memory slot holds one
 * utterance's encoder output projected per layer into int8 K/V pages
 * (BuildCrossMemory + per-(frame, head) quantize, src/Needle/Whistle.cs:
 * 886-914,789-790: every frame row quantized, W_ckv [2*dim][dim], each
 * head's 64 K and V values QuantizeInt8).  set_memory takes the fp16
 * [frames][dim] memory from the host; fill_memory_synthetic generates it as
 * fp16 N(0,1) from (seed, utterance) on the device.  The slot must be empty;
 * its length becomes `frames`.  attach_memory makes the rows of `slot` attend
 * to `memory_slot` (-1 detaches); beams of one utterance share it. */
NDL_API int ndl_slot_set_memory(ndl_engine *e, int slot, const uint16_t *memory, int frames);
NDL_API int ndl_slot_fill_memory_synthetic(ndl_engine *e, int slot, int frames, uint64_t seed, uint64_t utterance);
NDL_API int ndl_slot_attach_memory(ndl_engine *e, int slot, int memory_slot);
/* Copies slot `src` (its positions, pages and memory attachment) into `dst`,
 * replacing dst's content: the beam fork of Engine.CopyFrom
 * (src/Needle/Engine.cs:367-379). */
NDL_API int ndl_slot_copy(ndl_engine *e, int dst, int src);

/* Primed prefixes (Engine.PrimedPrefixBytes / ExportPrimedPrefix /
 * ImportPrimedPrefix, src/Needle/Engine.cs:398-464).  The blob holds the
 * slot's marked prefix (its length at ndl_slot_mark) in the reference's
 * layout: int32 length, then per layer keys int8 [len][heads*64], values
 * int8 [len][heads*64], key scales fp32 [len][heads], value scales fp32
 * [len][heads] (the synthetic decoders keep no recurrent engine state, so
 * the reference's state section is empty; a Needle-3 engine's blob carries
 * it, see ndl_engine_create_model).  Import replaces the slot's cache
 * and sets its length and mark to the blob's length; a short buffer or blob
 * and a length beyond the capacity are NDL_ERR_INVALID_ARG. */
NDL_API int ndl_slot_prefix_bytes(ndl_engine *e, int slot, size_t *bytes);
NDL_API int ndl_slot_export_prefix(ndl_engine *e, int slot, void *blob, size_t bytes);
NDL_API int ndl_slot_import_prefix(ndl_engine *e, int slot, const void *blob, size_t bytes);
/* Prefix sharing: `dst` (reset first) takes `src`'s marked prefix by
 * reference: whole KV pages are shared, the partial last page is copied, and
 * a later write into a shared page copies it first (copy on write).  dst's
 * length and mark become the prefix length. */
NDL_API int ndl_slot_share_prefix(ndl_engine *e, int dst, int src);
/* Times the last step's self-attention launch of `layer` alone: `reps`
 * back-to-back launches with the step's rows, pages and work list between two
 * events on the engine stream; *ms_per_launch = their average.  A measurement
 * aid (the attention roofline); it rewrites only the step's scratch outputs. */
NDL_API int ndl_engine_time_attention(ndl_engine *e, int layer, int reps, float *ms_per_launch);
/* Pool pages not held by any slot. */
NDL_API int ndl_engine_free_pages(ndl_engine *e, int *free_pages);

/* Beam search over many utterances at once: Whistle.BeamSearch
 * (src/Needle/Whistle.Decode.cs:224-350) for each utterance, every live
 * beam of every utterance in one forward_batch per step.  Utterance u uses
 * memory slot memory_slots[u] and the 2*width beam slots
 * beam_slots[u*2*width ...] (reset here).  Each beam starts from `prompt`;
 * per step the top-width of every beam's log-softmax (ids 0, 2, 3 excluded
 * when mask_special_023) extend it; candidates are ranked by score (equal
 * scores keep (beam, rank) order), eos ends a hypothesis; the search stops
 * when no beam stays live, when width hypotheses finished and the best
 * finished score/(len+1)^length_penalty beats the best live one, or after
 * max_steps.  tokens [utterances][max_steps], lengths, scores (normalised,
 * nullable) receive each utterance's winner; rows_run (nullable) the rows
 * (prompt positions and beam tokens) the search decoded. */
typedef struct {
    int width, max_steps, eos, mask_special_023;
    float length_penalty;
} ndl_beam_config;
NDL_API int ndl_beam_search(ndl_engine *e, const ndl_beam_config *cfg, int utterances, const int *memory_slots,
                            const int *beam_slots, const int32_t *prompt, int prompt_len, int32_t *tokens,
                            int *lengths, float *scores, long long *rows_run);

/* One batched step: EngineCore.ForwardBatch (src/Needle/Engine.cs:2303-2350)
 * via BatchedEngine.ForwardBatch (src/Needle/BatchEngine.cs:34).  Host
 * arrays.  Consecutive rows of one slot form a prefill run; logits are
 * computed for head_rows only (compact order).  Asynchronous on the engine
 * stream; NDL_FAIL_CONTEXT_EXHAUSTED when a slot would exceed capacity. */
NDL_API int ndl_forward_batch(ndl_engine *e, const int *tokens, const int *row_slots, int rows, const int *head_rows,
                              int heads);
/* BatchedEngine.BatchLogitsRow (src/Needle/BatchEngine.cs:37): host copy. */
NDL_API int ndl_batch_logits_row(ndl_engine *e, int compact_row, float *out);
/* Masked greedy selection on every head row of the last step
 * (Ops.ArgMaxMasked / ArgMaxMaskedWithProbability, src/Needle/Ops.cs:1223-1330).
 * masks: host [heads][words] uint32 (NULL = all allowed); probs nullable. */
NDL_API int ndl_sample_argmax(ndl_engine *e, const uint32_t *masks, int words, int *ids, float *probs);
/* Beam expansion (Ops.TopKLogSoftmax, src/Needle/Ops.cs:1092-1221) on every
 * head row: ids/log_probs/probs [heads][k], k <= 8; probs nullable. */
NDL_API int ndl_sample_topk(ndl_engine *e, int k, int mask_special_023, int *ids, float *log_probs, float *probs);

/* Per-slot vocabulary masks kept on the device, for callers that reuse one
 * mask for every step of a request (the reference's lanes keep their masks,
 * src/Needle/BatchedSession.cs:310-330).  set_mask: `words` uint32 words,
 * ids >= 32*words disallowed; NULL clears the slot's mask.
 * sample_argmax_slots: ArgMaxMasked on every head row of the last step with
 * the stored mask of slots[h] (negative or unmasked slot: no mask). */
NDL_API int ndl_engine_set_mask(ndl_engine *e, int slot, const uint32_t *mask, int words);
NDL_API int ndl_sample_argmax_slots(ndl_engine *e, const int *slots, int *ids, float *probs);

/* Grammar-constrained sparse head: Engine.LogitsForBatchRow
 * (src/Needle/Engine.cs:2683-2700; BatchedEngine.LogitsForBatchRow,
 * src/Needle/BatchEngine.cs:39-40) for n <= max_heads requests at once.
 * Request r asks for batch row rows[r] of the last forward_batch (any row,
 * head row or not) at the vocabulary ids ids[offsets[r] .. offsets[r+1])
 * (offsets[0] = 0, non-decreasing; ids in any order, repeats allowed).
 *   values: host float[offsets[n]] (nullable): the logits, equal bit for bit
 *           to the dense head's logits of that row at those ids.
 *   picks:  host int[n] (nullable): ArgMaxSparse
 *           (src/Needle/NeedleSession.cs:984-995), the first listed id
 *           holding the strict maximum, -1 for an empty list.
 *   probs:  host float[n] (nullable, needs picks): BestProbability over the
 *           request's values (0 for an empty list).
 * Errors: NDL_ERR_INVALID_ARG for a row outside the last step, an id outside
 * the vocabulary or decreasing offsets.  Synchronous. */
NDL_API int ndl_logits_sparse(ndl_engine *e, int n, const int *rows, const int *offsets, const int *ids,
                              float *values, int *picks, float *probs);

/* Engine limits. */
typedef struct {
    int slots, capacity, vocab, max_rows, max_heads, layers, dim, heads;
} ndl_engine_info;
NDL_API int ndl_engine_get_info(ndl_engine *e, ndl_engine_info *info);

/* ------------------------------------------------------------------ */
/* Continuous batching (replaces BatchedSession.RunBatch's loop,       */
/* src/Needle/BatchedSession.cs:218-268)                               */
/* ------------------------------------------------------------------ */
/* Each step packs every running request's decode row, then prompt chunks
 * (at most prefill_chunk positions of one request per step) up to max_rows,
 * runs one ndl_forward_batch and samples every head row with the request's
 * mask.  A request's tokens equal those it gets alone (rows are batch
 * invariant).  One host thread per scheduler. */
typedef struct ndl_sched ndl_sched;
typedef struct {
    int max_rows;      /* rows per step, <= the engine's max_rows and max_heads */
    int prefill_chunk; /* prompt positions of one request per step */
} ndl_sched_config;
typedef struct {
    int request;
    int kind;   /* 1: first token produced, 2: request finished */
    int token;  /* the token of this step (-1 if none) */
    int status; /* kind 2: 0 or a FailureReason (3 = ContextExhausted) */
} ndl_sched_event;
NDL_API int ndl_sched_create(ndl_engine *e, const ndl_sched_config *cfg, ndl_sched **out);
/* A scheduler without an engine: plans steps and returns token
 * (request * 7919 + produced) % vocab; for testing the packing on a host. */
NDL_API int ndl_sched_create_dry(const ndl_sched_config *cfg, int slots, int capacity, int vocab, ndl_sched **out);
NDL_API int ndl_sched_destroy(ndl_sched *s);
/* Queues a request (arrival order = admission order).  mask: `mask_words`
 * words, NULL = unmasked; stop_token < 0: none; generation ends after
 * max_new_tokens tokens or the stop token. */
NDL_API int ndl_sched_submit(ndl_sched *s, int request, const int32_t *prompt, int prompt_len, int max_new_tokens,
                             int stop_token, const uint32_t *mask, int mask_words);
/* Jump-forward (NeedleSession.GenerateCalls, src/Needle/NeedleSession.cs:
 * 538-662): `count` tokens the caller's grammar forces after a decoding
 * request's last pick (its mask allows one id at each), appended to the
 * request's output without logits.  The next step feeds the pick and the
 * forced tokens as one run of the request's slot and samples only at the
 * run's last row; the stream equals feeding them one per step.  Forced
 * tokens count toward max_new_tokens and end the request at the stop token.
 * NDL_ERR_INVALID_ARG for a request that is not decoding or a token outside
 * the vocabulary. */
NDL_API int ndl_sched_force(ndl_sched *s, int request, const int32_t *tokens, int count);
/* Runs one step (none if nothing is queued or running): events of this step
 * (at most `capacity` written, *count = all), rows and decode rows packed. */
NDL_API int ndl_sched_step(ndl_sched *s, ndl_sched_event *events, int capacity, int *count, int *rows,
                           int *decode_rows);
/* Tokens produced so far by a request (capacity entries at most; *count = all). */
NDL_API int ndl_sched_tokens(ndl_sched *s, int request, int32_t *tokens, int capacity, int *count);
NDL_API int ndl_sched_pending(ndl_sched *s, int *waiting, int *running);
/* The last step's packing (arrays of max_rows, nullable). */
NDL_API int ndl_sched_last_plan(ndl_sched *s, int *tokens, int *row_slots, int *rows, int *head_rows, int *heads);

/* ---- Needle-3 model archive (.cact) -------------------------------------
 * Replaces Model.FromBytes / FromMemory (src/Needle/Model.cs:307-404): the
 * record table is walked in the reference's order and each tensor is named
 * by its role and index (layer, site or probe head), e.g. "embedding" 0,
 * "layer.q" l, "layer.mlp.cond_u" l, "hyper.phi_pre" 0, "hyper.perm_a" 0,
 * "site.tables" s, "final_norm" 0, "manifest" 0, "probe.probe_vectors" h,
 * "audio" k (an audio section's records, untyped).  The archive is checked
 * with the reference's checks and messages: NDL_ERR_MALFORMED_MODEL where
 * it throws InvalidDataException (short, wrong magic, truncated, a record
 * of the wrong kind, no tokenizer) and NDL_ERR_UNSUPPORTED where it throws
 * NotSupportedException (head, MLP and convolution geometry; more than 4
 * orders or 16 sites).  Also malformed, where the reference reads out of
 * range: a walk past the table, a tensor larger than its bytes, fewer than
 * 28 codebook levels, a permutation entry outside [0, HadaN).
 * device >= 0 uploads the weights to that device in one allocation:
 *  - CQ codes and fp16 norms as stored, for ndl_cq_matmul / ndl_cq_gather_rows,
 *    with a host codebook;
 *  - dense tensors as fp32, converted by Scalar.HalfToSingle, or by
 *    HalfToSingleUpstream before the audio section of an audio-carrying
 *    archive;
 *  - permutations as int32;
 *  - the probe heads' CQ matrices also decoded to fp32 rows (Reader.Rows).
 * device < 0 parses and checks on the host only.  The archive is not
 * referenced after the call returns.  "layer.attn_gate" is the stored logit:
 * the reference keeps its sigmoid. */
typedef struct ndl_model ndl_model;
enum {
    NDL_TENSOR_DENSE = 0,       /* fp32 values [count] */
    NDL_TENSOR_CQ = 1,          /* indices, norms, book; rows x cols, bits */
    NDL_TENSOR_PERMUTATION = 2, /* int32 [count] */
    NDL_TENSOR_CQ_ROWS = 3,     /* a CQ matrix and its decoded rows: values [rows][cols] */
    NDL_TENSOR_RAW = 4
};
typedef struct {
    uint32_t magic;
    int tensors, codebook_entries;
    int64_t length, tokenizer_bytes;
    int has_audio, has_confidence, has_embedding_head;
    int probe_heads, confidence_head, embedding_head; /* head indices, -1: none */
    int probe_codes[16];                              /* ProbeHead codes: 1 embedding, 2 confidence, 3 router */
    /* Geometry (src/Needle/Model.cs:65-120), header words 3..48 */
    int vocab, dim, heads, kv_heads, layers, qk_dim, v_dim, max_seq, hada_n, lanes;
    int sliding_window, conv_taps, engram_slots, engram_sub, engram_tables;
    int engram_conv_taps, engram_dilation, engram_seed_heads, kv_window;
    int order_count, site_count;
    uint64_t global_mask;
    float rope_theta;
    int orders[4], sites[16];
    int hada_rows, hada_cols;
    int device; /* -1: host only */
    size_t device_bytes;
} ndl_model_info;
typedef struct {
    int kind, record, dtype, ndim;
    int64_t shape[4];
    uint64_t offset, bytes; /* the record's bytes in the archive */
    int64_t count;          /* elements of values / permutation */
    int rows, cols, bits;   /* CQ */
    /* device addresses after an upload (NULL otherwise) */
    const float *values;
    const int32_t *permutation;
    const uint8_t *indices;
    const uint16_t *norms;
    const ndl_kt_codebook *book; /* host */
} ndl_model_tensor;
NDL_API int ndl_model_load(const void *archive, size_t bytes, int device, ndl_model **out);
NDL_API int ndl_model_destroy(ndl_model *m);
NDL_API int ndl_model_get_info(const ndl_model *m, ndl_model_info *info);
NDL_API int ndl_model_tensor_count(const ndl_model *m, int *count);
NDL_API int ndl_model_tensor_name(const ndl_model *m, int i, const char **role, int *index);
NDL_API int ndl_model_get_tensor(const ndl_model *m, const char *role, int index, ndl_model_tensor *t);
/* The host copy of a dense (fp32) or permutation (int32) tensor. */
NDL_API int ndl_model_read_host(const ndl_model *m, const char *role, int index, void *destination, size_t bytes);
/* The tokenizer record's bytes (owned by the model). */
NDL_API int ndl_model_tokenizer(const ndl_model *m, const void **blob, size_t *bytes);

/* ---- Whistle encoder ---------------------------------------------------
 * Replaces Whistle.Encode + BuildCrossMemory (src/Needle/Whistle.cs:179-200,
 * 886-914) for a loaded archive with an audio section (AudioWeights,
 * src/Needle/Audio.cs:117-149), on the model's device: the log-mel front end
 * (FeatureJob, src/Needle/Frontend.cs:82-130), Normalize, the three-stage
 * stem, the encoder layers (RunEncoder, :794-828) and the final norm, then
 * every decoder layer's cross memory (int8 keys and values per (frame,
 * head) with fp32 scales, the layout of CrossMemory).  The scalar tier
 * throughout, with MathF.Exp and MathF.Log as the correctly rounded
 * functions, so every output equals the scalar chain bit for bit.
 * create: max_samples bounds the PCM per call (at most the reference's 30 s);
 * encode: host or device PCM samples in [-1, 1] (the first 30 s kept);
 *   *frames = encoder rows ((((samples / hop) + 1) / 2 + 1) / 2 + 1) / 2, 0
 *   below one hop; returns when the work is done.  encode_device queues the
 *   same work on ndl_whistle_stream without waiting (pcm device or host).
 * read: copies a result to host memory (bytes at least its size, *written
 *   its size): NDL_WHISTLE_MEL [mel frames][mels] after Normalize, _STEM
 *   [frames][dim], _ENCODER [frames][dim], and of decoder layer `layer`
 *   _KEYS int8 [frames][heads][qk], _KEY_SCALES fp32 [frames][heads],
 *   _VALUES int8 [frames][heads][v], _VALUE_SCALES fp32 [frames][heads].
 * NDL_ERR_UNSUPPORTED for an archive without audio or a geometry the device
 * encoder does not take (CQ widths not in 128-column groups, dim > 1024,
 * head dims > 64, more than 128 mels, fft > 4096 or not a power of two), or a
 * max_samples whose first stem stage (half the mel frames x 40 x the stem
 * width) would hold 2^31 elements or more. */
typedef struct ndl_whistle ndl_whistle;
enum {
    NDL_WHISTLE_MEL = 0,
    NDL_WHISTLE_STEM = 1,
    NDL_WHISTLE_ENCODER = 2,
    NDL_WHISTLE_KEYS = 3,
    NDL_WHISTLE_KEY_SCALES = 4,
    NDL_WHISTLE_VALUES = 5,
    NDL_WHISTLE_VALUE_SCALES = 6
};
NDL_API int ndl_whistle_create(const ndl_model *m, int max_samples, ndl_whistle **out);
NDL_API int ndl_whistle_encode(ndl_whistle *w, const float *pcm, int samples, int *frames);
NDL_API int ndl_whistle_encode_device(ndl_whistle *w, const float *pcm, int samples);
NDL_API int ndl_whistle_frames(const ndl_whistle *w, int *frames, int *mel_frames);
NDL_API int ndl_whistle_read(ndl_whistle *w, int what, int layer, void *dst, size_t bytes, size_t *written);
NDL_API void *ndl_whistle_stream(ndl_whistle *w);
NDL_API int ndl_whistle_destroy(ndl_whistle *w);

/* The Engram block of one site on a loaded model (EngineCore.ApplyEngramBatch,
 * src/Needle/Engine.cs:2405-2469), chained on `stream` over `count` tokens:
 *   rows = the n-gram hash rows (ndl_engram_hash, the model's orders, heads
 *          and table size);
 *   e[t] = FakeA8 of [GatherRow(site.tables, rows[t][0]) | ... ] (a -1 row
 *          gathers zeros);
 *   key, value = site.key / site.value times e prepared at 2 bits (CQ);
 *   conv = the dilated 4-tap conv of value over the slot's 9-entry history
 *          (ndl_engram_conv: history_out gets the batch slots' new
 *          histories, other slots' entries are left as they are);
 *   residual[t] += sigmoid(dot(RmsUnit(x[t]), RmsUnit(key[t])) / sqrt(dim)) * conv[t].
 * tokens, row_slots [count]; slot_length [slots]; slot_prev [slots][2];
 * history_in / history_out [slots][9][dim] (this site's); x, residual
 * [count][dim]: device memory.  workspace: device memory of at least
 * ndl_engram_workspace(m, count) bytes, 256-byte aligned.  The model must be
 * on a device; its tables must tile the input (EngramTables x EngramSub ==
 * Dim) and its key / value matrices be 2-bit Dim x Dim, else
 * NDL_ERR_UNSUPPORTED.  Bit-exact to the scalar chain, the gate's sigmoid
 * included (MathF.Exp as the correctly rounded exponential). */
/* HadamardMlp.Apply (src/Needle/Blocks.cs:1067-1093) on `count` residual
 * rows [count][Dim] (device memory, updated in place) with layer `layer`'s
 * MLP factors and pre-norm scale and the model's two permutations; `scale`
 * as MlpBatch.Scale.  One block per row, the same kernel as the KernelTable
 * slot (inner sums in the scalar order, MathF.Exp correctly rounded: bit for
 * bit the scalar code).  A tensor shorter than the HadaRows x HadaCols
 * split needs is NDL_ERR_UNSUPPORTED. */
NDL_API int ndl_mlp_apply(const ndl_model *m, int layer, float *residual, int count, float scale, void *stream);
NDL_API size_t ndl_engram_workspace(const ndl_model *m, int count);
NDL_API int ndl_engram_apply(const ndl_model *m, int site, const int32_t *tokens, const int32_t *row_slots, int count,
                             const int32_t *slot_length, const int32_t *slot_prev, int slots, const float *history_in,
                             float *history_out, const float *x, float *residual, void *workspace,
                             size_t workspace_bytes, void *stream);

/* A batched decode engine over a loaded Needle-3 model (Model.Open + new
 * BatchedEngine on a real archive; src/Needle/Model.cs:400-425,
 * src/Needle/BatchEngine.cs:9-14).  ndl_forward_batch then runs
 * EngineCore.ForwardBatch with RunLayerBatch (src/Needle/Engine.cs:
 * 2303-2596) on the device in the reference's scalar tier, bit for bit:
 * embedding GatherRow and scale, the hyper-connection prepare / phi matmuls /
 * gates / Mix4 / Sinkhorn, Engram at its site layers, attention (CQ
 * projections, 3-tap convs over each slot's two previous projections,
 * ZeroCenteredRms and RoPE per head, an int8 K / V cache per slot, grouped
 * heads with the sliding window on local layers, the gated output and
 * PostNormAdd), the Kronecker MLP and CombineDiff4x4, then the head rows'
 * logits over the vocabulary (PrepareHeadVectors and the tied embedding).
 * A run of rows of one slot is equivalent to feeding them one at a time, and
 * is computed that way.  Slot state (lengths, previous tokens, conv and
 * Engram histories, K / V cache) is per slot on the device; ndl_slot_reset
 * clears it, ndl_slot_mark / ndl_slot_rewind keep and restore it
 * (MarkView / RewindView, src/Needle/Engine.cs:2235-2255), and the primed-
 * prefix calls move a slot's marked prefix as the reference's blob with its
 * state section: int32 length; per layer the conv histories q | k | v (two
 * entries each, fp32); per Engram site the 9-entry history; the previous two
 * tokens; the confidence pools at their reset values (this engine does not
 * pool); then per layer keys [len][kv*qk], values [len][kv*v], key and value
 * scales [len][kv].  Sampling, masks, top-k and ndl_batch_logits_row work as
 * on the synthetic decoder.  Not available on this engine
 * (NDL_ERR_UNSUPPORTED): slot copies and shared prefixes, cross memory, the
 * sparse head, the page / tensor views and the attention timer.  The model must stay loaded while
 * the engine lives; capacity is at most 8192 and the model's head dims at
 * most 64. */
NDL_API int ndl_engine_create_model(const ndl_engine_config *engine, const ndl_model *model, ndl_engine **out);

#ifdef __cplusplus
}
#endif
#endif
