// Internal launch helpers shared between translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ndl {

int launch_quantize_rows(const float *x, const float *weight, int rows, int cols, int8_t *q, float *scales,
                         cudaStream_t stream);
// NDL_ERR_UNSUPPORTED when the CTA-per-row kernel cannot take the shape.
int launch_swiglu_quantize_rows(const float *gu, int rows, int ffn, int8_t *q, float *scales, cudaStream_t stream);

struct MatmulArgs {
    const int8_t *q;
    const float *sa;
    int m, k;
    const int8_t *w;
    const uint16_t *sw;
    int n;
    float *y;
    int ldy;
    const float *residual;
    int32_t *acc;
    long long w_stride, sw_stride, y_stride;
    int batch;
    int *status;  // nullable: kernels record timeouts here
};

// RoPE + int8 quantize of q (per head) and k, v (per position and head) into
// the paged cache.  qkv rows are [q heads | k heads | v heads].
struct KvWriteArgs {
    const float *qkv;
    int ld_qkv;
    const int32_t *row_slot, *row_pos;
    const int32_t *page_table;
    int max_pages;
    uint8_t *pool;
    long long page_bytes;
    int num_pages;
    const float *rope_cos, *rope_sin;  // [positions][32]
    int layer, heads, rows;
    int8_t *q8;  // [rows][heads][64]
    float *qs;   // [rows][heads]
    int *status;
};
int launch_kv_write(const KvWriteArgs &a, cudaStream_t stream);
// Cross-attention queries (per-head quantize, no RoPE) and the memory K/V of
// one layer written into a memory slot's pages.
int launch_cross_query(const float *q, int ldq, int heads, int rows, int8_t *q8, float *qs, cudaStream_t stream);
int launch_cross_kv_write(const float *y, int frames, int heads, const int32_t *page_row, int num_pages, uint8_t *pool,
                          long long page_bytes, int layer, int *status, cudaStream_t stream);

// The attention work list: one record per row position of the launch's row
// order, {row, attended positions, slot, pages (0: an out-of-range row)}
// followed by the row's page ids, padded to 16 bytes.  Built once per step
// by launch_attn_work; the kernel deals its (row, head) items dynamically.
__host__ __device__ __forceinline__ int attn_record_ints(int max_pages) { return 4 + ((max_pages + 3) & ~3); }
// Positions one (row, head) may attend to: its scores stay in shared memory.
constexpr int kAttnMaxPositions = 8192;

struct AttnArgs {
    const int8_t *q;  // [rows][heads][64], dims in k_slot order
    const float *qs;  // [rows][heads]
    const int32_t *row_slot, *row_pos, *row_order;
    const int32_t *page_table;
    int max_pages;
    const uint8_t *pool;
    long long page_bytes;
    int num_pages;
    int layer, heads, rows;
    float inv_sqrt_d;
    float *out;       // [rows][heads][64]
    int *status;
    int slots;        // rows of page_table (bounds check)
    // nullable: the row's heads x 64 outputs quantized per row
    // (Scalar.QuantizeInt8), the o-projection's input
    int8_t *q_out;    // [rows][heads * 64]
    float *s_out;     // [rows]
    int32_t *work;    // [rows][attn_record_ints(max_pages)]
    int *n_work;      // int[4]: the item count, the next dynamically dealt item, finished CTAs, unused
};
// Primed-prefix blobs (prefix.cu): bytes of a blob of `len` positions, and
// the move of a slot's first `len` positions between its pages and a blob
// (to_blob) or back.
size_t prefix_blob_bytes(int layers, int heads, int len);
int launch_prefix_move(bool to_blob, int layers, int heads, int len, const int32_t *pages, uint8_t *pool,
                       long long page_bytes, int num_pages, uint8_t *blob, int *status, cudaStream_t stream);

// Builds the work list of a launch shape (one small launch; the engine
// builds it once per step and reuses it for every layer).
int launch_attn_work(const AttnArgs &a, cudaStream_t stream);
// build_work: launch_attn_work first (callers without a prebuilt list);
// quantize: also quantize the outputs per row into q_out, s_out after it.
int launch_attn_decode(const AttnArgs &a, cudaStream_t stream, bool build_work = true, bool quantize = true);
// The per-row quantize of the attention outputs into q_out, s_out.
int launch_attn_quantize(const AttnArgs &a, cudaStream_t stream);

// Streaming int8 GEMV (mma.sync m16n8k32 per 32-column group), any m.
int launch_gemv_i8g32(const MatmulArgs &a, cudaStream_t stream);
// tcgen05 kind::i8 GEMM for m >= 64; returns NDL_ERR_UNSUPPORTED when the
// shape does not fit its tiling so the caller can fall back to the GEMV.
int launch_gemm_i8g32_tc(const MatmulArgs &a, cudaStream_t stream);

// CQ Prepare (Quant.PrepareRange's scalar branch) and MatMulRows on one
// matrix (ndl_cq_prepare / ndl_cq_matmul without the argument checks).
int launch_cq_prepare(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales, float *offsets,
                      int stride, cudaStream_t stream);
int launch_cq_matmul(const uint8_t *indices, const uint16_t *norms, const uint8_t *book_bytes, float byte_scale,
                     int cols, int bits, const int8_t *values, const float *scales, const float *offsets, int stride,
                     int tokens, float *y, int ldy, int row_start, int row_end, cudaStream_t stream);
// One CQ matrix (or row slice of one) for launch_cq_matmul_jobs: rows
// [row_start, row_end) of y [tokens][ldy] from the shared prepared
// activations; book_bytes is the host copy of the 16 codebook bytes.
struct CqMatmulJob {
    const uint8_t *indices;
    const uint16_t *norms;
    const uint8_t *book_bytes;
    float byte_scale;
    float *y;
    int ldy, row_start, row_end;
};
// Where a row op writes CQ Prepare's output (values [rows][n], scales and
// offsets [rows][stride]) instead of its rows.
struct CqPrepOut {
    int8_t *values;
    float *scales, *offsets;
    int stride, bits;
};
// CTA-per-row row ops (n % 4 == 0, n <= 4096, 16-byte aligned rows; n % 128
// == 0 with prep): mode 0 RmsUnit, 1 ZeroCenteredRms (aux = scale), 2
// MultiplyBySigmoid (aux = gate rows), 3 PostNormAdd (aux = scale, dst =
// residual, gate[row]; fake and prep not allowed), 4 ZeroCenteredRms then
// SiLU, 5 the row unchanged; fake adds Quant.FakeA8; prep (nullable) sends
// the rows into CQ Prepare instead of dst.  NDL_ERR_UNSUPPORTED (nothing
// launched) for a shape or alignment the kernel does not take.
int launch_row_op(int mode, bool fake, const float *x, const float *aux, const float *gate, int rows, int n,
                  float *dst, const CqPrepOut *prep, cudaStream_t stream);
// ndl_fake_a8_rows modes 0..2 followed by CQ Prepare of the rows, in one
// launch; NDL_ERR_UNSUPPORTED (nothing launched) unless n % 128 == 0,
// n <= 4096 and x / aux sit on 16-byte boundaries.
int launch_fake_a8_prepare(int mode, const float *x, const float *aux, int rows, int n, int bits, int8_t *values,
                           float *scales, float *offsets, int stride, cudaStream_t stream);
// The hyper-connection prepare of a layer after its phi matmuls, CTA per
// row: the pre / post gates and Sinkhorn logits of `layer` (pre, post [rows]
// [ld] with the layer's 4 at 4 * layer, res with its 16 at 16 * layer), u =
// Mix4(stream, hpre) also written to residual, mix = Sinkhorn4x4(logits).
int launch_hc_prepare(const float *pre, int ld_pre, const float *post, int ld_post, const float *res, int ld_res,
                      const float *a_pre, const float *b_pre, const float *a_post, const float *b_post,
                      const float *a_res, const float *b_res, int layer, const float *stream, int dim, int rows, float *u,
                      float *residual, float *post_gate, float *mix, cudaStream_t cs);
// HadamardMlp.Apply's operands (block b works on row b).  Optional around
// it, per row: a PostNormAdd before (pn_x non-null: residual += pn_gate[row]
// ((1 + pn_scale) pn_x) InverseRms(pn_x)) and a CombineDiff4x4 after
// (cb_next non-null: next lanes from the row's stream, mix, the final
// residual, u and post gates).
struct KtMlpArgs {
    const float *w[13];
    const float *pre_norm;
    const int32_t *perm_a, *perm_b;
    int dim, rows, cols;
    float scale;
    float *residual;
    long long row_stride;  // block b updates residual + b * row_stride (0: one row)
    const float *pn_x, *pn_scale, *pn_gate;
    const float *cb_stream, *cb_mix, *cb_u, *cb_post;
    float *cb_next;
};
int launch_slot_hadamard_mlp(const KtMlpArgs &a, cudaStream_t stream);
// The same kernel over `count` rows (a.row_stride apart).
int launch_mlp_rows(const KtMlpArgs &a, int count, cudaStream_t stream);
// HadamardMlp.Apply on `count` residual rows with explicit factors (d1, d2,
// b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b, cond_v, cond_u), block per row.
int launch_hadamard_mlp_rows(const float *const w[13], const float *pre_norm, const int32_t *perm_a,
                             const int32_t *perm_b, int dim, int rows, int cols, float scale, float *residual, int count,
                             cudaStream_t stream);
// Several matrices of the same width and bits over one Prepare, few launches.
int launch_cq_matmul_jobs(const CqMatmulJob *jobs, int n_jobs, int cols, int bits, const int8_t *values,
                          const float *scales, const float *offsets, int stride, int tokens, cudaStream_t stream);

}  // namespace ndl
