/*
 * needle_oracle.h - CPU restatement of the needle-cs batched decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA path in needle-cs_b200/.  It is imported by tests/, by
 * __graft_entry__.smoke() and by the cpu_baseline / --impl reference legs of
 * bench.py, and by nothing else.  The shipped library never links it.
 *
 * Every function restates one reference routine; the reference location is
 * cited per function (paths are relative to the needle-cs source tree).
 * Floating point follows the reference's scalar C# semantics: IEEE binary32,
 * no FMA contraction (compile with -ffp-contract=off), left-to-right
 * summation, MathF.Cos/Sin/Pow mapped to the C library's cosf/sinf/powf
 * (which is what .NET calls on Linux), and MathF.Exp to exp_rn, the float
 * exponential rounded to nearest, computed from the mathematics with IEEE
 * double operations (needle_oracle.c).  The decoder's attention and SiLU
 * restate the reference's AVX2 tier instead (Attention.GroupAvx2 and the
 * vector Silu/Glu, with Ops.Exp): fused multiply-adds where it uses them,
 * its partial sums in its order.
 */
#ifndef NEEDLE_ORACLE_H
#define NEEDLE_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- test-input generators (tests/Needle.Tests/Conformance/Conformance.cs:10-119) ---- */
uint64_t ndo_xorshift_next(uint64_t *state);
int ndo_xorshift_int(uint64_t *state, int lo, int hi);
float ndo_xorshift_float(uint64_t *state, float scale);
void ndo_fill_uniform(float *x, int n, uint64_t *state, float scale);
void ndo_fill_edges(float *x, int n, uint64_t *state, float scale);
void ndo_fill_sbyte(int8_t *x, int n, uint64_t *state, int extremes);
void ndo_fill_bytes(uint8_t *x, int n, uint64_t *state, int extremes);
uint16_t ndo_half_bits(float value);

/* ---- the benchmark configs' synthetic inputs (counter-based generator) ---- */
void ndo_synth_normal(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale, float *out);
void ndo_synth_uniform(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo, float hi, float *out);
void ndo_synth_int8(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out);

/* ---- the exponential (MathF.Exp) over an array ---- */
void ndo_exp_rn(const float *x, int n, float *y);
void ndo_exp_simd(const float *x, int n, float *y);

/* ---- row primitives (src/Needle/Scalar.cs) ---- */
float ndo_abs_max(const float *x, int n);
float ndo_quantize_int8(const float *x, int n, int8_t *dst);
void ndo_quantize_rows(const float *x, int rows, int cols, int8_t *q, float *scales);
float ndo_fake_a8(float *x, int n);
float ndo_half_to_single(uint16_t half);
void ndo_hadamard128(const float *src, float *dst);
void ndo_planes(const int8_t *quantized, int bits, int8_t *dst, int *sum);
float ndo_sigmoid(float x);
void ndo_softmax(float *s, int n);
void ndo_rope(float *x, int heads, int head_dim, const float *cos_t, const float *sin_t);
void ndo_rope_tables(float theta, int qk_dim, int positions, float *cos_t, float *sin_t);
float ndo_inverse_rms(const float *x, int n);
void ndo_rms_norm(const float *x, const float *weight, int n, float *dst);
void ndo_zero_centered_rms(const float *x, const float *scale, int n, float *dst);
void ndo_swiglu(const float *gate, const float *up, int n, float *dst);

/* ---- quantized matmul ---- */
/* Codebook (src/Needle/Model.cs:36-52). */
typedef struct {
    float levels[16];
    uint8_t bytes[32];
    float byte_scale;
} ndo_codebook;
void ndo_codebook_fill(ndo_codebook *book, const float *levels, int count);
/* Needle-3 row ops (Scalar.cs:250-439, Ops.cs:800-812) */
void ndo_mix4(const float *s, int dim, float w0, float w1, float w2, float w3, float *dst);
void ndo_combine4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *y, float post,
                  float *dst);
void ndo_combine_diff4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *x,
                       const float *u, float post, float *dst);
void ndo_combine_diff4x4(const float *s, int dim, const float *mix, const float *x, const float *u,
                         const float *post_gate, float *dst);
void ndo_taps3(const float *taps, int width, const float *current, float *dst);
void ndo_sinkhorn4x4(const float *logits, float *result);
void ndo_rms_fake_a8(const float *x, int n, float *dst);
void ndo_centered_rms_fake_a8(const float *x, const float *scale, int n, float *dst);
void ndo_gate_fake_a8(float *x, const float *gate, int n);
void ndo_post_norm_add(float *residual, const float *x, const float *scale, float gate, int n);
void ndo_engram_hash(const int32_t *tokens, const int32_t *row_slots, int count, const int32_t *slot_length,
                     const int32_t *slot_prev, const int32_t *orders, int order_count, int heads, int engram_slots,
                     int32_t *rows); /* Engine.cs:2652-2681 */
void ndo_engram_conv(const float *history_in, const float *values, const int32_t *row_slots, int count,
                     const float *taps, int dilation, int dim, float *out, float *history_out); /* Engine.cs:2421-2453 */
void ndo_engram_gate(const float *x, const float *key, const float *v, int dim, float *residual); /* Engine.cs:2455-2466 */
void ndo_conf_pool_update(int row, const float *streams, const int32_t *row_slots, int count, int initial,
                          const float *probe_vectors, int probes, int dim, int pool_rows, float *cell, float *pool_max,
                          float *pool_sum, float *pool_acc, const float *snap_max, const float *snap_sum,
                          const float *snap_acc, const uint8_t *pending); /* Engine.cs:2598-2650 */
float ndo_conf_logit(const float *pool_sum, const float *pool_acc, int pool_rows, int dim, const float *gain,
                     const float *query_vectors, const float *row_bias, float bias, const float *projection,
                     int queries, float *pooled_out); /* Engine.cs:2702-2738 */
void ndo_hadamard_mlp(const float *const *w, const float *pre_norm, const int32_t *perm_a, const int32_t *perm_b,
                      int dim, int rows, int cols, float scale, float *residual); /* Blocks.cs:1067-1093 */
void ndo_gather_row_cq(const uint8_t *indices, const uint16_t *norms, const float *levels, int cols, int bits, int row,
                       float *dst); /* Quant.cs:566-576 */

/* CQ activations prepare, scalar branch (src/Needle/Quant.cs:471-484). */
void ndo_prepare_cq(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales,
                    float *offsets, int stride);
/* CQ MatMulRows (src/Needle/Scalar.cs:146-192). */
void ndo_matmul_rows_cq(const uint8_t *indices, const uint16_t *norms, const ndo_codebook *book, int rows,
                        int cols, int bits, const int8_t *values, const float *scales, const float *offsets,
                        int stride, int tokens, float *y, int ldy, int row_start, int row_end);
/* I8G32: int8 weights [N][K], fp16 scale per (row, 32-column group).  Same
 * skeleton as Scalar.MatMulRows with a 32-group and raw int8 weights:
 *   D[t][n][g] = sum_{k in g} w[n][k] * q[t][k]                   (int32)
 *   y[t][n]    = sa[t] * (fma over g ascending of half(sw[n][g]) * D)  (fp32)
 * acc (nullable) receives D as [M][N][K/32]. */
void ndo_matmul_i8g32(const int8_t *w, const uint16_t *sw, int n_rows, int k, const int8_t *q, const float *sa,
                      int m, int32_t *acc, float *y, int ldy);

/* ---- attention ---- */
/* Scalar.AttentionHead (src/Needle/Scalar.cs:290-312) with qk/v widths as
 * parameters; inv_sqrt_dim replaces the hard-coded 1/sqrt(48). */
void ndo_attention_head(const int8_t *query, float query_scale, const int8_t *keys, const float *key_scales,
                        const int8_t *values, const float *value_scales, int key_stride, int value_stride,
                        int scale_stride, int first, int last, int qk_dim, int v_dim, float inv_sqrt_dim,
                        float *scores, float *output, float *probabilities);
void ndo_attention_head_simd(const int8_t *query, float query_scale, const int8_t *keys, const float *key_scales,
                             const int8_t *values, const float *value_scales, int key_stride, int value_stride,
                             int scale_stride, int first, int last, int qk_dim, int v_dim, float inv_sqrt_dim,
                             float *scores, float *output);
/* Attention.MergePartials scalar branch (src/Needle/Blocks.cs:750-817):
 * partial c = {out[heads*64] at c*stride, peak[h] at c*stride+peak_off,
 * sum[h] at c*stride+peak_off+8}. */
void ndo_merge_partials(const float *partials, int count, int heads, int stride, int peak_off, float *output);

/* ---- sampling ---- */
int ndo_argmax(const float *x, int n);                                       /* Ops.cs:1052-1090 scalar tail */
int ndo_argmax_masked(const float *x, const uint32_t *mask, int words, int length); /* Ops.cs:1236-1265 */
float ndo_best_probability(const float *values, int count, float best);      /* Ops.cs:1530-1535 */
int ndo_argmax_sparse(const float *values, const int32_t *rows, int count,
                      float *probability);                                   /* NeedleSession.cs:984-995 */
int ndo_argmax_masked_with_probability(const float *x, const uint32_t *mask, int words, int length,
                                       float *scratch, float *probability);  /* Ops.cs:1302-1330 */
void ndo_topk_logsoftmax(const float *x, int n, int k, int *indices, float *log_probs, float *probs,
                         int mask_special_023);                              /* Ops.cs:1092-1221 */

/* ---- synthetic decoder step ---- */
typedef struct {
    int layers, dim, heads, head_dim, ffn, vocab;
    float rope_theta, eps;
    /* per layer l (arrays of length layers): */
    const int8_t **w_qkv;  const uint16_t **s_qkv;   /* [3*dim][dim]      */
    const int8_t **w_o;    const uint16_t **s_o;     /* [dim][dim]        */
    const int8_t **w_gu;   const uint16_t **s_gu;    /* [2*ffn][dim]      */
    const int8_t **w_d;    const uint16_t **s_d;     /* [dim][ffn]        */
    const float **attn_norm, **ffn_norm;             /* [dim]             */
    const float *final_norm;                         /* [dim]             */
    const uint16_t *embedding;                       /* fp16 [vocab][dim] */
    const int8_t *w_head; const uint16_t *s_head;    /* [vocab][dim]      */
    /* cross-attention blocks (Whistle-shaped decoder; NULL w_cq: none):    */
    const int8_t **w_cq;   const uint16_t **s_cq;    /* [dim][dim]        */
    const int8_t **w_ckv;  const uint16_t **s_ckv;   /* [2*dim][dim]      */
    const int8_t **w_co;   const uint16_t **s_co;    /* [dim][dim]        */
    const float **cross_norm;                        /* [dim]             */
} ndo_decoder;

/* One decoder layer stack + head for one row at absolute position `pos`.
 * kv_k/kv_v: int8 [layers][capacity][heads*head_dim]; kv_ks/kv_vs: fp32
 * [layers][capacity][heads] (the reference slot layout,
 * src/Needle/Engine.cs:184-187,220-223). Positions [0,pos) must be filled;
 * this call writes position pos (KV write, src/Needle/Engine.cs:2552-2569)
 * and writes logits [vocab]. Returns 0, or -1 if scratch allocation failed. */
int ndo_decoder_row(const ndo_decoder *m, int token, int pos, int capacity, int8_t *kv_k, int8_t *kv_v,
                    float *kv_ks, float *kv_vs, const float *rope_cos, const float *rope_sin, float *logits);

/* The same row for a decoder with cross-attention blocks: after the
 * self-attention residual of layer l, x += W_co . Attn(W_cq . RMSNorm(x),
 * memory of layer l) over all `frames` memory positions (the reference's
 * cross branch, src/Needle/Engine.cs:1098-1184: Position 0, Window 0,
 * Frames span).  mem_k/mem_v int8 [layers][frames][heads*head_dim],
 * mem_ks/mem_vs fp32 [layers][frames][heads]. */
int ndo_decoder_row_cross(const ndo_decoder *m, int token, int pos, int capacity, int8_t *kv_k, int8_t *kv_v,
                          float *kv_ks, float *kv_vs, const float *rope_cos, const float *rope_sin, int frames,
                          const int8_t *mem_k, const int8_t *mem_v, const float *mem_ks, const float *mem_vs,
                          float *logits);

/* Cross memory of one layer (BuildCrossMemory + per-(frame, head) quantize,
 * src/Needle/Whistle.cs:886-914,789-790, with int8 projections): every
 * frame row of `memory` fp32 [frames][dim] is quantized (QuantizeInt8), put
 * through W_ckv[layer] (I8G32 [2*dim][dim]) and each head's 64 K and 64 V
 * values are quantized per (frame, head) into k/v [frames][heads*head_dim]
 * with scales ks/vs [frames][heads]. */
int ndo_cross_memory(const ndo_decoder *m, int layer, const float *memory, int frames, int8_t *k, int8_t *v, float *ks,
                     float *vs);

/* ---- the AVX2 CPU baseline (avx2_decoder.c) ---- */
typedef struct ndb_model ndb_model;
ndb_model *ndb_model_create(const ndo_decoder *m);
void ndb_model_destroy(ndb_model *b);
/* rows decode tokens[r] at pos[r] of their own caches (kv_k[r] etc.);
 * logits [rows][vocab]; equal to ndo_decoder_row per row, bit for bit. */
int ndb_decode_step(const ndb_model *b, int rows, const int32_t *tokens, const int32_t *pos, int capacity,
                    int8_t *const *kv_k, int8_t *const *kv_v, float *const *kv_ks, float *const *kv_vs,
                    const float *rope_cos, const float *rope_sin, float *logits, int threads);
/* the int8 linear alone: ndo_matmul_i8g32's y, bit for bit */
void ndb_matmul_i8g32(const int8_t *w, const uint16_t *sw, int n, int k, const int8_t *q, const float *sa, int m,
                      float *y, int ldy, int threads);
void *ndb_linear_create(const int8_t *w, const uint16_t *sw, int n, int k);
void ndb_linear_run(const void *linear, const int8_t *q, const float *sa, int m, float *y, int ldy, int threads);
void ndb_linear_destroy(void *linear);

#ifdef __cplusplus
}
#endif
#endif
