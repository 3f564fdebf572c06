/*
 * avx2_decoder.c - the CPU baseline: the synthetic decoder's batched decode
 * step written with the reference's AVX2 kernels' algorithms, on all host
 * cores (OpenMP).
 *
 * TEST AND BENCHMARK INFRASTRUCTURE ONLY: bench.py times it as the reference
 * arm and cpu_baseline ("AVX2 restatement"), tests/ check it against the
 * scalar oracle.  The shipped CUDA library never links it.
 *
 * What each part follows (paths relative to the needle-cs source tree):
 *  * the int8 linear: Gemv.Block (src/Needle/Gemv.cs:277-316) - a block of
 *    weight rows, per 32-column group the int32 dot of int8 pairs by
 *    maddubs/madd (the sign trick makes one operand unsigned, as the
 *    reference's codebook bytes are), one float fused multiply-add by the
 *    group scale per group; weight rows split across threads in contiguous
 *    ranges like MatMulBatch.RunShard (src/Needle/Quant.cs:717-723).  The 8
 *    lanes of a group's dot are reduced before the fold, and the fold runs
 *    one weight row per lane in ascending group order, so y equals the
 *    scalar oracle's (the reference folds lane-wise and sums lanes last,
 *    which rounds differently; its own tiers agree only to a tolerance);
 *  * attention: Attention.GroupAvx2 (src/Needle/Blocks.cs:178-541) per
 *    (row, head): int32 dots, s = (dot * ks) * (qs / sqrt(d)), Ops.Exp on
 *    8-position vectors, four partial sums by position modulo 4, 1 / total,
 *    acc = fma(e * vs, v, acc) on 8-dim vectors, out = acc * inverse;
 *  * SwiGLU: the vector Silu / Glu with Ops.Sigmoid (src/Needle/Ops.cs:
 *    36-40,90-105);
 *  * RMSNorm, the quantizer, RoPE and the KV write: the scalar oracle's
 *    routines (cheap beside the linears and attention).
 * Every float operation is the one the scalar oracle takes for the same
 * value, so the step's logits equal ndo_decoder_row's bit for bit.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include "needle_oracle.h"

/* ------------------------------------------------------------------------ */
/* model: the decoder's tensors plus the forms the AVX2 kernels read         */
/* ------------------------------------------------------------------------ */

/* One I8G32 weight matrix: |w| as unsigned bytes beside w (for the sign
 * trick) and the fp16 group scales as floats, transposed to [row block of
 * 8][group][8 rows] so one group's 8 scales are one vector. */
typedef struct {
    int n, k;
    const int8_t *w;
    uint8_t *abs_w;
    float *scales;
} ndb_linear;

struct ndb_model {
    const ndo_decoder *m;
    ndb_linear *qkv, *o, *gu, *down, head;
};

static int linear_init(ndb_linear *L, const int8_t *w, const uint16_t *sw, int n, int k) {
    L->n = n;
    L->k = k;
    L->w = w;
    const int groups = k / 32, blocks = (n + 7) / 8;
    L->abs_w = (uint8_t *)aligned_alloc(64, ((size_t)n * k + 63) / 64 * 64);
    L->scales = (float *)aligned_alloc(64, ((size_t)blocks * groups * 8 * sizeof(float) + 63) / 64 * 64);
    if (!L->abs_w || !L->scales) return -1;
    for (size_t i = 0; i < (size_t)n * k; i++) L->abs_w[i] = (uint8_t)(w[i] < 0 ? -w[i] : w[i]);
    for (int b = 0; b < blocks; b++)
        for (int g = 0; g < groups; g++)
            for (int r = 0; r < 8; r++) {
                const int row = b * 8 + r;
                L->scales[((size_t)b * groups + g) * 8 + r] =
                    row < n ? ndo_half_to_single(sw[(size_t)row * groups + g]) : 0.0f;
            }
    return 0;
}

static void linear_free(ndb_linear *L) {
    free(L->abs_w);
    free(L->scales);
}

ndb_model *ndb_model_create(const ndo_decoder *m) {
    ndb_model *b = (ndb_model *)calloc(1, sizeof(ndb_model));
    if (!b) return NULL;
    b->m = m;
    const int L = m->layers, d = m->dim, F = m->ffn;
    b->qkv = (ndb_linear *)calloc(L, sizeof(ndb_linear));
    b->o = (ndb_linear *)calloc(L, sizeof(ndb_linear));
    b->gu = (ndb_linear *)calloc(L, sizeof(ndb_linear));
    b->down = (ndb_linear *)calloc(L, sizeof(ndb_linear));
    int bad = !b->qkv || !b->o || !b->gu || !b->down;
    for (int l = 0; l < L && !bad; l++) {
        bad |= linear_init(&b->qkv[l], m->w_qkv[l], m->s_qkv[l], 3 * d, d);
        bad |= linear_init(&b->o[l], m->w_o[l], m->s_o[l], d, d);
        bad |= linear_init(&b->gu[l], m->w_gu[l], m->s_gu[l], 2 * F, d);
        bad |= linear_init(&b->down[l], m->w_d[l], m->s_d[l], d, F);
    }
    if (!bad) bad |= linear_init(&b->head, m->w_head, m->s_head, m->vocab, d);
    if (bad) {
        ndb_model_destroy(b);
        return NULL;
    }
    return b;
}

void ndb_model_destroy(ndb_model *b) {
    if (!b) return;
    for (int l = 0; l < b->m->layers; l++) {
        if (b->qkv) linear_free(&b->qkv[l]);
        if (b->o) linear_free(&b->o[l]);
        if (b->gu) linear_free(&b->gu[l]);
        if (b->down) linear_free(&b->down[l]);
    }
    linear_free(&b->head);
    free(b->qkv);
    free(b->o);
    free(b->gu);
    free(b->down);
    free(b);
}

/* ------------------------------------------------------------------------ */
/* the int8 linear                                                           */
/* ------------------------------------------------------------------------ */

/* Eight vectors of 8 int32 -> one vector whose lane r is the sum of vector r
 * (exact integer additions, so their order does not matter). */
static inline __m256i reduce8(const __m256i *v) {
    const __m256i a = _mm256_hadd_epi32(v[0], v[1]), b = _mm256_hadd_epi32(v[2], v[3]);
    const __m256i c = _mm256_hadd_epi32(v[4], v[5]), d = _mm256_hadd_epi32(v[6], v[7]);
    const __m256i ab = _mm256_hadd_epi32(a, b), cd = _mm256_hadd_epi32(c, d);
    return _mm256_add_epi32(_mm256_permute2x128_si256(ab, cd, 0x20), _mm256_permute2x128_si256(ab, cd, 0x31));
}

/* The int32 dot of 32 int8 pairs as 8 lanes: maddubs(|w|, sign(x, w)) then
 * madd with ones.  |w| <= 127 and |x| <= 127, so the 16-bit pair sums do not
 * saturate. */
static inline __m256i dot32(const uint8_t *abs_w, const int8_t *w, __m256i x, __m256i ones) {
    const __m256i aw = _mm256_loadu_si256((const __m256i *)abs_w);
    const __m256i sx = _mm256_sign_epi8(x, _mm256_loadu_si256((const __m256i *)w));
    return _mm256_madd_epi16(_mm256_maddubs_epi16(aw, sx), ones);
}

/* y[t][n] = (sum over groups g, ascending, of half(sw[n][g]) * D[t][n][g]
 * as fused multiply-adds) * sa[t], for rows [0, n) (the scalar oracle's
 * ndo_matmul_i8g32 bit for bit); residual: y = residual + that (residual may
 * alias y).  q rows hold values in [-127, 127] (the quantizer's range). */
static void linear_run(const ndb_linear *L, const int8_t *q, const float *sa, int m, float *y, int ldy,
                       const float *residual, int threads) {
    const int n = L->n, k = L->k, groups = k / 32, blocks = (n + 7) / 8;
    const __m256i ones = _mm256_set1_epi16(1);
#pragma omp parallel for schedule(static) num_threads(threads)
    for (int b = 0; b < blocks; b++) {
        const int rows = n - b * 8 < 8 ? n - b * 8 : 8;
        for (int t = 0; t < m; t++) {
            const int8_t *x = q + (size_t)t * k;
            __m256 acc = _mm256_setzero_ps();
            for (int g = 0; g < groups; g++) {
                const __m256i xv = _mm256_loadu_si256((const __m256i *)(x + g * 32));
                __m256i part[8];
                for (int r = 0; r < 8; r++) {
                    const size_t off = (size_t)(b * 8 + (r < rows ? r : 0)) * k + g * 32;
                    part[r] = dot32(L->abs_w + off, L->w + off, xv, ones);
                }
                const __m256 dots = _mm256_cvtepi32_ps(reduce8(part));
                acc = _mm256_fmadd_ps(_mm256_load_ps(L->scales + ((size_t)b * groups + g) * 8), dots, acc);
            }
            float out[8];
            _mm256_storeu_ps(out, _mm256_mul_ps(acc, _mm256_set1_ps(sa[t])));
            float *yt = y + (size_t)t * ldy + b * 8;
            const float *rt = residual ? residual + (size_t)t * ldy + b * 8 : NULL;
            for (int r = 0; r < rows; r++) yt[r] = rt ? rt[r] + out[r] : out[r];
        }
    }
}

/* The int8 linear alone (for the tests and the cfg1 baseline): the same
 * arguments as ndo_matmul_i8g32 without the accumulator dump. */
void ndb_matmul_i8g32(const int8_t *w, const uint16_t *sw, int n, int k, const int8_t *q, const float *sa, int m,
                      float *y, int ldy, int threads) {
    ndb_linear L;
    if (linear_init(&L, w, sw, n, k) != 0) return;
    linear_run(&L, q, sa, m, y, ldy, NULL, threads);
    linear_free(&L);
}

/* A prepared linear for repeated timing (the cfg1 baseline). */
void *ndb_linear_create(const int8_t *w, const uint16_t *sw, int n, int k) {
    ndb_linear *L = (ndb_linear *)calloc(1, sizeof(ndb_linear));
    if (!L || linear_init(L, w, sw, n, k) != 0) {
        if (L) linear_free(L);
        free(L);
        return NULL;
    }
    return L;
}
void ndb_linear_run(const void *L, const int8_t *q, const float *sa, int m, float *y, int ldy, int threads) {
    linear_run((const ndb_linear *)L, q, sa, m, y, ldy, NULL, threads);
}
void ndb_linear_destroy(void *L) {
    if (!L) return;
    linear_free((ndb_linear *)L);
    free(L);
}

/* ------------------------------------------------------------------------ */
/* Ops.Exp on 8 lanes (src/Needle/Ops.cs:16-31)                              */
/* ------------------------------------------------------------------------ */

static inline __m256 exp8(__m256 x) {
    x = _mm256_min_ps(_mm256_max_ps(x, _mm256_set1_ps(-87.3f)), _mm256_set1_ps(88.7f));
    const __m256 n = _mm256_round_ps(_mm256_mul_ps(x, _mm256_set1_ps(1.44269504f)),
                                     _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m256 r = _mm256_fnmadd_ps(n, _mm256_set1_ps(0.693359375f), x);
    r = _mm256_fnmadd_ps(n, _mm256_set1_ps(-2.12194440e-4f), r);
    __m256 p = _mm256_set1_ps(1.9875691500e-4f);
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.3981999507e-3f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(8.3334519073e-3f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(4.1665795894e-2f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(1.6666665459e-1f));
    p = _mm256_fmadd_ps(p, r, _mm256_set1_ps(5.0000001201e-1f));
    const __m256 y = _mm256_fmadd_ps(p, _mm256_mul_ps(r, r), _mm256_add_ps(r, _mm256_set1_ps(1.0f)));
    const __m256i bits = _mm256_slli_epi32(_mm256_add_epi32(_mm256_cvtps_epi32(n), _mm256_set1_epi32(127)), 23);
    return _mm256_mul_ps(y, _mm256_castsi256_ps(bits));
}

/* ------------------------------------------------------------------------ */
/* attention, one (row, head) of an unsplit tile (GroupAvx2)                  */
/* ------------------------------------------------------------------------ */

/* keys/values: the head's first position, strides in bytes per position;
 * scales: the head's first scale, stride per position.  scores: >= count + 8
 * floats of scratch. */
static void attention_head(const int8_t *query, float query_scale, const int8_t *keys, const float *key_scales,
                           const int8_t *values, const float *value_scales, int kv_stride, int scale_stride, int count,
                           float inv_sqrt_dim, float *scores, float *output) {
    const float scale = query_scale * inv_sqrt_dim;
    const __m256i ones = _mm256_set1_epi16(1);
    const __m256i q0 = _mm256_loadu_si256((const __m256i *)query);
    const __m256i q1 = _mm256_loadu_si256((const __m256i *)(query + 32));
    const __m256i aq0 = _mm256_abs_epi8(q0), aq1 = _mm256_abs_epi8(q1);
    __m256 peak8 = _mm256_set1_ps(-INFINITY);
    const __m256 vscale = _mm256_set1_ps(scale);
    for (int s0 = 0; s0 < count; s0 += 8) {
        __m256i part[8];
        for (int i = 0; i < 8; i++) {
            const int s = s0 + i < count ? s0 + i : count - 1;
            const int8_t *k = keys + (size_t)s * kv_stride;
            const __m256i k0 = _mm256_sign_epi8(_mm256_loadu_si256((const __m256i *)k), q0);
            const __m256i k1 = _mm256_sign_epi8(_mm256_loadu_si256((const __m256i *)(k + 32)), q1);
            part[i] = _mm256_add_epi32(_mm256_madd_epi16(_mm256_maddubs_epi16(aq0, k0), ones),
                                       _mm256_madd_epi16(_mm256_maddubs_epi16(aq1, k1), ones));
        }
        float ks[8];
        for (int i = 0; i < 8; i++)
            ks[i] = key_scales[(size_t)(s0 + i < count ? s0 + i : count - 1) * scale_stride];
        const __m256 sc = _mm256_mul_ps(_mm256_mul_ps(_mm256_cvtepi32_ps(reduce8(part)), _mm256_loadu_ps(ks)), vscale);
        _mm256_storeu_ps(scores + s0, sc);
        const int valid = count - s0 < 8 ? count - s0 : 8;
        const __m256 keep = _mm256_castsi256_ps(_mm256_cmpgt_epi32(_mm256_set1_epi32(valid),
                                                                    _mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7)));
        peak8 = _mm256_max_ps(peak8, _mm256_blendv_ps(_mm256_set1_ps(-INFINITY), sc, keep));
    }
    float pk[8];
    _mm256_storeu_ps(pk, peak8);
    float peak = pk[0];
    for (int i = 1; i < 8; i++) peak = pk[i] > peak ? pk[i] : peak;
    /* e = Ops.Exp(s - peak); four partial sums by position modulo 4 */
    const __m256 vpeak = _mm256_set1_ps(peak);
    for (int s0 = 0; s0 < count; s0 += 8)
        _mm256_storeu_ps(scores + s0, exp8(_mm256_sub_ps(_mm256_loadu_ps(scores + s0), vpeak)));
    __m128 sum4 = _mm_setzero_ps();
    int s = 0;
    for (; s + 4 <= count; s += 4) sum4 = _mm_add_ps(sum4, _mm_loadu_ps(scores + s));
    float sums[4];
    _mm_storeu_ps(sums, sum4);
    for (; s < count; s++) sums[0] += scores[s];
    const float inverse = 1.0f / ((sums[0] + sums[1]) + (sums[2] + sums[3]));
    /* w = e * vs; acc = fma(w, v, acc) in position order over 64 dims */
    __m256 acc[8];
    for (int j = 0; j < 8; j++) acc[j] = _mm256_setzero_ps();
    for (s = 0; s < count; s++) {
        const __m256 w = _mm256_set1_ps(scores[s] * value_scales[(size_t)s * scale_stride]);
        const int8_t *v = values + (size_t)s * kv_stride;
        for (int j = 0; j < 8; j++) {
            const __m256 vf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(v + 8 * j))));
            acc[j] = _mm256_fmadd_ps(w, vf, acc[j]);
        }
    }
    const __m256 vinv = _mm256_set1_ps(inverse);
    for (int j = 0; j < 8; j++) _mm256_storeu_ps(output + 8 * j, _mm256_mul_ps(acc[j], vinv));
}

/* ------------------------------------------------------------------------ */
/* one batched decode step                                                   */
/* ------------------------------------------------------------------------ */

/* SwiGLU on 8 lanes: (g * Ops.Sigmoid(g)) * u. */
static void swiglu(const float *gate, const float *up, int n, float *dst) {
    const __m256 one = _mm256_set1_ps(1.0f), zero = _mm256_setzero_ps();
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        const __m256 g = _mm256_loadu_ps(gate + i);
        const __m256 sig = _mm256_div_ps(one, _mm256_add_ps(one, exp8(_mm256_sub_ps(zero, g))));
        _mm256_storeu_ps(dst + i, _mm256_mul_ps(_mm256_mul_ps(g, sig), _mm256_loadu_ps(up + i)));
    }
    for (; i < n; i++) {
        float one_lane[8] = {gate[i]}, out[8];
        const __m256 g = _mm256_loadu_ps(one_lane);
        const __m256 sig = _mm256_div_ps(one, _mm256_add_ps(one, exp8(_mm256_sub_ps(zero, g))));
        _mm256_storeu_ps(out, sig);
        dst[i] = (gate[i] * out[0]) * up[i];
    }
}

/* Rows r of the batch decode token tokens[r] at position pos[r] of their own
 * caches (kv_k[r] etc., the oracle's [layers][capacity][width] layout), as
 * ForwardBatch does (src/Needle/Engine.cs:2303-2404): layer by layer for the
 * whole batch, each linear over all rows at once.  logits [rows][vocab].
 * Returns 0, or -1 if scratch allocation failed. */
int ndb_decode_step(const ndb_model *b, int rows, const int32_t *tokens, const int32_t *pos, int capacity,
                    int8_t *const *kv_k, int8_t *const *kv_v, float *const *kv_ks, float *const *kv_vs,
                    const float *rope_cos, const float *rope_sin, float *logits, int threads) {
    const ndo_decoder *m = b->m;
    const int d = m->dim, H = m->heads, hd = m->head_dim, F = m->ffn, width = H * hd, half = hd / 2;
    const float inv_sqrt = 1.0f / sqrtf((float)hd);
    const size_t R = (size_t)rows;
    float *x = (float *)malloc(R * d * sizeof(float)), *h = (float *)malloc(R * (2 * F) * sizeof(float));
    float *qkv = (float *)malloc(R * 3 * d * sizeof(float)), *o = (float *)malloc(R * d * sizeof(float));
    float *act = (float *)malloc(R * F * sizeof(float)), *sa = (float *)malloc(R * sizeof(float));
    float *qs = (float *)malloc(R * H * sizeof(float));
    int8_t *qa = (int8_t *)malloc(R * (F > d ? F : d)), *qq = (int8_t *)malloc(R * width + 64);
    float *scratch = (float *)malloc((size_t)threads * (capacity + 16) * sizeof(float));
    int rc = 0;
    if (!x || !h || !qkv || !o || !act || !sa || !qs || !qa || !qq || !scratch) {
        rc = -1;
        goto done;
    }
#pragma omp parallel for num_threads(threads)
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < d; i++) x[(size_t)r * d + i] = ndo_half_to_single(m->embedding[(size_t)tokens[r] * d + i]);
    for (int l = 0; l < m->layers; l++) {
#pragma omp parallel for num_threads(threads)
        for (int r = 0; r < rows; r++) {
            ndo_rms_norm(x + (size_t)r * d, m->attn_norm[l], d, h + (size_t)r * d);
            sa[r] = ndo_quantize_int8(h + (size_t)r * d, d, qa + (size_t)r * d);
        }
        linear_run(&b->qkv[l], qa, sa, rows, qkv, 3 * d, NULL, threads);
#pragma omp parallel for num_threads(threads)
        for (int r = 0; r < rows; r++) {
            float *q = qkv + (size_t)r * 3 * d, *k = q + d, *v = k + d;
            const int p = pos[r];
            ndo_rope(q, H, hd, rope_cos + (size_t)p * half, rope_sin + (size_t)p * half);
            ndo_rope(k, H, hd, rope_cos + (size_t)p * half, rope_sin + (size_t)p * half);
            int8_t *lk = kv_k[r] + (size_t)l * capacity * width, *lv = kv_v[r] + (size_t)l * capacity * width;
            float *lks = kv_ks[r] + (size_t)l * capacity * H, *lvs = kv_vs[r] + (size_t)l * capacity * H;
            for (int hh = 0; hh < H; hh++) {
                qs[(size_t)r * H + hh] = ndo_quantize_int8(q + hh * hd, hd, qq + (size_t)r * width + hh * hd);
                lks[(size_t)p * H + hh] = ndo_quantize_int8(k + hh * hd, hd, lk + (size_t)p * width + hh * hd);
                lvs[(size_t)p * H + hh] = ndo_quantize_int8(v + hh * hd, hd, lv + (size_t)p * width + hh * hd);
            }
        }
        /* Denormal operands are flushed to zero in this region (MXCSR FTZ and
         * DAZ, restored afterwards): on this data e * vs of positions far
         * below the peak is a denormal, and an x86 fma with a denormal operand
         * takes a microcode assist (the step ran about four times slower with
         * IEEE denormals).  The reference runs with IEEE denormals, so this
         * makes the baseline faster than the reference's code, not slower;
         * such a product is far below half an ulp of the accumulator, which
         * also holds the peak position's term, so the outputs do not change. */
#pragma omp parallel num_threads(threads)
        {
            const unsigned csr = _mm_getcsr();
            _mm_setcsr(csr | 0x8040u);
#pragma omp for schedule(dynamic, 1)
            for (int rh = 0; rh < rows * H; rh++) {
                const int r = rh / H, hh = rh % H;
                const int8_t *lk = kv_k[r] + (size_t)l * capacity * width + hh * hd;
                const int8_t *lv = kv_v[r] + (size_t)l * capacity * width + hh * hd;
                const float *lks = kv_ks[r] + (size_t)l * capacity * H + hh;
                const float *lvs = kv_vs[r] + (size_t)l * capacity * H + hh;
                attention_head(qq + (size_t)r * width + hh * hd, qs[rh], lk, lks, lv, lvs, width, H, pos[r] + 1,
                               inv_sqrt, scratch + (size_t)omp_get_thread_num() * (capacity + 16),
                               o + (size_t)r * d + hh * hd);
            }
            _mm_setcsr(csr);
        }
#pragma omp parallel for num_threads(threads)
        for (int r = 0; r < rows; r++) sa[r] = ndo_quantize_int8(o + (size_t)r * d, d, qa + (size_t)r * d);
        linear_run(&b->o[l], qa, sa, rows, x, d, x, threads);
#pragma omp parallel for num_threads(threads)
        for (int r = 0; r < rows; r++) {
            ndo_rms_norm(x + (size_t)r * d, m->ffn_norm[l], d, h + (size_t)r * d);
            sa[r] = ndo_quantize_int8(h + (size_t)r * d, d, qa + (size_t)r * d);
        }
        linear_run(&b->gu[l], qa, sa, rows, h, 2 * F, NULL, threads);
#pragma omp parallel for num_threads(threads)
        for (int r = 0; r < rows; r++) {
            const float *gu = h + (size_t)r * 2 * F;
            swiglu(gu, gu + F, F, act + (size_t)r * F);
            sa[r] = ndo_quantize_int8(act + (size_t)r * F, F, qa + (size_t)r * F);
        }
        linear_run(&b->down[l], qa, sa, rows, x, d, x, threads);
    }
#pragma omp parallel for num_threads(threads)
    for (int r = 0; r < rows; r++) {
        ndo_rms_norm(x + (size_t)r * d, m->final_norm, d, h + (size_t)r * d);
        sa[r] = ndo_quantize_int8(h + (size_t)r * d, d, qa + (size_t)r * d);
    }
    linear_run(&b->head, qa, sa, rows, logits, m->vocab, NULL, threads);
done:
    free(x);
    free(h);
    free(qkv);
    free(o);
    free(act);
    free(sa);
    free(qs);
    free(qa);
    free(qq);
    free(scratch);
    return rc;
}
