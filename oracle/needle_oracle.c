/*
 * needle_oracle.c - CPU restatement of the needle-cs batched decode path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA library, never
 * linked into it.  Each function cites the reference routine it restates
 * (paths relative to the needle-cs source tree).  Build with
 * -ffp-contract=off so that a*b+c stays two rounded operations, as in the
 * reference's scalar C#.
 */
#include "needle_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Test-input generators: tests/Needle.Tests/Conformance/Conformance.cs      */
/* ------------------------------------------------------------------------ */

/* XorShift64.Next (Conformance.cs:19-27); seed 0 is replaced by the golden
 * ratio constant (Conformance.cs:14-17) by the caller. */
uint64_t ndo_xorshift_next(uint64_t *state) {
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

/* XorShift64.NextInt (Conformance.cs:29-32). */
int ndo_xorshift_int(uint64_t *state, int lo, int hi) {
    return lo + (int)(ndo_xorshift_next(state) % (uint64_t)(hi - lo));
}

/* XorShift64.NextFloat (Conformance.cs:34-37): ulong->float, then float ops. */
float ndo_xorshift_float(uint64_t *state, float scale) {
    float u = (float)(ndo_xorshift_next(state) >> 11) * (1.0f / 9007199254740992.0f);
    return ((u - 0.5f) * 2.0f) * scale;
}

/* ConformanceInputs.FillUniform (Conformance.cs:42-48). */
void ndo_fill_uniform(float *x, int n, uint64_t *state, float scale) {
    for (int i = 0; i < n; i++) x[i] = ndo_xorshift_float(state, scale);
}

/* ConformanceInputs.FillEdges (Conformance.cs:50-68): zeros every 7th,
 * +-1e-38 denormals every 11th from 3, +-0.5*scale ties every 13th from 5. */
void ndo_fill_edges(float *x, int n, uint64_t *state, float scale) {
    for (int i = 0; i < n; i++) x[i] = ndo_xorshift_float(state, scale);
    for (int i = 0; i < n; i += 7) x[i] = 0.0f;
    for (int i = 3; i < n; i += 11) x[i] = 1e-38f * (i % 2 == 0 ? 1.0f : -1.0f);
    for (int i = 5; i < n; i += 13) x[i] = (i % 26 < 13 ? 0.5f : -0.5f) * scale;
}

/* ConformanceInputs.FillSByte (Conformance.cs:70-88). */
void ndo_fill_sbyte(int8_t *x, int n, uint64_t *state, int extremes) {
    for (int i = 0; i < n; i++) x[i] = (int8_t)ndo_xorshift_int(state, -128, 128);
    if (extremes && n > 0) {
        x[0] = -128;
        if (n > 1) x[1] = 127;
        for (int i = 2; i < n; i += 5) x[i] = (i % 2 == 0) ? (int8_t)-128 : (int8_t)127;
    }
}

/* ConformanceInputs.FillBytes (Conformance.cs:90-101). */
void ndo_fill_bytes(uint8_t *x, int n, uint64_t *state, int extremes) {
    for (int i = 0; i < n; i++) x[i] = (uint8_t)ndo_xorshift_int(state, 0, 256);
    if (extremes && n >= 2) {
        x[0] = 0x00;
        x[1] = 0xFF;
    }
}

/* ConformanceInputs.HalfBits (Conformance.cs:103-118): saturating, flush
 * below 2^-15, round-half-up on the dropped 13 bits. */
uint16_t ndo_half_bits(float value) {
    uint32_t bits;
    memcpy(&bits, &value, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    uint32_t magnitude = bits & 0x7FFFFFFFu;
    if (magnitude >= 0x47800000u) return (uint16_t)(sign | 0x7BFFu);
    if (magnitude <= 0x38000000u) return (uint16_t)sign;
    uint32_t rounded = (magnitude >> 13) + ((magnitude >> 12) & 1u);
    return (uint16_t)(sign | (rounded - 0x1C000u));
}

/* ------------------------------------------------------------------------ */
/* The benchmark configs' synthetic inputs                                   */
/* ------------------------------------------------------------------------ */
/* A counter-based generator: value i of stream `stream` under `seed` is a
 * function of (seed, stream, i) alone.  splitmix64 mixing (Steele, Lea and
 * Flood, 2014); normal = Irwin-Hall(12) - 6 from twelve 16-bit uniforms,
 * scaled to unit variance, in exact integer arithmetic; uniform = the top 24
 * bits of one hash, lo + (hi - lo) * u in float; int8 = hash mod 255 - 127.
 * The CUDA library generates the engine's weights and prefix caches with the
 * same definition; these host copies let the CPU baselines and tests build
 * them without it. */
static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static uint64_t synth_key(uint64_t seed, uint64_t stream) { return splitmix64(seed ^ (stream * 0x9E3779B97F4A7C15ull)); }
static uint64_t synth_hash(uint64_t key, uint64_t i) { return splitmix64(key + i * 0xD1B54A32D192ED03ull); }
static int sum16x4(uint64_t h) {
    return (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48);
}

void ndo_synth_normal(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float scale, float *out) {
    const uint64_t key = synth_key(seed, stream);
    for (size_t n = 0; n < count; n++) {
        const uint64_t i = first + n;
        const int s = sum16x4(synth_hash(key, 3 * i)) + sum16x4(synth_hash(key, 3 * i + 1)) +
                      sum16x4(synth_hash(key, 3 * i + 2));
        out[n] = ((float)(2 * s - 786420) * (1.0f / 131072.0f)) * scale;
    }
}

void ndo_synth_uniform(uint64_t seed, uint64_t stream, uint64_t first, size_t count, float lo, float hi, float *out) {
    const uint64_t key = synth_key(seed, stream);
    for (size_t n = 0; n < count; n++) {
        const float u = (float)(synth_hash(key, first + n) >> 40) * (1.0f / 16777216.0f);
        const float span = hi - lo;
        const float t = span * u;
        out[n] = lo + t;
    }
}

void ndo_synth_int8(uint64_t seed, uint64_t stream, uint64_t first, size_t count, int8_t *out) {
    const uint64_t key = synth_key(seed, stream);
    for (size_t n = 0; n < count; n++) out[n] = (int8_t)((int)(synth_hash(key, first + n) % 255u) - 127);
}

/* ------------------------------------------------------------------------ */
/* Row primitives: src/Needle/Scalar.cs                                      */
/* ------------------------------------------------------------------------ */

static const float kRoundBias = 12582912.0f;           /* Scalar.cs:51 */
static const float kHadamardScale = 0.08838834764831845f; /* Scalar.cs:49 */

/* Scalar.RoundEven (Scalar.cs:52-53): the 1.5*2^23 trick. */
static float round_even(float x) {
    volatile float t = x + kRoundBias; /* volatile keeps the two roundings */
    return t - kRoundBias;
}

/* MathF.Exp (.NET calls the C runtime's expf): exp of a float rounded to
 * nearest float, computed in double precision from the mathematics with
 * IEEE operations only.  Cody and Waite's argument reduction x = k*ln2 + r,
 * k = rint(x/ln2), with ln2 split into a high part whose products with k are
 * exact and a low part (the split published with fdlibm); exp(r) by its
 * Taylor series to degree 13 in Estrin's form with fused multiply-adds; scaled
 * by 2^k (exact) and rounded once to float.  The relative error before that
 * rounding is below 1e-15: the correctly rounded float unless exp(x) lies
 * within about 1e-15 of a rounding midpoint, where a C runtime's expf may
 * differ as well (the reference pins its own exp only to a tolerance,
 * tests/Needle.Tests/KernelTests.cs:35-46).  The CUDA kernels evaluate the
 * same steps, so softmax weights and SiLU gates compare bit for bit. */
static float exp_rn(float x) {
    if (x != x) return x;
    if (x > 89.0f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const double xd = (double)x;
    const double k = rint(xd * 1.4426950408889634);
    const double r = (xd - k * 6.93147180369123816490e-01) - k * 1.90821492927058770002e-10;
    /* the degree-13 Taylor polynomial by Estrin's scheme (pairs, then r^2, r^4,
     * r^8 levels): four dependent fused steps instead of thirteen */
    const double r2 = r * r, r4 = r2 * r2, r8 = r4 * r4;
    const double q0 = fma(1.0, r, 1.0);                                            /* 1 + r */
    const double q1 = fma(1.6666666666666666667e-01, r, 0.5);                      /* 1/2! + r/3! */
    const double q2 = fma(8.3333333333333333333e-03, r, 4.1666666666666666667e-02); /* 1/4!, 1/5! */
    const double q3 = fma(1.9841269841269841270e-04, r, 1.3888888888888888889e-03); /* 1/6!, 1/7! */
    const double q4 = fma(2.7557319223985890653e-06, r, 2.4801587301587301587e-05); /* 1/8!, 1/9! */
    const double q5 = fma(2.5052108385441718775e-08, r, 2.7557319223985890653e-07); /* 1/10!, 1/11! */
    const double q6 = fma(1.6059043836821614599e-10, r, 2.0876756987868098979e-09); /* 1/12!, 1/13! */
    const double s0 = fma(q1, r2, q0), s1 = fma(q3, r2, q2), s2 = fma(q5, r2, q4);
    const double t0 = fma(s1, r4, s0), t1 = fma(q6, r4, s2);
    const double p = fma(t1, r8, t0);
    return (float)scalbn(p, (int)k);
}

/* exp_rn over an array (the oracle's exponential, for the tests). */
void ndo_exp_rn(const float *x, int n, float *y) {
    for (int i = 0; i < n; i++) y[i] = exp_rn(x[i]);
}

/* Ops.Exp (src/Needle/Ops.cs:16-31), the reference's SIMD exponential, which
 * its AVX2 attention softmax (Blocks.cs:362-404) and vector sigmoid
 * (Ops.cs:36-40) use, restated for one lane: clamp to [-87.3, 88.7] (a NaN
 * becomes -87.3, as maxps returns its second operand), n = nearest integer of
 * x * log2(e), r = x - n*ln2 in two fused steps, a degree-5 polynomial by
 * fused multiply-adds, y = p*r^2 + (r + 1), times 2^n built in the exponent
 * bits.  Every step is one IEEE operation, so the CUDA kernels, which take the
 * same steps, return the same bits.  It agrees with expf to within about
 * 2e-6 relative (tests/Needle.Tests/KernelTests.cs:35-43). */
static float ops_exp(float x) {
    x = fminf(fmaxf(x, -87.3f), 88.7f);
    const float n = rintf(x * 1.44269504f);
    float r = fmaf(-n, 0.693359375f, x);
    r = fmaf(-n, -2.12194440e-4f, r);
    float p = 1.9875691500e-4f;
    p = fmaf(p, r, 1.3981999507e-3f);
    p = fmaf(p, r, 8.3334519073e-3f);
    p = fmaf(p, r, 4.1665795894e-2f);
    p = fmaf(p, r, 1.6666665459e-1f);
    p = fmaf(p, r, 5.0000001201e-1f);
    const float y = fmaf(p, r * r, r + 1.0f);
    const uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
    float scale;
    memcpy(&scale, &bits, sizeof scale);
    return y * scale;
}

/* Ops.Exp over an array (for the tests). */
void ndo_exp_simd(const float *x, int n, float *y) {
    for (int i = 0; i < n; i++) y[i] = ops_exp(x[i]);
}

/* Ops.Sigmoid (src/Needle/Ops.cs:36-40): 1 / (1 + Exp(0 - x)). */
static float ops_sigmoid(float x) { return 1.0f / (1.0f + ops_exp(0.0f - x)); }

static float maxf_cs(float a, float b) { return a > b ? a : (b > a ? b : (a == a ? a : b)); }

/* Scalar.AbsMax (Scalar.cs:55-60). */
float ndo_abs_max(const float *x, int n) {
    float peak = 0.0f;
    for (int i = 0; i < n; i++) peak = maxf_cs(peak, fabsf(x[i]));
    return peak;
}

static float clamp_q(float v) { return fminf(fmaxf(v, -128.0f), 127.0f); }

/* Scalar.QuantizeInt8 (Scalar.cs:67-74). */
float ndo_quantize_int8(const float *x, int n, int8_t *dst) {
    float peak = ndo_abs_max(x, n);
    float scale = peak > 0.0f ? peak / 127.0f : 1.0f;
    float inverse = 1.0f / scale;
    for (int i = 0; i < n; i++) dst[i] = (int8_t)clamp_q(round_even(x[i] * inverse));
    return scale;
}

/* Per-row QuantizeInt8 over a [rows][cols] matrix (the activation quantizer
 * applied to every linear input row, src/Needle/Quant.cs:103-132). */
void ndo_quantize_rows(const float *x, int rows, int cols, int8_t *q, float *scales) {
    for (int r = 0; r < rows; r++) scales[r] = ndo_quantize_int8(x + (size_t)r * cols, cols, q + (size_t)r * cols);
}

/* Quant.FakeA8 scalar path = AbsMax + Scalar.RoundTrip (Quant.cs:66-77,
 * Scalar.cs:62-65). */
float ndo_fake_a8(float *x, int n) {
    float peak = ndo_abs_max(x, n);
    float scale = peak > 0.0f ? peak / 127.0f : 1.0f;
    float inverse = 1.0f / scale;
    for (int i = 0; i < n; i++) x[i] = clamp_q(round_even(x[i] * inverse)) * scale;
    return scale;
}

/* Scalar.HalfToSingle (Scalar.cs:121-128): subnormals exact, no Inf/NaN
 * special case (0x7C00 decodes to 65536). */
float ndo_half_to_single(uint16_t half) {
    uint32_t magnitude = half & 0x7FFFu;
    if (magnitude == 0) return 0.0f;
    if (magnitude < 0x0400u)
        return (half & 0x8000u) ? -(float)magnitude * 5.9604645e-8f : (float)magnitude * 5.9604645e-8f;
    uint32_t bits = ((magnitude << 13) + 0x38000000u) | ((uint32_t)(half & 0x8000u) << 16);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Scalar.Hadamard (Scalar.cs:76-89): in-place FWHT over 128, then scale. */
void ndo_hadamard128(const float *src, float *p) {
    if (src != p)
        for (int i = 0; i < 128; i++) p[i] = src[i];
    for (int stride = 1; stride < 128; stride <<= 1)
        for (int block = 0; block < 128; block += stride * 2)
            for (int i = block; i < block + stride; i++) {
                float a = p[i], b = p[i + stride];
                p[i] = a + b;
                p[i + stride] = a - b;
            }
    for (int i = 0; i < 128; i++) p[i] *= kHadamardScale;
}

/* Scalar.Planes (Scalar.cs:91-111). */
void ndo_planes(const int8_t *quantized, int bits, int8_t *dst, int *sum) {
    int s = 0;
    if (bits == 2) {
        for (int j = 0; j < 32; j++)
            for (int p = 0; p < 4; p++) {
                int8_t q = quantized[4 * j + p];
                dst[p * 32 + j] = q;
                s += q;
            }
    } else {
        for (int half = 0; half < 2; half++)
            for (int j = 0; j < 32; j++)
                for (int p = 0; p < 2; p++) {
                    int8_t q = quantized[half * 64 + 2 * j + p];
                    dst[half * 64 + p * 32 + j] = q;
                    s += q;
                }
    }
    *sum = s;
}

/* Scalar.Sigmoid (Scalar.cs:194). */
float ndo_sigmoid(float x) { return 1.0f / (1.0f + exp_rn(-x)); }

/* Scalar.Softmax (Scalar.cs:220-231). */
void ndo_softmax(float *s, int n) {
    float peak = -INFINITY;
    for (int i = 0; i < n; i++) peak = maxf_cs(peak, s[i]);
    float total = 0.0f;
    for (int i = 0; i < n; i++) {
        s[i] = exp_rn(s[i] - peak);
        total += s[i];
    }
    for (int i = 0; i < n; i++) s[i] /= total;
}

/* Scalar.Rope (Scalar.cs:233-248): half-split rotation. */
void ndo_rope(float *x, int heads, int head_dim, const float *cos_t, const float *sin_t) {
    int half = head_dim / 2;
    for (int h = 0; h < heads; h++) {
        float *lo = x + h * head_dim, *hi = lo + half;
        for (int i = 0; i < half; i++) {
            float a = lo[i], b = hi[i];
            lo[i] = a * cos_t[i] - b * sin_t[i];
            hi[i] = b * cos_t[i] + a * sin_t[i];
        }
    }
}

/* EngineCore.RopeFrequencies + BuildRopeTables (src/Needle/Engine.cs:336-356). */
void ndo_rope_tables(float theta, int qk_dim, int positions, float *cos_t, float *sin_t) {
    int half = qk_dim / 2;
    float freq[512];
    for (int i = 0; i < half && i < 512; i++) freq[i] = 1.0f / powf(theta, 2.0f * (float)i / (float)qk_dim);
    for (int p = 0; p < positions; p++)
        for (int i = 0; i < half; i++) {
            float angle = (float)p * freq[i];
            cos_t[(size_t)p * half + i] = cosf(angle);
            sin_t[(size_t)p * half + i] = sinf(angle);
        }
}

/* Ops.InverseRms (src/Needle/Ops.cs:209) over Scalar.SumOfSquares
 * (Scalar.cs:206-211), epsilon 1e-6 (Ops.cs:12). */
float ndo_inverse_rms(const float *x, int n) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    return 1.0f / sqrtf(sum / (float)n + 1e-6f);
}

/* Synthetic RMSNorm: the scalar ZeroCenteredRms expression
 * (src/Needle/Ops.cs:233-255, (1+scale)*x*inv) with a plain weight w in
 * place of (1+scale): dst = (w*x)*inv. */
void ndo_rms_norm(const float *x, const float *weight, int n, float *dst) {
    float inv = ndo_inverse_rms(x, n);
    for (int i = 0; i < n; i++) dst[i] = (weight[i] * x[i]) * inv;
}

/* Ops.ZeroCenteredRms scalar branch (src/Needle/Ops.cs:243). */
void ndo_zero_centered_rms(const float *x, const float *scale, int n, float *dst) {
    float inv = ndo_inverse_rms(x, n);
    for (int i = 0; i < n; i++) dst[i] = ((1.0f + scale[i]) * x[i]) * inv;
}

/* SwiGLU from the reference's AVX2 Silu / Glu (src/Needle/Ops.cs:90-105,
 * 1013-1024: x * Sigmoid(x) on vectors): dst = (g * Ops.Sigmoid(g)) * u. */
void ndo_swiglu(const float *gate, const float *up, int n, float *dst) {
    for (int i = 0; i < n; i++) dst[i] = (gate[i] * ops_sigmoid(gate[i])) * up[i];
}

/* ------------------------------------------------------------------------ */
/* Needle-3 row ops: hyper-connections, conv taps, fake-A8 norms             */
/* ------------------------------------------------------------------------ */

/* Scalar.Mix4 (Scalar.cs:255-258): dst = w0*s0 + w1*s1 + w2*s2 + w3*s3. */
void ndo_mix4(const float *s, int dim, float w0, float w1, float w2, float w3, float *dst) {
    for (int c = 0; c < dim; c++) dst[c] = w0 * s[c] + w1 * s[dim + c] + w2 * s[2 * dim + c] + w3 * s[3 * dim + c];
}

/* Scalar.Combine4 (Scalar.cs:250-253): dst = post*y + mix. */
void ndo_combine4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *y, float post,
                  float *dst) {
    for (int c = 0; c < dim; c++)
        dst[c] = post * y[c] + w0 * s[c] + w1 * s[dim + c] + w2 * s[2 * dim + c] + w3 * s[3 * dim + c];
}

/* Scalar.CombineDiff4 (Scalar.cs:428-431): dst = post*(x - u) + mix. */
void ndo_combine_diff4(const float *s, int dim, float w0, float w1, float w2, float w3, const float *x,
                       const float *u, float post, float *dst) {
    for (int c = 0; c < dim; c++)
        dst[c] = post * (x[c] - u[c]) + w0 * s[c] + w1 * s[dim + c] + w2 * s[2 * dim + c] + w3 * s[3 * dim + c];
}

/* Ops.CombineDiff4x4 (Ops.cs:800-812): lane i of the next stream is
 * CombineDiff4 with weights mix[4i..4i+3] and gate post_gate[i]. */
void ndo_combine_diff4x4(const float *s, int dim, const float *mix, const float *x, const float *u,
                         const float *post_gate, float *dst) {
    for (int i = 0; i < 4; i++)
        ndo_combine_diff4(s, dim, mix[i * 4], mix[i * 4 + 1], mix[i * 4 + 2], mix[i * 4 + 3], x, u, post_gate[i],
                          dst + (size_t)i * dim);
}

/* Scalar.Taps3 (Scalar.cs:285-288): current[-2w .. w) holds three steps. */
void ndo_taps3(const float *taps, int width, const float *current, float *dst) {
    for (int c = 0; c < width; c++)
        dst[c] = taps[c] * current[c] + taps[width + c] * current[c - width] + taps[2 * width + c] * current[c - 2 * width];
}

/* Scalar.Sinkhorn4x4 (Scalar.cs:361-381): row-max exp, then 20 rounds of
 * row and column normalisation (a column of zeros is left alone). */
void ndo_sinkhorn4x4(const float *logits, float *result) {
    for (int r = 0; r < 4; r++) {
        float peak = maxf_cs(maxf_cs(logits[r * 4], logits[r * 4 + 1]), maxf_cs(logits[r * 4 + 2], logits[r * 4 + 3]));
        for (int c = 0; c < 4; c++) result[r * 4 + c] = exp_rn(logits[r * 4 + c] - peak);
    }
    for (int it = 0; it < 20; it++) {
        for (int r = 0; r < 4; r++) {
            float sum = result[r * 4] + result[r * 4 + 1] + result[r * 4 + 2] + result[r * 4 + 3];
            for (int c = 0; c < 4; c++) result[r * 4 + c] /= sum;
        }
        for (int c = 0; c < 4; c++) {
            float sum = result[c] + result[4 + c] + result[8 + c] + result[12 + c];
            if (sum > 0.0f)
                for (int r = 0; r < 4; r++) result[r * 4 + c] /= sum;
        }
    }
}

static float fake_round_trip(float *v, int n) {
    float peak = 0.0f;
    for (int i = 0; i < n; i++) peak = maxf_cs(peak, fabsf(v[i]));
    float scale = peak > 0.0f ? peak / 127.0f : 1.0f;
    float round = 1.0f / scale;
    for (int i = 0; i < n; i++) v[i] = clamp_q(round_even(v[i] * round)) * scale;
    return scale;
}

static float rms_inverse(const float *x, int n) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    return 1.0f / sqrtf(sum / (float)n + 1e-6f);
}

/* Scalar.RmsFakeA8 (Scalar.cs:381-395). */
void ndo_rms_fake_a8(const float *x, int n, float *dst) {
    float inverse = rms_inverse(x, n);
    for (int i = 0; i < n; i++) dst[i] = x[i] * inverse;
    fake_round_trip(dst, n);
}

/* Scalar.CenteredRmsFakeA8 (Scalar.cs:397-411). */
void ndo_centered_rms_fake_a8(const float *x, const float *scale, int n, float *dst) {
    float inverse = rms_inverse(x, n);
    for (int i = 0; i < n; i++) dst[i] = (1.0f + scale[i]) * x[i] * inverse;
    fake_round_trip(dst, n);
}

/* Scalar.GateFakeA8 (Scalar.cs:413-426): x *= sigmoid(gate), in place. */
void ndo_gate_fake_a8(float *x, const float *gate, int n) {
    for (int i = 0; i < n; i++) x[i] *= ndo_sigmoid(gate[i]);
    fake_round_trip(x, n);
}

/* Scalar.PostNormAdd (Scalar.cs:433-439). */
void ndo_post_norm_add(float *residual, const float *x, const float *scale, float gate, int n) {
    float inverse = rms_inverse(x, n);
    for (int i = 0; i < n; i++) residual[i] += gate * ((1.0f + scale[i]) * x[i] * inverse);
}

/* Scalar.Kron (Scalar.cs:441-460): result = left^T . z . right on a
 * (rows x cols) grid, active input rows and result rows given. */
static void kron(const float *z, int active_rows, const float *left, const float *right, int rows, int cols,
                 int result_rows, float *result) {
    float scratch[1024];
    for (int k = 0; k < result_rows; k++) {
        for (int c = 0; c < cols; c++) {
            float sum = 0.0f;
            for (int i = 0; i < active_rows; i++) sum += left[i * rows + k] * z[i * cols + c];
            scratch[c] = sum;
        }
        for (int c = 0; c < cols; c++) {
            float sum = 0.0f;
            for (int j = 0; j < cols; j++) sum += scratch[j] * right[j * cols + c];
            result[k * cols + c] = sum;
        }
    }
}

/* HadamardMlp.Apply, scalar path (src/Needle/Blocks.cs:1067-1093 with
 * Scalar.ConditionWeights / ScaleInput / PermuteModulateActivate /
 * PermuteScale / AccumulateOutput, Scalar.cs:323-358): the Kronecker-factored
 * MLP on one token's residual, in place.  w: d1, d2, b2, d3, d4, w1a, w1b,
 * w2a, w2b, w3a, w3b, cond_v, cond_u in MlpWeights order (Audio.cs:5-27). */
void ndo_hadamard_mlp(const float *const *w, const float *pre_norm, const int32_t *perm_a, const int32_t *perm_b,
                      int dim, int rows, int cols, float scale, float *residual) {
    const float *d1 = w[0], *d2 = w[1], *b2 = w[2], *d3 = w[3], *d4 = w[4], *w1a = w[5], *w1b = w[6], *w2a = w[7],
                *w2b = w[8], *w3a = w[9], *w3b = w[10], *cond_v = w[11], *cond_u = w[12];
    int width = rows * cols;
    int input_rows = (dim + cols - 1) / cols;
    int output_rows = rows < (input_rows + 3) / 4 * 4 ? rows : (input_rows + 3) / 4 * 4;
    float weights[8], normalized[8192], front[8192], back[8192];
    ndo_zero_centered_rms(residual, pre_norm, dim, normalized);
    for (int j = 0; j < 8; j++) {
        float sum = 0.0f;
        for (int i = 0; i < dim; i++) sum += normalized[i] * cond_v[i * 8 + j];
        weights[j] = sum;
    }
    ndo_softmax(weights, 8);
    for (int i = 0; i < dim; i++) front[i] = normalized[i] * d1[i];
    for (int i = dim; i < input_rows * cols; i++) front[i] = 0.0f;
    kron(front, input_rows, w1a, w1b, rows, cols, rows, back);
    for (int n = 0; n < width; n++) {
        float condition = 1.0f;
        for (int j = 0; j < 8; j++) condition += weights[j] * cond_u[j * width + n];
        float v = d2[n] * condition * back[perm_a[n]] + b2[n];
        front[n] = v * ndo_sigmoid(v);
    }
    kron(front, rows, w2a, w2b, rows, cols, rows, back);
    for (int n = 0; n < width; n++) front[n] = back[perm_b[n]] * d3[n];
    kron(front, rows, w3a, w3b, rows, cols, output_rows, back);
    for (int i = 0; i < dim; i++) residual[i] += scale * (back[i] * d4[i]);
}

/* ------------------------------------------------------------------------ */
/* Engram (Needle-3 n-gram memory)                                           */
/* ------------------------------------------------------------------------ */

/* EngineCore.EngramHashRowsBatch (src/Needle/Engine.cs:2652-2681): the table
 * row of every (token, table) from the token's n-gram; rows of consecutive
 * tokens of one slot form a run, earlier tokens come from the slot's last two
 * (slot_prev[slot][0..1]), -1 before the n-gram fits.  rows [count][tables]. */
void ndo_engram_hash(const int32_t *tokens, const int32_t *row_slots, int count, const int32_t *slot_length,
                     const int32_t *slot_prev, const int32_t *orders, int order_count, int heads, int engram_slots,
                     int32_t *rows) {
    int tables = order_count * heads;
    int run_start = 0;
    for (int t = 0; t < count; t++) {
        if (t == 0 || row_slots[t] != row_slots[t - 1]) run_start = t;
        const int32_t *prev = slot_prev + 2 * row_slots[t];
        int position = slot_length[row_slots[t]] + t - run_start;
        for (int o = 0; o < order_count; o++)
            for (int h = 0; h < heads; h++) {
                int table = o * heads + h, order = orders[o];
                if (position < order - 1) {
                    rows[t * tables + table] = -1;
                    continue;
                }
                uint32_t acc = 0x9E3779B9u * (uint32_t)(table + 1);
                for (int j = 0; j < order; j++) {
                    int back = t - run_start - j;
                    int token = back >= 0 ? tokens[run_start + back] : prev[back + 2];
                    acc = (acc ^ (uint32_t)token) * 0x01000193u;
                }
                acc ^= acc >> 15;
                rows[t * tables + table] = table * engram_slots + (int)(acc % (uint32_t)engram_slots);
            }
    }
}

/* The causal conv of ApplyEngramBatch (src/Needle/Engine.cs:2421-2453): per
 * token, a window of the slot's last 9 values and its own (history [slot][9]
 * [dim], values [count][dim]); out = sum_j taps[j] * window[9 - j*dilation],
 * j = 0..3 in order; a run's last window (minus its oldest entry) becomes the
 * slot's new history (history_out). */
void ndo_engram_conv(const float *history_in, const float *values, const int32_t *row_slots, int count,
                     const float *taps, int dilation, int dim, float *out, float *history_out) {
    enum { H = 9 };
    float *stage = (float *)malloc(sizeof(float) * (size_t)(H + 1) * dim);
    for (int rs = 0; rs < count;) {
        int slot = row_slots[rs], rk = rs;
        while (rk + 1 < count && row_slots[rk + 1] == slot) rk++;
        memcpy(stage, history_in + (size_t)slot * H * dim, sizeof(float) * (size_t)H * dim);
        for (int t = rs; t <= rk; t++) {
            if (t > rs) memmove(stage, stage + dim, sizeof(float) * (size_t)H * dim);
            memcpy(stage + (size_t)H * dim, values + (size_t)t * dim, sizeof(float) * (size_t)dim);
            float *o = out + (size_t)t * dim;
            for (int c = 0; c < dim; c++) o[c] = 0.0f;
            for (int j = 0; j < 4; j++)
                for (int c = 0; c < dim; c++) o[c] += taps[(size_t)j * dim + c] * stage[(size_t)(H - j * dilation) * dim + c];
        }
        memcpy(history_out + (size_t)slot * H * dim, stage + dim, sizeof(float) * (size_t)H * dim);
        rs = rk + 1;
    }
    free(stage);
}

/* The gate of ApplyEngramBatch (src/Needle/Engine.cs:2455-2466), one token:
 * residual += sigmoid(dot(RmsUnit(x), RmsUnit(key)) / sqrt(dim)) * v. */
void ndo_engram_gate(const float *x, const float *key, const float *v, int dim, float *residual) {
    float ia = ndo_inverse_rms(x, dim), ib = ndo_inverse_rms(key, dim);
    float dot = 0.0f;
    for (int i = 0; i < dim; i++) dot += (x[i] * ia) * (key[i] * ib);
    float alpha = ndo_sigmoid(dot * (1.0f / sqrtf((float)dim)));
    for (int i = 0; i < dim; i++) residual[i] += alpha * v[i];
}

/* ------------------------------------------------------------------------ */
/* Confidence head (Needle-3 probe pooling)                                  */
/* ------------------------------------------------------------------------ */

static float dot_seq(const float *a, const float *b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* EngineCore.PoolTokensBatch (src/Needle/Engine.cs:2598-2650) for one layer
 * row: per token the slot's cell (the mean of the 4 streams, or stream 0 for
 * the first token of an initial batch) scores against each probe, and the
 * probe's online-softmax pool (max, sum, acc [dim]) absorbs it.  State per
 * slot: cell [dim], pool_max / pool_sum [pool_rows], pool_acc [pool_rows][dim];
 * with pending[slot] set, a run's first token first restores the probe's pool
 * from the snapshot arrays. */
void ndo_conf_pool_update(int row, const float *streams, const int32_t *row_slots, int count, int initial,
                          const float *probe_vectors, int probes, int dim, int pool_rows, float *cell, float *pool_max,
                          float *pool_sum, float *pool_acc, const float *snap_max, const float *snap_sum,
                          const float *snap_acc, const uint8_t *pending) {
    float inverse_root = 1.0f / sqrtf((float)dim);
    float *c = (float *)malloc(sizeof(float) * (size_t)dim);
    for (int rs = 0; rs < count;) {
        int slot = row_slots[rs], rk = rs;
        while (rk + 1 < count && row_slots[rk + 1] == slot) rk++;
        memcpy(c, cell + (size_t)slot * dim, sizeof(float) * (size_t)dim);
        float *mx = pool_max + (size_t)slot * pool_rows, *sm = pool_sum + (size_t)slot * pool_rows;
        float *ac = pool_acc + (size_t)slot * pool_rows * dim;
        int restore = pending && pending[slot];
        for (int t = rs; t <= rk; t++) {
            const float *st = streams + (size_t)t * 4 * dim;
            if (initial && t == rs) memcpy(c, st, sizeof(float) * (size_t)dim);
            else ndo_mix4(st, dim, 0.25f, 0.25f, 0.25f, 0.25f, c);
            for (int pr = 0; pr < probes; pr++) {
                int index = row * probes + pr;
                float *acc = ac + (size_t)index * dim;
                if (restore && t == rs) {
                    mx[index] = snap_max[(size_t)slot * pool_rows + index];
                    sm[index] = snap_sum[(size_t)slot * pool_rows + index];
                    memcpy(acc, snap_acc + ((size_t)slot * pool_rows + index) * dim, sizeof(float) * (size_t)dim);
                }
                float score = dot_seq(c, probe_vectors + (size_t)index * dim, dim) * inverse_root;
                if (score > mx[index]) {
                    float rescale = exp_rn(mx[index] - score);
                    sm[index] = sm[index] * rescale + 1.0f;
                    for (int i = 0; i < dim; i++) acc[i] = rescale * acc[i] + 1.0f * c[i];
                    mx[index] = score;
                } else {
                    float weight = exp_rn(score - mx[index]);
                    sm[index] += weight;
                    for (int i = 0; i < dim; i++) acc[i] += weight * c[i];
                }
            }
        }
        memcpy(cell + (size_t)slot * dim, c, sizeof(float) * (size_t)dim);
        rs = rk + 1;
    }
    free(c);
}

/* EngineCore.ConfidenceLogitForSlot (src/Needle/Engine.cs:2702-2738) from a
 * slot's pools (rows = pool_rows): each pooled mean, RMS-normalised and
 * gained, forms the key of a row; each query attends over the rows
 * (softmax of dot / sqrt(dim) + row bias) and the pooled queries project to
 * the logit.  pooled_out [queries][dim] (nullable). */
float ndo_conf_logit(const float *pool_sum, const float *pool_acc, int pool_rows, int dim, const float *gain,
                     const float *query_vectors, const float *row_bias, float bias, const float *projection,
                     int queries, float *pooled_out) {
    float inverse_root = 1.0f / sqrtf((float)dim);
    float *v = (float *)malloc(sizeof(float) * (size_t)pool_rows * dim);
    float *w = (float *)malloc(sizeof(float) * (size_t)pool_rows);
    float *pooled = (float *)malloc(sizeof(float) * (size_t)queries * dim);
    for (int i = 0; i < pool_rows; i++) {
        float *vi = v + (size_t)i * dim;
        float inv_sum = 1.0f / pool_sum[i];
        for (int k = 0; k < dim; k++) vi[k] = 0.0f * 0.0f + inv_sum * pool_acc[(size_t)i * dim + k];
        float inv = ndo_inverse_rms(vi, dim);
        for (int k = 0; k < dim; k++) vi[k] = vi[k] * inv;
        for (int k = 0; k < dim; k++) vi[k] = gain[i] * vi[k] + 0.0f * vi[k];
    }
    float logit = bias;
    for (int q = 0; q < queries; q++) {
        for (int i = 0; i < pool_rows; i++)
            w[i] = dot_seq(v + (size_t)i * dim, query_vectors + (size_t)q * dim, dim) * inverse_root +
                   row_bias[q * pool_rows + i];
        ndo_softmax(w, pool_rows);
        float *pq = pooled + (size_t)q * dim;
        for (int k = 0; k < dim; k++) pq[k] = 0.0f;
        for (int i = 0; i < pool_rows; i++)
            for (int k = 0; k < dim; k++) pq[k] += w[i] * v[(size_t)i * dim + k];
    }
    logit += dot_seq(pooled, projection, queries * dim);
    if (pooled_out) memcpy(pooled_out, pooled, sizeof(float) * (size_t)queries * dim);
    free(v);
    free(w);
    free(pooled);
    return logit;
}

/* ------------------------------------------------------------------------ */
/* Quantized matmul                                                          */
/* ------------------------------------------------------------------------ */

/* Codebook.Fill (src/Needle/Model.cs:44-52); MathF.Round is half-to-even. */
void ndo_codebook_fill(ndo_codebook *book, const float *levels, int count) {
    float peak = 0.0f;
    for (int i = 0; i < count; i++) peak = maxf_cs(peak, fabsf(levels[i]));
    book->byte_scale = peak / 63.0f;
    for (int i = 0; i < 16; i++) book->levels[i] = levels[i % count];
    for (int i = 0; i < 32; i++)
        book->bytes[i] = i % 16 < count ? (uint8_t)(rintf(levels[i % 16] / book->byte_scale) + 63.0f) : 0;
}

/* Quant.PrepareRange scalar branch (src/Needle/Quant.cs:471-484): per
 * 128-group FWHT, int8 quantize, plane reorder, offset = 63*sum(q). */
void ndo_prepare_cq(const float *x, int tokens, int cols, int bits, int8_t *values, float *scales,
                    float *offsets, int stride) {
    int groups = cols / 128;
    float rotated[128];
    int8_t quantized[128];
    for (int t = 0; t < tokens; t++)
        for (int g = 0; g < groups; g++) {
            int slot = t * stride + g;
            int sum;
            ndo_hadamard128(x + (size_t)t * cols + g * 128, rotated);
            scales[slot] = ndo_quantize_int8(rotated, 128, quantized);
            ndo_planes(quantized, bits, values + ((size_t)t * groups + g) * 128, &sum);
            offsets[slot] = 63.0f * (float)sum;
        }
}

/* Quant.GatherRow scalar path (src/Needle/Quant.cs:566-576): Scalar.DecodeRow
 * (src/Needle/Scalar.cs:130-144), levels[index] * norm in natural column
 * order, then Scalar.Hadamard in place per 128-column group. */
void ndo_gather_row_cq(const uint8_t *indices, const uint16_t *norms, const float *levels, int cols, int bits, int row,
                       float *dst) {
    int groups = cols / 128;
    int row_bytes = cols * bits / 8;
    const uint8_t *idx = indices + (size_t)row * row_bytes;
    const uint16_t *nr = norms + (size_t)row * groups;
    for (int g = 0; g < groups; g++) {
        float norm = ndo_half_to_single(nr[g]);
        float *d = dst + g * 128;
        for (int i = 0; i < 128; i++)
            d[i] = bits == 2 ? levels[idx[g * 32 + i / 4] >> (i % 4 * 2) & 3] * norm
                             : levels[idx[g * 64 + i / 2] >> (i % 2 * 4) & 15] * norm;
        ndo_hadamard128(d, d);
    }
}

/* Scalar.MatMulRows (src/Needle/Scalar.cs:146-192). */
void ndo_matmul_rows_cq(const uint8_t *indices, const uint16_t *norms, const ndo_codebook *book, int rows,
                        int cols, int bits, const int8_t *values, const float *scales, const float *offsets,
                        int stride, int tokens, float *y, int ldy, int row_start, int row_end) {
    (void)rows;
    int groups = cols / 128;
    int row_bytes = cols * bits / 8;
    const uint8_t *table = book->bytes;
    float byte_scale = book->byte_scale;
    for (int t = 0; t < tokens; t++) {
        const int8_t *v = values + (size_t)t * cols;
        const float *sc = scales + (size_t)t * stride;
        const float *off = offsets + (size_t)t * stride;
        for (int n = row_start; n < row_end; n++) {
            const uint8_t *packed = indices + (size_t)n * row_bytes;
            const uint16_t *nr = norms + (size_t)n * groups;
            float accumulator = 0.0f, bias = 0.0f;
            for (int g = 0; g < groups; g++) {
                const int8_t *x = v + g * 128;
                int dot = 0;
                if (bits == 2) {
                    const uint8_t *p = packed + g * 32;
                    for (int j = 0; j < 32; j++) {
                        int b = p[j];
                        dot += table[b & 3] * x[j] + table[b >> 2 & 3] * x[32 + j] + table[b >> 4 & 3] * x[64 + j] +
                               table[b >> 6 & 3] * x[96 + j];
                    }
                } else {
                    const uint8_t *p = packed + g * 64;
                    for (int half = 0; half < 2; half++)
                        for (int j = 0; j < 32; j++) {
                            int b = p[half * 32 + j];
                            dot += table[b & 15] * x[2 * half * 32 + j] + table[b >> 4] * x[(2 * half + 1) * 32 + j];
                        }
                }
                float scaled = (ndo_half_to_single(nr[g]) * byte_scale) * sc[g];
                accumulator += scaled * (float)dot;
                bias += scaled * off[g];
            }
            y[(size_t)t * ldy + n] = accumulator - bias;
        }
    }
}

/* I8G32: the Scalar.MatMulRows skeleton (Scalar.cs:146-192) with raw int8
 * weights and 32-column groups.  The activation scale is one per row, so it
 * is factored out of the group sum:
 *   acc = fmaf(half(sw[n][g]), (float)D[t][n][g], acc)   for g ascending
 *   y[t][n] = acc * sa[t]
 * (the per-group fused multiply-add mirrors the reference's SIMD GEMV,
 * src/Needle/Gemv.cs:259-316, which folds each group's int32 dot into the
 * float accumulator with an FMA). */
void ndo_matmul_i8g32(const int8_t *w, const uint16_t *sw, int n_rows, int k, const int8_t *q, const float *sa,
                      int m, int32_t *acc, float *y, int ldy) {
    int groups = k / 32;
    for (int t = 0; t < m; t++) {
        const int8_t *x = q + (size_t)t * k;
        for (int n = 0; n < n_rows; n++) {
            const int8_t *row = w + (size_t)n * k;
            const uint16_t *scales = sw + (size_t)n * groups;
            float accumulator = 0.0f;
            for (int g = 0; g < groups; g++) {
                int dot = 0;
                for (int j = 0; j < 32; j++) dot += row[g * 32 + j] * x[g * 32 + j];
                if (acc) acc[((size_t)t * n_rows + n) * groups + g] = dot;
                accumulator = fmaf(ndo_half_to_single(scales[g]), (float)dot, accumulator);
            }
            y[(size_t)t * ldy + n] = accumulator * sa[t];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Attention                                                                 */
/* ------------------------------------------------------------------------ */

/* Scalar.AttentionHead (src/Needle/Scalar.cs:290-312). */
void ndo_attention_head(const int8_t *query, float query_scale, const int8_t *keys, const float *key_scales,
                        const int8_t *values, const float *value_scales, int key_stride, int value_stride,
                        int scale_stride, int first, int last, int qk_dim, int v_dim, float inv_sqrt_dim,
                        float *scores, float *output, float *probabilities) {
    int count = last - first + 1;
    float scale = query_scale * inv_sqrt_dim;
    for (int s = 0; s < count; s++) {
        const int8_t *key = keys + (size_t)(first + s) * key_stride;
        int dot = 0;
        for (int d = 0; d < qk_dim; d++) dot += query[d] * key[d];
        scores[s] = ((float)dot * key_scales[(size_t)(first + s) * scale_stride]) * scale;
    }
    ndo_softmax(scores, count);
    if (probabilities)
        for (int s = 0; s < count; s++) probabilities[first + s] = scores[s];
    for (int d = 0; d < v_dim; d++) output[d] = 0.0f;
    for (int s = 0; s < count; s++) {
        const int8_t *row = values + (size_t)(first + s) * value_stride;
        float weight = scores[s] * value_scales[(size_t)(first + s) * scale_stride];
        for (int d = 0; d < v_dim; d++) output[d] += weight * (float)row[d];
    }
}

/* Attention.GroupAvx2 (src/Needle/Blocks.cs:178-185) for one head of an
 * unsplit tile, the reference's AVX2 attention tier: ScoresAvx2 (:274-336,
 * exact int32 dots, s = (dot * ks) * (qs / sqrt(d))), Normalizers (:188-199)
 * with ExponentiateAcrossPositions (:362-404: e = Ops.Exp(s - max), summed in
 * four partial sums by position modulo 4 with the tail positions in the
 * first, combined as (s0 + s1) + (s2 + s3); inverse = 1 / total), ValuesFloat
 * (:413-420: w = e * vs) and AccumulateFloat (:494-541: acc = fma(w, v, acc)
 * in position order; out = acc * inverse). */
void ndo_attention_head_simd(const int8_t *query, float query_scale, const int8_t *keys, const float *key_scales,
                             const int8_t *values, const float *value_scales, int key_stride, int value_stride,
                             int scale_stride, int first, int last, int qk_dim, int v_dim, float inv_sqrt_dim,
                             float *scores, float *output) {
    int count = last - first + 1;
    float scale = query_scale * inv_sqrt_dim;
    float peak = -INFINITY;
    for (int s = 0; s < count; s++) {
        const int8_t *key = keys + (size_t)(first + s) * key_stride;
        int dot = 0;
        for (int d = 0; d < qk_dim; d++) dot += query[d] * key[d];
        scores[s] = ((float)dot * key_scales[(size_t)(first + s) * scale_stride]) * scale;
        peak = maxf_cs(peak, scores[s]);
    }
    float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int s = 0;
    for (; s + 4 <= count; s += 4)
        for (int k = 0; k < 4; k++) {
            scores[s + k] = ops_exp(scores[s + k] - peak);
            sum[k] += scores[s + k];
        }
    for (; s < count; s++) {
        scores[s] = ops_exp(scores[s] - peak);
        sum[0] += scores[s];
    }
    const float inverse = 1.0f / ((sum[0] + sum[1]) + (sum[2] + sum[3]));
    for (s = 0; s < count; s++) scores[s] *= value_scales[(size_t)(first + s) * scale_stride];
    for (int d = 0; d < v_dim; d++) output[d] = 0.0f;
    for (s = 0; s < count; s++) {
        const int8_t *row = values + (size_t)(first + s) * value_stride;
        for (int d = 0; d < v_dim; d++) output[d] = fmaf(scores[s], (float)row[d], output[d]);
    }
    for (int d = 0; d < v_dim; d++) output[d] *= inverse;
}

/* Attention.MergePartials, non-SIMD branch (src/Needle/Blocks.cs:750-817). */
void ndo_merge_partials(const float *partials, int count, int heads, int stride, int peak_off, float *output) {
    float weights[64];
    for (int h = 0; h < heads; h++) {
        if (count == 2) {
            float peak0 = partials[peak_off + h];
            float peak1 = partials[stride + peak_off + h];
            float pk = maxf_cs(peak0, peak1);
            float w0 = exp_rn(peak0 - pk), w1 = exp_rn(peak1 - pk);
            float tot = 0.0f;
            tot += w0 * partials[peak_off + 8 + h];
            tot += w1 * partials[stride + peak_off + 8 + h];
            float inv = 1.0f / tot;
            for (int d = 0; d < 64; d++)
                output[h * 64 + d] = (w0 * partials[h * 64 + d] + w1 * partials[stride + h * 64 + d]) * inv;
            continue;
        }
        float peak = -INFINITY;
        for (int c = 0; c < count; c++) peak = maxf_cs(peak, partials[c * stride + peak_off + h]);
        float total = 0.0f;
        for (int c = 0; c < count; c++) {
            weights[c] = exp_rn(partials[c * stride + peak_off + h] - peak);
            total += weights[c] * partials[c * stride + peak_off + 8 + h];
        }
        float inverse = 1.0f / total;
        for (int d = 0; d < 64; d++) {
            float sum = 0.0f;
            for (int c = 0; c < count; c++) sum += weights[c] * partials[c * stride + h * 64 + d];
            output[h * 64 + d] = sum * inverse;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Sampling: src/Needle/Ops.cs                                               */
/* ------------------------------------------------------------------------ */

/* Ops.ArgMax scalar loop (Ops.cs:1086-1089): strict >, first max wins. */
int ndo_argmax(const float *x, int n) {
    int best = 0;
    for (int i = 1; i < n; i++)
        if (x[i] > x[best]) best = i;
    return best;
}

static int tz32(uint32_t v) { return __builtin_ctz(v); }

/* Ops.ArgMaxMaskedScalar (Ops.cs:1236-1265). */
int ndo_argmax_masked(const float *x, const uint32_t *mask, int words, int length) {
    int best = -1;
    float peak = -INFINITY;
    for (int w = 0; w < words; w++) {
        uint32_t bits = mask[w];
        if (bits == 0) continue;
        int bottom = w * 32;
        if (bits == 0xFFFFFFFFu) {
            int top = bottom + 32 <= length ? bottom + 32 : length;
            for (int id = bottom; id < top; id++) {
                float value = x[id];
                if (value > peak) { peak = value; best = id; }
            }
            continue;
        }
        while (bits != 0) {
            int id = bottom + tz32(bits);
            bits &= bits - 1;
            if (id >= length) continue;
            float value = x[id];
            if (value > peak) { peak = value; best = id; }
        }
    }
    return best;
}

/* Ops.ScalarBestProbability (Ops.cs:1530-1535). */
float ndo_best_probability(const float *values, int count, float best) {
    float total = 0.0f;
    for (int i = 0; i < count; i++) total += exp_rn(values[i] - best);
    return 1.0f / total;
}

/* NeedleSession.ArgMaxSparse (src/Needle/NeedleSession.cs:984-995): over
 * the values of a sparse head list (Engine.LogitsForBatchRow order), the id
 * of the first entry holding the strict maximum (-1 when no value exceeds
 * -inf) and BestProbability over all listed values (0 when none). */
int ndo_argmax_sparse(const float *values, const int32_t *rows, int count, float *probability) {
    int best = -1;
    float peak = -INFINITY;
    for (int i = 0; i < count; i++) {
        float value = values[i];
        if (value > peak) { peak = value; best = rows[i]; }
    }
    *probability = best < 0 ? 0.0f : ndo_best_probability(values, count, peak);
    return best;
}

/* Ops.ArgMaxMaskedWithProbability scalar branch (Ops.cs:1302-1330). */
int ndo_argmax_masked_with_probability(const float *x, const uint32_t *mask, int words, int length,
                                       float *scratch, float *probability) {
    int best = -1, count = 0;
    float peak = -INFINITY;
    for (int w = 0; w < words; w++) {
        uint32_t bits = mask[w];
        while (bits != 0) {
            int id = w * 32 + tz32(bits);
            bits &= bits - 1;
            if (id >= length) continue;
            float value = x[id];
            scratch[count++] = value;
            if (value > peak) { peak = value; best = id; }
        }
    }
    if (best < 0) {
        *probability = 0.0f;
        return -1;
    }
    *probability = ndo_best_probability(scratch, count, peak);
    return best;
}

/* Ops.TopKLogSoftmax, scalar branch (Ops.cs:1092-1221): insertion top-k
 * ordered by (value desc, index asc); log-sum-exp accumulated in double. */
void ndo_topk_logsoftmax(const float *x, int n, int k, int *indices, float *log_probs, float *probs,
                         int mask_special_023) {
    float top_val[64];
    int top_idx[64];
    for (int i = 0; i < k; i++) { top_val[i] = -INFINITY; top_idx[i] = -1; }
    float min_val = -INFINITY;
    int min_idx = 0x7FFFFFFF;
    int start = 0;
    if (mask_special_023 && n > 1) {
        top_val[0] = x[1];
        top_idx[0] = 1;
        if (k == 1) { min_val = top_val[0]; min_idx = 1; }
        start = 4;
    }
    for (int i = start; i < n; i++) {
        if (mask_special_023 && (i == 0 || i == 2 || i == 3)) continue;
        float v = x[i];
        if (v > min_val || (v == min_val && i < min_idx)) {
            int pos = k - 1;
            while (pos > 0 && (v > top_val[pos - 1] || (v == top_val[pos - 1] && i < top_idx[pos - 1]))) {
                top_val[pos] = top_val[pos - 1];
                top_idx[pos] = top_idx[pos - 1];
                pos--;
            }
            top_val[pos] = v;
            top_idx[pos] = i;
            min_val = top_val[k - 1];
            min_idx = top_idx[k - 1];
        }
    }
    float peak = top_val[0];
    double total = 0.0;
    for (int i = 0; i < n; i++) {
        float v = mask_special_023 && (i == 0 || i == 2 || i == 3) ? -1e30f : x[i];
        total += exp((double)(v - peak));
    }
    float log_shift = peak + (float)log(total);
    for (int m = 0; m < k; m++) {
        indices[m] = top_idx[m];
        float lp = top_val[m] - log_shift;
        log_probs[m] = lp;
        if (probs) probs[m] = exp_rn(lp);
    }
}

/* ------------------------------------------------------------------------ */
/* Synthetic decoder: one row through every layer and the head.              */
/* Structure of EngineCore.ForwardBatch/RunAttentionBatch                    */
/* (src/Needle/Engine.cs:2303-2350, 2480-2596) with the synthetic block:     */
/* RMSNorm -> int8 QKV -> RoPE -> int8 q / KV write -> attention -> int8 O   */
/* -> residual; RMSNorm -> int8 gate/up -> SwiGLU -> int8 down -> residual.  */
/* ------------------------------------------------------------------------ */

int ndo_decoder_row(const ndo_decoder *m, int token, int pos, int capacity, int8_t *kv_k, int8_t *kv_v,
                    float *kv_ks, float *kv_vs, const float *rope_cos, const float *rope_sin, float *logits) {
    return ndo_decoder_row_cross(m, token, pos, capacity, kv_k, kv_v, kv_ks, kv_vs, rope_cos, rope_sin, 0, NULL, NULL,
                                 NULL, NULL, logits);
}

int ndo_decoder_row_cross(const ndo_decoder *m, int token, int pos, int capacity, int8_t *kv_k, int8_t *kv_v,
                          float *kv_ks, float *kv_vs, const float *rope_cos, const float *rope_sin, int frames,
                          const int8_t *mem_k, const int8_t *mem_v, const float *mem_ks, const float *mem_vs,
                          float *logits) {
    const int d = m->dim, H = m->heads, hd = m->head_dim, F = m->ffn, V = m->vocab;
    const int width = H * hd;
    const float inv_sqrt = 1.0f / sqrtf((float)hd);
    const int span = (pos + 1 > frames ? pos + 1 : frames);
    size_t floats = (size_t)d * 4 + 3 * (size_t)d + 2 * (size_t)F + F + (size_t)span + 64;
    float *buf = (float *)malloc(floats * sizeof(float));
    int8_t *qbuf = (int8_t *)malloc((size_t)(F > d ? F : d) + (size_t)width);
    if (!buf || !qbuf) {
        free(buf);
        free(qbuf);
        return -1;
    }
    float *x = buf, *h = x + d, *o = h + d, *proj = o + d, *qkv = proj + d, *gu = qkv + 3 * d, *act = gu + 2 * F,
          *scores = act + F;
    int8_t *qa = qbuf, *qq = qbuf + (F > d ? F : d);
    float qs[64];
    for (int i = 0; i < d; i++) x[i] = ndo_half_to_single(m->embedding[(size_t)token * d + i]);
    const int half = hd / 2;
    for (int l = 0; l < m->layers; l++) {
        float sa;
        ndo_rms_norm(x, m->attn_norm[l], d, h);
        sa = ndo_quantize_int8(h, d, qa);
        ndo_matmul_i8g32(m->w_qkv[l], m->s_qkv[l], 3 * d, d, qa, &sa, 1, NULL, qkv, 3 * d);
        float *q = qkv, *k = qkv + d, *v = qkv + 2 * d;
        ndo_rope(q, H, hd, rope_cos + (size_t)pos * half, rope_sin + (size_t)pos * half);
        ndo_rope(k, H, hd, rope_cos + (size_t)pos * half, rope_sin + (size_t)pos * half);
        int8_t *lk = kv_k + (size_t)l * capacity * width, *lv = kv_v + (size_t)l * capacity * width;
        float *lks = kv_ks + (size_t)l * capacity * H, *lvs = kv_vs + (size_t)l * capacity * H;
        for (int hh = 0; hh < H; hh++) qs[hh] = ndo_quantize_int8(q + hh * hd, hd, qq + hh * hd);
        for (int hh = 0; hh < H; hh++) {
            lks[(size_t)pos * H + hh] = ndo_quantize_int8(k + hh * hd, hd, lk + (size_t)pos * width + hh * hd);
            lvs[(size_t)pos * H + hh] = ndo_quantize_int8(v + hh * hd, hd, lv + (size_t)pos * width + hh * hd);
        }
        for (int hh = 0; hh < H; hh++)
            ndo_attention_head_simd(qq + hh * hd, qs[hh], lk + hh * hd, lks + hh, lv + hh * hd, lvs + hh, width, width,
                                    H, 0, pos, hd, hd, inv_sqrt, scores, o + hh * hd);
        sa = ndo_quantize_int8(o, d, qa);
        ndo_matmul_i8g32(m->w_o[l], m->s_o[l], d, d, qa, &sa, 1, NULL, proj, d);
        for (int i = 0; i < d; i++) x[i] = x[i] + proj[i];
        if (frames > 0 && m->w_cq) {
            /* cross block: queries from this row, keys/values from the memory */
            ndo_rms_norm(x, m->cross_norm[l], d, h);
            sa = ndo_quantize_int8(h, d, qa);
            ndo_matmul_i8g32(m->w_cq[l], m->s_cq[l], d, d, qa, &sa, 1, NULL, qkv, d);
            for (int hh = 0; hh < H; hh++) qs[hh] = ndo_quantize_int8(qkv + hh * hd, hd, qq + hh * hd);
            const int8_t *mk = mem_k + (size_t)l * frames * width, *mv = mem_v + (size_t)l * frames * width;
            const float *mks = mem_ks + (size_t)l * frames * H, *mvs = mem_vs + (size_t)l * frames * H;
            for (int hh = 0; hh < H; hh++)
                ndo_attention_head_simd(qq + hh * hd, qs[hh], mk + hh * hd, mks + hh, mv + hh * hd, mvs + hh, width,
                                        width, H, 0, frames - 1, hd, hd, inv_sqrt, scores, o + hh * hd);
            sa = ndo_quantize_int8(o, d, qa);
            ndo_matmul_i8g32(m->w_co[l], m->s_co[l], d, d, qa, &sa, 1, NULL, proj, d);
            for (int i = 0; i < d; i++) x[i] = x[i] + proj[i];
        }
        ndo_rms_norm(x, m->ffn_norm[l], d, h);
        sa = ndo_quantize_int8(h, d, qa);
        ndo_matmul_i8g32(m->w_gu[l], m->s_gu[l], 2 * F, d, qa, &sa, 1, NULL, gu, 2 * F);
        ndo_swiglu(gu, gu + F, F, act);
        sa = ndo_quantize_int8(act, F, qa);
        ndo_matmul_i8g32(m->w_d[l], m->s_d[l], d, F, qa, &sa, 1, NULL, proj, d);
        for (int i = 0; i < d; i++) x[i] = x[i] + proj[i];
    }
    {
        float sa;
        ndo_rms_norm(x, m->final_norm, d, h);
        sa = ndo_quantize_int8(h, d, qa);
        ndo_matmul_i8g32(m->w_head, m->s_head, V, d, qa, &sa, 1, NULL, logits, V);
    }
    free(buf);
    free(qbuf);
    return 0;
}

int ndo_cross_memory(const ndo_decoder *m, int layer, const float *memory, int frames, int8_t *k, int8_t *v, float *ks,
                     float *vs) {
    const int d = m->dim, H = m->heads, hd = m->head_dim, width = H * hd;
    int8_t *qa = (int8_t *)malloc((size_t)d);
    float *y = (float *)malloc((size_t)2 * d * sizeof(float));
    if (!qa || !y) {
        free(qa);
        free(y);
        return -1;
    }
    for (int f = 0; f < frames; f++) {
        float sa = ndo_quantize_int8(memory + (size_t)f * d, d, qa);
        ndo_matmul_i8g32(m->w_ckv[layer], m->s_ckv[layer], 2 * d, d, qa, &sa, 1, NULL, y, 2 * d);
        for (int h = 0; h < H; h++) {
            ks[(size_t)f * H + h] = ndo_quantize_int8(y + h * hd, hd, k + (size_t)f * width + h * hd);
            vs[(size_t)f * H + h] = ndo_quantize_int8(y + d + h * hd, hd, v + (size_t)f * width + h * hd);
        }
    }
    free(qa);
    free(y);
    return 0;
}
