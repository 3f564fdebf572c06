/*
 * whistle_oracle.c - CPU restatement of the Whistle encoder's front end
 * (mel features) and its table builders, the reference's scalar tier.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA library, never
 * linked into it.  Built with -ffp-contract=off, so every a*b+c below is two
 * rounded operations, as in the reference's scalar C#.  The encoder layers
 * are chained in oracle/whistle.py from needle_oracle.c's routines.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846 /* Math.PI */
#endif

/* log_rn: MathF.Log taken as the correctly rounded natural logarithm of a
 * float.  A double-precision restatement of the classic reduction: x = 2^k m
 * with m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s) with s = (m - 1)/(m + 1)
 * and the odd atanh series to s^23 (|s| <= 0.1716, so the next term is below
 * 2e-19), then k ln2 + log m with ln2 split into a 32-bit head and a tail as
 * in fdlibm.  The device's log_rn takes the same IEEE double steps (the
 * exponent from the bits, fused multiply-adds, one division), so both give
 * the same float. */
static double log_series(double s2) {
    double p = 1.0 / 23.0;
    p = fma(p, s2, 1.0 / 21.0);
    p = fma(p, s2, 1.0 / 19.0);
    p = fma(p, s2, 1.0 / 17.0);
    p = fma(p, s2, 1.0 / 15.0);
    p = fma(p, s2, 1.0 / 13.0);
    p = fma(p, s2, 1.0 / 11.0);
    p = fma(p, s2, 1.0 / 9.0);
    p = fma(p, s2, 1.0 / 7.0);
    p = fma(p, s2, 1.0 / 5.0);
    p = fma(p, s2, 1.0 / 3.0);
    return fma(p, s2, 1.0);
}

float ndo_log_rn(float x) {
    if (x != x) return x;
    if (x < 0.0f) return NAN;
    if (x == 0.0f) return -INFINITY;
    if (isinf(x)) return x;
    const double d = (double)x;  /* a float is a normal double */
    uint64_t bits;
    memcpy(&bits, &d, 8);
    int k = (int)((bits >> 52) & 0x7ff) - 1023;
    bits = (bits & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL; /* m in [1, 2) */
    double m;
    memcpy(&m, &bits, 8);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        k += 1;
    }
    const double s = (m - 1.0) / (m + 1.0);
    const double lm = 2.0 * s * log_series(s * s);
    const double ln2_hi = 6.93147180369123816490e-01, ln2_lo = 1.90821492927058770002e-10;
    return (float)((double)k * ln2_hi + fma((double)k, ln2_lo, lm));
}

void ndo_log_rn_array(const float *x, int n, float *y) {
    for (int i = 0; i < n; i++) y[i] = ndo_log_rn(x[i]);
}

/* Frontend.Create's tables (src/Needle/Frontend.cs:15-46): the Hann window
 * (0.5 - 0.5 cos(2 pi n / (window - 1)) in double), the twiddles cos and
 * -sin of 2 pi k / fft, the bit reversal and each bin's first mel and count
 * of mels between its first and last nonzero weight. */
void ndo_frontend_tables(int fft, int window, const float *mel_bank, int mels, float *hann, float *cosines,
                         float *sines, int32_t *bitrev, int32_t *mel_first, int32_t *mel_count) {
    for (int n = 0; n < window; n++) hann[n] = (float)(0.5 - 0.5 * cos(2 * M_PI * n / (window - 1)));
    for (int k = 0; k < fft / 2; k++) {
        cosines[k] = (float)cos(2 * M_PI * k / fft);
        sines[k] = (float)-sin(2 * M_PI * k / fft);
    }
    int bits = 0;
    while ((1 << (bits + 1)) <= fft) bits++;
    for (int i = 0; i < fft; i++) {
        int r = 0;
        for (int b = 0; b < bits; b++) r |= (i >> b & 1) << (bits - 1 - b);
        bitrev[i] = r;
    }
    for (int k = 0; k <= fft / 2; k++) {
        const float *row = mel_bank + (size_t)k * mels;
        int first = mels, last = -1;
        for (int m = 0; m < mels; m++)
            if (row[m] != 0.0f) {
                if (first == mels) first = m;
                last = m;
            }
        mel_first[k] = first;
        mel_count[k] = last >= first ? last - first + 1 : 0;
    }
}

/* FeatureJob.Execute for one frame (Frontend.cs:100-130) with the scalar
 * Butterflies (:205-225): the windowed segment in bit-reversed order, the
 * radix-2 stages (tr = re[b] c - im[b] s, ti = re[b] s + im[b] c, each
 * product and sum rounded), the power of bins 0..fft/2, and each mel the
 * sum of power[k] * bank[k][m] over the bins whose range holds m, in
 * ascending k (Scalar.AddScaled).  Returns the frame's peak mel. */
float ndo_mel_frame(const float *segment, int fft, int window, const float *hann, const float *cosines,
                    const float *sines, const int32_t *bitrev, const float *mel_bank, int mels,
                    const int32_t *mel_first, const int32_t *mel_count, float *mel_out) {
    static _Thread_local float re[8192], im[8192], power[4097];
    if (fft > 8192) return NAN;
    for (int i = 0; i < fft; i++) {
        re[bitrev[i]] = i < window ? segment[i] * hann[i] : 0.0f;
        im[i] = 0.0f;
    }
    for (int size = 2; size <= fft; size <<= 1) {
        const int half = size / 2, step = fft / size;
        for (int start = 0; start < fft; start += size)
            for (int k = 0; k < half; k++) {
                const float c = cosines[k * step], s = sines[k * step];
                const int a = start + k, b = a + half;
                const float tr = re[b] * c - im[b] * s;
                const float ti = re[b] * s + im[b] * c;
                re[b] = re[a] - tr;
                im[b] = im[a] - ti;
                re[a] += tr;
                im[a] += ti;
            }
    }
    for (int k = 0; k <= fft / 2; k++) power[k] = re[k] * re[k] + im[k] * im[k];
    float peak = 0.0f;
    for (int m = 0; m < mels; m++) mel_out[m] = 0.0f;
    for (int k = 0; k <= fft / 2; k++) {
        const int first = mel_first[k], count = mel_count[k];
        for (int m = first; m < first + count; m++) mel_out[m] += power[k] * mel_bank[(size_t)k * mels + m];
    }
    for (int m = 0; m < mels; m++) peak = fmaxf(peak, mel_out[m]);
    return peak;
}

/* Whistle.Normalize's scalar branch (src/Needle/Whistle.cs:263-272): per
 * column, in double, the mean over rows (sum in row order, / rows), the
 * sample standard deviation (squares of x - mean summed in row order,
 * / max(rows - 1, 1), sqrt) and x = (x - mean) / (std + 1e-5). */
void ndo_normalize_columns(float *x, int rows, int cols) {
    const int denom = rows - 1 > 1 ? rows - 1 : 1;
    for (int c = 0; c < cols; c++) {
        double sum = 0;
        for (int r = 0; r < rows; r++) sum += x[(size_t)r * cols + c];
        const double mean = sum / rows;
        double squares = 0;
        for (int r = 0; r < rows; r++) {
            const double dv = x[(size_t)r * cols + c] - mean;
            squares += dv * dv;
        }
        const double sd = sqrt(squares / denom);
        for (int r = 0; r < rows; r++) x[(size_t)r * cols + c] = (float)((x[(size_t)r * cols + c] - mean) / (sd + 1e-5));
    }
}

/* The encoder's RoPE tables (Whistle.AllocateBuffers, src/Needle/Whistle.cs:
 * 134-139): angle = p / MathF.Pow(theta, 2i / qk) in float, MathF.Cos / Sin. */
void ndo_whistle_rope_tables(float theta, int qk, int positions, float *cos_t, float *sin_t) {
    const int half = qk / 2;
    for (int p = 0; p < positions; p++)
        for (int i = 0; i < half; i++) {
            const float angle = (float)p / powf(theta, 2.0f * (float)i / (float)qk);
            cos_t[(size_t)p * half + i] = cosf(angle);
            sin_t[(size_t)p * half + i] = sinf(angle);
        }
}

/* The cross-memory position tables (Whistle.cs:142-152): angleStep =
 * -ln(10000) / (half - 1), invFreq = exp(angleStep i), sin / cos of p invFreq,
 * all in double, stored as float. */
void ndo_cross_position_tables(int dim, int positions, float *sin_t, float *cos_t) {
    const int half = dim / 2;
    const double step = -log(10000.0) / (half - 1);
    for (int i = 0; i < half; i++) {
        const double inv_freq = exp(step * i);
        for (int p = 0; p < positions; p++) {
            const double angle = p * inv_freq;
            sin_t[(size_t)p * half + i] = (float)sin(angle);
            cos_t[(size_t)p * half + i] = (float)cos(angle);
        }
    }
}

/* Scalar.Silu / Glu / MultiplyBySigmoid (src/Needle/Scalar.cs:194-204,280-283)
 * over arrays, with Sigmoid(x) = 1 / (1 + exp_rn(-x)). */
float ndo_sigmoid(float x);
void ndo_silu(float *x, int n) {
    for (int i = 0; i < n; i++) x[i] *= ndo_sigmoid(x[i]);
}
void ndo_glu(const float *value, const float *gate, float *dst, int n) {
    for (int i = 0; i < n; i++) dst[i] = value[i] * ndo_sigmoid(gate[i]);
}
void ndo_multiply_by_sigmoid(float *x, const float *gate, int n) {
    for (int i = 0; i < n; i++) x[i] *= ndo_sigmoid(gate[i]);
}
