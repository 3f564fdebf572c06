// The Whistle encoder on the device: Whistle.Encode and BuildCrossMemory
// (src/Needle/Whistle.cs:179-200, 886-914) for a loaded archive with an
// audio section (AudioWeights, src/Needle/Audio.cs:117-149), in the
// reference's scalar tier (MathF.Exp and MathF.Log as correctly rounded
// functions, every other step one IEEE rounding, as the C# loops):
//   front end   FeatureJob (Frontend.cs:82-130): CTA per frame, the Hann-
//               windowed segment in bit-reversed order in shared memory, the
//               radix-2 stages of Frontend.Butterflies' scalar loop (one
//               thread per butterfly, a barrier per stage), the power
//               spectrum, each mel summed over the bins in ascending order;
//               the peak by an integer max; log(x + floor); Normalize per mel
//               column in double, thread per column in row order
//   stem        (:282-470) thread per output element for the 3x3 convs
//               (AddScaled / MultiplyAccumulate in the (dt, df) order),
//               the 2-bit CQ pointwise matmuls over (row, frequency) tokens,
//               SiLU, the channel-major transpose, the StemOut matmul
//   encoder     (:794-828) per layer: RmsUnit + 4-bit Prepare in one kernel,
//               the three phi slices in one matmul launch, gates / Mix4 /
//               Sinkhorn4x4, MLP0 and MLP (HadamardMlp, scale 0.5), self-
//               attention (ZeroCenteredRms + Prepare, Q/K/V/gate in one
//               launch, per-head norms / RoPE at the frame index / int8,
//               every frame attending every frame, MultiplyBySigmoid +
//               Prepare, out, PostNormAdd), the convolution module (Pw1,
//               Glu, the depthwise conv over time, ZeroCenteredRms + SiLU +
//               Prepare, Pw2, residual add), CombineDiff4x4; then Mix4 by
//               1/4 and ZeroCenteredRms with the final norm
//   memory      (:755-792) the rows plus PositionMix times the position
//               tables, FakeA8 + Prepare; per decoder layer the cross K / V
//               matmuls and, warp per (frame, head), ZeroCenteredRms of the
//               key and int8 quantization of key and value.
#include <math.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "cq.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {
namespace {

constexpr int kWhWarps = 4;     // warps per CTA of the per-(frame, head) kernels
constexpr int kWhMaxFft = 4096;
constexpr int kWhMaxHead = 64;  // qk and v dims held in a warp's scratch

// log_rn: MathF.Log as the correctly rounded natural logarithm of a float, by
// a double-precision restatement of the classic reduction: x = 2^k m with m
// in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s), s = (m - 1) / (m + 1), the odd
// atanh series to s^23 (|s| <= 0.1716: the next term is below 2e-19), then
// k ln2 with ln2 split into a 32-bit head and a tail as in fdlibm.  The CPU
// restatement takes the same IEEE double steps.
__device__ __forceinline__ float log_rn(float x) {
    if (x != x) return x;
    if (x < 0.0f) return __int_as_float(0x7fc00000);
    if (x == 0.0f) return __int_as_float(0xff800000);
    if (isinf(x)) return x;
    const double d = (double)x;
    unsigned long long bits = (unsigned long long)__double_as_longlong(d);
    int k = (int)((bits >> 52) & 0x7ff) - 1023;
    bits = (bits & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;  // m in [1, 2)
    double m = __longlong_as_double((long long)bits);
    if (m > 1.4142135623730951) {
        m = __dmul_rn(m, 0.5);
        k += 1;
    }
    const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0)), s2 = __dmul_rn(s, s);
    double p = 1.0 / 23.0;
    p = __fma_rn(p, s2, 1.0 / 21.0);
    p = __fma_rn(p, s2, 1.0 / 19.0);
    p = __fma_rn(p, s2, 1.0 / 17.0);
    p = __fma_rn(p, s2, 1.0 / 15.0);
    p = __fma_rn(p, s2, 1.0 / 13.0);
    p = __fma_rn(p, s2, 1.0 / 11.0);
    p = __fma_rn(p, s2, 1.0 / 9.0);
    p = __fma_rn(p, s2, 1.0 / 7.0);
    p = __fma_rn(p, s2, 1.0 / 5.0);
    p = __fma_rn(p, s2, 1.0 / 3.0);
    p = __fma_rn(p, s2, 1.0);
    const double lm = __dmul_rn(__dmul_rn(2.0, s), p);
    const double ln2_hi = 6.93147180369123816490e-01, ln2_lo = 1.90821492927058770002e-10;
    return __double2float_rn(__dadd_rn(__dmul_rn((double)k, ln2_hi), __fma_rn((double)k, ln2_lo, lm)));
}

// FeatureJob.Execute for one frame per CTA (Frontend.cs:100-130) with the
// scalar Butterflies (:205-225).  Mel m sums the bins in [mel_lo[m],
// mel_hi[m]) whose range holds it (outside them no bin's range does), in
// ascending order.  peak_bits gets the max over frames as the bits of a
// nonnegative float (an integer max orders them the same way).
__global__ void __launch_bounds__(256) wh_mel_kernel(const float *__restrict__ padded, int hop, int fft, int window,
                                                     const float *__restrict__ hann, const float *__restrict__ cosines,
                                                     const float *__restrict__ sines, const int32_t *__restrict__ bitrev,
                                                     const float *__restrict__ bank, int mels,
                                                     const int32_t *__restrict__ mel_first,
                                                     const int32_t *__restrict__ mel_count,
                                                     const int32_t *__restrict__ mel_lo,
                                                     const int32_t *__restrict__ mel_hi, float *__restrict__ mel,
                                                     unsigned *__restrict__ peak_bits) {
    pdl_enter();
    extern __shared__ float wh_fft[];
    float *re = wh_fft, *im = re + fft, *power = im + fft;
    const int frame = blockIdx.x;
    const float *seg = padded + (size_t)frame * hop;
    for (int i = threadIdx.x; i < fft; i += blockDim.x) {
        re[bitrev[i]] = i < window ? __fmul_rn(seg[i], hann[i]) : 0.0f;
        im[i] = 0.0f;
    }
    __syncthreads();
    for (int size = 2; size <= fft; size <<= 1) {
        const int half = size >> 1, step = fft / size;
        for (int j = threadIdx.x; j < fft / 2; j += blockDim.x) {
            const int k = j % half, a = (j / half) * size + k, b = a + half;
            const float c = cosines[k * step], s = sines[k * step];
            const float rb = re[b], ib = im[b], ra = re[a], ia = im[a];
            const float tr = __fsub_rn(__fmul_rn(rb, c), __fmul_rn(ib, s));
            const float ti = __fadd_rn(__fmul_rn(rb, s), __fmul_rn(ib, c));
            re[b] = __fsub_rn(ra, tr);
            im[b] = __fsub_rn(ia, ti);
            re[a] = __fadd_rn(ra, tr);
            im[a] = __fadd_rn(ia, ti);
        }
        __syncthreads();
    }
    for (int k = threadIdx.x; k <= fft / 2; k += blockDim.x)
        power[k] = __fadd_rn(__fmul_rn(re[k], re[k]), __fmul_rn(im[k], im[k]));
    __syncthreads();
    for (int m = threadIdx.x; m < mels; m += blockDim.x) {
        float acc = 0.0f;
        for (int k = mel_lo[m]; k < mel_hi[m]; k++) {  // the bins whose range can hold m, ascending
            const int first = mel_first[k];
            if (m >= first && m < first + mel_count[k])
                acc = __fadd_rn(acc, __fmul_rn(power[k], bank[(size_t)k * mels + m]));
        }
        mel[(size_t)frame * mels + m] = acc;
        atomicMax(peak_bits, __float_as_uint(fmaxf(acc, 0.0f)));
    }
}

// FeatureJob.Logarithm (Frontend.cs:91-98): x = log(x + floor), floor =
// max(peak * 1e-8, 1e-30).
__global__ void wh_log_kernel(float *__restrict__ mel, long long n, const unsigned *__restrict__ peak_bits) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float floor = fmaxf(__fmul_rn(__uint_as_float(*peak_bits), 1e-8f), 1e-30f);
    mel[i] = log_rn(__fadd_rn(mel[i], floor));
}

// Whistle.Normalize's scalar branch (Whistle.cs:263-272): per column, in
// double, the sum in row order / rows, then the squares of x - mean in row
// order, sd = sqrt(squares / max(rows - 1, 1)); den = sd + 1e-5.  One CTA,
// a thread per column running its add chain over tiles of kMomRows rows in
// shared memory; thread 0 brings the next tile (one contiguous block of the
// [rows][cols] features) with a bulk copy while the chains run on the
// current one, so the chains never wait on global memory.  A wait that runs
// out sets *status (the encode then reports NDL_ERR_TIMEOUT).
constexpr int kMomRows = 128;
constexpr uint32_t kMomWaitLimit = 1u << 16;  // tests of about 1 us each

__global__ void __launch_bounds__(128) wh_moments_kernel(const float *__restrict__ x, int rows, int cols,
                                                         double *__restrict__ mean_out, double *__restrict__ den_out,
                                                         int *__restrict__ status) {
    pdl_enter();
    extern __shared__ __align__(16) float mom_tile[];  // [2][kMomRows][cols]
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int failed;
    const int tid = threadIdx.x;
    const int tiles = (rows + kMomRows - 1) / kMomRows, denom = rows - 1 > 1 ? rows - 1 : 1;
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_mbar_init();
        failed = 0;
    }
    __syncthreads();
    auto issue = [&](int g) {  // sweep-wide tile g into buffer g & 1 (thread 0)
        const int t = g % tiles, r0 = t * kMomRows, n = min(kMomRows, rows - r0);
        const uint32_t bytes = (uint32_t)(((size_t)n * cols * 4 + 15) & ~(size_t)15);
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&bars[g & 1], bytes);
        bulk_g2s(mom_tile + (size_t)(g & 1) * kMomRows * cols, x + (size_t)r0 * cols, bytes, &bars[g & 1]);
    };
    if (tid == 0) issue(0);
    double mean = 0.0;
    for (int pass = 0; pass < 2; pass++) {
        double acc = 0.0;
        for (int t = 0; t < tiles; t++) {
            const int g = pass * tiles + t;
            if (tid == 0 && g + 1 < 2 * tiles) issue(g + 1);  // its buffer was released by the barrier below
            if (!mbar_wait_bounded(&bars[g & 1], (uint32_t)(g >> 1) & 1u, kMomWaitLimit)) failed = 1;
            const float *cur = mom_tile + (size_t)(g & 1) * kMomRows * cols;
            if (tid < cols && !failed) {
                const int n = min(kMomRows, rows - t * kMomRows);
                int r = 0;
                for (; r + 16 <= n; r += 16) {  // 16 loads and conversions ahead of 16 chained adds
                    double v[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) v[k] = (double)cur[(r + k) * cols + tid];
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        if (pass == 0) {
                            acc = __dadd_rn(acc, v[k]);
                        } else {
                            const double dv = __dsub_rn(v[k], mean);
                            acc = __dadd_rn(acc, __dmul_rn(dv, dv));
                        }
                    }
                }
                for (; r < n; r++) {
                    const double v = (double)cur[r * cols + tid];
                    if (pass == 0) {
                        acc = __dadd_rn(acc, v);
                    } else {
                        const double dv = __dsub_rn(v, mean);
                        acc = __dadd_rn(acc, __dmul_rn(dv, dv));
                    }
                }
            }
            __syncthreads();
        }
        if (tid < cols) {
            if (pass == 0) {
                mean = __ddiv_rn(acc, (double)rows);
            } else {
                mean_out[tid] = mean;
                den_out[tid] = __dadd_rn(__dsqrt_rn(__ddiv_rn(acc, (double)denom)), 1e-5);
            }
        }
    }
    if (tid == 0 && failed) atomicOr(status, kStatusTimeout);
}

// x = (float)((x - mean) / den) per element.
__global__ void wh_standardize_kernel(float *__restrict__ x, long long n, int cols, const double *__restrict__ mean,
                                      const double *__restrict__ den) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int c = (int)(i % cols);
    x[i] = __double2float_rn(__ddiv_rn(__dsub_rn((double)x[i], mean[c]), den[c]));
}

// Stem stage 1 (ExecuteStageFirst, Whistle.cs:346-375): out[p][f][c] = SiLU
// of the 3x3 conv at stride 2 over (time, mel), AddScaled in (dt, df) order;
// rows outside [0, l0) read zeros, frequencies outside [0, mels) are skipped.
__global__ void wh_stem1_kernel(const float *__restrict__ feats, int l0, int mels, const float *__restrict__ w, int s,
                                int l1, float *__restrict__ out) {
    pdl_enter();
    // 32-bit index arithmetic (a stage holds fewer than 2^31 elements, checked when the encoder is created):
    // a 64-bit division is a long software sequence on the GPU
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (unsigned)l1 * 40u * (unsigned)s) return;
    const unsigned pf = i / (unsigned)s;
    const int c = (int)(i - pf * (unsigned)s), f = (int)(pf % 40u), p = (int)(pf / 40u);
    float o = 0.0f;
    for (int dt = 0; dt < 3; dt++) {
        const int r = 2 * p - 1 + dt;
        for (int df = 0; df < 3; df++) {
            const int freq = 2 * f - 1 + df;
            if (freq < 0 || freq >= mels) continue;
            const float v = r >= 0 && r < l0 ? feats[(size_t)r * mels + freq] : 0.0f;
            o = __fadd_rn(o, __fmul_rn(v, w[(dt * 3 + df) * s + c]));
        }
    }
    out[i] = __fmul_rn(o, sigmoid_rn(o));
}

// Whistle.Depthwise (Whistle.cs:326-344) at stride 2 in time and frequency:
// out[q][f][c] = sum over (dt, df) of src[2q-1+dt][2f-1+df][c] * w[dt*3+df][c]
// (MultiplyAccumulate order), rows outside [0, rows_in) zeros.
__global__ void wh_depthwise_kernel(const float *__restrict__ src, int rows_in, int freq_in,
                                    const float *__restrict__ w, int s, int rows_out, int freq_out,
                                    float *__restrict__ out) {
    pdl_enter();
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;  // 32-bit index arithmetic, as in wh_stem1_kernel
    if (i >= (unsigned)rows_out * (unsigned)freq_out * (unsigned)s) return;
    const unsigned pf = i / (unsigned)s;
    const int c = (int)(i - pf * (unsigned)s), f = (int)(pf % (unsigned)freq_out), q = (int)(pf / (unsigned)freq_out);
    float o = 0.0f;
    for (int dt = 0; dt < 3; dt++) {
        const int r = 2 * q - 1 + dt;
        for (int df = 0; df < 3; df++) {
            const int freq = 2 * f - 1 + df;
            if (freq < 0 || freq >= freq_in) continue;
            const float v = r >= 0 && r < rows_in ? src[((size_t)r * freq_in + freq) * s + c] : 0.0f;
            o = __fadd_rn(o, __fmul_rn(v, w[(dt * 3 + df) * s + c]));
        }
    }
    out[i] = o;
}

// Scalar.Silu in place.
__global__ void wh_silu_kernel(float *__restrict__ x, long long n) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fmul_rn(x[i], sigmoid_rn(x[i]));
}

// ExecuteStageThirdTranspose (Whistle.cs:427-440): SiLU, then flat[r][c*10 + f]
// = row[r][f][c].
__global__ void wh_silu_transpose_kernel(const float *__restrict__ src, int rows, int s, float *__restrict__ flat) {
    pdl_enter();
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;  // 32-bit index arithmetic, as in wh_stem1_kernel
    if (i >= (unsigned)rows * 10u * (unsigned)s) return;
    const unsigned pf = i / (unsigned)s;
    const int c = (int)(i - pf * (unsigned)s), f = (int)(pf % 10u), r = (int)(pf / 10u);
    const float v = src[i];
    flat[(size_t)r * 10 * s + (size_t)c * 10 + f] = __fmul_rn(v, sigmoid_rn(v));
}

// ExecuteCopyLanes (Whistle.cs:553-562): the stem rows into all four lanes.
__global__ void wh_lanes_kernel(const float *__restrict__ stem, long long frames, int dim, float *__restrict__ stream) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= frames * 4 * dim) return;
    const long long t = i / (4LL * dim);
    stream[i] = stem[t * dim + i % dim];
}

__device__ __forceinline__ float wh_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Ops.InverseRms over a warp's scratch: squares summed in order on lane 0.
__device__ __forceinline__ float wh_inverse_rms(const float *x, int n, int lane) {
    float sum = 0.0f;
    if (lane == 0)
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
    sum = __shfl_sync(0xffffffffu, sum, 0);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), 1e-6f)));
}

// Quant.QuantizeInt8 of a warp's scratch into dst; returns the scale.
__device__ __forceinline__ float wh_quantize(const float *x, int n, int8_t *dst, int lane) {
    float peak = 0.0f;
    for (int i = lane; i < n; i += 32) peak = fmaxf(peak, fabsf(x[i]));
    peak = wh_warp_max(peak);
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    for (int i = lane; i < n; i += 32) dst[i] = (int8_t)fminf(fmaxf(rintf(__fmul_rn(x[i], inverse)), -128.0f), 127.0f);
    return scale;
}

// ZeroCenteredRms of a head's qk values held in the warp's scratch b (in place).
__device__ __forceinline__ void wh_head_norm(float *b, const float *__restrict__ scale, int qk, int lane) {
    __syncwarp();
    const float inv = wh_inverse_rms(b, qk, lane);
    __syncwarp();
    for (int i = lane; i < qk; i += 32) b[i] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, scale[i]), b[i]), inv);
    __syncwarp();
}

// ExecuteAttnRopeQuantize (Whistle.cs:642-669), warp per (frame, head): q
// heads, then kv heads.  ZeroCenteredRms with q_norm / k_norm, RoPE at the
// frame index (half-split, Scalar.Rope), QuantizeInt8 per head; a kv head's
// value row is quantized as it is.
__global__ void __launch_bounds__(32 * kWhWarps) wh_qkv_kernel(
    const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v, int frames, int heads,
    int kv, int qk, int vd, const float *__restrict__ q_norm, const float *__restrict__ k_norm,
    const float *__restrict__ rope_cos, const float *__restrict__ rope_sin, int8_t *__restrict__ q8,
    float *__restrict__ qs, int8_t *__restrict__ keys, float *__restrict__ ks, int8_t *__restrict__ values,
    float *__restrict__ vs) {
    pdl_enter();
    __shared__ float buf[kWhWarps][kWhMaxHead];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * kWhWarps + warp;
    if (item >= frames * (heads + kv)) return;
    const int t = item / (heads + kv), h = item - t * (heads + kv);
    const bool is_q = h < heads;
    const int hh = is_q ? h : h - heads;
    const float *x = is_q ? q + (size_t)t * heads * qk + hh * qk : k + (size_t)t * kv * qk + hh * qk;
    float *b = buf[warp];
    for (int i = lane; i < qk; i += 32) b[i] = x[i];
    wh_head_norm(b, is_q ? q_norm : k_norm, qk, lane);
    const int half = qk / 2;
    const float *cs = rope_cos + (size_t)t * half, *sn = rope_sin + (size_t)t * half;
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
        const float s = wh_quantize(b, qk, q8 + (size_t)t * heads * qk + hh * qk, lane);
        if (lane == 0) qs[(size_t)t * heads + hh] = s;
        return;
    }
    const float kscale = wh_quantize(b, qk, keys + (size_t)t * kv * qk + hh * qk, lane);
    if (lane == 0) ks[(size_t)t * kv + hh] = kscale;
    __syncwarp();
    const float *vx = v + (size_t)t * kv * vd + hh * vd;
    for (int i = lane; i < vd; i += 32) b[i] = vx[i];
    __syncwarp();
    const float vscale = wh_quantize(b, vd, values + (size_t)t * kv * vd + hh * vd, lane);
    if (lane == 0) vs[(size_t)t * kv + hh] = vscale;
}

// Scalar.AttentionHead (src/Needle/Scalar.cs:290-312) over every frame
// (AttentionBatch.Span with Frames set: [0, frames), Blocks.cs:970-975).  CTA
// per (kv head, four (frame, grouped head) items): the kv head's int8 keys,
// values and scales of every frame are staged in shared memory once, then
// warp per item: s_j = (dot_j * ks_j) * (qs / sqrt(qk)) with dp4a dots;
// e_j = MathF.Exp(s_j - max) summed in frame order; w_j = (e_j / total) * vs_j;
// out[d] += w_j * v_j[d] in frame order, dims d and d + 32 of a lane side by
// side.
__global__ void __launch_bounds__(32 * kWhWarps) wh_attention_kernel(
    const int8_t *__restrict__ q8, const float *__restrict__ qs, int frames, int heads, int kv, int qk, int vd,
    float inv_sqrt, const int8_t *__restrict__ keys, const float *__restrict__ ks, const int8_t *__restrict__ values,
    const float *__restrict__ vs, float *__restrict__ out) {
    pdl_enter();
    extern __shared__ __align__(16) int wh_att[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, kh = blockIdx.y;
    const int group = heads / kv, kwords = qk / 4, vwords = vd / 4;
    int *kst = wh_att;                                               // [frames][qk / 4]
    int *vst = kst + (size_t)frames * kwords;                        // [frames][vd / 4]
    float *kss = reinterpret_cast<float *>(vst + (size_t)frames * vwords);  // [frames]
    float *vss = kss + frames;                                        // [frames]
    float *scores = vss + frames;                                     // [kWhWarps][frames]
    {  // stage the kv head: 4-byte words, 16 loads in flight per thread
        const int nk = frames * kwords, nv = frames * vwords, total = nk + nv + 2 * frames;
        for (int base = threadIdx.x; base < total; base += 16 * blockDim.x) {
            int v[16];
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int i = base + k * blockDim.x;
                if (i < nk) {
                    const int j = i / kwords, wd = i - j * kwords;
                    v[k] = reinterpret_cast<const int *>(keys + (size_t)j * kv * qk + kh * qk)[wd];
                } else if (i < nk + nv) {
                    const int j = (i - nk) / vwords, wd = i - nk - j * vwords;
                    v[k] = reinterpret_cast<const int *>(values + (size_t)j * kv * vd + kh * vd)[wd];
                } else if (i < nk + nv + frames) {
                    v[k] = __float_as_int(ks[(size_t)(i - nk - nv) * kv + kh]);
                } else if (i < total) {
                    v[k] = __float_as_int(vs[(size_t)(i - nk - nv - frames) * kv + kh]);
                }
            }
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int i = base + k * blockDim.x;
                if (i < total) wh_att[i] = v[k];  // kst, vst, kss, vss are contiguous in this order
            }
        }
    }
    __syncthreads();
    const int item = blockIdx.x * kWhWarps + warp;
    if (item >= frames * group) return;
    float *sc = scores + (size_t)warp * frames;
    const int t = item / group, h = kh * group + (item - (item / group) * group);
    // the query as int32 words (qk % 4 == 0): dp4a gives the same exact int32 dot
    int qw[kWhMaxHead / 4];
    const int *qrow = reinterpret_cast<const int *>(q8 + (size_t)t * heads * qk + h * qk);
#pragma unroll
    for (int i = 0; i < kWhMaxHead / 4; i++) qw[i] = i < kwords ? qrow[i] : 0;
    const float scale = __fmul_rn(qs[(size_t)t * heads + h], inv_sqrt);
    float peak = -INFINITY;
    for (int j = lane; j < frames; j += 32) {
        const int *kr = kst + (size_t)j * kwords;
        int dot = 0;
#pragma unroll
        for (int i = 0; i < kWhMaxHead / 4; i++)
            if (i < kwords) dot = __dp4a(kr[i], qw[i], dot);
        const float s = __fmul_rn(__fmul_rn(__int2float_rn(dot), kss[j]), scale);
        sc[j] = s;
        peak = fmaxf(peak, s);
    }
    peak = wh_warp_max(peak);
    for (int j = lane; j < frames; j += 32) sc[j] = exp_rn(__fsub_rn(sc[j], peak));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0)
        for (int j = 0; j < frames; j++) total = __fadd_rn(total, sc[j]);
    total = __shfl_sync(0xffffffffu, total, 0);
    // p_j = e_j / total, then the PV weight p_j * vs_j
    for (int j = lane; j < frames; j += 32) sc[j] = __fmul_rn(__fdiv_rn(sc[j], total), vss[j]);
    __syncwarp();
    const int8_t *vb = reinterpret_cast<const int8_t *>(vst);
    const int d0 = lane, d1 = lane + 32;
    const bool has0 = d0 < vd, has1 = d1 < vd;
    float a0 = 0.0f, a1 = 0.0f;
    int j = 0;
    for (; j + 8 <= frames; j += 8) {
        float w8[8], v0[8], v1[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            w8[u] = sc[j + u];
            v0[u] = has0 ? (float)vb[(size_t)(j + u) * vd + d0] : 0.0f;
            v1[u] = has1 ? (float)vb[(size_t)(j + u) * vd + d1] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            a0 = __fadd_rn(a0, __fmul_rn(w8[u], v0[u]));
            a1 = __fadd_rn(a1, __fmul_rn(w8[u], v1[u]));
        }
    }
    for (; j < frames; j++) {
        a0 = __fadd_rn(a0, __fmul_rn(sc[j], has0 ? (float)vb[(size_t)j * vd + d0] : 0.0f));
        a1 = __fadd_rn(a1, __fmul_rn(sc[j], has1 ? (float)vb[(size_t)j * vd + d1] : 0.0f));
    }
    float *o = out + (size_t)t * heads * vd + h * vd;
    if (has0) o[d0] = a0;
    if (has1) o[d1] = a1;
    for (int d = lane + 64; d < vd; d += 32) {  // v dims past 64 (not taken by the encoder's checks)
        float acc = 0.0f;
        for (int jj = 0; jj < frames; jj++) acc = __fadd_rn(acc, __fmul_rn(sc[jj], (float)vb[(size_t)jj * vd + d]));
        o[d] = acc;
    }
}

// ExecuteConvGlu (Whistle.cs:708-718): hidden = value * sigmoid(gate), value
// and gate the two halves of each Pw1 row (Scalar.Glu).
__global__ void wh_glu_kernel(const float *__restrict__ glu, long long frames, int dim, float *__restrict__ hidden) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= frames * dim) return;
    const long long t = i / dim;
    const int c = (int)(i - t * dim);
    const float *row = glu + t * 2 * dim;
    hidden[i] = __fmul_rn(row[c], sigmoid_rn(row[dim + c]));
}

// ExecuteConvDepthwisePrepare's conv (Whistle.cs:720-744): o[t][c] = sum over
// k of taps[k][c] * hidden[t + k - kernel/2][c] in k order (frames outside
// [0, frames) skipped).
__global__ void wh_time_conv_kernel(const float *__restrict__ hidden, int frames, int dim,
                                    const float *__restrict__ taps, int kernel, float *__restrict__ out) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)frames * dim) return;
    const int t = (int)(i / dim), c = (int)(i - (long long)t * dim), pad = kernel / 2;
    float o = 0.0f;
    for (int k = 0; k < kernel; k++) {
        const int src = t + k - pad;
        if (src < 0 || src >= frames) continue;
        o = __fadd_rn(o, __fmul_rn(taps[(size_t)k * dim + c], hidden[(size_t)src * dim + c]));
    }
    out[i] = o;
}

// ExecuteConvAdd (Whistle.cs:746-753): residual += 1 * proj.
__global__ void wh_add_kernel(float *__restrict__ residual, const float *__restrict__ proj, long long n) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) residual[i] = __fadd_rn(residual[i], proj[i]);
}

__global__ void wh_fill_kernel(float *__restrict__ x, long long n, float value) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = value;
}

// ExecuteCrossPrepare's sum (Whistle.cs:755-771): rows = encoder output, the
// first half plus mix * sin, the second plus mix * cos (AddScaled).
__global__ void wh_cross_rows_kernel(const float *__restrict__ enc, int frames, int dim, float mix,
                                     const float *__restrict__ sin_t, const float *__restrict__ cos_t,
                                     float *__restrict__ rows) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)frames * dim) return;
    const int t = (int)(i / dim), c = (int)(i - (long long)t * dim), half = dim / 2;
    const float pos = c < half ? sin_t[(size_t)t * half + c] : cos_t[(size_t)t * half + c - half];
    rows[i] = __fadd_rn(enc[i], __fmul_rn(mix, pos));
}

// ExecuteCrossQuantize (Whistle.cs:773-792), warp per (frame, head):
// ZeroCenteredRms of the key with k_norm, then QuantizeInt8 of key and value
// into the layer's memory.
__global__ void __launch_bounds__(32 * kWhWarps) wh_cross_quant_kernel(
    const float *__restrict__ kraw, const float *__restrict__ vraw, int frames, int heads, int qk, int vd,
    const float *__restrict__ k_norm, int8_t *__restrict__ keys, float *__restrict__ kscale,
    int8_t *__restrict__ values, float *__restrict__ vscale) {
    pdl_enter();
    __shared__ float buf[kWhWarps][kWhMaxHead];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * kWhWarps + warp;
    if (item >= frames * heads) return;
    float *b = buf[warp];
    const float *kx = kraw + (size_t)item * qk;
    for (int i = lane; i < qk; i += 32) b[i] = kx[i];
    wh_head_norm(b, k_norm, qk, lane);
    const float ks = wh_quantize(b, qk, keys + (size_t)item * qk, lane);
    if (lane == 0) kscale[item] = ks;
    __syncwarp();
    const float *vx = vraw + (size_t)item * vd;
    for (int i = lane; i < vd; i += 32) b[i] = vx[i];
    __syncwarp();
    const float s = wh_quantize(b, vd, values + (size_t)item * vd, lane);
    if (lane == 0) vscale[item] = s;
}

unsigned wh_blocks(long long threads, int per_block) { return (unsigned)((threads + per_block - 1) / per_block); }

// wh_attention_kernel's shared memory: keys and values of every frame, their
// scales, and kWhWarps score rows.
size_t wh_attention_smem(int frames, int qk, int vd) {
    return (size_t)frames * (qk + vd) + (size_t)frames * 4 * (2 + kWhWarps);
}

}  // namespace
}  // namespace ndl

using namespace ndl;

namespace {

struct WhCq {
    const uint8_t *indices = nullptr;
    const uint16_t *norms = nullptr;
    const ndl_kt_codebook *book = nullptr;
    int rows = 0, cols = 0, bits = 0;
};

struct WhLayer {
    const float *pre_mlp_norm0, *attn_norm, *post_attn_norm, *conv_norm, *conv_out_norm, *pre_mlp_norm;
    WhCq q, k, v, gate, out, pw1, pw2;
    const float *q_norm, *k_norm, *depthwise;
    float attn_gate;  // the stored logit's sigmoid
    const float *mlp0[13], *mlp[13];
};

struct WhCross {
    WhCq k, v;
    const float *k_norm;
};

}  // namespace

struct ndl_whistle {
    const ndl_model *model = nullptr;
    ndl_model_info info{};
    cudaStream_t stream = nullptr;
    // AudioWeights' manifest (src/Needle/Audio.cs:119-130)
    int encoder_layers = 0, conv_kernel = 0, stem_width = 0, mels = 0, rate = 0, fft = 0, window = 0, hop = 0;
    int max_samples = 0, max_l0 = 0, max_l1 = 0, max_l2 = 0, max_frames = 0;
    int frames = 0, l0 = 0;
    // views of the loaded weights
    std::vector<WhCross> cross;
    std::vector<WhLayer> layer;
    float position_mix = 0.0f;
    const float *a_pre, *a_post, *a_res, *b_pre, *b_post, *b_res, *final_norm, *stem_first, *stem_dw1, *stem_dw2, *bank;
    WhCq phi_pre, phi_post, phi_res, stem_pw1, stem_pw2, stem_out_w;
    const int32_t *perm_a = nullptr, *perm_b = nullptr;
    // device tables and buffers
    std::vector<void *> allocations;
    float *hann, *cosines, *sines, *rope_cos, *rope_sin, *pos_sin, *pos_cos;
    int32_t *bitrev, *mel_first, *mel_count, *mel_lo, *mel_hi;
    double *col_mean, *col_den;
    unsigned *peak;
    int *status;  // kStatusTimeout when a bounded wait ran out
    float *padded, *mel, *stage0, *dw, *pw, *flat, *stem_out, *stream_a, *stream_b, *u, *residual, *pre, *post, *res,
        *post_gate, *mix, *quarters, *q, *k, *v, *gate, *qs, *ks, *vs, *attn_out, *proj, *glu,
        *hidden, *conv, *gate_rows, *enc_out, *cross_rows, *cross_k, *cross_v;
    int8_t *q8, *keys, *values;
    int8_t *act_values;
    float *act_scales, *act_offsets;
    int act_stride = 0;
    int8_t *mem_keys, *mem_values;
    float *mem_kscale, *mem_vscale;
};

namespace {

int whistle_alloc(ndl_whistle *w, void **p, size_t bytes) {
    if (cudaMalloc(p, bytes < 16 ? 16 : bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "whistle: %zu bytes of device memory", bytes);
    }
    w->allocations.push_back(*p);
    return NDL_OK;
}

template <typename T>
int whistle_buf(ndl_whistle *w, T **p, size_t count) {
    return whistle_alloc(w, reinterpret_cast<void **>(p), count * sizeof(T));
}

// The reading walk of AudioWeights (src/Needle/Audio.cs:117-149) over the
// loader's "audio" records, with the shape checks the device kernels need.
struct AudioWalk {
    const ndl_model *m;
    int k = 1;  // record 0 is the manifest
    int dense(const float **dst, int64_t need) {
        ndl_model_tensor t;
        if (ndl_model_get_tensor(m, "audio", k, &t) != NDL_OK || t.kind != NDL_TENSOR_DENSE || t.count < need)
            return set_error(NDL_ERR_UNSUPPORTED, "audio record %d: a dense tensor of %lld values expected", k,
                             (long long)need);
        *dst = t.values;
        k++;
        return NDL_OK;
    }
    int scalar(float *dst) {
        float v = 0.0f;
        if (ndl_model_read_host(m, "audio", k, &v, sizeof(v)) != NDL_OK)
            return set_error(NDL_ERR_UNSUPPORTED, "audio record %d: a scalar expected", k);
        *dst = v;
        k++;
        return NDL_OK;
    }
    int cq(WhCq *dst, int rows, int cols, int bits) {
        ndl_model_tensor t;
        if (ndl_model_get_tensor(m, "audio", k, &t) != NDL_OK || t.kind != NDL_TENSOR_CQ || t.rows != rows ||
            t.cols != cols || t.bits != bits)
            return set_error(NDL_ERR_UNSUPPORTED, "audio record %d: a %d-bit %d x %d CQ matrix expected (%d x %d, %d)",
                             k, bits, rows, cols, t.rows, t.cols, t.bits);
        dst->indices = t.indices;
        dst->norms = t.norms;
        dst->book = t.book;
        dst->rows = t.rows;
        dst->cols = t.cols;
        dst->bits = t.bits;
        k++;
        return NDL_OK;
    }
};

#define WH_TRY(x)                         \
    do {                                  \
        int st_ = (x);                    \
        if (st_ != NDL_OK) return st_;    \
    } while (0)

int whistle_views(ndl_whistle *w) {
    const ndl_model_info &g = w->info;
    const int d = g.dim, H = g.heads, KV = g.kv_heads, QK = g.qk_dim, VD = g.v_dim, E = w->encoder_layers;
    const int s = w->stem_width;
    AudioWalk a{w->model};
    const int64_t mlp_sizes[13] = {d,
                                   g.hada_n,
                                   g.hada_n,
                                   g.hada_n,
                                   d,
                                   (int64_t)((d + g.hada_cols - 1) / g.hada_cols) * g.hada_rows,
                                   (int64_t)g.hada_cols * g.hada_cols,
                                   (int64_t)g.hada_rows * g.hada_rows,
                                   (int64_t)g.hada_cols * g.hada_cols,
                                   (int64_t)g.hada_rows * g.hada_rows,
                                   (int64_t)g.hada_cols * g.hada_cols,
                                   (int64_t)d * 8,
                                   (int64_t)8 * g.hada_n};
    w->cross.resize(g.layers);
    for (int l = 0; l < g.layers; l++) {  // CrossWeights (Audio.cs:63-75)
        WhCross &c = w->cross[l];
        const float *unused;
        WhCq skip;
        WH_TRY(a.dense(&unused, d));
        WH_TRY(a.cq(&skip, H * QK, d, 2));
        WH_TRY(a.cq(&c.k, H * QK, d, 2));
        WH_TRY(a.cq(&c.v, H * VD, d, 2));
        WH_TRY(a.cq(&skip, H * VD, d, 2));
        WH_TRY(a.cq(&skip, d, H * VD, 2));
        WH_TRY(a.dense(&unused, QK));
        WH_TRY(a.dense(&c.k_norm, QK));
        WH_TRY(a.dense(&unused, d));
        float mix_logit;
        WH_TRY(a.scalar(&mix_logit));
    }
    float pm;
    WH_TRY(a.scalar(&pm));
    w->position_mix = host_sigmoid_rn(pm);
    w->layer.resize(E);
    for (int l = 0; l < E; l++) {  // EncoderLayer (Audio.cs:85-104)
        WhLayer &L = w->layer[l];
        WH_TRY(a.dense(&L.pre_mlp_norm0, d));
        WH_TRY(a.dense(&L.attn_norm, d));
        WH_TRY(a.dense(&L.post_attn_norm, d));
        WH_TRY(a.dense(&L.conv_norm, d));
        WH_TRY(a.dense(&L.conv_out_norm, d));
        WH_TRY(a.dense(&L.pre_mlp_norm, d));
        WH_TRY(a.cq(&L.q, H * QK, d, 2));
        WH_TRY(a.cq(&L.k, KV * QK, d, 2));
        WH_TRY(a.cq(&L.v, KV * VD, d, 2));
        WH_TRY(a.cq(&L.gate, H * VD, d, 2));
        WH_TRY(a.cq(&L.out, d, H * VD, 2));
        WH_TRY(a.dense(&L.q_norm, QK));
        WH_TRY(a.dense(&L.k_norm, QK));
        float gate_logit;
        WH_TRY(a.scalar(&gate_logit));
        L.attn_gate = host_sigmoid_rn(gate_logit);
        WH_TRY(a.cq(&L.pw1, 2 * d, d, 2));
        WH_TRY(a.cq(&L.pw2, d, d, 2));
        WH_TRY(a.dense(&L.depthwise, (int64_t)w->conv_kernel * d));
        for (int i = 0; i < 13; i++) WH_TRY(a.dense(&L.mlp0[i], mlp_sizes[i]));
        for (int i = 0; i < 13; i++) WH_TRY(a.dense(&L.mlp[i], mlp_sizes[i]));
    }
    // HyperConnections(ref r, 0) (Model.cs:160-173): no permutations
    WH_TRY(a.dense(&w->a_pre, E));
    WH_TRY(a.dense(&w->a_post, E));
    WH_TRY(a.dense(&w->a_res, E));
    WH_TRY(a.dense(&w->b_pre, 4 * E));
    WH_TRY(a.dense(&w->b_post, 4 * E));
    WH_TRY(a.dense(&w->b_res, 16 * E));
    WH_TRY(a.cq(&w->phi_pre, 4 * E, 4 * d, 4));
    WH_TRY(a.cq(&w->phi_post, 4 * E, 4 * d, 4));
    WH_TRY(a.cq(&w->phi_res, 16 * E, 4 * d, 4));
    WH_TRY(a.dense(&w->final_norm, d));
    WH_TRY(a.dense(&w->stem_first, 9 * s));
    WH_TRY(a.dense(&w->stem_dw1, 9 * s));
    WH_TRY(a.cq(&w->stem_pw1, s, s, 2));
    WH_TRY(a.dense(&w->stem_dw2, 9 * s));
    WH_TRY(a.cq(&w->stem_pw2, s, s, 2));
    WH_TRY(a.cq(&w->stem_out_w, d, 10 * s, 2));
    WH_TRY(a.dense(&w->bank, (int64_t)(w->fft / 2 + 1) * w->mels));
    ndl_model_tensor t;
    if (ndl_model_get_tensor(w->model, "hyper.perm_a", 0, &t) != NDL_OK) return NDL_ERR_UNSUPPORTED;
    w->perm_a = t.permutation;
    if (ndl_model_get_tensor(w->model, "hyper.perm_b", 0, &t) != NDL_OK) return NDL_ERR_UNSUPPORTED;
    w->perm_b = t.permutation;
    return NDL_OK;
}

}  // namespace

namespace {

void whistle_free(ndl_whistle *w) {
    for (void *p : w->allocations) cudaFree(p);
    if (w->stream) cudaStreamDestroy(w->stream);
    delete w;
}

// Frontend.Create's tables (Frontend.cs:15-46), the encoder's RoPE tables
// (Whistle.cs:134-139: p / MathF.Pow(theta, 2i / qk), MathF.Cos / Sin) and
// the cross-memory position tables (Whistle.cs:142-152, in double), on the
// host with the C library's functions.
int whistle_tables(ndl_whistle *w) {
    const int fft = w->fft, window = w->window, mels = w->mels, F = w->max_frames, QK = w->info.qk_dim;
    const int half = w->info.dim / 2;
    std::vector<float> hann(window), cs(fft / 2), sn(fft / 2), bank((size_t)(fft / 2 + 1) * mels);
    std::vector<int32_t> bitrev(fft), first(fft / 2 + 1), count(fft / 2 + 1);
    const double pi = 3.14159265358979323846;  // Math.PI
    for (int n = 0; n < window; n++) hann[n] = (float)(0.5 - 0.5 * cos(2 * pi * n / (window - 1)));
    for (int k = 0; k < fft / 2; k++) {
        cs[k] = (float)cos(2 * pi * k / fft);
        sn[k] = (float)-sin(2 * pi * k / fft);
    }
    int bits = 0;
    while ((1 << (bits + 1)) <= fft) bits++;
    for (int i = 0; i < fft; i++) {
        int r = 0;
        for (int b = 0; b < bits; b++) r |= (i >> b & 1) << (bits - 1 - b);
        bitrev[i] = r;
    }
    NDL_CUDA(cudaMemcpy(bank.data(), w->bank, bank.size() * 4, cudaMemcpyDeviceToHost));
    for (int k = 0; k <= fft / 2; k++) {
        int f = mels, last = -1;
        for (int m = 0; m < mels; m++)
            if (bank[(size_t)k * mels + m] != 0.0f) {
                if (f == mels) f = m;
                last = m;
            }
        first[k] = f;
        count[k] = last >= f ? last - f + 1 : 0;
    }
    std::vector<int32_t> lo(mels, 0), hi(mels, 0);  // per mel, the bins [lo, hi) whose ranges can hold it
    for (int m = 0; m < mels; m++) {
        int a = -1, b = -1;
        for (int k = 0; k <= fft / 2; k++)
            if (m >= first[k] && m < first[k] + count[k]) {
                if (a < 0) a = k;
                b = k;
            }
        lo[m] = a < 0 ? 0 : a;
        hi[m] = a < 0 ? 0 : b + 1;
    }
    std::vector<float> rc((size_t)F * (QK / 2)), rs((size_t)F * (QK / 2)), ps((size_t)F * half), pc((size_t)F * half);
    for (int p = 0; p < F; p++)
        for (int i = 0; i < QK / 2; i++) {
            const float angle = (float)p / powf(w->info.rope_theta, 2.0f * (float)i / (float)QK);
            rc[(size_t)p * (QK / 2) + i] = cosf(angle);
            rs[(size_t)p * (QK / 2) + i] = sinf(angle);
        }
    const double step = -log(10000.0) / (half - 1);
    for (int i = 0; i < half; i++) {
        const double inv_freq = exp(step * i);
        for (int p = 0; p < F; p++) {
            const double angle = p * inv_freq;
            ps[(size_t)p * half + i] = (float)sin(angle);
            pc[(size_t)p * half + i] = (float)cos(angle);
        }
    }
    WH_TRY(whistle_buf(w, &w->hann, hann.size()));
    WH_TRY(whistle_buf(w, &w->cosines, cs.size()));
    WH_TRY(whistle_buf(w, &w->sines, sn.size()));
    WH_TRY(whistle_buf(w, &w->bitrev, bitrev.size()));
    WH_TRY(whistle_buf(w, &w->mel_first, first.size()));
    WH_TRY(whistle_buf(w, &w->mel_count, count.size()));
    WH_TRY(whistle_buf(w, &w->mel_lo, lo.size()));
    WH_TRY(whistle_buf(w, &w->mel_hi, hi.size()));
    WH_TRY(whistle_buf(w, &w->col_mean, (size_t)mels));
    WH_TRY(whistle_buf(w, &w->col_den, (size_t)mels));
    WH_TRY(whistle_buf(w, &w->rope_cos, rc.size()));
    WH_TRY(whistle_buf(w, &w->rope_sin, rs.size()));
    WH_TRY(whistle_buf(w, &w->pos_sin, ps.size()));
    WH_TRY(whistle_buf(w, &w->pos_cos, pc.size()));
    NDL_CUDA(cudaMemcpy(w->hann, hann.data(), hann.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->cosines, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->sines, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->bitrev, bitrev.data(), bitrev.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->mel_first, first.data(), first.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->mel_count, count.data(), count.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->mel_lo, lo.data(), lo.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->mel_hi, hi.data(), hi.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->rope_cos, rc.data(), rc.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->rope_sin, rs.data(), rs.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->pos_sin, ps.data(), ps.size() * 4, cudaMemcpyHostToDevice));
    NDL_CUDA(cudaMemcpy(w->pos_cos, pc.data(), pc.size() * 4, cudaMemcpyHostToDevice));
    return NDL_OK;
}

int whistle_buffers(ndl_whistle *w) {
    const ndl_model_info &g = w->info;
    const size_t d = g.dim, F = w->max_frames, s = w->stem_width, L = g.layers;
    const size_t H = g.heads, KV = g.kv_heads, QK = g.qk_dim, VD = g.v_dim;
    const size_t stem_tokens = std::max((size_t)w->max_l2 * 20, (size_t)F * 10);
    const size_t cols = std::max(std::max(s, 10 * s), std::max(4 * d, H * VD));
    const size_t tokens = std::max(stem_tokens, F);
    w->act_stride = (int)((cols / 128 + 7) & ~(size_t)7);
    // the stem kernels index their stages in 32 bits; the first stage is the largest
    if ((size_t)w->max_l1 * 40 * s >= ((size_t)1 << 31))
        return set_error(NDL_ERR_UNSUPPORTED, "whistle: %d samples at stem width %zu exceed the stem's 2^31 elements",
                         w->max_samples, s);
    WH_TRY(whistle_buf(w, &w->peak, 1));
    WH_TRY(whistle_buf(w, &w->status, 1));
    WH_TRY(whistle_buf(w, &w->padded, (size_t)w->window + w->max_samples + w->hop + w->fft));
    WH_TRY(whistle_buf(w, &w->mel, (size_t)w->max_l0 * w->mels + 4));  // + 4: the bulk copies round up to 16 bytes
    WH_TRY(whistle_buf(w, &w->stage0, (size_t)w->max_l1 * 40 * s));
    WH_TRY(whistle_buf(w, &w->dw, stem_tokens * s));
    WH_TRY(whistle_buf(w, &w->pw, stem_tokens * s));
    WH_TRY(whistle_buf(w, &w->flat, F * 10 * s));
    WH_TRY(whistle_buf(w, &w->act_values, tokens * cols));
    WH_TRY(whistle_buf(w, &w->act_scales, tokens * w->act_stride));
    WH_TRY(whistle_buf(w, &w->act_offsets, tokens * w->act_stride));
    float **fd[] = {&w->stem_out, &w->u, &w->residual, &w->proj, &w->hidden, &w->conv, &w->enc_out, &w->cross_rows};
    for (float **p : fd) WH_TRY(whistle_buf(w, p, F * d));
    WH_TRY(whistle_buf(w, &w->stream_a, F * 4 * d));
    WH_TRY(whistle_buf(w, &w->stream_b, F * 4 * d));
    WH_TRY(whistle_buf(w, &w->glu, F * 2 * d));
    float **f4[] = {&w->post_gate, &w->quarters};
    for (float **p : f4) WH_TRY(whistle_buf(w, p, F * 4));
    const size_t E = w->encoder_layers;
    WH_TRY(whistle_buf(w, &w->pre, F * 4 * E));
    WH_TRY(whistle_buf(w, &w->post, F * 4 * E));
    WH_TRY(whistle_buf(w, &w->res, F * 16 * E));
    WH_TRY(whistle_buf(w, &w->mix, F * 16));
    WH_TRY(whistle_buf(w, &w->gate_rows, F));
    WH_TRY(whistle_buf(w, &w->q, F * H * QK));
    WH_TRY(whistle_buf(w, &w->k, F * KV * QK));
    WH_TRY(whistle_buf(w, &w->v, F * KV * VD));
    WH_TRY(whistle_buf(w, &w->gate, F * H * VD));
    WH_TRY(whistle_buf(w, &w->attn_out, F * H * VD));
    WH_TRY(whistle_buf(w, &w->q8, F * H * QK));
    WH_TRY(whistle_buf(w, &w->qs, F * H));
    WH_TRY(whistle_buf(w, &w->keys, F * KV * QK));
    WH_TRY(whistle_buf(w, &w->ks, F * KV));
    WH_TRY(whistle_buf(w, &w->values, F * KV * VD));
    WH_TRY(whistle_buf(w, &w->vs, F * KV));
    WH_TRY(whistle_buf(w, &w->cross_k, F * H * QK));
    WH_TRY(whistle_buf(w, &w->cross_v, F * H * VD));
    WH_TRY(whistle_buf(w, &w->mem_keys, L * F * H * QK));
    WH_TRY(whistle_buf(w, &w->mem_values, L * F * H * VD));
    WH_TRY(whistle_buf(w, &w->mem_kscale, L * F * H));
    WH_TRY(whistle_buf(w, &w->mem_vscale, L * F * H));
    return NDL_OK;
}

CqMatmulJob wh_job(const WhCq &c, float *y, int ldy, int row_start, int row_end) {
    return CqMatmulJob{c.indices, c.norms, c.book->bytes, c.book->byte_scale, y, ldy, row_start, row_end};
}

int wh_matmul(ndl_whistle *w, const WhCq &c, int tokens, float *y) {
    const CqMatmulJob job = wh_job(c, y, c.rows, 0, c.rows);
    return launch_cq_matmul_jobs(&job, 1, c.cols, c.bits, w->act_values, w->act_scales, w->act_offsets, w->act_stride,
                                 tokens, w->stream);
}

int wh_prepare(ndl_whistle *w, const float *x, int tokens, int cols) {
    return launch_cq_prepare(x, tokens, cols, 2, w->act_values, w->act_scales, w->act_offsets, w->act_stride,
                             w->stream);
}

// A row op of the RMS family followed by a Prepare at `bits`.
int wh_row_prepare(ndl_whistle *w, int mode, bool fake, const float *x, const float *aux, int rows, int n, int bits) {
    const CqPrepOut prep{w->act_values, w->act_scales, w->act_offsets, w->act_stride, bits};
    return launch_row_op(mode, fake, x, aux, nullptr, rows, n, nullptr, &prep, w->stream);
}

}  // namespace

namespace {

#define WH_LAUNCH(name)                            \
    do {                                           \
        const int st_ = check_launch(name);        \
        if (st_ != NDL_OK) return st_;             \
    } while (0)

// Encode (Whistle.cs:179-200) and BuildCrossMemory (:886-914) of the PCM in
// w->padded (samples at offset window / 2, zeros around), on w->stream.
int whistle_run(ndl_whistle *w, int samples) {
    const ndl_model_info &g = w->info;
    cudaStream_t st = w->stream;
    const int hop = w->hop, fft = w->fft, window = w->window, mels = w->mels;
    const int l0 = samples / hop;
    w->l0 = l0 > 0 ? l0 : 0;
    w->frames = 0;
    if (l0 < 1) return NDL_OK;
    const int l1 = (l0 + 1) / 2, l2 = (l1 + 1) / 2, F = (l2 + 1) / 2;
    const int d = g.dim, s = w->stem_width, H = g.heads, KV = g.kv_heads, QK = g.qk_dim, VD = g.v_dim;
    const int E = w->encoder_layers;
    // front end
    NDL_CUDA(cudaMemsetAsync(w->peak, 0, sizeof(unsigned), st));
    NDL_CUDA(cudaMemsetAsync(w->status, 0, sizeof(int), st));
    launch_kernel(wh_mel_kernel, dim3((unsigned)l0), dim3(256), (size_t)(2 * fft + fft / 2 + 1) * 4, st, w->padded,
                  hop, fft, window, w->hann, w->cosines, w->sines, w->bitrev, w->bank, mels, w->mel_first,
                  w->mel_count, w->mel_lo, w->mel_hi, w->mel, w->peak);
    WH_LAUNCH("wh_mel");
    const long long nmel = (long long)l0 * mels;
    launch_kernel(wh_log_kernel, dim3(wh_blocks(nmel, 256)), dim3(256), 0, st, w->mel, nmel, (const unsigned *)w->peak);
    WH_LAUNCH("wh_log");
    {
        const size_t smem = (size_t)2 * kMomRows * mels * 4;
        static DeviceOnce smem_attribute;
        WH_TRY(smem_attribute.run([] {
            const cudaError_t e = cudaFuncSetAttribute(wh_moments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       2 * kMomRows * 128 * 4);
            return e == cudaSuccess ? (int)NDL_OK : set_error(NDL_ERR_CUDA, "wh_moments smem: %s", cudaGetErrorString(e));
        }));
        launch_kernel(wh_moments_kernel, dim3(1), dim3(128), smem, st, (const float *)w->mel, l0, mels, w->col_mean,
                      w->col_den, w->status);
    }
    WH_LAUNCH("wh_moments");
    launch_kernel(wh_standardize_kernel, dim3(wh_blocks(nmel, 256)), dim3(256), 0, st, w->mel, nmel, mels,
                  (const double *)w->col_mean, (const double *)w->col_den);
    WH_LAUNCH("wh_standardize");
    // stem
    const long long n0 = (long long)l1 * 40 * s;
    launch_kernel(wh_stem1_kernel, dim3(wh_blocks(n0, 256)), dim3(256), 0, st, (const float *)w->mel, l0, mels,
                  w->stem_first, s, l1, w->stage0);
    WH_LAUNCH("wh_stem1");
    const long long n1 = (long long)l2 * 20 * s;
    launch_kernel(wh_depthwise_kernel, dim3(wh_blocks(n1, 256)), dim3(256), 0, st, (const float *)w->stage0, l1, 40,
                  w->stem_dw1, s, l2, 20, w->dw);
    WH_LAUNCH("wh_depthwise1");
    WH_TRY(wh_prepare(w, w->dw, l2 * 20, s));
    WH_TRY(wh_matmul(w, w->stem_pw1, l2 * 20, w->pw));
    launch_kernel(wh_silu_kernel, dim3(wh_blocks(n1, 256)), dim3(256), 0, st, w->pw, n1);
    WH_LAUNCH("wh_silu");
    const long long n2 = (long long)F * 10 * s;
    launch_kernel(wh_depthwise_kernel, dim3(wh_blocks(n2, 256)), dim3(256), 0, st, (const float *)w->pw, l2, 20,
                  w->stem_dw2, s, F, 10, w->dw);
    WH_LAUNCH("wh_depthwise2");
    WH_TRY(wh_prepare(w, w->dw, F * 10, s));
    WH_TRY(wh_matmul(w, w->stem_pw2, F * 10, w->pw));
    launch_kernel(wh_silu_transpose_kernel, dim3(wh_blocks(n2, 256)), dim3(256), 0, st, (const float *)w->pw, F, s,
                  w->flat);
    WH_LAUNCH("wh_silu_transpose");
    WH_TRY(wh_prepare(w, w->flat, F, 10 * s));
    WH_TRY(wh_matmul(w, w->stem_out_w, F, w->stem_out));
    // encoder
    const long long nd = (long long)F * d;
    launch_kernel(wh_lanes_kernel, dim3(wh_blocks(nd * 4, 256)), dim3(256), 0, st, (const float *)w->stem_out,
                  (long long)F, d, w->stream_a);
    WH_LAUNCH("wh_lanes");
    launch_kernel(wh_fill_kernel, dim3(wh_blocks((long long)F * 4, 256)), dim3(256), 0, st, w->quarters,
                  (long long)F * 4, 0.25f);
    WH_LAUNCH("wh_fill");
    float *stream = w->stream_a, *next = w->stream_b;
    const float inv_sqrt = 1.0f / sqrtf((float)QK);
    for (int l = 0; l < E; l++) {
        const WhLayer &L = w->layer[l];
        // ExecuteRmsAndPrepareStream, the phi slices, ExecutePreHyper
        WH_TRY(wh_row_prepare(w, 0, false, stream, nullptr, F, 4 * d, 4));
        const CqMatmulJob phi[3] = {wh_job(w->phi_pre, w->pre, 4 * E, 4 * l, 4 * l + 4),
                                    wh_job(w->phi_post, w->post, 4 * E, 4 * l, 4 * l + 4),
                                    wh_job(w->phi_res, w->res, 16 * E, 16 * l, 16 * l + 16)};
        WH_TRY(launch_cq_matmul_jobs(phi, 3, 4 * d, 4, w->act_values, w->act_scales, w->act_offsets, w->act_stride, F,
                                     st));
        WH_TRY(launch_hc_prepare(w->pre, 4 * E, w->post, 4 * E, w->res, 16 * E, w->a_pre, w->b_pre, w->a_post,
                                 w->b_post, w->a_res, w->b_res, l, stream, d, F, w->u, w->residual, w->post_gate,
                                 w->mix, st));
        WH_TRY(launch_hadamard_mlp_rows(L.mlp0, L.pre_mlp_norm0, w->perm_a, w->perm_b, d, g.hada_rows, g.hada_cols,
                                        0.5f, w->residual, F, st));
        // RunSelfAttention (:840-862)
        WH_TRY(wh_row_prepare(w, 1, false, w->residual, L.attn_norm, F, d, 2));
        const CqMatmulJob proj[4] = {wh_job(L.q, w->q, H * QK, 0, H * QK), wh_job(L.k, w->k, KV * QK, 0, KV * QK),
                                     wh_job(L.v, w->v, KV * VD, 0, KV * VD), wh_job(L.gate, w->gate, H * VD, 0, H * VD)};
        WH_TRY(launch_cq_matmul_jobs(proj, 4, d, 2, w->act_values, w->act_scales, w->act_offsets, w->act_stride, F,
                                     st));
        launch_kernel(wh_qkv_kernel, dim3(wh_blocks((long long)F * (H + KV), kWhWarps)), dim3(32 * kWhWarps), 0, st,
                      (const float *)w->q, (const float *)w->k, (const float *)w->v, F, H, KV, QK, VD, L.q_norm,
                      L.k_norm, (const float *)w->rope_cos, (const float *)w->rope_sin, w->q8, w->qs, w->keys, w->ks,
                      w->values, w->vs);
        WH_LAUNCH("wh_qkv");
        static DeviceOnce attention_smem;
        WH_TRY(attention_smem.run([] {
            int dev = 0, optin = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
            const cudaError_t e =
                cudaFuncSetAttribute(wh_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
            return e == cudaSuccess ? (int)NDL_OK
                                    : set_error(NDL_ERR_CUDA, "wh_attention smem: %s", cudaGetErrorString(e));
        }));
        launch_kernel(wh_attention_kernel, dim3(wh_blocks((long long)F * (H / KV), kWhWarps), (unsigned)KV),
                      dim3(32 * kWhWarps), wh_attention_smem(F, QK, VD), st, (const int8_t *)w->q8,
                      (const float *)w->qs, F, H, KV, QK, VD, inv_sqrt, (const int8_t *)w->keys, (const float *)w->ks,
                      (const int8_t *)w->values, (const float *)w->vs, w->attn_out);
        WH_LAUNCH("wh_attention");
        WH_TRY(wh_row_prepare(w, 2, false, w->attn_out, w->gate, F, H * VD, 2));
        WH_TRY(wh_matmul(w, L.out, F, w->proj));
        launch_kernel(wh_fill_kernel, dim3(wh_blocks(F, 256)), dim3(256), 0, st, w->gate_rows, (long long)F,
                      L.attn_gate);
        WH_LAUNCH("wh_fill");
        WH_TRY(launch_row_op(3, false, w->proj, L.post_attn_norm, w->gate_rows, F, d, w->residual, nullptr, st));
        // RunConvolution (:864-876)
        WH_TRY(wh_row_prepare(w, 1, false, w->residual, L.conv_norm, F, d, 2));
        WH_TRY(wh_matmul(w, L.pw1, F, w->glu));
        launch_kernel(wh_glu_kernel, dim3(wh_blocks(nd, 256)), dim3(256), 0, st, (const float *)w->glu, (long long)F,
                      d, w->hidden);
        WH_LAUNCH("wh_glu");
        launch_kernel(wh_time_conv_kernel, dim3(wh_blocks(nd, 256)), dim3(256), 0, st, (const float *)w->hidden, F, d,
                      L.depthwise, w->conv_kernel, w->conv);
        WH_LAUNCH("wh_time_conv");
        WH_TRY(wh_row_prepare(w, 4, false, w->conv, L.conv_out_norm, F, d, 2));
        WH_TRY(wh_matmul(w, L.pw2, F, w->proj));
        launch_kernel(wh_add_kernel, dim3(wh_blocks(nd, 256)), dim3(256), 0, st, w->residual, (const float *)w->proj,
                      nd);
        WH_LAUNCH("wh_add");
        {  // MLP, then CombineDiff4x4 into the next streams, one kernel per frame
            KtMlpArgs a{};
            for (int k = 0; k < 13; k++) a.w[k] = L.mlp[k];
            a.pre_norm = L.pre_mlp_norm;
            a.perm_a = w->perm_a;
            a.perm_b = w->perm_b;
            a.dim = d;
            a.rows = g.hada_rows;
            a.cols = g.hada_cols;
            a.scale = 0.5f;
            a.residual = w->residual;
            a.row_stride = d;
            a.cb_stream = stream;
            a.cb_mix = w->mix;
            a.cb_u = w->u;
            a.cb_post = w->post_gate;
            a.cb_next = next;
            WH_TRY(launch_mlp_rows(a, F, st));
        }
        std::swap(stream, next);
    }
    // ExecuteEncoderFinal (:614-626)
    WH_TRY(ndl_hc_mix4(stream, d, w->quarters, F, w->u, st));
    WH_TRY(launch_row_op(1, false, w->u, w->final_norm, nullptr, F, d, w->enc_out, nullptr, st));
    // BuildCrossMemory
    launch_kernel(wh_cross_rows_kernel, dim3(wh_blocks(nd, 256)), dim3(256), 0, st, (const float *)w->enc_out, F, d,
                  w->position_mix, (const float *)w->pos_sin, (const float *)w->pos_cos, w->cross_rows);
    WH_LAUNCH("wh_cross_rows");
    WH_TRY(wh_row_prepare(w, 5, true, w->cross_rows, nullptr, F, d, 2));
    for (int l = 0; l < g.layers; l++) {
        const WhCross &c = w->cross[l];
        const CqMatmulJob kv[2] = {wh_job(c.k, w->cross_k, H * QK, 0, H * QK), wh_job(c.v, w->cross_v, H * VD, 0, H * VD)};
        WH_TRY(launch_cq_matmul_jobs(kv, 2, d, 2, w->act_values, w->act_scales, w->act_offsets, w->act_stride, F, st));
        const size_t slots = (size_t)l * F * H;
        launch_kernel(wh_cross_quant_kernel, dim3(wh_blocks((long long)F * H, kWhWarps)), dim3(32 * kWhWarps), 0, st,
                      (const float *)w->cross_k, (const float *)w->cross_v, F, H, QK, VD, c.k_norm,
                      w->mem_keys + slots * QK, w->mem_kscale + slots, w->mem_values + slots * VD,
                      w->mem_vscale + slots);
        WH_LAUNCH("wh_cross_quant");
    }
    w->frames = F;
    return NDL_OK;
}

}  // namespace

extern "C" NDL_API int ndl_whistle_create(const ndl_model *m, int max_samples, ndl_whistle **out) {
    NDL_REQUIRE(m && out, "null pointer");
    *out = nullptr;
    ndl_model_info info;
    if (ndl_model_get_info(m, &info) != NDL_OK) return NDL_ERR_INVALID_ARG;
    NDL_REQUIRE(info.has_audio, "the archive has no speech model (no audio section)");
    NDL_REQUIRE(info.device >= 0, "the model is not on a device (load it with a device)");
    NDL_REQUIRE(max_samples >= 1, "max_samples %d", max_samples);
    float manifest[13];
    if (ndl_model_read_host(m, "audio", 0, manifest, sizeof(manifest)) != NDL_OK)
        return set_error(NDL_ERR_UNSUPPORTED, "the audio section's manifest is not a 13-entry vector");
    ndl_whistle *w = new ndl_whistle;
    w->model = m;
    w->info = info;
    const int E = (int)manifest[3], conv = (int)manifest[5], s = (int)manifest[6], stages = (int)manifest[7];
    w->encoder_layers = E;
    w->conv_kernel = conv;
    w->stem_width = s;
    w->mels = (int)manifest[8];
    w->rate = (int)manifest[9];
    w->fft = (int)manifest[10];
    w->window = (int)manifest[11];
    w->hop = (int)manifest[12];
    const int d = info.dim;
    int rc = NDL_OK;
    if (stages != 3) rc = set_error(NDL_ERR_UNSUPPORTED, "three-stage stem expected, the manifest says %d", stages);
    else if (E < 1 || conv < 1 || w->mels < 1 || w->mels > 128 || w->hop < 1 || w->window < 2 || w->fft < 2 || w->fft > kWhMaxFft ||
             (w->fft & (w->fft - 1)) != 0 || w->window > w->fft || w->rate < 1)
        rc = set_error(NDL_ERR_UNSUPPORTED, "audio manifest: %d layers, kernel %d, %d mels, fft %d, window %d, hop %d",
                       E, conv, w->mels, w->fft, w->window, w->hop);
    else if (s < 128 || s % 128 != 0 || 10 * s > 8192 || d % 128 != 0 || 4 * d > 4096 ||
             (info.heads * info.v_dim) % 128 != 0 || info.qk_dim > kWhMaxHead || info.v_dim > kWhMaxHead ||
             info.qk_dim % 4 != 0 || info.kv_heads < 1 || info.heads % info.kv_heads != 0 || info.hada_n <= 0)
        rc = set_error(NDL_ERR_UNSUPPORTED,
                       "Whistle geometry: stem width %d, dim %d, heads %d x %d / %d, kv heads %d (the device encoder "
                       "takes CQ widths in 128-column groups, dim <= 1024, head dims <= %d)",
                       s, d, info.heads, info.qk_dim, info.v_dim, info.kv_heads, kWhMaxHead);
    const int rate_cap = 30 * w->rate;  // Whistle.MaxSeconds
    w->max_samples = max_samples < rate_cap ? max_samples : rate_cap;
    w->max_l0 = w->max_samples / (w->hop > 0 ? w->hop : 1);
    w->max_l1 = (w->max_l0 + 1) / 2;
    w->max_l2 = (w->max_l1 + 1) / 2;
    w->max_frames = (w->max_l2 + 1) / 2;
    if (rc == NDL_OK && w->max_l0 < 1) rc = set_error(NDL_ERR_INVALID_ARG, "max_samples %d is under one hop", max_samples);
    int dev = 0;
    if (rc == NDL_OK && cudaGetDevice(&dev) == cudaSuccess && dev != info.device) cudaSetDevice(info.device);
    if (rc == NDL_OK && cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        rc = set_error(NDL_ERR_CUDA, "whistle: stream creation failed");
    }
    if (rc == NDL_OK) rc = whistle_views(w);
    if (rc == NDL_OK) rc = whistle_tables(w);
    if (rc == NDL_OK) rc = whistle_buffers(w);
    if (rc != NDL_OK) {
        whistle_free(w);
        return rc;
    }
    *out = w;
    return NDL_OK;
}

extern "C" NDL_API int ndl_whistle_encode_device(ndl_whistle *w, const float *pcm, int samples) {
    NDL_REQUIRE(w, "null encoder");
    NDL_REQUIRE(samples >= 0 && samples <= w->max_samples, "samples %d (0..%d)", samples, w->max_samples);
    NDL_REQUIRE(samples == 0 || pcm, "null pcm");
    const int half = w->window / 2;
    const size_t total = (size_t)w->window + w->max_samples + w->hop + w->fft;
    NDL_CUDA(cudaMemsetAsync(w->padded, 0, total * 4, w->stream));
    if (samples > 0)
        NDL_CUDA(cudaMemcpyAsync(w->padded + half, pcm, (size_t)samples * 4, cudaMemcpyDefault, w->stream));
    return whistle_run(w, samples);
}

extern "C" NDL_API int ndl_whistle_encode(ndl_whistle *w, const float *pcm, int samples, int *frames) {
    NDL_REQUIRE(w && frames, "null pointer");
    samples = samples < w->max_samples ? samples : w->max_samples;  // Encode keeps the first MaxSeconds
    const int rc = ndl_whistle_encode_device(w, pcm, samples);
    if (rc != NDL_OK) return rc;
    NDL_CUDA(cudaStreamSynchronize(w->stream));
    int status = 0;
    NDL_CUDA(cudaMemcpy(&status, w->status, sizeof(int), cudaMemcpyDeviceToHost));
    if (status) return set_error(NDL_ERR_TIMEOUT, "whistle encode: a bounded wait ran out (status %d)", status);
    *frames = w->frames;
    return NDL_OK;
}

extern "C" NDL_API int ndl_whistle_read(ndl_whistle *w, int what, int layer, void *dst, size_t bytes,
                                        size_t *written) {
    NDL_REQUIRE(w && dst, "null pointer");
    const ndl_model_info &g = w->info;
    const size_t F = w->frames, H = g.heads, QK = g.qk_dim, VD = g.v_dim;
    const void *src = nullptr;
    size_t size = 0;
    if (what >= NDL_WHISTLE_KEYS)
        NDL_REQUIRE(layer >= 0 && layer < g.layers, "layer %d of %d", layer, g.layers);
    const size_t slots = (size_t)(layer > 0 ? layer : 0) * F * H;
    switch (what) {
        case NDL_WHISTLE_MEL: src = w->mel, size = (size_t)w->l0 * w->mels * 4; break;
        case NDL_WHISTLE_STEM: src = w->stem_out, size = F * g.dim * 4; break;
        case NDL_WHISTLE_ENCODER: src = w->enc_out, size = F * g.dim * 4; break;
        case NDL_WHISTLE_KEYS: src = w->mem_keys + slots * QK, size = F * H * QK; break;
        case NDL_WHISTLE_KEY_SCALES: src = w->mem_kscale + slots, size = F * H * 4; break;
        case NDL_WHISTLE_VALUES: src = w->mem_values + slots * VD, size = F * H * VD; break;
        case NDL_WHISTLE_VALUE_SCALES: src = w->mem_vscale + slots, size = F * H * 4; break;
        default: return set_error(NDL_ERR_INVALID_ARG, "what %d", what);
    }
    NDL_REQUIRE(bytes >= size, "%zu bytes for a %zu-byte result", bytes, size);
    NDL_CUDA(cudaStreamSynchronize(w->stream));
    if (size) NDL_CUDA(cudaMemcpy(dst, src, size, cudaMemcpyDeviceToHost));
    if (written) *written = size;
    return NDL_OK;
}

extern "C" NDL_API int ndl_whistle_frames(const ndl_whistle *w, int *frames, int *mel_frames) {
    NDL_REQUIRE(w, "null encoder");
    if (frames) *frames = w->frames;
    if (mel_frames) *mel_frames = w->l0;
    return NDL_OK;
}

extern "C" NDL_API void *ndl_whistle_stream(ndl_whistle *w) { return w ? (void *)w->stream : nullptr; }

extern "C" NDL_API int ndl_whistle_destroy(ndl_whistle *w) {
    if (!w) return NDL_OK;
    cudaStreamSynchronize(w->stream);
    whistle_free(w);
    return NDL_OK;
}
