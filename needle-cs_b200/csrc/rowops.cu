// Needle-3 row operations around a layer (the reference's hyper-connection
// streams, conv taps and fake-A8 norms), batched over tokens on the device.
//
// Hyper-connections (EngineCore.RunLayerBatch, src/Needle/Engine.cs:2352-2404):
// a token carries 4 streams of `dim` floats.  Before the layer the streams
// mix into the layer input (Mix4, Scalar.cs:255-258) and a 4x4 Sinkhorn
// matrix (Scalar.Sinkhorn4x4, Scalar.cs:361-381) is made from the layer's
// logits; after it, CombineDiff4x4 (Ops.cs:800-812) forms the next streams.
// Conv taps: Scalar.Taps3 (Scalar.cs:285-288) over a (t-2, t-1, t) triple
// (EngineCore.ChainTriple, Engine.cs:2471-2478).  Fake-A8 norms:
// Scalar.RmsFakeA8 / CenteredRmsFakeA8 / GateFakeA8 / PostNormAdd
// (Scalar.cs:381-439).
//
// The arithmetic follows the scalar code term by term (no contraction; sums
// of squares in ascending order on one lane), so every result except those
// through exp equals the scalar restatement bit for bit.
#include "common.cuh"
#include "cq.cuh"
#include "hc.cuh"
#include "kernels.cuh"

namespace ndl {

__device__ __forceinline__ float mix4_term(float acc, float w0, float w1, float w2, float w3, const float *s, int dim,
                                           int c) {
    acc = __fadd_rn(acc, __fmul_rn(w0, s[c]));
    acc = __fadd_rn(acc, __fmul_rn(w1, s[dim + c]));
    acc = __fadd_rn(acc, __fmul_rn(w2, s[2 * dim + c]));
    return __fadd_rn(acc, __fmul_rn(w3, s[3 * dim + c]));
}

// Mix4 per token: dst[t] = sum_i w[t][i] * s[t][i] (s [n][4][dim]).
__global__ void __launch_bounds__(256) mix4_kernel(const float *__restrict__ s, int dim, const float *__restrict__ w,
                                                   int n, float *__restrict__ dst) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * dim) return;
    const int t = (int)(i / dim), c = (int)(i - (long long)t * dim);
    const float *st = s + (size_t)t * 4 * dim, *wt = w + (size_t)t * 4;
    const float first = __fmul_rn(wt[0], st[c]);
    float acc = __fadd_rn(first, __fmul_rn(wt[1], st[dim + c]));
    acc = __fadd_rn(acc, __fmul_rn(wt[2], st[2 * dim + c]));
    dst[(size_t)t * dim + c] = __fadd_rn(acc, __fmul_rn(wt[3], st[3 * dim + c]));
}

// CombineDiff4x4 per token: stream i of dst[t] = post[t][i] * (x - u)
// + sum_j mix[t][4i + j] * s[t][j]; with kDiff false, Combine4 per token
// (x as y, u unused, one output stream).
template <bool kDiff>
__global__ void __launch_bounds__(256) combine4_kernel(const float *__restrict__ s, int dim,
                                                       const float *__restrict__ mix, const float *__restrict__ x,
                                                       const float *__restrict__ u, const float *__restrict__ post,
                                                       int n, float *__restrict__ dst) {
    pdl_enter();
    constexpr int kOut = kDiff ? 4 : 1;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * kOut * dim) return;
    const int t = (int)(i / (kOut * dim));
    const int rest = (int)(i - (long long)t * kOut * dim), o = rest / dim, c = rest - o * dim;
    const float *st = s + (size_t)t * 4 * dim, *m = mix + (size_t)t * (kDiff ? 16 : 4) + 4 * o;
    const float xv = x[(size_t)t * dim + c];
    const float head = kDiff ? __fmul_rn(post[(size_t)t * 4 + o], __fsub_rn(xv, u[(size_t)t * dim + c]))
                             : __fmul_rn(post[t], xv);
    dst[((size_t)t * kOut + o) * dim + c] = mix4_term(head, m[0], m[1], m[2], m[3], st, dim, c);
}

// Sinkhorn4x4 per token on 16 lanes (hc_sinkhorn16); lanes past the last
// token run on zeros and store nothing.
__global__ void __launch_bounds__(128) sinkhorn4x4_kernel(const float *__restrict__ logits, int n,
                                                          float *__restrict__ out) {
    pdl_enter();
    const long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long t = gt >> 4;
    const int lane = threadIdx.x & 31, e = lane & 15;
    const bool ok = t < n;
    const float r = hc_sinkhorn16(ok ? logits[t * 16 + e] : 0.0f, lane);
    if (ok) out[t * 16 + e] = r;
}

// The hyper-connection prepare after the phi matmuls (RunLayerBatch,
// src/Needle/Engine.cs:2366-2382; the encoder's ExecutePreHyper,
// src/Needle/Whistle.cs:578-601), CTA per row: hpre[i] = Sigmoid(a_pre[l]
// pre[i] + b_pre[4l + i] + (i == lane ? 4 : -4)), post_gate[i] = 2
// Sigmoid(a_post[l] post[i] + b_post[4l + i] + (i == lane ? 0 : -4)) on
// threads 0..3; the Sinkhorn logits a_res[l] res[j] + b_res[16l + j] on warp 1;
// then u = Mix4(stream, hpre), also copied to the residual, and
// mix = Sinkhorn4x4(logits) on warp 0.  Each sum left to right, one rounding
// per operation.
__global__ void __launch_bounds__(256) hc_prepare_kernel(
    const float *__restrict__ pre, int ld_pre, const float *__restrict__ post, int ld_post,
    const float *__restrict__ res, int ld_res, const float *__restrict__ a_pre, const float *__restrict__ b_pre,
    const float *__restrict__ a_post, const float *__restrict__ b_post, const float *__restrict__ a_res,
    const float *__restrict__ b_res, int layer, const float *__restrict__ stream, int dim, float *__restrict__ u,
    float *__restrict__ residual, float *__restrict__ post_gate, float *__restrict__ mix) {
    pdl_enter();
    __shared__ float sh[4 + 16];
    const int t = blockIdx.x, tid = threadIdx.x, lane = layer % 4;
    if (tid < 4) {
        const int i = tid;
        const float *pr = pre + (size_t)t * ld_pre + layer * 4, *po = post + (size_t)t * ld_post + layer * 4;
        const float zp = __fadd_rn(__fadd_rn(__fmul_rn(a_pre[layer], pr[i]), b_pre[layer * 4 + i]),
                                   i == lane ? 4.0f : -4.0f);
        sh[i] = sigmoid_rn(zp);
        const float zq = __fadd_rn(__fadd_rn(__fmul_rn(a_post[layer], po[i]), b_post[layer * 4 + i]),
                                   i == lane ? 0.0f : -4.0f);
        post_gate[t * 4 + i] = __fmul_rn(2.0f, sigmoid_rn(zq));
    } else if (tid >= 32 && tid < 48) {
        const int j = tid - 32;
        sh[4 + j] = __fadd_rn(__fmul_rn(a_res[layer], res[(size_t)t * ld_res + layer * 16 + j]), b_res[layer * 16 + j]);
    }
    __syncthreads();
    const float w0 = sh[0], w1 = sh[1], w2 = sh[2], w3 = sh[3];
    const float *st = stream + (size_t)t * 4 * dim;
    for (int c = tid; c < dim; c += blockDim.x) {
        const float x = hc_mix4(st, dim, c, w0, w1, w2, w3);
        u[(size_t)t * dim + c] = x;
        residual[(size_t)t * dim + c] = x;
    }
    if (tid < 32) {  // both half-warps hold the row's matrix; the first stores it
        const float r = hc_sinkhorn16(sh[4 + (tid & 15)], tid);
        if (tid < 16) mix[(size_t)t * 16 + tid] = r;
    }
}

// Taps3 on triples [n][3][width] = (x_{t-2}, x_{t-1}, x_t).
__global__ void __launch_bounds__(256) taps3_kernel(const float *__restrict__ taps, int width,
                                                    const float *__restrict__ triples, int n,
                                                    float *__restrict__ dst) {
    pdl_enter();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)n * width) return;
    const int t = (int)(i / width), c = (int)(i - (long long)t * width);
    const float *cur = triples + (size_t)t * 3 * width + 2 * width;
    float acc = __fmul_rn(taps[c], cur[c]);
    acc = __fadd_rn(acc, __fmul_rn(taps[width + c], cur[c - width]));
    dst[(size_t)t * width + c] = __fadd_rn(acc, __fmul_rn(taps[2 * width + c], cur[c - 2 * width]));
}

// Warp per row.  MODE 0 RmsFakeA8, 1 CenteredRmsFakeA8 (aux = scale),
// 2 GateFakeA8 (aux = gate), 3 PostNormAdd (aux = scale, dst = residual,
// gate[row]).  The sum of squares runs on lane 0 in ascending order.
template <int MODE>
__global__ void __launch_bounds__(256) fake_a8_kernel(const float *__restrict__ x, const float *__restrict__ aux,
                                                      const float *__restrict__ gate, int rows, int n,
                                                      float *__restrict__ dst) {
    pdl_enter();
    const int row = (int)(((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + (size_t)row * n;
    float *dr = dst + (size_t)row * n;
    float inverse = 0.0f;
    if (MODE != 2) {
        float sum = 0.0f;
        if (lane == 0)
            for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(xr[i], xr[i]));
        sum = __shfl_sync(0xffffffffu, sum, 0);
        inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), 1e-6f)));
    }
    if (MODE == 3) {
        const float g = gate[row];
        for (int i = lane; i < n; i += 32)
            dr[i] = __fadd_rn(dr[i], __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, aux[i]), xr[i]), inverse)));
        return;
    }
    float peak = 0.0f;
    for (int i = lane; i < n; i += 32) {
        float v;
        if (MODE == 0) v = __fmul_rn(xr[i], inverse);
        else if (MODE == 1) v = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, aux[i]), xr[i]), inverse);
        else v = __fmul_rn(xr[i], sigmoid_rn(aux[(size_t)row * n + i]));
        dr[i] = v;
        peak = fmaxf(peak, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float round = __fdiv_rn(1.0f, scale);
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
        // Scalar.RoundEven (Scalar.cs:52-53): x + 1.5*2^23 - 1.5*2^23, which also
        // turns -0 into +0 (rintf would keep the sign of a zero)
        const float r = __fsub_rn(__fadd_rn(__fmul_rn(dr[i], round), 12582912.0f), 12582912.0f);
        dr[i] = __fmul_rn(fminf(fmaxf(r, -128.0f), 127.0f), scale);
    }
}

// CTA-per-row row ops for rows of n % 4 == 0, n <= 4096 floats on 16-byte
// boundaries, the arithmetic of the scalar code element for element:
//  MODE 0 RmsUnit (x * inverse), 1 ZeroCenteredRms (((1 + aux) x) inverse),
//  2 MultiplyBySigmoid (x sigmoid(aux row)), 3 PostNormAdd (dst += gate[row]
//  ((1 + aux) x) inverse), 4 ZeroCenteredRms then SiLU, 5 the row as it is;
//  kFake adds Quant.FakeA8 (RmsFakeA8, CenteredRmsFakeA8, GateFakeA8 for
//  modes 0..2, FakeA8 for mode 5), as fake_a8_kernel does.
// The row stays in registers (float4 i on thread i % 128), the squares go
// through shared memory and thread 0 sums them in ascending order with its
// next four float4 loads issued ahead of the current adds (the add chain is
// the kernel's critical path); the peak is a max over the CTA.  With kPrep
// the rows go on into CQ Prepare (n % 128 == 0): warp w holds group w + 4 i
// of the row as four consecutive elements per lane, and the prepared values,
// scales and offsets are written instead of dst.
constexpr int kFakeThreads = 128;
constexpr int kFakeMaxVec = 8;

__device__ __forceinline__ float fake_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int MODE, bool kPrep, bool kFake>
__global__ void __launch_bounds__(kFakeThreads) row_op_kernel(const float *__restrict__ x,
                                                              const float *__restrict__ aux,
                                                              const float *__restrict__ gate, int n,
                                                              float *__restrict__ dst, CqPrepOut prep) {
    constexpr bool kRms = MODE == 0 || MODE == 1 || MODE == 3 || MODE == 4;
    pdl_enter();
    __shared__ float red[kFakeThreads / 32];
    __shared__ float4 squares[kRms ? kFakeThreads * kFakeMaxVec : 1];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nv = n >> 2;
    const float4 *in = reinterpret_cast<const float4 *>(x + (size_t)row * n);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v[kFakeMaxVec];
#pragma unroll
    for (int i = 0; i < kFakeMaxVec; i++) {
        const int idx = tid + i * kFakeThreads;
        v[i] = idx < nv ? in[idx] : zero;
    }
    float inverse = 0.0f;
    if (kRms) {
#pragma unroll
        for (int i = 0; i < kFakeMaxVec; i++) {
            const int idx = tid + i * kFakeThreads;
            if (idx < nv)
                squares[idx] = make_float4(__fmul_rn(v[i].x, v[i].x), __fmul_rn(v[i].y, v[i].y),
                                           __fmul_rn(v[i].z, v[i].z), __fmul_rn(v[i].w, v[i].w));
        }
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            float4 nxt[4];
#pragma unroll
            for (int j = 0; j < 4; j++) nxt[j] = j < nv ? squares[j] : zero;
            for (int i = 0; i < nv; i += 4) {
                float4 cur[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    cur[j] = nxt[j];
                    nxt[j] = i + 4 + j < nv ? squares[i + 4 + j] : zero;
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    if (i + j < nv) {
                        sum = __fadd_rn(sum, cur[j].x);
                        sum = __fadd_rn(sum, cur[j].y);
                        sum = __fadd_rn(sum, cur[j].z);
                        sum = __fadd_rn(sum, cur[j].w);
                    }
                }
            }
            red[0] = sum;
        }
        __syncthreads();
        const float sum = red[0];
        __syncthreads();  // red is reused for the peak
        inverse = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), 1e-6f)));
    }
    if (MODE == 3) {
        const float g = gate[row];
        const float4 *sv = reinterpret_cast<const float4 *>(aux);
        float4 *dv = reinterpret_cast<float4 *>(dst + (size_t)row * n);
#pragma unroll
        for (int i = 0; i < kFakeMaxVec; i++) {
            const int idx = tid + i * kFakeThreads;
            if (idx < nv) {
                const float4 s = sv[idx];
                float4 o = dv[idx];
                o.x = __fadd_rn(o.x, __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, s.x), v[i].x), inverse)));
                o.y = __fadd_rn(o.y, __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, s.y), v[i].y), inverse)));
                o.z = __fadd_rn(o.z, __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, s.z), v[i].z), inverse)));
                o.w = __fadd_rn(o.w, __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, s.w), v[i].w), inverse)));
                dv[idx] = o;
            }
        }
        return;
    }
    float peak = 0.0f;
#pragma unroll
    for (int i = 0; i < kFakeMaxVec; i++) {
        const int idx = tid + i * kFakeThreads;
        if (idx < nv) {
            float *e = reinterpret_cast<float *>(&v[i]);
            float4 a = zero;
            if (MODE == 1 || MODE == 4) a = reinterpret_cast<const float4 *>(aux)[idx];
            if (MODE == 2) a = reinterpret_cast<const float4 *>(aux + (size_t)row * n)[idx];
            const float *av = reinterpret_cast<const float *>(&a);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (MODE == 0) e[k] = __fmul_rn(e[k], inverse);
                else if (MODE == 1 || MODE == 4) e[k] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, av[k]), e[k]), inverse);
                else if (MODE == 2) e[k] = __fmul_rn(e[k], sigmoid_rn(av[k]));
                if (MODE == 4) e[k] = __fmul_rn(e[k], sigmoid_rn(e[k]));
                peak = fmaxf(peak, fabsf(e[k]));
            }
        }
    }
    float scale = 1.0f, round = 1.0f;
    if (kFake) {
        peak = fake_warp_max(peak);
        if (lane == 0) red[warp] = peak;
        __syncthreads();
        peak = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
        round = __fdiv_rn(1.0f, scale);
    }
#pragma unroll
    for (int i = 0; i < kFakeMaxVec; i++) {
        const int idx = tid + i * kFakeThreads;
        if (idx < nv) {  // warp-uniform when kPrep (nv % 32 == 0)
            float *e = reinterpret_cast<float *>(&v[i]);
            if (kFake) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    // Scalar.RoundEven as in fake_a8_kernel
                    const float r = __fsub_rn(__fadd_rn(__fmul_rn(e[k], round), 12582912.0f), 12582912.0f);
                    e[k] = __fmul_rn(fminf(fmaxf(r, -128.0f), 127.0f), scale);
                }
            }
            if (kPrep) {
                float w[4] = {e[0], e[1], e[2], e[3]};
                const int g = idx >> 5;
                cq_prepare_group_lane4(w, lane, prep.bits, prep.values + (size_t)row * n + (size_t)g * 128,
                                       prep.scales + (size_t)row * prep.stride + g,
                                       prep.offsets + (size_t)row * prep.stride + g);
            } else {
                reinterpret_cast<float4 *>(dst + (size_t)row * n)[idx] = v[i];
            }
        }
    }
}

// The plain float helper slots (Scalar.cs:206-248, Ops.cs:209-255, Quant.cs:69-80)
// on one warp: sums run on lane 0 in ascending order, so the results equal the
// scalar code (Softmax's exp aside).  MODE 0 RmsUnit, 1 ZeroCenteredRms
// (aux = scale), 2 AddScaled, 3 ScaleAdd, 4 MultiplyAccumulate (aux = b),
// 5 Dot (aux = b, result in out[0]), 6 Softmax (x in place), 7 FakeA8 (x in
// place, scale in out[0]).  dst is the slot's destination.
template <int MODE>
__global__ void __launch_bounds__(32) slot_vec_kernel(float *__restrict__ x, const float *__restrict__ aux,
                                                      float *__restrict__ dst, float s0, float s1, int n,
                                                      float *__restrict__ out) {
    const int lane = threadIdx.x;
    if (MODE == 0 || MODE == 1) {
        float sum = 0.0f;
        if (lane == 0)
            for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
        sum = __shfl_sync(0xffffffffu, sum, 0);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), 1e-6f)));
        for (int i = lane; i < n; i += 32)
            dst[i] = MODE == 0 ? __fmul_rn(x[i], inv) : __fmul_rn(__fmul_rn(__fadd_rn(1.0f, aux[i]), x[i]), inv);
    } else if (MODE == 2) {
        for (int i = lane; i < n; i += 32) dst[i] = __fadd_rn(dst[i], __fmul_rn(s0, x[i]));
    } else if (MODE == 3) {
        for (int i = lane; i < n; i += 32) dst[i] = __fadd_rn(__fmul_rn(s0, dst[i]), __fmul_rn(s1, x[i]));
    } else if (MODE == 4) {
        for (int i = lane; i < n; i += 32) dst[i] = __fadd_rn(dst[i], __fmul_rn(x[i], aux[i]));
    } else if (MODE == 5) {
        if (lane == 0) {
            float sum = 0.0f;
            for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(x[i], aux[i]));
            out[0] = sum;
        }
    } else if (MODE == 6) {
        float peak = -INFINITY;
        for (int i = lane; i < n; i += 32) peak = fmaxf(peak, x[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
        for (int i = lane; i < n; i += 32) x[i] = exp_rn(__fsub_rn(x[i], peak));
        __syncwarp();
        float total = 0.0f;
        if (lane == 0)
            for (int i = 0; i < n; i++) total = __fadd_rn(total, x[i]);
        total = __shfl_sync(0xffffffffu, total, 0);
        for (int i = lane; i < n; i += 32) x[i] = __fdiv_rn(x[i], total);
    } else {  // FakeA8: AbsMax, then RoundTrip with the reference's RoundEven
        float peak = 0.0f;
        for (int i = lane; i < n; i += 32) peak = fmaxf(peak, fabsf(x[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
        const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
        const float inverse = __fdiv_rn(1.0f, scale);
        for (int i = lane; i < n; i += 32) {
            const float r = __fsub_rn(__fadd_rn(__fmul_rn(x[i], inverse), 12582912.0f), 12582912.0f);
            x[i] = __fmul_rn(fminf(fmaxf(r, -128.0f), 127.0f), scale);
        }
        if (lane == 0) out[0] = scale;
    }
}

// Scalar.Rope (Scalar.cs:233-248): half-split rotation of each head, in place.
__global__ void __launch_bounds__(256) slot_rope_kernel(float *__restrict__ x, int heads, int head_dim,
                                                        const float *__restrict__ cs, const float *__restrict__ sn) {
    const int half = head_dim / 2;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= heads * half) return;
    const int h = k / half, i = k - h * half;
    float *lo = x + (size_t)h * head_dim, *hi = lo + half;
    const float a = lo[i], b = hi[i];
    lo[i] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(b, sn[i]));
    hi[i] = __fadd_rn(__fmul_rn(b, cs[i]), __fmul_rn(a, sn[i]));
}

int launch_slot_vec(int mode, float *x, const float *aux, float *dst, float s0, float s1, int n, float *out,
                    cudaStream_t stream) {
    switch (mode) {
        case 0: slot_vec_kernel<0><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 1: slot_vec_kernel<1><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 2: slot_vec_kernel<2><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 3: slot_vec_kernel<3><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 4: slot_vec_kernel<4><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 5: slot_vec_kernel<5><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        case 6: slot_vec_kernel<6><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
        default: slot_vec_kernel<7><<<1, 32, 0, stream>>>(x, aux, dst, s0, s1, n, out); break;
    }
    return check_launch("slot_vec");
}

int launch_slot_rope(float *x, int heads, int head_dim, const float *cs, const float *sn, cudaStream_t stream) {
    const int k = heads * (head_dim / 2);
    if (k == 0) return NDL_OK;
    slot_rope_kernel<<<(k + 255) / 256, 256, 0, stream>>>(x, heads, head_dim, cs, sn);
    return check_launch("slot_rope");
}

// Attention.Run / Scalar.AttentionTile (src/Needle/Blocks.cs:65-84,
// src/Needle/Scalar.cs:290-321) on the reference's tile: up to 6 query heads
// sharing one key / value span, keys of 48 int8, values of 64.  Warp per
// head.  Without peaks the outputs are normalized (Softmax, then the
// weighted value sum); with peaks (the split-position mode of the
// reference's vector path, Blocks.cs:188-199) the outputs stay unnormalized
// and the head's peak and exp sum are stored for MergePartials.  Positions
// are summed in ascending order.
struct KtTileArgs {
    const int8_t *q;
    const float *qs;
    int heads;
    const int8_t *keys;  // row 0 = the tile's first position
    const float *ks;
    const int8_t *values;
    const float *vs;
    int key_stride, value_stride, scale_stride, count;
    float *scores;  // [heads][count]
    float *output;  // [heads][64]
    float *probs;   // [heads][count] or null
    float *peaks, *sums;  // [heads] or null
};

__global__ void __launch_bounds__(192) slot_attention_tile_kernel(KtTileArgs a) {
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (h >= a.heads) return;
    const int8_t *q = a.q + h * 48;
    const float scale = __fmul_rn(a.qs[h], 0.14433756729740643f);
    float *sc = a.scores + (size_t)h * a.count;
    float peak = -INFINITY;
    for (int s = lane; s < a.count; s += 32) {
        const int8_t *k = a.keys + (size_t)s * a.key_stride;
        int dot = 0;
        for (int d = 0; d < 48; d++) dot += (int)q[d] * (int)k[d];
        const float v = __fmul_rn(__fmul_rn((float)dot, a.ks[(size_t)s * a.scale_stride]), scale);
        sc[s] = v;
        peak = fmaxf(peak, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    for (int s = lane; s < a.count; s += 32) sc[s] = exp_rn(__fsub_rn(sc[s], peak));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0)
        for (int s = 0; s < a.count; s++) total = __fadd_rn(total, sc[s]);
    total = __shfl_sync(0xffffffffu, total, 0);
    const bool partial = a.peaks != nullptr;
    if (!partial)
        for (int s = lane; s < a.count; s += 32) sc[s] = __fdiv_rn(sc[s], total);
    __syncwarp();
    if (a.probs)
        for (int s = lane; s < a.count; s += 32) a.probs[(size_t)h * a.count + s] = sc[s];
    float o0 = 0.0f, o1 = 0.0f;
    for (int s = 0; s < a.count; s++) {
        const float w = __fmul_rn(sc[s], a.vs[(size_t)s * a.scale_stride]);
        const int8_t *row = a.values + (size_t)s * a.value_stride;
        o0 = __fadd_rn(o0, __fmul_rn(w, (float)row[2 * lane]));
        o1 = __fadd_rn(o1, __fmul_rn(w, (float)row[2 * lane + 1]));
    }
    a.output[h * 64 + 2 * lane] = o0;
    a.output[h * 64 + 2 * lane + 1] = o1;
    if (partial && lane == 0) {
        a.peaks[h] = peak;
        a.sums[h] = total;
    }
}

// Attention.MergePartials (src/Needle/Blocks.cs:750-817) over `count`
// partial slots of 6*64 + 16 floats (outputs, peaks at 384 + h, sums at
// 392 + h): warp per head, lane owns dims 2*lane, 2*lane+1, the scalar
// branch's arithmetic (two-chunk form for count == 2).
__global__ void __launch_bounds__(192) slot_merge_partials_kernel(const float *__restrict__ p, int count, int heads,
                                                                  float *__restrict__ out) {
    constexpr int kStride = 6 * 64 + 16, kPeak = 6 * 64;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (h >= heads) return;
    for (int k = 0; k < 2; k++) {
        const int d = 2 * lane + k;
        float r;
        if (count == 2) {
            const float p0 = p[kPeak + h], p1 = p[kStride + kPeak + h];
            const float pk = fmaxf(p0, p1);
            const float w0 = exp_rn(__fsub_rn(p0, pk)), w1 = exp_rn(__fsub_rn(p1, pk));
            float tot = __fadd_rn(0.0f, __fmul_rn(w0, p[kPeak + 8 + h]));
            tot = __fadd_rn(tot, __fmul_rn(w1, p[kStride + kPeak + 8 + h]));
            const float inv = __fdiv_rn(1.0f, tot);
            r = __fmul_rn(__fadd_rn(__fmul_rn(w0, p[h * 64 + d]), __fmul_rn(w1, p[kStride + h * 64 + d])), inv);
        } else {
            float peak = -INFINITY;
            for (int c = 0; c < count; c++) peak = fmaxf(peak, p[c * kStride + kPeak + h]);
            float total = 0.0f, sum = 0.0f;
            for (int c = 0; c < count; c++) {
                const float w = exp_rn(__fsub_rn(p[c * kStride + kPeak + h], peak));
                total = __fadd_rn(total, __fmul_rn(w, p[c * kStride + kPeak + 8 + h]));
                sum = __fadd_rn(sum, __fmul_rn(w, p[c * kStride + h * 64 + d]));
            }
            r = __fmul_rn(sum, __fdiv_rn(1.0f, total));
        }
        out[h * 64 + d] = r;
    }
}

int launch_slot_attention_tile(const KtTileArgs &a, cudaStream_t stream) {
    slot_attention_tile_kernel<<<1, 192, 0, stream>>>(a);
    return check_launch("slot_attention_tile");
}
int launch_slot_merge_partials(const float *partials, int count, int heads, float *out, cudaStream_t stream) {
    slot_merge_partials_kernel<<<1, 192, 0, stream>>>(partials, count, heads, out);
    return check_launch("slot_merge_partials");
}

// HadamardMlp.Apply (src/Needle/Blocks.cs:1067-1093, scalar steps
// Scalar.cs:323-358,441-460) on one token: one CTA, each step's outputs in
// parallel, every inner sum sequential in the scalar order.  w holds the
// MlpWeights arrays (d1, d2, b2, d3, d4, w1a, w1b, w2a, w2b, w3a, w3b,
// cond_v, cond_u); smem: weights[8], normalized[dim], front / back / kron
// scratch [width] each.
// One Kronecker factor pair: tmp = left^T z (active_rows of z), then
// result = tmp right, every element a sum in ascending index order.  Each
// thread runs the chains of up to four elements (blockDim apart) side by
// side so their loads and adds overlap.
__device__ void mlp_kron(const float *z, int active_rows, const float *left, const float *right, int rows, int cols,
                         int result_rows, float *tmp, float *result) {
    const int n = result_rows * cols;
    for (int e0 = threadIdx.x; e0 < n; e0 += 4 * blockDim.x) {
        int kq[4], cq[4];
        float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int e = min(e0 + q * (int)blockDim.x, n - 1);
            kq[q] = e / cols;
            cq[q] = e - kq[q] * cols;
        }
#pragma unroll 4
        for (int i = 0; i < active_rows; i++)
#pragma unroll
            for (int q = 0; q < 4; q++) sum[q] = __fadd_rn(sum[q], __fmul_rn(left[i * rows + kq[q]], z[i * cols + cq[q]]));
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (e0 + q * (int)blockDim.x < n) tmp[e0 + q * blockDim.x] = sum[q];
    }
    __syncthreads();
    for (int e0 = threadIdx.x; e0 < n; e0 += 4 * blockDim.x) {
        int kq[4], cq[4];
        float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int e = min(e0 + q * (int)blockDim.x, n - 1);
            kq[q] = e / cols;
            cq[q] = e - kq[q] * cols;
        }
#pragma unroll 4
        for (int j = 0; j < cols; j++)
#pragma unroll
            for (int q = 0; q < 4; q++) sum[q] = __fadd_rn(sum[q], __fmul_rn(tmp[kq[q] * cols + j], right[j * cols + cq[q]]));
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (e0 + q * (int)blockDim.x < n) result[e0 + q * blockDim.x] = sum[q];
    }
    __syncthreads();
}

// mlp_kron with each thread on four adjacent columns of one output row
// (cols % 4 == 0, every array on 16-byte boundaries): per step one broadcast
// load of the left (or tmp) value and one 16-byte load of z (or right) feed
// four chains, the same products and sums in the same order.  tmp rows are
// cols + 4 floats apart, so the four rows a warp reads in the second product
// sit in four different banks (at a stride of cols they would share one).
__device__ void mlp_kron4(const float *z, int active_rows, const float *left, const float *right, int rows, int cols,
                          int result_rows, float *tmp, float *result) {
    const int quads = cols >> 2, n = result_rows * quads;
    for (int u = threadIdx.x; u < n; u += blockDim.x) {
        const int k = u / quads, c = (u - k * quads) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int i = 0; i < active_rows; i++) {
            const float l = left[i * rows + k];
            const float4 zz = *reinterpret_cast<const float4 *>(z + i * cols + c);
            acc.x = __fadd_rn(acc.x, __fmul_rn(l, zz.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(l, zz.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(l, zz.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(l, zz.w));
        }
        *reinterpret_cast<float4 *>(tmp + k * (cols + 4) + c) = acc;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < n; u += blockDim.x) {
        const int k = u / quads, c = (u - k * quads) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int j = 0; j < cols; j++) {
            const float t = tmp[k * (cols + 4) + j];
            const float4 rr = *reinterpret_cast<const float4 *>(right + j * cols + c);
            acc.x = __fadd_rn(acc.x, __fmul_rn(t, rr.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(t, rr.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(t, rr.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(t, rr.w));
        }
        *reinterpret_cast<float4 *>(result + k * cols + c) = acc;
    }
    __syncthreads();
}

// Shared floats of slot_hadamard_mlp_kernel: weights[8], normalized[dim],
// front / back [width], tmp [rows][cols + 4], scratch[8][dim + 4] (squares,
// then the ConditionWeights products, rows dim + 4 apart so that the eight
// products of one normalized element land in eight banks), the residual row
// [dim] and the six Kronecker factors (the first left factor's in_rows x
// rows, two more rows x rows, three cols x cols).
__host__ __device__ inline size_t mlp_smem_floats(int dim, int rows, int cols) {
    const size_t in_rows = (size_t)(dim + cols - 1) / cols;
    return 8 + (size_t)dim + 2 * (size_t)rows * cols + (size_t)rows * (cols + 4) + 8 * ((size_t)dim + 4) +
           (size_t)dim + (in_rows + 2 * (size_t)rows) * rows + 3 * (size_t)cols * cols;
}

// Element loop over [0, n) in which every thread issues the loads of kBatch
// of its elements (load(i), global) before it uses any of them (use(i, v)):
// one memory round trip per kBatch elements instead of one per element.
template <int kBatch, typename Load, typename Use>
__device__ __forceinline__ void mlp_batched(int n, int tid, int threads, Load load, Use use) {
    for (int base = tid; base < n; base += kBatch * threads) {
        decltype(load(0)) v[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int i = base + k * threads;
            if (i < n) v[k] = load(i);
        }
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int i = base + k * threads;
            if (i < n) use(i, v[k]);
        }
    }
}

// The ascending fp32 sum of x[0..n) (shared memory, 16-byte aligned) on one
// thread, its next four float4 loads issued ahead of the current adds.
__device__ __forceinline__ float mlp_ordered_sum(const float *x, int n) {
    float sum = 0.0f;
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) {  // rows of a width that is not a multiple of 4
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, x[i]);
        return sum;
    }
    const int nv = n >> 2;
    const float4 *v = reinterpret_cast<const float4 *>(x);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 nxt[4];
#pragma unroll
    for (int j = 0; j < 4; j++) nxt[j] = j < nv ? v[j] : zero;
    for (int i = 0; i < nv; i += 4) {
        float4 cur[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            cur[j] = nxt[j];
            nxt[j] = i + 4 + j < nv ? v[i + 4 + j] : zero;
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (i + j < nv) {
                sum = __fadd_rn(sum, cur[j].x);
                sum = __fadd_rn(sum, cur[j].y);
                sum = __fadd_rn(sum, cur[j].z);
                sum = __fadd_rn(sum, cur[j].w);
            }
    }
    for (int i = nv * 4; i < n; i++) sum = __fadd_rn(sum, x[i]);
    return sum;
}

struct MlpCondition {
    float w[8], d2, b2;
    int perm;
};

__global__ void __launch_bounds__(256) slot_hadamard_mlp_kernel(KtMlpArgs a) {
    extern __shared__ float sm[];
    float *const residual = a.residual + (size_t)blockIdx.x * a.row_stride;
    const int dim = a.dim, rows = a.rows, cols = a.cols, width = rows * cols;
    const int input_rows = (dim + cols - 1) / cols;
    const int output_rows = min(rows, (input_rows + 3) / 4 * 4);
    const int tid = threadIdx.x, nt = blockDim.x;
    float *weights = sm, *normalized = sm + 8, *front = normalized + dim, *back = front + width, *tmp = back + width;
    const int sd = dim + 4;  // scratch row stride
    float *scratch = tmp + rows * (cols + 4), *res = scratch + 8 * sd;
    float *left1 = res + dim, *right1 = left1 + input_rows * rows, *left2 = right1 + cols * cols;
    float *right2 = left2 + rows * rows, *left3 = right2 + cols * cols, *right3 = left3 + rows * rows;
    const float *__restrict__ d1 = a.w[0], *__restrict__ d2 = a.w[1], *__restrict__ b2 = a.w[2];
    const float *__restrict__ d3 = a.w[3], *__restrict__ d4 = a.w[4], *__restrict__ cond_v = a.w[11];
    const float *__restrict__ cond_u = a.w[12], *__restrict__ pre = a.pre_norm;
    const int32_t *__restrict__ perm_a = a.perm_a, *__restrict__ perm_b = a.perm_b;
    // the Kronecker products four columns a thread where the shared arrays sit on 16-byte boundaries
    const bool quads = dim % 4 == 0 && rows % 4 == 0 && cols % 4 == 0 && input_rows % 4 == 0;
    auto kron = [&](const float *z, int active, const float *l, const float *r, int rw, int cl, int res_rows,
                    float *t, float *out) {
        if (quads) mlp_kron4(z, active, l, r, rw, cl, res_rows, t, out);
        else mlp_kron(z, active, l, r, rw, cl, res_rows, t, out);
    };
    if (a.pn_x) {
        // Scalar.PostNormAdd first: the projection's squares summed in order, then
        // residual + gate ((1 + scale) x) inverse, kept in res
        const float *px = a.pn_x + (size_t)blockIdx.x * dim;
        mlp_batched<4>(dim, tid, nt, [&](int i) { return px[i]; }, [&](int i, float x) {
            normalized[i] = x;
            scratch[i] = __fmul_rn(x, x);
        });
        __syncthreads();
        if (tid == 0) {
            const float sum = mlp_ordered_sum(scratch, dim);
            weights[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)dim), 1e-6f)));
        }
        __syncthreads();
        const float pinv = weights[0], g = a.pn_gate[blockIdx.x];
        const float *__restrict__ ps = a.pn_scale;
        mlp_batched<4>(dim, tid, nt, [&](int i) { return make_float2(residual[i], __ldg(ps + i)); },
                       [&](int i, float2 rs) {
                           const float r = __fadd_rn(
                               rs.x, __fmul_rn(g, __fmul_rn(__fmul_rn(__fadd_rn(1.0f, rs.y), normalized[i]), pinv)));
                           res[i] = r;
                           scratch[i] = __fmul_rn(r, r);
                       });
    } else {
        // the residual row and its squares (ZeroCenteredRms)
        mlp_batched<4>(dim, tid, nt, [&](int i) { return residual[i]; }, [&](int i, float r) {
            res[i] = r;
            scratch[i] = __fmul_rn(r, r);
        });
    }
    __syncthreads();
    if (tid == 0) {  // the sum of squares in order
        const float sum = mlp_ordered_sum(scratch, dim);
        weights[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)dim), 1e-6f)));
    } else if (tid >= 32) {  // meanwhile the other warps stage the Kronecker factors
        const int sizes[6] = {input_rows * rows, cols * cols, rows * rows, cols * cols, rows * rows, cols * cols};
        float *dsts[6] = {left1, right1, left2, right2, left3, right3};
        const int t2 = tid - 32, n2 = nt - 32;
        int most = 0;
        for (int f = 0; f < 6; f++) most = max(most, sizes[f]);
        // every factor's loads of a chunk go out before any of its stores
        for (int base = t2; base < most; base += 4 * n2) {
            float v[6][4];
#pragma unroll
            for (int f = 0; f < 6; f++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int i = base + k * n2;
                    v[f][k] = i < sizes[f] ? __ldg(a.w[5 + f] + i) : 0.0f;
                }
#pragma unroll
            for (int f = 0; f < 6; f++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int i = base + k * n2;
                    if (i < sizes[f]) dsts[f][i] = v[f][k];
                }
        }
    }
    __syncthreads();
    const float inv = weights[0];
    mlp_batched<4>(dim, tid, nt, [&](int i) { return __ldg(pre + i); }, [&](int i, float p) {
        normalized[i] = __fmul_rn(__fmul_rn(__fadd_rn(1.0f, p), res[i]), inv);
    });
    __syncthreads();
    // ConditionWeights: products in parallel (weight j's row of dim contiguous),
    // weight j summed in order by thread j
    mlp_batched<8>(dim * 8, tid, nt, [&](int e) { return __ldg(cond_v + e); },
                   [&](int e, float w) { scratch[(e & 7) * sd + (e >> 3)] = __fmul_rn(normalized[e >> 3], w); });
    __syncthreads();
    if (tid < 8) weights[tid] = mlp_ordered_sum(scratch + tid * sd, dim);
    __syncthreads();
    // Softmax over the 8 weights: the peak and the exponentials on 8 threads, the
    // total in order and the divisions on thread 0
    if (tid < 8) {
        float peak = -INFINITY;
        for (int j = 0; j < 8; j++) peak = fmaxf(peak, weights[j]);
        scratch[tid] = exp_rn(__fsub_rn(weights[tid], peak));
    }
    __syncthreads();
    if (tid == 0) {
        float total = 0.0f;
        for (int j = 0; j < 8; j++) total = __fadd_rn(total, scratch[j]);
        for (int j = 0; j < 8; j++) weights[j] = __fdiv_rn(scratch[j], total);
    }
    mlp_batched<4>(input_rows * cols, tid, nt, [&](int i) { return i < dim ? __ldg(d1 + i) : 0.0f; },
                   [&](int i, float w) { front[i] = i < dim ? __fmul_rn(normalized[i], w) : 0.0f; });
    __syncthreads();
    kron(front, input_rows, left1, right1, rows, cols, rows, tmp, back);
    mlp_batched<4>(width, tid, nt,
                   [&](int n) {
                       MlpCondition c;
#pragma unroll
                       for (int j = 0; j < 8; j++) c.w[j] = __ldg(cond_u + j * width + n);
                       c.d2 = __ldg(d2 + n);
                       c.b2 = __ldg(b2 + n);
                       c.perm = __ldg(perm_a + n);
                       return c;
                   },
                   [&](int n, const MlpCondition &c) {
                       float condition = 1.0f;
#pragma unroll
                       for (int j = 0; j < 8; j++) condition = __fadd_rn(condition, __fmul_rn(weights[j], c.w[j]));
                       const float v = __fadd_rn(__fmul_rn(__fmul_rn(c.d2, condition), back[c.perm]), c.b2);
                       front[n] = __fmul_rn(v, sigmoid_rn(v));
                   });
    __syncthreads();
    kron(front, rows, left2, right2, rows, cols, rows, tmp, back);
    mlp_batched<4>(width, tid, nt, [&](int n) { return make_float2(__int_as_float(__ldg(perm_b + n)), __ldg(d3 + n)); },
                   [&](int n, float2 p) { front[n] = __fmul_rn(back[__float_as_int(p.x)], p.y); });
    __syncthreads();
    kron(front, rows, left3, right3, rows, cols, output_rows, tmp, back);
    mlp_batched<4>(dim, tid, nt, [&](int i) { return __ldg(d4 + i); }, [&](int i, float w) {
        const float r = __fadd_rn(res[i], __fmul_rn(a.scale, __fmul_rn(back[i], w)));
        residual[i] = r;
        res[i] = r;
    });
    if (a.cb_next) {
        // Ops.CombineDiff4x4 (Ops.cs:800-812) on the row: lane o of next =
        // post[o] (residual - u) + mix[4o..4o+3] . stream, left to right
        __syncthreads();
        const size_t row = blockIdx.x;
        const float *st = a.cb_stream + row * 4 * dim, *m = a.cb_mix + row * 16, *uu = a.cb_u + row * dim;
        const float *pg = a.cb_post + row * 4;
        float *nx = a.cb_next + row * 4 * dim;
        for (int e = tid; e < 4 * dim; e += nt) {
            const int o = e / dim, c = e - o * dim;
            const float head = __fmul_rn(pg[o], __fsub_rn(res[c], uu[c]));
            nx[e] = mix4_term(head, m[4 * o], m[4 * o + 1], m[4 * o + 2], m[4 * o + 3], st, dim, c);
        }
    }
}

int launch_mlp_rows(const KtMlpArgs &a, int count, cudaStream_t stream) {
    if (count == 0) return NDL_OK;
    const size_t smem = mlp_smem_floats(a.dim, a.rows, a.cols) * 4;
    if (smem > 200 * 1024) return set_error(NDL_ERR_UNSUPPORTED, "hadamard_mlp: dim %d x width %d too large", a.dim,
                                            a.rows * a.cols);
    NDL_CUDA(cudaFuncSetAttribute(slot_hadamard_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    launch_kernel(slot_hadamard_mlp_kernel, dim3((unsigned)count), dim3(256), smem, stream, a);
    return check_launch("hadamard_mlp_rows");
}

int launch_hadamard_mlp_rows(const float *const w[13], const float *pre_norm, const int32_t *perm_a,
                             const int32_t *perm_b, int dim, int rows, int cols, float scale, float *residual, int count,
                             cudaStream_t stream) {
    if (count == 0) return NDL_OK;
    KtMlpArgs a{};
    for (int k = 0; k < 13; k++) a.w[k] = w[k];
    a.pre_norm = pre_norm;
    a.perm_a = perm_a;
    a.perm_b = perm_b;
    a.dim = dim;
    a.rows = rows;
    a.cols = cols;
    a.scale = scale;
    a.residual = residual;
    a.row_stride = dim;
    const size_t smem = mlp_smem_floats(dim, rows, cols) * 4;
    if (smem > 200 * 1024) return set_error(NDL_ERR_UNSUPPORTED, "hadamard_mlp: dim %d x width %d too large", dim,
                                            rows * cols);
    NDL_CUDA(cudaFuncSetAttribute(slot_hadamard_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    launch_kernel(slot_hadamard_mlp_kernel, dim3((unsigned)count), dim3(256), smem, stream, a);
    return check_launch("hadamard_mlp_rows");
}

int launch_slot_hadamard_mlp(const KtMlpArgs &a, cudaStream_t stream) {
    const size_t smem = mlp_smem_floats(a.dim, a.rows, a.cols) * 4;
    if (smem > 200 * 1024) return set_error(NDL_ERR_UNSUPPORTED, "hadamard_mlp: dim %d x width %d too large", a.dim,
                                            a.rows * a.cols);
    NDL_CUDA(cudaFuncSetAttribute(slot_hadamard_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    slot_hadamard_mlp_kernel<<<1, 256, smem, stream>>>(a);
    return check_launch("slot_hadamard_mlp");
}

static unsigned blocks_for(long long threads, int per_block) {
    return (unsigned)((threads + per_block - 1) / per_block);
}

int launch_mix4(const float *s, int dim, const float *w, int n, float *dst, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    launch_kernel(mix4_kernel, dim3(blocks_for((long long)n * dim, 256)), dim3(256), 0, stream, s, dim, w, n, dst);
    return check_launch("mix4");
}
int launch_combine4(bool diff, const float *s, int dim, const float *mix, const float *x, const float *u,
                    const float *post, int n, float *dst, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    if (diff)
        launch_kernel(combine4_kernel<true>, dim3(blocks_for((long long)n * 4 * dim, 256)), dim3(256), 0, stream, s,
                      dim, mix, x, u, post, n, dst);
    else
        launch_kernel(combine4_kernel<false>, dim3(blocks_for((long long)n * dim, 256)), dim3(256), 0, stream, s, dim,
                      mix, x, u, post, n, dst);
    return check_launch("combine4");
}
int launch_hc_prepare(const float *pre, int ld_pre, const float *post, int ld_post, const float *res, int ld_res,
                      const float *a_pre, const float *b_pre, const float *a_post, const float *b_post,
                      const float *a_res, const float *b_res, int layer, const float *stream, int dim, int rows, float *u,
                      float *residual, float *post_gate, float *mix, cudaStream_t cs) {
    if (rows == 0) return NDL_OK;
    launch_kernel(hc_prepare_kernel, dim3((unsigned)rows), dim3(256), 0, cs, pre, ld_pre, post, ld_post, res, ld_res,
                  a_pre, b_pre, a_post, b_post, a_res, b_res, layer, stream, dim, u, residual, post_gate, mix);
    return check_launch("hc_prepare");
}
int launch_sinkhorn4x4(const float *logits, int n, float *out, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    launch_kernel(sinkhorn4x4_kernel, dim3(blocks_for((long long)n * 16, 128)), dim3(128), 0, stream, logits, n, out);
    return check_launch("sinkhorn4x4");
}
int launch_taps3(const float *taps, int width, const float *triples, int n, float *dst, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    launch_kernel(taps3_kernel, dim3(blocks_for((long long)n * width, 256)), dim3(256), 0, stream, taps, width,
                  triples, n, dst);
    return check_launch("taps3");
}
int launch_fake_a8(int mode, const float *x, const float *aux, const float *gate, int rows, int n, float *dst,
                   cudaStream_t stream) {
    if (rows == 0) return NDL_OK;
    if (n % 4 == 0 && n <= 4 * kFakeThreads * kFakeMaxVec && aligned(x, 16) && aligned(dst, 16) &&
        (mode == 0 || aligned(aux, 16))) {
        return launch_row_op(mode, mode != 3, x, aux, gate, rows, n, dst, nullptr, stream);
    }
    const dim3 grid(blocks_for((long long)rows * 32, 256)), block(256);
    switch (mode) {
        case 0: launch_kernel(fake_a8_kernel<0>, grid, block, 0, stream, x, aux, gate, rows, n, dst); break;
        case 1: launch_kernel(fake_a8_kernel<1>, grid, block, 0, stream, x, aux, gate, rows, n, dst); break;
        case 2: launch_kernel(fake_a8_kernel<2>, grid, block, 0, stream, x, aux, gate, rows, n, dst); break;
        default: launch_kernel(fake_a8_kernel<3>, grid, block, 0, stream, x, aux, gate, rows, n, dst); break;
    }
    return check_launch("fake_a8");
}

template <int MODE, bool kPrep, bool kFake>
static void row_op_launch(dim3 grid, const float *x, const float *aux, const float *gate, int n, float *dst,
                          const CqPrepOut &prep, cudaStream_t stream) {
    launch_kernel(row_op_kernel<MODE, kPrep, kFake>, grid, dim3(kFakeThreads), 0, stream, x, aux, gate, n, dst, prep);
}

template <int MODE>
static void row_op_dispatch(bool fake, bool with_prep, dim3 grid, const float *x, const float *aux, const float *gate,
                            int n, float *dst, const CqPrepOut &prep, cudaStream_t stream) {
    if (with_prep) {
        if (fake) row_op_launch<MODE, true, true>(grid, x, aux, gate, n, dst, prep, stream);
        else row_op_launch<MODE, true, false>(grid, x, aux, gate, n, dst, prep, stream);
    } else {
        if (fake) row_op_launch<MODE, false, true>(grid, x, aux, gate, n, dst, prep, stream);
        else row_op_launch<MODE, false, false>(grid, x, aux, gate, n, dst, prep, stream);
    }
}

int launch_row_op(int mode, bool fake, const float *x, const float *aux, const float *gate, int rows, int n,
                  float *dst, const CqPrepOut *prep, cudaStream_t stream) {
    const bool uses_aux = mode == 1 || mode == 2 || mode == 3 || mode == 4;
    if (mode < 0 || mode > 5 || (mode == 3 && (fake || prep)) || n % (prep ? 128 : 4) != 0 ||
        n > 4 * kFakeThreads * kFakeMaxVec || !aligned(x, 16) || (uses_aux && !aligned(aux, 16)) ||
        (!prep && !aligned(dst, 16)) || (prep && prep->stride < n / 128))
        return NDL_ERR_UNSUPPORTED;
    if (rows == 0) return NDL_OK;
    const dim3 grid((unsigned)rows);
    const CqPrepOut none{}, &p = prep ? *prep : none;
    const bool wp = prep != nullptr;
    switch (mode) {
        case 0: row_op_dispatch<0>(fake, wp, grid, x, aux, gate, n, dst, p, stream); break;
        case 1: row_op_dispatch<1>(fake, wp, grid, x, aux, gate, n, dst, p, stream); break;
        case 2: row_op_dispatch<2>(fake, wp, grid, x, aux, gate, n, dst, p, stream); break;
        case 3: row_op_launch<3, false, false>(grid, x, aux, gate, n, dst, p, stream); break;
        case 4: row_op_dispatch<4>(fake, wp, grid, x, aux, gate, n, dst, p, stream); break;
        default: row_op_dispatch<5>(fake, wp, grid, x, aux, gate, n, dst, p, stream); break;
    }
    return check_launch("row_op");
}

int launch_fake_a8_prepare(int mode, const float *x, const float *aux, int rows, int n, int bits, int8_t *values,
                           float *scales, float *offsets, int stride, cudaStream_t stream) {
    if (mode < 0 || mode > 2) return NDL_ERR_UNSUPPORTED;
    const CqPrepOut prep{values, scales, offsets, stride, bits};
    return launch_row_op(mode, true, x, aux, nullptr, rows, n, nullptr, &prep, stream);
}

}  // namespace ndl

using namespace ndl;

extern "C" NDL_API int ndl_hc_mix4(const float *s, int dim, const float *w, int n, float *dst, void *stream) {
    NDL_REQUIRE(dim >= 1 && n >= 0, "dim %d / n %d", dim, n);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(s && w && dst, "null pointer");
    return launch_mix4(s, dim, w, n, dst, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_hc_combine_diff4x4(const float *s, int dim, const float *mix, const float *x,
                                              const float *u, const float *post_gate, int n, float *dst,
                                              void *stream) {
    NDL_REQUIRE(dim >= 1 && n >= 0, "dim %d / n %d", dim, n);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(s && mix && x && u && post_gate && dst, "null pointer");
    return launch_combine4(true, s, dim, mix, x, u, post_gate, n, dst, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_hc_combine4(const float *s, int dim, const float *w, const float *y, const float *post,
                                       int n, float *dst, void *stream) {
    NDL_REQUIRE(dim >= 1 && n >= 0, "dim %d / n %d", dim, n);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(s && w && y && post && dst, "null pointer");
    return launch_combine4(false, s, dim, w, y, nullptr, post, n, dst, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_hc_sinkhorn4x4(const float *logits, int n, float *out, void *stream) {
    NDL_REQUIRE(n >= 0, "n %d", n);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(logits && out, "null pointer");
    return launch_sinkhorn4x4(logits, n, out, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_taps3(const float *taps, int width, const float *triples, int n, float *dst, void *stream) {
    NDL_REQUIRE(width >= 1 && n >= 0, "width %d / n %d", width, n);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(taps && triples && dst, "null pointer");
    return launch_taps3(taps, width, triples, n, dst, (cudaStream_t)stream);
}

extern "C" NDL_API int ndl_fake_a8_rows(int mode, const float *x, const float *aux, const float *gate, int rows,
                                        int n, float *dst, void *stream) {
    NDL_REQUIRE(mode >= 0 && mode <= 3, "mode %d (0..3)", mode);
    NDL_REQUIRE(rows >= 0 && n >= 1, "rows %d / n %d", rows, n);
    if (rows == 0) return NDL_OK;
    NDL_REQUIRE(x && dst && (mode == 0 || aux) && (mode != 3 || gate), "null pointer");
    return launch_fake_a8(mode, x, aux, gate, rows, n, dst, (cudaStream_t)stream);
}

// HadamardMlp.Apply (src/Needle/Blocks.cs:1067-1093) over `count` residual
// rows of a loaded model's layer, block per row: the layer's MLP factors and
// pre-norm scale, the model's two permutations, its HadaRows x HadaCols split.
extern "C" NDL_API int ndl_mlp_apply(const ndl_model *m, int layer, float *residual, int count, float scale,
                                     void *stream) {
    NDL_REQUIRE(m, "null model");
    ndl_model_info g;
    if (ndl_model_get_info(m, &g) != NDL_OK) return NDL_ERR_INVALID_ARG;
    NDL_REQUIRE(g.device >= 0, "the model is not on a device (load it with a device)");
    NDL_REQUIRE(layer >= 0 && layer < g.layers, "layer %d of %d", layer, g.layers);
    NDL_REQUIRE(count >= 0, "count %d", count);
    const int dim = g.dim, rows = g.hada_rows, cols = g.hada_cols, width = g.hada_n;
    const int in_rows = cols > 0 ? (dim + cols - 1) / cols : 0;
    if (width <= 0 || in_rows > rows)
        return set_error(NDL_ERR_UNSUPPORTED, "HadaN %d (%d x %d) cannot hold a %d-wide row", width, rows, cols, dim);
    static const char *names[13] = {"layer.mlp.d1",  "layer.mlp.d2",  "layer.mlp.b2",     "layer.mlp.d3",
                                    "layer.mlp.d4",  "layer.mlp.w1a", "layer.mlp.w1b",    "layer.mlp.w2a",
                                    "layer.mlp.w2b", "layer.mlp.w3a", "layer.mlp.w3b",    "layer.mlp.cond_v",
                                    "layer.mlp.cond_u"};
    const long long need[13] = {dim, width, width, width, dim, (long long)in_rows * rows, (long long)cols * cols,
                                (long long)rows * rows, (long long)cols * cols, (long long)rows * rows,
                                (long long)cols * cols, (long long)dim * 8, 8LL * width};
    KtMlpArgs a{};
    ndl_model_tensor t;
    for (int k = 0; k < 13; k++) {
        if (ndl_model_get_tensor(m, names[k], layer, &t) != NDL_OK) return NDL_ERR_INVALID_ARG;
        if (t.kind != NDL_TENSOR_DENSE || t.count < need[k])
            return set_error(NDL_ERR_UNSUPPORTED, "%s %d holds %lld values, %lld needed", names[k], layer,
                             (long long)t.count, need[k]);
        a.w[k] = t.values;
    }
    if (ndl_model_get_tensor(m, "layer.pre_hada", layer, &t) != NDL_OK) return NDL_ERR_INVALID_ARG;
    if (t.count < dim) return set_error(NDL_ERR_UNSUPPORTED, "layer.pre_hada %d holds %lld values", layer, (long long)t.count);
    a.pre_norm = t.values;
    if (ndl_model_get_tensor(m, "hyper.perm_a", 0, &t) != NDL_OK) return NDL_ERR_INVALID_ARG;
    a.perm_a = t.permutation;
    if (ndl_model_get_tensor(m, "hyper.perm_b", 0, &t) != NDL_OK) return NDL_ERR_INVALID_ARG;
    a.perm_b = t.permutation;
    if (count == 0) return NDL_OK;
    NDL_REQUIRE(residual, "null residual");
    a.dim = dim;
    a.rows = rows;
    a.cols = cols;
    a.scale = scale;
    a.residual = residual;
    a.row_stride = dim;
    const size_t smem = mlp_smem_floats(dim, rows, cols) * 4;
    if (smem > 200 * 1024) return set_error(NDL_ERR_UNSUPPORTED, "hadamard_mlp: dim %d x width %d too large", dim, width);
    NDL_CUDA(cudaFuncSetAttribute(slot_hadamard_mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    slot_hadamard_mlp_kernel<<<(unsigned)count, 256, smem, (cudaStream_t)stream>>>(a);
    return check_launch("hadamard_mlp_rows");
}
