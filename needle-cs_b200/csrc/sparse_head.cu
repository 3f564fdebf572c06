// Grammar-constrained sparse head.
//
// Engine.LogitsForBatchRow (src/Needle/Engine.cs:2683-2700) computes the
// logits of one batch row only at the vocabulary ids a grammar allows (the
// reference rounds each run of consecutive ids out to multiples of 4 for its
// SIMD rows; every logit is an independent row dot, so the values at the
// requested ids are the dense head's).  ArgMaxSparse
// (src/Needle/NeedleSession.cs:984-995) then picks the first id of the list
// holding the strict maximum and BestProbability over the list's values.
//
// Here one launch serves a batch of requests: request r asks for batch row
// rows[r] at ids[offsets[r] .. offsets[r+1]).  The head activations of the
// requested rows (final RMSNorm + per-row quantize) are made by the same
// kernels as the dense head, so a sparse logit equals the dense logit at
// that id bit for bit.
#include "common.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {

constexpr int kSparseWarps = 8;     // entries per CTA of sparse_head_kernel
constexpr int kSparseMaxK = 4096;   // model dim bound (per-warp chunk sums in shared memory)

// Warp per entry t: logit of vocabulary row ids[t] for the request owning t.
// The int32 dot of each 32-wide group is exact (dp4a over 16-byte chunks,
// two chunks per group); the fold is the I8G32 definition every dense
// kernel follows: acc = fma(half(sw[g]), float(D_g), acc) over ascending g,
// then y = acc * sa.
__global__ void __launch_bounds__(32 * kSparseWarps) sparse_head_kernel(
    const int8_t *__restrict__ w, const uint16_t *__restrict__ sw, int vocab, int k, const int8_t *__restrict__ qa,
    const float *__restrict__ sa, const int32_t *__restrict__ offsets, int n, const int32_t *__restrict__ ids,
    int total, float *__restrict__ out, int *status) {
    pdl_enter();
    __shared__ int chunk_dot[kSparseWarps][kSparseMaxK / 16];
    const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSparseWarps + wi;
    if (t >= total) return;  // the whole warp leaves together
    int lo = 0, hi = n - 1;  // the request: the last r with offsets[r] <= t
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= t)
            lo = mid;
        else
            hi = mid - 1;
    }
    const int r = lo, id = ids[t];
    if (id < 0 || id >= vocab) {  // the host checks ids; kept so a bad id can never read out of bounds
        if (lane == 0) {
            out[t] = 0.0f;
            if (status) atomicOr(status, kStatusBadPage);
        }
        return;
    }
    const int8_t *wr = w + (size_t)id * k, *xr = qa + (size_t)r * k;
    for (int c = lane; c < k / 16; c += 32) {
        const int4 a = *reinterpret_cast<const int4 *>(wr + 16 * c);
        const int4 b = *reinterpret_cast<const int4 *>(xr + 16 * c);
        int d = __dp4a(a.x, b.x, 0);
        d = __dp4a(a.y, b.y, d);
        d = __dp4a(a.z, b.z, d);
        d = __dp4a(a.w, b.w, d);
        chunk_dot[wi][c] = d;
    }
    __syncwarp();
    if (lane == 0) {
        const uint16_t *s = sw + (size_t)id * (k / 32);
        float acc = 0.0f;
        for (int g = 0; g < k / 32; g++)
            acc = fmaf(__half2float(__ushort_as_half(s[g])), __int2float_rn(chunk_dot[wi][2 * g] + chunk_dot[wi][2 * g + 1]),
                       acc);
        out[t] = __fmul_rn(acc, sa[r]);
    }
}

// CTA per request: ArgMaxSparse over values[offsets[r] .. offsets[r+1]) in
// list order (strict '>', so the first position holding the maximum wins;
// -1 when no value exceeds -inf) and p = 1 / sum exp(v - max) over the list
// (BestProbability, Ops.cs:1435-1470; tree sum, so tolerance-equal).
__global__ void __launch_bounds__(256) sparse_argmax_kernel(const float *__restrict__ values,
                                                            const int32_t *__restrict__ offsets,
                                                            const int32_t *__restrict__ ids, int n,
                                                            int32_t *__restrict__ picks, float *__restrict__ probs) {
    pdl_enter();
    __shared__ float s_val[256];
    __shared__ int s_pos[256];
    __shared__ float s_sum[256];
    const int r = blockIdx.x;
    if (r >= n) return;
    const int begin = offsets[r], end = offsets[r + 1];
    float best = -INFINITY;
    int best_pos = -1;
    for (int i = begin + threadIdx.x; i < end; i += blockDim.x) {
        const float v = values[i];
        if (v > best) {
            best = v;
            best_pos = i;
        }
    }
    s_val[threadIdx.x] = best;
    s_pos[threadIdx.x] = best_pos;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = s_val[threadIdx.x + s], mv = s_val[threadIdx.x];
            const int op = s_pos[threadIdx.x + s], mp = s_pos[threadIdx.x];
            if (op >= 0 && (mp < 0 || ov > mv || (ov == mv && op < mp))) {
                s_val[threadIdx.x] = ov;
                s_pos[threadIdx.x] = op;
            }
        }
        __syncthreads();
    }
    const int pos = s_pos[0];
    const float peak = s_val[0];
    float sum = 0.0f;
    if (pos >= 0)
        for (int i = begin + threadIdx.x; i < end; i += blockDim.x) sum += expf(values[i] - peak);
    s_sum[threadIdx.x] = sum;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) s_sum[threadIdx.x] += s_sum[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        picks[r] = pos >= 0 ? ids[pos] : -1;
        if (probs) probs[r] = pos >= 0 ? 1.0f / s_sum[0] : 0.0f;
    }
}

int launch_sparse_head(const int8_t *w, const uint16_t *sw, int vocab, int k, const int8_t *qa, const float *sa,
                       const int32_t *offsets, int n, const int32_t *ids, int total, float *out, int *status,
                       cudaStream_t stream) {
    if (n == 0 || total == 0) return NDL_OK;
    if (k % 32 != 0 || k > kSparseMaxK)
        return set_error(NDL_ERR_UNSUPPORTED, "sparse head: dim %d (a multiple of 32 up to %d)", k, kSparseMaxK);
    launch_kernel(sparse_head_kernel, dim3((unsigned)((total + kSparseWarps - 1) / kSparseWarps)),
                  dim3(32 * kSparseWarps), 0, stream, w, sw, vocab, k, qa, sa, offsets, n, ids, total, out, status);
    return check_launch("sparse_head");
}

int launch_sparse_argmax(const float *values, const int32_t *offsets, const int32_t *ids, int n, int32_t *picks,
                         float *probs, cudaStream_t stream) {
    if (n == 0) return NDL_OK;
    launch_kernel(sparse_argmax_kernel, dim3(n), dim3(256), 0, stream, values, offsets, ids, n, picks, probs);
    return check_launch("sparse_argmax");
}

}  // namespace ndl
