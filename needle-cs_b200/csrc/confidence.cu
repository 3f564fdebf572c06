// The Needle-3 confidence head on the device: probe pooling over the
// decoded tokens (EngineCore.PoolTokensBatch, src/Needle/Engine.cs:2598-2650)
// and the per-slot confidence logit (ConfidenceLogitForSlot, :2702-2738).
//
// Each slot keeps, per pool row (layer row x probe), an online softmax over
// its tokens: the peak score, the sum of exp(score - peak) and the
// exp-weighted sum of the token cells; the cell is the mean of the token's 4
// hyper-connection streams (stream 0 for the first token of an initial
// batch).  The logit attends, per query, over the pooled means (RMS-unit,
// gained, with a row bias) and projects the pooled queries.  State lives in
// caller-owned device arrays; the reference's snapshot / restore after a
// rewind is the optional snapshot arrays and per-slot pending flags.  Sums run
// in the scalar code's order and MathF.Exp is the correctly rounded
// exponential (exp_rn), so the results equal the scalar code's bit for bit.
#include "common.cuh"
#include "kernels.cuh"

namespace ndl {

struct ConfPoolArgs {
    int row;
    const float *streams;  // [count][4][dim]
    const int32_t *row_slots;
    int count, initial;
    const float *probes_v;  // [pool_rows][dim]
    int probes, dim, pool_rows, slots;
    float *cell, *pool_max, *pool_sum, *pool_acc;
    const float *snap_max, *snap_sum, *snap_acc;
    const uint8_t *pending;
};

// Block per (token, probe); only a run's first token works, walking its run.
__global__ void __launch_bounds__(256) conf_pool_kernel(ConfPoolArgs a) {
    extern __shared__ float cs[];  // cell [dim]
    __shared__ float factor;
    __shared__ int grow;
    pdl_enter();
    const int rs = blockIdx.x, p = blockIdx.y;
    const int slot = a.row_slots[rs];
    if (rs > 0 && a.row_slots[rs - 1] == slot) return;
    if (slot < 0 || slot >= a.slots) return;
    int rk = rs;
    while (rk + 1 < a.count && a.row_slots[rk + 1] == slot) rk++;
    const int dim = a.dim, index = a.row * a.probes + p;
    const size_t at = (size_t)slot * a.pool_rows + index;
    float *acc = a.pool_acc + at * dim;
    const float *probe = a.probes_v + (size_t)index * dim;
    const float inverse_root = __fdiv_rn(1.0f, __fsqrt_rn((float)dim));
    if (a.pending && a.pending[slot]) {
        for (int i = threadIdx.x; i < dim; i += blockDim.x) acc[i] = a.snap_acc[at * dim + i];
        if (threadIdx.x == 0) {
            a.pool_max[at] = a.snap_max[at];
            a.pool_sum[at] = a.snap_sum[at];
        }
    }
    __syncthreads();
    for (int t = rs; t <= rk; t++) {
        const float *st = a.streams + (size_t)t * 4 * dim;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) {
            if (a.initial && t == rs) {
                cs[i] = st[i];
            } else {
                float m = __fadd_rn(__fmul_rn(0.25f, st[i]), __fmul_rn(0.25f, st[dim + i]));
                m = __fadd_rn(m, __fmul_rn(0.25f, st[2 * dim + i]));
                cs[i] = __fadd_rn(m, __fmul_rn(0.25f, st[3 * dim + i]));
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float dot = 0.0f;
            for (int i = 0; i < dim; i++) dot = __fadd_rn(dot, __fmul_rn(cs[i], probe[i]));
            const float score = __fmul_rn(dot, inverse_root);
            const float mx = a.pool_max[at];
            if (score > mx) {
                const float rescale = exp_rn(__fsub_rn(mx, score));
                a.pool_sum[at] = __fadd_rn(__fmul_rn(a.pool_sum[at], rescale), 1.0f);
                a.pool_max[at] = score;
                factor = rescale;
                grow = 1;
            } else {
                const float weight = exp_rn(__fsub_rn(score, mx));
                a.pool_sum[at] = __fadd_rn(a.pool_sum[at], weight);
                factor = weight;
                grow = 0;
            }
        }
        __syncthreads();
        const float f = factor;
        if (grow)
            for (int i = threadIdx.x; i < dim; i += blockDim.x) acc[i] = __fadd_rn(__fmul_rn(f, acc[i]), cs[i]);
        else
            for (int i = threadIdx.x; i < dim; i += blockDim.x) acc[i] = __fadd_rn(acc[i], __fmul_rn(f, cs[i]));
        __syncthreads();
    }
    if (p == 0)
        for (int i = threadIdx.x; i < dim; i += blockDim.x) a.cell[(size_t)slot * dim + i] = cs[i];
}

struct ConfLogitArgs {
    const int32_t *slot_list;
    int n;
    const float *pool_sum, *pool_acc;
    int pool_rows, dim;
    const float *gain, *query_vectors, *row_bias;
    float bias;
    const float *projection;
    int queries;
    float *logits, *pooled_out;
};

// Block per listed slot; shared memory holds the row keys [pool_rows][dim],
// the pooled queries [queries][dim] and the weights [pool_rows].
__global__ void __launch_bounds__(256) conf_logit_kernel(ConfLogitArgs a) {
    extern __shared__ float sm[];
    pdl_enter();
    const int r = blockIdx.x, slot = a.slot_list[r], rows = a.pool_rows, dim = a.dim;
    float *v = sm, *pooled = v + (size_t)rows * dim, *w = pooled + (size_t)a.queries * dim;
    const float *sum = a.pool_sum + (size_t)slot * rows, *acc = a.pool_acc + (size_t)slot * rows * dim;
    const float inverse_root = __fdiv_rn(1.0f, __fsqrt_rn((float)dim));
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {  // thread per row, in the scalar order
        float *vi = v + (size_t)i * dim;
        const float inv_sum = __fdiv_rn(1.0f, sum[i]);
        float ss = 0.0f;
        for (int k = 0; k < dim; k++) {
            vi[k] = __fadd_rn(0.0f, __fmul_rn(inv_sum, acc[(size_t)i * dim + k]));
            ss = __fadd_rn(ss, __fmul_rn(vi[k], vi[k]));
        }
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)dim), 1e-6f)));
        for (int k = 0; k < dim; k++) {
            const float u = __fmul_rn(vi[k], inv);
            vi[k] = __fadd_rn(__fmul_rn(a.gain[i], u), __fmul_rn(0.0f, u));
        }
    }
    __syncthreads();
    for (int q = 0; q < a.queries; q++) {
        const float *qv = a.query_vectors + (size_t)q * dim;
        for (int i = threadIdx.x; i < rows; i += blockDim.x) {
            float d = 0.0f;
            for (int k = 0; k < dim; k++) d = __fadd_rn(d, __fmul_rn(v[(size_t)i * dim + k], qv[k]));
            w[i] = __fadd_rn(__fmul_rn(d, inverse_root), a.row_bias[q * rows + i]);
        }
        __syncthreads();
        if (threadIdx.x == 0) {  // Softmax over the rows
            float peak = -INFINITY, total = 0.0f;
            for (int i = 0; i < rows; i++) peak = fmaxf(peak, w[i]);
            for (int i = 0; i < rows; i++) {
                w[i] = exp_rn(__fsub_rn(w[i], peak));
                total = __fadd_rn(total, w[i]);
            }
            for (int i = 0; i < rows; i++) w[i] = __fdiv_rn(w[i], total);
        }
        __syncthreads();
        for (int k = threadIdx.x; k < dim; k += blockDim.x) {
            float s = 0.0f;
            for (int i = 0; i < rows; i++) s = __fadd_rn(s, __fmul_rn(w[i], v[(size_t)i * dim + k]));
            pooled[(size_t)q * dim + k] = s;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float d = 0.0f;
        for (int k = 0; k < a.queries * dim; k++) d = __fadd_rn(d, __fmul_rn(pooled[k], a.projection[k]));
        a.logits[r] = __fadd_rn(a.bias, d);
    }
    if (a.pooled_out)
        for (int k = threadIdx.x; k < a.queries * dim; k += blockDim.x)
            a.pooled_out[(size_t)r * a.queries * dim + k] = pooled[k];
}

}  // namespace ndl

using namespace ndl;

extern "C" NDL_API int ndl_conf_pool_update(int row, const float *streams, const int32_t *row_slots, int count,
                                            int initial, const float *probe_vectors, int probes, int dim,
                                            int pool_rows, int slots, float *cell, float *pool_max, float *pool_sum,
                                            float *pool_acc, const float *snap_max, const float *snap_sum,
                                            const float *snap_acc, const uint8_t *pending, void *stream) {
    NDL_REQUIRE(count >= 0 && probes >= 1 && dim >= 1 && slots >= 1, "count %d / probes %d / dim %d / slots %d", count,
                probes, dim, slots);
    NDL_REQUIRE(row >= 0 && (row + 1) * probes <= pool_rows, "row %d of %d probes outside %d pool rows", row, probes,
                pool_rows);
    NDL_REQUIRE((size_t)dim * 4 <= 48 * 1024, "dim %d too large", dim);
    if (count == 0) return NDL_OK;
    NDL_REQUIRE(streams && row_slots && probe_vectors && cell && pool_max && pool_sum && pool_acc, "null pointer");
    NDL_REQUIRE(!pending || (snap_max && snap_sum && snap_acc), "pending flags need the snapshot arrays");
    ConfPoolArgs a{row, streams, row_slots, count, initial, probe_vectors, probes, dim, pool_rows, slots, cell,
                   pool_max, pool_sum, pool_acc, snap_max, snap_sum, snap_acc, pending};
    launch_kernel(conf_pool_kernel, dim3((unsigned)count, (unsigned)probes), dim3(256), (size_t)dim * 4,
                  (cudaStream_t)stream, a);
    return check_launch("conf_pool");
}

extern "C" NDL_API int ndl_conf_logit(const int32_t *slot_list, int n, const float *pool_sum, const float *pool_acc,
                                      int pool_rows, int dim, const float *gain, const float *query_vectors,
                                      const float *row_bias, float bias, const float *projection, int queries,
                                      float *logits, float *pooled_out, void *stream) {
    NDL_REQUIRE(n >= 0 && pool_rows >= 1 && dim >= 1 && queries >= 1, "n %d / rows %d / dim %d / queries %d", n,
                pool_rows, dim, queries);
    const size_t smem = ((size_t)pool_rows * dim + (size_t)queries * dim + pool_rows) * 4;
    NDL_REQUIRE(smem <= 200 * 1024, "%d rows x %d dims do not fit one block's shared memory", pool_rows, dim);
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(slot_list && pool_sum && pool_acc && gain && query_vectors && row_bias && projection && logits,
                "null pointer");
    cudaError_t e = cudaFuncSetAttribute(conf_logit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "conf_logit smem attribute: %s", cudaGetErrorString(e));
    ConfLogitArgs a{slot_list, n, pool_sum, pool_acc, pool_rows, dim, gain, query_vectors, row_bias, bias,
                    projection, queries, logits, pooled_out};
    launch_kernel(conf_logit_kernel, dim3((unsigned)n), dim3(256), smem, (cudaStream_t)stream, a);
    return check_launch("conf_logit");
}
