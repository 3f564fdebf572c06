// Paged int8 KV cache: the KV-write epilogue and decode attention.
//
// KV write (src/Needle/Engine.cs:2552-2569): RoPE at the row's absolute
// position (half-split rotation, Scalar.Rope src/Needle/Scalar.cs:233-248),
// then QuantizeInt8 of q per head and of k, v per (position, head) into the
// slot's page.  Bit-exact: round-to-nearest products, no FMA.
//
// Decode attention, bit for bit the reference's AVX2 attention tier
// (Attention.GroupAvx2, src/Needle/Blocks.cs:178-541, on an unsplit tile):
// persistent warps stream (row, head) items from a work list built once per
// step.  Each page's (layer, head) record arrives in shared memory as two
// bulk copies (K half, V half) that the warp issues into its own ring
// (mbarrier completion, bounded waits).  Pass A: the int8 dots on tensor
// cores (mma.sync s8, exact int32), then (dot * ks) * (qs / sqrt(d)) per
// position into a shared score buffer.  Softmax in the reference's order:
// max, e = Ops.Exp(s - max) per position, their total in four partial sums
// by position modulo 4, inverse = 1 / total.  Pass B: w = e * vs, then
// acc[d] = fma(w, v[d], acc[d]) in position order, out = acc * inverse.
// Every rounding is the reference's, so the output is its result exactly.
// A row is never split, so no merge of partials is needed.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "kv.cuh"

namespace ndl {

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int8_t quant1(float x, float inverse) {
    float r = rintf(__fmul_rn(x, inverse));
    return (int8_t)(int)fminf(fmaxf(r, -128.0f), 127.0f);
}

// Quantizes the 64-vector held as (lo = v[lane], hi = v[lane+32]) across the
// warp; returns the scale.
__device__ __forceinline__ float warp_quantize64(float lo, float hi, int8_t &qlo, int8_t &qhi) {
    float peak = warp_max_f(fmaxf(fabsf(lo), fabsf(hi)));
    float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    float inverse = __fdiv_rn(1.0f, scale);
    qlo = quant1(lo, inverse);
    qhi = quant1(hi, inverse);
    return scale;
}

// ------------------------------------------------------------- KV write --
__global__ void __launch_bounds__(256) kv_write_kernel(KvWriteArgs a) {
    pdl_enter();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= a.rows * a.heads) return;
    const int row = warp / a.heads, head = warp - row * a.heads;
    const int pos = a.row_pos[row];
    const int slot = a.row_slot[row];
    const float *base = a.qkv + (size_t)row * a.ld_qkv + head * kHeadDim;
    const int width = a.heads * kHeadDim;
    const float c = a.rope_cos[(size_t)pos * (kHeadDim / 2) + lane];
    const float s = a.rope_sin[(size_t)pos * (kHeadDim / 2) + lane];
    int8_t lo8, hi8;
    // q: RoPE + per-head quantize
    {
        float x0 = base[lane], x1 = base[lane + 32];
        float lo = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float hi = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        float scale = warp_quantize64(lo, hi, lo8, hi8);
        int8_t *qo = a.q8 + ((size_t)row * a.heads + head) * kHeadDim;
        qo[k_slot(lane)] = lo8;
        qo[k_slot(lane + 32)] = hi8;
        if (lane == 0) a.qs[(size_t)row * a.heads + head] = scale;
    }
    const int pg = pos / kPagePositions, j = pos - pg * kPagePositions;
    int page = (pg < a.max_pages) ? a.page_table[(size_t)slot * a.max_pages + pg] : -1;
    bool ok = page >= 0 && page < a.num_pages;
    if (!ok && lane == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    uint8_t *blk = ok ? a.pool + (size_t)page * a.page_bytes + kv_block_offset(a.layer, head, a.heads) : nullptr;
    // k: RoPE + per-(position, head) quantize into the page
    {
        const float *kb = base + width;
        float x0 = kb[lane], x1 = kb[lane + 32];
        float lo = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        float hi = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        float scale = warp_quantize64(lo, hi, lo8, hi8);
        if (ok) {
            blk[k_byte(j, lane)] = (uint8_t)lo8;
            blk[k_byte(j, lane + 32)] = (uint8_t)hi8;
            if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[k_scale_index(j)] = scale;
        }
    }
    // v: per-(position, head) quantize into the page
    {
        const float *vb = base + 2 * width;
        float scale = warp_quantize64(vb[lane], vb[lane + 32], lo8, hi8);
        if (ok) {
            blk[v_byte(j, lane)] = (uint8_t)lo8;
            blk[v_byte(j, lane + 32)] = (uint8_t)hi8;
            if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[v_scale_index(j)] = scale;
        }
    }
}

int launch_kv_write(const KvWriteArgs &a, cudaStream_t stream) {
    int warps = a.rows * a.heads;
    if (warps == 0) return NDL_OK;
    launch_kernel(kv_write_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream, a);
    return check_launch("kv_write");
}

// ------------------------------------------------------- cross attention --
// Queries of the cross-attention block: per (row, head) quantize (no RoPE:
// the memory has no positions) into q8 in k_slot order.  Warp per (row, head).
__global__ void __launch_bounds__(256) cross_query_kernel(const float *__restrict__ q, int ldq, int heads, int rows,
                                                          int8_t *__restrict__ q8, float *__restrict__ qs) {
    pdl_enter();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows * heads) return;
    const int row = warp / heads, head = warp - row * heads;
    const float *src = q + (size_t)row * ldq + head * kHeadDim;
    int8_t lo8, hi8;
    const float scale = warp_quantize64(src[lane], src[lane + 32], lo8, hi8);
    int8_t *qo = q8 + ((size_t)row * heads + head) * kHeadDim;
    qo[k_slot(lane)] = lo8;
    qo[k_slot(lane + 32)] = hi8;
    if (lane == 0) qs[(size_t)row * heads + head] = scale;
}

int launch_cross_query(const float *q, int ldq, int heads, int rows, int8_t *q8, float *qs, cudaStream_t stream) {
    const int warps = rows * heads;
    if (warps == 0) return NDL_OK;
    launch_kernel(cross_query_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream, q, ldq, heads, rows, q8, qs);
    return check_launch("cross_query");
}

// Cross memory of one layer into the pages of a memory slot: y [frames][2*dim]
// holds the projected K | V of every frame; per (frame, head) the 64 K and 64
// V values are quantized (QuantizeInt8, src/Needle/Whistle.cs:789-790) and
// stored at the frame's position like self-attention keys.  Warp per
// (frame, head); page_row = the slot's page-table row.
__global__ void __launch_bounds__(256) cross_kv_write_kernel(const float *__restrict__ y, int frames, int heads,
                                                             const int32_t *__restrict__ page_row, int num_pages,
                                                             uint8_t *__restrict__ pool, long long page_bytes,
                                                             int layer, int *status) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= frames * heads) return;
    const int f = warp / heads, head = warp - f * heads;
    const int dim = heads * kHeadDim;
    const int page = page_row[f / kPagePositions], j = f % kPagePositions;
    if (page < 0 || page >= num_pages) {
        if (lane == 0 && status) atomicOr(status, kStatusBadPage);
        return;
    }
    uint8_t *blk = pool + (size_t)page * page_bytes + kv_block_offset(layer, head, heads);
    const float *kr = y + (size_t)f * 2 * dim + head * kHeadDim, *vr = kr + dim;
    int8_t lo8, hi8;
    float scale = warp_quantize64(kr[lane], kr[lane + 32], lo8, hi8);
    blk[k_byte(j, lane)] = (uint8_t)lo8;
    blk[k_byte(j, lane + 32)] = (uint8_t)hi8;
    if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[k_scale_index(j)] = scale;
    scale = warp_quantize64(vr[lane], vr[lane + 32], lo8, hi8);
    blk[v_byte(j, lane)] = (uint8_t)lo8;
    blk[v_byte(j, lane + 32)] = (uint8_t)hi8;
    if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[v_scale_index(j)] = scale;
}

int launch_cross_kv_write(const float *y, int frames, int heads, const int32_t *page_row, int num_pages, uint8_t *pool,
                          long long page_bytes, int layer, int *status, cudaStream_t stream) {
    const long long warps = (long long)frames * heads;
    if (warps == 0) return NDL_OK;
    cross_kv_write_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(y, frames, heads, page_row, num_pages,
                                                                           pool, page_bytes, layer, status);
    return check_launch("cross_kv_write");
}

// ------------------------------------------------------ decode attention --
constexpr int kAttnWarps = 4;   // warps per CTA; each works its own items
#ifndef NDL_ATTN_STAGES
#define NDL_ATTN_STAGES 3
#endif
constexpr int kAttnStages = NDL_ATTN_STAGES;  // ring stages (half records) per warp
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnPageRegs = kAttnMaxPositions / kPagePositions / 32;  // page ids per lane of an item
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr int kClaimLead = 4;  // pages of pass B left when a warp claims its next item

// Shared memory of one CTA for rows of at most max_pages pages: per warp
// [ring stages][64 PV weights][64 exponentials][stage page flags][scores],
// then the barriers full[warp][stage].
struct AttnSmem {
    int wbuf, ebuf, flags, scores, warp_bytes, bars, total;
};
__host__ __device__ __forceinline__ AttnSmem attn_smem(int max_pages) {
    AttnSmem s;
    s.wbuf = kAttnStages * kKvHalfBytes;
    s.ebuf = s.wbuf + kPagePositions * 4;
    s.flags = s.ebuf + kPagePositions * 4;
    s.scores = s.flags + 16;
    s.warp_bytes = s.scores + max_pages * kPagePositions * 4;
    s.bars = kAttnWarps * s.warp_bytes;
    s.total = s.bars + kAttnWarps * kAttnStages * 8;
    return s;
}

__device__ __forceinline__ void mma_s8s8_m16n8k32(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// The work list: CTA per row position ri of the launch's row order.  An
// out-of-range row (length or slot) gets zero pages, its status bit and NaN
// outputs.  CTA 0 sets the item count and clears the kernel's counters.
__global__ void __launch_bounds__(128) attn_work_kernel(AttnArgs a) {
    pdl_enter();
    const int ri = blockIdx.x;
    int32_t *rec = a.work + (size_t)ri * attn_record_ints(a.max_pages);
    const int row = a.row_order ? a.row_order[ri] : ri;
    const int len = a.row_pos[row] + 1, slot = a.row_slot[row];
    const bool valid = len >= 1 && len <= a.max_pages * kPagePositions && slot >= 0 && slot < a.slots;
    const int pages = valid ? (len + kPagePositions - 1) / kPagePositions : 0;
    if (threadIdx.x == 0) {
        *reinterpret_cast<int4 *>(rec) = make_int4(row, len, slot, pages);
        if (!valid && a.status) atomicOr(a.status, kStatusBadPage);
        if (ri == 0) {
            a.n_work[0] = a.rows * a.heads;
            a.n_work[1] = 0;
            a.n_work[2] = 0;
        }
    }
    for (int t = threadIdx.x; t < pages; t += blockDim.x)
        rec[4 + t] = a.page_table[(size_t)slot * a.max_pages + t];
    if (!valid)
        for (int t = threadIdx.x; t < a.heads * kHeadDim; t += blockDim.x)
            a.out[(size_t)row * a.heads * kHeadDim + t] = __int_as_float(0x7fc00000);
}

// One 16-position chunk of pass B for the lane's two dims: va / vb hold the
// chunk's V bytes of dim lane and lane + 32, w the chunk's 16 weights.
// Each int8 becomes an exact float through its biased byte (v ^ 0x80 as the
// low mantissa byte of 2^23), then acc = fma(w, v, acc) per position in
// order (AccumulateFloat's Fma.MultiplyAdd), both dims in one packed fma.
__device__ __forceinline__ uint64_t pv_chunk(uint64_t acc, const uint4 &va, const uint4 &vb, const float *w) {
    const uint32_t wa[4] = {va.x ^ 0x80808080u, va.y ^ 0x80808080u, va.z ^ 0x80808080u, va.w ^ 0x80808080u};
    const uint32_t wb[4] = {vb.x ^ 0x80808080u, vb.y ^ 0x80808080u, vb.z ^ 0x80808080u, vb.w ^ 0x80808080u};
    const uint64_t bias = f2_pack(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const float4 w4 = *reinterpret_cast<const float4 *>(w + 4 * q);
        const float ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float fa = __uint_as_float(__byte_perm(wa[q], 0x4B000000u, 0x7540u + i));
            const float fb = __uint_as_float(__byte_perm(wb[q], 0x4B000000u, 0x7540u + i));
            const uint64_t v = f2_add(f2_pack(fa, fb), bias);  // exact: both are integers below 2^24
            acc = f2_fma(f2_pack(ww[i], ww[i]), v, acc);
        }
    }
    return acc;
}

// One (row, head) item as a warp holds it in registers: its work record
// (row, attended positions, page count; lane l keeps page ids l, l+32, ...)
// and, once fetched, the query scale and the lane's 16 query bytes.
struct AttnItemRegs {
    int item, row, head, len, pages;
    int page[kAttnPageRegs];
    float qs;
    uint4 q;
};

// The record of `item` (no use of the result yet: the loads stay in flight).
__device__ __forceinline__ void item_fetch_record(const AttnArgs &a, int item, int n_work, int lane,
                                                  AttnItemRegs &it) {
    it.item = item;
    it.pages = 0;
    if (item >= n_work) return;
    const int32_t *rec = a.work + (size_t)(item / a.heads) * attn_record_ints(a.max_pages);
    const int4 h = __ldg(reinterpret_cast<const int4 *>(rec));
    it.head = item % a.heads;
    it.row = h.x;
    it.len = h.y;
    it.pages = h.w;
#pragma unroll
    for (int j = 0; j < kAttnPageRegs; j++) {
        const int idx = lane + 32 * j;
        it.page[j] = idx < a.max_pages ? __ldg(rec + 4 + idx) : -1;
    }
}
// The item's query scale and the lane's query chunk (k_slot chunk tig).
__device__ __forceinline__ void item_fetch_query(const AttnArgs &a, int lane, AttnItemRegs &it) {
    if (it.pages == 0) return;
    const size_t rh = (size_t)it.row * a.heads + it.head;
    it.qs = __ldg(a.qs + rh);
    it.q = __ldg(reinterpret_cast<const uint4 *>(a.q + rh * kHeadDim) + (lane & 3));
}
__device__ __forceinline__ int item_page(const AttnItemRegs &it, int pi) {
    const int j = pi >> 5;
    int v = it.page[0];
#pragma unroll
    for (int r = 1; r < kAttnPageRegs; r++)
        if (j == r) v = it.page[r];
    return __shfl_sync(0xffffffffu, v, pi & 31);
}

// A warp's copy stream: every item's K halves, then its V halves, into the
// warp's ring.  Copies of the current item go out first; those of the next
// item once its record is in registers (`next_ready`), so item boundaries
// overlap.  Lane 0 issues; all lanes keep the counters.
struct AttnStream {
    unsigned issued, consumed;
    int k_cur, k_next;
};
__device__ __forceinline__ void attn_issue(const AttnArgs &a, uint8_t *wsm, int *flags, uint64_t *full,
                                           AttnStream &st, const AttnItemRegs &cur, const AttnItemRegs &nx,
                                           bool next_ready, int lane) {
    while (st.issued - st.consumed < (unsigned)kAttnStages) {
        const bool use_cur = st.k_cur < 2 * cur.pages;  // lane-uniform
        if (!use_cur && !(next_ready && st.k_next < 2 * nx.pages)) break;
        const int k = use_cur ? st.k_cur++ : st.k_next++;
        const int pages = use_cur ? cur.pages : nx.pages, head = use_cur ? cur.head : nx.head;
        const bool v_half = k >= pages;
        const int pi = v_half ? k - pages : k;
        const int page = use_cur ? item_page(cur, pi) : item_page(nx, pi);
        const int stage = st.issued % kAttnStages;
        if (lane == 0) {
            const bool ok = page >= 0 && page < a.num_pages;
            flags[stage] = ok ? 1 : 0;
            if (!ok) {
                if (a.status) atomicOr(a.status, kStatusBadPage);
                mbar_arrive(&full[stage]);  // completes the phase without a copy; the stage holds stale bytes
            } else {
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&full[stage], kKvHalfBytes);
                bulk_g2s(wsm + stage * kKvHalfBytes,
                         a.pool + (size_t)page * a.page_bytes + kv_block_offset(a.layer, head, a.heads) +
                             (v_half ? kKvHalfBytes : 0),
                         kKvHalfBytes, &full[stage]);
            }
        }
        st.issued++;
    }
}

// Persistent warps, each working (row position, head) items of the work list
// (rows longest first, heads innermost): warp w of the grid takes item w
// first, then claims the next unclaimed item from a counter in global memory
// one item ahead, so warps that stream slower take fewer items and the
// launch's warps finish together.  Per item the warp streams 2 * pages half
// records through its 3-stage ring (cp.async.bulk, mbarrier completion,
// bounded waits), every page's K half, then every page's V half:
//  * pass A: the page's K fragments to registers, exact int32 dots on tensor
//    cores (mma.sync m16n8k32 s8, K as A, the query in every B column; lane
//    (gid, tig) keeps positions 16*tig + gid and + 8), then
//    s = (dot * ks) * (qs / sqrt(d)) into the warp's score buffer;
//  * the max over the row's scores;
//  * pass B, page by page: e = Ops.Exp(s - max) for every position, the four
//    partial sums of e by position modulo 4 (lanes 0..3), weights
//    w = e * vs, then acc[d] = fma(w, v[d], acc[d]) in position order, two
//    dims (lane, lane + 32) per lane; at the end out = acc * (1 / total)
//    with total = (s0 + s1) + (s2 + s3).  The total is needed only then, so
//    no separate softmax pass sits between the two.
// The next item's claim, record and query are loaded into registers while
// the current one computes, each used only a phase after its load was issued.
__global__ void __launch_bounds__(kAttnThreads, 3) attn_decode_kernel(AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const AttnSmem L = attn_smem(a.max_pages);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    uint8_t *wsm = smem + (size_t)warp * L.warp_bytes;
    float *wbuf = reinterpret_cast<float *>(wsm + L.wbuf);
    float *ebuf = reinterpret_cast<float *>(wsm + L.ebuf);
    int *flags = reinterpret_cast<int *>(wsm + L.flags);
    float *sc = reinterpret_cast<float *>(wsm + L.scores);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars) + warp * kAttnStages;
    if (lane == 0) {
        for (int i = 0; i < kAttnStages; i++) mbar_init(&full[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    pdl_wait();
    pdl_trigger();
    const int n_work = a.n_work[0];
    int *next_item = a.n_work + 1;
    const int W = gridDim.x * kAttnWarps;
    const int p0 = 16 * tig + gid, p1 = p0 + 8;  // the positions of this lane's two QK results
    const int swz = (lane >> 1) & 3;             // V chunk rotation of dims lane and lane + 32
    AttnStream st{0u, 0u, 0, 0};
    AttnItemRegs cur, nx;
    item_fetch_record(a, blockIdx.x * kAttnWarps + warp, n_work, lane, cur);
    bool query_ready = false;  // cur's query scale and bytes are in registers
    nx.item = n_work;
    nx.pages = 0;
    bool timed_out = false;
    while (cur.item < n_work && !timed_out) {
        if (cur.pages == 0) {  // an out-of-range row: nothing to attend (its outputs are NaN already)
            int claim = 0;
            if (lane == 0) claim = W + atomicAdd(next_item, 1);
            item_fetch_record(a, __shfl_sync(0xffffffffu, claim, 0), n_work, lane, cur);
            query_ready = false;
            st.k_cur = 0;
            continue;
        }
        // The next item is claimed late, kClaimLead pages before the end of pass B, so a warp commits
        // to more work only when its current item is nearly done (claims made at an item's start
        // left the launch's last warps up to a fifth of the kernel behind the others).  Its record
        // is fetched a page after the claim and used a page after that.  Short items claim at the
        // start and fetch the record after pass A.
        const int claim_at = cur.pages >= kClaimLead ? cur.pages - kClaimLead : -1;
        int claim = 0;
        if (claim_at < 0 && lane == 0) claim = W + atomicAdd(next_item, 1);
        bool next_ready = false;
        attn_issue(a, wsm, flags, full, st, cur, nx, next_ready, lane);
        if (!query_ready) item_fetch_query(a, lane, cur);  // lands while the first copies are in flight
        const float scale = __fmul_rn(cur.qs, a.inv_sqrt_d);
        const uint4 qv = cur.q;
        const int len = cur.len, n_pages = cur.pages;
        bool poisoned = false;
        float peak = -INFINITY;
        // ---- pass A: s_j = (dot_j * ks_j) * scale for every position ----
        for (int pg = 0; pg < n_pages; pg++) {
            const int stage = st.consumed % kAttnStages;
            if (!mbar_wait_bounded(&full[stage], (st.consumed / kAttnStages) & 1, kWaitLimit)) {
                timed_out = true;
                break;
            }
            const uint8_t *blk = wsm + stage * kKvHalfBytes;
            uint4 kf[4][2];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                kf[mt][0] = *reinterpret_cast<const uint4 *>(blk + mt * 1024 + lane * 16);
                kf[mt][1] = *reinterpret_cast<const uint4 *>(blk + mt * 1024 + 512 + lane * 16);
            }
            const float2 ks = *reinterpret_cast<const float2 *>(blk + kKScaleOffset + 8 * lane);
            if (!flags[stage]) poisoned = true;
            fence_proxy_async_smem();  // these reads before the stage's next copy
            __syncwarp();
            st.consumed++;
            attn_issue(a, wsm, flags, full, st, cur, nx, next_ready, lane);
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                int d[4] = {0, 0, 0, 0};
                mma_s8s8_m16n8k32(d, kf[mt][0], qv.x, qv.y);
                mma_s8s8_m16n8k32(d, kf[mt][1], qv.z, qv.w);
                if (mt == tig) dot0 = d[0], dot1 = d[2];
            }
            const int valid = min(kPagePositions, len - pg * kPagePositions);
            if (p0 < valid) {
                const float s0 = __fmul_rn(__fmul_rn(__int2float_rn(dot0), ks.x), scale);
                sc[pg * kPagePositions + p0] = s0;
                peak = fmaxf(peak, s0);
            }
            if (p1 < valid) {
                const float s1 = __fmul_rn(__fmul_rn(__int2float_rn(dot1), ks.y), scale);
                sc[pg * kPagePositions + p1] = s1;
                peak = fmaxf(peak, s1);
            }
        }
        if (timed_out) break;
        if (claim_at < 0)  // a short item: the next item's record (the claim has long returned)
            item_fetch_record(a, __shfl_sync(0xffffffffu, claim, 0), n_work, lane, nx);
        peak = warp_max_f(peak);
        __syncwarp();
        if (claim_at < 0) {
            item_fetch_query(a, lane, nx);
            next_ready = true;
        }
        // ---- pass B: per page e = Ops.Exp(s - peak) (ExponentiateAcrossPositions), the four
        // partial sums by position modulo 4 on lanes 0..3 (positions past the last whole quad
        // go to the first, in order), w = e * vs (ValuesFloat), acc[d] = fma(w, v[d], acc[d])
        // (AccumulateFloat) ----
        uint64_t acc = f2_pack(0.0f, 0.0f);  // dims lane, lane + 32
        const int quads = len & ~3;           // positions summed four ways
        float part = 0.0f;                    // lane k < 4: partial sum k
        for (int pg = 0; pg < n_pages; pg++) {
            if (pg == claim_at && lane == 0) claim = W + atomicAdd(next_item, 1);
            if (pg == claim_at + 1) item_fetch_record(a, __shfl_sync(0xffffffffu, claim, 0), n_work, lane, nx);
            if (pg == claim_at + 2) {
                item_fetch_query(a, lane, nx);
                next_ready = true;
            }
            const int stage = st.consumed % kAttnStages;
            if (!mbar_wait_bounded(&full[stage], (st.consumed / kAttnStages) & 1, kWaitLimit)) {
                timed_out = true;
                break;
            }
            const uint8_t *blk = wsm + stage * kKvHalfBytes;  // [V scales][V dim-major]
            const float *vs = reinterpret_cast<const float *>(blk);
            const int valid = min(kPagePositions, len - pg * kPagePositions);
            // positions past the row's end get weight 0: fma(0, v, acc) is acc
            const float e0 = lane < valid ? exp_simd(__fsub_rn(sc[pg * kPagePositions + lane], peak)) : 0.0f;
            const float e1 =
                lane + 32 < valid ? exp_simd(__fsub_rn(sc[pg * kPagePositions + lane + 32], peak)) : 0.0f;
            ebuf[(lane & 3) * 16 + (lane >> 2)] = e0;
            ebuf[(lane & 3) * 16 + 8 + (lane >> 2)] = e1;
            // (the V scales of positions past the row's end are stale page bytes: never multiplied)
            wbuf[lane] = lane < valid ? __fmul_rn(e0, vs[lane]) : 0.0f;
            wbuf[lane + 32] = lane + 32 < valid ? __fmul_rn(e1, vs[lane + 32]) : 0.0f;
            uint4 va[4], vb[4];
#pragma unroll
            for (int ch = 0; ch < 4; ch++) {
                va[ch] = *reinterpret_cast<const uint4 *>(blk + 256 + lane * 64 + ((ch ^ swz) << 4));
                vb[ch] = *reinterpret_cast<const uint4 *>(blk + 256 + (lane + 32) * 64 + ((ch ^ swz) << 4));
            }
            if (!flags[stage]) poisoned = true;
            fence_proxy_async_smem();
            __syncwarp();
            st.consumed++;
            attn_issue(a, wsm, flags, full, st, cur, nx, next_ready, lane);
#pragma unroll
            for (int ch = 0; ch < 4; ch++) acc = pv_chunk(acc, va[ch], vb[ch], wbuf + 16 * ch);
            if (lane < 4) {
                const int base = pg * kPagePositions;
                const float *el = ebuf + lane * 16;  // positions base + 4 i + lane, i ascending
                if (base + kPagePositions <= quads) {
#pragma unroll
                    for (int i = 0; i < 16; i += 4) {
                        const float4 e4 = *reinterpret_cast<const float4 *>(el + i);
                        part = __fadd_rn(part, e4.x);
                        part = __fadd_rn(part, e4.y);
                        part = __fadd_rn(part, e4.z);
                        part = __fadd_rn(part, e4.w);
                    }
                } else {
                    for (int i = 0; i < 16; i++)
                        if (base + 4 * i + lane < quads) part = __fadd_rn(part, el[i]);
                    if (lane == 0)
                        for (int p = max(quads, base); p < base + valid; p++) {
                            const int j = p - base;
                            part = __fadd_rn(part, ebuf[(j & 3) * 16 + (j >> 2)]);
                        }
                }
            }
            __syncwarp();  // the weights and exponentials are read before the next page rewrites them
        }
        if (timed_out) break;
        float *out = a.out + ((size_t)cur.row * a.heads + cur.head) * kHeadDim;
        const float s1 = __shfl_sync(0xffffffffu, part, 1), s2 = __shfl_sync(0xffffffffu, part, 2),
                    s3 = __shfl_sync(0xffffffffu, part, 3);
        const float inverse =
            __shfl_sync(0xffffffffu, __fdiv_rn(1.0f, __fadd_rn(__fadd_rn(part, s1), __fadd_rn(s2, s3))), 0);
        float acc_a, acc_b;
        f2_unpack(acc, acc_a, acc_b);
        const float nan = __int_as_float(0x7fc00000);
        out[lane] = poisoned ? nan : __fmul_rn(acc_a, inverse);
        out[lane + 32] = poisoned ? nan : __fmul_rn(acc_b, inverse);
        // the next item becomes current, with the copies already issued for it
        cur = nx;
        query_ready = true;
        st.k_cur = st.k_next;
        st.k_next = 0;
        nx.item = n_work;
        nx.pages = 0;
    }
    if (timed_out) {
        if (lane == 0 && a.status) atomicOr(a.status, kStatusTimeout);
        // every copy in flight lands before the warp exits (bounded)
        for (unsigned j = st.consumed; j < st.issued; j++)
            mbar_wait_bounded(&full[j % kAttnStages], (j / kAttnStages) & 1, kWaitLimit);
    }
    // the last CTA out resets the item counter and the finish count for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.n_work + 2, 1) == (int)gridDim.x - 1) {
            a.n_work[1] = 0;
            a.n_work[2] = 0;
            __threadfence();
        }
    }
}

// The per-row quantize of the attention output (the o-projection's input):
// CTA per row, warp per head; the row peak (exact max of |x| over heads x 64)
// goes through shared memory; scale, inverse and rounding as
// Scalar.QuantizeInt8 (src/Needle/Scalar.cs:67-74).
__global__ void __launch_bounds__(1024) attn_quantize_kernel(AttnArgs a) {
    pdl_enter();
    __shared__ float head_peak[32];
    const int row = blockIdx.x, head = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float2 v = *reinterpret_cast<const float2 *>(a.out + ((size_t)row * a.heads + head) * kHeadDim + 2 * lane);
    const float hp = warp_max_f(fmaxf(fabsf(v.x), fabsf(v.y)));
    if (lane == 0) head_peak[head] = hp;
    __syncthreads();
    float peak = 0.0f;
    for (int h = 0; h < a.heads; h++) peak = fmaxf(peak, head_peak[h]);
    const float scale = peak > 0.0f ? __fdiv_rn(peak, 127.0f) : 1.0f;
    const float inverse = __fdiv_rn(1.0f, scale);
    const uint32_t b0 = (uint8_t)quant1(v.x, inverse), b1 = (uint8_t)quant1(v.y, inverse);
    reinterpret_cast<uint16_t *>(a.q_out + (size_t)row * a.heads * kHeadDim)[head * 32 + lane] =
        (uint16_t)(b0 | (b1 << 8));
    if (threadIdx.x == 0) a.s_out[row] = scale;
}

int launch_attn_work(const AttnArgs &a, cudaStream_t stream) {
    if (a.rows == 0) return NDL_OK;
    if (!a.work || !a.n_work) return set_error(NDL_ERR_INVALID_ARG, "attention: no work list");
    launch_kernel(attn_work_kernel, dim3(a.rows), dim3(128), 0, stream, a);
    return check_launch("attn_work");
}

int launch_attn_quantize(const AttnArgs &a, cudaStream_t stream) {
    if (a.rows == 0 || !a.q_out) return NDL_OK;
    if (a.heads > 32) return set_error(NDL_ERR_INVALID_ARG, "attention: %d heads > 32", a.heads);
    launch_kernel(attn_quantize_kernel, dim3(a.rows), dim3(a.heads * 32), 0, stream, a);
    return check_launch("attn_quantize");
}

// CTAs of attn_decode_kernel that fit one SM at this shared-memory size,
// cached per device and size.
static int attn_ctas_per_sm(size_t smem) {
    struct Entry {
        int dev;
        size_t smem;
        int ctas;
    };
    static std::mutex mutex;
    static Entry cache[32];
    static int used = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 1;
    std::lock_guard<std::mutex> lock(mutex);
    for (int i = 0; i < used; i++)
        if (cache[i].dev == dev && cache[i].smem == smem) return cache[i].ctas;
    int ctas = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, attn_decode_kernel, kAttnThreads, smem) != cudaSuccess ||
        ctas < 1)
        ctas = 1;
    if (used < 32) cache[used++] = Entry{dev, smem, ctas};
    return ctas;
}

int launch_attn_decode(const AttnArgs &a, cudaStream_t stream, bool build_work, bool quantize) {
    if (a.rows == 0) return NDL_OK;
    if (a.max_pages < 1 || a.max_pages * kPagePositions > kAttnMaxPositions)
        return set_error(NDL_ERR_UNSUPPORTED, "attention: %d pages per row (at most %d positions)", a.max_pages,
                         kAttnMaxPositions);
    static DeviceOnce smem_attribute;  // the attribute belongs to the kernel on one device
    int st0 = smem_attribute.run([] {
        int dev = 0, optin = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
        return (int)NDL_OK;
    });
    if (st0 != NDL_OK) return st0;
    const size_t smem = (size_t)attn_smem(a.max_pages).total;
    const long long items = (long long)a.rows * a.heads;
    if (items > 0x7FFFFFFF) return set_error(NDL_ERR_INVALID_ARG, "attention: too many work items");
    if (build_work) {
        int st = launch_attn_work(a, stream);
        if (st != NDL_OK) return st;
    }
    long long blocks = (items + kAttnWarps - 1) / kAttnWarps;
    const long long resident = (long long)device_sm_count() * attn_ctas_per_sm(smem);
    if (blocks > resident) blocks = resident;
    launch_kernel(attn_decode_kernel, dim3((unsigned)blocks), dim3(kAttnThreads), smem, stream, a);
    int st = check_launch("attn_decode");
    if (st != NDL_OK || !quantize) return st;
    return launch_attn_quantize(a, stream);
}

}  // namespace ndl

using namespace ndl;

// Workspace: the work list [rows][attn_record_ints(max_pages)] int32 and 16
// bytes for the item count and the decode kernel's two counters.
extern "C" NDL_API size_t ndl_attention_paged_workspace(int rows, int heads, int max_pages) {
    if (rows <= 0 || heads <= 0 || max_pages <= 0) return 0;
    return (size_t)rows * attn_record_ints(max_pages) * sizeof(int32_t) + 16;
}

// Points a.work and a.n_work into a workspace of that layout.
static void abi_carve(AttnArgs &a, void *ws, int rows, int max_pages) {
    uint8_t *base = static_cast<uint8_t *>(ws);
    a.work = reinterpret_cast<int32_t *>(base);
    a.n_work = reinterpret_cast<int *>(base + (size_t)rows * attn_record_ints(max_pages) * sizeof(int32_t));
}

static int abi_check(const int8_t *q, const float *qs, const int32_t *row_slot, const int32_t *row_pos, int rows,
                     int heads, const int32_t *page_table, int slots, int max_pages, const uint8_t *pool,
                     size_t page_bytes, int num_pages, int layer, float *out) {
    NDL_REQUIRE(rows >= 0 && heads >= 1 && slots >= 1 && max_pages >= 1 && num_pages >= 1 && layer >= 0,
                "bad attention geometry");
    if (rows == 0) return NDL_OK;
    NDL_REQUIRE(q && qs && row_slot && row_pos && page_table && pool && out, "null pointer");
    NDL_REQUIRE(page_bytes % 16 == 0 && page_bytes >= kv_block_offset(layer, heads - 1, heads) + kKvBlockBytes,
                "page_bytes %zu cannot hold layer %d of %d heads", page_bytes, layer, heads);
    NDL_REQUIRE(aligned(q, 16) && aligned(pool, 16) && aligned(out, 16) && aligned(qs, 4), "misaligned pointer");
    if ((long long)max_pages * kPagePositions > kAttnMaxPositions)
        return set_error(NDL_ERR_UNSUPPORTED, "attention: %d pages per row; at most %d positions", max_pages,
                         kAttnMaxPositions);
    return NDL_OK;
}

extern "C" NDL_API int ndl_attention_paged(const int8_t *q, const float *qs, const int32_t *row_slot,
                                           const int32_t *row_pos, int rows, int heads, const int32_t *page_table,
                                           int slots, int max_pages, const uint8_t *pool, size_t page_bytes,
                                           int num_pages, int layer, float *out, void *workspace,
                                           size_t workspace_bytes, int *status, void *stream) {
    int rc = abi_check(q, qs, row_slot, row_pos, rows, heads, page_table, slots, max_pages, pool, page_bytes,
                       num_pages, layer, out);
    if (rc != NDL_OK || rows == 0) return rc;
    const size_t need = ndl_attention_paged_workspace(rows, heads, max_pages);
    cudaStream_t st = (cudaStream_t)stream;
    void *ws = workspace;
    if (ws) {
        NDL_REQUIRE(workspace_bytes >= need && aligned(ws, 16), "workspace of %zu bytes, %zu needed",
                    workspace_bytes, need);
    } else {
        NDL_CUDA(cudaMallocAsync(&ws, need, st));
    }
    AttnArgs a{q, qs, row_slot, row_pos, nullptr, page_table, max_pages, pool, (long long)page_bytes, num_pages,
               layer, heads, rows, 0.125f, out, status, slots, nullptr, nullptr, nullptr, nullptr};
    abi_carve(a, ws, rows, max_pages);
    rc = launch_attn_decode(a, st);
    if (!workspace) cudaFreeAsync(ws, st);
    return rc;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of ndl_attention_paged.
//
// Some hosts must not allocate memory while they serve a request: a game
// loop or job-system worker on a frame budget, an audio callback, or the
// reference's host worker, whose steady-state calls are held to zero
// allocations.  cudaMalloc can block for a long time, serialises on a
// driver-wide lock and can synchronise the device, so such callers cannot
// supply the workspace ndl_attention_paged needs, nor let it allocate one.
// This entry point keeps the work list (and the kernel's counters) in a
// fixed device array that the library owns instead.
//
// The array is a file-scope __device__ variable, so every GPU that loads
// this library holds its kNoAllocScratchBytes until the process exits.  On
// the host its name is only a stand-in: the real device address is looked
// up once per device with cudaGetSymbolAddress, the first time the entry
// point is called on that device (with that device current), and cached.
// Make that first call before any stream capture starts.
//
// Every call shares the one array.  Nothing in it has to start at zero: a
// launch's first kernel writes every work record and clears the counters
// before the attention kernel reads them.  Two calls whose work overlaps on
// the GPU (different streams, or no ordering between them) race on the
// array and can corrupt each other's results; callers must order them, for
// example by issuing them on one stream.
// ---------------------------------------------------------------------------
namespace {

// 4 MiB: a work record of 16 bytes plus 4 per page-table column (rounded up
// to 16) per row, plus 16 bytes of counters; 512 rows fit at any supported
// page-table width (at most 128 pages).
constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void *g_noalloc_address[kNoAllocMaxDevices];

// Device address of the scratch array on the current device (set-up on
// first use per device).
int noalloc_scratch(void **out) {
    int dev = 0;
    NDL_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(NDL_ERR_UNSUPPORTED, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_address[dev]) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return set_error(NDL_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        g_noalloc_address[dev] = ptr;
    }
    *out = g_noalloc_address[dev];
    return NDL_OK;
}

}  // namespace

extern "C" NDL_API int ndl_attention_paged_noalloc(const int8_t *q, const float *qs, const int32_t *row_slot,
                                                   const int32_t *row_pos, int rows, int heads,
                                                   const int32_t *page_table, int slots, int max_pages,
                                                   const uint8_t *pool, size_t page_bytes, int num_pages, int layer,
                                                   float *out, int *status, void *stream) {
    int rc = abi_check(q, qs, row_slot, row_pos, rows, heads, page_table, slots, max_pages, pool, page_bytes,
                       num_pages, layer, out);
    if (rc != NDL_OK || rows == 0) return rc;
    const size_t need = ndl_attention_paged_workspace(rows, heads, max_pages);
    if (need > kNoAllocScratchBytes)
        return set_error(NDL_ERR_INVALID_ARG,
                         "%d rows x %d pages need %zu bytes of scratch; the built-in buffer holds %zu", rows,
                         max_pages, need, kNoAllocScratchBytes);
    void *scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc != NDL_OK) return rc;
    AttnArgs a{q, qs, row_slot, row_pos, nullptr, page_table, max_pages, pool, (long long)page_bytes, num_pages,
               layer, heads, rows, 0.125f, out, status, slots, nullptr, nullptr, nullptr, nullptr};
    abi_carve(a, scratch, rows, max_pages);
    return launch_attn_decode(a, (cudaStream_t)stream);
}
