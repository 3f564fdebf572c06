// Paged int8 KV cache: the KV-write epilogue and split-K decode attention.
//
// KV write (src/Needle/Engine.cs:2552-2569): RoPE at the row's absolute
// position (half-split rotation, Scalar.Rope src/Needle/Scalar.cs:233-248),
// then QuantizeInt8 of q per head and of k, v per (position, head) into the
// slot's page.  Bit-exact: round-to-nearest products, no FMA.
//
// Decode attention (Scalar.AttentionHead src/Needle/Scalar.cs:290-312,
// AttentionBatch.ExecuteChunk + MergePartials src/Needle/Blocks.cs:750-990):
// persistent warps stream (row, head, chunk of pages) items from a work list
// built once per step.  Each page's 8704-byte (layer, head) record arrives
// in shared memory by one cp.async.bulk, issued by a producer warp into a
// 3-stage ring per consumer warp (mbarrier completion, bounded waits).
// Scores are exact int8 dots (mma.sync s8) scaled by ks * (qs / sqrt(d));
// softmax is online (running max, rescaled sum) in fp32 with expf; V is
// accumulated exactly by mma.sync s8 x u8 over 24-bit fixed-point
// probability weights.  A row longer than one chunk (a fixed number of
// pages, so the split depends only on the row's own length) writes (peak,
// sum, unnormalised output) partials that attn_merge_kernel combines with
// exp(peak - max) weights, like MergePartials.
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
            if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[scale_slot(j)] = scale;
        }
    }
    // v: per-(position, head) quantize into the page
    {
        const float *vb = base + 2 * width;
        float scale = warp_quantize64(vb[lane], vb[lane + 32], lo8, hi8);
        if (ok) {
            blk[v_byte(j, lane)] = (uint8_t)lo8;
            blk[v_byte(j, lane + 32)] = (uint8_t)hi8;
            if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[scale_slot(j)] = scale;
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
    if (lane == 0) reinterpret_cast<float *>(blk + kKScaleOffset)[scale_slot(j)] = scale;
    scale = warp_quantize64(vr[lane], vr[lane + 32], lo8, hi8);
    blk[v_byte(j, lane)] = (uint8_t)lo8;
    blk[v_byte(j, lane + 32)] = (uint8_t)hi8;
    if (lane == 0) reinterpret_cast<float *>(blk + kVScaleOffset)[scale_slot(j)] = scale;
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
constexpr int kAttnConsumers = 4;  // consumer warps per CTA; warp 4 is the producer
constexpr int kAttnStages = 3;     // ring stages per consumer
constexpr int kAttnThreads = 32 * (kAttnConsumers + 1);
constexpr int kAttnCtasPerSm = 2;  // 2 x 4 consumers x 3 stages x 8.7 KB = 209 KB of ring per SM
// Per-stage item header, written by the producer with the first page of an
// item: {row, head | chunk << 16, len, pages | chunks << 16} (row -1 = the
// list ended), the query scale at byte 16 and the 64 query bytes at byte 32.
// Every page also sets the int at byte 24: 1 if its copy was issued, 0 if
// its page id was outside the pool (the stage then holds stale bytes).
constexpr int kAttnHdrBytes = 96;
constexpr int kAttnHdrOffset = kAttnStages * kKvBlockBytes + 256;
// then the producer's landing slot for the consumer's next work-list record
constexpr int kAttnEntryOffset = kAttnHdrOffset + kAttnStages * kAttnHdrBytes;
constexpr int kConsumerSmem = kAttnEntryOffset + (int)sizeof(AttnWork);  // ring, digits, headers, record
static_assert(kConsumerSmem % 16 == 0 && kAttnEntryOffset % 16 == 0, "bulk copy destinations");
constexpr int kAttnBarOffset = kAttnConsumers * kConsumerSmem;  // full[c][s], empty[c][s], record[c]
constexpr int kAttnSmem = kAttnBarOffset + (2 * kAttnConsumers * kAttnStages + kAttnConsumers) * 8;
// A producer lane reads the result of its item claim (an atomic) and of a
// query-scale load only this many SM cycles after issuing them, so the
// warp's other lanes are not held on the load's scoreboard.
constexpr long long kAttnLatencyCycles = 1000;
// int32 PV accumulators gain at most 64 * 255 * 128 per page; flushing to
// fp32 every 1024 pages keeps them below 2^31.
constexpr int kHoldPages = 1024;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kPollLimit = 1u << 24;  // producer polls without progress (with a short sleep each)

// Work item i = (row in LPT order, head, chunk) with chunk innermost.
struct AttnItem {
    int row, head, chunk, n_chunks, first_page, n_pages, len, slot;
};

__device__ __forceinline__ bool attn_item(const AttnArgs &a, int i, AttnItem &it) {
    const int chunk = i % a.max_chunks;
    const int rh = i / a.max_chunks;
    it.head = rh % a.heads;
    const int ri = rh / a.heads;
    it.row = a.row_order ? a.row_order[ri] : ri;
    it.len = a.row_pos[it.row] + 1;
    it.slot = a.row_slot[it.row];
    if (it.len < 1 || it.len > a.max_pages * kPagePositions || it.slot < 0 || it.slot >= a.slots) {
        if (a.status) atomicOr(a.status, kStatusBadPage);  // out-of-range row: skipped
        return false;
    }
    const int pages = (it.len + kPagePositions - 1) / kPagePositions;
    it.n_chunks = (pages + a.chunk_pages - 1) / a.chunk_pages;
    if (chunk >= it.n_chunks) return false;
    it.chunk = chunk;
    it.first_page = chunk * a.chunk_pages;
    it.n_pages = min(pages, it.first_page + a.chunk_pages) - it.first_page;
    return true;
}

__device__ __forceinline__ void mma_s8s8_m16n8k32(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8u8_m16n8k32(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

__device__ __forceinline__ AttnWork attn_work_of(const AttnArgs &a, const AttnItem &it) {
    AttnWork w;
    w.row = it.row;
    w.head_chunk = it.head | (it.chunk << 16);
    w.len = it.len;
    w.pages_chunks = it.n_pages | (it.n_chunks << 16);
#pragma unroll
    for (int k = 0; k < kAttnMaxChunkPages; k++)
        w.page[k] = k < it.n_pages ? a.page_table[(size_t)it.slot * a.max_pages + it.first_page + k] : -1;
    return w;
}

// The compacted work list: CTA per row position ri of the LPT order.  Its
// items (head, chunk innermost) start after the items of rows 0..ri-1, so
// the CTA first sums those rows' chunk counts, then writes its own items
// with their page ids.
__global__ void __launch_bounds__(256) attn_work_kernel(AttnArgs a) {
    pdl_enter();
    __shared__ int warp_sum[8];
    const int ri = blockIdx.x;
    auto chunks_of = [&](int r) -> int {  // 0 for an out-of-range row
        const int row = a.row_order ? a.row_order[r] : r;
        const int len = a.row_pos[row] + 1, slot = a.row_slot[row];
        if (len < 1 || len > a.max_pages * kPagePositions || slot < 0 || slot >= a.slots) return 0;
        const int pages = (len + kPagePositions - 1) / kPagePositions;
        return (pages + a.chunk_pages - 1) / a.chunk_pages;
    };
    int part = 0;
    for (int r = threadIdx.x; r < ri; r += blockDim.x) part += chunks_of(r);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = part;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) before += warp_sum[w];
    const int base = a.heads * before;
    const int nc = chunks_of(ri);
    const int items = a.heads * nc;
    AttnItem it;
    if (nc == 0) {  // an out-of-range row: no items, status recorded, NaN output
        if (threadIdx.x == 0) attn_item(a, ri * a.heads * a.max_chunks, it);
        const int row = a.row_order ? a.row_order[ri] : ri;
        for (int t = threadIdx.x; t < a.heads * kHeadDim; t += blockDim.x)
            a.out[(size_t)row * a.heads * kHeadDim + t] = __int_as_float(0x7fc00000);
    }
    for (int t = threadIdx.x; t < items; t += blockDim.x) {
        const int head = t / nc, chunk = t - head * nc;
        if (attn_item(a, (ri * a.heads + head) * a.max_chunks + chunk, it)) a.work[base + t] = attn_work_of(a, it);
    }
    if (ri == a.rows - 1 && threadIdx.x == 0) {
        a.n_work[0] = base + items;
        a.n_work[1] = 0;  // the decode kernel's item counter and finish count
        a.n_work[2] = 0;
    }
}

// Persistent, warp-specialised.  The work list (rows sorted longest first,
// heads and chunks of a row adjacent) is dealt dynamically: consumer warp w
// takes item w first (its record and query scale loaded directly, as nothing
// is in flight yet to hide them behind); after that, whenever its producer lane starts
// issuing an item it claims the next unclaimed one from a counter in global
// memory.  Warps that stream slower (the rate differs by SM and over time)
// so take fewer items and the launch's warps finish together; claiming one
// item ahead keeps the claims in step with progress.
// Lane c of the producer warp feeds consumer c of its CTA.  It runs a small
// state machine per lane so that no lane's latency holds the warp: claim
// (atomic; its result read kAttnLatencyCycles later), fetch the item's
// 48-byte record into shared memory (cp.async.bulk, completion polled on
// its own mbarrier), load the query scale (read kAttnLatencyCycles later).
// It issues the consumer's page copies (one cp.async.bulk per 8704-byte
// page record) into the consumer's 3-stage ring as stages free up; with an
// item's first page it writes the item header (metadata, query scale) into
// the stage and copies the 64 query bytes beside it, so a consumer never
// loads metadata from global memory.
// A consumer waits for a page, moves its K and V^T fragments and scales to
// registers, frees the stage and computes, all products on int8 tensor cores:
//  * QK: mma.sync m16n8k32 s8, A = K (16 positions x 32 dims), B = the
//    query in every column: exact int32 dots.  Lane (gid, tig) keeps tile
//    tig, i.e. positions 16*tig + gid and 16*tig + gid + 8.
//  * PV: the weights w' = p * vs * 2^e (e keeps w' below 2^12, folded into
//    the online-softmax rescale) become 24-bit fixed point W = w' * 2^12,
//    split into three unsigned byte digits.  mma.sync m16n8k32 s8 x u8 with
//    A = V^T (16 dims x 32 positions) and B = the digits (column = digit)
//    gives exact int32 sums of digit x v, chained across pages in the
//    accumulator until the softmax rescale changes; the digits recombine
//    as D0 * 2^16 + D1 * 2^8 + D2 once per item.
// Every wait and the producer's polling are bounded.  The last CTA to finish
// returns the counters to zero for the next launch on the same list.
__device__ __forceinline__ void attn_producer(const AttnArgs &a, uint8_t *smem, uint64_t *full, uint64_t *empty,
                                              uint64_t *record_bar, int lane) {
    const int W = gridDim.x * kAttnConsumers;
    const int c = lane;
    const int n_work = a.n_work[0];
    int *next_item = a.n_work + 1;
    enum { kClaimed, kFetching, kScale, kReady, kExhausted };
    bool done = c >= kAttnConsumers, ending = false;
    uint8_t *record = smem + c * kConsumerSmem + kAttnEntryOffset;
    AttnWork cur{}, nx{};
    float qs_cur = 0.0f, qs_nx = 0.0f;
    int fs = kClaimed, claim = blockIdx.x * kAttnConsumers + c;  // the first item is this warp's own
    long long t_issue = clock64() - kAttnLatencyCycles;
    unsigned fetches = 0;
    if (!done) {  // the first record and scale load directly: nothing is in flight yet to hide them behind
        if (claim < n_work) {
            nx = a.work[claim];
            qs_nx = __ldg(a.qs + (size_t)nx.row * a.heads + (nx.head_chunk & 0xFFFF));
            fs = kReady;
        } else {
            fs = kExhausted;
        }
    }
    int k = 0, n_pages = 0;
    unsigned issued = 0;
    uint32_t idle = 0;
    bool timed_out = false;
    while (true) {
        bool send = false;
        int stage = 0;
        if (!done) {
            // one step of the next item's fetch
            if (fs == kClaimed && clock64() - t_issue >= kAttnLatencyCycles) {
                if (claim < n_work) {
                    uint64_t *bar = &record_bar[c];
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(bar, (uint32_t)sizeof(AttnWork));
                    bulk_g2s(record, a.work + claim, (uint32_t)sizeof(AttnWork), bar);
                    fs = kFetching;
                } else {
                    fs = kExhausted;
                }
            } else if (fs == kFetching && mbar_test_wait(&record_bar[c], fetches & 1)) {
                fetches++;
                nx = *reinterpret_cast<const AttnWork *>(record);
                qs_nx = __ldg(a.qs + (size_t)nx.row * a.heads + (nx.head_chunk & 0xFFFF));
                t_issue = clock64();
                fs = kScale;
            } else if (fs == kScale && clock64() - t_issue >= kAttnLatencyCycles) {
                fs = kReady;
            }
            // the next item starts once the current one is issued
            if (!ending && k == n_pages) {
                if (fs == kReady) {
                    cur = nx;
                    qs_cur = qs_nx;
                    n_pages = cur.pages_chunks & 0xFFFF;
                    k = 0;
                    claim = W + atomicAdd(next_item, 1);
                    t_issue = clock64();
                    fs = kClaimed;
                } else if (fs == kExhausted) {
                    ending = true;
                }
            }
            if (ending || k < n_pages) {
                stage = issued % kAttnStages;
                send = issued < (unsigned)kAttnStages ||
                       mbar_test_wait(&empty[c * kAttnStages + stage], ((issued / kAttnStages) - 1) & 1);
            }
        }
        if (send) {  // lanes with a free stage issue together
            uint64_t *bar = &full[c * kAttnStages + stage];
            uint8_t *hdr = smem + c * kConsumerSmem + kAttnHdrOffset + stage * kAttnHdrBytes;
            if (ending) {  // end marker: no copy, the consumer reads row -1 and stops
                *reinterpret_cast<int4 *>(hdr) = make_int4(-1, 0, 0, 0);
                mbar_arrive(bar);
                done = true;
            } else {
                const bool first = k == 0;
                int page = -1;
#pragma unroll
                for (int j = 0; j < kAttnMaxChunkPages; j++)
                    if (j == k) page = cur.page[j];
                k++;
                const bool page_ok = page >= 0 && page < a.num_pages;
                if (!page_ok && a.status) atomicOr(a.status, kStatusBadPage);
                const uint32_t tx = (page_ok ? kKvBlockBytes : 0) + (first ? kHeadDim : 0);
                const int head = cur.head_chunk & 0xFFFF;
                if (first) {
                    *reinterpret_cast<int4 *>(hdr) = make_int4(cur.row, cur.head_chunk, cur.len, cur.pages_chunks);
                    *reinterpret_cast<float *>(hdr + 16) = qs_cur;
                }
                *reinterpret_cast<int *>(hdr + 24) = page_ok ? 1 : 0;  // a skipped page poisons its item
                if (tx == 0) {
                    mbar_arrive(bar);
                } else {
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(bar, tx);
                    if (page_ok)
                        bulk_g2s(smem + c * kConsumerSmem + stage * kKvBlockBytes,
                                 a.pool + (size_t)page * a.page_bytes + kv_block_offset(a.layer, head, a.heads),
                                 kKvBlockBytes, bar);
                    if (first) bulk_g2s(hdr + 32, a.q + ((size_t)cur.row * a.heads + head) * kHeadDim, kHeadDim, bar);
                }
            }
            issued++;
        }
        const unsigned busy = __ballot_sync(0xffffffffu, !done), moved = __ballot_sync(0xffffffffu, send);
        if (!busy) break;
        if (moved) {
            idle = 0;
        } else if (++idle > kPollLimit) {
            timed_out = true;
            break;
        } else {
            __nanosleep(64);
        }
    }
    if (timed_out && lane == 0 && a.status) atomicOr(a.status, kStatusTimeout);
    // drain: every copy this lane issued lands before the CTA exits (bounded)
    if (fs == kFetching) mbar_wait_bounded(&record_bar[c], fetches & 1, kWaitLimit);
    for (unsigned j = issued > (unsigned)kAttnStages ? issued - kAttnStages : 0u; j < issued; j++)
        mbar_wait_bounded(&full[c * kAttnStages + j % kAttnStages], (j / kAttnStages) & 1, kWaitLimit);
}

__device__ __forceinline__ void attn_consumer(const AttnArgs &a, uint8_t *smem, uint64_t *full, uint64_t *empty,
                                              int warp, int lane) {
    const int gid = lane >> 2, tig = lane & 3;
    uint8_t *ring = smem + warp * kConsumerSmem;
    uint8_t *digits = ring + kAttnStages * kKvBlockBytes;  // [digit 0..2, unused zero row][tig][16 bytes]
    const uint8_t *headers = ring + kAttnHdrOffset;
    uint64_t *f_bar = full + warp * kAttnStages, *e_bar = empty + warp * kAttnStages;
    reinterpret_cast<uint2 *>(digits)[lane] = make_uint2(0u, 0u);
    __syncwarp();
    unsigned consumed = 0;
    bool timed_out = false;
    while (!timed_out) {
        // the item's first stage carries its header (or the end marker)
        const int stage0 = consumed % kAttnStages;
        if (!mbar_wait_bounded(&f_bar[stage0], (consumed / kAttnStages) & 1, kWaitLimit)) {
            timed_out = true;
            break;
        }
        const uint8_t *hdr = headers + stage0 * kAttnHdrBytes;
        const int4 meta = *reinterpret_cast<const int4 *>(hdr);
        if (meta.x < 0) break;  // the list ended for this warp
        const uint4 qv = *reinterpret_cast<const uint4 *>(hdr + 32 + tig * 16);  // K-dim chunk tig, both k-steps
        const float scale = __fmul_rn(*reinterpret_cast<const float *>(hdr + 16), a.inv_sqrt_d);
        AttnItem it;
        it.row = meta.x;
        it.head = meta.y & 0xFFFF;
        it.chunk = meta.y >> 16;
        it.len = meta.z;
        it.n_pages = meta.w & 0xFFFF;
        it.n_chunks = meta.w >> 16;
        it.first_page = it.chunk * a.chunk_pages;
        float m = -INFINITY, l = 0.0f;
        int e_acc = 12;  // power-of-two scale currently applied to the accumulators
        int acc_i[4][4];
        float acc_f[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; mt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc_i[mt][i] = 0, acc_f[mt][i] = 0.0f;
        int held = 0;  // pages summed in acc_i since the last flush
        bool poisoned = false;  // a page of this item was skipped: the item publishes NaN
        const int p0 = 16 * tig + gid, p1 = p0 + 8;
        for (int pg = 0; pg < it.n_pages; pg++) {
            const int stage = consumed % kAttnStages;
            if (pg > 0 && !mbar_wait_bounded(&f_bar[stage], (consumed / kAttnStages) & 1, kWaitLimit)) {
                timed_out = true;
                break;
            }
            const uint8_t *blk = ring + stage * kKvBlockBytes;
            const int valid = min(kPagePositions, it.len - (it.first_page + pg) * kPagePositions);
            // the page into registers (K and V^T fragments, scales); then the
            // stage goes back to the producer while this warp computes
            uint4 kf[4][2], vf[4][2];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                kf[mt][0] = *reinterpret_cast<const uint4 *>(blk + mt * 1024 + lane * 16);
                kf[mt][1] = *reinterpret_cast<const uint4 *>(blk + mt * 1024 + 512 + lane * 16);
                vf[mt][0] = *reinterpret_cast<const uint4 *>(blk + kVOffset + mt * 1024 + lane * 16);
                vf[mt][1] = *reinterpret_cast<const uint4 *>(blk + kVOffset + mt * 1024 + 512 + lane * 16);
            }
            const float2 ks = *reinterpret_cast<const float2 *>(blk + kKScaleOffset + 8 * lane);
            const float2 vs = *reinterpret_cast<const float2 *>(blk + kVScaleOffset + 8 * lane);
            if (!*reinterpret_cast<const int *>(headers + stage * kAttnHdrBytes + 24)) poisoned = true;
            __syncwarp();
            if (lane == 0) mbar_arrive(&e_bar[stage]);
            consumed++;
            // ---- QK ----
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                int d[4] = {0, 0, 0, 0};
                mma_s8s8_m16n8k32(d, kf[mt][0], qv.x, qv.y);
                mma_s8s8_m16n8k32(d, kf[mt][1], qv.z, qv.w);
                if (mt == tig) dot0 = d[0], dot1 = d[2];
            }
            const float s0 = p0 < valid ? __fmul_rn(__fmul_rn(__int2float_rn(dot0), ks.x), scale) : -INFINITY;
            const float s1 = p1 < valid ? __fmul_rn(__fmul_rn(__int2float_rn(dot1), ks.y), scale) : -INFINITY;
            // one combined warp reduction: the page's score max and V-scale max
            float smax = fmaxf(s0, s1);
            float vmax = fmaxf(p0 < valid ? vs.x : 0.0f, p1 < valid ? vs.y : 0.0f);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
                vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
            }
            const float m_new = fmaxf(m, smax);
            const float e0 = p0 < valid ? expf(s0 - m_new) : 0.0f;
            const float e1 = p1 < valid ? expf(s1 - m_new) : 0.0f;
            const float corr = expf(m - m_new);
            l = l * corr + (e0 + e1);  // this lane's share; reduced across the warp per item
            m = m_new;
            // power-of-two range guard: w' = p * vs * 2^e < 2^12 (p <= 1)
            int ex;
            frexpf(vmax, &ex);
            const int e_page = 12 - max(0, ex);
            const float rescale = corr * exp2f((float)(e_page - e_acc));
            e_acc = e_page;
            const float f = exp2f((float)(e_page + 12));
            // W = w' * 2^12 < 2^24 (an exact power-of-two scaling of w')
            const uint32_t W0 = p0 < valid ? __float2uint_rn(e0 * vs.x * f) : 0u;
            const uint32_t W1 = p1 < valid ? __float2uint_rn(e1 * vs.y * f) : 0u;
            // digits of this lane's two positions, at PV columns pv_col(p0) and pv_col(p0) + 1
            uint8_t *dg = digits + tig * 16 + 2 * gid;
            *reinterpret_cast<uint16_t *>(dg) = (uint16_t)__byte_perm(W0, W1, 0x0062);
            *reinterpret_cast<uint16_t *>(dg + 64) = (uint16_t)__byte_perm(W0, W1, 0x0051);
            *reinterpret_cast<uint16_t *>(dg + 128) = (uint16_t)__byte_perm(W0, W1, 0x0040);
            if (rescale != 1.0f || held == kHoldPages) {
#pragma unroll
                for (int mt = 0; mt < 4; mt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        acc_f[mt][i] = (acc_f[mt][i] + __int2float_rn(acc_i[mt][i])) * rescale;
                        acc_i[mt][i] = 0;
                    }
                held = 0;
            }
            held++;
            __syncwarp();
            // ---- PV: column n of B is digit n & 3 (digit 3 = the zero row) ----
            const uint4 b = *reinterpret_cast<const uint4 *>(digits + (gid & 3) * 64 + tig * 16);
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                mma_s8u8_m16n8k32(acc_i[mt], vf[mt][0], b.x, b.y);
                mma_s8u8_m16n8k32(acc_i[mt], vf[mt][1], b.z, b.w);
            }
            __syncwarp();  // the digits are read before the next page rewrites them
        }
        if (timed_out) break;
        l = warp_sum_f(l);
        // lane (gid, 0) holds digits 0 and 1 of dims 16*mt + gid (+8), lane
        // (gid, 1) digit 2: o = (D0 * 2^16 + D1 * 2^8 + D2) * 2^-(12 + e)
        const float unscale = exp2f((float)(-12 - e_acc));
        float o[4][2];
#pragma unroll
        for (int mt = 0; mt < 4; mt++) {
            float t[4];
#pragma unroll
            for (int i = 0; i < 4; i++) t[i] = acc_f[mt][i] + __int2float_rn(acc_i[mt][i]);
            const float d2a = __shfl_down_sync(0xffffffffu, t[0], 1);
            const float d2b = __shfl_down_sync(0xffffffffu, t[2], 1);
            o[mt][0] = fmaf(t[0], 65536.0f, fmaf(t[1], 256.0f, d2a)) * unscale;
            o[mt][1] = fmaf(t[2], 65536.0f, fmaf(t[3], 256.0f, d2b)) * unscale;
        }
        if (poisoned) {  // NaN output (or NaN partial, which the merge turns into a NaN output)
#pragma unroll
            for (int mt = 0; mt < 4; mt++) o[mt][0] = o[mt][1] = __int_as_float(0x7fc00000);
            m = l = __int_as_float(0x7fc00000);
        }
        const size_t rh_index = (size_t)it.row * a.heads + it.head;
        float *out = a.out + rh_index * kHeadDim;
        if (it.n_chunks == 1) {
            const float inv = 1.0f / l;
            if (tig == 0)
#pragma unroll
                for (int mt = 0; mt < 4; mt++) {
                    out[16 * mt + gid] = o[mt][0] * inv;
                    out[16 * mt + gid + 8] = o[mt][1] * inv;
                }
            continue;
        }
        // long row: publish this chunk's (unnormalised output, peak, sum);
        // attn_merge_kernel combines them after this launch
        float *part = a.partials + (rh_index * a.max_chunks + it.chunk) * kPartialFloats;
        if (tig == 0)
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                part[16 * mt + gid] = o[mt][0];
                part[16 * mt + gid + 8] = o[mt][1];
            }
        if (lane == 0) {
            part[64] = m;
            part[65] = l;
        }
    }
    if (timed_out && lane == 0 && a.status) atomicOr(a.status, kStatusTimeout);
}

__global__ void __launch_bounds__(kAttnThreads, kAttnCtasPerSm) attn_decode_kernel(AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kAttnBarOffset);  // [consumer][stage]
    uint64_t *empty = full + kAttnConsumers * kAttnStages;
    uint64_t *record_bar = empty + kAttnConsumers * kAttnStages;  // [consumer]
    if (threadIdx.x == 0) {
        for (int i = 0; i < kAttnConsumers * kAttnStages; i++) mbar_init(&full[i], 1), mbar_init(&empty[i], 1);
        for (int i = 0; i < kAttnConsumers; i++) mbar_init(&record_bar[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (warp == kAttnConsumers)
        attn_producer(a, smem, full, empty, record_bar, lane);
    else
        attn_consumer(a, smem, full, empty, warp, lane);
    // every producer lane has taken its last item: the last CTA out resets
    // the item counter and the finish count for the next launch
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

// Combines the chunks of every long row (Attention.MergePartials,
// src/Needle/Blocks.cs:750-817): out = sum_c w_c o_c / sum_c w_c l_c with
// w_c = exp(peak_c - max peak), chunks in ascending order.  Warp per
// (row, head); lane owns dims 2*lane, 2*lane+1.
__global__ void __launch_bounds__(256) attn_merge_kernel(AttnArgs a) {
    pdl_enter();
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= a.rows * a.heads) return;
    const int row = w / a.heads;
    const int len = a.row_pos[row] + 1, slot = a.row_slot[row];
    if (len < 1 || len > a.max_pages * kPagePositions || slot < 0 || slot >= a.slots) return;  // NaN already
    const int pages = (len + kPagePositions - 1) / kPagePositions;
    const int n_chunks = (pages + a.chunk_pages - 1) / a.chunk_pages;
    if (n_chunks < 2) return;
    const float *parts = a.partials + (size_t)w * a.max_chunks * kPartialFloats;
    float peak = -INFINITY;
    for (int c = 0; c < n_chunks; c++) peak = fmaxf(peak, parts[c * kPartialFloats + 64]);
    float total = 0.0f, m0 = 0.0f, m1 = 0.0f;
    for (int c = 0; c < n_chunks; c++) {
        const float *pc = parts + c * kPartialFloats;
        const float wgt = expf(pc[64] - peak);
        total += wgt * pc[65];
        const float2 v = *reinterpret_cast<const float2 *>(pc + 2 * lane);
        m0 += wgt * v.x;
        m1 += wgt * v.y;
    }
    const float inv = 1.0f / total;
    *reinterpret_cast<float2 *>(a.out + (size_t)w * kHeadDim + 2 * lane) = make_float2(m0 * inv, m1 * inv);
}

// attn_merge_kernel fused with the per-row quantize of the attention
// output (the o-projection's input), bit-identical to the two launches:
// CTA per row, warp per head; a head of a one-chunk row is read back from
// out.  The row peak (exact max of |x| over heads x 64) goes through shared
// memory; scale, inverse and rounding as Scalar.QuantizeInt8
// (src/Needle/Scalar.cs:67-74).
__global__ void __launch_bounds__(1024) attn_merge_quantize_kernel(AttnArgs a) {
    pdl_enter();
    __shared__ float head_peak[32];
    const int row = blockIdx.x, head = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = row * a.heads + head;
    const int len = a.row_pos[row] + 1, slot = a.row_slot[row];
    const bool valid = len >= 1 && len <= a.max_pages * kPagePositions && slot >= 0 && slot < a.slots;
    const int pages = (len + kPagePositions - 1) / kPagePositions;
    const int n_chunks = valid ? (pages + a.chunk_pages - 1) / a.chunk_pages : 1;
    float2 *o = reinterpret_cast<float2 *>(a.out + (size_t)w * kHeadDim + 2 * lane);
    float2 v;
    if (n_chunks >= 2) {
        const float *parts = a.partials + (size_t)w * a.max_chunks * kPartialFloats;
        float peak = -INFINITY;
        for (int c = 0; c < n_chunks; c++) peak = fmaxf(peak, parts[c * kPartialFloats + 64]);
        float total = 0.0f, m0 = 0.0f, m1 = 0.0f;
        for (int c = 0; c < n_chunks; c++) {
            const float *pc = parts + c * kPartialFloats;
            const float wgt = expf(pc[64] - peak);
            total += wgt * pc[65];
            const float2 pv = *reinterpret_cast<const float2 *>(pc + 2 * lane);
            m0 += wgt * pv.x;
            m1 += wgt * pv.y;
        }
        const float inv = 1.0f / total;
        v = make_float2(m0 * inv, m1 * inv);
        *o = v;
    } else {
        v = *o;
    }
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
    launch_kernel(attn_work_kernel, dim3(a.rows), dim3(256), 0, stream, a);
    return check_launch("attn_work");
}

int launch_attn_merge(const AttnArgs &a, cudaStream_t stream) {
    if (a.rows == 0) return NDL_OK;
    if (a.q_out) {
        if (a.heads > 32) return set_error(NDL_ERR_INVALID_ARG, "attention: %d heads > 32", a.heads);
        launch_kernel(attn_merge_quantize_kernel, dim3(a.rows), dim3(a.heads * 32), 0, stream, a);
        return check_launch("attn_merge_quantize");
    }
    if (a.max_chunks < 2) return NDL_OK;
    const int warps = a.rows * a.heads;
    launch_kernel(attn_merge_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream, a);
    return check_launch("attn_merge");
}

int launch_attn_decode(const AttnArgs &a, cudaStream_t stream, bool build_work, bool merge) {
    if (a.rows == 0) return NDL_OK;
    if (a.chunk_pages < 1 || a.chunk_pages > kAttnMaxChunkPages)
        return set_error(NDL_ERR_INVALID_ARG, "attention: %d pages per item (1..%d)", a.chunk_pages,
                         kAttnMaxChunkPages);
    static DeviceOnce smem_attribute;  // the attribute belongs to the kernel on one device
    int st0 = smem_attribute.run([] {
        cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kAttnSmem);
        if (e != cudaSuccess) return set_error(NDL_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
        return (int)NDL_OK;
    });
    if (st0 != NDL_OK) return st0;
    const int sms = device_sm_count();
    const long long items = (long long)a.rows * a.heads * a.max_chunks;
    if (items > 0x7FFFFFFF) return set_error(NDL_ERR_INVALID_ARG, "attention: too many work items");
    if (build_work) {
        int st = launch_attn_work(a, stream);
        if (st != NDL_OK) return st;
    }
    long long blocks = (items + kAttnConsumers - 1) / kAttnConsumers;
    const long long resident = (long long)sms * kAttnCtasPerSm;  // the CTAs that fit the shared memory
    if (blocks > resident) blocks = resident;
    launch_kernel(attn_decode_kernel, dim3((unsigned)blocks), dim3(kAttnThreads), kAttnSmem, stream, a);
    int st = check_launch("attn_decode");
    if (st != NDL_OK || !merge) return st;
    return launch_attn_merge(a, stream);
}

}  // namespace ndl

using namespace ndl;

static constexpr int kAbiChunkPages = 8;

// Workspace: the chunk partials [rows][heads][chunks][kPartialFloats] fp32,
// then the work list [rows * heads * chunks] and 16 bytes for its length and
// the decode kernel's two counters.
static size_t abi_partial_bytes(int rows, int heads, int max_pages) {
    const size_t chunks = (size_t)(max_pages + kAbiChunkPages - 1) / kAbiChunkPages;
    return ((size_t)rows * heads * chunks * kPartialFloats * sizeof(float) + 15) / 16 * 16;
}

extern "C" NDL_API size_t ndl_attention_paged_workspace(int rows, int heads, int max_pages) {
    if (rows <= 0 || heads <= 0 || max_pages <= 0) return 0;
    const size_t chunks = (size_t)(max_pages + kAbiChunkPages - 1) / kAbiChunkPages;
    return abi_partial_bytes(rows, heads, max_pages) + (size_t)rows * heads * chunks * sizeof(AttnWork) + 16;
}

// Points a.partials, a.work and a.n_work into a workspace of that layout.
static void abi_carve(AttnArgs &a, void *ws, int rows, int heads, int max_pages) {
    uint8_t *base = static_cast<uint8_t *>(ws);
    const size_t pb = abi_partial_bytes(rows, heads, max_pages);
    const size_t chunks = (size_t)(max_pages + kAbiChunkPages - 1) / kAbiChunkPages;
    a.partials = reinterpret_cast<float *>(base);
    a.work = reinterpret_cast<AttnWork *>(base + pb);
    a.n_work = reinterpret_cast<int *>(base + pb + (size_t)rows * heads * chunks * sizeof(AttnWork));
}

extern "C" NDL_API int ndl_attention_paged(const int8_t *q, const float *qs, const int32_t *row_slot,
                                           const int32_t *row_pos, int rows, int heads, const int32_t *page_table,
                                           int slots, int max_pages, const uint8_t *pool, size_t page_bytes,
                                           int num_pages, int layer, float *out, void *workspace,
                                           size_t workspace_bytes, int *status, void *stream) {
    NDL_REQUIRE(rows >= 0 && heads >= 1 && slots >= 1 && max_pages >= 1 && num_pages >= 1 && layer >= 0,
                "bad attention geometry");
    if (rows == 0) return NDL_OK;
    NDL_REQUIRE(q && qs && row_slot && row_pos && page_table && pool && out, "null pointer");
    NDL_REQUIRE(page_bytes % 16 == 0 && page_bytes >= kv_block_offset(layer, heads - 1, heads) + kKvBlockBytes,
                "page_bytes %zu cannot hold layer %d of %d heads", page_bytes, layer, heads);
    NDL_REQUIRE(aligned(q, 16) && aligned(pool, 16) && aligned(out, 16) && aligned(qs, 4), "misaligned pointer");
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
               layer, heads, rows, kAbiChunkPages, (max_pages + kAbiChunkPages - 1) / kAbiChunkPages,
               0.125f, out, nullptr, nullptr, status, slots};
    abi_carve(a, ws, rows, heads, max_pages);
    int rc = launch_attn_decode(a, st);
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
// This entry point keeps the chunk partials in a fixed device array that
// the library owns instead.
//
// The array is a file-scope __device__ variable, so every GPU that loads
// this library holds its kNoAllocScratchBytes until the process exits.  On
// the host its name is only a stand-in: the real device address is looked
// up once per device with cudaGetSymbolAddress, the first time the entry
// point is called on that device (with that device current), and cached.
// Make that first call before any stream capture starts.
//
// Every call shares the one array.  Nothing in it has to start at zero: a
// launch writes each chunk partial before the merge reads it.  Two calls
// whose work overlaps on the GPU (different streams, or no ordering between
// them) race on the array and can corrupt each other's results; callers
// must order them, for example by issuing them on one stream.
// ---------------------------------------------------------------------------
namespace {

// 4 MiB: 320 bytes per (row, head, 8-page chunk) item (a 272-byte partial
// and a 48-byte work record) plus 16 bytes of counters, so at most 13107
// items; 512 rows x 8 heads x 3 chunks (1536 positions) fit.
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
    NDL_REQUIRE(rows >= 0 && heads >= 1 && slots >= 1 && max_pages >= 1 && num_pages >= 1 && layer >= 0,
                "bad attention geometry");
    if (rows == 0) return NDL_OK;
    NDL_REQUIRE(q && qs && row_slot && row_pos && page_table && pool && out, "null pointer");
    NDL_REQUIRE(page_bytes % 16 == 0 && page_bytes >= kv_block_offset(layer, heads - 1, heads) + kKvBlockBytes,
                "page_bytes %zu cannot hold layer %d of %d heads", page_bytes, layer, heads);
    NDL_REQUIRE(aligned(q, 16) && aligned(pool, 16) && aligned(out, 16) && aligned(qs, 4), "misaligned pointer");
    const size_t need = ndl_attention_paged_workspace(rows, heads, max_pages);
    if (need > kNoAllocScratchBytes)
        return set_error(NDL_ERR_INVALID_ARG,
                         "%d rows x %d heads x %d pages need %zu bytes of scratch; the built-in buffer holds %zu",
                         rows, heads, max_pages, need, kNoAllocScratchBytes);
    void *scratch = nullptr;
    int st = noalloc_scratch(&scratch);
    if (st != NDL_OK) return st;
    AttnArgs a{q, qs, row_slot, row_pos, nullptr, page_table, max_pages, pool, (long long)page_bytes, num_pages,
               layer, heads, rows, kAbiChunkPages, (max_pages + kAbiChunkPages - 1) / kAbiChunkPages,
               0.125f, out, nullptr, nullptr, status, slots};
    abi_carve(a, scratch, rows, heads, max_pages);
    return launch_attn_decode(a, (cudaStream_t)stream);
}
