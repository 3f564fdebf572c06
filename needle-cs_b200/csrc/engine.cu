// Batched decode engine: the B200 replacement of BatchedEngine / EngineCore
// (src/Needle/BatchEngine.cs:5-50, src/Needle/Engine.cs:2255-2350).
//
// Owns the device weights of the synthetic decoder, the paged int8 KV pool,
// per-slot lengths / marks / page tables, and the step buffers.  One host
// thread per engine; all device work is ordered on the engine's stream.
//
// forward_batch(tokens, row_slots, rows, head_rows, heads) follows the
// reference's ForwardBatch contract: consecutive rows of one slot are a
// prefill run at positions len, len+1, ...; every row attends causally to
// its own slot; logits are produced only for head_rows (compact order).
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "needle3.cuh"
#include "kv.cuh"

namespace ndl {

int launch_step_prepare(const int32_t *updates, int32_t *page_table, int max_pages, const int32_t *tokens, int rows,
                        const uint16_t *embedding, int vocab, int dim, float *x, int *status, cudaStream_t stream);
int launch_swiglu_quantize(const float *gu, int rows, int ffn, float *act, int8_t *q, float *scales,
                           cudaStream_t stream);
int launch_gather_rows(const float *x, const int32_t *idx, int n, int dim, float *out, cudaStream_t stream);
int launch_argmax_masked(const float *x, long long ldx, const uint32_t *mask, int words, long long ldm,
                         const int32_t *mask_index, int length, int rows, int32_t *ids, float *probs,
                         cudaStream_t stream);
int launch_topk_logsoftmax(const float *x, long long ldx, int n, int k, int mask023, int rows, int32_t *idx,
                           float *logp, float *probs, cudaStream_t stream);
int launch_kv_fill(uint64_t seed, uint64_t session, int layers, int heads, int first, int count,
                   const int32_t *page_row, uint8_t *pool, long long page_bytes, cudaStream_t stream);
int launch_half_to_float(const uint16_t *src, long long n, float *dst, cudaStream_t stream);
int launch_sparse_head(const int8_t *w, const uint16_t *sw, int vocab, int k, const int8_t *qa, const float *sa,
                       const int32_t *offsets, int n, const int32_t *ids, int total, float *out, int *status,
                       cudaStream_t stream);
int launch_sparse_argmax(const float *values, const int32_t *offsets, const int32_t *ids, int n, int32_t *picks,
                         float *probs, cudaStream_t stream);

// Stream ids of the synthetic decoder tensors under the model seed.
enum : uint64_t {
    kStreamEmbedding = 1,
    kStreamFinalNorm = 2,
    kStreamLayerBase = 100,   // + 16 * layer + field
    kStreamCrossBase = 5000,  // + 16 * layer + cross field
};
enum : int { kFCqW, kFCqS, kFCkvW, kFCkvS, kFCoW, kFCoS, kFCrossNorm };
// fp16 N(0,1) encoder memory of an utterance: stream kStreamMemory + utterance
constexpr uint64_t kStreamMemory = 1ull << 40;
enum : int { kFQkvW, kFQkvS, kFOW, kFOS, kFGuW, kFGuS, kFDW, kFDS, kFAttnNorm, kFFfnNorm };

struct DeviceLayer {
    int8_t *w_qkv, *w_o, *w_gu, *w_d;
    uint16_t *s_qkv, *s_o, *s_gu, *s_d;
    float *attn_norm, *ffn_norm;
    // cross-attention block (decoders with `cross`)
    int8_t *w_cq = nullptr, *w_ckv = nullptr, *w_co = nullptr;
    uint16_t *s_cq = nullptr, *s_ckv = nullptr, *s_co = nullptr;
    float *cross_norm = nullptr;
};

}  // namespace ndl

struct ndl_engine {
    ndl_engine_config ec{};
    ndl_decoder_config dc{};
    ndl::N3State *n3 = nullptr;  // set: a Needle-3 engine over a loaded model (ndl_engine_create_model)
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::vector<void *> allocations;
    std::vector<ndl::DeviceLayer> layers;
    float *final_norm = nullptr;
    uint16_t *embedding = nullptr;
    int8_t *w_head = nullptr;
    uint16_t *s_head = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // KV
    int max_pages = 0;
    size_t page_bytes = 0;
    uint8_t *pool = nullptr;
    int32_t *d_page_table = nullptr;
    std::vector<int32_t> page_table;  // host mirror [slots][max_pages]
    std::vector<int32_t> free_pages;
    std::vector<int> page_refs;  // slots holding each pool page (shared prefixes hold one page in many)
    std::vector<int> slot_len, slot_mark;
    std::vector<int> cross_slot;  // memory slot attended by each slot's rows (-1: none)
    // step buffers
    float *x = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *act = nullptr, *head_x = nullptr;
    int8_t *qa = nullptr, *q8 = nullptr;
    float *sa = nullptr, *qs = nullptr;
    float *logits = nullptr;
    int32_t *d_meta = nullptr;
    int32_t *h_meta = nullptr;  // pinned staging
    size_t meta_ints = 0;
    int32_t *attn_work = nullptr, *cross_work = nullptr;  // per-step attention work lists
    int *n_work = nullptr;                                // their counters, int[4] each (self, cross)
    int *d_status = nullptr;
    int32_t *d_ids = nullptr;
    float *d_probs = nullptr, *d_logp = nullptr;
    uint32_t *d_masks = nullptr;
    // per-slot sampling masks held on the device ([slots][vocab words]),
    // allocated by the first ndl_engine_set_mask
    uint32_t *d_mask_table = nullptr;
    int32_t *d_mask_index = nullptr;
    std::vector<char> slot_has_mask;
    void *h_out = nullptr;  // pinned sampling results
    // sparse head staging (grown on demand): device and pinned host copies of
    // rows, offsets, picks, probs (max_heads each) then ids and values
    void *d_sparse = nullptr, *h_sparse = nullptr;
    size_t sparse_bytes = 0;
    // primed-prefix blob staging (grown on demand, kept across calls)
    uint8_t *d_prefix = nullptr;
    size_t prefix_bytes = 0;
    int last_rows = 0, last_heads = 0;
    // captured step graphs, keyed by (rows, heads)
    struct StepGraph {
        int rows, heads;
        cudaGraphExec_t exec;
        unsigned long long last_use;
    };
    std::vector<StepGraph> graphs;
    unsigned long long graph_clock = 0;
    bool use_graphs = true;
    bool use_pdl = true;  // step kernels overlap their launches (programmatic dependent launch)
    // per-kernel-class timing (CUDA events on the engine stream)
    bool profile = false;
    std::vector<cudaEvent_t> event_pool;
    size_t events_used = 0;
    std::vector<std::pair<int, size_t>> pending;  // (class, index of the start event)
    double prof_ms[NDL_PROF_CLASSES] = {0};
    long long prof_count[NDL_PROF_CLASSES] = {0};
    // offsets of the last step's metadata in d_meta
    int off_tokens = 0, off_slot = 0, off_pos = 0, off_order = 0, off_cslot = 0, off_cpos = 0, off_head = 0,
        off_updates = 0;
};

using namespace ndl;

namespace {

template <typename T>
int dalloc(ndl_engine *e, T **p, size_t count) {
    void *ptr = nullptr;
    cudaError_t err = cudaMalloc(&ptr, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu): %s", count * sizeof(T), cudaGetErrorString(err));
    }
    e->allocations.push_back(ptr);
    *p = static_cast<T *>(ptr);
    return NDL_OK;
}

#define TRY(x)                         \
    do {                               \
        int st_ = (x);                 \
        if (st_ != NDL_OK) return st_; \
    } while (0)

uint64_t layer_stream(int layer, int field) { return kStreamLayerBase + 16ull * layer + field; }

// Norm weights: 1 + 0.1 * normal (host, exact float ops).
void norm_values(uint64_t seed, uint64_t stream, int n, std::vector<float> &out) {
    out.resize(n);
    uint64_t key = synth_key(seed, stream);
    for (int i = 0; i < n; i++) {
        float z = synth_normal(key, i);
        float t = 0.1f * z;
        out[i] = 1.0f + t;
    }
}

int upload(ndl_engine *e, void *dst, const void *src, size_t bytes) {
    NDL_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, e->stream));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    return NDL_OK;
}

// LM head quantized from the fp16 embedding per (row, 32-group):
// s = fp16(max|e| / 127) (1 if the group is zero), w = clamp(rint(e * (1/float(s))), -127, 127).
void quantize_head(const std::vector<uint16_t> &emb, int vocab, int dim, std::vector<int8_t> &w,
                   std::vector<uint16_t> &s) {
    int G = dim / 32;
    w.resize((size_t)vocab * dim);
    s.resize((size_t)vocab * G);
    for (int r = 0; r < vocab; r++)
        for (int g = 0; g < G; g++) {
            const uint16_t *e = emb.data() + (size_t)r * dim + g * 32;
            float peak = 0.0f;
            for (int i = 0; i < 32; i++) peak = std::max(peak, std::fabs(half_to_float_ref(e[i])));
            uint16_t sh = peak > 0.0f ? float_to_half_rne(peak / 127.0f) : float_to_half_rne(1.0f);
            float sf = half_to_float_ref(sh);
            float inv = 1.0f / sf;
            s[(size_t)r * G + g] = sh;
            for (int i = 0; i < 32; i++) {
                float v = std::nearbyint(half_to_float_ref(e[i]) * inv);
                v = std::min(std::max(v, -127.0f), 127.0f);
                w[(size_t)r * dim + g * 32 + i] = (int8_t)v;
            }
        }
}

int build_weights(ndl_engine *e) {
    const ndl_decoder_config &c = e->dc;
    const int d = c.dim, F = c.ffn, V = c.vocab, G = d / 32, GF = F / 32;
    const uint64_t seed = c.seed;
    e->layers.resize(c.layers);
    std::vector<float> host;
    for (int l = 0; l < c.layers; l++) {
        DeviceLayer &L = e->layers[l];
        TRY(dalloc(e, &L.w_qkv, (size_t)3 * d * d));
        TRY(dalloc(e, &L.s_qkv, (size_t)3 * d * G));
        TRY(dalloc(e, &L.w_o, (size_t)d * d));
        TRY(dalloc(e, &L.s_o, (size_t)d * G));
        TRY(dalloc(e, &L.w_gu, (size_t)2 * F * d));
        TRY(dalloc(e, &L.s_gu, (size_t)2 * F * G));
        TRY(dalloc(e, &L.w_d, (size_t)d * F));
        TRY(dalloc(e, &L.s_d, (size_t)d * GF));
        TRY(dalloc(e, &L.attn_norm, d));
        TRY(dalloc(e, &L.ffn_norm, d));
        cudaStream_t s = e->stream;
        TRY(ndl_synth_int8_device(seed, layer_stream(l, kFQkvW), 0, (size_t)3 * d * d, L.w_qkv, s));
        TRY(ndl_synth_uniform_f16_device(seed, layer_stream(l, kFQkvS), 0, (size_t)3 * d * G, 0.001f, 0.02f,
                                         L.s_qkv, s));
        TRY(ndl_synth_int8_device(seed, layer_stream(l, kFOW), 0, (size_t)d * d, L.w_o, s));
        TRY(ndl_synth_uniform_f16_device(seed, layer_stream(l, kFOS), 0, (size_t)d * G, 0.001f, 0.02f, L.s_o, s));
        TRY(ndl_synth_int8_device(seed, layer_stream(l, kFGuW), 0, (size_t)2 * F * d, L.w_gu, s));
        TRY(ndl_synth_uniform_f16_device(seed, layer_stream(l, kFGuS), 0, (size_t)2 * F * G, 0.001f, 0.02f,
                                         L.s_gu, s));
        TRY(ndl_synth_int8_device(seed, layer_stream(l, kFDW), 0, (size_t)d * F, L.w_d, s));
        TRY(ndl_synth_uniform_f16_device(seed, layer_stream(l, kFDS), 0, (size_t)d * GF, 0.001f, 0.02f, L.s_d, s));
        norm_values(seed, layer_stream(l, kFAttnNorm), d, host);
        TRY(upload(e, L.attn_norm, host.data(), d * sizeof(float)));
        norm_values(seed, layer_stream(l, kFFfnNorm), d, host);
        TRY(upload(e, L.ffn_norm, host.data(), d * sizeof(float)));
        if (c.cross) {
            auto cs = [&](int f) { return (uint64_t)kStreamCrossBase + 16ull * l + (uint64_t)f; };
            TRY(dalloc(e, &L.w_cq, (size_t)d * d));
            TRY(dalloc(e, &L.s_cq, (size_t)d * G));
            TRY(dalloc(e, &L.w_ckv, (size_t)2 * d * d));
            TRY(dalloc(e, &L.s_ckv, (size_t)2 * d * G));
            TRY(dalloc(e, &L.w_co, (size_t)d * d));
            TRY(dalloc(e, &L.s_co, (size_t)d * G));
            TRY(dalloc(e, &L.cross_norm, d));
            TRY(ndl_synth_int8_device(seed, cs(kFCqW), 0, (size_t)d * d, L.w_cq, s));
            TRY(ndl_synth_uniform_f16_device(seed, cs(kFCqS), 0, (size_t)d * G, 0.001f, 0.02f, L.s_cq, s));
            TRY(ndl_synth_int8_device(seed, cs(kFCkvW), 0, (size_t)2 * d * d, L.w_ckv, s));
            TRY(ndl_synth_uniform_f16_device(seed, cs(kFCkvS), 0, (size_t)2 * d * G, 0.001f, 0.02f, L.s_ckv, s));
            TRY(ndl_synth_int8_device(seed, cs(kFCoW), 0, (size_t)d * d, L.w_co, s));
            TRY(ndl_synth_uniform_f16_device(seed, cs(kFCoS), 0, (size_t)d * G, 0.001f, 0.02f, L.s_co, s));
            norm_values(seed, cs(kFCrossNorm), d, host);
            TRY(upload(e, L.cross_norm, host.data(), d * sizeof(float)));
        }
    }
    TRY(dalloc(e, &e->final_norm, d));
    norm_values(seed, kStreamFinalNorm, d, host);
    TRY(upload(e, e->final_norm, host.data(), d * sizeof(float)));
    // embedding fp16 N(0, 0.02) and the int8 head quantized from it
    std::vector<uint16_t> emb((size_t)V * d);
    ndl_synth_normal_f16(seed, kStreamEmbedding, 0, emb.size(), 0.02f, emb.data());
    std::vector<int8_t> wh;
    std::vector<uint16_t> sh;
    quantize_head(emb, V, d, wh, sh);
    TRY(dalloc(e, &e->embedding, emb.size()));
    TRY(dalloc(e, &e->w_head, wh.size()));
    TRY(dalloc(e, &e->s_head, sh.size()));
    TRY(upload(e, e->embedding, emb.data(), emb.size() * 2));
    TRY(upload(e, e->w_head, wh.data(), wh.size()));
    TRY(upload(e, e->s_head, sh.data(), sh.size() * 2));
    // RoPE tables (EngineCore.RopeFrequencies/BuildRopeTables, src/Needle/Engine.cs:336-356)
    const int half = c.head_dim / 2, cap = e->ec.capacity;
    std::vector<float> freq(half), cs((size_t)cap * half), sn((size_t)cap * half);
    for (int i = 0; i < half; i++) freq[i] = 1.0f / powf(c.rope_theta, 2.0f * (float)i / (float)c.head_dim);
    for (int p = 0; p < cap; p++)
        for (int i = 0; i < half; i++) {
            float angle = (float)p * freq[i];
            cs[(size_t)p * half + i] = cosf(angle);
            sn[(size_t)p * half + i] = sinf(angle);
        }
    TRY(dalloc(e, &e->rope_cos, cs.size()));
    TRY(dalloc(e, &e->rope_sin, sn.size()));
    TRY(upload(e, e->rope_cos, cs.data(), cs.size() * 4));
    TRY(upload(e, e->rope_sin, sn.data(), sn.size() * 4));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    return NDL_OK;
}

int build_sampling_buffers(ndl_engine *e);

int build_buffers(ndl_engine *e) {
    const ndl_decoder_config &c = e->dc;
    const int R = e->ec.max_rows, Hd = e->ec.max_heads, d = c.dim, F = c.ffn;
    TRY(dalloc(e, &e->x, (size_t)R * d));
    TRY(dalloc(e, &e->qkv, (size_t)R * 3 * d));
    TRY(dalloc(e, &e->attn, (size_t)R * d));
    TRY(dalloc(e, &e->gu, (size_t)R * 2 * F));
    TRY(dalloc(e, &e->act, (size_t)R * F));
    TRY(dalloc(e, &e->head_x, (size_t)Hd * d));
    TRY(dalloc(e, &e->qa, (size_t)R * std::max(d, F)));
    TRY(dalloc(e, &e->q8, (size_t)R * d));
    TRY(dalloc(e, &e->sa, (size_t)R));
    TRY(dalloc(e, &e->qs, (size_t)R * c.heads));
    TRY(dalloc(e, &e->logits, (size_t)Hd * c.vocab));
    {
        const size_t records = (size_t)R * attn_record_ints(e->max_pages);
        TRY(dalloc(e, &e->attn_work, records));
        if (c.cross) TRY(dalloc(e, &e->cross_work, records));
        TRY(dalloc(e, &e->n_work, 8));  // int[4] per list (self, cross)
    }
    // metadata: tokens, slots, positions, order, memory slot, memory position
    // (R each) + head rows (Hd) + updates (3 per row + slack)
    e->meta_ints = (size_t)6 * R + Hd + 3 * (size_t)R + 64;
    TRY(dalloc(e, &e->d_meta, e->meta_ints));
    NDL_CUDA(cudaMallocHost(&e->h_meta, e->meta_ints * sizeof(int32_t)));
    return build_sampling_buffers(e);
}

// The logits, status word and sampling buffers every engine kind has.
int build_sampling_buffers(ndl_engine *e) {
    const int Hd = e->ec.max_heads, V = e->dc.vocab;
    if (!e->logits) TRY(dalloc(e, &e->logits, (size_t)Hd * V));
    TRY(dalloc(e, &e->d_status, 1));
    NDL_CUDA(cudaMemsetAsync(e->d_status, 0, sizeof(int), e->stream));
    TRY(dalloc(e, &e->d_ids, (size_t)Hd * 8));
    TRY(dalloc(e, &e->d_probs, (size_t)Hd * 8));
    TRY(dalloc(e, &e->d_logp, (size_t)Hd * 8));
    int words = (V + 31) / 32;
    TRY(dalloc(e, &e->d_masks, (size_t)Hd * words));
    NDL_CUDA(cudaMallocHost(&e->h_out, (size_t)Hd * 8 * 12 + (size_t)Hd * words * 4 + 64));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    return NDL_OK;
}

// A pool page for one slot (reference count 1), or -1 when the pool is empty.
int alloc_page(ndl_engine *e) {
    if (e->free_pages.empty()) return -1;
    const int page = e->free_pages.back();
    e->free_pages.pop_back();
    e->page_refs[page] = 1;
    return page;
}
// A slot drops its reference; the page returns to the pool with the last one.
void release_page(ndl_engine *e, int page) {
    if (--e->page_refs[page] == 0) e->free_pages.push_back(page);
}

void free_slot_pages(ndl_engine *e, int slot, int keep_pages, std::vector<int32_t> *updates) {
    int32_t *row = e->page_table.data() + (size_t)slot * e->max_pages;
    for (int i = keep_pages; i < e->max_pages; i++) {
        if (row[i] >= 0) {
            release_page(e, row[i]);
            row[i] = -1;
            if (updates) updates->insert(updates->end(), {slot, i, -1});
        }
    }
}

// Makes page index `pg` of `slot` writable by this slot alone: a missing
// page is allocated; a page another slot also holds (a shared prefix) is
// copied first (copy on write: the device copy is queued in `copies` as
// (from, to)).  Returns the page, or -1 when the pool is exhausted; a new
// entry is recorded in `updates` as (slot, index, page).
int writable_page(ndl_engine *e, int slot, int pg, std::vector<int32_t> &updates, std::vector<int32_t> &copies) {
    int32_t &entry = e->page_table[(size_t)slot * e->max_pages + pg];
    if (entry >= 0 && e->page_refs[entry] == 1) return entry;
    const int page = alloc_page(e);
    if (page < 0) return -1;
    if (entry >= 0) {
        copies.insert(copies.end(), {entry, page});
        release_page(e, entry);
    }
    entry = page;
    updates.insert(updates.end(), {slot, pg, page});
    return page;
}

// Queues the page copies of writable_page on the engine stream.
int copy_pages(ndl_engine *e, const std::vector<int32_t> &copies) {
    for (size_t i = 0; i < copies.size(); i += 2)
        NDL_CUDA(cudaMemcpyAsync(e->pool + (size_t)copies[i + 1] * e->page_bytes,
                                 e->pool + (size_t)copies[i] * e->page_bytes, e->page_bytes,
                                 cudaMemcpyDeviceToDevice, e->stream));
    return NDL_OK;
}

int check_status(ndl_engine *e) {
    int st = 0;
    NDL_CUDA(cudaMemcpyAsync(&st, e->d_status, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    if (st) {
        cudaMemsetAsync(e->d_status, 0, sizeof(int), e->stream);
        if (st & kStatusTimeout) return set_error(NDL_ERR_TIMEOUT, "a kernel wait gave up (status 0x%x)", st);
        return set_error(NDL_ERR_BOUNDS, "a kernel saw an out-of-range page or token (status 0x%x)", st);
    }
    return NDL_OK;
}

// Brings the device page table up to the host mirror for the entries that
// `updates` (slot, page, value triples) names: per touched slot one copy of
// the mirror's span from its lowest to its highest named page (the entries
// between hold the mirror's values already).  Small and synchronous.
int push_page_updates(ndl_engine *e, const std::vector<int32_t> &updates) {
    if (updates.empty()) return NDL_OK;
    std::vector<std::pair<int, std::pair<int, int>>> spans;  // slot -> [lo, hi]
    for (size_t i = 0; i < updates.size(); i += 3) {
        const int slot = updates[i], page = updates[i + 1];
        auto it = std::find_if(spans.begin(), spans.end(), [&](const auto &s) { return s.first == slot; });
        if (it == spans.end())
            spans.push_back({slot, {page, page}});
        else
            it->second = {std::min(it->second.first, page), std::max(it->second.second, page)};
    }
    for (const auto &s : spans) {
        const size_t at = (size_t)s.first * e->max_pages + s.second.first;
        NDL_CUDA(cudaMemcpyAsync(e->d_page_table + at, e->page_table.data() + at,
                                 sizeof(int32_t) * (size_t)(s.second.second - s.second.first + 1),
                                 cudaMemcpyHostToDevice, e->stream));
    }
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    return NDL_OK;
}

// Device staging for one primed-prefix blob, kept across calls so that an
// import or export does not allocate (and the pool does not trim) each time.
static int prefix_reserve(ndl_engine *e, size_t bytes) {
    if (bytes <= e->prefix_bytes) return NDL_OK;
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    if (e->d_prefix) cudaFree(e->d_prefix);
    e->d_prefix = nullptr;
    e->prefix_bytes = 0;
    if (cudaMalloc(reinterpret_cast<void **>(&e->d_prefix), bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "primed prefix staging (%zu bytes)", bytes);
    }
    e->prefix_bytes = bytes;
    return NDL_OK;
}

// Records a start event for `cls`; returns the pending index or -1.
long prof_begin(ndl_engine *e, int cls) {
    if (!e->profile) return -1;
    while (e->event_pool.size() < e->events_used + 2) {
        cudaEvent_t ev;
        if (cudaEventCreate(&ev) != cudaSuccess) return -1;
        e->event_pool.push_back(ev);
    }
    size_t i = e->events_used;
    e->events_used += 2;
    cudaEventRecord(e->event_pool[i], e->stream);
    e->pending.push_back({cls, i});
    return (long)i;
}
void prof_end(ndl_engine *e, long i) {
    if (i >= 0) cudaEventRecord(e->event_pool[i + 1], e->stream);
}
struct ProfScope {
    ndl_engine *e;
    long i;
    ProfScope(ndl_engine *e_, int cls) : e(e_), i(prof_begin(e_, cls)) {}
    ~ProfScope() { prof_end(e, i); }
};

int check_slot(ndl_engine *e, int slot) {
    if (!e) return set_error(NDL_ERR_INVALID_ARG, "engine is NULL");
    if (slot < 0 || slot >= e->ec.slots) return set_error(NDL_ERR_INVALID_ARG, "slot %d out of range", slot);
    return NDL_OK;
}

// The device work of one step.  Every kernel reads its per-step data from
// d_meta, so the sequence can be captured once per (rows, heads) and replayed.
int step_kernels(ndl_engine *e, int rows, int heads) {
    PdlScope pdl(e->use_pdl);
    const ndl_decoder_config &c = e->dc;
    cudaStream_t s = e->stream;
    const int32_t *d_tokens = e->d_meta + e->off_tokens, *d_slot = e->d_meta + e->off_slot;
    const int32_t *d_pos = e->d_meta + e->off_pos, *d_order = e->d_meta + e->off_order;
    const int32_t *d_head = e->d_meta + e->off_head;
    {
        ProfScope p(e, NDL_PROF_PREPARE);
        TRY(launch_step_prepare(e->d_meta + e->off_updates, e->d_page_table, e->max_pages, d_tokens, rows,
                                e->embedding, c.vocab, c.dim, e->x, e->d_status, s));
    }

    // the work lists (row records with their page ids) are the same for
    // every layer: built once per step.  A (row, head) is never split, so a
    // row's result depends only on its own positions (batch-invariant logits)
    {
        ProfScope p(e, NDL_PROF_PREPARE);
        AttnArgs w{e->q8, e->qs, d_slot, d_pos, d_order, e->d_page_table, e->max_pages, e->pool,
                   (long long)e->page_bytes, e->ec.kv_pages, 0, c.heads, rows, 0.0f, e->attn, e->d_status,
                   e->ec.slots, e->qa, e->sa, e->attn_work, e->n_work};
        TRY(launch_attn_work(w, s));
        if (c.cross) {
            w.row_slot = e->d_meta + e->off_cslot;
            w.row_pos = e->d_meta + e->off_cpos;
            w.work = e->cross_work;
            w.n_work = e->n_work + 4;
            TRY(launch_attn_work(w, s));
        }
    }

    const int d = c.dim, F = c.ffn;
    for (int l = 0; l < c.layers; l++) {
        const DeviceLayer &L = e->layers[l];
        {
            ProfScope p(e, NDL_PROF_NORM_QUANT);
            TRY(launch_quantize_rows(e->x, L.attn_norm, rows, d, e->qa, e->sa, s));
        }
        {
            ProfScope p(e, NDL_PROF_GEMM_QKV);
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_qkv, L.s_qkv, 3 * d, d, e->qkv, 3 * d, nullptr, nullptr, s));
        }
        {
            ProfScope p(e, NDL_PROF_KV_WRITE);
            KvWriteArgs kw{e->qkv, 3 * d, d_slot, d_pos, e->d_page_table, e->max_pages, e->pool,
                           (long long)e->page_bytes, e->ec.kv_pages, e->rope_cos, e->rope_sin, l, c.heads, rows,
                           e->q8, e->qs, e->d_status};
            TRY(launch_kv_write(kw, s));
        }
        const AttnArgs aa{e->q8, e->qs, d_slot, d_pos, d_order, e->d_page_table, e->max_pages, e->pool,
                          (long long)e->page_bytes, e->ec.kv_pages, l, c.heads, rows,
                          1.0f / sqrtf((float)c.head_dim), e->attn, e->d_status, e->ec.slots, e->qa, e->sa,
                          e->attn_work, e->n_work};
        {
            ProfScope p(e, NDL_PROF_ATTENTION);
            TRY(launch_attn_decode(aa, s, false, false));
        }
        {
            ProfScope p(e, NDL_PROF_NORM_QUANT);
            TRY(launch_attn_quantize(aa, s));  // the output quantized per row into qa, sa
        }
        {
            ProfScope p(e, NDL_PROF_GEMM_O);
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_o, L.s_o, d, d, e->x, d, e->x, nullptr, s));
        }
        if (c.cross) {
            // x += W_co . Attn(W_cq . RMSNorm(x), memory of the row's slot)
            ProfScope p(e, NDL_PROF_CROSS);
            const int32_t *d_cslot = e->d_meta + e->off_cslot, *d_cpos = e->d_meta + e->off_cpos;
            TRY(launch_quantize_rows(e->x, L.cross_norm, rows, d, e->qa, e->sa, s));
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_cq, L.s_cq, d, d, e->qkv, d, nullptr, nullptr, s));
            TRY(launch_cross_query(e->qkv, d, c.heads, rows, e->q8, e->qs, s));
            AttnArgs ca{e->q8, e->qs, d_cslot, d_cpos, d_order, e->d_page_table, e->max_pages, e->pool,
                        (long long)e->page_bytes, e->ec.kv_pages, l, c.heads, rows,
                        1.0f / sqrtf((float)c.head_dim), e->attn, e->d_status, e->ec.slots, e->qa, e->sa,
                        e->cross_work, e->n_work + 4};
            TRY(launch_attn_decode(ca, s, false));
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_co, L.s_co, d, d, e->x, d, e->x, nullptr, s));
        }
        {
            ProfScope p(e, NDL_PROF_NORM_QUANT);
            TRY(launch_quantize_rows(e->x, L.ffn_norm, rows, d, e->qa, e->sa, s));
        }
        {
            ProfScope p(e, NDL_PROF_GEMM_GATEUP);
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_gu, L.s_gu, 2 * F, d, e->gu, 2 * F, nullptr, nullptr, s));
        }
        {
            ProfScope p(e, NDL_PROF_SWIGLU);
            TRY(launch_swiglu_quantize(e->gu, rows, F, e->act, e->qa, e->sa, s));
        }
        {
            ProfScope p(e, NDL_PROF_GEMM_DOWN);
            TRY(ndl_matmul_i8g32(e->qa, e->sa, rows, L.w_d, L.s_d, d, F, e->x, d, e->x, nullptr, s));
        }
    }
    if (heads > 0) {
        ProfScope p(e, NDL_PROF_HEAD);
        TRY(launch_gather_rows(e->x, d_head, heads, d, e->head_x, s));
        TRY(launch_quantize_rows(e->head_x, e->final_norm, heads, d, e->qa, e->sa, s));
        TRY(ndl_matmul_i8g32(e->qa, e->sa, heads, e->w_head, e->s_head, c.vocab, d, e->logits, c.vocab, nullptr,
                             nullptr, s));
    }
    return NDL_OK;
}

int launch_step_graph(ndl_engine *e, int rows, int heads) {
    for (auto &g : e->graphs)
        if (g.rows == rows && g.heads == heads) {
            g.last_use = ++e->graph_clock;
            NDL_CUDA(cudaGraphLaunch(g.exec, e->stream));
            return NDL_OK;
        }
    cudaGraph_t graph = nullptr;
    NDL_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    int st = step_kernels(e, rows, heads);
    cudaError_t end = cudaStreamEndCapture(e->stream, &graph);
    if (st != NDL_OK || end != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        if (st != NDL_OK) return st;
        return set_error(NDL_ERR_CUDA, "step capture: %s", cudaGetErrorString(end));
    }
    cudaGraphExec_t exec = nullptr;
    cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) return set_error(NDL_ERR_CUDA, "step graph: %s", cudaGetErrorString(inst));
    if (e->graphs.size() >= 16) {  // evict the least recently used shape
        auto lru = std::min_element(e->graphs.begin(), e->graphs.end(),
                                    [](const ndl_engine::StepGraph &x, const ndl_engine::StepGraph &y) {
                                        return x.last_use < y.last_use;
                                    });
        cudaGraphExecDestroy(lru->exec);
        e->graphs.erase(lru);
    }
    e->graphs.push_back({rows, heads, exec, ++e->graph_clock});
    NDL_CUDA(cudaGraphLaunch(exec, e->stream));
    return NDL_OK;
}

}  // namespace

extern "C" {

NDL_API int ndl_engine_create(const ndl_engine_config *ec, const ndl_decoder_config *dc, ndl_engine **out) {
    NDL_REQUIRE(ec && dc && out, "null argument");
    *out = nullptr;
    NDL_REQUIRE(dc->head_dim == kHeadDim, "head_dim must be %d", kHeadDim);
    NDL_REQUIRE(dc->layers >= 1 && dc->heads >= 1 && dc->dim == dc->heads * dc->head_dim,
                "dim must equal heads * head_dim");
    NDL_REQUIRE(dc->ffn >= 32 && dc->ffn % 32 == 0 && dc->dim % 32 == 0, "dim and ffn must be multiples of 32");
    NDL_REQUIRE(dc->vocab >= 1, "vocab must be positive");
    NDL_REQUIRE(ec->slots >= 1 && ec->capacity >= kPagePositions && ec->capacity % kPagePositions == 0,
                "capacity must be a positive multiple of %d", kPagePositions);
    if (ec->capacity > kAttnMaxPositions)
        return set_error(NDL_ERR_UNSUPPORTED, "capacity %d: attention holds at most %d positions per row",
                         ec->capacity, kAttnMaxPositions);
    NDL_REQUIRE(ec->max_rows >= 1 && ec->max_heads >= 1 && ec->max_heads <= ec->max_rows, "bad row limits");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || ec->device < 0 || ec->device >= count) {
        cudaGetLastError();
        return set_error(NDL_ERR_NO_DEVICE, "device %d not available", ec->device);
    }
    NDL_CUDA(cudaSetDevice(ec->device));
    ndl_engine *e = new ndl_engine();
    e->ec = *ec;
    e->dc = *dc;
    if (e->dc.rope_theta <= 0.0f) e->dc.rope_theta = 10000.0f;
    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete e;
        return set_error(NDL_ERR_CUDA, "stream: %s", cudaGetErrorString(err));
    }
    e->own_stream = true;
    e->max_pages = ec->capacity / kPagePositions;
    e->page_bytes = kv_page_bytes(dc->layers, dc->heads);
    int pages = ec->kv_pages > 0 ? ec->kv_pages : ec->slots * e->max_pages;
    e->ec.kv_pages = pages;
    int st = NDL_OK;
    if (st == NDL_OK) st = dalloc(e, &e->pool, (size_t)pages * e->page_bytes);
    if (st == NDL_OK) st = dalloc(e, &e->d_page_table, (size_t)ec->slots * e->max_pages);
    if (st == NDL_OK) st = build_weights(e);
    if (st == NDL_OK) st = build_buffers(e);
    if (st != NDL_OK) {
        ndl_engine_destroy(e);
        return st;
    }
    e->page_table.assign((size_t)ec->slots * e->max_pages, -1);
    cudaMemcpy(e->d_page_table, e->page_table.data(), e->page_table.size() * 4, cudaMemcpyHostToDevice);
    e->free_pages.resize(pages);
    for (int i = 0; i < pages; i++) e->free_pages[i] = pages - 1 - i;  // pop_back yields 0, 1, 2, ...
    e->page_refs.assign(pages, 0);
    e->slot_len.assign(ec->slots, 0);
    e->slot_mark.assign(ec->slots, 0);
    e->cross_slot.assign(ec->slots, -1);
    *out = e;
    return NDL_OK;
}

// A Needle-3 engine over a loaded .cact model (ndl_model_load with a device):
// its steps are the model's RunLayerBatch chain (needle3.cu); sampling, masks
// and logits work as for the synthetic decoder.
NDL_API int ndl_engine_create_model(const ndl_engine_config *ec, const ndl_model *m, ndl_engine **out) {
    NDL_REQUIRE(ec && m && out, "null argument");
    *out = nullptr;
    ndl_model_info info;
    int st = ndl_model_get_info(m, &info);
    if (st != NDL_OK) return st;
    NDL_REQUIRE(info.device >= 0, "the model is not on a device");
    NDL_REQUIRE(ec->device == info.device, "engine device %d, model device %d", ec->device, info.device);
    NDL_REQUIRE(ec->slots >= 1 && ec->capacity >= 1, "slots and capacity must be positive");
    NDL_REQUIRE(ec->max_rows >= 1 && ec->max_heads >= 1 && ec->max_heads <= ec->max_rows, "bad row limits");
    NDL_CUDA(cudaSetDevice(ec->device));
    ndl_engine *e = new ndl_engine();
    e->ec = *ec;
    e->dc = ndl_decoder_config{};
    e->dc.layers = info.layers;
    e->dc.dim = info.dim;
    e->dc.heads = info.heads;
    e->dc.head_dim = info.qk_dim;
    e->dc.vocab = info.vocab;
    cudaError_t err = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) {
        delete e;
        return set_error(NDL_ERR_CUDA, "stream: %s", cudaGetErrorString(err));
    }
    e->own_stream = true;
    e->use_graphs = false;
    st = ndl::n3_create(m, ec->slots, ec->capacity, ec->max_rows, ec->max_heads, e->stream, &e->n3);
    if (st == NDL_OK) {
        e->dc.vocab = ndl::n3_vocab(e->n3);
        st = build_sampling_buffers(e);
    }
    if (st != NDL_OK) {
        ndl_engine_destroy(e);
        return st;
    }
    e->slot_len.assign(ec->slots, 0);
    e->slot_mark.assign(ec->slots, 0);
    e->cross_slot.assign(ec->slots, -1);
    *out = e;
    return NDL_OK;
}

NDL_API int ndl_engine_destroy(ndl_engine *e) {
    if (!e) return NDL_OK;
    if (e->stream) cudaStreamSynchronize(e->stream);
    ndl::n3_destroy(e->n3);
    for (auto &g : e->graphs) cudaGraphExecDestroy(g.exec);
    for (cudaEvent_t ev : e->event_pool) cudaEventDestroy(ev);
    for (void *p : e->allocations) cudaFree(p);
    if (e->h_meta) cudaFreeHost(e->h_meta);
    if (e->h_out) cudaFreeHost(e->h_out);
    if (e->d_sparse) cudaFree(e->d_sparse);
    if (e->h_sparse) cudaFreeHost(e->h_sparse);
    if (e->d_prefix) cudaFree(e->d_prefix);
    if (e->own_stream && e->stream) cudaStreamDestroy(e->stream);
    delete e;
    return NDL_OK;
}

NDL_API int ndl_engine_stream(ndl_engine *e, void **stream) {
    NDL_REQUIRE(e && stream, "null argument");
    *stream = e->stream;
    return NDL_OK;
}

NDL_API int ndl_engine_tensor(ndl_engine *e, const char *name, int layer, void **ptr, size_t *bytes) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_engine_tensor");
    NDL_REQUIRE(e && name && ptr && bytes, "null argument");
    const ndl_decoder_config &c = e->dc;
    const size_t d = c.dim, F = c.ffn, V = c.vocab, G = d / 32, GF = F / 32;
    std::string n(name);
    if (layer >= 0) {
        NDL_REQUIRE(layer < c.layers, "layer %d out of range", layer);
        DeviceLayer &L = e->layers[layer];
        if (n == "w_qkv") { *ptr = L.w_qkv; *bytes = 3 * d * d; }
        else if (n == "s_qkv") { *ptr = L.s_qkv; *bytes = 3 * d * G * 2; }
        else if (n == "w_o") { *ptr = L.w_o; *bytes = d * d; }
        else if (n == "s_o") { *ptr = L.s_o; *bytes = d * G * 2; }
        else if (n == "w_gu") { *ptr = L.w_gu; *bytes = 2 * F * d; }
        else if (n == "s_gu") { *ptr = L.s_gu; *bytes = 2 * F * G * 2; }
        else if (n == "w_d") { *ptr = L.w_d; *bytes = d * F; }
        else if (n == "s_d") { *ptr = L.s_d; *bytes = d * GF * 2; }
        else if (n == "attn_norm") { *ptr = L.attn_norm; *bytes = d * 4; }
        else if (n == "ffn_norm") { *ptr = L.ffn_norm; *bytes = d * 4; }
        else if (c.cross && n == "w_cq") { *ptr = L.w_cq; *bytes = d * d; }
        else if (c.cross && n == "s_cq") { *ptr = L.s_cq; *bytes = d * G * 2; }
        else if (c.cross && n == "w_ckv") { *ptr = L.w_ckv; *bytes = 2 * d * d; }
        else if (c.cross && n == "s_ckv") { *ptr = L.s_ckv; *bytes = 2 * d * G * 2; }
        else if (c.cross && n == "w_co") { *ptr = L.w_co; *bytes = d * d; }
        else if (c.cross && n == "s_co") { *ptr = L.s_co; *bytes = d * G * 2; }
        else if (c.cross && n == "cross_norm") { *ptr = L.cross_norm; *bytes = d * 4; }
        else return set_error(NDL_ERR_INVALID_ARG, "unknown layer tensor '%s'", name);
        return NDL_OK;
    }
    if (n == "final_norm") { *ptr = e->final_norm; *bytes = d * 4; }
    else if (n == "embedding") { *ptr = e->embedding; *bytes = V * d * 2; }
    else if (n == "w_head") { *ptr = e->w_head; *bytes = V * d; }
    else if (n == "s_head") { *ptr = e->s_head; *bytes = V * G * 2; }
    else if (n == "rope_cos") { *ptr = e->rope_cos; *bytes = (size_t)e->ec.capacity * (c.head_dim / 2) * 4; }
    else if (n == "rope_sin") { *ptr = e->rope_sin; *bytes = (size_t)e->ec.capacity * (c.head_dim / 2) * 4; }
    else if (n == "kv_pool") { *ptr = e->pool; *bytes = (size_t)e->ec.kv_pages * e->page_bytes; }
    else if (n == "page_table") { *ptr = e->d_page_table; *bytes = e->page_table.size() * 4; }
    else if (n == "logits") { *ptr = e->logits; *bytes = (size_t)e->ec.max_heads * V * 4; }
    else return set_error(NDL_ERR_INVALID_ARG, "unknown tensor '%s'", name);
    return NDL_OK;
}

NDL_API int ndl_engine_read_tensor(ndl_engine *e, const char *name, int layer, void *host, size_t bytes) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_engine_read_tensor");
    void *ptr = nullptr;
    size_t have = 0;
    TRY(ndl_engine_tensor(e, name, layer, &ptr, &have));
    NDL_REQUIRE(host && bytes <= have, "read of %zu bytes from a %zu-byte tensor", bytes, have);
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    NDL_CUDA(cudaMemcpy(host, ptr, bytes, cudaMemcpyDeviceToHost));
    return NDL_OK;
}

NDL_API int ndl_engine_page_bytes(ndl_engine *e, size_t *bytes) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_engine_page_bytes");
    NDL_REQUIRE(e && bytes, "null argument");
    *bytes = e->page_bytes;
    return NDL_OK;
}

NDL_API int ndl_slot_length(ndl_engine *e, int slot, int *length) {
    TRY(check_slot(e, slot));
    NDL_REQUIRE(length, "length is NULL");
    *length = e->slot_len[slot];
    return NDL_OK;
}

NDL_API int ndl_slot_page(ndl_engine *e, int slot, int index, int *page) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_page");
    TRY(check_slot(e, slot));
    NDL_REQUIRE(page && index >= 0 && index < e->max_pages, "bad page index");
    *page = e->page_table[(size_t)slot * e->max_pages + index];
    return NDL_OK;
}

// EngineCore.ResetSlot (src/Needle/Engine.cs:2267-2271): empty the slot.
NDL_API int ndl_slot_reset(ndl_engine *e, int slot) {
    TRY(check_slot(e, slot));
    if (e->n3) {
        TRY(ndl::n3_reset_slot(e->n3, slot, e->stream));
        e->slot_len[slot] = 0;
        e->slot_mark[slot] = 0;
        return NDL_OK;
    }
    std::vector<int32_t> updates;
    free_slot_pages(e, slot, 0, &updates);
    e->slot_len[slot] = 0;
    e->slot_mark[slot] = 0;
    return push_page_updates(e, updates);
}

// EngineCore.MarkSlot (src/Needle/Engine.cs:2273-2277): remember the length.
NDL_API int ndl_slot_mark(ndl_engine *e, int slot) {
    TRY(check_slot(e, slot));
    if (e->n3) {
        TRY(ndl::n3_mark(e->n3, slot, e->stream));
        e->slot_mark[slot] = e->slot_len[slot];
        return NDL_OK;
    }
    e->slot_mark[slot] = e->slot_len[slot];
    return NDL_OK;
}

// EngineCore.RewindSlot (src/Needle/Engine.cs:2279-2283): back to the mark;
// pages wholly past the mark are returned to the pool.
NDL_API int ndl_slot_rewind(ndl_engine *e, int slot) {
    TRY(check_slot(e, slot));
    if (e->n3) {
        TRY(ndl::n3_rewind(e->n3, slot, e->stream));
        e->slot_len[slot] = e->slot_mark[slot];
        return NDL_OK;
    }
    std::vector<int32_t> updates;
    int keep = (e->slot_mark[slot] + kPagePositions - 1) / kPagePositions;
    free_slot_pages(e, slot, keep, &updates);
    e->slot_len[slot] = e->slot_mark[slot];
    return push_page_updates(e, updates);
}

// Fills positions [len, len+count) of a slot with the synthetic prefix K/V
// (fp16 N(0,1) quantized on load) and advances its length.
NDL_API int ndl_slot_fill_synthetic(ndl_engine *e, int slot, int count, uint64_t seed, uint64_t session) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_fill_synthetic");
    TRY(check_slot(e, slot));
    NDL_REQUIRE(count >= 0, "count < 0");
    int first = e->slot_len[slot];
    if (first + count > e->ec.capacity)
        return set_error(NDL_FAIL_CONTEXT_EXHAUSTED, "slot %d: %d + %d exceeds capacity %d", slot, first, count,
                         e->ec.capacity);
    std::vector<int32_t> updates, copies;
    for (int p = first / kPagePositions; p * kPagePositions < first + count; p++)
        if (writable_page(e, slot, p, updates, copies) < 0)
            return set_error(NDL_ERR_PAGES_EXHAUSTED, "KV page pool exhausted");
    TRY(copy_pages(e, copies));
    TRY(push_page_updates(e, updates));
    TRY(launch_kv_fill(seed, session, e->dc.layers, e->dc.heads, first, count,
                       e->d_page_table + (size_t)slot * e->max_pages, e->pool, (long long)e->page_bytes,
                       e->stream));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    e->slot_len[slot] = first + count;
    return NDL_OK;
}

namespace {

// Pages for positions [first, first + count) of a slot (host mirror + device table).
int reserve_pages(ndl_engine *e, int slot, int first, int count) {
    std::vector<int32_t> updates, copies;
    for (int p = first / kPagePositions; p * kPagePositions < first + count; p++)
        if (writable_page(e, slot, p, updates, copies) < 0)
            return set_error(NDL_ERR_PAGES_EXHAUSTED, "KV page pool exhausted");
    TRY(copy_pages(e, copies));
    return push_page_updates(e, updates);
}

// Builds the memory K/V of every layer from fp16 memory already on the device.
int build_memory(ndl_engine *e, int slot, const uint16_t *d_mem16, int frames) {
    const int d = e->dc.dim;
    cudaStream_t s = e->stream;
    TRY(reserve_pages(e, slot, 0, frames));
    float *mem = nullptr, *y = nullptr, *sa = nullptr;
    int8_t *q = nullptr;
    int st = NDL_OK;
    auto cleanup = [&]() {
        cudaStreamSynchronize(s);
        cudaFree(mem);
        cudaFree(y);
        cudaFree(sa);
        cudaFree(q);
    };
    if (cudaMalloc(&mem, (size_t)frames * d * 4) != cudaSuccess || cudaMalloc(&y, (size_t)frames * 2 * d * 4) != cudaSuccess ||
        cudaMalloc(&sa, (size_t)frames * 4) != cudaSuccess || cudaMalloc(&q, (size_t)frames * d) != cudaSuccess) {
        cudaGetLastError();
        cleanup();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "cross memory scratch (%d frames)", frames);
    }
    st = launch_half_to_float(d_mem16, (long long)frames * d, mem, s);
    if (st == NDL_OK) st = launch_quantize_rows(mem, nullptr, frames, d, q, sa, s);
    for (int l = 0; l < e->dc.layers && st == NDL_OK; l++) {
        const DeviceLayer &L = e->layers[l];
        st = ndl_matmul_i8g32(q, sa, frames, L.w_ckv, L.s_ckv, 2 * d, d, y, 2 * d, nullptr, nullptr, s);
        if (st == NDL_OK)
            st = launch_cross_kv_write(y, frames, e->dc.heads, e->d_page_table + (size_t)slot * e->max_pages,
                                       e->ec.kv_pages, e->pool, (long long)e->page_bytes, l, e->d_status, s);
    }
    cleanup();
    if (st != NDL_OK) return st;
    TRY(check_status(e));
    e->slot_len[slot] = frames;
    return NDL_OK;
}

int check_memory_slot(ndl_engine *e, int slot, int frames) {
    TRY(check_slot(e, slot));
    NDL_REQUIRE(e->dc.cross, "the decoder has no cross-attention blocks");
    NDL_REQUIRE(e->slot_len[slot] == 0, "memory slot %d is not empty", slot);
    NDL_REQUIRE(frames >= 1 && frames <= e->ec.capacity, "frames %d outside 1..%d", frames, e->ec.capacity);
    return NDL_OK;
}

}  // namespace

NDL_API int ndl_slot_set_memory(ndl_engine *e, int slot, const uint16_t *memory, int frames) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_set_memory");
    NDL_REQUIRE(e && memory, "null argument");
    TRY(check_memory_slot(e, slot, frames));
    const size_t bytes = (size_t)frames * e->dc.dim * 2;
    uint16_t *d_mem = nullptr;
    if (cudaMalloc(&d_mem, bytes) != cudaSuccess) {
        cudaGetLastError();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "cross memory upload (%zu bytes)", bytes);
    }
    int st = cudaMemcpyAsync(d_mem, memory, bytes, cudaMemcpyHostToDevice, e->stream) == cudaSuccess
                 ? build_memory(e, slot, d_mem, frames)
                 : set_error(NDL_ERR_CUDA, "cross memory upload failed");
    cudaStreamSynchronize(e->stream);
    cudaFree(d_mem);
    return st;
}

NDL_API int ndl_slot_fill_memory_synthetic(ndl_engine *e, int slot, int frames, uint64_t seed, uint64_t utterance) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_fill_memory_synthetic");
    NDL_REQUIRE(e, "null engine");
    TRY(check_memory_slot(e, slot, frames));
    const size_t count = (size_t)frames * e->dc.dim;
    uint16_t *d_mem = nullptr;
    if (cudaMalloc(&d_mem, count * 2) != cudaSuccess) {
        cudaGetLastError();
        return set_error(NDL_ERR_OUT_OF_MEMORY, "cross memory (%zu values)", count);
    }
    int st = ndl_synth_normal_f16_device(seed, kStreamMemory + utterance, 0, count, 1.0f, d_mem, e->stream);
    if (st == NDL_OK) st = build_memory(e, slot, d_mem, frames);
    cudaStreamSynchronize(e->stream);
    cudaFree(d_mem);
    return st;
}

NDL_API int ndl_slot_attach_memory(ndl_engine *e, int slot, int memory_slot) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_attach_memory");
    NDL_REQUIRE(e, "null engine");
    TRY(check_slot(e, slot));
    NDL_REQUIRE(e->dc.cross, "the decoder has no cross-attention blocks");
    NDL_REQUIRE(memory_slot >= -1 && memory_slot < e->ec.slots && memory_slot != slot, "memory slot %d",
                memory_slot);
    e->cross_slot[slot] = memory_slot;
    return NDL_OK;
}

NDL_API int ndl_slot_copy(ndl_engine *e, int dst, int src) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_copy");
    NDL_REQUIRE(e, "null engine");
    TRY(check_slot(e, dst));
    TRY(check_slot(e, src));
    if (dst == src) return NDL_OK;
    std::vector<int32_t> updates;
    free_slot_pages(e, dst, 0, &updates);
    TRY(push_page_updates(e, updates));
    const int len = e->slot_len[src];
    TRY(reserve_pages(e, dst, 0, len));
    const int32_t *rs = e->page_table.data() + (size_t)src * e->max_pages;
    const int32_t *rd = e->page_table.data() + (size_t)dst * e->max_pages;
    for (int p = 0; p * kPagePositions < len; p++)
        NDL_CUDA(cudaMemcpyAsync(e->pool + (size_t)rd[p] * e->page_bytes, e->pool + (size_t)rs[p] * e->page_bytes,
                                 e->page_bytes, cudaMemcpyDeviceToDevice, e->stream));
    e->slot_len[dst] = len;
    e->slot_mark[dst] = e->slot_mark[src];
    e->cross_slot[dst] = e->cross_slot[src];
    return NDL_OK;
}

// EngineCore.ForwardBatch (src/Needle/Engine.cs:2303-2350).
NDL_API int ndl_forward_batch(ndl_engine *e, const int *tokens, const int *row_slots, int rows, const int *head_rows,
                              int heads) {
    NDL_REQUIRE(e, "engine is NULL");
    NDL_REQUIRE(rows >= 1 && rows <= e->ec.max_rows, "rows %d outside 1..%d", rows, e->ec.max_rows);
    NDL_REQUIRE(heads >= 0 && heads <= e->ec.max_heads && heads <= rows, "heads %d out of range", heads);
    NDL_REQUIRE(tokens && row_slots && (heads == 0 || head_rows), "null argument");
    if (e->n3) {
        int st = ndl::n3_forward(e->n3, e->stream, tokens, row_slots, rows, head_rows, heads, e->logits);
        if (st != NDL_OK) return st;
        for (int r = 0; r < rows; r++) e->slot_len[row_slots[r]]++;
        e->last_rows = rows;
        e->last_heads = heads;
        return NDL_OK;  // no Needle-3 kernel reports through the status word: nothing to wait for here
    }
    const ndl_decoder_config &c = e->dc;
    // positions, capacity check, page allocation (host)
    int32_t *m = e->h_meta;
    const int R = e->ec.max_rows;
    e->off_tokens = 0, e->off_slot = R, e->off_pos = 2 * R, e->off_order = 3 * R, e->off_cslot = 4 * R,
    e->off_cpos = 5 * R, e->off_head = 6 * R;
    e->off_updates = 6 * R + e->ec.max_heads;
    std::vector<int> advance;
    advance.reserve(rows);
    int max_len = 0;
    for (int r = 0; r < rows; r++) {
        int slot = row_slots[r];
        if (slot < 0 || slot >= e->ec.slots) return set_error(NDL_ERR_INVALID_ARG, "row %d: slot %d", r, slot);
        if (tokens[r] < 0 || tokens[r] >= c.vocab) return set_error(NDL_ERR_INVALID_ARG, "row %d: token %d", r, tokens[r]);
        int offset = (r > 0 && row_slots[r - 1] == slot) ? (m[e->off_pos + r - 1] - e->slot_len[slot] + 1) : 0;
        if (r > 0 && row_slots[r - 1] != slot)
            for (int q = 0; q < r; q++)
                if (row_slots[q] == slot) return set_error(NDL_ERR_INVALID_ARG, "slot %d rows are not consecutive", slot);
        int pos = e->slot_len[slot] + offset;
        if (pos >= e->ec.capacity)
            return set_error(NDL_FAIL_CONTEXT_EXHAUSTED, "slot %d: context capacity %d exceeded", slot, e->ec.capacity);
        m[e->off_tokens + r] = tokens[r];
        m[e->off_slot + r] = slot;
        m[e->off_pos + r] = pos;
        if (c.cross) {
            const int ms = e->cross_slot[slot];
            if (ms < 0 || e->slot_len[ms] < 1)
                return set_error(NDL_ERR_INVALID_ARG, "slot %d has no cross memory attached", slot);
            m[e->off_cslot + r] = ms;
            m[e->off_cpos + r] = e->slot_len[ms] - 1;
        }
        max_len = std::max(max_len, pos + 1);
    }
    for (int h = 0; h < heads; h++) {
        if (head_rows[h] < 0 || head_rows[h] >= rows) return set_error(NDL_ERR_INVALID_ARG, "head row %d", head_rows[h]);
        m[e->off_head + h] = head_rows[h];
    }
    // pages for the new positions; updates region = [count, (slot, index, page)...]
    // (a page another slot shares is copied first: copy on write)
    std::vector<int32_t> updates, copies;
    for (int r = 0; r < rows; r++)
        if (writable_page(e, m[e->off_slot + r], m[e->off_pos + r] / kPagePositions, updates, copies) < 0)
            return set_error(NDL_ERR_PAGES_EXHAUSTED, "KV page pool exhausted");
    const int n_updates = (int)(updates.size() / 3);
    int32_t *upd = m + e->off_updates;
    std::copy(updates.begin(), updates.end(), upd + 1);
    upd[0] = n_updates;
    TRY(copy_pages(e, copies));
    // longest rows first (LPT order for the attention work list)
    std::vector<int> order(rows);
    for (int r = 0; r < rows; r++) order[r] = r;
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return m[e->off_pos + a] > m[e->off_pos + b]; });
    for (int r = 0; r < rows; r++) m[e->off_order + r] = order[r];
    size_t meta_bytes = (size_t)(e->off_updates + 1 + 3 * n_updates) * sizeof(int32_t);
    NDL_CUDA(cudaMemcpyAsync(e->d_meta, m, meta_bytes, cudaMemcpyHostToDevice, e->stream));
    TRY(e->use_graphs && !e->profile ? launch_step_graph(e, rows, heads) : step_kernels(e, rows, heads));
    // bookkeeping (src/Needle/Engine.cs:2327-2340): lengths advance per slot run
    for (int r = 0; r < rows; r++) e->slot_len[m[e->off_slot + r]] = m[e->off_pos + r] + 1;
    e->last_rows = rows;
    e->last_heads = heads;
    return NDL_OK;
}

NDL_API int ndl_engine_use_pdl(ndl_engine *e, int enable) {
    NDL_REQUIRE(e, "engine is NULL");
    e->use_pdl = enable != 0;
    for (auto &g : e->graphs) cudaGraphExecDestroy(g.exec);  // graphs captured the old launch form
    e->graphs.clear();
    return NDL_OK;
}

NDL_API int ndl_engine_use_graphs(ndl_engine *e, int enable) {
    NDL_REQUIRE(e, "engine is NULL");
    e->use_graphs = enable != 0;
    return NDL_OK;
}

NDL_API int ndl_engine_profile(ndl_engine *e, int enable) {
    NDL_REQUIRE(e, "engine is NULL");
    e->profile = enable != 0;
    return NDL_OK;
}

NDL_API int ndl_engine_profile_read(ndl_engine *e, double *ms, long long *launches, int reset) {
    NDL_REQUIRE(e, "engine is NULL");
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    for (auto &pr : e->pending) {
        float t = 0.0f;
        NDL_CUDA(cudaEventElapsedTime(&t, e->event_pool[pr.second], e->event_pool[pr.second + 1]));
        e->prof_ms[pr.first] += t;
        e->prof_count[pr.first] += 1;
    }
    e->pending.clear();
    e->events_used = 0;
    for (int i = 0; i < NDL_PROF_CLASSES; i++) {
        if (ms) ms[i] = e->prof_ms[i];
        if (launches) launches[i] = e->prof_count[i];
        if (reset) e->prof_ms[i] = 0.0, e->prof_count[i] = 0;
    }
    return NDL_OK;
}

NDL_API int ndl_engine_sync(ndl_engine *e) {
    NDL_REQUIRE(e, "engine is NULL");
    return check_status(e);
}

// BatchedEngine.BatchLogitsRow (src/Needle/BatchEngine.cs:37): host copy of
// the logits of one compact head row of the last forward_batch.
NDL_API int ndl_batch_logits_row(ndl_engine *e, int compact_row, float *out) {
    NDL_REQUIRE(e && out, "null argument");
    NDL_REQUIRE(compact_row >= 0 && compact_row < e->last_heads, "compact row %d out of range", compact_row);
    NDL_CUDA(cudaMemcpyAsync(out, e->logits + (size_t)compact_row * e->dc.vocab, (size_t)e->dc.vocab * 4,
                             cudaMemcpyDeviceToHost, e->stream));
    return check_status(e);
}

// Greedy / grammar-masked selection over the head rows of the last step:
// Ops.ArgMaxMasked / ArgMaxMaskedWithProbability (src/Needle/Ops.cs:1223-1330).
// masks: host [heads][words] (NULL = everything allowed); probs nullable.
NDL_API int ndl_sample_argmax(ndl_engine *e, const uint32_t *masks, int words, int *ids, float *probs) {
    NDL_REQUIRE(e && ids, "null argument");
    const int n = e->last_heads, V = e->dc.vocab;
    if (n == 0) return NDL_OK;
    const int max_words = (V + 31) / 32;
    NDL_REQUIRE(!masks || (words >= 1 && words <= max_words), "words %d outside 1..%d", words, max_words);
    cudaStream_t s = e->stream;
    uint8_t *h = static_cast<uint8_t *>(e->h_out);
    if (masks) {
        memcpy(h + (size_t)e->ec.max_heads * 96, masks, (size_t)n * words * 4);
        NDL_CUDA(cudaMemcpyAsync(e->d_masks, h + (size_t)e->ec.max_heads * 96, (size_t)n * words * 4,
                                 cudaMemcpyHostToDevice, s));
    }
    {
        ProfScope p(e, NDL_PROF_SAMPLE);
        TRY(launch_argmax_masked(e->logits, V, masks ? e->d_masks : nullptr, words, words, nullptr, V, n, e->d_ids,
                                 probs ? e->d_probs : nullptr, s));
    }
    NDL_CUDA(cudaMemcpyAsync(h, e->d_ids, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    if (probs) NDL_CUDA(cudaMemcpyAsync(h + (size_t)n * 4, e->d_probs, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    TRY(check_status(e));
    memcpy(ids, h, (size_t)n * 4);
    if (probs) memcpy(probs, h + (size_t)n * 4, (size_t)n * 4);
    return NDL_OK;
}

NDL_API int ndl_engine_get_info(ndl_engine *e, ndl_engine_info *info) {
    NDL_REQUIRE(e && info, "null argument");
    *info = ndl_engine_info{e->ec.slots, e->ec.capacity, e->dc.vocab, e->ec.max_rows, e->ec.max_heads,
                            e->dc.layers, e->dc.dim, e->dc.heads};
    return NDL_OK;
}

// Times the last step's self-attention launch of `layer` alone: `reps`
// back-to-back launches (the step's rows, KV pages and work list) between
// two events on the engine stream; *ms = the average launch.  A measurement
// aid for the attention roofline: the launches rewrite the step's scratch
// outputs (the query is the last layer's), nothing a later step reads.
NDL_API int ndl_engine_time_attention(ndl_engine *e, int layer, int reps, float *ms) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_engine_time_attention");
    NDL_REQUIRE(e && ms, "null argument");
    NDL_REQUIRE(e->last_rows > 0, "no step has run");
    NDL_REQUIRE(layer >= 0 && layer < e->dc.layers && reps >= 1, "layer %d / reps %d out of range", layer, reps);
    const int rows = e->last_rows;
    const int32_t *d_slot = e->d_meta + e->off_slot, *d_pos = e->d_meta + e->off_pos;
    const int32_t *d_order = e->d_meta + e->off_order;
    const AttnArgs aa{e->q8, e->qs, d_slot, d_pos, d_order, e->d_page_table, e->max_pages, e->pool,
                      (long long)e->page_bytes, e->ec.kv_pages, layer, e->dc.heads, rows,
                      1.0f / sqrtf((float)e->dc.head_dim), e->attn, e->d_status, e->ec.slots, e->qa, e->sa,
                      e->attn_work, e->n_work};
    cudaEvent_t t0 = nullptr, t1 = nullptr;
    NDL_CUDA(cudaEventCreate(&t0));
    NDL_CUDA(cudaEventCreate(&t1));
    int st = cudaEventRecord(t0, e->stream) == cudaSuccess ? NDL_OK : set_error(NDL_ERR_CUDA, "event record");
    for (int r = 0; r < reps && st == NDL_OK; r++) st = launch_attn_decode(aa, e->stream, false, false);
    float total = 0.0f;
    if (st == NDL_OK && (cudaEventRecord(t1, e->stream) != cudaSuccess || cudaEventSynchronize(t1) != cudaSuccess ||
                         cudaEventElapsedTime(&total, t0, t1) != cudaSuccess))
        st = set_error(NDL_ERR_CUDA, "attention timing events");
    cudaEventDestroy(t0);
    cudaEventDestroy(t1);
    TRY(st);
    *ms = total / reps;
    return check_status(e);
}

// Pool pages not held by any slot.
NDL_API int ndl_engine_free_pages(ndl_engine *e, int *free_pages) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_engine_free_pages");
    NDL_REQUIRE(e && free_pages, "null argument");
    *free_pages = (int)e->free_pages.size();
    return NDL_OK;
}

// Engine.PrimedPrefixBytes (src/Needle/Engine.cs:398-400): bytes of the blob
// of the slot's marked prefix (its length at ndl_slot_mark).
NDL_API int ndl_slot_prefix_bytes(ndl_engine *e, int slot, size_t *bytes) {
    NDL_REQUIRE(e && bytes, "null argument");
    TRY(check_slot(e, slot));
    if (e->n3) {
        *bytes = ndl::n3_prefix_bytes(e->n3, e->slot_mark[slot]);
        return NDL_OK;
    }
    *bytes = prefix_blob_bytes(e->dc.layers, e->dc.heads, e->slot_mark[slot]);
    return NDL_OK;
}

// Engine.ExportPrimedPrefix (src/Needle/Engine.cs:402-427): the slot's
// marked prefix as a blob (layout in prefix.cu).
NDL_API int ndl_slot_export_prefix(ndl_engine *e, int slot, void *blob, size_t bytes) {
    NDL_REQUIRE(e && blob, "null argument");
    TRY(check_slot(e, slot));
    const int len = e->slot_mark[slot];
    if (e->n3) {
        const size_t n3_need = ndl::n3_prefix_bytes(e->n3, len);
        NDL_REQUIRE(bytes >= n3_need, "primed prefix buffer too small (%zu bytes, %zu needed)", bytes, n3_need);
        *static_cast<int32_t *>(blob) = len;
        return ndl::n3_prefix_move(e->n3, slot, true, static_cast<uint8_t *>(blob), len, e->stream);
    }
    const size_t need = prefix_blob_bytes(e->dc.layers, e->dc.heads, len);
    NDL_REQUIRE(bytes >= need, "primed prefix buffer too small (%zu bytes, %zu needed)", bytes, need);
    *static_cast<int32_t *>(blob) = len;
    if (len == 0) return NDL_OK;
    TRY(prefix_reserve(e, need));
    uint8_t *stage = e->d_prefix;
    TRY(launch_prefix_move(true, e->dc.layers, e->dc.heads, len, e->d_page_table + (size_t)slot * e->max_pages,
                           e->pool, (long long)e->page_bytes, e->ec.kv_pages, stage, e->d_status, e->stream));
    if (cudaMemcpyAsync(static_cast<uint8_t *>(blob) + 4, stage + 4, need - 4, cudaMemcpyDeviceToHost, e->stream) !=
        cudaSuccess)
        return set_error(NDL_ERR_CUDA, "primed prefix download failed");
    return check_status(e);
}

// Engine.ImportPrimedPrefix (src/Needle/Engine.cs:429-464): the slot's cache
// becomes the blob's prefix; its length and mark are the blob's length.
NDL_API int ndl_slot_import_prefix(ndl_engine *e, int slot, const void *blob, size_t bytes) {
    NDL_REQUIRE(e && blob, "null argument");
    TRY(check_slot(e, slot));
    NDL_REQUIRE(bytes >= 4, "primed prefix is truncated");
    const int len = *static_cast<const int32_t *>(blob);
    NDL_REQUIRE(len >= 0 && len <= e->ec.capacity, "primed prefix length exceeds context capacity");
    if (e->n3) {
        NDL_REQUIRE(bytes >= ndl::n3_prefix_bytes(e->n3, len), "primed prefix is truncated");
        TRY(ndl_slot_reset(e, slot));
        TRY(ndl::n3_prefix_move(e->n3, slot, false, static_cast<uint8_t *>(const_cast<void *>(blob)), len, e->stream));
        e->slot_len[slot] = len;
        e->slot_mark[slot] = len;
        return NDL_OK;
    }
    const size_t need = prefix_blob_bytes(e->dc.layers, e->dc.heads, len);
    NDL_REQUIRE(bytes >= need, "primed prefix is truncated");
    TRY(ndl_slot_reset(e, slot));
    if (len > 0) {
        TRY(reserve_pages(e, slot, 0, len));
        TRY(prefix_reserve(e, need));
        uint8_t *stage = e->d_prefix;
        if (cudaMemcpyAsync(stage, blob, need, cudaMemcpyHostToDevice, e->stream) != cudaSuccess)
            return set_error(NDL_ERR_CUDA, "primed prefix upload failed");
        TRY(launch_prefix_move(false, e->dc.layers, e->dc.heads, len, e->d_page_table + (size_t)slot * e->max_pages,
                               e->pool, (long long)e->page_bytes, e->ec.kv_pages, stage, e->d_status, e->stream));
        TRY(check_status(e));  // the blob is consumed once this returns
    }
    e->slot_len[slot] = len;
    e->slot_mark[slot] = len;
    return NDL_OK;
}

// Prefix sharing: `dst` takes `src`'s marked prefix by reference.  Whole
// pages are shared (one more reference each); the partial last page is
// copied.  A later write into a shared page copies it first (copy on write),
// so neither slot sees the other's new positions.
NDL_API int ndl_slot_share_prefix(ndl_engine *e, int dst, int src) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_slot_share_prefix");
    NDL_REQUIRE(e, "null engine");
    TRY(check_slot(e, dst));
    TRY(check_slot(e, src));
    NDL_REQUIRE(dst != src, "slot %d cannot share its own prefix", dst);
    const int len = e->slot_mark[src];
    TRY(ndl_slot_reset(e, dst));
    std::vector<int32_t> updates, copies;
    const int32_t *rs = e->page_table.data() + (size_t)src * e->max_pages;
    int32_t *rd = e->page_table.data() + (size_t)dst * e->max_pages;
    const int whole = len / kPagePositions;
    for (int p = 0; p < whole; p++) {
        rd[p] = rs[p];
        e->page_refs[rs[p]]++;
        updates.insert(updates.end(), {dst, p, rd[p]});
    }
    if (len % kPagePositions) {
        const int page = alloc_page(e);
        if (page < 0) {
            push_page_updates(e, updates);
            return set_error(NDL_ERR_PAGES_EXHAUSTED, "KV page pool exhausted");
        }
        copies.insert(copies.end(), {rs[whole], page});
        rd[whole] = page;
        updates.insert(updates.end(), {dst, whole, page});
    }
    TRY(copy_pages(e, copies));
    TRY(push_page_updates(e, updates));
    e->slot_len[dst] = len;
    e->slot_mark[dst] = len;
    e->cross_slot[dst] = e->cross_slot[src];
    return NDL_OK;
}

// Stores a vocabulary bitmask for `slot` on the device (NULL clears it):
// the scheduler uploads a request's mask once instead of every step.
NDL_API int ndl_engine_set_mask(ndl_engine *e, int slot, const uint32_t *mask, int words) {
    NDL_REQUIRE(e, "null engine");
    TRY(check_slot(e, slot));
    const int max_words = (e->dc.vocab + 31) / 32;
    if (!mask) {
        if (!e->slot_has_mask.empty()) e->slot_has_mask[slot] = 0;
        return NDL_OK;
    }
    NDL_REQUIRE(words >= 1 && words <= max_words, "words %d outside 1..%d", words, max_words);
    if (!e->d_mask_table) {
        TRY(dalloc(e, &e->d_mask_table, (size_t)e->ec.slots * max_words));
        TRY(dalloc(e, &e->d_mask_index, (size_t)e->ec.max_heads));
        e->slot_has_mask.assign(e->ec.slots, 0);
    }
    uint32_t *row = e->d_mask_table + (size_t)slot * max_words;
    NDL_CUDA(cudaMemsetAsync(row, 0, (size_t)max_words * 4, e->stream));
    // pageable source: the copy completes before the call returns
    NDL_CUDA(cudaMemcpyAsync(row, mask, (size_t)words * 4, cudaMemcpyHostToDevice, e->stream));
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    e->slot_has_mask[slot] = 1;
    return NDL_OK;
}

// Grows the sparse-head staging buffers to hold `total` ids: rows, offsets,
// picks and probs (max_heads + 1 words each), then ids and values.
static int sparse_reserve(ndl_engine *e, size_t total) {
    const size_t bytes = ((size_t)4 * (e->ec.max_heads + 1) + 2 * total) * 4;
    if (bytes <= e->sparse_bytes) return NDL_OK;
    NDL_CUDA(cudaStreamSynchronize(e->stream));
    if (e->d_sparse) cudaFree(e->d_sparse);
    if (e->h_sparse) cudaFreeHost(e->h_sparse);
    e->d_sparse = e->h_sparse = nullptr;
    e->sparse_bytes = 0;
    NDL_CUDA(cudaMalloc(&e->d_sparse, bytes));
    NDL_CUDA(cudaMallocHost(&e->h_sparse, bytes));
    e->sparse_bytes = bytes;
    return NDL_OK;
}

// Engine.LogitsForBatchRow (src/Needle/Engine.cs:2683-2700) for a batch of
// requests, with ArgMaxSparse (src/Needle/NeedleSession.cs:984-995) on top:
// request r wants batch row rows[r] of the last forward_batch at the
// vocabulary ids ids[offsets[r] .. offsets[r+1]).  One gather + final-norm
// quantize of the requested rows (the dense head's kernels), one sparse
// row-dot launch, one argmax launch.
NDL_API int ndl_logits_sparse(ndl_engine *e, int n, const int *rows, const int *offsets, const int *ids,
                              float *values, int *picks, float *probs) {
    if (e && e->n3) return set_error(NDL_ERR_UNSUPPORTED, "%s: not available on a Needle-3 engine", "ndl_logits_sparse");
    NDL_REQUIRE(e, "engine is NULL");
    const int Hd = e->ec.max_heads, V = e->dc.vocab, d = e->dc.dim;
    NDL_REQUIRE(n >= 0 && n <= Hd, "%d requests outside 0..%d", n, Hd);
    NDL_REQUIRE(!probs || picks, "probs need picks");
    if (n == 0) return NDL_OK;
    NDL_REQUIRE(rows && offsets, "null argument");
    NDL_REQUIRE(e->last_rows > 0, "no step has run");
    NDL_REQUIRE(offsets[0] == 0, "offsets[0] = %d, not 0", offsets[0]);
    for (int r = 0; r < n; r++) {
        NDL_REQUIRE(rows[r] >= 0 && rows[r] < e->last_rows, "request %d: row %d outside the last step's %d rows", r,
                    rows[r], e->last_rows);
        NDL_REQUIRE(offsets[r + 1] >= offsets[r], "offsets decrease at request %d", r);
    }
    const int total = offsets[n];
    NDL_REQUIRE(total == 0 || ids, "null ids");
    for (int t = 0; t < total; t++) NDL_REQUIRE(ids[t] >= 0 && ids[t] < V, "id %d outside the vocabulary", ids[t]);
    TRY(sparse_reserve(e, (size_t)total));
    cudaStream_t s = e->stream;
    int32_t *h_rows = static_cast<int32_t *>(e->h_sparse), *d_rows = static_cast<int32_t *>(e->d_sparse);
    const size_t o_off = Hd + 1, o_picks = 2 * o_off, o_probs = 3 * o_off, o_ids = 4 * o_off, o_vals = o_ids + total;
    memcpy(h_rows, rows, (size_t)n * 4);
    memcpy(h_rows + o_off, offsets, (size_t)(n + 1) * 4);
    if (total) memcpy(h_rows + o_ids, ids, (size_t)total * 4);
    NDL_CUDA(cudaMemcpyAsync(d_rows, h_rows, o_vals * 4, cudaMemcpyHostToDevice, s));
    float *d_vals = reinterpret_cast<float *>(d_rows + o_vals);
    {
        ProfScope p(e, NDL_PROF_HEAD);
        TRY(launch_gather_rows(e->x, d_rows, n, d, e->head_x, s));
        TRY(launch_quantize_rows(e->head_x, e->final_norm, n, d, e->qa, e->sa, s));
        TRY(launch_sparse_head(e->w_head, e->s_head, V, d, e->qa, e->sa, d_rows + o_off, n, d_rows + o_ids, total,
                               d_vals, e->d_status, s));
    }
    if (picks) {
        ProfScope p(e, NDL_PROF_SAMPLE);
        TRY(launch_sparse_argmax(d_vals, d_rows + o_off, d_rows + o_ids, n, d_rows + o_picks,
                                 probs ? reinterpret_cast<float *>(d_rows + o_probs) : nullptr, s));
        NDL_CUDA(cudaMemcpyAsync(h_rows + o_picks, d_rows + o_picks, (size_t)2 * o_off * 4, cudaMemcpyDeviceToHost, s));
    }
    if (values && total)
        NDL_CUDA(cudaMemcpyAsync(h_rows + o_vals, d_vals, (size_t)total * 4, cudaMemcpyDeviceToHost, s));
    TRY(check_status(e));
    if (values && total) memcpy(values, h_rows + o_vals, (size_t)total * 4);
    if (picks) memcpy(picks, h_rows + o_picks, (size_t)n * 4);
    if (probs) memcpy(probs, h_rows + o_probs, (size_t)n * 4);
    return NDL_OK;
}

// ArgMaxMasked over every head row of the last step, each row masked by the
// stored mask of slots[h] (negative, or a slot without a mask: unmasked).
NDL_API int ndl_sample_argmax_slots(ndl_engine *e, const int *slots, int *ids, float *probs) {
    NDL_REQUIRE(e && slots && ids, "null argument");
    const int n = e->last_heads, V = e->dc.vocab, max_words = (V + 31) / 32;
    if (n == 0) return NDL_OK;
    cudaStream_t s = e->stream;
    uint8_t *h = static_cast<uint8_t *>(e->h_out);
    int32_t *hidx = reinterpret_cast<int32_t *>(h + (size_t)e->ec.max_heads * 96);
    bool any = false;
    for (int i = 0; i < n; i++) {
        const int sl = slots[i];
        NDL_REQUIRE(sl < e->ec.slots, "head %d: slot %d out of range", i, sl);
        hidx[i] = (sl >= 0 && !e->slot_has_mask.empty() && e->slot_has_mask[sl]) ? sl : -1;
        any = any || hidx[i] >= 0;
    }
    if (any) NDL_CUDA(cudaMemcpyAsync(e->d_mask_index, hidx, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    {
        ProfScope p(e, NDL_PROF_SAMPLE);
        TRY(launch_argmax_masked(e->logits, V, any ? e->d_mask_table : nullptr, max_words, max_words,
                                 any ? e->d_mask_index : nullptr, V, n, e->d_ids, probs ? e->d_probs : nullptr, s));
    }
    NDL_CUDA(cudaMemcpyAsync(h, e->d_ids, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    if (probs) NDL_CUDA(cudaMemcpyAsync(h + (size_t)n * 4, e->d_probs, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    TRY(check_status(e));
    memcpy(ids, h, (size_t)n * 4);
    if (probs) memcpy(probs, h + (size_t)n * 4, (size_t)n * 4);
    return NDL_OK;
}

// Beam expansion: Ops.TopKLogSoftmax (src/Needle/Ops.cs:1092-1221) on every
// head row of the last step.  Outputs [heads][k] on the host.
NDL_API int ndl_sample_topk(ndl_engine *e, int k, int mask_special_023, int *ids, float *log_probs, float *probs) {
    NDL_REQUIRE(e && ids && log_probs, "null argument");
    NDL_REQUIRE(k >= 1 && k <= 8, "k=%d outside 1..8", k);
    const int n = e->last_heads;
    if (n == 0) return NDL_OK;
    cudaStream_t s = e->stream;
    {
        ProfScope p(e, NDL_PROF_SAMPLE);
        TRY(launch_topk_logsoftmax(e->logits, e->dc.vocab, e->dc.vocab, k, mask_special_023, n, e->d_ids, e->d_logp,
                                   probs ? e->d_probs : nullptr, s));
    }
    uint8_t *h = static_cast<uint8_t *>(e->h_out);
    size_t b = (size_t)n * k * 4;
    NDL_CUDA(cudaMemcpyAsync(h, e->d_ids, b, cudaMemcpyDeviceToHost, s));
    NDL_CUDA(cudaMemcpyAsync(h + b, e->d_logp, b, cudaMemcpyDeviceToHost, s));
    if (probs) NDL_CUDA(cudaMemcpyAsync(h + 2 * b, e->d_probs, b, cudaMemcpyDeviceToHost, s));
    TRY(check_status(e));
    memcpy(ids, h, b);
    memcpy(log_probs, h + b, b);
    if (probs) memcpy(probs, h + 2 * b, b);
    return NDL_OK;
}

}  // extern "C"
