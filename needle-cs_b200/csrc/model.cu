// The Needle-3 model archive (.cact) for the device.  This is the reference's
// loader: Model's constructor (src/Needle/Model.cs:307-361), RequireWellFormed
// (:365-384) and Reader (:200-283).  It is restated here as a host walk over
// the record table that names every tensor by its role ("layer.q", index =
// layer), with the reference's checks and messages.  Weights go up in one
// device allocation, in the forms the device kernels take:
//  * CQ matrices: their index and fp16 norm bytes as stored, with the two
//    codebooks filled on the host (Codebook.Fill, :44-52);
//  * dense tensors: fp32, fp16 records converted by the reference's rule
//    (Scalar.HalfToSingle, or HalfToSingleUpstream for the part of an
//    audio-carrying archive before its audio section, Scalar.cs:113-128);
//  * permutations: int32;
//  * the probe heads' CQ matrices: also decoded to fp32 rows (Reader.Rows) by
//    the GatherRow kernel.
// The checks the reference does not make, and this loader does, because a
// bad value would otherwise become an out-of-range device access:
//  * the walk stays inside the table;
//  * a tensor's elements fit its bytes;
//  * the codebook holds the 28 levels the two books read;
//  * a permutation entry lies in [0, HadaN).
// An audio section (Whistle's encoder, an archive whose next record after the
// final norm is the 13-entry fp32 vector) is kept as untyped records
// ("audio", index = position in the section).
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"

#define TRY(x)                         \
    do {                               \
        int st_ = (x);                 \
        if (st_ != NDL_OK) return st_; \
    } while (0)

namespace ndl {
namespace {

constexpr uint32_t kCactMagic = 0x05E12A84u;  // ModelInfo.SupportedMagic (src/Needle/ModelInfo.cs:7)
constexpr uint64_t kCactHeaderBytes = 196;     // ModelInfo.HeaderBytes (src/Needle/ModelInfo.cs:8)
constexpr const char *kGuidance =              // ModelInfo.RefreshGuidance (src/Needle/ModelInfo.cs:9)
    "If the upstream model changed, see CONTRIBUTING.md, section \"Refreshing the upstream model\".";
constexpr int kCqGroupCols = 128;   // Cq.GroupSize
constexpr int kCodebookLevels = 28;  // the 2-bit book reads levels 0..3, the 4-bit book levels 12..27
constexpr int kMaxProbeHeads = 16;

// Record (src/Needle/Model.cs:191-198), byte for byte.
#pragma pack(push, 1)
struct CactRecord {
    uint8_t dtype, ndim;
    uint16_t pad;
    uint32_t shape[4];
    uint64_t offset, bytes;
    uint32_t group, bits;
};
#pragma pack(pop)
static_assert(sizeof(CactRecord) == 44, "the archive's record is 44 bytes");

enum : uint8_t { kTypeFp16 = 1, kTypeFp32 = 2, kTypeCq = 3, kTypeRaw = 4 };  // Reader.Fp16 .. Raw

struct Entry {
    std::string role;
    int index = 0, record = 0, kind = NDL_TENSOR_DENSE;
    int64_t count = 0;         // elements: dense, permutation, decoded rows
    int rows = 0, cols = 0, bits = 0;
    size_t index_bytes = 0, norm_bytes = 0;
    std::vector<float> dense;  // host fp32 (dense)
    std::vector<int32_t> perm;
    size_t at_values = 0, at_perm = 0, at_indices = 0, at_norms = 0;  // offsets in the device block
};

// Scalar.HalfToSingle and Scalar.HalfToSingleUpstream (src/Needle/Scalar.cs:113-128):
// both map a zero magnitude to +0 and give exponent 31 no special meaning;
// the exact one scales subnormals, the upstream one treats them as normal.
float half_to_single(uint16_t half, bool exact) {
    const uint32_t magnitude = half & 0x7FFFu;
    if (magnitude == 0) return 0.0f;
    if (exact && magnitude < 0x0400u) {
        const float v = (float)magnitude * 5.9604645e-8f;
        return (half & 0x8000u) ? -v : v;
    }
    const uint32_t bits = ((magnitude << 13) + 0x38000000u) | ((uint32_t)(half & 0x8000u) << 16);
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

// Codebook.Fill (src/Needle/Model.cs:44-52): byte levels rounded half to even.
void fill_codebook(ndl_kt_codebook *book, const float *levels, int count) {
    float peak = 0.0f;
    for (int i = 0; i < count; i++) peak = fmaxf(peak, fabsf(levels[i]));
    book->byte_scale = peak / 63.0f;
    for (int i = 0; i < 16; i++) book->levels[i] = levels[i % count];
    for (int i = 0; i < 32; i++) {
        uint8_t b = 0;
        if (i % 16 < count) {
            const float r = rintf(levels[i % 16] / book->byte_scale) + 63.0f;
            b = isfinite(r) ? (uint8_t)(int)r : 0;
        }
        book->bytes[i] = b;
    }
}

// (uint)value's bit length (BitMath.BitLength, src/Needle/Model.cs:54-62).
int bit_length(uint32_t v) {
    int bits = 0;
    for (; v; v >>= 1) bits++;
    return bits;
}

}  // namespace
}  // namespace ndl

using namespace ndl;

struct ndl_model {
    ndl_model_info info{};
    std::vector<CactRecord> records;
    std::vector<Entry> entries;
    ndl_kt_codebook book2{}, book4{};
    std::vector<uint8_t> tokenizer;
    uint8_t *block = nullptr;
};

namespace ndl {
namespace {

int malformed(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
int malformed(const char *fmt, ...) {
    char facts[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(facts, sizeof(facts), fmt, ap);
    va_end(ap);
    return set_error(NDL_ERR_MALFORMED_MODEL, "%s. %s", facts, kGuidance);
}
int unsupported(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
int unsupported(const char *fmt, ...) {
    char facts[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(facts, sizeof(facts), fmt, ap);
    va_end(ap);
    return set_error(NDL_ERR_UNSUPPORTED, "%s. %s", facts, kGuidance);
}

// RequireWellFormed (src/Needle/Model.cs:365-384).
int require_well_formed(const uint8_t *map, uint64_t length, uint32_t *h) {
    if (length < kCactHeaderBytes)
        return malformed("not a Needle 3 .cact archive: the file has %llu bytes, shorter than the %llu-byte header",
                         (unsigned long long)length, (unsigned long long)kCactHeaderBytes);
    memcpy(h, map, kCactHeaderBytes);
    if (h[0] != kCactMagic)
        return malformed("not a supported Needle 3 .cact archive: found magic 0x%08X, supported magic is 0x%08X", h[0],
                         kCactMagic);
    const uint64_t count = h[1];
    const uint64_t table_end = kCactHeaderBytes + (uint64_t)h[2] * 4 + count * sizeof(CactRecord);
    if (count == 0 || table_end > length)
        return malformed("truncated or corrupt .cact archive: the header declares %llu tensors and %u codebook entries, "
                         "needing %llu bytes of tables, but the file has %llu bytes",
                         (unsigned long long)count, h[2], (unsigned long long)table_end, (unsigned long long)length);
    const uint8_t *table = map + kCactHeaderBytes + (size_t)h[2] * 4;
    for (uint64_t i = 0; i < count; i++) {
        CactRecord r;
        memcpy(&r, table + i * sizeof(CactRecord), sizeof(r));
        if (r.offset > length || r.bytes > length - r.offset)
            return malformed("truncated .cact archive: tensor %llu ends at byte %llu, but the file has %llu bytes",
                             (unsigned long long)i, (unsigned long long)(r.offset + r.bytes),
                             (unsigned long long)length);
    }
    if (h[26] > 4 || h[31] > 16)
        return unsupported("unsupported engram layout: found %u orders and %u sites; this build supports at most 4 "
                           "orders and 16 sites",
                           h[26], h[31]);
    return NDL_OK;
}

// The Geometry words (src/Needle/Model.cs:78-104) and the constructor's
// three geometry checks (:319-324).
int read_geometry(const uint32_t *h, ndl_model_info *g) {
    g->kv_window = (int)h[3];
    g->vocab = (int)h[5];
    g->dim = (int)h[7];
    g->heads = (int)h[8];
    g->kv_heads = (int)h[9];
    g->layers = (int)h[10];
    g->qk_dim = (int)h[11];
    g->v_dim = (int)h[12];
    g->max_seq = (int)h[13];
    g->hada_n = (int)h[14];
    g->lanes = (int)h[15];
    g->sliding_window = (int)h[16];
    g->global_mask = (uint64_t)h[17] | ((uint64_t)h[18] << 32);
    g->conv_taps = (int)h[19];
    g->engram_slots = (int)h[20];
    g->engram_sub = (int)h[21];
    g->engram_tables = (int)h[22];
    g->engram_conv_taps = (int)h[23];
    g->engram_dilation = (int)h[24];
    g->engram_seed_heads = (int)h[25];
    g->order_count = (int)h[26];
    g->site_count = (int)h[31];
    memcpy(&g->rope_theta, h + 48, 4);
    for (int i = 0; i < g->order_count; i++) g->orders[i] = (int)h[27 + i];
    for (int i = 0; i < g->site_count; i++) g->sites[i] = (int)h[32 + i];
    g->hada_rows = 1 << (bit_length((uint32_t)(g->hada_n - 1)) / 2);
    g->hada_cols = g->hada_n / g->hada_rows;
    if (!(g->qk_dim == 48 && g->v_dim == 64 && g->lanes == 4))
        return unsupported("unsupported head geometry: found QkDim=%d, VDim=%d, Lanes=%d; this build supports "
                           "QkDim=48, VDim=64, Lanes=4",
                           g->qk_dim, g->v_dim, g->lanes);
    if (!(g->hada_cols % 8 == 0 && g->hada_rows * g->hada_cols == g->hada_n))
        return unsupported("unsupported MLP geometry: found HadaN=%d; this build supports sizes that split into rows "
                           "by columns with columns divisible by 8",
                           g->hada_n);
    if (!(g->conv_taps == 3 && g->engram_conv_taps == 4 && g->dim % kCqGroupCols == 0))
        return unsupported("unsupported convolution geometry: found ConvTaps=%d, EngramConvTaps=%d, Dim=%d; this build "
                           "supports ConvTaps=3, EngramConvTaps=4 and Dim divisible by %d",
                           g->conv_taps, g->engram_conv_taps, g->dim, kCqGroupCols);
    return NDL_OK;
}

// Reader (src/Needle/Model.cs:200-283): takes records in order, each under a role.
struct Walker {
    const uint8_t *map;
    ndl_model *m;
    int next = 0;
    bool exact_halves = true;

    int count() const { return (int)m->records.size(); }

    int take(const char *role, int index, const CactRecord **r) {
        if (next >= count())
            return malformed("the tensor table ends after %d records, before %s %d", count(), role, index);
        *r = &m->records[next];
        Entry e;
        e.role = role;
        e.index = index;
        e.record = next++;
        m->entries.push_back(std::move(e));
        return NDL_OK;
    }

    static uint64_t elements(const CactRecord &r) {
        uint64_t n = 1;
        for (int i = 0; i < r.ndim; i++) n *= r.shape[i];
        return n;
    }

    int check_shape(const CactRecord &r, uint64_t element_bytes) {
        const Entry &e = m->entries.back();
        if (r.ndim > 4) return malformed("tensor %d (%s %d) has %d dimensions (at most 4)", e.record, e.role.c_str(), e.index, r.ndim);
        for (int i = 0; i < r.ndim; i++)
            if (r.shape[i] > 0x7FFFFFFFu)
                return malformed("tensor %d (%s %d) has a dimension of %u", e.record, e.role.c_str(), e.index, r.shape[i]);
        const uint64_t n = elements(r);
        if (n > (1ull << 40) || n * element_bytes > r.bytes)
            return malformed("tensor %d (%s %d) holds %llu bytes, %llu elements of %llu bytes need more", e.record,
                             e.role.c_str(), e.index, (unsigned long long)r.bytes, (unsigned long long)n,
                             (unsigned long long)element_bytes);
        return NDL_OK;
    }

    // Reader.Dense
    int dense(const char *role, int index, bool exact) {
        const CactRecord *r;
        TRY(take(role, index, &r));
        Entry &e = m->entries.back();
        if (r->dtype != kTypeFp16 && r->dtype != kTypeFp32)
            return malformed("dense tensor expected: tensor %d (%s %d) has dtype %d", e.record, role, index, r->dtype);
        TRY(check_shape(*r, r->dtype == kTypeFp16 ? 2 : 4));
        e.kind = NDL_TENSOR_DENSE;
        e.count = (int64_t)elements(*r);
        e.dense.resize((size_t)e.count);
        const uint8_t *src = map + r->offset;
        if (r->dtype == kTypeFp16) {
            for (int64_t i = 0; i < e.count; i++) {
                uint16_t hv;
                memcpy(&hv, src + 2 * i, 2);
                e.dense[(size_t)i] = half_to_single(hv, exact);
            }
        } else {
            memcpy(e.dense.data(), src, (size_t)e.count * 4);
        }
        return NDL_OK;
    }
    int dense(const char *role, int index) { return dense(role, index, exact_halves); }

    // Reader.Indices: an fp32 vector of `expected` entries, truncated to int.
    int indices(const char *role, int index, int expected) {
        const CactRecord *r;
        TRY(take(role, index, &r));
        Entry &e = m->entries.back();
        if (r->dtype != kTypeFp32 || r->ndim > 4 || elements(*r) != (uint64_t)expected)
            return malformed("permutation expected: tensor %d (%s %d) is not an fp32 vector of %d entries", e.record,
                             role, index, expected);
        TRY(check_shape(*r, 4));
        e.kind = NDL_TENSOR_PERMUTATION;
        e.count = expected;
        e.perm.resize((size_t)expected);
        for (int i = 0; i < expected; i++) {
            float f;
            memcpy(&f, map + r->offset + 4 * (size_t)i, 4);
            const int v = (f > -2147483648.0f && f < 2147483648.0f) ? (int)f : INT32_MIN;
            if (v < 0 || v >= expected)
                return malformed("permutation entry %d of tensor %d (%s %d) is %d, outside [0, %d)", i, e.record, role,
                                 index, v, expected);
            e.perm[(size_t)i] = v;
        }
        return NDL_OK;
    }

    // Reader.Quantized; `decode` also asks for the rows decoded (Reader.Rows).
    int quantized(const char *role, int index, bool decode = false) {
        const CactRecord *r;
        TRY(take(role, index, &r));
        Entry &e = m->entries.back();
        if (r->dtype != kTypeCq || (r->bits != 2 && r->bits != 4))
            return malformed("2- or 4-bit CQ tensor expected: tensor %d (%s %d) has dtype %d, %u bits", e.record, role,
                             index, r->dtype, r->bits);
        const uint64_t rows = r->shape[0], cols = r->shape[1];
        if (cols % kCqGroupCols != 0 || r->group != (uint32_t)kCqGroupCols)
            return malformed("CQ group of 128 expected: tensor %d (%s %d) has %llu columns, group %u", e.record, role,
                             index, (unsigned long long)cols, r->group);
        if (rows == 0 || cols == 0 || rows > 0x7FFFFFFFu || cols > 0x7FFFFFFFu)
            return malformed("tensor %d (%s %d) is a %llu x %llu CQ matrix", e.record, role, index,
                             (unsigned long long)rows, (unsigned long long)cols);
        e.index_bytes = (size_t)(rows * cols * r->bits / 8);
        e.norm_bytes = (size_t)(rows * (cols / kCqGroupCols) * 2);
        if ((uint64_t)e.index_bytes + e.norm_bytes > r->bytes)
            return malformed("tensor %d (%s %d) holds %llu bytes, its %llu x %llu %u-bit codes and norms need %llu",
                             e.record, role, index, (unsigned long long)r->bytes, (unsigned long long)rows,
                             (unsigned long long)cols, r->bits, (unsigned long long)(e.index_bytes + e.norm_bytes));
        e.kind = decode ? NDL_TENSOR_CQ_ROWS : NDL_TENSOR_CQ;
        e.rows = (int)rows;
        e.cols = (int)cols;
        e.bits = (int)r->bits;
        if (decode) e.count = (int64_t)rows * (int64_t)cols;
        return NDL_OK;
    }

    // MlpWeights (src/Needle/Audio.cs:5-27)
    int mlp(int layer) {
        static const char *names[13] = {"layer.mlp.d1",  "layer.mlp.d2",  "layer.mlp.b2",    "layer.mlp.d3",
                                        "layer.mlp.d4",  "layer.mlp.w1a", "layer.mlp.w1b",   "layer.mlp.w2a",
                                        "layer.mlp.w2b", "layer.mlp.w3a", "layer.mlp.w3b",   "layer.mlp.cond_v",
                                        "layer.mlp.cond_u"};
        for (const char *n : names) TRY(dense(n, layer));
        return NDL_OK;
    }

    // LayerWeights (src/Needle/Model.cs:122-150)
    int layer(int l) {
        TRY(dense("layer.norm_in", l));
        TRY(quantized("layer.q", l));
        TRY(quantized("layer.k", l));
        TRY(quantized("layer.v", l));
        TRY(dense("layer.q_taps", l));
        TRY(dense("layer.k_taps", l));
        TRY(dense("layer.v_taps", l));
        TRY(dense("layer.q_norm", l));
        TRY(dense("layer.k_norm", l));
        TRY(quantized("layer.gate", l));
        TRY(quantized("layer.out", l));
        TRY(dense("layer.post_norm", l));
        TRY(dense("layer.attn_gate", l));  // the logit; the reference keeps its sigmoid
        TRY(dense("layer.pre_hada", l));
        return mlp(l);
    }

    // HyperConnections (src/Needle/Model.cs:152-173)
    int hyper(int perm_length) {
        for (const char *n : {"hyper.a_pre", "hyper.a_post", "hyper.a_res", "hyper.b_pre", "hyper.b_post", "hyper.b_res"})
            TRY(dense(n, 0));
        TRY(quantized("hyper.phi_pre", 0));
        TRY(quantized("hyper.phi_post", 0));
        TRY(quantized("hyper.phi_res", 0));
        if (perm_length > 0) {
            TRY(indices("hyper.perm_a", 0, perm_length));
            TRY(indices("hyper.perm_b", 0, perm_length));
        }
        return NDL_OK;
    }

    // EngramSite (src/Needle/Model.cs:175-189)
    int site(int s) {
        TRY(quantized("site.tables", s));
        TRY(quantized("site.key", s));
        TRY(quantized("site.value", s));
        return dense("site.taps", s);
    }

    // ProbeHead (src/Needle/Audio.cs:29-56)
    int probe_head(int h, int code) {
        TRY(quantized("probe.probe_vectors", h, true));
        TRY(dense("probe.gain", h));
        TRY(quantized("probe.query_vectors", h, true));
        TRY(dense("probe.row_bias", h));
        TRY(quantized("probe.projection", h, true));
        TRY(dense("probe.bias", h));
        if (code == 3) TRY(dense("probe.router", h));  // ProbeHead.Router reads one more dense tensor
        return NDL_OK;
    }
};

// HasAudioWeights (src/Needle/Model.cs:386-391)
bool has_audio_weights(const std::vector<CactRecord> &records) {
    for (const CactRecord &r : records)
        if (r.dtype == kTypeFp32 && r.ndim == 1 && r.shape[0] == 13) return true;
    return false;
}

// MathF.Round: half to even.
int round_half_even(float v) { return (int)rintf(v); }

// The constructor's walk (src/Needle/Model.cs:307-361).
int parse(ndl_model *m, const uint8_t *map, uint64_t length) {
    uint32_t h[kCactHeaderBytes / 4];
    TRY(require_well_formed(map, length, h));
    ndl_model_info &g = m->info;
    g.magic = h[0];
    g.length = (int64_t)length;
    g.tensors = (int)h[1];
    g.codebook_entries = (int)h[2];
    g.device = -1;
    g.confidence_head = g.embedding_head = -1;
    TRY(read_geometry(h, &g));
    if (h[2] < (uint32_t)kCodebookLevels)
        return malformed("the codebook holds %u levels, the 2- and 4-bit books read %d", h[2], kCodebookLevels);
    float levels[kCodebookLevels];
    memcpy(levels, map + kCactHeaderBytes, sizeof(levels));
    fill_codebook(&m->book2, levels, 4);
    fill_codebook(&m->book4, levels + 12, 16);
    m->records.resize(h[1]);
    memcpy(m->records.data(), map + kCactHeaderBytes + (size_t)h[2] * 4, (size_t)h[1] * sizeof(CactRecord));

    Walker w{map, m};
    w.exact_halves = !has_audio_weights(m->records);
    TRY(w.quantized("embedding", 0));
    for (int l = 0; l < g.layers; l++) TRY(w.layer(l));
    TRY(w.hyper(g.hada_n));
    for (int s = 0; s < g.site_count; s++) TRY(w.site(s));
    TRY(w.dense("final_norm", 0));
    const int tail = w.count() - 1;
    if (w.next < w.count()) {
        const CactRecord &n = m->records[w.next];
        if (n.dtype == kTypeFp32 && n.ndim == 1 && n.shape[0] == 13) {
            g.has_audio = 1;  // AudioWeights: kept as records, exact halves from here on
            for (int k = 0; w.next < tail; k++) {
                const CactRecord &r = m->records[w.next];
                if (r.dtype == kTypeCq) TRY(w.quantized("audio", k));
                else if (r.dtype == kTypeFp16 || r.dtype == kTypeFp32) TRY(w.dense("audio", k, true));
                else return malformed("audio tensor %d has dtype %d", w.next, r.dtype);
            }
        } else if (w.next != tail) {
            TRY(w.dense("manifest", 0));
            const std::vector<float> manifest = m->entries.back().dense;
            for (int hd = 0; w.next < tail; hd++) {
                if (hd >= (int)manifest.size() || hd >= kMaxProbeHeads)
                    return malformed("probe head %d has no manifest entry (%zu entries, at most %d heads)", hd,
                                     manifest.size(), kMaxProbeHeads);
                const int code = round_half_even(manifest[(size_t)hd]);
                TRY(w.probe_head(hd, code));
                g.probe_codes[hd] = code;
                g.probe_heads = hd + 1;
                if (code == 2) {
                    g.confidence_head = hd;
                    g.has_confidence = 1;
                } else if (code == 1) {
                    g.embedding_head = hd;
                    g.has_embedding_head = 1;
                }
            }
        }
    }
    const CactRecord &tok = m->records[(size_t)tail];
    if (tok.dtype != kTypeRaw)
        return malformed("tokenizer blob missing: the last tensor has dtype %d, expected %d", tok.dtype, kTypeRaw);
    if (w.next > tail) return malformed("the weights run into the tokenizer record (tensor %d)", tail);
    m->tokenizer.assign(map + tok.offset, map + tok.offset + tok.bytes);
    g.tokenizer_bytes = (int64_t)tok.bytes;
    return NDL_OK;
}

// One device allocation for everything; the decoded probe rows come from the
// GatherRow kernel over the uploaded codes.
int upload(ndl_model *m, const uint8_t *map, int device) {
    size_t end = 0;
    auto place = [&](size_t bytes) {
        end = (end + 255) & ~(size_t)255;
        const size_t at = end;
        end += bytes;
        return at;
    };
    int max_rows = 0;
    for (Entry &e : m->entries) {
        if (e.kind == NDL_TENSOR_DENSE) e.at_values = place((size_t)e.count * 4);
        if (e.kind == NDL_TENSOR_PERMUTATION) e.at_perm = place((size_t)e.count * 4);
        if (e.kind == NDL_TENSOR_CQ || e.kind == NDL_TENSOR_CQ_ROWS) {
            e.at_indices = place(e.index_bytes);
            e.at_norms = place(e.norm_bytes);
        }
        if (e.kind == NDL_TENSOR_CQ_ROWS) {
            e.at_values = place((size_t)e.count * 4);
            max_rows = std::max(max_rows, e.rows);
        }
    }
    const size_t at_ids = place((size_t)max_rows * 4);
    const size_t total = end;
    std::vector<uint8_t> stage(total);
    for (const Entry &e : m->entries) {
        const CactRecord &r = m->records[(size_t)e.record];
        if (e.kind == NDL_TENSOR_DENSE) memcpy(stage.data() + e.at_values, e.dense.data(), (size_t)e.count * 4);
        if (e.kind == NDL_TENSOR_PERMUTATION) memcpy(stage.data() + e.at_perm, e.perm.data(), (size_t)e.count * 4);
        if (e.kind == NDL_TENSOR_CQ || e.kind == NDL_TENSOR_CQ_ROWS) {
            memcpy(stage.data() + e.at_indices, map + r.offset, e.index_bytes);
            memcpy(stage.data() + e.at_norms, map + r.offset + e.index_bytes, e.norm_bytes);
        }
    }
    for (int i = 0; i < max_rows; i++) {
        const int32_t v = i;
        memcpy(stage.data() + at_ids + 4 * (size_t)i, &v, 4);
    }
    int previous = 0;
    NDL_CUDA(cudaGetDevice(&previous));
    NDL_CUDA(cudaSetDevice(device));
    int st = NDL_OK;
    if (cudaMalloc(reinterpret_cast<void **>(&m->block), total) != cudaSuccess) {
        cudaGetLastError();
        m->block = nullptr;
        st = set_error(NDL_ERR_OUT_OF_MEMORY, "model weights (%zu bytes) on device %d", total, device);
    }
    if (st == NDL_OK && cudaMemcpy(m->block, stage.data(), total, cudaMemcpyHostToDevice) != cudaSuccess)
        st = set_error(NDL_ERR_CUDA, "model upload: %s", cudaGetErrorString(cudaGetLastError()));
    for (const Entry &e : m->entries) {
        if (st != NDL_OK || e.kind != NDL_TENSOR_CQ_ROWS) continue;
        const ndl_kt_codebook &book = e.bits == 2 ? m->book2 : m->book4;
        st = ndl_cq_gather_rows(m->block + e.at_indices, reinterpret_cast<const uint16_t *>(m->block + e.at_norms),
                                book.levels, e.rows, e.cols, e.bits,
                                reinterpret_cast<const int32_t *>(m->block + at_ids), e.rows,
                                reinterpret_cast<float *>(m->block + e.at_values), nullptr);
    }
    if (st == NDL_OK && cudaStreamSynchronize(nullptr) != cudaSuccess)
        st = set_error(NDL_ERR_CUDA, "model upload: %s", cudaGetErrorString(cudaGetLastError()));
    cudaSetDevice(previous);
    if (st != NDL_OK) return st;
    m->info.device = device;
    m->info.device_bytes = total;
    return NDL_OK;
}

const Entry *find(const ndl_model *m, const char *role, int index) {
    for (const Entry &e : m->entries)
        if (e.index == index && e.role == role) return &e;
    return nullptr;
}

}  // namespace
}  // namespace ndl

NDL_API int ndl_model_load(const void *archive, size_t bytes, int device, ndl_model **out) {
    NDL_REQUIRE(out, "null model handle");
    *out = nullptr;
    NDL_REQUIRE(archive || bytes == 0, "null archive of %zu bytes", bytes);
    static const uint8_t empty[1] = {0};
    const uint8_t *map = archive ? static_cast<const uint8_t *>(archive) : empty;
    ndl_model *m = new ndl_model();
    int st = parse(m, map, bytes);
    if (st == NDL_OK && device >= 0) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n) {
            cudaGetLastError();
            st = set_error(NDL_ERR_NO_DEVICE, "no CUDA device %d (%d present)", device, n);
        } else {
            st = upload(m, map, device);
        }
    }
    if (st != NDL_OK) {
        ndl_model_destroy(m);
        return st;
    }
    *out = m;
    return NDL_OK;
}

NDL_API int ndl_model_destroy(ndl_model *m) {
    if (!m) return NDL_OK;
    if (m->block) {
        int previous = 0;
        cudaGetDevice(&previous);
        cudaSetDevice(m->info.device);
        cudaFree(m->block);
        cudaSetDevice(previous);
    }
    delete m;
    return NDL_OK;
}

NDL_API int ndl_model_get_info(const ndl_model *m, ndl_model_info *info) {
    NDL_REQUIRE(m && info, "null argument");
    *info = m->info;
    return NDL_OK;
}

NDL_API int ndl_model_tensor_count(const ndl_model *m, int *count) {
    NDL_REQUIRE(m && count, "null argument");
    *count = (int)m->entries.size();
    return NDL_OK;
}

NDL_API int ndl_model_tensor_name(const ndl_model *m, int i, const char **role, int *index) {
    NDL_REQUIRE(m && role && index, "null argument");
    NDL_REQUIRE(i >= 0 && i < (int)m->entries.size(), "tensor %d of %zu", i, m->entries.size());
    *role = m->entries[(size_t)i].role.c_str();
    *index = m->entries[(size_t)i].index;
    return NDL_OK;
}

NDL_API int ndl_model_get_tensor(const ndl_model *m, const char *role, int index, ndl_model_tensor *t) {
    NDL_REQUIRE(m && role && t, "null argument");
    const Entry *e = find(m, role, index);
    NDL_REQUIRE(e, "the model has no tensor %s %d", role, index);
    const CactRecord &r = m->records[(size_t)e->record];
    memset(t, 0, sizeof(*t));
    t->kind = e->kind;
    t->record = e->record;
    t->dtype = r.dtype;
    t->ndim = r.ndim;
    for (int i = 0; i < 4; i++) t->shape[i] = r.shape[i];
    t->offset = r.offset;
    t->bytes = r.bytes;
    t->count = e->count;
    t->rows = e->rows;
    t->cols = e->cols;
    t->bits = e->bits;
    if (e->kind == NDL_TENSOR_CQ || e->kind == NDL_TENSOR_CQ_ROWS) t->book = e->bits == 2 ? &m->book2 : &m->book4;
    if (m->block) {
        if (e->kind == NDL_TENSOR_DENSE || e->kind == NDL_TENSOR_CQ_ROWS)
            t->values = reinterpret_cast<const float *>(m->block + e->at_values);
        if (e->kind == NDL_TENSOR_PERMUTATION) t->permutation = reinterpret_cast<const int32_t *>(m->block + e->at_perm);
        if (e->kind == NDL_TENSOR_CQ || e->kind == NDL_TENSOR_CQ_ROWS) {
            t->indices = m->block + e->at_indices;
            t->norms = reinterpret_cast<const uint16_t *>(m->block + e->at_norms);
        }
    }
    return NDL_OK;
}

NDL_API int ndl_model_read_host(const ndl_model *m, const char *role, int index, void *destination, size_t bytes) {
    NDL_REQUIRE(m && role && destination, "null argument");
    const Entry *e = find(m, role, index);
    NDL_REQUIRE(e, "the model has no tensor %s %d", role, index);
    NDL_REQUIRE(e->kind == NDL_TENSOR_DENSE || e->kind == NDL_TENSOR_PERMUTATION,
                "%s %d is a CQ matrix: its host form is the archive's own bytes", role, index);
    const size_t need = (size_t)e->count * 4;
    NDL_REQUIRE(bytes >= need, "%s %d needs %zu bytes, %zu given", role, index, need, bytes);
    memcpy(destination, e->kind == NDL_TENSOR_DENSE ? (const void *)e->dense.data() : (const void *)e->perm.data(), need);
    return NDL_OK;
}

NDL_API int ndl_model_tokenizer(const ndl_model *m, const void **blob, size_t *bytes) {
    NDL_REQUIRE(m && blob && bytes, "null argument");
    *blob = m->tokenizer.data();
    *bytes = m->tokenizer.size();
    return NDL_OK;
}
