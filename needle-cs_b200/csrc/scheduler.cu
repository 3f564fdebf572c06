// Continuous batching over one engine: requests arrive at any time, each
// step packs every running request's next decode row plus prompt chunks of
// waiting requests (at most `prefill_chunk` positions of one request per
// step) into one ndl_forward_batch, then samples every head row with the
// request's stored vocabulary mask (ArgMaxMasked).
//
// The reference's BatchedSession.RunBatch (src/Needle/BatchedSession.cs:
// 218-268) packs each lane's pending tokens (at most 4) into one
// ForwardBatch per step after prefilling every lane on its own
// (PrefillLane, :270-304); this scheduler keeps its step structure (collect
// pending rows, one forward, advance lanes, ContextExhausted check against
// the capacity, :242-246) and additionally mixes prompt chunks with decode
// rows.  Because a row's logits do not depend on the rest of the batch, a
// request's token stream is the one it would get alone.
//
// Jump-forward (NeedleSession.GenerateCalls, src/Needle/NeedleSession.cs:
// 538-662): tokens the caller's grammar forces (the mask allows one id) are
// appended to a decoding request's output without logits; the next step feeds
// the request's unfed tokens (its last pick and the forced ones) as one run
// and samples only at the run's last row, as the reference feeds its call
// chunk.  A run equals feeding the tokens one per step, so the stream does
// not change, only the number of forwards.
//
// Host code only; single-threaded like the engine (one host thread per
// engine).  A scheduler made by ndl_sched_create_dry has no engine: it plans
// steps and "samples" token (request * 7919 + produced) % vocab, which lets
// the packing be tested without a GPU.
#include <algorithm>
#include <deque>
#include <unordered_map>
#include <vector>

#include "common.cuh"

using namespace ndl;

namespace {

enum class State { Waiting, Prefill, Decode, Done };

struct Request {
    int id = 0;
    std::vector<int32_t> prompt;
    std::vector<uint32_t> mask;  // empty: unmasked
    int max_new = 0, stop = -1;
    int slot = -1, fed = 0;
    int unfed = 0;          // tokens at the end of `out` not yet fed (the last pick and forced tokens)
    bool finished = false;  // forced tokens reached max_new or the stop token: ends at the next step
    State state = State::Waiting;
    int status = NDL_OK;
    std::vector<int32_t> out;
};

}  // namespace

struct ndl_sched {
    ndl_engine *e = nullptr;
    ndl_sched_config cfg{};
    int slots = 0, capacity = 0, vocab = 0;
    std::unordered_map<int, Request> requests;
    std::deque<int> waiting;     // request ids, arrival order
    std::vector<int> admitted;   // running request ids, admission order
    std::vector<int> free_slots;
    std::vector<int> dry_len;    // dry mode: positions held per slot
    // last step's plan
    std::vector<int> tokens, row_slots, head_rows, head_request;
};

namespace {

int slot_length(ndl_sched *s, int slot, int *len) {
    if (!s->e) {
        *len = s->dry_len[slot];
        return NDL_OK;
    }
    return ndl_slot_length(s->e, slot, len);
}

int release(ndl_sched *s, Request &r) {
    if (r.slot >= 0) {
        if (s->e) {
            int st = ndl_slot_reset(s->e, r.slot);
            if (st != NDL_OK) return st;
            st = ndl_engine_set_mask(s->e, r.slot, nullptr, 0);
            if (st != NDL_OK) return st;
        } else {
            s->dry_len[r.slot] = 0;
        }
        s->free_slots.push_back(r.slot);
        r.slot = -1;
    }
    r.state = State::Done;
    return NDL_OK;
}

int admit(ndl_sched *s) {
    while (!s->waiting.empty() && !s->free_slots.empty()) {
        Request &r = s->requests[s->waiting.front()];
        s->waiting.pop_front();
        r.slot = s->free_slots.back();
        s->free_slots.pop_back();
        if (s->e) {
            int st = ndl_slot_reset(s->e, r.slot);
            if (st != NDL_OK) return st;
            st = r.mask.empty() ? ndl_engine_set_mask(s->e, r.slot, nullptr, 0)
                                : ndl_engine_set_mask(s->e, r.slot, r.mask.data(), (int)r.mask.size());
            if (st != NDL_OK) return st;
        } else {
            s->dry_len[r.slot] = 0;
        }
        r.state = State::Prefill;
        r.fed = 0;
        s->admitted.push_back(r.id);
    }
    return NDL_OK;
}

void push_event(ndl_sched_event *events, int capacity, int *count, int request, int kind, int token, int status) {
    if (events && *count < capacity) events[*count] = ndl_sched_event{request, kind, token, status};
    (*count)++;
}

}  // namespace

extern "C" {

NDL_API int ndl_sched_create(ndl_engine *e, const ndl_sched_config *cfg, ndl_sched **out) {
    NDL_REQUIRE(e && cfg && out, "null argument");
    NDL_REQUIRE(cfg->max_rows >= 1 && cfg->prefill_chunk >= 1, "max_rows=%d prefill_chunk=%d", cfg->max_rows,
                cfg->prefill_chunk);
    ndl_engine_info info{};
    int st = ndl_engine_get_info(e, &info);
    if (st != NDL_OK) return st;
    NDL_REQUIRE(cfg->max_rows <= info.max_rows && cfg->max_rows <= info.max_heads,
                "max_rows %d above the engine's rows (%d) or heads (%d)", cfg->max_rows, info.max_rows,
                info.max_heads);
    auto *s = new ndl_sched();
    s->e = e;
    s->cfg = *cfg;
    s->slots = info.slots;
    s->capacity = info.capacity;
    s->vocab = info.vocab;
    for (int i = s->slots - 1; i >= 0; i--) s->free_slots.push_back(i);
    *out = s;
    return NDL_OK;
}

NDL_API int ndl_sched_create_dry(const ndl_sched_config *cfg, int slots, int capacity, int vocab, ndl_sched **out) {
    NDL_REQUIRE(cfg && out, "null argument");
    NDL_REQUIRE(cfg->max_rows >= 1 && cfg->prefill_chunk >= 1 && slots >= 1 && capacity >= 1 && vocab >= 1,
                "bad dry scheduler configuration");
    auto *s = new ndl_sched();
    s->cfg = *cfg;
    s->slots = slots;
    s->capacity = capacity;
    s->vocab = vocab;
    s->dry_len.assign(slots, 0);
    for (int i = slots - 1; i >= 0; i--) s->free_slots.push_back(i);
    *out = s;
    return NDL_OK;
}

NDL_API int ndl_sched_destroy(ndl_sched *s) {
    delete s;
    return NDL_OK;
}

NDL_API int ndl_sched_submit(ndl_sched *s, int request, const int32_t *prompt, int prompt_len, int max_new_tokens,
                             int stop_token, const uint32_t *mask, int mask_words) {
    NDL_REQUIRE(s && prompt, "null argument");
    NDL_REQUIRE(prompt_len >= 1 && max_new_tokens >= 1, "prompt_len=%d max_new_tokens=%d", prompt_len,
                max_new_tokens);
    NDL_REQUIRE(!s->requests.count(request), "request %d already submitted", request);
    const int max_words = (s->vocab + 31) / 32;
    NDL_REQUIRE(!mask || (mask_words >= 1 && mask_words <= max_words), "mask_words %d outside 1..%d", mask_words,
                max_words);
    for (int i = 0; i < prompt_len; i++)
        NDL_REQUIRE(prompt[i] >= 0 && prompt[i] < s->vocab, "prompt token %d = %d outside the vocabulary", i,
                    prompt[i]);
    Request r;
    r.id = request;
    r.prompt.assign(prompt, prompt + prompt_len);
    if (mask) r.mask.assign(mask, mask + mask_words);
    r.max_new = max_new_tokens;
    r.stop = stop_token;
    s->requests.emplace(request, std::move(r));
    s->waiting.push_back(request);
    return NDL_OK;
}

// Jump-forward: `count` tokens the caller's grammar forces after the
// request's last pick, appended to its output without sampling; the next
// step feeds them with that pick as one run (see the file comment).  The
// request must be decoding; reaching max_new_tokens or the stop token among
// them ends it at the next step.
NDL_API int ndl_sched_force(ndl_sched *s, int request, const int32_t *tokens, int count) {
    NDL_REQUIRE(s && tokens, "null argument");
    NDL_REQUIRE(count >= 1, "count %d", count);
    auto it = s->requests.find(request);
    NDL_REQUIRE(it != s->requests.end(), "request %d was not submitted", request);
    Request &r = it->second;
    NDL_REQUIRE(r.state == State::Decode && !r.finished, "request %d is not decoding", request);
    for (int i = 0; i < count; i++)
        NDL_REQUIRE(tokens[i] >= 0 && tokens[i] < s->vocab, "forced token %d = %d outside the vocabulary", i,
                    tokens[i]);
    for (int i = 0; i < count && !r.finished; i++) {
        r.out.push_back(tokens[i]);
        r.unfed++;
        if ((int)r.out.size() >= r.max_new || tokens[i] == r.stop) r.finished = true;
    }
    return NDL_OK;
}

// One step.  Events: kind 1 = first token (token = its id), kind 2 = the
// request finished (status 0, or a FailureReason such as 3 ContextExhausted;
// token = the last id or -1).  *count is the number of events (those beyond
// `capacity` are dropped); rows / decode_rows report the step's size.
NDL_API int ndl_sched_step(ndl_sched *s, ndl_sched_event *events, int capacity, int *count, int *rows,
                           int *decode_rows) {
    NDL_REQUIRE(s && count, "null argument");
    *count = 0;
    int st = admit(s);
    if (st != NDL_OK) return st;
    s->tokens.clear();
    s->row_slots.clear();
    s->head_rows.clear();
    s->head_request.clear();
    const int budget = s->cfg.max_rows;
    int n_decode = 0;
    // decode rows first, in admission order: each request's unfed tokens (one,
    // or a jump-forward run), the logits at the last
    for (int id : s->admitted) {
        Request &r = s->requests[id];
        if (r.state != State::Decode) continue;
        if (r.finished) {
            push_event(events, capacity, count, id, 2, r.out.back(), r.status);
            if ((st = release(s, r)) != NDL_OK) return st;
            continue;
        }
        const int n = std::min(r.unfed, budget - (int)s->tokens.size());
        if (n <= 0) continue;
        int len = 0;
        if ((st = slot_length(s, r.slot, &len)) != NDL_OK) return st;
        if (len + n > s->capacity) {
            r.status = NDL_FAIL_CONTEXT_EXHAUSTED;
            push_event(events, capacity, count, id, 2, r.out.empty() ? -1 : r.out.back(), r.status);
            if ((st = release(s, r)) != NDL_OK) return st;
            continue;
        }
        const int first = (int)r.out.size() - r.unfed;
        for (int i = 0; i < n; i++) {
            s->tokens.push_back(r.out[first + i]);
            s->row_slots.push_back(r.slot);
        }
        r.unfed -= n;
        if (r.unfed == 0) {  // the run is complete: its last row samples the next token
            s->head_rows.push_back((int)s->tokens.size() - 1);
            s->head_request.push_back(id);
        }
        n_decode += n;
    }
    // then prompt chunks
    for (int id : s->admitted) {
        Request &r = s->requests[id];
        const int left = budget - (int)s->tokens.size();
        if (r.state != State::Prefill || left <= 0) continue;
        const int c = std::min({(int)r.prompt.size() - r.fed, s->cfg.prefill_chunk, left});
        int len = 0;
        if ((st = slot_length(s, r.slot, &len)) != NDL_OK) return st;
        if (len + c > s->capacity) {
            r.status = NDL_FAIL_CONTEXT_EXHAUSTED;
            push_event(events, capacity, count, id, 2, -1, r.status);
            if ((st = release(s, r)) != NDL_OK) return st;
            continue;
        }
        for (int i = 0; i < c; i++) {
            s->tokens.push_back(r.prompt[r.fed + i]);
            s->row_slots.push_back(r.slot);
        }
        r.fed += c;
        if (r.fed == (int)r.prompt.size()) {  // the prompt's last position samples the first token
            s->head_rows.push_back((int)s->tokens.size() - 1);
            s->head_request.push_back(id);
        }
    }
    const int R = (int)s->tokens.size(), H = (int)s->head_rows.size();
    if (rows) *rows = R;
    if (decode_rows) *decode_rows = n_decode;
    std::vector<int> ids(H);
    if (R > 0) {
        if (s->e) {
            st = ndl_forward_batch(s->e, s->tokens.data(), s->row_slots.data(), R, s->head_rows.data(), H);
            if (st != NDL_OK) return st;
            if (H > 0) {
                std::vector<int> head_slots(H);
                for (int h = 0; h < H; h++) head_slots[h] = s->row_slots[s->head_rows[h]];
                st = ndl_sample_argmax_slots(s->e, head_slots.data(), ids.data(), nullptr);
                if (st != NDL_OK) return st;
            }
        } else {
            for (int i = 0; i < R; i++) s->dry_len[s->row_slots[i]]++;
            for (int h = 0; h < H; h++) {
                const Request &r = s->requests[s->head_request[h]];
                ids[h] = (int)(((long long)r.id * 7919 + (long long)r.out.size()) % s->vocab);
            }
        }
    }
    for (int h = 0; h < H; h++) {
        Request &r = s->requests[s->head_request[h]];
        const int tok = ids[h];
        if (tok < 0) {  // the mask allowed nothing: the request ends (ArgMaxMasked returns -1)
            push_event(events, capacity, count, r.id, 2, -1, r.status);
            if ((st = release(s, r)) != NDL_OK) return st;
            continue;
        }
        r.out.push_back(tok);
        r.unfed = 1;
        if (r.state == State::Prefill) {
            r.state = State::Decode;
            push_event(events, capacity, count, r.id, 1, tok, NDL_OK);
        }
        if ((int)r.out.size() >= r.max_new || tok == r.stop) {
            push_event(events, capacity, count, r.id, 2, tok, r.status);
            if ((st = release(s, r)) != NDL_OK) return st;
        }
    }
    s->admitted.erase(std::remove_if(s->admitted.begin(), s->admitted.end(),
                                     [&](int id) { return s->requests[id].state == State::Done; }),
                      s->admitted.end());
    return NDL_OK;
}

NDL_API int ndl_sched_tokens(ndl_sched *s, int request, int32_t *tokens, int capacity, int *count) {
    NDL_REQUIRE(s && count, "null argument");
    auto it = s->requests.find(request);
    NDL_REQUIRE(it != s->requests.end(), "unknown request %d", request);
    const std::vector<int32_t> &out = it->second.out;
    *count = (int)out.size();
    if (tokens) std::copy(out.begin(), out.begin() + std::min<size_t>(out.size(), (size_t)std::max(capacity, 0)), tokens);
    return NDL_OK;
}

NDL_API int ndl_sched_pending(ndl_sched *s, int *waiting, int *running) {
    NDL_REQUIRE(s, "null scheduler");
    if (waiting) *waiting = (int)s->waiting.size();
    if (running) *running = (int)s->admitted.size();
    return NDL_OK;
}

// The last step's packing: tokens and slots per row, head rows.  Arrays of
// at least max_rows entries (NULL to skip).
NDL_API int ndl_sched_last_plan(ndl_sched *s, int *tokens, int *row_slots, int *rows, int *head_rows, int *heads) {
    NDL_REQUIRE(s && rows && heads, "null argument");
    *rows = (int)s->tokens.size();
    *heads = (int)s->head_rows.size();
    if (tokens) std::copy(s->tokens.begin(), s->tokens.end(), tokens);
    if (row_slots) std::copy(s->row_slots.begin(), s->row_slots.end(), row_slots);
    if (head_rows) std::copy(s->head_rows.begin(), s->head_rows.end(), head_rows);
    return NDL_OK;
}

}  // extern "C"
