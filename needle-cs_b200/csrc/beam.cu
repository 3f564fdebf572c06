// Beam search over many utterances at once (Whistle-shaped decoders).
//
// Whistle.BeamSearch (src/Needle/Whistle.Decode.cs:224-350) per utterance,
// with every live beam of every utterance in one ndl_forward_batch per step
// and one TopKLogSoftmax launch (ndl_sample_topk) for all of them.  Beams are
// engine slots: the utterance owns 2*width slots (`live` and `next`, as the
// reference owns 2*width engines); a child that is not its parent's last
// child starts as a copy of the parent (ndl_slot_copy, Engine.CopyFrom
// src/Needle/Engine.cs:367-379), the last child continues in the parent's
// slot.  Selection per step, as in the reference: candidates = beam score +
// log-prob (fp32), sorted by score descending (equal scores keep their
// (beam, rank) order: the reference's List.Sort leaves that order open), EOS
// candidates become finished hypotheses, at most `width` others stay live;
// the search of an utterance stops when nothing stays live, or when `width`
// hypotheses finished and the best normalised finished score
// score/(len+1)^penalty is at least the best normalised live one.  The
// winner is the best finished hypothesis, else the best live one
// (score/len^penalty).
//
// Host code; one host thread per engine.
#include <algorithm>
#include <cmath>
#include <vector>

#include "common.cuh"

namespace {

struct Cand {
    float score;
    int parent, token;
};

struct Utt {
    int memory;
    std::vector<int> live, next;  // slot ids
    std::vector<std::vector<int>> tokens;
    std::vector<float> scores;
    int live_count = 1;
    std::vector<std::pair<float, std::vector<int>>> finished;
    bool done = false;
};

float normalized(float score, int length, float penalty) {
    return penalty == 0.0f ? score : score / powf((float)length, penalty);
}

}  // namespace

extern "C" {

NDL_API int ndl_beam_search(ndl_engine *e, const ndl_beam_config *cfg, int utterances, const int *memory_slots,
                            const int *beam_slots, const int32_t *prompt, int prompt_len, int32_t *tokens,
                            int *lengths, float *scores, long long *rows_run) {
    NDL_REQUIRE(e && cfg && memory_slots && beam_slots && prompt && tokens && lengths, "null argument");
    const int W = cfg->width;
    NDL_REQUIRE(W >= 1 && W <= 8, "width %d outside 1..8", W);
    NDL_REQUIRE(utterances >= 1 && prompt_len >= 1 && cfg->max_steps >= 1, "utterances=%d prompt_len=%d",
                utterances, prompt_len);
    ndl_engine_info info{};
    int st = ndl_engine_get_info(e, &info);
    if (st != NDL_OK) return st;
    NDL_REQUIRE((long long)utterances * prompt_len <= info.max_rows && (long long)utterances * W <= info.max_heads &&
                    (long long)utterances * W <= info.max_rows,
                "%d utterances x beam %d (prompt %d) exceed the engine's rows %d / heads %d", utterances, W,
                prompt_len, info.max_rows, info.max_heads);
    std::vector<Utt> us(utterances);
    for (int u = 0; u < utterances; u++) {
        Utt &t = us[u];
        t.memory = memory_slots[u];
        t.live.assign(beam_slots + (size_t)u * 2 * W, beam_slots + (size_t)u * 2 * W + W);
        t.next.assign(beam_slots + (size_t)u * 2 * W + W, beam_slots + (size_t)(u + 1) * 2 * W);
        t.tokens.assign(W, {});
        t.scores.assign(W, 0.0f);
        for (int b = 0; b < 2 * W; b++) {
            const int sl = beam_slots[(size_t)u * 2 * W + b];
            if ((st = ndl_slot_reset(e, sl)) != NDL_OK) return st;
            if ((st = ndl_slot_attach_memory(e, sl, t.memory)) != NDL_OK) return st;
        }
    }
    // the prompt of every utterance in beam 0: one prefill run each
    std::vector<int> rows_tok, rows_slot, heads;
    for (int u = 0; u < utterances; u++) {
        for (int i = 0; i < prompt_len; i++) {
            rows_tok.push_back(prompt[i]);
            rows_slot.push_back(us[u].live[0]);
        }
        heads.push_back((int)rows_tok.size() - 1);
    }
    std::vector<int> head_utt(utterances), head_beam(utterances, 0);
    for (int u = 0; u < utterances; u++) head_utt[u] = u;
    std::vector<int> ids((size_t)utterances * W * W);
    std::vector<float> logp((size_t)utterances * W * W);
    long long rows_total = 0;
    for (int step = 0; step < cfg->max_steps; step++) {
        // logits of every live beam (step 0: the prompts), then their top-W
        rows_total += (long long)rows_tok.size();
        if ((st = ndl_forward_batch(e, rows_tok.data(), rows_slot.data(), (int)rows_tok.size(), heads.data(),
                                    (int)heads.size())) != NDL_OK)
            return st;
        if ((st = ndl_sample_topk(e, W, cfg->mask_special_023, ids.data(), logp.data(), nullptr)) != NDL_OK)
            return st;
        // candidates per utterance, in (beam, rank) order
        std::vector<std::vector<Cand>> cands(utterances);
        for (size_t h = 0; h < heads.size(); h++) {
            Utt &t = us[head_utt[h]];
            const int b = head_beam[h];
            for (int k = 0; k < W; k++)
                cands[head_utt[h]].push_back(Cand{t.scores[b] + logp[h * W + k], b, ids[h * W + k]});
        }
        rows_tok.clear();
        rows_slot.clear();
        heads.clear();
        head_utt.clear();
        head_beam.clear();
        for (int u = 0; u < utterances; u++) {
            Utt &t = us[u];
            if (t.done) continue;
            std::vector<Cand> &c = cands[u];
            std::stable_sort(c.begin(), c.end(), [](const Cand &a, const Cand &b) { return a.score > b.score; });
            std::vector<Cand> kept;
            for (const Cand &x : c) {
                if (x.token == cfg->eos)
                    t.finished.push_back({x.score, t.tokens[x.parent]});
                else
                    kept.push_back(x);
                if ((int)kept.size() >= W) break;
            }
            if (kept.empty()) {
                t.done = true;
                continue;
            }
            if ((int)t.finished.size() >= W) {
                float best_f = -INFINITY, best_l = -INFINITY;
                for (auto &f : t.finished)
                    best_f = std::max(best_f, normalized(f.first, (int)f.second.size() + 1, cfg->length_penalty));
                for (auto &k : kept)
                    best_l = std::max(best_l,
                                      normalized(k.score, (int)t.tokens[k.parent].size() + 1, cfg->length_penalty));
                if (best_f >= best_l) {
                    t.done = true;
                    continue;
                }
            }
            // fork as the reference does: children that are not their
            // parent's last start in next[j] as a copy of the parent; the
            // last child takes the parent's slot (swapped into next[j]);
            // then live and next trade places
            const int kc = (int)kept.size();
            std::vector<int> last_child(W, -1);
            for (int j = 0; j < kc; j++) last_child[kept[j].parent] = j;
            std::vector<std::vector<int>> new_tokens(W);
            std::vector<float> new_scores(W, 0.0f);
            for (int j = 0; j < kc; j++) {
                const int p = kept[j].parent;
                if (j == last_child[p]) continue;
                if ((st = ndl_slot_copy(e, t.next[j], t.live[p])) != NDL_OK) return st;
                new_tokens[j] = t.tokens[p];
                new_tokens[j].push_back(kept[j].token);
                new_scores[j] = kept[j].score;
            }
            for (int j = 0; j < kc; j++) {
                const int p = kept[j].parent;
                if (j != last_child[p]) continue;
                std::swap(t.next[j], t.live[p]);
                new_tokens[j] = t.tokens[p];
                new_tokens[j].push_back(kept[j].token);
                new_scores[j] = kept[j].score;
            }
            std::swap(t.live, t.next);
            t.tokens = new_tokens;
            t.scores = new_scores;
            t.live_count = kc;
            for (int j = 0; j < kc; j++) {
                rows_tok.push_back(kept[j].token);
                rows_slot.push_back(t.live[j]);
                heads.push_back((int)rows_tok.size() - 1);
                head_utt.push_back(u);
                head_beam.push_back(j);
            }
        }
        if (rows_tok.empty()) break;
    }
    if (rows_run) *rows_run = rows_total;
    // winners
    for (int u = 0; u < utterances; u++) {
        Utt &t = us[u];
        const std::vector<int> *best = nullptr;
        float best_score = -INFINITY;
        for (auto &f : t.finished) {
            const float v = normalized(f.first, (int)f.second.size() + 1, cfg->length_penalty);
            if (v > best_score) best_score = v, best = &f.second;
        }
        if (!best)
            for (int j = 0; j < t.live_count; j++) {
                const float v = normalized(t.scores[j], (int)t.tokens[j].size(), cfg->length_penalty);
                if (v > best_score) best_score = v, best = &t.tokens[j];
            }
        const int n = best ? std::min((int)best->size(), cfg->max_steps) : 0;
        for (int i = 0; i < n; i++) tokens[(size_t)u * cfg->max_steps + i] = (*best)[i];
        lengths[u] = n;
        if (scores) scores[u] = best_score;
    }
    return NDL_OK;
}

}  // extern "C"
