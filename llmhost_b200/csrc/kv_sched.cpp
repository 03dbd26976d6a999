// kv_sched.cpp -- the path's host-side callers: the draft-tree builder and the
// continuous-batching scheduler (C ABI in include/llmhost_kv.h).
//
// The reference has both only as placeholders: a DraftModel hook returning a
// token list and parent array (crates/llm-engine/src/draft.rs:9-23) and a
// Scheduler that tracks live sequence ids and packs them into a batch
// (crates/llm-engine/src/schedule.rs:8-48).  This file keeps their semantics
// and adds what feeding the kernels needs:
//   * kv_draft_tree_best_first: from a draft model's candidates (parent,
//     token, probability given the parent) pick the speculative tree by
//     cumulative probability, best first, within a node and depth budget;
//   * kv_sched_*: running set in insertion order (schedule.rs), queued
//     prompt tokens per sequence, a per-step planner under a token budget
//     (decode tokens first, then prefill chunks), and LPT assignment of
//     sessions to GPUs.
#include <algorithm>
#include <cstdint>
#include <new>
#include <queue>
#include <unordered_map>
#include <vector>

#include "../../include/llmhost_kv.h"

struct kv_sched {
    std::vector<uint64_t> running;                 // insertion order, no duplicates
    std::unordered_map<uint64_t, int64_t> pending;  // queued prompt tokens per running sequence
};

extern "C" {

int kv_draft_tree_best_first(const int32_t* cand_parent, const uint32_t* cand_token, const double* cand_prob,
                             int32_t n_cand, int32_t max_nodes, int32_t max_depth, uint32_t* tokens, int32_t* tree,
                             int32_t* picked, int32_t* n_out) {
    if (n_cand < 0 || max_nodes < 0 || max_depth < 0 || !n_out) return KV_ERR_INVALID;
    if (n_cand > 0 && (!cand_parent || !cand_token || !cand_prob)) return KV_ERR_INVALID;
    if (max_nodes > 0 && (!tokens || !tree)) return KV_ERR_INVALID;
    *n_out = 0;
    std::vector<double> score(static_cast<size_t>(n_cand));
    std::vector<int32_t> depth(static_cast<size_t>(n_cand));
    std::vector<std::vector<int32_t>> kids(static_cast<size_t>(n_cand));
    std::vector<int32_t> roots;
    for (int32_t c = 0; c < n_cand; ++c) {
        const int32_t p = cand_parent[c];
        const double pr = cand_prob[c];
        if (p < -1 || p >= c || !(pr >= 0.0 && pr <= 1.0)) return KV_ERR_INVALID;  // parents first, probabilities
        score[c] = (p < 0 ? 1.0 : score[p]) * pr;
        depth[c] = p < 0 ? 0 : depth[p] + 1;
        if (p < 0)
            roots.push_back(c);
        else
            kids[p].push_back(c);
    }
    // Eligible candidates: roots, and children of picked nodes, no deeper than
    // max_depth.  The most probable (cumulative) goes next; ties to the
    // lower candidate index.
    auto worse = [&](int32_t a, int32_t b) { return score[a] < score[b] || (score[a] == score[b] && a > b); };
    std::priority_queue<int32_t, std::vector<int32_t>, decltype(worse)> open(worse);
    for (int32_t c : roots)
        if (depth[c] <= max_depth) open.push(c);
    std::vector<int32_t> out_pos(static_cast<size_t>(n_cand), -1);
    int32_t n = 0;
    while (n < max_nodes && !open.empty()) {
        const int32_t c = open.top();
        open.pop();
        out_pos[c] = n;
        tokens[n] = cand_token[c];
        tree[n] = cand_parent[c] < 0 ? -1 : out_pos[cand_parent[c]];
        if (picked) picked[n] = c;
        ++n;
        for (int32_t k : kids[c])
            if (depth[k] <= max_depth) open.push(k);
    }
    *n_out = n;
    return KV_OK;
}

int kv_sched_create(kv_sched** out) {
    if (!out) return KV_ERR_INVALID;
    *out = new (std::nothrow) kv_sched();
    return *out ? KV_OK : KV_ERR_OOM;
}

int kv_sched_destroy(kv_sched* s) {
    if (!s) return KV_ERR_INVALID;
    delete s;
    return KV_OK;
}

// schedule.rs:23-27: a sequence already running is not added twice.
int kv_sched_add(kv_sched* s, uint64_t seq_id) {
    if (!s) return KV_ERR_INVALID;
    if (std::find(s->running.begin(), s->running.end(), seq_id) == s->running.end()) {
        s->running.push_back(seq_id);
        s->pending[seq_id] = 0;
    }
    return KV_OK;
}

// schedule.rs:29-31
int kv_sched_remove(kv_sched* s, uint64_t seq_id) {
    if (!s) return KV_ERR_INVALID;
    s->running.erase(std::remove(s->running.begin(), s->running.end(), seq_id), s->running.end());
    s->pending.erase(seq_id);
    return KV_OK;
}

// schedule.rs:34-37 (and schedule.rs:41-47: a batch holds these ids, in this order)
int kv_sched_running(const kv_sched* s, uint64_t* out, int64_t cap, int64_t* n) {
    if (!s || !n) return KV_ERR_INVALID;
    *n = static_cast<int64_t>(s->running.size());
    if (cap < *n || (*n > 0 && !out)) return KV_ERR_INVALID;
    std::copy(s->running.begin(), s->running.end(), out);
    return KV_OK;
}

int kv_sched_set_pending(kv_sched* s, uint64_t seq_id, int64_t prefill_tokens) {
    if (!s || prefill_tokens < 0) return KV_ERR_INVALID;
    auto it = s->pending.find(seq_id);
    if (it == s->pending.end()) return KV_ERR_UNKNOWN_SEQ;
    it->second = prefill_tokens;
    return KV_OK;
}

int kv_sched_plan_step(kv_sched* s, int64_t token_budget, int32_t chunk_tokens, uint64_t* seq_ids,
                       int32_t* n_tokens, int32_t* is_prefill, int32_t cap, int32_t* n_out) {
    if (!s || !n_out || token_budget < 0 || chunk_tokens <= 0 || cap < 0) return KV_ERR_INVALID;
    if (cap < static_cast<int64_t>(s->running.size())) return KV_ERR_INVALID;  // one entry per running sequence at most
    if (!s->running.empty() && (!seq_ids || !n_tokens || !is_prefill)) return KV_ERR_INVALID;
    int32_t n = 0;
    int64_t left = token_budget;
    for (uint64_t id : s->running) {  // decode tokens first: one per sequence with no prompt left
        if (left == 0) break;
        if (s->pending[id] == 0) {
            seq_ids[n] = id;
            n_tokens[n] = 1;
            is_prefill[n] = 0;
            ++n;
            --left;
        }
    }
    for (uint64_t id : s->running) {  // then prompt chunks while the budget lasts
        if (left == 0) break;
        int64_t& q = s->pending[id];
        if (q == 0) continue;
        const int64_t take = std::min<int64_t>({q, static_cast<int64_t>(chunk_tokens), left});
        seq_ids[n] = id;
        n_tokens[n] = static_cast<int32_t>(take);
        is_prefill[n] = 1;
        ++n;
        q -= take;
        left -= take;
    }
    *n_out = n;
    return KV_OK;
}

int kv_sched_lpt(const int64_t* weights, int32_t n, int32_t n_bins, int32_t* bins) {
    if (n < 0 || n_bins <= 0 || (n > 0 && (!weights || !bins))) return KV_ERR_INVALID;
    std::vector<int32_t> order(static_cast<size_t>(n));
    for (int32_t i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return weights[a] > weights[b]; });
    std::vector<int64_t> load(static_cast<size_t>(n_bins), 0);
    for (int32_t i : order) {
        int32_t b = 0;
        for (int32_t k = 1; k < n_bins; ++k)
            if (load[k] < load[b]) b = k;
        bins[i] = b;
        load[b] += weights[i];
    }
    return KV_OK;
}

}  // extern "C"
