// kv_state_capi.cpp -- C ABI over the host-side KV state (include/llmhost_kv.h).
//
// Output buffers are checked against their capacities before the state
// changes, so a call that returns an error leaves the state as it was
// (except forward, which drops the previous draft first, as the reference does).
#include <algorithm>
#include <new>

#include "../../include/llmhost_kv.h"
#include "kv_state.h"

using kvb200::KvState;
using kvb200::PageCopy;
using kvb200::SlotMove;
using kvb200::StateStatus;
using kvb200::TokenMove;
using kvb200::TreeError;

struct kv_state {
    KvState impl;
    kv_state(uint32_t n_pages, int n_layers, const uint32_t* order, size_t n_order, int page_tokens)
        : impl(n_pages, n_layers, order, n_order, page_tokens) {}
};

namespace {

int to_status(StateStatus s) { return static_cast<int>(s); }

void put_tree_error(const TreeError& e, kv_tree_error* out) {
    if (!out) return;
    out->kind = static_cast<int32_t>(e.kind);
    out->child = e.child;
    out->parent = e.parent;
    out->tree = e.tree;
    out->tokens = e.tokens;
}

bool put_copies(const std::vector<PageCopy>& v, uint32_t* src, uint32_t* dst, int32_t* n) {
    for (size_t i = 0; i < v.size(); ++i) {
        src[i] = v[i].src;
        dst[i] = v[i].dst;
    }
    if (n) *n = static_cast<int32_t>(v.size());
    return true;
}

void put_moves(const std::vector<SlotMove>& v, int32_t* src, int32_t* dst, int32_t* n) {
    for (size_t i = 0; i < v.size(); ++i) {
        src[i] = v[i].src;
        dst[i] = v[i].dst;
    }
    if (n) *n = static_cast<int32_t>(v.size());
}

}  // namespace

extern "C" {

int kv_tree_validate(const int32_t* tree, int32_t tree_len, int32_t tokens, kv_tree_error* err) {
    if ((!tree && tree_len > 0) || tree_len < 0 || tokens < 0) return KV_ERR_INVALID;
    const TreeError e = kvb200::validate_tree_for_tokens(tree, static_cast<size_t>(tree_len),
                                                         static_cast<size_t>(tokens));
    put_tree_error(e, err);
    return e.kind == kvb200::TreeErrorKind::None ? KV_OK : KV_ERR_TREE;
}

int kv_tree_validate_accept(const int32_t* tree, int32_t tree_len, const int64_t* accepted, int32_t n,
                            kv_tree_error* err) {
    if ((!tree && tree_len > 0) || tree_len < 0 || n < 0 || (!accepted && n > 0)) return KV_ERR_INVALID;
    const TreeError e = kvb200::validate_accept_path(tree, static_cast<size_t>(tree_len), accepted,
                                                     static_cast<size_t>(n));
    put_tree_error(e, err);
    return e.kind == kvb200::TreeErrorKind::None ? KV_OK : KV_ERR_TREE;
}

int kv_state_create(uint32_t n_pages, int32_t n_layers, int32_t page_tokens, const uint32_t* alloc_order,
                    uint32_t n_order, kv_state** out) {
    if (!out || n_pages == 0 || n_layers <= 0 || page_tokens <= 0) return KV_ERR_INVALID;
    *out = nullptr;
    if (alloc_order) {
        // The order must be a permutation of a subset of [0, n_pages): no repeats.
        std::vector<uint8_t> seen(n_pages, 0);
        for (uint32_t i = 0; i < n_order; ++i) {
            if (alloc_order[i] >= n_pages || seen[alloc_order[i]]) return KV_ERR_INVALID;
            seen[alloc_order[i]] = 1;
        }
    }
    kv_state* s = new (std::nothrow) kv_state(n_pages, n_layers, alloc_order, alloc_order ? n_order : 0, page_tokens);
    if (!s) return KV_ERR_OOM;
    *out = s;
    return KV_OK;
}

int kv_state_destroy(kv_state* st) {
    if (!st) return KV_ERR_INVALID;
    delete st;
    return KV_OK;
}

int kv_state_open(kv_state* st, uint64_t seq_id) {
    if (!st) return KV_ERR_INVALID;
    st->impl.open(seq_id);
    return KV_OK;
}

int kv_state_close(kv_state* st, uint64_t seq_id) {
    if (!st) return KV_ERR_INVALID;
    if (!st->impl.has(seq_id)) return KV_ERR_UNKNOWN_SEQ;
    st->impl.close(seq_id);
    return KV_OK;
}

int kv_state_fork(kv_state* st, uint64_t src, uint64_t dst) {
    if (!st) return KV_ERR_INVALID;
    return to_status(st->impl.fork(src, dst));
}

int kv_state_append(kv_state* st, uint64_t seq_id, const uint32_t* tokens, int32_t n, uint32_t* cow_src,
                    uint32_t* cow_dst, int32_t cow_cap, int32_t* n_cow) {
    if (!st || n < 0) return KV_ERR_INVALID;
    if (cow_cap < st->impl.n_layers() || !cow_src || !cow_dst) return KV_ERR_INVALID;
    std::vector<PageCopy> cow;
    const StateStatus s = st->impl.append(seq_id, tokens, n, &cow);
    if (s != StateStatus::Ok) return to_status(s);
    put_copies(cow, cow_src, cow_dst, n_cow);
    return KV_OK;
}

int kv_state_forward(kv_state* st, uint64_t seq_id, const uint32_t* tokens, int32_t n, const int32_t* tree,
                     int32_t tree_len, int32_t* slots, int32_t* positions, uint32_t* cow_src, uint32_t* cow_dst,
                     int32_t cow_cap, int32_t* n_cow, kv_tree_error* err) {
    if (!st || n < 0 || (n > 0 && !tokens) || (tree && tree_len < 0)) return KV_ERR_INVALID;
    if (cow_cap < st->impl.n_layers() || !cow_src || !cow_dst || (n > 0 && (!slots || !positions)))
        return KV_ERR_INVALID;
    std::vector<int32_t> sl, po;
    std::vector<PageCopy> cow;
    TreeError e;
    const StateStatus s = st->impl.forward(seq_id, tokens, static_cast<size_t>(n), tree,
                                           tree ? static_cast<size_t>(tree_len) : 0, &e, &sl, &po, &cow);
    put_tree_error(e, err);
    if (s != StateStatus::Ok) return to_status(s);
    for (size_t i = 0; i < sl.size(); ++i) {
        slots[i] = sl[i];
        positions[i] = po[i];
    }
    put_copies(cow, cow_src, cow_dst, n_cow);
    return KV_OK;
}

static int finish_commit(kv_state* st, uint64_t seq_id, bool is_accept, const int64_t* idx, int32_t n,
                         int32_t* move_src, int32_t* move_dst, int32_t move_cap, int32_t* n_moves,
                         kv_token_move* tok_moves, int32_t tok_cap, int32_t* n_tok_moves, int64_t* bad_index) {
    if (!st || n < 0 || (n > 0 && !idx)) return KV_ERR_INVALID;
    int64_t pend = 0;
    const StateStatus ps = st->impl.pending_size(seq_id, &pend);
    if (ps != StateStatus::Ok) return to_status(ps);
    if (pend > 0 && (move_cap < pend || !move_src || !move_dst)) return KV_ERR_INVALID;
    if (tok_moves && tok_cap < pend * st->impl.n_layers()) return KV_ERR_INVALID;
    std::vector<SlotMove> moves;
    std::vector<TokenMove> pages;
    std::vector<TokenMove>* pp = tok_moves ? &pages : nullptr;
    const StateStatus s = is_accept ? st->impl.accept(seq_id, idx, static_cast<size_t>(n), bad_index, &moves, pp)
                                    : st->impl.rollback(seq_id, idx, static_cast<size_t>(n), bad_index, &moves, pp);
    if (s != StateStatus::Ok) return to_status(s);
    put_moves(moves, move_src, move_dst, n_moves);
    if (tok_moves) {
        for (size_t i = 0; i < pages.size(); ++i)
            tok_moves[i] = kv_token_move{pages[i].src_page, pages[i].src_slot, pages[i].dst_page, pages[i].dst_slot};
        if (n_tok_moves) *n_tok_moves = static_cast<int32_t>(pages.size());
    } else if (n_tok_moves) {
        *n_tok_moves = 0;
    }
    return KV_OK;
}

int kv_state_accept(kv_state* st, uint64_t seq_id, const int64_t* accepted, int32_t n, int32_t* move_src,
                    int32_t* move_dst, int32_t move_cap, int32_t* n_moves, kv_token_move* tok_moves,
                    int32_t tok_cap, int32_t* n_tok_moves, int64_t* bad_index) {
    return finish_commit(st, seq_id, true, accepted, n, move_src, move_dst, move_cap, n_moves, tok_moves, tok_cap,
                         n_tok_moves, bad_index);
}

int kv_state_rollback(kv_state* st, uint64_t seq_id, const int64_t* rejected, int32_t n, int32_t* move_src,
                      int32_t* move_dst, int32_t move_cap, int32_t* n_moves, kv_token_move* tok_moves,
                      int32_t tok_cap, int32_t* n_tok_moves, int64_t* bad_index) {
    return finish_commit(st, seq_id, false, rejected, n, move_src, move_dst, move_cap, n_moves, tok_moves, tok_cap,
                         n_tok_moves, bad_index);
}

int kv_state_forward_batch(kv_state* st, const uint64_t* seq_ids, int32_t n_seqs, const uint32_t* tokens,
                           const int32_t* tok_off, const int32_t* trees, int32_t* tok_row, int32_t* slots,
                           int32_t* positions, int32_t* prefix, uint64_t* masks, uint32_t* cow_src,
                           uint32_t* cow_dst, int32_t cow_cap, int32_t* n_cow, uint32_t* tables, int32_t stride,
                           int32_t* n_done, kv_tree_error* err) {
    if (n_done) *n_done = 0;
    if (n_cow) *n_cow = 0;
    if (!st || n_seqs < 0) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (!seq_ids || !tok_off || tok_off[0] != 0 || !prefix || !tables || stride <= 0) return KV_ERR_INVALID;
    const int layers = st->impl.n_layers();
    if (static_cast<int64_t>(cow_cap) < static_cast<int64_t>(layers) * n_seqs || !cow_src || !cow_dst)
        return KV_ERR_INVALID;
    const int P = st->impl.page_tokens();
    for (int32_t i = 0; i < n_seqs; ++i) {
        const int32_t n = tok_off[i + 1] - tok_off[i];
        if (n < 0 || (masks && n > 64)) return KV_ERR_INVALID;
        // the draft's tables: the committed ones grown to hold L + n tokens
        int64_t L = 0, len = 0;
        if (st->impl.token_count(seq_ids[i], &L) == StateStatus::Ok) {
            for (int l = 0; l < layers; ++l) {
                const std::vector<uint32_t>* t = nullptr;
                st->impl.table(seq_ids[i], l, 0, &t);
                len = std::max<int64_t>(len, static_cast<int64_t>(t->size()));
            }
        }
        if (std::max<int64_t>(len, (L + n + P - 1) / P) > stride) return KV_ERR_INVALID;
    }
    const int32_t total = tok_off[n_seqs];
    if (total > 0 && (!tokens || !tok_row || !slots || !positions)) return KV_ERR_INVALID;
    std::vector<int32_t> sl, po;
    std::vector<PageCopy> cow;
    int32_t nc = 0;
    for (int32_t i = 0; i < n_seqs; ++i) {
        const int32_t off = tok_off[i], n = tok_off[i + 1] - off;
        const int32_t* tree = trees ? trees + off : nullptr;
        TreeError e;
        cow.clear();
        const StateStatus s = st->impl.forward(seq_ids[i], tokens + off, static_cast<size_t>(n), tree,
                                               tree ? static_cast<size_t>(n) : 0, &e, &sl, &po, &cow);
        put_tree_error(e, err);
        if (s != StateStatus::Ok) return to_status(s);
        for (int32_t k = 0; k < n; ++k) {
            tok_row[off + k] = i;
            slots[off + k] = sl[k];
            positions[off + k] = po[k];
        }
        if (masks) {  // ancestor-or-self bits; the tree was validated (parents precede)
            for (int32_t k = 0; k < n; ++k) {
                const int32_t par = tree ? tree[k] : k - 1;
                masks[off + k] = (par >= 0 ? masks[off + par] : 0ull) | (1ull << k);
            }
        }
        for (const PageCopy& c : cow) {
            cow_src[nc] = c.src;
            cow_dst[nc] = c.dst;
            ++nc;
        }
        int64_t base = 0;
        st->impl.pending_base(seq_ids[i], &base);
        prefix[i] = static_cast<int32_t>(base);
        if (n_done) *n_done = i + 1;
        if (n_cow) *n_cow = nc;
    }
    for (int l = 0; l < layers; ++l) {
        for (int32_t i = 0; i < n_seqs; ++i) {
            const std::vector<uint32_t>* t = nullptr;
            st->impl.table(seq_ids[i], l, 1, &t);
            uint32_t* row = tables + (static_cast<size_t>(l) * n_seqs + i) * stride;
            const int32_t m = static_cast<int32_t>(t->size());
            for (int32_t j = 0; j < stride; ++j) row[j] = j < m ? (*t)[j] : KV_PAGE_NONE;
        }
    }
    return KV_OK;
}

int kv_state_accept_batch(kv_state* st, const uint64_t* seq_ids, int32_t n_seqs, const int64_t* paths,
                          const int32_t* path_off, kv_token_move* tok_moves, int32_t tok_cap, int64_t* tok_need,
                          int32_t* group_off, int32_t* n_done, int64_t* bad_index) {
    if (n_done) *n_done = 0;
    if (tok_need) *tok_need = 0;
    if (!st || n_seqs < 0) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (!seq_ids || !path_off || path_off[0] != 0 || !group_off) return KV_ERR_INVALID;
    const int layers = st->impl.n_layers();
    int64_t need = 0;
    for (int32_t i = 0; i < n_seqs; ++i) {
        if (path_off[i + 1] < path_off[i]) return KV_ERR_INVALID;
        int64_t pend = 0;
        const StateStatus ps = st->impl.pending_size(seq_ids[i], &pend);
        if (ps != StateStatus::Ok) return to_status(ps);
        need += pend * layers;
    }
    if (tok_need) *tok_need = need;
    if (need > tok_cap || (need > 0 && !tok_moves) || (path_off[n_seqs] > 0 && !paths)) return KV_ERR_INVALID;
    std::vector<SlotMove> moves;
    std::vector<TokenMove> pages;
    int32_t nt = 0;
    group_off[0] = 0;
    for (int32_t i = 0; i < n_seqs; ++i) {
        const int32_t off = path_off[i], n = path_off[i + 1] - off;
        moves.clear();
        pages.clear();
        const StateStatus s = st->impl.accept(seq_ids[i], n ? paths + off : nullptr, static_cast<size_t>(n),
                                              bad_index, &moves, &pages);
        if (s != StateStatus::Ok) return to_status(s);
        const int32_t per = static_cast<int32_t>(pages.size()) / layers;  // layer-major, the same per layer
        for (int l = 0; l < layers; ++l) {
            for (int32_t k = 0; k < per; ++k) {
                const TokenMove& m = pages[static_cast<size_t>(l) * per + k];
                tok_moves[nt++] = kv_token_move{m.src_page, m.src_slot, m.dst_page, m.dst_slot};
            }
            group_off[i * layers + l + 1] = nt;
        }
        if (n_done) *n_done = i + 1;
    }
    return KV_OK;
}

int kv_state_evict_window(kv_state* st, uint64_t seq_id, int64_t window, int64_t* n_freed) {
    if (!st) return KV_ERR_INVALID;
    return to_status(st->impl.evict_window(seq_id, window, n_freed));
}

int kv_state_compact(kv_state* st, uint32_t* src, uint32_t* dst, int32_t cap, int32_t* n_moves) {
    if (!st) return KV_ERR_INVALID;
    const uint32_t need = st->impl.compact_moves();
    if (n_moves) *n_moves = static_cast<int32_t>(need);
    if (need > 0 && (cap < static_cast<int32_t>(need) || !src || !dst)) return KV_ERR_INVALID;
    std::vector<PageCopy> moves;
    st->impl.compact(&moves);
    put_copies(moves, src, dst, n_moves);
    return KV_OK;
}

int kv_state_token_count(const kv_state* st, uint64_t seq_id, int64_t* n) {
    if (!st || !n) return KV_ERR_INVALID;
    return to_status(st->impl.token_count(seq_id, n));
}

int kv_state_committed(const kv_state* st, uint64_t seq_id, uint32_t* tokens, int64_t cap, int64_t* n) {
    if (!st || !n) return KV_ERR_INVALID;
    const std::vector<uint32_t>* v = nullptr;
    const StateStatus s = st->impl.committed(seq_id, &v);
    if (s != StateStatus::Ok) return to_status(s);
    *n = static_cast<int64_t>(v->size());
    if (cap < *n || (*n > 0 && !tokens)) return KV_ERR_INVALID;
    for (size_t i = 0; i < v->size(); ++i) tokens[i] = (*v)[i];
    return KV_OK;
}

int kv_state_table(const kv_state* st, uint64_t seq_id, int32_t layer, int32_t which, uint32_t* out, int64_t cap,
                   int64_t* n) {
    if (!st || !n) return KV_ERR_INVALID;
    const std::vector<uint32_t>* t = nullptr;
    const StateStatus s = st->impl.table(seq_id, layer, which, &t);
    if (s != StateStatus::Ok) return to_status(s);
    *n = static_cast<int64_t>(t->size());
    if (cap < *n || (*n > 0 && !out)) return KV_ERR_INVALID;
    for (size_t i = 0; i < t->size(); ++i) out[i] = (*t)[i];
    return KV_OK;
}

int kv_state_export_tables(const kv_state* st, const uint64_t* seq_ids, int32_t n_seqs, int32_t layer,
                           int32_t which, uint32_t* out, int32_t stride) {
    if (!st || n_seqs < 0 || stride <= 0 || (n_seqs > 0 && (!seq_ids || !out))) return KV_ERR_INVALID;
    for (int32_t i = 0; i < n_seqs; ++i) {
        const std::vector<uint32_t>* t = nullptr;
        const StateStatus s = st->impl.table(seq_ids[i], layer, which, &t);
        if (s != StateStatus::Ok) return to_status(s);
        if (static_cast<int64_t>(t->size()) > stride) return KV_ERR_INVALID;
    }
    for (int32_t i = 0; i < n_seqs; ++i) {
        const std::vector<uint32_t>* t = nullptr;
        st->impl.table(seq_ids[i], layer, which, &t);
        uint32_t* row = out + static_cast<size_t>(i) * stride;
        for (int32_t j = 0; j < stride; ++j) row[j] = j < static_cast<int32_t>(t->size()) ? (*t)[j] : KV_PAGE_NONE;
    }
    return KV_OK;
}

int kv_state_free_list(const kv_state* st, uint32_t* out, int64_t cap, int64_t* n) {
    if (!st || !n) return KV_ERR_INVALID;
    const std::vector<uint32_t> f = st->impl.free_list();
    *n = static_cast<int64_t>(f.size());
    if (cap < *n || (*n > 0 && !out)) return KV_ERR_INVALID;
    for (size_t i = 0; i < f.size(); ++i) out[i] = f[i];
    return KV_OK;
}

int kv_state_refcount(const kv_state* st, uint32_t page, uint32_t* count) {
    if (!st || !count || page >= st->impl.n_pages()) return KV_ERR_INVALID;
    *count = st->impl.refcount(page);
    return KV_OK;
}

int kv_state_pending_base(const kv_state* st, uint64_t seq_id, int64_t* base) {
    if (!st || !base) return KV_ERR_INVALID;
    return to_status(st->impl.pending_base(seq_id, base));
}

}  // extern "C"
