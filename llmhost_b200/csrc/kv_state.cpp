// kv_state.cpp -- host-side KV state (see kv_state.h for the rules).
#include "kv_state.h"

#include <algorithm>
#include <unordered_set>

namespace kvb200 {

// ---- tree.rs:41-123 --------------------------------------------------------
std::vector<int32_t> linear_tree(size_t len) {
    std::vector<int32_t> t(len);
    for (size_t i = 0; i < len; ++i) t[i] = i == 0 ? -1 : static_cast<int32_t>(i - 1);
    return t;
}

TreeError validate_tree(const int32_t* tree, size_t n) {
    TreeError e;
    for (size_t child = 0; child < n; ++child) {
        const int32_t parent = tree[child];
        if (parent == -1) continue;
        if (parent < 0 || static_cast<size_t>(parent) >= n) {
            e.kind = TreeErrorKind::ParentOutOfRange;
            e.child = static_cast<int64_t>(child);
            e.parent = parent;
            return e;
        }
        if (static_cast<size_t>(parent) >= child) {
            e.kind = TreeErrorKind::ParentDoesNotPrecede;
            e.child = static_cast<int64_t>(child);
            e.parent = parent;
            return e;
        }
    }
    return e;
}

TreeError validate_tree_for_tokens(const int32_t* tree, size_t n, size_t tokens) {
    if (n != tokens) {
        TreeError e;
        e.kind = TreeErrorKind::LengthMismatch;
        e.tree = static_cast<int64_t>(n);
        e.tokens = static_cast<int64_t>(tokens);
        return e;
    }
    return validate_tree(tree, n);
}

TreeError validate_accept_path(const int32_t* tree, size_t n, const int64_t* accepted, size_t na) {
    TreeError e;
    std::unordered_set<int64_t> set(accepted, accepted + na);
    if (set.size() != na) {
        // A duplicate is reported as ParentDoesNotPrecede { child: first repeated index, parent: -2 }.
        int64_t dup = 0;
        for (size_t i = 0; i < na && dup == 0; ++i) {
            size_t count = 0;
            for (size_t j = 0; j < na; ++j) count += accepted[j] == accepted[i];
            if (count > 1) dup = accepted[i];
        }
        e.kind = TreeErrorKind::ParentDoesNotPrecede;
        e.child = dup;
        e.parent = -2;
        return e;
    }
    for (size_t i = 0; i < na; ++i) {
        const int64_t child = accepted[i];
        if (child < 0 || static_cast<size_t>(child) >= n) {
            e.kind = TreeErrorKind::ParentOutOfRange;
            e.child = child;
            e.parent = static_cast<int32_t>(child);
            return e;
        }
        const int32_t parent = tree[child];
        if (parent == -1) continue;
        if (parent < 0 || static_cast<size_t>(parent) >= n) {
            e.kind = TreeErrorKind::ParentOutOfRange;
            e.child = child;
            e.parent = parent;
            return e;
        }
        if (!set.count(parent)) {
            e.kind = TreeErrorKind::ParentDoesNotPrecede;
            e.child = child;
            e.parent = parent;
            return e;
        }
    }
    return e;
}

// ---- allocator ---------------------------------------------------------------
KvState::KvState(uint32_t n_pages, int n_layers, const uint32_t* order, size_t n_order, int page_tokens)
    : n_pages_(n_pages), n_layers_(n_layers), P_(page_tokens), ref_(n_pages, 0) {
    free_.reserve(n_pages);
    if (order && n_order) {
        for (size_t i = n_order; i-- > 0;) free_.push_back(order[i]);
    } else {
        for (uint32_t i = n_pages; i-- > 0;) free_.push_back(i);
    }
}

std::vector<uint32_t> KvState::free_list() const { return std::vector<uint32_t>(free_.rbegin(), free_.rend()); }

uint32_t KvState::alloc() {
    const uint32_t p = free_.back();
    free_.pop_back();
    ref_[p] = 1;
    return p;
}

void KvState::incref(uint32_t p) { ++ref_[p]; }

void KvState::decref(uint32_t p) {
    if (--ref_[p] == 0) free_.push_back(p);
}

void KvState::release_tables(std::vector<std::vector<uint32_t>>& tables) {
    for (auto& t : tables)
        for (uint32_t p : t)
            if (p != kNoPage) decref(p);
    tables.assign(n_layers_, {});
}

std::vector<std::vector<uint32_t>> KvState::share_tables(const std::vector<std::vector<uint32_t>>& tables) {
    for (const auto& t : tables)
        for (uint32_t p : t)
            if (p != kNoPage) incref(p);
    return tables;
}

int64_t KvState::pages_needed(const std::vector<std::vector<uint32_t>>& tables, int64_t start, int64_t n) const {
    if (n <= 0) return 0;
    int64_t need = 0;
    const int64_t want = (start + n + P_ - 1) / P_;
    for (const auto& t : tables) {
        if (start % P_ != 0) {
            const uint32_t tail = t[start / P_];
            if (tail != kNoPage && ref_[tail] > 1) ++need;
        }
        need += std::max<int64_t>(0, want - static_cast<int64_t>(t.size()));
    }
    return need;
}

void KvState::grow(std::vector<std::vector<uint32_t>>& tables, int64_t start, int64_t n, std::vector<PageCopy>* cow) {
    if (n <= 0) return;
    const size_t want = static_cast<size_t>((start + n + P_ - 1) / P_);
    for (auto& t : tables) {
        if (start % P_ != 0) {
            uint32_t& tail = t[start / P_];
            if (tail != kNoPage && ref_[tail] > 1) {  // copy-on-write of the shared partial page
                const uint32_t fresh = alloc();
                if (cow) cow->push_back({tail, fresh});
                decref(tail);
                tail = fresh;
            }
        }
        while (t.size() < want) t.push_back(alloc());
    }
}

// ---- sessions ------------------------------------------------------------------
void KvState::open(uint64_t seq) {
    close(seq);
    Session s;
    s.tables.assign(n_layers_, {});
    sessions_.emplace(seq, std::move(s));
}

void KvState::close(uint64_t seq) {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return;
    if (it->second.pending) release_tables(it->second.pending->tables);
    release_tables(it->second.tables);
    sessions_.erase(it);
}

StateStatus KvState::fork(uint64_t src, uint64_t dst) {
    auto it = sessions_.find(src);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    if (src == dst || sessions_.count(dst)) return StateStatus::Invalid;
    Session s;
    s.tables = share_tables(it->second.tables);
    s.n_tokens = it->second.n_tokens;
    s.committed = it->second.committed;
    sessions_.emplace(dst, std::move(s));
    return StateStatus::Ok;
}

StateStatus KvState::append(uint64_t seq, const uint32_t* tokens, int64_t n, std::vector<PageCopy>* cow) {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    Session& s = it->second;
    if (n < 0 || s.pending) return StateStatus::Invalid;
    if (pages_needed(s.tables, s.n_tokens, n) > static_cast<int64_t>(free_.size())) return StateStatus::Oom;
    grow(s.tables, s.n_tokens, n, cow);
    s.n_tokens += n;
    for (int64_t i = 0; i < n; ++i) s.committed.push_back(tokens ? tokens[i] : 0u);
    return StateStatus::Ok;
}

StateStatus KvState::forward(uint64_t seq, const uint32_t* tokens, size_t n, const int32_t* tree, size_t tree_len,
                             TreeError* terr,
                             std::vector<int32_t>* slots, std::vector<int32_t>* positions,
                             std::vector<PageCopy>* cow) {
    // effective_tree (tree.rs:75-83): a missing tree is a linear chain.
    std::vector<int32_t> t = tree ? std::vector<int32_t>(tree, tree + tree_len) : linear_tree(n);
    if (tree) {
        const TreeError e = validate_tree_for_tokens(t.data(), tree_len, n);
        if (e.kind != TreeErrorKind::None) {
            if (terr) *terr = e;
            return StateStatus::Tree;
        }
    }
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) {  // forward on an unknown sequence opens it (batch.rs:177-187)
        Session s;
        s.tables.assign(n_layers_, {});
        it = sessions_.emplace(seq, std::move(s)).first;
    }
    Session& s = it->second;
    if (s.pending) {  // a second forward drops the uncommitted draft (batch.rs:189-192)
        release_tables(s.pending->tables);
        s.pending.reset();
    }
    Draft d;
    d.tables = share_tables(s.tables);
    d.base = s.n_tokens;
    if (pages_needed(d.tables, d.base, static_cast<int64_t>(n)) > static_cast<int64_t>(free_.size())) {
        release_tables(d.tables);
        return StateStatus::Oom;
    }
    grow(d.tables, d.base, static_cast<int64_t>(n), cow);
    d.tokens.assign(tokens, tokens + n);
    d.tree = t;
    std::vector<int32_t> depth(n, 0);
    for (size_t i = 0; i < n; ++i) depth[i] = t[i] == -1 ? 0 : depth[static_cast<size_t>(t[i])] + 1;
    if (slots) slots->clear();
    if (positions) positions->clear();
    for (size_t i = 0; i < n; ++i) {
        if (slots) slots->push_back(static_cast<int32_t>(d.base + static_cast<int64_t>(i)));
        if (positions) positions->push_back(static_cast<int32_t>(d.base + depth[i]));
    }
    s.pending = std::move(d);
    return StateStatus::Ok;
}

StateStatus KvState::accept(uint64_t seq, const int64_t* accepted, size_t na, int64_t* bad_index,
                            std::vector<SlotMove>* moves, std::vector<TokenMove>* pages) {
    return commit(seq, std::vector<int64_t>(accepted, accepted + na), bad_index, moves, pages);
}

StateStatus KvState::rollback(uint64_t seq, const int64_t* rejected, size_t nr, int64_t* bad_index,
                              std::vector<SlotMove>* moves, std::vector<TokenMove>* pages) {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    if (!it->second.pending) return StateStatus::NoPending;
    std::unordered_set<int64_t> rej(rejected, rejected + nr);
    std::vector<int64_t> acc;
    for (size_t i = 0; i < it->second.pending->tokens.size(); ++i)
        if (!rej.count(static_cast<int64_t>(i))) acc.push_back(static_cast<int64_t>(i));
    return commit(seq, acc, bad_index, moves, pages);
}

StateStatus KvState::commit(uint64_t seq, const std::vector<int64_t>& accepted, int64_t* bad_index,
                            std::vector<SlotMove>* moves, std::vector<TokenMove>* pages) {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    Session& s = it->second;
    if (!s.pending) return StateStatus::NoPending;
    Draft& d = *s.pending;
    const TreeError e = validate_accept_path(d.tree.data(), d.tree.size(), accepted.data(), accepted.size());
    if (e.kind != TreeErrorKind::None) {
        if (bad_index)
            *bad_index = e.kind == TreeErrorKind::LengthMismatch ? (accepted.empty() ? 0 : accepted[0]) : e.child;
        return StateStatus::InvalidAccept;
    }
    for (int64_t idx : accepted)
        if (idx < 0 || static_cast<size_t>(idx) >= d.tokens.size()) {
            if (bad_index) *bad_index = idx;
            return StateStatus::InvalidAccept;
        }
    // Parents precede children, so index order follows the path (batch.rs:278-281).
    std::vector<int64_t> order = accepted;
    std::sort(order.begin(), order.end());
    order.erase(std::unique(order.begin(), order.end()), order.end());
    const int64_t a = static_cast<int64_t>(order.size());
    std::vector<SlotMove> mv;
    for (int64_t j = 0; j < a; ++j)
        if (order[j] != j) mv.push_back({static_cast<int32_t>(d.base + order[j]), static_cast<int32_t>(d.base + j)});
    if (pages) {
        pages->clear();
        for (const auto& t : d.tables)
            for (const SlotMove& m : mv)
                pages->push_back({t[m.src / P_], m.src % P_, t[m.dst / P_], m.dst % P_});
    }
    if (moves) *moves = mv;
    // Free the draft's pages past the accepted tokens (the rejected branches).
    const size_t keep = static_cast<size_t>((d.base + a + P_ - 1) / P_);
    for (auto& t : d.tables) {
        for (size_t i = t.size(); i-- > keep;)
            if (t[i] != kNoPage) decref(t[i]);
        if (t.size() > keep) t.resize(keep);
    }
    release_tables(s.tables);
    s.tables = std::move(d.tables);
    for (int64_t i : order) s.committed.push_back(d.tokens[static_cast<size_t>(i)]);
    s.n_tokens = d.base + a;
    s.pending.reset();
    return StateStatus::Ok;
}

StateStatus KvState::evict_window(uint64_t seq, int64_t window, int64_t* freed) {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    Session& s = it->second;
    if (window <= 0 || s.pending) return StateStatus::Invalid;
    const int64_t lo = std::max<int64_t>(0, s.n_tokens - window);
    int64_t count = 0;
    for (auto& t : s.tables) {
        const size_t end = std::min(t.size(), static_cast<size_t>(lo / P_));
        for (size_t i = 0; i < end; ++i)
            if (t[i] != kNoPage) {
                decref(t[i]);
                t[i] = kNoPage;
                ++count;
            }
    }
    if (freed) *freed = count;
    return StateStatus::Ok;
}

void KvState::compact(std::vector<PageCopy>* moves) {
    const uint32_t used = n_pages_ - static_cast<uint32_t>(free_.size());
    std::vector<uint32_t> holes, movers;
    for (uint32_t p = 0; p < used; ++p)
        if (ref_[p] == 0) holes.push_back(p);
    for (uint32_t p = used; p < n_pages_; ++p)
        if (ref_[p] > 0) movers.push_back(p);
    if (moves) moves->clear();
    if (!movers.empty()) {
        std::vector<uint32_t> remap(n_pages_);
        for (uint32_t p = 0; p < n_pages_; ++p) remap[p] = p;
        for (size_t i = 0; i < movers.size(); ++i) {
            remap[movers[i]] = holes[i];
            ref_[holes[i]] = ref_[movers[i]];
            ref_[movers[i]] = 0;
            if (moves) moves->push_back({movers[i], holes[i]});
        }
        auto fix = [&](std::vector<std::vector<uint32_t>>& tables) {
            for (auto& t : tables)
                for (uint32_t& p : t)
                    if (p != kNoPage) p = remap[p];
        };
        for (auto& kv : sessions_) {
            fix(kv.second.tables);
            if (kv.second.pending) fix(kv.second.pending->tables);
        }
    }
    free_.clear();
    for (uint32_t p = n_pages_; p-- > used;) free_.push_back(p);
}

StateStatus KvState::token_count(uint64_t seq, int64_t* n) const {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    *n = it->second.n_tokens;
    return StateStatus::Ok;
}

StateStatus KvState::committed(uint64_t seq, const std::vector<uint32_t>** tokens) const {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    *tokens = &it->second.committed;
    return StateStatus::Ok;
}

StateStatus KvState::table(uint64_t seq, int layer, int which, const std::vector<uint32_t>** t) const {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    if (layer < 0 || layer >= n_layers_) return StateStatus::Invalid;
    if (which == 0) {
        *t = &it->second.tables[layer];
        return StateStatus::Ok;
    }
    if (!it->second.pending) return StateStatus::NoPending;
    *t = &it->second.pending->tables[layer];
    return StateStatus::Ok;
}

StateStatus KvState::pending_size(uint64_t seq, int64_t* n) const {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    *n = it->second.pending ? static_cast<int64_t>(it->second.pending->tokens.size()) : 0;
    return StateStatus::Ok;
}

uint32_t KvState::compact_moves() const {
    const uint32_t used = n_pages_ - static_cast<uint32_t>(free_.size());
    uint32_t m = 0;
    for (uint32_t p = used; p < n_pages_; ++p) m += ref_[p] > 0;
    return m;
}

StateStatus KvState::pending_base(uint64_t seq, int64_t* base) const {
    auto it = sessions_.find(seq);
    if (it == sessions_.end()) return StateStatus::UnknownSeq;
    if (!it->second.pending) return StateStatus::NoPending;
    *base = it->second.pending->base;
    return StateStatus::Ok;
}

}  // namespace kvb200
