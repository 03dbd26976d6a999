// kv_state.h -- host-side KV state: page allocator, block tables, speculation.
//
// This is the state the reference keeps in llm-engine's Engine and PagedKv
// (crates/llm-engine/src/batch.rs:104-297, crates/llm-engine/src/cache.rs:12-51),
// with real pages behind it.  It runs on the host and only plans device work:
// calls return the page copies (copy-on-write, compaction) and token-slot
// moves (accepted draft tokens) that the caller runs with kv_copy_pages /
// kv_move_slots before it launches the next step.
//
// Build-defined rules (the reference has no allocator, fork or eviction):
//   * allocation pops a LIFO free stack seeded so the first page handed out is
//     order[0], then order[1], ...; a page returns to the top of the stack when
//     its reference count drops to 0;
//   * every operation walks layers 0..n_layers-1 in order, and pages of one
//     layer in table order;
//   * appending into a partially filled tail page that another table also
//     references first copies that page (copy-on-write), then new pages are
//     allocated for the rest;
//   * forward() forks a draft from the session (all pages shared); draft token
//     i goes to slot L + i at RoPE position L + depth(i) (depth(root) = 0);
//   * commit moves accepted token order[j] from slot L + order[j] to L + j,
//     frees the draft's pages past ceil((L + a) / P), releases the session's
//     old tables and installs the draft as the session's tables;
//   * evict_window frees, per layer, the pages wholly below n - window;
//   * compact moves every used page with id >= U (U = pages in use) to the
//     lowest free id, in ascending order, and re-seeds the free stack with
//     U, U+1, ... as the next pages to hand out.
#pragma once

#include <cstdint>
#include <optional>
#include <unordered_map>
#include <vector>

namespace kvb200 {

constexpr uint32_t kNoPage = 0xFFFFFFFFu;

// tree.rs:11-19
enum class TreeErrorKind : int32_t { None = 0, LengthMismatch = 1, ParentOutOfRange = 2, ParentDoesNotPrecede = 3 };

struct TreeError {
    TreeErrorKind kind = TreeErrorKind::None;
    int64_t child = 0;   // ParentOutOfRange / ParentDoesNotPrecede
    int64_t parent = 0;
    int64_t tree = 0;    // LengthMismatch
    int64_t tokens = 0;
};

// tree.rs:41-123
std::vector<int32_t> linear_tree(size_t len);
TreeError validate_tree(const int32_t* tree, size_t n);
TreeError validate_tree_for_tokens(const int32_t* tree, size_t n, size_t tokens);
TreeError validate_accept_path(const int32_t* tree, size_t n, const int64_t* accepted, size_t na);

struct PageCopy {
    uint32_t src, dst;
};
struct SlotMove {
    int32_t src, dst;
};
// One token's K/V (all heads of one layer) from one page slot to another.
struct TokenMove {
    uint32_t src_page;
    int32_t src_slot;
    uint32_t dst_page;
    int32_t dst_slot;
};

enum class StateStatus : int32_t {
    Ok = 0,
    Invalid = 1,
    Oom = 3,
    UnknownSeq = 8,
    NoPending = 9,
    InvalidAccept = 10,
    Tree = 11,
};

class KvState {
public:
    KvState(uint32_t n_pages, int n_layers, const uint32_t* order, size_t n_order, int page_tokens);

    uint32_t n_pages() const { return n_pages_; }
    int n_layers() const { return n_layers_; }
    int page_tokens() const { return P_; }
    uint32_t free_pages() const { return static_cast<uint32_t>(free_.size()); }
    uint32_t refcount(uint32_t page) const { return page < n_pages_ ? ref_[page] : 0; }
    // Pages in pop order (next page handed out first).
    std::vector<uint32_t> free_list() const;

    // Engine::open (batch.rs:138-150): replaces any state of seq_id.
    void open(uint64_t seq);
    void close(uint64_t seq);
    bool has(uint64_t seq) const { return sessions_.count(seq) != 0; }
    // New session dst sharing every page of src (copy-on-write later).
    StateStatus fork(uint64_t src, uint64_t dst);
    // Commit n tokens straight into the session (prefill / plain decode).
    StateStatus append(uint64_t seq, const uint32_t* tokens, int64_t n, std::vector<PageCopy>* cow);
    StateStatus pending_size(uint64_t seq, int64_t* n) const;
    // Page moves compact() would make (for sizing the caller's buffers).
    uint32_t compact_moves() const;

    // Engine::forward for one sequence (batch.rs:173-222).
    StateStatus forward(uint64_t seq, const uint32_t* tokens, size_t n, const int32_t* tree, size_t tree_len,
                        TreeError* terr,
                        std::vector<int32_t>* slots, std::vector<int32_t>* positions,
                        std::vector<PageCopy>* cow);
    // Engine::accept / rollback / commit (batch.rs:230-296).
    // `pages` receives the same moves per layer (layer-major), addressed by the
    // draft's pages before the commit frees any of them.
    StateStatus accept(uint64_t seq, const int64_t* accepted, size_t na, int64_t* bad_index,
                       std::vector<SlotMove>* moves, std::vector<TokenMove>* pages = nullptr);
    StateStatus rollback(uint64_t seq, const int64_t* rejected, size_t nr, int64_t* bad_index,
                         std::vector<SlotMove>* moves, std::vector<TokenMove>* pages = nullptr);

    StateStatus evict_window(uint64_t seq, int64_t window, int64_t* freed);
    void compact(std::vector<PageCopy>* moves);

    // Queries.
    StateStatus token_count(uint64_t seq, int64_t* n) const;
    StateStatus committed(uint64_t seq, const std::vector<uint32_t>** tokens) const;
    // which: 0 = committed tables, 1 = the pending draft's.
    StateStatus table(uint64_t seq, int layer, int which, const std::vector<uint32_t>** t) const;
    StateStatus pending_base(uint64_t seq, int64_t* base) const;

private:
    struct Draft {
        std::vector<uint32_t> tokens;
        std::vector<int32_t> tree;
        std::vector<std::vector<uint32_t>> tables;
        int64_t base = 0;
    };
    struct Session {
        std::vector<std::vector<uint32_t>> tables;
        int64_t n_tokens = 0;
        std::vector<uint32_t> committed;
        std::optional<Draft> pending;
    };

    uint32_t alloc();
    void incref(uint32_t p);
    void decref(uint32_t p);
    void release_tables(std::vector<std::vector<uint32_t>>& tables);
    std::vector<std::vector<uint32_t>> share_tables(const std::vector<std::vector<uint32_t>>& tables);
    // Pages an append of n tokens at `start` needs across all layers.
    int64_t pages_needed(const std::vector<std::vector<uint32_t>>& tables, int64_t start, int64_t n) const;
    void grow(std::vector<std::vector<uint32_t>>& tables, int64_t start, int64_t n, std::vector<PageCopy>* cow);
    StateStatus commit(uint64_t seq, const std::vector<int64_t>& accepted, int64_t* bad_index,
                       std::vector<SlotMove>* moves, std::vector<TokenMove>* pages);

    uint32_t n_pages_;
    int n_layers_;
    int P_;
    std::vector<uint32_t> ref_;
    std::vector<uint32_t> free_;  // top of the stack = back()
    std::unordered_map<uint64_t, Session> sessions_;
};

}  // namespace kvb200
