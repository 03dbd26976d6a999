// kv_copy.cu -- page-granular and token-granular copies inside the pool.
//
// These run the plans the host-side KV state returns (kv_state_*):
//   kv_copy_pages  copy-on-write page copies and compaction page moves.  The
//                  copies of one call are independent (a page is never both a
//                  source and a destination), so every 16-byte chunk of every
//                  page is copied in parallel: HBM-bound, read + write of
//                  2 * page_bytes per page.
//   kv_move_tokens accepted draft tokens moved into sequence order at commit,
//                  addressed by page.  Moves of one group (one sequence and
//                  layer) run in order, a chunk at a time: every source of a
//                  chunk is read into shared memory before any destination is
//                  written.  That is exact for the moves kv_state_accept /
//                  kv_state_rollback produce (a later move never reads a slot
//                  an earlier move wrote).  Groups run in parallel.  A token
//                  is its row of every page section (K and V; or K codes, V
//                  codes and scales of every head block in quantised pools).
// Page ids past the pool and slots past a page are skipped and flagged in the
// pool's error word.
#include <algorithm>

#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace kvb200 {
namespace {

__global__ void __launch_bounds__(256) copy_pages_kernel(uint4* __restrict__ pages, const uint32_t* src,
                                                         const uint32_t* dst, int n, uint32_t n_pages,
                                                         int page_vecs, int* err) {
    const int i = blockIdx.y;
    if (i >= n) return;
    const uint32_t s = __ldg(src + i), d = __ldg(dst + i);
    if (s >= n_pages || d >= n_pages) {
        if (blockIdx.x == 0 && threadIdx.x == 0) flag_error(err, kDevErrBadPage);
        return;
    }
    const uint4* from = pages + static_cast<size_t>(s) * page_vecs;
    uint4* to = pages + static_cast<size_t>(d) * page_vecs;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < page_vecs; v += gridDim.x * blockDim.x)
        to[v] = from[v];
}

constexpr int kMoveSmem = 48 * 1024;

// A page as sections: token (head h, slot j) of section i is the row of
// row[i] words at base[i] + h * head[i] + j * row[i].  f32 / bf16 pools: K
// rows then V rows, each [nkv][16][row] (16-byte words).  Quantised pools:
// nkv head blocks of K codes, V codes, scales (4-byte words, as the 8-byte
// scale rows need).
struct PageSections {
    int n;          // sections
    int row[4];     // words per (head, slot) row
    int base[4];    // section start in a page (head 0), in words
    int head[4];    // words between heads
    int tok_words;  // words of one token: nkv * sum(row)
    int page_words;
};

PageSections page_sections(const kv_pool* pool, int word_bytes) {
    PageSections ps{};
    const int nkv = pool->cfg.n_kv_heads;
    if (is_quant(pool->cfg.dtype)) {
        const int bytes[3] = {kHeadDim, quant_vrow(pool->cfg.dtype), 8};
        const int block = kPageTokens * (bytes[0] + bytes[1] + bytes[2]) / word_bytes;
        ps.n = 3;
        int at = 0;
        for (int i = 0; i < 3; ++i) {
            ps.row[i] = bytes[i] / word_bytes;
            ps.base[i] = at;
            ps.head[i] = block;
            at += kPageTokens * ps.row[i];
            ps.tok_words += nkv * ps.row[i];
        }
        ps.page_words = nkv * block;
    } else {
        const int r = kHeadDim * static_cast<int>(pool->elem_bytes) / word_bytes;
        ps.n = 2;
        for (int i = 0; i < 2; ++i) {
            ps.row[i] = r;
            ps.base[i] = i * nkv * kPageTokens * r;
            ps.head[i] = kPageTokens * r;
            ps.tok_words += nkv * r;
        }
        ps.page_words = 2 * nkv * kPageTokens * r;
    }
    return ps;
}

// One CTA per group of moves.  A token is its rows of every section, one row
// per (section, head).
template <typename Word>
__global__ void __launch_bounds__(256) move_tokens_kernel(Word* __restrict__ pages, const kv_token_move* moves,
                                                          const int32_t* group_off, int n_moves, int nkv,
                                                          const PageSections ps, uint32_t n_pages, int* err) {
    extern __shared__ uint4 buf_raw[];
    Word* buf = reinterpret_cast<Word*>(buf_raw);
    const int beg = __ldg(group_off + blockIdx.x), end = __ldg(group_off + blockIdx.x + 1);
    if (beg < 0 || end > n_moves || beg > end) {  // offsets outside the move array
        if (threadIdx.x == 0) flag_error(err, kDevErrBadPage);
        return;
    }
    const int tok_words = ps.tok_words;
    const int chunk = kMoveSmem / (tok_words * static_cast<int>(sizeof(Word)));
    // word v of the token in (page, slot), or nullptr if out of range.
    auto addr = [&](uint32_t page, int slot, int v) -> Word* {
        if (page >= n_pages || slot < 0 || slot >= kPageTokens) return nullptr;
        int sec = 0;
        while (sec + 1 < ps.n && v >= nkv * ps.row[sec]) v -= nkv * ps.row[sec++];
        const int head = v / ps.row[sec];
        return pages + static_cast<size_t>(page) * ps.page_words + ps.base[sec] +
               static_cast<size_t>(head) * ps.head[sec] + static_cast<size_t>(slot) * ps.row[sec] + v % ps.row[sec];
    };
    for (int c0 = beg; c0 < end; c0 += chunk) {
        const int cn = min(chunk, end - c0);
        for (int e = threadIdx.x; e < cn * tok_words; e += blockDim.x) {
            const kv_token_move m = moves[c0 + e / tok_words];
            const Word* p = addr(m.src_page, m.src_slot, e % tok_words);
            if (p) buf[e] = *p;
            else flag_error(err, kDevErrBadPage);
        }
        __syncthreads();
        for (int e = threadIdx.x; e < cn * tok_words; e += blockDim.x) {
            const kv_token_move m = moves[c0 + e / tok_words];
            Word* p = addr(m.dst_page, m.dst_slot, e % tok_words);
            if (p) *p = buf[e];
            else flag_error(err, kDevErrBadPage);
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace kvb200

extern "C" {

int kv_copy_pages(kv_pool* pool, const uint32_t* src, const uint32_t* dst, int32_t n, void* stream) {
    using namespace kvb200;
    if (!pool || n < 0) return KV_ERR_INVALID;
    if (n == 0) return KV_OK;
    if (!src || !dst) return KV_ERR_INVALID;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != pool->cfg.device) cudaSetDevice(pool->cfg.device);
    const int page_vecs = static_cast<int>(pool->page_bytes / 16);
    const unsigned gx = static_cast<unsigned>(std::min(8, (page_vecs + 255) / 256));
    constexpr int kMaxGridY = 65535;  // one launch per 65535 copies (grid.y limit)
    cudaError_t e = cudaSuccess;
    for (int32_t off = 0; off < n && e == cudaSuccess; off += kMaxGridY) {
        const int m = std::min<int32_t>(kMaxGridY, n - off);
        copy_pages_kernel<<<dim3(gx, m), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<uint4*>(pool->pages), src + off, dst + off, m, pool->cfg.n_pages, page_vecs,
            pool->dev_error);
        e = cudaGetLastError();
    }
    if (prev >= 0 && prev != pool->cfg.device) cudaSetDevice(prev);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

int kv_move_tokens(kv_pool* pool, const kv_token_move* moves, int32_t n_moves, const int32_t* group_offsets,
                   int32_t n_groups, void* stream) {
    using namespace kvb200;
    if (!pool || n_groups < 0 || n_moves < 0) return KV_ERR_INVALID;
    if (n_groups == 0 || n_moves == 0) return KV_OK;
    if (!moves || !group_offsets) return KV_ERR_INVALID;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != pool->cfg.device) cudaSetDevice(pool->cfg.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (is_quant(pool->cfg.dtype))
        move_tokens_kernel<uint32_t><<<n_groups, 256, kMoveSmem, st>>>(
            static_cast<uint32_t*>(pool->pages), moves, group_offsets, n_moves, pool->cfg.n_kv_heads,
            page_sections(pool, 4), pool->cfg.n_pages, pool->dev_error);
    else
        move_tokens_kernel<uint4><<<n_groups, 256, kMoveSmem, st>>>(
            static_cast<uint4*>(pool->pages), moves, group_offsets, n_moves, pool->cfg.n_kv_heads,
            page_sections(pool, 16), pool->cfg.n_pages, pool->dev_error);
    const cudaError_t e = cudaGetLastError();
    if (prev >= 0 && prev != pool->cfg.device) cudaSetDevice(prev);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // extern "C"
