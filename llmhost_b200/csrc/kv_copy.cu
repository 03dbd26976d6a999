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
//                  an earlier move wrote).  Groups run in parallel.
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

// One CTA per group of moves.  A token's K/V is 2 * nkv rows of row_vecs
// 16-byte chunks (K rows of every head, then V rows), one row per head.
__global__ void __launch_bounds__(256) move_tokens_kernel(uint4* __restrict__ pages, const kv_token_move* moves,
                                                          const int32_t* group_off, int n_moves, int nkv,
                                                          int row_vecs, uint32_t n_pages, int* err) {
    extern __shared__ uint4 buf[];
    const int beg = __ldg(group_off + blockIdx.x), end = __ldg(group_off + blockIdx.x + 1);
    if (beg < 0 || end > n_moves || beg > end) {  // offsets outside the move array
        if (threadIdx.x == 0) flag_error(err, kDevErrBadPage);
        return;
    }
    const int tok_vecs = 2 * nkv * row_vecs;
    const int page_vecs = tok_vecs * kPageTokens;
    const int chunk = kMoveSmem / (tok_vecs * 16);
    // 16-byte chunk v of the token in (page, slot), or nullptr if out of range.
    auto addr = [&](uint32_t page, int slot, int v) -> uint4* {
        if (page >= n_pages || slot < 0 || slot >= kPageTokens) return nullptr;
        const int row = v / row_vecs;  // K heads, then V heads
        return pages + static_cast<size_t>(page) * page_vecs +
               (static_cast<size_t>(row) * kPageTokens + slot) * row_vecs + v % row_vecs;
    };
    for (int c0 = beg; c0 < end; c0 += chunk) {
        const int cn = min(chunk, end - c0);
        for (int e = threadIdx.x; e < cn * tok_vecs; e += blockDim.x) {
            const kv_token_move m = moves[c0 + e / tok_vecs];
            const uint4* p = addr(m.src_page, m.src_slot, e % tok_vecs);
            if (p) buf[e] = *p;
            else flag_error(err, kDevErrBadPage);
        }
        __syncthreads();
        for (int e = threadIdx.x; e < cn * tok_vecs; e += blockDim.x) {
            const kv_token_move m = moves[c0 + e / tok_vecs];
            uint4* p = addr(m.dst_page, m.dst_slot, e % tok_vecs);
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
    const int row_vecs = kHeadDim * static_cast<int>(pool->elem_bytes) / 16;
    move_tokens_kernel<<<n_groups, 256, kMoveSmem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint4*>(pool->pages), moves, group_offsets, n_moves, pool->cfg.n_kv_heads, row_vecs,
        pool->cfg.n_pages, pool->dev_error);
    const cudaError_t e = cudaGetLastError();
    if (prev >= 0 && prev != pool->cfg.device) cudaSetDevice(prev);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // extern "C"
