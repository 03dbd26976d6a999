// kv_pool.cu -- pool lifetime and the C ABI entry points (include/llmhost_kv.h).
//
// A pool is what a `crates/llm-cuda` Backend (crates/llm-core/src/backend.rs:4-13)
// would own: the physical pages of every attention layer's paged KV, the RoPE
// cos/sin table, and the attention workspace.  Nothing is allocated after
// kv_pool_create; the hot entry points only validate arguments and launch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace {

// Runs the enclosing scope on `dev`, restoring the caller's device after.
struct DeviceScope {
    int prev = -1;
    bool ok = false;
    explicit DeviceScope(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) return;
        ok = (prev == dev) || cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceScope() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// k, v and q rows are read as 16-byte vectors (appends, the decode kernels' staging).
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_config(const kv_pool_config& c) {
    if (c.dtype != KV_DTYPE_F32 && c.dtype != KV_DTYPE_BF16 && c.dtype != KV_DTYPE_Q8 && c.dtype != KV_DTYPE_K8V4 &&
        c.dtype != KV_DTYPE_F16)
        return false;
    if (c.head_dim != kvb200::kHeadDim || c.page_tokens != kvb200::kPageTokens) return false;
    if (c.n_kv_heads != 1 && c.n_kv_heads != 2 && c.n_kv_heads != 4 && c.n_kv_heads != 8) return false;
    if (c.n_q_heads <= 0 || c.n_q_heads % c.n_kv_heads != 0) return false;
    if (c.n_pages == 0 || c.max_positions <= 0 || c.max_seqs <= 0 || c.max_seqs > 65536) return false;
    if (!(c.rope_theta > 0.f) || c.device < 0) return false;
    return true;
}

// RoPE table [max_pos][d/2] of (cos, sin): rope.rs:6-14 (inv_freq, fp32 powf)
// and rope.rs:30-41 (pos as f32, freq = pos * inv_freq[i], libm cosf/sinf).
void build_rope_table(int max_pos, int dim, float theta, std::vector<float2>& out) {
    const int half = dim / 2;
    std::vector<float> inv(half);
    const float dim_f = static_cast<float>(dim);
    for (int i = 0; i < dim; i += 2) {
        const float expo = static_cast<float>(i) / dim_f;
        inv[i / 2] = 1.0f / powf(theta, expo);
    }
    out.resize(static_cast<size_t>(max_pos) * half);
    const unsigned hw = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    const int chunk = (max_pos + static_cast<int>(hw) - 1) / static_cast<int>(hw);
    std::vector<std::thread> th;
    for (unsigned w = 0; w < hw; ++w) {
        const int b = static_cast<int>(w) * chunk, e = std::min(max_pos, b + chunk);
        if (b >= e) break;
        th.emplace_back([&, b, e] {
            for (int p = b; p < e; ++p) {
                const float pos = static_cast<float>(p);
                for (int i = 0; i < half; ++i) {
                    const float freq = pos * inv[i];
                    out[static_cast<size_t>(p) * half + i] = make_float2(cosf(freq), sinf(freq));
                }
            }
        });
    }
    for (auto& t : th) t.join();
}

// The pool as 128-byte rows (2D), 128-byte swizzle, boxes of box_rows rows.
int encode_row_map(kv_pool* p, CUtensorMap* map, cuuint32_t box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode),
                                cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !encode)
        return KV_ERR_CUDA;
    const int elem = static_cast<int>(p->elem_bytes);
    const cuuint64_t row_elems = 128 / elem;
    const cuuint64_t page_rows = p->page_bytes / 128;
    const cuuint64_t gdim[2] = {row_elems, static_cast<cuuint64_t>(p->cfg.n_pages) * page_rows};
    const cuuint64_t gstride[1] = {128};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(row_elems), box_rows};
    const cuuint32_t estride[2] = {1, 1};
    const CUtensorMapDataType dt = p->cfg.dtype == KV_DTYPE_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : p->cfg.dtype == KV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const CUresult r = encode(map, dt, 2, p->pages, gdim, gstride, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? KV_OK : KV_ERR_CUDA;
}

// page_map: a whole page per box (up to 256 rows; decode).  head_map: one
// head's page_tokens rows of K or V per box (prefill).
int encode_page_map(kv_pool* p) {
    const cuuint64_t page_rows = p->page_bytes / 128;
    const int rc = encode_row_map(p, &p->page_map, static_cast<cuuint32_t>(std::min<cuuint64_t>(256, page_rows)));
    if (rc != KV_OK) return rc;
    return encode_row_map(p, &p->head_map, static_cast<cuuint32_t>(p->cfg.page_tokens * p->elem_bytes / 2));
}

void free_pool(kv_pool* p) {
    if (!p) return;
    cudaFree(p->pages);
    cudaFree(p->rope);
    cudaFree(p->dev_error);
    cudaFree(p->part_o);
    cudaFree(p->part_ml);
    cudaFree(p->counters);
    cudaFree(p->pre_part);
    cudaFree(p->pre_counters);
    delete p;
}

int alloc_dev(void** ptr, size_t bytes) {
    const cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        return KV_ERR_OOM;
    }
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace

extern "C" {

const char* kv_status_str(int status) {
    switch (status) {
        case KV_OK: return "ok";
        case KV_ERR_INVALID: return "invalid argument";
        case KV_ERR_BAD_PAGE: return "page id out of range or not allocated";
        case KV_ERR_OOM: return "out of pages or device memory";
        case KV_ERR_TIMEOUT: return "device-side wait timed out";
        case KV_ERR_CUDA: return "CUDA error";
        case KV_ERR_UNSUPPORTED: return "shape not supported by this build";
        case KV_ERR_BAD_POS: return "RoPE position out of range";
        case KV_ERR_UNKNOWN_SEQ: return "unknown sequence";
        case KV_ERR_NO_PENDING: return "sequence has no pending forward to accept or roll back";
        case KV_ERR_INVALID_ACCEPT: return "accepted tokens are not a valid path";
        case KV_ERR_TREE: return "invalid parent-index tree";
        default: return "unknown status";
    }
}

int kv_api_version(void) { return KV_API_VERSION; }

int kv_pool_create(const kv_pool_config* cfg, kv_pool** out) {
    if (!cfg || !out) return KV_ERR_INVALID;
    *out = nullptr;
    if (!valid_config(*cfg)) return KV_ERR_INVALID;
    DeviceScope dev(cfg->device);
    if (!dev.ok) return KV_ERR_CUDA;
    kv_pool* p = new (std::nothrow) kv_pool();
    if (!p) return KV_ERR_OOM;
    p->cfg = *cfg;
    p->elem_bytes = cfg->dtype == KV_DTYPE_F32 ? 4 : 2;  // f16 and quantised pools take bf16 k, v, q, out
    p->page_bytes = kvb200::is_quant(cfg->dtype)
                        ? kvb200::quant_page_bytes(cfg->dtype, cfg->n_kv_heads)
                        : 2ull * cfg->n_kv_heads * cfg->page_tokens * cfg->head_dim * p->elem_bytes;
    if (static_cast<uint64_t>(cfg->n_pages) * (p->page_bytes / 128) >= (1ull << 31)) {
        delete p;
        return KV_ERR_INVALID;  // TMA row coordinates are int32
    }
    int rc = KV_OK;
    if (cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, cfg->device) !=
        cudaSuccess) {
        delete p;
        return KV_ERR_CUDA;
    }
    rc = kvb200::decode_setup(p);
    if (rc == KV_OK) rc = kvb200::prefill_setup(p);
    if (rc != KV_OK) {
        delete p;
        return rc;
    }
    const size_t pool_bytes = static_cast<size_t>(cfg->n_pages) * p->page_bytes;
    const size_t slots = kvb200::decode_workspace_slots(p);
    const size_t rope_elems = static_cast<size_t>(cfg->max_positions) * (cfg->head_dim / 2);
    if ((rc = alloc_dev(&p->pages, pool_bytes)) ||
        (rc = alloc_dev(reinterpret_cast<void**>(&p->rope), rope_elems * sizeof(float2))) ||
        (rc = alloc_dev(reinterpret_cast<void**>(&p->dev_error), sizeof(kvb200::DeviceWs))) ||
        (rc = alloc_dev(reinterpret_cast<void**>(&p->part_o),
                        slots * cfg->n_q_heads * cfg->head_dim * sizeof(float))) ||
        (rc = alloc_dev(reinterpret_cast<void**>(&p->part_ml), slots * cfg->n_q_heads * 2 * sizeof(float))) ||
        (rc = alloc_dev(reinterpret_cast<void**>(&p->counters), kvb200::decode_counter_count(p) * sizeof(int)))) {
        free_pool(p);
        return rc;
    }
    const size_t pre_bytes = kvb200::prefill_workspace_bytes(p);
    const size_t pre_counters = kvb200::prefill_counter_count(p);
    if (pre_bytes &&
        ((rc = alloc_dev(reinterpret_cast<void**>(&p->pre_part), pre_bytes)) ||
         (rc = alloc_dev(reinterpret_cast<void**>(&p->pre_counters), pre_counters * sizeof(int))))) {
        free_pool(p);
        return rc;
    }
    if (pre_counters && cudaMemset(p->pre_counters, 0, pre_counters * sizeof(int)) != cudaSuccess) {
        free_pool(p);
        return KV_ERR_CUDA;
    }
    std::vector<float2> table;
    build_rope_table(cfg->max_positions, cfg->head_dim, cfg->rope_theta, table);
    if (cudaMemset(p->pages, 0, pool_bytes) != cudaSuccess ||
        cudaMemset(p->dev_error, 0, sizeof(kvb200::DeviceWs)) != cudaSuccess ||
        cudaMemset(p->counters, 0, kvb200::decode_counter_count(p) * sizeof(int)) != cudaSuccess ||
        cudaMemcpy(p->rope, table.data(), rope_elems * sizeof(float2), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        free_pool(p);
        return KV_ERR_CUDA;
    }
    if (!kvb200::is_quant(cfg->dtype) && (rc = encode_page_map(p)) != KV_OK) {
        free_pool(p);
        return rc;
    }
    *out = p;
    return KV_OK;
}

int kv_pool_destroy(kv_pool* pool) {
    if (!pool) return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    cudaDeviceSynchronize();
    free_pool(pool);
    return KV_OK;
}

void* kv_pool_pages(const kv_pool* pool) { return pool ? pool->pages : nullptr; }

size_t kv_pool_page_bytes(const kv_pool* pool) { return pool ? pool->page_bytes : 0; }

static int copy_pages(kv_pool* pool, const uint32_t* ids, int32_t n, void* host, bool to_host) {
    if (!pool || n < 0 || (n > 0 && (!ids || !host))) return KV_ERR_INVALID;
    for (int32_t i = 0; i < n; ++i)
        if (ids[i] >= pool->cfg.n_pages) return KV_ERR_BAD_PAGE;
    DeviceScope dev(pool->cfg.device);
    const size_t pb = pool->page_bytes;
    char* dev_base = static_cast<char*>(pool->pages);
    char* h = static_cast<char*>(host);
    for (int32_t i = 0; i < n;) {  // one copy per run of consecutive page ids
        int32_t j = i + 1;
        while (j < n && ids[j] == ids[j - 1] + 1) ++j;
        const size_t bytes = static_cast<size_t>(j - i) * pb;
        char* d = dev_base + static_cast<size_t>(ids[i]) * pb;
        const cudaError_t e = to_host ? cudaMemcpy(h + i * pb, d, bytes, cudaMemcpyDeviceToHost)
                                      : cudaMemcpy(d, h + i * pb, bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return KV_ERR_CUDA;
        i = j;
    }
    return KV_OK;
}

int kv_pool_read_pages(kv_pool* pool, const uint32_t* page_ids, int32_t n, void* host_dst) {
    return copy_pages(pool, page_ids, n, host_dst, true);
}

int kv_pool_write_pages(kv_pool* pool, const uint32_t* page_ids, int32_t n, const void* host_src) {
    return copy_pages(pool, page_ids, n, const_cast<void*>(host_src), false);
}

int kv_last_error(kv_pool* pool) {
    if (!pool) return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    if (cudaDeviceSynchronize() != cudaSuccess) return KV_ERR_CUDA;
    int word = 0;
    if (cudaMemcpy(&word, pool->dev_error, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return KV_ERR_CUDA;
    if (word == 0) return KV_OK;
    cudaMemset(pool->dev_error, 0, sizeof(int));
    // A wait that gave up may have left a split counter half counted.
    cudaMemset(pool->counters, 0, kvb200::decode_counter_count(pool) * sizeof(int));
    cudaDeviceSynchronize();
    if (word & kvb200::kDevErrTimeout) return KV_ERR_TIMEOUT;
    if (word & kvb200::kDevErrBadPage) return KV_ERR_BAD_PAGE;
    if (word & kvb200::kDevErrBadPos) return KV_ERR_BAD_POS;
    if (word & kvb200::kDevErrBadArg) return KV_ERR_INVALID;
    return KV_ERR_CUDA;
}

int kv_append(kv_pool* pool, const void* k, const void* v, const int32_t* tok_seq,
              const int32_t* tok_slot, const int32_t* tok_pos, int32_t n_tokens,
              const uint32_t* block_tables, int32_t n_seqs, int32_t bt_stride, void* stream) {
    if (!pool || n_tokens < 0 || n_seqs < 0) return KV_ERR_INVALID;
    if (n_tokens == 0) return KV_OK;
    if (!k || !v || !tok_seq || !tok_slot || !tok_pos || !block_tables || bt_stride <= 0 ||
        n_seqs == 0 || !aligned16(k) || !aligned16(v))
        return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_append(pool, k, v, tok_seq, tok_slot, tok_pos, nullptr, n_tokens, n_seqs,
                                 block_tables, bt_stride, static_cast<cudaStream_t>(stream));
}

int kv_append_decode(kv_pool* pool, const void* k, const void* v, const uint32_t* block_tables,
                     int32_t bt_stride, const int32_t* seq_lens, int32_t n_seqs, void* stream) {
    if (!pool || n_seqs < 0) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (!k || !v || !block_tables || !seq_lens || bt_stride <= 0 || !aligned16(k) || !aligned16(v))
        return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_append(pool, k, v, nullptr, nullptr, nullptr, seq_lens, n_seqs, n_seqs,
                                 block_tables, bt_stride, static_cast<cudaStream_t>(stream));
}

int kv_decode_attn(kv_pool* pool, const void* q, const uint32_t* block_tables, int32_t bt_stride,
                   const int32_t* seq_lens, int32_t n_seqs, int32_t window, void* out,
                   void* stream) {
    if (!pool || n_seqs < 0 || window < 0) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (n_seqs > pool->cfg.max_seqs) return KV_ERR_INVALID;
    if (!q || !block_tables || !seq_lens || !out || bt_stride <= 0 || !aligned16(q)) return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_decode(pool, q, block_tables, bt_stride, seq_lens, n_seqs, window, out,
                                 static_cast<cudaStream_t>(stream));
}

int kv_append_decode_attn(kv_pool* pool, const void* k, const void* v, const void* q,
                          const uint32_t* block_tables, int32_t bt_stride, const int32_t* seq_lens,
                          int32_t n_seqs, int32_t window, void* out, void* stream) {
    if (!pool || n_seqs < 0 || window < 0) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (n_seqs > pool->cfg.max_seqs) return KV_ERR_INVALID;
    if (!k || !v || !q || !block_tables || !seq_lens || !out || bt_stride <= 0 || !aligned16(k) ||
        !aligned16(v) || !aligned16(q))
        return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_decode(pool, q, block_tables, bt_stride, seq_lens, n_seqs, window, out,
                                 static_cast<cudaStream_t>(stream), k, v);
}

int kv_norm_append_decode_attn(kv_pool* pool, const void* k, const void* v, const void* q, const float* q_norm,
                               const float* k_norm, float eps, const uint32_t* block_tables, int32_t bt_stride,
                               const int32_t* seq_lens, int32_t n_seqs, int32_t window, void* out, void* stream) {
    if (!pool || n_seqs < 0 || window < 0 || !(eps >= 0.f)) return KV_ERR_INVALID;
    if (n_seqs == 0) return KV_OK;
    if (n_seqs > pool->cfg.max_seqs) return KV_ERR_INVALID;
    if (!k || !v || !q || !q_norm || !k_norm || !block_tables || !seq_lens || !out || bt_stride <= 0 ||
        !aligned16(k) || !aligned16(v) || !aligned16(q) || !aligned16(q_norm) || !aligned16(k_norm))
        return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_decode(pool, q, block_tables, bt_stride, seq_lens, n_seqs, window, out,
                                 static_cast<cudaStream_t>(stream), k, v, q_norm, k_norm, eps);
}

int kv_prefill_attn(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_offsets,
                    const int32_t* prefix_lens, const uint64_t* tree_masks, const uint32_t* block_tables,
                    int32_t bt_stride, int32_t n_seqs, int32_t max_q_per_seq, void* out, void* stream) {
    if (!pool || n_seqs < 0 || max_q_per_seq < 0) return KV_ERR_INVALID;
    if (n_seqs == 0 || max_q_per_seq == 0) return KV_OK;
    if (!q || !q_pos || !q_offsets || !prefix_lens || !block_tables || !out || bt_stride <= 0 ||
        n_seqs > 65535 || (tree_masks && max_q_per_seq > 64))
        return KV_ERR_INVALID;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_prefill(pool, q, q_pos, q_offsets, prefix_lens,
                                  reinterpret_cast<const unsigned long long*>(tree_masks), n_seqs,
                                  max_q_per_seq, block_tables, bt_stride, out, static_cast<cudaStream_t>(stream));
}

size_t kv_prefill_shared_workspace_bytes(const kv_pool* pool, int32_t n_seqs, int32_t max_q_per_seq) {
    if (!pool || n_seqs <= 0 || max_q_per_seq <= 0) return 0;
    return kvb200::prefill_shared_workspace_bytes(pool, n_seqs, max_q_per_seq);
}

int kv_prefill_attn_shared(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_offsets,
                           const int32_t* prefix_lens, const uint64_t* tree_masks, const uint32_t* block_tables,
                           int32_t bt_stride, int32_t n_seqs, int32_t max_q_per_seq, int32_t shared_tokens,
                           void* workspace, void* out, void* stream) {
    if (!pool || n_seqs < 0 || max_q_per_seq < 0) return KV_ERR_INVALID;
    if (n_seqs == 0 || max_q_per_seq == 0) return KV_OK;
    if (!q || !q_pos || !q_offsets || !prefix_lens || !block_tables || !out || !workspace || bt_stride <= 0 ||
        n_seqs > 65535 || (tree_masks && max_q_per_seq > 64) || !aligned16(workspace))
        return KV_ERR_INVALID;
    if (shared_tokens <= 0 || shared_tokens % kvb200::kPageTokens != 0 ||
        shared_tokens / kvb200::kPageTokens > bt_stride)
        return KV_ERR_INVALID;
    if (pool->cfg.dtype != KV_DTYPE_BF16) return KV_ERR_UNSUPPORTED;
    DeviceScope dev(pool->cfg.device);
    return kvb200::launch_prefill_shared(pool, q, q_pos, q_offsets, prefix_lens,
                                         reinterpret_cast<const unsigned long long*>(tree_masks), n_seqs,
                                         max_q_per_seq, block_tables, bt_stride, shared_tokens, workspace, out,
                                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
