// kv_pool_impl.h -- the pool object behind the opaque `kv_pool` handle.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/llmhost_kv.h"

struct kv_pool {
    kv_pool_config cfg;
    int sm_count = 0;
    size_t page_bytes = 0;
    size_t elem_bytes = 0;
    void* pages = nullptr;        // n_pages * page_bytes, device
    float2* rope = nullptr;       // [max_positions][head_dim / 2] (cos, sin), device
    int* dev_error = nullptr;     // device error word
    // decode split workspace
    float* part_o = nullptr;      // [decode_workspace_slots][n_q][head_dim]
    float* part_ml = nullptr;     // [decode_workspace_slots][n_q][2]
    int* counters = nullptr;      // [decode_counter_count]: per sequence, then per CTA run
    int decode_grid = 0;
    size_t decode_smem = 0;
    // prefill split workspace (bf16 pools): partial rows of the units that the
    // persistent prefill schedule cuts between CTAs, and one merge counter per unit
    float* pre_part = nullptr;    // [prefill_workspace_slots][256 rows][head_dim + 2]
    int* pre_counters = nullptr;  // [prefill_counter_count]
    CUtensorMap page_map;         // TMA view of the pool as 128-byte rows
    CUtensorMap head_map;         // same rows, one head's page_tokens rows per box (bf16)
};

namespace kvb200 {

// Quantised pools (KV_DTYPE_Q8, KV_DTYPE_K8V4): per (head, token) 64 K code
// bytes, 64 (Q8) or 32 (K8V4) V code bytes and two f16 scales each for K and
// V.  A page is n_kv head blocks: K codes [16][64], V codes [16][vrow],
// scales [16 tokens][2 blocks][K, V].
inline bool is_quant(int dtype) { return dtype == KV_DTYPE_Q8 || dtype == KV_DTYPE_K8V4; }
// 16-bit float pages (bf16 or IEEE half) in the bf16 page layout.
inline bool is_half_page(int dtype) { return dtype == KV_DTYPE_BF16 || dtype == KV_DTYPE_F16; }
inline int quant_vrow(int dtype) { return dtype == KV_DTYPE_Q8 ? 64 : 32; }
inline size_t quant_head_block(int dtype) { return static_cast<size_t>(16) * (64 + quant_vrow(dtype) + 8); }
inline size_t quant_page_bytes(int dtype, int nkv) { return static_cast<size_t>(nkv) * quant_head_block(dtype); }

// Launchers implemented in the .cu files; they return a kv_status.
int launch_append(kv_pool* pool, const void* k, const void* v, const int32_t* tok_seq,
                  const int32_t* tok_slot, const int32_t* tok_pos, const int32_t* seq_lens,
                  int32_t n_tokens, int32_t n_seqs, const uint32_t* bt, int32_t bt_stride,
                  cudaStream_t stream, const float* k_norm = nullptr, float eps = 0.f);

// Raises a kernel's dynamic shared-memory limit on `device` to at least
// `bytes` (never lowers it: the attribute is shared by every pool).
int raise_smem_limit(const void* fn, int device, size_t bytes);

// Sets up the decode kernel for the pool (smem attribute, grid); called once
// at pool creation.  Returns KV_ERR_UNSUPPORTED for shapes not compiled.
int decode_setup(kv_pool* pool);
size_t decode_workspace_slots(const kv_pool* pool);
size_t decode_counter_count(const kv_pool* pool);
// new_k / new_v non-null: append each sequence's new token first (fused
// kv_append_decode; the last page of every sequence must be its own).
// q_norm / k_norm non-null: RMS-normalise each q head and the new k heads
// first (kv_norm_append_decode_attn).
int launch_decode(kv_pool* pool, const void* q, const uint32_t* bt, int32_t bt_stride,
                  const int32_t* seq_lens, int32_t n_seqs, int32_t window, void* out,
                  cudaStream_t stream, const void* new_k = nullptr, const void* new_v = nullptr,
                  const float* q_norm = nullptr, const float* k_norm = nullptr, float eps = 0.f);

// Decode attention on tcgen05 for bf16 and quantised pools (kv_decode_tc.cu);
// decode_setup and launch_decode route those pools here.
int decode_tc_setup(kv_pool* pool);
int launch_decode_tc(kv_pool* pool, const void* q, const uint32_t* bt, int32_t bt_stride, const int32_t* seq_lens,
                     int32_t n_seqs, int32_t window, void* out, cudaStream_t stream, const void* new_k,
                     const void* new_v, const float* q_norm, const float* k_norm, float eps);

// Prefill / tree-verify attention: tcgen05 for bf16 pools (kv_prefill.cu).
int prefill_setup(kv_pool* pool);
// Bytes of the prefill split workspace and of its counters (0 for fp32 pools).
size_t prefill_workspace_bytes(const kv_pool* pool);
size_t prefill_counter_count(const kv_pool* pool);
int launch_prefill(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                   const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                   const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream);
// Shared-prefix form (bf16 pools): every token against the first `shared`
// keys (table row 0) into ws, then each sequence against the rest, merged.
size_t prefill_shared_workspace_bytes(const kv_pool* pool, int32_t n_seqs, int32_t max_q);
int launch_prefill_shared(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                          const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                          const uint32_t* bt, int32_t bt_stride, int32_t shared, void* ws, void* out,
                          cudaStream_t stream);
// fp32 and quantised pools: CUDA-core kernel (kv_prefill_f32.cu), same arguments.
int launch_prefill_f32(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                       const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                       const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream);

// Decode launch on explicit workspace pointers and an explicit tensor map,
// for the entry point that owns no pool (kv_noalloc.cu).
struct DecodeRaw {
    int dtype, nkv, group;
    const CUtensorMap* map;
    const void* q;
    void* out;
    const uint32_t* bt;
    long long bt_stride;
    const int32_t* seq_lens;
    int n_seqs;
    int window;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    float* part_o;
    float* part_ml;
    int* counters;
    int* err;
    int grid;
    size_t smem;
};
// Sets the kernel's shared-memory attribute on the current device and
// returns its persistent grid size; call once per device and shape.
int decode_configure_raw(int dtype, int nkv, int group, int max_seqs, int device, int sm_count,
                         int* grid, size_t* smem);
int launch_decode_raw(const DecodeRaw& r, cudaStream_t stream);

}  // namespace kvb200
