// kv_append.cu -- K/V append into pages with RoPE on k, for sm_100a.
//
// Replaces the decode append (crates/llm-engine/src/lfm2.rs:828-832), the
// prefill K/V store (lfm2.rs:751-761) and the k-side RoPE before them
// (lfm2.rs:816-825 -> crates/llm-cpu/src/rope.rs:56-81).  The rotation is the
// reference's: for d < 32, k'[d] = k[d]*cos - k[d+32]*sin; for d >= 32,
// k'[d] = k[d]*cos + k[d-32]*sin, each as two rounded products and a rounded
// sum (Rust does not contract to FMA).  cos/sin come from the pool's table,
// computed with the same libm calls as rope.rs:30-41, so the stored K is
// bit-identical to the CPU path's (after bf16 rounding to nearest even).
//
// Thread mapping: 4 threads per (token, kv head); thread qd owns dims
// [8qd, 8qd+8) and their rotation partners [8qd+32, 8qd+40), so the four
// threads of a head write its 128-byte (bf16) row as 16-byte stores.
#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace kvb200 {
namespace {

struct AppendArgs {
    const void* k;
    const void* v;
    const int32_t* tok_seq;   // null: decode mode (token i = sequence i)
    const int32_t* tok_slot;
    const int32_t* tok_pos;
    const int32_t* seq_lens;  // decode mode: slot = pos = seq_lens[i] - 1
    int n_tokens;
    int n_seqs;  // rows of the block table
    int nkv;
    const uint32_t* bt;
    long long bt_stride;
    uint32_t n_pages;
    const float2* rope;
    int max_pos;
    int* err;
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = bf16x2_to_float2(w[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&x)[8]) {
    uint4 u;
    u.x = float2_to_bf16x2(x[0], x[1]);
    u.y = float2_to_bf16x2(x[2], x[3]);
    u.z = float2_to_bf16x2(x[4], x[5]);
    u.w = float2_to_bf16x2(x[6], x[7]);
    *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void store8(float* p, const float (&x)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

// V is copied as stored bits (no widening round trip).
__device__ __forceinline__ void copy8(__nv_bfloat16* dst, const __nv_bfloat16* src) {
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
}
__device__ __forceinline__ void copy8(float* dst, const float* src) {
    reinterpret_cast<float4*>(dst)[0] = __ldg(reinterpret_cast<const float4*>(src));
    reinterpret_cast<float4*>(dst)[1] = __ldg(reinterpret_cast<const float4*>(src) + 1);
}

template <typename T>
__global__ void __launch_bounds__(256) append_kernel(T* __restrict__ pages, const AppendArgs a) {
    const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per_tok = a.nkv * 4;
    const long long tok = gtid / per_tok;
    if (tok >= a.n_tokens) return;
    const int r = static_cast<int>(gtid % per_tok);
    const int h = r >> 2, qd = r & 3;
    int s, slot, pos;
    if (a.tok_seq) {
        s = __ldg(a.tok_seq + tok);
        slot = __ldg(a.tok_slot + tok);
        pos = __ldg(a.tok_pos + tok);
    } else {
        s = static_cast<int>(tok);
        slot = __ldg(a.seq_lens + tok) - 1;
        pos = slot;
        if (slot < 0) return;  // empty sequence: nothing to append
    }
    if (pos < 0 || pos >= a.max_pos) {
        if (r == 0) flag_error(a.err, kDevErrBadPos);
        return;
    }
    if (s < 0 || s >= a.n_seqs || slot < 0 || slot / kPageTokens >= a.bt_stride) {
        if (r == 0) flag_error(a.err, kDevErrBadPage);
        return;
    }
    const uint32_t page = __ldg(a.bt + static_cast<size_t>(s) * a.bt_stride + slot / kPageTokens);
    if (page >= a.n_pages) {
        if (r == 0) flag_error(a.err, kDevErrBadPage);
        return;
    }
    const int j = slot % kPageTokens;
    const size_t page_elems = static_cast<size_t>(2) * a.nkv * kPageTokens * kHeadDim;
    T* kdst = pages + page * page_elems + (static_cast<size_t>(h) * kPageTokens + j) * kHeadDim;
    T* vdst = pages + page * page_elems +
              (static_cast<size_t>(a.nkv + h) * kPageTokens + j) * kHeadDim;
    const T* ksrc = static_cast<const T*>(a.k) + (tok * a.nkv + h) * kHeadDim;
    const T* vsrc = static_cast<const T*>(a.v) + (tok * a.nkv + h) * kHeadDim;

    float x[8], y[8], xo[8], yo[8];
    load8(ksrc + 8 * qd, x);
    load8(ksrc + 8 * qd + 32, y);
    const float2* cs = a.rope + static_cast<size_t>(pos) * (kHeadDim / 2) + 8 * qd;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float2 c = __ldg(cs + e);
        xo[e] = __fadd_rn(__fmul_rn(x[e], c.x), __fmul_rn(-y[e], c.y));
        yo[e] = __fadd_rn(__fmul_rn(y[e], c.x), __fmul_rn(x[e], c.y));
    }
    store8(kdst + 8 * qd, xo);
    store8(kdst + 8 * qd + 32, yo);
    copy8(vdst + 8 * qd, vsrc + 8 * qd);
    copy8(vdst + 8 * qd + 32, vsrc + 8 * qd + 32);
}

}  // namespace

int launch_append(kv_pool* pool, const void* k, const void* v, const int32_t* tok_seq,
                  const int32_t* tok_slot, const int32_t* tok_pos, const int32_t* seq_lens,
                  int32_t n_tokens, int32_t n_seqs, const uint32_t* bt, int32_t bt_stride,
                  cudaStream_t stream) {
    AppendArgs a;
    a.k = k;
    a.v = v;
    a.tok_seq = tok_seq;
    a.tok_slot = tok_slot;
    a.tok_pos = tok_pos;
    a.seq_lens = seq_lens;
    a.n_tokens = n_tokens;
    a.n_seqs = n_seqs;
    a.nkv = pool->cfg.n_kv_heads;
    a.bt = bt;
    a.bt_stride = bt_stride;
    a.n_pages = pool->cfg.n_pages;
    a.rope = pool->rope;
    a.max_pos = pool->cfg.max_positions;
    a.err = pool->dev_error;
    const long long threads = static_cast<long long>(n_tokens) * a.nkv * 4;
    const int block = 256;
    const unsigned grid = static_cast<unsigned>((threads + block - 1) / block);
    if (pool->cfg.dtype == KV_DTYPE_BF16)
        append_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(
            static_cast<__nv_bfloat16*>(pool->pages), a);
    else
        append_kernel<float><<<grid, block, 0, stream>>>(static_cast<float*>(pool->pages), a);
    return cudaGetLastError() == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
