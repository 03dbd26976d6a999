// kv_append.cu -- K/V append into pages with RoPE on k, for sm_100a.
//
// Replaces the decode append (crates/llm-engine/src/lfm2.rs:828-832), the
// prefill K/V store (lfm2.rs:751-761) and the k-side RoPE before them
// (lfm2.rs:816-825 -> crates/llm-cpu/src/rope.rs:56-81).  The rotation is the
// reference's: for d < 32, k'[d] = k[d]*cos - k[d+32]*sin; for d >= 32,
// k'[d] = k[d]*cos + k[d-32]*sin, each as two rounded products and a rounded
// sum (Rust does not contract to FMA).  cos/sin come from the pool's table,
// computed with the same libm calls as rope.rs:30-41, so the stored K is
// bit-identical to the CPU path's (after bf16 or f16 rounding to nearest even).
//
// Thread mapping: 4 threads per (token, kv head); thread qd owns dims
// [8qd, 8qd+8) and their rotation partners [8qd+32, 8qd+40), so the four
// threads of a head write its 128-byte (bf16) row as 16-byte stores.
#include <cuda_fp16.h>

#include <type_traits>

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
    const float* k_norm;  // quantised pools: RMSNorm weights of k before RoPE (null: none)
    float eps;
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
__device__ __forceinline__ void store8(__half* p, const float (&x)[8]) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);  // low half: x[2i]
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(h);
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

// S: the page element (bf16, fp32, or IEEE half for KV_DTYPE_F16); I: the
// appended k / v element (S, or bf16 for half pages, whose V is then widened
// and rounded to half rather than copied).
template <typename S, typename I = S>
__global__ void __launch_bounds__(256) append_kernel(S* __restrict__ pages, const AppendArgs a) {
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
    S* kdst = pages + page * page_elems + (static_cast<size_t>(h) * kPageTokens + j) * kHeadDim;
    S* vdst = pages + page * page_elems +
              (static_cast<size_t>(a.nkv + h) * kPageTokens + j) * kHeadDim;
    const I* ksrc = static_cast<const I*>(a.k) + (tok * a.nkv + h) * kHeadDim;
    const I* vsrc = static_cast<const I*>(a.v) + (tok * a.nkv + h) * kHeadDim;

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
    if constexpr (std::is_same_v<S, I>) {
        copy8(vdst + 8 * qd, vsrc + 8 * qd);
        copy8(vdst + 8 * qd + 32, vsrc + 8 * qd + 32);
    } else {
        load8(vsrc + 8 * qd, x);
        load8(vsrc + 8 * qd + 32, y);
        store8(vdst + 8 * qd, x);
        store8(vdst + 8 * qd + 32, y);
    }
}

// ---- quantised pools (KV_DTYPE_Q8, KV_DTYPE_K8V4) ---------------------------
// K is rotated in fp32 exactly as above, then each 32-dim block quantised as
// BlockQ8_0::quantize (crates/llm-quant/src/lib.rs:26-36): scale =
// f16(max|x| / 127) to nearest even, inv = 1 / scale (0 for a zero scale),
// code = round-half-away(x * inv) clamped to [-127, 127].  V (bf16 in) is
// quantised the same way (Q8), or as BlockQ4::quantize (lib.rs:63-78, K8V4):
// scale f16(max|x| / 8), codes clamped to [-8, 7], element 2i in the low
// nibble of byte i.  The four threads of a (token, head) hold dims
// [8qd, 8qd+8) of block 0 and [32+8qd, ...) of block 1, so a block's max|x|
// is two shuffles inside the four-lane group (whose threads always exit
// together).

__device__ __forceinline__ float group4_max(float x, unsigned mask) {
    x = fmaxf(x, __shfl_xor_sync(mask, x, 1));
    return fmaxf(x, __shfl_xor_sync(mask, x, 2));
}

// The block's f16 scale bits and the reciprocal the codes are taken with.
__device__ __forceinline__ float block_inv(float amax, float div, uint16_t& bits) {
    const __half h = __float2half_rn(amax / div);
    bits = __half_as_ushort(h);
    const float sf = __half2float(h);
    return sf == 0.f ? 0.f : 1.f / sf;
}

__device__ __forceinline__ uint2 codes_q8(const float (&x)[8], float inv) {
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float q = fminf(fmaxf(roundf(__fmul_rn(x[e], inv)), -127.f), 127.f);
        w[e >> 2] |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xffu) << (8 * (e & 3));
    }
    return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ uint32_t codes_q4(const float (&x)[8], float inv) {
    uint32_t w = 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float q = fminf(fmaxf(roundf(__fmul_rn(x[e], inv)), -8.f), 7.f);
        w |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xfu) << (4 * e);
    }
    return w;
}

template <bool kV4>
__global__ void __launch_bounds__(256) append_q_kernel(uint8_t* __restrict__ pages, const AppendArgs a) {
    const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per_tok = a.nkv * 4;
    const long long tok = gtid / per_tok;
    if (tok >= a.n_tokens) return;
    const int r = static_cast<int>(gtid % per_tok);
    const int h = r >> 2, qd = r & 3;
    const unsigned mask = 0xfu << (threadIdx.x & 28);  // this (token, head)'s four lanes
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
    constexpr int kVRow = kV4 ? 32 : 64;
    constexpr size_t kHeadBlock = static_cast<size_t>(kPageTokens) * (64 + kVRow + 8);
    const size_t j = static_cast<size_t>(slot % kPageTokens);
    // the head's block of the page: K codes, V codes, K scales, V scales
    uint8_t* blk = pages + (static_cast<size_t>(page) * a.nkv + h) * kHeadBlock;
    uint8_t* kc = blk + j * 64;
    uint8_t* vc = blk + kPageTokens * 64 + j * kVRow;
    uint8_t* sc = blk + kPageTokens * (64 + kVRow) + j * 8;  // [block][K scale, V scale]
    const __nv_bfloat16* ksrc = static_cast<const __nv_bfloat16*>(a.k) + (tok * a.nkv + h) * kHeadDim;
    const __nv_bfloat16* vsrc = static_cast<const __nv_bfloat16*>(a.v) + (tok * a.nkv + h) * kHeadDim;

    float x[8], y[8], xo[8], yo[8];
    load8(ksrc + 8 * qd, x);
    load8(ksrc + 8 * qd + 32, y);
    if (a.k_norm) {
        // the row's RMSNorm (ops.rs:8-23, lfm2.rs:805-812) before RoPE; each of
        // the four threads works the row's scale out itself
        const float sc = rms_scale_row(ksrc, a.eps);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            x[e] = rms_apply(x[e], sc, __ldg(a.k_norm + 8 * qd + e));
            y[e] = rms_apply(y[e], sc, __ldg(a.k_norm + 32 + 8 * qd + e));
        }
    }
    const float2* cs = a.rope + static_cast<size_t>(pos) * (kHeadDim / 2) + 8 * qd;
    float ax = 0.f, ay = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float2 c = __ldg(cs + e);
        xo[e] = __fadd_rn(__fmul_rn(x[e], c.x), __fmul_rn(-y[e], c.y));
        yo[e] = __fadd_rn(__fmul_rn(y[e], c.x), __fmul_rn(x[e], c.y));
        ax = fmaxf(ax, fabsf(xo[e]));
        ay = fmaxf(ay, fabsf(yo[e]));
    }
    uint16_t kb0, kb1;
    const float kinv0 = block_inv(group4_max(ax, mask), 127.f, kb0);
    const float kinv1 = block_inv(group4_max(ay, mask), 127.f, kb1);
    *reinterpret_cast<uint2*>(kc + 8 * qd) = codes_q8(xo, kinv0);
    *reinterpret_cast<uint2*>(kc + 32 + 8 * qd) = codes_q8(yo, kinv1);

    load8(vsrc + 8 * qd, x);
    load8(vsrc + 8 * qd + 32, y);
    float vx = 0.f, vy = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        vx = fmaxf(vx, fabsf(x[e]));
        vy = fmaxf(vy, fabsf(y[e]));
    }
    uint16_t vb0, vb1;
    const float div = kV4 ? 8.f : 127.f;
    const float vinv0 = block_inv(group4_max(vx, mask), div, vb0);
    const float vinv1 = block_inv(group4_max(vy, mask), div, vb1);
    if constexpr (kV4) {
        *reinterpret_cast<uint32_t*>(vc + 4 * qd) = codes_q4(x, vinv0);
        *reinterpret_cast<uint32_t*>(vc + 16 + 4 * qd) = codes_q4(y, vinv1);
    } else {
        *reinterpret_cast<uint2*>(vc + 8 * qd) = codes_q8(x, vinv0);
        *reinterpret_cast<uint2*>(vc + 32 + 8 * qd) = codes_q8(y, vinv1);
    }
    if (qd == 0)
        *reinterpret_cast<uint2*>(sc) = make_uint2(static_cast<uint32_t>(kb0) | (static_cast<uint32_t>(vb0) << 16),
                                                  static_cast<uint32_t>(kb1) | (static_cast<uint32_t>(vb1) << 16));
}

}  // namespace

int launch_append(kv_pool* pool, const void* k, const void* v, const int32_t* tok_seq,
                  const int32_t* tok_slot, const int32_t* tok_pos, const int32_t* seq_lens,
                  int32_t n_tokens, int32_t n_seqs, const uint32_t* bt, int32_t bt_stride,
                  cudaStream_t stream, const float* k_norm, float eps) {
    if (k_norm && !is_quant(pool->cfg.dtype)) return KV_ERR_UNSUPPORTED;  // bf16 / f16 / fp32 fold it into the decode
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
    a.k_norm = k_norm;
    a.eps = eps;
    const long long threads = static_cast<long long>(n_tokens) * a.nkv * 4;
    const int block = 256;
    const unsigned grid = static_cast<unsigned>((threads + block - 1) / block);
    if (pool->cfg.dtype == KV_DTYPE_BF16)
        append_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(
            static_cast<__nv_bfloat16*>(pool->pages), a);
    else if (pool->cfg.dtype == KV_DTYPE_F16)
        append_kernel<__half, __nv_bfloat16><<<grid, block, 0, stream>>>(static_cast<__half*>(pool->pages), a);
    else if (pool->cfg.dtype == KV_DTYPE_Q8)
        append_q_kernel<false><<<grid, block, 0, stream>>>(static_cast<uint8_t*>(pool->pages), a);
    else if (pool->cfg.dtype == KV_DTYPE_K8V4)
        append_q_kernel<true><<<grid, block, 0, stream>>>(static_cast<uint8_t*>(pool->pages), a);
    else
        append_kernel<float><<<grid, block, 0, stream>>>(static_cast<float*>(pool->pages), a);
    return cudaGetLastError() == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
