// kv_prefill_f32.cu -- chunked-prefill and tree-verify attention for fp32 pools.
//
// The fp32 counterpart of kv_prefill.cu (same entry point, same masks: every
// cached key s < L, chunk key L + j when j <= i or, with tree masks, when bit j
// of the row's ancestor-or-self mask is set).  fp32 has no tensor-core path
// here, so this runs on the CUDA cores, in fp32 throughout, to stay within the
// 1e-5 relative bound of attention_forward (crates/llm-engine/src/lfm2.rs:
// 1058-1111).
//
// Quantised pools (KV_DTYPE_Q8, KV_DTYPE_K8V4) and half pools (KV_DTYPE_F16)
// run the same kernel: their pages are widened into the fp32 staging (code x
// f16 block scale, or the half value; both exact in fp32) and their q and out
// are bf16.
//
// One CTA (8 warps) per (sequence, kv head, kTokens query tokens); a row is a
// (token, query head of the group) pair, up to 32 rows per CTA.  Per page of
// 16 keys the CTA stages this head's K and V slices (4 KiB each) in shared
// memory, double-buffered with cp.async; each warp then serves its rows:
// lanes (2k, 2k+1) split key k's 64-dim dot product, the page maximum and sum
// are warp reductions, and lane l accumulates output dims 2l, 2l+1.  Scores
// are in log2 units (q pre-scaled by log2(e)/sqrt(d)) with an online max.
#include <cuda_fp16.h>

#include <cmath>

#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace kvb200 {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxRows = 32;          // query rows per CTA
constexpr int kHalf = 33;             // padded half-row of a staged K slice (floats)
constexpr int kKRow = 2 * kHalf;      // one key's 64 dims in two padded halves

struct PrefillF32Args {
    const void* q;        // fp32 (fp32 pools) or bf16 (quantised pools)
    const int32_t* q_pos;
    const int32_t* q_off;
    const int32_t* prefix;
    const unsigned long long* tree;
    const uint32_t* bt;
    long long bt_stride;
    int n_q, nkv, group, tokens, max_q;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    const void* pages;
    size_t page_bytes;
    void* out;            // as q
    int* err;
    float qscale;
};

__device__ __forceinline__ float ex2f(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

struct Stage {
    float k[kPageTokens * kKRow];   // key kk: dims [0,32) at kk*66, [32,64) at kk*66 + 33
    float v[kPageTokens * kHeadDim];
};

// kQ: 0 fp32 pages; 1 Q8, 2 K8V4, 3 IEEE-half pages (bf16 q and out)
template <int kQ>
__global__ void __launch_bounds__(kWarps * 32) prefill_f32_kernel(const PrefillF32Args a) {
    const int s = blockIdx.z, h = blockIdx.y;
    const int q0 = __ldg(a.q_off + s);
    const int T = __ldg(a.q_off + s + 1) - q0;
    const int L = __ldg(a.prefix + s);
    const bool tree = a.tree != nullptr;
    if (T < 0 || L < 0 || T > a.max_q || (tree && T > 64)) {
        if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0) flag_error(a.err, kDevErrBadArg);
        return;
    }
    const int t_begin = blockIdx.x * a.tokens;
    if (t_begin >= T) return;
    const int t_end = min(T, t_begin + a.tokens);
    const int n_rows = (t_end - t_begin) * a.group;
    const int kmax = tree ? L + T : L + t_end;
    const int np = (kmax + kPageTokens - 1) / kPageTokens;

    __shared__ __align__(16) float q_s[kMaxRows][kKRow];  // dims [0,32) at 0, [32,64) at kHalf
    __shared__ __align__(16) Stage stage[2];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // q rows: RoPE at q_pos (rope.rs:76 form), scaled into log2 units
    for (int e = threadIdx.x; e < n_rows * (kHeadDim / 2); e += blockDim.x) {
        const int row = e / (kHeadDim / 2), i = e % (kHeadDim / 2);
        const int tok = t_begin + row / a.group, g = row % a.group;
        const size_t qrow = (static_cast<size_t>(q0 + tok) * a.n_q + h * a.group + g) * kHeadDim;
        int pos = __ldg(a.q_pos + q0 + tok);
        if (pos < 0 || pos >= a.max_pos) {
            if (i == 0) flag_error(a.err, kDevErrBadPos);
            pos = 0;
        }
        const float2 c = __ldg(a.rope + static_cast<size_t>(pos) * (kHeadDim / 2) + i);
        float x, y;
        if constexpr (kQ == 0) {
            const float* src = static_cast<const float*>(a.q) + qrow;
            x = __ldg(src + i);
            y = __ldg(src + i + kHeadDim / 2);
        } else {
            const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(a.q) + qrow;
            x = __bfloat162float(src[i]);
            y = __bfloat162float(src[i + kHeadDim / 2]);
        }
        q_s[row][i] = __fadd_rn(__fmul_rn(x, c.x), __fmul_rn(-y, c.y)) * a.qscale;
        q_s[row][kHalf + i] = __fadd_rn(__fmul_rn(y, c.x), __fmul_rn(x, c.y)) * a.qscale;
    }

    // stage page p's K and V slices of head h (zeros past the table or the pool)
    auto load_page = [&](int p, Stage& dst) {
        uint32_t phys = kPageNone;
        if (p < a.bt_stride) phys = __ldg(a.bt + static_cast<size_t>(s) * a.bt_stride + p);
        const bool ok = phys < a.n_pages;
        if (!ok && threadIdx.x == 0) flag_error(a.err, kDevErrBadPage);
        // 16 keys x 64 dims = 256 float4 per slice: thread t moves one of K and one of V
        const int t = threadIdx.x, kk = t / 16, c4 = t % 16;  // dims 4*c4 .. 4*c4+3
        float* kdst = dst.k + kk * kKRow + (c4 < 8 ? 4 * c4 : kHalf + 4 * (c4 - 8));
        float* vdst = dst.v + kk * kHeadDim + 4 * c4;
        if (!ok) {
            kdst[0] = kdst[1] = kdst[2] = kdst[3] = 0.f;
            *reinterpret_cast<float4*>(vdst) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if constexpr (kQ == 0) {
            const float* kb = static_cast<const float*>(a.pages) + static_cast<size_t>(phys) * (a.page_bytes / 4) +
                              static_cast<size_t>(h) * kPageTokens * kHeadDim;
            const float* vb = kb + static_cast<size_t>(a.nkv) * kPageTokens * kHeadDim;
            // the padded K half-rows are not 16-byte aligned: plain loads there
            const float4 kv = __ldg(reinterpret_cast<const float4*>(kb + kk * kHeadDim) + c4);
            kdst[0] = kv.x;
            kdst[1] = kv.y;
            kdst[2] = kv.z;
            kdst[3] = kv.w;
            cp_async16(vdst, vb + kk * kHeadDim + 4 * c4);
        } else if constexpr (kQ == 3) {
            // half pages in the bf16 layout: K block [nkv][16][64], then V
            const __half* kb = reinterpret_cast<const __half*>(static_cast<const uint8_t*>(a.pages) +
                                                               static_cast<size_t>(phys) * a.page_bytes) +
                               static_cast<size_t>(h) * kPageTokens * kHeadDim;
            const __half* vb = kb + static_cast<size_t>(a.nkv) * kPageTokens * kHeadDim;
            const uint2 kw = __ldg(reinterpret_cast<const uint2*>(kb + kk * kHeadDim + 4 * c4));
            const uint2 vw = __ldg(reinterpret_cast<const uint2*>(vb + kk * kHeadDim + 4 * c4));
            const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
            const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
            const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vw.x));
            const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vw.y));
            kdst[0] = k0.x;
            kdst[1] = k0.y;
            kdst[2] = k1.x;
            kdst[3] = k1.y;
            *reinterpret_cast<float4*>(vdst) = make_float4(v0.x, v0.y, v1.x, v1.y);
        } else {
            // head block of the page: K codes [16][64], V codes [16][vrow],
            // scales [16][2 blocks][K, V]; dims 4 c4 .. lie in block c4 / 8
            constexpr int kVRow = kQ == 2 ? 32 : 64;
            const uint8_t* blk = static_cast<const uint8_t*>(a.pages) + static_cast<size_t>(phys) * a.page_bytes +
                                 static_cast<size_t>(h) * kPageTokens * (kHeadDim + kVRow + 8);
            const uint32_t sc = __ldg(reinterpret_cast<const uint32_t*>(blk + kPageTokens * (kHeadDim + kVRow) +
                                                                       kk * 8 + (c4 / 8) * 4));
            const float ks = __half2float(__ushort_as_half(static_cast<unsigned short>(sc & 0xffffu)));
            const float vs = __half2float(__ushort_as_half(static_cast<unsigned short>(sc >> 16)));
            const uint32_t kw = __ldg(reinterpret_cast<const uint32_t*>(blk + kk * kHeadDim + 4 * c4));
#pragma unroll
            for (int e = 0; e < 4; ++e)
                kdst[e] = static_cast<float>(static_cast<int8_t>((kw >> (8 * e)) & 0xffu)) * ks;
            float vv[4];
            if constexpr (kQ == 2) {
                const uint32_t vw = __ldg(reinterpret_cast<const unsigned short*>(blk + kPageTokens * kHeadDim +
                                                                                  kk * kVRow + 2 * c4));
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    vv[e] = static_cast<float>(static_cast<int>(vw << (28 - 4 * e)) >> 28) * vs;
            } else {
                const uint32_t vw = __ldg(reinterpret_cast<const uint32_t*>(blk + kPageTokens * kHeadDim +
                                                                           kk * kVRow + 4 * c4));
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    vv[e] = static_cast<float>(static_cast<int8_t>((vw >> (8 * e)) & 0xffu)) * vs;
            }
            *reinterpret_cast<float4*>(vdst) = make_float4(vv[0], vv[1], vv[2], vv[3]);
        }
        cp_async_commit();
    };

    // per-row online state: rows warp, warp + 8, ... (at most 4 per warp)
    float m[4], l[4];
    float2 acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
        acc[i] = make_float2(0.f, 0.f);
    }
    const int kk = lane >> 1, half = lane & 1;

    load_page(0, stage[0]);
    for (int p = 0; p < np; ++p) {
        Stage& cur = stage[p & 1];
        if (p + 1 < np) {
            __syncthreads();  // everyone is done with stage[(p+1) & 1] (page p-1)
            load_page(p + 1, stage[(p + 1) & 1]);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // page p staged (and, at p = 0, q_s)
        const int key = p * kPageTokens + kk;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = warp + kWarps * i;
            if (row >= n_rows) break;
            // score of key kk: lanes 2kk, 2kk+1 each take 32 dims
            const float* qr = q_s[row] + kHalf * half;
            const float* kr = cur.k + kk * kKRow + kHalf * half;
            float d0 = 0.f, d1 = 0.f;
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                d0 = fmaf(qr[e], kr[e], d0);
                d1 = fmaf(qr[e + 1], kr[e + 1], d1);
            }
            float sc = d0 + d1;
            sc += __shfl_xor_sync(0xffffffffu, sc, 1);
            // visibility
            const int tok = t_begin + row / a.group;
            bool vis;
            if (key < L) vis = true;
            else if (key >= L + T) vis = false;
            else if (tree) vis = (__ldg(a.tree + q0 + tok) >> (key - L)) & 1ull;
            else vis = (key - L) <= tok;
            if (!vis) sc = -INFINITY;
            float pm = sc;
#pragma unroll
            for (int o = 2; o < 32; o <<= 1) pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, o));
            const float mn = fmaxf(m[i], pm);
            const float mu = mn == -INFINITY ? 0.f : mn;
            const float alpha = ex2f(m[i] - mu);
            const float pk = ex2f(sc - mu);
            float ps = half ? 0.f : pk;  // one lane per key
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l[i] = l[i] * alpha + ps;
            m[i] = mn;
            float2 o2 = make_float2(acc[i].x * alpha, acc[i].y * alpha);
#pragma unroll
            for (int k2 = 0; k2 < kPageTokens; ++k2) {
                const float pv = __shfl_sync(0xffffffffu, pk, 2 * k2);
                const float2 vv = *reinterpret_cast<const float2*>(cur.v + k2 * kHeadDim + 2 * lane);
                o2.x = fmaf(pv, vv.x, o2.x);
                o2.y = fmaf(pv, vv.y, o2.y);
            }
            acc[i] = o2;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = warp + kWarps * i;
        if (row >= n_rows) break;
        const int tok = t_begin + row / a.group, g = row % a.group;
        const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
        const size_t orow = (static_cast<size_t>(q0 + tok) * a.n_q + h * a.group + g) * kHeadDim;
        if constexpr (kQ == 0)
            reinterpret_cast<float2*>(static_cast<float*>(a.out) + orow)[lane] =
                make_float2(acc[i].x * inv, acc[i].y * inv);
        else
            reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.out) + orow)[lane] =
                float2_to_bf16x2(acc[i].x * inv, acc[i].y * inv);
    }
}

}  // namespace

int launch_prefill_f32(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                       const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                       const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream) {
    const auto& c = pool->cfg;
    const int group = c.n_q_heads / c.n_kv_heads;
    if (group < 1 || group > kMaxRows) return KV_ERR_UNSUPPORTED;
    PrefillF32Args a;
    a.q = q;
    a.q_pos = q_pos;
    a.q_off = q_off;
    a.prefix = prefix;
    a.tree = tree;
    a.bt = bt;
    a.bt_stride = bt_stride;
    a.n_q = c.n_q_heads;
    a.nkv = c.n_kv_heads;
    a.group = group;
    a.tokens = kMaxRows / group;
    a.max_q = max_q;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.pages = pool->pages;
    a.page_bytes = pool->page_bytes;
    a.out = out;
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    const dim3 grid((max_q + a.tokens - 1) / a.tokens, c.n_kv_heads, n_seqs);
    if (c.dtype == KV_DTYPE_Q8)
        prefill_f32_kernel<1><<<grid, kWarps * 32, 0, stream>>>(a);
    else if (c.dtype == KV_DTYPE_K8V4)
        prefill_f32_kernel<2><<<grid, kWarps * 32, 0, stream>>>(a);
    else if (c.dtype == KV_DTYPE_F16)
        prefill_f32_kernel<3><<<grid, kWarps * 32, 0, stream>>>(a);
    else
        prefill_f32_kernel<0><<<grid, kWarps * 32, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
