// kv_decode.cu -- paged decode attention for sm_100a (split-K over pages).
//
// Replaces attention_decode_cached (crates/llm-engine/src/lfm2.rs:1006-1056)
// plus the q RoPE that precedes it (lfm2.rs:816-822).  Math per query head h
// (kv head h / g, lfm2.rs:1028): scores = (q . k) / sqrt(d), masked keys get
// -inf, softmax over the keys, out = sum_s w_s v_s.  Here the softmax is the
// online (running-max) form, so each split of the key range produces
// (max, sum, unnormalised out) and splits merge by the log-sum-exp identity
// (Milakov & Gimelshein 2018); the result equals the reference's to fp32
// rounding.
//
// Work split ("stream-K" over pages): the pages of all sequences are laid
// end to end (per-sequence page counts, exclusive-scanned in shared memory)
// and every CTA of a persistent grid (SMs x CTAs/SM) takes an equal slice of
// that list, so skewed sequence lengths cannot unbalance the SMs.  A sequence
// wholly inside one slice is finished by that CTA; a sequence cut by slice
// boundaries leaves one partial per CTA, and the last CTA to finish it
// (atomic counter, no waiting) merges the partials and resets the counter.
//
// Data path per CTA: warp 0 streams whole pages (K and V of all kv heads, one
// contiguous 4- to 64-KiB block) with TMA 2-D tile loads, 128-byte swizzled,
// STAGES-1 pages ahead of use, into a ring of STAGES page buffers guarded by
// full/empty mbarriers.  Two warps own each kv head and take alternate
// pages: QK^T with 4 lanes per key (16 dims each, FFMA2, 2 keys per lane),
// the page max in one redux.sync, p to shared memory as (p, p) pairs, then PV
// with each lane owning 2 output dims over the page's 16 keys.  The two
// warps' states merge through shared memory when a sequence's slice ends.
// Every wait is bounded by %globaltimer; a timeout sets the pool's error word
// and an abort flag so the CTA drains and exits instead of hanging.
#include <cmath>
#include <map>
#include <mutex>

#include "kv_common.cuh"
#include "kv_decode_sched.cuh"
#include "kv_pool_impl.h"

namespace kvb200 {
namespace {

template <typename T, int NKV>
struct Geom {
    static constexpr int kElem = sizeof(T);
    static constexpr int kRowsPerToken = kHeadDim * kElem / 128;  // 1 (bf16) or 2 (f32)
    static constexpr int kPageRows = 2 * NKV * kPageTokens * kRowsPerToken;
    static constexpr int kPageBytes = kPageRows * 128;
    static constexpr int kBoxRows = kPageRows > 256 ? 256 : kPageRows;
    static constexpr int kLoads = kPageRows / kBoxRows;
};

struct DecodeArgs {
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
    float qscale;  // log2(e) / sqrt(d): scores come out in log2 units
    // Fused append (kv_append_decode_attn): the new token's K and V,
    // [n_seqs, NKV, 64] each, stored at slot seq_lens[s] - 1 before it is
    // attended.  Null: plain decode.
    const void* new_k;
    const void* new_v;
    void* pages;
    // kv_norm_append_decode_attn: the attention layer's per-head RMSNorm of q
    // and of the new k before RoPE ([64] weights each; null: none).
    const float* q_norm;
    const float* k_norm;
    float eps;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (*abort_flag) return false;
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            flag_error(err, kDevErrTimeout);
            return false;
        }
    }
}

template <typename T> __device__ __forceinline__ T to_elem(float x);
template <> __device__ __forceinline__ float to_elem<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 to_elem<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// q for heads h*G .. h*G+G-1 of sequence s, dims [16*qd, 16*qd+16), rotated
// at `pos` exactly as rope.rs:56-81 (two products and a sum, no FMA) and
// scaled into log2 units.  Two dims at a time to keep few registers live.
__device__ __forceinline__ float2 load_pair(const __nv_bfloat16* p) {
    return bf16x2_to_float2(__ldg(reinterpret_cast<const unsigned int*>(p)));
}
__device__ __forceinline__ float2 load_pair(const float* p) {
    return __ldg(reinterpret_cast<const float2*>(p));
}

// With a.q_norm, each head row is first RMS-normalised (lfm2.rs:797-804):
// lanes 0..G-1 work out the scales of the G heads, one row each.
template <typename T, int G>
__device__ __forceinline__ void load_q(const DecodeArgs& a, int s, int nq, int h, int qd, int pos,
                                       float2 (&q2)[G][8], int lane) {
    const float4* cs = reinterpret_cast<const float4*>(a.rope + static_cast<size_t>(pos) * (kHeadDim / 2) +
                                                       ((16 * qd) & 31));
    const float sgn = qd < 2 ? -1.f : 1.f;
    const T* rows = static_cast<const T*>(a.q) + (static_cast<size_t>(s) * nq + h * G) * kHeadDim;
    float sc[G];
    if (a.q_norm != nullptr) {
        const float mine = lane < G ? rms_scale_row(rows + (lane < G ? lane : 0) * kHeadDim, a.eps) : 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = __shfl_sync(~0u, mine, g);
    }
    const int dx = 16 * qd, dy = (16 * qd + 32) & 63;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 c = __ldg(cs + i);  // (cos, sin) of dims 16qd+2i and 16qd+2i+1
        float2 wx = make_float2(1.f, 1.f), wy = make_float2(1.f, 1.f);
        if (a.q_norm != nullptr) {
            wx = __ldg(reinterpret_cast<const float2*>(a.q_norm + dx + 2 * i));
            wy = __ldg(reinterpret_cast<const float2*>(a.q_norm + dy + 2 * i));
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const T* row = rows + g * kHeadDim;
            float2 x = load_pair(row + dx + 2 * i);
            float2 y = load_pair(row + dy + 2 * i);
            if (a.q_norm != nullptr) {
                x = make_float2(rms_apply(x.x, sc[g], wx.x), rms_apply(x.y, sc[g], wx.y));
                y = make_float2(rms_apply(y.x, sc[g], wy.x), rms_apply(y.y, sc[g], wy.y));
            }
            const float r0 = __fadd_rn(__fmul_rn(x.x, c.x), __fmul_rn(sgn * y.x, c.y));
            const float r1 = __fadd_rn(__fmul_rn(x.y, c.z), __fmul_rn(sgn * y.y, c.w));
            q2[g][i] = make_float2(r0 * a.qscale, r1 * a.qscale);
        }
    }
}

// ---- per-lane shared-memory offsets ------------------------------------------
// The TMA writes each page with the 128-byte swizzle: 16-byte chunk c of
// 128-byte row R lands at chunk c ^ (R & 7).  The offsets below fold that in
// once per lane.  K: lane (j = lane/4, qd = lane%4) reads key j of its head,
// dims [16qd, 16qd+16); key j+8 sits kKey8 bytes further with the same
// swizzle.  V: lane (kh = lane/16, dg = lane%16) reads dims [4dg, 4dg+4) of
// key 8kh+t at vaddr(t), an XOR with a compile-time constant plus an
// immediate offset.
template <typename T> struct LaneOffsets;

template <> struct LaneOffsets<__nv_bfloat16> {
    static constexpr uint32_t kKey8 = 8 * 128;
    uint32_t k[2];
    uint32_t v;
    __device__ __forceinline__ LaneOffsets(int h, int lane, int nkv) {
        const uint32_t j = lane >> 2, qd = lane & 3;
        const uint32_t row = h * kPageTokens + j;
        k[0] = row * 128 + (((2 * qd) ^ j) << 4);
        k[1] = row * 128 + (((2 * qd + 1) ^ j) << 4);
        const uint32_t kh = lane >> 4, dg = lane & 15;
        v = ((nkv + h) * kPageTokens + 8 * kh) * 128 + ((dg >> 1) << 4) + (dg & 1) * 8;
    }
    // key 8kh + t, t in [0, 8): row & 7 == t
    __device__ __forceinline__ uint32_t vaddr(int t) const { return (v ^ (t << 4)) + t * 128; }
};

template <> struct LaneOffsets<float> {
    static constexpr uint32_t kKey8 = 8 * 256;
    uint32_t k[4];
    uint32_t v;
    __device__ __forceinline__ LaneOffsets(int h, int lane, int nkv) {
        const uint32_t j = lane >> 2, qd = lane & 3;
        const uint32_t R = (h * kPageTokens + j) * 2 + (qd >> 1);
#pragma unroll
        for (int c = 0; c < 4; ++c) k[c] = R * 128 + ((((qd & 1) * 4 + c) ^ (R & 7)) << 4);
        // dims [4dg, 4dg+4) of key row r = 16 bytes at r*256 + 16dg: 128-byte
        // row 2r + dg/8, chunk dg%8, and (2r + dg/8) & 7 = 2t + dg/8 for
        // r = 8kh + t (+ multiples of 16).
        const uint32_t kh = lane >> 4, dg = lane & 15, b = dg >> 3;
        v = ((nkv + h) * kPageTokens + 8 * kh) * 256 + b * 128 + (((dg & 7) ^ b) << 4);
    }
    __device__ __forceinline__ uint32_t vaddr(int t) const {
        return (v ^ (((2 * t) & 7) << 4)) + t * 256;
    }
};

__device__ __forceinline__ void load_key(const uint8_t* buf, const LaneOffsets<__nv_bfloat16>& o,
                                         uint32_t extra, float2 (&k)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(buf + o.k[0] + extra);
    const uint4 b = *reinterpret_cast<const uint4*>(buf + o.k[1] + extra);
    k[0] = bf16x2_to_float2(a.x); k[1] = bf16x2_to_float2(a.y);
    k[2] = bf16x2_to_float2(a.z); k[3] = bf16x2_to_float2(a.w);
    k[4] = bf16x2_to_float2(b.x); k[5] = bf16x2_to_float2(b.y);
    k[6] = bf16x2_to_float2(b.z); k[7] = bf16x2_to_float2(b.w);
}
__device__ __forceinline__ void load_key(const uint8_t* buf, const LaneOffsets<float>& o,
                                         uint32_t extra, float2 (&k)[8]) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const float4 f = *reinterpret_cast<const float4*>(buf + o.k[c] + extra);
        k[2 * c] = make_float2(f.x, f.y);
        k[2 * c + 1] = make_float2(f.z, f.w);
    }
}

// V of one key, the lane's 4 dims, as two float2.
__device__ __forceinline__ void load_v(const uint8_t* buf, const LaneOffsets<__nv_bfloat16>& o, int t,
                                       float2& v0, float2& v1) {
    const uint2 w = *reinterpret_cast<const uint2*>(buf + o.vaddr(t));
    v0 = bf16x2_to_float2(w.x);
    v1 = bf16x2_to_float2(w.y);
}
__device__ __forceinline__ void load_v(const uint8_t* buf, const LaneOffsets<float>& o, int t,
                                       float2& v0, float2& v1) {
    const float4 f = *reinterpret_cast<const float4*>(buf + o.vaddr(t));
    v0 = make_float2(f.x, f.y);
    v1 = make_float2(f.z, f.w);
}

// Byte offset in a staged page of byte b of token row r (the 128-byte
// swizzle of the TMA copy: chunk c of 128-byte row R sits at chunk c ^ (R & 7)).
template <typename T>
__device__ __forceinline__ uint32_t staged_offset(int r, int b) {
    constexpr int kRpt = kHeadDim * static_cast<int>(sizeof(T)) / 128;
    const int R = r * kRpt + (b >> 7);
    return static_cast<uint32_t>(R * 128 + ((((b & 127) >> 4) ^ (R & 7)) << 4) + (b & 15));
}

// Bytes a warp stages for a fused append: the new token's K and V rows of
// its kv head and the (cos, sin) row of its position.
template <typename T>
constexpr int patch_bytes() { return 2 * kHeadDim * static_cast<int>(sizeof(T)) + kHeadDim / 2 * 8; }

// Fused append, part 1 (when the warp starts the sequence): cp.async the
// inputs into the warp's staging area, so part 2 never waits on HBM while it
// holds a stage of the page ring.
template <typename T>
__device__ __forceinline__ void stage_patch_inputs(uint8_t* dst, const T* ks, const T* vs, const float2* cs,
                                                   int lane) {
    constexpr int nk = kHeadDim * static_cast<int>(sizeof(T)) / 16;  // 16-byte pieces of a row
    for (int c = lane; c < 2 * nk + 16; c += 32) {
        const void* src = c < nk       ? static_cast<const void*>(reinterpret_cast<const uint8_t*>(ks) + 16 * c)
                          : c < 2 * nk ? static_cast<const void*>(reinterpret_cast<const uint8_t*>(vs) + 16 * (c - nk))
                                       : static_cast<const void*>(reinterpret_cast<const uint8_t*>(cs) + 16 * (c - 2 * nk));
        cp_async16(dst + 16 * c, src);
    }
    cp_async_commit();
}

// Fused append, part 2: kv head h's new token (slot j of its page) written by
// the one warp that reads this head of the staged page, into the staged copy
// before the warp's first read of it and into the page in HBM (`gpage`).  K
// is rotated exactly as append_kernel does (two rounded products and a
// rounded sum per output, then rounding to the pool type), V copied as
// stored bits, so pages and attention are bit-identical to kv_append_decode
// followed by kv_decode_attn.  Lanes 0-15: K dims 2i, 2i+1 and their
// partners 32 + 2i, 33 + 2i; lanes 16-31: V dims [4i, 4i + 4).  Out of line:
// it runs once per sequence and head, and must not take registers from the
// page loop.
template <typename T, int NKV>
__device__ __noinline__ void patch_new_token(uint8_t* buf, uint8_t* gpage, const uint8_t* in, int h, int j,
                                             int lane, const float* k_norm, float eps) {
    constexpr int kE = static_cast<int>(sizeof(T));
    cp_async_wait<0>();
    __syncwarp();
    // With k_norm, the row is first RMS-normalised (lfm2.rs:805-812).
    float sc = 0.f;
    if (k_norm != nullptr) sc = __shfl_sync(~0u, lane == 0 ? rms_scale_row(reinterpret_cast<const T*>(in), eps) : 0.f, 0);
    const int i = lane & 15;
    if (lane < 16) {
        const int kr = h * kPageTokens + j;
        float2 x, y;
        if constexpr (kE == 2) {
            x = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(in + 4 * i));
            y = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(in + 64 + 4 * i));
        } else {
            x = *reinterpret_cast<const float2*>(in + 8 * i);
            y = *reinterpret_cast<const float2*>(in + 128 + 8 * i);
        }
        if (k_norm != nullptr) {
            const float2 wx = __ldg(reinterpret_cast<const float2*>(k_norm + 2 * i));
            const float2 wy = __ldg(reinterpret_cast<const float2*>(k_norm + 32 + 2 * i));
            x = make_float2(rms_apply(x.x, sc, wx.x), rms_apply(x.y, sc, wx.y));
            y = make_float2(rms_apply(y.x, sc, wy.x), rms_apply(y.y, sc, wy.y));
        }
        const float4 c = *reinterpret_cast<const float4*>(in + 2 * kHeadDim * kE + 16 * i);
        const float x0 = __fadd_rn(__fmul_rn(x.x, c.x), __fmul_rn(-y.x, c.y));
        const float x1 = __fadd_rn(__fmul_rn(x.y, c.z), __fmul_rn(-y.y, c.w));
        const float y0 = __fadd_rn(__fmul_rn(y.x, c.x), __fmul_rn(x.x, c.y));
        const float y1 = __fadd_rn(__fmul_rn(y.y, c.z), __fmul_rn(x.y, c.w));
        const int bx = 2 * i * kE, by = (32 + 2 * i) * kE;
        uint8_t* grow = gpage + kr * kHeadDim * kE;
        if constexpr (kE == 2) {
            const uint32_t wx = float2_to_bf16x2(x0, x1), wy = float2_to_bf16x2(y0, y1);
            *reinterpret_cast<uint32_t*>(buf + staged_offset<T>(kr, bx)) = wx;
            *reinterpret_cast<uint32_t*>(buf + staged_offset<T>(kr, by)) = wy;
            *reinterpret_cast<uint32_t*>(grow + bx) = wx;
            *reinterpret_cast<uint32_t*>(grow + by) = wy;
        } else {
            *reinterpret_cast<float2*>(buf + staged_offset<T>(kr, bx)) = make_float2(x0, x1);
            *reinterpret_cast<float2*>(buf + staged_offset<T>(kr, by)) = make_float2(y0, y1);
            *reinterpret_cast<float2*>(grow + bx) = make_float2(x0, x1);
            *reinterpret_cast<float2*>(grow + by) = make_float2(y0, y1);
        }
    } else {
        const int vr = (NKV + h) * kPageTokens + j;
        const int b = 4 * i * kE;
        const uint8_t* vin = in + kHeadDim * kE + b;
        uint8_t* grow = gpage + vr * kHeadDim * kE;
        if constexpr (kE == 2) {
            const uint2 w = *reinterpret_cast<const uint2*>(vin);
            *reinterpret_cast<uint2*>(buf + staged_offset<T>(vr, b)) = w;
            *reinterpret_cast<uint2*>(grow + b) = w;
        } else {
            const float4 w = *reinterpret_cast<const float4*>(vin);
            *reinterpret_cast<float4*>(buf + staged_offset<T>(vr, b)) = w;
            *reinterpret_cast<float4*>(grow + b) = w;
        }
    }
    // The stage is refilled by the TMA (async proxy) once it is handed back.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
}

// Warp-wide max in one instruction (sm_100a redux.sync on f32).
__device__ __forceinline__ float warp_max(float x) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
    return r;
}

// 2^x; 2^-inf = +0.  Scores are already in log2 units.
__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// One page (16 keys) of one kv head; keys [t0, t1) of the page are valid
// (all of them when kMasked is false).  QK: lane (j, qd) scores keys j and
// j+8 over dims [16qd, 16qd+16) and reduces over the 4 lanes of a key by
// shuffles; the page max is one redux; p goes to shared memory as (p, p)
// pairs.  PV: lane (kh, dg) accumulates dims [4dg, 4dg+4) over keys
// [8kh, 8kh+8); the two key halves are merged when the sequence is flushed.
template <typename T, int G, bool kMasked>
__device__ __forceinline__ void page_step(const uint8_t* buf, const LaneOffsets<T>& lo, int lane,
                                          int t0, int t1, const float2 (&q2)[G][8],
                                          float2 (&o2)[G][2], float (&lp)[G], float (&M)[G],
                                          float2* pb) {
    const int j = lane >> 2, qd = lane & 3;
    float sa[G], sb[G];
    {
        float2 kv[8];
        load_key(buf, lo, 0, kv);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = __ffma2_rn(q2[g][i], kv[i], acc);
            sa[g] = acc.x + acc.y;
        }
        load_key(buf, lo, LaneOffsets<T>::kKey8, kv);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = __ffma2_rn(q2[g][i], kv[i], acc);
            sb[g] = acc.x + acc.y;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        sa[g] += __shfl_xor_sync(~0u, sa[g], 1);
        sb[g] += __shfl_xor_sync(~0u, sb[g], 1);
        sa[g] += __shfl_xor_sync(~0u, sa[g], 2);
        sb[g] += __shfl_xor_sync(~0u, sb[g], 2);
    }
    bool va = true, vb = true;
    if constexpr (kMasked) {
        va = j >= t0 && j < t1;
        vb = j + 8 >= t0 && j + 8 < t1;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float xa = va ? sa[g] : -INFINITY;
        const float xb = vb ? sb[g] : -INFINITY;
        const float mn = fmaxf(M[g], warp_max(fmaxf(xa, xb)));
        // A full page always holds a finite score; a masked one may not.
        const float mu = (kMasked && mn == -INFINITY) ? 0.f : mn;
        const float alpha = ex2(M[g] - mu);
        const float pa = ex2(xa - mu);
        const float pbv = ex2(xb - mu);
        lp[g] = fmaf(lp[g], alpha, qd == 0 ? pa + pbv : 0.f);
        o2[g][0] = __fmul2_rn(o2[g][0], make_float2(alpha, alpha));
        o2[g][1] = __fmul2_rn(o2[g][1], make_float2(alpha, alpha));
        M[g] = mn;
        if (qd == 0) {
            pb[g * 16 + j] = make_float2(pa, pa);
            pb[g * 16 + j + 8] = make_float2(pbv, pbv);
        }
    }
    __syncwarp();
    const int kh = lane >> 4;
#pragma unroll
    for (int t2 = 0; t2 < 4; ++t2) {
        float4 pq[G];
#pragma unroll
        for (int g = 0; g < G; ++g)
            pq[g] = *reinterpret_cast<const float4*>(pb + g * 16 + 8 * kh + 2 * t2);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = 2 * t2 + u;
            float2 v0, v1;
            load_v(buf, lo, t, v0, v1);
            if constexpr (kMasked) {
                // Slots outside [t0, t1) may hold another sequence's stale
                // values: zero them so 0 * (inf or nan) cannot leak in.
                const int key = 8 * kh + t;
                if (key < t0 || key >= t1) {
                    v0 = make_float2(0.f, 0.f);
                    v1 = make_float2(0.f, 0.f);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float2 pp = u == 0 ? make_float2(pq[g].x, pq[g].y) : make_float2(pq[g].z, pq[g].w);
                o2[g][0] = __ffma2_rn(pp, v0, o2[g][0]);
                o2[g][1] = __ffma2_rn(pp, v1, o2[g][1]);
            }
        }
    }
    __syncwarp();  // pb is rewritten by this warp's next page
}

// Sixteen warps: W = 16 / NKV per kv head, warp (h, sub) taking the slice
// pages k with k % W == sub; warp 0 also issues the loads.  Few kv heads
// (one GPU's share of a head-sharded session) thus still fill an SM with one
// CTA, and a long sequence splits into at most one partial per SM.
template <typename T, int NKV, int G, int STAGES>
struct DecodeShape {
    static constexpr int W = 16 / NKV;
    static_assert(16 % NKV == 0, "kv heads must divide 16");
    // A stage's successive pages (k, k + STAGES) go to the same warp: the warp
    // that waits on a stage's next phase has seen its previous one, so a
    // parity wait can never pass on a stale phase.  And STAGES >= W keeps every
    // warp's next page within the issued window.
    static_assert(STAGES % W == 0, "the page ring must hold a multiple of W stages");
    using Geo = Geom<T, NKV>;
    static constexpr int kConsumers = 16;
    static constexpr int kThreads = kConsumers * 32;
    static size_t smem_bytes(int max_seqs) {
        return 1024 + static_cast<size_t>(STAGES) * Geo::kPageBytes   // page ring
               + 2 * STAGES * 8                                         // full/empty barriers
               + static_cast<size_t>(kConsumers) * G * 16 * 8           // (p, p) buffers
               + static_cast<size_t>(NKV) * (W - 1) * G * (kHeadDim + 4) * 4  // per-head merge buffers
               + static_cast<size_t>(kConsumers) * patch_bytes<T>()    // fused-append staging
               + 16 + (static_cast<size_t>(max_seqs) + 1) * 4;          // misc + page scan
    }
};

template <typename T, int NKV, int G, int STAGES>
__global__ void __launch_bounds__(DecodeShape<T, NKV, G, STAGES>::kThreads, 1)
decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a) {
    using Geo = Geom<T, NKV>;
    constexpr int NQ = NKV * G;
    constexpr int W = DecodeShape<T, NKV, G, STAGES>::W;  // warps per kv head
    constexpr int NCW = 16;                               // warps
    constexpr int NCONS = NCW * 32;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* stage = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(stage + STAGES * Geo::kPageBytes);
    uint64_t* empty = full + STAGES;
    float2* pbuf = reinterpret_cast<float2*>(empty + STAGES);  // [NCW][G][16]
    float* xbuf = reinterpret_cast<float*>(pbuf + NCW * G * 16);  // [NKV][W - 1][G][64 + 4]
    uint8_t* patch_in = reinterpret_cast<uint8_t*>(xbuf + NKV * (W - 1) * G * (kHeadDim + 4));  // [NCW][patch_bytes]
    int* misc = reinterpret_cast<int*>(patch_in + NCW * patch_bytes<T>());  // [0] counter, [1] abort
    int* pstart = misc + 4;                                               // [n_seqs + 1]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = a.n_seqs;

    if (threadIdx.x == 32) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NKV);  // each page is consumed by one warp per kv head
        }
        fence_mbar_init();
        prefetch_tmap(&tmap);
        misc[0] = 0;
        misc[1] = 0;
    }
    if (warp == 0) scan_pages(a.seq_lens, n, a.window, pstart, lane);  // exclusive scan of page counts
    __syncthreads();

    const int total = pstart[n];
    const int cta = blockIdx.x;
    // Slices of at least kMinSlicePages pages: a short batch uses fewer CTAs
    // rather than splitting each sequence over many (whose partials one CTA
    // would then merge).
    const int grid = max(1, min(static_cast<int>(gridDim.x), total / kMinSlicePages));
    for (int s = cta; s < n; s += gridDim.x) {  // sequences with no tokens: zeros
        if (__ldg(a.seq_lens + s) <= 0) {
            T* o = static_cast<T*>(a.out) + static_cast<size_t>(s) * NQ * kHeadDim;
            for (int i = threadIdx.x; i < NQ * kHeadDim; i += NCONS) o[i] = to_elem<T>(0.f);
        }
    }
    if (cta >= grid) return;
    const int gb = static_cast<int>((static_cast<long long>(cta) * total) / grid);
    const int ge = static_cast<int>((static_cast<long long>(cta + 1) * total) / grid);
    if (gb >= ge) return;
    volatile int* abort_flag = misc + 1;

    // ---- load issue (warp 0): page i of this slice goes to stage i % STAGES ----
    // Lane l of warp 0 holds the physical id of slice page bt_base + l.
    const int n_local = ge - gb;
    int bt_base = -32;
    uint32_t bt_batch = 0;
    int issued = 0;  // pages issued so far (warp 0 only)
    bool issuing = true;
    auto issue_upto = [&](int upto) {  // warp 0: issue slice pages [issued, upto)
        upto = min(upto, n_local);
        while (issuing && issued < upto) {
            if (issued >= bt_base + 32) {
                bt_base = issued & ~31;
                const int gq = gb + bt_base + lane;
                bt_batch = 0;
                if (gq < ge) {
                    const int sq = find_seq(pstart, n, gq);
                    const int ntq = __ldg(a.seq_lens + sq);
                    const int pg = seq_lo(ntq, a.window) / kPageTokens + (gq - pstart[sq]);
                    // A row holds bt_stride entries: never read past it.
                    bt_batch = pg < a.bt_stride
                                   ? __ldg(a.bt + static_cast<size_t>(sq) * a.bt_stride + pg)
                                   : kPageNone;
                    if (bt_batch >= a.n_pages) {
                        flag_error(a.err, kDevErrBadPage);
                        bt_batch = 0;
                    }
                }
            }
            const uint32_t ph = __shfl_sync(~0u, bt_batch, issued - bt_base);
            bool ok = true;
            if (lane == 0) {
                const int st = issued % STAGES;
                if (issued >= STAGES)
                    ok = wait_or_abort(&empty[st], static_cast<uint32_t>(issued / STAGES - 1) & 1u,
                                       abort_flag, a.err);
                if (ok) {
                    mbar_arrive_expect_tx(&full[st], Geo::kPageBytes);
                    uint8_t* dst = stage + st * Geo::kPageBytes;
#pragma unroll
                    for (int b = 0; b < Geo::kLoads; ++b)
                        tma_load_2d(dst + b * Geo::kBoxRows * 128, &tmap, &full[st], 0,
                                    static_cast<int>(ph) * Geo::kPageRows + b * Geo::kBoxRows);
                }
            }
            if (!__shfl_sync(~0u, ok, 0)) {
                issuing = false;  // stop; consumers' waits on full[] see the abort flag
                return;
            }
            ++issued;
        }
    };
    if (warp == 0) issue_upto(STAGES);

    // ---- consumers: warp w owns kv head w/2 and the slice pages of parity w%2 ----
    const int h = warp / W, sub = warp % W;
    const int qd = lane & 3;
    const LaneOffsets<T> lofs(h, lane, NKV);
    float2* my_pb = pbuf + warp * (G * 16);
    float* head_x = xbuf + h * (W - 1) * G * (kHeadDim + 4);  // slots of warps sub = 1 .. W - 1
    float2 q2[G][8];
    float2 o2[G][2];
    float lp[G], M[G];
    int s = find_seq(pstart, n, gb);
    int g = gb;
    while (g < ge) {
        const int nt = __ldg(a.seq_lens + s);
        const int lo = seq_lo(nt, a.window);
        const int plo = lo / kPageTokens;
        const int s_begin = pstart[s], s_end = pstart[s + 1];
        const int seg_end = min(ge, s_end);
        int pos = nt - 1;
        // The new token is appended by the warp of each head that reads the
        // sequence's last page, when this slice holds it.
        bool patch = a.new_k != nullptr && s_end <= ge;
        if (pos >= a.max_pos) {
            if (lane == 0) flag_error(a.err, kDevErrBadPos);
            pos = 0;
            patch = false;  // as kv_append_decode: nothing stored
        }
        // Of the warps of a head, the one that reads the last page appends.
        patch = patch && ((s_end - 1 - gb) % W == sub);
        uint8_t* my_patch_in = patch_in + warp * patch_bytes<T>();
        if (patch) {
            const size_t src = (static_cast<size_t>(s) * NKV + h) * kHeadDim;
            stage_patch_inputs<T>(my_patch_in, static_cast<const T*>(a.new_k) + src,
                                  static_cast<const T*>(a.new_v) + src,
                                  a.rope + static_cast<size_t>(pos) * (kHeadDim / 2), lane);
        }
        load_q<T, G>(a, s, NQ, h, qd, pos, q2, lane);
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
            o2[gg][0] = o2[gg][1] = make_float2(0.f, 0.f);
            lp[gg] = 0.f;
            M[gg] = -INFINITY;
        }
        // This warp's pages of the segment: slice page k = g - gb with k % W == sub.
        for (int gw = g + ((sub - (g - gb)) % W + W) % W; gw < seg_end; gw += W) {
            const int k = gw - gb;
            // Up to page k + STAGES - 1: it reuses the stage of page k - 1,
            // never the stage of page k that this warp is about to read.
            if (warp == 0) issue_upto(k + STAGES);
            const int st = k % STAGES;
            const uint32_t par = static_cast<uint32_t>(k / STAGES) & 1u;
            // A failed wait (timeout or abort) keeps the stage: it is never
            // handed back, so no copy can be issued over one still landing.
            if (!wait_or_abort(&full[st], par, abort_flag, a.err)) continue;
            uint8_t* buf = stage + st * Geo::kPageBytes;
            const int pg = plo + (gw - s_begin);
            if (patch && gw == s_end - 1) {
                // The loader flagged a bad entry already; store nothing then.
                const uint32_t page = pg < a.bt_stride
                                          ? __ldg(a.bt + static_cast<size_t>(s) * a.bt_stride + pg)
                                          : kPageNone;
                if (page < a.n_pages)
                    patch_new_token<T, NKV>(buf, static_cast<uint8_t*>(a.pages) + static_cast<size_t>(page) * Geo::kPageBytes,
                                            my_patch_in, h, pos % kPageTokens, lane, a.k_norm, a.eps);
            }
            const int t0 = max(lo - pg * kPageTokens, 0);
            const int t1 = min(nt - pg * kPageTokens, kPageTokens);
            if (t0 == 0 && t1 == kPageTokens)
                page_step<T, G, false>(buf, lofs, lane, t0, t1, q2, o2, lp, M, my_pb);
            else
                page_step<T, G, true>(buf, lofs, lane, t0, t1, q2, o2, lp, M, my_pb);
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        // Keep the ring full across the flush below; the pages this waits on
        // are released by the other warps before they reach the flush.
        if (warp == 0) issue_upto(seg_end - gb + STAGES - 1);
        g = seg_end;
        // ---- flush sequence s: sum lane partials, merge the key halves
        // (lanes l and l^16 hold the same dims), then the two warps of a head.
#pragma unroll
        for (int gg = 0; gg < G; ++gg) {
            float t = lp[gg];
            t += __shfl_xor_sync(~0u, t, 16);
            t += __shfl_xor_sync(~0u, t, 8);
            t += __shfl_xor_sync(~0u, t, 4);
            t += __shfl_xor_sync(~0u, t, 2);
            t += __shfl_xor_sync(~0u, t, 1);
            lp[gg] = t;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                o2[gg][c].x += __shfl_xor_sync(~0u, o2[gg][c].x, 16);
                o2[gg][c].y += __shfl_xor_sync(~0u, o2[gg][c].y, 16);
            }
        }
        const int dg = lane & 15;
        if (sub != 0 && lane < 16) {
            float* my_x = head_x + (sub - 1) * G * (kHeadDim + 4);
#pragma unroll
            for (int gg = 0; gg < G; ++gg) {
                *reinterpret_cast<float4*>(my_x + gg * (kHeadDim + 4) + 4 * dg) =
                    make_float4(o2[gg][0].x, o2[gg][0].y, o2[gg][1].x, o2[gg][1].y);
                if (lane == 0) {
                    my_x[gg * (kHeadDim + 4) + kHeadDim] = M[gg];
                    my_x[gg * (kHeadDim + 4) + kHeadDim + 1] = lp[gg];
                }
            }
        }
        named_bar_sync(2 + h, W * 32);
        if (sub == 0) {
            for (int j = 0; j < W - 1; ++j) {
                const float* ox_base = head_x + j * G * (kHeadDim + 4);
#pragma unroll
                for (int gg = 0; gg < G; ++gg) {
                    const float4 ox = *reinterpret_cast<const float4*>(ox_base + gg * (kHeadDim + 4) + 4 * dg);
                    const float mx = ox_base[gg * (kHeadDim + 4) + kHeadDim];
                    const float lx = ox_base[gg * (kHeadDim + 4) + kHeadDim + 1];
                    const float mn = fmaxf(M[gg], mx);
                    const float mu = (mn == -INFINITY) ? 0.f : mn;
                    const float wa = ex2(M[gg] - mu), wb = ex2(mx - mu);
                    lp[gg] = lp[gg] * wa + lx * wb;
                    o2[gg][0] = make_float2(fmaf(ox.x, wb, o2[gg][0].x * wa), fmaf(ox.y, wb, o2[gg][0].y * wa));
                    o2[gg][1] = make_float2(fmaf(ox.z, wb, o2[gg][1].x * wa), fmaf(ox.w, wb, o2[gg][1].y * wa));
                    M[gg] = mn;
                }
            }
        }
        named_bar_sync(2 + h, W * 32);  // xbuf is free again
        const bool whole = (s_begin >= gb) && (s_end <= ge);
        const bool writer = (sub == 0 && lane < 16);
        if (whole) {
            if (writer) {
#pragma unroll
                for (int gg = 0; gg < G; ++gg) {
                    const float inv = lp[gg] > 0.f ? 1.f / lp[gg] : 0.f;
                    T* orow = static_cast<T*>(a.out) +
                              (static_cast<size_t>(s) * NQ + h * G + gg) * kHeadDim + 4 * dg;
                    const float x0 = o2[gg][0].x * inv, x1 = o2[gg][0].y * inv;
                    const float x2 = o2[gg][1].x * inv, x3 = o2[gg][1].y * inv;
                    if constexpr (sizeof(T) == 2)
                        *reinterpret_cast<uint2*>(orow) =
                            make_uint2(float2_to_bf16x2(x0, x1), float2_to_bf16x2(x2, x3));
                    else
                        *reinterpret_cast<float4*>(orow) = make_float4(x0, x1, x2, x3);
                }
            }
        } else {
            const int slot = (s_begin < gb) ? 2 * cta : 2 * cta + 1;
            if (writer) {
#pragma unroll
                for (int gg = 0; gg < G; ++gg) {
                    const size_t row = static_cast<size_t>(slot) * NQ + h * G + gg;
                    *reinterpret_cast<float4*>(a.part_o + row * kHeadDim + 4 * dg) =
                        make_float4(o2[gg][0].x, o2[gg][0].y, o2[gg][1].x, o2[gg][1].y);
                    if (lane == 0)
                        *reinterpret_cast<float2*>(a.part_ml + row * 2) = make_float2(M[gg], lp[gg]);
                }
                __threadfence();
            }
            named_bar_sync(1, NCONS);
            if (threadIdx.x == 0) misc[0] = atomicAdd(a.counters + s, 1);
            named_bar_sync(1, NCONS);
            // Contributors: the CTAs whose slice holds a page of s.  With at
            // least one page per CTA (total >= grid) they are c_first..c_last;
            // with fewer pages than CTAs some slices are empty and each page
            // has a CTA of its own, so page s_begin + i belongs to contributor i.
            const int c_first = cta_of(s_begin, grid, total);
            const bool dense = total >= grid;
            const int n_contrib = dense ? cta_of(s_end - 1, grid, total) - c_first + 1 : s_end - s_begin;
            if (misc[0] == n_contrib - 1) {  // last contributor merges the splits
                __threadfence();
                auto slot_of = [&](int i) {
                    const int c = dense ? c_first + i : cta_of(s_begin + i, grid, total);
                    return (c == c_first) ? 2 * c + 1 : 2 * c;
                };
                // One warp folds a head's partial rows (256 bytes each, lane l
                // takes dims 2l, 2l+1) with an online max, kMergeBatch rows in
                // flight.  With fewer heads than warps, kWpq warps share a head
                // (strided over the splits) and combine through xbuf.
                constexpr int kWpq = NQ >= NCW ? 1 : NCW / NQ;
                auto fold = [&](int qh, int first, int step, float& Mr, float& Lr, float2& Or) {
                    Mr = -INFINITY;
                    Lr = 0.f;
                    Or = make_float2(0.f, 0.f);
                    for (int i0 = first; i0 < n_contrib; i0 += step * kMergeBatch) {
                        float2 ml[kMergeBatch], ov[kMergeBatch];
#pragma unroll
                        for (int u = 0; u < kMergeBatch; ++u) {
                            const int i = i0 + u * step;
                            if (i < n_contrib) {
                                const size_t row = static_cast<size_t>(slot_of(i)) * NQ + qh;
                                ml[u] = __ldcg(reinterpret_cast<const float2*>(a.part_ml + row * 2));
                                ov[u] = __ldcg(reinterpret_cast<const float2*>(a.part_o + row * kHeadDim) + lane);
                            } else {
                                ml[u] = make_float2(-INFINITY, 0.f);
                                ov[u] = make_float2(0.f, 0.f);
                            }
                        }
                        float bm = Mr;
#pragma unroll
                        for (int u = 0; u < kMergeBatch; ++u) bm = fmaxf(bm, ml[u].x);
                        const float mu = (bm == -INFINITY) ? 0.f : bm;
                        const float sc = ex2(Mr - mu);
                        Lr *= sc;
                        Or = make_float2(Or.x * sc, Or.y * sc);
#pragma unroll
                        for (int u = 0; u < kMergeBatch; ++u) {
                            const float w = ex2(ml[u].x - mu);
                            Lr = fmaf(ml[u].y, w, Lr);
                            Or = make_float2(fmaf(ov[u].x, w, Or.x), fmaf(ov[u].y, w, Or.y));
                        }
                        Mr = bm;
                    }
                };
                auto write_out = [&](int qh, float Lr, float2 Or) {
                    const float inv = Lr > 0.f ? 1.f / Lr : 0.f;
                    T* orow = static_cast<T*>(a.out) + (static_cast<size_t>(s) * NQ + qh) * kHeadDim + 2 * lane;
                    if constexpr (sizeof(T) == 2)
                        *reinterpret_cast<uint32_t*>(orow) = float2_to_bf16x2(Or.x * inv, Or.y * inv);
                    else
                        *reinterpret_cast<float2*>(orow) = make_float2(Or.x * inv, Or.y * inv);
                };
                if constexpr (kWpq == 1) {
                    for (int qh = warp; qh < NQ; qh += NCW) {
                        float Mr, Lr;
                        float2 Or;
                        fold(qh, 0, 1, Mr, Lr, Or);
                        write_out(qh, Lr, Or);
                    }
                } else {
                    const int qh = warp / kWpq, part = warp % kWpq;
                    float* st = xbuf + warp * (kHeadDim + 2);  // [NCW][64 + 2]
                    if (qh < NQ) {
                        float Mr, Lr;
                        float2 Or;
                        fold(qh, part, kWpq, Mr, Lr, Or);
                        *reinterpret_cast<float2*>(st + 2 * lane) = Or;
                        if (lane == 0) {
                            st[kHeadDim] = Mr;
                            st[kHeadDim + 1] = Lr;
                        }
                    }
                    named_bar_sync(1, NCONS);
                    if (warp < NQ) {
                        float Mr = -INFINITY;
                        for (int p = 0; p < kWpq; ++p) Mr = fmaxf(Mr, xbuf[(warp * kWpq + p) * (kHeadDim + 2) + kHeadDim]);
                        const float mu = (Mr == -INFINITY) ? 0.f : Mr;
                        float Lr = 0.f;
                        float2 Or = make_float2(0.f, 0.f);
                        for (int p = 0; p < kWpq; ++p) {
                            const float* sp = xbuf + (warp * kWpq + p) * (kHeadDim + 2);
                            const float w = ex2(sp[kHeadDim] - mu);
                            Lr = fmaf(sp[kHeadDim + 1], w, Lr);
                            const float2 o = *reinterpret_cast<const float2*>(sp + 2 * lane);
                            Or = make_float2(fmaf(o.x, w, Or.x), fmaf(o.y, w, Or.y));
                        }
                        write_out(warp, Lr, Or);
                    }
                }
                if (threadIdx.x == 0) a.counters[s] = 0;
            }
            named_bar_sync(1, NCONS);  // misc[0] is read by all before the next flush
        }
        if (g < ge) s = find_seq(pstart, n, g);
    }
    cp_async_wait<0>();  // a staged append skipped after a failed wait
    // Warp 0: do not leave while a copy issued here may still be landing.  A
    // stage is reused only after its previous page was handed back, so the
    // last page issued into each stage covers every copy in flight.
    if (warp == 0 && lane == 0) {
        for (int st = 0; st < STAGES && st < issued; ++st) {
            const int last = st + ((issued - 1 - st) / STAGES) * STAGES;
            mbar_wait(&full[st], static_cast<uint32_t>(last / STAGES) & 1u);
        }
    }
}
// ---------------------------------------------------------------------------
// Host side: one entry per compiled (dtype, n_kv, group) shape.
struct DecodeVariant {
    int dtype, nkv, group;
    const void* fn;
    size_t (*smem)(int);
    int threads;
};

template <typename T, int NKV, int G, int STAGES>
DecodeVariant make_variant(int dtype) {
    using S = DecodeShape<T, NKV, G, STAGES>;
    return DecodeVariant{dtype, NKV, G, reinterpret_cast<const void*>(&decode_kernel<T, NKV, G, STAGES>),
                         &S::smem_bytes, S::kThreads};
}

const DecodeVariant* find_variant(int dtype, int nkv, int group) {
    static const DecodeVariant table[] = {
        make_variant<__nv_bfloat16, 8, 3, 6>(KV_DTYPE_BF16),
        make_variant<__nv_bfloat16, 8, 4, 6>(KV_DTYPE_BF16),
        make_variant<__nv_bfloat16, 1, 4, 32>(KV_DTYPE_BF16),  // 32q/8kv split over 8 GPUs by KV head
        make_variant<__nv_bfloat16, 2, 4, 16>(KV_DTYPE_BF16),  // ... over 4 GPUs
        make_variant<__nv_bfloat16, 4, 4, 8>(KV_DTYPE_BF16),   // ... over 2 GPUs
        make_variant<float, 8, 3, 2>(KV_DTYPE_F32),
        make_variant<float, 8, 4, 2>(KV_DTYPE_F32),
        make_variant<float, 1, 4, 16>(KV_DTYPE_F32),
        make_variant<float, 2, 4, 8>(KV_DTYPE_F32),
        make_variant<float, 4, 4, 4>(KV_DTYPE_F32),
    };
    for (const auto& v : table)
        if (v.dtype == dtype && v.nkv == nkv && v.group == group) return &v;
    return nullptr;
}


}  // namespace

// A kernel's dynamic shared-memory limit is one attribute per device, shared
// by every pool and caller that launches it.  It only ever grows here, to the
// largest size any of them needs, so setting up a pool with a smaller
// workspace never breaks the launches of one created earlier.
int raise_smem_limit(const void* fn, int device, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> current;
    std::lock_guard<std::mutex> lock(mu);
    size_t& cur = current[{fn, device}];
    if (bytes <= cur) return KV_OK;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
        cudaSuccess)
        return KV_ERR_CUDA;
    cur = bytes;
    return KV_OK;
}

int decode_setup(kv_pool* pool) {
    const auto& c = pool->cfg;
    if (is_half_page(c.dtype) || is_quant(c.dtype)) return decode_tc_setup(pool);
    const DecodeVariant* v = find_variant(c.dtype, c.n_kv_heads, c.n_q_heads / c.n_kv_heads);
    if (!v) return KV_ERR_UNSUPPORTED;
    const size_t smem = v->smem(c.max_seqs);
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c.device) != cudaSuccess)
        return KV_ERR_CUDA;
    if (smem > static_cast<size_t>(optin)) return KV_ERR_INVALID;  // max_seqs too large
    if (raise_smem_limit(v->fn, c.device, smem) != KV_OK) return KV_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v->fn, v->threads, smem) !=
            cudaSuccess ||
        per_sm < 1)
        return KV_ERR_CUDA;
    pool->decode_grid = pool->sm_count * per_sm;
    pool->decode_smem = smem;
    return KV_OK;
}

// Partial rows: two per CTA; the tensor-core kernel (bf16, f16 and quantised pools) keeps two
// more per CTA for the run partials of a long sequence's two-level merge.
size_t decode_workspace_slots(const kv_pool* pool) {
    return (pool->cfg.dtype == KV_DTYPE_F32 ? 2 : 4) * static_cast<size_t>(pool->decode_grid);
}

// Merge counters: one per sequence, then two per CTA for the runs.
size_t decode_counter_count(const kv_pool* pool) {
    return static_cast<size_t>(pool->cfg.max_seqs) + 2 * static_cast<size_t>(pool->decode_grid);
}

int launch_decode(kv_pool* pool, const void* q, const uint32_t* bt, int32_t bt_stride,
                  const int32_t* seq_lens, int32_t n_seqs, int32_t window, void* out,
                  cudaStream_t stream, const void* new_k, const void* new_v, const float* q_norm,
                  const float* k_norm, float eps) {
    const auto& c = pool->cfg;
    if (is_half_page(c.dtype))
        return launch_decode_tc(pool, q, bt, bt_stride, seq_lens, n_seqs, window, out, stream, new_k, new_v, q_norm,
                                k_norm, eps);
    if (is_quant(c.dtype)) {
        // The append (k RMSNorm, RoPE, quantise on store) and the attention
        // (with the q RMSNorm) as two launches.
        if (new_k != nullptr) {
            const int rc = launch_append(pool, new_k, new_v, nullptr, nullptr, nullptr, seq_lens, n_seqs, n_seqs, bt,
                                         bt_stride, stream, k_norm, eps);
            if (rc != KV_OK) return rc;
        }
        return launch_decode_tc(pool, q, bt, bt_stride, seq_lens, n_seqs, window, out, stream, nullptr, nullptr,
                                q_norm, nullptr, eps);
    }
    const DecodeVariant* v = find_variant(c.dtype, c.n_kv_heads, c.n_q_heads / c.n_kv_heads);
    if (!v) return KV_ERR_UNSUPPORTED;
    DecodeArgs a;
    a.q = q;
    a.out = out;
    a.bt = bt;
    a.bt_stride = bt_stride;
    a.seq_lens = seq_lens;
    a.n_seqs = n_seqs;
    a.window = window;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.part_o = pool->part_o;
    a.part_ml = pool->part_ml;
    a.counters = pool->counters;
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    a.new_k = new_k;
    a.new_v = new_v;
    a.pages = pool->pages;
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.eps = eps;
    void* args[] = {&pool->page_map, &a};
    const cudaError_t e = cudaLaunchKernel(v->fn, dim3(pool->decode_grid), dim3(v->threads), args,
                                           pool->decode_smem, stream);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

// ---- decode on caller-supplied workspace (the allocation-free entry point) ----
int decode_configure_raw(int dtype, int nkv, int group, int max_seqs, int device, int sm_count,
                         int* grid, size_t* smem) {
    const DecodeVariant* v = find_variant(dtype, nkv, group);
    if (!v) return KV_ERR_UNSUPPORTED;
    const size_t bytes = v->smem(max_seqs);
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess)
        return KV_ERR_CUDA;
    if (bytes > static_cast<size_t>(optin)) return KV_ERR_INVALID;
    if (raise_smem_limit(v->fn, device, bytes) != KV_OK) return KV_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v->fn, v->threads, bytes) != cudaSuccess ||
        per_sm < 1)
        return KV_ERR_CUDA;
    *grid = sm_count * per_sm;
    *smem = bytes;
    return KV_OK;
}

int launch_decode_raw(const DecodeRaw& r, cudaStream_t stream) {
    const DecodeVariant* v = find_variant(r.dtype, r.nkv, r.group);
    if (!v) return KV_ERR_UNSUPPORTED;
    DecodeArgs a;
    a.q = r.q;
    a.out = r.out;
    a.bt = r.bt;
    a.bt_stride = r.bt_stride;
    a.seq_lens = r.seq_lens;
    a.n_seqs = r.n_seqs;
    a.window = r.window;
    a.rope = r.rope;
    a.max_pos = r.max_pos;
    a.n_pages = r.n_pages;
    a.part_o = r.part_o;
    a.part_ml = r.part_ml;
    a.counters = r.counters;
    a.err = r.err;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(kHeadDim)));
    a.new_k = nullptr;
    a.new_v = nullptr;
    a.pages = nullptr;
    a.q_norm = nullptr;
    a.k_norm = nullptr;
    a.eps = 0.f;
    CUtensorMap map = *r.map;
    void* args[] = {&map, &a};
    const cudaError_t e = cudaLaunchKernel(v->fn, dim3(r.grid), dim3(v->threads), args, r.smem, stream);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
