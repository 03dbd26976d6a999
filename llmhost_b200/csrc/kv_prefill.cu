// kv_prefill.cu -- chunked-prefill and tree-verify attention on tcgen05 (bf16).
//
// Replaces attention_forward (crates/llm-engine/src/lfm2.rs:1058-1111) for a
// chunk of T new tokens appended after L cached ones, the case the reference
// lacks (attn_prefill always starts at position 0, lfm2.rs:730).  Query token
// i (chunk-relative) sees cached key s < L, and chunk key L + j when j <= i
// (causal chunk) or, for a speculative tree, when bit j of its
// ancestor-or-self mask is set.  The chunk's K/V must already be in pages.
//
// One CTA per (sequence, kv head, 2 x 128 query rows); a row is a (token,
// query head of the group) pair.  Keys are consumed in blocks of 128 (8 pages).
// Roles:
//   warps 0-15  softmax, two threads per row: warps 8t..8t+7 own tile t, warp
//               8t + 4h + q rows 32q..32q+31 and keys 64h..64h+63 of each
//               block (TMEM lane quarter q); the halves of a row agree on the
//               block maximum through shared memory
//   warp 16     TMA producer: per page one {64 x 16} bf16 box of K and one of
//               V for this kv head (128-byte swizzle, no multicast) into a
//               4-stage ring
//   warp 17     TMEM owner; one thread issues the tensor-core MMAs:
//                 S_t  = Q_t K^T : M 128, N 128, K 64; Q_t and K K-major in
//                                  shared memory; fp32 S_t in TMEM
//                 O_t += P_t V   : M 128, N 64, K 128; P_t (bf16) in TMEM, V
//                                  MN-major straight from the page layout
// TMEM per tile (256 columns): S_t [0, 128), P_t [128, 192), O_t [192, 256).
// The softmax writes P_t group by group while it sweeps S_t.
//
// Softmax (log2 units: q is pre-scaled by log2(e)/sqrt(d)) keeps a per-row
// reference maximum m: P = 2^(S - m) is computed in the same pass that finds
// the block maximum, and only when a block maximum exceeds m by more than
// kLazyLog2 is m raised, O (in TMEM) and the row sum rescaled and P redone.
// P therefore stays below 2^kLazyLog2.  Pages past the sequence load as
// out-of-range boxes (zero fill).
#include <algorithm>
#include <cmath>

#include "kv_common.cuh"
#include "kv_pool_impl.h"
#include "kv_tc.cuh"

namespace kvb200 {
namespace {

constexpr int kRows = 128;                                // MMA M: query rows per tile
constexpr int kTiles = 2;                                 // query tiles per CTA
constexpr int kBlockKeys = 128;                           // keys per block (MMA N of S, K of PV)
constexpr int kPagesPerBlock = kBlockKeys / kPageTokens;  // 8
constexpr int kStages = 4;                                // K/V block ring
constexpr int kKvBytes = kBlockKeys * 128;                // 16 KiB: K (or V) of one block
constexpr int kSliceBytes = kPageTokens * 128;            // one page's K (or V) rows of one head
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTileCols = 256;                       // TMEM columns per tile
constexpr uint32_t kColP = 128, kColO = 192;              // within a tile; S at 0
constexpr int kHalves = 2;                                // softmax threads per row
constexpr int kHalfKeys = kBlockKeys / kHalves;           // keys of a block one thread sweeps
constexpr int kTileThreads = kRows * kHalves;             // softmax threads of one tile
constexpr int kSoftmaxThreads = kTiles * kTileThreads;    // warps 0-15
constexpr int kProducerWarp = kSoftmaxThreads / 32;       // warp 16: TMA
constexpr int kMmaWarp = kProducerWarp + 1;               // warp 17: TMEM owner, MMA issue
constexpr int kThreads = kSoftmaxThreads + 64;

// smem: Q tiles (128 rows x 128 B, 128-byte swizzle), the K/V ring (stage st:
// K at +0, V at +kKvBytes), then the barriers
constexpr int kQBytes = kRows * 128;
constexpr int kStageBytes = 2 * kKvBytes;
constexpr int kOffStage = kTiles * kQBytes;
constexpr int kOffBar = kOffStage + kStages * kStageBytes;
// float [3][kTiles][kHalves][kRows]: half-row maxima (slots 0, 1 by block
// parity) and half-row sums (slot 2) passed between the halves of a row
constexpr int kOffX = kOffBar + 256;
constexpr int kXBytes = 3 * kTiles * kHalves * kRows * 4;
// The CTA's work list: segments of units (see Seg), then its length and the
// merge flag
constexpr int kMaxSegs = 512;
constexpr int kOffSeg = kOffX + kXBytes;
constexpr int kOffSegN = kOffSeg + kMaxSegs * 32;
// persistent-grid set-up: each unit's visible key count and the inclusive
// prefix of the unit costs (64-bit), warp totals, and the parts this CTA
// merges at its end
constexpr int kOffScan = kOffSegN + 64;
constexpr int kScanBytes = kMaxSegs * 4 + kMaxSegs * 8 + 16 * 8 + 64;
constexpr int kSmemBytes = 1024 + kOffScan + kScanBytes;

// Work schedule.  A unit is one (sequence, kv head, pair of query tiles),
// the work of one CTA of the plain grid: its query rows against key blocks
// 0 .. nb-1.  With more units than SMs (and at most kPersistMaxUnits), the
// grid is persistent instead: the units' key blocks are laid end to end, each
// unit led by kLeadBlocks blocks of no work that stand for the cost of
// starting it (its Q tiles, the pipeline restart, its epilogue), and every
// CTA takes an equal run of that list.  A unit cut between CTAs is computed
// in parts; each part leaves its rows' unnormalised sums (reference maximum,
// row sum, O) in the pool's prefill workspace and the last part to arrive
// merges them (log-sum-exp of the parts, Milakov & Gimelshein 2018).
constexpr int kLeadBlocks = 1;
constexpr int kPersistMaxUnits = kMaxSegs;
constexpr int kPartRows = kTiles * kRows;                        // rows of a unit
constexpr size_t kSlotFloats = static_cast<size_t>(kPartRows) * (kHeadDim + 2);  // O rows, then (m, l) pairs
constexpr int kMergeBar = 3;                                     // named barrier of all softmax threads

// P entries stay below 2^kLazyLog2 times the row's reference maximum; the
// reference is raised only when a block's maximum exceeds it by more.
constexpr float kLazyLog2 = 8.f;

// One entry of a CTA's work list: unit u's key blocks [b0, b1) of nb, kmax
// its last visible key + 1; the unit's parts are computed by CTAs c_first ..
// c_first + n_parts - 1 (n_parts = 1: this CTA does the whole unit).
struct Seg {
    int u, b0, b1, nb, kmax, c_first, n_parts, pad;
};

struct PrefillArgs {
    const __nv_bfloat16* q;
    const int32_t* q_pos;
    const int32_t* q_off;
    const int32_t* prefix;
    const unsigned long long* tree;
    const uint32_t* bt;
    long long bt_stride;
    long long bt_cols;  // entries of a row from bt on (bt_stride, less the shared pages in the suffix pass)
    int n_q, nkv, group, tile_tokens, max_q;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    int page_rows;
    __nv_bfloat16* out;
    int* err;
    float qscale;
    int nx;           // query-tile pairs per (sequence, kv head)
    int n_seqs;
    int persist;      // 1: persistent grid over the unit list (gridDim.x CTAs)
    float* part;      // persistent: [2 gridDim.x][kSlotFloats] partial rows
    int* counters;    // persistent: [units] parts arrived (reset by the merger)
    // Shared-prefix (cascade) passes; row R = token * n_q + query head.
    int virt;         // 1: the prefix pass, one sequence of every token of the batch
    int virt_L;       //    (q_off[n_seqs] tokens) against the first virt_L keys of table row 0 only
    float* pout;      // non-null: rows written as (O [R][64] unnormalised, then (m, l) [R]) instead of out
    const float* pin; // non-null: rows merged with such partial rows before out is written
    long long prow_total;  // rows of pout / pin
    int L_off;        // the suffix pass: tokens of the shared prefix, left out of every prefix length
};

// Where unit u's rows are and which keys they can see.
struct UnitInfo {
    int s, h, q0, T, L, t_begin, t_end, kmax, nb;
    bool bad;  // sequence lengths out of range
};

__device__ __forceinline__ UnitInfo unit_info(const PrefillArgs& a, int u) {
    UnitInfo r;
    const int x = u % a.nx;
    r.h = (u / a.nx) % a.nkv;
    r.s = u / (a.nx * a.nkv);
    const bool tree = a.tree != nullptr;
    if (a.virt) {  // every token of the batch, the shared keys only
        r.s = 0;
        r.q0 = 0;
        r.T = __ldg(a.q_off + a.n_seqs);
        r.L = a.virt_L;
        r.bad = r.T < 0 || r.L < 0 || r.T > a.max_q;  // max_q: n_seqs x the per-sequence bound
    } else {
        r.q0 = __ldg(a.q_off + r.s);
        r.T = __ldg(a.q_off + r.s + 1) - r.q0;
        r.L = __ldg(a.prefix + r.s) - a.L_off;
        r.bad = r.T < 0 || r.L < 0 || r.T > a.max_q || (tree && r.T > 64);
    }
    r.t_begin = x * kTiles * a.tile_tokens;
    r.t_end = min(r.T, r.t_begin + kTiles * a.tile_tokens);
    // keys [0, kmax) can be visible to the unit
    r.kmax = a.virt ? r.L : tree ? r.L + r.T : r.L + r.t_end;
    r.nb = (r.bad || r.t_begin >= r.T) ? 0 : (r.kmax + kBlockKeys - 1) / kBlockKeys;
    return r;
}

// The CTA (of G) whose run of the unit list [c C / G, (c + 1) C / G) holds
// position p.
__device__ __forceinline__ int cta_of(long long p, long long C, long long G) {
    return static_cast<int>(((p + 1) * G + C - 1) / C - 1);
}

__device__ __forceinline__ int unit_cost(int kmax) {
    return kmax > 0 ? (kmax + kBlockKeys - 1) / kBlockKeys + kLeadBlocks : 0;
}

// This CTA's run of the persistent grid's unit list (one thread): the units'
// costs are laid end to end (prefix[u]: inclusive, 64-bit), the list of C
// positions is cut into G equal runs, and every unit whose work positions
// meet this CTA's run becomes a segment.  With C >= G every run holds at
// least one position, so the CTAs between a unit's first and last part all
// hold a part of it; with fewer positions than CTAs only the first C CTAs
// take one each.
__device__ int cut_run(int n_units, const int* ukmax, const long long* prefix, Seg* segs) {
    const long long C = n_units > 0 ? prefix[n_units - 1] : 0;
    const long long G = C < gridDim.x ? C : gridDim.x, c = blockIdx.x;
    if (c >= G) return 0;
    const long long gb = c * C / G, ge = (c + 1) * C / G;
    int lo = 0, hi = n_units;  // the first unit whose positions end past gb
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] > gb)
            hi = mid;
        else
            lo = mid + 1;
    }
    int n = 0;
    for (int u = lo; u < n_units; ++u) {
        const int cost = unit_cost(ukmax[u]);
        if (cost == 0) continue;
        const long long w1 = prefix[u], w0 = w1 - cost + kLeadBlocks;  // the unit's work positions
        if (w1 - cost >= ge) break;
        const long long b = max(gb, w0), e = min(ge, w1);
        if (b < e) {
            Seg sg;
            sg.u = u;
            sg.nb = cost - kLeadBlocks;
            sg.b0 = static_cast<int>(b - w0);
            sg.b1 = static_cast<int>(e - w0);
            sg.kmax = ukmax[u];
            sg.c_first = cta_of(w0, C, G);
            sg.n_parts = cta_of(w1 - 1, C, G) - sg.c_first + 1;
            sg.pad = 0;
            segs[n++] = sg;
        }
    }
    return n;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// max(m, v[0..15])
__device__ __forceinline__ float max16(float m, const float (&v)[16]) {
    const float a = max3f(v[0], v[1], v[2]), b = max3f(v[3], v[4], v[5]), c = max3f(v[6], v[7], v[8]);
    const float d = max3f(v[9], v[10], v[11]), e = max3f(v[12], v[13], v[14]), f = max3f(v[15], m, a);
    return max3f(max3f(b, c, d), e, f);
}

// Row visibility for keys that reach the chunk.
struct RowMask {
    int L, T, t_chunk;  // cached keys, chunk length, chunk-relative token of the row
    unsigned long long bits;
    bool tree, valid;
    __device__ __forceinline__ bool visible(int key) const {
        if (!valid) return false;
        if (key < L) return true;
        if (key >= L + T) return false;
        return tree ? ((bits >> (key - L)) & 1ull) != 0 : (key - L) <= t_chunk;
    }
};

// One 32-key group g of this thread's S row (keys k0 + 32 g .. k0 + 32 g + 31):
// folds it into the block maximum bm and writes P = 2^(S - mu) as bf16 pairs
// to TMEM columns t_p + 16 g .. + 15; adds P to sum2.  Masked keys are made
// -inf in place.
__device__ __forceinline__ void group32(uint32_t (&rr)[32], int g, int k0, bool need_mask, const RowMask& rm,
                                        float mu, uint32_t t_p, float& bm, float2 (&sum2)[2]) {
    if (need_mask) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (!rm.visible(k0 + 32 * g + i)) rr[i] = __float_as_uint(-INFINITY);
    }
    float t[11];
#pragma unroll
    for (int i = 0; i < 10; ++i)
        t[i] = max3f(__uint_as_float(rr[3 * i]), __uint_as_float(rr[3 * i + 1]), __uint_as_float(rr[3 * i + 2]));
    t[10] = max3f(__uint_as_float(rr[30]), __uint_as_float(rr[31]), bm);
    bm = max3f(max3f(t[0], t[1], t[2]), max3f(t[3], t[4], t[5]), max3f(max3f(t[6], t[7], t[8]), t[9], t[10]));
    const float2 nmu = make_float2(-mu, -mu);
    uint32_t w[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 d = __fadd2_rn(make_float2(__uint_as_float(rr[2 * i]), __uint_as_float(rr[2 * i + 1])), nmu);
        const float2 p = make_float2(ex2f(d.x), ex2f(d.y));
        sum2[i & 1] = __fadd2_rn(sum2[i & 1], p);
        w[i] = float2_to_bf16x2(p.x, p.y);
    }
    tmem_st16(t_p + 16 * g, w);
}

// One pass over this thread's two 32-key groups of its S row (t_s, keys k0
// ..: its half of the block): the half's maximum and P against the
// reference mu.  Warp-collective.
__device__ __forceinline__ void sweep_s(uint32_t t_s, uint32_t t_p, int k0, bool need_mask, const RowMask& rm,
                                        float mu, float& bm, float2 (&sum2)[2]) {
    uint32_t ra[32], rb[32];
    tmem_ld32(t_s, ra);
    tmem_ld32(t_s + 32, rb);
    tmem_wait32(ra);
    group32(ra, 0, k0, need_mask, rm, mu, t_p, bm, sum2);
    tmem_wait32(rb);
    group32(rb, 1, k0, need_mask, rm, mu, t_p, bm, sum2);
}

// S values of a 16-key group as floats, masked keys at -inf.
__device__ __forceinline__ void s_group(const uint32_t (&rr)[16], int key0, bool need_mask, const RowMask& rm,
                                        float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(rr[i]);
    if (need_mask) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (!rm.visible(key0 + i)) v[i] = -INFINITY;
    }
}

// Maximum of this thread's half of its S row (rarely needed: first block
// only).  A rolled loop, to keep the instruction footprint of the softmax small.
__device__ __forceinline__ float row_max(uint32_t taddr, int k0, bool need_mask, const RowMask& rm) {
    float bm = -INFINITY;
#pragma unroll 1
    for (int g = 0; g < kHalfKeys / 16; ++g) {
        uint32_t rr[16];
        tmem_ld16(taddr + 16 * g, rr);
        tmem_wait16(rr);
        float v[16];
        s_group(rr, k0 + 16 * g, need_mask, rm, v);
        bm = max16(bm, v);
    }
    return bm;
}

// P = 2^(S - mu) of this thread's half row straight into its P columns of
// TMEM (rarely needed: a block that raised a row's reference), plus the sum.
// Rolled loop.
__device__ __forceinline__ float2 row_exp_to_tmem(uint32_t t_s, uint32_t t_p, int k0, bool need_mask,
                                                  const RowMask& rm, float mu) {
    const float2 nmu = make_float2(-mu, -mu);
    float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int g = 0; g < kHalfKeys / 16; ++g) {
        uint32_t rr[16];
        tmem_ld16(t_s + 16 * g, rr);
        tmem_wait16(rr);
        float v[16];
        s_group(rr, k0 + 16 * g, need_mask, rm, v);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 d = __fadd2_rn(make_float2(v[2 * i], v[2 * i + 1]), nmu);
            const float2 p = make_float2(ex2f(d.x), ex2f(d.y));
            sum2 = __fadd2_rn(sum2, p);
            w[i] = float2_to_bf16x2(p.x, p.y);
        }
        tmem_st8(t_p + 8 * g, w);
    }
    return sum2;
}

// This thread's half of its O row (32 fp32 columns) scaled in place in TMEM.
// Warp-collective.
__device__ __forceinline__ void scale_o(uint32_t t_o, float f) {
    const float2 f2 = make_float2(f, f);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        uint32_t x[16];
        tmem_ld16(t_o + 16 * c, x);
        tmem_wait16(x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 u = __fmul2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), f2);
            x[2 * i] = __float_as_uint(u.x);
            x[2 * i + 1] = __float_as_uint(u.y);
        }
        tmem_st16(t_o + 16 * c, x);
    }
    tmem_wait_st();
}

// A row's final sums -- reference maximum m (log2 units), row sum l and the
// unnormalised O -- to their destination: the shared-prefix partial rows
// (pout), or bf16 out after an optional merge with a partial row (pin) by the
// log-sum-exp identity.  finish_begin once per row, then finish16 for each 16
// of this thread's dims (dims 32 hf + 16 c ..).
struct RowFinish {
    float f, g, inv;  // weights of this row's O and of the pin row's; 1 / merged row sum
};

__device__ __forceinline__ RowFinish finish_begin(const PrefillArgs& a, long long row, int hf, float m, float l) {
    RowFinish rf{1.f, 0.f, 0.f};
    if (a.pout) {
        if (hf == 0) reinterpret_cast<float2*>(a.pout + a.prow_total * kHeadDim)[row] = make_float2(m, l);
        return rf;
    }
    if (a.pin) {
        const float2 ml = __ldg(reinterpret_cast<const float2*>(a.pin + a.prow_total * kHeadDim) + row);
        const float M = fmaxf(m, ml.x);
        rf.f = m == -INFINITY ? 0.f : ex2f(m - M);
        rf.g = ml.x == -INFINITY ? 0.f : ex2f(ml.x - M);
        l = l * rf.f + ml.y * rf.g;
    }
    rf.inv = l > 0.f ? 1.f / l : 0.f;
    return rf;
}

__device__ __forceinline__ void finish16(const PrefillArgs& a, long long row, int hf, int c, const RowFinish& rf,
                                         float (&o)[16], __nv_bfloat16* dst) {
    const size_t at = static_cast<size_t>(row) * kHeadDim + kHeadDim / 2 * hf + 16 * c;
    if (a.pout) {
        float4* o4 = reinterpret_cast<float4*>(a.pout + at);
#pragma unroll
        for (int i = 0; i < 4; ++i) o4[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        return;
    }
    if (a.pin) {
        const float4* p4 = reinterpret_cast<const float4*>(a.pin + at);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 v = __ldg(p4 + i);
            o[4 * i] = o[4 * i] * rf.f + v.x * rf.g;
            o[4 * i + 1] = o[4 * i + 1] * rf.f + v.y * rf.g;
            o[4 * i + 2] = o[4 * i + 2] * rf.f + v.z * rf.g;
            o[4 * i + 3] = o[4 * i + 3] * rf.f + v.w * rf.g;
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
        reinterpret_cast<uint4*>(dst)[2 * c + i] =
            make_uint4(float2_to_bf16x2(o[8 * i] * rf.inv, o[8 * i + 1] * rf.inv),
                       float2_to_bf16x2(o[8 * i + 2] * rf.inv, o[8 * i + 3] * rf.inv),
                       float2_to_bf16x2(o[8 * i + 4] * rf.inv, o[8 * i + 5] * rf.inv),
                       float2_to_bf16x2(o[8 * i + 6] * rf.inv, o[8 * i + 7] * rf.inv));
}

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap hmap,
                                                              const __grid_constant__ PrefillArgs a) {
    const bool tree = a.tree != nullptr;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kOffBar);  // [kStages]
    uint64_t* empty = full + kStages;                               // [kStages]
    uint64_t* s_full = empty + kStages;                             // [kTiles]
    uint64_t* p_full = s_full + kTiles;                             // [kTiles]
    uint64_t* pv_full = p_full + kTiles;                            // [kTiles]
    uint64_t* mma_done = pv_full + kTiles;
    uint64_t* q_full = mma_done + 1;                                // a segment's Q tiles written
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    Seg* segs = reinterpret_cast<Seg*>(base + kOffSeg);
    int* n_segs_p = reinterpret_cast<int*>(base + kOffSegN);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int t = 0; t < kTiles; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], kTileThreads);  // every softmax thread of the tile arrives
            mbar_init(&pv_full[t], 1);
        }
        mbar_init(mma_done, 1);
        mbar_init(q_full, kSoftmaxThreads);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == kProducerWarp && lane == 0) prefetch_tmap(&hmap);
    // The work list: the whole unit of this CTA (plain grid), or this CTA's
    // run of every unit's key blocks (persistent grid: each softmax thread
    // works out one unit, the costs are scanned across the 512 softmax
    // threads, thread 0 cuts the run).
    int* ukmax = reinterpret_cast<int*>(base + kOffScan);                 // [kMaxSegs]
    long long* uprefix = reinterpret_cast<long long*>(ukmax + kMaxSegs);   // [kMaxSegs]
    long long* wsum = uprefix + kMaxSegs;                                   // [16]
    int* pend = reinterpret_cast<int*>(wsum + 16);                          // [4] segments to merge, then count
    if (a.persist) {
        if (threadIdx.x < kSoftmaxThreads) {
            const int n_units = a.nx * a.nkv * (a.virt ? 1 : a.n_seqs);  // the prefix pass: one sequence
            const int u = threadIdx.x;
            int km = 0;
            if (u < n_units) {
                const UnitInfo ui = unit_info(a, u);
                km = ui.nb > 0 ? ui.kmax : 0;
                if (ui.bad && blockIdx.x == 0 && u % (a.nx * a.nkv) == 0) flag_error(a.err, kDevErrBadArg);
            }
            ukmax[u] = km;
            long long incl = unit_cost(km);
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const long long t = __shfl_up_sync(0xffffffffu, incl, d);
                if (lane >= d) incl += t;
            }
            if (lane == 31) wsum[warp] = incl;
            named_bar_sync(kMergeBar, kSoftmaxThreads);
            if (warp == 0) {
                long long x = lane < kSoftmaxThreads / 32 ? wsum[lane] : 0;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const long long t = __shfl_up_sync(0xffffffffu, x, d);
                    if (lane >= d) x += t;
                }
                if (lane < kSoftmaxThreads / 32) wsum[lane] = x;
            }
            named_bar_sync(kMergeBar, kSoftmaxThreads);
            uprefix[u] = incl + (warp > 0 ? wsum[warp - 1] : 0);
            named_bar_sync(kMergeBar, kSoftmaxThreads);
            if (threadIdx.x == 0) {
                *n_segs_p = cut_run(n_units, ukmax, uprefix, segs);
                pend[3] = 0;
            }
        }
    } else if (threadIdx.x == 0) {
        const int u = (blockIdx.z * a.nkv + blockIdx.y) * a.nx + blockIdx.x;
        const UnitInfo ui = unit_info(a, u);
        if (ui.bad && blockIdx.x == 0 && blockIdx.y == 0) flag_error(a.err, kDevErrBadArg);
        int n = 0;
        if (ui.nb > 0) {
            segs[0] = Seg{u, 0, ui.nb, ui.nb, ui.kmax, 0, 1, 0};
            n = 1;
        }
        *n_segs_p = n;
        pend[3] = 0;
    }
    tc_fence_before();
    __syncthreads();  // the TMEM address, the barriers and the work list are published
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_segs = *n_segs_p;

    if (warp == kProducerWarp) {
        // ---------------- producer: K/V head slices, 8 pages per block ----------------
        // Lane i < 8 owns page i of every block: its block-table entry for the
        // next block (which may be the next segment's first) is loaded while
        // this block's stage is waited for, and it issues that page's K and V
        // boxes (lane 0 first sets the stage's expected bytes), so no copy
        // waits on a serial chain of loads.
        const int total_rows = static_cast<int>(a.n_pages) * a.page_rows;
        // page pi of the segment's sequence holds keys its unit can see
        auto used = [&](int k, int j) {
            return lane < kPagesPerBlock && (j * kPagesPerBlock + lane) * kPageTokens < segs[k].kmax;
        };
        auto seq_of = [&](int k) { return segs[k].u / (a.nx * a.nkv); };
        auto entry = [&](int k, int j) -> uint32_t {
            const int pi = j * kPagesPerBlock + lane;
            if (!used(k, j)) return 0u;
            return pi < a.bt_cols ? __ldg(a.bt + static_cast<size_t>(seq_of(k)) * a.bt_stride + pi) : kPageNone;
        };
        int issued = 0, J = 0;
        int k = 0, j = n_segs > 0 ? segs[0].b0 : 0;
        uint32_t next = n_segs > 0 ? entry(0, j) : 0u;
        while (k < n_segs) {
            const int st = J % kStages;
            const uint32_t phys = next;
            const int ck = k, cj = j;
            if (++j == segs[k].b1 && ++k < n_segs) j = segs[k].b0;
            if (k < n_segs) next = entry(k, j);  // in flight during the wait below
            bool ok = true;
            if (lane == 0 && J >= kStages)
                ok = wait_bar(&empty[st], static_cast<uint32_t>(J / kStages - 1) & 1u, abort_flag, a.err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            if (lane == 0) mbar_arrive_expect_tx(&full[st], kStageBytes);
            __syncwarp();
            if (lane < kPagesPerBlock) {
                const int h = (segs[ck].u / a.nx) % a.nkv;
                uint8_t* kt = base + kOffStage + st * kStageBytes;
                int rk = total_rows, rv = total_rows;  // out of range: zero fill
                if (used(ck, cj)) {
                    if (phys < a.n_pages) {
                        rk = static_cast<int>(phys) * a.page_rows + h * kPageTokens;
                        rv = static_cast<int>(phys) * a.page_rows + (a.nkv + h) * kPageTokens;
                    } else {
                        flag_error(a.err, kDevErrBadPage);
                    }
                }
                tma_load_2d(kt + lane * kSliceBytes, &hmap, &full[st], 0, rk);
                tma_load_2d(kt + kKvBytes + lane * kSliceBytes, &hmap, &full[st], 0, rv);
            }
            issued = ++J;
        }
        if (lane == 0 && *abort_flag) {  // wait (bounded) for the newest copy issued into each stage
            for (int st = 0; st < kStages && st < issued; ++st) {
                const int last = st + ((issued - 1 - st) / kStages) * kStages;
                mbar_wait(&full[st], static_cast<uint32_t>(last / kStages) & 1u);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (one thread) ----------------
        // Per block J (counted over all segments) and tile t: O_t += P_t(J-1)
        // V(J-1) once P_t(J-1) is written, then S_t(J).  tcgen05.mma executes in
        // issue order, so when S_t(J) completes P_t(J-1) V(J-1) has too: the
        // softmax may then overwrite P_t and rescale O_t.  The K/V stage of
        // block J-1 is released after the last tile's PV.  A segment's first S
        // waits for its Q tiles; its first P V starts O afresh, which the
        // softmax threads allow only after the previous segment's epilogue has
        // read O (they arrive on p_full for that block after it).
        if (lane == 0) {
            constexpr uint32_t kIdescS = instr_desc(kBlockKeys, kRows, false);
            constexpr uint32_t kIdescPV = instr_desc(kHeadDim, kRows, true);
            const uint32_t q_addr = smem_addr(base);
            const uint32_t stage_addr = smem_addr(base + kOffStage);
            int J = 0;
            bool prev_first = false;  // block J-1 opened its segment (its P V starts O)
            bool ok = true;
            auto issue_pv = [&](int t, int pst) {
                const uint32_t tt = tmem + kTileCols * t;
                const uint32_t v_addr = stage_addr + pst * kStageBytes + kKvBytes;
#pragma unroll
                for (int kk = 0; kk < kBlockKeys / 16; ++kk)
                    mma_ts(tt + kColO, tt + kColP + 8 * kk, smem_desc(v_addr + 2048 * kk, kKvBytes, 1024), kIdescPV,
                           !prev_first || kk > 0);
                mma_commit(&pv_full[t]);
            };
            for (int k = 0; ok && k < n_segs; ++k) {
                const int b0 = segs[k].b0, b1 = segs[k].b1;
                for (int j = b0; j < b1; ++j, ++J) {
                    const int st = J % kStages, pst = (J + kStages - 1) % kStages;
                    if (j == b0) {
                        // A segment's first block: the previous segment's last P V
                        // goes first (its epilogue waits for it), then the new Q
                        // tiles are waited for.
                        for (int t = 0; J > 0 && t < kTiles; ++t) {
                            if (!wait_bar(&p_full[t], static_cast<uint32_t>(J - 1) & 1u, abort_flag, a.err)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            issue_pv(t, pst);
                        }
                        if (!ok || !wait_bar(q_full, static_cast<uint32_t>(k) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                    }
                    if (!wait_bar(&full[st], static_cast<uint32_t>(J / kStages) & 1u, abort_flag, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int t = 0; t < kTiles; ++t) {
                        if (J > 0 && j > b0) {
                            if (!wait_bar(&p_full[t], static_cast<uint32_t>(J - 1) & 1u, abort_flag, a.err)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            issue_pv(t, pst);
                        }
                        const uint32_t tt = tmem + kTileCols * t;
                        const uint32_t k_addr = stage_addr + st * kStageBytes;
                        const uint32_t qa = q_addr + t * kQBytes;
#pragma unroll
                        for (int kk = 0; kk < kHeadDim / 16; ++kk)
                            mma_ss(tt, smem_desc(qa + 32 * kk, 16, 1024), smem_desc(k_addr + 32 * kk, 16, 1024), kIdescS,
                                   kk > 0);
                        mma_commit(&s_full[t]);
                    }
                    if (!ok) break;
                    if (J > 0) mma_commit(&empty[pst]);
                    prev_first = j == b0;
                }
            }
            if (ok && J > 0) {  // the last block's P V
                const int pst = (J - 1) % kStages;
                for (int t = 0; t < kTiles; ++t) {
                    if (!wait_bar(&p_full[t], static_cast<uint32_t>(J - 1) & 1u, abort_flag, a.err)) break;
                    tc_fence_after();
                    issue_pv(t, pst);
                }
                mma_commit(&empty[pst]);
            }
            // Every MMA issued above has finished before TMEM is released.
            mma_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else {
        // ---------------- softmax: thread (tq, hf, r) owns half hf of row r of tile tq ----------------
        // Row r of tile tq of a unit is (token t_begin + tq * tile_tokens + r / G,
        // head h*G + r % G).
        const int tq = (warp >> 3) & 1, hf = (warp >> 2) & 1, r = 32 * (warp & 3) + lane;
        const int rt = r / a.group, rg = r % a.group;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        const uint32_t t_tile = lane_base + kTileCols * tq;  // this thread's row of its tile
        // Q tiles of segment k: RoPE at q_pos (rope.rs:76 form), scaled into
        // log2 units, bf16, into shared memory; each half builds half of the
        // row's dims.  Then every softmax thread arrives on q_full.  Its
        // indices are worked out here again, so that none stays live through
        // the block loop.
        auto build_q = [&](int k) {
            const int w = threadIdx.x >> 5, tq = (w >> 3) & 1, hf = (w >> 2) & 1, r = 32 * (w & 3) + (threadIdx.x & 31);
            const int rt = r / a.group, rg = r % a.group;
            uint8_t* qrow = base + tq * kQBytes + r * 128;
            const UnitInfo ui = unit_info(a, segs[k].u);
            const int t_row = ui.t_begin + tq * a.tile_tokens + rt;
            if (rt < a.tile_tokens && t_row < ui.t_end) {
                const uint4* src = reinterpret_cast<const uint4*>(
                    a.q + (static_cast<size_t>(ui.q0 + t_row) * a.n_q + ui.h * a.group + rg) * kHeadDim);
                int pos = __ldg(a.q_pos + ui.q0 + t_row);
                if (pos < 0 || pos >= a.max_pos) {
                    flag_error(a.err, kDevErrBadPos);
                    pos = 0;
                }
                const float2* cs = a.rope + static_cast<size_t>(pos) * (kHeadDim / 2);
                // dims 8c .. 8c+7 rotate together with dims 32+8c .. 32+8c+7; this
                // half takes c = 2 hf, 2 hf + 1
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int c = 2 * hf + cc;
                    const uint4 u0 = __ldg(src + c), u1 = __ldg(src + c + 4);
                    const uint32_t w0[4] = {u0.x, u0.y, u0.z, u0.w}, w1[4] = {u1.x, u1.y, u1.z, u1.w};
                    uint32_t lo[4], hi[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 x = bf16x2_to_float2(w0[i]), y = bf16x2_to_float2(w1[i]);
                        const float2 c0 = __ldg(cs + 8 * c + 2 * i), c1 = __ldg(cs + 8 * c + 2 * i + 1);
                        const float a0 = __fadd_rn(__fmul_rn(x.x, c0.x), __fmul_rn(-y.x, c0.y)) * a.qscale;
                        const float a1 = __fadd_rn(__fmul_rn(x.y, c1.x), __fmul_rn(-y.y, c1.y)) * a.qscale;
                        const float b0 = __fadd_rn(__fmul_rn(y.x, c0.x), __fmul_rn(x.x, c0.y)) * a.qscale;
                        const float b1 = __fadd_rn(__fmul_rn(y.y, c1.x), __fmul_rn(x.y, c1.y)) * a.qscale;
                        lo[i] = float2_to_bf16x2(a0, a1);
                        hi[i] = float2_to_bf16x2(b0, b1);
                    }
                    *reinterpret_cast<uint4*>(qrow + ((c ^ (r & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4*>(qrow + (((c + 4) ^ (r & 7)) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                }
            } else {
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {
                    const int c = 2 * hf + (cc & 1) + 4 * (cc >> 1);  // 16-byte chunks 2hf, 2hf+1, 2hf+4, 2hf+5
                    *reinterpret_cast<uint4*>(qrow + (c << 4)) = make_uint4(0, 0, 0, 0);
                }
            }
            proxy_fence();  // the tensor core reads Q through the async proxy
            mbar_arrive(q_full);
        };
        // tcgen05.ld / st are warp-collective (.sync.aligned): every branch
        // around them below is decided by a warp vote, never per row.  The two
        // halves of a row sit in warps 4 apart and hold the same rows, so
        // their votes agree.
        constexpr unsigned kAll = 0xffffffffu;
        const uint32_t t_s = t_tile + kHalfKeys * hf;              // this half's S columns
        const uint32_t t_p = t_tile + kColP + kHalfKeys / 2 * hf;  // and P columns (bf16 pairs)
        const uint32_t t_o = t_tile + kColO + kHeadDim / 2 * hf;   // and O dims
        // Half-row maxima and sums pass between the halves through shared
        // memory (maxima double-buffered by block parity, sums in a third
        // slot), behind a named barrier of the tile's 256 softmax threads.
        // Every warp of the tile reaches that barrier once per block and once
        // after a segment's last, also a warp of padding rows and a warp that
        // gave up after a timed-out wait (it goes on without waiting or
        // working), so the counts always match.
        float* xch = reinterpret_cast<float*>(base + kOffX);
        auto xslot = [&](int par, int half) { return xch + ((par * kTiles + tq) * kHalves + half) * kRows + r; };
        const int xbar = 1 + tq;  // named barrier id of the tile
        bool dead = false;
        int J = 0;
        if (n_segs > 0) build_q(0);
        for (int k = 0; k < *n_segs_p; ++k) {
            // Only the row mask and the block range stay live through the block
            // loop; the rest is read again for the epilogue (register budget).
            RowMask rm;
            int b0, b1;
            {
                const Seg& sg = segs[k];
                b0 = sg.b0;
                b1 = sg.b1;
                const UnitInfo ui = unit_info(a, sg.u);
                const int t_row = ui.t_begin + tq * a.tile_tokens + rt;
                rm.L = ui.L;
                rm.T = a.virt ? 0 : ui.T;  // the prefix pass sees no chunk keys
                rm.t_chunk = t_row;
                rm.tree = tree;
                rm.valid = (rt < a.tile_tokens) && (t_row < ui.t_end);
                rm.bits = (tree && rm.valid) ? __ldg(a.tree + ui.q0 + t_row) : 0ull;
            }
            const bool row_valid = rm.valid;
            // m: the row's reference maximum (log2 units; -inf until a key is
            // seen).  O (in TMEM) and l are sums of 2^(S - m) terms.  Padding
            // rows (past the chunk, or the last rows of a tile when G does not
            // divide 128) have Q = 0, so S = 0 on unmasked keys: they start at
            // m = 0 and never ask for a first pass or a redo; their results are
            // not written.
            float m = row_valid ? -INFINITY : 0.f, l = 0.f;
            // A warp of padding rows only (the tail of the last tile) never
            // sweeps S: its P and O rows are never read back, and each row of
            // an MMA is independent of the others.  It still waits for each S
            // before it arrives on p_full, which keeps the barrier phases in step.
            const bool idle = __all_sync(kAll, !row_valid);
            for (int j = b0; j < b1; ++j, ++J) {
                if (!dead && !__all_sync(kAll, wait_bar(&s_full[tq], static_cast<uint32_t>(J) & 1u, abort_flag, a.err)))
                    dead = true;
                const bool work = !dead && !idle;
                const int k0 = j * kBlockKeys + kHalfKeys * hf;
                const bool need_mask = (j + 1) * kBlockKeys > rm.L;  // block-level, so warp-uniform
                float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                float bm = -INFINITY;
                bool first = false;
                if (work) {
                    tc_fence_after();
                    first = __any_sync(kAll, m == -INFINITY);  // some row has no reference yet
                    if (!first)  // one pass: the half's maximum and P against the current reference
                        sweep_s(t_s, t_p, k0, need_mask, rm, m, bm, sum2);
                    else
                        bm = row_max(t_s, k0, need_mask, rm);
                }
                // the row's block maximum over both halves
                *xslot(J & 1, hf) = bm;
                named_bar_sync(xbar, kTileThreads);
                bm = fmaxf(bm, *xslot(J & 1, hf ^ 1));
                if (work) {
                    // raise this row's reference to the block maximum?
                    const bool raise = bm > m + kLazyLog2 || (m == -INFINITY && bm != -INFINITY);
                    if (first || __any_sync(kAll, raise)) {
                        const bool rescale = raise && m != -INFINITY;
                        const float alpha = rescale ? ex2f(m - bm) : 1.f;
                        if (__any_sync(kAll, rescale)) scale_o(t_o, alpha);  // O *= alpha (1 for other rows)
                        l *= alpha;
                        if (raise) m = bm;
                        // P again for the whole warp; rows with no visible key yet
                        // have S = -inf everywhere, so mu = 0 gives P = 0
                        tmem_wait_st();
                        sum2[0] = row_exp_to_tmem(t_s, t_p, k0, need_mask, rm, m == -INFINITY ? 0.f : m);
                        sum2[1] = make_float2(0.f, 0.f);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                }
                if (!dead) mbar_arrive(&p_full[tq]);
                const float2 s01 = __fadd2_rn(sum2[0], sum2[1]);
                l += s01.x + s01.y;
            }
            // The next segment's Q tiles go in now: its first S can then run
            // while this segment's epilogue reads O (S of this segment's last
            // block has completed, so the tensor core is done with these tiles).
            if (k + 1 < *n_segs_p) build_q(k + 1);
            // the row sum over both halves
            *xslot(2, hf) = l;
            named_bar_sync(xbar, kTileThreads);
            const float lt = l + *xslot(2, hf ^ 1);
            const bool have_o = !dead && !idle &&
                                __all_sync(kAll, wait_bar(&pv_full[tq], static_cast<uint32_t>(J - 1) & 1u, abort_flag, a.err));
            if (have_o) tc_fence_after();
            const Seg sg = segs[k];
            __nv_bfloat16* dst;
            {
                const UnitInfo ui = unit_info(a, sg.u);
                dst = a.out + (static_cast<size_t>(ui.q0 + rm.t_chunk) * a.n_q + ui.h * a.group + rg) * kHeadDim +
                      kHeadDim / 2 * hf;
            }
            if (sg.n_parts == 1) {
                if (have_o) {
                    const bool write = row_valid && !*abort_flag;
                    long long row = 0;
                    RowFinish rf{};
                    if (write) {
                        const UnitInfo ui = unit_info(a, sg.u);
                        row = (static_cast<long long>(ui.q0) + rm.t_chunk) * a.n_q + ui.h * a.group + rg;
                        rf = finish_begin(a, row, hf, m, lt);
                    }
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t x[16];
                        tmem_ld16(t_o + 16 * c, x);
                        tmem_wait16(x);
                        float o[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] = __uint_as_float(x[i]);
                        if (write) finish16(a, row, hf, c, rf, o, dst);
                    }
                }
                continue;
            }
            // ---- a part of a unit: its rows' (m, l, O) into this CTA's slot;
            // the last part to arrive merges.  Slot 2c + 1 holds the part of the
            // unit's first CTA (its last segment), slot 2c the other parts (a
            // CTA's first segment), so no CTA needs both for one launch.
            const int prow = tq * kRows + r;
            float* slot = a.part + (2 * static_cast<size_t>(blockIdx.x) + (blockIdx.x == sg.c_first ? 1 : 0)) * kSlotFloats;
            if (have_o) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t x[16];
                    tmem_ld16(t_o + 16 * c, x);
                    tmem_wait16(x);
                    float4* o4 = reinterpret_cast<float4*>(slot + static_cast<size_t>(prow) * kHeadDim + kHeadDim / 2 * hf + 16 * c);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        o4[i] = make_float4(__uint_as_float(x[4 * i]), __uint_as_float(x[4 * i + 1]),
                                            __uint_as_float(x[4 * i + 2]), __uint_as_float(x[4 * i + 3]));
                }
                if (hf == 0)
                    reinterpret_cast<float2*>(slot + static_cast<size_t>(kPartRows) * kHeadDim)[prow] = make_float2(m, lt);
            }
            // bar.sync orders every softmax thread's stores before thread 0's
            // fence, which is cumulative, so one fence publishes the whole part
            // before its arrival is counted.  The other threads go straight on;
            // if this part arrived last, the unit is merged at the CTA's end.
            named_bar_sync(kMergeBar, kSoftmaxThreads);
            if (threadIdx.x == 0) {
                __threadfence();
                const int old = atomicAdd(a.counters + sg.u, 1);
                if (old == sg.n_parts - 1) {
                    a.counters[sg.u] = 0;  // ready for the next launch
                    pend[pend[3]++] = k;
                }
            }
        }
        // ---- the merges this CTA's parts arrived last for (at most two):
        // out = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p, M = max_p m_p
        named_bar_sync(kMergeBar, kSoftmaxThreads);  // pend is complete
        if (threadIdx.x == 0 && pend[3] > 0) __threadfence();
        named_bar_sync(kMergeBar, kSoftmaxThreads);
        for (int pm = 0; pm < pend[3]; ++pm) {
            const Seg sg = segs[pend[pm]];
            const UnitInfo ui = unit_info(a, sg.u);
            const int t_row = ui.t_begin + tq * a.tile_tokens + rt;
            if (!(rt < a.tile_tokens && t_row < ui.t_end) || *abort_flag) continue;
            __nv_bfloat16* dst = a.out + (static_cast<size_t>(ui.q0 + t_row) * a.n_q + ui.h * a.group + rg) * kHeadDim +
                                 kHeadDim / 2 * hf;
            const int prow = tq * kRows + r;
            auto pslot = [&](int c) {
                return a.part + (2 * static_cast<size_t>(c) + (c == sg.c_first ? 1 : 0)) * kSlotFloats;
            };
            auto ml_of = [&](int c) {
                return __ldcg(reinterpret_cast<const float2*>(pslot(c) + static_cast<size_t>(kPartRows) * kHeadDim) + prow);
            };
            // the parts' maxima, four loads in flight at a time
            float M = -INFINITY;
            for (int p0 = 0; p0 < sg.n_parts; p0 += 4) {
                float2 ml[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) ml[q] = p0 + q < sg.n_parts ? ml_of(sg.c_first + p0 + q) : make_float2(-INFINITY, 0.f);
#pragma unroll
                for (int q = 0; q < 4; ++q) M = fmaxf(M, ml[q].x);
            }
            // then 16 dims at a time, two parts' loads in flight at a time
            float lsum = 0.f;
            const long long row = (static_cast<long long>(ui.q0) + t_row) * a.n_q + ui.h * a.group + rg;
            RowFinish rf{};
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
                float o[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = 0.f;
                for (int p0 = 0; p0 < sg.n_parts; p0 += 2) {
                    float2 ml[2];
                    float4 v[2][4];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const bool have = p0 + q < sg.n_parts;
                        const int c = sg.c_first + p0 + (have ? q : 0);
                        ml[q] = have ? ml_of(c) : make_float2(-INFINITY, 0.f);
                        const float4* o4 = reinterpret_cast<const float4*>(pslot(c) + static_cast<size_t>(prow) * kHeadDim +
                                                                           kHeadDim / 2 * hf + 16 * hh);
#pragma unroll
                        for (int i = 0; i < 4; ++i) v[q][i] = have ? __ldcg(o4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const float f = ml[q].x == -INFINITY ? 0.f : ex2f(ml[q].x - M);
                        if (hh == 0) lsum += f * ml[q].y;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            o[4 * i] += f * v[q][i].x;
                            o[4 * i + 1] += f * v[q][i].y;
                            o[4 * i + 2] += f * v[q][i].z;
                            o[4 * i + 3] += f * v[q][i].w;
                        }
                    }
                }
                if (hh == 0) rf = finish_begin(a, row, hf, M, lsum);  // lsum is complete after the first pass
                finish16(a, row, hf, hh, rf, o, dst);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

int prefill_setup(kv_pool* pool) {
    if (pool->cfg.dtype != KV_DTYPE_BF16) return KV_OK;  // the tensor-core path is bf16
    if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
        return KV_ERR_CUDA;
    return KV_OK;
}

// Two slots per CTA of the persistent grid (at most one per SM).
size_t prefill_workspace_bytes(const kv_pool* pool) {
    if (pool->cfg.dtype != KV_DTYPE_BF16) return 0;
    return 2 * static_cast<size_t>(pool->sm_count) * kSlotFloats * sizeof(float);
}

size_t prefill_counter_count(const kv_pool* pool) {
    return pool->cfg.dtype == KV_DTYPE_BF16 ? static_cast<size_t>(kPersistMaxUnits) : 0;
}

namespace {

// One prefill_kernel launch.  shared > 0: the pass given by `pass` of the
// shared-prefix form (0: every token against the first `shared` keys into
// ws; 1: each sequence against the rest of its keys, merged with ws).
int launch_prefill_pass(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                        const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                        const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream, int shared, int pass,
                        float* ws) {
    const auto& c = pool->cfg;
    const int group = c.n_q_heads / c.n_kv_heads;
    if (group < 1 || group > kRows) return KV_ERR_UNSUPPORTED;
    PrefillArgs a{};
    const bool virt = shared > 0 && pass == 0;
    const int mq = virt ? n_seqs * max_q : max_q;  // the prefix pass is one sequence of every token
    a.q = static_cast<const __nv_bfloat16*>(q);
    a.q_pos = q_pos;
    a.q_off = q_off;
    a.prefix = prefix;
    a.tree = virt ? nullptr : tree;
    a.bt = (shared > 0 && pass == 1) ? bt + shared / kPageTokens : bt;
    a.bt_stride = bt_stride;
    a.bt_cols = (shared > 0 && pass == 1) ? bt_stride - shared / kPageTokens : bt_stride;
    a.n_q = c.n_q_heads;
    a.nkv = c.n_kv_heads;
    a.group = group;
    // Tokens per 128-row tile: as many as fit, except that chunks short
    // enough for one CTA are split evenly over its tiles, so that the rows
    // left over are whole warps of padding (which skip the softmax).
    const int fit = kRows / group;
    a.tile_tokens = mq <= kTiles * fit ? std::max(1, (mq + kTiles - 1) / kTiles) : fit;
    a.max_q = mq;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.page_rows = static_cast<int>(pool->page_bytes / 128);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    const int cta_tokens = kTiles * a.tile_tokens;
    a.nx = std::max(1, (mq + cta_tokens - 1) / cta_tokens);
    a.n_seqs = n_seqs;
    a.virt = virt ? 1 : 0;
    a.virt_L = virt ? shared : 0;
    a.L_off = (shared > 0 && pass == 1) ? shared : 0;
    a.prow_total = static_cast<long long>(n_seqs) * max_q * c.n_q_heads;
    a.pout = virt ? ws : nullptr;
    a.pin = (shared > 0 && pass == 1) ? ws : nullptr;
    // More units than SMs but few enough for one work list per CTA: the
    // persistent grid, one CTA per SM, each taking an equal run of the units'
    // key blocks (the plain grid would leave part of its last wave idle).
    const int seqs = virt ? 1 : n_seqs;
    const long long n_units = static_cast<long long>(a.nx) * c.n_kv_heads * seqs;
    a.persist = n_units > pool->sm_count && n_units <= kPersistMaxUnits && pool->pre_part && pool->pre_counters;
    a.part = pool->pre_part;
    a.counters = pool->pre_counters;
    const dim3 grid = a.persist ? dim3(pool->sm_count) : dim3(a.nx, c.n_kv_heads, seqs);
    void* args[] = {&pool->head_map, &a};
    const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(&prefill_kernel), grid, dim3(kThreads), args,
                                           kSmemBytes, stream);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace

int launch_prefill(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                   const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                   const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream) {
    if (pool->cfg.dtype != KV_DTYPE_BF16)  // fp32 and quantised pools: the CUDA-core kernel
        return launch_prefill_f32(pool, q, q_pos, q_off, prefix, tree, n_seqs, max_q, bt, bt_stride, out, stream);
    return launch_prefill_pass(pool, q, q_pos, q_off, prefix, tree, n_seqs, max_q, bt, bt_stride, out, stream, 0, 0,
                               nullptr);
}

size_t prefill_shared_workspace_bytes(const kv_pool* pool, int32_t n_seqs, int32_t max_q) {
    return static_cast<size_t>(n_seqs) * max_q * pool->cfg.n_q_heads * (kHeadDim + 2) * sizeof(float);
}

int launch_prefill_shared(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                          const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                          const uint32_t* bt, int32_t bt_stride, int32_t shared, void* ws, void* out,
                          cudaStream_t stream) {
    int rc = launch_prefill_pass(pool, q, q_pos, q_off, prefix, tree, n_seqs, max_q, bt, bt_stride, out, stream,
                                 shared, 0, static_cast<float*>(ws));
    if (rc != KV_OK) return rc;
    return launch_prefill_pass(pool, q, q_pos, q_off, prefix, tree, n_seqs, max_q, bt, bt_stride, out, stream, shared,
                               1, static_cast<float*>(ws));
}

}  // namespace kvb200
