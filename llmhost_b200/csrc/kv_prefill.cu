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
constexpr int kOffX = kOffBar + 256;  // float [2][kTiles][kHalves][kRows]: half-row maxima / sums
constexpr int kSmemBytes = 1024 + kOffX + 2 * kTiles * kHalves * kRows * 4;

// P entries stay below 2^kLazyLog2 times the row's reference maximum; the
// reference is raised only when a block's maximum exceeds it by more.
constexpr float kLazyLog2 = 8.f;

struct PrefillArgs {
    const __nv_bfloat16* q;
    const int32_t* q_pos;
    const int32_t* q_off;
    const int32_t* prefix;
    const unsigned long long* tree;
    const uint32_t* bt;
    long long bt_stride;
    int n_q, nkv, group, tile_tokens, max_q;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    int page_rows;
    __nv_bfloat16* out;
    int* err;
    float qscale;
};

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

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap hmap,
                                                              const PrefillArgs a) {
    const int s = blockIdx.z, h = blockIdx.y;
    const int q0 = __ldg(a.q_off + s);
    const int T = __ldg(a.q_off + s + 1) - q0;
    const int L = __ldg(a.prefix + s);
    const bool tree = a.tree != nullptr;
    const int cta_tokens = kTiles * a.tile_tokens;
    if (T < 0 || L < 0 || T > a.max_q || (tree && T > 64)) {
        if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0) flag_error(a.err, kDevErrBadArg);
        return;
    }
    const int t_begin = blockIdx.x * cta_tokens;
    if (t_begin >= T) return;
    const int t_end = min(T, t_begin + cta_tokens);
    const int kmax = tree ? L + T : L + t_end;  // keys [0, kmax) can be visible to this CTA
    const int nb = (kmax + kBlockKeys - 1) / kBlockKeys;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kOffBar);  // [kStages]
    uint64_t* empty = full + kStages;                               // [kStages]
    uint64_t* s_full = empty + kStages;                             // [kTiles]
    uint64_t* p_full = s_full + kTiles;                             // [kTiles]
    uint64_t* pv_full = p_full + kTiles;                            // [kTiles]
    uint64_t* mma_done = pv_full + kTiles;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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

    // ---- Q tiles (warps 0-15): thread = (tile tq, half hf, row r); row r of
    // tile tq is (token t_begin + tq * tile_tokens + r / G, head h*G + r % G).
    // RoPE at q_pos (rope.rs:76 form), scaled into log2 units, bf16, into
    // shared memory; each half builds half of the row's dims.
    const int tq = (warp >> 3) & 1, hf = (warp >> 2) & 1, r = 32 * (warp & 3) + lane;
    const int rt = r / a.group, rg = r % a.group;
    const int t_row = t_begin + tq * a.tile_tokens + rt;
    const bool row_valid = (threadIdx.x < kSoftmaxThreads) && (rt < a.tile_tokens) && (t_row < t_end);
    tc_fence_before();
    __syncthreads();  // the TMEM address is published
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    const uint32_t t_tile = lane_base + kTileCols * tq;  // this thread's row of its tile
    if (threadIdx.x < kSoftmaxThreads) {
        uint8_t* qrow = base + tq * kQBytes + r * 128;
        if (row_valid) {
            const uint4* src = reinterpret_cast<const uint4*>(
                a.q + (static_cast<size_t>(q0 + t_row) * a.n_q + h * a.group + rg) * kHeadDim);
            int pos = __ldg(a.q_pos + q0 + t_row);
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
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == kProducerWarp) {
        // ---------------- producer: K/V head slices, 8 pages per block ----------------
        // Lane i < 8 owns page i of every block: its block-table entry for
        // block j + 1 is loaded while block j's stage is waited for, and it
        // issues that page's K and V boxes (lane 0 first sets the stage's
        // expected bytes), so no copy waits on a serial chain of loads.
        const int total_rows = static_cast<int>(a.n_pages) * a.page_rows;
        // page pi of the sequence holds keys this CTA can see
        auto used = [&](int j) { return lane < kPagesPerBlock && (j * kPagesPerBlock + lane) * kPageTokens < kmax; };
        auto entry = [&](int j) -> uint32_t {
            const int pi = j * kPagesPerBlock + lane;
            if (!used(j)) return 0u;
            return pi < a.bt_stride ? __ldg(a.bt + static_cast<size_t>(s) * a.bt_stride + pi) : kPageNone;
        };
        int issued = 0;
        uint32_t next = nb > 0 ? entry(0) : 0u;
        for (int j = 0; j < nb; ++j) {
            const int st = j % kStages;
            const uint32_t phys = next;
            if (j + 1 < nb) next = entry(j + 1);  // in flight during the wait below
            bool ok = true;
            if (lane == 0 && j >= kStages)
                ok = wait_bar(&empty[st], static_cast<uint32_t>(j / kStages - 1) & 1u, abort_flag, a.err);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            if (lane == 0) mbar_arrive_expect_tx(&full[st], kStageBytes);
            __syncwarp();
            if (lane < kPagesPerBlock) {
                uint8_t* kt = base + kOffStage + st * kStageBytes;
                int rk = total_rows, rv = total_rows;  // out of range: zero fill
                if (used(j)) {
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
            issued = j + 1;
        }
        if (lane == 0 && *abort_flag) {  // wait (bounded) for the newest copy issued into each stage
            for (int st = 0; st < kStages && st < issued; ++st) {
                const int last = st + ((issued - 1 - st) / kStages) * kStages;
                mbar_wait(&full[st], static_cast<uint32_t>(last / kStages) & 1u);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer (one thread) ----------------
        // Per block j and tile t: O_t += P_t(j-1) V(j-1) once P_t(j-1) is
        // written, then S_t(j).  tcgen05.mma executes in issue order, so when
        // S_t(j) completes P_t(j-1) V(j-1) has too: the softmax may then
        // overwrite P_t and rescale O_t.  The K/V stage of block j-1 is
        // released after the last tile's PV.
        if (lane == 0) {
            constexpr uint32_t kIdescS = instr_desc(kBlockKeys, kRows, false);
            constexpr uint32_t kIdescPV = instr_desc(kHeadDim, kRows, true);
            const uint32_t q_addr = smem_addr(base);
            const uint32_t stage_addr = smem_addr(base + kOffStage);
            for (int j = 0; j <= nb; ++j) {
                const int st = j % kStages, pst = (j + kStages - 1) % kStages;
                if (j < nb && !wait_bar(&full[st], static_cast<uint32_t>(j / kStages) & 1u, abort_flag, a.err))
                    break;
                tc_fence_after();
                bool ok = true;
#pragma unroll
                for (int t = 0; t < kTiles; ++t) {
                    const uint32_t tt = tmem + kTileCols * t;
                    if (j > 0) {
                        if (!wait_bar(&p_full[t], static_cast<uint32_t>(j - 1) & 1u, abort_flag, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t v_addr = stage_addr + pst * kStageBytes + kKvBytes;
#pragma unroll
                        for (int kk = 0; kk < kBlockKeys / 16; ++kk)
                            mma_ts(tt + kColO, tt + kColP + 8 * kk, smem_desc(v_addr + 2048 * kk, kKvBytes, 1024),
                                   kIdescPV, j > 1 || kk > 0);
                        mma_commit(&pv_full[t]);
                    }
                    if (j < nb) {
                        const uint32_t k_addr = stage_addr + st * kStageBytes;
                        const uint32_t qa = q_addr + t * kQBytes;
#pragma unroll
                        for (int kk = 0; kk < kHeadDim / 16; ++kk)
                            mma_ss(tt, smem_desc(qa + 32 * kk, 16, 1024), smem_desc(k_addr + 32 * kk, 16, 1024), kIdescS,
                                   kk > 0);
                        mma_commit(&s_full[t]);
                    }
                }
                if (!ok) break;
                if (j > 0) mma_commit(&empty[pst]);
            }
            // Every MMA issued above has finished before TMEM is released.
            mma_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else {
        // ---------------- softmax: thread (tq, hf, r) owns half hf of row r of tile tq ----------------
        RowMask rm;
        rm.L = L;
        rm.T = T;
        rm.t_chunk = t_row;
        rm.tree = tree;
        rm.valid = row_valid;
        rm.bits = (tree && row_valid) ? __ldg(a.tree + q0 + t_row) : 0ull;
        // m: the row's reference maximum (log2 units; -inf until a key is seen).
        // O (in TMEM) and l are sums of 2^(S - m) terms.  Padding rows (past
        // the chunk, or the last rows of a tile when G does not divide 128)
        // have Q = 0, so S = 0 on unmasked keys: they start at m = 0 and never
        // ask for a first pass or a redo; their results are not written.
        float m = row_valid ? -INFINITY : 0.f, l = 0.f;
        // tcgen05.ld / st are warp-collective (.sync.aligned): every branch
        // around them below is decided by a warp vote, never per row.  The two
        // halves of a row sit in warps 4 apart and hold the same rows, so
        // their votes agree.
        constexpr unsigned kAll = 0xffffffffu;
        // A warp of padding rows only (the tail of the last tile) never
        // sweeps S: its P and O rows are never read back, and each row of an
        // MMA is independent of the others.  It still waits for each S before
        // it arrives on p_full, which keeps the barrier phases in step.
        const bool idle = __all_sync(kAll, !row_valid);
        const uint32_t t_s = t_tile + kHalfKeys * hf;         // this half's S columns
        const uint32_t t_p = t_tile + kColP + kHalfKeys / 2 * hf;  // and P columns (bf16 pairs)
        const uint32_t t_o = t_tile + kColO + kHeadDim / 2 * hf;   // and O dims
        // Half-row maxima and sums pass between the halves through shared
        // memory, double-buffered by block parity, behind a named barrier of
        // the tile's 256 softmax threads.  Every warp of the tile reaches that
        // barrier once per block and once after the last, also a warp of
        // padding rows and a warp that gave up after a timed-out wait (it
        // goes on without waiting or working), so the counts always match.
        float* xch = reinterpret_cast<float*>(base + kOffX);
        auto xslot = [&](int par, int half) { return xch + ((par * kTiles + tq) * kHalves + half) * kRows + r; };
        const int xbar = 1 + tq;  // named barrier id of the tile
        bool dead = false;
        for (int j = 0; j < nb; ++j) {
            if (!dead && !__all_sync(kAll, wait_bar(&s_full[tq], static_cast<uint32_t>(j) & 1u, abort_flag, a.err)))
                dead = true;
            const bool work = !dead && !idle;
            const int k0 = j * kBlockKeys + kHalfKeys * hf;
            const bool need_mask = (j + 1) * kBlockKeys > L;  // block-level, so warp-uniform
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
            *xslot(j & 1, hf) = bm;
            named_bar_sync(xbar, kTileThreads);
            bm = fmaxf(bm, *xslot(j & 1, hf ^ 1));
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
        // the row sum over both halves (slot parity nb & 1: its last readers
        // passed the barrier of block nb - 1)
        *xslot(nb & 1, hf) = l;
        named_bar_sync(xbar, kTileThreads);
        const float lt = l + *xslot(nb & 1, hf ^ 1);
        if (!dead && !idle &&
            __all_sync(kAll, wait_bar(&pv_full[tq], static_cast<uint32_t>(nb - 1) & 1u, abort_flag, a.err))) {
            tc_fence_after();
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
            __nv_bfloat16* dst = a.out + (static_cast<size_t>(q0 + t_row) * a.n_q + h * a.group + rg) * kHeadDim +
                                 kHeadDim / 2 * hf;
            const bool write = row_valid && !*abort_flag;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t x[16];
                tmem_ld16(t_o + 16 * c, x);
                tmem_wait16(x);
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    w[i] = float2_to_bf16x2(__uint_as_float(x[2 * i]) * inv, __uint_as_float(x[2 * i + 1]) * inv);
                if (write) {
                    reinterpret_cast<uint4*>(dst)[2 * c] = make_uint4(w[0], w[1], w[2], w[3]);
                    reinterpret_cast<uint4*>(dst)[2 * c + 1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
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

int launch_prefill(kv_pool* pool, const void* q, const int32_t* q_pos, const int32_t* q_off,
                   const int32_t* prefix, const unsigned long long* tree, int32_t n_seqs, int32_t max_q,
                   const uint32_t* bt, int32_t bt_stride, void* out, cudaStream_t stream) {
    const auto& c = pool->cfg;
    if (c.dtype == KV_DTYPE_F32)
        return launch_prefill_f32(pool, q, q_pos, q_off, prefix, tree, n_seqs, max_q, bt, bt_stride, out, stream);
    const int group = c.n_q_heads / c.n_kv_heads;
    if (group < 1 || group > kRows) return KV_ERR_UNSUPPORTED;
    PrefillArgs a;
    a.q = static_cast<const __nv_bfloat16*>(q);
    a.q_pos = q_pos;
    a.q_off = q_off;
    a.prefix = prefix;
    a.tree = tree;
    a.bt = bt;
    a.bt_stride = bt_stride;
    a.n_q = c.n_q_heads;
    a.nkv = c.n_kv_heads;
    a.group = group;
    // Tokens per 128-row tile: as many as fit, except that chunks short
    // enough for one CTA are split evenly over its tiles, so that the rows
    // left over are whole warps of padding (which skip the softmax).
    const int fit = kRows / group;
    a.tile_tokens = max_q <= kTiles * fit ? std::max(1, (max_q + kTiles - 1) / kTiles) : fit;
    a.max_q = max_q;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.page_rows = static_cast<int>(pool->page_bytes / 128);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    const int cta_tokens = kTiles * a.tile_tokens;
    const dim3 grid((max_q + cta_tokens - 1) / cta_tokens, c.n_kv_heads, n_seqs);
    void* args[] = {&pool->head_map, &a};
    const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(&prefill_kernel), grid, dim3(kThreads), args,
                                           kSmemBytes, stream);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
