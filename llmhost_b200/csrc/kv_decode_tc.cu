// kv_decode_tc.cu -- paged decode attention on tcgen05, for bf16 pools.
//
// Same contract as decode_kernel (kv_decode.cu): attention_decode_cached
// (crates/llm-engine/src/lfm2.rs:1006-1056) for one new token per sequence,
// q rotated at seq_lens[s] - 1 (crates/llm-cpu/src/rope.rs:56-81 form), the
// key range [lo, seq_lens[s]) of lfm2.rs:1032-1035 with the sliding window,
// split-K over pages with a last-arriving-contributor merge, and the fused
// append of kv_append_decode_attn.  The dot products run on the tensor cores:
//
//   unit    one kv head over a block of up to 8 pages (128 keys) of one
//           sequence.  A stage of the ring holds two units: K_0, K_1, V_0,
//           V_1, each a [128 keys x 64] bf16 tile of TMA boxes {64 x 16} (one
//           per page and head, 128-byte swizzle, no multicast).  Pages past
//           the block's end load as out-of-range boxes, which fill zeros.
//   S_u^T  = K_u Q_u^T        M 128 keys, N 16 (the unit's query heads, padded), K 64
//   O^T   += [V_0; V_1]^T P   M 128 (the 64 dims of each unit), N 16 (8 query
//                             columns per unit), K 128 keys
// With keys on the M axis each softmax thread owns one key of the block.
// The PV product of the two stacked V tiles yields two useful 64 x 8 blocks
// (unit u's dims x unit u's query heads) and two unused ones.  Units pair the
// kv heads (2p, 2p+1) of a block; with a single kv head they pair
// consecutive blocks of it.
//
// Roles (320 threads, one CTA per SM):
//   warps 0-3  Q tiles, softmax, epilogue and split merge; thread t is key t
//              of the block and TMEM lane t
//   warp 4     TMA producer (one box per lane per stage), and the fused
//              append: the new token's K/V rows are stored to the page in HBM
//              before the box that covers them is loaded
//   warp 5     TMEM owner; lane 0 issues the MMAs
//   warps 6-9  epilogue: a finished sequence segment's O (one of two TMEM
//              buffers), its normalisation or partial row, and the split
//              merge, while warps 0-3 go on with the next segment
//
// Softmax in log2 units (q is pre-scaled by log2(e)/sqrt(d)) against a
// reference maximum per query head, shared by the CTA: P = 2^(S - m), and m
// is raised (O and the row sums rescaled) only when a block's maximum passes
// it by more than kLazyLog2.  P is stored as bf16 and the row sums add the
// same rounded values.  Every wait is bounded; a timeout sets the error word
// and an abort flag, and the CTA runs its schedule out without work.
//
// Work split: every sequence's stages (one per head pair of each 8-page
// chunk), each sequence's list led by kLead stages that stand for the cost of
// opening it, are laid end to end and cut into equal slices, one per CTA of
// the persistent grid.  The kernel is launched with programmatic stream
// serialization: it reads nothing global before griddepcontrol.wait, and lets
// the next launch start on the SMs it has left.
#include <cuda_fp16.h>

#include <cmath>

#include "kv_common.cuh"
#include "kv_decode_sched.cuh"
#include "kv_pool_impl.h"
#include "kv_tc.cuh"

namespace kvb200 {
namespace {

constexpr int kUnitKeys = 128;                        // keys per unit (MMA M of S, K of PV)
constexpr int kUnitPages = kUnitKeys / kPageTokens;   // 8
constexpr int kUnitBytes = kUnitKeys * 128;           // 16 KiB: K (or V) of one unit
constexpr int kStageBytes = 4 * kUnitBytes;           // K_0 K_1 V_0 V_1
constexpr int kStagesBf16 = 3;                       // tile ring of bf16 pools
constexpr int kSoftThreads = 128;                     // warps 0-3
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kEpiWarp0 = 6;                          // warps 6-9
constexpr int kEpiThreads = 128;
constexpr int kThreads = 320;
// Quantised pools: a fourth warpgroup (warps 12-15) turns the pages' int8 /
// int4 codes into the f16 K and V tiles of a stage (in place of the TMA
// boxes); warps 10-11 have no role.  Sixteen warps launch with 128 registers
// each; the converters hand 32 of theirs to the softmax warpgroup
// (setmaxnreg: 4 x 96 + 4 x 160 + 8 x 128 = 16 x 128).
constexpr int kConvWarp0 = 12;                        // warps 12-15
constexpr int kConvWarps = 4;
constexpr int kConvRegs = 96;
constexpr int kSoftRegsQ = 160;
constexpr int kConvPages = kUnitPages / kConvWarps;   // pages of a unit per converter warp
constexpr int kPrefetchStages = 4;                    // L2 prefetch distance of quantised page blocks
template <int kQ>
__host__ __device__ constexpr int block_threads() { return (kQ == 1 || kQ == 2) ? 512 : kThreads; }
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0;   // S of buffer sb, unit u: columns kColS + 32 sb + 16 u ..
constexpr uint32_t kColO = 64;  // O of segment buffer e, accumulator c: kColO + 64 e + 16 c; unit u's queries at + 8 u
constexpr int kPBytes = 2 * 16 * 128;  // P: 16 rows x 128 keys as two 64-key atoms
constexpr float kLazyLog2 = 8.f;
constexpr int kSoftBar = 1;     // named barrier of the softmax warps
constexpr int kEpiBar = 2;      // named barrier of the epilogue warps
constexpr int kSetupBar = 3;    // the producer's scan is done (it arrives, the others wait)
constexpr unsigned kAll = 0xffffffffu;

struct TcArgs {
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    const uint32_t* bt;
    long long bt_stride;
    const int32_t* seq_lens;
    int n_seqs;
    int window;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    int page_rows;
    float* part_o;
    float* part_ml;
    int* counters;   // [n_seqs]: contributors (or runs) merged per sequence
    int* gcounters;  // [2 * gridDim.x]: contributors merged per run of a long sequence
    int* err;
    float qscale;
    const __nv_bfloat16* new_k;  // fused append (null: none)
    const __nv_bfloat16* new_v;
    uint8_t* pages;
    const float* q_norm;  // per-head RMSNorm weights of q and the new k (null: none)
    const float* k_norm;
    float eps;
};

// kQ: the page storage.  0 bf16 and 3 IEEE half (TMA boxes straight into the
// tile ring); 1 Q8 and 2 K8V4 (codes copied raw and converted in the CTA).
// Every kQ but 0 runs the MMAs on f16 operands.
template <int NKV, int G, int kQ = 0>
struct TcShape {
    static constexpr bool kConv = kQ == 1 || kQ == 2;
    static_assert(G >= 1 && G <= 4, "query heads per kv head");
    static_assert(NKV == 1 || NKV == 2 || NKV == 4 || NKV == 8, "kv heads");
    static constexpr int NQ = NKV * G;
    static constexpr int kPairs = NKV >= 2 ? NKV / 2 : 1;  // stages per block round = O accumulators
    // shared memory, from a 1024-aligned base
    // Tile ring: three stages for bf16 pools; two for quantised pools, which
    // also keep two stages of raw page blocks (8 pages x 2 units) that the
    // converter warps expand into the tiles.
    static constexpr int kRing = kConv ? 2 : kStagesBf16;
    static constexpr int kHeadBlock = kConv ? kPageTokens * (kHeadDim + (kQ == 2 ? 32 : 64) + 8) : 0;
    static constexpr int kRawStage = 2 * kUnitPages * kHeadBlock;
    static constexpr int kOffRaw = kRing * kStageBytes;
    static constexpr int kOffQ = kOffRaw + (kConv ? kRing * kRawStage : 0);  // Q tiles: head h at + 1024 h (8 rows)
    static constexpr int kOffP = kOffQ + (NKV + 1) * 1024;          // P, two buffers
    static constexpr int kOffStg = kOffP + 2 * kPBytes;             // fused append inputs
    static constexpr int kStgBytes = NKV * 256 + 256;               // per head K row, V row; RoPE row
    static constexpr int kOffQstg = kOffStg + kStgBytes;            // next segment's q rows and RoPE row
    static constexpr int kQstgBytes = NQ * 128 + 256;
    static constexpr int kOffQsc = kOffQstg + kQstgBytes;           // float [NQ]: q RMSNorm scales
    static constexpr int kOffQw = kOffQsc + ((NQ * 4 + 15) & ~15);  // float [64]: q RMSNorm weights
    static constexpr int kOffMax = kOffQw + 64 * 4;                 // float [2][4 warps][2 units][4]
    static constexpr int kOffM = kOffMax + 2 * 4 * 8 * 4;           // float [2 buffers][NQ]: reference maxima
    static constexpr int kOffL = kOffM + 2 * NQ * 4;                // float [2 buffers][4 warps][NQ]: row sums
    static constexpr int kOffOb = kOffL + 2 * 4 * NQ * 4;           // float [64][4]
    static constexpr int kBars = 28;                                // mbarrier slots (4 kRing + 16 used)
    static constexpr int kOffBar = (kOffOb + 64 * 4 * 4 + 7) & ~7;
    static constexpr int kOffInt = kOffBar + kBars * 8;             // int [16]
    static constexpr int kOffLdm = kOffInt + 16 * 4;                // int [4]: quantised pages loaded per stage
    static constexpr int kOffScan = kOffLdm + 4 * 4;                // int [n_seqs + 1]
    static size_t smem_bytes(int max_seqs) { return 1024 + kOffScan + (static_cast<size_t>(max_seqs) + 1) * 4; }
};

// Work is sliced in stages.  Every sequence's pages are cut into chunks from
// its first page (8 pages; 16 with a single kv head; the last chunk may be
// partial), each chunk into kStages stages (one per kv head pair), the
// stages of all sequences laid end to end, and each CTA takes an equal run
// of them.  A cut between CTAs never splits a block, only the head pairs of
// one chunk.
template <int NKV>
struct Chunk {
    static constexpr int kPages = NKV >= 2 ? kUnitPages : 2 * kUnitPages;
    static constexpr int kStages = NKV >= 2 ? NKV / 2 : 1;
};

// Slices are cut by cost, not by stages alone: the start of a sequence in a
// CTA (its Q tiles, a pipeline restart, a partial last chunk before it) costs
// about as much as kLead stages, so each sequence's stage list begins with
// kLead stages that hold no work.
constexpr int kLead = 2;

// One sequence's stages [g, min(ge, s_end)) inside this CTA's slice [gb, ge)
// (global stage indices; s_begin / s_end are the sequence's first and end
// stage, s_first = s_begin + kLead its first stage with work).  j0, j1: the
// stages with work counted from s_first (nst = j1 - j0, possibly none); c0:
// the chunk of stage j0; pg0, np: block-table index of chunk c0's first
// page, and the pages from there to the end of the segment's last chunk;
// last_chunk: the chunk holding the sequence's last page.
struct Seg {
    int s, nt, lo, pg0, np, s_begin, s_first, s_end, j0, j1, c0, nst, last_chunk;
};

template <int NKV>
__device__ __forceinline__ Seg make_seg(const TcArgs& a, const int* sstart, int s, int g, int ge) {
    constexpr int kCp = Chunk<NKV>::kPages, kSt = Chunk<NKV>::kStages;
    Seg q;
    q.s = s;
    q.nt = __ldg(a.seq_lens + s);
    q.lo = seq_lo(q.nt, a.window);
    q.s_begin = sstart[s];
    q.s_first = q.s_begin + kLead;
    q.s_end = sstart[s + 1];
    q.j0 = max(g, q.s_first) - q.s_first;
    q.j1 = min(ge, q.s_end) - q.s_first;
    q.nst = q.j1 - q.j0;
    q.c0 = q.np = q.pg0 = q.last_chunk = 0;
    if (q.nst <= 0) return q;  // only lead stages of s in this slice
    q.c0 = q.j0 / kSt;
    const int pages = seq_pages(q.nt, a.window);
    const int p0 = kCp * q.c0;
    const int p1 = min(pages, kCp * ((q.j1 - 1) / kSt + 1));
    q.np = p1 - p0;
    q.pg0 = q.lo / kPageTokens + p0;
    q.last_chunk = (pages - 1) / kCp;
    return q;
}

// The first segment with work at or after stage g of the slice; g moves to
// its start.  False if there is none.
template <int NKV>
__device__ __forceinline__ bool seek_seg(const TcArgs& a, const int* sstart, int n, int& g, int ge, Seg& q) {
    while (g < ge) {
        q = make_seg<NKV>(a, sstart, find_seq(sstart, n, g), g, ge);
        if (q.nst > 0) return true;
        g = min(ge, q.s_end);
    }
    return false;
}

// Stage jj of a segment: each unit's block (counted from chunk c0) and its
// page count, and the pair p.
template <int NKV>
__device__ __forceinline__ void stage_units(const Seg& q, int jj, int& b0, int& b1, int& n0, int& n1, int& p) {
    constexpr int kSt = Chunk<NKV>::kStages;
    const int j = q.j0 + jj;
    const int c = j / kSt - q.c0;
    p = j % kSt;
    if (NKV >= 2) {
        b0 = b1 = c;
    } else {
        b0 = 2 * c;
        b1 = 2 * c + 1;
    }
    n0 = max(0, min(kUnitPages, q.np - kUnitPages * b0));
    n1 = max(0, min(kUnitPages, q.np - kUnitPages * b1));
}

// Walks a CTA's stages in schedule order: stage i, stage j of segment q.
template <int NKV>
struct StageCursor {
    int i, j, g, seg_no, ge, n;
    bool done;
    Seg q;
    __device__ __forceinline__ void start(const TcArgs& a, const int* pstart, int n_, int gb, int ge_) {
        i = j = seg_no = 0;
        n = n_;
        ge = ge_;
        g = gb;
        done = !seek_seg<NKV>(a, pstart, n, g, ge, q);
    }
    __device__ __forceinline__ void next(const TcArgs& a, const int* pstart) {
        ++i;
        if (++j < q.nst) return;
        j = 0;
        g = min(ge, q.s_end);
        done = !seek_seg<NKV>(a, pstart, n, g, ge, q);
        ++seg_no;
    }
};

__device__ __forceinline__ float warp_maxf(float x) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
    return r;
}

// Warp reduce-scatter of N per-lane values: level LV (partner lane ^ (16 >>
// LV)) halves the vector while it splits evenly and did so at the level
// before, else adds the partner's whole vector.  Afterwards the lanes whose
// full-exchange bits are clear hold the warp sums of values [base, base +
// len) in v[0 .. len).
template <int N, int LEN, int LV, bool HALVING>
struct ReduceScatter {
    static constexpr bool kHalve = HALVING && LEN % 2 == 0;
    static constexpr int kNext = kHalve ? LEN / 2 : LEN;
    static constexpr int kFinal = ReduceScatter<N, kNext, LV + 1, kHalve>::kFinal;
    __device__ __forceinline__ static void run(float (&v)[N], int lane, int& base, int& full_mask) {
        constexpr int o = 16 >> LV;
        if constexpr (kHalve) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < kNext; ++j) {
                const float send = upper ? v[j] : v[j + kNext];
                const float keep = upper ? v[j + kNext] : v[j];
                v[j] = keep + __shfl_xor_sync(kAll, send, o);
            }
            if (upper) base += kNext;
        } else {
#pragma unroll
            for (int j = 0; j < LEN; ++j) v[j] += __shfl_xor_sync(kAll, v[j], o);
            full_mask |= o;
        }
        ReduceScatter<N, kNext, LV + 1, kHalve>::run(v, lane, base, full_mask);
    }
};
template <int N, int LEN, bool HALVING>
struct ReduceScatter<N, LEN, 5, HALVING> {
    static constexpr int kFinal = LEN;
    __device__ __forceinline__ static void run(float (&)[N], int, int&, int&) {}
};

// Warp sums of v[0 .. N) stored to dst[0 .. N).
template <int N>
__device__ __forceinline__ void warp_reduce_scatter_store(float (&v)[N], float* dst, int lane) {
    int base = 0, full_mask = 0;
    ReduceScatter<N, N, 0, true>::run(v, lane, base, full_mask);
    if ((lane & full_mask) == 0) {
#pragma unroll
        for (int j = 0; j < ReduceScatter<N, N, 0, true>::kFinal; ++j) dst[base + j] = v[j];
    }
}


// kNorm: the q/k RMSNorm of kv_norm_append_decode_attn is compiled in (a
// separate instantiation, so that the plain kernel's hot loops stay as they are).

// ---- quantised pages -------------------------------------------------------
// Prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void* gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// Plain (non-tensor, no multicast) bulk copy of `bytes` (a multiple of 16,
// both addresses 16-byte aligned) into this CTA's shared memory, completing
// on `bar`'s transaction count.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// Codes to f16 tile rows (quantised pools run the MMAs on f16 operands: the
// code-to-value steps then stay on the ALU and FMA pipes).  A code c biased
// to a byte u = c + o becomes the f16 1024 + u through the bit pattern
// 0x6400 | u (a byte permute places two at once), less 1024 + o gives c
// exactly, and c * scale (f16 scale, one f16 rounding to nearest even) is
// the dequantised element of crates/llm-quant/src/lib.rs (BlockQ8_0 and
// BlockQ4 dequantize) to f16 precision.
__device__ __forceinline__ uint2 codes4_to_f16(uint32_t biased, __half2 off, __half2 s) {
    const uint32_t lo = __byte_perm(biased, 0x64646464u, 0x5140);  // bytes 0, 1
    const uint32_t hi = __byte_perm(biased, 0x64646464u, 0x7362);  // bytes 2, 3
    __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&lo), off), s);
    __half2 b = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hi), off), s);
    return make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

// 16 int8 codes (one uint4) -> 16 f16 (two uint4); codes biased by 128.
__device__ __forceinline__ void q8x16_to_f16(uint4 c, __half2 s, uint4& o0, uint4& o1) {
    const __half2 off = __half2half2(__ushort_as_half(0x6480));  // 1152 = 1024 + 128
    const uint2 a = codes4_to_f16(c.x ^ 0x80808080u, off, s), b = codes4_to_f16(c.y ^ 0x80808080u, off, s);
    const uint2 d = codes4_to_f16(c.z ^ 0x80808080u, off, s), e = codes4_to_f16(c.w ^ 0x80808080u, off, s);
    o0 = make_uint4(a.x, a.y, b.x, b.y);
    o1 = make_uint4(d.x, d.y, e.x, e.y);
}

// 8 packed 4-bit codes (one word, element 2i in the low nibble of byte i) ->
// 8 f16 (one uint4); nibbles biased by 8.
__device__ __forceinline__ uint4 q4x8_to_f16(uint32_t w, __half2 s) {
    const __half2 off = __half2half2(__ushort_as_half(0x6408));     // 1032 = 1024 + 8
    const uint32_t even = (w & 0x0F0F0F0Fu) ^ 0x08080808u;         // elements 0, 2, 4, 6
    const uint32_t odd = ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;  // elements 1, 3, 5, 7
    const uint2 a = codes4_to_f16(__byte_perm(even, odd, 0x5140), off, s);  // elements 0..3
    const uint2 b = codes4_to_f16(__byte_perm(even, odd, 0x7362), off, s);  // elements 4..7
    return make_uint4(a.x, a.y, b.x, b.y);
}

// The 16-bit operand type of the MMAs: bf16 (bf16 pools) or f16 (quantised).
template <bool kF16>
__device__ __forceinline__ uint32_t pack_ab(float a, float b) {
    if constexpr (kF16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&h);
    } else {
        return float2_to_bf16x2(a, b);
    }
}

// x rounded to the operand type: its bits, and the rounded value in `xr`.
template <bool kF16>
__device__ __forceinline__ unsigned short round_ab(float x, float& xr) {
    if constexpr (kF16) {
        const __half h = __float2half_rn(x);
        xr = __half2float(h);
        return __half_as_ushort(h);
    } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(x);
        xr = __bfloat162float(h);
        return __bfloat16_as_ushort(h);
    }
}

template <int NKV, int G, bool kNorm, int kQ>
__global__ void __launch_bounds__(block_threads<kQ>(), 1) decode_tc_kernel(const __grid_constant__ CUtensorMap hmap,
                                                                           const TcArgs a) {
    constexpr int kNT = block_threads<kQ>();
    using Sh = TcShape<NKV, G, kQ>;
    constexpr bool kConv = Sh::kConv;  // quantised pages: converter warps
    constexpr bool kF16 = kQ != 0;     // f16 MMA operands (Q, P and the K / V tiles)
    constexpr int kRing = Sh::kRing;
    constexpr int NQ = Sh::NQ;
    constexpr int kPairs = Sh::kPairs;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // Every barrier's slot follows from kRing, so no ring depth can make two
    // of them share an mbarrier (a TMA's byte count and an MMA commit landing
    // on one barrier would corrupt both phases).
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + Sh::kOffBar);
    uint64_t* full = bars;                    // [kRing]    tiles landed (TMA) or written (converters)
    uint64_t* empty = full + kRing;           // [kRing]    PV done with the stage
    uint64_t* s_full = empty + kRing;         // [2]        S MMAs done
    uint64_t* s_free = s_full + 2;            // [2]        S read by the softmax
    uint64_t* p_full = s_free + 2;            // [2]        P (and zeroed V rows) written
    uint64_t* pv_done = p_full + 2;           // [2]        PV MMAs done
    uint64_t* q_full = pv_done + 2;           //            Q tiles of the next segment written
    uint64_t* mma_done = q_full + 1;
    uint64_t* o_full = mma_done + 1;          // [2]        a segment's last PV done (O buffer e)
    uint64_t* seg_done = o_full + 2;          // [2]        its reference maxima and row sums written
    uint64_t* o_free = seg_done + 2;          // [2]        the epilogue is done with O buffer e and its sums
    uint64_t* rfull = o_free + 2;             // [kRing]    quantised pools: a stage's page blocks landed
    uint64_t* rempty = rfull + kRing;         // [kRing]    and were read by the converters
    static_assert(4 * kRing + 16 <= Sh::kBars, "the barrier slots fit the reserved space");
    static_assert(kRing <= 4, "one loaded-page mask per stage");
    int* ldmask = reinterpret_cast<int*>(base + Sh::kOffLdm);
    int* ints = reinterpret_cast<int*>(base + Sh::kOffInt);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ints);
    volatile int* abort_flag = ints + 1;
    int* contrib = ints + 2;
    int* vote = ints + 8;             // [2][4]
    int* pstart = reinterpret_cast<int*>(base + Sh::kOffScan);  // stage starts, [n_seqs + 1]
    float* fmax = reinterpret_cast<float*>(base + Sh::kOffMax);
    float* fm = reinterpret_cast<float*>(base + Sh::kOffM);
    float* fl = reinterpret_cast<float*>(base + Sh::kOffL);
    float* fob = reinterpret_cast<float*>(base + Sh::kOffOb);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = a.n_seqs;
    static_assert(4 * kConvRegs + 4 * kSoftRegsQ + 8 * 128 == 16 * 128, "the register split adds up");
    // Set-up.  The producer warp initialises the barriers, scans the stage
    // counts and goes straight on to its first copies; the other warps clear
    // the Q padding and P buffers, allocate TMEM and wait for the scan.
    if (warp == kProducerWarp) {
        if (lane == 0) {
            for (int i = 0; i < kRing; ++i) {
                mbar_init(&full[i], kConv ? kConvWarps * 32 : 1);  // TMA arrival, or every converter thread
                mbar_init(&rfull[i], 1);
                mbar_init(&rempty[i], kConvWarps * 32);
                mbar_init(&empty[i], 1);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(&s_full[i], 1);
                mbar_init(&s_free[i], kSoftThreads);
                mbar_init(&p_full[i], kSoftThreads);
                mbar_init(&pv_done[i], 1);
            }
            mbar_init(q_full, kSoftThreads);
            mbar_init(mma_done, 1);
            for (int i = 0; i < 2; ++i) {
                mbar_init(&o_full[i], 1);
                mbar_init(&seg_done[i], kSoftThreads);
                mbar_init(&o_free[i], kEpiThreads);
            }
            *abort_flag = 0;
            fence_mbar_init();
            if constexpr (!kConv) prefetch_tmap(&hmap);
        }
        grid_dep_wait();  // the inputs are read from here on
        __syncwarp();
        scan_units(a.seq_lens, n, a.window, Chunk<NKV>::kPages, pstart, lane, Chunk<NKV>::kStages, kLead);
        __syncwarp();
        named_bar_arrive(kSetupBar, kNT);
    } else {
        if (threadIdx.x < kSoftThreads) {  // Q padding rows and P rows never written stay zero
            uint4* z = reinterpret_cast<uint4*>(base + Sh::kOffQ);
            for (int i = threadIdx.x; i < ((NKV + 1) * 1024 + 2 * kPBytes) / 16; i += kSoftThreads)
                z[i] = make_uint4(0, 0, 0, 0);
            proxy_fence();
        }
        if constexpr (kNorm) {  // the q RMSNorm weights, read where the Q tiles are built
            if (threadIdx.x < 64) {
                grid_dep_wait();
                reinterpret_cast<float*>(base + Sh::kOffQw)[threadIdx.x] = __ldg(a.q_norm + threadIdx.x);
            }
        }
        if (warp == kMmaWarp) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             smem_addr(tmem_slot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        grid_dep_wait();
        tc_fence_before();
        named_bar_sync(kSetupBar, kNT);
        tc_fence_after();
    }

    // The grid is persistent (every CTA resident at once), so the next
    // launch's CTAs can only take SMs this grid has left: let it launch now.
    grid_dep_trigger();
    const int total = pstart[n];
    const int cta = blockIdx.x;
    const int grid = max(1, min(static_cast<int>(gridDim.x), total));  // at least one stage per CTA
    const int gb = static_cast<int>((static_cast<long long>(cta) * total) / grid);
    const int ge = static_cast<int>((static_cast<long long>(cta + 1) * total) / grid);
    if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {  // sequences with no tokens: zeros (every CTA, idle ones too)
        for (int s = cta; s < n; s += gridDim.x) {
            if (__ldg(a.seq_lens + s) <= 0) {
                __nv_bfloat16* o = a.out + static_cast<size_t>(s) * NQ * kHeadDim;
                for (int i = threadIdx.x - kEpiWarp0 * 32; i < NQ * kHeadDim; i += kEpiThreads)
                    o[i] = __float2bfloat16_rn(0.f);
            }
        }
    }
    if (cta >= grid || gb >= ge) {  // no work: hand TMEM back and leave
        if (warp == kMmaWarp) {
            const uint32_t tm = *tmem_slot;
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tm), "r"(kTmemCols)
                         : "memory");
        }
        return;
    }
    const uint32_t tmem = *tmem_slot;  // read by the warps that waited on the set-up barrier

    if (warp == kProducerWarp) {
        // ---------------- producer ----------------
        // Software-pipelined: stage i + 1's block-table entries are loaded
        // (and, at a sequence boundary, its segment worked out) before stage
        // i waits for its ring slot, so the copies go out as the slot frees.
        // Lane: page k of the unit's block, K or V, unit u.  Lanes 4k .. 4k+3
        // read page k's K rows of both units' heads (adjacent in the page when
        // the units are heads 2p, 2p+1) and their V rows.
        const int total_rows = static_cast<int>(a.n_pages) * a.page_rows;
        uint8_t* stg = base + Sh::kOffStg;
        const int k = lane >> 2, kv = (lane >> 1) & 1, u = lane & 1;
        struct Fetch {
            uint32_t phys;
            bool load;  // false: past the block's pages (zero fill)
        };
        auto fetch = [&](const StageCursor<NKV>& c) -> Fetch {
            int b0, b1, n0, n1, p;
            stage_units<NKV>(c.q, c.j, b0, b1, n0, n1, p);
            if (k >= (u ? n1 : n0)) return Fetch{0u, false};
            const int pg = c.q.pg0 + kUnitPages * (u ? b1 : b0) + k;
            return Fetch{pg < a.bt_stride ? __ldg(a.bt + static_cast<size_t>(c.q.s) * a.bt_stride + pg) : kPageNone,
                         true};
        };
        // k RMSNorm weights of this lane's dims (2 ii, 2 ii + 1, 32 + 2 ii, 33 + 2 ii)
        float2 kwx = make_float2(1.f, 1.f), kwy = make_float2(1.f, 1.f);
        if constexpr (kNorm && !kConv) {  // quantised pools normalise k in their append launch (no k_norm here)
            kwx = __ldg(reinterpret_cast<const float2*>(a.k_norm) + (lane & 15));
            kwy = __ldg(reinterpret_cast<const float2*>(a.k_norm + 32) + (lane & 15));
        }
        StageCursor<NKV> cur;
        cur.start(a, pstart, n, gb, ge);
        Fetch fc = cur.done ? Fetch{0u, false} : fetch(cur);  // a slice may hold lead stages only
        // Quantised pools: the page blocks of the stage kPrefetchStages ahead
        // are prefetched into L2, so that the raw ring (two stages, all the
        // shared memory leaves) is filled from L2 rather than across the
        // whole HBM latency.
        StageCursor<NKV> pfc = cur;
        Fetch fpf{0u, false};
        int hpf = 0;  // head of this lane's unit in the prefetched stage
        auto fetch_pf = [&]() {
            fpf = pfc.done ? Fetch{0u, false} : fetch(pfc);
            if (!pfc.done) {
                int b0, b1, n0, n1, pp;
                stage_units<NKV>(pfc.q, pfc.j, b0, b1, n0, n1, pp);
                hpf = NKV >= 2 ? 2 * pp + u : 0;
            }
        };
        if constexpr (kConv) {
            for (int d = 0; d < kPrefetchStages && !pfc.done; ++d) pfc.next(a, pstart);
            fetch_pf();
        }
        int issued = 0;
        bool issuing = true, app = false, have_ksc = false;
        float ksc = 0.f;  // lane h < NKV: RMSNorm scale of the new k of head h
        // With k_norm: every head's scale, one lane per head, once the staged
        // rows have landed (kept off the stage that stores them).
        auto k_scales = [&]() {
            cp_async_wait<0>();
            __syncwarp();
            if (lane < NKV) ksc = rms_scale_row(reinterpret_cast<const __nv_bfloat16*>(stg + lane * 256), a.eps);
            have_ksc = true;
        };
        while (!cur.done) {
            const Seg& q = cur.q;
            if (cur.j == 0) {
                // Fused append: the new token (slot nt - 1, on the sequence's
                // last page) for the heads of this slice's stages of the last
                // chunk, when its position is valid.  Its inputs are staged now.
                if (app) cp_async_wait<0>();
                have_ksc = false;
                app = a.new_k != nullptr && (q.j1 - 1) / Chunk<NKV>::kStages == q.last_chunk &&
                      q.nt - 1 < a.max_pos;
                if (app) {
                    const __nv_bfloat16* kr = a.new_k + static_cast<size_t>(q.s) * NKV * kHeadDim;
                    const __nv_bfloat16* vr = a.new_v + static_cast<size_t>(q.s) * NKV * kHeadDim;
                    const uint8_t* cr =
                        reinterpret_cast<const uint8_t*>(a.rope + static_cast<size_t>(q.nt - 1) * (kHeadDim / 2));
                    for (int c = lane; c < NKV * 16 + 16; c += 32) {
                        if (c < NKV * 16) {
                            const int h = c >> 4, r = c & 15;
                            const __nv_bfloat16* src = (r < 8 ? kr : vr) + h * kHeadDim + (r & 7) * 8;
                            cp_async16(stg + h * 256 + (r >> 3) * 128 + (r & 7) * 16, src);
                        } else {
                            cp_async16(stg + NKV * 256 + (c - NKV * 16) * 16, cr + (c - NKV * 16) * 16);
                        }
                    }
                    cp_async_commit();
                }
            }
            if constexpr (kNorm)
                if (app && !have_ksc && cur.j == 1) k_scales();
            StageCursor<NKV> nxt = cur;
            nxt.next(a, pstart);
            const Fetch fn = nxt.done ? Fetch{0u, false} : fetch(nxt);  // in flight during the wait below
            const int i = cur.i, st = i % kRing;
            if (issuing) {
                bool ok = true;
                if (lane == 0 && i >= kRing)
                    ok = wait_bar(kConv ? &rempty[st] : &empty[st], static_cast<uint32_t>(i / kRing - 1) & 1u, abort_flag,
                                  a.err);
                issuing = __shfl_sync(kAll, ok, 0);
            }
            if (issuing) {
                int b0, b1, n0, n1, p;
                stage_units<NKV>(q, cur.j, b0, b1, n0, n1, p);
                if (app && (q.j0 + cur.j) / Chunk<NKV>::kStages == q.last_chunk) {
                    // Store the rotated K and the V rows of this stage's heads
                    // to the page, then let the async proxy (TMA) see them.
                    cp_async_wait<0>();
                    __syncwarp();
                    const int pgl = q.pg0 + q.np - 1;
                    const uint32_t page = pgl < a.bt_stride ? __ldg(a.bt + static_cast<size_t>(q.s) * a.bt_stride + pgl)
                                                            : kPageNone;
                    if (page < a.n_pages) {
                        const int jslot = (q.nt - 1) % kPageTokens;
                        uint8_t* gpage = a.pages + static_cast<size_t>(page) * a.page_rows * 128;
                        const float4 c = *reinterpret_cast<const float4*>(stg + NKV * 256 + 16 * (lane & 15));
                        const int ii = lane & 15;
                        // With k_norm, each head row is RMS-normalised first
                        // (lfm2.rs:805-812) with the scale lane h holds.
                        if constexpr (kNorm)
                            if (!have_ksc) k_scales();
#pragma unroll
                        for (int hh = 0; hh < (NKV >= 2 ? 2 : 1); ++hh) {
                            const int h = NKV >= 2 ? 2 * p + hh : 0;
                            const uint8_t* in = stg + h * 256;
                            float sc = 1.f;
                            if constexpr (kNorm) sc = __shfl_sync(kAll, ksc, h);
                            if (lane < 16) {
                                float2 x = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(in + 4 * ii));
                                float2 y = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(in + 64 + 4 * ii));
                                if constexpr (kNorm) {
                                    x = make_float2(rms_apply(x.x, sc, kwx.x), rms_apply(x.y, sc, kwx.y));
                                    y = make_float2(rms_apply(y.x, sc, kwy.x), rms_apply(y.y, sc, kwy.y));
                                }
                                const float x0 = __fadd_rn(__fmul_rn(x.x, c.x), __fmul_rn(-y.x, c.y));
                                const float x1 = __fadd_rn(__fmul_rn(x.y, c.z), __fmul_rn(-y.y, c.w));
                                const float y0 = __fadd_rn(__fmul_rn(y.x, c.x), __fmul_rn(x.x, c.y));
                                const float y1 = __fadd_rn(__fmul_rn(y.y, c.z), __fmul_rn(x.y, c.w));
                                uint8_t* row = gpage + (h * kPageTokens + jslot) * 128;
                                *reinterpret_cast<uint32_t*>(row + 4 * ii) = pack_ab<kF16>(x0, x1);
                                *reinterpret_cast<uint32_t*>(row + 64 + 4 * ii) = pack_ab<kF16>(y0, y1);
                            } else {
                                uint8_t* row = gpage + ((NKV + h) * kPageTokens + jslot) * 128;
                                const uint2 vb = *reinterpret_cast<const uint2*>(in + 128 + 8 * ii);
                                if constexpr (kF16) {  // half pages: bf16 V widened and rounded to half
                                    const float2 v0 = bf16x2_to_float2(vb.x), v1 = bf16x2_to_float2(vb.y);
                                    *reinterpret_cast<uint2*>(row + 8 * ii) =
                                        make_uint2(pack_ab<true>(v0.x, v0.y), pack_ab<true>(v1.x, v1.y));
                                } else {
                                    *reinterpret_cast<uint2*>(row + 8 * ii) = vb;
                                }
                            }
                        }
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                    }
                    __syncwarp();
                }
                const int hu = NKV >= 2 ? 2 * p + u : 0;
                if constexpr (!kConv) {
                    if (lane == 0) mbar_arrive_expect_tx(&full[st], kStageBytes);
                    __syncwarp();
                    int row = total_rows;  // out of range: zero fill
                    if (fc.load) {
                        if (fc.phys < a.n_pages)
                            row = static_cast<int>(fc.phys) * a.page_rows + (kv ? NKV + hu : hu) * kPageTokens;
                        else
                            flag_error(a.err, kDevErrBadPage);
                    }
                    tma_load_2d(base + st * kStageBytes + kv * 2 * kUnitBytes + u * kUnitBytes + k * 2048, &hmap,
                                &full[st], 0, row);
                } else {
                    // Quantised pages: each loaded page's head blocks (K codes,
                    // V codes, scales; heads 2p, 2p + 1 adjacent)
                    // with plain bulk copies (no multicast) into raw slot st,
                    // block (u, k) at (2k + u) head blocks: one copy of both
                    // units' blocks per page (lane (k, K, 0)), or one per unit
                    // with a single kv head (lanes (k, K, u)).  The mask of
                    // loaded pages goes with the stage.
                    constexpr uint32_t kHB = static_cast<uint32_t>(Sh::kHeadBlock);
                    const bool ld = fc.load && fc.phys < a.n_pages;
                    if (fc.load && !ld) flag_error(a.err, kDevErrBadPage);
                    const unsigned m = __ballot_sync(kAll, ld);
                    if (lane == 0) {
                        ldmask[st] = static_cast<int>(m);
                        mbar_arrive_expect_tx(&rfull[st], NKV >= 2 ? __popc(m & 0x11111111u) * 2 * kHB
                                                                   : __popc(m & 0x33333333u) * kHB);
                    }
                    __syncwarp();
                    if (ld && kv == 0 && (NKV == 1 || u == 0)) {
                        const uint8_t* blk = a.pages + (static_cast<size_t>(fc.phys) * NKV + hu) * kHB;
                        bulk_load(base + Sh::kOffRaw + st * Sh::kRawStage + (2 * k + u) * kHB, blk,
                                  NKV >= 2 ? 2 * kHB : kHB, &rfull[st]);
                    }
                    if (fpf.load && fpf.phys < a.n_pages && kv == 0 && (NKV == 1 || u == 0))
                        prefetch_l2(a.pages + (static_cast<size_t>(fpf.phys) * NKV + hpf) * kHB,
                                    NKV >= 2 ? 2 * kHB : kHB);
                    if (!pfc.done) {
                        pfc.next(a, pstart);
                        fetch_pf();
                    }
                }
                issued = i + 1;
            }
            cur = nxt;
            fc = fn;
        }
        if (app) cp_async_wait<0>();  // nothing left in flight into the staging area
        // Do not leave while a copy may still be landing: the newest copy
        // issued into each stage covers every older one.
        if (lane == 0) {
            for (int st = 0; st < kRing && st < issued; ++st) {
                const int last = st + ((issued - 1 - st) / kRing) * kRing;
                mbar_wait(kConv ? &rfull[st] : &full[st], static_cast<uint32_t>(last / kRing) & 1u);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer ----------------
        // Two cursors over the schedule: S(si) once its K tiles have landed,
        // its S buffer is free and its segment's Q is written; PV(pi) once
        // P(pi) is written.  Neither waits on the other: a PV (which hands
        // its stage back to the producer) never queues behind the next
        // stage's copy.  PV(pi) is issued only after S(pi).
        if (lane == 0) {
            constexpr uint32_t kIdS = instr_desc(16, 128, false, false, kF16);
            constexpr uint32_t kIdPV = instr_desc(16, 128, false, true, kF16);
            const uint32_t st_addr = smem_addr(base), q_addr = smem_addr(base + Sh::kOffQ);
            const uint32_t p_addr = smem_addr(base + Sh::kOffP);
            StageCursor<NKV> sc, pc;
            sc.start(a, pstart, n, gb, ge);
            pc.start(a, pstart, n, gb, ge);
            bool q_ready = false;
            uint64_t t_last = global_timer_ns();
            while (!pc.done) {
                if (*abort_flag) break;
                bool progress = false;
                // first PV into its accumulator in this segment: every pair
                // occurs once in any kPairs consecutive stages
                const bool first = pc.j < kPairs;
                const int eb = pc.seg_no & 1;      // O buffer of the segment
                if (pc.i < sc.i && mbar_test(&p_full[pc.i & 1], static_cast<uint32_t>(pc.i >> 1) & 1u) &&
                    (!first || pc.seg_no < 2 ||
                     mbar_test(&o_free[eb], static_cast<uint32_t>((pc.seg_no - 2) >> 1) & 1u))) {
                    tc_fence_after();
                    const int pcc = NKV >= 2 ? (pc.q.j0 + pc.j) % kPairs : 0;
                    const uint32_t va = st_addr + (pc.i % kRing) * kStageBytes + 2 * kUnitBytes;
                    const uint32_t pa = p_addr + (pc.i & 1) * kPBytes;
#pragma unroll
                    for (int kk = 0; kk < kUnitKeys / 16; ++kk)
                        mma_ss(tmem + kColO + 64 * eb + 16 * pcc, smem_desc(va + 2048 * kk, kUnitBytes, 1024),
                               smem_desc(pa + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), kIdPV, !first || kk > 0);
                    mma_commit(&pv_done[pc.i & 1]);
                    mma_commit(&empty[pc.i % kRing]);
                    if (pc.j == pc.q.nst - 1) mma_commit(&o_full[eb]);
                    pc.next(a, pstart);
                    progress = true;
                }
                if (!sc.done) {
                    const int st = sc.i % kRing, sb = sc.i & 1;
                    if (!q_ready) q_ready = mbar_test(q_full, static_cast<uint32_t>(sc.seg_no) & 1u);
                    if (q_ready && mbar_test(&full[st], static_cast<uint32_t>(sc.i / kRing) & 1u) &&
                        (sc.i < 2 || mbar_test(&s_free[sb], static_cast<uint32_t>((sc.i - 2) >> 1) & 1u))) {
                        tc_fence_after();
                        int b0, b1, n0, n1, p;
                        stage_units<NKV>(sc.q, sc.j, b0, b1, n0, n1, p);
                        const uint32_t ka = st_addr + st * kStageBytes;
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            if ((u ? n1 : n0) == 0) continue;
                            const int hu = NKV >= 2 ? 2 * p + u : 0;
#pragma unroll
                            for (int kk = 0; kk < kHeadDim / 16; ++kk)
                                mma_ss(tmem + kColS + 32 * sb + 16 * u,
                                       smem_desc(ka + u * kUnitBytes + 32 * kk, 16, 1024),
                                       smem_desc(q_addr + hu * 1024 + 32 * kk, 16, 1024), kIdS, kk > 0);
                        }
                        mma_commit(&s_full[sb]);
                        const int seg = sc.seg_no;
                        sc.next(a, pstart);
                        if (sc.seg_no != seg) q_ready = false;
                        progress = true;
                    }
                }
                if (progress) {
                    t_last = global_timer_ns();
                } else if (global_timer_ns() - t_last > kWaitLimitNs) {
                    *abort_flag = 1;
                    flag_error(a.err, kDevErrTimeout);
                    break;
                }
            }
            // Every MMA issued above has finished before TMEM is released.
            mma_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else if (warp < kProducerWarp) {
        // ---------------- softmax and Q tiles (warps 0-3) ----------------
        // (quantised pools: with the registers the converter warpgroup gives up)
        if constexpr (kConv) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftRegsQ));
        const int t = threadIdx.x;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);
        const int kp = t >> 4, slot = t & 15;  // page of the block and slot of this thread's key
        const int ut = t >> 6;                 // O rows of this thread's TMEM lane: unit ut
        // Q tiles of a segment: item (h, n, c) rotates dims [8c, 8c+8) with
        // [32+8c, 32+8c+8) of query head h*G + n (rope.rs:76 form), scales them
        // into log2 units and stores bf16 row n of head h's 8-row group.
        // A segment's q rows and RoPE row are fetched into shared memory
        // (cp.async) while the segment before it streams, so that building its
        // Q tiles at the boundary waits on no global load.
        uint8_t* qstg = base + Sh::kOffQstg;
        auto seg_pos = [&](const Seg& q) { return q.nt - 1 < a.max_pos ? q.nt - 1 : 0; };
        auto prefetch_q = [&](const Seg& q) {
            const uint8_t* src = reinterpret_cast<const uint8_t*>(a.q + static_cast<size_t>(q.s) * NQ * kHeadDim);
            const uint8_t* cr = reinterpret_cast<const uint8_t*>(a.rope + static_cast<size_t>(seg_pos(q)) * (kHeadDim / 2));
            for (int c = t; c < NQ * 8 + 16; c += kSoftThreads)
                cp_async16(qstg + 16 * c, c < NQ * 8 ? src + 16 * c : cr + 16 * (c - NQ * 8));
            cp_async_commit();
        };
        // Q tiles: item (h, n, c) rotates dims [8c, 8c+8) with [32+8c, 32+8c+8)
        // of query head h*G + n (rope.rs:76 form), scales them into log2 units
        // and stores bf16 row n of head h's 8-row group.
        // With q_norm: the RMSNorm scale of each staged q row (lfm2.rs:797-804),
        // one thread per row; worked out during the segment before when it
        // has a second stage, where the softmax warps have slack.
        float* qsc = reinterpret_cast<float*>(base + Sh::kOffQsc);
        const float* qw = reinterpret_cast<const float*>(base + Sh::kOffQw);
        bool qsc_ready = false;
        auto q_scales = [&]() {
            cp_async_wait<0>();
            named_bar_sync(kSoftBar, kSoftThreads);  // every thread's pieces have landed
            if (t < NQ) qsc[t] = rms_scale_row(reinterpret_cast<const __nv_bfloat16*>(qstg + t * 128), a.eps);
            qsc_ready = true;
        };
        auto build_q = [&](const Seg& q) {
            if (q.nt - 1 >= a.max_pos && t == 0) flag_error(a.err, kDevErrBadPos);
            constexpr bool norm = kNorm;
            if constexpr (kNorm)
                if (!qsc_ready) q_scales();
            cp_async_wait<0>();
            named_bar_sync(kSoftBar, kSoftThreads);  // the staged rows (and scales) are visible
            qsc_ready = false;
            if (t < NQ * 4) {
                const int h = t / (G * 4), n_ = (t >> 2) % G, c = t & 3;
                const uint8_t* row_in = qstg + (h * G + n_) * 128;
                const float2* cs = reinterpret_cast<const float2*>(qstg + NQ * 128) + 8 * c;
                const float sc = norm ? qsc[h * G + n_] : 1.f;
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float2 x = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(row_in + 16 * c + 4 * e));
                    float2 y = bf16x2_to_float2(*reinterpret_cast<const uint32_t*>(row_in + 64 + 16 * c + 4 * e));
                    if constexpr (kNorm) {
                        const float2 wx = reinterpret_cast<const float2*>(qw)[4 * c + e];
                        const float2 wy = reinterpret_cast<const float2*>(qw)[16 + 4 * c + e];
                        x = make_float2(rms_apply(x.x, sc, wx.x), rms_apply(x.y, sc, wx.y));
                        y = make_float2(rms_apply(y.x, sc, wy.x), rms_apply(y.y, sc, wy.y));
                    }
                    const float2 c0 = cs[2 * e], c1 = cs[2 * e + 1];
                    const float a0 = __fadd_rn(__fmul_rn(x.x, c0.x), __fmul_rn(-y.x, c0.y)) * a.qscale;
                    const float a1 = __fadd_rn(__fmul_rn(x.y, c1.x), __fmul_rn(-y.y, c1.y)) * a.qscale;
                    const float b0 = __fadd_rn(__fmul_rn(y.x, c0.x), __fmul_rn(x.x, c0.y)) * a.qscale;
                    const float b1 = __fadd_rn(__fmul_rn(y.y, c1.x), __fmul_rn(x.y, c1.y)) * a.qscale;
                    lo[e] = pack_ab<kF16>(a0, a1);
                    hi[e] = pack_ab<kF16>(b0, b1);
                }
                uint8_t* row = base + Sh::kOffQ + h * 1024 + n_ * 128;
                *reinterpret_cast<uint4*>(row + ((c ^ n_) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4*>(row + (((c + 4) ^ n_) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            }
            proxy_fence();  // the tensor core reads Q through the async proxy
            mbar_arrive(q_full);
            named_bar_sync(kSoftBar, kSoftThreads);  // the staging area is free again
        };

        float m[NKV][G], l[NKV][G];
        int i = 0, segk = 0;
        Seg q;
        int g0 = gb;
        const bool any = seek_seg<NKV>(a, pstart, n, g0, ge, q);
        if (any) {
            prefetch_q(q);
            build_q(q);
        }
        for (; any;) {
            // the next segment of this slice, its q fetched while this one streams
            int g_next = min(ge, q.s_end);
            Seg nq = q;
            const bool more = seek_seg<NKV>(a, pstart, n, g_next, ge, nq);
            if (more) prefetch_q(nq);
#pragma unroll
            for (int h = 0; h < NKV; ++h)
#pragma unroll
                for (int c = 0; c < G; ++c) {
                    m[h][c] = -INFINITY;
                    l[h][c] = 0.f;
                }
            // chunks of the segment; a head pair outside [j0, j1) is another CTA's
            const int c_end = (q.j1 - 1) / kPairs;
            for (int cc = q.c0; cc <= c_end; ++cc) {
#pragma unroll
                for (int p = 0; p < kPairs; ++p) {
                    const int jseq = cc * kPairs + p;
                    if (jseq < q.j0 || jseq >= q.j1) continue;
                    const int j = jseq - q.j0;
                    int b0, b1, n0, n1, pp;
                    stage_units<NKV>(q, j, b0, b1, n0, n1, pp);
                    constexpr int kH1 = NKV >= 2 ? 1 : 0;
                    const int h0 = NKV >= 2 ? 2 * p : 0;
                    const int h1 = h0 + kH1;
                    const int sb = i & 1, st = i % kRing;
                    uint8_t* stage = base + st * kStageBytes;
                    // ---- S of this stage: key t's scores for each unit's query heads
                    const bool okS =
                        __all_sync(kAll, wait_bar(&s_full[sb], static_cast<uint32_t>(i >> 1) & 1u, abort_flag, a.err));
                    uint32_t r0[4] = {0, 0, 0, 0}, r1[4] = {0, 0, 0, 0};
                    if (okS) {
                        tc_fence_after();
                        tmem_ld4(lane_base + kColS + 32 * sb, r0);
                        tmem_ld4(lane_base + kColS + 32 * sb + 16, r1);
                        tmem_wait4x2(r0, r1);
                    }
                    tc_fence_before();
                    mbar_arrive(&s_free[sb]);
                    const int tok0 = (q.pg0 + kUnitPages * b0 + kp) * kPageTokens + slot;
                    const int tok1 = (q.pg0 + kUnitPages * b1 + kp) * kPageTokens + slot;
                    const bool v0 = okS && kp < n0 && tok0 >= q.lo && tok0 < q.nt;
                    const bool v1 = okS && kp < n1 && tok1 >= q.lo && tok1 < q.nt;
                    float s0[G], s1[G];
                    bool exceed = false;
#pragma unroll
                    for (int c = 0; c < G; ++c) {
                        s0[c] = v0 ? __uint_as_float(r0[c]) : -INFINITY;
                        s1[c] = v1 ? __uint_as_float(r1[c]) : -INFINITY;
                        exceed |= s0[c] > m[h0][c] + kLazyLog2;
                        exceed |= s1[c] > m[h1][c] + kLazyLog2;
                    }
                    // ---- raise references?  (decided for the whole CTA: every
                    // key of the block is multiplied into the same O)
                    int* vt = vote + 4 * (i & 1);
                    const unsigned bal = __ballot_sync(kAll, exceed);
                    if (lane == 0) vt[warp] = bal != 0u;
                    named_bar_sync(kSoftBar, kSoftThreads);
                    if (vt[0] | vt[1] | vt[2] | vt[3]) {
                        float* mx = fmax + 32 * (i & 1);  // [warp][unit][4]
#pragma unroll
                        for (int c = 0; c < G; ++c) {
                            const float x0 = warp_maxf(s0[c]), x1 = warp_maxf(s1[c]);
                            if (lane == 0) {
                                mx[warp * 8 + c] = x0;
                                mx[warp * 8 + 4 + c] = x1;
                            }
                        }
                        named_bar_sync(kSoftBar, kSoftThreads);
                        float f0[G], f1[G];
                        bool resc = false;
#pragma unroll
                        for (int c = 0; c < G; ++c) {
                            float bm0 = fmaxf(fmaxf(mx[c], mx[8 + c]), fmaxf(mx[16 + c], mx[24 + c]));
                            float bm1 = fmaxf(fmaxf(mx[4 + c], mx[12 + c]), fmaxf(mx[20 + c], mx[28 + c]));
                            if (NKV == 1) bm0 = bm1 = fmaxf(bm0, bm1);
                            {
                                const float mo = m[h0][c];
                                const float mn = bm0 > mo + kLazyLog2 ? bm0 : mo;
                                f0[c] = (mn == mo || mo == -INFINITY) ? 1.f : ex2f(mo - mn);
                                resc |= mn != mo && mo != -INFINITY;
                                l[h0][c] *= f0[c];
                                m[h0][c] = mn;
                            }
                            if (NKV == 1) {
                                f1[c] = f0[c];
                            } else {
                                const float mo = m[h1][c];
                                const float mn = bm1 > mo + kLazyLog2 ? bm1 : mo;
                                f1[c] = (mn == mo || mo == -INFINITY) ? 1.f : ex2f(mo - mn);
                                resc |= mn != mo && mo != -INFINITY;
                                l[h1][c] *= f1[c];
                                m[h1][c] = mn;
                            }
                        }
                        if (resc) {
                            // O of accumulator p holds this segment's earlier
                            // blocks; the PV issued last (stage i - 1) covers them.
                            const bool okP = __all_sync(
                                kAll, wait_bar(&pv_done[(i - 1) & 1], static_cast<uint32_t>((i - 1) >> 1) & 1u,
                                               abort_flag, a.err));
                            if (okP) {
                                tc_fence_after();
                                const uint32_t to = lane_base + kColO + 64 * (segk & 1) + 16 * p + 8 * ut;
                                uint32_t o[4];
                                tmem_ld4(to, o);
                                tmem_wait4(o);
#pragma unroll
                                for (int c = 0; c < G; ++c)
                                    o[c] = __float_as_uint(__uint_as_float(o[c]) * (ut ? f1[c] : f0[c]));
                                tmem_st4(to, o);
                                tmem_wait_st();
                            }
                        }
                    }
                    // ---- P = 2^(S - m) as bf16 into P[i & 1]; zero the V rows
                    // of keys outside the range on loaded pages (stale slots)
                    if (i >= 2) wait_bar(&pv_done[sb], static_cast<uint32_t>((i - 2) >> 1) & 1u, abort_flag, a.err);
                    uint8_t* prow = base + Sh::kOffP + sb * kPBytes + (t >> 6) * 2048;
                    const int chunk = (t & 63) >> 3, within = (t & 7) * 2;
#pragma unroll
                    for (int c = 0; c < G; ++c) {
                        float r0, r1;
                        const unsigned short p0 = round_ab<kF16>(v0 ? ex2f(s0[c] - m[h0][c]) : 0.f, r0);
                        const unsigned short p1 = round_ab<kF16>(v1 ? ex2f(s1[c] - m[h1][c]) : 0.f, r1);
                        l[h0][c] += r0;
                        l[h1][c] += r1;
                        *reinterpret_cast<unsigned short*>(prow + c * 128 + ((chunk ^ c) << 4) + within) = p0;
                        *reinterpret_cast<unsigned short*>(prow + (8 + c) * 128 + ((chunk ^ c) << 4) + within) = p1;
                    }
                    if (okS && !v0 && kp < n0) {
                        uint4* vrow = reinterpret_cast<uint4*>(stage + 2 * kUnitBytes + t * 128);
#pragma unroll
                        for (int c = 0; c < 8; ++c) vrow[c] = make_uint4(0, 0, 0, 0);
                    }
                    if (okS && !v1 && kp < n1) {
                        uint4* vrow = reinterpret_cast<uint4*>(stage + 3 * kUnitBytes + t * 128);
#pragma unroll
                        for (int c = 0; c < 8; ++c) vrow[c] = make_uint4(0, 0, 0, 0);
                    }
                    proxy_fence();
                    tc_fence_before();
                    mbar_arrive(&p_full[sb]);
                    ++i;
                    if constexpr (kNorm)
                        if (more && j == 1) q_scales();  // the next segment's
                }
            }
            // ---- segment done: Q of the next segment first (every S of this
            // one has completed), then hand its reference maxima and row sums
            // to the epilogue warps (O buffer segk & 1), once the epilogue of
            // segment segk - 2 is done with that buffer.
            if (more) {
                q = nq;
                build_q(q);
            }
            const int eb = segk & 1;
            if (segk >= 2) wait_bar(&o_free[eb], static_cast<uint32_t>((segk - 2) >> 1) & 1u, abort_flag, a.err);
            float lv[NQ];
#pragma unroll
            for (int h = 0; h < NKV; ++h)
#pragma unroll
                for (int c = 0; c < G; ++c) {
                    lv[h * G + c] = l[h][c];
                    if (t == 0) fm[eb * NQ + h * G + c] = m[h][c];
                }
            warp_reduce_scatter_store<NQ>(lv, fl + (eb * 4 + warp) * NQ, lane);
            mbar_arrive(&seg_done[eb]);
            ++segk;
            if (!more) break;
        }
    } else if (kConv && warp >= kConvWarp0) {
        // ---------------- converters (quantised pools, warps 12-15) ----------------
        // Warp w expands pages [w P, w P + P) (P = kConvPages) of both units
        // of a stage from its raw slot (head blocks the producer copied) into
        // the tile slot once the PV before it has released that slot: lane
        // (r, hb) takes key r's 32-dim block hb of K and of V and writes it
        // as four 16-byte chunks of f16 in the 128-byte-swizzled tile row
        // (the layout the TMA boxes give bf16 pools).  A page not loaded
        // (past the block's end, or a bad id) is written as zeros.
        if constexpr (kConv) {
            asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kConvRegs));
            constexpr int kVRow = kQ == 2 ? 32 : 64;
            constexpr int kHB = Sh::kHeadBlock;
            const int cw = warp - kConvWarp0, r = lane >> 1, hb = lane & 1;
            const uint32_t sw = static_cast<uint32_t>(r & 7);
            StageCursor<NKV> cur;
            cur.start(a, pstart, n, gb, ge);
            bool going = true;
            while (!cur.done) {
                const int i = cur.i, st = i % kRing;
                if (going) {
                    bool ok = true;
                    if (lane == 0) {
                        ok = wait_bar(&rfull[st], static_cast<uint32_t>(i / kRing) & 1u, abort_flag, a.err);
                        if (ok && i >= kRing)
                            ok = wait_bar(&empty[st], static_cast<uint32_t>(i / kRing - 1) & 1u, abort_flag, a.err);
                    }
                    going = __shfl_sync(kAll, ok, 0);
                }
                if (going) {
                    const unsigned m = static_cast<unsigned>(ldmask[st]);
                    const uint8_t* raw = base + Sh::kOffRaw + st * Sh::kRawStage;
                    uint8_t* stage = base + st * kStageBytes;
#pragma unroll 1
                    for (int e = 0; e < kConvPages; ++e) {
                        const int k = kConvPages * cw + e;
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const bool ld = (m >> (4 * k + u)) & 1u;  // lane (k, K, u) saw this page loaded
                            const uint8_t* blk = raw + (2 * k + u) * kHB;
                            uint4 ko[4], vo[4];
                            if (ld) {
                                const uint4* kr = reinterpret_cast<const uint4*>(blk + r * kHeadDim + 32 * hb);
                                const uint4* vr = reinterpret_cast<const uint4*>(blk + kPageTokens * kHeadDim +
                                                                                 r * kVRow + (kVRow / 2) * hb);
                                // this block's scale pair: K scale, V scale
                                const uint32_t scw = *reinterpret_cast<const uint32_t*>(
                                    blk + kPageTokens * (kHeadDim + kVRow) + r * 8 + hb * 4);
                                const __half2 ks = __half2half2(__ushort_as_half(static_cast<unsigned short>(scw & 0xffffu)));
                                const __half2 vs = __half2half2(__ushort_as_half(static_cast<unsigned short>(scw >> 16)));
                                q8x16_to_f16(kr[0], ks, ko[0], ko[1]);
                                q8x16_to_f16(kr[1], ks, ko[2], ko[3]);
                                if constexpr (kQ == 2) {
                                    const uint4 v = vr[0];
                                    vo[0] = q4x8_to_f16(v.x, vs);
                                    vo[1] = q4x8_to_f16(v.y, vs);
                                    vo[2] = q4x8_to_f16(v.z, vs);
                                    vo[3] = q4x8_to_f16(v.w, vs);
                                } else {
                                    q8x16_to_f16(vr[0], vs, vo[0], vo[1]);
                                    q8x16_to_f16(vr[1], vs, vo[2], vo[3]);
                                }
                            } else {
#pragma unroll
                                for (int x = 0; x < 4; ++x) ko[x] = vo[x] = make_uint4(0, 0, 0, 0);
                            }
                            uint8_t* krow = stage + u * kUnitBytes + k * 2048 + r * 128;
                            uint8_t* vrow = krow + 2 * kUnitBytes;
#pragma unroll
                            for (int x = 0; x < 4; ++x) {
                                const uint32_t off = (static_cast<uint32_t>(4 * hb + x) ^ sw) << 4;
                                *reinterpret_cast<uint4*>(krow + off) = ko[x];
                                *reinterpret_cast<uint4*>(vrow + off) = vo[x];
                            }
                        }
                    }
                    proxy_fence();  // generic-proxy tile writes, read by the MMAs
                    mbar_arrive(&full[st]);
                    mbar_arrive(&rempty[st]);  // the raw slot may take the next copies
                }
                cur.next(a, pstart);
            }
        }
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
        // ---------------- epilogue (warps 6-9) ----------------
        // Segment k: O buffer k & 1 once its last PV is done (o_full) and its
        // maxima and row sums are written (seg_done).  TMEM lane r holds head
        // dim r & 63 of unit r >> 6 (the pair's second kv head, or for a
        // single kv head the odd blocks' share of the same head).
        const int e = threadIdx.x - kEpiWarp0 * 32;
        const int row = 32 * (warp & 3) + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        const int ut = row >> 6, d = row & 63;
        const int ew = warp - kEpiWarp0;  // 0-3
        int k = 0;
        int g = gb;
        Seg cur;
        while (seek_seg<NKV>(a, pstart, n, g, ge, cur)) {
            const int eb = k & 1;
            const uint32_t ph = static_cast<uint32_t>(k >> 1) & 1u;
            const bool okE = __all_sync(kAll, wait_bar(&o_full[eb], ph, abort_flag, a.err)) &&
                             __all_sync(kAll, wait_bar(&seg_done[eb], ph, abort_flag, a.err));
            float ov[kPairs][G], Lv[kPairs][G], Mv[kPairs][G];
            uint32_t oa[kPairs][4];
            if (okE) {
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < kPairs; ++p) tmem_ld4(lane_base + kColO + 64 * eb + 16 * p + 8 * ut, oa[p]);
#pragma unroll
                for (int p = 0; p < kPairs; ++p) tmem_wait4(oa[p]);  // one wait; the rest tie the registers
            } else {
#pragma unroll
                for (int p = 0; p < kPairs; ++p) oa[p][0] = oa[p][1] = oa[p][2] = oa[p][3] = 0u;
            }
#pragma unroll
            for (int p = 0; p < kPairs; ++p) {
                uint32_t o[4] = {oa[p][0], oa[p][1], oa[p][2], oa[p][3]};
                const int h = NKV >= 2 ? 2 * p + ut : 0;
#pragma unroll
                for (int c = 0; c < G; ++c) {
                    const int qh = h * G + c;
                    const float* lb = fl + eb * 4 * NQ;
                    Lv[p][c] = lb[qh] + lb[NQ + qh] + lb[2 * NQ + qh] + lb[3 * NQ + qh];
                    Mv[p][c] = fm[eb * NQ + qh];
                    // a head pair with no stage in this segment (another CTA
                    // took its part of the chunk): its O columns are stale
                    ov[p][c] = Lv[p][c] > 0.f ? __uint_as_float(o[c]) : 0.f;
                }
            }
            if (NKV == 1) {  // the odd blocks accumulate in lanes 64-127: add them in
                if (ut == 1)
#pragma unroll
                    for (int c = 0; c < G; ++c) fob[d * 4 + c] = ov[0][c];
                named_bar_sync(kEpiBar, kEpiThreads);
                if (ut == 0)
#pragma unroll
                    for (int c = 0; c < G; ++c) ov[0][c] += fob[d * 4 + c];
                named_bar_sync(kEpiBar, kEpiThreads);  // fob is free again
            }
            tc_fence_before();
            mbar_arrive(&o_free[eb]);  // O buffer eb and its sums may be reused
            // whole: this CTA holds every stage of s with work; otherwise its
            // partial goes to slot 2 cta + 1 if it holds the first such stage
            const bool whole = cur.s_first >= gb && cur.s_end <= ge;
            const int pslot = (cur.s_first < gb) ? 2 * cta : 2 * cta + 1;
            if (NKV >= 2 || ut == 0) {
#pragma unroll
                for (int p = 0; p < kPairs; ++p) {
                    const int h = NKV >= 2 ? 2 * p + ut : 0;
#pragma unroll
                    for (int c = 0; c < G; ++c) {
                        const int qh = h * G + c;
                        if (whole) {
                            const float inv = Lv[p][c] > 0.f ? 1.f / Lv[p][c] : 0.f;
                            a.out[(static_cast<size_t>(cur.s) * NQ + qh) * kHeadDim + d] =
                                __float2bfloat16_rn(ov[p][c] * inv);
                        } else {
                            const size_t prow = static_cast<size_t>(pslot) * NQ + qh;
                            a.part_o[prow * kHeadDim + d] = ov[p][c];
                            if (d == 0) *reinterpret_cast<float2*>(a.part_ml + prow * 2) = make_float2(Mv[p][c], Lv[p][c]);
                        }
                    }
                }
            }
            if (!whole) {
                // Contributors: the CTAs whose slice holds a stage of s with
                // work; those stages are consecutive, so are they.  CTA c
                // wrote its partial to slot 2c + (c == c_first).  Up to kGroup
                // contributors: the last to arrive merges them all.  More: the
                // last of each run of kGroup contributors merges its run into
                // the run's slot in the second half of the workspace, and the
                // last run to finish merges the run partials.
                const int c_first = cta_of(cur.s_first, grid, total);
                const int n_contrib = cta_of(cur.s_end - 1, grid, total) - c_first + 1;
                auto slot_of = [&](int c) { return static_cast<size_t>((c == c_first) ? 2 * c + 1 : 2 * c); };
                constexpr int kGroup = 16;
                const int n_groups = (n_contrib + kGroup - 1) / kGroup;
                const int g_first = c_first + ((cta - c_first) / kGroup) * kGroup;
                const int g_size = min(kGroup, c_first + n_contrib - g_first);
                const size_t run_base = 2 * static_cast<size_t>(gridDim.x);
                // Warp w folds query heads w, w + 4, ..., kMH of them at a time,
                // each row a partial (256 bytes, lane takes dims 2 lane, 2 lane
                // + 1) into an online maximum, kMB rows of each head in flight;
                // the result goes to the output (normalised) or to a partial slot.
                auto merge = [&](int n_rows, auto row_slot, bool to_out, size_t dst_slot) {
                    constexpr int kMH = 3, kMB = 8;
                    for (int qb = ew; qb < NQ; qb += 4 * kMH) {
                        float Mr[kMH], Lr[kMH];
                        float2 Or[kMH];
#pragma unroll
                        for (int hh = 0; hh < kMH; ++hh) {
                            Mr[hh] = -INFINITY;
                            Lr[hh] = 0.f;
                            Or[hh] = make_float2(0.f, 0.f);
                        }
                        for (int i0 = 0; i0 < n_rows; i0 += kMB) {
                            float2 ml[kMH][kMB], pv[kMH][kMB];
#pragma unroll
                            for (int u = 0; u < kMB; ++u) {
                                const int ic = i0 + u;
                                const size_t sl = row_slot(ic < n_rows ? ic : 0);
#pragma unroll
                                for (int hh = 0; hh < kMH; ++hh) {
                                    const int qh = qb + 4 * hh;
                                    if (ic < n_rows && qh < NQ) {
                                        const size_t prow = sl * NQ + qh;
                                        ml[hh][u] = __ldcg(reinterpret_cast<const float2*>(a.part_ml + prow * 2));
                                        pv[hh][u] = __ldcg(reinterpret_cast<const float2*>(a.part_o + prow * kHeadDim) + lane);
                                    } else {
                                        ml[hh][u] = make_float2(-INFINITY, 0.f);
                                        pv[hh][u] = make_float2(0.f, 0.f);
                                    }
                                }
                            }
#pragma unroll
                            for (int hh = 0; hh < kMH; ++hh) {
                                float bm = Mr[hh];
#pragma unroll
                                for (int u = 0; u < kMB; ++u) bm = fmaxf(bm, ml[hh][u].x);
                                const float mu = (bm == -INFINITY) ? 0.f : bm;
                                const float sc = ex2f(Mr[hh] - mu);
                                Lr[hh] *= sc;
                                Or[hh] = make_float2(Or[hh].x * sc, Or[hh].y * sc);
#pragma unroll
                                for (int u = 0; u < kMB; ++u) {
                                    const float w = ex2f(ml[hh][u].x - mu);
                                    Lr[hh] = fmaf(ml[hh][u].y, w, Lr[hh]);
                                    Or[hh] = make_float2(fmaf(pv[hh][u].x, w, Or[hh].x), fmaf(pv[hh][u].y, w, Or[hh].y));
                                }
                                Mr[hh] = bm;
                            }
                        }
#pragma unroll
                        for (int hh = 0; hh < kMH; ++hh) {
                            const int qh = qb + 4 * hh;
                            if (qh >= NQ) continue;
                            if (to_out) {
                                const float inv = Lr[hh] > 0.f ? 1.f / Lr[hh] : 0.f;
                                *reinterpret_cast<uint32_t*>(a.out + (static_cast<size_t>(cur.s) * NQ + qh) * kHeadDim +
                                                             2 * lane) = float2_to_bf16x2(Or[hh].x * inv, Or[hh].y * inv);
                            } else {
                                const size_t prow = dst_slot * NQ + qh;
                                *(reinterpret_cast<float2*>(a.part_o + prow * kHeadDim) + lane) = Or[hh];
                                if (lane == 0)
                                    *reinterpret_cast<float2*>(a.part_ml + prow * 2) = make_float2(Mr[hh], Lr[hh]);
                            }
                        }
                    }
                };
                __threadfence();
                named_bar_sync(kEpiBar, kEpiThreads);
                if (e == 0)
                    *contrib = atomicAdd(n_groups == 1 ? a.counters + cur.s : a.gcounters + slot_of(g_first), 1);
                named_bar_sync(kEpiBar, kEpiThreads);
                if (n_groups == 1) {
                    if (*contrib == n_contrib - 1) {
                        __threadfence();
                        merge(n_contrib, [&](int r) { return slot_of(c_first + r); }, true, 0);
                        if (e == 0) a.counters[cur.s] = 0;
                    }
                } else if (*contrib == g_size - 1) {
                    __threadfence();
                    merge(g_size, [&](int r) { return slot_of(g_first + r); }, false, run_base + slot_of(g_first));
                    if (e == 0) a.gcounters[slot_of(g_first)] = 0;
                    __threadfence();
                    named_bar_sync(kEpiBar, kEpiThreads);  // every thread has read contrib
                    if (e == 0) *contrib = atomicAdd(a.counters + cur.s, 1);
                    named_bar_sync(kEpiBar, kEpiThreads);
                    if (*contrib == n_groups - 1) {
                        __threadfence();
                        merge(n_groups, [&](int r) { return run_base + slot_of(c_first + r * kGroup); }, true, 0);
                        if (e == 0) a.counters[cur.s] = 0;
                    }
                }
                named_bar_sync(kEpiBar, kEpiThreads);  // contrib is read by all before the next segment
            }
            ++k;
            g = min(ge, cur.s_end);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------
struct TcVariant {
    int nkv, group;
    const void* fn;       // bf16 pages
    const void* fn_norm;  // bf16 pages, with the q/k RMSNorm
    const void* fn_q8;    // KV_DTYPE_Q8 pages (codes converted in the CTA)
    const void* fn_k8v4;  // KV_DTYPE_K8V4 pages
    const void* fn_q8_norm;  // the same with the q RMSNorm
    const void* fn_k8v4_norm;
    const void* fn_f16;       // KV_DTYPE_F16 pages (TMA, f16 operands)
    const void* fn_f16_norm;
    size_t (*smem)(int);  // dynamic shared memory of each, by max_seqs
    size_t (*smem_q8)(int);
    size_t (*smem_k8v4)(int);
    size_t (*smem_f16)(int);
};

template <int NKV, int G>
TcVariant make_tc_variant() {
    return TcVariant{NKV,
                     G,
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, false, 0>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, true, 0>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, false, 1>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, false, 2>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, true, 1>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, true, 2>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, false, 3>),
                     reinterpret_cast<const void*>(&decode_tc_kernel<NKV, G, true, 3>),
                     &TcShape<NKV, G, 0>::smem_bytes, &TcShape<NKV, G, 1>::smem_bytes,
                     &TcShape<NKV, G, 2>::smem_bytes, &TcShape<NKV, G, 3>::smem_bytes};
}

const TcVariant* find_tc_variant(int nkv, int group) {
    static const TcVariant table[] = {
        make_tc_variant<8, 3>(), make_tc_variant<8, 4>(), make_tc_variant<1, 4>(),
        make_tc_variant<2, 4>(), make_tc_variant<4, 4>(),
    };
    for (const auto& v : table)
        if (v.nkv == nkv && v.group == group) return &v;
    return nullptr;
}

// The kernel for a pool's storage type, plain or with the q/k RMSNorm.
const void* tc_kernel_for(const TcVariant* v, int dtype, bool norm) {
    if (dtype == KV_DTYPE_Q8) return norm ? v->fn_q8_norm : v->fn_q8;
    if (dtype == KV_DTYPE_K8V4) return norm ? v->fn_k8v4_norm : v->fn_k8v4;
    if (dtype == KV_DTYPE_F16) return norm ? v->fn_f16_norm : v->fn_f16;
    return norm ? v->fn_norm : v->fn;
}

int tc_threads_for(int dtype) { return is_quant(dtype) ? block_threads<1>() : block_threads<0>(); }

}  // namespace

int decode_tc_setup(kv_pool* pool) {
    const auto& c = pool->cfg;
    const TcVariant* v = find_tc_variant(c.n_kv_heads, c.n_q_heads / c.n_kv_heads);
    if (!v) return KV_ERR_UNSUPPORTED;
    const size_t smem = (c.dtype == KV_DTYPE_Q8     ? v->smem_q8
                         : c.dtype == KV_DTYPE_K8V4 ? v->smem_k8v4
                         : c.dtype == KV_DTYPE_F16  ? v->smem_f16
                                                    : v->smem)(c.max_seqs);
    int optin = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c.device) != cudaSuccess)
        return KV_ERR_CUDA;
    if (smem > static_cast<size_t>(optin)) return KV_ERR_INVALID;  // max_seqs too large
    const void* fn = tc_kernel_for(v, c.dtype, false);
    if (raise_smem_limit(fn, c.device, smem) != KV_OK ||
        raise_smem_limit(tc_kernel_for(v, c.dtype, true), c.device, smem) != KV_OK)
        return KV_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, tc_threads_for(c.dtype), smem) != cudaSuccess ||
        per_sm < 1)
        return KV_ERR_CUDA;
    pool->decode_grid = pool->sm_count * per_sm;
    pool->decode_smem = smem;
    return KV_OK;
}

int launch_decode_tc(kv_pool* pool, const void* q, const uint32_t* bt, int32_t bt_stride, const int32_t* seq_lens,
                     int32_t n_seqs, int32_t window, void* out, cudaStream_t stream, const void* new_k,
                     const void* new_v, const float* q_norm, const float* k_norm, float eps) {
    const auto& c = pool->cfg;
    const TcVariant* v = find_tc_variant(c.n_kv_heads, c.n_q_heads / c.n_kv_heads);
    if (!v) return KV_ERR_UNSUPPORTED;
    // Quantised pools: the append (with the k norm) is its own launch.
    if (is_quant(c.dtype) && (new_k != nullptr || k_norm != nullptr)) return KV_ERR_UNSUPPORTED;
    TcArgs a;
    a.q = static_cast<const __nv_bfloat16*>(q);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.bt = bt;
    a.bt_stride = bt_stride;
    a.seq_lens = seq_lens;
    a.n_seqs = n_seqs;
    a.window = window;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.page_rows = static_cast<int>(pool->page_bytes / 128);
    a.part_o = pool->part_o;
    a.part_ml = pool->part_ml;
    a.counters = pool->counters;
    a.gcounters = pool->counters + c.max_seqs;
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    a.new_k = static_cast<const __nv_bfloat16*>(new_k);
    a.new_v = static_cast<const __nv_bfloat16*>(new_v);
    a.pages = static_cast<uint8_t*>(pool->pages);
    a.q_norm = q_norm;
    a.k_norm = k_norm;
    a.eps = eps;
    void* args[] = {&pool->head_map, &a};
    // Programmatic serialization: this launch may start while the kernel
    // before it in the stream finishes; it reads nothing before that kernel
    // has completed (grid_dep_wait), so stream order holds for the data.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(pool->decode_grid);
    lc.blockDim = dim3(tc_threads_for(c.dtype));
    lc.dynamicSmemBytes = pool->decode_smem;
    lc.stream = stream;
    lc.attrs = attr;
    lc.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelExC(&lc, tc_kernel_for(v, c.dtype, q_norm != nullptr), args);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
