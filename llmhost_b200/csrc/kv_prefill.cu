// kv_prefill.cu -- chunked-prefill and tree-verify attention on tcgen05 (bf16).
//
// Replaces attention_forward (crates/llm-engine/src/lfm2.rs:1058-1111) for a
// chunk of T new tokens appended after L cached ones, the case the reference
// lacks (attn_prefill always starts at position 0, lfm2.rs:730).  Query token
// i (chunk-relative) sees cached key s < L, and chunk key L + j when j <= i
// (causal chunk) or, for a speculative tree, when bit j of its
// ancestor-or-self mask is set.  The chunk's K/V must already be in pages.
//
// One CTA per (sequence, kv head, tile of 128 query rows); a row is a
// (token, query head of the group) pair.  Warps 0-3 own one row per thread
// (softmax), warp 4 streams K/V head slices page by page with TMA (one
// {64 x 16} bf16 box per page and per K / V, 128-byte swizzle, no multicast)
// into a 2-stage ring of 128-key blocks, warp 5 allocates TMEM and issues the
// tensor-core MMAs from one thread:
//   S  = Q K^T  : M 128, N 128, K 64, bf16 operands K-major, fp32 in TMEM;
//   PV = P V    : M 128, N 64,  K 128, P K-major from shared memory, V
//                 MN-major straight from the page layout, fp32 in TMEM.
// The softmax threads read their row of S from TMEM, keep the running max
// and sum in log2 units (q is pre-scaled by log2(e)/sqrt(d)), write P as bf16
// to shared memory, then fold PV into an fp32 accumulator in registers.
// Pages past the sequence load as out-of-range boxes (zero fill).
#include <cmath>

#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace kvb200 {
namespace {

constexpr int kRows = 128;                                // MMA M
constexpr int kBlockKeys = 128;                           // keys per block (MMA N of S)
constexpr int kPagesPerBlock = kBlockKeys / kPageTokens;  // 8
constexpr int kStages = 2;
constexpr int kTile = kRows * 128;                        // 16 KiB: 128 rows of 64 bf16
constexpr int kSliceBytes = kPageTokens * 128;            // one page's K (or V) rows of one head
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColPV = 128;
constexpr int kThreads = 192;

// smem offsets from the 1024-aligned base
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kTile;                      // 2 sub-tiles (keys 0-63, 64-127)
constexpr int kOffStage = kOffP + 2 * kTile;              // stage st: K at +0, V at +kTile
constexpr int kStageBytes = 2 * kTile;
constexpr int kOffBar = kOffStage + kStages * kStageBytes;
constexpr int kSmemBytes = 1024 + kOffBar + 128;

struct PrefillArgs {
    const __nv_bfloat16* q;
    const int32_t* q_pos;
    const int32_t* q_off;
    const int32_t* prefix;
    const unsigned long long* tree;
    const uint32_t* bt;
    long long bt_stride;
    int n_q, nkv, group, tile_tokens;
    const float2* rope;
    int max_pos;
    uint32_t n_pages;
    int page_rows;
    __nv_bfloat16* out;
    int* err;
    float qscale;
};

// tcgen05 shared-memory descriptor: 128-byte swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (static_cast<uint64_t>((addr >> 4) & 0x3FFFu)) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B.
__host__ __device__ constexpr uint32_t instr_desc(int n, int m, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc ? 1 : 0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2f(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// Bounded wait that gives up (and raises the CTA abort flag) after the time limit.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
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

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap hmap,
                                                              const PrefillArgs a) {
    const int s = blockIdx.z, h = blockIdx.y;
    const int q0 = __ldg(a.q_off + s);
    const int T = __ldg(a.q_off + s + 1) - q0;
    const int L = __ldg(a.prefix + s);
    const bool tree = a.tree != nullptr;
    if (T < 0 || L < 0 || T > static_cast<int>(gridDim.x) * a.tile_tokens || (tree && T > 64)) {
        if (blockIdx.x == 0 && h == 0 && threadIdx.x == 0) flag_error(a.err, kDevErrBadArg);
        return;
    }
    const int t_begin = blockIdx.x * a.tile_tokens;
    if (t_begin >= T) return;
    const int t_end = min(T, t_begin + a.tile_tokens);
    const int kmax = tree ? L + T : L + t_end;  // keys [0, kmax) can be visible to this tile
    const int nb = (kmax + kBlockKeys - 1) / kBlockKeys;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + kOffBar);  // [kStages]
    uint64_t* empty = full + kStages;                               // [kStages]
    uint64_t* s_full = empty + kStages;
    uint64_t* p_full = s_full + 1;
    uint64_t* pv_full = p_full + 1;
    uint64_t* mma_done = pv_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(p_full, kRows);  // every softmax thread arrives
        mbar_init(pv_full, 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) {  // TMEM: S at columns [0, 128), PV at [128, 192)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (warp == 4 && lane == 0) prefetch_tmap(&hmap);

    // ---- Q tile (warps 0-3): row r = (token t_begin + r / G, head h*G + r % G),
    // RoPE at q_pos (rope.rs:76 form), scaled into log2 units, bf16, swizzled.
    const int r = threadIdx.x;
    const int rt = r / a.group, rg = r % a.group;
    const int t_row = t_begin + rt;
    const bool row_valid = (r < kRows) && (rt < a.tile_tokens) && (t_row < t_end);
    if (r < kRows) {
        uint4 packed[8];
        if (row_valid) {
            const __nv_bfloat16* src = a.q + (static_cast<size_t>(q0 + t_row) * a.n_q + h * a.group + rg) * kHeadDim;
            float x[kHeadDim];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + c);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 f = bf16x2_to_float2(w[i]);
                    x[8 * c + 2 * i] = f.x;
                    x[8 * c + 2 * i + 1] = f.y;
                }
            }
            int pos = __ldg(a.q_pos + q0 + t_row);
            if (pos < 0 || pos >= a.max_pos) {
                flag_error(a.err, kDevErrBadPos);
                pos = 0;
            }
            const float2* cs = a.rope + static_cast<size_t>(pos) * (kHeadDim / 2);
            float y[kHeadDim];
#pragma unroll
            for (int i = 0; i < kHeadDim / 2; ++i) {
                const float2 c = __ldg(cs + i);
                y[i] = __fadd_rn(__fmul_rn(x[i], c.x), __fmul_rn(-x[i + 32], c.y)) * a.qscale;
                y[i + 32] = __fadd_rn(__fmul_rn(x[i + 32], c.x), __fmul_rn(x[i], c.y)) * a.qscale;
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
                packed[c] = make_uint4(float2_to_bf16x2(y[8 * c], y[8 * c + 1]), float2_to_bf16x2(y[8 * c + 2], y[8 * c + 3]),
                                       float2_to_bf16x2(y[8 * c + 4], y[8 * c + 5]),
                                       float2_to_bf16x2(y[8 * c + 6], y[8 * c + 7]));
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) packed[c] = make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
            *reinterpret_cast<uint4*>(base + kOffQ + r * 128 + ((c ^ (r & 7)) << 4)) = packed[c];
        proxy_fence();  // the tensor core reads Q through the async proxy
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ---------------- producer: K/V head slices, 8 pages per block ----------------
        if (lane == 0) {
            const int total_rows = static_cast<int>(a.n_pages) * a.page_rows;
            int issued = 0;
            for (int j = 0; j < nb; ++j) {
                const int st = j % kStages;
                if (j >= kStages &&
                    !wait_bar(&empty[st], static_cast<uint32_t>(j / kStages - 1) & 1u, abort_flag, a.err))
                    break;
                mbar_arrive_expect_tx(&full[st], kStageBytes);
                uint8_t* kt = base + kOffStage + st * kStageBytes;
                for (int i = 0; i < kPagesPerBlock; ++i) {
                    const int pi = j * kPagesPerBlock + i;
                    int rk = total_rows, rv = total_rows;  // out of range: zero fill
                    if (pi * kPageTokens < kmax) {
                        const uint32_t phys = pi < a.bt_stride ? __ldg(a.bt + static_cast<size_t>(s) * a.bt_stride + pi)
                                                               : kPageNone;
                        if (phys < a.n_pages) {
                            rk = static_cast<int>(phys) * a.page_rows + h * kPageTokens;
                            rv = static_cast<int>(phys) * a.page_rows + (a.nkv + h) * kPageTokens;
                        } else {
                            flag_error(a.err, kDevErrBadPage);
                        }
                    }
                    tma_load_2d(kt + i * kSliceBytes, &hmap, &full[st], 0, rk);
                    tma_load_2d(kt + kTile + i * kSliceBytes, &hmap, &full[st], 0, rv);
                }
                issued = j + 1;
            }
            if (*abort_flag) {  // wait (bounded) for the newest copy issued into each stage
                for (int st = 0; st < kStages && st < issued; ++st) {
                    const int last = st + ((issued - 1 - st) / kStages) * kStages;
                    mbar_wait(&full[st], static_cast<uint32_t>(last / kStages) & 1u);
                }
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            constexpr uint32_t kIdescS = instr_desc(kBlockKeys, kRows, false);
            constexpr uint32_t kIdescPV = instr_desc(kHeadDim, kRows, true);
            const uint32_t q_addr = smem_addr(base + kOffQ);
            const uint32_t p_addr = smem_addr(base + kOffP);
            for (int j = 0; j < nb; ++j) {
                const int st = j % kStages;
                if (!wait_bar(&full[st], static_cast<uint32_t>(j / kStages) & 1u, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t k_addr = smem_addr(base + kOffStage + st * kStageBytes);
                const uint32_t v_addr = k_addr + kTile;
#pragma unroll
                for (int kk = 0; kk < kHeadDim / 16; ++kk)
                    mma_f16(tmem + kColS, smem_desc(q_addr + 32 * kk, 16, 1024), smem_desc(k_addr + 32 * kk, 16, 1024),
                            kIdescS, kk > 0);
                mma_commit(s_full);
                if (!wait_bar(p_full, static_cast<uint32_t>(j) & 1u, abort_flag, a.err)) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kBlockKeys / 16; ++kk)
                    mma_f16(tmem + kColPV, smem_desc(p_addr + (kk / 4) * kTile + 32 * (kk % 4), 16, 1024),
                            smem_desc(v_addr + 2048 * kk, kTile, 1024), kIdescPV, kk > 0);
                mma_commit(pv_full);
                mma_commit(&empty[st]);
            }
            // Every MMA issued above has finished before TMEM is released.
            mma_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
    } else {
        // ---------------- softmax: thread r owns row r ----------------
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(32 * warp) << 16);
        const int t_chunk = rt + t_begin;  // chunk-relative token of this row
        const unsigned long long tmask = (tree && row_valid) ? __ldg(a.tree + q0 + t_row) : 0ull;
        float o[kHeadDim];
#pragma unroll
        for (int i = 0; i < kHeadDim; ++i) o[i] = 0.f;
        float m = -INFINITY, l = 0.f;
        for (int j = 0; j < nb; ++j) {
            if (!wait_bar(s_full, static_cast<uint32_t>(j) & 1u, abort_flag, a.err)) break;
            tc_fence_after();
            float sv[kBlockKeys];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float part[32];
                tmem_ld32(t_lane + kColS + 32 * c, part);
#pragma unroll
                for (int i = 0; i < 32; ++i) sv[32 * c + i] = part[i];
            }
            tmem_wait_ld();
            const int k0 = j * kBlockKeys;
            if (k0 + kBlockKeys > L) {  // the block reaches the chunk: mask per key
#pragma unroll
                for (int c = 0; c < kBlockKeys; ++c) {
                    const int key = k0 + c;
                    bool vis;
                    if (key < L) vis = true;
                    else if (key >= L + T) vis = false;
                    else if (tree) vis = (tmask >> (key - L)) & 1ull;
                    else vis = (key - L) <= t_chunk;
                    if (!vis || !row_valid) sv[c] = -INFINITY;
                }
            }
            float bm = -INFINITY;
#pragma unroll
            for (int c = 0; c < kBlockKeys; ++c) bm = fmaxf(bm, sv[c]);
            const float mn = fmaxf(m, bm);
            const float mu = (mn == -INFINITY) ? 0.f : mn;
            const float alpha = ex2f(m - mu);
            float sum = 0.f;
            uint8_t* prow = base + kOffP + r * 128;
#pragma unroll
            for (int c8 = 0; c8 < kBlockKeys / 8; ++c8) {
                float p[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    p[i] = ex2f(sv[8 * c8 + i] - mu);
                    sum += p[i];
                }
                const uint4 u = make_uint4(float2_to_bf16x2(p[0], p[1]), float2_to_bf16x2(p[2], p[3]),
                                           float2_to_bf16x2(p[4], p[5]), float2_to_bf16x2(p[6], p[7]));
                *reinterpret_cast<uint4*>(prow + (c8 / 8) * kTile + (((c8 % 8) ^ (r & 7)) << 4)) = u;
            }
            l = l * alpha + sum;
            m = mn;
            proxy_fence();  // P is read by the tensor core (async proxy)
            tc_fence_before();
            mbar_arrive(p_full);
            if (!wait_bar(pv_full, static_cast<uint32_t>(j) & 1u, abort_flag, a.err)) break;
            tc_fence_after();
            float pv[kHeadDim];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float part[32];
                tmem_ld32(t_lane + kColPV + 32 * c, part);
#pragma unroll
                for (int i = 0; i < 32; ++i) pv[32 * c + i] = part[i];
            }
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < kHeadDim; ++i) o[i] = fmaf(o[i], alpha, pv[i]);
        }
        if (row_valid && !*abort_flag) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            __nv_bfloat16* dst = a.out + (static_cast<size_t>(q0 + t_row) * a.n_q + h * a.group + rg) * kHeadDim;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                reinterpret_cast<uint4*>(dst)[c] =
                    make_uint4(float2_to_bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv),
                               float2_to_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                               float2_to_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                               float2_to_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 5)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
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
    if (c.dtype != KV_DTYPE_BF16) return KV_ERR_UNSUPPORTED;
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
    a.tile_tokens = kRows / group;
    a.rope = pool->rope;
    a.max_pos = c.max_positions;
    a.n_pages = c.n_pages;
    a.page_rows = static_cast<int>(pool->page_bytes / 128);
    a.out = static_cast<__nv_bfloat16*>(out);
    a.err = pool->dev_error;
    a.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(c.head_dim)));
    const dim3 grid((max_q + a.tile_tokens - 1) / a.tile_tokens, c.n_kv_heads, n_seqs);
    void* args[] = {&pool->head_map, &a};
    const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(&prefill_kernel), grid, dim3(kThreads), args,
                                           kSmemBytes, stream);
    return e == cudaSuccess ? KV_OK : KV_ERR_CUDA;
}

}  // namespace kvb200
