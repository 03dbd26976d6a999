// kv_common.cuh -- shared device helpers for the sm_100a paged-KV kernels.
//
// Page layout (build-defined; the reference's KV is a contiguous
// [n_kv, cap, head_dim] fp32 buffer per layer, crates/llm-engine/src/lfm2.rs:188-203):
//   page p = K block [n_kv][P][d] followed by V block [n_kv][P][d], element
//   type T (float or bf16).  Token t of a sequence sits in page bt[t / P],
//   slot t % P.  Viewed as 128-byte rows, one page is PAGE_ROWS rows, which is
//   how the TMA tensor map addresses it (row coordinate = page * PAGE_ROWS).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/llmhost_kv.h"

namespace kvb200 {

constexpr int kHeadDim = 64;
constexpr int kPageTokens = 16;
constexpr uint32_t kPageNone = 0xFFFFFFFFu;

// Device error word bits (read back by kv_last_error).
constexpr int kDevErrBadPage = 1;   // a block-table entry was >= n_pages
constexpr int kDevErrTimeout = 2;   // an mbarrier wait ran past its time limit
constexpr int kDevErrBadPos = 4;    // a RoPE position was >= max_positions
constexpr int kDevErrBadArg = 8;    // a device-side length or offset was out of range

// A bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Workspace shared by the kernels of one pool (device memory).
struct DeviceWs {
    int error;      // OR of kDevErr* bits
    int pad[31];
};

__device__ __forceinline__ void flag_error(int* err, int bits) { atomicOr(err, bits); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy (cp.async, L2 only) and its group controls.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier ------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// Test whether the phase with the given parity has completed.  The waiting
// thread may be suspended by the hardware for up to kSuspendHintNs (it wakes
// as soon as the phase completes), so a waiting warp does not spin on the
// issue slots that computing warps need.
constexpr uint32_t kSuspendHintNs = 1000000u;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// kWaitLimitNs.  Returns false on timeout (the caller flags the error word).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// ---- TMA (no multicast anywhere in this library) --------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch.  grid_dep_wait: block until the grids this
// one depends on have completed and their memory is visible (a no-op when the
// launch has no programmatic dependency); every global access of a kernel
// launched with programmatic serialization comes after it.
// grid_dep_trigger: let the next grid in the stream launch once every CTA of
// this one has triggered or exited (its CTAs then do their set-up on SMs this
// grid has left and wait in grid_dep_wait).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrive at a named barrier without waiting for it.
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- element helpers -------------------------------------------------------
// Two bf16 packed in a 32-bit word -> float2 (exact widening).
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ uint32_t float2_to_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // round to nearest even
    return *reinterpret_cast<uint32_t*>(&h);
}

// 128-byte swizzle used by the TMA loads: 16-byte chunk c of 128-byte row r
// lands at chunk c ^ (r & 7).  Returns the byte offset inside a 1024-byte
// aligned buffer of the chunk that holds linear byte offset `lin`.
__device__ __forceinline__ uint32_t swz128(uint32_t lin) {
    const uint32_t row = lin >> 7;
    const uint32_t chunk = (lin >> 4) & 7u;
    return (row << 7) | (((chunk ^ (row & 7u)) << 4)) | (lin & 15u);
}


// RMSNorm scale of one head row of 64 values (crates/llm-cpu/src/ops.rs:12-18):
// the sum of squares in double, in dimension order, as separate rounded
// products and sums (Rust does not contract), then
// (float)(1 / sqrt(sumsq / 64 + eps)) with IEEE square root and reciprocal.
// The row is read with 16-byte loads (it must be 16-byte aligned) and each
// chunk's squares are taken before the running sum reaches them, so the
// 64-term chain of rounded adds is the only serial part.  Out of line:
// called once per row, it must not grow the kernels' hot code.
__device__ __forceinline__ float rms_mean_to_scale(double s, float eps) {
    const double m = __dadd_rn(__dmul_rn(s, 1.0 / 64.0), static_cast<double>(eps));
    return __double2float_rn(__drcp_rn(__dsqrt_rn(m)));
}
static __device__ __noinline__ float rms_scale_row(const __nv_bfloat16* row, float eps) {
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    double s = 0.0;
    uint4 w = r4[0];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 wn = r4[c < 7 ? c + 1 : c];  // the next chunk in flight
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        double sq[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = bf16x2_to_float2(u[e]);
            sq[2 * e] = __dmul_rn(static_cast<double>(f.x), static_cast<double>(f.x));
            sq[2 * e + 1] = __dmul_rn(static_cast<double>(f.y), static_cast<double>(f.y));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) s = __dadd_rn(s, sq[i]);
        w = wn;
    }
    return rms_mean_to_scale(s, eps);
}
static __device__ __noinline__ float rms_scale_row(const float* row, float eps) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    double s = 0.0;
    float4 w = r4[0];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const float4 wn = r4[c < 15 ? c + 1 : c];
        const double sq[4] = {__dmul_rn(static_cast<double>(w.x), static_cast<double>(w.x)),
                              __dmul_rn(static_cast<double>(w.y), static_cast<double>(w.y)),
                              __dmul_rn(static_cast<double>(w.z), static_cast<double>(w.z)),
                              __dmul_rn(static_cast<double>(w.w), static_cast<double>(w.w))};
#pragma unroll
        for (int i = 0; i < 4; ++i) s = __dadd_rn(s, sq[i]);
        w = wn;
    }
    return rms_mean_to_scale(s, eps);
}

// x' = w * (x * scale): RMSNorm's two rounded products (ops.rs:19-21).
__device__ __forceinline__ float rms_apply(float x, float scale, float w) { return __fmul_rn(w, __fmul_rn(x, scale)); }

}  // namespace kvb200
