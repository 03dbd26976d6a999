// kv_decode_sched.cuh -- how the decode kernels split their work: every
// sequence's pages laid end to end (a scan over seq_lens), equal slices of
// at least kMinSlicePages pages per CTA of a persistent grid, and the
// contributor numbering of a sequence cut by slices.
#pragma once

#include "kv_common.cuh"

namespace kvb200 {

__device__ __forceinline__ int seq_lo(int n_tok, int window) {
    return (window > 0 && n_tok > window) ? n_tok - window : 0;
}

__device__ __forceinline__ int seq_pages(int n_tok, int window) {
    if (n_tok <= 0) return 0;
    return (n_tok + kPageTokens - 1) / kPageTokens - seq_lo(n_tok, window) / kPageTokens;
}

// Largest s in [0, n) with pstart[s] <= g (pstart is nondecreasing, pstart[0] = 0).
__device__ __forceinline__ int find_seq(const int* pstart, int n, int g) {
    int lo = 0, hi = n;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (pstart[mid] <= g) lo = mid; else hi = mid;
    }
    return lo;
}

// Fewest pages a CTA's slice holds (unless the batch has fewer in total).
constexpr int kMinSlicePages = 8;
// Partial rows a merging warp has in flight at once.
constexpr int kMergeBatch = 16;

// CTA whose slice [floor(c*T/G), floor((c+1)*T/G)) holds global page x.
__device__ __forceinline__ int cta_of(int x, int grid, int total) {
    return static_cast<int>(((static_cast<long long>(x) + 1) * grid - 1) / total);
}

// Warp 0 (all lanes): start[s] = units of unit_pages pages (the last one of
// a sequence may be partial) in sequences before s, start[n] = all units.
// With mult > 1, each unit counts mult times (work items per unit); a
// sequence with pages counts lead more (a cost charged to its start).
__device__ __forceinline__ void scan_units(const int32_t* seq_lens, int n, int window, int unit_pages, int* start,
                                           int lane, int mult = 1, int lead = 0) {
    const int per = (n + 31) >> 5;
    const int b = min(n, lane * per), e = min(n, b + per);
    auto units = [&](int s) {
        const int pages = seq_pages(__ldg(seq_lens + s), window);
        return pages > 0 ? mult * ((pages + unit_pages - 1) / unit_pages) + lead : 0;
    };
    int local = 0;
    for (int s = b; s < e; ++s) local += units(s);
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(~0u, incl, off);
        if (lane >= off) incl += y;
    }
    int run = incl - local;
    for (int s = b; s < e; ++s) {
        start[s] = run;
        run += units(s);
    }
    if (lane == 31) start[n] = incl;
}

// pstart[s] = pages of sequences before s, pstart[n] = all pages.
__device__ __forceinline__ void scan_pages(const int32_t* seq_lens, int n, int window, int* pstart, int lane) {
    scan_units(seq_lens, n, window, 1, pstart, lane);
}

}  // namespace kvb200
