// kv_noalloc.cu -- paged decode attention that allocates no device memory.
//
// Who this is for: callers that cannot call cudaMalloc -- for example a host
// runtime whose device memory all comes from a fixed arena it manages
// itself, or a caller that is not allowed to grow its device footprint after
// start-up.  Such a caller cannot create a kv_pool (creation allocates the
// pages, the RoPE table and the split workspace), so this entry point takes
// every input and output from the caller and keeps its only scratch -- the
// per-split partial results and the per-sequence merge counters of the
// decode kernel -- in one file-scope __device__ array, g_scratch.
//
// Limits: 4 MiB of scratch per device, at most kNoAllocMaxSeqs sequences and
// kNoAllocMaxQHeads query heads per call; larger requests are rejected with
// KV_ERR_INVALID before anything is launched.  Every GPU that loads this
// library holds the 4 MiB until the process exits.
//
// Sharing: all calls on a device use the same array.  A call clears the
// counters it uses (cudaMemsetAsync on its stream) before its kernel runs;
// the partial results need no clearing (each call writes them before it
// reads them).  Two calls whose kernels overlap on the GPU -- on different
// streams, or from different host threads -- race on the array; serialise
// them, e.g. on one stream.
//
// Set-up: the first call on a device, with that device current, looks up
// the array's device address (cudaGetSymbolAddress), the SM count and the
// kernel's launch shape; later calls reuse them.  Make that first call
// before any stream capture begins.  The address is kept until the process
// exits, so a device reset after the first call is not supported.
//
// Kernel: the CUDA-core decode kernel for both dtypes (kv_decode_attn runs
// the tensor-core kernel for bf16 pools), through its raw launch interface.
#include <cudaTypedefs.h>

#include <mutex>

#include "kv_common.cuh"
#include "kv_pool_impl.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kNoAllocMaxSeqs = 1024;
constexpr int kNoAllocMaxQHeads = 32;
constexpr size_t kCountersBytes = kNoAllocMaxSeqs * sizeof(int);
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code `g_scratch` names a host-side stand-in,
// not device memory: kernels are given the address cudaGetSymbolAddress
// returns for the current device.
static __device__ __align__(256) unsigned char g_scratch[kNoAllocScratchBytes];

struct ShapeSetup {
    int dtype = -1, nkv = 0, group = 0;
    int grid = 0;
    size_t smem = 0;
};

struct DeviceSetup {
    bool ready = false;
    unsigned char* scratch = nullptr;  // device address of g_scratch on this device
    int sm_count = 0;
    ShapeSetup shapes[8];
    int n_shapes = 0;
};

std::mutex g_mu;
DeviceSetup g_dev[kMaxDevices];
// The driver's tensor-map encoder; looked up once, under g_mu.
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int setup_device(int dev, DeviceSetup& d) {
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return KV_ERR_CUDA;
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_scratch) != cudaSuccess || ptr == nullptr) return KV_ERR_CUDA;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return KV_ERR_CUDA;
    d.scratch = static_cast<unsigned char*>(ptr);
    d.ready = true;
    return KV_OK;
}

const ShapeSetup* setup_shape(int dev, DeviceSetup& d, int dtype, int nkv, int group, int* rc) {
    for (int i = 0; i < d.n_shapes; ++i)
        if (d.shapes[i].dtype == dtype && d.shapes[i].nkv == nkv && d.shapes[i].group == group)
            return &d.shapes[i];
    if (d.n_shapes == 8) {
        *rc = KV_ERR_UNSUPPORTED;
        return nullptr;
    }
    ShapeSetup s;
    s.dtype = dtype;
    s.nkv = nkv;
    s.group = group;
    *rc = kvb200::decode_configure_raw(dtype, nkv, group, kNoAllocMaxSeqs, dev, d.sm_count, &s.grid,
                                       &s.smem);
    if (*rc != KV_OK) return nullptr;
    d.shapes[d.n_shapes] = s;
    return &d.shapes[d.n_shapes++];
}

int encode_map(PFN_cuTensorMapEncodeTiled_v12000 encode, const void* pages, uint32_t n_pages, int dtype, int nkv,
               CUtensorMap* map) {
    const cuuint64_t elem = dtype == KV_DTYPE_BF16 ? 2 : 4;
    const cuuint64_t row_elems = 128 / elem;
    const cuuint64_t page_rows = 2ull * nkv * kvb200::kPageTokens * kvb200::kHeadDim * elem / 128;
    const cuuint64_t gdim[2] = {row_elems, static_cast<cuuint64_t>(n_pages) * page_rows};
    const cuuint64_t gstride[1] = {128};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(row_elems),
                               static_cast<cuuint32_t>(page_rows < 256 ? page_rows : 256)};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode(map,
                              dtype == KV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                              2, const_cast<void*>(pages), gdim, gstride, box, estride,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? KV_OK : KV_ERR_INVALID;
}

}  // namespace

extern "C" int kv_decode_attn_noalloc(const void* pages, uint32_t n_pages, int32_t dtype,
                                      int32_t n_q_heads, int32_t n_kv_heads, const void* rope_cs,
                                      int32_t max_positions, const void* q,
                                      const uint32_t* block_tables, int32_t bt_stride,
                                      const int32_t* seq_lens, int32_t n_seqs, int32_t window,
                                      void* out, int32_t* status, void* stream) {
    using namespace kvb200;
    if (dtype != KV_DTYPE_F32 && dtype != KV_DTYPE_BF16) return KV_ERR_INVALID;
    if (n_kv_heads <= 0 || n_q_heads <= 0 || n_q_heads % n_kv_heads != 0) return KV_ERR_INVALID;
    if (n_q_heads > kNoAllocMaxQHeads || n_seqs < 0 || n_seqs > kNoAllocMaxSeqs) return KV_ERR_INVALID;
    if (!status || window < 0) return KV_ERR_INVALID;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n_seqs == 0) return cudaMemsetAsync(status, 0, sizeof(int32_t), st) == cudaSuccess ? KV_OK : KV_ERR_CUDA;
    if (!pages || n_pages == 0 || !rope_cs || max_positions <= 0 || !q || !block_tables ||
        bt_stride <= 0 || !seq_lens || !out)
        return KV_ERR_INVALID;
    const uint64_t page_rows = 2ull * n_kv_heads * kPageTokens * kHeadDim * (dtype == KV_DTYPE_BF16 ? 2 : 4) / 128;
    if (static_cast<uint64_t>(n_pages) * page_rows >= (1ull << 31)) return KV_ERR_INVALID;

    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return KV_ERR_CUDA;
    const ShapeSetup* shape = nullptr;
    unsigned char* scratch = nullptr;
    PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        DeviceSetup& d = g_dev[dev];
        if (!d.ready) {
            const int rc = setup_device(dev, d);
            if (rc != KV_OK) return rc;
        }
        int rc = KV_OK;
        shape = setup_shape(dev, d, dtype, n_kv_heads, n_q_heads / n_kv_heads, &rc);
        if (!shape) return rc;
        scratch = d.scratch;
        encode = g_encode;
    }
    // Scratch layout: merge counters, then (max, sum) pairs, then partial outputs.
    const size_t slots = 2 * static_cast<size_t>(shape->grid);
    const size_t ml_bytes = slots * n_q_heads * 2 * sizeof(float);
    const size_t o_bytes = slots * n_q_heads * kHeadDim * sizeof(float);
    if (kCountersBytes + ml_bytes + o_bytes > kNoAllocScratchBytes) return KV_ERR_INVALID;

    CUtensorMap map;
    int rc = encode_map(encode, pages, n_pages, dtype, n_kv_heads, &map);
    if (rc != KV_OK) return rc;

    int* counters = reinterpret_cast<int*>(scratch);
    if (cudaMemsetAsync(counters, 0, static_cast<size_t>(n_seqs) * sizeof(int), st) != cudaSuccess ||
        cudaMemsetAsync(status, 0, sizeof(int32_t), st) != cudaSuccess)
        return KV_ERR_CUDA;

    DecodeRaw r;
    r.dtype = dtype;
    r.nkv = n_kv_heads;
    r.group = n_q_heads / n_kv_heads;
    r.map = &map;
    r.q = q;
    r.out = out;
    r.bt = block_tables;
    r.bt_stride = bt_stride;
    r.seq_lens = seq_lens;
    r.n_seqs = n_seqs;
    r.window = window;
    r.rope = static_cast<const float2*>(rope_cs);
    r.max_pos = max_positions;
    r.n_pages = n_pages;
    r.part_ml = reinterpret_cast<float*>(scratch + kCountersBytes);
    r.part_o = reinterpret_cast<float*>(scratch + kCountersBytes + ml_bytes);
    r.counters = counters;
    r.err = status;
    r.grid = shape->grid;
    r.smem = shape->smem;
    return launch_decode_raw(r, st);
}
