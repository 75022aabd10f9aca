// rsort_keys_static: the in-place full-width keys sort with all of its scratch
// (scratch keys, digit bins, look-back words, pass counters) taken from one
// file-scope device array instead of caller-provided memory.
//
// Who needs it: callers that cannot allocate device memory at the point where
// they sort.  Code recording a CUDA graph by stream capture may not call
// cudaMalloc while capturing; a plugin hosted by a framework that owns every
// device byte through its own pool (PyTorch's caching allocator, an RMM pool,
// rccl-memory's DeviceAllocator) may have no way to reach that pool from the
// sorting call site; and latency-critical loops cannot afford an allocation
// and the synchronization it can imply.  The regular entry points stay
// allocation free as well, but they need the caller to own the workspace;
// this one needs nothing but the keys.
//
// Limits and sharing:
//  - at most RSORT_STATIC_MAX_ITEMS keys per call (any of the six key types);
//    larger inputs are rejected with RSORT_WORKSPACE_TOO_SMALL
//  - the array (RSORT_STATIC_SCRATCH_BYTES) is part of the library's device
//    image, so every GPU that loads the library holds it until process exit
//  - every call on a device uses the same array and leaves its contents
//    behind: calls whose work overlaps on the GPU (other streams, other host
//    threads) race on it and must be serialized by the caller
//  - the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current, and looks it up again
//    when a different context is current on that device (after a device
//    reset); make that first call before any stream capture begins
//  - a bounded device wait that gives up is not reported by this call (the
//    sticky status word lives in the shared array and is cleared by the next
//    call); the output is then unspecified
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/rsort_b200.h"
#include "rsort_internal.cuh"
#include "rsort_kernels.cuh"

namespace {

constexpr size_t kMaxItems = RSORT_STATIC_MAX_ITEMS;
constexpr size_t kAlign = 256;
constexpr size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Region layout inside the static array (bytes).
constexpr size_t kKeysBytes = align_up(kMaxItems * 8);
constexpr size_t kBinsBytes = align_up(8 * 256 * sizeof(uint64_t));
constexpr size_t kCountersBytes = align_up(rsort::CTR_WORDS * sizeof(int32_t));
// Look-back words: 256 64-bit words per tile; the smallest keys-only tile
// (8-byte keys) gives the largest tile count.
constexpr size_t kMinTile = size_t(rsort::onesweep_tile(8, 0)) < size_t(rsort::onesweep_tile(4, 0))
                                ? size_t(rsort::onesweep_tile(8, 0))
                                : size_t(rsort::onesweep_tile(4, 0));
constexpr size_t kMaxTiles = (kMaxItems + kMinTile - 1) / kMinTile;
constexpr size_t kLookbackBytes = align_up(kMaxTiles * 256 * sizeof(uint64_t));
constexpr size_t kTotalBytes = kKeysBytes + kBinsBytes + kCountersBytes + kLookbackBytes;
static_assert(kTotalBytes <= RSORT_STATIC_SCRATCH_BYTES, "static scratch too small");

}  // namespace

// The scratch array.  In host code this name is only a stand-in for the
// symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_rsort_static_scratch[RSORT_STATIC_SCRATCH_BYTES];

namespace {

// Cached device address of the array, per device ordinal and the context that
// was current when it was resolved: a context that is torn down and recreated
// (cudaDeviceReset) may load the module at another address, so a different
// current context resolves the address again.
struct StaticAddress {
    void *ctx = nullptr;
    unsigned char *ptr = nullptr;
};
std::mutex g_static_mutex;
StaticAddress g_static_addr[64];

// Once per device (and context), with that device current: resolve the
// array's device address.
rsort_status static_scratch(unsigned char **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return rsort::record_failure(RSORT_CUDA_ERROR, "static scratch: cudaGetDevice");
    if (dev < 0 || dev >= 64)
        return rsort::record_failure(RSORT_UNSUPPORTED_TARGET, "static scratch: device ordinal");
    void *ctx = nullptr;
    if (rsort::current_context(&ctx) != cudaSuccess)
        return rsort::record_failure(RSORT_CUDA_ERROR, "static scratch: current context");
    std::lock_guard<std::mutex> lock(g_static_mutex);
    StaticAddress &a = g_static_addr[dev];
    if (!a.ptr || a.ctx != ctx) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_rsort_static_scratch);
        if (e != cudaSuccess || !p)
            return rsort::record_failure(RSORT_CUDA_ERROR, "static scratch: cudaGetSymbolAddress");
        a.ptr = static_cast<unsigned char *>(p);
        a.ctx = ctx;
    }
    *out = a.ptr;
    return RSORT_OK;
}

}  // namespace

extern "C" rsort_status rsort_keys_static(rsort_key_t key, int descending, void *d_keys, size_t n,
                                          rsort_stream_t stream) {
    if (int(key) < RSORT_U32 || int(key) > RSORT_F64)
        return rsort::record_failure(RSORT_BAD_ARGUMENT, "static keys: key type (32/64-bit keys)");
    if (n > kMaxItems)
        return rsort::record_failure(RSORT_WORKSPACE_TOO_SMALL,
                                     "static keys (at most RSORT_STATIC_MAX_ITEMS)", kMaxItems, n);
    if (n == 0) return RSORT_OK;
    if (!d_keys) return rsort::record_failure(RSORT_BAD_ARGUMENT, "static keys: null buffer");
    rsort_controls c{};
    rsort_status st = rsort_controls_query(key, 0, n, &c);
    if (st != RSORT_OK) return st;
    if (c.lookback * sizeof(int32_t) > kLookbackBytes)
        return rsort::record_failure(RSORT_WORKSPACE_TOO_SMALL, "static keys: look-back region",
                                     kLookbackBytes, c.lookback * sizeof(int32_t));
    if (c.bins * sizeof(uint64_t) > kBinsBytes)
        return rsort::record_failure(RSORT_WORKSPACE_TOO_SMALL, "static keys: bins region",
                                     kBinsBytes, c.bins * sizeof(uint64_t));
    if (c.counters * sizeof(int32_t) > kCountersBytes)
        return rsort::record_failure(RSORT_WORKSPACE_TOO_SMALL, "static keys: counters region",
                                     kCountersBytes, c.counters * sizeof(int32_t));
    unsigned char *base = nullptr;
    st = static_scratch(&base);
    if (st != RSORT_OK) return st;
    unsigned char *scratch_keys = base;
    uint64_t *bins = reinterpret_cast<uint64_t *>(base + kKeysBytes);
    int32_t *counters = reinterpret_cast<int32_t *>(base + kKeysBytes + kBinsBytes);
    int32_t *lookback = reinterpret_cast<int32_t *>(base + kKeysBytes + kBinsBytes + kCountersBytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The previous call's contents stay in the array: the pass counters and
    // the sticky status word must start at zero (the sort itself zeroes its
    // bins and look-back words).
    if (c.counters) {
        const cudaError_t e = cudaMemsetAsync(counters, 0, c.counters * sizeof(int32_t), s);
        if (e != cudaSuccess)
            return rsort::record_failure(RSORT_CUDA_ERROR, "static keys: counters reset");
    }
    return rsort_keys(key, descending, d_keys, scratch_keys, n, n, c.bins ? bins : nullptr, c.bins,
                      c.lookback ? lookback : nullptr, c.lookback,
                      c.counters ? counters : nullptr, c.counters, stream);
}
