// C ABI of the B200 radix sort: validation, control-region sizing and the
// pass schedule of one sort.  Replaces the reference's Rust pass control
// (rccl-cub/src/radix.rs:364-876) together with the kernel-trait seam it
// drives (rccl-cub/src/radix.rs:205-362).
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/rsort_b200.h"
#include "rsort_device.cuh"
#include "rsort_dist.cuh"
#include "rsort_internal.cuh"
#include "rsort_kernels.cuh"
#include "rsort_records.cuh"

using namespace rsort;

namespace {

thread_local rsort_error_info g_last_error = {RSORT_OK, "", 0, 0, 0, 0, 0};
thread_local uint64_t g_launches = 0;

// Benchmark instrumentation: when enabled, every kernel launch of the calling
// host thread is bracketed by two CUDA events on the launch stream.
struct ProfiledLaunch {
    int kernel;
    cudaEvent_t start, stop;
};
thread_local bool g_profile = false;
thread_local std::vector<ProfiledLaunch> g_profiled;
thread_local std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pooled_event() {
    if (!g_event_pool.empty()) {
        cudaEvent_t e = g_event_pool.back();
        g_event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

}  // namespace

namespace rsort {

LaunchScope::LaunchScope(int k, cudaStream_t s) : kernel(k), stream(s), on(g_profile), rec(nullptr) {
    ++g_launches;
    if (on) {
        auto *r = new ProfiledLaunch{k, pooled_event(), pooled_event()};
        cudaEventRecord(r->start, stream);
        rec = r;
    }
}

LaunchScope::~LaunchScope() {
    if (on) {
        auto *r = static_cast<ProfiledLaunch *>(rec);
        cudaEventRecord(r->stop, stream);
        g_profiled.push_back(*r);
        delete r;
    }
}

rsort_status record_failure(rsort_status s, const char *role, size_t expected, size_t actual) {
    g_last_error.status = s;
    g_last_error.role = role;
    g_last_error.expected = expected;
    g_last_error.actual = actual;
    g_last_error.begin_bit = g_last_error.end_bit = g_last_error.key_bits = 0;
    return s;
}

cudaError_t current_context(void **ctx) {
    using Fn = CUresult (*)(CUcontext *);
    static Fn fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !f) return cudaErrorNotSupported;
        fn = reinterpret_cast<Fn>(f);
    }
    CUcontext c = nullptr;
    if (fn(&c) != CUDA_SUCCESS) return cudaErrorInvalidValue;
    *ctx = c;
    return cudaSuccess;
}

}  // namespace rsort

namespace {

rsort_status fail(rsort_status s, const char *role, size_t expected = 0, size_t actual = 0) {
    return record_failure(s, role, expected, actual);
}

rsort_status fail_bits(unsigned begin, unsigned end, unsigned key_bits) {
    fail(RSORT_INVALID_BIT_RANGE, "radix bit range");
    g_last_error.begin_bit = begin;
    g_last_error.end_bit = end;
    g_last_error.key_bits = key_bits;
    return RSORT_INVALID_BIT_RANGE;
}

rsort_status cuda_fail(cudaError_t e, const char *role) {
    (void)e;
    return fail(RSORT_CUDA_ERROR, role);
}

// A scratch blob is carved into 256-byte aligned regions (8-byte keys,
// 16-byte aligned look-back words), so the blob must start on 256 bytes.
// Checked before any launch: a misaligned region would fault the kernels.
rsort_status check_blob(const void *d_scratch, const char *role) {
    if ((reinterpret_cast<uintptr_t>(d_scratch) & 255) != 0)
        return fail(RSORT_BAD_ARGUMENT, role, 256, reinterpret_cast<uintptr_t>(d_scratch) & 255);
    return RSORT_OK;
}

// bytes_per_item * n bytes of a scratch region, or false past the radix item
// limit or past 2^56 bytes (far beyond any device, and small enough that a
// layout's sum of regions cannot wrap a size_t).
bool region_bytes(size_t bytes_per_item, size_t n, size_t *out) {
    constexpr size_t kMaxRegion = size_t(1) << 56;
    if (n > RSORT_MAX_ITEMS || (bytes_per_item && n > kMaxRegion / bytes_per_item)) return false;
    *out = bytes_per_item * n;
    return true;
}

bool key_ok(rsort_key_t k) { return int(k) >= RSORT_U32 && int(k) <= RSORT_BF16; }
int key_bytes(rsort_key_t k) {
    switch (k) {
        case RSORT_U8:
        case RSORT_I8: return 1;
        case RSORT_U16:
        case RSORT_I16:
        case RSORT_F16:
        case RSORT_BF16: return 2;
        case RSORT_U64:
        case RSORT_I64:
        case RSORT_F64: return 8;
        default: return 4;
    }
}
int key_kind(rsort_key_t k) {
    switch (k) {
        case RSORT_I32:
        case RSORT_I64:
        case RSORT_I8:
        case RSORT_I16: return KIND_SINT;
        case RSORT_F32:
        case RSORT_F64:
        case RSORT_F16:
        case RSORT_BF16: return KIND_FLOAT;
        default: return KIND_UINT;
    }
}
// The sample-sort steps and the merges are built for 32- and 64-bit keys.
bool wide_key(rsort_key_t k) { return key_ok(k) && key_bytes(k) >= 4; }
bool value_ok(size_t vb) { return vb == 0 || vb == 1 || vb == 2 || vb == 4 || vb == 8 || vb == 16; }

struct DeviceInfo {
    int sm_count = 0;
    bool supported = false;
    bool probed = false;
};

std::mutex g_dev_mutex;
DeviceInfo g_dev[64];

rsort_status device_info(DeviceInfo *out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(RSORT_UNSUPPORTED_TARGET, "device ordinal");
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceInfo &d = g_dev[dev];
    if (!d.probed) {
        int major = 0, sms = 0;
        e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        d.sm_count = sms;
        d.supported = major == 10;  // the kernels are built for sm_100a only
        d.probed = true;
    }
    *out = d;
    if (!d.supported)
        return fail(RSORT_UNSUPPORTED_TARGET, "radix sort is built for sm_100a (B200) only");
    return RSORT_OK;
}

}  // namespace

rsort_status rsort::current_sm_count(int *sm_count) {
    DeviceInfo d;
    const rsort_status st = device_info(&d);
    if (st == RSORT_OK) *sm_count = d.sm_count;
    return st;
}

namespace {

size_t tiles_for(size_t n, int kb, int vb) {
    const size_t tile = size_t(onesweep_tile(kb, vb));
    return (n + tile - 1) / tile;
}

bool single_route(size_t n, int kb, int vb) { return n <= policy800_single_tile_items(kb, vb); }

struct Controls {
    uint64_t *bins;
    size_t nbins;
    int32_t *lookback;
    size_t nlookback;
    int32_t *counters;
    size_t ncounters;
};

// rccl-cub/src/radix.rs:388-423 validate_controls, with the lengths taken from
// rsort_controls_query.
rsort_status validate_controls(const Controls &c, size_t n, int kb, int vb) {
    const size_t passes = size_t(kb);  // full-width passes: 8 * kb bits / 8
    const size_t need_bins = passes * RADIX;
    const size_t need_lookback = tiles_for(n, kb, vb) * RADIX * 2;
    if (c.nbins < need_bins) return fail(RSORT_WORKSPACE_TOO_SMALL, "radix bins", need_bins, c.nbins);
    if (c.nlookback != need_lookback)
        return fail(RSORT_LENGTH_MISMATCH, "radix lookback", need_lookback, c.nlookback);
    if (c.ncounters < size_t(CTR_WORDS))
        return fail(RSORT_WORKSPACE_TOO_SMALL, "radix pass counters", CTR_WORDS, c.ncounters);
    if (!c.bins || !c.lookback || !c.counters) return fail(RSORT_BAD_ARGUMENT, "null control region");
    if ((reinterpret_cast<uintptr_t>(c.lookback) & 15) != 0)
        return fail(RSORT_BAD_ARGUMENT, "radix lookback alignment (16 bytes)");
    if ((reinterpret_cast<uintptr_t>(c.bins) & 7) != 0)
        return fail(RSORT_BAD_ARGUMENT, "radix bins alignment (8 bytes)");
    return RSORT_OK;
}

// One sort over a DoubleBuffer.  values == nullptr pointers for keys-only.
// total: float keys in IEEE total order (no zero fold; the named-order merge
// sort entry points), else the reference's radix order.
rsort_status sort_buffer(rsort_key_t key, int descending, void *kf, void *ks, void *vf, void *vs,
                         size_t vb, size_t n, unsigned begin_bit, unsigned end_bit,
                         int *current_is_first, const Controls &c, cudaStream_t stream,
                         bool total = false) {
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    if (!value_ok(vb)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    if (!current_is_first) return fail(RSORT_BAD_ARGUMENT, "null selector");
    const int kb = key_bytes(key);
    const unsigned kbits = unsigned(kb) * 8;
    // rccl-cub/src/radix.rs:370-376
    if (begin_bit > end_bit || end_bit > kbits) return fail_bits(begin_bit, end_bit, kbits);
    const unsigned passes = (end_bit - begin_bit + 7) / 8;
    // rccl-cub/src/radix.rs:467-469
    if (n == 0 || passes == 0) return RSORT_OK;
    if (n > RSORT_MAX_ITEMS)
        return fail(RSORT_SIZE_OVERFLOW, "radix item count (at most RSORT_MAX_ITEMS)",
                    RSORT_MAX_ITEMS, n);
    if (!kf || !ks || (vb && (!vf || !vs))) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    {
        rsort_status st = check_alignment(addr(kf) | addr(ks), size_t(kb), "radix keys alignment");
        if (st == RSORT_OK)
            st = check_alignment(addr(vf) | addr(vs), vb, "radix values alignment");
        if (st != RSORT_OK) return st;
    }
    const bool cur_first = *current_is_first != 0;
    void *kin = cur_first ? kf : ks;
    void *kout = cur_first ? ks : kf;
    void *vin = cur_first ? vf : vs;
    void *vout = cur_first ? vs : vf;
    const int kind = total && key_kind(key) == KIND_FLOAT ? KIND_FLOAT_TOTAL : key_kind(key);

    // rccl-cub/src/radix.rs:470-492: single-tile route, one selector flip.
    DeviceInfo dev;
    rsort_status st;
    if (single_route(n, kb, int(vb))) {
        st = device_info(&dev);
        if (st != RSORT_OK) return st;
        SingleArgs a{kin, kout, vin, vout, uint32_t(n), begin_bit, end_bit, kind, descending ? 1 : 0};
        cudaError_t e;
        {
            LaunchScope scope(RSORT_KERNEL_SINGLE_TILE, stream);
            e = launch_single_tile(kb, int(vb), a, stream);
        }
        if (e != cudaSuccess) return cuda_fail(e, "single-tile launch");
        *current_is_first = cur_first ? 0 : 1;
        return RSORT_OK;
    }

    st = validate_controls(c, n, kb, int(vb));
    if (st != RSORT_OK) return st;
    st = device_info(&dev);
    if (st != RSORT_OK) return st;
    const size_t tiles = tiles_for(n, kb, int(vb));
    if (tiles > 0x7fffffffull) return fail(RSORT_SIZE_OVERFLOW, "radix tile count");

    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_INIT, stream);
        // The status word (CTR_STATUS) is sticky: only rsort_check_device_status
        // clears it, so a give-up in any earlier sort stays visible.
        e = launch_init(c.bins, size_t(passes) * RADIX, c.counters, CTR_STATUS, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "init launch");

    HistArgs h{};
    h.keys = kin;
    h.n = n;
    h.bins = c.bins;
    h.lookback = reinterpret_cast<uint64_t *>(c.lookback);
    h.lookback_words = uint64_t(tiles) * RADIX;
    h.done = c.counters + CTR_HIST_DONE;
    h.passes = passes;
    h.begin_bit = begin_bit;
    h.end_bit = end_bit;
    h.kind = kind;
    h.desc = descending ? 1 : 0;
    h.vector_ok = (reinterpret_cast<uintptr_t>(kin) & 15) == 0;
    h.hot = c.counters + CTR_HOT_FLAGS;
    {
        LaunchScope scope(RSORT_KERNEL_HISTOGRAM, stream);
        e = launch_histogram(kb, h, dev.sm_count, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "histogram launch");

    // rccl-cub/src/radix.rs:518-552: one onesweep pass per 8-bit digit, each
    // flipping the selector.
    bool first_is_src = cur_first;
    for (unsigned p = 0; p < passes; ++p) {
        PassArgs a{};
        a.keys_in = first_is_src ? kf : ks;
        a.keys_out = first_is_src ? ks : kf;
        a.values_in = first_is_src ? vf : vs;
        a.values_out = first_is_src ? vs : vf;
        a.n = n;
        a.bins = c.bins + size_t(p) * RADIX;
        a.lookback = reinterpret_cast<uint64_t *>(c.lookback);
        a.tile_counter = c.counters + CTR_TILE + p;
        a.status = c.counters + CTR_STATUS;
        a.shift = begin_bit + 8 * p;
        const unsigned bits = (end_bit - a.shift) < 8 ? (end_bit - a.shift) : 8;
        a.mask = (1u << bits) - 1;
        a.kind = kind;
        a.desc = descending ? 1 : 0;
        a.first = p == 0;
        a.last = p + 1 == passes;
        a.tag = p + 1;
        a.hot = c.counters + CTR_HOT_FLAGS;
        a.pass = p;
        // Passes after the first: the RANK_RUNS form goes first and takes
        // the pass when it and the pass before are hot (long runs of equal
        // keys); otherwise it exits and the plain pass claims every tile.
        if (p > 0 && kb >= 4 && n >= RUNS_MIN_ITEMS) {
            LaunchScope scope(RSORT_KERNEL_ONESWEEP_RUNS, stream);
            e = launch_onesweep_runs(kb, int(vb), a, tiles, stream);
            if (e != cudaSuccess) return cuda_fail(e, "onesweep launch");
        }
        {
            LaunchScope scope(RSORT_KERNEL_ONESWEEP, stream);
            e = launch_onesweep(kb, int(vb), a, tiles, stream);
        }
        if (e != cudaSuccess) return cuda_fail(e, "onesweep launch");
        first_is_src = !first_is_src;
    }
    *current_is_first = first_is_src ? 1 : 0;
    return RSORT_OK;
}

}  // namespace

extern "C" {

rsort_status rsort_controls_query(rsort_key_t key, size_t value_bytes, size_t n,
                                  rsort_controls *out) {
    if (!out) return fail(RSORT_BAD_ARGUMENT, "null output");
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    if (!value_ok(value_bytes)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    if (n > RSORT_MAX_ITEMS)
        return fail(RSORT_SIZE_OVERFLOW, "radix item count (at most RSORT_MAX_ITEMS)",
                    RSORT_MAX_ITEMS, n);
    const int kb = key_bytes(key);
    if (single_route(n, kb, int(value_bytes))) {
        out->bins = out->lookback = out->counters = 0;
        return RSORT_OK;
    }
    out->bins = size_t(kb) * RADIX;
    out->lookback = tiles_for(n, kb, int(value_bytes)) * RADIX * 2;
    out->counters = CTR_WORDS;
    return RSORT_OK;
}

rsort_status rsort_keys_buffer(rsort_key_t key, int descending, void *d_first, void *d_second,
                               size_t n, unsigned begin_bit, unsigned end_bit,
                               int *current_is_first, uint64_t *bins, size_t nbins,
                               int32_t *lookback, size_t nlookback, int32_t *counters,
                               size_t ncounters, rsort_stream_t stream) {
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return sort_buffer(key, descending, d_first, d_second, nullptr, nullptr, 0, n, begin_bit,
                       end_bit, current_is_first, c, reinterpret_cast<cudaStream_t>(stream));
}

rsort_status rsort_pairs_buffer(rsort_key_t key, int descending, void *d_keys_first,
                                void *d_keys_second, void *d_values_first, void *d_values_second,
                                size_t value_bytes, size_t n, unsigned begin_bit, unsigned end_bit,
                                int *current_is_first, uint64_t *bins, size_t nbins,
                                int32_t *lookback, size_t nlookback, int32_t *counters,
                                size_t ncounters, rsort_stream_t stream) {
    if (value_bytes == 0) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return sort_buffer(key, descending, d_keys_first, d_keys_second, d_values_first,
                       d_values_second, value_bytes, n, begin_bit, end_bit, current_is_first, c,
                       reinterpret_cast<cudaStream_t>(stream));
}

namespace {

rsort_status keys_in_place(rsort_key_t key, int descending, bool total, void *d_keys,
                           void *d_scratch, size_t nscratch, size_t n, const Controls &c,
                           cudaStream_t s) {
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    // rccl-cub/src/radix.rs:591-600
    if (nscratch != n) return fail(RSORT_LENGTH_MISMATCH, "radix scratch keys", n, nscratch);
    const int kb = key_bytes(key);
    if (n > 0 && single_route(n, kb, 0)) {
        // The single-tile kernel reads its whole input before writing, so it
        // sorts in place and the reference's copy-back (radix.rs:617-621) is
        // not needed.
        int sel = 0;
        return sort_buffer(key, descending, d_keys, d_keys, nullptr, nullptr, 0, n, 0,
                           unsigned(kb) * 8, &sel, c, s, total);
    }
    int current_is_first = 1;
    rsort_status st = sort_buffer(key, descending, d_keys, d_scratch, nullptr, nullptr, 0, n, 0,
                                  unsigned(kb) * 8, &current_is_first, c, s, total);
    if (st != RSORT_OK) return st;
    if (!current_is_first && n > 0) {
        cudaError_t e = cudaMemcpyAsync(d_keys, d_scratch, n * size_t(kb), cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "copy back");
    }
    return RSORT_OK;
}

rsort_status pairs_in_place(rsort_key_t key, int descending, bool total, void *d_keys,
                            void *d_values, size_t value_bytes, void *d_scratch_keys,
                            size_t nscratch_keys, void *d_scratch_values, size_t nscratch_values,
                            size_t n, const Controls &c, cudaStream_t s) {
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    if (value_bytes == 0 || !value_ok(value_bytes))
        return fail(RSORT_BAD_ARGUMENT, "radix value width");
    // rccl-cub/src/radix.rs:833-844
    if (nscratch_keys != n) return fail(RSORT_LENGTH_MISMATCH, "radix scratch keys", n, nscratch_keys);
    if (nscratch_values != n)
        return fail(RSORT_LENGTH_MISMATCH, "radix scratch values", n, nscratch_values);
    const int kb = key_bytes(key);
    if (n > 0 && single_route(n, kb, int(value_bytes))) {
        int sel = 0;
        return sort_buffer(key, descending, d_keys, d_keys, d_values, d_values, value_bytes, n, 0,
                           unsigned(kb) * 8, &sel, c, s, total);
    }
    int current_is_first = 1;
    rsort_status st = sort_buffer(key, descending, d_keys, d_scratch_keys, d_values,
                                  d_scratch_values, value_bytes, n, 0, unsigned(kb) * 8,
                                  &current_is_first, c, s, total);
    if (st != RSORT_OK) return st;
    if (!current_is_first && n > 0) {
        cudaError_t e = cudaMemcpyAsync(d_keys, d_scratch_keys, n * size_t(kb),
                                        cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_values, d_scratch_values, n * value_bytes,
                                cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "copy back");
    }
    return RSORT_OK;
}

bool order_ok(rsort_order_t o) { return int(o) >= 0 && int(o) <= 3; }
bool order_desc(rsort_order_t o) {
    return o == RSORT_ORDER_DESCENDING || o == RSORT_ORDER_TOTAL_DESCENDING;
}
bool order_total(rsort_order_t o) {
    return o == RSORT_ORDER_TOTAL_ASCENDING || o == RSORT_ORDER_TOTAL_DESCENDING;
}

}  // namespace

rsort_status rsort_keys(rsort_key_t key, int descending, void *d_keys, void *d_scratch,
                        size_t nscratch, size_t n, uint64_t *bins, size_t nbins, int32_t *lookback,
                        size_t nlookback, int32_t *counters, size_t ncounters,
                        rsort_stream_t stream) {
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return keys_in_place(key, descending, false, d_keys, d_scratch, nscratch, n, c,
                         reinterpret_cast<cudaStream_t>(stream));
}

rsort_status rsort_merge_sort_keys(rsort_key_t key, rsort_order_t order, void *d_keys,
                                   void *d_scratch, size_t nscratch, size_t n, uint64_t *bins,
                                   size_t nbins, int32_t *lookback, size_t nlookback,
                                   int32_t *counters, size_t ncounters, rsort_stream_t stream) {
    if (!order_ok(order)) return fail(RSORT_BAD_ARGUMENT, "sort order");
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return keys_in_place(key, order_desc(order) ? 1 : 0, order_total(order), d_keys, d_scratch,
                         nscratch, n, c, reinterpret_cast<cudaStream_t>(stream));
}

rsort_status rsort_pairs(rsort_key_t key, int descending, void *d_keys, void *d_values,
                         size_t value_bytes, void *d_scratch_keys, size_t nscratch_keys,
                         void *d_scratch_values, size_t nscratch_values, size_t n, uint64_t *bins,
                         size_t nbins, int32_t *lookback, size_t nlookback, int32_t *counters,
                         size_t ncounters, rsort_stream_t stream) {
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return pairs_in_place(key, descending, false, d_keys, d_values, value_bytes, d_scratch_keys,
                          nscratch_keys, d_scratch_values, nscratch_values, n, c,
                          reinterpret_cast<cudaStream_t>(stream));
}

rsort_status rsort_merge_sort_pairs(rsort_key_t key, rsort_order_t order, void *d_keys,
                                    void *d_values, size_t value_bytes, void *d_scratch_keys,
                                    size_t nscratch_keys, void *d_scratch_values,
                                    size_t nscratch_values, size_t n, uint64_t *bins, size_t nbins,
                                    int32_t *lookback, size_t nlookback, int32_t *counters,
                                    size_t ncounters, rsort_stream_t stream) {
    if (!order_ok(order)) return fail(RSORT_BAD_ARGUMENT, "sort order");
    Controls c{bins, nbins, lookback, nlookback, counters, ncounters};
    return pairs_in_place(key, order_desc(order) ? 1 : 0, order_total(order), d_keys, d_values,
                          value_bytes, d_scratch_keys, nscratch_keys, d_scratch_values,
                          nscratch_values, n, c, reinterpret_cast<cudaStream_t>(stream));
}

rsort_status rsort_check_device_status(int32_t *counters, size_t ncounters,
                                       rsort_stream_t stream) {
    if (!counters || ncounters < size_t(CTR_WORDS)) return RSORT_OK;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t word = 0;
    cudaError_t e = cudaMemcpyAsync(&word, counters + CTR_STATUS, sizeof(word),
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "status read");
    if (word == 0) return RSORT_OK;
    const int32_t zero = 0;
    e = cudaMemcpyAsync(counters + CTR_STATUS, &zero, sizeof(zero), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (word == DEV_STATUS_TIMEOUT) return fail(RSORT_TIMEOUT, "radix look-back wait");
    return fail(RSORT_CUDA_ERROR, "radix scatter bounds check");
}

size_t rsort_single_tile_items(rsort_key_t key, size_t value_bytes) {
    if (!key_ok(key)) return 0;
    return policy800_single_tile_items(key_bytes(key), int(value_bytes));
}

int rsort_selector_flips(rsort_key_t key, size_t value_bytes, size_t n, unsigned begin_bit,
                         unsigned end_bit) {
    if (!key_ok(key) || begin_bit > end_bit || end_bit > unsigned(key_bytes(key)) * 8) return 0;
    const unsigned passes = (end_bit - begin_bit + 7) / 8;
    if (n == 0 || passes == 0) return 0;
    return single_route(n, key_bytes(key), int(value_bytes)) ? 1 : int(passes);
}

const char *rsort_status_string(rsort_status s) {
    switch (s) {
        case RSORT_OK: return "ok";
        case RSORT_INVALID_BIT_RANGE: return "radix bit range is outside 0..=key_bits or reversed";
        case RSORT_LENGTH_MISMATCH: return "length does not match required length";
        case RSORT_WORKSPACE_TOO_SMALL: return "workspace is smaller than required length";
        case RSORT_UNSUPPORTED_TARGET: return "unsupported target (sm_100a required)";
        case RSORT_SIZE_OVERFLOW: return "combined device range length overflowed";
        case RSORT_CUDA_ERROR: return "CUDA error";
        case RSORT_TIMEOUT: return "bounded device wait gave up";
        case RSORT_BAD_ARGUMENT: return "invalid argument";
    }
    return "unknown status";
}

void rsort_last_error(rsort_error_info *out) {
    if (out) *out = g_last_error;
}

uint64_t rsort_launch_count(void) { return g_launches; }
void rsort_launch_count_reset(void) { g_launches = 0; }

// ---------------------------------------------------------------------------
// Multi-GPU sample sort device steps (no reference counterpart).
// ---------------------------------------------------------------------------

rsort_status rsort_dist_samples(rsort_key_t key, int descending, const void *d_sorted_keys,
                                size_t m, unsigned rank, unsigned samples, void *d_samples,
                                rsort_stream_t stream) {
    if (!wide_key(key)) return fail(RSORT_BAD_ARGUMENT, "key type (32- or 64-bit keys only)");
    if (m >= (size_t(1) << POS_BITS) || rank >= (1u << (64 - POS_BITS)))
        return fail(RSORT_SIZE_OVERFLOW, "sample position");
    if (samples == 0) return RSORT_OK;
    if (!d_samples || (m && !d_sorted_keys)) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    if (check_alignment(addr(d_sorted_keys), size_t(key_bytes(key)), "sample keys alignment") ||
        check_alignment(addr(d_samples), 8, "samples alignment (8 bytes)"))
        return RSORT_BAD_ARGUMENT;
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_DIST, s);
        e = launch_samples(key_bytes(key), d_sorted_keys, m, rank, samples,
                           KeyXform{key_kind(key), descending ? 1 : 0},
                           static_cast<Composite *>(d_samples), s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "samples launch");
}

rsort_status rsort_dist_splitters(const void *d_samples, size_t total, unsigned world,
                                  void *d_splitters, rsort_stream_t stream) {
    if (world < 1) return fail(RSORT_BAD_ARGUMENT, "world size");
    if (total > MAX_SPLITTER_SAMPLES)
        return fail(RSORT_WORKSPACE_TOO_SMALL, "splitter sample set", MAX_SPLITTER_SAMPLES, total);
    if (world == 1) return RSORT_OK;
    if (!d_samples || !d_splitters) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    if (check_alignment(addr(d_samples) | addr(d_splitters), 8, "samples alignment (8 bytes)"))
        return RSORT_BAD_ARGUMENT;
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_DIST, s);
        e = launch_splitters(static_cast<const Composite *>(d_samples), uint32_t(total), world,
                             static_cast<Composite *>(d_splitters), s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "splitters launch");
}

rsort_status rsort_dist_bounds(rsort_key_t key, int descending, const void *d_sorted_keys,
                               size_t m, unsigned rank, const void *d_splitters, unsigned world,
                               uint64_t *d_bounds, rsort_stream_t stream) {
    if (!wide_key(key)) return fail(RSORT_BAD_ARGUMENT, "key type (32- or 64-bit keys only)");
    if (world < 1 || !d_bounds || (world > 1 && !d_splitters))
        return fail(RSORT_BAD_ARGUMENT, "null buffer");
    if (m >= (size_t(1) << POS_BITS)) return fail(RSORT_SIZE_OVERFLOW, "sample position");
    if (check_alignment(addr(d_sorted_keys), size_t(key_bytes(key)), "bound keys alignment") ||
        check_alignment(addr(d_splitters), 8, "splitters alignment (8 bytes)") ||
        check_alignment(addr(d_bounds), 8, "bounds alignment"))
        return RSORT_BAD_ARGUMENT;
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_DIST, s);
        e = launch_bounds(key_bytes(key), d_sorted_keys, m, rank,
                          static_cast<const Composite *>(d_splitters), world,
                          KeyXform{key_kind(key), descending ? 1 : 0}, d_bounds, s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "bounds launch");
}

rsort_status rsort_ipc_export(const void *d_ptr, void *handle, uint64_t *offset) {
    if (!d_ptr || !handle || !offset) return fail(RSORT_BAD_ARGUMENT, "null argument");
    uintptr_t base = 0;
    cudaError_t e = allocation_base(d_ptr, &base);
    if (e != cudaSuccess) return cuda_fail(e, "allocation base of the exported pointer");
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == RSORT_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    *offset = uint64_t(reinterpret_cast<uintptr_t>(d_ptr) - base);
    return RSORT_OK;
}

rsort_status rsort_ipc_import(const void *handle, void **d_base) {
    if (!handle || !d_base) return fail(RSORT_BAD_ARGUMENT, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(d_base, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

rsort_status rsort_ipc_release(void *d_base) {
    if (!d_base) return fail(RSORT_BAD_ARGUMENT, "null argument");
    const cudaError_t e = cudaIpcCloseMemHandle(d_base);
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

rsort_status rsort_gather_segments(unsigned nseg, const void *const *d_src, const uint64_t *bytes,
                                   void *d_dst, rsort_stream_t stream) {
    if (nseg > unsigned(GATHER_MAX_SEGMENTS))
        return fail(RSORT_BAD_ARGUMENT, "gather segment count", GATHER_MAX_SEGMENTS, nseg);
    if (nseg == 0) return RSORT_OK;
    if (!d_src || !bytes) return fail(RSORT_BAD_ARGUMENT, "null argument");
    GatherArgs a{};
    a.nseg = nseg;
    a.dst = static_cast<char *>(d_dst);
    uint64_t total = 0;
    for (unsigned q = 0; q < nseg; ++q) {
        a.dst_start[q] = total;
        a.src[q] = static_cast<const char *>(d_src[q]);
        if (bytes[q] && !d_src[q]) return fail(RSORT_BAD_ARGUMENT, "null segment");
        const uint64_t align = uint64_t(reinterpret_cast<uintptr_t>(d_src[q])) |
                               uint64_t(reinterpret_cast<uintptr_t>(a.dst) + total) | bytes[q];
        int lg = 0;
        while (lg < 4 && !(align & (uint64_t(1) << lg))) ++lg;
        a.unit_log2[q] = uint8_t(lg);
        total += bytes[q];
    }
    a.dst_start[nseg] = total;
    if (total == 0) return RSORT_OK;
    if (!d_dst) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_GATHER, s);
        e = launch_gather(a, dev.sm_count, s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "gather launch");
}

// ---------------------------------------------------------------------------
// Segmented radix sort (no reference counterpart)
// ---------------------------------------------------------------------------
namespace {

struct SegLayout {
    size_t keys, values, bins, lookback, counters, ids, total;
    rsort_controls c;
};

rsort_status seg_layout(rsort_key_t key, size_t vb, size_t n, size_t nseg, SegLayout *L) {
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    if (nseg > 0xffffffffull) return fail(RSORT_SIZE_OVERFLOW, "segment count");
    rsort_controls c{};
    // Controls sized for a segment of all n items bound every segment.
    rsort_status st = rsort_controls_query(key, vb, n, &c);
    if (st != RSORT_OK) return st;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = (off + bytes + 255) / 256 * 256;
        return at;
    };
    L->keys = take(size_t(key_bytes(key)) * n);
    L->values = take(vb * n);
    L->bins = take(8 * c.bins);
    L->lookback = take(4 * c.lookback);
    L->counters = take(4 * c.counters);
    L->ids = take(4 * nseg);
    L->total = off;
    L->c = c;
    return RSORT_OK;
}

}  // namespace

size_t rsort_segmented_scratch_bytes(rsort_key_t key, size_t value_bytes, size_t n, size_t nseg) {
    SegLayout L{};
    return seg_layout(key, value_bytes, n, nseg, &L) == RSORT_OK ? L.total : 0;
}

rsort_status rsort_segmented_sort(rsort_key_t key, int descending, const void *d_keys_in,
                                  void *d_keys_out, const void *d_values_in, void *d_values_out,
                                  size_t value_bytes, size_t n, size_t nseg,
                                  const uint64_t *d_begin_offsets, const uint64_t *d_end_offsets,
                                  unsigned begin_bit, unsigned end_bit, void *d_scratch,
                                  size_t scratch_bytes, rsort_stream_t stream) {
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "radix key type");
    if (!value_ok(value_bytes)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    const int kb = key_bytes(key);
    const unsigned kbits = unsigned(kb) * 8;
    if (begin_bit > end_bit || end_bit > kbits) return fail_bits(begin_bit, end_bit, kbits);
    if (nseg == 0 || n == 0) return RSORT_OK;
    if (nseg > 0xffffffffull) return fail(RSORT_SIZE_OVERFLOW, "segment count");
    if (!d_keys_in || !d_keys_out || !d_begin_offsets || !d_end_offsets ||
        (value_bytes && (!d_values_in || !d_values_out)))
        return fail(RSORT_BAD_ARGUMENT, "null buffer");
    {
        rsort_status st = check_alignment(addr(d_keys_in) | addr(d_keys_out), size_t(kb),
                                          "segmented keys alignment");
        if (st == RSORT_OK)
            st = check_alignment(addr(d_values_in) | addr(d_values_out), value_bytes,
                                 "segmented values alignment");
        if (st == RSORT_OK)
            st = check_alignment(addr(d_begin_offsets) | addr(d_end_offsets), 8,
                                 "segment offsets alignment");
        if (st != RSORT_OK) return st;
    }
    SegLayout L{};
    rsort_status st = seg_layout(key, value_bytes, n, nseg, &L);
    if (st != RSORT_OK) return st;
    if (!d_scratch || scratch_bytes < L.total)
        return fail(RSORT_WORKSPACE_TOO_SMALL, "segmented sort scratch", L.total, scratch_bytes);
    st = check_blob(d_scratch, "segmented sort scratch alignment (256 bytes)");
    if (st != RSORT_OK) return st;
    DeviceInfo dev;
    st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The segment extents are read on the host (one synchronization).
    std::vector<uint64_t> b(nseg), e(nseg);
    cudaError_t ce = cudaMemcpyAsync(b.data(), d_begin_offsets, 8 * nseg, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(e.data(), d_end_offsets, 8 * nseg, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return cuda_fail(ce, "segment offsets");
    const size_t single = policy800_single_tile_items(kb, int(value_bytes));
    std::vector<uint32_t> small;
    std::vector<size_t> large;
    for (size_t i = 0; i < nseg; ++i) {
        if (b[i] > e[i] || e[i] > n) return fail(RSORT_BAD_ARGUMENT, "segment offsets out of range");
        const uint64_t len = e[i] - b[i];
        if (len == 0) continue;
        if (len <= single) small.push_back(uint32_t(i));
        else large.push_back(i);
    }
    char *base = static_cast<char *>(d_scratch);
    const int kind = key_kind(key);
    if (!small.empty()) {
        uint32_t *ids = reinterpret_cast<uint32_t *>(base + L.ids);
        ce = cudaMemcpyAsync(ids, small.data(), 4 * small.size(), cudaMemcpyHostToDevice, s);
        if (ce != cudaSuccess) return cuda_fail(ce, "segment ids");
        SingleArgs a{d_keys_in, d_keys_out, d_values_in, d_values_out, 0, begin_bit, end_bit, kind,
                     descending ? 1 : 0};
        a.seg_begin = d_begin_offsets;
        a.seg_end = d_end_offsets;
        a.seg_ids = ids;
        a.seg_count = uint32_t(small.size());
        {
            LaunchScope scope(RSORT_KERNEL_SINGLE_TILE, s);
            ce = launch_single_tile(kb, int(value_bytes), a, s);
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "segmented single-tile launch");
    }
    if (!large.empty()) {
        Controls c{reinterpret_cast<uint64_t *>(base + L.bins), L.c.bins,
                   reinterpret_cast<int32_t *>(base + L.lookback), L.c.lookback,
                   reinterpret_cast<int32_t *>(base + L.counters), L.c.counters};
        if (L.c.counters) {
            ce = cudaMemsetAsync(c.counters, 0, 4 * L.c.counters, s);
            if (ce != cudaSuccess) return cuda_fail(ce, "segmented sort counters");
        }
        char *sk = base + L.keys;
        char *sv = base + L.values;
        for (size_t i : large) {
            const size_t len = size_t(e[i] - b[i]);
            char *ok = static_cast<char *>(d_keys_out) + b[i] * kb;
            char *ov = value_bytes ? static_cast<char *>(d_values_out) + b[i] * value_bytes : nullptr;
            ce = cudaMemcpyAsync(ok, static_cast<const char *>(d_keys_in) + b[i] * kb, len * kb,
                                 cudaMemcpyDeviceToDevice, s);
            if (ce == cudaSuccess && value_bytes)
                ce = cudaMemcpyAsync(ov, static_cast<const char *>(d_values_in) + b[i] * value_bytes,
                                     len * value_bytes, cudaMemcpyDeviceToDevice, s);
            if (ce != cudaSuccess) return cuda_fail(ce, "segment copy");
            // The look-back region must have this segment's exact length
            // (the LengthMismatch rule): pass that prefix of the scratch.
            rsort_controls cs{};
            st = rsort_controls_query(key, value_bytes, len, &cs);
            if (st != RSORT_OK) return st;
            const Controls cseg{c.bins, cs.bins, c.lookback, cs.lookback, c.counters, cs.counters};
            int cur_first = 1;
            st = sort_buffer(key, descending, ok, sk, ov, value_bytes ? sv : nullptr, value_bytes, len,
                             begin_bit, end_bit, &cur_first, cseg, s);
            if (st != RSORT_OK) return st;
            if (!cur_first) {
                ce = cudaMemcpyAsync(ok, sk, len * kb, cudaMemcpyDeviceToDevice, s);
                if (ce == cudaSuccess && value_bytes)
                    ce = cudaMemcpyAsync(ov, sv, len * value_bytes, cudaMemcpyDeviceToDevice, s);
                if (ce != cudaSuccess) return cuda_fail(ce, "segment copy back");
            }
        }
    }
    return RSORT_OK;
}

// ---------------------------------------------------------------------------
// Lexicographic record sort (rccl-thrust/src/record_sort.rs:144-300)
// ---------------------------------------------------------------------------
namespace {

struct RowsLayout {
    size_t keys, keys_alt, perm, perm_alt, bins, lookback, counters, rows, payload, total;
    rsort_controls c;
};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

rsort_status rows_layout(size_t words, size_t payload_bytes, size_t n, RowsLayout *L) {
    if (words > (size_t(1) << 20)) return fail(RSORT_BAD_ARGUMENT, "record width");
    size_t row_region = 0, payload_region = 0;
    if (!region_bytes(4 * words, n, &row_region) || !region_bytes(payload_bytes, n, &payload_region))
        return fail(RSORT_SIZE_OVERFLOW, "record sort scratch size");
    rsort_controls c{};
    rsort_status st = rsort_controls_query(RSORT_U64, 4, n, &c);
    if (st != RSORT_OK) return st;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    L->keys = take(8 * n);
    L->keys_alt = take(8 * n);
    L->perm = take(4 * n);
    L->perm_alt = take(4 * n);
    L->bins = take(8 * c.bins);
    L->lookback = take(4 * c.lookback);
    L->counters = take(4 * c.counters);
    L->rows = take(row_region);
    L->payload = take(payload_region);
    L->total = off;
    L->c = c;
    return RSORT_OK;
}

}  // namespace

size_t rsort_rows_scratch_bytes(size_t words, size_t payload_bytes, size_t n) {
    RowsLayout L{};
    return rows_layout(words, payload_bytes, n, &L) == RSORT_OK ? L.total : 0;
}

rsort_status rsort_rows_lexicographic(size_t words, void *d_rows, void *d_payload,
                                      size_t payload_bytes, size_t n, void *d_scratch,
                                      size_t scratch_bytes, rsort_stream_t stream) {
    if (words == 0 || n <= 1) return RSORT_OK;
    if (n > 0xffffffffull) return fail(RSORT_SIZE_OVERFLOW, "record count (32-bit permutation)");
    if (words > (size_t(1) << 20)) return fail(RSORT_BAD_ARGUMENT, "record width");
    if (!d_rows || (payload_bytes && !d_payload)) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    if (check_alignment(addr(d_rows), 4, "record rows alignment (32-bit words)") != RSORT_OK)
        return RSORT_BAD_ARGUMENT;
    RowsLayout L{};
    rsort_status st = rows_layout(words, payload_bytes, n, &L);
    if (st != RSORT_OK) return st;
    if (!d_scratch || scratch_bytes < L.total)
        return fail(RSORT_WORKSPACE_TOO_SMALL, "record sort scratch", L.total, scratch_bytes);
    st = check_blob(d_scratch, "record sort scratch alignment (256 bytes)");
    if (st != RSORT_OK) return st;
    DeviceInfo dev;
    st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    char *base = static_cast<char *>(d_scratch);
    uint64_t *keys = reinterpret_cast<uint64_t *>(base + L.keys);
    uint64_t *keys_alt = reinterpret_cast<uint64_t *>(base + L.keys_alt);
    uint32_t *perm = reinterpret_cast<uint32_t *>(base + L.perm);
    uint32_t *perm_alt = reinterpret_cast<uint32_t *>(base + L.perm_alt);
    Controls c{reinterpret_cast<uint64_t *>(base + L.bins), L.c.bins,
               reinterpret_cast<int32_t *>(base + L.lookback), L.c.lookback,
               reinterpret_cast<int32_t *>(base + L.counters), L.c.counters};
    const uint32_t *rows = static_cast<const uint32_t *>(d_rows);
    cudaError_t e = L.c.counters ? cudaMemsetAsync(c.counters, 0, 4 * L.c.counters, s) : cudaSuccess;
    if (e != cudaSuccess) return cuda_fail(e, "record sort counters");
    {
        LaunchScope scope(RSORT_KERNEL_RECORDS, s);
        e = launch_iota(perm, n, dev.sm_count, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "record sort permutation");
    // LSD over 64-bit chunks of the row, least significant chunk (the last
    // words) first; every pass is a stable sort of (chunk key, permutation).
    const size_t chunks = (words + 1) / 2;
    for (size_t j = chunks; j-- > 0;) {
        const uint32_t first = uint32_t(2 * j);
        const uint32_t count = uint32_t(words - 2 * j < 2 ? words - 2 * j : 2);
        {
            LaunchScope scope(RSORT_KERNEL_RECORDS, s);
            e = launch_chunk_keys(rows, uint32_t(words), j + 1 == chunks ? nullptr : perm, n, first,
                                  count, keys, dev.sm_count, s);
        }
        if (e != cudaSuccess) return cuda_fail(e, "record sort chunk keys");
        int cur_first = 1;
        st = sort_buffer(RSORT_U64, 0, keys, keys_alt, perm, perm_alt, 4, n, 0, 32 * count,
                         &cur_first, c, s);
        if (st != RSORT_OK) return st;
        if (!cur_first) {
            e = cudaMemcpyAsync(perm, perm_alt, 4 * n, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "record sort permutation copy");
        }
    }
    // Apply the permutation to the rows and payloads.
    char *rows_tmp = base + L.rows;
    {
        LaunchScope scope(RSORT_KERNEL_RECORDS, s);
        e = launch_permute(d_rows, perm, n, 4 * words, rows_tmp, dev.sm_count, s);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_rows, rows_tmp, 4 * words * n, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && payload_bytes) {
        char *pay_tmp = base + L.payload;
        {
            LaunchScope scope(RSORT_KERNEL_RECORDS, s);
            e = launch_permute(d_payload, perm, n, payload_bytes, pay_tmp, dev.sm_count, s);
        }
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_payload, pay_tmp, payload_bytes * n, cudaMemcpyDeviceToDevice, s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "record sort permutation");
}

// ---------------------------------------------------------------------------
// Comparator-program sort: DeviceMergeSort by a chain of projected-field
// comparisons (rccl-cub/src/dispatch.rs:170-193, 1113-1146 with the closures
// of rccl-thrust/examples/sort.rs:101-113), on the stable radix path.
// ---------------------------------------------------------------------------
namespace {

struct SortByLayout {
    size_t keys, keys_alt, perm, perm_alt, bins, lookback, counters, records, values, total;
    rsort_controls c, c32, c64;  // region sizes; the exact counts of each key width
};

rsort_status sort_by_layout(size_t record_bytes, size_t value_bytes, size_t n, SortByLayout *L) {
    size_t record_region = 0, value_region = 0;
    if (!region_bytes(record_bytes, n, &record_region) || !region_bytes(value_bytes, n, &value_region))
        return fail(RSORT_SIZE_OVERFLOW, "sort_by scratch size");
    // The groups sort 32- or 64-bit keys with 4-byte indices: controls for
    // the larger of the two shapes serve both.
    rsort_controls c64{}, c32{};
    rsort_status st = rsort_controls_query(RSORT_U64, 4, n, &c64);
    if (st == RSORT_OK) st = rsort_controls_query(RSORT_U32, 4, n, &c32);
    if (st != RSORT_OK) return st;
    const rsort_controls c{std::max(c64.bins, c32.bins), std::max(c64.lookback, c32.lookback),
                           std::max(c64.counters, c32.counters)};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align256(off + bytes);
        return at;
    };
    L->keys = take(8 * n);
    L->keys_alt = take(8 * n);
    L->perm = take(4 * n);
    L->perm_alt = take(4 * n);
    L->bins = take(8 * c.bins);
    L->lookback = take(4 * c.lookback);
    L->counters = take(4 * c.counters);
    L->records = take(record_region);
    L->values = take(value_region);
    L->total = off;
    L->c = c;
    L->c32 = c32;
    L->c64 = c64;
    return RSORT_OK;
}

unsigned bit_length(uint64_t v) { return v ? 64u - unsigned(__builtin_clzll(v)) : 0u; }

// Checks one term and fills its device form, including the window of order
// image bits that can differ between records (width 0: the term compares
// every record equal).
rsort_status prepare_term(const rsort_compare_term &t, size_t record_bytes, uintptr_t records,
                          CompareTerm *out) {
    const rsort_key_t key = rsort_key_t(t.type);
    if (!key_ok(key)) return fail(RSORT_BAD_ARGUMENT, "comparator term type");
    if (!order_ok(rsort_order_t(t.order))) return fail(RSORT_BAD_ARGUMENT, "comparator term order");
    const unsigned bytes = unsigned(key_bytes(key)), W = 8 * bytes;
    if (size_t(t.offset) + bytes > record_bytes)
        return fail(RSORT_BAD_ARGUMENT, "comparator term field (offset + width <= record_bytes)",
                    record_bytes, size_t(t.offset) + bytes);
    const int kind0 = key_kind(key);
    const int kind = kind0 == KIND_FLOAT && order_total(rsort_order_t(t.order)) ? KIND_FLOAT_TOTAL
                                                                               : kind0;
    const int proj = t.projection;
    if (proj < RSORT_PROJ_IDENTITY || proj > RSORT_PROJ_REM)
        return fail(RSORT_BAD_ARGUMENT, "comparator term projection");
    if (kind0 == KIND_FLOAT && proj != RSORT_PROJ_IDENTITY)
        return fail(RSORT_BAD_ARGUMENT, "comparator term projection (floats: identity only)");
    const uint64_t wmask = W == 64 ? ~uint64_t(0) : (uint64_t(1) << W) - 1;
    const int64_t smin = W == 64 ? INT64_MIN : -(int64_t(1) << (W - 1));
    const int64_t smax = W == 64 ? INT64_MAX : (int64_t(1) << (W - 1)) - 1;
    const bool is_signed = kind0 == KIND_SINT;
    // The operand must be a value of the field's type (a 64-bit unsigned
    // operand is passed as its bits).
    const bool representable = is_signed ? (t.operand >= smin && t.operand <= smax)
                                          : (W == 64 || (t.operand >= 0 && uint64_t(t.operand) <= wmask));
    unsigned lo = 0, width = W;
    const uint64_t op = uint64_t(t.operand) & wmask;
    switch (proj) {
        case RSORT_PROJ_AND:
            if (!representable) return fail(RSORT_BAD_ARGUMENT, "comparator term mask");
            // Without the sign bit the masked value is non-negative and the
            // signed image's sign bit is constant: only the mask bits vary.
            if (!is_signed || !(op >> (W - 1))) {
                if (op == 0) {
                    width = 0;
                } else {
                    lo = unsigned(__builtin_ctzll(op));
                    width = bit_length(op) - lo;
                }
            }
            break;
        case RSORT_PROJ_SHR:
            if (t.operand < 0 || uint64_t(t.operand) >= W)
                return fail(RSORT_BAD_ARGUMENT, "comparator term shift (0 <= shift < width)", W,
                            size_t(t.operand));
            if (!is_signed) width = W - unsigned(t.operand);
            break;
        case RSORT_PROJ_DIV:
        case RSORT_PROJ_REM:
            if (!representable || op == 0 || (is_signed && t.operand == -1))
                return fail(RSORT_BAD_ARGUMENT, "comparator term divisor (non-zero; not -1 for signed)");
            if (!is_signed) width = proj == RSORT_PROJ_DIV ? bit_length(wmask / op) : bit_length(op - 1);
            break;
        default: break;
    }
    const bool aligned = records % bytes == 0 && record_bytes % bytes == 0 && t.offset % bytes == 0;
    *out = CompareTerm{t.offset,
                       uint8_t(bytes),
                       uint8_t(kind),
                       uint8_t(proj),
                       uint8_t(order_desc(rsort_order_t(t.order)) ? 1 : 0),
                       uint8_t(aligned ? 1 : 0),
                       uint8_t(lo),
                       uint8_t(width),
                       int64_t(op)};
    if (is_signed) out->operand = t.operand;
    return RSORT_OK;
}

}  // namespace

size_t rsort_sort_by_scratch_bytes(size_t record_bytes, size_t value_bytes, size_t n) {
    SortByLayout L{};
    return sort_by_layout(record_bytes, value_bytes, n, &L) == RSORT_OK ? L.total : 0;
}

rsort_status rsort_sort_by(const rsort_compare_term *terms, size_t nterms, void *d_records,
                           size_t record_bytes, void *d_values, size_t value_bytes, size_t n,
                           void *d_scratch, size_t scratch_bytes, rsort_stream_t stream) {
    if (nterms > RSORT_MAX_TERMS)
        return fail(RSORT_BAD_ARGUMENT, "comparator terms (at most RSORT_MAX_TERMS)", RSORT_MAX_TERMS,
                    nterms);
    if (nterms && !terms) return fail(RSORT_BAD_ARGUMENT, "null comparator terms");
    if (record_bytes == 0) return fail(RSORT_BAD_ARGUMENT, "record width");
    if (n > 0xffffffffull) return fail(RSORT_SIZE_OVERFLOW, "record count (32-bit permutation)");
    if (n > 1 && (!d_records || (value_bytes && !d_values))) return fail(RSORT_BAD_ARGUMENT, "null buffer");
    // Groups of terms packed into one key, least significant group first;
    // each group's terms most significant first.
    std::vector<CompareGroup> groups;
    {
        std::vector<CompareTerm> kept;
        for (size_t i = 0; i < nterms; ++i) {
            CompareTerm ct{};
            rsort_status st = prepare_term(terms[i], record_bytes,
                                           reinterpret_cast<uintptr_t>(d_records), &ct);
            if (st != RSORT_OK) return st;
            if (ct.width) kept.push_back(ct);
        }
        for (size_t i = kept.size(); i-- > 0;) {
            if (groups.empty() || groups.back().total_bits + kept[i].width > 64 ||
                groups.back().nterms == COMPARE_GROUP_MAX)
                groups.push_back(CompareGroup{});
            CompareGroup &g = groups.back();
            // prepend: terms run most significant first within a group
            for (uint32_t k = g.nterms; k > 0; --k) g.term[k] = g.term[k - 1];
            g.term[0] = kept[i];
            ++g.nterms;
            g.total_bits += kept[i].width;
        }
    }
    if (n <= 1 || groups.empty()) return RSORT_OK;
    SortByLayout L{};
    rsort_status st = sort_by_layout(record_bytes, value_bytes, n, &L);
    if (st != RSORT_OK) return st;
    if (!d_scratch || scratch_bytes < L.total)
        return fail(RSORT_WORKSPACE_TOO_SMALL, "sort_by scratch", L.total, scratch_bytes);
    st = check_blob(d_scratch, "sort_by scratch alignment (256 bytes)");
    if (st != RSORT_OK) return st;
    DeviceInfo dev;
    st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    char *base = static_cast<char *>(d_scratch);
    void *keys = base + L.keys;
    void *keys_alt = base + L.keys_alt;
    uint32_t *perm = reinterpret_cast<uint32_t *>(base + L.perm);
    uint32_t *perm_alt = reinterpret_cast<uint32_t *>(base + L.perm_alt);
    // One set of control regions, sized for the larger shape; each group's
    // sort gets the exact counts of its key width.
    auto controls = [&](const rsort_controls &k) {
        return Controls{reinterpret_cast<uint64_t *>(base + L.bins), k.bins,
                        reinterpret_cast<int32_t *>(base + L.lookback), k.lookback,
                        reinterpret_cast<int32_t *>(base + L.counters), k.counters};
    };
    const Controls c32 = controls(L.c32), c64 = controls(L.c64);
    const uint8_t *records = static_cast<const uint8_t *>(d_records);
    cudaError_t e = L.c.counters ? cudaMemsetAsync(c64.counters, 0, 4 * L.c.counters, s)
                                 : cudaSuccess;
    if (e != cudaSuccess) return cuda_fail(e, "sort_by counters");
    {
        LaunchScope scope(RSORT_KERNEL_RECORDS, s);
        e = launch_iota(perm, n, dev.sm_count, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "sort_by permutation");
    // LSD over the groups; every group is a stable sort of (key, index).
    for (size_t gi = 0; gi < groups.size(); ++gi) {
        const CompareGroup &g = groups[gi];
        {
            LaunchScope scope(RSORT_KERNEL_RECORDS, s);
            e = launch_compare_keys(records, record_bytes, gi == 0 ? nullptr : perm, n, g, keys,
                                    dev.sm_count, s);
        }
        if (e != cudaSuccess) return cuda_fail(e, "sort_by keys");
        int cur_first = 1;
        const bool narrow = g.total_bits <= 32;
        st = sort_buffer(narrow ? RSORT_U32 : RSORT_U64, 0, keys, keys_alt, perm, perm_alt, 4, n, 0,
                         g.total_bits, &cur_first, narrow ? c32 : c64, s);
        if (st != RSORT_OK) return st;
        if (!cur_first) std::swap(perm, perm_alt);
    }
    // Apply the permutation to the records and values.
    char *rec_tmp = base + L.records;
    {
        LaunchScope scope(RSORT_KERNEL_RECORDS, s);
        e = launch_permute(d_records, perm, n, record_bytes, rec_tmp, dev.sm_count, s);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_records, rec_tmp, record_bytes * n, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && value_bytes) {
        char *val_tmp = base + L.values;
        {
            LaunchScope scope(RSORT_KERNEL_RECORDS, s);
            e = launch_permute(d_values, perm, n, value_bytes, val_tmp, dev.sm_count, s);
        }
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_values, val_tmp, value_bytes * n, cudaMemcpyDeviceToDevice, s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "sort_by permutation");
}

// One word per merge tile plus one, and one more per pair of a batched round
// (rsort_merge_runs / rsort_merge_segments launch up to MERGE_MAX_PAIRS pair
// merges at once, each with its own closing word).
size_t rsort_merge_partition_words(size_t total) {
    return merge_partition_words(total, 0) + MERGE_MAX_PAIRS;
}

namespace {
rsort_status merge_impl(rsort_key_t key, int descending, bool total, const void *a_keys,
                        const void *a_values, size_t na, const void *b_keys, const void *b_values,
                        size_t nb, void *out_keys, void *out_values, size_t value_bytes,
                        uint64_t *d_partitions, size_t npartitions, rsort_stream_t stream);
}

rsort_status rsort_merge(rsort_key_t key, int descending, const void *a_keys,
                         const void *a_values, size_t na, const void *b_keys, const void *b_values,
                         size_t nb, void *out_keys, void *out_values, size_t value_bytes,
                         uint64_t *d_partitions, size_t npartitions, rsort_stream_t stream) {
    return merge_impl(key, descending, false, a_keys, a_values, na, b_keys, b_values, nb, out_keys,
                      out_values, value_bytes, d_partitions, npartitions, stream);
}

rsort_status rsort_merge_ordered(rsort_key_t key, rsort_order_t order, const void *a_keys,
                                 const void *a_values, size_t na, const void *b_keys,
                                 const void *b_values, size_t nb, void *out_keys,
                                 void *out_values, size_t value_bytes, uint64_t *d_partitions,
                                 size_t npartitions, rsort_stream_t stream) {
    if (!order_ok(order)) return fail(RSORT_BAD_ARGUMENT, "sort order");
    return merge_impl(key, order_desc(order) ? 1 : 0, order_total(order), a_keys, a_values, na,
                      b_keys, b_values, nb, out_keys, out_values, value_bytes, d_partitions,
                      npartitions, stream);
}

namespace {
rsort_status merge_impl(rsort_key_t key, int descending, bool total, const void *a_keys,
                        const void *a_values, size_t na, const void *b_keys, const void *b_values,
                        size_t nb, void *out_keys, void *out_values, size_t value_bytes,
                        uint64_t *d_partitions, size_t npartitions, rsort_stream_t stream) {
    if (!wide_key(key)) return fail(RSORT_BAD_ARGUMENT, "key type (32- or 64-bit keys only)");
    if (!value_ok(value_bytes)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    if (na + nb == 0) return RSORT_OK;
    if (!out_keys || (na && !a_keys) || (nb && !b_keys) ||
        (value_bytes && (!out_values || (na && !a_values) || (nb && !b_values))))
        return fail(RSORT_BAD_ARGUMENT, "null buffer");
    {
        rsort_status st = check_alignment(addr(a_keys) | addr(b_keys) | addr(out_keys),
                                          size_t(key_bytes(key)), "merge keys alignment");
        if (st == RSORT_OK)
            st = check_alignment(addr(a_values) | addr(b_values) | addr(out_values), value_bytes,
                                 "merge values alignment");
        if (st == RSORT_OK) st = check_alignment(addr(d_partitions), 8, "merge partitions alignment");
        if (st != RSORT_OK) return st;
    }
    if (merge_partition_words(na, nb) > 0x7fffffffull) return fail(RSORT_SIZE_OVERFLOW, "merge tiles");
    if (!d_partitions || npartitions < merge_partition_words(na, nb))
        return fail(RSORT_WORKSPACE_TOO_SMALL, "merge partitions", merge_partition_words(na, nb),
                    npartitions);
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int kind = total && key_kind(key) == KIND_FLOAT ? KIND_FLOAT_TOTAL : key_kind(key);
    MergeArgs p{a_keys, a_values, na, b_keys, b_values, nb, out_keys, out_values, kind,
                descending ? 1 : 0};
    cudaError_t e;
    {
        LaunchScope scope(RSORT_KERNEL_MERGE, s);
        e = launch_merge(key_bytes(key), int(value_bytes), p, d_partitions, s);
    }
    return e == cudaSuccess ? RSORT_OK : cuda_fail(e, "merge launch");
}
}  // namespace

namespace {

// A round of a merge tree: independent two-run merges launched together, at
// most MERGE_MAX_PAIRS per launch, so every pair (and every peer a pair reads)
// progresses at once.
struct PairMerge {
    const void *ak, *av;
    size_t na;
    const void *bk, *bv;
    size_t nb;
    void *ok, *ov;
};

rsort_status merge_round(rsort_key_t key, int descending, const std::vector<PairMerge> &pairs,
                         size_t value_bytes, uint64_t *d_partitions, size_t npartitions,
                         cudaStream_t s) {
    const int kind = key_kind(key);
    for (size_t first = 0; first < pairs.size(); first += MERGE_MAX_PAIRS) {
        const size_t count = std::min<size_t>(MERGE_MAX_PAIRS, pairs.size() - first);
        MergeBatch b{};
        b.npairs = uint32_t(count);
        uint64_t words = 0;
        for (size_t q = 0; q < count; ++q) {
            const PairMerge &m = pairs[first + q];
            if (merge_partition_words(m.na, m.nb) > 0x7fffffffull)
                return fail(RSORT_SIZE_OVERFLOW, "merge tiles");
            b.pair[q] = MergeArgs{m.ak, m.av, m.na, m.bk, m.bv, m.nb, m.ok, m.ov, kind,
                                  descending ? 1 : 0};
            b.split_start[q] = words;
            words += merge_partition_words(m.na, m.nb);
        }
        b.split_start[count] = words;
        if (!d_partitions || npartitions < words)
            return fail(RSORT_WORKSPACE_TOO_SMALL, "merge partitions", words, npartitions);
        cudaError_t e;
        {
            LaunchScope scope(RSORT_KERNEL_MERGE, s);
            e = launch_merge_batch(key_bytes(key), int(value_bytes), b, d_partitions, s);
        }
        if (e != cudaSuccess) return cuda_fail(e, "merge launch");
    }
    return RSORT_OK;
}

}  // namespace

rsort_status rsort_merge_runs(rsort_key_t key, int descending, void *keys, void *values,
                              size_t value_bytes, const size_t *run_lengths, unsigned runs,
                              void *scratch_keys, void *scratch_values, uint64_t *d_partitions,
                              size_t npartitions, int *result_in_scratch, rsort_stream_t stream) {
    if (!wide_key(key)) return fail(RSORT_BAD_ARGUMENT, "key type (32- or 64-bit keys only)");
    if (!value_ok(value_bytes)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    if (!result_in_scratch || (runs && !run_lengths)) return fail(RSORT_BAD_ARGUMENT, "null argument");
    const size_t kb = size_t(key_bytes(key));
    std::vector<size_t> len(run_lengths, run_lengths + runs), off(runs, 0);
    size_t total = 0;
    for (unsigned r = 0; r < runs; ++r) {
        off[r] = total;
        total += len[r];
    }
    *result_in_scratch = 0;
    if (runs > 1 && total > 0) {
        if (!keys || !scratch_keys || (value_bytes && (!values || !scratch_values)))
            return fail(RSORT_BAD_ARGUMENT, "null buffer");
        rsort_status sa = check_alignment(addr(keys) | addr(scratch_keys), size_t(kb),
                                          "merge keys alignment");
        if (sa == RSORT_OK)
            sa = check_alignment(addr(values) | addr(scratch_values), value_bytes,
                                 "merge values alignment");
        if (sa != RSORT_OK) return sa;
        DeviceInfo dev;
        rsort_status st = device_info(&dev);
        if (st != RSORT_OK) return st;
    }
    // Pairwise merge tree: runs (0,1), (2,3), ... each round, one batched
    // launch per round; ties keep the lower run first, so the result is
    // stable across runs in run order.
    char *src_k = static_cast<char *>(keys), *dst_k = static_cast<char *>(scratch_keys);
    char *src_v = static_cast<char *>(values), *dst_v = static_cast<char *>(scratch_values);
    bool in_scratch = false;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    while (len.size() > 1) {
        std::vector<size_t> nlen, noff;
        std::vector<PairMerge> pairs;
        for (size_t r = 0; r < len.size(); r += 2) {
            if (r + 1 < len.size()) {
                pairs.push_back(PairMerge{
                    src_k + off[r] * kb, value_bytes ? src_v + off[r] * value_bytes : nullptr,
                    len[r], src_k + off[r + 1] * kb,
                    value_bytes ? src_v + off[r + 1] * value_bytes : nullptr, len[r + 1],
                    dst_k + off[r] * kb, value_bytes ? dst_v + off[r] * value_bytes : nullptr});
                nlen.push_back(len[r] + len[r + 1]);
            } else {
                if (len[r]) {
                    cudaError_t e = cudaMemcpyAsync(dst_k + off[r] * kb, src_k + off[r] * kb,
                                                    len[r] * kb, cudaMemcpyDeviceToDevice, s);
                    if (e == cudaSuccess && value_bytes)
                        e = cudaMemcpyAsync(dst_v + off[r] * value_bytes,
                                            src_v + off[r] * value_bytes, len[r] * value_bytes,
                                            cudaMemcpyDeviceToDevice, s);
                    if (e != cudaSuccess) return cuda_fail(e, "merge run copy");
                }
                nlen.push_back(len[r]);
            }
            noff.push_back(off[r]);
        }
        rsort_status st = merge_round(key, descending, pairs, value_bytes, d_partitions,
                                      npartitions, s);
        if (st != RSORT_OK) return st;
        len.swap(nlen);
        off.swap(noff);
        std::swap(src_k, dst_k);
        std::swap(src_v, dst_v);
        in_scratch = !in_scratch;
    }
    *result_in_scratch = in_scratch ? 1 : 0;
    return RSORT_OK;
}


rsort_status rsort_merge_segments(rsort_key_t key, int descending, unsigned runs,
                                  const void *const *run_keys, const void *const *run_values,
                                  const size_t *run_lengths, size_t value_bytes, void *out_keys,
                                  void *out_values, void *scratch_keys, void *scratch_values,
                                  uint64_t *d_partitions, size_t npartitions,
                                  int *result_in_scratch, unsigned first_pair,
                                  rsort_stream_t stream) {
    if (!wide_key(key)) return fail(RSORT_BAD_ARGUMENT, "key type (32- or 64-bit keys only)");
    if (!value_ok(value_bytes)) return fail(RSORT_BAD_ARGUMENT, "radix value width");
    if (!result_in_scratch || (runs && (!run_lengths || !run_keys || (value_bytes && !run_values))))
        return fail(RSORT_BAD_ARGUMENT, "null argument");
    *result_in_scratch = 0;
    const size_t kb = size_t(key_bytes(key));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    char *ok = static_cast<char *>(out_keys), *ov = static_cast<char *>(out_values);
    // First round straight from the given runs (a peer's memory is read once,
    // by the merge itself): pairs (0,1), (2,3), ... into out, all in one
    // batched launch whose blocks interleave the pairs, so every peer is read
    // at once.  Pairs are listed from first_pair on (wrapping): ranks starting
    // at different pairs begin their reads on different peers.  The output
    // layout does not depend on the order.
    const unsigned pairs = (runs + 1) / 2;
    std::vector<size_t> len(pairs), at(pairs);
    size_t off = 0;
    for (unsigned p = 0; p < pairs; ++p) {
        const unsigned r = 2 * p;
        len[p] = run_lengths[r] + (r + 1 < runs ? run_lengths[r + 1] : 0);
        at[p] = off;
        off += len[p];
    }
    if (off > 0) {
        if (!ok || (value_bytes && !ov)) return fail(RSORT_BAD_ARGUMENT, "null buffer");
        uintptr_t kbits = addr(ok), vbits = addr(ov);
        for (unsigned r = 0; r < runs; ++r) {
            kbits |= addr(run_keys[r]);
            if (value_bytes) vbits |= addr(run_values[r]);
        }
        rsort_status sa = check_alignment(kbits, size_t(kb), "merge keys alignment");
        if (sa == RSORT_OK) sa = check_alignment(vbits, value_bytes, "merge values alignment");
        if (sa != RSORT_OK) return sa;
        DeviceInfo dev;
        rsort_status st = device_info(&dev);
        if (st != RSORT_OK) return st;
    }
    std::vector<PairMerge> first;
    for (unsigned k = 0; k < pairs; ++k) {
        const unsigned p = (first_pair + k) % pairs;
        const unsigned r = 2 * p;
        const size_t o = at[p];
        if (r + 1 < runs) {
            if ((run_lengths[r] && !run_keys[r]) || (run_lengths[r + 1] && !run_keys[r + 1]))
                return fail(RSORT_BAD_ARGUMENT, "null run");
            first.push_back(PairMerge{run_keys[r], value_bytes ? run_values[r] : nullptr,
                                      run_lengths[r], run_keys[r + 1],
                                      value_bytes ? run_values[r + 1] : nullptr,
                                      run_lengths[r + 1], ok + o * kb,
                                      value_bytes ? ov + o * value_bytes : nullptr});
        } else if (run_lengths[r]) {
            cudaError_t e = cudaMemcpyAsync(ok + o * kb, run_keys[r], run_lengths[r] * kb,
                                            cudaMemcpyDeviceToDevice, s);
            if (e == cudaSuccess && value_bytes)
                e = cudaMemcpyAsync(ov + o * value_bytes, run_values[r],
                                    run_lengths[r] * value_bytes, cudaMemcpyDeviceToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, "merge run copy");
        }
    }
    rsort_status st = merge_round(key, descending, first, value_bytes, d_partitions, npartitions, s);
    if (st != RSORT_OK) return st;
    if (len.size() <= 1) return RSORT_OK;
    // Later rounds in local memory, between out and scratch.
    return rsort_merge_runs(key, descending, out_keys, out_values, value_bytes, len.data(),
                            unsigned(len.size()), scratch_keys, scratch_values, d_partitions,
                            npartitions, result_in_scratch, stream);
}

// Failure-detection self test: one onesweep CTA is handed tile 1 of a
// two-tile input whose tile 0 is never processed, so its look-back waits on a
// word nothing publishes.  The wait must give up within its bound, set the
// status word and skip its writes; the call returns the status the host reads.
rsort_status rsort_selftest_lookback_timeout(rsort_stream_t stream) {
    DeviceInfo dev;
    rsort_status st = device_info(&dev);
    if (st != RSORT_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const size_t tile = size_t(onesweep_tile(4, 0));
    const size_t n = 2 * tile;
    uint32_t *keys = nullptr, *out = nullptr;
    uint64_t *bins = nullptr, *lookback = nullptr;
    int32_t *counters = nullptr;
    cudaError_t e = cudaMalloc(&keys, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&out, n * 4);
    if (e == cudaSuccess) e = cudaMalloc(&bins, RADIX * 8);
    if (e == cudaSuccess) e = cudaMalloc(&lookback, 2 * RADIX * 8);
    if (e == cudaSuccess) e = cudaMalloc(&counters, CTR_WORDS * 4);
    if (e == cudaSuccess) e = cudaMemsetAsync(keys, 0, n * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(out, 0, n * 4, s);
    // Two non-empty digit buckets (digit 0 and digit 255, n/2 keys each), so
    // the pass is not a one-bucket identity copy and the tile must look back.
    std::vector<uint64_t> host_bins(RADIX, n / 2);
    host_bins[0] = 0;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(bins, host_bins.data(), RADIX * 8, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(lookback, 0, 2 * RADIX * 8, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(counters, 0, CTR_WORDS * 4, s);
    const int32_t one = 1;  // the single CTA claims tile 1
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(counters + CTR_TILE, &one, sizeof(one), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        PassArgs a{};
        a.keys_in = keys;
        a.keys_out = out;
        a.n = n;
        a.bins = bins;
        a.lookback = lookback;
        a.tile_counter = counters + CTR_TILE;
        a.status = counters + CTR_STATUS;
        a.shift = 0;
        a.mask = 0xff;
        a.kind = KIND_UINT;
        a.first = 1;
        a.last = 1;
        a.tag = 1;
        e = launch_onesweep(4, 0, a, 1, s);
    }
    int32_t word = 0;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(&word, counters + CTR_STATUS, sizeof(word), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(keys);
    cudaFree(out);
    cudaFree(bins);
    cudaFree(lookback);
    cudaFree(counters);
    if (e != cudaSuccess) return cuda_fail(e, "self test");
    if (word == DEV_STATUS_TIMEOUT) return fail(RSORT_TIMEOUT, "radix look-back wait (self test)");
    return word == 0 ? RSORT_OK : fail(RSORT_CUDA_ERROR, "radix scatter bounds check");
}

void rsort_profile_enable(int enable) { g_profile = enable != 0; }

size_t rsort_profile_read(int32_t *kernel_ids, float *milliseconds, size_t capacity) {
    size_t n = 0;
    for (const ProfiledLaunch &r : g_profiled) {
        float ms = 0.f;
        if (cudaEventSynchronize(r.stop) == cudaSuccess) cudaEventElapsedTime(&ms, r.start, r.stop);
        if (n < capacity) {
            if (kernel_ids) kernel_ids[n] = r.kernel;
            if (milliseconds) milliseconds[n] = ms;
        }
        ++n;
        g_event_pool.push_back(r.start);
        g_event_pool.push_back(r.stop);
    }
    g_profiled.clear();
    return n;
}

}  // extern "C"
