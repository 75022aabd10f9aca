// C++ mirror (include/rsort_b200.hpp) tests.  Without arguments: host-only
// checks (validation errors, workspace counts); with --gpu: device sorts
// checked against std::stable_sort restatements of the probes' expectations.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <random>
#include <vector>

#include "rsort_b200.hpp"

using namespace rccl_b200::cub;

#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            std::fprintf(stderr, "FAILED %s:%d %s\n", __FILE__, __LINE__, #cond); \
            return 1;                                                        \
        }                                                                    \
    } while (0)

static int host_checks() {
    // rccl-cub/examples/device_radix_sort_keys_probe.rs:360-376: InvalidBitRange{25,17,32}
    uint32_t *fake = reinterpret_cast<uint32_t *>(uintptr_t(256));
    DoubleBuffer<uint32_t> b(fake, fake + 64, 4);
    DeviceRadixSortBufferWorkspace ws{};
    bool threw = false;
    try {
        device_radix_sort_keys_buffer(nullptr, b, 25, 17, ws);
    } catch (const DeviceAlgorithmError &e) {
        threw = true;
        CHECK(e.kind == RSORT_INVALID_BIT_RANGE);
        CHECK(e.begin == 25 && e.end == 17 && e.key_bits == 32);
    }
    CHECK(threw);
    CHECK(b.current_is_first);
    // Empty window: no launch, no selector change (radix.rs:467-469).
    device_radix_sort_keys_buffer(nullptr, b, 12, 12, ws);
    CHECK(b.current_is_first);
    // Controls are empty on the single-tile route (workspace.rs:96-106).
    rsort_controls c = workspace_counts<uint32_t>(4864);
    CHECK(c.bins == 0 && c.lookback == 0 && c.counters == 0);
    c = workspace_counts<uint64_t, uint32_t>(1 << 20);
    CHECK(c.bins == 8 * 256 && c.lookback > 0);
    // LengthMismatch on the look-back region.
    c = workspace_counts<uint32_t>(100000);
    DeviceRadixSortBufferWorkspace bad{reinterpret_cast<uint64_t *>(uintptr_t(4096)), c.bins,
                                       reinterpret_cast<int32_t *>(uintptr_t(8192)), c.lookback + 2,
                                       reinterpret_cast<int32_t *>(uintptr_t(65536)), c.counters};
    DoubleBuffer<uint32_t> big(fake, fake + 64, 100000);
    threw = false;
    try {
        device_radix_sort_keys_buffer(nullptr, big, 0, 32, bad);
    } catch (const DeviceAlgorithmError &e) {
        threw = true;
        CHECK(e.kind == RSORT_LENGTH_MISMATCH && e.role == "radix lookback");
        CHECK(e.expected == c.lookback && e.actual == c.lookback + 2);
    }
    CHECK(threw);
    std::printf("host checks: PASS\n");
    return 0;
}

template <typename T>
static T *dev_copy(const std::vector<T> &h) {
    T *d = nullptr;
    cudaMalloc(reinterpret_cast<void **>(&d), std::max<size_t>(1, h.size()) * sizeof(T));
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

template <typename T>
static std::vector<T> host_copy(const T *d, size_t n) {
    std::vector<T> h(n);
    cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
    return h;
}

static DeviceRadixSortBufferWorkspace make_ws(rsort_controls c) {
    DeviceRadixSortBufferWorkspace ws{};
    ws.nbins = c.bins;
    ws.nlookback = c.lookback;
    ws.ncounters = c.counters;
    if (c.bins) cudaMalloc(reinterpret_cast<void **>(&ws.bins), c.bins * 8);
    if (c.lookback) cudaMalloc(reinterpret_cast<void **>(&ws.lookback), c.lookback * 4);
    if (c.counters) {
        cudaMalloc(reinterpret_cast<void **>(&ws.counters), c.counters * 4);
        cudaMemset(ws.counters, 0, c.counters * 4);
    }
    return ws;
}

static int gpu_checks() {
    std::mt19937_64 rng(11);
    // Stable u64/u32 pairs, ascending (BASELINE config 2 shape, smaller n).
    const size_t n = 1 << 20;
    std::vector<uint64_t> keys(n);
    for (auto &k : keys) k = rng() & 0xffffffffffull;  // duplicates
    std::vector<uint32_t> vals(n);
    std::iota(vals.begin(), vals.end(), 0u);
    uint64_t *dk = dev_copy(keys), *sk = dev_copy(keys);
    uint32_t *dv = dev_copy(vals), *sv = dev_copy(vals);
    auto ws = make_ws(workspace_counts<uint64_t, uint32_t>(n));
    device_radix_sort_pairs(nullptr, dk, dv, sk, sv, n, ws);
    std::vector<size_t> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return keys[a] < keys[b]; });
    auto gk = host_copy(dk, n);
    auto gv = host_copy(dv, n);
    for (size_t i = 0; i < n; ++i) {
        CHECK(gk[i] == keys[order[i]]);
        CHECK(gv[i] == order[i]);
    }
    // i32 descending probe (device_radix_sort_keys_probe.rs:75-83).
    std::vector<int32_t> si{0, -1, INT32_MIN, 7, -9, INT32_MAX, -1, 0};
    int32_t *ds = dev_copy(si), *ss = dev_copy(si);
    device_radix_sort_keys_descending(nullptr, ds, ss, si.size(), make_ws(workspace_counts<int32_t>(8)));
    auto gs = host_copy(ds, si.size());
    const int32_t want[] = {INT32_MAX, 7, 0, 0, -1, -1, -9, INT32_MIN};
    CHECK(std::equal(gs.begin(), gs.end(), want));
    // DoubleBuffer window 0..24 (device_radix_sort_keys_probe.rs:300-339): 3 passes.
    std::vector<uint32_t> w(10003);
    for (uint32_t i = 0; i < w.size(); ++i) w[i] = ((i & 0xff) << 24) | ((i * 2654435761u) & 0xffffff);
    uint32_t *wf = dev_copy(w), *ws2 = dev_copy(w);
    DoubleBuffer<uint32_t> db(wf, ws2, w.size());
    device_radix_sort_keys_buffer(nullptr, db, 0, 24, make_ws(workspace_counts<uint32_t>(w.size())));
    CHECK(!db.current_is_first);
    auto gw = host_copy(db.current(), w.size());
    std::vector<uint32_t> ew = w;
    std::stable_sort(ew.begin(), ew.end(), [](uint32_t a, uint32_t b) { return (a & 0xffffff) < (b & 0xffffff); });
    CHECK(gw == ew);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    std::printf("gpu checks: PASS\n");
    return 0;
}

int main(int argc, char **argv) {
    if (host_checks()) return 1;
    if (argc > 1 && std::strcmp(argv[1], "--gpu") == 0) return gpu_checks();
    return 0;
}
