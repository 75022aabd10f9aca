// CPU comparison-sort stand-ins for the benchmark's CPU baseline.
//
// TEST INFRASTRUCTURE ONLY (the benchmark's CPU baseline leg).  The benchmark
// asks for Rust `slice::sort_unstable` (single core) and rayon
// `par_sort_unstable` (all cores); neither Rust nor rayon exists in this
// environment, so these are the C++ standard library's equivalents:
//   - one thread: std::sort (keys; unstable like sort_unstable) or
//     std::stable_sort (key/value pairs, whose order must be stable);
//   - T threads: T chunks sorted by std::thread workers, then pairwise
//     std::merge rounds (stable: ties take the earlier chunk), each round's
//     merges on their own threads.
// The order is the radix order of the reference (the order image of
// radix_oracle.c: to_ordered plus the float zero fold), compared directly.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "radix_oracle.h"

namespace {

template <typename B>
struct Img {
    int kt, desc;
    uint64_t operator()(B raw) const { return orc_fold(kt, orc_to_ordered(kt, desc, uint64_t(raw))); }
};

template <typename T, typename Less>
void chunked_sort(T *data, size_t n, int threads, bool stable, Less less) {
    if (threads <= 1 || n < 4096) {
        if (stable) std::stable_sort(data, data + n, less);
        else std::sort(data, data + n, less);
        return;
    }
    std::vector<size_t> bounds;
    for (int t = 0; t <= threads; ++t) bounds.push_back(n * size_t(t) / size_t(threads));
    {
        std::vector<std::thread> pool;
        for (int t = 0; t < threads; ++t)
            pool.emplace_back([&, t] {
                if (stable) std::stable_sort(data + bounds[t], data + bounds[t + 1], less);
                else std::sort(data + bounds[t], data + bounds[t + 1], less);
            });
        for (auto &th : pool) th.join();
    }
    std::vector<T> tmp(n);
    T *src = data, *dst = tmp.data();
    while (bounds.size() > 2) {
        std::vector<size_t> next;
        std::vector<std::thread> pool;
        for (size_t i = 0; i + 1 < bounds.size(); i += 2) {
            const size_t a = bounds[i], b = bounds[i + 1];
            const size_t c = i + 2 < bounds.size() ? bounds[i + 2] : b;
            next.push_back(a);
            pool.emplace_back([=] {
                if (c > b) std::merge(src + a, src + b, src + b, src + c, dst + a, less);
                else std::copy(src + a, src + b, dst + a);
            });
        }
        next.push_back(bounds.back());
        for (auto &th : pool) th.join();
        bounds.swap(next);
        std::swap(src, dst);
    }
    if (src != data) std::copy(src, src + n, data);
}

template <typename B>
int sort_typed(int kt, int desc, int stable, B *keys, uint32_t *values, size_t n, int threads) {
    const Img<B> img{kt, desc};
    if (!values) {
        // Sort order images, then map back: the comparison costs one integer
        // compare, as a Rust sort of primitive keys does.
        std::vector<uint64_t> v(n);
        for (size_t i = 0; i < n; ++i) v[i] = img(keys[i]);
        if (stable) {
            // Keep the input order of equal images (the two float zeros).
            struct KI { uint64_t k; B raw; };
            std::vector<KI> kv(n);
            for (size_t i = 0; i < n; ++i) kv[i] = {v[i], keys[i]};
            chunked_sort(kv.data(), n, threads, true,
                         [](const KI &a, const KI &b) { return a.k < b.k; });
            for (size_t i = 0; i < n; ++i) keys[i] = kv[i].raw;
        } else {
            chunked_sort(v.data(), n, threads, false, std::less<uint64_t>());
            for (size_t i = 0; i < n; ++i) keys[i] = B(orc_from_ordered(kt, desc, v[i]));
        }
        return ORC_OK;
    }
    struct KV { uint64_t k; B raw; uint32_t v; };
    std::vector<KV> kv(n);
    for (size_t i = 0; i < n; ++i) kv[i] = {img(keys[i]), keys[i], values[i]};
    chunked_sort(kv.data(), n, threads, stable != 0,
                 [](const KV &a, const KV &b) { return a.k < b.k; });
    for (size_t i = 0; i < n; ++i) {
        keys[i] = kv[i].raw;
        values[i] = kv[i].v;
    }
    return ORC_OK;
}

}  // namespace

extern "C" int orc_cpu_sort(int key_type, int descending, int stable, void *keys,
                            uint32_t *values, size_t n, int threads) {
    if (key_type < ORC_U32 || key_type > ORC_F64 || (n && !keys)) return ORC_BAD_ARGUMENT;
    if (orc_key_bytes(key_type) == 4)
        return sort_typed(key_type, descending, stable, static_cast<uint32_t *>(keys), values, n,
                          threads);
    return sort_typed(key_type, descending, stable, static_cast<uint64_t *>(keys), values, n,
                      threads);
}
