// Comparator only, never part of the product: CUB's own DeviceRadixSort
// (the CCCL headers shipped with the CUDA toolkit, built for sm_100a), which
// the reference's radix path ports.  The reference's cuda-oxide build cannot
// run here, so bench.py --cub-proxy times this beside librsort_b200 on the
// same inputs.  Built by bench.py into baseline/_cub/.
#include <cstddef>
#include <cstdint>

#include <cub/device/device_radix_sort.cuh>
#include <cuda_runtime.h>

namespace {

// kind: 0 = u64 keys / u32 values ascending, 1 = f32 keys descending,
//       2 = u32 keys ascending
template <typename F>
int dispatch(int kind, F &&f) {
    switch (kind) {
        case 0: return f(static_cast<uint64_t *>(nullptr), static_cast<uint32_t *>(nullptr), false);
        case 1: return f(static_cast<float *>(nullptr), static_cast<cub::NullType *>(nullptr), true);
        case 2: return f(static_cast<uint32_t *>(nullptr), static_cast<cub::NullType *>(nullptr), false);
        default: return int(cudaErrorInvalidValue);
    }
}

}  // namespace

// Temporary storage CUB needs for n items (DoubleBuffer form).
extern "C" int cub_proxy_temp_bytes(int kind, size_t n, size_t *bytes) {
    return dispatch(kind, [&](auto *k, auto *v, bool desc) -> int {
        using K = std::remove_pointer_t<decltype(k)>;
        using V = std::remove_pointer_t<decltype(v)>;
        cub::DoubleBuffer<K> keys(nullptr, nullptr);
        cudaError_t e;
        if constexpr (std::is_same_v<V, cub::NullType>) {
            e = desc ? cub::DeviceRadixSort::SortKeysDescending(nullptr, *bytes, keys, int(n))
                     : cub::DeviceRadixSort::SortKeys(nullptr, *bytes, keys, int(n));
        } else {
            cub::DoubleBuffer<V> values(nullptr, nullptr);
            e = cub::DeviceRadixSort::SortPairs(nullptr, *bytes, keys, values, int(n));
        }
        return int(e);
    });
}

// One full-width sort; *selector is which buffer (0 = first) holds the result.
extern "C" int cub_proxy_sort(int kind, void *k0, void *k1, void *v0, void *v1, size_t n, void *temp,
                              size_t temp_bytes, int *selector, cudaStream_t stream) {
    return dispatch(kind, [&](auto *k, auto *v, bool desc) -> int {
        using K = std::remove_pointer_t<decltype(k)>;
        using V = std::remove_pointer_t<decltype(v)>;
        cub::DoubleBuffer<K> keys(static_cast<K *>(k0), static_cast<K *>(k1));
        cudaError_t e;
        if constexpr (std::is_same_v<V, cub::NullType>) {
            e = desc ? cub::DeviceRadixSort::SortKeysDescending(temp, temp_bytes, keys, int(n), 0,
                                                                int(sizeof(K) * 8), stream)
                     : cub::DeviceRadixSort::SortKeys(temp, temp_bytes, keys, int(n), 0,
                                                      int(sizeof(K) * 8), stream);
        } else {
            cub::DoubleBuffer<V> values(static_cast<V *>(v0), static_cast<V *>(v1));
            e = cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys, values, int(n), 0,
                                                int(sizeof(K) * 8), stream);
        }
        *selector = keys.selector;
        return int(e);
    });
}
