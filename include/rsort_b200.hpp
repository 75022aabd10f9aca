// rsort_b200.hpp -- header-only C++17 mirror of rccl-cub's DeviceRadixSort API
// over the C ABI in rsort_b200.h.
//
// Same names, argument meaning and error behaviour as the reference's public
// radix functions (rccl-cub/src/dispatch.rs:2091-2942), DoubleBuffer
// (rccl-cub/src/double_buffer.rs:6-130) and DeviceAlgorithmError
// (rccl-cub/src/error.rs:1-84).  Device memory is plain caller-owned device
// pointers; calls are asynchronous on the given stream.
#ifndef RSORT_B200_HPP
#define RSORT_B200_HPP

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>

#include <cuda_runtime_api.h>

#include "rsort_b200.h"

namespace rccl_b200 {
namespace cub {

// The sealed RadixKey set (rccl-cub/src/radix.rs:114-173).
template <typename K> struct RadixKey;
template <> struct RadixKey<uint32_t> { static constexpr rsort_key_t code = RSORT_U32; };
template <> struct RadixKey<int32_t> { static constexpr rsort_key_t code = RSORT_I32; };
template <> struct RadixKey<float> { static constexpr rsort_key_t code = RSORT_F32; };
template <> struct RadixKey<uint64_t> { static constexpr rsort_key_t code = RSORT_U64; };
template <> struct RadixKey<int64_t> { static constexpr rsort_key_t code = RSORT_I64; };
template <> struct RadixKey<double> { static constexpr rsort_key_t code = RSORT_F64; };
// Small integer keys (no reference counterpart).  Half and bfloat16 keys go
// through the C ABI with RSORT_F16 / RSORT_BF16 on their 16-bit storage.
template <> struct RadixKey<uint8_t> { static constexpr rsort_key_t code = RSORT_U8; };
template <> struct RadixKey<int8_t> { static constexpr rsort_key_t code = RSORT_I8; };
template <> struct RadixKey<uint16_t> { static constexpr rsort_key_t code = RSORT_U16; };
template <> struct RadixKey<int16_t> { static constexpr rsort_key_t code = RSORT_I16; };

// DeviceAlgorithmError: one exception type whose `kind` names the variant and
// whose fields carry that variant's payload.
class DeviceAlgorithmError : public std::runtime_error {
  public:
    explicit DeviceAlgorithmError(const rsort_error_info &info, rsort_status status)
        : std::runtime_error(describe(info, status)), kind(status), role(info.role ? info.role : ""),
          expected(info.expected), actual(info.actual), begin(info.begin_bit), end(info.end_bit),
          key_bits(info.key_bits) {}
    rsort_status kind;
    std::string role;
    size_t expected, actual;
    unsigned begin, end, key_bits;

  private:
    static std::string describe(const rsort_error_info &i, rsort_status s) {
        switch (s) {
            case RSORT_INVALID_BIT_RANGE:
                return "radix bit range " + std::to_string(i.begin_bit) + ".." +
                       std::to_string(i.end_bit) + " is outside 0..=" + std::to_string(i.key_bits) +
                       " or reversed";
            case RSORT_LENGTH_MISMATCH:
                return std::string(i.role ? i.role : "") + " length " + std::to_string(i.actual) +
                       " does not match required length " + std::to_string(i.expected);
            case RSORT_WORKSPACE_TOO_SMALL:
                return std::string(i.role ? i.role : "") + " length " + std::to_string(i.actual) +
                       " is smaller than required length " + std::to_string(i.expected);
            default:
                return std::string(rsort_status_string(s)) + (i.role ? std::string(": ") + i.role : "");
        }
    }
};

inline void check(rsort_status s) {
    if (s == RSORT_OK) return;
    rsort_error_info info{};
    rsort_last_error(&info);
    throw DeviceAlgorithmError(info, s);
}

// Two same-shaped ranges used by ping-pong sorts (double_buffer.rs:6-130).
template <typename K>
struct DoubleBuffer {
    K *first, *second;
    size_t len;
    bool current_is_first = true;
    DoubleBuffer(K *f, K *s, size_t n) : first(f), second(s), len(n) {}
    K *current() const { return current_is_first ? first : second; }
    K *alternate() const { return current_is_first ? second : first; }
    void swap() { current_is_first = !current_is_first; }
};

// Paired form: one selector for keys and values (DoubleBuffer::paired).
template <typename K, typename V>
struct PairedDoubleBuffer {
    K *first_keys, *second_keys;
    V *first_values, *second_values;
    size_t len;
    bool current_is_first = true;
    K *current_keys() const { return current_is_first ? first_keys : second_keys; }
    V *current_values() const { return current_is_first ? first_values : second_values; }
};

// The three control regions of DeviceRadixSortBufferWorkspace (caller owned).
struct DeviceRadixSortBufferWorkspace {
    uint64_t *bins = nullptr;
    size_t nbins = 0;
    int32_t *lookback = nullptr;
    size_t nlookback = 0;
    int32_t *counters = nullptr;
    size_t ncounters = 0;
};

// Element counts the workspace needs (workspace.rs:68-106 counterpart).
template <typename K, typename V = void>
inline rsort_controls workspace_counts(size_t n) {
    rsort_controls c{};
    const size_t vb = std::is_void<V>::value ? 0 : sizeof(typename std::conditional<
                                                       std::is_void<V>::value, char, V>::type);
    check(rsort_controls_query(RadixKey<K>::code, vb, n, &c));
    return c;
}

// --- keys ------------------------------------------------------------------
template <typename K>
inline void device_radix_sort_keys(cudaStream_t stream, K *keys, K *scratch, size_t n,
                                   const DeviceRadixSortBufferWorkspace &ws) {
    check(rsort_keys(RadixKey<K>::code, 0, keys, scratch, n, n, ws.bins, ws.nbins, ws.lookback,
                     ws.nlookback, ws.counters, ws.ncounters,
                     reinterpret_cast<rsort_stream_t>(stream)));
}

template <typename K>
inline void device_radix_sort_keys_descending(cudaStream_t stream, K *keys, K *scratch, size_t n,
                                              const DeviceRadixSortBufferWorkspace &ws) {
    check(rsort_keys(RadixKey<K>::code, 1, keys, scratch, n, n, ws.bins, ws.nbins, ws.lookback,
                     ws.nlookback, ws.counters, ws.ncounters,
                     reinterpret_cast<rsort_stream_t>(stream)));
}

template <typename K>
inline void device_radix_sort_keys_buffer_impl(cudaStream_t stream, DoubleBuffer<K> &b,
                                               unsigned begin, unsigned end,
                                               const DeviceRadixSortBufferWorkspace &ws, int desc) {
    int sel = b.current_is_first ? 1 : 0;
    check(rsort_keys_buffer(RadixKey<K>::code, desc, b.first, b.second, b.len, begin, end, &sel,
                            ws.bins, ws.nbins, ws.lookback, ws.nlookback, ws.counters,
                            ws.ncounters, reinterpret_cast<rsort_stream_t>(stream)));
    b.current_is_first = sel != 0;
}

template <typename K>
inline void device_radix_sort_keys_buffer(cudaStream_t stream, DoubleBuffer<K> &b, unsigned begin,
                                          unsigned end, const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_keys_buffer_impl(stream, b, begin, end, ws, 0);
}

template <typename K>
inline void device_radix_sort_keys_buffer_descending(cudaStream_t stream, DoubleBuffer<K> &b,
                                                     unsigned begin, unsigned end,
                                                     const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_keys_buffer_impl(stream, b, begin, end, ws, 1);
}

// --- pairs -----------------------------------------------------------------
template <typename K, typename V>
inline void device_radix_sort_pairs_impl(cudaStream_t stream, K *keys, V *values, K *scratch_keys,
                                         V *scratch_values, size_t n,
                                         const DeviceRadixSortBufferWorkspace &ws, int desc) {
    check(rsort_pairs(RadixKey<K>::code, desc, keys, values, sizeof(V), scratch_keys, n,
                      scratch_values, n, n, ws.bins, ws.nbins, ws.lookback, ws.nlookback,
                      ws.counters, ws.ncounters, reinterpret_cast<rsort_stream_t>(stream)));
}

template <typename K, typename V>
inline void device_radix_sort_pairs(cudaStream_t stream, K *keys, V *values, K *scratch_keys,
                                    V *scratch_values, size_t n,
                                    const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_pairs_impl(stream, keys, values, scratch_keys, scratch_values, n, ws, 0);
}

template <typename K, typename V>
inline void device_radix_sort_pairs_descending(cudaStream_t stream, K *keys, V *values,
                                               K *scratch_keys, V *scratch_values, size_t n,
                                               const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_pairs_impl(stream, keys, values, scratch_keys, scratch_values, n, ws, 1);
}

template <typename K, typename V>
inline void device_radix_sort_pairs_buffer_impl(cudaStream_t stream, PairedDoubleBuffer<K, V> &b,
                                                unsigned begin, unsigned end,
                                                const DeviceRadixSortBufferWorkspace &ws,
                                                int desc) {
    int sel = b.current_is_first ? 1 : 0;
    check(rsort_pairs_buffer(RadixKey<K>::code, desc, b.first_keys, b.second_keys,
                             b.first_values, b.second_values, sizeof(V), b.len, begin, end, &sel,
                             ws.bins, ws.nbins, ws.lookback, ws.nlookback, ws.counters,
                             ws.ncounters, reinterpret_cast<rsort_stream_t>(stream)));
    b.current_is_first = sel != 0;
}

template <typename K, typename V>
inline void device_radix_sort_pairs_buffer(cudaStream_t stream, PairedDoubleBuffer<K, V> &b,
                                           unsigned begin, unsigned end,
                                           const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_pairs_buffer_impl(stream, b, begin, end, ws, 0);
}

template <typename K, typename V>
inline void device_radix_sort_pairs_buffer_descending(cudaStream_t stream,
                                                      PairedDoubleBuffer<K, V> &b, unsigned begin,
                                                      unsigned end,
                                                      const DeviceRadixSortBufferWorkspace &ws) {
    device_radix_sort_pairs_buffer_impl(stream, b, begin, end, ws, 1);
}

// --- DeviceMergeSort / DeviceMerge for named orders -------------------------
// (rccl-cub dispatch.rs:170-193, 1113-1146, 1570-1601 take a comparator
// closure; here the comparator is one of the named orders of rsort_order_t.)
enum class Order : int {
    Ascending = RSORT_ORDER_ASCENDING,
    Descending = RSORT_ORDER_DESCENDING,
    TotalAscending = RSORT_ORDER_TOTAL_ASCENDING,
    TotalDescending = RSORT_ORDER_TOTAL_DESCENDING,
};

template <typename K>
inline void device_merge_sort_keys(cudaStream_t stream, K *keys, K *scratch, size_t n,
                                   const DeviceRadixSortBufferWorkspace &ws, Order order) {
    check(rsort_merge_sort_keys(RadixKey<K>::code, static_cast<rsort_order_t>(order), keys,
                                scratch, n, n, ws.bins, ws.nbins, ws.lookback, ws.nlookback,
                                ws.counters, ws.ncounters, reinterpret_cast<rsort_stream_t>(stream)));
}

template <typename K, typename V>
inline void device_merge_sort_pairs(cudaStream_t stream, K *keys, V *values, K *scratch_keys,
                                    V *scratch_values, size_t n,
                                    const DeviceRadixSortBufferWorkspace &ws, Order order) {
    check(rsort_merge_sort_pairs(RadixKey<K>::code, static_cast<rsort_order_t>(order), keys,
                                 values, sizeof(V), scratch_keys, n, scratch_values, n, n, ws.bins,
                                 ws.nbins, ws.lookback, ws.nlookback, ws.counters, ws.ncounters,
                                 reinterpret_cast<rsort_stream_t>(stream)));
}

// d_partitions: rsort_merge_partition_words(na + nb) words.
template <typename K>
inline void device_merge_keys(cudaStream_t stream, const K *first, size_t na, const K *second,
                              size_t nb, uint64_t *d_partitions, size_t npartitions, K *output,
                              Order order) {
    check(rsort_merge_ordered(RadixKey<K>::code, static_cast<rsort_order_t>(order), first, nullptr,
                              na, second, nullptr, nb, output, nullptr, 0, d_partitions,
                              npartitions, reinterpret_cast<rsort_stream_t>(stream)));
}

template <typename K, typename V>
inline void device_merge_pairs(cudaStream_t stream, const K *first_keys, const V *first_values,
                               size_t na, const K *second_keys, const V *second_values, size_t nb,
                               uint64_t *d_partitions, size_t npartitions, K *output_keys,
                               V *output_values, Order order) {
    check(rsort_merge_ordered(RadixKey<K>::code, static_cast<rsort_order_t>(order), first_keys,
                              first_values, na, second_keys, second_values, nb, output_keys,
                              output_values, sizeof(V), d_partitions, npartitions,
                              reinterpret_cast<rsort_stream_t>(stream)));
}

}  // namespace cub
}  // namespace rccl_b200

#endif  // RSORT_B200_HPP
