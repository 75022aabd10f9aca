// Launchers of the lexicographic record sort's gathers (rsort_records.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace rsort {

// keys[i] = words [first, first + count) of row perm[i] (count 1 or 2, word
// `first` in the high half); perm == nullptr means the identity.
cudaError_t launch_chunk_keys(const uint32_t *rows, uint32_t words, const uint32_t *perm,
                              uint64_t n, uint32_t first, uint32_t count, uint64_t *keys,
                              int sm_count, cudaStream_t s);
// perm[i] = i
cudaError_t launch_iota(uint32_t *perm, uint64_t n, int sm_count, cudaStream_t s);
// dst item i = src item perm[i] (items of item_bytes)
cudaError_t launch_permute(const void *src, const uint32_t *perm, uint64_t n, size_t item_bytes,
                           void *dst, int sm_count, cudaStream_t s);

// One term of a comparator program, prepared on the host: the field (byte
// offset, width in bytes, key kind), the projection and its operand, the
// direction, and the bit window [lo, lo + width) of the projected value's
// order image that can differ between records (the only bits the key needs).
struct CompareTerm {
    uint32_t offset;
    uint8_t bytes;       // 1, 2, 4 or 8
    uint8_t kind;        // KeyKind
    uint8_t projection;  // rsort_projection_t
    uint8_t desc;
    uint8_t aligned;     // every record's field is aligned to `bytes`
    uint8_t lo, width;
    int64_t operand;
};

// Terms whose windows are packed into one sort key, most significant first;
// total_bits <= 64 (<= 32: the key is 32-bit).
constexpr int COMPARE_GROUP_MAX = 16;
struct CompareGroup {
    CompareTerm term[COMPARE_GROUP_MAX];
    uint32_t nterms;
    uint32_t total_bits;
};

// keys[i] = the group's packed window bits of record perm[i] (perm ==
// nullptr: the identity); 32-bit keys when total_bits <= 32, else 64-bit.
cudaError_t launch_compare_keys(const uint8_t *records, size_t record_bytes, const uint32_t *perm,
                                uint64_t n, const CompareGroup &group, void *keys, int sm_count,
                                cudaStream_t s);

}  // namespace rsort
