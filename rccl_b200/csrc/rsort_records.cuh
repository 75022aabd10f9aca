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

}  // namespace rsort
