// Gathers of the lexicographic record sort (rccl-thrust/src/record_sort.rs
// semantics: stable ascending order of padding-free [u32; N] rows, word 0
// most significant, payloads in lockstep).  The sort itself is multi-word
// LSD over the stable pairs radix sort; these kernels build each pass's
// 64-bit chunk keys through the current permutation and apply the final
// permutation to the rows and payloads.
#include <cstdint>

#include <cuda_runtime.h>

#include "rsort_records.cuh"

namespace rsort {

namespace {

constexpr int GATHER_BLOCK = 256;

// keys[i] = words [first, first + count) of row perm[i], big-endian within
// the 64-bit key (count is 1 or 2); perm == nullptr means the identity.
__global__ void __launch_bounds__(GATHER_BLOCK)
    chunk_keys_kernel(const uint32_t *rows, uint32_t words, const uint32_t *perm, uint64_t n,
                      uint32_t first, uint32_t count, uint64_t *keys) {
    const uint64_t stride = uint64_t(gridDim.x) * GATHER_BLOCK;
    for (uint64_t i = uint64_t(blockIdx.x) * GATHER_BLOCK + threadIdx.x; i < n; i += stride) {
        const uint64_t r = perm ? perm[i] : i;
        const uint32_t *row = rows + r * words + first;
        keys[i] = count == 2 ? (uint64_t(row[0]) << 32) | row[1] : uint64_t(row[0]);
    }
}

__global__ void __launch_bounds__(GATHER_BLOCK) iota_kernel(uint32_t *perm, uint64_t n) {
    const uint64_t stride = uint64_t(gridDim.x) * GATHER_BLOCK;
    for (uint64_t i = uint64_t(blockIdx.x) * GATHER_BLOCK + threadIdx.x; i < n; i += stride)
        perm[i] = uint32_t(i);
}

// dst item i = src item perm[i], items of `unit` bytes (1, 2, 4 or 8) times
// `units` per item.
template <typename U>
__global__ void __launch_bounds__(GATHER_BLOCK)
    permute_kernel(const U *src, const uint32_t *perm, uint64_t n, uint32_t units, U *dst) {
    const uint64_t total = n * units;
    const uint64_t stride = uint64_t(gridDim.x) * GATHER_BLOCK;
    for (uint64_t k = uint64_t(blockIdx.x) * GATHER_BLOCK + threadIdx.x; k < total; k += stride) {
        const uint64_t i = k / units, u = k - i * units;
        dst[k] = src[uint64_t(perm[i]) * units + u];
    }
}

unsigned grid_for(uint64_t items, int sm_count) {
    const uint64_t want = (items + GATHER_BLOCK - 1) / GATHER_BLOCK;
    const uint64_t cap = uint64_t(sm_count) * 8;
    return unsigned(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

cudaError_t launch_chunk_keys(const uint32_t *rows, uint32_t words, const uint32_t *perm,
                              uint64_t n, uint32_t first, uint32_t count, uint64_t *keys,
                              int sm_count, cudaStream_t s) {
    chunk_keys_kernel<<<grid_for(n, sm_count), GATHER_BLOCK, 0, s>>>(rows, words, perm, n, first,
                                                                     count, keys);
    return cudaGetLastError();
}

cudaError_t launch_iota(uint32_t *perm, uint64_t n, int sm_count, cudaStream_t s) {
    iota_kernel<<<grid_for(n, sm_count), GATHER_BLOCK, 0, s>>>(perm, n);
    return cudaGetLastError();
}

cudaError_t launch_permute(const void *src, const uint32_t *perm, uint64_t n, size_t item_bytes,
                           void *dst, int sm_count, cudaStream_t s) {
    // The copy unit must divide the item width and both base addresses: a
    // 4-byte aligned row array must not be moved with 8-byte accesses.
    const uint64_t align = uint64_t(item_bytes) | uint64_t(reinterpret_cast<uintptr_t>(src)) |
                           uint64_t(reinterpret_cast<uintptr_t>(dst));
    int lg = 3;
    while (lg > 0 && align % (uint64_t(1) << lg) != 0) --lg;
    const uint32_t units = uint32_t(item_bytes >> lg);
    const unsigned grid = grid_for(n * units, sm_count);
    switch (lg) {
        case 3:
            permute_kernel<uint64_t><<<grid, GATHER_BLOCK, 0, s>>>(
                static_cast<const uint64_t *>(src), perm, n, units, static_cast<uint64_t *>(dst));
            break;
        case 2:
            permute_kernel<uint32_t><<<grid, GATHER_BLOCK, 0, s>>>(
                static_cast<const uint32_t *>(src), perm, n, units, static_cast<uint32_t *>(dst));
            break;
        case 1:
            permute_kernel<uint16_t><<<grid, GATHER_BLOCK, 0, s>>>(
                static_cast<const uint16_t *>(src), perm, n, units, static_cast<uint16_t *>(dst));
            break;
        default:
            permute_kernel<uint8_t><<<grid, GATHER_BLOCK, 0, s>>>(
                static_cast<const uint8_t *>(src), perm, n, units, static_cast<uint8_t *>(dst));
            break;
    }
    return cudaGetLastError();
}

}  // namespace rsort
