// Gathers of the lexicographic record sort (rccl-thrust/src/record_sort.rs
// semantics: stable ascending order of padding-free [u32; N] rows, word 0
// most significant, payloads in lockstep).  The sort itself is multi-word
// LSD over the stable pairs radix sort; these kernels build each pass's
// 64-bit chunk keys through the current permutation and apply the final
// permutation to the rows and payloads.  The comparator-program sort
// (rsort_sort_by) uses the same scheme with keys packed from its terms'
// projected fields (compare_keys_kernel).
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/rsort_b200.h"
#include "rsort_device.cuh"
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

// Order image of one projected field (the radix order of the projected
// value: unsigned as is, signed with the sign bit flipped, floats sign-
// magnitude to unsigned with -0.0 folded onto +0.0 unless the order is
// total), complemented for a descending term.
template <typename U>
__device__ __forceinline__ uint64_t term_image(U v, const CompareTerm &t) {
    using S = typename KeyBits<U>::Signed;
    constexpr U SIGN = KeyBits<U>::SIGN;
    constexpr int W = KeyBits<U>::WIDTH;
    if (t.kind == KIND_SINT) {
        S x = S(v);
        const S op = S(t.operand);
        switch (t.projection) {
            case RSORT_PROJ_AND: x = S(U(x) & U(op)); break;
            case RSORT_PROJ_SHR: x = S(x >> int(t.operand)); break;
            case RSORT_PROJ_DIV: x = S(x / op); break;
            case RSORT_PROJ_REM: x = S(x % op); break;
            default: break;
        }
        v = U(U(x) ^ SIGN);
    } else if (t.kind == KIND_UINT) {
        const U op = U(t.operand);
        switch (t.projection) {
            case RSORT_PROJ_AND: v = U(v & op); break;
            case RSORT_PROJ_SHR: v = U(v >> int(t.operand)); break;
            case RSORT_PROJ_DIV: v = U(v / op); break;
            case RSORT_PROJ_REM: v = U(v % op); break;
            default: break;
        }
    } else {
        v = U(v ^ (U(S(v) >> (W - 1)) | SIGN));
        if (t.kind == KIND_FLOAT && v == U(SIGN - 1)) v = SIGN;
    }
    if (t.desc) v = U(~v);
    return uint64_t(v);
}

template <typename U>
__device__ __forceinline__ U load_field(const uint8_t *p, bool aligned) {
    if (aligned) return *reinterpret_cast<const U *>(p);
    U v = 0;
#pragma unroll
    for (int b = 0; b < int(sizeof(U)); ++b) v |= U(U(p[b]) << (8 * b));
    return v;
}

__device__ __forceinline__ uint64_t term_bits(const uint8_t *rec, const CompareTerm &t) {
    const uint8_t *p = rec + t.offset;
    const bool al = t.aligned != 0;
    uint64_t img;
    switch (t.bytes) {
        case 1: img = term_image<uint8_t>(p[0], t); break;
        case 2: img = term_image<uint16_t>(load_field<uint16_t>(p, al), t); break;
        case 4: img = term_image<uint32_t>(load_field<uint32_t>(p, al), t); break;
        default: img = term_image<uint64_t>(load_field<uint64_t>(p, al), t); break;
    }
    const uint64_t mask = t.width >= 64 ? ~uint64_t(0) : (uint64_t(1) << t.width) - 1;
    return (img >> t.lo) & mask;
}

template <typename K>
__global__ void __launch_bounds__(GATHER_BLOCK)
    compare_keys_kernel(const uint8_t *records, uint64_t record_bytes, const uint32_t *perm,
                        uint64_t n, const __grid_constant__ CompareGroup g, K *keys) {
    const uint64_t stride = uint64_t(gridDim.x) * GATHER_BLOCK;
    for (uint64_t i = uint64_t(blockIdx.x) * GATHER_BLOCK + threadIdx.x; i < n; i += stride) {
        const uint64_t r = perm ? perm[i] : i;
        const uint8_t *rec = records + r * record_bytes;
        uint64_t key = 0;
        for (uint32_t k = 0; k < g.nterms; ++k) {
            const CompareTerm &t = g.term[k];
            // width 64 only when the group is this one term
            key = (t.width >= 64 ? 0 : key << t.width) | term_bits(rec, t);
        }
        keys[i] = K(key);
    }
}

}  // namespace

cudaError_t launch_compare_keys(const uint8_t *records, size_t record_bytes, const uint32_t *perm,
                                uint64_t n, const CompareGroup &group, void *keys, int sm_count,
                                cudaStream_t s) {
    if (group.total_bits <= 32)
        compare_keys_kernel<uint32_t><<<grid_for(n, sm_count), GATHER_BLOCK, 0, s>>>(
            records, record_bytes, perm, n, group, static_cast<uint32_t *>(keys));
    else
        compare_keys_kernel<uint64_t><<<grid_for(n, sm_count), GATHER_BLOCK, 0, s>>>(
            records, record_bytes, perm, n, group, static_cast<uint64_t *>(keys));
    return cudaGetLastError();
}

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
