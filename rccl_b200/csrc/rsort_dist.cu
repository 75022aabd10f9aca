// Device steps of the multi-GPU sample sort (no reference counterpart: the
// reference is single-GPU).  Every element is ordered by the composite
// (order image, rank, position in the rank's locally sorted shard), which is
// the global stable order because the input shards are contiguous slices.
//
//   samples    regular samples of the locally sorted shard
//   splitters  sort the world's samples (bitonic, one CTA) and pick W-1
//   bounds     lower bound of every splitter in the local shard
//   merge      stable merge-path merge of two sorted runs (ties: first run)
#include "rsort_device.cuh"
#include "rsort_dist.cuh"

namespace rsort {

template <typename B>
__device__ __forceinline__ uint64_t image_of(B raw, KeyXform xf) {
    return uint64_t(fold_zero(to_ordered(raw, xf), xf.kind));
}

// ---------------------------------------------------------------------------
// Regular samples: sample i sits at floor((i + 1) * m / (S + 1)).
// ---------------------------------------------------------------------------
template <typename B>
__global__ void samples_kernel(const B *keys, uint64_t m, uint32_t rank, uint32_t S,
                               KeyXform xf, Composite *out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S) return;
    if (m == 0) {
        out[i] = Composite{~0ull, ~0ull};
        return;
    }
    const uint64_t p = (uint64_t(i) + 1) * m / (uint64_t(S) + 1);
    out[i] = Composite{image_of(keys[p], xf), (uint64_t(rank) << POS_BITS) | p};
}

__device__ __forceinline__ bool comp_less(const Composite &a, const Composite &b) {
    return a.key < b.key || (a.key == b.key && a.pos < b.pos);
}

// ---------------------------------------------------------------------------
// Splitters: one CTA bitonic-sorts the padded sample set in shared memory;
// splitter j (1 <= j < W) is sample floor(j * valid / W).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) splitters_kernel(const Composite *samples, uint32_t total,
                                                         uint32_t world, Composite *splitters) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Composite *s = reinterpret_cast<Composite *>(smem_raw);
    __shared__ uint32_t valid;
    uint32_t np = 1;
    while (np < total) np <<= 1;
    if (threadIdx.x == 0) valid = 0;
    __syncthreads();
    uint32_t my_valid = 0;
    for (uint32_t i = threadIdx.x; i < np; i += blockDim.x) {
        const Composite c = i < total ? samples[i] : Composite{~0ull, ~0ull};
        s[i] = c;
        if (c.pos != ~0ull) ++my_valid;
    }
    atomicAdd(&valid, my_valid);
    __syncthreads();
    for (uint32_t k = 2; k <= np; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t i = threadIdx.x; i < np; i += blockDim.x) {
                const uint32_t partner = i ^ j;
                if (partner > i) {
                    const bool up = (i & k) == 0;
                    const Composite a = s[i], b = s[partner];
                    if (comp_less(b, a) == up) {
                        s[i] = b;
                        s[partner] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (uint32_t j = threadIdx.x + 1; j < world; j += blockDim.x) {
        splitters[j - 1] = valid ? s[uint64_t(j) * valid / world] : Composite{~0ull, ~0ull};
    }
}

// ---------------------------------------------------------------------------
// Bucket bounds: bounds[j] = #{ local i : (image_i, rank, i) < splitter_j }.
// ---------------------------------------------------------------------------
template <typename B>
__global__ void bounds_kernel(const B *keys, uint64_t m, uint32_t rank, const Composite *splitters,
                              uint32_t world, KeyXform xf, uint64_t *bounds) {
    const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j > world) return;
    if (j == 0) {
        bounds[0] = 0;
        return;
    }
    if (j == world) {
        bounds[world] = m;
        return;
    }
    const Composite sp = splitters[j - 1];
    uint64_t lo = 0, hi = m;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        const Composite c{image_of(keys[mid], xf), (uint64_t(rank) << POS_BITS) | mid};
        if (comp_less(c, sp))
            lo = mid + 1;
        else
            hi = mid;
    }
    bounds[j] = lo;
}

// ---------------------------------------------------------------------------
// Stable merge of two sorted runs A then B (ties take A first), merge-path
// partitioned: every CTA owns MERGE_TILE outputs, finds its A/B split with a
// binary search on the cross diagonal, stages both segments in shared memory,
// merges MERGE_ITEMS outputs per thread and writes the tile out coalesced.
// ---------------------------------------------------------------------------
#ifndef RSORT_MERGE_THREADS
#define RSORT_MERGE_THREADS 256
#endif
constexpr int MERGE_THREADS = RSORT_MERGE_THREADS;
// Odd, so the serial per-thread merges of neighbouring lanes (which start
// MERGE_ITEMS items apart in shared memory) fall into different banks.
#ifndef RSORT_MERGE_ITEMS
#define RSORT_MERGE_ITEMS 13
#endif
constexpr int MERGE_ITEMS = RSORT_MERGE_ITEMS;
constexpr int MERGE_TILE = MERGE_THREADS * MERGE_ITEMS;

template <typename B>
__device__ __forceinline__ uint64_t merge_path(const B *a, uint64_t na, const B *b, uint64_t nb,
                                               uint64_t diag, KeyXform xf) {
    uint64_t lo = diag > nb ? diag - nb : 0;
    uint64_t hi = diag < na ? diag : na;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        if (image_of(a[mid], xf) <= image_of(b[diag - 1 - mid], xf))
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// Merge-path partitions: split[i] = number of A items among the first
// i * MERGE_TILE outputs (one thread per tile boundary).
template <typename B>
__device__ __forceinline__ uint64_t merge_split(const MergeArgs &p, uint64_t i) {
    const uint64_t total = p.na + p.nb;
    const uint64_t diag = i * MERGE_TILE < total ? i * MERGE_TILE : total;
    return merge_path(static_cast<const B *>(p.a_keys), p.na, static_cast<const B *>(p.b_keys),
                      p.nb, diag, KeyXform{p.kind, p.desc});
}

template <typename B>
__global__ void merge_partition_kernel(MergeArgs p, uint64_t *split, uint64_t nsplit) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nsplit) return;
    split[i] = merge_split<B>(p, i);
}

// Partitions of every pair of a batch: pair q's words start at split_start[q].
template <typename B>
__global__ void merge_partition_batch_kernel(const __grid_constant__ MergeBatch b,
                                             uint64_t *split) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= b.split_start[b.npairs]) return;
    uint32_t q = 0;
    while (i >= b.split_start[q + 1]) ++q;
    split[i] = merge_split<B>(b.pair[q], i - b.split_start[q]);
}

template <typename B, int VB>
struct MergeSmem {
    static constexpr int VSIZE = VB > 0 ? VB : 1;
    static constexpr size_t KEYS = 0;                                  // A then B segment
    static constexpr size_t VALS = KEYS + size_t(MERGE_TILE) * sizeof(B);
    static constexpr size_t BYTES = VALS + (VB > 0 ? size_t(MERGE_TILE) * VSIZE : 0);
};

template <int VB> struct MergeValue;
template <> struct MergeValue<0> { using type = uint8_t; };
template <> struct MergeValue<1> { using type = uint8_t; };
template <> struct MergeValue<2> { using type = uint16_t; };
template <> struct MergeValue<4> { using type = uint32_t; };
template <> struct MergeValue<8> { using type = uint64_t; };
template <> struct MergeValue<16> { using type = uint4; };

// One CTA per MERGE_TILE outputs: stage the A and B segments given by the
// precomputed partitions, let every thread merge MERGE_ITEMS outputs from its
// own merge-path split, gather through shared memory and write the tile out
// coalesced.
template <typename B, int VB>
__device__ __forceinline__ void merge_tile(const MergeArgs &p, const uint64_t *split,
                                           uint64_t tile) {
    using S = MergeSmem<B, VB>;
    using VT = typename MergeValue<VB>::type;
    extern __shared__ __align__(16) uint8_t smem[];
    B *sk = reinterpret_cast<B *>(smem + S::KEYS);
    VT *sv = reinterpret_cast<VT *>(smem + S::VALS);
    const KeyXform xf{p.kind, p.desc};
    const B *ak = static_cast<const B *>(p.a_keys);
    const B *bk = static_cast<const B *>(p.b_keys);
    const VT *av = static_cast<const VT *>(p.a_values);
    const VT *bv = static_cast<const VT *>(p.b_values);
    const uint64_t total = p.na + p.nb;
    const uint64_t d0 = tile * MERGE_TILE;
    const uint64_t d1 = d0 + MERGE_TILE < total ? d0 + MERGE_TILE : total;
    const uint64_t a0 = split[tile], a1 = split[tile + 1];
    const uint64_t b0 = d0 - a0, b1 = d1 - a1;
    const uint32_t la = uint32_t(a1 - a0), lb = uint32_t(b1 - b0);
    const uint32_t n = la + lb;
    {
        // Every load of the thread is issued before the first shared store,
        // so MERGE_ITEMS keys (and values) per thread are in flight at once:
        // the runs may be a peer's memory, microseconds away over NVLink.
        B kreg[MERGE_ITEMS];
        VT vreg[VB > 0 ? MERGE_ITEMS : 1];
#pragma unroll
        for (int k = 0; k < MERGE_ITEMS; ++k) {
            const uint32_t i = threadIdx.x + uint32_t(k) * MERGE_THREADS;
            if (i < n) {
                const bool in_a = i < la;
                kreg[k] = in_a ? ak[a0 + i] : bk[b0 + i - la];
                if constexpr (VB > 0) vreg[k] = in_a ? av[a0 + i] : bv[b0 + i - la];
            }
        }
#pragma unroll
        for (int k = 0; k < MERGE_ITEMS; ++k) {
            const uint32_t i = threadIdx.x + uint32_t(k) * MERGE_THREADS;
            if (i < n) {
                sk[i] = kreg[k];
                if constexpr (VB > 0) sv[i] = vreg[k];
            }
        }
    }
    __syncthreads();
    const B *ta = sk;
    const B *tb = sk + la;
    const uint32_t diag = min(uint32_t(threadIdx.x) * MERGE_ITEMS, n);
    uint32_t lo = diag > lb ? diag - lb : 0, hi = diag < la ? diag : la;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (image_of(ta[mid], xf) <= image_of(tb[diag - 1 - mid], xf))
            lo = mid + 1;
        else
            hi = mid;
    }
    uint32_t ia = lo, ib = diag - lo;
    B ok[MERGE_ITEMS];
    VT ov[VB > 0 ? MERGE_ITEMS : 1];
    uint64_t ima = ia < la ? image_of(ta[ia], xf) : 0;
    uint64_t imb = ib < lb ? image_of(tb[ib], xf) : 0;
#pragma unroll
    for (int k = 0; k < MERGE_ITEMS; ++k) {
        const bool take_a = ib >= lb || (ia < la && ima <= imb);
        const uint32_t src = take_a ? ia : la + ib;
        if (diag + k < n) {
            ok[k] = sk[src];
            if constexpr (VB > 0) ov[k] = sv[src];
        }
        if (take_a) {
            ++ia;
            if (ia < la) ima = image_of(ta[ia], xf);
        } else {
            ++ib;
            if (ib < lb) imb = image_of(tb[ib], xf);
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < MERGE_ITEMS; ++k) {
        if (diag + k < n) {
            sk[diag + k] = ok[k];
            if constexpr (VB > 0) sv[diag + k] = ov[k];
        }
    }
    __syncthreads();
    B *outk = static_cast<B *>(p.out_keys) + d0;
    VT *outv = static_cast<VT *>(p.out_values) + d0;
    for (uint32_t i = threadIdx.x; i < n; i += MERGE_THREADS) {
        outk[i] = sk[i];
        if constexpr (VB > 0) outv[i] = sv[i];
    }
}

template <typename B, int VB>
__global__ void __launch_bounds__(MERGE_THREADS) merge_kernel(MergeArgs p, const uint64_t *split) {
    merge_tile<B, VB>(p, split, blockIdx.x);
}

// All pairs of a batch in one launch.  Block k merges tile k / npairs of pair
// k % npairs, so every pair (and every peer a pair reads) progresses at once.
template <typename B, int VB>
__global__ void __launch_bounds__(MERGE_THREADS)
    merge_batch_kernel(const __grid_constant__ MergeBatch b, const uint64_t *split) {
    const uint32_t q = blockIdx.x % b.npairs;
    const uint64_t t = blockIdx.x / b.npairs;
    const uint64_t tiles = b.split_start[q + 1] - b.split_start[q] - 1;
    if (t >= tiles) return;
    merge_tile<B, VB>(b.pair[q], split + b.split_start[q], t);
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
namespace {

template <typename B, int VB>
cudaError_t merge_t(const MergeArgs &p, uint64_t *split, cudaStream_t s) {
    using S = MergeSmem<B, VB>;
    const uint64_t total = p.na + p.nb;
    if (total == 0) return cudaSuccess;
    const uint64_t blocks = (total + MERGE_TILE - 1) / MERGE_TILE;
    const uint64_t nsplit = blocks + 1;
    merge_partition_kernel<B><<<dim3(uint32_t((nsplit + 255) / 256)), 256, 0, s>>>(p, split, nsplit);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto k = merge_kernel<B, VB>;
    if (S::BYTES > 32 * 1024) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::BYTES));
        if (e != cudaSuccess) return e;
    }
    k<<<dim3(uint32_t(blocks)), MERGE_THREADS, S::BYTES, s>>>(p, split);
    return cudaGetLastError();
}

template <typename B, int VB>
cudaError_t merge_batch_t(const MergeBatch &b, uint64_t *split, cudaStream_t s) {
    using S = MergeSmem<B, VB>;
    const uint64_t words = b.split_start[b.npairs];
    uint64_t max_tiles = 0;
    for (uint32_t q = 0; q < b.npairs; ++q) {
        const uint64_t t = b.split_start[q + 1] - b.split_start[q] - 1;
        max_tiles = t > max_tiles ? t : max_tiles;
    }
    if (max_tiles == 0) return cudaSuccess;
    merge_partition_batch_kernel<B><<<dim3(uint32_t((words + 255) / 256)), 256, 0, s>>>(b, split);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    auto k = merge_batch_kernel<B, VB>;
    if (S::BYTES > 32 * 1024) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::BYTES));
        if (e != cudaSuccess) return e;
    }
    k<<<dim3(uint32_t(max_tiles * b.npairs)), MERGE_THREADS, S::BYTES, s>>>(b, split);
    return cudaGetLastError();
}

template <typename B>
cudaError_t merge_batch_vb(int vb, const MergeBatch &b, uint64_t *split, cudaStream_t s) {
    switch (vb) {
        case 0: return merge_batch_t<B, 0>(b, split, s);
        case 1: return merge_batch_t<B, 1>(b, split, s);
        case 2: return merge_batch_t<B, 2>(b, split, s);
        case 4: return merge_batch_t<B, 4>(b, split, s);
        case 8: return merge_batch_t<B, 8>(b, split, s);
        case 16: return merge_batch_t<B, 16>(b, split, s);
        default: return cudaErrorInvalidValue;
    }
}

template <typename B>
cudaError_t merge_vb(int vb, const MergeArgs &p, uint64_t *split, cudaStream_t s) {
    switch (vb) {
        case 0: return merge_t<B, 0>(p, split, s);
        case 1: return merge_t<B, 1>(p, split, s);
        case 2: return merge_t<B, 2>(p, split, s);
        case 4: return merge_t<B, 4>(p, split, s);
        case 8: return merge_t<B, 8>(p, split, s);
        case 16: return merge_t<B, 16>(p, split, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_samples(int key_bytes, const void *keys, uint64_t m, uint32_t rank, uint32_t S,
                           KeyXform xf, Composite *out, cudaStream_t s) {
    const uint32_t blocks = (S + 255) / 256;
    if (blocks == 0) return cudaSuccess;
    if (key_bytes == 4)
        samples_kernel<uint32_t><<<blocks, 256, 0, s>>>(static_cast<const uint32_t *>(keys), m,
                                                       rank, S, xf, out);
    else
        samples_kernel<uint64_t><<<blocks, 256, 0, s>>>(static_cast<const uint64_t *>(keys), m,
                                                       rank, S, xf, out);
    return cudaGetLastError();
}

cudaError_t launch_splitters(const Composite *samples, uint32_t total, uint32_t world,
                             Composite *splitters, cudaStream_t s) {
    uint32_t np = 1;
    while (np < total) np <<= 1;
    const size_t bytes = size_t(np) * sizeof(Composite);
    if (bytes > 32 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(splitters_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
        if (e != cudaSuccess) return e;
    }
    splitters_kernel<<<1, 1024, bytes, s>>>(samples, total, world, splitters);
    return cudaGetLastError();
}

cudaError_t launch_bounds(int key_bytes, const void *keys, uint64_t m, uint32_t rank,
                          const Composite *splitters, uint32_t world, KeyXform xf,
                          uint64_t *bounds, cudaStream_t s) {
    const uint32_t blocks = (world + 1 + 63) / 64;
    if (key_bytes == 4)
        bounds_kernel<uint32_t><<<blocks, 64, 0, s>>>(static_cast<const uint32_t *>(keys), m, rank,
                                                     splitters, world, xf, bounds);
    else
        bounds_kernel<uint64_t><<<blocks, 64, 0, s>>>(static_cast<const uint64_t *>(keys), m, rank,
                                                     splitters, world, xf, bounds);
    return cudaGetLastError();
}

size_t merge_partition_words(uint64_t na, uint64_t nb) {
    return size_t((na + nb + MERGE_TILE - 1) / MERGE_TILE + 1);
}

cudaError_t launch_merge(int key_bytes, int value_bytes, const MergeArgs &p, uint64_t *split,
                         cudaStream_t s) {
    return key_bytes == 4 ? merge_vb<uint32_t>(value_bytes, p, split, s)
                          : merge_vb<uint64_t>(value_bytes, p, split, s);
}

cudaError_t launch_merge_batch(int key_bytes, int value_bytes, const MergeBatch &b,
                               uint64_t *split, cudaStream_t s) {
    if (b.npairs == 0) return cudaSuccess;
    return key_bytes == 4 ? merge_batch_vb<uint32_t>(value_bytes, b, split, s)
                          : merge_batch_vb<uint64_t>(value_bytes, b, split, s);
}

}  // namespace rsort
