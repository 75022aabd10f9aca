// Bucket exchange of the multi-GPU sample sort over NVLink peer memory (no
// reference counterpart: the reference is single-GPU).
//
// Each rank exports its sorted shard (keys, values) with CUDA IPC and every
// peer maps it once.  The default exchange then merges the buckets straight
// out of the peers' shards (rsort_merge_segments); the "peer-copy" exchange
// instead PULLS every bucket with rsort_gather_segments, the SM-driven copy
// kernel below reading the peers' HBM over NVLink / NVSwitch, all peers at
// the same time, with no staging buffers or proxy copies.  Also here: the
// allocation-base lookup that CUDA IPC export needs.
//
// The kernel waits on nothing: the caller orders it after the peers' sorts
// (a collective that every rank enters after its own sort) and orders the
// peers' next writes of their shards after it (a collective after the copy).
#include <cstdint>
#include <cstring>

#include <cuda.h>
#include <cuda_runtime.h>

#include "rsort_dist.cuh"

namespace rsort {

namespace {

constexpr int GATHER_THREADS = 512;
constexpr int GATHER_UNROLL = 4;

// Copies n units of type U, threads of `groups` CTAs interleaved.
template <typename U>
__device__ __forceinline__ void copy_units(const char *src, char *dst, uint64_t n, uint64_t first,
                                           uint64_t stride) {
    const U *s = reinterpret_cast<const U *>(src);
    U *d = reinterpret_cast<U *>(dst);
    for (uint64_t i = first; i < n; i += stride * GATHER_UNROLL) {
        U v[GATHER_UNROLL];
#pragma unroll
        for (int k = 0; k < GATHER_UNROLL; ++k) {
            const uint64_t idx = i + uint64_t(k) * stride;
            if (idx < n) v[k] = s[idx];
        }
#pragma unroll
        for (int k = 0; k < GATHER_UNROLL; ++k) {
            const uint64_t idx = i + uint64_t(k) * stride;
            if (idx < n) d[idx] = v[k];
        }
    }
}

// CTA b copies segment b % nseg together with the other CTAs of that
// segment, so all segments (peers) are read concurrently.
__global__ void __launch_bounds__(GATHER_THREADS) gather_kernel(GatherArgs a) {
    const uint32_t q = blockIdx.x % a.nseg;
    const uint32_t g = blockIdx.x / a.nseg;
    const uint32_t groups = gridDim.x / a.nseg;
    const uint64_t bytes = a.dst_start[q + 1] - a.dst_start[q];
    if (bytes == 0) return;
    const char *src = a.src[q];
    char *dst = a.dst + a.dst_start[q];
    const int lg = a.unit_log2[q];
    const uint64_t n = bytes >> lg;
    const uint64_t first = uint64_t(g) * GATHER_THREADS + threadIdx.x;
    const uint64_t stride = uint64_t(groups) * GATHER_THREADS;
    switch (lg) {
        case 4: copy_units<uint4>(src, dst, n, first, stride); break;
        case 3: copy_units<uint2>(src, dst, n, first, stride); break;
        case 2: copy_units<uint32_t>(src, dst, n, first, stride); break;
        case 1: copy_units<uint16_t>(src, dst, n, first, stride); break;
        default: copy_units<uint8_t>(src, dst, n, first, stride); break;
    }
}

}  // namespace

cudaError_t launch_gather(const GatherArgs &a, int sm_count, cudaStream_t s) {
    if (a.nseg == 0) return cudaSuccess;
    // About two CTAs per SM in total, the same number for every segment.
    uint32_t groups = uint32_t((2 * sm_count + int(a.nseg) - 1) / int(a.nseg));
    if (groups == 0) groups = 1;
    gather_kernel<<<groups * a.nseg, GATHER_THREADS, 0, s>>>(a);
    return cudaGetLastError();
}

// Allocation base of a device pointer, through the driver entry point (the
// library does not link the driver library itself).
cudaError_t allocation_base(const void *p, uintptr_t *base) {
    using Fn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
    static Fn fn = nullptr;
    if (!fn) {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || !f) return cudaErrorNotSupported;
        fn = reinterpret_cast<Fn>(f);
    }
    CUdeviceptr b = 0;
    size_t size = 0;
    if (fn(&b, &size, CUdeviceptr(reinterpret_cast<uintptr_t>(p))) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    *base = uintptr_t(b);
    return cudaSuccess;
}

}  // namespace rsort
