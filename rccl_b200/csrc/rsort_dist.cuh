// Shared declarations of the sample-sort device steps.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "rsort_device.cuh"

namespace rsort {

// Composite sort position of one element: order image of the key, then
// (rank << POS_BITS | position in the rank's locally sorted shard).
struct Composite {
    uint64_t key;
    uint64_t pos;
};
constexpr int POS_BITS = 40;

// Largest sample set the one-CTA splitter kernel sorts (power of two; 16 bytes
// per composite in shared memory).
constexpr uint32_t MAX_SPLITTER_SAMPLES = 8192;

struct MergeArgs {
    const void *a_keys;
    const void *a_values;
    uint64_t na;
    const void *b_keys;
    const void *b_values;
    uint64_t nb;
    void *out_keys;
    void *out_values;
    int kind, desc;
};

cudaError_t launch_samples(int key_bytes, const void *keys, uint64_t m, uint32_t rank, uint32_t S,
                           KeyXform xf, Composite *out, cudaStream_t s);
cudaError_t launch_splitters(const Composite *samples, uint32_t total, uint32_t world,
                             Composite *splitters, cudaStream_t s);
cudaError_t launch_bounds(int key_bytes, const void *keys, uint64_t m, uint32_t rank,
                          const Composite *splitters, uint32_t world, KeyXform xf,
                          uint64_t *bounds, cudaStream_t s);
// Words of the merge-path partition array a merge of na + nb items needs.
size_t merge_partition_words(uint64_t na, uint64_t nb);
cudaError_t launch_merge(int key_bytes, int value_bytes, const MergeArgs &p, uint64_t *split,
                         cudaStream_t s);

// Several independent two-run merges in one launch (a round of a merge tree).
// Pair q's merge-path partitions take split_start[q + 1] - split_start[q]
// words (merge_partition_words of the pair) of the split array.
constexpr uint32_t MERGE_MAX_PAIRS = 32;
struct MergeBatch {
    MergeArgs pair[MERGE_MAX_PAIRS];
    uint64_t split_start[MERGE_MAX_PAIRS + 1];
    uint32_t npairs;
};
cudaError_t launch_merge_batch(int key_bytes, int value_bytes, const MergeBatch &b,
                               uint64_t *split, cudaStream_t s);

// Segment gather of the bucket exchange: segment q (src[q], a peer's or the
// local shard) lands at dst + dst_start[q]; unit_log2[q] is the copy width
// (log2 bytes, at most 4) that divides both addresses and the length.
constexpr int GATHER_MAX_SEGMENTS = 64;
struct GatherArgs {
    const char *src[GATHER_MAX_SEGMENTS];
    uint64_t dst_start[GATHER_MAX_SEGMENTS + 1];
    uint8_t unit_log2[GATHER_MAX_SEGMENTS];
    char *dst;
    uint32_t nseg;
};
cudaError_t launch_gather(const GatherArgs &a, int sm_count, cudaStream_t s);
// Base address of the device allocation that contains p.
cudaError_t allocation_base(const void *p, uintptr_t *base);

}  // namespace rsort
