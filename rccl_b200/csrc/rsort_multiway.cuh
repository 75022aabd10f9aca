// Shared declarations of the single-pass W-way merge (rsort_multiway.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace rsort {

constexpr int MW_MAX_RUNS = 64;
#ifndef RSORT_MW_THREADS
#define RSORT_MW_THREADS 512
#endif
constexpr int MW_THREADS = RSORT_MW_THREADS;

// Outputs per thread and merge round; the CTA's capacity is MW_THREADS times
// this.  Odd, so the serial merges of neighbouring threads (which start this
// many items apart in shared memory) fall into different banks; smaller for
// wide items so two buffers still fit in shared memory.
#ifndef RSORT_MW_ITEMS
#define RSORT_MW_ITEMS 9
#endif
constexpr int mw_items(int key_bytes, int value_bytes) {
    return key_bytes + value_bytes <= 12 ? RSORT_MW_ITEMS : (RSORT_MW_ITEMS + 1) / 2;
}

struct MultiwayArgs {
    const void *keys[MW_MAX_RUNS];
    const void *values[MW_MAX_RUNS];
    uint64_t len[MW_MAX_RUNS];
    uint64_t pivot_start[MW_MAX_RUNS + 1];  // prefix sums of the runs' pivot counts
    uint32_t runs;
    uint32_t stride;  // S: a run contributes a pivot every S items
    uint32_t group;   // G: pivot intervals per CTA
    uint64_t pivots;  // P
    uint64_t *table;  // (P + 1) rows of `runs` counts
    void *out_keys;
    void *out_values;
    int kind, desc;
};

cudaError_t launch_multiway(int key_bytes, int value_bytes, MultiwayArgs &a, cudaStream_t s);

}  // namespace rsort
