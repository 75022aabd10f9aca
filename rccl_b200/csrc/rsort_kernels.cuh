// Kernel argument blocks, tile shapes and launch entry points shared by the
// kernel translation unit and the host pass control.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace rsort {

// Tile shape of the onesweep pass for a (key bytes, value bytes) pair.  The
// shapes are B200 choices (148 SMs, 228 KB shared memory per SM, two resident
// 512-thread CTAs per SM), not the reference's Policy800 constants; only the
// single-tile routing threshold keeps Policy800's value because it decides an
// observable DoubleBuffer selector outcome.
#ifndef RSORT_ONESWEEP_THREADS
#define RSORT_ONESWEEP_THREADS 512
#endif
constexpr int ONESWEEP_THREADS = RSORT_ONESWEEP_THREADS;

// Items per thread, tuned on B200 (bigger tiles shorten the look-back chain;
// beyond these the 64-register budget spills).
#ifndef RSORT_ITEMS_KEYS32
#define RSORT_ITEMS_KEYS32 24
#endif
#ifndef RSORT_ITEMS_KEYS64
#define RSORT_ITEMS_KEYS64 15
#endif
#ifndef RSORT_ITEMS_PAIRS64_32
#define RSORT_ITEMS_PAIRS64_32 12
#endif
#ifndef RSORT_ITEMS_PAIRS32_32
#define RSORT_ITEMS_PAIRS32_32 16
#endif
// 1- and 2-byte keys take the 4-byte shapes (a key occupies one register
// either way).
constexpr int onesweep_items(int key_bytes_, int value_bytes) {
    const int key_bytes = key_bytes_ < 4 ? 4 : key_bytes_;
    return (value_bytes == 0 && key_bytes == 4) ? RSORT_ITEMS_KEYS32
         : (value_bytes == 0 && key_bytes == 8) ? RSORT_ITEMS_KEYS64
         : (value_bytes == 4 && key_bytes == 8) ? RSORT_ITEMS_PAIRS64_32
         : (value_bytes == 4 && key_bytes == 4) ? RSORT_ITEMS_PAIRS32_32
         : value_bytes == 0 ? (key_bytes == 4 ? 16 : 8)
         : value_bytes == 16 ? (key_bytes == 4 ? 6 : 4)
         : key_bytes == 4 ? (value_bytes <= 4 ? 12 : 8)
         : value_bytes == 8 ? 7
         : 8;
}

constexpr int onesweep_tile(int key_bytes, int value_bytes) {
    return ONESWEEP_THREADS * onesweep_items(key_bytes, value_bytes);
}

// Policy800 single-tile extent (rccl-cub/src/workspace.rs:23-66):
// 256 threads * max(1, 19*4 / max(item_size, 4)) items, where item_size is
// the key size for keys-only and max(key, value) size for pairs.
constexpr size_t policy800_single_tile_items(int key_bytes, int value_bytes) {
    const int item = key_bytes > value_bytes ? key_bytes : value_bytes;
    const int divisor = item > 4 ? item : 4;
    const int items = 19 * 4 / divisor;
    return 256u * size_t(items < 1 ? 1 : items);
}

constexpr int SINGLE_THREADS = 512;

// Counters region layout (int32 words).
constexpr int CTR_TILE = 0;     // [0, 8): dynamic tile counter of each pass
constexpr int CTR_HIST_DONE = 8;
constexpr int CTR_STATUS = 9;
constexpr int CTR_HOT_FLAGS = 10;  // bit p: pass p is hot (HOT_SHARE), from the histogram
constexpr int CTR_WORDS = 16;

struct HistArgs {
    const void *keys;
    uint64_t n;
    uint64_t *bins;       // passes * 256
    uint64_t *lookback;   // zeroed here
    uint64_t lookback_words;
    int *done;
    uint32_t passes;
    uint32_t begin_bit, end_bit;
    int kind, desc;
    int vector_ok;  // keys pointer is 16-byte aligned
    int *hot;       // counters + CTR_HOT_FLAGS, or nullptr
};

struct PassArgs {
    const void *keys_in;
    void *keys_out;
    const void *values_in;
    void *values_out;
    uint64_t n;
    const uint64_t *bins;  // this pass's 256 global digit starts
    uint64_t *lookback;
    int *tile_counter;
    int *status;
    uint32_t shift, mask;
    int kind, desc;
    int first, last;  // apply the raw->ordered / ordered->raw transform
    uint32_t tag;
    const int *hot;    // counters + CTR_HOT_FLAGS (RANK_RUNS kernel only), or nullptr
    uint32_t pass;     // index of this pass within the sort
};

struct SingleArgs {
    const void *keys_in;
    void *keys_out;
    const void *values_in;
    void *values_out;
    uint32_t n;
    uint32_t begin_bit, end_bit;
    int kind, desc;
    // Segmented sort: when seg_ids is set, seg_count CTAs run and CTA b
    // sorts segment s = seg_ids[b], items [seg_begin[s], seg_end[s]) of the
    // arrays above (at most the single-tile extent); n is unused.
    const uint64_t *seg_begin = nullptr;
    const uint64_t *seg_end = nullptr;
    const uint32_t *seg_ids = nullptr;
    uint32_t seg_count = 0;
};

// Host-side launchers (defined in rsort_kernels.cu).  Each returns the CUDA
// error of the launch.
cudaError_t launch_init(uint64_t *bins, size_t nbins, int *counters, size_t ncounters,
                        cudaStream_t stream);
cudaError_t launch_histogram(int key_bytes, const HistArgs &a, int sm_count, cudaStream_t stream);
cudaError_t launch_onesweep(int key_bytes, int value_bytes, const PassArgs &a, uint64_t tiles,
                            cudaStream_t stream);
// Sorts shorter than this skip the RANK_RUNS form: its launch, which exits
// at once on passes without runs, would cost a measurable share of a small
// sort (2^20 u32 keys: 0.106 -> 0.14 ms on B200).
constexpr uint64_t RUNS_MIN_ITEMS = uint64_t(1) << 25;
// The RANK_RUNS form of the pass (4- and 8-byte keys; a persistent grid):
// it sorts the pass when the histogram marked this pass and the one before
// hot, and otherwise exits without claiming a tile.  Launched just before
// launch_onesweep, whose tile claims then find the pass done.
cudaError_t launch_onesweep_runs(int key_bytes, int value_bytes, const PassArgs &a,
                                 uint64_t tiles, cudaStream_t stream);
cudaError_t launch_single_tile(int key_bytes, int value_bytes, const SingleArgs &a,
                               cudaStream_t stream);

}  // namespace rsort
