/*
 * CPU restatement of the reference DeviceRadixSort ordering rules.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * product path: only the test suite, the smoke check and the benchmark's CPU
 * baseline leg load it.  The product library (librsort_b200.so) never links
 * or calls it.
 *
 * Parity is pinned against the reference's own golden vectors (the probes in
 * rccl-cub/examples/device_radix_sort_*_probe.rs and
 * rccl-thrust/examples/sort.rs, transcribed into tests/golden/ and
 * tests/test_oracle.py).  The reference itself (Rust + cuda-oxide, sm_80..89
 * only) cannot be built in this environment.
 *
 * Reference files restated here (paths inside the reference project):
 *   rccl-cub/src/ordering_backend/radix.rs:73-337   bit transforms, zero fold, digits
 *   rccl-cub/src/ordering_kernels.rs:677-702        which transform each route uses
 *   rccl-cub/src/ordering_backend/radix.rs:366-505  single-tile rank (6-bit, reversed lanes)
 *   rccl-cub/src/radix.rs:364-554, 625-778         pass control, selector, bit windows
 *   rccl-cub/src/workspace.rs:23-66                 Policy800 single-tile threshold
 */
#ifndef RSORT_ORACLE_H
#define RSORT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Key type codes; identical to rsort_key_t in include/rsort_b200.h. */
enum { ORC_U32 = 0, ORC_I32 = 1, ORC_F32 = 2, ORC_U64 = 3, ORC_I64 = 4, ORC_F64 = 5 };

/* Status codes; identical to rsort_status in include/rsort_b200.h. */
enum { ORC_OK = 0, ORC_INVALID_BIT_RANGE = 1, ORC_BAD_ARGUMENT = 8 };

unsigned orc_key_bytes(int key_type);
unsigned orc_key_bits(int key_type);

/* Order-preserving transform of the raw key bits (zero-extended to 64 bits).
 * radix.rs:73-235. */
uint64_t orc_to_ordered(int key_type, int descending, uint64_t raw);
uint64_t orc_from_ordered(int key_type, int descending, uint64_t ordered);

/* The float digit functions first fold the ordered image of -0.0 (ascending)
 * onto +0.0 so that both zeros are equal radix keys.  radix.rs:257-337. */
uint64_t orc_fold(int key_type, uint64_t ordered);

/* Policy800 single-tile extent (workspace.rs:23-66): 256 * items with
 * items = max(1, 19*4 / max(item_size, 4)), item_size = key bytes for
 * keys-only, max(key, value) bytes for pairs. */
size_t orc_single_tile_items(unsigned key_bytes, unsigned value_bytes);

/* The 64-bit sort key the reference's pass schedule orders by, for a call
 * with n items.  The sort is a stable ascending sort by this key. */
uint64_t orc_sort_key(int key_type, int descending, unsigned begin_bit, unsigned end_bit,
                      int single_tile_route, uint64_t raw);

/* Sort host arrays in place with the reference's observable semantics.
 *   keys:   n keys of orc_key_bytes(key_type) bytes
 *   values: n values of value_bytes bytes (value_bytes 0 = keys only)
 *   swaps:  out, number of DoubleBuffer selector flips the reference performs
 *           (0 no-op, 1 single-tile route, ceil((end-begin)/8) onesweep)
 *   threads: host threads to use (>= 1)
 * Returns ORC_OK or ORC_INVALID_BIT_RANGE (arrays unchanged). */
int orc_radix_sort(int key_type, int descending, void *keys, void *values, size_t n,
                   unsigned value_bytes, unsigned begin_bit, unsigned end_bit, int threads,
                   int *swaps);

/* Stable ascending sort of (sort_key, payload index): writes the permutation
 * perm[i] = input index of the i-th output.  Exposed for the sample-sort
 * restatement. */
void orc_stable_order(const uint64_t *sort_keys, size_t n, unsigned key_bits, int threads,
                      uint64_t *perm);

/* Restatement of the multi-GPU sample-sort partition rule used by
 * rccl_b200.dist (no reference counterpart): given the world's contiguous
 * input shards (already concatenated, shard sizes in shard_sizes[world]),
 * compute how many items every rank owns after the exchange.
 *   samples_per_rank: regular samples taken from each locally sorted shard
 * out_counts[world] receives the per-rank output sizes. */
int orc_sample_partition(int key_type, int descending, const void *keys, const size_t *shard_sizes,
                         int world, unsigned samples_per_rank, int threads, size_t *out_counts);

/* CPU baseline stand-ins (oracle/cpu_sorts.cpp): std::sort (stable = 0) or
 * std::stable_sort (stable = 1) by the order image on one thread, or chunked
 * on `threads` threads with pairwise std::merge rounds.  values: n u32
 * values moved with their keys, or NULL. */
int orc_cpu_sort(int key_type, int descending, int stable, void *keys, uint32_t *values,
                 size_t n, int threads);

#ifdef __cplusplus
}
#endif

#endif
