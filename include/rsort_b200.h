/*
 * rsort_b200 -- B200 (sm_100a) DeviceRadixSort behind a C ABI.
 *
 * This is the drop-in seam for rccl-cub's radix pass control.  In the
 * reference the pass schedule lives in Rust (rccl-cub/src/radix.rs:425-876)
 * and calls the kernel traits RadixKernel / RadixKeysKernel /
 * RadixPairsKernel (rccl-cub/src/radix.rs:205-362).  Here one C call owns the
 * whole schedule for one sort, so the Rust side replaces the bodies of
 * device_radix_sort_keys_buffer / device_radix_sort_pairs_buffer with a single
 * call each.
 *
 * Conventions (rccl-cub semantics kept):
 *  - All device memory is owned by the caller (keys, values, scratch and the
 *    three control regions).  The single-GPU entry points never allocate.
 *  - Calls are asynchronous on `stream`; nothing synchronizes the stream
 *    (rccl-cub/src/radix.rs:425-554 never synchronizes either).
 *  - Validation errors leave every buffer and the selector unchanged.
 *  - `n == 0` or an empty bit window returns RSORT_OK with no launch and no
 *    selector change (rccl-cub/src/radix.rs:467-469).
 *  - The reference's "Policy800 one-portion maximum" length limit
 *    (rccl-cub/src/radix.rs:377-384) is deliberately lifted: offsets are 64-bit.
 *    A sort takes at most RSORT_MAX_ITEMS items (RSORT_SIZE_OVERFLOW beyond):
 *    the decoupled look-back counts are 48-bit and the tile counters 32-bit.
 *  - The entry points whose scratch is one blob carved into regions
 *    (rsort_segmented_sort, rsort_rows_lexicographic, rsort_sort_by) want it
 *    256-byte aligned and reject other addresses with RSORT_BAD_ARGUMENT
 *    before any device work; allocations from cudaMalloc or PyTorch are.
 */
#ifndef RSORT_B200_H
#define RSORT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same binary layout as cudaStream_t. */
typedef struct CUstream_st *rsort_stream_t;

/* The six RadixKey implementations (rccl-cub/src/radix.rs:114-173), then the
 * small keys the reference lists as missing (no reference counterpart):
 * u8/i8/u16/i16, IEEE half (F16) and bfloat16 (BF16), ordered by the same
 * rules (floats: -0.0 == +0.0 in the radix order, NaNs by bit pattern).  The
 * small keys are accepted by the single-GPU sorts (rsort_keys*, rsort_pairs*,
 * rsort_merge_sort_*) but not by the sample-sort steps, the merges or
 * rsort_keys_static. */
typedef enum {
    RSORT_U32 = 0,
    RSORT_I32 = 1,
    RSORT_F32 = 2,
    RSORT_U64 = 3,
    RSORT_I64 = 4,
    RSORT_F64 = 5,
    RSORT_U8 = 6,
    RSORT_I8 = 7,
    RSORT_U16 = 8,
    RSORT_I16 = 9,
    RSORT_F16 = 10,
    RSORT_BF16 = 11
} rsort_key_t;

/* Maps 1:1 onto rccl_cub::DeviceAlgorithmError (rccl-cub/src/error.rs:3-25). */
typedef enum {
    RSORT_OK = 0,
    RSORT_INVALID_BIT_RANGE = 1,   /* InvalidBitRange { begin, end, key_bits } */
    RSORT_LENGTH_MISMATCH = 2,     /* LengthMismatch { role, expected, actual } */
    RSORT_WORKSPACE_TOO_SMALL = 3, /* WorkspaceTooSmall { role, required, actual } */
    RSORT_UNSUPPORTED_TARGET = 4,  /* UnsupportedTarget: device is not sm_100 */
    RSORT_SIZE_OVERFLOW = 5,       /* SizeOverflow */
    RSORT_CUDA_ERROR = 6,          /* Driver / Launch */
    RSORT_TIMEOUT = 7,             /* a bounded device wait gave up (no reference variant) */
    RSORT_BAD_ARGUMENT = 8         /* unsupported layout, null pointer, misalignment */
} rsort_status;

/* Element counts of the three control regions, in the element types of
 * rccl-cub's DeviceRadixSortBufferWorkspace (bins: u64, lookback: i32,
 * counters: i32; rccl-cub/src/workspace.rs:68-106).  Zero for inputs the
 * single-tile route sorts, as in radix_control_lengths (workspace.rs:96-106). */
typedef struct {
    size_t bins;     /* uint64_t elements */
    size_t lookback; /* int32_t elements; the region must be 16-byte aligned */
    size_t counters; /* int32_t elements */
} rsort_controls;

/* Details of the last non-OK status returned on the calling host thread
 * (the payload of the matching DeviceAlgorithmError variant). */
typedef struct {
    rsort_status status;
    const char *role;  /* static string, e.g. "radix lookback" */
    size_t expected;   /* expected / required length */
    size_t actual;
    unsigned begin_bit, end_bit, key_bits; /* InvalidBitRange payload */
} rsort_error_info;

#define RSORT_MAX_ITEMS ((size_t)1 << 40)

/* Control-region sizes for `n` items (replaces
 * rccl-cub/src/workspace.rs:68-106 device_radix_sort_*workspace_counts).
 * value_bytes = 0 for keys-only; otherwise 1, 2, 4, 8 or 16. */
rsort_status rsort_controls_query(rsort_key_t key, size_t value_bytes, size_t n,
                                  rsort_controls *out);

/* Keys-only DoubleBuffer sort over bits [begin_bit, end_bit)
 * (replaces rccl-cub/src/radix.rs:425-554 device_radix_sort_keys_buffer and
 * the eight-kernel RadixKeysKernel seam it drives).  *current_is_first is the
 * DoubleBuffer selector: read on entry, updated on success exactly as the
 * reference's swaps update it. */
rsort_status rsort_keys_buffer(rsort_key_t key, int descending, void *d_first, void *d_second,
                               size_t n, unsigned begin_bit, unsigned end_bit,
                               int *current_is_first, uint64_t *bins, size_t nbins,
                               int32_t *lookback, size_t nlookback, int32_t *counters,
                               size_t ncounters, rsort_stream_t stream);

/* Key/value DoubleBuffer sort (replaces rccl-cub/src/radix.rs:625-778
 * device_radix_sort_pairs_buffer and the RadixPairsKernel seam).  Values are
 * opaque value_bytes-wide items (1, 2, 4, 8 or 16 bytes) moved stably with
 * their keys. */
rsort_status rsort_pairs_buffer(rsort_key_t key, int descending, void *d_keys_first,
                                void *d_keys_second, void *d_values_first, void *d_values_second,
                                size_t value_bytes, size_t n, unsigned begin_bit, unsigned end_bit,
                                int *current_is_first, uint64_t *bins, size_t nbins,
                                int32_t *lookback, size_t nlookback, int32_t *counters,
                                size_t ncounters, rsort_stream_t stream);

/* In-place full-width keys sort with caller scratch (replaces
 * rccl-cub/src/radix.rs:556-623 device_radix_sort_keys; scratch must hold n
 * keys).  The sorted keys always end in d_keys. */
rsort_status rsort_keys(rsort_key_t key, int descending, void *d_keys, void *d_scratch,
                        size_t nscratch, size_t n, uint64_t *bins, size_t nbins, int32_t *lookback,
                        size_t nlookback, int32_t *counters, size_t ncounters,
                        rsort_stream_t stream);

/* In-place full-width pairs sort (replaces rccl-cub/src/radix.rs:780-876
 * device_radix_sort_pairs). */
rsort_status rsort_pairs(rsort_key_t key, int descending, void *d_keys, void *d_values,
                         size_t value_bytes, void *d_scratch_keys, size_t nscratch_keys,
                         void *d_scratch_values, size_t nscratch_values, size_t n, uint64_t *bins,
                         size_t nbins, int32_t *lookback, size_t nlookback, int32_t *counters,
                         size_t ncounters, rsort_stream_t stream);

/* Synchronizes `stream` and reports whether a bounded device wait of an
 * earlier sort using these counters gave up (RSORT_TIMEOUT), then clears the
 * flag.  The flag is sticky across sorts; a fresh counters region must be
 * zeroed once (as rccl-cub's workspace constructors zero theirs,
 * rccl-cub/src/workspace.rs:114-119).  No reference counterpart: the reference's look-back spin is
 * unbounded (rccl-cub/src/ordering_backend/radix.rs:991-1011). */
rsort_status rsort_check_device_status(int32_t *counters, size_t ncounters,
                                       rsort_stream_t stream);

/* Failure-detection self test (no reference counterpart).  Runs one onesweep
 * CTA whose look-back waits on a predecessor that never publishes; the bounded
 * wait (about one second) must give up.  Returns RSORT_TIMEOUT when it does
 * (the expected result) and leaves the context usable.  Synchronizes
 * `stream` and allocates its own small buffers (test hook, not a sort path). */
rsort_status rsort_selftest_lookback_timeout(rsort_stream_t stream);

/* Single-tile extent used for routing: identical to the reference's Policy800
 * threshold (rccl-cub/src/workspace.rs:43-66). */
size_t rsort_single_tile_items(rsort_key_t key, size_t value_bytes);

/* Number of DoubleBuffer selector flips a successful call performs. */
int rsort_selector_flips(rsort_key_t key, size_t value_bytes, size_t n, unsigned begin_bit,
                         unsigned end_bit);

/* ---------------------------------------------------------------------------
 * Multi-GPU sample sort device steps.  No reference counterpart: the
 * reference is single-GPU.  Each rank sorts its contiguous input shard with
 * rsort_pairs / rsort_keys, then:
 *   1. rsort_dist_samples   regular samples of the sorted shard
 *   2. (all-gather of every rank's samples over NCCL, by the caller)
 *   3. rsort_dist_splitters W-1 splitters from the gathered samples
 *   4. rsort_dist_bounds    W+1 bucket bounds of the local shard
 *   5. (all-to-all of the buckets over NCCL, by the caller)
 *   6. rsort_merge_runs     stable merge of the W received runs
 * Elements are ordered by the 16-byte composite (order image of the key,
 * rank << 40 | position in the sorted shard), which is the global stable
 * order, so the concatenation of the ranks' outputs is the stable sort of the
 * concatenated inputs.
 * ------------------------------------------------------------------------- */

/* Composite size in bytes (samples and splitters are arrays of composites). */
#define RSORT_COMPOSITE_BYTES 16
/* Largest total sample count rsort_dist_splitters accepts. */
#define RSORT_MAX_SPLITTER_SAMPLES 8192

rsort_status rsort_dist_samples(rsort_key_t key, int descending, const void *d_sorted_keys,
                                size_t m, unsigned rank, unsigned samples, void *d_samples,
                                rsort_stream_t stream);
rsort_status rsort_dist_splitters(const void *d_samples, size_t total, unsigned world,
                                  void *d_splitters, rsort_stream_t stream);
rsort_status rsort_dist_bounds(rsort_key_t key, int descending, const void *d_sorted_keys,
                               size_t m, unsigned rank, const void *d_splitters, unsigned world,
                               uint64_t *d_bounds, rsort_stream_t stream);

/* uint64 words of merge-path partition scratch a merge of `total` items needs
 * (rsort_merge, and every round of rsort_merge_runs / rsort_merge_segments,
 * which launch up to 32 pair merges at once). */
size_t rsort_merge_partition_words(size_t total);

/* Stable merge of two sorted runs (a then b; equal keys keep a first).
 * d_partitions: caller scratch of rsort_merge_partition_words(na + nb) words. */
rsort_status rsort_merge(rsort_key_t key, int descending, const void *a_keys,
                         const void *a_values, size_t na, const void *b_keys, const void *b_values,
                         size_t nb, void *out_keys, void *out_values, size_t value_bytes,
                         uint64_t *d_partitions, size_t npartitions, rsort_stream_t stream);

/* Stable merge of `runs` consecutive sorted runs held in keys/values
 * (run_lengths is a host array).  The result is in keys/values, or in the
 * scratch buffers when *result_in_scratch is set on return.  d_partitions
 * needs rsort_merge_partition_words(total items) words. */
rsort_status rsort_merge_runs(rsort_key_t key, int descending, void *keys, void *values,
                              size_t value_bytes, const size_t *run_lengths, unsigned runs,
                              void *scratch_keys, void *scratch_values, uint64_t *d_partitions,
                              size_t npartitions, int *result_in_scratch, rsort_stream_t stream);

/* Stable merge of `runs` sorted runs that may live anywhere the device can
 * read -- this GPU's memory or a peer's (IPC-mapped): the first round merges
 * runs (0,1), (2,3), ... straight from the given pointers into out, so a
 * peer's run crosses NVLink once, inside the merge; later rounds go between
 * out and scratch.  Host arrays of run pointers and lengths; ties keep the
 * lower run first.  The result is in out, or in scratch when
 * *result_in_scratch is set.  d_partitions as for rsort_merge_runs.
 * first_pair: the first-round pair launched first (the others follow,
 * wrapping); ranks starting at different pairs spread their peer reads over
 * different peers.  It does not change the result. */
rsort_status rsort_merge_segments(rsort_key_t key, int descending, unsigned runs,
                                  const void *const *run_keys, const void *const *run_values,
                                  const size_t *run_lengths, size_t value_bytes, void *out_keys,
                                  void *out_values, void *scratch_keys, void *scratch_values,
                                  uint64_t *d_partitions, size_t npartitions,
                                  int *result_in_scratch, unsigned first_pair,
                                  rsort_stream_t stream);

/* Single-pass stable merge of `runs` sorted runs (1..64; ties keep the lower
 * run first), for the last step of the sample sort.  Host arrays of run
 * pointers (this GPU's memory or a peer's) and lengths; out_* receive the
 * merged items.  Every run contributes a pivot every S items; a binary search
 * per pivot and run places the pivots in merged order, and one CTA merges the
 * runs' segments between consecutive pivots in shared memory, so every item
 * is read once and written once (the pairwise rsort_merge_runs reads and
 * writes everything log2(runs) times, but on B200 its two-run kernel keeps
 * more work in flight and is the faster of the two for runs in this GPU's
 * memory).  d_scratch: 8-byte aligned,
 * rsort_multiway_scratch_bytes(key, value_bytes, runs, total items) bytes. */
size_t rsort_multiway_scratch_bytes(rsort_key_t key, size_t value_bytes, unsigned runs,
                                    size_t total);
rsort_status rsort_merge_multiway(rsort_key_t key, int descending, unsigned runs,
                                  const void *const *run_keys, const void *const *run_values,
                                  const size_t *run_lengths, size_t value_bytes, void *out_keys,
                                  void *out_values, void *d_scratch, size_t scratch_bytes,
                                  rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * Whole multi-GPU sample sort behind one call (no reference counterpart; the
 * survey's rsort_dist_pairs(world, devices, comms, streams, ...)).  The steps
 * above run with no host code in between except one read of the gathered
 * bucket bounds (the receive sizes are data dependent):
 *   local sort (in place in d_keys / d_values) -> samples -> NCCL all-gather
 *   -> splitters -> bucket bounds -> NCCL all-gather of the bounds ->
 *   exchange -> stable merge of the W received runs into d_out_*.
 *
 * rsort_dist_pairs drives `world` GPUs from one host thread: devices[r],
 * comms[r] (an ncclComm_t of rank r in a communicator of `world` ranks, for
 * example from ncclCommInitAll) and streams[r] belong to rank r, as do the
 * per-rank arrays.  Collectives of all ranks are issued inside one NCCL
 * group, as NCCL requires for a single thread.  rsort_dist_pairs_rank is the
 * same sort for one process (or thread) per GPU: each rank calls it with its
 * own comm and stream.
 *
 * value_bytes 0 sorts keys only (d_values / d_out_values may be NULL).
 * n_local[r] items per rank (any sizes, zero allowed); the global input is
 * the ranks' shards concatenated in rank order, and the output is its stable
 * sort, partitioned contiguously: rank r receives n_out[r] items into
 * d_out_keys[r] / d_out_values[r] (out_capacity[r] items available).  When
 * any rank's part does not fit, every rank returns RSORT_WORKSPACE_TOO_SMALL
 * after filling n_out and before the exchange (the inputs are then sorted
 * locally, which a repeated call with larger outputs accepts).  d_scratch[r] holds
 * rsort_dist_scratch_bytes(key, value_bytes, n_local[r], out_capacity[r],
 * world) bytes, 256-byte aligned.  Keys: the six 32/64-bit RadixKey types.
 *
 * exchange: RSORT_EXCHANGE_NCCL moves the buckets with grouped
 * ncclSend/ncclRecv; RSORT_EXCHANGE_PEER (rsort_dist_pairs only) reads them
 * straight out of the peers' sorted shards with one copy kernel per rank over
 * NVLink (peer access is enabled by the call; where a pair of devices cannot
 * access each other it falls back to NCCL), and synchronizes the streams
 * before returning so no peer read outlives the call.
 * The NCCL library is resolved at run time (the libnccl.so.2 already loaded
 * into the process, else the one on the library path); without it these
 * calls return RSORT_UNSUPPORTED_TARGET.
 * ------------------------------------------------------------------------- */
typedef struct ncclComm *rsort_nccl_comm_t; /* the same type as NCCL's ncclComm_t */

typedef enum { RSORT_EXCHANGE_NCCL = 0, RSORT_EXCHANGE_PEER = 1 } rsort_exchange_t;

size_t rsort_dist_scratch_bytes(rsort_key_t key, size_t value_bytes, size_t n_local,
                                size_t out_capacity, unsigned world);

rsort_status rsort_dist_pairs(rsort_key_t key, int descending, size_t value_bytes, int world,
                              const int *devices, rsort_nccl_comm_t const *comms,
                              rsort_stream_t const *streams, void *const *d_keys,
                              void *const *d_values, const size_t *n_local,
                              void *const *d_out_keys, void *const *d_out_values,
                              const size_t *out_capacity, void *const *d_scratch,
                              const size_t *scratch_bytes, rsort_exchange_t exchange,
                              size_t *n_out);

rsort_status rsort_dist_pairs_rank(rsort_key_t key, int descending, size_t value_bytes,
                                   int rank, int world, rsort_nccl_comm_t comm,
                                   rsort_stream_t stream, void *d_keys, void *d_values,
                                   size_t n_local, void *d_out_keys, void *d_out_values,
                                   size_t out_capacity, void *d_scratch, size_t scratch_bytes,
                                   size_t *n_out);

/* ---------------------------------------------------------------------------
 * DeviceMergeSort / DeviceMerge for named orders.
 *
 * rccl-cub's merge sort and merge (rccl-cub/src/dispatch.rs:170-193,
 * 1572-1601; the Thrust sort_by / sort_unstable_by lowering,
 * rccl-thrust/src/backend.rs:39-63, 112-150) take a comparator closure
 * compiled to device code, which a C ABI cannot carry.  These entry points
 * take the comparators such closures almost always are:
 *   RSORT_ORDER_ASCENDING        |a, b| a.cmp(b); floats a.partial_cmp(b),
 *                                -0.0 == +0.0 (the radix order)
 *   RSORT_ORDER_DESCENDING       |a, b| b.cmp(a)
 *   RSORT_ORDER_TOTAL_ASCENDING  |a, b| a.total_cmp(b): -0.0 < +0.0, NaNs by
 *                                sign and payload (integers: as ASCENDING)
 *   RSORT_ORDER_TOTAL_DESCENDING |a, b| b.total_cmp(a)
 * The sorts are stable, like rccl-cub's merge sort, so their output equals
 * the comparator sort's for these orders; they run on the radix path (no
 * comparisons), with the radix workspace (rsort_controls_query) and
 * scratch, result in place.  rsort_merge_ordered merges two sorted runs
 * (ties: a first) with rsort_merge's partitions.
 * ------------------------------------------------------------------------- */
typedef enum {
    RSORT_ORDER_ASCENDING = 0,
    RSORT_ORDER_DESCENDING = 1,
    RSORT_ORDER_TOTAL_ASCENDING = 2,
    RSORT_ORDER_TOTAL_DESCENDING = 3
} rsort_order_t;

rsort_status rsort_merge_sort_keys(rsort_key_t key, rsort_order_t order, void *d_keys,
                                   void *d_scratch, size_t nscratch, size_t n, uint64_t *bins,
                                   size_t nbins, int32_t *lookback, size_t nlookback,
                                   int32_t *counters, size_t ncounters, rsort_stream_t stream);
rsort_status rsort_merge_sort_pairs(rsort_key_t key, rsort_order_t order, void *d_keys,
                                    void *d_values, size_t value_bytes, void *d_scratch_keys,
                                    size_t nscratch_keys, void *d_scratch_values,
                                    size_t nscratch_values, size_t n, uint64_t *bins, size_t nbins,
                                    int32_t *lookback, size_t nlookback, int32_t *counters,
                                    size_t ncounters, rsort_stream_t stream);
rsort_status rsort_merge_ordered(rsort_key_t key, rsort_order_t order, const void *a_keys,
                                 const void *a_values, size_t na, const void *b_keys,
                                 const void *b_values, size_t nb, void *out_keys,
                                 void *out_values, size_t value_bytes, uint64_t *d_partitions,
                                 size_t npartitions, rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * Segmented radix sort (no reference counterpart; the reference lists it as
 * missing).  Sorts each segment [d_begin_offsets[i], d_end_offsets[i]) of
 * the input (uint64 device arrays) into the same items of the output, stably,
 * by bits [begin_bit, end_bit), exactly as rsort_keys_buffer / _pairs_buffer
 * would sort an array of that segment's length.  Segments must not overlap;
 * items outside every segment are left as they are in the output.
 * Segments up to the single-tile extent are sorted one CTA each in one
 * launch, longer ones by the onesweep path one after another.  The call reads
 * the offsets on the host (it synchronizes the stream).  value_bytes 0 =
 * keys only.  d_scratch: rsort_segmented_scratch_bytes(..) bytes.
 * ------------------------------------------------------------------------- */
size_t rsort_segmented_scratch_bytes(rsort_key_t key, size_t value_bytes, size_t n, size_t nseg);
rsort_status rsort_segmented_sort(rsort_key_t key, int descending, const void *d_keys_in,
                                  void *d_keys_out, const void *d_values_in, void *d_values_out,
                                  size_t value_bytes, size_t n, size_t nseg,
                                  const uint64_t *d_begin_offsets, const uint64_t *d_end_offsets,
                                  unsigned begin_bit, unsigned end_bit, void *d_scratch,
                                  size_t scratch_bytes, rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * Lexicographic record sort (rccl-thrust/src/record_sort.rs:144-300).
 *
 * Stable ascending sort of n padding-free rows of `words` uint32 each (word 0
 * most significant; SRDatalog/HISA records), in place.  An optional payload
 * of payload_bytes per row (0 = none) moves in lockstep; equal rows keep
 * their input order.  Multi-word LSD over the stable pairs radix sort: one
 * pass per 64-bit chunk of the row, then one gather of rows and payloads.
 * d_scratch: rsort_rows_scratch_bytes(words, payload_bytes, n) bytes, 256-byte
 * aligned.  n must fit a 32-bit permutation.
 * ------------------------------------------------------------------------- */
size_t rsort_rows_scratch_bytes(size_t words, size_t payload_bytes, size_t n);
rsort_status rsort_rows_lexicographic(size_t words, void *d_rows, void *d_payload,
                                      size_t payload_bytes, size_t n, void *d_scratch,
                                      size_t scratch_bytes, rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * DeviceMergeSort by a comparator program.
 *
 * rccl-cub's merge sort (rccl-cub/src/dispatch.rs:170-193, 1113-1146) and
 * Thrust's sort_by lowering (rccl-thrust/src/backend.rs:39-63) take any
 * `Fn(&K, &K) -> Ordering` closure over any DeviceCopy record.  The closures
 * the reference's own callers pass are key projections chained with
 * then_with and optionally reversed:
 *   |l, r| (l & 1).cmp(&(r & 1)).then_with(|| l.cmp(r))  rccl-thrust/examples/sort.rs:101
 *   |l, r| (l / 10).cmp(&(r / 10))                        rccl-thrust/examples/sort.rs:111
 *   |l, r| r.cmp(l)                                       rccl-thrust/examples/sort.rs:133
 *   |l, r| l.key.cmp(&r.key) on a struct                  rccl-thrust/examples/set_operations_tests.rs:143-151
 *   sort_by_key(|k| k & 0x00ff_ffff)                      rccl-cub/examples/device_ordering_benchmark.rs:162
 * A comparator program states such a closure as data: `nterms` terms, most
 * significant first; two records compare by the first term whose projected
 * values differ.  Term t reads the field of type t.type at byte offset
 * t.offset of the record, applies t.projection with t.operand (in the
 * field's type, with Rust's integer semantics), and compares the results by
 * t.order (rsort_order_t: floats by partial_cmp with -0.0 == +0.0, or by
 * total_cmp; DESCENDING reverses the term).  nterms == 0 compares every
 * record equal.
 *   RSORT_PROJ_IDENTITY  v                   any type
 *   RSORT_PROJ_AND       v & operand         integers
 *   RSORT_PROJ_SHR       v >> operand        integers (arithmetic for signed),
 *                                            0 <= operand < width
 *   RSORT_PROJ_DIV       v / operand         integers, truncating; operand != 0,
 *                                            and != -1 for signed types
 *   RSORT_PROJ_REM       v % operand         integers, the dividend's sign;
 *                                            same operand rules as DIV
 * The sort is stable (equal records keep their input order), so its result
 * is the comparator sort's.  It runs on the stable radix path: the terms'
 * significant bits are packed into 64-bit keys, least significant group
 * first, each group one stable (key, index) sort; then the records and the
 * optional values (value_bytes each, 0 = none) are permuted in place.
 * Fields may sit at any byte offset.  d_scratch:
 * rsort_sort_by_scratch_bytes(record_bytes, value_bytes, n) bytes, 256-byte
 * aligned; n must fit a 32-bit permutation; at most RSORT_MAX_TERMS terms.
 * ------------------------------------------------------------------------- */
#define RSORT_MAX_TERMS 16

typedef enum {
    RSORT_PROJ_IDENTITY = 0,
    RSORT_PROJ_AND = 1,
    RSORT_PROJ_SHR = 2,
    RSORT_PROJ_DIV = 3,
    RSORT_PROJ_REM = 4
} rsort_projection_t;

typedef struct {
    uint32_t offset;               /* byte offset of the field in the record */
    int32_t type;                  /* rsort_key_t of the field */
    int32_t projection;            /* rsort_projection_t */
    int32_t order;                 /* rsort_order_t */
    int64_t operand;               /* mask, shift or divisor (the field's bits
                                      for unsigned 64-bit masks) */
} rsort_compare_term;

size_t rsort_sort_by_scratch_bytes(size_t record_bytes, size_t value_bytes, size_t n);
rsort_status rsort_sort_by(const rsort_compare_term *terms, size_t nterms, void *d_records,
                           size_t record_bytes, void *d_values, size_t value_bytes, size_t n,
                           void *d_scratch, size_t scratch_bytes, rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * Bucket exchange over NVLink peer memory (no reference counterpart).
 *
 * Replaces step 5 above (the NCCL all-to-all): every rank exports its sorted
 * shard with CUDA IPC, maps the peers' shards once, and either merges its
 * buckets straight out of the peers' shards (rsort_merge_segments) or pulls
 * them with one copy kernel reading peer HBM directly.
 *   rsort_ipc_export   IPC handle (RSORT_IPC_HANDLE_BYTES) of the device
 *                      allocation holding d_ptr, and d_ptr's byte offset in it
 *   rsort_ipc_import   maps a peer's handle (same node); d_base + offset is
 *                      the peer's pointer; undo with rsort_ipc_release
 *   rsort_gather_segments  copies nseg device segments (peer or local, host
 *                      arrays of pointers and byte lengths) back to back into
 *                      d_dst on `stream`; nseg <= RSORT_GATHER_MAX_SEGMENTS
 * The kernel does not wait for the peers: order it after every peer's sort
 * (for example a collective entered after the sort) and order the peers'
 * next writes of their shards after it (a collective after the copy).
 * ------------------------------------------------------------------------- */
#define RSORT_IPC_HANDLE_BYTES 64
#define RSORT_GATHER_MAX_SEGMENTS 64

rsort_status rsort_ipc_export(const void *d_ptr, void *handle, uint64_t *offset);
rsort_status rsort_ipc_import(const void *handle, void **d_base);
rsort_status rsort_ipc_release(void *d_base);
rsort_status rsort_gather_segments(unsigned nseg, const void *const *d_src, const uint64_t *bytes,
                                   void *d_dst, rsort_stream_t stream);

/* ---------------------------------------------------------------------------
 * Allocation-free keys sort (no reference counterpart).
 *
 * For callers that cannot allocate device memory where they sort: code
 * recording a CUDA graph by stream capture (cudaMalloc is not allowed while
 * capturing), plugins whose host framework owns every device byte through its
 * own pool, and latency-critical loops that cannot take an allocation.  Same
 * result as rsort_keys (in-place, full width, either direction, all six key
 * types), but every scratch byte comes from one static device array inside
 * the library instead of the caller.
 *
 * Limits: n <= RSORT_STATIC_MAX_ITEMS, else RSORT_WORKSPACE_TOO_SMALL.  The
 * array (RSORT_STATIC_SCRATCH_BYTES) is held by every GPU that loads the
 * library until exit.  All calls on a device share it, so calls whose work
 * overlaps on the GPU race and must be serialized by the caller.  The first
 * call on each device resolves the array's address; make it before any stream
 * capture starts.  A bounded device wait that gives up is not reported here
 * (the output is then unspecified).
 * ------------------------------------------------------------------------- */
#define RSORT_STATIC_MAX_ITEMS ((size_t)1 << 20)
#define RSORT_STATIC_SCRATCH_BYTES ((size_t)9 << 20)

rsort_status rsort_keys_static(rsort_key_t key, int descending, void *d_keys, size_t n,
                               rsort_stream_t stream);

const char *rsort_status_string(rsort_status status);
void rsort_last_error(rsort_error_info *out);

/* Kernel launches issued by the calling host thread since the last reset
 * (instrumentation for benchmarks; no reference counterpart). */
uint64_t rsort_launch_count(void);
void rsort_launch_count_reset(void);

/* Kernel ids reported by rsort_profile_read. */
enum { RSORT_KERNEL_INIT = 0, RSORT_KERNEL_HISTOGRAM = 1, RSORT_KERNEL_ONESWEEP = 2,
       RSORT_KERNEL_SINGLE_TILE = 3, RSORT_KERNEL_DIST = 4, RSORT_KERNEL_MERGE = 5,
       RSORT_KERNEL_GATHER = 6, RSORT_KERNEL_RECORDS = 7,
       /* the uniform-step form of a pass after the first (4- and 8-byte keys):
        * it sorts passes where runs of equal keys are expected and exits at
        * once elsewhere, so a pass costs this launch plus the onesweep launch */
       RSORT_KERNEL_ONESWEEP_RUNS = 8 };

/* Benchmark instrumentation (no reference counterpart): while enabled, every
 * kernel launch of the calling host thread is bracketed by CUDA events on its
 * stream.  rsort_profile_read waits for the recorded launches, writes up to
 * `capacity` (kernel id, duration in ms) pairs, clears the record and returns
 * the number of launches recorded. */
void rsort_profile_enable(int enable);
size_t rsort_profile_read(int32_t *kernel_ids, float *milliseconds, size_t capacity);

#ifdef __cplusplus
}
#endif

#endif /* RSORT_B200_H */
