// B200 radix sort kernels: fused multi-digit histogram (+ look-back zeroing and
// bin scan), the onesweep digit-scatter pass with bounded decoupled look-back,
// and the one-CTA small-input sort.
//
// Reference counterparts (semantics, not structure):
//   histogram + exclusive sum  rccl-cub/src/ordering_backend/radix.rs:717-895
//   onesweep keys / pairs      rccl-cub/src/ordering_backend/radix.rs:1022-1687
//   single tile keys / pairs   rccl-cub/src/ordering_backend/radix.rs:535-715
#include "rsort_device.cuh"
#include "rsort_kernels.cuh"

namespace rsort {

template <int VB> struct ValueType;
template <> struct ValueType<0> { using type = uint8_t; };
template <> struct ValueType<1> { using type = uint8_t; };
template <> struct ValueType<2> { using type = uint16_t; };
template <> struct ValueType<4> { using type = uint32_t; };
template <> struct ValueType<8> { using type = uint64_t; };
template <> struct ValueType<16> { using type = uint4; };

// ---------------------------------------------------------------------------
// Init: zero the bins and the counters region.
// ---------------------------------------------------------------------------
__global__ void init_kernel(uint64_t *bins, uint32_t nbins, int *counters, uint32_t ncounters) {
    for (uint32_t i = threadIdx.x; i < nbins; i += blockDim.x) bins[i] = 0;
    for (uint32_t i = threadIdx.x; i < ncounters; i += blockDim.x) counters[i] = 0;
}

// ---------------------------------------------------------------------------
// Histogram of every digit pass in one read of the keys.  Also zeroes the
// look-back words for the whole sort, and the last CTA to finish turns the
// digit counts into global exclusive digit offsets (one scan per pass).
//
// Counter layout: one column of counters per lane, counter (row, digit,
// column) at word (row * 256 + digit) * 32 + column.  Lane l of every warp
// adds into column l, so the 32 lanes of one shared atomic hit 32 different
// banks whatever the digits are: the count runs at the shared-atomic issue
// rate, also on skewed inputs where a single-copy histogram serializes on one
// address.  Keys of up to 4 bytes have one row of 32-bit counters per pass.
// 8-byte keys (8 passes) would need 256 KB that way; they keep 16-bit
// counters instead, passes p and p + 4 in the low and high halves of row
// p % 4's words, and every CTA adds its counts into the bins and clears them
// before any counter can reach 2^16 (HistShape::FLUSH_KEYS).  (With 16
// columns of 32-bit counters, lanes l and l + 16 shared a bank, so every
// atomic took two shared-memory cycles: 0.59 ms for config 2's 2^28 u64 keys
// against 0.33 ms of HBM time.)  The 128 KB of counters take the shared
// memory of one 1024-thread CTA per SM.
// ---------------------------------------------------------------------------
constexpr int HIST_THREADS = 1024;
constexpr int HIST_UNROLL = 4;

template <typename B> struct HistShape {
    static constexpr int MAX_PASSES = int(sizeof(B));  // 8-bit digits
    static constexpr bool PACKED = sizeof(B) == 8;
    static constexpr int COLS = 32;
    static constexpr int ROWS = PACKED ? 4 : MAX_PASSES;
    static constexpr size_t WORDS = size_t(ROWS) * RADIX * COLS;
    static constexpr size_t BYTES = WORDS * 4;
    // PACKED: keys one thread may count between two flushes.  A column is
    // shared by lane l of the CTA's 32 warps, and each key adds one to one
    // counter of every pass, so a counter stays at most 32 * FLUSH_KEYS.
    static constexpr uint32_t FLUSH_KEYS = 65535 / (HIST_THREADS / 32);
    static_assert(uint64_t(FLUSH_KEYS) * (HIST_THREADS / 32) <= 0xffffu,
                  "a 16-bit counter stays below 2^16 between flushes");
};

// Counts one key into every pass's digit counters (column already applied to
// `hc`).  FULL: the bit window is the whole key, so every shift is a
// compile-time constant.
template <typename B, int KIND, bool FULL>
__device__ __forceinline__ void hist_count(B raw, B dmask, uint32_t passes, uint32_t begin_bit,
                                           uint32_t last_mask, uint32_t *hc) {
    using S = HistShape<B>;
    using T = KeyBits<B>;
    B o = to_ordered_k<KIND>(raw, dmask);
    if constexpr (KIND == KIND_FLOAT) {
        if (o == B(T::SIGN - 1)) o = B(T::SIGN);
    }
#pragma unroll
    for (int p = 0; p < S::MAX_PASSES; ++p) {
        uint32_t d;
        if constexpr (FULL) {
            d = uint32_t(o >> (8 * p)) & 0xffu;
        } else {
            if (uint32_t(p) >= passes) break;
            const uint32_t mask = uint32_t(p) + 1 == passes ? last_mask : 0xffu;
            d = uint32_t(o >> (begin_bit + 8 * p)) & mask;
        }
        if constexpr (S::PACKED)
            atomicAdd(hc + ((p & 3) * RADIX + d) * S::COLS, 1u << (16 * (p >> 2)));
        else
            atomicAdd(hc + (p * RADIX + d) * S::COLS, 1u);
    }
}

template <typename B, int KIND, bool FULL>
__global__ void __launch_bounds__(HIST_THREADS, 1) histogram_kernel(HistArgs a) {
    using S = HistShape<B>;
    extern __shared__ __align__(16) uint32_t h[];
    __shared__ int is_last;
    const uint32_t tid = threadIdx.x, lane = tid & 31;
    {
        uint4 *h4 = reinterpret_cast<uint4 *>(h);
        for (uint32_t i = tid; i < S::WORDS / 4; i += HIST_THREADS) h4[i] = make_uint4(0, 0, 0, 0);
    }

    // Zero this sort's look-back words (grid-stride, 16-byte stores).
    {
        const uint64_t words = a.lookback_words;
        const uint64_t stride = uint64_t(gridDim.x) * HIST_THREADS;
        uint4 *lb4 = reinterpret_cast<uint4 *>(a.lookback);
        const uint64_t n4 = words / 2;
        for (uint64_t i = uint64_t(blockIdx.x) * HIST_THREADS + tid; i < n4; i += stride)
            lb4[i] = make_uint4(0, 0, 0, 0);
        if ((words & 1) && blockIdx.x == 0 && tid == 0) a.lookback[words - 1] = 0;
    }
    __syncthreads();

    const B dmask = a.desc ? B(~B(0)) : B(0);
    const uint32_t passes = a.passes, begin_bit = a.begin_bit;
    const uint32_t last_bits = a.end_bit - (begin_bit + 8 * (passes - 1));
    const uint32_t last_mask = (1u << last_bits) - 1;
    uint32_t *hc = h + (lane % S::COLS);
    auto count = [&](B raw) {
        hist_count<B, KIND, FULL>(raw, dmask, passes, begin_bit, last_mask, hc);
    };
    const uint64_t stride = uint64_t(gridDim.x) * HIST_THREADS;
    const uint64_t gtid = uint64_t(blockIdx.x) * HIST_THREADS + tid;
    const B *keys = static_cast<const B *>(a.keys);

    // Column sums into the global bins; each lane starts at a different
    // column so the reads of a warp spread over the banks.
    auto add_columns = [&]() {
        for (uint32_t i = tid; i < passes * RADIX; i += HIST_THREADS) {
            const uint32_t p = i / RADIX, d = i % RADIX;
            const uint32_t row = S::PACKED ? (p & 3) * RADIX + d : i;
            const uint32_t sh = S::PACKED ? 16 * (p >> 2) : 0;
            uint32_t c = 0;
#pragma unroll 8
            for (int k = 0; k < S::COLS; ++k) {
                const uint32_t w = h[row * S::COLS + ((k + lane) % S::COLS)];
                c += S::PACKED ? (w >> sh) & 0xffffu : w;
            }
            if (c) atomicAdd(reinterpret_cast<unsigned long long *>(&a.bins[i]),
                             static_cast<unsigned long long>(c));
        }
    };
    // PACKED: between two chunks of the key range, every CTA adds its counts
    // into the bins and clears them.  The chunk loops below are uniform over
    // the grid, so every thread of a CTA reaches these barriers together.
    auto flush = [&]() {
        __syncthreads();
        add_columns();
        __syncthreads();
        uint4 *h4 = reinterpret_cast<uint4 *>(h);
        for (uint32_t i = tid; i < S::WORDS / 4; i += HIST_THREADS) h4[i] = make_uint4(0, 0, 0, 0);
        __syncthreads();
    };

    uint64_t scalar_begin = 0;
    if (a.vector_ok) {
        // HIST_UNROLL independent 16-byte loads per thread are in flight
        // before any counting, so the SM keeps enough bytes outstanding to
        // cover DRAM latency.
        constexpr int PER = 16 / sizeof(B);
        const uint64_t nvec = a.n / PER;
        const uint4 *kv = reinterpret_cast<const uint4 *>(keys);
        const uint64_t step = stride * HIST_UNROLL;
        auto count_block = [&](uint64_t i) {
            uint4 v[HIST_UNROLL];
#pragma unroll
            for (int u = 0; u < HIST_UNROLL; ++u) {
                const uint64_t idx = i + uint64_t(u) * stride;
                v[u] = idx < nvec ? ld_stream(kv + idx) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < HIST_UNROLL; ++u) {
                if (i + uint64_t(u) * stride >= nvec) break;
                if constexpr (sizeof(B) == 1 || sizeof(B) == 2) {
                    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
#pragma unroll
                        for (int b = 0; b < 4 / int(sizeof(B)); ++b)
                            count(B(w[q] >> (8 * sizeof(B) * b)));
                    }
                } else if constexpr (sizeof(B) == 4) {
                    count(v[u].x);
                    count(v[u].y);
                    count(v[u].z);
                    count(v[u].w);
                } else {
                    count((uint64_t(v[u].y) << 32) | v[u].x);
                    count((uint64_t(v[u].w) << 32) | v[u].z);
                }
            }
        };
        if constexpr (S::PACKED) {
            // One iteration of a thread counts HIST_UNROLL * PER keys from the
            // grid's step-aligned block of `step` vectors, so a chunk of whole
            // blocks holds every load its iterations issue.
            // A chunk's iterations count at most FLUSH_KEYS - (PER - 1) keys
            // per thread, leaving room for the scalar loop's last keys.
            static_assert((S::FLUSH_KEYS / (HIST_UNROLL * PER)) * HIST_UNROLL * PER + PER - 1 <=
                              S::FLUSH_KEYS,
                          "vector chunk within the flush bound");
            const uint64_t chunk = step * (S::FLUSH_KEYS / (HIST_UNROLL * PER));
            for (uint64_t c0 = 0; c0 < nvec; c0 += chunk) {
                const uint64_t c1 = nvec - c0 < chunk ? nvec : c0 + chunk;
                for (uint64_t i = c0 + gtid; i < c1; i += step) count_block(i);
                if (c1 < nvec) flush();
            }
        } else {
            for (uint64_t i = gtid; i < nvec; i += step) count_block(i);
        }
        scalar_begin = nvec * PER;
    }
    // Keys the vector loop did not take (an unaligned input, or the last
    // PER - 1 keys): one key per thread and iteration; PACKED counters in
    // chunks of FLUSH_KEYS iterations.
    if constexpr (S::PACKED) {
        const uint64_t chunk = stride * S::FLUSH_KEYS;
        for (uint64_t c0 = scalar_begin; c0 < a.n; c0 += chunk) {
            const uint64_t c1 = a.n - c0 < chunk ? a.n : c0 + chunk;
            for (uint64_t i = c0 + gtid; i < c1; i += stride) count(keys[i]);
            if (c1 < a.n) flush();
        }
    } else {
        for (uint64_t i = scalar_begin + gtid; i < a.n; i += stride) count(keys[i]);
    }
    __syncthreads();
    add_columns();
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.done, 1) == int(gridDim.x) - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // Every pass at once: thread t takes bin base + t, so each group of 8
    // warps holds one pass's 256 digits and scans them (a warp scan, then
    // the sums of the group's earlier warps).  One round for up to 4
    // passes, two for 8.
    static_assert(HIST_THREADS % RADIX == 0, "whole passes per round");
    __shared__ uint64_t wsum[HIST_THREADS / 32];
    __shared__ uint32_t hot;  // bit p: pass p is hot
    if (tid == 0) hot = 0;
    __syncthreads();
    const uint32_t warp = tid >> 5, total = a.passes * RADIX;
    for (uint32_t base = 0; base < total; base += HIST_THREADS) {
        const uint32_t i = base + tid, p = i / RADIX;
        const uint64_t v = i < total ? __ldcg(&a.bins[i]) : 0;
        if (i < total && v != a.n && v * HOT_SHARE >= a.n && p < 32) atomicOr(&hot, 1u << p);
        uint64_t inc = v;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= uint32_t(off)) inc += y;
        }
        if (lane == 31) wsum[warp] = inc;
        __syncthreads();
        uint64_t before = 0;
        for (uint32_t w = warp & ~uint32_t(RADIX / 32 - 1); w < warp; ++w) before += wsum[w];
        if (i < total) a.bins[i] = before + inc - v;
        __syncthreads();  // wsum is rewritten by the next round
    }
    if (a.hot && tid == 0) *a.hot = int(hot);
}

// ---------------------------------------------------------------------------
// Onesweep digit-scatter pass.
//
// One CTA per tile; the tile id comes from a per-pass atomic counter, so a
// tile only ever waits on tiles that were claimed earlier by running CTAs.
//  1. warp-striped coalesced loads of the tile (pass 0 applies the
//     raw->ordered transform)
//  2. stable warp multi-split rank with __match_any_sync over warp-private
//     256-bin histograms
//  3. per-digit tile totals, published as look-back aggregates, then a
//     bounded walk back for the exclusive prefix across tiles
//  4. keys scattered into shared memory at their tile rank, then written out
//     by consecutive threads to consecutive addresses of each digit run
//     (the last pass applies the ordered->raw transform)
//  5. pairs: values follow through the same shared-memory permutation
// ---------------------------------------------------------------------------
#ifndef RSORT_MIN_BLOCKS
#define RSORT_MIN_BLOCKS 2
#endif
constexpr int WHIST_WORDS = RADIX;

template <typename B, int VB, int ITEMS>
struct OnesweepSmem {
    static constexpr int THREADS = ONESWEEP_THREADS;
    static constexpr int WARPS = THREADS / 32;
    static constexpr int TILE = THREADS * ITEMS;
    static constexpr int VSIZE = VB > 0 ? VB : 1;
    // The rank-phase mask arrays (WMASK) and the scatter-phase key/value
    // staging (KEYS, VALS) are never live at the same time: they share one
    // region, separated by the __syncthreads after ranking.
    static constexpr size_t WHIST = 0;
    static constexpr size_t TSTART = WHIST + size_t(WARPS) * WHIST_WORDS * 4;
    static constexpr size_t GBASE = TSTART + RADIX * 4;
    static constexpr size_t WSUMS = GBASE + RADIX * 8;
    static constexpr size_t CTL = WSUMS + 8 * 4;
    static constexpr size_t WMASK = (CTL + 16 + 15) / 16 * 16;
    static constexpr size_t MASK_BYTES = size_t(WARPS) * RANK_MASK_SETS * RADIX * 4;
    static constexpr size_t KEYS = WMASK;
    static constexpr size_t VALS = KEYS + size_t(TILE) * sizeof(B);
    static constexpr size_t STAGE_BYTES = size_t(TILE) * sizeof(B) + (VB > 0 ? size_t(TILE) * VSIZE : 0);
    static constexpr size_t BYTES = WMASK + (MASK_BYTES > STAGE_BYTES ? MASK_BYTES : STAGE_BYTES);
};

template <bool V> struct BoolTag {
    static constexpr bool value = V;
};
template <int V> struct IntTag {
    static constexpr int value = V;
};

// PERSIST: a persistent grid whose CTAs claim tiles until none are left and
// load the next tile while writing out the current one (measured faster for
// 8-byte keys); otherwise one tile per CTA (faster for 4-byte keys, whose
// tiles are larger).  The per-tile body is compiled twice, for full tiles
// (no per-item bounds tests, fully unrolled write-out) and for the last,
// partial tile.
// RUNS: the RANK_RUNS form (persistent grids only): it sorts the pass only
// when this pass and the one before are hot, else it returns at once.
template <typename B, int VB, int ITEMS, int KIND, bool PERSIST, bool RUNS = false>
__global__ void __launch_bounds__(ONESWEEP_THREADS, RSORT_MIN_BLOCKS) onesweep_kernel(PassArgs a) {
    if constexpr (RUNS) {
        static_assert(PERSIST, "the RANK_RUNS form runs on a persistent grid");
        const int hot = a.hot && a.pass >= 1 && a.pass < 32 ? *a.hot : 0;
        if (!((hot >> a.pass) & (hot >> (a.pass - 1)) & 1)) return;
    }
    using L = OnesweepSmem<B, VB, ITEMS>;
    using VT = typename ValueType<VB>::type;
    constexpr int THREADS = L::THREADS, WARPS = L::WARPS, TILE = L::TILE;
    static_assert((WARPS * WHIST_WORDS) % 4 == 0 && (WARPS * RANK_MASK_SETS * RADIX) % 4 == 0, "");
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *whist = reinterpret_cast<uint32_t *>(smem + L::WHIST);
    uint32_t *wmask = reinterpret_cast<uint32_t *>(smem + L::WMASK);
    uint32_t *tstart = reinterpret_cast<uint32_t *>(smem + L::TSTART);
    int64_t *gbase = reinterpret_cast<int64_t *>(smem + L::GBASE);
    uint32_t *wsums = reinterpret_cast<uint32_t *>(smem + L::WSUMS);
    int *ctl = reinterpret_cast<int *>(smem + L::CTL);
    B *skey = reinterpret_cast<B *>(smem + L::KEYS);
    VT *sval = reinterpret_cast<VT *>(smem + L::VALS);

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const B dmask = a.desc ? B(~B(0)) : B(0);
    const int64_t tiles = int64_t((a.n + TILE - 1) / TILE);
    const uint32_t seg = warp * 32 * ITEMS;
    B *kout = static_cast<B *>(a.keys_out);
    VT *vout = static_cast<VT *>(a.values_out);

    auto zero_scratch = [&]() {
        uint4 *w4 = reinterpret_cast<uint4 *>(whist);
        for (uint32_t i = tid; i < WARPS * WHIST_WORDS / 4; i += THREADS) w4[i] = make_uint4(0, 0, 0, 0);
        uint4 *m4 = reinterpret_cast<uint4 *>(wmask);
        for (uint32_t i = tid; i < WARPS * RANK_MASK_SETS * RADIX / 4; i += THREADS)
            m4[i] = make_uint4(0, 0, 0, 0);
    };

    // Tiles are claimed from the pass's atomic counter.  A tile only ever
    // waits (look-back) on tiles with smaller ids, and every claimed tile
    // belongs to a running CTA that has finished all of its own smaller
    // tiles, so the waits always end.
    if (tid == 0) {
        ctl[0] = atomicAdd(a.tile_counter, 1);
        ctl[1] = 0;
        ctl[3] = 0;
    }
    zero_scratch();
    __syncthreads();
    int64_t tile = ctl[0];
    if (tile >= tiles) return;

    // Warp-striped coalesced loads of one tile's keys and values.
    // (t >= tiles loads nothing; the call is unconditional so the previous
    // tile's registers are dead after its scatter on every path.)
    B key[ITEMS];
    VT val[VB > 0 ? ITEMS : 1];
    auto load_values = [&](int64_t t) {
        const uint64_t base = t < tiles ? uint64_t(t) * TILE : 0;
        const uint64_t remain = t < tiles ? a.n - base : 0;
        const VT *vin = static_cast<const VT *>(a.values_in) + base;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const uint32_t pos = seg + j * 32 + lane;
            if (pos < remain) val[j] = vin[pos];
        }
    };
    auto load_tile = [&](int64_t t) {
        const uint64_t base = t < tiles ? uint64_t(t) * TILE : 0;
        const uint64_t remain = t < tiles ? a.n - base : 0;
        const B *kin = static_cast<const B *>(a.keys_in) + base;
        if (remain >= uint64_t(TILE)) {
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) key[j] = ld_stream(kin + seg + j * 32 + lane);
        } else {
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                const uint32_t pos = seg + j * 32 + lane;
                key[j] = pos < remain ? kin[pos] : B(0);
            }
        }
        if constexpr (VB > 0) load_values(t);
    };
    load_tile(tile);

    // One-bucket fast path: when one digit holds all n keys the pass is the
    // identity permutation, so every tile is copied through in place (with
    // the first / last pass transforms) at HBM speed.  The bins are the same
    // for every CTA, so all CTAs take the same path and no tile waits on
    // another.  The pass still writes the alternate buffer, so the selector
    // outcome is unchanged.
    if (tid < RADIX) {
        const uint64_t lo = a.bins[tid];
        const uint64_t hi = tid + 1 < RADIX ? a.bins[tid + 1] : a.n;
        if (hi - lo == a.n) ctl[3] = 1;
    }
    __syncthreads();
    if (ctl[3]) {
        for (;;) {
            const uint64_t base = uint64_t(tile) * TILE;
            const uint64_t remain = a.n - base;
            if constexpr (PERSIST) {
                if (tid == 0) ctl[2] = atomicAdd(a.tile_counter, 1);
            }
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                const uint32_t pos = seg + j * 32 + lane;
                if (pos < remain) {
                    B k = key[j];
                    if (a.first) k = to_ordered_k<KIND>(k, dmask);
                    if (a.last) k = from_ordered_k<KIND>(k, dmask);
                    kout[base + pos] = k;
                    if constexpr (VB > 0) vout[base + pos] = val[j];
                }
            }
            if constexpr (!PERSIST) break;
            __syncthreads();
            const int64_t next = ctl[2];
            __syncthreads();  // the next claim rewrites ctl[2]
            if (next >= tiles) break;
            tile = next;
            load_tile(tile);
        }
        return;
    }

    // One tile: rank, totals and scan, scatter into shared memory, look-back,
    // write-out.  Returns the next tile id.
    auto tile_body = [&](auto full_tag, auto mode_tag, const int64_t tile,
                         const uint32_t count) -> int64_t {
        constexpr bool FULL = decltype(full_tag)::value;
        constexpr int MODE = decltype(mode_tag)::value;
        auto live = [&](int j) { return FULL || seg + j * 32 + lane < count; };

        // 1. Stable warp multi-split rank over warp-private histograms.
        uint32_t rank[ITEMS];
        if (a.first) {
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) key[j] = to_ordered_k<KIND>(key[j], dmask);
        }
        auto digit_at = [&](int j) {
            return live(j) ? digit_k<KIND>(key[j], a.shift, a.mask) : INVALID_DIGIT;
        };
        warp_rank_items_or3<ITEMS, FULL, MODE>(digit_at, rank, whist + warp * WHIST_WORDS,
                                               wmask + warp * RANK_MASK_SETS * RADIX);
        __syncthreads();
        const int64_t next = PERSIST ? int64_t(ctl[2]) : tiles;

        // 2. Per-digit tile totals -> look-back aggregate, warp offsets, tile scan.
        uint32_t total = 0;
        uint64_t *my_lb = a.lookback + uint64_t(tile) * RADIX + tid;
        // Each warp's digit counts become absolute tile positions (tile digit
        // start + the counts of that digit in earlier warps), so the scatter
        // needs one shared load per key.
        if (tid < RADIX) {
#pragma unroll 4
            for (int w = 0; w < WARPS; ++w) total += whist[w * RADIX + tid];
            st_relaxed_gpu(my_lb, lb_word(tile == 0 ? LB_INCLUSIVE : LB_AGGREGATE, a.tag, total));
        }
        const uint32_t tile_excl = block_exclusive_scan_256(total, wsums, nullptr);
        if (tid < RADIX) {
            tstart[tid] = tile_excl;
            uint32_t run = tile_excl;
#pragma unroll 4
            for (int w = 0; w < WARPS; ++w) {
                const uint32_t t = whist[w * RADIX + tid];
                whist[w * RADIX + tid] = run;
                run += t;
            }
        }
        __syncthreads();

        // 3. Scatter keys and values into shared memory at their tile rank.
        bool bad = false;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            if (live(j)) {
                const uint32_t d = rank[j] >> 16;
                const uint32_t rj = rank[j] & 0xffffu;
                const uint32_t r = whist[warp * RADIX + d] + rj;
                if (r < count) {
                    skey[r] = key[j];
                    if constexpr (VB > 0) sval[r] = val[j];
                } else {
                    bad = true;
                }
            }
        }

        // 4. Look-back for the exclusive prefix of this tile's digits.
        if (tid < RADIX) {
            uint64_t excl = 0;
            if (tile > 0) {
                bool gave_up = false;
                excl = lookback_exclusive(a.lookback, tile, tid, a.tag, a.status, &gave_up);
                st_relaxed_gpu(my_lb, lb_word(LB_INCLUSIVE, a.tag, excl + total));
                if (gave_up) ctl[1] = 1;
            }
            gbase[tid] = int64_t(a.bins[tid] + excl) - int64_t(tile_excl);
        }
        __syncthreads();
        const bool abort = ctl[1] != 0;

        // 5. The key and value registers are free again: start loading the
        //    next tile so its DRAM latency overlaps the write-out.
        if constexpr (PERSIST) load_tile(next);

        // 6. Consecutive threads write consecutive tile positions, i.e. runs
        //    of consecutive addresses within each digit's output range.
        auto write_out = [&](auto last_tag) {
            constexpr bool LAST = decltype(last_tag)::value;
            auto put = [&](uint32_t i) {
                const B k = skey[i];
                const uint32_t d = digit_k<KIND>(k, a.shift, a.mask);
                const uint64_t dst = uint64_t(gbase[d] + int64_t(i));
                if (dst < a.n) {
                    kout[dst] = LAST ? from_ordered_k<KIND>(k, dmask) : k;
                    if constexpr (VB > 0) vout[dst] = sval[i];
                } else {
                    bad = true;
                }
            };
            if constexpr (FULL) {
                // Fully unrolled unless the next tile's keys are already
                // loaded (persistent grid), where registers are short.
                constexpr int WU = PERSIST ? 2 : ITEMS;
#pragma unroll WU
                for (int k = 0; k < ITEMS; ++k) put(tid + uint32_t(k) * THREADS);
            } else {
                for (uint32_t i = tid; i < count; i += THREADS) put(i);
            }
        };
        if (!abort) {
            if (a.last)
                write_out(BoolTag<true>{});
            else
                write_out(BoolTag<false>{});
        }
        if (bad) atomicExch(a.status, DEV_STATUS_BOUNDS);
        return next;
    };

    for (;;) {
        const uint64_t remain = a.n - uint64_t(tile) * TILE;
        const uint32_t count = remain < uint64_t(TILE) ? uint32_t(remain) : uint32_t(TILE);
        // Claim the next tile now; it is read after the rank barrier.
        if constexpr (PERSIST) {
            if (tid == 0) ctl[2] = atomicAdd(a.tile_counter, 1);
        }
        // Full tiles of the RUNS form take the uniform-step rank (a per-tile
        // choice between the two ranks measured slower on skewed passes).
        const int64_t next =
            count == uint32_t(TILE)
                ? tile_body(BoolTag<true>{}, IntTag<(RUNS ? RANK_RUNS : RANK_PLAIN)>{}, tile, count)
                : tile_body(BoolTag<false>{}, IntTag<RANK_PLAIN>{}, tile, count);
        if (!PERSIST || next >= tiles) break;

        // The staging area aliases the mask arrays: every write-out read is
        // done before they are cleared for the next tile.
        __syncthreads();
        zero_scratch();
        __syncthreads();
        tile = next;
    }
}

// ---------------------------------------------------------------------------
// Single-tile sort: one CTA sorts n <= the Policy800 single-tile extent in
// shared memory.  Like the reference's single-tile route it orders by the
// ascending-space digits of fold(to_ordered_ascending(key)) and reverses each
// digit for descending order (rccl-cub/src/ordering_kernels.rs:1229-1234,
// rccl-cub/src/ordering_backend/radix.rs:413-420); the digit width is 8 bits.
// ---------------------------------------------------------------------------
template <typename B, int VB>
struct SingleShape {
    static constexpr int TILE_MAX = int(policy800_single_tile_items(int(sizeof(B)), VB));
    static constexpr int ITEMS = (TILE_MAX + SINGLE_THREADS - 1) / SINGLE_THREADS;
    static constexpr int TILE = ITEMS * SINGLE_THREADS;
    static constexpr int WARPS = SINGLE_THREADS / 32;
    static constexpr int VSIZE = VB > 0 ? VB : 1;
    static constexpr size_t WHIST = 0;
    static constexpr size_t TSTART = WHIST + size_t(WARPS) * RADIX * 4;
    static constexpr size_t WSUMS = TSTART + RADIX * 4;
    static constexpr size_t KEYS = (WSUMS + 8 * 4 + 15) / 16 * 16;
    static constexpr size_t VALS = KEYS + size_t(TILE) * sizeof(B);
    static constexpr size_t BYTES = VALS + (VB > 0 ? size_t(TILE) * VSIZE : 0);
};

template <typename B, int VB>
__global__ void __launch_bounds__(SINGLE_THREADS, 1) single_tile_kernel(SingleArgs a) {
    using S = SingleShape<B, VB>;
    using VT = typename ValueType<VB>::type;
    constexpr int ITEMS = S::ITEMS, WARPS = S::WARPS, THREADS = SINGLE_THREADS;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *whist = reinterpret_cast<uint32_t *>(smem + S::WHIST);
    uint32_t *tstart = reinterpret_cast<uint32_t *>(smem + S::TSTART);
    uint32_t *wsums = reinterpret_cast<uint32_t *>(smem + S::WSUMS);
    B *skey = reinterpret_cast<B *>(smem + S::KEYS);
    VT *sval = reinterpret_cast<VT *>(smem + S::VALS);

    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t seg = warp * 32 * ITEMS;
    uint64_t base = 0;
    uint32_t n = a.n;
    if (a.seg_ids) {
        const uint32_t s = a.seg_ids[blockIdx.x];
        base = a.seg_begin[s];
        const uint64_t len = a.seg_end[s] - base;
        n = len < uint64_t(S::TILE_MAX) ? uint32_t(len) : uint32_t(S::TILE_MAX);
    }
    const KeyXform asc{a.kind, 0};
    const B *kin = static_cast<const B *>(a.keys_in) + base;
    const VT *vin = VB > 0 ? static_cast<const VT *>(a.values_in) + base : nullptr;

    B key[ITEMS];
    VT val[VB > 0 ? ITEMS : 1];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const uint32_t pos = seg + j * 32 + lane;
        key[j] = pos < n ? to_ordered(kin[pos], asc) : B(0);
        if constexpr (VB > 0) {
            if (pos < n) val[j] = vin[pos];
        }
    }

    for (uint32_t bit = a.begin_bit; bit < a.end_bit; bit += 8) {
        const uint32_t bits = min(8u, a.end_bit - bit);
        const uint32_t mask = (1u << bits) - 1;
        for (uint32_t i = tid; i < WARPS * RADIX; i += THREADS) whist[i] = 0;
        __syncthreads();
        uint32_t dig[ITEMS], rank[ITEMS];
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const uint32_t pos = seg + j * 32 + lane;
            uint32_t d = digit_of(key[j], a.kind, bit, mask);
            if (a.desc) d = mask - d;
            dig[j] = pos < n ? d : INVALID_DIGIT;
        }
        warp_rank_items<ITEMS>([&](int j) { return dig[j]; }, rank, whist + warp * RADIX, true);
        __syncthreads();
        uint32_t total = 0;
        if (tid < RADIX) {
            for (int w = 0; w < WARPS; ++w) {
                const uint32_t t = whist[w * RADIX + tid];
                whist[w * RADIX + tid] = total;
                total += t;
            }
        }
        const uint32_t ex = block_exclusive_scan_256(total, wsums, nullptr);
        if (tid < RADIX) tstart[tid] = ex;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            if (dig[j] < RADIX) {
                const uint32_t r = tstart[dig[j]] + whist[warp * RADIX + dig[j]] + rank[j];
                if (r < n) {
                    skey[r] = key[j];
                    if constexpr (VB > 0) sval[r] = val[j];
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const uint32_t pos = seg + j * 32 + lane;
            if (pos < n) {
                key[j] = skey[pos];
                if constexpr (VB > 0) val[j] = sval[pos];
            }
        }
        __syncthreads();
    }

    B *kout = static_cast<B *>(a.keys_out) + base;
    VT *vout = VB > 0 ? static_cast<VT *>(a.values_out) + base : nullptr;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const uint32_t pos = seg + j * 32 + lane;
        if (pos < n) {
            kout[pos] = from_ordered(key[j], asc);
            if constexpr (VB > 0) vout[pos] = val[j];
        }
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
namespace {

template <typename Kernel>
cudaError_t ensure_smem(Kernel k, size_t bytes) {
    // cudaFuncSetAttribute is per function and device; calling it each launch
    // is cheap next to a sort and keeps the launcher stateless.
    if (bytes <= 32 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
}

// RUNS: the RANK_RUNS form, always on a persistent grid.
template <typename B, int VB, bool RUNS = false>
cudaError_t onesweep_t(const PassArgs &a, uint64_t tiles, cudaStream_t s) {
    constexpr int ITEMS = onesweep_items(int(sizeof(B)), VB);
    using L = OnesweepSmem<B, VB, ITEMS>;
    constexpr bool P = RUNS || sizeof(B) == 8;
    auto k = a.kind == KIND_FLOAT         ? onesweep_kernel<B, VB, ITEMS, KIND_FLOAT, P, RUNS>
             : a.kind == KIND_FLOAT_TOTAL ? onesweep_kernel<B, VB, ITEMS, KIND_FLOAT_TOTAL, P, RUNS>
             : a.kind == KIND_SINT        ? onesweep_kernel<B, VB, ITEMS, KIND_SINT, P, RUNS>
                                          : onesweep_kernel<B, VB, ITEMS, KIND_UINT, P, RUNS>;
    cudaError_t e = ensure_smem(k, L::BYTES);
    if (e != cudaSuccess) return e;
    if (!P) {
        k<<<dim3(uint32_t(tiles)), ONESWEEP_THREADS, L::BYTES, s>>>(a);
        return cudaGetLastError();
    }
    // Persistent grid: every CTA that fits on the device at once.
    int dev = 0, sms = 0, per_sm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, ONESWEEP_THREADS, L::BYTES)) !=
        cudaSuccess)
        return e;
    const uint64_t resident = uint64_t(sms) * uint64_t(per_sm > 0 ? per_sm : 1);
    const uint64_t grid = tiles < resident ? tiles : resident;
    k<<<dim3(uint32_t(grid)), ONESWEEP_THREADS, L::BYTES, s>>>(a);
    return cudaGetLastError();
}

template <typename B, int VB>
cudaError_t single_t(const SingleArgs &a, cudaStream_t s) {
    using S = SingleShape<B, VB>;
    auto k = single_tile_kernel<B, VB>;
    cudaError_t e = ensure_smem(k, S::BYTES);
    if (e != cudaSuccess) return e;
    k<<<a.seg_ids ? a.seg_count : 1u, SINGLE_THREADS, S::BYTES, s>>>(a);
    return cudaGetLastError();
}

template <typename B, bool RUNS = false>
cudaError_t onesweep_vb(int vb, const PassArgs &a, uint64_t tiles, cudaStream_t s) {
    switch (vb) {
        case 0: return onesweep_t<B, 0, RUNS>(a, tiles, s);
        case 1: return onesweep_t<B, 1, RUNS>(a, tiles, s);
        case 2: return onesweep_t<B, 2, RUNS>(a, tiles, s);
        case 4: return onesweep_t<B, 4, RUNS>(a, tiles, s);
        case 8: return onesweep_t<B, 8, RUNS>(a, tiles, s);
        case 16: return onesweep_t<B, 16, RUNS>(a, tiles, s);
        default: return cudaErrorInvalidValue;
    }
}

template <typename B>
cudaError_t single_vb(int vb, const SingleArgs &a, cudaStream_t s) {
    switch (vb) {
        case 0: return single_t<B, 0>(a, s);
        case 1: return single_t<B, 1>(a, s);
        case 2: return single_t<B, 2>(a, s);
        case 4: return single_t<B, 4>(a, s);
        case 8: return single_t<B, 8>(a, s);
        case 16: return single_t<B, 16>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_init(uint64_t *bins, size_t nbins, int *counters, size_t ncounters,
                        cudaStream_t stream) {
    init_kernel<<<1, 256, 0, stream>>>(bins, uint32_t(nbins), counters, uint32_t(ncounters));
    return cudaGetLastError();
}

template <typename B, int KIND, bool FULL>
static cudaError_t histogram_launch(const HistArgs &a, int blocks, cudaStream_t stream) {
    constexpr size_t smem = HistShape<B>::BYTES;
    static_assert(smem + 256 <= 227 * 1024, "histogram shared memory");
    cudaError_t e = cudaFuncSetAttribute(histogram_kernel<B, KIND, FULL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    histogram_kernel<B, KIND, FULL><<<blocks, HIST_THREADS, smem, stream>>>(a);
    return cudaGetLastError();
}

template <typename B, int KIND>
static cudaError_t histogram_full(const HistArgs &a, int blocks, cudaStream_t stream) {
    const bool full = a.begin_bit == 0 && a.end_bit == 8 * sizeof(B);
    return full ? histogram_launch<B, KIND, true>(a, blocks, stream)
                : histogram_launch<B, KIND, false>(a, blocks, stream);
}

template <typename B>
static cudaError_t histogram_kind(const HistArgs &a, int blocks, cudaStream_t stream) {
    switch (a.kind) {
        case KIND_SINT: return histogram_full<B, KIND_SINT>(a, blocks, stream);
        case KIND_FLOAT: return histogram_full<B, KIND_FLOAT>(a, blocks, stream);
        case KIND_FLOAT_TOTAL: return histogram_full<B, KIND_FLOAT_TOTAL>(a, blocks, stream);
        default: return histogram_full<B, KIND_UINT>(a, blocks, stream);
    }
}

cudaError_t launch_histogram(int key_bytes, const HistArgs &a, int sm_count, cudaStream_t stream) {
    // One 1024-thread CTA per SM (the counters fill the SM's shared memory).
    const int blocks = sm_count;
    switch (key_bytes) {
        case 1: return histogram_kind<uint8_t>(a, blocks, stream);
        case 2: return histogram_kind<uint16_t>(a, blocks, stream);
        case 4: return histogram_kind<uint32_t>(a, blocks, stream);
        case 8: return histogram_kind<uint64_t>(a, blocks, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_onesweep(int key_bytes, int value_bytes, const PassArgs &a, uint64_t tiles,
                            cudaStream_t stream) {
    switch (key_bytes) {
        case 1: return onesweep_vb<uint8_t>(value_bytes, a, tiles, stream);
        case 2: return onesweep_vb<uint16_t>(value_bytes, a, tiles, stream);
        case 4: return onesweep_vb<uint32_t>(value_bytes, a, tiles, stream);
        case 8: return onesweep_vb<uint64_t>(value_bytes, a, tiles, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_onesweep_runs(int key_bytes, int value_bytes, const PassArgs &a,
                                 uint64_t tiles, cudaStream_t stream) {
    switch (key_bytes) {
        case 4: return onesweep_vb<uint32_t, true>(value_bytes, a, tiles, stream);
        case 8: return onesweep_vb<uint64_t, true>(value_bytes, a, tiles, stream);
        default: return cudaSuccess;  // 1- and 2-byte keys: the plain pass only
    }
}

cudaError_t launch_single_tile(int key_bytes, int value_bytes, const SingleArgs &a,
                               cudaStream_t stream) {
    switch (key_bytes) {
        case 1: return single_vb<uint8_t>(value_bytes, a, stream);
        case 2: return single_vb<uint16_t>(value_bytes, a, stream);
        case 4: return single_vb<uint32_t>(value_bytes, a, stream);
        case 8: return single_vb<uint64_t>(value_bytes, a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace rsort
